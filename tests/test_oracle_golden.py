"""CPU: the oracle against the reference's own golden vectors.

* INT4_B32 packing: the oracle's quantiser vs bytes produced by the reference's
  tools/export_mamba2.py:68-103 (bit-exact), and the dequant layout of
  shaders/linear.metal:38-61.
* Whole-model: the oracle's prefill / decode logits and greedy ids vs HF
  transformers' Mamba2ForCausalLM run on the exact weights of .ssm files written by
  the reference exporter (the ground truth of tests/test_ssd_parity.cpp).
"""

import numpy as np
import pytest

import pyoracle as po


def test_fp16_conversion_matches_numpy():
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 10.0 ** rng.integers(-8, 5, 20000),
                           np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e-8, 5.96e-8, 2.98e-8, np.inf, -np.inf],
                                    dtype=np.float32)]).astype(np.float32)
    ours = np.zeros(len(vals), dtype=np.uint16)
    po.lib().lssm_oracle_f32_to_f16(po.ptr(vals), po.ptr(ours), len(vals))
    with np.errstate(over="ignore"):   # 65520 and the 10^4-scaled samples round to inf on purpose
        want = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, want)
    back = np.zeros(len(vals), dtype=np.float32)
    po.lib().lssm_oracle_f16_to_f32(po.ptr(ours), po.ptr(back), len(vals))
    assert np.array_equal(back, ours.view(np.float16).astype(np.float32))


def test_int4_quantizer_bit_exact_vs_reference(golden):
    g = np.load(golden / "int4_pack.npz")
    w = g["w_f16"].view(np.float16).astype(np.float32)
    N, K = w.shape
    packed = np.zeros((N, K // 2), dtype=np.uint8)
    scales = np.zeros((N, K // 32), dtype=np.uint16)
    po.lib().lssm_oracle_int4_quantize(po.ptr(np.ascontiguousarray(w)), N, K, po.ptr(packed), po.ptr(scales))
    assert np.array_equal(scales, g["scales"])
    assert np.array_equal(packed, g["packed"])


def test_int4_dequant_layout(golden):
    g = np.load(golden / "int4_pack.npz")
    packed, scales = g["packed"], g["scales"]
    N, K = packed.shape[0], packed.shape[1] * 2
    out = np.zeros((N, K), dtype=np.float32)
    po.lib().lssm_oracle_int4_dequant(po.ptr(packed), po.ptr(scales), po.ptr(out), N, K)
    lo = (packed & 0xF).astype(np.int32)
    hi = (packed >> 4).astype(np.int32)
    q = np.empty((N, K), np.int32)
    q[:, 0::2], q[:, 1::2] = lo, hi
    q = np.where(q < 8, q, q - 16)
    expect = q * np.repeat(scales.view(np.float16).astype(np.float32), 32, axis=1)
    assert np.array_equal(out, expect)


@pytest.mark.parametrize("tag", ["tinyA", "tinyB"])
@pytest.mark.parametrize("quant", ["fp16", "int4"])
def test_oracle_matches_hf(golden, tag, quant):
    g = np.load(golden / f"{tag}_{quant}_hf.npz")
    for mode, tol in ((1, 2e-3), (0, 0.1)):
        m = po.OracleModel(golden / f"{tag}_{quant}.ssm", mode=mode)
        toks, pl, sl = m.generate(g["prompt"], len(g["tokens"]), teacher=g["tokens"])
        assert np.abs(pl - g["prefill_logits"]).max() < tol
        assert np.abs(sl - g["step_logits"][1:]).max() < tol
        assert np.array_equal(toks, g["tokens"])


def test_ssd_chunked_equals_sequential_recurrence():
    rng = np.random.default_rng(1)
    Bt, L, H, P, N, G = 2, 37, 4, 8, 16, 2
    X = rng.standard_normal((Bt, L, H, P)).astype(np.float32)
    Bm = rng.standard_normal((Bt, L, G, N)).astype(np.float32)
    Cm = rng.standard_normal((Bt, L, G, N)).astype(np.float32)
    dt = (rng.standard_normal((Bt, L, H)) - 2).astype(np.float32)
    db = np.zeros(H, np.float32)
    alog = np.log(rng.uniform(1, 16, H)).astype(np.float32)
    D = rng.standard_normal(H).astype(np.float32)
    s0 = rng.standard_normal((Bt, H, P, N)).astype(np.float32) * 0.1
    ys, ss = np.zeros_like(X), s0.copy()
    po.lib().lssm_oracle_ssd_sequential_f64(*map(po.ptr, (X, Bm, Cm, dt, db, alog, D, ys, ss)), Bt, L, H, P, N, G,
                                            1e-6, 1e6, 1)
    for C in (1, 8, 16, 64):
        yc, sc = np.zeros_like(X), s0.copy()
        po.lib().lssm_oracle_ssd_chunked_f32(*map(po.ptr, (X, Bm, Cm, dt, db, alog, D, yc, sc)), Bt, L, H, P, N, G,
                                             C, 1e-6, 1e6, 1, 1)
        assert np.abs(yc - ys).max() < 1e-4 * (1 + np.abs(ys).max())
        assert np.abs(sc - ss).max() < 1e-4 * (1 + np.abs(ss).max())


def test_argmax_first_max_rule():
    v = np.array([1.0, 3.0, 3.0, 2.0], dtype=np.float32)
    assert po.lib().lssm_oracle_argmax_f32(po.ptr(v), 4) == 1
    v = np.array([np.nan, 5.0, 6.0], dtype=np.float32)
    assert po.lib().lssm_oracle_argmax_f32(po.ptr(v), 3) == 0
