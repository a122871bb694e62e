"""GPU: parity at the benchmark configurations themselves, not only at reduced shapes.

  * 130M fp32 config: 24 layers, d_model 768, 24 heads x 64, d_state 128, vocab 50288,
    random init from seed, 256 uniform prompt ids + 64 greedy tokens. The engine's ids
    must equal the oracle's FREE-RUNNING ids (fp16-faithful and fp32 modes); the max-abs
    logits error against the fp32 oracle is printed and held to the reference's 0.5
    criterion (tests/test_ssd_parity.cpp:148-153 of the reference).
  * 2.7B INT4 headline model at full depth (64 layers): 32-token prompt, 8 greedy tokens
    through the persistent decode kernel, ids and last-step logits vs the oracle.
  * Batched decode at M = 64 on the 2.7B widths (64 sequences in one session: split-K
    INT4 GEMMs at M = 64), sampled sequences vs the oracle.
  * The SSD-op config at full size: batch 8, L 4096, 80 heads x 64, d_state 128, bf16
    in, fp32 out; sequences 0 and 7 vs the fp64 token-by-token recurrence.

Excused near-tie flips are counted and capped (parity_util).
"""

import numpy as np
import pytest

import lssm
import pyoracle as po
from parity_util import assert_ids, first_divergence, flip_cap

pytestmark = pytest.mark.gpu

HP130 = dict(d_model=768, n_layer=24, d_state=128, d_conv=4, expand=2, vocab_size=50288, n_heads=24, d_head=64,
             chunk_size=256, n_groups=1, norm_before_gate=0)
HP27 = dict(d_model=2560, n_layer=64, d_state=128, d_conv=4, expand=2, vocab_size=50288, n_heads=80, d_head=64,
            chunk_size=256, n_groups=1, norm_before_gate=0)


def logits_tolerance(pre, last):
    """Logits bound against the fp16-faithful oracle: twice the spread between the oracle's
    own fp16-faithful and fp32 runs on the same rows (floor 0.1). The engine and the faithful
    oracle share every fp16 rounding point and differ only in fp32 summation order, which
    flips single fp16 roundings deep in the residual stream; the fp16-vs-fp32 spread is the
    size such flips reach at this depth and logit scale."""
    noise = max(np.abs(pre[0] - pre[1]).max(), np.abs(last[0] - last[1]).max())
    return max(0.1, 2.0 * float(noise))


def _free_running_check(gpu_toks, ora: po.OracleModel, prompt, label):
    """Free-running comparison: the oracle generates on its own; up to the first
    difference the histories are identical. A difference is allowed only at a near tie
    of the oracle's logits (counted); after it the rest is checked teacher-forced."""
    n = len(gpu_toks)
    otoks, opre, ostep = ora.generate(prompt, n)
    rows = np.concatenate([opre[None], ostep])
    d = first_divergence(gpu_toks, otoks)
    print(f"[parity] {label}: free-running ids equal for {d} of {n} tokens")
    if d == n:
        return rows, 0
    # diverged: the ids from d on are conditioned on different histories, so re-run teacher-forced
    ttoks, tpre, tstep = ora.generate(prompt, n, teacher=gpu_toks)
    trows = np.concatenate([tpre[None], tstep])
    return trows, assert_ids(gpu_toks, ttoks, trows, label + " (teacher-forced after divergence)")


def test_130m_fp32_config_free_running(ctx):
    hp = lssm.hparams(**HP130)
    model = lssm.Model.synthesize(ctx, hp, seed=130, int4=False)
    image = model.download_bytes()
    assert image == po.synthesize(HP130, 130, False), "synthesized 130M image differs from the CPU generator"
    prompt = np.random.default_rng(130).integers(0, 50280, size=256).astype(np.uint32)
    sess = lssm.Session(ctx, model, batch=1, max_seq_len=256)
    first = sess.prefill(prompt[None])
    pre_gpu = sess.logits()[0]
    rest = sess.decode(first, 63)[0]
    last_gpu = sess.logits()[0]
    toks = np.concatenate([first, rest])
    flips, pre, last = 0, {}, {}
    for mode, name in ((0, "fp16-faithful"), (1, "fp32")):
        ora = po.OracleModel(image, mode=mode)
        rows, f = _free_running_check(toks, ora, prompt, f"130M x24 vs {name} oracle")
        flips += f
        _, _, tstep = ora.generate(prompt, 64, teacher=toks)
        pre[mode], last[mode] = rows[0], tstep[62]
    assert flips <= flip_cap(64)
    tol = logits_tolerance(pre, last)
    e16 = max(np.abs(pre_gpu - pre[0]).max(), np.abs(last_gpu - last[0]).max())
    e32 = max(np.abs(pre_gpu - pre[1]).max(), np.abs(last_gpu - last[1]).max())
    print(f"[parity] 130M x24: max|dlogits| vs fp16-faithful oracle {e16:.4f} (tolerance {tol:.4f}), "
          f"vs fp32 oracle {e32:.4f} (reference criterion 0.5)")
    assert e16 <= tol
    assert e32 < 0.5     # tests/test_ssd_parity.cpp:148-153 of the reference, on the model class it targets
    sess.close()
    model.close()


def test_2p7b_int4_full_depth(ctx):
    """The headline model (64 layers, INT4_B32 in/out_proj) through prefill and the
    persistent decode kernel: free-running ids equal to the oracle's, logits within the
    fp16 noise band of the reference arithmetic."""
    hp = lssm.hparams(**HP27)
    model = lssm.Model.synthesize(ctx, hp, seed=0, int4=True)
    prompt = np.random.default_rng(27).integers(0, 50280, size=32).astype(np.uint32)
    sess = lssm.Session(ctx, model, batch=1, max_seq_len=32)
    first = sess.prefill(prompt[None])
    pre_gpu = sess.logits()[0]
    toks = np.concatenate([first, sess.decode(first, 8)[0]])
    assert sess.launches()[1] == 1, "the persistent decode kernel did not run"
    last_gpu = sess.logits()[0]
    image = po.synthesize(HP27, 0, True)
    pre, last = {}, {}
    for mode in (0, 1):
        ora = po.OracleModel(image, mode=mode)
        rows, f = _free_running_check(toks, ora, prompt, f"2.7B INT4 x64 vs oracle mode {mode}")
        assert f <= flip_cap(9)
        _, _, tstep = ora.generate(prompt, 9, teacher=toks)
        pre[mode], last[mode] = rows[0], tstep[-1]
    tol = logits_tolerance(pre, last)
    e16 = max(np.abs(pre_gpu - pre[0]).max(), np.abs(last_gpu - last[0]).max())
    e32 = max(np.abs(pre_gpu - pre[1]).max(), np.abs(last_gpu - last[1]).max())
    print(f"[parity] 2.7B INT4 x64: max|dlogits| vs fp16-faithful oracle {e16:.4f} (tolerance {tol:.4f}), "
          f"vs fp32 oracle {e32:.4f}, max|logit| {np.abs(pre[1]).max():.1f}")
    assert e16 <= tol
    sess.close()
    model.close()


def test_batched_64_sequences_2p7b_width(ctx):
    """64 sequences in one session on the 2.7B widths (4 layers): the M = 64 split-K INT4
    GEMMs and the batched ssd_step; sequences 0, 21, 42 and 63 vs the oracle (ids
    teacher-forced, last-step logits within logits_tolerance)."""
    hp = dict(HP27, n_layer=4)
    model = lssm.Model.synthesize(ctx, lssm.hparams(**hp), seed=64, int4=True)
    prompts = np.random.default_rng(64).integers(0, 50280, size=(64, 96)).astype(np.uint32)
    sess = lssm.Session(ctx, model, batch=64, max_seq_len=96)
    toks = sess.generate(prompts, 8)
    last = sess.logits()
    image = po.synthesize(hp, 64, True)
    ora16, ora32 = po.OracleModel(image, mode=0), po.OracleModel(image, mode=1)
    for b in (0, 21, 42, 63):
        otoks, opre, ostep = ora16.generate(prompts[b], 8, teacher=toks[b])
        assert_ids(toks[b], otoks, np.concatenate([opre[None], ostep]), f"batch-64 2.7B-width x4, sequence {b}")
        _, pre32, step32 = ora32.generate(prompts[b], 8, teacher=toks[b])
        tol = logits_tolerance({0: opre, 1: pre32}, {0: ostep[6], 1: step32[6]})
        err = float(np.abs(last[b] - ostep[6]).max())
        print(f"[parity] batch-64 sequence {b}: last-step max|dlogits| {err:.4f} (tolerance {tol:.4f})")
        assert err <= tol


def _bf16(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    bits = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return bits, (bits.astype(np.uint32) << 16).view(np.float32)


def test_ssd_op_config_full_size(ctx):
    """batch 8, L 4096, 80 heads x 64, N 128, G 1, chunk 256; x, B, C ~ N(0,1) bf16;
    dt = softplus(N(0,1) - 2) (dt_raw = N(0,1) - 2, dt_bias = 0); A = -exp(U[log 1, log 16]);
    D ~ N(0,1); zero initial state; fp32 state and output. 32 chunks of carried state:
    y within 1.5e-2 of max|y| and the final state within 1.5e-2 of max|S| (bf16 operand
    rounding, as at short L), against the fp64 recurrence."""
    Bt, L, H, P, N, G = 8, 4096, 80, 64, 128, 1
    r = np.random.default_rng(4096)
    alog = np.log(r.uniform(1, 16, H)).astype(np.float32)
    D = r.standard_normal(H).astype(np.float32)
    zero = np.zeros(H, np.float32)
    check = (0, 7)
    Xb = np.empty((Bt, L, H, P), np.uint16)
    Bb = np.empty((Bt, L, G, N), np.uint16)
    Cb = np.empty((Bt, L, G, N), np.uint16)
    dtf = np.empty((Bt, L, H), np.float32)
    ref_in = {}
    for b in range(Bt):
        Xb[b], xr = _bf16(r.standard_normal((L, H, P), dtype=np.float32))
        Bb[b], br = _bf16(r.standard_normal((L, G, N), dtype=np.float32))
        Cb[b], cr = _bf16(r.standard_normal((L, G, N), dtype=np.float32))
        dtf[b] = r.standard_normal((L, H), dtype=np.float32) - 2.0
        if b in check:
            ref_in[b] = (xr, br, cr, dtf[b].copy())
    bufs = [lssm.DeviceBuffer.from_array(ctx, a) for a in (Xb, Bb, Cb, dtf, zero, alog, D)]
    del Xb
    bY = lssm.DeviceBuffer(ctx, Bt * L * H * P * 4)
    bS = lssm.DeviceBuffer.from_array(ctx, np.zeros((Bt, H, P, N), np.float32))
    lssm.Ops(ctx).ssd_chunked_batched(*bufs, bY, bS, lssm.SSDBatchedDims(Bt, L, H, P, N, G, 256, 1e-6, 1e6, 1,
                                                                         lssm.DT_BF16, lssm.DT_F32, lssm.DT_F32,
                                                                         lssm.DT_F32))
    for b in check:
        xr, br, cr, dr = ref_in[b]
        ye = np.zeros((1, L, H, P), np.float32)
        se = np.zeros((1, H, P, N), np.float32)
        po.lib().lssm_oracle_ssd_sequential_f64(*(po.ptr(np.ascontiguousarray(a)) for a in (xr, br, cr, dr, zero, alog, D)),
                                                po.ptr(ye), po.ptr(se), 1, L, H, P, N, G, 1e-6, 1e6, 1)
        y = bY.download(np.float32, L * H * P, b * L * H * P * 4).reshape(ye.shape)
        s = bS.download(np.float32, H * P * N, b * H * P * N * 4).reshape(se.shape)
        ey, es = np.abs(y - ye).max() / np.abs(ye).max(), np.abs(s - se).max() / np.abs(se).max()
        # error of the last chunk vs the first: a compounding state-carry error would grow with L
        e_first = np.abs(y[0, :256] - ye[0, :256]).max() / np.abs(ye).max()
        e_last = np.abs(y[0, -256:] - ye[0, -256:]).max() / np.abs(ye).max()
        print(f"[parity] SSD-op config sequence {b}: max|dy|/max|y| {ey:.3e} (first chunk {e_first:.3e}, "
              f"last chunk {e_last:.3e}), max|dS|/max|S| {es:.3e}")
        assert ey <= 1.5e-2
        assert es <= 1.5e-2
