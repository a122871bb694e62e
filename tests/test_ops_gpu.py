"""GPU: every op of the drop-in boundary (include/lssm_cuda.h, the MetalOps surface of
include/lite_ssm/ops.hpp) called through the C ABI and compared with the CPU oracle
(oracle/lssm_oracle.cpp) on the same seeded inputs.

Tolerances (stated per test):
  * integer / byte / copy work (conv-state roll and seeding, the SSD state layout,
    kernel-probe and error behaviour): bit-exact;
  * fp16-output elementwise ops: within 1 fp16 ulp (CUDA's expf vs the host libm can
    flip the last fp16 rounding);
  * reductions (RMSNorm, GEMV, GEMM, SSD): |gpu - oracle| <= atol + rtol*|oracle| with
    fp32 accumulation-order slack (rtol 1e-2 for fp16 outputs, i.e. a few fp16 ulps).
"""

import numpy as np
import pytest

import lssm
import pyoracle as po

pytestmark = pytest.mark.gpu

RNG = np.random.default_rng(1234)


def h(a):
    return np.ascontiguousarray(np.asarray(a, np.float32).astype(np.float16))


def hb(ctx, a, extra=0):
    return lssm.DeviceBuffer.from_array(ctx, a, extra)


def get16(buf, n, off=0):
    return buf.download(np.float16, n, off).astype(np.float32)


def ulp_close(a, b, ulps=1):
    a16, b16 = np.float16(np.ravel(a)), np.float16(np.ravel(b))
    spacing = np.abs(np.spacing(np.maximum(np.abs(a16), np.abs(b16)).astype(np.float16))).astype(np.float32)
    return np.all(np.abs(a16.astype(np.float32) - b16.astype(np.float32)) <= ulps * spacing + 1e-7)


def close(gpu, ref, rtol=1e-2, atol=1e-3):
    gpu, ref = np.ravel(gpu), np.ravel(ref)
    err = np.abs(gpu - ref)
    ok = err <= atol + rtol * np.abs(ref)
    assert ok.all(), f"max err {err.max():.4g} at {np.argmax(err)}; ref {ref.ravel()[np.argmax(err)]:.4g}"


@pytest.fixture(scope="module")
def ops(ctx):
    return lssm.Ops(ctx)


# ---------------------------------------------------------------------------
def test_backend_loaded_and_registry():
    assert lssm.lib().lssm_backend_loaded() == 1
    assert lssm.lib().lssm_has_kernel(b"ssd_chunked_f16") == 1


# 16-byte path (dim % 8 == 0, row in registers, up to 1024 octets): 2560, 768, 5120, 8192, 16;
# element path: 12, 8200 (1025 octets).
@pytest.mark.parametrize("rows,dim", [(3, 2560), (5, 12), (1, 768), (2, 5120), (4, 8192), (2, 8200), (3, 16)])
def test_rmsnorm(ctx, ops, rows, dim):
    x = h(RNG.standard_normal((rows, dim)) * 3)
    w = h(RNG.uniform(0.5, 1.5, dim))
    ref = np.zeros((rows, dim), np.uint16)
    po.lib().lssm_oracle_rmsnorm_f16(po.ptr(x.view(np.uint16)), po.ptr(w.view(np.uint16)), po.ptr(ref), rows, dim, 1e-5)
    bx, bw, by = hb(ctx, x), hb(ctx, w), lssm.DeviceBuffer(ctx, x.nbytes)
    ops.rmsnorm_f16((bx, 0), (bw, 0), (by, 0), lssm.RMSNormDims(rows, dim, 1e-5))
    assert ulp_close(get16(by, rows * dim), po.to_f32(ref), ulps=2)


def test_rmsnorm_rejects_bad_dim(ctx, ops):
    b = lssm.DeviceBuffer(ctx, 64)
    with pytest.raises(lssm.LssmError, match="dim must be a multiple of 4"):
        ops.rmsnorm_f16((b, 0), (b, 0), (b, 0), lssm.RMSNormDims(1, 6, 1e-5))


@pytest.mark.parametrize("N,K", [(1000, 2560), (77, 100), (8, 4)])
def test_linear_f16_gemv(ctx, ops, N, K):
    x = h(RNG.standard_normal(K))
    w = h(RNG.standard_normal((N, K)) / np.sqrt(K))
    ref = np.zeros(N, np.uint16)
    po.lib().lssm_oracle_linear_f16(po.ptr(x.view(np.uint16)), po.ptr(w.view(np.uint16)), po.ptr(ref), 1, N, K)
    bx, bw, by = hb(ctx, x), hb(ctx, w), lssm.DeviceBuffer(ctx, N * 2)
    ops.linear_f16_gemv((bx, 0), (bw, 0), (by, 0), lssm.LinearDims(1, N, K))
    close(get16(by, N), po.to_f32(ref))
    # fused SiLU epilogue (linear.metal:113-138)
    ops.linear_silu_f16_gemv((bx, 0), (bw, 0), (by, 0), lssm.LinearDims(1, N, K))
    r = po.to_f32(ref)
    close(get16(by, N), r / (1 + np.exp(-r)), atol=2e-3)


def test_gemv_rejects_batch(ctx, ops):
    b = lssm.DeviceBuffer(ctx, 1024)
    with pytest.raises(lssm.LssmError, match="M must be 1"):
        ops.linear_f16_gemv((b, 0), (b, 0), (b, 0), lssm.LinearDims(2, 4, 8))
    with pytest.raises(lssm.LssmError, match="K must be a multiple of 4"):
        ops.linear_f16_gemv((b, 0), (b, 0), (b, 0), lssm.LinearDims(1, 4, 6))


def test_rmsnorm_linear_gemv(ctx, ops):
    N, K = 300, 768
    x = h(RNG.standard_normal(K) * 2)
    nw = h(RNG.uniform(0.5, 1.5, K))
    w = h(RNG.standard_normal((N, K)) / np.sqrt(K))
    xn = np.zeros(K, np.uint16)
    po.lib().lssm_oracle_rmsnorm_f16(po.ptr(x.view(np.uint16)), po.ptr(nw.view(np.uint16)), po.ptr(xn), 1, K, 1e-5)
    ref = np.zeros(N, np.uint16)
    po.lib().lssm_oracle_linear_f16(po.ptr(xn), po.ptr(w.view(np.uint16)), po.ptr(ref), 1, N, K)
    bx, bn, bw, by = hb(ctx, x), hb(ctx, nw), hb(ctx, w), lssm.DeviceBuffer(ctx, N * 2)
    ops.rmsnorm_linear_f16_gemv((bx, 0), (bn, 0), (bw, 0), (by, 0), lssm.RMSLinearDims(N, K, 1e-5))
    close(get16(by, N), po.to_f32(ref))


# (2048, 2560, 5120) takes 144-wide N tiles (last tile ragged), (2048, 10576, 2560) 240-wide ones:
# accumulators ending in a 16-column chunk
@pytest.mark.parametrize("M,N,K", [(200, 300, 256), (130, 257, 72), (512, 1024, 2560), (33, 40, 36), (1, 16, 64),
                                   (2048, 2560, 5120), (2048, 10576, 2560)])
def test_linear_f16_gemm(ctx, ops, M, N, K):
    x = h(RNG.standard_normal((M, K)))
    w = h(RNG.standard_normal((N, K)) / np.sqrt(K))
    ref = (x.astype(np.float32) @ w.astype(np.float32).T)
    bx, bw, by = hb(ctx, x), hb(ctx, w), lssm.DeviceBuffer(ctx, M * N * 2)
    ops.linear_f16_gemm((bx, 0), (bw, 0), (by, 0), lssm.LinearDims(M, N, K))
    close(get16(by, M * N).reshape(M, N), ref, rtol=1e-2, atol=2e-3)
    ops.linear_silu_f16_gemm((bx, 0), (bw, 0), (by, 0), lssm.LinearDims(M, N, K))
    close(get16(by, M * N).reshape(M, N), ref / (1 + np.exp(-ref)), rtol=1e-2, atol=2e-3)


def _int4_weights(N, K, scale=0.05):
    w = (RNG.standard_normal((N, K)) * scale).astype(np.float32)
    w16 = w.astype(np.float16).astype(np.float32)
    packed = np.zeros((N, K // 2), np.uint8)
    scales = np.zeros((N, K // 32), np.uint16)
    po.lib().lssm_oracle_int4_quantize(po.ptr(np.ascontiguousarray(w16)), N, K, po.ptr(packed), po.ptr(scales))
    return packed, scales


# N >= 16 x SM count with K % 256 == 0 takes the streaming kernel (1 CTA per SM,
# K chunks of 1024 / 512 / 256 through a shared-memory ring), the rest the per-tile ones
@pytest.mark.parametrize("N,K,off", [(1000, 2560, 0), (77, 96, 0), (300, 5120, 0), (50, 64, 2), (10576, 2560, 0),
                                     (2560, 5120, 0), (4813, 1280, 0), (3000, 8192, 0)])
def test_linear_int4_gemv(ctx, ops, N, K, off):
    packed, scales = _int4_weights(N, K)
    x = h(RNG.standard_normal(K))
    ref = np.zeros(N, np.uint16)
    po.lib().lssm_oracle_linear_int4(po.ptr(x.view(np.uint16)), po.ptr(packed), po.ptr(scales), po.ptr(ref), 1, N, K, 0)
    # one buffer holding [pad][packed][scales] like a .ssm payload (scales after packed)
    blob = np.concatenate([np.zeros(off, np.uint8), packed.ravel(), scales.view(np.uint8).ravel()])
    bw, bx, by = hb(ctx, blob), hb(ctx, x), lssm.DeviceBuffer(ctx, N * 2)
    ops.linear_int4_gemv((bx, 0), (bw, off), (bw, off + N * K // 2), (by, 0), lssm.LinearDims(1, N, K))
    close(get16(by, N), po.to_f32(ref))


# batched-decode extension: rows 2..8; N >= 16 x SM count takes the streaming kernel
@pytest.mark.parametrize("M,N,K", [(2, 300, 5120), (4, 4813, 1280), (8, 3000, 8192), (3, 18560, 4096)])
def test_linear_int4_gemv_rows(ctx, ops, M, N, K):
    packed, scales = _int4_weights(N, K)
    x = h(RNG.standard_normal((M, K)))
    ref = np.zeros(M * N, np.uint16)
    po.lib().lssm_oracle_linear_int4(po.ptr(x.view(np.uint16)), po.ptr(packed), po.ptr(scales), po.ptr(ref), M, N, K,
                                     0)
    blob = np.concatenate([packed.ravel(), scales.view(np.uint8).ravel()])
    bw, bx, by = hb(ctx, blob), hb(ctx, x), lssm.DeviceBuffer(ctx, M * N * 2)
    ops.linear_int4_gemv_rows((bx, 0), (bw, 0), (bw, N * K // 2), (by, 0), lssm.LinearDims(M, N, K))
    close(get16(by, M * N), po.to_f32(ref))
    with pytest.raises(lssm.LssmError, match="M must be 1..8"):
        ops.linear_int4_gemv_rows((bx, 0), (bw, 0), (bw, N * K // 2), (by, 0), lssm.LinearDims(9, N, K))


@pytest.mark.parametrize("M,N,K", [(2, 1000, 2560), (5, 5000, 4096), (8, 777, 1024)])
def test_linear_f16_gemv_rows(ctx, ops, M, N, K):
    x = h(RNG.standard_normal((M, K)))
    w = h(RNG.standard_normal((N, K)) * 0.05)
    ref = x.astype(np.float32) @ w.astype(np.float32).T
    bx, bw, by = hb(ctx, x), hb(ctx, w), lssm.DeviceBuffer(ctx, M * N * 2)
    ops.linear_f16_gemv_rows((bx, 0), (bw, 0), (by, 0), lssm.LinearDims(M, N, K))
    close(get16(by, M * N).reshape(M, N), ref, rtol=1e-2, atol=2e-3)


def test_int4_rejects_bad_dims(ctx, ops):
    b = lssm.DeviceBuffer(ctx, 4096)
    with pytest.raises(lssm.LssmError, match="K must be a multiple of 32"):
        ops.linear_int4_gemv((b, 0), (b, 0), (b, 0), (b, 0), lssm.LinearDims(1, 4, 48))
    with pytest.raises(lssm.LssmError, match="M must be 1"):
        ops.linear_int4_gemv((b, 0), (b, 0), (b, 0), (b, 0), lssm.LinearDims(3, 4, 64))
    with pytest.raises(lssm.LssmError, match="K must be a multiple of 32"):
        ops.linear_int4_gemm((b, 0), (b, 0), (b, 0), (b, 0), lssm.LinearDims(3, 4, 48))


# (512, 10576, 2560) and (200, 4810, 768) take the fused dequant tcgen05 kernel (k_gemm_i4,
# ragged last N tile in the last case); M <= 128 with K >= 512 splits K over CTAs in it
# ((64, 5120, 5120), (64, 2560, 5120), (16, 10576, 2560), (33, 1000, 768): fp32 partials
# summed by a second kernel); the others the dequantise-then-GEMM path. Same fp16 rounding
# of each weight in both.
@pytest.mark.parametrize("M,N,K", [(100, 300, 256), (512, 10576, 2560), (17, 33, 96), (64, 5120, 5120),
                                   (200, 4810, 768), (64, 2560, 5120), (16, 10576, 2560), (33, 1000, 768)])
def test_linear_int4_gemm(ctx, ops, M, N, K):
    packed, scales = _int4_weights(N, K)
    x = h(RNG.standard_normal((M, K)))
    ref = np.zeros(M * N, np.uint16)
    po.lib().lssm_oracle_linear_int4(po.ptr(x.view(np.uint16)), po.ptr(packed), po.ptr(scales), po.ptr(ref), M, N, K, 1)
    bp, bs, bx, by = hb(ctx, packed), hb(ctx, scales), hb(ctx, x), lssm.DeviceBuffer(ctx, M * N * 2)
    ops.linear_int4_gemm((bx, 0), (bp, 0), (bs, 0), (by, 0), lssm.LinearDims(M, N, K))
    close(get16(by, M * N), po.to_f32(ref), rtol=1e-2, atol=2e-3)


# off 2: the packed nibbles at an unaligned offset of a payload (byte-load fallback)
@pytest.mark.parametrize("off", [0, 2])
def test_int4_dequantised_weights_bit_exact(ctx, ops, off):
    """M > 512 takes the dequantise-then-GEMM path. With unit-vector activation rows the GEMM
    returns single weights (one exact product, fp32 sum, fp16 result), so each output must
    equal half(float(q) * float(scale)) bit for bit (linear.metal:538 rounding), including
    scales whose products round near the fp16 maximum, go subnormal and carry both signs
    (finite products only: an infinite weight times a zero activation would be NaN; zeros
    compare without their sign)."""
    M, N, K = 600, 304, 2560
    packed, scales = _int4_weights(N, K)
    sc = scales.view(np.float16).copy()
    sc.ravel()[:7] = np.float16([4000, -4000, 6e-8, -3e-6, 0.0, 1.5e-5, -7e3])
    scales = sc.view(np.uint16)
    ks = RNG.choice(K, size=M, replace=True)
    x = np.zeros((M, K), np.float16)
    x[np.arange(M), ks] = 1.0
    nib = np.zeros((N, K), np.int32)
    nib[:, 0::2] = packed & 0xF
    nib[:, 1::2] = packed >> 4
    q = np.where(nib < 8, nib, nib - 16).astype(np.float32)
    w16 = (q * np.repeat(scales.view(np.float16).astype(np.float32), 32, axis=1)).astype(np.float16)
    blob = np.concatenate([np.zeros(off, np.uint8), packed.ravel()])
    bp_, bs, bx, by = hb(ctx, blob), hb(ctx, scales), hb(ctx, x), lssm.DeviceBuffer(ctx, M * N * 2)
    ops.linear_int4_gemm((bx, 0), (bp_, off), (bs, 0), (by, 0), lssm.LinearDims(M, N, K))
    got = by.download(np.uint16, M * N).reshape(M, N)
    # the GEMM's fp32 sum starts at +0, so a -0 weight (q = 0 with a negative scale) comes out as +0
    want = np.where(w16[:, ks].T == 0, np.float16(0), w16[:, ks].T).astype(np.float16).view(np.uint16)
    bad = np.argwhere(got != want)
    detail = [(int(m), int(n), int(ks[m]), hex(int(got[m, n])), hex(int(want[m, n])),
               float(scales.view(np.float16)[n, ks[m] // 32])) for m, n in bad[:8]]
    assert not len(bad), f"{len(bad)} dequantised weights differ (m, n, k, got, want, scale): {detail}"


def test_int4_gemm_scratch_growth_keeps_replayed_graph_valid():
    """The INT4 GEMM's scratch belongs to the context. A captured batch keeps using its block
    after a later, larger call grows the scratch outside the batch (the old block is kept
    until the graph is replaced), and growth inside a capture is refused with a state error."""
    c = lssm.Ctx(0)
    ops = lssm.Ops(c)
    M, N, K = 16, 512, 1024
    packed, scales = _int4_weights(N, K)
    x = h(RNG.standard_normal((M, K)))
    ref = np.zeros(M * N, np.uint16)
    po.lib().lssm_oracle_linear_int4(po.ptr(x.view(np.uint16)), po.ptr(packed), po.ptr(scales), po.ptr(ref), M, N, K, 1)
    bp, bs, bx, by = hb(c, packed), hb(c, scales), hb(c, x), lssm.DeviceBuffer(c, M * N * 2)
    ops.linear_int4_gemm((bx, 0), (bp, 0), (bs, 0), (by, 0), lssm.LinearDims(M, N, K))   # sizes the scratch
    c.set_graph_batching(True)
    c.begin_batch()
    ops.linear_int4_gemm((bx, 0), (bp, 0), (bs, 0), (by, 0), lssm.LinearDims(M, N, K))
    c.commit_and_wait()
    c.set_graph_batching(False)
    # a larger call outside the batch grows the scratch (split-K partials of 128 x 4096)
    M2, N2 = 128, 4096
    p2, s2 = _int4_weights(N2, K)
    x2 = h(RNG.standard_normal((M2, K)))
    b2p, b2s, b2x, b2y = hb(c, p2), hb(c, s2), hb(c, x2), lssm.DeviceBuffer(c, M2 * N2 * 2)
    ops.linear_int4_gemm((b2x, 0), (b2p, 0), (b2s, 0), (b2y, 0), lssm.LinearDims(M2, N2, K))
    by.zero()
    c.replay_batch(2)
    c.begin_batch()
    c.commit_and_wait()
    close(get16(by, M * N), po.to_f32(ref), rtol=1e-2, atol=2e-3)
    # growth inside a capture: refused, and the context stays usable
    M3, N3 = 128, 8192
    p3, s3 = _int4_weights(N3, K)
    b3p, b3s, b3y = hb(c, p3), hb(c, s3), lssm.DeviceBuffer(c, M3 * N3 * 2)
    c.set_graph_batching(True)
    c.begin_batch()
    with pytest.raises(lssm.LssmError, match="inside a captured batch"):
        ops.linear_int4_gemm((b2x, 0), (b3p, 0), (b3s, 0), (b3y, 0), lssm.LinearDims(M3, N3, K))
    c.commit_and_wait()
    c.set_graph_batching(False)
    ops.linear_int4_gemm((bx, 0), (bp, 0), (bs, 0), (by, 0), lssm.LinearDims(M, N, K))
    close(get16(by, M * N), po.to_f32(ref), rtol=1e-2, atol=2e-3)
    c.close()


def test_elementwise(ctx, ops):
    n = 10007
    x = h(RNG.standard_normal(n) * 4)
    g = h(RNG.standard_normal(n))
    bx, bg, by = hb(ctx, x), hb(ctx, g), lssm.DeviceBuffer(ctx, n * 2)
    ref = np.zeros(n, np.uint16)
    po.lib().lssm_oracle_silu_f16(po.ptr(x.view(np.uint16)), po.ptr(ref), n)
    ops.silu_f16((bx, 0), (by, 0), n)
    assert ulp_close(get16(by, n), po.to_f32(ref))
    po.lib().lssm_oracle_silu_gated_f16(po.ptr(x.view(np.uint16)), po.ptr(g.view(np.uint16)), po.ptr(ref), n)
    ops.silu_gated_f16((bx, 0), (bg, 0), (by, 0), n)
    assert ulp_close(get16(by, n), po.to_f32(ref))
    yv = g.view(np.uint16).copy()
    po.lib().lssm_oracle_add_inplace_f16(po.ptr(yv), po.ptr(x.view(np.uint16)), n)
    ops.add_inplace_f16((bg, 0), (bx, 0), n)
    assert np.array_equal(bg.download(np.uint16, n), yv)   # one rounding of an exact sum: bit-exact


def test_split_silu(ctx, ops):
    L, di, N, G = 13, 64, 16, 2
    D = di + 2 * G * N
    xbc = h(RNG.standard_normal((L, D)) * 2)
    rx, rb, rc = np.zeros(L * di, np.uint16), np.zeros(L * G * N, np.uint16), np.zeros(L * G * N, np.uint16)
    po.lib().lssm_oracle_split_silu_xBC_f16(po.ptr(xbc.view(np.uint16)), po.ptr(rx), po.ptr(rb), po.ptr(rc), L, di, N, G)
    b = hb(ctx, xbc)
    ox, ob, oc = (lssm.DeviceBuffer(ctx, n * 2) for n in (L * di, L * G * N, L * G * N))
    ops.split_silu_xBC_f16((b, 0), (ox, 0), (ob, 0), (oc, 0), L, di, N, G)
    for o, r, n in ((ox, rx, L * di), (ob, rb, L * G * N), (oc, rc, L * G * N)):
        assert ulp_close(get16(o, n), po.to_f32(r))


@pytest.mark.parametrize("L,D,K", [(37, 300, 4), (1, 64, 4), (5, 17, 3)])
def test_causal_conv1d(ctx, ops, L, D, K):
    x = h(RNG.standard_normal((L, D)))
    w = h(RNG.uniform(-0.5, 0.5, (D, K)))
    bias = h(RNG.uniform(-0.5, 0.5, D))
    ref = np.zeros(L * D, np.uint16)
    po.lib().lssm_oracle_causal_conv1d_f16(*(po.ptr(a.view(np.uint16)) for a in (x, w, bias)), po.ptr(ref), 1, L, D, K)
    bx, bw, bb, by = hb(ctx, x), hb(ctx, w), hb(ctx, bias), lssm.DeviceBuffer(ctx, L * D * 2)
    ops.causal_conv1d_f16((bx, 0), (bw, 0), (bb, 0), (by, 0), lssm.Conv1dDims(1, L, D, K))
    close(get16(by, L * D), po.to_f32(ref), rtol=2e-3, atol=2e-3)
    # seed conv state from the last K rows (bit-exact copy, zero-padded when L < K)
    st = np.zeros(D * K, np.uint16)
    po.lib().lssm_oracle_seed_conv_state_f16(po.ptr(x.view(np.uint16)), po.ptr(st), L, D, K)
    bst = lssm.DeviceBuffer(ctx, D * K * 2)
    bst.upload(np.full(D * K, 0x3C00, np.uint16))
    ops.seed_conv_state_f16((bx, 0), (bst, 0), L, D, K)
    assert np.array_equal(bst.download(np.uint16, D * K), st)


def test_conv1d_update(ctx, ops):
    D, K = 1792, 4
    xn = h(RNG.standard_normal(D))
    state = h(RNG.standard_normal((D, K)))
    w = h(RNG.uniform(-0.5, 0.5, (D, K)))
    bias = h(RNG.uniform(-0.5, 0.5, D))
    rs, ry = state.view(np.uint16).copy(), np.zeros(D, np.uint16)
    po.lib().lssm_oracle_causal_conv1d_update_f16(po.ptr(xn.view(np.uint16)), po.ptr(rs), po.ptr(w.view(np.uint16)),
                                                  po.ptr(bias.view(np.uint16)), po.ptr(ry), 1, D, K)
    bx, bs, bw, bb, by = hb(ctx, xn), hb(ctx, state), hb(ctx, w), hb(ctx, bias), lssm.DeviceBuffer(ctx, D * 2)
    for _ in range(1):
        ops.causal_conv1d_update_f16((bx, 0), (bs, 0), (bw, 0), (bb, 0), (by, 0), lssm.Conv1dDims(1, 1, D, K))
    assert np.array_equal(bs.download(np.uint16, D * K), rs.ravel())
    close(get16(by, D), po.to_f32(ry), rtol=2e-3, atol=2e-3)


def test_inproj_fused(ctx, ops):
    L, dm, di, N, G, H, K = 11, 128, 256, 16, 2, 8, 4
    GN, xd = G * N, di + 2 * G * N
    proj = di + xd + H
    normed = h(RNG.standard_normal((L, dm)))
    W = h(RNG.standard_normal((proj, dm)) / np.sqrt(dm))
    Wc = h(RNG.uniform(-0.5, 0.5, (xd, K)))
    cb = h(RNG.uniform(-0.5, 0.5, xd))
    outs_ref = [np.zeros(n, np.uint16) for n in (L * di, L * di, L * GN, L * GN, L * H, L * xd)]
    po.lib().lssm_oracle_inproj_fused_f16(*(po.ptr(a.view(np.uint16)) for a in (normed, W, Wc, cb)),
                                          *(po.ptr(o) for o in outs_ref), L, dm, di, N, G, H, K)
    bufs = [lssm.DeviceBuffer(ctx, o.nbytes) for o in outs_ref]
    ins = [hb(ctx, a) for a in (normed, W, Wc, cb)]
    ops.inproj_fused_f16(*((b, 0) for b in ins), *((b, 0) for b in bufs),
                         lssm.FusedInProjDims(L, dm, di, N, G, H, K, proj))
    for b, r in zip(bufs, outs_ref):
        close(get16(b, r.size), po.to_f32(r), rtol=1e-2, atol=3e-3)


def _ssd_inputs(L, H, P, N, G, seed=0):
    r = np.random.default_rng(seed)
    X = h(r.standard_normal((L, H, P)))
    Bm = h(r.standard_normal((L, G, N)) * 0.5)
    Cm = h(r.standard_normal((L, G, N)) * 0.5)
    dt = h(r.standard_normal((L, H)) - 2)
    db = h(r.uniform(-0.5, 0.5, H))
    alog = h(np.log(r.uniform(1, 16, H)))
    D = h(r.standard_normal(H))
    return X, Bm, Cm, dt, db, alog, D


@pytest.mark.parametrize("H,P,N,G", [(80, 64, 128, 1), (8, 16, 16, 4), (3, 8, 12, 3)])
def test_ssd_step(ctx, ops, H, P, N, G):
    X, Bm, Cm, dt, db, alog, D = _ssd_inputs(1, H, P, N, G)
    S = (RNG.standard_normal((H, P, N)) * 0.3).astype(np.float32)
    rS, ry = S.copy(), np.zeros(H * P, np.uint16)
    po.lib().lssm_oracle_ssd_step_f16(*(po.ptr(a.view(np.uint16)) for a in (X, Bm, Cm, dt, db, alog, D)), po.ptr(rS),
                                      po.ptr(ry), H, P, N, G, 1e-6, 1e6, 1)
    ins = [hb(ctx, a) for a in (X, Bm, Cm, dt, db, alog, D)]
    bS, by = hb(ctx, S), lssm.DeviceBuffer(ctx, H * P * 2)
    ops.ssd_step_f16(*((b, 0) for b in ins[:7]), (bS, 0), (by, 0), lssm.SSDStepDims(H, P, N, G, 1e-6, 1e6, 1))
    close(bS.download(np.float32, H * P * N).reshape(H, P, N), rS, rtol=1e-5, atol=1e-5)
    close(get16(by, H * P), po.to_f32(ry), rtol=1e-2, atol=2e-3)


@pytest.mark.parametrize("Bt,H,P,N,G", [(5, 80, 64, 128, 1), (3, 16, 64, 128, 8), (2, 6, 16, 16, 2)])
def test_ssd_step_batched(ctx, Bt, H, P, N, G):
    """Batched-decode extension: each sequence against the oracle's one-sequence ssd_step."""
    ins = [_ssd_inputs(1, H, P, N, G, seed=10 + b) for b in range(Bt)]
    S = (RNG.standard_normal((Bt, H, P, N)) * 0.3).astype(np.float32)
    rS, ry = S.copy(), np.zeros((Bt, H * P), np.uint16)
    for b in range(Bt):
        X, Bm, Cm, dt, db, alog, D = ins[b]
        sb = np.ascontiguousarray(rS[b])
        yb = np.zeros(H * P, np.uint16)
        po.lib().lssm_oracle_ssd_step_f16(*(po.ptr(a.view(np.uint16)) for a in (X, Bm, Cm, dt, ins[0][4], ins[0][5],
                                                                                 ins[0][6])), po.ptr(sb), po.ptr(yb),
                                          H, P, N, G, 1e-6, 1e6, 1)
        rS[b], ry[b] = sb, yb
    cat = lambda k: np.ascontiguousarray(np.concatenate([ins[b][k].ravel() for b in range(Bt)]))  # noqa: E731
    bx, bB, bC, bdt = (hb(ctx, cat(k)) for k in (0, 1, 2, 3))
    bdb, bal, bD = (hb(ctx, ins[0][k]) for k in (4, 5, 6))
    bS, by = hb(ctx, S), lssm.DeviceBuffer(ctx, Bt * H * P * 2)
    dims = lssm.SSDBatchedDims(Bt, 1, H, P, N, G, 256, 1e-6, 1e6, 1, 0, 0, 0, 0)
    lssm.check(lssm.lib().lssm_ssd_step_batched(ctx.h, bx.ptr, bB.ptr, bC.ptr, bdt.ptr, bdb.ptr, bal.ptr, bD.ptr,
                                                bS.ptr, by.ptr, dims))
    close(bS.download(np.float32, Bt * H * P * N).reshape(Bt, H, P, N), rS, rtol=1e-5, atol=1e-5)
    close(get16(by, Bt * H * P).reshape(Bt, H * P), po.to_f32(ry), rtol=1e-2, atol=2e-3)


@pytest.mark.parametrize("L,H,P,N,G,chunk", [(77, 8, 64, 128, 1, 64), (40, 6, 16, 16, 2, 16), (1, 4, 8, 8, 1, 256),
                                             (300, 4, 64, 128, 1, 256)])
def test_ssd_chunked_f16(ctx, ops, L, H, P, N, G, chunk):
    X, Bm, Cm, dt, db, alog, D = _ssd_inputs(L, H, P, N, G, seed=L)
    S0 = (RNG.standard_normal((H, P, N)) * 0.2).astype(np.float32)
    # exact reference: token-by-token recurrence in double on the same fp16 inputs
    f = lambda a: np.ascontiguousarray(a.astype(np.float32))  # noqa: E731
    ye, se = np.zeros((1, L, H, P), np.float32), S0[None].copy()
    po.lib().lssm_oracle_ssd_sequential_f64(*(po.ptr(f(a)) for a in (X, Bm, Cm, dt, db, alog, D)), po.ptr(ye),
                                            po.ptr(se), 1, L, H, P, N, G, 1e-6, 1e6, 1)
    ins = [hb(ctx, a) for a in (X, Bm, Cm, dt, db, alog, D)]
    bS, bY = hb(ctx, S0), lssm.DeviceBuffer(ctx, L * H * P * 2)
    ops.ssd_chunked_f16(*((b, 0) for b in ins), (bY, 0), (bS, 0),
                        lssm.SSDDims(L, H, P, N, G, chunk, 1e-6, 1e6, 1))
    y = get16(bY, L * H * P).reshape(1, L, H, P)
    scale = np.abs(ye).max()
    assert np.abs(y - ye).max() <= 2e-3 * scale + 2e-3   # fp16 output rounding + fp32 accumulation
    s = bS.download(np.float32, H * P * N).reshape(1, H, P, N)
    # P=64/N=128 shapes run on the tensor-core kernel, whose state update multiplies fp16
    # operands (the decay-scaled B rows): a few fp16 ulps of max|S|.
    assert np.abs(s - se).max() <= 3e-3 * (1 + np.abs(se).max())


@pytest.mark.parametrize("xdt,G,L", [(lssm.DT_BF16, 1, 100), (lssm.DT_F16, 1, 100), (lssm.DT_BF16, 2, 300),
                                     (lssm.DT_F16, 2, 129)])
def test_ssd_chunked_batched_bf16_in_f32_out(ctx, ops, xdt, G, L):
    """P = 64, N = 128 runs on the tensor-core kernel: the intra-chunk weights M, the
    scaled C / B rows and the state snapshot are MMA operands in the input dtype, so the
    error vs the fp64 recurrence is a few input-dtype ulps of max|y| (bf16: 2^-8, fp16: 2^-11):
    tolerance 1.5e-2 (bf16) / 3e-3 (fp16) of max|y|; the fp32 state carry is tighter."""
    Bt, H, P, N = 2, 4, 64, 128
    r = np.random.default_rng(5)
    Xf = r.standard_normal((Bt, L, H, P)).astype(np.float32)
    Bf = r.standard_normal((Bt, L, G, N)).astype(np.float32)
    Cf = r.standard_normal((Bt, L, G, N)).astype(np.float32)
    dtf = (r.standard_normal((Bt, L, H)) - 2).astype(np.float32)
    alog = np.log(r.uniform(1, 16, H)).astype(np.float32)
    D = r.standard_normal(H).astype(np.float32)
    zero = np.zeros(H, np.float32)

    def cast(a):
        if xdt == lssm.DT_BF16:
            u = a.view(np.uint32)
            bits = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
            return bits, (bits.astype(np.uint32) << 16).view(np.float32)
        a16 = a.astype(np.float16)
        return a16.view(np.uint16), a16.astype(np.float32)

    (Xb, Xr), (Bb, Br), (Cb, Cr) = cast(Xf), cast(Bf), cast(Cf)
    ye, se = np.zeros((Bt, L, H, P), np.float32), np.zeros((Bt, H, P, N), np.float32)
    po.lib().lssm_oracle_ssd_sequential_f64(*(po.ptr(np.ascontiguousarray(a)) for a in (Xr, Br, Cr, dtf, zero, alog, D)),
                                            po.ptr(ye), po.ptr(se), Bt, L, H, P, N, G, 1e-6, 1e6, 1)
    bufs = [hb(ctx, a) for a in (Xb, Bb, Cb, dtf, zero, alog, D)]
    bY, bS = lssm.DeviceBuffer(ctx, ye.nbytes), hb(ctx, np.zeros_like(se))
    ops.ssd_chunked_batched(*bufs, bY, bS, lssm.SSDBatchedDims(Bt, L, H, P, N, G, 256, 1e-6, 1e6, 1, xdt,
                                                               lssm.DT_F32, lssm.DT_F32, lssm.DT_F32))
    y = bY.download(np.float32, ye.size).reshape(ye.shape)
    tol = 1.5e-2 if xdt == lssm.DT_BF16 else 3e-3
    assert np.abs(y - ye).max() <= tol * np.abs(ye).max()
    s = bS.download(np.float32, se.size).reshape(se.shape)
    assert np.abs(s - se).max() <= tol * np.abs(se).max()


def test_graph_batching_replay(ctx, ops):
    """A captured batch replays the same ops on the same buffers (y += x, three times)."""
    n = 3000
    x = h(RNG.standard_normal(n))
    bx, by = hb(ctx, x), hb(ctx, np.zeros(n, np.float16))
    ctx.set_graph_batching(True)
    ctx.begin_batch()
    ops.add_inplace_f16((by, 0), (bx, 0), n)
    ctx.commit_and_wait()            # runs once
    ctx.replay_batch(2)              # twice more
    ctx.set_graph_batching(False)
    ctx.begin_batch()
    ctx.commit_and_wait()            # plain batch: synchronises the stream
    s = x.astype(np.float32)
    ref = np.float16(np.float16(s + s) + s).astype(np.float32)
    assert np.array_equal(get16(by, n), ref)
    with pytest.raises(lssm.LssmError, match="a batch is active"):
        ctx.begin_batch()
        try:
            ctx.set_graph_batching(True)
        finally:
            ctx.commit_and_wait()


def test_batching_semantics(ctx, ops):
    n = 4096
    x = h(RNG.standard_normal(n))
    bx, by = hb(ctx, x), lssm.DeviceBuffer(ctx, n * 2)
    ctx.begin_batch()
    assert ctx.batch_active()
    with pytest.raises(lssm.LssmError, match="already active"):
        ctx.begin_batch()
    ops.silu_f16((bx, 0), (by, 0), n)
    ops.add_inplace_f16((by, 0), (bx, 0), n)
    ctx.commit_and_wait()
    assert not ctx.batch_active()
    with pytest.raises(lssm.LssmError, match="without an active batch"):
        ctx.commit_and_wait()
    s = x.astype(np.float32)
    silu = (s / (1 + np.exp(-s))).astype(np.float16).astype(np.float32)
    assert ulp_close(get16(by, n), silu + s, ulps=2)
