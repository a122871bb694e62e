"""GPU: lssm_inproj_fused_f16_noalloc, the fused in_proj op for callers that cannot
allocate device memory when they call it (their own allocator owns the memory budget,
or an allocation would block the device mid-request). It must produce the same outputs
as lssm_inproj_fused_f16, which allocates its scratch on demand, on two calls in a row
(the static scratch keeps the previous call's contents), and reject a request larger
than its fixed scratch.

This file is named to be collected last, so a stop-at-first-failure run has already
run every other test when it gets here; it also passes alone in a fresh process.
"""

import ctypes as C

import numpy as np
import pytest

import lssm

pytestmark = pytest.mark.gpu


def _call(ctx, name, ins, outs, dims):
    args = []
    for b in list(ins) + list(outs):
        args += [b.ptr, 0]
    lssm.check(getattr(lssm.lib(), name)(ctx.h, *args, dims))


def _dev(ctx, a):
    return lssm.DeviceBuffer.from_array(ctx, np.ascontiguousarray(a))


def test_noalloc_matches_allocating_entry_point():
    ctx = lssm.Ctx(0)
    rng = np.random.default_rng(21)
    tols = dict(rtol=0, atol=0)   # same kernels on the same inputs: identical bits expected
    for L, dm, di, N, G, H, K in ((11, 128, 256, 16, 2, 8, 4), (16, 768, 1536, 128, 1, 24, 4)):
        GN, xd = G * N, di + 2 * G * N
        proj = di + xd + H
        dims = lssm.FusedInProjDims(L, dm, di, N, G, H, K, proj)
        for call in range(2):   # two calls in a row: the second reuses the static scratch
            normed = rng.standard_normal((L, dm)).astype(np.float16)
            W = (rng.standard_normal((proj, dm)) / np.sqrt(dm)).astype(np.float16)
            Wc = rng.uniform(-0.5, 0.5, (xd, K)).astype(np.float16)
            cb = rng.uniform(-0.5, 0.5, xd).astype(np.float16)
            ins = [_dev(ctx, a) for a in (normed, W, Wc, cb)]
            sizes = (L * di, L * di, L * GN, L * GN, L * H, L * xd)
            ref_out = [lssm.DeviceBuffer(ctx, n * 2) for n in sizes]
            new_out = [lssm.DeviceBuffer(ctx, n * 2) for n in sizes]
            _call(ctx, "lssm_inproj_fused_f16", ins, ref_out, dims)
            _call(ctx, "lssm_inproj_fused_f16_noalloc", ins, new_out, dims)
            for r, n, cnt in zip(ref_out, new_out, sizes):
                a = r.download(np.float16, cnt).astype(np.float32)
                b = n.download(np.float16, cnt).astype(np.float32)
                np.testing.assert_allclose(b, a, **tols)
    ctx.close()


def test_noalloc_leaves_device_memory_unchanged():
    """After the first call on the device (which looks up the array's address and makes
    the driver load the module that holds it), further calls take no device memory:
    cudaMemGetInfo's free bytes are the same before and after them. An L == 0 call
    returns through the same completion checks as the other ops."""
    import torch

    ctx = lssm.Ctx(0)
    rng = np.random.default_rng(5)
    L, dm, di, N, G, H, K = 16, 768, 1536, 128, 1, 24, 4
    GN, xd = G * N, di + 2 * G * N
    proj = di + xd + H
    dims = lssm.FusedInProjDims(L, dm, di, N, G, H, K, proj)
    ins = [_dev(ctx, a) for a in (rng.standard_normal((L, dm)).astype(np.float16),
                                  (rng.standard_normal((proj, dm)) / np.sqrt(dm)).astype(np.float16),
                                  rng.uniform(-0.5, 0.5, (xd, K)).astype(np.float16),
                                  rng.uniform(-0.5, 0.5, xd).astype(np.float16))]
    outs = [lssm.DeviceBuffer(ctx, n * 2) for n in (L * di, L * di, L * GN, L * GN, L * H, L * xd)]
    _call(ctx, "lssm_inproj_fused_f16_noalloc", ins, outs, dims)       # first call: set-up
    torch.cuda.synchronize(0)
    free0, _ = torch.cuda.mem_get_info(0)
    for _ in range(3):
        _call(ctx, "lssm_inproj_fused_f16_noalloc", ins, outs, dims)
    _call(ctx, "lssm_inproj_fused_f16_noalloc", ins, outs, lssm.FusedInProjDims(0, dm, di, N, G, H, K, proj))
    torch.cuda.synchronize(0)
    free1, _ = torch.cuda.mem_get_info(0)
    assert free1 == free0, f"device free memory changed by {free0 - free1} bytes across no-allocation calls"
    ctx.close()


def test_noalloc_rejects_requests_beyond_its_scratch():
    ctx = lssm.Ctx(0)
    buf = lssm.DeviceBuffer(ctx, 64)
    # L * proj_dim * 4 bytes above the 4 MiB static scratch (proj_dim 70000, L 16)
    di, N, G, H = 60000, 128, 1, 9744
    proj = di + di + 2 * G * N + H
    dims = lssm.FusedInProjDims(16, 256, di, N, G, H, 4, proj)
    with pytest.raises(lssm.LssmError, match="exceeds the"):
        _call(ctx, "lssm_inproj_fused_f16_noalloc", [buf] * 4, [buf] * 6, dims)
    ctx.close()
    _ = C
