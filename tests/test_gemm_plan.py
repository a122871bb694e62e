"""CPU: the launch plan of the fused INT4 GEMM (lssm_plan_int4_gemm, the host function the
launcher uses), over decode, batched and prefill shapes: which shapes the fused kernel takes,
the N tile, and the K split at decode-size M, against the plan's invariants and the choices
measured on B200 for the batched in_proj / out_proj."""

import ctypes as C
import itertools

import pytest

import lssm

SMS = 148


def plan(M, N, K, ws_bytes, sms=SMS):
    bn, sp = C.c_uint32(), C.c_uint32()
    fused = lssm.lib().lssm_plan_int4_gemm(M, N, K, sms, ws_bytes, C.byref(bn), C.byref(sp))
    return fused, bn.value, sp.value


def unit(tile, m_tiles, n_tiles, splits, nk):
    out = (C.c_uint32 * 5)()
    lssm.lib().lssm_int4_gemm_unit(tile, m_tiles, n_tiles, splits, nk, out)
    return tuple(out)


def k_ranges(nk, splits, m_tiles=1, n_tiles=1):
    """K-block range of each split, from the kernel's own unit function (every (m, n) tile
    of a split gets the same range)."""
    mn = m_tiles * n_tiles
    r = []
    for s in range(splits):
        units = [unit(s * mn + t, m_tiles, n_tiles, splits, nk) for t in range(mn)]
        assert len({u[3:] for u in units}) == 1 and all(u[2] == s for u in units)
        assert sorted((u[0], u[1]) for u in units) == [(m, n) for m in range(m_tiles) for n in range(n_tiles)]
        r.append(units[0][3:])
    return r


@pytest.mark.parametrize("M,N,K,bn,splits", [
    (64, 10576, 2560, 256, 3),    # batched in_proj: 42 N tiles x 3 splits = 126 CTAs
    (64, 2560, 5120, 128, 7),     # batched out_proj: 20 N tiles x 7 splits = 140 CTAs
    (64, 5120, 5120, 256, 7),
    (16, 10576, 2560, 256, 3),
])
def test_measured_choices(M, N, K, bn, splits):
    assert plan(M, N, K, 8 * M * N * 4) == (1, bn, splits)


def test_without_scratch_no_split():
    # no workspace: no split; out_proj's 40 N tiles are then too few for the fused kernel
    assert plan(64, 10576, 2560, 0) == (1, 128, 1)
    assert plan(64, 2560, 5120, 0)[0] == 0


def test_not_taken():
    assert plan(100, 300, 256, 1 << 30)[0] == 0     # one K group: no split, too few N tiles
    assert plan(17, 33, 96, 1 << 30)[0] == 0        # K % 256
    assert plan(513, 10576, 2560, 1 << 30)[0] == 0  # beyond a few M tiles: dequantise once
    assert plan(2048, 10576, 2560, 1 << 30)[0] == 0


@pytest.mark.parametrize("M,N,K", list(itertools.product(
    [1, 9, 16, 33, 64, 100, 128, 129, 256, 512], [300, 1000, 2560, 4810, 5120, 10576, 50288],
    [256, 768, 2560, 5120])))
def test_plan_invariants(M, N, K):
    for ws in (0, 1 << 20, 8 * M * N * 4):
        fused, bn, sp = plan(M, N, K, ws)
        if not fused:
            assert bn == 0 and sp == 1
            continue
        assert bn in (64, 128, 256) and M <= 512 and K % 256 == 0
        tiles = -(-M // 128) * -(-N // bn)
        if sp == 1:
            assert (N + 63) // 64 >= SMS // 2
            continue
        assert M <= 128 and ws > 0
        assert 2 <= sp <= min(8, K // 256)
        assert sp * M * N * 4 <= ws              # partials fit the scratch
        assert tiles * sp <= SMS                  # one wave of CTAs
        r = k_ranges(K // 64, sp, -(-M // 128), -(-N // bn))   # every K block in exactly one split
        assert all(a % 4 == 0 for a, _ in r)      # splits start on 256-wide scale groups
        assert r[0][0] == 0 and r[-1][1] == K // 64
        assert all(a < b for a, b in r) and all(r[i][1] == r[i + 1][0] for i in range(sp - 1))


def test_split_needs_room_for_two_partials():
    """Splitting K needs ws_bytes >= 2*M*N*4 (the fp32 partials of two splits)."""
    M, N, K = 64, 10576, 2560
    assert plan(M, N, K, 2 * M * N * 4)[2] >= 2
    assert plan(M, N, K, 2 * M * N * 4 - 16)[2] == 1


# ---------------------------------------------------------------------------
# fp16 tensor-core GEMM: the N tile the launcher picks (lssm_plan_gemm_f16, its own function)
def tile_f16(M, N, sms=SMS):
    return lssm.lib().lssm_plan_gemm_f16(M, N, sms)


def test_f16_gemm_tiles_of_the_2p7b_prefill():
    """2048-token prefill: in_proj (N 10576) takes 240-wide tiles (720 tiles = 4.86 waves on 148 SMs;
    256 would leave 672 = 4.54 waves), out_proj (N 2560) 144-wide ones (288 tiles = 1.95 waves; 160
    gives 256 = 1.73)."""
    assert tile_f16(2048, 10576) == 240
    assert tile_f16(2048, 2560) == 144


@pytest.mark.parametrize("M,N", [(2048, 10576), (2048, 2560), (512, 1024), (200, 300), (16384, 2320), (16384, 4096),
                                 (1, 16), (4096, 18560)])
def test_f16_gemm_tile_is_a_compiled_width_with_best_fill(M, N):
    bn = tile_f16(M, N)
    assert bn in (128, 144, 160, 192, 240, 256)
    # no other width fills the persistent waves better without a lower shared-memory factor
    def fill(c):
        tiles = -(-M // 128) * -(-N // c)
        waves = -(-tiles // SMS)
        return M * N / (waves * SMS * 128 * c)
    assert fill(bn) >= 0.8 * max(fill(c) for c in (128, 144, 160, 192, 240, 256))
