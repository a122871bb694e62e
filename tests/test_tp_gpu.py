"""GPU: the head-tensor-parallel session (lssm_session_create_tp) through the C ABI.

* one rank (a world-1 communicator, no NCCL): the sharded path with its fp32 out_proj
  partials, all-reduced sum of squares and (value, index) argmax merge must give the
  normal session's greedy tokens and logits;
* two ranks on two GPUs (skipped with fewer): decode all-reduces over the peer-memory
  exchange and over NCCL; tokens and logits against the fp16-faithful oracle with the model
  test's criteria (logits < 0.1, greedy ids equal up to near-ties inside that tolerance), and
  the two exchanges against each other;
* the exchange's bounded wait, run out on one GPU against a flag nothing sets.
"""

import os

import numpy as np
import pytest

import lssm
import pyoracle as po

pytestmark = pytest.mark.gpu

PROMPTS = np.array([[5, 17, 3, 250, 99, 1, 42, 7, 64, 128, 11, 200],
                    [9, 8, 7, 6, 5, 4, 3, 2, 1, 100, 101, 102]], dtype=np.uint32)
N_NEW = 6


def _run(sess):
    first = sess.prefill(PROMPTS)
    pre = sess.logits()
    rest = sess.decode(first, N_NEW - 1)
    return np.concatenate([first[:, None], rest], 1), pre, sess.logits()


@pytest.mark.parametrize("name", ["tinyB_fp16", "tinyB_int4"])
def test_tp_world1_matches_session(ctx, golden, name):
    model = lssm.Model.load(ctx, golden / f"{name}.ssm")
    ref = _run(lssm.Session(ctx, model, batch=2, max_seq_len=PROMPTS.shape[1]))
    comm = lssm.Comm(ctx, 0, 1, bytes(lssm.COMM_ID_BYTES))
    got = _run(lssm.Session(ctx, model, batch=2, max_seq_len=PROMPTS.shape[1], comm=comm))
    assert np.array_equal(got[0], ref[0])
    assert np.abs(got[1] - ref[1]).max() < 0.02
    assert np.abs(got[2] - ref[2]).max() < 0.02


def _tp_rank(rank, world, uid, path, out_dir):
    ctx = lssm.Ctx(rank)
    comm = lssm.Comm(ctx, rank, world, uid)
    model = lssm.Model.load(ctx, path)
    res = {}
    for p2p in (1, 0):
        sess = lssm.Session(ctx, model, batch=2, max_seq_len=PROMPTS.shape[1], comm=comm)
        sess.set_option("tp_p2p", p2p)
        toks, pre, last = _run(sess)
        res.update({f"toks{p2p}": toks, f"pre{p2p}": pre, f"last{p2p}": last})
        sess.close()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **res)
    ctx.close()


@pytest.mark.parametrize("name", ["tinyB_fp16", "tinyB_int4"])
def test_tp2_matches_oracle(golden, tmp_path, name):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    path = str(golden / f"{name}.ssm")
    uid = lssm.Comm.unique_id()
    mp.start_processes(_tp_rank, args=(2, uid, path, str(tmp_path)), nprocs=2, start_method="spawn")
    r0, r1 = (np.load(tmp_path / f"rank{r}.npz") for r in range(2))
    for k in ("toks1", "pre1", "last1", "toks0", "pre0", "last0"):
        assert np.array_equal(r0[k], r1[k]), k  # every rank holds the same tokens and gathered logits
    # peer exchange vs NCCL: same sums (two ranks, one addition), prefill identical
    assert np.array_equal(r0["toks1"], r0["toks0"])
    assert np.array_equal(r0["pre1"], r0["pre0"])
    assert np.abs(r0["last1"] - r0["last0"]).max() < 2e-2
    ora = po.OracleModel(path, mode=0)
    for b in range(2):
        toks = r0["toks1"][b]
        otoks, opre, ostep = ora.generate(PROMPTS[b], N_NEW, teacher=toks)
        assert np.abs(r0["pre1"][b] - opre).max() < 0.1
        assert np.abs(r0["last1"][b] - ostep[N_NEW - 2]).max() < 0.1
        rows = np.concatenate([opre[None], ostep])
        for i, (a, o) in enumerate(zip(toks, otoks)):
            assert a == o or abs(rows[i][a] - rows[i][o]) <= 0.1


def test_peer_exchange_wait_times_out(ctx, golden):
    """The exchange kernel's flag wait is bounded: with a flag nothing sets it gives up after
    the limit, the host gets LSSM_ERR_TIMEOUT, and the context keeps working."""
    with pytest.raises(lssm.LssmError, match="timed out"):
        lssm.check(lssm.lib().lssm_p2p_wait_selftest(ctx.h, 20_000_000))
    model = lssm.Model.load(ctx, golden / "tinyB_fp16.ssm")
    out = lssm.Session(ctx, model, batch=1, max_seq_len=8).generate(np.array([[1, 2, 3]], np.uint32), 3)
    assert out.shape == (1, 3)


def _ar_rank(rank, world, uid, out_dir):
    import torch

    torch.cuda.set_device(rank)
    ctx = lssm.Ctx(rank)
    comm = lssm.Comm(ctx, rank, world, uid)
    res = {}
    for n in (1000, 16384, 200000):   # peer exchange (ragged / decode size), NCCL (large)
        x = torch.arange(n, device="cuda", dtype=torch.float32) * (rank + 1) + 0.25 * rank
        torch.cuda.synchronize()
        comm.allreduce_f32(x.data_ptr(), n)
        comm.allreduce_f32(x.data_ptr(), n)   # a second call: next epoch, other parity
        res[f"n{n}"] = x.cpu().numpy()
    np.savez(os.path.join(out_dir, f"ar{rank}.npz"), **res)
    comm.close()
    ctx.close()


def test_comm_allreduce_two_ranks(tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    uid = lssm.Comm.unique_id()
    mp.start_processes(_ar_rank, args=(2, uid, str(tmp_path)), nprocs=2, start_method="spawn")
    for n in (1000, 16384, 200000):
        base = np.arange(n, dtype=np.float32)
        once = base * 1 + base * 2 + np.float32(0.25)        # rank 0 + rank 1
        want = once * 2                                       # summed again
        for r in range(2):
            got = np.load(tmp_path / f"ar{r}.npz")[f"n{n}"]
            np.testing.assert_allclose(got, want, rtol=1e-6)
