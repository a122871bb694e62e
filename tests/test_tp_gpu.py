"""GPU: the head-tensor-parallel session (lssm_session_create_tp) through the C ABI.

* one rank (a world-1 communicator, no NCCL): the sharded path with its fp32 out_proj
  partials, all-reduced sum of squares and (value, index) argmax merge must give the
  normal session's greedy tokens and logits;
* two ranks on two GPUs (skipped with fewer): NCCL all-reduces over NVLink; tokens and
  logits against the fp16-faithful oracle with the model test's criteria (logits < 0.1,
  greedy ids equal up to near-ties inside that tolerance).
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
    toks, pre, last = _run(lssm.Session(ctx, model, batch=2, max_seq_len=PROMPTS.shape[1], comm=comm))
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), toks=toks, pre=pre, last=last)
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
    for k in ("toks", "pre", "last"):
        assert np.array_equal(r0[k], r1[k]), k  # every rank holds the same tokens and gathered logits
    ora = po.OracleModel(path, mode=0)
    for b in range(2):
        toks = r0["toks"][b]
        otoks, opre, ostep = ora.generate(PROMPTS[b], N_NEW, teacher=toks)
        assert np.abs(r0["pre"][b] - opre).max() < 0.1
        assert np.abs(r0["last"][b] - ostep[N_NEW - 2]).max() < 0.1
        rows = np.concatenate([opre[None], ostep])
        for i, (a, o) in enumerate(zip(toks, otoks)):
            assert a == o or abs(rows[i][a] - rows[i][o]) <= 0.1
