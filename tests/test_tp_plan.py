"""CPU: head tensor parallelism decomposes the Mamba-2 model exactly (up to fp32 summation
order). Each of two `gloo` ranks takes the rows / columns `lssm.tp_shard_plan` assigns it
(the copy plan lssm_session_create_tp performs on the device), runs the block with the
two all-reduces of the device path (sum of squares of the gated slice, fp32 out_proj
partials) and the vocab-split lm_head with an all-gather, and must reproduce the
single-rank model's prefill and decode logits and greedy tokens.

The model arithmetic is a plain fp32 numpy statement of the block
(src/model/mamba2_block.cpp:170-289 of the reference: in_proj -> causal conv + SiLU ->
selective scan -> gate -> RMSNorm over d_inner -> out_proj -> residual), shared by the
full and the sharded runs, so the comparison isolates the decomposition.
"""

import os
import socket

import numpy as np
import pytest

import lssm
import pyoracle as po

EPS = 1e-5


def _load(path):
    buf = open(path, "rb").read()
    hdr, t = po.parse_ssm(buf)
    raw = np.frombuffer(buf, dtype=np.uint8)

    def get(name):
        ti = t[name]
        blob = raw[ti.offset:ti.offset + ti.nbytes]
        if ti.dtype == po.DTYPE_INT4_B32:
            N, K = ti.shape
            packed = np.ascontiguousarray(blob[:N * K // 2]).reshape(N, K // 2)
            scales = np.ascontiguousarray(blob[N * K // 2:]).view(np.uint16).reshape(N, K // 32)
            out = np.zeros((N, K), dtype=np.float32)
            po.lib().lssm_oracle_int4_dequant(po.ptr(packed), po.ptr(scales), po.ptr(out), N, K)
            return out
        return blob.view(np.float16).astype(np.float32).reshape(ti.shape)

    hp = dict(d_model=hdr.d_model, n_layer=hdr.n_layer, d_state=hdr.d_state, d_conv=hdr.d_conv,
              expand=hdr.expand, vocab_size=hdr.vocab_size, n_heads=hdr.n_heads, d_head=hdr.d_head,
              chunk_size=hdr.chunk_size, n_groups=hdr.n_groups)
    W = {"embed": get("backbone.embeddings.weight"), "norm_f": get("backbone.norm_f.weight"),
         "lm_head": get("lm_head.weight" if "lm_head.weight" in t else "backbone.embeddings.weight"), "layers": []}
    for i in range(hdr.n_layer):
        p = f"backbone.layers.{i}."
        W["layers"].append({k: get(p + n) for k, n in (
            ("norm", "norm.weight"), ("in_w", "mixer.in_proj.weight"), ("conv_w", "mixer.conv1d.weight"),
            ("conv_b", "mixer.conv1d.bias"), ("dt_bias", "mixer.dt_bias"), ("A_log", "mixer.A_log"),
            ("D", "mixer.D"), ("mixer_norm", "mixer.norm.weight"), ("out_w", "mixer.out_proj.weight"))})
    return hp, W


def _shard(hp, W, rank, world):
    """This rank's copy of the weights under lssm.tp_shard_plan."""
    plan = lssm.tp_shard_plan(hp, rank, world)
    cat = lambda a, segs: np.concatenate([a[o:o + n] for o, n in segs], axis=0)  # noqa: E731
    h0, hn = plan["heads"]
    c0, cn = plan["inner_cols"]
    v0, vn = plan["vocab"]
    out = {"embed": W["embed"], "norm_f": W["norm_f"], "lm_head": W["lm_head"][v0:v0 + vn], "layers": []}
    for L in W["layers"]:
        out["layers"].append({
            "norm": L["norm"], "in_w": cat(L["in_w"], plan["in_rows"]),
            "conv_w": cat(L["conv_w"].reshape(L["conv_w"].shape[0], -1), plan["conv_channels"]),
            "conv_b": cat(L["conv_b"], plan["conv_channels"]),
            "dt_bias": L["dt_bias"][h0:h0 + hn], "A_log": L["A_log"][h0:h0 + hn], "D": L["D"][h0:h0 + hn],
            "mixer_norm": L["mixer_norm"][c0:c0 + cn], "out_w": L["out_w"][:, c0:c0 + cn]})
    return out, plan


def _rms(x, w, sumsq=None, dim=None):
    ss = (x * x).sum(-1, keepdims=True) if sumsq is None else sumsq
    return x * w / np.sqrt(ss / (dim or x.shape[-1]) + EPS)


def _silu(x):
    return x / (1.0 + np.exp(-x))


def _softplus(x):
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


class Runner:
    """fp32 model over (possibly sharded) weights; `ar` all-reduces a float32 array in
    place across ranks, `ag` all-gathers a float32 array along the last axis."""

    def __init__(self, hp, W, world=1, ar=None, ag=None):
        self.hp, self.W, self.world = hp, W, world
        self.ar = ar or (lambda a: a)
        self.ag = ag or (lambda a: a)
        H = hp["n_heads"] // world
        G = hp["n_groups"] // world
        self.H, self.G, self.P, self.N = H, G, hp["d_head"], hp["d_state"]
        self.di_total = hp["expand"] * hp["d_model"]
        self.di = H * self.P
        self.xd = self.di + 2 * G * self.N
        K = hp["d_conv"]
        self.conv = [np.zeros((self.xd, K), np.float32) for _ in W["layers"]]
        self.ssd = [np.zeros((H, self.P, self.N), np.float32) for _ in W["layers"]]

    def block(self, l, hid):
        L = self.W["layers"][l]
        di, xd, H, G, P, N = self.di, self.xd, self.H, self.G, self.P, self.N
        K = self.hp["d_conv"]
        proj = _rms(hid, L["norm"]) @ L["in_w"].T
        z, xbc, dt = proj[:, :di], proj[:, di:di + xd], proj[:, di + xd:]
        cw = L["conv_w"].reshape(xd, K)
        ys = np.zeros((hid.shape[0], di), np.float32)
        A = -np.exp(L["A_log"])
        for t in range(hid.shape[0]):
            st = self.conv[l]
            st[:, :-1] = st[:, 1:]
            st[:, -1] = xbc[t]
            c = _silu((st * cw).sum(1) + L["conv_b"])
            x, B, C = c[:di].reshape(H, P), c[di:di + G * N].reshape(G, N), c[di + G * N:].reshape(G, N)
            d = np.clip(_softplus(dt[t] + L["dt_bias"]), 1e-6, 1e6)
            g = np.arange(H) // (H // G)
            S = self.ssd[l]
            S[:] = np.exp(A * d)[:, None, None] * S + (d[:, None] * x)[:, :, None] * B[g][:, None, :]
            ys[t] = ((S * C[g][:, None, :]).sum(-1) + L["D"][:, None] * x).reshape(-1)
        gated = _silu(z) * ys
        ss = self.ar((gated * gated).sum(-1, keepdims=True).astype(np.float32))
        mo = _rms(gated, L["mixer_norm"], ss, self.di_total)
        return hid + self.ar((mo @ L["out_w"].T).astype(np.float32))

    def forward(self, toks):
        hid = self.W["embed"][np.asarray(toks)]
        for l in range(len(self.W["layers"])):
            hid = self.block(l, hid)
        last = _rms(hid[-1:], self.W["norm_f"])
        return self.ag((last @ self.W["lm_head"].T).astype(np.float32))[0]


def _generate(runner, prompt, n_new):
    logits = [runner.forward(prompt)]
    toks = [int(np.argmax(logits[-1]))]
    for _ in range(n_new - 1):
        logits.append(runner.forward([toks[-1]]))
        toks.append(int(np.argmax(logits[-1])))
    return np.stack(logits), toks


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, path, prompt, n_new, out_dir):
    import torch
    import torch.distributed as dist

    os.environ["OMP_NUM_THREADS"] = "1"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        hp, W = _load(path)
        Ws, plan = _shard(hp, W, rank, world)

        def ar(a):
            t = torch.from_numpy(np.ascontiguousarray(a))
            dist.all_reduce(t)
            return t.numpy()

        vmax = -(-hp["vocab_size"] // world)

        def ag(a):
            pad = np.full(a.shape[:-1] + (vmax,), -np.inf, np.float32)
            pad[..., :a.shape[-1]] = a
            parts = [torch.empty_like(torch.from_numpy(pad)) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(pad))
            return np.concatenate([p.numpy() for p in parts], -1)[..., :hp["vocab_size"]]

        logits, toks = _generate(Runner(hp, Ws, world, ar, ag), prompt, n_new)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), logits=logits, toks=np.array(toks))
    finally:
        dist.destroy_process_group()


def test_shard_plan_covers_every_row_once():
    hp = dict(d_model=4096, n_layer=56, d_state=128, d_conv=4, expand=2, vocab_size=256000, n_heads=128,
              d_head=64, chunk_size=256, n_groups=8)
    di, GN, H = 8192, 8 * 128, 128
    proj = 2 * di + 2 * GN + H
    for world in (1, 2, 4, 8):
        rows, cols, vocab, heads = [], [], [], []
        for r in range(world):
            p = lssm.tp_shard_plan(hp, r, world)
            rows += [i for o, n in p["in_rows"] for i in range(o, o + n)]
            cols += list(range(p["inner_cols"][0], sum(p["inner_cols"])))
            vocab += list(range(p["vocab"][0], sum(p["vocab"])))
            heads += list(range(p["heads"][0], sum(p["heads"])))
        assert sorted(rows) == list(range(proj))
        assert sorted(cols) == list(range(di)) and sorted(heads) == list(range(H))
        assert sorted(vocab) == list(range(hp["vocab_size"]))
    with pytest.raises(ValueError):
        lssm.tp_shard_plan(dict(hp, n_groups=1), 0, 2)


@pytest.mark.parametrize("name", ["tinyB_fp16", "tinyB_int4"])
def test_tp2_matches_single_rank_gloo(golden, tmp_path, name):
    import torch.multiprocessing as mp

    path = str(golden / f"{name}.ssm")
    prompt = [5, 17, 3, 250, 99, 1, 42, 7, 64, 128, 11]
    n_new = 4
    hp, W = _load(path)
    ref_logits, ref_toks = _generate(Runner(hp, W), prompt, n_new)
    mp.start_processes(_rank_main, args=(2, _free_port(), path, prompt, n_new, str(tmp_path)), nprocs=2,
                       start_method="spawn")
    for r in range(2):
        got = np.load(tmp_path / f"rank{r}.npz")
        assert list(got["toks"]) == ref_toks
        # fp32 with a different summation order (per-rank partial sums): relative 1e-4
        np.testing.assert_allclose(got["logits"], ref_logits, rtol=1e-4, atol=1e-4 * np.abs(ref_logits).max())


@pytest.mark.parametrize("name", ["tinyB_fp16", "tinyB_int4"])
def test_numpy_model_matches_fp32_oracle(golden, name):
    """The shared fp32 statement used above is the oracle's fp32 model (mode 1)."""
    path = golden / f"{name}.ssm"
    prompt = [5, 17, 3, 250, 99, 1, 42, 7, 64, 128, 11]
    hp, W = _load(str(path))
    logits, toks = _generate(Runner(hp, W), prompt, 4)
    o_toks, o_pl, o_sl = po.OracleModel(path, mode=1).generate(np.array(prompt), 4)
    assert toks == [int(t) for t in o_toks]
    scale = np.abs(o_pl).max()
    np.testing.assert_allclose(logits[0], o_pl, atol=1e-5 * scale)
    np.testing.assert_allclose(logits[1:], o_sl, atol=1e-5 * scale)
