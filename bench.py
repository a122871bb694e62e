"""Benchmark of the B200 Mamba-2 hot path (the headline metric: 2.7B-shape INT4
decode / prefill tokens per second, with roofline fractions).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload decode27b|batched|tp8b]

Default workload (N=1): the Mamba-2 2.7B shape (64 layers, d_model 2560, d_inner 5120,
80 heads x 64, d_state 128, ngroups 1, vocab 50288), in_proj/out_proj packed INT4_B32 as
the reference exporter writes them, random init from seed 0; one step = one request:
prefill 2048 random prompt ids + 512 greedy decode tokens, batch 1. `value` is decode
tokens/s (whole job), `prefill_tok_s` the prefill rate. Under torchrun each rank serves
its own independent request (sequences sharded across GPUs, no data-path collective):
weak scaling. Timing: W untimed steps, then K steps bracketed by a barrier and a device
synchronize; prefill and decode are timed with CUDA events on the engine's stream; the
max over ranks is reported. `e2e` repeats the request through the C ABI call with the
prompt in pinned host memory and the generated ids copied back, timed on the host.

The default line also carries `sharded_workloads`: at every N, on the same ranks, the two
workloads that shard across GPUs (strong scaling, 1 warm-up + 2 timed steps each): the
64-sequence batched decode with the sequences split over the GPUs, and the 8B shape with
its heads tensor-parallel over all N GPUs (TP8 at N = 8).

--impl reference times the reference's math on the host CPU (the reference has no CPU
compute path of its own: its kernels are Metal shaders; the oracle under oracle/ is the
C++ restatement of them) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "lite-ssm_b200"))

METRIC = "decode tok/s & prefill tok/s (2.7B quant) at 1/2/4/8 B200; % HBM/tensor roofline"
HP27 = dict(d_model=2560, n_layer=64, d_state=128, d_conv=4, expand=2, vocab_size=50288, n_heads=80, d_head=64,
            chunk_size=256, n_groups=1, norm_before_gate=0)
HP8B = dict(d_model=4096, n_layer=56, d_state=128, d_conv=4, expand=2, vocab_size=256000, n_heads=128, d_head=64,
            chunk_size=256, n_groups=8, norm_before_gate=0)
PROMPT, NEW = 2048, 512
VOCAB_IDS = 50280


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), float(j.get("bf16_tflops_sustained", 0)), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def decode_bytes_per_token(hp) -> dict:
    """Algorithmic HBM bytes of one batch-1 decode token (each byte read/written once)."""
    dm, di, H, P, N = hp["d_model"], hp["expand"] * hp["d_model"], hp["n_heads"], hp["d_head"], hp["d_state"]
    G = hp["n_groups"]
    xd = di + 2 * G * N
    proj = di + xd + H
    int4 = lambda n, k: n * k // 2 + (n * k // 32) * 2  # noqa: E731
    per_layer = {
        "in_proj_int4": int4(proj, dm),
        "out_proj_int4": int4(dm, di),
        "ssd_state_rw": 2 * H * P * N * 4,
        "conv_state_rw": 2 * xd * hp["d_conv"] * 2,
        "small": (xd * hp["d_conv"] + xd + 3 * H + dm + di) * 2,
    }
    layers = hp["n_layer"] * sum(per_layer.values())
    lm = hp["vocab_size"] * dm * 2 + dm * 2
    return dict(per_layer=per_layer, total=layers + lm, lm_head=lm)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines = []          # (monotonic time, line)
        self.t_begin = self.t_end = None

    def start(self):
        """Starts nvidia-smi ahead of the timed region (its start-up is not timed work)
        and waits up to 3 s for the first sample; call mark_begin() when timing starts."""
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.monotonic()
            while not self.lines and time.monotonic() - t0 < 3.0:
                time.sleep(0.02)
        except OSError:
            self.proc = None

    def mark_begin(self):
        self.t_begin = time.monotonic()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def stop(self):
        self.t_end = time.monotonic()
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        t_begin = self.t_begin if self.t_begin is not None else 0.0
        inside = [ln for t, ln in self.lines if t_begin <= t <= self.t_end]
        if not inside and self.lines:   # timed region shorter than one sampling period
            inside = [min(self.lines, key=lambda tl: abs(tl[0] - t_begin))[1]]
        for ln in inside:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local, dist


def barrier(dist, local):
    if dist is not None:
        import torch
        dist.barrier(device_ids=[local])
        torch.cuda.synchronize()


def allreduce_max(dist, vals, local):
    if dist is None:
        return vals
    import torch
    t = torch.tensor(vals, dtype=torch.float64, device=f"cuda:{local}")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def graph_timed(ctx, stream, call, n, replays=4):
    """Average device time of one `call` (a C-ABI op launch): the n calls are captured
    once into a CUDA graph through the library's graph batching and the graph is
    replayed, so the CUDA events measure kernels back to back, not host submission."""
    import torch
    call(0)                            # eager first call: loads kernels, sizes scratch outside capture
    torch.cuda.synchronize()
    ctx.set_graph_batching(True)
    try:
        ctx.begin_batch()
        for i in range(n):
            call(i)
        ctx.commit_and_wait()          # instantiate + one warm run
        ctx.replay_batch(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        ctx.replay_batch(replays)
        e1.record(stream)
        e1.synchronize()
    finally:
        ctx.set_graph_batching(False)
    return e0.elapsed_time(e1) / (n * replays)


def time_kernel_int4_gemv(lssm, ctx, model, hp, reps=128):
    """Average device time of the dominant decode kernel (the in_proj INT4 GEMV,
    N = 10576, K = 2560) on layer 0's weights, CUDA events on the launching stream."""
    import ctypes as C

    import torch
    dm = hp["d_model"]
    # every launch reads a different layer's in_proj (64 x 15 MB >> L2), as in a decode token
    offs = [model.tensor(f"backbone.layers.{i}.mixer.in_proj.weight")[0] for i in range(hp["n_layer"])]
    _, nb, _ = model.tensor("backbone.layers.0.mixer.in_proj.weight")
    N = (2 * hp["expand"] * dm + 2 * hp["n_groups"] * hp["d_state"] + hp["n_heads"])
    calls = [0]
    base = lssm.lib().lssm_model_device_base(model.h)
    x = lssm.DeviceBuffer(ctx, dm * 2)
    x.upload(np.random.default_rng(0).standard_normal(dm).astype(np.float16))
    y = lssm.DeviceBuffer(ctx, N * 2)
    stream = torch.cuda.ExternalStream(ctx.stream())
    dims = lssm.LinearDims(1, N, dm)
    L = lssm.lib()

    class _B:
        pass

    def call():
        off = offs[calls[0] % len(offs)]
        calls[0] += 1
        lssm.check(L.lssm_linear_int4_gemv(ctx.h, x.ptr, 0, base, off, base, off + N * dm // 2, y.ptr, 0, dims))

    ms = graph_timed(ctx, stream, lambda i: call(), reps)
    bytes_alg = nb + dm * 2 + N * 2
    _ = C
    return ms, bytes_alg


_ORACLE_CACHE = {}


def cpu_baseline_sample(seed=0, prompt=32, new=8, hp=None):
    """The oracle (C++ restatement of the reference's kernels) on the host cores:
    a bounded sample of the same workload (same model bytes, shorter request)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import pyoracle as po
    # every host core this process may run on (torchrun exports OMP_NUM_THREADS=1)
    try:
        cores = len(os.sched_getaffinity(0))
    except AttributeError:
        cores = os.cpu_count() or 1
    po.lib().lssm_oracle_set_num_threads(cores)
    hp = hp or HP27
    key = (seed, tuple(sorted(hp.items())))
    if key not in _ORACLE_CACHE:   # the model is synthesised once per process, not timed
        t0 = time.time()
        img = po.synthesize(hp, seed, True)
        _ORACLE_CACHE[key] = (po.OracleModel(img, mode=0), time.time() - t0)
        del img
    m, t_synth = _ORACLE_CACHE[key]
    rng = np.random.default_rng(seed + 1)
    toks = rng.integers(0, VOCAB_IDS, size=prompt).astype(np.uint32)
    # prefill alone
    t0 = time.time()
    m.generate(toks, 1, want_logits=False)
    t_pre = time.time() - t0
    # the full sample keeps its ids and logits (copying them out is not measurable next to
    # the model math): the GPU engine is checked against them on the same prompt
    t0 = time.time()
    ids, pre_logits, step_logits = m.generate(toks, new + 1, want_logits=True)
    t_all = time.time() - t0
    t_dec = max(t_all - t_pre, 1e-9)
    return dict(prefill_tok_s=prompt / t_pre, decode_tok_s=new / t_dec, cores=po.lib().lssm_oracle_num_threads(),
                sample=f"prompt {prompt} + {new} greedy tokens, full 64-layer 2.7B INT4 model (synth {t_synth:.1f}s)",
                seconds=t_pre + t_all, prompt=toks, ids=ids, pre_logits=pre_logits, last_logits=step_logits[-1],
                oracle=m)


def oracle_fp32_rows(cb):
    """The same sample through the oracle's fp32 mode (not timed): prefill and last-step
    logits, conditioned on the fp16-faithful run's ids."""
    m = cb["oracle"]
    m.desc.mode = 1
    try:
        _, pre, steps = m.generate(cb["prompt"], len(cb["ids"]), teacher=cb["ids"])
    finally:
        m.desc.mode = 0
    return pre, steps[-1]


def parity_vs_oracle(sess, cb):
    """The GPU engine on the CPU sample's prompt (same 64-layer model bytes): greedy ids must
    equal the fp16-faithful oracle's free-running ids, and the prefill / last-step logits must
    be within twice the oracle's own fp16-faithful vs fp32 spread on the same rows (floor 0.1):
    the engine and the faithful oracle share every fp16 rounding point and differ only in fp32
    summation order."""
    n = len(cb["ids"])
    sess.reset()
    first = sess.prefill(cb["prompt"][None])
    pre = sess.logits()[0]
    rest = sess.decode(first, n - 1)[0]
    last = sess.logits()[0]
    ids = np.concatenate([first, rest])
    diff = np.nonzero(ids != cb["ids"])[0]
    d = int(diff[0]) if len(diff) else n
    pre32, last32 = oracle_fp32_rows(cb)
    noise = max(float(np.abs(cb["pre_logits"] - pre32).max()), float(np.abs(cb["last_logits"] - last32).max()))
    tol = max(0.1, 2.0 * noise)
    e_pre = float(np.abs(pre - cb["pre_logits"]).max())
    e_last = float(np.abs(last - cb["last_logits"]).max()) if d == n else None
    ok = d == n and e_pre <= tol and e_last <= tol
    return {"ok": bool(ok), "ids_equal": d == n, "tokens": n, "first_divergence": d, "prompt": len(cb["prompt"]),
            "max_abs_logits_prefill": e_pre, "max_abs_logits_last": e_last, "tolerance": tol,
            "oracle_fp16_vs_fp32_spread": noise, "max_abs_logit": float(np.abs(pre32).max()),
            "max_abs_logits_vs_fp32": float(max(np.abs(pre - pre32).max(), np.abs(last - last32).max())),
            "oracle": "fp16-faithful C++ oracle, free-running, same synthesized 64-layer 2.7B INT4 model",
            "decode_path": "persistent" if n_dec_launches(sess) == 1 else "per-op graph"}


def run_reference(args, world, rank):
    if rank != 0:
        return 0
    res = []
    for i in range(args.warmup + args.steps):
        r = cpu_baseline_sample(prompt=args.ref_prompt, new=args.ref_new)
        if i >= args.warmup:
            res.append(r)
    dec = float(np.median([r["decode_tok_s"] for r in res]))
    pre = float(np.median([r["prefill_tok_s"] for r in res]))
    secs = float(np.mean([r["seconds"] for r in res]))
    line = {
        "impl": "reference", "metric": METRIC, "value": dec, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": secs * 1000.0, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16 activations, int4_b32 weights, f32 accum",
        "data": "synthetic (seeded random-init weights and prompt ids)",
        "config": {"workload": "2.7B-int4 batch-1 decode (CPU bounded sample)", "model": "mamba2-2.7b-shape",
                   "global_batch": 1, "seq_len": args.ref_prompt, "parallelism": "host threads"},
        "prefill_tok_s": pre,
        "cpu_baseline": {"value": dec, "unit": "tok/s", "cores": res[0]["cores"], "kind": "port",
                         "sample": res[0]["sample"]},
        "e2e": {"value": dec, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def n_dec_launches(sess):
    return sess.launches()[1]


def run_ours(args, world, rank, local, dist):
    import lssm
    import torch
    hbm, tflops, tflops_sus, peak_kind = measured_peaks()
    ctx = lssm.Ctx(local)
    hp = lssm.hparams(**HP27)
    model = lssm.Model.synthesize(ctx, hp, seed=0, int4=True)
    sess = lssm.Session(ctx, model, batch=1, max_seq_len=PROMPT)
    rng = np.random.default_rng(1000 + rank)
    prompt = rng.integers(0, VOCAB_IDS, size=(1, PROMPT)).astype(np.uint32)

    def step():
        sess.reset()
        first = sess.prefill(prompt)
        p_ms, _ = sess.timing()
        sess.decode(first, NEW - 1)   # NEW tokens total: 1 from prefill + NEW-1 decode steps
        _, d_ms = sess.timing()
        return p_ms, d_ms

    clocks = ClockSampler(local)
    clocks.start()
    for _ in range(args.warmup):
        step()
    barrier(dist, local)
    torch.cuda.synchronize()
    clocks.mark_begin()
    pre_ms, dec_ms = [], []
    w0 = time.time()
    for _ in range(args.steps):
        p, d = step()
        pre_ms.append(p)
        dec_ms.append(d)
    torch.cuda.synchronize()
    wall = time.time() - w0
    barrier(dist, local)
    clk = clocks.stop()
    tot_pre, tot_dec = allreduce_max(dist, [sum(pre_ms), sum(dec_ms)], local)
    dec_tokens = (NEW - 1) * args.steps * world
    pre_tokens = PROMPT * args.steps * world
    decode_tok_s = dec_tokens / (tot_dec / 1000.0)
    prefill_tok_s = pre_tokens / (tot_pre / 1000.0)

    # e2e through the C ABI with host buffers (prompt H2D + generated ids D2H in the timed region)
    pinned = torch.from_numpy(prompt).pin_memory()
    ptoks = pinned.numpy()
    barrier(dist, local)
    e_t = []
    for _ in range(max(1, min(args.steps, 3))):
        t0 = time.perf_counter()
        out = sess.generate(ptoks, NEW)
        e_t.append(time.perf_counter() - t0)
    (e_max,) = allreduce_max(dist, [float(np.sum(e_t))], local)
    e2e = NEW * len(e_t) * world / e_max   # generated tokens per request-second (prefill + decode + copies)
    assert out.shape == (1, NEW)

    # Dominant kernel: the persistent decode kernel (one launch = NEW - 1 tokens), timed
    # by the session's CUDA events on the launching stream; algorithmic bytes per token
    # = weights + ssd/conv state read and written once (decode_bytes_per_token).
    bpt = decode_bytes_per_token(HP27)
    persistent = n_dec_launches(sess) == 1
    k_ms = tot_dec / args.steps                      # one decode launch per step
    k_bytes = bpt["total"] * (NEW - 1)
    achieved = k_bytes / (k_ms / 1000.0) / 1e9
    step_gbs = bpt["total"] * (decode_tok_s / world) / 1e9
    prof = ROOT / "profiles" / "decode_persist_traffic.json"
    traffic = None
    if prof.exists():
        tpt = json.loads(prof.read_text()).get("dram_bytes_per_token")
        traffic = tpt * (NEW - 1) if tpt else None
    # secondary: the standalone INT4 GEMV kernel of the per-op path (graph-timed, cold L2)
    g_ms, g_bytes = time_kernel_int4_gemv(lssm, ctx, model, HP27)
    n_pre, n_dec = sess.launches()
    launches = args.steps * (n_pre + n_dec)   # n_dec: launches of the whole decode call
    prefill_flops = 2 * PROMPT * (HP27["n_layer"] * ((2 * 5120 + 256 + 80) * 2560 + 2560 * 5120))

    # the workloads that shard across GPUs, measured at every N on the same ranks (collective):
    # batched decode (sequences split over the GPUs) and the 8B shape (heads tensor-parallel)
    sharded = None
    if not args.no_sharded:
        bl = run_batched(args, world, rank, local, dist, ctx=ctx, model=model, steps=2, warmup=1, emit=False)
        tl = run_tp8b(args, world, rank, local, dist, ctx=ctx, steps=2, warmup=1, emit=False)
        if rank == 0:
            def brief(r):
                return {"value": r["value"], "unit": r["unit"], "scaling": r["scaling"],
                        "prefill_tok_s": r["prefill_tok_s"], "decode_ms_per_step": r["decode_ms_per_step"],
                        "roofline_frac": r["roofline"]["frac"], "bytes_per_step_per_gpu": r["roofline"][
                            "bytes_per_step_per_gpu"], "e2e": r["e2e"], "steps": r["steps"], "warmup": r["warmup"],
                        "workload": r["config"]["workload"], "parallelism": r["config"]["parallelism"],
                        "clocks": r["clocks"]}
            sharded = {"batched": brief(bl), "tp8b": brief(tl)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": decode_tok_s, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": (tot_pre + tot_dec) / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16 activations, int4_b32 weights, f32 accum",
            "data": "synthetic (seeded random-init weights in the reference .ssm INT4_B32 layout, random prompt ids)",
            "config": {"workload": "2.7B-int4 batch-1 per GPU: prefill 2048 + 512 greedy decode tokens",
                       "model": "mamba2-2.7b-shape (64L, d_model 2560, 80x64 heads, d_state 128, vocab 50288)",
                       "global_batch": world, "seq_len": PROMPT, "parallelism": f"independent sequences x{world}",
                       "l2": "no flush: each decode token streams 2.05 GB of weights + state (> 126 MB L2)"},
            "prefill_tok_s": prefill_tok_s,
            "decode_ms_per_token": tot_dec / ((NEW - 1) * args.steps),
            "prefill_ms": tot_pre / args.steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "traffic": traffic,
                         "kernel": ("k_decode_persist (all layers + lm_head + argmax, NEW-1 tokens per launch)"
                                    if persistent else "decode step (per-op CUDA graph)"),
                         "kernel_ms": k_ms, "bytes_per_launch": k_bytes,
                         "bytes_per_token": bpt["total"], "peak_kind": f"{peak_kind} hbm_gbs (burst copy)"},
            "gemv_microbench": {"kernel": "int4 GEMV in_proj (N=10576, K=2560), per-op path", "ms": g_ms,
                                "gbs": g_bytes / (g_ms / 1000.0) / 1e9, "frac": g_bytes / (g_ms / 1000.0) / 1e9 / hbm},
            "decode_step_roofline": {"bytes_per_token": bpt["total"], "achieved_gbs": step_gbs, "peak": hbm,
                                     "frac": step_gbs / hbm},
            # prefill is a ~30 ms stretch of back-to-back GEMMs: the sustained (power-capped) peak
            "prefill_tensor_roofline": {"flops": prefill_flops,
                                        "achieved_tflops": prefill_flops / (tot_pre / args.steps / 1000) / 1e12,
                                        "peak": tflops_sus or tflops,
                                        "peak_kind": f"{peak_kind} bf16_tflops_sustained" if tflops_sus else
                                        f"{peak_kind} bf16_tflops",
                                        "frac": prefill_flops / (tot_pre / args.steps / 1000) / 1e12 / (tflops_sus or tflops)},
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": PROMPT * 4, "d2h_bytes_per_step": NEW * 4},
            "gpu_launches": launches, "clocks": clk, "wall_s": wall,
        }
        if sharded is not None:
            line["sharded_workloads"] = sharded
        if world == 1 and not args.no_cpu_baseline:
            cb = cpu_baseline_sample(prompt=args.ref_prompt, new=args.ref_new)
            line["cpu_baseline"] = {"value": cb["decode_tok_s"], "unit": "tok/s", "cores": cb["cores"], "kind": "port",
                                    "sample": cb["sample"], "prefill_tok_s": cb["prefill_tok_s"]}
            line["parity"] = parity_vs_oracle(sess, cb)
        print(json.dumps(line), flush=True)
    sess.close()
    model.close()
    ctx.close()
    return 0


def run_kernel_bench(args):
    """Single-kernel microbenchmarks at the benchmark shapes (used for the roofline
    numbers and as small, bounded cases for ncu). Weights / states are cycled over
    64 distinct layer slices so every launch reads from HBM (> 126 MB L2), like a
    real decode token does."""
    import ctypes as C

    import lssm
    import torch
    hbm, tflops, _, peak_kind = measured_peaks()
    ctx = lssm.Ctx(0)
    L = lssm.lib()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.ExternalStream(ctx.stream())
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    reps = args.reps
    out = {"kernel": args.kernel}

    def timed(call, n):
        return graph_timed(ctx, stream, call, n)

    if args.kernel in ("int4_gemv", "int4_gemv_out"):
        if args.kernel == "int4_gemv":
            N, K = 10576, 2560
        else:
            N, K = 2560, 5120
        N, K = args.gemv_n or N, args.gemv_k or K
        R = args.rows
        per = N * K // 2 + N * K // 16
        nl = 64
        W = torch.randint(0, 256, (nl * per,), dtype=torch.uint8, device=dev, generator=g)
        sc = (torch.rand((nl, N * K // 32), device=dev, generator=g) * 0.01 + 1e-3).half()
        Wv = W.view(nl, per)
        Wv[:, N * K // 2:] = sc.view(torch.uint8).view(nl, -1)
        x = torch.randn(R, K, device=dev, generator=g).half()
        y = torch.empty(R, N, device=dev, dtype=torch.half)
        torch.cuda.synchronize()
        dims = lssm.LinearDims(R, N, K)
        base = W.data_ptr()
        fn = L.lssm_linear_int4_gemv if R == 1 else L.lssm_linear_int4_gemv_rows

        def call(i):
            o = (i % nl) * per
            lssm.check(fn(ctx.h, x.data_ptr(), 0, base, o, base, o + N * K // 2, y.data_ptr(), 0, dims))
        call(0)   # loads the kernel outside the graph capture
        torch.cuda.synchronize()
        ms = timed(call, reps)
        b = per + R * K * 2 + R * N * 2
        out.update(shape=[R, N, K], us=ms * 1e3, bytes=b, gbs=b / ms / 1e6, frac=b / ms / 1e6 / hbm)
    elif args.kernel == "f16_gemv":
        N, K, R = args.gemv_n or 50288, args.gemv_k or 2560, args.rows
        per = N * K * 2
        nl = max(2, min(64, int(4e9 // per)))
        W = (torch.randn(nl * N * K, device=dev, generator=g) * 0.05).half()
        x = torch.randn(R, K, device=dev, generator=g).half()
        y = torch.empty(R, N, device=dev, dtype=torch.half)
        torch.cuda.synchronize()
        dims = lssm.LinearDims(R, N, K)
        base = W.data_ptr()
        fn = L.lssm_linear_f16_gemv if R == 1 else L.lssm_linear_f16_gemv_rows

        def call(i):
            lssm.check(fn(ctx.h, x.data_ptr(), 0, base, (i % nl) * per, y.data_ptr(), 0, dims))
        call(0)
        torch.cuda.synchronize()
        ms = timed(call, reps)
        b = per + R * K * 2 + R * N * 2
        out.update(shape=[R, N, K], us=ms * 1e3, bytes=b, gbs=b / ms / 1e6, frac=b / ms / 1e6 / hbm)
    elif args.kernel in ("gemm_f16", "int4_gemm"):
        M, N, K = args.m, args.n, args.k
        X = torch.randn(M, K, device=dev, generator=g).half()
        Y = torch.empty(M, N, device=dev, dtype=torch.half)
        # call i reads weight copy i % nl; the copies one timed graph touches (min(nl, reps)) exceed
        # the 126 MB L2 when reps >= nl, so the weights stream from HBM as in a model's layers
        if args.kernel == "gemm_f16":
            per = N * K * 2
            nl = max(1, min(64, -(-(512 << 20) // per)))
            Wt = (torch.randn(nl, N, K, device=dev, generator=g) / K ** 0.5).half()
            torch.cuda.synchronize()

            def call(i):
                lssm.check(L.lssm_linear_f16_gemm(ctx.h, X.data_ptr(), 0, Wt.data_ptr(), (i % nl) * per,
                                                  Y.data_ptr(), 0, lssm.LinearDims(M, N, K)))
        else:
            per = N * K // 2 + N * K // 16   # packed nibbles, then fp16 scales
            stride = (per + 255) // 256 * 256
            nl = max(1, min(64, -(-(512 << 20) // per)))
            Wq = torch.randint(0, 256, (nl * stride,), dtype=torch.uint8, device=dev, generator=g)
            Wv = Wq.view(nl, stride)
            Wv[:, N * K // 2:per] = ((torch.rand((nl, N * K // 32), device=dev, generator=g) * 0.01).half()
                                     .view(torch.uint8))
            torch.cuda.synchronize()

            def call(i):
                off = (i % nl) * stride
                lssm.check(L.lssm_linear_int4_gemm(ctx.h, X.data_ptr(), 0, Wq.data_ptr(), off, Wq.data_ptr(),
                                                   off + N * K // 2, Y.data_ptr(), 0, lssm.LinearDims(M, N, K)))
        ms = timed(call, reps)
        fl = 2.0 * M * N * K
        out.update(shape=[M, N, K], us=ms * 1e3, tflops=fl / ms / 1e9, frac=fl / ms / 1e9 / tflops,
                   weight_copies=min(nl, reps), weight_bytes=per)
    elif args.kernel == "ssd_chunked":
        Bt, Ls, H, P, N, G = args.ssd_batch, args.ssd_len, 80, 64, 128, 1
        X = torch.randn(Bt, Ls, H, P, device=dev, generator=g).bfloat16()
        Bm = torch.randn(Bt, Ls, G, N, device=dev, generator=g).bfloat16()
        Cm = torch.randn(Bt, Ls, G, N, device=dev, generator=g).bfloat16()
        dt = torch.randn(Bt, Ls, H, device=dev, generator=g) - 2.0
        db = torch.zeros(H, device=dev)
        alog = torch.empty(H, device=dev).uniform_(0.0, float(np.log(16.0)), generator=g)
        Dd = torch.randn(H, device=dev, generator=g)
        Y = torch.empty(Bt, Ls, H, P, device=dev)
        S = torch.zeros(Bt, H, P, N, device=dev)
        torch.cuda.synchronize()
        dims = lssm.SSDBatchedDims(Bt, Ls, H, P, N, G, 256, 1e-6, 1e6, 1, lssm.DT_BF16, lssm.DT_F32, lssm.DT_F32,
                                   lssm.DT_F32)

        def call(i):
            lssm.check(L.lssm_ssd_chunked_batched(ctx.h, X.data_ptr(), Bm.data_ptr(), Cm.data_ptr(), dt.data_ptr(),
                                                  db.data_ptr(), alog.data_ptr(), Dd.data_ptr(), Y.data_ptr(),
                                                  S.data_ptr(), dims))
        ms = timed(call, reps)
        b = X.numel() * 2 + Bm.numel() * 2 * 2 + dt.numel() * 4 + Y.numel() * 4 + 2 * S.numel() * 4
        out.update(shape=[Bt, Ls, H, P, N], us=ms * 1e3, bytes=b, gbs=b / ms / 1e6, frac=b / ms / 1e6 / hbm)
    elif args.kernel == "ssd_step":
        H, P, N = 80, 64, 128
        Bt = args.step_batch
        per = Bt * H * P * N                   # state floats per slice
        nl = max(2, min(64, int(2e9 // (per * 4))))
        S = torch.zeros(nl * per, device=dev)
        x = torch.randn(Bt * H * P, device=dev, generator=g).half()
        Bm = torch.randn(Bt * N, device=dev, generator=g).half()
        Cm = torch.randn(Bt * N, device=dev, generator=g).half()
        dt = torch.randn(Bt * H, device=dev, generator=g).half()
        par = torch.zeros(H, device=dev).half()
        y = torch.empty(Bt * H * P, device=dev, dtype=torch.half)
        torch.cuda.synchronize()
        if Bt == 1:
            dims = lssm.SSDStepDims(H, P, N, 1, 1e-6, 1e6, 1)

            def call(i):
                so = (i % nl) * per * 4
                lssm.check(L.lssm_ssd_step_f16(ctx.h, x.data_ptr(), 0, Bm.data_ptr(), 0, Cm.data_ptr(), 0, dt.data_ptr(),
                                               0, par.data_ptr(), 0, par.data_ptr(), 0, par.data_ptr(), 0, S.data_ptr(),
                                               so, y.data_ptr(), 0, dims))
        else:
            bdims = lssm.SSDBatchedDims(Bt, 1, H, P, N, 1, 256, 1e-6, 1e6, 1, 0, 0, 0, 0)

            def call(i):
                lssm.check(L.lssm_ssd_step_batched(ctx.h, x.data_ptr(), Bm.data_ptr(), Cm.data_ptr(), dt.data_ptr(),
                                                   par.data_ptr(), par.data_ptr(), par.data_ptr(),
                                                   S.data_ptr() + (i % nl) * per * 4, y.data_ptr(), bdims))
        call(0)
        torch.cuda.synchronize()
        ms = timed(call, reps)
        b = 2 * per * 4 + Bt * H * P * 4
        out.update(shape=[Bt, H, P, N], us=ms * 1e3, bytes=b, gbs=b / ms / 1e6, frac=b / ms / 1e6 / hbm)
    out["peak"] = f"{peak_kind} (hbm {hbm} GB/s, bf16 {tflops} TF/s)"
    print(json.dumps(out), flush=True)
    _ = C
    ctx.close()
    return 0


def run_batched(args, world, rank, local, dist, ctx=None, model=None, steps=None, warmup=None, emit=True):
    """Batched decode (the batched benchmark config): `--seqs` independent sequences (default
    64), each a 512-token prompt + 256 greedy decode steps, sharded over the ranks (seqs /
    world per GPU, weights replicated, no data-path collective): strong scaling. With `model`
    given (the default run embeds this workload) it reuses that 2.7B model; returns the
    record (rank 0) and prints it when `emit`."""
    import lssm
    import torch
    hbm, _, _, peak_kind = measured_peaks()
    total = args.seqs
    if total % world:
        raise SystemExit(f"--seqs {total} is not divisible by {world} ranks")
    per = total // world
    plen, steps_new = args.batched_prompt, args.batched_new
    n_steps = args.steps if steps is None else steps
    n_warm = args.warmup if warmup is None else warmup
    own = model is None
    if ctx is None:
        ctx = lssm.Ctx(local)
    if own:
        model = lssm.Model.synthesize(ctx, lssm.hparams(**HP27), seed=0, int4=True)
    sess = lssm.Session(ctx, model, batch=per, max_seq_len=plen)
    rng = np.random.default_rng(2000 + rank)
    prompts = rng.integers(0, VOCAB_IDS, size=(per, plen)).astype(np.uint32)

    def step():
        sess.reset()
        first = sess.prefill(prompts)
        p_ms, _ = sess.timing()
        sess.decode(first, steps_new)
        _, d_ms = sess.timing()
        return p_ms, d_ms

    clocks = ClockSampler(local)
    clocks.start()
    for _ in range(n_warm):
        step()
    barrier(dist, local)
    torch.cuda.synchronize()
    clocks.mark_begin()
    pre, dec = [], []
    w0 = time.time()
    for _ in range(n_steps):
        p_ms, d_ms = step()
        pre.append(p_ms)
        dec.append(d_ms)
    torch.cuda.synchronize()
    wall = time.time() - w0
    barrier(dist, local)
    clk = clocks.stop()
    tot_pre, tot_dec = allreduce_max(dist, [sum(pre), sum(dec)], local)
    decode_tok_s = total * steps_new * n_steps / (tot_dec / 1000.0)
    prefill_tok_s = total * plen * n_steps / (tot_pre / 1000.0)
    # e2e: the same requests through lssm_generate, prompts from pinned host memory
    pinned = torch.from_numpy(prompts).pin_memory().numpy()
    barrier(dist, local)
    t0 = time.perf_counter()
    out = sess.generate(pinned, steps_new + 1)
    e_s = time.perf_counter() - t0
    (e_max,) = allreduce_max(dist, [e_s], local)
    assert out.shape == (per, steps_new + 1)
    bpt = decode_bytes_per_token(HP27)
    state_b = HP27["n_layer"] * (bpt["per_layer"]["ssd_state_rw"] + bpt["per_layer"]["conv_state_rw"])
    step_bytes = (bpt["total"] - HP27["n_layer"] * (bpt["per_layer"]["ssd_state_rw"] + bpt["per_layer"]["conv_state_rw"])
                  + per * state_b)   # weights once per step per GPU + every sequence's state R+W
    ms_step = tot_dec / n_steps / steps_new
    n_pre, n_dec = sess.launches()
    if rank == 0:
        line = {
            "metric": METRIC, "value": decode_tok_s, "unit": "tok/s", "n_gpus": world, "steps": n_steps,
            "warmup": n_warm, "ms_per_step": (tot_pre + tot_dec) / n_steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16 activations, int4_b32 weights, f32 accum",
            "data": "synthetic (seeded random-init weights in the reference .ssm INT4_B32 layout, random prompt ids)",
            "config": {"workload": f"batched decode: {total} sequences x ({plen} prompt + {steps_new} greedy steps)",
                       "model": "mamba2-2.7b-shape (64L, d_model 2560, 80x64 heads, d_state 128, vocab 50288)",
                       "global_batch": total, "seq_len": plen, "parallelism": f"sequences sharded {per} per GPU x{world}",
                       "l2": f"no flush: each step streams {step_bytes / 1e9:.2f} GB per GPU (> 126 MB L2)"},
            "prefill_tok_s": prefill_tok_s,
            "decode_ms_per_step": ms_step,
            "roofline": {"bound": "hbm", "achieved": step_bytes / (ms_step / 1000.0) / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": step_bytes / (ms_step / 1000.0) / 1e9 / hbm, "traffic": None,
                         "kernel": "decode step (per-op CUDA graph)", "bytes_per_step_per_gpu": step_bytes,
                         "peak_kind": f"{peak_kind} hbm_gbs"},
            "e2e": {"value": total * (steps_new + 1) / e_max, "unit": "tok/s", "h2d_bytes_per_step": per * plen * 4,
                    "d2h_bytes_per_step": per * (steps_new + 1) * 4},
            "gpu_launches": n_steps * (n_pre + n_dec), "clocks": clk, "wall_s": wall,
        }
        if emit:
            print(json.dumps(line), flush=True)
    sess.close()
    if own:
        model.close()
    return line if rank == 0 else None


def run_tp8b(args, world, rank, local, dist, ctx=None, steps=None, warmup=None, emit=True):
    """The 8B-shape config: 4 sequences, prefill 4096 random ids + 128 greedy decode tokens,
    the heads (and groups, d_inner channels, lm_head vocab rows) tensor-parallel over the
    ranks with NCCL all-reduces after out_proj (and of the gated-norm sum of squares);
    one GPU runs the unsharded session. Strong scaling (the job is fixed)."""
    import lssm
    import torch
    hbm, _, _, peak_kind = measured_peaks()
    B, plen, steps_new = args.tp_batch, args.tp_prompt, args.tp_new
    n_steps = args.steps if steps is None else steps
    n_warm = args.warmup if warmup is None else warmup
    if ctx is None:
        ctx = lssm.Ctx(local)
    model = lssm.Model.synthesize(ctx, lssm.hparams(**HP8B), seed=0, int4=True)
    comm = None
    if world > 1:
        uid = torch.zeros(lssm.COMM_ID_BYTES, dtype=torch.uint8, device=f"cuda:{local}")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(lssm.Comm.unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        comm = lssm.Comm(ctx, rank, world, bytes(uid.cpu().numpy()))
    sess = lssm.Session(ctx, model, batch=B, max_seq_len=plen, comm=comm)
    rng = np.random.default_rng(8000)
    prompts = rng.integers(0, 255990, size=(B, plen)).astype(np.uint32)   # same on every rank

    def step():
        sess.reset()
        first = sess.prefill(prompts)
        p_ms, _ = sess.timing()
        toks = sess.decode(first, steps_new)
        _, d_ms = sess.timing()
        return p_ms, d_ms, toks

    clocks = ClockSampler(local)
    clocks.start()
    for _ in range(n_warm):
        step()
    barrier(dist, local)
    torch.cuda.synchronize()
    clocks.mark_begin()
    pre, dec = [], []
    w0 = time.time()
    for _ in range(n_steps):
        p_ms, d_ms, toks = step()
        pre.append(p_ms)
        dec.append(d_ms)
    torch.cuda.synchronize()
    wall = time.time() - w0
    barrier(dist, local)
    clk = clocks.stop()
    tot_pre, tot_dec = allreduce_max(dist, [sum(pre), sum(dec)], local)
    decode_tok_s = B * steps_new * n_steps / (tot_dec / 1000.0)
    prefill_tok_s = B * plen * n_steps / (tot_pre / 1000.0)
    pinned = torch.from_numpy(prompts).pin_memory().numpy()
    barrier(dist, local)
    t0 = time.perf_counter()
    out = sess.generate(pinned, steps_new + 1)
    e_s = time.perf_counter() - t0
    (e_max,) = allreduce_max(dist, [e_s], local)
    assert out.shape == (B, steps_new + 1)
    bpt = decode_bytes_per_token(HP8B)
    state_b = HP8B["n_layer"] * (bpt["per_layer"]["ssd_state_rw"] + bpt["per_layer"]["conv_state_rw"])
    step_bytes = (bpt["total"] - state_b + B * state_b) / world   # weights once per step + B states, per GPU
    ms_step = tot_dec / n_steps / steps_new
    n_pre, n_dec = sess.launches()
    if rank == 0:
        line = {
            "metric": METRIC, "value": decode_tok_s, "unit": "tok/s", "n_gpus": world, "steps": n_steps,
            "warmup": n_warm, "ms_per_step": (tot_pre + tot_dec) / n_steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16 activations, int4_b32 weights, f32 accum",
            "data": "synthetic (seeded random-init weights in the reference .ssm INT4_B32 layout, random prompt ids)",
            "config": {"workload": f"8B-shape: batch {B}, prefill {plen} + {steps_new} greedy decode tokens",
                       "model": "mamba2-8b-shape (56L, d_model 4096, 128x64 heads, 8 groups, d_state 128, vocab 256000)",
                       "global_batch": B, "seq_len": plen,
                       "parallelism": (f"heads tensor-parallel x{world} (decode all-reduces by peer-memory exchange "
                                       "over NVLink when every rank has its own GPU, else NCCL; prefill NCCL)")
                       if world > 1
                       else "one GPU, unsharded",
                       "l2": f"no flush: each decode step streams {step_bytes / 1e9:.2f} GB per GPU (> 126 MB L2)"},
            "prefill_tok_s": prefill_tok_s,
            "decode_ms_per_step": ms_step,
            "roofline": {"bound": "hbm", "achieved": step_bytes / (ms_step / 1000.0) / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": step_bytes / (ms_step / 1000.0) / 1e9 / hbm, "traffic": None,
                         "kernel": "decode step (per-op CUDA graph incl. NCCL)", "bytes_per_step_per_gpu": step_bytes,
                         "peak_kind": f"{peak_kind} hbm_gbs"},
            "e2e": {"value": B * (steps_new + 1) / e_max, "unit": "tok/s", "h2d_bytes_per_step": B * plen * 4,
                    "d2h_bytes_per_step": B * (steps_new + 1) * 4},
            "gpu_launches": n_steps * (n_pre + n_dec), "clocks": clk, "wall_s": wall,
        }
        if emit:
            print(json.dumps(line), flush=True)
    sess.close()
    if comm is not None:
        comm.close()
    model.close()
    return line if rank == 0 else None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="decode27b", choices=["decode27b", "batched", "tp8b"],
                    help="decode27b: the headline batch-1 request per GPU; batched: --seqs sequences sharded over "
                         "GPUs; tp8b: the 8B shape, heads tensor-parallel over GPUs")
    ap.add_argument("--tp-batch", type=int, default=4)
    ap.add_argument("--tp-prompt", type=int, default=4096)
    ap.add_argument("--tp-new", type=int, default=128)
    ap.add_argument("--seqs", type=int, default=64)
    ap.add_argument("--batched-prompt", type=int, default=512)
    ap.add_argument("--batched-new", type=int, default=256)
    ap.add_argument("--kernel", default=None,
                    choices=["int4_gemv", "int4_gemv_out", "f16_gemv", "gemm_f16", "int4_gemm", "ssd_chunked",
                             "ssd_step"],
                    help="single-kernel microbenchmark instead of the model bench")
    ap.add_argument("--reps", type=int, default=64)
    ap.add_argument("--rows", type=int, default=1, help="activation rows of the GEMV microbenchmarks (1..8)")
    ap.add_argument("--gemv-n", type=int, default=0, help="GEMV microbenchmark N (0: the 2.7B shape)")
    ap.add_argument("--gemv-k", type=int, default=0, help="GEMV microbenchmark K (0: the 2.7B shape)")
    ap.add_argument("--m", type=int, default=2048)
    ap.add_argument("--n", type=int, default=10576)
    ap.add_argument("--k", type=int, default=2560)
    ap.add_argument("--ssd-batch", type=int, default=8)
    ap.add_argument("--step-batch", type=int, default=1, help="sequences of the ssd_step microbenchmark")
    ap.add_argument("--ssd-len", type=int, default=4096)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ref-prompt", type=int, default=32)
    ap.add_argument("--ref-new", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the batched / tensor-parallel workloads the default run also measures")
    ap.add_argument("--prompt-len", type=int, default=PROMPT,
                    help="prompt tokens per request (the metric's workload is 2048; smaller only for profiling)")
    ap.add_argument("--decode-tokens", type=int, default=NEW,
                    help="generated tokens per request (the metric's workload is 512; smaller only for profiling)")
    args = ap.parse_args()
    globals()["PROMPT"], globals()["NEW"] = args.prompt_len, args.decode_tokens
    if args.kernel:
        return run_kernel_bench(args)
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        return run_reference(args, world, rank)
    world, rank, local, dist = dist_setup(args.gpus)
    try:
        if args.workload == "batched":
            run_batched(args, world, rank, local, dist)
            return 0
        if args.workload == "tp8b":
            run_tp8b(args, world, rank, local, dist)
            return 0
        return run_ours(args, world, rank, local, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
