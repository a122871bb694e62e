"""ctypes front end of the CPU oracle (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm
import this module. It loads oracle/_build/liblssm_oracle.so (built from
oracle/lssm_oracle.cpp by oracle/build_oracle.py) and offers:
  * a .ssm reader (header + tensor index), restating
    include/lite_ssm/ssm_format.hpp:22-128 and src/core/ssm_loader.cpp:48-139;
  * thin wrappers over the oracle's per-kernel restatements;
  * OracleModel: prefill + greedy decode of a whole .ssm model on the CPU.
"""

from __future__ import annotations

import ctypes as C
import os
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liblssm_oracle.so"

DTYPE_F16, DTYPE_BF16, DTYPE_F32, DTYPE_I8, DTYPE_U8, DTYPE_I32, DTYPE_INT4_B32 = range(7)
HEADER_FMT = "<4sIIIQQIIIIIIIIIIII4I"
HEADER_SIZE = 96
INDEX_PREFIX_FMT = "<IIIIQQ"


def _align(x: int, a: int) -> int:
    return (x + a - 1) & ~(a - 1)


@dataclass
class TensorInfo:
    name: str
    dtype: int
    shape: tuple
    offset: int
    nbytes: int


@dataclass
class SSMHeader:
    n_tensors: int
    index_offset: int
    data_offset: int
    d_model: int
    n_layer: int
    d_state: int
    d_conv: int
    expand: int
    vocab_size: int
    n_heads: int
    d_head: int
    chunk_size: int
    default_dtype: int
    n_groups: int
    norm_before_gate: int


def packed_nbytes(dtype: int, numel: int) -> int:
    if dtype == DTYPE_INT4_B32:
        return numel // 2 + (numel // 32) * 2
    return numel * {DTYPE_F16: 2, DTYPE_BF16: 2, DTYPE_F32: 4, DTYPE_I8: 1, DTYPE_U8: 1, DTYPE_I32: 4}[dtype]


def parse_ssm(buf: bytes):
    """Parse header + index; raises ValueError with the reference loader's checks."""
    if len(buf) < HEADER_SIZE:
        raise ValueError("file too small to contain a header")
    f = struct.unpack(HEADER_FMT, buf[:HEADER_SIZE])
    if f[0] != b"LSSM":
        raise ValueError("bad magic")
    if f[1] != 1:
        raise ValueError("unsupported version")
    if f[2] != HEADER_SIZE:
        raise ValueError("header_size mismatch")
    hdr = SSMHeader(n_tensors=f[3], index_offset=f[4], data_offset=f[5], d_model=f[6], n_layer=f[7],
                    d_state=f[8], d_conv=f[9], expand=f[10], vocab_size=f[11], n_heads=f[12],
                    d_head=f[13], chunk_size=f[14], default_dtype=f[15], n_groups=f[16] or 1,
                    norm_before_gate=f[17])
    pos = hdr.index_offset
    tensors = {}
    for _ in range(hdr.n_tensors):
        name_len, rank, dtype, _pad, off, nb = struct.unpack(INDEX_PREFIX_FMT, buf[pos:pos + 32])
        pos += 32
        shape = struct.unpack(f"<{rank}Q", buf[pos:pos + 8 * rank])
        pos += 8 * rank
        name = buf[pos:pos + name_len].decode()
        pos += name_len
        raw = 32 + 8 * rank + name_len
        pos += _align(raw, 8) - raw
        numel = int(np.prod(shape))
        if off + nb > len(buf) or packed_nbytes(dtype, numel) != nb:
            raise ValueError(f"bad payload for {name}")
        tensors[name] = TensorInfo(name, dtype, tuple(shape), off, nb)
    return hdr, tensors


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            from build_oracle import build  # type: ignore  # noqa: E402
            build()
        _lib = C.CDLL(str(LIB_PATH))
        _declare(_lib)
    return _lib


def _declare(L):
    P = C.c_void_p
    u32, f32 = C.c_uint32, C.c_float
    L.lssm_oracle_h2f.restype = C.c_float
    L.lssm_oracle_h2f.argtypes = [C.c_uint16]
    L.lssm_oracle_f2h.restype = C.c_uint16
    L.lssm_oracle_f2h.argtypes = [C.c_float]
    L.lssm_oracle_num_threads.restype = C.c_int
    L.lssm_oracle_set_num_threads.argtypes = [C.c_int]
    L.lssm_oracle_rmsnorm_f16.argtypes = [P, P, P, u32, u32, f32]
    L.lssm_oracle_int4_dequant.argtypes = [P, P, P, u32, u32]
    L.lssm_oracle_int4_quantize.argtypes = [P, u32, u32, P, P]
    L.lssm_oracle_linear_f16.argtypes = [P, P, P, u32, u32, u32]
    L.lssm_oracle_linear_int4.argtypes = [P, P, P, P, u32, u32, u32, C.c_int]
    L.lssm_oracle_silu_f16.argtypes = [P, P, u32]
    L.lssm_oracle_add_inplace_f16.argtypes = [P, P, u32]
    L.lssm_oracle_silu_gated_f16.argtypes = [P, P, P, u32]
    L.lssm_oracle_split_silu_xBC_f16.argtypes = [P, P, P, P, u32, u32, u32, u32]
    L.lssm_oracle_causal_conv1d_f16.argtypes = [P, P, P, P, u32, u32, u32, u32]
    L.lssm_oracle_causal_conv1d_update_f16.argtypes = [P, P, P, P, P, u32, u32, u32]
    L.lssm_oracle_seed_conv_state_f16.argtypes = [P, P, u32, u32, u32]
    L.lssm_oracle_inproj_fused_f16.argtypes = [P] * 10 + [u32] * 7
    L.lssm_oracle_ssd_step_f16.argtypes = [P] * 9 + [u32] * 4 + [f32, f32, u32]
    L.lssm_oracle_ssd_chunked_f16.argtypes = [P] * 9 + [u32] * 6 + [f32, f32, u32]
    L.lssm_oracle_ssd_chunked_f32.argtypes = [P] * 9 + [u32] * 7 + [f32, f32, u32, C.c_int]
    L.lssm_oracle_ssd_sequential_f64.argtypes = [P] * 9 + [u32] * 6 + [f32, f32, u32]
    L.lssm_oracle_argmax_f32.restype = u32
    L.lssm_oracle_argmax_f32.argtypes = [P, u32]
    L.lssm_oracle_generate.restype = C.c_int
    L.lssm_oracle_generate.argtypes = [P, P, P, P, u32, u32, P, P, P, P]


def ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


class LayerOffsets(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("norm_w", "in_proj_w", "conv1d_w", "conv1d_b", "dt_bias", "A_log",
                                          "D", "mixer_norm_w", "out_proj_w")] + \
               [("in_proj_int4", C.c_uint32), ("out_proj_int4", C.c_uint32)]


class ModelDesc(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("d_model", "n_layer", "d_state", "d_conv", "expand", "vocab",
                                          "n_heads", "d_head", "chunk", "n_groups")] + \
               [("embed_off", C.c_uint64), ("norm_f_off", C.c_uint64), ("lm_head_off", C.c_uint64),
                ("lm_head_int4", C.c_uint32), ("mode", C.c_uint32)]


class OracleModel:
    """Whole-model CPU oracle over a .ssm file (bytes or path). mode 0 = faithful fp16, 1 = fp32."""

    def __init__(self, ssm, mode: int = 0):
        buf = Path(ssm).read_bytes() if isinstance(ssm, (str, os.PathLike)) else bytes(ssm)
        self.buf = np.frombuffer(buf, dtype=np.uint8).copy()
        self.hdr, self.tensors = parse_ssm(buf)
        h = self.hdr
        t = self.tensors
        lm = t.get("lm_head.weight", t["backbone.embeddings.weight"])
        self.desc = ModelDesc(h.d_model, h.n_layer, h.d_state, h.d_conv, h.expand, h.vocab_size, h.n_heads,
                              h.d_head, h.chunk_size, h.n_groups, t["backbone.embeddings.weight"].offset,
                              t["backbone.norm_f.weight"].offset, lm.offset,
                              1 if lm.dtype == DTYPE_INT4_B32 else 0, mode)
        arr = (LayerOffsets * h.n_layer)()
        for i in range(h.n_layer):
            p = f"backbone.layers.{i}."
            g = lambda n: t[p + n]  # noqa: E731
            arr[i] = LayerOffsets(g("norm.weight").offset, g("mixer.in_proj.weight").offset,
                                  g("mixer.conv1d.weight").offset, g("mixer.conv1d.bias").offset,
                                  g("mixer.dt_bias").offset, g("mixer.A_log").offset, g("mixer.D").offset,
                                  g("mixer.norm.weight").offset, g("mixer.out_proj.weight").offset,
                                  int(g("mixer.in_proj.weight").dtype == DTYPE_INT4_B32),
                                  int(g("mixer.out_proj.weight").dtype == DTYPE_INT4_B32))
        self.layers = arr

    def generate(self, prompt, n_new: int, teacher=None, want_logits: bool = True):
        prompt = np.ascontiguousarray(prompt, dtype=np.uint32)
        V = self.hdr.vocab_size
        toks = np.zeros(n_new, dtype=np.uint32)
        pl = np.zeros(V, dtype=np.float32) if want_logits else None
        sl = np.zeros((max(n_new - 1, 1), V), dtype=np.float32) if want_logits else None
        tch = None if teacher is None else np.ascontiguousarray(teacher, dtype=np.uint32)
        rc = lib().lssm_oracle_generate(ptr(self.buf), C.byref(self.desc), self.layers, ptr(prompt), len(prompt),
                                        n_new, None if tch is None else ptr(tch), ptr(toks),
                                        None if pl is None else ptr(pl), None if sl is None else ptr(sl))
        if rc != 0:
            raise RuntimeError(f"oracle generate failed rc={rc}")
        return toks, pl, sl


def mamba2_tensor_list(hp: dict, int4: bool):
    """(name, dtype, shape) of a Mamba2ForCausalLM state_dict in its order — the order
    the reference exporter writes (tools/export_mamba2.py:162-195); in_proj/out_proj
    are INT4_B32 when int4 (export_mamba2.py:55-65)."""
    dm, di = hp["d_model"], hp["expand"] * hp["d_model"]
    G = hp.get("n_groups", 1) or 1
    xd = di + 2 * G * hp["d_state"]
    proj = di + xd + hp["n_heads"]
    lin = DTYPE_INT4_B32 if int4 else DTYPE_F16
    out = [("backbone.embeddings.weight", DTYPE_F16, (hp["vocab_size"], dm))]
    for i in range(hp["n_layer"]):
        p = f"backbone.layers.{i}."
        out += [(p + "norm.weight", DTYPE_F16, (dm,)), (p + "mixer.dt_bias", DTYPE_F16, (hp["n_heads"],)),
                (p + "mixer.A_log", DTYPE_F16, (hp["n_heads"],)), (p + "mixer.D", DTYPE_F16, (hp["n_heads"],)),
                (p + "mixer.conv1d.weight", DTYPE_F16, (xd, 1, hp["d_conv"])),
                (p + "mixer.conv1d.bias", DTYPE_F16, (xd,)),
                (p + "mixer.in_proj.weight", lin if dm % 32 == 0 else DTYPE_F16, (proj, dm)),
                (p + "mixer.norm.weight", DTYPE_F16, (di,)),
                (p + "mixer.out_proj.weight", lin if di % 32 == 0 else DTYPE_F16, (dm, di))]
    out += [("backbone.norm_f.weight", DTYPE_F16, (dm,)), ("lm_head.weight", DTYPE_F16, (hp["vocab_size"], dm))]
    return out


def plan_layout(hp: dict, tensors):
    """Header + index bytes and payload offsets, restating tools/ssm_format.py:197-340."""
    idx_size = sum(_align(32 + 8 * len(s) + len(n.encode()), 8) for n, _, s in tensors)
    data_off = _align(HEADER_SIZE + idx_size, 64)
    cur, placed = data_off, []
    for n, dt, s in tensors:
        nb = packed_nbytes(dt, int(np.prod(s)))
        placed.append(TensorInfo(n, dt, tuple(s), cur, nb))
        cur = _align(cur + nb, 64)
    header = struct.pack(HEADER_FMT, b"LSSM", 1, HEADER_SIZE, len(tensors), HEADER_SIZE, data_off, hp["d_model"],
                         hp["n_layer"], hp["d_state"], hp["d_conv"], hp["expand"], hp["vocab_size"], hp["n_heads"],
                         hp["d_head"], hp.get("chunk_size", 256), DTYPE_F16, hp.get("n_groups", 1) or 1,
                         hp.get("norm_before_gate", 0), 0, 0, 0, 0)
    index = b""
    for t in placed:
        body = struct.pack(INDEX_PREFIX_FMT, len(t.name.encode()), len(t.shape), t.dtype, 0, t.offset, t.nbytes)
        body += struct.pack(f"<{len(t.shape)}Q", *t.shape) + t.name.encode()
        index += body + b"\0" * (_align(len(body), 8) - len(body))
    return header + index, placed, _align(cur, 64)


def _host_vector(kind: str, seed: int, stream: int, n: int) -> np.ndarray:
    import math
    lib().lssm_oracle_synth_f32.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float]
    u = np.zeros(n, dtype=np.float32)
    lib().lssm_oracle_synth_f32(ptr(u), n, seed, stream, 1.0)
    out = np.zeros(n, dtype=np.float16)
    for i in range(n):
        uu = 0.5 * (float(u[i]) + 1.0)
        if kind == "A_log":
            v = math.log(1.0 + 15.0 * uu)
        elif kind == "dt_bias":
            dt = math.exp(math.log(1e-3) + uu * math.log(100.0))
            v = dt + math.log(-math.expm1(-dt))
        elif kind == "D":
            v = 0.5 + uu
        else:
            v = 0.9 + 0.2 * uu
        out[i] = np.float16(np.float32(v))
    return out


def synthesize(hp: dict, seed: int, int4: bool) -> bytes:
    """CPU copy of the engine's seeded random-init model (.ssm image bytes)."""
    L = lib()
    L.lssm_oracle_synth_f16.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float]
    L.lssm_oracle_synth_int4.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint64, C.c_uint64, C.c_float]
    tl = mamba2_tensor_list(hp, int4)
    head, placed, total = plan_layout(hp, tl)
    img = np.zeros(total, dtype=np.uint8)
    img[: len(head)] = np.frombuffer(head, dtype=np.uint8)
    sqrt3 = 1.7320508075688772
    for i, t in enumerate(placed):
        stream = i + 1
        view = img[t.offset: t.offset + t.nbytes]
        addr = view.ctypes.data_as(C.c_void_p)
        n = t.name
        if n.endswith("embeddings.weight") or n == "lm_head.weight":
            L.lssm_oracle_synth_f16(addr, int(np.prod(t.shape)), seed, 1 if n == "lm_head.weight" else stream,
                                    float(np.float32(0.5 * sqrt3)))
        elif n.endswith("in_proj.weight") or n.endswith("out_proj.weight"):
            amp = float(np.float32(sqrt3 / np.sqrt(float(t.shape[1]))))
            if t.dtype == DTYPE_INT4_B32:
                L.lssm_oracle_synth_int4(addr, t.shape[0], t.shape[1], seed, stream, amp)
            else:
                L.lssm_oracle_synth_f16(addr, int(np.prod(t.shape)), seed, stream, amp)
        elif n.endswith("conv1d.weight") or n.endswith("conv1d.bias"):
            L.lssm_oracle_synth_f16(addr, int(np.prod(t.shape)), seed, stream, 0.5)
        else:
            kind = "A_log" if n.endswith("A_log") else "dt_bias" if n.endswith("dt_bias") else \
                "D" if n.endswith(".D") else "norm"
            view[:] = np.frombuffer(_host_vector(kind, seed, stream, int(np.prod(t.shape))).tobytes(), np.uint8)
    return img.tobytes()


def f16(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32).astype(np.float16).view(np.uint16))


def to_f32(h: np.ndarray) -> np.ndarray:
    return np.asarray(h).view(np.float16).astype(np.float32)
