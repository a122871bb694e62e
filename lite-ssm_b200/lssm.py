"""ctypes binding of liblssm_cuda.so (include/lssm_cuda.h).

This is the Python host side of the drop-in boundary: the same operations as
lite_ssm::MetalOps (include/lite_ssm/ops.hpp:57-244), with the same argument
meaning ((buffer, byte offset) pairs plus the POD dims structs) and the same
error behaviour (a failing call raises RuntimeError carrying the library's
message, where MetalOps throws std::runtime_error). Buffers are device
allocations (DeviceBuffer) instead of MTLBuffers.

There is no CPU fallback: if the library or a CUDA device is missing, every
entry point raises.
"""

from __future__ import annotations

import atexit
import ctypes as C
import os
import weakref
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liblssm_cuda.so"

P = C.c_void_p
u32, u64, f32, sz = C.c_uint32, C.c_uint64, C.c_float, C.c_size_t


class LinearDims(C.Structure):
    _fields_ = [("M", u32), ("N", u32), ("K", u32)]


class RMSNormDims(C.Structure):
    _fields_ = [("rows", u32), ("dim", u32), ("eps", f32)]


class RMSLinearDims(C.Structure):
    _fields_ = [("N", u32), ("K", u32), ("eps", f32)]


class Conv1dDims(C.Structure):
    _fields_ = [("B", u32), ("L", u32), ("D", u32), ("K", u32)]


class SSDDims(C.Structure):
    _fields_ = [("L", u32), ("H", u32), ("P", u32), ("N", u32), ("n_groups", u32), ("chunk_size", u32),
                ("dt_min", f32), ("dt_max", f32), ("has_D", u32)]


class SSDStepDims(C.Structure):
    _fields_ = [("H", u32), ("P", u32), ("N", u32), ("n_groups", u32), ("dt_min", f32), ("dt_max", f32),
                ("has_D", u32)]


class FusedInProjDims(C.Structure):
    _fields_ = [(n, u32) for n in ("L", "d_model", "d_inner", "d_state", "n_groups", "n_heads", "d_conv",
                                   "proj_dim")]


class SSDBatchedDims(C.Structure):
    _fields_ = [("batch", u32), ("L", u32), ("H", u32), ("P", u32), ("N", u32), ("n_groups", u32),
                ("chunk_size", u32), ("dt_min", f32), ("dt_max", f32), ("has_D", u32), ("x_dtype", u32),
                ("dt_dtype", u32), ("param_dtype", u32), ("y_dtype", u32)]


class HParams(C.Structure):
    _fields_ = [(n, u32) for n in ("d_model", "n_layer", "d_state", "d_conv", "expand", "vocab_size", "n_heads",
                                   "d_head", "chunk_size", "default_dtype", "n_groups", "norm_before_gate")]


DT_F16, DT_BF16, DT_F32 = 0, 1, 2

# (name, argtypes) for every exported function; restype is lssm_status (int) unless listed.
_SIGS = {
    "lssm_ctx_create": [C.c_int, C.POINTER(P)],
    "lssm_ctx_destroy": [P],
    "lssm_ctx_set_stream": [P, P],
    "lssm_begin_batch": [P],
    "lssm_commit_and_wait": [P],
    "lssm_ctx_set_graph_batching": [P, C.c_int],
    "lssm_replay_batch": [P, u32],
    "lssm_alloc": [P, sz, C.POINTER(P)],
    "lssm_free": [P, P],
    "lssm_upload": [P, P, sz, P, sz],
    "lssm_download": [P, P, P, sz, sz],
    "lssm_memset": [P, P, sz, C.c_int, sz],
    "lssm_rmsnorm_f16": [P, P, sz, P, sz, P, sz, RMSNormDims],
    "lssm_linear_f16_gemv": [P, P, sz, P, sz, P, sz, LinearDims],
    "lssm_linear_silu_f16_gemv": [P, P, sz, P, sz, P, sz, LinearDims],
    "lssm_rmsnorm_linear_f16_gemv": [P, P, sz, P, sz, P, sz, P, sz, RMSLinearDims],
    "lssm_linear_f16_gemm": [P, P, sz, P, sz, P, sz, LinearDims],
    "lssm_linear_silu_f16_gemm": [P, P, sz, P, sz, P, sz, LinearDims],
    "lssm_linear_int4_gemv": [P, P, sz, P, sz, P, sz, P, sz, LinearDims],
    "lssm_linear_int4_gemv_rows": [P, P, sz, P, sz, P, sz, P, sz, LinearDims],
    "lssm_linear_f16_gemv_rows": [P, P, sz, P, sz, P, sz, LinearDims],
    "lssm_ssd_step_batched": [P, P, P, P, P, P, P, P, P, P, SSDBatchedDims],
    "lssm_linear_int4_gemm": [P, P, sz, P, sz, P, sz, P, sz, LinearDims],
    "lssm_silu_f16": [P, P, sz, P, sz, u32],
    "lssm_add_inplace_f16": [P, P, sz, P, sz, u32],
    "lssm_split_silu_xBC_f16": [P, P, sz, P, sz, P, sz, P, sz, u32, u32, u32, u32],
    "lssm_silu_gated_f16": [P, P, sz, P, sz, P, sz, u32],
    "lssm_causal_conv1d_f16": [P, P, sz, P, sz, P, sz, P, sz, Conv1dDims],
    "lssm_causal_conv1d_update_f16": [P, P, sz, P, sz, P, sz, P, sz, P, sz, Conv1dDims],
    "lssm_seed_conv_state_f16": [P, P, sz, P, sz, u32, u32, u32],
    "lssm_inproj_fused_f16": [P] + [P, sz] * 10 + [FusedInProjDims],
    "lssm_inproj_fused_f16_noalloc": [P] + [P, sz] * 10 + [FusedInProjDims],
    "lssm_ssd_chunked_f16": [P] + [P, sz] * 9 + [SSDDims],
    "lssm_ssd_step_f16": [P] + [P, sz] * 9 + [SSDStepDims],
    "lssm_ssd_chunked_batched": [P] * 10 + [SSDBatchedDims],
    "lssm_model_load": [P, C.c_char_p, C.POINTER(P)],
    "lssm_model_load_bytes": [P, P, sz, C.POINTER(P)],
    "lssm_model_synthesize": [P, C.POINTER(HParams), u64, C.c_int, C.POINTER(P)],
    "lssm_model_save": [P, C.c_char_p],
    "lssm_model_config": [P, C.POINTER(HParams)],
    "lssm_model_tensor": [P, C.c_char_p, C.POINTER(u64), C.POINTER(u64), C.POINTER(u32)],
    "lssm_model_destroy": [P],
    "lssm_session_create": [P, P, u32, u32, C.POINTER(P)],
    "lssm_session_create_tp": [P, P, P, u32, u32, C.POINTER(P)],
    "lssm_comm_unique_id": [P],
    "lssm_comm_init": [P, C.c_int, C.c_int, P, C.POINTER(P)],
    "lssm_comm_destroy": [P],
    "lssm_p2p_wait_selftest": [P, u64],
    "lssm_comm_allreduce_f32": [P, P, sz],
    "lssm_session_destroy": [P],
    "lssm_session_reset": [P],
    "lssm_prefill": [P, P, u32, P],
    "lssm_decode": [P, P, u32, P],
    "lssm_generate": [P, P, u32, u32, u32, P, C.POINTER(u32)],
    "lssm_session_logits": [P, P],
    "lssm_session_timing": [P, C.POINTER(f32), C.POINTER(f32)],
    "lssm_session_set_option": [P, C.c_char_p, C.c_int64],
    "lssm_session_launches": [P, C.POINTER(u64), C.POINTER(u64)],
    "lssm_session_trace": [P, C.POINTER(u64), u64, C.POINTER(u64)],
}
_OTHER = {
    "lssm_last_error": (C.c_char_p, []),
    "lssm_version": (C.c_char_p, []),
    "lssm_backend_loaded": (C.c_int, []),
    "lssm_has_kernel": (C.c_int, [C.c_char_p]),
    "lssm_comm_rank": (C.c_int, [P]),
    "lssm_comm_world": (C.c_int, [P]),
    "lssm_batch_active": (C.c_int, [P]),
    "lssm_ctx_stream": (P, [P]),
    "lssm_model_nbytes": (sz, [P]),
    "lssm_model_device_base": (P, [P]),
    "lssm_plan_layout": (sz, [C.POINTER(HParams), C.c_int, P, sz, C.POINTER(u64), C.POINTER(u64)]),
    "lssm_parse_header": (C.c_int, [P, sz, C.POINTER(HParams), C.POINTER(u32), C.c_char_p, sz]),
    "lssm_plan_int4_gemm": (C.c_int, [u32, u32, u32, C.c_int, sz, C.POINTER(u32), C.POINTER(u32)]),
    "lssm_int4_gemm_unit": (None, [u32, u32, u32, u32, u32, C.POINTER(u32)]),
    "lssm_persist_in_deal": (None, [u32, u32, u32, u32, C.POINTER(u32)]),
    "lssm_plan_gemm_f16": (C.c_int, [u32, u32, C.c_int]),
}

_lib = None


def lib():
    """Load liblssm_cuda.so (building it first if it is missing)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            import importlib.util
            spec = importlib.util.spec_from_file_location("lssm_build", HERE / "build.py")
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)  # type: ignore
            mod.build()
        L = C.CDLL(str(LIB_PATH))
        for n, a in _SIGS.items():
            fn = getattr(L, n)
            fn.argtypes = a
            fn.restype = C.c_int
        for n, (r, a) in _OTHER.items():
            fn = getattr(L, n)
            fn.argtypes = a
            fn.restype = r
        _lib = L
    return _lib


class LssmError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(msg)
        self.status = status


def check(st: int):
    if st != 0:
        raise LssmError(st, lib().lssm_last_error().decode(errors="replace"))


def cuda_available() -> bool:
    try:
        return lib().lssm_backend_loaded() == 1
    except OSError:
        return False


_LIVE_CTX: "weakref.WeakSet[Ctx]" = weakref.WeakSet()


@atexit.register
def _close_live_contexts():
    """At interpreter exit, while the library and this module are still whole, close every
    context that is still open (its sessions, models and buffers first), instead of leaving
    the native teardown to the order in which module globals happen to be cleared."""
    for c in list(_LIVE_CTX):
        try:
            c.close()
        except Exception:
            pass


class Ctx:
    """One per host thread (MetalOps' threading model)."""

    def __init__(self, device: int = 0):
        h = P()
        check(lib().lssm_ctx_create(device, C.byref(h)))
        self.h = h
        self.device = device
        self._deps = []   # weak refs to sessions / models / buffers made on this context
        _LIVE_CTX.add(self)

    def _track(self, obj):
        if len(self._deps) > 256:
            self._deps = [r for r in self._deps if r() is not None]
        self._deps.append(weakref.ref(obj))

    def close(self):
        """Destroys what was made on this context (newest first), then the context, so no
        native object outlives the context it points to."""
        if self.h:
            for r in reversed(self._deps):
                o = r()
                if o is not None:
                    try:
                        (o.close if hasattr(o, "close") else o.free)()
                    except Exception:
                        pass
            self._deps.clear()
            lib().lssm_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # batching (MetalOps::begin_batch / commit_and_wait)
    def begin_batch(self):
        check(lib().lssm_begin_batch(self.h))

    def commit_and_wait(self):
        check(lib().lssm_commit_and_wait(self.h))

    def set_graph_batching(self, enable: bool):
        check(lib().lssm_ctx_set_graph_batching(self.h, 1 if enable else 0))

    def replay_batch(self, times: int = 1):
        check(lib().lssm_replay_batch(self.h, times))

    def batch_active(self) -> bool:
        return lib().lssm_batch_active(self.h) == 1

    def stream(self) -> int:
        return lib().lssm_ctx_stream(self.h) or 0


class DeviceBuffer:
    """Device allocation (stands in for DeviceBuffer / UnifiedBuffer)."""

    def __init__(self, ctx: Ctx, nbytes: int):
        self.ctx = ctx
        self.nbytes = int(nbytes)
        p = P()
        check(lib().lssm_alloc(ctx.h, max(self.nbytes, 1), C.byref(p)))
        self.ptr = p
        ctx._track(self)

    @classmethod
    def from_array(cls, ctx: Ctx, a: np.ndarray, extra: int = 0):
        a = np.ascontiguousarray(a)
        b = cls(ctx, a.nbytes + extra)
        b.upload(a)
        return b

    def upload(self, a: np.ndarray, off: int = 0):
        a = np.ascontiguousarray(a)
        check(lib().lssm_upload(self.ctx.h, self.ptr, off, a.ctypes.data_as(P), a.nbytes))

    def download(self, dtype, count: int, off: int = 0) -> np.ndarray:
        out = np.empty(count, dtype=dtype)
        check(lib().lssm_download(self.ctx.h, out.ctypes.data_as(P), self.ptr, off, out.nbytes))
        return out

    def zero(self):
        check(lib().lssm_memset(self.ctx.h, self.ptr, 0, 0, self.nbytes))

    def free(self):
        if self.ptr:
            lib().lssm_free(self.ctx.h, self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Ops:
    """lite_ssm::MetalOps, method for method. Every tensor argument is a
    (DeviceBuffer, byte_offset) pair; dims are the ops.hpp POD structs."""

    def __init__(self, ctx: Ctx):
        self.ctx = ctx

    @staticmethod
    def _b(x):
        buf, off = x
        return buf.ptr, off

    def _call(self, name, *args):
        check(getattr(lib(), name)(self.ctx.h, *args))

    def rmsnorm_f16(self, x, w, y, dims: RMSNormDims):
        self._call("lssm_rmsnorm_f16", *self._b(x), *self._b(w), *self._b(y), dims)

    def linear_f16_gemv(self, x, w, y, dims: LinearDims):
        self._call("lssm_linear_f16_gemv", *self._b(x), *self._b(w), *self._b(y), dims)

    def linear_silu_f16_gemv(self, x, w, y, dims: LinearDims):
        self._call("lssm_linear_silu_f16_gemv", *self._b(x), *self._b(w), *self._b(y), dims)

    def rmsnorm_linear_f16_gemv(self, x, w_norm, w, y, dims: RMSLinearDims):
        self._call("lssm_rmsnorm_linear_f16_gemv", *self._b(x), *self._b(w_norm), *self._b(w), *self._b(y), dims)

    def linear_f16_gemm(self, x, w, y, dims: LinearDims):
        self._call("lssm_linear_f16_gemm", *self._b(x), *self._b(w), *self._b(y), dims)

    def linear_silu_f16_gemm(self, x, w, y, dims: LinearDims):
        self._call("lssm_linear_silu_f16_gemm", *self._b(x), *self._b(w), *self._b(y), dims)

    def linear_int4_gemv(self, x, w_packed, w_scales, y, dims: LinearDims):
        self._call("lssm_linear_int4_gemv", *self._b(x), *self._b(w_packed), *self._b(w_scales), *self._b(y), dims)

    def linear_int4_gemv_rows(self, x, w_packed, w_scales, y, dims: LinearDims):
        """Batched-decode extension: 1..8 activation rows, weights read once."""
        self._call("lssm_linear_int4_gemv_rows", *self._b(x), *self._b(w_packed), *self._b(w_scales), *self._b(y),
                   dims)

    def linear_f16_gemv_rows(self, x, w, y, dims: LinearDims):
        """Batched-decode extension: 1..8 activation rows, weights read once."""
        self._call("lssm_linear_f16_gemv_rows", *self._b(x), *self._b(w), *self._b(y), dims)

    def linear_int4_gemm(self, x, w_packed, w_scales, y, dims: LinearDims):
        self._call("lssm_linear_int4_gemm", *self._b(x), *self._b(w_packed), *self._b(w_scales), *self._b(y), dims)

    def silu_f16(self, x, y, n):
        self._call("lssm_silu_f16", *self._b(x), *self._b(y), n)

    def add_inplace_f16(self, y, x, n):
        self._call("lssm_add_inplace_f16", *self._b(y), *self._b(x), n)

    def split_silu_xBC_f16(self, xBC, x_out, B_out, C_out, L, d_inner, d_state, n_groups):
        self._call("lssm_split_silu_xBC_f16", *self._b(xBC), *self._b(x_out), *self._b(B_out), *self._b(C_out), L,
                   d_inner, d_state, n_groups)

    def silu_gated_f16(self, x, gate, y, n):
        self._call("lssm_silu_gated_f16", *self._b(x), *self._b(gate), *self._b(y), n)

    def causal_conv1d_f16(self, x, w, bias, y, dims: Conv1dDims):
        self._call("lssm_causal_conv1d_f16", *self._b(x), *self._b(w), *self._b(bias), *self._b(y), dims)

    def causal_conv1d_update_f16(self, x_new, state, w, bias, y, dims: Conv1dDims):
        self._call("lssm_causal_conv1d_update_f16", *self._b(x_new), *self._b(state), *self._b(w), *self._b(bias),
                   *self._b(y), dims)

    def seed_conv_state_f16(self, xBC, state, L, D, K):
        self._call("lssm_seed_conv_state_f16", *self._b(xBC), *self._b(state), L, D, K)

    def inproj_fused_f16(self, normed, W_in, W_conv, conv_b, proj_z, ssd_x, ssd_B, ssd_C, proj_dt, proj_xBC,
                         dims: FusedInProjDims):
        args = []
        for t in (normed, W_in, W_conv, conv_b, proj_z, ssd_x, ssd_B, ssd_C, proj_dt, proj_xBC):
            args += self._b(t)
        self._call("lssm_inproj_fused_f16", *args, dims)

    def ssd_chunked_f16(self, X, B, Cm, dt_raw, dt_bias, A_log, D_skip, Y, state_io, dims: SSDDims):
        args = []
        for t in (X, B, Cm, dt_raw, dt_bias, A_log, D_skip, Y, state_io):
            args += self._b(t)
        self._call("lssm_ssd_chunked_f16", *args, dims)

    def ssd_step_f16(self, x, B, Cm, dt_raw, dt_bias, A_log, D_skip, state, y, dims: SSDStepDims):
        args = []
        for t in (x, B, Cm, dt_raw, dt_bias, A_log, D_skip, state, y):
            args += self._b(t)
        self._call("lssm_ssd_step_f16", *args, dims)

    def ssd_chunked_batched(self, X, B, Cm, dt_raw, dt_bias, A_log, D_skip, Y, state_io, dims: SSDBatchedDims):
        self._call("lssm_ssd_chunked_batched", X.ptr, B.ptr, Cm.ptr, dt_raw.ptr, dt_bias.ptr, A_log.ptr, D_skip.ptr,
                   Y.ptr, state_io.ptr, dims)


class Model:
    """A .ssm model resident in HBM (SSMFile + Mamba2Model)."""

    def __init__(self, ctx: Ctx, handle):
        self.ctx = ctx
        self.h = handle
        ctx._track(self)

    @classmethod
    def load(cls, ctx: Ctx, path: str):
        h = P()
        check(lib().lssm_model_load(ctx.h, str(path).encode(), C.byref(h)))
        return cls(ctx, h)

    @classmethod
    def load_bytes(cls, ctx: Ctx, data: bytes):
        h = P()
        buf = C.create_string_buffer(data, len(data))
        check(lib().lssm_model_load_bytes(ctx.h, C.cast(buf, P), len(data), C.byref(h)))
        return cls(ctx, h)

    @classmethod
    def synthesize(cls, ctx: Ctx, hp: HParams, seed: int, int4: bool):
        h = P()
        check(lib().lssm_model_synthesize(ctx.h, C.byref(hp), seed, 1 if int4 else 0, C.byref(h)))
        return cls(ctx, h)

    def save(self, path: str):
        check(lib().lssm_model_save(self.h, str(path).encode()))

    def config(self) -> HParams:
        hp = HParams()
        check(lib().lssm_model_config(self.h, C.byref(hp)))
        return hp

    def nbytes(self) -> int:
        return int(lib().lssm_model_nbytes(self.h))

    def tensor(self, name: str):
        off, nb, dt = u64(), u64(), u32()
        check(lib().lssm_model_tensor(self.h, name.encode(), C.byref(off), C.byref(nb), C.byref(dt)))
        return off.value, nb.value, dt.value

    def download_bytes(self) -> bytes:
        n = self.nbytes()
        out = np.empty(n, dtype=np.uint8)
        base = lib().lssm_model_device_base(self.h)
        check(lib().lssm_download(self.ctx.h, out.ctypes.data_as(P), base, 0, n))
        return out.tobytes()

    def close(self):
        if self.h:
            lib().lssm_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


COMM_ID_BYTES = 128


class Comm:
    """NCCL communicator of one rank (head tensor parallelism): rank 0 makes the id with
    Comm.unique_id(), the caller shares it (e.g. torch.distributed broadcast), every rank
    builds Comm(ctx, rank, world, uid)."""

    @staticmethod
    def unique_id() -> bytes:
        buf = (C.c_uint8 * COMM_ID_BYTES)()
        check(lib().lssm_comm_unique_id(C.cast(buf, P)))
        return bytes(buf)

    def __init__(self, ctx: Ctx, rank: int, world: int, uid: bytes):
        if len(uid) != COMM_ID_BYTES:
            raise ValueError(f"unique id must be {COMM_ID_BYTES} bytes")
        buf = (C.c_uint8 * COMM_ID_BYTES).from_buffer_copy(uid)
        h = P()
        check(lib().lssm_comm_init(ctx.h, rank, world, C.cast(buf, P), C.byref(h)))
        self.h = h
        self.ctx = ctx
        self.rank, self.world = rank, world
        ctx._track(self)

    def allreduce_f32(self, ptr: int, n: int):
        """Sum n fp32 device values at ptr in place across the ranks (collective)."""
        check(lib().lssm_comm_allreduce_f32(self.h, ptr, n))

    def close(self):
        if self.h:
            lib().lssm_comm_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    """Mamba2State + Mamba2Workspace for `batch` independent sequences. With `comm`, a
    head-tensor-parallel session over this rank's shard of the model (calls are then
    collective: every rank runs them with the same tokens)."""

    def __init__(self, ctx: Ctx, model: Model, batch: int, max_seq_len: int, comm: "Comm | None" = None):
        self.ctx = ctx
        self.model = model
        self.batch = batch
        self.vocab = model.config().vocab_size
        self.comm = comm
        h = P()
        if comm is None:
            check(lib().lssm_session_create(ctx.h, model.h, batch, max_seq_len, C.byref(h)))
        else:
            check(lib().lssm_session_create_tp(ctx.h, model.h, comm.h, batch, max_seq_len, C.byref(h)))
        self.h = h
        ctx._track(self)

    def reset(self):
        check(lib().lssm_session_reset(self.h))

    def set_option(self, key: str, value: int):
        check(lib().lssm_session_set_option(self.h, key.encode(), int(value)))

    def prefill(self, tokens: np.ndarray) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32).reshape(self.batch, -1)
        nxt = np.zeros(self.batch, dtype=np.uint32)
        check(lib().lssm_prefill(self.h, t.ctypes.data_as(P), t.shape[1], nxt.ctypes.data_as(P)))
        return nxt

    def decode(self, first: np.ndarray, n_steps: int) -> np.ndarray:
        f = np.ascontiguousarray(first, dtype=np.uint32).reshape(self.batch)
        out = np.zeros((self.batch, n_steps), dtype=np.uint32)
        check(lib().lssm_decode(self.h, f.ctypes.data_as(P), n_steps, out.ctypes.data_as(P)))
        return out

    def generate(self, prompt: np.ndarray, max_new: int, eos: int = 0xFFFFFFFF) -> np.ndarray:
        t = np.ascontiguousarray(prompt, dtype=np.uint32).reshape(self.batch, -1)
        out = np.zeros((self.batch, max_new), dtype=np.uint32)
        n = u32()
        check(lib().lssm_generate(self.h, t.ctypes.data_as(P), t.shape[1], max_new, eos, out.ctypes.data_as(P),
                                  C.byref(n)))
        return out[:, : n.value]

    def logits(self) -> np.ndarray:
        out = np.zeros((self.batch, self.vocab), dtype=np.float32)
        check(lib().lssm_session_logits(self.h, out.ctypes.data_as(P)))
        return out

    def timing(self):
        a, b = f32(), f32()
        check(lib().lssm_session_timing(self.h, C.byref(a), C.byref(b)))
        return a.value, b.value

    def launches(self):
        a, b = u64(), u64()
        check(lib().lssm_session_launches(self.h, C.byref(a), C.byref(b)))
        return a.value, b.value

    def trace(self) -> np.ndarray:
        """Phase stamps of the last persistent decode (set_option("trace", 1) first):
        (sm_count, n_layer * 10 + 6) uint64, layout as lssm_session_trace documents."""
        n = u64()
        check(lib().lssm_session_trace(self.h, None, 0, C.byref(n)))
        out = np.zeros(n.value, dtype=np.uint64)
        check(lib().lssm_session_trace(self.h, out.ctypes.data_as(C.POINTER(u64)), n.value, C.byref(n)))
        return out.reshape(-1, self.model.config().n_layer * 10 + 6)

    def close(self):
        if self.h:
            lib().lssm_session_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def tp_shard_plan(hp: dict, rank: int, world: int) -> dict:
    """Which model rows / columns rank `rank` of `world` holds under head tensor
    parallelism (the layout lssm_session_create_tp copies): in_proj row segments
    [z | x | B | C | dt], conv channel segments [x | B | C], the head slice, the d_inner
    column slice of out_proj / mixer norm, and the lm_head vocab slice."""
    H, G, P, N = hp["n_heads"], hp["n_groups"], hp["d_head"], hp["d_state"]
    if H % world or G % world:
        raise ValueError("n_heads and n_groups must divide by the world size")
    di = hp["expand"] * hp["d_model"]
    GN, Hr, Gr = G * N, H // world, G // world
    dir_, GNr = Hr * P, Gr * N
    xd = di + 2 * GN
    V = hp["vocab_size"]
    vmax = -(-V // world)
    voff = min(V, rank * vmax)
    return {
        "in_rows": [(rank * dir_, dir_), (di + rank * dir_, dir_), (2 * di + rank * GNr, GNr),
                    (2 * di + GN + rank * GNr, GNr), (di + xd + rank * Hr, Hr)],
        "conv_channels": [(rank * dir_, dir_), (di + rank * GNr, GNr), (di + GN + rank * GNr, GNr)],
        "heads": (rank * Hr, Hr),
        "inner_cols": (rank * dir_, dir_),
        "vocab": (voff, min(vmax, V - voff)),
    }


def hparams(**kw) -> HParams:
    hp = HParams()
    defaults = dict(d_conv=4, expand=2, chunk_size=256, default_dtype=0, n_groups=1, norm_before_gate=0)
    defaults.update(kw)
    for k, v in defaults.items():
        setattr(hp, k, int(v))
    return hp


def f16(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32).astype(np.float16))


if os.environ.get("LSSM_EAGER_LOAD"):
    lib()
