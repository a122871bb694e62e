"""CPU: liblssm_cuda.so loads and exports every symbol include/lssm_cuda.h declares,
and answers the kernel-presence probe for the reference's kernel list
(tests/test_metal_ops.cpp:31-49). No compute calls (no GPU here)."""

import ctypes as C
import re
from pathlib import Path

import lssm

ROOT = Path(__file__).resolve().parent.parent

REFERENCE_KERNELS = [
    "lite_ssm_common_noop", "rmsnorm_f16", "silu_f16", "silu_gated_f16", "linear_f16_gemv",
    "linear_silu_f16_gemv", "rmsnorm_linear_f16_gemv", "linear_f16_gemm", "linear_silu_f16_gemm",
    "causal_conv1d_f16", "causal_conv1d_update_f16", "ssd_chunked_f16", "ssd_step_f16", "linear_int4_gemv",
    "linear_int4_gemm", "seed_conv_state_f16", "inproj_fused_f16",
]


def declared_symbols():
    text = (ROOT / "include" / "lssm_cuda.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lssm_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = C.CDLL(str(lssm.LIB_PATH))
    names = declared_symbols()
    assert len(names) > 40
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_kernel_registry_lists_reference_kernels():
    for k in REFERENCE_KERNELS:
        assert lssm.lib().lssm_has_kernel(k.encode()) == 1, k
    assert lssm.lib().lssm_has_kernel(b"not_a_kernel") == 0


def test_version_and_errors_without_device():
    assert b"sm_100a" in lssm.lib().lssm_version()
    # No CUDA device in the build container: the backend reports not loaded and
    # context creation fails loudly instead of falling back to the CPU.
    if lssm.lib().lssm_backend_loaded() == 0:
        h = C.c_void_p()
        rc = lssm.lib().lssm_ctx_create(0, C.byref(h))
        assert rc != 0
        assert lssm.lib().lssm_last_error()
