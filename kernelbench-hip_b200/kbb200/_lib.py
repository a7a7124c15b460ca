"""ctypes binding of libkbb200.so — the C ABI declared in include/kbb200.h.

The library is loaded from this package directory (built in-tree by
kernelbench-hip_b200/build.py).  There is no fallback: if the shared library
is missing or a symbol is absent, importing this module raises, so no
operator can silently run anywhere but on the CUDA kernels.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(os.environ.get("KBB200_LIB", Path(__file__).resolve().parent / "libkbb200.so"))

_p = C.c_void_p
_f = C.POINTER(C.c_float)
_i64 = C.c_int64
_sz = C.c_size_t
_int = C.c_int
_float = C.c_float

# name -> (restype, argtypes); must match include/kbb200.h exactly
SIGNATURES: dict[str, tuple] = {
    "kb_version": (_int, []),
    "kb_status_string": (C.c_char_p, [_int]),
    "kb_last_error": (C.c_char_p, []),
    "kb_device_sm_count": (_int, [_int]),
    "kb_read_fault": (_int, [_int, C.POINTER(C.c_int)]),
    "kb_gelu_tanh_f32": (_int, [_p, _p, _i64, _p]),
    "kb_gelu_erf_f32": (_int, [_p, _p, _i64, _p]),
    "kb_swish_f32": (_int, [_p, _p, _i64, _p]),
    "kb_relu_f32": (_int, [_p, _p, _i64, _p]),
    "kb_diag_matmul_f32": (_int, [_p, _p, _p, _i64, _i64, _p]),
    "kb_layernorm_f32": (_int, [_p, _p, _p, _p, _i64, _i64, _float, _p]),
    "kb_rmsnorm_f32": (_int, [_p, _p, _p, _i64, _i64, _i64, _float, _p]),
    "kb_softmax_f32": (_int, [_p, _p, _i64, _i64, _p]),
    "kb_logsoftmax_f32": (_int, [_p, _p, _i64, _i64, _p]),
    "kb_sum_dim1_f32": (_int, [_p, _p, _i64, _i64, _i64, _p]),
    "kb_mean_dim1_f32": (_int, [_p, _p, _i64, _i64, _i64, _p]),
    "kb_argmax_dim1_f32": (_int, [_p, _p, _i64, _i64, _i64, _p]),
    "kb_mse_workspace_size": (_sz, [_i64]),
    "kb_mse_f32": (_int, [_p, _p, _p, _i64, _p, _sz, _p]),
    "kb_mse_partial_f64": (_int, [_p, _p, _p, _i64, _p, _sz, _p]),
    "kb_mse_finalize_f32": (_int, [_p, _p, _i64, _p]),
    "kb_frobenius_workspace_size": (_sz, [_i64]),
    "kb_frobenius_normalize_f32": (_int, [_p, _p, _i64, _p, _sz, _p]),
    "kb_sumsq_partial_f64": (_int, [_p, _p, _i64, _p, _sz, _p]),
    "kb_scale_by_inv_norm_f32": (_int, [_p, _p, _i64, _p, _p]),
    "kb_maxpool2d_f32": (_int, [_p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _int, _int, _int, _int, _p]),
    "kb_batchnorm_workspace_size": (_sz, [_i64, _i64, _i64]),
    "kb_batchnorm_train_f32": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _float, _float, _p, _p, _p, _sz, _p]),
    "kb_batchnorm_train_f32_noalloc": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _float, _float, _p, _p, _p]),
    "kb_batchnorm_stats_f64": (_int, [_p, _p, _i64, _i64, _i64, _p, _sz, _p]),
    "kb_batchnorm_apply_f32": (_int, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _float, _float, _p, _p, _p]),
    "kb_sgemm_3xtf32": (_int, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _int, _p]),
    "kb_sgemm_workspace_size": (_sz, [_i64, _i64, _i64, _int]),
    "kb_sgemm_3xtf32_ws": (_int, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "kb_bgemm_3xtf32": (_int, [_p, _p, _p, _i64, _i64, _i64, _i64, _p]),
    "kb_gemm_splitk_workspace_size": (_sz, [_i64, _i64, _i64]),
    "kb_gemm_splitk_3xtf32": (_int, [_p, _p, _p, _i64, _i64, _i64, _p, _sz, _p]),
    "kb_gemv_f32": (_int, [_p, _p, _p, _i64, _i64, _p]),
    "kb_avgpool2d_f32": (_int, [_p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _int, _int, _int, _int, _int,
                                _p]),
    "kb_cumsum_f32": (_int, [_p, _p, _i64, _i64, _i64, _p]),
    "kb_cross_entropy_workspace_size": (_sz, [_i64]),
    "kb_cross_entropy_f32": (_int, [_p, _p, _p, _i64, _i64, _i64, _p, _sz, _p]),
    "kb_cross_entropy_partial_f64": (_int, [_p, _p, _p, _i64, _i64, _i64, _p, _sz, _p]),
    "kb_cross_entropy_finalize_f32": (_int, [_p, _p, _p]),
    "kb_p2p_header_bytes": (_sz, []),
    "kb_p2p_buffer_bytes": (_sz, [_sz, _int]),
    "kb_p2p_buffer_alloc": (_int, [_sz, C.POINTER(C.c_void_p)]),
    "kb_p2p_buffer_free": (_int, [_p]),
    "kb_p2p_ipc_handle": (_int, [_p, _p]),
    "kb_p2p_ipc_open": (_int, [_p, C.POINTER(C.c_void_p)]),
    "kb_p2p_ipc_close": (_int, [_p]),
    "kb_p2p_read_fault": (_int, [_int, C.POINTER(C.c_int)]),
    "kb_p2p_allreduce_f64": (_int, [_p, _int, _int, _sz, _p, _p, _i64, C.c_uint, C.c_uint64, _p]),
    "kb_p2p_allreduce_f32": (_int, [_p, _int, _int, _sz, _p, _p, _i64, C.c_uint, C.c_uint64, _p]),
    "kb_p2p_splitk_allreduce_f32": (_int, [_p, _int, _int, _sz, _p, _int, _p, _i64, C.c_uint, C.c_uint64,
                                           _p]),
    "kb_sharded_workspace_size": (_sz, []),
    "kb_mse_sharded_f32": (_int, [_p, _p, _p, _i64, _p, _sz, _p, _int, _int, _sz, C.c_uint, C.c_uint64, _p]),
    "kb_sumsq_sharded_f64": (_int, [_p, _p, _i64, _p, _sz, _p, _int, _int, _sz, C.c_uint, C.c_uint64, _p]),
    "kb_batchnorm_sharded_workspace_size": (_sz, [_i64, _i64, _i64]),
    "kb_batchnorm_stats_sharded_f64": (_int, [_p, _p, _i64, _i64, _i64, _p, _sz, _p, _int, _int, _sz, C.c_uint,
                                              C.c_uint64, _p]),
    "kb_gemm_splitk_partials_workspace_size": (_sz, [_i64, _i64, _i64]),
    "kb_gemm_splitk_partials_3xtf32": (_int, [_p, _p, _i64, _i64, _i64, _p, _sz, C.POINTER(C.c_int), _p]),
}


class KbError(RuntimeError):
    """A C-ABI entry returned a non-zero kbStatus."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed with status {status}: {msg}")
        self.fn, self.status, self.msg = fn, status, msg


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python kernelbench-hip_b200/build.py` "
            "(the operators have no non-CUDA fallback)")
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError if the symbol is not exported
        fn.restype = res
        fn.argtypes = args
    return lib


LIB = _load()


def check(fn_name: str, status: int) -> None:
    if status != 0:
        msg = LIB.kb_last_error().decode(errors="replace")
        raise KbError(fn_name, status, msg)


def read_fault(clear: bool = True) -> int:
    """Device fault word (nonzero if a kernel abandoned a bounded wait)."""
    v = C.c_int(0)
    check("kb_read_fault", LIB.kb_read_fault(1 if clear else 0, C.byref(v)))
    return v.value


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
