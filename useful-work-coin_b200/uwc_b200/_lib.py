"""ctypes binding of libuwcb200.so (include/uwc_b200.h).

The library must have been built (useful-work-coin_b200/build.py, or __graft_entry__.build()).
There is no fallback: if it is missing, every operation raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libuwcb200.so")

OK, ERR_ARG, ERR_SHAPE, ERR_ALIGN, ERR_CUDA, ERR_DEVICE, ERR_SCRATCH = range(7)
DEV_TIMEOUT = 1
HOOK_WAIT_NS, HOOK_WITHHOLD, HOOK_STREAM_PDL, HOOK_TP_TWO_PHASE = 1, 2, 3, 4

# (name, restype, argtypes) for every function declared in include/uwc_b200.h
_P, _U32, _U64, _I32, _F64 = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int, ctypes.c_double
_I64, _F32 = ctypes.c_longlong, ctypes.c_float
SIGNATURES = {
    "uwc_version": (_I32, []),
    "uwc_launch_count": (_U64, []),
    "uwc_test_hook": (_I32, [_I32, _I64]),
    "uwc_status_string": (ctypes.c_char_p, [_I32]),
    "uwc_device_status": (_I32, [ctypes.POINTER(ctypes.c_uint32), _I32]),
    "uwc_b3_scratch_words": (_U64, [_U64]),
    "uwc_b3_root_and_seed": (_I32, [_P, _U64, _P, _P, _P, _U32, _P, _P, _P, _U64, _P]),
    "uwc_b3_noalloc_max_bytes": (_U64, []),
    "uwc_b3_noalloc_forget": (None, []),
    "uwc_b3_root_and_seed_noalloc": (_I32, [_P, _U64, _P, _P, _P, _U32, _P, _P, _P]),
    "uwc_noise_uniform": (_I32, [_P, _U64, _P, _P, _P, _I32, _P]),
    "uwc_noise_perm": (_I32, [_P, _U32, _U32, _P, _P, _P]),
    "uwc_noise_rows": (_I32, [_P, _I32, _I32, _I32, _P, _P, _P, _P, _P, _I32, _I32, _P, _I32, _P]),
    "uwc_proj_matrix": (_I32, [_P, _I32, _I32, _P, _P]),
    "uwc_proj_corr": (_I32, [_P, _I32, _I32, _P, _I32, _P, _I32, _P]),
    "uwc_gemm_workspace_bytes": (_U64, [_I32, _I32, _I32, _I32]),
    "uwc_gemm": (_I32, [_P, _P, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _I32, _P, _P, _P, _I32, _P, _P, _P, _I32,
                        _P, _U64, _P]),
    "uwc_gemm_stream": (_I32, [_P, _P, _I32, _I32, _I32, _P, _P, _P, _P, _I32, _P]),
    "uwc_gemm_epi_workspace_bytes": (_U64, [_I32, _I32, _I32]),
    "uwc_gemm_epi": (_I32, [_P, _P, _I32, _I32, _I32, _P, _P, _P, _P, _I32, _P, _U64, _P]),
    "uwc_tp_buffer_bytes": (_U64, [_I32, _I32]),
    "uwc_tp_alloc": (_I32, [_I32, _I32, _P]),
    "uwc_tp_free": (_I32, [_P]),
    "uwc_ipc_handle": (_I32, [_P, _P]),
    "uwc_ipc_open": (_I32, [_P, _P]),
    "uwc_ipc_close": (_I32, [_P]),
    "uwc_tp_barrier": (_I32, [_P, _P]),
    "uwc_quant_act_tp": (_I32, [_P, _I32, _I32, _I32, _P, _P, _P, _P]),
    "uwc_gemm_stream_tp": (_I32, [_P, _P, _I32, _I32, _I32, _P, _P, _P, _P, _I32, _P, _P]),
    "uwc_mined_block_layout": (_I32, [_I32, _I32, _I32, _P]),
    "uwc_mined_workspace_layout": (_I32, [_I32, _I32, _I32, _I32, _I32, _I32, _I32, _P]),
    "uwc_mined_setup_block": (_I32, [_P, _I32, _I32, _I32, _P, _P, _P, _U64, _P, _U64, _P]),
    "uwc_mine_attempt": (_I32, [_P, _I32, _I32, _I32, _I32, _P, _P, _I32, _P, _U64, _P]),
    "uwc_mined_forward": (_I32, [_P, _I32, _I32, _I32, _I32, _P, _P, _P, _I32, _P, _I32, _P, _I32, _P, _U64, _P]),
    "uwc_peak_i8": (_I32, [_I32, _P]),
    "uwc_peak_i8_ops": (ctypes.c_double, [_I32]),
    "uwc_quant_act": (_I32, [_P, _I32, _I32, _I32, _P, _P, _P]),
    "uwc_quant_rows_had": (_I32, [_P, _I32, _I32, _I32, _P, _P, _P]),
    "uwc_fwht_absmax": (_I32, [_P, _I32, _I32, _I32, _P, _P]),
    "uwc_quant_act_global": (_I32, [_P, _I32, _I32, _I32, _P, _P, _P, _P]),
    "uwc_rmsnorm_quant": (_I32, [_P, _P, _I32, _I32, _I32, _F64, _P, _P, _P]),
    "uwc_swiglu_quant": (_I32, [_P, _P, _P, _I32, _I32, _I32, _P, _P, _P]),
    "uwc_swiglu": (_I32, [_P, _P, _P, _I32, _I32, _P, _P]),
    "uwc_dequant_residual": (_I32, [_P, _P, _P, _P, _I32, _I32, _P, _P]),
    "uwc_qkv_post": (_I32, [_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _F64, _I32, _P, _P, _P, _P, _P, _P,
                            _P]),
    "uwc_attention": (_I32, [_P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I64, _I64, _I64, _I64, _I64, _I64,
                             _F32, _P, _P]),
    "uwc_attention_tc_workspace_bytes": (_U64, [_I32, _I32, _I32, _I32, _I32]),
    "uwc_attention_tc": (_I32, [_P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I64, _I64, _I64, _I64, _I64,
                                _I64, _F32, _P, _P, _U64, _P]),
    "uwc_gemm_batched": (_I32, [_P, _P, _I32, _I32, _I32, _I32, _I64, _I64, _I32, _I32, _I32, _I32, _P, _P]),
    "uwc_attention_at": (_I32, [_P, _P, _P, _P, _P, _P, _I32, _I32, _P, _I32, _I32, _I32, _I64, _I64, _I64, _I64,
                                _I64, _I64, _F32, _P, _P]),
    "uwc_kv_append": (_I32, [_P, _P, _P, _P, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P]),
    "uwc_qkv_post_at": (_I32, [_P, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _F64, _I32, _P, _P, _P, _P,
                               _P, _P, _P]),
    "uwc_qkv_post_kv": (_I32, [_P, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _F64, _I32, _P, _P, _P, _P,
                               _P, _P, _I32, _P]),
    "uwc_rmsnorm": (_I32, [_P, _P, _I32, _I32, _F64, _P, _P]),
    "uwc_logprobs": (_I32, [_P, _I32, _I32, _P, _P, _P]),
    "uwc_stage_scratch_words": (_U64, [_I64, _I32]),
    "uwc_stage_out_leaves": (_I32, [_P, _I64, _I32, _I32, _P, _U64, _P, _P]),
    "uwc_stage_roots": (_I32, [_P, _I32, _I32, _I32, _P, _U64, _P, _P]),
}

_LIB = None


class UWCError(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise UWCError(f"{LIB_PATH} is missing: build it with useful-work-coin_b200/build.py "
                           "(there is no CPU or library fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def check(rc: int, what: str) -> None:
    """Raise like the reference does: shape/alignment/argument violations are AssertionErrors
    (ops.py:191-192 asserts), CUDA/device problems are RuntimeErrors."""
    if rc == OK:
        return
    msg = f"{what}: {lib().uwc_status_string(rc).decode()} (status {rc})"
    if rc in (ERR_ARG, ERR_SHAPE, ERR_ALIGN, ERR_SCRATCH):
        raise AssertionError(msg)
    raise UWCError(msg)


def launch_count() -> int:
    """Kernels this library has launched in this process so far (a counter in the library)."""
    return int(lib().uwc_launch_count())


def device_status(clear: bool = True) -> int:
    """Sticky device-side error bits (DEV_TIMEOUT); synchronizes the current device."""
    v = ctypes.c_uint32(0)
    check(lib().uwc_device_status(ctypes.byref(v), 1 if clear else 0), "uwc_device_status")
    return int(v.value)
