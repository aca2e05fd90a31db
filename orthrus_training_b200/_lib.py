"""ctypes binding of liborthrus_b200.so (the C ABI in include/orthrus_b200.h).

The library is built in-tree by ``build_lib.py``. There is no fallback: on a machine with a GPU,
every op of this package runs through the library, and importing an op without it raises.
"""

from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_size_t, c_uint, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "liborthrus_b200.so"

OK, EINVAL, ECUDA, EWORKSPACE, EDEVICE = 0, -1, -2, -3, -4
BF16, F32 = 0, 1
MASK_CAUSAL, MASK_DUAL, MASK_DRAFT, MASK_TREE = 0, 1, 2, 3
ERR_TIMEOUT, ERR_BOUNDS = 1, 2

_P = c_void_p
_SIGNATURES = {
    "orthrus_version": (c_int, []),
    "orthrus_launch_count": (ctypes.c_ulonglong, []),
    "orthrus_device_error": (c_int, [c_int, ctypes.POINTER(c_uint), c_int]),
    "orthrus_selftest_bounded_wait": (c_int, [_P, ctypes.c_uint64, _P, _P]),
    "orthrus_gemm_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64]),
    "orthrus_gemm_bf16": (c_int, [_P, c_int64, _P, c_int64, _P, c_int64, c_int64, c_int64, c_int64,
                                  c_int, c_int, _P, c_size_t, _P]),
    "orthrus_gemm2_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64]),
    "orthrus_gemm2_bf16": (c_int, [_P, c_int64, c_int, _P, c_int64, c_int, _P, c_int64, _P, c_int64,
                                   c_int64, c_int64, c_int64, c_int, _P, c_size_t, _P]),
    "orthrus_linear_bf16": (c_int, [_P, c_int64, _P, c_int64, _P, _P, c_int64, c_int64, c_int64,
                                    c_int64, c_int, _P]),
    "orthrus_linear_skinny_bf16": (c_int, [_P, c_int64, _P, c_int64, _P, _P, c_int64, c_int64, c_int64,
                                           c_int64, c_int, _P]),
    "orthrus_linear_swiglu_keep_bf16": (c_int, [_P, _P, c_int64, c_int64, c_int64, _P, _P, _P]),
    "orthrus_linear_qkv_rope_keep_bf16": (c_int, [_P, _P, _P, _P, _P, _P, c_int64, _P, c_int64, c_int64,
                                                  c_int64, c_int, c_int, c_float, _P, _P, _P, _P, _P, _P]),
    "orthrus_rope_table_bf16": (c_int, [_P, c_int64, c_int, _P, _P, _P]),
    "orthrus_linear_qkv_rope_bf16": (c_int, [_P, _P, _P, _P, _P, _P, c_int64, c_int64, c_int64, c_int,
                                             c_int, c_float, _P, _P, _P, _P]),
    "orthrus_gemm_simt_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64]),
    "orthrus_gemm_simt": (c_int, [_P, c_int64, _P, c_int64, _P, c_int64, c_int64, c_int64, c_int64,
                                  c_int, _P, c_size_t, _P]),
    "orthrus_rmsnorm": (c_int, [_P, _P, c_int64, c_int, c_float, _P, _P, c_int, _P]),
    "orthrus_rmsnorm_bwd_add": (c_int, [_P, _P, _P, _P, _P, c_int64, c_int, _P, _P]),
    "orthrus_rmsnorm_bwd": (c_int, [_P, _P, _P, _P, c_int64, c_int, _P, c_int, _P]),
    "orthrus_swiglu_fwd": (c_int, [_P, c_int64, c_int, _P, c_int, _P]),
    "orthrus_swiglu_bwd": (c_int, [_P, _P, c_int64, c_int, _P, c_int, _P]),
    "orthrus_qkv_prep_fwd": (c_int, [_P, _P, _P, _P, _P, c_int64, c_int64, c_int, c_int, c_int, c_int,
                                     c_float, _P, _P, _P, c_int64, _P, _P, c_int, _P]),
    "orthrus_qkv_prep_bwd_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int]),
    "orthrus_qkv_prep_bwd": (c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, c_int64, c_int64, c_int,
                                     c_int, c_int, c_int, _P, _P, _P, _P, c_size_t, c_int, _P]),
    "orthrus_attn_tilemap": (c_int, [_P, c_int64, c_int64, c_int, c_int64, _P, _P]),
    "orthrus_attn_fwd": (c_int, [_P, _P, _P, c_int64, c_int64, c_int64, _P, _P, c_int64, c_int64,
                                 c_int64, c_int64, c_int, c_int, c_int64, c_int, c_int, c_float, c_int,
                                 _P, c_int64, c_int, _P, _P, _P, _P, c_int, _P]),
    "orthrus_attn_fwd_doc": (c_int, [_P, _P, _P, c_int64, c_int64, c_int64, _P, _P, c_int64, c_int64,
                                     c_int64, c_int64, c_int, c_int, c_int64, c_int, c_int, c_float, c_int,
                                     _P, c_int64, c_int, _P, _P, _P, _P, _P, c_int, _P]),
    "orthrus_attn_bwd_doc": (c_int, [_P, _P, _P, c_int64, c_int64, c_int64, _P, _P, c_int64, c_int64,
                                     c_int64, c_int64, c_int, c_int, c_int64, c_int, c_int, c_float, _P,
                                     c_int64, c_int, _P, _P, _P, _P, _P, _P, _P, _P, c_size_t, c_int, _P]),
    "orthrus_attn_bwd_workspace_bytes": (c_size_t, [c_int64, c_int, c_int64]),
    "orthrus_attn_decode_workspace_bytes": (c_size_t, [c_int64, c_int, c_int64, c_int64]),
    "orthrus_attn_decode_fwd": (c_int, [_P, _P, _P, c_int64, c_int64, c_int64, _P, _P, c_int64, c_int64,
                                        c_int64, c_int64, c_int, c_int, c_int64, c_float, c_int, _P, _P, _P,
                                        _P, c_size_t, _P]),
    "orthrus_attn_bwd": (c_int, [_P, _P, _P, c_int64, c_int64, c_int64, _P, _P, c_int64, c_int64,
                                 c_int64, c_int64, c_int, c_int, c_int64, c_int, c_int, c_float, _P,
                                 c_int64, c_int, _P, _P, _P, _P, _P, _P, _P, c_size_t, c_int, _P]),
    "orthrus_attn_bwd_noalloc": (c_int, [_P, _P, _P, c_int64, c_int64, c_int64, _P, _P, c_int64,
                                         c_int64, c_int64, c_int64, c_int, c_int, c_int64, c_int,
                                         c_int, c_float, _P, c_int64, c_int, _P, _P, _P, _P, _P, _P,
                                         c_int, _P]),
    "orthrus_lmhead_kl_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int64,
                                                     c_int]),
    "orthrus_lmhead_kl_fwd": (c_int, [_P, c_int64, _P, c_int64, _P, _P, c_int64, c_int64, _P, _P,
                                      c_int, _P, _P, _P, _P, _P, _P, c_int64, _P, c_size_t, c_int,
                                      _P]),
    "orthrus_lmhead_kl_bwd": (c_int, [_P, _P, _P, c_int64, c_int, _P]),
    "orthrus_argmax_rows": (c_int, [_P, c_int64, c_int64, c_int64, _P, _P]),
    "orthrus_decode_draft": (c_int, [_P, c_int64, c_int, c_int64, _P, _P, _P, _P]),
    "orthrus_decode_verify_accept": (c_int, [_P, c_int64, c_int, c_int64, _P, _P, _P, c_int, _P, _P,
                                             _P, _P, _P, _P, c_int64, _P, _P, c_int64, _P]),
    "orthrus_sample_probs": (c_int, [_P, c_int64, c_int, c_float, c_int, c_float, _P, _P]),
    "orthrus_sample_rows": (c_int, [_P, _P, c_int64, c_int, c_float, c_int, c_float, ctypes.c_uint64, _P,
                                    _P, _P]),
    "orthrus_decode_sample_draft": (c_int, [_P, _P, c_int64, c_int, c_int, c_float, c_int, c_float,
                                            ctypes.c_uint64, _P, _P, _P, _P, _P, _P]),
    "orthrus_decode_sample_accept": (c_int, [_P, _P, _P, _P, c_int64, c_int, c_int, c_float, c_int,
                                             c_float, ctypes.c_uint64, _P, _P, c_int, _P, _P, _P, _P, _P,
                                             _P, c_int64, _P, _P, c_int64, _P]),
    "orthrus_philox4x32_10": (c_int, [_P, c_int64, _P, _P]),
    "orthrus_lmhead_argmax_workspace_bytes": (c_size_t, [c_int64]),
    "orthrus_lmhead_argmax_bf16": (c_int, [_P, c_int64, _P, c_int64, c_int64, _P, _P, c_size_t, _P]),
    "orthrus_decode_draft_ids": (c_int, [_P, c_int64, c_int, _P, _P, _P, _P]),
    "orthrus_decode_accept_ids": (c_int, [_P, c_int64, c_int, _P, _P, c_int, _P, _P, _P, _P, _P, _P, c_int64,
                                          _P, _P, c_int64, _P]),
}

_lib = None


class OrthrusError(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it has not been built (no fallback path exists)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise OrthrusError(
                f"{LIB_PATH.name} is not built: run `python -m orthrus_training_b200.build_lib`")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(handle, name, None)
            if fn is None:
                continue
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def check(status: int, what: str) -> None:
    if status == OK:
        return
    if status == EINVAL:
        raise ValueError(f"{what}: invalid arguments (shape, dtype or alignment)")
    if status == EWORKSPACE:
        raise OrthrusError(f"{what}: workspace too small")
    raise OrthrusError(f"{what}: CUDA error (status {status})")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return BF16
    if dtype == torch.float32:
        return F32
    raise ValueError(f"unsupported dtype {dtype}: the kernels take bfloat16 or float32")


def launch_count() -> int:
    return int(lib().orthrus_launch_count())


def device_error(device: int = 0, clear: bool = True) -> int:
    word = c_uint(0)
    lib().orthrus_device_error(device, ctypes.byref(word), int(clear))
    return word.value


def raise_on_device_error(device: int = 0) -> None:
    word = device_error(device, clear=True)
    if word:
        kinds = [n for bit, n in ((ERR_TIMEOUT, "bounded wait timed out"),
                                  (ERR_BOUNDS, "index out of bounds")) if word & bit]
        raise OrthrusError(f"device error word {word:#x}: {', '.join(kinds)}")
