"""ctypes binding of ``libnl_ops.so`` — the C ABI declared in ``include/nl_ops.h``.

This is the same binding a ctypes- or FFI-based caller of the reference would
add for its custom-call targets: plain pointers, sizes and a stream handle.
Tensors are passed as ``tensor.data_ptr()``; the stream is the current torch
CUDA stream, so kernels order with surrounding torch work and are captured by
CUDA graphs.

There is no fallback: if the library is missing, importing an operator that
needs it raises, naming the build command.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_longlong, c_size_t, c_ulonglong, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libnl_ops.so")

STATUS = {0: "NL_OK", -1: "NL_ERR_SHAPE", -2: "NL_ERR_ALIGN", -3: "NL_ERR_LAUNCH", -4: "NL_ERR_CUDA",
          -5: "NL_ERR_DTYPE", -6: "NL_ERR_WORKSPACE", -7: "NL_ERR_TOO_LARGE"}
F32, BF16 = 0, 1
EPI_STORE, EPI_ACCUM, EPI_BIAS, EPI_BIAS_GELU, EPI_RESID, EPI_DGELU = 0, 1, 2, 3, 4, 5

# name -> argtypes (restype is int unless listed in _RESTYPE)
SIGNATURES: dict[str, list] = {
    "nl_version": [],
    "nl_get_device_error": [c_void_p],
    "nl_launch_count": [],
    "nl_gemm": [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p],
    "nl_gemm_ex": [c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int,
                   c_float, c_int, c_void_p, c_void_p, c_void_p, c_void_p],
    "nl_ce_fwd": [c_void_p, c_longlong, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p],
    "nl_ce_bwd": [c_void_p, c_longlong, c_int, c_void_p, c_void_p, c_void_p, c_longlong, c_int, c_int, c_int,
                  c_float, c_void_p],
    "nl_ce_fwd_bwd": [c_void_p, c_longlong, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_longlong, c_int,
                      c_int, c_int, c_float, c_void_p],
    "nl_flash_attention_fwd": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p],
    "nl_flash_attention_bwd": [c_void_p] * 11 + [c_int, c_int, c_int, c_void_p],
    "nl_flash_attention_bwd_dq": [c_void_p] * 8 + [c_int, c_int, c_int, c_void_p],
    "nl_flash_attention_bwd_dkdv": [c_void_p] * 8 + [c_int, c_int, c_int, c_void_p],
    "nl_flash_attention_workspace_bytes": [c_int, c_int, c_int, c_int, c_int],
    "nl_flash_attention_fwd_dt": [c_void_p] * 5 + [c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p],
    "nl_flash_attention_bwd_dq_dt": [c_void_p] * 7 + [c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p],
    "nl_flash_attention_bwd_dkdv_dt": [c_void_p] * 8 + [c_int, c_int, c_int, c_int, c_void_p, c_size_t,
                                                        c_void_p],
    "nl_flash_attention_bwd_noalloc_max_rows": [],
    "nl_flash_attention_bwd_noalloc": [c_void_p] * 9 + [c_int, c_int, c_int, c_void_p],
    "nl_flash_attention_fwd_strided": [c_void_p] * 3 + [c_longlong] * 3 + [c_void_p] + [c_longlong] * 3 +
                                      [c_void_p, c_int, c_int, c_int, c_int, c_void_p],
    "nl_flash_attention_bwd_strided": [c_void_p] * 3 + [c_longlong] * 3 + [c_void_p] * 2 + [c_longlong] * 3 +
                                      [c_void_p] * 6 + [c_int, c_int, c_int, c_int, c_void_p],
    "nl_embed_fwd": [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p],
    "nl_embed_bwd": [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p],
    "nl_layernorm_fwd": [c_void_p] * 6 + [c_int, c_int, c_float, c_void_p],
    "nl_layernorm_bwd": [c_void_p] * 10 + [c_int, c_int, c_int, c_void_p],
    "nl_colsum_bf16": [c_void_p, c_void_p, c_int, c_int, c_void_p],
    "nl_adamw_step": [c_void_p] * 5 + [c_longlong, c_void_p, c_float, c_float, c_float, c_float, c_int, c_void_p],
    "nl_adamw_schedule": [c_void_p, c_void_p, c_float, c_int, c_int, c_float, c_float, c_float, c_void_p],
    "nl_decode_embed": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p],
    "nl_decode_workspace_bytes": [c_int, c_int, c_int],
    "nl_decode_attention": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_int, c_int, c_int, c_int,
                            c_void_p],
    "nl_sample_tokens": [c_void_p, c_longlong, c_int, c_float, c_ulonglong, c_void_p, c_void_p, c_void_p,
                         c_longlong, c_int, c_void_p],
    "nl_decode_advance": [c_void_p, c_void_p],
    "nl_linear_ln_small": [c_void_p, c_longlong, c_void_p, c_void_p, c_float, c_void_p, c_longlong, c_void_p,
                           c_longlong, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p],
    "nl_cast_bf16": [c_void_p, c_void_p, c_longlong, c_void_p],
    "nl_rows_mark": [c_void_p, c_longlong, c_void_p, c_int, c_void_p],
    "nl_rows_compact": [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p],
    "nl_rows_gather": [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p],
    "nl_rows_scatter": [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p],
    "nl_adamw_rows": [c_void_p] * 7 + [c_int, c_int, c_void_p, c_float, c_float, c_float, c_float, c_int,
                                       c_void_p],
    "nl_lce_workspace_bytes": [c_int, c_int, c_int],
    "nl_lce_fwd": [c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_size_t,
                   c_int, c_int, c_int, c_void_p],
    "nl_lce_bwd_ex": [c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_int, c_int,
                      c_void_p, c_int, c_int, c_void_p, ctypes.c_size_t, c_int, c_int, c_int, c_int, c_void_p],
    "nl_lce_bwd": [c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p,
                   c_int, c_int, c_void_p, ctypes.c_size_t, c_int, c_int, c_int, c_int, c_void_p],
}
_RESTYPE = {"nl_version": ctypes.c_char_p, "nl_launch_count": c_longlong,
            "nl_flash_attention_bwd_noalloc_max_rows": c_longlong, "nl_flash_attention_workspace_bytes": c_size_t, "nl_lce_workspace_bytes": ctypes.c_size_t,
            "nl_decode_workspace_bytes": ctypes.c_size_t}


class NlError(RuntimeError):
    """A kernel entry point returned a non-zero nl_status."""


class _Lib:
    def __init__(self) -> None:
        self._dll = None

    def _load(self):
        if self._dll is None:
            if not LIB_PATH.exists():
                raise ImportError(f"{LIB_PATH} is missing: build it with `python -m nlearn_b200.build` "
                                  "(there is no CPU fallback for the hot path)")
            dll = ctypes.CDLL(str(LIB_PATH))
            for name, args in SIGNATURES.items():
                fn = getattr(dll, name)
                fn.argtypes = args
                fn.restype = _RESTYPE.get(name, c_int)
            self._dll = dll
        return self._dll

    def __getattr__(self, name):
        if name.startswith("nl_"):
            return getattr(self._load(), name)
        raise AttributeError(name)


lib = _Lib()


def check(status: int, what: str) -> None:
    if status != 0:
        raise NlError(f"{what} returned {STATUS.get(status, status)}")


def stream_handle():
    import torch
    return c_void_p(torch.cuda.current_stream().cuda_stream)


def ptr(t) -> c_void_p:
    return c_void_p(0 if t is None else t.data_ptr())


def device_error() -> int:
    """Read and clear the kernels' device error word: 1 = a bounded wait gave
    up, 2 = misaligned shared memory, 3 = a decode position outside the cache
    or the output row (the cache and the output row are not written; the
    attention output keeps its previous contents, the sampled token is still
    written)."""
    return lib.nl_get_device_error(stream_handle())


__all__ = ["lib", "check", "ptr", "stream_handle", "device_error", "NlError", "LIB_PATH", "SIGNATURES",
           "F32", "BF16", "EPI_STORE", "EPI_ACCUM", "EPI_BIAS", "EPI_BIAS_GELU", "EPI_RESID", "EPI_DGELU",
           "c_longlong"]
