"""ctypes binding of libvdn_b200.so (the C ABI declared in include/vdn_b200.h).

The library is loaded once, lazily, from this package directory.  There is no
fallback: if the shared library is missing or does not export a declared
symbol, every op raises RuntimeError.  Status codes map to the reference's
exception split (ValueError for bad metadata and non-finite data, TypeError for
bad dtypes, RuntimeError for unsupported hardware and failed launches).
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libvdn_b200.so"

VDN_OK, VDN_ERR_VALUE, VDN_ERR_TYPE, VDN_ERR_RUNTIME, VDN_ERR_NONFINITE, VDN_ERR_TIMEOUT = range(6)
DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
ACT_GELU_TANH, ACT_GELU_ERF, ACT_SWIGLU = 1, 2, 3

_i64, _i32, _f32, _sz = C.c_int64, C.c_int, C.c_float, C.c_size_t
_p = C.c_void_p

# name -> (restype, argtypes); the complete exported surface of include/vdn_b200.h.
SIGNATURES = {
    "vdn_last_error": (C.c_char_p, []),
    "vdn_abi_version": (_i32, []),
    "vdn_device_supported": (_i32, [_i32, C.POINTER(_i32)]),
    "vdn_mxfp8_padded_shape": (_i32, [_i64, _i64, C.POINTER(_i64), C.POINTER(_i64)]),
    "vdn_mxfp8_quantize": (_i32, [_p, _i64, _i64, _i64, _p, _p, _p, _p]),
    "vdn_mxfp8_act_quantize": (_i32, [_i32, _p, _i64, _i64, _i64, _p, _p, _p, _p]),
    "vdn_mxfp8_prenorm_quantize": (_i32, [_p, _i64, _i64, _i64, _p, _i32, _f32, _p, _i64, _p,
                                          _i64, _p, _p, _p, _p, _p, _p]),
    "vdn_finite_parts": (_i32, [_p, _i64, _i32, _i32, _p, _p]),
    "vdn_mxfp8_quantize_host": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _i32]),
    "vdn_mxfp8_gemm": (_i32, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _i64, _p, _p]),
    "vdn_mxfp8_gemm_fused": (_i32, [_p, _p, _p, _p, _i64, _p, _p, _p, _p, _i64, _p, _i64, _i64, _i64,
                                    _i64, _p, _i64, _p, _i64, _p, _p, _p]),
    "vdn_gate_gemm": (_i32, [_p, _i64, _p, _i64, _p, _i64, _i64, _i64, _i64, _p, _i64, _p, _p]),
    "vdn_mxfp8_quantize_grouped": (_i32, [_p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p]),
    "vdn_mxfp8_gemm_scatter": (_i32, [_p, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _p, _i64, _i64,
                                      _p, _p]),
    "vdn_mxfp8_gemm_act_quantize": (_i32, [_p, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _i32, _p,
                                           _p, _p, _p]),
    "vdn_peer_alloc": (_i32, [C.c_size_t, C.POINTER(_p)]),
    "vdn_peer_free": (_i32, [_p]),
    "vdn_ipc_handle": (_i32, [_p, _p]),
    "vdn_ipc_open": (_i32, [_p, C.POINTER(_p)]),
    "vdn_ipc_close": (_i32, [_p]),
    "vdn_copy_async": (_i32, [_p, _p, C.c_size_t, _p]),
    "vdn_peer_broadcast": (_i32, [_p, C.c_size_t, _i32, _p, _p]),
    "vdn_peer_fence": (_i32, [_i32, _p, _p, _i32, _p, _p, _p]),
    "vdn_mxfp8_quantize_scatter": (_i32, [_p, _i64, _i32, _i32, _i64, _i64, _i32, _i64, _i32, _p, _p, _p,
                                          _p, _p]),
    "vdn_window_merge": (_i32, [_i32, _p, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _p, _i64, _i64, _p,
                                _i64, _i64, _p, _p, _p]),
    "vdn_sepconv": (_i32, [_p, _i64, _i32, _i32, _i32, _i32, _p, _p, _p, _p, _i64, _p]),
    "vdn_frame_alpha": (_i32, [_p, _i32, _i32, _p, _i32, _p, _p, _p, _i32, _i32, _p, _p, _p]),
    "vdn_frame_sums": (_i32, [_p, _i64, _i64, _i64, _p, _i32, _f32, _p, _p]),
    "vdn_delta_factors": (_i32, [_p, _p, _p, _i64, _i32, _p, _p, _p]),
    "vdn_vda_statistics": (_i32, [_p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p, _i64, _i64, _i64,
                                  _i32, _i32, _i32, _i32, _i32, _p, _p, _p]),
    "vdn_vda_scan": (_i32, [_p, _p, _p, _i32, _i32, _i32, _p, _p, _p]),
    "vdn_vda_gather": (_i32, [_p, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _p, _i32, _p]),
    "vdn_vda_readout": (_i32, [_p, _i64, _i64, _i64, _p, _p, _i64, _i64, _i64, _p, _f32, _i32, _i32,
                               _i32, _i32, _p, _p]),
    "vdn_vda_factor_inverse": (_i32, [_p, _i64, _p, _p]),
    "vdn_vda_scan_tc": (_i32, [_p, _p, _p, _p, _i32, _i32, _p, _p, _p, _p]),
    "vdn_vda_scan_tc_bf16": (_i32, [_p, _p, _p, _p, _i32, _i32, _p, _p, _p, _p]),
    "vdn_vda_workspace_size": (_sz, [_i32, _i32, _i32, _i32]),
    "vdn_vda_forward": (_i32, [_p, _p, _p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _p, _f32,
                               _p, _p, _i32, _i32, _i32, _i32, _i32, _p, _p, _sz, _p]),
    "vdn_vda_forward_noalloc": (_i32, [_p, _p, _p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _p,
                                       _f32, _p, _p, _i32, _i32, _i32, _i32, _i32, _p, _p]),
}

_LOCK = threading.Lock()
_LIB = None


def load() -> C.CDLL:
    """Load the library once; raise RuntimeError (no fallback) when unavailable."""
    global _LIB
    with _LOCK:
        if _LIB is None:
            if not LIB_PATH.is_file():
                raise RuntimeError(
                    f"vdn_b200 native library missing ({LIB_PATH.name}); build it with "
                    "`python -m vdn_b200.csrc.build` -- there is no fallback path")
            lib = C.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)  # AttributeError -> missing export
                fn.restype, fn.argtypes = res, args
            _LIB = lib
    return _LIB


def call(name: str, *args) -> int:
    rc = getattr(load(), name)(*args)
    if rc != VDN_OK:
        raise_status(rc)
    return rc


def raise_status(rc: int):
    msg = load().vdn_last_error().decode(errors="replace")
    if rc in (VDN_ERR_VALUE, VDN_ERR_NONFINITE):
        raise ValueError(msg)
    if rc == VDN_ERR_TYPE:
        raise TypeError(msg)
    raise RuntimeError(msg)


def ptr(t: torch.Tensor | None):
    return None if t is None else C.c_void_p(t.data_ptr())


def stream_of(device: torch.device):
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


_SUPPORTED: dict[int, bool] = {}


def require_device(t: torch.Tensor, what: str = "tensor") -> None:
    """Raise RuntimeError unless t lives on an sm_100 CUDA device (no fallback)."""
    if t.device.type != "cuda":
        raise ValueError(f"{what} must be a CUDA tensor")
    idx = t.device.index if t.device.index is not None else torch.cuda.current_device()
    ok = _SUPPORTED.get(idx)
    if ok is None:
        flag = C.c_int(0)
        call("vdn_device_supported", idx, C.byref(flag))
        ok = _SUPPORTED[idx] = bool(flag.value)
    if not ok:
        raise RuntimeError("vdn_b200 kernels require an sm_100 (B200) GPU; no fallback")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return {torch.float32: DTYPE_F32, torch.bfloat16: DTYPE_BF16, torch.float16: DTYPE_F16}[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}") from None
