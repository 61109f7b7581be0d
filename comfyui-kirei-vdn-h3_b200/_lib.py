"""ctypes binding of the C-ABI library ``libvdn_b200.so`` (declared in include/vdn_b200.h).

The library is loaded from this package directory only.  There is no fallback: if the
library is missing, or a call is made without a CUDA device, the call raises.  Every
entry point is stream-ordered on the caller's current CUDA stream and returns an int
status that :func:`check` maps onto the exception types the reference raises
(``ValueError`` for bad geometry/arguments, ``RuntimeError`` for launch failures).
"""

from __future__ import annotations

import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libvdn_b200.so")

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_longlong
_F = ctypes.c_float

# name -> argument types (all return int status)
SIGNATURES: dict[str, list] = {
    "vdn_gemm": [_I, _P, _L, _P, _L, _L, _P, _L, _P, _L, _I, _I, _I, _I, _F, _P, _P, _P, _P, _P, _I, _P, _L, _P, _P],
    "vdn_gemm_grouped_k": [_I, _P, _L, _L, _I, _I, _P, _L, _P, _L, _I, _I, _I, _F, _P, _P, _P, _P, _P, _I, _P, _L,
                           _P, _P],
    "vdn_qkv_gemm": [_I, _P, _L, _P, _L, _I, _I, _I, _I, _I, _P, _F, _F, _P, _P, _P, _P, _P, _L, _P, _L, _P, _L,
                     _P, _I, _I, _I, _P, _P],
    "vdn_adaln_rmsnorm": [_P, _L, _I, _I, _P, _F, _P, _P, _L, _P, _P, _L, _P, _L, _P, _P],
    "vdn_gemm_block": [_I, _P, _L, _P, _L, _L, _L, _I, _P, _L, _P, _L, _I, _I, _I, _F, _P, _P, _P, _P, _P, _I, _P,
                       _L, _P, _P, _L, _P, _P, _P],
    "vdn_quant_int8_rows_amax": [_P, _L, _I, _I, _P, _P, _L, _P, _P],
    "vdn_window_attention": [_P, _L, _P, _L, _P, _L, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _P, _P, _I, _P,
                             _P, _P, _P, _L, _P, _L, _I, _P, _P, _P, _P],
    "vdn_spatial_conv": [_P, _L, _P, _I, _I, _I, _I, _I, _I, _P, _L, _P],
    "vdn_temporal_act": [_P, _L, _P, _I, _I, _I, _I, _I, _I, _P, _P],
    "vdn_conv_features": [_P, _L, _P, _I, _I, _P, _I, _I, _I, _I, _I, _I, _I, _P, _P],
    "vdn_alpha_gate": [_P, _L, _I, _I, _I, _P, _P, _P, _I, _I, _P, _P],
    "vdn_frame_stats": [_P, _P, _I, _I, _I, _I, _P, _L, _I, _P, _P, _P],
    "vdn_frame_stats_tc": [_P, _P, _I, _I, _I, _P, _L, _I, _P, _P, _P, _P],
    "vdn_readout_tc": [_P, _I, _I, _I, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _L, _L, _I, _I, _P, _P],
    "vdn_delta_factor": [_P, _P, _I, _I, _I, _P, _P, _I, _F, _P, _P, _P],
    "vdn_rope_split_half": [_P, _L, _I, _I, _I, _I, _P, _L, _P],
    "vdn_sana_factor": [_P, _P, _I, _I, _I, _F, _P, _P, _I, _F, _F, _P, _P],
    "vdn_bidir_scan": [_P, _P, _P, _P, _I, _I, _I, _F, _P, _P, _P],
    "vdn_bidir_scan_tc": [_P, _P, _P, _P, _I, _I, _I, _F, _P, _P, _P, _P],
    "vdn_readout": [_P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _I, _P, _P, _L, _P, _L, _L, _I, _I, _P],
    "vdn_cast_rows": [_P, _L, _I, _I, _I, _P, _L, _P],
    "vdn_quant_int8_rows": [_I, _P, _L, _I, _I, _P, _L, _P, _P],
    "vdn_quant_int8_rows_convrot": [_P, _L, _I, _I, _I, _P, _L, _P, _P],
    "vdn_fp8_amax": [_I, _P, _L, _I, _I, _P, _P],
    "vdn_fp8_cast": [_I, _P, _L, _I, _I, _P, _P, _L, _P, _P],
    "vdn_quant_fp8_tensor": [_I, _P, _L, _I, _I, _P, _L, _P, _P, _P],
    "vdn_fp8_linear_noalloc": [_P, _L, _I, _I, _P, _L, _I, _P, _P, _L, _P, _P],
}

_STATUS = {
    -1: (ValueError, "invalid argument"),
    -2: (ValueError, "geometry not supported by the sm_100a kernels"),
    -3: (RuntimeError, "TMA tensor-map encoding failed"),
    -4: (RuntimeError, "CUDA launch failed"),
    -5: (ValueError, "pointer or row pitch is not 16-byte aligned"),
    -6: (ValueError, "problem is larger than the library's fixed device scratch area"),
}

DEVICE_ERRORS = {
    1: "TMA producer timed out waiting for a free stage",
    2: "MMA issuer timed out waiting for operands",
    3: "epilogue/softmax warps timed out waiting for the accumulator",
    4: "device wait timed out",
}

_lib = None


def library() -> ctypes.CDLL:
    """Load (once) and return the C-ABI library; raise if it is not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with build.py (nvcc, sm_100a). "
                "There is no CPU or library fallback for the VDN-H3 B200 path."
            )
        lib = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        lib.vdn_launch_count.argtypes = []
        lib.vdn_launch_count.restype = ctypes.c_longlong
        _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    if status == 0:
        return
    exc, msg = _STATUS.get(status, (RuntimeError, f"status {status}"))
    if status == -4:
        err = torch.cuda.current_device() if torch.cuda.is_available() else None
        msg = f"{msg} on cuda:{err}"
    raise exc(f"{what}: {msg}")


def call(name: str, *args) -> None:
    check(getattr(library(), name)(*args), name)


def launch_count() -> int:
    """Kernels launched by the library so far (host-side count; diff it around a region)."""
    return int(library().vdn_launch_count())


def ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


def stream_handle(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("the VDN-H3 B200 path takes CUDA tensors only (no CPU fallback)")


class DeviceStatus:
    """Device-resident status words checked once per forward (deferred, like the
    reference's deferred Cholesky validation, branch.py:27-59).

    word 0: first kernel wait-timeout code (0 = none).
    word 1: work-queue counter of the persistent attention kernel (zeroed per launch).
    """

    def __init__(self, device):
        self.words = torch.zeros(4, dtype=torch.int32, device=device)

    @property
    def err_ptr(self) -> int:
        return self.words.data_ptr()

    @property
    def counter_ptr(self) -> int:
        return self.words.data_ptr() + 4

    def reset(self):
        self.words.zero_()

    def raise_if_failed(self):
        code = int(self.words[0].item())
        if code:
            self.words.zero_()
            raise RuntimeError(f"VDN-H3 kernel aborted: {DEVICE_ERRORS.get(code, code)}")
