"""ctypes binding of the sm_100a C-ABI library (``include/loraforge_b200.h``).

The library is loaded lazily on first use.  There is no fallback: if the library
is missing every operator raises, so a CUDA path can never silently turn into a
CPU or library computation.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "_lib" / "liblfb200.so"

LF_F32, LF_F16, LF_BF16 = 0, 1, 2
LF_E_INVALID, LF_E_CUDA, LF_E_UNSUPPORTED = -1, -2, -3

_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float


class SliceDesc(ctypes.Structure):
    """Mirror of ``lf_slice_desc``."""

    _fields_ = [
        ("ptr", ctypes.c_void_p),
        ("slot_stride", ctypes.c_int64),
        ("row_stride", ctypes.c_int64),
        ("rows", ctypes.c_int64),
    ]


# name -> argument types (all entry points return int status).
SIGNATURES = {
    "lf_group_tokens": [_p, _i64, _i32, _i32, _p, _p, _p, _p, _p],
    "lf_split_runs": [_p, _p, _p, _p, _i64, _i32, _p, _p, _p, _p],
    "lf_group_token_runs": [_p, _i64, _i32, _i32, _p, _p, _p, _p, _p],
    "lf_row_shrink": [_p, _i64, _p, _p, _p, _p, _i64, _i64, _i32, _i32, _i32, _i32, _p],
    "lf_row_expand": [
        _p, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p,
        _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _p,
    ],
    "lf_bgmv_shrink": [_i32, _p, _i64, _p, _p, _p, _p, _i32, _i64, _i64, _i32, _i32, _i32, _p],
    "lf_bgmv_expand": [
        _i32, _p, _p, _p, _p, _i32, _p, _i32, _p, _i32, _p, _i64, _i64, _i64, _i32, _i32,
        _i32, _i32, _p,
    ],
    "lf_vllm_shrink": [_i32, _p, _i64, _p, _i32, _i32, _p, _p, _i64, _i64, _i32, _f32, _p],
    "lf_vllm_expand": [_i32, _p, _p, _i32, _i32, _p, _i64, _p, _i64, _i32, _i64, _i32, _p],
    "lf_fused_shrink_expand": [
        _p, _i64, _p, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _i64,
        _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _p,
    ],
    "lf_sgmv_prefill": [
        _p, _i64, _p, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _i64,
        _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _p,
    ],
    "lf_sgmv_shrink": [
        _p, _i64, _p, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _i64,
        _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _p,
    ],
    "lf_sgmv_expand": [
        _p, _i64, _p, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _i64,
        _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _p,
    ],
    "lf_fused_z_rows": [_i64, _i64, _i32, _i32, _p, _p],
    "lf_fused_shrink_expand_noalloc": [
        _p, _i64, _p, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p,
        _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _p,
    ],
    "lf_device_wait_timeouts": [_p, _i32],
    "lf_segment_routes": [_p, _p, _p, _p, _i32, _i64, _i64, _p, _p],
    "lf_peer_alloc": [_i64, _p, _p],
    "lf_peer_open": [_p, _p],
    "lf_peer_close": [_p],
    "lf_peer_free": [_p],
    "lf_peer_status": [_p, _p, _i32],
    "lf_peer_sum": [_p, _i32, _i32, _p, _i64, _i64, _i64, _p],
    "lf_fused_workspace_reset": [_p, _i64, _i64, _i64, _i32, _i32, _p],
    "lf_lora_base_gemm": [
        _p, _i64, _p, _i64, _p, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _i64,
        _i64, _i64, _i32, _i32, _i32, _i32, _i32, _p,
    ],
    "lf_fused_noalloc_reset": [_p],
}

_lock = threading.Lock()
_lib = None


def exported_symbols() -> tuple[str, ...]:
    """Every symbol the header declares (checked by the CPU test suite)."""
    return ("lf_version", "lf_last_error_string", "lf_fused_workspace_floats",
            "lf_sgmv_prefill_workspace_floats", "lf_lora_base_gemm_workspace_floats",
            "lf_peer_buffer_bytes", "lf_peer_handle_bytes", *SIGNATURES)


def library() -> ctypes.CDLL:
    """Load and type the C-ABI library once per process."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIBRARY.exists():
                raise RuntimeError(
                    f"loraforge_b200 native library missing at {LIBRARY}; "
                    "build it with `python -m loraforge_b200._build`"
                )
            lib = ctypes.CDLL(str(LIBRARY))
            lib.lf_version.restype = ctypes.c_int
            lib.lf_version.argtypes = []
            lib.lf_last_error_string.restype = ctypes.c_char_p
            lib.lf_last_error_string.argtypes = []
            for name, args in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = ctypes.c_int
                fn.argtypes = args
            for sizer in ("lf_fused_workspace_floats", "lf_sgmv_prefill_workspace_floats",
                          "lf_lora_base_gemm_workspace_floats"):
                getattr(lib, sizer).restype = ctypes.c_int64
                getattr(lib, sizer).argtypes = [_i64, _i64, _i32, _i32]
            lib.lf_peer_buffer_bytes.restype = ctypes.c_int64
            lib.lf_peer_buffer_bytes.argtypes = [_i64]
            lib.lf_peer_handle_bytes.restype = ctypes.c_int
            lib.lf_peer_handle_bytes.argtypes = []
            _lib = lib
    return _lib


def call(name: str, *args) -> None:
    """Invoke an entry point; non-zero status raises RuntimeError with its message."""
    lib = library()
    status = getattr(lib, name)(*args)
    if status != 0:
        message = lib.lf_last_error_string().decode(errors="replace")
        raise RuntimeError(message or f"{name} failed with status {status}")


def fused_workspace_floats(num_tokens: int, width: int, num_slices: int, capacity: int) -> int:
    """FP32 workspace size of lf_fused_shrink_expand for these sizes."""
    n = library().lf_fused_workspace_floats(num_tokens, width, num_slices, capacity)
    if n < 0:
        raise ValueError("invalid sizes for the fused workspace")
    return n


def prefill_workspace_floats(num_tokens: int, width: int, num_slices: int, capacity: int) -> int:
    """FP32 workspace size of lf_sgmv_prefill for these sizes."""
    n = library().lf_sgmv_prefill_workspace_floats(num_tokens, width, num_slices, capacity)
    if n < 0:
        raise ValueError("invalid sizes for the prefill workspace")
    return n


def lora_base_gemm_workspace_floats(num_tokens: int, width: int, num_slices: int, capacity: int) -> int:
    """FP32 workspace size of lf_lora_base_gemm for these sizes."""
    n = library().lf_lora_base_gemm_workspace_floats(num_tokens, width, num_slices, capacity)
    if n < 0:
        raise ValueError("invalid sizes for the base GEMM workspace")
    return n


def fused_z_rows(num_tokens: int, width: int, num_slices: int, capacity: int) -> tuple[int, int]:
    """(offset, floats per row) of the z rows lf_sgmv_shrink leaves in the workspace."""
    offset, row = ctypes.c_int64(0), ctypes.c_int64(0)
    call("lf_fused_z_rows", num_tokens, width, num_slices, capacity, ctypes.byref(offset),
         ctypes.byref(row))
    return offset.value, row.value


def device_wait_timeouts(reset: bool = False) -> int:
    """Expired bounded device waits since the last reset (synchronous)."""
    count = ctypes.c_int32(0)
    call("lf_device_wait_timeouts", ctypes.byref(count), 1 if reset else 0)
    return count.value


def stream_of(device) -> int:
    """Raw handle of PyTorch's current stream on ``device``."""
    import torch

    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dtype) -> int:
    import torch

    codes = {torch.float32: LF_F32, torch.float16: LF_F16, torch.bfloat16: LF_BF16}
    return codes[dtype]
