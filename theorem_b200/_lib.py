"""ctypes binding of the C ABI in include/theorem_b200.h.

The shared library ``theorem_b200/libtheorem_b200.so`` is built in-tree by
``theorem_b200.build``. There is no CPU fallback: if the library is missing,
or a call returns a non-zero status, an exception is raised.

Status mapping mirrors the reference's error behaviour: its launchers
``assert`` on shape / dtype / contiguity (e.g.
kernels/causal_conv1d/kernel.py:184-192), so THM_ERR_INVALID /
THM_ERR_UNSUPPORTED / THM_ERR_ALIGNMENT raise ``AssertionError``; launch,
timeout and driver failures raise ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libtheorem_b200.so"

THM_OK, THM_ERR_INVALID, THM_ERR_UNSUPPORTED, THM_ERR_ALIGNMENT = 0, 1, 2, 3
THM_ERR_CUDA, THM_ERR_TIMEOUT, THM_ERR_NO_DRIVER = 4, 5, 6
THM_F32, THM_BF16 = 0, 1
THM_LAYOUT_BDS, THM_LAYOUT_BSD = 0, 1
THM_ACT_NONE, THM_ACT_SILU = 0, 1

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float

_SIGNATURES = {
    "thm_causal_conv1d_fwd": [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P],
    "thm_causal_conv1d_pair_fwd": [_P] * 8 + [_I] * 7 + [_P],
    "thm_recompute_w_u_fwd": [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P],
    "thm_chunk_fwd_h_fwd": [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P],
    "thm_chunk_fwd_o_fwd": [_P, _P, _P, _P, _P, _P, _F, _I, _I, _I, _I, _I, _I, _I, _P],
    "thm_recompute_w_u_conv_fwd": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P],
    "thm_build_A_fwd": [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P],
    "thm_chunk_local_cumsum_fwd": [_P, _P, _I, _I, _I, _F, _P],
    "thm_gated_delta_fwd_ho": [_P, _P, _P, _P, _P, _P, _P, _P, _F, _I, _I, _I, _I, _I, _I, _P],
    "thm_sp_prefix_fold": [_P, _P, _P, _P, _I, _I, _I, _I, _P],
    "thm_selftest_wait_timeout": [ctypes.c_longlong, _P, _P],
    "thm_status_string": [_I],
    "thm_get_device_status": [ctypes.POINTER(_I), _I],
    "thm_version": [],
}

_lib = None
_lock = threading.Lock()


def load():
    """Load (once) and return the ctypes handle of the CUDA library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is not built; run `python -m theorem_b200.build` "
                    "(nvcc for sm_100a). There is no CPU fallback.")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, args in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = ctypes.c_char_p if name == "thm_status_string" else _I
            _lib = lib
    return _lib


def exported_symbols():
    return tuple(_SIGNATURES)


def status_string(code: int) -> str:
    return load().thm_status_string(int(code)).decode()


def check(code: int, what: str) -> None:
    """Raise the exception class the reference would for a non-zero status."""
    if code == THM_OK:
        return
    msg = f"{what}: {status_string(code)}"
    if code in (THM_ERR_INVALID, THM_ERR_UNSUPPORTED, THM_ERR_ALIGNMENT):
        raise AssertionError(msg)
    raise RuntimeError(msg)


def device_status(reset: bool = False) -> int:
    """In-kernel error word of the current device (synchronizes)."""
    out = _I(0)
    check(load().thm_get_device_status(ctypes.byref(out), int(bool(reset))), "thm_get_device_status")
    return out.value


def ptr(t) -> int | None:
    """Device address of a torch tensor (None for None)."""
    return None if t is None else t.data_ptr()


def stream_of(t) -> int:
    """Raw cudaStream_t of torch's current stream on the tensor's device."""
    import torch
    return torch.cuda.current_stream(t.device).cuda_stream


def dtype_code(t) -> int:
    import torch
    if t.dtype == torch.float32:
        return THM_F32
    if t.dtype == torch.bfloat16:
        return THM_BF16
    raise AssertionError(f"unsupported dtype {t.dtype} (float32 or bfloat16)")


if os.environ.get("THEOREM_B200_EAGER_LOAD") == "1":  # pragma: no cover
    load()
