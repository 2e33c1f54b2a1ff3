"""ctypes binding of libgptq_b200.so (the C ABI declared in include/gptq_b200.h).

The library is the only compute path: if it is missing, or no CUDA device is
present, calls raise instead of falling back to anything else.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libgptq_b200.so")

GQ_OK, GQ_ERR_ARG, GQ_ERR_NOT_PD, GQ_ERR_CUDA, GQ_ERR_TIMEOUT = 0, 1, 2, 3, 4
GQ_F32, GQ_BF16, GQ_F16 = 0, 1, 2
GQ_AFFINE, GQ_MXFP4, GQ_MXFP8 = 0, 1, 2
GQ_CLIP_MINMAX, GQ_CLIP_MSE = 0, 1
GQ_MX_GROUPWISE, GQ_MX_SAFE_SCALE_SEARCH = 0, 1

DTYPE_CODE = {torch.float32: GQ_F32, torch.bfloat16: GQ_BF16, torch.float16: GQ_F16}
MODE_CODE = {"affine": GQ_AFFINE, "mxfp4": GQ_MXFP4, "mxfp8": GQ_MXFP8}
CLIP_CODE = {"minmax": GQ_CLIP_MINMAX, "mse": GQ_CLIP_MSE}

P, I64, I32, F32, SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_size_t

# name -> (restype, argtypes); must match include/gptq_b200.h
SIGNATURES = {
    "gq_abi_version": (I32, []),
    "gq_status_string": (ctypes.c_char_p, [I32]),
    "gq_last_error": (ctypes.c_char_p, []),
    "gq_selftest_wait_timeout": (I32, [ctypes.c_ulonglong, P, P, P]),
    "gq_hessian_bf16": (I32, [P, I64, I64, I64, P, I64, F32, F32, P, P]),
    "gq_hessian_tile_count": (I64, [I64]),
    "gq_hessian_concurrent_tiles": (I64, [I64]),
    "gq_hessian_bf16_range": (I32, [P, I64, I64, I64, P, I64, F32, F32, I64, I64, P, P]),
    "gq_hessian_grouped_workspace_size": (SZ, [P, I64, I64]),
    "gq_hessian_grouped_bf16": (I32, [P, I64, I64, I64, P, P, P, I64, P, F32, F32, P, SZ, P, P]),
    "gq_hessian_spans_workspace_size": (SZ, [P, I64, I64]),
    "gq_hessian_spans_bf16": (I32, [P, I64, I64, I64, P, I64, P, F32, F32, P, SZ, P, P]),
    "gq_hessian_merge_pieces": (I32, [P, I64, I64, P, P, P, P]),
    "gq_dead_columns": (I32, [P, I64, I64, P, P]),
    "gq_mx_prepare_hinv": (I32, [P, I64, I64, F32, P, P, P, P]),
    "gq_prepare_hinv_workspace_size": (SZ, [I64, I64]),
    "gq_prepare_hinv": (I32, [P, I64, I64, F32, P, P, P, P, SZ, P, P]),
    "gq_gptq_mxfp_workspace_size": (SZ, [I64, I64, I64]),
    "gq_gptq_mxfp": (I32, [P, I32, P, P, P, P, I64, I64, I64, I32, I32, P, P, P, P, I32, P, P, SZ, P]),
    "gq_gptq_mxfp_noalloc": (I32, [P, I32, P, P, P, P, I64, I64, I64, I32, I32, P, P, P, P, I32, P, P]),
    "gq_gptq_affine_workspace_size": (SZ, [I64, I64, I64, I32, I32]),
    "gq_gptq_affine": (I32, [P, P, I32, P, I64, I64, I64, I32, I32, I32, I32, I32, P, P, P, P, P, SZ, P, P]),
    "gq_gemm_f32": (I32, [P, P, P, I64, I64, I64, I64, I64, I64, I32, I32, I64, I64, I64, I64, I64, I64, I64, I64,
                          F32, F32, P, I32, P, P]),
    "gq_prepare_weights": (I32, [P, I32, P, I64, I64, I64, P, P]),
    "gq_rtn_affine": (I32, [P, I32, I64, I64, I32, I32, I32, I32, P, P, P, P, I32, P]),
    "gq_rtn_mxfp": (I32, [P, I32, I64, I64, I32, P, P, P, P, I32, P]),
    "gq_dequantize": (I32, [P, P, P, I32, I64, I64, I32, I32, P, P]),
    "gq_pack_q": (I32, [P, I64, I64, I32, P, P]),
    "gq_unpack_q": (I32, [P, I64, I64, I32, I64, P, P]),
    "gq_pack_nibbles": (I32, [P, I64, I64, P, P]),
    "gq_unpack_nibbles": (I32, [P, I64, I64, P, P]),
}

_lib = None
_lock = threading.Lock()


class GQError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def lib() -> ctypes.CDLL:
    """Load the library once (raises if it has not been built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is missing: build it with `python mlx-gptq-mxfp_b200/build.py`")
                handle = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().gq_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str) -> None:
    """Map a C status code to the reference's exception types."""
    if status == GQ_OK:
        return
    msg = f"{what}: {last_error() or lib().gq_status_string(status).decode()}"
    if status == GQ_ERR_ARG:
        raise ValueError(msg)
    raise GQError(status, msg)


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    """The library computes on CUDA devices only; there is no CPU path."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("mlx_gptq_b200 computes on CUDA devices only; got a tensor on "
                               f"{t.device} (move it to a cuda device first)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    return dev


_status_words: dict[int, torch.Tensor] = {}


def status_word(device: torch.device | int | None = None) -> torch.Tensor:
    """The device's int32 status word (zero at creation). Kernels with bounded waits
    (the Hessians) write GQ_ERR_TIMEOUT into it when a wait gives up, instead of
    hanging; the product path passes it to every such launch and reads it with
    raise_on_device_timeout before results are used."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    w = _status_words.get(idx)
    if w is None:
        with _lock:
            w = _status_words.get(idx)
            if w is None:
                w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
                _status_words[idx] = w
    return w


def raise_on_device_timeout(device: torch.device | int | None = None) -> None:
    """Read the device's status word (a synchronizing copy on the current stream) and
    raise GQError(GQ_ERR_TIMEOUT) if a bounded device wait gave up since the last
    check; a reported failure is cleared from the word."""
    w = status_word(device)
    v = int(w.item())
    if v != GQ_OK:
        w.zero_()
        raise GQError(v, f"a device-side wait gave up (status {v}: "
                         f"{lib().gq_status_string(v).decode()}); the results of the launch are incomplete")


def aligned(t: torch.Tensor) -> torch.Tensor:
    """Contiguous and 16-byte aligned (copies otherwise)."""
    if not t.is_contiguous() or t.data_ptr() % 16:
        t = t.contiguous()
        if t.data_ptr() % 16:
            t = t.clone()
    return t
