"""ctypes binding of librecavsr_b200.so (the C ABI in include/recavsr_b200.h).

PyTorch only supplies device memory and the current CUDA stream; every
computation is a call into the library. There is no fallback: if the library
is missing or the device is not a B200-class (sm_100) GPU the calls raise.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librecavsr_b200.so")

RC_OK, RC_ERR_ARG, RC_ERR_CUDA, RC_ERR_TIMEOUT, RC_ERR_UNSUPPORTED = range(5)
EPI_BIAS, EPI_GATED_RESIDUAL, EPI_RESIDUAL, EPI_GELU_NVFP4, EPI_SWIGLU = range(5)

_P, _I, _LL, _F = C.c_void_p, C.c_int, C.c_longlong, C.c_float
_SIGNATURES = {
    "rc_abi_version": [],
    "rc_get_last_error": [C.c_char_p, C.c_size_t],
    "rc_read_device_error": [C.POINTER(C.c_uint)],
    "rc_nvfp4_quantize": [_P, _I, _I, _LL, _F, _P, _P, _P],
    "rc_fp8_quantize": [_P, _I, _I, _LL, _P, _P, _P, _P],
    "rc_nvfp4_gemm": [_P, _P, _P, _P, _P, _I, _I, _I, _F, _I, _P, _LL, _P, _P, _P, _F, _P],
    "rc_gemm_split_workspace": [],
    "rc_nvfp4_gemm_ws": [_P, _P, _P, _P, _P, _I, _I, _I, _F, _I, _P, _LL, _P, _P, _P, _F, _P, _LL, _P],
    "rc_fp8_gemm": [_P, _P, _P, _P, _P, _I, _I, _I, _F, _I, _P, _LL, _P, _P],
    "rc_bf16_gemm": [_P, _P, _P, _I, _I, _I, _I, _P, _LL, _P, _P],
    "rc_bf16_gemm_ws": [_P, _P, _P, _I, _I, _I, _I, _P, _LL, _P, _P, _LL, _P],
    "rc_ln_modulate_quant": [_P, _LL, _I, _I, _P, _P, _P, _P, _F, _P, _LL, _P, _P, _F, _P],
    "rc_layer_norm": [_P, _I, _LL, _I, _I, _P, _P, _F, _I, _P, _LL, _P],
    "rc_rmsnorm_rope": [_I, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _F, _P],
    "rc_temporal_rope": [_P, _LL, _P, _LL, _P, _P, _P, _I, _I, _I, _I, _I, _P],
    "rc_kv_commit": [_P, _P, _LL, _P, _P, _LL, _I, _I, _I, _P, _P, _P],
    "rc_paired_attention": [_P] * 11 + [_I] * 10 + [_P, _LL, _P, _LL, _P, _P, _P],
    "rc_paired_attention_workspace": [_I] * 7,
    "rc_cross_attention": [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _LL, _P, _P, _P],
    "rc_cross_attention_workspace": [],
    "rc_cross_attention_ws": [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _LL, _P, _P, _P, _LL, _P],
    "rc_paired_attention_static_scratch": [_P] * 11 + [_I] * 10 + [_P, _LL, _P, _P, _P],
    "rc_kv_commit_planned": [_P, _P, _LL, _LL, _P, _P, _LL, _I, _I, _I, _I, _P, _P],
    "rc_conv3d_im2col": [_P, _LL, _LL, _LL, _LL, _I, _I, _I, _I, _I, _I, _I, _I, _P, _LL, _P],
    "rc_channel_rmsnorm_silu": [_P, _LL, _I, _I, _P, _F, _P, _LL, _P],
    "rc_patchify": [_P, _I, _LL, _LL, _LL, _I, _I, _I, _I, _I, _I, _P, _LL, _P],
    "rc_enlarge_block": [_P, _LL, _LL, _I, _I, _I, _I, _I, _I, _I, _P, _P],
    "rc_strip_blend": [_I, _P, _P, _P, _P, _P, _P, _I, _I, _P, _LL, _P],
    "rc_local_gqa_attention": [_P, _P, _P, _P] + [_I] * 13 + [_P, _P, _P],
    "rc_fd_latent_in": [_P, _LL, _I, _P, _P, _P, _P],
    "rc_cf_adain_workspace": [_I, _LL],
    "rc_cf_adain": [_P, _I, _P, _I, _I, _LL, _P, _LL, _P, _P],
    "rc_cf_bicubic_u8": [_P, _I, _I, _I, _I, _I, _P, _P],
    "rc_cf_wavelet_level": [_P, _I, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P],
    "rc_fd_lr_unshuffle": [_P, _I, _P, _I, _I, _I, _P, _P],
    "rc_fd_lr_group": [_P, _LL, _I, _I, _P, _P, _P],
    "rc_fd_kv_norm": [_P, _LL, _I, _I, _I, _P, _P, _F, _P, _P, _LL, _LL, _P],
    "rc_fd_rope_gather": [_P, _LL] + [_I] * 9 + [_P, _P, _LL, _P, _I, _P, _P, _P, _P],
    "rc_fd_silu": [_P, _I, _I, _I, _P, _P],
    "rc_fd_pixel_shuffle": [_P, _LL, _I, _I, _I, _I, _I, _P, _P],
    "rc_unpatchify_residual": [_P, _LL, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P],
}
_RESTYPES = {"rc_paired_attention_workspace": C.c_longlong, "rc_gemm_split_workspace": C.c_longlong,
             "rc_cross_attention_workspace": C.c_longlong, "rc_cf_adain_workspace": C.c_longlong}

_lib = None
_lock = threading.Lock()


def library() -> C.CDLL:
    """Load the library once; raise loudly if it is absent."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is missing: build it with `python -m recavsr_b200.build` "
                        "(there is no CPU fallback)")
                lib = C.CDLL(LIB_PATH)
                for name, args in _SIGNATURES.items():
                    fn = getattr(lib, name, None)
                    if fn is None:
                        continue
                    fn.argtypes = args
                    fn.restype = _RESTYPES.get(name, C.c_int)
                _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    lib = library()
    return [n for n in _SIGNATURES if hasattr(lib, n)]


def last_error() -> str:
    buf = C.create_string_buffer(2048)
    library().rc_get_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int, name: str) -> None:
    if status == RC_OK:
        return
    msg = last_error() or name
    if status in (RC_ERR_ARG, RC_ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(f"{msg} (status {status})")


def call(name: str, *args) -> None:
    check(getattr(library(), name)(*args), name)


def read_device_error() -> int:
    """Read and clear the kernels' device error word (synchronizes)."""
    word = C.c_uint(0)
    check(library().rc_read_device_error(C.byref(word)), "rc_read_device_error")
    return int(word.value)


def stream(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def require_cuda(t: torch.Tensor, what: str) -> None:
    if t.device.type != "cuda":
        raise ValueError(f"{what}: the B200 kernels need CUDA tensors (got {t.device})")
