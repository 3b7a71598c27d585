"""ctypes binding of libivonar_b200.so (declared in include/ivonar_b200.h).

The library is the only compute path of this package: importing works without it, but every
entry point raises KernelError when the shared object is missing or cannot run on the device.
Replaces the reference's NVRTC/driver runtime (src/ivonar_inference/kernels/runtime.py).
"""

from __future__ import annotations

import ctypes
import glob
import os
from ctypes import POINTER, Structure, c_char_p, c_float, c_int32, c_int64, c_uint64, c_void_p
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
LIBRARY = PACKAGE / "libivonar_b200.so"

IVB_ABI_VERSION = 2
IVB_OK, IVB_EINVAL, IVB_ECUDA, IVB_ETIMEOUT, IVB_ECAPACITY, IVB_EUNSUPPORTED = range(6)
IVB_EPI_STORE, IVB_EPI_RESIDUAL, IVB_EPI_SILU_PAIR = range(3)
IVB_MAMBA, IVB_MLA = 0, 1
IVB_RUN_SAMPLE, IVB_RUN_SAMPLE_ONLY, IVB_RUN_HEAD_ALL = 1, 2, 4


class KernelError(RuntimeError):
    """The sm_100a kernels cannot run here or reported a failure (reference kernels/runtime.py:27)."""


class IvbTernary(Structure):
    _fields_ = [
        ("packed", c_void_p),
        ("scales", c_void_p),
        ("bias", c_void_p),
        ("rows", c_int32),
        ("in_features", c_int32),
        ("row_bytes", c_int32),
        ("scale_stride", c_int32),
    ]


IVB_CHECK_PACKED = 0
IVB_CHECK_SCALES = 1


class IvbCheckBuffer(Structure):
    _fields_ = [("data", c_void_p), ("count", c_int64), ("kind", c_int32), ("pad", c_int32)]


class IvbLayerDesc(Structure):
    _fields_ = [
        ("kind", c_int32),
        ("mixer_norm", c_void_p),
        ("mixer_norm_eps", c_float),
        ("ffn_norm", c_void_p),
        ("ffn_norm_eps", c_float),
        ("entry", IvbTernary),
        ("out", IvbTernary),
        ("gate_up", IvbTernary),
        ("down", IvbTernary),
        ("decay", c_void_p),
        ("theta", c_void_p),
        ("skip", c_void_p),
        ("conv_weight", c_void_p),
        ("conv_bias", c_void_p),
        ("ssm_state", c_void_p),
        ("prev_force", c_void_p),
        ("conv_state", c_void_p),
        ("conv_taps", c_int32),
        ("half_dt_min", c_float),
        ("half_dt_range", c_float),
        ("k_nope_up", IvbTernary),
        ("v_up", IvbTernary),
        ("rope", c_void_p),
        ("latent_q", c_void_p),
        ("latent_scale", c_void_p),
        ("k_rope_cache", c_void_p),
        ("attn_scale", c_float),
        ("k_cache", c_void_p),
        ("v_cache", c_void_p),
    ]


class IvbModelDesc(Structure):
    _fields_ = [
        ("abi_version", c_int32),
        ("vocab", c_int32),
        ("hidden", c_int32),
        ("heads", c_int32),
        ("head_dim", c_int32),
        ("state_dim", c_int32),
        ("latent_dim", c_int32),
        ("rope_dim", c_int32),
        ("nope_dim", c_int32),
        ("dense", c_int32),
        ("num_layers", c_int32),
        ("max_len", c_int32),
        ("max_top_k", c_int32),
        ("act_eps", c_float),
        ("norm_clip", c_float),
        ("head", IvbTernary),
        ("final_norm", c_void_p),
        ("final_norm_eps", c_float),
        ("layers", POINTER(IvbLayerDesc)),
        ("logits", c_void_p),
        ("token", c_void_p),
        ("position", c_void_p),
        ("seen", c_void_p),
        ("history", c_void_p),
        ("history_len", c_int32),
        ("sampling", c_void_p),
        ("top_k", c_void_p),
        ("rng", c_void_p),
    ]


# (name, restype, argtypes) for every function declared in include/ivonar_b200.h
class IvbBatchLayer(Structure):
    _fields_ = [
        ("ssm_state", c_void_p),
        ("prev_force", c_void_p),
        ("conv_state", c_void_p),
        ("latent_q", c_void_p),
        ("latent_scale", c_void_p),
        ("k_rope_cache", c_void_p),
    ]


class IvbBatch(Structure):
    _fields_ = [
        ("batch", c_int32),
        ("layers", POINTER(IvbBatchLayer)),
        ("tokens", c_void_p),
        ("positions", c_void_p),
        ("logits", c_void_p),
        ("seen", c_void_p),
        ("rng", c_void_p),
        ("history", c_void_p),
        ("history_len", c_int32),
        ("step", c_void_p),
        ("sampling", c_void_p),
        ("top_k", c_void_p),
    ]


SIGNATURES = {
    "ivb_abi_version": (c_int32, []),
    "ivb_last_error": (c_char_p, []),
    "ivb_device_supported": (c_int32, []),
    "ivb_quantize": (c_int32, [c_void_p, c_void_p, c_int32, c_float, c_float, c_float, c_void_p, c_void_p, c_void_p, c_void_p]),
    "ivb_ternary_group_dots": (c_int32, [POINTER(IvbTernary), c_void_p, c_void_p, c_void_p]),
    "ivb_ternary_gemv": (c_int32, [POINTER(IvbTernary), c_void_p, c_void_p, c_float, c_float, c_float, c_int32, c_void_p, c_void_p]),
    "ivb_quantize_rows": (c_int32, [c_void_p, c_int32, c_int32, c_void_p, c_float, c_float, c_float, c_void_p, c_int32, c_void_p, c_void_p, c_void_p]),
    "ivb_ternary_gemm": (c_int32, [POINTER(IvbTernary), c_void_p, c_int32, c_void_p, c_int32, c_int32, c_void_p, c_int32, c_void_p, c_void_p]),
    "ivb_decode_rows": (c_int32, [c_void_p, c_int32, c_int32, c_int32, c_int32, c_float, c_void_p, c_int32, c_int32, c_void_p, c_void_p]),
    "ivb_ternary_gemv_splitk": (c_int32, [POINTER(IvbTernary), c_void_p, c_void_p, c_float, c_float, c_float, c_int32, c_void_p, c_void_p]),
    "ivb_sample": (c_int32, [c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p]),
    "ivb_probe_wait_timeout": (c_int32, [c_void_p, c_void_p, c_uint64, c_void_p]),
    "ivb_decoder_create": (c_int32, [POINTER(IvbModelDesc), c_int32, POINTER(c_void_p)]),
    "ivb_decoder_destroy": (None, [c_void_p]),
    "ivb_decoder_workspace_bytes": (c_uint64, [c_void_p]),
    "ivb_decoder_num_phases": (c_int32, [c_void_p]),
    "ivb_decoder_ctas": (c_int32, [c_void_p]),
    "ivb_decoder_bind": (c_int32, [c_void_p, c_void_p, c_void_p]),
    "ivb_decoder_run": (c_int32, [c_void_p, c_int32, c_void_p, c_int32, c_uint64, c_void_p]),
    "ivb_decoder_trace": (c_int32, [c_void_p, c_void_p, c_int32]),
    "ivb_decoder_prefill_workspace_bytes": (c_uint64, [c_void_p, c_int32]),
    "ivb_decoder_prefill": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_uint64, c_void_p]),
    "ivb_batch_workspace_bytes": (c_uint64, [c_void_p, c_int32]),
    "ivb_batch_decode": (c_int32, [c_void_p, POINTER(IvbBatch), c_int32, c_void_p, c_uint64, c_void_p]),
    "ivb_batch_embed": (c_int32, [POINTER(IvbTernary), c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p]),
    "ivb_batch_ssm": (c_int32, [POINTER(IvbLayerDesc), POINTER(IvbBatchLayer), c_void_p, c_int32, c_int32, c_int32, c_int32,
                                c_int32, c_int32, c_void_p, c_void_p]),
    "ivb_batch_mla": (c_int32, [POINTER(IvbLayerDesc), POINTER(IvbBatchLayer), c_void_p, c_int32, c_void_p, c_int32, c_int32,
                                c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_float, c_void_p, c_void_p, c_void_p]),
    "ivb_batch_sample": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_int32, c_void_p, c_void_p,
                                   c_void_p, c_void_p, c_int32, c_void_p, c_void_p]),
    "ivb_validate_buffers": (c_int32, [c_void_p, c_int32, c_void_p, c_void_p]),
    "ivb_batch_topk_slice": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_int32,
                                       c_int32, c_void_p, c_void_p, c_void_p]),
    "ivb_batch_sample_merge": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p, c_int32, c_void_p,
                                         c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_int32, c_void_p]),
    "ivb_rows_amax": (c_int32, [c_void_p, c_int32, c_int32, c_void_p, c_void_p]),
    "ivb_quantize_rows_amax": (c_int32, [c_void_p, c_int32, c_int32, c_void_p, c_float, c_void_p, c_int32, c_void_p, c_void_p]),
    "ivb_decoder_check": (c_int32, [c_void_p, c_void_p]),
}

_lib: ctypes.CDLL | None = None


def _preload_cudart() -> None:
    import torch  # noqa: F401  (loads the CUDA runtime torch ships with)

    candidates = []
    for site in {os.path.dirname(os.path.dirname(torch.__file__))}:
        candidates += glob.glob(os.path.join(site, "nvidia", "cuda_runtime", "lib", "libcudart.so.12*"))
    candidates += ["/usr/local/cuda/lib64/libcudart.so.12"]
    for path in candidates:
        try:
            ctypes.CDLL(path, mode=ctypes.RTLD_GLOBAL)
            return
        except OSError:
            continue


def library() -> ctypes.CDLL:
    """Load libivonar_b200.so once; raises KernelError if it is missing."""

    global _lib
    if _lib is not None:
        return _lib
    if not LIBRARY.exists():
        raise KernelError(f"{LIBRARY.name} is not built (python -m ivonar_inference_b200.build)")
    try:
        lib = ctypes.CDLL(str(LIBRARY))
    except OSError:
        _preload_cudart()
        try:
            lib = ctypes.CDLL(str(LIBRARY))
        except OSError as exc:
            raise KernelError(f"cannot load {LIBRARY.name}: {exc}") from exc
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    if lib.ivb_abi_version() != IVB_ABI_VERSION:
        raise KernelError("libivonar_b200.so has a different ABI version than this package")
    _lib = lib
    return lib


def last_error() -> str:
    message = library().ivb_last_error()
    return message.decode(errors="replace") if message else ""


def check(rc: int, what: str) -> None:
    if rc == IVB_OK:
        return
    message = last_error()
    if rc == IVB_ECAPACITY:
        raise ValueError(message or "the decoder has no free position left")
    raise KernelError(f"{what} failed ({rc}): {message}")


def ternary(packed, scales, bias, rows: int, in_features: int) -> IvbTernary:
    """IvbTernary over device tensors (packed [rows, row_bytes] uint8, scales [rows, stride] fp16)."""

    return IvbTernary(
        packed.data_ptr(),
        scales.data_ptr(),
        0 if bias is None else bias.data_ptr(),
        int(rows),
        int(in_features),
        int(packed.shape[1]),
        int(scales.shape[1]),
    )
