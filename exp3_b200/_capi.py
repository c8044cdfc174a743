"""ctypes binding of libfpx.so (the C ABI declared in include/fpx.h).

The library is loaded once, on first use. If it is missing or cannot be loaded
the ops raise: there is no CPU or PyTorch fallback.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libfpx.so"

c_int, c_i64, c_size, c_double, c_void_p = ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_double, ctypes.c_void_p
P = c_void_p  # device pointers and the stream travel as void*

STATUS = {0: "ok", -1: "invalid argument", -2: "inconsistent shapes", -3: "unsupported",
          -4: "CUDA launch failed", -5: "workspace too small or misaligned", -6: "device wait timed out"}

METHOD_IDS = {"dense": 0, "fp_v1": 1, "mean_native": 2, "mean_balanced": 3, "cgf_mean": 4,
              "dispersion_mean": 5, "fp_v1_rescue": 6, "fp_v1_rescue_v2": 7}
STAGE_ROUTE, STAGE_EXACT, STAGE_MEAN, STAGE_ALL = 1, 2, 4, 7

S3 = [c_i64, c_i64, c_i64]
SIGNATURES = {
    "fpx_status_string": ([c_int], ctypes.c_char_p),
    "fpx_version": ([], c_int),
    "fpx_set_option": ([c_int, c_int], c_int),
    "fpx_device_error": ([ctypes.POINTER(c_int), c_int], c_int),
    "fpx_block_mean_k": ([P, *S3, c_int, c_int, c_int, c_int, c_int, P, P], c_int),
    "fpx_block_descriptors": ([P, *S3, P, *S3, c_int, c_int, c_int, c_int, c_int, P, P, P, P, P, P], c_int),
    "fpx_v1_scores": ([P, *S3, P, c_int, c_int, c_int, c_int, c_int, c_int, c_double, P, P], c_int),
    "fpx_deal_output_score": ([P, c_int, c_int, c_int, c_int, c_int, c_double, c_int, c_int, P, P, P], c_int),
    "fpx_selector_scores": ([P, *S3, P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_double,
                             P, P], c_int),
    "fpx_protected_selection": ([P, c_int, c_int, c_int, c_double, c_int, c_int, c_int, P, P], c_int),
    "fpx_indices_from_mask": ([P, c_int, c_int, c_int, P, P, P], c_int),
    "fpx_mask_from_indices": ([P, P, c_int, c_int, c_int, P, P], c_int),
    "fpx_selection_accounting": ([P, c_int, c_int, c_int, c_int, c_int, P, P], c_int),
    "fpx_exact_attention": ([P, *S3, P, *S3, P, *S3, P, P, c_int, c_int, c_int, c_int, c_int, c_int,
                             c_double, P, P, P], c_int),
    "fpx_mean_tail": ([P, *S3, P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_double, P, P, P], c_int),
    "fpx_merge_exact_mean": ([P, P, P, P, c_i64, c_int, P, P, P], c_int),
    "fpx_rescue_tail_workspace_bytes": ([c_int, c_int, c_int, c_int, c_int, c_int], c_size),
    "fpx_rescue_tail": ([P, *S3, P, *S3, P, *S3, P, c_int, c_int, c_int, c_int, c_int, c_int, c_double, c_int,
                         P, P, P, c_size, P], c_int),
    "fpx_prefill_workspace_bytes": ([c_int, c_int, c_int, c_int, c_int, c_int, c_int], c_size),
    "fpx_prefill_attention": ([c_int, c_double, c_int, c_int, c_int, P, *S3, P, *S3, P, *S3,
                               c_int, c_int, c_int, c_int, c_int, c_int, c_double,
                               c_int, c_int, c_int, c_int, P, *S3, P, P, c_size, c_int, P], c_int),
    "fpx_decode_workspace_bytes": ([c_int, c_int, c_int, c_int, c_int, c_int], c_size),
    "fpx_decode_attention": ([P, *S3, P, *S3, P, *S3, c_int, c_int, c_int, c_int, c_int, c_int, c_double,
                              P, *S3, P, P, c_size, P], c_int),
    "fpx_decode_attention_at": ([P, *S3, P, *S3, P, *S3, c_int, c_int, c_int, P, c_int, c_int, c_int, c_double,
                                 P, *S3, P, P, c_size, P], c_int),
    "fpx_decode_attention_noalloc": ([P, *S3, P, *S3, P, *S3, c_int, c_int, c_int, c_int, c_int, c_int,
                                      c_double, P, *S3, P, P], c_int),
    "fpx_ar_buffer_bytes": ([c_int], c_size),
    "fpx_ar_create": ([c_size, ctypes.POINTER(c_void_p), ctypes.POINTER(ctypes.c_char)], c_int),
    "fpx_ar_open": ([ctypes.POINTER(ctypes.c_char), ctypes.POINTER(c_void_p)], c_int),
    "fpx_ar_close": ([P], c_int),
    "fpx_ar_destroy": ([P], c_int),
    "fpx_ar_error": ([P, ctypes.POINTER(c_int)], c_int),
    "fpx_allreduce_bf16": ([P, c_i64, ctypes.POINTER(c_void_p), c_int, c_int, c_int, P], c_int),
    "fpx_rmsnorm": ([P, P, P, c_double, c_i64, c_int, P, P, P], c_int),
    "fpx_rope_neox": ([P, *S3, c_int, c_int, c_int, c_int, c_int, c_double, P], c_int),
    "fpx_rope_neox_at": ([P, *S3, c_int, c_int, c_int, c_int, P, c_double, P], c_int),
    "fpx_silu_mul": ([P, c_i64, c_int, P, P], c_int),
    "fpx_prefill_export_routing": ([c_int, c_int, c_int, c_int, c_int, c_int, c_int, P, c_size, P, P, P, P],
                                   c_int),
}

_lib = None
_lock = threading.Lock()


class FpxError(RuntimeError):
    pass


def lib():
    """The loaded library (raises FpxError when it is absent)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise FpxError(f"{LIB_PATH} is missing: build it with `python -m exp3_b200.build`")
                handle = ctypes.CDLL(str(LIB_PATH))
                for name, (args, res) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.argtypes, fn.restype = args, res
                _lib = handle
    return _lib


def call(name: str, *args) -> None:
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        cuda = ""
        if rc == -4:
            try:
                torch.cuda.synchronize()
            except RuntimeError as exc:  # surfaces the launch error text
                cuda = f": {exc}"
        raise FpxError(f"{name} failed with status {rc} ({STATUS.get(rc, 'unknown')}){cuda}")


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if t.device.type != "cuda":
            raise FpxError("fpx ops run on CUDA tensors only (there is no CPU path)")
    return dev


def strides3(t: torch.Tensor):
    """Element strides of dims 0..2 of a [B, L, heads, d] tensor whose last dim is contiguous."""
    if t.stride(-1) != 1:
        raise FpxError("the last dimension must be contiguous")
    return t.stride(0), t.stride(1), t.stride(2)


def device_error(reset: bool = True) -> int:
    """The device error word of libfpx (1 = a bounded wait in a kernel gave up); synchronises."""
    code = ctypes.c_int(0)
    rc = lib().fpx_device_error(ctypes.byref(code), 1 if reset else 0)
    if rc != 0:
        raise FpxError(f"fpx_device_error failed with status {rc}")
    return code.value


def set_exact_kernel(name: str) -> None:
    """Selects the exact-attention kernel at head dim 128: "tcgen05" (two query tiles per CTA),
    "tcgen05_single" (one tile per CTA, double-buffered S) or "mma" (the mma.sync cross-check)."""
    call("fpx_set_option", 1, {"tcgen05": 0, "mma": 1, "tcgen05_single": 2}[name])


def set_route_kernel(name: str) -> None:
    """Selects the V1 routing kernel: "tcgen05" (the default) or "mma" (the mma.sync cross-check)."""
    call("fpx_set_option", 3, {"tcgen05": 0, "mma": 1}[name])


def set_mean_kernel(name: str) -> None:
    """Selects the fused path's tail kernels (block-mean and rescue tails): "tcgen05" (the
    default) or "fp32" (the CUDA-core cross-check)."""
    call("fpx_set_option", 4, {"tcgen05": 0, "fp32": 1}[name])


def set_selector_kernel(name: str) -> None:
    """Selects the fused path's routing kernel for mean_balanced / cgf_mean / dispersion_mean:
    "tcgen05" (the default) or "fp32" (the CUDA-core cross-check)."""
    call("fpx_set_option", 5, {"tcgen05": 0, "fp32": 1}[name])


def set_exp_emulation(pairs_of_8: int) -> None:
    """How many of every 8 exp2 pairs the tcgen05 kernel evaluates on the FMA pipe (0, 2, 3)."""
    call("fpx_set_option", 2, int(pairs_of_8))
