"""Loads libh3b.so (the sm_100a kernels behind the C ABI of include/h3b.h).

There is no fallback: if the library is missing or a call fails the error is
raised, so a run can never silently compute somewhere else.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libh3b.so")

_lib = None

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_int64 = ctypes.c_int64
c_float = ctypes.c_float


class MaskParams(ctypes.Structure):
    """h3b_mask_params (include/h3b.h)."""

    _fields_ = [
        ("mode", c_int),
        ("budget", c_void_p),
        ("protected_key_blocks", c_int64),
        ("keep_first_column", c_int),
        ("keep_diagonal", c_int),
        ("temporal_radius", c_int),
        ("temporal_spatial_radius", c_int),
        ("frames", c_int64),
        ("frame_tokens", c_int64),
        ("protected_tokens", c_int64),
        ("query_tokens", c_int64),
        ("query_indices", c_void_p),
        ("protected_query_blocks", c_int64),
    ]


# name -> argtypes (all return int status unless listed in _RESTYPES)
_SIGNATURES = {
    "h3b_version": [],
    "h3b_last_error": [],
    "h3b_device_status": [c_int, ctypes.POINTER(c_int), c_int],
    "h3b_selftest_bounded_wait": [c_int64, c_void_p],
    "h3b_quantize_int8_rowwise": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p],
    "h3b_quantize_int8_rowwise_convrot": [c_void_p, c_int64, c_int64, c_int64, c_int, c_int, c_void_p, c_void_p,
                                          c_void_p],
    "h3b_rms_adaln_quantize_int8": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_float, c_int, c_void_p, c_void_p, c_void_p],
    "h3b_int8_gemm_dequant": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int64,
                              c_int64, c_int64, c_int, c_void_p],
    "h3b_int8_gemm_dequant_qk_rope": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int64,
                                      c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                                      c_void_p, c_void_p, c_int, c_float, c_void_p],
    "h3b_int8_gemm_gated_residual": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                                     c_int64, c_int64, c_int64, c_int64, c_void_p],
    "h3b_int8_gemm_i32": [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p],
    "h3b_int8_gemm_gelu_convrot": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int64,
                                   c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p],
    "h3b_quantize_rotated_int8": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p,
                                  c_void_p, c_void_p],
    "h3b_dequant_int4_grouped_to_int8": [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                         c_void_p],
    "h3b_w4a8_group_sums": [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p],
    "h3b_bf16_gemm_accumulate": [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p],
    "h3b_adaln_projection": [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p],
    "h3b_key_mean_workspace_bytes": [c_int64, c_int64],
    "h3b_key_mean": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_void_p],
    "h3b_key_mean_no_alloc": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p],
    "h3b_pool_sim_quant": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
                           c_void_p, c_void_p, c_int64, c_void_p],
    "h3b_quantize_per_thread_int8": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_void_p, c_void_p,
                                     c_int64, c_void_p],
    "h3b_pool_sim_quant_slab": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
                                c_void_p, c_void_p, c_int64, c_int64, c_void_p],
    "h3b_value_fp8_given_absmax": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_void_p,
                                   c_void_p],
    "h3b_qk_rmsnorm_rope": [c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                            c_void_p, c_int, c_float, c_void_p],
    "h3b_value_fp8": [c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p],
    "h3b_ulysses_pack": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_void_p],
    "h3b_ulysses_unpack": [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p],
    "h3b_block_mask": [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int64,
                       ctypes.POINTER(MaskParams), c_void_p, c_void_p],
    "h3b_bitmap_to_lut": [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p],
    "h3b_attention": [c_void_p, c_void_p, c_int, c_int, c_int64, c_int64, c_void_p, c_void_p, c_int, c_int64,
                      c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_float, c_void_p, c_int64, c_void_p],
}
_RESTYPES = {"h3b_version": ctypes.c_char_p, "h3b_last_error": ctypes.c_char_p,
             "h3b_key_mean_workspace_bytes": c_int64}

EXPORTED = tuple(_SIGNATURES)


H3B_ERR_UNSUPPORTED = -2


class H3BError(RuntimeError):
    pass


def lib():
    """The loaded library; raises if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise H3BError(
                f"{LIB_PATH} is missing: build it with `python x-minimaxh3_b200/build.py` "
                "(the CUDA path has no fallback)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, argtypes in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = argtypes
            fn.restype = _RESTYPES.get(name, c_int)
        _lib = handle
    return _lib


# kernels each entry launches (for the benchmark's launch count); default 1
_KERNELS_PER_CALL = {"value_fp8": 3, "key_mean": 2, "key_mean_no_alloc": 2}
_launches = 0


def reset_launch_count() -> None:
    global _launches
    _launches = 0


def launch_count() -> int:
    return _launches


def check(status: int, what: str) -> None:
    global _launches
    _launches += _KERNELS_PER_CALL.get(what, 1)
    if status != 0:
        msg = lib().h3b_last_error().decode(errors="replace")
        raise H3BError(f"{what} failed with status {status}: {msg}")


def device_status(device: int = 0, reset: bool = True) -> int:
    """The device status word (0 = no kernel reported a timeout); clears it by default."""
    out = c_int(0)
    check(lib().h3b_device_status(device, ctypes.byref(out), int(reset)), "h3b_device_status")
    return out.value
