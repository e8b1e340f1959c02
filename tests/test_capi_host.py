"""CPU-side checks of the C ABI library and the host logic (no GPU needed).

The library must load, export every entry point include/h3b.h declares, and
reject bad arguments with a status code and message before touching CUDA.
"""

import ctypes
import os
import re

import pytest
import torch

import h3b
from h3b import ops
from h3b._lib import EXPORTED, lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    text = open(os.path.join(ROOT, "include", "h3b.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(h3b_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    declared = header_symbols()
    assert declared, "no declarations parsed"
    handle = ctypes.CDLL(h3b.LIB_PATH)
    for name in declared:
        assert hasattr(handle, name), f"{name} declared in include/h3b.h but not exported"
    assert set(declared) == set(EXPORTED), "ctypes signature table and header disagree"


def _header_declarations():
    """name -> (return type, [parameter type]) for every entry point of include/h3b.h."""
    text = open(os.path.join(ROOT, "include", "h3b.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    decls = {}
    for ret, name, params in re.findall(r"([A-Za-z_][\w ]*?\**)\s*\b(h3b_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text,
                                        flags=re.S):
        params = " ".join(params.split())
        types = [] if params in ("", "void") else [p.strip().rsplit(" ", 1)[0] if "*" not in p.strip().rsplit(" ", 1)[-1]
                                                   else p.strip() for p in params.split(",")]
        decls[name] = (" ".join(ret.split()), types)
    return decls


def _category(c_type: str) -> str:
    if "*" in c_type:
        return "pointer"
    return {"int64_t": "int64", "int": "int", "float": "float"}[c_type.replace("const ", "").strip()]


def _ctypes_category(t) -> str:
    if t is ctypes.c_void_p or (isinstance(t, type) and issubclass(t, ctypes._Pointer)):
        return "pointer"
    return {ctypes.c_int64: "int64", ctypes.c_int: "int", ctypes.c_float: "float"}[t]


def test_ctypes_signatures_match_the_header_parameter_by_parameter():
    from h3b._lib import _RESTYPES, _SIGNATURES

    decls = _header_declarations()
    assert set(decls) == set(_SIGNATURES)
    for name, (ret, params) in decls.items():
        restype = _RESTYPES.get(name, ctypes.c_int)
        assert (ret, restype) in (("int", ctypes.c_int), ("int64_t", ctypes.c_int64),
                                  ("const char*", ctypes.c_char_p)), f"{name} returns {ret}, ctypes {restype}"
        argtypes = _SIGNATURES[name]
        assert len(params) == len(argtypes), f"{name}: header has {len(params)} parameters, ctypes {len(argtypes)}"
        for i, (c_type, t) in enumerate(zip(params, argtypes)):
            assert _category(c_type) == _ctypes_category(t), f"{name} parameter {i}: {c_type} vs {t}"


def test_version_and_error_string():
    assert lib().h3b_version().startswith(b"h3b")
    assert lib().h3b_last_error() is not None


def test_null_pointer_is_rejected_without_cuda():
    st = lib().h3b_quantize_int8_rowwise(None, 4, 256, 256, None, None, None)
    assert st == -1
    assert b"null" in lib().h3b_last_error()


def test_unsupported_shapes_are_rejected():
    dummy = ctypes.c_void_p(16)
    assert lib().h3b_quantize_int8_rowwise_convrot(dummy, 4, 300, 300, 256, 0, dummy, dummy, None) == -2
    assert lib().h3b_quantize_int8_rowwise_convrot(dummy, 4, 256, 256, 128, 0, dummy, dummy, None) == -2
    assert lib().h3b_quantize_int8_rowwise_convrot(dummy, 4, 256, 256, 256, 7, dummy, dummy, None) == -1
    assert lib().h3b_int8_gemm_dequant(dummy, dummy, dummy, dummy, 1, None, dummy, 8, 8, 24, 8, 2, None) == -2
    assert lib().h3b_int8_gemm_dequant(dummy, dummy, dummy, dummy, 1, None, dummy, 8, 8, 32, 8, 0, None) == -2
    assert lib().h3b_dequant_int4_grouped_to_int8(dummy, dummy, 0, None, dummy, 8, 64, 3, None) == -2
    assert lib().h3b_attention(dummy, dummy, 0, 96, 10, 128, dummy, dummy, 0, 10, 128, dummy, dummy, 1, None,
                               0.1, dummy, 128, None) == -2
    assert lib().h3b_attention(dummy, dummy, 2, 128, 10, 128, dummy, dummy, 0, 10, 128, dummy, dummy, 1, None,
                               0.1, dummy, 128, None) == -1
    assert lib().h3b_attention(dummy, ctypes.c_void_p(20), 0, 128, 10, 128, dummy, ctypes.c_void_p(20), 1, 10, 128,
                               dummy, dummy, 1, None, 0.1, dummy, 128, None) == -2
    assert lib().h3b_quantize_per_thread_int8(dummy, 10, 1, 128, None, 2, dummy, dummy, 128, None) == -1
    assert lib().h3b_selftest_bounded_wait(0, None) == -1
    assert lib().h3b_selftest_bounded_wait(2_000_000_000, None) == -1
    assert lib().h3b_bf16_gemm_accumulate(dummy, dummy, dummy, 8, 8, 12, 8, None) == -2
    assert lib().h3b_adaln_projection(dummy, dummy, None, 9, 64, 64, dummy, None) == -2    # 1..8 rows
    assert lib().h3b_adaln_projection(dummy, dummy, None, 1, 64, 12, dummy, None) == -1    # K % 8
    assert lib().h3b_adaln_projection(dummy, ctypes.c_void_p(24), None, 1, 64, 64, dummy, None) == -2


def test_qkv_qk_rope_entry_rejects_what_it_does_not_take():
    """The fused QKV + q/k norm/RoPE entry answers 'unsupported' (-2) for the cases its
    caller must route to the two-call path, and 'invalid' (-1) for bad arguments, all
    before any CUDA call."""
    d, odd = ctypes.c_void_p(16), ctypes.c_void_p(18)

    def call(D=d, ws_numel=1, M=4096, N=3072, stride=3072, H=8, q_off=0, k_off=1024, rot=128, qw=d):
        return lib().h3b_int8_gemm_dequant_qk_rope(d, d, d, d, ws_numel, None, D, M, N, 256, stride, H, q_off,
                                                   k_off, qw, d, d, d, rot, 1e-6, None)

    assert call(rot=64) == -2                      # rotary width without a fused epilogue
    assert call(k_off=512) == -2                   # Q and K head ranges overlap
    assert call(k_off=2560) == -2                  # K heads run past N
    assert call(q_off=64) == -2                    # head not at a 128-column boundary
    assert call(D=odd) == -2                       # unaligned output rows
    assert call(stride=3076) == -2                 # row stride not a multiple of 8
    assert call(ws_numel=7) == -1
    assert call(qw=None) == -1
    assert call(H=0) == -1
    assert b"H <= 0" in lib().h3b_last_error()
    assert call(rot=64) == -2
    assert b"rot_dim" in lib().h3b_last_error()


def test_empty_inputs_are_no_ops():
    assert lib().h3b_quantize_int8_rowwise(None, 0, 256, 256, None, None, None) == 0
    assert lib().h3b_int8_gemm_dequant(None, None, ctypes.c_void_p(16), ctypes.c_void_p(16), 1, None,
                                       ctypes.c_void_p(16), 0, 8, 32, 8, 2, None) == 0


def test_key_mean_workspace_size():
    # one fp64 partial sum per (1024-token chunk, head, channel)
    assert lib().h3b_key_mean_workspace_bytes(111600, 32) == 109 * 32 * 128 * 8


def test_ops_refuse_cpu_tensors():
    x = torch.zeros(4, 256, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.quantize_int8_rowwise(x)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.int8_linear(x, torch.zeros(8, 256, dtype=torch.int8), torch.ones(8))


def test_segment_rows():
    assert ops.segment_rows(None, 10, "cpu") is None
    assert ops.segment_rows(((0, 10, 0),), 10, "cpu") is None
    seg = ops.segment_rows(((0, 3, 1), (3, 10, 2)), 10, "cpu")
    assert seg.tolist() == [1, 1, 1, 2, 2, 2, 2, 2, 2, 2]
    with pytest.raises(ValueError):
        ops.segment_rows(((0, 3, 1), (4, 10, 2)), 10, "cpu")
    with pytest.raises(ValueError):
        ops.segment_rows(((0, 9, 1),), 10, "cpu")


def test_act_code_validation():
    assert ops.act_code(None) == 0 and ops.act_code("gelu_tanh") == 1 and ops.act_code("swiglu") == 2
    with pytest.raises(ValueError, match="unsupported input_act"):
        ops.act_code("relu")
