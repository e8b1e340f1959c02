"""Torch-facing operators over libh3b.so.

Each function mirrors the comfy_kitchen operator the X-MinimaxH3 native engine
calls for this path (same name, argument meaning and validation errors), but
runs the sm_100a kernels through the C ABI.  Tensors must already be on a CUDA
device: there is no CPU or eager fallback, and a missing library raises.

    quantize_int8_rowwise            comfy_kitchen eager/quantization.py:857-875 (cuda launcher int8_linear.cu:1035)
    quantize_int8_rowwise_convrot64  comfy_kitchen backends/cuda/__init__.py:2041-2053 (int8_linear.cu:943-1030)
    rms_adaln_quantize_int8          model/kernels.py:7594-7642 fused with the quantizer above
    int8_linear                      comfy_kitchen __init__.py:722-769 / cuda/__init__.py:1960-2081
    int8_linear_prequantized         comfy_kitchen cuda/__init__.py:1934-1957
    int8_linear_gated_residual_      int8_linear + residual.addcmul_ (model/fused_mlp.py:393-425)
    dequant_int4_grouped_to_int8     comfy_kitchen eager/w4a8_int8.py:344-363 (w4a8_gemm.cu:36-90)
    w4a8_int8_linear                 comfy_kitchen tensor/w4a8_int8.py:89-115 (cuda/__init__.py:2139-2298)
"""

from __future__ import annotations

import ctypes

import torch

from ._lib import H3B_ERR_UNSUPPORTED, check, lib

_ACT_CODES = {None: 0, "none": 0, "gelu_tanh": 1, "swiglu": 2}


def _p(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _cuda(name: str, *tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(f"{name} runs only on CUDA tensors (the B200 library has no CPU path)")


def _rows(x: torch.Tensor) -> torch.Tensor:
    """2-D view with unit column stride (row stride may be larger)."""
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1 or x2.data_ptr() % 16 or x2.stride(0) % 8:
        x2 = x2.contiguous()
    return x2


def act_code(input_act: str | None) -> int:
    try:
        return _ACT_CODES[input_act]
    except KeyError:
        known = sorted(k for k in _ACT_CODES if k is not None)
        raise ValueError(f"unsupported input_act: {input_act!r} (expected one of {known})") from None


# ----------------------------------------------------------------------------- quantization


def quantize_int8_rowwise(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row INT8 codes and fp32 scales ([..., K] -> int8 [M, K], f32 [M, 1])."""
    _cuda("quantize_int8_rowwise", x)
    if x.dtype != torch.bfloat16:
        raise ValueError("quantize_int8_rowwise expects bfloat16 activations")
    x2 = _rows(x)
    M, K = x2.shape
    q = torch.empty((M, K), device=x.device, dtype=torch.int8)
    s = torch.empty((M, 1), device=x.device, dtype=torch.float32)
    check(lib().h3b_quantize_int8_rowwise(_p(x2), M, K, x2.stride(0), _p(q), _p(s), _stream(x)),
          "quantize_int8_rowwise")
    return q, s


def quantize_int8_rowwise_convrot64(x: torch.Tensor, group_size: int = 256, input_act: str | None = None,
                                    ) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused activation + ConvRot-256 + per-row INT8 quantization."""
    _cuda("quantize_int8_rowwise_convrot64", x)
    if x.dtype != torch.bfloat16:
        raise ValueError("quantize_int8_rowwise_convrot64 expects bfloat16 activations")
    code = act_code(input_act)
    x2 = _rows(x)
    M, W = x2.shape
    K = W // 2 if code == 2 else W
    if code == 2 and W % 2:
        raise ValueError("swiglu input must have an even width [gate | up]")
    if group_size != 256 or K % group_size:
        raise ValueError(f"ConvRot group size {group_size} must be 256 and divide the input width {K}")
    q = torch.empty((M, K), device=x.device, dtype=torch.int8)
    s = torch.empty((M, 1), device=x.device, dtype=torch.float32)
    check(lib().h3b_quantize_int8_rowwise_convrot(_p(x2), M, K, x2.stride(0), group_size, code, _p(q), _p(s),
                                                  _stream(x)), "quantize_int8_rowwise_convrot64")
    return q, s


def segment_rows(segments, rows: int, device) -> torch.Tensor | None:
    """Per-token modulation-table row for AdaLN segments ((start, stop, row), ...);
    None when every token uses row 0."""
    if not segments:
        return None
    segments = tuple(segments)
    if len(segments) == 1 and int(segments[0][2]) == 0:
        start, stop, _ = segments[0]
        if int(start) != 0 or int(stop) != rows:
            raise ValueError("modulation segments do not cover the packed sequence")
        return None
    out = torch.empty(rows, dtype=torch.int32)
    prev = 0
    for start, stop, row in segments:
        if int(start) != prev or int(stop) <= int(start):
            raise ValueError("modulation segments must be an ordered partition")
        out[int(start):int(stop)] = int(row)
        prev = int(stop)
    if prev != rows:
        raise ValueError("modulation segments do not cover the packed sequence")
    return out.to(device)


def rms_adaln_quantize_int8(x: torch.Tensor, norm_weight: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor,
                            segments=None, eps: float = 1e-5, convrot_group_size: int = 256,
                            ) -> tuple[torch.Tensor, torch.Tensor]:
    """RMSNorm(norm_weight) + AdaLN (x * (1 + scale) + shift, bf16 boundaries) + ConvRot + INT8.

    scale / shift: bf16 [K] or per-segment tables [R, K]; segments as in
    model/layers.py:916-941.
    """
    _cuda("rms_adaln_quantize_int8", x, norm_weight, scale, shift)
    x2 = _rows(x)
    M, K = x2.shape
    w = norm_weight.to(torch.bfloat16).contiguous()
    sc = scale.to(torch.bfloat16).reshape(-1, K).contiguous()
    sh = shift.to(torch.bfloat16).reshape(-1, K).contiguous()
    seg = segment_rows(segments, M, x.device)
    q = torch.empty((M, K), device=x.device, dtype=torch.int8)
    s = torch.empty((M, 1), device=x.device, dtype=torch.float32)
    check(lib().h3b_rms_adaln_quantize_int8(_p(x2), M, K, x2.stride(0), _p(w), _p(sc), _p(sh), _p(seg), float(eps),
                                            int(convrot_group_size), _p(q), _p(s), _stream(x)),
          "rms_adaln_quantize_int8")
    return q, s


def qk_rmsnorm_rope_(qkv: torch.Tensor, heads: int, q_offset: int, k_offset: int, q_weight: torch.Tensor,
                     k_weight: torch.Tensor, cos_table: torch.Tensor, sin_table: torch.Tensor,
                     eps: float = 1e-6) -> torch.Tensor:
    """In-place per-head RMSNorm + split-half partial RoPE of the Q and K heads of
    projection rows qkv [L, W] (bf16); cos/sin tables bf16 [L, rot_dim/2]
    (model/layers.py:72-149)."""
    _cuda("qk_rmsnorm_rope_", qkv, q_weight, k_weight, cos_table, sin_table)
    if qkv.dtype != torch.bfloat16 or qkv.ndim != 2 or qkv.stride(1) != 1:
        raise ValueError("qkv must be bfloat16 rows [L, W] with unit column stride")
    L = qkv.shape[0]
    rot = 2 * cos_table.shape[-1]
    if cos_table.shape != (L, rot // 2) or sin_table.shape != cos_table.shape:
        raise ValueError("rotation tables must be [L, rot_dim/2]")
    qw = q_weight.to(torch.bfloat16).contiguous()
    kw = k_weight.to(torch.bfloat16).contiguous()
    ct = cos_table.to(torch.bfloat16).contiguous()
    st = sin_table.to(torch.bfloat16).contiguous()
    check(lib().h3b_qk_rmsnorm_rope(_p(qkv), L, heads, qkv.stride(0), q_offset, k_offset, _p(qw), _p(kw), _p(ct),
                                    _p(st), rot, float(eps), _stream(qkv)), "qk_rmsnorm_rope_")
    return qkv


# ----------------------------------------------------------------------------- GEMM


def _weight_scale(weight_scale: torch.Tensor, n: int, device) -> torch.Tensor:
    ws = weight_scale.to(device=device, dtype=torch.float32).reshape(-1).contiguous()
    if ws.numel() not in (1, n):
        raise ValueError(f"INT8 weight scale must be scalar or per-output-channel, got {tuple(weight_scale.shape)}")
    return ws


def _bias_f32(bias: torch.Tensor | None, n: int, device) -> torch.Tensor | None:
    if bias is None:
        return None
    b = bias.to(device=device, dtype=torch.float32).reshape(-1).contiguous()
    if b.numel() != n:
        raise ValueError("bias does not match the weight's output rows")
    return b


def int8_mm_i32(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """int32 acc[M, N] = a[M, K] . b[N, K]^T on the tcgen05 pipeline (verification)."""
    _cuda("int8_mm_i32", a, b)
    a = a.contiguous()
    b = b.contiguous()
    M, K = a.shape
    N = b.shape[0]
    acc = torch.empty((M, N), device=a.device, dtype=torch.int32)
    check(lib().h3b_int8_gemm_i32(_p(a), _p(b), _p(acc), M, N, K, _stream(a)), "int8_mm_i32")
    return acc


def int8_linear_prequantized(xq: torch.Tensor, xs: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor,
                             bias: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16,
                             out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16(xq . weight^T * xs * ws + bias) for already-quantized rows."""
    _cuda("int8_linear_prequantized", xq, xs, weight)
    if out_dtype != torch.bfloat16:
        raise ValueError("the B200 INT8 GEMM writes bfloat16 output")
    if weight.dtype != torch.int8 or weight.ndim != 2:
        raise ValueError("weight must be a rank-two int8 tensor")
    xq2 = xq if xq.is_contiguous() else xq.contiguous()
    M, K = xq2.shape
    N = weight.shape[0]
    if weight.shape[1] != K:
        raise ValueError(f"Input and weight inner dimensions must match, got {K} and {weight.shape[1]}")
    w = weight if weight.is_contiguous() else weight.contiguous()
    ws = _weight_scale(weight_scale, N, xq.device)
    b = _bias_f32(bias, N, xq.device)
    xs2 = xs.reshape(-1).to(torch.float32).contiguous()
    if out is None:
        out = torch.empty((M, N), device=xq.device, dtype=torch.bfloat16)
    check(lib().h3b_int8_gemm_dequant(_p(xq2), _p(w), _p(xs2), _p(ws), ws.numel(), _p(b), _p(out), M, N, K,
                                      out.stride(0), 2, _stream(xq)), "int8_linear_prequantized")
    return out


def int8_linear_prequantized_qk_rope(xq: torch.Tensor, xs: torch.Tensor, weight: torch.Tensor,
                                     weight_scale: torch.Tensor, bias: torch.Tensor | None, out: torch.Tensor,
                                     heads: int, q_offset: int, k_offset: int, q_weight: torch.Tensor,
                                     k_weight: torch.Tensor, cos_table: torch.Tensor, sin_table: torch.Tensor,
                                     eps: float = 1e-6) -> torch.Tensor:
    """The QKV projection into `out` with the per-head q/k RMSNorm + split-half RoPE
    applied in the GEMM epilogue (model/layers.py:277-295 then 72-149).  Bit-identical
    to int8_linear_prequantized followed by qk_rmsnorm_rope_, which it runs instead
    when the library reports the shape unsupported by the fused epilogue (GEMMs that
    take the 1-SM kernel, rotary widths other than 96 and 128)."""
    _cuda("int8_linear_prequantized_qk_rope", xq, xs, weight, out, q_weight, k_weight, cos_table, sin_table)
    if weight.dtype != torch.int8 or weight.ndim != 2:
        raise ValueError("weight must be a rank-two int8 tensor")
    if out.dtype != torch.bfloat16 or out.ndim != 2 or out.stride(1) != 1:
        raise ValueError("out must be bfloat16 rows [M, N] with unit column stride")
    xq2 = xq if xq.is_contiguous() else xq.contiguous()
    M, K = xq2.shape
    N = weight.shape[0]
    if weight.shape[1] != K or tuple(out.shape) != (M, N):
        raise ValueError(f"shape mismatch: xq {tuple(xq.shape)}, weight {tuple(weight.shape)}, out {tuple(out.shape)}")
    rot = 2 * cos_table.shape[-1]
    if cos_table.shape != (M, rot // 2) or sin_table.shape != cos_table.shape:
        raise ValueError("rotation tables must be [M, rot_dim/2]")
    w = weight if weight.is_contiguous() else weight.contiguous()
    ws = _weight_scale(weight_scale, N, xq.device)
    b = _bias_f32(bias, N, xq.device)
    xs2 = xs.reshape(-1).to(torch.float32).contiguous()
    qw = q_weight.to(torch.bfloat16).contiguous()
    kw = k_weight.to(torch.bfloat16).contiguous()
    ct = cos_table.to(torch.bfloat16).contiguous()
    st = sin_table.to(torch.bfloat16).contiguous()
    status = lib().h3b_int8_gemm_dequant_qk_rope(_p(xq2), _p(w), _p(xs2), _p(ws), ws.numel(), _p(b), _p(out), M, N,
                                                 K, out.stride(0), heads, q_offset, k_offset, _p(qw), _p(kw), _p(ct),
                                                 _p(st), rot, float(eps), _stream(xq))
    if status != H3B_ERR_UNSUPPORTED:
        check(status, "int8_linear_prequantized_qk_rope")
        return out
    int8_linear_prequantized(xq2, xs2, w, ws, b, out=out)
    return qk_rmsnorm_rope_(out, heads, q_offset, k_offset, qw, kw, ct, st, eps)


def quantize_rotated_int8(rot: torch.Tensor, amax: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row INT8 codes and scales of GELU + ConvRot rotated bf16 rows whose absmax is
    spread over amax [M, C] (the output of the fused FC1 epilogue)."""
    _cuda("quantize_rotated_int8", rot, amax)
    if rot.dtype != torch.bfloat16 or rot.ndim != 2 or rot.stride(1) != 1:
        raise ValueError("rot must be bfloat16 rows [M, K] with unit column stride")
    if amax.dtype != torch.float32 or amax.ndim != 2 or amax.shape[0] != rot.shape[0] or amax.stride(1) != 1:
        raise ValueError("amax must be float32 [M, C] with unit column stride")
    M, K = rot.shape
    q = torch.empty((M, K), device=rot.device, dtype=torch.int8)
    s = torch.empty((M, 1), device=rot.device, dtype=torch.float32)
    check(lib().h3b_quantize_rotated_int8(_p(rot), M, K, rot.stride(0), _p(amax), amax.stride(0), amax.shape[1],
                                          _p(q), _p(s), _stream(rot)), "quantize_rotated_int8")
    return q, s


def int8_linear_gelu_convrot_quantize(xq: torch.Tensor, xs: torch.Tensor, weight: torch.Tensor,
                                      weight_scale: torch.Tensor, bias: torch.Tensor | None = None,
                                      ) -> tuple[torch.Tensor, torch.Tensor]:
    """FC1 of the GELU MLP and the next layer's input quantizer (tanh-GELU, ConvRot-256,
    per-row INT8) in two launches: the GEMM epilogue applies the GELU and the rotation,
    a light pass forms the codes (model/fused_mlp.py:269-426 with comfy_kitchen
    int8_linear.cu:943-1030).  Bit-identical to int8_linear_prequantized followed by
    quantize_int8_rowwise_convrot64(h, 256, "gelu_tanh"), which it runs instead when
    the library reports the shape unsupported by the fused epilogue (GEMMs that take
    the 1-SM kernel, widths that are not a multiple of 256 or above 16384)."""
    _cuda("int8_linear_gelu_convrot_quantize", xq, xs, weight)
    if weight.dtype != torch.int8 or weight.ndim != 2:
        raise ValueError("weight must be a rank-two int8 tensor")
    xq2 = xq if xq.is_contiguous() else xq.contiguous()
    M, K = xq2.shape
    N = weight.shape[0]
    if weight.shape[1] != K:
        raise ValueError(f"Input and weight inner dimensions must match, got {K} and {weight.shape[1]}")
    w = weight if weight.is_contiguous() else weight.contiguous()
    ws = _weight_scale(weight_scale, N, xq.device)
    b = _bias_f32(bias, N, xq.device)
    xs2 = xs.reshape(-1).to(torch.float32).contiguous()
    rot = torch.empty((M, N), device=xq.device, dtype=torch.bfloat16)
    amax = torch.empty((M, max(N // 128, 1)), device=xq.device, dtype=torch.float32)
    status = lib().h3b_int8_gemm_gelu_convrot(_p(xq2), _p(w), _p(xs2), _p(ws), ws.numel(), _p(b), _p(rot), M, N, K,
                                              rot.stride(0), _p(amax), amax.stride(0), _stream(xq))
    if status != H3B_ERR_UNSUPPORTED:
        check(status, "int8_linear_gelu_convrot_quantize")
        return quantize_rotated_int8(rot, amax)
    del amax
    int8_linear_prequantized(xq2, xs2, w, ws, b, out=rot)
    return quantize_int8_rowwise_convrot64(rot, 256, "gelu_tanh")


def _quantize_for_linear(x, convrot, convrot_groupsize, input_act):
    if convrot:
        return quantize_int8_rowwise_convrot64(x, convrot_groupsize, input_act)
    if act_code(input_act):
        raise ValueError("input_act is fused only into the ConvRot quantizer")
    return quantize_int8_rowwise(x)


def int8_linear(x: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor, bias: torch.Tensor | None = None,
                out_dtype: torch.dtype = torch.bfloat16, convrot: bool = False, convrot_groupsize: int = 256,
                input_act: str | None = None) -> torch.Tensor:
    """Dynamic per-token INT8 quantization (optionally activation + ConvRot) + INT8 GEMM."""
    _cuda("int8_linear", x, weight)
    in_w = x.shape[-1] // (2 if act_code(input_act) == 2 else 1)
    if in_w != weight.shape[-1]:
        raise ValueError(f"Input and weight inner dimensions must match, got {in_w} and {weight.shape[-1]}")
    xq, xs = _quantize_for_linear(x, convrot, convrot_groupsize, input_act)
    out = int8_linear_prequantized(xq, xs, weight, weight_scale, bias, out_dtype)
    return out.reshape(*x.shape[:-1], weight.shape[0])


def int8_linear_gated_residual_(residual: torch.Tensor, gate: torch.Tensor, xq: torch.Tensor, xs: torch.Tensor,
                                weight: torch.Tensor, weight_scale: torch.Tensor,
                                bias: torch.Tensor | None = None) -> torch.Tensor:
    """residual += bf16(xq . weight^T * xs * ws + bias) * gate, in place (one bf16 rounding)."""
    _cuda("int8_linear_gated_residual_", residual, gate, xq, weight)
    M, K = xq.shape
    N = weight.shape[0]
    if residual.shape[-1] != N or residual.reshape(-1, N).shape[0] != M:
        raise ValueError("residual does not match the linear's output")
    if residual.dtype != torch.bfloat16 or residual.stride(-1) != 1:
        raise ValueError("residual must be a bfloat16 tensor with unit column stride")
    r2 = residual.view(-1, N) if residual.is_contiguous() else residual
    g = gate.to(device=residual.device, dtype=torch.bfloat16).reshape(-1).contiguous()
    if g.numel() != N:
        raise ValueError("gate must have one value per output column")
    ws = _weight_scale(weight_scale, N, xq.device)
    b = _bias_f32(bias, N, xq.device)
    xs2 = xs.reshape(-1).to(torch.float32).contiguous()
    w = weight if weight.is_contiguous() else weight.contiguous()
    check(lib().h3b_int8_gemm_gated_residual(_p(xq.contiguous()), _p(w), _p(xs2), _p(ws), ws.numel(), _p(b), _p(g),
                                             _p(r2), M, N, K, r2.stride(0), _stream(xq)),
          "int8_linear_gated_residual_")
    return residual


# ----------------------------------------------------------------------------- W4A8


def dequant_int4_grouped_to_int8(qdata: torch.Tensor, s_rel: torch.Tensor, codebook: torch.Tensor | None,
                                 group_size: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Packed int4 [N, K/2] + s_rel [N, K/G] (f32 or e4m3) -> int8 grid [N, K]."""
    _cuda("dequant_int4_grouped_to_int8", qdata, s_rel, codebook)
    if qdata.dtype != torch.int8 or qdata.ndim != 2:
        raise ValueError("packed weight must be a 2D int8 tensor")
    N, Kh = qdata.shape
    K = Kh * 2
    if s_rel.dtype == torch.float8_e4m3fn:
        kind, sr = 1, s_rel.contiguous().view(torch.uint8)
    elif s_rel.dtype == torch.float32:
        kind, sr = 0, s_rel.contiguous()
    else:
        raise ValueError("s_rel must be float32 or float8_e4m3fn")
    if tuple(s_rel.shape) != (N, K // group_size):
        raise ValueError(f"s_rel must have shape {(N, K // group_size)}, got {tuple(s_rel.shape)}")
    cb = None if codebook is None else codebook.to(torch.float32).contiguous()
    if cb is not None and cb.numel() != 16:
        raise ValueError("codebook must have 16 entries")
    if out is None:
        out = torch.empty((N, K), device=qdata.device, dtype=torch.int8)
    check(lib().h3b_dequant_int4_grouped_to_int8(_p(qdata.contiguous()), _p(sr), kind, _p(cb), _p(out), N, K,
                                                 int(group_size), _stream(qdata)), "dequant_int4_grouped_to_int8")
    return out


def w4a8_int8_linear(x: torch.Tensor, qdata: torch.Tensor, s_rel: torch.Tensor, s_channel: torch.Tensor,
                     codebook: torch.Tensor | None = None, correction: torch.Tensor | None = None,
                     bias: torch.Tensor | None = None, group_size: int = 16, convrot_groupsize: int = 256,
                     out_dtype: torch.dtype = torch.bfloat16, input_act: str | None = None) -> torch.Tensor:
    """x @ W^T + bias with W stored as grouped packed int4 (mandatory ConvRot)."""
    _cuda("w4a8_int8_linear", x, qdata, s_rel, s_channel)
    N, Kh = qdata.shape
    K = Kh * 2
    if group_size < 4 or K % 16 or K % group_size or K % convrot_groupsize or (
            16 % group_size != 0 and group_size % 16 != 0):
        raise ValueError(f"K={K} must be divisible by 16, group_size={group_size}, and "
                         f"convrot_groupsize={convrot_groupsize}; group_size must be >=4 "
                         f"and divide 16 or be a multiple of 16")
    if tuple(s_channel.shape) != (N,):
        raise ValueError(f"s_channel must have shape {(N,)}, got {tuple(s_channel.shape)}")
    in_w = x.shape[-1] // (2 if act_code(input_act) == 2 else 1)
    if in_w != K:
        raise ValueError(f"Input K={in_w} does not match qdata K={K}")
    w8 = dequant_int4_grouped_to_int8(qdata, s_rel, codebook, group_size)
    xq, xs = quantize_int8_rowwise_convrot64(x, convrot_groupsize, input_act)
    out = int8_linear_prequantized(xq, xs, w8, s_channel, bias, out_dtype)
    if correction is not None:
        w4a8_group_correction_(out, xq, xs, correction, group_size)
    return out.reshape(*x.shape[:-1], N)


def correction_operand(correction: torch.Tensor) -> torch.Tensor:
    """correction [K/G, N] -> the bf16 B operand [N, pad8(K/G)] of the correction GEMM
    (transposed so each output column's groups are contiguous; zero columns pad K to 8).
    A weight: build it once per layer."""
    groups, N = correction.shape
    kp = (groups + 7) // 8 * 8
    op = torch.zeros((N, kp), device=correction.device, dtype=torch.bfloat16)
    op[:, :groups] = correction.to(torch.bfloat16).t()
    return op


def w4a8_group_correction_(out: torch.Tensor, xq: torch.Tensor, xs: torch.Tensor, correction: torch.Tensor,
                           group_size: int, operand: torch.Tensor | None = None) -> torch.Tensor:
    """out += (sum of each group's activation codes * xs) @ correction [K/G, N], in bf16 with
    fp32 accumulation (comfy_kitchen backends/cuda/__init__.py:2294-2297): the group sums
    (h3b_w4a8_group_sums) then a tcgen05 bf16 GEMM accumulating into out
    (h3b_bf16_gemm_accumulate).  `operand`: correction_operand(correction), if cached."""
    _cuda("w4a8_group_correction_", out, xq, xs, correction)
    M, K = xq.shape
    groups = K // group_size
    N = out.shape[-1]
    if tuple(correction.shape) != (groups, N):
        raise ValueError(f"correction must have shape {(groups, N)}, got {tuple(correction.shape)}")
    if out.dtype != torch.bfloat16 or out.stride(-1) != 1:
        raise ValueError("the W4A8 correction accumulates into bfloat16 rows")
    op = correction_operand(correction) if operand is None else operand
    kp = op.shape[1]
    sx = torch.empty((M, kp), device=xq.device, dtype=torch.bfloat16)
    xs2 = xs.reshape(-1).to(torch.float32).contiguous()
    check(lib().h3b_w4a8_group_sums(_p(xq.contiguous()), _p(xs2), M, K, group_size, _p(sx), kp, _stream(xq)),
          "w4a8_group_sums")
    out2 = out.view(-1, N) if out.is_contiguous() else out
    check(lib().h3b_bf16_gemm_accumulate(_p(sx), _p(op), _p(out2), M, N, kp, out2.stride(0), _stream(xq)),
          "bf16_gemm_accumulate")
    return out


# ----------------------------------------------------------------------------- AdaLN projection


def adaln_projection(weight: torch.Tensor, bias: torch.Tensor | None, t: torch.Tensor) -> torch.Tensor:
    """bf16 [R, N] = bf16(t @ weight^T + bias) with fp32 products and sums on the GPU, for
    t [K] or [R, K] (rounded to bf16 first, as the engine's bf16 projector linear sees
    it) and a bf16 weight [N, K] (the engine's adaln_projector, model/layers.py:1083-1085)."""
    _cuda("adaln_projection", weight, t)
    if weight.dtype != torch.bfloat16 or weight.ndim != 2:
        raise ValueError("the AdaLN projection weight must be a bfloat16 matrix [N, K]")
    N, K = weight.shape
    t2 = t.reshape(-1, K).to(torch.bfloat16).contiguous()
    w = weight if weight.is_contiguous() else weight.contiguous()
    b = None
    if bias is not None:
        b = bias.to(torch.bfloat16).reshape(-1).contiguous()
        if b.numel() != N:
            raise ValueError("bias does not match the projection's output width")
    out = torch.empty((t2.shape[0], N), device=weight.device, dtype=torch.bfloat16)
    for r0 in range(0, t2.shape[0], 8):
        rows = min(8, t2.shape[0] - r0)
        check(lib().h3b_adaln_projection(_p(w), _p(t2[r0:r0 + rows]), _p(b), rows, N, K, _p(out[r0:r0 + rows]),
                                         _stream(w)), "adaln_projection")
    return out
