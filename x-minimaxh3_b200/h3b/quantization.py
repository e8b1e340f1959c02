"""Quantized linear layers of the H3 checkpoint contract, running on the B200 kernels.

Mirrors model/quantization.py of the native engine:
  * ComfyQuantSpec     (:96-138)  the `<prefix>.comfy_quant` payload (uint8 JSON bytes,
                                  bytes, str or a mapping), `int8_tensorwise` only;
  * W4A8QuantSpec      (:151-187) the file-level layer spec, `asym_w4a8_int8` only;
  * Int8Linear         ConvRotInt8Linear (:210-255, from_state_dict :233-255);
  * W4A8Linear         ConvRotW4A8Linear (:416-476).
The constructors make the same checks with the same exception types and messages.

The forward runs on this package's kernels and never on the host:
  INT8:  row INT8 (ConvRot or plain) quantizer -> tcgen05 INT8 GEMM, dequant epilogue;
  W4A8:  packed-nibble decode to the INT8 grid -> the same GEMM with s_channel in the
         epilogue -> optional group correction (comfy_kitchen w4a8 contract).
A layer also exposes the two halves separately (`quantize`, `forward_prequantized`)
and the gated-residual epilogue (`gated_residual_`), which is how the DiT block uses it.

The B200 quantizer implements the ConvRot group of 256, the value every H3
checkpoint records; a spec with another power-of-four group is refused with
ValueError when the layer is built.
"""

from __future__ import annotations

import json
from collections.abc import Mapping
from dataclasses import dataclass

import torch

from . import ops

CONVROT_GROUP = 256


def _power_of_four(size: int) -> bool:
    return not (size < 4 or size & (size - 1) or size.bit_length() % 2 == 0)


@dataclass(frozen=True, slots=True)
class ComfyQuantSpec:
    format: str
    convrot: bool = False
    convrot_groupsize: int = 256

    @classmethod
    def decode(cls, raw: object) -> "ComfyQuantSpec":
        if isinstance(raw, torch.Tensor):
            payload = bytes(raw.detach().cpu().to(torch.uint8).tolist())
        elif isinstance(raw, (bytes, bytearray, memoryview)):
            payload = bytes(raw)
        elif isinstance(raw, str):
            payload = raw.encode("utf-8")
        elif isinstance(raw, Mapping):
            return cls._from_mapping(dict(raw))
        else:
            raise TypeError(f"unsupported comfy_quant payload: {type(raw).__name__}")
        return cls._from_mapping(json.loads(payload.decode("utf-8")))

    @classmethod
    def _from_mapping(cls, data: Mapping[str, object]) -> "ComfyQuantSpec":
        params = data.get("params", {})
        if not isinstance(params, Mapping):
            params = {}
        return cls(format=str(data.get("format", "")),
                   convrot=bool(data.get("convrot", params.get("convrot", False))),
                   convrot_groupsize=int(data.get("convrot_groupsize", params.get("convrot_groupsize", 256))))

    def encode(self) -> torch.Tensor:
        """The uint8 JSON payload a checkpoint stores under `<prefix>.comfy_quant`."""
        body = json.dumps({"format": self.format,
                           "params": {"convrot": self.convrot, "convrot_groupsize": self.convrot_groupsize}})
        return torch.tensor(list(body.encode("utf-8")), dtype=torch.uint8)

    def validate_supported(self) -> None:
        if self.format != "int8_tensorwise":
            raise ValueError(f"native core currently supports int8_tensorwise, got {self.format!r}")
        if self.convrot and not _power_of_four(self.convrot_groupsize):
            raise ValueError("ConvRot group size must be a power of four")


@dataclass(frozen=True, slots=True)
class W4A8QuantSpec:
    """Physical layout recorded by the mixed W4A8 checkpoints."""

    format: str = "asym_w4a8_int8"
    group_size: int = 16
    convrot: bool = True
    convrot_groupsize: int = 256

    @classmethod
    def from_mapping(cls, data: Mapping[str, object]) -> "W4A8QuantSpec":
        return cls(format=str(data.get("format", "")), group_size=int(data.get("group_size", 16)),
                   convrot=bool(data.get("convrot", True)),
                   convrot_groupsize=int(data.get("convrot_groupsize", 256)))

    def to_mapping(self) -> dict[str, object]:
        return {"format": self.format, "group_size": self.group_size, "convrot": self.convrot,
                "convrot_groupsize": self.convrot_groupsize}

    def validate_supported(self) -> None:
        if self.format != "asym_w4a8_int8":
            raise ValueError(f"native core currently supports asym_w4a8_int8, got {self.format!r}")
        if self.group_size < 4 or (16 % self.group_size != 0 and self.group_size % 16 != 0):
            raise ValueError("W4A8 group size must be >=4 and divide 16 or be a multiple of 16")
        if not self.convrot:
            raise ValueError("the H3 W4A8 checkpoint requires ConvRot")
        if not _power_of_four(self.convrot_groupsize):
            raise ValueError("ConvRot group size must be a power of four")


def _check_b200_convrot(convrot: bool, size: int) -> None:
    if convrot and size != CONVROT_GROUP:
        raise ValueError(f"the B200 quantizer implements ConvRot group {CONVROT_GROUP}, got {size}")


class _QuantLinear:
    """Shared forward of the two layer kinds; subclasses provide `int8_weight()`."""

    spec_convrot: bool
    bias: torch.Tensor | None

    @property
    def bias_f32(self) -> torch.Tensor | None:
        """The bias as the fp32 vector the GEMM epilogues read, converted once."""
        b = self.bias
        if b is None:
            return None
        cached = getattr(self, "_bias_f32", None)
        if cached is None or cached[0] is not b:
            cached = (b, b.to(torch.float32).reshape(-1).contiguous())
            self._bias_f32 = cached
        return cached[1]

    @property
    def convrot_group_size(self) -> int:
        """ConvRot group of the activation quantizer, 0 for a plain row quantizer."""
        return CONVROT_GROUP if self.spec_convrot else 0

    def quantize(self, x: torch.Tensor, input_act: str | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """Per-token INT8 codes and scales of x with this layer's rotation (and input activation)."""
        if self.spec_convrot:
            return ops.quantize_int8_rowwise_convrot64(x, CONVROT_GROUP, input_act)
        if ops.act_code(input_act):
            raise ValueError("input_act is fused only into the ConvRot quantizer")
        return ops.quantize_int8_rowwise(x)

    def forward_prequantized(self, xq: torch.Tensor, xs: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """bf16 [M, N] from quantized rows; `out` (bf16 rows with unit column stride) receives it when given."""
        w8, ws = self.int8_weight()
        out = ops.int8_linear_prequantized(xq, xs, w8, ws, self.bias_f32, out=out)
        self._correct_(out, xq, xs)
        return out

    def forward_prequantized_for(self, next_layer: "_QuantLinear", xq: torch.Tensor, xs: torch.Tensor,
                                 input_act: str | None) -> tuple[torch.Tensor, torch.Tensor]:
        """This layer's output quantized as `next_layer`'s input with `input_act` applied
        (the MLP's FC1 feeding FC2, model/fused_mlp.py:269-426).  With a ConvRot next
        layer, tanh-GELU and no post-GEMM correction on this layer, the activation and
        the rotation run in this GEMM's epilogue; the codes and scales are the same
        either way."""
        if (input_act == "gelu_tanh" and next_layer.spec_convrot
                and getattr(self, "correction", None) is None):
            w8, ws = self.int8_weight()
            return ops.int8_linear_gelu_convrot_quantize(xq, xs, w8, ws, self.bias_f32)
        h = self.forward_prequantized(xq, xs)
        return next_layer.quantize(h, input_act)

    def forward_prequantized_qk_rope(self, xq: torch.Tensor, xs: torch.Tensor, out: torch.Tensor, heads: int,
                                     q_offset: int, k_offset: int, q_weight: torch.Tensor, k_weight: torch.Tensor,
                                     cos_table: torch.Tensor, sin_table: torch.Tensor, eps: float) -> torch.Tensor:
        """The QKV projection into `out` followed by the per-head q/k RMSNorm + RoPE
        (model/layers.py:277-295), fused into the GEMM epilogue when this layer has no
        post-GEMM correction; the same values either way."""
        if getattr(self, "correction", None) is None:
            w8, ws = self.int8_weight()
            return ops.int8_linear_prequantized_qk_rope(xq, xs, w8, ws, self.bias_f32, out, heads, q_offset, k_offset,
                                                        q_weight, k_weight, cos_table, sin_table, eps)
        self.forward_prequantized(xq, xs, out=out)
        return ops.qk_rmsnorm_rope_(out, heads, q_offset, k_offset, q_weight, k_weight, cos_table, sin_table, eps)

    def gated_residual_(self, residual: torch.Tensor, gate: torch.Tensor, xq: torch.Tensor,
                        xs: torch.Tensor) -> torch.Tensor:
        """residual += bf16(layer(x)) * gate with one bf16 rounding (model/layers.py:944-960)."""
        if getattr(self, "correction", None) is None:
            w8, ws = self.int8_weight()
            return ops.int8_linear_gated_residual_(residual, gate, xq, xs, w8, ws, self.bias_f32)
        update = self.forward_prequantized(xq, xs)
        return residual.addcmul_(update, gate.to(update.dtype))

    def _correct_(self, out, xq, xs) -> None:
        pass

    def __call__(self, x: torch.Tensor, input_act: str | None = None) -> torch.Tensor:
        xq, xs = self.quantize(x.reshape(-1, x.shape[-1]), input_act)
        return self.forward_prequantized(xq, xs).reshape(*x.shape[:-1], self.out_features)


class Int8Linear(_QuantLinear):
    """ConvRot INT8 layer: weight int8 [N, K] (stored rotated), weight_scale f32 [N] or [1],
    optional bias [N]."""

    def __init__(self, qweight: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor | None = None, *,
                 spec: ComfyQuantSpec, output_dtype: torch.dtype | None = None) -> None:
        spec.validate_supported()
        if qweight.ndim != 2 or qweight.dtype != torch.int8:
            raise ValueError("qweight must be a rank-two int8 tensor")
        if scale.numel() not in (1, qweight.shape[0]):
            raise ValueError("INT8 scale must be scalar or one value per output row")
        if bias is not None and bias.numel() != qweight.shape[0]:
            raise ValueError("bias does not match qweight output rows")
        if spec.convrot and qweight.shape[1] % spec.convrot_groupsize:
            raise ValueError("qweight input width is not divisible by ConvRot group size")
        _check_b200_convrot(spec.convrot, spec.convrot_groupsize)
        if output_dtype not in (None, torch.bfloat16):
            raise ValueError("the B200 INT8 GEMM writes bfloat16 output")
        self.qweight = qweight.contiguous()
        self.scale = scale.to(torch.float32).reshape(-1).contiguous()
        self.bias = bias
        self.spec = spec
        self.spec_convrot = spec.convrot

    @classmethod
    def from_state_dict(cls, state: Mapping[str, torch.Tensor], prefix: str, *,
                        output_dtype: torch.dtype | None = None) -> "Int8Linear":
        try:
            spec = ComfyQuantSpec.decode(state[f"{prefix}.comfy_quant"])
            qweight = state[f"{prefix}.weight"]
            scale = state[f"{prefix}.weight_scale"]
        except KeyError as error:
            raise KeyError(f"incomplete quantized layer {prefix!r}: missing {error.args[0]!r}") from error
        return cls(qweight, scale, state.get(f"{prefix}.bias"), spec=spec, output_dtype=output_dtype)

    @property
    def in_features(self) -> int:
        return int(self.qweight.shape[1])

    @property
    def out_features(self) -> int:
        return int(self.qweight.shape[0])

    def int8_weight(self) -> tuple[torch.Tensor, torch.Tensor]:
        return self.qweight, self.scale

    def dense_weight(self) -> torch.Tensor:
        """fp32 [N, K] weight the layer applies (in the rotated input basis when ConvRot)."""
        return self.qweight.float() * self.scale.view(-1, 1)


class W4A8Linear(_QuantLinear):
    """Packed W4 layer: qdata int8 [N, K/2] (even column in the low nibble), s_rel
    e4m3 or f32 [N, K/G], s_channel f32 [N], optional codebook [16], correction
    [K/G, N] and bias [N].  ConvRot is mandatory."""

    def __init__(self, qdata: torch.Tensor, s_rel: torch.Tensor, s_channel: torch.Tensor, *,
                 codebook: torch.Tensor | None = None, correction: torch.Tensor | None = None,
                 bias: torch.Tensor | None = None, spec: W4A8QuantSpec = W4A8QuantSpec(),
                 output_dtype: torch.dtype | None = None) -> None:
        spec.validate_supported()
        if qdata.ndim != 2 or qdata.dtype != torch.int8:
            raise ValueError("packed W4 weight must be a rank-two int8 tensor")
        out_features, packed_width = qdata.shape
        in_features = packed_width * 2
        if in_features % 16 or in_features % spec.group_size:
            raise ValueError("W4A8 input width is incompatible with its group size")
        if in_features % spec.convrot_groupsize:
            raise ValueError("W4A8 input width is incompatible with ConvRot")
        groups = in_features // spec.group_size
        if tuple(s_rel.shape) != (out_features, groups):
            raise ValueError(f"s_rel must be {(out_features, groups)}, got {tuple(s_rel.shape)}")
        if tuple(s_channel.shape) != (out_features,):
            raise ValueError(f"s_channel must be {(out_features,)}, got {tuple(s_channel.shape)}")
        if codebook is not None and tuple(codebook.shape) != (16,):
            raise ValueError("W4A8 codebook must contain 16 entries")
        if correction is not None and tuple(correction.shape) != (groups, out_features):
            raise ValueError("W4A8 correction must be [groups, out_features]")
        if bias is not None and bias.numel() != out_features:
            raise ValueError("bias does not match W4A8 output rows")
        _check_b200_convrot(True, spec.convrot_groupsize)
        if output_dtype not in (None, torch.bfloat16):
            raise ValueError("the B200 INT8 GEMM writes bfloat16 output")
        self.qdata = qdata.contiguous()
        self.s_rel = s_rel.contiguous()
        self.s_channel = s_channel.to(torch.float32).contiguous()
        self.codebook = codebook
        self.correction = correction
        self.bias = bias
        self.spec = spec
        self.spec_convrot = True

    @property
    def in_features(self) -> int:
        return int(self.qdata.shape[1]) * 2

    @property
    def out_features(self) -> int:
        return int(self.qdata.shape[0])

    def int8_weight(self) -> tuple[torch.Tensor, torch.Tensor]:
        """The INT8 grid decoded on the GPU for this call (the packed weight stays resident)."""
        return ops.dequant_int4_grouped_to_int8(self.qdata, self.s_rel, self.codebook, self.spec.group_size), \
            self.s_channel

    def _correct_(self, out, xq, xs) -> None:
        if self.correction is not None:
            if getattr(self, "_correction_operand", None) is None:
                self._correction_operand = ops.correction_operand(self.correction)
            ops.w4a8_group_correction_(out, xq, xs, self.correction, self.spec.group_size,
                                       self._correction_operand)

    def dense_weight(self) -> torch.Tensor:
        """fp32 [N, K] weight (model/quantization.py:486-516 decode order)."""
        packed = self.qdata.to(torch.int32) & 0xFF
        codes = torch.empty(self.out_features, self.in_features, dtype=torch.int64, device=packed.device)
        codes[:, 0::2] = packed & 0xF
        codes[:, 1::2] = (packed >> 4) & 0xF
        values = codes.float() - 8.0 if self.codebook is None else self.codebook.float()[codes]
        groups = self.in_features // self.spec.group_size
        grid = (values.view(self.out_features, groups, self.spec.group_size)
                * self.s_rel.float().unsqueeze(-1)).round().clamp_(-127, 127)
        weight = grid * self.s_channel.view(-1, 1, 1)
        if self.correction is not None:
            weight = weight + self.correction.float().T.unsqueeze(-1)
        return weight.reshape(self.out_features, self.in_features)
