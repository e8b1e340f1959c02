"""Pruned H3 checkpoints (`*_pruned_int8_convrot.safetensors`, `*_pruned_w4a8_mixed.safetensors`)
assembled into B200 DiT blocks.

Mirrors model/assembly.py of the native engine:
  * TensorSource, MappingTensorSource, SafeTensorSource (:64-150): the safetensors reader
    and the per-layer W4A8 specs under the file metadata key `_quantization_metadata`
    (JSON `{"layers": {prefix: spec}}`), with the same errors;
  * quant_linear = _quant_linear (:166-228): `<prefix>.weight_scale` present -> ConvRot
    INT8 from (weight, weight_scale, comfy_quant); else `weight_s_rel` and
    `weight_s_channel` -> packed W4A8 (weight, optional weight_codebook,
    weight_correction, bias) with the layer's spec, or the H3 default
    {asym_w4a8_int8, group 16, ConvRot 256} when the source records none; else KeyError;
  * load_block = assemble_pruned_block (:259-333): the tensor names of block i
    (blocks.{i}.attn.qkv_proj / attn.out_proj / mlp.fc1 / mlp.fc2, attn.q_norm.weight,
    attn.k_norm.weight, norm1.weight, norm2.weight, adaln_proj.linear.{weight,bias}).
The block dimensions are read from the tensors themselves.  The AdaLN projection is
kept as stored (18 * hidden rows in H3: three modulation rows per timestep row,
model/layers.py:910-913) and is evaluated in fp32 over bf16-rounded weights, as the
engine does (assembly.py:306-315).  LoRA updates are outside this path.
"""

from __future__ import annotations

import json
from collections.abc import Mapping
from typing import Protocol

import torch

from . import attention as A
from .block import BlockConfig, DiTBlockB200
from .quantization import Int8Linear, W4A8Linear, W4A8QuantSpec

H3_NUM_LAYERS = 50          # model/config.py:12-17
H3_NORM_EPS = 1e-5
H3_QK_NORM_EPS = 1e-5
_DEFAULT_W4A8_SPEC = {"format": "asym_w4a8_int8", "group_size": 16, "convrot": True, "convrot_groupsize": 256}


class TensorSource(Protocol):
    def tensor(self, key: str) -> torch.Tensor: ...

    def has_tensor(self, key: str) -> bool: ...

    def quantization_spec(self, prefix: str) -> Mapping[str, object] | None: ...


class MappingTensorSource:
    def __init__(self, state: Mapping[str, torch.Tensor], *,
                 quantization_metadata: Mapping[str, Mapping[str, object]] | None = None) -> None:
        self.state = state
        self._quantization_metadata = dict(quantization_metadata or {})

    def tensor(self, key: str) -> torch.Tensor:
        return self.state[key]

    def has_tensor(self, key: str) -> bool:
        return key in self.state

    def quantization_spec(self, prefix: str) -> Mapping[str, object] | None:
        return self._quantization_metadata.get(prefix)


def parse_quantization_metadata(metadata: Mapping[str, str] | None) -> dict[str, dict[str, object]]:
    """Per-layer specs from safetensors file metadata (`_quantization_metadata`)."""
    raw = (metadata or {}).get("_quantization_metadata")
    if not raw:
        return {}
    try:
        decoded = json.loads(raw)
        layers = decoded.get("layers", {})
        if not isinstance(layers, Mapping):
            raise TypeError("layers must be a mapping")
        return {str(name): dict(spec) for name, spec in layers.items() if isinstance(spec, Mapping)}
    except (json.JSONDecodeError, TypeError, ValueError, AttributeError) as error:
        raise ValueError("invalid safetensors _quantization_metadata") from error


class SafeTensorSource:
    """Lazy safetensors reader; keep its context open while assembling blocks."""

    def __init__(self, path: str) -> None:
        self.path = path
        self._reader = None
        self._keys: set[str] = set()
        self._quantization_metadata: dict[str, dict[str, object]] = {}

    def __enter__(self) -> "SafeTensorSource":
        try:
            from safetensors import safe_open
        except ImportError as error:
            raise RuntimeError("safetensors is required to load H3 weights") from error
        reader = safe_open(self.path, framework="pt", device="cpu")
        reader.__enter__()
        try:
            self._quantization_metadata = parse_quantization_metadata(reader.metadata())
        except ValueError:
            reader.__exit__(None, None, None)
            raise
        self._reader = reader
        self._keys = set(reader.keys())
        return self

    def __exit__(self, *args) -> None:
        if self._reader is not None:
            self._reader.__exit__(*args)
        self._reader = None
        self._keys.clear()
        self._quantization_metadata.clear()

    def _open(self):
        if self._reader is None:
            raise RuntimeError("SafeTensorSource must be used as a context manager")
        return self._reader

    def tensor(self, key: str) -> torch.Tensor:
        return self._open().get_tensor(key)

    def has_tensor(self, key: str) -> bool:
        self._open()
        return key in self._keys

    def quantization_spec(self, prefix: str) -> Mapping[str, object] | None:
        self._open()
        return self._quantization_metadata.get(prefix)


def quant_linear(source: TensorSource, prefix: str, *, device="cuda",
                 output_dtype: torch.dtype | None = None) -> Int8Linear | W4A8Linear:
    """The layer stored under `prefix`, INT8 or W4A8 by its tensor names."""
    if source.has_tensor(f"{prefix}.weight_scale"):
        state = {f"{prefix}.weight": source.tensor(f"{prefix}.weight").to(device),
                 f"{prefix}.weight_scale": source.tensor(f"{prefix}.weight_scale").to(device),
                 f"{prefix}.comfy_quant": source.tensor(f"{prefix}.comfy_quant")}
        return Int8Linear.from_state_dict(state, prefix, output_dtype=output_dtype)
    required = (f"{prefix}.weight_s_rel", f"{prefix}.weight_s_channel")
    if not all(source.has_tensor(key) for key in required):
        raise KeyError(f"quantized layer {prefix!r} is neither ConvRot INT8 nor W4A8")
    raw_spec = source.quantization_spec(prefix)
    spec = W4A8QuantSpec.from_mapping(_DEFAULT_W4A8_SPEC if raw_spec is None else raw_spec)

    def optional(name: str) -> torch.Tensor | None:
        key = f"{prefix}.{name}"
        return source.tensor(key).to(device) if source.has_tensor(key) else None

    return W4A8Linear(source.tensor(f"{prefix}.weight").to(device), source.tensor(f"{prefix}.weight_s_rel").to(device),
                      source.tensor(f"{prefix}.weight_s_channel").to(device), codebook=optional("weight_codebook"),
                      correction=optional("weight_correction"), bias=optional("bias"), spec=spec,
                      output_dtype=output_dtype)


def load_block(index: int, source: TensorSource, *, num_layers: int = H3_NUM_LAYERS, device="cuda",
               head_dim: int = 128, mask: A.MaskConfig | None = None, norm_eps: float = H3_NORM_EPS,
               qk_norm_eps: float = H3_QK_NORM_EPS, group=None) -> DiTBlockB200:
    """Block `index` of a pruned H3 checkpoint as a B200 block (assembly.py:259-333).

    mask: the Sparge selection the attention runs with (None: dense).  The MLP input
    activation is SwiGLU when FC1 has twice FC2's input width (model/layers.py:900-907),
    else tanh-GELU.  RoPE tables come with each forward (`rope_tables_from_frequencies`)."""
    if not 0 <= index < num_layers:
        raise IndexError(index)
    prefix = f"blocks.{index}"
    dev = torch.device(device)

    def vector(name: str) -> torch.Tensor:
        return source.tensor(f"{prefix}.{name}").to(device=dev, dtype=torch.bfloat16).reshape(-1).contiguous()

    qkv = quant_linear(source, f"{prefix}.attn.qkv_proj", device=dev)
    out = quant_linear(source, f"{prefix}.attn.out_proj", device=dev)
    fc1 = quant_linear(source, f"{prefix}.mlp.fc1", device=dev)
    fc2 = quant_linear(source, f"{prefix}.mlp.fc2", device=dev)
    q_norm, k_norm = vector("attn.q_norm.weight"), vector("attn.k_norm.weight")
    norm1, norm2 = vector("norm1.weight"), vector("norm2.weight")
    ada_w = source.tensor(f"{prefix}.adaln_proj.linear.weight").to(device=dev, dtype=torch.bfloat16).contiguous()
    ada_b = vector("adaln_proj.linear.bias")

    hidden = norm1.numel()
    if q_norm.numel() != head_dim:
        raise ValueError(f"q_norm has {q_norm.numel()} entries, the B200 attention needs head_dim {head_dim}")
    if qkv.out_features % (3 * head_dim):
        raise ValueError("qkv_proj rows are not three whole sets of heads")
    heads = qkv.out_features // (3 * head_dim)
    ffn = fc2.in_features
    if fc1.out_features == 2 * ffn:
        act = "swiglu"
    elif fc1.out_features == ffn:
        act = "gelu_tanh"
    else:
        raise ValueError(f"fc1 has {fc1.out_features} rows, fc2 takes {ffn} inputs")
    cfg = BlockConfig(hidden=hidden, heads=heads, head_dim=head_dim, ffn=ffn, mlp_act=act,
                      w4_group=fc1.spec.group_size if isinstance(fc1, W4A8Linear) else 128,
                      convrot=256, eps=norm_eps, qk_eps=qk_norm_eps, t_dim=int(ada_w.shape[1]), mask=mask)
    return DiTBlockB200.from_parts(cfg, ada_w=ada_w, ada_b=ada_b, norm1=norm1, norm2=norm2, q_norm=q_norm,
                                   k_norm=k_norm, qkv=qkv, out=out, fc1=fc1, fc2=fc2, device=dev, group=group)
