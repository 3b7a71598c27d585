"""Packed Ivonar checkpoint container, independent of the reference package.

It reads the reference's packed checkpoint (``format = ivonar_packed_ternary_inference``, schema 1,
``src/ivonar_inference/loader.py:17-18,212-258``) and exposes the same attribute tree the reference
``IvonarModel`` has (``config``, ``blocks[i].mixer_type / mixer_norm / mixer / ffn_norm / ffn``,
``token_io.projection``, ``final_norm``), so ``B200Decoder`` accepts either object. Nothing here does
arithmetic on the token loop; it only holds tensors.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch
from torch import Tensor

PACKED_FORMAT = "ivonar_packed_ternary_inference"
PACKED_SCHEMA_VERSION = 1
TERNARY_GROUP_SIZE = 128

# reference config.py:6-17
REQUIRED_CONTRACT = {
    "architecture": "ivonar_native_ternary",
    "architecture_version": 1,
    "ternary_group_size": 128,
    "ternary_storage": "q2_g128",
    "activation_quantization": "int8_per_token",
    "output_head_type": "tied_ternary_embedding_head",
    "mla_rope_layout": "decoupled_direct_rope",
    "mamba_implementation": "ivonar_mamba3_conv_et_mimo",
    "mamba_variant": "MIMO",
    "tie_embeddings": True,
}


@dataclass(frozen=True)
class ModelConfig:
    """The fields of a checkpoint configuration the token loop needs (reference config.py:21-74)."""

    name: str
    vocab_size: int
    seq_len: int
    hidden_dim: int
    num_layers: int
    num_heads: int
    state_dim: int
    layer_types: tuple[str, ...]
    dense_dim: int
    latent_dim: int
    base_context: int
    final_context: int
    rope_base: float
    longrope_scaling: str

    @classmethod
    def from_payload(cls, config: Any) -> "ModelConfig":
        if not isinstance(config, dict):
            raise ValueError("checkpoint config is invalid")
        mismatches = [f"{k}={config.get(k)!r}" for k, v in REQUIRED_CONTRACT.items() if config.get(k) != v]
        if mismatches:
            raise ValueError("incompatible Ivonar checkpoint: " + ", ".join(mismatches))
        if int(config.get("num_experts", 0)) > 0:
            raise ValueError("mixture-of-experts checkpoints are not supported")
        hidden = int(config["hidden_dim"])
        layers = int(config["num_layers"])
        kinds = tuple(str(k) for k in config.get("layer_types") or ()) or tuple("mamba" for _ in range(layers))
        if len(kinds) != layers or any(k not in {"mamba", "mla"} for k in kinds):
            raise ValueError("layer_types must name mamba or mla for every layer")
        return cls(
            name=str(config.get("name", "")),
            vocab_size=int(config["vocab_size"]),
            seq_len=int(config["seq_len"]),
            hidden_dim=hidden,
            num_layers=layers,
            num_heads=int(config["num_heads"]),
            state_dim=int(config["state_dim"]),
            layer_types=kinds,
            dense_dim=int(config.get("dense_intermediate_dim", 0) or max(int(config.get("intermediate_dim", 0)), 4 * hidden)),
            latent_dim=int(config.get("mla_latent_dim", 0) or max(128, hidden // 4)),
            base_context=int(config.get("base_context", 8192)),
            final_context=int(config.get("final_context", 8192)),
            rope_base=float(config.get("rope_base", 10000.0)),
            longrope_scaling=str(config.get("longrope_scaling", "linear")),
        )


class Ternary:
    """One packed projection: uint8 codes [out, ceil(in/4)], fp16 scales [out, ceil(in/128)], fp32 bias."""

    def __init__(self, packed_weight: Tensor, weight_scales: Tensor, in_features: int, bias: Tensor | None = None,
                 eps: float = 1e-5, group_size: int = TERNARY_GROUP_SIZE) -> None:
        if packed_weight.ndim != 2 or packed_weight.dtype != torch.uint8:
            raise ValueError("packed_weight must be a two-dimensional uint8 tensor")
        self.in_features = int(in_features)
        self.out_features = int(packed_weight.shape[0])
        self.group_size = int(group_size)
        self.eps = float(eps)
        want_packed = (self.out_features, math.ceil(self.in_features / 4))
        want_scales = (self.out_features, math.ceil(self.in_features / self.group_size))
        if tuple(packed_weight.shape) != want_packed:
            raise ValueError(f"invalid packed shape: expected {want_packed}, got {tuple(packed_weight.shape)}")
        if tuple(weight_scales.shape) != want_scales:
            raise ValueError(f"invalid scale shape: expected {want_scales}, got {tuple(weight_scales.shape)}")
        if bias is not None and tuple(bias.shape) != (self.out_features,):
            raise ValueError(f"invalid bias shape: expected ({self.out_features},), got {tuple(bias.shape)}")
        self.packed_weight = packed_weight.contiguous()
        self.weight_scales = weight_scales.contiguous()
        self.bias = None if bias is None else bias.detach().clone().float()

    def to(self, device: torch.device | str) -> "Ternary":
        self.packed_weight = self.packed_weight.to(device)
        self.weight_scales = self.weight_scales.to(device)
        if self.bias is not None:
            self.bias = self.bias.to(device)
        return self


class Norm:
    """RMSNorm parameters (reference layers.py:10-25: eps 1e-6, clip 8)."""

    def __init__(self, weight: Tensor, eps: float = 1e-6, clip: float = 8.0) -> None:
        if weight.ndim != 1:
            raise ValueError("RMSNorm weight must be one-dimensional")
        self.weight = weight.detach().clone().float()
        self.hidden_dim = int(weight.shape[0])
        self.eps = float(eps)
        self.clip = float(clip)


class Rotary:
    """RoPE parameters of the latent attention (reference attention.py:18-72)."""

    def __init__(self, head_dim: int, base_context: int, active_context: int, rope_base: float = 10000.0,
                 scaling_strategy: str = "linear") -> None:
        if head_dim % 2:
            raise ValueError("head_dim must be even for rotary position encoding")
        self.head_dim = int(head_dim)
        self.base_context = int(base_context)
        self.active_context = int(active_context)
        self.rope_base = float(rope_base)
        self.scaling_strategy = scaling_strategy.strip().lower()
        if self.scaling_strategy not in {"linear", "yarn_like", "none"}:
            raise ValueError("Rotary scaling_strategy must be linear, yarn_like, or none")


class RecurrentMixer:
    """SSM mixer parameters (reference recurrent.py:41-105)."""

    def __init__(self, in_proj: Ternary, bc_dt_proj: Ternary, out_proj: Ternary, log_decay: Tensor, theta: Tensor,
                 skip: Tensor, conv_weight: Tensor, conv_bias: Tensor, num_heads: int, state_dim: int,
                 dt_min: float = 1e-3, dt_max: float = 0.1) -> None:
        self.hidden_dim = int(in_proj.in_features)
        self.num_heads = int(num_heads)
        self.state_dim = int(state_dim)
        if self.hidden_dim % self.num_heads:
            raise ValueError("hidden_dim must be divisible by num_heads")
        self.head_dim = self.hidden_dim // self.num_heads
        self.dt_min = float(dt_min)
        self.dt_max = float(dt_max)
        if tuple(log_decay.shape) != (self.num_heads, self.state_dim) or tuple(theta.shape) != (self.num_heads, self.state_dim):
            raise ValueError("log_decay and theta must have shape [num_heads, state_dim]")
        if tuple(skip.shape) != (self.num_heads, self.head_dim):
            raise ValueError("skip must have shape [num_heads, head_dim]")
        if conv_weight.ndim != 3 or conv_weight.shape[0] != self.hidden_dim or conv_weight.shape[1] != 1:
            raise ValueError("conv_weight must have shape [hidden_dim, 1, conv_kernel_size]")
        self.conv_kernel_size = int(conv_weight.shape[2])
        self.in_proj, self.bc_dt_proj, self.out_proj = in_proj, bc_dt_proj, out_proj
        self.log_decay = log_decay.detach().clone().float()
        self.theta = theta.detach().clone().float()
        self.skip = skip.detach().clone().float()
        self.conv_weight = conv_weight.detach().clone().float()
        self.conv_bias = conv_bias.detach().clone().float()


class LatentAttention:
    """Latent (MLA) attention parameters (reference attention.py:75-134)."""

    def __init__(self, q_proj: Ternary, kv_down_proj: Ternary, k_nope_up_proj: Ternary, k_rope_proj: Ternary,
                 v_up_proj: Ternary, out_proj: Ternary, num_heads: int, base_context: int, active_context: int,
                 rope_base: float = 10000.0, scaling_strategy: str = "linear") -> None:
        self.hidden_dim = int(q_proj.in_features)
        self.num_heads = int(num_heads)
        if self.hidden_dim % self.num_heads:
            raise ValueError("hidden_dim must be divisible by num_heads")
        self.head_dim = self.hidden_dim // self.num_heads
        if self.head_dim < 4:
            raise ValueError("head_dim must be at least 4 for MLA decoupled RoPE")
        self.rope_dim = max(2, (self.head_dim // 2) // 2 * 2)
        self.nope_dim = self.head_dim - self.rope_dim
        self.latent_dim = int(kv_down_proj.out_features)
        expected = {
            "q_proj": (q_proj, (self.hidden_dim, self.hidden_dim)),
            "kv_down_proj": (kv_down_proj, (self.hidden_dim, self.latent_dim)),
            "k_nope_up_proj": (k_nope_up_proj, (self.latent_dim, self.num_heads * self.nope_dim)),
            "k_rope_proj": (k_rope_proj, (self.hidden_dim, self.num_heads * self.rope_dim)),
            "v_up_proj": (v_up_proj, (self.latent_dim, self.hidden_dim)),
            "out_proj": (out_proj, (self.hidden_dim, self.hidden_dim)),
        }
        for name, (proj, shape) in expected.items():
            if (proj.in_features, proj.out_features) != shape:
                raise ValueError(f"{name} has shape {(proj.in_features, proj.out_features)}, expected {shape}")
        self.q_proj, self.kv_down_proj, self.k_nope_up_proj = q_proj, kv_down_proj, k_nope_up_proj
        self.k_rope_proj, self.v_up_proj, self.out_proj = k_rope_proj, v_up_proj, out_proj
        self.rope = Rotary(self.rope_dim, base_context, active_context, rope_base, scaling_strategy)


class FeedForward:
    def __init__(self, gate_proj: Ternary, up_proj: Ternary, down_proj: Ternary) -> None:
        self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj


class Block:
    def __init__(self, mixer_type: str, mixer_norm: Norm, mixer, ffn_norm: Norm, ffn: FeedForward) -> None:
        if mixer_type not in {"mamba", "mla"}:
            raise ValueError("layer type must be mamba or mla")
        self.mixer_type, self.mixer_norm, self.mixer, self.ffn_norm, self.ffn = mixer_type, mixer_norm, mixer, ffn_norm, ffn


class TokenHead:
    def __init__(self, projection: Ternary) -> None:
        self.projection = projection
        self.vocab_size = int(projection.out_features)
        self.hidden_dim = int(projection.in_features)


class PackedModel:
    """The whole packed model (same attribute tree as the reference IvonarModel)."""

    def __init__(self, config: ModelConfig, token_io: TokenHead, blocks: list[Block], final_norm: Norm) -> None:
        if len(blocks) != config.num_layers:
            raise ValueError(f"expected {config.num_layers} blocks, got {len(blocks)}")
        self.config, self.token_io, self.blocks, self.final_norm = config, token_io, blocks, final_norm

    @property
    def device(self) -> torch.device:
        return self.token_io.projection.packed_weight.device

    def projections(self) -> list[Ternary]:
        out = [self.token_io.projection]
        for block in self.blocks:
            m = block.mixer
            if block.mixer_type == "mamba":
                out += [m.in_proj, m.bc_dt_proj, m.out_proj]
            else:
                out += [m.q_proj, m.kv_down_proj, m.k_nope_up_proj, m.k_rope_proj, m.v_up_proj, m.out_proj]
            out += [block.ffn.gate_proj, block.ffn.up_proj, block.ffn.down_proj]
        return out


def validate_state(state: dict[str, Tensor]) -> None:
    """Reject malformed packed buffers (reference loader.py:94-112)."""

    for key, value in state.items():
        if not isinstance(value, torch.Tensor):
            raise RuntimeError(f"model_state entry is not a tensor: {key}")
        if key.endswith(".packed_weight"):
            if value.dtype != torch.uint8:
                raise RuntimeError(f"packed ternary buffer must be uint8: {key}")
            flat = value.reshape(-1)
            for start in range(0, flat.numel(), 8 << 20):
                chunk = flat[start : start + (8 << 20)]
                if bool((chunk & (chunk >> 1) & 0x55).any()):
                    raise RuntimeError(f"packed ternary buffer contains the reserved code 3: {key}")
        elif key.endswith(".weight_scales"):
            if value.dtype != torch.float16:
                raise RuntimeError(f"g128 scale buffer must be float16: {key}")
            if value.numel() and not bool(torch.isfinite(value).all()):
                raise RuntimeError(f"g128 scale buffer must contain only finite values: {key}")
            if value.numel() and not bool((value > 0).all()):
                raise RuntimeError(f"g128 scale buffer must contain only positive values: {key}")


def build_model(config: ModelConfig | dict, state: dict[str, Tensor], validate: bool = True) -> PackedModel:
    """Assemble a PackedModel from a packed state dict with the reference key layout (loader.py:146-203)."""

    if isinstance(config, dict):
        config = ModelConfig.from_payload(config)
    if validate:
        validate_state(state)
    used: set[str] = set()

    def take(key: str) -> Tensor:
        if key not in state:
            raise RuntimeError(f"model_state is missing {key}")
        used.add(key)
        return state[key]

    def linear(prefix: str, in_features: int) -> Ternary:
        bias_key = f"{prefix}.bias"
        bias = None
        if bias_key in state:
            used.add(bias_key)
            bias = state[bias_key]
        return Ternary(take(f"{prefix}.packed_weight"), take(f"{prefix}.weight_scales"), in_features, bias=bias)

    hidden = config.hidden_dim
    token_io = TokenHead(linear("token_io.projection", hidden))
    if token_io.vocab_size != config.vocab_size:
        raise RuntimeError(f"token weight has {token_io.vocab_size} rows, config says {config.vocab_size}")
    blocks = []
    for index, kind in enumerate(config.layer_types):
        p = f"blocks.{index}"
        if kind == "mamba":
            mixer = RecurrentMixer(
                linear(f"{p}.mixer.in_proj", hidden), linear(f"{p}.mixer.bc_dt_proj", hidden),
                linear(f"{p}.mixer.out_proj", hidden), take(f"{p}.mixer.log_decay"), take(f"{p}.mixer.theta"),
                take(f"{p}.mixer.skip"), take(f"{p}.mixer.conv_weight"), take(f"{p}.mixer.conv_bias"),
                num_heads=config.num_heads, state_dim=config.state_dim,
            )
        else:
            mixer = LatentAttention(
                linear(f"{p}.mixer.q_proj", hidden), linear(f"{p}.mixer.kv_down_proj", hidden),
                linear(f"{p}.mixer.k_nope_up_proj", config.latent_dim), linear(f"{p}.mixer.k_rope_proj", hidden),
                linear(f"{p}.mixer.v_up_proj", config.latent_dim), linear(f"{p}.mixer.out_proj", hidden),
                num_heads=config.num_heads, base_context=config.base_context, active_context=config.seq_len,
                rope_base=config.rope_base, scaling_strategy=config.longrope_scaling,
            )
        ffn = FeedForward(linear(f"{p}.ffn.gate_proj", hidden), linear(f"{p}.ffn.up_proj", hidden),
                          linear(f"{p}.ffn.down_proj", config.dense_dim))
        blocks.append(Block(kind, Norm(take(f"{p}.mixer_norm.weight")), mixer, Norm(take(f"{p}.ffn_norm.weight")), ffn))
    final_norm = Norm(take("final_norm.weight"))
    unused = sorted(set(state) - used)
    if unused:
        raise RuntimeError(f"model_state has entries the model does not use: {', '.join(unused[:5])}")
    return PackedModel(config, token_io, blocks, final_norm)


def load_checkpoint(path: str | Path) -> PackedModel:
    """Read a packed checkpoint file (reference loader.py:212-258, without the tokenizer check)."""

    payload = torch.load(Path(path), map_location="cpu", weights_only=True)
    if not isinstance(payload, dict):
        raise RuntimeError(f"invalid Ivonar checkpoint: {path}")
    if payload.get("format") != PACKED_FORMAT or payload.get("schema_version") != PACKED_SCHEMA_VERSION:
        raise RuntimeError(f"unsupported checkpoint format; expected {PACKED_FORMAT} schema {PACKED_SCHEMA_VERSION}")
    state = payload.get("model_state")
    if not isinstance(state, dict):
        raise RuntimeError("checkpoint model_state is invalid")
    return build_model(ModelConfig.from_payload(payload.get("config")), state)


def rope_table(rotary, max_len: int) -> Tensor:
    """[max_len, rope_dim/2, 2] (cos, sin) of the rotary of one attention layer, fp32 on the CPU.

    Same positions and frequencies as reference attention.py:39-72 (linear / yarn_like / none).
    """

    dim = int(rotary.head_dim)
    inv_freq = 1.0 / (float(rotary.rope_base) ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    positions = torch.arange(0, max_len, dtype=torch.float32)
    base, active = int(rotary.base_context), int(rotary.active_context)
    ratio = active / base if active > base else 1.0
    strategy = str(rotary.scaling_strategy)
    if strategy == "linear" and ratio > 1.0:
        positions = positions / ratio
    if strategy == "yarn_like" and ratio > 1.0:
        ramp = torch.linspace(0.0, 1.0, steps=inv_freq.numel())
        inv_freq = inv_freq / (1.0 + (ratio - 1.0) * ramp.square())
    freqs = torch.einsum("s,d->sd", positions, inv_freq)
    return torch.stack((freqs.cos(), freqs.sin()), dim=-1).contiguous()
