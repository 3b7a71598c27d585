"""Seeded synthetic Ivonar models with the benchmark's weight distributions.

There is no public checkpoint in this environment, so tests and benchmarks use random-init models
of the named shapes, built as packed state dicts with the reference key layout (the layout
``src/ivonar_inference/loader.py:146-203`` reads). Distributions:
  codes: P(value 0) = 0.4, P(-1) = P(+1) = 0.3; fp16 group scales exp(N(log 0.02, 0.3));
  norm weights 1 + 0.1 N; biases N(0, 0.02) on every projection except the tied head;
  SSM constants as the reference tests build them (tests/conftest.py:88-94).
``style="reference_tests"`` reproduces the reference test distribution instead (uniform codes,
scales U(0.01, 0.06)). Generation uses one CPU torch.Generator, so a (config, seed) pair gives
the same bytes on every machine with the same torch build. The models are the reference's own
``IvonarModel`` objects: the payload is parsed by the reference's ``ModelConfig.from_payload`` and the
state dict assembled (and validated) by its ``build_model`` (src/ivonar_inference/config.py:39,
loader.py:146).
"""

from __future__ import annotations

import math

import torch

from . import _reference

# The checkpoint contract every Ivonar packed checkpoint declares (the keys and values the reference
# loader requires, src/ivonar_inference/config.py:6-17): a format, restated here as data only.
CONTRACT = {
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


def config_payload(name: str, vocab: int, hidden: int, layers: list[str], heads: int, state_dim: int, latent: int,
                   dense: int, seq_len: int) -> dict:
    return {
        **CONTRACT,
        "name": name,
        "vocab_size": vocab,
        "seq_len": seq_len,
        "hidden_dim": hidden,
        "num_layers": len(layers),
        "num_heads": heads,
        "state_dim": state_dim,
        "layer_types": list(layers),
        "dense_intermediate_dim": dense,
        "mla_latent_dim": latent,
        "base_context": seq_len,
        "final_context": seq_len,
        "num_experts": 0,
    }


def config0(seq_len: int = 64) -> dict:
    """Benchmark config 0: tiny CPU-runnable hybrid (vocab 512, d 128, 4 blocks)."""
    return config_payload("CONFIG0", 512, 128, ["mamba", "mla"] * 2, 4, 16, 64, 384, seq_len)


def config1(seq_len: int = 8192) -> dict:
    """Benchmark config 1/2/3: Nano-shaped (vocab 32768, d 1024, 24 blocks, 16x64 heads, latent 256, F 2816)."""
    return config_payload("NANO", 32768, 1024, ["mamba", "mla"] * 12, 16, 16, 256, 2816, seq_len)


def config4(seq_len: int = 2048) -> dict:
    """Benchmark config 4: 7B-shaped (vocab 32768, d 4096, 32 blocks, 32x128 heads, latent 512, F 11008)."""
    return config_payload("SEVEN_B", 32768, 4096, ["mamba", "mla"] * 16, 32, 16, 512, 11008, seq_len)


def tiny(hidden: int = 16, heads: int = 4, state_dim: int = 3, latent: int = 8, dense: int = 32, vocab: int = 300,
         seq_len: int = 32, layers: tuple[str, ...] = ("mamba", "mla", "mamba")) -> dict:
    """The reference test shapes (tests/conftest.py:34-52, tests/test_kernels.py:23-41)."""
    return config_payload("TINY", vocab, hidden, list(layers), heads, state_dim, latent, dense, seq_len)


def _codes(gen: torch.Generator, rows: int, cols: int, style: str) -> torch.Tensor:
    if style == "reference_tests":
        return torch.randint(0, 3, (rows, cols), generator=gen, dtype=torch.uint8)
    if style == "fast":  # the same code distribution, drawn on the generator's device
        r = torch.randint(0, 10, (rows, cols), generator=gen, dtype=torch.uint8, device=gen.device)
        return (r >= 3).to(torch.uint8) + (r >= 7).to(torch.uint8)
    r = torch.rand(rows, cols, generator=gen)
    return (r >= 0.3).to(torch.uint8) + (r >= 0.7).to(torch.uint8)


def _packed(gen: torch.Generator, rows: int, cols: int, style: str) -> tuple[torch.Tensor, torch.Tensor]:
    width = math.ceil(cols / 4)
    codes = _codes(gen, rows, width * 4, style).view(rows, width, 4)
    packed = codes[..., 0] | (codes[..., 1] << 2) | (codes[..., 2] << 4) | (codes[..., 3] << 6)
    groups = math.ceil(cols / 128)
    if style == "reference_tests":
        scales = (torch.rand(rows, groups, generator=gen) * 0.05 + 0.01).half()
    else:
        scales = torch.exp(math.log(0.02) + 0.3 * torch.randn(rows, groups, generator=gen, device=gen.device)).half()
    return packed.contiguous().cpu(), scales.cpu()


def synthetic_state(payload: dict, seed: int = 0, style: str = "baseline") -> dict[str, torch.Tensor]:
    """A packed state dict for ``payload`` (see the module docstring for the distributions)."""

    config = _reference.module("config").ModelConfig.from_payload(payload)
    gen = torch.Generator().manual_seed(int(seed))
    # "fast": the packed matrices are drawn on the GPU when there is one (the 7B-shaped model in seconds)
    big = gen
    if style == "fast" and torch.cuda.is_available():
        big = torch.Generator(device="cuda").manual_seed(int(seed))
    state: dict[str, torch.Tensor] = {}

    def linear(prefix: str, rows: int, cols: int, bias: bool = True) -> None:
        packed, scales = _packed(big, rows, cols, style)
        state[f"{prefix}.packed_weight"] = packed
        state[f"{prefix}.weight_scales"] = scales
        if bias:
            state[f"{prefix}.bias"] = torch.randn(rows, generator=gen) * 0.02

    d, h, s = config.hidden_dim, config.num_heads, config.state_dim
    hd = d // h
    linear("token_io.projection", config.vocab_size, d, bias=False)
    for index, kind in enumerate(config.layer_types):
        p = f"blocks.{index}"
        state[f"{p}.mixer_norm.weight"] = 1.0 + 0.1 * torch.randn(d, generator=gen)
        state[f"{p}.ffn_norm.weight"] = 1.0 + 0.1 * torch.randn(d, generator=gen)
        if kind == "mamba":
            linear(f"{p}.mixer.in_proj", 2 * d, d)
            linear(f"{p}.mixer.bc_dt_proj", 3 * h * s, d)
            linear(f"{p}.mixer.out_proj", d, d)
            state[f"{p}.mixer.log_decay"] = torch.rand(h, s, generator=gen) * 0.5 - 1.0
            state[f"{p}.mixer.theta"] = torch.rand(h, s, generator=gen) * math.pi
            state[f"{p}.mixer.skip"] = 1.0 + 0.1 * torch.randn(h, hd, generator=gen)
            conv = 0.1 * torch.randn(d, 1, 4, generator=gen)
            conv[:, :, -1] += 1.0
            state[f"{p}.mixer.conv_weight"] = conv
            state[f"{p}.mixer.conv_bias"] = 0.01 * torch.randn(d, generator=gen)
        else:
            rope = max(2, (hd // 2) // 2 * 2)
            nope = hd - rope
            linear(f"{p}.mixer.q_proj", d, d)
            linear(f"{p}.mixer.kv_down_proj", config.latent_dim, d)
            linear(f"{p}.mixer.k_nope_up_proj", h * nope, config.latent_dim)
            linear(f"{p}.mixer.k_rope_proj", h * rope, d)
            linear(f"{p}.mixer.v_up_proj", d, config.latent_dim)
            linear(f"{p}.mixer.out_proj", d, d)
        linear(f"{p}.ffn.gate_proj", config.dense_dim, d)
        linear(f"{p}.ffn.up_proj", config.dense_dim, d)
        linear(f"{p}.ffn.down_proj", d, config.dense_dim)
    state["final_norm.weight"] = 1.0 + 0.1 * torch.randn(d, generator=gen)
    return state


def synthetic_model(payload: dict, seed: int = 0, style: str = "baseline"):
    """The reference ``IvonarModel`` of ``payload`` with the synthetic weights (on the CPU)."""

    config = _reference.module("config").ModelConfig.from_payload(payload)
    model = _reference.module("loader").build_model(config, synthetic_state(payload, seed, style))
    return model.eval()


def random_prompt(vocab: int, length: int, seed: int = 0, low: int = 0) -> torch.Tensor:
    """Seeded uniform token ids [1, length] (int64)."""
    gen = torch.Generator().manual_seed(int(seed))
    return torch.randint(low, vocab, (1, length), generator=gen, dtype=torch.int64)
