"""The algorithmic byte counts behind bench.py's roofline figures, recomputed from the model's own tensors
and shapes on the CPU: what one decode token must read (every packed byte, scale and bias once, the
recurrent state read and written, the key/value cache up to its position plus the append)."""

from __future__ import annotations

import sys

import torch

from conftest import ROOT


def _bench():
    if str(ROOT) not in sys.path:
        sys.path.insert(0, str(ROOT))
    import bench

    return bench


def test_decode_bytes_of_config1() -> None:
    from ivonar_inference_b200 import synthetic

    bench = _bench()
    model = synthetic.synthetic_model(synthetic.config1(seq_len=320), 0)
    total, parts = bench.decode_bytes(model, 36, 256)
    state = model.state_dict()
    weights = sum(t.numel() for k, t in state.items() if k.endswith(".packed_weight"))
    weights += sum(2 * t.numel() for k, t in state.items() if k.endswith(".weight_scales"))
    weights += sum(4 * t.numel() for k, t in state.items() if k.endswith(".bias"))
    assert parts["weights_per_token"] == weights == 88_072_192
    mla = [b for b in model.blocks if b.mixer_type != "mamba"]
    assert len(mla) == 12 and mla[0].mixer.num_heads == 16 and mla[0].mixer.head_dim == 64
    # fp32 key and value rows of 16 heads x 64 dims per position per attention layer
    assert parts["kv_bytes_per_position"] == 12 * 16 * 2 * 64 * 4 == 98_304
    # recurrent state, fp32, read and written every token: per mamba block the heads x state x head_dim
    # state in two components (ssm_state), the previous step's input term of one component (prev_force)
    # and the conv tail of (kernel - 1) inputs per channel (conv_state)
    mamba = [b.mixer for b in model.blocks if b.mixer_type == "mamba"]
    hsd = mamba[0].num_heads * mamba[0].state_dim * mamba[0].head_dim
    assert len(mamba) == 12 and hsd == 16 * 16 * 64 and mamba[0].conv_kernel_size == 4
    assert parts["state_per_token"] == 12 * 2 * 4 * (3 * hsd + 1024 * 3) == 5_013_504
    # 256 tokens at positions 36..291: each reads the cache up to and including its own position and
    # appends one row
    attended = sum(p + 1 for p in range(36, 36 + 256)) + 256
    assert total == 256 * (weights + 5_013_504) + 98_304 * attended


def test_batched_roofline_counts_weights_once_per_step() -> None:
    from ivonar_inference_b200 import synthetic

    bench = _bench()
    model = synthetic.synthetic_model(synthetic.config1(seq_len=320), 0)
    _, parts = bench.decode_bytes(model, 128, 1, cache="latent")
    one = bench.batch_roofline(model, 1, 128, 10, 1.0)
    many = bench.batch_roofline(model, 256, 128, 10, 1.0)
    # 255 more sequences add their state and cache, not the weights
    per_seq = 10 * parts["state_per_token"] + sum(parts["kv_bytes_per_position"] * (p + 2) for p in range(128, 138))
    assert many["bytes_per_gpu"] - one["bytes_per_gpu"] == 255 * per_seq
    assert one["bytes_per_gpu"] == 10 * parts["weights_per_token"] + per_seq
    assert torch.isclose(torch.tensor(many["achieved"]), torch.tensor(many["bytes_per_gpu"] / 1e-3 / 1e9))
