"""Checkpoint ingest fast path (ingest.load_model) against the reference's load_model: the same model
tensors bit for bit, the same decoder outputs, and the reference's errors for corrupted checkpoints."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref_module(name: str):
    from ivonar_inference_b200 import _reference

    return _reference.module(name)


def _write_checkpoint(path, payload: dict, state: dict) -> None:
    loader = _ref_module("loader")
    torch.save({"format": loader.PACKED_FORMAT, "schema_version": loader.PACKED_SCHEMA_VERSION, "config": payload,
                "model_state": state, "tokenizer_sha256": "0" * 64, "step": 7}, path)


def _reference_error(path) -> str:
    loader = _ref_module("loader")
    with pytest.raises(RuntimeError) as info:
        loader.load_model(path, "cpu", materialize=False)
    return str(info.value)


def test_ingest_matches_the_reference_loader(tmp_path) -> None:
    from ivonar_inference_b200 import B200Decoder, ingest, synthetic

    payload = synthetic.config0(seq_len=64)
    state = synthetic.synthetic_state(payload, 3)
    path = tmp_path / "model.pt"
    _write_checkpoint(path, payload, state)
    ref = _ref_module("loader").load_model(path, "cpu", materialize=False)
    ours = ingest.load_model(path, "cuda", materialize=False)
    assert ours.step == 7 and ours.tokenizer_sha256 == "0" * 64 and ours.config == ref.config
    ref_state, our_state = ref.model.state_dict(), ours.model.state_dict()
    assert set(ref_state) == set(our_state)
    for key, value in ref_state.items():
        got = our_state[key]
        assert got.device.type == "cuda", key
        assert value.dtype == got.dtype and torch.equal(value, got.cpu()), key
    # materialised (the reference's default): the unpacked weights match the reference's on the GPU
    ref_m = _ref_module("loader").load_model(path, "cuda").model.state_dict()
    ours_m = ingest.load_model(path, "cuda").model.state_dict()
    assert set(ref_m) == set(ours_m)
    for key, value in ref_m.items():
        assert value.dtype == ours_m[key].dtype and torch.equal(value, ours_m[key]), key
    # the decoder bound to either model computes the same logits
    prompt = synthetic.random_prompt(int(payload["vocab_size"]), 12, seed=1)
    a = B200Decoder(ref.model, max_len=64, device="cuda")
    b = B200Decoder(ours.model, max_len=64, device="cuda")
    assert torch.equal(a.prefill(prompt), b.prefill(prompt))
    for tok in (5, 17, 3):
        assert torch.equal(a.step(torch.tensor([tok])), b.step(torch.tensor([tok])))


def test_ingest_of_an_archive_the_direct_reader_hands_to_torch_load(tmp_path) -> None:
    """An entry saved as a Parameter (a global the direct reader leaves to torch.load): the memory-mapped
    load and one-block copy give the reference's model all the same."""
    from ivonar_inference_b200 import ingest, synthetic

    payload = synthetic.config0(seq_len=64)
    state = synthetic.synthetic_state(payload, 5)
    state["final_norm.weight"] = torch.nn.Parameter(state["final_norm.weight"], requires_grad=False)
    path = tmp_path / "model.pt"
    _write_checkpoint(path, payload, state)
    assert ingest._read_archive(path, torch.device("cuda")) is None
    ref = _ref_module("loader").load_model(path, "cpu", materialize=False).model.state_dict()
    ours = ingest.load_model(path, "cuda", materialize=False).model.state_dict()
    assert set(ref) == set(ours)
    for key, value in ref.items():
        assert ours[key].device.type == "cuda" and torch.equal(value, ours[key].cpu()), key


@pytest.mark.parametrize("damage", ["code3", "nan_scale", "zero_scale", "negative_scale", "dtype"])
def test_ingest_reports_the_reference_errors(tmp_path, damage: str) -> None:
    from ivonar_inference_b200 import ingest, synthetic

    payload = synthetic.config0(seq_len=64)
    state = synthetic.synthetic_state(payload, 4)
    packed = [k for k in state if k.endswith(".packed_weight")]
    scales = [k for k in state if k.endswith(".weight_scales")]
    if damage == "code3":
        key = packed[len(packed) // 2]
        state[key] = state[key].clone()
        state[key].view(-1)[1234 % state[key].numel()] = 0b00110100  # field 2 holds the reserved code 3
    elif damage == "dtype":
        key = scales[3]
        state[key] = state[key].float()
    else:
        key = scales[len(scales) // 2]
        state[key] = state[key].clone()
        state[key].view(-1)[5] = {"nan_scale": float("nan"), "zero_scale": 0.0, "negative_scale": -0.5}[damage]
        # a later buffer broken too: the first one in the reference's order is reported
        late = scales[-1]
        state[late] = state[late].clone()
        state[late].view(-1)[0] = 0.0
    path = tmp_path / "model.pt"
    _write_checkpoint(path, payload, state)
    expected = _reference_error(path)
    with pytest.raises(RuntimeError) as info:
        ingest.load_model(path, "cuda", materialize=False)
    assert str(info.value) == expected
    assert key in expected
