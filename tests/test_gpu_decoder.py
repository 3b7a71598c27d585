"""B200Decoder (persistent sm_100a decode kernel) against the CPU oracle and the reference goldens."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu


def _model(payload, seed=0, style="baseline"):
    from ivonar_inference_b200 import synthetic

    return synthetic.synthetic_model(payload, seed, style)


def _first_difference(a, b) -> int:
    return next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), min(len(a), len(b)))


@pytest.mark.parametrize("name", ["model_config0", "model_tiny"])
def test_decoder_matches_the_oracle_and_the_reference(oracle_lib, name: str) -> None:
    from ivonar_inference_b200 import B200Decoder, synthetic

    g = golden(name)
    payload = synthetic.config0() if name == "model_config0" else synthetic.tiny(seq_len=64)
    style = "baseline" if name == "model_config0" else "reference_tests"
    model = _model(payload, int(g["seed"]), style)
    dec = B200Decoder(model, device="cuda", sampling=True)
    ora = oracle_lib.OracleDecoder(model)
    prompt = torch.from_numpy(g["prompt"]).view(1, -1)
    gpu = dec.prefill(prompt)[0].cpu().numpy()
    cpu = ora.prefill(g["prompt"]).copy()
    assert float(np.abs(gpu - cpu).max()) < 0.02
    assert float(np.abs(gpu - g["prefill_logits"]).max()) < 0.05
    assert dec.host_position == len(g["prompt"]) and int(dec.position) == len(g["prompt"])
    # teacher forcing along the reference's penalized greedy stream
    stream = g["torch_greedy_rp"]
    worst_oracle = worst_ref = 0.0
    for i, tok in enumerate(stream[:-1]):
        out = dec.step(torch.tensor([int(tok)]))[0].cpu().numpy()
        ref = ora.step(int(tok))
        worst_oracle = max(worst_oracle, float(np.abs(out - ref).max()))
        worst_ref = max(worst_ref, float(np.abs(out - g["torch_greedy_rp_step_logits"][i]).max()))
    assert worst_oracle < 0.02 and worst_ref < 0.05
    # free-running penalized greedy: the reference's tokens
    dec.prefill(prompt)
    dec.configure_sampling(temperature=1.0, top_k=1, repetition_penalty=4.0)
    tokens = [dec.sample()] + dec.advance_many(len(stream) - 1)
    assert tokens == stream.tolist()


@pytest.mark.parametrize("layers", [("mamba",), ("mla",), ("mla", "mamba")])
def test_nano_width_blocks_match_the_oracle_closely(oracle_lib, layers) -> None:
    # One or two blocks at the Nano width (d 1024, 16x64 heads, latent 256, F 2816, vocab 32768):
    # little room for quantisation flips to compound, so any kernel error would stand out.
    from ivonar_inference_b200 import B200Decoder, synthetic

    payload = synthetic.config_payload("NANO_SLICE", 32768, 1024, list(layers), 16, 16, 256, 2816, 512)
    model = _model(payload, 9)
    dec = B200Decoder(model, device="cuda", max_len=128)
    ora = oracle_lib.OracleDecoder(model, max_len=128)
    prompt = synthetic.random_prompt(32768, 40, seed=9)
    gpu = dec.prefill(prompt)[0].cpu().numpy()
    cpu = ora.prefill(prompt[0].numpy()).copy()
    diff = np.abs(gpu - cpu)
    print(f"{layers}: max {diff.max():.2e} mean {diff.mean():.2e} logit std {cpu.std():.3f}")
    # Identical codes give identical logits (a lone mamba block prefilled bit-identically); an
    # activation code on the other side of a rounding boundary moves every logit by ~1e-3; the
    # reference's own fp16-KV GPU arithmetic differs from its fp32-KV CPU arithmetic on one such
    # attention block by 0.009-0.013 mean / 0.05-0.08 max |dlogit|. A kernel error would move the
    # logits by their own scale (std ~0.54). Bound: twice the reference spread.
    assert float(diff.mean()) < 0.025 and float(diff.max()) < 0.16
    for t in prompt[0, :8].tolist():
        out = dec.step(torch.tensor([t]))[0].cpu().numpy()
        ref = ora.step(t)
        assert float(np.abs(out - ref).mean()) < 0.025 and float(np.abs(out - ref).max()) < 0.16


def test_nano_decoder_matches_the_oracle(oracle_lib) -> None:
    from ivonar_inference_b200 import B200Decoder, synthetic

    g = golden("model_config1")
    model = _model(synthetic.config1(seq_len=2048), 0)
    dec = B200Decoder(model, max_len=256, device="cuda", sampling=True)
    ora = oracle_lib.OracleDecoder(model, max_len=256)
    prompt = torch.from_numpy(g["prompt"]).view(1, -1)
    gpu = dec.prefill(prompt)[0].cpu().numpy()
    cpu = ora.prefill(g["prompt"]).copy()
    diff = np.abs(gpu - cpu)
    # 24 quantised blocks amplify rounding-order differences chaotically; the reference's own torch
    # and numba paths differ by 0.21 max / 0.033 mean on this model, which is the bar here.
    assert float(diff.max()) < 0.25 and float(diff.mean()) < 0.04, (float(diff.max()), float(diff.mean()))
    # The argmax itself may land on either side of a near-tie (on this prompt the oracle's two leading
    # logits are 0.008 apart): the GPU's pick must be within the same spread of the oracle's maximum.
    assert float(cpu.max() - cpu[int(gpu.argmax())]) < 0.25
    dec.configure_sampling(1.0, 1, 1.0)
    tokens = [dec.sample()] + dec.advance_many(47)
    # Every greedy token of the GPU must be a near-argmax of the oracle's logits when the oracle is
    # teacher-forced along the GPU's own stream (streams may split at near-ties, as the reference's
    # own torch and numba paths do after 8 tokens on this model).
    worst_gap = 0.0
    gaps = []
    logits = cpu
    for i, tok in enumerate(tokens):
        gap = float(logits.max() - logits[tok])
        gaps.append(gap)
        worst_gap = max(worst_gap, gap)
        if i + 1 < len(tokens):
            logits = ora.step(tok)
    agree = _first_difference(tokens, g["numba_stepped_greedy"].tolist())
    print(f"nano greedy: agreement with reference numba {agree}/48, worst oracle gap {worst_gap:.3e}, "
          f"exact argmax {sum(x == 0.0 for x in gaps)}/48")
    stats = (agree, worst_gap, sum(x == 0.0 for x in gaps))
    # bound: the reference's own torch/numba logit spread on this model (0.21 max)
    assert worst_gap < 0.25, stats
    # most picks are the oracle's exact argmax; the rest are near-ties inside the bound above. The count
    # moves with the prefill's fp32 order (tensor-core prefill vs oracle: max 0.219 / mean 0.036, the
    # token-by-token prefill: max 0.202 / mean 0.033), so it is held to two thirds of the stream.
    assert sum(x == 0.0 for x in gaps) >= 32, stats


def test_sampled_stream_matches_the_oracle_with_the_same_seed(oracle_lib) -> None:
    from ivonar_inference_b200 import B200Decoder, synthetic

    model = _model(synthetic.config0(), 3)
    dec = B200Decoder(model, device="cuda", sampling=True, seed=1234)
    ora = oracle_lib.OracleDecoder(model, seed=1234)
    prompt = synthetic.random_prompt(512, 16, seed=3)
    dec.prefill(prompt)
    ora.prefill(prompt[0].numpy())
    dec.configure_sampling(0.5, 40, 1.15)
    ora.configure_sampling(0.5, 40, 1.15)
    tokens = [dec.sample()] + dec.advance_many(31)
    ref = [ora.sample()]
    ref += ora.generate(ref[0], 31)
    assert _first_difference(tokens, ref) >= 16, (tokens, ref)
    assert int(dec.rng[1]) == 32


def test_bursts_produce_the_same_tokens_as_single_steps() -> None:
    from ivonar_inference_b200 import B200Decoder, synthetic
    from ivonar_inference_b200.decoder import BURST

    model = _model(synthetic.tiny(seq_len=64), 21, "reference_tests")
    dec = B200Decoder(model, device="cuda", sampling=True, seed=5)
    assert dec.capture()
    assert dec.burst_size == BURST
    prompt = torch.tensor([[5, 9, 14, 3]])
    runs = []
    for bursts in (True, False):
        dec.prefill(prompt)
        dec.configure_sampling(temperature=1.0, top_k=1, repetition_penalty=50.0)
        first = dec.sample()
        rest = dec.advance_many(2 * BURST + 3) if bursts else [dec.advance() for _ in range(2 * BURST + 3)]
        runs.append([first, *rest])
        assert dec.host_position == 4 + 2 * BURST + 3
    assert runs[0] == runs[1]
    assert len(set(runs[0])) > 1


def test_graph_replay_matches_eager_steps() -> None:
    from ivonar_inference_b200 import B200Decoder, synthetic

    model = _model(synthetic.config0(), 4)
    dec = B200Decoder(model, device="cuda")
    assert dec.graph is None and dec.attention_lengths == (dec.max_len,)
    ids = synthetic.random_prompt(512, 20, seed=4)[0].tolist()
    def run():
        out = [dec.prefill(torch.tensor([ids[:8]]))[0].cpu().clone()]
        for t in ids[8:]:
            out.append(dec.step(torch.tensor([t]))[0].cpu().clone())
        return torch.stack(out)
    eager = run()
    assert dec.capture() is True
    assert set(dec.graphs) == {dec.max_len}
    replayed = run()
    assert torch.equal(eager, replayed)


def test_capacity_and_input_errors() -> None:
    from ivonar_inference_b200 import B200Decoder, synthetic

    model = _model(synthetic.tiny(), 5, "reference_tests")
    dec = B200Decoder(model, max_len=8, device="cuda", sampling=True)
    with pytest.raises(ValueError, match="capacity"):
        dec.prefill(torch.randint(2, 300, (1, 9)))
    with pytest.raises(IndexError):
        dec.prefill(torch.tensor([[1, 2, 300]]))
    dec.prefill(torch.randint(2, 300, (1, 6)))
    dec.configure_sampling(1.0, 4, 1.0)
    dec.sample()
    tokens = dec.advance_many(2)
    assert len(tokens) == 2 and dec.host_position == 8
    with pytest.raises(ValueError, match="no free position"):
        dec.advance()
    with pytest.raises(RuntimeError):
        B200Decoder(model, max_len=8, device="cuda").sample()
    with pytest.raises(ValueError):
        dec.configure_sampling(0.0, 4, 1.0)


def test_self_check_and_build_decoder() -> None:
    from ivonar_inference_b200 import B200Decoder, build_decoder, synthetic

    model = _model(synthetic.config0(), 6)
    decoder, backend, note = build_decoder(model, "cuda", sampling=True)
    assert isinstance(decoder, B200Decoder) and backend == "ternary" and note is None
    assert int(decoder.position) == 0 and decoder.host_position == 0
