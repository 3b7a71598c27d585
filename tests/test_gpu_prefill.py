"""Tensor-core prompt prefill (ivb_decoder_prefill) against the token-by-token decode path on a B200."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import check_greedy_stream, golden

pytestmark = pytest.mark.gpu


def _model(payload, seed=0, style="baseline"):
    from ivonar_inference_b200 import synthetic

    return synthetic.synthetic_model(payload, seed, style)


@pytest.mark.parametrize("name", ["model_config0", "model_tiny"])
def test_gemm_prefill_matches_the_step_prefill_and_the_oracle(oracle_lib, name: str) -> None:
    from ivonar_inference_b200 import B200Decoder, synthetic

    g = golden(name)
    seq_len = int(g["seq_len"])
    payload = synthetic.config0(seq_len=seq_len) if name == "model_config0" else synthetic.tiny(seq_len=seq_len)
    model = _model(payload, int(g["seed"]), "baseline" if name == "model_config0" else "reference_tests")
    prompt = torch.from_numpy(g["prompt"]).view(1, -1)
    fast = B200Decoder(model, device="cuda", sampling=True)
    slow = B200Decoder(model, device="cuda", sampling=True, prefill="steps")
    a = fast.prefill(prompt)[0].cpu().numpy()
    b = slow.prefill(prompt)[0].cpu().numpy()
    ref = oracle_lib.OracleDecoder(model).prefill(g["prompt"]).copy()
    # same arithmetic up to fp32 accumulation order (per 128-group vs per 64-chunk) and the fp16 rounding
    # of the current position's k_rope: the decoder-vs-oracle bar of the decode tests
    assert float(np.abs(a - b).max()) < 0.02
    assert float(np.abs(a - ref).max()) < 0.02
    assert fast.host_position == slow.host_position == len(g["prompt"])
    assert int(fast.position) == int(slow.position) and int(fast.token) == int(prompt[0, -1])
    # decoding continues from the prefilled caches and state: the reference's 256-token penalised greedy
    # stream (identical, or parting only at a near-tie of the reference's scores, as in the decode tests)
    stream = g["torch_greedy_rp"]
    fast.configure_sampling(temperature=1.0, top_k=1, repetition_penalty=4.0)
    tokens = [fast.sample()] + fast.advance_many(len(stream) - 1)
    check_greedy_stream(tokens, stream, g["prefill_logits"], g["torch_greedy_rp_step_logits"], 4.0, 0.1)


def test_chunked_prefill_equals_one_call() -> None:
    from ivonar_inference_b200 import B200Decoder, synthetic

    model = _model(synthetic.config0(), 4)
    prompt = synthetic.random_prompt(512, 45, seed=4)
    whole = B200Decoder(model, device="cuda")
    parts = B200Decoder(model, device="cuda", prefill_chunk=7)
    a = whole.prefill(prompt)[0].cpu().numpy()
    b = parts.prefill(prompt)[0].cpu().numpy()
    # every token row is computed the same way whatever the chunking (caches and state carry over)
    assert float(np.abs(a - b).max()) < 1e-5
    for t in (3, 17, 250):
        x = whole.step(torch.tensor([t]))[0].cpu().numpy()
        y = parts.step(torch.tensor([t]))[0].cpu().numpy()
        assert float(np.abs(x - y).max()) < 1e-5


def test_nano_prefill_matches_the_oracle(oracle_lib) -> None:
    from ivonar_inference_b200 import B200Decoder, synthetic

    g = golden("model_config1")
    model = _model(synthetic.config1(seq_len=2048), 0)
    dec = B200Decoder(model, max_len=256, device="cuda")
    gpu = dec.prefill(torch.from_numpy(g["prompt"]).view(1, -1))[0].cpu().numpy()
    cpu = oracle_lib.OracleDecoder(model, max_len=256).prefill(g["prompt"]).copy()
    diff = np.abs(gpu - cpu)
    # the reference's own torch and numba paths differ by 0.21 max / 0.033 mean on this model
    assert float(diff.max()) < 0.25 and float(diff.mean()) < 0.04, (float(diff.max()), float(diff.mean()))
