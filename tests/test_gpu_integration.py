"""B200Decoder behind the reference's own callers: Engine.load, stream_text, check_decoder and run_benchmark.

The reference package (installed unmodified under baseline/_ref) is imported as is. The only change is
the one binding a maintainer adds: the reference's CUDA slot ``decoder._kernel_decoder`` points at
``ivonar_inference_b200.decoder.kernel_decoder``. Everything else (checkpoint loading, tokenizer, prompt
rendering, sampling settings, graph capture, streaming, verification, the benchmark) is reference code.
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(name: str):
    from ivonar_inference_b200 import _reference

    return _reference.module(name)


def _tokenizer_file(path: Path, vocab: int) -> Path:
    """A byte-level tokenizer (no merges) whose vocabulary fills `vocab` ids: the reserved tokens, the
    256 bytes, then two-letter pieces, so that any sampled id decodes."""
    tokenizer = _ref("tokenizer").TernaryTokenizer()
    pieces = {idx: list(value) for idx, value in tokenizer.vocab.items()}
    letters = b"abcdefghijklmnopqrstuvwxyz"
    for extra, idx in enumerate(range(tokenizer.next_id, vocab)):
        pieces[idx] = [letters[extra % 26], letters[(extra // 26) % 26]]
    payload = {"format": "ivonar_tokenizer_v1", "backend": "python_byte_bpe", "special_tokens": tokenizer.special_tokens,
               "vocab": {str(idx): value for idx, value in sorted(pieces.items())}, "merges": [], "next_id": vocab}
    path.write_text(json.dumps(payload), encoding="utf-8")
    return path


def _checkpoint(path: Path, payload: dict, tokenizer_file: Path, seed: int) -> Path:
    from ivonar_inference_b200 import synthetic

    loader = _ref("loader")
    torch.save({"format": loader.PACKED_FORMAT, "schema_version": loader.PACKED_SCHEMA_VERSION, "config": payload,
                "model_state": synthetic.synthetic_state(payload, seed, "reference_tests"),
                "tokenizer_sha256": _ref("tokenizer").tokenizer_file_sha256(tokenizer_file)}, path)
    return path


@pytest.fixture
def b200_slot(monkeypatch):
    """The reference's build_decoder with its CUDA slot bound to the B200 decoder."""
    from ivonar_inference_b200 import decoder

    monkeypatch.setattr(_ref("decoder"), "_kernel_decoder", decoder.kernel_decoder)
    return decoder


@pytest.fixture
def served(tmp_path: Path):
    from ivonar_inference_b200 import synthetic

    payload = synthetic.tiny(hidden=64, heads=4, state_dim=5, latent=24, dense=96, vocab=300, seq_len=96)
    tokenizer_file = _tokenizer_file(tmp_path / "tokenizer.json", 300)
    return _checkpoint(tmp_path / "packed_inference_checkpoint.pt", payload, tokenizer_file, 7), tokenizer_file


def test_engine_load_serves_the_b200_decoder(b200_slot, served) -> None:
    engine_mod = _ref("engine")
    model_file, _ = served
    engine = engine_mod.Engine.load(model_file, device="cuda")
    assert isinstance(engine.decoder, b200_slot.B200Decoder)
    assert engine.info.backend == "ternary"
    assert engine.info.graph is True and engine.decoder.burst_size == b200_slot.BURST
    assert engine.info.notes == ()
    # the packed weights are all the kernels read: nothing was materialised on the GPU
    assert engine.model.token_io.projection.cached_runtime_weight("cuda") is None
    result = engine.complete([{"role": "user", "content": "hi"}], engine_mod.GenerationSettings(max_tokens=24))
    assert isinstance(result.text, str) and result.completion_tokens >= 1
    assert result.finish_reason in {"stop", "length"}
    pieces = list(engine.stream([{"role": "user", "content": "hello there"}], engine_mod.GenerationSettings(max_tokens=24)))
    assert all(isinstance(piece, str) for piece in pieces)


def test_stream_text_greedy_matches_the_reference_decoder(b200_slot, served) -> None:
    """Greedy answers through stream_text: the B200 decoder and the reference's own decoder (torch, fp32 on
    the CPU) produce the same text."""
    generation, loader = _ref("generation"), _ref("loader")
    model_file, tokenizer_file = served
    tokenizer = _ref("tokenizer").TernaryTokenizer.load(tokenizer_file)
    gpu_model = loader.load_model(model_file, device="cuda", materialize=False).model
    cpu_model = loader.load_model(model_file, device="cpu").model
    ours = b200_slot.B200Decoder(gpu_model, device="cuda", sampling=True)
    assert ours.capture()
    reference = _ref("decoder").StaticDecoder(cpu_model, device="cpu", sampling=True)
    prompt = "<|im_start|>user\nwhy is the sky blue<|im_end|>\n<|im_start|>assistant\n"
    texts = []
    for decoder in (ours, reference):
        texts.append("".join(generation.stream_text(tokenizer, decoder, prompt, max_new_tokens=40, temperature=1.0,
                                                     top_k=1, repetition_penalty=1.3)))
    assert texts[0] == texts[1]
    produced = ours.host_position - len(tokenizer.encode(prompt))
    assert 0 <= produced <= 40


def test_check_decoder_passes_eager_and_replayed(b200_slot, served) -> None:
    """The reference's verify.check_decoder: teacher-forced predictions against the model's one-pass fp32
    forward, eager and through the captured graph (which must give the same numbers)."""
    verify, loader = _ref("verify"), _ref("loader")
    model_file, _ = served
    reference = loader.load_model(model_file, device="cpu").model
    gpu_model = loader.load_model(model_file, device="cuda", materialize=False).model
    decoder = b200_slot.B200Decoder(gpu_model, device="cuda")
    ids = torch.randint(2, 300, (60,), generator=torch.Generator().manual_seed(3)).tolist()
    eager = verify.check_decoder(reference, decoder, ids, split=17)
    assert eager.positions == 43
    assert eager.passed, eager.lines()
    assert eager.max_abs_diff < 0.05
    assert abs(eager.decoder_log_prob - eager.reference_log_prob) < 0.05
    assert decoder.capture() is True and decoder.graph is not None
    replayed = verify.check_decoder(reference, decoder, ids, split=17)
    assert replayed.decoder_log_prob == eager.decoder_log_prob
    decoder.reset()
    again = verify.check_decoder(reference, decoder, ids, split=17)
    assert again.decoder_log_prob == replayed.decoder_log_prob


@pytest.mark.parametrize("graph", [True, False])
def test_run_benchmark_through_the_engine(b200_slot, served, graph: bool) -> None:
    bench, engine_mod = _ref("bench"), _ref("engine")
    model_file, _ = served
    engine = engine_mod.Engine.load(model_file, device="cuda", graph=graph)
    assert isinstance(engine.decoder, b200_slot.B200Decoder) and engine.info.graph is graph
    result = bench.run_benchmark(engine, prompt="hi", tokens=32)
    assert result.prompt_tokens > 0
    assert 1 <= result.step_tokens <= 32
    assert result.step_tokens_per_second > 0
    assert len(result.lines()) == 3


def test_build_decoder_falls_back_to_the_reference_when_the_slot_fails(monkeypatch, served) -> None:
    """A B200 decoder that cannot be built leaves the reference's own torch decoder serving, with a note."""
    from ivonar_inference_b200 import decoder

    def broken(*args, **kwargs):
        raise decoder.KernelError("no sm_100 device")

    model_file, _ = served
    model = _ref("loader").load_model(model_file, device="cuda", materialize=False).model
    monkeypatch.setattr(decoder, "kernel_decoder", broken)
    served_decoder, backend, note = decoder.build_decoder(model, "cuda", sampling=True)
    assert type(served_decoder) is _ref("decoder").StaticDecoder
    assert backend == "torch" and "no sm_100 device" in note
