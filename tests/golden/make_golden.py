"""Generate the golden vectors that pin the CPU oracle to the reference implementation.

Run where the reference package (ivonar_inference) is importable, for example after installing it
under baseline/_ref as bench.py's reference arm does; IVONAR_HOME must name a writable directory
for its numba cache:

    IVONAR_HOME=<writable dir> PYTHONPATH=<reference install or its src/> python tests/golden/make_golden.py

The generated fixtures are committed, so the tests need only this repository.

It imports LuisOezdem/ivonar-inference unmodified and records, on seeded synthetic inputs:
  quantizer.npz   numba norm_quantize / quantize_into (cpu_decoder.py:30-70)
  ternary.npz     per-128-group integer dots through numba row_dot (cpu_decoder.py:73-86) with
                  one-hot scales, and fp32 outputs of numba gemv / normed_gemv / normed_gemv_silu
  ssm.npz         numba recurrent_step (cpu_decoder.py:137-183) over 4 consecutive steps
  attention.npz   numba attention_step (cpu_decoder.py:186-231) over 6 positions
  sampler.npz     greedy (top_k = 1) picks of the torch sampler with a repetition penalty
                  (decoder.py:324-333)
  model_*.npz     whole-model runs: torch StaticDecoder (fp32) prefill logits and 256-token greedy and
                  penalised-greedy streams (config 0 and tiny: the penalised stream's per-step logits),
                  numba CpuDecoder greedy streams (from the torch prefill, and stepped through the prompt);
                  config 1 also the reference's own spread: per-step mean and max |torch - numba| of the
                  logits, both decoders teacher-forced along the torch greedy stream (ref_spread_*)
Everything is generated from this repository's synthetic models (ivonar_inference_b200.synthetic),
whose state dicts the reference loader reads as-is.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
STREAM = 256           # tokens of every recorded greedy stream
STREAM_CONTEXT = 288   # context of the config-0 and tiny models the streams run on
sys.path.insert(0, str(ROOT))
OUT = Path(__file__).resolve().parent

from ivonar_inference_b200 import synthetic  # noqa: E402


def _reference():
    import ivonar_inference.cpu_decoder as cpu
    from ivonar_inference.config import ModelConfig
    from ivonar_inference.decoder import StaticDecoder
    from ivonar_inference.loader import build_model, materialize_weights
    from ivonar_inference.quantization import TernaryLinear

    return cpu, ModelConfig, StaticDecoder, build_model, materialize_weights, TernaryLinear


def quantizer_vectors(cpu) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(1)
    out: dict[str, np.ndarray] = {}
    cases = [(16, 1.0), (128, 1.0), (200, 3.0), (1024, 1.0), (1024, 40.0), (2816, 0.5), (256, 0.0)]
    for k, (n, spread) in enumerate(cases):
        x = (rng.standard_normal(n) * spread).astype(np.float32)
        if n >= 200:
            x[rng.integers(0, n, 3)] *= 30.0  # outliers beyond the RMSNorm clip
        w = (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        padded = (n + 127) // 128 * 128
        q = np.zeros(padded, np.int32)
        gsum = np.zeros(padded // 128, np.int32)
        work = np.zeros(padded, np.float32)
        s_norm = cpu.norm_quantize(x, w, np.float32(1e-6), np.float32(8.0), work, q, gsum)
        out[f"x{k}"], out[f"w{k}"] = x, w
        out[f"norm_q{k}"], out[f"norm_scale{k}"] = q[:n].astype(np.int8), np.float32(s_norm)
        q2 = np.zeros(padded, np.int32)
        s_plain = cpu.quantize_into(x, q2, gsum)
        out[f"plain_q{k}"], out[f"plain_scale{k}"] = q2[:n].astype(np.int8), np.float32(s_plain)
    out["count"] = np.int32(len(cases))
    return out


def ternary_vectors(cpu, TernaryLinear) -> dict[str, np.ndarray]:
    gen = torch.Generator().manual_seed(2)
    rng = np.random.default_rng(2)
    out: dict[str, np.ndarray] = {}
    shapes = [(64, 1024), (48, 2816), (40, 256), (24, 100), (8, 16), (6, 130)]
    for k, (rows, cols) in enumerate(shapes):
        packed, scales = synthetic._packed(gen, rows, cols, "baseline")
        bias = torch.randn(rows, generator=gen) * 0.02
        lin = TernaryLinear(packed, scales, cols, bias=bias)
        planes, s_np, b_np = cpu.planes_of([lin])
        groups = planes.shape[1] // cpu.PLANE
        x = rng.standard_normal(cols).astype(np.float32)
        q = np.zeros(groups * 128, np.int32)
        gsum = np.zeros(groups, np.int32)
        act_scale = cpu.quantize_into(x, q, gsum)
        q8_plain = q[:cols].astype(np.int8).copy()
        dots = np.zeros((rows, groups), np.int32)
        for g in range(groups):
            onehot = np.zeros_like(s_np)
            onehot[:, g] = 1.0
            for r in range(rows):
                dots[r, g] = int(cpu.row_dot(planes, onehot, r, q, gsum))
        y = np.zeros(rows, np.float32)
        cpu.gemv(x, planes, s_np, b_np, q, gsum, y, False)
        w = (1.0 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
        work = np.zeros(groups * 128, np.float32)
        yn = np.zeros(rows, np.float32)
        cpu.normed_gemv(x, w, np.float32(1e-6), np.float32(8.0), work, planes, s_np, b_np, q, gsum, yn)
        out[f"packed{k}"] = packed.numpy()
        out[f"scales{k}"] = scales.view(torch.int16).numpy().view(np.uint16)
        out[f"bias{k}"] = bias.numpy().astype(np.float32)
        out[f"in{k}"] = np.int32(cols)
        out[f"x{k}"], out[f"w{k}"] = x, w
        out[f"q8_{k}"], out[f"act_scale{k}"] = q8_plain, np.float32(act_scale)
        out[f"dots{k}"], out[f"gemv{k}"], out[f"normed_gemv{k}"] = dots, y, yn
        if rows % 2 == 0:
            # SwiGLU pair over two halves of the matrix used as gate and up projections
            half = rows // 2
            gate = TernaryLinear(packed[:half], scales[:half], cols, bias=bias[:half])
            up = TernaryLinear(packed[half:], scales[half:], cols, bias=bias[half:])
            p2, s2, b2 = cpu.planes_of([gate, up])
            mid = np.zeros(half, np.float32)
            cpu.normed_gemv_silu(x, w, np.float32(1e-6), np.float32(8.0), work, p2, s2, b2, q, gsum, mid)
            out[f"silu{k}"] = mid
    out["count"] = np.int32(len(shapes))
    return out


def ssm_vectors(cpu) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(3)
    hidden, heads, state, hd, taps = 128, 4, 16, 32, 4
    width = 2 * hidden + 3 * heads * state
    conv_taps = (0.1 * rng.standard_normal((hidden, taps))).astype(np.float32)
    conv_taps[:, -1] += 1.0
    conv_bias = (0.01 * rng.standard_normal(hidden)).astype(np.float32)
    log_decay = (rng.random((heads, state)) * 0.5 - 1.0).astype(np.float32)
    decay = (-np.log1p(np.exp(log_decay))).astype(np.float32)
    theta = (rng.random((heads, state)) * np.pi).astype(np.float32)
    skip = (1.0 + 0.1 * rng.standard_normal((heads, hd))).astype(np.float32)
    conv_state = np.zeros((hidden, taps - 1), np.float32)
    ssm_state = np.zeros((heads, state, hd, 2), np.float32)
    prev = np.zeros((heads, state, hd), np.float32)
    values = np.zeros(hidden, np.float32)
    out = {"conv_taps": conv_taps.copy(), "conv_bias": conv_bias, "decay": decay, "theta": theta, "skip": skip}
    for step in range(4):
        mixer_in = rng.standard_normal(width).astype(np.float32)
        y = np.zeros(hidden, np.float32)
        cpu.recurrent_step(mixer_in, hidden, heads, state, hd, conv_taps, conv_bias, conv_state, decay, theta, skip,
                           ssm_state, prev, np.float32(0.5e-3), np.float32(0.5 * (0.1 - 1e-3)), values, y)
        out[f"in{step}"], out[f"y{step}"] = mixer_in, y.copy()
    out["ssm_state"], out["prev_force"], out["conv_state"] = ssm_state, prev, conv_state
    return out


def attention_vectors(cpu) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(4)
    heads, hd, nope, rope, latent, max_len = 4, 32, 16, 16, 64, 8
    hidden = heads * hd
    width = hidden + latent + heads * rope
    ang = rng.random((max_len, rope // 2)).astype(np.float32) * 3.0
    table = np.stack([np.cos(ang), np.sin(ang)], axis=-1).astype(np.float32)
    full = np.concatenate([np.stack([np.ones((max_len, nope // 2)), np.zeros((max_len, nope // 2))], -1), table], axis=1)
    full = np.ascontiguousarray(full.astype(np.float32))
    k_cache = np.zeros((heads, max_len, hd), np.float32)
    v_cache = np.zeros((heads, max_len, hd), np.float32)
    out = {"rope": table}
    scale = np.float32(1.0 / np.sqrt(hd))
    for pos in range(6):
        mixer_in = rng.standard_normal(width).astype(np.float32)
        kv = rng.standard_normal(heads * nope + hidden).astype(np.float32)
        y = np.zeros(hidden, np.float32)
        cpu.attention_step(mixer_in, kv, full, pos, k_cache, v_cache, y, heads, hd, nope, rope, latent, scale)
        out[f"in{pos}"], out[f"kv{pos}"], out[f"y{pos}"] = mixer_in, kv, y.copy()
    return out


def sampler_vectors(StaticDecoder, model) -> dict[str, np.ndarray]:
    gen = torch.Generator().manual_seed(5)
    dec = StaticDecoder(model, max_len=8, device="cpu", sampling=True)
    out = {}
    for k in range(6):
        logits = torch.randn(1, model.config.vocab_size, generator=gen) * (1 + k)
        top = int(logits.argmax())
        penalized = [top] if k % 2 else []
        dec.configure_sampling(temperature=0.7, top_k=1, repetition_penalty=3.0, penalized_ids=penalized)
        dec.logits.copy_(logits)
        out[f"logits{k}"] = logits[0].numpy()
        out[f"penalized{k}"] = np.array(penalized, np.int64)
        out[f"token{k}"] = np.int64(dec.sample())
    return out


def model_run(ref, payload: dict, seed: int, style: str, prompt_len: int, steps: int, keep_logits: bool, numba: bool):
    cpu, ModelConfig, StaticDecoder, build_model, materialize_weights, _ = ref
    state = synthetic.synthetic_state(payload, seed, style)
    model = build_model(ModelConfig.from_payload(payload), state).eval()
    materialize_weights(model, torch.float32)
    vocab = payload["vocab_size"]
    prompt = synthetic.random_prompt(vocab, prompt_len, seed=seed)
    out = {"prompt": prompt[0].numpy(), "seed": np.int64(seed)}
    dec = StaticDecoder(model, max_len=payload["seq_len"], device="cpu", sampling=True)
    out["prefill_logits"] = dec.prefill(prompt)[0].clone().numpy()
    for tag, rp in (("greedy", 1.0), ("greedy_rp", 4.0)):
        dec.prefill(prompt)
        dec.configure_sampling(temperature=1.0, top_k=1, repetition_penalty=rp)
        tokens = [dec.sample()]
        logits = []
        for _ in range(steps - 1):
            tokens.append(dec.advance())
            if keep_logits and tag == "greedy_rp":
                logits.append(dec.logits[0].clone().numpy())
        out[f"torch_{tag}"] = np.array(tokens, np.int64)
        if logits:
            # logits after each fed token: step_logits[i] chose stream[i + 1] (prefill_logits chose stream[0])
            out[f"torch_{tag}_step_logits"] = np.stack(logits)
    if numba:
        cdec = cpu.CpuDecoder(model, max_len=payload["seq_len"], sampling=True)
        for tag, rp in (("greedy", 1.0), ("greedy_rp", 4.0)):
            cdec.prefill(prompt)
            cdec.configure_sampling(temperature=1.0, top_k=1, repetition_penalty=rp)
            out[f"numba_{tag}"] = np.array([cdec.sample(), *cdec.advance_many(steps - 1)], np.int64)
        # the numba decoder stepping through the prompt too (no torch prefill state)
        cdec.prefill(prompt[:, :1])
        for i in range(1, prompt.shape[1]):
            cdec.step(prompt[:, i])
        out["numba_stepped_logits"] = cdec.logits[0].clone().numpy()
        cdec.configure_sampling(temperature=1.0, top_k=1, repetition_penalty=1.0)
        out["numba_stepped_greedy"] = np.array([cdec.sample(), *cdec.advance_many(steps - 1)], np.int64)
    return out, model


def spread_run(ref, payload: dict, seed: int, style: str, data: dict, max_len: int) -> dict:
    """The reference's own fp32 spread on a model: its torch StaticDecoder and numba CpuDecoder
    prefill the same prompt and are teacher-forced along the torch greedy stream; per step the mean and
    max |logit difference|."""
    cpu, ModelConfig, StaticDecoder, build_model, materialize_weights, _ = ref
    state = synthetic.synthetic_state(payload, seed, style)
    model = build_model(ModelConfig.from_payload(payload), state).eval()
    materialize_weights(model, torch.float32)
    prompt = torch.from_numpy(data["prompt"]).view(1, -1)
    dec = StaticDecoder(model, max_len=max_len, device="cpu", sampling=True)
    cdec = cpu.CpuDecoder(model, max_len=max_len, sampling=True)
    dec.prefill(prompt)
    cdec.prefill(prompt)
    means, maxes = [], []
    for tok in data["torch_greedy"][:-1]:
        a = dec.step(torch.tensor([int(tok)]))[0].numpy()
        b = cdec.step(torch.tensor([int(tok)]))[0].numpy()
        d = np.abs(a - b)
        means.append(d.mean())
        maxes.append(d.max())
    return {"ref_spread_mean": np.array(means, np.float32), "ref_spread_max": np.array(maxes, np.float32)}


def main() -> None:
    if "--spread-only" in sys.argv:
        # add the spread arrays to an existing config-1 fixture (its other arrays stay as they are)
        ref = _reference()
        path = OUT / "model_config1.npz"
        data = dict(np.load(path))
        data.update(spread_run(ref, synthetic.config1(seq_len=2048), 0, "baseline", data, 320))
        np.savez_compressed(path, **data)
        print(f"{path.name}: {path.stat().st_size} bytes")
        return
    ref = _reference()
    cpu, ModelConfig, StaticDecoder, build_model, materialize_weights, TernaryLinear = ref
    np.savez_compressed(OUT / "quantizer.npz", **quantizer_vectors(cpu))
    np.savez_compressed(OUT / "ternary.npz", **ternary_vectors(cpu, TernaryLinear))
    np.savez_compressed(OUT / "ssm.npz", **ssm_vectors(cpu))
    np.savez_compressed(OUT / "attention.npz", **attention_vectors(cpu))
    # 256-token streams; the models' contexts hold the prompt and every generated token
    data, model0 = model_run(ref, synthetic.config0(seq_len=STREAM_CONTEXT), 0, "baseline", 16, STREAM, True, True)
    np.savez_compressed(OUT / "model_config0.npz", seq_len=np.int64(STREAM_CONTEXT), **data)
    np.savez_compressed(OUT / "sampler.npz", **sampler_vectors(StaticDecoder, model0))
    data, _ = model_run(ref, synthetic.tiny(seq_len=STREAM_CONTEXT), 3, "reference_tests", 8, STREAM, True, True)
    np.savez_compressed(OUT / "model_tiny.npz", seq_len=np.int64(STREAM_CONTEXT), **data)
    if "--no-nano" not in sys.argv:
        data, _ = model_run(ref, synthetic.config1(seq_len=2048), 0, "baseline", 36, STREAM, False, True)
        data.update(spread_run(ref, synthetic.config1(seq_len=2048), 0, "baseline", data, 320))
        np.savez_compressed(OUT / "model_config1.npz", seq_len=np.int64(2048), **data)
    for path in sorted(OUT.glob("*.npz")):
        print(f"{path.name}: {path.stat().st_size} bytes")


if __name__ == "__main__":
    main()
