#!/usr/bin/env python
"""Benchmark of the Ivonar token loop on B200 (one JSON line on stdout from rank 0).

Workload (benchmark configuration 1): Nano-shaped ternary hybrid (vocab 32768, d 1024, 24 blocks), batch 1,
a 36-token random prompt, then 256 sampled decode tokens (T 0.5, top-k 40, repetition penalty 1.15).
A step is one such generation. `value` is decode tokens/s of the persistent decode kernel with the
prompt already prefilled in HBM (CUDA events around the one launch that decodes 256 tokens; L2 is
flushed by a 256 MB write before every step, outside the timed region). `e2e` is the same metric
through the public decoder API with the prompt in pinned host memory: prefill + sample + 16 bursts of
advance_many(16), host copies included. With --gpus N (torchrun) every rank decodes its own
independent sequences on its own GPU (data parallel, no collective on the data path); value is the
total over ranks divided by the slowest rank's time.

Secondary, rank 0 (benchmark configuration 2): prompt prefill tok/s at 512, 2048 and 8192 tokens through
B200Decoder.prefill (tcgen05 GEMMs, recurrent scan, latent-cache fill and causal attention) at batch 1
and at batch 8 (eight independent prompts, one decoder and one CUDA stream each, timed together), and
the int8 tensor-core throughput of the prefill GEMM alone on the gate/up shape at 2048 tokens.

Secondary, every rank (benchmark configuration 3): batched serving, 256 independent sequences split evenly over
the N GPUs (data parallel, no collective on the data path), each a 128-token random prompt and then
sampled tokens (T 0.5, top-k 40, rp 1.15, per-sequence seeds) through B200BatchDecoder; `batched.value`
is the aggregate decode tok/s (all sequences' tokens over the slowest rank's CUDA-event time of the
timed decode steps).

Secondary, every rank (benchmark configuration 4): the 7B-shaped model (weights drawn on the GPU) tensor
parallel over the N ranks (`tp`): a 512-token random prompt teacher-forced, then sampled decode at batch
1 and batch 32, tok/s over the slowest rank's CUDA-event time.

Secondary, rank 0 (`gpu_reference`): the reference's own GPU decoder (KernelDecoder, NVRTC-compiled CUDA,
installed unmodified in baseline/_ref) and B200Decoder timed by the same procedure through the reference
API on the same GPU: prefill, configure_sampling, sample, then CUDA events around advance_many bursts that
produce the 256 decode tokens (the reference eager and with its CUDA graphs captured).

Secondary, rank 0 at N=1 (`ingest`): loading the config-1 checkpoint (88.8 MB, in the page cache) to
the GPU through the reference's load_model and through ingest.load_model, median wall-clock ms of 3
loads each with the device synchronised, and the device validation call alone.

--impl reference times the reference's own CPU decoder (the numba CpuDecoder chosen by the reference's
build_decoder for device "cpu", installed unmodified in baseline/_ref) on this host's cores, rank 0 only:
each timed step decodes the workload's 256 sampled tokens after an untimed prefill.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PROMPT = 36
TOKENS = 256
TEMPERATURE, TOP_K, PENALTY = 0.5, 40, 1.15
WORKLOAD = "config1 nano b=1: 36-token random prompt + 256 sampled decode tokens (T 0.5, top-k 40, rp 1.15)"


def log(*args) -> None:
    print(*args, file=sys.stderr, flush=True)


def parse() -> argparse.Namespace:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--tokens", type=int, default=TOKENS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--no-gpu-reference", action="store_true", help="skip the reference KernelDecoder on this GPU")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-batch", action="store_true")
    ap.add_argument("--no-ingest", action="store_true", help="skip the checkpoint-load measurement (N=1 only)")
    ap.add_argument("--tp", action="store_true", help="also measure config 4 (7B-shaped, tensor parallel over the ranks) at N=1")
    ap.add_argument("--no-tp", action="store_true", help="skip config 4, which runs by default on more than one GPU")
    ap.add_argument("--only", choices=("prefill", "gemm", "tp", "batch", "ingest"), default=None,
                    help="run one secondary measurement alone (for profiler captures): a prefill of "
                         "--prefill-tokens tokens, the prefill GEMM on the gate/up shape, config 4, or "
                         "config 3 (--batch-tokens decode tokens per sequence), or the checkpoint load")
    ap.add_argument("--prefill-tokens", type=int, default=2048)
    ap.add_argument("--batch-tokens", type=int, default=512, help="decode tokens per sequence of --only batch")
    ap.add_argument("--kernel-table", action="store_true", help="--only batch: per-kernel device time of a step")
    return ap.parse_args()


def measured_peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# dram__bytes_read.sum + dram__bytes_write.sum of one ncu capture (--set full) of a 16-token
# grid_decode_kernel launch of this workload (1,870,212,352 + 65,810,688 bytes), per token; scaled to a
# launch by the tokens it runs.
NCU_DRAM_BYTES_PER_TOKEN = (1_870_212_352 + 65_810_688) / 16
TRAFFIC_SOURCE = ("ncu --set full capture of a 16-token grid_decode_kernel launch at positions 37-52 "
                  "(python bench.py --steps 1 --warmup 1 --tokens 16 ...), scaled by tokens per launch")


def decode_bytes(model, first_position: int, tokens: int, cache: str = "kv") -> tuple[float, dict]:
    """Algorithmic HBM bytes of `tokens` decode steps starting at `first_position`.

    Per token: every packed ternary byte + fp16 scale + fp32 bias once, the recurrent state read and
    written, and the attention cache read up to the current position plus its append. cache "kv": the
    single-sequence decoder's fp32 key and value rows (heads x 2 x head_dim padded to 4 floats per
    position per attention layer); "latent": the batched decoder's compressed cache (latent codes +
    scale + fp16 k_rope).
    """
    cfg = model.config
    weights = 0
    for proj in model.modules():
        if getattr(proj, "packed_weight", None) is None:
            continue
        weights += proj.packed_weight.numel() + proj.weight_scales.numel() * 2
        if proj.bias is not None:
            weights += proj.bias.numel() * 4
    state = 0
    per_pos = 0
    for block in model.blocks:
        m = block.mixer
        if block.mixer_type == "mamba":
            hsd = m.num_heads * m.state_dim * m.head_dim
            state += 2 * 4 * (2 * hsd + hsd + cfg.hidden_dim * (m.conv_kernel_size - 1))
        elif cache == "kv":
            per_pos += m.num_heads * 2 * ((m.head_dim + 3) // 4 * 4) * 4
        else:
            per_pos += m.latent_dim + 4 + m.num_heads * m.rope_dim * 2
    kv = sum(per_pos * (p + 1) for p in range(first_position, first_position + tokens)) + per_pos * tokens
    total = tokens * (weights + state) + kv
    return float(total), {"weights_per_token": weights, "state_per_token": state, "kv_bytes_per_position": per_pos}


def batch_roofline(model, sequences: int, first_position: int, steps: int, ms: float) -> dict:
    """Per-GPU HBM roofline of config 3's timed decode steps: every step reads the packed weights once
    for all of the GPU's sequences, and each sequence's recurrent state (read and written) and latent
    cache up to its position."""
    per_step_weights, parts = decode_bytes(model, first_position, 1, cache="latent")
    weights, state, per_pos = parts["weights_per_token"], parts["state_per_token"], parts["kv_bytes_per_position"]
    kv = sum(per_pos * (p + 2) for p in range(first_position, first_position + steps))
    total = steps * (weights + sequences * state) + sequences * kv
    peak, peak_kind = measured_peaks()
    achieved = total / (ms / 1000.0) / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "peak_source": peak_kind, "bytes_per_gpu": total,
            "bytes": "per step: packed weights once + per sequence (SSM state read+write + latent cache to its position)"}


class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,utilization.gpu,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, enabled: bool = True) -> None:
        self.index, self.proc, self.path = index, None, None
        if not enabled:
            return
        self.path = Path(tempfile.mkdtemp(prefix="ivb_clocks_")) / f"clocks_rank{index}.csv"
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        loaded = [r for r in rows if r[3].isdigit() and int(r[3]) > 0] or rows
        mhz = [float(r[1]) for r in loaded if r[1].replace(".", "").isdigit()]
        reasons = sorted({names[i] for r in loaded for i in range(4) if r[5 + i].lower() == "active"})
        return {
            "sm_mhz": statistics.median(mhz) if mhz else None,
            "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
            "reasons": reasons,
            "samples": len(rows),
            "samples_under_load": len(loaded),
        }


def reference_environment() -> None:
    """The reference keeps its numba and NVRTC caches under IVONAR_HOME: a temporary directory, set before
    its modules are imported."""
    os.environ.setdefault("IVONAR_HOME", str(Path(tempfile.gettempdir()) / "ivb_reference_home"))


def host_cpu() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def reference_cpu_decoder(model):
    """The decoder the reference serves on device "cpu": its build_decoder picks the numba CpuDecoder
    after that decoder's self-check (the torch StaticDecoder when the check fails)."""
    reference_environment()
    from ivonar_inference_b200 import _reference

    decoder, backend, note = _reference.module("decoder").build_decoder(model, "cpu", sampling=True, kernels=True)
    if backend == "ternary":
        import numba

        threads = int(numba.get_num_threads())
        label = "reference CpuDecoder (numba)"
    else:
        import torch

        threads = int(torch.get_num_threads())
        label = f"reference torch StaticDecoder ({note})"
    return decoder, threads, label


def reference_cpu_rate(decoder, prompt, tokens: int) -> float:
    """Seconds for `tokens` sampled decode tokens after an untimed prefill (reference decoder API)."""
    decoder.prefill(prompt)
    decoder.configure_sampling(TEMPERATURE, TOP_K, PENALTY)
    decoder.sample()
    start = time.perf_counter()
    decoder.advance_many(tokens)
    return time.perf_counter() - start


def cpu_baseline(model, tokens: int) -> dict:
    """The reference's CPU decoder on this host's cores, on a bounded sample (rank 0, N=1)."""
    from ivonar_inference_b200 import synthetic

    decoder, threads, label = reference_cpu_decoder(model)
    reference_cpu_rate(decoder, synthetic.random_prompt(32768, PROMPT, seed=98), 4)  # numba warm-up
    seconds = reference_cpu_rate(decoder, synthetic.random_prompt(32768, PROMPT, seed=99), tokens)
    return {"value": tokens / seconds, "unit": "tok/s", "cores": threads, "kind": "reference",
            "cpu": host_cpu(),
            "sample": f"config1 model, {PROMPT}-token prompt prefilled (untimed), {tokens} sampled decode tokens "
                      f"timed; {label}, {threads} threads, from baseline/_ref",
            "seconds": seconds}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from ivonar_inference_b200 import synthetic

    tokens = int(args.tokens)
    model = synthetic.synthetic_model(synthetic.config1(seq_len=2048), seed=0)
    decoder, threads, label = reference_cpu_decoder(model)
    times = []
    for step in range(args.warmup + args.steps):
        prompt = synthetic.random_prompt(32768, PROMPT, seed=100 + step)
        seconds = reference_cpu_rate(decoder, prompt, tokens if step >= args.warmup else 8)
        if step >= args.warmup:
            times.append(seconds)
    value = args.steps * tokens / sum(times)
    sample = (f"each step: config1 model, {PROMPT}-token prompt prefilled (untimed), {tokens} sampled decode tokens "
              f"timed (warm-up steps decode 8); {label}, {threads} threads, from baseline/_ref")
    line = {
        "impl": "reference", "metric": "decode tok/s (b=1)", "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * sum(times) / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic", "config": {"workload": WORKLOAD, "runs_on": "host CPU"},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "reference", "sample": sample,
                         "cpu": host_cpu()},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def api_decode_rate(decoder, prompt, tokens: int) -> float:
    """Decode tok/s through the reference decoder API: prefill, configure_sampling, sample and 16 warm
    tokens untimed, then CUDA events around the advance_many bursts that produce `tokens` tokens."""
    import torch

    decoder.prefill(prompt)
    decoder.configure_sampling(TEMPERATURE, TOP_K, PENALTY)
    decoder.sample()
    decoder.advance_many(16)
    torch.cuda.synchronize(decoder.device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    done = 0
    while done < tokens:
        done += len(decoder.advance_many(min(decoder.burst_size, tokens - done)))
    end.record()
    torch.cuda.synchronize(decoder.device)
    return tokens / (start.elapsed_time(end) / 1000.0)


def gpu_reference(device, tokens: int) -> dict:
    """The reference KernelDecoder and B200Decoder on this GPU, timed by the same procedure."""
    import torch

    reference_environment()
    from ivonar_inference_b200 import B200Decoder, _reference, synthetic

    model = synthetic.synthetic_model(synthetic.config1(seq_len=2048), seed=0).to(device)
    prompt = synthetic.random_prompt(32768, PROMPT, seed=4242).to(device)
    max_len = PROMPT + tokens + 64
    out: dict = {"procedure": f"{PROMPT}-token prompt, then {tokens} sampled tokens through advance_many bursts "
                              "(CUDA events), reference decoder API", "unit": "tok/s"}
    try:
        kernel_decoder = _reference.module("kernel_decoder").KernelDecoder
        ref = kernel_decoder(model, max_len=max_len, device=device, sampling=True)
        ref.self_check()
        out["reference_kernel_decoder"] = {"eager": api_decode_rate(ref, prompt, tokens)}
        out["reference_kernel_decoder"]["graph_captured"] = bool(ref.capture())
        out["reference_kernel_decoder"]["graph"] = max(api_decode_rate(ref, prompt, tokens) for _ in range(2))
        out["reference_kernel_decoder"]["burst"] = int(ref.burst_size)
        del ref
    except Exception as exc:  # the reference's NVRTC build can be missing on a box
        out["reference_kernel_decoder"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    torch.cuda.empty_cache()
    ours = B200Decoder(model, max_len=max_len, device=device, sampling=True, seed=5)
    ours.capture()
    out["b200_decoder"] = {"graph": max(api_decode_rate(ours, prompt, tokens) for _ in range(2)),
                           "burst": int(ours.burst_size)}
    return out


INT8_NOMINAL_TOPS = 4500.0  # B200 dense int8 tensor-core peak (nominal)
BATCH_SEQUENCES, BATCH_PROMPT, BATCH_TOKENS, BATCH_WARM = 256, 128, 512, 8


def batch_measure(device, world: int, rank: int, tokens: int = BATCH_TOKENS, kernel_table: bool = False) -> dict:
    """Config 3 on this rank: BATCH_SEQUENCES / world sequences decoded together (B200BatchDecoder);
    `tokens` decode tokens per sequence (config 3: 512; fewer only for profiler captures). kernel_table:
    after the timed steps, 4 more steps under the torch profiler (CUPTI) give the device time per kernel
    of a step (in `kernels`), outside the timed region."""
    import torch

    from ivonar_inference_b200 import synthetic
    from ivonar_inference_b200.batch import B200BatchDecoder

    per_rank = max(1, BATCH_SEQUENCES // world)
    model = synthetic.synthetic_model(synthetic.config1(seq_len=2048), seed=0)
    room = 8 if kernel_table else 0  # positions and history slots for the profiled steps
    max_len = BATCH_PROMPT + tokens + 8 + room
    batch = B200BatchDecoder(model, per_rank, max_len=max_len, device=device, history_len=tokens + room)
    first = rank * per_rank
    prompts = [synthetic.random_prompt(32768, BATCH_PROMPT, seed=50_000 + first + i)[0] for i in range(per_rank)]
    batch.start(prompts, [first + i for i in range(per_rank)], TEMPERATURE, TOP_K, PENALTY)
    batch.decode(BATCH_WARM)  # includes the graph capture
    torch.cuda.synchronize(device)
    timed = tokens - 1 - BATCH_WARM
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    batch.decode(timed)
    end.record()
    torch.cuda.synchronize(device)
    out = {"sequences_per_gpu": per_rank, "ms": start.elapsed_time(end), "steps": timed}
    if kernel_table:
        from torch.profiler import ProfilerActivity, profile

        extra = 4
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            batch.decode(extra)
            torch.cuda.synchronize(device)
        rows = [(e.key, e.count // extra, e.device_time_total / extra) for e in prof.key_averages() if e.device_time_total > 0]
        out["kernels"] = [{"kernel": k.replace("(anonymous namespace)::", "").split("(")[0], "launches_per_step": c, "us_per_step": round(t, 1)}
                          for k, c, t in sorted(rows, key=lambda r: -r[2])]
    return out


PREFILL_BATCH = 8


def prefill_measure(device, lengths=((512, 3), (2048, 2), (8192, 1)), gemm_reps: int = 20, batch: int = PREFILL_BATCH) -> dict:
    """Config 2: prefill tok/s per prompt length at batch 1 and at batch `batch` (that many independent
    requests, each its own B200Decoder prefilling its own prompt on its own stream, so their kernels
    overlap), and the GEMM's int8 tensor-core throughput."""
    import ctypes

    import torch

    from ivonar_inference_b200 import B200Decoder, synthetic
    from ivonar_inference_b200 import _native as native

    model = synthetic.synthetic_model(synthetic.config1(seq_len=8192), seed=0)
    result: dict = {"batch": [1, batch], "tok_s": {}, "ms": {}, "tok_s_batch": {}, "ms_batch": {},
                    "batch_note": f"{batch} independent prompts of the same length, one decoder and one CUDA stream each, "
                                  "timed together (CUDA events on the launching stream, all streams joined)"}
    longest = max((length for length, _ in lengths), default=0)
    decs = [B200Decoder(model, max_len=longest, device=device) for _ in range(batch)] if lengths else []
    streams = [torch.cuda.Stream(device=device) for _ in range(batch)]
    for length, reps in lengths:
        prompts = [synthetic.random_prompt(32768, length, seed=length + i).to(device) for i in range(batch)]
        decs[0].prefill(prompts[0])
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(reps):
            decs[0].prefill(prompts[0])
        end.record()
        torch.cuda.synchronize(device)
        ms = start.elapsed_time(end) / reps
        result["tok_s"][str(length)] = length / (ms / 1000.0)
        result["ms"][str(length)] = ms
        main = torch.cuda.current_stream(device)

        def all_prefills() -> None:
            for dec, prompt, st in zip(decs, prompts, streams):
                st.wait_stream(main)
                with torch.cuda.stream(st):
                    dec.prefill(prompt)
            for st in streams:
                main.wait_stream(st)

        all_prefills()  # warm-up (workspaces, tensor maps)
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(reps):
            all_prefills()
        end.record()
        torch.cuda.synchronize(device)
        ms_b = start.elapsed_time(end) / reps
        result["tok_s_batch"][str(length)] = batch * length / (ms_b / 1000.0)
        result["ms_batch"][str(length)] = ms_b
    del decs
    torch.cuda.empty_cache()
    lib = native.library()
    gen = torch.Generator().manual_seed(0)
    rows, cols, tokens = 5632, 1024, 2048
    packed, scales = synthetic._packed(gen, rows, cols, "baseline")
    weights = (packed.to(device).contiguous(), scales.view(torch.int16).to(device).contiguous())
    desc = native.ternary(weights[0], weights[1], None, rows, cols)
    x = torch.randn(tokens, cols, device=device)
    q8 = torch.zeros(tokens, cols, dtype=torch.int8, device=device)
    act = torch.empty(tokens, device=device)
    out = torch.empty(tokens, rows, device=device)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device).cuda_stream
    native.check(lib.ivb_quantize_rows(x.data_ptr(), tokens, cols, 0, 1e-6, 8.0, 1e-5, q8.data_ptr(), cols, act.data_ptr(),
                                       None, stream), "ivb_quantize_rows")

    def gemm() -> None:
        native.check(lib.ivb_ternary_gemm(ctypes.byref(desc), q8.data_ptr(), cols, act.data_ptr(), tokens, 0,
                                          out.data_ptr(), rows, err.data_ptr(), stream), "ivb_ternary_gemm")

    if gemm_reps <= 0:
        return result
    for _ in range(3):
        gemm()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(gemm_reps):
        gemm()
    end.record()
    torch.cuda.synchronize(device)
    if int(err.item()) != 0:
        raise RuntimeError("prefill GEMM reported a timeout")
    us = start.elapsed_time(end) / gemm_reps * 1000.0
    tops = 2.0 * rows * cols * tokens / (us * 1e-6) / 1e12
    result["gemm"] = {"shape": f"{rows}x{cols} weights x {tokens} tokens", "us": us, "tops_int8": tops,
                      "frac_of_nominal_int8_peak": tops / INT8_NOMINAL_TOPS, "peak_tops": INT8_NOMINAL_TOPS,
                      "peak_source": "nominal dense int8 (no measured int8 peak in MEASURED_PEAKS.json)"}
    return result


TP_PROMPT, TP_TOKENS, TP_WARM = 512, 256, 4


def tp_measure(device, world: int, rank: int) -> dict:
    """Config 4 on this rank's shard: B200TensorParallel at batch 1 and 32, `world`-way tensor parallel."""
    import torch
    import torch.distributed as dist

    from ivonar_inference_b200 import synthetic
    from ivonar_inference_b200.tp import B200TensorParallel

    model = synthetic.synthetic_model(synthetic.config4(seq_len=TP_PROMPT + TP_TOKENS + 16), seed=0, style="fast")
    out: dict = {"metric": "decode tok/s, config 4 (7B-shaped), tensor parallel", "unit": "tok/s", "tp": world,
                 "prompt": TP_PROMPT}
    for batch in (1, 32):
        tp = B200TensorParallel(model, rank, world, None, batch=batch, max_len=TP_PROMPT + TP_TOKENS + 8, device=device,
                                history_len=TP_TOKENS)
        prompts = synthetic.random_prompt(32768, TP_PROMPT, seed=777)[0].repeat(batch, 1)
        prompts[:, -1] = torch.arange(batch) % 32768  # distinct last tokens
        tp.start(prompts, list(range(batch)), TEMPERATURE, TOP_K, PENALTY)
        tp.decode(TP_WARM)
        torch.cuda.synchronize(device)
        timed = TP_TOKENS - 1 - TP_WARM
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        tp.decode(timed)
        end.record()
        torch.cuda.synchronize(device)
        ms = torch.tensor([start.elapsed_time(end)], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        out[f"b{batch}"] = {"value": batch * timed / (float(ms.item()) / 1000.0), "ms_per_step": float(ms.item()) / timed,
                            "timed_steps": timed}
        del tp
        torch.cuda.empty_cache()
    return out


def ingest_measure(device, reps: int) -> dict:
    """Checkpoint load of config 1 (packed, on local disk, in the page cache after one untimed load):
    the reference's load_model to the GPU and ingest.load_model, wall clock with the device synchronised
    (median of `reps`), and the one-launch device validation alone (CUDA events)."""
    import torch

    from ivonar_inference_b200 import _reference, ingest, synthetic

    loader = _reference.module("loader")
    payload = synthetic.config1(seq_len=PROMPT + TOKENS + 16)
    state = {k: v.cpu() for k, v in synthetic.synthetic_state(payload, 0, "fast").items()}
    checked = {k: v for k, v in state.items() if k.endswith((".packed_weight", ".weight_scales"))}
    checked_bytes = sum(v.numel() * v.element_size() for v in checked.values())
    out: dict = {"metric": "checkpoint load ms, config 1", "unit": "ms", "reps": reps}
    with tempfile.TemporaryDirectory() as tmp:
        path = Path(tmp) / "packed_inference_checkpoint.pt"
        torch.save({"format": loader.PACKED_FORMAT, "schema_version": loader.PACKED_SCHEMA_VERSION,
                    "config": payload, "model_state": state}, path)
        out["file_bytes"] = path.stat().st_size
        for name, load in (("reference", loader.load_model), ("b200", ingest.load_model)):
            times = []
            for i in range(reps + 1):
                torch.cuda.synchronize(device)
                t0 = time.perf_counter()
                loaded = load(path, device, materialize=False)
                torch.cuda.synchronize(device)
                if i:
                    times.append((time.perf_counter() - t0) * 1000.0)
                del loaded
            out[name] = {"ms": statistics.median(times), "min_ms": min(times)}
    on_device = {k: v.to(device) for k, v in checked.items()}
    ingest.validate_state_device(on_device, device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        ingest.validate_state_device(on_device, device)
    end.record()
    torch.cuda.synchronize(device)
    ms = start.elapsed_time(end) / reps
    peak, peak_kind = measured_peaks()
    out["validate"] = {"buffers": len(checked), "bytes": checked_bytes, "ms": ms,
                       "gbs": checked_bytes / (ms / 1000.0) / 1e9, "peak_gbs": peak, "peak_kind": peak_kind,
                       "note": "per call: descriptor copy, one launch, one synchronising read of 12 bytes"}
    out["speedup"] = out["reference"]["ms"] / out["b200"]["ms"]
    return out


def run_b200(args) -> None:
    import torch
    import torch.distributed as dist

    from ivonar_inference_b200 import B200Decoder, synthetic
    from ivonar_inference_b200 import _native as native

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    tokens = int(args.tokens)
    model = synthetic.synthetic_model(synthetic.config1(seq_len=2048), seed=0)
    dec = B200Decoder(model, max_len=512, device=device, sampling=True, seed=1000 + rank)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    def barrier() -> None:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    # ---- device-timed decode (prompt already prefilled in HBM) --------------------------------
    step_ms = []
    clocks = None
    for step in range(args.warmup + args.steps):
        prompt = synthetic.random_prompt(32768, PROMPT, seed=10_000 * rank + step)
        dec.prefill(prompt)
        dec.configure_sampling(TEMPERATURE, TOP_K, PENALTY)
        dec.sample()
        flush.zero_()
        if step == args.warmup:
            barrier()
            clocks = ClockSampler(local, enabled=not args.no_clocks and rank == 0)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        dec._launch(tokens, None, native.IVB_RUN_SAMPLE)
        end.record(stream)
        dec._check()
        if step >= args.warmup:
            step_ms.append(start.elapsed_time(end))
    barrier()
    clock_info = clocks.stop() if clocks is not None else None
    total_ms = torch.tensor([sum(step_ms)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(total_ms, op=dist.ReduceOp.MAX)
    max_ms = float(total_ms.item())
    value = world * args.steps * tokens / (max_ms / 1000.0)

    # ---- end to end through the public API with host buffers ----------------------------------
    dec.capture()
    e2e_ms = []
    h2d = d2h = 0
    for step in range(args.warmup + args.steps):
        prompt = synthetic.random_prompt(32768, PROMPT, seed=20_000 * rank + step).pin_memory()
        flush.zero_()
        barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        dec.prefill(prompt)
        dec.configure_sampling(TEMPERATURE, TOP_K, PENALTY)
        produced = [dec.sample()]
        while len(produced) < tokens + 1:
            produced += dec.advance_many(min(dec.burst_size, tokens + 1 - len(produced)))
        end.record(stream)
        torch.cuda.synchronize(device)
        if step >= args.warmup:
            e2e_ms.append(start.elapsed_time(end))
        bursts = -(-tokens // max(dec.burst_size, 1))
        h2d = prompt.numel() * prompt.element_size()
        d2h = 8 * (tokens + 1) + 4 * (bursts + 2)
    e2e_total = torch.tensor([sum(e2e_ms)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(e2e_total, op=dist.ReduceOp.MAX)
    e2e_value = world * args.steps * tokens / (float(e2e_total.item()) / 1000.0)

    ctas, phases = dec.ctas, dec.num_phases
    tp_line = None
    if args.tp or (world > 1 and not args.no_tp):
        tp_line = tp_measure(device, world, rank)
    batched = None
    if not args.no_batch:
        del dec
        torch.cuda.empty_cache()
        part = batch_measure(device, world, rank)
        batch_ms = torch.tensor([part["ms"]], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(batch_ms, op=dist.ReduceOp.MAX)
        seqs = part["sequences_per_gpu"] * world
        batched = {"metric": "batched decode tok/s (aggregate, config 3)", "value": seqs * part["steps"] / (float(batch_ms.item()) / 1000.0),
                   "unit": "tok/s", "sequences": seqs, "sequences_per_gpu": part["sequences_per_gpu"],
                   "prompt": BATCH_PROMPT, "timed_steps": part["steps"], "ms": float(batch_ms.item()),
                   "ms_per_step": float(batch_ms.item()) / part["steps"], "parallelism": f"dp{world}"}
        batched["roofline"] = batch_roofline(model, part["sequences_per_gpu"], BATCH_PROMPT + 1 + BATCH_WARM, part["steps"],
                                             float(batch_ms.item()))

    if rank == 0:
        peak, peak_kind = measured_peaks()
        nbytes, parts = decode_bytes(model, PROMPT + 1, tokens)
        launch_s = (sum(step_ms) / len(step_ms)) / 1000.0
        achieved = nbytes / launch_s / 1e9
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                    "traffic": NCU_DRAM_BYTES_PER_TOKEN * tokens, "traffic_source": TRAFFIC_SOURCE,
                    "peak_source": peak_kind, "kernel": "ivb::grid_decode_kernel",
                    "algorithmic_bytes_per_launch": nbytes, **parts}
        line = {
            "metric": "decode tok/s (b=1)", "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": max_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": WORKLOAD, "l2": "flushed (256 MB write) before every step", "parallelism": f"dp{world}",
                       "ctas": ctas, "phases_per_token": phases},
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": args.steps,
            "roofline": roofline,
            "clocks": clock_info,
        }
        if batched is not None:
            line["batched"] = batched
        if tp_line is not None:
            line["tp"] = tp_line
        if not args.no_prefill:
            line["prefill"] = prefill_measure(device)
        if not args.no_gpu_reference:
            line["gpu_reference"] = gpu_reference(device, tokens)
        if world == 1 and not args.no_ingest:
            try:
                line["ingest"] = ingest_measure(device, 3)
            except Exception as exc:  # a secondary measurement must not cost the main line
                line["ingest"] = {"error": f"{type(exc).__name__}: {exc}"}
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(model, 32)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    args = parse()
    if args.only == "tp":
        import datetime

        import torch
        import torch.distributed as dist

        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
        if world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
        result = tp_measure(device, world, rank)
        if rank == 0:
            print(json.dumps(result), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.only is not None:
        import torch

        torch.cuda.set_device(0)
        device = torch.device("cuda", 0)
        if args.only == "prefill":
            print(json.dumps(prefill_measure(device, lengths=((args.prefill_tokens, args.steps),), gemm_reps=0)), flush=True)
        elif args.only == "ingest":
            print(json.dumps(ingest_measure(device, args.steps)), flush=True)
        elif args.only == "batch":
            r = batch_measure(device, 1, 0, tokens=args.batch_tokens, kernel_table=args.kernel_table)
            r["tok_s"] = r["sequences_per_gpu"] * r["steps"] / (r["ms"] / 1000.0)
            print(json.dumps(r), flush=True)
        else:
            print(json.dumps(prefill_measure(device, lengths=(), gemm_reps=args.steps)["gemm"]), flush=True)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
