"""B200Decoder: the reference decoder interface over the sm_100a whole-GPU decode kernel.

Drop-in for ``ivonar_inference.kernel_decoder.KernelDecoder`` behind ``build_decoder`` (reference
src/ivonar_inference/decoder.py:61-466 for the interface, 479-529 for the dispatch). Like the
reference's own GPU decoder it is a subclass of the reference's ``StaticDecoder``
(kernel_decoder.py:145-170): the constructor, attributes (device, max_len, batch_size, burst_size,
position, host_position, logits, token, seen, graph, graphs, attention_lengths), ``step``,
``advance``, ``configure_sampling``, ``reset`` and ``attention_length`` are the reference's own; this
class overrides what the kernels run (``prefill``, the per-token ``_step`` and ``_sample``,
``advance_many``, ``capture``, ``self_check``).

The model is the reference ``IvonarModel``; only its packed tensors are read. Weights stay in the
q2_g128 format; rows are stacked per fused projection (entry, gate/up interleaved) and padded to
16-byte rows, as the reference Matrix does (kernel_decoder.py:84-142). The attention cache is the
compressed latent (int8 codes + scale per position, fp16 rotated k_rope) instead of the reference's
decompressed fp16 K/V.
"""

from __future__ import annotations

import ctypes
import math

import torch
import torch.nn.functional as F
from torch import Tensor

from . import _native as native
from . import _reference
from ._native import KernelError

StaticDecoder = _reference.module("decoder").StaticDecoder

BURST = 16
SELF_CHECK_TOLERANCE = 0.25
DEFAULT_TIMEOUT_NS = 2_000_000_000
PREFILL_CHUNK = 2048  # prompt tokens per tensor-core prefill call (workspace grows with it)


def _pad_rows(packed: Tensor) -> Tensor:
    row_bytes = int(packed.shape[1])
    padded = (row_bytes + 15) // 16 * 16
    return F.pad(packed, (0, padded - row_bytes)) if padded != row_bytes else packed


def _stack(tensors: list[Tensor], interleave: bool) -> Tensor:
    if len(tensors) == 1:
        return tensors[0]
    if interleave:
        return torch.stack(tensors, dim=1).reshape(-1, *tensors[0].shape[1:])
    return torch.cat(tensors, dim=0)


class DeviceMatrix:
    """A row-stack of packed projections on the device, in the layout the kernels read."""

    def __init__(self, projections: list, device: torch.device, interleave: bool = False, scale_align: int = 1) -> None:
        first = projections[0]
        self.in_features = int(first.in_features)
        for proj in projections:
            if int(proj.in_features) != self.in_features:
                raise KernelError("fused projections must share their input width")
            if int(getattr(proj, "group_size", 128)) != 128:
                raise KernelError("ternary kernels need group size 128")
            if proj.weight_scales.dtype != torch.float16:
                raise KernelError("ternary kernels need float16 group scales")
            if interleave and int(proj.out_features) != int(first.out_features):
                raise KernelError("interleaved projections must share their output width")
        packed = _stack([p.packed_weight.to(device) for p in projections], interleave)
        self.packed = _pad_rows(packed).contiguous()
        scales = _stack([p.weight_scales.to(device) for p in projections], interleave)
        stride = (int(scales.shape[1]) + scale_align - 1) // scale_align * scale_align
        if stride != int(scales.shape[1]):
            scales = F.pad(scales, (0, stride - int(scales.shape[1])))
        self.scales = scales.contiguous()
        biases = [p.bias for p in projections]
        if all(b is None for b in biases):
            self.bias = None
        else:
            filled = [torch.zeros(int(p.out_features)) if b is None else b.float() for p, b in zip(projections, biases)]
            self.bias = _stack([b.to(device) for b in filled], interleave).contiguous()
        self.rows = int(self.packed.shape[0])

    def desc(self) -> native.IvbTernary:
        return native.ternary(self.packed, self.scales, self.bias, self.rows, self.in_features)

    @property
    def nbytes(self) -> int:
        return self.packed.numel() + self.scales.numel() * 2 + (0 if self.bias is None else self.bias.numel() * 4)


def rope_from_rotary(rotary, max_len: int) -> Tensor:
    """[max_len, rope_dim/2, 2] (cos, sin) of one attention layer, computed by the reference's own
    ``Rotary.rotate`` on unit vectors (as StaticDecoder._prepare_attention does, decoder.py:177-181)."""

    dim = int(rotary.head_dim)
    unit = torch.zeros(1, max_len, 1, dim, dtype=torch.float32)
    unit[..., 0::2] = 1.0
    return rotary.rotate(unit, offset=0).reshape(max_len, dim // 2, 2).contiguous()


class B200Decoder(StaticDecoder):
    """Batch-1 decoder whose whole token step is one persistent sm_100a kernel launch."""

    backend_name = "ternary-b200"

    def __init__(
        self,
        model,
        max_len: int | None = None,
        device: str | torch.device | None = None,
        sampling: bool = False,
        max_top_k: int = 256,
        ctas: int = 0,
        seed: int | None = None,
        timeout_ns: int = DEFAULT_TIMEOUT_NS,
        prefill: str = "gemm",
        prefill_chunk: int = PREFILL_CHUNK,
    ) -> None:
        target = model.device if device is None else torch.device(device)
        if target.type != "cuda":
            raise KernelError("ternary kernels need a CUDA device")
        if target.index is None:
            target = torch.device("cuda", torch.cuda.current_device())
        if prefill not in ("gemm", "steps"):
            raise ValueError("prefill must be 'gemm' (tensor-core prefill) or 'steps' (token by token)")
        self.lib = native.library()
        with torch.cuda.device(target):
            if not self.lib.ivb_device_supported():
                raise KernelError(f"{torch.cuda.get_device_name(target)} is not an sm_100 GPU this build runs on")
        capacity = int(model.config.seq_len if max_len is None else max_len)
        super().__init__(model, max_len=capacity, batch_size=1, device=target, sampling=sampling, max_top_k=max_top_k,
                         attention_lengths=(capacity,), fuse_projections=False)
        # the kernels keep their own compressed latent cache: the reference's fp16 K/V caches go
        self.attention_caches = {}
        self.prefill_mode = prefill
        self.prefill_chunk = max(1, int(prefill_chunk))
        self._prefill_ws: Tensor | None = None
        self.vocab = int(model.config.vocab_size)
        self._burst_graph: torch.cuda.CUDAGraph | None = None
        self.timeout_ns = int(timeout_ns)
        dev = self.device
        # temperature, penalty and inverse penalty side by side (the kernels read one [3] array); the
        # reference's configure_sampling fills these views
        self._sampling = torch.ones(3, dtype=torch.float32, device=dev)
        self.temperature = self._sampling[0:1]
        self.penalty = self._sampling[1:2]
        self.inverse_penalty = self._sampling[2:3]
        self.history = torch.zeros(max(self.max_len, BURST), dtype=torch.int64, device=dev)
        if seed is None:
            seed = int(torch.randint(0, 2**62, (1,)).item())
        self.rng = torch.tensor([int(seed), 0], dtype=torch.int64, device=dev)
        self._ctas_request = int(ctas)
        self._pending_check = False
        self._build(model, dev)

    # ------------------------------------------------------------------------------------------
    def _build(self, model, dev: torch.device) -> None:
        config = model.config
        hidden, heads = int(config.hidden_dim), int(config.num_heads)
        head_dim = hidden // heads
        self.head = DeviceMatrix([model.token_io.projection], dev)
        self.final_norm = model.final_norm.weight.float().to(dev).contiguous()
        self.layer_matrices: list[dict[str, DeviceMatrix]] = []
        self.latent_caches: dict[int, tuple[Tensor, Tensor, Tensor]] = {}
        self.kv_caches: dict[int, tuple[Tensor, Tensor]] = {}
        self._keep: list[Tensor] = []
        layers = (native.IvbLayerDesc * len(model.blocks))()
        dims = {"state": int(config.state_dim), "latent": int(config.latent_dim), "rope": 2, "nope": head_dim - 2}
        clip = 8.0
        for index, block in enumerate(model.blocks):
            mixer = block.mixer
            kind = getattr(block, "mixer_type", None)
            desc = layers[index]
            mats: dict[str, DeviceMatrix] = {}
            norm_m = block.mixer_norm.weight.float().to(dev).contiguous()
            norm_f = block.ffn_norm.weight.float().to(dev).contiguous()
            self._keep += [norm_m, norm_f]
            clip = float(getattr(block.mixer_norm, "clip", 8.0))
            desc.mixer_norm = norm_m.data_ptr()
            desc.mixer_norm_eps = float(block.mixer_norm.eps)
            desc.ffn_norm = norm_f.data_ptr()
            desc.ffn_norm_eps = float(block.ffn_norm.eps)
            if kind == "mamba":
                desc.kind = native.IVB_MAMBA
                mats["entry"] = DeviceMatrix([mixer.in_proj, mixer.bc_dt_proj], dev)
                mats["out"] = DeviceMatrix([mixer.out_proj], dev)
                taps = int(mixer.conv_kernel_size)
                consts = {
                    "decay": (-F.softplus(mixer.log_decay.float())).contiguous(),
                    "theta": mixer.theta.float().contiguous(),
                    "skip": mixer.skip.float().reshape(-1).contiguous(),
                    "conv_weight": mixer.conv_weight.float().reshape(hidden, taps).contiguous(),
                    "conv_bias": mixer.conv_bias.float().contiguous(),
                }
                consts = {k: v.to(dev) for k, v in consts.items()}
                self._keep += list(consts.values())
                # the reference's recurrent state buffers (StaticDecoder._prepare_recurrent): [1, H, S, hd, 2],
                # [1, H, S, hd], [1, hidden, taps - 1] fp32, the layout the kernels read
                state = self.recurrent_states[index]
                if taps < 2:
                    raise KernelError("the B200 kernels need a causal convolution of at least 2 taps")
                for key in ("decay", "theta", "skip", "conv_weight", "conv_bias"):
                    setattr(desc, key, consts[key].data_ptr())
                desc.ssm_state = state["ssm_state"].data_ptr()
                desc.prev_force = state["prev_force"].data_ptr()
                desc.conv_state = state["conv_state"].data_ptr()
                desc.conv_taps = taps
                desc.half_dt_min = 0.5 * float(mixer.dt_min)
                desc.half_dt_range = 0.5 * (float(mixer.dt_max) - float(mixer.dt_min))
                dims["state"] = int(mixer.state_dim)
            elif kind == "mla":
                desc.kind = native.IVB_MLA
                mats["entry"] = DeviceMatrix([mixer.q_proj, mixer.kv_down_proj, mixer.k_rope_proj], dev)
                mats["out"] = DeviceMatrix([mixer.out_proj], dev)
                # up-projections are read by bulk copies: 16-byte scale rows
                mats["k_nope_up"] = DeviceMatrix([mixer.k_nope_up_proj], dev, scale_align=8)
                mats["v_up"] = DeviceMatrix([mixer.v_up_proj], dev, scale_align=8)
                rope = rope_from_rotary(mixer.rope, self.max_len).to(dev)
                # compressed cache: int8 latent codes (rows padded to 16 bytes), one scale per
                # position (padded to a multiple of 4), head-major fp16 k_rope (rows padded to 8)
                lpad = (int(mixer.latent_dim) + 15) // 16 * 16
                rpad = (int(mixer.rope_dim) + 7) // 8 * 8
                latent_q = torch.zeros(self.max_len, lpad, dtype=torch.int8, device=dev)
                # bulk copies read scales in 16-byte units: pad so a tile ending at max_len stays inside
                latent_scale = torch.zeros((self.max_len + 7) // 4 * 4, dtype=torch.float32, device=dev)
                k_rope = torch.zeros(mixer.num_heads, self.max_len, rpad, dtype=torch.float16, device=dev)
                # the decode kernel's decompressed cache: per head and position, fp32 keys [k_nope |
                # rotated k_rope] and values, rows padded to 16 bytes
                kvpad = (int(mixer.head_dim) + 3) // 4 * 4
                k_cache = torch.zeros(mixer.num_heads, self.max_len, kvpad, dtype=torch.float32, device=dev)
                v_cache = torch.zeros_like(k_cache)
                self._keep.append(rope)
                self.latent_caches[index] = (latent_q, latent_scale, k_rope)
                self.kv_caches[index] = (k_cache, v_cache)
                desc.k_nope_up = mats["k_nope_up"].desc()
                desc.v_up = mats["v_up"].desc()
                desc.rope = rope.data_ptr()
                desc.latent_q = latent_q.data_ptr()
                desc.latent_scale = latent_scale.data_ptr()
                desc.k_rope_cache = k_rope.data_ptr()
                desc.k_cache = k_cache.data_ptr()
                desc.v_cache = v_cache.data_ptr()
                desc.attn_scale = 1.0 / math.sqrt(mixer.head_dim)
                dims.update(latent=int(mixer.latent_dim), rope=int(mixer.rope_dim), nope=int(mixer.nope_dim))
            else:
                raise KernelError(f"unsupported mixer for the B200 kernels: {type(mixer).__name__}")
            mats["gate_up"] = DeviceMatrix([block.ffn.gate_proj, block.ffn.up_proj], dev, interleave=True)
            mats["down"] = DeviceMatrix([block.ffn.down_proj], dev)
            desc.entry = mats["entry"].desc()
            desc.out = mats["out"].desc()
            desc.gate_up = mats["gate_up"].desc()
            desc.down = mats["down"].desc()
            self.layer_matrices.append(mats)
        self._layers = layers
        md = native.IvbModelDesc()
        md.abi_version = native.IVB_ABI_VERSION
        md.vocab = self.vocab
        md.hidden = hidden
        md.heads = heads
        md.head_dim = head_dim
        md.state_dim = dims["state"]
        md.latent_dim = dims["latent"]
        md.rope_dim = dims["rope"]
        md.nope_dim = dims["nope"]
        md.dense = int(config.dense_dim)
        md.num_layers = len(model.blocks)
        md.max_len = self.max_len
        md.max_top_k = self.max_top_k
        md.act_eps = float(getattr(model.token_io.projection, "eps", 1e-5))
        md.norm_clip = clip
        md.head = self.head.desc()
        md.final_norm = self.final_norm.data_ptr()
        md.final_norm_eps = float(model.final_norm.eps)
        md.layers = ctypes.cast(layers, ctypes.POINTER(native.IvbLayerDesc))
        md.logits = self.logits.data_ptr()
        md.token = self.token.data_ptr()
        md.position = self.position.data_ptr()
        md.seen = self.seen.data_ptr()
        md.history = self.history.data_ptr()
        md.history_len = int(self.history.numel())
        md.sampling = self._sampling.data_ptr()
        md.top_k = self.top_k.data_ptr()
        md.rng = self.rng.data_ptr()
        self._desc = md
        handle = ctypes.c_void_p()
        with torch.cuda.device(dev):
            native.check(self.lib.ivb_decoder_create(ctypes.byref(md), self._ctas_request, ctypes.byref(handle)),
                         "ivb_decoder_create")
            self._plan = handle
            self.workspace = torch.zeros(int(self.lib.ivb_decoder_workspace_bytes(handle)), dtype=torch.uint8, device=dev)
            native.check(self.lib.ivb_decoder_bind(handle, self.workspace.data_ptr(), self._stream()), "ivb_decoder_bind")
        self.ctas = int(self.lib.ivb_decoder_ctas(handle))
        self.num_phases = int(self.lib.ivb_decoder_num_phases(handle))

    def __del__(self) -> None:
        plan = getattr(self, "_plan", None)
        lib = getattr(self, "lib", None)
        if plan is not None and lib is not None:
            try:
                lib.ivb_decoder_destroy(plan)
            except Exception:
                pass
            self._plan = None

    # ------------------------------------------------------------------------------------------
    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def _launch(self, steps: int, feed: Tensor | None, flags: int) -> None:
        with torch.cuda.device(self.device):
            rc = self.lib.ivb_decoder_run(
                self._plan, int(steps), 0 if feed is None else feed.data_ptr(), int(flags), self.timeout_ns, self._stream()
            )
            native.check(rc, "ivb_decoder_run")

    def _check(self) -> None:
        self._pending_check = False
        with torch.cuda.device(self.device):
            native.check(self.lib.ivb_decoder_check(self._plan, self._stream()), "decode kernel")

    def trace(self, step: int | None) -> Tensor | None:
        """Record a per-phase, per-CTA device timeline of step `step` of each following run
        (None stops). Returns the int64 [num_phases, ctas, 8] globaltimer buffer (ns): work start,
        marks inside the phase, work end."""
        if step is None:
            native.check(self.lib.ivb_decoder_trace(self._plan, None, 0), "ivb_decoder_trace")
            self._trace = None
            return None
        self._trace = torch.zeros(self.num_phases, self.ctas, 8, dtype=torch.int64, device=self.device)
        native.check(self.lib.ivb_decoder_trace(self._plan, self._trace.data_ptr(), int(step)), "ivb_decoder_trace")
        return self._trace

    def phase_kinds(self) -> list[str]:
        """Names of the ops of one token, in the order of the trace buffer's first axis."""
        kinds = []
        for index in range(len(self.layer_matrices)):
            if index in self.recurrent_states:
                kinds += [f"L{index}.entry_ssm", f"L{index}.out", f"L{index}.gate_up", f"L{index}.down"]
            else:
                kinds += [f"L{index}.entry", f"L{index}.attention", f"L{index}.out", f"L{index}.gate_up", f"L{index}.down"]
        return kinds + ["head", "merge"]

    @property
    def weight_bytes(self) -> int:
        total = self.head.nbytes
        for mats in self.layer_matrices:
            total += sum(m.nbytes for m in mats.values())
        return total

    @property
    def tile_prefill(self) -> bool:
        return True

    @property
    def persisted_bytes(self) -> int:
        return 0

    # ------------------------------------------------------------------------------------------
    @torch.no_grad()
    def prefill(self, input_ids: Tensor) -> Tensor:
        """Run the prompt and return its last logits (tensor-core prefill, or token by token)."""

        if input_ids.ndim != 2 or input_ids.shape[0] != self.batch_size:
            raise ValueError(f"input_ids must have shape [{self.batch_size}, seq_len]")
        length = int(input_ids.shape[1])
        if length == 0 or length > self.max_len:
            raise ValueError("prompt length must lie within the decoder capacity")
        if input_ids.device.type == "cpu" and input_ids.numel():
            low, high = int(input_ids.min()), int(input_ids.max())
            if low < 0 or high >= self.vocab:
                raise IndexError(f"token id is out of range for vocab_size={self.vocab}")
        ids = input_ids[0].to(device=self.device, dtype=torch.int64).contiguous()
        for state in self.recurrent_states.values():
            for buffer in state.values():
                buffer.zero_()
        self.position.zero_()
        self.host_position = 0
        self._feed = ids
        if self.prefill_mode == "steps":
            self._launch(length, ids, 0)
        else:
            self._prefill_gemm(ids)
        # the device error word is read by the next step or sample (as the reference's prefill, this
        # call does not wait for the GPU, so prefills of several decoders on their own streams overlap)
        self._pending_check = True
        self.host_position = length
        return self.logits

    def _prefill_gemm(self, ids: Tensor) -> None:
        """All prompt tokens per layer at once (tcgen05 GEMMs), in chunks of prefill_chunk tokens."""

        chunk = min(self.prefill_chunk, self.max_len)
        with torch.cuda.device(self.device):
            nbytes = int(self.lib.ivb_decoder_prefill_workspace_bytes(self._plan, chunk))
            if self._prefill_ws is None or self._prefill_ws.numel() < nbytes:
                self._prefill_ws = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
            for start in range(0, int(ids.numel()), chunk):
                part = ids[start:start + chunk]
                rc = self.lib.ivb_decoder_prefill(self._plan, part.data_ptr(), int(part.numel()), start,
                                                  self._prefill_ws.data_ptr(), self._prefill_ws.numel(), self._stream())
                native.check(rc, "ivb_decoder_prefill")

    def _step(self, length: int) -> None:
        """One token through the kernel (the reference step's contract, decoder.py:307-322): feeds
        self.token, advances self.position and, when sampling, samples the next token into it."""

        if self._pending_check and not torch.cuda.is_current_stream_capturing():
            self._check()  # a failed prefill is reported before anything runs on its state
        self._launch(1, self.token, native.IVB_RUN_SAMPLE if self.sampling else 0)
        if not torch.cuda.is_current_stream_capturing():
            self._check()

    def _run_step(self) -> None:
        super()._run_step()
        self._check()  # errors of a replayed graph surface here

    def _sample(self) -> None:
        if self._pending_check and not torch.cuda.is_current_stream_capturing():
            self._check()
        self._launch(0, None, native.IVB_RUN_SAMPLE_ONLY)
        if not torch.cuda.is_current_stream_capturing():
            self._check()

    @torch.no_grad()
    def advance_many(self, count: int) -> list[int]:
        """Produce ``count`` tokens, each fed back into the next step, in one kernel launch."""

        if not self.sampling:
            raise RuntimeError("this decoder was created without sampling")
        count = int(count)
        if count <= 0:
            return []
        room = self.max_len - self.host_position
        run = min(count, room)
        tokens: list[int] = []
        if run > 0:
            if run == BURST and self._burst_graph is not None:
                self._burst_graph.replay()
            else:
                self._launch(run, None, native.IVB_RUN_SAMPLE)
            self._check()
            tokens = self.history[:run].tolist()
            self.host_position += run
        if run < count:
            self.attention_length(self.host_position)
        return tokens

    @torch.no_grad()
    def capture(self, warmup_steps: int = 2) -> bool:
        """The reference's one-step graph (decoder.py:403-433) plus a 16-token burst graph when sampling
        (as kernel_decoder.py:482-512 adds); the decoder state the warm-up steps touch is restored."""

        if self.device.type != "cuda" or not torch.cuda.is_available():
            return False
        saved_rng = self.rng.clone()
        saved_seen = self.seen.clone()
        saved_states = {i: {k: v.clone() for k, v in s.items()} for i, s in self.recurrent_states.items()}
        saved_position = int(self.position)
        saved_token = self.token.clone()
        captured = super().capture(warmup_steps)
        burst = None
        if captured and self.sampling and self.max_len >= BURST:
            try:
                stream = torch.cuda.Stream(device=self.device)
                stream.wait_stream(torch.cuda.current_stream(self.device))
                with torch.cuda.stream(stream):
                    self.position.zero_()
                    self._launch(BURST, None, native.IVB_RUN_SAMPLE)
                    torch.cuda.synchronize(self.device)
                    graph = torch.cuda.CUDAGraph()
                    self.position.zero_()
                    with torch.cuda.graph(graph, stream=stream):
                        self._launch(BURST, None, native.IVB_RUN_SAMPLE)
                torch.cuda.synchronize(self.device)
                self._check()
                burst = graph
            except Exception:
                burst = None
        self._burst_graph = burst
        self.burst_size = BURST if burst is not None else 1
        self.position.fill_(saved_position)
        self.token.copy_(saved_token)
        self.rng.copy_(saved_rng)
        self.seen.copy_(saved_seen)
        for i, state in saved_states.items():
            for key, value in state.items():
                self.recurrent_states[i][key].copy_(value)
        return captured

    @torch.no_grad()
    def self_check(self) -> None:
        """Prefill a prompt whole and token by token; both must agree (reference kernel_decoder.py:525-549)."""

        vocab = self.vocab
        length = min(32 + 16 + 1, self.max_len)
        ids = torch.randint(2, vocab, (1, length), generator=torch.Generator().manual_seed(0))
        whole = self.prefill(ids).clone()
        self._check()
        self.prefill(ids[:, :1])
        for index in range(1, length):
            self.step(ids[:, index])
        stepped = self.logits.clone()
        sampled = int(self.token[0])
        self.reset()
        scale = float(whole.norm())
        if not (bool(torch.isfinite(whole).all()) and bool(torch.isfinite(stepped).all())) or scale == 0.0:
            raise KernelError("the B200 kernels produced invalid numbers on this GPU")
        difference = float((whole - stepped).norm()) / scale
        if difference > SELF_CHECK_TOLERANCE:
            raise KernelError(f"the B200 kernels disagree with themselves on this GPU ({difference:.1e})")
        if not 0 <= sampled < vocab:
            raise KernelError("the B200 sampler returned an invalid token on this GPU")


def kernel_decoder(model, target: torch.device, sampling: bool, max_top_k: int) -> tuple[B200Decoder, str | None]:
    """Drop-in for the reference's CUDA slot ``_kernel_decoder(model, target, sampling, max_top_k)``
    (decoder.py:518-529): a self-checked decoder and no note (prompts always run through the tensor-core
    prefill, so no torch weights are materialised). Binding it there makes the reference's build_decoder,
    Engine.load, verify_model and run_benchmark serve B200Decoder."""

    decoder = B200Decoder(model, device=target, sampling=sampling, max_top_k=max_top_k)
    decoder.self_check()
    return decoder, None


def build_decoder(model, device: str | torch.device, sampling: bool = False, max_top_k: int = 256,
                  kernels: bool = True) -> tuple[object, str, str | None]:
    """The decoder the engine serves (reference decoder.py:479-507 with its CUDA kernel slot,
    ``_kernel_decoder`` at :518-529, filled by ``kernel_decoder``).

    CUDA with kernels: a self-checked B200Decoder, backend "ternary". When it cannot run there, or for
    any other device, the reference's own ``build_decoder`` decides (its numba CPU decoder or its torch
    decoder), with the B200 failure as the note.
    """

    target = torch.device(device)
    reference_build = _reference.module("decoder").build_decoder
    if kernels and target.type == "cuda":
        try:
            decoder, note = kernel_decoder(model, target, sampling, max_top_k)
            return decoder, "ternary", note
        except Exception as exc:
            note = f"B200 ternary kernels unavailable, using the torch decoder: {exc}"
        decoder, backend, _ = reference_build(model, target, sampling=sampling, max_top_k=max_top_k, kernels=False)
        return decoder, backend, note
    return reference_build(model, target, sampling=sampling, max_top_k=max_top_k, kernels=kernels)
