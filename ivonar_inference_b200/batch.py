"""Batched decode of independent sequences on one B200 (benchmark configuration 3).

`B200BatchDecoder` advances `batch` sequences one token per step together through
`ivb_batch_decode`: every projection of every layer runs once per step as a tcgen05 GEMM over the
batch (the weights stream once for all sequences), while the SSM step, the latent-cache append, the
latent attention and the sampler run per sequence on that sequence's own state. Prompts are prefilled
one sequence at a time by a `B200Decoder` (the tensor-core prefill) whose state is then copied into
the sequence's slot. The reference's `StaticDecoder` takes a `batch_size` (decoder.py:67,96) but its
GPU kernels decode one sequence; there is no batched kernel path to mirror beyond that surface.
"""

from __future__ import annotations

import ctypes
from collections.abc import Sequence

import torch
from torch import Tensor

from . import _native as native
from .decoder import B200Decoder


class B200BatchDecoder:
    """`batch` sequences of one model decoded together; sampling per sequence (own seed and flags)."""

    def __init__(self, model, batch: int, max_len: int | None = None, device: str | torch.device | None = None,
                 max_top_k: int = 256, history_len: int = 1024, graphs: bool = True) -> None:
        if batch <= 0:
            raise ValueError("batch must be positive")
        self.base = B200Decoder(model, max_len=max_len, device=device, sampling=True, max_top_k=max_top_k)
        base = self.base
        dev = base.device
        self.device = dev
        self.batch = int(batch)
        self.max_len = base.max_len
        self.vocab = base.vocab
        self.lib = native.library()
        layers = (native.IvbBatchLayer * len(base.layer_matrices))()
        self.states: dict[int, dict[str, Tensor]] = {}
        self.caches: dict[int, tuple[Tensor, Tensor, Tensor]] = {}
        for index in range(len(base.layer_matrices)):
            desc = layers[index]
            if index in base.recurrent_states:
                one = base.recurrent_states[index]
                taps = int(base._layers[index].conv_taps)
                hidden = int(one["conv_state"].shape[1])
                state = {
                    "ssm_state": torch.zeros((batch,) + tuple(one["ssm_state"].shape[1:]), device=dev),
                    "prev_force": torch.zeros((batch,) + tuple(one["prev_force"].shape[1:]), device=dev),
                    "conv_state": torch.zeros(batch, hidden, taps - 1, device=dev),
                }
                self.states[index] = state
                desc.ssm_state = state["ssm_state"].data_ptr()
                desc.prev_force = state["prev_force"].data_ptr()
                desc.conv_state = state["conv_state"].data_ptr() if state["conv_state"].numel() else None
            else:
                latent_q, latent_scale, k_rope = base.latent_caches[index]
                cache = (
                    torch.zeros((batch,) + tuple(latent_q.shape), dtype=torch.int8, device=dev),
                    torch.zeros(batch, self.max_len, dtype=torch.float32, device=dev),
                    torch.zeros((batch,) + tuple(k_rope.shape), dtype=torch.float16, device=dev),
                )
                self.caches[index] = cache
                desc.latent_q = cache[0].data_ptr()
                desc.latent_scale = cache[1].data_ptr()
                desc.k_rope_cache = cache[2].data_ptr()
        self._layers = layers
        self.tokens = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.positions = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.logits = torch.zeros(batch, self.vocab, dtype=torch.float32, device=dev)
        self.seen = torch.zeros(batch, self.vocab, dtype=torch.uint8, device=dev)
        self.rng = torch.zeros(batch, 2, dtype=torch.int64, device=dev)
        self.history = torch.zeros(batch, int(history_len), dtype=torch.int64, device=dev)
        self.step_counter = torch.zeros(1, dtype=torch.int32, device=dev)
        self.use_graphs = bool(graphs)
        self._graph: torch.cuda.CUDAGraph | None = None
        self.host_positions = [0] * batch
        spec = native.IvbBatch()
        spec.batch = batch
        spec.layers = ctypes.cast(layers, ctypes.POINTER(native.IvbBatchLayer))
        spec.tokens = self.tokens.data_ptr()
        spec.positions = self.positions.data_ptr()
        spec.logits = self.logits.data_ptr()
        spec.seen = self.seen.data_ptr()
        spec.rng = self.rng.data_ptr()
        spec.history = self.history.data_ptr()
        spec.history_len = int(history_len)
        spec.step = self.step_counter.data_ptr()
        spec.sampling = base._sampling.data_ptr()
        spec.top_k = base.top_k.data_ptr()
        self._spec = spec
        nbytes = int(self.lib.ivb_batch_workspace_bytes(base._plan, batch))
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=dev)

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    @torch.no_grad()
    def start(self, prompts: Sequence[Tensor], seeds: Sequence[int], temperature: float, top_k: int,
              repetition_penalty: float = 1.0) -> list[int]:
        """Prefill every sequence's prompt and sample its first token; returns those tokens."""

        if len(prompts) != self.batch or len(seeds) != self.batch:
            raise ValueError(f"need {self.batch} prompts and seeds")
        base = self.base
        first: list[int] = []
        for b, (prompt, seed) in enumerate(zip(prompts, seeds)):
            ids = prompt.reshape(1, -1)
            base.prefill(ids)
            base.configure_sampling(temperature, top_k, repetition_penalty)
            base.rng.copy_(torch.tensor([int(seed), 0], dtype=torch.int64))
            first.append(base.sample())
            for index, state in self.states.items():
                one = base.recurrent_states[index]
                state["ssm_state"][b].copy_(one["ssm_state"][0])
                state["prev_force"][b].copy_(one["prev_force"][0])
                if state["conv_state"].numel():
                    state["conv_state"][b].copy_(one["conv_state"][0, :, : state["conv_state"].shape[2]])
            for index, cache in self.caches.items():
                latent_q, latent_scale, k_rope = base.latent_caches[index]
                cache[0][b].copy_(latent_q)
                cache[1][b].copy_(latent_scale[: self.max_len])
                cache[2][b].copy_(k_rope)
            self.tokens[b] = base.token[0]
            self.positions[b] = base.host_position
            self.seen[b].copy_(base.seen[0].to(torch.uint8))
            self.rng[b].copy_(base.rng)
            self.logits[b].copy_(base.logits[0])
            self.host_positions[b] = base.host_position
        self.step_counter.zero_()
        return first

    @torch.no_grad()
    def decode(self, steps: int) -> Tensor:
        """Feed every sequence's last token `steps` times; returns the sampled tokens [batch, steps]."""

        steps = int(steps)
        if steps <= 0:
            return self.history[:, :0]
        if max(self.host_positions) + steps > self.max_len:
            raise ValueError("the batch has no free position left (capacity)")
        done = int(self.step_counter.item())
        if done + steps > self.history.shape[1]:
            raise ValueError("steps exceed the history length of this batch decoder")
        if not self.use_graphs:
            self._launch(steps)
        else:
            run = steps
            if self._graph is None:
                # one step runs eagerly (first-use setup happens outside capture), then one step is captured
                self._launch(1)
                run -= 1
                if run > 0:
                    self._capture()
            for _ in range(run):
                self._graph.replay()
        self.base._check()
        self.host_positions = [p + steps for p in self.host_positions]
        return self.history[:, done:done + steps]

    def _launch(self, steps: int) -> None:
        rc = self.lib.ivb_batch_decode(self.base._plan, ctypes.byref(self._spec), steps, self.workspace.data_ptr(),
                                       self.workspace.numel(), self._stream())
        native.check(rc, "ivb_batch_decode")

    def _capture(self) -> None:
        """One batched step as a CUDA graph (its launches replayed without host work per kernel)."""

        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            rc = self.lib.ivb_batch_decode(self.base._plan, ctypes.byref(self._spec), 1, self.workspace.data_ptr(),
                                           self.workspace.numel(), self._stream())
        native.check(rc, "ivb_batch_decode (capture)")
        self._graph = graph
