"""Tensor-parallel batched decode (benchmark configuration 4: the 7B-shaped model over 2/4/8 B200).

Each rank holds a shard of every block: the mixer by heads (mamba: the value/gate channels and the
B, C, dt rows of its heads, their SSM constants and state; mla: the q and k_rope rows, k_nope/v
up-projection rows of its heads, the latent projection replicated), the FFN by 128-input groups of the
hidden dimension (gate/up rows column-parallel, down columns row-parallel), and the out projections
row-parallel. Per block and step:

    quantise(resid, norm) -> entry GEMM (shard) -> mixer (shard heads) -> all-reduce MAX of the row amax
    -> quantise(y shard, global amax) -> out GEMM (shard columns, partial) -> all-reduce SUM -> resid +=
    quantise(resid, ffn norm) -> gate/up GEMM (shard) -> all-reduce MAX -> quantise(h shard, global amax)
    -> down GEMM (shard columns, partial) -> all-reduce SUM -> resid +=

The all-reduces are NCCL collectives over NVLink (torch.distributed, backend "nccl") on the stream
the kernels run on; the global amax keeps every shard's activation codes equal to the unsharded
quantiser's, so a sharded step differs from one GPU's only in the order of the fp32 partial sums.
The embedding is replicated; the head is sharded by vocabulary rows: each rank computes the logits of
its slice and their top-k candidates (`ivb_batch_topk_slice`), an NCCL all-gather brings every rank's
candidates to every rank, and each rank runs the same merge and Philox draw (`ivb_batch_sample_merge`),
so all ranks sample the token the unsharded sampler would (same seeds). The kernels are the batched
decode's unit steps (`ivb_batch_*`, `ivb_ternary_gemm`, `ivb_quantize_rows[_amax]`). Prompts run through
the same step teacher-forced, one token per step.
"""

from __future__ import annotations

import ctypes
import math

import torch
import torch.nn.functional as F
from torch import Tensor

from . import _native as native
from .decoder import DeviceMatrix, rope_from_rotary


def split_even(total: int, parts: int, unit: int = 1) -> list[tuple[int, int]]:
    """`total` items in `parts` contiguous ranges whose bounds are multiples of `unit` (the last may end at
    `total`), sizes differing by at most one unit."""

    units = math.ceil(total / unit)
    base, extra = divmod(units, parts)
    out, lo = [], 0
    for p in range(parts):
        n = base + (1 if p < extra else 0)
        hi = min(total, (lo // unit + n) * unit) if n else lo
        out.append((lo, hi))
        lo = hi
    return out


class Shard:
    """A slice of a packed projection: the attributes DeviceMatrix reads (packed uint8 rows, fp16 group
    scales, optional fp32 bias, widths), in the checkpoint's q2_g128 layout."""

    def __init__(self, packed_weight: Tensor, weight_scales: Tensor, in_features: int, bias: Tensor | None,
                 group_size: int = 128, eps: float = 1e-5) -> None:
        self.packed_weight = packed_weight
        self.weight_scales = weight_scales
        self.in_features = int(in_features)
        self.out_features = int(packed_weight.shape[0])
        self.bias = bias
        self.group_size = int(group_size)
        self.eps = float(eps)


def row_slice(t, r0: int, r1: int) -> Shard:
    bias = None if t.bias is None else t.bias[r0:r1]
    return Shard(t.packed_weight[r0:r1], t.weight_scales[r0:r1], t.in_features, bias, group_size=t.group_size, eps=t.eps)


def col_slice(t, k0: int, k1: int, keep_bias: bool) -> Shard:
    """Inputs [k0, k1) of a matrix. The shard keeps the q2_g128 layout: either it starts on a 128-input
    group boundary (and ends on one, or at the end), or it lies inside one group (its one scale column)."""

    inside = k0 % 4 == 0 and k0 // 128 == (k1 - 1) // 128
    aligned = k0 % 128 == 0 and (k1 % 128 == 0 or k1 == t.in_features)
    if not (inside or aligned):
        raise ValueError("column shards must follow the 128-input scale groups")
    packed = t.packed_weight[:, k0 // 4: (k1 + 3) // 4]
    scales = t.weight_scales[:, k0 // 128: (k1 - 1) // 128 + 1]
    return Shard(packed.contiguous(), scales.contiguous(), k1 - k0, t.bias if keep_bias else None,
                 group_size=t.group_size, eps=t.eps)


class B200TensorParallel:
    """`batch` sequences decoded with the blocks sharded over `world` ranks (this process is `rank`)."""

    def __init__(self, model, rank: int, world: int, group=None, batch: int = 1, max_len: int = 1024,
                 device: str | torch.device | None = None, max_top_k: int = 256, history_len: int = 1024,
                 graphs: bool = True) -> None:
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.device, self.rank, self.world, self.group = dev, int(rank), int(world), group
        self.batch, self.max_len, self.max_top_k = int(batch), int(max_len), int(max_top_k)
        self.lib = native.library()
        config = model.config
        d, H = int(config.hidden_dim), int(config.num_heads)
        hd = d // H
        if H % world:
            raise ValueError(f"{H} heads do not split over {world} ranks")
        self.hidden, self.heads_local, self.head_dim = d, H // world, hd
        h0, h1 = rank * self.heads_local, (rank + 1) * self.heads_local
        c0, c1 = h0 * hd, h1 * hd
        self.channels = c1 - c0
        self.vocab = int(model.token_io.projection.out_features)
        first = model.blocks[0].ffn.down_proj
        self.f_range = split_even(int(first.in_features), world, 128)[rank]
        f0, f1 = self.f_range
        self.ffn_local = f1 - f0
        if self.ffn_local <= 0:
            raise ValueError(f"{first.in_features} FFN inputs do not fill {world} shards of 128-input groups")
        self.head = DeviceMatrix([model.token_io.projection], dev)  # the embedding rows (replicated)
        # this rank's vocabulary slice of the head (rows in 128-row units, so the slices tile the GEMM)
        self.v_range = split_even(self.vocab, world, 128)[rank]
        v0, v1 = self.v_range
        self.vloc = v1 - v0
        if self.vloc <= 0:
            raise ValueError(f"{self.vocab} vocabulary rows do not fill {world} shards of 128 rows")
        self.head_shard = DeviceMatrix([row_slice(model.token_io.projection, v0, v1)], dev)
        self.final_norm = model.final_norm.weight.float().to(dev).contiguous()
        self.final_eps = float(model.final_norm.eps)
        self.act_eps = float(getattr(model.token_io.projection, "eps", 1e-5))
        self._keep: list = []
        self.layers = []
        self.batch_layers = (native.IvbBatchLayer * len(model.blocks))()
        self.descs = (native.IvbLayerDesc * len(model.blocks))()
        B = self.batch
        ent_rows = 0
        for index, block in enumerate(model.blocks):
            mixer, kind = block.mixer, getattr(block, "mixer_type", None)
            desc, state = self.descs[index], self.batch_layers[index]
            norm_m = block.mixer_norm.weight.float().to(dev).contiguous()
            norm_f = block.ffn_norm.weight.float().to(dev).contiguous()
            self.norm_clip = float(getattr(block.mixer_norm, "clip", 8.0))
            desc.mixer_norm, desc.mixer_norm_eps = norm_m.data_ptr(), float(block.mixer_norm.eps)
            desc.ffn_norm, desc.ffn_norm_eps = norm_f.data_ptr(), float(block.ffn_norm.eps)
            keep = [norm_m, norm_f]
            if kind == "mamba":
                desc.kind = native.IVB_MAMBA
                S = int(mixer.state_dim)
                value = row_slice(mixer.in_proj, c0, c1)
                gate = row_slice(mixer.in_proj, d + c0, d + c1)
                bcdt = row_slice(mixer.bc_dt_proj, h0 * 3 * S, h1 * 3 * S)
                entry = DeviceMatrix([value, gate, bcdt], dev)
                taps = int(mixer.conv_kernel_size)
                consts = {
                    "decay": (-F.softplus(mixer.log_decay.float()))[h0:h1].contiguous(),
                    "theta": mixer.theta.float()[h0:h1].contiguous(),
                    "skip": mixer.skip.float().reshape(-1)[c0:c1].contiguous(),
                    "conv_weight": mixer.conv_weight.float().reshape(d, taps)[c0:c1].contiguous(),
                    "conv_bias": mixer.conv_bias.float()[c0:c1].contiguous(),
                }
                consts = {k: v.to(dev) for k, v in consts.items()}
                keep += list(consts.values())
                for key in ("decay", "theta", "skip", "conv_weight", "conv_bias"):
                    setattr(desc, key, consts[key].data_ptr())
                desc.conv_taps = taps
                desc.half_dt_min = 0.5 * float(mixer.dt_min)
                desc.half_dt_range = 0.5 * (float(mixer.dt_max) - float(mixer.dt_min))
                st = {
                    "ssm_state": torch.zeros(B, self.heads_local, S, hd, 2, device=dev),
                    "prev_force": torch.zeros(B, self.heads_local, S, hd, device=dev),
                    "conv_state": torch.zeros(B, self.channels, max(taps - 1, 0), device=dev),
                }
                keep += list(st.values())
                state.ssm_state, state.prev_force = st["ssm_state"].data_ptr(), st["prev_force"].data_ptr()
                state.conv_state = st["conv_state"].data_ptr() if st["conv_state"].numel() else None
                self.state_dim = S
                layer = {"kind": "mamba", "entry": entry, "state": st}
            elif kind == "mla":
                desc.kind = native.IVB_MLA
                rope, nope, Lt = int(mixer.rope_dim), int(mixer.nope_dim), int(mixer.latent_dim)
                q = row_slice(mixer.q_proj, c0, c1)
                k_rope = row_slice(mixer.k_rope_proj, h0 * rope, h1 * rope)
                entry = DeviceMatrix([q, mixer.kv_down_proj, k_rope], dev)
                kn = DeviceMatrix([row_slice(mixer.k_nope_up_proj, h0 * nope, h1 * nope)], dev, scale_align=8)
                vu = DeviceMatrix([row_slice(mixer.v_up_proj, c0, c1)], dev, scale_align=8)
                table = rope_from_rotary(mixer.rope, self.max_len).to(dev)
                lpad, rpad = (Lt + 15) // 16 * 16, (rope + 7) // 8 * 8
                cache = (
                    torch.zeros(B, self.max_len, lpad, dtype=torch.int8, device=dev),
                    torch.zeros(B, self.max_len, dtype=torch.float32, device=dev),
                    torch.zeros(B, self.heads_local, self.max_len, rpad, dtype=torch.float16, device=dev),
                )
                keep += [table, *cache]
                desc.k_nope_up, desc.v_up = kn.desc(), vu.desc()
                desc.rope = table.data_ptr()
                desc.attn_scale = 1.0 / math.sqrt(hd)
                state.latent_q, state.latent_scale, state.k_rope_cache = (c.data_ptr() for c in cache)
                self.latent, self.rope, self.nope = Lt, rope, nope
                layer = {"kind": "mla", "entry": entry, "k_nope_up": kn, "v_up": vu, "cache": cache}
            else:
                raise native.KernelError(f"unsupported mixer for the B200 kernels: {type(mixer).__name__}")
            out = DeviceMatrix([col_slice(mixer.out_proj, c0, c1, keep_bias=rank == 0)], dev)
            gate_up = DeviceMatrix([row_slice(block.ffn.gate_proj, f0, f1), row_slice(block.ffn.up_proj, f0, f1)], dev,
                                   interleave=True)
            down = DeviceMatrix([col_slice(block.ffn.down_proj, f0, f1, keep_bias=rank == 0)], dev)
            layer.update(out=out, gate_up=gate_up, down=down)
            desc.entry, desc.out, desc.gate_up, desc.down = (layer[k].desc() for k in ("entry", "out", "gate_up", "down"))
            ent_rows = max(ent_rows, layer["entry"].rows)
            self._keep.append(keep)
            self.layers.append(layer)
        ldq = (max(d, self.ffn_local, self.channels) + 127) // 128 * 128
        rows128 = (B + 127) // 128 * 128
        f32 = dict(dtype=torch.float32, device=dev)
        self.resid, self.partial = torch.zeros(B, d, **f32), torch.zeros(B, d, **f32)
        self.ent = torch.zeros(B, ent_rows, **f32)
        self.y = torch.zeros(B, self.channels, **f32)
        self.h = torch.zeros(B, self.ffn_local, **f32)
        self.q8 = torch.zeros(rows128, ldq, dtype=torch.int8, device=dev)
        self.act_scale, self.amax = torch.zeros(B, **f32), torch.zeros(B, **f32)
        self.logits = torch.zeros(B, self.vloc, **f32)  # this rank's slice
        self.seen = torch.zeros(B, self.vloc, dtype=torch.uint8, device=dev)
        # sampler candidates: this rank's top-k per sequence, and every rank's after the all-gather
        self.kc = max(2, min(self.max_top_k, self.vocab, 256))
        self.cand_keys = torch.zeros(B, self.kc, dtype=torch.int32, device=dev)
        self.cand_ids = torch.zeros(B, self.kc, dtype=torch.int32, device=dev)
        self.all_keys = torch.zeros(world, B, self.kc, dtype=torch.int32, device=dev)
        self.all_ids = torch.zeros(world, B, self.kc, dtype=torch.int32, device=dev)
        self.tokens = torch.zeros(B, dtype=torch.int64, device=dev)
        self.positions = torch.zeros(B, dtype=torch.int64, device=dev)
        self.rng = torch.zeros(B, 2, dtype=torch.int64, device=dev)
        self.history = torch.zeros(B, int(history_len), dtype=torch.int64, device=dev)
        self.step_counter = torch.zeros(1, dtype=torch.int32, device=dev)
        self.sampling = torch.ones(3, **f32)
        self.top_k = torch.ones(1, dtype=torch.int64, device=dev)
        self.error = torch.zeros(1, dtype=torch.int32, device=dev)
        self.host_position = 0
        self.use_graphs = bool(graphs)
        self._graph: torch.cuda.CUDAGraph | None = None

    # ------------------------------------------------------------------------------------------
    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def _all_reduce(self, t: Tensor, op) -> None:
        if self.world > 1:
            torch.distributed.all_reduce(t, op=op, group=self.group)

    def _quant(self, x: Tensor, n: int, norm, eps: float) -> None:
        ldq = (n + 127) // 128 * 128
        native.check(self.lib.ivb_quantize_rows(x.data_ptr(), self.batch, n, norm, eps, self.norm_clip, self.act_eps,
                                                self.q8.data_ptr(), ldq, self.act_scale.data_ptr(), None, self._stream()),
                     "ivb_quantize_rows")

    def _quant_shard(self, x: Tensor, n: int) -> None:
        """Quantise a row-parallel input shard with the amax of the whole row."""

        native.check(self.lib.ivb_rows_amax(x.data_ptr(), self.batch, n, self.amax.data_ptr(), self._stream()), "ivb_rows_amax")
        self._all_reduce(self.amax, torch.distributed.ReduceOp.MAX if self.world > 1 else None)
        ldq = (n + 127) // 128 * 128
        native.check(self.lib.ivb_quantize_rows_amax(x.data_ptr(), self.batch, n, self.amax.data_ptr(), self.act_eps,
                                                     self.q8.data_ptr(), ldq, self.act_scale.data_ptr(), self._stream()),
                     "ivb_quantize_rows_amax")

    def _sample(self, history: bool) -> None:
        """Every rank draws the same token per sequence from the candidates of all vocabulary slices."""

        st = self._stream()
        v0 = self.v_range[0]
        native.check(self.lib.ivb_batch_topk_slice(self.logits.data_ptr(), self.seen.data_ptr(), self.vloc, v0, self.vocab,
                                                   self.batch, self.sampling.data_ptr(), self.top_k.data_ptr(),
                                                   self.max_top_k, self.kc, self.cand_keys.data_ptr(),
                                                   self.cand_ids.data_ptr(), st), "ivb_batch_topk_slice")
        if self.world > 1:
            torch.distributed.all_gather_into_tensor(self.all_keys, self.cand_keys, group=self.group)
            torch.distributed.all_gather_into_tensor(self.all_ids, self.cand_ids, group=self.group)
        else:
            self.all_keys[0].copy_(self.cand_keys)
            self.all_ids[0].copy_(self.cand_ids)
        native.check(self.lib.ivb_batch_sample_merge(
            self.all_keys.data_ptr(), self.all_ids.data_ptr(), self.world, self.batch, self.kc, self.vocab,
            self.top_k.data_ptr(), self.max_top_k, self.rng.data_ptr(), self.tokens.data_ptr(), self.positions.data_ptr(),
            self.history.data_ptr() if history else None, self.history.shape[1] if history else 0,
            self.step_counter.data_ptr() if history else None, self.seen.data_ptr(), v0, self.vloc, st),
            "ivb_batch_sample_merge")

    def _gemm(self, m: DeviceMatrix, epilogue: int, out: Tensor, ldo: int) -> None:
        desc = m.desc()
        ldq = (m.in_features + 127) // 128 * 128
        native.check(self.lib.ivb_ternary_gemm(ctypes.byref(desc), self.q8.data_ptr(), ldq, self.act_scale.data_ptr(),
                                               self.batch, epilogue, out.data_ptr(), ldo, self.error.data_ptr(),
                                               self._stream()), "ivb_ternary_gemm")

    def _row_parallel(self, m: DeviceMatrix) -> None:
        """partial = shard product (bias on rank 0 only); resid += all-reduce SUM(partial)."""

        self._gemm(m, native.IVB_EPI_STORE, self.partial, self.hidden)
        self._all_reduce(self.partial, torch.distributed.ReduceOp.SUM if self.world > 1 else None)
        self.resid.add_(self.partial)

    @torch.no_grad()
    def step(self, feed: Tensor | None = None, sample: bool = True) -> None:
        """One token for every sequence: `feed` [batch] teacher-forces the input tokens (no sampling)."""

        if self.host_position >= self.max_len:
            raise ValueError("the decoder has no free position left (capacity)")
        if feed is not None:
            self.tokens.copy_(feed.to(self.device, torch.int64))
        st = self._stream()
        head = self.head.desc()
        native.check(self.lib.ivb_batch_embed(ctypes.byref(head), self.tokens.data_ptr(), self.batch, self.hidden,
                                              self.resid.data_ptr(), self.step_counter.data_ptr() if sample else None, st),
                     "ivb_batch_embed")
        for index, layer in enumerate(self.layers):
            desc = self.descs[index]
            self._quant(self.resid, self.hidden, desc.mixer_norm, desc.mixer_norm_eps)
            ld = layer["entry"].rows
            self._gemm(layer["entry"], native.IVB_EPI_STORE, self.ent, ld)
            if layer["kind"] == "mamba":
                rc = self.lib.ivb_batch_ssm(ctypes.byref(desc), ctypes.byref(self.batch_layers[index]), self.ent.data_ptr(), ld,
                                            self.batch, self.channels, self.heads_local, self.head_dim, self.state_dim,
                                            self.y.data_ptr(), st)
                native.check(rc, "ivb_batch_ssm")
            else:
                rc = self.lib.ivb_batch_mla(ctypes.byref(desc), ctypes.byref(self.batch_layers[index]), self.ent.data_ptr(), ld,
                                            self.positions.data_ptr(), self.batch, self.channels, self.latent,
                                            self.heads_local, self.head_dim, self.rope, self.nope, self.max_len,
                                            self.act_eps, self.error.data_ptr(), self.y.data_ptr(), st)
                native.check(rc, "ivb_batch_mla")
            self._quant_shard(self.y, self.channels)
            self._row_parallel(layer["out"])
            self._quant(self.resid, self.hidden, desc.ffn_norm, desc.ffn_norm_eps)
            self._gemm(layer["gate_up"], native.IVB_EPI_SILU_PAIR, self.h, self.ffn_local)
            self._quant_shard(self.h, self.ffn_local)
            self._row_parallel(layer["down"])
        self._quant(self.resid, self.hidden, self.final_norm.data_ptr(), self.final_eps)
        self._gemm(self.head_shard, native.IVB_EPI_STORE, self.logits, self.vloc)
        if sample:
            self._sample(history=True)
        else:
            self.positions.add_(1)
        self.host_position += 1

    @torch.no_grad()
    def start(self, prompts: Tensor, seeds, temperature: float, top_k: int, repetition_penalty: float = 1.0) -> None:
        """Run the prompts [batch, T] teacher-forced, then configure sampling (per-sequence seeds)."""

        if prompts.shape[0] != self.batch:
            raise ValueError(f"prompts must have {self.batch} rows")
        if temperature <= 0 or repetition_penalty <= 0:
            raise ValueError("temperature and repetition_penalty must be positive")
        for t in (self.positions, self.seen, self.step_counter, self.error):
            t.zero_()
        for layer in self.layers:
            for buf in layer.get("state", {}).values():
                buf.zero_()
        self.host_position = 0
        for t in range(int(prompts.shape[1])):
            self.step(prompts[:, t], sample=False)
        self.sampling[0], self.sampling[1], self.sampling[2] = float(temperature), float(repetition_penalty), 1.0 / float(repetition_penalty)
        self.top_k.fill_(int(top_k) if 0 < int(top_k) <= self.max_top_k else self.max_top_k)
        self.rng[:, 0] = torch.as_tensor([int(s) for s in seeds], dtype=torch.int64, device=self.device)
        self.rng[:, 1] = 0
        # the first sampled token comes from the prompt's last logits
        self._sample(history=False)
        self.positions.sub_(1)  # the sampler advanced the position; the sampled token is fed at the same slot

    @torch.no_grad()
    def decode(self, steps: int) -> Tensor:
        """`steps` sampled tokens per sequence (each fed back); returns them [batch, steps]. After one eager
        step, a whole step (kernels and NCCL all-reduces) is captured once as a CUDA graph and replayed."""

        steps = int(steps)
        done = int(self.step_counter.item())
        if self.host_position + steps > self.max_len:
            raise ValueError("the decoder has no free position left (capacity)")
        run = steps
        if self.use_graphs and run > 0 and self._graph is None:
            self.step()
            run -= 1
            if run > 0:
                graph = torch.cuda.CUDAGraph()
                position = self.host_position
                with torch.cuda.graph(graph):
                    self.step()
                self.host_position = position  # capture records the step without running it
                self._graph = graph
        for _ in range(run):
            if self._graph is not None:
                self._graph.replay()
                self.host_position += 1
            else:
                self.step()
        if int(self.error.item()) != 0:
            raise native.KernelError(f"tensor-parallel step reported error {int(self.error.item())}")
        return self.history[:, done:done + int(steps)]
