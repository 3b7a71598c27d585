"""CPU oracle of the Ivonar token loop. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module; the
product package (ivonar_inference_b200) never does. It drives the C restatement in
ivonar_oracle.c (liboracle.so) through the reference's decode order:
  embed -> per block [norm+quant -> entry GEMV -> recurrent step | (latent quant -> up GEMV ->
  attention with an fp32 K/V cache)] -> quant -> out GEMV (+=) -> norm+quant -> gate/up SwiGLU ->
  quant -> down GEMV (+=) -> final norm+quant -> head GEMV -> (sample)
following src/ivonar_inference/cpu_decoder.py:457-497 (CpuDecoder._numba_step) and
kernel_decoder.py:234-269 (launch order of the reference GPU decoder).
"""

from __future__ import annotations

import ctypes
import math
import subprocess
from ctypes import POINTER, c_float, c_int, c_int64, c_uint64, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "_build" / "liboracle.so"

_lib: ctypes.CDLL | None = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIBRARY


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            build()
        L = ctypes.CDLL(str(LIBRARY))
        L.orc_quantize.restype = c_float
        L.orc_quantize.argtypes = [c_void_p, c_void_p, c_int, c_float, c_float, c_float, c_void_p, c_void_p]
        L.orc_group_dots.restype = None
        L.orc_group_dots.argtypes = [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_int]
        L.orc_gemv.restype = None
        L.orc_gemv.argtypes = [c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_void_p, c_float, c_void_p, c_int, c_int]
        L.orc_embed.restype = None
        L.orc_embed.argtypes = [c_void_p, c_void_p, c_int, c_int, c_int, c_int64, c_void_p]
        L.orc_ssm_step.restype = None
        L.orc_ssm_step.argtypes = [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                   c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_float, c_void_p]
        L.orc_attention_step.restype = None
        L.orc_attention_step.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int,
                                         c_int, c_int, c_int, c_float, c_void_p]
        L.orc_sample.restype = c_int64
        L.orc_sample.argtypes = [c_void_p, c_void_p, c_int, c_float, c_float, c_float, c_int64, c_int, POINTER(c_uint64)]
        L.orc_philox_uniform.restype = c_float
        L.orc_philox_uniform.argtypes = [c_uint64, c_uint64]
        L.orc_philox4x32_10.restype = None
        L.orc_philox4x32_10.argtypes = [c_void_p, c_void_p, c_void_p]
        L.orc_set_kv_half.restype = None
        L.orc_set_kv_half.argtypes = [c_int]
        L.orc_max_threads.restype = c_int
        _lib = L
    return _lib


def _p(a: np.ndarray | None) -> int:
    return 0 if a is None else a.ctypes.data


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


# ---- primitives -------------------------------------------------------------------------------
def quantize(x, norm_w=None, norm_eps: float = 1e-6, clip: float = 8.0, act_eps: float = 1e-5):
    """(q8 int8 [n], scale float, xsum int32 [ceil(n/64)])."""
    x = _f32(x)
    w = None if norm_w is None else _f32(norm_w)
    n = x.shape[0]
    q = np.zeros(n, dtype=np.int8)
    xs = np.zeros((n + 63) // 64, dtype=np.int32)
    s = lib().orc_quantize(_p(x), _p(w), n, norm_eps, clip, act_eps, _p(q), _p(xs))
    return q, float(np.float32(s)), xs


class Matrix:
    """Row-stacked packed projections in host memory (rows padded to 16 bytes)."""

    def __init__(self, projections, interleave: bool = False) -> None:
        packed = [np.asarray(p.packed_weight.cpu().numpy(), dtype=np.uint8) for p in projections]
        scales = [p.weight_scales.cpu().contiguous().view(dtype=_torch().int16).numpy().view(np.uint16) for p in projections]
        self.in_features = int(projections[0].in_features)
        if len(projections) > 1 and interleave:
            packed_s = np.stack(packed, axis=1).reshape(-1, packed[0].shape[1])
            scales_s = np.stack(scales, axis=1).reshape(-1, scales[0].shape[1])
        else:
            packed_s = np.concatenate(packed, axis=0)
            scales_s = np.concatenate(scales, axis=0)
        rb = packed_s.shape[1]
        pad = (rb + 15) // 16 * 16
        if pad != rb:
            packed_s = np.pad(packed_s, ((0, 0), (0, pad - rb)))
        self.packed = np.ascontiguousarray(packed_s)
        self.scales = np.ascontiguousarray(scales_s)
        biases = [p.bias for p in projections]
        if all(b is None for b in biases):
            self.bias = None
        else:
            parts = [np.zeros(int(p.out_features), np.float32) if b is None else b.cpu().float().numpy() for p, b in zip(projections, biases)]
            self.bias = np.ascontiguousarray(np.stack(parts, axis=1).reshape(-1) if interleave else np.concatenate(parts))
        self.rows = self.packed.shape[0]

    @classmethod
    def raw(cls, packed: np.ndarray, scales_u16: np.ndarray, in_features: int, bias: np.ndarray | None = None) -> "Matrix":
        m = cls.__new__(cls)
        rb = packed.shape[1]
        pad = (rb + 15) // 16 * 16
        m.packed = np.ascontiguousarray(np.pad(packed, ((0, 0), (0, pad - rb))) if pad != rb else packed)
        m.scales = np.ascontiguousarray(scales_u16)
        m.bias = None if bias is None else _f32(bias)
        m.in_features = int(in_features)
        m.rows = m.packed.shape[0]
        return m

    def gemv(self, q8: np.ndarray, act_scale: float, out: np.ndarray, epilogue: int = 0, threads: int = 0) -> None:
        threads = threads or lib().orc_max_threads()
        lib().orc_gemv(_p(self.packed), _p(self.scales), self.scales.shape[1], _p(self.bias), self.rows, self.in_features,
                       self.packed.shape[1], _p(q8), act_scale, _p(out), epilogue, threads)

    def group_dots(self, q8: np.ndarray, threads: int = 0) -> np.ndarray:
        groups = (self.in_features + 127) // 128
        dots = np.zeros((self.rows, groups), dtype=np.int32)
        lib().orc_group_dots(_p(self.packed), self.rows, self.in_features, self.packed.shape[1], _p(np.ascontiguousarray(q8)),
                             _p(dots), threads or lib().orc_max_threads())
        return dots


def _torch():
    import torch

    return torch


def rope_table_np(rotary, max_len: int) -> np.ndarray:
    """[max_len, head_dim/2, (cos, sin)] of the reference RotaryEmbedding (attention.py:41-72: scaled
    inverse frequencies and positions, then cos/sin of their outer product)."""
    torch = _torch()
    dim = int(rotary.head_dim)
    inv_freq = 1.0 / (float(rotary.rope_base) ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    positions = torch.arange(0, max_len, dtype=torch.float32)
    base, active = int(rotary.base_context), int(rotary.active_context)
    ratio = active / base if active > base else 1.0
    if rotary.scaling_strategy == "linear" and ratio > 1.0:
        positions = positions / ratio
    if rotary.scaling_strategy == "yarn_like" and ratio > 1.0:
        ramp = torch.linspace(0.0, 1.0, steps=inv_freq.numel())
        inv_freq = inv_freq / (1.0 + (ratio - 1.0) * ramp.square())
    freqs = torch.einsum("s,d->sd", positions, inv_freq)
    return np.ascontiguousarray(torch.stack((freqs.cos(), freqs.sin()), dim=-1).numpy())


class OracleDecoder:
    """Batch-1 CPU decoder over the packed weights, restating the reference token loop."""

    def __init__(self, model, max_len: int | None = None, threads: int = 0, seed: int = 0) -> None:
        torch = _torch()
        cfg = model.config
        self.max_len = int(cfg.seq_len if max_len is None else max_len)
        self.vocab = int(cfg.vocab_size)
        self.hidden = int(cfg.hidden_dim)
        self.threads = threads or lib().orc_max_threads()
        self.head = Matrix([model.token_io.projection])
        self.final_norm = _f32(model.final_norm.weight.float().numpy())
        self.final_eps = float(model.final_norm.eps)
        self.act_eps = float(getattr(model.token_io.projection, "eps", 1e-5))
        self.layers = []
        mixer_width = self.hidden
        for block in model.blocks:
            m = block.mixer
            L = {
                "kind": block.mixer_type,
                "mixer_norm": _f32(block.mixer_norm.weight.float().numpy()),
                "mixer_eps": float(block.mixer_norm.eps),
                "clip": float(block.mixer_norm.clip),
                "ffn_norm": _f32(block.ffn_norm.weight.float().numpy()),
                "ffn_eps": float(block.ffn_norm.eps),
                "gate_up": Matrix([block.ffn.gate_proj, block.ffn.up_proj], interleave=True),
                "down": Matrix([block.ffn.down_proj]),
            }
            if block.mixer_type == "mamba":
                taps = int(m.conv_kernel_size)
                L.update(
                    entry=Matrix([m.in_proj, m.bc_dt_proj]), out=Matrix([m.out_proj]), heads=m.num_heads,
                    state_dim=m.state_dim, head_dim=m.head_dim, taps=taps,
                    conv_w=_f32(m.conv_weight.float().reshape(self.hidden, taps).numpy()),
                    conv_b=_f32(m.conv_bias.float().numpy()),
                    decay=_f32((-torch.nn.functional.softplus(m.log_decay.float())).numpy()),
                    theta=_f32(m.theta.float().numpy()), skip=_f32(m.skip.float().reshape(-1).numpy()),
                    hdmin=0.5 * float(m.dt_min), hdrange=0.5 * (float(m.dt_max) - float(m.dt_min)),
                )
            else:
                L.update(
                    entry=Matrix([m.q_proj, m.kv_down_proj, m.k_rope_proj]), up=Matrix([m.k_nope_up_proj, m.v_up_proj]),
                    out=Matrix([m.out_proj]), heads=m.num_heads, head_dim=m.head_dim, nope=m.nope_dim, rope=m.rope_dim,
                    latent=m.latent_dim, rope_tab=rope_table_np(m.rope, self.max_len), scale=1.0 / math.sqrt(m.head_dim),
                )
            mixer_width = max(mixer_width, L["entry"].rows)
            self.layers.append(L)
        self.mixer_in = np.zeros(mixer_width, np.float32)
        self.y = np.zeros(self.hidden, np.float32)
        self.mid = np.zeros(int(cfg.dense_dim), np.float32)
        self.kv = np.zeros(max(1, max((L["up"].rows for L in self.layers if L["kind"] == "mla"), default=1)), np.float32)
        self.residual = np.zeros(self.hidden, np.float32)
        self.logits = np.zeros(self.vocab, np.float32)
        self.seen = np.zeros(self.vocab, np.uint8)
        self.rng = (c_uint64 * 2)(int(seed), 0)
        self.temperature, self.penalty, self.inverse_penalty = 1.0, 1.0, 1.0
        self.top_k = 256
        self.max_top_k = 256
        self.reset_state()

    def reset_state(self) -> None:
        self.position = 0
        for L in self.layers:
            if L["kind"] == "mamba":
                H, S, hd = L["heads"], L["state_dim"], L["head_dim"]
                L["ssm_state"] = np.zeros((H, S, hd, 2), np.float32)
                L["prev_force"] = np.zeros((H, S, hd), np.float32)
                L["conv_state"] = np.zeros((self.hidden, max(L["taps"] - 1, 1)), np.float32)
            else:
                L["k_cache"] = np.zeros((L["heads"], self.max_len, L["head_dim"]), np.float32)
                L["v_cache"] = np.zeros((L["heads"], self.max_len, L["head_dim"]), np.float32)

    def _quant(self, x, norm=None, eps=1e-6, clip=8.0):
        q, s, _ = quantize(x, norm, eps, clip, self.act_eps)
        return q, s

    def step(self, token: int, head: bool = True) -> np.ndarray:
        if self.position >= self.max_len:
            raise ValueError("the decoder has no free position left")
        L0 = lib()
        x = self.residual
        L0.orc_embed(_p(self.head.packed), _p(self.head.scales), self.head.scales.shape[1], self.head.packed.shape[1],
                     self.hidden, int(token), _p(x))
        t = self.threads
        for L in self.layers:
            q, s = self._quant(x, L["mixer_norm"], L["mixer_eps"], L["clip"])
            mix = self.mixer_in[: L["entry"].rows]
            L["entry"].gemv(q, s, mix, 0, t)
            if L["kind"] == "mamba":
                L0.orc_ssm_step(_p(mix), self.hidden, L["heads"], L["state_dim"], L["head_dim"], L["taps"], _p(L["conv_w"]),
                                _p(L["conv_b"]), _p(L["conv_state"]), _p(L["decay"]), _p(L["theta"]), _p(L["skip"]),
                                _p(L["ssm_state"]), _p(L["prev_force"]), L["hdmin"], L["hdrange"], _p(self.y))
            else:
                lat = np.ascontiguousarray(mix[self.hidden : self.hidden + L["latent"]])
                ql, sl = self._quant(lat)
                kv = self.kv[: L["up"].rows]
                L["up"].gemv(ql, sl, kv, 0, t)
                L0.orc_attention_step(_p(mix), _p(kv), _p(L["rope_tab"]), self.position, _p(L["k_cache"]), _p(L["v_cache"]),
                                      self.max_len, L["heads"], L["head_dim"], L["nope"], L["rope"], L["latent"], L["scale"],
                                      _p(self.y))
            q, s = self._quant(self.y)
            L["out"].gemv(q, s, x, 1, t)
            q, s = self._quant(x, L["ffn_norm"], L["ffn_eps"], L["clip"])
            L["gate_up"].gemv(q, s, self.mid, 2, t)
            q, s = self._quant(self.mid)
            L["down"].gemv(q, s, x, 1, t)
        if head:
            q, s = self._quant(x, self.final_norm, self.final_eps, self.layers[0]["clip"] if self.layers else 8.0)
            self.head.gemv(q, s, self.logits, 0, t)
        self.position += 1
        return self.logits

    def prefill(self, ids) -> np.ndarray:
        ids = [int(i) for i in np.asarray(ids).reshape(-1)]
        if not ids or len(ids) > self.max_len:
            raise ValueError("prompt length must lie within the decoder capacity")
        self.reset_state()
        for i, tok in enumerate(ids):
            self.step(tok, head=i == len(ids) - 1)
        return self.logits

    def configure_sampling(self, temperature: float, top_k: int, repetition_penalty: float = 1.0, penalized_ids=(),
                           max_top_k: int = 256) -> None:
        self.temperature = float(temperature)
        self.penalty = float(repetition_penalty)
        self.inverse_penalty = float(np.float32(1.0) / np.float32(repetition_penalty))
        self.max_top_k = min(int(max_top_k), self.vocab)
        self.top_k = int(top_k) if 0 < int(top_k) <= self.max_top_k else self.max_top_k
        self.seen[:] = 0
        for t in penalized_ids:
            if 0 <= int(t) < self.vocab:
                self.seen[int(t)] = 1

    def sample(self) -> int:
        return int(lib().orc_sample(_p(self.logits), _p(self.seen), self.vocab, self.temperature, self.penalty,
                                    self.inverse_penalty, self.top_k, self.max_top_k, self.rng))

    def generate(self, first: int, count: int) -> list[int]:
        """Feed `first`, then sample and feed back `count` tokens."""
        out = []
        tok = first
        for _ in range(count):
            self.step(tok)
            tok = self.sample()
            out.append(tok)
        return out
