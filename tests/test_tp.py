"""Tensor-parallel sharding on CPU: the row/column shards of packed ternary matrices and their all-reduce
reassemble the unsharded products (world_size 2 over gloo; the same plan the NCCL ranks use on B200)."""

from __future__ import annotations

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _dense(t) -> torch.Tensor:
    """Dequantised weights [out, in] (code - 1) * scale, float64."""
    packed = t.packed_weight.to(torch.int64)
    codes = torch.stack([(packed >> (2 * f)) & 3 for f in range(4)], dim=2).reshape(packed.shape[0], -1)[:, : t.in_features]
    scales = t.weight_scales.double().repeat_interleave(128, dim=1)[:, : t.in_features]
    return (codes.double() - 1.0) * scales


def test_split_even_covers_the_groups() -> None:
    from ivonar_inference_b200.tp import split_even

    for total, parts in ((11008, 8), (11008, 2), (384, 2), (384, 3), (4096, 8), (100, 1)):
        ranges = split_even(total, parts, 128)
        assert ranges[0][0] == 0 and ranges[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        assert all(lo % 128 == 0 and hi > lo for lo, hi in ranges)
        sizes = [-(-(hi - lo) // 128) for lo, hi in ranges]
        assert max(sizes) - min(sizes) <= 1


def _worker(rank: int, world: int, port: int, result) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ivonar_inference_b200 import synthetic
        from ivonar_inference_b200.tp import col_slice, row_slice, split_even

        model = synthetic.synthetic_model(synthetic.config0(), 0)
        block = model.blocks[0]
        gen = torch.Generator().manual_seed(1)
        d = int(model.config.hidden_dim)
        x = torch.randn(3, d, generator=gen, dtype=torch.float64)
        # row-parallel FFN down projection: inputs split on 128-groups, partial products summed
        F = int(block.ffn.down_proj.in_features)
        f0, f1 = split_even(F, world, 128)[rank]
        h = torch.randn(3, F, generator=gen, dtype=torch.float64)
        part = h[:, f0:f1] @ _dense(col_slice(block.ffn.down_proj, f0, f1, keep_bias=rank == 0)).T
        dist.all_reduce(part)
        full = h @ _dense(block.ffn.down_proj).T
        # column-parallel gate: rows of this rank, gathered
        g_rows = _dense(row_slice(block.ffn.gate_proj, f0, f1))
        ranges = split_even(F, world, 128)
        width = max(hi - lo for lo, hi in ranges)  # gloo gathers equal sizes: pad, then trim
        mine = torch.zeros(3, width, dtype=torch.float64)
        mine[:, : f1 - f0] = x @ g_rows.T
        gathered = [torch.zeros(3, width, dtype=torch.float64) for _ in ranges]
        dist.all_gather(gathered, mine)
        gathered = [g[:, : hi - lo] for g, (lo, hi) in zip(gathered, ranges)]
        gate_full = x @ _dense(block.ffn.gate_proj).T
        # mixer heads: out projection row-parallel over head channels
        H = int(model.config.num_heads)
        hd = d // H
        c0, c1 = rank * (H // world) * hd, (rank + 1) * (H // world) * hd
        y = torch.randn(3, d, generator=gen, dtype=torch.float64)
        out_part = y[:, c0:c1] @ _dense(col_slice(block.mixer.out_proj, c0, c1, keep_bias=rank == 0)).T
        dist.all_reduce(out_part)
        out_full = y @ _dense(block.mixer.out_proj).T
        if rank == 0:
            result["down"] = float((part - full).abs().max())
            result["gate"] = float((torch.cat(gathered, dim=1) - gate_full).abs().max())
            result["out"] = float((out_part - out_full).abs().max())
    finally:
        dist.destroy_process_group()


def test_shards_reassemble_the_unsharded_products_over_gloo() -> None:
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    manager = mp.get_context("spawn").Manager()
    result = manager.dict()
    mp.start_processes(_worker, args=(2, port, result), nprocs=2, join=True, start_method="spawn")
    assert result["down"] < 1e-9 and result["gate"] < 1e-9 and result["out"] < 1e-9, dict(result)


def _topk_order(keys: torch.Tensor, ids: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """The k best (key desc, id asc), as the samplers order their candidates."""
    order = sorted(range(keys.numel()), key=lambda i: (-float(keys[i]), int(ids[i])))[:k]
    return keys[order], ids[order]


def _vocab_worker(rank: int, world: int, port: int, result) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ivonar_inference_b200.tp import split_even

        vocab, k, batch = 700, 40, 3
        gen = torch.Generator().manual_seed(7)
        # scores with many exact ties (rounded), the same on every rank
        scores = torch.round(torch.randn(batch, vocab, generator=gen, dtype=torch.float64) * 4.0) / 4.0
        ranges = split_even(vocab, world, 128)
        v0, v1 = ranges[rank]
        kc = k
        keys = torch.full((batch, kc), -1e30, dtype=torch.float64)
        ids = torch.zeros(batch, kc, dtype=torch.int64)
        for b in range(batch):
            local = scores[b, v0:v1]
            kk, ii = _topk_order(local, torch.arange(v0, v1), min(k, v1 - v0))
            keys[b, : kk.numel()], ids[b, : ii.numel()] = kk, ii
            ids[b, ii.numel():] = vocab + torch.arange(kc - ii.numel())
        all_keys = [torch.zeros_like(keys) for _ in range(world)]
        all_ids = [torch.zeros_like(ids) for _ in range(world)]
        dist.all_gather(all_keys, keys)
        dist.all_gather(all_ids, ids)
        # rank-major candidates: equal keys appear in id order, so ranking them by position (as the merge
        # kernel does) ranks them by id
        ok = True
        for b in range(batch):
            ck = torch.cat([a[b] for a in all_keys])
            ci = torch.cat([a[b] for a in all_ids])
            pos = torch.arange(ck.numel())
            mk, mp = _topk_order(ck, pos, k)
            gk, gi = _topk_order(scores[b], torch.arange(vocab), k)
            ok = ok and torch.equal(mk, gk) and torch.equal(ci[mp], gi)
        if rank == 0:
            result["ok"] = bool(ok)
            result["ranges"] = ranges
    finally:
        dist.destroy_process_group()


def test_vocabulary_shards_merge_to_the_unsharded_top_k_over_gloo() -> None:
    """The sharded head's sampler plan (tp.py, ivb_batch_topk_slice + ivb_batch_sample_merge): per-slice
    top-k candidates, gathered rank-major and merged by position, give the unsharded top-k with its id
    order among equal scores."""
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    manager = mp.get_context("spawn").Manager()
    result = manager.dict()
    mp.start_processes(_vocab_worker, args=(2, port, result), nprocs=2, join=True, start_method="spawn")
    assert result["ok"], dict(result)
    assert result["ranges"] == [(0, 384), (384, 700)]
