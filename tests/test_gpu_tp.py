"""Tensor-parallel batched decode (config 4 path) on B200: one rank against the reference's greedy stream,
two NCCL ranks against one rank."""

from __future__ import annotations

import os

import pytest
import torch
import torch.multiprocessing as mp

from conftest import check_greedy_stream, golden

pytestmark = pytest.mark.gpu


def _stream(model, rank: int, world: int, prompt: torch.Tensor, count: int, group=None) -> list[int]:
    from ivonar_inference_b200.tp import B200TensorParallel

    tp = B200TensorParallel(model, rank, world, group, batch=1, max_len=64, device=f"cuda:{rank}")
    tp.start(prompt.view(1, -1), [7], 1.0, 1, 4.0)
    first = int(tp.tokens[0])
    rest = tp.decode(count - 1)[0].tolist()
    return [first] + rest


def test_one_rank_continues_the_reference_greedy_stream() -> None:
    from ivonar_inference_b200 import synthetic

    g = golden("model_config0")
    model = synthetic.synthetic_model(synthetic.config0(seq_len=int(g["seq_len"])), int(g["seed"]))
    stream = g["torch_greedy_rp"].tolist()[:40]
    got = _stream(model, 0, 1, torch.from_numpy(g["prompt"]), len(stream))
    check_greedy_stream(got, stream, g["prefill_logits"], g["torch_greedy_rp_step_logits"], 4.0, 0.1)


def _rank(rank: int, world: int, port: int, prompt, count: int, result) -> None:
    import torch.distributed as dist

    from ivonar_inference_b200 import synthetic

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        model = synthetic.synthetic_model(synthetic.config0(), 0)
        result[rank] = _stream(model, rank, world, prompt, count)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_decode_the_stream_of_one() -> None:
    import socket

    from ivonar_inference_b200 import synthetic

    g = golden("model_config0")
    prompt = torch.from_numpy(g["prompt"])
    count = 24
    want = _stream(synthetic.synthetic_model(synthetic.config0(), 0), 0, 1, prompt, count)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    result = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_rank, args=(2, port, prompt, count, result), nprocs=2, join=True, start_method="spawn")
    assert result[0] == result[1] == want, (result[0], result[1], want)
