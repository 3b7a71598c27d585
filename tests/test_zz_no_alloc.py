"""ivb_ternary_gemv_splitk (static scratch, no allocation) against the CPU oracle on a B200.

The split-K entry point serves callers that may not allocate device memory when they call it (a server
whose memory pool already holds the GPU, or a path that cannot take cudaMalloc's synchronisation).

Collected last on purpose: it must pass alone and after the other GPU tests, which exercises the
once-per-device scratch lookup both cold and after other kernels ran.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from ivonar_inference_b200 import _native

    return _native, _native.library()


def _matrix(gen, rows: int, cols: int):
    from ivonar_inference_b200 import _native, synthetic

    packed, scales = synthetic._packed(gen, rows, cols, "baseline")
    rb = packed.shape[1]
    pad = (rb + 15) // 16 * 16
    p = torch.nn.functional.pad(packed, (0, pad - rb)).cuda().contiguous()
    s = scales.view(torch.int16).cuda().contiguous()
    b = (torch.randn(rows, generator=gen) * 0.02).cuda()
    return _native.ternary(p, s, b, rows, cols), (p, s, b)


@pytest.mark.parametrize("epilogue", [0, 1, 2])
@pytest.mark.parametrize("normed", [False, True])
def test_splitk_matches_the_oracle_and_repeats_bit_for_bit(oracle_lib, epilogue: int, normed: bool) -> None:
    """Against the CPU oracle's quantiser and GEMV (same codes, fp32 sums in another order), up to the
    largest input the scratch takes (16384); two calls in a row give the same bits (the column blocks'
    partial sums are added in a fixed order)."""
    nat, lib = _lib()
    gen = torch.Generator().manual_seed(70 + 3 * epilogue + int(normed))
    stream = torch.cuda.current_stream().cuda_stream
    for rows, cols in ((1024, 2816), (64, 100), (5632, 1024), (32768, 1024), (8, 11008), (64, 16384)):
        desc, (p, sc, b) = _matrix(gen, rows, cols)
        x = torch.randn(cols, generator=gen)
        w = 1.0 + 0.1 * torch.randn(cols, generator=gen)
        out_rows = rows // 2 if epilogue == 2 else rows
        base = torch.randn(out_rows, generator=gen)
        q8, act_scale, _ = oracle_lib.quantize(x.numpy(), w.numpy() if normed else None, 1e-6, 8.0, 1e-5)
        mat = oracle_lib.Matrix.raw(p.cpu().numpy(), sc.cpu().numpy().view(np.uint16), cols, b.cpu().numpy())
        want = base.numpy().copy()
        mat.gemv(q8, act_scale, want, epilogue)
        results = []
        xd, wd = x.cuda(), w.cuda()  # kept alive until the kernels ran (the allocator reuses freed blocks)
        for call in range(2):
            got = base.cuda()
            nat.check(lib.ivb_ternary_gemv_splitk(ctypes.byref(desc), xd.data_ptr(), wd.data_ptr() if normed else 0,
                                                  1e-6, 8.0, 1e-5, epilogue, got.data_ptr(), stream), "ivb_ternary_gemv_splitk")
            torch.cuda.synchronize()
            results.append(got.cpu().numpy())
        assert np.array_equal(results[0], results[1]), f"{rows}x{cols}: two calls differ"
        scale = float(np.abs(want).max()) + 1e-6
        # same integer chunk dots; fp32 group sums in another order (and CUDA's expf in the SwiGLU)
        np.testing.assert_allclose(results[0], want, rtol=2e-5, atol=2e-5 * scale, err_msg=f"{rows}x{cols}")


def test_splitk_rejects_inputs_larger_than_its_scratch() -> None:
    nat, lib = _lib()
    gen = torch.Generator().manual_seed(5)
    stream = torch.cuda.current_stream().cuda_stream
    desc, keep = _matrix(gen, 32770, 64)
    x = torch.randn(64, generator=gen).cuda()
    out = torch.zeros(32770, device="cuda")
    rc = lib.ivb_ternary_gemv_splitk(ctypes.byref(desc), x.data_ptr(), 0, 1e-6, 8.0, 1e-5, 0, out.data_ptr(), stream)
    assert rc == nat.IVB_EINVAL
    assert "static scratch" in nat.last_error()
    desc, keep = _matrix(gen, 4, 16448)
    x = torch.randn(16448, generator=gen).cuda()
    rc = lib.ivb_ternary_gemv_splitk(ctypes.byref(desc), x.data_ptr(), 0, 1e-6, 8.0, 1e-5, 0, out.data_ptr(), stream)
    assert rc == nat.IVB_EINVAL
    assert "input limit" in nat.last_error()
