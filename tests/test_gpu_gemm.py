"""Prefill path on a B200: ivb_quantize_rows and the tcgen05 ternary GEMM against the CPU oracle."""

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
    p = torch.nn.functional.pad(packed, (0, pad - rb)).contiguous()
    s = scales.view(torch.int16).contiguous()
    b = torch.randn(rows, generator=gen) * 0.02
    desc = _native.ternary(p.cuda(), s.cuda(), b.cuda(), rows, cols)
    keep = (p.cuda(), s.cuda(), b.cuda())
    desc = _native.ternary(keep[0], keep[1], keep[2], rows, cols)
    return desc, keep, (p.numpy()[:, :rb], s.numpy().view(np.uint16), b.numpy())


def _quantize_rows(x: torch.Tensor, w: torch.Tensor | None):
    nat, lib = _lib()
    rows, n = x.shape
    ldq = (n + 127) // 128 * 128
    q8 = torch.zeros((rows + 127) // 128 * 128, ldq, dtype=torch.int8, device="cuda")  # whole 128-token tiles
    scale = torch.empty(rows, dtype=torch.float32, device="cuda")
    gsum = torch.empty(rows, (n + 127) // 128, dtype=torch.int32, device="cuda")
    xd = x.float().cuda().contiguous()
    wd = None if w is None else w.float().cuda().contiguous()
    nat.check(lib.ivb_quantize_rows(xd.data_ptr(), rows, n, 0 if wd is None else wd.data_ptr(), 1e-6, 8.0, 1e-5,
                                    q8.data_ptr(), ldq, scale.data_ptr(), gsum.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream), "ivb_quantize_rows")
    return q8, scale, gsum, ldq


def _q8_offsets(rows: int, ldq: int) -> np.ndarray:
    """Byte offset of (token t, input i) in the tiled GEMM activation layout documented in ivonar_b200.h."""
    t = np.arange(rows)[:, None]
    i = np.arange(ldq)[None, :]
    k = i >> 4
    r = t & 127
    tile = ((t >> 7) * (ldq >> 7) + (k >> 3)) * 16384
    core = (((r >> 3) << 3) + (k & 7)) * 128 + ((r & 7) << 4)
    return tile + core + ((i & 3) << 2) + ((i >> 2) & 3)


def test_quantize_rows_matches_the_oracle_quantiser(oracle_lib) -> None:
    gen = torch.Generator().manual_seed(3)
    for rows, n, normed in ((5, 1024, True), (37, 2816, False), (3, 100, True), (130, 256, False)):
        x = torch.randn(rows, n, generator=gen) * 2.0
        w = 1.0 + 0.1 * torch.randn(n, generator=gen)
        q8, scale, gsum, ldq = _quantize_rows(x, w if normed else None)
        flat = q8.cpu().numpy().reshape(-1)
        natural = flat[_q8_offsets(rows, ldq)]
        for t in range(rows):
            q, s, _ = oracle_lib.quantize(x[t].numpy(), w.numpy() if normed else None)
            np.testing.assert_array_equal(natural[t, :n], q)
            assert np.all(natural[t, n:] == 0)
            assert np.float32(scale[t].item()) == s
            groups = (n + 127) // 128
            want = [int(q[g * 128:(g + 1) * 128].astype(np.int64).sum()) for g in range(groups)]
            assert gsum[t].cpu().tolist() == want


@pytest.mark.parametrize("epilogue", [0, 1, 2])
def test_gemm_matches_the_oracle_gemv_per_token(oracle_lib, epilogue: int) -> None:
    nat, lib = _lib()
    gen = torch.Generator().manual_seed(20 + epilogue)
    stream = torch.cuda.current_stream().cuda_stream
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    # the first four and the last split K (few row x token tiles); the others run every epilogue in the
    # GEMM itself, over several tiles per CTA, ragged row and token tiles included
    for rows, cols, tokens in ((128, 1024, 1), (256, 1024, 37), (1792, 1024, 130), (1024, 2816, 64), (64, 100, 3),
                               (256, 384, 200), (1216, 1024, 1300), (5632, 1024, 16)):
        desc, keep, (p, s, b) = _matrix(gen, rows, cols)
        x = torch.randn(tokens, cols, generator=gen)
        w = 1.0 + 0.1 * torch.randn(cols, generator=gen)
        q8, scale, gsum, ldq = _quantize_rows(x, w)
        out_rows = rows // 2 if epilogue == 2 else rows
        base = torch.randn(tokens, out_rows, generator=gen)
        out = base.clone().cuda()
        nat.check(lib.ivb_ternary_gemm(ctypes.byref(desc), q8.data_ptr(), ldq, scale.data_ptr(), tokens, epilogue,
                                       out.data_ptr(), out_rows, err.data_ptr(), stream), "ivb_ternary_gemm")
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        got = out.cpu().numpy()
        mat = oracle_lib.Matrix.raw(p, s, cols, b)
        for t in range(tokens):
            q, sc, _ = oracle_lib.quantize(x[t].numpy(), w.numpy())
            want = base[t].numpy().copy()
            mat.gemv(q, sc, want, epilogue)
            tol = float(np.abs(want).max()) + 1e-6
            # per-group fp32 accumulation against the GEMV's per-chunk order: the GEMV bar
            np.testing.assert_allclose(got[t], want, rtol=2e-5, atol=2e-5 * tol, err_msg=f"{rows}x{cols} token {t}")
