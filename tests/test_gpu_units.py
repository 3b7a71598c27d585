"""Unit kernels of libivonar_b200.so on a B200 against the CPU oracle (bit-exact where integer)."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu


def _native():
    from ivonar_inference_b200 import _native

    return _native


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _gpu_quantize(x: torch.Tensor, w: torch.Tensor | None, eps=1e-6, clip=8.0, act_eps=1e-5):
    nat = _native()
    lib = nat.library()
    n = x.numel()
    xd = x.float().cuda().contiguous()
    wd = None if w is None else w.float().cuda().contiguous()
    q = torch.empty(n, dtype=torch.int8, device="cuda")
    s = torch.empty(1, dtype=torch.float32, device="cuda")
    xs = torch.empty((n + 63) // 64, dtype=torch.int32, device="cuda")
    rc = lib.ivb_quantize(xd.data_ptr(), 0 if wd is None else wd.data_ptr(), n, eps, clip, act_eps, q.data_ptr(),
                          s.data_ptr(), xs.data_ptr(), _stream())
    nat.check(rc, "ivb_quantize")
    torch.cuda.synchronize()
    return q.cpu().numpy(), np.float32(s.item()), xs.cpu().numpy()


def test_quantizer_is_bit_exact_with_the_oracle(oracle_lib) -> None:
    gen = torch.Generator().manual_seed(0)
    for n in (1, 16, 100, 128, 256, 1000, 1024, 2816, 4096, 11008):
        for spread in (1e-9, 1.0, 50.0):
            x = torch.randn(n, generator=gen) * spread
            if n > 8:
                x[torch.randint(0, n, (3,), generator=gen)] *= 40.0
            w = 1.0 + 0.1 * torch.randn(n, generator=gen)
            for norm in (None, w):
                q, s, xs = _gpu_quantize(x, norm)
                rq, rs, rxs = oracle_lib.quantize(x.numpy(), None if norm is None else norm.numpy())
                assert s == np.float32(rs), (n, spread, norm is None)
                np.testing.assert_array_equal(q, rq)
                np.testing.assert_array_equal(xs, rxs)
    q, s, _ = _gpu_quantize(torch.zeros(300), None)
    assert s == np.float32(1e-5) and not q.any()


def _device_matrix(packed: np.ndarray, scales: np.ndarray, bias: np.ndarray | None, in_features: int):
    nat = _native()
    rb = packed.shape[1]
    pad = (rb + 15) // 16 * 16
    p = torch.from_numpy(np.pad(packed, ((0, 0), (0, pad - rb)))).cuda().contiguous()
    s = torch.from_numpy(scales.view(np.int16).copy()).cuda().contiguous()
    b = None if bias is None else torch.from_numpy(np.ascontiguousarray(bias, np.float32)).cuda()
    return nat.ternary(p, s, b, packed.shape[0], in_features), (p, s, b)


def _random_matrix(gen, rows, cols):
    from ivonar_inference_b200 import synthetic

    packed, scales = synthetic._packed(gen, rows, cols, "baseline")
    bias = torch.randn(rows, generator=gen) * 0.02
    return packed.numpy(), scales.view(torch.int16).numpy().view(np.uint16), bias.numpy()


def test_integer_group_dots_are_bit_exact(oracle_lib) -> None:
    nat = _native()
    lib = nat.library()
    cases = []
    g = golden("ternary")
    for k in range(int(g["count"])):
        cases.append((g[f"packed{k}"], g[f"scales{k}"], g[f"bias{k}"], int(g[f"in{k}"]), g[f"q8_{k}"], g[f"dots{k}"]))
    gen = torch.Generator().manual_seed(1)
    for rows, cols in ((1, 64), (300, 1024), (37, 2816), (5, 11008), (64, 256), (3, 1)):
        p, s, b = _random_matrix(gen, rows, cols)
        q8 = torch.randint(-127, 128, (cols,), generator=gen, dtype=torch.int8).numpy()
        cases.append((p, s, b, cols, q8, None))
    for packed, scales, bias, n, q8, ref in cases:
        desc, keep = _device_matrix(packed, scales, bias, n)
        groups = (n + 127) // 128
        dots = torch.empty(packed.shape[0] * groups, dtype=torch.int32, device="cuda")
        q = torch.from_numpy(q8.copy()).cuda()
        nat.check(lib.ivb_ternary_group_dots(ctypes.byref(desc), q.data_ptr(), dots.data_ptr(), _stream()), "dots")
        got = dots.view(packed.shape[0], groups).cpu().numpy()
        want = oracle_lib.Matrix.raw(packed, scales, n, bias).group_dots(q8)
        np.testing.assert_array_equal(got, want)
        if ref is not None:
            np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("epilogue", [0, 1, 2])
@pytest.mark.parametrize("normed", [False, True])
def test_gemv_matches_the_oracle(oracle_lib, epilogue: int, normed: bool) -> None:
    nat = _native()
    lib = nat.library()
    gen = torch.Generator().manual_seed(10 + epilogue)
    for rows, cols in ((2, 16), (64, 100), (1792, 1024), (2816, 1024), (1024, 2816), (5632, 1024), (4096, 256),
                       (32768, 1024), (8, 11008)):
        p, s, b = _random_matrix(gen, rows, cols)
        x = torch.randn(cols, generator=gen)
        w = 1.0 + 0.1 * torch.randn(cols, generator=gen)
        desc, keep = _device_matrix(p, s, b, cols)
        out_rows = rows // 2 if epilogue == 2 else rows
        base = torch.randn(out_rows, generator=gen)
        out = base.clone().cuda()
        xd, wd = x.cuda(), w.cuda()
        rc = lib.ivb_ternary_gemv(ctypes.byref(desc), xd.data_ptr(), wd.data_ptr() if normed else 0, 1e-6, 8.0, 1e-5,
                                  epilogue, out.data_ptr(), _stream())
        nat.check(rc, "gemv")
        got = out.cpu().numpy()
        q, sc, _ = oracle_lib.quantize(x.numpy(), w.numpy() if normed else None)
        want = base.numpy().copy()
        oracle_lib.Matrix.raw(p, s, cols, b).gemv(q, sc, want, epilogue)
        scale = float(np.abs(want).max()) + 1e-6
        np.testing.assert_allclose(got, want, rtol=2e-5, atol=2e-5 * scale, err_msg=f"{rows}x{cols}")


def test_gemv_matches_the_reference_numba_gemv() -> None:
    nat = _native()
    lib = nat.library()
    g = golden("ternary")
    for k in range(int(g["count"])):
        n = int(g[f"in{k}"])
        desc, keep = _device_matrix(g[f"packed{k}"], g[f"scales{k}"], g[f"bias{k}"], n)
        out = torch.zeros(g[f"packed{k}"].shape[0], device="cuda")
        x = torch.from_numpy(g[f"x{k}"]).cuda()
        nat.check(lib.ivb_ternary_gemv(ctypes.byref(desc), x.data_ptr(), 0, 1e-6, 8.0, 1e-5, 0, out.data_ptr(), _stream()), "gemv")
        np.testing.assert_allclose(out.cpu().numpy(), g[f"gemv{k}"], rtol=1e-5, atol=1e-6)


def _gpu_sample(logits: np.ndarray, seen: np.ndarray, temperature, penalty, top_k, max_top_k, rng: list[int]):
    nat = _native()
    lib = nat.library()
    L = torch.from_numpy(np.ascontiguousarray(logits, np.float32)).cuda()
    S = torch.from_numpy(seen.astype(np.uint8)).cuda()
    params = torch.tensor([temperature, penalty, float(np.float32(1.0 / penalty))], dtype=torch.float32).cuda()
    k = torch.tensor([top_k], dtype=torch.int64).cuda()
    r = torch.tensor(rng, dtype=torch.int64).cuda()
    tok = torch.zeros(1, dtype=torch.int64).cuda()
    hist = torch.zeros(1, dtype=torch.int64).cuda()
    nat.check(lib.ivb_sample(L.data_ptr(), S.data_ptr(), logits.size, params.data_ptr(), k.data_ptr(), max_top_k,
                             r.data_ptr(), tok.data_ptr(), hist.data_ptr(), _stream()), "sample")
    torch.cuda.synchronize()
    return int(tok.item()), S.cpu().numpy(), r.cpu().tolist(), int(hist.item())


def test_sampler_draws_the_oracle_token_for_the_same_philox_state(oracle_lib) -> None:
    gen = torch.Generator().manual_seed(3)
    same = total = 0
    for vocab in (300, 1000, 32768):
        for trial in range(12):
            logits = (torch.randn(vocab, generator=gen) * (0.5 + trial % 4)).numpy()
            seen = (torch.rand(vocab, generator=gen) < 0.05).numpy().astype(np.uint8)
            T = (0.5, 0.7, 1.0)[trial % 3]
            rp = (1.0, 1.15, 3.0)[trial % 3]
            top_k = (1, 5, 40, 256)[trial % 4]
            key = 1000 + trial
            tok, seen_after, rng_after, hist = _gpu_sample(logits, seen.copy(), T, rp, top_k, 256, [key, trial])
            seen_o = seen.copy()
            rng_o = (oracle_lib.c_uint64 * 2)(key, trial)
            want = oracle_lib.lib().orc_sample(oracle_lib._p(logits), oracle_lib._p(seen_o), vocab, T, rp,
                                               float(np.float32(1.0 / rp)), top_k, 256, rng_o)
            assert rng_after == [key, trial + 1]
            assert hist == tok and seen_after[tok] == 1
            # the kernel and the oracle weigh the candidates with the same exponential and add them in
            # the same order: the same Philox state draws the same token, every time
            assert tok == want, (vocab, trial, tok, want)
            same += int(tok == want)
            total += 1
    assert same == total == 36


def test_sampler_follows_the_top_k_distribution() -> None:
    # same statistical check as the reference (tests/test_kernels.py:130-164)
    gen = torch.Generator().manual_seed(21)
    logits = (torch.randn(300, generator=gen) * 3).numpy()
    draws = 2000
    counts = np.zeros(300)
    for i in range(draws):
        tok, *_ = _gpu_sample(logits, np.zeros(300, np.uint8), 0.7, 1.0, 8, 16, [77, i])
        counts[tok] += 1
    values, indices = torch.topk(torch.from_numpy(logits) / 0.7, 8)
    expected = torch.softmax(values, 0).numpy()
    assert counts[[i for i in range(300) if i not in indices.tolist()]].sum() == 0
    freq = counts[indices.numpy()] / draws
    tol = 5 * np.sqrt(expected * (1 - expected) / draws) + 0.005
    assert (np.abs(freq - expected) <= tol).all()
    top = int(indices[0])
    seen = np.zeros(300, np.uint8)
    seen[top] = 1
    hits = sum(_gpu_sample(logits, seen.copy(), 0.7, 2.0, 8, 16, [99, i])[0] == top for i in range(draws))
    assert hits / draws < float(expected[0]) * 0.8


def test_sampler_breaks_ties_by_lower_index() -> None:
    logits = np.zeros(1000, np.float32)
    logits[[10, 500, 999]] = 5.0
    for i in range(20):
        tok, *_ = _gpu_sample(logits, np.zeros(1000, np.uint8), 1.0, 1.0, 1, 256, [5, i])
        assert tok == 10
    flat = np.zeros(777, np.float32)
    picks = {_gpu_sample(flat, np.zeros(777, np.uint8), 1.0, 1.0, 4, 256, [6, i])[0] for i in range(60)}
    assert picks <= {0, 1, 2, 3} and len(picks) > 1


def test_a_wait_that_never_completes_gives_up_and_the_gpu_stays_usable() -> None:
    nat = _native()
    lib = nat.library()
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    word = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.ivb_probe_wait_timeout(counter.data_ptr(), word.data_ptr(), 50_000_000, _stream())
    assert rc == nat.IVB_ETIMEOUT
    assert int(word.item()) == nat.IVB_ETIMEOUT
    assert int(counter.item()) == 1
    x = torch.arange(10, device="cuda", dtype=torch.float32)
    assert float((x * 2).sum()) == 90.0


def _stream_chunk(packed: np.ndarray, scales_u16: np.ndarray, bias, in_n: int) -> tuple[torch.Tensor, int, int]:
    """One weight-stream chunk of the decode kernel: packed rows padded to 16 bytes (plus 16 when a
    multiple of 128, as the plan lays them out), the fp16 scale rows padded to 8 entries, the biases."""
    rows = packed.shape[0]
    rb = (packed.shape[1] + 15) // 16 * 16
    if rb % 128 == 0:
        rb += 16
    stride = ((in_n + 127) // 128 + 7) // 8 * 8
    w = np.zeros((rows, rb), np.uint8)
    w[:, : packed.shape[1]] = packed
    sc = np.zeros((rows, stride), np.uint16)
    sc[:, : scales_u16.shape[1]] = scales_u16
    blob = w.tobytes() + sc.tobytes()
    blob += b"\0" * ((-len(blob)) % 16)
    if bias is not None:
        blob += np.asarray(bias, np.float32).tobytes()
    return torch.from_numpy(np.frombuffer(blob, np.uint8).copy()).cuda(), rb, stride


def _decode_rows(chunk, rows, rb, stride, has_bias, act_scale, q8, in_n, lg) -> np.ndarray:
    nat = _native()
    q = torch.from_numpy(np.ascontiguousarray(q8, np.int8)).cuda()
    out = torch.zeros(rows, dtype=torch.float32, device="cuda")
    nat.check(nat.library().ivb_decode_rows(chunk.data_ptr(), rows, rb, stride, int(has_bias), float(act_scale), q.data_ptr(),
                                            in_n, lg, out.data_ptr(), _stream()), "ivb_decode_rows")
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_decode_row_routine_gives_the_reference_integer_dots() -> None:
    """The decode kernel's GEMV row routine at every lane width it can run with: with a one-hot group
    scale (1.0) and act_scale 1 each output is the exact integer dot of one 128-input group, equal bit
    for bit to the reference's numba row_dot on the same codes (tests/golden/ternary.npz)."""
    g = golden("ternary")
    checked = 0
    for k in range(int(g["count"])):
        packed, scales, q8, dots = g[f"packed{k}"], g[f"scales{k}"], g[f"q8_{k}"], g[f"dots{k}"]
        rows, groups = dots.shape
        in_n = int(g[f"in{k}"])
        chunks = (in_n + 63) // 64
        for lg in (-1, 0, 1, 2, 3, 4):  # -1: the routine the decode kernel picks for the shape
            if chunks > 4 << max(lg, 4 if lg < 0 else lg):
                continue
            for grp in range(groups):
                onehot = np.zeros_like(scales)
                onehot[:, grp] = 0x3C00  # fp16 1.0
                chunk, rb, stride = _stream_chunk(packed, onehot, None, in_n)
                out = _decode_rows(chunk, rows, rb, stride, False, 1.0, q8, in_n, lg)
                assert np.array_equal(out, dots[:, grp].astype(np.float32)), (k, lg, grp)
                checked += 1
    assert checked == 112  # every group of the six golden shapes, every lane width that holds them and the kernel's pick


def test_decode_row_routine_matches_the_reference_gemv(oracle_lib) -> None:
    """With the real group scales and biases the row routine equals the reference's numba gemv output
    (its fp32 sum over groups, here over 64-input chunks: same float tolerance as the unit GEMV) and the
    oracle's GEMV, for every lane width."""
    g = golden("ternary")
    for k in range(int(g["count"])):
        packed, scales, q8, bias = g[f"packed{k}"], g[f"scales{k}"], g[f"q8_{k}"], g[f"bias{k}"]
        in_n = int(g[f"in{k}"])
        rows = packed.shape[0]
        act_scale = float(g[f"act_scale{k}"])
        mat = oracle_lib.Matrix.raw(packed, scales, in_n, bias)
        want = np.zeros(rows, np.float32)
        mat.gemv(np.ascontiguousarray(q8, np.int8), act_scale, want)
        chunks = (in_n + 63) // 64
        chunk, rb, stride = _stream_chunk(packed, scales, bias, in_n)
        for lg in (-1, 0, 1, 2, 3, 4):
            if chunks > 4 << max(lg, 4 if lg < 0 else lg):
                continue
            out = _decode_rows(chunk, rows, rb, stride, True, act_scale, q8, in_n, lg)
            np.testing.assert_allclose(out, g[f"gemv{k}"], rtol=1e-5, atol=1e-6)
            np.testing.assert_allclose(out, want, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("rows,cols", [(8, 1024), (16, 1024), (64, 1024), (200, 1024), (8, 2816), (6, 2816), (10, 1024)])
def test_decode_row_geometries_give_the_oracle_integer_dots(oracle_lib, rows: int, cols: int) -> None:
    """Every compile-time row geometry of the decode kernel (16 lanes x 1 row, 8 lanes x 2 and x 8 rows,
    32 lanes for long inputs) against the oracle's exact integer group dots (one-hot group scales)."""
    from ivonar_inference_b200 import synthetic

    gen = torch.Generator().manual_seed(rows * 7 + cols)
    packed, scales = synthetic._packed(gen, rows, cols, "baseline")
    packed = packed.numpy()
    scales = scales.view(torch.int16).numpy().view(np.uint16)
    x = torch.randn(cols, generator=gen).numpy()
    q8, _, _ = oracle_lib.quantize(x)
    want = oracle_lib.Matrix.raw(packed, scales, cols).group_dots(q8)
    for grp in range(want.shape[1]):
        onehot = np.zeros_like(scales)
        onehot[:, grp] = 0x3C00
        chunk, rb, stride = _stream_chunk(packed, onehot, None, cols)
        out = _decode_rows(chunk, rows, rb, stride, False, 1.0, q8, cols, -1)
        assert np.array_equal(out, want[:, grp].astype(np.float32)), (rows, cols, grp)
