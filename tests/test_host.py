"""Host-side checks that need no GPU: the C ABI, the checkpoint container and the decoder guards."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest
import torch

from conftest import ROOT

HEADER = ROOT / "include" / "ivonar_b200.h"


def _declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(ivb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_entry_point() -> None:
    from ivonar_inference_b200 import _native

    lib = _native.library()
    names = _declared_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
        assert name in _native.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_native.SIGNATURES) == set(names)
    assert lib.ivb_abi_version() == _native.IVB_ABI_VERSION


def test_ctypes_structs_match_the_c_layout(tmp_path: Path) -> None:
    from ivonar_inference_b200 import _native

    structs = [_native.IvbTernary, _native.IvbLayerDesc, _native.IvbModelDesc, _native.IvbCheckBuffer]
    lines = ['#include <cstddef>', '#include <cstdio>', '#include "ivonar_b200.h"', "int main() {"]
    for st in structs:
        lines.append(f'  printf("{st.__name__} sizeof %zu\\n", sizeof({st.__name__}));')
        for field, _ in st._fields_:
            lines.append(f'  printf("{st.__name__} {field} %zu\\n", offsetof({st.__name__}, {field}));')
    lines.append("  return 0;\n}")
    src = tmp_path / "layout.cpp"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    compiler = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"
    subprocess.run([compiler, "-std=c++17", f"-I{HEADER.parent}", str(src), "-o", str(exe)], check=True)
    printed = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    expected = {}
    for st in structs:
        expected[f"{st.__name__} sizeof"] = ctypes.sizeof(st)
        for field, _ in st._fields_:
            expected[f"{st.__name__} {field}"] = getattr(st, field).offset
    got = {" ".join(line.split()[:2]): int(line.split()[2]) for line in printed if line.strip()}
    assert got == expected


def test_last_error_reports_bad_arguments() -> None:
    from ivonar_inference_b200 import _native

    lib = _native.library()
    rc = lib.ivb_ternary_group_dots(None, None, None, None)
    assert rc == _native.IVB_EINVAL
    assert "null" in _native.last_error()
    handle = ctypes.c_void_p()
    assert lib.ivb_decoder_create(None, 0, ctypes.byref(handle)) == _native.IVB_EINVAL


def test_synthetic_models_are_the_reference_model_built_by_its_loader(tmp_path: Path) -> None:
    from ivonar_inference_b200 import _reference, synthetic

    payload = synthetic.tiny()
    model = synthetic.synthetic_model(payload, 0, "reference_tests")
    assert isinstance(model, _reference.module("model").IvonarModel)
    assert [b.mixer_type for b in model.blocks] == ["mamba", "mla", "mamba"]
    assert model.blocks[1].mixer.rope_dim == 2 and model.blocks[1].mixer.nope_dim == 2
    # the reference loader validates what the generator emits: no reserved code 3, positive scales
    state = synthetic.synthetic_state(payload, 0, "reference_tests")
    bad = dict(state)
    bad["blocks.0.ffn.down_proj.packed_weight"] = bad["blocks.0.ffn.down_proj.packed_weight"].clone()
    bad["blocks.0.ffn.down_proj.packed_weight"][0, 0] = 0xFF
    config = _reference.module("config").ModelConfig.from_payload(payload)
    with pytest.raises(RuntimeError, match="code 3"):
        _reference.module("loader").build_model(config, bad)
    # a packed checkpoint of it loads through the reference's load_model unchanged
    path = tmp_path / "packed.pt"
    loader = _reference.module("loader")
    torch.save({"format": loader.PACKED_FORMAT, "schema_version": loader.PACKED_SCHEMA_VERSION, "config": payload,
                "model_state": state}, path)
    loaded = loader.load_model(path, materialize=False).model
    assert torch.equal(loaded.token_io.projection.packed_weight, state["token_io.projection.packed_weight"])


def test_synthetic_models_are_reproducible_and_follow_the_distribution() -> None:
    from ivonar_inference_b200 import synthetic

    payload = synthetic.config0()
    a = synthetic.synthetic_state(payload, 5)
    b = synthetic.synthetic_state(payload, 5)
    assert all(torch.equal(a[k], b[k]) for k in a)
    packed = a["blocks.0.ffn.gate_proj.packed_weight"]
    codes = torch.stack([(packed >> s) & 3 for s in (0, 2, 4, 6)], -1).flatten()
    frac = torch.bincount(codes.long(), minlength=4).float() / codes.numel()
    assert abs(float(frac[1]) - 0.4) < 0.02 and abs(float(frac[0]) - 0.3) < 0.02 and float(frac[3]) == 0.0
    scales = a["blocks.0.ffn.gate_proj.weight_scales"].float()
    assert abs(float(scales.log().mean()) - torch.log(torch.tensor(0.02)).item()) < 0.05


def test_rope_table_is_the_reference_decoders_rotary_table() -> None:
    from ivonar_inference_b200 import _reference, synthetic
    from ivonar_inference_b200.decoder import rope_from_rotary

    model = synthetic.synthetic_model(synthetic.tiny(hidden=64, latent=24, dense=96, seq_len=64), 0, "reference_tests")
    static = _reference.module("decoder").StaticDecoder(model, device="cpu")
    mixer = model.blocks[1].mixer
    table = rope_from_rotary(mixer.rope, 64)
    assert table.shape == (64, mixer.rope_dim // 2, 2)
    reference = torch.view_as_real(static.rope_tables[1][:, mixer.nope_dim // 2:])
    torch.testing.assert_close(table, reference, rtol=0, atol=0)


def test_the_b200_decoder_refuses_a_cpu_device() -> None:
    from ivonar_inference_b200 import B200Decoder, KernelError, synthetic

    model = synthetic.synthetic_model(synthetic.tiny(), 0, "reference_tests")
    with pytest.raises(KernelError, match="CUDA"):
        B200Decoder(model, device="cpu")


def test_build_decoder_leaves_other_devices_to_the_reference_dispatch() -> None:
    from ivonar_inference_b200 import _reference, decoder, synthetic

    model = synthetic.synthetic_model(synthetic.tiny(), 0, "reference_tests")
    dec, backend, note = decoder.build_decoder(model, "cpu", kernels=False)
    assert isinstance(dec, _reference.module("decoder").StaticDecoder) and backend == "torch" and note is None


def test_ingest_leaves_other_devices_to_the_reference_loader(tmp_path: Path) -> None:
    from ivonar_inference_b200 import _reference, ingest, synthetic

    payload = synthetic.tiny()
    state = synthetic.synthetic_state(payload, 0, "reference_tests")
    loader = _reference.module("loader")
    path = tmp_path / "packed.pt"
    torch.save({"format": loader.PACKED_FORMAT, "schema_version": loader.PACKED_SCHEMA_VERSION, "config": payload,
                "model_state": state, "step": 3}, path)
    ours = ingest.load_model(path, "cpu", materialize=False)
    ref = loader.load_model(path, "cpu", materialize=False)
    assert isinstance(ours, loader.LoadedModel) and ours.step == 3 and ours.config == ref.config
    for key, value in ref.model.state_dict().items():
        assert torch.equal(value, ours.model.state_dict()[key]), key
    # a corrupted checkpoint raises the reference's own error
    state["blocks.1.ffn.up_proj.weight_scales"] = -state["blocks.1.ffn.up_proj.weight_scales"]
    torch.save({"format": loader.PACKED_FORMAT, "schema_version": loader.PACKED_SCHEMA_VERSION, "config": payload,
                "model_state": state}, path)
    with pytest.raises(RuntimeError, match="positive values: blocks.1.ffn.up_proj.weight_scales"):
        ingest.load_model(path, "cpu")


def test_ingest_block_copy_rebuilds_every_tensor_at_its_offset(tmp_path: Path) -> None:
    """The one-block copy of a memory-mapped checkpoint, aimed at the host: every tensor (views that share
    a storage, a strided view, an empty tensor, non-tensor entries) comes back equal at its offset."""
    from ivonar_inference_b200 import ingest, synthetic

    state = dict(synthetic.synthetic_state(synthetic.tiny(), 0, "reference_tests"))
    base = torch.arange(60, dtype=torch.float32).view(6, 10)
    state.update({"shared.a": base, "shared.b": base[2:5, 1:7:2], "shared.t": base.t(), "empty": torch.empty(0, 3),
                  "half": torch.randn(7, dtype=torch.float16), "note": "text"})
    path = tmp_path / "state.pt"
    torch.save(state, path)
    mapped = torch.load(path, map_location="cpu", weights_only=True, mmap=True)
    out = ingest._state_to_device(mapped, torch.device("cpu"), path.stat().st_size)
    assert out.keys() == state.keys() and out["note"] == "text"
    for key, value in state.items():
        if isinstance(value, torch.Tensor):
            assert out[key].dtype == value.dtype and out[key].shape == value.shape, key
            assert torch.equal(out[key], value), key
    # views of one saved storage stay views of one block
    assert out["shared.b"].untyped_storage().data_ptr() == out["shared.a"].untyped_storage().data_ptr()


def test_ingest_archive_reader_matches_torch_load(tmp_path: Path) -> None:
    """The direct reader of a torch.save archive, aimed at the host: the same payload as torch.load
    (nested config, shared and strided storages, empty tensors), and None (torch.load takes over) for an
    archive holding anything else."""
    from ivonar_inference_b200 import ingest, synthetic

    payload = synthetic.tiny()
    state = dict(synthetic.synthetic_state(payload, 0, "reference_tests"))
    base = torch.arange(60, dtype=torch.float32).view(6, 10)
    state.update({"shared.a": base, "shared.b": base[2:5, 1:7:2], "shared.t": base.t(), "empty": torch.empty(0, 3),
                  "bf16": torch.randn(5, dtype=torch.bfloat16), "ids": torch.arange(9)})
    path = tmp_path / "model.pt"
    torch.save({"format": "f", "config": payload, "model_state": state, "step": 4, "none": None}, path)
    got = ingest._read_archive(path, torch.device("cpu"))
    want = torch.load(path, map_location="cpu", weights_only=True)
    assert got is not None and got.keys() == want.keys() and got["config"] == want["config"] and got["none"] is None
    for key, value in want["model_state"].items():
        ours = got["model_state"][key]
        assert ours.dtype == value.dtype and ours.shape == value.shape and ours.stride() == value.stride(), key
        assert torch.equal(ours, value), key
    torch.save({"p": torch.nn.Parameter(torch.ones(3))}, path)
    assert ingest._read_archive(path, torch.device("cpu")) is None
    path.write_bytes(b"not an archive")
    assert ingest._read_archive(path, torch.device("cpu")) is None


def _device_checks_on_the_host(state: dict, checked: list) -> tuple[int, int, int]:
    """What ivb_validate_buffers reports, computed with numpy: the lowest index into `checked` of a
    packed buffer holding code 3, of a scale buffer with a non-finite value, and of one with a
    non-positive value (len(checked) when none)."""
    import numpy as np

    bad = [len(checked)] * 3
    for i, (_, key, kind) in enumerate(checked):
        if kind == 0:
            b = state[key].numpy().reshape(-1).astype(np.uint32)
            flags = (bool(np.any(b & (b >> 1) & 0x55)), False, False)
        else:
            h = state[key].view(torch.int16).numpy().reshape(-1).astype(np.uint32) & 0xFFFF
            flags = (False, bool(np.any((h & 0x7C00) == 0x7C00)), bool(np.any(((h & 0x8000) != 0) | ((h & 0x7FFF) == 0))))
        for j in range(3):
            if flags[j]:
                bad[j] = min(bad[j], i)
    return tuple(bad)


def test_ingest_reports_the_reference_loaders_first_error() -> None:
    """The order in which the device-checked state raises: for random corruptions (reserved codes,
    NaN/inf/zero/negative scales, wrong dtypes, non-tensors, several at once) the message chosen from
    the device's per-check lowest indices is the one the reference's own _validate_state raises."""
    from ivonar_inference_b200 import _reference, ingest, synthetic

    loader = _reference.module("loader")
    clean = synthetic.synthetic_state(synthetic.tiny(), 0, "reference_tests")
    keys = list(clean)
    gen = torch.Generator().manual_seed(11)
    for trial in range(200):
        state = {k: v.clone() for k, v in clean.items()}
        for _ in range(int(torch.randint(0, 4, (1,), generator=gen))):
            key = keys[int(torch.randint(0, len(keys), (1,), generator=gen))]
            value = state[key]
            kind = int(torch.randint(0, 6, (1,), generator=gen))
            if not isinstance(value, torch.Tensor):
                continue
            flat = value.view(-1)
            at = int(torch.randint(0, flat.numel(), (1,), generator=gen))
            if key.endswith(".packed_weight") and kind < 3:
                flat[at] = int(flat[at]) | (3 << (2 * (kind % 4)))
            elif key.endswith(".weight_scales") and kind < 4:
                flat[at] = (float("nan"), float("inf"), 0.0, -0.25)[kind]
            elif kind == 4 and value.dtype in (torch.uint8, torch.float16):
                state[key] = value.float()
            elif kind == 5:
                state[key] = [1, 2, 3]
        errors, checked = ingest._plan_checks(state)
        bad = _device_checks_on_the_host(state, checked)
        ours = ingest._first_error(errors, checked, bad)
        try:
            loader._validate_state(state)
            expected = None
        except RuntimeError as exc:
            expected = str(exc)
        assert ours == expected, (trial, ours, expected)
