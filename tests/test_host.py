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

    structs = [_native.IvbTernary, _native.IvbLayerDesc, _native.IvbModelDesc]
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


def test_build_model_uses_every_state_entry() -> None:
    from ivonar_inference_b200 import model as M
    from ivonar_inference_b200 import synthetic

    payload = synthetic.tiny()
    state = synthetic.synthetic_state(payload, 0, "reference_tests")
    built = M.build_model(payload, state)
    assert [b.mixer_type for b in built.blocks] == ["mamba", "mla", "mamba"]
    assert built.blocks[1].mixer.rope_dim == 2 and built.blocks[1].mixer.nope_dim == 2
    extra = dict(state)
    extra["blocks.0.mixer.unknown"] = torch.zeros(1)
    with pytest.raises(RuntimeError, match="does not use"):
        M.build_model(payload, extra)
    missing = dict(state)
    del missing["final_norm.weight"]
    with pytest.raises(RuntimeError, match="missing final_norm.weight"):
        M.build_model(payload, missing)
    bad = dict(state)
    bad["blocks.0.ffn.down_proj.packed_weight"] = bad["blocks.0.ffn.down_proj.packed_weight"].clone()
    bad["blocks.0.ffn.down_proj.packed_weight"][0, 0] = 0xFF
    with pytest.raises(RuntimeError, match="reserved code 3"):
        M.build_model(payload, bad)
    with pytest.raises(ValueError, match="incompatible"):
        M.ModelConfig.from_payload({**payload, "architecture_version": 2})
    with pytest.raises(ValueError, match="mixture-of-experts"):
        M.ModelConfig.from_payload({**payload, "num_experts": 4})


def test_checkpoint_round_trip(tmp_path: Path) -> None:
    from ivonar_inference_b200 import model as M
    from ivonar_inference_b200 import synthetic

    payload = synthetic.config0()
    state = synthetic.synthetic_state(payload, 1)
    path = tmp_path / "packed.pt"
    torch.save({"format": M.PACKED_FORMAT, "schema_version": 1, "config": payload, "model_state": state}, path)
    loaded = M.load_checkpoint(path)
    assert loaded.config.vocab_size == 512 and len(loaded.blocks) == 4
    assert torch.equal(loaded.token_io.projection.packed_weight, state["token_io.projection.packed_weight"])
    torch.save({"format": "other", "schema_version": 1, "config": payload, "model_state": state}, path)
    with pytest.raises(RuntimeError, match="unsupported checkpoint format"):
        M.load_checkpoint(path)


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


def test_rope_table_matches_the_reference_rotary_layout() -> None:
    from ivonar_inference_b200.model import Rotary, rope_table

    rot = Rotary(16, base_context=32, active_context=64, scaling_strategy="linear")
    table = rope_table(rot, 64)
    assert table.shape == (64, 8, 2)
    inv = 1.0 / (10000.0 ** (torch.arange(0, 16, 2, dtype=torch.float32) / 16))
    pos = torch.arange(64, dtype=torch.float32) / 2.0
    torch.testing.assert_close(table[..., 0], torch.cos(pos[:, None] * inv), rtol=0, atol=0)
    yarn = rope_table(Rotary(16, 32, 64, scaling_strategy="yarn_like"), 4)
    none = rope_table(Rotary(16, 32, 64, scaling_strategy="none"), 4)
    assert not torch.equal(yarn, none)


def test_the_b200_decoder_refuses_a_cpu_device() -> None:
    from ivonar_inference_b200 import B200Decoder, KernelError, synthetic

    model = synthetic.synthetic_model(synthetic.tiny(), 0, "reference_tests")
    with pytest.raises(KernelError, match="CUDA"):
        B200Decoder(model, device="cpu")


def test_build_decoder_has_no_cpu_fallback_without_the_reference(monkeypatch) -> None:
    from ivonar_inference_b200 import KernelError, decoder, synthetic

    monkeypatch.setattr(decoder, "_reference_static_decoder", lambda: None)
    model = synthetic.synthetic_model(synthetic.tiny(), 0, "reference_tests")
    with pytest.raises(KernelError):
        decoder.build_decoder(model, "cpu")
