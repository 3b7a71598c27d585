"""Checkpoint ingest straight to the GPU: the fast path of the reference's ``load_model``
(``loader.py:212-258``).

The reference reads the whole checkpoint into host memory (``torch.load(map_location="cpu")``), checks
every packed buffer on the CPU in 8 Mi chunks and every scale buffer (``_validate_state``,
``loader.py:94-112``), assembles the model on the CPU and then moves it to the device. Here the file is
memory-mapped and its tensor records are copied to the device as one block; all packed buffers and
scales are checked on the device by one kernel (``ivb_validate_buffers``), and the reference's own
``build_model`` assembles the model from the device tensors, its host-side content checks replaced by
the device ones. Errors are the reference's, raised for the same entry: the entries are walked in the
reference's order and the first failing check (not a tensor, wrong dtype, the reserved code 3, a scale
that is not finite, a scale that is not positive) raises the reference's message. The result is the
reference's ``LoadedModel``; other devices take the reference's loader unchanged.
"""

from __future__ import annotations

import collections
import contextlib
import ctypes
import io
import pickle
import struct
import threading
import zipfile
from pathlib import Path
from typing import Any

import numpy as np
import torch

from . import _native as native
from . import _reference

_PATCH_LOCK = threading.Lock()


def _plan_checks(state: dict[str, Any]) -> tuple[dict[int, str], list[tuple[int, str, int]]]:
    """The host part of the reference's state checks (``loader.py:94-112``): the type and dtype errors by
    entry position, and the (position, key, kind) of every buffer whose content the device checks."""

    errors: dict[int, str] = {}
    checked: list[tuple[int, str, int]] = []
    for pos, (key, value) in enumerate(state.items()):
        if not isinstance(value, torch.Tensor):
            errors[pos] = f"model_state entry is not a tensor: {key}"
        elif key.endswith(".packed_weight"):
            if value.dtype != torch.uint8:
                errors[pos] = f"packed ternary buffer must be uint8: {key}"
            else:
                checked.append((pos, key, native.IVB_CHECK_PACKED))
        elif key.endswith(".weight_scales"):
            if value.dtype != torch.float16:
                errors[pos] = f"g128 scale buffer must be float16: {key}"
            else:
                checked.append((pos, key, native.IVB_CHECK_SCALES))
    return errors, checked


def _first_error(errors: dict[int, str], checked: list[tuple[int, str, int]], bad: tuple[int, int, int]) -> str | None:
    """The message the reference raises first: `bad` holds the device's lowest failing index into
    `checked` per content check (reserved code 3, non-finite scale, non-positive scale; len(checked)
    when none failed). Entries are taken in state order, and one scale buffer fails "finite" before
    "positive", as the reference tests them."""

    errors = dict(errors)
    for idx, message in zip(bad, ("packed ternary buffer contains the reserved code 3: {}",
                                  "g128 scale buffer must contain only finite values: {}",
                                  "g128 scale buffer must contain only positive values: {}")):
        if 0 <= idx < len(checked):
            pos, key, _ = checked[idx]
            errors.setdefault(pos, message.format(key))
    return errors[min(errors)] if errors else None


def validate_state_device(state: dict[str, Any], device: torch.device) -> None:
    """The reference's state checks (``loader.py:94-112``) with the content checks on the device: one
    launch over every packed and scale buffer of the right dtype, one synchronisation. Then the entries
    are walked in the reference's order and the first failing check raises the reference's message."""

    errors, checked = _plan_checks(state)
    bad = (len(checked),) * 3
    if checked:
        lib = native.library()
        descs = (native.IvbCheckBuffer * len(checked))()
        keep = []
        for i, (_, key, kind) in enumerate(checked):
            t = state[key].contiguous()
            keep.append(t)
            descs[i].data = t.data_ptr() if t.numel() else None
            descs[i].count = t.numel()
            descs[i].kind = kind
        raw = torch.frombuffer(bytearray(ctypes.string_at(ctypes.addressof(descs), ctypes.sizeof(descs))), dtype=torch.uint8)
        dev_descs = raw.to(device)
        out = torch.empty(3, dtype=torch.int32, device=device)
        stream = torch.cuda.current_stream(device).cuda_stream
        native.check(lib.ivb_validate_buffers(dev_descs.data_ptr(), len(checked), out.data_ptr(), stream),
                     "ivb_validate_buffers")
        bad = tuple(int(v) for v in out.cpu())
    message = _first_error(errors, checked, bad)
    if message is not None:
        raise RuntimeError(message)


_STORAGE_DTYPES = {
    "ByteStorage": torch.uint8, "CharStorage": torch.int8, "ShortStorage": torch.int16, "IntStorage": torch.int32,
    "LongStorage": torch.int64, "HalfStorage": torch.float16, "BFloat16Storage": torch.bfloat16,
    "FloatStorage": torch.float32, "DoubleStorage": torch.float64, "BoolStorage": torch.bool,
}


class _Unsupported(Exception):
    """The archive holds something the direct reader does not handle; ``torch.load`` reads it instead."""


class _StorageType:
    def __init__(self, dtype: torch.dtype) -> None:
        self.dtype = dtype


class _ArchiveUnpickler(pickle.Unpickler):
    """The ``data.pkl`` of a ``torch.save`` archive with every storage resolved to a view of one device
    block. Only the globals a state-dict checkpoint uses are resolved (``OrderedDict``, the typed storage
    classes, ``torch._utils._rebuild_tensor_v2``), all of which ``torch.load(weights_only=True)`` allows;
    any other global stops the reader and ``torch.load`` takes over, with its own checks and errors."""

    def __init__(self, data: bytes, records: dict[str, tuple[int, int]], block: torch.Tensor) -> None:
        super().__init__(io.BytesIO(data))
        self.records = records  # storage key -> (offset in the block, bytes)
        self.block = block
        self.views: dict[str, torch.Tensor] = {}

    def find_class(self, module: str, name: str):
        if module == "collections" and name == "OrderedDict":
            return collections.OrderedDict
        if module == "torch" and name in _STORAGE_DTYPES:
            return _StorageType(_STORAGE_DTYPES[name])
        if module == "torch._utils" and name == "_rebuild_tensor_v2":
            return self._rebuild
        raise _Unsupported(f"{module}.{name}")

    def persistent_load(self, pid):
        if not (isinstance(pid, tuple) and len(pid) == 5 and pid[0] == "storage" and isinstance(pid[1], _StorageType)):
            raise _Unsupported("persistent id")
        _, kind, key, _location, numel = pid
        view = self.views.get(key)
        if view is None:
            offset, nbytes = self.records.get(f"data/{key}", (0, -1))
            if nbytes != int(numel) * kind.dtype.itemsize or offset % kind.dtype.itemsize:
                raise _Unsupported(f"storage {key}")
            view = self.block[offset:offset + nbytes].view(kind.dtype)
            self.views[key] = view
        return view

    @staticmethod
    def _rebuild(storage, storage_offset, size, stride, requires_grad, backward_hooks, metadata=None):
        if not isinstance(storage, torch.Tensor) or backward_hooks or metadata:
            raise _Unsupported("tensor")
        out = storage.as_strided(tuple(size), tuple(stride), storage.storage_offset() + int(storage_offset))
        return out.requires_grad_() if requires_grad else out


def _read_archive(path: Path, target: torch.device):
    """A ``torch.save`` archive read straight to `target`: the zip directory gives every storage record's
    place in the file (records are stored uncompressed), the span holding them is copied to the device
    in one block from a memory map of the file, and ``data.pkl`` is unpickled with each tensor rebuilt as
    a view of that block. Returns None when the archive is not of that form (``torch.load`` then reads
    it, and reports what is wrong with it as the reference does)."""

    try:
        with zipfile.ZipFile(path) as archive, open(path, "rb") as raw:
            infos = archive.infolist()
            pickles = [i for i in infos if i.filename.endswith("/data.pkl") and i.filename.count("/") == 1]
            if len(pickles) != 1:
                return None
            prefix = pickles[0].filename[:-len("data.pkl")]
            if prefix + "byteorder" in archive.namelist() and archive.read(prefix + "byteorder") != b"little":
                return None
            records: dict[str, tuple[int, int]] = {}
            for info in infos:
                name = info.filename[len(prefix):] if info.filename.startswith(prefix) else ""
                if not name.startswith("data/"):
                    continue
                if info.compress_type != zipfile.ZIP_STORED:
                    return None
                raw.seek(info.header_offset)
                header = raw.read(30)
                if len(header) != 30 or header[:4] != b"PK\x03\x04":
                    return None
                name_len, extra_len = struct.unpack("<HH", header[26:30])
                records[name] = (info.header_offset + 30 + name_len + extra_len, info.file_size)
            data = archive.read(pickles[0])
        lo = min((off for off, _ in records.values()), default=0)
        hi = max((off + n for off, n in records.values()), default=0)
        if records and hi > path.stat().st_size:
            return None
        if records:
            mapped = np.memmap(path, dtype=np.uint8, mode="c", offset=lo, shape=(hi - lo,))
            block = torch.from_numpy(mapped).to(target)
            del mapped
        else:
            block = torch.empty(0, dtype=torch.uint8, device=target)
        relative = {name: (off - lo, n) for name, (off, n) in records.items()}
        return _ArchiveUnpickler(data, relative, block).load()
    except (_Unsupported, zipfile.BadZipFile, pickle.UnpicklingError, ValueError, OSError, EOFError):
        return None


def _state_to_device(state: dict[str, Any], target: torch.device, file_bytes: int) -> dict[str, Any]:
    """The checkpoint's tensors on `target` in one host-to-device copy. ``torch.load(mmap=True)`` maps
    the file once and every storage is a slice of that mapping, so the span from the lowest to the
    highest storage byte (at most the file's size) is copied as one block and each tensor becomes a view
    of the device block at its storage's offset (records are 64-byte aligned in the file, so every view
    keeps its dtype's alignment). Anything else (a storage outside one mapping, a non-CPU tensor) is
    copied tensor by tensor."""

    tensors = [v for v in state.values() if isinstance(v, torch.Tensor) and v.untyped_storage().nbytes()]
    spans = [(t.untyped_storage().data_ptr(), t.untyped_storage().nbytes()) for t in tensors]
    lo = min((ptr for ptr, _ in spans), default=0)
    hi = max((ptr + n for ptr, n in spans), default=0)
    if not tensors or hi - lo > file_bytes or any(t.device.type != "cpu" for t in tensors):
        return {key: value.to(target) if isinstance(value, torch.Tensor) else value for key, value in state.items()}
    host = torch.frombuffer((ctypes.c_uint8 * (hi - lo)).from_address(lo), dtype=torch.uint8)
    block = host.to(target)
    out: dict[str, Any] = {}
    for key, value in state.items():
        if not isinstance(value, torch.Tensor):
            out[key] = value
            continue
        storage = value.untyped_storage()
        if not storage.nbytes():
            out[key] = torch.empty_strided(value.shape, value.stride(), dtype=value.dtype, device=target)
            continue
        start = storage.data_ptr() - lo
        flat = block[start:start + storage.nbytes()].view(value.dtype)
        out[key] = flat.as_strided(value.shape, value.stride(), flat.storage_offset() + value.storage_offset())
    return out


@contextlib.contextmanager
def _checked_on_device(loader):
    """While held, the reference loader's host-side state checks are skipped (the caller has run them on
    the device): ``build_model`` calls the module-level ``_validate_state``."""

    with _PATCH_LOCK:
        original = loader._validate_state
        loader._validate_state = lambda state: None
        try:
            yield
        finally:
            loader._validate_state = original


def load_model(path: str | Path, device: str | torch.device = "cuda", expected_tokenizer_sha256: str | None = None,
               materialize: bool = True):
    """The reference's ``load_model`` (same arguments and defaults, checks, errors and ``LoadedModel``
    result) with the checkpoint streamed to `device` and validated there. ``materialize`` unpacks the
    weights for the torch path as the reference does; callers that serve through the B200 kernels pass
    False (the kernels read the packed weights), as the reference's own kernel callers do."""

    loader = _reference.module("loader")
    target = torch.device(device)
    if target.type != "cuda":
        return loader.load_model(path, target, expected_tokenizer_sha256, materialize)
    config_mod = _reference.module("config")
    quantization = _reference.module("quantization")
    model_file = Path(path)
    if target.index is None:
        target = torch.device("cuda", torch.cuda.current_device())
    payload = _read_archive(model_file, target)
    direct = payload is not None
    if not direct:
        payload = torch.load(model_file, map_location="cpu", weights_only=True, mmap=True)
    if not isinstance(payload, dict):
        raise RuntimeError(f"invalid Ivonar checkpoint: {model_file}")
    if payload.get("format") != loader.PACKED_FORMAT or payload.get("schema_version") != loader.PACKED_SCHEMA_VERSION:
        raise RuntimeError(
            f"unsupported checkpoint format; expected {loader.PACKED_FORMAT} schema {loader.PACKED_SCHEMA_VERSION}")
    config = config_mod.ModelConfig.from_payload(payload.get("config"))
    tokenizer_sha256 = str(payload["tokenizer_sha256"]) if payload.get("tokenizer_sha256") else None
    if expected_tokenizer_sha256 is not None:
        if tokenizer_sha256 is None:
            raise RuntimeError("checkpoint is missing tokenizer_sha256")
        if tokenizer_sha256 != str(expected_tokenizer_sha256):
            raise RuntimeError(
                f"tokenizer SHA-256 mismatch: expected {expected_tokenizer_sha256}, found {tokenizer_sha256}")
    state = payload.get("model_state")
    if not isinstance(state, dict):
        raise RuntimeError("checkpoint model_state is invalid")
    on_device = dict(state) if direct else _state_to_device(state, target, model_file.stat().st_size)
    validate_state_device(on_device, target)
    with _checked_on_device(loader):
        model = loader.build_model(config, on_device)
    model.to(target)  # modules the loader creates from constants (none hold checkpoint bytes)
    model.eval()
    if materialize:
        loader.materialize_weights(model, quantization.runtime_dtype(target))
    return loader.LoadedModel(
        model=model,
        config=config,
        path=model_file,
        lineup=str(payload["lineup"]) if payload.get("lineup") is not None else None,
        stage=str(payload["stage"]) if payload.get("stage") is not None else None,
        phase=str(payload["phase"]) if payload.get("phase") is not None else None,
        step=int(payload.get("step", 0) or 0),
        tokenizer_sha256=tokenizer_sha256,
    )
