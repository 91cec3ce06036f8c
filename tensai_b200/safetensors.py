"""Safetensors checkpoints for quantize-on-load: the reader and writer of
tensai's encoding/safetensors package (safetensors.go) in Python, plus the
B200 path from a checkpoint's raw bytes to a resident quantized matrix.

The format: an 8-byte little-endian header length, a JSON header mapping each
tensor name to {dtype, shape, data_offsets} (and an optional __metadata__ of
strings), then the raw little-endian buffer. As in the Go package
(safetensors.go:66-118), Open parses only the header and checks it (length
below 100 MB, offsets ordered, no negative dimension, byte size matching the
shape for the known dtypes); each tensor is read on demand from a memory map.
Tensor() widens F16, BF16 and F64 to float32 on the host like
safetensors.go:165-237; DeviceTensor() instead copies the stored bytes as
they are to the GPU, and QuantizeLinear() hands a BF16 / F16 / F32 Linear
weight ([out, in], as Hugging Face checkpoints store it) to the device
quantizer (tq_quantize4_linear_dev / tq_quantize8_linear_dev: transpose,
widening and QuantizeMatrix4 or QuantizeMatrix in one kernel), so a 7B
checkpoint needs no float32 copy anywhere. OpenSharded reads a
model.safetensors.index.json (safetensors.go:305-364). Save writes F32
(safetensors.go:252-303).
"""
from __future__ import annotations

import json
import mmap
import os
import struct

import numpy as np

__all__ = ["File", "Open", "Shards", "OpenSharded", "Save", "SaveFile"]

_MAX_HEADER = 100 << 20
_SIZES = {"F32": 4, "F16": 2, "BF16": 2, "F64": 8}


def _f16_to_f32(h: np.ndarray) -> np.ndarray:
    """IEEE binary16 bits to float32, subnormals, infinities and NaNs included."""
    h = h.astype(np.uint32)
    sign = (h >> 15) << 31
    exp = (h >> 10) & 0x1F
    frac = h & 0x3FF
    out = sign | ((exp + 112) << 23) | (frac << 13)  # normal: rebias 15 -> 127
    out = np.where(exp == 0x1F, sign | (0xFF << 23) | (frac << 13), out)  # inf / NaN
    # zero and subnormals: frac * 2^-24 exactly, with the sign
    sub = (frac.astype(np.float32) * np.float32(2.0 ** -24)).view(np.uint32) | sign
    out = np.where(exp == 0, sub, out)
    return out.astype(np.uint32).view(np.float32)


class File:
    """An open safetensors checkpoint; tensor data is read on demand."""

    def __init__(self, path: str):
        self._fh = open(path, "rb")
        try:
            head = self._fh.read(8)
            if len(head) < 8:
                raise ValueError("safetensors: reading header length: file too short")
            (n,) = struct.unpack("<Q", head)
            if n == 0 or n >= _MAX_HEADER:
                raise ValueError(f"safetensors: implausible header length {n}")
            header = self._fh.read(n)
            if len(header) < n:
                raise ValueError("safetensors: reading header: file too short")
            try:
                raw = json.loads(header)
            except ValueError as e:
                raise ValueError(f"safetensors: parsing header: {e}") from None
            self._data_off = 8 + n
            self._entries, self._meta = {}, None
            for name, e in raw.items():
                if name == "__metadata__":
                    self._meta = {str(k): str(v) for k, v in e.items()}
                    continue
                lo, hi = (int(x) for x in e["data_offsets"])
                shape = [int(d) for d in e["shape"]]
                if lo < 0 or hi < lo:
                    raise ValueError(f"safetensors: entry {name!r} has invalid offsets {[lo, hi]}")
                if any(d < 0 for d in shape):
                    raise ValueError(f"safetensors: entry {name!r} has negative dimension in {shape}")
                size = _SIZES.get(e["dtype"])
                if size is not None and int(np.prod(shape, dtype=np.int64)) * size != hi - lo:
                    raise ValueError(f"safetensors: entry {name!r}: shape {shape} does not match {hi - lo} bytes")
                self._entries[name] = (e["dtype"], shape, lo, hi)
            self._names = sorted(self._entries)
            size = os.fstat(self._fh.fileno()).st_size
            self._map = mmap.mmap(self._fh.fileno(), 0, access=mmap.ACCESS_READ) if size else None
        except Exception:
            self._fh.close()
            raise

    def Close(self) -> None:
        if self._map is not None:
            self._map.close()
            self._map = None
        self._fh.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.Close()

    def Names(self) -> list[str]:
        """Tensor names, sorted."""
        return list(self._names)

    def Metadata(self):
        """The free-form __metadata__ strings, or None."""
        return None if self._meta is None else dict(self._meta)

    def Info(self, name: str):
        """(dtype, shape, True) without loading the data, or ("", None, False)."""
        e = self._entries.get(name)
        if e is None:
            return "", None, False
        return e[0], list(e[1]), True

    def Raw(self, name: str) -> np.ndarray:
        """The tensor's stored bytes (a read-only view of the file)."""
        dtype, shape, lo, hi = self._entry(name)
        if self._data_off + hi > len(self._map if self._map is not None else b""):
            raise ValueError(f"safetensors: reading tensor {name!r}: file too short")
        return np.frombuffer(self._map, np.uint8, hi - lo, self._data_off + lo)

    def Tensor(self, name: str) -> np.ndarray:
        """The tensor as float32 (F16, BF16 and F64 widened or rounded); a
        scalar (empty shape) comes back with shape [1]."""
        dtype, shape, _, _ = self._entry(name)
        if dtype not in _SIZES:
            raise ValueError(f"safetensors: unsupported dtype {dtype!r} (tensor {name!r})")
        b = self.Raw(name)
        if dtype == "F32":
            v = b.view("<f4").astype(np.float32)
        elif dtype == "F16":
            v = _f16_to_f32(b.view("<u2"))
        elif dtype == "BF16":
            v = (b.view("<u2").astype(np.uint32) << 16).view(np.float32)
        else:
            v = b.view("<f8").astype(np.float32)
        return v.reshape(shape if shape else [1])

    def DeviceTensor(self, name: str, device="cuda"):
        """The stored values on the GPU in their own dtype (torch float32,
        float16 or bfloat16), copied from the file without conversion."""
        import torch
        dtype, shape, _, _ = self._entry(name)
        kinds = {"F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16}
        if dtype not in kinds:
            raise ValueError(f"safetensors: {dtype} tensor {name!r} has no device form")
        host = torch.from_numpy(self.Raw(name).copy())
        return host.to(device).view(kinds[dtype]).reshape(shape if shape else [1])

    def QuantizeLinear(self, name: str, bits: int = 4, stream=None) -> int:
        """A resident int4 (or int8) matrix handle of the Linear weight `name`
        ([out, in] in the file): the matrix the Go loader builds with
        Matrix().T() and QuantizeMatrix4 (_example/qwen/model.go:126-140),
        quantized on the GPU from the file's own bytes."""
        from .quant import quantize_linear_dev
        w = self.DeviceTensor(name)
        if w.dim() != 2:
            raise ValueError(f"safetensors: {name!r} is not a 2-D Linear weight")
        h = quantize_linear_dev(w, bits, stream)
        if stream is not None:
            stream.synchronize()
        else:
            import torch
            torch.cuda.synchronize()
        return h

    def _entry(self, name: str):
        e = self._entries.get(name)
        if e is None:
            raise KeyError(f"safetensors: no tensor {name!r}")
        return e


def Open(path: str) -> File:
    """Opens a safetensors file, parsing its header."""
    return File(path)


class Shards:
    """A checkpoint split over several files by a model.safetensors.index.json."""

    def __init__(self, index_path: str):
        with open(index_path, "rb") as fh:
            try:
                idx = json.load(fh)
            except ValueError as e:
                raise ValueError(f"safetensors: parsing index: {e}") from None
        wm = idx.get("weight_map") or {}
        if not wm:
            raise ValueError("safetensors: index has no weight_map")
        d = os.path.dirname(index_path)
        self._files: dict[str, File] = {}
        self._by_name: dict[str, File] = {}
        try:
            for name, shard in wm.items():
                f = self._files.get(shard)
                if f is None:
                    f = self._files[shard] = File(os.path.join(d, shard))
                if not f.Info(name)[2]:
                    raise ValueError(f"safetensors: index maps {name!r} to {shard}, which lacks it")
                self._by_name[name] = f
        except Exception:
            self.Close()
            raise
        self._names = sorted(self._by_name)

    def Close(self) -> None:
        for f in self._files.values():
            f.Close()
        self._files.clear()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.Close()

    def Names(self) -> list[str]:
        return list(self._names)

    def Info(self, name: str):
        f = self._by_name.get(name)
        return ("", None, False) if f is None else f.Info(name)

    def File(self, name: str) -> File:
        """The shard holding `name`."""
        f = self._by_name.get(name)
        if f is None:
            raise KeyError(f"safetensors: no tensor {name!r}")
        return f

    def Tensor(self, name: str) -> np.ndarray:
        return self.File(name).Tensor(name)

    def QuantizeLinear(self, name: str, bits: int = 4, stream=None) -> int:
        return self.File(name).QuantizeLinear(name, bits, stream)


def OpenSharded(index_path: str) -> Shards:
    """Opens a sharded checkpoint through its index; shards are resolved
    relative to the index file."""
    return Shards(index_path)


def Save(fh, tensors: dict, meta: dict | None = None) -> None:
    """Writes float32 tensors, names sorted, with optional __metadata__; the
    header is padded with spaces so the buffer starts 8-byte aligned."""
    if "__metadata__" in tensors:
        raise ValueError("safetensors: '__metadata__' is a reserved name")
    names = sorted(tensors)
    arrays = [np.ascontiguousarray(tensors[n], dtype="<f4") for n in names]
    head = {}
    if meta:
        head["__metadata__"] = {str(k): str(v) for k, v in meta.items()}
    off = 0
    for n, a in zip(names, arrays):
        head[n] = {"dtype": "F32", "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes
    hb = json.dumps(head, separators=(",", ":")).encode("utf-8")
    hb += b" " * ((8 - (8 + len(hb)) % 8) % 8)
    fh.write(struct.pack("<Q", len(hb)))
    fh.write(hb)
    for a in arrays:
        fh.write(a.tobytes())


def SaveFile(path: str, tensors: dict, meta: dict | None = None) -> None:
    with open(path, "wb") as fh:
        Save(fh, tensors, meta)
