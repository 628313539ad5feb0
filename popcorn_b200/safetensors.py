"""Safetensors archives and the Gemma weight loader (the input side of the
decode path).

The reference reads weights through MTLSafeTensors (a Swift package pinned
only to `branch: "main"` in Examples/GemmaCLI/Package.swift:15, not vendored)
and Examples/GemmaCLI/Sources/GemmaCLI/Gemma4WeightLoader.swift. The format
is the published safetensors layout: an 8-byte little-endian header length
N, N bytes of JSON {name: {"dtype", "shape", "data_offsets": [begin, end]},
"__metadata__": {...}}, then the tensor bytes, offsets counted from the end
of the header, packed with no padding. Tensors are read as numpy views of a
read-only memory map; `to_device` copies one into a freshly allocated (so
256-byte aligned) torch tensor — which also cures the case
Gemma4WeightLoader.swift:99-105 copies for: a U32 tensor that follows an
odd-length 16-bit tensor sits at a 2-byte file offset.
"""
import json
import mmap
import os
import struct

import numpy as np

# safetensors dtype -> (numpy storage type, torch dtype name)
_DTYPES = {
    "F32": (np.float32, "float32"), "F16": (np.float16, "float16"), "BF16": (np.uint16, "bfloat16"),
    "F64": (np.float64, "float64"), "I8": (np.int8, "int8"), "I16": (np.int16, "int16"),
    "I32": (np.int32, "int32"), "I64": (np.int64, "int64"), "U8": (np.uint8, "uint8"),
    "U16": (np.uint16, "uint16"), "U32": (np.uint32, "uint32"), "U64": (np.uint64, "uint64"),
    "BOOL": (np.bool_, "bool"),
}


class SafeTensorsError(Exception):
    pass


class SafeTensors:
    """One archive file, or every `*.safetensors` file of a directory (the
    names of all shards in one table)."""

    def __init__(self, path):
        files = ([os.path.join(path, f) for f in sorted(os.listdir(path)) if f.endswith(".safetensors")]
                 if os.path.isdir(path) else [path])
        if not files:
            raise SafeTensorsError("no .safetensors files in %s" % path)
        self._maps = []
        self._entries = {}
        self.metadata = {}
        for f in files:
            with open(f, "rb") as fh:
                mm = mmap.mmap(fh.fileno(), 0, access=mmap.ACCESS_READ)
            if len(mm) < 8:
                raise SafeTensorsError("%s: file too short" % f)
            (n,) = struct.unpack("<Q", mm[:8])
            if 8 + n > len(mm):
                raise SafeTensorsError("%s: header length %d beyond the file" % (f, n))
            try:
                header = json.loads(bytes(mm[8:8 + n]).decode("utf-8"))
            except ValueError as e:
                raise SafeTensorsError("%s: bad JSON header (%s)" % (f, e))
            base = 8 + n
            self.metadata.update(header.pop("__metadata__", {}) or {})
            for name, e in header.items():
                dt = e.get("dtype")
                if dt not in _DTYPES:
                    raise SafeTensorsError("%s: tensor %s has unknown dtype %r" % (f, name, dt))
                shape = tuple(int(d) for d in e.get("shape", []))
                b, end = (int(v) for v in e["data_offsets"])
                count = int(np.prod(shape)) if shape else 1
                if end - b != count * np.dtype(_DTYPES[dt][0]).itemsize or base + end > len(mm) or b < 0:
                    raise SafeTensorsError("%s: tensor %s: data_offsets %r do not fit dtype / shape / file"
                                           % (f, name, [b, end]))
                if name in self._entries:
                    raise SafeTensorsError("tensor %s appears in two shards" % name)
                self._entries[name] = (len(self._maps), dt, shape, base + b, end - b)
            self._maps.append(mm)

    @property
    def names(self):
        return list(self._entries)

    def __contains__(self, name):
        return name in self._entries

    def info(self, name):
        """(dtype, shape, file offset, bytes)."""
        if name not in self._entries:
            raise SafeTensorsError("tensor %s not in the archive" % name)
        _, dt, shape, off, nb = self._entries[name]
        return dt, shape, off, nb

    def array(self, name):
        """A read-only numpy view (bf16 as uint16 bits); unaligned offsets allowed."""
        if name not in self._entries:
            raise SafeTensorsError("tensor %s not in the archive" % name)
        i, dt, shape, off, nb = self._entries[name]
        a = np.frombuffer(self._maps[i], dtype=_DTYPES[dt][0], count=nb // np.dtype(_DTYPES[dt][0]).itemsize,
                          offset=off)
        return a.reshape(shape)

    def to_device(self, name, device="cuda"):
        """A torch tensor of the stored dtype on `device`, in its own
        (aligned) allocation."""
        import torch
        dt = self.info(name)[0]
        host = torch.from_numpy(np.ascontiguousarray(self.array(name)).copy())
        if dt == "BF16":
            host = host.view(torch.int16).view(torch.bfloat16)
        elif dt == "U32":
            host = host.view(torch.int32).view(torch.uint32) if hasattr(torch, "uint32") else host.view(torch.int32)
        return host.to(device)

    def close(self):
        for m in self._maps:
            m.close()
        self._maps = []


def save(path, tensors, metadata=None):
    """Writes {name: (numpy array, safetensors dtype)} as one archive (bf16
    arrays as uint16 bits), tensors packed in the given order with no padding."""
    header, blobs, off = {}, [], 0
    for name, (a, dt) in tensors.items():
        a = np.ascontiguousarray(a, dtype=_DTYPES[dt][0])
        raw = a.tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode("utf-8")
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


class Quantization:
    """The config's top-level `quantization` block (bits, group_size)."""

    def __init__(self, bits=4, group_size=64):
        self.bits, self.group_size = int(bits), int(group_size)


class WeightLoader:
    """Gemma4WeightLoader.swift:13-123: hides the MLX vs Transformers tensor
    naming (`language_model.model.*` vs `model.language_model.*`, detected
    at load) and per-tensor quantization: `<name>.weight` is an affine
    4-bit tensor when `<name>.scales` and `<name>.biases` exist and the
    config has a quantization block. Tensors land on `device`."""

    def __init__(self, archive, quantization=None, device="cuda"):
        self.archive, self.quantization, self.device = archive, quantization, device
        names = archive.names
        if any(n.startswith("language_model.model.") for n in names):
            self.prefix = "language_model.model"
        elif any(n.startswith("model.language_model.") for n in names):
            self.prefix = "model.language_model"
        else:
            raise SafeTensorsError("Could not find Gemma language model weights in archive.")

    def qualify(self, relative):
        return "%s.%s" % (self.prefix, relative)

    def layer_prefix(self, index):
        return self.qualify("layers.%d" % index)

    def linear(self, name):
        """LinearWeight: a dense [out, in] tensor or an AffineQuantizedTensor."""
        q = self._maybe_quantized(name)
        return q if q is not None else self.archive.to_device(name + ".weight", self.device)

    def embedding(self, name):
        """EmbeddingTable: dense [vocab, hidden] or quantized, as linear()."""
        return self.linear(name)

    def norm_weight(self, name):
        """A norm weight as f32 on the device: bf16 values widened
        (Support.swift:24-38), other dtypes as stored."""
        import torch
        dt = self.archive.info(name)[0]
        a = self.archive.array(name)
        if dt == "BF16":
            a = (a.astype(np.uint32) << 16).view(np.float32)
        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(self.device)

    def _maybe_quantized(self, name):
        from .api import AffineQuantizedTensor
        if self.quantization is None:
            return None
        w, s, b = name + ".weight", name + ".scales", name + ".biases"
        if not (w in self.archive and s in self.archive and b in self.archive):
            return None
        dt, shape, _, _ = self.archive.info(w)
        if dt != "U32":
            raise SafeTensorsError("Expected U32 packed weights for %s, got %s." % (w, dt))
        import torch
        packed = torch.from_numpy(np.ascontiguousarray(self.archive.array(w)).view(np.int32).copy()).to(self.device)
        per_word = 32 // self.quantization.bits
        out_f, inner = shape
        qt = AffineQuantizedTensor(packed, self.archive.to_device(s, self.device),
                                   self.archive.to_device(b, self.device), (out_f, inner * per_word),
                                   bits=self.quantization.bits, group_size=self.quantization.group_size)
        return qt


__all__ = ["SafeTensors", "SafeTensorsError", "save", "Quantization", "WeightLoader"]
