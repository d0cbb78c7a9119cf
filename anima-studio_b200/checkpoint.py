"""safetensors checkpoints on disk: the reader of app/weights.js:29-99 (SafeTensors.open, has,
info, bytes, f32) and a writer, with no dependency on the safetensors package.

File format (the one the reference parses): an 8-byte little-endian header length n, n bytes of
JSON mapping each tensor name to {"dtype", "shape", "data_offsets": [begin, end]} (offsets into
the data section that follows the header; an optional "__metadata__" entry holds string pairs),
then the data section, each tensor row-major and little-endian.

`SafeTensors(path, prefix)` maps the file and hands out CPU tensors by name, with the reference's
prefix convention (app/weights.js:29-41: the DiT lives under "model.diffusion_model." in the
published checkpoints, tools/reference.py:281). `checkpoint.mapping()` is a read-only dict view
that loads each tensor when it is first asked for, so AnimaDiT, linear_weights and load_lora take a
file exactly as they take an in-memory dict; quantized linears keep their comfy_quant companions
(weight, weight_scale, weight_s_rel, weight_s_channel, weight_codebook and the JSON comfy_quant
tensor) as stored.
"""

from __future__ import annotations

import json
import mmap
import os
import struct
from collections.abc import Mapping

import numpy as np
import torch

# safetensors dtype names -> (torch dtype, bytes per element)
DTYPES = {
    "F64": (torch.float64, 8), "F32": (torch.float32, 4), "F16": (torch.float16, 2), "BF16": (torch.bfloat16, 2),
    "I64": (torch.int64, 8), "I32": (torch.int32, 4), "I16": (torch.int16, 2), "I8": (torch.int8, 1),
    "U8": (torch.uint8, 1), "BOOL": (torch.bool, 1), "F8_E4M3": (torch.float8_e4m3fn, 1),
    "F8_E5M2": (torch.float8_e5m2, 1),
}
NAMES = {dt: name for name, (dt, _) in DTYPES.items()}
MAX_HEADER = 100 << 20  # a header larger than this is a corrupt file, not a checkpoint


class SafeTensors:
    """One safetensors file, memory-mapped; names are looked up under `prefix`."""

    def __init__(self, path: str, prefix: str = ""):
        self.path = path
        self.prefix = prefix
        self._f = open(path, "rb")
        size = os.fstat(self._f.fileno()).st_size
        if size < 8:
            raise ValueError(f"{path}: {size} bytes is too short for a safetensors file")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        (n,) = struct.unpack("<Q", self._mm[:8])
        if n > MAX_HEADER or 8 + n > size:
            raise ValueError(f"{path}: header length {n} does not fit the {size}-byte file")
        try:
            header = json.loads(bytes(self._mm[8:8 + n]).decode("utf-8"))
        except (UnicodeDecodeError, json.JSONDecodeError) as e:
            raise ValueError(f"{path}: header is not JSON ({e})") from None
        if not isinstance(header, dict):
            raise ValueError(f"{path}: header is not a JSON object")
        self.metadata = header.pop("__metadata__", None) or {}
        self.data_start = 8 + n
        data_len = size - self.data_start
        self.header = {}
        for name, t in header.items():
            try:
                dtype, shape, (a, b) = t["dtype"], [int(d) for d in t["shape"]], t["data_offsets"]
            except (KeyError, TypeError, ValueError):
                raise ValueError(f"{path}: malformed entry for {name}") from None
            if dtype not in DTYPES:
                raise ValueError(f"{path}: {name} has unsupported dtype {dtype}")
            nbytes = int(np.prod(shape, dtype=np.int64)) * DTYPES[dtype][1]
            if not (0 <= a <= b <= data_len) or b - a != nbytes:
                raise ValueError(f"{path}: {name} data_offsets [{a}, {b}) do not hold {dtype}{shape} inside "
                                 f"the {data_len}-byte data section")
            self.header[name] = (dtype, shape, (int(a), int(b)))

    def close(self):
        self._mm.close()
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def keys(self) -> list[str]:
        """Tensor names under the prefix, with the prefix removed."""
        p = len(self.prefix)
        return [k[p:] for k in self.header if k.startswith(self.prefix)]

    def has(self, name: str) -> bool:
        return self.prefix + name in self.header

    def info(self, name: str):
        """(dtype name, shape, (begin, end)) of `name` (app/weights.js:44-48)."""
        t = self.header.get(self.prefix + name)
        if t is None:
            raise KeyError(f"missing tensor {self.prefix + name}")
        return t

    def bytes(self, name: str) -> memoryview:
        """The raw little-endian bytes of `name` (app/weights.js:50-54), a view into the file."""
        _, _, (a, b) = self.info(name)
        return memoryview(self._mm)[self.data_start + a:self.data_start + b]

    def tensor(self, name: str) -> torch.Tensor:
        """`name` as a CPU tensor of its stored dtype (a copy: the file stays read-only)."""
        dtype, shape, (a, b) = self.info(name)
        tdt, _ = DTYPES[dtype]
        if a == b:
            return torch.empty(shape, dtype=tdt)
        raw = torch.frombuffer(bytearray(self.bytes(name)), dtype=torch.uint8)
        return raw.view(tdt).reshape(shape)

    def f32(self, name: str) -> torch.Tensor:
        """`name` converted to fp32, as app/weights.js:60-71 does for vectors and LoRA alphas."""
        return self.tensor(name).to(torch.float32)

    def mapping(self) -> "LazyTensors":
        return LazyTensors(self)


class LazyTensors(Mapping):
    """Read-only name -> tensor view of a SafeTensors file that loads each tensor on first use."""

    def __init__(self, st: SafeTensors):
        self.st = st
        self._names = st.keys()
        self._cache: dict = {}

    def __getitem__(self, name):
        t = self._cache.get(name)
        if t is None:
            t = self._cache[name] = self.st.tensor(name)
        return t

    def __contains__(self, name):
        return self.st.has(name)

    def __iter__(self):
        return iter(self._names)

    def __len__(self):
        return len(self._names)

    def release(self):
        """Drop the host copies (after the weights are on the device)."""
        self._cache.clear()


def save_file(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """Write tensors (name -> CPU or device tensor) as a safetensors file: data in name order with
    no gaps (readers reject holes in the data section), the header padded with spaces so the data
    starts 8-byte aligned."""
    entries, blobs, off = {}, [], 0
    for name in sorted(tensors):
        t = tensors[name].detach().to("cpu").contiguous()
        if t.dtype not in NAMES:
            raise ValueError(f"{name}: dtype {t.dtype} has no safetensors name")
        raw = t.reshape(-1).view(torch.uint8).numpy().tobytes() if t.numel() else b""
        entries[name] = {"dtype": NAMES[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        entries["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    head = json.dumps(entries, separators=(",", ":")).encode()
    head += b" " * ((-len(head)) % 8)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(head)))
        f.write(head)
        for b in blobs:
            f.write(b)
    os.replace(tmp, path)


def open_dit(path: str, prefix: str = "model.diffusion_model.") -> LazyTensors:
    """The DiT tensors of a checkpoint file, named as AnimaDiT expects ("blocks.0...")."""
    st = SafeTensors(path, prefix)
    if not st.keys():
        st.close()
        raise ValueError(f"{path}: no tensors under {prefix!r}")
    return st.mapping()
