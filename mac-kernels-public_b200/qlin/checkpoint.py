"""Checkpoint readers: packed linears straight from GGUF and safetensors files.

The reference reads GGUF headers itself (`bench/gguf_headers.py:93-110`, `read_header`) and its
loaders hand ComfyUI a raw-block tensor per layer, which the GPU path repacks once.  Here the file
is memory-mapped, each quantized 2-D tensor's bytes are copied to the GPU once (no intermediate
torch tensor of the whole file), and the resident stage layout is built next to it:

    lin = load_gguf_linears("model.gguf", "cuda")     # name -> GGUFLinear (repacked, cached)
    y = lin["blk.0.attn_qkv.weight"](x)

    w = load_int8_linears("model_int8.safetensors", "cuda")   # "<layer>.weight" int8 + "<layer>.weight_scale"
    y = w["blocks.0.attn.wq"](x, convrot=True, convrot_groupsize=256)

Formats, as written by gguf-py 0.19.0 (`GGUFWriter`) and the safetensors reference writer:
  GGUF v2/v3: "GGUF", u32 version, u64 tensor count, u64 key-value count; key-value pairs
  (u64-length string key, u32 value type, value; arrays as u32 element type, u64 count, elements);
  tensor infos (name, u32 n_dims, u64 dims innermost first, u32 ggml type, u64 offset); tensor data
  from the header's end rounded up to `general.alignment` (32 when absent).  Little-endian only.
  safetensors: u64 header length, a JSON header {name: {dtype, shape, data_offsets}}, the data.
"""
from __future__ import annotations

import json
import math
import mmap
import os
import struct
from dataclasses import dataclass

import numpy as np
import torch

_GGUF_SCALARS = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q",
                 12: "<d"}
# ggml type id -> (values per block, bytes per block) for the types a loader meets in DiT files
GGML_BLOCKS = {0: (1, 4), 1: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34),
               10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210), 20: (32, 18),
               23: (256, 136), 30: (1, 2)}


@dataclass
class TensorInfo:
    name: str
    shape: tuple      # torch order (outermost first)
    qtype: int        # ggml type id (GGUF) or -1 (safetensors)
    dtype: str        # safetensors dtype string, or the ggml type id as text
    offset: int       # absolute byte offset in the file
    nbytes: int


class _Reader:
    def __init__(self, buf):
        self.buf, self.pos = buf, 0

    def take(self, n):
        if self.pos + n > len(self.buf):
            raise ValueError("truncated GGUF header")
        b = self.buf[self.pos:self.pos + n]
        self.pos += n
        return b

    def scalar(self, fmt):
        return struct.unpack(fmt, self.take(struct.calcsize(fmt)))[0]

    def string(self):
        return bytes(self.take(self.scalar("<Q"))).decode("utf-8")

    def value(self, vtype):
        if vtype in _GGUF_SCALARS:
            return self.scalar(_GGUF_SCALARS[vtype])
        if vtype == 8:
            return self.string()
        if vtype == 9:
            etype, n = self.scalar("<I"), self.scalar("<Q")
            return [self.value(etype) for _ in range(n)]
        raise ValueError(f"unknown GGUF value type {vtype}")


class _Mapped:
    def __init__(self, path):
        self.path = os.fspath(path)
        self._f = open(self.path, "rb")
        size = os.fstat(self._f.fileno()).st_size
        # copy-on-write mapping: writable views for torch.frombuffer, the file is never modified
        self.mm = mmap.mmap(self._f.fileno(), size, access=mmap.ACCESS_COPY) if size else b""
        self.tensors: dict[str, TensorInfo] = {}

    def close(self):
        if isinstance(self.mm, mmap.mmap):
            self.mm.close()
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def raw(self, name) -> torch.Tensor:
        """The tensor's bytes as a CPU uint8 tensor over the mapping (no copy; valid while the
        file is open)."""
        t = self.tensors[name]
        if t.nbytes < 0:
            raise ValueError(f"{name}: ggml type {t.qtype} is not sized by this reader")
        if t.nbytes == 0:
            return torch.empty(0, dtype=torch.uint8)
        return torch.frombuffer(self.mm, dtype=torch.uint8, count=t.nbytes, offset=t.offset)


class GGUFFile(_Mapped):
    """Header of a GGUF file plus zero-copy access to each tensor's bytes."""

    def __init__(self, path):
        super().__init__(path)
        mv = memoryview(self.mm)
        try:
            self._parse(_Reader(mv))
        except Exception:
            mv.release()
            self.close()
            raise
        mv.release()

    def _parse(self, r):
        if bytes(r.take(4)) != b"GGUF":
            raise ValueError(f"{self.path}: not a GGUF file")
        self.version = r.scalar("<I")
        if self.version not in (2, 3):
            raise ValueError(f"{self.path}: GGUF version {self.version} is not supported")
        n_tensors, n_kv = r.scalar("<Q"), r.scalar("<Q")
        self.kv = {}
        for _ in range(n_kv):
            key = r.string()
            self.kv[key] = r.value(r.scalar("<I"))
        infos = []
        for _ in range(n_tensors):
            name = r.string()
            dims = [r.scalar("<Q") for _ in range(r.scalar("<I"))]
            infos.append((name, dims, r.scalar("<I"), r.scalar("<Q")))
        align = int(self.kv.get("general.alignment", 32))
        data0 = (r.pos + align - 1) // align * align
        for name, dims, qtype, off in infos:
            numel = math.prod(dims)
            if qtype not in GGML_BLOCKS:
                nbytes = -1  # a type this reader does not size; its bytes are not accessible
            else:
                qk, ts = GGML_BLOCKS[qtype]
                nbytes = numel // qk * ts
            self.tensors[name] = TensorInfo(name, tuple(reversed(dims)), qtype, str(qtype), data0 + off, nbytes)
            if nbytes > 0 and data0 + off + nbytes > len(self.mm):
                raise ValueError(f"{self.path}: tensor {name} runs past the end of the file")

    def orig_shape(self, name):
        """ComfyUI-GGUF's `comfy.gguf.orig_shape.<name>` entry (the torch shape when rows straddle
        blocks), or None."""
        v = self.kv.get(f"comfy.gguf.orig_shape.{name}")
        return tuple(v) if v is not None else None


_ST_DTYPES = {"F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
              "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
              "BOOL": torch.bool, "F8_E4M3": torch.float8_e4m3fn}


class SafetensorsFile(_Mapped):
    """Header of a safetensors file plus zero-copy access to each tensor."""

    def __init__(self, path):
        super().__init__(path)
        try:
            self._parse()
        except Exception:
            self.close()
            raise

    def _parse(self):
        if len(self.mm) < 8:
            raise ValueError(f"{self.path}: not a safetensors file")
        (hlen,) = struct.unpack("<Q", self.mm[:8])
        if 8 + hlen > len(self.mm):
            raise ValueError(f"{self.path}: header runs past the end of the file")
        header = json.loads(bytes(self.mm[8:8 + hlen]).decode("utf-8"))
        self.metadata = header.pop("__metadata__", {}) or {}
        for name, d in header.items():
            b0, b1 = d["data_offsets"]
            if b1 < b0 or 8 + hlen + b1 > len(self.mm):
                raise ValueError(f"{self.path}: tensor {name} has bad offsets")
            self.tensors[name] = TensorInfo(name, tuple(d["shape"]), -1, d["dtype"], 8 + hlen + b0, b1 - b0)

    def tensor(self, name) -> torch.Tensor:
        """The tensor as a CPU torch tensor over the mapping (no copy; valid while the file is
        open)."""
        t = self.tensors[name]
        dt = _ST_DTYPES.get(t.dtype)
        if dt is None:
            raise ValueError(f"{name}: dtype {t.dtype} is not supported")
        return self.raw(name).view(dt).reshape(t.shape)


class GGUFLinear:
    """One GGUF linear resident on the GPU: the raw blocks (kept, as the kitchen op takes them)
    and the cached repacked stages."""

    def __init__(self, raw, qtype, shape):
        from . import repack_gguf
        self.raw, self.qtype, self.shape = raw, int(qtype), tuple(shape)
        repack_gguf(raw, self.qtype, self.shape)

    def __call__(self, x, bias=None, out_dtype=None, **lora):
        from . import gguf_linear
        return gguf_linear(x, self.raw, self.qtype, self.shape, bias=bias, out_dtype=out_dtype, **lora)


def load_gguf_linears(path, device, names=None):
    """Every 2-D tensor of a GGUF type the GEMM supports (whole blocks per row), copied from the
    mapped file to `device` and repacked once.  Returns {name: GGUFLinear}; other tensors (norms,
    F16 / F32 matrices, rows straddling blocks) are left to the caller's stock path."""
    from . import GGUF_TYPES
    out = {}
    with GGUFFile(path) as f:
        for name, t in f.tensors.items():
            if names is not None and name not in names:
                continue
            if t.qtype not in GGUF_TYPES or len(t.shape) != 2 or t.nbytes <= 0:
                continue
            n, k = t.shape
            if f.orig_shape(name) not in (None, (n, k)):
                continue
            raw = f.raw(name).to(device, copy=True).reshape(n, -1)
            out[name] = GGUFLinear(raw, t.qtype, (n, k))
    return out


class Int8Linear:
    """One INT8 (ConvRot) linear resident on the GPU: int8 weight [N, K] and its per-channel scale."""

    def __init__(self, qdata, scale):
        self.qdata, self.scale = qdata, scale

    def __call__(self, x, bias=None, out_dtype=None, convrot=False, convrot_groupsize=256, **lora):
        from . import int8_linear
        return int8_linear(x, self.qdata, self.scale, bias, out_dtype, convrot, convrot_groupsize, **lora)


def load_int8_linears(path, device, names=None):
    """Every `<layer>.weight` int8 matrix with a `<layer>.weight_scale` beside it (the kitchen's
    TensorWiseINT8Layout as saved in the reference's INT8 checkpoints, `bench/bench_int8_backward.py:43-45`),
    copied from the mapped file to `device`.  Returns {layer: Int8Linear}."""
    out = {}
    with SafetensorsFile(path) as f:
        for name, t in f.tensors.items():
            if not name.endswith(".weight") or t.dtype != "I8" or len(t.shape) != 2:
                continue
            layer = name[: -len(".weight")]
            if names is not None and layer not in names:
                continue
            sname = f"{layer}.weight_scale"
            if sname not in f.tensors:
                continue
            q = f.tensor(name).to(device, copy=True)
            s = f.tensor(sname).to(device, copy=True).reshape(-1)
            out[layer] = Int8Linear(q, s)
    return out
