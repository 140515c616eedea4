"""Minimal GGUF v3 reader/writer used for synthetic NomicBERT-MoE model files.

The container format follows the published GGUF v3 layout that the reference
loads through ``gguf_init_from_file`` (src/crispembed.cpp:365-373) and writes
through gguf-py in models/convert-bert-to-gguf.py:

    header   : magic "GGUF", u32 version (3), u64 n_tensors, u64 n_kv
    kv pairs : gguf-string key, u32 value type, value
    infos    : gguf-string name, u32 n_dims, u64 ne[n_dims] (ne0 fastest),
               u32 ggml type, u64 offset (relative to the data section)
    data     : tensors, each aligned to ``general.alignment`` (default 32)

Quantized rows are stored as ggml blocks (Q8_0: 34 B per 32 values,
Q4_K: 144 B per 256 values), see ``crispembed_b200.quant``.
"""
from __future__ import annotations

import io
import struct
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Tuple, Union

import numpy as np

GGUF_MAGIC = b"GGUF"
GGUF_VERSION = 3
DEFAULT_ALIGNMENT = 32

# gguf value types
T_UINT8, T_INT8, T_UINT16, T_INT16, T_UINT32, T_INT32, T_FLOAT32, T_BOOL, T_STRING, T_ARRAY, T_UINT64, T_INT64, T_FLOAT64 = range(13)

# ggml tensor types the library reads (ggml's numbering)
GGML_F32 = 0
GGML_F16 = 1
GGML_Q4_0 = 2
GGML_Q4_1 = 3
GGML_Q5_0 = 6
GGML_Q5_1 = 7
GGML_Q8_0 = 8
GGML_Q4_K = 12
GGML_Q5_K = 13
GGML_Q6_K = 14
GGML_IQ4_NL = 20
GGML_IQ4_XS = 23
GGML_BF16 = 30

# (block elements, block bytes)
BLOCK_INFO = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_Q4_0: (32, 18), GGML_Q4_1: (32, 20), GGML_Q5_0: (32, 22),
              GGML_Q5_1: (32, 24), GGML_Q8_0: (32, 34), GGML_Q4_K: (256, 144), GGML_Q5_K: (256, 176),
              GGML_Q6_K: (256, 210), GGML_IQ4_NL: (32, 18), GGML_IQ4_XS: (256, 136), GGML_BF16: (1, 2)}
TYPE_NAMES = {GGML_F32: "F32", GGML_F16: "F16", GGML_Q4_0: "Q4_0", GGML_Q4_1: "Q4_1", GGML_Q5_0: "Q5_0",
              GGML_Q5_1: "Q5_1", GGML_Q8_0: "Q8_0", GGML_Q4_K: "Q4_K", GGML_Q5_K: "Q5_K", GGML_Q6_K: "Q6_K",
              GGML_IQ4_NL: "IQ4_NL", GGML_IQ4_XS: "IQ4_XS", GGML_BF16: "BF16"}

_SCALAR_FMT = {
    T_UINT8: "<B", T_INT8: "<b", T_UINT16: "<H", T_INT16: "<h", T_UINT32: "<I", T_INT32: "<i",
    T_FLOAT32: "<f", T_BOOL: "<?", T_UINT64: "<Q", T_INT64: "<q", T_FLOAT64: "<d",
}


def row_bytes(ggml_type: int, ne0: int) -> int:
    be, bb = BLOCK_INFO[ggml_type]
    if ne0 % be:
        raise ValueError(f"row of {ne0} elements is not a multiple of the {TYPE_NAMES[ggml_type]} block ({be})")
    return ne0 // be * bb


def tensor_bytes(ggml_type: int, ne: Tuple[int, ...]) -> int:
    n_rows = 1
    for d in ne[1:]:
        n_rows *= d
    return row_bytes(ggml_type, ne[0]) * n_rows


@dataclass
class _PendingTensor:
    name: str
    ne: Tuple[int, ...]  # ggml order: ne0 fastest
    ggml_type: int
    nbytes: int
    produce: Callable[[], np.ndarray]  # returns the raw bytes (uint8) or a typed array


class GGUFWriter:
    """Streaming writer: tensors are produced lazily at write time so that a
    ~1 GB model never needs to sit in memory twice."""

    def __init__(self, path: str, alignment: int = DEFAULT_ALIGNMENT):
        self.path = path
        self.alignment = alignment
        self.kv: List[Tuple[str, int, object]] = []
        self.tensors: List[_PendingTensor] = []

    # ---- key/value -----------------------------------------------------
    def add_u32(self, key: str, v: int):
        self.kv.append((key, T_UINT32, int(v)))

    def add_i32(self, key: str, v: int):
        self.kv.append((key, T_INT32, int(v)))

    def add_f32(self, key: str, v: float):
        self.kv.append((key, T_FLOAT32, float(v)))

    def add_bool(self, key: str, v: bool):
        self.kv.append((key, T_BOOL, bool(v)))

    def add_str(self, key: str, v: str):
        self.kv.append((key, T_STRING, str(v)))

    def add_str_array(self, key: str, values: List[str]):
        self.kv.append((key, T_ARRAY, (T_STRING, list(values))))

    def add_f32_array(self, key: str, values):
        self.kv.append((key, T_ARRAY, (T_FLOAT32, [float(x) for x in values])))

    # ---- tensors -------------------------------------------------------
    def add_tensor(self, name: str, ne: Tuple[int, ...], ggml_type: int,
                   produce: Union[np.ndarray, Callable[[], np.ndarray]]):
        ne = tuple(int(x) for x in ne)
        nbytes = tensor_bytes(ggml_type, ne)
        if isinstance(produce, np.ndarray):
            arr = produce
            produce = lambda a=arr: a
        self.tensors.append(_PendingTensor(name, ne, ggml_type, nbytes, produce))

    # ---- serialisation -------------------------------------------------
    @staticmethod
    def _w_str(f, s: str):
        b = s.encode("utf-8")
        f.write(struct.pack("<Q", len(b)))
        f.write(b)

    def _w_value(self, f, vtype: int, v):
        if vtype == T_STRING:
            self._w_str(f, v)
        elif vtype == T_ARRAY:
            etype, items = v
            f.write(struct.pack("<IQ", etype, len(items)))
            if etype == T_STRING:
                buf = io.BytesIO()
                for s in items:
                    b = s.encode("utf-8")
                    buf.write(struct.pack("<Q", len(b)))
                    buf.write(b)
                f.write(buf.getvalue())
            else:
                f.write(np.asarray(items, dtype=np.dtype(_SCALAR_FMT[etype][1:]).newbyteorder("<")).tobytes())
        else:
            f.write(struct.pack(_SCALAR_FMT[vtype], v))

    def write(self):
        kv = list(self.kv)
        if self.alignment != DEFAULT_ALIGNMENT:
            kv.append(("general.alignment", T_UINT32, self.alignment))
        offsets = []
        off = 0
        for t in self.tensors:
            off = (off + self.alignment - 1) // self.alignment * self.alignment
            offsets.append(off)
            off += t.nbytes
        with open(self.path, "wb") as f:
            f.write(GGUF_MAGIC)
            f.write(struct.pack("<IQQ", GGUF_VERSION, len(self.tensors), len(kv)))
            for key, vtype, v in kv:
                self._w_str(f, key)
                f.write(struct.pack("<I", vtype))
                self._w_value(f, vtype, v)
            for t, o in zip(self.tensors, offsets):
                self._w_str(f, t.name)
                f.write(struct.pack("<I", len(t.ne)))
                f.write(struct.pack(f"<{len(t.ne)}Q", *t.ne))
                f.write(struct.pack("<IQ", t.ggml_type, o))
            pos = f.tell()
            pad = (-pos) % self.alignment
            f.write(b"\0" * pad)
            base = f.tell()
            for t, o in zip(self.tensors, offsets):
                cur = f.tell() - base
                if cur < o:
                    f.write(b"\0" * (o - cur))
                data = np.ascontiguousarray(t.produce())
                raw = data.view(np.uint8).reshape(-1)
                if raw.size != t.nbytes:
                    raise ValueError(f"tensor {t.name}: produced {raw.size} bytes, expected {t.nbytes}")
                f.write(raw.tobytes())


@dataclass
class GGUFTensor:
    name: str
    ne: Tuple[int, ...]
    ggml_type: int
    offset: int  # absolute file offset
    nbytes: int


@dataclass
class GGUFFile:
    path: str
    kv: Dict[str, object] = field(default_factory=dict)
    tensors: Dict[str, GGUFTensor] = field(default_factory=dict)
    _mm: Optional[np.memmap] = None

    def raw(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        if self._mm is None:
            self._mm = np.memmap(self.path, dtype=np.uint8, mode="r")
        return self._mm[t.offset:t.offset + t.nbytes]


def read_gguf(path: str) -> GGUFFile:
    """Parse header, kv pairs and tensor infos; tensor data stays on disk (memmap)."""
    out = GGUFFile(path)
    with open(path, "rb") as f:
        if f.read(4) != GGUF_MAGIC:
            raise ValueError(f"{path}: not a GGUF file")
        version, n_tensors, n_kv = struct.unpack("<IQQ", f.read(20))
        if version not in (2, 3):
            raise ValueError(f"{path}: unsupported GGUF version {version}")

        def r_str():
            (n,) = struct.unpack("<Q", f.read(8))
            return f.read(n).decode("utf-8", errors="replace")

        def r_val(vtype):
            if vtype == T_STRING:
                return r_str()
            if vtype == T_ARRAY:
                etype, n = struct.unpack("<IQ", f.read(12))
                if etype == T_STRING:
                    return [r_str() for _ in range(n)]
                dt = np.dtype(_SCALAR_FMT[etype][1:]).newbyteorder("<")
                return np.frombuffer(f.read(n * dt.itemsize), dtype=dt).tolist()
            fmt = _SCALAR_FMT[vtype]
            (v,) = struct.unpack(fmt, f.read(struct.calcsize(fmt)))
            return v

        for _ in range(n_kv):
            key = r_str()
            (vtype,) = struct.unpack("<I", f.read(4))
            out.kv[key] = r_val(vtype)
        infos = []
        for _ in range(n_tensors):
            name = r_str()
            (nd,) = struct.unpack("<I", f.read(4))
            ne = struct.unpack(f"<{nd}Q", f.read(8 * nd))
            gtype, off = struct.unpack("<IQ", f.read(12))
            infos.append((name, tuple(ne), gtype, off))
        align = int(out.kv.get("general.alignment", DEFAULT_ALIGNMENT))
        pos = f.tell()
        base = (pos + align - 1) // align * align
        for name, ne, gtype, off in infos:
            out.tensors[name] = GGUFTensor(name, ne, gtype, base + off, tensor_bytes(gtype, ne))
    return out
