"""GGUF version 3: header decoding (metadata and tensor records) and a file
builder.

The decoder restates the checks of TR's gguf.Decode
(internal/compute/gguf/gguf.go, decoder.go, types.go): the file is untrusted
input, so every count, length, alignment, offset and size is checked against
the bytes that remain before anything is allocated, and the layout of the data
section (tensors in order, aligned, back to back, inside the file) is verified
without reading the data.  Errors are GGUFError with the kind of the failure;
the TR message code each kind corresponds to is in KINDS.

The builder writes valid files (TR's gguftest.Builder, gguftest/build.go):
metadata keys in order, tensor records with offsets padded to the alignment,
the data section aligned.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

MAGIC = b"GGUF"
VERSION = 3
DEFAULT_ALIGNMENT = 32
ALIGNMENT_KEY = "general.alignment"
MAX_TENSOR_NAME = 63  # bytes (ggml's 64-byte name with its NUL)
MAX_DIMS = 4
MIN_KV = 13      # smallest key record: name length 8, type 4, value 1
MIN_TENSOR = 25  # smallest tensor record: length 8, name 1, dims 4, type 4, offset 8
INT64_MAX = (1 << 63) - 1

# the failure kinds and TR's message codes for them
KINDS = {
    "magic": "H6676", "version": "H6656", "counts": "H6657", "truncated": "H6658", "length": "H6659",
    "utf8": "H6663", "duplicate": "H6664", "alignment": "H6665", "name": "H6666", "dims": "H6667",
    "dim": "H6668", "size": "H6669", "type": "H6670", "block": "H6671", "offset": "H6672", "range": "H6673",
    "value_type": "H6660", "nested": "H6661", "bool": "H6662",
}

# tensor types: id -> (name, elements per block, bytes per block); every ggml
# type, so the layout of files holding types this library does not read can
# still be checked (the on-disk format's own table)
TYPES = {
    0: ("F32", 1, 4), 1: ("F16", 1, 2), 2: ("Q4_0", 32, 18), 3: ("Q4_1", 32, 20),
    6: ("Q5_0", 32, 22), 7: ("Q5_1", 32, 24), 8: ("Q8_0", 32, 34), 9: ("Q8_1", 32, 36),
    10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110), 12: ("Q4_K", 256, 144), 13: ("Q5_K", 256, 176),
    14: ("Q6_K", 256, 210), 15: ("Q8_K", 256, 292), 16: ("IQ2_XXS", 256, 66), 17: ("IQ2_XS", 256, 74),
    18: ("IQ3_XXS", 256, 98), 19: ("IQ1_S", 256, 50), 20: ("IQ4_NL", 32, 18), 21: ("IQ3_S", 256, 110),
    22: ("IQ2_S", 256, 82), 23: ("IQ4_XS", 256, 136), 24: ("I8", 1, 1), 25: ("I16", 1, 2),
    26: ("I32", 1, 4), 27: ("I64", 1, 8), 28: ("F64", 1, 8), 29: ("IQ1_M", 256, 56),
    30: ("BF16", 1, 2), 34: ("TQ1_0", 256, 54), 35: ("TQ2_0", 256, 66), 39: ("MXFP4", 32, 17),
    40: ("NVFP4", 64, 36), 41: ("Q1_0", 128, 18), 42: ("Q2_0", 64, 18), 43: ("F8_E4M3", 1, 1),
}
F32, F16, Q4_0, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 2, 8, 12, 14, 30

# metadata value types
U8, I8, U16, I16, U32, I32, F32V, BOOL, STRING, ARRAY, U64, I64, F64V = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32V: "<f", BOOL: "<B",
           U64: "<Q", I64: "<q", F64V: "<d"}


def _width(vt: int) -> int:
    """bytes of one value of type vt in the file (a string's length field)."""
    if vt in (U8, I8, BOOL):
        return 1
    if vt in (U16, I16):
        return 2
    if vt in (U32, I32, F32V):
        return 4
    return 8


class GGUFError(ValueError):
    def __init__(self, kind: str, detail: str):
        super().__init__(f"gguf {kind} ({KINDS.get(kind, '?')}): {detail}")
        self.kind = kind
        self.code = KINDS.get(kind)


@dataclass
class Value:
    type: int
    data: object
    elem: int | None = None  # element type of an array


@dataclass
class Tensor:
    name: str
    dims: list   # file order: dims[0] is the innermost (last) axis
    type: int
    offset: int  # from the start of the data section
    size: int = 0

    def shape(self) -> tuple:
        """TR's shape: the file's dims reversed."""
        return tuple(reversed(self.dims))


@dataclass
class File:
    keys: list = field(default_factory=list)
    values: dict = field(default_factory=dict)
    tensors: list = field(default_factory=list)
    header_end: int = 0
    data_start: int = 0
    alignment: int = DEFAULT_ALIGNMENT

    def tensor(self, name: str) -> Tensor:
        for t in self.tensors:
            if t.name == name:
                return t
        raise KeyError(name)


class _Reader:
    def __init__(self, buf, size: int):
        self.buf = memoryview(buf)
        self.size = max(0, min(int(size), len(self.buf)))
        self.off = 0

    @property
    def remaining(self) -> int:
        return self.size - self.off

    def take(self, n: int, kind: str) -> memoryview:
        if n > self.remaining:
            raise GGUFError("truncated", f"{kind} at byte {self.off}")
        b = self.buf[self.off:self.off + n]
        self.off += n
        return b

    def u32(self, kind: str) -> int:
        return struct.unpack("<I", self.take(4, kind))[0]

    def u64(self, kind: str) -> int:
        return struct.unpack("<Q", self.take(8, kind))[0]

    def length(self, count: int, width: int):
        """count items of at least width bytes must fit in what remains (no
        allocation sized by an untrusted count)."""
        if count * width > self.remaining:
            raise GGUFError("length", f"at byte {self.off}: {count} items, {self.remaining} bytes left")

    def text(self, kind: str) -> str:
        n = self.u64(kind)
        self.length(n, 1)
        start = self.off
        raw = bytes(self.take(n, kind))
        try:
            return raw.decode("utf-8")
        except UnicodeDecodeError:
            raise GGUFError("utf8", f"at byte {start}") from None

    def value(self, vt: int, in_array: bool = False):
        if vt in _SCALAR:
            v = struct.unpack(_SCALAR[vt], self.take(_width(vt), "value"))[0]
            if vt == BOOL:
                if v > 1:
                    raise GGUFError("bool", f"bool byte {v} at byte {self.off - 1}")
                return bool(v)
            return v
        if vt == STRING:
            return self.text("value")
        if vt == ARRAY:
            if in_array:
                raise GGUFError("nested", f"array inside an array at byte {self.off}")
            et = self.u32("value")
            if et > F64V:
                raise GGUFError("value_type", f"array element type {et}")
            if et == ARRAY:
                raise GGUFError("nested", f"array of arrays at byte {self.off}")
            n = self.u64("value")
            self.length(n, _width(et))
            return Value(ARRAY, [self.value(et, True) for _ in range(n)], et)
        raise GGUFError("value_type", f"type {vt}")


def _pad(n: int, a: int) -> int:
    return (n + a - 1) & ~(a - 1)


def decode(buf, size: int | None = None) -> File:
    """Decode and check the header of a GGUF file held in buf (bytes,
    bytearray, mmap or memoryview) of size bytes (default: len(buf)); the
    decoder never reads past size.  The tensor data is not read."""
    r = _Reader(buf, len(buf) if size is None else size)
    if bytes(r.take(4, "header")) != MAGIC:
        raise GGUFError("magic", "not a GGUF file")
    v = r.u32("header")
    if v != VERSION:
        order = "big-endian " if v != 0 and v & 0xFFFF == 0 else ""
        raise GGUFError("version", f"{order}version {int.from_bytes(v.to_bytes(4, 'little'), 'big') if order else v}")
    n_tensors = r.u64("header")
    n_keys = r.u64("header")
    if n_keys * MIN_KV + n_tensors * MIN_TENSOR > r.remaining:
        raise GGUFError("counts", f"{n_keys} keys and {n_tensors} tensors cannot fit in {r.remaining} bytes")
    f = File()
    for _ in range(n_keys):
        key = r.text("key")
        if key in f.values:
            raise GGUFError("duplicate", f"key {key[:64]!r}")
        vt = r.u32("value")
        if vt > F64V:
            raise GGUFError("value_type", f"type {vt} of key {key[:64]!r}")
        val = r.value(vt)
        f.keys.append(key)
        f.values[key] = val if isinstance(val, Value) else Value(vt, val)
    if ALIGNMENT_KEY in f.values:
        a = f.values[ALIGNMENT_KEY]
        if a.type != U32:
            raise GGUFError("alignment", f"{ALIGNMENT_KEY} of type {a.type}, not UINT32")
        if a.data == 0 or a.data & (a.data - 1):
            raise GGUFError("alignment", f"{a.data} is not a power of two")
        f.alignment = a.data
    seen = set()
    for _ in range(n_tensors):
        name = r.text("tensor")
        nb = len(name.encode("utf-8"))
        if nb == 0 or nb > MAX_TENSOR_NAME:
            raise GGUFError("name", f"tensor name of {nb} bytes")
        if name in seen:
            raise GGUFError("duplicate", f"tensor {name!r}")
        seen.add(name)
        nd = r.u32("tensor")
        if nd > MAX_DIMS:
            raise GGUFError("dims", f"{name}: {nd} axes")
        dims = [r.u64("tensor") for _ in range(nd)]
        for d in dims:
            if d > INT64_MAX:
                raise GGUFError("dim", f"{name}: axis of {d}")
        t = Tensor(name, dims, r.u32("tensor"), r.u64("tensor"))
        _measure(t)
        f.tensors.append(t)
    f.header_end = r.off
    _layout(f, r.size)
    return f


def _measure(t: Tensor):
    """check the type and shape; the tensor's bytes (an axis of 0 counts as 1
    in the overflow check: it holds no data but shapes the operations)."""
    if t.type not in TYPES:
        raise GGUFError("type", f"{t.name}: unknown type {t.type}")
    _, blk, bb = TYPES[t.type]
    last = t.dims[0] if t.dims else 1
    if last % blk:
        raise GGUFError("block", f"{t.name}: last axis {last} not a multiple of {blk} ({TYPES[t.type][0]})")
    count, limit = 1, 1
    for n in t.dims:
        limit *= max(n, 1)
        if limit > INT64_MAX:
            raise GGUFError("size", f"{t.name}: element count overflows")
        count *= n
    size = count // blk * bb
    if size > INT64_MAX:
        raise GGUFError("size", f"{t.name}: byte size overflows")
    t.size = size


def _layout(f: File, size: int):
    """tensors in file order, each at the running padded offset, all inside
    the file; the data section starts aligned when there are tensors."""
    f.data_start = f.header_end
    if not f.tensors:
        return
    start = _pad(f.header_end, f.alignment)
    f.data_start = start
    expected = 0
    for t in f.tensors:
        if t.offset != expected:
            raise GGUFError("offset", f"{t.name}: offset {t.offset}, expected {expected}")
        end = start + expected + t.size
        if end > size:
            raise GGUFError("range", f"{t.name}: data ends at {end}, file has {size} bytes")
        expected += _pad(t.size, f.alignment)


def tensor_bytes(buf, f: File, t: Tensor) -> memoryview:
    """the tensor's data (a view of buf; nothing is copied)."""
    s = f.data_start + t.offset
    return memoryview(buf)[s:s + t.size]


# ---------------------------------------------------------------- builder

def _enc_value(v) -> tuple:
    """(value type, bytes) of a Python value: int -> by the tag of a
    (type, value) tuple or INT32/UINT64 by range, float -> FLOAT32, bool,
    str, list (array of the first element's type)."""
    if isinstance(v, tuple):
        vt, x = v
        if vt == STRING:
            b = x.encode("utf-8")
            return STRING, struct.pack("<Q", len(b)) + b
        if vt == ARRAY:
            et, items = x
            body = b"".join(_enc_value((et, it))[1] for it in items)
            return ARRAY, struct.pack("<IQ", et, len(items)) + body
        return vt, struct.pack(_SCALAR[vt], int(x) if vt != F32V and vt != F64V else float(x))
    if isinstance(v, bool):
        return _enc_value((BOOL, int(v)))
    if isinstance(v, int):
        return _enc_value((I32, v) if -(1 << 31) <= v < (1 << 31) else (U64, v))
    if isinstance(v, float):
        return _enc_value((F32V, v))
    if isinstance(v, str):
        return _enc_value((STRING, v))
    if isinstance(v, list):
        first = _enc_value(v[0])[0] if v else U8
        return _enc_value((ARRAY, (first, [x if not isinstance(x, tuple) else x[1] for x in v])))
    raise TypeError(f"no GGUF type for {type(v)}")


class Builder:
    """A valid GGUF v3 file (TR's gguftest.Builder).  kv(key, value) adds a
    metadata key (Python value, or a (type, value) tuple for an explicit
    type); tensor(name, type, dims, data) adds a tensor with file-order dims
    (dims[0] innermost)."""

    def __init__(self, alignment: int = 0):
        self.alignment = alignment
        self.kvs = []
        self.tensors = []

    def kv(self, key: str, value) -> "Builder":
        if self.alignment and key == ALIGNMENT_KEY:
            raise ValueError("set the alignment through Builder(alignment=...)")
        self.kvs.append((key, value))
        return self

    def tensor(self, name: str, ttype: int, dims, data) -> "Builder":
        self.tensors.append((name, int(ttype), [int(d) for d in dims], bytes(data)))
        return self

    def to_bytes(self) -> bytes:
        a = self.alignment or DEFAULT_ALIGNMENT
        kvs = list(self.kvs)
        if self.alignment:
            kvs.insert(0, (ALIGNMENT_KEY, (U32, self.alignment)))
        out = bytearray(MAGIC + struct.pack("<IQQ", VERSION, len(self.tensors), len(kvs)))
        for k, v in kvs:
            kb = k.encode("utf-8")
            vt, body = _enc_value(v)
            out += struct.pack("<Q", len(kb)) + kb + struct.pack("<I", vt) + body
        off = 0
        for name, tt, dims, data in self.tensors:
            nb = name.encode("utf-8")
            out += struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims))
            out += b"".join(struct.pack("<Q", d) for d in dims)
            out += struct.pack("<IQ", tt, off)
            off += _pad(len(data), a)
        if self.tensors:
            out += bytes(_pad(len(out), a) - len(out))
        for i, (_, _, _, data) in enumerate(self.tensors):
            out += data
            if i + 1 < len(self.tensors):
                out += bytes(_pad(len(data), a) - len(data))
        return bytes(out)

    def write(self, path: str):
        with open(path, "wb") as fh:
            fh.write(self.to_bytes())
