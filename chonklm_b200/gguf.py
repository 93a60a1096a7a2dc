"""GGUF v3 container: header parser and a writer for synthetic models.

The parser follows the reference's `src/lib/gguf.ts`:
  * magic / version / tensor and KV counts            (gguf.ts:59-68)
  * KV value decoding, types 0..12                     (gguf.ts:238-284)
  * tensor infos: name, dims, ggml type, offset        (gguf.ts:75-89)
  * per-type byte lengths with block-multiple checks   (gguf.ts:103-130, 155-159)
  * data offset = header end aligned to 32             (gguf.ts:99, 161-163)

The writer is the inverse and is used to build the seeded synthetic models the
tests and the benchmark load (there are no real model files on these boxes).
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

GGUF_MAGIC = 0x46554747  # "GGUF" little-endian (gguf.ts:3)


class GGML_TYPE:
    """GGML tensor type ids the reference accepts (gguf.ts:5-14)."""
    F32 = 0
    F16 = 1
    Q5_0 = 6
    Q5_1 = 7
    Q8_0 = 8
    Q4_K = 12
    Q5_K = 13
    Q6_K = 14


# (weights per block, bytes per block), gguf.ts:103-130
BLOCK_LAYOUT: Dict[int, Tuple[int, int]] = {
    GGML_TYPE.F32: (1, 4),
    GGML_TYPE.F16: (1, 2),
    GGML_TYPE.Q5_0: (32, 22),
    GGML_TYPE.Q5_1: (32, 24),
    GGML_TYPE.Q8_0: (32, 34),
    GGML_TYPE.Q4_K: (256, 144),
    GGML_TYPE.Q5_K: (256, 176),
    GGML_TYPE.Q6_K: (256, 210),
}

TYPE_NAMES = {
    GGML_TYPE.F32: "F32", GGML_TYPE.F16: "F16", GGML_TYPE.Q5_0: "Q5_0",
    GGML_TYPE.Q5_1: "Q5_1", GGML_TYPE.Q8_0: "Q8_0", GGML_TYPE.Q4_K: "Q4_K",
    GGML_TYPE.Q5_K: "Q5_K", GGML_TYPE.Q6_K: "Q6_K",
}


def ggml_type_name(t: int) -> str:
    """gguf.ts:132-153."""
    return TYPE_NAMES.get(t, f"type-{t}")


def ggml_tensor_byte_length(t: int, n_elements: int) -> int:
    """Byte length of a tensor; raises like gguf.ts:103-130 on a partial block."""
    if t not in BLOCK_LAYOUT:
        raise ValueError(f"unsupported GGML tensor type {t}")
    block, nbytes = BLOCK_LAYOUT[t]
    if n_elements % block != 0:
        raise ValueError(f"GGML tensor type {t} requires {block}-element blocks, got {n_elements}")
    return (n_elements // block) * nbytes


# --- metadata value types (gguf.ts:238-284) --------------------------------
VT_U8, VT_I8, VT_U16, VT_I16, VT_U32, VT_I32, VT_F32, VT_BOOL, VT_STR, VT_ARR, VT_U64, VT_I64, VT_F64 = range(13)
_SCALAR_FMT = {VT_U8: "<B", VT_I8: "<b", VT_U16: "<H", VT_I16: "<h", VT_U32: "<I", VT_I32: "<i",
               VT_F32: "<f", VT_U64: "<Q", VT_I64: "<q", VT_F64: "<d"}


@dataclass
class GgufValue:
    type: str
    value: Any


@dataclass
class GgufTensorInfo:
    name: str
    shape: List[int]          # ggml order: shape[0] is the contiguous (row) length
    type: int
    offset: int               # relative to data_offset
    n_elements: int
    n_bytes: int


@dataclass
class GgufFile:
    version: int
    tensor_count: int
    kv_count: int
    kv: Dict[str, GgufValue]
    tensors: List[GgufTensorInfo]
    tensor_map: Dict[str, GgufTensorInfo]
    data_offset: int


class _Reader:
    def __init__(self, buf: bytes):
        self.buf = buf
        self.off = 0

    def take(self, fmt: str):
        v = struct.unpack_from(fmt, self.buf, self.off)[0]
        self.off += struct.calcsize(fmt)
        return v

    def u64n(self) -> int:
        v = self.take("<Q")
        if v > 2 ** 53 - 1:  # gguf.ts:214-219
            raise ValueError(f"GGUF uint64 exceeds JS safe integer: {v}")
        return v

    def string(self) -> str:
        n = self.u64n()
        if self.off + n > len(self.buf):
            raise ValueError("GGUF string runs past buffer")
        s = self.buf[self.off:self.off + n].decode("utf-8", errors="replace")
        self.off += n
        return s

    def value(self, vt: int) -> GgufValue:
        if vt in _SCALAR_FMT:
            names = {VT_U8: "uint8", VT_I8: "int8", VT_U16: "uint16", VT_I16: "int16", VT_U32: "uint32",
                     VT_I32: "int32", VT_F32: "float32", VT_U64: "uint64", VT_I64: "int64", VT_F64: "float64"}
            return GgufValue(names[vt], self.take(_SCALAR_FMT[vt]))
        if vt == VT_BOOL:
            return GgufValue("bool", self.take("<B") != 0)
        if vt == VT_STR:
            return GgufValue("string", self.string())
        if vt == VT_ARR:
            item_t = self.take("<I")
            n = self.u64n()
            return GgufValue("array", [self.value(item_t) for _ in range(n)])
        raise ValueError(f"unsupported GGUF metadata value type {vt}")


def parse_gguf(buf: bytes) -> GgufFile:
    """Parse a GGUF header (gguf.ts:59-101). `buf` must hold at least the header."""
    r = _Reader(buf)
    magic = r.take("<I")
    if magic != GGUF_MAGIC:
        raise ValueError(f"invalid GGUF magic: 0x{magic:x}")
    version = r.take("<I")
    tensor_count = r.u64n()
    kv_count = r.u64n()
    kv: Dict[str, GgufValue] = {}
    for _ in range(kv_count):
        key = r.string()
        vt = r.take("<I")
        kv[key] = r.value(vt)
    tensors: List[GgufTensorInfo] = []
    tmap: Dict[str, GgufTensorInfo] = {}
    for _ in range(tensor_count):
        name = r.string()
        nd = r.take("<I")
        shape = [r.u64n() for _ in range(nd)]
        t = r.take("<I")
        off = r.u64n()
        ne = 1
        for s in shape:
            ne *= s
        info = GgufTensorInfo(name, shape, t, off, ne, ggml_tensor_byte_length(t, ne))
        tensors.append(info)
        tmap[name] = info
    data_offset = (r.off + 31) // 32 * 32
    return GgufFile(version, tensor_count, kv_count, kv, tensors, tmap, data_offset)


def fetch_gguf_header(src: "ByteSource") -> GgufFile:
    """Retry with doubling prefixes 4 MiB..64 MiB, as gguf.ts:42-57 does."""
    size = 4 * 1024 * 1024
    last: Optional[Exception] = None
    while size <= 64 * 1024 * 1024:
        n = min(size, src.total_size)
        buf = src.read(0, n)
        try:
            parsed = parse_gguf(buf)
            if parsed.data_offset <= len(buf):
                return parsed
            last = ValueError(f"GGUF header extends past {size} bytes")
        except (struct.error, ValueError) as e:
            last = e
        if n == src.total_size:
            break
        size *= 2
    raise ValueError(f"could not parse GGUF header for {src.name}: {last}")


# --- byte sources: plain file or shard directory (cache.ts:262-467) ---------
class ByteSource:
    """Logical byte range reader over a GGUF file or a shard directory.

    A path without a file extension is a shard directory holding
    `manifest.json` in the format written by the reference's
    `scripts/shard-gguf.mjs:152-164` (`{version, totalSize, shardSize,
    shardCount, shards: [{index, name, offset, size}]}`); a range read is
    stitched from the intersecting shards as in `cache.ts:422-467`.
    """

    def __init__(self, path: str):
        self.name = path
        tail = os.path.basename(path.rstrip("/"))
        self.sharded = os.path.isdir(path) or ("." not in tail)  # cache.ts:282-288
        if self.sharded:
            with open(os.path.join(path, "manifest.json"), "r") as f:
                m = json.load(f)
            if not isinstance(m.get("totalSize"), int) or not isinstance(m.get("shards"), list):
                raise ValueError(f"invalid manifest at {path}/manifest.json")
            self.manifest = m
            self.total_size = m["totalSize"]
        else:
            self.total_size = os.path.getsize(path)

    def read(self, offset: int, length: int) -> bytes:
        if offset < 0 or length < 0 or offset + length > self.total_size:
            raise ValueError(f"range out of bounds for {self.name}: offset={offset} length={length} "
                             f"totalSize={self.total_size}")
        if not self.sharded:
            with open(self.name, "rb") as f:
                f.seek(offset)
                b = f.read(length)
            if len(b) != length:
                raise ValueError(f"short read from {self.name}")
            return b
        out = bytearray(length)
        end = offset + length
        for s in self.manifest["shards"]:
            s_end = s["offset"] + s["size"]
            if s_end <= offset:
                continue
            if s["offset"] >= end:
                break
            lo = max(0, offset - s["offset"])
            hi = min(s["size"], end - s["offset"])
            with open(os.path.join(self.name, s["name"]), "rb") as f:
                f.seek(lo)
                chunk = f.read(hi - lo)
            if len(chunk) != hi - lo:
                raise ValueError(f"shard {s['name']} is shorter than its manifest entry")
            dst = s["offset"] + lo - offset
            out[dst:dst + len(chunk)] = chunk
        return bytes(out)


def shard_gguf(src_path: str, out_dir: str, shard_size: int = 24 * 1024 * 1024) -> dict:
    """Split a GGUF into byte shards + manifest.json in the reference's format
    (`scripts/shard-gguf.mjs:31` shard size, `:152-164` manifest fields)."""
    os.makedirs(out_dir, exist_ok=True)
    total = os.path.getsize(src_path)
    shards = []
    with open(src_path, "rb") as f:
        idx = 0
        off = 0
        while off < total:
            data = f.read(shard_size)
            name = f"shard-{idx:04d}.bin"
            with open(os.path.join(out_dir, name), "wb") as g:
                g.write(data)
            shards.append({"index": idx, "name": name, "offset": off, "size": len(data)})
            off += len(data)
            idx += 1
    manifest = {"version": 1, "quant": os.path.basename(out_dir), "totalSize": total,
                "shardSize": shard_size, "shardCount": len(shards), "shards": shards}
    with open(os.path.join(out_dir, "manifest.json"), "w") as g:
        json.dump(manifest, g, indent=2)
        g.write("\n")
    return manifest


# --- writer ------------------------------------------------------------------
def _pack_string(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _pack_value(v: Any, vt: Optional[int] = None, item_t: Optional[int] = None) -> Tuple[int, bytes]:
    if vt is None:
        if isinstance(v, bool):
            vt = VT_BOOL
        elif isinstance(v, int):
            vt = VT_U32 if 0 <= v < 2 ** 32 else VT_I64
        elif isinstance(v, float):
            vt = VT_F32
        elif isinstance(v, str):
            vt = VT_STR
        elif isinstance(v, (list, tuple)):
            vt = VT_ARR
        else:
            raise TypeError(f"cannot encode {type(v)}")
    if vt in _SCALAR_FMT:
        return vt, struct.pack(_SCALAR_FMT[vt], v)
    if vt == VT_BOOL:
        return vt, struct.pack("<B", 1 if v else 0)
    if vt == VT_STR:
        return vt, _pack_string(v)
    if vt == VT_ARR:
        items = list(v)
        if item_t is None:
            item_t = _pack_value(items[0])[0] if items else VT_U32
        body = b"".join(_pack_value(it, item_t)[1] for it in items)
        return vt, struct.pack("<IQ", item_t, len(items)) + body
    raise ValueError(vt)


def write_gguf(path: str, kv: Dict[str, Any], tensors: List[Tuple[str, List[int], int, bytes]],
               alignment: int = 32) -> None:
    """Write a GGUF v3 file.

    kv: metadata; a value may be `(value, value_type)` to force the type, or
    `(items, VT_ARR, item_type)` for an array of a given item type.
    tensors: `(name, ggml_shape, ggml_type, payload_bytes)`; ggml_shape[0] is
    the contiguous dimension (row length), as in the GGUF spec.
    """
    head = bytearray()
    head += struct.pack("<IIQQ", GGUF_MAGIC, 3, len(tensors), len(kv))
    for key, val in kv.items():
        if isinstance(val, tuple) and len(val) == 3:
            vt, body = _pack_value(val[0], val[1], val[2])
        elif isinstance(val, tuple):
            vt, body = _pack_value(val[0], val[1])
        else:
            vt, body = _pack_value(val)
        head += _pack_string(key) + struct.pack("<I", vt) + body
    offsets = []
    off = 0
    for name, shape, t, payload in tensors:
        ne = 1
        for s in shape:
            ne *= s
        if ggml_tensor_byte_length(t, ne) != len(payload):
            raise ValueError(f"{name}: payload {len(payload)} B != expected {ggml_tensor_byte_length(t, ne)}")
        offsets.append(off)
        off += (len(payload) + alignment - 1) // alignment * alignment
    for (name, shape, t, payload), o in zip(tensors, offsets):
        head += _pack_string(name) + struct.pack("<I", len(shape))
        head += b"".join(struct.pack("<Q", s) for s in shape)
        head += struct.pack("<IQ", t, o)
    pad = (-len(head)) % alignment
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * pad)
        for (name, shape, t, payload), o in zip(tensors, offsets):
            f.write(payload)
            f.write(b"\0" * ((-len(payload)) % alignment))


def metadata_number(v: Any) -> Optional[float]:
    """gguf.ts-side `ggufMetadataNumber` (llama-wgsl-runtime.ts:496-503)."""
    if isinstance(v, bool):
        return None
    if isinstance(v, (int, float)):
        return v
    if isinstance(v, GgufValue):
        return metadata_number(v.value)
    return None
