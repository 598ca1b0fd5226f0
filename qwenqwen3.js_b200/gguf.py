"""GGUF v3 reader and writer.

``GGUFReader`` mirrors the reference loader's public API (gguf.js:1-375): the same method
names (``getKeyValue``, ``getTensorMetaByName``, ``getArch`` ...), the same meta object
``{buffer, offset, nbytes, shape, type}`` with ``nbytes`` padded to 256 bytes
(gguf.js:78-79) and the data section aligned to ``general.alignment`` (default 32,
gguf.js:85-87).  It hands raw tensor bytes to the CUDA backend unchanged, as gguf.js hands
``new Uint8Array(meta.buffer, meta.offset, meta.nbytes)`` to the WebGPU upload.

``GGUFWriter`` writes the files the synthetic-model generator produces.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

# KV value types (gguf.js:18-22)
KV_TYPES = dict(UINT8=0, INT8=1, UINT16=2, INT16=3, UINT32=4, INT32=5, FLOAT32=6, BOOL=7, STRING=8, ARRAY=9,
                UINT64=10, INT64=11, FLOAT64=12)
_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}

# tensor types (gguf.js:25-34)
TYPE_F32 = 0
TYPE_F16 = 1
TYPE_Q8_0 = 8
TYPE_Q2_K, TYPE_Q3_K, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K = 10, 11, 12, 13, 14

# (values per block, bytes per block), as _tensorNbytes (gguf.js:302-341) sizes them over all
# elements.  The 32-value legacy types take the ggml block sizes: gguf.js gives Q4_0/Q4_1/Q5_0/
# Q5_1 32 quant bytes per block (34/36/42/44) where a block holds 16 (18/20/22/24); no matmul of
# the reference reads those types.
_BLOCKS = {TYPE_F32: (1, 4), TYPE_F16: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24),
           TYPE_Q8_0: (32, 34), 9: (32, 36), TYPE_Q2_K: (256, 84), TYPE_Q3_K: (256, 110), TYPE_Q4_K: (256, 144),
           TYPE_Q5_K: (256, 176), TYPE_Q6_K: (256, 210)}


def tensor_nbytes(shape, ggml_type: int) -> int:
    """Exact byte size of a tensor of this shape and ggml type.  An unknown type is an error (the
    JS assumes F32 with a warning, which misplaces every later tensor's bytes)."""
    n = int(np.prod([int(s) for s in shape], dtype=np.int64))
    if ggml_type not in _BLOCKS:
        raise ValueError(f"unsupported tensor type {ggml_type}")
    per, size = _BLOCKS[ggml_type]
    return -(-n // per) * size


@dataclass
class TensorMeta:
    """The meta object of gguf.js:235-254."""

    buffer: np.ndarray  # uint8 view of the whole file (or of this tensor's slice)
    offset: int
    nbytes: int  # padded to 256 as the reference does
    shape: list
    type: int
    name: str = ""

    @property
    def exact_nbytes(self) -> int:
        return tensor_nbytes(self.shape, self.type)

    def raw(self) -> np.ndarray:
        """The tensor's exact bytes (no padding), as a uint8 view."""
        return self.buffer[self.offset: self.offset + self.exact_nbytes]


class GGUFReader:
    SIGNATURE = b"GGUF"
    VERSION = 3
    KV_TYPES = KV_TYPES

    def __init__(self, buffer):
        if isinstance(buffer, (bytes, bytearray, memoryview)):
            buffer = np.frombuffer(buffer, dtype=np.uint8)
        self.buffer = buffer
        self._mv = memoryview(buffer)
        self._kvs: list[tuple[str, int, int]] = []
        self._tensors: list[dict] = []
        self._parse_header()

    @classmethod
    def fromFile(cls, path) -> "GGUFReader":
        return cls(np.memmap(Path(path), dtype=np.uint8, mode="r"))

    # --- header (gguf.js:37-94)
    def _u32(self, off):
        return struct.unpack_from("<I", self._mv, off)[0]

    def _u64(self, off):
        return struct.unpack_from("<Q", self._mv, off)[0]

    def _str(self, off, n):
        return bytes(self._mv[off: off + n]).decode("utf-8")

    def _parse_header(self):
        sig = bytes(self._mv[0:4])
        if sig != self.SIGNATURE:
            raise ValueError(f"Invalid signature: {sig!r}")
        self.version = self._u32(4)
        self._tensorCount = self._u64(8)
        self._kvCount = self._u64(16)
        off = 24
        for _ in range(self._kvCount):
            klen = self._u64(off)
            key = self._str(off + 8, klen)
            t = self._u32(off + 8 + klen)
            voff = off + 8 + klen + 4
            self._kvs.append((key, t, voff))
            off = self._skip(t, voff)
        for _ in range(self._tensorCount):
            nlen = self._u64(off)
            off += 8
            name = self._str(off, nlen)
            off += nlen
            nd = self._u32(off)
            off += 4
            shape = [self._u64(off + 8 * i) for i in range(nd)]
            off += 8 * nd
            t = self._u32(off)
            off += 4
            rel = self._u64(off)
            off += 8
            nbytes = tensor_nbytes(shape, t)
            self._tensors.append(dict(name=name, shape=shape, type=t, rel=rel, nbytes=-(-nbytes // 256) * 256))
        align = int(self.getKeyValue("general.alignment", 0) or 32)
        start = off + (align - off % align) % align
        for t in self._tensors:
            t["dataOffset"] = start + t.pop("rel")

    def _skip(self, t, off):
        if t in _SCALAR:
            return off + struct.calcsize(_SCALAR[t])
        if t == KV_TYPES["STRING"]:
            return off + 8 + self._u64(off)
        if t == KV_TYPES["ARRAY"]:
            at = self._u32(off)
            n = self._u64(off + 4)
            o = off + 12
            if at in _SCALAR:
                return o + n * struct.calcsize(_SCALAR[at])
            for _ in range(n):
                o = self._skip(at, o)
            return o
        raise ValueError(f"Unknown KV type: {t}")

    def _read(self, t, off):
        if t in _SCALAR:
            return struct.unpack_from(_SCALAR[t], self._mv, off)[0]
        if t == KV_TYPES["STRING"]:
            return self._str(off + 8, self._u64(off))
        if t == KV_TYPES["ARRAY"]:
            at = self._u32(off)
            n = self._u64(off + 4)
            o = off + 12
            if at in _SCALAR:
                return list(np.frombuffer(self._mv[o: o + n * struct.calcsize(_SCALAR[at])], dtype=_SCALAR[at]).tolist())
            out = []
            for _ in range(n):
                out.append(self._read(at, o))
                o = self._skip(at, o)
            return out
        raise ValueError(f"Unsupported KV type: {t}")

    # --- public API (gguf.js:157-291)
    def getHeader(self):
        return dict(signature="GGUF", version=self.version, tensorCount=self._tensorCount, kvCount=self._kvCount,
                    fileSize=len(self.buffer))

    def getKVCount(self):
        return self._kvCount

    def getKVKey(self, i):
        return self._kvs[i][0]

    def getKVType(self, i):
        return self._kvs[i][1]

    def getKVValue(self, i):
        _, t, off = self._kvs[i]
        return self._read(t, off)

    def findKey(self, key):
        for i, (k, _, _) in enumerate(self._kvs):
            if k == key:
                return i
        return -1

    def getKeyValue(self, key, default=None):
        i = self.findKey(key)
        return default if i < 0 else self.getKVValue(i)

    def getTensorCount(self):
        return self._tensorCount

    def getTensorName(self, i):
        return self._tensors[i]["name"]

    def getTensorShape(self, i):
        return self._tensors[i]["shape"]

    def getTensorType(self, i):
        return self._tensors[i]["type"]

    def getTensorMeta(self, i) -> TensorMeta:
        t = self._tensors[i]
        return TensorMeta(self.buffer, t["dataOffset"], t["nbytes"], list(t["shape"]), t["type"], t["name"])

    def getTensorMetaByName(self, name):
        for i, t in enumerate(self._tensors):
            if t["name"] == name:
                return self.getTensorMeta(i)
        return None

    def getArch(self):
        """gguf.js:264-291."""
        arch = self.getKeyValue("general.architecture", "unknown")
        p = arch + "."
        hkv = self.getKeyValue(p + "attention.head_count_kv")
        head_kv = max(v for v in hkv if v > 0) if isinstance(hkv, list) else (hkv if hkv is not None else None)

        def num(key, default=None):
            v = self.getKeyValue(key)
            return default if v is None else v

        rope = self.getKeyValue(p + "rope.freq_base") or self.getKeyValue(p + "rope_freq_base")
        return dict(
            architecture=arch,
            vocabSize=num(p + "vocab_size"),
            contextLength=num(p + "context_length"),
            embeddingLength=num(p + "embedding_length"),
            blockCount=num(p + "block_count"),
            feedForwardLength=num(p + "feed_forward_length"),
            headCount=num(p + "attention.head_count"),
            headCountKV=head_kv,
            layerNormRmsEps=self.getKeyValue(p + "attention.layer_norm_rms_epsilon"),
            ropeFreqBase=rope,
            expertFeedForwardLength=num(p + "expert_feed_forward_length", 0) or 0,
            leadingDenseBlockCount=num(p + "leading_dense_block_count", 0) or 0,
            expertGatingFunc=num(p + "expert_gating_func", 0) or 0,
            shortconvLCache=num(p + "shortconv.l_cache", 0) or 0,
        )


class GGUFWriter:
    """Minimal GGUF v3 writer (tensors aligned to `alignment`, general.alignment recorded)."""

    def __init__(self, alignment: int = 32):
        self.alignment = alignment
        self.kvs: list[tuple[str, int, object, int | None]] = []
        self.tensors: list[tuple[str, list, int, np.ndarray]] = []
        self.add_kv("general.alignment", KV_TYPES["UINT32"], alignment)

    def add_kv(self, key: str, vtype: int, value, array_type: int | None = None):
        self.kvs.append((key, vtype, value, array_type))

    def add_tensor(self, name: str, shape, ggml_type: int, raw: np.ndarray):
        raw = np.ascontiguousarray(raw).view(np.uint8).reshape(-1)
        if raw.nbytes != tensor_nbytes(shape, ggml_type):
            raise ValueError(f"{name}: {raw.nbytes} bytes for shape {shape} type {ggml_type}")
        self.tensors.append((name, [int(s) for s in shape], ggml_type, raw))

    @staticmethod
    def _enc_str(s: str) -> bytes:
        b = s.encode("utf-8")
        return struct.pack("<Q", len(b)) + b

    def _enc_val(self, t, v, at=None) -> bytes:
        if t in _SCALAR:
            return struct.pack(_SCALAR[t], v)
        if t == KV_TYPES["STRING"]:
            return self._enc_str(v)
        if t == KV_TYPES["ARRAY"]:
            head = struct.pack("<IQ", at, len(v))
            if at in _SCALAR:
                return head + np.asarray(v, dtype=_SCALAR[at]).tobytes()
            return head + b"".join(self._enc_val(at, x) for x in v)
        raise ValueError(t)

    def write(self, path) -> None:
        head = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(self.tensors), len(self.kvs)))
        for k, t, v, at in self.kvs:
            head += self._enc_str(k) + struct.pack("<I", t) + self._enc_val(t, v, at)
        offs, off = [], 0
        for name, shape, t, raw in self.tensors:
            offs.append(off)
            off += raw.nbytes
            off += (self.alignment - off % self.alignment) % self.alignment
        for (name, shape, t, raw), o in zip(self.tensors, offs):
            head += self._enc_str(name) + struct.pack("<I", len(shape)) + struct.pack(f"<{len(shape)}Q", *shape)
            head += struct.pack("<IQ", t, o)
        head += b"\0" * ((self.alignment - len(head) % self.alignment) % self.alignment)
        with open(path, "wb") as f:
            f.write(head)
            pos = 0
            for (name, shape, t, raw), o in zip(self.tensors, offs):
                if o > pos:
                    f.write(b"\0" * (o - pos))
                    pos = o
                f.write(raw.tobytes())
                pos += raw.nbytes
            # trailing pad so that padded 256-byte slices of the last tensor stay in the file
            f.write(b"\0" * 256)
