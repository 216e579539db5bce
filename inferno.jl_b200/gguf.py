"""GGUF v3 reader and writer (host side).

The reader mirrors the reference's src/GGUF.jl:119-165 (`read_gguf`):
metadata key/values, tensor infos (name, dims with dims[0] the fastest, GGML
type, offset relative to the aligned data section), `general.alignment`
(default 32, GGUF.jl:152-156) and a memory map of the file.  The writer emits
the same layout; it is used to produce the seeded synthetic models.
"""
import mmap
import struct

import numpy as np

GGUF_MAGIC = 0x46554747
GGUF_VERSION = 3

# value types, src/GGUF.jl:9-23
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)
_SCALAR = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f",
           T_BOOL: "<?", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}

# GGML tensor types used on the verify path (src/GGUF.jl:25-60)
GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K = 0, 1, 8, 12, 13, 14
BLOCK = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_Q8_0: (32, 34), GGML_Q4_K: (256, 144),
         GGML_Q5_K: (256, 176), GGML_Q6_K: (256, 210)}


def tensor_nbytes(ggml_type, n_elements):
    be, bb = BLOCK[ggml_type]
    if n_elements % be:
        raise ValueError(f"{n_elements} elements not a multiple of the block ({be})")
    return n_elements // be * bb


class TensorInfo:
    def __init__(self, name, dims, ggml_type, offset):
        self.name, self.dims, self.type, self.offset = name, list(dims), ggml_type, offset

    @property
    def n_elements(self):
        n = 1
        for d in self.dims:
            n *= d
        return n

    @property
    def nbytes(self):
        return tensor_nbytes(self.type, self.n_elements)


class GGUFFile:
    """read_gguf (src/GGUF.jl:119-165): metadata, tensor infos, mapped data"""

    def __init__(self, path):
        self.path = path
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        buf = self._mm
        pos = 0

        def rd(fmt):
            nonlocal pos
            v = struct.unpack_from(fmt, buf, pos)
            pos += struct.calcsize(fmt)
            return v[0]

        def rd_str():
            n = rd("<Q")
            if n > 1 << 20:
                raise ValueError("string length exceeds 1 MB")  # GGUF.jl:96-99
            nonlocal pos
            s = bytes(buf[pos:pos + n]).decode("utf-8")
            pos += n
            return s

        def rd_val(t):
            if t in _SCALAR:
                return rd(_SCALAR[t])
            if t == T_STR:
                return rd_str()
            if t == T_ARR:
                at = rd("<I")
                n = rd("<Q")
                return [rd_val(at) for _ in range(n)]
            raise ValueError(f"unknown GGUF value type {t}")

        if rd("<I") != GGUF_MAGIC:
            raise ValueError("Not a valid GGUF file")
        self.version = rd("<I")
        n_tensors = rd("<Q")
        n_kv = rd("<Q")
        self.metadata = {}
        for _ in range(n_kv):
            k = rd_str()
            t = rd("<I")
            self.metadata[k] = rd_val(t)
        self.tensors = {}
        for _ in range(n_tensors):
            name = rd_str()
            nd = rd("<I")
            dims = [rd("<Q") for _ in range(nd)]
            t = rd("<I")
            off = rd("<Q")
            self.tensors[name] = TensorInfo(name, dims, t, off)
        align = int(self.metadata.get("general.alignment", 32))
        if pos % align:
            pos += align - pos % align
        self.data_offset = pos

    def raw(self, name):
        """the tensor's bytes as a read-only numpy view of the mapped file"""
        ti = self.tensors[name]
        start = self.data_offset + ti.offset
        return np.frombuffer(self._mm, dtype=np.uint8, count=ti.nbytes, offset=start)

    def f32(self, name):
        ti = self.tensors[name]
        if ti.type != GGML_F32:
            raise TypeError(f"{name} is not F32")
        return self.raw(name).view(np.float32)

    def close(self):
        self._mm.close()
        self._f.close()


class GGUFWriter:
    def __init__(self, path, alignment=32):
        self.path, self.alignment = path, alignment
        self.kv = []
        self.tensors = []  # (name, dims, type, bytes)

    def add(self, key, value, vtype=None):
        if vtype is None:
            if isinstance(value, bool):
                vtype = T_BOOL
            elif isinstance(value, int):
                vtype = T_U32 if value >= 0 else T_I32
            elif isinstance(value, float):
                vtype = T_F32
            elif isinstance(value, str):
                vtype = T_STR
            else:
                raise TypeError(f"give vtype for {key}")
        self.kv.append((key, vtype, value))

    def add_tensor(self, name, dims, ggml_type, data):
        data = np.ascontiguousarray(data).view(np.uint8).ravel()
        n = 1
        for d in dims:
            n *= d
        if data.size != tensor_nbytes(ggml_type, n):
            raise ValueError(f"{name}: {data.size} bytes for dims {dims} type {ggml_type}")
        self.tensors.append((name, list(dims), ggml_type, data))

    @staticmethod
    def _str(s):
        b = s.encode("utf-8")
        return struct.pack("<Q", len(b)) + b

    def _val(self, t, v):
        if t in _SCALAR:
            return struct.pack(_SCALAR[t], v)
        if t == T_STR:
            return self._str(v)
        raise TypeError("arrays not needed here")

    def write(self):
        head = bytearray()
        head += struct.pack("<IIQQ", GGUF_MAGIC, GGUF_VERSION, len(self.tensors), len(self.kv) + 1)
        head += self._str("general.alignment") + struct.pack("<I", T_U32) + struct.pack("<I", self.alignment)
        for k, t, v in self.kv:
            head += self._str(k) + struct.pack("<I", t) + self._val(t, v)
        offs, off = [], 0
        for name, dims, t, data in self.tensors:
            offs.append(off)
            off += data.size
            off += (-off) % self.alignment
        for (name, dims, t, data), o in zip(self.tensors, offs):
            head += self._str(name) + struct.pack("<I", len(dims))
            head += b"".join(struct.pack("<Q", d) for d in dims)
            head += struct.pack("<IQ", t, o)
        head += b"\0" * ((-len(head)) % self.alignment)
        with open(self.path, "wb") as f:
            f.write(head)
            pos = 0
            for (name, dims, t, data), o in zip(self.tensors, offs):
                if o > pos:
                    f.write(b"\0" * (o - pos))
                    pos = o
                f.write(data.tobytes())
                pos += data.size
