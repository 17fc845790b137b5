"""The GGUF container subset a Kev packed backbone uses (version 3).

A reference packed artifact (crates/huncho-backend/src/qwen_quantized.rs:
91-208, written through candle's gguf_file) holds string metadata
(`general.architecture`, `huncho.quantization`, `huncho.config_json`,
`huncho.input_widths`) and tensors of type F32, Q8_0 or Q4_0. Layout (GGUF
v3): magic "GGUF", version, tensor count, metadata count; metadata as
(string key, u32 value type, value); tensor infos as (string name, u32 n_dims,
u64 dims innermost first, u32 type, u64 data offset); padding to the
alignment (`general.alignment`, default 32); tensor data, each tensor at an
aligned offset. Strings are u64 length + UTF-8 bytes.
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

MAGIC = b"GGUF"
VERSION = 3
ALIGNMENT = 32

TYPE_F32, TYPE_F16, TYPE_Q4_0, TYPE_Q8_0 = 0, 1, 2, 8
BLOCK = 32
# bytes per 32-value block: fp16 scale + payload
BLOCK_BYTES = {TYPE_Q8_0: 2 + 32, TYPE_Q4_0: 2 + 16}

# metadata value types
_VT = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
VT_STRING, VT_ARRAY, VT_UINT32 = 8, 9, 4


def tensor_nbytes(ggml_type: int, shape) -> int:
    """Bytes of a tensor of `shape` (row-major, last dim innermost)."""
    n = int(np.prod(shape)) if len(shape) else 1
    if ggml_type == TYPE_F32:
        return 4 * n
    if ggml_type == TYPE_F16:
        return 2 * n
    if ggml_type in BLOCK_BYTES:
        if shape[-1] % BLOCK:
            raise ValueError("quantized rows must be a multiple of 32 wide")
        return n // BLOCK * BLOCK_BYTES[ggml_type]
    raise ValueError(f"unsupported GGUF tensor type {ggml_type}")


def _str(b: bytes) -> bytes:
    return struct.pack("<Q", len(b)) + b


def write(path, metadata: dict, tensors: dict, alignment: int = ALIGNMENT) -> None:
    """Write `tensors` {name: (ggml_type, shape, raw bytes)} and string or u32
    `metadata` in name order."""
    head = bytearray(MAGIC + struct.pack("<IQQ", VERSION, len(tensors), len(metadata)))
    for k, v in metadata.items():
        head += _str(k.encode())
        if isinstance(v, str):
            head += struct.pack("<I", VT_STRING) + _str(v.encode())
        elif isinstance(v, int):
            head += struct.pack("<II", VT_UINT32, v)
        else:
            raise TypeError(f"metadata {k}: only strings and u32 are written")
    offset = 0
    layout = []
    for name, (t, shape, raw) in tensors.items():
        if len(raw) != tensor_nbytes(t, shape):
            raise ValueError(f"{name}: {len(raw)} bytes for shape {shape} type {t}")
        head += _str(name.encode()) + struct.pack("<I", len(shape))
        for d in reversed(shape):
            head += struct.pack("<Q", d)
        head += struct.pack("<IQ", t, offset)
        layout.append((offset, raw))
        offset += -(-len(raw) // alignment) * alignment
    head += b"\0" * (-len(head) % alignment)
    data = bytearray(offset)
    for off, raw in layout:
        data[off:off + len(raw)] = raw
    Path(path).write_bytes(bytes(head) + bytes(data))


def read(path):
    """(metadata {key: value}, tensors {name: (ggml_type, shape, raw bytes)})."""
    buf = Path(path).read_bytes()
    if buf[:4] != MAGIC:
        raise ValueError("not a GGUF file")
    version, n_t, n_kv = struct.unpack_from("<IQQ", buf, 4)
    if version not in (2, 3):
        raise ValueError(f"unsupported GGUF version {version}")
    pos = 24

    def rd(fmt):
        nonlocal pos
        v = struct.unpack_from(fmt, buf, pos)
        pos += struct.calcsize(fmt)
        return v[0] if len(v) == 1 else v

    def rstr():
        nonlocal pos
        n = rd("<Q")
        s = buf[pos:pos + n].decode()
        pos += n
        return s

    def rval(vt):
        if vt == VT_STRING:
            return rstr()
        if vt == VT_ARRAY:
            et, n = rd("<I"), rd("<Q")
            return [rval(et) for _ in range(n)]
        return rd(_VT[vt])

    meta = {}
    for _ in range(n_kv):
        k = rstr()
        meta[k] = rval(rd("<I"))
    infos = []
    for _ in range(n_t):
        name = rstr()
        nd = rd("<I")
        dims = [rd("<Q") for _ in range(nd)]
        t, off = rd("<I"), rd("<Q")
        infos.append((name, t, tuple(reversed(dims)), off))
    align = int(meta.get("general.alignment", ALIGNMENT))
    base = pos + (-pos % align)
    tensors = {}
    for name, t, shape, off in infos:
        n = tensor_nbytes(t, shape)
        tensors[name] = (t, shape, buf[base + off:base + off + n])
    return meta, tensors
