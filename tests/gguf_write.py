"""A GGUF file writer for the loader tests, written from the GGUF format
(version 3: header, metadata, tensor records, aligned tensor data), with
switches for the damaged files the reader must reject."""
import struct

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f",
        BOOL: "<B", U64: "<Q", I64: "<q", F64: "<d"}


def _str(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(t, v):
    if t == STR:
        return _str(v)
    if t == ARR:
        et, items = v
        out = struct.pack("<IQ", et, len(items))
        return out + b"".join(_value(et, x) for x in items)
    return struct.pack(_FMT[t], v)


def gguf_bytes(kv, tensors, version=3, alignment=32, magic=0x46554747, offsets=None):
    """kv: [(key, type, value)], arrays as (ARR, (elem_type, [items]));
    tensors: [(name, dims (contiguous axis first), ggml_type, raw bytes)].
    Tensor data follows the records, each tensor at a multiple of
    `alignment` (pass general.alignment in kv for a non-default one);
    `offsets` overrides the recorded data offsets."""
    head = struct.pack("<IIQQ", magic, version, len(tensors), len(kv))
    head += b"".join(_str(k) + struct.pack("<I", t) + _value(t, v) for k, t, v in kv)
    data, offs = b"", []
    for _, _, _, raw in tensors:
        data += b"\0" * (-len(data) % alignment)
        offs.append(len(data))
        data += raw
    if offsets is not None:
        offs = offsets
    for (name, dims, gt, _), off in zip(tensors, offs):
        head += _str(name) + struct.pack("<I", len(dims)) + b"".join(
            struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", gt, off)
    head += b"\0" * (-len(head) % alignment)
    return head + data


def write_gguf(path, kv, tensors, **kw):
    with open(path, "wb") as f:
        f.write(gguf_bytes(kv, tensors, **kw))
    return path
