"""Minimal GGUF v3 reader in Python (public GGUF spec), independent of the
C++ reader in the product library.  Used by the tests to hand tensors to the
oracle."""
import struct

import numpy as np

_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
BLOCK = {0: (1, 4), 1: (1, 2), 30: (1, 2), 2: (32, 18), 6: (32, 22), 8: (32, 34), 12: (256, 144), 13: (256, 176),
         14: (256, 210), 34: (256, 54), 35: (256, 66), 10: (256, 84), 11: (256, 110)}


class Tensor:
    def __init__(self, name, dims, qtype, data):
        self.name, self.dims, self.qtype, self.data = name, dims, qtype, data

    @property
    def nbytes(self):
        return self.data.nbytes


def parse(buf):
    buf = memoryview(np.asarray(buf, dtype=np.uint8)).cast("B")
    pos = 0

    def take(fmt):
        nonlocal pos
        v = struct.unpack_from(fmt, buf, pos)[0]
        pos += struct.calcsize(fmt)
        return v

    def string():
        nonlocal pos
        n = take("<Q")
        s = bytes(buf[pos:pos + n]).decode()
        pos += n
        return s

    def value(t):
        if t in _SCALAR:
            return take(_SCALAR[t])
        if t == 8:
            return string()
        if t == 9:
            et, n = take("<I"), take("<Q")
            return [value(et) for _ in range(n)]
        raise ValueError(f"bad GGUF value type {t}")

    assert take("<I") == 0x46554747, "bad magic"
    version = take("<I")
    assert version in (2, 3)
    n_t, n_kv = take("<Q"), take("<Q")
    kv = {}
    for _ in range(n_kv):
        k = string()
        kv[k] = value(take("<I"))
    infos = []
    for _ in range(n_t):
        name = string()
        nd = take("<I")
        dims = [take("<Q") for _ in range(nd)]
        infos.append((name, dims, take("<I"), take("<Q")))
    align = kv.get("general.alignment", 32)
    start = (pos + align - 1) // align * align
    arr = np.frombuffer(buf, dtype=np.uint8)
    tensors = {}
    for name, dims, qt, off in infos:
        e, b = BLOCK[qt]
        n = int(np.prod(dims))
        nbytes = n // e * b
        tensors[name] = Tensor(name, dims, qt, arr[start + off:start + off + nbytes])
    return kv, tensors


def _pack_value(v):
    """(type id, payload) for a Python value: int -> u32, float -> f32, str,
    bool, or ('f32[]' | 'u32[]', list)."""
    if isinstance(v, bool):
        return 7, struct.pack("<?", v)
    if isinstance(v, int):
        return 4, struct.pack("<I", v)
    if isinstance(v, float):
        return 6, struct.pack("<f", v)
    if isinstance(v, str):
        b = v.encode()
        return 8, struct.pack("<Q", len(b)) + b
    kind, items = v
    et = {"f32[]": 6, "u32[]": 4, "str[]": 8}[kind]
    body = struct.pack("<IQ", et, len(items))
    for it in items:
        body += _pack_value(it)[1] if et != 4 else struct.pack("<I", it)
    return 9, body


def write(kvs, tensors, align=32):
    """GGUF v3 bytes.  kvs: list of (key, value); tensors: list of
    (name, type, dims, payload bytes or None for zeros)."""
    out = bytearray(struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(kvs)))
    for k, v in kvs:
        kb = k.encode()
        t, payload = _pack_value(v)
        out += struct.pack("<Q", len(kb)) + kb + struct.pack("<I", t) + payload
    offs, off = [], 0
    sizes = []
    for name, qt, dims, payload in tensors:
        e, b = BLOCK[qt]
        n = int(np.prod(dims)) // e * b
        sizes.append(n)
        offs.append(off)
        off = (off + n + align - 1) // align * align
    for (name, qt, dims, payload), o in zip(tensors, offs):
        nb = name.encode()
        out += struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims))
        for d in dims:
            out += struct.pack("<Q", d)
        out += struct.pack("<IQ", qt, o)
    out += b"\0" * ((-len(out)) % align)
    base = len(out)
    out += b"\0" * off
    for (name, qt, dims, payload), o, n in zip(tensors, offs, sizes):
        if payload is not None:
            pb = bytes(payload)
            assert len(pb) == n, (name, len(pb), n)
            out[base + o:base + o + n] = pb
    return np.frombuffer(bytes(out), dtype=np.uint8)
