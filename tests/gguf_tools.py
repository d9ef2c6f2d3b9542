"""Minimal GGUF reader/writer for tests: parses files the way gguf.rs:193-311 does and writes
them the way scripts/quantize.py:119-199 does, so malformed variants can be built."""
from __future__ import annotations

import struct
from typing import Dict, List, Tuple

import numpy as np


def read_gguf(buf: bytes) -> Tuple[int, Dict[str, dict], int]:
    pos = 0

    def rd(fmt):
        nonlocal pos
        v = struct.unpack_from("<" + fmt, buf, pos)
        pos += struct.calcsize("<" + fmt)
        return v[0]

    def rdstr():
        nonlocal pos
        n = rd("Q")
        s = buf[pos:pos + n].decode("utf-8")
        pos += n
        return s

    fixed = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}

    def skip(t):
        nonlocal pos
        if t == 8:
            rdstr()
        elif t == 9:
            et, cnt = rd("I"), rd("Q")
            for _ in range(cnt):
                skip(et)
        else:
            pos += fixed[t]

    assert rd("I") == 0x46554747
    version = rd("I")
    nt, nm = rd("Q"), rd("Q")
    for _ in range(nm):
        rdstr()
        skip(rd("I"))
    tensors = {}
    order = []
    for _ in range(nt):
        name = rdstr()
        nd = rd("I")
        dims = [rd("Q") for _ in range(nd)]
        dtype = rd("I")
        off = rd("Q")
        tensors[name] = dict(dims=dims, dtype=dtype, offset=off, order=len(order))
        order.append(name)
    data_off = (pos + 31) // 32 * 32
    return version, tensors, data_off


def tensor_bytes(dtype: int, numel: int) -> int:
    return {0: numel * 4, 1: numel * 2, 30: numel * 2, 2: numel // 32 * 18}[dtype]


def write_gguf(tensors: List[Tuple[str, Tuple[int, ...], int, bytes]], metadata: Dict[str, object] | None = None,
               version: int = 3, magic: int = 0x46554747) -> bytes:
    """tensors: (name, shape in PyTorch order, ggml dtype, data bytes)."""
    out = bytearray()
    out += struct.pack("<II", magic, version)
    out += struct.pack("<Q", len(tensors))
    metadata = metadata or {}
    out += struct.pack("<Q", len(metadata))
    for k, v in metadata.items():
        kb = k.encode()
        out += struct.pack("<Q", len(kb)) + kb
        if isinstance(v, str):
            vb = v.encode()
            out += struct.pack("<I", 8) + struct.pack("<Q", len(vb)) + vb
        elif isinstance(v, tuple) and v[0] == "raw":   # (raw, type, payload bytes)
            out += struct.pack("<I", v[1]) + v[2]
        elif isinstance(v, int):
            out += struct.pack("<II", 4, v)
        else:
            out += struct.pack("<If", 6, v)
    off = 0
    for name, shape, dtype, data in tensors:
        nb = name.encode()
        out += struct.pack("<Q", len(nb)) + nb
        out += struct.pack("<I", len(shape))
        for d in reversed(shape):
            out += struct.pack("<Q", d)
        out += struct.pack("<IQ", dtype, off)
        off += len(data)
    out += b"\x00" * ((32 - len(out) % 32) % 32)
    for _, _, _, data in tensors:
        out += data
    return bytes(out)


def split_tensors(buf: bytes):
    """(name, shape, dtype, bytes) for every tensor of a GGUF buffer, in file order."""
    _, ts, data_off = read_gguf(buf)
    res = []
    for name, t in sorted(ts.items(), key=lambda kv: kv[1]["order"]):
        numel = int(np.prod(t["dims"])) if t["dims"] else 1
        n = tensor_bytes(t["dtype"], numel)
        res.append((name, tuple(reversed(t["dims"])), t["dtype"], bytes(buf[data_off + t["offset"]:data_off + t["offset"] + n])))
    return res
