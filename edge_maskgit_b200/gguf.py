"""Minimal GGUF v3 reader (the format of mg-model.cpp:139-201): metadata and tensors as numpy
views of a read-only memory map, plus row slicing of Q8_0 / Q4_K / F32 weights (a row's
blocks are contiguous, so rows [a, b) of an [N][K] weight are one byte range)."""
from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np

_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<B", 10: "<Q", 11: "<q", 12: "<d"}


@dataclass
class Tensor:
    name: str
    ne: tuple          # innermost first (ggml order)
    type: int          # 0 F32, 8 Q8_0, 12 Q4_K
    data: np.ndarray   # uint8 view of the tensor bytes

    @property
    def row_bytes(self) -> int:
        K = self.ne[0]
        return {0: K * 4, 8: K // 32 * 34, 12: K // 256 * 144}[self.type]

    def rows(self, a: int, b: int) -> np.ndarray:
        """Bytes of rows [a, b) of a 2-D weight (ne = {K, N})."""
        rb = self.row_bytes
        return self.data[a * rb:b * rb]

    def f32(self) -> np.ndarray:
        if self.type != 0:
            raise TypeError(f"{self.name} is not F32")
        return self.data.view(np.float32).reshape(tuple(reversed(self.ne)))


class GGUF:
    def __init__(self, path):
        self.buf = np.memmap(path, dtype=np.uint8, mode="r")
        b = self.buf
        p = 0

        def rd(fmt):
            nonlocal p
            v = struct.unpack_from(fmt, b, p)[0]
            p += struct.calcsize(fmt)
            return v

        def rstr():
            nonlocal p
            n = rd("<Q")
            s = bytes(b[p:p + n]).decode()
            p += n
            return s

        if rd("<I") != 0x46554747 or rd("<I") != 3:
            raise ValueError("not a GGUF v3 file")
        nt, nkv = rd("<Q"), rd("<Q")
        self.meta = {}
        for _ in range(nkv):
            k, t = rstr(), rd("<I")
            if t == 8:
                self.meta[k] = rstr()
            elif t == 9:
                sub, n = rd("<I"), rd("<Q")
                vals = [rstr() if sub == 8 else rd(_SCALAR[sub]) for _ in range(n)]
                self.meta[k] = vals
            else:
                self.meta[k] = rd(_SCALAR[t])
        infos = []
        for _ in range(nt):
            name = rstr()
            nd = rd("<I")
            ne = tuple(rd("<Q") for _ in range(nd))
            typ, off = rd("<I"), rd("<Q")
            infos.append((name, ne, typ, off))
        align = int(self.meta.get("general.alignment", 32))
        base = (p + align - 1) // align * align
        self.tensors = {}
        for name, ne, typ, off in infos:
            n = int(np.prod(ne))
            nbytes = {0: n * 4, 8: n // 32 * 34, 12: n // 256 * 144}.get(typ, 0)
            self.tensors[name] = Tensor(name, ne, typ, b[base + off:base + off + nbytes])

    def __getitem__(self, name) -> Tensor:
        return self.tensors[name]

    def hp(self, key, default=None):
        return self.meta.get("maskgit." + key, default)
