""".fgm model files, read from Python: the mirror of the C++ loader
(host/fgm_model.hpp) and of the reference's fgm-core Model
(crates/fgm-core/src/model.rs:117-221), for the format that the reference's
convert/fgm.py writes:

    [0, 8)    magic b"FASTGEM1"
    [8, 12)   u32 little-endian header length
    [12, ..)  JSON header {"arch", "config", "meta", "tensors"}
    ...       tensor blobs, 64-byte aligned, already in the kernels' layouts

The file is memory-mapped; views are numpy arrays over the mapping.
``register_linears`` makes the quantised weights resident on the device
through the library's registry (``fgm_cuda_register``).
"""
from __future__ import annotations

import json
import struct

import numpy as np

MAGIC = b"FASTGEM1"
_DTYPES = {"f32": np.float32, "f16": np.uint16, "q8c": np.int8, "q4g": np.uint8,
           "q8r": np.int8, "q4r": np.uint8}


class FgmError(ValueError):
    """A malformed file, a missing tensor or a non-linear dtype (the
    reference panics in these cases)."""


class FgmFile:
    def __init__(self, path: str):
        self.path = path
        self._mm = np.memmap(path, dtype=np.uint8, mode="r")
        mm = self._mm
        if mm.size < 12 or bytes(mm[:8]) != MAGIC:
            raise FgmError(f"{path}: not a .fgm file")
        (hlen,) = struct.unpack("<I", bytes(mm[8:12]))
        if hlen > mm.size - 12:
            raise FgmError(f"{path}: header length past the end of the file")
        try:
            h = json.loads(bytes(mm[12:12 + hlen]))
        except (UnicodeDecodeError, json.JSONDecodeError) as e:
            raise FgmError(f"{path}: bad header: {e}") from None
        if not isinstance(h, dict) or "config" not in h or not isinstance(h.get("tensors"), dict):
            raise FgmError(f"{path}: header lacks config / tensors")
        self.config = h["config"]
        self.meta = h.get("meta", {})
        self.arch = h.get("arch")
        self.tensors = h["tensors"]
        for name, e in self.tensors.items():
            if e["offset"] < 0 or e["nbytes"] < 0 or e["offset"] + e["nbytes"] > mm.size:
                raise FgmError(f"{path}: tensor {name} lies past the end of the file")

    # ---------------------------------------------------------------- views
    def has(self, name: str) -> bool:
        return name in self.tensors

    def entry(self, name: str) -> dict:
        try:
            return self.tensors[name]
        except KeyError:
            raise FgmError(f"missing tensor {name}") from None

    def shape(self, name: str) -> list:
        return self.entry(name)["shape"]

    def raw(self, name: str) -> np.ndarray:
        e = self.entry(name)
        return self._mm[e["offset"]: e["offset"] + e["nbytes"]]

    def array(self, name: str) -> np.ndarray:
        """The tensor's bytes viewed as its dtype (f16 as raw uint16 bits)."""
        return self.raw(name).view(_DTYPES.get(self.entry(name)["dtype"], np.uint8))

    def linear(self, name: str) -> dict:
        """model.rs:169-194: blob, scales and geometry of a quantised linear."""
        e = self.entry(name)
        if e["dtype"] not in ("q4g", "q8c"):
            raise FgmError(f"tensor {name} has non-linear dtype {e['dtype']}")
        if len(e["shape"]) < 2:
            raise FgmError(f"tensor {name} is not a matrix")
        n, k = e["shape"][0], e["shape"][1]
        meta = e.get("meta") or {}
        had = int(meta.get("hadamard", 0) or 0)
        if e["dtype"] == "q4g":
            return {"bits": 4, "n": n, "k": k, "q": self.raw(name),
                    "scale": self.raw(name + ".scale").view(np.uint16),
                    "group": int(meta.get("group", 64) or 64), "hadamard": had}
        return {"bits": 8, "n": n, "k": k, "q": self.raw(name).view(np.int8),
                "scale": self.raw(name + ".scale").view(np.float32),
                "group": 0, "hadamard": had}

    def dual(self, name: str):
        """model.rs:196-208: (primary, int8 twin or None)."""
        alt = name + ".i8"
        return self.linear(name), (self.linear(alt) if self.has(alt) else None)

    def total_bytes(self) -> int:
        return sum(e["nbytes"] for e in self.tensors.values())

    # -------------------------------------------------------------- device
    def _linear_blobs(self):
        for name, e in self.tensors.items():
            if e["dtype"] in ("q4g", "q8c"):
                yield self.raw(name)
                if self.has(name + ".scale"):
                    yield self.raw(name + ".scale")

    def register_linears(self) -> int:
        """Upload every quantised weight and its scales to the device
        registry; GEMMs given these host addresses then read the device
        copies.  Returns the bytes registered."""
        from ._lib import call
        total = 0
        for b in self._linear_blobs():
            if b.size:
                call("fgm_cuda_register", b.ctypes.data, b.size)
                total += b.size
        return total

    def unregister_linears(self) -> None:
        from ._lib import call
        for b in self._linear_blobs():
            if b.size:
                call("fgm_cuda_unregister", b.ctypes.data)
