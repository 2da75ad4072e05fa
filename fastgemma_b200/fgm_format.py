"""The ``.fgm`` weight and activation layouts the kernels consume.

Restated from the reference's format producer so that synthetic weights carry
exactly the bytes a converted model file would:

* ``pack_b_tiles`` -- W[N, K] int8 into tiles ``[N/16][K/64][k/4][n%16][k%4]``
  (convert/quant.py:96-107).  Streaming one n-block walks K contiguously.
* ``pack_nibbles`` -- 64-value blocks, value i (< 32) in the low nibble of byte
  i and value i + 32 in the high nibble, two's complement
  (convert/quant.py:76-82; sign extension ``(v ^ 8) - 8``, amx_gemm.c:84-86).
* q4g scales: f16 ``[K/group][N]`` (convert/quant.py:149-165, model.rs:182).
* q8c scales: f32 ``[N]`` (convert/quant.py:110-117).
* packed activations: ``[ceil(M/16)][K/64][16][64]`` int8 with zero padding
  rows (ops.c:279-290; ``packed_a_len``, lib.rs:155-157).

The synthetic generators follow the seeded distributions of the benchmark
configurations: int4 values uniform in [-8, 7], int8 uniform in [-127, 127],
f16 group scales ~ U(0.005, 0.02), f32 channel scales ~ U(0.001, 0.01),
activations ~ N(0, 1).
"""
from __future__ import annotations

import numpy as np

TILE_N = 16
TILE_K = 64
Q4_TILE = 512
Q8_TILE = 1024


def packed_a_len(m: int, k: int) -> int:
    """Bytes of the tile-packed copy of an ``m x k`` activation (lib.rs:155-157)."""
    return (m + 15) // 16 * 16 * k


def pack_b_tiles(q: np.ndarray) -> np.ndarray:
    """W[N, K] int8 -> flat tile order ``[nb][kb][k/4][n][k%4]``."""
    n, k = q.shape
    assert n % TILE_N == 0 and k % TILE_K == 0, (n, k)
    t = q.reshape(n // TILE_N, TILE_N, k // TILE_K, TILE_K // 4, 4)
    return np.ascontiguousarray(t.transpose(0, 2, 3, 1, 4)).reshape(-1)


def unpack_b_tiles(blob: np.ndarray, n: int, k: int) -> np.ndarray:
    """Inverse of :func:`pack_b_tiles`."""
    t = blob.reshape(n // TILE_N, k // TILE_K, TILE_K // 4, TILE_N, 4)
    return np.ascontiguousarray(t.transpose(0, 3, 1, 2, 4)).reshape(n, k)


def pack_nibbles(flat_i8: np.ndarray) -> np.ndarray:
    """Half-split nibble packing of 64-value blocks."""
    assert flat_i8.size % 64 == 0
    b = flat_i8.reshape(-1, 64).astype(np.uint8)
    return ((b[:, :32] & 0x0F) | ((b[:, 32:] & 0x0F) << 4)).astype(np.uint8).reshape(-1)


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    """Inverse of :func:`pack_nibbles`, two's-complement sign extension."""
    p = packed.reshape(-1, 32)
    lo = ((p & 0x0F).astype(np.int16) ^ 8) - 8
    hi = (((p >> 4) & 0x0F).astype(np.int16) ^ 8) - 8
    return np.concatenate([lo, hi], axis=1).astype(np.int8).reshape(-1)


def pack_q4g(q: np.ndarray) -> np.ndarray:
    """W[N, K] with values in [-8, 7] -> the q4g blob (N*K/2 bytes)."""
    return pack_nibbles(pack_b_tiles(q))


def pack_a(a: np.ndarray) -> np.ndarray:
    """Row-major int8 [M, K] -> tile-packed ``[ceil(M/16)][K/64][16][64]``."""
    m, k = a.shape
    mp = (m + 15) // 16 * 16
    pad = np.zeros((mp, k), np.int8)
    pad[:m] = a
    t = pad.reshape(mp // 16, 16, k // 64, 64).transpose(0, 2, 1, 3)
    return np.ascontiguousarray(t).reshape(-1)


def q4g_column_shard(bq: np.ndarray, scale: np.ndarray, n: int, k: int,
                     nb0: int, nb1: int):
    """Bytes of n-blocks ``[nb0, nb1)`` of a q4g weight.

    The tile order makes a column shard one contiguous byte range of the blob;
    the ``[K/group][N]`` scales need one strided slice per group row.
    """
    per_nb = (k // TILE_K) * Q4_TILE
    w = bq[nb0 * per_nb: nb1 * per_nb]
    s = np.ascontiguousarray(scale.reshape(-1, n)[:, nb0 * 16: nb1 * 16])
    return w, s


def q8c_column_shard(b: np.ndarray, scale: np.ndarray, n: int, k: int, nb0: int, nb1: int):
    """Bytes of n-blocks ``[nb0, nb1)`` of a q8c weight."""
    per_nb = (k // TILE_K) * Q8_TILE
    return b[nb0 * per_nb: nb1 * per_nb], scale[nb0 * 16: nb1 * 16]


# ------------------------------------------------------------- synthetic data
def synth_q4g(n: int, k: int, group: int, seed: int, *, structured: bool = True):
    """Seeded q4g weight: (blob uint8 [N*K/2], scales f16 [K/group, N]).

    ``structured`` draws W[N, K] and packs it through the format; otherwise the
    blob bytes are drawn directly (every nibble uniform over its 16 codes, the
    same distribution, without materialising W -- used for large benches).
    """
    assert group % 64 == 0 and k % group == 0 and n % 16 == 0
    rng = np.random.default_rng(seed)
    if structured:
        q = rng.integers(-8, 8, size=(n, k), dtype=np.int8)
        blob = pack_q4g(q)
    else:
        blob = rng.integers(0, 256, size=n * k // 2, dtype=np.uint8)
    s = rng.uniform(0.005, 0.02, size=(k // group, n)).astype(np.float16)
    return blob, s


def synth_q8c(n: int, k: int, seed: int, *, structured: bool = True):
    """Seeded q8c weight: (blob int8 [N*K], scales f32 [N])."""
    assert k % 64 == 0 and n % 16 == 0
    rng = np.random.default_rng(seed)
    q = rng.integers(-127, 128, size=(n, k) if structured else n * k, dtype=np.int8)
    blob = pack_b_tiles(q) if structured else q
    s = rng.uniform(0.001, 0.01, size=n).astype(np.float32)
    return blob, s


def synth_x(m: int, k: int, seed: int) -> np.ndarray:
    """Seeded activations X ~ N(0, 1), f32 [M, K]."""
    return np.random.default_rng(seed).standard_normal((m, k), dtype=np.float32)
