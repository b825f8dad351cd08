"""Seeded synthetic GGUF blocks with the value distributions of the
benchmark configurations (there are no model files on the box):

  Q8_0  32 int8 codes uniform in [-127, 127], fp16 d = |N(0, 0.02)| / 127
  Q4_0  32 nibbles uniform in [0, 15] (offset -8), fp16 d as for Q8_0
  Q4_K  6-bit sub-scales and mins uniform in [0, 63] packed as llama.cpp's
        get_scale_min_k4 reads them (TR tensor/quant.go:158-163), nibbles
        uniform, fp16 d and dmin ~ |N(0, 0.01)|
  Q6_K  6-bit codes uniform, int8 sub-scales uniform, fp16 d ~ |N(0, 0.01)|

Blocks are generated with numpy on the host (vectorised) and uploaded
verbatim; the layout is the GGUF one byte for byte.

Decoder parity models use two variants of the K-quant blocks (`centered`,
`d_band`): with mins equal to the sub-scales and dmin = 7.5 d, a Q4_K
sub-block dequantises to d*sc*(q - 7.5), zero-mean over uniform codes.  The
benchmark's uncentred blocks carry a per-sub-block offset far larger than
their spread, so a decoder's embedding rows sit near a 16-dimensional
subspace and a handful of tokens win every greedy pick; the centred blocks
keep the token stream varied.  d_band draws the block scales uniformly from
a narrow band so that no output row (a head row of a few blocks) has a norm
far above the others.
"""
from __future__ import annotations

import numpy as np

Q4_0, Q8_0, Q4_K, Q6_K = 2, 8, 12, 14
BLOCK = {Q8_0: (32, 34), Q4_0: (32, 18), Q4_K: (256, 144), Q6_K: (256, 210)}


def _f16_bytes(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float16).view(np.uint8).reshape(-1, 2)


def pack_q4k_scales(sc: np.ndarray, m: np.ndarray) -> np.ndarray:
    """[nb, 8] 6-bit scales and mins -> [nb, 12] packed bytes."""
    sc = sc.astype(np.uint8)
    m = m.astype(np.uint8)
    q = np.zeros((sc.shape[0], 12), np.uint8)
    q[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    q[:, 4:8] = (m[:, 0:4] & 63) | ((m[:, 4:8] >> 4) << 6)
    q[:, 8:12] = (sc[:, 4:8] & 0xF) | ((m[:, 4:8] & 0xF) << 4)
    return q


def blocks(wtype: int, nblocks: int, seed: int, d_std: float | None = None, centered: bool = False,
           d_band: tuple | None = None) -> np.ndarray:
    """nblocks blocks of wtype as a flat uint8 array; d_std replaces the
    standard deviation of the K-quant fp16 block scales (Q4_K d and dmin,
    Q6_K d) when given.  centered (Q4_K): mins = sub-scales and
    dmin = 7.5 d.  d_band = (lo, hi): K-quant d uniform in [lo, hi)."""
    rng = np.random.default_rng(seed)
    e, size = BLOCK[wtype]
    out = np.empty((nblocks, size), np.uint8)
    if wtype == Q8_0:
        out[:, 0:2] = _f16_bytes(np.abs(rng.normal(0, 0.02, nblocks)) / 127)
        out[:, 2:] = rng.integers(-127, 128, (nblocks, 32), dtype=np.int8).view(np.uint8)
    elif wtype == Q4_0:
        out[:, 0:2] = _f16_bytes(np.abs(rng.normal(0, 0.02, nblocks)) / 127)
        out[:, 2:] = rng.integers(0, 256, (nblocks, 16), dtype=np.uint8)
    elif wtype == Q4_K:
        ds = 0.01 if d_std is None else d_std
        out[:, 0:2] = _f16_bytes(np.abs(rng.normal(0, ds, nblocks)))
        out[:, 2:4] = _f16_bytes(np.abs(rng.normal(0, ds, nblocks)))
        out[:, 4:16] = pack_q4k_scales(rng.integers(0, 64, (nblocks, 8)), rng.integers(0, 64, (nblocks, 8)))
        out[:, 16:] = rng.integers(0, 256, (nblocks, 128), dtype=np.uint8)
        if d_band is not None:
            out[:, 0:2] = _f16_bytes(rng.uniform(d_band[0], d_band[1], nblocks))
        if centered:
            sc = rng.integers(0, 64, (nblocks, 8))
            out[:, 4:16] = pack_q4k_scales(sc, sc)
            d = out[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(-1)
            out[:, 2:4] = _f16_bytes(d * np.float32(7.5))
    elif wtype == Q6_K:
        out[:, 0:192] = rng.integers(0, 256, (nblocks, 192), dtype=np.uint8)
        out[:, 192:208] = rng.integers(-128, 128, (nblocks, 16), dtype=np.int8).view(np.uint8)
        out[:, 208:210] = _f16_bytes(np.abs(rng.normal(0, 0.01 if d_std is None else d_std, nblocks)))
        if d_band is not None:
            out[:, 208:210] = _f16_bytes(rng.uniform(d_band[0], d_band[1], nblocks))
    else:
        raise ValueError(wtype)
    return out.reshape(-1)


def weight(wtype: int, N: int, K: int, seed: int, d_std: float | None = None, centered: bool = False,
           d_band: tuple | None = None) -> np.ndarray:
    """An [N, K] weight as its block store."""
    e, _ = BLOCK[wtype]
    assert K % e == 0
    return blocks(wtype, N * K // e, seed, d_std, centered, d_band)


def activations(M: int, K: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal((M, K), dtype=np.float32)
