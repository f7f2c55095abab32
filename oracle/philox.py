"""Philox4x32-10 counter-based generator in numpy (test infrastructure only).

Restates the published algorithm of Salmon, Moraes, Dror and Shaw, "Parallel
random numbers: as easy as 1, 2, 3" (SC'11): ten rounds of two 32x32->64
multiplies with the round keys bumped by the golden-ratio Weyl constants.

The select-step kernels draw their in-kernel Gumbel noise from this generator,
so this module is the checker for that noise.  Counter layout (shared with
``yapd_b200/csrc/philox.cuh``):

* token noise for (request b, position l, token v) of an L-wide block:
  counter ``(v >> 2, b*L + l, off_lo, off_hi & 0x7fffffff)``, output word ``v & 3``;
* position noise for flat position ``p = b*L + l``:
  counter ``(p >> 2, 0xffffffff, off_lo, off_hi | 0x80000000)``, word ``p & 3``;
* key ``(seed_lo, seed_hi)``.

A word ``w`` maps to the uniform ``(w >> 8) * 2**-24`` in ``[0, 1)``.
"""
from __future__ import annotations

import numpy as np
import torch

M0 = np.uint64(0xD2511F53)
M1 = np.uint64(0xCD9E8D57)
W0 = np.uint32(0x9E3779B9)
W1 = np.uint32(0xBB67AE85)
MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(ctr: np.ndarray, key: tuple[int, int]) -> np.ndarray:
    """``ctr``: ``(N, 4)`` uint32 counters -> ``(N, 4)`` uint32 outputs."""
    c = [ctr[:, i].astype(np.uint64) for i in range(4)]
    k0 = np.uint64(key[0] & 0xFFFFFFFF)
    k1 = np.uint64(key[1] & 0xFFFFFFFF)
    for r in range(10):
        p0 = M0 * c[0]
        p1 = M1 * c[2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & MASK32
        hi1, lo1 = p1 >> np.uint64(32), p1 & MASK32
        c = [(hi1 ^ c[1] ^ k0) & MASK32, lo1, (hi0 ^ c[3] ^ k1) & MASK32, lo0]
        if r < 9:
            k0 = (k0 + np.uint64(W0)) & MASK32
            k1 = (k1 + np.uint64(W1)) & MASK32
    return np.stack(c, axis=1).astype(np.uint32)


def _uniform_from_words(w: np.ndarray) -> torch.Tensor:
    u = (w >> np.uint32(8)).astype(np.float32) * np.float32(2.0 ** -24)
    return torch.from_numpy(u)


def token_uniforms(seed: int, offset: int, B: int, L: int, V: int) -> torch.Tensor:
    """``(B, L, V)`` float32 uniforms for the token Gumbel noise."""
    nq = (V + 3) // 4
    pos = np.arange(B * L, dtype=np.uint32)
    q = np.arange(nq, dtype=np.uint32)
    ctr = np.empty((B * L, nq, 4), dtype=np.uint32)
    ctr[:, :, 0] = q[None, :]
    ctr[:, :, 1] = pos[:, None]
    ctr[:, :, 2] = np.uint32(offset & 0xFFFFFFFF)
    ctr[:, :, 3] = np.uint32((offset >> 32) & 0x7FFFFFFF)
    out = philox4x32_10(ctr.reshape(-1, 4), (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))
    words = out.reshape(B * L, nq * 4)[:, :V]
    return _uniform_from_words(words).reshape(B, L, V)


def position_uniforms(seed: int, offset: int, B: int, L: int) -> torch.Tensor:
    """``(B, L)`` float32 uniforms for the position Gumbel noise."""
    n = B * L
    p = np.arange(n, dtype=np.uint32)
    ctr = np.empty((n, 4), dtype=np.uint32)
    ctr[:, 0] = p >> np.uint32(2)
    ctr[:, 1] = np.uint32(0xFFFFFFFF)
    ctr[:, 2] = np.uint32(offset & 0xFFFFFFFF)
    ctr[:, 3] = np.uint32(((offset >> 32) & 0x7FFFFFFF) | 0x80000000)
    out = philox4x32_10(ctr, (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))
    words = out[np.arange(n), p & np.uint32(3)]
    return _uniform_from_words(words).reshape(B, L)


def token_uniforms_at(seed: int, offset: int, flat_pos: np.ndarray, V: int) -> torch.Tensor:
    """``(n, V)`` token uniforms of the given flat positions ``b*L + l`` (the
    same counters as ``token_uniforms``, for a subset of a large batch)."""
    nq = (V + 3) // 4
    pos = np.asarray(flat_pos, dtype=np.uint32)
    ctr = np.empty((pos.size, nq, 4), dtype=np.uint32)
    ctr[:, :, 0] = np.arange(nq, dtype=np.uint32)[None, :]
    ctr[:, :, 1] = pos[:, None]
    ctr[:, :, 2] = np.uint32(offset & 0xFFFFFFFF)
    ctr[:, :, 3] = np.uint32((offset >> 32) & 0x7FFFFFFF)
    out = philox4x32_10(ctr.reshape(-1, 4), (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))
    return _uniform_from_words(out.reshape(pos.size, nq * 4)[:, :V])


def position_uniforms_at(seed: int, offset: int, flat_pos: np.ndarray) -> torch.Tensor:
    """``(n,)`` position uniforms of the given flat positions."""
    p = np.asarray(flat_pos, dtype=np.uint32)
    ctr = np.empty((p.size, 4), dtype=np.uint32)
    ctr[:, 0] = p >> np.uint32(2)
    ctr[:, 1] = np.uint32(0xFFFFFFFF)
    ctr[:, 2] = np.uint32(offset & 0xFFFFFFFF)
    ctr[:, 3] = np.uint32(((offset >> 32) & 0x7FFFFFFF) | 0x80000000)
    out = philox4x32_10(ctr, (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))
    return _uniform_from_words(out[np.arange(p.size), p & np.uint32(3)])
