"""Training-mode dropout of the pair layer -- TEST INFRASTRUCTURE ONLY.

Only ``tests/`` may import this module, as the checker of the dropout paths of the B200
package. It restates:

* ``DropoutRowwise`` / ``DropoutColumnwise`` (reference src/genie_tk/pair_transform.py:26-61):
  one multiplier tensor ([B, 1, N, C] resp. [B, N, 1, C]: ``nn.Dropout`` applied to ones, so
  0 or 1 / (1 - p)) broadcast over the rows resp. the columns of the update;
* ``PairTransformLayer.forward`` in training mode (:162-195): each of the four triangle
  updates is multiplied by its multiplier tensor before its residual add, in the order
  tri_mul_out, tri_mul_in, tri_att_start (rowwise) and tri_att_end (columnwise);
* the keep-bit form the kernels consume (128 bits per (b, residue), bit c = channel c kept);
* Philox4x32-10, the counter-based generator of Salmon, Moraes, Dror and Shaw ("Parallel
  random numbers: as easy as 1, 2, 3", SC'11), restated from the paper in numpy uint32
  arithmetic and pinned by the paper's published known-answer vectors
  (``tests/test_dropout_cpu.py``), with the bit assignment of gtk_dropout_keep_bits_philox.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from .triangle_oracle import layer_tail, triatt_forward, trimul_forward

Params = Dict[str, torch.Tensor]

# Philox-4x32 round multipliers and Weyl key increments (SC'11, section 5).
PHILOX_M0 = np.uint64(0xD2511F53)
PHILOX_M1 = np.uint64(0xCD9E8D57)
PHILOX_W0 = np.uint32(0x9E3779B9)
PHILOX_W1 = np.uint32(0xBB67AE85)
_MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(ctr: np.ndarray, key: np.ndarray) -> np.ndarray:
    """Philox4x32 with 10 rounds. ``ctr`` uint32 [..., 4], ``key`` uint32 [..., 2] (broadcast);
    returns uint32 [..., 4]. Round: (hi0, lo0) = M0 * c0, (hi1, lo1) = M1 * c2,
    c = (hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0); the key is bumped by (W0, W1) before every
    round but the first."""
    c = [np.asarray(ctr[..., i], dtype=np.uint32).astype(np.uint64) for i in range(4)]
    k0 = np.asarray(key[..., 0], dtype=np.uint32).astype(np.uint64)
    k1 = np.asarray(key[..., 1], dtype=np.uint32).astype(np.uint64)
    for r in range(10):
        if r > 0:
            k0 = (k0 + np.uint64(PHILOX_W0)) & _MASK32
            k1 = (k1 + np.uint64(PHILOX_W1)) & _MASK32
        p0 = PHILOX_M0 * c[0]
        p1 = PHILOX_M1 * c[2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & _MASK32
        hi1, lo1 = p1 >> np.uint64(32), p1 & _MASK32
        c = [hi1 ^ c[1] ^ k0, lo1, hi0 ^ c[3] ^ k1, lo0]
    return np.stack([x.astype(np.uint32) for x in c], axis=-1)


def keep_bits_philox(seed: int, offset: int, p: float, n_vectors: int) -> np.ndarray:
    """uint32 [n_vectors, 4]: channel c of vector v is kept when word c % 4 of
    Philox(counter = (v*32 + c//4 as two 32-bit halves, offset as two halves), key = seed)
    is >= floor(p * 2^32)."""
    threshold = min(int(np.floor(p * 4294967296.0)), 0xFFFFFFFF)
    blocks = np.arange(n_vectors * 32, dtype=np.uint64)
    ctr = np.stack([blocks & _MASK32, blocks >> np.uint64(32),
                    np.full_like(blocks, offset & 0xFFFFFFFF), np.full_like(blocks, (offset >> 32) & 0xFFFFFFFF)],
                   axis=-1).astype(np.uint32)
    key = np.array([seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF], dtype=np.uint32)
    r = philox4x32_10(ctr, key)                            # [n*32, 4]: channels 4g .. 4g+3
    keep = (r.astype(np.uint64) >= np.uint64(threshold)).reshape(n_vectors, 128)
    return pack_keep(keep)


def pack_keep(keep: np.ndarray) -> np.ndarray:
    """bool [n, 128] -> uint32 [n, 4] (bit c % 32 of word c // 32)."""
    k = np.asarray(keep, dtype=np.uint64).reshape(-1, 4, 32)
    return (k << np.arange(32, dtype=np.uint64)).sum(axis=-1).astype(np.uint32)


def unpack_keep(bits: np.ndarray) -> np.ndarray:
    """uint32 [n, 4] -> bool [n, 128]."""
    b = np.asarray(bits, dtype=np.uint32).astype(np.uint64).reshape(-1, 4, 1)
    return ((b >> np.arange(32, dtype=np.uint64)) & np.uint64(1)).astype(bool).reshape(-1, 128)


def multipliers_from_bits(bits: np.ndarray, scale: float, B: int, N: int, rowwise: bool) -> torch.Tensor:
    """The multiplier tensor a keep-bit array stands for: [B, 1, N, 128 G] (rowwise) or
    [B, N, 1, 128 G] (columnwise) for G 128-bit groups per (b, residue), kept channels =
    scale, dropped = 0."""
    m = torch.from_numpy(unpack_keep(bits).astype(np.float32) * np.float32(scale)).reshape(B, N, -1)
    return m.unsqueeze(1) if rowwise else m.unsqueeze(2)


def pair_layer_forward(z: torch.Tensor, mask: torch.Tensor, lp: Dict[str, Params], no_heads: int,
                       drop_mults: Optional[Sequence[torch.Tensor]] = None, chunk_rows: int = 0) -> torch.Tensor:
    """PairTransformLayer.forward (pair_transform.py:162-195). ``drop_mults``: the four
    multiplier tensors in the reference's draw order (None: eval mode, no dropout)."""
    z = z.float().clone()
    m: List = [1.0] * 4 if drop_mults is None else [t.to(z.device).float() for t in drop_mults]
    z = z + trimul_forward(z, mask, lp["tri_mul_out"], outgoing=True) * m[0]
    z = z + trimul_forward(z, mask, lp["tri_mul_in"], outgoing=False) * m[1]
    z = z + triatt_forward(z, mask, lp["tri_att_start"], starting=True, no_heads=no_heads,
                           chunk_rows=chunk_rows) * m[2]
    z = z + triatt_forward(z, mask, lp["tri_att_end"], starting=False, no_heads=no_heads,
                           chunk_rows=chunk_rows) * m[3]
    return layer_tail(z, mask, lp["pair_transition"])
