"""Seeded synthetic packed weights and activations for the benchmark configs.

The reference measures only a real 96 GB checkpoint that is not available
here, so every input is synthetic with the configs' shapes and value
distributions: packed blocks are uniform random bytes except the binary16
scale fields d (and dmin for K-quants), which are drawn from U(lo, hi) and
rounded to binary16, so every scale is finite; activations are N(0, 1); the
F32 router is N(0, 0.02).

Two generators give the same distributions: numpy (host; parity tests, the
CPU baseline) and torch on the device (the benchmark's multi-GB tables).
Also holds planar_np, a numpy restatement of the planar layout that the CPU
tests use to pin the device repack kernel.
"""

from __future__ import annotations

import numpy as np

TYPE_F32, TYPE_Q4_K, TYPE_Q5_K, TYPE_IQ3_S, TYPE_IQ2_S = 0, 12, 13, 21, 22
BLOCK_BYTES = {TYPE_Q4_K: 144, TYPE_Q5_K: 176, TYPE_IQ2_S: 82, TYPE_IQ3_S: 110}
SCALE_FIELDS = {TYPE_Q4_K: 2, TYPE_Q5_K: 2, TYPE_IQ2_S: 1, TYPE_IQ3_S: 1}
# d ranges of the configs: K-quants U(0.001, 0.02), IQ U(0.001, 0.01)
D_RANGE = {TYPE_Q4_K: (0.001, 0.02), TYPE_Q5_K: (0.001, 0.02), TYPE_IQ2_S: (0.001, 0.01), TYPE_IQ3_S: (0.001, 0.01)}


def matrix_bytes(ty: int, in_w: int, out_w: int) -> int:
    return in_w // 256 * BLOCK_BYTES[ty] * out_w


def packed_np(rng: np.random.Generator, ty: int, in_w: int, out_w: int, d_range=None) -> np.ndarray:
    """GGUF-layout packed matrix [in_w, out_w] as uint8 (host)."""
    lo, hi = d_range or D_RANGE[ty]
    bb = BLOCK_BYTES[ty]
    nblk = in_w // 256 * out_w
    w = rng.integers(0, 256, size=(nblk, bb), dtype=np.uint8)
    for f in range(SCALE_FIELDS[ty]):
        d = rng.uniform(lo, hi, size=nblk).astype(np.float16)
        w[:, 2 * f : 2 * f + 2] = d.view(np.uint8).reshape(nblk, 2)
    return w.reshape(-1)


def packed_torch(gen, ty: int, in_w: int, out_w: int, device, d_range=None):
    """Same distribution, generated on the device with a seeded torch.Generator."""
    import torch

    lo, hi = d_range or D_RANGE[ty]
    bb = BLOCK_BYTES[ty]
    nblk = in_w // 256 * out_w
    w = torch.randint(0, 256, (nblk, bb), dtype=torch.uint8, device=device, generator=gen)
    for f in range(SCALE_FIELDS[ty]):
        d = torch.empty(nblk, dtype=torch.float32, device=device).uniform_(lo, hi, generator=gen).to(torch.float16)
        w[:, 2 * f : 2 * f + 2] = d.view(torch.uint8).view(nblk, 2)
    return w.view(-1)


# ---------------------------------------------------------------- planar

_FIELDS = {  # (GGUF offset, bytes per block, permutation) in plane order
    # permutation: False none, True lane-major, "qh" / "sgn" bit-transposed words
    TYPE_IQ2_S: [(2, 32, False), (34, 32, "sgn"), (66, 8, "qh"), (74, 8, False), (0, 2, False)],
    TYPE_IQ3_S: [(2, 64, False), (74, 32, "sgn"), (66, 8, "qh"), (106, 4, False), (0, 2, False)],
    TYPE_Q4_K: [(16, 128, True), (4, 12, False), (0, 4, False)],
    TYPE_Q5_K: [(48, 128, True), (16, 32, True), (4, 12, False), (0, 4, False)],
}


def _lane_major(field: np.ndarray) -> np.ndarray:
    # per 32-byte group: new[4k+i] = old[k+8i]
    n = field.shape[0]
    g = field.reshape(n, -1, 4, 8)  # [blk, group, i, k] with old index k + 8i
    return g.transpose(0, 1, 3, 2).reshape(n, -1)  # [blk, group, k, i] -> index 4k + i


def _lane_major_inv(field: np.ndarray) -> np.ndarray:
    n = field.shape[0]
    g = field.reshape(n, -1, 8, 4)  # [blk, group, k, i]
    return g.transpose(0, 1, 3, 2).reshape(n, -1)


def qh_transpose(w: np.ndarray) -> np.ndarray:
    """Transpose of the 4x4 matrix of 2-bit cells of each uint32 (cell (r, c)
    at bit 8r + 2c); its own inverse."""
    w = w.astype(np.uint32)
    t = ((w >> np.uint32(12)) ^ w) & np.uint32(0x0000F0F0)
    w = w ^ t ^ (t << np.uint32(12))
    t = ((w >> np.uint32(6)) ^ w) & np.uint32(0x00CC00CC)
    return w ^ t ^ (t << np.uint32(6))


def _qh_words(field: np.ndarray) -> np.ndarray:
    words = np.ascontiguousarray(field).view("<u4")
    return qh_transpose(words).astype("<u4").view(np.uint8).reshape(field.shape)


def _delta_swap(w: np.ndarray, mask: int, d: int) -> np.ndarray:
    t = ((w >> np.uint32(d)) ^ w) & np.uint32(mask)
    return w ^ t ^ (t << np.uint32(d))


_SIGN_SWAPS = [(0x22222222, 1), (0x0C0C0C0C, 2), (0x00AA00AA, 7), (0x0000CCCC, 14)]


def sign_transpose(w: np.ndarray, inverse: bool = False) -> np.ndarray:
    """Sign words of the planar IQ layout: bit 8l + i (subgroup l, lane i) ->
    bit 4i + l, by four delta swaps (the inverse applies them in reverse)."""
    w = np.asarray(w, dtype=np.uint32)
    for mask, d in (reversed(_SIGN_SWAPS) if inverse else _SIGN_SWAPS):
        w = _delta_swap(w, mask, d)
    return w


def _sign_words(field: np.ndarray, inverse: bool) -> np.ndarray:
    words = np.ascontiguousarray(field).view("<u4")
    return sign_transpose(words, inverse).astype("<u4").view(np.uint8).reshape(field.shape)


def _permute(field: np.ndarray, how, inverse: bool) -> np.ndarray:
    if how == "qh":
        return _qh_words(field)
    if how == "sgn":
        return _sign_words(field, inverse)
    if how:
        return _lane_major_inv(field) if inverse else _lane_major(field)
    return field


def planar_row_bytes(ty: int, in_w: int) -> int:
    """Row stride of the planar layout: GGUF row bytes rounded up to 16."""
    return (in_w // 256 * BLOCK_BYTES[ty] + 15) // 16 * 16


def planar_bytes(ty: int, in_w: int, out_w: int) -> int:
    return planar_row_bytes(ty, in_w) * out_w


def planar_np(ty: int, gguf: np.ndarray, in_w: int) -> np.ndarray:
    """GGUF bytes -> planar bytes (the layout of lbk_repack): per row, one
    plane per field over the row's blocks, rows padded with zeros to 16 bytes."""
    bb = BLOCK_BYTES[ty]
    nb = in_w // 256
    blocks = gguf.reshape(-1, nb, bb)
    rows = blocks.shape[0]
    out = np.zeros((rows, planar_row_bytes(ty, in_w)), dtype=np.uint8)
    pos = 0
    for off, nbytes, lm in _FIELDS[ty]:
        f = blocks[:, :, off : off + nbytes].reshape(rows * nb, nbytes)
        out[:, pos : pos + nb * nbytes] = _permute(f, lm, False).reshape(rows, nb * nbytes)
        pos += nb * nbytes
    return out.reshape(-1)


def gguf_from_planar_np(ty: int, planar: np.ndarray, in_w: int) -> np.ndarray:
    bb = BLOCK_BYTES[ty]
    nb = in_w // 256
    rs = planar_row_bytes(ty, in_w)
    rows = planar.size // rs
    p = planar.reshape(rows, rs)
    out = np.zeros((rows, nb, bb), dtype=np.uint8)
    pos = 0
    for off, nbytes, lm in _FIELDS[ty]:
        f = np.ascontiguousarray(p[:, pos : pos + nb * nbytes]).reshape(rows * nb, nbytes)
        out[:, :, off : off + nbytes] = _permute(f, lm, True).reshape(rows, nb, nbytes)
        pos += nb * nbytes
    return out.reshape(-1)
