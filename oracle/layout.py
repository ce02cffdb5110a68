"""CPU restatement of this build's kernel weight layout (numpy, integer only).

Test infrastructure (see ``oracle/__init__.py``). The layout is this build's
own design (documented in mtp_b200/csrc/gptq.cu); this module states it a
second time, independently of the CUDA repack, so the GPU repack can be
checked bit-exactly and so a CPU decode of the layout can be checked against
the reference dequantisation (repack/gptq_unpack.py:88-131).
"""
from __future__ import annotations

import numpy as np

from . import gptq


def _round256(v: int) -> int:
    return (v + 255) // 256 * 256


def expert_layout(hidden: int, inter: int, group: int) -> dict[str, int]:
    def sizes(n, k):
        return n * k // 2, n * (k // group) * 2, n * (k // group) // 2
    a, b = sizes(2 * inter, hidden), sizes(hidden, inter)
    off = {}
    o = 0
    for name, size in (("w13_qweight", a[0]), ("w13_scales", a[1]), ("w13_zeros", a[2]),
                       ("w2_qweight", b[0]), ("w2_scales", b[1]), ("w2_zeros", b[2])):
        off[name] = o
        o = _round256(o + size)
    off["bytes"] = o
    return off


def block_rows(n: int, gated: bool) -> np.ndarray:
    """[n/128, 128] source row of each row of each 128-row block: for a gated
    projection (w13, n = 2I) block b is gate rows 64b..64b+63 then up rows
    I+64b..I+64b+63; otherwise rows 128b..128b+127."""
    nb = n // 128
    r = np.arange(128)
    if gated:
        half = n // 2
        return np.stack([np.where(r < 64, 64 * b + r, half + 64 * b + (r - 64)) for b in range(nb)])
    return np.stack([128 * b + r for b in range(nb)])


def repack_projection(qweight: np.ndarray, qzeros: np.ndarray, scales: np.ndarray, group: int,
                      gated: bool = False):
    """GPTQ [K/8, N] / [K/G, N/8] / [K/G, N] -> (weights bytes, scales bytes, zeros bytes)."""
    q = gptq.unpack_rows(qweight)            # [K, N] values 0..15
    z = gptq.unpack_cols(qzeros)             # [K/G, N]
    s = np.ascontiguousarray(scales).view(np.uint16)  # [K/G, N]
    k, n = q.shape
    rows = block_rows(n, gated)              # [nb, 128]
    nb, chunks, groups = n // 128, k // 32, k // group
    # words[b, c, r, j]: k0 = 32c + 8j; byte t = q(k0 + t) | q(k0 + 4 + t) << 4
    qt = q.T.astype(np.uint32)               # [N, K]
    qb = qt[rows]                            # [nb, 128, K]
    qb = qb.reshape(nb, 128, chunks, 4, 2, 4)  # [.., c, j, half, t]: k = 32c + 8j + 4 half + t
    lo, hi = qb[..., 0, :], qb[..., 1, :]      # [nb, 128, c, j, t]
    shifts = (8 * np.arange(4)).astype(np.uint32)
    words = ((lo | (hi << np.uint32(4))) << shifts).sum(axis=-1).astype(np.uint32)  # [nb, 128, c, j]
    words = words.transpose(0, 2, 1, 3)      # [nb, c, 128, j]
    sc = s.T[rows].transpose(0, 2, 1)        # [nb, groups, 128]
    zt = z.T[rows].transpose(0, 2, 1).astype(np.uint8)  # [nb, groups, 128]
    zp = (zt[..., 0::2] | (zt[..., 1::2] << 4)).astype(np.uint8)  # [nb, groups, 64]
    return (np.ascontiguousarray(words).view(np.uint8).reshape(-1),
            np.ascontiguousarray(sc).view(np.uint8).reshape(-1), np.ascontiguousarray(zp).reshape(-1))


def repack_expert(t: dict, e: int | None, hidden: int, inter: int, group: int) -> np.ndarray:
    """One expert blob (uint8 [bytes]) from GPTQ tensors (numpy or torch)."""
    def get(name):
        v = t[name] if e is None else t[name][e]
        return v.numpy() if hasattr(v, "numpy") else np.asarray(v)
    L = expert_layout(hidden, inter, group)
    blob = np.zeros(L["bytes"], dtype=np.uint8)
    for p in ("w13", "w2"):
        qw, sc, zp = repack_projection(get(f"{p}_qweight"), get(f"{p}_qzeros"), get(f"{p}_scales"), group,
                                       gated=(p == "w13"))
        blob[L[f"{p}_qweight"]:L[f"{p}_qweight"] + qw.size] = qw
        blob[L[f"{p}_scales"]:L[f"{p}_scales"] + sc.size] = sc
        blob[L[f"{p}_zeros"]:L[f"{p}_zeros"] + zp.size] = zp
    return blob


def decode_projection(blob: np.ndarray, off_q: int, off_s: int, off_z: int, n: int, k: int, group: int,
                      zero_mode: str = "raw", gated: bool = False) -> np.ndarray:
    """Inverse: kernel layout -> fp32 [N, K] (Linear orientation), computed as the
    kernel's dequantisation defines it: (q - z) * s per element."""
    nb, chunks, groups = n // 128, k // 32, k // group
    words = blob[off_q:off_q + n * k // 2].view(np.uint32).reshape(nb, chunks, 128, 4)
    sc = blob[off_s:off_s + n * groups * 2].view(np.float16).reshape(nb, groups, 128).astype(np.float32)
    zp = blob[off_z:off_z + n * groups // 2].reshape(nb, groups, 64)
    zr = np.empty((nb, groups, 128), dtype=np.float32)
    zr[..., 0::2] = zp & 0xF
    zr[..., 1::2] = zp >> 4
    if zero_mode == "sym8":
        zr[:] = 8.0
    t = np.arange(4, dtype=np.uint32)
    lo = (words[..., None] >> (8 * t)) & np.uint32(0xF)           # [nb, c, 128, j, t]
    hi = (words[..., None] >> (8 * t + 4)) & np.uint32(0xF)
    q = np.stack([lo, hi], axis=-2).astype(np.float32)             # [nb, c, 128, j, half, t]
    q = q.transpose(0, 2, 1, 3, 4, 5).reshape(nb, 128, k)          # k = 32c + 8j + 4 half + t
    gidx = np.arange(k) // group
    deq = (q - zr.transpose(0, 2, 1)[:, :, gidx]) * sc.transpose(0, 2, 1)[:, :, gidx]
    out = np.zeros((n, k), dtype=np.float32)
    out[block_rows(n, gated).reshape(-1)] = deq.reshape(nb * 128, k)
    return out
