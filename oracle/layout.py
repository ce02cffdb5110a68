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


def repack_projection(qweight: np.ndarray, qzeros: np.ndarray, scales: np.ndarray, group: int):
    """GPTQ [K/8, N] / [K/G, N/8] / [K/G, N] -> (weights bytes, scales bytes, zeros bytes)."""
    q = gptq.unpack_rows(qweight)            # [K, N] values 0..15
    z = gptq.unpack_cols(qzeros)             # [K/G, N]
    s = np.ascontiguousarray(scales).view(np.uint16)  # [K/G, N]
    k, n = q.shape
    strips, chunks, groups = n // 16, k // 64, k // group
    # words[s, c, lane, kk]: row 16s + g + 8(kk & 1), k base 64c + 32(kk >> 1) + 4t;
    # byte b = q(row, kb + b) | q(row, kb + 16 + b) << 4
    lane = np.arange(32)
    g, t = lane // 4, lane % 4
    words = np.zeros((strips, chunks, 32, 4), dtype=np.uint32)
    for si in range(strips):
        for c in range(chunks):
            for kk in range(4):
                r = 16 * si + g + 8 * (kk & 1)
                kb = 64 * c + 32 * (kk >> 1) + 4 * t
                w = np.zeros(32, dtype=np.uint32)
                for b in range(4):
                    byte = q[kb + b, r].astype(np.uint32) | (q[kb + 16 + b, r].astype(np.uint32) << np.uint32(4))
                    w |= byte << np.uint32(8 * b)
                words[si, c, :, kk] = w
    sc = np.zeros((strips, groups, 8, 2), dtype=np.uint16)
    zp = np.zeros((strips, groups, 8), dtype=np.uint8)
    for si in range(strips):
        for gr in range(groups):
            rows = 16 * si + np.arange(8)
            sc[si, gr, :, 0] = s[gr, rows]
            sc[si, gr, :, 1] = s[gr, rows + 8]
            zp[si, gr, :] = (z[gr, rows] | (z[gr, rows + 8] << 4)).astype(np.uint8)
    return words.view(np.uint8).reshape(-1), sc.view(np.uint8).reshape(-1), zp.reshape(-1)


def repack_expert(t: dict, e: int | None, hidden: int, inter: int, group: int) -> np.ndarray:
    """One expert blob (uint8 [bytes]) from GPTQ tensors (numpy or torch)."""
    def get(name):
        v = t[name] if e is None else t[name][e]
        return v.numpy() if hasattr(v, "numpy") else np.asarray(v)
    L = expert_layout(hidden, inter, group)
    blob = np.zeros(L["bytes"], dtype=np.uint8)
    for p in ("w13", "w2"):
        qw, sc, zp = repack_projection(get(f"{p}_qweight"), get(f"{p}_qzeros"), get(f"{p}_scales"), group)
        blob[L[f"{p}_qweight"]:L[f"{p}_qweight"] + qw.size] = qw
        blob[L[f"{p}_scales"]:L[f"{p}_scales"] + sc.size] = sc
        blob[L[f"{p}_zeros"]:L[f"{p}_zeros"] + zp.size] = zp
    return blob


def decode_projection(blob: np.ndarray, off_q: int, off_s: int, off_z: int, n: int, k: int, group: int,
                      zero_mode: str = "raw") -> np.ndarray:
    """Inverse: kernel layout -> fp32 [N, K] (Linear orientation), computed as the
    kernel's dequantisation defines it: (q - z) * s per element."""
    strips, chunks, groups = n // 16, k // 64, k // group
    words = blob[off_q:off_q + n * k // 2].view(np.uint32).reshape(strips, chunks, 32, 4)
    sc = blob[off_s:off_s + n * groups * 2].view(np.float16).reshape(strips, groups, 8, 2)
    zp = blob[off_z:off_z + n * groups // 2].reshape(strips, groups, 8)
    out = np.zeros((n, k), dtype=np.float32)
    lane = np.arange(32)
    g, t = lane // 4, lane % 4
    for si in range(strips):
        for c in range(chunks):
            for kk in range(4):
                w = words[si, c, :, kk]
                rr = 16 * si + g + 8 * (kk & 1)
                kb = 64 * c + 32 * (kk >> 1) + 4 * t
                for b in range(4):
                    byte = (w >> np.uint32(8 * b)) & np.uint32(0xFF)
                    for kc, qv in ((kb + b, byte & np.uint32(0xF)), (kb + 16 + b, byte >> np.uint32(4))):
                        grp = kc // group
                        zbyte = zp[si, grp, g]
                        zrow = np.where((kk & 1) == 0, zbyte & 0xF, zbyte >> 4).astype(np.float32)
                        if zero_mode == "sym8":
                            zrow = np.float32(8.0)
                        srow = np.where((kk & 1) == 0, sc[si, grp, g, 0], sc[si, grp, g, 1]).astype(np.float32)
                        out[rr, kc] = (qv.astype(np.float32) - zrow) * srow
    return out
