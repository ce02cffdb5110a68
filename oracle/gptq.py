"""GPTQ int4 pack / unpack / dequantise, restated in numpy.

Test infrastructure (see ``oracle/__init__.py``): never imported by the
shipped package.

Reference: src/mtp_expert_prefetch/repack/gptq_unpack.py
  * ``unpack_cols``  :54-68  - int32 words packed along the column (N) axis;
                               nibble i of word j is column 8j+i.
  * ``unpack_rows``  :71-85  - int32 words packed along the row (K) axis;
                               nibble i of word j is row 8j+i.
  * ``dequantize_gptq_projection`` :88-131 - fp32 ``(q - z[g_idx]) * s[g_idx]``,
                               transposed to Linear orientation [out, in].
  * ``synthesize_g_idx`` :134-148 - ``arange(K) // group_size``.
The pack helpers restate the inverse used by the reference tests
(tests/test_gptq_unpack.py:17-38).
"""
from __future__ import annotations

import numpy as np

PACK = 8  # int4 values per int32 word
MASK = 0xF


def _as_u32(packed: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(packed).view(np.uint32)


def unpack_rows(packed: np.ndarray) -> np.ndarray:
    """[R, C] int32 -> [R*8, C] int32; row 8j+i of the result is nibble i of row j."""
    words = _as_u32(packed).astype(np.uint64)
    rows, cols = words.shape
    out = np.empty((rows * PACK, cols), dtype=np.int32)
    for i in range(PACK):
        out[i::PACK, :] = ((words >> np.uint64(4 * i)) & np.uint64(MASK)).astype(np.int32)
    return out


def unpack_cols(packed: np.ndarray) -> np.ndarray:
    """[R, C] int32 -> [R, C*8] int32; column 8j+i of the result is nibble i of column j."""
    words = _as_u32(packed).astype(np.uint64)
    rows, cols = words.shape
    out = np.empty((rows, cols * PACK), dtype=np.int32)
    for i in range(PACK):
        out[:, i::PACK] = ((words >> np.uint64(4 * i)) & np.uint64(MASK)).astype(np.int32)
    return out


def pack_rows(values: np.ndarray) -> np.ndarray:
    """Inverse of :func:`unpack_rows` (tests/test_gptq_unpack.py:17-26)."""
    v = np.asarray(values).astype(np.uint64) & np.uint64(MASK)
    rows, cols = v.shape
    assert rows % PACK == 0, "row count must be a multiple of 8"
    out = np.zeros((rows // PACK, cols), dtype=np.uint64)
    for i in range(PACK):
        out |= v[i::PACK, :] << np.uint64(4 * i)
    return out.astype(np.uint32).view(np.int32)


def pack_cols(values: np.ndarray) -> np.ndarray:
    """Inverse of :func:`unpack_cols` (tests/test_gptq_unpack.py:29-38)."""
    v = np.asarray(values).astype(np.uint64) & np.uint64(MASK)
    rows, cols = v.shape
    assert cols % PACK == 0, "column count must be a multiple of 8"
    out = np.zeros((rows, cols // PACK), dtype=np.uint64)
    for i in range(PACK):
        out |= v[:, i::PACK] << np.uint64(4 * i)
    return out.astype(np.uint32).view(np.int32)


def synthesize_g_idx(in_features: int, group_size: int = 128) -> np.ndarray:
    """gptq_unpack.py:134-148."""
    return (np.arange(in_features, dtype=np.int64) // int(group_size)).astype(np.int32)


def dequantize(
    qweight: np.ndarray,
    qzeros: np.ndarray,
    scales: np.ndarray,
    g_idx: np.ndarray | None = None,
    *,
    group_size: int = 128,
    zero_mode: str = "raw",
    linear_weight: bool = True,
) -> np.ndarray:
    """fp32 dequantisation of one projection (gptq_unpack.py:88-131).

    ``zero_mode``:
      * ``"raw"``  - the stored zero point as is (the reference torch oracle,
                     gptq_unpack.py:104,127-128).
      * ``"sym8"`` - the constant 8 that vLLM's symmetric GPTQ path uses and the
                     stored zeros ignored (vllm_wna16_group_plan.py:410-416).
    Returns [out, in] (Linear orientation) when ``linear_weight``.
    """
    q = unpack_rows(qweight)                       # [K, N]
    k = q.shape[0]
    if g_idx is None:
        g_idx = synthesize_g_idx(k, group_size)
    g_idx = np.asarray(g_idx, dtype=np.int64)
    s = np.asarray(scales).astype(np.float32)[g_idx]  # fp16 -> fp32 exact
    if zero_mode == "raw":
        z = unpack_cols(qzeros).astype(np.float32)[g_idx]
    elif zero_mode == "sym8":
        z = np.float32(8.0)
    else:
        raise ValueError(f"unknown zero_mode {zero_mode!r}")
    w = (q.astype(np.float32) - z) * s
    if linear_weight:
        w = np.ascontiguousarray(w.T)
    return w.astype(np.float32)
