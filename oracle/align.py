"""moe_align_block_size restated in numpy with a canonical (stable) order.

Test infrastructure (see ``oracle/__init__.py``).

Reference: vLLM 0.22.0 ``model_executor/layers/fused_moe/moe_align_block_size.py``
``moe_align_block_size`` (wrapper docstring and buffer sizing), as called by the
reference at src/mtp_expert_prefetch/tracing/vllm_router_trace.py:19648-19659
with ``ignore_invalid_experts=True``. The vLLM op itself is compiled code and
is not read; its documented contract is restated here:

* the flat pair index ``t*top_k + j`` of every routed (token, slot) is grouped
  by expert into blocks of ``block_size``; each expert's run is padded up to a
  multiple of ``block_size`` with the sentinel ``numel = M*top_k``;
* ``expert_ids[b]`` is the expert that owns block ``b``;
* ``num_tokens_post_padded`` is the padded total;
* buffer length ``numel + E*(block_size-1)`` (rounded up to ``block_size`` when
  ``pad_sorted_ids``), capped at ``numel*block_size`` when ``numel < E``;
* with ``expert_map`` and ``ignore_invalid_experts`` the pairs whose expert maps
  to -1 are dropped and ``expert_ids`` holds the mapped (local) ids; without
  ``ignore_invalid_experts`` every pair counts and ``expert_ids`` is mapped
  through ``expert_map`` afterwards (so non-local blocks read -1).

Canonical order (what vLLM's atomics leave unspecified): experts in ascending
global id, and inside an expert ascending flat index. This reproduces the
docstring's worked example. Positions past ``num_tokens_post_padded`` hold the
sentinel and blocks past the last used block hold -1.

``segments`` is this build's extra output: one row per expert that owns at
least one block, ``(expert, first_block, block_count)``, ascending expert.
"""
from __future__ import annotations

import numpy as np


def cdiv(a: int, b: int) -> int:
    return -(-a // b)


def buffer_sizes(numel: int, num_experts: int, block_size: int, pad_sorted_ids: bool = False):
    cap = numel + num_experts * (block_size - 1)
    if pad_sorted_ids:
        cap = cdiv(cap, block_size) * block_size
    if numel < num_experts:
        cap = min(numel * block_size, cap)
    return cap, cdiv(cap, block_size)


def moe_align_block_size(
    topk_ids: np.ndarray,
    block_size: int,
    num_experts: int,
    expert_map: np.ndarray | None = None,
    pad_sorted_ids: bool = False,
    ignore_invalid_experts: bool = False,
):
    ids = np.asarray(topk_ids, dtype=np.int64).reshape(-1)
    numel = ids.size
    cap, max_blocks = buffer_sizes(numel, num_experts, block_size, pad_sorted_ids)
    sorted_ids = np.full(cap, numel, dtype=np.int32)
    expert_ids = np.full(max_blocks, -1, dtype=np.int32)

    valid = (ids >= 0) & (ids < num_experts)
    if expert_map is not None and ignore_invalid_experts:
        emap = np.asarray(expert_map, dtype=np.int64)
        mapped = np.where(valid, emap[np.clip(ids, 0, num_experts - 1)], -1)
        valid &= mapped >= 0

    pos = 0
    segments = []
    for e in range(num_experts):
        flat = np.nonzero(valid & (ids == e))[0]          # ascending flat index
        cnt = flat.size
        if cnt == 0:
            continue
        padded = cdiv(cnt, block_size) * block_size
        sorted_ids[pos:pos + cnt] = flat.astype(np.int32)
        b0 = pos // block_size
        nb = padded // block_size
        if expert_map is not None:
            tag = int(np.asarray(expert_map)[e])
        else:
            tag = e
        expert_ids[b0:b0 + nb] = tag
        segments.append((e, b0, nb))
        pos += padded
    ntpp = np.array([pos], dtype=np.int32)
    seg = np.array(segments, dtype=np.int32).reshape(-1, 3)
    return sorted_ids, expert_ids, ntpp, seg
