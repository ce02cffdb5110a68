"""Host API of the W4A16 MoE path: torch tensors in, C-ABI calls out.

Names and argument meanings follow the reference interfaces this path drops
in for (paths relative to the reference project; vLLM 0.22.0 paths relative to
the package):

* :func:`topk_softmax`          - vLLM ``topk_softmax`` (restated at
                                  tracing/vllm_router_trace.py:4201-4227);
* :func:`moe_align_block_size`  - vLLM ``fused_moe/moe_align_block_size.py``;
* :func:`dequantize_gptq_projection` - repack/gptq_unpack.py:88-131;
* :func:`fused_experts`         - vLLM ``fused_experts`` (signature probed by the
                                  reference, replaced at vllm_router_trace.py:19330-19840);
* :func:`moe_layer_w4a16`       - router + fused_experts + shared expert, the
                                  ``FusedMoE.forward_impl`` boundary (17977) and
                                  ``MtpExtraRunner.moe_tokens`` (mtp/extra_tensors.py:544-598).

Shape and dtype errors raise ``ValueError`` before any launch (as
gptq_unpack.py:374-417 and the reference invokers do); a non-zero C status
raises :class:`mtp_b200._lib.MtpError`. Every call is asynchronous on the
current torch CUDA stream. There is no CPU path.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib

ZERO_MODES = {"raw": _lib.MTP_ZERO_RAW, "sym8": _lib.MTP_ZERO_SYM8}


def _p(t: torch.Tensor | None):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(t: torch.Tensor):
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _check_cuda(name: str, t: torch.Tensor | None, dtype: torch.dtype | None = None, ndim: int | None = None):
    if t is None:
        return
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor, got device {t.device}")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if ndim is not None and t.ndim != ndim:
        raise ValueError(f"{name} must be {ndim}-D, got shape {tuple(t.shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


# ---------------------------------------------------------------------------
# router
# ---------------------------------------------------------------------------
def topk_softmax(gating_output: torch.Tensor, topk: int, renormalize: bool = True):
    """softmax -> top-k -> (optional) renormalise. Returns
    ``(topk_weights fp32 [M,k], topk_ids int32 [M,k], token_expert_indices int32 [M,k])``."""
    _check_cuda("gating_output", gating_output, torch.float32, 2)
    m, e = gating_output.shape
    if not 0 < topk <= min(e, 32):
        raise ValueError(f"topk must be in [1, {min(e, 32)}], got {topk}")
    if e > 1024:
        raise ValueError(f"at most 1024 experts are supported, got {e}")
    dev = gating_output.device
    w = torch.empty((m, topk), dtype=torch.float32, device=dev)
    ids = torch.empty((m, topk), dtype=torch.int32, device=dev)
    tei = torch.empty((m, topk), dtype=torch.int32, device=dev)
    if m:
        _lib.call("mtp_router_topk", _p(gating_output), m, e, topk, int(bool(renormalize)),
                  _p(w), _p(ids), _p(tei), _stream(gating_output))
    return w, ids, tei


# ---------------------------------------------------------------------------
# align
# ---------------------------------------------------------------------------
def moe_align_block_size(topk_ids: torch.Tensor, block_size: int, num_experts: int,
                         expert_map: torch.Tensor | None = None, pad_sorted_ids: bool = False,
                         ignore_invalid_experts: bool = False, *, return_segments: bool = False):
    """Same contract as vLLM's wrapper; the order inside an expert is the
    ascending flat index ``t*top_k + j`` (deterministic). With
    ``return_segments`` also returns ``(segments [max_seg, 3], num_segments [1])``."""
    if topk_ids.dtype != torch.int32:
        raise ValueError(f"topk_ids must be int32, got {topk_ids.dtype}")
    _check_cuda("topk_ids", topk_ids)
    if expert_map is not None:
        _check_cuda("expert_map", expert_map, torch.int32, 1)
        if expert_map.numel() != num_experts:
            raise ValueError("expert_map must have num_experts entries")
    numel = topk_ids.numel()
    cap, blocks, max_seg = _lib.align_sizes(numel, num_experts, block_size, pad_sorted_ids)
    dev = topk_ids.device
    sorted_ids = torch.empty(cap, dtype=torch.int32, device=dev)
    expert_ids = torch.empty(blocks, dtype=torch.int32, device=dev)
    ntpp = torch.empty(1, dtype=torch.int32, device=dev)
    segs = torch.empty((max(max_seg, 1), 3), dtype=torch.int32, device=dev) if return_segments else None
    nseg = torch.empty(1, dtype=torch.int32, device=dev) if return_segments else None
    _lib.call("mtp_moe_align", _p(topk_ids), numel, num_experts, block_size, _p(expert_map),
              int(bool(ignore_invalid_experts)), int(bool(pad_sorted_ids)), _p(sorted_ids),
              _p(expert_ids), _p(ntpp), _p(segs), _p(nseg), _stream(topk_ids))
    if return_segments:
        return sorted_ids, expert_ids, ntpp, segs[:max_seg], nseg
    return sorted_ids, expert_ids, ntpp


# ---------------------------------------------------------------------------
# GPTQ weights
# ---------------------------------------------------------------------------
def dequantize_gptq_projection(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
                               g_idx: torch.Tensor | None = None, *, group_size: int = 128,
                               zero_mode: str = "raw", dtype: torch.dtype = torch.float32,
                               linear_weight: bool = True) -> torch.Tensor:
    """fp32 ``(q - z[g_idx]) * s[g_idx]`` on the GPU; [out, in] when ``linear_weight``."""
    _check_cuda("qweight", qweight, torch.int32, 2)
    _check_cuda("qzeros", qzeros, torch.int32, 2)
    _check_cuda("scales", scales, torch.float16, 2)
    _check_cuda("g_idx", g_idx, torch.int32, 1)
    k = qweight.shape[0] * 8
    n = qweight.shape[1]
    if scales.shape[1] != n or qzeros.shape[1] * 8 != n or scales.shape != (qzeros.shape[0], n):
        raise ValueError(f"inconsistent GPTQ shapes: qweight {tuple(qweight.shape)}, "
                         f"qzeros {tuple(qzeros.shape)}, scales {tuple(scales.shape)}")
    if g_idx is not None and g_idx.numel() != k:
        raise ValueError(f"g_idx has {g_idx.numel()} entries, expected {k}")
    if zero_mode not in ZERO_MODES:
        raise ValueError(f"zero_mode must be one of {sorted(ZERO_MODES)}")
    out = torch.empty((n, k), dtype=torch.float32, device=qweight.device)
    _lib.call("mtp_gptq_dequant", _p(qweight), _p(qzeros), _p(scales.view(torch.int16)), _p(g_idx),
              k, n, group_size, ZERO_MODES[zero_mode], _p(out), _stream(qweight))
    if not linear_weight:
        out = out.t().contiguous()
    return out.to(dtype)


@dataclass
class W4A16Experts:
    """E routed experts in the kernel layout: ``blobs`` uint8 [E, layout.bytes]."""

    blobs: torch.Tensor | None
    num_experts: int
    hidden: int
    inter: int
    group_size: int
    layout: _lib.MtpExpertLayout

    @property
    def expert_bytes(self) -> int:
        return int(self.layout.bytes)

    @classmethod
    def from_gptq(cls, w13_qweight, w13_qzeros, w13_scales, w2_qweight, w2_qzeros, w2_scales,
                  *, group_size: int = 128) -> "W4A16Experts":
        """Repack GPTQ checkpoint tensors (leading E axis) once into the kernel
        layout. w13 = [gate; up] rows: qweight [E, H/8, 2I]; w2: qweight [E, I/8, H]."""
        for name, t, dt in (("w13_qweight", w13_qweight, torch.int32), ("w13_qzeros", w13_qzeros, torch.int32),
                            ("w13_scales", w13_scales, torch.float16), ("w2_qweight", w2_qweight, torch.int32),
                            ("w2_qzeros", w2_qzeros, torch.int32), ("w2_scales", w2_scales, torch.float16)):
            _check_cuda(name, t, dt, 3)
        e, h8, two_i = w13_qweight.shape
        hidden, inter = h8 * 8, two_i // 2
        if w2_qweight.shape != (e, inter // 8, hidden):
            raise ValueError(f"w2_qweight must be {(e, inter // 8, hidden)}, got {tuple(w2_qweight.shape)}")
        if w13_scales.shape != (e, hidden // group_size, two_i) or w2_scales.shape != (e, inter // group_size, hidden):
            raise ValueError("scales do not match group_size")
        if w13_qzeros.shape != (e, hidden // group_size, two_i // 8) or w2_qzeros.shape != (e, inter // group_size, hidden // 8):
            raise ValueError("qzeros do not match group_size")
        layout = _lib.expert_layout(hidden, inter, group_size)
        blobs = torch.zeros((e, layout.bytes), dtype=torch.uint8, device=w13_qweight.device)
        _lib.call("mtp_w4a16_repack_gptq", _p(w13_qweight), _p(w13_qzeros), _p(w13_scales.view(torch.int16)),
                  _p(w2_qweight), _p(w2_qzeros), _p(w2_scales.view(torch.int16)), e, hidden, inter,
                  group_size, _p(blobs), _stream(w13_qweight))
        return cls(blobs, e, hidden, inter, group_size, layout)

    def shard(self, rank: int, world: int) -> "W4A16Experts":
        """The experts [rank * E / world, (rank + 1) * E / world) as a view: the
        local expert set of one rank of an expert-parallel group."""
        if world < 1 or not 0 <= rank < world or self.num_experts % world:
            raise ValueError(f"{self.num_experts} experts do not shard evenly over {world} ranks")
        n = self.num_experts // world
        return W4A16Experts(self.blobs[rank * n:(rank + 1) * n], n, self.hidden, self.inter,
                            self.group_size, self.layout)


@dataclass
class SharedExpert:
    """The sigmoid-gated shared expert: one blob [layout.bytes] + gate weight [H] bf16."""

    blob: torch.Tensor
    gate_weight: torch.Tensor

    @classmethod
    def from_gptq(cls, w13_qweight, w13_qzeros, w13_scales, w2_qweight, w2_qzeros, w2_scales,
                  gate_weight, *, group_size: int = 128) -> "SharedExpert":
        ex = W4A16Experts.from_gptq(w13_qweight[None], w13_qzeros[None], w13_scales[None],
                                    w2_qweight[None], w2_qzeros[None], w2_scales[None],
                                    group_size=group_size)
        gw = gate_weight.reshape(-1)
        _check_cuda("gate_weight", gw, torch.bfloat16, 1)
        if gw.numel() != ex.hidden:
            raise ValueError("gate_weight must have hidden entries")
        return cls(ex.blobs[0], gw.contiguous())


# ---------------------------------------------------------------------------
# the layer
# ---------------------------------------------------------------------------
def layer_workspace(m: int, experts: W4A16Experts, top_k: int, device) -> torch.Tensor:
    nbytes = _lib.layer_workspace_bytes(m, experts.num_experts, top_k, experts.hidden, experts.inter)
    # zero-filled once: the layer keeps its call counters there and leaves
    # them zero after every call
    return torch.zeros(nbytes, dtype=torch.uint8, device=device)


# Average routed pairs per expert from which the automatic path choice runs a
# call on the prefill kernels (128-pair bf16 tiles) instead of the decode
# kernel (8-pair int8 tiles, exact dequantisation).
PREFILL_MIN_PAIRS_PER_EXPERT = 32


def layer_path(m: int, num_experts: int, top_k: int) -> str:
    """"prefill" when the call has enough pairs per expert for 128-pair tiles,
    else "decode" (the automatic choice of :func:`moe_layer_w4a16`)."""
    return "prefill" if m * top_k >= PREFILL_MIN_PAIRS_PER_EXPERT * num_experts else "decode"


def prefill_workspace(m: int, experts: W4A16Experts, top_k: int, device) -> torch.Tensor:
    """Workspace of the prefill path (no zero fill needed)."""
    nbytes = _lib.prefill_workspace_bytes(m, experts.num_experts, top_k, experts.hidden, experts.inter)
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def moe_layer_w4a16(hidden_states: torch.Tensor, router_logits: torch.Tensor | None,
                    experts: W4A16Experts, top_k: int, renormalize: bool = True,
                    shared: SharedExpert | None = None, *,
                    topk_weights: torch.Tensor | None = None, topk_ids: torch.Tensor | None = None,
                    slot_table: torch.Tensor | None = None, slot_cache: torch.Tensor | None = None,
                    host_store: torch.Tensor | None = None, zero_mode: str = "raw",
                    out: torch.Tensor | None = None, out_f32: torch.Tensor | None = None,
                    topk_out: tuple[torch.Tensor, torch.Tensor] | None = None,
                    demand_log: torch.Tensor | None = None, status: torch.Tensor | None = None,
                    workspace: torch.Tensor | None = None, path: str = "auto",
                    expert_map: torch.Tensor | None = None,
                    shared_rows: tuple[int, int] | None = None) -> torch.Tensor:
    """One W4A16 MoE layer forward: router (when ``router_logits`` is given,
    else the given ``topk_weights``/``topk_ids``), align, gate_up + SiLU*up,
    down + routed weight, top-k sum and the sigmoid-gated shared expert.

    Weights: ``experts.blobs`` (slot = expert), or with ``slot_table`` [E]
    int32 the slot cache ``slot_cache`` [S, bytes] (slot -1 = not resident,
    read from the pinned ``host_store`` [E, bytes] through its device
    mapping). Returns ``out`` [M, H] bf16.

    ``path``: "decode" (the persistent layer kernel), "prefill" (128-pair
    bf16 tiles; every expert resident, no ``slot_table`` / ``demand_log``) or
    "auto": prefill when :func:`layer_path` says so, the call allows it and a
    given ``workspace`` is large enough for it.

    Expert parallelism: ``expert_map`` [global E] int32 (vLLM's expert_map)
    takes global ``topk_ids`` to this shard's experts (-1: another rank's,
    the pair contributes nothing); ``shared_rows`` = (begin, end) restricts
    the shared expert to those rows."""
    _check_cuda("hidden_states", hidden_states, torch.bfloat16, 2)
    m, h = hidden_states.shape
    if h != experts.hidden:
        raise ValueError(f"hidden_states last dim {h} != experts hidden {experts.hidden}")
    e = experts.num_experts
    if router_logits is not None:
        _check_cuda("router_logits", router_logits, torch.float32, 2)
        if router_logits.shape != (m, e):
            raise ValueError(f"router_logits must be {(m, e)}, got {tuple(router_logits.shape)}")
    else:
        if topk_weights is None or topk_ids is None:
            raise ValueError("give router_logits or topk_weights and topk_ids")
        _check_cuda("topk_weights", topk_weights, torch.float32, 2)
        _check_cuda("topk_ids", topk_ids, torch.int32, 2)
        if topk_weights.shape != (m, top_k) or topk_ids.shape != (m, top_k):
            raise ValueError(f"topk_weights/topk_ids must be {(m, top_k)}")
    if zero_mode not in ZERO_MODES:
        raise ValueError(f"zero_mode must be one of {sorted(ZERO_MODES)}")
    blobs = experts.blobs
    if slot_table is not None:
        _check_cuda("slot_table", slot_table, torch.int32, 1)
        if slot_table.numel() != e:
            raise ValueError("slot_table must have num_experts entries")
        blobs = slot_cache
        if slot_cache is None and host_store is None:
            raise ValueError("slot_table needs slot_cache and/or host_store")
    if blobs is not None:
        _check_cuda("expert blobs", blobs, torch.uint8)
    host_ptr = None
    if host_store is not None:
        if not host_store.is_pinned():
            raise ValueError("host_store must be pinned host memory")
        host_ptr = C.c_void_p(_lib.host_device_pointer(host_store.data_ptr()))
    dev = hidden_states.device
    if out is None:
        out = torch.empty((m, h), dtype=torch.bfloat16, device=dev)
    _check_cuda("out", out, torch.bfloat16, 2)
    _check_cuda("out_f32", out_f32, torch.float32, 2)
    if path not in ("auto", "decode", "prefill"):
        raise ValueError('path must be "auto", "decode" or "prefill"')
    if path == "prefill" and (slot_table is not None or demand_log is not None):
        raise ValueError("the prefill path needs every expert resident and writes no demand_log")
    if path == "auto":
        path = "decode"
        if slot_table is None and demand_log is None and layer_path(m, e, top_k) == "prefill":
            need = _lib.prefill_workspace_bytes(m, e, top_k, h, experts.inter)
            if workspace is None or workspace.numel() >= need:
                path = "prefill"
    if workspace is None:
        workspace = (prefill_workspace if path == "prefill" else layer_workspace)(m, experts, top_k, dev)
    args = _lib.MtpMoeLayerArgs()
    args.num_tokens, args.hidden, args.inter, args.num_experts = m, h, experts.inter, e
    args.top_k, args.group_size, args.renormalize = top_k, experts.group_size, int(bool(renormalize))
    args.zero_mode = ZERO_MODES[zero_mode]
    args.hidden_states = hidden_states.data_ptr()
    args.router_logits = router_logits.data_ptr() if router_logits is not None else None
    args.topk_weights = topk_weights.data_ptr() if topk_weights is not None else None
    args.topk_ids = topk_ids.data_ptr() if topk_ids is not None else None
    args.expert_blobs = blobs.data_ptr() if blobs is not None else None
    args.expert_bytes = experts.expert_bytes
    args.slot_table = slot_table.data_ptr() if slot_table is not None else None
    args.host_blobs = host_ptr.value if host_ptr is not None else None
    args.shared_blob = shared.blob.data_ptr() if shared is not None else None
    args.shared_gate_weight = shared.gate_weight.data_ptr() if shared is not None else None
    args.out = out.data_ptr()
    args.out_f32 = out_f32.data_ptr() if out_f32 is not None else None
    if topk_out is not None:
        args.topk_weights_out = topk_out[0].data_ptr()
        args.topk_ids_out = topk_out[1].data_ptr()
    args.demand_log = demand_log.data_ptr() if demand_log is not None else None
    args.status = status.data_ptr() if status is not None else None
    args.workspace = workspace.data_ptr()
    args.workspace_bytes = workspace.numel()
    if expert_map is not None:
        if router_logits is not None:
            raise ValueError("expert_map needs given topk_ids (global ids), not router_logits")
        _check_cuda("expert_map", expert_map, torch.int32, 1)
        args.expert_map = expert_map.data_ptr()
        args.global_num_experts = expert_map.numel()
    if shared_rows is not None:
        b, e_ = int(shared_rows[0]), int(shared_rows[1])
        if not 0 <= b <= e_ <= m:
            raise ValueError(f"shared_rows {shared_rows} outside [0, {m}]")
        if b == e_:
            raise ValueError("an empty shared_rows range: pass shared=None instead")
        args.shared_rows_begin, args.shared_rows_end = b, e_
    _lib.call("mtp_w4a16_moe_prefill" if path == "prefill" else "mtp_w4a16_moe_layer", C.byref(args),
              _stream(hidden_states))
    return out


def vllm_wna16_to_gptq(w13_qweight: torch.Tensor, w2_qweight: torch.Tensor, w13_scales: torch.Tensor,
                       w2_scales: torch.Tensor) -> dict:
    """vLLM's moe_wna16 GPTQ tensors back to the checkpoint form.

    vLLM keeps, per expert, ``qweight.T.contiguous().view(uint8)`` ([N, K/2],
    low nibble = even k) and ``scales.T`` ([N, K/g]) (moe_wna16.py
    create_weights and moe_wna16_weight_loader, GPTQ branch); a symmetric
    checkpoint has no zero points there (the kernel subtracts 8), so the
    returned qzeros hold 8 in every nibble. Shapes: w13 [E, 2I, H/2] and
    [E, 2I, H/g], w2 [E, H, I/2] and [E, H, I/g]; returns the ``from_gptq``
    keys (qweight [E, K/8, N] int32, qzeros [E, K/g, N/8] int32, scales
    [E, K/g, N] fp16)."""
    out = {}
    for name, q, sc in (("w13", w13_qweight, w13_scales), ("w2", w2_qweight, w2_scales)):
        if q.dtype != torch.uint8 or q.dim() != 3 or sc.dim() != 3 or q.shape[:2] != sc.shape[:2]:
            raise ValueError(f"{name}: expected uint8 [E, N, K/2] weights and [E, N, K/g] scales, got "
                             f"{tuple(q.shape)} {q.dtype} and {tuple(sc.shape)}")
        e, n, k_half = q.shape
        out[f"{name}_qweight"] = q.contiguous().view(torch.int32).transpose(1, 2).contiguous()
        out[f"{name}_scales"] = sc.transpose(1, 2).contiguous().to(torch.float16)
        zero8 = torch.tensor(0x88888888 - (1 << 32), dtype=torch.int32)
        out[f"{name}_qzeros"] = zero8.expand(e, sc.shape[2], n // 8).contiguous().to(q.device)
    return out


_VLLM_REPACKED: dict = {}


def experts_from_vllm_wna16(w1: torch.Tensor, w2: torch.Tensor, quant_config) -> W4A16Experts:
    """The kernel-layout experts for vLLM's (w1, w2, quant_config) triple,
    repacked once and cached on the identity of the four tensors (the cache
    holds them, so an id cannot be reused while the entry lives)."""
    s1, s2 = getattr(quant_config, "w1_scale", None), getattr(quant_config, "w2_scale", None)
    if s1 is None or s2 is None:
        raise ValueError("quant_config must carry w1_scale and w2_scale (vLLM int4_w4a16)")
    if getattr(quant_config, "w1_zp", None) is not None or getattr(quant_config, "w2_zp", None) is not None:
        raise ValueError("zero points in vLLM's moe_wna16 layout are not supported (symmetric GPTQ only)")
    key = tuple(id(t) for t in (w1, w2, s1, s2))
    hit = _VLLM_REPACKED.get(key)
    if hit is not None and all(a is b for a, b in zip(hit[0], (w1, w2, s1, s2))):
        return hit[1]
    g = vllm_wna16_to_gptq(w1, w2, s1, s2)
    hidden = w1.shape[2] * 2
    experts = W4A16Experts.from_gptq(g["w13_qweight"], g["w13_qzeros"], g["w13_scales"], g["w2_qweight"],
                                     g["w2_qzeros"], g["w2_scales"], group_size=hidden // s1.shape[2])
    _VLLM_REPACKED[key] = ((w1, w2, s1, s2), experts)
    return experts


def fused_experts(hidden_states: torch.Tensor, w1, w2=None,
                  topk_weights: torch.Tensor | None = None, topk_ids: torch.Tensor | None = None,
                  inplace: bool = False, activation="silu",
                  apply_router_weight_on_input: bool = False, global_num_experts: int = -1,
                  expert_map: torch.Tensor | None = None, quant_config=None, *,
                  shared: SharedExpert | None = None, zero_mode: str = "raw") -> torch.Tensor:
    """vLLM ``fused_experts`` shape: routed experts given by ``topk_weights`` /
    ``topk_ids``. Weights either as vLLM passes them for int4_w4a16 (``w1``
    [E, 2I, H/2] and ``w2`` [E, H, I/2] uint8 in the moe_wna16 GPTQ layout,
    ``quant_config.w1_scale`` / ``w2_scale``; repacked once, see
    :func:`experts_from_vllm_wna16`), or as one :class:`W4A16Experts` in
    ``w1`` (``w2`` None or the same object). ``expert_map`` [global E] maps
    global ids to local ones (-1: not on this rank, the pair is skipped)."""
    name = str(getattr(activation, "value", getattr(activation, "name", activation))).lower()
    if name != "silu":
        raise ValueError(f"only SiLU is supported, got {activation!r}")
    if apply_router_weight_on_input:
        raise ValueError("apply_router_weight_on_input is not supported")
    if isinstance(w1, W4A16Experts):
        if w2 is not None and w2 is not w1:
            raise ValueError("with a W4A16Experts in w1, w2 must be None or the same object")
        experts = w1
    elif isinstance(w1, torch.Tensor) and isinstance(w2, torch.Tensor):
        experts = experts_from_vllm_wna16(w1, w2, quant_config)
        zero_mode = "sym8"
    else:
        raise ValueError("w1 / w2 must be vLLM int4_w4a16 tensors or one W4A16Experts")
    if topk_ids is None or topk_weights is None:
        raise ValueError("topk_weights and topk_ids are required")
    if topk_ids.dtype != torch.int32:
        topk_ids = topk_ids.to(torch.int32)
    if topk_weights.dtype != torch.float32:
        topk_weights = topk_weights.to(torch.float32)
    if expert_map is not None:
        if global_num_experts not in (-1, expert_map.numel()):
            raise ValueError("expert_map must have global_num_experts entries")
        ids = topk_ids.long()
        ok = (ids >= 0) & (ids < expert_map.numel())
        topk_ids = torch.where(ok, expert_map.to(ids.device)[ids.clamp(0, expert_map.numel() - 1)].long(),
                               torch.full_like(ids, -1)).to(torch.int32)
    elif global_num_experts not in (-1, experts.num_experts):
        raise ValueError("global_num_experts must equal the experts' count (or give expert_map)")
    out = moe_layer_w4a16(hidden_states, None, experts, int(topk_ids.shape[1]), shared=shared,
                          topk_weights=topk_weights.contiguous(), topk_ids=topk_ids.contiguous(),
                          zero_mode=zero_mode)
    if inplace:
        # The layer reads hidden_states until its last kernel, so the result is
        # written to a separate buffer first.
        hidden_states.copy_(out)
        return hidden_states
    return out


# ---------------------------------------------------------------------------
# MTP expert-demand predictor
# ---------------------------------------------------------------------------
class MtpPredictor:
    """BF16 predictor ``logits = W2 . silu(W1 . h + b1) + b2`` (hidden -> width
    -> future x experts) with per-future-layer top-k, the forward of the
    reference's predictor family (training/hidden_residual.py:44-134) at the
    BASELINE shape. Weights are prepacked once for the kernel."""

    def __init__(self, w1: torch.Tensor, b1: torch.Tensor | None, w2: torch.Tensor, b2: torch.Tensor | None,
                 *, future: int, experts: int):
        _check_cuda("w1", w1, torch.bfloat16, 2)
        _check_cuda("w2", w2, torch.bfloat16, 2)
        _check_cuda("b1", b1, torch.bfloat16, 1)
        _check_cuda("b2", b2, torch.bfloat16, 1)
        width, hidden = w1.shape
        if w2.shape != (future * experts, width):
            raise ValueError(f"w2 must be [{future * experts}, {width}], got {tuple(w2.shape)}")
        if b1 is not None and b1.numel() != width:
            raise ValueError("b1 must have width entries")
        if b2 is not None and b2.numel() != future * experts:
            raise ValueError("b2 must have future * experts entries")
        self.hidden, self.width, self.future, self.experts = hidden, width, future, experts
        self.w1p = torch.empty_like(w1)
        self.w2p = torch.empty_like(w2)
        _lib.call("mtp_predictor_pack", _p(w1), width, hidden, _p(self.w1p), _stream(w1))
        _lib.call("mtp_predictor_pack", _p(w2), future * experts, width, _p(self.w2p), _stream(w2))
        self.b1, self.b2 = b1, b2

    def workspace(self, m: int, device) -> torch.Tensor:
        return torch.empty(_lib.predictor_workspace_bytes(m, self.width, self.future, self.experts),
                           dtype=torch.uint8, device=device)

    def predict_topk(self, hidden: torch.Tensor, top_k: int, *, logits_out: torch.Tensor | None = None,
                     ids_out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
        """ids [M, future, top_k] int32 of the predicted experts per future layer."""
        _check_cuda("hidden", hidden, torch.bfloat16, 2)
        m = hidden.shape[0]
        if hidden.shape[1] != self.hidden:
            raise ValueError(f"hidden must be [M, {self.hidden}]")
        ids = ids_out if ids_out is not None else torch.empty(m, self.future, top_k, dtype=torch.int32,
                                                              device=hidden.device)
        _check_cuda("ids_out", ids, torch.int32)
        _check_cuda("logits_out", logits_out, torch.float32)
        ws = workspace if workspace is not None else self.workspace(m, hidden.device)
        _lib.call("mtp_predict_topk", _p(hidden), m, self.hidden, _p(self.w1p), _p(self.b1), self.width,
                  _p(self.w2p), _p(self.b2), self.future, self.experts, top_k, _p(logits_out), _p(ids),
                  _p(ws), ws.numel(), _stream(hidden))
        return ids


class HiddenResidualPredictor:
    """The reference's ``HiddenResidualExpertPredictor`` forward on the GPU
    (training/hidden_residual.py:44-103): encoder Linear -> SiLU -> LayerNorm,
    plus a layer embedding and a per-delta embedding, SiLU, and one shared
    classifier over experts for every future delta; then top-k per delta.
    ``from_module`` takes the weights of a reference module (cast to bf16)."""

    def __init__(self, w1, b1, ln_weight, ln_bias, layer_emb, delta_emb, wc, bc, *, ln_eps: float = 1e-5):
        for name, t in (("w1", w1), ("layer_emb", layer_emb), ("delta_emb", delta_emb), ("wc", wc)):
            _check_cuda(name, t, torch.bfloat16, 2)
        for name, t in (("b1", b1), ("ln_weight", ln_weight), ("ln_bias", ln_bias), ("bc", bc)):
            _check_cuda(name, t, torch.bfloat16, 1)
        self.width, self.hidden = w1.shape
        self.experts = wc.shape[0]
        self.num_layers, self.future = layer_emb.shape[0], delta_emb.shape[0]
        if wc.shape[1] != self.width or layer_emb.shape[1] != self.width or delta_emb.shape[1] != self.width:
            raise ValueError("classifier and embeddings must have width columns")
        self.w1p = torch.empty_like(w1)
        self.wcp = torch.empty_like(wc)
        _lib.call("mtp_predictor_pack", _p(w1), self.width, self.hidden, _p(self.w1p), _stream(w1))
        _lib.call("mtp_predictor_pack", _p(wc), self.experts, self.width, _p(self.wcp), _stream(wc))
        self.b1, self.ln_weight, self.ln_bias, self.bc = b1, ln_weight, ln_bias, bc
        self.layer_emb, self.delta_emb = layer_emb.contiguous(), delta_emb.contiguous()
        self.ln_eps = float(ln_eps)

    @classmethod
    def from_module(cls, module, device) -> "HiddenResidualPredictor":
        enc, ln = module.encoder[0], module.encoder[2]
        bf = lambda t: None if t is None else t.detach().to(device=device, dtype=torch.bfloat16).contiguous()
        return cls(bf(enc.weight), bf(enc.bias), bf(ln.weight), bf(ln.bias), bf(module.layer_embedding.weight),
                   bf(module.delta_embedding.weight), bf(module.classifier.weight), bf(module.classifier.bias),
                   ln_eps=float(ln.eps))

    def workspace(self, m: int, device) -> torch.Tensor:
        out = _lib.i64()
        _lib.call("mtp_predictor_hr_workspace_size", m, self.width, self.future, self.experts, C.byref(out))
        return torch.empty(out.value, dtype=torch.uint8, device=device)

    def predict_topk(self, hidden: torch.Tensor, layer_ids: torch.Tensor | None, top_k: int, *,
                     logits_out: torch.Tensor | None = None, ids_out: torch.Tensor | None = None,
                     workspace: torch.Tensor | None = None) -> torch.Tensor:
        """ids [M, future, top_k] int32; ``layer_ids`` [M] int32 (None = layer 0)."""
        _check_cuda("hidden", hidden, torch.bfloat16, 2)
        _check_cuda("layer_ids", layer_ids, torch.int32, 1)
        m = hidden.shape[0]
        if hidden.shape[1] != self.hidden:
            raise ValueError(f"hidden must be [M, {self.hidden}]")
        ids = ids_out if ids_out is not None else torch.empty(m, self.future, top_k, dtype=torch.int32,
                                                              device=hidden.device)
        _check_cuda("ids_out", ids, torch.int32)
        _check_cuda("logits_out", logits_out, torch.float32)
        ws = workspace if workspace is not None else self.workspace(m, hidden.device)
        _lib.call("mtp_predict_topk_hidden_residual", _p(hidden), _p(layer_ids), m, self.hidden, _p(self.w1p),
                  _p(self.b1), self.width, _p(self.ln_weight), _p(self.ln_bias), C.c_float(self.ln_eps),
                  _p(self.layer_emb), self.num_layers, _p(self.delta_emb), self.future, _p(self.wcp), _p(self.bc),
                  self.experts, top_k, _p(logits_out), _p(ids), _p(ws), ws.numel(), _stream(hidden))
        return ids


# ---------------------------------------------------------------------------
# expert prefetch session (premap slot cache)
# ---------------------------------------------------------------------------
class PrefetchSession:
    """Per-layer HBM slot cache filled from a pinned host store on a side
    stream, with the expert -> slot tables the layer kernel reads. Counters
    follow the reference's cache managers (runtime/cache_manager.py:193-578).

    ``host_store`` is a pinned uint8 tensor [layers, experts, expert_bytes]
    (or None with ``simulate=True``, bookkeeping only)."""

    def __init__(self, num_layers: int, num_experts: int, slots_per_layer: int, expert_bytes: int,
                 host_store: torch.Tensor | None = None, device=None, simulate: bool = False,
                 shared_host_layers: bool = False):
        import numpy as np  # noqa: F401  (host arrays below)
        self.num_layers, self.num_experts, self.slots = num_layers, num_experts, slots_per_layer
        self.expert_bytes = expert_bytes
        self.host_store = host_store
        if simulate:
            self.cache = self.slot_tables = None
            dev_index = 0
        else:
            if host_store is None or not host_store.is_pinned():
                raise ValueError("host_store must be a pinned host tensor")
            want = (1 if shared_host_layers else num_layers) * num_experts * expert_bytes
            if host_store.numel() != want:
                raise ValueError("host_store must be [layers, experts, expert_bytes] bytes "
                                 "([experts, expert_bytes] with shared_host_layers)")
            device = torch.device(device)
            dev_index = device.index if device.index is not None else torch.cuda.current_device()
            # 256-byte aligned slots: expert_bytes is a multiple of 256 (expert layout)
            self.cache = torch.empty(num_layers * slots_per_layer * expert_bytes, dtype=torch.uint8, device=device)
            self.slot_tables = torch.empty(num_layers, num_experts, dtype=torch.int32, device=device)
        self.shared_host_layers = shared_host_layers
        cfg = _lib.MtpPrefetchConfig(dev_index, num_layers, num_experts, slots_per_layer, expert_bytes,
                                     None if simulate else host_store.data_ptr(),
                                     None if simulate else self.cache.data_ptr(),
                                     None if simulate else self.slot_tables.data_ptr(), int(simulate),
                                     -1 if shared_host_layers else 0)
        h = _lib.u64()
        _lib.call("mtp_prefetch_session_create", C.byref(cfg), C.byref(h))
        self.handle = h.value

    @staticmethod
    def _ids(experts):
        import numpy as np
        a = np.ascontiguousarray(np.asarray(experts, dtype=np.int32).reshape(-1))
        return a, a.ctypes.data_as(C.c_void_p)

    def issue(self, layer: int, experts) -> int:
        a, p = self._ids(experts)
        out = i32_()
        _lib.call("mtp_prefetch_issue", self.handle, layer, p, a.size, C.byref(out))
        return out.value

    def demand(self, layer: int, experts, insert_on_miss: bool = True) -> int:
        a, p = self._ids(experts)
        out = i32_()
        _lib.call("mtp_prefetch_demand", self.handle, layer, p, a.size, int(insert_on_miss), C.byref(out))
        return out.value

    def wait(self, layer: int, experts, stream: torch.cuda.Stream | None = None):
        """Make ``stream`` wait for the in-flight copies of these experts."""
        a, p = self._ids(experts)
        st = stream if stream is not None else torch.cuda.current_stream()
        _lib.call("mtp_prefetch_wait", self.handle, layer, p, a.size, C.c_void_p(st.cuda_stream))

    def layer_used(self, layer: int, stream: torch.cuda.Stream | None = None):
        st = stream if stream is not None else torch.cuda.current_stream()
        _lib.call("mtp_prefetch_layer_used", self.handle, layer, C.c_void_p(st.cuda_stream))

    def poll(self) -> dict:
        out = _lib.MtpPrefetchStats()
        _lib.call("mtp_prefetch_poll", self.handle, C.byref(out))
        return {name: getattr(out, name) for name, _ in out._fields_}

    def sync(self):
        _lib.call("mtp_prefetch_sync", self.handle)

    def layer_views(self, layer: int):
        """(expert_blobs, slot_table, host_blobs) of one layer, for moe_layer_w4a16."""
        s0 = layer * self.slots * self.expert_bytes
        e0 = 0 if self.shared_host_layers else layer * self.num_experts * self.expert_bytes
        return (self.cache[s0:s0 + self.slots * self.expert_bytes], self.slot_tables[layer],
                self.host_store.reshape(-1)[e0:e0 + self.num_experts * self.expert_bytes])

    def close(self):
        if getattr(self, "handle", 0):
            _lib.call("mtp_prefetch_session_destroy", self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


i32_ = C.c_int32
