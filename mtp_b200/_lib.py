"""ctypes binding of libmtp_b200.so (the C ABI declared in include/mtp_b200.h).

The library is loaded from the package's ``lib/`` directory, where
``python -m mtp_b200.build`` (or ``__graft_entry__.build()``) puts it. There is
no fallback: if the library is missing or does not load, every operation
raises.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libmtp_b200.so"

# Every symbol include/mtp_b200.h declares (checked by the tests).
EXPORTS = (
    "mtp_status_string",
    "mtp_abi_version",
    "mtp_host_device_pointer",
    "mtp_router_topk",
    "mtp_moe_align_sizes",
    "mtp_moe_align",
    "mtp_gptq_dequant",
    "mtp_w4a16_expert_layout",
    "mtp_w4a16_repack_gptq",
    "mtp_w4a16_moe_layer_workspace_size",
    "mtp_w4a16_moe_layer",
    "mtp_w4a16_moe_layer_timeouts",
    "mtp_w4a16_moe_layer_noalloc",
    "mtp_w4a16_moe_prefill_workspace_size",
    "mtp_w4a16_moe_prefill",
    "mtp_w4a16_moe_prefill_tables",
    "mtp_predictor_pack",
    "mtp_predictor_workspace_size",
    "mtp_predict_topk",
    "mtp_predictor_hr_workspace_size",
    "mtp_predict_topk_hidden_residual",
    "mtp_prefetch_session_create",
    "mtp_prefetch_session_destroy",
    "mtp_prefetch_issue",
    "mtp_prefetch_layer_used",
    "mtp_prefetch_demand",
    "mtp_prefetch_wait",
    "mtp_prefetch_poll",
    "mtp_prefetch_sync",
)

MTP_ZERO_RAW = 0
MTP_ZERO_SYM8 = 1

vp = C.c_void_p
i32 = C.c_int32
i64 = C.c_int64


class MtpExpertLayout(C.Structure):
    _fields_ = [("w13_qweight", i64), ("w13_scales", i64), ("w13_zeros", i64),
                ("w2_qweight", i64), ("w2_scales", i64), ("w2_zeros", i64), ("bytes", i64)]


class MtpMoeLayerArgs(C.Structure):
    _fields_ = [
        ("num_tokens", i32), ("hidden", i32), ("inter", i32), ("num_experts", i32),
        ("top_k", i32), ("group_size", i32), ("renormalize", i32), ("zero_mode", i32),
        ("hidden_states", vp), ("router_logits", vp), ("topk_weights", vp), ("topk_ids", vp),
        ("expert_blobs", vp), ("expert_bytes", i64), ("slot_table", vp), ("host_blobs", vp),
        ("shared_blob", vp), ("shared_gate_weight", vp), ("out", vp), ("out_f32", vp),
        ("topk_weights_out", vp), ("topk_ids_out", vp), ("demand_log", vp), ("status", vp),
        ("workspace", vp), ("workspace_bytes", i64),
        ("expert_map", vp), ("global_num_experts", i32), ("shared_rows_begin", i32), ("shared_rows_end", i32),
    ]


class MtpPrefillTables(C.Structure):
    _fields_ = [("pair_expert_ids", i64), ("sorted_token_ids", i64), ("expert_ids", i64),
                ("num_tokens_post_padded", i64), ("capacity", i32), ("max_blocks", i32),
                ("pairs_per_token", i32), ("block_size", i32)]


class MtpPrefetchConfig(C.Structure):
    _fields_ = [("device", i32), ("num_layers", i32), ("num_experts", i32), ("slots_per_layer", i32),
                ("expert_bytes", i64), ("host_store", vp), ("cache_base", vp), ("slot_tables", vp),
                ("simulate", i32), ("host_layer_stride", i64)]


class MtpPrefetchStats(C.Structure):
    _fields_ = [(n, i64) for n in (
        "issued_fetch_count", "used_fetch_count", "unused_fetch_count", "demand_count", "demand_hit_count",
        "demand_miss_count", "evicted_before_use_count", "ready_late_miss_count", "inflight_count",
        "resident_count", "bytes_copied")]


u64 = C.c_uint64

_SIGS = {
    "mtp_status_string": (C.c_char_p, [C.c_int]),
    "mtp_abi_version": (C.c_int, []),
    "mtp_host_device_pointer": (C.c_int, [vp, C.POINTER(vp)]),
    "mtp_router_topk": (C.c_int, [vp, i32, i32, i32, i32, vp, vp, vp, vp]),
    "mtp_moe_align_sizes": (C.c_int, [i32, i32, i32, i32, C.POINTER(i32), C.POINTER(i32), C.POINTER(i32)]),
    "mtp_moe_align": (C.c_int, [vp, i32, i32, i32, vp, i32, i32, vp, vp, vp, vp, vp, vp]),
    "mtp_gptq_dequant": (C.c_int, [vp, vp, vp, vp, i32, i32, i32, i32, vp, vp]),
    "mtp_w4a16_expert_layout": (C.c_int, [i32, i32, i32, C.POINTER(MtpExpertLayout)]),
    "mtp_w4a16_repack_gptq": (C.c_int, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp, vp]),
    "mtp_w4a16_moe_layer_workspace_size": (C.c_int, [i32, i32, i32, i32, i32, C.POINTER(i64)]),
    "mtp_w4a16_moe_layer": (C.c_int, [C.POINTER(MtpMoeLayerArgs), vp]),
    "mtp_w4a16_moe_layer_noalloc": (C.c_int, [C.POINTER(MtpMoeLayerArgs), vp]),
    "mtp_w4a16_moe_layer_timeouts": (C.c_int, [vp, C.POINTER(i32), vp]),
    "mtp_w4a16_moe_prefill_tables": (C.c_int, [i32, i32, i32, i32, i32, i32, C.POINTER(MtpPrefillTables)]),
    "mtp_w4a16_moe_prefill_workspace_size": (C.c_int, [i32, i32, i32, i32, i32, C.POINTER(i64)]),
    "mtp_w4a16_moe_prefill": (C.c_int, [C.POINTER(MtpMoeLayerArgs), vp]),
    "mtp_predictor_pack": (C.c_int, [vp, i32, i32, vp, vp]),
    "mtp_predictor_workspace_size": (C.c_int, [i32, i32, i32, i32, C.POINTER(i64)]),
    "mtp_predict_topk": (C.c_int, [vp, i32, i32, vp, vp, i32, vp, vp, i32, i32, i32, vp, vp, vp, i64, vp]),
    "mtp_predictor_hr_workspace_size": (C.c_int, [i32, i32, i32, i32, C.POINTER(i64)]),
    "mtp_predict_topk_hidden_residual": (C.c_int, [vp, vp, i32, i32, vp, vp, i32, vp, vp, C.c_float, vp, i32, vp,
                                                   i32, vp, vp, i32, i32, vp, vp, vp, i64, vp]),
    "mtp_prefetch_session_create": (C.c_int, [C.POINTER(MtpPrefetchConfig), C.POINTER(u64)]),
    "mtp_prefetch_session_destroy": (C.c_int, [u64]),
    "mtp_prefetch_issue": (C.c_int, [u64, i32, vp, i32, C.POINTER(i32)]),
    "mtp_prefetch_layer_used": (C.c_int, [u64, i32, vp]),
    "mtp_prefetch_demand": (C.c_int, [u64, i32, vp, i32, i32, C.POINTER(i32)]),
    "mtp_prefetch_wait": (C.c_int, [u64, i32, vp, i32, vp]),
    "mtp_prefetch_poll": (C.c_int, [u64, C.POINTER(MtpPrefetchStats)]),
    "mtp_prefetch_sync": (C.c_int, [u64]),
}

_lock = threading.Lock()
_lib = None


class MtpError(RuntimeError):
    def __init__(self, fn: str, status: int, message: str):
        super().__init__(f"{fn} failed with status {status}: {message}")
        self.status = status


def load() -> C.CDLL:
    """Load (once) and return the library; raises if it is absent."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m mtp_b200.build` "
                    "(there is no CPU fallback for mtp_b200 operations)")
            lib = C.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGS.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
        return _lib


def call(name: str, *args) -> None:
    lib = load()
    status = getattr(lib, name)(*args)
    if status != 0:
        msg = lib.mtp_status_string(status).decode()
        raise MtpError(name, status, msg)


def expert_layout(hidden: int, inter: int, group_size: int) -> MtpExpertLayout:
    out = MtpExpertLayout()
    call("mtp_w4a16_expert_layout", hidden, inter, group_size, C.byref(out))
    return out


def align_sizes(numel: int, num_experts: int, block_size: int, pad_sorted_ids: bool = False):
    cap, blocks, segs = i32(), i32(), i32()
    call("mtp_moe_align_sizes", numel, num_experts, block_size, int(pad_sorted_ids),
         C.byref(cap), C.byref(blocks), C.byref(segs))
    return cap.value, blocks.value, segs.value


def layer_workspace_bytes(m: int, e: int, k: int, hidden: int, inter: int) -> int:
    out = i64()
    call("mtp_w4a16_moe_layer_workspace_size", m, e, k, hidden, inter, C.byref(out))
    return out.value


def prefill_tables(m: int, e: int, k: int, hidden: int, inter: int, has_shared: bool) -> MtpPrefillTables:
    out = MtpPrefillTables()
    call("mtp_w4a16_moe_prefill_tables", m, e, k, hidden, inter, int(has_shared), C.byref(out))
    return out


def prefill_workspace_bytes(m: int, e: int, k: int, hidden: int, inter: int) -> int:
    out = i64()
    call("mtp_w4a16_moe_prefill_workspace_size", m, e, k, hidden, inter, C.byref(out))
    return out.value


def host_device_pointer(host_ptr: int) -> int:
    """Device address of a pinned host buffer (cudaHostGetDevicePointer)."""
    out = vp()
    call("mtp_host_device_pointer", vp(host_ptr), C.byref(out))
    return int(out.value)


def predictor_workspace_bytes(m: int, width: int, future: int, experts: int) -> int:
    out = i64()
    call("mtp_predictor_workspace_size", m, width, future, experts, C.byref(out))
    return out.value
