"""ctypes binding of libdsca_b200.so (include/dsca_b200.h).

The library is the only compute path: if it is missing or the device is not an sm_100 part,
every call raises; there is no CPU or eager-PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "lib", "libdsca_b200.so")

# status codes / enums (include/dsca_b200.h)
OK, ERR_BAD_ARG, ERR_CAPACITY, ERR_WAIT_TIMEOUT, ERR_CUDA, ERR_DEVICE_INDEX, ERR_UNSUPPORTED = range(7)
F32, BF16, F8E4M3 = 0, 1, 2
ROUTE_SWITCH_TOP1, ROUTE_SOFTMAX_TOPK = 0, 1
ACT_RELU, ACT_SWIGLU = 0, 1
ROUTER_TOKENS = 32
MAX_EXPERTS = 64
MAX_TOPK = 8

_vp = ctypes.c_void_p
_i = ctypes.c_int


class RouterArgs(ctypes.Structure):
    _fields_ = [("x", _vp), ("w_router", _vp), ("w_shared_gate", _vp),
                ("T", _i), ("d", _i), ("E", _i), ("top_k", _i), ("dtype", _i), ("mode", _i),
                ("norm_topk", _i), ("weight_round_bf16", _i),
                ("logits", _vp), ("topk_ids", _vp), ("topk_w", _vp), ("expert_index", _vp),
                ("shared_gate", _vp), ("block_hist", _vp), ("local_rank", _vp),
                ("counts", _vp), ("offsets", _vp), ("block_base", _vp), ("done_counter", _vp),
                ("w_slices", _vp), ("w_exp", _vp), ("x_slices", _vp), ("x_exp", _vp), ("logits_f32", _vp),
                ("err", _vp), ("first_counts", _vp)]


class ScanArgs(ctypes.Structure):
    _fields_ = [("block_hist", _vp), ("nblocks", _i), ("E", _i), ("counts", _vp), ("offsets", _vp),
                ("block_base", _vp)]


class PermuteArgs(ctypes.Structure):
    _fields_ = [("x", _vp), ("T", _i), ("d", _i), ("E", _i), ("top_k", _i), ("dtype", _i),
                ("topk_ids", _vp), ("local_rank", _vp), ("block_base", _vp), ("offsets", _vp),
                ("G", _i), ("cum_split", _vp), ("dest_base", _vp), ("capacity", _i), ("out", _vp),
                ("token_row", _vp), ("err", _vp), ("out_f16", _i), ("x_f16", _vp),
                ("out_e4m3", _i), ("out_scale", _vp), ("x_q", _vp), ("x_scale", _vp)]


class SplitArgs(ctypes.Structure):
    _fields_ = [("src", _vp), ("ld", _i), ("rows", _i), ("K", _i), ("rows_dev", _vp), ("dst", _vp),
                ("inv_scale", _vp)]


class FfnArgs(ctypes.Structure):
    _fields_ = [("dtype", _i), ("act", _i), ("d", _i), ("n1p", _i), ("ip", _i), ("dp", _i),
                ("num_groups", _i), ("group_offsets", _vp), ("group_weight", _vp),
                ("num_experts_w", _i), ("capacity", _i), ("a", _vp), ("w1", _vp), ("w2", _vp),
                ("h", _vp), ("y", _vp), ("shared_rows", _i), ("shared_n1p", _i), ("shared_ip", _i),
                ("xs", _vp), ("ws1", _vp), ("ws2", _vp), ("hs", _vp), ("ys", _vp), ("err", _vp),
                ("num_ctas", _i), ("phases", _i), ("ep_ctx", _vp), ("segments", _i),
                ("w1_scale", _vp), ("w2_scale", _vp), ("ws1_scale", _vp), ("ws2_scale", _vp),
                ("tile_rows", _i), ("pdl_after_permute", _i), ("group_order", _vp), ("cache_hints", _i), ("tile_order", _i),
                ("f8_split", _i), ("a_scale", _vp), ("xs_scale", _vp), ("hq", _vp), ("hsq", _vp), ("h_scale", _vp),
                ("hs_scale", _vp), ("tile_counters", _vp), ("shared_handoff", _i)]


MAX_GPUS = 8


class EpSetup(ctypes.Structure):
    _fields_ = [("G", _i), ("E", _i), ("me", _i), ("d", _i), ("elem_bytes", _i),
                ("recv_capacity", _i), ("ret_capacity", _i), ("eq_tokens", _i), ("start_epoch", ctypes.c_uint),
                ("expert_to_gpu", _vp), ("flags", _vp * MAX_GPUS), ("meta", _vp * MAX_GPUS),
                ("recv", _vp * MAX_GPUS), ("ret", _vp * MAX_GPUS)]


class EpDispatchArgs(ctypes.Structure):
    _fields_ = [("x", _vp), ("T", _i), ("d", _i), ("top_k", _i), ("dtype", _i), ("topk_ids", _vp),
                ("local_rank", _vp), ("block_base", _vp), ("ctx", _vp), ("token_row", _vp), ("err", _vp),
                ("out_f16", _i), ("x_f16", _vp)]


class CombineArgs(ctypes.Structure):
    _fields_ = [("T", _i), ("d", _i), ("top_k", _i), ("dtype", _i), ("y", _vp), ("token_row", _vp),
                ("topk_w", _vp), ("ys", _vp), ("shared_gate", _vp), ("rows", _i), ("out", _vp),
                ("err", _vp), ("pdl", _i)]


class QosArgs(ctypes.Structure):
    _fields_ = [("x", _vp), ("x_prev", _vp), ("logits", _vp), ("dtype", _i), ("topk_ids", _vp),
                ("seq_priority", _vp), ("remaining", _vp), ("valid", _vp), ("T", _i), ("d", _i), ("E", _i),
                ("top_k", _i), ("attention_mode", _i), ("alpha", ctypes.c_float), ("beta", ctypes.c_float),
                ("delta", ctypes.c_float), ("target_batch", ctypes.c_float), ("epsilon", ctypes.c_float),
                ("token_score", _vp), ("expert_priority", _vp), ("err", _vp),
                ("first_counts", _vp), ("partial", _vp), ("done_counter", _vp)]


# every symbol include/dsca_b200.h declares
EXPORTED = ["dsca_version", "dsca_status_string", "dsca_device_info", "dsca_router_topk",
            "dsca_dispatch_scan", "dsca_permute", "dsca_grouped_ffn", "dsca_combine",
            "dsca_plan_harmony", "dsca_plan_layout", "dsca_check_error", "dsca_exp_neg_eval",
            "dsca_grouped_ffn_static_scratch", "dsca_ep_ctx_bytes", "dsca_ep_init", "dsca_ep_group_offsets",
            "dsca_ep_plan", "dsca_ep_plan_counts", "dsca_ep_priority", "dsca_ep_group_order", "dsca_ep_dispatch", "dsca_ep_wait", "dsca_ep_plan_eval", "dsca_ipc_export",
            "dsca_ipc_import", "dsca_ipc_close", "dsca_ep_read_plan", "dsca_ep_region_alloc",
            "dsca_ep_region_free", "dsca_ep_return", "dsca_qos_priority", "dsca_router_pack_i8", "dsca_split_rows"]
STATIC_SCRATCH_BYTES = 16 << 20

_LIB = None


class DscaError(RuntimeError):
    def __init__(self, code: int, where: str):
        self.code = code
        super().__init__(f"{where}: dsca status {code} ({status_string(code)})")


def load():
    """Load the library (raises if it has not been built)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"libdsca_b200.so not found at {LIB_PATH}: run `python -m dsca_moe_b200.build` "
                           "(there is no fallback path)")
    lib = ctypes.CDLL(LIB_PATH)
    p = ctypes.POINTER
    lib.dsca_version.restype = ctypes.c_char_p
    lib.dsca_status_string.restype = ctypes.c_char_p
    lib.dsca_status_string.argtypes = [_i]
    lib.dsca_device_info.argtypes = [p(_i), p(_i)]
    lib.dsca_router_topk.argtypes = [p(RouterArgs), _vp]
    lib.dsca_dispatch_scan.argtypes = [p(ScanArgs), _vp]
    lib.dsca_permute.argtypes = [p(PermuteArgs), _vp]
    lib.dsca_split_rows.argtypes = [p(SplitArgs), _vp]
    lib.dsca_grouped_ffn.argtypes = [p(FfnArgs), _vp]
    lib.dsca_grouped_ffn_static_scratch.argtypes = [p(FfnArgs), _vp]
    u64 = ctypes.c_uint64
    lib.dsca_ep_ctx_bytes.restype = ctypes.c_size_t
    lib.dsca_ep_ctx_bytes.argtypes = []
    lib.dsca_ep_init.argtypes = [_vp, p(EpSetup), _vp]
    lib.dsca_ep_group_offsets.restype = _vp
    lib.dsca_ep_group_offsets.argtypes = [_vp]
    lib.dsca_ep_group_order.restype = _vp
    lib.dsca_ep_group_order.argtypes = [_vp]
    lib.dsca_ep_plan.argtypes = [_vp, _vp, _vp, u64, _vp, _vp]
    lib.dsca_ep_plan_counts.argtypes = [_vp, _vp, u64, _vp, _vp]
    lib.dsca_ep_priority.argtypes = [_vp, _vp, u64, _vp, _vp]
    lib.dsca_ep_dispatch.argtypes = [p(EpDispatchArgs), _vp]
    lib.dsca_ep_wait.argtypes = [_vp, _i, u64, _vp, _vp]
    lib.dsca_ep_plan_eval.argtypes = [_vp, _i, _i, _vp, _i, _vp, _vp]
    lib.dsca_ipc_export.argtypes = [_vp, _vp, p(ctypes.c_size_t)]
    lib.dsca_ipc_import.argtypes = [_vp, ctypes.c_size_t, p(_vp)]
    lib.dsca_ipc_close.argtypes = [_vp, ctypes.c_size_t]
    lib.dsca_ep_read_plan.argtypes = [_vp, _vp, _vp, _vp]
    lib.dsca_ep_region_alloc.argtypes = [ctypes.c_size_t, p(_vp)]
    lib.dsca_ep_region_free.argtypes = [_vp]
    lib.dsca_ep_return.argtypes = [_vp, _vp, _i, _i, _i, _vp, _vp]
    lib.dsca_combine.argtypes = [p(CombineArgs), _vp]
    lib.dsca_qos_priority.argtypes = [p(QosArgs), _vp]
    lib.dsca_router_pack_i8.argtypes = [_vp, _i, _i, _vp, _vp, _vp]
    lib.dsca_plan_harmony.argtypes = [_vp, _i, _i, _vp, _i, _vp]
    lib.dsca_plan_layout.argtypes = [_vp, _i, _i, _i, p(_i), _vp, _vp, _vp, _vp, _vp, _vp, _vp]
    lib.dsca_check_error.argtypes = [_vp, _vp]
    lib.dsca_exp_neg_eval.argtypes = [_vp, _vp, _i, _vp]
    for name in EXPORTED:
        getattr(lib, name).restype = getattr(lib, name).restype or _i
    lib.dsca_version.restype = ctypes.c_char_p
    lib.dsca_status_string.restype = ctypes.c_char_p
    _LIB = lib
    return lib


def status_string(code: int) -> str:
    try:
        return load().dsca_status_string(code).decode()
    except Exception:  # noqa: BLE001 - only used to format an error message
        return "?"


def check(code: int, where: str):
    if code != OK:
        raise DscaError(code, where)


def call(name: str, *args):
    check(getattr(load(), name)(*args), name)
