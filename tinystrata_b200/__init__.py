"""tinystrata_b200 - TinyStrata's MoE expert-layer path on B200 (sm_100a).

The product is ``libtsb_moe.so`` (C ABI in include/tsb_moe.h).  This module is the host-side mirror of the reference's
expert-layer entry points over that ABI (same names, argument meaning and error behaviour: a failing call raises
``TsbError`` where the reference throws or exits), taking torch CUDA tensors for device memory and streams.  There is no
CPU fallback: without the built library every call raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtsb_moe.so")

T_Q4_0, T_Q8_0, T_Q4_K, T_Q6_K, T_IQ3_XXS, T_IQ3_S = 2, 8, 12, 14, 18, 21
ACT_SWIGLU, ACT_GELU_TANH, ACT_SWIGLU_CLAMP = 0, 1, 2
Q8_1_BYTES = 36


class TsbError(RuntimeError):
    pass


class GgufTensorInfo(C.Structure):
    """tsb_gguf_tensor_info: a tensor of a mapped GGUF file."""
    _fields_ = [("type", C.c_int32), ("n_dims", C.c_int32), ("ne", C.c_int64 * 4), ("bytes", C.c_uint64),
                ("data", C.c_void_p)]


class MmvqSlots(C.Structure):
    """tsb_mmvq_slots (the reference's MmvqSlots, include/strata/gemma4/matvec.hpp:149-153)."""
    _fields_ = [("w", C.c_void_p * 32), ("x", C.c_void_p * 32), ("y", C.c_void_p * 32)]


class MmvqIds(C.Structure):
    """tsb_mmvq_ids (the reference's MmvqIds, include/strata/gemma4/matvec.hpp:158-167)."""
    _fields_ = [("table", C.c_void_p), ("ids", C.c_void_p), ("offset", C.c_uint64), ("x", C.c_void_p),
                ("x_stride", C.c_uint64), ("x_every", C.c_int32), ("y", C.c_void_p), ("y_stride", C.c_uint64)]


class DecodeLayer(C.Structure):
    """tsb_decode_layer: device pointers of one layer for the fused decode path."""
    _fields_ = [("blobs", C.c_void_p), ("router", C.c_void_p), ("sh_blob", C.c_void_p), ("logit_prior", C.c_void_p)]


class DecodeDesc(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("n_layers", C.c_int32), ("n_tok", C.c_int32), ("n_embd", C.c_int32),
                ("n_ff", C.c_int32), ("n_expert", C.c_int32), ("n_used", C.c_int32), ("sh_n_ff", C.c_int32),
                ("gu_type", C.c_int32), ("d_type", C.c_int32), ("sh_gu_type", C.c_int32), ("sh_d_type", C.c_int32),
                ("eps", C.c_float)]


class DecodeActDesc(C.Structure):
    """tsb_decode_act_desc: the Gemma 4 / LFM2 decode MoE block of one launch."""
    _fields_ = [("struct_size", C.c_uint32), ("n_tok", C.c_int32), ("n_embd", C.c_int32), ("n_ff", C.c_int32),
                ("n_expert", C.c_int32), ("n_used", C.c_int32), ("sh_n_ff", C.c_int32), ("gu_type", C.c_int32),
                ("d_type", C.c_int32), ("act", C.c_int32), ("sh_act", C.c_int32), ("limit", C.c_float),
                ("gate", C.c_int32), ("in_scale", C.c_float), ("norm", C.c_int32), ("w_scale", C.c_float)]


class ExpertLayout(C.Structure):
    """tsb_expert_layout (the reference's NativeExpertLayout, iq_kernels.hpp:45-53)."""
    _fields_ = [("gu_type", C.c_int32), ("d_type", C.c_int32), ("n_embd", C.c_int64), ("n_ff", C.c_int64),
                ("gu_row", C.c_uint64), ("d_row", C.c_uint64), ("up_off", C.c_uint64), ("down_off", C.c_uint64),
                ("bytes", C.c_uint64)]


_lib = None
_lock = threading.Lock()
_p, _i32, _i64, _u64, _f = C.c_void_p, C.c_int32, C.c_int64, C.c_uint64, C.c_float

# name -> (restype, argtypes); every symbol of include/tsb_moe.h
SIGNATURES = {
    "tsb_moe_abi_version": (C.c_int, []),
    "tsb_last_error": (C.c_char_p, []),
    "tsb_device_error": (C.c_int, [C.POINTER(C.c_uint), C.c_int]),
    "tsb_type_supported": (C.c_int, [C.c_int]),
    "tsb_row_bytes": (_i64, [C.c_int, _i64]),
    "tsb_native_expert_layout": (C.c_int, [C.c_int, C.c_int, _i64, _i64, C.POINTER(ExpertLayout)]),
    "tsb_native_expert_supported": (C.c_int, [C.c_int, C.c_int, _i64, _i64]),
    "tsb_native_expert_scratch_bytes": (_u64, [_i64, _i64]),
    "tsb_quantize_q8_1_rows": (C.c_int, [_p, _i64, _i64, _p, _p]),
    "tsb_router_logits_f32": (C.c_int, [_p, _p, _p, C.c_int, C.c_int, C.c_int, C.c_int, _p]),
    "tsb_native_router_topk": (C.c_int, [_p, _p, _p, C.c_int, C.c_int, C.c_int, C.c_int, _p]),
    "tsb_route_rows": (C.c_int, [_p, C.c_int, C.c_int, C.c_int, C.c_int, _f, _p, _p, C.c_int, _f, _p, _p, _p]),
    "tsb_moe_group": (C.c_int, [_p, C.c_int, C.c_int, C.c_int, _p, _u64, _p, _p, _p, _p, _p, _p]),
    "tsb_native_expert_grouped": (C.c_int, [C.POINTER(ExpertLayout), _p, _p, _p, _p, _p, _i64, _i64, _p, _p, _p, _p,
                                            _i64]),
    "tsb_native_expert_grouped_act": (C.c_int, [C.POINTER(ExpertLayout), _p, _p, _p, _p, _p, _i64, _i64, _p, _p, _p,
                                                C.c_int, _f, _p]),
    "tsb_moe_dispatch": (C.c_int, [_p, C.c_int, C.c_int, C.c_int, _p, _p, _p, _p, _p]),
    "tsb_mmq_act_bytes": (_u64, [_i64, _i64]),
    "tsb_mmq_quantize": (C.c_int, [_p, _i64, _p, C.c_int, C.c_int, _p, _p]),
    "tsb_mmq_from_q8_1": (C.c_int, [_p, _p, C.c_int, C.c_int, _p, _p]),
    "tsb_moe_prefill_gu": (C.c_int, [C.POINTER(ExpertLayout), _p, _u64, _p, C.c_int, C.c_int, _p, _p, C.c_int, _f,
                                     _p]),
    "tsb_moe_prefill_down": (C.c_int, [C.POINTER(ExpertLayout), _p, _u64, _p, C.c_int, C.c_int, _p, _p, _p]),
    "tsb_debug_mmq_block_sums": (C.c_int, [C.POINTER(ExpertLayout), C.c_int, _p, C.c_int, _p, _p, _p, _p, _p]),
    "tsb_native_expert_grouped_noalloc": (C.c_int, [C.POINTER(ExpertLayout), _p, _p, _p, _p, _p, _i64, _i64, _p, _p,
                                                    _p]),
    "tsb_moe_combine": (C.c_int, [_p, _p, _p, _p, C.c_int, _p, _p, C.c_int, _p, _p, _p, C.c_int, _f, C.c_int, _p]),
    "tsb_moe_sum": (C.c_int, [_p, _p, _p, C.c_int, C.c_int, C.c_int, _p]),
    "tsb_rms_norm_q8_1": (C.c_int, [_p, _p, _p, _p, C.c_int, _f, C.c_int, _p]),
    "tsb_native_expert_set_phase": (C.c_int, [C.c_int]),
    "tsb_debug_row_calls": (C.c_int, [C.c_int, _p, _p, _i64, _p, _p, _p]),
    "tsb_moe_decode_workspace_bytes": (_u64, [C.POINTER(DecodeDesc)]),
    "tsb_moe_decode_layers": (C.c_int, [C.POINTER(DecodeDesc), _p, _p, _p, _p, _p, _p, _u64, _p]),
    "tsb_moe_decode_error": (C.c_int, [C.POINTER(DecodeDesc), _p, _p]),
    "tsb_decode_last_error": (C.c_char_p, []),
    "tsb_moe_decode_set_trace": (C.c_int, [_p]),
    "tsb_moe_decode_set_debug": (C.c_int, [C.c_int]),
    "tsb_add_scaled": (C.c_int, [_p, C.c_int, C.c_int, _p]),
    "tsb_mmq_product": (C.c_int, [_p, C.c_int, _i64, _i64, C.c_uint64, C.c_int, _p, _p, _p, _i64, _p, _i64, _p]),
    "tsb_gguf_open": (C.c_int, [C.c_char_p, C.POINTER(C.c_void_p)]),
    "tsb_gguf_close": (C.c_int, [_p]),
    "tsb_gguf_tensor_count": (C.c_int, [_p]),
    "tsb_gguf_tensor_name": (C.c_int, [_p, C.c_int, C.c_char_p, C.c_int]),
    "tsb_gguf_tensor": (C.c_int, [_p, C.c_char_p, C.POINTER(GgufTensorInfo)]),
    "tsb_gguf_kv_int": (C.c_int, [_p, C.c_char_p, C.POINTER(_i64)]),
    "tsb_gguf_kv_float": (C.c_int, [_p, C.c_char_p, C.POINTER(C.c_double)]),
    "tsb_gguf_kv_str": (C.c_int, [_p, C.c_char_p, C.c_char_p, C.c_int]),
    "tsb_gguf_expert_layer": (C.c_int, [_p, C.c_char_p, C.POINTER(ExpertLayout), C.POINTER(C.c_uint64),
                                        C.POINTER(C.c_int32)]),
    "tsb_gguf_repack_experts": (C.c_int, [_p, C.c_char_p, C.c_int, C.c_int, _p, C.c_uint64]),
    "tsb_mmvq_supported": (C.c_int, [C.c_int]),
    "tsb_mmvq_run_slots": (C.c_int, [C.c_int, C.POINTER(MmvqSlots), C.c_int, C.c_int, C.c_int, _p]),
    "tsb_mmvq_run_ids": (C.c_int, [C.c_int, C.POINTER(MmvqIds), C.c_int, C.c_int, C.c_int, _p]),
    "tsb_ep_unique_id": (C.c_int, [_p]),
    "tsb_ep_create": (C.c_int, [_p, C.c_int, C.c_int, C.POINTER(ExpertLayout), _p, C.c_uint64, C.c_int, C.c_int,
                                C.c_int, C.c_int, C.c_int, _f, C.POINTER(C.c_void_p)]),
    "tsb_ep_set_timeout_ns": (C.c_int, [_p, C.c_uint64]),
    "tsb_ep_dispatch": (C.c_int, [_p, _p, _p, _p, C.c_int, C.c_int, _p]),
    "tsb_ep_combine": (C.c_int, [_p, _p, C.c_int, _p, _p, C.c_int, C.c_int, _p]),
    "tsb_ep_stats": (C.c_int, [_p, C.POINTER(_i64), C.POINTER(_i64), C.POINTER(_i64)]),
    "tsb_ep_synchronize": (C.c_int, [_p]),
    "tsb_ep_destroy": (C.c_int, [_p]),
    "tsb_moe_layer_tail": (C.c_int, [_p, _p, _p, _p, _p, _f, C.c_int, C.c_int, _f, _p]),
    "tsb_set_wait_limit_ns": (C.c_int, [_u64]),
    "tsb_moe_decode_act_workspace_bytes": (_u64, [C.POINTER(DecodeActDesc)]),
    "tsb_moe_decode_act_set_trace": (C.c_int, [_p]),
    "tsb_moe_decode_act": (C.c_int, [C.POINTER(DecodeActDesc), _p, _p, _p, _p, _p, _p, _u64, _p, _p, C.c_int, _p, _p,
                                     _p, _p, _u64, _p]),
    "tsb_moe_group_staged": (C.c_int, [_p, C.c_int, C.c_int, C.c_int, _p, C.c_int, _p, _p, _u64, _p, C.c_int, _p, _p,
                                       _p, _p, _p, _p, _p]),
    "tsb_staged_rebalance": (C.c_int, [_p, C.c_int, C.c_int, _p, _p, C.c_int, _p, _p]),
    "tsb_staged_load": (C.c_int, [_p, _p, _u64, _u64, _p, _p, C.c_int, C.c_int, C.c_int, _p]),
    "tsb_stage_layer": (C.c_int, [_p, C.c_int, C.c_int, _p, _p, _u64, _p, C.c_int, _p]),
}


def lib():
    """The loaded libtsb_moe.so (raises when it has not been built: there is no fallback)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise TsbError(f"{LIB_PATH} is missing: run `python -m tinystrata_b200.build` (no CPU fallback)")
            L = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name, None)
                if fn is None:
                    continue
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def last_error() -> str:
    return lib().tsb_last_error().decode()


def _check(rc: int, what: str):
    if rc != 0:
        raise TsbError(f"{what}: status {rc}: {last_error()}")


def _ptr(t):
    if t is None:
        return None
    return C.c_void_p(t.data_ptr())


def _stream(stream):
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return C.c_void_p(stream.cuda_stream)


# ------------------------------------------------------------------------------------------------ formats
def row_bytes(ggml_type: int, n: int) -> int:
    return int(lib().tsb_row_bytes(ggml_type, n))


def native_expert_layout(gu_type: int, d_type: int, n_embd: int, n_ff: int) -> ExpertLayout:
    L = ExpertLayout()
    _check(lib().tsb_native_expert_layout(gu_type, d_type, n_embd, n_ff, C.byref(L)), "native_expert_layout")
    return L


def native_expert_supported(gu_type, d_type, n_embd, n_ff) -> bool:
    return bool(lib().tsb_native_expert_supported(gu_type, d_type, n_embd, n_ff))


def native_expert_scratch_bytes(cap_entries: int, n_ff: int) -> int:
    return int(lib().tsb_native_expert_scratch_bytes(cap_entries, n_ff))


# ------------------------------------------------------------------------------------------------ entry points
def quantize_q8_1_rows(x, y=None, stream=None):
    """fp32 [rows, n] -> q8_1 uint8 [rows, n / 32 * 36] (quantize_q8_1_rows, iq_kernels.hpp:24)."""
    import torch
    rows, n = x.shape
    if y is None:
        y = torch.empty((rows, n // 32 * Q8_1_BYTES), dtype=torch.uint8, device=x.device)
    _check(lib().tsb_quantize_q8_1_rows(_ptr(x), rows, n, _ptr(y), _stream(stream)), "quantize_q8_1_rows")
    return y


def router_logits_f32(W, h, logits=None, ld=None, stream=None):
    import torch
    n_out, n_in = W.shape
    T = h.shape[0]
    ld = ld or n_out
    if logits is None:
        logits = torch.empty((T, ld), dtype=torch.float32, device=h.device)
    _check(lib().tsb_router_logits_f32(_ptr(W), _ptr(h), _ptr(logits), n_in, n_out, T, ld, _stream(stream)),
           "router_logits_f32")
    return logits


def native_router_topk(logits, k: int, n_expert: int | None = None, ids=None, w=None, stream=None):
    """Softmax top-k (native_router_topk, native_router.hpp:5-6); logits [T, ld >= n_expert]."""
    import torch
    T, ld = logits.shape
    n_expert = n_expert or ld
    ids = ids if ids is not None else torch.empty((T, k), dtype=torch.int32, device=logits.device)
    w = w if w is not None else torch.empty((T, k), dtype=torch.float32, device=logits.device)
    _check(lib().tsb_native_router_topk(_ptr(logits), _ptr(ids), _ptr(w), n_expert, k, T, ld, _stream(stream)),
           "native_router_topk")
    return ids, w


def route_rows(logits, n_used, gate, in_scale=1.0, bias=None, escale=None, norm=True, w_scale=0.0, stream=None):
    """Gemma 4 / LFM2 routing (route_rows, gemma4/kernels.cu:289-356)."""
    import torch
    rows, E = logits.shape
    ids = torch.empty((rows, n_used), dtype=torch.int32, device=logits.device)
    w = torch.empty((rows, n_used), dtype=torch.float32, device=logits.device)
    _check(lib().tsb_route_rows(_ptr(logits), E, n_used, rows, gate, in_scale, _ptr(bias), _ptr(escale), int(norm),
                                w_scale, _ptr(ids), _ptr(w), _stream(stream)), "route_rows")
    return ids, w


class Groups:
    """Device group tables (k_group's outputs) for up to cap entries."""

    def __init__(self, cap_entries: int, device):
        import torch
        self.cap = cap_entries
        self.grp_ptr = torch.zeros(cap_entries, dtype=torch.int64, device=device)
        self.grp_start = torch.zeros(cap_entries + 1, dtype=torch.int32, device=device)
        self.n_groups = torch.zeros(1, dtype=torch.int32, device=device)
        self.ent_dst = torch.zeros(cap_entries, dtype=torch.int32, device=device)
        self.ent_tok = torch.zeros(cap_entries, dtype=torch.int32, device=device)


def moe_group(ids, n_expert: int, blobs, blob_stride: int, groups: Groups | None = None, stream=None) -> Groups:
    """Decode grouping (k_group, q36_engine.cu:396-422); blobs = device base of the layer's expert blobs."""
    T, K = ids.shape
    groups = groups or Groups(T * K, ids.device)
    base = blobs.data_ptr() if hasattr(blobs, "data_ptr") else int(blobs)
    _check(lib().tsb_moe_group(_ptr(ids), T * K, K, n_expert, C.c_void_p(base), blob_stride, _ptr(groups.grp_ptr),
                               _ptr(groups.grp_start), _ptr(groups.n_groups), _ptr(groups.ent_dst),
                               _ptr(groups.ent_tok), _stream(stream)), "moe_group")
    return groups


def decode_act_desc(cfg: dict, n_tok: int, shared: bool) -> DecodeActDesc:
    """The descriptor of a Gemma / LFM layer config (router_mode softmax_scaled: gate 0; sigmoid: gate 1)."""
    d = DecodeActDesc()
    d.struct_size = C.sizeof(DecodeActDesc)
    d.n_tok, d.n_embd, d.n_ff = n_tok, cfg["n_embd"], cfg["n_ff"]
    d.n_expert, d.n_used = cfg["n_expert"], cfg["n_used"]
    d.sh_n_ff = (cfg.get("sh_n_ff") or 0) if shared else 0
    d.gu_type, d.d_type = cfg["gu_type"], cfg["d_type"]
    d.act, d.sh_act = cfg["act"], cfg.get("sh_act", cfg["act"])
    d.limit = cfg.get("limit", float("inf"))
    sig = cfg["router_mode"] == "sigmoid"
    d.gate = 1 if sig else 0
    d.in_scale = 1.0 if sig else cfg.get("in_scale", 1.0)
    d.norm = 1
    d.w_scale = cfg.get("w_scale", 0.0) if sig else 0.0
    return d


def moe_decode_act(desc: DecodeActDesc, router, h, hq, blobs, blob_stride: int, out, ws, bias=None, escale=None,
                   sh_blob=None, sh_out=None, ids=None, w=None, accumulate: bool = True, stream=None):
    """The Gemma / LFM decode MoE block in one launch (tsb_moe_decode_act)."""
    _check(lib().tsb_moe_decode_act(C.byref(desc), _ptr(router), _ptr(bias), _ptr(escale), _ptr(h), _ptr(hq),
                                    _ptr(blobs), blob_stride, _ptr(sh_blob), _ptr(out), int(accumulate), _ptr(sh_out),
                                    _ptr(ids), _ptr(w), _ptr(ws), ws.numel() * ws.element_size(), _stream(stream)),
           "moe_decode_act")
    return out


def moe_group_staged(ids, n_expert: int, slot_of, n_slots: int, slots, host_blobs, blob_stride: int, stage,
                     stage_cap: int, groups: Groups | None = None, counts=None, stream=None) -> Groups:
    """Grouping of a host-staged layer (k_group_hy, q36_engine.cu:423-452, with the missed experts fetched into
    stage by the GPU): slot_of int32 [n_expert] on the device, host_blobs a pinned host tensor."""
    T, K = ids.shape
    groups = groups or Groups(T * K, ids.device)
    _check(lib().tsb_moe_group_staged(_ptr(ids), T * K, K, n_expert, _ptr(slot_of), n_slots, _ptr(slots),
                                      _ptr(host_blobs), blob_stride, _ptr(stage), stage_cap, _ptr(groups.grp_ptr),
                                      _ptr(groups.grp_start), _ptr(groups.n_groups), _ptr(groups.ent_dst),
                                      _ptr(groups.ent_tok), _ptr(counts), _stream(stream)), "moe_group_staged")
    return groups


def staged_rebalance(score, slot_of, exp_in_slot, max_swaps: int):
    """The reference's rebalance of one layer (q36_engine.cu:3215-3265) on host numpy arrays (score float64,
    slot_of / exp_in_slot int32, updated in place).  Returns the moves as (experts, slots) int32 arrays."""
    import numpy as np
    for a, dt in ((score, np.float64), (slot_of, np.int32), (exp_in_slot, np.int32)):
        assert a.dtype == dt and a.flags.c_contiguous
    me = np.zeros(max(max_swaps, 1), np.int32)
    ms = np.zeros(max(max_swaps, 1), np.int32)
    n = lib().tsb_staged_rebalance(score.ctypes.data, score.size, exp_in_slot.size, slot_of.ctypes.data,
                                   exp_in_slot.ctypes.data, max_swaps, me.ctypes.data, ms.ctypes.data)
    _check(min(n, 0), "staged_rebalance")
    return me[:n], ms[:n]


def staged_load(host_blobs, slots, blob_stride: int, blob_bytes: int, move_expert, move_slot, n_expert: int,
                n_slots: int, stream=None):
    """The moved experts' blobs host to device into their slots (cudaMemcpyAsync on `stream`)."""
    _check(lib().tsb_staged_load(_ptr(host_blobs), _ptr(slots), blob_stride, blob_bytes, move_expert.ctypes.data,
                                 move_slot.ctypes.data, len(move_expert), n_expert, n_slots, _stream(stream)),
           "staged_load")


def stage_layer(slot_of, n_slots: int, slots, host_blobs, blob_stride: int, stage, whole: bool = False,
                stream=None) -> int:
    """The streamed prompt layer (stream_kick, q36_engine.cu:3001-3033): every blob into stage in expert order;
    slot_of a host int32 numpy array.  Returns the copies issued."""
    import numpy as np
    assert slot_of.dtype == np.int32 and slot_of.flags.c_contiguous
    n = lib().tsb_stage_layer(slot_of.ctypes.data, slot_of.size, n_slots, _ptr(slots), _ptr(host_blobs), blob_stride,
                              _ptr(stage), int(whole), _stream(stream))
    _check(min(n, 0), "stage_layer")
    return n


def native_expert_grouped(L: ExpertLayout, groups: Groups, cap_groups: int, cap_entries: int, x_q8_1, scratch, out,
                          act: int = ACT_SWIGLU, limit: float = float("inf"), stream=None):
    """Grouped experts (native_expert_grouped, iq_kernels.hpp:75-78); act selects the Gemma/LFM activations."""
    args = (C.byref(L), _ptr(groups.grp_ptr), _ptr(groups.grp_start), _ptr(groups.n_groups), _ptr(groups.ent_dst),
            _ptr(groups.ent_tok), cap_groups, cap_entries, _ptr(x_q8_1), _ptr(scratch), _ptr(out))
    if act == ACT_SWIGLU:
        _check(lib().tsb_native_expert_grouped(*args, _stream(stream), 0), "native_expert_grouped")
    else:
        _check(lib().tsb_native_expert_grouped_act(*args, act, limit, _stream(stream)), "native_expert_grouped_act")
    return out


def native_expert_grouped_noalloc(L: ExpertLayout, groups: Groups, cap_groups: int, cap_entries: int, x_q8_1, out,
                                  stream=None):
    """native_expert_grouped (SwiGLU) with the library's fixed 1 MiB device scratch instead of a caller buffer; one
    copy per device, so calls must not overlap in time."""
    _check(lib().tsb_native_expert_grouped_noalloc(C.byref(L), _ptr(groups.grp_ptr), _ptr(groups.grp_start),
                                                   _ptr(groups.n_groups), _ptr(groups.ent_dst), _ptr(groups.ent_tok),
                                                   cap_groups, cap_entries, _ptr(x_q8_1), _ptr(out), _stream(stream)),
           "native_expert_grouped_noalloc")
    return out


# ------------------------------------------------------------------------------------------------ prefill
def moe_dispatch(ids, n_expert: int, stream=None):
    """Stable sort of the entries by expert (q36_engine.cu:486-510): (bounds [E+1], row_ent, row_tok, rinv)."""
    import torch
    T, K = ids.shape
    n = T * K
    dev = ids.device
    bounds = torch.empty(n_expert + 1, dtype=torch.int32, device=dev)
    row_ent = torch.empty(n, dtype=torch.int32, device=dev)
    row_tok = torch.empty(n, dtype=torch.int32, device=dev)
    rinv = torch.empty(n, dtype=torch.int32, device=dev)
    _check(lib().tsb_moe_dispatch(_ptr(ids), n, K, n_expert, _ptr(bounds), _ptr(row_ent), _ptr(row_tok), _ptr(rinv),
                                  _stream(stream)), "moe_dispatch")
    return bounds, row_ent, row_tok, rinv


class MmqAct:
    """Activations in the tensor-core ("mmq") layout for `rows` rows of K values: one 256-byte aligned device buffer of
    tsb_mmq_act_bytes(rows, K) bytes holding int8 codes [rows][K], fp32 d [rows][ldS] and d * sum(codes) [rows][ldS]
    (ldS = K / 32 rounded up to 4).  The role of the reference's block_q8_1_mmq (moe_mmq.hpp:37)."""

    def __init__(self, rows: int, K: int, device, buf=None):
        import torch
        self.rows, self.K = rows, K
        self.ldS = (K // 32 + 3) // 4 * 4
        nbytes = int(lib().tsb_mmq_act_bytes(rows, K))
        if buf is None:
            buf = torch.empty(nbytes + 256, dtype=torch.uint8, device=device)
        assert buf.numel() >= nbytes
        off = (-buf.data_ptr()) % 256
        self._store = buf
        self.buf = buf[off:off + max(nbytes, 1)]

    def data_ptr(self):
        return self.buf.data_ptr()

    @property
    def codes(self):
        import torch
        return self.buf[:self.rows * self.K].view(torch.int8).view(self.rows, self.K)

    def _al(self, v):
        return (v + 255) // 256 * 256

    @property
    def d(self):
        import torch
        o = self._al(self.rows * self.K)
        return self.buf[o:o + self.rows * self.ldS * 4].view(torch.float32).view(self.rows, self.ldS)

    @property
    def s(self):
        import torch
        o = self._al(self.rows * self.K) + self._al(self.rows * self.ldS * 4)
        return self.buf[o:o + self.rows * self.ldS * 4].view(torch.float32).view(self.rows, self.ldS)


def mmq_quantize(x, row_src=None, n_rows: int | None = None, out: MmqAct | None = None, stream=None) -> MmqAct:
    """fp32 rows -> mmq layout; output row r from x[row_src[r]] (tsb_mmq_quantize; the reference's mmq::quantize)."""
    n_rows = x.shape[0] if n_rows is None else n_rows
    K = x.shape[1]
    out = out if out is not None else MmqAct(n_rows, K, x.device)
    _check(lib().tsb_mmq_quantize(_ptr(x), x.stride(0), _ptr(row_src), n_rows, K, C.c_void_p(out.data_ptr()),
                                  _stream(stream)), "mmq_quantize")
    return out


def mmq_from_q8_1(x_q8_1, K: int, row_src=None, n_rows: int | None = None, out: MmqAct | None = None,
                  stream=None) -> MmqAct:
    """q8_1 rows (uint8 [rows, K / 32 * 36]) -> mmq layout, output row r from row row_src[r]."""
    n_rows = x_q8_1.shape[0] if n_rows is None else n_rows
    out = out if out is not None else MmqAct(n_rows, K, x_q8_1.device)
    _check(lib().tsb_mmq_from_q8_1(_ptr(x_q8_1), _ptr(row_src), n_rows, K, C.c_void_p(out.data_ptr()),
                                   _stream(stream)), "mmq_from_q8_1")
    return out


def moe_prefill_gu(L: ExpertLayout, blobs, blob_stride: int, bounds, n_groups: int, n_rows: int, x_act: MmqAct,
                   act: int = ACT_SWIGLU, limit: float = float("inf"), h: MmqAct | None = None, stream=None) -> MmqAct:
    """Grouped gate/up + activation on the tensor cores (kind::i8): x_act rows (expert-sorted) -> the hidden vectors
    in the mmq layout."""
    h = h if h is not None else MmqAct(n_rows, int(L.n_ff), x_act.buf.device)
    _check(lib().tsb_moe_prefill_gu(C.byref(L), _ptr(blobs), blob_stride, _ptr(bounds), n_groups, n_rows,
                                    C.c_void_p(x_act.data_ptr()), C.c_void_p(h.data_ptr()), act, limit,
                                    _stream(stream)), "moe_prefill_gu")
    return h


def moe_prefill_down(L: ExpertLayout, blobs, blob_stride: int, bounds, n_groups: int, n_rows: int, h_act: MmqAct,
                     out=None, stream=None):
    """Grouped down on the tensor cores: moe_prefill_gu's hidden rows -> fp32 [n_rows, n_embd]."""
    import torch
    if out is None:
        out = torch.empty((n_rows, L.n_embd), dtype=torch.float32, device=h_act.buf.device)
    _check(lib().tsb_moe_prefill_down(C.byref(L), _ptr(blobs), blob_stride, _ptr(bounds), n_groups, n_rows,
                                      C.c_void_p(h_act.data_ptr()), _ptr(out), _stream(stream)), "moe_prefill_down")
    return out


def mmq_product(w, ggml_type: int, w_rows: int, w_cols: int, stride: int, n: int, x_act: MmqAct, bounds=None,
                ids=None, total_rows: int | None = None, dst=None, ld_dst: int | None = None, stream=None):
    """The grouped tensor-core product with fp32 output (tsb_mmq_product; mmq::Context::run / gemma4::Mmq::mul)."""
    import torch
    total_rows = x_act.rows if total_rows is None else total_rows
    if dst is None:
        dst = torch.empty((total_rows, w_rows), dtype=torch.float32, device=x_act.buf.device)
    ld_dst = dst.stride(0) if ld_dst is None else ld_dst
    _check(lib().tsb_mmq_product(_ptr(w), ggml_type, w_rows, w_cols, stride, n, C.c_void_p(x_act.data_ptr()),
                                 _ptr(bounds), _ptr(ids), total_rows, _ptr(dst), ld_dst, _stream(stream)),
           "mmq_product")
    return dst


def mmvq_slots(ggml_type: int, ws, xs, ys, n_in: int, n_out: int, stream=None):
    """Up to 32 products y[i] = W[i] x[i] (q8_1 columns) in one launch (gemma_native_mmvq_slots)."""
    S = MmvqSlots()
    for i, (w, x, y) in enumerate(zip(ws, xs, ys)):
        S.w[i], S.x[i], S.y[i] = w.data_ptr(), x.data_ptr(), y.data_ptr()
    _check(lib().tsb_mmvq_run_slots(ggml_type, C.byref(S), len(ws), n_in, n_out, _stream(stream)), "mmvq_run_slots")


def mmvq_ids(ggml_type: int, table, ids, offset: int, x, x_stride: int, x_every: int, y, y_stride: int, count: int,
             n_in: int, n_out: int, stream=None):
    """The products of matrices table[ids[j]] + offset (device table and ids), gemma_native_mmvq_ids."""
    M = MmvqIds(table.data_ptr(), ids.data_ptr(), offset, x.data_ptr(), x_stride, x_every, y.data_ptr(), y_stride)
    _check(lib().tsb_mmvq_run_ids(ggml_type, C.byref(M), count, n_in, n_out, _stream(stream)), "mmvq_run_ids")


def debug_mmq_block_sums(L: ExpertLayout, mode: int, blob, n_rows: int, x_act: MmqAct, stream=None):
    """The int32 block sums of the first tile of one prefill launch (mode 0 gate/up, 1 down) over one expert blob:
    [K / 32, split, 128 rows, 128 tile columns]."""
    import torch
    K = int(L.n_embd if mode == 0 else L.n_ff)
    split = 2 if (L.d_type if mode == 1 else L.gu_type) == T_Q6_K else 1
    sums = torch.zeros((K // 32, split, 128, 128), dtype=torch.int32, device=blob.device)
    h = MmqAct(n_rows, int(L.n_ff), blob.device) if mode == 0 else None
    out = torch.empty((n_rows, int(L.n_embd)), dtype=torch.float32, device=blob.device) if mode == 1 else None
    _check(lib().tsb_debug_mmq_block_sums(C.byref(L), mode, _ptr(blob), n_rows, C.c_void_p(x_act.data_ptr()),
                                          C.c_void_p(h.data_ptr()) if h is not None else None, _ptr(out), _ptr(sums),
                                          _stream(stream)), "debug_mmq_block_sums")
    return sums, (h if mode == 0 else out)


def moe_combine(x, parts, wts, K, shared=None, sgate=None, sg_stride=1, prow=None, wn=None, h=None, hq=None,
                eps=1e-6, stream=None):
    """x += sum_k w part + sigmoid(sgate) shared; h = rms(x) wn; hq = q8_1(h) (k_moe_out, q36_engine.cu:307-332)."""
    T, n = x.shape
    _check(lib().tsb_moe_combine(_ptr(x), _ptr(parts), _ptr(prow), _ptr(wts), K, _ptr(shared), _ptr(sgate), sg_stride,
                                 _ptr(wn), _ptr(h), _ptr(hq), n, eps, T, _stream(stream)), "moe_combine")
    return x


def rms_norm_q8_1(x, h=None, hq=None, wn=None, eps=1e-6, stream=None):
    """h = rms(x) * wn and its q8_1 image (the layer input's norm, q36_kernels.cuh:222-250 without the add)."""
    T_, n = x.shape
    _check(lib().tsb_rms_norm_q8_1(_ptr(x), _ptr(wn), _ptr(h), _ptr(hq), n, eps, T_, _stream(stream)), "rms_norm_q8_1")


def native_expert_set_phase(phase: int):
    _check(lib().tsb_native_expert_set_phase(phase), "native_expert_set_phase")


def moe_sum(x, w, acc, n_used, stream=None):
    rows, n = acc.shape
    _check(lib().tsb_moe_sum(_ptr(x), _ptr(w), _ptr(acc), n, n_used, rows, _stream(stream)), "moe_sum")
    return acc


class ScaledRows(C.Structure):
    """tsb_scaled_rows (the reference's ScaledRows, include/strata/gemma4/kernels.hpp:51-56)."""
    _fields_ = [("x", C.c_void_p * 32), ("acc", C.c_void_p * 32), ("w", C.c_float * 32)]


def add_scaled(xs, accs, ws, stream=None):
    """accs[k] += xs[k] * ws[k] for k in order (add_scaled, src/gemma4/kernels.cu:245-249)."""
    R = ScaledRows()
    for k, (x, a, w) in enumerate(zip(xs, accs, ws)):
        R.x[k], R.acc[k], R.w[k] = x.data_ptr(), a.data_ptr(), float(w)
    _check(lib().tsb_add_scaled(C.byref(R), len(xs), xs[0].numel(), _stream(stream)), "add_scaled")


def moe_layer_tail(moe, r, post_moe=None, mlp=None, post_ffn=None, out_scale=1.0, eps=1e-6, stream=None):
    """The Gemma 4 layer tail (gemma4.cpp:560-568): r = (r + rms(rms(moe) post_moe + mlp) post_ffn) out_scale."""
    rows, n = moe.shape
    _check(lib().tsb_moe_layer_tail(_ptr(moe), _ptr(post_moe), _ptr(mlp), _ptr(post_ffn), _ptr(r), out_scale, n, rows,
                                    eps, _stream(stream)), "moe_layer_tail")
    return r


def debug_row_calls(ggml_type: int, row, x_q8_1, n: int, stream=None):
    import torch
    qk = {T_Q4_0: 32, T_Q8_0: 32, T_Q4_K: 256, T_Q6_K: 256, T_IQ3_XXS: 256, T_IQ3_S: 256}[ggml_type]
    cpb = {T_Q4_0: 2, T_Q8_0: 4, T_Q4_K: 16, T_Q6_K: 32, T_IQ3_XXS: 8, T_IQ3_S: 8}[ggml_type]
    calls = n // qk * cpb
    s = torch.empty(calls, dtype=torch.int32, device=row.device)
    v = torch.empty(calls, dtype=torch.float32, device=row.device)
    _check(lib().tsb_debug_row_calls(ggml_type, _ptr(row), _ptr(x_q8_1), n, _ptr(s), _ptr(v), _stream(stream)),
           "debug_row_calls")
    return s, v


def set_wait_limit_ns(ns: int):
    """The bound of every spin-wait in the library's kernels on the current device (default 2e9 ns)."""
    _check(lib().tsb_set_wait_limit_ns(int(ns)), "set_wait_limit_ns")


def decode_set_debug(withhold_cta: int):
    """Tests of the bounded waits: CTA withhold_cta - 1 of later fused-decode launches skips publishing its layer-0
    router logits (0 turns it off)."""
    _check(lib().tsb_moe_decode_set_debug(int(withhold_cta)), "moe_decode_set_debug")


def device_error(clear: bool = True) -> int:
    code = C.c_uint(0)
    _check(lib().tsb_device_error(C.byref(code), int(clear)), "device_error")
    return int(code.value)


class DecodeStack:
    """The fused decode path over n_layers resident layers: one persistent launch per step
    (tsb_moe_decode_layers).  blobs [L][E][bytes] uint8, routers [L][E + 1][H] fp32, sh_blobs [L][bytes] uint8,
    priors (optional) [L][n_tok][E] fp32 added to the router logits.  record: keep every layer's routing (ids, w);
    record_x: also x after every layer (x_rec [L][n_tok][H])."""

    def __init__(self, cfg: dict, blobs, routers, sh_blobs, n_tok: int, eps: float = 1e-6, record: bool = True,
                 priors=None, record_x: bool = False):
        import torch
        self.cfg = cfg
        L = blobs.shape[0]
        self.desc = DecodeDesc(C.sizeof(DecodeDesc), L, n_tok, cfg["n_embd"], cfg["n_ff"], cfg["n_expert"],
                               cfg["n_used"], cfg["sh_n_ff"], cfg["gu_type"], cfg["d_type"], cfg["sh_gu_type"],
                               cfg["sh_d_type"], eps)
        dev = blobs.device
        tab = torch.tensor([[blobs[l].data_ptr(), routers[l].data_ptr(), sh_blobs[l].data_ptr(),
                             priors[l].data_ptr() if priors is not None else 0] for l in range(L)], dtype=torch.int64)
        self.layers = tab.to(dev)
        self.ws_bytes = int(lib().tsb_moe_decode_workspace_bytes(C.byref(self.desc)))
        self.ws = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=dev)
        K = cfg["n_used"]
        self.ids = torch.zeros((L, n_tok, K), dtype=torch.int32, device=dev) if record else None
        self.w = torch.zeros((L, n_tok, K), dtype=torch.float32, device=dev) if record else None
        self.x_rec = torch.zeros((L, n_tok, cfg["n_embd"]), dtype=torch.float32, device=dev) if record_x else None
        self._keep = (blobs, routers, sh_blobs, priors)

    def forward(self, x, stream=None):
        rc = lib().tsb_moe_decode_layers(C.byref(self.desc), _ptr(self.layers), _ptr(x), _ptr(self.ids), _ptr(self.w),
                                         _ptr(self.x_rec), _ptr(self.ws), self.ws_bytes, _stream(stream))
        if rc != 0:
            raise TsbError(f"moe_decode_layers: status {rc}: {lib().tsb_decode_last_error().decode()}")
        return x

    def trace(self, x, stream=None):
        """One traced step: per layer, per phase the mean / max over CTAs of the stamp offsets (us from the launch's
        first stamp).  Returns (stamps [L][16][CTAs] int64 tensor, summary dict)."""
        import torch
        L = self.desc.n_layers
        sms = torch.cuda.get_device_properties(x.device).multi_processor_count
        buf = torch.zeros((L, 16, sms), dtype=torch.int64, device=x.device)
        _check(lib().tsb_moe_decode_set_trace(_ptr(buf)), "set_trace")
        try:
            self.forward(x, stream)
            torch.cuda.synchronize()
        finally:
            lib().tsb_moe_decode_set_trace(None)
        return buf.cpu()

    def error(self) -> int:
        code = (C.c_uint * 128)()
        _check(lib().tsb_moe_decode_error(C.byref(self.desc), _ptr(self.ws), code), "moe_decode_error")
        self.error_detail = [hex(int(c)) for c in code[:106]] + ["layout"] + [hex(int(c)) for c in code[110:117]]
        if code[0]:
            import torch
            w = self.ws.view(torch.int32)
            # progress words after the error record: (layer << 8) | phase stamp of each CTA
            off = (self.ws_bytes - 8192) // 4 + 128
            prog = w[off:off + torch.cuda.get_device_properties(self.ws.device).multi_processor_count].cpu().tolist()
            from collections import Counter
            self.error_detail.append(sorted(Counter(hex(v) for v in prog).items()))
        return int(code[0])


from .layer import MoELayer, StagedExperts  # noqa: E402  (host mirror of the engines' MoE block)
