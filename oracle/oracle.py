"""oracle/oracle.py - TEST INFRASTRUCTURE: numpy face on the C restatement (tsb_oracle.c) and on the reference's own
compiled CPU kernels (oracle/_ref/libtsb_ref_cpu.so).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's ``cpu_baseline`` leg import this module, and only as the
checker.  Each function names the reference code it restates (paths inside the TinyStrata tree).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None
_lock = threading.Lock()

Q8_1_BYTES = 36
T_Q4_0, T_Q8_0, T_Q4_K, T_Q6_K, T_IQ3_XXS, T_IQ3_S = 2, 8, 12, 14, 18, 21
ACT_SWIGLU, ACT_GELU_TANH, ACT_SWIGLU_CLAMP = 0, 1, 2

_p = C.c_void_p
_i64 = C.c_int64
_i32 = C.c_int32
_f = C.c_float


def reference_dir() -> str:
    """The TinyStrata source tree the `ref` builds compile from: $REF when set, else a `reference` directory beside
    this repository (the same rule as oracle/Makefile)."""
    return os.environ.get("REF") or os.path.abspath(os.path.join(HERE, "..", "..", "reference"))


def build(ref: bool = True) -> None:
    """make the C restatement, and the reference CPU kernels when the reference tree is present."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    if ref and os.path.isdir(reference_dir()):
        subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)


def lib():
    global _LIB
    with _lock:
        if _LIB is None:
            path = os.path.join(HERE, "libtsb_oracle.so")
            if not os.path.exists(path):
                build(ref=False)
            L = C.CDLL(path)
            L.or_half_to_float.restype = _f
            L.or_half_to_float.argtypes = [C.c_uint16]
            L.or_float_to_half.restype = C.c_uint16
            L.or_float_to_half.argtypes = [_f]
            L.or_q8_1_block.argtypes = [_p, _p]
            L.or_quantize_q8_1_rows.argtypes = [_p, _i64, _i64, _p]
            for fn in ("or_block_values", "or_block_bytes", "or_calls_per_block"):
                getattr(L, fn).restype = C.c_int
                getattr(L, fn).argtypes = [C.c_int]
            L.or_row_bytes.restype = _i64
            L.or_row_bytes.argtypes = [C.c_int, _i64]
            L.or_row_calls.restype = _i64
            L.or_row_calls.argtypes = [C.c_int, _i64]
            L.or_row_dot_calls.argtypes = [C.c_int, _p, _p, _i64, _p, _p]
            L.or_row_dot.restype = C.c_double
            L.or_row_dot.argtypes = [C.c_int, _p, _p, _i64]
            L.or_mat_vec.argtypes = [C.c_int, _p, _p, _i64, _i64, _p]
            L.or_dequant_row.argtypes = [C.c_int, _p, _i64, _p]
            L.or_weight_codes.argtypes = [C.c_int, _p, _i64, _p]
            L.or_router_softmax_topk.restype = C.c_int
            L.or_router_softmax_topk.argtypes = [_p, C.c_int, C.c_int, C.c_int, C.c_int, _p, _p, _f]
            L.or_route_rows.argtypes = [_p, C.c_int, C.c_int, C.c_int, C.c_int, _f, _p, _p, C.c_int, _f, _p, _p]
            L.or_group.restype = C.c_int
            L.or_group.argtypes = [_p, C.c_int, C.c_int, C.c_int, _p, _p, _p, _p]
            L.or_dispatch.restype = C.c_int
            L.or_dispatch.argtypes = [_p, C.c_int, C.c_int, C.c_int, _p, _p, _p, _p]
            L.or_expert_ffn.argtypes = [C.c_int, C.c_int, _p, _i64, _i64, C.c_int, _f, _p, _p, _p]
            L.or_combine_token.argtypes = [_p, _p, _p, C.c_int, _p, _f, _i64, _p]
            L.or_rms_q8_1.argtypes = [_p, _p, _i64, _f, _p, _p]
            _LIB = L
    return _LIB


def ref_cpu():
    """The reference's own CPU expert kernels (oracle/_ref/libtsb_ref_cpu.so), or None when not built."""
    global _REF
    with _lock:
        if _REF is None:
            path = os.path.join(HERE, "_ref", "libtsb_ref_cpu.so")
            if not os.path.exists(path):
                return None
            R = C.CDLL(path)
            R.ref_cpu_isa.restype = C.c_int
            R.ref_q8k_quant.argtypes = [_p, _p, _i64]
            R.ref_gu_rows.restype = C.c_int
            R.ref_gu_rows.argtypes = [C.c_int, _p, C.c_size_t, C.c_size_t, C.c_int, _p, C.c_int, _p, C.c_int, C.c_int]
            R.ref_rows.restype = C.c_int
            R.ref_rows.argtypes = [C.c_int, _p, C.c_size_t, C.c_int, _p, C.c_int, _p, C.c_int, C.c_int]
            R.ref_cpu_moe_decode.restype = C.c_double
            R.ref_cpu_moe_decode.argtypes = [C.c_int, C.c_int, _p, C.c_size_t, C.c_int, C.c_int, C.c_size_t,
                                             C.c_size_t, _p, _p, C.c_int, _p, C.c_int, _p, C.c_int]
            _REF = R
    return _REF


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_p)


# ------------------------------------------------------------------------------------------------ formats
def block_values(t: int) -> int:
    return lib().or_block_values(t)


def block_bytes(t: int) -> int:
    return lib().or_block_bytes(t)


def row_bytes(t: int, n: int) -> int:
    return int(lib().or_row_bytes(t, n))


def calls_per_block(t: int) -> int:
    return lib().or_calls_per_block(t)


def half_to_float(h: int) -> float:
    return lib().or_half_to_float(h)


def float_to_half(f: float) -> int:
    return lib().or_float_to_half(f)


# ------------------------------------------------------------------------------------------------ q8_1
def quantize_q8_1(x: np.ndarray) -> np.ndarray:
    """fp32 [rows, n] -> q8_1 bytes [rows, n/32*36] (iq_kernels.cu:1469-1494, IEEE division)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, n = x.reshape(-1, x.shape[-1]).shape
    y = np.zeros((rows, n // 32 * Q8_1_BYTES), np.uint8)
    lib().or_quantize_q8_1_rows(_ptr(x), rows, n, _ptr(y))
    return y.reshape(x.shape[:-1] + (n // 32 * Q8_1_BYTES,))


def q8_1_unpack(q: np.ndarray):
    """q8_1 bytes [..., nb*36] -> (d fp32 [..., nb], sum fp32 [..., nb], codes int8 [..., nb, 32])."""
    q = np.ascontiguousarray(q, dtype=np.uint8)
    nb = q.shape[-1] // Q8_1_BYTES
    b = q.reshape(q.shape[:-1] + (nb, Q8_1_BYTES))
    d = b[..., 0:2].copy().view(np.float16)[..., 0].astype(np.float32)
    s = b[..., 2:4].copy().view(np.float16)[..., 0].astype(np.float32)
    codes = b[..., 4:].view(np.int8)
    return d, s, codes


def q8_1_compare(a: np.ndarray, b: np.ndarray, x: np.ndarray | None = None):
    """Compare two q8_1 images: returns (n blocks whose d or sum differ, n codes that differ, max |code diff|)."""
    da, sa, ca = q8_1_unpack(a)
    db, sb, cb = q8_1_unpack(b)
    bad_ds = int(np.count_nonzero((da != db) | (sa != sb)))
    diff = np.abs(ca.astype(np.int32) - cb.astype(np.int32))
    return bad_ds, int(np.count_nonzero(diff)), int(diff.max(initial=0))


# ------------------------------------------------------------------------------------------------ dots
def row_dot_calls(t: int, row: np.ndarray, xq: np.ndarray, n: int):
    """Per-call integer sums and float values of one row against one q8_1 activation (row_dot's call order)."""
    ncalls = int(lib().or_row_calls(t, n))
    s = np.zeros(ncalls, np.int32)
    v = np.zeros(ncalls, np.float32)
    lib().or_row_dot_calls(t, _ptr(np.ascontiguousarray(row)), _ptr(np.ascontiguousarray(xq)), n, _ptr(s), _ptr(v))
    return s, v


def mat_vec(t: int, w: np.ndarray, xq: np.ndarray, n_in: int, n_out: int) -> np.ndarray:
    y = np.zeros(n_out, np.float32)
    lib().or_mat_vec(t, _ptr(np.ascontiguousarray(w)), _ptr(np.ascontiguousarray(xq)), n_in, n_out, _ptr(y))
    return y


def weight_codes(t: int, rows: np.ndarray, n: int) -> np.ndarray:
    """int8 [rows, n]: the integer weight codes the block dots multiply the activation codes by (or_weight_codes)."""
    rows = np.ascontiguousarray(rows, dtype=np.uint8).reshape(-1, row_bytes(t, n))
    out = np.empty((rows.shape[0], n), dtype=np.int8)
    for r in range(rows.shape[0]):
        lib().or_weight_codes(t, _ptr(rows[r]), n, _ptr(out[r]))
    return out


def dequant_row(t: int, row: np.ndarray, n: int) -> np.ndarray:
    y = np.zeros(n, np.float32)
    lib().or_dequant_row(t, _ptr(np.ascontiguousarray(row)), n, _ptr(y))
    return y


# ------------------------------------------------------------------------------------------------ routing
def router_softmax_topk(logits: np.ndarray, k: int, n_expert: int | None = None, tie_ulps: float = 4.0):
    """native_router.cu:44-95: softmax, k argmax picks, renormalised (floor 6.103515625e-5).
    Returns (ids int32 [T,k], w fp32 [T,k], near_ties)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T, ld = logits.shape
    n_expert = n_expert or ld
    ids = np.zeros((T, k), np.int32)
    w = np.zeros((T, k), np.float32)
    nt = lib().or_router_softmax_topk(_ptr(logits), T, n_expert, ld, k, _ptr(ids), _ptr(w), tie_ulps)
    return ids, w, nt


def route_rows(logits: np.ndarray, n_used: int, gate: int, in_scale: float = 1.0, bias=None, escale=None,
               norm: bool = True, w_scale: float = 0.0):
    """gemma4/kernels.cu:289-356 (route_rows): gate 0 softmax(logit*in_scale), 1 sigmoid; pick on p+bias."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = logits.shape
    ids = np.zeros((T, n_used), np.int32)
    w = np.zeros((T, n_used), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    s = None if escale is None else np.ascontiguousarray(escale, dtype=np.float32)
    lib().or_route_rows(_ptr(logits), E, n_used, T, gate, in_scale, None if b is None else _ptr(b),
                        None if s is None else _ptr(s), int(norm), w_scale, _ptr(ids), _ptr(w))
    return ids, w


def group(ids: np.ndarray, n_expert: int):
    """q36_engine.cu:396-422 (k_group): groups by ascending expert id, entries in entry order."""
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    T, K = ids.shape
    n_ent = T * K
    ge = np.zeros(n_ent, np.int32)
    gs = np.zeros(n_ent + 1, np.int32)
    dst = np.zeros(n_ent, np.int32)
    tok = np.zeros(n_ent, np.int32)
    g = lib().or_group(_ptr(ids), n_ent, K, n_expert, _ptr(ge), _ptr(gs), _ptr(dst), _ptr(tok))
    return ge[:g].copy(), gs[:g + 1].copy(), dst, tok


def dispatch(ids: np.ndarray, n_expert: int):
    """q36_engine.cu:486-510 in the stable (expert, entry) order: bounds, dst, src, inv, max_rows."""
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    T, K = ids.shape
    n_ent = T * K
    bounds = np.zeros(n_expert + 1, np.int32)
    dst = np.zeros(n_ent, np.int32)
    src = np.zeros(n_ent, np.int32)
    inv = np.zeros(n_ent, np.int32)
    mx = lib().or_dispatch(_ptr(ids), n_ent, K, n_expert, _ptr(bounds), _ptr(dst), _ptr(src), _ptr(inv))
    return bounds, dst, src, inv, mx


def staged_rebalance(score: np.ndarray, slot_of: np.ndarray, exp_in_slot: np.ndarray, max_swaps: int):
    """The hybrid mode's placement of one layer, src/qwen35/q36_engine.cu:3215-3265 (the non-fair scan), with
    std::sort's unspecified tie order fixed as the lower id / lower slot first, and the age of
    include/strata/qwen35/cache_policy.hpp:28-30.  Updates the arrays in place; returns the moves [(expert, slot)]."""
    E, S = score.size, exp_in_slot.size
    moves = []
    if S <= 0 or S >= E:
        return moves
    order = sorted(range(E), key=lambda x: (-score[x], x))
    victims = sorted(range(S), key=lambda s: (score[exp_in_slot[s]], s))
    vi, left = 0, max_swaps
    for i in range(S):
        if left <= 0:
            break
        x = order[i]
        if slot_of[x] >= 0:
            continue
        if vi >= len(victims):
            break
        s = victims[vi]
        y = exp_in_slot[s]
        if score[y] >= score[x]:
            break
        vi += 1
        slot_of[y] = -1
        slot_of[x] = s
        exp_in_slot[s] = x
        moves.append((x, s))
        left -= 1
    score *= 0.5
    return moves


# ------------------------------------------------------------------------------------------------ experts
def expert_ffn(gu_type: int, d_type: int, blob: np.ndarray, n_embd: int, n_ff: int, xq_row: np.ndarray,
               act: int = ACT_SWIGLU, limit: float = float("inf"), want_h: bool = False):
    out = np.zeros(n_embd, np.float32)
    h = np.zeros(n_ff, np.float32) if want_h else None
    lib().or_expert_ffn(gu_type, d_type, _ptr(np.ascontiguousarray(blob)), n_embd, n_ff, act, limit,
                        _ptr(np.ascontiguousarray(xq_row)), _ptr(out), None if h is None else _ptr(h))
    return (out, h) if want_h else out


def experts_for_tokens(gu_type, d_type, blobs, n_embd, n_ff, xq, ids, act=ACT_SWIGLU, limit=float("inf"),
                       threads: int | None = None):
    """parts[t, k] = expert ids[t, k] applied to token t (fp32 [T, K, n_embd]); blobs [E, blob_bytes]."""
    T, K = ids.shape
    parts = np.zeros((T, K, n_embd), np.float32)

    def one(tk):
        t, k = divmod(tk, K)
        parts[t, k] = expert_ffn(gu_type, d_type, blobs[ids[t, k]], n_embd, n_ff, xq[t], act, limit)

    with ThreadPoolExecutor(max_workers=threads or os.cpu_count()) as ex:
        list(ex.map(one, range(T * K)))
    return parts


def combine(x, parts, wts, shared=None, gs=None):
    """k_moe_out (q36_engine.cu:307-332) in double: x + sum_k w_k part_k + gs * shared."""
    T, K, n = parts.shape
    acc = np.einsum("tk,tkn->tn", wts.astype(np.float64), parts.astype(np.float64))
    if shared is not None:
        g = np.ones(T) if gs is None else np.asarray(gs, np.float64)
        acc += g[:, None] * shared.astype(np.float64)
    base = np.zeros((T, n)) if x is None else x.astype(np.float64)
    return (base + acc).astype(np.float32)


def rms_q8_1(x: np.ndarray, wn=None, eps: float = 1e-6):
    """The combine epilogue (q36_kernels.cuh:252-290): h = x * rsqrt(mean x^2 + eps) * wn, and q8_1(h)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    T, n = x.shape
    h = np.zeros_like(x)
    hq = np.zeros((T, n // 32 * Q8_1_BYTES), np.uint8)
    w = None if wn is None else np.ascontiguousarray(wn, dtype=np.float32)
    for t in range(T):
        lib().or_rms_q8_1(_ptr(x[t]), None if w is None else _ptr(w), n, eps, _ptr(h[t]), _ptr(hq[t]))
    return h, hq


def sigmoid(v):
    return 1.0 / (1.0 + np.exp(-np.asarray(v, np.float64)))


def moe_layer(layer: dict, h: np.ndarray, logits: np.ndarray | None = None, threads: int | None = None) -> dict:
    """The whole MoE block for tokens h (fp32 [T, H]) of a synthetic layer (tinystrata_b200.synth):
    router -> routing -> experts -> shared expert -> combine, the reference's call stack A/C
    (q36_engine.cu:2821-2925; gemma4 engine.cpp:2436-2457).  Returns ids, w, parts, shared, out (no residual)."""
    cfg = layer["cfg"]
    H, E, K = cfg["n_embd"], cfg["n_expert"], cfg["n_used"]
    T = h.shape[0]
    if logits is None:
        W = layer["router"].astype(np.float64)
        logits = (h.astype(np.float64) @ W.T).astype(np.float32)
    xq = quantize_q8_1(h)
    mode = cfg["router_mode"]
    gs = None
    if mode == "softmax":
        ids, w, _ = router_softmax_topk(logits[:, :E], K, E)
        if cfg.get("shared_gate"):
            gs = sigmoid(logits[:, E])
    elif mode == "softmax_scaled":
        ids, w = route_rows(logits[:, :E], K, 0, cfg.get("in_scale", 1.0), None, layer.get("escale"), True, 0.0)
    else:
        ids, w = route_rows(logits[:, :E], K, 1, 1.0, layer.get("bias"), None, True, cfg.get("w_scale", 0.0))
    act = cfg["act"]
    parts = experts_for_tokens(cfg["gu_type"], cfg["d_type"], layer["blobs"], H, cfg["n_ff"], xq, ids, act,
                               cfg.get("limit", float("inf")), threads)
    shared = None
    if cfg.get("sh_n_ff"):
        shared = np.stack([expert_ffn(cfg["sh_gu_type"], cfg["sh_d_type"], layer["sh_blob"], H, cfg["sh_n_ff"], xq[t],
                                      cfg.get("sh_act", act), cfg.get("limit", float("inf"))) for t in range(T)])
    out = combine(None, parts, w, shared, gs)
    return {"logits": logits, "ids": ids, "w": w, "parts": parts, "shared": shared, "gs": gs, "out": out, "xq": xq}


# ------------------------------------------------------------------------------------------------ CPU baseline
def physical_cores() -> int:
    """Physical cores of this host (the reference pins one worker per physical core, pool.hpp:45-109)."""
    try:
        seen = set()
        for cpu in os.listdir("/sys/devices/system/cpu"):
            if cpu.startswith("cpu") and cpu[3:].isdigit():
                base = f"/sys/devices/system/cpu/{cpu}/topology/"
                with open(base + "physical_package_id") as f1, open(base + "core_id") as f2:
                    seen.add((f1.read().strip(), f2.read().strip()))
        if seen:
            return len(seen)
    except OSError:
        pass
    return os.cpu_count() or 1


def cpu_baseline_decode(cfg: dict, seconds: float = 10.0, threads: int | None = None, seed: int = 1,
                        chunk: int = 16) -> dict:
    """Time the reference's own CPU expert path (oracle/_ref, ref_cpu_moe_decode) on decode tokens of one layer with
    every expert resident in host memory, random distinct top-K routing per token, for about `seconds`.
    Returns tokens/s through one MoE layer (routed experts), the threads used and the sample description."""
    import time
    from tinystrata_b200 import synth
    R = ref_cpu()
    if R is None:
        raise RuntimeError("oracle/_ref/libtsb_ref_cpu.so is not built")
    threads = threads or physical_cores()
    layer = synth.make_layer(cfg, seed)
    blobs = np.ascontiguousarray(layer["blobs"])
    E, K, H, F = cfg["n_expert"], cfg["n_used"], cfg["n_embd"], cfg["n_ff"]
    L = synth.blob_layout(cfg)
    rng = np.random.default_rng(seed)
    done, times = 0, []
    t_end = time.time() + seconds
    while time.time() < t_end or done < chunk:
        ids = np.stack([rng.choice(E, K, replace=False) for _ in range(chunk)]).astype(np.int32)
        w = rng.dirichlet(np.ones(K), size=chunk).astype(np.float32)
        x = synth.rms_normed(rng, chunk, H)
        out = np.zeros((chunk, H), np.float32)
        times.append(R.ref_cpu_moe_decode(cfg["gu_type"], cfg["d_type"], _ptr(blobs), L["bytes"], H, F, L["gu_row"],
                                          L["d_row"], _ptr(ids), _ptr(w), K, _ptr(x), chunk, _ptr(out), threads))
        done += chunk
    # the median chunk: a chunk that the shared host interrupted does not pull the rate down (the mean rate beside it)
    t_med = float(np.median(times))
    return {"value": chunk / t_med, "unit": "tokens/s", "cores": threads, "kind": "reference",
            "mean_value": done / float(np.sum(times)),
            "sample": f"{done} decode tokens x 1 layer ({cfg['name']}, {K} routed experts each of {E} resident in host "
                      f"memory, reference iq512/iq256 rows + q8k_quant_avx2, {threads} worker threads), "
                      f"{float(np.sum(times)):.1f} s; value = {chunk} tokens / the median of {len(times)} chunk times"}


_CX = None


def cx_port():
    """oracle/libcx_port.so: the C restatement of the reference's CPU expert path (cpu_experts_port.c)."""
    global _CX
    with _lock:
        if _CX is None:
            path = os.path.join(HERE, "libcx_port.so")
            if not os.path.exists(path):
                build(ref=False)
            L = C.CDLL(path)
            L.cx_moe_experts_q4_0.restype = C.c_int
            L.cx_moe_experts_q4_0.argtypes = [_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_int, C.c_int, _p, C.c_int,
                                              _p, _p, C.c_int, C.c_int, _f, C.c_int, _p]
            _CX = L
    return _CX


def cx_moe_experts_q4_0(blobs, layout: dict, n_embd: int, n_ff: int, x, ids, w, gelu: bool, limit=float("inf"),
                        threads: int = 1):
    """The routed experts of `x` (fp32 [rows, n_embd]) through cpu_experts_port.c: fp32 [rows, n_embd]."""
    blobs = np.ascontiguousarray(blobs)
    x = np.ascontiguousarray(x, dtype=np.float32)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, K = ids.shape
    out = np.zeros((rows, n_embd), np.float32)
    rc = cx_port().cx_moe_experts_q4_0(_ptr(blobs), blobs.shape[1], layout["up_off"], layout["down_off"], n_embd,
                                       n_ff, _ptr(x), rows, _ptr(ids), _ptr(w), K, int(gelu), limit, threads,
                                       _ptr(out))
    if rc != 0:
        raise ValueError("cx_moe_experts_q4_0: arguments")
    return out


def cpu_baseline_prefill(cfg: dict, seconds: float = 10.0, threads: int | None = None, seed: int = 2,
                         chunk: int = 256) -> dict:
    """C2's routed experts (Q4_0 Gemma-4-shaped layer, every expert in host memory, uniform routing) through the C
    restatement of the reference's CPU expert path (cpu_experts_port.c, gemma4/cpu_experts.cpp:145-235) on this host's
    cores, prompt chunks of `chunk` tokens for about `seconds`: tokens/s through the layer's routed experts."""
    import time
    from tinystrata_b200 import synth
    threads = threads or physical_cores()
    layer = synth.make_layer(cfg, seed)
    blobs = np.ascontiguousarray(layer["blobs"])
    E, K, H, F = cfg["n_expert"], cfg["n_used"], cfg["n_embd"], cfg["n_ff"]
    L = synth.blob_layout(cfg)
    rng = np.random.default_rng(seed)
    done, elapsed = 0, 0.0
    t_end = time.time() + seconds
    while time.time() < t_end or done < chunk:
        ids = np.stack([rng.choice(E, K, replace=False) for _ in range(chunk)]).astype(np.int32)
        w = rng.dirichlet(np.ones(K), size=chunk).astype(np.float32)
        x = synth.rms_normed(rng, chunk, H)
        t0 = time.perf_counter()
        cx_moe_experts_q4_0(blobs, L, H, F, x, ids, w, gelu=True, threads=threads)
        elapsed += time.perf_counter() - t0
        done += chunk
    return {"value": done / elapsed, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{done} prompt tokens in chunks of {chunk} x 1 layer ({cfg['name']}, {K} of {E} Q4_0 routed "
                      f"experts resident in host memory; shared FFN, router and combine not included), C restatement "
                      f"of gemma4/cpu_experts.cpp:145-235 with ggml's Q4_0 x Q8_0 dot, {threads} worker threads, "
                      f"{elapsed:.1f} s"}
