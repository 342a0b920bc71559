"""Expert-parallel prefill (the multi-GPU row of the expert path): experts [r E/G, (r+1) E/G) live on rank r (block
placement), or experts r, r + G, r + 2G, ... (cyclic placement: a popularity-ordered expert set -- a skewed router's
head -- spreads over the ranks instead of landing on rank 0), every rank routes its own tokens, and two all-to-all
exchanges move the work (the layout TinyStrata's serving layer would shard
its prompt path with; the reference itself runs a single GPU, src/gemma4/engine.cpp:2436-2457 is the per-GPU body).

One forward:
  1. destinations: rank of each pick (expert // (E / G), or expert % G when cyclic); a token goes to a rank once,
     whatever number of its picks live there (deduplicated), in token order;
  2. counts exchange (all_to_all_single of G int64);
  3. dispatch exchange: the tokens' q8_1 rows and, per row, the local expert ids of its picks on that rank (-1 for the
     others) and their weights (0 for the others);
  4. local experts: expert_fn(rows, ids, w) -> per received row the weighted partial sum of its picks on this rank;
  5. return exchange of the partial rows (fp32), and each token's output = the partials of the ranks it went to, added
     in rank order (no atomics: a rank's rows come back in the token order they were sent in).

torch.distributed is the plumbing: NCCL over NVLink on B200s, gloo for the CPU tests.  expert_fn is the local
compute: the tensor-core prefill path on a GPU (gpu_expert_fn), anything with the same contract in tests.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist


class EPPlan:
    """Where each local token goes: per destination rank the tokens (ascending) and their picks on that rank (local
    expert ids: the expert's index among its rank's experts)."""

    def __init__(self, ids: torch.Tensor, w: torch.Tensor, n_expert: int, world: int, cyclic: bool = False):
        T, K = ids.shape
        if n_expert % world:
            raise ValueError(f"expert parallelism: {n_expert} experts do not split evenly over {world} ranks")
        per = n_expert // world
        if cyclic:
            dest = torch.remainder(ids.long(), world)                                   # [T, K]
            local = torch.div(ids.long(), world, rounding_mode="floor")
        else:
            dest = torch.div(ids.long(), per, rounding_mode="floor")
            local = ids.long() - dest * per
        self.world = world
        self.per = per
        ranks = torch.arange(world, device=ids.device).view(world, 1, 1)
        hit = dest.unsqueeze(0) == ranks                                              # [G, T, K]
        mask = hit.any(dim=2)                                                         # [G, T]
        self.counts = mask.sum(dim=1)                                                 # [G]
        toks = [torch.nonzero(mask[d], as_tuple=False).view(-1) for d in range(world)]
        self.send_tok = toks                                                          # per destination, ascending
        self.send_idx = torch.cat(toks) if T else torch.zeros(0, dtype=torch.long, device=ids.device)
        lid = local.unsqueeze(0).expand(world, T, K)                                  # local ids on each rank
        lid = torch.where(hit, lid, torch.full_like(lid, -1))
        wl = torch.where(hit, w.unsqueeze(0).expand(world, T, K), torch.zeros_like(w).unsqueeze(0).expand(world, T, K))
        self.send_ids = torch.cat([lid[d][toks[d]] for d in range(world)]).to(torch.int32)      # [S, K]
        self.send_w = torch.cat([wl[d][toks[d]] for d in range(world)]).to(torch.float32)       # [S, K]


def _a2a(out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits, group):
    dist.all_to_all_single(out, inp.contiguous(), output_split_sizes=out_splits, input_split_sizes=in_splits,
                           group=group)
    return out


def ep_forward(xq: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, n_expert: int, n_embd: int, expert_fn,
               group=None, cyclic: bool = False) -> torch.Tensor:
    """The routed part of the layer for this rank's T tokens: xq [T, row bytes] (uint8 q8_1 rows), ids / w [T, K] ->
    fp32 [T, n_embd].  expert_fn(rows uint8 [R, row bytes], ids int32 [R, K] (local expert, -1 = none), w [R, K]) ->
    fp32 [R, n_embd].  cyclic: expert e lives on rank e % G as local expert e // G (else on rank e // (E / G))."""
    world = dist.get_world_size(group)
    plan = EPPlan(ids, w, n_expert, world, cyclic)
    dev = xq.device
    send_counts = plan.counts.to(torch.int64)
    recv_counts = torch.empty_like(send_counts)
    _a2a(recv_counts, send_counts, None, None, group)
    s_split = [int(c) for c in send_counts.cpu()]
    r_split = [int(c) for c in recv_counts.cpu()]
    R = sum(r_split)
    K = ids.shape[1]
    rows = _a2a(torch.empty((R, xq.shape[1]), dtype=xq.dtype, device=dev), xq[plan.send_idx], r_split, s_split, group)
    rids = _a2a(torch.empty((R, K), dtype=torch.int32, device=dev), plan.send_ids, r_split, s_split, group)
    rw = _a2a(torch.empty((R, K), dtype=torch.float32, device=dev), plan.send_w, r_split, s_split, group)
    partial = expert_fn(rows, rids, rw) if R else torch.zeros((0, n_embd), dtype=torch.float32, device=dev)
    back = _a2a(torch.empty((sum(s_split), n_embd), dtype=torch.float32, device=dev), partial, s_split, r_split, group)
    out = torch.zeros((ids.shape[0], n_embd), dtype=torch.float32, device=dev)
    o = 0
    for d in range(world):   # rank order, each rank's rows in token order: a fixed summation order
        n = s_split[d]
        if n:
            out[plan.send_tok[d]] += back[o:o + n]
        o += n
    return out


def gpu_expert_fn(L, blobs, blob_stride: int, act: int, limit: float = float("inf"), stream=None):
    """The local experts on the tensor cores: dispatch of the received picks, grouped gate/up + down, and the weighted
    partial sum per received row.  blobs: this rank's E / G expert blobs."""
    import tinystrata_b200 as T

    n_local = blobs.shape[0]

    def fn(rows, rids, rw):
        R, K = rids.shape
        bounds, row_ent, row_tok, rinv = T.moe_dispatch(rids, n_local, stream=stream)
        n = int(bounds[-1].item())
        xa = T.mmq_from_q8_1(rows, int(L.n_embd), row_src=row_tok, n_rows=n, stream=stream)
        h = T.moe_prefill_gu(L, blobs, blob_stride, bounds, n_local, n, xa, act, limit, stream=stream)
        parts = T.moe_prefill_down(L, blobs, blob_stride, bounds, n_local, n, h, stream=stream)
        valid = rinv.view(R, K) >= 0
        idx = torch.where(valid, rinv.view(R, K), torch.zeros_like(rinv.view(R, K))).long()
        gathered = parts[idx.view(-1)].view(R, K, -1)
        wk = torch.where(valid, rw, torch.zeros_like(rw))
        acc = gathered[:, 0] * wk[:, 0:1]
        for k in range(1, K):   # pick order, as the combine does
            acc = torch.addcmul(acc, gathered[:, k], wk[:, k:k + 1])
        return acc

    return fn


class ExpertParallel:
    """The device path of expert parallelism (libtsb_moe.so's tsb_ep_*): plan, pack, unpack, local experts, partial
    sums and the ordered gather as kernels, the exchanges as NCCL point-to-point calls on the library's own
    communicator, one host synchronisation per step (the row counts).  The same placement and per-token result as
    ep_forward above, which stays the CPU statement of the algorithm (gloo tests).

    Collective: every rank of `group` constructs it (the NCCL id travels through torch.distributed, the plumbing).
    blobs: this rank's n_expert / G expert blobs in local order (expert e = local l: cyclic e = l * G + rank).

    One step: dispatch(xq, ids, w) queues the exchanges and returns; work the caller queues on the same stream next
    (the shared expert) runs while the rows travel; combine(out, ...) computes the local experts per micro-batch as
    their rows arrive and writes out = (out if accumulate) + the partials in rank order + sigmoid(sgate) shared."""

    def __init__(self, L, blobs, blob_stride: int, n_expert: int, n_used: int, act: int, limit: float = float("inf"),
                 max_tokens: int = 8192, cyclic: bool = True, group=None):
        from . import _check, lib
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        uid = (C.c_char * 128)()
        if self.rank == 0:
            _check(lib().tsb_ep_unique_id(uid), "ep_unique_id")
        obj = [bytes(uid)]
        dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        uid = (C.c_char * 128).from_buffer_copy(obj[0])
        self.L = L
        self.blobs = blobs                       # held: the library keeps the pointer
        self.h = C.c_void_p()
        _check(lib().tsb_ep_create(uid, self.rank, self.world, C.byref(L), C.c_void_p(blobs.data_ptr()), blob_stride,
                                   n_expert, n_used, int(cyclic), max_tokens, act, limit, C.byref(self.h)),
               "ep_create")

    def dispatch(self, xq, ids, w, micro_batches: int = 2, stream=None):
        from . import _check, _stream, lib
        T = ids.shape[0]
        _check(lib().tsb_ep_dispatch(self.h, C.c_void_p(xq.data_ptr()) if T else None,
                                     C.c_void_p(ids.data_ptr()) if T else None, C.c_void_p(w.data_ptr()) if T else None,
                                     T, micro_batches, _stream(stream)), "ep_dispatch")

    def combine(self, out, accumulate: bool = False, shared=None, sgate=None, sg_stride: int = 1, bf16: bool = False,
                stream=None):
        from . import _check, _ptr, _stream, lib
        _check(lib().tsb_ep_combine(self.h, _ptr(out) if out is not None and out.numel() else None, int(accumulate),
                                    _ptr(shared), _ptr(sgate), sg_stride, int(bf16), _stream(stream)), "ep_combine")
        return out

    def synchronize(self):
        """Wait (bounded) for every exchange issued so far; TsbError (status -6) when a peer never answers."""
        from . import _check, lib
        _check(lib().tsb_ep_synchronize(self.h), "ep_synchronize")

    def set_timeout(self, seconds: float):
        from . import _check, lib
        _check(lib().tsb_ep_set_timeout_ns(self.h, int(seconds * 1e9)), "ep_set_timeout_ns")

    def stats(self) -> dict:
        from . import _check, lib
        a, b, c = C.c_int64(), C.c_int64(), C.c_int64()
        _check(lib().tsb_ep_stats(self.h, C.byref(a), C.byref(b), C.byref(c)), "ep_stats")
        return {"rows_sent": a.value, "rows_received": b.value, "picks": c.value}

    def close(self):
        from . import _check, lib
        if self.h:
            h, self.h = self.h, C.c_void_p()
            _check(lib().tsb_ep_destroy(h), "ep_destroy")

    def __del__(self):
        try:
            if self.h:
                self.close()
        except Exception:
            pass
