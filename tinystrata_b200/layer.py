"""The engines' MoE block as a sequence of expert-layer entry points (the reference's call stacks A and C:
src/qwen35/q36_engine.cu:2821-2925 and src/gemma4/engine.cpp:2436-2457), over device buffers owned here.

Qwen decode (router_mode "softmax"): router GEMV (+ shared-gate row) -> native_router_topk -> moe_group ->
native_expert_grouped -> shared expert (one more group) -> moe_combine (x += ..., next RMS + q8_1).
Gemma / LFM: route_rows (softmax-scaled / sigmoid+bias) and the GELU-tanh / clamped-SwiGLU activations, moe_sum.
"""
from __future__ import annotations

import torch

import numpy as np

from . import (ACT_SWIGLU, Groups, Q8_1_BYTES, decode_act_desc, lib, moe_combine, moe_decode_act, moe_group,
               moe_group_staged, moe_sum, native_expert_grouped, native_expert_layout, native_expert_scratch_bytes,
               native_router_topk, route_rows, router_logits_f32, staged_load, staged_rebalance)


class StagedExperts:
    """A layer's experts in pinned host memory, n_slots of them resident in HBM slots: the reference's hybrid-mode
    state of a layer (q36_engine.cu: slot_of / exp_in_slot / score, k_group_hy 423-452, rebalance 3215-3265).

    host_blobs: pinned uint8 [E, stride] (every expert); resident: the experts to place first (default 0..n_slots-1).
    Entries of experts without a slot are fetched by the GPU into a stage buffer of min(max_entries, E) blobs."""

    def __init__(self, host_blobs: torch.Tensor, blob_bytes: int, n_slots: int, max_entries: int, device,
                 resident=None, stream=None):
        assert host_blobs.is_pinned() and host_blobs.dim() == 2 and host_blobs.dtype == torch.uint8
        self.host = host_blobs
        self.E, self.stride = host_blobs.shape[0], int(host_blobs.stride(0))
        self.blob_bytes, self.n_slots = int(blob_bytes), int(n_slots)
        assert 0 <= self.n_slots <= self.E
        self.slots = torch.empty((max(self.n_slots, 1), self.stride), dtype=torch.uint8, device=device)
        self.stage_cap = min(max_entries, self.E)
        self.stage = torch.empty((self.stage_cap, self.stride), dtype=torch.uint8, device=device)
        self.counts = torch.zeros(self.E, dtype=torch.int32, device=device)
        self.score = np.zeros(self.E, np.float64)
        self.slot_of = np.full(self.E, -1, np.int32)
        first = np.arange(self.n_slots, dtype=np.int32) if resident is None else np.asarray(resident, np.int32)
        assert first.size == self.n_slots and len(set(first.tolist())) == first.size
        self.exp_in_slot = first.copy()
        self.slot_of[first] = np.arange(self.n_slots, dtype=np.int32)
        self.slot_of_d = torch.from_numpy(self.slot_of).to(device)
        staged_load(self.host, self.slots, self.stride, self.blob_bytes, first, np.arange(self.n_slots, dtype=np.int32),
                    self.E, self.n_slots, stream=stream)
        self.swaps = 0

    def group(self, ids, groups: Groups, stream=None) -> Groups:
        return moe_group_staged(ids, self.E, self.slot_of_d, self.n_slots, self.slots, self.host, self.stride,
                                self.stage, self.stage_cap, groups, counts=self.counts, stream=stream)

    def rebalance(self, max_swaps: int, stream=None) -> int:
        """Between steps: the usage counts into the scores, the reference's placement, the moved blobs and the new
        slot table uploaded on `stream` (in that order).  Reads the counts (a host synchronisation)."""
        cs = torch.cuda.current_stream() if stream is None else stream
        with torch.cuda.stream(cs):
            self.score += self.counts.cpu().numpy().astype(np.float64)
            self.counts.zero_()
            me, ms = staged_rebalance(self.score, self.slot_of, self.exp_in_slot, max_swaps)
            if len(me):
                staged_load(self.host, self.slots, self.stride, self.blob_bytes, me, ms, self.E, self.n_slots,
                            stream=cs)
                self.slot_of_d.copy_(torch.from_numpy(self.slot_of))
        self.swaps += len(me)
        return len(me)


class MoELayer:
    """One MoE layer's device weights and work buffers for up to max_tokens tokens.

    blobs: uint8 [E, blob_bytes] (the layer's expert blobs); router: fp32 [E (+1), H]; sh_blob: uint8 [bytes] or None.
    """

    def __init__(self, cfg: dict, blobs: torch.Tensor | None, router: torch.Tensor, sh_blob: torch.Tensor | None = None,
                 max_tokens: int = 16, escale=None, bias=None, staged: StagedExperts | None = None):
        self.cfg = cfg
        self.H, self.F, self.E, self.K = cfg["n_embd"], cfg["n_ff"], cfg["n_expert"], cfg["n_used"]
        self.dev = router.device
        self.blobs, self.router, self.sh_blob = blobs, router.contiguous(), sh_blob
        self.staged = staged
        self.L = native_expert_layout(cfg["gu_type"], cfg["d_type"], self.H, self.F)
        if staged is not None:
            assert blobs is None and staged.E == self.E and staged.blob_bytes == self.L.bytes
            self.stride = staged.stride
        else:
            assert blobs.shape[-1] == self.L.bytes
            self.stride = int(blobs.stride(0)) if blobs.dim() > 1 else int(self.L.bytes)
        self.escale, self.bias = escale, bias
        self.max_tokens = max_tokens
        n_ent = max_tokens * self.K
        dev = self.dev
        self.rows = self.router.shape[0]
        self.logits = torch.empty((max_tokens, self.rows), dtype=torch.float32, device=dev)
        self.ids = torch.empty((max_tokens, self.K), dtype=torch.int32, device=dev)
        self.w = torch.empty((max_tokens, self.K), dtype=torch.float32, device=dev)
        self.groups = Groups(n_ent, dev)
        self.scratch = torch.empty(native_expert_scratch_bytes(n_ent, max(self.F, cfg.get("sh_n_ff") or 0)) // 4 + 64,
                                   dtype=torch.float32, device=dev)
        self.parts = torch.empty((n_ent, self.H), dtype=torch.float32, device=dev)
        self.Ls = None
        if sh_blob is not None and cfg.get("sh_n_ff"):
            self.Ls = native_expert_layout(cfg["sh_gu_type"], cfg["sh_d_type"], self.H, cfg["sh_n_ff"])
            self.shared = torch.empty((max_tokens, self.H), dtype=torch.float32, device=dev)
            self.sh_groups = Groups(max_tokens, dev)
            self.sh_groups.grp_ptr[0] = sh_blob.data_ptr()
            self.sh_groups.ent_dst.copy_(torch.arange(max_tokens, dtype=torch.int32))
            self.sh_groups.ent_tok.copy_(torch.arange(max_tokens, dtype=torch.int32))
            self.sh_groups.n_groups.fill_(1)
            self._sh_T = -1

    def forward_fused(self, x: torch.Tensor, h: torch.Tensor, hq: torch.Tensor, stream=None):
        """Gemma / LFM decode (router_mode softmax_scaled or sigmoid) in one launch (tsb_moe_decode_act): the same
        values as forward bit for bit -- x += the picks' weighted sum (+ the shared MLP's output); ids, w, shared and
        the logits (self.fused_logits) as forward leaves them."""
        import ctypes as C
        cfg = self.cfg
        assert cfg["router_mode"] in ("softmax_scaled", "sigmoid") and self.staged is None
        T = x.shape[0]
        shared = self.Ls is not None
        if getattr(self, "_act_ws", None) is None:
            big = decode_act_desc(cfg, self.max_tokens, shared)
            n = int(lib().tsb_moe_decode_act_workspace_bytes(C.byref(big)))
            self._act_ws = torch.empty(n // 4 + 64, dtype=torch.float32, device=self.dev)
        d = decode_act_desc(cfg, T, shared)
        sig = cfg["router_mode"] == "sigmoid"
        moe_decode_act(d, self.router, h, hq, self.blobs, self.stride, x, self._act_ws,
                       bias=self.bias if sig else None, escale=None if sig else self.escale,
                       sh_blob=self.sh_blob if shared else None, sh_out=self.shared[:T] if shared else None,
                       ids=self.ids[:T], w=self.w[:T], accumulate=True, stream=stream)
        self.fused_logits = self._act_ws[:T * self.E].view(T, self.E)
        if shared:
            x.add_(self.shared[:T])
        return x

    def _shared_for(self, T: int):
        if self._sh_T != T:
            self.sh_groups.grp_start[0] = 0
            self.sh_groups.grp_start[1] = T
            self._sh_T = T

    def forward(self, x: torch.Tensor, h: torch.Tensor, hq: torch.Tensor, h_next: torch.Tensor | None = None,
                hq_next: torch.Tensor | None = None, eps: float = 1e-6, stream=None, prior: torch.Tensor | None = None):
        """x += MoE(h) for T = x.shape[0] tokens; h (fp32) feeds the router, hq (q8_1) the experts.  With h_next /
        hq_next the next layer's RMS-normed input and its q8_1 image are written too.  prior (optional, [T, E]) is
        added to the router logits before the softmax, as the fused decode path's logit_prior."""
        cfg = self.cfg
        T = x.shape[0]
        K, E = self.K, self.E
        logits = self.logits[:T]
        router_logits_f32(self.router, h, logits, ld=self.rows, stream=stream)
        if prior is not None:
            with torch.cuda.stream(stream) if stream is not None else torch.cuda.stream(torch.cuda.current_stream()):
                logits[:, :E].add_(prior)
        mode = cfg["router_mode"]
        if mode == "softmax":
            native_router_topk(logits, K, E, self.ids[:T], self.w[:T], stream=stream)
        elif mode == "softmax_scaled":
            ids, w = route_rows(logits[:, :E].contiguous(), K, 0, cfg.get("in_scale", 1.0), None, self.escale, True,
                                0.0, stream=stream)
            self.ids[:T].copy_(ids)
            self.w[:T].copy_(w)
        else:
            ids, w = route_rows(logits[:, :E].contiguous(), K, 1, 1.0, self.bias, None, True, cfg.get("w_scale", 0.0),
                                stream=stream)
            self.ids[:T].copy_(ids)
            self.w[:T].copy_(w)
        if self.staged is not None:
            self.staged.group(self.ids[:T], self.groups, stream=stream)
        else:
            moe_group(self.ids[:T], E, self.blobs, self.stride, self.groups, stream=stream)
        n_ent = T * K
        native_expert_grouped(self.L, self.groups, n_ent, n_ent, hq, self.scratch, self.parts, cfg["act"],
                              cfg.get("limit", float("inf")), stream=stream)
        shared = None
        if self.Ls is not None:
            self._shared_for(T)
            native_expert_grouped(self.Ls, self.sh_groups, 1, T, hq, self.scratch, self.shared[:T],
                                  cfg.get("sh_act", cfg["act"]), cfg.get("limit", float("inf")), stream=stream)
            shared = self.shared[:T]
        if mode == "softmax":
            sg = logits[:, E:] if cfg.get("shared_gate") else None
            moe_combine(x, self.parts, self.w[:T], K, shared, sg, self.rows, h=h_next, hq=hq_next, eps=eps,
                        stream=stream)
        else:
            moe_sum(self.parts, self.w[:T], x, K, stream=stream)
            if shared is not None:
                x.add_(shared)
        return x


class PrefillLayer:
    """One MoE layer's prompt path for up to max_tokens tokens on the tensor cores (the reference's call stack C, the
    prompt branch: router, routing, permutation, MMQ gate/up + activation, MMQ down, shared expert, moe_sum;
    src/gemma4/engine.cpp:2436-2457 with src/prefill/moe_mmq.cu:334-384).  Weights as MoELayer's, in any format the
    tensor-core path takes (Q4_0, Q8_0, Q4_K, Q6_K, IQ3_XXS, IQ3_S)."""

    def __init__(self, cfg: dict, blobs, router, sh_blob=None, max_tokens: int = 8192, escale=None, bias=None):
        import torch
        from . import MmqAct, native_expert_layout
        self.cfg = cfg
        self.H, self.F, self.E, self.K = cfg["n_embd"], cfg["n_ff"], cfg["n_expert"], cfg["n_used"]
        self.blobs, self.router, self.sh_blob = blobs, router.contiguous(), sh_blob
        self.L = native_expert_layout(cfg["gu_type"], cfg["d_type"], self.H, self.F)
        self.stride = int(blobs.stride(0))
        self.escale, self.bias = escale, bias
        dev = blobs.device
        T, K, H = max_tokens, self.K, self.H
        self.max_tokens = T
        self.rows = self.router.shape[0]         # E, or E + 1 with Qwen's shared-expert gate row
        self.logits = torch.empty((T, self.rows), dtype=torch.float32, device=dev)
        self._ids = torch.empty((T, self.K), dtype=torch.int32, device=dev)
        self._w = torch.empty((T, self.K), dtype=torch.float32, device=dev)
        self.xa = MmqAct(T * K, H, dev)            # the routed rows in expert order (tensor-core layout)
        self.ha = MmqAct(T * K, self.F, dev)       # their hidden vectors
        self.parts = torch.empty((T * K, H), dtype=torch.float32, device=dev)
        self.Ls = None
        if sh_blob is not None and cfg.get("sh_n_ff"):
            self.Ls = native_expert_layout(cfg["sh_gu_type"], cfg["sh_d_type"], H, cfg["sh_n_ff"])
            self.xs = MmqAct(T, H, dev)
            self.hs = MmqAct(T, cfg["sh_n_ff"], dev)
            self.shared = torch.empty((T, H), dtype=torch.float32, device=dev)

    def forward(self, x, h, stream=None, h_next=None, hq_next=None, eps: float = 1e-6, prior=None):
        """x += MoE(h) for T = x.shape[0] tokens (h fp32 [T, H], the layer's normed input).  Qwen's routing
        (router_mode "softmax": softmax top-k, q36_engine.cu:2821-2840) gates the shared expert by the sigmoid of the
        router's extra row, and with h_next / hq_next also writes the next layer's normed input and its q8_1 image
        (k_moe_out, q36_engine.cu:307-332); Gemma / LFM2 route by route_rows.  prior (optional, [T, E]) is added to
        the router logits before routing, as MoELayer's."""
        from . import (MmqAct, mmq_quantize, moe_combine, moe_dispatch, moe_prefill_down, moe_prefill_gu,
                       native_router_topk, route_rows, router_logits_f32)
        cfg = self.cfg
        T = x.shape[0]
        K, E = self.K, self.E
        mode = cfg["router_mode"]
        logits = router_logits_f32(self.router, h, self.logits[:T], ld=self.rows, stream=stream)
        if prior is not None:
            with torch.cuda.stream(stream) if stream is not None else torch.cuda.stream(torch.cuda.current_stream()):
                logits[:, :E].add_(prior)
        if mode == "softmax":
            ids, w = native_router_topk(logits, K, E, self._ids[:T], self._w[:T], stream=stream)
        elif mode == "softmax_scaled":
            ids, w = route_rows(logits[:, :E].contiguous(), K, 0, cfg.get("in_scale", 1.0), None, self.escale, True,
                                0.0, stream=stream)
        else:
            ids, w = route_rows(logits[:, :E].contiguous(), K, 1, 1.0, self.bias, None, True, cfg.get("w_scale", 0.0),
                                stream=stream)
        bounds, row_ent, row_tok, rinv = moe_dispatch(ids, E, stream=stream)
        n = T * K
        xa = self.xa if T == self.max_tokens else MmqAct(n, self.H, x.device, buf=self.xa._store)
        ha = self.ha if T == self.max_tokens else MmqAct(n, self.F, x.device, buf=self.ha._store)
        mmq_quantize(h, row_src=row_tok, n_rows=n, out=xa, stream=stream)
        moe_prefill_gu(self.L, self.blobs, self.stride, bounds, E, n, xa, cfg["act"], cfg.get("limit", float("inf")),
                       h=ha, stream=stream)
        parts = moe_prefill_down(self.L, self.blobs, self.stride, bounds, E, n, ha, out=self.parts[:n], stream=stream)
        shared = None
        if self.Ls is not None:
            FS = self.cfg["sh_n_ff"]
            xs = self.xs if T == self.max_tokens else MmqAct(T, self.H, x.device, buf=self.xs._store)
            hs = self.hs if T == self.max_tokens else MmqAct(T, FS, x.device, buf=self.hs._store)
            mmq_quantize(h, n_rows=T, out=xs, stream=stream)
            moe_prefill_gu(self.Ls, self.sh_blob, 0, None, 1, T, xs, cfg.get("sh_act", cfg["act"]),
                           cfg.get("limit", float("inf")), h=hs, stream=stream)
            shared = moe_prefill_down(self.Ls, self.sh_blob, 0, None, 1, T, hs, out=self.shared[:T], stream=stream)
        sg = logits[:, E:] if mode == "softmax" and cfg.get("shared_gate") and shared is not None else None
        moe_combine(x, parts, w, K, shared=shared, sgate=sg, sg_stride=self.rows, prow=rinv, h=h_next, hq=hq_next,
                    eps=eps, stream=stream)
        self.ids, self.w, self.rinv, self.bounds = ids, w, rinv, bounds
        return x
