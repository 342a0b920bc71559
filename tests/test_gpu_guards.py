"""The device-side guards, exercised on purpose without faulting the GPU.

* A bounded wait that runs out: with a short bound (20 ms) and CTA 0 of the fused decode kernel told to withhold its
  layer-0 router logits, every other CTA's wait for them gives up; the kernel returns, the error record names the
  routing wait's site, and the same context then runs a normal step whose output equals a fresh run.
* Device counts beyond the caller's capacities: a group count far above cap_groups is clamped by the grouped expert
  kernels (nothing past the caller's tables is read or written), the clamp is reported in the device error word, and
  the result equals the unclamped call's.
"""
import numpy as np
import pytest
import torch

import tinystrata_b200 as T
from oracle import oracle as O
from tinystrata_b200 import synth

pytestmark = pytest.mark.gpu

SITE_ROUTING_LOGITS = 0x345   # the routing warps' wait for every CTA's router logits (tsb_decode.cuh)
SITE_GU_GROUPS = 0x110        # k_expert_gu: the device group count exceeded cap_groups


def test_bounded_wait_gives_up_and_context_survives(cuda):
    cfg = synth.QWEN
    st = synth.device_layers(cfg, 2, seed=21, device=cuda)
    D = T.DecodeStack(cfg, st["blobs"], st["routers"], st["sh_blobs"], n_tok=1)
    x0 = torch.from_numpy(synth.rms_normed(np.random.default_rng(21), 1, cfg["n_embd"])).to(cuda)
    good = x0.clone()
    D.forward(good)
    torch.cuda.synchronize()
    assert D.error() == 0
    ids_good = D.ids.clone()

    x = x0.clone()
    T.set_wait_limit_ns(20_000_000)
    T.decode_set_debug(1)   # CTA 0 withholds its layer-0 logits: nobody can route
    try:
        D.forward(x)
        torch.cuda.synchronize()
    finally:
        T.decode_set_debug(0)
        T.set_wait_limit_ns(2_000_000_000)
    assert D.error() == SITE_ROUTING_LOGITS, D.error_detail

    # the context is usable: the same step again gives the first run's output and routing
    x = x0.clone()
    D.forward(x)
    torch.cuda.synchronize()
    assert D.error() == 0
    assert torch.equal(x, good)
    assert torch.equal(D.ids, ids_good)
    assert T.device_error() == 0


def test_group_count_beyond_capacity_is_clamped(cuda):
    cfg = synth.QWEN
    H, F, K = cfg["n_embd"], cfg["n_ff"], cfg["n_used"]
    layer = synth.make_layer(cfg, 31, n_expert=16)
    rng = np.random.default_rng(31)
    ids = np.stack([rng.choice(16, K, replace=False) for _ in range(2)]).astype(np.int32)
    xq = torch.from_numpy(O.quantize_q8_1(synth.rms_normed(rng, 2, H))).to(cuda)
    blobs = torch.from_numpy(layer["blobs"]).to(cuda)
    L = T.native_expert_layout(cfg["gu_type"], cfg["d_type"], H, F)
    g = T.moe_group(torch.from_numpy(ids).to(cuda), 16, blobs, int(L.bytes))
    n_ent = 2 * K
    scratch = torch.empty(T.native_expert_scratch_bytes(n_ent, F) // 4, dtype=torch.float32, device=cuda)
    ref = torch.empty((n_ent, H), device=cuda)
    T.native_expert_grouped(L, g, n_ent, n_ent, xq, scratch, ref)
    torch.cuda.synchronize()
    assert T.device_error() == 0
    n_real = int(g.n_groups.item())

    g.n_groups.fill_(1 << 20)   # a count far past every table the caller sized for n_real groups
    out = torch.full_like(ref, float("nan"))
    T.native_expert_grouped(L, g, n_real, n_ent, xq, scratch, out)
    torch.cuda.synchronize()
    assert T.device_error() == SITE_GU_GROUPS
    assert torch.equal(out, ref)
