"""Parity at the benchmark configurations' own shapes (all experts of the layer resident, full token counts):

* Qwen3.6-shaped layer (hidden 2048, 256 IQ3_XXS experts, top-8 softmax, sigmoid-gated Q8_0 shared expert), T = 512,
  through both the decode-kernel layer (MoELayer) and the tensor-core prompt layer (PrefillLayer), every token against
  the oracle's restatement of call stack A (q36_engine.cu:2821-2925).
* Gemma-4-shaped prefill (hidden 2816, 128 Q4_0 experts, top-8, GELU-tanh, Q4_0 dense shared FFN), T = 8192.
* LFM2.5-shaped prefill (hidden 2048, 64 experts, Q4_K gate/up + Q6_K down, top-4 sigmoid + bias), T = 2048.
* The expert-parallel Qwen layer (IQ3_XXS gate/up, IQ3_S down) with Zipf(1.1)-skewed router logits, T = 4096 on one
  device (the per-rank work of the sharded run).

At the full prompt sizes the routing of every token is checked bit for bit against the oracle's routing of the same
logits; a seeded sample of tokens is checked against the oracle's whole layer; and every token's output is checked
against the decode-kernel layer on the same weights (whose grouped expert kernels are bit for bit the reference's,
test_gpu_parity), a second implementation that shares no product code with the tensor-core path.  Layer tolerance:
max-abs <= 1e-2 of the RMS and cosine >= 0.9999.
"""
import numpy as np
import pytest
import torch

import tinystrata_b200 as T
from oracle import oracle as O
from tinystrata_b200 import synth
from tinystrata_b200.layer import MoELayer, PrefillLayer

pytestmark = pytest.mark.gpu

ERR, COS = 1e-2, 0.9999


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def tol(mine, ref):
    mine = np.asarray(mine, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    rms = np.sqrt(np.mean(ref ** 2))
    return float(np.abs(mine - ref).max() / rms), float(mine @ ref / (np.linalg.norm(mine) * np.linalg.norm(ref)))


def oracle_routing(cfg, layer, logits):
    E, K = cfg["n_expert"], cfg["n_used"]
    if cfg["router_mode"] == "softmax":
        ids, w, _ = O.router_softmax_topk(logits[:, :E], K, E)
    elif cfg["router_mode"] == "softmax_scaled":
        ids, w = O.route_rows(logits[:, :E], K, 0, cfg.get("in_scale", 1.0), None, layer.get("escale"), True, 0.0)
    else:
        ids, w = O.route_rows(logits[:, :E], K, 1, 1.0, layer.get("bias"), None, True, cfg.get("w_scale", 0.0))
    return ids, w


def layers_for(cfg, layer, T_tok):
    kw = dict(escale=dev(layer["escale"]) if layer.get("escale") is not None else None,
              bias=dev(layer["bias"]) if layer.get("bias") is not None else None)
    sh = dev(layer["sh_blob"]) if layer.get("sh_blob") is not None else None
    blobs, router = dev(layer["blobs"]), dev(layer["router"])
    P = PrefillLayer(cfg, blobs, router, sh, max_tokens=T_tok, **kw)
    M = MoELayer(cfg, blobs, router, sh, max_tokens=T_tok, **kw)
    return P, M


def run_both(P, M, h, prior=None):
    T_tok, H = h.shape
    hd = dev(h)
    xp = torch.zeros((T_tok, H), device="cuda")
    P.forward(xp, hd, prior=prior)
    xm = torch.zeros((T_tok, H), device="cuda")
    M.forward(xm, hd, T.quantize_q8_1_rows(hd), prior=prior)
    torch.cuda.synchronize()
    assert T.device_error() == 0
    return xp.cpu().numpy(), xm.cpu().numpy()


def check_layer(cfg, layer, h, prior=None, n_sample=None, seed=0):
    T_tok = h.shape[0]
    P, M = layers_for(cfg, layer, T_tok)
    xp, xm = run_both(P, M, h, prior)
    logits = P.logits[:T_tok].cpu().numpy()
    assert np.array_equal(logits, M.logits[:T_tok].cpu().numpy())       # one router kernel, same input (+ prior)
    ids, w = oracle_routing(cfg, layer, logits)
    assert np.array_equal(P.ids[:T_tok].cpu().numpy(), ids)
    assert np.array_equal(M.ids[:T_tok].cpu().numpy(), ids)
    assert np.allclose(P.w[:T_tok].cpu().numpy(), w, rtol=2e-6, atol=0)
    # every token: the tensor-core layer against the decode-kernel layer
    err, cos = tol(xp, xm)
    assert err <= ERR and cos >= COS, ("prefill vs decode kernels", err, cos)
    # the oracle's whole layer on every token, or on a seeded sample
    rows = np.arange(T_tok) if n_sample is None else np.sort(
        np.random.default_rng(seed).choice(T_tok, n_sample, replace=False))
    ref = O.moe_layer(layer, h[rows], logits=np.ascontiguousarray(logits[rows]))
    assert np.array_equal(ref["ids"], ids[rows])
    for name, mine in (("prefill", xp[rows]), ("decode kernels", xm[rows])):
        err, cos = tol(mine, ref["out"])
        assert err <= ERR and cos >= COS, (name, err, cos)
    return P, M


def test_qwen_layer_T512_every_token(cuda):
    cfg = synth.QWEN
    layer = synth.make_layer(cfg, seed=0)
    h = synth.rms_normed(np.random.default_rng(0), 512, cfg["n_embd"])
    check_layer(cfg, layer, h)


def test_gemma_prefill_T8192(cuda):
    cfg = synth.GEMMA
    layer = synth.make_layer(cfg, seed=2)
    h = synth.rms_normed(np.random.default_rng(2), 8192, cfg["n_embd"])
    P, _ = check_layer(cfg, layer, h, n_sample=96, seed=2)
    # every expert of the 128 received rows (the full-size case exercises every group of the grouped products)
    assert int((P.bounds[1:] - P.bounds[:-1]).gt(0).sum()) == cfg["n_expert"]


def test_lfm_prefill_T2048(cuda):
    cfg = synth.LFM
    layer = synth.make_layer(cfg, seed=3)
    h = synth.rms_normed(np.random.default_rng(3), 2048, cfg["n_embd"])
    check_layer(cfg, layer, h, n_sample=128, seed=3)


def test_qwen_ep_prefill_zipf_T4096(cuda):
    cfg = synth.QWEN_EP
    E = cfg["n_expert"]
    layer = synth.make_layer(cfg, seed=4)
    h = synth.rms_normed(np.random.default_rng(4), 4096, cfg["n_embd"])
    prior = torch.tensor(-1.1 * np.log(np.arange(1, E + 1)), dtype=torch.float32, device="cuda")
    prior = prior.expand(4096, E).contiguous()
    P, _ = check_layer(cfg, layer, h, prior=prior, n_sample=64, seed=4)
    counts = (P.bounds[1:] - P.bounds[:-1]).cpu().numpy()
    assert counts[0] > 4 * counts[E // 2]     # the skew reached the dispatch (hot experts hold many more rows)
