"""Parity at the benchmark configurations' own shapes (all experts of the layer resident, full token counts):

* Qwen3.6-shaped layer (hidden 2048, 256 IQ3_XXS experts, top-8 softmax, sigmoid-gated Q8_0 shared expert), T = 512,
  through both the decode-kernel layer (MoELayer) and the tensor-core prompt layer (PrefillLayer), against the
  oracle's restatement of call stack A (q36_engine.cu:2821-2925).
* Gemma-4-shaped prefill (hidden 2816, 128 Q4_0 experts, top-8, GELU-tanh, Q4_0 dense shared FFN), T = 8192.
* LFM2.5-shaped prefill (hidden 2048, 64 experts, Q4_K gate/up + Q6_K down, top-4 sigmoid + bias), T = 2048.
* The expert-parallel Qwen layer (IQ3_XXS gate/up, IQ3_S down) with Zipf(1.1)-skewed router logits, T = 4096 on one
  device (the per-rank work of the sharded run).

Routing of every token against the oracle's routing of the same logits (bit for bit but for near ties of the two
expf implementations); every token's output against the decode-kernel layer on the same weights (whose grouped expert
kernels are bit for bit the reference's, test_gpu_parity), a second implementation sharing no product code with the
tensor-core path; a seeded sample of tokens against fp64 on the layer's own hidden codes (the north star's bar:
max-abs <= 1e-2 of the RMS, cosine >= 0.9999), its hidden codes against the oracle's, and the oracle's whole layer.
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


def routing_vs_oracle(cfg, layer, logits, ids_gpu):
    """The GPU's picks against the oracle's on the same logits.  The oracle's libm expf and CUDA's expf may differ in
    the last bit, so a row may differ where two candidates' probabilities tie within a few ulps; such rows are allowed
    (at most one in a thousand), any other difference fails.  Returns the oracle's ids and weights and the rows whose
    picks agree."""
    ids, w = oracle_routing(cfg, layer, logits)
    bad = np.nonzero(np.any(ids != ids_gpu, axis=1))[0]
    E = cfg["n_expert"]
    for r in bad:
        lg = logits[r, :E].astype(np.float64) * (cfg.get("in_scale", 1.0) if cfg["router_mode"] == "softmax_scaled"
                                                 else 1.0)
        if cfg["router_mode"] == "sigmoid":
            p = 1.0 / (1.0 + np.exp(-lg)) + (layer["bias"].astype(np.float64) if layer.get("bias") is not None else 0)
        else:
            p = np.exp(lg - lg.max())
            p /= p.sum()
        only_gpu = sorted(set(ids_gpu[r]) - set(ids[r]))
        only_ora = sorted(set(ids[r]) - set(ids_gpu[r]))
        assert len(only_gpu) == len(only_ora), (r, ids[r], ids_gpu[r])
        if only_gpu:   # a different pick at the boundary of the set
            gap = max(abs(p[a] - p[b]) for a, b in zip(only_gpu, only_ora))
        else:          # the same picks, two of them in the other order
            diff = np.nonzero(ids[r] != ids_gpu[r])[0]
            gap = max(abs(p[ids[r][i]] - p[ids_gpu[r][i]]) for i in diff)
        assert gap <= 1e-6 * p.max(), ("routing differs beyond a near tie", r, only_gpu, only_ora, gap)
    assert len(bad) <= max(1, len(ids) // 1000), len(bad)
    return ids, w, np.setdiff1d(np.arange(len(ids)), bad)


def teacher_forced(cfg, layer, P, rows, logits):
    """The layer output of `rows` recomputed in fp64 from the prompt layer's own routing and its own hidden codes
    (codes x d of the q8_1-quantised hidden vectors the down products read): exact products of the dequantised down
    weights with those hidden values, summed as the combine does.  What is left between this and the GPU's output is
    the fp32 accumulation of the products alone."""
    H, F, K, E = cfg["n_embd"], cfg["n_ff"], cfg["n_used"], cfg["n_expert"]
    L = synth.blob_layout(cfg)
    ids = P.ids.cpu().numpy()[rows]
    w = P.w.cpu().numpy()[rows].astype(np.float64)
    rinv = P.rinv.cpu().numpy()
    codes = P.ha.codes.cpu().numpy()
    d = P.ha.d.cpu().numpy()[:, :F // 32]

    def hval(r):
        return codes[r].astype(np.float64) * np.repeat(d[r].astype(np.float64), 32)

    cache = {}

    def down(e):
        if e not in cache:
            blob = layer["blobs"][e]
            rb = L["d_row"]
            dn = blob[L["down_off"]:L["down_off"] + H * rb].reshape(H, rb)
            cache[e] = np.stack([O.dequant_row(cfg["d_type"], dn[i], F) for i in range(H)]).astype(np.float64)
        return cache[e]

    out = np.zeros((len(rows), H))
    for i, t in enumerate(rows):
        for k in range(K):
            out[i] += w[i, k] * (down(int(ids[i, k])) @ hval(rinv[t * K + k]))
    if P.Ls is not None:
        FS = cfg["sh_n_ff"]
        Ls = synth.blob_layout(cfg, shared=True)
        rb = Ls["d_row"]
        dn = layer["sh_blob"][Ls["down_off"]:Ls["down_off"] + H * rb].reshape(H, rb)
        Wd = np.stack([O.dequant_row(cfg["sh_d_type"], dn[i], FS) for i in range(H)]).astype(np.float64)
        sc, sd = P.hs.codes.cpu().numpy(), P.hs.d.cpu().numpy()[:, :FS // 32]
        g = (1.0 / (1.0 + np.exp(-logits[rows, E].astype(np.float64))) if cfg["router_mode"] == "softmax"
             and cfg.get("shared_gate") else np.ones(len(rows)))
        for i, t in enumerate(rows):
            out[i] += g[i] * (Wd @ (sc[t].astype(np.float64) * np.repeat(sd[t].astype(np.float64), 32)))
    return out


def check_layer(cfg, layer, h, prior=None, n_sample=None, seed=0):
    """Layer bar (the north star's): max-abs <= 1e-2 of the RMS and cosine >= 0.9999 against the fp64 result on the
    same routing and the same hidden codes (teacher_forced), with the hidden codes themselves checked against the
    oracle's fp64 hidden vectors quantised (at most one quantisation step apart, and rarely: a value within rounding of
    a code boundary).  Against the oracle's own hidden codes, and against the decode-kernel layer (the reference's own
    kernels, which quantise the hidden vectors from dp4a sums), the single-step hidden-code differences reach the
    output: there cosine >= 0.9999 and max-abs <= 3e-2 of the RMS."""
    T_tok = h.shape[0]
    P, M = layers_for(cfg, layer, T_tok)
    xp, xm = run_both(P, M, h, prior)
    logits = P.logits[:T_tok].cpu().numpy()
    assert np.array_equal(logits, M.logits[:T_tok].cpu().numpy())       # one router kernel, same input (+ prior)
    ids_gpu = P.ids[:T_tok].cpu().numpy()
    assert np.array_equal(M.ids[:T_tok].cpu().numpy(), ids_gpu)          # one routing kernel per mode, both paths
    ids, w, agree = routing_vs_oracle(cfg, layer, logits, ids_gpu)
    assert np.allclose(P.w[:T_tok].cpu().numpy()[agree], w[agree], rtol=2e-6, atol=0)
    # every token: the tensor-core layer against the decode-kernel layer
    err, cos = tol(xp, xm)
    assert err <= 3e-2 and cos >= COS, ("prefill vs decode kernels", err, cos)
    rows = agree if n_sample is None else np.sort(np.random.default_rng(seed).choice(agree, n_sample, replace=False))
    # the north star's bar given the same routing and hidden codes
    tf = teacher_forced(cfg, layer, P, rows, logits)
    err, cos = tol(xp[rows], tf)
    assert err <= ERR and cos >= COS, ("prefill vs fp64 on its own hidden codes", err, cos)
    # the hidden codes against the oracle's fp64 hidden vectors, quantised
    K, F = cfg["n_used"], cfg["n_ff"]
    xq = O.quantize_q8_1(h[rows])
    rinv = P.rinv.cpu().numpy()
    codes, dd = P.ha.codes.cpu().numpy(), P.ha.d.cpu().numpy()[:, :F // 32]
    href = np.stack([O.expert_ffn(cfg["gu_type"], cfg["d_type"], layer["blobs"][ids[t, k]], cfg["n_embd"], F, xq[i],
                                  cfg["act"], cfg.get("limit", float("inf")), want_h=True)[1]
                     for i, t in enumerate(rows) for k in range(K)])
    ref_q = O.quantize_q8_1(href)
    ref_q.reshape(len(href), -1, 36)[:, :, 2:4] = 0
    sel = np.array([rinv[t * K + k] for t in rows for k in range(K)])
    mine_q = np.zeros_like(ref_q).reshape(len(sel), F // 32, 36)
    mine_q[:, :, 0:2] = dd[sel].astype(np.float16).view(np.uint8).reshape(len(sel), F // 32, 2)
    mine_q[:, :, 4:] = codes[sel].reshape(len(sel), F // 32, 32).view(np.uint8)
    bad_ds, bad_codes, max_step = O.q8_1_compare(mine_q.reshape(len(sel), -1), ref_q)
    assert max_step <= 1 and bad_codes <= max(2, len(sel) * F // 2000), (bad_ds, bad_codes, max_step)
    # the oracle's whole layer (its own hidden codes) on the same rows
    ref = O.moe_layer(layer, h[rows], logits=np.ascontiguousarray(logits[rows]))
    assert np.array_equal(ref["ids"], ids[rows])
    for name, mine in (("prefill", xp[rows]), ("decode kernels", xm[rows])):
        err, cos = tol(mine, ref["out"])
        assert err <= 3e-2 and cos >= COS, (name, err, cos)
    return P, M


def test_qwen_layer_T512(cuda):
    cfg = synth.QWEN
    layer = synth.make_layer(cfg, seed=0)
    h = synth.rms_normed(np.random.default_rng(0), 512, cfg["n_embd"])
    check_layer(cfg, layer, h, n_sample=128, seed=0)


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
