"""The prefill path on the tensor cores: the dispatch permutation bit for bit against the oracle's restatement of
q36_engine.cu:486-510, and the grouped gate/up + down products (routed and dense shared expert) against the oracle's
fp64-accumulated block dots and against the reference's own decode kernels on the same q8_1 activations, within the
layer tolerance (max-abs <= 1e-2 of the RMS, cosine >= 0.9999); the hidden vectors' q8_1 codes against the oracle's."""
import numpy as np
import pytest
import torch

import tinystrata_b200 as T
from oracle import oracle as O
from tinystrata_b200 import synth

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def tol(mine, ref):
    mine = np.asarray(mine, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    rms = np.sqrt(np.mean(ref ** 2))
    return float(np.abs(mine - ref).max() / rms), float(mine @ ref / (np.linalg.norm(mine) * np.linalg.norm(ref)))


@pytest.mark.parametrize("T_tok,K,E", [(300, 8, 128), (1, 8, 256), (4096, 4, 64), (257, 2, 8)])
def test_dispatch_matches_oracle(cuda, T_tok, K, E):
    rng = np.random.default_rng(T_tok + E)
    # Zipf-skewed picks, distinct per token (some experts get nothing)
    p = 1.0 / np.arange(1, E + 1) ** 1.1
    p /= p.sum()
    ids = np.stack([rng.choice(E, K, replace=False, p=p) for _ in range(T_tok)]).astype(np.int32)
    bounds, row_ent, row_tok, rinv = T.moe_dispatch(dev(ids), E)
    b, dst, src, inv, _ = O.dispatch(ids, E)
    assert np.array_equal(bounds.cpu().numpy(), b)
    assert np.array_equal(row_ent.cpu().numpy(), dst)
    assert np.array_equal(row_tok.cpu().numpy(), src)
    assert np.array_equal(rinv.cpu().numpy(), inv)


def _routed_case(cfg, T_tok, K, E_mat, seed):
    layer = synth.make_layer(cfg, seed, n_expert=E_mat)
    rng = np.random.default_rng(seed)
    H, F = cfg["n_embd"], cfg["n_ff"]
    x = synth.rms_normed(rng, T_tok, H)
    ids = np.stack([rng.choice(E_mat, K, replace=False) for _ in range(T_tok)]).astype(np.int32)
    return layer, x, ids


# weight formats: Q4_0 (Gemma, C2), Q4_K gate/up + Q6_K down (LFM2, C3), IQ3_XXS (Qwen, C1 weights),
# IQ3_XXS gate/up + IQ3_S down (Qwen expert-parallel, C4)
CASES = [("gemma", 200, 2), ("gemma", 37, 8), ("lfm", 150, 4), ("qwen", 120, 8), ("qwen_ep", 96, 8)]
CFGS = {"gemma": synth.GEMMA, "lfm": synth.LFM, "qwen": synth.QWEN, "qwen_ep": synth.QWEN_EP}


@pytest.mark.parametrize("name,T_tok,K", CASES)
def test_prefill_routed_vs_oracle(cuda, name, T_tok, K):
    cfg = CFGS[name]
    H, F, E_mat = cfg["n_embd"], cfg["n_ff"], 8
    layer, x, ids = _routed_case(cfg, T_tok, K, E_mat, seed=21)
    L = T.native_expert_layout(cfg["gu_type"], cfg["d_type"], H, F)
    blobs = dev(layer["blobs"])
    xqd = T.quantize_q8_1_rows(dev(x))   # the reference quantiser's blocks (bitwise, test_gpu_parity)
    bounds, row_ent, row_tok, rinv = T.moe_dispatch(dev(ids), E_mat)
    n = T_tok * K
    h = T.moe_prefill_gu(L, blobs, int(L.bytes), bounds, E_mat, n, xqd, row_tok, act=cfg["act"])
    out = T.moe_prefill_down(L, blobs, int(L.bytes), bounds, E_mat, n, h)
    torch.cuda.synchronize()
    assert T.device_error() == 0
    mine = out.cpu().numpy()[rinv.cpu().numpy()]          # back to entry order
    assert np.all(np.isfinite(mine))
    xq = xqd.cpu().numpy()
    ref = O.experts_for_tokens(cfg["gu_type"], cfg["d_type"], layer["blobs"], H, F, xq, ids, cfg["act"]).reshape(n, H)
    err, cos = tol(mine, ref)
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)
    # the reference's own decode kernels on the same activations (test_gpu_parity pins them bitwise)
    g = T.moe_group(dev(ids), E_mat, blobs, int(L.bytes))
    scratch = torch.empty(T.native_expert_scratch_bytes(n, F) // 4, dtype=torch.float32, device="cuda")
    outd = torch.full((n, H), float("nan"), device="cuda")
    T.native_expert_grouped(L, g, n, n, xqd, scratch, outd, cfg["act"])
    err, cos = tol(mine, outd.cpu().numpy())
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)
    # the hidden vectors' q8_1 blocks against the oracle's quantisation of its fp64-summed hidden vectors: codes may
    # differ only where the value sits within rounding of a code boundary (a handful)
    hq = h.cpu().numpy()[rinv.cpu().numpy()]
    href = np.stack([O.expert_ffn(cfg["gu_type"], cfg["d_type"], layer["blobs"][ids[e // K, e % K]], H, F, xq[e // K],
                                  cfg["act"], want_h=True)[1] for e in range(n)])
    bad_ds, bad_codes, max_step = O.q8_1_compare(hq, O.quantize_q8_1(href))
    assert max_step <= 1 and bad_codes <= n * F // 2000, (bad_ds, bad_codes, max_step)


@pytest.mark.parametrize("name", ["gemma", "qwen"])   # Q4_0 (Gemma) and Q8_0 (Qwen) dense shared experts
def test_prefill_dense_shared_vs_oracle(cuda, name):
    cfg = CFGS[name]
    H, FS = cfg["n_embd"], cfg["sh_n_ff"]
    layer = synth.make_layer(cfg, 31, n_expert=1)
    rng = np.random.default_rng(31)
    T_tok = 150
    x = synth.rms_normed(rng, T_tok, H)
    Ls = T.native_expert_layout(cfg["sh_gu_type"], cfg["sh_d_type"], H, FS)
    sh = dev(layer["sh_blob"])
    xqd = T.quantize_q8_1_rows(dev(x))
    h = T.moe_prefill_gu(Ls, sh, 0, None, 1, T_tok, xqd, None, act=cfg.get("sh_act", cfg["act"]))
    out = T.moe_prefill_down(Ls, sh, 0, None, 1, T_tok, h)
    torch.cuda.synchronize()
    xq = xqd.cpu().numpy()
    ref = np.stack([O.expert_ffn(cfg["sh_gu_type"], cfg["sh_d_type"], layer["sh_blob"], H, FS, xq[t],
                                 cfg.get("sh_act", cfg["act"]))
                    for t in range(T_tok)])
    err, cos = tol(out.cpu().numpy(), ref)
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)


def test_prefill_rejects_unsupported(cuda):
    # expert widths that do not fill the kernel's 64-value stages are refused (UNSUPPORTED), nothing is launched
    H, F = 2048, 96
    L = T.native_expert_layout(synth.T_Q4_0, synth.T_Q4_0, H, F)
    blobs = torch.zeros(int(L.bytes), dtype=torch.uint8, device="cuda")
    xq = torch.zeros((4, H // 32 * 36), dtype=torch.uint8, device="cuda")
    with pytest.raises(T.TsbError, match="status -2"):
        T.moe_prefill_gu(L, blobs, int(L.bytes), None, 1, 4, xq)


def test_prefill_layer_gemma_vs_oracle(cuda):
    """The whole prompt-path layer (router GEMM, routing, q8_1, dispatch, grouped products, shared FFN, combine)."""
    from tinystrata_b200.layer import PrefillLayer
    cfg = dict(synth.GEMMA, n_expert=16)
    H = cfg["n_embd"]
    layer = synth.make_layer(cfg, 41)
    rng = np.random.default_rng(41)
    T_tok = 100
    x = synth.rms_normed(rng, T_tok, H)
    P = PrefillLayer(cfg, dev(layer["blobs"]), dev(layer["router"]), dev(layer["sh_blob"]), max_tokens=T_tok,
                     escale=dev(layer["escale"]))
    xd = torch.zeros((T_tok, H), device="cuda")
    P.forward(xd, dev(x))
    torch.cuda.synchronize()
    assert T.device_error() == 0
    ref = O.moe_layer(layer, x)
    assert np.array_equal(P.ids.cpu().numpy(), ref["ids"])
    err, cos = tol(xd.cpu().numpy(), ref["out"])
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)
