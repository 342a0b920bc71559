"""The prefill path on the tensor cores: the dispatch permutation bit for bit against the oracle's restatement of
q36_engine.cu:486-510; the tensor-core activation layout (codes and scales) bit for bit against the q8_1 quantiser;
the int32 block sums in tensor memory bit for bit against the integer dot of the activation codes with the oracle's
weight codes, for every weight format, gate/up and down; the grouped gate/up + down products (routed and dense shared
expert) against the oracle's fp64-accumulated block dots and against the reference's own decode kernels on the same
q8_1 activations, within the layer tolerance (max-abs <= 1e-2 of the RMS, cosine >= 0.9999); the hidden vectors'
q8_1 codes against the oracle's."""
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


def act_to_q8_1(a: "T.MmqAct", rows=None) -> np.ndarray:
    """The codes and d of an mmq-layout buffer as q8_1 bytes (sum field zero) for O.q8_1_compare on codes and d."""
    codes = a.codes.cpu().numpy()
    d = a.d.cpu().numpy()[:, :a.K // 32]
    if rows is not None:
        codes, d = codes[rows], d[rows]
    n, K = codes.shape
    out = np.zeros((n, K // 32, 36), np.uint8)
    out[:, :, 0:2] = d.astype(np.float16).view(np.uint8).reshape(n, K // 32, 2)
    out[:, :, 4:] = codes.reshape(n, K // 32, 32).view(np.uint8)
    return out.reshape(n, -1)


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


def test_mmq_layout_is_the_q8_1_quantiser(cuda):
    """mmq_quantize (fp32, gathered rows) and mmq_from_q8_1 give the q8_1 quantiser's codes and fp16 scales bit for
    bit, and the code-sum term exactly d * sum(codes)."""
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, size=(300, 704)).astype(np.float32)
    x[::7, :64] *= 300.0
    x[5] = 0.0
    src = rng.integers(0, 300, size=500).astype(np.int32)
    xd = dev(x)
    a = T.mmq_quantize(xd, row_src=dev(src), n_rows=500)
    q = T.quantize_q8_1_rows(xd).cpu().numpy()[src]
    d_ref, _, c_ref = O.q8_1_unpack(q)
    assert np.array_equal(a.codes.cpu().numpy(), c_ref.reshape(500, 704))
    assert np.array_equal(a.d.cpu().numpy()[:, :22], d_ref)
    csum = c_ref.astype(np.int64).sum(-1)
    assert np.array_equal(a.s.cpu().numpy()[:, :22], (d_ref.astype(np.float32) * csum.astype(np.float32)))
    b = T.mmq_from_q8_1(T.quantize_q8_1_rows(xd), 704, row_src=dev(src), n_rows=500)
    torch.cuda.synchronize()
    for u, v in ((a.codes, b.codes), (a.d, b.d), (a.s, b.s)):
        assert torch.equal(u[:, :22] if u.dtype == torch.float32 else u, v[:, :22] if v.dtype == torch.float32 else v)


# ------------------------------------------------------------------------------------------------ block sums
FORMAT_CFGS = [   # (gate/up type, down type, n_embd, n_ff): every weight format on each side of the products
    (synth.T_Q4_0, synth.T_Q4_0, 2816, 704),
    (synth.T_Q8_0, synth.T_Q8_0, 2048, 512),
    (synth.T_Q4_K, synth.T_Q6_K, 2048, 512),
    (synth.T_IQ3_XXS, synth.T_IQ3_S, 2048, 512),
]


@pytest.mark.parametrize("gu,dn,H,F", FORMAT_CFGS)
@pytest.mark.parametrize("mode", [0, 1])
def test_block_sums_bit_exact(cuda, gu, dn, H, F, mode):
    """The tensor core's int32 sum of every 32-value block (Q6_K: 16-value half) of the first output tile equals the
    integer dot of the q8_1 activation codes with the weight codes the reference's block dots multiply
    (or_weight_codes, restating iq_kernels.cu:188-236, 314-386, 457-474, 523-566)."""
    rng = np.random.default_rng(7 + gu + dn + mode)
    cfg = dict(gu_type=gu, d_type=dn, n_embd=H, n_ff=F)
    L = T.native_expert_layout(gu, dn, H, F)
    blob = np.concatenate([synth.gen_matrix(rng, gu, F, H, 0.02), synth.gen_matrix(rng, gu, F, H, 0.02),
                           synth.gen_matrix(rng, dn, H, F, 0.02)])
    assert blob.size == L.bytes
    Kc = H if mode == 0 else F
    x = rng.normal(0, 1, size=(128, Kc)).astype(np.float32)
    x[::5, :96] *= 40.0
    xa = T.mmq_quantize(dev(x))
    sums, _ = T.debug_mmq_block_sums(L, mode, dev(blob), 128, xa)
    torch.cuda.synchronize()
    assert T.device_error() == 0
    xc = xa.codes.cpu().numpy().astype(np.int64)                 # [128, Kc]
    if mode == 0:
        t, rb = gu, int(L.gu_row)
        gate = blob[:F * rb].reshape(F, rb)
        up = blob[int(L.up_off):int(L.up_off) + F * rb].reshape(F, rb)
        cols = [(up if (c & 32) else gate)[(c >> 6) * 32 + (c & 31)] for c in range(128)]
    else:
        t, rb = dn, int(L.d_row)
        down = blob[int(L.down_off):].reshape(H, rb)
        cols = [down[c] for c in range(128)]
    wc = O.weight_codes(t, np.stack(cols), Kc).astype(np.int64)  # [128 columns, Kc]
    got = sums.cpu().numpy().astype(np.int64)                    # [Kc / 32, split, 128, 128]
    nb = Kc // 32
    seg = 16 if t == synth.T_Q6_K else 32                        # Q6_K: one sum per 16-value half
    want = np.stack([xc[:, o:o + seg] @ wc[:, o:o + seg].T for o in range(0, Kc, seg)])
    want = want.reshape(nb, 32 // seg, 128, 128)
    assert np.array_equal(got, want), np.argwhere(got != want)[:5]


# ------------------------------------------------------------------------------------------------ products
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
    xd = dev(x)
    xqd = T.quantize_q8_1_rows(xd)   # the reference quantiser's blocks (bitwise, test_gpu_parity)
    bounds, row_ent, row_tok, rinv = T.moe_dispatch(dev(ids), E_mat)
    n = T_tok * K
    xa = T.mmq_quantize(xd, row_src=row_tok, n_rows=n)
    h = T.moe_prefill_gu(L, blobs, int(L.bytes), bounds, E_mat, n, xa, act=cfg["act"])
    out = T.moe_prefill_down(L, blobs, int(L.bytes), bounds, E_mat, n, h)
    torch.cuda.synchronize()
    assert T.device_error() == 0
    inv = rinv.cpu().numpy()
    mine = out.cpu().numpy()[inv]          # back to entry order
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
    # the hidden vectors' q8_1 codes and scales against the oracle's quantisation of its fp64-summed hidden vectors:
    # codes may differ only where the value sits within rounding of a code boundary (a handful)
    hq = act_to_q8_1(h, inv)
    href = np.stack([O.expert_ffn(cfg["gu_type"], cfg["d_type"], layer["blobs"][ids[e // K, e % K]], H, F, xq[e // K],
                                  cfg["act"], want_h=True)[1] for e in range(n)])
    ref_q = O.quantize_q8_1(href)
    ref_q.reshape(n, -1, 36)[:, :, 2:4] = 0   # the sum field is not part of the tensor-core layout
    bad_ds, bad_codes, max_step = O.q8_1_compare(hq, ref_q)
    assert max_step <= 1 and bad_codes <= n * F // 2000 and bad_ds <= n * F // 32 // 500, (bad_ds, bad_codes, max_step)


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
    xd = dev(x)
    xqd = T.quantize_q8_1_rows(xd)
    xa = T.mmq_quantize(xd)
    h = T.moe_prefill_gu(Ls, sh, 0, None, 1, T_tok, xa, act=cfg.get("sh_act", cfg["act"]))
    out = T.moe_prefill_down(Ls, sh, 0, None, 1, T_tok, h)
    torch.cuda.synchronize()
    assert T.device_error() == 0
    xq = xqd.cpu().numpy()
    ref = np.stack([O.expert_ffn(cfg["sh_gu_type"], cfg["sh_d_type"], layer["sh_blob"], H, FS, xq[t],
                                 cfg.get("sh_act", cfg["act"]))
                    for t in range(T_tok)])
    err, cos = tol(out.cpu().numpy(), ref)
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)


def test_prefill_rejects_unsupported(cuda):
    # expert widths that do not fill the kernel's 64-value tiles are refused (UNSUPPORTED), nothing is launched
    H, F = 2048, 96
    L = T.native_expert_layout(synth.T_Q4_0, synth.T_Q4_0, H, F)
    blobs = torch.zeros(int(L.bytes), dtype=torch.uint8, device="cuda")
    xa = T.mmq_quantize(torch.zeros((4, H), device="cuda"))
    with pytest.raises(T.TsbError, match="status -2"):
        T.moe_prefill_gu(L, blobs, int(L.bytes), None, 1, 4, xa)


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


@pytest.mark.parametrize("t,w_rows,w_cols", [(synth.T_Q4_0, 192, 2816), (synth.T_IQ3_S, 256, 512),
                                             (synth.T_Q6_K, 128, 1792)])
def test_mmq_product_groups_row_map_and_stride(cuda, t, w_rows, w_cols):
    """tsb_mmq_product (mmq::Context::run / gemma4::Mmq::mul): three matrices over their row ranges, each row's
    product scattered to dst row ids[i] of a wider dst (ld_dst > w_rows), against fp64 of the dequantised weights and
    the activation values (codes x d) the kernel read."""
    rng = np.random.default_rng(90 + t)
    n, rows = 3, 300
    rb = synth.row_bytes(t, w_cols)
    mats = [synth.gen_matrix(rng, t, w_rows, w_cols, 0.02).reshape(w_rows, rb) for _ in range(n)]
    stride = (w_rows * rb + 255) // 256 * 256
    wbuf = np.zeros(n * stride, np.uint8)
    for e in range(n):
        wbuf[e * stride:e * stride + w_rows * rb] = mats[e].ravel()
    bounds = np.array([0, 70, 70 + 161, rows], np.int32)
    ids = rng.permutation(rows).astype(np.int32)
    x = rng.normal(0, 1, size=(rows, w_cols)).astype(np.float32)
    xa = T.mmq_quantize(dev(x))
    ld = w_rows + 36
    dst = torch.full((rows, ld), float("nan"), device="cuda")
    T.mmq_product(dev(wbuf), t, w_rows, w_cols, stride, n, xa, bounds=dev(bounds), ids=dev(ids), dst=dst, ld_dst=ld)
    torch.cuda.synchronize()
    assert T.device_error() == 0
    got = dst.cpu().numpy()
    xv = xa.codes.cpu().numpy().astype(np.float64) * np.repeat(xa.d.cpu().numpy()[:, :w_cols // 32], 32, axis=1)
    for e in range(n):
        W = np.stack([O.dequant_row(t, mats[e][i], w_cols) for i in range(w_rows)]).astype(np.float64)
        for r in range(bounds[e], bounds[e + 1]):
            want = W @ xv[r]
            err = np.abs(got[ids[r], :w_rows] - want).max() / np.sqrt(np.mean(want ** 2))
            assert err <= 1e-4, (e, r, err)
    assert np.all(np.isnan(got[:, w_rows:]))   # nothing written past the rows' w_rows values
