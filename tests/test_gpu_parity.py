"""GPU parity of the CUDA path (called through the C ABI) against the oracle and against the reference's own decode
kernels compiled for sm_100a (oracle/_ref/libtsb_ref_gpu.so), on the same seeded inputs.

Bar: integer work bit-exact (per-call integer sums, routing ids, groups); the q8_1 quantiser, the (256, 8) router and
the grouped experts bit-exact against the reference's GPU kernels; layer outputs within max-abs 1e-2 x RMS and cosine
>= 0.9999 against the oracle."""
import numpy as np
import pytest
import torch

import tinystrata_b200 as T
from oracle import oracle as O
from tinystrata_b200 import synth
from tests import refgpu

pytestmark = pytest.mark.gpu

FORMATS = [synth.T_IQ3_XXS, synth.T_IQ3_S, synth.T_Q4_0, synth.T_Q8_0, synth.T_Q4_K, synth.T_Q6_K]
EXACT_FLOAT = {synth.T_IQ3_XXS, synth.T_IQ3_S, synth.T_Q4_0, synth.T_Q8_0}   # no fused multiply-add in the call value


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def ref_or_skip():
    R = refgpu.lib()
    if R is None:
        pytest.skip("oracle/_ref/libtsb_ref_gpu.so not built")
    return R


def layer_tolerance(mine, ref):
    mine = np.asarray(mine, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    rms = np.sqrt(np.mean(ref ** 2))
    cos = float(mine @ ref / (np.linalg.norm(mine) * np.linalg.norm(ref)))
    return float(np.abs(mine - ref).max() / rms), cos


# ------------------------------------------------------------------------------------------------ block dots
@pytest.mark.parametrize("t", FORMATS)
@pytest.mark.parametrize("n", [512, 2048])
def test_row_calls_bit_exact(cuda, t, n):
    rng = np.random.default_rng(1000 * t + n)
    W = synth.gen_matrix(rng, t, 1, n, 0.02)
    x = rng.normal(0, 1, size=(1, n)).astype(np.float32)
    x[0, :64] *= 50.0   # some large blocks
    xq = O.quantize_q8_1(x)[0]
    s, v = T.debug_row_calls(t, dev(W), dev(xq), n)
    so, vo = O.row_dot_calls(t, W, xq, n)
    assert np.array_equal(s.cpu().numpy(), so)
    if t in EXACT_FLOAT:
        assert np.array_equal(v.cpu().numpy(), vo)
    else:
        assert np.allclose(v.cpu().numpy(), vo, rtol=1e-6, atol=1e-6 * np.abs(vo).max())


# ------------------------------------------------------------------------------------------------ q8_1
def test_quantize_q8_1_matches_reference_gpu_bitwise(cuda):
    R = ref_or_skip()
    rng = np.random.default_rng(5)
    x = rng.normal(0, 2, size=(64, 2048)).astype(np.float32)
    x[3, :32] = 0.0
    x[4, 32:64] = 1e5    # sums past fp16: clamped to 65504 (q8_1_finite)
    x[5, 7] = -3e6
    xd = dev(x)
    mine = T.quantize_q8_1_rows(xd)
    ref = torch.zeros_like(mine)
    R.ref_quantize_q8_1_rows(refgpu.ptr(xd), 64, 2048, refgpu.ptr(ref), refgpu.stream())
    torch.cuda.synchronize()
    assert torch.equal(mine, ref)
    bad_ds, bad_codes, maxd = O.q8_1_compare(mine.cpu().numpy(), O.quantize_q8_1(x))
    assert maxd <= 1 and bad_codes <= x.size // 2000   # only values within a few ulp of a rounding boundary


def test_quantize_empty_and_errors(cuda):
    x = torch.zeros((0, 64), device="cuda")
    assert T.lib().tsb_quantize_q8_1_rows(T._ptr(x), 0, 64, T._ptr(x), None) == 0
    assert T.lib().tsb_quantize_q8_1_rows(T._ptr(x), 1, 33, T._ptr(x), None) == -1


# ------------------------------------------------------------------------------------------------ routers
@pytest.mark.parametrize("ld", [256, 257])
def test_router_topk_vs_reference_and_oracle(cuda, ld):
    rng = np.random.default_rng(ld)
    logits = rng.normal(0, 2, size=(100, ld)).astype(np.float32)
    lg = dev(logits)
    ids, w = T.native_router_topk(lg, 8, 256)
    oi, ow, near = O.router_softmax_topk(logits, 8, 256)
    assert near == 0
    assert np.array_equal(ids.cpu().numpy(), oi)
    assert np.allclose(w.cpu().numpy(), ow, rtol=2e-6)
    if ld == 256:
        R = ref_or_skip()
        ri = torch.zeros_like(ids)
        rw = torch.zeros_like(w)
        s = torch.cuda.Stream()   # the reference rejects the legacy default stream (native_router.cu:104)
        with torch.cuda.stream(s):
            assert R.ref_native_router_topk(refgpu.ptr(lg), refgpu.ptr(ri), refgpu.ptr(rw), 256, 8, 100,
                                            refgpu.stream()) == 0
        torch.cuda.synchronize()
        assert torch.equal(ids, ri) and torch.equal(w, rw)


@pytest.mark.parametrize("E,K", [(64, 4), (128, 8), (512, 16)])
def test_router_topk_other_shapes(cuda, E, K):
    rng = np.random.default_rng(E)
    logits = rng.normal(0, 2, size=(33, E)).astype(np.float32)
    ids, w = T.native_router_topk(dev(logits), K, E)
    oi, ow, near = O.router_softmax_topk(logits, K, E)
    assert near == 0 and np.array_equal(ids.cpu().numpy(), oi)
    assert np.allclose(w.cpu().numpy(), ow, rtol=2e-6)


@pytest.mark.parametrize("gate", [0, 1])
def test_route_rows_vs_oracle(cuda, gate):
    rng = np.random.default_rng(40 + gate)
    E, K = (128, 8) if gate == 0 else (64, 4)
    logits = rng.normal(0, 2, size=(50, E)).astype(np.float32)
    bias = rng.normal(0, 0.05, size=E).astype(np.float32) if gate == 1 else None
    esc = rng.uniform(0.5, 1.5, size=E).astype(np.float32) if gate == 0 else None
    scale = 1.0 / np.sqrt(2816.0) if gate == 0 else 1.0
    ids, w = T.route_rows(dev(logits), K, gate, scale, None if bias is None else dev(bias),
                          None if esc is None else dev(esc), True, 0.0)
    oi, ow = O.route_rows(logits, K, gate, scale, bias, esc, True, 0.0)
    assert np.array_equal(ids.cpu().numpy(), oi)
    assert np.allclose(w.cpu().numpy(), ow, rtol=1e-5)


@pytest.mark.parametrize("gate", [0, 1])
def test_route_rows_vs_reference_gpu(cuda, gate):
    """route_rows bit for bit against the reference's own route_kernel (src/gemma4/kernels.cu:289-356): Gemma's
    softmax of scaled logits with per-expert scales, LFM2's sigmoid picked by gate + bias, with and without the weight
    scale."""
    R = ref_or_skip()
    rng = np.random.default_rng(140 + gate)
    E, K, rows = (128, 8, 300) if gate == 0 else (64, 4, 300)
    logits = dev(rng.normal(0, 2, size=(rows, E)).astype(np.float32))
    bias = dev(rng.normal(0, 0.05, size=E).astype(np.float32)) if gate == 1 else None
    esc = dev(rng.uniform(0.5, 1.5, size=E).astype(np.float32)) if gate == 0 else None
    scale = 1.0 / np.sqrt(2816.0) if gate == 0 else 1.0
    for w_scale in (0.0, 2.5):
        ids, w = T.route_rows(logits, K, gate, scale, bias, esc, True, w_scale)
        rids = torch.zeros_like(ids)
        rw = torch.zeros_like(w)
        assert R.ref_route_rows(refgpu.ptr(logits), E, K, rows, gate, scale, refgpu.ptr(bias), refgpu.ptr(esc), 1,
                                w_scale, refgpu.ptr(rids), refgpu.ptr(rw), refgpu.stream()) == 0
        torch.cuda.synchronize()
        assert torch.equal(ids, rids)
        assert torch.equal(w, rw)


def test_moe_sum_and_add_scaled_vs_reference_gpu(cuda):
    """moe_sum and add_scaled bit for bit against the reference's (src/gemma4/kernels.cu:245-249, 358-366)."""
    R = ref_or_skip()
    rng = np.random.default_rng(150)
    rows, K, n = 37, 8, 2816
    x = dev(rng.normal(0, 1, size=(rows * K, n)).astype(np.float32))
    w = dev(rng.random((rows, K)).astype(np.float32))
    acc0 = rng.normal(0, 1, size=(rows, n)).astype(np.float32)
    mine, ref = dev(acc0), dev(acc0)
    T.moe_sum(x, w, mine, K)
    R.ref_moe_sum(refgpu.ptr(x), refgpu.ptr(w), refgpu.ptr(ref), n, K, rows, refgpu.stream())
    torch.cuda.synchronize()
    assert torch.equal(mine, ref)
    # add_scaled with repeated sums (the same vector added into twice) and 5 vectors
    xs = [dev(rng.normal(0, 1, size=n).astype(np.float32)) for _ in range(5)]
    a0 = [rng.normal(0, 1, size=n).astype(np.float32) for _ in range(3)]
    accs_m = [dev(a) for a in a0]
    accs_r = [dev(a) for a in a0]
    ws = [0.5, -1.25, 3.0, 0.125, 7.0]
    pick = [0, 1, 0, 2, 1]
    T.add_scaled(xs, [accs_m[i] for i in pick], ws)
    import ctypes as C
    xp = (C.c_void_p * 5)(*[x.data_ptr() for x in xs])
    ap = (C.c_void_p * 5)(*[accs_r[i].data_ptr() for i in pick])
    wp = (C.c_float * 5)(*ws)
    assert R.ref_add_scaled(xp, ap, wp, 5, n, refgpu.stream()) == 0
    torch.cuda.synchronize()
    for a, b in zip(accs_m, accs_r):
        assert torch.equal(a, b)


def test_moe_layer_tail_vs_fp64(cuda):
    """The Gemma 4 layer tail (gemma4.cpp:560-568) against an fp64 restatement of its norms and adds."""
    rng = np.random.default_rng(151)
    rows, n, eps, scale = 9, 2816, 1e-6, 0.75
    moe = rng.normal(0, 3, size=(rows, n))
    mlp = rng.normal(0, 1, size=(rows, n))
    pm = rng.uniform(0.5, 1.5, size=n)
    pf = rng.uniform(0.5, 1.5, size=n)
    r0 = rng.normal(0, 1, size=(rows, n))

    def rms(v):
        return v / np.sqrt(np.mean(v * v, axis=1, keepdims=True) + eps)

    want = (r0 + rms(rms(moe) * pm + mlp) * pf) * scale
    r = dev(r0.astype(np.float32))
    f = lambda a: dev(np.asarray(a, np.float32))
    T.moe_layer_tail(f(moe), r, f(pm), f(mlp), f(pf), scale, eps)
    torch.cuda.synchronize()
    err, cos = layer_tolerance(r.cpu().numpy(), want)
    assert err <= 1e-5 and cos >= 0.999999, (err, cos)


def test_router_logits(cuda):
    rng = np.random.default_rng(9)
    W = rng.normal(0, 0.02, size=(257, 2048)).astype(np.float32)
    h = rng.normal(0, 1, size=(5, 2048)).astype(np.float32)
    lg = T.router_logits_f32(dev(W), dev(h))
    ref = h.astype(np.float64) @ W.T.astype(np.float64)
    assert np.allclose(lg.cpu().numpy(), ref, rtol=1e-4, atol=1e-4)


# ------------------------------------------------------------------------------------------------ grouping
def test_group_matches_oracle(cuda):
    rng = np.random.default_rng(21)
    T_, K, E = 16, 8, 256
    ids = np.stack([rng.choice(40, K, replace=False) for _ in range(T_)]).astype(np.int32)   # many shared experts
    base = torch.zeros(1, dtype=torch.uint8, device="cuda")
    stride = 1204224
    g = T.moe_group(dev(ids), E, base, stride)
    ge, gs, dst, tok = O.group(ids, E)
    ng = int(g.n_groups.item())
    assert ng == len(ge)
    assert np.array_equal(g.grp_start[:ng + 1].cpu().numpy(), gs)
    assert np.array_equal(g.ent_dst.cpu().numpy(), dst)
    assert np.array_equal(g.ent_tok.cpu().numpy(), tok)
    assert np.array_equal(g.grp_ptr[:ng].cpu().numpy() - base.data_ptr(), ge.astype(np.int64) * stride)


# ------------------------------------------------------------------------------------------------ grouped experts
def _grouped_case(cfg, E_mat, ids, seed, act=T.ACT_SWIGLU, limit=float("inf")):
    layer = synth.make_layer(cfg, seed, n_expert=E_mat)
    rng = np.random.default_rng(seed)
    Tn, K = ids.shape
    H, F = cfg["n_embd"], cfg["n_ff"]
    h = synth.rms_normed(rng, Tn, H)
    xq = O.quantize_q8_1(h)
    blobs = dev(layer["blobs"])
    L = T.native_expert_layout(cfg["gu_type"], cfg["d_type"], H, F)
    g = T.moe_group(dev(ids), E_mat, blobs, int(L.bytes))
    n_ent = Tn * K
    scratch = torch.empty(T.native_expert_scratch_bytes(n_ent, F) // 4, dtype=torch.float32, device="cuda")
    out = torch.full((n_ent, H), float("nan"), device="cuda")
    xqd = dev(xq)
    T.native_expert_grouped(L, g, n_ent, n_ent, xqd, scratch, out, act, limit)
    torch.cuda.synchronize()
    assert T.device_error() == 0
    return layer, xq, xqd, g, out, blobs


def _oracle_parts(cfg, layer, xq, ids, act=O.ACT_SWIGLU, limit=float("inf")):
    Tn, K = ids.shape
    return O.experts_for_tokens(cfg["gu_type"], cfg["d_type"], layer["blobs"], cfg["n_embd"], cfg["n_ff"], xq, ids,
                                act, limit).reshape(Tn * K, -1)


@pytest.mark.parametrize("Tn", [1, 4])
def test_expert_grouped_qwen_vs_reference_gpu_and_oracle(cuda, Tn):
    cfg = synth.QWEN
    rng = np.random.default_rng(77 + Tn)
    ids = np.stack([rng.choice(12, 8, replace=False) for _ in range(Tn)]).astype(np.int32)
    layer, xq, xqd, g, out, blobs = _grouped_case(cfg, 12, ids, seed=3)
    mine = out.cpu().numpy()
    assert np.all(np.isfinite(mine))
    ref_parts = _oracle_parts(cfg, layer, xq, ids)
    err, cos = layer_tolerance(mine, ref_parts)
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)
    R = refgpu.lib()
    if R is not None:
        n_ent = Tn * 8
        rs = torch.zeros(R.ref_native_expert_scratch_bytes(n_ent, 512) // 4 + 64, device="cuda")
        rout = torch.full_like(out, float("nan"))
        R.ref_native_expert_grouped(18, 18, 2048, 512, refgpu.ptr(g.grp_ptr), refgpu.ptr(g.grp_start),
                                    refgpu.ptr(g.n_groups), refgpu.ptr(g.ent_dst), refgpu.ptr(g.ent_tok), n_ent, n_ent,
                                    refgpu.ptr(xqd), refgpu.ptr(rs), refgpu.ptr(rout), refgpu.stream())
        torch.cuda.synchronize()
        r = rout.cpu().numpy()
        assert np.array_equal(mine, r), layer_tolerance(mine, r)   # the reference's native_expert_grouped, bit for bit


def test_expert_grouped_many_entries_per_group(cuda):
    """16 tokens all routed to the same 8 experts: groups of 16 entries, taken 4 at a time."""
    cfg = synth.QWEN
    ids = np.tile(np.arange(8, dtype=np.int32), (16, 1))
    layer, xq, xqd, g, out, blobs = _grouped_case(cfg, 8, ids, seed=4)
    err, cos = layer_tolerance(out.cpu().numpy(), _oracle_parts(cfg, layer, xq, ids))
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)


def test_expert_grouped_iq3s_down(cuda):
    cfg = synth.QWEN_EP
    rng = np.random.default_rng(8)
    ids = np.stack([rng.choice(10, 8, replace=False) for _ in range(2)]).astype(np.int32)
    layer, xq, xqd, g, out, blobs = _grouped_case(cfg, 10, ids, seed=5)
    err, cos = layer_tolerance(out.cpu().numpy(), _oracle_parts(cfg, layer, xq, ids))
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)


def test_expert_grouped_gemma_q4_0_gelu(cuda):
    cfg = dict(synth.GEMMA, n_expert=16)
    rng = np.random.default_rng(9)
    ids = np.stack([rng.choice(16, 8, replace=False) for _ in range(3)]).astype(np.int32)
    layer, xq, xqd, g, out, blobs = _grouped_case(cfg, 16, ids, seed=6, act=T.ACT_GELU_TANH)
    err, cos = layer_tolerance(out.cpu().numpy(), _oracle_parts(cfg, layer, xq, ids, O.ACT_GELU_TANH))
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)


def test_expert_grouped_lfm_q4k_q6k(cuda):
    cfg = dict(synth.LFM, n_expert=8)
    rng = np.random.default_rng(10)
    ids = np.stack([rng.choice(8, 4, replace=False) for _ in range(3)]).astype(np.int32)
    layer, xq, xqd, g, out, blobs = _grouped_case(cfg, 8, ids, seed=7, act=T.ACT_SWIGLU_CLAMP, limit=float("inf"))
    err, cos = layer_tolerance(out.cpu().numpy(), _oracle_parts(cfg, layer, xq, ids, O.ACT_SWIGLU_CLAMP))
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)


# ------------------------------------------------------------------------------------------------ combine, layer
def test_combine_vs_reference_gpu_and_oracle(cuda):
    rng = np.random.default_rng(31)
    Tn, K, H = 3, 8, 2048
    x = rng.normal(0, 1, size=(Tn, H)).astype(np.float32)
    parts = rng.normal(0, 1, size=(Tn * K, H)).astype(np.float32)
    w = rng.uniform(0, 0.3, size=(Tn, K)).astype(np.float32)
    shared = rng.normal(0, 1, size=(Tn, H)).astype(np.float32)
    sg = rng.normal(0, 1, size=(Tn, 257)).astype(np.float32)
    xd, pd, wd, sd, sgd = dev(x), dev(parts), dev(w), dev(shared), dev(sg)
    h = torch.empty((Tn, H), device="cuda")
    hq = torch.empty((Tn, H // 32 * 36), dtype=torch.uint8, device="cuda")
    wn = torch.ones(H, device="cuda")   # the reference's combine computes h only with a norm weight
    T.moe_combine(xd, pd, wd, K, sd, sgd[:, 256:], 257, wn=wn, h=h, hq=hq)
    gs = O.sigmoid(sg[:, 256])
    ref = O.combine(x, parts.reshape(Tn, K, H), w, shared, gs)
    assert np.allclose(xd.cpu().numpy(), ref, rtol=1e-5, atol=1e-5)
    hr, hqr = O.rms_q8_1(ref)
    assert np.allclose(h.cpu().numpy(), hr, rtol=1e-5, atol=1e-5)
    R = refgpu.lib()
    if R is not None:
        x2 = dev(x)
        h2 = torch.empty_like(h)
        hq2 = torch.empty_like(hq)
        R.ref_moe_out_small(refgpu.ptr(x2), refgpu.ptr(pd), None, refgpu.ptr(wd), K, refgpu.ptr(sd),
                            C_ptr(sgd, 256), 257, refgpu.ptr(wn), refgpu.ptr(h2), H, 1e-6, refgpu.ptr(hq2), Tn,
                            refgpu.stream())
        torch.cuda.synchronize()
        assert np.allclose(x2.cpu().numpy(), xd.cpu().numpy(), rtol=1e-6, atol=1e-6)
        assert np.allclose(h2.cpu().numpy(), h.cpu().numpy(), rtol=1e-6, atol=1e-6)
        # the reference's h through the quantiser pinned bitwise to the reference's own gives this combine's hq
        assert torch.equal(T.quantize_q8_1_rows(h2), hq) or not torch.equal(h2, h)
        bad_ds, bad_codes, maxd = O.q8_1_compare(hq.cpu().numpy(), hq2.cpu().numpy())
        assert maxd <= 1 and bad_codes <= 8
    bad_ds, bad_codes, maxd = O.q8_1_compare(hq.cpu().numpy(), hqr)
    assert maxd <= 1 and bad_codes <= 8


def C_ptr(t, offset_elems):
    import ctypes
    return ctypes.c_void_p(t.data_ptr() + offset_elems * t.element_size())


def test_moe_layer_qwen_end_to_end(cuda):
    """The whole decode block (router GEMV, top-8, grouping, experts, shared expert, gated combine) through MoELayer,
    against the oracle's restatement of call stack A."""
    cfg = synth.QWEN
    layer = synth.make_layer(cfg, seed=0)
    rng = np.random.default_rng(0)
    Tn = 4
    h = synth.rms_normed(rng, Tn, cfg["n_embd"])
    M = T.MoELayer(cfg, dev(layer["blobs"]), dev(layer["router"]), dev(layer["sh_blob"]), max_tokens=8)
    x = torch.zeros((Tn, cfg["n_embd"]), device="cuda")
    hd = dev(h)
    hq = T.quantize_q8_1_rows(hd)
    M.forward(x, hd, hq)
    torch.cuda.synchronize()
    logits = M.logits[:Tn].cpu().numpy()
    ref = O.moe_layer(layer, h, logits=logits)
    assert np.array_equal(M.ids[:Tn].cpu().numpy(), ref["ids"])
    assert np.allclose(M.w[:Tn].cpu().numpy(), ref["w"], rtol=2e-6)
    err, cos = layer_tolerance(x.cpu().numpy(), ref["out"])
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)
    assert T.device_error() == 0


# ------------------------------------------------------------------------------------------------ slot products
@pytest.mark.parametrize("t,n_in,n_out", [(synth.T_Q4_0, 2816, 704), (synth.T_Q4_0, 704, 2816), (synth.T_Q8_0, 2048, 512),
                                          (synth.T_Q4_K, 2048, 1792), (synth.T_Q6_K, 1792, 2048),
                                          (synth.T_IQ3_XXS, 2048, 512), (synth.T_IQ3_S, 512, 2048)])
def test_mmvq_slots_and_ids_vs_reference_mmvq(cuda, t, n_in, n_out):
    """tsb_mmvq_run_slots / _ids (gemma_native_mmvq_slots / _ids): 32 matrices, each with its own q8_1 column, in one
    launch, against the reference's own iq_mmvq one matrix at a time on the same buffers -- bit for bit for the
    formats whose call values carry no fused multiply-add, within 1e-6 relative otherwise -- and the ids form (device
    table of matrices, ids with repeats, columns shared by x_every entries) against the slots form."""
    R = ref_or_skip()
    rng = np.random.default_rng(200 + t)
    n = 32
    rb = synth.row_bytes(t, n_in)
    mats = [dev(synth.gen_matrix(rng, t, n_out, n_in, 0.02)) for _ in range(n)]
    xs = [dev(O.quantize_q8_1(rng.normal(0, 1, size=(1, n_in)).astype(np.float32))[0]) for _ in range(n)]
    ys = [torch.full((n_out,), float("nan"), device="cuda") for _ in range(n)]
    T.mmvq_slots(t, mats, xs, ys, n_in, n_out)
    ref = [torch.zeros(n_out, device="cuda") for _ in range(n)]
    if t != synth.T_Q6_K:   # the reference's iq_mmvq has no Q6_K (STRATA_MMVQ_FMTS, iq_kernels.cu:705): the oracle
        for i in range(n):
            R.ref_iq_mmvq(t, refgpu.ptr(mats[i]), refgpu.ptr(xs[i]), refgpu.ptr(ref[i]), n_in, n_out, 1,
                          refgpu.stream())
    torch.cuda.synchronize()
    assert T.device_error() == 0
    for i in range(n):
        a = ys[i].cpu().numpy()
        if t == synth.T_Q6_K:
            b = O.mat_vec(t, mats[i].cpu().numpy(), xs[i].cpu().numpy(), n_in, n_out)
            assert np.allclose(a, b, rtol=1e-5, atol=1e-5 * np.abs(b).max()), i
            continue
        b = ref[i].cpu().numpy()
        if t in EXACT_FLOAT:
            assert np.array_equal(a, b), i
        else:
            assert np.allclose(a, b, rtol=1e-6, atol=1e-6 * np.abs(b).max()), i
    # the ids form: matrix j = table[ids[j]], column j // 4, outputs y_stride apart
    table = torch.tensor([m.data_ptr() for m in mats], dtype=torch.int64, device="cuda")
    ids = torch.from_numpy(rng.integers(0, n, size=16).astype(np.int32)).cuda()
    xcat = torch.stack(xs[:4])                       # 4 columns, each shared by 4 entries
    y_stride = n_out + 16
    ycat = torch.full((16, y_stride), float("nan"), device="cuda")
    T.mmvq_ids(t, table, ids, 0, xcat, xcat.stride(0), 4, ycat, y_stride, 16, n_in, n_out)
    want = [torch.full((n_out,), float("nan"), device="cuda") for _ in range(16)]
    idl = ids.cpu().tolist()
    T.mmvq_slots(t, [mats[idl[j]] for j in range(16)], [xs[j // 4] for j in range(16)], want, n_in, n_out)
    torch.cuda.synchronize()
    for j in range(16):
        assert torch.equal(ycat[j, :n_out], want[j]), j
    assert torch.isnan(ycat[:, n_out:]).all()
