"""The fused decode kernel (tsb_moe_decode_layers, one persistent launch for every layer of a step) against the
layer-by-layer entry points (MoELayer, whose pieces test_gpu_parity pins to the reference's kernels and the oracle),
and its first layer against the oracle's restatement of the whole block, on the same device weights."""
import numpy as np
import pytest
import torch

import tinystrata_b200 as T
from oracle import oracle as O
from tinystrata_b200 import synth

pytestmark = pytest.mark.gpu


def tol(mine, ref):
    mine = np.asarray(mine, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    rms = np.sqrt(np.mean(ref ** 2))
    return float(np.abs(mine - ref).max() / rms), float(mine @ ref / (np.linalg.norm(mine) * np.linalg.norm(ref)))


@pytest.fixture(scope="module")
def stack(cuda):
    cfg = synth.QWEN
    st = synth.device_layers(cfg, 3, seed=11, device=cuda)
    torch.cuda.synchronize()
    return cfg, st


@pytest.mark.parametrize("Tn", [1, 4, 16])
def test_fused_decode_matches_layerwise(cuda, stack, Tn):
    cfg, st = stack
    H = cfg["n_embd"]
    rng = np.random.default_rng(Tn)
    x0 = torch.from_numpy(rng.normal(0, 1, size=(Tn, H)).astype(np.float32)).to(cuda)
    # layer by layer
    layers = [T.MoELayer(cfg, st["blobs"][l], st["routers"][l], st["sh_blobs"][l], max_tokens=Tn) for l in range(3)]
    x1 = x0.clone()
    h = torch.empty_like(x1)
    hq = torch.empty((Tn, H // 32 * 36), dtype=torch.uint8, device=cuda)
    T.rms_norm_q8_1(x1, h, hq)
    ids_ref = []
    for M in layers:
        M.forward(x1, h, hq, h_next=h, hq_next=hq)
        ids_ref.append(M.ids[:Tn].clone())
    # fused
    D = T.DecodeStack(cfg, st["blobs"], st["routers"], st["sh_blobs"], n_tok=Tn)
    x2 = x0.clone()
    D.forward(x2)
    torch.cuda.synchronize()
    assert D.error() == 0, " ".join(str(v) for v in D.error_detail)
    assert T.device_error() == 0
    for l in range(3):
        assert torch.equal(D.ids[l], ids_ref[l]), f"layer {l} routing"
    err, cos = tol(x2.cpu().numpy(), x1.cpu().numpy())
    assert err <= 1e-4 and cos >= 0.999999, (err, cos)


def test_fused_decode_first_layer_vs_oracle(cuda, stack):
    cfg, st = stack
    H = cfg["n_embd"]
    rng = np.random.default_rng(5)
    x0 = synth.rms_normed(rng, 2, H)
    one = {k: v[:1] for k, v in st.items() if k in ("blobs", "routers", "sh_blobs")}
    D = T.DecodeStack(cfg, one["blobs"], one["routers"], one["sh_blobs"], n_tok=2)
    x = torch.from_numpy(x0).to(cuda)
    D.forward(x)
    torch.cuda.synchronize()
    assert D.error() == 0
    layer = {"cfg": cfg, "blobs": st["blobs"][0].cpu().numpy(), "router": st["routers"][0].cpu().numpy(),
             "sh_blob": st["sh_blobs"][0].cpu().numpy()}
    h, _ = O.rms_q8_1(x0)
    ref = O.moe_layer(layer, h)
    assert np.array_equal(D.ids[0].cpu().numpy(), ref["ids"])
    err, cos = tol(x.cpu().numpy() - x0, ref["out"])
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)


def test_fused_decode_rejects_unsupported(cuda, stack):
    cfg, st = stack
    bad = dict(cfg, n_ff=1024)
    with pytest.raises(Exception):
        T.DecodeStack(bad, st["blobs"], st["routers"], st["sh_blobs"], n_tok=1).forward(
            torch.zeros((1, cfg["n_embd"]), device=cuda))
    with pytest.raises(Exception):
        T.DecodeStack(cfg, st["blobs"], st["routers"], st["sh_blobs"], n_tok=17).forward(
            torch.zeros((17, cfg["n_embd"]), device=cuda))
