"""The Gemma 4 / LFM2 decode MoE block in one launch (tsb_moe_decode_act) against the layer-by-layer entry points
(route_rows, grouping, grouped experts with GELU-tanh / clamped SwiGLU, moe_sum, the dense shared MLP) on the same
device weights: logits, picks, weights, the shared MLP's output and the layer output bit for bit, at 1, 4 and 16
tokens, with and without per-expert scales / routing bias."""
import numpy as np
import pytest
import torch

import tinystrata_b200 as T
from tinystrata_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", params=["GEMMA", "LFM"])
def stack(request, cuda):
    cfg = dict(getattr(synth, request.param))
    st = synth.device_layers(cfg, 1, seed=21, device=cuda)
    torch.cuda.synchronize()
    return cfg, st


@pytest.mark.parametrize("Tn,route_extra", [(1, False), (4, True), (16, True)])
def test_fused_act_decode_equals_layerwise(cuda, stack, Tn, route_extra):
    cfg, st = stack
    H, E = cfg["n_embd"], cfg["n_expert"]
    rng = np.random.default_rng(Tn)
    kw = {}
    if cfg["router_mode"] == "softmax_scaled":
        es = rng.uniform(0.5, 1.5, E).astype(np.float32) if route_extra else np.ones(E, np.float32)
        kw["escale"] = torch.from_numpy(es).to(cuda)
    else:
        b = rng.normal(0, 0.01, E).astype(np.float32) if route_extra else np.zeros(E, np.float32)
        kw["bias"] = torch.from_numpy(b).to(cuda)
    sh = st["sh_blobs"][0] if cfg.get("sh_n_ff") else None
    M = T.MoELayer(cfg, st["blobs"][0], st["routers"][0], sh, max_tokens=16, **kw)
    h = torch.from_numpy(synth.rms_normed(rng, Tn, H)).to(cuda)
    hq = T.quantize_q8_1_rows(h)
    x0 = torch.from_numpy(rng.normal(0, 1, size=(Tn, H)).astype(np.float32)).to(cuda)
    xm = x0.clone()
    M.forward(xm, h, hq)
    torch.cuda.synchronize()
    ids_m, w_m, lg_m = M.ids[:Tn].clone(), M.w[:Tn].clone(), M.logits[:Tn, :E].clone()
    sh_m = M.shared[:Tn].clone() if sh is not None else None
    M.ids.fill_(-1)
    M.w.zero_()
    if sh is not None:
        M.shared.zero_()
    xf = x0.clone()
    M.forward_fused(xf, h, hq)
    torch.cuda.synchronize()
    assert T.device_error() == 0
    assert torch.equal(M.fused_logits, lg_m), "router logits differ"
    assert torch.equal(M.ids[:Tn], ids_m), "picks differ"
    assert torch.equal(M.w[:Tn], w_m), "weights differ"
    if sh is not None:
        assert torch.equal(M.shared[:Tn], sh_m), "shared MLP output differs"
    assert torch.equal(xf, xm), f"layer output differs: max {float((xf - xm).abs().max())}"


def test_fused_act_decode_refuses_what_it_does_not_run(cuda):
    cfg = dict(synth.GEMMA, n_tok=1)
    d = T.decode_act_desc(synth.GEMMA, 17, True)   # 17 tokens
    ws = torch.empty(1 << 20, dtype=torch.float32, device=cuda)
    x = torch.zeros((17, cfg["n_embd"]), device=cuda)
    with pytest.raises(T.TsbError):
        T.moe_decode_act(d, x, x, x, x, 0, x, ws)
    d = T.decode_act_desc(dict(synth.QWEN, router_mode="sigmoid"), 1, False)   # IQ3_XXS experts
    with pytest.raises(T.TsbError):
        T.moe_decode_act(d, x, x, x, x, 0, x, ws)
