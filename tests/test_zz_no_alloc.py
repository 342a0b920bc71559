"""tsb_native_expert_grouped_noalloc (the library's fixed device scratch) against tsb_native_expert_grouped (a caller
scratch buffer) on the same inputs: two calls in a row with different routing, each equal to the caller-scratch entry
point, and an oversize call refused before any launch.  Collected last on purpose (file name), so it also runs after
every other GPU test has used the library."""
import numpy as np
import pytest
import torch

import tinystrata_b200 as T
from oracle import oracle as O
from tinystrata_b200 import synth

pytestmark = pytest.mark.gpu

TOL = 1e-6   # max-abs over RMS; the two entry points run the same kernels, so the results are expected bit for bit


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def _case(cfg, n_mat, ids, seed):
    layer = synth.make_layer(cfg, seed, n_expert=n_mat)
    rng = np.random.default_rng(seed)
    Tn, K = ids.shape
    H, F = cfg["n_embd"], cfg["n_ff"]
    xq = _dev(O.quantize_q8_1(synth.rms_normed(rng, Tn, H)))
    blobs = _dev(layer["blobs"])
    L = T.native_expert_layout(cfg["gu_type"], cfg["d_type"], H, F)
    g = T.moe_group(_dev(ids), n_mat, blobs, int(L.bytes))
    n_ent = Tn * K
    scratch = torch.empty(T.native_expert_scratch_bytes(n_ent, F) // 4, dtype=torch.float32, device="cuda")
    ref = torch.full((n_ent, H), float("nan"), device="cuda")
    T.native_expert_grouped(L, g, n_ent, n_ent, xq, scratch, ref)
    return L, g, xq, n_ent, ref, blobs


def _close(a, b):
    rms = float(torch.sqrt(torch.mean(b.double() ** 2)))
    return float((a.double() - b.double()).abs().max()) / rms


@pytest.mark.parametrize("cfg_name", ["QWEN", "LFM"])
def test_noalloc_matches_caller_scratch_twice(cuda, cfg_name):
    cfg = getattr(synth, cfg_name)
    K = cfg["n_used"]
    rng = np.random.default_rng(2024)
    ids_a = np.stack([rng.choice(12, K, replace=False) for _ in range(4)]).astype(np.int32)
    ids_b = np.stack([rng.choice(12, K, replace=False) for _ in range(2)]).astype(np.int32)
    A = _case(cfg, 12, ids_a, seed=5)
    B = _case(cfg, 12, ids_b, seed=6)
    outs = []
    for L, g, xq, n_ent, ref, _ in (A, B):   # two calls in a row, different routing and tokens
        out = torch.full_like(ref, float("nan"))
        T.native_expert_grouped_noalloc(L, g, n_ent, n_ent, xq, out)
        outs.append(out)
    torch.cuda.synchronize()
    for out, case in zip(outs, (A, B)):
        ref = case[4]
        assert torch.isfinite(out).all()
        assert _close(out, ref) <= TOL
    assert T.device_error() == 0


def test_noalloc_refuses_oversize(cuda):
    cfg = synth.QWEN
    rng = np.random.default_rng(7)
    ids = np.stack([rng.choice(12, 8, replace=False) for _ in range(2)]).astype(np.int32)
    L, g, xq, n_ent, ref, _ = _case(cfg, 12, ids, seed=8)
    out = torch.full_like(ref, float("nan"))
    too_many = (1 << 20) // (cfg["n_ff"] * 4) + 1   # one entry more than the fixed 1 MiB holds at n_ff 512
    with pytest.raises(T.TsbError, match="status -5"):
        T.native_expert_grouped_noalloc(L, g, n_ent, too_many, xq, out)
    torch.cuda.synchronize()
    assert torch.isnan(out).all()   # nothing was launched
