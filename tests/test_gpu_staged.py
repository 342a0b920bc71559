"""Host-staged experts (the reference's hybrid mode, src/qwen35/q36_engine.cu:423-452, 2995-3049, 3052-3265): a layer
whose experts live in pinned host memory with some of them in HBM slots gives the resident layer's outputs bit for
bit -- the entries of experts without a slot run on the GPU after the kernel pulled their blobs over the host link --
before and after a rebalance moves experts into the slots, and inside a captured CUDA graph.  The streamed prompt
layer (tsb_stage_layer) assembles the layer's bytes exactly with the reference's runs of copies."""
import numpy as np
import pytest
import torch

import tinystrata_b200 as T
from tinystrata_b200 import synth
from tinystrata_b200.layer import MoELayer, StagedExperts

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def pinned_blobs(blobs: np.ndarray) -> torch.Tensor:
    """Every expert's blob in pinned host memory, rows 16-byte aligned (stride rounded up to 16)."""
    E, nb = blobs.shape
    stride = (nb + 15) // 16 * 16
    h = torch.zeros((E, stride), dtype=torch.uint8).pin_memory()
    h[:, :nb] = torch.from_numpy(blobs)
    return h


def layer_kw(layer):
    return dict(escale=dev(layer["escale"]) if layer.get("escale") is not None else None,
                bias=dev(layer["bias"]) if layer.get("bias") is not None else None)


@pytest.mark.parametrize("name,n_expert,n_slots,Tn", [("QWEN", 64, 24, 1), ("QWEN", 64, 24, 16), ("LFM", 64, 20, 8),
                                                      ("GEMMA", 32, 0, 4), ("QWEN", 32, 32, 4)])
def test_staged_layer_equals_resident(cuda, name, n_expert, n_slots, Tn):
    cfg = dict(getattr(synth, name), n_expert=n_expert)
    layer = synth.make_layer(cfg, seed=40 + n_slots + Tn)
    rng = np.random.default_rng(Tn)
    h = synth.rms_normed(rng, Tn, cfg["n_embd"])
    hd = dev(h)
    hq = T.quantize_q8_1_rows(hd)
    sh = dev(layer["sh_blob"]) if layer.get("sh_blob") is not None else None
    router = dev(layer["router"])
    R = MoELayer(cfg, dev(layer["blobs"]), router, sh, max_tokens=Tn, **layer_kw(layer))
    host = pinned_blobs(layer["blobs"])
    S = StagedExperts(host, layer["blobs"].shape[1], n_slots, Tn * cfg["n_used"], cuda)
    M = MoELayer(cfg, None, router, sh, max_tokens=Tn, staged=S, **layer_kw(layer))
    xr = torch.zeros((Tn, cfg["n_embd"]), device=cuda)
    R.forward(xr, hd, hq)
    xs = torch.zeros_like(xr)
    M.forward(xs, hd, hq)
    torch.cuda.synchronize()
    assert T.device_error() == 0
    ids = R.ids[:Tn].cpu().numpy()
    assert np.array_equal(M.ids[:Tn].cpu().numpy(), ids)
    n_ent = Tn * cfg["n_used"]
    assert torch.equal(M.parts[:n_ent], R.parts[:n_ent]), "staged expert rows differ from the resident layer's"
    assert torch.equal(xs, xr)
    # the usage record: one count per entry
    want = np.bincount(ids.ravel(), minlength=n_expert)
    assert np.array_equal(S.counts.cpu().numpy(), want)
    # which groups were staged: the used experts without a slot, each fetched once, bytes equal to the host blob
    used = np.unique(ids)
    missed = [x for x in used if S.slot_of[x] < 0]
    nb = layer["blobs"].shape[1]
    for m, x in enumerate(missed):
        assert torch.equal(S.stage[m, :nb].cpu(), host[x, :nb]), f"stage blob {m} is not expert {x}"
    # rebalance: the most-used experts take slots (copies on the stream, then the slot table); outputs unchanged
    if 0 < n_slots < n_expert:
        moved = S.rebalance(max_swaps=n_slots)
        torch.cuda.synchronize()
        assert moved > 0 or not missed
        if len(used) <= n_slots:   # every used expert outranks the unused residents: all of them now have slots
            assert all(S.slot_of[x] >= 0 for x in used)
        for s_, x in enumerate(S.exp_in_slot):
            assert S.slot_of[x] == s_
            assert torch.equal(S.slots[s_, :nb].cpu(), host[x, :nb]), f"slot {s_} does not hold expert {x}"
        assert np.array_equal(S.slot_of_d.cpu().numpy(), S.slot_of)
        xs2 = torch.zeros_like(xr)
        M.forward(xs2, hd, hq)
        torch.cuda.synchronize()
        assert torch.equal(xs2, xr)


def test_staged_layer_in_a_cuda_graph(cuda):
    """The staged step (routing, grouping with the host fetch, experts, combine) captured once and replayed on new
    inputs: the replay equals the resident layer's eager step on the same inputs."""
    cfg = dict(synth.QWEN, n_expert=64)
    layer = synth.make_layer(cfg, seed=7)
    Tn = 4
    host = pinned_blobs(layer["blobs"])
    S = StagedExperts(host, layer["blobs"].shape[1], 16, Tn * cfg["n_used"], cuda)
    sh, router = dev(layer["sh_blob"]), dev(layer["router"])
    R = MoELayer(cfg, dev(layer["blobs"]), router, sh, max_tokens=Tn)
    M = MoELayer(cfg, None, router, sh, max_tokens=Tn, staged=S)
    hd = torch.zeros((Tn, cfg["n_embd"]), device=cuda)
    hq = torch.empty((Tn, cfg["n_embd"] // 32 * 36), dtype=torch.uint8, device=cuda)
    xs = torch.zeros((Tn, cfg["n_embd"]), device=cuda)
    s = torch.cuda.Stream()
    rng = np.random.default_rng(3)
    hd.copy_(dev(synth.rms_normed(rng, Tn, cfg["n_embd"])))
    with torch.cuda.stream(s):   # warm-up outside the capture (first-call lookups)
        T.quantize_q8_1_rows(hd, hq, stream=s)
        M.forward(xs, hd, hq, stream=s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        xs.zero_()
        T.quantize_q8_1_rows(hd, hq, stream=s)
        M.forward(xs, hd, hq, stream=s)
    for seed in (11, 12):
        h = synth.rms_normed(np.random.default_rng(seed), Tn, cfg["n_embd"])
        hd.copy_(dev(h))
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        xr = torch.zeros_like(xs)
        R.forward(xr, hd, T.quantize_q8_1_rows(hd))
        torch.cuda.synchronize()
        assert torch.equal(xs, xr)
    assert T.device_error() == 0
    del g


def expected_runs(slot_of, n_slots, E):
    runs, x = 0, 0
    res = lambda i: 0 <= slot_of[i] < n_slots   # noqa: E731
    while x < E:
        y = x + 1
        if res(x):
            while y < E and res(y) and slot_of[y] == slot_of[y - 1] + 1:
                y += 1
        else:
            while y < E and not res(y):
                y += 1
        runs += 1
        x = y
    return runs


@pytest.mark.parametrize("n_slots,whole", [(40, False), (40, True), (10, False), (64, False)])
def test_stage_layer_assembles_the_layer(cuda, n_slots, whole):
    """The streamed prompt layer: runs of consecutive slots device to device, runs of unplaced experts host to device
    (one whole-layer copy below half residency or when asked); the stage buffer equals the host layer byte for byte
    and, as the tensor-core prompt products' weights, gives the resident layer's outputs."""
    cfg = dict(synth.GEMMA, n_expert=64)
    rng = np.random.default_rng(n_slots)
    E = cfg["n_expert"]
    blobs = np.stack([synth.gen_blob(rng, cfg) for _ in range(E)])
    host = pinned_blobs(blobs)
    # slots 0 .. n_slots/2 - 1 hold experts 5, 6, ... (one device-to-device run), the rest a random choice
    block = np.arange(5, 5 + n_slots // 2, dtype=np.int32)
    rest = rng.permutation(np.setdiff1d(np.arange(E), block))[: n_slots - block.size]
    resident = np.concatenate([block, rest]).astype(np.int32)
    S = StagedExperts(host, blobs.shape[1], n_slots, 8, cuda, resident=resident)
    stage = torch.empty((E, S.stride), dtype=torch.uint8, device=cuda)
    n = T.stage_layer(S.slot_of, n_slots, S.slots, host, S.stride, stage, whole=whole)
    torch.cuda.synchronize()
    want = 1 if (whole or 2 * n_slots < E) else expected_runs(S.slot_of, n_slots, E)
    assert n == want
    assert torch.equal(stage.cpu(), host)
    # the prompt products on the staged layer: bit for bit the resident layer's
    layer = synth.make_layer(cfg, seed=5, n_expert=1)
    layer["blobs"] = blobs
    Tn = 48
    h = synth.rms_normed(rng, Tn, cfg["n_embd"])
    kw = layer_kw(layer)
    sh, router = dev(layer["sh_blob"]), dev(layer["router"])
    from tinystrata_b200.layer import PrefillLayer
    P1 = PrefillLayer(cfg, dev(blobs), router, sh, max_tokens=Tn, **kw)
    P2 = PrefillLayer(cfg, stage[:, :blobs.shape[1]], router, sh, max_tokens=Tn, **kw)
    x1 = torch.zeros((Tn, cfg["n_embd"]), device=cuda)
    x2 = torch.zeros_like(x1)
    P1.forward(x1, dev(h))
    P2.forward(x2, dev(h))
    torch.cuda.synchronize()
    assert torch.equal(x1, x2)
    assert T.device_error() == 0
