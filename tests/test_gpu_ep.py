"""Expert-parallel prefill on 2 GPUs over NCCL: each rank holds half the experts of a Gemma-shaped Q4_0 layer and
routes its own tokens; the routed outputs (dispatch all-to-all, tensor-core experts, return all-to-all) against the
oracle's fp64-accumulated experts for the same tokens within the layer tolerance.  Needs two GPUs (skipped with one);
the host logic is covered bit for bit on CPU ranks by test_ep.py."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

T_TOK = 96


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        import tinystrata_b200 as T
        from oracle import oracle as O
        from tinystrata_b200 import synth
        from tinystrata_b200.ep import ep_forward, gpu_expert_fn
        cfg = dict(synth.GEMMA, n_expert=16)
        E, K, H, F = cfg["n_expert"], cfg["n_used"], cfg["n_embd"], cfg["n_ff"]
        layer = synth.make_layer(cfg, 51)   # the same weights on every rank
        per = E // world
        L = T.native_expert_layout(cfg["gu_type"], cfg["d_type"], H, F)
        mine = torch.from_numpy(layer["blobs"][rank * per:(rank + 1) * per].copy()).to(dev)
        rng = np.random.default_rng(60 + rank)
        x = synth.rms_normed(rng, T_TOK, H)
        ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T_TOK)]).astype(np.int32)
        w = rng.random((T_TOK, K)).astype(np.float32)
        xq = T.quantize_q8_1_rows(torch.from_numpy(x).to(dev))
        out = ep_forward(xq, torch.from_numpy(ids).to(dev), torch.from_numpy(w).to(dev), E, H,
                         gpu_expert_fn(L, mine, int(L.bytes), cfg["act"]))
        torch.cuda.synchronize()
        parts = O.experts_for_tokens(cfg["gu_type"], cfg["d_type"], layer["blobs"], H, F, xq.cpu().numpy(), ids,
                                     cfg["act"])
        ref = O.combine(None, parts, w)
        m = out.cpu().numpy().astype(np.float64).ravel()
        r = np.asarray(ref, np.float64).ravel()
        err = float(np.abs(m - r).max() / np.sqrt(np.mean(r ** 2)))
        cos = float(m @ r / (np.linalg.norm(m) * np.linalg.norm(r)))
        q.put((rank, err, cos, T.device_error()))
    except Exception as e:   # reported to the parent, which fails the test
        q.put((rank, repr(e), None, None))
    finally:
        dist.destroy_process_group()


def test_ep_prefill_two_gpus_vs_oracle():
    if torch.cuda.device_count() < 2:
        pytest.skip("expert parallelism needs two GPUs")
    import torch.multiprocessing as mp
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, err, cos, derr in res:
        assert cos is not None, (rank, err)
        assert err <= 1e-2 and cos >= 0.9999 and derr == 0, (rank, err, cos, derr)
