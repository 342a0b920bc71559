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


# ------------------------------------------------------------------------------------------------ the device path
def _ep_worker(rank, world, port, q, scenario):
    import datetime
    import torch.distributed as dist
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    # gloo carries only the NCCL id: the exchanges run on the library's own communicator
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import tinystrata_b200 as T
        from oracle import oracle as O
        from tinystrata_b200 import synth
        from tinystrata_b200.ep import ExpertParallel
        cfg = dict(synth.QWEN_EP, n_expert=16)
        E, K, H, F, FS = cfg["n_expert"], cfg["n_used"], cfg["n_embd"], cfg["n_ff"], cfg["sh_n_ff"]
        layer = synth.make_layer(cfg, 71)   # the same weights on every rank
        L = T.native_expert_layout(cfg["gu_type"], cfg["d_type"], H, F)
        Ls = T.native_expert_layout(cfg["sh_gu_type"], cfg["sh_d_type"], H, FS)
        mine = torch.from_numpy(layer["blobs"][rank::world].copy()).to(dev)   # cyclic placement
        sh = torch.from_numpy(layer["sh_blob"]).to(dev)
        ep = ExpertParallel(L, mine, int(L.bytes), E, K, cfg["act"], max_tokens=160, cyclic=True)
        ep.set_timeout(3.0 if scenario == "timeout" else 60.0)
        results = []
        steps = [(1, False, 100), (2, False, 100), (3, True, 100), (2, False, 0 if rank == 1 else 37)]
        if scenario == "timeout":
            steps = steps[:1] + [(2, False, 50)]
        for i, (mb, bf16, T_tok) in enumerate(steps):
            if scenario == "timeout" and i == 1 and rank == 1:
                q.put((rank, "left", None))
                q.close()
                q.join_thread()   # the message is out of this process before it ends
                os._exit(0)   # between steps, nothing in flight: the peer never answers the next exchange
            rng = np.random.default_rng(80 + 10 * rank + i)
            x = synth.rms_normed(rng, T_tok, H) if T_tok else np.zeros((0, H), np.float32)
            xd = torch.from_numpy(x).to(dev)
            ids = (np.stack([rng.choice(E, K, replace=False) for _ in range(T_tok)]).astype(np.int32) if T_tok
                   else np.zeros((0, K), np.int32))
            w = rng.random((T_tok, K)).astype(np.float32)
            sg = rng.normal(0, 1, size=T_tok).astype(np.float32)
            xq = T.quantize_q8_1_rows(xd) if T_tok else torch.zeros((0, H // 32 * 36), dtype=torch.uint8, device=dev)
            out = torch.full((T_tok, H), float("nan"), device=dev)
            try:
                ep.dispatch(xq, torch.from_numpy(ids).to(dev), torch.from_numpy(w).to(dev), micro_batches=mb)
            except T.TsbError as e:
                results.append(("error", str(e)))
                break
            shared = None
            if T_tok:   # the shared expert on the caller's stream while the rows travel
                hs = T.moe_prefill_gu(Ls, sh, 0, None, 1, T_tok, T.mmq_quantize(xd), cfg["act"])
                shared = T.moe_prefill_down(Ls, sh, 0, None, 1, T_tok, hs)
            sgd = torch.from_numpy(sg).to(dev)
            ep.combine(out, accumulate=False, shared=shared, sgate=sgd if T_tok else None, bf16=bf16)
            ep.synchronize()           # bounded: a peer that never answers ends here with an error
            torch.cuda.synchronize()
            st = ep.stats()
            if T_tok == 0:
                results.append(("empty", out.numel(), st))
                continue
            xqn = xq.cpu().numpy()
            parts = O.experts_for_tokens(cfg["gu_type"], cfg["d_type"], layer["blobs"], H, F, xqn, ids, cfg["act"])
            shr = np.stack([O.expert_ffn(cfg["sh_gu_type"], cfg["sh_d_type"], layer["sh_blob"], H, FS, xqn[t],
                                         cfg["act"]) for t in range(T_tok)])
            ref = O.combine(None, parts, w, shr, O.sigmoid(sg))
            m = out.cpu().numpy().astype(np.float64).ravel()
            r = np.asarray(ref, np.float64).ravel()
            err = float(np.abs(m - r).max() / np.sqrt(np.mean(r ** 2)))
            cos = float(m @ r / (np.linalg.norm(m) * np.linalg.norm(r)))
            results.append((mb, bf16, err, cos, st))
        q.put((rank, results, T.device_error()))
        ep.close()
    except Exception as e:   # reported to the parent, which fails the test
        import traceback
        q.put((rank, "exception: " + repr(e) + traceback.format_exc(), None))
    finally:
        dist.destroy_process_group()


def _run_ep(scenario):
    import torch.multiprocessing as mp
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_ep_worker, args=(r, world, port, q, scenario)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict((r, (a, b)) for r, a, b in (q.get(timeout=600) for _ in range(world)))
    for p in procs:
        p.join(timeout=60)
    return res


def test_ep_device_path_two_gpus_vs_oracle():
    """tsb_ep_* on 2 GPUs (Qwen-EP formats: IQ3_XXS gate/up, IQ3_S down, Q8_0 shared expert gated by a sigmoid),
    cyclic placement, 1 / 2 / 3 micro-batches, fp32 and bf16 returns, and a step where one rank has no tokens: every
    token's layer output against the oracle's fp64-accumulated experts within the layer tolerance."""
    if torch.cuda.device_count() < 2:
        pytest.skip("expert parallelism needs two GPUs")
    res = _run_ep("normal")
    sent_total = 0
    recv_total = 0
    for rank, (results, derr) in res.items():
        assert isinstance(results, list), (rank, results)
        assert derr == 0, (rank, derr)
        for item in results:
            if item[0] == "empty":
                continue
            mb, bf16, err, cos, st = item
            # fp32 returns meet the layer bar; bf16 returns (half the return bytes) round each partial row to 8
            # significant bits, which moves the worst single value to ~1.6 % of the RMS at cosine 0.999999: the
            # library's default and the bench use fp32, and bf16 is held to 3e-2 here
            assert err <= (3e-2 if bf16 else 1e-2) and cos >= 0.9999, (rank, mb, bf16, err, cos)
        sent_total += results[0][4]["rows_sent"]
        recv_total += results[0][4]["rows_received"]
    assert sent_total == recv_total   # every row sent was received


def test_ep_peer_that_leaves_times_out():
    """A rank that leaves between steps: the other rank's next counts exchange gives up after its 3 s bound with
    TSB_ERR_COMM (the communicator aborted, the context still usable), instead of waiting for ever."""
    if torch.cuda.device_count() < 2:
        pytest.skip("expert parallelism needs two GPUs")
    res = _run_ep("timeout")
    assert res[1][0] == "left"
    results, derr = res[0]
    assert isinstance(results, list), results
    assert results[0][2] <= 1e-2, results[0]
    assert results[-1][0] == "error" and "status -6" in results[-1][1], results[-1]
    assert derr == 0
