"""Expert-parallel prefill on CPU ranks (gloo): the destination plan, the deduplicated dispatch of q8_1 rows with their
local picks, the return of the partial rows and the rank-ordered sum, bit for bit against a single-process
computation of the same per-rank partial sums (a synthetic expert function stands in for the GPU experts)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

E, K, H, T = 16, 4, 64, 37


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tokens(rank):
    g = torch.Generator().manual_seed(100 + rank)
    xq = torch.randint(0, 256, (T, H // 32 * 36), generator=g, dtype=torch.uint8)
    ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(torch.int32)
    w = torch.rand((T, K), generator=g)
    return xq, ids, w


def _expert(rows, e):
    """A stand-in expert: the q8_1 row's code bytes as floats, scaled and shifted per global expert id e."""
    codes = rows.view(rows.shape[0], -1, 36)[:, :, 4:].reshape(rows.shape[0], -1).to(torch.int8).float()
    return codes * (1.0 + 0.01 * e.float().unsqueeze(1)) + e.float().unsqueeze(1)


def _partials(rows, rids, rw, base, stride=1):
    """The expert_fn contract: per row sum over k of w_k expert(row, base + stride id_k), ids < 0 weigh 0 (pick
    order); stride 1 for block placement (base = first expert of the rank), G for cyclic (base = the rank)."""
    R, Kk = rids.shape
    valid = rids >= 0
    gid = torch.where(valid, rids * stride + base, torch.full_like(rids, base))
    wk = torch.where(valid, rw, torch.zeros_like(rw))
    acc = _expert(rows, gid[:, 0]) * wk[:, 0:1]
    for k in range(1, Kk):
        acc = torch.addcmul(acc, _expert(rows, gid[:, k]), wk[:, k:k + 1])
    return acc


def _reference(xq, ids, w, world, cyclic):
    per = E // world
    out = torch.zeros((T, H))
    dest = ids.long() % world if cyclic else ids.long() // per
    local = ids.long() // world if cyclic else ids.long() - dest * per
    for d in range(world):
        sel = (dest == d).any(dim=1).nonzero().view(-1)
        if len(sel) == 0:
            continue
        lid = torch.where(dest[sel] == d, local[sel], torch.full_like(local[sel], -1)).to(torch.int32)
        out[sel] += _partials(xq[sel], lid, w[sel], d if cyclic else d * per, world if cyclic else 1)
    return out


def _worker(rank, world, port, q, cyclic):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from tinystrata_b200.ep import EPPlan, ep_forward
        xq, ids, w = _tokens(rank)
        per = E // world
        base, stride = (rank, world) if cyclic else (rank * per, 1)
        out = ep_forward(xq, ids, w, E, H, lambda rows, rids, rw: _partials(rows, rids, rw, base, stride),
                         cyclic=cyclic)
        ref = _reference(xq, ids, w, world, cyclic)
        plan = EPPlan(ids, w, E, world, cyclic)
        dedup = int(plan.counts.sum())
        dest = ids.long() % world if cyclic else ids.long() // per
        q.put((rank, bool(torch.equal(out, ref)), float((out - ref).abs().max()), dedup,
               int((dest.unsqueeze(2) == torch.arange(world)).any(1).sum())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,cyclic", [(2, False), (4, False), (2, True), (4, True)])
def test_ep_forward_matches_single_process(world, cyclic):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, cyclic)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, equal, err, dedup, distinct in res:
        assert equal, (rank, err)
        assert dedup == distinct   # one row per (token, destination rank), not per pick


def test_ep_plan_dedup_and_order():
    from tinystrata_b200.ep import EPPlan
    ids = torch.tensor([[0, 5, 6, 15], [8, 9, 1, 2], [12, 13, 14, 3]], dtype=torch.int32)
    w = torch.arange(12, dtype=torch.float32).view(3, 4)
    p = EPPlan(ids, w, 16, 4)   # 4 experts per rank
    assert p.counts.tolist() == [3, 1, 1, 2]
    assert [t.tolist() for t in p.send_tok] == [[0, 1, 2], [0], [1], [0, 2]]
    # token 1's row for rank 0 carries its picks 1 and 2 (local ids 1, 2) and nothing else
    assert p.send_ids[1].tolist() == [-1, -1, 1, 2]
    assert p.send_w[1].tolist() == [0.0, 0.0, 6.0, 7.0]


def test_ep_plan_cyclic():
    from tinystrata_b200.ep import EPPlan
    ids = torch.tensor([[0, 5, 6, 15], [8, 9, 1, 2]], dtype=torch.int32)
    w = torch.arange(8, dtype=torch.float32).view(2, 4)
    p = EPPlan(ids, w, 16, 4, cyclic=True)   # expert e on rank e % 4 as local expert e // 4
    assert p.counts.tolist() == [2, 2, 2, 1]   # token 0 reaches every rank, token 1 ranks 0, 1, 2
    assert [t.tolist() for t in p.send_tok] == [[0, 1], [0, 1], [0, 1], [0]]
    # rows in rank order: row 2 is token 0's for rank 1 (pick 1: expert 5 -> local 1), row 3 token 1's for rank 1
    # (picks 9 and 1 -> local 2 and 0)
    assert p.send_ids[2].tolist() == [-1, 1, -1, -1]
    assert p.send_ids[3].tolist() == [-1, 2, 0, -1]
