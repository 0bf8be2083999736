"""Expert parallelism on the host (no GPU): the placement of hobbylm_b200.ep, the dispatch / expert
/ combine dataflow of the GPU kernels (ep.cu) restated over gloo ranks, and the rendezvous timeout.

The dataflow test runs W = 2 and 4 CPU ranks. Each rank routes its own tokens, packs every (token,
rank) row into a fixed-size block for the expert's owner (row count first, as k_ep_pack /
k_ep_headers do), exchanges blocks with one send/recv pair per peer (the NCCL group's shape),
computes only its own experts on the rows it received, sends the outputs back in the same slots,
and combines them in rank order followed by the shared expert (model.rs:300-323). The result must
equal the one-process MoE of the CPU oracle bit for bit, which is what lets the GPU engine split
experts across GPUs without changing a logit.
"""
import os
import socket
import time
from datetime import timedelta

import numpy as np
import pytest
import torch.multiprocessing as mp

from hobbylm_b200 import ep

K = 6


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_placement_splits_experts_evenly():
    for ne, world in ((36, 1), (36, 2), (36, 4), (64, 8), (32, 4)):
        owners = [ep.owner(e, ne, world) for e in range(ne)]
        for q in range(world):
            mine = list(ep.local_experts(q, ne, world))
            assert mine == [e for e in range(ne) if owners[e] == q]
            assert len(mine) == ne // world
    with pytest.raises(ValueError):
        ep.experts_per_rank(36, 5)


def _exchange(dist, blocks):
    """One fixed-size block to and from every peer, as one group of send/recv pairs."""
    rank, world = dist.get_rank(), dist.get_world_size()
    import torch

    out = [torch.empty_like(b) for b in blocks]
    reqs = []
    for p in range(world):
        if p == rank:
            out[p].copy_(blocks[p])
            continue
        reqs.append(dist.isend(blocks[p], p))
        reqs.append(dist.irecv(out[p], p))
    for r in reqs:
        r.wait()
    return out


def _rank_main(rank, world, port, tokens_per_rank, result_q):
    import torch
    import torch.distributed as dist

    import oracle
    from hobbylm_b200 import synth

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        inp = synth.moe_op_inputs(seed=2, T=world * tokens_per_rank)
        moe = oracle.Moe(inp["router"], inp["bias"], inp["gate_exps"], inp["up_exps"], inp["down_exps"],
                         inp["gate_sh"], inp["up_sh"], inp["down_sh"], top_k=K)
        ne, d = moe.ne, moe.d
        x = inp["x"][rank * tokens_per_rank:(rank + 1) * tokens_per_rank]
        y_ref, sel, w = moe.run(x, mode=0)  # the one-process MoE of these tokens, and their routing
        cap = tokens_per_rank * K
        # dispatch: [count, rows of (h, expert)] per destination
        send = [torch.zeros(1 + cap * (d + 1)) for _ in range(world)]
        sent = [[] for _ in range(world)]  # (t, r) of each sent slot
        for t in range(tokens_per_rank):
            for r in range(K):
                p = ep.owner(int(sel[t, r]), ne, world)
                i = len(sent[p])
                row = send[p][1 + i * (d + 1):1 + (i + 1) * (d + 1)]
                row[:d] = torch.from_numpy(x[t])
                row[d] = float(sel[t, r])
                sent[p].append((t, r))
        for p in range(world):
            send[p][0] = len(sent[p])
        recv = _exchange(dist, send)
        # this rank's experts on every received row; outputs go back in the same slots
        back = [torch.zeros(cap * d) for _ in range(world)]
        for p in range(world):
            n = int(recv[p][0])
            for i in range(n):
                row = recv[p][1 + i * (d + 1):1 + (i + 1) * (d + 1)].numpy()
                e = int(row[d])
                assert e in ep.local_experts(rank, ne, world), "row sent to a rank that does not own its expert"
                back[p][i * d:(i + 1) * d] = torch.from_numpy(moe.expert(row[:d].astype(np.float32), e))
        ret = _exchange(dist, back)
        ybuf = np.zeros((tokens_per_rank, K, d), np.float32)
        for p in range(world):
            for i, (t, r) in enumerate(sent[p]):
                ybuf[t, r] = ret[p][i * d:(i + 1) * d].numpy()
        # rank-order combine, then the shared expert (model.rs:300-323), in f32 without fusion
        out = np.zeros((tokens_per_rank, d), np.float32)
        for t in range(tokens_per_rank):
            o = np.zeros(d, np.float32)
            for r in range(K):
                o = o + np.float32(w[t, r] * np.float32(1.0)) * ybuf[t, r]
            o = o + moe.expert(x[t], -1)
            out[t] = o
        result_q.put((rank, bool(np.array_equal(out.view(np.uint32), y_ref.view(np.uint32))),
                      float(np.abs(out - y_ref).max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_dispatch_expert_combine_matches_one_process(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, 6, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok, err in sorted(results):
        assert ok, f"rank {rank}: max |d| {err}"


def _timeout_main(rank, world, port, result_q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    if rank != 0:
        time.sleep(12)  # joined the group but never reaches the id exchange
        result_q.put((rank, "idle", 0.0))
        return
    t0 = time.time()
    try:
        ep.exchange_id(lambda: b"\x01" * 128)
        result_q.put((rank, "returned", time.time() - t0))
    except Exception as ex:  # the process group's timeout ends the broadcast with an error
        result_q.put((rank, type(ex).__name__, time.time() - t0))


def test_id_exchange_times_out_when_a_rank_never_joins():
    """A rank that never takes part makes rank 0's rendezvous fail on the host within the process
    group's timeout (3 s here), before any NCCL communicator is created."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_timeout_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, what, secs = q.get(timeout=120)
        res[rank] = (what, secs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    what, secs = res[0]
    assert what not in ("returned", "idle"), res
    assert secs < 30, res
