"""Expert parallelism on GPUs (hg_engine_ep_init): two ranks, each decoding its own sequences with
the routed experts split between them, must give every sequence exactly the logits and ids of
the one-GPU engine. Needs two GPUs (skipped otherwise); the ranks run as spawned processes with
NVLS off, and every wait is bounded by the process group's timeout."""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _gpus() -> int:
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, model, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist

    from hobbylm_b200 import Engine, ep, synth

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    ok, msg = True, ""
    try:
        prompts = [synth.prompt_ids(40 + 31 * i + 7 * rank, 100 * rank + i) for i in range(5)]
        ref = Engine.load(model, device=rank, max_batch=8)
        eng = Engine.load(model, device=rank, max_batch=8)
        ep.setup(eng)
        cr = [ref.new_cache() for _ in prompts]
        ce = [eng.new_cache() for _ in prompts]
        toks = []
        for p, a, b in zip(prompts, cr, ce):
            la = ref.prefill(a, p)
            lb = eng.prefill(b, p)
            assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
            la[50257:] = -np.inf
            toks.append(int(np.argmax(la)))
        ta, tb = list(toks), list(toks)
        for step in range(6):
            na, la = ref.decode_batch(cr, ta, want_logits=True)
            nb, lb = eng.decode_batch(ce, tb, want_logits=True)
            if not np.array_equal(la.view(np.uint32), lb.view(np.uint32)):
                ok, msg = False, f"step {step}: logits differ (max |d| {np.abs(la - lb).max()})"
                break
            ta, tb = [int(v) for v in na], [int(v) for v in nb]
        if ok:
            ga = ref.decode_greedy(cr, ta, 5)
            gb = eng.decode_greedy(ce, tb, 5)
            if not np.array_equal(ga, gb):
                ok, msg = False, "device-driven greedy ids differ"
        for c in cr + ce:
            c.close()
        eng.close()
        ref.close()
    except Exception as ex:  # report instead of hanging the other rank
        ok, msg = False, f"{type(ex).__name__}: {ex}"
    q.put((rank, ok, msg))
    dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < 2, reason="expert parallelism needs two GPUs")
@pytest.mark.parametrize("preset", ["130M", "500M"])
def test_expert_parallel_two_ranks_equal_one_gpu(preset):
    import torch.multiprocessing as mp

    from hobbylm_b200 import synth

    model = synth.cached_model(preset, 0)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, model, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    for rank, ok, msg in sorted(res):
        assert ok, f"rank {rank}: {msg}"
