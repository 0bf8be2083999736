#!/usr/bin/env python
"""Decode throughput of the hobbylm_b200 engine (the hobby-rs decode path on B200).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one process per GPU)

Workload (the headline): the 500M preset, random-init seed 0, Q8_0 GGUF
(context_length 16384 so prompt + decode fits), 256 sequences with prompt lengths ~ U[1024, 8192]
of random ids (torch.Generator seed 5). Sequences are sharded over the ranks with replicated
weights and no collective on the decode path (strong scaling: the 256 are fixed). A step
is one batched greedy decode step of every sequence (sequences are placed on ranks balanced by
prompt length); value = tokens of all ranks / max-over-ranks
device time. At N=1 the line also carries config 4 (bs1: 2048-token prompt seed 4, 512 greedy
steps) under "bs1". The reference arm (--impl reference) times the CPU oracle (a C++ restatement
of hobby-rs, which cannot be built here) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (bs1, bs256) 500M Q8_0 at 1/2/4/8 B200; HBM GB/s vs ~8 TB/s"
N_SEQS = 256
CTX = 16384
VALID = 50257


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-bs1", action="store_true", help="skip the config-4 bs1 sub-measurement")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--bs1-only", action="store_true", help="run only the config-4 bs1 measurement (one GPU)")
    ap.add_argument("--diffusion", action="store_true",
                    help="measure diffusion decode (Engine::generate_diffusion) instead of the headline (one GPU)")
    ap.add_argument("--seqs", type=int, default=N_SEQS, help=argparse.SUPPRESS)
    # profiling aid: shorter prompts (same batch) make the untimed prefill quick when only the
    # context-independent kernels are of interest; the headline always uses U[1024, 8192]
    ap.add_argument("--prompt-range", type=int, nargs=2, default=(1024, 8192), help=argparse.SUPPRESS)
    ap.add_argument("--ep", action="store_true",
                    help="expert parallelism under torchrun: the routed experts split across the ranks, "
                         "(token, expert) rows exchanged with NCCL inside each step (config 5's variant)")
    ap.add_argument("--prefill-case", action="store_true",
                    help="time the prefill alone: --seqs prompts of --lo ids each (500M, one GPU)")
    ap.add_argument("--attn-case", action="store_true",
                    help="time the decode-attention op alone on a config-3-shaped case (one GPU); "
                         "--seqs/--lo/--hi/--pages/--layers shape it")
    ap.add_argument("--lo", type=int, default=512, help=argparse.SUPPRESS)
    ap.add_argument("--hi", type=int, default=4096, help=argparse.SUPPRESS)
    ap.add_argument("--pages", choices=("random", "ordered"), default="random", help=argparse.SUPPRESS)
    ap.add_argument("--layers", type=int, default=0, help=argparse.SUPPRESS)
    return ap.parse_args()


def workload(n_seqs: int = N_SEQS, seed: int = 5, lo: int = 1024, hi: int = 8192):
    """Prompt lengths ~ U[lo, hi] (config 5: U[1024, 8192]) and ids ~ U[0, 50257) from
    torch.Generator(seed)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(lo, hi + 1, (n_seqs,), generator=g).tolist()
    prompts = [torch.randint(0, VALID, (n,), generator=g).numpy().astype("uint32") for n in lens]
    return prompts


def shard(lengths, rank: int, world: int) -> list[int]:
    """Sequence indices of `rank`: sequences sorted by prompt length (longest first, ties by index)
    are dealt in snake order (0..w-1, w-1..0, ...), so every rank holds n/world sequences with
    nearly the same total context, i.e. the same KV bytes per step. No collective on the decode path."""
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    mine = []
    for j, i in enumerate(order):
        blk, pos = divmod(j, world)
        if (pos if blk % 2 == 0 else world - 1 - pos) == rank:
            mine.append(i)
    return mine


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "200", "-i", str(device)], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        self.f.seek(0)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta

        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=timedelta(seconds=900))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def reduce_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reduce_sum(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def model_path(rank: int, world: int) -> str:
    from hobbylm_b200 import synth

    if rank == 0:
        p = synth.cached_model("500M", 0, context_length=CTX)
    barrier(world)
    if rank != 0:
        p = synth.cached_model("500M", 0, context_length=CTX)
    return p


def kv_bytes_per_pos(cfg) -> int:
    return cfg["n_layers"] * 2 * cfg["n_kv_heads"] * cfg["head_dim"] * 4


def weight_bytes_per_token(cfg) -> int:
    """Algorithmic weight bytes one bs1 token streams: int8 + f32 scale per 32 of every matrix a
    token touches (attention, dense layers, k routed + shared experts, lm_head) + the f32 router."""
    d, f, df, L, nd = cfg["d_model"], cfg["expert_ffn"], cfg["dense_ffn"], cfg["n_layers"], cfg["n_dense"]
    qd, kvd = cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"]
    k, nsh, ne, V = cfg["top_k"], cfg["n_shared"], cfg["n_experts"], cfg["vocab_size"]
    q8 = lambda r, c: r * c * 1.125  # int8 + one f32 scale per 32
    per_layer_attn = q8(qd + 2 * kvd, d) + q8(d, qd)
    dense = q8(2 * df, d) + q8(d, df)
    expert = q8(2 * f, d) + q8(d, f)
    moe = (k + nsh) * expert + ne * d * 4
    return int(L * per_layer_attn + nd * dense + (L - nd) * moe + q8(V, d))


def run_ours(args):
    import numpy as np
    import torch

    from hobbylm_b200 import Engine, synth

    rank, world, local = dist_setup(args)
    torch.cuda.set_device(local)
    path = model_path(rank, world)
    prompts_all = workload(args.seqs, lo=args.prompt_range[0], hi=args.prompt_range[1])
    mine = shard([len(p) for p in prompts_all], rank, world)
    prompts = [prompts_all[i] for i in mine]
    n_local = len(prompts)
    total_steps = args.warmup + 2 * args.steps + 2
    pool = sum(len(p) + total_steps + 32 for p in prompts)
    eng = Engine.load(path, device=local, max_batch=max(n_local, 1), kv_pool_tokens=pool)
    cfg = eng.cfg
    t0 = time.time()
    caches, toks = [], []
    for p in prompts:
        c = eng.new_cache()
        lg = eng.prefill(c, p)
        lg[VALID:] = -np.inf
        caches.append(c)
        toks.append(int(np.argmax(lg)))
    prefill_s = time.time() - t0
    if args.ep and world > 1:  # before the first decode step: the step graphs hold the exchanges
        from hobbylm_b200 import ep

        ep.setup(eng)
    stream = torch.cuda.ExternalStream(eng.stream(), device=local)
    # warm-up (captures the step graph)
    if args.warmup:
        out = eng.decode_greedy(caches, toks, args.warmup)
        toks = [int(v) for v in out[-1]]
    kernels_per_step = eng.decode_kernel_count(n_local)
    ctx_start = [c.len for c in caches]
    # ---- timed: K steps driven on the device (inputs resident in HBM) ----
    barrier(world)
    torch.cuda.synchronize()
    clocks = Clocks(local)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    out = eng.decode_greedy(caches, toks, args.steps, want_ids=True)
    ev1.record(stream)
    ev1.synchronize()
    clk = clocks.stop()
    torch.cuda.synchronize()
    barrier(world)
    dev_s = ev0.elapsed_time(ev1) / 1e3
    toks = [int(v) for v in out[-1]]
    max_s = reduce_max(dev_s, world)
    total_tokens = reduce_sum(n_local * args.steps, world)
    value = total_tokens / max_s
    # ---- e2e: the same steps through the per-step C-ABI call with host buffers ----
    barrier(world)
    torch.cuda.synchronize()
    w0 = time.perf_counter()
    for _ in range(args.steps):
        nxt, _ = eng.decode_batch(caches, toks)
        toks = [int(v) for v in nxt]
    torch.cuda.synchronize()
    e2e_s = reduce_max(time.perf_counter() - w0, world)
    # ---- attention roofline (the dominant kernels) on this step's state ----
    ms_s, ms_o = eng.time_attention(caches, iters=5)
    ctx_now = [c.len for c in caches]
    kvd = cfg["n_kv_heads"] * cfg["head_dim"]
    kv_bytes = sum(2 * n * kvd * 4 for n in ctx_now)  # K + V read by one layer's attention
    hbm, peak_kind = peaks()
    att_gbs = kv_bytes / ((ms_s + ms_o) / 1e3) / 1e9
    traffic = None
    tf = os.path.join(ROOT, "profiles", "attention_traffic.txt")
    if os.path.exists(tf):
        with open(tf) as f:
            bpp = [float(ln.split(":", 1)[1]) for ln in f if ln.startswith("bytes_per_position:")]
        # captured on a smaller case; DRAM bytes scale with the positions read
        if bpp:
            traffic = int(bpp[0] * sum(ctx_now))
    res = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(max_s / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8 dot / f32",
        "data": "synthetic (random-init seed-0 weights, random prompt ids)",
        "config": {"workload": f"config5: 500M Q8_0, {args.seqs} seqs, prompts U[{args.prompt_range[0]},"
                               f"{args.prompt_range[1]}] seed 5, greedy decode",
                   "global_batch": args.seqs, "seqs_per_gpu": n_local,
                   "parallelism": (f"seq-shard x{world} + experts split over {world} ranks (NCCL send/recv)"
                                   if args.ep and world > 1 else f"seq-shard x{world}"),
                   "context_at_start": {"min": int(reduce_min(min(ctx_start) if ctx_start else 0, world)),
                                        "mean": reduce_sum(sum(ctx_start), world) / max(total_tokens / args.steps, 1)},
                   "l2": "inputs larger than L2 (KV cache ~60 GB)", "prefill_s_rank0": round(prefill_s, 1)},
        "e2e": {"value": round(total_tokens / e2e_s, 1), "unit": "tok/s",
                "h2d_bytes_per_step": int(reduce_sum(n_local * 12, world)),
                "d2h_bytes_per_step": int(reduce_sum(n_local * 8 + 4, world))},
        "roofline": {"bound": "hbm", "kernel": "attention (k_qk_prep + k_attn_scores + k_attn_softmax + k_attn_pv), one layer",
                     "achieved": round(att_gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(att_gbs / hbm, 4), "peak_kind": peak_kind,
                     "traffic": traffic, "ms_scores": round(ms_s, 4), "ms_out": round(ms_o, 4),
                     "algorithmic_bytes": kv_bytes},
        "clocks": clk,
        "gpu_launches": int(reduce_sum(kernels_per_step * args.steps, world)),
    }
    if world == 1 and not args.no_bs1:
        res["bs1"] = run_bs1(eng_path=path, local=local)
    if world == 1 and not args.no_cpu and rank == 0:
        res["cpu_baseline"] = cpu_sample(path, prompts_all, steps=4, n_sample=2)
    for c in caches:
        c.close()
    eng.close()
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def reduce_min(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return float(t.item())


def run_bs1(eng_path: str, local: int, prompt_len: int = 2048, steps: int = 512) -> dict:
    """Config 4: 500M, bs1, 2048-token prompt (seed 4), 512 greedy steps (device-driven)."""
    import numpy as np
    import torch

    from hobbylm_b200 import Engine, synth

    eng = Engine.load(eng_path, device=local, max_batch=1, kv_pool_tokens=prompt_len + steps + 64)
    cfg = eng.cfg
    with eng.new_cache() as kv:
        lg = eng.prefill(kv, synth.prompt_ids(prompt_len, 4))
        lg[VALID:] = -np.inf
        tok = int(np.argmax(lg))
        out = eng.decode_greedy([kv], [tok], 8)
        tok = int(out[-1][0])
        n0 = kv.len
        stream = torch.cuda.ExternalStream(eng.stream(), device=local)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        eng.decode_greedy([kv], [tok], steps, want_ids=False)
        e1.record(stream)
        e1.synchronize()
        s = e0.elapsed_time(e1) / 1e3
        n1 = kv.len
    eng.close()
    mean_ctx = (n0 + n1) / 2
    bytes_tok = weight_bytes_per_token(cfg) + kv_bytes_per_pos(cfg) * (mean_ctx + 1)
    hbm, kind = peaks()
    gbs = bytes_tok * steps / s / 1e9
    return {"workload": "config4: 500M Q8_0 bs1, 2048-token prompt seed 4, 512 greedy steps",
            "tok_s": round(steps / s, 1), "us_per_token": round(s / steps * 1e6, 1),
            "algorithmic_bytes_per_token": int(bytes_tok), "achieved_gbs": round(gbs, 1),
            "roofline_frac": round(gbs / hbm, 4), "peak_kind": kind}


def cpu_sample(path: str, prompts_all, steps: int = 4, n_sample: int = 2) -> dict:
    """The CPU oracle (hobby-rs restated, OpenMP over output rows like rayon) decoding `steps`
    tokens for `n_sample` sequences of the workload. Their prompt K/V are synthetic (random) rows:
    the decode cost depends only on the context length, and a CPU prefill of these prompts would
    take minutes."""
    import numpy as np

    import oracle

    ora = oracle.Engine(path, quant=True)
    kvd = ora.cfg["n_kv_heads"] * ora.cfg["head_dim"]
    rng = np.random.default_rng(0)
    tot_s, tot_tok, ctxs = 0.0, 0, []
    for p in prompts_all[:n_sample]:
        c = ora.new_cache()
        n = len(p)
        c.fill(rng.standard_normal((n, kvd)).astype(np.float32), rng.standard_normal((n, kvd)).astype(np.float32))
        tok = int(p[-1])
        for i in range(steps):
            t = time.perf_counter()
            lg = ora.forward(c, tok, n + i)
            tot_s += time.perf_counter() - t
            tot_tok += 1
            lg[VALID:] = -np.inf
            tok = int(np.argmax(lg))
        ctxs.append(n)
        c.close()
    ora.close()
    return {"value": round(tot_tok / tot_s, 2), "unit": "tok/s", "cores": oracle.num_threads(), "kind": "port",
            "sample": f"{n_sample} sequences x {steps} decode tokens at contexts {ctxs} (synthetic prompt KV), "
                      f"500M Q8_0, sequential like hobby-rs"}


DIFF_PROMPT = 64


def diffusion_cpu_sample(path: str, prompt) -> tuple[dict, list]:
    """The oracle's generate_diffusion on one block: 32 ids, 8 denoising passes (the per-block
    schedule of the defaults, round(32 * 32 / 128) = 8) after the bidirectional prompt encode."""
    import oracle

    ora = oracle.Engine(path, quant=True)
    t = time.perf_counter()
    ids = ora.generate_diffusion(prompt, gen_len=32, block=32, steps=8)
    s = time.perf_counter() - t
    ora.close()
    return ({"value": round(len(ids) / s, 2), "unit": "tok/s", "cores": oracle.num_threads(), "kind": "port",
             "sample": f"one 32-id block (8 passes + finalize) after a {len(prompt)}-id prompt encode, 500M Q8_0"},
            [int(i) for i in ids])


def run_diffusion(args):
    """Diffusion decode on one GPU: Engine::generate_diffusion (lib.rs:211-495) with DiffOpts
    defaults (gen_len 128, block 32, 32 steps, greedy, presence penalty 1.4, prefix-cached) after a
    64-id prompt, wall clock per call (the block scoring runs on the host between GPU passes)."""
    import torch

    from hobbylm_b200 import DiffOpts, Engine, synth

    path = synth.cached_model("500M", 0, context_length=CTX)
    prompt = synth.prompt_ids(DIFF_PROMPT, 6)
    eng = Engine.load(path, device=0, max_batch=1, kv_pool_tokens=4096)
    first = eng.generate_diffusion(prompt, DiffOpts(gen_len=32, block=32, steps=8))
    for _ in range(args.warmup):
        eng.generate_diffusion(prompt, DiffOpts())
    res = {}
    for name, o in (("cached", DiffOpts()), ("uncached", DiffOpts(cached=False))):
        times, n = [], 0
        for _ in range(args.steps):
            torch.cuda.synchronize()
            t = time.perf_counter()
            n = len(eng.generate_diffusion(prompt, o))
            times.append(time.perf_counter() - t)
        res[name] = (n, statistics.median(times))
    # one denoising pass of the cached path: a 32-row block after the prompt, logits to the host
    with eng.new_cache() as kv:
        eng.run_block(kv, prompt, n_logits=0, commit=True)
        blk = [eng.cfg["mask_token_id"]] * 32
        for _ in range(3):
            eng.run_block(kv, blk)
        t = time.perf_counter()
        for _ in range(20):
            eng.run_block(kv, blk)
        pass_ms = (time.perf_counter() - t) / 20 * 1e3
    eng.close()
    cpu = None if args.no_cpu else diffusion_cpu_sample(path, prompt)
    n, s = res["cached"]
    line = {"metric": "diffusion decode tok/s (500M Q8_0, DiffOpts defaults, prefix-cached)", "value": round(n / s, 1),
            "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(s * 1e3, 2), "higher_is_better": True, "scaling": "replicas only",
            "vs_baseline": None, "dtype": "int8 dot / f32", "data": "synthetic",
            "config": {"workload": f"500M Q8_0 seed 0, {DIFF_PROMPT}-id prompt (seed 6), gen_len 128, block 32, "
                                   "32 steps, temp 0, rep_penalty 1.4; a step = one generate_diffusion call"},
            "generated": n, "pass_ms_32_rows": round(pass_ms, 3),
            "uncached": {"value": round(res["uncached"][0] / res["uncached"][1], 1), "unit": "tok/s",
                         "ms_per_call": round(res["uncached"][1] * 1e3, 2)}}
    if cpu is not None:
        line["cpu_baseline"] = cpu[0]
        line["first_block_equals_oracle"] = cpu[1] == first
    print(json.dumps(line), flush=True)


def run_reference(args):
    """The reference arm: the CPU oracle on the host cores, rank 0 only."""
    rank, world, local = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), 0
    if rank != 0:
        return
    import numpy as np

    import oracle
    from hobbylm_b200 import synth

    path = synth.cached_model("500M", 0, context_length=CTX)
    prompts_all = workload(args.seqs)
    ora = oracle.Engine(path, quant=True)
    kvd = ora.cfg["n_kv_heads"] * ora.cfg["head_dim"]
    rng = np.random.default_rng(0)
    sample = prompts_all[:2]
    caches, toks = [], []
    for p in sample:
        c = ora.new_cache()
        n = len(p)
        c.fill(rng.standard_normal((n, kvd)).astype(np.float32), rng.standard_normal((n, kvd)).astype(np.float32))
        caches.append(c)
        toks.append(int(p[-1]))

    def step():
        for i, c in enumerate(caches):
            lg = ora.forward(c, toks[i], len(c))
            lg[VALID:] = -np.inf
            toks[i] = int(np.argmax(lg))

    for _ in range(args.warmup):
        step()
    t = time.perf_counter()
    for _ in range(args.steps):
        step()
    s = time.perf_counter() - t
    v = len(sample) * args.steps / s
    res = {"metric": METRIC, "value": round(v, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(s / args.steps * 1e3, 2), "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": "int8 dot / f32", "impl": "reference",
           "data": "synthetic", "config": {"workload": "config5 sample: the first 2 of the 256 sequences",
                                          "global_batch": args.seqs},
           "cpu_baseline": {"value": round(v, 2), "unit": "tok/s", "cores": oracle.num_threads(), "kind": "port",
                            "sample": f"2 sequences (contexts {[len(p) for p in sample]}, synthetic prompt KV) "
                                      f"x {args.steps} steps; hobby-rs serves sequences one after another"},
           "e2e": {"value": round(v, 2), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(res), flush=True)


def run_attn_case(args):
    """The decode-attention op alone (hg_op_kv_attn: QK-norm + RoPE + KV append, scores, softmax,
    value sums) on a config-3-shaped case, for timing and profiling the attention kernels: --seqs
    sequences with contexts U[--lo, --hi] (seed 3), the 500M head shapes (12 q / 3 kv heads,
    head_dim 128), 16-position pages placed by a random permutation (--pages ordered: consecutive
    pages), K/V/q ~ N(0,1), QK-norm gains 1, RoPE base 1e4. --layers L lays the pool out as the
    engine does for an L-layer model (one page holds K and V of every layer; layer 0 is read).
    Each step is one call; inputs are created on the device and outputs are not checked here (the
    parity tests compare this entry point with the oracle)."""
    import ctypes as C

    import numpy as np
    import torch

    from hobbylm_b200 import _native as native

    nh, nkv, hd, eps, theta = 12, 3, 128, 1e-5, 10000.0
    rng = np.random.default_rng(3)
    ctx = rng.integers(args.lo, args.hi + 1, args.seqs)
    max_pos = int(ctx.max()) + args.steps + 1
    bt_stride = (max_pos + 15) // 16
    n_pages = args.seqs * bt_stride
    perm = rng.permutation(n_pages).astype(np.int32).reshape(args.seqs, bt_stride)
    if args.pages == "ordered":
        perm = np.arange(n_pages, dtype=np.int32).reshape(args.seqs, bt_stride)
    page_floats = nkv * 16 * hd
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(3)
    page_stride = page_floats
    if args.layers > 0:  # [page][layer][K | V]
        pool = torch.zeros((n_pages, args.layers, 2, page_floats), device=dev)
        pool[:, 0].normal_(generator=g)
        k_pool, v_pool = pool[:, 0, 0], pool[:, 0, 1]
        page_stride = args.layers * 2 * page_floats
    else:
        k_pool = torch.randn((n_pages, page_floats), generator=g, device=dev)
        v_pool = torch.randn((n_pages, page_floats), generator=g, device=dev)
    cos = torch.empty((max_pos, hd // 2), dtype=torch.float32)
    sin = torch.empty_like(cos)
    native.check(native.lib().hg_rope_tables(hd, max_pos, theta, cos.data_ptr(), sin.data_ptr()))
    d_cos, d_sin = cos.to(dev), sin.to(dev)
    ones = torch.ones(hd, device=dev)
    d_bt = torch.from_numpy(perm).to(dev)
    pos = torch.from_numpy(ctx.astype(np.int32)).to(dev)
    qkv = torch.randn((args.seqs, (nh + 2 * nkv) * hd), generator=g, device=dev)
    out = torch.empty((args.seqs, nh * hd), device=dev)
    a = native.KvAttnArgs()
    a.n_seqs, a.n_heads, a.n_kv_heads, a.head_dim, a.max_pos, a.eps = args.seqs, nh, nkv, hd, max_pos, eps
    a.qkv, a.q_norm, a.k_norm = qkv.data_ptr(), ones.data_ptr(), ones.data_ptr()
    a.rope_cos, a.rope_sin, a.pos, a.block_table = d_cos.data_ptr(), d_sin.data_ptr(), pos.data_ptr(), d_bt.data_ptr()
    a.bt_stride, a.k_pool, a.v_pool, a.page_stride, a.out = (
        bt_stride, k_pool.data_ptr(), v_pool.data_ptr(), page_stride, out.data_ptr())
    scratch = torch.empty(native.lib().hg_op_kv_attn_scratch_bytes(C.byref(a)), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    times = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        native.check(native.lib().hg_op_kv_attn(C.byref(a), scratch.data_ptr(), C.c_void_p(stream.cuda_stream)))
        e1.record(stream)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
        pos += 1
    kv_bytes = 2 * nkv * hd * 4 * (int(ctx.sum()) + args.seqs * args.steps)  # K + V rows read per call (upper)
    best = min(times[1:] if len(times) > 1 else times)
    print(json.dumps({"attn_case": True, "seqs": args.seqs, "pages": args.pages, "layers": args.layers,
                      "contexts": [int(ctx.min()), int(ctx.mean()), int(ctx.max())],
                      "ms_per_call": round(best, 4), "kv_gb_per_s": round(kv_bytes / (best / 1e3) / 1e9, 1)}))


def run_prefill_case(args):
    """Model::prefill alone (the exact-order prefill kernels) on the 500M model: --seqs prompts of
    --lo random ids each (seed 100 + i), one at a time, wall clock per prompt after a first prompt
    that loads the kernels."""
    import numpy as np

    from hobbylm_b200 import Engine, synth

    n, length = max(1, args.seqs), max(1, args.lo)
    eng = Engine.load(synth.cached_model("500M", 0, context_length=CTX), device=0, max_batch=1,
                      kv_pool_tokens=(n + 1) * (length + 64))
    times = []
    for i in range(n + 1):
        c = eng.new_cache()
        t0 = time.time()
        lg = eng.prefill(c, synth.prompt_ids(length, 100 + i))
        dt = time.time() - t0
        if i > 0:
            times.append(round(dt, 4))
        assert np.isfinite(lg).all()
        c.close()
    eng.close()
    print(json.dumps({"prefill_case": True, "prompts": n, "tokens": length, "s_per_prompt": times,
                      "tok_s": round(length * n / sum(times), 1)}), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.diffusion:
        run_diffusion(args)
    elif args.attn_case:
        run_attn_case(args)
    elif args.prefill_case:
        run_prefill_case(args)
    elif args.bs1_only:
        from hobbylm_b200 import synth

        print(json.dumps(run_bs1(synth.cached_model("500M", 0, context_length=CTX), 0)), flush=True)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
