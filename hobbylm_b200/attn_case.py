"""A config-3-shaped decode-attention case on the GPU, for timing and profiling the attention
kernels alone: n sequences with contexts U[lo, hi] (seed 3), the 500M head shapes (12 q / 3 kv
heads, head_dim 128), 16-position pages placed by a random permutation, K/V/q ~ N(0,1), QK-norm
gains 1, RoPE base 1e4. Each step is one hg_op_kv_attn call (append + attention for every
sequence). Inputs are created on the device; outputs are not checked here (the parity tests
compare this entry point with the oracle).

    python -m hobbylm_b200.attn_case [--seqs 64] [--lo 512] [--hi 4096] [--steps 5] [--pages random|ordered]

--pages ordered gives each sequence consecutive pages of the pool instead of the permutation.
--layers L lays the pool out as the engine does for an L-layer model (one page holds K and V of
every layer; this case reads layer 0), instead of separate dense K and V pools.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json

import numpy as np


def main() -> None:
    import torch

    from hobbylm_b200 import _native as native

    ap = argparse.ArgumentParser()
    ap.add_argument("--seqs", type=int, default=64)
    ap.add_argument("--lo", type=int, default=512)
    ap.add_argument("--hi", type=int, default=4096)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--pages", choices=("random", "ordered"), default="random")
    ap.add_argument("--layers", type=int, default=0)
    a = ap.parse_args()
    nh, nkv, hd, eps, theta = 12, 3, 128, 1e-5, 10000.0
    rng = np.random.default_rng(3)
    ctx = rng.integers(a.lo, a.hi + 1, a.seqs)
    max_pos = int(ctx.max()) + a.steps + 1
    bt_stride = (max_pos + 15) // 16
    n_pages = a.seqs * bt_stride
    perm = rng.permutation(n_pages).astype(np.int32).reshape(a.seqs, bt_stride)
    if a.pages == "ordered":
        perm = np.arange(n_pages, dtype=np.int32).reshape(a.seqs, bt_stride)
    page_floats = nkv * 16 * hd
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(3)
    page_stride = page_floats
    if a.layers > 0:  # [page][layer][K | V]
        pool = torch.zeros((n_pages, a.layers, 2, page_floats), device=dev)
        pool[:, 0].normal_(generator=g)
        k_pool, v_pool = pool[:, 0, 0], pool[:, 0, 1]
        page_stride = a.layers * 2 * page_floats
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
    qkv = torch.randn((a.seqs, (nh + 2 * nkv) * hd), generator=g, device=dev)
    out = torch.empty((a.seqs, nh * hd), device=dev)
    args = native.KvAttnArgs()
    args.n_seqs, args.n_heads, args.n_kv_heads, args.head_dim, args.max_pos, args.eps = a.seqs, nh, nkv, hd, max_pos, eps
    args.qkv, args.q_norm, args.k_norm = qkv.data_ptr(), ones.data_ptr(), ones.data_ptr()
    args.rope_cos, args.rope_sin, args.pos, args.block_table = d_cos.data_ptr(), d_sin.data_ptr(), pos.data_ptr(), d_bt.data_ptr()
    args.bt_stride, args.k_pool, args.v_pool, args.page_stride, args.out = (
        bt_stride, k_pool.data_ptr(), v_pool.data_ptr(), page_stride, out.data_ptr())
    scratch = torch.empty(native.lib().hg_op_kv_attn_scratch_bytes(C.byref(args)), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    times = []
    for _ in range(a.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        native.check(native.lib().hg_op_kv_attn(C.byref(args), scratch.data_ptr(), C.c_void_p(stream.cuda_stream)))
        e1.record(stream)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
        pos += 1
    kv_bytes = 2 * nkv * hd * 4 * (int(ctx.sum()) + a.seqs * a.steps)  # K + V rows read per call (upper)
    best = min(times[1:] if len(times) > 1 else times)
    print(json.dumps({"seqs": a.seqs, "pages": a.pages, "layers": a.layers, "contexts": [int(ctx.min()), int(ctx.mean()), int(ctx.max())],
                      "ms_per_call": round(best, 4), "kv_gb_per_s": round(kv_bytes / (best / 1e3) / 1e9, 1)}))


if __name__ == "__main__":
    main()
