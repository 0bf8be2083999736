"""Kernel-level parity through the C ABI (device pointers) against the CPU oracle.

Q8 matvec / matmul, the MoE layer and KV append + decode attention must be bit-exact with the
oracle's restatement of hobby-rs (quant.rs, model.rs).
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# (rows, cols) of every matrix shape of the two presets (quant.rs matvec inputs)
SHAPES = [(2304, 768), (768, 1536), (320, 768), (768, 320), (2304, 768), (768, 2304), (512, 512), (192, 512),
          (512, 192), (1536, 512), (512, 1536), (96, 4128)]


def _dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _pack(native, w):
    rows, cols = w.shape
    ss = native.lib().hg_q8_scale_stride(cols)
    qs = np.empty((rows, cols), np.int8)
    sc = np.empty((rows, ss), np.float32)
    native.check(native.lib().hg_q8_pack(w.ctypes.data, rows, cols, qs.ctypes.data, sc.ctypes.data))
    return qs, sc


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("rows,cols", SHAPES)
@pytest.mark.parametrize("ntok", [1, 3, 17, 40, 256])
def test_q8_matvec_bitexact(native, oracle_mod, rows, cols, ntok):
    """Decode matvec order (quant.rs:44-67) for one to 256 tokens. From 32 tokens on, rows whose
    width is a multiple of 128 take the tensor-core kernel (exact int32 lane partials from
    tcgen05.mma kind::i8, f32 chains on the CUDA cores); the others and smaller steps take dp4a."""
    import torch

    rng = np.random.default_rng(rows * 7 + cols + ntok)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    x = rng.standard_normal((ntok, cols)).astype(np.float32)
    qs, sc = _pack(native, w)
    oq, osc = oracle_mod.q8_quantize(w)
    dq, ds, dx = _dev(qs), _dev(sc), _dev(x)
    dy = torch.empty((ntok, rows), dtype=torch.float32, device="cuda")
    native.check(native.lib().hg_op_q8_matvec(dq.data_ptr(), ds.data_ptr(), rows, cols, dx.data_ptr(), dy.data_ptr(),
                                              ntok, None))
    torch.cuda.synchronize()
    y = dy.cpu().numpy()
    for t in range(ntok):
        ref = oracle_mod.q8_matvec(oq, osc, x[t])
        assert np.array_equal(_bits(y[t]), _bits(ref)), f"token {t}: max |d| {np.abs(y[t] - ref).max()}"


@pytest.mark.parametrize("rows,cols", [(2304, 768), (320, 768), (768, 320), (768, 2304), (512, 192)])
@pytest.mark.parametrize("ntok", [1, 37, 130])
def test_q8_matmul_bitexact(native, oracle_mod, rows, cols, ntok):
    import torch

    rng = np.random.default_rng(rows + cols * 3 + ntok)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    x = rng.standard_normal((ntok, cols)).astype(np.float32)
    qs, sc = _pack(native, w)
    oq, osc = oracle_mod.q8_quantize(w)
    dq, ds, dx = _dev(qs), _dev(sc), _dev(x)
    dy = torch.empty((ntok, rows), dtype=torch.float32, device="cuda")
    native.check(native.lib().hg_op_q8_matmul(dq.data_ptr(), ds.data_ptr(), rows, cols, dx.data_ptr(), dy.data_ptr(),
                                              ntok, None))
    torch.cuda.synchronize()
    ref = oracle_mod.q8_matmul(oq, osc, x)
    assert np.array_equal(_bits(dy.cpu().numpy()), _bits(ref))


def _moe_weights(native, inp, k, n_shared):
    ne, f, d = inp["gate_exps"].shape
    keep = {}

    def pk(name, arr3):
        cnt, r, c = arr3.shape
        qs, sc = _pack(native, arr3.reshape(cnt * r, c))
        keep[name + "_qs"], keep[name + "_sc"] = _dev(qs), _dev(sc)

    pk("gate", inp["gate_exps"])
    pk("up", inp["up_exps"])
    pk("down", inp["down_exps"])
    if n_shared:
        pk("sh_gate", inp["gate_sh"][None])
        pk("sh_up", inp["up_sh"][None])
        pk("sh_down", inp["down_sh"][None])
    keep["router"], keep["bias"] = _dev(inp["router"]), _dev(inp["bias"])
    w = native.MoeWeights()
    w.d_model, w.expert_ffn, w.n_experts, w.top_k, w.n_shared = d, f, ne, k, n_shared
    w.gating_sigmoid, w.weights_norm, w.weights_scale = 1, 0, 1.0
    for name, t in keep.items():
        setattr(w, name, t.data_ptr())
    return w, keep


@pytest.fixture(scope="module")
def moe_inputs():
    from hobbylm_b200 import synth

    return synth.moe_op_inputs(seed=2, T=256)


@pytest.mark.parametrize("T", [1, 8, 64, 256])
def test_moe_op_config2_bitexact(native, oracle_mod, moe_inputs, T):
    """Config 2: 500M MoE dims, Q8_0 experts with int8 ~ U[-127,127] and |N(0,0.01)| fp16 scales
    (re-quantized as Model::load does), router N(0,0.02), bias N(0,0.1), x ~ N(0,1)."""
    import torch

    inp = moe_inputs
    k = 6
    w, keep = _moe_weights(native, inp, k, 1)
    x = np.ascontiguousarray(inp["x"][:T])
    dx = _dev(x)
    dy = torch.empty((T, x.shape[1]), dtype=torch.float32, device="cuda")
    dsel = torch.empty((T, k), dtype=torch.int32, device="cuda")
    nbytes = native.lib().hg_op_moe_scratch_bytes(C.byref(w), T)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    native.check(native.lib().hg_op_moe_ffn(C.byref(w), dx.data_ptr(), T, dy.data_ptr(), dsel.data_ptr(),
                                            scratch.data_ptr(), None))
    torch.cuda.synchronize()
    moe = oracle_mod.Moe(inp["router"], inp["bias"], inp["gate_exps"], inp["up_exps"], inp["down_exps"],
                         inp["gate_sh"], inp["up_sh"], inp["down_sh"], top_k=k)
    y_ref, sel_ref, _ = moe.run(x, mode=0)
    assert np.array_equal(dsel.cpu().numpy(), sel_ref), "expert selection differs"
    y = dy.cpu().numpy()
    assert np.array_equal(_bits(y), _bits(y_ref)), f"max |d| {np.abs(y - y_ref).max()}"


def _oracle_attn_steps(oracle_mod, rope, caches, qkv, pos, nh, nkv, hd, eps, ones):
    """One oracle attention step (append + attend) per sequence, sequences in parallel threads
    (the oracle call is single-threaded, stateless and releases the GIL)."""
    from concurrent.futures import ThreadPoolExecutor

    def one(s):
        kc, vc = caches[s]
        return oracle_mod.attn_step(rope, nh, nkv, hd, eps, ones, ones, qkv[s].copy(), int(pos[s]), kc, vc)

    with ThreadPoolExecutor(max_workers=16) as ex:
        return list(ex.map(one, range(len(caches))))


@pytest.mark.parametrize("n_seqs,steps", [(64, 256), (72, 24)])
def test_kv_attn_config3(native, oracle_mod, n_seqs, steps):
    """Config 3: 64 sequences, ctx ~ U[512, 4096] (seed 3), 500M head shapes, K/V/Q ~ N(0,1),
    QK-norm gains 1, RoPE base 1e4, 16-token pages placed by a random permutation, one appended
    and attended token per sequence per step for all 256 steps. Every sequence's output is
    bit-compared with the oracle at every step, and at the end every appended K and V row of every
    sequence. 72 sequences (216 (sequence, kv head) pairs) take the large-batch kernel path."""
    import torch

    nh, nkv, hd, eps, theta = 12, 3, 128, 1e-5, 10000.0
    rng = np.random.default_rng(3)
    ctx = rng.integers(512, 4097, n_seqs)
    max_pos = int(ctx.max()) + steps + 1
    bt_stride = (max_pos + 15) // 16
    n_pages = n_seqs * bt_stride
    perm = rng.permutation(n_pages).astype(np.int32).reshape(n_seqs, bt_stride)
    kvd = nkv * hd
    page_floats = nkv * 16 * hd
    k_pool = np.zeros((n_pages, nkv, 16, hd), np.float32)
    v_pool = np.zeros((n_pages, nkv, 16, hd), np.float32)
    caches = []
    for s in range(n_seqs):
        kc = np.zeros((max_pos, kvd), np.float32)
        vc = np.zeros((max_pos, kvd), np.float32)
        n = int(ctx[s])
        kc[:n] = rng.standard_normal((n, kvd)).astype(np.float32)
        vc[:n] = rng.standard_normal((n, kvd)).astype(np.float32)
        p = np.arange(n)
        k_pool[perm[s, p // 16], :, p % 16] = kc[:n].reshape(n, nkv, hd)
        v_pool[perm[s, p // 16], :, p % 16] = vc[:n].reshape(n, nkv, hd)
        caches.append((kc, vc))
    rope = oracle_mod.Rope(hd, max_pos, theta)
    cos, sin = rope.tables()
    ones = np.ones(hd, np.float32)
    d_k, d_v = _dev(k_pool.reshape(n_pages, page_floats)), _dev(v_pool.reshape(n_pages, page_floats))
    d_bt, d_cos, d_sin, d_g = _dev(perm), _dev(cos), _dev(sin), _dev(ones)
    pos = ctx.astype(np.int32).copy()
    a = native.KvAttnArgs()
    a.n_seqs, a.n_heads, a.n_kv_heads, a.head_dim, a.max_pos, a.eps = n_seqs, nh, nkv, hd, max_pos, eps
    a.q_norm, a.k_norm = d_g.data_ptr(), d_g.data_ptr()
    a.rope_cos, a.rope_sin, a.block_table = d_cos.data_ptr(), d_sin.data_ptr(), d_bt.data_ptr()
    a.bt_stride, a.k_pool, a.v_pool, a.page_stride = bt_stride, d_k.data_ptr(), d_v.data_ptr(), page_floats
    scratch = torch.empty(native.lib().hg_op_kv_attn_scratch_bytes(C.byref(a)), dtype=torch.uint8, device="cuda")
    worst = 0.0
    for step in range(steps):
        qkv = rng.standard_normal((n_seqs, (nh + 2 * nkv) * hd)).astype(np.float32)
        d_qkv, d_pos = _dev(qkv), _dev(pos)
        d_out = torch.empty((n_seqs, nh * hd), dtype=torch.float32, device="cuda")
        a.qkv, a.pos, a.out = d_qkv.data_ptr(), d_pos.data_ptr(), d_out.data_ptr()
        native.check(native.lib().hg_op_kv_attn(C.byref(a), scratch.data_ptr(), None))
        refs = _oracle_attn_steps(oracle_mod, rope, caches, qkv, pos, nh, nkv, hd, eps, ones)
        out = d_out.cpu().numpy()
        for s in range(n_seqs):
            ref = refs[s]
            rel = np.linalg.norm(out[s] - ref) / np.linalg.norm(ref)
            worst = max(worst, rel)
            assert np.array_equal(_bits(out[s]), _bits(ref)), f"step {step} seq {s}: rel L2 {rel}"
        pos += 1
    # every appended K (QK-normed + roped) and V row of every sequence equals the oracle's cache row
    kp = d_k.cpu().numpy().reshape(n_pages, nkv, 16, hd)
    vp = d_v.cpu().numpy().reshape(n_pages, nkv, 16, hd)
    for s in range(n_seqs):
        kc, vc = caches[s]
        p = np.arange(int(ctx[s]), int(pos[s]))
        got_k = kp[perm[s, p // 16], :, p % 16].reshape(len(p), kvd)
        got_v = vp[perm[s, p // 16], :, p % 16].reshape(len(p), kvd)
        assert np.array_equal(_bits(got_k), _bits(kc[p])), f"seq {s}: appended K rows differ"
        assert np.array_equal(_bits(got_v), _bits(vc[p])), f"seq {s}: appended V rows differ"
