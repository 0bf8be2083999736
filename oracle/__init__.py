"""TEST INFRASTRUCTURE ONLY — ctypes binding of the CPU oracle (oracle/hobby_oracle.cpp).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs import this
package, as the checker or the timed CPU baseline. The product (hobbylm_b200) never imports it.

The oracle restates hobby-rs (harishsg993010/HobbyLM, hobby-rs/src/{gguf,config,quant,ops,model,
lib,sample}.rs); see the header of hobby_oracle.cpp for the per-function citations and arithmetic
pins. Parity pins: the synthetic-model producer is pinned bit-exactly to the reference's own
PyTorch init + exporter (tests/golden/synth_digests_*.json) and the oracle's F32 mode is pinned to
the reference's PyTorch forward: causal (tests/golden/torch_logits_130M.npz), on caller rows
(torch_embeds_logits_130M.npz) and bidirectional (torch_bidir_logits_130M.npz), and its greedy
uncached diffusion loop to the reference's own sampler (torch_diffusion_generate_130M.json). The
Q8 path has no reference
output to pin against (hobby-rs cannot be built here and has no tests or fixtures for this path):
its Q8 arithmetic is a restatement of quant.rs and is therefore "parity unpinned" for Q8.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "hobby_oracle.cpp")
LIB = os.path.join(HERE, "_build", "libhobby_oracle.so")
CXXFLAGS = ["-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared", "-std=c++17"]


def build(force: bool = False) -> str:
    """Compile the oracle (g++) unless an up-to-date library exists."""
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    tmp = LIB + f".tmp{os.getpid()}"
    subprocess.check_call(["g++", *CXXFLAGS, SRC, "-o", tmp])
    os.replace(tmp, LIB)
    return LIB


_lib = None

f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


def lib():
    global _lib
    if _lib is not None:
        return _lib
    L = C.CDLL(build())
    vp, i, f, d = C.c_void_p, C.c_int, C.c_float, C.c_double
    sig = {
        "hor_last_error": (C.c_char_p, []),
        "hor_set_exp_mode": (None, [i]),
        "hor_num_threads": (i, []),
        "hor_set_num_threads": (None, [i]),
        "hor_engine_load": (i, [C.c_char_p, i, C.POINTER(vp)]),
        "hor_engine_free": (None, [vp]),
        "hor_engine_config": (i, [vp, i32p, f32p]),
        "hor_engine_weight_bytes": (C.c_uint64, [vp]),
        "hor_cache_new": (i, [vp, C.POINTER(vp)]),
        "hor_cache_free": (None, [vp]),
        "hor_cache_len": (i, [vp]),
        "hor_cache_read": (i, [vp, i, f32p, f32p]),
        "hor_cache_fill": (i, [vp, vp, f32p, f32p, i]),
        "hor_prefill": (i, [vp, vp, u32p, i, f32p]),
        "hor_prefill_embeds": (i, [vp, vp, f32p, i, f32p]),
        "hor_forward_x": (i, [vp, vp, f32p, i, f32p]),
        "hor_run_block": (i, [vp, vp, u32p, i, i, vp]),
        "hor_sample": (i, [f32p, i, f, f, C.POINTER(C.c_uint64), C.POINTER(C.c_uint32)]),
        "hor_score_block": (i, [f32p, i, u32p, i, vp, i, C.c_uint32, f, f, C.POINTER(C.c_uint64), u32p, f32p, f32p]),
        "hor_forward_bidir": (i, [vp, u32p, i, f32p]),
        "hor_generate_embeds": (i, [vp, f32p, i, vp, i, i, f, f, C.c_uint64, f, u32p, C.POINTER(i)]),
        "hor_generate_diffusion": (i, [vp, u32p, i, i, i, i, f, f, i, f, C.c_uint64, i, f, u32p, C.POINTER(i)]),
        "hor_forward": (i, [vp, vp, C.c_uint32, i, f32p]),
        "hor_last_routing": (i, [vp, i32p, f32p]),
        "hor_generate": (i, [vp, u32p, i, i, f, f, C.c_uint64, f, u32p, vp, C.POINTER(i), C.POINTER(d),
                             C.POINTER(d)]),
        "hor_q8_quantize": (i, [f32p, i, i, i8p, f32p]),
        "hor_q8_quant_act": (i, [f32p, i, i8p, f32p]),
        "hor_q8_matvec": (i, [i8p, f32p, i, i, f32p, f32p]),
        "hor_q8_matmul": (i, [i8p, f32p, i, i, f32p, f32p, i]),
        "hor_dequant": (i, [i, u8p, C.c_size_t, f32p]),
        "hor_dot": (f, [f32p, f32p, i]),
        "hor_rmsnorm": (None, [f32p, f32p, f, f32p, i]),
        "hor_expf": (f, [f]),
        "hor_sigmoid": (f, [f]),
        "hor_silu": (f, [f]),
        "hor_moe_create": (i, [i, i, i, i, i, i, i, f, f32p, f32p, f32p, f32p, f32p, vp, vp, vp, C.POINTER(vp)]),
        "hor_moe_free": (None, [vp]),
        "hor_moe_run": (i, [vp, f32p, i, i, f32p, vp, vp]),
        "hor_moe_sel_scores": (i, [vp, f32p, f32p]),
        "hor_moe_expert": (i, [vp, f32p, i, f32p]),
        "hor_rope_create": (i, [i, i, f, C.POINTER(vp)]),
        "hor_rope_free": (None, [vp]),
        "hor_rope_tables": (i, [vp, f32p, f32p]),
        "hor_attn_step": (i, [vp, i, i, i, f, f32p, f32p, f32p, i, f32p, f32p, f32p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


class OracleError(RuntimeError):
    pass


def _check(rc: int) -> None:
    if rc != 0:
        raise OracleError(lib().hor_last_error().decode())


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


CONFIG_INTS = ("d_model", "n_layers", "n_dense", "n_heads", "n_kv_heads", "head_dim", "dense_ffn", "expert_ffn",
               "n_experts", "top_k", "n_shared", "vocab_size", "context_length", "expert_weights_norm",
               "gating_sigmoid", "eos", "diffusion", "mask_token_id", "block_size")
CONFIG_FLOATS = ("rms_eps", "rope_theta", "expert_weights_scale")


def set_exp_mode(libm: bool) -> None:
    lib().hor_set_exp_mode(1 if libm else 0)


def num_threads() -> int:
    return lib().hor_num_threads()


class Engine:
    """hobby-rs ``Engine`` restated (lib.rs:78-162) over token ids."""

    def __init__(self, path: str, quant: bool = True):
        h = C.c_void_p()
        _check(lib().hor_engine_load(path.encode(), 1 if quant else 0, C.byref(h)))
        self.h = h
        ints = np.zeros(len(CONFIG_INTS), np.int32)
        fl = np.zeros(3, np.float32)
        _check(lib().hor_engine_config(self.h, ints, fl))
        self.cfg = {k: int(v) for k, v in zip(CONFIG_INTS, ints)}
        self.cfg.update({k: float(v) for k, v in zip(CONFIG_FLOATS, fl)})

    def close(self):
        if self.h:
            lib().hor_engine_free(self.h)
            self.h = None

    __del__ = close

    @property
    def vocab(self) -> int:
        return self.cfg["vocab_size"]

    def weight_bytes(self) -> int:
        return int(lib().hor_engine_weight_bytes(self.h))

    def new_cache(self) -> "Cache":
        return Cache(self)

    def prefill(self, cache: "Cache", ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.zeros(self.vocab, np.float32)
        _check(lib().hor_prefill(self.h, cache.h, ids, len(ids), out))
        return out

    def prefill_embeds(self, cache: "Cache", rows) -> np.ndarray:
        rows = np.ascontiguousarray(rows, dtype=np.float32)
        out = np.zeros(self.vocab, np.float32)
        _check(lib().hor_prefill_embeds(self.h, cache.h, rows, rows.shape[0], out))
        return out

    def forward_x(self, cache: "Cache", row, pos: int) -> np.ndarray:
        row = np.ascontiguousarray(row, dtype=np.float32)
        out = np.zeros(self.vocab, np.float32)
        _check(lib().hor_forward_x(self.h, cache.h, row, int(pos), out))
        return out

    def forward(self, cache: "Cache", token: int, pos: int) -> np.ndarray:
        out = np.zeros(self.vocab, np.float32)
        _check(lib().hor_forward(self.h, cache.h, int(token), int(pos), out))
        return out

    def generate_embeds(self, rows, ids, max_new: int, temp: float = 0.0, top_p: float = 0.95, seed: int = 1234,
                        rep_penalty: float = 1.0) -> np.ndarray:
        """Engine::generate with embeds (lib.rs:107-126): rows [n][d_model] before the prompt ids."""
        rows = np.ascontiguousarray(rows, dtype=np.float32).reshape(-1, self.cfg["d_model"])
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.zeros(max(max_new, 1), np.uint32)
        n = C.c_int()
        _check(lib().hor_generate_embeds(self.h, rows, rows.shape[0], ids.ctypes.data if len(ids) else None, len(ids),
                                         max_new, temp, top_p, seed, rep_penalty, out, C.byref(n)))
        return out[:n.value].copy()

    def run_block(self, cache: "Cache", ids, commit: bool = False, want_logits: bool = True):
        """Model::run_block (model.rs:472-510) at base = len(cache): logits [n][vocab] (or None);
        commit appends the block's K/V to the cache (lib.rs:386-391)."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.zeros((len(ids), self.vocab), np.float32) if want_logits else None
        _check(lib().hor_run_block(self.h, cache.h, ids, len(ids), 1 if commit else 0, _ptr(out)))
        return out

    def forward_bidir(self, ids) -> np.ndarray:
        """Model::forward_bidir (model.rs:441-470): logits [n][vocab] of every position."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.zeros((len(ids), self.vocab), np.float32)
        _check(lib().hor_forward_bidir(self.h, ids, len(ids), out))
        return out

    def generate_diffusion(self, ids, gen_len: int = 128, block: int = 32, steps: int = 32, temp: float = 0.0,
                           rep_penalty: float = 1.4, remask_steps: int = 0, remask_frac: float = 0.3,
                           seed: int = 1234, cached: bool = True, threshold: float = 0.0) -> np.ndarray:
        """Engine::generate_diffusion (lib.rs:211-220) on token ids; DiffOpts defaults (lib.rs:59-63)."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.zeros(max(gen_len, 1), np.uint32)
        n = C.c_int()
        _check(lib().hor_generate_diffusion(self.h, ids, len(ids), gen_len, block, steps, temp, rep_penalty,
                                            remask_steps, remask_frac, seed, 1 if cached else 0, threshold, out,
                                            C.byref(n)))
        return out[:n.value].copy()

    def last_routing(self):
        n = self.cfg["n_layers"] * self.cfg["top_k"]
        sel = np.zeros(n, np.int32)
        w = np.zeros(n, np.float32)
        _check(lib().hor_last_routing(self.h, sel, w))
        return sel.reshape(self.cfg["n_layers"], -1), w.reshape(self.cfg["n_layers"], -1)

    def generate(self, ids, max_new: int, temp: float = 0.0, top_p: float = 0.95, seed: int = 1234,
                 rep_penalty: float = 1.0, want_logits: bool = False):
        """Returns (token ids, logits [n][vocab] or None, forward seconds, prefill seconds)."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.zeros(max(max_new, 1), np.uint32)
        logits = np.zeros((max(max_new, 1), self.vocab), np.float32) if want_logits else None
        n = C.c_int()
        fs, ps = C.c_double(), C.c_double()
        _check(lib().hor_generate(self.h, ids, len(ids), max_new, temp, top_p, seed, rep_penalty, out,
                                  _ptr(logits), C.byref(n), C.byref(fs), C.byref(ps)))
        k = n.value
        return out[:k].copy(), (logits[:k].copy() if want_logits else None), fs.value, ps.value


class Cache:
    def __init__(self, eng: Engine):
        h = C.c_void_p()
        _check(lib().hor_cache_new(eng.h, C.byref(h)))
        self.h, self.eng = h, eng

    def close(self):
        if self.h:
            lib().hor_cache_free(self.h)
            self.h = None

    __del__ = close

    def __len__(self):
        return lib().hor_cache_len(self.h)

    def layer(self, li: int):
        kvd = self.eng.cfg["n_kv_heads"] * self.eng.cfg["head_dim"]
        n = len(self)
        k = np.zeros((n, kvd), np.float32)
        v = np.zeros((n, kvd), np.float32)
        _check(lib().hor_cache_read(self.h, li, k, v))
        return k, v

    def fill(self, k: np.ndarray, v: np.ndarray) -> None:
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        _check(lib().hor_cache_fill(self.eng.h, self.h, k, v, k.shape[0]))


# ---- op level ------------------------------------------------------------------------------
def q8_quantize(w: np.ndarray):
    """Q8Tensor::quantize (quant.rs:78-102): returns (int8 [out, in], f32 scales [out, in/32])."""
    w = np.ascontiguousarray(w, np.float32)
    out, inn = w.shape
    qs = np.zeros((out, inn), np.int8)
    sc = np.zeros((out, inn // 32), np.float32)
    _check(lib().hor_q8_quantize(w, out, inn, qs, sc))
    return qs, sc


def q8_quant_act(x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32)
    qx = np.zeros(x.shape[0], np.int8)
    dx = np.zeros(x.shape[0] // 32, np.float32)
    _check(lib().hor_q8_quant_act(x, x.shape[0], qx, dx))
    return qx, dx


def q8_matvec(qs, sc, x) -> np.ndarray:
    out, inn = qs.shape
    y = np.zeros(out, np.float32)
    _check(lib().hor_q8_matvec(np.ascontiguousarray(qs), np.ascontiguousarray(sc), out, inn,
                               np.ascontiguousarray(x, np.float32), y))
    return y


def q8_matmul(qs, sc, x) -> np.ndarray:
    out, inn = qs.shape
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros((x.shape[0], out), np.float32)
    _check(lib().hor_q8_matmul(np.ascontiguousarray(qs), np.ascontiguousarray(sc), out, inn, x, y, x.shape[0]))
    return y


def dequant(ggml_type: int, raw: np.ndarray, n: int) -> np.ndarray:
    y = np.zeros(n, np.float32)
    _check(lib().hor_dequant(ggml_type, np.ascontiguousarray(raw, np.uint8), n, y))
    return y


def dot(a, b) -> float:
    a = np.ascontiguousarray(a, np.float32)
    return float(lib().hor_dot(a, np.ascontiguousarray(b, np.float32), a.shape[0]))


def rmsnorm(x, w, eps) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    lib().hor_rmsnorm(x, np.ascontiguousarray(w, np.float32), eps, out, x.shape[0])
    return out


def expf(x: float) -> float:
    return float(lib().hor_expf(x))


def sample(logits, temp: float, top_p: float, state: int) -> tuple[int, int]:
    """sample.rs:66-112; returns (id, advanced xorshift64* state)."""
    st, out = C.c_uint64(state), C.c_uint32()
    _check(lib().hor_sample(np.ascontiguousarray(logits, np.float32), len(logits), temp, top_p, C.byref(st),
                            C.byref(out)))
    return int(out.value), int(st.value)


def score_block(logits, blk, committed, mask: int, rep_penalty: float, temp: float, state: int):
    """lib.rs:221-263 over rows of logits [blk_len][vocab]; returns (pred, pconf, cconf, state)."""
    logits = np.ascontiguousarray(logits, np.float32)
    blk = np.ascontiguousarray(blk, np.uint32)
    committed = np.ascontiguousarray(committed, np.uint32)
    n = len(blk)
    pred, pconf, cconf = np.zeros(n, np.uint32), np.zeros(n, np.float32), np.zeros(n, np.float32)
    st = C.c_uint64(state)
    _check(lib().hor_score_block(logits, logits.shape[1], blk, n, committed.ctypes.data if len(committed) else None,
                                 len(committed), mask, rep_penalty, temp, C.byref(st), pred, pconf, cconf))
    return pred, pconf, cconf, int(st.value)


class Moe:
    """A standalone Ffn::Moe (model.rs:29-38) over f32 expert stacks, re-quantized like Model::load."""

    def __init__(self, router, bias, gate_exps, up_exps, down_exps, gate_sh=None, up_sh=None, down_sh=None,
                 top_k=6, gating_sigmoid=True, weights_norm=False, weights_scale=1.0):
        ne, f, d = gate_exps.shape
        n_shared = 0 if gate_sh is None else 1
        self.d, self.f, self.ne, self.top_k = d, f, ne, top_k
        c = lambda a: np.ascontiguousarray(a, np.float32)
        self._keep = [c(router), c(bias), c(gate_exps), c(up_exps), c(down_exps)]
        sh = [c(a) for a in (gate_sh, up_sh, down_sh)] if n_shared else [None, None, None]
        self._keep += [a for a in sh if a is not None]
        h = C.c_void_p()
        _check(lib().hor_moe_create(d, f, ne, top_k, n_shared, int(gating_sigmoid), int(weights_norm),
                                    weights_scale, *self._keep[:5], *[_ptr(a) for a in sh], C.byref(h)))
        self.h = h

    def close(self):
        if self.h:
            lib().hor_moe_free(self.h)
            self.h = None

    __del__ = close

    def run(self, x, mode: int = 0):
        """mode 0: per-token ffn (decode); mode 1: ffn_prefill. Returns (y, sel, gate weights)."""
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        y = np.zeros((T, self.d), np.float32)
        sel = np.zeros((T, self.top_k), np.int32)
        w = np.zeros((T, self.top_k), np.float32)
        _check(lib().hor_moe_run(self.h, x, T, mode, y, _ptr(sel), _ptr(w)))
        return y, sel, w

    def expert(self, x, e: int) -> np.ndarray:
        """Expert e's SwiGLU output on one row (e = -1: the shared expert), unscaled."""
        y = np.zeros(self.d, np.float32)
        _check(lib().hor_moe_expert(self.h, np.ascontiguousarray(x, np.float32), int(e), y))
        return y

    def sel_scores(self, x) -> np.ndarray:
        out = np.zeros(self.ne, np.float32)
        _check(lib().hor_moe_sel_scores(self.h, np.ascontiguousarray(x, np.float32), out))
        return out


class Rope:
    def __init__(self, hd: int, max_pos: int, theta: float):
        h = C.c_void_p()
        _check(lib().hor_rope_create(hd, max_pos, theta, C.byref(h)))
        self.h, self.hd, self.max_pos = h, hd, max_pos

    def close(self):
        if self.h:
            lib().hor_rope_free(self.h)
            self.h = None

    __del__ = close

    def tables(self):
        c = np.zeros((self.max_pos, self.hd // 2), np.float32)
        s = np.zeros_like(c)
        _check(lib().hor_rope_tables(self.h, c, s))
        return c, s


def attn_step(rope: Rope, n_heads, n_kv_heads, hd, eps, q_norm, k_norm, qkv, pos, k_cache, v_cache) -> np.ndarray:
    """One layer's decode attention (model.rs:199-233). k_cache/v_cache: [>= pos+1, kv_dim], updated."""
    out = np.zeros(n_heads * hd, np.float32)
    _check(lib().hor_attn_step(rope.h, n_heads, n_kv_heads, hd, eps, np.ascontiguousarray(q_norm, np.float32),
                               np.ascontiguousarray(k_norm, np.float32), qkv, pos, k_cache, v_cache, out))
    return out
