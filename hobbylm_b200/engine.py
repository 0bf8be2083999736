"""Python mirror of the hobby-rs engine surface over libhobbygpu.so.

Names and behaviour follow hobby-rs/src/lib.rs (``Engine::load``, ``generate``, ``eos``,
``weight_bytes``, ``GenOpts``) and hobby-rs/src/model.rs (``KvCache``, ``Model::prefill``,
``Model::forward``). Token ids replace text at this boundary: the tokenizer (tokenizer.rs) is
host-side text I/O outside the decode path, so ``generate`` takes prompt ids and streams ids.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Callable, Iterable, Sequence

import numpy as np

from ._native import BLOCK_CB, Config, DiffOptsC, EngineOpts, GenOptsC, HgError, TOKEN_CB, check, lib

GPT2_VALID = 50257  # lib.rs:26


@dataclass
class GenOpts:
    """lib.rs:29-41 (same defaults)."""
    max_new: int = 256
    temp: float = 0.0
    top_p: float = 0.95
    seed: int = 1234
    rep_penalty: float = 1.0

    def c(self) -> GenOptsC:
        return GenOptsC(self.max_new, self.temp, self.top_p, self.seed, self.rep_penalty)


@dataclass
class DiffOpts:
    """DiffOpts (lib.rs:43-63, same defaults). block 0 takes the model's diffusion.block_size."""
    gen_len: int = 128
    block: int = 32
    steps: int = 32
    temp: float = 0.0
    rep_penalty: float = 1.4
    remask_steps: int = 0
    remask_frac: float = 0.3
    seed: int = 1234
    cached: bool = True
    threshold: float = 0.0

    def c(self) -> DiffOptsC:
        return DiffOptsC(self.gen_len, self.block, self.steps, self.temp, self.rep_penalty, self.remask_steps,
                         self.remask_frac, self.seed, 1 if self.cached else 0, self.threshold)


def _u32(ids) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(ids, dtype=np.int64).astype(np.uint32))


class KvCache:
    """A sequence's paged KV cache on the GPU (model.rs:60-75). Free with close()."""

    def __init__(self, eng: "Engine", max_ctx: int = 0):
        h = C.c_void_p()
        check(lib().hg_seq_create(eng.h, int(max_ctx), C.byref(h)))
        self.h, self.eng = h, eng

    @property
    def len(self) -> int:
        return lib().hg_seq_len(self.h)

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().hg_seq_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class Engine:
    """A loaded model on one GPU (lib.rs:78-102). Weights are re-quantized on the host exactly as
    Model::load does and uploaded to HBM once."""

    def __init__(self, h: C.c_void_p):
        self.h = h
        cfg = Config()
        check(lib().hg_engine_config(self.h, C.byref(cfg)))
        self.cfg = cfg.as_dict()

    @classmethod
    def load(cls, path: str, quant: bool = True, device: int = 0, max_batch: int = 1, kv_pool_tokens: int = 0,
             kv_page_shuffle: int = 0) -> "Engine":
        if not quant:
            raise ValueError("the GPU engine runs the Q8 path (hobby-rs --quant q8); --quant f32 is CPU-only")
        opts = EngineOpts(device, max_batch, kv_pool_tokens, kv_page_shuffle)
        h = C.c_void_p()
        check(lib().hg_engine_load_ex(str(path).encode(), C.byref(opts), C.byref(h)))
        return cls(h)

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().hg_engine_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # lib.rs:94-102
    def eos(self) -> int:
        return int(lib().hg_engine_eos(self.h))

    def weight_bytes(self) -> int:
        return int(lib().hg_engine_weight_bytes(self.h))

    def device_bytes(self) -> int:
        return int(lib().hg_engine_device_bytes(self.h))

    @property
    def vocab(self) -> int:
        return self.cfg["vocab_size"]

    def new_cache(self, max_ctx: int = 0) -> KvCache:
        return KvCache(self, max_ctx)

    def prefill(self, cache: KvCache, ids: Sequence[int]) -> np.ndarray:
        """Model::prefill on token ids; returns the last position's logits."""
        ids = _u32(ids)
        out = np.empty(self.vocab, np.float32)
        check(lib().hg_prefill(self.h, cache.h, ids.ctypes.data, len(ids), out.ctypes.data))
        return out

    def prefill_embeds(self, cache: KvCache, rows) -> np.ndarray:
        """Model::prefill on caller rows (n x d_model f32, e.g. modality embeddings spliced before a
        prompt, lib.rs:118-121); returns the last position's logits."""
        rows = np.ascontiguousarray(rows, dtype=np.float32)
        if rows.ndim != 2 or rows.shape[1] != self.cfg["d_model"]:
            raise HgError(-1, f"rows must be n x {self.cfg['d_model']}")
        out = np.empty(self.vocab, np.float32)
        check(lib().hg_prefill_embeds(self.h, cache.h, rows.ctypes.data, rows.shape[0], out.ctypes.data))
        return out

    def forward_x(self, cache: KvCache, row, want_logits: bool = True):
        """Model::forward_x (model.rs:160): one decode step from a d_model-float row instead of a
        token embedding. Returns (logits or None, greedy next id with ids >= 50257 masked)."""
        row = np.ascontiguousarray(row, dtype=np.float32)
        if row.shape != (self.cfg["d_model"],):
            raise HgError(-1, f"row must have {self.cfg['d_model']} floats")
        out = np.empty(self.vocab, np.float32) if want_logits else None
        nxt = C.c_uint32()
        check(lib().hg_forward_x(self.h, cache.h, row.ctypes.data, out.ctypes.data if want_logits else None,
                                 C.byref(nxt)))
        return out, int(nxt.value)

    def forward(self, cache: KvCache, token: int, pos: int | None = None, want_logits: bool = True):
        """Model::forward(token, pos, cache). pos, if given, must equal the cache length.
        Returns (logits or None, greedy next id with ids >= 50257 masked)."""
        if pos is not None and pos != cache.len:
            raise HgError(-1, f"pos {pos} != cache length {cache.len}")
        out = np.empty(self.vocab, np.float32) if want_logits else None
        nxt = C.c_uint32()
        check(lib().hg_forward(self.h, cache.h, int(token), out.ctypes.data if want_logits else None, C.byref(nxt)))
        return out, int(nxt.value)

    def decode_batch(self, caches: Sequence[KvCache], tokens: Sequence[int], want_logits: bool = False):
        n = len(caches)
        arr = (C.c_void_p * n)(*[c.h.value for c in caches])
        toks = _u32(tokens)
        nxt = np.empty(n, np.uint32)
        logits = np.empty((n, self.vocab), np.float32) if want_logits else None
        check(lib().hg_decode_batch(self.h, arr, n, toks.ctypes.data, nxt.ctypes.data,
                                    logits.ctypes.data if want_logits else None))
        return nxt, logits

    def decode_greedy(self, caches: Sequence[KvCache], tokens: Sequence[int], steps: int,
                      want_ids: bool = True):
        """``steps`` greedy steps for the batch, driven on the device; returns [steps][n] ids."""
        n = len(caches)
        arr = (C.c_void_p * n)(*[c.h.value for c in caches])
        toks = _u32(tokens)
        out = np.empty((steps, n), np.uint32) if want_ids else None
        check(lib().hg_decode_greedy(self.h, arr, n, toks.ctypes.data, steps,
                                     out.ctypes.data if want_ids else None))
        return out

    def stream(self) -> int:
        return int(lib().hg_engine_stream(self.h) or 0)

    @staticmethod
    def ep_unique_id() -> bytes:
        """A new NCCL unique id (128 bytes) for expert parallelism (hobbylm_b200.ep)."""
        buf = C.create_string_buffer(128)
        check(lib().hg_ep_unique_id(buf))
        return buf.raw

    def ep_init(self, nccl_id: bytes, rank: int, world: int) -> None:
        """Split the routed experts over `world` ranks (hg_engine_ep_init); call on every rank
        before the first decode step. hobbylm_b200.ep.setup does the id exchange."""
        if len(nccl_id) != 128:
            raise HgError(-1, "an NCCL unique id is 128 bytes")
        buf = C.create_string_buffer(bytes(nccl_id), 128)
        check(lib().hg_engine_ep_init(self.h, buf, int(rank), int(world)))

    def decode_kernel_count(self, n: int) -> int:
        return check(lib().hg_decode_kernel_count(self.h, n))

    def time_attention(self, caches: Sequence[KvCache], iters: int = 10):
        n = len(caches)
        arr = (C.c_void_p * n)(*[c.h.value for c in caches])
        a, b = C.c_float(), C.c_float()
        check(lib().hg_debug_time_attention(self.h, arr, n, iters, C.byref(a), C.byref(b)))
        return a.value, b.value

    def last_routing(self, slot: int = 0) -> np.ndarray:
        sel = np.empty((self.cfg["n_layers"], self.cfg["top_k"]), np.int32)
        check(lib().hg_debug_last_routing(self.h, slot, sel.ctypes.data))
        return sel

    def run_block(self, cache: KvCache, ids, n_logits: int | None = None, commit: bool = False):
        """Model::run_block (model.rs:472-510) at position cache.len: the rows attend to the prefix and
        to each other. Returns the logits [n_logits][vocab] of the last n_logits rows (default all, 0
        for none); commit appends the block's K/V to the sequence (lib.rs:386-391)."""
        ids = _u32(list(ids))
        nl = len(ids) if n_logits is None else int(n_logits)
        out = np.empty((nl, self.vocab), np.float32) if nl > 0 else None
        check(lib().hg_run_block(self.h, cache.h, ids.ctypes.data, len(ids), nl, 1 if commit else 0,
                                 out.ctypes.data if out is not None else None))
        return out

    def generate_diffusion(self, prompt_ids: Iterable[int], opts: DiffOpts | None = None,
                           on_block: Callable[[list[int]], bool] | None = None) -> list[int]:
        """Engine::generate_diffusion (lib.rs:211-495) on token ids. on_block(ids) receives each
        finished block's new ids (up to the first eos) and returns False to stop."""
        opts = opts or DiffOpts()
        ids = _u32(list(prompt_ids))
        out = np.empty(max(opts.gen_len, 1), np.uint32)
        err: list[BaseException] = []

        def cb(p, n, _user):
            if on_block is None:
                return 1
            try:
                return 1 if on_block([int(p[i]) for i in range(n)]) else 0
            except BaseException as ex:  # stop generation and re-raise after the call returns
                err.append(ex)
                return 0

        cfun = BLOCK_CB(cb)
        o = opts.c()
        n = check(lib().hg_generate_diffusion(self.h, ids.ctypes.data if len(ids) else None, len(ids), C.byref(o),
                                              cfun, None, out.ctypes.data))
        if err:
            raise err[0]
        return [int(t) for t in out[:n]]

    def generate(self, prompt_ids: Iterable[int], opts: GenOpts | None = None,
                 on_token: Callable[[int], bool] | None = None, embeds=None) -> list[int]:
        """Engine::generate (lib.rs:107-162) on token ids. on_token(id) returns False to stop.
        embeds: optional [n][d_model] rows prefilled before the prompt (lib.rs:118-121)."""
        opts = opts or GenOpts()
        ids = _u32(list(prompt_ids))
        rows = None
        if embeds is not None:
            rows = np.ascontiguousarray(embeds, dtype=np.float32).reshape(-1, self.cfg["d_model"])
        out = np.empty(max(opts.max_new, 1), np.uint32)
        err: list[BaseException] = []

        def cb(tok, _user):
            if on_token is None:
                return 1
            try:
                return 1 if on_token(int(tok)) else 0
            except BaseException as ex:  # stop generation and re-raise after the call returns
                err.append(ex)
                return 0

        cfun = TOKEN_CB(cb)
        o = opts.c()
        if rows is None:
            n = check(lib().hg_generate(self.h, ids.ctypes.data, len(ids), C.byref(o), cfun, None, out.ctypes.data))
        else:
            n = check(lib().hg_generate_embeds(self.h, rows.ctypes.data if len(rows) else None, len(rows),
                                               ids.ctypes.data if len(ids) else None, len(ids), C.byref(o), cfun,
                                               None, out.ctypes.data))
        if err:
            raise err[0]
        return [int(t) for t in out[:n]]
