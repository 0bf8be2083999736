"""ctypes binding of libhobbygpu.so (include/hobbygpu.h).

The library is built in-tree by ``python -m hobbylm_b200.build``. There is no fallback: if the
shared library is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libhobbygpu.so")

HG_OK = 0
ERRORS = {
    -1: "HG_ERR_INVALID", -2: "HG_ERR_IO", -3: "HG_ERR_FORMAT", -4: "HG_ERR_MISSING", -5: "HG_ERR_CUDA",
    -6: "HG_ERR_POOL_EXHAUSTED", -7: "HG_ERR_CONTEXT", -8: "HG_ERR_TOKEN", -9: "HG_ERR_TIMEOUT",
}

# every symbol include/hobbygpu.h declares
EXPORTS = (
    "hg_last_error", "hg_engine_load", "hg_engine_load_ex", "hg_engine_free", "hg_engine_config", "hg_gguf_config",
    "hg_gguf_tensor_f32", "hg_prefill_embeds", "hg_forward_x", "hg_run_block", "hg_generate_diffusion",
    "hg_engine_weight_bytes", "hg_engine_eos", "hg_engine_device_bytes", "hg_seq_create", "hg_seq_free",
    "hg_seq_len", "hg_prefill", "hg_forward", "hg_decode_batch", "hg_generate", "hg_debug_last_routing",
    "hg_q8_pack", "hg_q8_scale_stride", "hg_q8_unpack_qs", "hg_op_q8_matvec", "hg_op_q8_matmul",
    "hg_op_moe_scratch_bytes", "hg_op_moe_ffn", "hg_op_kv_attn_scratch_bytes", "hg_op_kv_attn", "hg_rope_tables",
    "hg_decode_greedy", "hg_engine_stream", "hg_decode_kernel_count", "hg_debug_time_attention",
    "hg_op_q8_matvec_noalloc", "hg_host_sample", "hg_host_score_block", "hg_generate_embeds",
    "hg_ep_unique_id", "hg_engine_ep_init",
)
NOALLOC_SCRATCH_BYTES = 4 << 20  # HG_NOALLOC_SCRATCH_BYTES


class HgError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


class Config(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "d_model", "n_layers", "n_dense", "n_heads", "n_kv_heads", "head_dim", "dense_ffn", "expert_ffn",
        "n_experts", "top_k", "n_shared", "vocab_size", "context_length", "expert_weights_norm",
        "gating_sigmoid", "eos_token")] + [("rms_eps", C.c_float), ("rope_theta", C.c_float),
                                           ("expert_weights_scale", C.c_float)] + [
        (n, C.c_int32) for n in ("diffusion", "mask_token_id", "block_size")]

    def as_dict(self) -> dict:
        return {n: getattr(self, n) for n, _ in self._fields_}


class EngineOpts(C.Structure):
    _fields_ = [("device", C.c_int32), ("max_batch", C.c_int32), ("kv_pool_tokens", C.c_int64),
                ("kv_page_shuffle", C.c_uint64)]


class GenOptsC(C.Structure):
    _fields_ = [("max_new", C.c_int32), ("temp", C.c_float), ("top_p", C.c_float), ("seed", C.c_uint64),
                ("rep_penalty", C.c_float)]


class DiffOptsC(C.Structure):
    _fields_ = [("gen_len", C.c_int32), ("block", C.c_int32), ("steps", C.c_int32), ("temp", C.c_float),
                ("rep_penalty", C.c_float), ("remask_steps", C.c_int32), ("remask_frac", C.c_float),
                ("seed", C.c_uint64), ("cached", C.c_int32), ("threshold", C.c_float)]


class MoeWeights(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("d_model", "expert_ffn", "n_experts", "top_k", "n_shared",
                                         "gating_sigmoid", "weights_norm")] + [("weights_scale", C.c_float)] + [
        (n, C.c_void_p) for n in ("router", "bias", "gate_qs", "gate_sc", "up_qs", "up_sc", "down_qs", "down_sc",
                                  "sh_gate_qs", "sh_gate_sc", "sh_up_qs", "sh_up_sc", "sh_down_qs", "sh_down_sc")]


class KvAttnArgs(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("n_seqs", "n_heads", "n_kv_heads", "head_dim", "max_pos")] + [
        ("eps", C.c_float)] + [(n, C.c_void_p) for n in ("qkv", "q_norm", "k_norm", "rope_cos", "rope_sin", "pos",
                                                         "block_table")] + [
        ("bt_stride", C.c_int32), ("k_pool", C.c_void_p), ("v_pool", C.c_void_p), ("page_stride", C.c_int64),
        ("out", C.c_void_p)]


TOKEN_CB = C.CFUNCTYPE(C.c_int, C.c_uint32, C.c_void_p)
BLOCK_CB = C.CFUNCTYPE(C.c_int, C.POINTER(C.c_uint32), C.c_int, C.c_void_p)

_lib = None


def lib():
    """Load libhobbygpu.so (raises if it is missing: the CUDA path is the only path)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing; build it with `python -m hobbylm_b200.build`")
    L = C.CDLL(LIB_PATH)
    vp, i32, i64, u32, u64, f32, sz = C.c_void_p, C.c_int, C.c_int64, C.c_uint32, C.c_uint64, C.c_float, C.c_size_t
    sig = {
        "hg_last_error": (C.c_char_p, []),
        "hg_engine_load": (i32, [C.c_char_p, i32, C.POINTER(vp)]),
        "hg_engine_load_ex": (i32, [C.c_char_p, C.POINTER(EngineOpts), C.POINTER(vp)]),
        "hg_engine_free": (None, [vp]),
        "hg_engine_config": (i32, [vp, C.POINTER(Config)]),
        "hg_gguf_config": (i32, [C.c_char_p, C.POINTER(Config)]),
        "hg_gguf_tensor_f32": (i32, [C.c_char_p, C.c_char_p, vp, i64]),
        "hg_engine_weight_bytes": (u64, [vp]),
        "hg_engine_eos": (u32, [vp]),
        "hg_engine_device_bytes": (u64, [vp]),
        "hg_seq_create": (i32, [vp, i32, C.POINTER(vp)]),
        "hg_seq_free": (None, [vp]),
        "hg_seq_len": (i32, [vp]),
        "hg_prefill": (i32, [vp, vp, vp, i32, vp]),
        "hg_prefill_embeds": (i32, [vp, vp, vp, i32, vp]),
        "hg_forward": (i32, [vp, vp, u32, vp, vp]),
        "hg_forward_x": (i32, [vp, vp, vp, vp, vp]),
        "hg_decode_batch": (i32, [vp, vp, i32, vp, vp, vp]),
        "hg_generate": (i32, [vp, vp, i32, C.POINTER(GenOptsC), TOKEN_CB, vp, vp]),
        "hg_generate_embeds": (i32, [vp, vp, i32, vp, i32, C.POINTER(GenOptsC), TOKEN_CB, vp, vp]),
        "hg_run_block": (i32, [vp, vp, vp, i32, i32, i32, vp]),
        "hg_host_sample": (i32, [vp, i32, f32, f32, C.POINTER(u64), vp]),
        "hg_host_score_block": (i32, [vp, i32, vp, i32, vp, i32, u32, f32, f32, C.POINTER(u64), vp, vp, vp]),
        "hg_generate_diffusion": (i32, [vp, vp, i32, C.POINTER(DiffOptsC), BLOCK_CB, vp, vp]),
        "hg_debug_last_routing": (i32, [vp, i32, vp]),
        "hg_q8_pack": (i32, [vp, i64, i64, vp, vp]),
        "hg_q8_scale_stride": (i32, [i64]),
        "hg_q8_unpack_qs": (i32, [vp, i64, i64, vp]),
        "hg_op_q8_matvec": (i32, [vp, vp, i64, i64, vp, vp, i32, vp]),
        "hg_op_q8_matmul": (i32, [vp, vp, i64, i64, vp, vp, i32, vp]),
        "hg_op_q8_matvec_noalloc": (i32, [vp, vp, i64, i64, vp, vp, i32, vp]),
        "hg_op_moe_scratch_bytes": (sz, [C.POINTER(MoeWeights), i32]),
        "hg_op_moe_ffn": (i32, [C.POINTER(MoeWeights), vp, i32, vp, vp, vp, vp]),
        "hg_op_kv_attn_scratch_bytes": (sz, [C.POINTER(KvAttnArgs)]),
        "hg_op_kv_attn": (i32, [C.POINTER(KvAttnArgs), vp, vp]),
        "hg_rope_tables": (i32, [i32, i32, f32, vp, vp]),
        "hg_decode_greedy": (i32, [vp, vp, i32, vp, i32, vp]),
        "hg_engine_stream": (vp, [vp]),
        "hg_ep_unique_id": (i32, [vp]),
        "hg_engine_ep_init": (i32, [vp, vp, i32, i32]),
        "hg_decode_kernel_count": (i32, [vp, i32]),
        "hg_debug_time_attention": (i32, [vp, vp, i32, i32, C.POINTER(f32), C.POINTER(f32)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(rc: int) -> int:
    if rc < 0:
        raise HgError(rc, lib().hg_last_error().decode(errors="replace"))
    return rc
