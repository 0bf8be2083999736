"""Host-side checks of libhobbygpu.so that need no GPU: exported symbols, the load-time
re-quantization + lane-chunked packing, RoPE tables, GGUF parsing and its error paths."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from hobbylm_b200 import _native, synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_functions():
    txt = open(os.path.join(ROOT, "include", "hobbygpu.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(hg_[a-z0-9_]+)\s*\(", txt)))


def test_library_exports_every_header_symbol(native):
    names = _header_functions()
    assert names, "no functions parsed from include/hobbygpu.h"
    lib = native.lib()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert sorted(set(native.EXPORTS)) == names


def test_integration_guide_covers_every_entry_point():
    """The binding guide a hobby-rs maintainer follows names every function of the header."""
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    assert not [n for n in _header_functions() if n not in doc]


def _pack(native, w):
    rows, cols = w.shape
    ss = native.lib().hg_q8_scale_stride(cols)
    qs = np.empty((rows, cols), np.int8)
    sc = np.empty((rows, ss), np.float32)
    native.check(native.lib().hg_q8_pack(w.ctypes.data, rows, cols, qs.ctypes.data, sc.ctypes.data))
    un = np.empty_like(qs)
    native.check(native.lib().hg_q8_unpack_qs(qs.ctypes.data, rows, cols, un.ctypes.data))
    return un, sc, qs


@pytest.mark.parametrize("rows,cols", [(7, 768), (5, 320), (3, 192), (4, 2304), (9, 64), (2, 4128)])
def test_q8_pack_equals_oracle_requant(native, oracle_mod, rows, cols):
    rng = np.random.default_rng(rows * cols)
    w = (rng.standard_normal((rows, cols)) * 0.05).astype(np.float32)
    w[0, :32] = 0.0  # an all-zero block (d = 0, id = 0)
    w[1, 5] = 0.5 / 127.0 * np.abs(w[1, :32]).max() * 127.0  # values near rounding ties
    un, sc, packed = _pack(native, w)
    oq, osc = oracle_mod.q8_quantize(w)
    nb = cols // 32
    assert np.array_equal(un, oq)
    assert np.array_equal(sc[:, :nb].view(np.uint32), osc.view(np.uint32))
    assert not sc[:, nb:].any()
    # the lane-chunked permutation: lane l of a 4-block chunk holds bytes 4l..4l+3 of each block
    if nb >= 4:
        for l in range(8):
            for b in range(4):
                assert np.array_equal(packed[:, l * 16 + b * 4: l * 16 + b * 4 + 4], oq[:, b * 32 + 4 * l: b * 32 + 4 * l + 4])


def test_q8_pack_from_q8_0_blocks_matches_oracle(native, oracle_mod):
    """Config-2 style weights (int8 ~ U[-127,127] with |N(0,0.01)| f16 scales, dequantized as
    gguf.rs does) through the re-quantizer: bit-identical codes and scales."""
    inp = synth.moe_op_inputs(seed=2, T=1)
    w = inp["down_exps"][0]
    un, sc, _ = _pack(native, w)
    oq, osc = oracle_mod.q8_quantize(w)
    assert np.array_equal(un, oq) and np.array_equal(sc[:, : w.shape[1] // 32], osc)


def test_rope_tables_match_oracle(native, oracle_mod):
    hd, mp, theta = 128, 300, 10000.0
    c = np.empty((mp, hd // 2), np.float32)
    s = np.empty_like(c)
    native.check(native.lib().hg_rope_tables(hd, mp, theta, c.ctypes.data, s.ctypes.data))
    r = oracle_mod.Rope(hd, mp, theta)
    oc, os_ = r.tables()
    assert np.array_equal(c, oc) and np.array_equal(s, os_)


def _config(native, path):
    cfg = native.Config()
    rc = native.lib().hg_gguf_config(str(path).encode(), C.byref(cfg))
    return rc, cfg


def test_gguf_config_matches_oracle(native, oracle_mod, model130):
    rc, cfg = _config(native, model130)
    assert rc == 0
    ora = oracle_mod.Engine(model130, quant=True)
    d = cfg.as_dict()
    for k, v in ora.cfg.items():
        key = "eos_token" if k == "eos" else k
        assert d[key] == pytest.approx(v), k


def _write_gguf(path, meta: dict, tensors: dict, arch="hobbylm"):
    import gguf

    w = gguf.GGUFWriter(str(path), arch)
    for k, v in meta.items():
        if isinstance(v, bool):
            w.add_bool(f"{arch}.{k}", v)
        elif isinstance(v, int):
            w.add_uint32(f"{arch}.{k}", v)
        elif isinstance(v, float):
            w.add_float32(f"{arch}.{k}", v)
    for name, arr in tensors.items():
        w.add_tensor(name, arr)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def test_config_defaults_follow_config_rs(native, tmp_path):
    """Optional keys take config.rs's defaults: leading_dense_block_count 1, expert_shared_count 0,
    context_length 8192, rms_eps 1e-5, rope.freq_base 1e6, expert_weights_scale 1, head_dim = d/h,
    vocab from token_embd rows."""
    p = tmp_path / "m.gguf"
    meta = {"embedding_length": 64, "block_count": 2, "attention.head_count": 2, "attention.head_count_kv": 1,
            "feed_forward_length": 64, "expert_feed_forward_length": 32, "expert_count": 4, "expert_used_count": 2}
    _write_gguf(p, meta, {"token_embd.weight": np.zeros((123, 64), np.float32)})
    rc, cfg = _config(native, p)
    assert rc == 0
    c = cfg.as_dict()
    assert (c["n_dense"], c["n_shared"], c["context_length"], c["head_dim"], c["vocab_size"]) == (1, 0, 8192, 32, 123)
    assert c["rms_eps"] == pytest.approx(1e-5) and c["rope_theta"] == 1e6 and c["expert_weights_scale"] == 1.0
    assert c["gating_sigmoid"] == 1 and c["expert_weights_norm"] == 0 and c["eos_token"] == 50256


def test_diffusion_keys_follow_config_rs(native, tmp_path):
    """diffusion.enabled / mask_token_id / block_size (config.rs:92-94) carry no architecture prefix;
    absent they default to false / 50257 / 32."""
    import gguf

    meta = {"embedding_length": 64, "block_count": 2, "attention.head_count": 2, "attention.head_count_kv": 1,
            "feed_forward_length": 64, "expert_feed_forward_length": 32, "expert_count": 4, "expert_used_count": 2}
    p = tmp_path / "d.gguf"
    w = gguf.GGUFWriter(str(p), "hobbylm")
    for k, v in meta.items():
        w.add_uint32(f"hobbylm.{k}", v)
    w.add_bool("diffusion.enabled", True)
    w.add_uint32("diffusion.mask_token_id", 100)
    w.add_uint32("diffusion.block_size", 16)
    w.add_tensor("token_embd.weight", np.zeros((123, 64), np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    rc, cfg = _config(native, p)
    assert rc == 0
    c = cfg.as_dict()
    assert (c["diffusion"], c["mask_token_id"], c["block_size"]) == (1, 100, 16)
    q = tmp_path / "e.gguf"
    _write_gguf(q, meta, {"token_embd.weight": np.zeros((123, 64), np.float32)})
    rc, cfg = _config(native, q)
    assert rc == 0 and (cfg.diffusion, cfg.mask_token_id, cfg.block_size) == (0, 50257, 32)


def test_gguf_errors(native, tmp_path):
    lib = native.lib()
    h = C.c_void_p()
    assert lib.hg_engine_load(str(tmp_path / "missing.gguf").encode(), 0, C.byref(h)) == -2
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + b"\0" * 64)
    assert lib.hg_engine_load(str(bad).encode(), 0, C.byref(h)) == -3
    assert b"bad magic" in lib.hg_last_error()
    v2 = tmp_path / "v2.gguf"
    v2.write_bytes(b"GGUF" + (2).to_bytes(4, "little") + b"\0" * 16)
    assert lib.hg_engine_load(str(v2).encode(), 0, C.byref(h)) == -3
    assert b"version 2" in lib.hg_last_error()
    good = tmp_path / "g.gguf"
    meta = {"embedding_length": 64, "block_count": 2, "attention.head_count": 2, "attention.head_count_kv": 1,
            "feed_forward_length": 64, "expert_feed_forward_length": 32, "expert_count": 4, "expert_used_count": 2}
    _write_gguf(good, meta, {"token_embd.weight": np.zeros((16, 64), np.float32)})
    data = good.read_bytes()
    trunc = tmp_path / "t.gguf"
    trunc.write_bytes(data[:40])
    assert lib.hg_engine_load(str(trunc).encode(), 0, C.byref(h)) == -3
    assert b"unexpected end of file" in lib.hg_last_error()
    # missing required metadata / tensors
    nometa = tmp_path / "nm.gguf"
    _write_gguf(nometa, {k: v for k, v in meta.items() if k != "expert_count"},
                {"token_embd.weight": np.zeros((16, 64), np.float32)})
    assert lib.hg_engine_load(str(nometa).encode(), 0, C.byref(h)) == -4
    assert b"expert_count" in lib.hg_last_error()
    # the tokenizer arrays are required (tokenizer.rs:55-61) before any GPU work
    assert lib.hg_engine_load(str(good).encode(), 0, C.byref(h)) == -4
    assert b"tokenizer" in lib.hg_last_error()


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    """No fallback: without libhobbygpu.so every entry point raises."""
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setattr(_native, "LIB_PATH", str(tmp_path / "nope.so"))
    with pytest.raises(ImportError):
        _native.lib()


# block layouts (bytes per block, elements per block, byte offsets of the f16 scale fields)
_QBLOCKS = {
    "Q8_0": (34, 32, (0,)),
    "Q5_0": (22, 32, (0,)),
    "Q4_K": (144, 256, (0, 2)),
    "Q6_K": (210, 256, (208,)),
}


def _random_blocks(qtype, rows, cols, rng):
    nbytes, nel, f16_at = _QBLOCKS[qtype]
    nblk = cols // nel
    raw = rng.integers(0, 256, (rows, nblk, nbytes), dtype=np.uint8)
    for off in f16_at:  # finite scales
        d = (rng.standard_normal((rows, nblk)) * 0.02).astype(np.float16)
        raw[:, :, off:off + 2] = d.view(np.uint8).reshape(rows, nblk, 2)
    return raw.reshape(rows, nblk * nbytes)


@pytest.mark.parametrize("qtype", ["F16", "Q8_0", "Q5_0", "Q4_K", "Q6_K"])
def test_gguf_tensor_dequant_matches_gguf_py(native, tmp_path, qtype):
    """Gguf::load (gguf.rs:250-269, 329-468) on every supported quantized type: the library's host
    dequantization equals gguf-py's, bit for bit, on random valid blocks."""
    import gguf

    rng = np.random.default_rng(7)
    rows, cols = 6, 512
    w = gguf.GGUFWriter(str(tmp_path / "q.gguf"), "hobbylm")
    if qtype == "F16":
        data = (rng.standard_normal((rows, cols)) * 0.5).astype(np.float16)
        w.add_tensor("t", data)
        ref = data.astype(np.float32)
    else:
        qt = getattr(gguf.GGMLQuantizationType, qtype)
        data = _random_blocks(qtype, rows, cols, rng)
        w.add_tensor("t", data, raw_dtype=qt)
        ref = np.asarray(gguf.quants.dequantize(data, qt), dtype=np.float32).reshape(rows, cols)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    out = np.empty(rows * cols, np.float32)
    lib = native.lib()
    native.check(lib.hg_gguf_tensor_f32(str(tmp_path / "q.gguf").encode(), b"t", out.ctypes.data, out.size))
    assert np.array_equal(out.view(np.uint32), ref.ravel().view(np.uint32))
    # wrong element count and missing tensor are errors, not silent truncation
    assert lib.hg_gguf_tensor_f32(str(tmp_path / "q.gguf").encode(), b"t", out.ctypes.data, out.size - 1) == -1
    assert lib.hg_gguf_tensor_f32(str(tmp_path / "q.gguf").encode(), b"nope", out.ctypes.data, out.size) == -4


def test_noalloc_matvec_rejects_out_of_range_shapes_before_any_device_work(native):
    """Rows or columns beyond INT_MAX, or a column count whose scratch size would wrap, are
    rejected from the arguments alone (dummy non-null pointers; no device is touched)."""
    lib = native.lib()
    p = C.c_void_p(16)
    for rows, cols, ntok in ((64, 1 << 62, 4), (1 << 31, 768, 1), (64, (1 << 31) + 32, 1)):
        rc = lib.hg_op_q8_matvec_noalloc(p, p, rows, cols, p, p, ntok, None)
        assert rc == -1, (rows, cols, ntok)  # HG_ERR_INVALID
        assert b"INT_MAX" in lib.hg_last_error()
