"""CPU checks that pin the synthetic-model producer and the oracle to the reference's own code.

* synth_digests_*.json: per-tensor digests of the F32 GGUF written by the reference exporter
  (export/to_gguf.py) from the reference's seed-0 MoETransformer (tests/golden/make_golden.py);
  hobbylm_b200.synth must reproduce every tensor bit for bit.
* torch_logits_130M.npz: the reference PyTorch forward (hobbylm/model.py) of the 130M model;
  the oracle's F32 path (hobby-rs --quant f32 semantics) must match it within f32 reordering
  tolerance (the two sum in different orders).
"""
import json
import os

import numpy as np
import pytest

from hobbylm_b200 import synth

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("preset", ["130M", "500M", "1B"])
def test_synth_matches_reference_export(preset):
    with open(os.path.join(GOLDEN, f"synth_digests_{preset}.json")) as f:
        g = json.load(f)
    got = synth.digests(preset, seed=0)
    assert set(got) == set(g["digests"])
    bad = [k for k, v in g["digests"].items() if got[k] != v]
    assert not bad, f"{len(bad)} tensors differ, e.g. {bad[:3]}"
    m = g["meta"]
    p = synth.PRESETS[preset]
    assert m["hobbylm.embedding_length"] == p.d_model and m["hobbylm.block_count"] == p.n_layers
    assert m["hobbylm.expert_used_count"] == p.top_k and m["hobbylm.rope.freq_base"] == p.rope_theta


def test_oracle_f32_matches_reference_torch(oracle_mod):
    g = np.load(os.path.join(GOLDEN, "torch_logits_130M.npz"))
    path = synth.cached_model("130M", 0, quant="f32", rms_eps=1e-6)
    eng = oracle_mod.Engine(path, quant=False)
    c = eng.new_cache()
    last = eng.prefill(c, g["ids"])
    rel = np.linalg.norm(last - g["last"]) / np.linalg.norm(g["last"])
    assert rel < 1e-5, rel
    assert np.array_equal(np.argsort(-last)[:8], g["top_ids"][-1])
    # the decode path (Model::forward) over the same tokens, one position at a time
    c2 = eng.new_cache()
    lg = eng.prefill(c2, g["ids"][:1])
    for pos in range(1, len(g["ids"])):
        top = np.argsort(-lg)[:8]
        assert np.array_equal(top, g["top_ids"][pos - 1]), pos
        lse = np.log(np.exp(lg - lg.max()).sum()) + lg.max()
        assert abs(lse - g["lse"][pos - 1]) < 1e-4
        lg = eng.forward(c2, int(g["ids"][pos]), pos)
    rel = np.linalg.norm(lg - g["last"]) / np.linalg.norm(g["last"])
    assert rel < 1e-5, rel


def test_oracle_forward_bidir_matches_reference_torch(oracle_mod):
    """Model::forward_bidir (model.rs:441-470), the pass the diffusion decode is built on, against
    the reference PyTorch model in its diffusion mode (bidirectional attention,
    hobbylm/model.py:225-226) on a canvas of 12 prompt ids and 6 [MASK] ids."""
    g = np.load(os.path.join(GOLDEN, "torch_bidir_logits_130M.npz"))
    path = synth.cached_model("130M", 0, quant="f32", rms_eps=1e-6)
    eng = oracle_mod.Engine(path, quant=False)
    lg = eng.forward_bidir(g["ids"])
    for r, full in zip(g["rows"], g["full"]):
        rel = np.linalg.norm(lg[r] - full) / np.linalg.norm(full)
        assert rel < 1e-5, (int(r), rel)
    for pos in range(len(g["ids"])):
        assert np.array_equal(np.argsort(-lg[pos])[:8], g["top_ids"][pos]), pos
        lse = np.log(np.exp(lg[pos] - lg[pos].max()).sum()) + lg[pos].max()
        assert abs(lse - g["lse"][pos]) < 1e-4, pos
    # a causal pass over the same canvas differs at the prompt positions, which now see the masks
    c = eng.new_cache()
    causal_first = eng.prefill(c, g["ids"][:1])
    assert np.linalg.norm(causal_first - g["full"][0]) / np.linalg.norm(g["full"][0]) > 1e-3


def test_oracle_diffusion_loop_matches_reference_sampler(oracle_mod):
    """The uncached denoising loop (hobby-rs lib.rs:409-495) at temperature 0 against the
    reference's own greedy sampler (hobbylm/diffusion.py:92-176) on the F32 model: same ids for
    three schedules, with and without the presence penalty and a remasking pass."""
    with open(os.path.join(GOLDEN, "torch_diffusion_generate_130M.json")) as f:
        g = json.load(f)
    path = synth.cached_model("130M", 0, quant="f32", rms_eps=1e-6)
    eng = oracle_mod.Engine(path, quant=False)
    prompt = np.array(g["prompt"], np.uint32)
    for case in g["cases"]:
        got = eng.generate_diffusion(prompt, cached=False, temp=0.0, **case["opts"])
        assert [int(t) for t in got] == case["ids"], case["opts"]


def test_oracle_rows_match_reference_inputs_embeds(oracle_mod):
    """Model::prefill and forward_x on caller rows (model.rs:160, 340) against the reference model's
    inputs_embeds forward (hobbylm/model.py:325-333): 4 rows spliced before 8 token embeddings."""
    g = np.load(os.path.join(GOLDEN, "torch_embeds_logits_130M.npz"))
    path = synth.cached_model("130M", 0, quant="f32", rms_eps=1e-6)
    eng = oracle_mod.Engine(path, quant=False)
    rows = g["rows"]
    last = eng.prefill_embeds(eng.new_cache(), rows)
    rel = np.linalg.norm(last - g["last"]) / np.linalg.norm(g["last"])
    assert rel < 1e-5, rel
    c = eng.new_cache()
    lg = eng.prefill_embeds(c, rows[:1])
    for pos in range(1, len(rows)):
        assert np.array_equal(np.argsort(-lg)[:8], g["top_ids"][pos - 1]), pos
        lse = np.log(np.exp(lg - lg.max()).sum()) + lg.max()
        assert abs(lse - g["lse"][pos - 1]) < 1e-4, pos
        lg = eng.forward_x(c, rows[pos], pos)
    rel = np.linalg.norm(lg - g["last"]) / np.linalg.norm(g["last"])
    assert rel < 1e-5, rel


def test_q8_0_fixture_dequant_matches_gguf_py(oracle_mod):
    """The oracle's Q8_0 dequant (gguf.rs:365-375) equals gguf-py's on a synthetic file's tensor."""
    import gguf

    path = synth.cached_model("130M", 0)
    r = gguf.GGUFReader(path)
    t = next(t for t in r.tensors if t.name == "blk.1.attn_qkv.weight")
    raw = np.asarray(t.data).view(np.uint8).ravel()
    n = int(np.prod(t.shape))
    ours = oracle_mod.dequant(8, raw, n)
    ref = gguf.quants.dequantize(np.asarray(t.data), gguf.GGMLQuantizationType.Q8_0).ravel()
    assert np.array_equal(ours.view(np.uint32), ref.astype(np.float32).view(np.uint32))


def test_requant_is_identity_on_full_range_blocks(oracle_mod):
    """quant.rs:78-102 applied to Q8_0 data whose blocks reach +-127 returns the same int8 codes and
    the f16 scale as f32 (the model weights' case); blocks without +-127 are rescaled."""
    rng = np.random.default_rng(0)
    q = rng.integers(-127, 128, (64, 256)).astype(np.float32)
    q[:, ::32] = 127.0  # every block holds +127
    d16 = (np.abs(rng.standard_normal((64, 8))) * 0.01).astype(np.float16).astype(np.float32)
    w = (q.reshape(64, 8, 32) * d16[:, :, None]).reshape(64, 256).astype(np.float32)
    qs, sc = oracle_mod.q8_quantize(w)
    assert np.array_equal(qs.astype(np.float32), q)
    assert np.array_equal(sc, d16)
    q2 = q.copy()
    q2[:, ::32] = 100.0
    q2 = np.clip(q2, -100, 100)
    w2 = (q2.reshape(64, 8, 32) * d16[:, :, None]).reshape(64, 256).astype(np.float32)
    qs2, sc2 = oracle_mod.q8_quantize(w2)
    assert np.abs(qs2).max() == 127 and not np.array_equal(sc2, d16)


def test_oracle_exp_pin(oracle_mod):
    """The oracle pins f32::exp to (float)exp((double)x); libm mode switches to glibc expf."""
    xs = np.linspace(-30, 30, 2001, dtype=np.float32)
    ours = np.array([oracle_mod.expf(float(x)) for x in xs], np.float32)
    ref = np.exp(xs.astype(np.float64)).astype(np.float32)
    assert np.array_equal(ours.view(np.uint32), ref.view(np.uint32))
    oracle_mod.set_exp_mode(True)
    try:
        libm = np.array([oracle_mod.expf(float(x)) for x in xs], np.float32)
    finally:
        oracle_mod.set_exp_mode(False)
    # glibc's expf differs from the correctly rounded value on a small fraction of inputs, by 1 ulp
    d = np.abs(libm.view(np.int32).astype(np.int64) - ours.view(np.int32).astype(np.int64))
    assert d.max() <= 1


def test_oracle_exp_choice_keeps_config1_tokens(oracle_mod):
    """The exp pin does not change config 1's greedy tokens (libm expf vs correctly rounded)."""
    path = synth.cached_model("130M", 0)
    ids = synth.prompt_ids(128, 1)
    eng = oracle_mod.Engine(path, quant=True)
    a, _, _, _ = eng.generate(ids, 32)
    oracle_mod.set_exp_mode(True)
    try:
        b, _, _, _ = eng.generate(ids, 32)
    finally:
        oracle_mod.set_exp_mode(False)
    assert list(a) == list(b)
