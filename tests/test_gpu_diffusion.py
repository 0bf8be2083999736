"""GPU parity of the diffusion decode through the C ABI, bit for bit against the oracle:
Model::run_block and forward_bidir (model.rs:441-587) and Engine::generate_diffusion
(lib.rs:211-495) on the cached and uncached paths, greedy, Gumbel, remasking and threshold."""
import numpy as np
import pytest

from hobbylm_b200 import DiffOpts, HgError, synth

pytestmark = pytest.mark.gpu
MASK = 50257


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def test_run_block_matches_oracle(engine130, oracle130):
    """A bidirectional block over a committed prefix: the logits of every row equal the oracle's,
    the sequence keeps its length until commit, and a rerun overwrites the block's K/V."""
    ids = synth.prompt_ids(40, 6)
    blk = [MASK] * 6 + list(synth.prompt_ids(10, 7))
    oc = oracle130.new_cache()
    with engine130.new_cache() as kv:
        assert engine130.run_block(kv, ids, n_logits=0, commit=True) is None
        oracle130.run_block(oc, ids, commit=True, want_logits=False)
        assert kv.len == 40
        for b in (blk, [MASK] * 16, blk):
            got = engine130.run_block(kv, b)
            ref = oracle130.run_block(oc, b)
            assert kv.len == 40
            assert np.array_equal(_bits(got), _bits(ref))
        engine130.run_block(kv, blk, n_logits=0, commit=True)
        oracle130.run_block(oc, blk, commit=True, want_logits=False)
        assert kv.len == 56
        got = engine130.run_block(kv, [MASK] * 8, n_logits=3)
        ref = oracle130.run_block(oc, [MASK] * 8)[-3:]
        assert np.array_equal(_bits(got), _bits(ref))


def test_canvas_pass_matches_forward_bidir(engine130, oracle130):
    """On an empty sequence a block is Model::forward_bidir (the uncached path's pass)."""
    ids = list(synth.prompt_ids(50, 8)) + [MASK] * 14
    with engine130.new_cache() as kv:
        got = engine130.run_block(kv, ids, n_logits=14)
        assert kv.len == 0
    ref = oracle130.forward_bidir(ids)[-14:]
    assert np.array_equal(_bits(got), _bits(ref))


@pytest.mark.parametrize("kw", [
    dict(),
    dict(cached=False),
    dict(temp=0.8, remask_steps=1, seed=9),
    dict(threshold=0.05),
    dict(cached=False, temp=0.7, steps=5, remask_steps=2, remask_frac=0.5, seed=3),
    dict(rep_penalty=1.0, steps=3),
])
def test_generate_diffusion_matches_oracle(engine130, oracle130, kw):
    ids = synth.prompt_ids(24, 11)
    opts = dict(gen_len=20, block=8, steps=8)
    opts.update(kw)
    ref = oracle130.generate_diffusion(ids, **opts)
    got = engine130.generate_diffusion(ids, DiffOpts(**opts))
    assert got == [int(t) for t in ref]


def test_generate_diffusion_streams_blocks_and_stops(engine130):
    ids = synth.prompt_ids(24, 11)
    o = DiffOpts(gen_len=24, block=8, steps=8)
    full = engine130.generate_diffusion(ids, o)
    if engine130.eos() in full[:16]:
        pytest.skip("eos inside the first two blocks")
    seen = []
    got = engine130.generate_diffusion(ids, o, on_block=lambda b: seen.append(b) or len(seen) < 2)
    assert len(seen) == 2 and seen[0] + seen[1] == got == full[:16]


def test_run_block_errors(engine130):
    with engine130.new_cache() as kv:
        for call, code in ((lambda: engine130.run_block(kv, [1] * 1025), -1),
                           (lambda: engine130.run_block(kv, [1, 2], n_logits=3), -1),
                           (lambda: engine130.run_block(kv, [60000]), -8)):
            with pytest.raises(HgError) as ei:
                call()
            assert ei.value.code == code
    with engine130.new_cache(max_ctx=20) as kv:
        with pytest.raises(HgError) as ei:
            engine130.run_block(kv, [1] * 21)
        assert ei.value.code == -7
        engine130.run_block(kv, [1] * 20, n_logits=1)
