"""CPU checks of the oracle's diffusion decode (hobby-rs model.rs:441-587, lib.rs:164-495): the
equivalences the GPU path is built on, and the determinism of the denoising loops."""
import numpy as np
import pytest

from hobbylm_b200 import synth


@pytest.fixture(scope="module")
def eng(oracle_mod):
    return oracle_mod.Engine(synth.cached_model("130M", 0), quant=True)


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def test_forward_bidir_is_run_block_on_an_empty_prefix(eng):
    """forward_bidir (model.rs:441-470) and run_block at base 0 (model.rs:472-510) take the same
    arithmetic: the GPU's uncached path runs the canvas as one block at position 0."""
    ids = synth.prompt_ids(21, 3)
    c = eng.new_cache()
    assert np.array_equal(_bits(eng.forward_bidir(ids)), _bits(eng.run_block(c, ids)))


def test_run_block_is_non_destructive_until_commit(eng):
    ids = synth.prompt_ids(10, 4)
    blk = [50257] * 5 + [11, 12, 13]
    c = eng.new_cache()
    eng.run_block(c, ids, commit=True, want_logits=False)
    assert len(c) == 10
    a = eng.run_block(c, blk)
    eng.run_block(c, [7] * 8)
    b = eng.run_block(c, blk)
    assert len(c) == 10 and np.array_equal(_bits(a), _bits(b))
    eng.run_block(c, blk, commit=True, want_logits=False)
    assert len(c) == 18


def test_one_row_block_keys_equal_causal_prefill(eng):
    """A block of one row attends to the prefix and itself: the causal prefill attention at that
    position, so the K/V it commits equal a one-token prefill's at every layer."""
    ids = synth.prompt_ids(17, 5)
    a, b = eng.new_cache(), eng.new_cache()
    eng.prefill(a, ids[:16])
    eng.prefill(b, ids[:16])
    eng.prefill(a, ids[16:])
    eng.run_block(b, ids[16:], commit=True, want_logits=False)
    for li in range(eng.cfg["n_layers"]):
        ka, va = a.layer(li)
        kb, vb = b.layer(li)
        assert np.array_equal(_bits(ka), _bits(kb)) and np.array_equal(_bits(va), _bits(vb)), li


def test_diffusion_config_defaults(eng):
    assert (eng.cfg["diffusion"], eng.cfg["mask_token_id"], eng.cfg["block_size"]) == (0, 50257, 32)


@pytest.mark.parametrize("kw", [dict(), dict(cached=False), dict(temp=0.8, remask_steps=1, seed=9),
                                dict(threshold=0.05)])
def test_generate_diffusion_is_deterministic(eng, kw):
    ids = synth.prompt_ids(12, 5)
    a = eng.generate_diffusion(ids, gen_len=16, block=8, steps=8, **kw)
    b = eng.generate_diffusion(ids, gen_len=16, block=8, steps=8, **kw)
    assert list(a) == list(b) and len(a) <= 16
    assert all(t < 50257 for t in a)


def test_gumbel_sampling_depends_on_the_seed(eng):
    ids = synth.prompt_ids(12, 5)
    a = eng.generate_diffusion(ids, gen_len=16, block=8, steps=8, temp=1.0, seed=1)
    b = eng.generate_diffusion(ids, gen_len=16, block=8, steps=8, temp=1.0, seed=2)
    g = eng.generate_diffusion(ids, gen_len=16, block=8, steps=8)
    assert list(a) != list(b) and list(a) != list(g)
