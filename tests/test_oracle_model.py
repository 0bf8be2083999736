"""CPU self-consistency of the oracle's model paths (hobby-rs model.rs:152-184, 340-439), the
properties the GPU parity tests also assert of the CUDA path."""
import numpy as np
import pytest

from hobbylm_b200 import synth


@pytest.fixture(scope="module")
def eng(oracle_mod):
    return oracle_mod.Engine(synth.cached_model("130M", 0), quant=True)


@pytest.fixture(scope="module")
def emb(native, eng):
    path = synth.cached_model("130M", 0)
    d, vocab = eng.cfg["d_model"], eng.vocab
    out = np.empty(vocab * d, np.float32)
    native.check(native.lib().hg_gguf_tensor_f32(path.encode(), b"token_embd.weight", out.ctypes.data, out.size))
    return out.reshape(vocab, d)


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def test_forward_x_of_the_embedding_row_is_forward(eng, emb):
    """Model::forward is forward_x of the token's embedding row (model.rs:152-160)."""
    ids = synth.prompt_ids(20, 21)
    a, b = eng.new_cache(), eng.new_cache()
    eng.prefill(a, ids)
    eng.prefill(b, ids)
    for i, tok in enumerate([5, 777, 50000]):
        la = eng.forward(a, tok, 20 + i)
        lb = eng.forward_x(b, emb[tok], 20 + i)
        assert np.array_equal(_bits(la), _bits(lb))


def test_prefill_of_embedding_rows_is_prefill_of_ids(eng, emb):
    """Engine::generate feeds prefill the token embeddings (lib.rs:118-126)."""
    ids = synth.prompt_ids(33, 22)
    a, b = eng.new_cache(), eng.new_cache()
    assert np.array_equal(_bits(eng.prefill(a, ids)), _bits(eng.prefill_embeds(b, emb[ids])))


def test_chunked_prefill_equals_one_prefill(eng):
    """Rows are independent in the prefill matmuls and each row's attention reads keys 0..pos, so
    prefilling in two calls gives the same logits and cache as one call."""
    ids = synth.prompt_ids(40, 23)
    a, b = eng.new_cache(), eng.new_cache()
    la = eng.prefill(a, ids)
    eng.prefill(b, ids[:17])
    lb = eng.prefill(b, ids[17:])
    assert np.array_equal(_bits(la), _bits(lb))
    for li in (0, eng.cfg["n_layers"] - 1):
        ka, va = a.layer(li)
        kb, vb = b.layer(li)
        assert np.array_equal(_bits(ka), _bits(kb)) and np.array_equal(_bits(va), _bits(vb))


def test_generate_is_prefill_then_greedy_forward(eng):
    """Engine::generate at temp 0 (lib.rs:107-162): masked argmax of the prefill logits, then of
    each forward step, stopping on eos."""
    ids = synth.prompt_ids(16, 24)
    toks, _, _, _ = eng.generate(ids, 6)
    c = eng.new_cache()
    lg = eng.prefill(c, ids)
    out = []
    for i in range(6):
        lg[50257:] = -np.inf
        t = int(np.argmax(lg))
        if t == eng.cfg["eos"]:
            break
        out.append(t)
        lg = eng.forward(c, t, 16 + i)
    assert list(toks) == out


def test_config2_router_margins_are_logged(oracle_mod, record_property):
    """The top-k cut of config 2's router (model.rs:270-293): the gap between the 6th and 7th
    selection scores of every token is recorded (a GPU/oracle selection flip on a near-tie can be
    told apart from a real fault) and is never an exact tie, where sort order would decide."""
    inp = synth.moe_op_inputs(seed=2, T=256)
    moe = oracle_mod.Moe(inp["router"], inp["bias"], inp["gate_exps"], inp["up_exps"], inp["down_exps"],
                         inp["gate_sh"], inp["up_sh"], inp["down_sh"], top_k=6)
    margins = []
    for x in inp["x"]:
        s = np.sort(moe.sel_scores(x))[::-1]
        margins.append(float(s[5] - s[6]))
    record_property("min_top6_top7_margin", min(margins))
    record_property("median_top6_top7_margin", float(np.median(margins)))
    print(f"config 2 router: min top-6/7 margin {min(margins):.3e}, median {np.median(margins):.3e}")
    assert min(margins) > 0.0


def test_generate_with_embedding_rows_is_generate_of_ids(eng, emb):
    """lib.rs:118-121: `embeds` rows that are the prompt's own token embeddings, ahead of the rest of
    the prompt (or instead of it), generate exactly what the ids do."""
    ids = synth.prompt_ids(16, 25)
    a, _, _, _ = eng.generate(ids, 8, rep_penalty=1.3)
    b = eng.generate_embeds(emb[ids[:5]], ids[5:], 8, rep_penalty=1.3)
    c = eng.generate_embeds(emb[ids], [], 8, rep_penalty=1.3)
    assert list(a) == list(b) == list(c)
