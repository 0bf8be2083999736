"""End-to-end parity of the decode engine against the CPU oracle (configs 1 and 4).

Both prefill and decode follow the reference's arithmetic order (sequential sums where hobby-rs
sums sequentially), so logits must be bit-identical to the oracle at every step; the north-star
tolerance (1e-3 relative L2) is also asserted so a failure shows its size. Greedy tokens and
router selections must be identical.
"""
import numpy as np
import pytest

from hobbylm_b200 import GenOpts, HgError, synth

pytestmark = pytest.mark.gpu

TOL_REL_L2 = 1e-3


def _rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_prefill_bitexact_config1(engine130, oracle130):
    ids = synth.prompt_ids(128, 1)
    with engine130.new_cache() as kv:
        lg = engine130.prefill(kv, ids)
        assert kv.len == 128
    oc = oracle130.new_cache()
    ref = oracle130.prefill(oc, ids)
    assert np.array_equal(lg.view(np.uint32), ref.view(np.uint32)), f"rel {_rel(lg, ref)}"


def test_prefill_chunked_equals_whole(engine130):
    ids = synth.prompt_ids(4400, 7)  # spans two 4096-row prefill chunks
    with engine130.new_cache() as a, engine130.new_cache() as b:
        whole = engine130.prefill(a, ids)
        engine130.prefill(b, ids[:300])
        split = engine130.prefill(b, ids[300:])
        assert np.array_equal(whole.view(np.uint32), split.view(np.uint32))


def test_device_greedy_equals_host_loop(engine130):
    """hg_decode_greedy (argmax fed back on the device) equals step-by-step hg_decode_batch."""
    prompts = [synth.prompt_ids(n, 40 + n) for n in (33, 80, 150)]
    ca = [engine130.new_cache() for _ in prompts]
    cb = [engine130.new_cache() for _ in prompts]
    t0 = []
    for p, a, b in zip(prompts, ca, cb):
        la = engine130.prefill(a, p)
        engine130.prefill(b, p)
        la[50257:] = -np.inf
        t0.append(int(np.argmax(la)))
    dev = engine130.decode_greedy(ca, t0, 70)  # crosses the 64-step id ring
    toks = list(t0)
    for k in range(70):
        nxt, _ = engine130.decode_batch(cb, toks)
        assert [int(v) for v in nxt] == [int(v) for v in dev[k]], f"step {k}"
        toks = [int(v) for v in nxt]
    assert [c.len for c in ca] == [c.len for c in cb]
    for c in ca + cb:
        c.close()


def test_greedy_decode_config1(engine130, oracle130):
    """Config 1: 130M, 128-token prompt (seed 1), 128 greedy tokens; identical tokens, per-step
    logits within 1e-3 relative L2, identical expert selection at every MoE layer."""
    ids = synth.prompt_ids(128, 1)
    steps = 128
    ref_toks, ref_logits, _, _ = oracle130.generate(ids, steps, want_logits=True)
    assert len(ref_toks) == steps
    oc = oracle130.new_cache()
    oracle130.prefill(oc, ids)
    with engine130.new_cache() as kv:
        lg = engine130.prefill(kv, ids)
        worst, sel_mismatch = 0.0, 0
        for i in range(steps):
            lm = lg.copy()
            lm[50257:] = -np.inf
            tok = int(np.argmax(lm))
            assert tok == ref_toks[i], f"step {i}: token {tok} != {ref_toks[i]}"
            rel = _rel(lg[:50257], ref_logits[i][:50257])  # the oracle records masked logits
            worst = max(worst, rel)
            assert rel < TOL_REL_L2, f"step {i}: rel L2 {rel}"
            assert np.array_equal(lg[:50257].view(np.uint32), ref_logits[i][:50257].view(np.uint32)), \
                f"step {i}: logits not bit-identical (rel L2 {rel:.2e})"
            lg, nxt = engine130.forward(kv, tok)
            oracle130.forward(oc, tok, 128 + i)
            gsel = engine130.last_routing()
            osel, _ = oracle130.last_routing()
            sel_mismatch += int((gsel != osel).any())
        print(f"worst per-step rel L2 {worst:.3e}")
        assert sel_mismatch == 0, f"{sel_mismatch} steps with a different expert selection"


def test_generate_api_matches_oracle(engine130, oracle130):
    ids = synth.prompt_ids(64, 11)
    got = []
    n = engine130.generate(ids, GenOpts(max_new=40), on_token=lambda t: got.append(t) or True)
    ref, _, _, _ = oracle130.generate(ids, 40)
    assert n == list(ref) and got == list(ref)
    # the callback can stop generation (lib.rs:152)
    stop = engine130.generate(ids, GenOpts(max_new=40), on_token=lambda t: False)
    assert len(stop) == 1


@pytest.mark.parametrize("temp,top_p,rep", [(0.8, 0.9, 1.3), (1.0, 1.0, 1.0), (0.0, 0.9, 1.5), (0.7, 0.5, 1.0)])
def test_sampling_matches_oracle(engine130, oracle130, temp, top_p, rep):
    """Temperature / top-p sampling and the repetition penalty (sample.rs, lib.rs:125-142) drawn on
    the GPU from the step's logits, with the RNG state on the device: the same ids as the oracle,
    through the nucleus, the plain draw and the penalised argmax."""
    ids = synth.prompt_ids(32, 5)
    o = GenOpts(max_new=24, temp=temp, top_p=top_p, seed=77, rep_penalty=rep)
    got = engine130.generate(ids, o)
    ref, _, _, _ = oracle130.generate(ids, 24, temp=temp, top_p=top_p, seed=77, rep_penalty=rep)
    assert got == list(ref)


def test_batched_decode_equals_single(engine130):
    prompts = [synth.prompt_ids(n, 20 + n) for n in (40, 97, 130, 64)]
    caches_b = [engine130.new_cache() for _ in prompts]
    caches_s = [engine130.new_cache() for _ in prompts]
    toks = []
    for p, cb, cs in zip(prompts, caches_b, caches_s):
        l1 = engine130.prefill(cb, p)
        engine130.prefill(cs, p)
        l1[50257:] = -np.inf
        toks.append(int(np.argmax(l1)))
    tb = list(toks)
    ts = list(toks)
    for _ in range(6):
        nb, lb = engine130.decode_batch(caches_b, tb, want_logits=True)
        for i, c in enumerate(caches_s):
            ls, n1 = engine130.forward(c, ts[i])
            assert np.array_equal(ls.view(np.uint32), lb[i].view(np.uint32))
            ts[i] = n1
        tb = [int(v) for v in nb]
        assert tb == ts
    for c in caches_b + caches_s:
        c.close()


def test_wide_batch_equals_single(model130):
    """48 sequences fill enough (token, kv head) CTAs for the split softmax / value-sum kernels;
    each row must equal the one-sequence path bit for bit (lengths cross page, 64-position chunk
    and 1024-position softmax chunk boundaries)."""
    from hobbylm_b200 import Engine

    lens = [1, 15, 16, 17, 63, 64, 65, 127, 1023, 1024, 1025, 2100] + [30 + 37 * i for i in range(36)]
    eng = Engine.load(model130, max_batch=96, kv_pool_tokens=80000)
    try:
        prompts = [synth.prompt_ids(n, 500 + i) for i, n in enumerate(lens)]
        cb = [eng.new_cache() for _ in prompts]
        cs = [eng.new_cache() for _ in prompts]
        toks = []
        for p, a, b in zip(prompts, cb, cs):
            la = eng.prefill(a, p)
            eng.prefill(b, p)
            la[50257:] = -np.inf
            toks.append(int(np.argmax(la)))
        tb, ts = list(toks), list(toks)
        for _ in range(3):
            nb, lb = eng.decode_batch(cb, tb, want_logits=True)
            for i, c in enumerate(cs):
                ls, n1 = eng.forward(c, ts[i])
                assert np.array_equal(ls.view(np.uint32), lb[i].view(np.uint32)), (i, lens[i])
                ts[i] = n1
            tb = [int(v) for v in nb]
            assert tb == ts
        for c in cb + cs:
            c.close()
    finally:
        eng.close()


def test_engine_freed_before_its_caches(model130):
    """Sequences left open when their engine is freed can still be closed (no use after free)."""
    from hobbylm_b200 import Engine

    eng = Engine.load(model130, max_batch=2)
    a, b = eng.new_cache(), eng.new_cache()
    eng.prefill(a, [1, 2, 3])
    eng.close()
    assert a.len == 3
    a.close()
    b.close()


def test_prefill_embeds_splice_matches_oracle(engine130, oracle130, model130, native):
    """Model::prefill on caller rows (model.rs:340; lib.rs:118-121 splices modality rows before the
    prompt's token embeddings): the token-embedding rows of a prompt give its ids' logits, and three
    spliced rows + the prompt, then greedy decode, equal the oracle bit for bit."""
    ids = synth.prompt_ids(40, 9)
    d, vocab = engine130.cfg["d_model"], engine130.vocab
    emb = np.empty(vocab * d, np.float32)
    native.check(native.lib().hg_gguf_tensor_f32(str(model130).encode(), b"token_embd.weight", emb.ctypes.data, emb.size))
    emb = emb.reshape(vocab, d)
    with engine130.new_cache() as a, engine130.new_cache() as b:
        la = engine130.prefill(a, ids)
        lb = engine130.prefill_embeds(b, emb[ids])
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    extra = (np.random.default_rng(11).standard_normal((3, d)) * 0.02).astype(np.float32)
    oc = oracle130.new_cache()
    ref = oracle130.prefill_embeds(oc, np.concatenate([extra, emb[ids]]))
    with engine130.new_cache() as kv:
        engine130.prefill_embeds(kv, extra)
        lg = engine130.prefill(kv, ids)
        n = kv.len
        assert n == 3 + len(ids)
        for i in range(8):
            assert np.array_equal(lg.view(np.uint32), ref.view(np.uint32)), f"step {i}: rel L2 {_rel(lg, ref)}"
            lm = lg.copy()
            lm[50257:] = -np.inf
            tok = int(np.argmax(lm))
            lg, _ = engine130.forward(kv, tok)
            ref = oracle130.forward(oc, tok, n + i)


def test_forward_x_matches_forward_and_oracle(engine130, oracle130, model130, native):
    """Model::forward_x (model.rs:160): a decode step from a token's own embedding row equals the step
    from its id, and steps from arbitrary rows between token steps equal the oracle bit for bit."""
    ids = synth.prompt_ids(30, 13)
    d, vocab = engine130.cfg["d_model"], engine130.vocab
    emb = np.empty(vocab * d, np.float32)
    native.check(native.lib().hg_gguf_tensor_f32(str(model130).encode(), b"token_embd.weight", emb.ctypes.data, emb.size))
    emb = emb.reshape(vocab, d)
    rows = (np.random.default_rng(17).standard_normal((2, d)) * 0.02).astype(np.float32)
    oc = oracle130.new_cache()
    oracle130.prefill(oc, ids)
    with engine130.new_cache() as a, engine130.new_cache() as b:
        engine130.prefill(a, ids)
        engine130.prefill(b, ids)
        la, na = engine130.forward(a, 1234)
        lb, nb = engine130.forward_x(b, emb[1234])
        assert na == nb and np.array_equal(la.view(np.uint32), lb.view(np.uint32))
        ref = oracle130.forward(oc, 1234, len(ids))
        assert np.array_equal(lb.view(np.uint32), ref.view(np.uint32))
        pos, tok = len(ids) + 1, nb
        for step in range(6):
            if step in (1, 4):
                lg, nxt = engine130.forward_x(b, rows[0 if step == 1 else 1])
                ref = oracle130.forward_x(oc, rows[0 if step == 1 else 1], pos)
            else:
                lg, nxt = engine130.forward(b, tok)
                ref = oracle130.forward(oc, tok, pos)
            assert np.array_equal(lg.view(np.uint32), ref.view(np.uint32)), f"step {step}: rel L2 {_rel(lg, ref)}"
            pos, tok = pos + 1, nxt


def test_generate_with_embeds_matches_oracle(engine130, oracle130):
    """Engine::generate with `embeds` (lib.rs:107-126): caller rows before the prompt ids, greedy and
    sampled, and rows alone, token for token against the oracle's single prefill over all inputs."""
    d = engine130.cfg["d_model"]
    rows = (np.random.default_rng(31).standard_normal((3, d)) * 0.02).astype(np.float32)
    ids = synth.prompt_ids(20, 32)
    for o in (GenOpts(max_new=12), GenOpts(max_new=12, temp=0.8, top_p=0.9, seed=5, rep_penalty=1.2)):
        ref = oracle130.generate_embeds(rows, ids, o.max_new, o.temp, o.top_p, o.seed, o.rep_penalty)
        assert engine130.generate(ids, o, embeds=rows) == [int(t) for t in ref]
    ref = oracle130.generate_embeds(rows, [], 6)
    assert engine130.generate([], GenOpts(max_new=6), embeds=rows) == [int(t) for t in ref]


def test_errors(engine130, model130):
    from hobbylm_b200 import Engine

    with engine130.new_cache() as kv:
        with pytest.raises(HgError) as ei:
            engine130.prefill(kv, [60000])
        assert ei.value.code == -8
        engine130.prefill(kv, [1, 2, 3])
        with pytest.raises(HgError) as ei:
            engine130.forward(kv, 50304)
        assert ei.value.code == -8
    with engine130.new_cache(max_ctx=20) as kv:
        engine130.prefill(kv, list(range(19)))
        engine130.forward(kv, 5)
        with pytest.raises(HgError) as ei:
            engine130.forward(kv, 5)
        assert ei.value.code == -7
    small = Engine.load(model130, kv_pool_tokens=64)
    try:
        with small.new_cache() as kv:
            small.prefill(kv, list(range(60)))
            with pytest.raises(HgError) as ei:
                small.prefill(kv, list(range(20)))
            assert ei.value.code == -6
    finally:
        small.close()


@pytest.mark.slow
def test_greedy_decode_config4(model500, oracle_mod):
    """Config 4 (500M, 2048-token prompt, seed 4): prefill bit-exact, the first 128 greedy tokens
    identical, per-step logits within 1e-3 relative L2."""
    from hobbylm_b200 import Engine

    ids = synth.prompt_ids(2048, 4)
    steps = 128
    ora = oracle_mod.Engine(model500, quant=True)
    ref_toks, ref_logits, _, _ = ora.generate(ids, steps, want_logits=True)
    eng = Engine.load(model500)
    try:
        with eng.new_cache() as kv:
            lg = eng.prefill(kv, ids)
            v = 50257
            assert np.array_equal(lg[:v].view(np.uint32), ref_logits[0][:v].view(np.uint32))
            for i in range(steps):
                lm = lg.copy()
                lm[v:] = -np.inf
                tok = int(np.argmax(lm))
                assert tok == ref_toks[i], f"step {i}"
                assert _rel(lg[:v], ref_logits[i][:v]) < TOL_REL_L2
                assert np.array_equal(lg[:v].view(np.uint32), ref_logits[i][:v].view(np.uint32)), f"step {i}"
                lg, _ = eng.forward(kv, tok)
    finally:
        eng.close()


def _oracle_prefills(ora, prompts):
    caches, logits = [], []
    for p in prompts:
        c = ora.new_cache()
        logits.append(ora.prefill(c, p))
        caches.append(c)
    return caches, logits


def _masked_argmax(lg):
    lm = lg.copy()
    lm[50257:] = -np.inf
    return int(np.argmax(lm))


def _batched_vs_oracle(model, oracle_mod, n_seqs, lo, hi, seed, steps, greedy_steps):
    """n_seqs sequences of the model (prompt lengths U[lo, hi]) prefilled on the GPU and by the
    oracle, then `steps` batched decode steps through hg_decode_batch with every sequence's logits
    and next id bit-compared with the oracle's one-sequence Model::forward, then `greedy_steps`
    device-driven steps (hg_decode_greedy) whose ids must equal the oracle's greedy ids."""
    from hobbylm_b200 import Engine

    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi + 1, n_seqs)
    prompts = [synth.prompt_ids(int(n), seed * 1000 + i) for i, n in enumerate(lens)]
    ora = oracle_mod.Engine(model, quant=True)
    eng = Engine.load(model, max_batch=n_seqs, kv_pool_tokens=int(lens.sum()) + n_seqs * (steps + greedy_steps + 32))
    caches = []
    try:
        ocs, olg = _oracle_prefills(ora, prompts)
        toks = []
        for i, p in enumerate(prompts):
            c = eng.new_cache()
            caches.append(c)
            lg = eng.prefill(c, p)
            assert np.array_equal(lg.view(np.uint32), olg[i].view(np.uint32)), f"prefill seq {i}"
            toks.append(_masked_argmax(lg))
        for step in range(steps):
            nb, lb = eng.decode_batch(caches, toks, want_logits=True)
            for i in range(n_seqs):
                ref = ora.forward(ocs[i], toks[i], int(lens[i]) + step)
                assert np.array_equal(lb[i].view(np.uint32), ref.view(np.uint32)), \
                    f"step {step} seq {i} (context {int(lens[i]) + step}): rel L2 {_rel(lb[i], ref)}"
                assert int(nb[i]) == _masked_argmax(ref), f"step {step} seq {i}: next id"
            toks = [int(v) for v in nb]
        if greedy_steps:
            dev = eng.decode_greedy(caches, toks, greedy_steps)
            for i in range(n_seqs):
                t = toks[i]
                for k in range(greedy_steps):
                    t = _masked_argmax(ora.forward(ocs[i], t, int(lens[i]) + steps + k))
                    assert int(dev[k][i]) == t, f"greedy step {k} seq {i}"
        for c in ocs:
            c.close()
    finally:
        for c in caches:
            c.close()
        eng.close()
        ora.close()


def test_batched_500m_large_batch_kernels_match_oracle(model500, oracle_mod):
    """The 500M engine with 80 sequences (240 (token, kv head) pairs: the large-batch attention
    kernels on the engine's layered KV pool, head_dim 128), prompts of 64-300 ids: 8 batched steps
    bit-identical to the oracle sequence by sequence, then 4 device-driven greedy steps."""
    _batched_vs_oracle(model500, oracle_mod, 80, 64, 300, 81, 8, 4)


@pytest.mark.slow
def test_batched_500m_config5_batch_matches_oracle(model500, oracle_mod):
    """The config-5 batch size (256 sequences, the step graph without programmatic launches, the
    lm_head's 64-token chunks, expert groups of many entries) on short prompts (8-64 ids): 4
    batched steps bit-identical to the oracle sequence by sequence, then 2 greedy steps."""
    _batched_vs_oracle(model500, oracle_mod, 256, 8, 64, 82, 4, 2)


# The 1B preset's attention and expert shapes (hobbylm/config.py:130-134: d 1024, 16 q / 8 kv heads
# of 128, GQA group 2, 64 experts top-8 of width 224, dense 2816) on two layers, so the model stays
# small enough to generate and check quickly.
PRESET_1B_2L = synth.Preset(1024, 2, 1, 16, 8, 128, 2816, 224, 64, 8, 1)


@pytest.fixture(scope="module")
def model1b2l():
    return synth.cached_model(PRESET_1B_2L, 0)


def test_gqa_group2_1b_shapes_match_oracle(model1b2l, oracle_mod):
    """A GQA group-2 model with the 1B preset's widths: prefill, then batch 1 (the small-batch
    kernels) and batch 30 (240 (token, kv head) pairs: the large-batch kernels) bit-identical to
    the oracle, then device-driven greedy ids."""
    _batched_vs_oracle(model1b2l, oracle_mod, 1, 40, 40, 91, 12, 8)
    _batched_vs_oracle(model1b2l, oracle_mod, 30, 16, 80, 92, 6, 4)
