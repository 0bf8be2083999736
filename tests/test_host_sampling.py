"""Host-side token selection of the library (hg_host_sample, hg_host_score_block) against the
oracle's restatement of sample.rs:3-112 and lib.rs:221-263, bit for bit, including the advanced
xorshift64* state. No GPU."""
import ctypes as C

import numpy as np
import pytest

VOCAB, VALID, MASK = 50304, 50257, 50257


def _logits(rng, n, kind):
    if kind == "normal":
        x = rng.standard_normal(n).astype(np.float32) * 3
    elif kind == "flat":
        x = rng.standard_normal(n).astype(np.float32) * 0.01
    else:  # coarse values: many exact ties, so the order of equal probabilities matters
        x = np.round(rng.standard_normal(n) * 2).astype(np.float32)
    x[VALID:] = -np.inf
    return x


def _lib_sample(native, x, temp, top_p, state):
    st, out = C.c_uint64(state), C.c_uint32()
    native.check(native.lib().hg_host_sample(x.ctypes.data, len(x), temp, top_p, C.byref(st), C.byref(out)))
    return int(out.value), int(st.value)


@pytest.mark.parametrize("kind", ["normal", "flat", "ties"])
def test_host_sample_matches_oracle(native, oracle_mod, kind):
    rng = np.random.default_rng({"normal": 1, "flat": 2, "ties": 3}[kind])
    for temp, top_p in [(0.0, 0.9), (0.8, 0.95), (1.0, 0.0), (1.3, 1.0), (0.5, 0.5), (2.0, 0.99)]:
        x = _logits(rng, VOCAB, kind)
        s_lib = s_ora = 1234
        for _ in range(4):  # chained draws: the state must advance identically
            a, s_lib = _lib_sample(native, x, temp, top_p, s_lib)
            b, s_ora = oracle_mod.sample(x, temp, top_p, s_ora)
            assert (a, s_lib) == (b, s_ora), (kind, temp, top_p)


@pytest.mark.parametrize("temp,rep", [(0.0, 1.4), (0.8, 1.4), (0.0, 1.0), (1.2, 1.0)])
def test_host_score_block_matches_oracle(native, oracle_mod, temp, rep):
    rng = np.random.default_rng(int(temp * 10 + rep * 100))
    blk_len = 16
    logits = np.stack([_logits(rng, VOCAB, "normal") for _ in range(blk_len)])
    blk = rng.integers(0, VALID, blk_len).astype(np.uint32)
    blk[::3] = MASK
    committed = rng.integers(0, VALID, 40).astype(np.uint32)
    pred = np.zeros(blk_len, np.uint32)
    pconf = np.zeros(blk_len, np.float32)
    cconf = np.zeros(blk_len, np.float32)
    st = C.c_uint64(99)
    native.check(native.lib().hg_host_score_block(logits.ctypes.data, VOCAB, blk.ctypes.data, blk_len,
                                                  committed.ctypes.data, len(committed), MASK, rep, temp,
                                                  C.byref(st), pred.ctypes.data, pconf.ctypes.data, cconf.ctypes.data))
    rp, rpc, rcc, rst = oracle_mod.score_block(logits, blk, committed, MASK, rep, temp, 99)
    assert np.array_equal(pred, rp)
    assert np.array_equal(pconf.view(np.uint32), rpc.view(np.uint32))
    assert np.array_equal(cconf.view(np.uint32), rcc.view(np.uint32))
    assert int(st.value) == rst
    assert np.all(cconf[::3] == 0.0)  # a [MASK] row's current id is banned: probability 0


def test_host_sampling_errors(native):
    lib = native.lib()
    st, out = C.c_uint64(1), C.c_uint32()
    assert lib.hg_host_sample(None, 10, 1.0, 0.9, C.byref(st), C.byref(out)) == -1
    x = np.zeros((1, 8), np.float32)
    blk = np.array([9], np.uint32)
    p, f1, f2 = np.zeros(1, np.uint32), np.zeros(1, np.float32), np.zeros(1, np.float32)
    assert lib.hg_host_score_block(x.ctypes.data, 8, blk.ctypes.data, 1, None, 0, 7, 1.0, 0.0, C.byref(st),
                                   p.ctypes.data, f1.ctypes.data, f2.ctypes.data) == -8


def test_generate_embeds_binding_rejects_null_engine(native):
    """hg_generate_embeds checks its arguments before any GPU work (the call works without a GPU)."""
    rows = np.zeros((2, 8), np.float32)
    out = np.zeros(4, np.uint32)
    rc = native.lib().hg_generate_embeds(None, rows.ctypes.data, 2, None, 0, None, native.TOKEN_CB(lambda t, u: 1),
                                         None, out.ctypes.data)
    assert rc == -1 and b"null argument" in native.lib().hg_last_error()


@pytest.mark.parametrize("case", ["one_finite", "tiny_top_p", "huge_temp", "n1"])
def test_host_sample_edge_cases_match_oracle(native, oracle_mod, case):
    rng = np.random.default_rng(11)
    x = _logits(rng, VOCAB, "normal")
    temp, top_p = 0.8, 0.9
    if case == "one_finite":
        x[:] = -np.inf
        x[4242] = 1.0
    elif case == "tiny_top_p":
        top_p = 1e-7
    elif case == "huge_temp":
        temp = 1e6
    else:
        x = np.array([0.5], np.float32)
    s_lib = s_ora = 7
    for _ in range(3):
        a, s_lib = _lib_sample(native, x, temp, top_p, s_lib)
        b, s_ora = oracle_mod.sample(x, temp, top_p, s_ora)
        assert (a, s_lib) == (b, s_ora), case
    if case == "one_finite":
        assert a == 4242
