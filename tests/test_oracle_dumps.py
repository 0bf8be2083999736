"""The oracle against its own committed greedy dumps for configs 1 and 4 (tests/golden/
make_oracle_dumps.py): ids and per-step logit digests, bit for bit, so any change to the oracle's
arithmetic shows up here before it can move the GPU parity target."""
import json
import os

import pytest

from hobbylm_b200 import synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
VALID = 50257


@pytest.mark.parametrize("name,steps", [("config1", None), ("config4", 48)])
def test_oracle_reproduces_its_greedy_dump(oracle_mod, name, steps):
    with open(os.path.join(GOLDEN, f"oracle_{name}_greedy.json")) as f:
        g = json.load(f)
    n = g["steps"] if steps is None else steps
    eng = oracle_mod.Engine(synth.cached_model(g["preset"], 0), quant=True)
    toks, logits, _, _ = eng.generate(synth.prompt_ids(g["prompt_len"], g["prompt_seed"]), n, want_logits=True)
    eng.close()
    assert [int(t) for t in toks] == g["tokens"][:n]
    assert [synth.tensor_digest(lg[:VALID]) for lg in logits] == g["logit_digests"][:n]
