"""Generate the oracle's golden greedy dumps for configs 1 and 4 (tokens and per-step logit digests).

    python tests/golden/make_oracle_dumps.py

Config 1: the 130M Q8_0 model (seed 0), a 128-id prompt (seed 1), 128 greedy steps. Config 4: the
500M Q8_0 model (seed 0), a 2048-id prompt (seed 4), 512 greedy steps. For each step the file holds
the generated id and the sha256 (first 32 hex digits) of that step's logits over ids < 50257 as f32
bytes, the logits the id was chosen from (step 0: the prefill's). tests/test_oracle_dumps.py checks
that the oracle still reproduces them bit for bit, so a change to the oracle cannot go unnoticed.
"""
from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

VALID = 50257
CASES = {"config1": ("130M", 128, 1, 128), "config4": ("500M", 2048, 4, 512)}


def dump(preset: str, prompt_len: int, seed: int, steps: int) -> dict:
    import oracle
    from hobbylm_b200 import synth

    eng = oracle.Engine(synth.cached_model(preset, 0), quant=True)
    ids = synth.prompt_ids(prompt_len, seed)
    toks, logits, _, _ = eng.generate(ids, steps, want_logits=True)
    eng.close()
    return {"preset": preset, "prompt_len": prompt_len, "prompt_seed": seed, "steps": steps,
            "tokens": [int(t) for t in toks], "logit_digests": [synth.tensor_digest(lg[:VALID]) for lg in logits]}


def main():
    for name, case in CASES.items():
        d = dump(*case)
        with open(os.path.join(HERE, f"oracle_{name}_greedy.json"), "w") as f:
            json.dump(d, f)
        print(name, len(d["tokens"]), "tokens")


if __name__ == "__main__":
    main()
