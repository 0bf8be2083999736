"""hobbylm_b200 — a B200 (sm_100a) decode engine for hobbylm GGUF models, the hobby-rs decode path.

    from hobbylm_b200 import Engine, GenOpts
    eng = Engine.load("model.gguf")
    ids = eng.generate(prompt_ids, GenOpts(max_new=64))

The compute runs in libhobbygpu.so (hand-written CUDA for sm_100a behind the C ABI in
include/hobbygpu.h); this package is the host-side mirror of hobby-rs's Engine / KvCache API.
"""
from .engine import GPT2_VALID, DiffOpts, Engine, GenOpts, KvCache  # noqa: F401
from ._native import HgError  # noqa: F401
