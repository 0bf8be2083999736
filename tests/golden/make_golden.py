"""Generate the golden fixtures that pin the synthetic-model producer and the oracle's semantics.

Run here (where the reference checkout is readable), never on the GPU box:

    python tests/golden/make_golden.py --reference /path/to/HobbyLM

It imports the reference's own Python code and writes, under tests/golden/:

* synth_digests_{130M,500M,1B}.json — per-tensor sha256 (f32 row-major bytes) of the F32 GGUF written by
  the reference exporter (export/to_gguf.py:38-133) from ``MoETransformer(get_config(preset))``
  after ``torch.manual_seed(0)`` (hobbylm/model.py:259-313). The exporter's HF-hub tokenizer download
  (to_gguf.py:18-35) is replaced by placeholder tokens, and the 130M preset (no shared expert) gets
  zero shared-expert tensors in its checkpoint so the exporter's unconditional shared-expert export
  (to_gguf.py:126-129) can run.
* torch_logits_130M.npz — the reference PyTorch model's f32 logits (hobbylm/model.py:322-356, MoE
  ``expert_backend="bmm"``, hobbylm/moe.py:121-135) for a 12-token prompt (ids from
  ``torch.Generator().manual_seed(1)``): the full last-position row plus per-position top-8 ids,
  values and logsumexp. hobby-rs reads rms_eps from GGUF metadata while the PyTorch RMSNorm uses
  1e-6, so the oracle is compared on a file written with rms_eps=1e-6.
* torch_bidir_logits_130M.npz — the same model with ``cfg.diffusion = True``, whose attention is
  bidirectional (hobbylm/model.py:225-226; the flag changes nothing else at inference), on an
  18-position canvas: 12 prompt ids (seed 1) then 6 [MASK] ids (50257, hobbylm/config.py:48):
  per-position top-8 ids, values and logsumexp, and the full rows of positions 0, 12 and 17.
  This is the reference for Model::forward_bidir (hobby-rs model.rs:441-470).
* torch_diffusion_generate_130M.json — the reference's own greedy denoising sampler
  (hobbylm/diffusion.py:92-176: num_transfer schedule, presence penalty, confidence-ordered
  commits, low-confidence remasking, each pass over the canvas prefix x[:b1]) on that model after
  the 12-id prompt, for three option sets. hobby-rs's uncached path (lib.rs:409-495) runs the same
  loop; at temperature 0 no random draws are involved, so its ids must equal these.
* torch_embeds_logits_130M.npz — the causal model on caller rows (``inputs_embeds``,
  hobbylm/model.py:325-333): 4 rows ~ N(0, 0.02^2) (numpy seed 7) spliced before the embeddings of
  an 8-id prompt (seed 1), as lib.rs:118-121 splices modality rows; the full last row plus
  per-position top-8 ids, values and logsumexp. The reference for Model::prefill / forward_x on rows.
"""
from __future__ import annotations

import argparse
import dataclasses
import importlib.util
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))


def reference_gguf_digests(ref: str, preset: str) -> dict:
    import torch
    import gguf
    from hobbylm_b200.synth import tensor_digest

    sys.path.insert(0, ref)
    from hobbylm.config import get_config
    from hobbylm.model import MoETransformer

    cfg = get_config(preset)
    torch.manual_seed(0)
    model = MoETransformer(cfg)
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    if cfg.n_shared == 0:
        for i in range(cfg.n_dense_layers, cfg.n_layers):
            sd[f"blocks.{i}.ffn.shared.w13"] = torch.zeros(1, cfg.d_model, 2 * cfg.expert_ffn)
            sd[f"blocks.{i}.ffn.shared.w2"] = torch.zeros(1, cfg.expert_ffn, cfg.d_model)
    spec = importlib.util.spec_from_file_location("ref_to_gguf", os.path.join(ref, "export", "to_gguf.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)

    def placeholder_tokenizer(vocab_size):
        toks = [f"<|tok_{i}|>" for i in range(vocab_size)]
        toks[50256] = "<|endoftext|>"
        return toks, [3 if i == 50256 else 1 for i in range(vocab_size)], ["Ġ t"]

    mod._gpt2_tokenizer = placeholder_tokenizer
    with tempfile.TemporaryDirectory() as td:
        ck = os.path.join(td, "ck", "model.pt")
        os.makedirs(os.path.dirname(ck))
        torch.save({"model": sd, "config": dataclasses.asdict(cfg)}, ck)
        out = os.path.join(td, "ref.gguf")
        argv = sys.argv
        sys.argv = ["to_gguf.py", "--ckpt", ck, "--out", out]
        try:
            mod.main()
        finally:
            sys.argv = argv
        r = gguf.GGUFReader(out)
        digests = {}
        for t in r.tensors:
            arr = np.asarray(t.data, dtype=np.float32).reshape([int(x) for x in reversed(t.shape)])
            digests[t.name] = tensor_digest(arr)
        meta = {}
        for k in ("hobbylm.context_length", "hobbylm.embedding_length", "hobbylm.block_count",
                  "hobbylm.attention.layer_norm_rms_epsilon", "hobbylm.rope.freq_base",
                  "hobbylm.expert_used_count", "hobbylm.expert_shared_count"):
            f = r.fields[k]
            meta[k] = float(f.parts[f.data[0]][0])
    return {"preset": preset, "seed": 0, "digests": digests, "meta": meta}


def reference_torch_logits(ref: str) -> dict:
    import torch

    sys.path.insert(0, ref)
    from hobbylm.config import get_config
    from hobbylm.model import MoETransformer
    from hobbylm_b200.synth import prompt_ids

    cfg = get_config("130M")
    cfg.expert_backend = "bmm"
    torch.manual_seed(0)
    model = MoETransformer(cfg).eval()
    ids = torch.from_numpy(prompt_ids(12, 1).astype(np.int64)).view(1, -1)
    with torch.no_grad():
        logits, _ = model(ids)
    lg = logits[0].float().numpy()
    top_ids = np.argsort(-lg, axis=1)[:, :8]
    top_vals = np.take_along_axis(lg, top_ids, axis=1)
    lse = np.log(np.exp(lg - lg.max(1, keepdims=True)).sum(1)) + lg.max(1)
    return {"ids": ids[0].numpy().astype(np.uint32), "last": lg[-1].astype(np.float32),
            "top_ids": top_ids.astype(np.int32), "top_vals": top_vals.astype(np.float32),
            "lse": lse.astype(np.float32)}


BIDIR_ROWS = (0, 12, 17)


def reference_torch_bidir_logits(ref: str) -> dict:
    import torch

    sys.path.insert(0, ref)
    from hobbylm.config import get_config
    from hobbylm.model import MoETransformer
    from hobbylm_b200.synth import prompt_ids

    cfg = get_config("130M")
    cfg.expert_backend = "bmm"
    cfg.diffusion = True
    torch.manual_seed(0)
    model = MoETransformer(cfg).eval()
    canvas = np.concatenate([prompt_ids(12, 1).astype(np.int64), np.full(6, cfg.mask_token_id, np.int64)])
    ids = torch.from_numpy(canvas).view(1, -1)
    with torch.no_grad():
        logits, _ = model(ids)
    lg = logits[0].float().numpy()
    top_ids = np.argsort(-lg, axis=1)[:, :8]
    top_vals = np.take_along_axis(lg, top_ids, axis=1)
    lse = np.log(np.exp(lg - lg.max(1, keepdims=True)).sum(1)) + lg.max(1)
    return {"ids": canvas.astype(np.uint32), "rows": np.array(BIDIR_ROWS, np.int32),
            "full": lg[list(BIDIR_ROWS)].astype(np.float32), "top_ids": top_ids.astype(np.int32),
            "top_vals": top_vals.astype(np.float32), "lse": lse.astype(np.float32)}


DIFF_CASES = (dict(gen_len=24, block=8, steps=8, rep_penalty=1.4),
              dict(gen_len=24, block=8, steps=12, rep_penalty=1.4, remask_steps=1),
              dict(gen_len=20, block=8, steps=5, rep_penalty=1.0))


def reference_diffusion_generate(ref: str) -> dict:
    import torch

    sys.path.insert(0, ref)
    from hobbylm import diffusion
    from hobbylm.config import get_config
    from hobbylm.model import MoETransformer
    from hobbylm_b200.synth import prompt_ids

    cfg = get_config("130M")
    cfg.expert_backend = "bmm"
    cfg.diffusion = True
    torch.manual_seed(0)
    model = MoETransformer(cfg).eval()
    prompt = prompt_ids(12, 1).astype(np.int64)
    cases = []
    for kw in DIFF_CASES:
        out = diffusion.generate(model, torch.from_numpy(prompt).view(1, -1), temperature=0.0, **kw)
        cases.append({"opts": kw, "ids": [int(t) for t in out[0]]})
    return {"prompt": [int(t) for t in prompt], "cases": cases}


def reference_torch_embeds_logits(ref: str) -> dict:
    import torch

    sys.path.insert(0, ref)
    from hobbylm.config import get_config
    from hobbylm.model import MoETransformer
    from hobbylm_b200.synth import prompt_ids

    cfg = get_config("130M")
    cfg.expert_backend = "bmm"
    torch.manual_seed(0)
    model = MoETransformer(cfg).eval()
    extra = (np.random.default_rng(7).standard_normal((4, cfg.d_model)) * 0.02).astype(np.float32)
    ids = torch.from_numpy(prompt_ids(8, 1).astype(np.int64))
    with torch.no_grad():
        rows = torch.cat([torch.from_numpy(extra), model.embed(ids)], 0)
        logits, _ = model(inputs_embeds=rows.unsqueeze(0))
    lg = logits[0].float().numpy()
    top_ids = np.argsort(-lg, axis=1)[:, :8]
    top_vals = np.take_along_axis(lg, top_ids, axis=1)
    lse = np.log(np.exp(lg - lg.max(1, keepdims=True)).sum(1)) + lg.max(1)
    return {"rows": rows.numpy().astype(np.float32), "last": lg[-1].astype(np.float32),
            "top_ids": top_ids.astype(np.int32), "top_vals": top_vals.astype(np.float32),
            "lse": lse.astype(np.float32)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("HOBBYLM_REFERENCE", ""))
    ap.add_argument("--only", choices=("all", "bidir", "embeds", "digests"), default="all",
                    help="bidir: only the diffusion fixtures; embeds: only the inputs_embeds fixture; "
                         "digests: only the synth_digests files of --presets")
    ap.add_argument("--presets", default="130M,500M,1B", help="presets whose exporter digests are written")
    a = ap.parse_args()
    if not a.reference or not os.path.isdir(a.reference):
        raise SystemExit("--reference must point at the HobbyLM checkout")
    if a.only == "digests":
        for preset in a.presets.split(","):
            d = reference_gguf_digests(a.reference, preset)
            with open(os.path.join(HERE, f"synth_digests_{preset}.json"), "w") as f:
                json.dump(d, f, indent=1, sort_keys=True)
            print(preset, len(d["digests"]), "tensors")
        return
    if a.only in ("all", "embeds"):
        el = reference_torch_embeds_logits(a.reference)
        np.savez(os.path.join(HERE, "torch_embeds_logits_130M.npz"), **el)
        print("embeds logits", el["top_ids"].shape)
        if a.only == "embeds":
            return
    bl = reference_torch_bidir_logits(a.reference)
    np.savez(os.path.join(HERE, "torch_bidir_logits_130M.npz"), **bl)
    print("bidir logits", bl["top_ids"].shape)
    dg = reference_diffusion_generate(a.reference)
    with open(os.path.join(HERE, "torch_diffusion_generate_130M.json"), "w") as f:
        json.dump(dg, f)
    print("diffusion cases", len(dg["cases"]))
    if a.only == "bidir":
        return
    for preset in a.presets.split(","):
        d = reference_gguf_digests(a.reference, preset)
        with open(os.path.join(HERE, f"synth_digests_{preset}.json"), "w") as f:
            json.dump(d, f, indent=1, sort_keys=True)
        print(preset, len(d["digests"]), "tensors")
    lg = reference_torch_logits(a.reference)
    np.savez(os.path.join(HERE, "torch_logits_130M.npz"), **lg)
    print("logits", lg["last"].shape)


if __name__ == "__main__":
    main()
