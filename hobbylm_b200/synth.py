"""Seeded synthetic hobbylm checkpoints written as GGUF (the input producer of the decode path).

The decode engine's benchmark and parity inputs are random-init hobbylm models (no trained
checkpoint is available offline). This module reproduces, in its own code, the two reference steps
that produce such a file:

* the model's random init: ``MoETransformer(get_config(preset))`` after ``torch.manual_seed(seed)``
  (hobbylm/model.py:259-313, hobbylm/moe.py:33-66, hobbylm/config.py:118-135). Module construction
  draws from the global generator (``nn.Embedding`` normal init, ``nn.Linear`` kaiming-uniform init,
  including the tied lm_head), then ``self.apply(self._init)`` redraws every Linear / Embedding /
  SwiGLU stack as N(0, init_std) in post-order, then residual projections are scaled by
  1/sqrt(2 L) and the router by 0.1. The same torch modules are constructed and the same draws are
  made in the same order, so the weights are bit-identical (pinned by tests/golden/synth_*.json).
* the exporter: export/to_gguf.py:38-133 (metadata keys, tensor names, the expert transposes, the
  fused qkv). Differences, each needed to run offline: the GPT-2 vocab/merges (downloaded from the
  HF hub by to_gguf.py:18-35) are replaced by placeholder token strings and one merge; a preset
  without a shared expert gets zero-filled ``*_shexp`` tensors (to_gguf.py:126-129 and
  model.rs:99-101 require them; ``expert_shared_count=0`` makes hobby-rs skip them); weight
  matrices are stored as Q8_0 (the role of ``llama-quantize``; gguf-py's quantizer is bit-exact with
  ggml's ``quantize_row_q8_0_ref``) while norms, ``exp_probs_b`` and the router stay F32.
"""
from __future__ import annotations

import hashlib
import dataclasses
import os
import tempfile
from dataclasses import dataclass

import numpy as np

VOCAB = 50304
EOS = 50256


@dataclass(frozen=True)
class Preset:
    d_model: int
    n_layers: int
    n_dense_layers: int
    n_q_heads: int
    n_kv_heads: int
    head_dim: int
    dense_ffn: int
    expert_ffn: int
    n_experts: int
    top_k: int
    n_shared: int
    vocab_size: int = VOCAB
    rope_theta: float = 10000.0
    init_std: float = 0.02


# hobbylm/config.py:118-134
PRESETS = {
    "130M": Preset(512, 12, 1, 8, 2, 64, 1536, 192, 32, 8, 0),
    "500M": Preset(768, 16, 1, 12, 3, 128, 2304, 320, 36, 6, 1),
    "1B": Preset(1024, 20, 1, 16, 8, 128, 2816, 224, 64, 8, 1),
}
# a few-MB model of the same architecture for smoke runs (not a reference preset)
TINY = Preset(256, 2, 1, 4, 1, 64, 512, 128, 8, 2, 1)


def init_weights(preset: str | Preset, seed: int = 0) -> dict:
    """Random-init weights in the reference's draw order. Returns torch f32 tensors keyed by the
    reference state_dict names (embed.weight, blocks.{i}.attn.qkv.weight, ...)."""
    import torch
    import torch.nn as nn

    p = PRESETS[preset] if isinstance(preset, str) else preset
    torch.manual_seed(seed)
    d, L = p.d_model, p.n_layers
    qkv_out = (p.n_q_heads + 2 * p.n_kv_heads) * p.head_dim
    # --- construction-time draws (module registration order) ---
    embed = nn.Embedding(p.vocab_size, d)
    blocks = []
    for i in range(L):
        b = {"qkv": nn.Linear(d, qkv_out, bias=False), "proj": nn.Linear(p.n_q_heads * p.head_dim, d, bias=False)}
        if i >= p.n_dense_layers:
            b["gate"] = nn.Linear(d, p.n_experts, bias=False)
            b["ew13"] = torch.empty(p.n_experts, d, 2 * p.expert_ffn)
            b["ew2"] = torch.empty(p.n_experts, p.expert_ffn, d)
            if p.n_shared > 0:
                b["sw13"] = torch.empty(p.n_shared, d, 2 * p.expert_ffn)
                b["sw2"] = torch.empty(p.n_shared, p.expert_ffn, d)
        else:
            b["w13"] = nn.Linear(d, 2 * p.dense_ffn, bias=False)
            b["w2"] = nn.Linear(p.dense_ffn, d, bias=False)
        blocks.append(b)
    nn.Linear(d, p.vocab_size, bias=False)  # the lm_head's own init draw; its weight is then tied
    # --- self.apply(_init): post-order over children ---
    std = p.init_std
    with torch.no_grad():
        nn.init.normal_(embed.weight, 0.0, std)
        for i, b in enumerate(blocks):
            nn.init.normal_(b["qkv"].weight, 0.0, std)
            nn.init.normal_(b["proj"].weight, 0.0, std)
            if i >= p.n_dense_layers:
                nn.init.normal_(b["gate"].weight, 0.0, std)
                nn.init.normal_(b["ew13"], 0.0, std)
                nn.init.normal_(b["ew2"], 0.0, std)
                if p.n_shared > 0:
                    nn.init.normal_(b["sw13"], 0.0, std)
                    nn.init.normal_(b["sw2"], 0.0, std)
            else:
                nn.init.normal_(b["w13"].weight, 0.0, std)
                nn.init.normal_(b["w2"].weight, 0.0, std)
        nn.init.normal_(embed.weight, 0.0, std)  # the tied lm_head is visited last
        # --- _scale_residual_init ---
        scale = (2 * L) ** -0.5
        for i, b in enumerate(blocks):
            b["proj"].weight.mul_(scale)
            if i >= p.n_dense_layers:
                b["ew2"].mul_(scale)
                if p.n_shared > 0:
                    b["sw2"].mul_(scale)
                b["gate"].weight.mul_(0.1)
            else:
                b["w2"].weight.mul_(scale)
    sd = {"embed.weight": embed.weight.detach(), "final_norm.weight": torch.ones(d)}
    for i, b in enumerate(blocks):
        pre = f"blocks.{i}."
        sd[pre + "attn_norm.weight"] = torch.ones(d)
        sd[pre + "ffn_norm.weight"] = torch.ones(d)
        sd[pre + "attn.qkv.weight"] = b["qkv"].weight.detach()
        sd[pre + "attn.proj.weight"] = b["proj"].weight.detach()
        sd[pre + "attn.q_norm.weight"] = torch.ones(p.head_dim)
        sd[pre + "attn.k_norm.weight"] = torch.ones(p.head_dim)
        if i >= p.n_dense_layers:
            sd[pre + "ffn.gate.weight"] = b["gate"].weight.detach()
            sd[pre + "ffn.expert_bias"] = torch.zeros(p.n_experts)
            sd[pre + "ffn.experts.w13"] = b["ew13"]
            sd[pre + "ffn.experts.w2"] = b["ew2"]
            if p.n_shared > 0:
                sd[pre + "ffn.shared.w13"] = b["sw13"]
                sd[pre + "ffn.shared.w2"] = b["sw2"]
        else:
            sd[pre + "ffn.w13.weight"] = b["w13"].weight.detach()
            sd[pre + "ffn.w2.weight"] = b["w2"].weight.detach()
    return sd


def gguf_tensors(preset: str | Preset, sd: dict) -> list:
    """(name, f32 numpy array in row-major [rows, cols] order) in export/to_gguf.py:101-129 order."""
    import torch

    p = PRESETS[preset] if isinstance(preset, str) else preset
    f, df = p.expert_ffn, p.dense_ffn
    out = []

    def t(name, arr):
        out.append((name, np.ascontiguousarray(arr.detach().to(torch.float32).numpy())))

    t("token_embd.weight", sd["embed.weight"])
    t("output_norm.weight", sd["final_norm.weight"])
    t("output.weight", sd.get("lm_head.weight", sd["embed.weight"]))
    for i in range(p.n_layers):
        pre = f"blocks.{i}."
        t(f"blk.{i}.attn_norm.weight", sd[pre + "attn_norm.weight"])
        t(f"blk.{i}.attn_qkv.weight", sd[pre + "attn.qkv.weight"])
        t(f"blk.{i}.attn_q_norm.weight", sd[pre + "attn.q_norm.weight"])
        t(f"blk.{i}.attn_k_norm.weight", sd[pre + "attn.k_norm.weight"])
        t(f"blk.{i}.attn_output.weight", sd[pre + "attn.proj.weight"])
        t(f"blk.{i}.ffn_norm.weight", sd[pre + "ffn_norm.weight"])
        if i < p.n_dense_layers:
            w13 = sd[pre + "ffn.w13.weight"]
            t(f"blk.{i}.ffn_gate.weight", w13[:df])
            t(f"blk.{i}.ffn_up.weight", w13[df:])
            t(f"blk.{i}.ffn_down.weight", sd[pre + "ffn.w2.weight"])
        else:
            t(f"blk.{i}.ffn_gate_inp.weight", sd[pre + "ffn.gate.weight"])
            t(f"blk.{i}.exp_probs_b.bias", sd[pre + "ffn.expert_bias"])
            ew13, ew2 = sd[pre + "ffn.experts.w13"], sd[pre + "ffn.experts.w2"]
            t(f"blk.{i}.ffn_gate_exps.weight", ew13[..., :f].transpose(1, 2).contiguous())
            t(f"blk.{i}.ffn_up_exps.weight", ew13[..., f:].transpose(1, 2).contiguous())
            t(f"blk.{i}.ffn_down_exps.weight", ew2.transpose(1, 2).contiguous())
            if pre + "ffn.shared.w13" in sd:
                sw13, sw2 = sd[pre + "ffn.shared.w13"], sd[pre + "ffn.shared.w2"]
                t(f"blk.{i}.ffn_gate_shexp.weight", sw13[0, :, :f].t().contiguous())
                t(f"blk.{i}.ffn_up_shexp.weight", sw13[0, :, f:].t().contiguous())
                t(f"blk.{i}.ffn_down_shexp.weight", sw2[0].t().contiguous())
            else:
                z = torch.zeros
                t(f"blk.{i}.ffn_gate_shexp.weight", z(f, p.d_model))
                t(f"blk.{i}.ffn_up_shexp.weight", z(f, p.d_model))
                t(f"blk.{i}.ffn_down_shexp.weight", z(p.d_model, f))
    return out


def keep_f32(name: str, arr: np.ndarray) -> bool:
    """Tensors stored F32 in the Q8_0 file: 1-D norms and biases, and the router."""
    return arr.ndim < 2 or name.endswith("ffn_gate_inp.weight")


def tensor_digest(arr: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(arr, dtype=np.float32).tobytes()).hexdigest()[:32]


def write_gguf(path: str, preset: str | Preset, tensors: list, *, quant: str = "q8_0",
               context_length: int = 8192, rms_eps: float = 1e-5, arch: str = "hobbylm") -> None:
    """Write a GGUF v3 file with export/to_gguf.py's metadata (to_gguf.py:59-96)."""
    import gguf

    p = PRESETS[preset] if isinstance(preset, str) else preset
    w = gguf.GGUFWriter(path, arch)
    w.add_name("HobbyLM (synthetic)")
    w.add_context_length(context_length)
    w.add_embedding_length(p.d_model)
    w.add_block_count(p.n_layers)
    w.add_feed_forward_length(p.dense_ffn)
    w.add_head_count(p.n_q_heads)
    w.add_head_count_kv(p.n_kv_heads)
    w.add_key_length(p.head_dim)
    w.add_value_length(p.head_dim)
    w.add_layer_norm_rms_eps(rms_eps)
    w.add_rope_freq_base(p.rope_theta)
    w.add_expert_count(p.n_experts)
    w.add_expert_used_count(p.top_k)
    w.add_expert_feed_forward_length(p.expert_ffn)
    w.add_expert_shared_count(p.n_shared)
    w.add_expert_shared_feed_forward_length(p.expert_ffn)
    w.add_leading_dense_block_count(p.n_dense_layers)
    w.add_expert_gating_func(gguf.ExpertGatingFuncType.SIGMOID)
    w.add_expert_weights_norm(False)
    w.add_expert_weights_scale(1.0)
    w.add_vocab_size(p.vocab_size)
    w.add_uint32(f"{arch}.nextn_predict_layers", 0)
    toks = [f"<|tok_{i}|>" for i in range(p.vocab_size)]
    toks[EOS] = "<|endoftext|>"
    w.add_tokenizer_model("gpt2")
    w.add_tokenizer_pre("gpt-2")
    w.add_token_list(toks)
    w.add_token_types([3 if i == EOS else 1 for i in range(p.vocab_size)])
    w.add_token_merges(["Ġ t"])
    w.add_bos_token_id(EOS)
    w.add_eos_token_id(EOS)
    w.add_add_bos_token(False)
    for name, arr in tensors:
        if quant == "q8_0" and not keep_f32(name, arr):
            q = gguf.quants.quantize(arr, gguf.GGMLQuantizationType.Q8_0)
            w.add_tensor(name, q, raw_dtype=gguf.GGMLQuantizationType.Q8_0)
        else:
            w.add_tensor(name, np.ascontiguousarray(arr, dtype=np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def make_model_gguf(path: str, preset: str = "130M", seed: int = 0, *, quant: str = "q8_0",
                    context_length: int = 8192, rms_eps: float = 1e-5) -> str:
    """Seed-``seed`` random-init ``preset`` model written to ``path`` (skipped if it exists)."""
    if os.path.exists(path):
        return path
    tmp = path + f".tmp{os.getpid()}"
    sd = init_weights(preset, seed)
    write_gguf(tmp, preset, gguf_tensors(preset, sd), quant=quant, context_length=context_length,
               rms_eps=rms_eps)
    os.replace(tmp, path)
    return path


def cached_model(preset: str = "130M", seed: int = 0, *, quant: str = "q8_0", context_length: int = 8192,
                 rms_eps: float = 1e-5, cache_dir: str | None = None) -> str:
    """Path of a cached synthetic GGUF (generated on first use)."""
    root = cache_dir or os.environ.get("HOBBYLM_B200_CACHE") or os.path.join(
        tempfile.gettempdir(), "hobbylm_b200_cache")
    os.makedirs(root, exist_ok=True)
    eps_tag = f"{rms_eps:g}".replace("-", "m")
    tag = preset if isinstance(preset, str) else "p" + "x".join(str(getattr(preset, f.name))
                                                               for f in dataclasses.fields(preset))
    name = f"hobbylm-{tag}-s{seed}-{quant}-ctx{context_length}-eps{eps_tag}.gguf"
    return make_model_gguf(os.path.join(root, name), preset, seed, quant=quant,
                           context_length=context_length, rms_eps=rms_eps)


def prompt_ids(n: int, seed: int, vocab: int = 50257) -> np.ndarray:
    """Token ids ~ U[0, vocab) from torch.Generator().manual_seed(seed) (the configs' prompts)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n,), generator=g).numpy().astype(np.uint32)


def moe_op_inputs(seed: int = 2, d: int = 768, f: int = 320, ne: int = 36, n_shared: int = 1,
                  T: int = 256) -> dict:
    """The op-level MoE inputs: expert weights as Q8_0 blocks with int8 ~ U[-127, 127] and fp16
    scales |N(0, 0.01)| (dequantized to f32 here, which is what Model::load hands to the
    re-quantizer), router W ~ N(0, 0.02), bias ~ N(0, 0.1), activations x ~ N(0, 1)."""
    import torch

    g = torch.Generator().manual_seed(seed)

    def q8(rows, cols, count):
        q = torch.randint(-127, 128, (count, rows, cols), generator=g, dtype=torch.int32).to(torch.float32)
        s = torch.randn(count, rows, cols // 32, generator=g).abs() * 0.01
        s = s.to(torch.float16).to(torch.float32)
        return (q.view(count, rows, cols // 32, 32) * s.unsqueeze(-1)).reshape(count, rows, cols).numpy()

    out = {
        "router": (torch.randn(ne, d, generator=g) * 0.02).numpy(),
        "bias": (torch.randn(ne, generator=g) * 0.1).numpy(),
        "gate_exps": q8(f, d, ne),
        "up_exps": q8(f, d, ne),
        "down_exps": q8(d, f, ne),
    }
    if n_shared:
        out["gate_sh"], out["up_sh"], out["down_sh"] = q8(f, d, 1)[0], q8(f, d, 1)[0], q8(d, f, 1)[0]
    out["x"] = torch.randn(T, d, generator=g).numpy()
    return {k: np.ascontiguousarray(v, dtype=np.float32) for k, v in out.items()}


def digests(preset: str, seed: int = 0) -> dict:
    sd = init_weights(preset, seed)
    return {name: tensor_digest(arr) for name, arr in gguf_tensors(preset, sd)}
