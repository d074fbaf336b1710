"""Synthetic HF-layout checkpoints and tokenizers (no network needed).

Writes ``config.json``, ``model.safetensors`` (N(0, std) weights, norm
weights 1, optional Qwen3 ``k_norm`` drawn with |w| up to a bound) and a
word-level ``tokenizer.json`` whose vocabulary has exactly ``vocab_size``
entries, so both this engine and the reference load it unchanged through
``AutoConfig`` / ``AutoTokenizer`` / safetensors.
"""
from __future__ import annotations

import json
import os
from typing import Optional

import torch

PRESETS = {
    # CPU fp32 plumbing/correctness model (2 layers, hidden 256)
    "tiny-llama": dict(model_type="llama", hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                       num_key_value_heads=2, head_dim=64, intermediate_size=688, vocab_size=1024,
                       rms_norm_eps=1e-6, rope_theta=10000.0, max_position_embeddings=4096,
                       tie_word_embeddings=False),
    "tiny-qwen3": dict(model_type="qwen3", hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                       num_key_value_heads=2, head_dim=64, intermediate_size=768, vocab_size=1024,
                       rms_norm_eps=1e-6, rope_theta=1000000.0, max_position_embeddings=4096,
                       tie_word_embeddings=True, attention_bias=False),
    "qwen3-0.6b": dict(model_type="qwen3", hidden_size=1024, num_hidden_layers=28, num_attention_heads=16,
                       num_key_value_heads=8, head_dim=128, intermediate_size=3072, vocab_size=151936,
                       rms_norm_eps=1e-6, rope_theta=1000000.0, max_position_embeddings=40960,
                       tie_word_embeddings=True, attention_bias=False),
    "tinyllama-1.1b": dict(model_type="llama", hidden_size=2048, num_hidden_layers=22, num_attention_heads=32,
                           num_key_value_heads=4, head_dim=64, intermediate_size=5632, vocab_size=32000,
                           rms_norm_eps=1e-5, rope_theta=10000.0, max_position_embeddings=4096,
                           tie_word_embeddings=False),
    "llama3-8b": dict(model_type="llama", hidden_size=4096, num_hidden_layers=32, num_attention_heads=32,
                      num_key_value_heads=8, head_dim=128, intermediate_size=14336, vocab_size=128256,
                      rms_norm_eps=1e-5, rope_theta=500000.0, max_position_embeddings=8192,
                      tie_word_embeddings=False),
    "llama3-70b": dict(model_type="llama", hidden_size=8192, num_hidden_layers=80, num_attention_heads=64,
                       num_key_value_heads=8, head_dim=128, intermediate_size=28672, vocab_size=128256,
                       rms_norm_eps=1e-5, rope_theta=500000.0, max_position_embeddings=16384,
                       tie_word_embeddings=False),
    "tiny-gpt2": dict(model_type="gpt2", n_embd=256, n_layer=2, n_head=4, n_inner=1024, vocab_size=1024,
                      n_positions=1024, layer_norm_epsilon=1e-5),
    "tiny-ernie": dict(model_type="ernie4_5", hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                       num_key_value_heads=2, head_dim=64, intermediate_size=704, vocab_size=1024,
                       rms_norm_eps=1e-5, rope_theta=500000.0, max_position_embeddings=4096,
                       tie_word_embeddings=True, use_bias=False),
}


def hf_config(preset: str, **over) -> dict:
    cfg = dict(PRESETS[preset])
    cfg.update(over)
    mt = cfg["model_type"]
    arch = {"llama": "LlamaForCausalLM", "qwen3": "Qwen3ForCausalLM", "gpt2": "GPT2LMHeadModel",
            "ernie4_5": "Ernie4_5ForCausalLM"}[mt]
    cfg.setdefault("architectures", [arch])
    cfg.setdefault("torch_dtype", "bfloat16")
    cfg.setdefault("bos_token_id", 1)
    cfg.setdefault("eos_token_id", 2)
    if mt != "gpt2":
        cfg.setdefault("hidden_act", "silu")
        cfg.setdefault("attention_bias", False)
    return cfg


def hf_state_dict(cfg: dict, seed: int = 0, std: float = 0.02, k_norm_range: Optional[float] = None,
                  dtype=torch.float32, norm_jitter: float = 0.0) -> dict:
    """HF-named tensors; norm weights are 1, or uniform in [1 - j, 1 + j] with
    ``norm_jitter`` j (exercises the folding of RMSNorm weights into GEMMs)."""
    g = torch.Generator().manual_seed(seed)

    def rnd(*shape):
        return (torch.randn(*shape, generator=g) * std).to(dtype)

    def norm_w(n):
        if norm_jitter <= 0:
            return torch.ones(n, dtype=dtype)
        return (1 + (torch.rand(n, generator=g) * 2 - 1) * norm_jitter).to(dtype)

    sd = {}
    if cfg["model_type"] == "gpt2":
        H, I, V = cfg["n_embd"], cfg.get("n_inner") or 4 * cfg["n_embd"], cfg["vocab_size"]
        sd["transformer.wte.weight"] = rnd(V, H)
        sd["transformer.wpe.weight"] = rnd(cfg["n_positions"], H) * 0.5
        for i in range(cfg["n_layer"]):
            p = f"transformer.h.{i}."
            sd[p + "ln_1.weight"] = torch.ones(H, dtype=dtype)
            sd[p + "ln_1.bias"] = torch.zeros(H, dtype=dtype)
            sd[p + "attn.c_attn.weight"] = rnd(H, 3 * H)
            sd[p + "attn.c_attn.bias"] = rnd(3 * H)
            sd[p + "attn.c_proj.weight"] = rnd(H, H)
            sd[p + "attn.c_proj.bias"] = rnd(H)
            sd[p + "ln_2.weight"] = torch.ones(H, dtype=dtype)
            sd[p + "ln_2.bias"] = torch.zeros(H, dtype=dtype)
            sd[p + "mlp.c_fc.weight"] = rnd(H, I)
            sd[p + "mlp.c_fc.bias"] = rnd(I)
            sd[p + "mlp.c_proj.weight"] = rnd(I, H)
            sd[p + "mlp.c_proj.bias"] = rnd(H)
        sd["transformer.ln_f.weight"] = torch.ones(H, dtype=dtype)
        sd["transformer.ln_f.bias"] = torch.zeros(H, dtype=dtype)
        return sd
    H, I, V = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    nh, nkv = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    D = cfg.get("head_dim") or H // nh
    bias = cfg.get("attention_bias", False) or cfg.get("use_bias", False)
    sd["model.embed_tokens.weight"] = rnd(V, H)
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}."
        sd[p + "input_layernorm.weight"] = norm_w(H)
        sd[p + "post_attention_layernorm.weight"] = norm_w(H)
        sd[p + "self_attn.q_proj.weight"] = rnd(nh * D, H)
        sd[p + "self_attn.k_proj.weight"] = rnd(nkv * D, H)
        sd[p + "self_attn.v_proj.weight"] = rnd(nkv * D, H)
        if bias:
            sd[p + "self_attn.q_proj.bias"] = rnd(nh * D)
            sd[p + "self_attn.k_proj.bias"] = rnd(nkv * D)
            sd[p + "self_attn.v_proj.bias"] = rnd(nkv * D)
        sd[p + "self_attn.o_proj.weight"] = rnd(H, nh * D)
        if cfg["model_type"] == "qwen3":
            sd[p + "self_attn.q_norm.weight"] = norm_w(D)
            kn = torch.ones(D, dtype=dtype)
            if k_norm_range is not None:
                kn = (torch.rand(D, generator=g) * 2 - 1).mul(k_norm_range).to(dtype)
            sd[p + "self_attn.k_norm.weight"] = kn
        sd[p + "mlp.gate_proj.weight"] = rnd(I, H)
        sd[p + "mlp.up_proj.weight"] = rnd(I, H)
        sd[p + "mlp.down_proj.weight"] = rnd(H, I)
    sd["model.norm.weight"] = norm_w(H)
    if not cfg.get("tie_word_embeddings", False):
        sd["lm_head.weight"] = rnd(V, H)
    return sd


def write_tokenizer(path: str, vocab_size: int, chat_template: bool = False) -> None:
    """Word-level tokenizer: token ``i`` is the word ``w{i}``; ids 0/1/2 are unk/bos/eos."""
    from tokenizers import Tokenizer, models, pre_tokenizers, decoders

    vocab = {f"w{i}": i for i in range(vocab_size)}
    specials = {0: "<unk>", 1: "<s>", 2: "</s>"}
    for i, s in specials.items():
        if i < vocab_size:
            del vocab[f"w{i}"]
            vocab[s] = i
    tok = Tokenizer(models.WordLevel(vocab=vocab, unk_token="<unk>"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tok.decoder = decoders.WordPiece(prefix="##")  # joins words with spaces
    from tokenizers import AddedToken

    tok.add_special_tokens([AddedToken(s, special=True) for s in specials.values()])
    tok.save(os.path.join(path, "tokenizer.json"))
    tc = {"tokenizer_class": "PreTrainedTokenizerFast", "unk_token": "<unk>", "bos_token": "<s>",
          "eos_token": "</s>", "model_max_length": 1 << 20, "add_bos_token": False}
    if chat_template:
        tc["chat_template"] = ("{% for m in messages %}<s> w3 {{ m['role'] }} {{ m['content'] }} </s> "
                               "{% endfor %}{% if add_generation_prompt %}<s> w4 {% endif %}")
    with open(os.path.join(path, "tokenizer_config.json"), "w") as f:
        json.dump(tc, f)
    with open(os.path.join(path, "special_tokens_map.json"), "w") as f:
        json.dump({"unk_token": "<unk>", "bos_token": "<s>", "eos_token": "</s>"}, f)


def make_checkpoint(path: str, preset: str, seed: int = 0, std: float = 0.02,
                    k_norm_range: Optional[float] = None, write_weights: bool = True,
                    chat_template: bool = False, dtype=torch.bfloat16, norm_jitter: float = 0.0, **over) -> str:
    """Create an HF-layout checkpoint directory and return its path."""
    os.makedirs(path, exist_ok=True)
    cfg = hf_config(preset, **over)
    cfg["torch_dtype"] = str(dtype).replace("torch.", "")
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    write_tokenizer(path, cfg["vocab_size"], chat_template)
    if write_weights:
        from safetensors.torch import save_file

        sd = hf_state_dict(cfg, seed=seed, std=std, k_norm_range=k_norm_range, dtype=dtype, norm_jitter=norm_jitter)
        save_file({k: v.contiguous() for k, v in sd.items()}, os.path.join(path, "model.safetensors"))
    return path
