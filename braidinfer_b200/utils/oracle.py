"""Independent fp32 CPU oracle: a straight-line HF-semantics forward over a
whole token sequence with an explicit attention mask.

It shares no code with the engine's paged/cascade path (no pages, no
segments, no query-side RoPE): it rotates keys at their *global* positions and
applies a dense boolean mask, which is what the cascade must reproduce.
``block_causal_mask`` builds the mask that independently cached chunks imply.
"""
from __future__ import annotations

from typing import List, Sequence

import torch
import torch.nn.functional as F

from ..ops.rope import inv_freq


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _rope(x, pos, cos_tab, sin_tab, interleaved=False):
    # x [N, H, D]
    c = cos_tab[pos][:, None, :]
    s = sin_tab[pos][:, None, :]
    if interleaved:
        x1, x2 = x[..., 0::2], x[..., 1::2]
        o1, o2 = x1 * c - x2 * s, x2 * c + x1 * s
        return torch.stack([o1, o2], -1).flatten(-2)
    d2 = x.shape[-1] // 2
    x1, x2 = x[..., :d2], x[..., d2:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)


def block_causal_mask(blocks: Sequence[int], private_from: int) -> torch.Tensor:
    """``blocks[i]`` is token i's chunk index.  Tokens of blocks ``< private_from``
    are cached chunks (causal inside their own chunk only); the rest are the
    private prompt and generated tokens (see every chunk, causal among
    themselves)."""
    b = torch.as_tensor(blocks)
    n = len(b)
    i = torch.arange(n)[:, None]
    j = torch.arange(n)[None, :]
    causal = j <= i
    same = b[:, None] == b[None, :]
    chunk_i = b[:, None] < private_from
    chunk_j = b[None, :] < private_from
    return torch.where(chunk_i, same & causal, chunk_j | (causal & ~chunk_j))


@torch.no_grad()
def forward(cfg: dict, sd: dict, ids: List[int], positions: List[int], mask: torch.Tensor) -> torch.Tensor:
    sd = {k: v.float() for k, v in sd.items()}
    ids_t = torch.as_tensor(ids)
    pos = torch.as_tensor(positions)
    if cfg["model_type"] == "gpt2":
        return _gpt2(cfg, sd, ids_t, pos, mask)
    H, nh, nkv = cfg["hidden_size"], cfg["num_attention_heads"], cfg["num_key_value_heads"]
    D = cfg.get("head_dim") or H // nh
    eps = cfg.get("rms_norm_eps", 1e-6)
    inv = inv_freq(D, cfg.get("rope_theta", 10000.0), cfg.get("rope_scaling"))
    ang = torch.outer(torch.arange(int(pos.max()) + 1, dtype=torch.float32), inv)
    cos_t, sin_t = ang.cos(), ang.sin()
    inter = cfg["model_type"] == "ernie4_5"
    N = len(ids)
    h = sd["model.embed_tokens.weight"][ids_t]
    neg = torch.where(mask, 0.0, float("-inf"))
    for li in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{li}."
        x = _rms(h, sd[p + "input_layernorm.weight"], eps)
        q = F.linear(x, sd[p + "self_attn.q_proj.weight"], sd.get(p + "self_attn.q_proj.bias")).view(N, nh, D)
        k = F.linear(x, sd[p + "self_attn.k_proj.weight"], sd.get(p + "self_attn.k_proj.bias")).view(N, nkv, D)
        v = F.linear(x, sd[p + "self_attn.v_proj.weight"], sd.get(p + "self_attn.v_proj.bias")).view(N, nkv, D)
        if p + "self_attn.q_norm.weight" in sd:
            q = _rms(q, sd[p + "self_attn.q_norm.weight"], eps)
            k = _rms(k, sd[p + "self_attn.k_norm.weight"], eps)
        q = _rope(q, pos, cos_t, sin_t, inter)
        k = _rope(k, pos, cos_t, sin_t, inter)
        g = nh // nkv
        k = k.repeat_interleave(g, 1)
        v = v.repeat_interleave(g, 1)
        sc = torch.einsum("ihd,jhd->hij", q, k) / D ** 0.5 + neg
        o = torch.einsum("hij,jhd->ihd", sc.softmax(-1), v).reshape(N, nh * D)
        h = h + F.linear(o, sd[p + "self_attn.o_proj.weight"])
        x = _rms(h, sd[p + "post_attention_layernorm.weight"], eps)
        a = F.silu(F.linear(x, sd[p + "mlp.gate_proj.weight"])) * F.linear(x, sd[p + "mlp.up_proj.weight"])
        h = h + F.linear(a, sd[p + "mlp.down_proj.weight"])
    h = _rms(h, sd["model.norm.weight"], eps)
    head = sd.get("lm_head.weight", sd["model.embed_tokens.weight"])
    return F.linear(h, head)


def _gpt2(cfg, sd, ids, pos, mask):
    H, nh = cfg["n_embd"], cfg["n_head"]
    D = H // nh
    eps = cfg.get("layer_norm_epsilon", 1e-5)
    N = len(ids)
    h = sd["transformer.wte.weight"][ids] + sd["transformer.wpe.weight"][pos]
    neg = torch.where(mask, 0.0, float("-inf"))
    for li in range(cfg["n_layer"]):
        p = f"transformer.h.{li}."
        x = F.layer_norm(h, (H,), sd[p + "ln_1.weight"], sd[p + "ln_1.bias"], eps)
        qkv = x @ sd[p + "attn.c_attn.weight"] + sd[p + "attn.c_attn.bias"]
        q, k, v = qkv.split(H, -1)
        q, k, v = (t.view(N, nh, D) for t in (q, k, v))
        sc = torch.einsum("ihd,jhd->hij", q, k) / D ** 0.5 + neg
        o = torch.einsum("hij,jhd->ihd", sc.softmax(-1), v).reshape(N, H)
        h = h + o @ sd[p + "attn.c_proj.weight"] + sd[p + "attn.c_proj.bias"]
        x = F.layer_norm(h, (H,), sd[p + "ln_2.weight"], sd[p + "ln_2.bias"], eps)
        m = x @ sd[p + "mlp.c_fc.weight"] + sd[p + "mlp.c_fc.bias"]
        m = 0.5 * m * (1 + torch.tanh(0.7978845608028654 * (m + 0.044715 * m ** 3)))
        h = h + m @ sd[p + "mlp.c_proj.weight"] + sd[p + "mlp.c_proj.bias"]
    h = F.layer_norm(h, (H,), sd["transformer.ln_f.weight"], sd["transformer.ln_f.bias"], eps)
    return F.linear(h, sd["transformer.wte.weight"])


def greedy(cfg, sd, prompt_ids, blocks, private_from, n_new, positions=None):
    """Greedy continuation under the block-causal mask; returns (tokens, logits list)."""
    ids = list(prompt_ids)
    blocks = list(blocks)
    pos = list(positions) if positions is not None else list(range(len(ids)))
    toks, logits = [], []
    for _ in range(n_new):
        m = block_causal_mask(blocks, private_from)
        lg = forward(cfg, sd, ids, pos, m)[-1]
        t = int(lg.argmax())
        toks.append(t)
        logits.append(lg)
        ids.append(t)
        blocks.append(max(blocks) + 1 if blocks[-1] < private_from else blocks[-1])
        pos.append(pos[-1] + 1)
    return toks, logits
