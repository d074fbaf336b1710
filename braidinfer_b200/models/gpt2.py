"""GPT-2 (learned absolute positions, LayerNorm, tanh-GELU MLP, tied head).

Parity with ``braidinfer/models/gpt2.py``: HF ``Conv1D`` weights are stored
``[in, out]`` and are transposed at load time (``gpt2.py:59-63`` did the same
for ``c_attn``); the LM head is tied to ``wte`` (``gpt2.py:192``).  Attention
goes through the same paged cascade kernel with RoPE disabled, so GPT-2 gets
chunk composition too (positions come from ``wpe`` at the composed position).
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import torch

from .. import ops
from ..config import ModelSpec
from ..parallel import comm
from ..parallel.layout import TPLayout
from ..parallel.state import TPState


class GPT2LM:
    packed_modules_mapping: dict = {}

    def __init__(self, spec: ModelSpec, tp: TPState, dtype: torch.dtype, device: torch.device, max_pos: int):
        self.spec, self.tp, self.dtype, self.device = spec, tp, dtype, device
        self.layout = TPLayout(tp.size, tp.rank, spec.num_heads, spec.num_kv_heads, spec.head_dim,
                               spec.intermediate_size, spec.vocab_size)
        L, H, D = self.layout, spec.hidden_size, spec.head_dim
        kw = dict(dtype=dtype, device=device)
        self.qkv_rows = 3 * L.q_heads * D
        self.inter_local = spec.intermediate_size // tp.size
        self.layers = []
        for _ in range(spec.num_layers):
            self.layers.append(dict(
                ln1_w=torch.ones(H, **kw), ln1_b=torch.zeros(H, **kw),
                qkv_w=torch.empty(self.qkv_rows, H, **kw), qkv_b=torch.zeros(self.qkv_rows, **kw),
                o_w=torch.empty(H, L.q_heads * D, **kw), o_b=torch.zeros(H, **kw),
                ln2_w=torch.ones(H, **kw), ln2_b=torch.zeros(H, **kw),
                fc_w=torch.empty(self.inter_local, H, **kw), fc_b=torch.zeros(self.inter_local, **kw),
                proj_w=torch.empty(H, self.inter_local, **kw), proj_b=torch.zeros(H, **kw)))
        self.embed = torch.empty(L.vocab_local, H, **kw)
        self.wpe = torch.empty(spec.max_position_embeddings, H, **kw)
        self.lnf_w = torch.ones(H, **kw)
        self.lnf_b = torch.zeros(H, **kw)
        self.lm_head = self.embed
        self.cos = self.sin = torch.zeros(1, max(1, D // 2), device=device)
        self.scale = 1.0 / math.sqrt(D)

    def random_init(self, seed: int = 0, std: float = 0.02, k_norm_range=None) -> None:
        g = torch.Generator(device=self.device)
        g.manual_seed(seed + 7919 * self.tp.rank)
        for w in self.layers:
            for k in ("qkv_w", "o_w", "fc_w", "proj_w"):
                w[k].normal_(0.0, std, generator=g)
        self.embed.normal_(0.0, std, generator=g)
        self.wpe.normal_(0.0, std / 2, generator=g)

    def load_hf_tensor(self, name: str, t: torch.Tensor) -> bool:
        L, S = self.layout, self.spec
        D, H = S.head_dim, S.hidden_size
        t = t.to(self.dtype)
        name = name[len("transformer."):] if name.startswith("transformer.") else name
        if name == "wte.weight":
            self.embed.copy_(t[L.vocab_start:L.vocab_start + L.vocab_local])
            return True
        if name == "wpe.weight":
            self.wpe.copy_(t[: self.wpe.shape[0]])
            return True
        if name == "ln_f.weight":
            self.lnf_w.copy_(t)
            return True
        if name == "ln_f.bias":
            self.lnf_b.copy_(t)
            return True
        if name == "lm_head.weight":
            return True
        if not name.startswith("h."):
            return False
        parts = name.split(".")
        w = self.layers[int(parts[1])]
        sub = ".".join(parts[2:])
        q0, nq = L.q_head_start * D, L.q_heads * D
        i0, ni = self.tp.rank * self.inter_local, self.inter_local
        if sub.endswith(".attn.bias") or sub.endswith("masked_bias") or sub == "attn.bias":
            return True
        if sub == "ln_1.weight":
            w["ln1_w"].copy_(t)
        elif sub == "ln_1.bias":
            w["ln1_b"].copy_(t)
        elif sub == "ln_2.weight":
            w["ln2_w"].copy_(t)
        elif sub == "ln_2.bias":
            w["ln2_b"].copy_(t)
        elif sub == "attn.c_attn.weight":  # Conv1D [H, 3H]
            tt = t.t()
            w["qkv_w"].copy_(torch.cat([tt[j * H + q0:j * H + q0 + nq] for j in range(3)]))
        elif sub == "attn.c_attn.bias":
            w["qkv_b"].copy_(torch.cat([t[j * H + q0:j * H + q0 + nq] for j in range(3)]))
        elif sub == "attn.c_proj.weight":  # [H_in, H_out]
            w["o_w"].copy_(t.t()[:, q0:q0 + nq])
        elif sub == "attn.c_proj.bias":
            w["o_b"].copy_(t if self.tp.rank == 0 else torch.zeros_like(t))
        elif sub == "mlp.c_fc.weight":
            w["fc_w"].copy_(t.t()[i0:i0 + ni])
        elif sub == "mlp.c_fc.bias":
            w["fc_b"].copy_(t[i0:i0 + ni])
        elif sub == "mlp.c_proj.weight":
            w["proj_w"].copy_(t.t()[:, i0:i0 + ni])
        elif sub == "mlp.c_proj.bias":
            w["proj_b"].copy_(t if self.tp.rank == 0 else torch.zeros_like(t))
        else:
            return False
        return True

    def finalize(self) -> None:
        pass

    def embed_tokens(self, input_ids, positions):
        h = ops.embedding(input_ids, self.embed, self.layout.vocab_start)
        if self.tp.size > 1:
            h = comm.all_reduce(h)
        return (h.float() + self.wpe[positions.long()].float()).to(self.dtype)

    def forward(self, input_ids, positions, slot_mapping, meta, kv_cache, workspace: Optional[Dict] = None):
        S, L = self.spec, self.layout
        h = self.embed_tokens(input_ids, positions)
        eps = S.rms_norm_eps
        for i, w in enumerate(self.layers):
            x = ops.layer_norm(h, w["ln1_w"], w["ln1_b"], eps)
            qkv = ops.linear(x, w["qkv_w"], w["qkv_b"])
            q = ops.qkv_prepare(qkv, positions, slot_mapping, kv_cache[i], L.q_heads, L.q_heads, S.head_dim,
                                self.cos, self.sin, None, None, eps, False)
            o = ops.attention(q, kv_cache[i], meta, self.cos, self.sin, self.scale, False, workspace)
            if self.tp.size == 1:
                h = ops.linear(o, w["o_w"], w["o_b"], residual=h)
            else:
                h = (h.float() + comm.all_reduce(ops.linear(o, w["o_w"], w["o_b"])).float()).to(self.dtype)
            x = ops.layer_norm(h, w["ln2_w"], w["ln2_b"], eps)
            m = ops.gelu_new(ops.linear(x, w["fc_w"], w["fc_b"]))
            if self.tp.size == 1:
                h = ops.linear(m, w["proj_w"], w["proj_b"], residual=h)
            else:
                h = (h.float() + comm.all_reduce(ops.linear(m, w["proj_w"], w["proj_b"])).float()).to(self.dtype)
        return h

    def final_hidden(self, h):
        return ops.layer_norm(h, self.lnf_w, self.lnf_b, self.spec.rms_norm_eps)

    def compute_logits(self, hn):
        local = ops.linear(hn, self.lm_head)
        if self.tp.size > 1:
            return comm.all_gather_last(local, self.spec.vocab_size)
        return local
