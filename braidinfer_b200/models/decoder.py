"""Llama-style decoder (Llama / TinyLlama / Llama-3, Qwen3, ERNIE-4.5).

One implementation serves the reference's three RMSNorm/SwiGLU/RoPE model
files (``braidinfer/models/llama.py``, ``qwen3.py``, ``ernie.py``); the
differences are data: Qwen3's per-head ``q_norm``/``k_norm``, optional QKV
bias, tied embeddings, and ERNIE's interleaved ("GLM") rotary pairs, which
are turned into the neox half-split convention by permuting each head's q/k
projection rows at load time (a permutation applied to both q and k leaves
q·k unchanged).

HF semantics are kept where the reference deviated: no ``1/sqrt(hidden)``
embedding scaling for Qwen3 (``braidinfer/models/qwen3.py:465``), ``lm_head``
tied to ``embed_tokens`` when ``tie_word_embeddings`` is set, K cached after
k_norm and RoPE and never re-normalised at attention time.

Per layer the forward runs five kernels: QKV GEMM (input RMSNorm fused: the
norm weight is folded into the weight columns at load time and each token's
1/rms is applied in the epilogue, then bias, q/k-norm, RoPE(k) and the paged
KV append) → cascade attention (query-side differential RoPE) → o_proj GEMM
with the residual add in its epilogue (or the TP reduction) → gate/up GEMM
(post-attention RMSNorm fused the same way, SwiGLU in the epilogue) → down
GEMM + residual.  The final norm is folded into a copy of the LM head.
"""
from __future__ import annotations

import math
import os
from typing import Dict, Optional

import torch

from .. import ops
from ..config import ModelSpec
from ..parallel import comm
from ..parallel.layout import TPLayout
from ..parallel.state import TPState

PREFETCH_ALL = os.environ.get("BRAID_PREFETCH_ALL", "0") == "1"
# decode attention pulls the o_proj weight into L2 while it streams K/V
PREFETCH_ATTN = os.environ.get("BRAID_PREFETCH_ATTN", "0") == "1"
# the down-projection GEMM pulls the next layer's QKV weight into L2 (TP1)
PREFETCH_QKV = os.environ.get("BRAID_PREFETCH_QKV", "0") == "1"


class LayerWeights:
    __slots__ = ("in_norm", "qkv_w", "qkv_b", "q_norm", "k_norm", "o_w", "o_b", "post_norm", "gu_w",
                 "down_w", "in_norm_b", "post_norm_b", "fc_b", "down_b")

    def __init__(self):
        for s in self.__slots__:
            setattr(self, s, None)


class DecoderLM:
    packed_modules_mapping = {
        "q_proj": ("qkv_proj", "q"),
        "k_proj": ("qkv_proj", "k"),
        "v_proj": ("qkv_proj", "v"),
        "gate_proj": ("gate_up_proj", 0),
        "up_proj": ("gate_up_proj", 1),
    }

    def __init__(self, spec: ModelSpec, tp: TPState, dtype: torch.dtype, device: torch.device,
                 max_pos: int):
        self.spec = spec
        self.tp = tp
        self.dtype = dtype
        self.device = device
        self.layout = TPLayout(tp.size, tp.rank, spec.num_heads, spec.num_kv_heads, spec.head_dim,
                               spec.intermediate_size, spec.vocab_size)
        L = self.layout
        D = spec.head_dim
        H = spec.hidden_size
        kw = dict(dtype=dtype, device=device)
        self.qkv_rows = (L.q_heads + 2 * L.kv_heads) * D
        self.layers = []
        for _ in range(spec.num_layers):
            w = LayerWeights()
            w.in_norm = torch.ones(H, **kw)
            w.qkv_w = torch.empty(self.qkv_rows, H, **kw)
            if spec.attention_bias:
                w.qkv_b = torch.zeros(self.qkv_rows, **kw)
            if spec.qk_norm:
                w.q_norm = torch.ones(D, **kw)
                w.k_norm = torch.ones(D, **kw)
            w.o_w = torch.empty(H, L.q_heads * D, **kw)
            w.post_norm = torch.ones(H, **kw)
            w.gu_w = torch.zeros(2 * L.inter_pad, H, **kw)
            w.down_w = torch.zeros(H, L.inter_pad, **kw)
            self.layers.append(w)
        # The input embedding is replicated on every rank (a gather needs no
        # collective); the LM head is vocab-parallel (rows [vocab_start, +local)).
        self.embed = torch.empty(spec.vocab_size, H, **kw)
        self.final_norm = torch.ones(H, **kw)
        self.lm_head = None if spec.tie_word_embeddings else torch.empty(L.vocab_local, H, **kw)
        self.lm_head_folded = None  # lm_head * final_norm, built by finalize()
        self.finalized = False
        # RoPE tables: room for query positions shifted by chunk deltas.
        self.rope_len = 2 * max_pos + 16
        if spec.use_rope:
            self.cos, self.sin = ops.build_cos_sin(D, spec.rope_theta, self.rope_len, spec.rope_scaling, device)
        else:
            self.cos = self.sin = torch.zeros(1, max(1, D // 2), device=device)
        self.scale = 1.0 / math.sqrt(D)
        # ERNIE: interleaved rotary pairs -> neox half split by a row permutation.
        self.rope_perm = None
        if spec.family == "ernie":
            self.rope_perm = torch.cat([torch.arange(0, D, 2), torch.arange(1, D, 2)])

    # ------------------------------------------------------------------ init
    def random_init(self, seed: int = 0, std: float = 0.02, k_norm_range: Optional[float] = None) -> None:
        g = torch.Generator(device=self.device)
        g.manual_seed(seed + 7919 * self.tp.rank)

        def fill(t):
            t.normal_(0.0, std, generator=g)

        L = self.layout
        for w in self.layers:
            fill(w.qkv_w)
            fill(w.o_w)
            gu = w.gu_w.view(-1, 2 * L.block, w.gu_w.shape[1])
            # only the unpadded intermediate rows carry weights
            n_blocks = -(-L.inter // L.block)
            fill(gu[:n_blocks])
            if L.inter % L.block:
                tail = L.inter % L.block
                gu[n_blocks - 1, tail:L.block].zero_()
                gu[n_blocks - 1, L.block + tail:].zero_()
            fill(w.down_w[:, :L.inter])
            if k_norm_range is not None and w.k_norm is not None:
                w.k_norm.uniform_(-k_norm_range, k_norm_range, generator=g)
        if self.tp.size > 1:
            # identical replicated table on every rank
            ge = torch.Generator(device=self.device)
            ge.manual_seed(seed + 104729)
            self.embed.normal_(0.0, std, generator=ge)
        else:
            fill(self.embed)
        if self.lm_head is not None:
            fill(self.lm_head)

    # --------------------------------------------------------------- loading
    def load_hf_tensor(self, name: str, t: torch.Tensor) -> bool:
        """Copy one HF checkpoint tensor (full, unsharded) into this rank's shard."""
        L, S = self.layout, self.spec
        D = S.head_dim
        t = t.to(self.dtype)
        if name in ("model.embed_tokens.weight", "embed_tokens.weight"):
            self.embed.copy_(t)
            return True
        if name in ("lm_head.weight",):
            if self.lm_head is None:
                return True
            self.lm_head.copy_(t[L.vocab_start:L.vocab_start + L.vocab_local])
            return True
        if name in ("model.norm.weight", "norm.weight"):
            self.final_norm.copy_(t)
            return True
        if not name.startswith("model.layers."):
            return False
        parts = name.split(".")
        li = int(parts[2])
        w = self.layers[li]
        sub = ".".join(parts[3:])
        qh0, qh = L.q_head_start, L.q_heads
        kh0, kh = L.kv_head_start, L.kv_heads
        q_rows, kv_rows = qh * D, kh * D

        def head_rows(x, h0, nh, permute):
            x = x.view(-1, D, *x.shape[1:])[h0:h0 + nh]
            if permute and self.rope_perm is not None:
                x = x[:, self.rope_perm.to(x.device)]
            return x.reshape(nh * D, *x.shape[2:])

        if sub == "input_layernorm.weight":
            w.in_norm.copy_(t)
        elif sub == "post_attention_layernorm.weight":
            w.post_norm.copy_(t)
        elif sub in ("self_attn.q_proj.weight", "self_attn.q_proj.bias"):
            dst = w.qkv_w if sub.endswith("weight") else w.qkv_b
            if dst is None:
                return True
            dst[:q_rows].copy_(head_rows(t, qh0, qh, True))
        elif sub in ("self_attn.k_proj.weight", "self_attn.k_proj.bias"):
            dst = w.qkv_w if sub.endswith("weight") else w.qkv_b
            if dst is None:
                return True
            dst[q_rows:q_rows + kv_rows].copy_(head_rows(t, kh0, kh, True))
        elif sub in ("self_attn.v_proj.weight", "self_attn.v_proj.bias"):
            dst = w.qkv_w if sub.endswith("weight") else w.qkv_b
            if dst is None:
                return True
            dst[q_rows + kv_rows:q_rows + 2 * kv_rows].copy_(head_rows(t, kh0, kh, False))
        elif sub == "self_attn.q_norm.weight":
            if w.q_norm is not None:
                w.q_norm.copy_(t)
        elif sub == "self_attn.k_norm.weight":
            if w.k_norm is not None:
                w.k_norm.copy_(t)
        elif sub == "self_attn.o_proj.weight":
            w.o_w.copy_(t[:, qh0 * D:(qh0 + qh) * D])
        elif sub in ("mlp.gate_proj.weight", "mlp.up_proj.weight"):
            rows = t[L.inter_start:L.inter_start + L.inter]
            gu = w.gu_w.view(-1, 2, L.block, t.shape[1])
            half = 0 if "gate" in sub else 1
            flat = gu[:, half].reshape(-1, t.shape[1])
            flat[:L.inter].copy_(rows)
            gu[:, half].copy_(flat.view(-1, L.block, t.shape[1]))
        elif sub == "mlp.down_proj.weight":
            w.down_w[:, :L.inter].copy_(t[:, L.inter_start:L.inter_start + L.inter])
        elif sub.endswith("rotary_emb.inv_freq"):
            pass
        else:
            return False
        return True

    def finalize(self) -> None:
        """Fold each RMSNorm weight into the columns of the GEMM that consumes
        the normalised activations (``W' = W diag(g)``); the GEMM epilogue then
        only scales each token's row by ``1/rms(x)``.  Called once after the
        weights are loaded or initialised."""
        if self.finalized:
            return

        def fold(wt, g):
            wt.copy_((wt.float() * g.float()[None, :]).to(wt.dtype))

        for w in self.layers:
            fold(w.qkv_w, w.in_norm)
            fold(w.gu_w, w.post_norm)
        L = self.layout
        head = self.lm_head if self.lm_head is not None else self.embed[L.vocab_start:L.vocab_start + L.vocab_local]
        folded = (head.float() * self.final_norm.float()[None, :]).to(self.dtype)
        if folded.shape[0] < L.vocab_per_rank:  # equal shards for the logits all-gather
            folded = torch.cat([folded, folded.new_zeros(L.vocab_per_rank - folded.shape[0], folded.shape[1])])
        self.lm_head_folded = folded.contiguous()
        self.finalized = True

    # --------------------------------------------------------------- forward
    def embed_tokens(self, input_ids: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        return ops.embedding(input_ids, self.embed, 0)

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor, slot_mapping: torch.Tensor,
                meta, kv_cache: torch.Tensor, workspace: Optional[Dict] = None) -> torch.Tensor:
        """Return the residual stream ``[T, hidden]`` after the last layer (pre final norm)."""
        S, L = self.spec, self.layout
        assert self.finalized, "call finalize() after loading weights"
        eps = S.rms_norm_eps
        fc = comm.get_fused_comm() if self.tp.size > 1 else None
        if fc is not None and input_ids.is_cuda and fc.can_sp(input_ids.shape[0]):
            return self._forward_sp(fc, input_ids, positions, slot_mapping, meta, kv_cache, workspace)
        # Decode under tensor parallelism: the reduce kernel that waits for the
        # peers' partials pulls leading K-blocks of the next GEMM's weight into
        # L2 meanwhile (HBM is idle then).  BRAID_PREFETCH_ALL=1 makes every
        # launch prefetch the following GEMM's weight too (measured slower on
        # B200 at TP1/TP2: the extra traffic competes with the running kernel).
        T = input_ids.shape[0]
        nxt = ops.prefetch_next if PREFETCH_ALL else (lambda w, t, skip=0: skip)
        residual = self.embed_tokens(input_ids, positions)
        for i, w in enumerate(self.layers):
            following = self.layers[i + 1].qkv_w if i + 1 < len(self.layers) else self.lm_head_folded
            nxt(w.o_w, T)
            q = ops.qkv_gemm(residual, w.qkv_w, w.qkv_b, eps, positions, slot_mapping, kv_cache[i], L.q_heads,
                             L.kv_heads, S.head_dim, self.cos, self.sin, w.q_norm, w.k_norm, eps, S.use_rope)
            gu_done = nxt(w.gu_w, T)
            if PREFETCH_ATTN and not PREFETCH_ALL:
                ops.prefetch_next(w.o_w, T)
            o = ops.attention(q, kv_cache[i], meta, self.cos, self.sin, self.scale, S.use_rope, workspace)
            residual = self._row_parallel(o, w.o_w, residual, w.gu_w, gu_done)
            nxt(w.down_w, T)
            g = ops.linear_swiglu(residual, w.gu_w, rms_eps=eps)
            residual = self._row_parallel(g, w.down_w, residual, following,
                                          pull_next=PREFETCH_QKV and i + 1 < len(self.layers))
        return residual

    def _forward_sp(self, fc, input_ids, positions, slot_mapping, meta, kv_cache, workspace) -> torch.Tensor:
        """Tensor-parallel prefill, sequence-parallel residual stream.

        The residual ``G`` lives in the peer-mapped comm buffer.  Per layer:
        QKV GEMM (waits tile by tile for gathered rows, 1/rms pushed with them)
        → attention → o_proj GEMM → reduce-scatter in its epilogue → owner
        reduce + all-gather of rows and 1/rms → gate/up GEMM (same waits) →
        down GEMM → reduce-scatter → reduce + all-gather.  Replaces the
        all-reduce that the reference's ``RowParallelLinear`` never issued
        (``braidinfer/layers/linear_distributed.py:170-174``).
        """
        S, L = self.spec, self.layout
        eps = S.rms_norm_eps
        G, rstd = fc.sp_begin(input_ids.shape[0])
        ops.embedding(input_ids, self.embed, 0, out=G)
        ops.row_rstd(G, eps, rstd)
        for i, w in enumerate(self.layers):
            q = ops.qkv_gemm(G, w.qkv_w, w.qkv_b, eps, positions, slot_mapping, kv_cache[i], L.q_heads,
                             L.kv_heads, S.head_dim, self.cos, self.sin, w.q_norm, w.k_norm, eps, S.use_rope,
                             rs_vec=rstd, sp=fc.sp_params())
            o = ops.attention(q, kv_cache[i], meta, self.cos, self.sin, self.scale, S.use_rope, workspace)
            fc.sp_linear_reduce_scatter(o.view(o.shape[0], -1), w.o_w, G)
            fc.sp_reduce_allgather(eps)
            g = ops.linear_swiglu(G, w.gu_w, rms_eps=eps, rs_vec=rstd, sp=fc.sp_params())
            fc.sp_linear_reduce_scatter(g, w.down_w, G)
            fc.sp_reduce_allgather(eps)
        fc.sp_wait()
        return G.clone()

    def _row_parallel(self, x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor,
                      w_next: Optional[torch.Tensor] = None, skip: int = 0, pull_next: bool = False) -> torch.Tensor:
        """``residual += x @ w.T`` summed over tensor-parallel ranks; the
        GEMM (and the reduce kernel after it) prefetch ``w_next`` into L2,
        past the ``skip`` leading K-blocks per slice already requested
        (``pull_next``: the single-GPU GEMM prefetches it as well)."""
        T = x.shape[0]
        done = ops.prefetch_next(w_next, T, skip) if PREFETCH_ALL else skip
        if pull_next and not PREFETCH_ALL and self.tp.size == 1:
            ops.prefetch_next(w_next, T)
        if self.tp.size == 1:
            return ops.linear(x, w, residual=residual, out=residual)
        fc = comm.get_fused_comm()
        if fc is not None and fc.can_all_reduce(residual):
            return fc.linear_all_reduce_add(x, w, residual, w_next, done)
        return comm.all_reduce_add(ops.linear(x, w), residual)

    def final_hidden(self, h: torch.Tensor) -> torch.Tensor:
        """Rows fed to the LM head; the final RMSNorm is fused into ``compute_logits``."""
        return h

    def sample_tp(self, h: torch.Tensor, temperature, top_k, top_p, min_p, seed, step, out: torch.Tensor):
        """Tensor parallelism: LM head on this rank's vocab shard (final norm
        folded in), then the sampler exchange over peer memory — no logits
        all-gather.  Returns ``out`` (one token per row, same on every rank)."""
        fc = comm.get_fused_comm()
        local = ops.linear(h, self.lm_head_folded, rms_eps=self.spec.rms_norm_eps)
        return fc.sample(local, self.layout.vocab_start, self.spec.vocab_size, temperature, top_k, top_p, min_p,
                         seed, step, out)

    def compute_logits(self, h: torch.Tensor) -> torch.Tensor:
        """Full-vocabulary logits ``[B, V]`` from residual-stream rows ``h``."""
        local = ops.linear(h, self.lm_head_folded, rms_eps=self.spec.rms_norm_eps)
        if self.tp.size > 1:
            return comm.all_gather_last(local, self.spec.vocab_size)
        return local
