"""Engine configuration.

Field names and defaults of the reference ``Config`` are kept
(``braidinfer/config.py:7-53``) so ``LLM(model, **kwargs)`` accepts the same
keyword arguments; the post-init checks are the same (page size multiple of
16, ``max_model_len`` clamped to the model's position limit, token budget at
least one full sequence).  Added fields cover what the B200 build needs:
tensor parallelism, CUDA-graph decode, device/dtype selection and the
communication timeout of the bounded device-side waits.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from typing import Any, Optional

import torch

from .errors import ConfigurationError


@dataclass
class ModelSpec:
    """Architecture facts extracted from an HF ``config.json``."""

    model_type: str
    family: str  # "llama" | "qwen3" | "gpt2" | "ernie"
    num_layers: int
    hidden_size: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate_size: int
    vocab_size: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    rope_scaling: Optional[dict] = None
    max_position_embeddings: int = 4096
    tie_word_embeddings: bool = False
    attention_bias: bool = False
    qk_norm: bool = False
    use_rope: bool = True
    norm_type: str = "rms"  # "rms" | "layer"
    act: str = "silu"
    eos_token_id: Any = None
    bos_token_id: Any = None
    torch_dtype: str = "bfloat16"

    @classmethod
    def from_hf(cls, hf: Any) -> "ModelSpec":
        get = (lambda k, d=None: hf.get(k, d)) if isinstance(hf, dict) else (lambda k, d=None: getattr(hf, k, d))
        mt = get("model_type")
        if mt == "gpt2":
            hidden = get("n_embd")
            nh = get("n_head")
            inter = get("n_inner") or 4 * hidden
            return cls(model_type=mt, family="gpt2", num_layers=get("n_layer"), hidden_size=hidden,
                       num_heads=nh, num_kv_heads=nh, head_dim=hidden // nh, intermediate_size=inter,
                       vocab_size=get("vocab_size"), rms_norm_eps=get("layer_norm_epsilon", 1e-5),
                       max_position_embeddings=get("n_positions", 1024), tie_word_embeddings=True,
                       attention_bias=True, use_rope=False, norm_type="layer", act="gelu_new",
                       eos_token_id=get("eos_token_id"), bos_token_id=get("bos_token_id"),
                       torch_dtype=str(get("torch_dtype") or get("dtype") or "float32").replace("torch.", ""))
        if mt in ("qwen3", "qwen2"):
            family = "qwen3"
        elif mt in ("llama", "mistral"):
            family = "llama"
        elif mt in ("ernie4_5", "ernie"):
            family = "ernie"
        else:
            raise ConfigurationError(f"unsupported model_type {mt!r}")
        hidden = get("hidden_size")
        nh = get("num_attention_heads")
        hd = get("head_dim") or hidden // nh
        dtype = get("torch_dtype") or get("dtype") or "bfloat16"
        return cls(model_type=mt, family=family, num_layers=get("num_hidden_layers"), hidden_size=hidden,
                   num_heads=nh, num_kv_heads=get("num_key_value_heads") or nh, head_dim=hd,
                   intermediate_size=get("intermediate_size"), vocab_size=get("vocab_size"),
                   rms_norm_eps=get("rms_norm_eps", 1e-6), rope_theta=get("rope_theta", 10000.0) or 10000.0,
                   rope_scaling=get("rope_scaling"), max_position_embeddings=get("max_position_embeddings", 4096),
                   tie_word_embeddings=bool(get("tie_word_embeddings", False)),
                   attention_bias=bool(get("attention_bias", mt == "qwen2") or get("use_bias", False)),
                   qk_norm=(mt == "qwen3"), eos_token_id=get("eos_token_id"), bos_token_id=get("bos_token_id"),
                   torch_dtype=str(dtype).replace("torch.", ""))

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    def param_count(self) -> int:
        h, i, v = self.hidden_size, self.intermediate_size, self.vocab_size
        attn = h * (self.q_size + 2 * self.kv_size) + self.q_size * h
        mlp = (3 if self.act == "silu" else 2) * h * i
        emb = v * h * (1 if self.tie_word_embeddings else 2)
        return self.num_layers * (attn + mlp) + emb


def load_hf_config(model: str) -> dict:
    """Read ``config.json`` of a local checkpoint directory (no network)."""
    path = os.path.join(model, "config.json")
    if not os.path.isfile(path):
        try:
            from transformers import AutoConfig

            return AutoConfig.from_pretrained(model, trust_remote_code=True).to_dict()
        except Exception as e:  # pragma: no cover - depends on HF cache
            raise ConfigurationError(f"Model {model!r} is neither a local directory nor a cached HF id: {e}")
    with open(path) as f:
        return json.load(f)


@dataclass
class Config:
    model: str
    max_num_batched_tokens: int = 16384
    max_num_seqs: int = 256
    max_model_len: int = 4096
    gpu_memory_utilization: float = 0.85
    enforce_eager: bool = False
    hf_config: Any = None
    eos: int = -1
    bos: int = -1
    kvcache_block_size: int = 256
    num_kvcache_blocks: int = -1
    chunk_page_ratio: float = 0.5
    chunk_registry_size: int = 1000
    chunk_persistence_dir: Optional[str] = None
    # --- additions of this build ------------------------------------------
    tensor_parallel_size: int = 1
    device: str = "auto"          # "auto" | "cpu" | "cuda" | "cuda:N"
    dtype: str = "auto"           # "auto" (bf16 on GPU, fp32 on CPU) | "bfloat16" | "float32"
    page_size: Optional[int] = None  # alias of kvcache_block_size
    max_graph_batch: int = 64     # largest decode batch captured in a CUDA graph
    max_prefill_graph_tokens: int = 256  # single-sequence prefills up to this many tokens replay a graph
    comm_backend: str = "fused"   # "fused" (in-kernel peer stores) | "nccl" (baseline)
    comm_timeout_s: float = 5.0
    heartbeat_every: int = 64      # TP: check peer liveness every N engine steps (0 = off)
    shared_prefix_batching: bool = True  # decode: attend once to segments shared by several sequences
    validate_plans: bool = False   # check every step's metadata on the host before upload (also BRAID_VALIDATE_PLAN=1)
    seed: int = 0
    load_weights: bool = True     # False: random-init weights (synthetic benchmarks)
    init_std: float = 0.02
    init_k_norm_range: Optional[float] = None  # random init: Qwen3 k_norm weights uniform in [-r, r]
    spec: Optional[ModelSpec] = field(default=None, repr=False)

    def __post_init__(self):
        if self.page_size is not None:
            self.kvcache_block_size = self.page_size
        self.page_size = self.kvcache_block_size
        if self.hf_config is None:
            self.hf_config = load_hf_config(self.model)
        if self.spec is None:
            self.spec = ModelSpec.from_hf(self.hf_config)
        if self.kvcache_block_size % 16 != 0:
            raise ConfigurationError("kvcache_block_size must be a multiple of 16")
        self.max_model_len = min(self.max_model_len, self.spec.max_position_embeddings)
        if self.max_num_batched_tokens < self.max_model_len:
            raise ConfigurationError("max_num_batched_tokens must be >= max_model_len")
        if self.tensor_parallel_size not in (1, 2, 4, 8):
            raise ConfigurationError("tensor_parallel_size must be 1, 2, 4 or 8")
        if self.comm_backend not in ("fused", "nccl"):
            raise ConfigurationError("comm_backend must be 'fused' or 'nccl'")

    # -- resolved runtime properties ----------------------------------------
    @property
    def torch_device(self) -> torch.device:
        if self.device == "auto":
            if torch.cuda.is_available():
                return torch.device("cuda", torch.cuda.current_device())
            return torch.device("cpu")
        return torch.device(self.device)

    @property
    def torch_dtype(self) -> torch.dtype:
        if self.dtype == "auto":
            return torch.bfloat16 if self.torch_device.type == "cuda" else torch.float32
        return getattr(torch, self.dtype)

    @property
    def use_cuda_graphs(self) -> bool:
        return (not self.enforce_eager) and self.torch_device.type == "cuda"
