"""braidinfer_b200 — a Blackwell-native (sm_100a) LLM inference engine with
chunk-based context management (content-addressed chunks, paged HND KV,
cascade attention with differential RoPE, output-KV retention) and tensor
parallelism over NVLink.

Public API (same names as the reference package ``braidinfer``):
``LLM``, ``SamplingParams``, ``ChunkedLLM``, ``ChunkType``.
"""
from .chunked_llm import ChunkedLLM
from .chunks import Chunk, ChunkType
from .config import Config
from .llm import LLM
from .sampling_params import SamplingParams

__all__ = ["LLM", "SamplingParams", "ChunkedLLM", "ChunkType", "Chunk", "Config"]
__version__ = "0.1.0"
