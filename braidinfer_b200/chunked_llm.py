"""``ChunkedLLM``: the chunk-based context API.

Method names, arguments and return dictionaries follow
``braidinfer/chunked_llm.py:16-707``: ``register_chunk``, ``list_chunks``,
``get_chunk``, ``delete_chunk``, ``clear_chunks``, ``evict_unused_chunks``,
``generate_from_chunks``, ``batch_generate_from_chunks``,
``preview_composition``, ``generate``, ``get_chunk_stats``,
``register_output_chunk_from_retained``, ``generate_and_retain_output``.

Semantics are the intended ones rather than the reference's defects:

* a chunk is prefilled *once*, independently (causal within itself) at the
  position it first appears, and reused in any later composition through
  query-side differential RoPE;
* the query chunk is by default the request's private prompt, so it attends
  to the system prompt and contexts (``cache_query_chunks=True`` prefills it
  independently too, for exact block-causal semantics);
* ``batch_generate_from_chunks`` batches the compositions in one engine run
  and reuses their chunk KV (the reference re-templated strings);
* retained outputs become OUTPUT chunks that *keep their KV pages*
  (refcounted), so reusing them costs no prefill;
* memory statistics count real pages of this model and layout.
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Union

from .chunk_registry import ChunkRegistry
from .chunks import Chunk, ChunkNotFoundError, ChunkType, InvalidCompositionError
from .llm import LLM
from .sampling_params import SamplingParams

CASCADE_LEVEL = {ChunkType.SYSTEM_PROMPT: 0, ChunkType.CONTEXT: 1, ChunkType.OUTPUT: 1, ChunkType.QUERY: 2}


def _sp(sampling_params) -> SamplingParams:
    if sampling_params is None:
        return SamplingParams()
    if isinstance(sampling_params, SamplingParams):
        return sampling_params
    return SamplingParams(**sampling_params)


class ChunkedLLM:
    def __init__(self, model_path: str, max_chunks: int = 1000, chunk_memory_ratio: float = 0.5,
                 enable_deduplication: bool = True, cache_query_chunks: bool = False, **llm_kwargs):
        self.model_path = model_path
        self.chunk_memory_ratio = chunk_memory_ratio
        self.cache_query_chunks = cache_query_chunks
        self.llm = LLM(model_path, **llm_kwargs)
        self.tokenizer = self.llm.tokenizer
        self.page_manager = self.llm.page_manager
        self.registry = ChunkRegistry(max_chunks=max_chunks, enable_deduplication=enable_deduplication,
                                      page_manager=self.page_manager)
        self.page_manager.evictor = self._evict_one
        self._allocated_chunks: Dict[str, int] = {}

    # ----------------------------------------------------------- helpers
    def _evict_one(self) -> bool:
        return self.registry.evict_lru_with_kv(lambda c: self.page_manager.is_shared(c.page_table or []))

    def _chunk_pages_budget_ok(self) -> None:
        """Honour ``chunk_memory_ratio`` as a soft cap on chunk-owned pages."""
        pm = self.page_manager
        cap = int(self.chunk_memory_ratio * (pm.num_pages - 1))
        while pm.stats()["chunk_pages"] > cap and self._evict_one():
            pass

    # ------------------------------------------------------------ registry
    def register_chunk(self, content: str, chunk_type: ChunkType, metadata: Optional[Dict[str, Any]] = None,
                       global_position_start: Optional[int] = None, token_ids: Optional[List[int]] = None) -> str:
        role = (metadata or {}).get("role")
        if token_ids is None:
            token_ids = self.llm.chat.chunk_tokens(chunk_type, content, role)
        chunk = Chunk.from_content(content, chunk_type, metadata=metadata, token_ids=token_ids)
        if global_position_start is not None:
            chunk.global_position_start = chunk.cached_position_start = global_position_start
        return self.registry.register(chunk)

    def list_chunks(self, chunk_type: Optional[ChunkType] = None,
                    metadata_filter: Optional[Dict[str, Any]] = None) -> List[Dict[str, Any]]:
        return self.registry.list_chunks(chunk_type, metadata_filter)

    def get_chunk(self, chunk_id: str) -> Dict[str, Any]:
        c = self.registry.get(chunk_id)
        return {"chunk_id": c.chunk_id, "chunk_type": c.chunk_type.value, "content": c.content,
                "token_count": c.token_count, "metadata": c.metadata, "created_at": c.created_at,
                "last_accessed": c.last_accessed, "access_count": c.access_count,
                "kv_cache_allocated": c.kv_cache_allocated, "cascade_level": c.cascade_level}

    def delete_chunk(self, chunk_id: str) -> bool:
        self._allocated_chunks.pop(chunk_id, None)
        return self.registry.delete(chunk_id)

    def clear_chunks(self, chunk_type: Optional[ChunkType] = None) -> int:
        n = self.registry.clear(chunk_type)
        self._allocated_chunks = {k: v for k, v in self._allocated_chunks.items() if k in self.registry}
        return n

    def evict_unused_chunks(self, max_age_seconds: float = 3600) -> int:
        n = self.registry.evict_unused_chunks(max_age_seconds)
        self._allocated_chunks = {k: v for k, v in self._allocated_chunks.items() if k in self.registry}
        return n

    # --------------------------------------------------------- generation
    def _resolve(self, system_chunk_id: str, query_chunk_id: str, context_chunk_ids: Optional[List[str]]):
        sysc = self.registry.get(system_chunk_id)
        if sysc.chunk_type != ChunkType.SYSTEM_PROMPT:
            raise InvalidCompositionError(f"Chunk {system_chunk_id} is not a system prompt")
        q = self.registry.get(query_chunk_id)
        if q.chunk_type != ChunkType.QUERY:
            raise InvalidCompositionError(f"Chunk {query_chunk_id} is not a query")
        ctx = []
        for cid in context_chunk_ids or []:
            c = self.registry.get(cid)
            if c.chunk_type not in (ChunkType.CONTEXT, ChunkType.OUTPUT):
                raise InvalidCompositionError(f"Chunk {cid} is not a context or output chunk")
            ctx.append(c)
        return sysc, ctx, q

    def _place(self, sysc: Chunk, ctx: List[Chunk], q: Chunk) -> List[Chunk]:
        """Assign global positions; return the chunks whose KV must be computed."""
        pos, todo = 0, []
        cached = [sysc] + ctx + ([q] if self.cache_query_chunks else [])
        for c in [sysc] + ctx + [q]:
            c.global_position_start = pos
            c.global_position_end = pos + len(c.token_ids)
            pos = c.global_position_end
        for c in cached:
            if not c.kv_cache_allocated:
                c.cached_position_start = c.global_position_start
                c.cascade_level = CASCADE_LEVEL[c.chunk_type]
                todo.append(c)
        return todo

    def _ensure_kv(self, chunks: List[Chunk]) -> None:
        if chunks:
            self.llm.prefill_chunks(chunks)
            for c in chunks:
                self._allocated_chunks[c.chunk_id] = c.cascade_level
            self._chunk_pages_budget_ok()

    def generate_from_chunks(self, system_chunk_id: str, query_chunk_id: str,
                             context_chunk_ids: Optional[List[str]] = None, sampling_params=None,
                             stream: bool = False):
        sysc, ctx, q = self._resolve(system_chunk_id, query_chunk_id, context_chunk_ids)
        self._ensure_kv(self._place(sysc, ctx, q))
        comp = {"system_chunk": sysc, "context_chunks": ctx, "query_chunk": q}
        gen = self.llm.generate_from_chunks(comp, _sp(sampling_params), stream)
        if stream:
            return gen
        final = None
        for item in gen:
            final = item
        return final if final else {"text": "", "token_ids": []}

    def batch_generate_from_chunks(self, requests: List[Dict[str, Any]], sampling_params=None) -> List[Dict[str, Any]]:
        sp = _sp(sampling_params)
        comps, todo = [], []
        for r in requests:
            sysc, ctx, q = self._resolve(r["system_chunk_id"], r["query_chunk_id"], r.get("context_chunk_ids"))
            # positions differ per composition; chunks keep the position of their first prefill
            for c in self._place(sysc, ctx, q):
                if c not in todo:
                    todo.append(c)
            comps.append({"system_chunk": sysc, "context_chunks": ctx, "query_chunk": q})
        self._ensure_kv(todo)
        seqs = [self.llm.add_composition(c, sp) for c in comps]
        self.llm._run_until(seqs)
        return [{"text": o["text"], "token_ids": o["token_ids"]} for o in (self.llm._output(s) for s in seqs)]

    def preview_composition(self, system_chunk_id: str, query_chunk_id: str,
                            context_chunk_ids: Optional[List[str]] = None) -> Dict[str, Any]:
        sysc = self.registry.get(system_chunk_id)
        q = self.registry.get(query_chunk_id)
        ctx = [self.registry.get(c) for c in context_chunk_ids or []]
        total = sysc.token_count + q.token_count + sum(c.token_count for c in ctx)
        per_tok = self.page_manager.bytes_per_page / self.page_manager.page_size
        uncached = sum(c.token_count for c in [sysc] + ctx if not c.kv_cache_allocated)
        return {"total_tokens": total, "num_levels": 1 + (1 if ctx else 0) + 1,
                "memory_bytes": int(total * per_tok), "tokens_to_prefill": uncached + q.token_count,
                "chunks": {"system": sysc.chunk_id, "contexts": [c.chunk_id for c in ctx], "query": q.chunk_id}}

    def generate(self, system_prompt: str, query: str, context: Optional[Union[str, List[str]]] = None,
                 sampling_params=None, persist_chunks: bool = True) -> Dict[str, Any]:
        sid = self.register_chunk(system_prompt, ChunkType.SYSTEM_PROMPT)
        qid = self.register_chunk(query, ChunkType.QUERY)
        cids = []
        if context:
            for c in [context] if isinstance(context, str) else context:
                cids.append(self.register_chunk(c, ChunkType.CONTEXT))
        out = self.generate_from_chunks(sid, qid, cids or None, sampling_params)
        out["chunk_ids"] = {"system": sid, "context": cids, "query": qid}
        if not persist_chunks:
            for cid in [sid, qid] + cids:
                self.delete_chunk(cid)
        return out

    def get_chunk_stats(self) -> Dict[str, Any]:
        st = self.registry.get_stats()
        pm = self.page_manager
        pages = set()
        tokens = 0
        for c in self.registry.chunks():
            tokens += c.token_count
            if c.kv_cache_allocated and c.page_table:
                pages.update(c.page_table)
        st["memory_used_mb"] = len(pages) * pm.bytes_per_page / (1024 * 1024)
        st["total_tokens"] = tokens
        st["kv_pages_used"] = len(pages)
        return st

    # ---------------------------------------------------------- retention
    def register_output_chunk_from_retained(self, seq_id: int, metadata: Optional[Dict[str, Any]] = None) -> Optional[str]:
        info = self.llm.get_retained_sequences().get(seq_id)
        seq = self.llm.retained_sequence(seq_id)
        if not info or seq is None:
            return None
        md = dict(metadata or {})
        md.update({"source": "output", "seq_id": seq_id, "prompt_length": info["prompt_length"],
                   "completion_length": info["completion_length"],
                   "has_think_tags": info["think_positions"] is not None})
        comp = list(seq.completion_token_ids)
        cid = self.register_chunk(info["text"], ChunkType.OUTPUT, metadata=md, token_ids=comp)
        c = self.registry.get(cid)
        if not c.kv_cache_allocated and comp:
            ps = self.page_manager.page_size
            k0 = seq.num_prompt_tokens
            pages = seq.pages[k0 // ps: -(-seq.num_tokens // ps)]
            self.page_manager.adopt_for_chunk(cid, pages, len(comp))
            c.page_table, c.kv_offset, c.kv_length = list(pages), k0 % ps, len(comp)
            c.cached_position_start = seq.pos_base + k0
            c.kv_cache_allocated = True
        c.cascade_level = 1
        self._allocated_chunks[cid] = 1
        return cid

    def generate_and_retain_output(self, system_prompt: str, query: str,
                                   context: Optional[Union[str, List[str]]] = None, sampling_params=None,
                                   persist_chunks: bool = True) -> Dict[str, Any]:
        if isinstance(sampling_params, SamplingParams):
            sp = dict(sampling_params.__dict__)
        else:
            sp = dict(sampling_params or {})
        sp["retain_output_cache"] = True
        out = self.generate(system_prompt, query, context, sp, persist_chunks)
        sid = out.get("seq_id")
        if sid is None:
            ret = self.llm.get_retained_sequences()
            sid = max(ret) if ret else None
        if sid is not None:
            out["output_chunk_id"] = self.register_output_chunk_from_retained(sid, metadata={"query": query})
            out["retained_seq_id"] = sid
        return out

    # Convenience passthroughs
    def get_retained_sequences(self):
        return self.llm.get_retained_sequences()

    def release_retained_sequence(self, seq_id: int) -> bool:
        return self.llm.release_retained_sequence(seq_id)
