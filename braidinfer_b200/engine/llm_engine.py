"""The engine: request intake, the step loop, streaming and output retention.

Public surface of ``braidinfer/engine/llm_engine.py:19-567``: ``add_request``,
``step``, ``generate(prompts, sampling_params, stream)`` returning
``[{"text", "token_ids"}]``, the streaming dict protocol (``text``,
``token_ids``, ``cumulative_text``, ``finished`` and a final ``final_output``
record), think-tag aware retention (``get_retained_sequences``,
``release_retained_sequence``, ``release_all_retained_sequences``) and
``generate_from_chunks(composition, ...)``.

Tensor parallelism is SPMD: every rank of a ``torchrun`` job constructs the
engine with the same arguments and issues the same calls; every rank samples
the same token (identical all-gathered logits and counter-based RNG), so the
ranks' schedulers stay in lockstep without exchanging decisions.
"""
from __future__ import annotations

import atexit
import time
from typing import Any, Dict, Iterable, List, Optional, Tuple, Union

from ..config import Config
from ..errors import ConfigurationError
from ..parallel.state import get_tp, init_tp
from ..sampling_params import SamplingParams
from ..utils.logging import get_logger
from ..utils.tracing import nvtx_range
from .chat_format import ChatFormat
from .metrics import MetricsCollector
from .model_runner import ModelRunner
from .scheduler import Scheduler
from .sequence import SegmentRef, Sequence, SequenceStatus

log = get_logger("engine")

THINK_START_DEFAULT = 151667  # Qwen3 "<think>"
THINK_END_DEFAULT = 151668    # Qwen3 "</think>"


def _load_tokenizer(path: str):
    try:
        from transformers import AutoTokenizer

        return AutoTokenizer.from_pretrained(path, use_fast=True, trust_remote_code=True)
    except Exception as e:  # tokenizer-less checkpoints still serve token ids
        log.warning("no tokenizer loaded from %s (%s); text I/O disabled", path, e)
        return None


class LLMEngine:
    def __init__(self, model: str, **kwargs):
        config = Config(model, **kwargs)
        tp = init_tp(config.tensor_parallel_size, timeout_s=max(60.0, config.comm_timeout_s * 6))
        if config.device == "auto" and tp.size > 1 and tp.backend == "nccl":
            import torch

            config.device = f"cuda:{torch.cuda.current_device()}"
        self.config = config
        self.tp = tp
        self.model_runner = ModelRunner(config, tp)
        if tp.size > 1 and config.comm_backend == "fused" and self.model_runner.device.type == "cuda":
            from ..parallel.symm import maybe_enable_fused_comm

            maybe_enable_fused_comm(config, self.model_runner)
        self.page_manager = self.model_runner.allocate_kv()
        self.tokenizer = _load_tokenizer(config.model)
        spec = config.spec
        eos = spec.eos_token_id
        eos_ids = list(eos) if isinstance(eos, (list, tuple)) else [eos]
        if self.tokenizer is not None and self.tokenizer.eos_token_id is not None:
            eos_ids.append(self.tokenizer.eos_token_id)
        eos_ids = [e for e in eos_ids if e is not None]
        config.eos = eos_ids[0] if eos_ids else -1
        bos = spec.bos_token_id
        config.bos = (bos[0] if isinstance(bos, (list, tuple)) else bos) if bos is not None else -1
        self.scheduler = Scheduler(config, self.page_manager, eos_ids)
        self.chat = ChatFormat(self.tokenizer)
        self.metrics = MetricsCollector()
        self._timing_stats: List[float] = []
        self._retained_sequences: Dict[int, Tuple[Sequence, Dict[str, Any]]] = {}
        self.think_token_ids = (THINK_START_DEFAULT, THINK_END_DEFAULT)
        if self.tokenizer is not None:
            ids = [self.tokenizer.convert_tokens_to_ids(t) for t in ("<think>", "</think>")]
            unk = self.tokenizer.unk_token_id
            if all(i is not None and i != unk for i in ids):
                self.think_token_ids = tuple(ids)
        self._heartbeat = None
        self._steps = 0
        if tp.size > 1 and config.heartbeat_every > 0:
            from ..parallel.health import Heartbeat

            self._heartbeat = Heartbeat(timeout_s=max(1.0, config.comm_timeout_s))
        if config.use_cuda_graphs:
            self.model_runner.capture_all(min(config.max_graph_batch, config.max_num_seqs))
        self._closed = False
        atexit.register(self.exit)

    # ----------------------------------------------------------- lifecycle
    def exit(self) -> None:
        if getattr(self, "_closed", True):
            return
        self._closed = True
        try:
            atexit.unregister(self.exit)  # a closed engine can be freed (weights, KV pool)
        except Exception:
            pass
        try:
            self.release_all_retained_sequences()
            # graphs may hold NCCL calls (TP): release them before the process group goes away
            # (the prebuilt next-step plan refers to its graph slot too)
            self.model_runner._spec = None
            self.model_runner.graphs.clear()
            self.model_runner.graphs_gather.clear()
            self.model_runner.graphs_shared.clear()
            self.model_runner.prefill_graphs.clear()
            if self.model_runner.device.type == "cuda":
                import torch

                torch.cuda.synchronize(self.model_runner.device)
        except Exception:
            pass

    def __del__(self):
        try:
            self.exit()
        except Exception:
            pass

    # ------------------------------------------------------------- intake
    def encode(self, text: str) -> List[int]:
        if self.tokenizer is None:
            raise ConfigurationError("no tokenizer: pass token ids")
        return list(self.tokenizer.encode(text))

    def decode(self, ids: List[int]) -> str:
        if self.tokenizer is None or not ids:
            return ""
        return self.tokenizer.decode(ids, skip_special_tokens=False)

    def _prepare(self, seq: Sequence, sp: SamplingParams) -> None:
        for st in sp.stop_strings():
            if self.tokenizer is None:
                continue
            toks = list(self.tokenizer.encode(st, add_special_tokens=False))
            if len(toks) == 1:
                if toks[0] not in seq.stop_token_ids:
                    seq.stop_token_ids.append(toks[0])
            elif toks:
                seq.stop_sequences.append(toks)
        seq.arrival_time = time.perf_counter()

    def add_request(self, prompt: Union[str, List[int]], sampling_params: SamplingParams,
                    segments: Optional[List[SegmentRef]] = None, pos_base: int = 0,
                    first_hidden=None) -> Sequence:
        if isinstance(prompt, str):
            prompt = self.encode(prompt)
        seq = Sequence(prompt, sampling_params, segments=segments, pos_base=pos_base)
        seq.first_hidden = first_hidden
        if seq.num_tokens == 0 and first_hidden is None:
            raise ConfigurationError("empty prompt")
        self._prepare(seq, sampling_params)
        self.scheduler.add(seq)
        return seq

    # --------------------------------------------------------------- step
    def step(self) -> List[Sequence]:
        self._steps += 1
        if self._heartbeat is not None and self._steps % self.config.heartbeat_every == 0:
            self._heartbeat.check(self._steps)  # PeerFailureError before any collective of this step
        seqs, is_prefill = self.scheduler.schedule()
        if not seqs:
            return []
        t0 = time.perf_counter()
        ntok = sum(max(1, s.num_tokens - s.num_cached_tokens) for s in seqs)
        with nvtx_range(f"{'prefill' if is_prefill else 'decode'} b={len(seqs)} t={ntok}"):
            token_ids = self.model_runner.run(seqs, is_prefill)
        now = time.perf_counter()
        dt = now - t0
        self._timing_stats.append(dt)
        self.metrics.record_step(is_prefill, ntok if is_prefill else len(seqs), dt)
        for s in seqs:
            if s.first_token_time is None:
                s.first_token_time = now
                self.metrics.record_ttft(now - s.arrival_time)
        finished = self.scheduler.postprocess(seqs, token_ids)
        for seq in finished:
            if seq.retain_output_cache:
                self._retained_sequences[seq.seq_id] = (seq, self.page_manager.get_sequence_cache_info(seq))
        if finished:
            self.metrics.record_finished(len(finished))
        return finished

    def _run_until(self, seqs: List[Sequence]) -> None:
        pending = {s.seq_id for s in seqs}
        while pending:
            for s in self.step():
                pending.discard(s.seq_id)
            if not self.scheduler.running and not self.scheduler.waiting and pending:
                raise RuntimeError("scheduler drained with unfinished sequences")

    def _output(self, seq: Sequence) -> Dict[str, Any]:
        return {"text": self.decode(seq.completion_token_ids), "token_ids": list(seq.completion_token_ids),
                "seq_id": seq.seq_id, "finish_reason": seq.finish_reason}

    def generate(self, prompts, sampling_params: Optional[Union[SamplingParams, List[SamplingParams]]] = None,
                 stream: bool = False, use_tqdm: bool = False):
        if isinstance(prompts, str) or (isinstance(prompts, list) and prompts and isinstance(prompts[0], int)):
            prompts = [prompts]
        sps = sampling_params if isinstance(sampling_params, list) else [sampling_params or SamplingParams()] * len(prompts)
        self._timing_stats = []
        seqs = [self.add_request(p, sp) for p, sp in zip(prompts, sps)]
        if stream:
            return self._generate_stream(seqs)
        self._run_until(seqs)
        return [self._output(s) for s in seqs]

    def _generate_stream(self, seqs: List[Sequence]) -> Iterable[Dict[str, Any]]:
        sent = {s.seq_id: 0 for s in seqs}
        pending = {s.seq_id: s for s in seqs}
        while pending:
            finished = self.step()
            for s in list(pending.values()):
                comp = s.completion_token_ids
                if len(comp) > sent[s.seq_id]:
                    new = comp[sent[s.seq_id]:]
                    sent[s.seq_id] = len(comp)
                    yield {"text": self.decode(new), "token_ids": new, "cumulative_text": self.decode(comp),
                           "finished": False, "seq_id": s.seq_id}
            for s in finished:
                if s.seq_id in pending:
                    del pending[s.seq_id]
                    comp = s.completion_token_ids
                    yield {"text": "", "token_ids": [], "cumulative_text": self.decode(comp), "finished": True,
                           "seq_id": s.seq_id, "final_output": self._output(s)}
            if not self.scheduler.running and not self.scheduler.waiting and pending:
                raise RuntimeError("scheduler drained with unfinished sequences")

    # ----------------------------------------------------------- metrics
    def get_metrics(self) -> Dict[str, Any]:
        m = self.metrics.summary()
        m["kv_pool"] = self.page_manager.stats()
        m["preemptions"] = self.scheduler.num_preemptions
        return m

    # ------------------------------------------------------------ retention
    def _find_think_tag_positions(self, token_ids: List[int]) -> Optional[Tuple[int, int]]:
        t0, t1 = self.think_token_ids
        start = None
        for i, t in enumerate(token_ids):
            if t == t0 and start is None:
                start = i
            elif t == t1 and start is not None:
                return (start, i)
        return (start, len(token_ids) - 1) if start is not None else None

    def get_retained_sequences(self) -> Dict[int, Dict[str, Any]]:
        out = {}
        for sid, (seq, info) in self._retained_sequences.items():
            comp = seq.completion_token_ids
            tp_ = self._find_think_tag_positions(comp)
            visible = comp[:tp_[0]] + comp[tp_[1] + 1:] if tp_ else comp
            out[sid] = {"text": self.decode(visible), "token_ids": list(comp), "think_positions": tp_,
                        "cache_info": info, "prompt_length": seq.total_prompt_len,
                        "completion_length": seq.num_completion_tokens}
        return out

    def retained_sequence(self, seq_id: int) -> Optional[Sequence]:
        e = self._retained_sequences.get(seq_id)
        return e[0] if e else None

    def release_retained_sequence(self, seq_id: int) -> bool:
        e = self._retained_sequences.pop(seq_id, None)
        if e is None:
            return False
        self.page_manager.deallocate(e[0])
        return True

    def release_all_retained_sequences(self) -> None:
        for sid in list(self._retained_sequences):
            self.release_retained_sequence(sid)

    # --------------------------------------------------------------- chunks
    def prefill_chunks(self, chunks: List[Any]) -> None:
        """Allocate pages and run the independent causal prefill of ``chunks``.

        Each chunk is rotated at ``chunk.cached_position_start`` and stores the
        final hidden state of its last token.
        """
        jobs, todo = [], []
        for c in chunks:
            if c.kv_cache_allocated:
                continue
            if not c.token_ids:
                c.page_table, c.kv_length, c.kv_offset = [], 0, 0
                c.kv_cache_allocated = True
                continue
            pages = self.page_manager.allocate_for_chunk(c.chunk_id, len(c.token_ids))
            c.page_table, c.kv_length, c.kv_offset = pages, len(c.token_ids), 0
            jobs.append((list(c.token_ids), c.cached_position_start, pages))
            todo.append(c)
        if not jobs:
            return
        hn = self.model_runner.prefill_chunks(jobs)
        for i, c in enumerate(todo):
            c.last_hidden = hn[i].detach().clone()
            c.kv_cache_allocated = True

    def generate_from_chunks(self, composition: Dict[str, Any], sampling_params: SamplingParams,
                             stream: bool = False):
        """Run a composition ``{system_chunk, context_chunks, query_chunk}``.

        Chunks with KV are attended through the cascade; a query chunk without
        KV (the default) is prefilled as the request's private prompt so it
        attends to every chunk before it.  Yields stream records, or (non-stream)
        a single final ``{"text", "token_ids"}`` dict.
        """
        seq = self.add_composition(composition, sampling_params)
        if stream:
            yield from self._generate_stream([seq])
            return
        self._run_until([seq])
        yield self._output(seq)

    def add_composition(self, composition: Dict[str, Any], sampling_params: SamplingParams) -> Sequence:
        sysc = composition.get("system_chunk")
        ctx = list(composition.get("context_chunks") or [])
        q = composition.get("query_chunk")
        cached = [c for c in [sysc] + ctx if c is not None]
        private: List[int] = []
        if q is not None:
            if q.kv_cache_allocated:
                cached.append(q)
            else:
                private.extend(q.token_ids)
        private.extend(self.chat.generation_prompt())
        segs, pos = [], 0
        for c in cached:
            n = c.kv_length if c.kv_cache_allocated else 0
            if n:
                segs.append(SegmentRef(pages=list(c.page_table), offset=c.kv_offset, length=n, pos0=pos,
                                       delta=pos - c.cached_position_start, chunk=c))
            pos += n
        first_hidden = None
        if not private:
            last = next((c for c in reversed(cached) if c.kv_length), None)
            if last is None:
                raise ConfigurationError("composition has no tokens")
            first_hidden = last.last_hidden
            if first_hidden is None:
                # retained output chunk: no stored hidden; re-feed its last token privately
                raise ConfigurationError("composition ends on a chunk without a stored final state; "
                                         "add a query chunk")
        return self.add_request(private, sampling_params, segments=segs, pos_base=pos, first_hidden=first_hidden)
