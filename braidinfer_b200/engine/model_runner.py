"""Runs the model: builds the per-step plan, executes eager prefill and
CUDA-graph decode, samples on the device.

Responsibilities of ``braidinfer/engine/model_runner.py:17-307`` (prepare
inputs, run model, sample, chunk prefill) re-designed for throughput:

* one packed int32 metadata buffer per step (one H2D copy);
* decode runs as a captured CUDA graph per batch bucket (the reference
  stored ``enforce_eager`` and never read it); padded rows write to the pool's
  scratch page;
* tokens are sampled on the device and read back once per step (the only
  D2H copy), instead of per-layer ``.item()`` syncs;
* chunk prefill is a normal batched forward with causal attention restricted
  to the chunk (the reference returned zeros from chunk prefill,
  ``braidinfer/layers/attention.py:143-144``).
"""
from __future__ import annotations

import os
import time
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from .. import ops
from ..config import Config
from ..errors import PlanValidationError
from ..models import build_model
from ..parallel.state import TPState
from ..utils.logging import get_logger
from ..utils.tracing import nvtx_range
from .batch import FwdItem, Plan, build_plan, find_shared_group, make_meta, pack, unpack, validate_plan
from .page_manager import PageManager
from .sequence import Sequence

log = get_logger("runner")

GRAPH_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 192, 256)
# token counts of single-sequence prefill graphs (a query or turn appended to cached chunks)
PREFILL_BUCKETS = (16, 32, 64, 128, 256)


def _num_sms(device) -> int:
    if device.type == "cuda":
        return torch.cuda.get_device_properties(device).multi_processor_count
    return 1


class _GraphSlot:
    def __init__(self):
        self.graph = None
        self.meta_buf = None
        self.sizes = None
        self.fbuf = None
        self.ibuf = None
        self.lbuf = None
        self.out = None
        self.hidden = None
        self.seg_cap = 0
        self.page_cap = 0
        self.num_splits = 1
        self.launches = 0
        self.dev_all = None  # device buffer of fbuf / ibuf / lbuf / meta_buf (views)
        self.pin_all = None  # its pinned host mirror (pin_l / pin_f / pin_k / pin_meta are numpy views)
        self.pin_meta = self.pin_f = self.pin_k = self.pin_l = self.pin_out = self.pin_status = None


class ModelRunner:
    def __init__(self, config: Config, tp: TPState):
        self.config = config
        self.tp = tp
        self.device = config.torch_device
        self.dtype = config.torch_dtype
        spec = config.spec
        self.spec = spec
        t0 = time.time()
        self.model = build_model(spec, tp, self.dtype, self.device, config.max_model_len)
        if config.load_weights:
            from ..utils.loader import load_model

            load_model(self.model, config.model)
        else:
            self.model.random_init(seed=config.seed, std=config.init_std, k_norm_range=config.init_k_norm_range)
        self.model.finalize()
        log.info("model ready in %.1fs", time.time() - t0)
        self.page_manager: Optional[PageManager] = None
        self.page_size = config.kvcache_block_size
        # decode graphs per batch bucket; under tensor parallelism with the
        # peer-memory runtime these sample through the record exchange, and
        # steps whose settings need the full distribution replay the
        # logits-all-gather variant (graphs_gather)
        self.graphs: Dict[int, _GraphSlot] = {}
        self.graphs_gather: Dict[int, _GraphSlot] = {}
        # decode graphs for steps with a shared-prefix group, keyed (bucket, TP sampling)
        self.graphs_shared: Dict[Tuple[int, bool], _GraphSlot] = {}
        self.sms = _num_sms(self.device)
        self.timing = {"steps": 0, "prefill_tokens": 0, "decode_tokens": 0}
        self.capture_logits: Optional[list] = None  # debug/test hook (eager steps only)
        self._spec = None  # (graph slot, batch state key, packed plan) of the next decode step
        self.validate = config.validate_plans or os.environ.get("BRAID_VALIDATE_PLAN") == "1"
        self.event_log: Optional[list] = None  # (start, end) CUDA events around each graph replay
        self.fused_comm = None  # set when the peer-memory TP runtime is enabled
        self.prefill_graphs: Dict[int, _GraphSlot] = {}
        self.last_h2d_bytes = 0

    # ------------------------------------------------------------- KV pool
    def kv_bytes_per_page(self) -> int:
        L = self.model.layout
        return 2 * self.spec.num_layers * L.kv_heads * self.page_size * self.spec.head_dim * \
            torch.tensor([], dtype=self.dtype).element_size()

    def auto_num_pages(self) -> int:
        cfg = self.config
        if cfg.num_kvcache_blocks > 0:
            return cfg.num_kvcache_blocks
        if self.device.type != "cuda":
            return 64
        free, total = torch.cuda.mem_get_info(self.device)
        used = total - free
        act = cfg.max_num_batched_tokens * self.spec.hidden_size * 64 + (2 << 30)
        budget = total * cfg.gpu_memory_utilization - used - act
        n = int(budget // self.kv_bytes_per_page())
        if self.tp.size > 1:
            import torch.distributed as dist

            t = torch.tensor([n], device=self.device)
            dist.all_reduce(t, op=dist.ReduceOp.MIN, group=self.tp.group)
            n = int(t.item())
        return max(n, 16)

    def allocate_kv(self) -> PageManager:
        L = self.model.layout
        n = self.auto_num_pages()
        self.page_manager = PageManager(n, self.page_size, self.spec.num_layers, L.kv_heads, self.spec.head_dim,
                                        self.dtype, self.device)
        log.info("KV pool: %d pages x %d tokens (%.2f GB)", n, self.page_size,
                 n * self.kv_bytes_per_page() / 1e9)
        return self.page_manager

    # ------------------------------------------------------------ forward
    def _decode_splits(self, batch: int, max_kv: Optional[int] = None) -> int:
        L = self.model.layout
        work = max(1, batch * L.kv_heads)
        # as many key splits as keep every CTA resident in one wave (2 per SM);
        # past 16 the split merge costs more than the shorter key loops save
        ns = max(1, min(16, (2 * self.sms) // work))
        if max_kv is not None:
            ns = max(1, min(ns, -(-max_kv // 64)))
        return ns

    def _upload(self, plan: Plan):
        host = pack(plan)
        if self.device.type == "cuda":
            buf = torch.from_numpy(host).pin_memory().to(self.device, non_blocking=True)
        else:
            buf = torch.from_numpy(host)
        return unpack(buf, plan.sizes)

    def _sampling_tensors(self, seqs: List[Sequence], pad: int = 0):
        n = len(seqs) + pad
        f = np.zeros((3, n), dtype=np.float32)
        k = np.zeros(n, dtype=np.int32)
        l = np.zeros((2, n), dtype=np.int64)
        for i, s in enumerate(seqs):
            f[0, i], f[1, i], f[2, i] = s.temperature, s.top_p, s.min_p
            k[i] = s.top_k
            l[0, i], l[1, i] = s.seed, s.num_completion_tokens
        f[1, len(seqs):] = 1.0
        return f, k, l

    def _check_plan(self, plan: Plan) -> None:
        if self.validate:
            validate_plan(plan, self.page_size, self.page_manager.num_pages, getattr(self.model, "rope_len", None))

    def _to_dev(self, a: np.ndarray) -> torch.Tensor:
        t = torch.from_numpy(a)
        if self.device.type == "cuda":
            return t.pin_memory().to(self.device, non_blocking=True)
        return t

    def forward_items(self, items: List[FwdItem], group: Optional[tuple] = None) -> torch.Tensor:
        """Eager forward; returns final-normed hidden rows of items with ``logits=True``.
        ``group``: shared-prefix group of a decode batch (members first)."""
        plan = build_plan(items, self.page_size, group=group)
        self._check_plan(plan)
        views = self._upload(plan)
        ns = self._decode_splits(plan.num_seqs, plan.max_kv_len) if plan.decode else 1
        sh = self._shared_splits(plan.num_seqs, ns) if group is not None and group[0] > 0 else 0
        meta = make_meta(views, plan, ns, shared_splits=sh)
        kv = self.page_manager.kv_cache
        with nvtx_range(f"forward t={plan.sizes['input_ids']}"):
            h = self.model.forward(views["input_ids"], views["positions"], views["slots"], meta, kv)
        rows = h.index_select(0, views["logits_idx"].long()) if plan.sizes["logits_idx"] else h[:0]
        return self.model.final_hidden(rows)

    def _items_for(self, seqs: List[Sequence]) -> List[FwdItem]:
        items = []
        for s in seqs:
            k0 = s.num_cached_tokens
            toks = s.token_ids[k0:]
            items.append(FwdItem(tokens=toks, pos0=s.pos_base + k0, priv_index0=k0, priv_pages=s.pages,
                                 priv_pos0=s.pos_base, segments=s.segments, logits=True))
        return items

    def sample(self, hn: torch.Tensor, seqs: List[Sequence]) -> torch.Tensor:
        with nvtx_range("sample"):
            return self._sample(hn, seqs)

    def _sample(self, hn: torch.Tensor, seqs: List[Sequence]) -> torch.Tensor:
        logits = self.model.compute_logits(hn)
        if self.capture_logits is not None:
            self.capture_logits.append(logits.float().cpu())
        f, k, l = self._sampling_tensors(seqs)
        ft, kt, lt = self._to_dev(f), self._to_dev(k), self._to_dev(l)
        return ops.sample(logits, ft[0], kt, ft[1], ft[2], lt[0], lt[1],
                          all_greedy=all(s.temperature == 0 for s in seqs))

    # ------------------------------------------------- shared-prefix decode
    def _shared_splits(self, n_seqs: int, own_splits: int) -> int:
        """Key splits of the shared-prefix pass: about one wave of resident
        CTAs over (query tiles x KV heads), within the 32 partial slots.  The
        tcgen05 prefill kernel takes 256-row tiles at one CTA per SM, the
        mma.sync kernel 64-row tiles at two."""
        L = self.model.layout
        G = max(1, L.q_heads // max(1, L.kv_heads))
        rows = 64
        if self.device.type == "cuda":
            from ..ops._ext import ext
            rows = int(ext().attn_prefill_tile_rows(L.head_dim))
        per_sm = 1 if rows > 64 else 2
        qt = -(-n_seqs * G // rows)
        want = max(1, (per_sm * self.sms) // max(1, qt * L.kv_heads))
        return max(1, min(want, 32 - own_splits, 24))

    def _shared_group(self, seqs: List[Sequence]):
        """Reorder a decode batch so a shared-prefix group comes first; returns
        ``(seqs, items, group)`` (``group`` None when no segment is shared)."""
        items = self._items_for(seqs)
        if not self.config.shared_prefix_batching or len(seqs) < 2 or not hasattr(self.model, "layout"):
            return seqs, items, None
        found = find_shared_group(items, self.page_size)
        if found is None:
            return seqs, items, None
        members, keys = found
        rest = [i for i in range(len(seqs)) if i not in set(members)]
        order = members + rest
        return [seqs[i] for i in order], [items[i] for i in order], (len(members), keys)

    def run(self, seqs: List[Sequence], is_prefill: bool) -> List[int]:
        """One engine step for ``seqs``; returns one sampled token per sequence."""
        self.timing["steps"] += 1
        if not is_prefill and all(s.num_tokens > s.num_cached_tokens for s in seqs):
            ordered, items, group = self._shared_group(seqs)
            if group is not None:
                out = None
                if self.config.use_cuda_graphs and len(seqs) <= self.config.max_graph_batch:
                    out = self._run_graph(ordered, items, group)
                if out is None:
                    hn = self.forward_items(items, group)
                    out = self.sample(hn, ordered).tolist()
                    if self.fused_comm is not None:
                        self.fused_comm.check()
                self.timing["decode_tokens"] += len(seqs)
                by_id = {sq.seq_id: t for sq, t in zip(ordered, out)}
                return [by_id[sq.seq_id] for sq in seqs]
        if not is_prefill and self.config.use_cuda_graphs and len(seqs) <= self.config.max_graph_batch:
            out = self._run_graph(seqs)
            if out is not None:
                self.timing["decode_tokens"] += len(seqs)
                return out
        if is_prefill and self.config.use_cuda_graphs and len(seqs) == 1 and self.capture_logits is None:
            out = self._run_prefill_graph(seqs[0])
            if out is not None:
                self.timing["prefill_tokens"] += seqs[0].num_tokens - seqs[0].num_cached_tokens
                return out
        with_tokens = [s for s in seqs if s.num_tokens > s.num_cached_tokens]
        rows = []
        if with_tokens:
            hn = self.forward_items(self._items_for(with_tokens))
            rows.append(hn)
            self.timing["prefill_tokens" if is_prefill else "decode_tokens"] += sum(
                s.num_tokens - s.num_cached_tokens for s in with_tokens)
        empty = [s for s in seqs if s.num_tokens <= s.num_cached_tokens]
        for s in empty:
            if s.first_hidden is None:
                raise RuntimeError(f"sequence {s.seq_id} has nothing to process")
            rows.append(s.first_hidden.to(self.device, self.dtype).view(1, -1))
        order = with_tokens + empty
        hn = torch.cat(rows) if len(rows) > 1 else rows[0]
        toks = self.sample(hn, order).tolist()
        if self.fused_comm is not None:
            self.fused_comm.check()
        by_id = {s.seq_id: t for s, t in zip(order, toks)}
        return [by_id[s.seq_id] for s in seqs]

    def prefill_chunks(self, jobs: List[Tuple[List[int], int, List[int]]]) -> torch.Tensor:
        """Independent causal prefill of chunks: ``(tokens, cached_pos0, pages)`` each.

        Returns the final-normed hidden state of each chunk's last token.
        """
        items = [FwdItem(tokens=t, pos0=p0, priv_index0=0, priv_pages=pg, priv_pos0=p0, segments=[], logits=True)
                 for t, p0, pg in jobs]
        budget = self.config.max_num_batched_tokens
        outs, cur, n = [], [], 0
        for it in items:
            if cur and n + len(it.tokens) > budget:
                outs.append(self.forward_items(cur))
                cur, n = [], 0
            cur.append(it)
            n += len(it.tokens)
        if cur:
            outs.append(self.forward_items(cur))
        self.timing["prefill_tokens"] += sum(len(t) for t, _, _ in jobs)
        return torch.cat(outs) if len(outs) > 1 else outs[0]

    # --------------------------------------------------------- CUDA graphs
    def _bucket(self, n: int) -> int:
        for b in GRAPH_BUCKETS:
            if b >= n and b <= self.config.max_graph_batch:
                return b
        return -1

    def _graph_caps(self, B: int) -> Tuple[int, int]:
        max_segs = 16
        pages_per_seq = -(-self.config.max_model_len // self.page_size) + max_segs
        return B * max_segs, B * pages_per_seq

    def _tp_sampling(self, seqs: List[Sequence]) -> bool:
        """True when this step samples through the vocab-parallel record
        exchange (TP with the peer-memory runtime, every row's settings exact there)."""
        fc = self.fused_comm
        if fc is None or self.tp.size == 1 or not hasattr(self.model, "sample_tp"):
            return False
        return all(fc.can_sample(s.temperature, s.top_k, s.top_p, s.min_p) for s in seqs)

    def _capture(self, B: int, prefill_tokens: int = 0, tp_sampling: bool = False, shared: bool = False) -> _GraphSlot:
        """Capture one engine step: a decode step of ``B`` sequences, or (with
        ``prefill_tokens``) a prefill of one sequence padded to that many tokens.
        ``tp_sampling``: sample through the vocab-parallel record exchange;
        ``shared``: decode with a shared-prefix group (the group's metadata is
        refreshed with every replay)."""
        g = _GraphSlot()
        g.seg_cap, g.page_cap = self._graph_caps(B)
        if shared:
            g.seg_cap += 16  # the group's shared segments, listed once
        pm = self.page_manager
        if prefill_tokens:
            g.seg_cap, g.page_cap = g.seg_cap + 1, g.page_cap + 1  # + the padding sequence
            dummy = FwdItem(tokens=[0], pos0=0, priv_index0=0, priv_pages=[pm.scratch_page], priv_pos0=0)
            plan = build_plan([dummy], self.page_size, scratch_page=pm.scratch_page, seg_cap=g.seg_cap,
                              page_cap=g.page_cap, pad_tokens=prefill_tokens - 1)
        else:
            plan = build_plan([], self.page_size, pad_seqs=B, scratch_page=pm.scratch_page,
                              seg_cap=g.seg_cap, page_cap=g.page_cap, group=(0, set()) if shared else None)
        g.sizes = plan.sizes
        # One device buffer holds the step's sampling settings and packed plan
        # (int64 [2, B] | float32 [3, B] | int32 [B] | int32 plan), so a replay
        # uploads them with ONE host->device copy from a pinned mirror.
        packed0 = pack(plan)
        nl, nf, nk = 16 * B, 12 * B, 4 * B
        g.dev_all = torch.zeros(nl + nf + nk + 4 * packed0.size, dtype=torch.uint8, device=self.device)
        g.lbuf = g.dev_all[:nl].view(torch.int64).view(2, B)
        g.fbuf = g.dev_all[nl:nl + nf].view(torch.float32).view(3, B)
        g.ibuf = g.dev_all[nl + nf:nl + nf + nk].view(torch.int32)
        g.meta_buf = g.dev_all[nl + nf + nk:].view(torch.int32)
        g.meta_buf.copy_(torch.from_numpy(packed0))
        views = unpack(g.meta_buf, g.sizes)
        g.num_splits = 1 if prefill_tokens else self._decode_splits(B)
        meta = make_meta(views, plan, g.num_splits,
                         shared_splits=self._shared_splits(B, g.num_splits) if shared else 0)
        meta.decode = not prefill_tokens
        meta.max_q_len = prefill_tokens or 1
        meta.max_kv_len = self.config.max_model_len
        g.fbuf[1].fill_(1.0)
        g.out = torch.zeros(B, dtype=torch.int32, device=self.device)
        kv = pm.kv_cache

        def body():
            h = self.model.forward(views["input_ids"], views["positions"], views["slots"], meta, kv)
            if prefill_tokens:
                h = h.index_select(0, views["logits_idx"].long())
            hn = self.model.final_hidden(h)
            if tp_sampling:
                self.model.sample_tp(hn, g.fbuf[0], g.ibuf, g.fbuf[1], g.fbuf[2], g.lbuf[0], g.lbuf[1], g.out)
            else:
                logits = self.model.compute_logits(hn)
                ops.sample(logits, g.fbuf[0], g.ibuf, g.fbuf[1], g.fbuf[2], g.lbuf[0], g.lbuf[1], out=g.out)

        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                body()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        from ..ops import _ext

        n0 = _ext.launches
        with torch.cuda.graph(graph, pool=self._graph_pool()):
            body()
        g.launches = _ext.launches - n0
        torch.cuda.synchronize(self.device)
        g.graph = graph
        self._pinned_meta = getattr(self, "_pinned_meta", {})
        return g

    def _graph_pool(self):
        if not hasattr(self, "_pool"):
            self._pool = torch.cuda.graph_pool_handle()
        return self._pool

    def capture_all(self, max_batch: Optional[int] = None) -> None:
        mb = min(max_batch or self.config.max_graph_batch, self.config.max_graph_batch)
        tps = self.fused_comm is not None and self.tp.size > 1 and hasattr(self.model, "sample_tp")
        for b in sorted(GRAPH_BUCKETS, reverse=True):
            if b <= mb and b not in self.graphs:
                self.graphs[b] = self._capture(b, tp_sampling=tps)

    def _run_graph(self, seqs: List[Sequence], items: Optional[List[FwdItem]] = None,
                   group: Optional[tuple] = None) -> Optional[List[int]]:
        B = self._bucket(len(seqs))
        if B < 0:
            return None
        tps = self._tp_sampling(seqs)
        if group is not None:
            key = (B, tps)
            g = self.graphs_shared.get(key)
            if g is None:
                g = self.graphs_shared[key] = self._capture(B, tp_sampling=tps, shared=True)
        else:
            if not tps and self.fused_comm is not None and self.tp.size > 1 and hasattr(self.model, "sample_tp"):
                table = self.graphs_gather  # settings that need the whole distribution
            else:
                table = self.graphs
            g = table.get(B)
            if g is None:
                g = table[B] = self._capture(B, tp_sampling=tps)
        plain = items is None and group is None
        spec, self._spec = self._spec, None
        if plain and spec is not None and spec[0] is g and spec[1] == self._decode_key(seqs, 0):
            # this step's plan was built while the previous step ran on the GPU;
            # only the sampled tokens (input ids lead the packed plan) are new
            packed = spec[2]
            packed[:len(seqs)] = [s.token_ids[-1] for s in seqs]
            return self._replay(g, packed, seqs, B, speculate=True)
        try:
            plan = build_plan(items if items is not None else self._items_for(seqs), self.page_size,
                              pad_seqs=B - len(seqs), scratch_page=self.page_manager.scratch_page,
                              seg_cap=g.seg_cap, page_cap=g.page_cap, group=group)
        except OverflowError:
            return None
        if plan.sizes != g.sizes:
            return None
        self._check_plan(plan)
        return self._replay(g, pack(plan), seqs, B, speculate=plain)

    @staticmethod
    def _decode_key(seqs: List[Sequence], ahead: int) -> tuple:
        """State of a decode batch that a prebuilt plan depends on, ``ahead``
        steps from now (every sequence one token longer per step)."""
        return tuple((s.seq_id, s.num_cached_tokens + ahead, s.num_tokens + ahead, s.pos_base, tuple(s.pages),
                      tuple(id(sg) for sg in s.segments)) for s in seqs)

    def _speculate(self, g: "_GraphSlot", seqs: List[Sequence], B: int):
        """The NEXT decode step's packed plan, assuming the same sequences each
        grow by one token (its id is filled in when the step runs) and no new
        KV page is needed; None when that cannot be prebuilt."""
        items = []
        for s in seqs:
            L = s.num_tokens
            if s.num_cached_tokens != L - 1 or L // self.page_size >= len(s.pages):
                return None
            items.append(FwdItem(tokens=[0], pos0=s.pos_base + L, priv_index0=L, priv_pages=s.pages,
                                 priv_pos0=s.pos_base, segments=s.segments, logits=True))
        try:
            plan = build_plan(items, self.page_size, pad_seqs=B - len(seqs), scratch_page=self.page_manager.scratch_page,
                              seg_cap=g.seg_cap, page_cap=g.page_cap)
        except OverflowError:
            return None
        if plan.sizes != g.sizes:
            return None
        try:
            self._check_plan(plan)
        except PlanValidationError:
            return None  # not prebuilt; the step's own plan is built and checked when it runs
        return (g, self._decode_key(seqs, 1), pack(plan))

    def _prefill_bucket(self, n: int) -> int:
        cap = self.config.max_prefill_graph_tokens
        for b in PREFILL_BUCKETS:
            if n <= b <= cap:
                return b
        return -1

    def _run_prefill_graph(self, seq: Sequence) -> Optional[List[int]]:
        """Prefill of one short token run (a query or a new turn over cached
        chunk KV) replayed from a CUDA graph captured per token bucket."""
        n = seq.num_tokens - seq.num_cached_tokens
        Tb = self._prefill_bucket(n) if n > 0 else -1
        if Tb < 0:
            return None
        g = self.prefill_graphs.get(Tb)
        if g is None:
            g = self.prefill_graphs[Tb] = self._capture(1, prefill_tokens=Tb)
        try:
            plan = build_plan(self._items_for([seq]), self.page_size, scratch_page=self.page_manager.scratch_page,
                              seg_cap=g.seg_cap, page_cap=g.page_cap, pad_tokens=Tb - n)
        except OverflowError:
            return None
        if plan.sizes != g.sizes:
            return None
        self._check_plan(plan)
        return self._replay(g, pack(plan), [seq], 1)

    def _replay(self, g: _GraphSlot, packed: np.ndarray, seqs: List[Sequence], B: int,
                speculate: bool = False) -> List[int]:
        with nvtx_range(f"graph replay b={B}"):
            return self._replay_graph(g, packed, seqs, B, speculate)

    def _replay_graph(self, g: _GraphSlot, packed: np.ndarray, seqs: List[Sequence], B: int,
                      speculate: bool) -> List[int]:
        """Upload the packed plan and sampling settings, replay the captured
        step, read the tokens back.  ``speculate``: while the GPU runs, prebuild
        the next decode step's plan (``_speculate``)."""
        # Persistent pinned staging: the previous step's copies completed at its
        # token read-back, so the buffers are free to overwrite.
        if g.pin_all is None:
            g.pin_all = torch.empty(g.dev_all.numel(), dtype=torch.uint8).pin_memory()
            a = g.pin_all.numpy()
            nl, nf, nk = 16 * B, 12 * B, 4 * B
            g.pin_l = a[:nl].view(np.int64).reshape(2, B)
            g.pin_f = a[nl:nl + nf].view(np.float32).reshape(3, B)
            g.pin_k = a[nl + nf:nl + nf + nk].view(np.int32)
            g.pin_meta = a[nl + nf + nk:].view(np.int32)
            g.pin_out = torch.empty(B, dtype=torch.int32).pin_memory()
        g.pin_meta[:] = packed
        f, k, l = self._sampling_tensors(seqs, pad=B - len(seqs))
        g.pin_f[:] = f
        g.pin_k[:] = k
        g.pin_l[:] = l
        g.dev_all.copy_(g.pin_all, non_blocking=True)
        self.last_h2d_bytes = g.pin_all.numel()
        if self.event_log is not None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.graph.replay()
            e1.record()
            self.event_log.append((e0, e1))
        else:
            g.graph.replay()
        g.pin_out.copy_(g.out, non_blocking=True)
        if self.fused_comm is not None:
            if g.pin_status is None:
                g.pin_status = torch.zeros(4, dtype=torch.int32).pin_memory()
            g.pin_status.copy_(self.fused_comm.status, non_blocking=True)
        if speculate:
            self._spec = self._speculate(g, seqs, B)
        torch.cuda.current_stream(self.device).synchronize()
        if self.fused_comm is not None and int(g.pin_status[0]) != 0:
            self.fused_comm.check()
        return g.pin_out[: len(seqs)].tolist()

    def launches_per_decode_step(self, batch: int) -> int:
        g = self.graphs.get(self._bucket(batch))
        return getattr(g, "launches", 0) if g is not None else 0
