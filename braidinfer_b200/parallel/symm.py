"""Peer-memory communication runtime for tensor parallelism (one process per GPU).

Each rank ``cudaMalloc``s one communication buffer (receive slots for decode
partials + per-source arrival counters), exports a CUDA IPC handle, and the
handles are exchanged over the process group; every rank then maps every
peer's buffer.  The fused collectives run as native kernels that store into
peer memory over NVLink (``csrc/comm.cu``, ``csrc/gemm_tcgen05.cu`` epi 3):

* ``linear_all_reduce_add(x, w, residual)``: the row-parallel GEMM (o_proj /
  down_proj) pushes its bf16 result tiles straight from the epilogue into every
  peer's slot, then ``tp_reduce_add`` waits — with a wall-clock bound — for all
  sources, sums in fp32 and adds the residual.  One NVLink hop, no NCCL call.
* ``all_reduce(x)``: the same protocol for a tensor computed elsewhere.

Prefill-sized batches (``maxT < T <= sp_max_tokens``) run sequence-parallel:
token rows are owned by ranks in blocks of ``ceil(T / tp)`` and the residual
stream lives in a gathered buffer ``G [T, hidden]`` inside the comm buffer.

* ``sp_linear_reduce_scatter(x, w)``: o_proj / down_proj GEMM whose epilogue
  stores each output row straight into its owner's receive slot (GEMM →
  reduce-scatter in one kernel; each rank sends ``(tp-1)/tp`` of its partial).
* ``sp_reduce_allgather(eps)``: the owner sums the partials, adds the residual,
  computes the row's ``1/rms`` and stores row + ``1/rms`` into every rank's
  ``G`` (all-gather by peer stores).
* the next QKV / gate_up GEMM (input RMSNorm fused) waits per 128-row tile
  for that tile's owners and then TMA-loads ``G`` locally (all-gather → GEMM);
  tiles whose rows have arrived run while others are still in flight.

Counters are cumulative; the expected values are tracked here on the host,
so these prefill calls are never captured in a CUDA graph.

Every wait is bounded (``comm_timeout_s``); an expired wait leaves a status
word that :meth:`FusedComm.check` turns into ``CommTimeoutError``.  No NVLS
multicast object and no TMA load of peer memory is used.  The NCCL path stays
the baseline (``comm_backend="nccl"``) and handles shapes above ``max_tokens``.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from ..errors import CommTimeoutError
from ..utils.logging import get_logger
from .state import TPState

log = get_logger("symm")


class FusedComm:
    def __init__(self, tp: TPState, hidden: int, device: torch.device, max_tokens: int = 64,
                 timeout_s: float = 5.0, sp_max_tokens: int = 0):
        from ..ops._ext import ext

        self.tp = tp
        self.H = hidden
        self.maxT = max_tokens
        self.device = device
        self.timeout_s = timeout_s
        self._C = ext()
        dev = device.index

        def align(n: int) -> int:
            return (n + 255) // 256 * 256

        data = 2 * tp.size * max_tokens * hidden * 2
        self.flags_off = align(data)
        off = self.flags_off + align(8 * tp.size)
        # per-(source, output tile) flags of the in-GEMM all-reduce: 128 features x up to 4 token tiles
        self.max_tiles = -(-hidden // 128) * 4
        self.tile_flags_off = off
        off += align(8 * tp.size * self.max_tiles)
        # sequence-parallel prefill region
        self.sp_max = sp_max_tokens if sp_max_tokens > max_tokens else 0
        self.rs_flags_off = off
        off += align(8 * tp.size)
        self.ag_flags_off = off
        off += align(8 * tp.size)
        self.g_off = off
        off += align(self.sp_max * hidden * 2)
        self.rstd_off = off
        off += align(self.sp_max * 4)
        self.recv_off = off
        off += align(tp.size * (-(-self.sp_max // tp.size)) * hidden * 2)
        # vocab-parallel sampling: per-row records [2 slots][tp][max_tokens] + per-source counters
        self.rec_bytes = int(self._C.tp_sample_record_bytes())
        self.sample_recv_off = off
        off += align(2 * tp.size * max_tokens * self.rec_bytes)
        self.sample_flags_off = off
        off += align(8 * tp.size)
        nbytes = off + 256
        self.sp_rs_expected = 0
        self.sp_ag_expected = 0
        self.sp_T = 0
        self.sp_rpr = 0
        ptr, handle = self._C.comm_alloc(nbytes, dev)
        self.local_ptr = int(ptr.item())
        handles = [None] * tp.size
        dist.all_gather_object(handles, handle.numpy().tobytes(), group=tp.group)
        self.peer_ptrs = []
        for r, h in enumerate(handles):
            if r == tp.rank:
                self.peer_ptrs.append(self.local_ptr)
            else:
                t = torch.frombuffer(bytearray(h), dtype=torch.uint8)
                self.peer_ptrs.append(int(self._C.comm_open(t, dev)))
        self.peers = torch.tensor(self.peer_ptrs, dtype=torch.int64, device=device)
        # [0] epoch (completed calls), [1] cumulative expected arrivals, [2] CTA done counter
        self.epoch_state = torch.zeros(4, dtype=torch.int64, device=device)
        self.sample_state = torch.zeros(4, dtype=torch.int64, device=device)  # sampler calls, expected, rows done
        self.status = torch.zeros(4, dtype=torch.int32, device=device)
        self.push_fault = False  # test hook: skip the push (a peer that never signals)
        import os
        self.fused_reduce = os.environ.get("BRAID_TP_FUSED_REDUCE", "0") == "1"
        dist.barrier(group=tp.group)
        log.info("fused comm ready: tp=%d maxT=%d hidden=%d (%.1f MB buffer)", tp.size, max_tokens, hidden,
                 nbytes / 1e6)

    # ------------------------------------------------------------- checks
    def can_all_reduce(self, x: torch.Tensor) -> bool:
        return x.is_cuda and x.dim() == 2 and x.shape[0] <= self.maxT and x.shape[1] == self.H and \
            x.dtype == torch.bfloat16

    def check(self) -> None:
        st = self.status.tolist()
        if st[0] != 0:
            self.status.zero_()
            what = {1: "all-reduce", 2: "all-gather", 3: "reduce-scatter", 4: "sampler exchange"}.get(st[0],
                                                                                                  "collective")
            raise CommTimeoutError(
                f"rank {st[1]} timed out after {self.timeout_s}s waiting for rank {st[2]} ({what} #{st[3]})",
                {"code": st[0], "rank": st[1], "peer": st[2], "epoch": st[3]})

    # ------------------------------------------ sequence-parallel prefill
    def can_sp(self, T: int) -> bool:
        # host-tracked counters: never inside a CUDA-graph capture (NCCL there)
        return self.maxT < T <= self.sp_max and not torch.cuda.is_current_stream_capturing()

    def sp_begin(self, T: int):
        """Start a sequence-parallel forward of ``T`` tokens; returns views of
        the gathered residual ``G [T, H]`` and its per-row ``1/rms [T]``."""
        assert self.can_sp(T)
        self.sp_T = T
        self.sp_rpr = -(-T // self.tp.size)
        dev = self.device.index
        G = self._C.comm_tensor(self.local_ptr, self.g_off, [T, self.H], 0, dev)
        rstd = self._C.comm_tensor(self.local_ptr, self.rstd_off, [T], 1, dev)
        return G, rstd

    def sp_params(self, wait: bool = True) -> torch.Tensor:
        """Parameter block of the GEMM's sequence-parallel mode (CPU int64)."""
        return torch.tensor([self.peers.data_ptr(), self.recv_off, self.rs_flags_off, self.ag_flags_off,
                             self.sp_ag_expected if wait else 0, self.status.data_ptr(),
                             int(self.timeout_s * 1e9), self.tp.rank, self.tp.size, self.sp_rpr, self.H],
                            dtype=torch.int64)

    def sp_linear_reduce_scatter(self, x: torch.Tensor, w: torch.Tensor, G: torch.Tensor) -> None:
        """Row-parallel GEMM whose epilogue pushes each row to its owner."""
        n = self._C.gemm(G, x, w, None, None, 4, -1.0, None, self.sp_params(wait=False))
        self.sp_rs_expected += int(n)

    def sp_reduce_allgather(self, eps: float) -> None:
        n = self._C.sp_reduce_allgather(self.peers, self.recv_off, self.rs_flags_off, self.ag_flags_off, self.g_off,
                                        self.rstd_off, self.tp.rank, self.tp.size, self.sp_rpr, self.sp_T, self.H,
                                        self.sp_rs_expected, float(eps), self.status, self.timeout_s)
        self.sp_ag_expected += int(n)

    def sp_wait(self) -> None:
        """Make all of ``G`` readable by ordinary kernels later on the stream."""
        self._C.sp_wait(self.local_ptr, self.ag_flags_off, self.tp.size, self.tp.rank, self.sp_ag_expected,
                        self.status, self.timeout_s)

    # -------------------------------------------------------- collectives
    def _reduce(self, out: torch.Tensor, residual: Optional[torch.Tensor], arrivals: int) -> torch.Tensor:
        self._C.tp_reduce_add(out, residual if residual is not None else out, residual is not None,
                              self.local_ptr, self.flags_off, self.tp.size, self.maxT, self.tp.rank, arrivals,
                              self.epoch_state, self.status, self.timeout_s)
        return out

    def _push_arrivals(self, x: torch.Tensor) -> int:
        T, H = x.shape
        return max(1, min(32, T * H // 8 // 256))

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        x = x.contiguous()
        if not self.push_fault:
            self._C.tp_push(x, self.peers, self.flags_off, self.tp.rank, self.tp.size, self.maxT, self.epoch_state)
        return self._reduce(x, None, self._push_arrivals(x))

    def all_reduce_add(self, partial: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
        partial = partial.contiguous()
        if not self.push_fault:
            self._C.tp_push(partial, self.peers, self.flags_off, self.tp.rank, self.tp.size, self.maxT,
                            self.epoch_state)
        return self._reduce(residual, residual, self._push_arrivals(partial))

    def linear_all_reduce_add(self, x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor,
                              w_next: Optional[torch.Tensor] = None, skip: int = 0) -> torch.Tensor:
        """``residual += sum_ranks(x @ w.T)`` in ONE kernel: each 128-feature tile
        is pushed to every peer from the GEMM epilogue, the tile's CTA waits for
        the peers' copies of the same tile and reduces them with the residual.
        ``fused_reduce = False`` keeps the two-kernel form (push epilogue, then
        ``tp_reduce_add``)."""
        if self.fused_reduce and residual.is_contiguous() and self.tp.size <= 8:
            self._C.gemm_allreduce_add(residual, x, w, self.peers, self.flags_off, self.tile_flags_off,
                                       self.max_tiles, self.tp.rank, self.tp.size, self.maxT, self.epoch_state,
                                       self.status, self.timeout_s)
            return residual
        arrivals = self._C.gemm_push(x, w, self.peers, self.flags_off, self.tp.rank, self.tp.size, self.maxT,
                                     self.epoch_state)
        if w_next is not None and x.shape[0] <= 64:  # the reduce kernel prefetches further while it waits
            self._C.gemm_prefetch_next(w_next, x.shape[0], skip)
        return self._reduce(residual, residual, arrivals)

    # --------------------------------------------------------- sampling
    TP_SAMPLE_MAX_TOP_K = 32  # candidates per rank and row in the sampler records

    def can_sample(self, temperature: float, top_k: int, top_p: float, min_p: float) -> bool:
        """Settings the record exchange samples exactly (else: logits all-gather)."""
        if temperature <= 0:
            return True
        if top_k <= 0:
            return top_p >= 1.0 and min_p <= 0.0
        return top_k <= self.TP_SAMPLE_MAX_TOP_K

    def sample(self, local_logits: torch.Tensor, vocab_start: int, vocab_size: int, temperature, top_k, top_p,
               min_p, seed, step, out: torch.Tensor) -> torch.Tensor:
        """Token per row from this rank's vocab shard of the logits: per-shard
        records are exchanged over peer memory and merged on every rank."""
        self._C.tp_sample(out, local_logits, int(vocab_start), int(vocab_size), temperature, top_k, top_p, min_p,
                          seed, step, self.peers, self.sample_recv_off, self.sample_flags_off, self.tp.rank,
                          self.tp.size, self.maxT, self.sample_state, self.status, self.timeout_s)
        return out

    def all_reduce_add_rms_norm(self, partial, residual, w, eps, out=None):
        from ..ops.norm import rms_norm

        self.all_reduce_add(partial, residual)
        return rms_norm(residual, w, eps, out), residual

    def close(self) -> None:
        dev = self.device.index
        try:
            torch.cuda.synchronize(self.device)
            for r, p in enumerate(self.peer_ptrs):
                if r != self.tp.rank:
                    self._C.comm_close(p, dev)
            self._C.comm_free(self.local_ptr, dev)
        except Exception:  # pragma: no cover - best effort at shutdown
            pass


def maybe_enable_fused_comm(config, runner) -> Optional[FusedComm]:
    """Create the peer-memory runtime for this TP group and route the model's
    collectives through it: one-shot push all-reduce for decode shapes,
    sequence-parallel reduce-scatter / all-gather for prefill batches up to
    ``max_num_batched_tokens``; larger tensors use NCCL."""
    from . import comm
    from .state import get_tp

    tp = get_tp()
    if tp.size == 1 or runner.device.type != "cuda":
        return None
    fc = FusedComm(tp, config.spec.hidden_size, runner.device, max_tokens=min(64, config.max_graph_batch or 64),
                   timeout_s=config.comm_timeout_s, sp_max_tokens=config.max_num_batched_tokens)
    comm.set_fused_comm(fc)
    runner.fused_comm = fc
    return fc
