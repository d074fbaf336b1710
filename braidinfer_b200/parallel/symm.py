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
                 timeout_s: float = 5.0):
        from ..ops._ext import ext

        self.tp = tp
        self.H = hidden
        self.maxT = max_tokens
        self.device = device
        self.timeout_s = timeout_s
        self._C = ext()
        dev = device.index
        data = 2 * tp.size * max_tokens * hidden * 2
        self.flags_off = (data + 255) // 256 * 256
        nbytes = self.flags_off + 8 * tp.size + 256
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
        self.status = torch.zeros(4, dtype=torch.int32, device=device)
        self.push_fault = False  # test hook: skip the push (a peer that never signals)
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
            raise CommTimeoutError(
                f"rank {st[1]} timed out after {self.timeout_s}s waiting for rank {st[2]} (all-reduce #{st[3]})",
                {"code": st[0], "rank": st[1], "peer": st[2], "epoch": st[3]})

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

    def linear_all_reduce_add(self, x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
        """``residual += sum_ranks(x @ w.T)`` with the push fused into the GEMM epilogue."""
        arrivals = self._C.gemm_push(x, w, self.peers, self.flags_off, self.tp.rank, self.tp.size, self.maxT,
                                     self.epoch_state)
        return self._reduce(residual, residual, arrivals)

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
    collectives through it (decode shapes); prefill-sized tensors use NCCL."""
    from . import comm
    from .state import get_tp

    tp = get_tp()
    if tp.size == 1 or runner.device.type != "cuda":
        return None
    fc = FusedComm(tp, config.spec.hidden_size, runner.device, max_tokens=min(64, config.max_graph_batch or 64),
                   timeout_s=config.comm_timeout_s)
    comm.set_fused_comm(fc)
    runner.fused_comm = fc
    return fc
