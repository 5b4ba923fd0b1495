"""Value-head-sharded decode across GPUs (one process per GPU).

Every (batch, value head) state evolves independently, so N ranks each own
Hv/N value heads' states for the whole run and a decode step needs no
communication.  The only exchange is an optional all-gather of the per-rank
outputs o[B, Hv/N, d_v] (NCCL over NVLink when the process group uses the
nccl backend) into the full o[B, Hv, d_v], done only when the caller asks.

The reference is single-GPU only (METHODOLOGY.md:80); this is the multi-GPU
layer BASELINE config 4 adds.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class HeadShard:
    h0: int   # first value head owned
    h1: int   # one past the last value head owned
    hq0: int  # first query/key head read
    hq1: int  # one past the last query/key head read


def shard_heads(Hv: int, Hqk: int, world_size: int, rank: int) -> HeadShard:
    """Contiguous value-head range of ``rank`` and the q/k heads it reads
    (value head h reads q/k head h // (Hv // Hqk))."""
    if Hv % Hqk:
        raise ValueError("Hv must be a multiple of Hqk")
    if Hv % world_size:
        raise ValueError(f"Hv={Hv} value heads do not split over {world_size} ranks")
    per = Hv // world_size
    group = Hv // Hqk
    h0, h1 = rank * per, (rank + 1) * per
    return HeadShard(h0, h1, h0 // group, (h1 - 1) // group + 1)


class ShardedGDNDecoder:
    """Holds this rank's slice of the recurrent state and runs decode steps.

    ``state`` is the local shard [B, Hv/N, d_k, d_v] (fp32, resident on this
    rank's GPU).  ``step`` takes the FULL per-token inputs (q, k [B, Hqk, d_k],
    v [B, Hv, d_v], g, beta [B, Hv]) or their local slices, and returns the
    local output; with ``gather=True`` it returns the full o [B, Hv, d_v].

    ``step_fn`` defaults to :func:`gdn_decode` (``kda=True``: :func:`kda_decode`);
    tests substitute a CPU function to exercise the sharding logic on gloo.
    """

    def __init__(self, B: int, Hqk: int, Hv: int, dk: int = 128, dv: int = 128, *,
                 group=None, device=None, state: torch.Tensor | None = None,
                 kda: bool = False, io_dtype=torch.bfloat16, step_fn: Callable | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.shard = shard_heads(Hv, Hqk, self.world, self.rank)
        self.B, self.Hqk, self.Hv, self.dk, self.dv = B, Hqk, Hv, dk, dv
        self.kda = kda
        self.device = torch.device(device) if device is not None else (
            torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available()
            else torch.device("cpu"))
        per = self.shard.h1 - self.shard.h0
        if state is None:
            state = torch.zeros((B, per, dk, dv), dtype=torch.float32, device=self.device)
        if tuple(state.shape) != (B, per, dk, dv):
            raise ValueError(f"local state must be {(B, per, dk, dv)}")
        self.state = state
        if step_fn is None:
            from .api import gdn_decode, kda_decode
            step_fn = kda_decode if kda else gdn_decode
        self.step_fn = step_fn
        self._gather_buf = None
        self.io_dtype = io_dtype

    def local_slices(self, q, k, v, g, beta):
        """Slices full-head inputs down to this rank's heads (views, no copy)."""
        s = self.shard
        if q.shape[1] == self.Hqk:
            q, k = q[:, s.hq0:s.hq1], k[:, s.hq0:s.hq1]
        if v.shape[1] == self.Hv:
            v, g, beta = v[:, s.h0:s.h1], g[:, s.h0:s.h1], beta[:, s.h0:s.h1]
        return q, k, v, g, beta

    def step(self, q, k, v, g, beta, *, gather: bool = False, scale: float = 1.0):
        ql, kl, vl, gl, bl = self.local_slices(q, k, v, g, beta)
        o_local = self.step_fn(ql, kl, vl, gl, bl, self.state, scale=scale)
        if not gather:
            return o_local
        return self.gather(o_local)

    def gather(self, o_local: torch.Tensor) -> torch.Tensor:
        """All-gathers rank-major [N, B, Hv/N, d_v] and returns [B, Hv, d_v]."""
        if self.world == 1:
            return o_local
        o_local = o_local.contiguous()
        n = self.world
        if self._gather_buf is None or self._gather_buf.dtype != o_local.dtype \
                or self._gather_buf.device != o_local.device:
            self._gather_buf = torch.empty((n,) + tuple(o_local.shape), dtype=o_local.dtype,
                                           device=o_local.device)
        buf = self._gather_buf
        if hasattr(dist, "all_gather_into_tensor") and o_local.device.type == "cuda":
            dist.all_gather_into_tensor(buf.view(-1), o_local.view(-1), group=self.group)
        else:
            dist.all_gather(list(buf.unbind(0)), o_local, group=self.group)
        # rank-major -> head-major: [N, B, Hv/N, d_v] -> [B, N*Hv/N, d_v]
        return buf.permute(1, 0, 2, 3).reshape(self.B, self.Hv, o_local.shape[-1])
