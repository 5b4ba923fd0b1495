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

import ctypes
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


class PeerGather:
    """All-gather of equal per-rank slices with the copy engines over NVLink.

    Every rank holds two slots of a rank-major buffer ``[2][N][slice]`` plus
    ``ready[N]`` and ``free[N]`` step counters, all exported through CUDA IPC.
    ``push(src, step)`` (on a side stream) waits until every rank has freed the
    slot of ``step`` (used by ``step - 2``), copies ``src`` into slot
    ``step % 2`` at row ``rank`` of every rank's buffer (DMA, no SMs), then
    sets ``ready[rank] = step`` on every rank.  ``wait(step)`` makes a stream
    wait until all ranks' slices of ``step`` have landed; ``release(step)``
    tells every producer that this rank is done reading that slot.  Steps
    start at 1.  All waits are GPU stream waits: no host synchronisation.
    """

    def __init__(self, slice_numel: int, dtype, device, group=None):
        from . import _lib
        self._lib = _lib.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        self.slice_numel = slice_numel
        # one allocation (one IPC handle per rank): the two buffer slots, then
        # the ready[N] | free[N] counters at a 256-byte boundary
        esz = torch.empty((), dtype=dtype).element_size()
        buf_bytes = 2 * self.world * slice_numel * esz
        flag_off = (buf_bytes + 255) // 256 * 256
        self.raw = torch.zeros(flag_off + 8 * self.world, dtype=torch.uint8, device=self.device)
        self.buf = self.raw[:buf_bytes].view(dtype).view(2, self.world, slice_numel)
        self.flags = self.raw[flag_off:].view(torch.int32)
        h = self._handle(self.raw)
        allh = [None] * self.world
        dist.all_gather_object(allh, h, group=group)
        self._opened = []
        bases = []
        for p, hp in enumerate(allh):
            bases.append(self.raw.data_ptr() if p == self.rank else self._open(hp))
        bufs = bases
        flags = [bp + flag_off for bp in bases]
        n = self.world
        slice_bytes = slice_numel * esz
        VP = ctypes.c_void_p * n
        # destinations of this rank's slice in each slot, and the flag words it writes
        self._dst = [VP(*[bufs[p] + (slot * n + self.rank) * slice_bytes for p in range(n)])
                     for slot in range(2)]
        self._ready = VP(*[flags[p] + 4 * self.rank for p in range(n)])
        self._free = VP(*[flags[p] + 4 * (n + self.rank) for p in range(n)])
        self._slice_bytes = slice_bytes
        dist.barrier(group=group)

    def _handle(self, t):
        """(IPC handle of t's allocation, byte offset of t inside it)."""
        from ._lib import IPC_HANDLE_BYTES, check
        h = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        off = ctypes.c_uint64()
        check(self._lib.gdn_ipc_handle(t.data_ptr(), h, ctypes.byref(off)), "gdn_ipc_handle")
        return h.raw, off.value

    def _open(self, handle_and_offset) -> int:
        from ._lib import check
        handle, offset = handle_and_offset
        ptr, base = ctypes.c_void_p(), ctypes.c_void_p()
        check(self._lib.gdn_ipc_open(handle, offset, ctypes.byref(ptr), ctypes.byref(base)),
              "gdn_ipc_open")
        self._opened.append(base.value)
        return ptr.value

    @staticmethod
    def _s(stream):
        return (stream or torch.cuda.current_stream()).cuda_stream

    def push(self, src: torch.Tensor, step: int, stream=None, peer_streams=None) -> None:
        """Sends ``src`` to every rank.  With ``peer_streams`` (one stream per
        rank) the copies to different ranks run on separate copy engines in
        parallel; otherwise they queue on ``stream``."""
        from ._lib import check
        n = self.world
        if peer_streams is None:
            s = self._s(stream)
            if step > 2:  # every consumer is done with the slot this step overwrites
                check(self._lib.gdn_gather_wait(self.flags.data_ptr() + 4 * n, n, step - 2, s),
                      "gdn_gather_wait")
            check(self._lib.gdn_gather_push(src.data_ptr(), self._slice_bytes, self._dst[step % 2],
                                            self._ready, n, step, s), "gdn_gather_push")
            return
        VP1 = ctypes.c_void_p * 1
        for p in range(n):
            s = peer_streams[p].cuda_stream
            if step > 2:  # rank p is done with the slot this step overwrites
                check(self._lib.gdn_gather_wait(self.flags.data_ptr() + 4 * (n + p), 1, step - 2, s),
                      "gdn_gather_wait")
            check(self._lib.gdn_gather_push(src.data_ptr(), self._slice_bytes,
                                            VP1(self._dst[step % 2][p]), VP1(self._ready[p]), 1,
                                            step, s), "gdn_gather_push")

    def wait(self, step: int, stream=None) -> torch.Tensor:
        """Stream-waits for every slice of ``step``; returns the slot [N, slice]."""
        from ._lib import check
        check(self._lib.gdn_gather_wait(self.flags.data_ptr(), self.world, step, self._s(stream)),
              "gdn_gather_wait")
        return self.buf[step % 2]

    def release(self, step: int, stream=None) -> None:
        from ._lib import check
        # zero-byte copies, then the free-flag writes on every producer
        check(self._lib.gdn_gather_push(self.flags.data_ptr(), 0, self._free, self._free,
                                        self.world, step, self._s(stream)), "gdn_gather_push")

    def close(self) -> None:
        for p in self._opened:
            self._lib.gdn_ipc_close(p)
        self._opened = []


class FusedGather:
    """Output all-gather fused into the decode kernel (gdn_peer_out_t).

    Every rank holds two full output buffers ``out[slot]`` [B, Hv, d_v]
    (head-major: the gathered result needs no permute), an arrival counter,
    a finished-CTA counter and ``free[N]`` flags, in one allocation exported
    through CUDA IPC.  ``decode_step(...)`` binds a :class:`DecodeStep` whose
    kernel writes this rank's heads of step s into slot ``s % 2`` of every
    rank's buffer with plain NVLink stores and signals arrival itself; no copy
    engine, collective or host synchronisation runs per step.

    Use: ``launch(steps)`` runs the next step (``steps`` = the two bound
    DecodeSteps, one per slot) and returns its step number; ``wait(step)``
    makes the current stream wait (bounded, on the GPU) until every rank's
    outputs of that step are in ``out[step % 2]``.  Reads of a step's
    outputs must be stream-ordered before this rank's next ``launch``.
    Every rank must launch the same sequence of steps.
    """

    def __init__(self, B: int, Hv: int, dv: int, h0: int, hv: int, dtype, device, group=None):
        from . import _lib
        self._lib = _lib.load()
        self._L = _lib
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 2 <= self.world <= 8:
            raise ValueError("the fused gather spans 2..8 ranks")
        self.device = torch.device(device)
        self.B, self.Hv, self.dv, self.h0, self.hv = B, Hv, dv, h0, hv
        esz = torch.empty((), dtype=dtype).element_size()
        slot_bytes = B * Hv * dv * esz
        flag_off = (2 * slot_bytes + 255) // 256 * 256
        n = self.world
        self.raw = torch.zeros(flag_off + 8 + 4 * n, dtype=torch.uint8, device=self.device)
        self.out = [self.raw[s * slot_bytes:(s + 1) * slot_bytes].view(dtype).view(B, Hv, dv)
                    for s in range(2)]
        flags = self.raw[flag_off:].view(torch.int32)
        self.arrive = flags[0:1]
        h = PeerGather._handle(self, self.raw)
        allh = [None] * n
        dist.all_gather_object(allh, h, group=group)
        self._opened = []
        bases = [self.raw.data_ptr() if p == self.rank else PeerGather._open(self, hp)
                 for p, hp in enumerate(allh)]
        head_off = h0 * dv * esz
        self._po = []
        for slot in range(2):
            po = _lib.PeerOut()
            peers = [bases[p] + slot * slot_bytes + head_off for p in range(n) if p != self.rank]
            for i, ptr in enumerate(peers):
                po.o_peer[i] = ptr
            for p in range(n):
                po.arrive[p] = bases[p] + flag_off
                po.free_flags[p] = bases[p] + flag_off + 8
            po.cta_done = bases[self.rank] + flag_off + 4
            po.n_ranks, po.rank, po.step = n, self.rank, 1
            self._po.append(po)
        self.step = 0
        self.group = group
        dist.barrier(group=group)

    def local_out(self, slot: int) -> torch.Tensor:
        """This rank's heads inside its own buffer of ``slot`` (the ``out``
        a DecodeStep writes)."""
        return self.out[slot][:, self.h0:self.h0 + self.hv]

    def decode_step(self, slot: int, q, k, v, g, beta, state, **kw):
        from .api import DecodeStep
        return DecodeStep(q, k, v, g, beta, state, out=self.local_out(slot),
                          peer_out=self._po[slot], **kw)

    def launch(self, steps) -> int:
        """Runs the next decode step through ``steps[slot]`` and returns its
        1-based step number."""
        self.step += 1
        slot = self.step % 2
        self._po[slot].step = self.step
        steps[slot]()
        return self.step

    def wait(self, step: int, stream=None) -> torch.Tensor:
        """Stream-waits until every rank's outputs of ``step`` have arrived;
        returns the gathered [B, Hv, d_v] buffer of that step."""
        from .api import status_word
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        self._L.check(self._lib.gdn_gather_wait_counter(
            self.arrive.data_ptr(), (step * self.world) & 0xFFFFFFFF,
            status_word(self.device).data_ptr(), s), "gdn_gather_wait_counter")
        return self.out[step % 2]

    def close(self) -> None:
        for p in self._opened:
            self._lib.gdn_ipc_close(p)
        self._opened = []


def gdn_prefill_seqpar(q, k, v, g, beta, initial_state=None, *, group=None, scale: float = 1.0):
    """Sequence-parallel GDN prefill: rank j of the group holds the j-th
    contiguous T-segment of every sequence (q, k [B, T_j, Hqk, d], v [B, T_j,
    Hv, d], g, beta [B, T_j, Hv]) and gets back that segment's outputs plus the
    state after its segment (on the last rank: the final state).

    The delta-rule recurrence is affine in the state over a segment,
    S_end = M S_start + L, with M = prod_t a_t (I - beta_t k_t k_t^T) (d_k x d_k)
    and L the segment's state from zero.  A middle rank obtains M by running
    the chunked prefill from the identity state with v = 0, and L by running
    it from zero.  Rank 0 without an initial state starts from zero, so its
    segment run already yields L_0 (and M_0 is never needed); the last rank's
    (M, L) are needed by nobody.  One all-gather exchanges the (M_j, L_j);
    each rank scans the segment start states in fp32 and runs its segment from
    its start state for exact outputs.  The critical path is three prefills
    of length T/N (two for N = 2) plus an all-gather of 2 x [B, Hv, d, d]
    fp32.  ``initial_state`` (the state before segment 0) must be given on
    every rank or on none.
    """
    from .api import gdn_prefill
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, T, _, dk = q.shape
    Hv, dv = v.shape[2], v.shape[3]
    if dk != dv:
        raise ValueError("sequence-parallel prefill needs d_k == d_v (M is d_k x d_v)")
    dev = q.device
    zero_start = initial_state is None
    ML = torch.zeros((2, B, Hv, dk, dv), dtype=torch.float32, device=dev)
    first = None
    if rank == 0 and zero_start:
        first = gdn_prefill(q, k, v, g, beta, None, scale=scale)  # its end state is L_0
        ML[1].copy_(first[1])
    elif rank < world - 1:
        eye = torch.eye(dk, dtype=torch.float32, device=dev).expand(B, Hv, dk, dk).contiguous()
        gdn_prefill(q, k, torch.zeros_like(v), g, beta, eye, scale=scale, final_state=ML[0])
        gdn_prefill(q, k, v, g, beta, None, scale=scale, final_state=ML[1])
    allml = torch.empty((world,) + tuple(ML.shape), dtype=ML.dtype, device=dev)
    dist.all_gather_into_tensor(allml.view(-1), ML.reshape(-1), group=group)
    if first is not None:
        return first
    S = (initial_state.float() if not zero_start
         else torch.zeros((B, Hv, dk, dv), dtype=torch.float32, device=dev))
    from . import _lib
    L_ = _lib.load()
    nmat = B * Hv
    for j in range(rank):  # start state of this rank's segment: S <- M_j S + L_j (fp32)
        if j == 0 and zero_start:
            S = allml[0, 1].clone()
        else:
            S = S.contiguous()
            S_next = torch.empty_like(S)
            _lib.check(L_.gdn_state_affine(allml[j, 0].data_ptr(), allml[j, 1].data_ptr(),
                                           S.data_ptr(), S_next.data_ptr(), nmat, dk,
                                           torch.cuda.current_stream(dev).cuda_stream),
                       "gdn_state_affine")
            S = S_next
    return gdn_prefill(q, k, v, g, beta, S.contiguous(), scale=scale)
