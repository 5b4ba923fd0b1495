"""Multi-GPU paths on 2 GPUs: value-head-sharded decode (NCCL gather), the
copy-engine gather, and the sequence-parallel prefill.  The decode and the
prefill are checked against the C oracle (the restatement of the reference's
gdn_decode_reference, pytorch_reference_gdn.py:38-91).  Skipped with fewer
than two GPUs."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import O_ATOL, O_RTOL, S_ATOL, graft

pytestmark = pytest.mark.gpu

B, HQK, HV, D, STEPS = 64, 16, 32, 128, 8


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        pkg = graft.package()
        inputs = graft.submodule("inputs")
        sh = graft.submodule("sharded")
        x = inputs.make_decode_inputs(STEPS, B, HQK, HV, D, seed=17)
        s = sh.shard_heads(HV, HQK, world, rank)
        dev = torch.device("cuda", rank)
        dec = sh.ShardedGDNDecoder(B, HQK, HV, D, D, device=dev,
                                   state=x.state[:, s.h0:s.h1].contiguous().to(dev))
        outs = []
        for t in range(STEPS):
            o = dec.step(x.q[t].to(dev), x.k[t].to(dev), x.v[t].to(dev), x.g[t].to(dev),
                         x.beta[t].to(dev), gather=True)
            outs.append(o.float().cpu())
        pkg.check_device_status(dev)
        states = [torch.empty_like(dec.state) for _ in range(world)]
        dist.all_gather(states, dec.state)
        if rank == 0:
            q.put((torch.stack(outs).numpy(), torch.cat([t.cpu() for t in states], 1).numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_sharded_decode_two_gpus_matches_oracle(orc, inputs):
    """8 steps on 2 ranks (16 value heads each): every gathered output row and
    every state shard against the oracle over all 32 heads."""
    x = inputs.make_decode_inputs(STEPS, B, HQK, HV, D, seed=17)
    ref_o, ref_s = orc.gdn_decode_steps(x.q, x.k, x.v, x.g, x.beta, x.state)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    o, s = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    np.testing.assert_allclose(o, ref_o, rtol=O_RTOL, atol=O_ATOL)
    assert np.abs(s - ref_s).max() < S_ATOL


def _gather_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        sh = graft.submodule("sharded")
        dev = torch.device("cuda", rank)
        n = 4096 + 8
        pg = sh.PeerGather(n, torch.bfloat16, dev)
        side = torch.cuda.Stream(dev)
        peers = [torch.cuda.Stream(dev) for _ in range(world)]
        ok = True
        for step in range(1, 7):
            src = torch.full((n,), float(100 * step + rank), dtype=torch.bfloat16, device=dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            if step % 2:
                pg.push(src, step, side)
            else:  # one stream (copy engine) per destination rank
                for ps in peers:
                    ps.wait_stream(side)
                pg.push(src, step, peer_streams=peers)
                for ps in peers:
                    side.wait_stream(ps)
            got = pg.wait(step, side)
            with torch.cuda.stream(side):
                snap = got.clone()
            pg.release(step, side)
            side.synchronize()
            want = torch.tensor([100.0 * step + r for r in range(world)]).view(world, 1).expand(world, n)
            want = want.to(torch.bfloat16).float()  # same rounding as the pushed data
            ok = ok and torch.equal(snap.float().cpu(), want)
        dist.barrier()
        pg.close()
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_copy_engine_gather_two_gpus():
    """The copy-engine all-gather delivers every rank's slice, step after step,
    through both buffer slots."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res == {0: True, 1: True}


def _seqpar_worker(rank, world, port, q, with_init=True):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        torch.backends.cuda.matmul.allow_tf32 = False
        sh = graft.submodule("sharded")
        inputs = graft.submodule("inputs")
        p = inputs.make_prefill_inputs(1, 300, 2, 4, 128, seed=9)
        S0 = torch.randn((1, 4, 128, 128), generator=torch.Generator().manual_seed(3)) * 0.02
        cut = [0, 128, 300]  # uneven segments, the second one ragged
        seg = [t[:, cut[rank]:cut[rank + 1]].contiguous().cuda() for t in (p.q, p.k, p.v, p.g, p.beta)]
        o, S = sh.gdn_prefill_seqpar(*seg, S0.cuda() if with_init else None)
        q.put((rank, o.float().cpu().numpy(), S.cpu().numpy()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
@pytest.mark.parametrize("with_init", [True, False])
def test_sequence_parallel_prefill_two_gpus(with_init):
    """T split over two GPUs: outputs of both segments and the final state
    match the sequential recurrence over the whole sequence (with an initial
    state, and from zero, where rank 0's own run supplies its segment map)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_seqpar_worker, args=(r, 2, port, q, with_init)) for r in range(2)]
    for p in procs:
        p.start()
    res = {r: (o, S) for r, o, S in (q.get(timeout=300) for _ in range(2))}
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    inputs = graft.submodule("inputs")
    p = inputs.make_prefill_inputs(1, 300, 2, 4, 128, seed=9)
    S0 = torch.randn((1, 4, 128, 128), generator=torch.Generator().manual_seed(3)) * 0.02
    o_ref, s_ref = graft.oracle().gdn_prefill(p.q, p.k, p.v, p.g, p.beta, S0 if with_init else None)
    o = np.concatenate([res[0][0], res[1][0]], axis=1)
    np.testing.assert_allclose(o, o_ref, rtol=2e-2, atol=1e-2)
    assert np.abs(res[1][1] - s_ref).max() < 1e-3


def _fused_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        pkg = graft.package()
        inputs = graft.submodule("inputs")
        sh = graft.submodule("sharded")
        dev = torch.device("cuda", rank)
        x = inputs.make_decode_inputs(STEPS, B, HQK, HV, D, seed=23)
        s = sh.shard_heads(HV, HQK, world, rank)
        hv = s.h1 - s.h0
        state = x.state[:, s.h0:s.h1].contiguous().to(dev)
        fg = sh.FusedGather(B, HV, D, s.h0, hv, torch.bfloat16, dev)
        outs = []
        for t in range(STEPS):
            ins = [x.q[t, :, s.hq0:s.hq1], x.k[t, :, s.hq0:s.hq1], x.v[t, :, s.h0:s.h1],
                   x.g[t, :, s.h0:s.h1], x.beta[t, :, s.h0:s.h1]]
            ins = [u.contiguous().to(dev) for u in ins]
            pair = [fg.decode_step(slot, *ins, state) for slot in range(2)]
            step = fg.launch(pair)
            full = fg.wait(step)
            outs.append(full.float().cpu())  # read before the next launch
        pkg.check_device_status(dev)
        states = [torch.empty_like(state) for _ in range(world)]
        dist.all_gather(states, state)
        dist.barrier()
        fg.close()
        if rank == 0:
            q.put((torch.stack(outs).numpy(), torch.cat([t.cpu() for t in states], 1).numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_fused_gather_decode_two_gpus_matches_oracle(orc, inputs):
    """Decode with the output all-gather fused into the kernel: every step's
    gathered [B, Hv, d] on rank 0 and the state shards against the oracle."""
    x = inputs.make_decode_inputs(STEPS, B, HQK, HV, D, seed=23)
    ref_o, ref_s = orc.gdn_decode_steps(x.q, x.k, x.v, x.g, x.beta, x.state)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_fused_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    o, s = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    np.testing.assert_allclose(o, ref_o, rtol=O_RTOL, atol=O_ATOL)
    assert np.abs(s - ref_s).max() < S_ATOL
