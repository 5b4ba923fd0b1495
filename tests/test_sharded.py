"""Head-sharded decode: shard arithmetic, and the 2-rank gather path on gloo
(CPU) with the oracle standing in for the per-rank kernel."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import graft


def test_shard_heads_partition():
    sh = graft.submodule("sharded")
    for world in (1, 2, 4, 8):
        seen = []
        for r in range(world):
            s = sh.shard_heads(32, 16, world, r)
            assert s.h1 - s.h0 == 32 // world
            assert s.hq0 == s.h0 // 2 and s.hq1 == (s.h1 - 1) // 2 + 1
            seen += list(range(s.h0, s.h1))
        assert seen == list(range(32))
    with pytest.raises(ValueError):
        sh.shard_heads(32, 16, 3, 0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_step(q, k, v, g, beta, state, scale=1.0):
    orc = graft.oracle()
    o, S = orc.gdn_decode_steps(q[None], k[None], v[None], g[None], beta[None], state,
                                scale=scale)
    state.copy_(torch.from_numpy(S))
    return torch.from_numpy(o[0])


def _worker(rank, world, port, steps, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = graft.submodule("sharded")
        inputs = graft.submodule("inputs")
        x = inputs.make_decode_inputs(steps, 2, 4, 8, 64, seed=11)
        s = sh.shard_heads(8, 4, world, rank)
        dec = sh.ShardedGDNDecoder(2, 4, 8, 64, 64, device="cpu",
                                   state=x.state[:, s.h0:s.h1].clone(), step_fn=_oracle_step)
        outs = [dec.step(x.q[t], x.k[t], x.v[t], x.g[t], x.beta[t], gather=True).numpy()
                for t in range(steps)]
        full_state = [torch.empty_like(dec.state) for _ in range(world)]
        dist.all_gather(full_state, dec.state)
        if rank == 0:
            result_q.put((np.stack(outs), torch.cat(full_state, dim=1).numpy()))
    finally:
        dist.destroy_process_group()


def test_sharded_gather_matches_unsharded_gloo():
    steps, world = 3, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, _free_port_once(), steps, q))
             for r in range(world)]
    for p in procs:
        p.start()
    o_sh, S_sh = q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    inputs = graft.submodule("inputs")
    x = inputs.make_decode_inputs(steps, 2, 4, 8, 64, seed=11)
    o, S = graft.oracle().gdn_decode_steps(x.q, x.k, x.v, x.g, x.beta, x.state)
    assert np.array_equal(o_sh, o)
    assert np.array_equal(S_sh, S)


_PORT = None


def _free_port_once():
    global _PORT
    if _PORT is None:
        _PORT = _free_port()
    return _PORT
