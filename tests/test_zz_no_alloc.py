"""gdn_prefill_launch_noalloc, the chunked prefill that allocates nothing.

Some callers of this library cannot allocate device memory: a plugin inside
a host framework that owns the GPU memory pool and gives the plugin no
allocator, or a serving path that must not run into cudaMalloc's implicit
device synchronisation.  For them the C ABI offers one entry point whose
workspace is a fixed array inside the library instead of caller memory.
This test calls it through the C ABI and checks that two calls in a row give
the results of the allocating entry point (gdn_prefill_launch with a
caller-owned workspace), within the tolerances of the other parity tests,
and that a problem larger than the fixed array is refused before launch.

The file name sorts last so that a run stopping at the first failure has
already run every other test; the test also passes alone in a fresh process.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import O_ATOL, O_RTOL, S_ATOL, graft

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _noalloc(pkg, api, q, k, v, g, beta, S0, out, final_state):
    L = pkg._lib.load()
    a = api._prefill_args(q, k, v, g, beta, S0, final_state, out, 64, 1.0)
    a.workspace, a.workspace_bytes = None, 0  # ignored by the no-alloc entry point
    return L.gdn_prefill_launch_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)


def test_noalloc_prefill_matches_allocating_entry_point(pkg, inputs):
    api = graft.submodule("api")
    torch.cuda.set_device(0)
    B, T, Hqk, Hv = 2, 200, 2, 4  # 2 x 4 x 4 = 32 workspace records
    for call, seed in enumerate((41, 42)):  # two calls in a row, different inputs
        p = inputs.make_prefill_inputs(B, T, Hqk, Hv, 128, seed=seed)
        x = [t.to(DEV) for t in (p.q, p.k, p.v, p.g, p.beta)]
        S0 = (torch.randn((B, Hv, 128, 128), generator=torch.Generator().manual_seed(seed)) * 0.02
              ).to(DEV)
        o_ref, s_ref = pkg.gdn_prefill(*x, S0, check=True)
        o = torch.full_like(o_ref, float("nan"))
        fs = torch.full_like(s_ref, float("nan"))
        rc = _noalloc(pkg, api, *x, S0, o, fs)
        assert rc == 0, f"call {call}: {pkg._lib.status_string(rc)}"
        pkg.check_device_status(torch.device(DEV))
        np.testing.assert_allclose(o.float().cpu().numpy(), o_ref.float().cpu().numpy(),
                                   rtol=O_RTOL, atol=O_ATOL)
        assert float((fs - s_ref).abs().max()) < S_ATOL


def test_noalloc_prefill_rejects_problems_beyond_its_scratch(pkg, inputs):
    api = graft.submodule("api")
    # 1 x 32 x ceil(4096 / 64) = 2048 records > the 668 the fixed array holds
    p = inputs.make_prefill_inputs(1, 4096, 16, 32, 128, seed=1)
    x = [t.to(DEV) for t in (p.q, p.k, p.v, p.g, p.beta)]
    o = torch.empty((1, 4096, 32, 128), dtype=torch.bfloat16, device=DEV)
    fs = torch.empty((1, 32, 128, 128), dtype=torch.float32, device=DEV)
    rc = _noalloc(pkg, api, *x, None, o, fs)
    assert rc == 7, pkg._lib.status_string(rc)  # GDN_ERR_WORKSPACE, nothing launched
