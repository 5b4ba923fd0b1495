"""GPU parity of the tcgen05 chunked prefill against the sequential recurrence
(the reference defines prefill only as T decode steps).  Tolerances: bf16
outputs rtol 2e-2 / atol 1e-2; final state max-abs 1e-3."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import O_ATOL, O_RTOL, S_ATOL

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _dev(p):
    return [t.to(DEV) for t in (p.q, p.k, p.v, p.g, p.beta)]


def test_golden_reference_sequential(pkg, golden):
    """Fixture produced by the reference's gdn_decode_reference, token by token."""
    z = golden("baseline_gdn_prefill.npz")
    bf = lambda a: torch.from_numpy(a).to(DEV, torch.bfloat16)
    o, S = pkg.gdn_prefill(bf(z["q"]), bf(z["k"]), bf(z["v"]), bf(z["g"]), bf(z["beta"]),
                           check=True)
    np.testing.assert_allclose(o.float().cpu().numpy(), z["o"], rtol=O_RTOL, atol=O_ATOL)
    assert np.abs(S.cpu().numpy() - z["S_final"]).max() < S_ATOL


@pytest.mark.parametrize("B,T,Hqk,Hv,init,dtype", [
    (1, 64, 1, 1, False, torch.bfloat16),     # one chunk
    (2, 512, 2, 4, False, torch.bfloat16),    # GQA group 2, 8 chunks
    (1, 100, 1, 2, True, torch.bfloat16),     # ragged tail chunk, initial state
    (1, 37, 2, 2, True, torch.bfloat16),      # shorter than one chunk
    (1, 256, 1, 4, True, torch.float16),      # f16 I/O, group 4
])
def test_prefill_matches_oracle(pkg, inputs, orc, B, T, Hqk, Hv, init, dtype):
    p = inputs.make_prefill_inputs(B, T, Hqk, Hv, 128, seed=T + Hv, io_dtype=dtype)
    S0 = (torch.randn((B, Hv, 128, 128), generator=torch.Generator().manual_seed(5)) * 0.02
          if init else None)
    o_ref, s_ref = orc.gdn_prefill(p.q, p.k, p.v, p.g, p.beta, S0)
    o, S = pkg.gdn_prefill(*_dev(p), None if S0 is None else S0.to(DEV), check=True)
    np.testing.assert_allclose(o.float().cpu().numpy(), o_ref, rtol=O_RTOL, atol=O_ATOL)
    assert np.abs(S.cpu().numpy() - s_ref).max() < S_ATOL


def test_prefill_config3_full(pkg, inputs, orc):
    """BASELINE config 3 at full size: B=4, T=4096, Hqk=16, Hv=32, zero state."""
    p = inputs.make_prefill_inputs(4, 4096, 16, 32, 128, seed=3)
    o, S = pkg.gdn_prefill(*_dev(p), check=True)
    o_ref, s_ref = orc.gdn_prefill(p.q, p.k, p.v, p.g, p.beta)
    np.testing.assert_allclose(o.float().cpu().numpy(), o_ref, rtol=O_RTOL, atol=O_ATOL)
    assert np.abs(S.cpu().numpy() - s_ref).max() < S_ATOL


def test_prefill_then_decode_continues(pkg, inputs, orc):
    """A prefill's final state is a valid decode state: prefill T tokens, then
    decode 4 more, against the oracle over all T + 4 tokens."""
    B, T, Hqk, Hv = 2, 192, 2, 4
    p = inputs.make_prefill_inputs(B, T + 4, Hqk, Hv, 128, seed=21)
    pre = [t[:, :T].contiguous().to(DEV) for t in (p.q, p.k, p.v, p.g, p.beta)]
    o, S = pkg.gdn_prefill(*pre, check=True)
    outs = []
    for t in range(T, T + 4):
        outs.append(pkg.gdn_decode(p.q[:, t].to(DEV), p.k[:, t].to(DEV), p.v[:, t].to(DEV),
                                   p.g[:, t].to(DEV), p.beta[:, t].to(DEV), S).float().cpu())
    o_ref, s_ref = orc.gdn_prefill(p.q, p.k, p.v, p.g, p.beta)
    np.testing.assert_allclose(torch.stack(outs, 1).numpy(), o_ref[:, T:], rtol=O_RTOL, atol=O_ATOL)
    assert np.abs(S.cpu().numpy() - s_ref).max() < S_ATOL


def test_prefill_deterministic(pkg, inputs):
    p = inputs.make_prefill_inputs(1, 256, 2, 4, 128, seed=1)
    d = _dev(p)
    o1, s1 = pkg.gdn_prefill(*d)
    o2, s2 = pkg.gdn_prefill(*d)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(s1, s2)


def test_prefill_rejects_bad_sizes(pkg, inputs):
    p = inputs.make_prefill_inputs(1, 64, 1, 1, 64, seed=0)
    with pytest.raises(pkg.GDNError):
        pkg.gdn_prefill(*_dev(p))  # d = 64 is not a prefill size


@pytest.mark.parametrize("count,d", [(3, 128), (2, 64), (1, 256)])
def test_state_affine_matches_fp64(pkg, count, d):
    """gdn_state_affine (the sequence-parallel start-state step) against
    M S + L in float64."""
    gen = torch.Generator().manual_seed(count + d)
    M, L, S = (torch.randn((count, d, d), generator=gen) * 0.1 for _ in range(3))
    Md, Ld, Sd = (t.to("cuda:0") for t in (M, L, S))
    out = torch.empty_like(Sd)
    rc = pkg._lib.load().gdn_state_affine(Md.data_ptr(), Ld.data_ptr(), Sd.data_ptr(),
                                         out.data_ptr(), count, d,
                                         torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    ref = (M.double() @ S.double() + L.double()).numpy()
    assert np.abs(out.cpu().double().numpy() - ref).max() < 1e-5
