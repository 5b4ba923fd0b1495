"""GPU parity of the KDA prefill against the reference KDA step applied token
by token (float64 oracle).  Tolerances: bf16 outputs rtol 2e-2 / atol 1e-2;
final state max-abs 1e-3.  Both forms are covered: the chunked tensor-core
form (d = 128, the default there) and the recurrent form (every d)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import O_ATOL, O_RTOL, S_ATOL

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _dev(p):
    return [t.to(DEV) for t in (p.q, p.k, p.v, p.g, p.beta)]


def _state(B, H, d, seed=5):
    return torch.randn((B, H, d, d), generator=torch.Generator().manual_seed(seed)) * 0.02


@pytest.mark.parametrize("B,T,Hqk,Hv,d,init,io,gdt", [
    (1, 16, 1, 1, 128, False, torch.bfloat16, torch.float32),   # one staged chunk
    (2, 100, 2, 4, 128, True, torch.bfloat16, torch.float32),   # ragged tail, GQA 2
    (1, 37, 1, 2, 64, True, torch.float16, torch.bfloat16),     # d = 64, f16 I/O, bf16 gate
    (1, 40, 2, 2, 256, True, torch.bfloat16, torch.float32),    # d = 256 (Qwen3-Next geometry)
    (3, 1, 1, 1, 128, True, torch.bfloat16, torch.float32),     # a single token
])
def test_kda_prefill_matches_oracle(pkg, inputs, orc, B, T, Hqk, Hv, d, init, io, gdt):
    p = inputs.make_kda_prefill_inputs(B, T, Hqk, Hv, d, seed=T + d, io_dtype=io, g_dtype=gdt)
    S0 = _state(B, Hv, d) if init else None
    o_ref, s_ref = orc.kda_prefill(p.q, p.k, p.v, p.g, p.beta,
                                   None if S0 is None else S0.double().numpy(), scale=0.75)
    o, S = pkg.kda_prefill(*_dev(p), None if S0 is None else S0.to(DEV), scale=0.75, check=True)
    np.testing.assert_allclose(o.float().cpu().numpy(), o_ref, rtol=O_RTOL, atol=O_ATOL)
    assert np.abs(S.cpu().numpy() - s_ref).max() < S_ATOL


@pytest.mark.parametrize("dk,dv", [(128, 64), (64, 256), (256, 128)])
def test_kda_prefill_unequal_head_dims(pkg, inputs, orc, dk, dv):
    """d_k != d_v: the state is [B, Hv, d_k, d_v], the gate [B, T, Hv, d_k]
    and v / o have d_v columns split into slabs."""
    B, T, Hqk, Hv = 2, 45, 1, 2
    p = inputs.make_kda_prefill_inputs(B, T, Hqk, Hv, dk, seed=dk + dv)
    v = torch.randn((B, T, Hv, dv), generator=torch.Generator().manual_seed(dv)).to(torch.bfloat16)
    S0 = torch.randn((B, Hv, dk, dv), generator=torch.Generator().manual_seed(3)) * 0.02
    o_ref, s_ref = orc.kda_prefill(p.q, p.k, v, p.g, p.beta, S0.double().numpy())
    o, S = pkg.kda_prefill(p.q.to(DEV), p.k.to(DEV), v.to(DEV), p.g.to(DEV), p.beta.to(DEV),
                           S0.to(DEV), check=True)
    assert tuple(o.shape) == (B, T, Hv, dv) and tuple(S.shape) == (B, Hv, dk, dv)
    np.testing.assert_allclose(o.float().cpu().numpy(), o_ref, rtol=O_RTOL, atol=O_ATOL)
    assert np.abs(S.cpu().numpy() - s_ref).max() < S_ATOL


@pytest.mark.parametrize("form", ["chunked", "recurrent"])
def test_kda_prefill_long_sequence(pkg, inputs, orc, form):
    """T = 4096 (the prefill length of the GDN prefill config), 8 heads."""
    p = inputs.make_kda_prefill_inputs(1, 4096, 8, 8, 128, seed=4)
    o, S = pkg.kda_prefill(*_dev(p), form=form, check=True)
    o_ref, s_ref = orc.kda_prefill(p.q, p.k, p.v, p.g, p.beta)
    np.testing.assert_allclose(o.float().cpu().numpy(), o_ref, rtol=O_RTOL, atol=O_ATOL)
    assert np.abs(S.cpu().numpy() - s_ref).max() < S_ATOL


def test_kda_prefill_then_decode_continues(pkg, inputs, orc):
    """The prefill's final state continues under kda_decode: prefill T tokens
    in place on the initial state, decode 3 more, against the oracle."""
    B, T, H, d = 2, 50, 2, 128
    p = inputs.make_kda_prefill_inputs(B, T + 3, H, H, d, seed=8)
    S = _state(B, H, d).to(DEV)
    S0 = S.double().cpu().numpy()
    pre = [t[:, :T].contiguous().to(DEV) for t in (p.q, p.k, p.v, p.g, p.beta)]
    pkg.kda_prefill(*pre, S, final_state=S, check=True)  # in place
    outs = []
    for t in range(T, T + 3):
        outs.append(pkg.kda_decode(p.q[:, t].to(DEV), p.k[:, t].to(DEV), p.v[:, t].to(DEV),
                                   p.g[:, t].to(DEV), p.beta[:, t].float().to(DEV), S)
                    .float().cpu())
    o_ref, s_ref = orc.kda_prefill(p.q, p.k, p.v, p.g, p.beta, S0)
    np.testing.assert_allclose(torch.stack(outs, 1).numpy(), o_ref[:, T:], rtol=O_RTOL,
                               atol=O_ATOL)
    assert np.abs(S.cpu().numpy() - s_ref).max() < S_ATOL


def test_kda_prefill_deterministic(pkg, inputs):
    p = inputs.make_kda_prefill_inputs(1, 64, 2, 4, 128, seed=1)
    d = _dev(p)
    o1, s1 = pkg.kda_prefill(*d)
    o2, s2 = pkg.kda_prefill(*d)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(s1, s2)


def test_kda_prefill_rejects_bad_args(pkg, inputs):
    p = inputs.make_kda_prefill_inputs(1, 16, 1, 1, 96, seed=0)
    with pytest.raises(pkg.GDNError):
        pkg.kda_prefill(*_dev(p))  # d = 96 is not a kernel size
    p = inputs.make_kda_prefill_inputs(1, 16, 1, 1, 128, seed=0)
    q, k, v, g, beta = _dev(p)
    with pytest.raises(pkg.GDNError):
        pkg.kda_prefill(q, k, v, g[..., 0].contiguous(), beta)  # a GDN (per-head) gate


@pytest.mark.parametrize("form", ["chunked", "recurrent"])
@pytest.mark.parametrize("kind", ["strong", "underflow"])
def test_kda_prefill_extreme_gates(pkg, inputs, orc, kind, form):
    """Gates far outside the config distribution: strong decay (g down to -30
    per token) and gates whose exp() underflows to zero (g = -200).  The
    kernel's rescaled state must renormalise mid-chunk and stay finite."""
    p = inputs.make_kda_prefill_inputs(2, 70, 2, 2, 128, seed=31)
    gen = torch.Generator().manual_seed(7)
    if kind == "strong":
        g = -30.0 * torch.rand(p.g.shape, generator=gen)
    else:
        g = torch.where(torch.rand(p.g.shape, generator=gen) < 0.1, -200.0, -0.05)
    S0 = _state(2, 2, 128)
    o_ref, s_ref = orc.kda_prefill(p.q, p.k, p.v, g, p.beta, S0.double().numpy())
    o, S = pkg.kda_prefill(p.q.to(DEV), p.k.to(DEV), p.v.to(DEV), g.to(DEV), p.beta.to(DEV),
                           S0.to(DEV), form=form, check=True)
    assert torch.isfinite(o.float()).all() and torch.isfinite(S).all()
    np.testing.assert_allclose(o.float().cpu().numpy(), o_ref, rtol=O_RTOL, atol=O_ATOL)
    assert np.abs(S.cpu().numpy() - s_ref).max() < S_ATOL


@pytest.mark.parametrize("B,T,Hqk,Hv,init,io,gdt", [
    (1, 64, 1, 1, False, torch.bfloat16, torch.float32),    # one whole chunk
    (2, 100, 2, 4, True, torch.bfloat16, torch.float32),    # ragged tail, GQA 2
    (1, 200, 1, 2, True, torch.float16, torch.bfloat16),    # f16 I/O, bf16 gate, 4 chunks
    (1, 77, 2, 2, True, torch.bfloat16, torch.float16),     # f16 gate
    (3, 1, 1, 1, True, torch.bfloat16, torch.float32),      # a single token
])
def test_kda_chunked_matches_oracle(pkg, inputs, orc, B, T, Hqk, Hv, init, io, gdt):
    """The chunked form on its own (d = 128): ragged chunks, GQA, gate and I/O
    dtypes, against the float64 reference recurrence."""
    p = inputs.make_kda_prefill_inputs(B, T, Hqk, Hv, 128, seed=T + 7, io_dtype=io, g_dtype=gdt)
    S0 = _state(B, Hv, 128) if init else None
    o_ref, s_ref = orc.kda_prefill(p.q, p.k, p.v, p.g, p.beta,
                                   None if S0 is None else S0.double().numpy(), scale=0.75)
    o, S = pkg.kda_prefill(*_dev(p), None if S0 is None else S0.to(DEV), scale=0.75,
                           form="chunked", check=True)
    np.testing.assert_allclose(o.float().cpu().numpy(), o_ref, rtol=O_RTOL, atol=O_ATOL)
    assert np.abs(S.cpu().numpy() - s_ref).max() < S_ATOL


def test_kda_chunked_equals_recurrent_at_config_size(pkg, inputs):
    """B = 4, T = 4096, H = 32 (the bench workload): the two forms agree on
    every output and state element (the oracle would take minutes here; the
    recurrent form is itself pinned to it above)."""
    p = inputs.make_kda_prefill_inputs(4, 4096, 32, 32, 128, seed=3, device=DEV)
    x = (p.q, p.k, p.v, p.g, p.beta)
    oc, sc = pkg.kda_prefill(*x, form="chunked", check=True)
    orr, sr = pkg.kda_prefill(*x, form="recurrent", check=True)
    np.testing.assert_allclose(oc.float().cpu().numpy(), orr.float().cpu().numpy(),
                               rtol=O_RTOL, atol=O_ATOL)
    assert float((sc - sr).abs().max()) < S_ATOL


def test_kda_chunked_rejects_other_head_dims(pkg, inputs):
    p = inputs.make_kda_prefill_inputs(1, 16, 1, 1, 64, seed=0)
    with pytest.raises(pkg.GDNError):
        pkg.kda_prefill(*_dev(p), form="chunked")


def test_kda_chunked_rejects_small_or_foreign_workspace(pkg, inputs):
    """A caller-supplied workspace must be on the inputs' device and large
    enough; both are refused before any launch."""
    p = inputs.make_kda_prefill_inputs(1, 128, 1, 1, 128, seed=0)
    x = _dev(p)
    with pytest.raises(pkg.GDNError):
        pkg.kda_prefill(*x, form="chunked", workspace=torch.empty(1024, dtype=torch.uint8, device=DEV))
    with pytest.raises(pkg.GDNError):
        pkg.kda_prefill(*x, form="chunked", workspace=torch.empty(1 << 20, dtype=torch.uint8))
