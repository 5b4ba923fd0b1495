"""GPU parity of the decode kernels against the oracle (tolerances from
BASELINE: bf16 outputs rtol 2e-2 / atol 1e-2, state max-abs 1e-3; the
reference's own f16 harness tolerance 5e-3 for the reference-layout calls)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import O_ATOL, O_RTOL, S_ATOL

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _run_gdn(pkg, x, steps=None, **kw):
    st = x.state.to(DEV)
    outs = []
    for t in range(x.q.shape[0] if steps is None else steps):
        o = pkg.gdn_decode(x.q[t].to(DEV), x.k[t].to(DEV), x.v[t].to(DEV), x.g[t].to(DEV),
                           x.beta[t].to(DEV), st, **kw)
        outs.append(o.float().cpu())
    pkg.check_device_status()
    return torch.stack(outs).numpy(), st.cpu().numpy()


def test_golden_baseline_gdn_64_steps(pkg, golden):
    """BASELINE config-0 distributions, 64 steps, against the reference's own
    recurrence (fixture made by the reference code)."""
    z = golden("baseline_gdn_decode.npz")
    st = torch.from_numpy(z["S0"]).to(DEV)
    bf = lambda a: torch.from_numpy(a).to(DEV, torch.bfloat16)
    for t in range(z["q"].shape[0]):
        o = pkg.gdn_decode(bf(z["q"][t]), bf(z["k"][t]), bf(z["v"][t]),
                           torch.from_numpy(z["g"][t]).to(DEV), torch.from_numpy(z["beta"][t]).to(DEV),
                           st)
        np.testing.assert_allclose(o.float().cpu().numpy(), z["o"][t], rtol=O_RTOL, atol=O_ATOL)
    pkg.check_device_status()
    assert np.abs(st.cpu().numpy() - z["S_final"]).max() < S_ATOL


def test_golden_reference_layout_f16(pkg, golden):
    """The reference's own inputs through the reference-layout entry point."""
    z = golden("ref_gdn_correctness.npz")
    B, H, dk = z["q_f16"].shape
    dv = z["v_f16"].shape[-1]
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    Q, K, V = t(z["q_f16"].reshape(B * H, dk)), t(z["k_f16"].reshape(B * H, dk)), t(z["v_f16"].reshape(B * H, dv))
    A, Bt = t(z["alpha_f16"].reshape(B * H, 1)), t(z["beta_f16"].reshape(B * H, 1))
    S_in = t(z["S_in"].reshape(B * H * dk, dv))
    S_out = torch.zeros_like(S_in)
    O = torch.zeros((B * H, dv), dtype=torch.float16, device=DEV)
    pkg.gdn_decode_ref(Q, K, V, A, Bt, S_in, S_out, O, batch=B, n_heads=H, d_k=dk, d_v=dv)
    torch.cuda.synchronize()
    np.testing.assert_allclose(O.float().cpu().numpy().reshape(B, H, dv),
                               z["o_expected_f16"].astype(np.float32), atol=5e-3, rtol=5e-3)
    assert np.abs(S_out.cpu().numpy().reshape(B, H, dk, dv) - z["S_out_expected"]).max() < 5e-6
    assert torch.equal(S_in.cpu(), torch.from_numpy(z["S_in"].reshape(B * H * dk, dv)))  # untouched


def test_golden_reference_layout_kda_f16(pkg, golden):
    z = golden("ref_kda_correctness.npz")
    B, H, dk = z["q_f16"].shape
    dv = z["v_f16"].shape[-1]
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    S_in = t(z["S_in_f32"].reshape(B * H * dk, dv))
    O = torch.zeros((B * H, dv), dtype=torch.float16, device=DEV)
    pkg.kda_decode_ref(t(z["q_f16"].reshape(B * H, dk)), t(z["k_f16"].reshape(B * H, dk)),
                       t(z["v_f16"].reshape(B * H, dv)), t(z["g_f16"].reshape(B * H, dk)),
                       t(z["beta_f16"].reshape(B * H, 1)), S_in, S_in, O,
                       batch=B, n_heads=H, d_k=dk, d_v=dv)  # in place
    torch.cuda.synchronize()
    np.testing.assert_allclose(O.float().cpu().numpy().reshape(B, H, dv),
                               z["o_expected_f16"].astype(np.float32), atol=5e-3, rtol=5e-3)
    assert np.abs(S_in.cpu().numpy().reshape(B, H, dk, dv) - z["S_out_expected_f32"]).max() < 1e-5


def test_golden_baseline_kda_16_steps(pkg, golden):
    z = golden("baseline_kda_decode.npz")
    st = torch.from_numpy(z["S0"]).to(DEV)
    bf = lambda a: torch.from_numpy(a).to(DEV, torch.bfloat16)
    for t in range(z["q"].shape[0]):
        o = pkg.kda_decode(bf(z["q"][t]), bf(z["k"][t]), bf(z["v"][t]),
                           torch.from_numpy(z["g"][t]).to(DEV), torch.from_numpy(z["beta"][t]).to(DEV),
                           st)
        np.testing.assert_allclose(o.float().cpu().numpy(), z["o"][t], rtol=O_RTOL, atol=O_ATOL)
    pkg.check_device_status()
    assert np.abs(st.cpu().numpy() - z["S_final"]).max() < S_ATOL


@pytest.mark.parametrize("B,Hqk,Hv,d,steps", [
    (8, 16, 32, 128, 64),     # config 0 (32-column TMA tile slabs: few heads)
    (10, 16, 32, 128, 4),     # 64-column TMA tile slabs
    (64, 16, 32, 128, 4),     # config 1 smallest batch (whole-row bulk-copy slabs)
    (3, 1, 4, 128, 8),        # group of 4, ragged batch
    (2, 2, 2, 64, 8),         # d = 64
    (1, 2, 4, 256, 4),        # d = 256 (reference qwen3 head size), 32-column slabs
    (40, 2, 4, 256, 2),       # d = 256, 64-column slabs
])
def test_gdn_decode_matches_oracle(pkg, inputs, orc, B, Hqk, Hv, d, steps):
    x = inputs.make_decode_inputs(steps, B, Hqk, Hv, d, seed=B * 7 + d)
    o_ref, s_ref = orc.gdn_decode_steps(x.q, x.k, x.v, x.g, x.beta, x.state)
    o, s = _run_gdn(pkg, x)
    np.testing.assert_allclose(o, o_ref, rtol=O_RTOL, atol=O_ATOL)
    assert np.abs(s - s_ref).max() < S_ATOL


@pytest.mark.parametrize("B,H,steps", [(64, 32, 64), (2, 4, 8)])
def test_kda_decode_matches_oracle(pkg, inputs, orc, B, H, steps):
    """Config 2 (B=64, H=32, 64 steps) against the float64 oracle."""
    x = inputs.make_decode_inputs(steps, B, H, H, 128, kda=True, seed=2)
    o_ref, s_ref = orc.kda_decode_steps(x.q, x.k, x.v, x.g, x.beta, x.state)
    st = x.state.to(DEV)
    for t in range(steps):
        o = pkg.kda_decode(x.q[t].to(DEV), x.k[t].to(DEV), x.v[t].to(DEV), x.g[t].to(DEV),
                           x.beta[t].to(DEV), st)
        np.testing.assert_allclose(o.float().cpu().numpy(), o_ref[t], rtol=O_RTOL, atol=O_ATOL)
    pkg.check_device_status()
    assert np.abs(st.cpu().numpy() - s_ref).max() < S_ATOL


def test_large_batch_single_step_sampled(pkg, inputs, orc):
    """Config 1 at B=1024: one in-place step on the GPU; a sample of sequences
    is checked against the oracle (the oracle runs on the sampled rows only)."""
    B, Hqk, Hv, d = 1024, 16, 32, 128
    x = inputs.make_decode_inputs(1, B, Hqk, Hv, d, seed=123)
    o, s = _run_gdn(pkg, x)
    idx = np.array([0, 1, 77, 511, 512, 1000, 1023])
    sub = lambda t: t[:, idx] if t.dim() >= 3 else t
    o_ref, s_ref = orc.gdn_decode_steps(sub(x.q), sub(x.k), sub(x.v), x.g[:, idx], x.beta[:, idx],
                                        x.state[idx])
    np.testing.assert_allclose(o[:, idx], o_ref, rtol=O_RTOL, atol=O_ATOL)
    assert np.abs(s[idx] - s_ref).max() < S_ATOL
    assert np.isfinite(s).all()


def test_strided_inputs_and_out_of_place(pkg, inputs, orc):
    """q/k/v as slices of a fused projection buffer; state written out of place."""
    B, Hqk, Hv, d = 4, 2, 4, 128
    x = inputs.make_decode_inputs(1, B, Hqk, Hv, d, seed=9)
    fused = torch.zeros((B, 2 * Hqk + Hv + 1, d), dtype=torch.bfloat16, device=DEV)
    fused[:, :Hqk] = x.q[0].to(DEV)
    fused[:, Hqk:2 * Hqk] = x.k[0].to(DEV)
    fused[:, 2 * Hqk:2 * Hqk + Hv] = x.v[0].to(DEV)
    q, k, v = fused[:, :Hqk], fused[:, Hqk:2 * Hqk], fused[:, 2 * Hqk:2 * Hqk + Hv]
    S_in = x.state.to(DEV)
    S_out = torch.full_like(S_in, float("nan"))
    o = pkg.gdn_decode(q, k, v, x.g[0].to(DEV), x.beta[0].to(DEV), S_in, state_out=S_out,
                       check=True)
    o_ref, s_ref = orc.gdn_decode_steps(x.q, x.k, x.v, x.g, x.beta, x.state)
    np.testing.assert_allclose(o.float().cpu().numpy(), o_ref[0], rtol=O_RTOL, atol=O_ATOL)
    assert np.abs(S_out.cpu().numpy() - s_ref).max() < S_ATOL  # NaN canary fully overwritten
    assert torch.equal(S_in.cpu(), x.state)


def test_bf16_gates_and_linear_gate(pkg, inputs, orc):
    B, Hqk, Hv, d = 2, 2, 4, 128
    x = inputs.make_decode_inputs(1, B, Hqk, Hv, d, seed=4)
    g16, b16 = x.g.to(torch.bfloat16), x.beta.to(torch.bfloat16)
    o_ref, s_ref = orc.gdn_decode_steps(x.q, x.k, x.v, g16.float(), b16.float(), x.state)
    st = x.state.to(DEV)
    o = pkg.gdn_decode(x.q[0].to(DEV), x.k[0].to(DEV), x.v[0].to(DEV), g16[0].to(DEV),
                       b16[0].to(DEV), st, check=True)
    np.testing.assert_allclose(o.float().cpu().numpy(), o_ref[0], rtol=O_RTOL, atol=O_ATOL)
    assert np.abs(st.cpu().numpy() - s_ref).max() < S_ATOL
    # linear gate: alpha passed directly
    st = x.state.to(DEV)
    o = pkg.gdn_decode(x.q[0].to(DEV), x.k[0].to(DEV), x.v[0].to(DEV), torch.exp(x.g[0]).to(DEV),
                       x.beta[0].to(DEV), st, gate="linear", check=True)
    o_ref, s_ref = orc.gdn_decode_steps(x.q, x.k, x.v, torch.exp(x.g), x.beta, x.state,
                                        gate="linear")
    np.testing.assert_allclose(o.float().cpu().numpy(), o_ref[0], rtol=O_RTOL, atol=O_ATOL)
    assert np.abs(st.cpu().numpy() - s_ref).max() < S_ATOL


def test_scale_argument(pkg, inputs, orc):
    x = inputs.make_decode_inputs(1, 2, 2, 2, 128, seed=6)
    st = x.state.to(DEV)
    o = pkg.gdn_decode(x.q[0].to(DEV), x.k[0].to(DEV), x.v[0].to(DEV), x.g[0].to(DEV),
                       x.beta[0].to(DEV), st, scale=0.0883883)
    o_ref, _ = orc.gdn_decode_steps(x.q, x.k, x.v, x.g, x.beta, x.state, scale=0.0883883)
    np.testing.assert_allclose(o.float().cpu().numpy(), o_ref[0], rtol=O_RTOL, atol=O_ATOL)


def test_deterministic_and_graph_capturable(pkg, inputs):
    """Bitwise repeatable (no atomics), and a captured CUDA graph of the bound
    launch gives the same state as eager calls."""
    x = inputs.make_decode_inputs(4, 16, 16, 32, 128, seed=8)
    dq = [t.to(DEV) for t in (x.q, x.k, x.v, x.g, x.beta)]
    s1, s2 = x.state.to(DEV), x.state.to(DEV)
    for t in range(4):
        pkg.gdn_decode(dq[0][t], dq[1][t], dq[2][t], dq[3][t], dq[4][t], s1)
    bufs = [d[0].clone() for d in dq]
    step = pkg.DecodeStep(*bufs, s2)
    step()  # warm-up (sets the kernel attributes outside capture)
    s2.copy_(x.state.to(DEV))
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            step()
    for t in range(4):
        for b, d in zip(bufs, dq):
            b.copy_(d[t])
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(s1, s2)
    pkg.check_device_status()


def test_bad_shapes_raise(pkg):
    q = torch.zeros(2, 2, 128, dtype=torch.bfloat16, device=DEV)
    v = torch.zeros(2, 3, 128, dtype=torch.bfloat16, device=DEV)
    g = torch.zeros(2, 3, device=DEV)
    S = torch.zeros(2, 3, 128, 128, device=DEV)
    with pytest.raises(pkg.GDNError):
        pkg.gdn_decode(q, q, v, g, g, S)  # Hv=3 not a multiple of Hqk=2
    with pytest.raises(pkg.GDNError):
        pkg.gdn_decode(q.float(), q.float(), v.float(), g, g, S)  # fp32 I/O


def test_fused_layer_preprocessing(pkg, inputs, orc):
    """Raw projections in, fused preprocessing in the kernel: q/k L2-normalised
    per head and the log gate computed from the raw gate projection a as
    -exp(A_log) * softplus(a + dt_bias), against the oracle fed with the
    preprocessed values."""
    import torch.nn.functional as F
    steps, B, Hqk, Hv, d = 8, 4, 2, 4, 128
    gen = torch.Generator().manual_seed(31)
    q = (torch.randn((steps, B, Hqk, d), generator=gen) * 3).to(torch.bfloat16)
    k = (torch.randn((steps, B, Hqk, d), generator=gen) * 3).to(torch.bfloat16)
    v = torch.randn((steps, B, Hv, d), generator=gen).to(torch.bfloat16)
    a = torch.randn((steps, B, Hv), generator=gen)
    beta = torch.sigmoid(torch.randn((steps, B, Hv), generator=gen))
    A_log = torch.log(1 + 15 * torch.rand(Hv, generator=gen))
    dt_bias = -4 + 3 * torch.rand(Hv, generator=gen)
    S0 = torch.randn((B, Hv, d, d), generator=gen) * 0.02
    eps = 1e-6
    nrm = lambda x: x.float() / torch.sqrt((x.float() ** 2).sum(-1, keepdim=True) + eps)
    g = -torch.exp(A_log) * F.softplus(a + dt_bias)
    o_ref, s_ref = orc.gdn_decode_steps(nrm(q), nrm(k), v, g, beta, S0)
    st = S0.to(DEV)
    Ad, dd = A_log.to(DEV), dt_bias.to(DEV)
    for t in range(steps):
        o = pkg.gdn_decode(q[t].to(DEV), k[t].to(DEV), v[t].to(DEV), a[t].to(DEV),
                           beta[t].to(DEV), st, l2norm_qk=True, l2_eps=eps, A_log=Ad, dt_bias=dd)
        np.testing.assert_allclose(o.float().cpu().numpy(), o_ref[t], rtol=O_RTOL, atol=O_ATOL)
    pkg.check_device_status()
    assert np.abs(st.cpu().numpy() - s_ref).max() < S_ATOL
    # KDA with in-kernel L2 normalisation
    x = inputs.make_decode_inputs(4, 2, 2, 2, 128, kda=True, seed=7)
    qr, kr = (x.q.float() * 5).to(torch.bfloat16), (x.k.float() * 0.5).to(torch.bfloat16)
    ko, ks = orc.kda_decode_steps(nrm(qr), nrm(kr), x.v, x.g, x.beta, x.state)
    st = x.state.to(DEV)
    for t in range(4):
        o = pkg.kda_decode(qr[t].to(DEV), kr[t].to(DEV), x.v[t].to(DEV), x.g[t].to(DEV),
                           x.beta[t].to(DEV), st, l2norm_qk=True, l2_eps=eps)
        np.testing.assert_allclose(o.float().cpu().numpy(), ko[t], rtol=O_RTOL, atol=O_ATOL)
    assert np.abs(st.cpu().numpy() - ks).max() < S_ATOL


@pytest.mark.parametrize("B,steps", [(8, 64), (64, 8), (10, 4)])
def test_fp16_state_characterisation(pkg, inputs, orc, B, steps):
    """Characterisation (not a parity test) of the optional fp16 state (half
    the streamed bytes, fp32 arithmetic) against the fp32 recurrence.  Outputs
    meet the BASELINE bf16 tolerance.  The state cannot meet the BASELINE 1e-3
    max-abs gate: at |S| near 1.1 (reached after 64 steps) one fp16 rounding
    alone is up to 4.9e-4, and after 64 steps the error is 1.25e-3 with
    round-to-nearest (stochastic rounding, emulated, is worse: 1.6e-3).  The
    option is therefore off by default; this test pins its measured error
    below 2e-3.  Covers 32-, 64- and 128-column slabs."""
    x = inputs.make_decode_inputs(steps, B, 16, 32, 128, seed=40 + B)
    o_ref, s_ref = orc.gdn_decode_steps(x.q, x.k, x.v, x.g, x.beta, x.state)
    st = x.state.to(DEV, torch.float16)
    for t in range(steps):
        o = pkg.gdn_decode(x.q[t].to(DEV), x.k[t].to(DEV), x.v[t].to(DEV), x.g[t].to(DEV),
                           x.beta[t].to(DEV), st)
        np.testing.assert_allclose(o.float().cpu().numpy(), o_ref[t], rtol=O_RTOL, atol=O_ATOL)
    pkg.check_device_status()
    assert np.abs(st.float().cpu().numpy() - s_ref).max() < 2e-3  # fp16-state bound, see docstring


def test_fused_layer_step_with_output_norm_gate(pkg, orc):
    """The whole layer step in one kernel: raw q/k (L2-normalised in-kernel),
    raw gate projection, and the output gated RMSNorm
    o <- RMSNorm(o) * w * silu(z) (norm before gate), against the oracle plus
    the same post-processing in fp32."""
    import torch.nn.functional as F
    steps, B, Hqk, Hv, d = 4, 4, 2, 4, 128
    gen = torch.Generator().manual_seed(77)
    q = (torch.randn((steps, B, Hqk, d), generator=gen) * 2).to(torch.bfloat16)
    k = (torch.randn((steps, B, Hqk, d), generator=gen) * 2).to(torch.bfloat16)
    v = torch.randn((steps, B, Hv, d), generator=gen).to(torch.bfloat16)
    z = torch.randn((steps, B, Hv, d), generator=gen).to(torch.bfloat16)
    a = torch.randn((steps, B, Hv), generator=gen)
    beta = torch.sigmoid(torch.randn((steps, B, Hv), generator=gen))
    A_log = torch.log(1 + 15 * torch.rand(Hv, generator=gen))
    dt_bias = -4 + 3 * torch.rand(Hv, generator=gen)
    w = 0.5 + torch.rand(d, generator=gen)
    S0 = torch.randn((B, Hv, d, d), generator=gen) * 0.02
    eps = 1e-6
    nrm = lambda x: x.float() / torch.sqrt((x.float() ** 2).sum(-1, keepdim=True) + eps)
    g = -torch.exp(A_log) * F.softplus(a + dt_bias)
    o_ref, s_ref = orc.gdn_decode_steps(nrm(q), nrm(k), v, g, beta, S0)
    o_ref = torch.from_numpy(o_ref)
    rms = torch.rsqrt((o_ref ** 2).mean(-1, keepdim=True) + eps)
    o_ref = (o_ref * rms * w * F.silu(z.float())).numpy()
    st = S0.to(DEV)
    for t in range(steps):
        o = pkg.gdn_decode(q[t].to(DEV), k[t].to(DEV), v[t].to(DEV), a[t].to(DEV),
                           beta[t].to(DEV), st, l2norm_qk=True, l2_eps=eps,
                           A_log=A_log.to(DEV), dt_bias=dt_bias.to(DEV),
                           z=z[t].to(DEV), norm_weight=w.to(DEV), norm_eps=eps)
        np.testing.assert_allclose(o.float().cpu().numpy(), o_ref[t], rtol=O_RTOL, atol=O_ATOL)
    pkg.check_device_status()
    assert np.abs(st.cpu().numpy() - s_ref).max() < S_ATOL
