"""Generates the golden fixtures in this directory by running the REFERENCE's
own oracle functions (imported from a checkout of baladithyab/cuda-oxide-bench).

Run once in a container that has the reference checkout:

    python tests/golden/make_golden.py [path/to/reference]

The fixtures are committed; nothing at test time reads the reference.

Files written (all numpy .npz):

* ref_gdn_correctness.npz — the reference's own inputs
  (pytorch_reference_gdn.make_inputs(SHAPE_CORRECTNESS, seed=0xC0FFEE),
  pytorch_reference_gdn.py:126-165; f16) and the outputs of its fused
  ``gdn_decode_reference`` (:38-91) and ``gdn_decode_reference_canonical``
  (:94-123).
* ref_kda_correctness.npz — pytorch_reference_kda.make_inputs(SHAPE_CORRECTNESS,
  seed=17) (pytorch_reference_kda.py:74-…), which includes the f64 oracle
  outputs of ``naive_recurrent_kda_step`` (:42-71).
* baseline_gdn_decode.npz — BASELINE config-0 distributions at a reduced size
  (B=1, Hqk=2, Hv=4, d=128, 64 steps, seed 0) run through the reference's
  ``gdn_decode_reference`` step by step with the BASELINE adapter
  (alpha = exp(g), q/k repeat_interleave over the GQA group).
* baseline_kda_decode.npz — BASELINE config-2 distributions (B=1, H=2, d=128,
  16 steps, seed 0) through ``naive_recurrent_kda_step`` step by step.
* baseline_gdn_prefill.npz — BASELINE config-3 distributions (B=1, T=128,
  Hqk=1, Hv=2, d=128, bf16 inputs, seed 0, zero initial state) through
  ``gdn_decode_reference`` token by token (the sequential recurrence that
  defines prefill).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


def _ref_modules(ref_root: Path):
    sys.path.insert(0, str(ref_root / "analysis" / "wave15-attention-architecture" / "reference"))
    import pytorch_reference_gdn as rg  # noqa: E402
    import pytorch_reference_kda as rk  # noqa: E402
    import shapes_gdn as sg  # noqa: E402
    return rg, rk, sg


def _inputs_module():
    sys.path.insert(0, str(ROOT))
    import __graft_entry__ as ge
    return ge.submodule("inputs")


def f32(t) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def main(ref_root: Path) -> None:
    rg, rk, sg = _ref_modules(ref_root)
    inputs = _inputs_module()
    torch.set_num_threads(8)

    # 1) reference inputs + reference outputs (GDN correctness shape)
    inp = rg.make_inputs(sg.SHAPE_CORRECTNESS, seed=0xC0FFEE)
    with torch.no_grad():
        o_f, S_f = rg.gdn_decode_reference(inp["q_f16"], inp["k_f16"], inp["v_f16"],
                                           inp["alpha_f16"], inp["beta_f16"], inp["S_in_f32"])
        o_c, S_c = rg.gdn_decode_reference_canonical(inp["q_f16"], inp["k_f16"], inp["v_f16"],
                                                     inp["alpha_f16"], inp["beta_f16"],
                                                     inp["S_in_f32"])
    np.savez_compressed(
        HERE / "ref_gdn_correctness.npz",
        q_f16=inp["q_f16"].numpy(), k_f16=inp["k_f16"].numpy(), v_f16=inp["v_f16"].numpy(),
        alpha_f16=inp["alpha_f16"].numpy(), beta_f16=inp["beta_f16"].numpy(),
        S_in=inp["S_in_f32"].numpy(), o_expected_f16=o_f.numpy(), S_out_expected=S_f.numpy(),
        o_canonical_f16=o_c.numpy(), S_out_canonical=S_c.numpy())

    # 2) reference KDA inputs + f64 oracle outputs
    kin = rk.make_inputs(rk.SHAPE_CORRECTNESS, seed=17)
    np.savez_compressed(HERE / "ref_kda_correctness.npz",
                        **{k: kin[k] for k in ("q_f16", "k_f16", "v_f16", "g_f16", "beta_f16",
                                               "S_in_f32", "o_expected_f16",
                                               "S_out_expected_f32")})

    # 3) BASELINE config-0 distributions, 64 steps, through the reference step
    steps, B, Hqk, Hv, d = 64, 1, 2, 4, 128
    x = inputs.make_decode_inputs(steps, B, Hqk, Hv, d, seed=0)
    grp = Hv // Hqk
    S = x.state.clone()
    o_all = []
    with torch.no_grad():
        for t in range(steps):
            qe = x.q[t].repeat_interleave(grp, dim=1)
            ke = x.k[t].repeat_interleave(grp, dim=1)
            o16, S = rg.gdn_decode_reference(qe, ke, x.v[t], torch.exp(x.g[t]), x.beta[t], S)
            # the reference returns o as f16; keep the fp32 value of the same
            # contraction (o = S_out^T q, step (5)) for a tighter comparison
            o_all.append(torch.einsum("bhk,bhkv->bhv", qe.float(), S))
    np.savez_compressed(HERE / "baseline_gdn_decode.npz",
                        q=f32(x.q), k=f32(x.k), v=f32(x.v), g=f32(x.g), beta=f32(x.beta),
                        S0=f32(x.state), o=f32(torch.stack(o_all)), S_final=f32(S))

    # 4) BASELINE config-2 (KDA) distributions, 16 steps
    steps, B, H = 16, 1, 2
    y = inputs.make_decode_inputs(steps, B, H, H, d, kda=True, seed=0)
    Sk = f32(y.state).astype(np.float64)
    ok = []
    for t in range(steps):
        o64, Sk = rk.naive_recurrent_kda_step(f32(y.q[t]), f32(y.k[t]), f32(y.v[t]), f32(y.g[t]),
                                              f32(y.beta[t]), Sk, scale=1.0)
        ok.append(o64)
    np.savez_compressed(HERE / "baseline_kda_decode.npz",
                        q=f32(y.q), k=f32(y.k), v=f32(y.v), g=f32(y.g), beta=f32(y.beta),
                        S0=f32(y.state), o=np.stack(ok), S_final=Sk)

    # 5) BASELINE config-3 distributions: sequential-recurrence prefill
    B, T, Hqk, Hv = 1, 128, 1, 2
    p = inputs.make_prefill_inputs(B, T, Hqk, Hv, d, seed=0)
    grp = Hv // Hqk
    S = torch.zeros((B, Hv, d, d))
    o_all = []
    with torch.no_grad():
        for t in range(T):
            qe = p.q[:, t].repeat_interleave(grp, dim=1)
            ke = p.k[:, t].repeat_interleave(grp, dim=1)
            _, S = rg.gdn_decode_reference(qe, ke, p.v[:, t], torch.exp(p.g[:, t].float()),
                                           p.beta[:, t], S)
            o_all.append(torch.einsum("bhk,bhkv->bhv", qe.float(), S))
    np.savez_compressed(HERE / "baseline_gdn_prefill.npz",
                        q=f32(p.q), k=f32(p.k), v=f32(p.v), g=f32(p.g), beta=f32(p.beta),
                        o=f32(torch.stack(o_all, dim=1)), S_final=f32(S))
    for f in sorted(HERE.glob("*.npz")):
        print(f"{f.name}: {f.stat().st_size / 1024:.0f} KiB")


if __name__ == "__main__":
    import os
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GDN_REFERENCE_ROOT")
    if not ref:
        sys.exit("usage: make_golden.py <reference checkout> (or set GDN_REFERENCE_ROOT)")
    main(Path(ref))
