"""Host-side argument validation of the Python entry points (no GPU needed):
a tensor on the wrong device must raise GDNError before any pointer reaches
the library."""
from __future__ import annotations

import pytest
import torch


def _api():
    import __graft_entry__ as graft
    return graft.submodule("api")


def _prefill(B=1, T=8, H=1, d=128, dev="cpu"):
    q = torch.zeros((B, T, H, d), dtype=torch.bfloat16, device=dev)
    g = torch.zeros((B, T, H), dtype=torch.float32, device=dev)
    return q, q.clone(), q.clone(), g, g.clone()


@pytest.mark.parametrize("which", ["initial_state", "final_state", "out"])
def test_prefill_rejects_state_or_out_on_another_device(pkg, which):
    api = _api()
    q, k, v, g, beta = _prefill()
    S = torch.zeros((1, 1, 128, 128), dtype=torch.float32)
    o = torch.zeros_like(v)
    args = {"initial_state": S, "final_state": S.clone(), "out": o}
    args[which] = torch.empty(args[which].shape, dtype=args[which].dtype, device="meta")
    with pytest.raises(pkg.GDNError, match=which):
        api._prefill_args(q, k, v, g, beta, args["initial_state"], args["final_state"],
                          args["out"], 64, 1.0)


@pytest.mark.parametrize("which", ["state_out", "out"])
def test_decode_rejects_state_out_or_out_on_another_device(pkg, which):
    api = _api()
    B, H, d = 2, 2, 128
    q = torch.zeros((B, H, d), dtype=torch.bfloat16)
    g = torch.zeros((B, H), dtype=torch.float32)
    S = torch.zeros((B, H, d, d), dtype=torch.float32)
    args = {"state_out": S.clone(), "out": torch.zeros_like(q)}
    args[which] = torch.empty(args[which].shape, dtype=args[which].dtype, device="meta")
    with pytest.raises(pkg.GDNError, match=which):
        api._decode_args(q, q.clone(), q.clone(), g, g.clone(), S, args["state_out"],
                         args["out"], 1.0, "log", False)


def test_cpu_inputs_are_rejected(pkg):
    q, k, v, g, beta = _prefill()
    with pytest.raises(pkg.GDNError):
        pkg.gdn_prefill(q, k, v, g, beta)
    with pytest.raises(pkg.GDNError):
        pkg.gdn_decode(q[:, 0], k[:, 0], v[:, 0], g[:, 0], beta[:, 0],
                       torch.zeros((1, 1, 128, 128)))
