"""Seeded synthetic inputs with the BASELINE distributions.

BASELINE names no dataset; every config uses these generators (seed 0 unless
stated).  Distributions:

* q, k: N(0, 1), L2-normalised per head (in fp32), then cast to the I/O dtype.
* v: N(0, 1) in the I/O dtype.
* beta = sigmoid(N(0, 1)) per (b, h) [per token].
* GDN log gate g = -exp(A) * softplus(a + dt_bias), A ~ U(0, ln 16),
  dt_bias ~ U(-4, -1) drawn once per (b, h) (they are per-head parameters in a
  model) and a ~ N(0, 1) drawn per token.
* KDA log gate g[b, h, k] = -softplus(N(0, 1)) * exp(U(-5, 0)) per token.
* state: fp32 N(0, 0.02) (std 0.02).

The reference's own generator (pytorch_reference_gdn.py:126-165) draws
pre-scaled q/k and a direct alpha instead; those inputs appear only in the
reference-generated golden fixtures.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F


def _gen(seed: int, device) -> torch.Generator:
    return torch.Generator(device=device).manual_seed(seed)


def _l2norm(x: torch.Tensor) -> torch.Tensor:
    return x / x.norm(dim=-1, keepdim=True).clamp_min(1e-6)


def gdn_gate_params(B: int, Hv: int, gen: torch.Generator, device):
    A = torch.rand((B, Hv), generator=gen, device=device) * math.log(16.0)
    dt_bias = -4.0 + 3.0 * torch.rand((B, Hv), generator=gen, device=device)
    return A, dt_bias


def gdn_log_gate(A, dt_bias, a):
    return -torch.exp(A) * F.softplus(a + dt_bias)


@dataclass
class DecodeInputs:
    q: torch.Tensor      # [steps, B, Hqk, dk]
    k: torch.Tensor
    v: torch.Tensor      # [steps, B, Hv, dv]
    g: torch.Tensor      # [steps, B, Hv] (GDN) or [steps, B, Hv, dk] (KDA), fp32
    beta: torch.Tensor   # [steps, B, Hv] fp32
    state: torch.Tensor  # [B, Hv, dk, dv] fp32


def make_decode_inputs(steps: int, B: int, Hqk: int, Hv: int, d: int = 128, *, kda: bool = False,
                       seed: int = 0, device="cpu", io_dtype=torch.bfloat16,
                       state_std: float = 0.02) -> DecodeInputs:
    """Inputs for ``steps`` decode tokens (configs 0, 1, 2, 4)."""
    gen = _gen(seed, device)
    q = _l2norm(torch.randn((steps, B, Hqk, d), generator=gen, device=device)).to(io_dtype)
    k = _l2norm(torch.randn((steps, B, Hqk, d), generator=gen, device=device)).to(io_dtype)
    v = torch.randn((steps, B, Hv, d), generator=gen, device=device).to(io_dtype)
    beta = torch.sigmoid(torch.randn((steps, B, Hv), generator=gen, device=device))
    if kda:
        n = torch.randn((steps, B, Hv, d), generator=gen, device=device)
        u = -5.0 * torch.rand((steps, B, Hv, d), generator=gen, device=device)
        g = -F.softplus(n) * torch.exp(u)
    else:
        A, dt_bias = gdn_gate_params(B, Hv, gen, device)
        a = torch.randn((steps, B, Hv), generator=gen, device=device)
        g = gdn_log_gate(A, dt_bias, a)
    state = torch.randn((B, Hv, d, d), generator=gen, device=device) * state_std
    return DecodeInputs(q, k, v, g.float(), beta.float(), state)


@dataclass
class PrefillInputs:
    q: torch.Tensor     # [B, T, Hqk, dk]
    k: torch.Tensor
    v: torch.Tensor     # [B, T, Hv, dv]
    g: torch.Tensor     # [B, T, Hv]
    beta: torch.Tensor  # [B, T, Hv]


def make_prefill_inputs(B: int, T: int, Hqk: int, Hv: int, d: int = 128, *, seed: int = 0,
                        device="cpu", io_dtype=torch.bfloat16) -> PrefillInputs:
    """Config 3: bf16 q/k/v/beta/g drawn per token as in config 0."""
    gen = _gen(seed, device)
    q = _l2norm(torch.randn((B, T, Hqk, d), generator=gen, device=device)).to(io_dtype)
    k = _l2norm(torch.randn((B, T, Hqk, d), generator=gen, device=device)).to(io_dtype)
    v = torch.randn((B, T, Hv, d), generator=gen, device=device).to(io_dtype)
    beta = torch.sigmoid(torch.randn((B, T, Hv), generator=gen, device=device)).to(io_dtype)
    A, dt_bias = gdn_gate_params(B, Hv, gen, device)
    a = torch.randn((B, T, Hv), generator=gen, device=device)
    g = gdn_log_gate(A[:, None, :], dt_bias[:, None, :], a).to(io_dtype)
    return PrefillInputs(q, k, v, g, beta)


def make_kda_prefill_inputs(B: int, T: int, Hqk: int, Hv: int, d: int = 128, *, seed: int = 0,
                            device="cpu", io_dtype=torch.bfloat16,
                            g_dtype=torch.float32) -> PrefillInputs:
    """KDA prefill: the config 2 distributions drawn per token, g [B,T,Hv,d]."""
    gen = _gen(seed, device)
    q = _l2norm(torch.randn((B, T, Hqk, d), generator=gen, device=device)).to(io_dtype)
    k = _l2norm(torch.randn((B, T, Hqk, d), generator=gen, device=device)).to(io_dtype)
    v = torch.randn((B, T, Hv, d), generator=gen, device=device).to(io_dtype)
    beta = torch.sigmoid(torch.randn((B, T, Hv), generator=gen, device=device)).to(io_dtype)
    n = torch.randn((B, T, Hv, d), generator=gen, device=device)
    u = -5.0 * torch.rand((B, T, Hv, d), generator=gen, device=device)
    g = (-F.softplus(n) * torch.exp(u)).to(g_dtype)
    return PrefillInputs(q, k, v, g, beta)


def kda_prefill_bytes(B: int, T: int, Hqk: int, Hv: int, d: int = 128, io_bytes: int = 2,
                      g_bytes: int = 4) -> int:
    """Compulsory HBM bytes: q, k, v, g, beta read once, o and the final state
    written once (zero initial state)."""
    tok = B * T
    return tok * (2 * Hqk * d * io_bytes + Hv * d * io_bytes * 2 + Hv * d * g_bytes
                  + Hv * io_bytes) + B * Hv * d * d * 4


def kda_recurrent_ops(B: int, T: int, Hv: int, d: int = 128) -> int:
    """fp32 operations of the recurrent form: per token and head, the decay,
    the two column sums and the rank-1 update, d*d each (FMA counted as 2
    except the decay multiply)."""
    return B * T * Hv * d * d * 7


# Algorithmic bytes / FLOPs (the numerators of every roofline figure).

def gdn_decode_bytes(B: int, Hqk: int, Hv: int, dk: int = 128, dv: int = 128,
                     io_bytes: int = 2, gate_bytes: int = 4) -> int:
    """State read + write, q/k read, v read + o write, g/beta read."""
    return B * (Hv * dk * dv * 4 * 2 + Hqk * dk * io_bytes * 2 + Hv * dv * io_bytes * 2
                + Hv * 2 * gate_bytes)


def kda_decode_bytes(B: int, Hqk: int, Hv: int, dk: int = 128, dv: int = 128,
                     io_bytes: int = 2, gate_bytes: int = 4) -> int:
    return B * (Hv * dk * dv * 4 * 2 + Hqk * dk * io_bytes * 2 + Hv * dk * gate_bytes
                + Hv * dv * io_bytes * 2 + Hv * gate_bytes)


def gdn_prefill_flops(B: int, T: int, Hqk: int, Hv: int, d: int = 128, C: int = 64) -> float:
    """Chunked-form FLOPs: per qk head-chunk KK^T and QK^T (2*2C^2 d); per
    value head-chunk the solve (C^3/3 *2), W, U (2*2C^2 d), (QK^T.M)V' (2C^2 d)
    and W S, Q S, K^T V' (3 * 2 C d^2)."""
    n_qk = B * Hqk * T // C
    n_v = B * Hv * T // C
    return n_qk * (2 * 2 * C * C * d) + n_v * (3 * 2 * C * C * d + 3 * 2 * C * d * d
                                               + (2.0 / 3.0) * C ** 3)
