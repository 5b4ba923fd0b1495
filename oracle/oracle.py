"""CPU oracle for the gated delta-rule path — TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use
this module, as the checker.  The CUDA product path never imports it.

Two restatements of the reference recurrence live here:

* ``gdn_decode_step_np`` / ``kda_decode_step_np`` — numpy, literal operation
  order of the reference functions
  ``gdn_decode_reference``  (analysis/wave15-attention-architecture/reference/
  pytorch_reference_gdn.py:38-91, fp32) and ``naive_recurrent_kda_step``
  (pytorch_reference_kda.py:42-71, float64).
* ``gdn_decode_steps`` / ``kda_decode_steps`` / ``gdn_prefill`` — the same
  arithmetic in C (``gdn_oracle.c``, OpenMP over heads) for multi-step and
  full-size cases.

BASELINE adapters (applied identically to kernel and oracle): value head h
uses q/k head ``h // (Hv // Hqk)`` (torch.repeat_interleave), alpha = exp(g)
for a log gate, scale = 1.0 by default.

Parity is pinned against golden vectors produced by the reference itself
(tests/golden/make_golden.py).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_DIR = Path(__file__).resolve().parent
_LIB_PATH = _DIR / "_build" / "liboracle.so"
_lib = None


def build(force: bool = False) -> Path:
    """Compiles liboracle.so with gcc (make) if it is missing or stale."""
    src = _DIR / "gdn_oracle.c"
    if force or not _LIB_PATH.exists() or src.stat().st_mtime > _LIB_PATH.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_DIR), "-B" if force else "_build/liboracle.so"],
                       check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(_LIB_PATH))
        f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
        f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
        i = ctypes.c_int
        L.oracle_gdn_decode.argtypes = [f32p] * 7 + [i] * 7 + [ctypes.c_float]
        L.oracle_gdn_decode.restype = None
        L.oracle_gdn_prefill.argtypes = [f32p] * 7 + [i] * 6 + [ctypes.c_float]
        L.oracle_gdn_prefill.restype = None
        L.oracle_kda_decode.argtypes = [f32p] * 5 + [f64p, f64p] + [i] * 6 + [ctypes.c_float]
        L.oracle_kda_decode.restype = None
        L.oracle_num_threads.restype = ctypes.c_int
        L.oracle_set_num_threads.argtypes = [i]
        _lib = L
    return _lib


def num_threads() -> int:
    return lib().oracle_num_threads()


def set_num_threads(n: int) -> None:
    lib().oracle_set_num_threads(int(n))


def _f32(x) -> np.ndarray:
    if hasattr(x, "detach"):  # torch tensor
        x = x.detach().float().cpu().numpy()
    return np.ascontiguousarray(x, dtype=np.float32)


# --------------------------------------------------------------------------
# numpy restatements (single step; small shapes)
# --------------------------------------------------------------------------

def gdn_decode_step_np(q, k, v, alpha, beta, S_in):
    """gdn_decode_reference (pytorch_reference_gdn.py:38-91) in numpy fp32.

    q, k (B,H,dk); v (B,H,dv); alpha, beta (B,H); S_in (B,H,dk,dv).
    Returns (o fp32 (B,H,dv), S_out fp32).  The reference returns o as f16;
    callers compare against that with an f16-rounding tolerance.
    """
    qf, kf, vf = _f32(q), _f32(k), _f32(v)
    af, bf = _f32(alpha), _f32(beta)
    S = _f32(S_in)
    S_scaled = af[:, :, None, None] * S                          # (1)
    u = np.einsum("bhk,bhkv->bhv", kf, S_scaled)                 # (2)
    residual = vf - u                                            # (3)
    outer = np.einsum("bhk,bhv->bhkv", kf, residual)             # (4)
    S_out = S_scaled + bf[:, :, None, None] * outer
    o = np.einsum("bhk,bhkv->bhv", qf, S_out)                    # (5)
    return o.astype(np.float32), S_out.astype(np.float32)


def kda_decode_step_np(q, k, v, g, beta, S_in, scale=1.0):
    """naive_recurrent_kda_step (pytorch_reference_kda.py:42-71), float64."""
    q = _f32(q).astype(np.float64) * scale
    k = _f32(k).astype(np.float64)
    v = _f32(v).astype(np.float64)
    g = _f32(g).astype(np.float64)
    beta = _f32(beta).astype(np.float64)
    S = np.asarray(S_in, dtype=np.float64)
    S = S * np.exp(g)[..., None]
    u = (k[..., None] * S).sum(axis=-2)
    residual = v - u
    S = S + (beta[..., None] * k)[..., None] * residual[..., None, :]
    o = np.einsum("bhk,bhkv->bhv", q, S)
    return o, S


# --------------------------------------------------------------------------
# C-backed multi-step drivers
# --------------------------------------------------------------------------

def gdn_decode_steps(q, k, v, g, beta, S0, *, gate="log", scale=1.0):
    """Runs the GDN recurrence over ``steps`` tokens.

    q, k [steps,B,Hqk,dk]; v [steps,B,Hv,dv]; g, beta [steps,B,Hv];
    S0 [B,Hv,dk,dv].  Returns (o [steps,B,Hv,dv] fp32, S_final fp32).
    """
    q, k, v, g, beta = map(_f32, (q, k, v, g, beta))
    S = _f32(S0).copy()
    steps, B, Hqk, dk = q.shape
    Hv, dv = v.shape[2], v.shape[3]
    assert k.shape == q.shape and v.shape[:2] == (steps, B)
    assert g.shape == (steps, B, Hv) and beta.shape == (steps, B, Hv)
    assert S.shape == (B, Hv, dk, dv) and Hv % Hqk == 0
    o = np.zeros((steps, B, Hv, dv), np.float32)
    lib().oracle_gdn_decode(q, k, v, g, beta, S, o, steps, B, Hqk, Hv, dk, dv,
                            1 if gate == "log" else 0, float(scale))
    return o, S


def kda_decode_steps(q, k, v, g, beta, S0, *, scale=1.0):
    """KDA recurrence (float64) over ``steps`` tokens.

    q, k [steps,B,Hqk,dk]; g [steps,B,Hv,dk] (log gate); v [steps,B,Hv,dv];
    beta [steps,B,Hv]; S0 [B,Hv,dk,dv].  Returns (o f64, S_final f64).
    """
    q, k, v, g, beta = map(_f32, (q, k, v, g, beta))
    S = np.ascontiguousarray(np.asarray(S0 if not hasattr(S0, "detach") else S0.detach().cpu().numpy(),
                                        dtype=np.float64)).copy()
    steps, B, Hqk, dk = q.shape
    Hv, dv = v.shape[2], v.shape[3]
    assert g.shape == (steps, B, Hv, dk) and beta.shape == (steps, B, Hv)
    o = np.zeros((steps, B, Hv, dv), np.float64)
    lib().oracle_kda_decode(q, k, v, g, beta, S, o, steps, B, Hqk, Hv, dk, dv, float(scale))
    return o, S


def gdn_prefill(q, k, v, g, beta, S0=None, *, scale=1.0):
    """Sequential-recurrence prefill oracle.

    q, k [B,T,Hqk,dk]; v [B,T,Hv,dv]; g (log gate), beta [B,T,Hv];
    S0 [B,Hv,dk,dv] or None.  Returns (o [B,T,Hv,dv] fp32, S_final fp32).
    """
    q, k, v, g, beta = map(_f32, (q, k, v, g, beta))
    B, T, Hqk, dk = q.shape
    Hv, dv = v.shape[2], v.shape[3]
    S = np.zeros((B, Hv, dk, dv), np.float32) if S0 is None else _f32(S0).copy()
    o = np.zeros((B, T, Hv, dv), np.float32)
    lib().oracle_gdn_prefill(q, k, v, g, beta, S, o, B, T, Hqk, Hv, dk, dv, float(scale))
    return o, S


if __name__ == "__main__":
    print(build(force=True), "threads:", num_threads())


def kda_prefill(q, k, v, g, beta, S0=None, *, scale=1.0):
    """KDA prefill oracle: T applications of the reference KDA step
    (naive_recurrent_kda_step, pytorch_reference_kda.py:42-71) in float64.

    q, k [B,T,Hqk,dk]; v [B,T,Hv,dv]; g [B,T,Hv,dk]; beta [B,T,Hv];
    S0 [B,Hv,dk,dv] or None.  Returns (o [B,T,Hv,dv] f64, S_final f64).
    """
    tm = lambda x: np.ascontiguousarray(np.swapaxes(_f32(x), 0, 1))  # [B,T,..] -> [T,B,..]
    q, k, v, g, beta = map(tm, (q, k, v, g, beta))
    B, Hv, dk, dv = q.shape[1], v.shape[2], q.shape[3], v.shape[3]
    S = np.zeros((B, Hv, dk, dv)) if S0 is None else S0
    o, S = kda_decode_steps(q, k, v, g, beta, S, scale=scale)
    return np.ascontiguousarray(np.swapaxes(o, 0, 1)), S
