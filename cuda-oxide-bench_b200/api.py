"""PyTorch-facing entry points of the gated delta-rule path.

The calls mirror the reference harness functions (``gdn_decode`` /
``kda_decode`` kernels launched by cutile-attn-gdn/main.py:116,268-271 and
cutile-attn-kda/main.py:206-269) in the argument form the BASELINE configs
use: q, k, v, g, beta and an fp32 recurrent state updated in place.  Every
call goes through the C ABI of ``libgdn_b200.so``; there is no Python or CPU
fallback.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import GDNError

_DTYPES = {torch.float32: _lib.DT_F32, torch.bfloat16: _lib.DT_BF16, torch.float16: _lib.DT_F16}
_status_words: dict[int, torch.Tensor] = {}


def _dt(t: torch.Tensor, what: str) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise GDNError(f"{what}: unsupported dtype {t.dtype}", 4) from None


def status_word(device: torch.device | int | None = None) -> torch.Tensor:
    """The per-device int32 word the kernels OR GDN_DEVERR_* bits into."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index or 0))
    w = _status_words.get(dev.index)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=dev)
        _status_words[dev.index] = w
    return w


def check_device_status(device=None) -> None:
    """Synchronises and raises GDNError if any kernel reported a device error."""
    w = status_word(device)
    val = int(w.item())
    if val:
        w.zero_()
        raise GDNError(f"device-side failure: {_lib.describe_device_status(val)}",
                       _lib.ERR_DEVICE_WAIT)


def _require_cuda(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    if dev.type != "cuda":
        raise GDNError("tensors must be CUDA tensors (there is no CPU implementation)", 6)
    for t in ts:
        if t.device != dev:
            raise GDNError(f"all tensors must be on {dev}, got {t.device}", 2)
    return dev


def _same_device(ref: torch.Tensor, **named) -> None:
    """Every named tensor (None = absent) must live on ref's CUDA device: a
    pointer to host memory or to another GPU would reach the kernel as an
    address it cannot (or must not) use."""
    for name, t in named.items():
        if t is not None and t.device != ref.device:
            raise GDNError(f"{name} must be on {ref.device}, got {t.device}", 2)


def _stream_ptr(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _decode_args(q, k, v, g, beta, state, state_out, o, scale, gate, kda,
                 sm_reserve: int = 0, l2norm_qk: bool = False, l2_eps: float = 1e-6,
                 A_log=None, dt_bias=None, z=None, norm_weight=None,
                 norm_eps: float = 1e-6) -> _lib.DecodeArgs:
    if q.dim() != 3 or k.shape != q.shape or v.dim() != 3:
        raise GDNError("q, k must be [B, Hqk, d_k] and v [B, Hv, d_v]", 2)
    B, Hqk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    if v.shape[0] != B:
        raise GDNError("q and v disagree on the batch size", 2)
    if kda:
        if tuple(g.shape) != (B, Hv, dk):
            raise GDNError(f"KDA gate must be [B, Hv, d_k] = {(B, Hv, dk)}, got {tuple(g.shape)}", 2)
        if g.stride(-1) != 1:
            raise GDNError("KDA gate rows must be contiguous", 3)
    elif tuple(g.shape) != (B, Hv):
        raise GDNError(f"GDN gate must be [B, Hv] = {(B, Hv)}, got {tuple(g.shape)}", 2)
    if tuple(beta.shape) != (B, Hv):
        raise GDNError(f"beta must be [B, Hv] = {(B, Hv)}, got {tuple(beta.shape)}", 2)
    for name, t in (("state", state), ("state_out", state_out)):
        if t.dtype not in (torch.float32, torch.float16) or t.dtype != state.dtype \
                or tuple(t.shape) != (B, Hv, dk, dv) or not t.is_contiguous():
            raise GDNError(f"{name} must be a contiguous fp32 (or fp16) [B, Hv, d_k, d_v] = "
                           f"{(B, Hv, dk, dv)} tensor", 2)
    if tuple(o.shape) != (B, Hv, dv) or o.dtype != q.dtype:
        raise GDNError("out must be [B, Hv, d_v] with the dtype of q", 2)
    _same_device(q, state=state, state_out=state_out, out=o)
    for name, t in (("q", q), ("k", k), ("v", v), ("out", o)):
        if t.stride(-1) != 1:
            raise GDNError(f"{name}: the innermost dimension must be contiguous", 3)
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise GDNError("q, k, v must share one dtype (bf16 or f16)", 4)
    a = _lib.DecodeArgs()
    a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    a.g, a.beta = g.data_ptr(), beta.data_ptr()
    a.state_in, a.state_out, a.o = state.data_ptr(), state_out.data_ptr(), o.data_ptr()
    a.q_sb, a.q_sh = q.stride(0), q.stride(1)
    a.k_sb, a.k_sh = k.stride(0), k.stride(1)
    a.v_sb, a.v_sh = v.stride(0), v.stride(1)
    a.o_sb, a.o_sh = o.stride(0), o.stride(1)
    a.g_sb, a.g_sh = g.stride(0), g.stride(1)
    a.beta_sb, a.beta_sh = beta.stride(0), beta.stride(1)
    a.B, a.Hqk, a.Hv, a.dk, a.dv = B, Hqk, Hv, dk, dv
    a.io_dtype = _dt(q, "q")
    a.g_dtype = _dt(g, "g")
    a.beta_dtype = _dt(beta, "beta")
    if gate not in ("log", "linear"):
        raise GDNError("gate must be 'log' (decay = exp(g)) or 'linear' (decay = g)", 4)
    a.gate_kind = _lib.GATE_LOG if gate == "log" else _lib.GATE_LINEAR
    a.scale = float(scale)
    a.status = status_word(q.device).data_ptr()
    a.sm_reserve = int(sm_reserve)
    a.state_dtype = _lib.DT_F16 if state.dtype == torch.float16 else _lib.DT_F32
    a.flags = _lib.DECODE_L2NORM_QK if l2norm_qk else 0
    a.l2_eps = float(l2_eps)
    if (A_log is None) != (dt_bias is None):
        raise GDNError("A_log and dt_bias go together (raw-gate mode)", 1)
    if A_log is not None:
        if kda:
            raise GDNError("the raw-gate formula is the scalar GDN gate; not for KDA", 4)
        for name, t in (("A_log", A_log), ("dt_bias", dt_bias)):
            if t.dtype != torch.float32 or tuple(t.shape) != (Hv,) or not t.is_contiguous() \
                    or t.device != q.device:
                raise GDNError(f"{name} must be a contiguous fp32 [Hv] tensor on {q.device}", 2)
        a.flags |= _lib.DECODE_GATE_RAW
        a.A_log, a.dt_bias = A_log.data_ptr(), dt_bias.data_ptr()
    if (z is None) != (norm_weight is None):
        raise GDNError("z and norm_weight go together (output norm/gate)", 1)
    if z is not None:
        if tuple(z.shape) != (B, Hv, dv) or z.dtype != q.dtype or z.stride(-1) != 1 \
                or z.device != q.device:
            raise GDNError("z must be [B, Hv, d_v] in q's dtype with contiguous rows", 2)
        if norm_weight.dtype != torch.float32 or tuple(norm_weight.shape) != (dv,) \
                or not norm_weight.is_contiguous() or norm_weight.device != q.device:
            raise GDNError("norm_weight must be a contiguous fp32 [d_v] tensor", 2)
        a.flags |= _lib.DECODE_OUT_NORM_GATE
        a.z, a.z_sb, a.z_sh = z.data_ptr(), z.stride(0), z.stride(1)
        a.norm_weight, a.norm_eps = norm_weight.data_ptr(), float(norm_eps)
    return a


class DecodeStep:
    """A decode launch bound to fixed tensors: ``step()`` re-launches it with
    no per-call validation or argument marshalling (the form to capture in a
    CUDA graph or to call in a tight decode loop).  The bound tensors' storage
    must stay alive and in place while the object is used."""

    def __init__(self, q, k, v, g, beta, state, *, out=None, state_out=None, scale=1.0,
                 gate="log", kda=False, sm_reserve=0, l2norm_qk=False, l2_eps=1e-6,
                 A_log=None, dt_bias=None, z=None, norm_weight=None, norm_eps=1e-6,
                 peer_out=None):
        dev = _require_cuda(q, k, v, g, beta, state)
        self.out = out if out is not None else torch.empty(
            (v.shape[0], v.shape[1], v.shape[2]), dtype=q.dtype, device=dev)
        state_out = state if state_out is None else state_out
        self._keep = (q, k, v, g, beta, state, state_out, self.out, A_log, dt_bias, z,
                      norm_weight)
        self._args = _decode_args(q, k, v, g, beta, state, state_out, self.out, scale, gate, kda,
                                  sm_reserve, l2norm_qk, l2_eps, A_log, dt_bias, z, norm_weight,
                                  norm_eps)
        if peer_out is not None:  # a _lib.PeerOut owned by sharded.FusedGather
            self._peer = peer_out
            self._args.peer_out = ctypes.addressof(peer_out)
        self._argp = ctypes.byref(self._args)
        L = _lib.load()
        self._fn = L.kda_decode_launch if kda else L.gdn_decode_launch
        self._dev = dev
        self._what = "kda_decode" if kda else "gdn_decode"

    def __call__(self, stream: int | None = None) -> torch.Tensor:
        rc = self._fn(self._argp, _stream_ptr(self._dev) if stream is None else stream)
        if rc:
            _lib.check(rc, self._what)
        return self.out


def gdn_decode(q, k, v, g, beta, state, *, scale: float = 1.0, out=None, gate: str = "log",
               state_out=None, check: bool = False, sm_reserve: int = 0,
               l2norm_qk: bool = False, l2_eps: float = 1e-6, A_log=None,
               dt_bias=None, z=None, norm_weight=None, norm_eps: float = 1e-6) -> torch.Tensor:
    """One GDN decode step; ``state`` is updated in place (or written to
    ``state_out``).  Returns o [B, Hv, d_v] in q's dtype.

    q, k [B, Hqk, d_k] bf16/f16; v [B, Hv, d_v]; g, beta [B, Hv] (any float
    dtype; ``gate='log'`` means decay = exp(g)); state fp32 [B, Hv, d_k, d_v].
    ``check=True`` synchronises and raises on a device-side failure.
    ``sm_reserve`` leaves that many SMs free for a concurrent kernel (the
    persistent decode otherwise occupies every SM).

    Fused layer preprocessing: ``l2norm_qk=True`` L2-normalises q and k per
    head inside the kernel (x / sqrt(sum x^2 + l2_eps)); with ``A_log`` and
    ``dt_bias`` ([Hv] fp32) ``g`` is the raw gate projection ``a`` and the log
    gate is -exp(A_log) * softplus(a + dt_bias); with ``z`` ([B, Hv, d_v]) and
    ``norm_weight`` ([d_v] fp32) the output becomes
    RMSNorm(o) * norm_weight * silu(z) per head (d_v in {64, 128}).
    """
    dev = _require_cuda(q, k, v, g, beta, state)
    if out is None:
        out = torch.empty((v.shape[0], v.shape[1], v.shape[2]), dtype=q.dtype, device=dev)
    so = state if state_out is None else state_out
    a = _decode_args(q, k, v, g, beta, state, so, out, scale, gate, False, sm_reserve,
                     l2norm_qk, l2_eps, A_log, dt_bias, z, norm_weight, norm_eps)
    _lib.check(_lib.load().gdn_decode_launch(ctypes.byref(a), _stream_ptr(dev)), "gdn_decode")
    if check:
        check_device_status(dev)
    return out


def kda_decode(q, k, v, g, beta, state, *, scale: float = 1.0, out=None, gate: str = "log",
               state_out=None, check: bool = False, l2norm_qk: bool = False,
               l2_eps: float = 1e-6) -> torch.Tensor:
    """One KDA decode step (per-channel gate g [B, Hv, d_k]); otherwise as
    :func:`gdn_decode` (``l2norm_qk`` included; no raw-gate mode)."""
    dev = _require_cuda(q, k, v, g, beta, state)
    if out is None:
        out = torch.empty((v.shape[0], v.shape[1], v.shape[2]), dtype=q.dtype, device=dev)
    so = state if state_out is None else state_out
    a = _decode_args(q, k, v, g, beta, state, so, out, scale, gate, True, 0, l2norm_qk, l2_eps)
    _lib.check(_lib.load().kda_decode_launch(ctypes.byref(a), _stream_ptr(dev)), "kda_decode")
    if check:
        check_device_status(dev)
    return out


def gdn_decode_ref(Q, K, V, Alpha, Beta, S_in, S_out, O, *, batch: int, n_heads: int,
                   d_k: int, d_v: int) -> None:
    """Reference-layout GDN decode: the (Q, K, V, Alpha, Beta, S_in, S_out, O)
    argument list of the reference kernels (cutile-attn-gdn/main.py:116,
    cuda-attn-gdn/attn_gdn.cu:343) with their 2-D layouts — Q,K (B*H, d_k),
    V,O (B*H, d_v), Alpha,Beta (B*H, 1) in f16/bf16 with alpha used directly,
    S_in/S_out (B*H*d_k, d_v) fp32 (may alias)."""
    dev = _require_cuda(Q, K, V, Alpha, Beta, S_in, S_out, O)
    for t in (Q, K, V, Alpha, Beta, S_in, S_out, O):
        if not t.is_contiguous():
            raise GDNError("reference-layout tensors must be contiguous", 3)
    rc = _lib.load().gdn_decode_ref_launch(
        batch, n_heads, d_k, d_v, Q.data_ptr(), K.data_ptr(), V.data_ptr(), Alpha.data_ptr(),
        Beta.data_ptr(), S_in.data_ptr(), S_out.data_ptr(), O.data_ptr(), _dt(Q, "Q"),
        _stream_ptr(dev))
    _lib.check(rc, "gdn_decode_ref")


def kda_decode_ref(Q, K, V, G, Beta, S_in, S_out, O, *, batch: int, n_heads: int,
                   d_k: int, d_v: int) -> None:
    """Reference-layout KDA decode (cutile-attn-kda/main.py:207,
    cuda-attn-kda/attn_kda.cu:327): G (B*H, d_k) log gate, otherwise as
    :func:`gdn_decode_ref`."""
    dev = _require_cuda(Q, K, V, G, Beta, S_in, S_out, O)
    for t in (Q, K, V, G, Beta, S_in, S_out, O):
        if not t.is_contiguous():
            raise GDNError("reference-layout tensors must be contiguous", 3)
    rc = _lib.load().kda_decode_ref_launch(
        batch, n_heads, d_k, d_v, Q.data_ptr(), K.data_ptr(), V.data_ptr(), G.data_ptr(),
        Beta.data_ptr(), S_in.data_ptr(), S_out.data_ptr(), O.data_ptr(), _dt(Q, "Q"),
        _stream_ptr(dev))
    _lib.check(rc, "kda_decode_ref")


def _prefill_args(q, k, v, g, beta, initial_state, final_state, o, chunk, scale, kda=False):
    if q.dim() != 4 or k.shape != q.shape or v.dim() != 4:
        raise GDNError("q, k must be [B, T, Hqk, d_k] and v [B, T, Hv, d_v]", 2)
    B, T, Hqk, dk = q.shape
    Hv, dv = v.shape[2], v.shape[3]
    g_shape = (B, T, Hv, dk) if kda else (B, T, Hv)
    if tuple(v.shape[:2]) != (B, T) or tuple(g.shape) != g_shape or tuple(beta.shape) != (B, T, Hv):
        raise GDNError(f"v [B,T,Hv,d_v], g {'[B,T,Hv,d_k]' if kda else '[B,T,Hv]'} and beta "
                       "[B,T,Hv] must match q [B,T,Hqk,d_k]", 2)
    for name, t in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta), ("out", o)):
        if not t.is_contiguous():
            raise GDNError(f"{name} must be contiguous", 3)
    if k.dtype != q.dtype or v.dtype != q.dtype or o.dtype != q.dtype:
        raise GDNError("q, k, v and out must share one dtype (bf16 or f16)", 4)
    for name, t in (("initial_state", initial_state), ("final_state", final_state)):
        if t is not None and (t.dtype != torch.float32 or tuple(t.shape) != (B, Hv, dk, dv)
                              or not t.is_contiguous()):
            raise GDNError(f"{name} must be a contiguous fp32 [B, Hv, d_k, d_v] tensor", 2)
    _same_device(q, initial_state=initial_state, final_state=final_state, out=o)
    a = _lib.PrefillArgs()
    a.q, a.k, a.v, a.g, a.beta = q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr()
    a.initial_state = initial_state.data_ptr() if initial_state is not None else None
    a.final_state = final_state.data_ptr()
    a.o = o.data_ptr()
    a.B, a.T, a.Hqk, a.Hv, a.dk, a.dv, a.chunk = B, T, Hqk, Hv, dk, dv, chunk
    a.io_dtype, a.g_dtype, a.beta_dtype = _dt(q, "q"), _dt(g, "g"), _dt(beta, "beta")
    a.scale = float(scale)
    a.status = status_word(q.device).data_ptr()
    return a


_workspaces: dict[int, torch.Tensor] = {}


def _workspace(dev, need: int, given):
    """The caller's workspace tensor, or a per-device cached one of at least
    ``need`` bytes (grown when a larger problem comes).  The cached one is
    shared by every gdn_prefill / kda_prefill call on the device, so calls
    whose kernels may overlap on the GPU (different streams or threads) must
    each pass their own ``workspace``."""
    if given is not None:
        if given.device != dev or not given.is_contiguous():
            raise GDNError(f"workspace must be a contiguous tensor on {dev}", 2)
        if given.numel() * given.element_size() < need:
            raise GDNError(f"workspace holds {given.numel() * given.element_size()} bytes; "
                           f"these shapes need {need}", 7)
        return given
    ws = _workspaces.get(dev.index)
    if ws is None or ws.numel() < need:
        _workspaces.pop(dev.index, None)
        ws = torch.empty(need, dtype=torch.uint8, device=dev)
        _workspaces[dev.index] = ws
    return ws


def gdn_prefill(q, k, v, g, beta, initial_state=None, *, chunk_size: int = 64,
                scale: float = 1.0, out=None, final_state=None, workspace=None,
                check: bool = False):
    """GDN chunked prefill over T tokens.  Returns (o [B,T,Hv,d_v], final_state
    fp32 [B,Hv,d_k,d_v]).  Equivalent to T decode steps (log gate g)."""
    dev = _require_cuda(q, k, v, g, beta)
    B, T, _, dk = q.shape
    Hv, dv = v.shape[2], v.shape[3]
    if out is None:
        out = torch.empty((B, T, Hv, dv), dtype=q.dtype, device=dev)
    if final_state is None:
        final_state = torch.empty((B, Hv, dk, dv), dtype=torch.float32, device=dev)
    a = _prefill_args(q, k, v, g, beta, initial_state, final_state, out, chunk_size, scale)
    L = _lib.load()
    need = L.gdn_prefill_workspace_size(ctypes.byref(a))
    if need:
        workspace = _workspace(dev, need, workspace)
        a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    _lib.check(L.gdn_prefill_launch(ctypes.byref(a), _stream_ptr(dev)), "gdn_prefill")
    if check:
        check_device_status(dev)
    return out, final_state


def kda_prefill(q, k, v, g, beta, initial_state=None, *, scale: float = 1.0, out=None,
                final_state=None, form: str = "auto", workspace=None, check: bool = False):
    """KDA prefill over T tokens: T applications of the reference's
    naive_recurrent_kda_step (pytorch_reference_kda.py:42-71) with the state
    threaded through.  q, k [B,T,Hqk,d_k]; v [B,T,Hv,d_v]; g [B,T,Hv,d_k]
    per-channel log gate; beta [B,T,Hv].  Returns (o [B,T,Hv,d_v],
    final_state fp32 [B,Hv,d_k,d_v]).  ``final_state`` may be the
    ``initial_state`` tensor (updated in place).

    ``form``: "chunked" (tensor cores, 64-token chunks; d_k = d_v = 128 only),
    "recurrent" (state on chip, CUDA cores; d in {64, 128, 256}) or "auto"
    (chunked where it exists).  The chunked form uses a device workspace
    (cached per device unless ``workspace`` is given)."""
    if form not in ("auto", "chunked", "recurrent"):
        raise GDNError(f"form must be 'auto', 'chunked' or 'recurrent', not {form!r}", 2)
    dev = _require_cuda(q, k, v, g, beta)
    B, T, _, dk = q.shape
    Hv, dv = v.shape[2], v.shape[3]
    if out is None:
        out = torch.empty((B, T, Hv, dv), dtype=q.dtype, device=dev)
    if final_state is None:
        final_state = torch.empty((B, Hv, dk, dv), dtype=torch.float32, device=dev)
    a = _prefill_args(q, k, v, g, beta, initial_state, final_state, out, 0, scale, kda=True)
    L = _lib.load()
    if form != "recurrent":
        need = L.kda_prefill_workspace_size(ctypes.byref(a))
        if not need and form == "chunked":
            raise GDNError("the chunked KDA prefill needs d_k = d_v = 128", 2)
        if need:
            workspace = _workspace(dev, need, workspace)
            a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    _lib.check(L.kda_prefill_launch(ctypes.byref(a), _stream_ptr(dev)), "kda_prefill")
    if check:
        check_device_status(dev)
    return out, final_state
