"""ctypes binding of ``libgdn_b200.so`` (the C ABI declared in include/gdn_b200.h).

The library is loaded lazily on first use.  If it is missing or cannot be
loaded, every entry point raises :class:`GDNError` — there is no fallback
implementation.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

_PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = _PKG_DIR / "libgdn_b200.so"

# enums mirrored from include/gdn_b200.h
DT_F32, DT_BF16, DT_F16 = 0, 1, 2
GATE_LOG, GATE_LINEAR = 0, 1
DECODE_L2NORM_QK, DECODE_GATE_RAW, DECODE_OUT_NORM_GATE = 1, 2, 4
OK = 0
ERR_DEVICE_WAIT = 8

DEVERR_BITS = {
    1 << 0: "consumer timed out waiting for a staged slab",
    1 << 1: "producer timed out waiting for a free ring slot",
    1 << 2: "tensor-core completion was never signalled",
    1 << 3: "copies in flight never landed while aborting",
    1 << 4: "a peer rank never released a gathered-output slot",
}

# Every function the header declares (checked by the CPU test suite).
EXPORTED = (
    "gdn_abi_version",
    "gdn_status_string",
    "gdn_decode_launch",
    "kda_decode_launch",
    "gdn_decode_ref_launch",
    "kda_decode_ref_launch",
    "gdn_prefill_workspace_size",
    "gdn_prefill_launch",
    "gdn_prefill_launch_noalloc",
    "kda_prefill_launch",
    "kda_prefill_workspace_size",
    "gdn_ipc_handle",
    "gdn_ipc_open",
    "gdn_ipc_close",
    "gdn_gather_push",
    "gdn_gather_wait",
    "gdn_gather_wait_counter",
    "gdn_state_affine",
)
IPC_HANDLE_BYTES = 64


class GDNError(RuntimeError):
    """A gdn_b200 call failed; ``code`` is the GDN_ERR_* value (or -1)."""

    def __init__(self, msg: str, code: int = -1):
        super().__init__(msg)
        self.code = code


class PeerOut(ctypes.Structure):
    _fields_ = [
        ("o_peer", ctypes.c_void_p * 7),
        ("arrive", ctypes.c_void_p * 8),
        ("free_flags", ctypes.c_void_p * 8),
        ("cta_done", ctypes.c_void_p),
        ("n_ranks", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("step", ctypes.c_uint32),
        ("reserved", ctypes.c_int32),
    ]


class DecodeArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("g", ctypes.c_void_p), ("beta", ctypes.c_void_p),
        ("state_in", ctypes.c_void_p), ("state_out", ctypes.c_void_p), ("o", ctypes.c_void_p),
        ("q_sb", ctypes.c_int64), ("q_sh", ctypes.c_int64),
        ("k_sb", ctypes.c_int64), ("k_sh", ctypes.c_int64),
        ("v_sb", ctypes.c_int64), ("v_sh", ctypes.c_int64),
        ("o_sb", ctypes.c_int64), ("o_sh", ctypes.c_int64),
        ("g_sb", ctypes.c_int64), ("g_sh", ctypes.c_int64),
        ("beta_sb", ctypes.c_int64), ("beta_sh", ctypes.c_int64),
        ("B", ctypes.c_int32), ("Hqk", ctypes.c_int32), ("Hv", ctypes.c_int32),
        ("dk", ctypes.c_int32), ("dv", ctypes.c_int32),
        ("io_dtype", ctypes.c_int32), ("g_dtype", ctypes.c_int32),
        ("beta_dtype", ctypes.c_int32), ("gate_kind", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("status", ctypes.c_void_p),
        ("sm_reserve", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("l2_eps", ctypes.c_float),
        ("A_log", ctypes.c_void_p),
        ("dt_bias", ctypes.c_void_p),
        ("state_dtype", ctypes.c_int32),
        ("z", ctypes.c_void_p),
        ("z_sb", ctypes.c_int64), ("z_sh", ctypes.c_int64),
        ("norm_weight", ctypes.c_void_p),
        ("norm_eps", ctypes.c_float),
        ("peer_out", ctypes.c_void_p),
    ]


class PrefillArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("g", ctypes.c_void_p), ("beta", ctypes.c_void_p),
        ("initial_state", ctypes.c_void_p), ("final_state", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("B", ctypes.c_int32), ("T", ctypes.c_int32), ("Hqk", ctypes.c_int32),
        ("Hv", ctypes.c_int32), ("dk", ctypes.c_int32), ("dv", ctypes.c_int32),
        ("chunk", ctypes.c_int32),
        ("io_dtype", ctypes.c_int32), ("g_dtype", ctypes.c_int32), ("beta_dtype", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
        ("status", ctypes.c_void_p),
    ]


_lock = threading.Lock()
_lib = None


def load(path: str | Path | None = None):
    """Loads (once) and returns the library handle.  Raises GDNError if absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise GDNError(
                f"{p.name} is not built ({p}); run __graft_entry__.build() or "
                "python cuda-oxide-bench_b200/build.py — there is no CPU fallback")
        try:
            L = ctypes.CDLL(str(p))
        except OSError as e:
            raise GDNError(f"cannot load {p}: {e}") from e
        vp, i32 = ctypes.c_void_p, ctypes.c_int32
        L.gdn_abi_version.restype = ctypes.c_int
        L.gdn_status_string.restype = ctypes.c_char_p
        L.gdn_status_string.argtypes = [ctypes.c_int]
        for fn in (L.gdn_decode_launch, L.kda_decode_launch):
            fn.argtypes = [ctypes.POINTER(DecodeArgs), vp]
            fn.restype = ctypes.c_int
        for fn in (L.gdn_decode_ref_launch, L.kda_decode_ref_launch):
            fn.argtypes = [i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, i32, vp]
            fn.restype = ctypes.c_int
        L.gdn_prefill_workspace_size.argtypes = [ctypes.POINTER(PrefillArgs)]
        L.gdn_prefill_workspace_size.restype = ctypes.c_size_t
        L.gdn_prefill_launch.argtypes = [ctypes.POINTER(PrefillArgs), vp]
        L.gdn_prefill_launch.restype = ctypes.c_int
        L.gdn_prefill_launch_noalloc.argtypes = [ctypes.POINTER(PrefillArgs), vp]
        L.gdn_prefill_launch_noalloc.restype = ctypes.c_int
        L.kda_prefill_launch.argtypes = [ctypes.POINTER(PrefillArgs), vp]
        L.kda_prefill_launch.restype = ctypes.c_int
        L.kda_prefill_workspace_size.argtypes = [ctypes.POINTER(PrefillArgs)]
        L.kda_prefill_workspace_size.restype = ctypes.c_size_t
        L.gdn_ipc_handle.argtypes = [vp, vp, ctypes.POINTER(ctypes.c_uint64)]
        L.gdn_ipc_open.argtypes = [vp, ctypes.c_uint64, ctypes.POINTER(vp), ctypes.POINTER(vp)]
        L.gdn_ipc_close.argtypes = [vp]
        L.gdn_gather_push.argtypes = [vp, ctypes.c_size_t, ctypes.POINTER(vp), ctypes.POINTER(vp),
                                      i32, ctypes.c_uint32, vp]
        L.gdn_gather_wait.argtypes = [vp, i32, ctypes.c_uint32, vp]
        L.gdn_gather_wait_counter.argtypes = [vp, ctypes.c_uint32, vp, vp]
        L.gdn_gather_wait_counter.restype = ctypes.c_int
        L.gdn_state_affine.argtypes = [vp, vp, vp, vp, i32, i32, vp]
        L.gdn_state_affine.restype = ctypes.c_int
        for fn in (L.gdn_ipc_handle, L.gdn_ipc_open, L.gdn_ipc_close, L.gdn_gather_push,
                   L.gdn_gather_wait):
            fn.restype = ctypes.c_int
        if path is None:
            _lib = L
        return L


def status_string(code: int) -> str:
    return load().gdn_status_string(int(code)).decode()


def check(code: int, what: str) -> None:
    if code != OK:
        raise GDNError(f"{what}: {status_string(code)} (code {code})", code)


def describe_device_status(word: int) -> str:
    parts = [txt for bit, txt in DEVERR_BITS.items() if word & bit]
    return "; ".join(parts) if parts else f"status word 0x{word:x}"
