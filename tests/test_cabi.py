"""The C ABI without a GPU: the library loads, exports every function the
header declares, its struct layouts match the ctypes mirrors, and argument
validation rejects bad calls before touching the device."""
from __future__ import annotations

import ctypes
import re
import subprocess

import pytest

from conftest import ROOT, has_gpu

HEADER = ROOT / "include" / "gdn_b200.h"


def header_functions() -> set[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(\w+)\s*\(", text, flags=re.M))


def test_library_exports_every_declared_function(pkg):
    L = pkg._lib.load()
    declared = header_functions()
    assert declared == set(pkg._lib.EXPORTED)
    for name in declared:
        assert hasattr(L, name), f"{name} not exported"


def test_version_and_status_strings(pkg):
    L = pkg._lib.load()
    assert L.gdn_abi_version() == 1
    assert pkg._lib.status_string(0) == "ok"
    assert "aligned" in pkg._lib.status_string(3)
    assert "unknown" in pkg._lib.status_string(99)


def test_struct_layout_matches_header(pkg, tmp_path):
    """sizeof/offsetof from the C compiler equal the ctypes mirrors."""
    src = tmp_path / "layout.c"
    fields_d = [f for f, _ in pkg._lib.DecodeArgs._fields_]
    fields_p = [f for f, _ in pkg._lib.PrefillArgs._fields_]
    fields_o = [f for f, _ in pkg._lib.PeerOut._fields_]
    body = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void){",
            'printf("%zu\\n", sizeof(gdn_decode_args_t));',
            'printf("%zu\\n", sizeof(gdn_prefill_args_t));',
            'printf("%zu\\n", sizeof(gdn_peer_out_t));']
    body += [f'printf("%zu\\n", offsetof(gdn_decode_args_t, {f}));' for f in fields_d]
    body += [f'printf("%zu\\n", offsetof(gdn_prefill_args_t, {f}));' for f in fields_p]
    body += [f'printf("%zu\\n", offsetof(gdn_peer_out_t, {f}));' for f in fields_o]
    body += ["return 0;}"]
    src.write_text("\n".join(body))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", str(src), "-o", str(exe)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True,
                                           check=True).stdout.split()]
    D, P, O = pkg._lib.DecodeArgs, pkg._lib.PrefillArgs, pkg._lib.PeerOut
    expect = [ctypes.sizeof(D), ctypes.sizeof(P), ctypes.sizeof(O)]
    expect += [getattr(D, f).offset for f in fields_d] + [getattr(P, f).offset for f in fields_p]
    expect += [getattr(O, f).offset for f in fields_o]
    assert vals == expect


def _valid_args(pkg, **over):
    a = pkg._lib.DecodeArgs()
    base = 0x7F0000000000
    for i, name in enumerate(("q", "k", "v", "g", "beta", "state_in", "state_out", "o")):
        setattr(a, name, base + i * (1 << 32))
    B, Hqk, Hv, d = 4, 2, 4, 128
    a.q_sb, a.q_sh, a.k_sb, a.k_sh = Hqk * d, d, Hqk * d, d
    a.v_sb, a.v_sh, a.o_sb, a.o_sh = Hv * d, d, Hv * d, d
    a.g_sb, a.g_sh, a.beta_sb, a.beta_sh = Hv, 1, Hv, 1
    a.B, a.Hqk, a.Hv, a.dk, a.dv = B, Hqk, Hv, d, d
    a.io_dtype, a.g_dtype, a.beta_dtype, a.gate_kind = 1, 0, 0, 0
    a.scale = 1.0
    for k, v in over.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("over,code", [
    ({"q": 0}, 1),
    ({"state_out": 0}, 1),
    ({"Hv": 3}, 2),              # not a multiple of Hqk
    ({"dk": 96}, 2),
    ({"dv": 96}, 2),
    ({"B": 0}, 2),
    ({"io_dtype": 0}, 4),        # fp32 I/O is not a kernel dtype
    ({"g_dtype": 7}, 4),
    ({"gate_kind": 5}, 4),
    ({"q": 0x7F0000000008}, 3),  # 8-byte aligned only
    ({"v_sh": 100}, 3),          # 200-byte head stride
    ({"flags": 8}, 4),           # unknown option bit
    ({"flags": 2}, 1),           # raw gate without A_log / dt_bias
    ({"flags": 1, "l2_eps": -1.0}, 2),
    ({"flags": 4}, 1),           # output norm/gate without z / norm_weight
])
def test_decode_validation_rejects(pkg, over, code):
    L = pkg._lib.load()
    a = _valid_args(pkg, **over)
    assert L.gdn_decode_launch(ctypes.byref(a), None) == code
    assert L.kda_decode_launch(ctypes.byref(a), None) in (code, 3, 4)


def test_overlapping_out_of_place_state_rejected(pkg):
    L = pkg._lib.load()
    a = _valid_args(pkg)
    a.state_out = a.state_in + 4096
    assert L.gdn_decode_launch(ctypes.byref(a), None) == 2


@pytest.mark.skipif(has_gpu(), reason="checks the no-device path")
def test_valid_call_without_gpu_reports_no_device(pkg):
    L = pkg._lib.load()
    a = _valid_args(pkg)
    assert L.gdn_decode_launch(ctypes.byref(a), None) == 6


def test_python_api_refuses_cpu_tensors(pkg):
    import torch
    q = torch.zeros(1, 1, 128, dtype=torch.bfloat16)
    v = torch.zeros(1, 1, 128, dtype=torch.bfloat16)
    g = torch.zeros(1, 1)
    S = torch.zeros(1, 1, 128, 128)
    with pytest.raises(pkg.GDNError):
        pkg.gdn_decode(q, q, v, g, g, S)
    with pytest.raises(pkg.GDNError):
        pkg.gdn_prefill(q[:, None], q[:, None], v[:, None], g[:, None], g[:, None])


def test_missing_library_fails_loudly(pkg, tmp_path):
    with pytest.raises(pkg.GDNError, match="not built"):
        pkg._lib.load(tmp_path / "libgdn_b200.so")
