"""C ABI checks that need no GPU.

* libhofa_b200.so loads and exports every function include/hofa.h declares;
* the ctypes mirror of every argument struct has the C compiler's size and
  field offsets (a small C program built with gcc against include/hofa.h);
* host-side validation rejects bad arguments with the documented status and
  never reaches a launch (the rejected calls carry fake device pointers).
"""
import os
import re
import subprocess

import pytest

from conftest import ROOT
from outlierneuronattention_b200 import _capi

HEADER = os.path.join(ROOT, "include", "hofa.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s+(hofa_[a-z_0-9]+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    names = declared_functions()
    assert "hofa_decode_fwd" in names and "hofa_prefill_gla_fwd" in names and len(names) >= 9
    L = _capi.lib()
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/hofa.h but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", _capi.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (hofa_[a-z_0-9]+)$", out, flags=re.M))
    assert set(names) <= exported


STRUCTS = {
    "hofa_tensor": (_capi.HofaTensor, ["data", "dtype", "ndim", "shape", "stride"]),
    "hofa_decode_args": (_capi.DecodeArgs, [f for f, _ in _capi.DecodeArgs._fields_]),
    "hofa_gla_args": (_capi.GlaArgs, [f for f, _ in _capi.GlaArgs._fields_]),
    "hofa_outlier_args": (_capi.OutlierArgs, [f for f, _ in _capi.OutlierArgs._fields_]),
    "hofa_prep_args": (_capi.PrepArgs, [f for f, _ in _capi.PrepArgs._fields_]),
    "hofa_linear_args": (_capi.LinearArgs, [f for f, _ in _capi.LinearArgs._fields_]),
}


def test_struct_layout_matches_c(tmp_path):
    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void){"]
    for cname, (_, fields) in STRUCTS.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for f in fields:
            lines.append(f'printf("{cname} {f} %zu\\n", offsetof({cname}, {f}));')
    lines.append("return 0;}")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-o", str(exe), str(src)], check=True)
    got = {}
    for line in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.splitlines():
        s, f, v = line.split()
        got[(s, f)] = int(v)
    for cname, (cls, fields) in STRUCTS.items():
        import ctypes
        assert got[(cname, "size")] == ctypes.sizeof(cls), cname
        for f in fields:
            assert got[(cname, f)] == getattr(cls, f).offset, (cname, f)
        assert _capi.FORMATS.get(cls, None) is None or _capi.FORMATS[cls].size == ctypes.sizeof(cls)


FAKE = 0x10000  # never dereferenced: every call below fails validation first


def tv(shape, dtype=1, stride=None, ptr=FAKE):
    nd = len(shape)
    if stride is None:
        stride, acc = [], 1
        for s in reversed(shape):
            stride.insert(0, acc)
            acc *= s
    return (ptr, dtype, nd) + tuple(shape) + (1,) * (4 - nd) + tuple(stride) + (0,) * (4 - nd)


def decode_vals(B=1, H=2, D=64, R=16, L=32, seq_len=8, **over):
    J = D - R
    t = dict(q=tv([B, H, 1, D]), k=tv([B, H, 1, D]), v=tv([B, H, 1, D]),
             cache_k=tv([B, H, L, R]), cache_v=tv([B, H, L, D]),
             state_in=tv([B, H, J, D], 0, ptr=FAKE), state_out=tv([B, H, J, D], 0, ptr=2 * FAKE),
             log_gamma=tv([B, H, 1], 0), mix_g=tv([B, H, 1]), norm_w=tv([H, D], 0),
             log_alpha=_capi.ABSENT, y=tv([B, H, 1, D]))
    t.update({k: v for k, v in over.items() if k in t})
    sc = dict(R=R, seq_len=seq_len, seq_len_dev=0, sm_scale=2.0, eps=1e-7, split_k=0,
              workspace=FAKE, workspace_bytes=1 << 30)
    sc.update({k: v for k, v in over.items() if k in sc})
    return _capi.flat(*[t[n] for n in ("q", "k", "v", "cache_k", "cache_v", "state_in", "state_out", "log_gamma",
                                       "mix_g", "norm_w", "log_alpha", "y")],
                      *[sc[n] for n in ("R", "seq_len", "seq_len_dev", "sm_scale", "eps", "split_k", "workspace",
                                        "workspace_bytes")])


def expect(status, fn, cls, vals, pattern):
    with pytest.raises(_capi.HofaError) as e:
        _capi.call(fn, cls, vals, 0)
    assert e.value.status == status, str(e.value)
    assert re.search(pattern, str(e.value)), str(e.value)


def test_decode_validation():
    D = _capi.DecodeArgs
    expect(1, "hofa_decode_fwd", D, decode_vals(seq_len=0), "seq_len=0")
    expect(1, "hofa_decode_fwd", D, decode_vals(seq_len=33), "seq_len=33")
    expect(1, "hofa_decode_fwd", D, decode_vals(R=65), "R=65")
    expect(2, "hofa_decode_fwd", D, decode_vals(D=96, R=16), "head dim 96")
    expect(1, "hofa_decode_fwd", D, decode_vals(state_in=tv([1, 2, 48, 64], 1)), "float32")
    expect(1, "hofa_decode_fwd", D, decode_vals(state_out=tv([1, 2, 48, 64], 0, ptr=FAKE)), "alias")
    expect(1, "hofa_decode_fwd", D, decode_vals(y=tv([1, 2, 1, 64], 0)), "share one dtype")
    expect(1, "hofa_decode_fwd", D, decode_vals(mix_g=tv([1, 3, 1])), "mix_g")
    expect(4, "hofa_decode_fwd", D, decode_vals(workspace_bytes=16), "workspace needs")
    expect(3, "hofa_decode_fwd", D, decode_vals(state_in=tv([1, 2, 48, 64], 0, ptr=FAKE + 4)), "16-byte")
    expect(1, "hofa_decode_fwd", D, decode_vals(split_k=65), "split_k=65")


def test_prefill_validation():
    B, H, T, D, R = 1, 2, 16, 64, 16
    g = _capi.flat(tv([B, H, T, D]), tv([B, H, T, D]), tv([B, H, T, D]), tv([B, H, T], 0), _capi.ABSENT,
                   _capi.ABSENT, _capi.ABSENT, _capi.ABSENT, tv([B, H, T, D + 1]), _capi.ABSENT,
                   R, 64, 1e-5, 0, 0, 0)
    expect(1, "hofa_prefill_gla_fwd", _capi.GlaArgs, g, "y: dim 3")
    o = _capi.flat(tv([B, H, T, D]), tv([B, H, T, D]), tv([B, H, T, D]), tv([B, H, T]), tv([B, H, T, D]),
                   R, -1, 2.0, 1)
    expect(1, "hofa_prefill_outlier_fwd", _capi.OutlierArgs, o, "q_offset")
    o = _capi.flat(tv([B, H, T, D]), tv([B, H, T, D]), tv([B, H, T, D]), tv([B, H, T]), tv([B, H, T, D]),
                   0, 0, 2.0, 1)
    expect(1, "hofa_prefill_outlier_fwd", _capi.OutlierArgs, o, "R=0")


def test_choose_split_and_workspace_size():
    L = _capi.lib()
    assert L.hofa_decode_choose_split(4, 16, 4096, 148) == 4     # 256 CTAs, clusters of 4
    assert L.hofa_decode_choose_split(1, 16, 4096, 148) == 8     # clusters capped at 8
    assert L.hofa_decode_choose_split(2, 16, 4096, 148) == 6     # 8-CTA clusters would need 256 CTAs
    assert L.hofa_decode_choose_split(1, 16, 65536, 148) == 18   # workspace combine above 16
    assert L.hofa_decode_choose_split(64, 16, 16384, 148) == 1
    assert L.hofa_decode_choose_split(1, 1, 10, 148) == 1
    # workspace: status + tickets + (4 + 2D) floats per (b,h,split)
    assert L.hofa_decode_workspace_size(1, 1, 64, 1) == 256 + 256 + (4 + 128) * 4


def test_decode_step_validation():
    """hofa_decode_step_fwd refuses mismatched tensors before any device work."""
    B, H, D, R, L = 1, 2, 64, 16, 32
    dvals = decode_vals(B=B, H=H, D=D, R=R, L=L)

    def prep_vals(q_ptr=FAKE, mix_out=True, cache_k=True):
        return _capi.flat(tv([B, H, 1, D], ptr=q_ptr), tv([B, H, 1, D]), tv([B, H, 1, D]), tv([H, 2 * D], 0),
                          tv([H], 0), tv([H, 2 * D], 0), tv([H], 0), _capi.ABSENT, tv([4096, R], 0), tv([4096, R], 0),
                          tv([B, H, 1], 0), tv([B, H, 1]) if mix_out else _capi.ABSENT,
                          tv([B, H, L, R]) if cache_k else _capi.ABSENT, tv([B, H, L, D]), R, 0, 0, 1)

    fn = _capi.lib().hofa_decode_step_fwd
    cases = [(prep_vals(q_ptr=3 * FAKE), "same q, k, v"), (prep_vals(mix_out=False), "mix_out is required"),
             (prep_vals(cache_k=False), "append to the decode's caches")]
    for pv, pattern in cases:
        st = fn(_capi.FORMATS[_capi.DecodeArgs].pack(*dvals), _capi.FORMATS[_capi.PrepArgs].pack(*pv), 0)
        assert st == 1
        assert re.search(pattern, _capi.lib().hofa_last_error().decode())
