"""hofa_decode_fwd_noalloc: the decode step for callers that cannot allocate.

Some callers of this library cannot allocate device memory: a host runtime
that owns every allocation and gives plugins no allocator, a real-time decode
loop that must never enter the driver's allocator, or glue code that only
holds borrowed pointers to its inputs and outputs.  For them the library has
one entry point that uses a scratch array built into the library instead of a
caller-provided workspace.  These tests call it through the C ABI and check
that it returns what the ordinary entry point (hofa_decode_fwd with its own
workspace) returns, on two calls in a row, and that shapes needing more
scratch than the array holds are refused with a clear message.

This file is collected last on purpose (``test_zz_``): if it fails, a run
that stops at the first failure has already run every other test.
"""
import ctypes

import pytest
import torch
import torch.nn.functional as F

from outlierneuronattention_b200 import _capi

TOL = 2e-2  # bf16 outputs, as in the other decode tests


def _noalloc_fn():
    fn = _capi.lib().hofa_decode_fwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    return fn


def _inputs(B, H, D, R, L, seed):
    g = torch.Generator().manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=g)
    bf = lambda t: t.to(torch.bfloat16).cuda()
    return dict(q=bf(rn(B, H, 1, D)), k=bf(rn(B, H, 1, D)), v=bf(rn(B, H, 1, D)),
                cache_k=bf(rn(B, H, L, R)), cache_v=bf(rn(B, H, L, D)),
                state=(rn(B, H, D - R, D) * 0.1).cuda(),
                log_gamma=F.logsigmoid(rn(B, H, 1)).cuda(), mix=bf(torch.sigmoid(rn(B, H, 1))),
                norm_w=(1 + 0.2 * rn(H, D)).cuda())


def _values(x, state_in, state_out, y, R, seq_len, split_k, seq_len_dev=None):
    # the workspace fields are ignored by the no-alloc entry point
    from outlierneuronattention_b200.hofa_decode import decode_args
    dummy = torch.empty(0, dtype=torch.uint8, device="cuda")
    return decode_args(x["q"], x["k"], x["v"], x["cache_k"], x["cache_v"], state_in, state_out, x["log_gamma"],
                       x["mix"], x["norm_w"], R, seq_len, 2.0, y, split_k=split_k, workspace=dummy,
                       seq_len_dev=seq_len_dev)


def _read_status(stream):
    fn = _capi.lib().hofa_decode_noalloc_read_status
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32)]
    out = ctypes.c_int32(-1)
    assert fn(stream, ctypes.byref(out)) == 0, _capi.lib().hofa_last_error().decode()
    return out.value


@pytest.mark.gpu
@pytest.mark.parametrize("device_len", [False, True])  # seq_len as a host int, or read from device memory
@pytest.mark.parametrize("split_k", [0, 4, 24])  # 0: automatic; 4: cluster combine; 24: combine through the scratch
def test_noalloc_matches_workspace_entry_point_two_calls(split_k, device_len):
    from outlierneuronattention_b200 import fused_hofa_decode
    B, H, D, R, L = 2, 4, 64, 16, 1500
    fn = _noalloc_fn()
    stream = _capi.stream_handle(torch.device("cuda"))
    x = _inputs(B, H, D, R, L, seed=split_k + 100 * device_len)
    lens = (L, L - 7)
    devs = [torch.tensor([n], dtype=torch.int32, device="cuda") if device_len else None for n in lens]
    s0 = x["state"]
    s1_ref, s1 = torch.empty_like(s0), torch.empty_like(s0)
    s2_ref, s2 = torch.empty_like(s0), torch.empty_like(s0)
    # two decode steps in a row through each entry point (the second reads the first's state)
    y1_ref = fused_hofa_decode(x["q"], x["k"], x["v"], x["cache_k"], x["cache_v"], s0, s1_ref, x["log_gamma"],
                               x["mix"], x["norm_w"], R, lens[0], 2.0, split_k=split_k or None, seq_len_dev=devs[0])
    y2_ref = fused_hofa_decode(x["q"], x["k"], x["v"], x["cache_k"], x["cache_v"], s1_ref, s2_ref, x["log_gamma"],
                               x["mix"], x["norm_w"], R, lens[1], 2.0, split_k=split_k or None, seq_len_dev=devs[1])
    y1, y2 = torch.empty_like(x["q"]), torch.empty_like(x["q"])
    buf1 = _capi.FORMATS[_capi.DecodeArgs].pack(*_values(x, s0, s1, y1, R, lens[0], split_k, devs[0]))
    assert fn(buf1, stream) == 0, _capi.lib().hofa_last_error().decode()
    buf2 = _capi.FORMATS[_capi.DecodeArgs].pack(*_values(x, s1, s2, y2, R, lens[1], split_k, devs[1]))
    assert fn(buf2, stream) == 0, _capi.lib().hofa_last_error().decode()
    torch.cuda.synchronize()
    for got, ref in ((y1, y1_ref), (y2, y2_ref)):
        assert torch.isfinite(got).all()
        assert (got.float() - ref.float()).abs().max().item() <= TOL
    for got, ref in ((s1, s1_ref), (s2, s2_ref)):
        torch.testing.assert_close(got, ref, atol=1e-5, rtol=1e-5)
    assert _read_status(stream) == 0


@pytest.mark.gpu
def test_noalloc_status_reports_a_clamped_device_length():
    """A device-side seq_len beyond the cache is clamped by the kernel and
    flagged (bit 1); the flag is readable through the no-alloc status reader,
    which then clears it."""
    B, H, D, R, L = 1, 2, 64, 16, 300
    fn = _noalloc_fn()
    stream = _capi.stream_handle(torch.device("cuda"))
    x = _inputs(B, H, D, R, L, seed=7)
    assert _read_status(stream) == 0
    bad = torch.tensor([L + 50], dtype=torch.int32, device="cuda")
    s1, y = torch.empty_like(x["state"]), torch.empty_like(x["q"])
    assert fn(_capi.FORMATS[_capi.DecodeArgs].pack(*_values(x, x["state"], s1, y, R, L, 0, bad)), stream) == 0
    assert _read_status(stream) & 1
    assert _read_status(stream) == 0
    assert torch.isfinite(y.float()).all()


def test_noalloc_rejects_shapes_beyond_its_scratch():
    """B*H*split partials larger than the built-in array: refused before any
    device work (fake pointers are never touched)."""
    fn = _noalloc_fn()
    B, H, D, R, L = 256, 16, 64, 16, 4096

    def tv(shape, dtype=1, ptr=0x10000):
        st, acc = [], 1
        for s in reversed(shape):
            st.insert(0, acc)
            acc *= s
        n = len(shape)
        return (ptr, dtype, n) + tuple(shape) + (1,) * (4 - n) + tuple(st) + (0,) * (4 - n)

    vals = _capi.flat(tv([B, H, 1, D]), tv([B, H, 1, D]), tv([B, H, 1, D]), tv([B, H, L, R]), tv([B, H, L, D]),
                      tv([B, H, D - R, D], 0), tv([B, H, D - R, D], 0, 0x20000), tv([B, H, 1], 0), tv([B, H, 1]),
                      tv([H, D], 0), _capi.ABSENT, tv([B, H, 1, D]), R, L, 0, 2.0, 1e-7, 8, 0, 0)
    st = fn(_capi.FORMATS[_capi.DecodeArgs].pack(*vals), 0)
    assert st == 4  # HOFA_ERR_WORKSPACE
    msg = _capi.lib().hofa_last_error().decode()
    assert "needs" in msg and "built-in array holds 2097152" in msg


def test_noalloc_rejects_bad_split_before_any_device_work():
    """An out-of-range split_k is refused by the same validation as
    hofa_decode_fwd, before the entry point issues anything (the fake
    pointers are never touched, and no device is needed)."""
    fn = _noalloc_fn()
    B, H, D, R, L = 1, 2, 64, 16, 256

    def tv(shape, dtype=1, ptr=0x10000):
        st, acc = [], 1
        for s in reversed(shape):
            st.insert(0, acc)
            acc *= s
        n = len(shape)
        return (ptr, dtype, n) + tuple(shape) + (1,) * (4 - n) + tuple(st) + (0,) * (4 - n)

    vals = _capi.flat(tv([B, H, 1, D]), tv([B, H, 1, D]), tv([B, H, 1, D]), tv([B, H, L, R]), tv([B, H, L, D]),
                      tv([B, H, D - R, D], 0), tv([B, H, D - R, D], 0, 0x20000), tv([B, H, 1], 0), tv([B, H, 1]),
                      tv([H, D], 0), _capi.ABSENT, tv([B, H, 1, D]), R, L, 0, 2.0, 1e-7, 65, 0, 0)
    st = fn(_capi.FORMATS[_capi.DecodeArgs].pack(*vals), 0)
    assert st == 1  # HOFA_ERR_INVALID_ARGUMENT
    assert "split_k=65" in _capi.lib().hofa_last_error().decode()
