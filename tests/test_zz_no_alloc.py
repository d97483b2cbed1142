"""ta_v_update_noalloc (static device scratch) against ta_v_update (caller
workspace), both called through the C ABI.

Collected last (file name) so it also runs after every other test has used
the library in the same process; it must pass alone in a fresh process too.
"""
import ctypes

import numpy as np
import pytest
import torch

from turboadam_b200 import _lib

pytestmark = pytest.mark.gpu

MAX_N = 1 << 20  # TA_V_UPDATE_NOALLOC_MAX_N in include/turboadam_b200.h
BS = 128


def _state(n, v_bits, gen):
    """A valid 1Q state: indices < 2^v_bits, headers (lmin <= lmax) in fp16."""
    nblk = (n + BS - 1) // BS
    idx = torch.randint(0, 1 << v_bits, (nblk * BS,), generator=gen, dtype=torch.int64)
    lo = -20.0 + 4.0 * torch.rand(nblk, generator=gen)
    hi = lo + 6.0 * torch.rand(nblk, generator=gen)
    hdr = torch.stack([lo, hi], dim=1).to(torch.float16).reshape(-1)
    return idx.to(torch.uint8).cuda(), hdr.cuda()


def _call(lib, fn, idx, hdr, g, n, v_bits, uni, seed, step, ws=None):
    dev = g.device
    out_idx = torch.empty_like(idx)
    out_hdr = torch.empty_like(hdr)
    v = torch.empty(n, dtype=torch.float32, device=dev)
    dt = _lib.TA_BF16 if g.dtype == torch.bfloat16 else _lib.TA_F32
    args = [idx.data_ptr(), hdr.data_ptr(), g.data_ptr(), dt, n, BS, v_bits, 0.999,
            uni.data_ptr() if uni is not None else None, seed, 7, step,
            out_idx.data_ptr(), out_hdr.data_ptr(), v.data_ptr()]
    if ws is not None:
        args += [ws.data_ptr(), ws.numel()]
    rc = getattr(lib, fn)(*args, _lib.stream_ptr(dev))
    assert rc == 0, f"{fn}: {lib.ta_last_error().decode()}"
    return out_idx, out_hdr, v


@pytest.mark.parametrize("n,v_bits,dtype,use_uni", [
    (1000, 4, torch.float32, False),
    (MAX_N, 4, torch.float32, False),
    (300001, 3, torch.bfloat16, True),
])
def test_noalloc_matches_workspace_entry_point(n, v_bits, dtype, use_uni):
    lib = _lib.load()
    gen = torch.Generator().manual_seed(n + v_bits)
    idx, hdr = _state(n, v_bits, gen)
    nblk = (n + BS - 1) // BS
    ws = torch.zeros(lib.ta_aux_workspace_size(n), dtype=torch.uint8, device="cuda")
    grads = [(1e-3 * torch.randn(n, generator=gen)).to(dtype).cuda() for _ in range(2)]
    unis = [torch.rand(nblk * BS, generator=gen).cuda() if use_uni else None for _ in range(2)]
    torch.cuda.synchronize()

    # two calls in a row, each fed the previous call's state
    a_idx, a_hdr = idx, hdr
    b_idx, b_hdr = idx, hdr
    for k in range(2):
        ra = _call(lib, "ta_v_update", a_idx, a_hdr, grads[k], n, v_bits, unis[k], 11, k + 1,
                   ws=ws)
        reserved = torch.cuda.memory_reserved()
        rb = _call(lib, "ta_v_update_noalloc", b_idx, b_hdr, grads[k], n, v_bits, unis[k], 11,
                   k + 1)
        torch.cuda.synchronize()
        assert torch.cuda.memory_reserved() == reserved
        # tolerance: exact -- both run the same kernels on the same inputs
        assert torch.equal(ra[0], rb[0]), f"indices differ on call {k}"
        assert torch.equal(ra[1].view(torch.int16), rb[1].view(torch.int16)), \
            f"headers differ on call {k}"
        np.testing.assert_array_equal(ra[2].cpu().numpy().view(np.uint32),
                                      rb[2].cpu().numpy().view(np.uint32))
        a_idx, a_hdr = ra[0], ra[1]
        b_idx, b_hdr = rb[0], rb[1]


def test_noalloc_status_reports_nonfinite_gradient_per_call():
    """A NaN gradient sets TA_STATUS_NONFINITE_GRAD in the static array's
    status word; the next call (finite gradient) starts from a clear word, and
    clear=1 zeroes it after the read."""
    lib = _lib.load()
    n, v_bits = 5000, 4
    gen = torch.Generator().manual_seed(3)
    idx, hdr = _state(n, v_bits, gen)
    stream = _lib.stream_ptr(torch.device("cuda"))

    def status(clear):
        v = ctypes.c_uint32(0)
        rc = lib.ta_v_update_noalloc_status(int(clear), ctypes.byref(v), stream)
        assert rc == 0, lib.ta_last_error().decode()
        return v.value

    g = (1e-3 * torch.randn(n, generator=gen)).cuda()
    g_bad = g.clone()
    g_bad[17] = float("nan")   # full block: fast path flags it, exact path reports it
    g_bad[n - 3] = float("inf")  # ragged tail block: general path
    _call(lib, "ta_v_update_noalloc", idx, hdr, g_bad, n, v_bits, None, 5, 1)
    assert status(clear=False) & _lib.TA_STATUS_NONFINITE_GRAD
    assert status(clear=True) & _lib.TA_STATUS_NONFINITE_GRAD  # still set, then cleared
    assert status(clear=False) == 0
    _call(lib, "ta_v_update_noalloc", idx, hdr, g_bad, n, v_bits, None, 5, 2)
    assert status(clear=False) & _lib.TA_STATUS_NONFINITE_GRAD
    _call(lib, "ta_v_update_noalloc", idx, hdr, g, n, v_bits, None, 5, 3)
    assert status(clear=False) == 0  # each call reports only itself


def test_noalloc_rejects_oversize():
    lib = _lib.load()
    rc = lib.ta_v_update_noalloc(None, None, None, _lib.TA_F32, MAX_N + 1, BS, 4, 0.999, None,
                                 0, 0, 1, None, None, None, _lib.stream_ptr(torch.device("cuda")))
    assert rc == 3  # TA_ERR_UNSUPPORTED
    msg = lib.ta_last_error().decode()
    assert "exceeds the static scratch limit" in msg and str(MAX_N) in msg
    assert ctypes.sizeof(ctypes.c_void_p) == 8
