"""Device checks of the properties behind the fast paths of pass 1: the
certified re-quantisation (exact indices from an approximate log plus a
per-quad error test) needs the hardware lg2 estimate within its assumed bound
and the checker's log monotone; the default parameter update uses a
reciprocal that is correctly rounded after one Newton step; bf16 parameters
are rounded by the hardware pair conversion, which must equal the portable
round-to-nearest-even. All are checked over every normal binary32 input (the
bf16 rounding over every non-NaN one).
"""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_fast_math_properties_exhaustive():
    from turboadam_b200 import _lib

    lib = _lib.load()
    out = torch.zeros(6, dtype=torch.int64, device="cuda")
    _lib.check(lib.ta_selftest_fast_math(out.data_ptr(), torch.cuda.current_stream().cuda_stream),
               "ta_selftest_fast_math")
    torch.cuda.synchronize()
    words = out.cpu().numpy().astype(np.uint64)
    max_err = float(words[:1].view(np.float64)[0])
    assert int(words[1]) == 0, "ta_logf is not monotone on the normal floats"
    assert 0.0 < max_err <= 2.0 ** -16, f"lg2.approx error {max_err} (2^{math.log2(max_err):.2f})"
    assert int(words[2]) == 0, "rcp.approx + one Newton step is not RN(1/x) everywhere"
    rs, rc = (float(x) for x in words[3:5].view(np.float64))
    assert 0.0 < rs <= 2.0 ** -22, f"rsqrt.approx relative error 2^{math.log2(rs):.2f}"
    assert 0.0 < rc <= 2.0 ** -22, f"rcp.approx relative error 2^{math.log2(rc):.2f}"
    assert int(words[5]) == 0, "cvt.rn.bf16x2.f32 differs from the portable bf16 rounding"


@pytest.mark.parametrize("v_bits", [2, 4, 8])
def test_boundary_heavy_blocks_bitexact(oracle, v_bits):
    """Gradients built so that many elements sit on or near re-quantisation
    decision points (constant blocks, repeated values, two magnitudes, tiny
    and graded spans, zero rows): the step must still match the checker bit
    for bit in every index, header and parameter, in both random modes."""
    from turboadam_b200 import TurboAdam

    rng = np.random.default_rng(11 + v_bits)
    n = 128 * 64
    kw = dict(lr=6e-4, betas=(0.9, 0.999), weight_decay=0.01, v_bits=v_bits)
    init = (rng.standard_normal(n) * 0.02).astype(np.float32)
    tp = torch.nn.Parameter(torch.from_numpy(init.copy()).cuda())
    op = oracle.OracleParam(init.copy())
    opt = TurboAdam([tp], seed=3, exact_params=True, **kw)
    oopt = oracle.OracleTurboAdam([oracle.OracleTurboAdam.make_group([op], **kw)])
    for step in range(8):
        g = (rng.standard_normal(n) * 1e-3).astype(np.float32)
        gb = g.reshape(64, 128)
        gb[0:8] = 1e-3                                    # constant blocks
        gb[8:16] = gb[8:16, :1]                           # constant per block
        gb[16:24] = np.where(rng.random((8, 128)) < 0.5, 1e-3, -1e-3)
        gb[24:32] *= np.float32(1e-4)                     # tiny gradients
        gb[32:40] = (np.arange(128) * 1e-5).astype(np.float32)  # graded
        gb[40:44] = 0.0                                   # zero rows
        tp.grad = torch.from_numpy(g.copy()).cuda()
        op.grad = g.copy()
        parity = step % 2 == 1
        if parity:
            u = rng.random(n, np.float32)
            u.reshape(64, 128)[:, ::3] = rng.integers(0, 2, (64, 43)).astype(np.float32) * 0.5
            opt._parity = {"uniforms": {tp: torch.from_numpy(u).cuda()}}
            ufn = lambda i, st, npad, u=u: u  # noqa: E731
        else:
            opt._parity = None
            ufn = lambda i, st, npad: oracle.sr_uniforms(op.n, i, st, 3)  # noqa: E731
        opt.step()
        oopt.step(uniforms=ufn)
        torch.cuda.synchronize()
        st = opt.state[tp]
        ost = oopt.state[id(op)]
        tag = f"step {step} parity {parity}"
        np.testing.assert_array_equal(st["compressed_v"]["indices"].cpu().numpy(), ost.v_idx,
                                      err_msg=tag)
        hdr = st["compressed_v"]["scales"].contiguous().view(torch.int16).cpu().numpy()
        np.testing.assert_array_equal(hdr.view(np.uint16).reshape(-1), ost.v_hdr, err_msg=tag)
        got = tp.detach().cpu().numpy()
        assert np.array_equal(got.view(np.uint32), op.data.view(np.uint32)), tag


def test_nonfinite_headers_and_wild_indices_bitexact(oracle):
    """State a checkpoint could hold but a step never writes -- NaN / inf /
    huge log-scale headers and indices >= 2^v_bits -- must take the exact
    path and still match the checker bit for bit."""
    from turboadam_b200 import TurboAdam

    rng = np.random.default_rng(21)
    n = 128 * 48
    kw = dict(lr=1e-3, betas=(0.9, 0.999), weight_decay=0.0, v_bits=4, compress_m=False)
    init = (rng.standard_normal(n) * 0.02).astype(np.float32)
    tp = torch.nn.Parameter(torch.from_numpy(init.copy()).cuda())
    op = oracle.OracleParam(init.copy())
    opt = TurboAdam([tp], seed=9, exact_params=True, **kw)
    oopt = oracle.OracleTurboAdam([oracle.OracleTurboAdam.make_group([op], **kw)])
    h16 = lambda x: np.float16(x).view(np.uint16)  # noqa: E731
    for step in range(3):
        g = (rng.standard_normal(n) * 1e-3).astype(np.float32)
        tp.grad = torch.from_numpy(g.copy()).cuda()
        op.grad = g.copy()
        if step == 1:
            st, ost = opt.state[tp], oopt.state[id(op)]
            hdr = ost.v_hdr.reshape(-1, 2).copy()
            hdr[0] = [h16(np.nan), h16(-10.0)]
            hdr[1] = [h16(-20.0), h16(np.inf)]
            hdr[2] = [h16(-np.inf), h16(-5.0)]
            hdr[3] = [h16(-60000.0), h16(60000.0)]
            hdr[4] = [h16(50.0), h16(90.0)]
            idx = ost.v_idx.copy()
            idx[5 * 128:5 * 128 + 7] = [16, 17, 100, 255, 31, 64, 200]
            ost.v_hdr[:] = hdr.reshape(-1)
            ost.v_idx[:] = idx
            cv = st["compressed_v"]
            cv["scales"].view(torch.int16).reshape(-1)[: hdr.size].copy_(
                torch.from_numpy(hdr.reshape(-1).view(np.int16)))
            cv["indices"][: idx.size].copy_(torch.from_numpy(idx))
        opt.step()
        oopt.step(uniforms=lambda i, st_, npad: oracle.sr_uniforms(op.n, i, st_, 9))
        torch.cuda.synchronize()
        st, ost = opt.state[tp], oopt.state[id(op)]
        tag = f"step {step}"
        np.testing.assert_array_equal(st["compressed_v"]["indices"].cpu().numpy()[: ost.v_idx.size],
                                      ost.v_idx, err_msg=tag)
        hdr = st["compressed_v"]["scales"].contiguous().view(torch.int16).cpu().numpy()
        got_h = hdr.view(np.uint16).reshape(-1)[: ost.v_hdr.size]
        nan_ref = np.isnan(ost.v_hdr.view(np.float16).astype(np.float32))
        np.testing.assert_array_equal(got_h[~nan_ref], ost.v_hdr[~nan_ref], err_msg=tag)
        assert np.isnan(got_h[nan_ref].view(np.float16).astype(np.float32)).all(), tag
        got = tp.detach().cpu().numpy()
        same = (got.view(np.uint32) == op.data.view(np.uint32)) | (np.isnan(got) & np.isnan(op.data))
        assert same.all(), tag


@pytest.mark.gpu
def test_bounded_wait_runs_out_and_reports():
    """The pipelines' bounded mbarrier wait (ta_selftest_wait_timeout): a
    stage armed for a copy that never lands makes every consumer warp's wait
    and then the producer's run out after the limit; the kernel returns, the
    status word reads TA_STATUS_WAIT_TIMEOUT and the context stays usable."""
    from turboadam_b200 import _lib

    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.zeros(2, dtype=torch.int64, device="cuda")
    limit_ns = 20_000_000  # 20 ms
    rc = lib.ta_selftest_wait_timeout(limit_ns, status.data_ptr(), out.data_ptr(),
                                      _lib.stream_ptr(torch.device("cuda")))
    assert rc == 0, lib.ta_last_error().decode()
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.TA_STATUS_WAIT_TIMEOUT
    elapsed, timeouts = (int(x) for x in out.tolist())
    assert timeouts == 5  # 4 consumer warps + the producer
    assert limit_ns <= elapsed < 1_000_000_000
    assert torch.ones(4, device="cuda").sum().item() == 4.0
    assert lib.ta_selftest_wait_timeout(0, status.data_ptr(), out.data_ptr(), None) == 1
    assert lib.ta_selftest_wait_timeout(3_000_000_000, status.data_ptr(), out.data_ptr(),
                                        None) == 1
