"""Checkpoint format: dense n-bit index packing, portable (package-free,
compact) state dicts, and bit-exact resume."""
import io

import numpy as np
import pytest
import torch

from turboadam_b200.checkpoint import (load_portable_state_dict, pack_indices,
                                       portable_state_dict, unpack_indices)


@pytest.mark.parametrize("n_bits", [1, 2, 3, 4, 6, 8])
@pytest.mark.parametrize("count", [1, 7, 128, 1000, 4099])
def test_pack_unpack_roundtrip(n_bits, count):
    rng = np.random.default_rng(n_bits * 7919 + count)
    idx = torch.from_numpy(rng.integers(0, 1 << n_bits, count, dtype=np.uint8))
    packed = pack_indices(idx, n_bits)
    assert packed.numel() == (count * n_bits + 7) // 8
    assert torch.equal(unpack_indices(packed, n_bits, count), idx)


def test_pack_layout_is_lsb_first():
    idx = torch.tensor([1, 2, 3, 0], dtype=torch.uint8)  # 2-bit: 01 10 11 00
    assert pack_indices(idx, 2).tolist() == [0b00111001]
    with pytest.raises(ValueError):
        pack_indices(torch.tensor([4], dtype=torch.uint8), 2)


def _make(seed_data=0):
    g = torch.Generator().manual_seed(seed_data)
    shapes = [(300, 200), (3000,), (4096 + 77,)]
    ps = [torch.nn.Parameter((torch.randn(s, generator=g) * 0.02).cuda()) for s in shapes]
    ps.append(torch.nn.Parameter((torch.randn(257, 64, generator=g) * 0.02).to(torch.bfloat16).cuda()))
    return ps


def _grads(ps, step):
    g = torch.Generator().manual_seed(500 + step)
    return [(torch.randn(p.shape, generator=g) * 1e-3).to(p.dtype).cuda() for p in ps]


@pytest.mark.gpu
@pytest.mark.parametrize("pack,ef", [(False, False), (True, False), (False, True)])
def test_bitexact_resume_from_portable_checkpoint(pack, ef):
    from turboadam_b200 import TurboAdam

    kw = dict(lr=6e-4, weight_decay=0.01, v_bits=3, error_feedback=ef)
    a = _make()
    oa = TurboAdam(a, seed=1234, **kw)
    for s in range(5):
        for p, g in zip(a, _grads(a, s)):
            p.grad = g
        oa.step()

    b = _make()
    ob = TurboAdam(b, seed=1234, **kw)
    for s in range(3):
        for p, g in zip(b, _grads(b, s)):
            p.grad = g
        ob.step()
    buf = io.BytesIO()
    torch.save(portable_state_dict(ob, pack=pack), buf)
    buf.seek(0)
    sd = torch.load(buf, weights_only=False)
    c = [torch.nn.Parameter(p.detach().clone()) for p in b]
    oc = TurboAdam(c, seed=99, **kw)  # the checkpoint's seed wins
    load_portable_state_dict(oc, sd)
    for s in range(3, 5):
        for p, g in zip(c, _grads(c, s)):
            p.grad = g
        oc.step()
    torch.cuda.synchronize()
    for pa, pc in zip(a, c):
        assert torch.equal(pa.detach().view(-1).view(torch.uint8), pc.detach().view(-1).view(torch.uint8))
        sa, sc = oa.state[pa], oc.state[pc]
        assert sa["step"] == sc["step"]
        assert torch.equal(sa["compressed_v"]["indices"], sc["compressed_v"]["indices"])
        assert torch.equal(sa["compressed_v"]["scales"].view(torch.int16),
                           sc["compressed_v"]["scales"].view(torch.int16))
        if "m_mgr" in sa:
            ea, ec = sa["m_mgr"]._encoded, sc["m_mgr"]._encoded
            for k in ("labels", "sign_packed", "block_norms"):
                assert torch.equal(ea[k].view(torch.uint8), ec[k].view(torch.uint8)), k
            ra, rc = sa["m_mgr"]._ef_residual, sc["m_mgr"]._ef_residual
            assert (ra is None) == (rc is None) and (ra is not None) == ef
            if ef:
                assert torch.equal(ra.view(torch.int32), rc.view(torch.int32))
        if "exp_avg" in sa:
            assert torch.equal(sa["exp_avg"], sc["exp_avg"])
