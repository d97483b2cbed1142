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


# ---------------------------------------------------------------------------
# reference checkpoints (tests/golden/ref_ckpt.pt: the reference's own
# torch.save(opt.state_dict()) after 3 steps; ckpt_cont.npz: its next 2 steps)
# ---------------------------------------------------------------------------

def _ref_ckpt_path():
    import os

    return os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_ckpt.pt")


def test_reference_state_dict_loads_without_the_reference_package():
    import sys

    from turboadam_b200.checkpoint import ReferenceCoStateManager, load_reference_state_dict
    from turboadam_b200.costate import CoStateManager

    assert "turboadam" not in sys.modules  # nothing of the reference is importable here
    sd = load_reference_state_dict(_ref_ckpt_path())
    assert [g["params"] for g in sd["param_groups"]] == [[0, 1, 2], [3, 4]]
    kinds = {k: type(st.get("m_mgr")).__name__ for k, st in sd["state"].items()}
    assert kinds == {0: "ReferenceCoStateManager", 1: "ReferenceCoStateManager",
                     2: "NoneType", 3: "ReferenceCoStateManager", 4: "ReferenceCoStateManager"}
    st = sd["state"][3]
    assert st["step"] == 3 and st["compressed_v"]["n_bits"] == 3
    ref = st["m_mgr"]
    assert isinstance(ref, ReferenceCoStateManager)
    assert ref._encoded["scales"].dtype == torch.float16 and ref._ef_residual.shape == (4133,)
    mgr = CoStateManager.from_reference(ref)
    assert (mgr.block_size, mgr._null_pct, mgr._amp_pct) == (128, 0.10, 0.90)
    assert mgr._has_state and mgr._error_feedback and mgr._original_numel == 4133
    assert float(mgr._alpha) == float(ref._alpha)
    assert torch.equal(mgr._encoded["sign_packed"], ref._encoded["sign_packed"])


def test_reference_loader_refuses_other_reference_classes(tmp_path):
    import pickle
    import sys
    import types

    from turboadam_b200.checkpoint import load_reference_state_dict

    mod = types.ModuleType("turboadam.quantize")

    class Other:  # a class of the reference package that is not optimizer state
        pass

    Other.__module__ = "turboadam.quantize"
    Other.__qualname__ = "Other"
    mod.Other = Other
    pkg = types.ModuleType("turboadam")
    saved = {k: sys.modules.get(k) for k in ("turboadam", "turboadam.quantize")}
    sys.modules["turboadam"] = pkg
    sys.modules["turboadam.quantize"] = mod
    try:
        path = tmp_path / "bad.pt"
        torch.save({"state": {0: {"x": Other()}}, "param_groups": []}, path)
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
    with pytest.raises(pickle.UnpicklingError, match="not part of a TurboAdam optimizer state"):
        load_reference_state_dict(path)


def _continue_from_reference(sd, exact_params):
    """Loads `sd` into a TurboAdam on the GPU, runs the reference's next 2
    steps (its gradients, uniforms and alpha injected) and compares every
    output with the reference's own continuation."""
    import golden_util as GU
    from turboadam_b200 import TurboAdam

    gmod = GU.load_module("make_golden.py")
    pspecs, gkw, _, n_after = gmod.CKPT_SPEC
    d = GU.load("ckpt_cont.npz")
    params = [torch.nn.Parameter(torch.from_numpy(d[f"p{pi}_ckpt"].copy()).cuda())
              for pi in range(len(pspecs))]
    groups = [dict(params=[params[i] for i, s in enumerate(pspecs) if s[1] == gi], **kw)
              for gi, kw in enumerate(gkw)]
    opt = TurboAdam(groups, exact_params=exact_params)
    opt.load_state_dict(sd)
    prev, scale = {}, {}
    for s in range(n_after):
        uni, alph = {}, {}
        for pi, p in enumerate(params):
            p.grad = torch.from_numpy(d[f"s{s}_g{pi}"]).cuda()
            uni[p] = torch.from_numpy(d[f"s{s}_u{pi}"]).cuda()
            if f"s{s}_alpha{pi}" in d:
                alph[p] = torch.from_numpy(d[f"s{s}_alpha{pi}"]).cuda()
        opt._parity = {"uniforms": uni, "alpha": alph}
        opt.step()
        torch.cuda.synchronize()
        for pi, p in enumerate(params):
            tag = f"continuation step {s} param {pi}"
            st = opt.state[p]
            assert st["step"] == int(d[f"s{s}_step{pi}"][0]) == 4 + s, tag
            ref = d[f"s{s}_p{pi}"].reshape(-1)
            before = prev.get(pi, d[f"p{pi}_ckpt"].reshape(-1))
            scale[pi] = np.maximum(scale.get(pi, 0.0), np.abs(ref.astype(np.float64) - before))
            ok = GU.p_close(p.detach().cpu().numpy().reshape(-1), ref, scale[pi])
            assert ok.all(), f"{tag}: {np.sum(~ok)} params off"
            prev[pi] = ref
            cv = st["compressed_v"]
            assert np.array_equal(cv["indices"].cpu().numpy(), d[f"s{s}_vidx{pi}"]), tag
            assert np.array_equal(cv["scales"].contiguous().view(torch.int16).cpu().numpy()
                                  .view(np.uint16).reshape(-1), d[f"s{s}_vhdr{pi}"].reshape(-1)), tag
            if "exp_avg" in st:
                assert np.array_equal(st["exp_avg"].cpu().numpy().reshape(-1),
                                      d[f"s{s}_m{pi}"].reshape(-1)), tag
            if "m_mgr" in st:
                enc = st["m_mgr"]._encoded
                for k, key in (("labels", "labels"), ("sign_packed", "signs"),
                               ("block_norms", "norms")):
                    assert np.array_equal(enc[k].cpu().numpy(), d[f"s{s}_{key}{pi}"]), (tag, k)
                assert np.array_equal(enc["scales"].view(torch.int16).cpu().numpy()
                                      .view(np.uint16), d[f"s{s}_amp{pi}"]), tag
                if f"s{s}_ef{pi}" in d:
                    ef = st["m_mgr"]._ef_residual
                    assert tuple(ef.shape) == tuple(pspecs[pi][0]), tag
                    assert np.array_equal(ef.cpu().numpy().reshape(-1).view(np.uint32),
                                          d[f"s{s}_ef{pi}"].reshape(-1).view(np.uint32)), tag


@pytest.mark.gpu
@pytest.mark.parametrize("exact_params", [True, False])
def test_resume_reference_checkpoint_matches_reference_continuation(exact_params):
    """Reference checkpoint -> TurboAdam.load_state_dict -> 2 more steps:
    indices, headers, labels, sign bits, norms, fp16 scales, error-feedback
    residuals and exp_avg bit-exact vs the reference's own continuation;
    parameters within 1e-6 of the step scale."""
    from turboadam_b200.checkpoint import load_reference_state_dict

    _continue_from_reference(load_reference_state_dict(_ref_ckpt_path()), exact_params)


@pytest.mark.gpu
def test_resume_reference_checkpoint_with_reference_classes_importable(monkeypatch):
    """With the reference package installed, torch.load gives its own
    CoStateManager objects; load_state_dict converts them just the same.
    (The reference is not importable on the GPU machine, so a class of the
    same module path and attributes stands in for it.)"""
    import sys
    import types

    pkg = types.ModuleType("turboadam")
    mod = types.ModuleType("turboadam.costate")

    class CoStateManager:  # the reference's class: plain attributes, no methods needed
        pass

    CoStateManager.__module__ = "turboadam.costate"
    mod.CoStateManager = CoStateManager
    pkg.costate = mod
    monkeypatch.setitem(sys.modules, "turboadam", pkg)
    monkeypatch.setitem(sys.modules, "turboadam.costate", mod)
    sd = torch.load(_ref_ckpt_path(), weights_only=False)
    assert type(sd["state"][0]["m_mgr"]) is CoStateManager
    _continue_from_reference(sd, exact_params=True)
