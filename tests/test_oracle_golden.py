"""Pin the CPU checker (oracle/) against golden vectors produced by the
reference implementation itself (tests/golden/make_golden.py).

What is pinned:
  * fused_v_update (quantize.py:222-299): new indices and fp16 headers
    bit-exact; fp32 v_new within 1e-6 relative (torch's CPU exp is not
    correctly rounded, ours is faithful: they differ by <= 1 ulp);
  * CoStateManager.update (costate.py:367-464) with the reference's alpha
    injected: m_new, ratios, thresholds, labels, sign bits, block norms and
    fp16 scales all bit-exact; the checker's own alpha (canonical fixed-order
    reduction) within 1e-6 relative of the reference's MKL sdot result;
  * whole TurboAdam.step runs (optimizer.py:88-292), incl. multiple groups,
    v-only / m-only, bf16 params and grad-None params: every packed state
    tensor bit-exact, parameters within 1e-6 of the step scale.
"""
import numpy as np
import pytest

import golden_util as GU


def _ulps(a, b):
    a = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(a - b)


def test_v_update_golden(oracle):
    d = GU.load("v_update.npz")
    beta2 = float(d["beta2"][0])
    n_idx = 0
    for c in range(int(d["n_cases"][0])):
        k = f"c{c:03d}"
        nbits, n, ns = (int(x) for x in d[k + "_meta"])
        for s in range(ns):
            oi, oh, v = oracle.v_update(d[f"{k}_s{s}_idx_in"], d[f"{k}_s{s}_hdr_in"],
                                        d[f"{k}_s{s}_g"], nbits, beta2, d[f"{k}_s{s}_u"])
            np.testing.assert_array_equal(oi, d[f"{k}_s{s}_idx_out"], err_msg=f"{k} s{s} idx")
            np.testing.assert_array_equal(oh, d[f"{k}_s{s}_hdr_out"].reshape(-1),
                                          err_msg=f"{k} s{s} hdr")
            rv = d[f"{k}_s{s}_v_out"]
            assert _ulps(v, rv).max() <= 1, f"{k} s{s} v_new differs by > 1 ulp"
            rel = np.abs(v.astype(np.float64) - rv) / np.maximum(np.abs(rv), 1e-45)
            assert rel.max() <= 1e-6
            n_idx += oi.size
    assert n_idx > 500_000


def test_v_decode_golden(oracle):
    """decompress_v (oneq.py:51-67, quantize.py:183-214): the checker's
    decode within 1 ulp of torch's exp for every v_bits, odd tails included."""
    d = GU.load("v_decode.npz")
    n_el = 0
    for c in range(int(d["n_cases"][0])):
        k = f"c{c:03d}"
        nbits, n = (int(x) for x in d[k + "_meta"])
        v = oracle.v_decode(d[f"{k}_idx"], d[f"{k}_hdr"], n, nbits)
        rv = d[f"{k}_v"]
        assert v.shape == rv.shape == (n,), k
        assert _ulps(v, rv).max() <= 1, f"{k}: decoded v differs by > 1 ulp"
        n_el += n
    assert n_el > 80_000


def test_v_init_matches_reference(oracle):
    d = GU.load("v_update.npz")
    for c in range(int(d["n_cases"][0])):
        k = f"c{c:03d}"
        nbits, n, _ = (int(x) for x in d[k + "_meta"])
        if c % 2:  # even cases start from the fresh (1e-30) state
            continue
        idx, hdr = oracle.v_init(n)
        np.testing.assert_array_equal(idx, d[f"{k}_s0_idx_in"])
        np.testing.assert_array_equal(hdr, d[f"{k}_s0_hdr_in"].reshape(-1))
    assert np.float16(oracle.v_init(1)[1].view(np.float16)[0]) == np.float16(-69.0625)


@pytest.mark.parametrize("inject", [True, False])
def test_costate_golden(oracle, inject):
    d = GU.load("costate.npz")
    for c in range(int(d["n_cases"][0])):
        k = f"c{c:03d}"
        n, ns = (int(x) for x in d[k + "_meta"])
        lo, hi = (float(x) for x in d[k + "_pct"])
        mgr = oracle.CoStateOracle(n, 128, lo, hi)
        for s in range(ns):
            ra = float(d[f"{k}_s{s}_alpha"][0])
            if not inject:
                # alpha of the same inputs: checker's own reduction vs MKL sdot
                ref_mgr = oracle.CoStateOracle(n, 128, lo, hi)
                ref_mgr.__dict__.update({kk: (vv.copy() if isinstance(vv, np.ndarray) else vv)
                                         for kk, vv in mgr.__dict__.items()})
                ref_mgr.update(d[f"{k}_s{s}_g"], 0.9, None)
                assert abs(ref_mgr.alpha - ra) <= 1e-6 * max(abs(ra), 1e-30), (k, s)
            m = mgr.update(d[f"{k}_s{s}_g"], 0.9, ra)
            tag = f"{k} step {s}"
            np.testing.assert_array_equal(m, d[f"{k}_s{s}_m_new"], err_msg=tag)
            np.testing.assert_array_equal(mgr.last_ratios, d[f"{k}_s{s}_ratios"], err_msg=tag)
            np.testing.assert_array_equal(mgr.last_tau, d[f"{k}_s{s}_tau"], err_msg=tag)
            np.testing.assert_array_equal(mgr.labels, d[f"{k}_s{s}_labels"], err_msg=tag)
            np.testing.assert_array_equal(mgr.signs, d[f"{k}_s{s}_signs"], err_msg=tag)
            np.testing.assert_array_equal(mgr.norms, d[f"{k}_s{s}_norms"], err_msg=tag)
            np.testing.assert_array_equal(mgr.amp, d[f"{k}_s{s}_amp"], err_msg=tag)
            if not inject:
                break  # later steps of an un-injected run legitimately diverge


def test_costate_error_feedback_golden(oracle):
    """CoStateManager(error_feedback=True) sequences (costate.py:410-437) with the
    reference's alpha injected: every encoding and the fp32 residual bit-exact."""
    d = GU.load("costate_ef.npz")
    for c in range(int(d["n_cases"][0])):
        k = f"c{c:03d}"
        n, ns = (int(x) for x in d[k + "_meta"])
        lo, hi = (float(x) for x in d[k + "_pct"])
        mgr = oracle.CoStateOracle(n, 128, lo, hi, error_feedback=True)
        for s in range(ns):
            m = mgr.update(d[f"{k}_s{s}_g"], 0.9, float(d[f"{k}_s{s}_alpha"][0]))
            tag = f"{k} step {s}"
            np.testing.assert_array_equal(m, d[f"{k}_s{s}_m_new"], err_msg=tag)
            np.testing.assert_array_equal(mgr.labels, d[f"{k}_s{s}_labels"], err_msg=tag)
            np.testing.assert_array_equal(mgr.signs, d[f"{k}_s{s}_signs"], err_msg=tag)
            np.testing.assert_array_equal(mgr.norms, d[f"{k}_s{s}_norms"], err_msg=tag)
            np.testing.assert_array_equal(mgr.amp, d[f"{k}_s{s}_amp"], err_msg=tag)
            np.testing.assert_array_equal(mgr.ef_residual.view(np.uint32),
                                          d[f"{k}_s{s}_ef_residual"].view(np.uint32), err_msg=tag)


def replay_optimizer_run(oracle, name, inject_alpha=True):
    """Replays one golden optimizer run in the checker; yields per-step
    (step, params, oracle_state, fixture)."""
    pspecs, gkw, nsteps, none_set = GU.runs()[name]
    d = GU.load(f"opt_{name}.npz")
    params = []
    for pi, (shape, dt, gi) in enumerate(pspecs):
        params.append(oracle.OracleParam(d[f"p{pi}_init"].reshape(-1).copy(), bf16=dt == "bf16"))
    groups = [oracle.OracleTurboAdam.make_group(
        [params[i] for i, s in enumerate(pspecs) if s[2] == gi], **kw) for gi, kw in enumerate(gkw)]
    opt = oracle.OracleTurboAdam(groups)
    for s in range(nsteps):
        for pi, p in enumerate(params):
            if (s, pi) in none_set:
                p.grad = None
                continue
            g = d[f"s{s}_g{pi}"].reshape(-1)
            p.grad = GU.bf16_to_f32(g) if pspecs[pi][1] == "bf16" else g.astype(np.float32)
        opt.step(uniforms=lambda i, st, npad, s=s: d[f"s{s}_u{i}"],
                 alpha_inject=(lambda i, st, s=s: float(d[f"s{s}_alpha{i}"][0]))
                 if inject_alpha else (lambda i, st: None))
        yield s, params, opt, d


@pytest.mark.parametrize("name", ["block", "groups", "bf16", "gradnone", "ef"])
def test_optimizer_runs_golden(oracle, name):
    pspecs = GU.runs()[name][0]
    prev, scale = {}, {}
    for s, params, opt, d in replay_optimizer_run(oracle, name):
        for pi, p in enumerate(params):
            if f"s{s}_p{pi}" not in d:
                continue
            tag = f"{name} step {s} param {pi}"
            st = opt.state[id(p)]
            assert st.step == int(d[f"s{s}_step{pi}"][0]), tag
            rp = d[f"s{s}_p{pi}"].reshape(-1)
            if p.bf16:
                ours, ref = GU.bf16_to_f32(p.data), GU.bf16_to_f32(rp)
            else:
                ours, ref = p.data, rp
            before = prev.get(pi, GU.bf16_to_f32(d[f"p{pi}_init"].reshape(-1))
                              if p.bf16 else d[f"p{pi}_init"].reshape(-1))
            scale[pi] = np.maximum(scale.get(pi, 0.0), np.abs(ref.astype(np.float64) - before))
            ok = GU.p_close(ours, ref, scale[pi])
            assert ok.all(), f"{tag}: {np.sum(~ok)} params off"
            prev[pi] = ref
            if st.v_idx is not None:
                np.testing.assert_array_equal(st.v_idx, d[f"s{s}_vidx{pi}"], err_msg=tag)
                np.testing.assert_array_equal(st.v_hdr, d[f"s{s}_vhdr{pi}"].reshape(-1),
                                              err_msg=tag)
            if st.mgr is not None:
                np.testing.assert_array_equal(st.mgr.labels, d[f"s{s}_labels{pi}"], err_msg=tag)
                np.testing.assert_array_equal(st.mgr.signs, d[f"s{s}_signs{pi}"], err_msg=tag)
                np.testing.assert_array_equal(st.mgr.norms, d[f"s{s}_norms{pi}"], err_msg=tag)
                np.testing.assert_array_equal(st.mgr.amp, d[f"s{s}_amp{pi}"], err_msg=tag)
                if f"s{s}_ef{pi}" in d:
                    np.testing.assert_array_equal(st.mgr.ef_residual.view(np.uint32),
                                                  d[f"s{s}_ef{pi}"].reshape(-1).view(np.uint32),
                                                  err_msg=tag)
            if st.exp_avg is not None:
                np.testing.assert_array_equal(st.exp_avg, d[f"s{s}_m{pi}"].reshape(-1),
                                              err_msg=tag)
            if st.exp_avg_sq is not None:
                np.testing.assert_array_equal(st.exp_avg_sq, d[f"s{s}_vsq{pi}"].reshape(-1),
                                              err_msg=tag)
    assert pspecs


def test_threshold_ranks_match_python(oracle):
    rng = np.random.default_rng(5)
    Bs = list(range(1, 400)) + [int(x) for x in rng.integers(1, 10**7, 2000)]
    for pcts in [(0.1, 0.9), (0.2, 0.7), (0.05, 0.95), (0.33, 0.66)]:
        for B in Bs:
            lo, hi = oracle.threshold_ranks(B, *pcts)
            assert lo == max(0, int(pcts[0] * B) - 1)
            assert hi == min(B - 1, int(pcts[1] * B))
