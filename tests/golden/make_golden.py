"""Generate golden vectors by running the reference TurboAdam (CPU path).

Usage (in a container that has the reference checkout):
    python tests/golden/make_golden.py [--ref /path/to/turboadam] [--out tests/golden]

The reference is imported from ``<ref>/src``; its stochastic rounding draw
(``torch.rand_like`` at reference ``quantize.py:291``) is replaced by seeded
uniform tensors that are stored in the fixtures, so the checker and the CUDA
path can be fed exactly the same draws. The reference's own alpha (the
``CoStateManager._alpha`` it stores, ``costate.py:443-456``) and its P10/P90
thresholds (``compute_thresholds``, ``costate.py:94-118``) are recorded per
step, so integer state can be compared with alpha injected.

Fixtures are compressed .npz files; the whole set stays a few MB.
"""
from __future__ import annotations

import argparse
import contextlib
import os
import sys
import zlib

import numpy as np
import torch


def _import_reference(ref: str):
    sys.path.insert(0, os.path.join(ref, "src"))
    import turboadam  # noqa: F401
    from turboadam import costate, oneq, optimizer, quantize

    return turboadam, costate, oneq, optimizer, quantize


class UniformFeed:
    """Replaces torch.rand_like with a queue of prepared tensors."""

    def __init__(self):
        self.queue = []
        self.orig = torch.rand_like

    def push(self, arr: np.ndarray):
        self.queue.append(torch.from_numpy(np.ascontiguousarray(arr, np.float32)))

    def __call__(self, like, *a, **k):
        assert self.queue, "reference drew more uniforms than prepared"
        t = self.queue.pop(0)
        assert t.numel() == like.numel(), (t.numel(), like.numel())
        return t.reshape(like.shape).to(like.dtype)

    @contextlib.contextmanager
    def active(self):
        torch.rand_like = self
        try:
            yield self
        finally:
            torch.rand_like = self.orig
            assert not self.queue, "unused uniforms left in the feed"


def h16(t: torch.Tensor) -> np.ndarray:
    """fp16 tensor -> uint16 bit patterns."""
    return t.detach().to(torch.float16).contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16).copy()


# ---------------------------------------------------------------------------
# A. fused_v_update (quantize.py:222-299)
# ---------------------------------------------------------------------------


def gen_v_cases(mods, out_dir):
    _, _, oneq, _, quantize = mods
    rng = np.random.default_rng(1234)
    feed = UniformFeed()
    cases = {}
    ci = 0
    for nbits in (2, 3, 4, 6, 8):
        for n in (1, 129, 1000, 16384 + 37):
            for init in ("fresh", "random"):
                B = (n + 127) // 128
                if init == "fresh":
                    v0 = torch.full((n,), 1e-30, dtype=torch.float32)
                else:
                    v0 = torch.from_numpy(
                        (rng.random(n) * 10.0 ** rng.uniform(-12, -2, n)).astype(np.float32))
                cv = oneq.compress_v_logscale(v0, n_bits=nbits, block_size=128,
                                              stochastic_round=False)
                idx = cv["indices"].clone()
                hdr = cv["scales"].clone()
                steps = []
                for s in range(3):
                    kind = (ci + s) % 3
                    if kind == 0:
                        g = rng.standard_normal(n) * 1e-3
                    elif kind == 1:
                        g = rng.standard_t(3, n) * 1e-3
                    else:
                        g = rng.standard_normal(n) * 10.0 ** rng.uniform(-6, 0, n)
                        g[rng.random(n) < 0.1] = 0.0
                    g = g.astype(np.float32)
                    u = rng.random(B * 128).astype(np.float32)
                    feed.push(u)
                    with feed.active():
                        ni, nh, v = quantize.fused_v_update(
                            idx, hdr, torch.from_numpy(g), 0.999, nbits, 128, n)
                    steps.append(dict(idx_in=idx.numpy().copy(), hdr_in=h16(hdr), g=g, u=u,
                                      idx_out=ni.numpy().copy(), hdr_out=h16(nh),
                                      v_out=v.numpy().copy()))
                    idx, hdr = ni, nh
                key = f"c{ci:03d}"
                for s, d in enumerate(steps):
                    for k, v in d.items():
                        cases[f"{key}_s{s}_{k}"] = v
                cases[f"{key}_meta"] = np.array([nbits, n, 3], np.int64)
                ci += 1
    cases["n_cases"] = np.array([ci], np.int64)
    cases["beta2"] = np.array([0.999], np.float64)
    np.savez_compressed(os.path.join(out_dir, "v_update.npz"), **cases)
    print("v_update cases:", ci)


def gen_v_decode_cases(mods, out_dir):
    """decompress_v (oneq.py:51-67 -> quantize.py:183-214) of states made by
    compress_v_logscale (oneq.py:13-48) from random v, every v_bits."""
    _, _, oneq, _, _ = mods
    rng = np.random.default_rng(4321)
    cases = {}
    ci = 0
    for nbits in (2, 3, 4, 6, 8):
        for n in (1, 129, 16384 + 37):
            v0 = torch.from_numpy(
                (rng.random(n) * 10.0 ** rng.uniform(-14, 0, n)).astype(np.float32))
            cv = oneq.compress_v_logscale(v0, n_bits=nbits, block_size=128,
                                          stochastic_round=False)
            v = oneq.decompress_v(cv)
            key = f"c{ci:03d}"
            cases[f"{key}_idx"] = cv["indices"].numpy().copy()
            cases[f"{key}_hdr"] = h16(cv["scales"])
            cases[f"{key}_v"] = v.reshape(-1).numpy().copy()
            cases[f"{key}_meta"] = np.array([nbits, n], np.int64)
            ci += 1
    cases["n_cases"] = np.array([ci], np.int64)
    np.savez_compressed(os.path.join(out_dir, "v_decode.npz"), **cases)
    print("v_decode cases:", ci)


# ---------------------------------------------------------------------------
# B. CoStateManager.update sequences (costate.py:367-464)
# ---------------------------------------------------------------------------


COSTATE_SPECS = [
    (4096, 0.10, 0.90, 5),
    (4133, 0.10, 0.90, 5),
    (384, 0.10, 0.90, 4),
    (300, 0.10, 0.90, 4),
    (65536 + 11, 0.10, 0.90, 4),
    (20000, 0.20, 0.70, 4),
    (128, 0.10, 0.90, 3),
]
# error_feedback=True sequences (costate.py:410-437), written to costate_ef.npz
COSTATE_EF_SPECS = [
    (4096, 0.10, 0.90, 5),
    (4133, 0.10, 0.90, 5),
    (20000, 0.20, 0.70, 4),
]


def gen_costate_cases(mods, out_dir, ef=False):
    _, costate, _, _, _ = mods
    rng = np.random.default_rng(199 if ef else 99)
    cases = {}
    specs = COSTATE_EF_SPECS if ef else COSTATE_SPECS
    rec = {}
    orig_thr = costate.compute_thresholds

    def thr(ratios, null_pct=0.10, amp_pct=0.90):
        t0, t1 = orig_thr(ratios, null_pct, amp_pct)
        rec["ratios"] = ratios.detach().numpy().copy()
        rec["tau"] = np.array([float(t0), float(t1)], np.float32)
        return t0, t1

    costate.compute_thresholds = thr
    try:
        for ci, (n, lo, hi, nsteps) in enumerate(specs):
            mgr = costate.CoStateManager(block_size=128, null_pct=lo, amp_pct=hi,
                                         error_feedback=ef)
            key = f"c{ci:03d}"
            for s in range(nsteps):
                scale = 10.0 ** rng.uniform(-5, -2)
                g = (rng.standard_normal(n) * scale).astype(np.float32)
                if s == 2:
                    g[: n // 7] = 0.0  # a run of zero gradient
                m_new = mgr.update(torch.from_numpy(g), 0.9)
                enc = mgr._encoded
                d = dict(g=g, m_new=m_new.numpy().copy(),
                         alpha=np.array([float(mgr._alpha)], np.float32),
                         labels=enc["labels"].numpy().copy(),
                         signs=enc["sign_packed"].numpy().copy(),
                         norms=enc["block_norms"].numpy().copy(),
                         amp=h16(enc["scales"]), ratios=rec["ratios"], tau=rec["tau"])
                if ef:
                    d["ef_residual"] = mgr._ef_residual.numpy().copy()
                for k, v in d.items():
                    cases[f"{key}_s{s}_{k}"] = v
            cases[f"{key}_meta"] = np.array([n, nsteps], np.int64)
            cases[f"{key}_pct"] = np.array([lo, hi], np.float64)
    finally:
        costate.compute_thresholds = orig_thr
    cases["n_cases"] = np.array([len(specs)], np.int64)
    name = "costate_ef.npz" if ef else "costate.npz"
    np.savez_compressed(os.path.join(out_dir, name), **cases)
    print(name, "cases:", len(specs))


# ---------------------------------------------------------------------------
# C. Whole TurboAdam.step runs (optimizer.py:88-292)
# ---------------------------------------------------------------------------

RUNS = {
    # name: (list of (shape, dtype, group), group kwargs list, steps, grad_none)
    "block": (
        [((64, 64), "f32", 0), ((96, 50), "f32", 0), ((128,), "f32", 0), ((33,), "f32", 0)],
        [dict(lr=6e-4, betas=(0.9, 0.999), weight_decay=0.01, v_bits=4)],
        5, {},
    ),
    "groups": (
        [((64, 80), "f32", 0), ((70,), "f32", 0), ((50, 90), "f32", 1), ((4500,), "f32", 2),
         ((20,), "f32", 2)],
        [dict(lr=1e-3, weight_decay=0.0, v_bits=3),
         dict(lr=3e-4, weight_decay=0.05, v_bits=8, compress_m=False),
         dict(lr=2e-3, weight_decay=0.1, v_bits=6, compress_v=False)],
        5, {},
    ),
    "bf16": (
        [((64, 64), "bf16", 0), ((40,), "bf16", 0), ((4099,), "bf16", 0)],
        [dict(lr=1e-3, weight_decay=0.01, v_bits=3)],
        4, {},
    ),
    "gradnone": (
        [((4096,), "f32", 0), ((130,), "f32", 0), ((4200,), "f32", 0)],
        [dict(lr=1e-3, weight_decay=0.02, v_bits=2, min_m_compress_elements=4100)],
        5, {(2, 1), (3, 0)},  # (step, param) pairs with grad None
    ),
    "ef": (
        [((64, 80), "f32", 0), ((4133,), "f32", 0), ((90,), "f32", 0), ((48, 100), "f32", 1)],
        [dict(lr=1e-3, weight_decay=0.01, v_bits=4, error_feedback=True),
         dict(lr=5e-4, weight_decay=0.0, v_bits=3, error_feedback=True, compress_v=False)],
        5, {(2, 1)},
    ),
}


def gen_optimizer_runs(mods, out_dir):
    turboadam, _, _, _, _ = mods
    TurboAdam = turboadam.TurboAdam
    feed = UniformFeed()
    for name, (pspecs, gkw, nsteps, none_set) in RUNS.items():
        rng = np.random.default_rng(zlib.crc32(name.encode()))
        params = []
        data = {}
        for pi, (shape, dt, gi) in enumerate(pspecs):
            init = (rng.standard_normal(shape) * 0.02).astype(np.float32)
            t = torch.from_numpy(init)
            if dt == "bf16":
                t = t.to(torch.bfloat16)
            p = torch.nn.Parameter(t)
            params.append(p)
            data[f"p{pi}_init"] = bf16_bits(p.data) if dt == "bf16" else p.data.numpy().copy()
        groups = []
        for gi, kw in enumerate(gkw):
            groups.append(dict(params=[params[i] for i, s in enumerate(pspecs) if s[2] == gi],
                               **kw))
        opt = TurboAdam(groups)
        for s in range(nsteps):
            for pi, p in enumerate(params):
                if (s, pi) in none_set:
                    p.grad = None
                    continue
                g = (rng.standard_normal(p.shape) * 10.0 ** rng.uniform(-4, -2)).astype(np.float32)
                gt = torch.from_numpy(g)
                if pspecs[pi][1] == "bf16":
                    gt = gt.to(torch.bfloat16)
                    data[f"s{s}_g{pi}"] = bf16_bits(gt)
                else:
                    data[f"s{s}_g{pi}"] = g
                p.grad = gt
            # uniforms: one draw per compress_v param with grad, in step order
            for pi, p in enumerate(params):
                if p.grad is None:
                    continue
                grp = next(g for g in opt.param_groups if any(q is p for q in g["params"]))
                if not grp["compress_v"]:
                    continue
                B = (p.numel() + 127) // 128
                u = rng.random(B * 128).astype(np.float32)
                feed.push(u)
                data[f"s{s}_u{pi}"] = u
            with feed.active():
                opt.step()
            for pi, p in enumerate(params):
                st = opt.state.get(p, {})
                if not st:
                    continue
                data[f"s{s}_p{pi}"] = (bf16_bits(p.data) if pspecs[pi][1] == "bf16"
                                       else p.data.numpy().copy())
                data[f"s{s}_step{pi}"] = np.array([st["step"]], np.int64)
                if "compressed_v" in st:
                    data[f"s{s}_vidx{pi}"] = st["compressed_v"]["indices"].numpy().copy()
                    data[f"s{s}_vhdr{pi}"] = h16(st["compressed_v"]["scales"])
                if "exp_avg" in st:
                    data[f"s{s}_m{pi}"] = st["exp_avg"].numpy().copy()
                if "exp_avg_sq" in st:
                    data[f"s{s}_vsq{pi}"] = st["exp_avg_sq"].numpy().copy()
                if "m_mgr" in st:
                    mg = st["m_mgr"]
                    if mg._ef_residual is not None:
                        data[f"s{s}_ef{pi}"] = mg._ef_residual.numpy().copy()
                    data[f"s{s}_alpha{pi}"] = np.array([float(mg._alpha)], np.float32)
                    data[f"s{s}_labels{pi}"] = mg._encoded["labels"].numpy().copy()
                    data[f"s{s}_signs{pi}"] = mg._encoded["sign_packed"].numpy().copy()
                    data[f"s{s}_norms{pi}"] = mg._encoded["block_norms"].numpy().copy()
                    data[f"s{s}_amp{pi}"] = h16(mg._encoded["scales"])
        data["meta_nsteps"] = np.array([nsteps], np.int64)
        np.savez_compressed(os.path.join(out_dir, f"opt_{name}.npz"), **data)
        print("optimizer run:", name)


# ---------------------------------------------------------------------------
# D. A reference checkpoint and its continuation (optimizer.py:194-218)
# ---------------------------------------------------------------------------

CKPT_SPEC = (
    [((64, 64), 0), ((96, 50), 0), ((130,), 0), ((4133,), 1), ((80, 64), 1)],
    [dict(lr=6e-4, betas=(0.9, 0.999), weight_decay=0.01, v_bits=4),
     dict(lr=1e-3, weight_decay=0.0, v_bits=3, error_feedback=True)],
    3, 2,  # steps before the checkpoint, steps after it
)


def gen_checkpoint_run(mods, out_dir):
    """torch.save of the reference optimizer's state_dict() after 3 steps
    (ref_ckpt.pt: pickled turboadam.costate.CoStateManager objects), then the
    reference's next 2 steps from that state (ckpt_cont.npz: gradients,
    uniforms, alpha and every output), all with injected uniforms."""
    turboadam, _, _, _, _ = mods
    pspecs, gkw, n_before, n_after = CKPT_SPEC
    rng = np.random.default_rng(777)
    feed = UniformFeed()
    params = [torch.nn.Parameter(torch.from_numpy(
        (rng.standard_normal(shape) * 0.02).astype(np.float32))) for shape, _ in pspecs]
    groups = [dict(params=[params[i] for i, s in enumerate(pspecs) if s[1] == gi], **kw)
              for gi, kw in enumerate(gkw)]
    opt = turboadam.TurboAdam(groups)
    order = [i for gi in range(len(gkw)) for i, s in enumerate(pspecs) if s[1] == gi]
    data = {}

    def one_step(s, record):
        for pi, p in enumerate(params):
            g = (rng.standard_normal(p.shape) * 10.0 ** rng.uniform(-4, -2)).astype(np.float32)
            p.grad = torch.from_numpy(g)
            if record:
                data[f"s{s}_g{pi}"] = g
        for pi in order:  # the reference draws in step (group, param) order
            B = (params[pi].numel() + 127) // 128
            u = rng.random(B * 128).astype(np.float32)
            feed.push(u)
            if record:
                data[f"s{s}_u{pi}"] = u
        with feed.active():
            opt.step()

    for s in range(n_before):
        one_step(s, False)
    torch.save(opt.state_dict(), os.path.join(out_dir, "ref_ckpt.pt"))
    for pi, p in enumerate(params):
        data[f"p{pi}_ckpt"] = p.data.numpy().copy()
    for s in range(n_after):
        one_step(s, True)
        for pi, p in enumerate(params):
            st = opt.state[p]
            data[f"s{s}_p{pi}"] = p.data.numpy().copy()
            data[f"s{s}_step{pi}"] = np.array([st["step"]], np.int64)
            data[f"s{s}_vidx{pi}"] = st["compressed_v"]["indices"].numpy().copy()
            data[f"s{s}_vhdr{pi}"] = h16(st["compressed_v"]["scales"])
            if "exp_avg" in st:
                data[f"s{s}_m{pi}"] = st["exp_avg"].numpy().copy()
            if "m_mgr" in st:
                mg = st["m_mgr"]
                data[f"s{s}_alpha{pi}"] = np.array([float(mg._alpha)], np.float32)
                data[f"s{s}_labels{pi}"] = mg._encoded["labels"].numpy().copy()
                data[f"s{s}_signs{pi}"] = mg._encoded["sign_packed"].numpy().copy()
                data[f"s{s}_norms{pi}"] = mg._encoded["block_norms"].numpy().copy()
                data[f"s{s}_amp{pi}"] = h16(mg._encoded["scales"])
                if mg._ef_residual is not None:
                    data[f"s{s}_ef{pi}"] = mg._ef_residual.numpy().copy()
    np.savez_compressed(os.path.join(out_dir, "ckpt_cont.npz"), **data)
    print("checkpoint run: ref_ckpt.pt + ckpt_cont.npz")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("TURBOADAM_REF"),
                    help="checkout of the reference repository (or set TURBOADAM_REF)")
    ap.add_argument("--out", default=os.path.dirname(os.path.abspath(__file__)))
    ap.add_argument("--only", nargs="*", default=None,
                    help="generate only these sets (v, v_decode, costate, costate_ef, runs, "
                         "checkpoint)")
    a = ap.parse_args()
    if not a.ref:
        ap.error("--ref (or TURBOADAM_REF) must name the reference checkout")
    torch.set_num_threads(1)
    mods = _import_reference(a.ref)
    sets = {
        "v": lambda: gen_v_cases(mods, a.out),
        "v_decode": lambda: gen_v_decode_cases(mods, a.out),
        "costate": lambda: gen_costate_cases(mods, a.out),
        "costate_ef": lambda: gen_costate_cases(mods, a.out, ef=True),
        "runs": lambda: gen_optimizer_runs(mods, a.out),
        "checkpoint": lambda: gen_checkpoint_run(mods, a.out),
    }
    for name, fn in sets.items():
        if a.only is None or name in a.only:
            fn()


if __name__ == "__main__":
    main()
