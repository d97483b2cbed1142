"""CPU checker for the TurboAdam step -- TEST INFRASTRUCTURE ONLY.

ctypes wrapper around ``oracle/_build/libta_oracle.so`` (built from
``oracle/ta_oracle.c`` by ``oracle/Makefile``) plus a numpy replay of
``TurboAdam.step`` (reference ``src/turboadam/optimizer.py:88-292``).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of
``bench.py`` import this module. The product package never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libta_oracle.so")
_lib = None

BLOCK_SIZE = 128


def build() -> str:
    """Compile the checker library (gcc, seconds)."""
    subprocess.check_call(["make", "-s", "-C", _HERE])
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_D = ctypes.c_double
_F = ctypes.c_float
_U32 = ctypes.c_uint32
_U64 = ctypes.c_uint64


def _declare(L):
    sig = {
        "orc_v_init": (None, [_I64, _I, _P, _P]),
        "orc_v_update": (None, [_P, _P, _P, _I64, _I, _I, _D, _P, _P, _P, _P]),
        "orc_v_decode": (None, [_P, _P, _I64, _I, _I, _P]),
        "orc_block_ratios": (None, [_P, _P, _I64, _I, _P, _P]),
        "orc_threshold_ranks": (None, [_I64, _D, _D, _P, _P]),
        "orc_thresholds": (None, [_P, _I64, _D, _D, _P, _P]),
        "orc_classify": (None, [_P, _I64, _F, _F, _P]),
        "orc_encode": (None, [_P, _I64, _I, _P, _P, _P]),
        "orc_decode": (None, [_P, _P, _P, _P, _F, _P, _I64, _I, _P]),
        "orc_alpha": (_F, [_P, _P, _I64, _I]),
        "orc_costate_update": (
            None,
            [_P, _P, _P, _P, _F, _I, _P, _I64, _I, _D, _D, _D, _P, _P, _P, _P, _P, _P, _I],
        ),
        "orc_weight_decay": (None, [_P, _I, _I64, _D, _D]),
        "orc_exp_avg": (None, [_P, _P, _I64, _D]),
        "orc_exp_avg_sq": (None, [_P, _P, _I64, _D]),
        "orc_adam_apply": (None, [_P, _I, _P, _P, _I64, _D, _D, _F, _F]),
        "orc_sr_uniforms": (None, [_I64, _I, _U32, _U32, _U64, _P]),
        "orc_sr_uniforms_at": (None, [_I64, _I64, _I, _U32, _U32, _U64, _P]),
        "orc_philox": (None, [_U32, _U32, _U32, _U32, _U32, _U32, _P]),
        "orc_logf_array": (None, [_P, _I64, _P]),
        "orc_logf_fast_array": (None, [_P, _I64, _P]),
        "orc_expf_array": (None, [_P, _I64, _P]),
        "orc_f32_to_f16_array": (None, [_P, _I64, _P]),
        "orc_scan_log": (_D, [_U32, _U32, _P]),
        "orc_scan_exp": (_D, [_U32, _U32, _P]),
        "orc_threads": (_I, []),
        "orc_set_threads": (None, [_I]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def n_blocks(n: int, bs: int = BLOCK_SIZE) -> int:
    return (n + bs - 1) // bs


# ---------------------------------------------------------------------------
# Primitive wrappers
# ---------------------------------------------------------------------------


def v_init(n: int, bs: int = BLOCK_SIZE):
    B = n_blocks(n, bs)
    idx = np.zeros(B * bs, np.uint8)
    hdr = np.zeros(B * 2, np.uint16)
    lib().orc_v_init(B, bs, _ptr(idx), _ptr(hdr))
    return idx, hdr


def v_update(idx, hdr, g, nbits, beta2, u, bs: int = BLOCK_SIZE):
    """quantize.py:222-299. Returns (new_idx, new_hdr_bits, v_new)."""
    g = np.ascontiguousarray(g, np.float32).reshape(-1)
    n = g.size
    B = n_blocks(n, bs)
    idx = np.ascontiguousarray(idx, np.uint8)
    hdr = np.ascontiguousarray(hdr, np.uint16).reshape(-1)
    u = np.ascontiguousarray(u, np.float32).reshape(-1)
    assert idx.size == B * bs and hdr.size == 2 * B and u.size == B * bs
    oi = np.empty(B * bs, np.uint8)
    oh = np.empty(2 * B, np.uint16)
    v = np.empty(n, np.float32)
    lib().orc_v_update(_ptr(idx), _ptr(hdr), _ptr(g), n, bs, nbits, float(beta2), _ptr(u),
                       _ptr(oi), _ptr(oh), _ptr(v))
    return oi, oh, v


def v_decode(idx, hdr, n, nbits, bs: int = BLOCK_SIZE):
    v = np.empty(n, np.float32)
    lib().orc_v_decode(_ptr(np.ascontiguousarray(idx, np.uint8)),
                       _ptr(np.ascontiguousarray(hdr, np.uint16).reshape(-1)), n, bs, nbits,
                       _ptr(v))
    return v


def threshold_ranks(B: int, null_pct: float, amp_pct: float):
    lo = ctypes.c_int64()
    hi = ctypes.c_int64()
    lib().orc_threshold_ranks(B, float(null_pct), float(amp_pct), ctypes.byref(lo),
                              ctypes.byref(hi))
    return lo.value, hi.value


def alpha(m, g, bs: int = BLOCK_SIZE) -> float:
    m = np.ascontiguousarray(m, np.float32).reshape(-1)
    g = np.ascontiguousarray(g, np.float32).reshape(-1)
    return lib().orc_alpha(_ptr(m), _ptr(g), m.size, bs)


def sr_uniforms(n: int, tensor_id: int, step: int, seed: int, bs: int = BLOCK_SIZE):
    B = n_blocks(n, bs)
    u = np.empty(B * bs, np.float32)
    lib().orc_sr_uniforms(B, bs, tensor_id & 0xFFFFFFFF, step & 0xFFFFFFFF,
                          seed & 0xFFFFFFFFFFFFFFFF, _ptr(u))
    return u


def sr_uniforms_at(b0: int, n_blocks: int, tensor_id: int, step: int, seed: int,
                   bs: int = BLOCK_SIZE):
    """The draws of blocks b0 .. b0 + n_blocks - 1 of a tensor (a slice)."""
    u = np.empty(n_blocks * bs, np.float32)
    lib().orc_sr_uniforms_at(int(b0), int(n_blocks), bs, tensor_id & 0xFFFFFFFF,
                             step & 0xFFFFFFFF, seed & 0xFFFFFFFFFFFFFFFF, _ptr(u))
    return u


def costate_decode(labels, signs, norms, amp_bits, alpha, g, bs: int = BLOCK_SIZE):
    """decode_blocks (costate.py:261-323): m_hat = alpha g + scale sign."""
    g = np.ascontiguousarray(g, np.float32).reshape(-1)
    out = np.empty(g.size, np.float32)
    lib().orc_decode(_ptr(np.ascontiguousarray(labels, np.uint8)),
                     _ptr(np.ascontiguousarray(signs, np.uint8)),
                     _ptr(np.ascontiguousarray(norms, np.float32)),
                     _ptr(np.ascontiguousarray(amp_bits, np.uint16)), float(alpha), _ptr(g),
                     g.size, bs, _ptr(out))
    return out


def costate_encode(delta, bs: int = BLOCK_SIZE):
    """encode_blocks (costate.py:213-258): (MSB-first sign bytes, block norms,
    fp16 scale bits)."""
    d = np.ascontiguousarray(delta, np.float32).reshape(-1)
    B = n_blocks(d.size, bs)
    signs = np.zeros((d.size + 7) // 8, np.uint8)
    norms = np.empty(B, np.float32)
    amp = np.empty(B, np.uint16)
    lib().orc_encode(_ptr(d), d.size, bs, _ptr(signs), _ptr(norms), _ptr(amp))
    return signs, norms, amp


def threads() -> int:
    return int(lib().orc_threads())


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def philox(ctr, key):
    out = np.empty(4, np.uint32)
    lib().orc_philox(*[int(c) for c in ctr], *[int(k) for k in key], _ptr(out))
    return out


def logf(x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().orc_logf_array(_ptr(x), x.size, _ptr(y))
    return y


def logf_fast(x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().orc_logf_fast_array(_ptr(x), x.size, _ptr(y))
    return y


def expf(x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().orc_expf_array(_ptr(x), x.size, _ptr(y))
    return y


def f32_to_f16_bits(x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_f16_array(_ptr(x), x.size, _ptr(y))
    return y


def scan_log(lo: int, hi: int):
    bad = ctypes.c_int64()
    me = lib().orc_scan_log(lo, hi, ctypes.byref(bad))
    return me, bad.value


def scan_exp(lo: int, hi: int):
    bad = ctypes.c_int64()
    me = lib().orc_scan_exp(lo, hi, ctypes.byref(bad))
    return me, bad.value


# ---------------------------------------------------------------------------
# CoState
# ---------------------------------------------------------------------------


@dataclass
class CoStateOracle:
    """State of reference CoStateManager (costate.py:350-365)."""

    n: int
    bs: int = BLOCK_SIZE
    null_pct: float = 0.10
    amp_pct: float = 0.90
    has_state: bool = False
    alpha: float = 0.0
    labels: np.ndarray = None
    signs: np.ndarray = None
    norms: np.ndarray = None
    amp: np.ndarray = None  # fp16 bits
    last_ratios: np.ndarray = None
    last_tau: np.ndarray = None
    error_feedback: bool = False
    ef_residual: np.ndarray = None  # fp32 [n] once the first step has run

    def __post_init__(self):
        B = n_blocks(self.n, self.bs)
        self.labels = np.zeros(B, np.uint8)
        self.signs = np.zeros((self.n + 7) // 8, np.uint8)
        self.norms = np.zeros(B, np.float32)
        self.amp = np.zeros(B, np.uint16)

    def update(self, g, beta1, alpha_inject=None):
        """costate.py:367-464. Returns m_new."""
        g = np.ascontiguousarray(g, np.float32).reshape(-1)
        B = n_blocks(self.n, self.bs)
        m_new = np.empty(self.n, np.float32)
        a_out = np.zeros(1, np.float32)
        ratios = np.empty(B, np.float32)
        tau = np.empty(2, np.float32)
        inj = None
        if alpha_inject is not None:
            inj_arr = np.array([alpha_inject], np.float32)
            inj = _ptr(inj_arr)
        ef_mode = 0
        if self.error_feedback:
            ef_mode = 2 if self.ef_residual is not None else 1
            if self.ef_residual is None:
                self.ef_residual = np.zeros(self.n, np.float32)
        lib().orc_costate_update(
            _ptr(self.labels), _ptr(self.signs), _ptr(self.norms), _ptr(self.amp),
            float(self.alpha), int(self.has_state), _ptr(g), self.n, self.bs, float(beta1),
            float(self.null_pct), float(self.amp_pct), inj, _ptr(m_new), _ptr(a_out),
            _ptr(ratios), _ptr(tau), _ptr(self.ef_residual) if ef_mode else None, ef_mode)
        self.alpha = float(a_out[0])
        self.has_state = True
        self.last_ratios = ratios
        self.last_tau = tau
        return m_new


# ---------------------------------------------------------------------------
# Whole optimizer step (optimizer.py:88-292)
# ---------------------------------------------------------------------------


@dataclass
class ParamState:
    step: int = 0
    compress_m: bool = False
    mgr: CoStateOracle = None
    exp_avg: np.ndarray = None
    exp_avg_sq: np.ndarray = None
    v_idx: np.ndarray = None
    v_hdr: np.ndarray = None
    group: int = 0


@dataclass
class OracleParam:
    """A parameter: flat data (fp32 array, or uint16 bf16 bits) + shape."""

    data: np.ndarray
    bf16: bool = False
    grad: np.ndarray = None  # fp32 view of the gradient (bf16 grads widened)

    @property
    def n(self):
        return self.data.size


@dataclass
class OracleTurboAdam:
    """numpy replay of TurboAdam.step on flat arrays.

    ``uniforms(param_index, step, n_padded)`` supplies the stochastic-rounding
    draws; ``alpha_inject(param_index, step)`` may return an alpha replacing the
    canonical reduction (reference-parity mode) or None.
    """

    groups: list  # list of dicts: params (list[OracleParam]), lr, betas, eps, ...
    state: dict = field(default_factory=dict)

    @staticmethod
    def make_group(params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0,
                   block_size=128, v_bits=4, compress_m=True, compress_v=True, null_pct=0.10,
                   amp_pct=0.90, min_m_compress_elements=4096, error_feedback=False):
        return dict(params=list(params), lr=lr, betas=betas, eps=eps,
                    weight_decay=weight_decay, block_size=block_size, v_bits=v_bits,
                    compress_m=compress_m, compress_v=compress_v, null_pct=null_pct,
                    amp_pct=amp_pct, min_m_compress_elements=min_m_compress_elements,
                    error_feedback=error_feedback)

    def step(self, uniforms, alpha_inject=lambda i, s: None):
        pid = 0
        index = {}
        for gi, group in enumerate(self.groups):
            for p in group["params"]:
                index[id(p)] = pid
                pid += 1
        # lazy init (optimizer.py:232-286)
        for gi, group in enumerate(self.groups):
            bs = group["block_size"]
            for p in group["params"]:
                if p.grad is None:
                    continue
                st = self.state.get(id(p))
                if st is None:
                    st = ParamState(group=gi)
                    st.compress_m = bool(group["compress_m"]
                                         and p.n >= group["min_m_compress_elements"])
                    if st.compress_m:
                        st.mgr = CoStateOracle(p.n, bs, group["null_pct"], group["amp_pct"],
                                               error_feedback=bool(group.get("error_feedback")))
                    else:
                        st.exp_avg = np.zeros(p.n, np.float32)
                    if not group["compress_v"]:
                        st.exp_avg_sq = np.zeros(p.n, np.float32)
                    self.state[id(p)] = st
                if group["compress_v"] and st.v_idx is None:
                    st.v_idx, st.v_hdr = v_init(p.n, bs)
        # bias corrections, last param with state wins (optimizer.py:172-188)
        bcs = {}
        for gi, group in enumerate(self.groups):
            b1, b2 = group["betas"]
            for p in group["params"]:
                st = self.state.get(id(p))
                if st is None:
                    continue
                nxt = st.step + 1
                bcs[gi] = (np.float32(1.0 - b1 ** nxt), np.float32(1.0 - b2 ** nxt))
        # per-param step (optimizer.py:88-170)
        for gi, group in enumerate(self.groups):
            lr = group["lr"]
            b1, b2 = group["betas"]
            for p in group["params"]:
                if p.grad is None:
                    continue
                st = self.state[id(p)]
                st.step += 1
                i = index[id(p)]
                g = np.ascontiguousarray(p.grad, np.float32).reshape(-1)
                lib().orc_weight_decay(_ptr(p.data), int(p.bf16), p.n, float(lr),
                                       float(group["weight_decay"]))
                if st.compress_m:
                    m_new = st.mgr.update(g, b1, alpha_inject(i, st.step))
                else:
                    lib().orc_exp_avg(_ptr(st.exp_avg), _ptr(g), p.n, float(b1))
                    m_new = st.exp_avg
                bc1, bc2 = bcs[gi]
                if group["compress_v"]:
                    bs = group["block_size"]
                    u = uniforms(i, st.step, n_blocks(p.n, bs) * bs)
                    st.v_idx, st.v_hdr, v = v_update(st.v_idx, st.v_hdr, g,
                                                     group["v_bits"], b2, u, bs)
                else:
                    lib().orc_exp_avg_sq(_ptr(st.exp_avg_sq), _ptr(g), p.n, float(b2))
                    v = st.exp_avg_sq
                lib().orc_adam_apply(_ptr(p.data), int(p.bf16), _ptr(m_new), _ptr(v), p.n,
                                     float(lr), float(group["eps"]), float(bc1), float(bc2))
