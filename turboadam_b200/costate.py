"""CoState first-moment state and its device seams.

Mirrors reference ``src/turboadam/costate.py``: ``CoStateManager`` keeps the
same attribute names (``block_size, _null_pct, _amp_pct, _has_state, _alpha,
_encoded{labels, sign_packed, block_norms, scales}, _original_numel,
_error_feedback, _ef_residual``) so optimizer state dicts have the reference
shape. The tensors in ``_encoded`` are views of device buffers padded to whole
16-block tiles (the layout the fused kernels stream).

``decode_blocks`` / ``encode_blocks`` / ``compute_thresholds`` /
``CoStateManager.update`` run the sm_100a kernels through the C ABI; they take
CUDA tensors only.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from .utils import BLOCK_SIZE


def _n_blocks(n: int, bs: int) -> int:
    return (n + bs - 1) // bs


def padded_blocks(n: int, bs: int = BLOCK_SIZE) -> int:
    return int(_lib.load().ta_state_padded_blocks(n, bs))


class CoStateManager:
    """Per-tensor CoState state (reference costate.py:332-464).

    Device buffers are created by :meth:`allocate`; until the first update
    ``_has_state`` is False and ``_encoded`` is None, as in the reference.
    """

    def __init__(self, block_size: int = BLOCK_SIZE, error_feedback: bool = False,
                 null_pct: float = 0.10, amp_pct: float = 0.90) -> None:
        self.block_size = block_size
        self._null_pct = null_pct
        self._amp_pct = amp_pct
        self._has_state = False
        self._alpha = 0.0
        self._encoded = None
        self._original_numel = 0
        self._error_feedback = error_feedback
        self._ef_residual = None
        self._bufs = None  # padded device buffers

    @classmethod
    def from_reference(cls, obj) -> "CoStateManager":
        """A manager holding the state of another object with the reference's
        CoStateManager attributes (costate.py:350-365) -- the reference's own
        class, when a checkpoint was loaded with the reference installed, or
        the stand-in of ``checkpoint.load_reference_state_dict``. The tensors
        move to the device on :meth:`adopt`."""
        mgr = cls(block_size=int(getattr(obj, "block_size", BLOCK_SIZE)),
                  error_feedback=bool(getattr(obj, "_error_feedback", False)),
                  null_pct=float(getattr(obj, "_null_pct", 0.10)),
                  amp_pct=float(getattr(obj, "_amp_pct", 0.90)))
        mgr._has_state = bool(getattr(obj, "_has_state", False))
        mgr._alpha = getattr(obj, "_alpha", 0.0)
        enc = getattr(obj, "_encoded", None)
        mgr._encoded = None if enc is None else dict(enc)
        mgr._original_numel = int(getattr(obj, "_original_numel", 0))
        mgr._ef_residual = getattr(obj, "_ef_residual", None)
        return mgr

    # -- storage ---------------------------------------------------------
    def allocate(self, n: int, device, shape=None) -> None:
        bs = self.block_size
        B = _n_blocks(n, bs)
        P = padded_blocks(n, bs)
        z = dict(device=device)
        self._bufs = {
            "labels": torch.zeros(P, dtype=torch.uint8, **z),
            "sign_packed": torch.zeros(P * bs // 8, dtype=torch.uint8, **z),
            "block_norms": torch.zeros(P, dtype=torch.float32, **z),
            "scales": torch.zeros(P, dtype=torch.float16, **z),
            "alpha": torch.zeros(1, dtype=torch.float32, **z),
        }
        if self._error_feedback:  # the residual (costate.py:428-437), fp32 like g
            self._bufs["ef"] = torch.zeros(n, dtype=torch.float32, **z)
        self._n = n
        self._B = B
        self._shape = tuple(shape) if shape is not None else (n,)

    def _views(self):
        b = self._bufs
        return {
            "labels": b["labels"][: self._B],
            "sign_packed": b["sign_packed"][: (self._n + 7) // 8],
            "block_norms": b["block_norms"][: self._B],
            "scales": b["scales"][: self._B],
        }

    def mark_updated(self) -> None:
        """Expose the device state under the reference attribute names."""
        if self._encoded is None:
            self._encoded = self._views()
            self._alpha = self._bufs["alpha"].view(())
        if self._error_feedback and self._ef_residual is None:
            # the reference keeps the residual in the gradient's shape
            self._ef_residual = self._bufs["ef"].view(self._shape)
        self._original_numel = self._n
        self._has_state = True

    def ef_pointer(self) -> int:
        """Device address of the error-feedback residual buffer (0 without)."""
        ef = self._bufs.get("ef") if self._bufs else None
        return ef.data_ptr() if ef is not None else 0

    def pointers(self):
        b = self._bufs
        return (b["labels"].data_ptr(), b["sign_packed"].data_ptr(), b["block_norms"].data_ptr(),
                b["scales"].data_ptr(), b["alpha"].data_ptr())

    def adopt(self, n: int, device, shape=None) -> None:
        """Re-home loaded state (any dtype/device, unpadded) into padded buffers."""
        enc = self._encoded
        alpha = self._alpha
        ef = getattr(self, "_ef_residual", None)
        self._ef_residual = None
        self.allocate(n, device, shape)
        if ef is not None and self._error_feedback:
            self._bufs["ef"].copy_(ef.reshape(-1).to(device=device, dtype=torch.float32))
            self._ef_residual = self._bufs["ef"].view(self._shape)
        if enc is not None:
            for k, v in self._views().items():
                src = enc[k].reshape(-1).to(device=device)
                v.copy_(src.to(v.dtype))
            a = alpha if isinstance(alpha, torch.Tensor) else torch.tensor(float(alpha))
            self._bufs["alpha"].copy_(a.reshape(1).to(device=device, dtype=torch.float32))
            self._encoded = None
            self.mark_updated()

    # -- reference API ----------------------------------------------------
    def update(self, g: torch.Tensor, beta1: float) -> torch.Tensor:
        """One CoState step (costate.py:367-464); returns fp32 m_new."""
        from .optimizer import _single_costate_update

        return _single_costate_update(self, g, beta1)


# ---------------------------------------------------------------------------
# Functional seams (costate.py:213-323, :94-149)
# ---------------------------------------------------------------------------


def decode_blocks(encoded: dict, alpha, g: torch.Tensor, block_size: int = BLOCK_SIZE,
                  original_numel: int | None = None) -> torch.Tensor:
    """m_hat = alpha*g + delta_hat (costate.py:261-323) on the device."""
    _lib.require_cuda(g)
    lib = _lib.load()
    n = g.numel() if original_numel is None else original_numel
    dev = g.device
    gf = g.reshape(-1).contiguous()
    if gf.dtype not in (torch.float32, torch.bfloat16):
        gf = gf.float()
    lab = encoded["labels"].to(device=dev, dtype=torch.uint8).contiguous()
    sgn = encoded["sign_packed"].to(device=dev, dtype=torch.uint8).contiguous()
    nrm = encoded["block_norms"].to(device=dev, dtype=torch.float32).contiguous()
    amp = encoded["scales"].to(device=dev, dtype=torch.float16).contiguous()
    a = alpha if isinstance(alpha, torch.Tensor) else torch.tensor(float(alpha))
    a = a.reshape(1).to(device=dev, dtype=torch.float32).contiguous()
    out = torch.empty(n, dtype=torch.float32, device=dev)
    _lib.check(lib.ta_costate_decode(lab.data_ptr(), sgn.data_ptr(), nrm.data_ptr(),
                                     amp.data_ptr(), a.data_ptr(), gf.data_ptr(),
                                     _lib.TA_BF16 if gf.dtype == torch.bfloat16 else _lib.TA_F32,
                                     n, block_size, out.data_ptr(), _lib.stream_ptr(dev)),
               "ta_costate_decode")
    return out.reshape(g.shape)


def encode_blocks(delta: torch.Tensor, labels: torch.Tensor,
                  block_size: int = BLOCK_SIZE) -> dict:
    """Block norms, fp16 scales, MSB-first signs (costate.py:213-258)."""
    _lib.require_cuda(delta)
    lib = _lib.load()
    d = delta.reshape(-1).float().contiguous()
    n = d.numel()
    B = _n_blocks(n, block_size)
    dev = d.device
    sgn = torch.zeros((n + 7) // 8, dtype=torch.uint8, device=dev)
    nrm = torch.empty(B, dtype=torch.float32, device=dev)
    amp = torch.empty(B, dtype=torch.float16, device=dev)
    _lib.check(lib.ta_costate_encode(d.data_ptr(), n, block_size, sgn.data_ptr(), nrm.data_ptr(),
                                     amp.data_ptr(), _lib.stream_ptr(dev)), "ta_costate_encode")
    return {"labels": labels, "sign_packed": sgn, "block_norms": nrm, "scales": amp}


def compute_thresholds(ratios: torch.Tensor, null_pct: float = 0.10, amp_pct: float = 0.90):
    """(tau0, tau1) as 0-dim device tensors (costate.py:94-118), exact."""
    tau, _ = _select(ratios, null_pct, amp_pct, want_labels=False)
    return tau[0], tau[1]


def classify_with_thresholds(ratios: torch.Tensor, null_pct: float = 0.10,
                             amp_pct: float = 0.90):
    """compute_thresholds followed by classify_blocks (costate.py:126-149)."""
    tau, labels = _select(ratios, null_pct, amp_pct, want_labels=True)
    return tau, labels


def _select(ratios, null_pct, amp_pct, want_labels):
    _lib.require_cuda(ratios)
    lib = _lib.load()
    r = ratios.reshape(-1).float().contiguous()
    B = r.numel()
    dev = r.device
    ws = torch.zeros(lib.ta_aux_workspace_size(B * BLOCK_SIZE), dtype=torch.uint8, device=dev)
    tau = torch.empty(2, dtype=torch.float32, device=dev)
    labels = torch.empty(B, dtype=torch.uint8, device=dev) if want_labels else None
    _lib.check(lib.ta_thresholds(r.data_ptr(), B, float(null_pct), float(amp_pct),
                                 tau.data_ptr(), labels.data_ptr() if want_labels else None,
                                 ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev)),
               "ta_thresholds")
    return tau, labels


def sqrt_block(block_size: int = BLOCK_SIZE) -> float:
    return math.sqrt(block_size)

