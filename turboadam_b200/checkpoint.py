"""Checkpoint format of the packed optimizer state.

``TurboAdam.state_dict()`` already has the reference's keys, dtypes and
shapes (views of the padded device buffers), and ``load_state_dict`` adopts a
reference checkpoint. This module adds the on-disk forms:

* ``load_reference_state_dict(f)``: reads a ``torch.save``'d state dict of the
  reference optimizer without the reference package installed (its
  ``turboadam.costate.CoStateManager`` objects unpickle as a plain stand-in
  with the same attributes, which ``TurboAdam.load_state_dict`` converts);

* ``portable_state_dict(opt, pack=False)``: compact tensors (no tile padding),
  each ``CoStateManager`` replaced by a plain dict (so the file loads without
  this package), the stochastic-rounding seed included so a resumed run
  continues bit for bit, and -- with ``pack=True`` -- the 1Q indices stored
  densely at n bits each (``pack_indices``) instead of one byte each.
* ``load_portable_state_dict(opt, sd)``: the inverse.

Dense packing: index e of a tensor occupies bits [e*n, e*n + n) of the byte
stream, least significant bit first (byte k holds bits 8k..8k+7).
"""
from __future__ import annotations

import copy

import numpy as np
import torch

from .costate import CoStateManager
from .oneq import adopt_compressed_v

FORMAT = "turboadam_b200/portable-1"


class ReferenceCoStateManager:
    """What a pickled reference ``turboadam.costate.CoStateManager`` loads as
    without the reference installed: an attribute bag with the reference's
    attribute names (costate.py:350-365); ``TurboAdam.load_state_dict``
    turns it into this package's manager."""

    def __setstate__(self, state):
        self.__dict__.update(state)


# classes of the reference package that an optimizer state dict may hold
_REFERENCE_CLASSES = {("turboadam.costate", "CoStateManager"): ReferenceCoStateManager}


def load_reference_state_dict(f, map_location="cpu"):
    """``torch.load`` of a reference TurboAdam ``state_dict()`` (a path or a
    file object) that does not need the reference package: its
    CoStateManager objects come back as :class:`ReferenceCoStateManager`.
    Any other class of the reference package is refused. Like
    ``torch.load(weights_only=False)`` this unpickles general Python objects:
    load only checkpoints you trust."""
    import pickle
    import types

    class _Unpickler(pickle.Unpickler):
        def find_class(self, module, name):
            if module == "turboadam" or module.startswith("turboadam."):
                cls = _REFERENCE_CLASSES.get((module, name))
                if cls is None:
                    raise pickle.UnpicklingError(
                        f"{module}.{name} is not part of a TurboAdam optimizer state")
                return cls
            return super().find_class(module, name)

    mod = types.ModuleType("turboadam_b200_reference_pickle")
    mod.Unpickler = _Unpickler
    mod.load = lambda file, **kw: _Unpickler(file, **kw).load()
    mod.__dict__.update({k: getattr(pickle, k) for k in ("UnpicklingError", "HIGHEST_PROTOCOL")})
    return torch.load(f, map_location=map_location, pickle_module=mod, weights_only=False)


def pack_indices(idx: torch.Tensor, n_bits: int) -> torch.Tensor:
    """u8 indices (each < 2^n_bits) -> dense little-endian n-bit stream (u8)."""
    if not 1 <= n_bits <= 8:
        raise ValueError("n_bits must be in 1..8")
    v = idx.reshape(-1).to("cpu", torch.uint8).numpy()
    if v.size and int(v.max()) >> n_bits:
        raise ValueError(f"index >= 2^{n_bits}")
    bits = np.unpackbits(v[:, None], axis=1, bitorder="little")[:, :n_bits].reshape(-1)
    return torch.from_numpy(np.packbits(bits, bitorder="little"))


def unpack_indices(packed: torch.Tensor, n_bits: int, count: int) -> torch.Tensor:
    """Inverse of pack_indices: the first `count` indices as u8."""
    bits = np.unpackbits(packed.reshape(-1).to("cpu", torch.uint8).numpy(), bitorder="little")
    bits = bits[: count * n_bits].reshape(count, n_bits)
    full = np.zeros((count, 8), np.uint8)
    full[:, :n_bits] = bits
    return torch.from_numpy(np.packbits(full, axis=1, bitorder="little").reshape(-1))


def _compact(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to("cpu").clone().contiguous()


def portable_state_dict(opt, pack: bool = False) -> dict:
    """Compact, package-free checkpoint of a TurboAdam (see module doc)."""
    sd = opt.state_dict()
    out_state = {}
    for k, st in sd["state"].items():
        o = {}
        for name, v in st.items():
            if name == "compressed_v":
                cv = dict(v)
                B = cv["scales"].shape[0]
                idx = _compact(cv["indices"])[: B * int(cv["block_size"])]
                if pack:
                    cv["indices"] = pack_indices(idx, int(cv["n_bits"]))
                    cv["packed"] = True
                else:
                    cv["indices"] = idx
                cv["scales"] = _compact(cv["scales"])
                o[name] = cv
            elif isinstance(v, CoStateManager):
                enc = v._encoded
                o[name] = {
                    "kind": "CoStateManager",
                    "block_size": v.block_size,
                    "null_pct": v._null_pct,
                    "amp_pct": v._amp_pct,
                    "has_state": bool(v._has_state),
                    "alpha": float(v._alpha),
                    "original_numel": int(v._original_numel),
                    "error_feedback": bool(v._error_feedback),
                    "encoded": None if enc is None else {kk: _compact(t) for kk, t in enc.items()},
                    "ef_residual": (None if v._ef_residual is None
                                    else _compact(v._ef_residual)),
                }
            elif isinstance(v, torch.Tensor):
                o[name] = _compact(v)
            else:
                o[name] = copy.deepcopy(v)
        out_state[k] = o
    return {"format": FORMAT, "seed": int(opt._seed), "state": out_state,
            "param_groups": copy.deepcopy(sd["param_groups"])}


def load_portable_state_dict(opt, sd: dict) -> None:
    """Load a portable_state_dict (also packed) into a TurboAdam."""
    if sd.get("format") != FORMAT:
        raise ValueError(f"not a {FORMAT} checkpoint")
    state = {}
    for k, st in sd["state"].items():
        o = {}
        for name, v in st.items():
            if name == "compressed_v":
                cv = dict(v)
                if cv.pop("packed", False):
                    B = cv["scales"].shape[0]
                    cv["indices"] = unpack_indices(cv["indices"], int(cv["n_bits"]),
                                                   B * int(cv["block_size"]))
                o[name] = cv
            elif isinstance(v, dict) and v.get("kind") == "CoStateManager":
                mgr = CoStateManager(block_size=v["block_size"], error_feedback=v["error_feedback"],
                                     null_pct=v["null_pct"], amp_pct=v["amp_pct"])
                mgr._has_state = v["has_state"]
                mgr._alpha = v["alpha"]
                mgr._original_numel = v["original_numel"]
                mgr._encoded = None if v["encoded"] is None else dict(v["encoded"])
                mgr._ef_residual = v.get("ef_residual")
                o[name] = mgr
            else:
                o[name] = v
        state[k] = o
    opt.load_state_dict({"state": state, "param_groups": sd["param_groups"]})
    # torch casts floating state to the parameter's dtype on load (lossy for
    # bf16 parameters: fp16 headers, fp32 moments); put the exact values back
    ids = [i for g in sd["param_groups"] for i in g["params"]]
    params = [p for g in opt.param_groups for p in g["params"]]
    for k, p in zip(ids, params):
        if k not in state or p not in opt.state:
            continue
        src, dst = state[k], opt.state[p]
        if "compressed_v" in src:
            dst["compressed_v"] = adopt_compressed_v(src["compressed_v"], p.device)
        for name in ("exp_avg", "exp_avg_sq"):
            if name in src:
                dst[name] = src[name].to(device=p.device, dtype=torch.float32).contiguous()
    opt._plans = None
    opt._seed = int(sd["seed"]) & 0xFFFFFFFFFFFFFFFF
