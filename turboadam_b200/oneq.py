"""1Q second-moment codec on the device (reference oneq.py / quantize.py).

State layout is the reference's: ``indices`` u8 [B*block] (one bucket index
per byte), ``scales`` fp16 [B, 2] = (log_min, log_max) of ln v, plus the
metadata keys of ``compress_v_logscale`` (oneq.py:41-48). The index/scale
tensors are views of buffers padded to whole 16-block tiles.
"""
from __future__ import annotations

import torch

from . import _lib
from .utils import BLOCK_SIZE


def _n_blocks(n: int, bs: int) -> int:
    return (n + bs - 1) // bs


def init_compressed_v(shape, n_bits: int, device, block_size: int = BLOCK_SIZE) -> dict:
    """State of optimizer.py:273-280: compress_v_logscale(full(1e-30),
    stochastic_round=False) -- indices 0, both headers fp16(ln 1e-30)."""
    lib = _lib.load()
    n = 1
    for s in shape:
        n *= int(s)
    B = _n_blocks(n, block_size)
    P = int(lib.ta_state_padded_blocks(n, block_size))
    idx = torch.empty(P * block_size, dtype=torch.uint8, device=device)
    hdr = torch.empty(P * 2, dtype=torch.float16, device=device)
    _lib.check(lib.ta_v_init(P * block_size, block_size, idx.data_ptr(), hdr.data_ptr(),
                             _lib.stream_ptr(device)), "ta_v_init")
    return _wrap(idx, hdr, n, B, n_bits, block_size, torch.Size(shape))


def _wrap(idx, hdr, n, B, n_bits, block_size, shape):
    return {
        "indices": idx[: B * block_size],
        "scales": hdr[: 2 * B].view(B, 2),
        "n_bits": n_bits,
        "original_shape": shape,
        "original_length": n,
        "block_size": block_size,
    }


def storage_capacity(t: torch.Tensor) -> int:
    """Bytes of t's storage from its first element on (padding included)."""
    return t.untyped_storage().nbytes() - t.storage_offset() * t.element_size()


def is_padded(cv: dict, device) -> bool:
    """True if the 1Q tensors are on `device` in whole-tile padded storage."""
    idx, hdr = cv["indices"], cv["scales"]
    if idx.device != device or hdr.device != device or hdr.dtype != torch.float16:
        return False
    if idx.dtype != torch.uint8 or not idx.is_contiguous() or not hdr.is_contiguous():
        return False
    n, bs = int(cv["original_length"]), int(cv["block_size"])
    P = int(_lib.load().ta_state_padded_blocks(n, bs))
    return (storage_capacity(idx) >= P * bs and storage_capacity(hdr) >= P * 4
            and idx.data_ptr() % 16 == 0 and hdr.data_ptr() % 16 == 0)


def adopt_compressed_v(cv: dict, device) -> dict:
    """Copy loaded (possibly cast / unpadded) 1Q state into padded buffers."""
    lib = _lib.load()
    n = int(cv["original_length"])
    bs = int(cv["block_size"])
    B = _n_blocks(n, bs)
    P = int(lib.ta_state_padded_blocks(n, bs))
    idx = torch.zeros(P * bs, dtype=torch.uint8, device=device)
    hdr = torch.zeros(P * 2, dtype=torch.float16, device=device)
    idx[: B * bs].copy_(cv["indices"].reshape(-1).to(device=device, dtype=torch.uint8))
    # load_state_dict casts floating state to the param dtype (the reference
    # reads it back with .to(float32), quantize.py:253-254); store fp16 again.
    hdr[: 2 * B].copy_(cv["scales"].reshape(-1).to(device=device).to(torch.float16))
    return _wrap(idx, hdr, n, B, int(cv["n_bits"]), bs, cv.get("original_shape", torch.Size([n])))


def decompress_v(compressed: dict) -> torch.Tensor:
    """fp32 v of the original shape (oneq.py:51-67)."""
    idx = compressed["indices"]
    _lib.require_cuda(idx)
    lib = _lib.load()
    n = int(compressed["original_length"])
    hdr = compressed["scales"].to(torch.float16).contiguous()
    idx = idx.to(torch.uint8).contiguous()
    out = torch.empty(n, dtype=torch.float32, device=idx.device)
    _lib.check(lib.ta_v_decode(idx.data_ptr(), hdr.data_ptr(), n, int(compressed["block_size"]),
                               int(compressed["n_bits"]), out.data_ptr(),
                               _lib.stream_ptr(idx.device)), "ta_v_decode")
    return out.reshape(compressed["original_shape"])


def fused_v_update(indices, scales, grad, beta2, n_bits, block_size, original_numel,
                   rand_buf=None, out_indices=None, out_scales=None, *, seed: int = 0,
                   tensor_id: int = 0, step: int = 1):
    """Decompress -> EMA -> recompress (quantize.py:222-299 /
    triton_kernels.py:105-165). ``rand_buf`` (padded-length fp32 uniforms)
    replaces the stochastic-rounding draws, as in the reference's CUDA path;
    otherwise Philox keyed by (seed, tensor_id, step) draws them.
    Returns (new_indices, new_scales, v_flat[original_numel])."""
    _lib.require_cuda(grad)
    lib = _lib.load()
    dev = grad.device
    n = int(original_numel)
    g = grad.reshape(-1)
    if g.dtype not in (torch.float32, torch.bfloat16):
        g = g.float()
    g = g.contiguous()
    idx = indices.to(torch.uint8).contiguous()
    hdr = scales.to(torch.float16).contiguous()
    new_idx = torch.empty_like(idx) if out_indices is None else out_indices
    new_hdr = torch.empty_like(hdr) if out_scales is None else out_scales
    v = torch.empty(n, dtype=torch.float32, device=dev)
    ws = torch.empty(lib.ta_aux_workspace_size(n), dtype=torch.uint8, device=dev)
    u = None
    if rand_buf is not None:
        u = rand_buf.reshape(-1).to(torch.float32).contiguous()
    _lib.check(lib.ta_v_update(idx.data_ptr(), hdr.data_ptr(), g.data_ptr(),
                               _lib.TA_BF16 if g.dtype == torch.bfloat16 else _lib.TA_F32, n,
                               int(block_size), int(n_bits), float(beta2),
                               u.data_ptr() if u is not None else None, seed, tensor_id, step,
                               new_idx.data_ptr(), new_hdr.data_ptr(), v.data_ptr(),
                               ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev)), "ta_v_update")
    return new_idx, new_hdr.reshape(-1, 2), v
