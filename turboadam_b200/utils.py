"""Block helpers (reference src/turboadam/utils.py)."""
from __future__ import annotations

import torch

BLOCK_SIZE = 128


def pad_to_blocks(tensor: torch.Tensor, block_size: int = BLOCK_SIZE,
                  pad_value: float = 0.0) -> tuple[torch.Tensor, int]:
    """Pad a flat tensor to a multiple of block_size (utils.py:27-53)."""
    n = tensor.shape[0]
    rem = n % block_size
    if rem == 0:
        return tensor, n
    fill = tensor.new_full((block_size - rem,), pad_value)
    return torch.cat([tensor, fill]), n


def unpad_from_blocks(padded: torch.Tensor, original_length: int) -> torch.Tensor:
    return padded[:original_length]
