"""Block size of the packed state (reference src/turboadam/utils.py:19).

The reference pads each tensor to whole blocks on every step
(``pad_to_blocks``, utils.py:27-66); here the state buffers are allocated
padded to whole 16-block tiles once, so no padding helper exists.
"""
BLOCK_SIZE = 128
