"""Drop-in for inference/hf/mode_attention.py: the attention of a multi-mode (MFD) draft step on B200.

Every query of mode m (K mode blocks of bs tokens, side by side) attends to the whole context and to the bs keys
of its own block (block-diagonal, not causal, inference/hf/mode_attention.py:153-164).  That is the tree-masked
verify attention with a different visibility: the context plays the prefix and each block key is visible to the
rows of its own mode, so mode_block_attention runs mfd_tree_attention with a block-diagonal bitset (built once per
(K, bs, device) and cached).  Signatures follow inference/hf/mode_attention.py:24-30 and 120-150; the tuning
arguments (modes_per_program, target_programs, block_n) are accepted and ignored.
"""

from __future__ import annotations

import torch

from . import ops

_MASKS: dict = {}


class ModeBlocks:
    """Passed as the attention mask of forward_modes in place of the dense mask: the layers then call
    mode_block_attention for (num_modes, block_size).  `exact` is kept for signature parity; the CUDA kernel runs
    either way."""

    def __init__(self, num_modes: int, block_size: int, exact: bool = False):
        self.mode_blocks = (num_modes, block_size)
        self.exact = exact


def block_bits(num_modes: int, block_size: int, device: torch.device) -> torch.Tensor:
    """[1, K*bs, words] int64 bitsets: row i sees block keys of its own mode (i // bs)."""
    key = (num_modes, block_size, device)
    bits = _MASKS.get(key)
    if bits is None:
        T = num_modes * block_size
        words = (T + 63) // 64
        rows = torch.arange(T) // block_size
        vis = rows[:, None] == rows[None, :]                       # [T, T] bool
        pad = torch.zeros(T, words * 64, dtype=torch.bool)
        pad[:, :T] = vis
        w = pad.view(T, words, 64).to(torch.int64)
        shifts = torch.arange(64, dtype=torch.int64)
        packed = (w << shifts).sum(-1)                             # bit b of word j = key 64 j + b (wraps to int64)
        bits = packed.view(1, T, words).to(device)
        _MASKS[key] = bits
    return bits


def mode_block_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, num_modes: int, block_size: int,
                         scaling: float, modes_per_program: int = 2, target_programs: int = 384,
                         block_n: int = 64) -> torch.Tensor:
    """Attention of the K mode blocks. q: [1, heads, K * bs, D]; k, v: [1, KV heads, context + K * bs, D] (the
    draft cache after the update, the blocks last). Returns [1, K * bs, heads, D]."""
    _, num_heads, num_queries, head_dim = q.shape
    total = k.shape[2]
    if num_queries != num_modes * block_size or num_heads % k.shape[1]:
        raise RuntimeError("mode_block_attention: q must hold num_modes * block_size queries per head")
    ctx = total - num_queries
    bits = block_bits(num_modes, block_size, q.device)
    qv = q.transpose(1, 2)  # [1, K*bs, heads, D] view: strides carry the layout, nothing is copied
    return ops.tree_attention(qv, k, v, bits, ctx, scaling)
