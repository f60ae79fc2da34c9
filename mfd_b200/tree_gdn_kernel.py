"""Drop-in for inference/hf/tree_gdn_kernel.py: tree verification of a gated delta rule layer on B200.

tree_gdn keeps the reference's signature (inference/hf/tree_gdn_kernel.py:153-171); block_t / block_v are
accepted and ignored (the CUDA kernel solves the tree by depth levels, one CTA per (head, 16 value columns)).
tree_gdn_states additionally returns every node's state S_i = e^{G_i} S0 + sum_{j in anc(i)} e^{G_i-G_j} k_j u_j^T,
the per-node form of the commit formula (inference/hf/qwen35_tree.py:134-137).
"""

from __future__ import annotations

import torch

from . import ops


def tree_gdn(q, k, v, g_cum, beta, s0, anc8, block_t: int = 64, block_v: int = 32):
    """q, k: [n, H_k, K] bf16 (l2-normalized, q scaled; value head h uses key head h // (H // H_k));
    v: [n, H, V] bf16; g_cum, beta: [n, H] fp32; s0: [H, K, V]; anc8: [n, n] int8, ancestors or self.
    Returns u and o, [n, H, V] fp32."""
    return ops.tree_gdn(q, k, v, g_cum, beta, s0, anc8)


def tree_gdn_states(q, k, v, g_cum, beta, s0, anc8):
    """As tree_gdn, plus the per-node states [n, H, K, V] fp32."""
    return ops.tree_gdn(q, k, v, g_cum, beta, s0, anc8, emit_states=True)


def tree_prep(x, conv_state, conv_index, conv_w, num_k_heads: int, num_v_heads: int, head_dim: int,
              block_n: int = 16):
    """The short convolution over each node's window + SiLU + l2norm (and q scale), as
    inference/hf/tree_gdn_kernel.py:135-150.  x [n, conv_dim]; conv_state [conv_dim, KC]; conv_index [n, KC] int32
    into [conv_state ; nodes]; conv_w [conv_dim, KC].  Returns q, k [n, H_k, D] and v [n, H, D] bf16."""
    return ops.tree_prep(x, conv_state, conv_index, conv_w, num_k_heads, num_v_heads, head_dim)
