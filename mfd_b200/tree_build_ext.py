"""Drop-in for inference/hf/tree_build_ext.py: build_single / build_mixture on given candidates.

Same arguments and return values as the reference (tree_build_ext.py:226-234): CPU candidate tables in,
(node_token_ids i64 [n], node_depths i64 [n], parents list [n+1], Tree, visibility bool [n+1, n+1]) out,
with identical pop order and tie-breaks (checked against the reference's own compiled builder in tests).
The heap runs on the GPU (mfd_build_trees); the Tree walks on the GPU.
"""

from __future__ import annotations

import torch

from . import ops
from .ddtree import Tree

_MODULE = None


def load_module():
    """The reference compiles its C++ here; the B200 library is loaded instead (and built if missing)."""
    from . import _lib

    return _lib.load()


def _run(lp: torch.Tensor, ids: torch.Tensor, prior: torch.Tensor | None, budget: int, single: bool):
    dev = torch.device("cuda", torch.cuda.current_device())
    K, L, k = lp.shape
    lp_d = lp.to(device=dev, dtype=torch.float32).contiguous().view(1, K, L, k)
    ids_d = ids.to(device=dev, dtype=torch.int64).contiguous().view(1, K, L, k)
    pr = None if prior is None else prior.to(device=dev, dtype=torch.float32).view(1, K)
    if budget <= 0 or L == 0:
        vis = torch.ones(1, 1, dtype=torch.bool)
        t = torch.zeros(1, dtype=torch.long, device=dev)
        p = torch.full((1,), -1, dtype=torch.long, device=dev)
        return torch.empty(0, dtype=torch.long), torch.empty(0, dtype=torch.long), [-1], Tree(t, p, 1), vis
    tree, counts, _, vis = ops.build_trees(lp_d, ids_d, pr, budget, single=single, want_anc=False, want_vis=True)
    tree_cpu = tree[0].cpu()
    n = int(counts[0].item())
    return (tree_cpu[0, 1: n + 1].clone(), tree_cpu[1, 1: n + 1].clone(), tree_cpu[2, : n + 1].tolist(),
            Tree(tree[0, 0], tree[0, 2], n + 1, tree_cpu[0], tree_cpu[2]),
            vis[0, : n + 1, : n + 1].cpu().to(torch.bool))


def build_single(top_log_probs: torch.Tensor, top_token_ids: torch.Tensor, budget: int):
    """[L, k] float32 / int64 -> (node_token_ids, node_depths, parents, child_maps, visibility)."""
    return _run(top_log_probs.unsqueeze(0), top_token_ids.unsqueeze(0), None, budget, single=True)


def build_mixture(top_log_probs: torch.Tensor, top_token_ids: torch.Tensor, log_prior: torch.Tensor, budget: int):
    """[K, L, k] float32 / int64 and [K] float32 -> as build_single."""
    return _run(top_log_probs, top_token_ids, log_prior, budget, single=False)
