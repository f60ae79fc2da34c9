"""Drop-in for inference/hf/tree_logits.py: the logits step of tree construction in one pass.

row_logsumexp(x) -> float32 [..., 1]       (tree_logits.py:34-39)
top_candidates(logits, k) -> (float32 CPU [..., k], int64 CPU [..., k])   (tree_logits.py:42-46)

Both run mfd_topk_logz: one HBM pass yields log Z and the top-k (value descending, equal values by lower
index first) of float32 or bf16 rows.
"""

from __future__ import annotations

import torch

from . import ops


def row_logsumexp(x: torch.Tensor) -> torch.Tensor:
    """logsumexp over the last dim of a CUDA tensor, as float32 with keepdim."""
    _, _, logz = ops.topk_logz(x, 1, ids_dtype=torch.int32)
    return logz.unsqueeze(-1)


def top_candidates(logits: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(top-k log-probabilities as float32 on CPU, their token ids as int64 on CPU) of [..., V] draft logits."""
    top, ids, _ = ops.topk_logz(logits, k, ids_dtype=torch.int64)
    return top.to(device="cpu"), ids.to(device="cpu")
