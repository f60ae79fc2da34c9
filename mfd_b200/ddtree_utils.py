"""Drop-in for the tree ops of the SGLang patch's ddtree_utils.py (sglang-v0.5.22-mfd.patch:1027-1948).

  build_trees_cpu(*, top_log_probs, top_ids, log_prior, bs, budget, tree, counts)   patch:1431-1445
  build_trees(...)   same, device tensors, no host round trip (stream-ordered, CUDA-graph safe)
  row_logsumexp(x, out=None)                                                     patch:1472-1482
  DDTreeDraftTopK(weight, block_size, num_modes, budget, max_bs, vocab_ids=None)  patch:1485-1550
  ddtree_verify_inputs(*, root_tokens, prefix_lens, tokens, depths, parents, mask_offsets, ids_out,
                       positions_out, mask_out, max_depth)                        patch:1670-1703
  ddtree_follow(*, posterior, verify_ids, parents, window, prefix_lens, <outs>)   patch:1844-1885
  ancestor_visibility_reference(parents)                                          patch:1938-1948
  DDTreeKVCompactor(kv_pool)(move_src=, move_tgt=)                              patch:1769-1841

The host builder of the reference (C++ on CPU, fed through pinned buffers) becomes the GPU builder, so the
draft top-k, tree build, verify inputs and walk all stay on the device.
"""

from __future__ import annotations

import json
import os
from typing import Optional

import torch

from . import ops


def build_trees(*, top_log_probs: torch.Tensor, top_ids: torch.Tensor, log_prior: torch.Tensor, bs: int, budget: int,
                tree: torch.Tensor, counts: torch.Tensor, anc: bool = False):
    """Device build into caller-owned device buffers tree [bs, 3, B+1] int64 and counts [bs] int64.
    K == 1 uses the single-mode heap (as the SGLang builder does).  Returns the ancestor bitsets if asked."""
    K = top_log_probs.shape[1]
    _, _, a, _ = ops.build_trees(top_log_probs[:bs], top_ids[:bs], log_prior[:bs] if log_prior is not None else None,
                                 budget, single=(K == 1), tree=tree, counts=counts, want_anc=anc)
    return a


def build_trees_cpu(*, top_log_probs: torch.Tensor, top_ids: torch.Tensor, log_prior: torch.Tensor, bs: int,
                    budget: int, tree: torch.Tensor, counts: torch.Tensor) -> None:
    """The reference's host-build signature: CPU (or CUDA) tensors in, results written into `tree` / `counts`.
    The build itself runs on the GPU."""
    dev = torch.device("cuda", torch.cuda.current_device())
    lp = top_log_probs[:bs].to(dev, non_blocking=True)
    ids = top_ids[:bs].to(dev, non_blocking=True)
    pr = log_prior[:bs].to(dev, non_blocking=True) if log_prior is not None else None
    if tree.is_cuda and counts.is_cuda:
        build_trees(top_log_probs=lp, top_ids=ids, log_prior=pr, bs=bs, budget=budget, tree=tree, counts=counts)
        return
    t = torch.empty((bs, 3, budget + 1), dtype=torch.int64, device=dev)
    c = torch.empty((bs,), dtype=torch.int64, device=dev)
    build_trees(top_log_probs=lp, top_ids=ids, log_prior=pr, bs=bs, budget=budget, tree=t, counts=c)
    tree[:bs].copy_(t)
    counts[:bs].copy_(c)


def row_logsumexp(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """log-sum-exp over the last dim of a 2D row-major CUDA tensor, float32 [rows]."""
    assert x.ndim == 2 and x.stride(1) == 1
    rows = x.shape[0]
    if out is None:
        out = torch.empty(rows, device=x.device, dtype=torch.float32)
    if rows > 0:
        top = torch.empty(rows, 1, dtype=torch.float32, device=x.device)
        ids = torch.empty(rows, 1, dtype=torch.int32, device=x.device)
        ops.topk_logz(x, 1, ids_dtype=torch.int32, out=(top, ids, out))
    return out


def ddtree_draft_vocab_path() -> str:
    """Token-id list of the reduced draft vocabulary ("" = the full vocabulary): the SGLANG_DFLASH_DDTREE_DRAFT_VOCAB
    setting of the SGLang patch (P:1221-1223), read from the environment."""
    return str(os.environ.get("SGLANG_DFLASH_DDTREE_DRAFT_VOCAB", "") or "").strip()


def load_draft_vocab(path: str, *, vocab_size: int) -> torch.Tensor:
    """The draft vocabulary at ``path`` (P:1226-1244) as sorted unique int64 token ids on the CPU: a JSON list, a
    JSON object with "token_ids", or whitespace-separated ids.  Sorting keeps the full vocabulary's relative order
    in the subset.  Ids outside [0, vocab_size), or none at all, raise ValueError."""
    with open(path) as f:
        text = f.read()
    try:
        spec = json.loads(text)
        ids = spec["token_ids"] if isinstance(spec, dict) else spec
    except ValueError:
        ids = text.split()
    ids = sorted({int(i) for i in ids})
    if not ids or ids[0] < 0 or ids[-1] >= vocab_size:
        raise ValueError(
            f"SGLANG_DFLASH_DDTREE_DRAFT_VOCAB={path!r}: token ids must lie in [0, {vocab_size}), "
            f"got {len(ids)} ids in [{ids[0] if ids else None}, {ids[-1] if ids else None}].")
    return torch.tensor(ids, dtype=torch.int64)


class DDTreeDraftTopK:
    """Top-k candidates of every drafted position into static buffers (graph safe).

    Called on the draft hidden states [bs * num_modes * block_size, H] (each block: the anchor then the
    block_size - 1 drafted positions): logits = hs @ weight.T (the caller's LM head, cuBLAS), then one
    mfd_topk_logz pass writes top_logp [bs, K, L, k] (float32 log-probabilities) and top_ids [bs, K, L, k]
    (int32).  With vocab_ids the head covers a vocabulary subset and ids map back through vocab_ids."""

    def __init__(self, *, weight: torch.Tensor, block_size: int, num_modes: int, budget: int, max_bs: int,
                 vocab_ids: Optional[torch.Tensor] = None):
        self.weight = weight
        self.block_size = int(block_size)
        self.num_modes = int(num_modes)
        self.vocab = int(weight.shape[0])
        if vocab_ids is not None:
            assert vocab_ids.dtype == torch.int32 and vocab_ids.shape == (self.vocab,), (vocab_ids.dtype,
                                                                                      vocab_ids.shape, weight.shape)
        self.vocab_ids = vocab_ids
        self.topk = int(min(budget, self.vocab))
        self.max_bs = int(max_bs)
        device = weight.device
        rows = self.max_bs * self.num_modes * (self.block_size - 1)
        self.top_logp = torch.empty((rows, self.topk), dtype=torch.float32, device=device)
        self.top_ids = torch.empty((rows, self.topk), dtype=torch.int32, device=device)
        self.log_z = torch.empty((rows,), dtype=torch.float32, device=device)
        self._idx = torch.empty((rows, self.topk), dtype=torch.int32, device=device) if vocab_ids is not None else None

    def __call__(self, hidden_states: torch.Tensor, input_ids=None) -> None:
        del input_ids
        L = self.block_size
        groups = hidden_states.shape[0] // L
        hs = hidden_states.view(groups, L, -1)[:, 1:, :].reshape(-1, hidden_states.shape[-1])
        if hs.dtype != self.weight.dtype:
            hs = hs.to(self.weight.dtype)
        n = hs.shape[0]
        logits = torch.matmul(hs, self.weight.T)
        if self.vocab_ids is None:
            ops.topk_logz(logits, self.topk, ids_dtype=torch.int32,
                          out=(self.top_logp[:n], self.top_ids[:n], self.log_z[:n]))
        else:
            ops.topk_logz(logits, self.topk, ids_dtype=torch.int32,
                          out=(self.top_logp[:n], self._idx[:n], self.log_z[:n]))
            torch.index_select(self.vocab_ids, 0, self._idx[:n].view(-1).long(), out=self.top_ids[:n].view(-1))

    def outputs(self, bs: int):
        rows = bs * self.num_modes * (self.block_size - 1)
        shape = (bs, self.num_modes, self.block_size - 1, self.topk)
        return self.top_logp[:rows].view(shape), self.top_ids[:rows].view(shape)


def ddtree_verify_inputs(*, root_tokens, prefix_lens, tokens, depths, parents, mask_offsets, ids_out, positions_out,
                         mask_out, max_depth: int) -> None:
    bs, W = tokens.shape
    if bs == 0:
        return
    ops.verify_inputs(root_tokens, prefix_lens, tokens, depths, parents, mask_offsets, ids_out, positions_out,
                      mask_out.view(torch.int8), max_depth)


def ddtree_follow(*, posterior, verify_ids, parents, window, prefix_lens, accept_len_out, commit_lens_out, bonus_out,
                  out_tokens_out, new_seq_lens_out, move_src_out, move_tgt_out, hidden_index_out) -> None:
    """Walk each request's tree along the target's token at each node (at most L-1 edges, L =
    out_tokens_out.shape[1]) and emit the commit outputs, as the reference kernel does."""
    bs, W = verify_ids.shape
    if bs == 0:
        return
    L = int(out_tokens_out.shape[1])
    outs = {"accept_len": accept_len_out, "commit_lens": commit_lens_out, "bonus": bonus_out,
            "out_tokens": out_tokens_out, "new_seq_lens": new_seq_lens_out, "move_src": move_src_out,
            "move_tgt": move_tgt_out, "hidden_index": hidden_index_out}
    ops.follow(posterior, verify_ids, parents, max_steps=L - 1, out_len=L, window=window, prefix_lens=prefix_lens,
               outs=outs)


def ancestor_visibility_reference(parents: torch.Tensor) -> torch.Tensor:
    """[W, W] bool ancestor-or-self matrix of one tree (tests only)."""
    W = parents.numel()
    vis = torch.zeros((W, W), dtype=torch.bool)
    p = parents.tolist()
    for i in range(W):
        j = i
        while j >= 0:
            vis[i, j] = True
            j = p[j] if j > 0 else -1
    return vis


class DDTreeKVCompactor:
    """Commit-time KV moves of DDTree rounds on a token-major pool (patch:1769-1841): only the moves that change a
    slot, every source read before any store, all of the pool's buffers in one launch (mfd_commit_kv_moves).
    kv_pool needs `data_ptrs` (device int64 tensor of buffer base addresses) and `data_strides` (bytes per slot,
    one value, a multiple of 8)."""

    def __init__(self, kv_pool):
        strides = {int(s) for s in kv_pool.data_strides.tolist()}
        if len(strides) != 1 or next(iter(strides)) % 8:
            raise ValueError(f"DDTree KV compaction needs one slot stride (multiple of 8 bytes), got {strides}")
        self.data_ptrs = kv_pool.data_ptrs
        self.slot_bytes = next(iter(strides))
        # the alignment every buffer base has (read once here, so the call itself does no host read) and the
        # pool's slot count when the pool exposes its buffers (slot ids beyond it are skipped, not dereferenced)
        bases = [int(b) for b in kv_pool.data_ptrs.tolist()]
        if any(b % 8 for b in bases):
            raise ValueError("DDTree KV compaction needs buffer bases aligned to 8 bytes")
        self.base_align = 16 if all(b % 16 == 0 for b in bases) else 8
        bufs = getattr(kv_pool, "k_buffer", None)
        self.pool_slots = int(bufs[0].shape[0]) if bufs else 0

    @staticmethod
    def supports(kv_pool) -> bool:
        """A plain token-major pool: one slot stride, no per-head layout switch, no scale buffers (the conditions of
        patch:1797-1807, read from the pool's attributes rather than its class)."""
        try:
            strides = {int(s) for s in kv_pool.data_strides.tolist()}
        except AttributeError:
            return False
        return (len(strides) == 1 and next(iter(strides)) % 8 == 0 and not getattr(kv_pool, "use_hnd", False)
                and not getattr(kv_pool, "use_native_move_kv_cache", False)
                and getattr(kv_pool, "native_k_scale_buffer", None) is None
                and getattr(kv_pool, "k_scale_buffer", None) is None and getattr(kv_pool, "layer_num", 1) > 0)

    def __call__(self, *, move_src: torch.Tensor, move_tgt: torch.Tensor) -> None:
        if move_src.shape[0] == 0:
            return
        ops.commit_kv_moves(self.data_ptrs, self.slot_bytes, move_src, move_tgt, base_align=self.base_align,
                            pool_slots=self.pool_slots)
