"""Drop-in for the SGLang patch's python/sglang/srt/speculative/ddtree_mode_attention.py: the paged multi-mode draft
attention of a serving batch on B200 (sglang-v0.5.22-mfd.patch:593-1026).

The K mode blocks of a request sit side by side (K x block_size queries, mode-major).  Every query attends to the
request's whole context -- the draft KV cache read through ``req_to_token`` -- and to the block_size keys of its own
mode block, taken from this step's projected k/v (never written to the cache).  One launch of the tcgen05 attention
kernel does it: its producer warp gathers each 128-key tile straight from the paged cache (16-byte cp.async copies
into the swizzled layout the tensor cores read, slot ids from the request's req_to_token row), the block keys come
from k_new / v_new, and the block-diagonal visibility is the same bitset the dense mode attention uses.  The grid
is fixed by (splits, M-tiles, KV heads, requests) and every CTA reads its context length on the device, so the
lengths can change between calls without a host round trip.

Signatures follow the reference (paged_mode_block_attention P:897-962, resolve_ctx_splits P:886-894,
PagedModeAttention P:991-1026).  ``num_ctx_splits``: > 0 splits the keys of every request into that many ranges (the
last CTA of a (request, KV head, M-tile) merges them); 0 runs one range; < 0 picks a split count that fills the SMs.
The tuning arguments ``modes_per_program``, ``block_n``, ``min_chunk`` and ``num_warps`` are accepted and ignored.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import ops
from .mode_attention import block_bits

_SM_COUNT: dict = {}


def _sm_count(device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SM_COUNT:
        _SM_COUNT[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SM_COUNT[idx]


def resolve_ctx_splits(num_ctx_splits: int, *, programs: int, device) -> int:
    """num_ctx_splits > 0: that many key ranges per request; 0: one; < 0: auto, enough ranges for the
    (request, KV head, M-tile pair) CTAs to cover the SMs once (at most 16)."""
    if num_ctx_splits > 0:
        return int(num_ctx_splits)
    if num_ctx_splits == 0:
        return 1
    return int(min(16, max(1, _sm_count(device) // max(1, programs))))


def paged_mode_block_attention(
    *,
    q: torch.Tensor,
    k_new: torch.Tensor,
    v_new: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    req_to_token: torch.Tensor,
    req_pool_indices: torch.Tensor,
    ctx_lens: torch.Tensor,
    num_modes: int,
    block_size: int,
    scaling: float,
    num_ctx_splits: int,
    out: Optional[torch.Tensor] = None,
    modes_per_program: int = 2,
    block_n: int = 64,
    min_chunk: int = 64,
    num_warps: Optional[int] = None,
) -> torch.Tensor:
    """q [T, H, D], k_new/v_new [T, Hkv, D] with T = bs * K * block_size (mode-major per request);
    k_cache/v_cache [slots, Hkv, D]; the context of request b is req_to_token[req_pool_indices[b], :ctx_lens[b]].
    Returns [T, H, D] (``out`` if given)."""
    del modes_per_program, block_n, min_chunk, num_warps
    T, H, D = q.shape
    Hkv = k_new.shape[1]
    KL = num_modes * block_size
    bs = T // KL
    if T != bs * KL or H % Hkv:
        raise AssertionError(f"paged_mode_block_attention: T={T} not a multiple of K*block_size={KL} or H % Hkv")
    if out is None:
        out = torch.empty((T, H, D), device=q.device, dtype=q.dtype)
    if bs == 0:
        return out
    splits = resolve_ctx_splits(num_ctx_splits, programs=ops.attention_ctas(bs, KL, H, Hkv, paged=True), device=q.device)
    bits = block_bits(num_modes, block_size, q.device)
    return ops.paged_mode_attention(q, k_new, v_new, k_cache, v_cache, req_to_token, req_pool_indices, ctx_lens,
                                    bits, num_modes, block_size, scaling, splits, out=out)


class PagedModeAttention:
    """Called by DFlashAttention (its ``mode_attention`` hook) in place of RadixAttention for the multi-mode draft
    forward: q/k/v as [T, heads * D] slices of the fused qkv; returns [T, heads * D].  The step's block keys are not
    written to the cache.  impl "triton" (the reference's default name) and "cuda" run the B200 kernel; the
    reference's float32 "reference" implementation is test infrastructure here and is not provided."""

    def __init__(self, *, kv_pool, req_to_token, num_modes: int, block_size: int, num_heads: int, num_kv_heads: int,
                 head_dim: int, scaling: float, num_ctx_splits: int, impl: str):
        if impl not in ("triton", "cuda"):
            raise ValueError(f"PagedModeAttention: impl {impl!r} is not provided (use 'triton' or 'cuda')")
        self.kv_pool = kv_pool
        self.req_to_token = req_to_token
        self.num_modes = int(num_modes)
        self.block_size = int(block_size)
        self.num_heads = int(num_heads)
        self.num_kv_heads = int(num_kv_heads)
        self.head_dim = int(head_dim)
        self.scaling = float(scaling)
        self.num_ctx_splits = int(num_ctx_splits)
        self.impl = impl

    def __call__(self, q, k, v, forward_batch, layer_id: int) -> torch.Tensor:
        T = q.shape[0]
        qh = q.view(T, self.num_heads, self.head_dim)
        kh = k.view(T, self.num_kv_heads, self.head_dim)
        vh = v.view(T, self.num_kv_heads, self.head_dim)
        k_cache, v_cache = self.kv_pool.get_kv_buffer(layer_id)
        bs = T // (self.num_modes * self.block_size)
        out = paged_mode_block_attention(
            q=qh, k_new=kh, v_new=vh, k_cache=k_cache, v_cache=v_cache, req_to_token=self.req_to_token,
            req_pool_indices=forward_batch.req_pool_indices[:bs], ctx_lens=forward_batch.seq_lens[:bs],
            num_modes=self.num_modes, block_size=self.block_size, scaling=self.scaling,
            num_ctx_splits=self.num_ctx_splits)
        return out.view(T, self.num_heads * self.head_dim)
