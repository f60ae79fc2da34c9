"""Drop-in for the tree operations of inference/hf/ddtree.py (hhhhhhy5/multi-future-drafting), B200-native.

Same names, arguments, return types and edge cases as the reference:

  build_ddtree_tree(draft_logits [L, V], budget)                   ddtree.py:115-211
  build_mixture_tree(draft_logits [K, L, V], mode_log_prior [K], budget)   ddtree.py:214-314
  compile_ddtree_tree(...)                                          ddtree.py:317-357
  multi_mode_draft_mask(context_length, num_modes, block_size, dtype, device)   ddtree.py:360-365
  follow_verified_tree(child_maps, posterior [1, n])                ddtree.py:368-382
  enable_cpp_tree / enable_mode_attention                           ddtree.py:95-112
  compact_dynamic_cache(past_key_values, past_length, keep_current_indices)   ddtree.py:406-436
  _compact_appended_window(cache_tensor, past_length, keep_current_indices)  ddtree.py:385-403

The builders run the logits step (mfd_topk_logz) and the exact heap (mfd_build_trees) on the GPU and
return CPU tensors as the reference does (its callers index them on the host).  The fourth value is a Tree
(as tree_build_ext returns with the C++ builder): follow(posterior) walks the verified path on the GPU;
children(i) returns node i's {token: child} dict.  ddtree_generate (the decode loop) is the caller and is
not part of this package.
"""

from __future__ import annotations

import time

import torch

from . import ops

DDTREE_STAGE_ORDER = ("draft", "tree_build", "tree_compile", "verify", "commit")
DDTREE_TREE_BUILD_STAGE_ORDER = ("tree_build_copy", "tree_build_heap", "tree_build_visibility")

# The reference switches between its Python heap, its C++ heap and a fused logits step
# (inference/hf/ddtree.py:87-103) and between SDPA and a Triton mode-attention kernel (105-112).  Here every
# variant is the same B200 path; the switches are kept so callers that set them keep working.
_CPP_TREE_ENABLED = False
_FUSED_LOGITS = False
_MODE_ATTN = False


def enable_cpp_tree(enabled: bool, fused_logits: bool = False) -> None:
    global _CPP_TREE_ENABLED, _FUSED_LOGITS
    _CPP_TREE_ENABLED = enabled
    _FUSED_LOGITS = enabled and fused_logits


def enable_mode_attention(enabled: bool) -> None:
    global _MODE_ATTN
    _MODE_ATTN = enabled


def empty_stage_times(order) -> dict[str, float]:
    return {name: 0.0 for name in order}


class Tree:
    """Child maps of a built tree, kept on the device.  follow(posterior) -> (accepted node list, next token)."""

    def __init__(self, tokens: torch.Tensor, parents: torch.Tensor, n: int, tokens_cpu=None, parents_cpu=None):
        # tokens/parents: [W] int64 CUDA (index 0 = root); n = number of nodes including the root
        self._tokens = tokens
        self._parents = parents
        self._n = int(n)
        self._tokens_cpu = tokens_cpu
        self._parents_cpu = parents_cpu

    def __len__(self) -> int:
        return self._n

    def follow(self, posterior: torch.Tensor):
        post = posterior.reshape(-1).to(device=self._tokens.device, dtype=torch.long)
        W = self._tokens.shape[0]
        if post.numel() < W:
            post = torch.cat([post, post.new_zeros(W - post.numel())])
        o = ops.follow(post[:W].view(1, W), self._tokens.view(1, W), self._parents.view(1, W), max_steps=-1,
                       out_len=W)
        n = int(o["accept_len"][0].item())
        accepted = o["accepted"][0, : n + 1].tolist()
        return accepted, int(o["bonus"][0].item())

    def children(self, i: int) -> dict[int, int]:
        if self._tokens_cpu is None:
            self._tokens_cpu = self._tokens.cpu()
            self._parents_cpu = self._parents.cpu()
        out = {}
        for j in range(1, self._n):
            if int(self._parents_cpu[j]) == i:
                out[int(self._tokens_cpu[j])] = j
        return out


def _trivial(build_subtimes):
    visibility = torch.zeros((1, 1), dtype=torch.bool)
    visibility[0, 0] = True
    return (torch.empty(0, dtype=torch.long), torch.empty(0, dtype=torch.long), [-1],
            _EmptyTree(), visibility, build_subtimes)


class _EmptyTree(list):
    """The reference returns [dict()] for an empty tree; a list of one empty dict walks the same way."""

    def __init__(self):
        super().__init__([dict()])


def _build(draft_logits: torch.Tensor, prior: torch.Tensor | None, budget: int, single: bool):
    """draft_logits [K, L, V] on CUDA -> the reference's 6-tuple."""
    build_subtimes = empty_stage_times(DDTREE_TREE_BUILD_STAGE_ORDER)
    K, L, V = draft_logits.shape
    topk = min(budget, V)
    t0 = time.perf_counter()
    x = draft_logits if draft_logits.dtype in (torch.float32, torch.bfloat16) else draft_logits.float()
    top, ids, _ = ops.topk_logz(x.reshape(K * L, V), topk, ids_dtype=torch.int32)
    prior_dev = None if prior is None else prior.to(device=draft_logits.device, dtype=torch.float32).view(1, K)
    tree, counts, _, vis = ops.build_trees(top.view(1, K, L, topk), ids.view(1, K, L, topk), prior_dev, budget,
                                           single=single, want_anc=False, want_vis=True)
    t1 = time.perf_counter()
    tree_cpu = tree[0].cpu()
    n = int(counts[0].item())
    vis_cpu = vis[0, : n + 1, : n + 1].cpu().to(torch.bool)
    build_subtimes["tree_build_heap"] = t1 - t0
    build_subtimes["tree_build_copy"] = time.perf_counter() - t1
    node_token_ids = tree_cpu[0, 1 : n + 1].clone()
    node_depths = tree_cpu[1, 1 : n + 1].clone()
    parents = tree_cpu[2, : n + 1].tolist()
    child_maps = Tree(tree[0, 0], tree[0, 2], n + 1, tree_cpu[0], tree_cpu[2])
    return node_token_ids, node_depths, parents, child_maps, vis_cpu, build_subtimes


def build_ddtree_tree(draft_logits: torch.Tensor, budget: int):
    """DDTree over one draft distribution [L, V] (single-mode heap, rank-tuple tie-break)."""
    if budget <= 0 or draft_logits.shape[0] == 0:
        return _trivial(empty_stage_times(DDTREE_TREE_BUILD_STAGE_ORDER))
    ops.require_cuda(draft_logits)
    return _build(draft_logits.unsqueeze(0), None, budget, single=True)


def build_mixture_tree(draft_logits: torch.Tensor, mode_log_prior: torch.Tensor, budget: int):
    """MFD mixture tree: the `budget` distinct prefixes with the largest max_k [log pi_k + log q_k(prefix)]."""
    num_modes, depth_limit = int(draft_logits.shape[0]), int(draft_logits.shape[1])
    if budget <= 0 or depth_limit == 0:
        return build_ddtree_tree(draft_logits[0], budget)
    ops.require_cuda(draft_logits)
    return _build(draft_logits, mode_log_prior, budget, single=False)


def compile_ddtree_tree(root_token_id, start, node_token_ids, node_depths, visibility_cpu, past_length, dtype,
                        device, verify_input_ids_buffer, verify_position_ids_buffer, attention_mask_buffer,
                        tree_visibility_buffer, previous_tree_start, previous_tree_length):
    """Verify inputs and the additive tree mask in the caller's buffers (inference/hf/ddtree.py:317-357)."""
    current_length = 1 + int(node_token_ids.numel())
    if previous_tree_length > 0:
        attention_mask_buffer[0, 0, :previous_tree_length,
                              previous_tree_start: previous_tree_start + previous_tree_length] = 0
    verify_input_ids = verify_input_ids_buffer[:, :current_length]
    verify_input_ids[0, 0] = root_token_id
    if current_length > 1:
        verify_input_ids[0, 1:current_length].copy_(node_token_ids, non_blocking=False)
    verify_position_ids = verify_position_ids_buffer[:, :current_length]
    verify_position_ids[0, 0] = start
    if current_length > 1:
        verify_position_ids[0, 1:current_length].copy_(node_depths, non_blocking=False)
        verify_position_ids[0, 1:current_length].add_(start)
    visibility = tree_visibility_buffer[:current_length, :current_length]
    visibility.copy_(visibility_cpu, non_blocking=False)
    tree_block = attention_mask_buffer[0, 0, :current_length, past_length: past_length + current_length]
    tree_block.fill_(torch.finfo(dtype).min)
    tree_block.masked_fill_(visibility, 0)
    attention_mask = attention_mask_buffer[:, :, :current_length, : past_length + current_length]
    return verify_input_ids, verify_position_ids, attention_mask, past_length, current_length


def multi_mode_draft_mask(context_length: int, num_modes: int, block_size: int, dtype: torch.dtype,
                          device: torch.device) -> torch.Tensor:
    """Additive [1, 1, K*bs, context + K*bs] mask of a multi-mode draft step (inference/hf/ddtree.py:360-365)."""
    query_block = torch.arange(num_modes * block_size, device=device) // block_size
    mask = torch.zeros((num_modes * block_size, context_length + num_modes * block_size), dtype=dtype, device=device)
    mask[:, context_length:].masked_fill_(query_block.unsqueeze(1) != query_block.unsqueeze(0), torch.finfo(dtype).min)
    return mask.view(1, 1, *mask.shape)


def follow_verified_tree(child_maps, posterior: torch.Tensor):
    """(accepted node indices, next token): follow the target's token at each node from the root."""
    if isinstance(child_maps, Tree):
        return child_maps.follow(posterior[0])
    posterior_tokens = posterior[0].tolist()
    accepted_indices = [0]
    current_index = 0
    next_token = int(posterior_tokens[current_index])
    while next_token in child_maps[current_index]:
        current_index = child_maps[current_index][next_token]
        accepted_indices.append(current_index)
        next_token = int(posterior_tokens[current_index])
    return accepted_indices, next_token


# ----------------------------------------------------------------------------------------------- commit step

def _compact_appended_window(cache_tensor: torch.Tensor, past_length: int, keep_current_indices: torch.Tensor) -> None:
    """Rows past_length + keep[i] -> past_length + i along dim -2, in place (inference/hf/ddtree.py:385-403): a
    no-op when the appended window is empty, keep is empty or keep covers the whole window."""
    ops.compact_tail([cache_tensor], past_length, keep_current_indices)


def compact_dynamic_cache(past_key_values, past_length: int, keep_current_indices: list[int]) -> None:
    """Keep only the accepted rows of the appended tree window in every layer's keys and values, then crop the
    cache to past_length + len(keep) (inference/hf/ddtree.py:406-436).  All layers' K and V move in one launch."""
    if len(keep_current_indices) == 0:
        past_key_values.crop(past_length)
        return
    if hasattr(past_key_values, "key_cache") and hasattr(past_key_values, "value_cache"):
        tensors = list(past_key_values.key_cache) + list(past_key_values.value_cache)
    elif hasattr(past_key_values, "layers"):
        tensors = []
        for layer in past_key_values.layers:
            if not hasattr(layer, "keys") or layer.keys is None or layer.keys.numel() == 0:
                continue
            tensors += [layer.keys, layer.values]
    else:
        raise RuntimeError("Unsupported DynamicCache layout for DDTree cache compaction.")
    by_device: dict = {}
    for t in tensors:
        by_device.setdefault(t.device, []).append(t)
    for group in by_device.values():
        ops.compact_tail(group, past_length, keep_current_indices)
    past_key_values.crop(past_length + len(keep_current_indices))
