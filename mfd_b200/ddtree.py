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
    """The root-only tree the reference returns for budget <= 0 or no drafted positions."""
    return (torch.empty(0, dtype=torch.long), torch.empty(0, dtype=torch.long), [-1],
            _EmptyTree(), torch.ones((1, 1), dtype=torch.bool), build_subtimes)


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
    # the device copies travel with the host tensors the reference's callers receive, so compile_ddtree_tree and
    # qwen35_tree.tree_verify read the tree where it was built instead of copying it back to the device
    node_token_ids._mfd_tree = tree[0]
    vis_cpu._mfd_vis = vis[0]
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
    """Verify inputs and the additive tree mask in the caller's buffers (inference/hf/ddtree.py:317-357): one
    mfd_compile_tree launch writes the ids, the positions, the visibility and the tree's block of the mask, and
    resets the previous round's block.  A tree from this package's builders is read on the device where it was
    built (nothing crosses the bus, nothing waits for the host); a tree built elsewhere is copied over once."""
    n = 1 + int(node_token_ids.numel())
    dev = attention_mask_buffer.device
    tree = getattr(node_token_ids, "_mfd_tree", None)
    vis = getattr(visibility_cpu, "_mfd_vis", None)
    if tree is None or vis is None or tree.device != dev or vis.device != dev:
        host = torch.zeros(2, n, dtype=torch.long)
        host[0, 1:] = node_token_ids.reshape(-1)
        host[1, 1:] = node_depths.reshape(-1)
        tree = host.to(dev)
        vis = visibility_cpu.to(device=dev, dtype=torch.uint8)
    if isinstance(root_token_id, torch.Tensor) and root_token_id.device == dev:
        root = root_token_id.reshape(1).to(torch.long)
    else:
        root = torch.tensor([int(root_token_id)], dtype=torch.long, device=dev)
    mask2d = attention_mask_buffer[0, 0]
    ops.compile_tree(root, tree[0], tree[1], vis, n, start, past_length, previous_tree_start, previous_tree_length,
                     verify_input_ids_buffer[0], verify_position_ids_buffer[0], mask2d, torch.finfo(dtype).min,
                     tree_visibility_buffer)
    return (verify_input_ids_buffer[:, :n], verify_position_ids_buffer[:, :n],
            attention_mask_buffer[:, :, :n, : past_length + n], past_length, n)


def multi_mode_draft_mask(context_length: int, num_modes: int, block_size: int, dtype: torch.dtype,
                          device: torch.device) -> torch.Tensor:
    """Additive [1, 1, K*bs, context + K*bs] mask of a multi-mode draft step (inference/hf/ddtree.py:360-365): the
    context is open to every query; the block part is closed except on the K diagonal blocks, where a mode's
    queries see their own block's keys (not causal inside a block)."""
    rows = num_modes * block_size
    mask = torch.full((rows, context_length + rows), torch.finfo(dtype).min, dtype=dtype, device=device)
    mask[:, :context_length] = 0
    # [K, bs, K, bs] view of the block part; its diagonal over the two mode axes is the K own-mode blocks
    mask[:, context_length:].unflatten(0, (num_modes, block_size)).unflatten(2, (num_modes, block_size)) \
        .diagonal(dim1=0, dim2=2).zero_()
    return mask[None, None]


def follow_verified_tree(child_maps, posterior: torch.Tensor):
    """(accepted node indices, next token): from the root, step to the child whose token the target produced at the
    current node, while there is one.  A Tree (this package's builders) walks on the device (mfd_follow); a list of
    {token: child} dicts (the reference's Python child maps, or the root-only tree) walks here."""
    if isinstance(child_maps, Tree):
        return child_maps.follow(posterior[0])
    target = [int(t) for t in posterior[0].tolist()]
    path = [0]
    while True:
        child = child_maps[path[-1]].get(target[path[-1]])
        if child is None:
            return path, target[path[-1]]
        path.append(child)


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
