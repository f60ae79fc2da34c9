"""Drop-in for inference/hf/qwen35_tree.py: exact tree verification of the Gated-DeltaNet (GDN) layers of a hybrid
target, B200-native.

A GDN layer carries a recurrent state that every token rewrites, so a draft tree cannot be verified as one flat
sequence: each node's output must come from the state propagated along its own root path only.  While a
TreeContext is active (tree_verify), every patched GDN layer evaluates all nodes from the committed state S0 at
once; commit() then moves each layer's state and conv window to the deepest accepted node.

Public surface (signatures of the reference, qwen35_tree.py:33-171): TreeContext, tree_verify, install, commit,
chain_tree, hybrid_layers, is_hybrid, conv_kernel, new_cache.  The work per layer runs in this package's kernels:
  tree_prep   (mfd_tree_prep)   the causal conv through parent-pointer windows, SiLU, l2norm, q scale;
  tree_gates  (mfd_tree_gates)  beta, the per-token log decay and its sum along each root path, in one launch;
  tree_gdn    (mfd_tree_gdn)    the ancestor-restricted delta rule (u, o);
  commit      (mfd_gdn_commit, mfd_conv_commit)  every layer's state and conv window in one launch each.
A tree built by mfd_b200.ddtree is read on the device where it was built: the context copies nothing back.
"""

from __future__ import annotations

import contextlib
from dataclasses import dataclass

import torch

_ACTIVE = None  # the TreeContext of the verify forward in progress


def _conv_windows(parents: list[int], kernel: int) -> list[list[int]]:
    """Each node's conv window, oldest first, as indices into [cached conv inputs (kernel of them) ; the nodes].

    Going back d steps from node i (d = 0 is i itself) lands on its d-th ancestor a_d, index kernel + a_d, while
    d <= depth(i); past the root it lands on cached input kernel - 1 - (d - depth(i) - 1) = kernel + depth(i) - d.
    The ancestors at distances 0..kernel-1 come from kernel - 1 gathers through the parent array."""
    n = len(parents)
    if n == 0:
        return []
    par = torch.tensor(list(parents) + [-1], dtype=torch.long)  # index n: the parent of "no node"
    hop = [torch.arange(n)]
    for _ in range(1, kernel):
        prev = hop[-1]
        hop.append(par[torch.where(prev >= 0, prev, torch.full_like(prev, n))])
    anc = torch.stack(hop, dim=1)                    # [n, kernel], column d = d-th ancestor or -1
    on_path = anc >= 0
    depth = on_path.sum(dim=1, keepdim=True) - 1     # ancestors within reach (capped at kernel - 1)
    d = torch.arange(kernel)[None]
    idx = torch.where(on_path, kernel + anc, kernel + depth - d)
    return idx.flip(1).tolist()


@dataclass
class _LayerRecord:
    """What commit() needs of one GDN layer's verify pass: u [n, H, Dv] float32, the l2-normed keys k [n, HK, Dk]
    bf16, the path log decays G [n, H] float32 and the layer's conv inputs x [n, conv_dim]."""
    u: torch.Tensor
    k: torch.Tensor
    G: torch.Tensor
    x: torch.Tensor


class TreeContext:
    """One tree under verification: its ancestor-or-self matrix `anc` [n, n] (bool, and `anc_f` float, `anc8` int8),
    the parent array on the device, each node's conv window (`conv_index` [n, kernel] int32 and `conv_index_cpu`),
    and the per-layer records the verify pass leaves for commit()."""

    def __init__(self, parents: list[int], visibility: torch.Tensor, conv_kernel: int, device: torch.device):
        n = len(parents)
        dev = torch.device(device)
        self.parents = list(parents)
        built = getattr(visibility, "_mfd_vis", None)  # the builder's device copy of this tree
        if built is not None and built.device == dev and built.shape[0] >= n:
            self.anc8 = built[:n, :n].to(torch.int8)
        else:
            self.anc8 = visibility.to(device=dev, dtype=torch.int8)
        self.anc = self.anc8.bool()
        self.anc_f = self.anc8.float()
        self.parents_dev = torch.tensor(self.parents, dtype=torch.long, device=dev)
        self.conv_index_cpu = _conv_windows(self.parents, conv_kernel)
        self.conv_index = torch.tensor(self.conv_index_cpu, dtype=torch.int32, device=dev)
        self.records: dict[int, _LayerRecord] = {}


@contextlib.contextmanager
def tree_verify(parents: list[int], visibility: torch.Tensor, conv_kernel: int, device: torch.device):
    """Activate a TreeContext for the target forward over the tree's nodes (patched GDN layers take the tree
    path while it is active)."""
    global _ACTIVE
    ctx = TreeContext(parents, visibility, conv_kernel, device)
    _ACTIVE = ctx
    try:
        yield ctx
    finally:
        _ACTIVE = None


def chain_tree(length: int) -> tuple[list[int], torch.Tensor]:
    """parents and ancestor visibility of a chain [root, d_1, ..., d_{length-1}] (a chain is the one-path tree)."""
    return list(range(-1, length - 1)), torch.tril(torch.ones(length, length, dtype=torch.bool))


def _tree_forward(layer, hidden_states: torch.Tensor, cache_params, ctx: TreeContext) -> torch.Tensor:
    """A GDN layer over the tree's nodes: the caller's projections (cuBLAS), then this package's kernels for the
    windowed conv, the gates and the tree-restricted delta rule; the output gate norm and out_proj are the layer's
    own modules."""
    from . import ops
    from .tree_gdn_kernel import tree_gdn, tree_prep

    if layer.conv1d.bias is not None or layer.head_k_dim != layer.head_v_dim:
        raise RuntimeError("qwen35_tree: the tree path needs a bias-free conv and equal key / value head dims")
    cache = cache_params.layers[layer.layer_idx]
    tokens = hidden_states[0]                                    # [n, hidden]
    x = layer.in_proj_qkv(tokens)                                # conv inputs [n, conv_dim]
    q, k, v = tree_prep(x, cache.conv_states[0], ctx.conv_index, layer.conv1d.weight.squeeze(1),
                        layer.num_k_heads, layer.num_v_heads, layer.head_k_dim)
    beta, G = ops.tree_gates(layer.in_proj_a(tokens), layer.in_proj_b(tokens), layer.A_log, layer.dt_bias,
                             ctx.parents_dev)
    u, o = tree_gdn(q, k, v, G, beta, cache.recurrent_states[0], ctx.anc8)
    ctx.records[layer.layer_idx] = _LayerRecord(u=u, k=k, G=G, x=x)
    gate = layer.in_proj_z(tokens).view(-1, layer.head_v_dim)
    core = layer.norm(o.view(-1, layer.head_v_dim).to(tokens.dtype), gate)
    return layer.out_proj(core.view(1, tokens.shape[0], -1))


class _GdnRouter:
    """The forward of a patched GDN layer: the tree path while a TreeContext is active, the layer's own forward
    otherwise (same arguments)."""

    def __init__(self, layer, native):
        self.layer = layer
        self.native = native

    def __call__(self, hidden_states, cache_params=None, attention_mask=None, **kwargs):
        ctx = _ACTIVE
        if ctx is None:
            return self.native(hidden_states, cache_params=cache_params, attention_mask=attention_mask, **kwargs)
        return _tree_forward(self.layer, hidden_states, cache_params, ctx)


def hybrid_layers(target) -> list:
    """The target's Gated-DeltaNet layers (HF Qwen3.5 / Qwen3.6 class name)."""
    return [m for m in target.modules() if type(m).__name__ == "Qwen3_5GatedDeltaNet"]


def is_hybrid(target) -> bool:
    return len(hybrid_layers(target)) > 0


def conv_kernel(target) -> int:
    return hybrid_layers(target)[0].conv_kernel_size


def new_cache(target):
    """A cache with GDN layer states for a hybrid target (a bare DynamicCache() builds attention layers only)."""
    from transformers import DynamicCache

    return DynamicCache(config=target.config) if is_hybrid(target) else DynamicCache()


def install(target) -> int:
    """Route every GDN layer of the target through the tree path while a TreeContext is active; returns the
    number of layers newly routed (layers already routed are left as they are)."""
    routed = 0
    for layer in hybrid_layers(target):
        if isinstance(layer.forward, _GdnRouter):
            continue
        layer.forward = _GdnRouter(layer, layer.forward)
        layer._tree_patched = True
        routed += 1
    return routed


@torch.no_grad()
def commit(cache, ctx: TreeContext, accepted: list[int], past_length: int, compact_attention) -> None:
    """Advance every GDN layer to the deepest accepted node a = accepted[-1] and keep only the accepted KV:
    S_a = e^{G_a} S0 + sum_{j on the path} e^{G_a - G_j} k_j u_j^T for all layers in one launch (ops.gdn_commit),
    their conv windows set to node a's in another (ops.conv_commit), in place in the cache's own tensors; then
    compact_attention(cache, past_length, accepted) (qwen35_tree.py:122-148)."""
    from . import ops

    layers = sorted(ctx.records)
    if layers:
        n = ctx.anc.shape[0]
        if any(not (0 <= int(a) < n) for a in accepted):
            raise RuntimeError("commit: accepted node outside the tree")
        recs = [ctx.records[i] for i in layers]
        states = [cache.layers[i].recurrent_states for i in layers]
        convs = [cache.layers[i].conv_states for i in layers]
        ops.gdn_commit([s_[0] if s_.dim() == 4 else s_ for s_ in states], [r.u for r in recs], [r.k for r in recs],
                       [r.G for r in recs], accepted)
        ops.conv_commit([c_[0] if c_.dim() == 3 else c_ for c_ in convs], [r.x for r in recs],
                        ctx.conv_index[accepted[-1]])
    ctx.records.clear()
    compact_attention(cache, past_length, accepted)
