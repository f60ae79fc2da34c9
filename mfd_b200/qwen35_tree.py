"""Drop-in for inference/hf/qwen35_tree.py: exact tree verification of Gated-DeltaNet layers.

TreeContext / tree_verify / chain_tree keep the reference's signatures (qwen35_tree.py:33-64, 169-171):
ancestor matrices of the tree and each node's causal-conv window gathered through parent pointers
(oldest first, indices into [cached conv state ; nodes]).  _tree_forward / install route a patched layer's
GDN core through mfd_b200.tree_gdn_kernel.tree_gdn (the B200 kernel); commit (the state at the deepest
accepted node and its conv window, qwen35_tree.py:122-148) runs the mfd_gdn_commit / mfd_conv_commit kernels.
"""

from __future__ import annotations

import contextlib

import torch
import torch.nn.functional as F

_ACTIVE = None


class TreeContext:
    def __init__(self, parents: list[int], visibility: torch.Tensor, conv_kernel: int, device: torch.device):
        n = len(parents)
        self.parents = list(parents)
        self.anc = visibility.to(device=device, dtype=torch.bool)  # [n, n]: row i = ancestors of i and i
        self.anc_f = self.anc.float()
        self.anc8 = self.anc.to(torch.int8)
        windows = []
        for i in range(n):
            # newest first: the node itself, then its ancestors, then the cached inputs, newest cached first
            newest_first = [conv_kernel + i]
            p = parents[i]
            while len(newest_first) < conv_kernel and p >= 0:
                newest_first.append(conv_kernel + p)
                p = parents[p]
            cached = conv_kernel - 1
            while len(newest_first) < conv_kernel:
                newest_first.append(cached)
                cached -= 1
            windows.append(list(reversed(newest_first)))
        self.conv_index_cpu = windows
        self.conv_index = torch.tensor(windows, dtype=torch.int32, device=device)
        self.stash = {}


@contextlib.contextmanager
def tree_verify(parents: list[int], visibility: torch.Tensor, conv_kernel: int, device: torch.device):
    global _ACTIVE
    ctx = TreeContext(parents, visibility, conv_kernel, device)
    _ACTIVE = ctx
    try:
        yield ctx
    finally:
        _ACTIVE = None


def chain_tree(length: int) -> tuple[list[int], torch.Tensor]:
    """parents and ancestor visibility of a chain [root, d_1, ..., d_{length-1}]."""
    return [-1] + list(range(length - 1)), torch.ones(length, length, dtype=torch.bool).tril()


def _tree_forward(layer, hidden_states: torch.Tensor, cache_params, ctx: TreeContext) -> torch.Tensor:
    from .tree_gdn_kernel import tree_gdn, tree_prep

    assert layer.conv1d.bias is None and layer.head_k_dim == layer.head_v_dim
    state = cache_params.layers[layer.layer_idx]
    h = hidden_states[0]
    n, dtype = h.shape[0], h.dtype
    x = layer.in_proj_qkv(h)
    q, k, v = tree_prep(x, state.conv_states[0], ctx.conv_index, layer.conv1d.weight.squeeze(1),
                        layer.num_k_heads, layer.num_v_heads, layer.head_k_dim)
    beta = layer.in_proj_b(h).float().sigmoid()
    g = -layer.A_log.float().exp() * F.softplus(layer.in_proj_a(h).float() + layer.dt_bias.float())
    G = ctx.anc_f @ g
    u, o = tree_gdn(q, k, v, G, beta, state.recurrent_states[0], ctx.anc8)
    z = layer.in_proj_z(h).reshape(-1, layer.head_v_dim)
    core = layer.norm(o.reshape(-1, layer.head_v_dim).to(dtype), z)
    ctx.stash[layer.layer_idx] = (u, k, G, x)
    return layer.out_proj(core.reshape(1, n, -1))


def install(target) -> int:
    """Route the target's GDN layers through _tree_forward while a TreeContext is active."""
    count = 0
    for module in target.modules():
        if type(module).__name__ != "Qwen3_5GatedDeltaNet" or getattr(module, "_tree_patched", False):
            continue
        native = module.forward

        def forward(hidden_states, cache_params=None, attention_mask=None, _native=native, _layer=module, **kwargs):
            if _ACTIVE is None:
                return _native(hidden_states, cache_params=cache_params, attention_mask=attention_mask, **kwargs)
            return _tree_forward(_layer, hidden_states, cache_params, _ACTIVE)

        module.forward = forward
        module._tree_patched = True
        count += 1
    return count


@torch.no_grad()
def commit(cache, ctx: TreeContext, accepted: list[int], past_length: int, compact_attention) -> None:
    """Advance every GDN layer to the deepest accepted node and keep only the accepted KV (qwen35_tree.py:122-148):
    the states S_a of all layers in one launch (ops.gdn_commit) and their conv windows in another (ops.conv_commit),
    in place in the cache's own state tensors; then compact_attention(cache, past_length, accepted)."""
    from . import ops

    layers = sorted(ctx.stash)
    if layers:
        last = accepted[-1]
        n = ctx.anc.shape[0]
        if any(not (0 <= int(a) < n) for a in accepted):
            raise RuntimeError("commit: accepted node outside the tree")
        states = [cache.layers[i].recurrent_states for i in layers]
        convs = [cache.layers[i].conv_states for i in layers]
        ops.gdn_commit([s_[0] if s_.dim() == 4 else s_ for s_ in states], [ctx.stash[i][0] for i in layers],
                       [ctx.stash[i][1] for i in layers], [ctx.stash[i][2] for i in layers], accepted)
        ops.conv_commit([c_[0] if c_.dim() == 3 else c_ for c_ in convs], [ctx.stash[i][3] for i in layers],
                        ctx.conv_index[last])
    ctx.stash.clear()
    compact_attention(cache, past_length, accepted)


@torch.no_grad()
def commit_state(s0: torch.Tensor, u: torch.Tensor, k: torch.Tensor, G: torch.Tensor, path: list[int]) -> torch.Tensor:
    """State at the deepest accepted node a = path[-1]: S_a = e^{G_a} S0 + sum_{j on path} e^{G_a - G_j} k_j u_j^T
    (qwen35_tree.py:134-137).  s0 [H, Dk, Dv], u [n, H, Dv], k [n, HK, Dk], G [n, H] -> [H, Dk, Dv] float32."""
    last = path[-1]
    idx = torch.tensor(path, dtype=torch.long, device=u.device)
    uu = u[idx].transpose(0, 1).float()                     # [H, p, Dv]
    kk = k[idx].float().transpose(0, 1)                      # [HK, p, Dk]
    rep = uu.shape[0] // kk.shape[0]
    if rep > 1:
        kk = kk.repeat_interleave(rep, dim=0)
    GG = G.transpose(0, 1).float()                           # [H, n]
    w = (GG[:, last:last + 1] - GG[:, idx]).exp()            # [H, p]
    return GG[:, last].exp()[:, None, None] * s0.float() + (kk * w[..., None]).transpose(-1, -2) @ uu
