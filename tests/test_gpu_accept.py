"""GPU parity: acceptance (argmax / reproducible sample + walk), the walk alone, verify inputs."""
import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def random_tree(g, W):
    parents = [-1] + [int(torch.randint(0, i, (1,), generator=g)) for i in range(1, W)]
    tokens = [0] * W
    for i in range(1, W):
        # distinct tokens among siblings
        used = {tokens[j] for j in range(1, i) if parents[j] == parents[i]}
        t = int(torch.randint(0, 50, (1,), generator=g))
        while t in used:
            t = (t + 1) % 50
        tokens[i] = t
    return tokens, parents


def python_follow(tokens, parents, posterior, L):
    """tests/sglang_kernels/test_ddtree_kernels.py:12-24 semantics (at most L-1 edges)."""
    children = {}
    for node in range(1, len(parents)):
        if parents[node] >= 0:
            children.setdefault(parents[node], {})[tokens[node]] = node
    accepted, cur = [0], 0
    nxt = posterior[0]
    while nxt in children.get(cur, {}) and len(accepted) < L:
        cur = children[cur][nxt]
        accepted.append(cur)
        nxt = posterior[cur]
    return accepted, nxt


@pytest.mark.parametrize("V", [50, 1000, 151936])
def test_greedy_accept_vs_oracle(V):
    from mfd_b200 import ops
    g = torch.Generator().manual_seed(V)
    bs, W = 3, 17
    trees = [random_tree(g, W) for _ in range(bs)]
    tokens = torch.tensor([t for t, _ in trees])
    parents = torch.tensor([p for _, p in trees])
    logits = torch.randn(bs, W, V, generator=g)
    # force the argmax to follow some edges
    for b in range(bs):
        for i in range(1, W):
            if torch.rand((), generator=g) < 0.7:
                logits[b, parents[b, i], tokens[b, i] % V] = 8.0
    logits = logits.to(torch.bfloat16)
    o = ops.accept(logits.to(DEV), tokens.to(DEV), parents.to(DEV), temperature=0.0)
    bits = logits.view(torch.int16).numpy().astype(np.uint16).reshape(bs * W, V)
    post = oracle.argmax_rows(bits).reshape(bs, W)
    assert np.array_equal(o["posterior"].cpu().numpy(), post)
    assert np.array_equal(post, torch.argmax(logits.float(), -1).numpy())
    for b in range(bs):
        acc, bonus = oracle.follow(tokens[b].numpy(), parents[b].numpy(), post[b])
        n = len(acc) - 1
        assert int(o["accept_len"][b]) == n and int(o["bonus"][b]) == bonus
        assert o["accepted"][b, :n + 1].tolist() == acc


@pytest.mark.parametrize("V,T", [(64, 1.0), (3001, 0.7), (151936, 1.0)])
def test_stochastic_accept_bit_exact_vs_oracle(V, T):
    from mfd_b200 import ops
    g = torch.Generator().manual_seed(V + 7)
    bs, W = 2, 65
    trees = [random_tree(g, W) for _ in range(bs)]
    tokens = torch.tensor([t for t, _ in trees])
    parents = torch.tensor([p for _, p in trees])
    logits = (torch.randn(bs, W, V, generator=g) * 1.5).to(torch.bfloat16)
    u = torch.rand(bs, W, generator=g, dtype=torch.float64)
    o = ops.accept(logits.to(DEV), tokens.to(DEV), parents.to(DEV), temperature=T, uniforms=u.to(DEV))
    bits = logits.view(torch.int16).numpy().astype(np.uint16).reshape(bs * W, V)
    inv_t = float(np.float32(1.0) / np.float32(T))
    post = oracle.sample_rows(bits, inv_t, u.numpy().reshape(-1)).reshape(bs, W)
    assert np.array_equal(o["posterior"].cpu().numpy(), post)
    for b in range(bs):
        acc, bonus = oracle.follow(tokens[b].numpy(), parents[b].numpy(), post[b])
        assert int(o["accept_len"][b]) == len(acc) - 1 and int(o["bonus"][b]) == bonus


def test_sample_tokens_edge_rows_bit_exact():
    """-inf entries, a single finite logit, a peaked row, u at the ends of [0, 1), vocab not a multiple of 8 (rows
    start at unaligned addresses), and a row of all -inf (sampled token V - 1, as the oracle defines it)."""
    from mfd_b200 import ops
    V = 5003
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(8, V, generator=g) * 2).to(torch.bfloat16)
    x[0, ::2] = float("-inf")
    x[1, :] = float("-inf")
    x[1, 4321] = 3.0
    x[2, 17] = 40.0
    x[3, :] = float("-inf")
    u = torch.tensor([0.0, 0.5, 0.999999, 0.3, 0.0, 0.9999999999, 0.25, 0.75], dtype=torch.float64)
    post = ops.sample_tokens(x.to(DEV), temperature=0.8, uniforms=u.to(DEV))
    bits = x.view(torch.int16).numpy().astype(np.uint16)
    inv_t = float(np.float32(1.0) / np.float32(0.8))
    ref = oracle.sample_rows(bits, inv_t, u.numpy())
    assert np.array_equal(post.cpu().numpy(), ref)
    assert int(post[1]) == 4321 and int(post[3]) == V - 1


@pytest.mark.parametrize("scale,shift,T", [(1.5, 0.0, 1.0), (0.5, -3.0, 0.1), (3.0, 0.0, 10.0), (0.001, 0.0, 1.0),
                                           (300.0, 20.0, 2.0), (1.0, -50.0, 0.7)])
def test_sample_tokens_value_regimes(scale, shift, T):
    """Rows whose max is positive, negative, zero (all logits <= 0), tiny or large, at small and large
    temperatures (block maxima far apart, weights that underflow to 0 within a block or across blocks): the
    one-pass kernel's block sums, block weights and fixed-order run sums reproduce the oracle's token bit for
    bit."""
    from mfd_b200 import ops
    V = 151936
    g = torch.Generator().manual_seed(int(scale * 7 + T * 13))
    x = (torch.randn(6, V, generator=g) * scale + shift).to(torch.bfloat16)
    if shift == 0.0 and scale == 0.001:
        x = -x.abs()
        x[:, 7] = 0.0  # max exactly 0
    u = torch.rand(6, generator=g, dtype=torch.float64)
    post = ops.sample_tokens(x.to(DEV), temperature=T, uniforms=u.to(DEV))
    bits = x.view(torch.int16).numpy().astype(np.uint16)
    inv_t = float(np.float32(1.0) / np.float32(T))
    assert np.array_equal(post.cpu().numpy(), oracle.sample_rows(bits, inv_t, u.numpy()))


def test_sglang_follow_outputs():
    from mfd_b200 import ddtree_utils
    g = torch.Generator().manual_seed(11)
    L = 16
    for trial in range(20):
        bs = 1 + trial % 3
        W = (17, 33, 65)[trial % 3]
        trees = [random_tree(g, W) for _ in range(bs)]
        vids = torch.tensor([t for t, _ in trees])
        par = torch.tensor([p for _, p in trees])
        posterior = torch.randint(0, 50, (bs, W), generator=g)
        for b in range(bs):
            for node in range(1, W):
                if torch.rand((), generator=g) < 0.7:
                    posterior[b, par[b, node]] = vids[b, node]
        window = torch.randint(1, 10 ** 6, (bs, W), generator=g)
        prefix = torch.randint(5, 300, (bs,), generator=g)
        outs = dict(
            accept_len_out=torch.empty(bs, dtype=torch.int32, device=DEV),
            commit_lens_out=torch.empty(bs, dtype=torch.int32, device=DEV),
            bonus_out=torch.empty(bs, dtype=torch.int64, device=DEV),
            out_tokens_out=torch.empty((bs, L), dtype=torch.int64, device=DEV),
            new_seq_lens_out=torch.empty(bs, dtype=torch.int64, device=DEV),
            move_src_out=torch.empty((bs, L), dtype=torch.int64, device=DEV),
            move_tgt_out=torch.empty((bs, L), dtype=torch.int64, device=DEV),
            hidden_index_out=torch.empty((bs, L), dtype=torch.int64, device=DEV),
        )
        ddtree_utils.ddtree_follow(posterior=posterior.to(DEV), verify_ids=vids.to(DEV), parents=par.to(DEV),
                                   window=window.to(DEV), prefix_lens=prefix.to(DEV), **outs)
        o = {k: v.cpu() for k, v in outs.items()}
        for b in range(bs):
            acc, bonus = python_follow(vids[b].tolist(), par[b].tolist(), posterior[b].tolist(), L)
            n = len(acc) - 1
            assert int(o["accept_len_out"][b]) == n
            assert int(o["commit_lens_out"][b]) == n + 1
            assert int(o["bonus_out"][b]) == bonus
            assert int(o["new_seq_lens_out"][b]) == int(prefix[b]) + n + 1
            emitted = [posterior[b, a].item() for a in acc[:-1]] + [bonus]
            assert o["out_tokens_out"][b, : n + 1].tolist() == emitted
            assert o["hidden_index_out"][b, : n + 1].tolist() == [b * W + a for a in acc]
            assert o["move_src_out"][b, : n + 1].tolist() == [int(window[b, a]) for a in acc]
            assert o["move_tgt_out"][b, : n + 1].tolist() == [int(window[b, j]) for j in range(n + 1)]
            assert (o["move_src_out"][b, n + 1:] == 0).all() and (o["move_tgt_out"][b, n + 1:] == 0).all()


def test_verify_inputs_vs_reference_semantics():
    from mfd_b200 import ddtree_utils
    from oracle import oracle as orc
    g = torch.Generator().manual_seed(2)
    L = 16
    for trial in range(12):
        bs = 1 + trial % 3
        B = (16, 32, 64)[trial % 3]
        W = B + 1
        K = 1
        lp_logits = (torch.randn(bs, K, L - 1, 300, generator=g) * 3).to(torch.bfloat16).float()
        top, ids = torch.topk(lp_logits, k=B, dim=-1)
        logp = (top - torch.logsumexp(lp_logits, -1, keepdim=True)).float().contiguous()
        tree_np, counts = orc.build_trees(logp.numpy(), ids.to(torch.int32).numpy(), np.zeros((bs, K), np.float32), B)
        tree = torch.from_numpy(tree_np)
        prefix = torch.randint(5, 300, (bs,), generator=g)
        roots = torch.randint(0, 300, (bs,), generator=g)
        offsets, off = [], 0
        for p in prefix.tolist():
            offsets.append(off)
            off += W * (p + W)
        tg = tree.to(DEV)
        mask = torch.empty(off, dtype=torch.bool, device=DEV)
        vids = torch.empty((bs, W), dtype=torch.long, device=DEV)
        vpos = torch.empty((bs, W), dtype=torch.long, device=DEV)
        ddtree_utils.ddtree_verify_inputs(root_tokens=roots.to(DEV), prefix_lens=prefix.to(DEV), tokens=tg[:, 0],
                                          depths=tg[:, 1], parents=tg[:, 2],
                                          mask_offsets=torch.tensor(offsets, device=DEV), ids_out=vids,
                                          positions_out=vpos, mask_out=mask, max_depth=L - 1)
        mc = mask.cpu()
        for b in range(bs):
            p = int(prefix[b])
            ref_ids = tree[b, 0].clone()
            ref_ids[0] = roots[b]
            assert torch.equal(vids[b].cpu(), ref_ids)
            assert torch.equal(vpos[b].cpu(), p + tree[b, 1])
            m = mc[offsets[b]: offsets[b] + W * (p + W)].view(W, p + W)
            assert m[:, :p].all()
            assert torch.equal(m[:, p:], ddtree_utils.ancestor_visibility_reference(tree[b, 2]))
