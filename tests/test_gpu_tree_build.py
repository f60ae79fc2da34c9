"""GPU parity: logits step (mfd_topk_logz) and exact tree builders (mfd_build_trees) vs the oracle and the
reference fixtures.  Integer outputs are compared bit for bit; log-probabilities within 2e-6 absolute
(the reference's own check allows 1e-4, inference/hf/tree_logits.py:58)."""
import numpy as np
import pytest
import torch

from oracle import oracle
from tests._golden import cases

pytestmark = pytest.mark.gpu

DEV = "cuda"
V0, K0, L0, B0 = 151936, 8, 16, 64


def config0_logits(seed, K=K0, L=L0, V=V0, sharp=False):
    """N(0,1) logits, 4 ids per (mode, position) boosted by U(4,10) (sharp: 1 id by U(12,16))."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(K, L, V, generator=g)
    nb = 1 if sharp else 4
    ids = torch.randint(0, V, (K, L, nb), generator=g)
    boost = torch.rand(K, L, nb, generator=g) * 4 + 12 if sharp else torch.rand(K, L, nb, generator=g) * 6 + 4
    x.scatter_add_(2, ids, boost)
    return x


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("R,V,k", [(1, 64, 64), (3, 1000, 8), (5, 4099, 100), (2, 70000, 256), (128, V0, 64), (7, 333, 1)])
def test_topk_logz_vs_oracle(dtype, R, V, k):
    from mfd_b200 import ops
    g = torch.Generator().manual_seed(R * 1000 + V + k)
    x = (torch.randn(R, V, generator=g) * 3).to(dtype)
    if dtype == torch.bfloat16 and V < 5000:
        x = ((x.float() * 2).round() / 2).to(dtype)  # many exact ties
    top, ids, lz = ops.topk_logz(x.to(DEV), k)
    xo = x.float().numpy()
    ref_lp, ref_ids, ref_lz = oracle.topk_logz(xo, k)
    assert np.array_equal(ids.cpu().numpy(), ref_ids)
    np.testing.assert_allclose(lz.cpu().numpy(), ref_lz, rtol=0, atol=4e-6 * max(1.0, float(np.abs(ref_lz).max()) / 8))
    np.testing.assert_allclose(top.cpu().numpy(), ref_lp, rtol=0, atol=8e-6)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("pattern", ["constant", "two_levels", "first_batch_high", "ascending", "few_values"])
def test_topk_adversarial_rows(dtype, pattern):
    """Rows that defeat the speculative floor: every element passes it (constant and tie-heavy rows overflow the
    candidate buffer, so the piece is rescanned with a raised key threshold, twice when ties fill it again), or the
    first batch overstates the row (too few candidates, rescan against the valid bound).  Ties order by index."""
    from mfd_b200 import ops
    R, V, k = 24, 151936, 64
    g = torch.Generator().manual_seed(11)
    if pattern == "constant":
        x = torch.full((R, V), 0.5)
    elif pattern == "two_levels":
        x = (torch.rand(R, V, generator=g) < 0.3).float()
    elif pattern == "first_batch_high":
        x = torch.randn(R, V, generator=g)
        x[:, :9000] += 8.0
    elif pattern == "ascending":
        x = torch.linspace(-4, 4, V).repeat(R, 1)
    else:
        x = torch.randint(0, 6, (R, V), generator=g).float() * 0.25
    x = x.to(dtype)
    top, ids, lz = ops.topk_logz(x.to(DEV), k)
    ref_lp, ref_ids, ref_lz = oracle.topk_logz(x.float().numpy(), k)
    assert np.array_equal(ids.cpu().numpy(), ref_ids)
    np.testing.assert_allclose(lz.cpu().numpy(), ref_lz, rtol=0, atol=4e-6 * max(1.0, float(np.abs(ref_lz).max()) / 8))
    np.testing.assert_allclose(top.cpu().numpy(), ref_lp, rtol=0, atol=8e-6)


def test_topk_repeatable_at_batch_size():
    """The bench's logits-step size (4096 rows): two calls give identical ids and log Z."""
    from mfd_b200 import ops
    x = torch.randn(4096, V0, generator=torch.Generator(device=DEV).manual_seed(5), device=DEV)
    a = [t.clone() for t in ops.topk_logz(x, 64, ids_dtype=torch.int32)]
    b = ops.topk_logz(x, 64, ids_dtype=torch.int32)
    assert torch.equal(a[1], b[1]) and torch.equal(a[2], b[2]) and torch.equal(a[0], b[0])
    rows = torch.arange(0, 4096, 97)
    ref_lp, ref_ids, _ = oracle.topk_logz(x[rows].cpu().numpy(), 64)
    assert np.array_equal(a[1][rows].cpu().numpy(), ref_ids)


def test_topk_strided_rows_and_int32_ids():
    from mfd_b200 import ops
    g = torch.Generator().manual_seed(3)
    base = torch.randn(6, 5003, generator=g)
    x = base.to(DEV)[:, 1:5001]  # misaligned starts, stride 5003
    top, ids, lz = ops.topk_logz(x, 33, ids_dtype=torch.int32)
    ref_lp, ref_ids, _ = oracle.topk_logz(base[:, 1:5001].numpy(), 33)
    assert ids.dtype == torch.int32 and np.array_equal(ids.cpu().numpy(), ref_ids)
    np.testing.assert_allclose(top.cpu().numpy(), ref_lp, rtol=0, atol=8e-6)


def test_builders_on_reference_tie_cases():
    from mfd_b200 import ops
    for i, c in enumerate(cases("candidates_ties.npz")):
        B = int(c["budget"])
        lp = torch.from_numpy(c["lp"]).to(DEV)[None]
        ids = torch.from_numpy(c["ids"]).to(DEV)[None]
        pr = torch.from_numpy(c["prior"]).to(DEV)[None]
        tree, counts, anc, vis = ops.build_trees(lp, ids, pr, B, single=bool(int(c["single"])), want_vis=True)
        n = int(counts[0])
        t = tree[0].cpu().numpy()
        assert n == len(c["tokens"]), f"case {i}"
        assert np.array_equal(t[0, 1:n + 1], c["tokens"]), f"case {i}"
        assert np.array_equal(t[1, 1:n + 1], c["depths"]), f"case {i}"
        assert np.array_equal(t[2, :n + 1], c["parents"]), f"case {i}"
        assert np.array_equal(vis[0, :n + 1, :n + 1].cpu().numpy().astype(bool), c["vis"]), f"case {i}"


def test_batched_builder_matches_reference_sglang_layout():
    from mfd_b200 import ddtree_utils
    for i, c in enumerate(cases("sglang_build_trees.npz")):
        bs = c["lp"].shape[0]
        B = int(c["budget"])
        tree = torch.empty((bs, 3, B + 1), dtype=torch.long, device=DEV)
        counts = torch.empty((bs,), dtype=torch.long, device=DEV)
        ddtree_utils.build_trees(top_log_probs=torch.from_numpy(c["lp"]).to(DEV),
                                 top_ids=torch.from_numpy(c["ids"]).to(DEV),
                                 log_prior=torch.from_numpy(c["prior"]).to(DEV), bs=bs, budget=B, tree=tree,
                                 counts=counts)
        assert np.array_equal(tree.cpu().numpy(), c["tree"]), f"case {i}"
        assert np.array_equal(counts.cpu().numpy(), c["counts"]), f"case {i}"
        # the host-signature variant writes into CPU tensors
        tcpu = torch.empty((bs, 3, B + 1), dtype=torch.long)
        ccpu = torch.empty((bs,), dtype=torch.long)
        ddtree_utils.build_trees_cpu(top_log_probs=torch.from_numpy(c["lp"]), top_ids=torch.from_numpy(c["ids"]),
                                     log_prior=torch.from_numpy(c["prior"]), bs=bs, budget=B, tree=tcpu, counts=ccpu)
        assert np.array_equal(tcpu.numpy(), c["tree"]), f"case {i} (cpu signature)"


def test_hf_build_mixture_tree_end_to_end_vs_reference():
    from mfd_b200 import ddtree
    for i, c in enumerate(cases("mixture_e2e.npz")):
        logits = torch.from_numpy(c["logits"]).to(DEV)
        B = int(c["budget"])
        if int(c["single"]):
            out = ddtree.build_ddtree_tree(logits[0], B)
        else:
            out = ddtree.build_mixture_tree(logits, torch.from_numpy(c["prior"]).to(DEV), B)
        assert np.array_equal(out[0].numpy(), c["tokens"]), f"case {i}"
        assert np.array_equal(out[1].numpy(), c["depths"]), f"case {i}"
        assert out[2] == c["parents"].tolist(), f"case {i}"
        assert np.array_equal(out[4].numpy(), c["vis"]), f"case {i}"
        acc, bonus = ddtree.follow_verified_tree(out[3], torch.from_numpy(c["post"]).view(1, -1))
        assert acc == c["accepted"].tolist() and bonus == int(c["bonus"]), f"case {i} walk"


@pytest.mark.parametrize("seed", range(4))
@pytest.mark.parametrize("sharp", [False, True])
def test_config0_tree_vs_oracle(seed, sharp):
    """Full config-0 size: GPU top-k/logZ + GPU heap == oracle heap fed with the GPU's candidates (bit-exact),
    and == the oracle's own candidates unless a score near-tie below 1e-5 separates them."""
    from mfd_b200 import ops
    x = config0_logits(seed, sharp=sharp)
    xd = x.to(DEV)
    top, ids, _ = ops.topk_logz(xd.view(K0 * L0, V0), B0, ids_dtype=torch.int32)
    prior = torch.zeros(1, K0, device=DEV)
    tree, counts, anc, _ = ops.build_trees(top.view(1, K0, L0, B0), ids.view(1, K0, L0, B0), prior, B0)
    n = int(counts[0])
    t = tree[0].cpu().numpy()
    lp_np = top.view(K0, L0, B0).cpu().numpy()
    ids_np = ids.view(K0, L0, B0).cpu().numpy().astype(np.int64)
    tok, dep, par = oracle.build_mixture(lp_np, ids_np, np.zeros(K0, np.float32), B0)
    assert n == len(tok)
    assert np.array_equal(t[0, 1:n + 1], tok) and np.array_equal(t[1, 1:n + 1], dep)
    assert np.array_equal(t[2, :n + 1], par)
    # ancestor bitsets equal the oracle visibility
    vis = oracle.visibility(par)
    a = anc[0].cpu().numpy().view(np.uint64)
    for i in range(n + 1):
        bits = [(int(a[i, j >> 6]) >> (j & 63)) & 1 for j in range(n + 1)]
        assert bits == vis[i].astype(int).tolist()
    # against the oracle's own candidates (float64 log Z)
    ref_lp, ref_ids, _ = oracle.topk_logz(x.view(K0 * L0, V0).numpy(), B0)
    assert np.array_equal(ref_ids.reshape(K0, L0, B0), ids_np)
    assert np.abs(ref_lp.reshape(K0, L0, B0) - lp_np).max() < 1e-5


def test_single_mode_heap_matches_reference_on_ties():
    from mfd_b200 import tree_build_ext
    g = torch.Generator().manual_seed(5)
    for trial in range(20):
        L = 1 + trial % 9
        logits = ((torch.randn(L, 40, generator=g) * 3 * 2).round() / 2).to(torch.bfloat16).float()
        top, ids = torch.topk(logits, 16, dim=-1)
        lp = (top - torch.logsumexp(logits, -1, keepdim=True)).float()
        got = tree_build_ext.build_single(lp, ids, 16)
        tok, dep, par = oracle.build_single(lp.numpy(), ids.numpy(), 16)
        assert np.array_equal(got[0].numpy(), tok) and np.array_equal(got[1].numpy(), dep)
        assert list(got[2]) == par.tolist()


def _candidate_tables(g, K, L, k, vocab, kind):
    """Sorted per-(mode, depth) candidate log-probabilities [K, L, k] f32 and distinct ids per row [K, L, k] i64,
    drawn from a small vocabulary so that modes share prefixes (duplicates across modes)."""
    scale = {"peaked": 4.0, "flat": 0.3}.get(kind, 1.5)
    x = torch.randn(K, L, vocab, generator=g) * scale
    if kind == "peaked":
        x[..., 0] += 12.0
    lp_full = torch.log_softmax(x, -1)
    top, idx = torch.topk(lp_full, k, dim=-1)
    perm = torch.stack([torch.randperm(vocab, generator=g) for _ in range(K * L)]).view(K, L, vocab)
    ids = torch.gather(perm, 2, idx)
    if kind == "quantized":  # exact ties inside modes (the heap's global tie-breaks decide)
        top = (top * 2).round() / 2
    if kind == "dup_modes" and K > 1:  # identical modes: every entry ties across modes
        top[1] = top[0]
        ids[1] = ids[0]
    return top.float().contiguous(), ids.long().contiguous()


@pytest.mark.parametrize("K,L,k,B", [(8, 16, 64, 64), (8, 15, 64, 64), (1, 16, 64, 64), (2, 3, 5, 40),
                                     (3, 5, 16, 95), (16, 16, 32, 64), (8, 4, 64, 96), (8, 16, 64, 200),
                                     (5, 1, 7, 30), (4, 31, 3, 50), (8, 16, 1, 10)])
@pytest.mark.parametrize("kind", ["normal", "peaked", "flat", "quantized", "dup_modes"])
def test_mixture_builder_sweep_vs_oracle(K, L, k, B, kind):
    """Mixture trees over shapes on both sides of the one-warp-per-mode builder's limits (K <= 16, B <= 95),
    with shared prefixes across modes, exact ties across modes (identical modes) and inside modes (quantized
    log-probabilities, replayed by the serial heap), random priors: bit-exact against the oracle heap."""
    from mfd_b200 import ops
    g = torch.Generator().manual_seed(K * 7919 + L * 131 + k * 17 + B + len(kind))
    bs = 5
    lps, idss, priors = [], [], []
    for t in range(bs):
        lp, ids = _candidate_tables(g, K, L, k, max(k, 24), kind)
        lps.append(lp)
        idss.append(ids)
        priors.append(torch.log_softmax(torch.randn(K, generator=g), -1) if t % 2 else torch.zeros(K))
    lp = torch.stack(lps)
    ids = torch.stack(idss)
    pr = torch.stack(priors).float()
    tree, counts, _, _ = ops.build_trees(lp.to(DEV), ids.to(DEV).to(torch.int32), pr.to(DEV), B)
    tree = tree.cpu().numpy()
    counts = counts.cpu().numpy()
    for t in range(bs):
        tok, dep, par = oracle.build_mixture(lp[t].numpy(), ids[t].numpy(), pr[t].numpy(), B)
        n = len(tok)
        assert counts[t] == n, (t, counts[t], n)
        assert np.array_equal(tree[t, 0, 1:n + 1], tok), t
        assert np.array_equal(tree[t, 1, 1:n + 1], dep), t
        assert np.array_equal(tree[t, 2, :n + 1], par), t
        assert (tree[t, 2, n + 1:] == -1).all() and (tree[t, 0, n + 1:] == 0).all()
