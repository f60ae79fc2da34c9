"""Tree gated-delta-rule verification (mfd_tree_gdn) and its input prep (mfd_tree_prep) against the oracle.

The oracle's chunk form is pinned to the reference's node-by-node recurrence in test_oracle_golden.py; here the
GPU path is compared with it on the same bf16-rounded inputs: u, o within 2e-2 absolute (bf16 tolerance; the
fp32 kernel lands near 1e-5) and the per-node float32 states within 1e-3 relative to their largest entry."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle
from tests._golden import cases

DEV = "cuda"


def random_parents(n, seed):
    g = np.random.default_rng(seed)
    return np.array([-1] + [int(g.integers(0, i)) for i in range(1, n)], np.int64)


def gdn_inputs(n, H, HK, D, parents, seed, s0_std=0.02):
    """q, k N(0,1) l2-normalised (q also scaled by D^-0.5), v N(0,1) bf16, beta = sigmoid(N(0,1)),
    g = -softplus(N(0,1)) summed along root paths, S0 N(0, s0_std)."""
    gen = torch.Generator().manual_seed(seed)
    q = F.normalize(torch.randn(n, HK, D, generator=gen), dim=-1) * D ** -0.5
    k = F.normalize(torch.randn(n, HK, D, generator=gen), dim=-1)
    v = torch.randn(n, H, D, generator=gen)
    beta = torch.sigmoid(torch.randn(n, H, generator=gen))
    g = -F.softplus(torch.randn(n, H, generator=gen))
    s0 = torch.randn(H, D, D, generator=gen) * s0_std
    G = torch.zeros(n, H)
    for i in range(n):
        G[i] = (G[parents[i]] if parents[i] >= 0 else 0) + g[i]
    return q.bfloat16(), k.bfloat16(), v.bfloat16(), G, beta, s0


def anc8_of(parents):
    return torch.from_numpy(oracle.visibility(parents).astype(np.int8))


def check_against_oracle(q, k, v, G, beta, s0, parents, emit_states):
    from mfd_b200 import ops
    anc = anc8_of(parents)
    status = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    res = ops.tree_gdn(q.to(DEV), k.to(DEV), v.to(DEV), G.to(DEV), beta.to(DEV), s0.to(DEV), anc.to(DEV),
                       emit_states=emit_states, status=status)
    assert int(status.item()) == 0
    ru, ro, rst = oracle.tree_gdn(q.float().numpy(), k.float().numpy(), v.float().numpy(), G.numpy(), beta.numpy(),
                                  s0.numpy(), parents, emit_states=emit_states)
    np.testing.assert_allclose(res[0].cpu().numpy(), ru, rtol=0, atol=2e-2)
    np.testing.assert_allclose(res[1].cpu().numpy(), ro, rtol=0, atol=2e-2)
    err_u = np.abs(res[0].cpu().numpy() - ru).max()
    err_o = np.abs(res[1].cpu().numpy() - ro).max()
    assert err_u < 1e-3 * max(1.0, np.abs(ru).max()) and err_o < 1e-3 * max(1.0, np.abs(ro).max())
    if emit_states:
        st = res[2].cpu().numpy()
        scale = np.abs(rst).max()
        assert np.abs(st - rst).max() <= 1e-3 * scale


@pytest.mark.gpu
@pytest.mark.parametrize("n,H,HK,D,seed", [(65, 32, 16, 128, 0), (64, 32, 16, 128, 1), (37, 4, 4, 64, 2),
                                          (128, 8, 2, 128, 3), (1, 2, 1, 128, 4), (200, 8, 4, 128, 6),
                                          (257, 32, 16, 128, 9), (257, 8, 4, 128, 10), (384, 4, 2, 128, 11)])
def test_tree_gdn_vs_oracle(n, H, HK, D, seed):
    """Odd seeds check u and o, even seeds the per-node states too; 200, 257 and 384 nodes span two and three
    128-node tiles (257 = a budget-256 tree with its root, the size the reference's guide times)."""
    parents = random_parents(n, seed)
    check_against_oracle(*gdn_inputs(n, H, HK, D, parents, seed), parents, emit_states=(seed % 2 == 0))


@pytest.mark.gpu
def test_tree_gdn_chain_and_star():
    n = 128
    chain = np.arange(-1, n - 1, dtype=np.int64)  # the longest root paths the kernel accepts
    check_against_oracle(*gdn_inputs(n, 4, 2, 128, chain, 7), chain, emit_states=True)
    star = np.array([-1] + [0] * (n - 1), np.int64)
    check_against_oracle(*gdn_inputs(n, 4, 2, 128, star, 8), star, emit_states=True)


@pytest.mark.gpu
def test_tree_gdn_reports_ancestor_pairs_beyond_capacity():
    """A 257-node chain has 33153 ancestor pairs, more than the u/o kernel holds at that size: the status word says
    MFD_ERR_CAPACITY (4) instead of computing from a truncated path table."""
    from mfd_b200 import ops
    n = 257
    chain = np.arange(-1, n - 1, dtype=np.int64)
    q, k, v, G, beta, s0 = gdn_inputs(n, 2, 1, 128, chain, 12)
    status = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    ops.tree_gdn(q.to(DEV), k.to(DEV), v.to(DEV), G.to(DEV), beta.to(DEV), s0.to(DEV), anc8_of(chain).to(DEV),
                 status=status)
    assert int(status.item()) == 4


@pytest.mark.gpu
def test_tree_gdn_reference_recurrence_cases():
    """The reference test's trees (tests/test_gdn_tree_math.py tree_case, Dk 16, Dv 12): the GPU output on
    bf16-rounded inputs against the float64 node-by-node recurrence on the exact inputs."""
    from mfd_b200 import ops
    for c in cases("gdn_tree.npz"):
        n, dk = c["k"].shape
        par = c["parents"]
        G = np.zeros(n)
        for j in range(n):
            G[j] = (G[par[j]] if par[j] >= 0 else 0.0) + c["g"][j]
        q = torch.from_numpy(c["q"][:, None, :]).bfloat16()
        k = torch.from_numpy(c["k"][:, None, :]).bfloat16()
        v = torch.from_numpy(c["v"][:, None, :]).bfloat16()
        s0 = torch.from_numpy(c["s0"].T[None].copy()).float()
        u, o, st = ops.tree_gdn(q.to(DEV), k.to(DEV), v.to(DEV), torch.from_numpy(G[:, None]).float().to(DEV),
                                torch.from_numpy(c["beta"][:, None]).float().to(DEV), s0.to(DEV),
                                anc8_of(par).to(DEV), emit_states=True)
        # bf16 rounding of q, k, v (relative 2^-9) is the only approximation: within 0.5% of the largest entry
        np.testing.assert_allclose(o[:, 0].cpu().numpy(), c["o"], rtol=0, atol=5e-3 * np.abs(c["o"]).max())
        np.testing.assert_allclose(st[:, 0].cpu().numpy().transpose(0, 2, 1), c["states"], rtol=0,
                                   atol=5e-3 * np.abs(c["states"]).max())
        check_against_oracle(q, k, v, torch.from_numpy(G[:, None]).float(),
                             torch.from_numpy(c["beta"][:, None]).float(), s0, par, emit_states=True)


@pytest.mark.gpu
def test_tree_gdn_rejects_a_mask_that_is_not_a_tree():
    from mfd_b200 import ops
    n = 8
    q, k, v, G, beta, s0 = gdn_inputs(n, 2, 1, 128, random_parents(n, 0), 0)
    anc = anc8_of(np.array([-1, 0, 0, 1, 1, 2, 2, 3]))
    anc[5, 1] = 1  # node 5 claims ancestors 1 and 2, which lie on different branches
    status = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    ops.tree_gdn(q.to(DEV), k.to(DEV), v.to(DEV), G.to(DEV), beta.to(DEV), s0.to(DEV), anc.to(DEV), status=status)
    assert int(status.item()) == 1


@pytest.mark.gpu
def test_commit_of_a_path_matches_emitted_node_state():
    """mfd_gdn_commit at the end of a root path equals the state mfd_tree_gdn emits for that node, and both equal
    the commit formula (oracle.commit_state, float64)."""
    from mfd_b200 import ops
    n = 65
    parents = random_parents(n, 11)
    q, k, v, G, beta, s0 = gdn_inputs(n, 8, 4, 128, parents, 11)
    u, o, st = ops.tree_gdn(q.to(DEV), k.to(DEV), v.to(DEV), G.to(DEV), beta.to(DEV), s0.to(DEV),
                            anc8_of(parents).to(DEV), emit_states=True)
    leaf = n - 1
    path = [leaf]
    while parents[path[-1]] >= 0:
        path.append(int(parents[path[-1]]))
    path = path[::-1]
    S = s0.float().clone().to(DEV)
    ops.gdn_commit([S], [u], [k.to(DEV)], [G.float().to(DEV)], path)
    torch.testing.assert_close(S, st[leaf], rtol=0, atol=1e-5)
    ref = oracle.commit_state(s0.numpy(), u.cpu().numpy(), k.float().numpy(), G.float().numpy(), path)
    np.testing.assert_allclose(S.cpu().numpy(), ref, rtol=0, atol=1e-4 * float(np.abs(ref).max()))


# ------------------------------------------------------------------------------------------------ tree_prep

def prep_inputs(n, HK, H, D, kc, parents, seed):
    from mfd_b200 import qwen35_tree
    gen = torch.Generator().manual_seed(seed)
    cd = (2 * HK + H) * D
    x = torch.randn(n, cd, generator=gen).bfloat16()
    cs = torch.randn(cd, kc, generator=gen).bfloat16()
    w = (torch.randn(cd, kc, generator=gen) * 0.5).bfloat16()
    vis = torch.from_numpy(oracle.visibility(parents))
    ctx = qwen35_tree.TreeContext([int(p) for p in parents], vis, kc, torch.device("cpu"))
    return x, cs, w, ctx.conv_index


def test_prep_oracle_is_the_causal_conv_on_a_chain():
    """On a chain the windowed convolution is torch's causal depthwise conv over [cached inputs ; tokens]."""
    n, HK, H, D, kc = 9, 2, 4, 16, 4
    chain = np.arange(-1, n - 1, dtype=np.int64)
    x, cs, w, idx = prep_inputs(n, HK, H, D, kc, chain, 0)
    q, k, v = oracle.tree_prep(x.float().numpy(), cs.float().numpy(), idx.numpy(), w.float().numpy(), HK, H, D,
                               D ** -0.5)
    seq = torch.cat([cs.float(), x.float().T], dim=1)  # [CD, KC + n]
    conv = F.conv1d(seq[None], w.float()[:, None, :], groups=seq.shape[0])[0, :, 1:].T  # node i: window ending at i
    y = F.silu(conv).bfloat16().float()
    qr = F.normalize(y[:, : HK * D].reshape(n, HK, D), dim=-1, eps=0) * D ** -0.5
    kr = F.normalize(y[:, HK * D: 2 * HK * D].reshape(n, HK, D), dim=-1, eps=0)
    vr = y[:, 2 * HK * D:].reshape(n, H, D)
    np.testing.assert_allclose(q, qr.bfloat16().float().numpy(), rtol=1e-2, atol=1e-3)
    np.testing.assert_allclose(k, kr.bfloat16().float().numpy(), rtol=1e-2, atol=1e-3)
    np.testing.assert_array_equal(v, vr.numpy())


@pytest.mark.gpu
@pytest.mark.parametrize("n,HK,H,D,seed", [(65, 16, 32, 128, 0), (20, 2, 4, 64, 1)])
def test_tree_prep_vs_oracle(n, HK, H, D, seed):
    from mfd_b200 import ops
    parents = random_parents(n, seed)
    x, cs, w, idx = prep_inputs(n, HK, H, D, 4, parents, seed)
    q, k, v = ops.tree_prep(x.to(DEV), cs.to(DEV), idx.to(DEV), w.to(DEV), HK, H, D)
    rq, rk, rv = oracle.tree_prep(x.float().numpy(), cs.float().numpy(), idx.numpy(), w.float().numpy(), HK, H, D,
                                  D ** -0.5)
    # bf16 outputs: at most one bf16 rounding step apart
    np.testing.assert_allclose(q.float().cpu().numpy(), rq, rtol=8e-3, atol=1e-6)
    np.testing.assert_allclose(k.float().cpu().numpy(), rk, rtol=8e-3, atol=1e-6)
    np.testing.assert_allclose(v.float().cpu().numpy(), rv, rtol=8e-3, atol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("n,H,dtype", [(65, 32, torch.bfloat16), (257, 16, torch.float32), (1, 4, torch.bfloat16)])
def test_tree_gates_vs_oracle(n, H, dtype):
    """beta, the softplus log decay and its sum along each root path (mfd_tree_gates) against the reference's
    formulas in float64 (oracle.tree_gates: sigmoid, -exp(A_log) softplus(a + dt_bias), G = anc @ g); inputs reach
    softplus's linear branch (a + dt_bias > 20)."""
    from mfd_b200 import ops
    g = torch.Generator().manual_seed(n + H)
    parents = random_parents(n, n)
    a = (torch.randn(n, H, generator=g) * 3).to(dtype)
    a[0, 0] = 30.0
    b = torch.randn(n, H, generator=g).to(dtype)
    a_log = torch.randn(H, generator=g) * 0.5
    dt_bias = torch.randn(H, generator=g)
    beta, G = ops.tree_gates(a.to(DEV), b.to(DEV), a_log.to(DEV), dt_bias.to(DEV),
                             torch.from_numpy(np.asarray(parents)).to(DEV))
    rb, rG = oracle.tree_gates(a.float().numpy(), b.float().numpy(), a_log.numpy(), dt_bias.numpy(), parents)
    np.testing.assert_allclose(beta.cpu().numpy(), rb, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(G.cpu().numpy(), rG, rtol=1e-4, atol=1e-4)
