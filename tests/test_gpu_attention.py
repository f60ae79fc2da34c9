"""GPU parity: tree-masked GQA verify attention vs the oracle / the reference mask + SDPA.
bf16 inputs, float32 accumulation; tolerance max |err| <= 2e-2 (the reference's kernel checks use 2e-2,
inference/hf/mode_attention.py:242)."""
import numpy as np
import pytest
import torch

from oracle import oracle
from tests._golden import bf16_from_i16, load

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 2e-2


def anc_bits(parents, words):
    n = len(parents)
    a = np.zeros((n, words), np.uint64)
    for i in range(n):
        j = i
        while j >= 0:
            a[i, j >> 6] |= np.uint64(1) << np.uint64(j & 63)
            j = parents[j]
    return torch.from_numpy(a.view(np.int64))


def test_verify_attention_vs_reference_fixture():
    from mfd_b200 import ops
    z = load("verify_attention.npz")
    q = torch.from_numpy(bf16_from_i16(z["q"])).to(torch.bfloat16)  # [1, H, n, D]
    k = torch.from_numpy(bf16_from_i16(z["k"])).to(torch.bfloat16)  # [1, Hkv, P+n, D]
    v = torch.from_numpy(bf16_from_i16(z["v"])).to(torch.bfloat16)
    parents = z["parents"].tolist()
    n = len(parents)
    P = int(z["prefix"])
    anc = anc_bits(parents, 1)[None].to(DEV)
    out = ops.tree_attention(q.transpose(1, 2).contiguous().to(DEV), k.to(DEV), v.to(DEV), anc, P, 128 ** -0.5)
    ref = torch.from_numpy(z["out"]).transpose(1, 2)  # [1, n, H, D]
    err = (out.float().cpu() - ref).abs().max().item()
    assert err <= TOL, err


@pytest.mark.parametrize("P,n,H,Hkv,splits", [(4096, 65, 32, 8, None), (100, 65, 32, 8, 3), (0, 17, 8, 8, 1),
                                              (1000, 64, 32, 8, 7), (77, 257, 16, 4, 2), (300, 100, 16, 8, 1),
                                              (2500, 130, 8, 2, None), (129, 33, 32, 8, 1)])
def test_tree_attention_vs_oracle(P, n, H, Hkv, splits):
    from mfd_b200 import ops
    g = torch.Generator().manual_seed(P + n + H)
    parents = [-1] + [int(torch.randint(0, i, (1,), generator=g)) for i in range(1, n)]
    D = 128
    q = torch.randn(1, n, H, D, generator=g).to(torch.bfloat16)
    k = (torch.randn(1, Hkv, P + n, D, generator=g) * 0.5).to(torch.bfloat16)
    v = (torch.randn(1, Hkv, P + n, D, generator=g) * 0.5).to(torch.bfloat16)
    words = (n + 63) // 64
    anc = anc_bits(parents, words)[None].to(DEV)
    out = ops.tree_attention(q.to(DEV), k.to(DEV), v.to(DEV), anc, P, D ** -0.5, splits=splits)
    kk = k[0].transpose(0, 1).float().numpy()
    vv = v[0].transpose(0, 1).float().numpy()
    ref = oracle.tree_attention(q[0].float().numpy(), kk[:P], vv[:P], kk[P:], vv[P:], parents, D ** -0.5)
    err = np.abs(out[0].float().cpu().numpy() - ref).max()
    assert err <= TOL, err
    assert ops.tree_attention_status() == 0  # no wait gave up, no CTA skipped


def test_tree_attention_batched_variable_prefix():
    from mfd_b200 import ops
    g = torch.Generator().manual_seed(9)
    bs, n, H, Hkv, D, S = 3, 33, 16, 4, 128, 700
    prefixes = [10, 300, 667]
    q = torch.randn(bs, n, H, D, generator=g).to(torch.bfloat16)
    k = (torch.randn(bs, Hkv, S, D, generator=g) * 0.5).to(torch.bfloat16)
    v = (torch.randn(bs, Hkv, S, D, generator=g) * 0.5).to(torch.bfloat16)
    trees = [[-1] + [int(torch.randint(0, i, (1,), generator=g)) for i in range(1, n)] for _ in range(bs)]
    anc = torch.stack([anc_bits(t, 1) for t in trees]).to(DEV)
    pl = torch.tensor(prefixes, dtype=torch.int32, device=DEV)
    out = ops.tree_attention(q.to(DEV), k.to(DEV), v.to(DEV), anc, pl, D ** -0.5, splits=4)
    for b in range(bs):
        P = prefixes[b]
        kk = k[b].transpose(0, 1).float().numpy()
        vv = v[b].transpose(0, 1).float().numpy()
        ref = oracle.tree_attention(q[b].float().numpy(), kk[:P], vv[:P], kk[P:P + n], vv[P:P + n], trees[b],
                                    D ** -0.5)
        err = np.abs(out[b].float().cpu().numpy() - ref).max()
        assert err <= TOL, (b, err)


@pytest.mark.parametrize("bs", [40, 70])
def test_tree_attention_many_requests_tied_prefixes(bs):
    """Launch order by prefix length (longest first, ties by request index) for up to 64 requests, natural order
    above that: every request's rows match the oracle either way."""
    from mfd_b200 import ops
    g = torch.Generator().manual_seed(bs)
    n, H, Hkv, D = 9, 8, 2, 128
    prefixes = [int(x) for x in torch.randint(0, 4, (bs,), generator=g) * 60 + 1]  # 1, 61, 121, 181: many ties
    S = max(prefixes) + n
    q = torch.randn(bs, n, H, D, generator=g).to(torch.bfloat16)
    k = (torch.randn(bs, Hkv, S, D, generator=g) * 0.5).to(torch.bfloat16)
    v = (torch.randn(bs, Hkv, S, D, generator=g) * 0.5).to(torch.bfloat16)
    trees = [[-1] + [int(torch.randint(0, i, (1,), generator=g)) for i in range(1, n)] for _ in range(bs)]
    anc = torch.stack([anc_bits(t, 1) for t in trees]).to(DEV)
    pl = torch.tensor(prefixes, dtype=torch.int32, device=DEV)
    out = ops.tree_attention(q.to(DEV), k.to(DEV), v.to(DEV), anc, pl, D ** -0.5).float().cpu().numpy()
    for b in range(bs):
        P = prefixes[b]
        kk = k[b].transpose(0, 1).float().numpy()
        vv = v[b].transpose(0, 1).float().numpy()
        ref = oracle.tree_attention(q[b].float().numpy(), kk[:P], vv[:P], kk[P:P + n], vv[P:P + n], trees[b],
                                    D ** -0.5)
        assert np.abs(out[b] - ref).max() <= TOL, b
    assert ops.tree_attention_status() == 0


def test_tree_attention_workspace_reused_across_sizes():
    """One workspace serves calls of different sizes in any order: a call that fills it with split partials
    (one request, 16 splits), then calls with more (request, KV head, M-tile) units and other split counts all
    match the oracle (their tickets live in the ticket-only buffer, never on the earlier partials)."""
    from mfd_b200 import ops
    g = torch.Generator().manual_seed(31)
    n, H, Hkv, D = 65, 32, 8, 128
    for bs, splits in [(1, 16), (5, 4), (2, 7), (6, 3)]:
        S = 600 + n
        prefixes = [int(x) for x in torch.randint(100, 600, (bs,), generator=g)]
        q = torch.randn(bs, n, H, D, generator=g).to(torch.bfloat16)
        k = (torch.randn(bs, Hkv, S, D, generator=g) * 0.5).to(torch.bfloat16)
        v = (torch.randn(bs, Hkv, S, D, generator=g) * 0.5).to(torch.bfloat16)
        trees = [[-1] + [int(torch.randint(0, i, (1,), generator=g)) for i in range(1, n)] for _ in range(bs)]
        anc = torch.stack([anc_bits(t, 2) for t in trees]).to(DEV)
        pl = torch.tensor(prefixes, dtype=torch.int32, device=DEV)
        out = ops.tree_attention(q.to(DEV), k.to(DEV), v.to(DEV), anc, pl, D ** -0.5, splits=splits)
        out = out.float().cpu().numpy()
        for b in range(bs):
            P = prefixes[b]
            kk = k[b].transpose(0, 1).float().numpy()
            vv = v[b].transpose(0, 1).float().numpy()
            ref = oracle.tree_attention(q[b].float().numpy(), kk[:P], vv[:P], kk[P:P + n], vv[P:P + n], trees[b],
                                        D ** -0.5)
            assert np.abs(out[b] - ref).max() <= TOL, (bs, splits, b)
    assert ops.tree_attention_status() == 0


@pytest.mark.parametrize("splits", [1, 2, 3])
def test_tree_attention_ignores_nan_beyond_each_requests_keys(splits):
    """A KV buffer holds whatever the caller left beyond a request's keys (here NaN, in K and V alike, and under
    a shorter constant prefix too): masked keys of a tile that runs past the request's last key must contribute
    nothing, as keys the reference's mask + SDPA never sees."""
    from mfd_b200 import ops
    g = torch.Generator().manual_seed(90 + splits)
    bs, n, H, Hkv, D, S = 3, 65, 32, 8, 128, 1500
    prefixes = [1413, 700, 1000]
    parents = [[-1] + [int(torch.randint(0, i, (1,), generator=g)) for i in range(1, n)] for _ in range(bs)]
    q = torch.randn(bs, n, H, D, generator=g).to(torch.bfloat16)
    k = torch.full((bs, Hkv, S, D), float("nan")).to(torch.bfloat16)
    v = torch.full((bs, Hkv, S, D), float("nan")).to(torch.bfloat16)
    for b, p in enumerate(prefixes):
        k[b, :, :p + n] = (torch.randn(Hkv, p + n, D, generator=g) * 0.5).to(torch.bfloat16)
        v[b, :, :p + n] = (torch.randn(Hkv, p + n, D, generator=g) * 0.5).to(torch.bfloat16)
    anc = torch.stack([anc_bits(par, 2) for par in parents]).to(DEV)
    pl = torch.tensor(prefixes, dtype=torch.int32, device=DEV)
    out = ops.tree_attention(q.to(DEV), k.to(DEV), v.to(DEV), anc, pl, D ** -0.5, splits=splits).float().cpu()
    assert torch.isfinite(out).all()
    for b, p in enumerate(prefixes):
        kk = k[b, :, :p + n].transpose(0, 1).float().numpy()
        vv = v[b, :, :p + n].transpose(0, 1).float().numpy()
        ref = oracle.tree_attention(q[b].float().numpy(), kk[:p], vv[:p], kk[p:], vv[p:], parents[b], D ** -0.5)
        assert np.abs(out[b].numpy() - ref).max() <= TOL
    # one constant prefix shorter than the buffer: the keys after prefix + n are NaN as well
    p = 700
    kc, vc = k[1:2].clone(), v[1:2].clone()
    out1 = ops.tree_attention(q[1:2].to(DEV), kc.to(DEV), vc.to(DEV), anc[1:2], p, D ** -0.5, splits=splits)
    assert torch.isfinite(out1.float()).all()
    assert torch.equal(out1.cpu(), out[1:2].to(torch.bfloat16)) or \
        (out1.float().cpu() - out[1:2]).abs().max() <= TOL


@pytest.mark.parametrize("n,splits", [(65, 1), (65, 3), (64, 2), (100, 1)])
def test_tree_attention_rescales_on_growing_scores(n, splits):
    """Scores that grow along the keys (K scaled by a ramp from 1 to 6) raise each row's running maximum by far
    more than 2^8 several times, so every M-tile of a CTA (one or two per CTA) takes the O rescale path; the result
    still matches the oracle."""
    from mfd_b200 import ops
    g = torch.Generator().manual_seed(500 + n + splits)
    P, H, Hkv, D = 1500, 32, 8, 128
    parents = [-1] + [int(torch.randint(0, i, (1,), generator=g)) for i in range(1, n)]
    ramp = torch.linspace(1.0, 6.0, P + n).view(1, 1, P + n, 1)
    q = (torch.randn(1, n, H, D, generator=g) * 2).to(torch.bfloat16)
    k = (torch.randn(1, Hkv, P + n, D, generator=g) * 0.5 * ramp).to(torch.bfloat16)
    v = (torch.randn(1, Hkv, P + n, D, generator=g) * 0.5).to(torch.bfloat16)
    anc = anc_bits(parents, (n + 63) // 64)[None].to(DEV)
    out = ops.tree_attention(q.to(DEV), k.to(DEV), v.to(DEV), anc, P, D ** -0.5, splits=splits)
    kk = k[0].transpose(0, 1).float().numpy()
    vv = v[0].transpose(0, 1).float().numpy()
    ref = oracle.tree_attention(q[0].float().numpy(), kk[:P], vv[:P], kk[P:], vv[P:], parents, D ** -0.5)
    assert np.abs(out[0].float().cpu().numpy() - ref).max() <= TOL
    assert ops.tree_attention_status() == 0


@pytest.mark.parametrize("splits", [1, 2])
def test_tree_attention_rescales_across_a_wide_score_range(splits):
    """Scores whose base-2 exponent grows by hundreds along the keys (K scaled by a ramp from 1 to 40): the running
    max is raised, and O rescaled in TMEM, on most key tiles, and the result is finite and matches the oracle."""
    from mfd_b200 import ops
    g = torch.Generator().manual_seed(700 + splits)
    P, n, H, Hkv, D = 1500, 65, 32, 8, 128
    parents = [-1] + [int(torch.randint(0, i, (1,), generator=g)) for i in range(1, n)]
    ramp = torch.linspace(1.0, 40.0, P + n).view(1, 1, P + n, 1)
    q = (torch.randn(1, n, H, D, generator=g) * 2).to(torch.bfloat16)
    k = (torch.randn(1, Hkv, P + n, D, generator=g) * 0.5 * ramp).to(torch.bfloat16)
    v = (torch.randn(1, Hkv, P + n, D, generator=g) * 0.5).to(torch.bfloat16)
    anc = anc_bits(parents, (n + 63) // 64)[None].to(DEV)
    out = ops.tree_attention(q.to(DEV), k.to(DEV), v.to(DEV), anc, P, D ** -0.5, splits=splits)
    kk = k[0].transpose(0, 1).float().numpy()
    vv = v[0].transpose(0, 1).float().numpy()
    ref = oracle.tree_attention(q[0].float().numpy(), kk[:P], vv[:P], kk[P:], vv[P:], parents, D ** -0.5)
    got = out[0].float().cpu().numpy()
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() <= TOL
    assert ops.tree_attention_status() == 0
