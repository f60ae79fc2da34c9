"""GPU parity of the benchmarked step itself: bench.Batch + bench.Step (configs[4]: drafter logits with 4 boosted
ids per row, B=64 mixture trees, verify attention over prefixes U(1024, 8192), stochastic acceptance at T=1 with
seeded uniforms) against the oracle chain -- oracle.topk_logz -> build_mixture -> sample_rows -> follow, and
oracle.tree_attention -- plus the independence of every request's results from the partition of the job over
GPUs (the same request ids as one batch and as the two halves bench.partition deals to two ranks).

Also configs[3]'s acceptance at its stated shape: a mixture tree of sharp drafter logits, target logits N(0,1)
with the argmax forced along a seeded depth-9 path, and the greedy walk, which must accept exactly that path."""
import numpy as np
import pytest
import torch

import bench
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
K, L, V, B, W = bench.K_MODES, bench.L_BLOCK, bench.VOCAB, bench.BUDGET, bench.W


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.cpu().view(torch.int16).numpy().astype(np.uint16)


def _run(reqs, prefixes, splits=None):
    batch = bench.Batch(reqs, prefixes, DEV)
    step = bench.Step(batch, splits=splits)
    o = step.run()
    torch.cuda.synchronize()
    return batch, {k: v.cpu() for k, v in o.items()}


def test_bench_step_matches_oracle_chain():
    prefixes = bench.prefix_lengths(bench.TOTAL_REQUESTS)
    reqs = [3, 17, 40, 101, 200, 255]
    batch, o = _run(reqs, prefixes)
    top = batch.top.view(len(reqs), K, L, B).cpu().numpy()
    ids = batch.ids.view(len(reqs), K, L, B).cpu().numpy().astype(np.int64)
    tree = batch.tree.cpu().numpy()
    counts = batch.counts.cpu().numpy()
    for i, r in enumerate(reqs):
        x = batch.draft[i].view(K * L, V).cpu().numpy()
        ref_lp, ref_ids, _ = oracle.topk_logz(x, B)
        assert np.array_equal(ref_ids.reshape(K, L, B), ids[i]), f"request {r}: top-k ids"
        assert np.abs(ref_lp.reshape(K, L, B) - top[i]).max() <= 8e-6, f"request {r}: top-k log-probs"
        tok, dep, par = oracle.build_mixture(top[i], ids[i], np.zeros(K, np.float32), B)
        n = len(tok)
        assert int(counts[i]) == n
        assert np.array_equal(tree[i, 0, 1:n + 1], tok) and np.array_equal(tree[i, 1, 1:n + 1], dep)
        assert np.array_equal(tree[i, 2, :n + 1], par), f"request {r}: parents"
        # the oracle's own candidates give the same tree (no near-tie on these inputs)
        tok2, _, par2 = oracle.build_mixture(ref_lp.reshape(K, L, B), ref_ids.reshape(K, L, B).astype(np.int64),
                                             np.zeros(K, np.float32), B)
        assert np.array_equal(tok2, tok) and np.array_equal(par2, par)
        # stochastic acceptance at T = 1: the sampling rule per node, then the walk over at most L - 1 edges
        post = oracle.sample_rows(_bits(batch.target[i]).reshape(W, V), 1.0, batch.u[i].cpu().numpy())
        assert np.array_equal(o["posterior"][i].numpy(), post), f"request {r}: samples"
        acc, bonus = oracle.follow(tree[i, 0], tree[i, 2], post, max_steps=L - 1)
        m = len(acc) - 1
        assert int(o["accept_len"][i]) == m and int(o["bonus"][i]) == bonus
        assert o["accepted"][i, :m + 1].tolist() == list(acc)
        assert o["out_tokens"][i, :m + 1].tolist() == [int(post[a]) for a in acc[:-1]] + [bonus]
    # verify attention of two requests (the shortest and the longest prefix) against the oracle
    for i in (int(np.argmin(batch.prefix)), int(np.argmax(batch.prefix))):
        p = batch.prefix[i]
        q = batch.q[i].float().cpu().numpy()
        kk = batch.k[i, :, :p + W].transpose(0, 1).float().cpu().numpy()
        vv = batch.v[i, :, :p + W].transpose(0, 1).float().cpu().numpy()
        ref = oracle.tree_attention(q, kk[:p], vv[:p], kk[p:], vv[p:], tree[i, 2].tolist(), bench.D ** -0.5)
        n = int(counts[i]) + 1
        err = np.abs(batch.attn_out[i].float().cpu().numpy()[:n] - ref[:n]).max()
        assert err <= 2e-2, f"request {reqs[i]}: attention max |err| {err}"


def test_results_independent_of_partition():
    total = 8
    prefixes = bench.prefix_lengths(total)
    whole = bench.partition(total, 1, 0, prefixes)
    splits = 2
    b1, o1 = _run(whole, prefixes, splits=splits)
    by_req = {}
    for rank in range(2):
        part = bench.partition(total, 2, rank, prefixes)
        b2, o2 = _run(part, prefixes, splits=splits)
        for j, r in enumerate(part):
            by_req[r] = (b2, o2, j)
    assert sorted(by_req) == sorted(whole)
    for i, r in enumerate(whole):
        b2, o2, j = by_req[r]
        assert torch.equal(b1.top[i * K * L:(i + 1) * K * L].cpu(), b2.top[j * K * L:(j + 1) * K * L].cpu())
        assert torch.equal(b1.tree[i].cpu(), b2.tree[j].cpu()), f"request {r}: tree"
        for key in ("posterior", "accept_len", "bonus", "accepted", "out_tokens"):
            assert torch.equal(o1[key][i], o2[key][j]), f"request {r}: {key}"
        n = int(b1.counts[i]) + 1
        assert torch.equal(b1.attn_out[i, :n].cpu(), b2.attn_out[j, :n].cpu()), f"request {r}: attention"


@pytest.mark.parametrize("seed", [3, 4])
def test_config3_forced_depth9_path_accepted(seed):
    from mfd_b200 import ops
    batch = bench.Batch([0], [64], DEV, temperature=0.0, target_std=1.0, uniform_prefix=64)
    bench.sharp_draft_logits(seed, DEV, batch.draft[0])
    bench.Step(batch).run()
    t = batch.tree[0].cpu().tolist()
    n = int(batch.counts[0])
    assert max(t[1][:n + 1]) >= 9, "the sharp generator's tree reaches depth 9"
    path = bench.forced_path(t[0], t[2], t[1], 9, seed=seed)
    assert len(path) == 10
    bench.force_argmax(batch.target[0], t[0], path)
    o = ops.accept(batch.target, batch.tree[:, 0], batch.tree[:, 2], temperature=0.0, max_steps=L - 1, out_len=L)
    post = oracle.argmax_rows(_bits(batch.target[0]).reshape(W, V))
    assert np.array_equal(o["posterior"][0].cpu().numpy(), post)
    acc, bonus = oracle.follow(np.array(t[0]), np.array(t[2]), post, max_steps=L - 1)
    assert list(acc) == path and int(o["accept_len"][0]) == 9
    assert o["accepted"][0, :10].tolist() == path and int(o["bonus"][0]) == bonus
