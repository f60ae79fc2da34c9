"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run in a container where the reference checkout is mounted (its root in MFD_REFERENCE_ROOT, else the mount
point the build container uses):

    python tests/golden/make_golden.py

Sources of truth, all the reference's own code (imported read-only, never copied):
  - inference/hf/ddtree.py build_mixture_tree / build_ddtree_tree (Python heaps, float32 top-k +
    logsumexp on CPU) and follow_verified_tree;
  - inference/hf/tree_build_ext.py's C++ builders (build_single / build_mixture / Tree.follow) and the
    SGLang patch's C++ build_trees, compiled from the reference sources by oracle/build_ref.py;
  - inference/hf/mode_attention.py `reference` (float32 masked SDPA);
  - inference/hf/ddtree.py compile_ddtree_tree (the additive verify mask) + torch SDPA in float64, and the
    verify inputs it writes over consecutive rounds (compile_tree.npz);
  - tests/test_gdn_tree_math.py's tree_case inputs and its node-by-node recurrence.
  - inference/hf/ddtree.py _compact_appended_window / compact_dynamic_cache (the commit step's cache
    compaction, its index_select path) on CPU tensors and a transformers DynamicCache.
Inputs are seeded; each fixture stores inputs and expected outputs.  Top-k on CPU leaves equal values in
unspecified order, so end-to-end (logits -> tree) fixtures use continuous float32 logits (no ties) and the
tie-heavy cases enter at the candidate level (top-k already given), exactly as the reference's own
tree_build_ext.check_equal and test_sglang_tree_builder do.
"""

from __future__ import annotations

import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
REF = os.environ.get("MFD_REFERENCE_ROOT", "/root/reference")
sys.dont_write_bytecode = True
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(REF, "inference", "hf"))
sys.path.insert(0, os.path.join(REF, "tests"))

import ddtree  # noqa: E402  (reference)
import mode_attention as ref_mode_attention  # noqa: E402  (reference)
import qwen35_tree as ref_qwen35_tree  # noqa: E402  (reference)
import test_gdn_tree_math as ref_gdn_test  # noqa: E402  (reference)

from oracle import build_ref  # noqa: E402

ddtree.cuda_time = time.perf_counter  # the reference tests do this on CPU-only machines


def save(name: str, **arrays) -> None:
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **arrays)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


def mixture_end_to_end():
    """Continuous float32 logits -> reference Python mixture/ddtree builders (float32 topk + logsumexp)."""
    gen = torch.Generator().manual_seed(1234)
    cases = []
    for trial in range(24):
        K = (1, 2, 4, 8)[trial % 4]
        L = int(torch.randint(1, 16, (1,), generator=gen))
        V = (64, 200, 500)[trial % 3]
        B = (5, 16, 31, 64)[(trial // 2) % 4]
        logits = torch.randn(K, L, V, generator=gen) * 3
        prior = torch.log_softmax(torch.randn(K, generator=gen), -1) if trial % 2 else torch.zeros(K)
        if K == 1 and trial % 8 == 0:
            out = ddtree.build_ddtree_tree(logits[0], B)
            single = 1
        else:
            out = ddtree.build_mixture_tree(logits, prior, B)
            single = 0
        n = len(out[2])
        post = torch.randint(0, V, (n,), generator=gen)
        # follow some edges so walks are long
        for node in range(1, n):
            if torch.rand((), generator=gen) < 0.6:
                post[out[2][node]] = int(out[0][node - 1])
        acc, bonus = ddtree.follow_verified_tree(out[3], post.view(1, n))
        cases.append(dict(logits=logits.numpy(), prior=prior.numpy().astype(np.float32), budget=B, single=single,
                          tokens=out[0].numpy(), depths=out[1].numpy(), parents=np.array(out[2], np.int64),
                          vis=out[4].numpy(), post=post.numpy(), accepted=np.array(acc, np.int64), bonus=bonus))
    flat = {}
    for i, c in enumerate(cases):
        for k, v in c.items():
            flat[f"c{i}_{k}"] = np.asarray(v)
    flat["n"] = np.array(len(cases))
    save("mixture_e2e.npz", **flat)


def candidates_with_ties():
    """bf16-like logits with many exact ties -> reference C++ builders on the float32 top-k candidates."""
    hf = build_ref.load("hf")
    gen = torch.Generator().manual_seed(99)
    flat = {}
    n = 0
    for trial in range(60):
        K = (1, 2, 8)[trial % 3]
        L = int(torch.randint(1, 16, (1,), generator=gen))
        V = 64 if trial % 5 else 512
        B = (16, 64, 255)[(trial // 3) % 3]
        logits = torch.randn(K, L, V, generator=gen) * 3
        if trial % 2 == 0:
            logits = (logits * 2).round() / 2
        logits = logits.to(torch.bfloat16).float()
        prior = torch.log_softmax(torch.randn(K, generator=gen), -1) if trial % 4 == 1 else torch.zeros(K)
        k = min(B, V)
        top, ids = torch.topk(logits, k=k, dim=-1)
        lp = (top - torch.logsumexp(logits, -1, keepdim=True)).float().contiguous()
        single = 1 if (K == 1 and trial % 2 == 0) else 0
        if single:
            out = hf.build_single(lp[0].contiguous(), ids[0].contiguous(), B)
        else:
            out = hf.build_mixture(lp, ids.contiguous(), prior.float().contiguous(), B)
        m = len(out[2])
        post = torch.randint(0, V, (m,), generator=gen)
        toks = [0] + out[0].tolist()
        for node in range(1, m):
            if torch.rand((), generator=gen) < 0.7:
                post[out[2][node]] = toks[node]
        acc, bonus = out[3].follow(post)
        flat.update({f"c{n}_lp": lp.numpy(), f"c{n}_ids": ids.numpy(), f"c{n}_prior": prior.numpy().astype(np.float32),
                     f"c{n}_budget": np.array(B), f"c{n}_single": np.array(single),
                     f"c{n}_tokens": out[0].numpy(), f"c{n}_depths": out[1].numpy(),
                     f"c{n}_parents": np.array(list(out[2]), np.int64), f"c{n}_vis": out[4].numpy(),
                     f"c{n}_post": post.numpy(), f"c{n}_accepted": np.array(list(acc), np.int64),
                     f"c{n}_bonus": np.array(int(bonus))})
        n += 1
    flat["n"] = np.array(n)
    save("candidates_ties.npz", **flat)


def sglang_batched():
    """The SGLang patch's C++ build_trees, batched (tail convention included)."""
    sg = build_ref.load("sglang")
    gen = torch.Generator().manual_seed(7)
    flat = {}
    n = 0
    for trial in range(20):
        K = (1, 2, 8)[trial % 3]
        L = int(torch.randint(1, 16, (1,), generator=gen))
        V = 64 if trial % 4 else 512
        B = (16, 31, 63, 128, 255)[trial % 5]
        bs = 1 + trial % 3
        logits = torch.randn(bs, K, L, V, generator=gen) * 3
        if trial % 3 == 0:
            logits = (logits * 2).round() / 2
        logits = logits.to(torch.bfloat16).float()
        k = min(B, V)
        top, ids = torch.topk(logits, k=k, dim=-1)
        lp = (top - torch.logsumexp(logits, -1, keepdim=True)).float().contiguous()
        prior = torch.zeros(bs, K)
        tree = torch.empty((bs, 3, B + 1), dtype=torch.long)
        counts = torch.empty((bs,), dtype=torch.long)
        sg.build_trees(lp, ids.to(torch.int32).contiguous(), prior, bs, B, tree, counts)
        flat.update({f"c{n}_lp": lp.numpy(), f"c{n}_ids": ids.to(torch.int32).numpy(), f"c{n}_prior": prior.numpy(),
                     f"c{n}_budget": np.array(B), f"c{n}_tree": tree.numpy(), f"c{n}_counts": counts.numpy()})
        n += 1
    flat["n"] = np.array(n)
    save("sglang_build_trees.npz", **flat)


def topk_rows():
    """float32 top-k + logsumexp on CPU (hf/ddtree.py:240-244), tie-free rows."""
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(12, 3001, generator=gen) * 2
    ids = torch.randint(0, 3001, (12, 3), generator=gen)
    x.scatter_add_(1, ids, torch.rand(12, 3, generator=gen) * 6 + 4)
    top, tid = torch.topk(x, 64, dim=-1)
    lz = torch.logsumexp(x, -1, keepdim=True)
    save("topk_logz.npz", x=x.numpy(), top_logp=(top - lz).numpy(), ids=tid.numpy(), logz=lz[:, 0].numpy())


def mode_attention_case():
    gen = torch.Generator().manual_seed(11)
    K, bs, H, Hkv, D = 4, 8, 4, 2, 128
    flat = {}
    for i, ctx in enumerate((1, 37, 130)):
        q = torch.randn(1, H, K * bs, D, generator=gen).to(torch.bfloat16)
        k = (torch.randn(1, Hkv, ctx + K * bs, D, generator=gen) * 2).to(torch.bfloat16)
        v = torch.randn(1, Hkv, ctx + K * bs, D, generator=gen).to(torch.bfloat16)
        ref = ref_mode_attention.reference(q, k, v, K, bs, D ** -0.5)  # [1, K*bs, H, D] float32
        flat.update({f"c{i}_q": q.view(torch.int16).numpy(), f"c{i}_k": k.view(torch.int16).numpy(),
                     f"c{i}_v": v.view(torch.int16).numpy(), f"c{i}_out": ref.numpy(), f"c{i}_ctx": np.array(ctx)})
    flat.update(n=np.array(3), K=np.array(K), bs=np.array(bs))
    save("mode_attention.npz", **flat)


def verify_attention_case():
    """compile_ddtree_tree's additive mask + SDPA (float64) on a small tree."""
    gen = torch.Generator().manual_seed(21)
    n, P, H, Hkv, D = 17, 40, 8, 2, 128
    parents = [-1] + [int(torch.randint(0, i, (1,), generator=gen)) for i in range(1, n)]
    vis = torch.zeros(n, n, dtype=torch.bool)
    for i in range(n):
        j = i
        while j >= 0:
            vis[i, j] = True
            j = parents[j]
    depths = torch.zeros(n - 1, dtype=torch.long)
    for i in range(1, n):
        depths[i - 1] = (depths[parents[i] - 1] + 1) if parents[i] > 0 else 1
    ids_buf = torch.zeros(1, 64, dtype=torch.long)
    pos_buf = torch.zeros(1, 64, dtype=torch.long)
    mask_buf = torch.zeros(1, 1, 64, P + 64, dtype=torch.float32)
    vis_buf = torch.zeros(64, 64, dtype=torch.bool)
    _, _, mask, _, _ = ddtree.compile_ddtree_tree(torch.tensor(5), P, torch.arange(1, n), depths, vis, P,
                                                  torch.float32, torch.device("cpu"), ids_buf, pos_buf, mask_buf,
                                                  vis_buf, 0, 0)
    q = torch.randn(1, H, n, D, generator=gen).to(torch.bfloat16)
    k = (torch.randn(1, Hkv, P + n, D, generator=gen) * 0.5).to(torch.bfloat16)
    v = (torch.randn(1, Hkv, P + n, D, generator=gen) * 0.5).to(torch.bfloat16)
    G = H // Hkv
    out = torch.nn.functional.scaled_dot_product_attention(
        q.double(), k.double().repeat_interleave(G, 1), v.double().repeat_interleave(G, 1),
        attn_mask=mask.double(), scale=D ** -0.5)
    save("verify_attention.npz", q=q.view(torch.int16).numpy(), k=k.view(torch.int16).numpy(),
         v=v.view(torch.int16).numpy(), parents=np.array(parents, np.int64), prefix=np.array(P),
         mask=mask.numpy(), out=out.float().numpy())


def compile_tree_case():
    """compile_ddtree_tree over consecutive rounds into the same buffers: each round's tree block overlaps the
    previous one (the prefix advances by less than the previous tree), bf16 and float32 masks."""
    gen = torch.Generator().manual_seed(31)
    flat = {}
    max_nodes, max_len = 24, 100
    for d, dtype in enumerate((torch.bfloat16, torch.float32)):
        ids_buf = torch.zeros(1, max_nodes, dtype=torch.long)
        pos_buf = torch.zeros(1, max_nodes, dtype=torch.long)
        mask_buf = torch.zeros(1, 1, max_nodes, max_len + max_nodes, dtype=dtype)
        vis_buf = torch.zeros(max_nodes, max_nodes, dtype=torch.bool)
        prev_start, prev_len, start = 0, 0, 40
        for r, n in enumerate((17, 13, 21)):
            parents = [-1] + [int(torch.randint(0, i, (1,), generator=gen)) for i in range(1, n)]
            vis = torch.zeros(n, n, dtype=torch.bool)
            depths = [0] * n
            for i in range(n):
                j = i
                while j >= 0:
                    vis[i, j] = True
                    j = parents[j]
                if i:
                    depths[i] = depths[parents[i]] + 1
            tokens = torch.randint(0, 1000, (n - 1,), generator=gen)
            root = int(torch.randint(0, 1000, (1,), generator=gen))
            pre = f"d{d}r{r}_"
            flat.update({pre + "parents": np.array(parents, np.int64), pre + "tokens": tokens.numpy(),
                         pre + "depths": np.array(depths[1:], np.int64), pre + "vis": vis.numpy(),
                         pre + "root": np.int64(root), pre + "start": np.int64(start),
                         pre + "prev": np.array([prev_start, prev_len], np.int64)})
            _, _, _, prev_start, prev_len = ddtree.compile_ddtree_tree(
                torch.tensor(root), start, tokens, torch.tensor(depths[1:], dtype=torch.long), vis, start, dtype,
                torch.device("cpu"), ids_buf, pos_buf, mask_buf, vis_buf, prev_start, prev_len)
            flat.update({pre + "ids": ids_buf.numpy().copy(), pre + "pos": pos_buf.numpy().copy(),
                         pre + "mask_bits": mask_buf.view(torch.int16 if dtype == torch.bfloat16 else torch.int32)
                         .numpy().copy(), pre + "vis_buf": vis_buf.numpy().copy()})
            start += 1 + int(torch.randint(0, 4, (1,), generator=gen))
    flat["dims"] = np.array([max_nodes, max_len], np.int64)
    save("compile_tree.npz", **flat)


def gdn_case():
    """tests/test_gdn_tree_math.py tree_case (seeds 0..2) and its node-by-node recurrence, float64."""
    flat = {}
    for seed in range(3):
        parents, k, q, v, beta, g, s0 = ref_gdn_test.tree_case(seed, n=24)
        n, dk = k.shape
        states, o_ref = [None] * n, torch.zeros(n, v.shape[1], dtype=torch.float64)
        for i in range(n):
            sp = s0 if parents[i] < 0 else states[parents[i]]
            states[i] = g[i].exp() * sp @ (torch.eye(dk, dtype=torch.float64) - beta[i] * torch.outer(k[i], k[i])) + \
                beta[i] * torch.outer(v[i], k[i])
            o_ref[i] = states[i] @ q[i]
        flat.update({f"c{seed}_parents": np.array(parents, np.int64), f"c{seed}_k": k.numpy(), f"c{seed}_q": q.numpy(),
                     f"c{seed}_v": v.numpy(), f"c{seed}_beta": beta.numpy(), f"c{seed}_g": g.numpy(),
                     f"c{seed}_s0": s0.numpy(), f"c{seed}_o": o_ref.numpy(),
                     f"c{seed}_states": torch.stack(states).numpy()})
    flat["n"] = np.array(3)
    save("gdn_tree.npz", **flat)


def tree_context_case():
    """qwen35_tree.TreeContext conv windows and chain_tree."""
    parents = [-1, 0, 0, 1, 3, 2, 5, 5]
    n = len(parents)
    vis = torch.zeros(n, n, dtype=torch.bool)
    for i in range(n):
        j = i
        while j >= 0:
            vis[i, j] = True
            j = parents[j]
    ctx = ref_qwen35_tree.TreeContext(parents, vis, 4, torch.device("cpu"))
    cp, cv = ref_qwen35_tree.chain_tree(6)
    save("tree_context.npz", parents=np.array(parents, np.int64), conv_index=np.array(ctx.conv_index_cpu, np.int64),
         chain_parents=np.array(cp, np.int64), chain_vis=cv.numpy())


def compact_case():
    """The commit step's cache compaction: ddtree._compact_appended_window (its index_select path) on cache tensors
    with monotone and permuted keep lists, an empty list and a whole-window list (both early returns), and
    compact_dynamic_cache on a transformers DynamicCache of two layers."""
    ddtree._CPP_COMPACT_ENABLED = False
    g = torch.Generator().manual_seed(17)
    cases = [((2, 3, 50, 16), 30, [0, 2, 5, 7]), ((1, 4, 40, 8), 25, [6, 1, 0, 9, 3]), ((2, 2, 20, 4), 12, []),
             ((1, 2, 24, 8), 16, [7, 6, 5, 4, 3, 2, 1, 0]), ((3, 1, 33, 32), 0, [4, 5, 30])]
    flat = {}
    for i, (shape, past, keep) in enumerate(cases):
        x = torch.randn(*shape, generator=g)
        y = x.clone()
        ddtree._compact_appended_window(y, past, torch.tensor(keep, dtype=torch.long))
        flat.update({f"c{i}_in": x.numpy(), f"c{i}_past": np.int64(past), f"c{i}_keep": np.array(keep, np.int64),
                     f"c{i}_out": y.numpy()})
    from transformers import DynamicCache

    cache = DynamicCache()
    ks = [torch.randn(1, 2, 14, 8, generator=g) for _ in range(2)]
    vs = [torch.randn(1, 2, 14, 8, generator=g) for _ in range(2)]
    for layer in range(2):
        cache.update(ks[layer].clone(), vs[layer].clone(), layer)
    ddtree.compact_dynamic_cache(cache, 9, [0, 3, 4])
    for layer in range(2):
        flat[f"dyn_k{layer}_in"], flat[f"dyn_v{layer}_in"] = ks[layer].numpy(), vs[layer].numpy()
        flat[f"dyn_k{layer}_out"] = cache.layers[layer].keys.numpy()
        flat[f"dyn_v{layer}_out"] = cache.layers[layer].values.numpy()
    flat["dyn_past"], flat["dyn_keep"] = np.int64(9), np.array([0, 3, 4], np.int64)
    flat["dyn_len"] = np.int64(cache.get_seq_length())
    save("compact_cache.npz", **flat)


if __name__ == "__main__":
    build_ref.build()
    mixture_end_to_end()
    candidates_with_ties()
    sglang_batched()
    topk_rows()
    mode_attention_case()
    verify_attention_case()
    compile_tree_case()
    gdn_case()
    tree_context_case()
    compact_case()
