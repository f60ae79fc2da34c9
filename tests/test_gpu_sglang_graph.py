"""The SGLang-facing draft-and-verify ops are CUDA-graph safe (the patch captures them, sglang-v0.5.22-mfd.patch:
1485-1493, 606-609): DDTreeDraftTopK (LM head GEMM + logits step into static buffers) -> build_trees into caller
buffers -> ddtree_follow, captured once after a warm-up and replayed with new hidden states and posteriors,
give exactly the eager results."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_draft_build_follow_in_cuda_graph():
    from mfd_b200 import ddtree_utils
    g = torch.Generator(device=DEV).manual_seed(21)
    bs, K, L, B, Hd, Vd = 2, 8, 16, 64, 256, 4096
    W = B + 1
    weight = (torch.randn(Vd, Hd, generator=g, device=DEV) * 0.2).bfloat16()
    head = ddtree_utils.DDTreeDraftTopK(weight=weight, block_size=L, num_modes=K, budget=B, max_bs=bs)
    hidden = torch.randn(bs * K * L, Hd, generator=g, device=DEV).bfloat16()
    prior = torch.zeros(bs, K, device=DEV)
    tree = torch.empty(bs, 3, W, dtype=torch.int64, device=DEV)
    counts = torch.empty(bs, dtype=torch.int64, device=DEV)
    posterior = torch.randint(0, Vd, (bs, W), generator=g, device=DEV)
    window = torch.arange(bs * W, device=DEV).view(bs, W)
    prefix = torch.full((bs,), 100, dtype=torch.int64, device=DEV)
    outs = dict(accept_len_out=torch.empty(bs, dtype=torch.int32, device=DEV),
                commit_lens_out=torch.empty(bs, dtype=torch.int32, device=DEV),
                bonus_out=torch.empty(bs, dtype=torch.int64, device=DEV),
                out_tokens_out=torch.empty(bs, L, dtype=torch.int64, device=DEV),
                new_seq_lens_out=torch.empty(bs, dtype=torch.int64, device=DEV),
                move_src_out=torch.empty(bs, L, dtype=torch.int64, device=DEV),
                move_tgt_out=torch.empty(bs, L, dtype=torch.int64, device=DEV),
                hidden_index_out=torch.empty(bs, L, dtype=torch.int64, device=DEV))

    def step():
        head(hidden)
        lp, ids = head.outputs(bs)
        ddtree_utils.build_trees(top_log_probs=lp, top_ids=ids, log_prior=prior, bs=bs, budget=B, tree=tree,
                                 counts=counts)
        ddtree_utils.ddtree_follow(posterior=posterior, verify_ids=tree[:, 0], parents=tree[:, 2], window=window,
                                   prefix_lens=prefix, **outs)

    def snapshot():
        lp, ids = head.outputs(bs)
        return [t.clone() for t in (lp, ids, tree, counts, *outs.values())]

    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for trial in range(3):
        hidden.copy_(torch.randn(bs * K * L, Hd, generator=g, device=DEV).bfloat16())
        posterior.copy_(torch.randint(0, Vd, (bs, W), generator=g, device=DEV))
        graph.replay()
        torch.cuda.synchronize()
        got = snapshot()
        step()
        torch.cuda.synchronize()
        want = snapshot()
        for a, b in zip(got, want):
            assert torch.equal(a, b), trial
        assert int(counts.min()) > 0
    del graph
