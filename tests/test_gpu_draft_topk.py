"""GPU parity of the SGLang draft top-k head (DDTreeDraftTopK, P:1501-1550) with and without a reduced draft
vocabulary: logits = hs @ W.T over the (subset) head, top-k per drafted position with log Z, and with vocab_ids
the subset indices mapped back to full-vocabulary ids (P:1545's index_select).  Checked against the oracle's
top-k + logsumexp on the same logits: ids bit-exact (equal values ordered by lower index, which a sorted subset
keeps in full-vocabulary order), log-probabilities within 8e-6.  The subset head has rows that tie exactly."""
import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("subset", [None, 65536])
def test_draft_topk_head_vs_oracle(subset):
    from mfd_b200.ddtree_utils import DDTreeDraftTopK

    g = torch.Generator().manual_seed(41 + (subset or 0))
    V, Hd, K, L, budget, bs = 151936, 256, 8, 16, 64, 2
    vocab_ids = None
    rows_w = V
    if subset is not None:
        vocab_ids = torch.randperm(V, generator=g)[:subset].sort().values.to(torch.int32)
        rows_w = subset
    weight = (torch.randn(rows_w, Hd, generator=g) * 0.05)
    # exact ties: some head rows duplicated, so their logits are bit-identical
    dup = torch.randint(0, rows_w, (64, 2), generator=g)
    weight[dup[:, 1]] = weight[dup[:, 0]]
    weight = weight.to(torch.bfloat16).to(DEV)
    hidden = (torch.randn(bs * K * L, Hd, generator=g)).to(torch.bfloat16).to(DEV)
    head = DDTreeDraftTopK(weight=weight, block_size=L, num_modes=K, budget=budget, max_bs=bs,
                           vocab_ids=vocab_ids.to(DEV) if vocab_ids is not None else None)
    head(hidden)
    top_logp, top_ids = head.outputs(bs)
    torch.cuda.synchronize()
    hs = hidden.view(bs * K, L, Hd)[:, 1:, :].reshape(-1, Hd)
    logits = torch.matmul(hs, weight.T).float().cpu().numpy()
    ref_lp, ref_idx, _ = oracle.topk_logz(logits, budget)
    ref_ids = ref_idx if vocab_ids is None else vocab_ids.numpy()[ref_idx]
    got_ids = top_ids.reshape(-1, budget).cpu().numpy()
    got_lp = top_logp.reshape(-1, budget).cpu().numpy()
    assert np.array_equal(got_ids, ref_ids)
    assert np.abs(got_lp - ref_lp).max() <= 8e-6
    # equal values did reach the candidate lists (duplicated rows and bf16 rounding of the logits)
    assert (np.diff(ref_lp, axis=1) == 0).any()
