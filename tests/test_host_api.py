"""Host-side behaviour of the drop-in API that needs no GPU: edge cases and loud failure without CUDA."""
import pytest
import torch

from mfd_b200 import ddtree, ddtree_utils, qwen35_tree
from tests._golden import load


def test_trivial_trees_match_reference_edge_cases():
    # inference/hf/ddtree.py:121-131 and 230-231
    out = ddtree.build_ddtree_tree(torch.zeros(0, 10), 8)
    assert out[0].numel() == 0 and out[2] == [-1] and out[4].tolist() == [[True]]
    out = ddtree.build_mixture_tree(torch.zeros(2, 3, 10), torch.zeros(2), 0)
    assert out[2] == [-1]
    acc, nxt = ddtree.follow_verified_tree(out[3], torch.tensor([[7]]))
    assert acc == [0] and nxt == 7


def test_no_cpu_fallback():
    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    with pytest.raises(RuntimeError, match="CUDA"):
        ddtree.build_mixture_tree(torch.randn(2, 3, 50), torch.zeros(2), 8)


def test_multi_mode_draft_mask():
    m = ddtree.multi_mode_draft_mask(3, 2, 2, torch.float32, torch.device("cpu"))
    assert m.shape == (1, 1, 4, 7)
    assert (m[0, 0, :, :3] == 0).all()
    assert m[0, 0, 0, 3] == 0 and m[0, 0, 0, 5] < -1e30 and m[0, 0, 2, 5] == 0


def test_ancestor_visibility_reference():
    vis = ddtree_utils.ancestor_visibility_reference(torch.tensor([-1, 0, 0, 1, -1]))
    assert vis[3].tolist() == [True, True, False, True, False]
    assert vis[4].tolist() == [False, False, False, False, True]


def test_tree_context_conv_windows_match_reference():
    z = load("tree_context.npz")
    parents = z["parents"].tolist()
    vis = torch.zeros(len(parents), len(parents), dtype=torch.bool)
    for i in range(len(parents)):
        j = i
        while j >= 0:
            vis[i, j] = True
            j = parents[j]
    ctx = qwen35_tree.TreeContext(parents, vis, 4, torch.device("cpu"))
    assert ctx.conv_index_cpu == z["conv_index"].tolist()
    cp, cv = qwen35_tree.chain_tree(6)
    assert cp == z["chain_parents"].tolist() and torch.equal(cv, torch.from_numpy(z["chain_vis"]))


def test_load_draft_vocab_formats(tmp_path, monkeypatch):
    """The reduced draft vocabulary loader (P:1226-1244): JSON list, JSON object with "token_ids", whitespace
    separated ids; sorted unique int64; out-of-range or empty lists raise ValueError."""
    a = tmp_path / "a.json"
    a.write_text("[5, 3, 3, 9]")
    b = tmp_path / "b.json"
    b.write_text('{"token_ids": [7, 1]}')
    c = tmp_path / "c.txt"
    c.write_text("4 2\n8")
    assert ddtree_utils.load_draft_vocab(str(a), vocab_size=10).tolist() == [3, 5, 9]
    assert ddtree_utils.load_draft_vocab(str(b), vocab_size=10).tolist() == [1, 7]
    t = ddtree_utils.load_draft_vocab(str(c), vocab_size=10)
    assert t.tolist() == [2, 4, 8] and t.dtype == torch.int64
    with pytest.raises(ValueError):
        ddtree_utils.load_draft_vocab(str(a), vocab_size=9)
    d = tmp_path / "d.json"
    d.write_text("[]")
    with pytest.raises(ValueError):
        ddtree_utils.load_draft_vocab(str(d), vocab_size=9)
    monkeypatch.setenv("SGLANG_DFLASH_DDTREE_DRAFT_VOCAB", f" {a} ")
    assert ddtree_utils.ddtree_draft_vocab_path() == str(a)
    monkeypatch.delenv("SGLANG_DFLASH_DDTREE_DRAFT_VOCAB")
    assert ddtree_utils.ddtree_draft_vocab_path() == ""


def test_compact_tail_routes_8_byte_aligned_bases_to_the_8_byte_path():
    from mfd_b200 import ops
    buf = torch.zeros(2 * 40 * 16 + 1, dtype=torch.int64)
    base = buf[: 2 * 40 * 16].view(2, 40, 16)        # 16-byte rows, base aligned as allocated
    shifted = buf[1:].view(2, 40, 16)                  # same layout, base 8 bytes further on
    assert base.data_ptr() % 16 == 0 and shifted.data_ptr() % 16 == 8
    keys = ops.compact_tail_groups([base, shifted])
    assert len(keys) == 2 and keys[0][-1] == 16 and keys[1][-1] == 8
    assert keys[0][:-1] == keys[1][:-1]  # only the alignment separates the two launches
