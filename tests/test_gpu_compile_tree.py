"""GPU parity of ddtree.compile_ddtree_tree (mfd_compile_tree) with the reference's (inference/hf/ddtree.py:
317-357) over consecutive rounds into the same buffers, bit for bit: the verify ids, positions, the bool
visibility and the whole additive mask buffer, whose tree blocks overlap from one round to the next.  Trees come
either from the host (the reference's fixture, copied over once) or from this package's builder (read on the
device where they were built)."""
import numpy as np
import pytest
import torch

from oracle import oracle
from tests._golden import load

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("d,dtype", [(0, torch.bfloat16), (1, torch.float32)])
def test_compile_tree_rounds_match_reference_fixture(d, dtype):
    from mfd_b200 import ddtree
    z = load("compile_tree.npz")
    max_nodes, max_len = [int(v) for v in z["dims"]]
    ids_buf = torch.zeros(1, max_nodes, dtype=torch.long, device=DEV)
    pos_buf = torch.zeros(1, max_nodes, dtype=torch.long, device=DEV)
    mask_buf = torch.zeros(1, 1, max_nodes, max_len + max_nodes, dtype=dtype, device=DEV)
    vis_buf = torch.zeros(max_nodes, max_nodes, dtype=torch.bool, device=DEV)
    bits = torch.int16 if dtype == torch.bfloat16 else torch.int32
    prev_start, prev_len = 0, 0
    for r in range(3):
        pre = f"d{d}r{r}_"
        assert [prev_start, prev_len] == z[pre + "prev"].tolist()
        start = int(z[pre + "start"])
        root = torch.tensor(int(z[pre + "root"]), device=DEV)
        ids, pos, mask, prev_start, prev_len = ddtree.compile_ddtree_tree(
            root, start, torch.from_numpy(z[pre + "tokens"]), torch.from_numpy(z[pre + "depths"]),
            torch.from_numpy(z[pre + "vis"]), start, dtype, DEV, ids_buf, pos_buf, mask_buf, vis_buf, prev_start,
            prev_len)
        n = len(z[pre + "parents"])
        assert prev_start == start and prev_len == n
        assert ids.shape == (1, n) and pos.shape == (1, n) and mask.shape == (1, 1, n, start + n)
        assert np.array_equal(ids_buf.cpu().numpy(), z[pre + "ids"])
        assert np.array_equal(pos_buf.cpu().numpy(), z[pre + "pos"])
        assert np.array_equal(vis_buf.cpu().numpy(), z[pre + "vis_buf"])
        assert np.array_equal(mask_buf.view(bits).cpu().numpy(), z[pre + "mask_bits"]), f"round {r}: mask"


def test_compile_tree_from_the_device_builder_matches_oracle():
    from mfd_b200 import ddtree
    g = torch.Generator().manual_seed(8)
    K, L, V, B = 8, 16, 4096, 64
    max_nodes, max_len = B + 1, 600
    ids_buf = torch.zeros(1, max_nodes, dtype=torch.long, device=DEV)
    pos_buf = torch.zeros(1, max_nodes, dtype=torch.long, device=DEV)
    mask_buf = torch.zeros(1, 1, max_nodes, max_len + max_nodes, dtype=torch.bfloat16, device=DEV)
    vis_buf = torch.zeros(max_nodes, max_nodes, dtype=torch.bool, device=DEV)
    ref_ids, ref_pos = np.zeros(max_nodes, np.int64), np.zeros(max_nodes, np.int64)
    ref_mask = np.zeros((max_nodes, max_len + max_nodes), np.float32)
    ref_vis = np.zeros((max_nodes, max_nodes), bool)
    prev_start, prev_len, start = 0, 0, 300
    for r in range(3):
        x = torch.randn(K, L, V, generator=g)
        x.scatter_add_(2, torch.randint(0, V, (K, L, 2), generator=g), torch.rand(K, L, 2, generator=g) * 8 + 4)
        tok, dep, parents, _, vis, _ = ddtree.build_mixture_tree(x.to(DEV), torch.zeros(K, device=DEV), B)
        assert hasattr(tok, "_mfd_tree") and hasattr(vis, "_mfd_vis")  # read on the device, not copied back
        root = torch.tensor(17 + r, device=DEV)
        oracle.compile_tree(17 + r, start, tok.numpy(), dep.numpy(), vis.numpy(), start, prev_start, prev_len,
                            ref_ids, ref_pos, ref_mask, ref_vis, float(torch.finfo(torch.bfloat16).min))
        _, _, _, prev_start, prev_len = ddtree.compile_ddtree_tree(
            root, start, tok, dep, vis, start, torch.bfloat16, DEV, ids_buf, pos_buf, mask_buf, vis_buf, prev_start,
            prev_len)
        n = len(parents)
        assert np.array_equal(ids_buf[0, :n].cpu().numpy(), ref_ids[:n])
        assert np.array_equal(pos_buf[0, :n].cpu().numpy(), ref_pos[:n])
        assert np.array_equal(vis_buf[:n, :n].cpu().numpy(), ref_vis[:n, :n])
        want = torch.from_numpy(ref_mask).to(torch.bfloat16).view(torch.int16)
        assert torch.equal(mask_buf[0, 0].cpu().view(torch.int16), want), f"round {r}"
        start += 2 + r
