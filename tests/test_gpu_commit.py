"""GPU parity of the commit step's KV moves (mfd_commit_kv_moves, mfd_compact_tail) against the oracle and the
reference's own cache compaction (golden fixture).  Bit-exact: the kernels only move bytes."""
import numpy as np
import pytest
import torch

from oracle import oracle
from tests._golden import load

pytestmark = pytest.mark.gpu

DEV = "cuda"


def test_compact_tail_vs_reference_fixture():
    from mfd_b200 import ddtree, ops
    f = load("compact_cache.npz")
    i = 0
    while f"c{i}_in" in f:
        x = torch.from_numpy(f[f"c{i}_in"]).to(DEV)
        ddtree._compact_appended_window(x, int(f[f"c{i}_past"]), torch.from_numpy(f[f"c{i}_keep"]).to(DEV))
        assert np.array_equal(x.cpu().numpy(), f[f"c{i}_out"]), i
        i += 1
    assert ops.compact_tail is not None and i == 5


class _Layer:
    def __init__(self, k, v):
        self.keys, self.values = k, v


class _Cache:
    """The `layers` form of a DynamicCache (keys / values per layer and crop), as compact_dynamic_cache reads it."""

    def __init__(self, ks, vs):
        self.layers = [_Layer(k, v) for k, v in zip(ks, vs)]

    def crop(self, n):
        for layer in self.layers:
            layer.keys = layer.keys[..., :n, :]
            layer.values = layer.values[..., :n, :]


def test_compact_dynamic_cache_vs_reference_fixture():
    from mfd_b200 import ddtree
    f = load("compact_cache.npz")
    ks = [torch.from_numpy(f[f"dyn_k{i}_in"]).to(DEV) for i in range(2)]
    vs = [torch.from_numpy(f[f"dyn_v{i}_in"]).to(DEV) for i in range(2)]
    cache = _Cache(ks, vs)
    ddtree.compact_dynamic_cache(cache, int(f["dyn_past"]), [int(i) for i in f["dyn_keep"]])
    for i in range(2):
        assert cache.layers[i].keys.shape[-2] == int(f["dyn_len"])
        assert np.array_equal(cache.layers[i].keys.cpu().numpy(), f[f"dyn_k{i}_out"])
        assert np.array_equal(cache.layers[i].values.cpu().numpy(), f[f"dyn_v{i}_out"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_compact_tail_many_layers_one_launch(dtype):
    from mfd_b200 import ops
    g = torch.Generator().manual_seed(3)
    tensors = [torch.randn(2, 8, 97, 128, generator=g).to(dtype) for _ in range(6)]
    past = 32
    keep = [0, 1, 3, 4, 9, 17, 30, 64]  # an accepted path of the 65-node window
    ref = [oracle.compact_tail(t.float().numpy(), past, keep) for t in tensors]
    dev = [t.to(DEV) for t in tensors]
    ops.compact_tail(dev, past, keep)
    for r, d in zip(ref, dev):
        assert np.array_equal(d.float().cpu().numpy(), r)


def test_compact_tail_edges():
    from mfd_b200 import ops
    x = torch.randn(1, 2, 30, 8, device=DEV)
    y = x.clone()
    ops.compact_tail([y], 20, [])  # empty keep: no change
    assert torch.equal(x, y)
    ops.compact_tail([y], 20, list(range(9, -1, -1)))  # keeps the whole window: no change (early return)
    assert torch.equal(x, y)
    ops.compact_tail([y], 30, [])  # empty window
    assert torch.equal(x, y)
    with pytest.raises(RuntimeError):
        ops.compact_tail([y], 20, [10])  # outside the window
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.compact_tail([y], 20, torch.tensor([0, 12], device=DEV), status=st)  # device keep, out of range: flagged
    assert int(st.item()) != 0


@pytest.mark.parametrize("slot_bytes", [2048, 40])
def test_commit_kv_moves_vs_oracle(slot_bytes):
    """Three requests owning disjoint slot ranges; move lists with no-ops, a chain of overlapping moves and the
    zeros past the path (as ddtree_follow writes them); 16-byte and 8-byte slot units."""
    from mfd_b200 import ddtree_utils, ops
    g = torch.Generator().manual_seed(slot_bytes)
    nbuf, nslots, width = 5, 300, 16
    words = slot_bytes // 8
    pool = torch.randint(-2**62, 2**62, (nbuf, nslots, words), generator=g, dtype=torch.int64)
    src = np.zeros((3, width), np.int64)
    tgt = np.zeros((3, width), np.int64)
    for b, base in enumerate((10, 110, 200)):
        path = [base + 40 + j for j in (0, 3, 4, 9, 12)]
        for i, s in enumerate(path):
            src[b, i], tgt[b, i] = s, base + 40 + i  # window slot of node -> slot of position i
        src[b, 5], tgt[b, 5] = base + 2, base + 2   # a no-op
        src[b, 6], tgt[b, 6] = base + 44, base + 45  # chain: 44 -> 45 while 45 -> ... above
    ref = oracle.commit_kv_moves(pool.numpy(), src, tgt)
    bufs = [pool[i].clone().to(DEV) for i in range(nbuf)]
    ops.commit_kv_moves(bufs, slot_bytes, torch.from_numpy(src).to(DEV), torch.from_numpy(tgt).to(DEV))
    for i in range(nbuf):
        assert np.array_equal(bufs[i].cpu().numpy(), ref[i]), i

    class Pool:  # the attributes DDTreeKVCompactor reads from SGLang's MHATokenToKVPool
        pass

    kv_pool = Pool()
    bufs2 = [pool[i].clone().to(DEV) for i in range(nbuf)]
    kv_pool.data_ptrs = torch.tensor([t.data_ptr() for t in bufs2], dtype=torch.int64, device=DEV)
    kv_pool.data_strides = torch.tensor([slot_bytes] * nbuf, dtype=torch.int64)
    assert ddtree_utils.DDTreeKVCompactor.supports(kv_pool)
    ddtree_utils.DDTreeKVCompactor(kv_pool)(move_src=torch.from_numpy(src).to(DEV),
                                            move_tgt=torch.from_numpy(tgt).to(DEV))
    for i in range(nbuf):
        assert np.array_equal(bufs2[i].cpu().numpy(), ref[i]), i


# ------------------------------------------------------------------------------------------------ GDN commit

@pytest.mark.parametrize("state_dtype", [torch.float32, torch.bfloat16])
def test_gdn_commit_matches_node_state_of_the_oracle(state_dtype):
    """Three layers: each state becomes S at the deepest accepted node, the oracle's per-node state (the formula
    of inference/hf/qwen35_tree.py:134-137 for every node), within 1e-3 of the state's scale (bf16: its rounding)."""
    from mfd_b200 import ops
    from tests.test_gdn import gdn_inputs, random_parents
    n, H, HK, D = 65, 8, 4, 128
    parents = random_parents(n, 5)
    leaf = n - 1
    path = [leaf]
    while parents[path[-1]] >= 0:
        path.append(int(parents[path[-1]]))
    path = path[::-1]
    states, us, ks, gs, refs = [], [], [], [], []
    for layer in range(3):
        q, k, v, G, beta, s0 = gdn_inputs(n, H, HK, D, parents, 40 + layer, s0_std=0.05)
        ru, _, rst = oracle.tree_gdn(q.float().numpy(), k.float().numpy(), v.float().numpy(), G.numpy(),
                                     beta.numpy(), s0.numpy(), parents, emit_states=True)
        states.append(s0.to(state_dtype).to(DEV))
        us.append(torch.from_numpy(ru).float().to(DEV))
        ks.append(k.bfloat16().to(DEV))
        gs.append(G.float().to(DEV))
        refs.append(rst[leaf])
    ops.gdn_commit(states, us, ks, gs, path)
    for s_, r in zip(states, refs):
        tol = (1e-3 if state_dtype == torch.float32 else 1e-2) * float(np.abs(r).max())
        np.testing.assert_allclose(s_.float().cpu().numpy(), r, rtol=0, atol=tol)


def test_conv_commit_matches_window_gather():
    from mfd_b200 import ops, qwen35_tree
    from tests.test_gdn import random_parents
    n, conv_dim, kernel = 65, 384, 4
    parents = list(random_parents(n, 7))
    ctx = qwen35_tree.TreeContext(parents, torch.from_numpy(oracle.visibility(np.array(parents))).bool(), kernel, DEV)
    g = torch.Generator().manual_seed(1)
    for node in (0, 5, n - 1):
        convs = [torch.randn(conv_dim, kernel, generator=g).bfloat16() for _ in range(2)]
        xs = [torch.randn(n, conv_dim, generator=g).bfloat16() for _ in range(2)]
        win = ctx.conv_index_cpu[node]
        refs = [torch.stack([c[:, i] if i < kernel else x[i - kernel] for i in win], dim=-1) for c, x in zip(convs, xs)]
        dc = [c.to(DEV) for c in convs]
        ops.conv_commit(dc, [x.to(DEV) for x in xs], ctx.conv_index[node])
        for d, r in zip(dc, refs):
            assert torch.equal(d.cpu(), r), node


def test_qwen35_commit_end_to_end():
    """qwen35_tree.commit on a cache of two GDN layers: states as the reference's commit formula gives them
    (oracle.commit_state, float64) and conv windows as its gather, then compact_attention is called."""
    from mfd_b200 import qwen35_tree
    from tests.test_gdn import gdn_inputs, random_parents
    n, H, HK, D, kernel = 33, 4, 2, 128, 4
    parents = list(random_parents(n, 9))
    ctx = qwen35_tree.TreeContext(parents, torch.from_numpy(oracle.visibility(np.array(parents))).bool(), kernel, DEV)
    conv_dim = (2 * HK + H) * D
    g = torch.Generator().manual_seed(2)

    class Layer:
        pass

    class Cache:
        layers = {}

    cache = Cache()
    expect = {}
    leaf = n - 1
    accepted = [leaf]
    while parents[accepted[-1]] >= 0:
        accepted.append(int(parents[accepted[-1]]))
    accepted = accepted[::-1]
    for li in (1, 3):
        q, k, v, G, beta, s0 = gdn_inputs(n, H, HK, D, np.array(parents), li)
        u = torch.randn(n, H, D, generator=g)
        x = torch.randn(n, conv_dim, generator=g).bfloat16()
        layer = Layer()
        layer.recurrent_states = s0[None].clone().to(DEV)
        layer.conv_states = torch.randn(1, conv_dim, kernel, generator=g).bfloat16().to(DEV)
        cache.layers[li] = layer
        ctx.records[li] = qwen35_tree._LayerRecord(u=u.to(DEV), k=k.bfloat16().to(DEV), G=G.float().to(DEV),
                                                   x=x.to(DEV))
        win = ctx.conv_index_cpu[accepted[-1]]
        conv_old = layer.conv_states[0].cpu()
        s_ref = oracle.commit_state(s0.numpy(), u.numpy(), k.bfloat16().float().numpy(), G.float().numpy(), accepted)
        expect[li] = (torch.from_numpy(s_ref).float(),
                      torch.stack([conv_old[:, i] if i < kernel else x[i - kernel] for i in win], dim=-1))
    called = []
    qwen35_tree.commit(cache, ctx, accepted, 100, lambda c, past, acc: called.append((past, list(acc))))
    assert called == [(100, accepted)] and ctx.records == {}
    for li, (s_ref, c_ref) in expect.items():
        torch.testing.assert_close(cache.layers[li].recurrent_states[0].cpu(), s_ref, rtol=0,
                                   atol=1e-5 * float(s_ref.abs().max()))
        assert torch.equal(cache.layers[li].conv_states[0].cpu(), c_ref)


def test_commit_kv_moves_skips_slot_ids_beyond_the_pool():
    from mfd_b200 import ops
    g = torch.Generator().manual_seed(5)
    nslots, width = 64, 8
    bufs = [torch.randint(-2**62, 2**62, (nslots, 256), generator=g, dtype=torch.int64).to(DEV) for _ in range(3)]
    before = [b.clone() for b in bufs]
    src = torch.zeros(2, width, dtype=torch.int64)
    tgt = torch.zeros(2, width, dtype=torch.int64)
    src[0, 0], tgt[0, 0] = 10, 3          # a valid move
    src[1, 0], tgt[1, 0] = nslots + 5, 4  # source beyond the pool
    src[1, 1], tgt[1, 1] = 6, 1 << 40     # target beyond the pool
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.commit_kv_moves(bufs, 2048, src.to(DEV), tgt.to(DEV), pool_slots=nslots, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 1  # MFD_ERR_INVALID
    for b, o in zip(bufs, before):
        want = o.clone()
        want[3] = o[10]
        assert torch.equal(b, want)  # only the valid move happened


def test_compact_tail_on_an_8_byte_aligned_view():
    from mfd_b200 import ops
    g = torch.Generator().manual_seed(6)
    flat = torch.randint(-2**62, 2**62, (2 * 30 * 16 + 1,), generator=g, dtype=torch.int64)
    view_cpu = flat[1:].view(2, 30, 16)
    ref = oracle.compact_tail(view_cpu.numpy(), 20, [3, 5, 9])
    dflat = flat.to(DEV)
    view = dflat[1:].view(2, 30, 16)
    assert view.data_ptr() % 16 == 8
    ops.compact_tail([view], 20, [3, 5, 9])
    assert np.array_equal(view.cpu().numpy(), ref)
