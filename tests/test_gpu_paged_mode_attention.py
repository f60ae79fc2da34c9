"""Paged drafter mode attention (the SGLang patch's paged_mode_block_attention, sglang-v0.5.22-mfd.patch:897-962):
the tcgen05 kernel gathering the context from a paged KV cache through req_to_token, against the oracle restatement
of paged_mode_block_attention_reference (patch:965-989), which composes the gather with the mode-attention reference
pinned in test_oracle_golden.py.  bf16 tolerance: max abs error <= 2e-2."""
import numpy as np
import pytest
import torch

from mfd_b200 import ops
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _batch(seed, ctx_lens, K=8, bs=16, H=32, Hkv=8, D=128, slots=None, pool_rows=None, width=None):
    g = torch.Generator().manual_seed(seed)
    nreq = len(ctx_lens)
    KL = K * bs
    T = nreq * KL
    width = width or max(max(ctx_lens), 1) + 5
    slots = slots or (sum(ctx_lens) + 257)
    pool_rows = pool_rows or nreq + 3
    q = torch.randn(T, H, D, generator=g).bfloat16()
    k_new = (torch.randn(T, Hkv, D, generator=g) * 1.5).bfloat16()
    v_new = torch.randn(T, Hkv, D, generator=g).bfloat16()
    k_cache = (torch.randn(slots, Hkv, D, generator=g) * 1.5).bfloat16()
    v_cache = torch.randn(slots, Hkv, D, generator=g).bfloat16()
    req_to_token = torch.randint(0, slots, (pool_rows, width), generator=g, dtype=torch.int32)
    perm = torch.randperm(slots, generator=g)
    rpi = torch.randperm(pool_rows, generator=g)[:nreq].to(torch.int64)
    off = 0
    for b, c in enumerate(ctx_lens):  # each request's context: distinct slots scattered over the pool
        req_to_token[rpi[b], :c] = perm[off:off + c].to(torch.int32)
        off += c
    ctx = torch.tensor(ctx_lens, dtype=torch.int64)
    return q, k_new, v_new, k_cache, v_cache, req_to_token, rpi, ctx


def _ref(host, ctx_list, K, bs, scale):
    return oracle.paged_mode_attention(host[0].float().numpy(), host[1].float().numpy(), host[2].float().numpy(),
                                       host[3].float().numpy(), host[4].float().numpy(), host[5].numpy(),
                                       host[6].numpy(), np.asarray(ctx_list), K, bs, scale)


def _check(host, K, bs, scale, splits):
    from mfd_b200.ddtree_mode_attention import paged_mode_block_attention
    q, k_new, v_new, k_cache, v_cache, r2t, rpi, ctx = [t.to(DEV) for t in host]
    got = paged_mode_block_attention(q=q, k_new=k_new, v_new=v_new, k_cache=k_cache, v_cache=v_cache,
                                     req_to_token=r2t, req_pool_indices=rpi, ctx_lens=ctx, num_modes=K, block_size=bs,
                                     scaling=scale, num_ctx_splits=splits)
    assert got.shape == q.shape and got.dtype == torch.bfloat16
    err = np.abs(got.float().cpu().numpy() - _ref(host, host[7].numpy(), K, bs, scale)).max()
    assert err <= 2e-2, err
    assert ops.tree_attention_status(purpose="paged_attn") == 0
    return got


@pytest.mark.parametrize("splits", [-1, 0, 3])
def test_paged_mode_attention_vs_oracle(splits):
    """Four requests with contexts of every alignment (multiple of 128, odd, shorter than a tile)."""
    _check(_batch(1, [1024, 37, 130, 4099]), 8, 16, 128 ** -0.5, splits)


@pytest.mark.parametrize("ctx_lens", [[0, 5], [1], [127, 128, 129, 3], [2048] * 6])
def test_paged_mode_attention_context_edges(ctx_lens):
    """Empty and one-token contexts (block keys only), tile-boundary lengths, and a larger batch."""
    _check(_batch(sum(ctx_lens) + len(ctx_lens), ctx_lens), 8, 16, 128 ** -0.5, -1)


@pytest.mark.parametrize("splits", [1, 2, 4, 7])
def test_paged_mode_attention_split_counts(splits):
    """Fixed split counts over mixed tiles (context and block keys in one tile), splits past the keys, and a
    request whose block keys form a split of their own."""
    _check(_batch(5, [77, 900, 512]), 8, 16, 128 ** -0.5, splits)


def test_paged_mode_attention_other_shapes_and_strided_cache():
    """Other mode counts, block sizes and head ratios; caches that are views of a wider pool buffer (row stride
    larger than Hkv * 128, as a K/V buffer with extra heads)."""
    from mfd_b200.ddtree_mode_attention import paged_mode_block_attention
    for K, bs, H, Hkv, ctx_lens in [(4, 8, 16, 16, [300, 64]), (2, 15, 8, 2, [129]), (16, 4, 32, 4, [64, 0, 700])]:
        host = _batch(K * 100 + bs, ctx_lens, K=K, bs=bs, H=H, Hkv=Hkv)
        q, k_new, v_new, k_cache, v_cache, r2t, rpi, ctx = host
        wide_k = torch.zeros(k_cache.shape[0], Hkv + 2, 128, dtype=torch.bfloat16)
        wide_v = torch.zeros_like(wide_k)
        wide_k[:, 1:Hkv + 1] = k_cache
        wide_v[:, 1:Hkv + 1] = v_cache
        got = paged_mode_block_attention(q=q.to(DEV), k_new=k_new.to(DEV), v_new=v_new.to(DEV),
                                         k_cache=wide_k.to(DEV)[:, 1:Hkv + 1], v_cache=wide_v.to(DEV)[:, 1:Hkv + 1],
                                         req_to_token=r2t.to(DEV), req_pool_indices=rpi.to(DEV),
                                         ctx_lens=ctx.to(DEV), num_modes=K, block_size=bs, scaling=128 ** -0.5,
                                         num_ctx_splits=-1)
        ref = _ref(host, ctx.numpy(), K, bs, 128 ** -0.5)
        assert np.abs(got.float().cpu().numpy() - ref).max() <= 2e-2, (K, bs, H, Hkv, ctx_lens)


def test_paged_matches_dense_mode_attention():
    """The paged kernel equals the dense mode attention on the same keys gathered contiguously (one request)."""
    from mfd_b200.ddtree_mode_attention import paged_mode_block_attention
    from mfd_b200.mode_attention import mode_block_attention
    K, bs, ctx = 8, 16, 1500
    q, k_new, v_new, k_cache, v_cache, r2t, rpi, ctx_t = _batch(7, [ctx])
    slots = r2t[rpi[0], :ctx].long()
    kd = torch.cat([k_cache[slots], k_new], 0).transpose(0, 1)[None].contiguous()  # [1, Hkv, ctx + KL, D]
    vd = torch.cat([v_cache[slots], v_new], 0).transpose(0, 1)[None].contiguous()
    dense = mode_block_attention(q.to(DEV).transpose(0, 1)[None], kd.to(DEV), vd.to(DEV), K, bs, 128 ** -0.5)
    paged = paged_mode_block_attention(q=q.to(DEV), k_new=k_new.to(DEV), v_new=v_new.to(DEV), k_cache=k_cache.to(DEV),
                                       v_cache=v_cache.to(DEV), req_to_token=r2t.to(DEV), req_pool_indices=rpi.to(DEV),
                                       ctx_lens=ctx_t.to(DEV), num_modes=K, block_size=bs, scaling=128 ** -0.5,
                                       num_ctx_splits=-1)
    assert (dense[0].float() - paged.float()).abs().max().item() <= 2e-2


def test_paged_mode_attention_cuda_graph():
    """Captured in a CUDA graph after a warm-up call: a replay with new context lengths (read on the device) equals
    an eager call with them, and both match the oracle."""
    from mfd_b200.ddtree_mode_attention import paged_mode_block_attention
    K, bs = 8, 16
    host = _batch(3, [500, 900, 33])
    q, k_new, v_new, k_cache, v_cache, r2t, rpi, ctx = [t.to(DEV) for t in host]
    out = torch.empty_like(q)
    kw = dict(q=q, k_new=k_new, v_new=v_new, k_cache=k_cache, v_cache=v_cache, req_to_token=r2t, req_pool_indices=rpi,
              ctx_lens=ctx, num_modes=K, block_size=bs, scaling=128 ** -0.5, num_ctx_splits=4, out=out)
    paged_mode_block_attention(**kw)
    assert np.abs(out.float().cpu().numpy() - _ref(host, [500, 900, 33], K, bs, 128 ** -0.5)).max() <= 2e-2
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        paged_mode_block_attention(**kw)
    new_ctx = [77, 900, 512]
    ctx.copy_(torch.tensor(new_ctx, device=DEV))
    g.replay()
    torch.cuda.synchronize()
    got = out.clone()
    want = paged_mode_block_attention(**{**kw, "out": None})
    ref = _ref(host, new_ctx, K, bs, 128 ** -0.5)
    assert np.abs(got.float().cpu().numpy() - ref).max() <= 2e-2
    assert np.abs(want.float().cpu().numpy() - ref).max() <= 2e-2
    assert torch.equal(got, want)
    assert ops.tree_attention_status(purpose="paged_attn") == 0
