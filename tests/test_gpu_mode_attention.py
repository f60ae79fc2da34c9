"""Drafter mode attention (mode_block_attention, the masked split-KV kernel with a block-diagonal visibility) against
the oracle restatement of inference/hf/mode_attention.py:153-164 (`reference`, pinned to the reference's own output in
test_oracle_golden.py) and against that fixture directly.  bf16 tolerance: max abs error <= 2e-2 (the reference's own
check, inference/hf/mode_attention.py:178)."""
import numpy as np
import pytest
import torch

from oracle import oracle
from tests._golden import bf16_from_i16, load

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("ctx", [1, 37, 500, 2048, 4096])
def test_mode_attention_vs_oracle(ctx):
    from mfd_b200.mode_attention import mode_block_attention
    K, bs, H, Hkv, D = 8, 16, 32, 8, 128
    g = torch.Generator().manual_seed(ctx)
    q = torch.randn(1, H, K * bs, D, generator=g).bfloat16()
    k = (torch.randn(1, Hkv, ctx + K * bs, D, generator=g) * 2).bfloat16()
    v = torch.randn(1, Hkv, ctx + K * bs, D, generator=g).bfloat16()
    got = mode_block_attention(q.to(DEV), k.to(DEV), v.to(DEV), K, bs, D ** -0.5)
    assert got.shape == (1, K * bs, H, D) and got.dtype == torch.bfloat16
    ref = oracle.mode_attention(q[0].float().numpy(), k[0].float().numpy(), v[0].float().numpy(), K, bs, D ** -0.5)
    assert np.abs(got[0].float().cpu().numpy() - ref).max() <= 2e-2


def test_mode_attention_other_shapes():
    """Other mode counts / block sizes / head ratios, q given as a strided view."""
    from mfd_b200.mode_attention import mode_block_attention
    for K, bs, H, Hkv, ctx in [(4, 8, 16, 16, 300), (2, 15, 8, 2, 129), (16, 4, 32, 4, 64)]:
        g = torch.Generator().manual_seed(K * 100 + bs)
        qf = torch.randn(1, K * bs, H, 128, generator=g).bfloat16()
        q = qf.to(DEV).transpose(1, 2)  # [1, H, T, D] with non-contiguous strides
        k = torch.randn(1, Hkv, ctx + K * bs, 128, generator=g).bfloat16()
        v = torch.randn(1, Hkv, ctx + K * bs, 128, generator=g).bfloat16()
        got = mode_block_attention(q, k.to(DEV), v.to(DEV), K, bs, 128 ** -0.5)
        ref = oracle.mode_attention(qf[0].transpose(0, 1).float().numpy(), k[0].float().numpy(), v[0].float().numpy(),
                                    K, bs, 128 ** -0.5)
        assert np.abs(got[0].float().cpu().numpy() - ref).max() <= 2e-2, (K, bs, H, Hkv, ctx)


def test_mode_attention_reference_fixture():
    """The reference's own masked-SDPA outputs (K=4, bs=8, 4/2 heads)."""
    from mfd_b200.mode_attention import mode_block_attention
    z = load("mode_attention.npz")
    K, bs = int(z["K"]), int(z["bs"])
    for i in range(int(z["n"])):
        q, k, v = (torch.from_numpy(bf16_from_i16(z[f"c{i}_{t}"])).bfloat16() for t in "qkv")
        got = mode_block_attention(q.to(DEV), k.to(DEV), v.to(DEV), K, bs, 128 ** -0.5)
        assert np.abs(got.float().cpu().numpy() - z[f"c{i}_out"]).max() <= 2e-2, i
