"""mfd_topk_logz_static (the allocation-free logits step) against mfd_topk_logz, both through the C ABI.

Named to be collected last, so it runs both after the rest of the suite and, on its own, in a fresh process
(the first call there also resolves the static scratch's device address)."""
import numpy as np
import pytest
import torch

from mfd_b200 import _lib
from mfd_b200._lib import MFD_BF16, MFD_F32, MFD_I64


def _run_workspace(lib, x, k, stream):
    R, V = x.shape
    top = torch.empty(R, k, dtype=torch.float32, device=x.device)
    ids = torch.empty(R, k, dtype=torch.int64, device=x.device)
    lz = torch.empty(R, dtype=torch.float32, device=x.device)
    ws = torch.empty(lib.mfd_topk_logz_workspace(R, V, k), dtype=torch.uint8, device=x.device)
    tk = torch.zeros(R, dtype=torch.int32, device=x.device)
    rc = lib.mfd_topk_logz(x.data_ptr(), MFD_BF16 if x.dtype == torch.bfloat16 else MFD_F32, R, V, x.stride(0), k,
                           top.data_ptr(), ids.data_ptr(), MFD_I64, lz.data_ptr(), ws.data_ptr(), ws.numel(),
                           tk.data_ptr(), tk.numel(), stream)
    _lib.check(rc, "mfd_topk_logz")
    return top, ids, lz


def _run_static(lib, x, k, stream):
    R, V = x.shape
    top = torch.full((R, k), float("nan"), dtype=torch.float32, device=x.device)
    ids = torch.full((R, k), -7, dtype=torch.int64, device=x.device)
    lz = torch.full((R,), float("nan"), dtype=torch.float32, device=x.device)
    rc = lib.mfd_topk_logz_static(x.data_ptr(), MFD_BF16 if x.dtype == torch.bfloat16 else MFD_F32, R, V,
                                  x.stride(0), k, top.data_ptr(), ids.data_ptr(), MFD_I64, lz.data_ptr(), stream)
    _lib.check(rc, "mfd_topk_logz_static")
    return top, ids, lz


@pytest.mark.gpu
def test_static_scratch_matches_workspace_entry_point_twice_in_a_row():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    # two different shapes back to back: the second call reuses scratch the first one left behind
    shapes = [(128, 151936, 64, torch.float32, 11), (37, 50021, 8, torch.bfloat16, 12)]
    for R, V, k, dtype, seed in shapes:
        g = torch.Generator().manual_seed(seed)
        x = (torch.randn(R, V, generator=g) * 3).to(dtype).to(dev)
        want = _run_workspace(lib, x, k, stream)
        got = _run_static(lib, x, k, stream)
        torch.cuda.synchronize()
        assert torch.equal(got[1], want[1])
        np.testing.assert_allclose(got[0].cpu().numpy(), want[0].cpu().numpy(), rtol=0, atol=1e-6)
        np.testing.assert_allclose(got[2].cpu().numpy(), want[2].cpu().numpy(), rtol=0, atol=1e-6)


def test_static_scratch_rejects_oversize_requests():
    lib = _lib.load()
    # 16385 rows exceed the ticket capacity; 8192 rows of a 151936 vocabulary exceed the partial records
    for R, V, k in [(16385, 1024, 8), (8192, 151936, 64)]:
        rc = lib.mfd_topk_logz_static(None, MFD_F32, R, V, V, k, None, None, MFD_I64, None, None)
        assert rc == 2
        assert b"static scratch" in lib.mfd_last_error()
    # invalid arguments report MFD_ERR_INVALID before any capacity check (k = 2^31 would overflow a doubling loop)
    for R, V, k in [(8192, 151936, 1 << 31), (4, 100, 257), (4, 100, 101)]:
        rc = lib.mfd_topk_logz_static(None, MFD_F32, R, V, V, k, None, None, MFD_I64, None, None)
        assert rc == 1
        assert b"invalid sizes" in lib.mfd_last_error()
    assert lib.mfd_topk_logz_workspace(8192, 151936, 1 << 31) == 0
