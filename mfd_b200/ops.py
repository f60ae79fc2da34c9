"""Torch-facing wrappers of the C ABI: device tensors in, device tensors out, launches on the current stream.

These are the building blocks; the reference-shaped entry points live in ddtree.py, tree_build_ext.py,
tree_logits.py, ddtree_utils.py (SGLang), mode_attention.py, tree_gdn_kernel.py and qwen35_tree.py.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import MFD_BF16, MFD_F32, MFD_I32, MFD_I64, Workspace, check, ptr, require_cuda, stream_ptr


def _ids_code(dtype: torch.dtype) -> int:
    if dtype == torch.int32:
        return MFD_I32
    if dtype == torch.int64:
        return MFD_I64
    raise RuntimeError(f"ids must be int32 or int64, got {dtype}")


# ----------------------------------------------------------------------------------------------- logits step

def topk_logz(x: torch.Tensor, k: int, ids_dtype: torch.dtype = torch.int64, out=None):
    """x [..., V] float32/bf16 (CUDA, last dim contiguous) -> (top_logp f32 [..., k], ids [..., k], logz f32 [...]).

    top_logp = top - logsumexp(row); ids ordered by value descending, equal values by lower index first."""
    dev = require_cuda(x)
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise RuntimeError(f"topk_logz: x must be float32 or bfloat16, got {x.dtype}")
    V = x.shape[-1]
    rows2d = x.reshape(-1, V)
    if rows2d.stride(-1) != 1:
        rows2d = rows2d.contiguous()
    R = rows2d.shape[0]
    if out is None:
        top = torch.empty(R, k, dtype=torch.float32, device=dev)
        ids = torch.empty(R, k, dtype=ids_dtype, device=dev)
        logz = torch.empty(R, dtype=torch.float32, device=dev)
    else:
        top, ids, logz = out
    L = _lib.lib()
    ws_bytes = L.mfd_topk_logz_workspace(R, V, k)
    ws = Workspace.get(dev, "topk", ws_bytes)
    tk = Workspace.tickets(dev, R)
    rc = L.mfd_topk_logz(rows2d.data_ptr(), MFD_BF16 if x.dtype == torch.bfloat16 else MFD_F32, R, V,
                         rows2d.stride(0), k, top.data_ptr(), ids.data_ptr(), _ids_code(ids.dtype),
                         ptr(logz), ws.data_ptr(), ws.numel(), tk.data_ptr(), tk.numel(), stream_ptr(dev))
    check(rc, "mfd_topk_logz")
    lead = x.shape[:-1]
    return top.view(*lead, k), ids.view(*lead, k), logz.view(*lead)


# ----------------------------------------------------------------------------------------------- builders

def build_trees(top_logp: torch.Tensor, top_ids: torch.Tensor, log_prior: torch.Tensor | None, budget: int,
                single: bool = False, tree: torch.Tensor | None = None, counts: torch.Tensor | None = None,
                want_anc: bool = True, want_vis: bool = False, status: torch.Tensor | None = None):
    """top_logp [bs, K, L, k] f32, top_ids [bs, K, L, k] i32/i64, log_prior [bs, K] or None.

    Returns (tree [bs, 3, B+1] i64, counts [bs] i64, anc [bs, B+1, words] u64 as int64 or None,
    vis [bs, B+1, B+1] u8 or None)."""
    dev = require_cuda(top_logp, top_ids, log_prior)
    bs, K, L, k = top_logp.shape
    W = budget + 1
    if top_logp.dtype != torch.float32:
        raise RuntimeError("build_trees: top_logp must be float32")
    top_logp = top_logp.contiguous()
    top_ids = top_ids.contiguous()
    if log_prior is not None:
        log_prior = log_prior.to(torch.float32).contiguous()
    if tree is None:
        tree = torch.empty(bs, 3, W, dtype=torch.int64, device=dev)
    if counts is None:
        counts = torch.empty(bs, dtype=torch.int64, device=dev)
    words = (W + 63) // 64
    anc = torch.empty(bs, W, words, dtype=torch.int64, device=dev) if want_anc else None
    vis = torch.empty(bs, W, W, dtype=torch.uint8, device=dev) if want_vis else None
    rc = _lib.lib().mfd_build_trees(top_logp.data_ptr(), top_ids.data_ptr(), _ids_code(top_ids.dtype),
                                    ptr(log_prior), bs, K, L, k, budget, 1 if single else 0, tree.data_ptr(),
                                    counts.data_ptr(), ptr(anc), ptr(vis), ptr(status), stream_ptr(dev))
    check(rc, "mfd_build_trees")
    return tree, counts, anc, vis


# ----------------------------------------------------------------------------------------------- acceptance

def accept(logits: torch.Tensor, tokens: torch.Tensor, parents: torch.Tensor, temperature: float = 0.0,
           uniforms: torch.Tensor | None = None, max_steps: int = -1, out_len: int | None = None,
           window: torch.Tensor | None = None, prefix_lens: torch.Tensor | None = None):
    """logits [bs, W, V] bf16 (rows contiguous), tokens/parents [bs, W] i64 -> dict of device outputs."""
    dev = require_cuda(logits, tokens, parents, uniforms, window, prefix_lens)
    if logits.dtype != torch.bfloat16:
        raise RuntimeError("accept: logits must be bfloat16")
    bs, W, V = logits.shape
    rows = logits.reshape(bs * W, V)
    if rows.stride(-1) != 1:
        rows = rows.contiguous()
    if out_len is None:
        out_len = W if max_steps < 0 else max_steps + 1
    if tokens.stride(-1) != 1 or parents.stride(-1) != 1:
        raise RuntimeError("accept: tokens/parents need a contiguous last dim")
    if uniforms is not None:
        uniforms = uniforms.to(torch.float64).contiguous()
    o = {
        "posterior": torch.empty(bs, W, dtype=torch.int64, device=dev),
        "accept_len": torch.empty(bs, dtype=torch.int32, device=dev),
        "commit_lens": torch.empty(bs, dtype=torch.int32, device=dev),
        "bonus": torch.empty(bs, dtype=torch.int64, device=dev),
        "out_tokens": torch.empty(bs, out_len, dtype=torch.int64, device=dev),
        "accepted": torch.empty(bs, out_len, dtype=torch.int64, device=dev),
        "new_seq_lens": torch.empty(bs, dtype=torch.int64, device=dev),
        "hidden_index": torch.empty(bs, out_len, dtype=torch.int64, device=dev),
    }
    if window is not None:
        o["move_src"] = torch.empty(bs, out_len, dtype=torch.int64, device=dev)
        o["move_tgt"] = torch.empty(bs, out_len, dtype=torch.int64, device=dev)
    L = _lib.lib()
    ws = Workspace.get(dev, "accept", L.mfd_accept_workspace(bs, W))
    tk = Workspace.tickets(dev, L.mfd_accept_tickets(bs, W))
    rc = L.mfd_accept(rows.data_ptr(), rows.stride(0), V, bs, W, tokens.data_ptr(), tokens.stride(0),
                      parents.data_ptr(), parents.stride(0), float(temperature), ptr(uniforms), max_steps,
                      ptr(window), ptr(prefix_lens), out_len, o["posterior"].data_ptr(), o["accept_len"].data_ptr(),
                      o["commit_lens"].data_ptr(), o["bonus"].data_ptr(), o["out_tokens"].data_ptr(),
                      o["accepted"].data_ptr(), o["new_seq_lens"].data_ptr(), ptr(o.get("move_src")),
                      ptr(o.get("move_tgt")), o["hidden_index"].data_ptr(), ws.data_ptr(), ws.numel(),
                      tk.data_ptr(), tk.numel(), stream_ptr(dev))
    check(rc, "mfd_accept")
    return o


def sample_tokens(logits: torch.Tensor, temperature: float = 0.0, uniforms: torch.Tensor | None = None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """logits [..., V] bf16 -> int64 [...]: argmax (temperature < 1e-5) or the reproducible sample."""
    dev = require_cuda(logits, uniforms)
    if logits.dtype != torch.bfloat16:
        raise RuntimeError("sample_tokens: logits must be bfloat16")
    V = logits.shape[-1]
    rows = logits.reshape(-1, V)
    if rows.stride(-1) != 1:
        rows = rows.contiguous()
    R = rows.shape[0]
    if out is None:
        out = torch.empty(R, dtype=torch.int64, device=dev)
    if uniforms is not None:
        uniforms = uniforms.to(torch.float64).reshape(-1).contiguous()
    L = _lib.lib()
    ws = Workspace.get(dev, "accept", L.mfd_sample_tokens_workspace(R))
    tk = Workspace.tickets(dev, R + 1)
    rc = L.mfd_sample_tokens(rows.data_ptr(), rows.stride(0), V, R, float(temperature), ptr(uniforms),
                             out.data_ptr(), ws.data_ptr(), ws.numel(), tk.data_ptr(), tk.numel(), stream_ptr(dev))
    check(rc, "mfd_sample_tokens")
    return out.view(logits.shape[:-1])


def follow(posterior: torch.Tensor, tokens: torch.Tensor, parents: torch.Tensor, max_steps: int = -1,
           out_len: int | None = None, window: torch.Tensor | None = None, prefix_lens: torch.Tensor | None = None,
           outs: dict | None = None):
    """Walk only: posterior/tokens/parents [bs, W] i64 (CUDA)."""
    dev = require_cuda(posterior, tokens, parents, window, prefix_lens)
    bs, W = posterior.shape
    if out_len is None:
        out_len = W if max_steps < 0 else max_steps + 1
    posterior = posterior.contiguous()
    if outs is None:
        outs = {
            "accept_len": torch.empty(bs, dtype=torch.int32, device=dev),
            "commit_lens": torch.empty(bs, dtype=torch.int32, device=dev),
            "bonus": torch.empty(bs, dtype=torch.int64, device=dev),
            "out_tokens": torch.empty(bs, out_len, dtype=torch.int64, device=dev),
            "accepted": torch.empty(bs, out_len, dtype=torch.int64, device=dev),
            "new_seq_lens": torch.empty(bs, dtype=torch.int64, device=dev),
            "hidden_index": torch.empty(bs, out_len, dtype=torch.int64, device=dev),
        }
        if window is not None:
            outs["move_src"] = torch.empty(bs, out_len, dtype=torch.int64, device=dev)
            outs["move_tgt"] = torch.empty(bs, out_len, dtype=torch.int64, device=dev)
    rc = _lib.lib().mfd_follow(posterior.data_ptr(), tokens.data_ptr(), tokens.stride(0), parents.data_ptr(),
                               parents.stride(0), bs, W, max_steps, ptr(window), ptr(prefix_lens), out_len,
                               ptr(outs.get("accept_len")), ptr(outs.get("commit_lens")), ptr(outs.get("bonus")),
                               ptr(outs.get("out_tokens")), ptr(outs.get("accepted")), ptr(outs.get("new_seq_lens")),
                               ptr(outs.get("move_src")), ptr(outs.get("move_tgt")), ptr(outs.get("hidden_index")),
                               stream_ptr(dev))
    check(rc, "mfd_follow")
    return outs


# ----------------------------------------------------------------------------------------------- verify inputs

def verify_inputs(root_tokens, prefix_lens, tokens, depths, parents, mask_offsets, ids_out, positions_out,
                  mask_out, max_depth: int) -> None:
    dev = require_cuda(root_tokens, prefix_lens, tokens, depths, parents, mask_offsets, ids_out, positions_out,
                       mask_out)
    bs, W = tokens.shape
    if not (tokens.stride() == depths.stride() == parents.stride() and tokens.stride(1) == 1):
        raise RuntimeError("verify_inputs: tokens/depths/parents must share a row-contiguous layout")
    rc = _lib.lib().mfd_verify_inputs(root_tokens.data_ptr(), prefix_lens.data_ptr(), tokens.data_ptr(),
                                      depths.data_ptr(), parents.data_ptr(), tokens.stride(0),
                                      mask_offsets.data_ptr(), bs, W, max_depth, ids_out.data_ptr(),
                                      positions_out.data_ptr(), mask_out.data_ptr(), stream_ptr(dev))
    check(rc, "mfd_verify_inputs")


def compile_tree(root: torch.Tensor, tokens: torch.Tensor, depths: torch.Tensor, vis: torch.Tensor, n: int, start: int,
                 past_length: int, prev_start: int, prev_length: int, ids_out: torch.Tensor, positions_out: torch.Tensor,
                 mask: torch.Tensor, min_value: float, vis_out: torch.Tensor) -> None:
    """One tree's HF verify inputs (mfd_compile_tree): root int64 [1] / 0-dim, tokens and depths int64 [>= n] (slot 0
    the root), vis uint8 [>= n, >= n] (row-contiguous), all on the device; ids_out / positions_out int64 [>= n];
    mask [rows, cols] (bf16 / fp16 / fp32, last dim contiguous); vis_out bool [>= n, >= n].  min_value is written
    where a tree key is not visible, in mask's dtype."""
    dev = require_cuda(root, tokens, depths, vis, ids_out, positions_out, mask, vis_out)
    if mask.dim() != 2 or mask.stride(1) != 1 or mask.element_size() not in (2, 4):
        raise RuntimeError("compile_tree: mask must be 2-D with a contiguous last dim, 2- or 4-byte elements")
    if vis.stride(1) != 1 or vis_out.stride(1) != 1 or ids_out.stride(-1) != 1 or positions_out.stride(-1) != 1:
        raise RuntimeError("compile_tree: vis, vis_out, ids and positions need a contiguous last dim")
    bits_t = torch.int16 if mask.element_size() == 2 else torch.int32
    min_bits = int(torch.tensor(min_value, dtype=mask.dtype).view(bits_t).item()) & (0xFFFF if bits_t == torch.int16
                                                                                      else 0xFFFFFFFF)
    rc = _lib.lib().mfd_compile_tree(root.data_ptr(), tokens.data_ptr(), depths.data_ptr(), int(n), vis.data_ptr(),
                                     vis.stride(0), int(start), int(past_length), int(prev_start), int(prev_length),
                                     ids_out.data_ptr(), positions_out.data_ptr(), mask.data_ptr(), mask.element_size(),
                                     mask.stride(0), mask.shape[0], mask.shape[1], min_bits, vis_out.data_ptr(),
                                     vis_out.stride(0), stream_ptr(dev))
    check(rc, "mfd_compile_tree")


# ----------------------------------------------------------------------------------------------- attention

def attention_ctas(bs: int, n: int, num_heads: int, num_kv_heads: int, paged: bool = False) -> int:
    """CTAs of one key split of the attention kernel: one per (request, KV head, 128-row M-tile of the packed rows
    (node, query head of the group)); the paged launch pairs its M-tiles (one when there is only one)."""
    mtiles = (n * (num_heads // num_kv_heads) + 127) // 128
    return bs * num_kv_heads * ((mtiles + 1) // 2 if paged and mtiles >= 2 else mtiles)


def default_splits(bs: int, n: int, num_heads: int, num_kv_heads: int, keys: int) -> int:
    """Key splits of the attention: at most one wave of CTAs (one CTA per SM), each split at least 2 key tiles of
    128 (shorter splits would spend more on their partial (o, lse) records than on keys)."""
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    units = attention_ctas(bs, n, num_heads, num_kv_heads)
    want = max(1, sms // units)
    max_splits = max(1, (keys + 255) // 256)
    return int(min(want, max_splits))


def tree_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, anc: torch.Tensor, prefix_lens,
                   scale: float, splits: int | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """q [bs, n, H, D], k/v [bs, Hkv, S, D] bf16 (prefix keys then the n tree keys), anc [bs, n, words] i64,
    prefix_lens: int (same for all) or int32 [bs] CUDA tensor.  Returns [bs, n, H, D] bf16."""
    dev = require_cuda(q, k, v, anc)
    bs, n, H, D = q.shape
    Hkv = k.shape[1]
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise RuntimeError("tree_attention: q, k, v must be bfloat16")
    if q.stride(-1) != 1 or k.stride(-1) != 1 or v.stride(-1) != 1:
        raise RuntimeError("tree_attention: the head dim must be contiguous")
    if out is None:
        out = torch.empty(bs, n, H, D, dtype=torch.bfloat16, device=dev)
    if isinstance(prefix_lens, torch.Tensor):
        pl_t, pl_c = prefix_lens.to(torch.int32).contiguous(), 0
        max_keys = k.shape[2]
    else:
        pl_t, pl_c = None, int(prefix_lens)
        max_keys = pl_c + n
    if splits is None:
        splits = default_splits(bs, n, H, Hkv, max_keys)
    L = _lib.lib()
    ws = Workspace.get(dev, "attn", L.mfd_tree_attention_workspace(bs, n, H, Hkv, splits))
    nt = L.mfd_tree_attention_tickets(bs, n, H, Hkv)
    tk = Workspace.tickets(dev, nt)
    rc = L.mfd_tree_attention(q.data_ptr(), q.stride(0), q.stride(1), q.stride(2), k.data_ptr(), k.stride(0),
                              k.stride(1), k.stride(2), v.data_ptr(), v.stride(0), v.stride(1), v.stride(2),
                              k.shape[2], ptr(pl_t), pl_c, anc.data_ptr(), anc.shape[-1], bs, n, H, Hkv, D,
                              float(scale), splits, out.data_ptr(), out.stride(0), out.stride(1), out.stride(2),
                              ws.data_ptr(), ws.numel(), tk.data_ptr(), tk.numel(), stream_ptr(dev))
    check(rc, "mfd_tree_attention")
    return out


def paged_mode_attention(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, k_cache: torch.Tensor,
                         v_cache: torch.Tensor, req_to_token: torch.Tensor, req_pool_indices: torch.Tensor,
                         ctx_lens: torch.Tensor, block_bits: torch.Tensor, num_modes: int, block_size: int,
                         scale: float, splits: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """q [T, H, 128], k_new/v_new [T, Hkv, 128] (T = bs * K * block_size, mode-major per request); k_cache/v_cache
    [slots, Hkv, 128]; request b's context is k_cache[req_to_token[req_pool_indices[b], :ctx_lens[b]]].
    block_bits [1, K*block_size, words] int64: the block-diagonal visibility.  Returns [T, H, 128] bf16."""
    dev = require_cuda(q, k_new, v_new, k_cache, v_cache, req_to_token, req_pool_indices, ctx_lens, block_bits)
    T, H, D = q.shape
    Hkv = k_new.shape[1]
    n = num_modes * block_size
    bs = T // n if n > 0 else 0
    if T != bs * n:
        raise RuntimeError(f"paged_mode_attention: {T} queries are not a multiple of num_modes * block_size = {n}")
    for t in (q, k_new, v_new, k_cache, v_cache):
        if t.dtype != torch.bfloat16:
            raise RuntimeError("paged_mode_attention: q, k, v and the caches must be bfloat16")
    if req_to_token.dtype != torch.int32:
        req_to_token = req_to_token.to(torch.int32)
    if req_to_token.stride(1) != 1:
        req_to_token = req_to_token.contiguous()
    rpi = req_pool_indices[:bs].to(torch.int64).contiguous()
    ctx = ctx_lens[:bs].to(torch.int64).contiguous()
    if out is None:
        out = torch.empty(T, H, D, dtype=torch.bfloat16, device=dev)
    if bs == 0:
        return out
    L = _lib.lib()
    ws = Workspace.get(dev, "paged_attn", L.mfd_tree_attention_workspace(bs, n, H, Hkv, splits))
    tk = Workspace.tickets(dev, L.mfd_tree_attention_tickets(bs, n, H, Hkv))
    rc = L.mfd_paged_mode_attention(q.data_ptr(), q.stride(0), q.stride(1), k_new.data_ptr(), k_new.stride(0),
                                    k_new.stride(1), v_new.data_ptr(), v_new.stride(0), v_new.stride(1),
                                    k_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1), v_cache.data_ptr(),
                                    v_cache.stride(0), v_cache.stride(1), k_cache.shape[0], req_to_token.data_ptr(),
                                    req_to_token.shape[0], req_to_token.shape[1], req_to_token.stride(0),
                                    rpi.data_ptr(), ctx.data_ptr(), block_bits.data_ptr(), block_bits.shape[-1], bs,
                                    num_modes, block_size, H, Hkv, D, float(scale), splits, out.data_ptr(),
                                    out.stride(0), out.stride(1), ws.data_ptr(), ws.numel(), tk.data_ptr(),
                                    tk.numel(), stream_ptr(dev))
    check(rc, "mfd_paged_mode_attention")
    return out


def tree_attention_status(device=None, purpose: str = "attn") -> int:
    """The sticky status word at the head of an attention workspace (the first int32 at its 256-byte aligned base):
    0; 1 once a bounded wait in the kernel gave up; 2 when a CTA found its shared-memory base misaligned beyond the
    reserved slack and did no work.  0 when no such call has run on the device.  purpose "attn": tree_attention
    and the dense mode attention; "paged_attn": paged_mode_attention."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    ws = Workspace._cache.get((dev.index if dev.index is not None else torch.cuda.current_device(), purpose))
    if ws is None:
        return 0
    off = (-ws.data_ptr()) % 256
    return int(ws[off:off + 4].view(torch.int32).item())


# ----------------------------------------------------------------------------------------------- tree GDN

def tree_gdn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g_cum: torch.Tensor, beta: torch.Tensor,
             s0: torch.Tensor, anc8: torch.Tensor, emit_states: bool = False, out=None, status=None):
    """q, k [n, HK, Dk] bf16, v [n, H, Dv] bf16, g_cum/beta [n, H] f32, s0 [H, Dk, Dv] f32, anc8 [n, n] int8.

    Returns (u, o) float32 [n, H, Dv], plus the per-node states float32 [n, H, Dk, Dv] when emit_states."""
    dev = require_cuda(q, k, v, g_cum, beta, s0, anc8)
    n, HK, Dk = k.shape
    H, Dv = v.shape[1], v.shape[2]
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise RuntimeError("tree_gdn: q, k, v must be bfloat16")
    if q.shape != k.shape or v.shape[0] != n or tuple(anc8.shape) != (n, n):
        raise RuntimeError("tree_gdn: inconsistent shapes")
    q = q if q.stride(2) == 1 and q.stride(1) == Dk else q.contiguous()
    k = k if k.stride(2) == 1 and k.stride(1) == Dk else k.contiguous()
    v = v if v.stride(2) == 1 and v.stride(1) == Dv else v.contiguous()
    g_cum = g_cum.float()
    beta = beta.float()
    g_cum = g_cum if g_cum.stride(1) == 1 else g_cum.contiguous()
    beta = beta if beta.stride(1) == 1 else beta.contiguous()
    s0 = s0.float().contiguous()
    anc8 = anc8.to(torch.int8)
    anc8 = anc8 if anc8.stride(1) == 1 else anc8.contiguous()
    if out is None:
        u = torch.empty(n, H, Dv, dtype=torch.float32, device=dev)
        o = torch.empty(n, H, Dv, dtype=torch.float32, device=dev)
        st = torch.empty(n, H, Dk, Dv, dtype=torch.float32, device=dev) if emit_states else None
    else:
        u, o, st = out
    rc = _lib.lib().mfd_tree_gdn(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
                                 g_cum.data_ptr(), g_cum.stride(0), beta.data_ptr(), beta.stride(0), s0.data_ptr(),
                                 anc8.data_ptr(), anc8.stride(0), n, H, HK, Dk, Dv, u.data_ptr(), o.data_ptr(),
                                 ptr(st), ptr(status), stream_ptr(dev))
    check(rc, "mfd_tree_gdn")
    return (u, o, st) if emit_states else (u, o)


def tree_gates(a: torch.Tensor, b: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor, parents: torch.Tensor,
               status: torch.Tensor | None = None):
    """a, b [n, H] (the layer's in_proj_a / in_proj_b outputs, bf16 or float32), a_log, dt_bias [H], parents [n]
    int64 on the device -> (beta, G) float32 [n, H]: sigmoid(b) and the per-token log decay
    -exp(A_log) softplus(a + dt_bias) summed along each node's root path."""
    dev = require_cuda(a, b, a_log, dt_bias, parents, status)
    n, H = a.shape
    if b.shape != a.shape or b.dtype != a.dtype or a.dtype not in (torch.bfloat16, torch.float32):
        raise RuntimeError("tree_gates: a and b must be [n, H] of one dtype, bf16 or float32")
    a = a if a.stride(1) == 1 else a.contiguous()
    b = b if b.stride(1) == 1 else b.contiguous()
    a_log = a_log.float().contiguous()
    dt_bias = dt_bias.float().contiguous()
    parents = parents.to(torch.int64).contiguous()
    beta = torch.empty(n, H, dtype=torch.float32, device=dev)
    G = torch.empty(n, H, dtype=torch.float32, device=dev)
    rc = _lib.lib().mfd_tree_gates(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0),
                                   MFD_BF16 if a.dtype == torch.bfloat16 else MFD_F32, a_log.data_ptr(),
                                   dt_bias.data_ptr(), parents.data_ptr(), n, H, beta.data_ptr(), G.data_ptr(),
                                   ptr(status), stream_ptr(dev))
    check(rc, "mfd_tree_gates")
    return beta, G


def tree_prep(x: torch.Tensor, conv_state: torch.Tensor, conv_index: torch.Tensor, conv_w: torch.Tensor,
              num_k_heads: int, num_v_heads: int, head_dim: int):
    """x [n, conv_dim] bf16, conv_state [conv_dim, KC] bf16, conv_index [n, KC] int32, conv_w [conv_dim, KC] bf16.

    Returns q (l2-normalised, scaled by head_dim^-0.5), k (l2-normalised) [n, H_k, D] and v [n, H, D], bf16."""
    dev = require_cuda(x, conv_state, conv_index, conv_w)
    n, cd = x.shape
    kc = conv_w.shape[1]
    x = x.to(torch.bfloat16).contiguous()
    conv_state = conv_state.to(torch.bfloat16).contiguous()
    conv_w = conv_w.to(torch.bfloat16).contiguous()
    conv_index = conv_index.to(torch.int32).contiguous()
    q = torch.empty(n, num_k_heads, head_dim, dtype=torch.bfloat16, device=dev)
    k = torch.empty_like(q)
    v = torch.empty(n, num_v_heads, head_dim, dtype=torch.bfloat16, device=dev)
    rc = _lib.lib().mfd_tree_prep(x.data_ptr(), conv_state.data_ptr(), conv_index.data_ptr(), conv_w.data_ptr(), n,
                                  cd, kc, num_k_heads, num_v_heads, head_dim, float(head_dim ** -0.5), q.data_ptr(),
                                  k.data_ptr(), v.data_ptr(), stream_ptr(dev))
    check(rc, "mfd_tree_prep")
    return q, k, v


# ----------------------------------------------------------------------------------------------- commit step

_PTR_CACHE: dict = {}


def _pointer_array(tensors, dev, extra=()) -> torch.Tensor:
    """A device int64 array of the tensors' base addresses (then `extra` values), cached by its contents: a call
    on the same buffers (a serving loop, a captured graph) copies nothing to the device."""
    key = (dev.index if dev.index is not None else torch.cuda.current_device(),
           tuple(t.data_ptr() for t in tensors) + tuple(int(v) for v in extra))
    arr = _PTR_CACHE.get(key)
    if arr is None:
        if len(_PTR_CACHE) >= 256:
            _PTR_CACHE.clear()
        arr = torch.tensor(list(key[1]), dtype=torch.int64, device=dev)
        _PTR_CACHE[key] = arr
    return arr


def _base_align(addr: int) -> int:
    return 16 if addr % 16 == 0 else 8


def commit_kv_moves(buffers, slot_bytes: int, move_src: torch.Tensor, move_tgt: torch.Tensor,
                    base_align: int | None = None, pool_slots: int = 0, status: torch.Tensor | None = None) -> None:
    """The commit step's KV moves in a token-major pool: for request b and i < width, slot move_src[b, i] moves to
    move_tgt[b, i] in every buffer when they differ, every source read before any store.  buffers: a list of
    CUDA tensors (one per layer K / V buffer, slot_bytes per slot) or a device int64 tensor of base addresses
    (the pool's data_ptrs, with `base_align` the alignment all of them have; 8 when not given).  move_src,
    move_tgt [bs, width] int64 on the device.  pool_slots > 0: moves with a slot id >= pool_slots are skipped and
    flagged in `status` (device int32).  One launch."""
    dev = require_cuda(move_src, move_tgt, status)
    if isinstance(buffers, torch.Tensor) and buffers.dtype == torch.int64 and buffers.dim() == 1:
        ptrs = buffers.to(dev)
        align = 8 if base_align is None else int(base_align)
    else:
        buffers = list(buffers)
        for t in buffers:
            if not t.is_cuda or t.data_ptr() % 8:
                raise RuntimeError("commit_kv_moves: buffers must be CUDA tensors aligned to 8 bytes")
        align = min([_base_align(t.data_ptr()) for t in buffers] or [16])
        ptrs = _pointer_array(buffers, dev)
    src = move_src.to(torch.int64).contiguous()
    tgt = move_tgt.to(torch.int64).contiguous()
    if src.shape != tgt.shape or src.dim() != 2:
        raise RuntimeError("commit_kv_moves: move_src and move_tgt must both be [bs, width]")
    rc = _lib.lib().mfd_commit_kv_moves(ptrs.data_ptr(), ptrs.numel(), int(slot_bytes), align, src.data_ptr(),
                                        tgt.data_ptr(), src.shape[0], src.shape[1], int(pool_slots), ptr(status),
                                        stream_ptr(dev))
    check(rc, "mfd_commit_kv_moves")


def compact_tail(tensors, past_length: int, keep, status: torch.Tensor | None = None) -> None:
    """Row past_length + keep[i] -> past_length + i along dim -2 of every tensor (HF caches [..., S, D]), in place,
    all tensors of one layout and base alignment in one launch; no-op when the appended window is empty or keep is
    empty or keeps the whole window (the reference's early returns).  keep: a list of ints or a device int64
    tensor.  A tensor whose base is only 8-byte aligned goes to the 8-byte path."""
    tensors = [t for t in tensors if t is not None and t.numel() > 0]
    if not tensors:
        return
    dev = require_cuda(*tensors)
    if isinstance(keep, torch.Tensor):
        keep_t = keep.to(device=dev, dtype=torch.int64).contiguous()
    else:
        keep_l = [int(i) for i in keep]
        S = tensors[0].shape[-2]
        if any(i < 0 or past_length + i >= S for i in keep_l):
            raise RuntimeError("compact_tail: keep index outside the appended window")
        keep_t = torch.tensor(keep_l, dtype=torch.int64, device=dev)
    groups: dict = {}
    for t in tensors:
        if t.dim() < 2 or t.stride(-1) != 1:
            raise RuntimeError("compact_tail: tensors need a contiguous last dim")
        if t.data_ptr() % 8:
            raise RuntimeError("compact_tail: tensors must start on an 8-byte boundary")
        outer = t.numel() // (t.shape[-2] * t.shape[-1])
        try:
            v = t.view(outer, t.shape[-2], t.shape[-1]) if t.dim() != 3 or outer != t.shape[0] else t
        except RuntimeError as e:
            raise RuntimeError("compact_tail: the dims before the last two must collapse into one stride") from e
        es = t.element_size()
        key = (tuple(v.shape), v.stride(0) * es, v.stride(1) * es, v.shape[2] * es, _base_align(v.data_ptr()))
        groups.setdefault(key, []).append(v)
    L = _lib.lib()
    for (shape, outer_stride, row_stride, row_bytes, align), views in groups.items():
        ptrs = _pointer_array(views, dev)
        rc = L.mfd_compact_tail(ptrs.data_ptr(), ptrs.numel(), shape[0], outer_stride, shape[1], row_stride, row_bytes,
                                align, int(past_length), keep_t.data_ptr(), keep_t.numel(), ptr(status),
                                stream_ptr(dev))
        check(rc, "mfd_compact_tail")


def compact_tail_groups(tensors) -> list:
    """The launch groups compact_tail forms for these tensors: (shape, outer stride, row stride, row bytes, base
    alignment) per group, in first-seen order.  Host logic only (no launch)."""
    keys = []
    for t in tensors:
        outer = t.numel() // (t.shape[-2] * t.shape[-1])
        es = t.element_size()
        v = t.view(outer, t.shape[-2], t.shape[-1]) if t.dim() != 3 or outer != t.shape[0] else t
        key = (tuple(v.shape), v.stride(0) * es, v.stride(1) * es, v.shape[2] * es, _base_align(v.data_ptr()))
        if key not in keys:
            keys.append(key)
    return keys


def gdn_commit(states, us, ks, gs, path) -> None:
    """Every layer's recurrent state (in place) -> the state at the deepest accepted node path[-1]:
    S_a = e^{G_a} S0 + sum_{j in path} e^{G_a - G_j} k_j u_j^T.  states: per layer [H, Dk, Dv] (or [1, H, Dk, Dv])
    float32 / bf16; us [n, H, Dv] float32, ks [n, HK, Dk] bf16, gs [n, H] float32 per layer; path: list or device
    int64 tensor.  One launch for all layers."""
    states = list(states)
    if not states:
        return
    dev = require_cuda(*states)
    H, Dk, Dv = states[0].shape[-3:]
    n, HK = ks[0].shape[0], ks[0].shape[1]
    sdt = states[0].dtype
    if sdt not in (torch.float32, torch.bfloat16):
        raise RuntimeError("gdn_commit: states must be float32 or bfloat16")
    for s_, u_, k_, g_ in zip(states, us, ks, gs):
        if (not s_.is_contiguous() or s_.dtype != sdt or tuple(s_.shape[-3:]) != (H, Dk, Dv) or s_.numel() != H * Dk * Dv
                or u_.dtype != torch.float32 or not u_.is_contiguous() or tuple(u_.shape) != (n, H, Dv)
                or k_.dtype != torch.bfloat16 or not k_.is_contiguous() or tuple(k_.shape) != (n, HK, Dk)
                or g_.dtype != torch.float32 or not g_.is_contiguous() or tuple(g_.shape) != (n, H)):
            raise RuntimeError("gdn_commit: per-layer tensors must be contiguous with the documented shapes/dtypes")
        if s_.data_ptr() % 16 or u_.data_ptr() % 16 or Dv % 4:
            raise RuntimeError("gdn_commit: states and u need 16-byte aligned bases and Dv a multiple of 4")
    # one device array: the four per-layer address lists, then the path (a device path tensor is used as given)
    nl = len(states)
    on_device = isinstance(path, torch.Tensor)
    if on_device:
        path_t, plist = path.to(device=dev, dtype=torch.int64).contiguous(), ()
    else:
        plist = tuple(int(i) for i in path)
        if not plist or any(not (0 <= i < n) for i in plist):
            raise RuntimeError("gdn_commit: the path must be a non-empty list of nodes of the tree")
    arr = _pointer_array(list(states) + list(us) + list(ks) + list(gs), dev, plist)
    base = arr.data_ptr()
    path_ptr = path_t.data_ptr() if on_device else base + 8 * 4 * nl
    plen = path_t.numel() if on_device else len(plist)
    rc = _lib.lib().mfd_gdn_commit(base, MFD_F32 if sdt == torch.float32 else MFD_BF16, base + 8 * nl,
                                   base + 16 * nl, base + 24 * nl, nl, path_ptr, plen, n, H, HK, Dk, Dv,
                                   stream_ptr(dev))
    check(rc, "mfd_gdn_commit")


def conv_commit(conv_states, xs, window) -> None:
    """Every layer's conv window (in place): column t = old column window[t] (< kernel) or x[window[t] - kernel].
    conv_states per layer [conv_dim, kernel] (or [1, conv_dim, kernel]); xs per layer [n, conv_dim] of the same
    dtype; window: the accepted node's window (list or device int tensor).  One launch for all layers."""
    conv_states = list(conv_states)
    if not conv_states:
        return
    dev = require_cuda(*conv_states)
    conv_dim, kernel = conv_states[0].shape[-2:]
    for c_, x_ in zip(conv_states, xs):
        if (not c_.is_contiguous() or not x_.is_contiguous() or x_.dtype != c_.dtype or x_.shape[-1] != conv_dim
                or tuple(c_.shape[-2:]) != (conv_dim, kernel)):
            raise RuntimeError("conv_commit: conv states [conv_dim, kernel] and inputs [n, conv_dim] of one dtype")
    win = window.to(device=dev, dtype=torch.int32).contiguous() if isinstance(window, torch.Tensor) else \
        torch.tensor([int(i) for i in window], dtype=torch.int32, device=dev)
    # (the pointer array is cached, so it stays alive while the kernel reads it)
    pa = _pointer_array(conv_states + list(xs), dev)
    nl = len(conv_states)
    rc = _lib.lib().mfd_conv_commit(pa.data_ptr(), pa.data_ptr() + 8 * nl, conv_states[0].element_size(), nl,
                                    conv_dim, kernel, win.data_ptr(), stream_ptr(dev))
    check(rc, "mfd_conv_commit")
