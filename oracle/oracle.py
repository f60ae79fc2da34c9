"""CPU oracle for the MFD verify step -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs import
this module, and only as the checker.  The product package (mfd_b200) never imports it.

Integer and index work (tree builders, visibility, walk, sampling rule, argmax) runs in the plain-C
restatement oracle/mfd_oracle.c through ctypes.  Floating-point paths are restated with numpy:

  topk_logz          hf/ddtree.py:240-244 (float32 top-k and logsumexp); ties ordered by lower index
                     first (this build's contract; torch's CPU top-k leaves tie order unspecified)
  tree_attention     hf/ddtree.py:352-356 (mask: prefix visible, tree block ancestor-only, the
                     compile_ddtree_tree mask) + SDPA with GQA head repetition
  mode_attention     hf/mode_attention.py:216-227 (`reference`: whole context + own mode block)
  tree_gdn           tests/test_gdn_tree_math.py:29-60 (chunk form with ancestor mask, one
                     triangular solve) with the GQA key-head map of hf/tree_gdn_kernel.py:71, 101,
                     per-node states by the commit formula hf/qwen35_tree.py:134-137
  compile_tree       hf/ddtree.py:317-357 (compile_ddtree_tree: verify ids, positions, additive tree mask)
  tree_gates         hf/qwen35_tree.py:77-79 (beta, softplus decay, G = anc_f @ g)
  tree_prep          hf/tree_gdn_kernel.py:27-56 (_tree_prep: windowed conv through parent pointers,
                     SiLU rounded to bf16, l2norm + q scale); pinned against torch's causal conv1d on chains

Parity pins: tests/golden/ holds fixtures made by tests/golden/make_golden.py from the reference
itself (its Python builders, compiled C++ builders, walk, mode-attention reference and verify mask);
tests/test_oracle_golden.py checks this oracle against them.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libmfd_oracle.so")
_LIB = None

_i64p = ctypes.POINTER(ctypes.c_int64)
_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_f64p = ctypes.POINTER(ctypes.c_double)


def build() -> str:
    """Compile oracle/mfd_oracle.c (gcc) into oracle/_build/libmfd_oracle.so."""
    src = os.path.join(_HERE, "mfd_oracle.c")
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-C", _HERE, "-s"], check=True)
    return _LIB_PATH


def lib():
    global _LIB
    if _LIB is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        L.oracle_build_mixture.restype = ctypes.c_int64
        L.oracle_build_mixture.argtypes = [_f32p, _i64p, _f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_int64, _i64p, _i64p, _i64p, _i64p]
        L.oracle_build_single.restype = ctypes.c_int64
        L.oracle_build_single.argtypes = [_f32p, _i64p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                          _i64p, _i64p, _i64p, _i64p]
        L.oracle_build_trees.restype = None
        L.oracle_build_trees.argtypes = [_f32p, _i32p, _f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int64, ctypes.c_int64, _i64p, _i64p]
        L.oracle_visibility.restype = None
        L.oracle_visibility.argtypes = [_i64p, ctypes.c_int64, _u8p]
        L.oracle_follow.restype = ctypes.c_int64
        L.oracle_follow.argtypes = [_i64p, _i64p, ctypes.c_int64, _i64p, ctypes.c_int64, _i64p, _i64p]
        L.oracle_sample_rows.restype = None
        L.oracle_sample_rows.argtypes = [_u16p, ctypes.c_int64, ctypes.c_int64, ctypes.c_float, _f64p, _i64p]
        L.oracle_argmax_rows.restype = None
        L.oracle_argmax_rows.argtypes = [_u16p, ctypes.c_int64, ctypes.c_int64, _i64p]
        L.oracle_exp32.restype = ctypes.c_float
        L.oracle_exp32.argtypes = [ctypes.c_float]
        _LIB = L
    return _LIB


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


# ------------------------------------------------------------------------------------------ builders

def build_mixture(top_logp: np.ndarray, top_ids: np.ndarray, prior: np.ndarray, budget: int, stats=None):
    """[K, L, k] float32 / int64, [K] float32 -> (tokens [n], depths [n], parents [n+1]) int64."""
    lp = np.ascontiguousarray(top_logp, dtype=np.float32)
    ids = np.ascontiguousarray(top_ids, dtype=np.int64)
    pr = np.ascontiguousarray(prior, dtype=np.float32)
    K, L, k = lp.shape
    tok = np.empty(max(budget, 1), np.int64)
    dep = np.empty(max(budget, 1), np.int64)
    par = np.empty(max(budget, 0) + 1, np.int64)
    pops = np.zeros(1, np.int64)
    n = lib().oracle_build_mixture(_p(lp, _f32p), _p(ids, _i64p), _p(pr, _f32p), K, L, k, budget,
                                   _p(tok, _i64p), _p(dep, _i64p), _p(par, _i64p), _p(pops, _i64p))
    if stats is not None:
        stats["pops"] = int(pops[0])
    return tok[:n].copy(), dep[:n].copy(), par[:n + 1].copy()


def build_single(top_logp: np.ndarray, top_ids: np.ndarray, budget: int, stats=None):
    """[L, k] float32 / int64 -> (tokens [n], depths [n], parents [n+1]) int64."""
    lp = np.ascontiguousarray(top_logp, dtype=np.float32)
    ids = np.ascontiguousarray(top_ids, dtype=np.int64)
    L, k = lp.shape
    tok = np.empty(max(budget, 1), np.int64)
    dep = np.empty(max(budget, 1), np.int64)
    par = np.empty(max(budget, 0) + 1, np.int64)
    pops = np.zeros(1, np.int64)
    n = lib().oracle_build_single(_p(lp, _f32p), _p(ids, _i64p), L, k, budget, _p(tok, _i64p), _p(dep, _i64p),
                                  _p(par, _i64p), _p(pops, _i64p))
    if stats is not None:
        stats["pops"] = int(pops[0])
    return tok[:n].copy(), dep[:n].copy(), par[:n + 1].copy()


def build_trees(top_logp: np.ndarray, top_ids: np.ndarray, prior: np.ndarray, budget: int):
    """SGLang layout: [bs, K, L, k] float32 / int32, [bs, K] -> tree [bs, 3, B+1] int64, counts [bs]."""
    lp = np.ascontiguousarray(top_logp, dtype=np.float32)
    ids = np.ascontiguousarray(top_ids, dtype=np.int32)
    pr = np.ascontiguousarray(prior, dtype=np.float32)
    bs, K, L, k = lp.shape
    tree = np.empty((bs, 3, budget + 1), np.int64)
    counts = np.empty(bs, np.int64)
    lib().oracle_build_trees(_p(lp, _f32p), _p(ids, _i32p), _p(pr, _f32p), bs, K, L, k, budget,
                             _p(tree, _i64p), _p(counts, _i64p))
    return tree, counts


def visibility(parents) -> np.ndarray:
    par = np.ascontiguousarray(parents, dtype=np.int64)
    m = par.shape[0]
    vis = np.empty((m, m), np.uint8)
    lib().oracle_visibility(_p(par, _i64p), m, _p(vis, _u8p))
    return vis.astype(bool)


def follow(tokens_with_root, parents, posterior, max_steps: int = -1):
    """tokens_with_root [m] (index 0 unused), parents [m], posterior [m] -> (accepted list, bonus)."""
    tok = np.ascontiguousarray(tokens_with_root, dtype=np.int64)
    par = np.ascontiguousarray(parents, dtype=np.int64)
    post = np.ascontiguousarray(posterior, dtype=np.int64)
    m = par.shape[0]
    acc = np.empty(m + 1, np.int64)
    bonus = np.zeros(1, np.int64)
    n = lib().oracle_follow(_p(tok, _i64p), _p(par, _i64p), m, _p(post, _i64p), max_steps, _p(acc, _i64p),
                            _p(bonus, _i64p))
    return acc[:n].tolist(), int(bonus[0])


def sample_rows(rows_bf16_u16: np.ndarray, inv_temp: float, u: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(rows_bf16_u16, dtype=np.uint16)
    R, V = x.shape
    uu = np.ascontiguousarray(u, dtype=np.float64)
    out = np.empty(R, np.int64)
    lib().oracle_sample_rows(_p(x, _u16p), R, V, ctypes.c_float(inv_temp), _p(uu, _f64p), _p(out, _i64p))
    return out


def argmax_rows(rows_bf16_u16: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(rows_bf16_u16, dtype=np.uint16)
    R, V = x.shape
    out = np.empty(R, np.int64)
    lib().oracle_argmax_rows(_p(x, _u16p), R, V, _p(out, _i64p))
    return out


def exp32(y: float) -> float:
    return float(lib().oracle_exp32(ctypes.c_float(y)))


# ------------------------------------------------------------------------------------------ float paths

def bf16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    return (np.asarray(u16, dtype=np.uint32) << 16).view(np.float32)


def topk_logz(x: np.ndarray, k: int):
    """x [R, V] float32 -> (top_logp [R, k] float32, ids [R, k] int64, logz [R] float32).

    logz is the float64 logsumexp rounded once to float32; top_logp = float32(top) - logz in float32, as
    hf/ddtree.py:243 subtracts.  Order: value descending, equal values by lower index first."""
    x = np.asarray(x, dtype=np.float32)
    R, V = x.shape
    xd = x.astype(np.float64)
    m = xd.max(axis=1, keepdims=True)
    logz = (m[:, 0] + np.log(np.exp(xd - m).sum(axis=1))).astype(np.float32)
    ids = np.empty((R, k), np.int64)
    top = np.empty((R, k), np.float32)
    idx = np.arange(V)
    for r in range(R):
        order = np.lexsort((idx, -x[r].astype(np.float64)))[:k]
        ids[r] = order
        top[r] = x[r, order]
    return (top - logz[:, None]).astype(np.float32), ids, logz


def tree_attention(q, k_prefix, v_prefix, k_tree, v_tree, parents, scale):
    """q [n, H, D], prefix K/V [P, Hkv, D], tree K/V [n, Hkv, D] (float arrays), parents [n] (parents[0] = -1).
    Row i sees every prefix key and the tree keys of its ancestors and itself.  Returns [n, H, D] float32."""
    q = np.asarray(q, np.float32)
    n, H, D = q.shape
    Hkv = k_tree.shape[1]
    G = H // Hkv
    vis = visibility(parents)
    kk = np.concatenate([np.asarray(k_prefix, np.float32), np.asarray(k_tree, np.float32)], 0)
    vv = np.concatenate([np.asarray(v_prefix, np.float32), np.asarray(v_tree, np.float32)], 0)
    P = k_prefix.shape[0]
    mask = np.zeros((n, P + n), bool)
    mask[:, :P] = True
    mask[:, P:] = vis
    out = np.empty((n, H, D), np.float32)
    for h in range(H):
        kv = h // G
        s = (q[:, h, :].astype(np.float64) @ kk[:, kv, :].astype(np.float64).T) * scale
        s = np.where(mask, s, -np.inf)
        s = s - s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[:, h, :] = (p @ vv[:, kv, :].astype(np.float64)).astype(np.float32)
    return out


def mode_attention(q, k, v, num_modes, block_size, scale):
    """hf/mode_attention.py reference: q [H, K*bs, D], k/v [Hkv, ctx + K*bs, D] -> [K*bs, H, D] float32."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    H, T, D = q.shape
    Hkv, total, _ = k.shape
    G = H // Hkv
    ctx = total - num_modes * block_size
    qb = np.arange(T) // block_size
    mask = np.ones((T, total), bool)
    mask[:, ctx:] = qb[:, None] == qb[None, :]
    out = np.empty((T, H, D), np.float32)
    for h in range(H):
        s = (q[h] @ k[h // G].T) * scale
        s = np.where(mask, s, -np.inf)
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[:, h, :] = (p @ v[h // G]).astype(np.float32)
    return out


def tree_gdn(q, k, v, g_cum, beta, s0, parents, emit_states=False):
    """Chunk form of the tree gated delta rule in float64.

    q, k [n, HK, Dk] (q already l2-normalised and scaled, k l2-normalised), v [n, H, Dv], g_cum/beta [n, H]
    (g_cum = log decay summed along the root path), s0 [H, Dk, Dv] (fla layout, o = S^T q), parents [n]
    (-1 = the committed state).  Returns u, o [n, H, Dv] and, if asked, per-node states [n, H, Dk, Dv]."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    G = np.asarray(g_cum, np.float64)
    beta = np.asarray(beta, np.float64)
    s0 = np.asarray(s0, np.float64)
    n, HK, Dk = k.shape
    H, Dv = v.shape[1], v.shape[2]
    anc = np.zeros((n, n), bool)
    for i in range(n):
        p = int(parents[i])
        if p >= 0:
            anc[i] = anc[p]
        anc[i, i] = True
    strict = anc & ~np.eye(n, dtype=bool)
    u = np.empty((n, H, Dv))
    o = np.empty((n, H, Dv))
    states = np.empty((n, H, Dk, Dv)) if emit_states else None
    for h in range(H):
        hk = h // (H // HK)
        kh, qh, Gh = k[:, hk], q[:, hk], G[:, h]
        gamma = np.where(anc, np.exp(np.where(anc, Gh[:, None] - Gh[None, :], 0.0)), 0.0)
        lower = beta[:, h, None] * gamma * (kh @ kh.T) * strict
        rhs = beta[:, h, None] * (v[:, h] - np.exp(Gh)[:, None] * (kh @ s0[h]))
        A = np.eye(n) + lower
        uh = np.zeros((n, Dv))
        for i in range(n):  # forward substitution (unit lower triangular)
            uh[i] = rhs[i] - A[i, :i] @ uh[:i]
        u[:, h] = uh
        o[:, h] = np.exp(Gh)[:, None] * (qh @ s0[h]) + (gamma * (qh @ kh.T) * anc) @ uh
        if emit_states:
            for i in range(n):
                w = gamma[i] * anc[i]
                states[i, h] = np.exp(Gh[i]) * s0[h] + (kh * w[:, None]).T @ uh
    return u, o, states


def commit_state(s0, u, k, G, path):
    """The state at the deepest accepted node a = path[-1] (inference/hf/qwen35_tree.py:134-137) in float64:
    S_a = e^{G_a} S0 + sum_{j on path} e^{G_a - G_j} k_j u_j^T, value head h reading key head h // (H / HK).
    s0 [H, Dk, Dv], u [n, H, Dv], k [n, HK, Dk], G [n, H] -> [H, Dk, Dv]."""
    s0 = np.asarray(s0, np.float64)
    u = np.asarray(u, np.float64)
    k = np.asarray(k, np.float64)
    G = np.asarray(G, np.float64)
    H, HK = u.shape[1], k.shape[1]
    a = path[-1]
    out = np.exp(G[a])[:, None, None] * s0
    for j in path:
        w = np.exp(G[a] - G[j])  # [H]
        kk = k[j][np.arange(H) // (H // HK)]  # [H, Dk]
        out += w[:, None, None] * kk[:, :, None] * u[j][:, None, :]
    return out


def gdn_recurrence(q, k, v, g, beta, s0, parents):
    """Node-by-node gated delta rule (tests/test_gdn_tree_math.py:38-44, fla layout S [Dk, Dv]):
    S_i = exp(g_i) S_p (I - beta_i k_i k_i^T)... written as S_i = e^{g_i}(S_p - beta_i k_i (k_i^T S_p)) +
    beta_i k_i v_i^T, o_i = S_i^T q_i.  float64; returns o [n, H, Dv] and states [n, H, Dk, Dv]."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    g = np.asarray(g, np.float64)
    beta = np.asarray(beta, np.float64)
    s0 = np.asarray(s0, np.float64)
    n, HK, Dk = k.shape
    H, Dv = v.shape[1], v.shape[2]
    states = np.empty((n, H, Dk, Dv))
    o = np.empty((n, H, Dv))
    for i in range(n):
        p = int(parents[i])
        for h in range(H):
            hk = h // (H // HK)
            sp = s0[h] if p < 0 else states[p, h]
            ki = k[i, hk]
            s = np.exp(g[i, h]) * (sp - beta[i, h] * np.outer(ki, ki @ sp)) + beta[i, h] * np.outer(ki, v[i, h])
            states[i, h] = s
            o[i, h] = s.T @ q[i, hk]
    return o, states


def tree_gates(a, b, a_log, dt_bias, parents):
    """inference/hf/qwen35_tree.py:77-79 in float64: beta = sigmoid(b), g = -exp(A_log) softplus(a + dt_bias)
    (torch's softplus: x above 20), G = anc @ g with anc the ancestor-or-self matrix of the parents."""
    a = np.asarray(a, np.float64)
    x = a + np.asarray(dt_bias, np.float64)[None]
    sp = np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20))))
    g = -np.exp(np.asarray(a_log, np.float64))[None] * sp
    beta = 1.0 / (1.0 + np.exp(-np.asarray(b, np.float64)))
    G = visibility(list(parents)).astype(np.float64) @ g
    return beta, G


def bf16_round(x) -> np.ndarray:
    """float32 -> nearest bfloat16 (ties to even), returned as float32."""
    b = np.ascontiguousarray(np.asarray(x, np.float32)).view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def tree_prep(x, conv_state, conv_index, conv_w, num_k_heads, num_v_heads, head_dim, scale):
    """hf/tree_gdn_kernel.py:27-56 in float32.  x [n, CD], conv_state [CD, KC], conv_index [n, KC] (indices into
    [conv_state columns ; nodes]), conv_w [CD, KC], all bf16-valued.  Returns q, k [n, HK, D], v [n, H, D] as
    bf16-valued float32 arrays."""
    x = np.asarray(x, np.float32)
    cs = np.asarray(conv_state, np.float32)
    w = np.asarray(conv_w, np.float32)
    idx = np.asarray(conv_index, np.int64)
    n, cd = x.shape
    kc = w.shape[1]
    X = np.concatenate([cs.T, x], axis=0)  # [KC + n, CD]: cached inputs then the nodes
    acc = np.zeros((n, cd), np.float32)
    for t in range(kc):  # sequential fp32 accumulation over the window, oldest first
        acc = (acc + X[idx[:, t]] * w[None, :, t]).astype(np.float32)
    y = bf16_round(acc / (np.float32(1) + np.exp(-acc, dtype=np.float32)))
    HK, H, D = num_k_heads, num_v_heads, head_dim
    q = y[:, : HK * D].reshape(n, HK, D)
    k = y[:, HK * D: 2 * HK * D].reshape(n, HK, D)
    v = y[:, 2 * HK * D:].reshape(n, H, D)

    def l2n(a):
        return a / np.sqrt((a * a).sum(-1, keepdims=True, dtype=np.float32) + np.float32(1e-6), dtype=np.float32)

    return bf16_round(l2n(q) * np.float32(scale)), bf16_round(l2n(k)), bf16_round(v)


def compile_tree(root, start, tokens, depths, vis, past, prev_start, prev_len, ids_buf, pos_buf, mask_buf,
                 vis_buf, min_value):
    """The HF verify inputs of one round (inference/hf/ddtree.py:317-357) written into numpy buffers in place:
    the previous round's block of the additive mask reset to 0, ids = [root, tokens], positions = start +
    [0, depths], the visibility copied, and the new block set to min_value except where visible (0).  ids_buf and
    pos_buf [max_nodes], mask_buf [max_nodes, max_cols], vis_buf [max_nodes, max_nodes]."""
    n = 1 + len(tokens)
    if prev_len > 0:
        mask_buf[:prev_len, prev_start:prev_start + prev_len] = 0
    ids_buf[0] = root
    ids_buf[1:n] = tokens
    pos_buf[0] = start
    pos_buf[1:n] = np.asarray(depths) + start
    vis = np.asarray(vis, bool)
    vis_buf[:n, :n] = vis
    mask_buf[:n, past:past + n] = np.where(vis, 0, min_value)
    return n


def compact_tail(cache, past_length, keep):
    """The commit step's cache compaction (inference/hf/ddtree.py:385-403, the index_select path): rows
    past + keep[i] of dim -2 move to past + i; nothing when the appended window is empty, keep is empty or keep has
    the window's length.  Returns a new array."""
    cache = np.asarray(cache)
    keep = [int(i) for i in keep]
    cur = cache.shape[-2] - past_length
    out = cache.copy()
    if cur <= 0 or len(keep) == 0 or len(keep) == cur:
        return out
    tail = cache[..., past_length:, :]
    out[..., past_length:past_length + len(keep), :] = tail[..., keep, :]
    return out


def commit_kv_moves(pool, move_src, move_tgt):
    """Token-major pool moves (sglang-v0.5.22-mfd.patch:1769-1841): pool [buffers, slots, ...]; for request b the
    moves (src, tgt) of row b with src != tgt, every source read before any store.  Requests are taken in order
    (they own disjoint slots in the callers).  Returns a new array."""
    out = np.array(pool, copy=True)
    for b in range(move_src.shape[0]):
        moves = [(int(s), int(t)) for s, t in zip(move_src[b], move_tgt[b]) if int(s) != int(t)]
        vals = [out[:, s].copy() for s, _ in moves]
        for (_, t), v in zip(moves, vals):
            out[:, t] = v
    return out


def paged_mode_attention(q, k_new, v_new, k_cache, v_cache, req_to_token, req_pool_indices, ctx_lens, num_modes,
                         block_size, scale):
    """SGLang paged_mode_block_attention_reference (sglang-v0.5.22-mfd.patch:965-989): per request, the context
    rows k_cache[req_to_token[req_pool_indices[b], :ctx_lens[b]]] followed by the request's K*block_size new keys,
    then the mode-block attention of mode_attention (block-diagonal over the new keys).
    q [T, H, D], k_new/v_new [T, Hkv, D], caches [slots, Hkv, D] -> [T, H, D] float32."""
    q = np.asarray(q, np.float32)
    T, H, D = q.shape
    KL = num_modes * block_size
    out = np.empty((T, H, D), np.float32)
    for b in range(T // KL):
        ctx = int(ctx_lens[b])
        slots = np.asarray(req_to_token[int(req_pool_indices[b]), :ctx], np.int64)
        rows = slice(b * KL, (b + 1) * KL)
        kk = np.concatenate([np.asarray(k_cache)[slots], np.asarray(k_new)[rows]], 0)  # [ctx + KL, Hkv, D]
        vv = np.concatenate([np.asarray(v_cache)[slots], np.asarray(v_new)[rows]], 0)
        out[rows] = mode_attention(q[rows].transpose(1, 0, 2), kk.transpose(1, 0, 2), vv.transpose(1, 0, 2),
                                   num_modes, block_size, scale)
    return out
