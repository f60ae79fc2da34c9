// tree_attention.cu -- C ABI of the tree-masked GQA verify attention (the kernel is tree_attention_tc.cu).
//
// softmax(q k^T * scale + mask) v for the B+1 tree rows of every request, where row i sees every
// prefix key and, among the tree keys, exactly its ancestors and itself (the additive mask of
// inference/hf/ddtree.py:352-356, the flashinfer custom mask of sglang-v0.5.22-mfd.patch:1625-1703).
// The mask comes from the builder's ancestor bitsets, never a dense [n, prefix + n] tensor.
//
// Layout: q, out [bs, n, H, 128] (any strides in elements that are multiples of 8, head dim contiguous); k, v
// [bs, Hkv, max_keys, 128] (the prefix keys [0, prefix_b) followed by the n tree keys [prefix_b, prefix_b + n));
// anc [bs, n, words].  Workspace: [status word | pad to 256 B][o partials][lse partials].  Tickets (one per
// (request, KV head, M-tile)) live in a separate ticket-only buffer: kept inside the workspace, they would land on
// an earlier call's partials whenever the workspace is reused with other sizes.
#include "common.cuh"
#include "tree_attention_tc.cuh"

using namespace mfd;

namespace {
struct WsLayout {
    size_t o_part, lse, total;
    int64_t units;
};
WsLayout ws_layout(int64_t bs, int64_t n, int64_t num_heads, int64_t num_kv_heads, int64_t splits) {
    const int64_t G = num_heads / num_kv_heads;
    const int64_t mtiles = (n * G + tca::kM - 1) / tca::kM;
    const size_t units = (size_t)bs * num_kv_heads * mtiles;
    const size_t rows = (size_t)splits * units * tca::kM;
    WsLayout w;
    w.units = (int64_t)units;
    w.o_part = 256;
    w.lse = w.o_part + rows * 128 * sizeof(float);
    w.total = w.lse + rows * sizeof(float) + 256;  // + alignment slack of the base
    return w;
}
}  // namespace

extern "C" int64_t mfd_tree_attention_tickets(int64_t bs, int64_t n, int64_t num_heads, int64_t num_kv_heads) {
    if (bs <= 0 || n <= 0 || num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads) return 1;
    return 3 * ws_layout(bs, n, num_heads, num_kv_heads, 1).units;  // [arrived, claimed, finished] per unit
}

extern "C" size_t mfd_tree_attention_workspace(int64_t bs, int64_t n, int64_t num_heads, int64_t num_kv_heads,
                                               int64_t splits) {
    if (bs <= 0 || n <= 0 || num_heads <= 0 || num_kv_heads <= 0 || splits <= 0 || num_heads % num_kv_heads)
        return 0;
    return ws_layout(bs, n, num_heads, num_kv_heads, splits).total;
}

extern "C" int mfd_tree_attention(const void* q, int64_t sq_b, int64_t sq_n, int64_t sq_h, const void* k,
                                  int64_t sk_b, int64_t sk_h, int64_t sk_s, const void* v, int64_t sv_b,
                                  int64_t sv_h, int64_t sv_s, int64_t max_keys, const int32_t* prefix_lens,
                                  int64_t prefix_len, const uint64_t* anc_bits, int64_t anc_words, int64_t bs,
                                  int64_t n, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim, float scale,
                                  int64_t splits, void* out, int64_t so_b, int64_t so_n, int64_t so_h,
                                  void* workspace, size_t workspace_bytes, unsigned int* tickets,
                                  int64_t tickets_len, void* stream) {
    if (bs < 0 || n < 1 || num_heads < 1 || num_kv_heads < 1 || num_heads % num_kv_heads || splits < 1 ||
        anc_words < (n + 63) / 64 || max_keys < 1) {
        set_error("mfd_tree_attention: invalid sizes bs=%lld n=%lld H=%lld Hkv=%lld splits=%lld words=%lld keys=%lld",
                  (long long)bs, (long long)n, (long long)num_heads, (long long)num_kv_heads, (long long)splits,
                  (long long)anc_words, (long long)max_keys);
        return MFD_ERR_INVALID;
    }
    const int64_t G = num_heads / num_kv_heads;
    if (head_dim != 128 || tca::kM % G) {
        set_error("mfd_tree_attention: head_dim must be 128 and H / Hkv divide 128 (got %lld, %lld)",
                  (long long)head_dim, (long long)G);
        return MFD_ERR_UNSUPPORTED;
    }
    if (bs == 0) return MFD_OK;
    if (!q || !k || !v || !anc_bits || !out) {
        set_error("mfd_tree_attention: null pointer");
        return MFD_ERR_INVALID;
    }
    if (!prefix_lens && prefix_len + n > max_keys) {
        set_error("mfd_tree_attention: prefix_len + n = %lld exceeds the %lld stored keys", (long long)(prefix_len + n),
                  (long long)max_keys);
        return MFD_ERR_INVALID;
    }
    const WsLayout wl = ws_layout(bs, n, num_heads, num_kv_heads, splits);
    if (!workspace || workspace_bytes < wl.total) {
        set_error("mfd_tree_attention: workspace of %zu bytes needed", wl.total);
        return MFD_ERR_INVALID;
    }
    if (splits > 1 && (!tickets || tickets_len < 3 * wl.units)) {
        set_error("mfd_tree_attention: a zeroed ticket buffer of %lld words is needed", (long long)(3 * wl.units));
        return MFD_ERR_INVALID;
    }
    // TMA: 16-byte aligned bases and strides
    const int64_t strides[] = {sq_b, sq_n, sq_h, sk_b, sk_h, sk_s, sv_b, sv_h, sv_s};
    for (int64_t s : strides)
        if (s % 8 || s <= 0) {
            set_error("mfd_tree_attention: strides must be positive multiples of 8 elements");
            return MFD_ERR_INVALID;
        }
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15u || so_n % 8 || so_h % 8) {
        set_error("mfd_tree_attention: q, k, v, out must be 16-byte aligned with 16-byte aligned rows");
        return MFD_ERR_INVALID;
    }
    char* ws = (char*)(((uintptr_t)workspace + 255) & ~(uintptr_t)255);
    tca::Shape sh{q, sq_b, sq_n, sq_h, k, sk_b, sk_h, sk_s, v, sv_b, sv_h, sv_s, max_keys};
    tca::Params p = {};
    p.out = (__nv_bfloat16*)out;
    p.so_b = so_b;
    p.so_n = so_n;
    p.so_h = so_h;
    p.prefix = prefix_lens;
    p.prefix_const = (int)prefix_len;
    p.anc = anc_bits;
    p.words = (int)anc_words;
    p.n = (int)n;
    p.H = (int)num_heads;
    p.Hkv = (int)num_kv_heads;
    p.G = (int)G;
    p.mtiles = (int)((n * G + tca::kM - 1) / tca::kM);
    p.scale_log2 = scale * 1.4426950408889634f;
    p.splits = (int)splits;
    p.o_part = (float*)(ws + wl.o_part);
    p.lse_part = (float*)(ws + wl.lse);
    p.tickets = tickets;
    p.status = (int*)ws;  // sticky: set to 1 if a bounded wait in the kernel ever gave up
    p.bs = (int)bs;
    return tca::launch(sh, p, (cudaStream_t)stream);
}

extern "C" int mfd_paged_mode_attention(const void* q, int64_t sq_t, int64_t sq_h, const void* k_new, int64_t skn_t,
                                        int64_t skn_h, const void* v_new, int64_t svn_t, int64_t svn_h,
                                        const void* k_cache, int64_t skc_t, int64_t skc_h, const void* v_cache,
                                        int64_t svc_t, int64_t svc_h, int64_t num_slots, const int32_t* req_to_token,
                                        int64_t r2t_rows, int64_t r2t_cols, int64_t r2t_stride,
                                        const int64_t* req_pool_indices, const int64_t* ctx_lens,
                                        const uint64_t* block_bits, int64_t bits_words, int64_t bs, int64_t num_modes,
                                        int64_t block_size, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                                        float scale, int64_t splits, void* out, int64_t so_t, int64_t so_h,
                                        void* workspace, size_t workspace_bytes, unsigned int* tickets,
                                        int64_t tickets_len, void* stream) {
    const int64_t n = num_modes * block_size;
    if (bs < 0 || num_modes < 1 || block_size < 1 || num_heads < 1 || num_kv_heads < 1 ||
        num_heads % num_kv_heads || splits < 1 || bits_words < (n + 63) / 64 || num_slots < 1 ||
        num_slots > 0x7fffffff || r2t_rows < 1 || r2t_cols < 0 || r2t_stride < r2t_cols) {
        set_error("mfd_paged_mode_attention: invalid sizes bs=%lld K=%lld block=%lld H=%lld Hkv=%lld splits=%lld "
                  "words=%lld slots=%lld req_to_token=[%lld, %lld] stride %lld",
                  (long long)bs, (long long)num_modes, (long long)block_size, (long long)num_heads,
                  (long long)num_kv_heads, (long long)splits, (long long)bits_words, (long long)num_slots,
                  (long long)r2t_rows, (long long)r2t_cols, (long long)r2t_stride);
        return MFD_ERR_INVALID;
    }
    const int64_t G = num_heads / num_kv_heads;
    if (head_dim != 128 || tca::kM % G) {
        set_error("mfd_paged_mode_attention: head_dim must be 128 and H / Hkv divide 128 (got %lld, %lld)",
                  (long long)head_dim, (long long)G);
        return MFD_ERR_UNSUPPORTED;
    }
    if (bs == 0) return MFD_OK;
    if (!q || !k_new || !v_new || !k_cache || !v_cache || !req_to_token || !req_pool_indices || !ctx_lens ||
        !block_bits || !out) {
        set_error("mfd_paged_mode_attention: null pointer");
        return MFD_ERR_INVALID;
    }
    // the gathered rows hold a token's KV heads contiguously (head stride 128) at 16-byte aligned offsets
    if (skn_h != 128 || svn_h != 128 || skc_h != 128 || svc_h != 128 || sq_h % 8 || sq_t % 8 || skn_t % 8 ||
        svn_t % 8 || skc_t % 8 || svc_t % 8 || so_t % 8 || so_h % 8 || sq_h <= 0 || sq_t <= 0 ||
        skn_t < num_kv_heads * 128 || svn_t < num_kv_heads * 128 || skc_t < num_kv_heads * 128 ||
        svc_t < num_kv_heads * 128) {
        set_error("mfd_paged_mode_attention: k/v rows must hold the KV heads contiguously (head stride 128) and every "
                  "stride must be a positive multiple of 8 elements");
        return MFD_ERR_INVALID;
    }
    if (skc_t != svc_t || skn_t != svn_t) {
        set_error("mfd_paged_mode_attention: K and V must share their token strides (cache %lld / %lld, new %lld / "
                  "%lld)", (long long)skc_t, (long long)svc_t, (long long)skn_t, (long long)svn_t);
        return MFD_ERR_INVALID;
    }
    if (((uintptr_t)q | (uintptr_t)k_new | (uintptr_t)v_new | (uintptr_t)k_cache | (uintptr_t)v_cache |
         (uintptr_t)out) & 15u) {
        set_error("mfd_paged_mode_attention: q, k, v, caches and out must be 16-byte aligned");
        return MFD_ERR_INVALID;
    }
    const WsLayout wl = ws_layout(bs, n, num_heads, num_kv_heads, splits);
    if (!workspace || workspace_bytes < wl.total) {
        set_error("mfd_paged_mode_attention: workspace of %zu bytes needed", wl.total);
        return MFD_ERR_INVALID;
    }
    if (splits > 1 && (!tickets || tickets_len < 3 * wl.units)) {
        set_error("mfd_paged_mode_attention: a zeroed ticket buffer of %lld words is needed",
                  (long long)(3 * wl.units));
        return MFD_ERR_INVALID;
    }
    char* ws = (char*)(((uintptr_t)workspace + 255) & ~(uintptr_t)255);
    // q / out as [bs, n, H, 128]: request b's n rows are tokens b n .. b n + n - 1
    tca::Shape sh{q, n * sq_t, sq_t, sq_h, nullptr, 0, 0, 0, nullptr, 0, 0, 0, 0};
    tca::Params p = {};
    p.out = (__nv_bfloat16*)out;
    p.so_b = n * so_t;
    p.so_n = so_t;
    p.so_h = so_h;
    p.anc = block_bits;
    p.words = (int)bits_words;
    p.n = (int)n;
    p.H = (int)num_heads;
    p.Hkv = (int)num_kv_heads;
    p.G = (int)G;
    p.mtiles = (int)((n * G + tca::kM - 1) / tca::kM);
    p.scale_log2 = scale * 1.4426950408889634f;
    p.splits = (int)splits;
    p.o_part = (float*)(ws + wl.o_part);
    p.lse_part = (float*)(ws + wl.lse);
    p.tickets = tickets;
    p.status = (int*)ws;
    p.bs = (int)bs;
    p.paged = 1;
    p.r2t = req_to_token;
    p.r2t_stride = r2t_stride;
    p.r2t_rows = r2t_rows;
    p.r2t_cols = r2t_cols;
    p.rpi = req_pool_indices;
    p.ctx = ctx_lens;
    p.kc = (const __nv_bfloat16*)k_cache;
    p.vc = (const __nv_bfloat16*)v_cache;
    p.kn = (const __nv_bfloat16*)k_new;
    p.vn = (const __nv_bfloat16*)v_new;
    p.skc_t = skc_t;
    p.skn_t = skn_t;
    p.slots = num_slots;
    return tca::launch(sh, p, (cudaStream_t)stream);
}
