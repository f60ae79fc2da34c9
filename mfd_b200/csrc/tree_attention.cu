// tree_attention.cu -- C ABI of the tree-masked GQA verify attention (the kernel is tree_attention_tc.cu).
//
// softmax(q k^T * scale + mask) v for the B+1 tree rows of every request, where row i sees every
// prefix key and, among the tree keys, exactly its ancestors and itself (the additive mask of
// inference/hf/ddtree.py:352-356, the flashinfer custom mask of sglang-v0.5.22-mfd.patch:1625-1703).
// The mask comes from the builder's ancestor bitsets, never a dense [n, prefix + n] tensor.
//
// Layout: q, out [bs, n, H, 128] (any strides in elements that are multiples of 8, head dim contiguous); k, v
// [bs, Hkv, max_keys, 128] (the prefix keys [0, prefix_b) followed by the n tree keys [prefix_b, prefix_b + n));
// anc [bs, n, words].  Workspace: [status word | pad to 256 B][tickets][o partials][lse partials].
#include "common.cuh"

namespace mfd {
namespace tca {
constexpr int kM = 128;
struct Params {
    __nv_bfloat16* out;
    int64_t so_b, so_n, so_h;
    const int32_t* prefix;
    int prefix_const;
    const uint64_t* anc;
    int words;
    int n, H, Hkv, G;
    int mtiles;
    float scale_log2;
    int splits;
    float* o_part;
    float* lse_part;
    unsigned int* tickets;
    int* status;
    int bs;
};
struct Shape {
    const void* q;
    int64_t sq_b, sq_n, sq_h;
    const void* k;
    int64_t sk_b, sk_h, sk_s;
    const void* v;
    int64_t sv_b, sv_h, sv_s;
    int64_t max_keys;
};
int launch(const Shape& sh, const Params& p, cudaStream_t stream);
}  // namespace tca
}  // namespace mfd

using namespace mfd;

namespace {
struct WsLayout {
    size_t tickets, o_part, lse, total;
};
WsLayout ws_layout(int64_t bs, int64_t n, int64_t num_heads, int64_t num_kv_heads, int64_t splits) {
    const int64_t G = num_heads / num_kv_heads;
    const int64_t mtiles = (n * G + tca::kM - 1) / tca::kM;
    const size_t units = (size_t)bs * num_kv_heads * mtiles;
    const size_t rows = (size_t)splits * units * tca::kM;
    WsLayout w;
    w.tickets = 256;
    w.o_part = w.tickets + (units * 4 + 255) / 256 * 256;
    w.lse = w.o_part + rows * 128 * sizeof(float);
    w.total = w.lse + rows * sizeof(float) + 256;  // + alignment slack of the base
    return w;
}
}  // namespace

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
                                  void* workspace, size_t workspace_bytes, void* stream) {
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
    tca::Params p;
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
    p.tickets = (unsigned int*)(ws + wl.tickets);
    p.status = (int*)ws;  // sticky: set to 1 if a bounded wait in the kernel ever gave up
    p.bs = (int)bs;
    return tca::launch(sh, p, (cudaStream_t)stream);
}
