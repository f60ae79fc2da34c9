// accept.cu -- the acceptance step: the target's token at every tree node (greedy argmax, or one
// reproducible sample per node) and the walk along the verified path.
//
// Greedy: post[i] = first index of the row maximum (torch.argmax; inference/hf/model/utils.py:28-30,
//   SGLang _target_tokens patch:2990-2991).
// Stochastic (temperature T): the reference draws torch.multinomial(softmax(x/T)) (hf/model/utils.py:31-35),
//   which is not reproducible.  This build's rule, identical on CPU and GPU bit for bit:
//     m = max x;  e_i = exp32((x_i - m) * (1/T))  (Cody-Waite reduction + degree-7 Taylor polynomial, fmaf);
//     E_i = trunc(e_i * 2^40) as uint64;  Z = sum E_i (integer: exact in any order);
//     token = min { j : sum_{i<=j} E_i > floor(u * Z) }   for the node's uniform u in [0, 1).
// Walk: from node 0 follow the child whose token equals post[current] (inference/hf/ddtree.py:368-382,
//   tree_build_ext.py:70-83; SGLang _ddtree_follow_kernel patch:1706-1766 and its outputs: accepted length,
//   commit length, bonus, emitted tokens, KV move lists, hidden-row indices, new sequence lengths).
//
// One CTA per logits row; the last CTA to finish a request's rows (an atomic ticket per request, no
// waiting) walks that request's tree.  Tickets reset themselves.
#include "common.cuh"

namespace mfd {
namespace accept {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;

// exp(y), y <= 0, float32: Cody & Waite range reduction (ln 2 = 0.693359375 - 2.12194440e-4) and the
// degree-7 Taylor polynomial of exp evaluated by Horner's rule; every operation individually rounded.
__device__ __forceinline__ float exp32_rule(float y) {
    if (!(y > -87.0f)) return 0.0f;
    const float n = rintf(__fmul_rn(y, 1.44269504088896341f));
    float r = __fmaf_rn(n, -0.693359375f, y);
    r = __fmaf_rn(n, 2.12194440e-4f, r);
    float q = 1.0f / 5040.0f;
    q = __fmaf_rn(q, r, 1.0f / 720.0f);
    q = __fmaf_rn(q, r, 1.0f / 120.0f);
    q = __fmaf_rn(q, r, 1.0f / 24.0f);
    q = __fmaf_rn(q, r, 1.0f / 6.0f);
    q = __fmaf_rn(q, r, 0.5f);
    q = __fmaf_rn(q, r, 1.0f);
    q = __fmaf_rn(q, r, 1.0f);
    const int ni = (int)n;
    return __uint_as_float(__float_as_uint(q) + ((uint32_t)ni << 23));
}
__device__ __forceinline__ uint64_t fixed40(float x, float m, float inv_t) {
    const float e = exp32_rule(__fmul_rn(__fsub_rn(x, m), inv_t));
    return (uint64_t)__fmul_rn(e, 1099511627776.0f);  // 2^40; float -> uint64 truncates toward zero
}

struct Params {
    const uint16_t* logits;  // bf16 rows, row r = b * width + i
    int64_t row_stride;      // elements
    int64_t vocab;
    int64_t bs, width;
    float temperature;       // < 1e-5: greedy
    const double* uniforms;  // [bs * width]
    int64_t* posterior;      // [bs * width]
    // walk (optional)
    int walk;
    const int64_t* tokens;   // [bs, width] stride tokens_stride
    int64_t tokens_stride;
    const int64_t* parents;  // [bs, width] stride parents_stride
    int64_t parents_stride;
    int64_t max_steps;       // < 0: unbounded
    const int64_t* window;   // [bs, width] or null
    const int64_t* prefix_lens;  // [bs] or null
    int64_t out_len;         // columns of the per-request outputs
    int32_t* accept_len;
    int32_t* commit_lens;
    int64_t* bonus;
    int64_t* out_tokens;
    int64_t* accepted;
    int64_t* new_seq_lens;
    int64_t* move_src;
    int64_t* move_tgt;
    int64_t* hidden_index;
    unsigned int* tickets;   // [bs]
};

__device__ __forceinline__ uint64_t block_reduce_max_u64(uint64_t v, uint64_t* red) {
    v = warp_max_u64(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    uint64_t r = (lane < kWarps) ? red[lane] : 0ull;
    return warp_max_u64(r);
}
__device__ __forceinline__ uint64_t block_reduce_sum_u64(uint64_t v, uint64_t* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += shfl_xor_u64(v, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    uint64_t r = (lane < kWarps) ? red[lane] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) r += shfl_xor_u64(r, o);
    return r;
}

// walk request b along its verified path (one warp); SGLang follow-kernel outputs
__device__ void walk_request(const Params& p, int64_t b) {
    const int lane = threadIdx.x & 31;
    const int64_t W = p.width;
    const int64_t* par = p.parents + b * p.parents_stride;
    const int64_t* tok = p.tokens + b * p.tokens_stride;
    const int64_t* post = p.posterior + b * W;
    const int64_t L = p.out_len;
    const int64_t limit = p.max_steps < 0 ? W : p.max_steps;
    int64_t cur = 0, n = 0;
    for (int64_t step = 0; step < limit; ++step) {
        const int64_t t = __ldcg(post + cur);
        int64_t child = -1;
        for (int64_t base = 1; base < W && child < 0; base += 32) {
            const int64_t j = base + lane;
            const bool hit = j < W && __ldcg(par + j) == cur && __ldcg(tok + j) == t;
            const uint32_t bal = __ballot_sync(MFD_FULL_MASK, hit);
            if (bal) child = base + (__ffs(bal) - 1);
        }
        if (child < 0) break;
        ++n;
        if (lane == 0 && n < L) {
            if (p.accepted) p.accepted[b * L + n] = child;
            if (p.out_tokens) p.out_tokens[b * L + n - 1] = t;
            if (p.hidden_index) p.hidden_index[b * L + n] = b * W + child;
            if (p.move_src && p.window) p.move_src[b * L + n] = p.window[b * W + child];
            if (p.move_tgt && p.window) p.move_tgt[b * L + n] = p.window[b * W + n];
        }
        cur = child;
    }
    const int64_t bon = __ldcg(post + cur);
    if (lane == 0) {
        if (p.accepted) p.accepted[b * L + 0] = 0;
        if (p.hidden_index) p.hidden_index[b * L + 0] = b * W;
        if (p.move_src && p.window) p.move_src[b * L + 0] = p.window[b * W + 0];
        if (p.move_tgt && p.window) p.move_tgt[b * L + 0] = p.window[b * W + 0];
        if (p.out_tokens && n < L) p.out_tokens[b * L + n] = bon;
        if (p.accept_len) p.accept_len[b] = (int32_t)n;
        if (p.commit_lens) p.commit_lens[b] = (int32_t)(n + 1);
        if (p.bonus) p.bonus[b] = bon;
        if (p.new_seq_lens) p.new_seq_lens[b] = (p.prefix_lens ? p.prefix_lens[b] : 0) + n + 1;
    }
    // tails past the path: zeros (accepted -1, hidden index b*W as the reference kernel leaves it)
    for (int64_t j = n + 1 + lane; j < L; j += 32) {
        if (p.accepted) p.accepted[b * L + j] = -1;
        if (p.out_tokens) p.out_tokens[b * L + j] = 0;
        if (p.hidden_index) p.hidden_index[b * L + j] = b * W;
        if (p.move_src) p.move_src[b * L + j] = 0;
        if (p.move_tgt) p.move_tgt[b * L + j] = 0;
    }
}

__global__ void __launch_bounds__(kThreads) accept_kernel(Params p) {
    __shared__ uint64_t red[kWarps];
    __shared__ int flag;
    const int64_t row = blockIdx.x;
    const int64_t b = row / p.width;
    const uint16_t* x = p.logits + row * p.row_stride;
    const int64_t V = p.vocab;
    const bool vec = ((((uintptr_t)x) & 15u) == 0) && (V % 8 == 0);
    const int64_t nv = vec ? V / 8 : 0;

    // pass 1: max (and first index of it)
    float bv = -INFINITY;
    uint32_t bi = 0xffffffffu;
    for (int64_t v = threadIdx.x; v < nv; v += kThreads) {
        const uint4 w = ldg_stream_u4(x + v * 8);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float a = bf16lo(ws[q]), c = bf16hi(ws[q]);
            if (a > bv || bi == 0xffffffffu) { bv = a; bi = (uint32_t)(v * 8 + 2 * q); }
            if (c > bv) { bv = c; bi = (uint32_t)(v * 8 + 2 * q + 1); }
        }
    }
    for (int64_t c = nv * 8 + threadIdx.x; c < V; c += kThreads) {
        const float a = bf16_at(x + c);
        if (a > bv || bi == 0xffffffffu) { bv = a; bi = (uint32_t)c; }
    }
    const uint64_t mine = (bi == 0xffffffffu) ? 0ull : topk_key(bv, bi);
    const uint64_t best = block_reduce_max_u64(mine, red);
    int64_t token = (int64_t)key_index(best);

    if (p.temperature >= 1e-5f) {
        // stochastic: pass 2 (Z), pass 3 (the crossing), both from L2
        const float m = key_value(best);
        const float inv_t = __frcp_rn(p.temperature);
        uint64_t z = 0;
        for (int64_t c = threadIdx.x; c < V; c += kThreads) z += fixed40(bf16_at(x + c), m, inv_t);
        const uint64_t Z = block_reduce_sum_u64(z, red);
        const double u = p.uniforms[row];
        const uint64_t target = (uint64_t)floor(u * (double)Z);
        // scan tiles of kThreads consecutive elements in order; thread t holds element tile*kThreads + t
        uint64_t acc = 0;
        token = V - 1;
        for (int64_t t0 = 0; t0 < V; t0 += kThreads) {
            const int64_t c = t0 + threadIdx.x;
            const uint64_t e = c < V ? fixed40(bf16_at(x + c), m, inv_t) : 0ull;
            // inclusive scan over the tile in thread order
            uint64_t incl = e;
            const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint64_t y = shfl_u64(incl, lane >= o ? lane - o : lane);
                if (lane >= o) incl += y;
            }
            __syncthreads();
            if (lane == 31) red[warp] = incl;
            __syncthreads();
            uint64_t before = 0, tile = 0;
            for (int w2 = 0; w2 < kWarps; ++w2) {
                const uint64_t s = red[w2];
                if (w2 < warp) before += s;
                tile += s;
            }
            const uint64_t cum = acc + before + incl;
            const bool cross = c < V && cum > target;
            // first crossing element in the tile
            const uint32_t bal = __ballot_sync(MFD_FULL_MASK, cross);
            __syncthreads();
            if (lane == 0) red[warp] = bal ? (uint64_t)(warp * 32 + __ffs(bal) - 1) : ~0ull;
            __syncthreads();
            uint64_t first = ~0ull;
            for (int w2 = 0; w2 < kWarps; ++w2) first = red[w2] < first ? red[w2] : first;
            if (first != ~0ull) {
                token = t0 + (int64_t)first;
                break;
            }
            acc += tile;
        }
    }
    if (threadIdx.x == 0) p.posterior[row] = token;

    if (!p.walk) return;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int t = atomicAdd(p.tickets + b, 1u);
        flag = (t == (unsigned int)(p.width - 1));
    }
    __syncthreads();
    if (!flag) return;
    __threadfence();
    if (threadIdx.x < 32) walk_request(p, b);
    if (threadIdx.x == 0) p.tickets[b] = 0u;
}

// walk only, posterior given (SGLang ddtree_follow)
__global__ void follow_kernel(Params p) {
    const int64_t b = (int64_t)blockIdx.x;
    if (threadIdx.x < 32) walk_request(p, b);
}

}  // namespace accept
}  // namespace mfd

using namespace mfd;

static int accept_common_checks(const char* fn, int64_t bs, int64_t width, const int64_t* tokens,
                                const int64_t* parents, int64_t out_len) {
    if (bs < 0 || width < 1 || out_len < 1) {
        set_error("%s: invalid sizes bs=%lld width=%lld out_len=%lld", fn, (long long)bs, (long long)width,
                  (long long)out_len);
        return MFD_ERR_INVALID;
    }
    if (bs > 0 && (!tokens || !parents)) {
        set_error("%s: tokens and parents are required", fn);
        return MFD_ERR_INVALID;
    }
    return MFD_OK;
}

extern "C" size_t mfd_accept_workspace(int64_t bs) { return (size_t)(bs > 0 ? bs : 1) * sizeof(unsigned int); }

extern "C" int mfd_accept(const void* logits, int64_t row_stride, int64_t vocab, int64_t bs, int64_t width,
                          const int64_t* tokens, int64_t tokens_stride, const int64_t* parents,
                          int64_t parents_stride, float temperature, const double* uniforms, int64_t max_steps,
                          const int64_t* window, const int64_t* prefix_lens, int64_t out_len, int64_t* posterior,
                          int32_t* accept_len, int32_t* commit_lens, int64_t* bonus, int64_t* out_tokens,
                          int64_t* accepted, int64_t* new_seq_lens, int64_t* move_src, int64_t* move_tgt,
                          int64_t* hidden_index, void* workspace, size_t workspace_bytes, void* stream) {
    int rc = accept_common_checks("mfd_accept", bs, width, tokens, parents, out_len);
    if (rc) return rc;
    if (vocab < 1 || vocab >= 0x7fffffff || row_stride < vocab) {
        set_error("mfd_accept: invalid vocab=%lld row_stride=%lld", (long long)vocab, (long long)row_stride);
        return MFD_ERR_INVALID;
    }
    if (bs == 0) return MFD_OK;
    if (!logits || !posterior) {
        set_error("mfd_accept: logits and posterior are required");
        return MFD_ERR_INVALID;
    }
    if (temperature >= 1e-5f && !uniforms) {
        set_error("mfd_accept: temperature > 0 needs uniforms");
        return MFD_ERR_INVALID;
    }
    if (!workspace || workspace_bytes < mfd_accept_workspace(bs)) {
        set_error("mfd_accept: workspace of %zu bytes needed", mfd_accept_workspace(bs));
        return MFD_ERR_INVALID;
    }
    accept::Params p = {};
    p.logits = (const uint16_t*)logits;
    p.row_stride = row_stride;
    p.vocab = vocab;
    p.bs = bs;
    p.width = width;
    p.temperature = temperature;
    p.uniforms = uniforms;
    p.posterior = posterior;
    p.walk = 1;
    p.tokens = tokens;
    p.tokens_stride = tokens_stride;
    p.parents = parents;
    p.parents_stride = parents_stride;
    p.max_steps = max_steps;
    p.window = window;
    p.prefix_lens = prefix_lens;
    p.out_len = out_len;
    p.accept_len = accept_len;
    p.commit_lens = commit_lens;
    p.bonus = bonus;
    p.out_tokens = out_tokens;
    p.accepted = accepted;
    p.new_seq_lens = new_seq_lens;
    p.move_src = move_src;
    p.move_tgt = move_tgt;
    p.hidden_index = hidden_index;
    p.tickets = (unsigned int*)workspace;
    const int64_t rows = bs * width;
    accept::accept_kernel<<<(unsigned)rows, accept::kThreads, 0, (cudaStream_t)stream>>>(p);
    MFD_CHECK_LAUNCH("mfd_accept");
    return MFD_OK;
}

extern "C" int mfd_sample_tokens(const void* logits, int64_t row_stride, int64_t vocab, int64_t rows,
                                 float temperature, const double* uniforms, int64_t* posterior, void* stream) {
    if (rows < 0 || vocab < 1 || vocab >= 0x7fffffff || row_stride < vocab) {
        set_error("mfd_sample_tokens: invalid sizes rows=%lld vocab=%lld", (long long)rows, (long long)vocab);
        return MFD_ERR_INVALID;
    }
    if (rows == 0) return MFD_OK;
    if (!logits || !posterior || (temperature >= 1e-5f && !uniforms)) {
        set_error("mfd_sample_tokens: null pointer");
        return MFD_ERR_INVALID;
    }
    accept::Params p = {};
    p.logits = (const uint16_t*)logits;
    p.row_stride = row_stride;
    p.vocab = vocab;
    p.bs = rows;
    p.width = 1;
    p.temperature = temperature;
    p.uniforms = uniforms;
    p.posterior = posterior;
    p.walk = 0;
    accept::accept_kernel<<<(unsigned)rows, accept::kThreads, 0, (cudaStream_t)stream>>>(p);
    MFD_CHECK_LAUNCH("mfd_sample_tokens");
    return MFD_OK;
}

extern "C" int mfd_follow(const int64_t* posterior, const int64_t* tokens, int64_t tokens_stride,
                          const int64_t* parents, int64_t parents_stride, int64_t bs, int64_t width,
                          int64_t max_steps, const int64_t* window, const int64_t* prefix_lens, int64_t out_len,
                          int32_t* accept_len, int32_t* commit_lens, int64_t* bonus, int64_t* out_tokens,
                          int64_t* accepted, int64_t* new_seq_lens, int64_t* move_src, int64_t* move_tgt,
                          int64_t* hidden_index, void* stream) {
    int rc = accept_common_checks("mfd_follow", bs, width, tokens, parents, out_len);
    if (rc) return rc;
    if (bs == 0) return MFD_OK;
    if (!posterior) {
        set_error("mfd_follow: posterior is required");
        return MFD_ERR_INVALID;
    }
    accept::Params p = {};
    p.posterior = (int64_t*)posterior;
    p.bs = bs;
    p.width = width;
    p.walk = 1;
    p.tokens = tokens;
    p.tokens_stride = tokens_stride;
    p.parents = parents;
    p.parents_stride = parents_stride;
    p.max_steps = max_steps;
    p.window = window;
    p.prefix_lens = prefix_lens;
    p.out_len = out_len;
    p.accept_len = accept_len;
    p.commit_lens = commit_lens;
    p.bonus = bonus;
    p.out_tokens = out_tokens;
    p.accepted = accepted;
    p.new_seq_lens = new_seq_lens;
    p.move_src = move_src;
    p.move_tgt = move_tgt;
    p.hidden_index = hidden_index;
    accept::follow_kernel<<<(unsigned)bs, 32, 0, (cudaStream_t)stream>>>(p);
    MFD_CHECK_LAUNCH("mfd_follow");
    return MFD_OK;
}
