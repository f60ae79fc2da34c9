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
// Greedy: the rows are split over several CTAs when there are few of them; the last CTA of a row merges its
// parts.  Sampling: one CTA per row.  In both, the last CTA to finish a request's rows (an atomic ticket per
// request, no waiting) walks that request's tree.  Tickets reset themselves.
#include "common.cuh"

namespace mfd {
namespace accept {


// exp(y), y <= 0, float32: Cody & Waite range reduction (ln 2 = 0.693359375 - 2.12194440e-4) and the
// degree-7 Taylor polynomial of exp evaluated by Horner's rule; every operation individually rounded.
// n = rint(y log2 e) is formed by adding 1.5 * 2^23 (the sum rounds to the nearest integer, ties to even, exactly
// as rintf) so that neither the rounding nor the float -> int conversion uses the slow conversion pipe.
__device__ __forceinline__ float exp32_rule(float y) {
    const bool ok = y > -87.0f;  // also false for NaN
    y = ok ? y : 0.0f;
    const float t = __fadd_rn(__fmul_rn(y, 1.44269504088896341f), 12582912.0f);
    const float n = __fsub_rn(t, 12582912.0f);
    const int ni = __float_as_int(t) - 0x4B400000;
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
    return ok ? __uint_as_float(__float_as_uint(q) + ((uint32_t)ni << 23)) : 0.0f;
}
// trunc(e * 2^40) for 0 <= e < 2 from e's fields: e = M * 2^(k - 23) with M the 24-bit significand, so
// e * 2^40 = M * 2^(k + 17) (exact: the conversion truncates only the fraction); tiny e gives 0.
__device__ __forceinline__ uint64_t fixed40(float x, float m, float inv_t) {
    const uint32_t u = __float_as_uint(exp32_rule(__fmul_rn(__fsub_rn(x, m), inv_t)));
    const int s = (int)(u >> 23) - 127 + 17;
    const uint32_t M = (u & 0x7FFFFFu) | 0x800000u;
    if (u == 0u) return 0ull;
    return s >= 0 ? ((uint64_t)M << s) : (uint64_t)(M >> min(-s, 31));
}

struct Params {
    const uint16_t* logits;  // bf16 rows, row r = b * width + i
    int64_t row_stride;      // elements
    int64_t vocab;
    int64_t bs, width;
    float temperature;       // < 1e-5: greedy
    const double* uniforms;  // [bs * width]
    int64_t* posterior;      // [bs * width]
    int parts;               // greedy: CTAs per row
    uint64_t* part_keys;     // [rows, parts] (greedy, parts > 1)
    unsigned int* row_tickets;  // [rows] (greedy, parts > 1)
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

// Shared-memory staging for the walk: a request's parents, tokens and posterior (widths up to kWalkStage), so
// that each step of the walk costs shared-memory reads instead of dependent L2 round trips.
constexpr int kWalkStage = 256;
struct WalkStage {
    int64_t tok[kWalkStage];
    int64_t post[kWalkStage];
    int32_t par[kWalkStage];
};

// walk request b along its verified path (one warp); SGLang follow-kernel outputs.  `st`: shared staging
// (used when the width fits), or null.
__device__ void walk_request(const Params& p, int64_t b, WalkStage* st) {
    const int lane = threadIdx.x & 31;
    const int64_t W = p.width;
    const int64_t* par = p.parents + b * p.parents_stride;
    const int64_t* tok = p.tokens + b * p.tokens_stride;
    const int64_t* post = p.posterior + b * W;
    const int64_t L = p.out_len;
    const int64_t limit = p.max_steps < 0 ? W : p.max_steps;
    const bool staged = st != nullptr && W <= kWalkStage;
    if (staged) {
        for (int j = lane; j < (int)W; j += 32) {
            const int64_t pj = __ldcg(par + j);
            st->par[j] = (pj < -1 || pj >= W) ? -2 : (int32_t)pj;  // out-of-range parents match no node
            st->tok[j] = __ldcg(tok + j);
            st->post[j] = __ldcg(post + j);
        }
        __syncwarp();
    }
    int64_t cur = 0, n = 0;
    for (int64_t step = 0; step < limit; ++step) {
        const int64_t t = staged ? st->post[cur] : __ldcg(post + cur);
        int64_t child = -1;
        for (int64_t base = 1; base < W && child < 0; base += 32) {
            const int64_t j = base + lane;
            const bool hit = j < W && (staged ? (st->par[j] == (int32_t)cur && st->tok[j] == t)
                                              : (__ldcg(par + j) == cur && __ldcg(tok + j) == t));
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
    const int64_t bon = staged ? st->post[cur] : __ldcg(post + cur);
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

template <int NT>
__device__ __forceinline__ uint64_t block_reduce_max_u64(uint64_t v, uint64_t* red) {
    constexpr int NW = NT / 32;
    v = warp_max_u64(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    uint64_t r = (lane < NW) ? red[lane] : 0ull;
    return warp_max_u64(r);
}

// 16-byte loads in flight per thread in the argmax (8 measured no faster than 4 at 10 parts per row)
constexpr int kGreedyLoads = 4;

// Best (value, first index) key over columns [c0, c1) of row x, one thread's share (vector loads when aligned).
template <int NT>
__device__ __forceinline__ uint64_t argmax_share(const uint16_t* x, int64_t c0, int64_t c1) {
    float bv = -INFINITY;
    uint32_t bi = 0xffffffffu;
    const bool vec = ((((uintptr_t)(x + c0)) & 15u) == 0);
    int64_t c = c0;
    if (vec) {
        const int64_t nv = (c1 - c0) / 8;
        const uint16_t* xv = x + c0;
        for (int64_t v0 = 0; v0 < nv; v0 += kGreedyLoads * NT) {
            uint4 w[kGreedyLoads];
#pragma unroll
            for (int u = 0; u < kGreedyLoads; ++u) {
                const int64_t vi = v0 + (int64_t)u * NT + threadIdx.x;
                w[u] = vi < nv ? ldg_stream_u4(xv + vi * 8) : make_uint4(0xff80ff80u, 0xff80ff80u, 0xff80ff80u, 0xff80ff80u);
            }
#pragma unroll
            for (int u = 0; u < kGreedyLoads; ++u) {
                const int64_t vi = v0 + (int64_t)u * NT + threadIdx.x;
                // the vector's maximum by three packed bf16 maxima; only a vector that beats the running maximum
                // (rare after the first few) is searched for the first index of its maximum, so the thread keeps
                // the first index of its largest value, as an element-by-element strict comparison would
                const __nv_bfloat162 m2 =
                    __hmax2(__hmax2(*reinterpret_cast<const __nv_bfloat162*>(&w[u].x),
                                    *reinterpret_cast<const __nv_bfloat162*>(&w[u].y)),
                            __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&w[u].z),
                                    *reinterpret_cast<const __nv_bfloat162*>(&w[u].w)));
                const float vm = fmaxf(__low2float(m2), __high2float(m2));
                if (vi < nv && (vm > bv || bi == 0xffffffffu)) {
                    const uint32_t ws[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
                    const uint32_t base = (uint32_t)(c0 + vi * 8);
                    uint32_t at = 7;
#pragma unroll
                    for (int q = 3; q >= 0; --q) {  // lowest position holding vm
                        if (bf16hi(ws[q]) == vm) at = 2 * q + 1;
                        if (bf16lo(ws[q]) == vm) at = 2 * q;
                    }
                    if (bi == 0xffffffffu && !(vm == vm)) {  // (a vector of NaNs first: its first element)
                        bv = bf16lo(ws[0]);
                        bi = base;
                    } else {
                        bv = vm;
                        bi = base + at;
                    }
                }
            }
        }
        c = c0 + nv * 8;
    }
    for (int64_t cc = c + threadIdx.x; cc < c1; cc += NT) {
        const float a = bf16_at(x + cc);
        if (a > bv || bi == 0xffffffffu) { bv = a; bi = (uint32_t)cc; }
    }
    return bi == 0xffffffffu ? 0ull : topk_key(bv, bi);
}

constexpr int kGreedyThreads = 256;

// greedy: CTA (row, part) reduces its part; the last part of a row reduces the parts; the last row of a
// request walks the tree
__global__ void __launch_bounds__(kGreedyThreads) greedy_kernel(Params p) {
    __shared__ uint64_t red[kGreedyThreads / 32];
    __shared__ int flag;
    __shared__ WalkStage stage;
    const int64_t row = blockIdx.x / p.parts;
    const int part = blockIdx.x % p.parts;
    const int64_t b = row / p.width;
    const uint16_t* x = p.logits + row * p.row_stride;
    const int64_t V = p.vocab;
    int64_t chunk = (V + p.parts - 1) / p.parts;
    chunk = (chunk + 7) / 8 * 8;
    const int64_t c0 = min(V, (int64_t)part * chunk), c1 = min(V, c0 + chunk);
    const uint64_t best = block_reduce_max_u64<kGreedyThreads>(argmax_share<kGreedyThreads>(x, c0, c1), red);
    if (p.parts > 1) {
        if (threadIdx.x == 0) {
            p.part_keys[row * p.parts + part] = best;
            __threadfence();
            const unsigned int t = atomicAdd(p.row_tickets + row, 1u);
            flag = (t == (unsigned int)(p.parts - 1));
        }
        __syncthreads();
        if (!flag) return;
        if (threadIdx.x < 32) {
            __threadfence();
            uint64_t k = 0;
            for (int i = threadIdx.x; i < p.parts; i += 32) {
                const uint64_t v = __ldcg(p.part_keys + row * p.parts + i);
                k = v > k ? v : k;
            }
            k = warp_max_u64(k);
            if (threadIdx.x == 0) {
                p.posterior[row] = (int64_t)key_index(k);
                p.row_tickets[row] = 0u;
            }
        }
    } else if (threadIdx.x == 0) {
        p.posterior[row] = (int64_t)key_index(best);
    }
    if (!p.walk) return;
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned int t = atomicAdd(p.tickets + b, 1u);
        flag = (t == (unsigned int)(p.width - 1));
    }
    __syncthreads();
    if (!flag) return;
    __threadfence();
    if (threadIdx.x < 32) walk_request(p, b, &stage);
    if (threadIdx.x == 0) p.tickets[b] = 0u;
}

// sum of the fixed-point weights of x[c0, c1) (one thread, sequential, vector loads when aligned)
__device__ __forceinline__ uint64_t weight_sum(const uint16_t* x, int64_t c0, int64_t c1, float m, float inv_t) {
    uint64_t z = 0;
    int64_t c = c0;
    if ((((uintptr_t)(x + c)) & 15u) == 0) {
        for (; c + 8 <= c1; c += 8) {
            const uint4 w = *reinterpret_cast<const uint4*>(x + c);
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) z += fixed40(bf16lo(ws[q]), m, inv_t) + fixed40(bf16hi(ws[q]), m, inv_t);
        }
    }
    for (; c < c1; ++c) z += fixed40(bf16_at(x + c), m, inv_t);
    return z;
}

constexpr int kSampleThreads = 768;
constexpr int kSampleWarps = kSampleThreads / 32;
constexpr int kMaxRounds = 64;
constexpr int kUnroll = 4;      // rounds whose loads are in flight together  // rows up to 64 rounds x 768 threads x 8 elements = 393216 logits

__device__ __forceinline__ uint64_t warp_sum_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += shfl_xor_u64(v, o);
    return v;
}
// the weights of vector v (elements 8v .. 8v+7 of the row) and its float maximum; absent elements weigh 0
__device__ __forceinline__ uint4 load_vec8(const uint16_t* x, int64_t v, int64_t V, bool aligned) {
    const int64_t e0 = v * 8;
    if (aligned && e0 + 8 <= V) return ldg_stream_u4(x + e0);
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint32_t lo = e0 + 2 * q < V ? x[e0 + 2 * q] : 0xFF80u;      // bf16 -inf
        const uint32_t hi = e0 + 2 * q + 1 < V ? x[e0 + 2 * q + 1] : 0xFF80u;
        w[q] = lo | (hi << 16);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ uint64_t vec8_weight(uint4 w, float m, float inv_t) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    uint64_t z = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) z += fixed40(bf16lo(ws[q]), m, inv_t) + fixed40(bf16hi(ws[q]), m, inv_t);
    return z;
}

// The weight of a logit depends only on its bf16 bit pattern (m and T are fixed per row), so each row first
// tabulates fixed40 over the patterns it can contain and pass 2 looks weights up instead of evaluating the
// exponential 150k times.  Table: for each sign, H + 1 entries indexed by t = clamp(magnitude - lo + 1, 0, H):
//   * t = 0, magnitudes below lo (|x| < tau): every such pattern has the weight of x = 0: with m != 0,
//     tau = 2^(e_m - 26) is under a quarter ulp of m, so fsub(x, m) == -m exactly; with m == 0, tau = 2^(e_T - 28)
//     keeps |x / T| < 2^-26, where the polynomial rounds to exactly 1.0, as it does for x = 0;
//   * t = 1 .. H - 1, magnitudes lo .. hi with hi = the bf16 magnitude at or above 90 T + |m|: fixed40 of the
//     pattern (positive patterns above m cannot occur: m is the row max);
//   * t = H, magnitudes beyond hi: (x - m) / T < -88 after rounding for negatives, weight 0 (positives cannot
//     occur), as for the infinities and NaNs, whose direct weight is 0 too.
// The clamp runs on both halves of a 32-bit word at once (16-bit SIMD add + min with relu).  Every entry is
// fixed40 itself, an integer below 2^41, so a thread adds its looked-up weights exactly in double (partial sums stay
// below 2^53) on the FP64 pipe, and pass 2 sums exactly the values the direct evaluation would.
constexpr int kTableCap = 12 * 1024;  // entries; rows needing more are evaluated directly

struct RowTable {
    int lo, H;  // magnitude offset and clamp limit; H < 0: no table
};

__device__ __forceinline__ int bf16_mag_ceil(float v) {  // smallest bf16 magnitude pattern >= v (v >= 0, finite)
    uint32_t u = __float_as_uint(v);
    uint32_t hi = u >> 16;
    if (u & 0xFFFFu) ++hi;
    return (int)min(hi, 0x7F80u);
}

__device__ RowTable plan_table(float m, float inv_t) {
    RowTable t;
    t.H = -1;
    t.lo = 0;
    if (!isfinite(m) || !(inv_t > 0.f) || !isfinite(inv_t)) return t;
    const float T = 1.0f / inv_t;
    float tau;
    if (m != 0.0f && fabsf(m) >= 1e-30f) {
        const int e_m = ((__float_as_uint(m) >> 23) & 0xFF) - 127;
        tau = ldexpf(1.0f, e_m - 26);
    } else if (m == 0.0f) {
        const int e_t = ((__float_as_uint(T) >> 23) & 0xFF) - 127;
        tau = ldexpf(1.0f, max(e_t - 28, -126));
    } else {
        return t;  // a tiny nonzero max: evaluate directly
    }
    const int lo = (int)(__float_as_uint(tau) >> 16);  // tau is a power of two: exact as bf16 (lo >= 0x80)
    const int hi = bf16_mag_ceil(90.0f * T + fabsf(m));
    const int H = max(hi - lo + 2, 1);
    if (2 * (H + 1) > kTableCap) return t;
    t.lo = lo;
    t.H = H;
    return t;
}

// stochastic: one 768-thread CTA per row (two resident per SM, so about 300 rows are in flight and the second
// pass over a row hits L2).  Vector v = r * 768 + t (8 logits) belongs to thread t in round r, so every load is
// coalesced and the rounds are in row order.  Pass 1: the row max.  Table of weights.  Pass 2: per round, each
// warp's 256-logit weight sum.  Warp 0 scans the (round, warp) sums in row order to find the one holding
// floor(u * Z) and searches its 256 logits.  All sums are integers, so no order changes the result.
__global__ void __launch_bounds__(kSampleThreads, 2) sample_kernel(Params p) {
    extern __shared__ __align__(16) double table[];  // [2][H + 1] (<= kTableCap)
    __shared__ uint64_t wsum[kMaxRounds * kSampleWarps];
    __shared__ float wmax[kSampleWarps];
    __shared__ int flag;
    __shared__ int64_t s_token;
    const int64_t row = blockIdx.x;
    const int64_t b = row / p.width;
    const uint16_t* x = p.logits + row * p.row_stride;
    const int64_t V = p.vocab;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool aligned = (((uintptr_t)x) & 15u) == 0;
    const int64_t nv = (V + 7) / 8;
    const int rounds = (int)((nv + kSampleThreads - 1) / kSampleThreads);
    // ---- pass 1: max (bf16 pairs), kUnroll rounds' loads in flight per thread; absent elements read as -inf
    __nv_bfloat162 mx2 = __floats2bfloat162_rn(-INFINITY, -INFINITY);
    for (int r0 = 0; r0 < rounds; r0 += kUnroll) {
        uint4 w[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t v = (int64_t)(r0 + u) * kSampleThreads + threadIdx.x;
            w[u] = v < nv ? load_vec8(x, v, V, aligned) : make_uint4(0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const uint32_t ws[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
#pragma unroll
            for (int q = 0; q < 4; ++q) mx2 = __hmax2(mx2, *reinterpret_cast<const __nv_bfloat162*>(&ws[q]));
        }
    }
    float mx = fmaxf(__low2float(mx2), __high2float(mx2));
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(MFD_FULL_MASK, mx, o));
    if (lane == 0) wmax[warp] = mx;
    __syncthreads();
    float m = wmax[0];
#pragma unroll 8
    for (int w = 1; w < kSampleWarps; ++w) m = fmaxf(m, wmax[w]);
    const float inv_t = __frcp_rn(p.temperature);
    // ---- the row's weight table
    const RowTable tb = plan_table(m, inv_t);
    if (tb.H >= 0) {
        const int half = tb.H + 1;
        for (int i = threadIdx.x; i < 2 * half; i += kSampleThreads) {
            const int sg = i >= half ? 1 : 0, t = i - sg * half;
            uint64_t e;
            if (t == 0) {
                e = fixed40(0.0f, m, inv_t);  // every magnitude below tau
            } else if (t < tb.H) {
                const uint32_t pat = ((uint32_t)sg << 15) | (uint32_t)(tb.lo + t - 1);
                const float v = __uint_as_float(pat << 16);
                e = (sg == 0 && v > m) ? 0ull : fixed40(v, m, inv_t);  // (positives above m cannot occur)
            } else {
                e = 0ull;  // beyond the cut, infinities, NaNs
            }
            table[i] = (double)e;  // exact: e < 2^41
        }
        __syncthreads();
    }
    const uint32_t add2 = (uint32_t)(uint16_t)(1 - tb.lo) * 0x10001u;  // both halves: 1 - lo
    const uint32_t lim2 = (uint32_t)(uint16_t)max(tb.H, 0) * 0x10001u;  // both halves: H
    const int half_entries = tb.H + 1;
    // the weight of 8 logits as an exact double (an integer below 2^44)
    auto vec_weight = [&](uint4 w) -> double {
        if (tb.H < 0) return (double)vec8_weight(w, m, inv_t);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        double z = 0.0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            // t for both halves at once: clamp(magnitude - lo + 1, 0, H)
            const uint32_t t2 = __viaddmin_s16x2_relu(ws[q] & 0x7FFF7FFFu, add2, lim2);
            const int i_lo = (int)(t2 & 0xFFFFu) + (int)((ws[q] >> 15) & 1u) * half_entries;
            const int i_hi = (int)(t2 >> 16) + (int)(ws[q] >> 31) * half_entries;
            z += table[i_lo];
            z += table[i_hi];
        }
        return z;
    };
    // ---- pass 2: the weight of each (round, warp) block of 256 logits
    for (int r0 = 0; r0 < rounds; r0 += kUnroll) {
        uint4 w[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t v = (int64_t)(r0 + u) * kSampleThreads + threadIdx.x;
            w[u] = v < nv ? load_vec8(x, v, V, aligned) : make_uint4(0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            if (r0 + u >= rounds) break;
            // a block of 256 weights sums below 2^52: exact in double; absent elements (-inf) weigh 0
            double z = vec_weight(w[u]);
#pragma unroll
            for (int o = 16; o; o >>= 1) z += __shfl_xor_sync(MFD_FULL_MASK, z, o);
            if (lane == 0) wsum[(r0 + u) * kSampleWarps + warp] = (uint64_t)z;
        }
    }
    __syncthreads();
    if (warp == 0) {
        // exclusive scan over the rounds x warps block sums in row order, a contiguous run of entries per lane
        const int ne = rounds * kSampleWarps;
        const int per = (ne + 31) / 32;
        const int e0 = min(lane * per, ne), e1 = min(e0 + per, ne);
        uint64_t tot = 0;
        for (int e = e0; e < e1; ++e) tot += wsum[e];
        uint64_t incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint64_t y = shfl_u64(incl, lane >= o ? lane - o : lane);
            if (lane >= o) incl += y;
        }
        const uint64_t Z = shfl_u64(incl, 31);
        const uint64_t target = (uint64_t)floor(p.uniforms[row] * (double)Z);
        uint64_t run = incl - tot;
        int hit = -1;
        uint64_t before = 0;
        for (int e = e0; e < e1; ++e) {
            const uint64_t w = wsum[e];
            if (hit < 0 && run + w > target) {
                hit = e;
                before = run;
            }
            run += w;
        }
        const uint32_t bal = __ballot_sync(MFD_FULL_MASK, hit >= 0);
        int64_t tok = V - 1;  // Z == 0 (every logit -inf): no crossing
        if (bal) {
            const int src = __ffs(bal) - 1;  // blocks are in lane order: the first lane with a hit holds it
            const int eh = __shfl_sync(MFD_FULL_MASK, hit, src);
            const uint64_t base = shfl_u64(before, src);
            // block eh = (round eh / warps, warp eh % warps): 32 consecutive vectors, one per lane
            const int64_t v = (int64_t)(eh / kSampleWarps) * kSampleThreads + (eh % kSampleWarps) * 32 + lane;
            const uint4 w = v < nv ? load_vec8(x, v, V, aligned)
                                   : make_uint4(0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u);
            const uint64_t ls = v < nv ? vec8_weight(w, m, inv_t) : 0ull;
            uint64_t li = ls;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint64_t y = shfl_u64(li, lane >= o ? lane - o : lane);
                if (lane >= o) li += y;
            }
            const uint64_t lex = base + li - ls;
            const bool in_me = ls > 0 && lex <= target && target < lex + ls;
            const uint32_t b2 = __ballot_sync(MFD_FULL_MASK, in_me);
            const int owner = b2 ? __ffs(b2) - 1 : 0;
            if (b2 && lane == owner) {
                const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
                uint64_t c = lex;
                tok = v * 8 + 7;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float xv = (q & 1) ? bf16hi(ws[q >> 1]) : bf16lo(ws[q >> 1]);
                    c += fixed40(xv, m, inv_t);
                    if (c > target) {
                        tok = v * 8 + q;
                        break;
                    }
                }
            }
            tok = __shfl_sync(MFD_FULL_MASK, (long long)tok, owner);
        }
        if (lane == 0) s_token = tok;
    }
    __syncthreads();
    if (threadIdx.x == 0) p.posterior[row] = s_token;
    if (!p.walk) return;
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned int t = atomicAdd(p.tickets + b, 1u);
        flag = (t == (unsigned int)(p.width - 1));
    }
    __syncthreads();
    if (!flag) return;
    __threadfence();
    if (threadIdx.x < 32) walk_request(p, b, sizeof(WalkStage) <= kTableCap * sizeof(double) ? reinterpret_cast<WalkStage*>(table) : nullptr);
    if (threadIdx.x == 0) p.tickets[b] = 0u;
}

// walk only, posterior given (SGLang ddtree_follow)
__global__ void follow_kernel(Params p) {
    __shared__ WalkStage stage;
    const int64_t b = (int64_t)blockIdx.x;
    if (threadIdx.x < 32) walk_request(p, b, &stage);
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

static int greedy_parts(int64_t rows) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t want = 4LL * sms;
    int64_t parts = (want + rows - 1) / rows;
    return (int)(parts < 1 ? 1 : (parts > 32 ? 32 : parts));
}

// scratch: part keys [rows * 32]; tickets (a buffer that is only ever used for tickets and is left zeroed):
// request tickets [bs] then row tickets [rows]
static size_t accept_scratch(int64_t rows) { return (size_t)(rows > 0 ? rows : 1) * 32 * 8; }

static int launch_accept(accept::Params& p, int64_t rows, void* scratch, unsigned int* tickets, cudaStream_t stream,
                         const char* fn) {
    p.tickets = tickets;
    p.row_tickets = tickets + (p.bs > 0 ? p.bs : 1);
    p.part_keys = (uint64_t*)scratch;
    if (p.temperature < 1e-5f) {
        p.parts = greedy_parts(rows);
        accept::greedy_kernel<<<(unsigned)(rows * p.parts), accept::kGreedyThreads, 0, stream>>>(p);
    } else {
        p.parts = 1;
        const int smem = accept::kTableCap * (int)sizeof(uint64_t);
        cudaError_t e = cudaFuncSetAttribute(accept::sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) {
            set_error("%s: %s", fn, cudaGetErrorString(e));
            return MFD_ERR_CUDA;
        }
        accept::sample_kernel<<<(unsigned)rows, accept::kSampleThreads, smem, stream>>>(p);
    }
    MFD_CHECK_LAUNCH(fn);
    return MFD_OK;
}

extern "C" size_t mfd_accept_workspace(int64_t bs, int64_t width) { return accept_scratch(bs * width); }

extern "C" int64_t mfd_accept_tickets(int64_t bs, int64_t width) { return (bs > 0 ? bs : 1) + bs * width; }

extern "C" int mfd_accept(const void* logits, int64_t row_stride, int64_t vocab, int64_t bs, int64_t width,
                          const int64_t* tokens, int64_t tokens_stride, const int64_t* parents,
                          int64_t parents_stride, float temperature, const double* uniforms, int64_t max_steps,
                          const int64_t* window, const int64_t* prefix_lens, int64_t out_len, int64_t* posterior,
                          int32_t* accept_len, int32_t* commit_lens, int64_t* bonus, int64_t* out_tokens,
                          int64_t* accepted, int64_t* new_seq_lens, int64_t* move_src, int64_t* move_tgt,
                          int64_t* hidden_index, void* workspace, size_t workspace_bytes, unsigned int* tickets,
                          int64_t tickets_len, void* stream) {
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
    if (temperature >= 1e-5f && vocab > (int64_t)accept::kMaxRounds * accept::kSampleThreads * 8) {
        set_error("mfd_accept: sampling supports vocab <= %d", accept::kMaxRounds * accept::kSampleThreads * 8);
        return MFD_ERR_UNSUPPORTED;
    }
    if (!workspace || workspace_bytes < mfd_accept_workspace(bs, width) || !tickets ||
        tickets_len < mfd_accept_tickets(bs, width)) {
        set_error("mfd_accept: workspace of %zu bytes and %lld zeroed tickets needed", mfd_accept_workspace(bs, width),
                  (long long)mfd_accept_tickets(bs, width));
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
    return launch_accept(p, bs * width, workspace, tickets, (cudaStream_t)stream, "mfd_accept");
}

extern "C" size_t mfd_sample_tokens_workspace(int64_t rows) { return accept_scratch(rows); }

extern "C" int mfd_sample_tokens(const void* logits, int64_t row_stride, int64_t vocab, int64_t rows,
                                 float temperature, const double* uniforms, int64_t* posterior, void* workspace,
                                 size_t workspace_bytes, unsigned int* tickets, int64_t tickets_len, void* stream) {
    if (rows < 0 || vocab < 1 || vocab >= 0x7fffffff || row_stride < vocab) {
        set_error("mfd_sample_tokens: invalid sizes rows=%lld vocab=%lld", (long long)rows, (long long)vocab);
        return MFD_ERR_INVALID;
    }
    if (rows == 0) return MFD_OK;
    if (!logits || !posterior || (temperature >= 1e-5f && !uniforms)) {
        set_error("mfd_sample_tokens: null pointer");
        return MFD_ERR_INVALID;
    }
    if (temperature >= 1e-5f && vocab > (int64_t)accept::kMaxRounds * accept::kSampleThreads * 8) {
        set_error("mfd_sample_tokens: sampling supports vocab <= %d", accept::kMaxRounds * accept::kSampleThreads * 8);
        return MFD_ERR_UNSUPPORTED;
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
    if (!workspace || workspace_bytes < mfd_sample_tokens_workspace(rows) || !tickets || tickets_len < rows + 1) {
        set_error("mfd_sample_tokens: workspace of %zu bytes and %lld zeroed tickets needed",
                  mfd_sample_tokens_workspace(rows), (long long)(rows + 1));
        return MFD_ERR_INVALID;
    }
    return launch_accept(p, rows, workspace, tickets, (cudaStream_t)stream, "mfd_sample_tokens");
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
