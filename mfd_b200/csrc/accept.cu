// accept.cu -- the acceptance step: the target's token at every tree node (greedy argmax, or one
// reproducible sample per node) and the walk along the verified path.
//
// Greedy: post[i] = first index of the row maximum (torch.argmax; inference/hf/model/utils.py:28-30,
//   SGLang _target_tokens patch:2990-2991).
// Stochastic (temperature T): the reference draws torch.multinomial(softmax(x/T)) (hf/model/utils.py:31-35),
//   which is not reproducible.  This build's rule, identical on CPU (oracle/mfd_oracle.c, sample_row) and GPU
//   bit for bit, is an inverse-CDF sample of softmax(x/T) whose every sum has a fixed order:
//     blocks of 256 logits, lane l of a block holding 8 of them; per block the maximum M_b, the weights
//     e_i = exp32((x_i - M_b) * (1/T)) (Cody-Waite reduction + a fitted degree-5 polynomial, fmaf), lane sums left to
//     right and their butterfly sum S_b (float32); block weights w_b = S_b * exp32((M_b - m) / T) in double
//     (m = row max); 32 runs of consecutive blocks summed left to right, the runs summed in order to Z; then the
//     target u Z is located run -> block -> lane -> logit, each level summing left to right (a level that
//     rounding leaves without a crossing yields its last logit of positive weight).
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


// exp(y), y <= 0, float32: Cody & Waite range reduction (ln 2 = 0.693359375 - 2.12194440e-4) and a degree-5
// polynomial of exp on |r| <= ln2/2 evaluated by Horner's rule; every operation individually rounded.  The
// polynomial 1 + c1 r + ... + c5 r^5 (constant term fixed at 1, so exp32_rule(0) = 1 exactly) was fitted for the
// least maximum relative error by iteratively reweighted least squares (Lawson's method) on 40001 points of
// [-ln2/2, ln2/2]: 9.2e-8 before rounding, within 4 ulp of a correctly rounded expf over the sampling domain.
// n = rint(y log2 e) is formed by adding 1.5 * 2^23 (the sum rounds to the nearest integer, ties to even, exactly
// as rintf) so that neither the rounding nor the float -> int conversion uses the slow conversion pipe.
constexpr float kExpC1 = 0.9999997f, kExpC2 = 0.4999915f, kExpC3 = 0.16667636f, kExpC4 = 0.041897807f,
                kExpC5 = 0.008290256f;
__device__ __forceinline__ float exp32_rule(float y) {
    const bool ok = y > -87.0f;  // also false for NaN
    y = ok ? y : 0.0f;
    const float t = __fadd_rn(__fmul_rn(y, 1.44269504088896341f), 12582912.0f);
    const float n = __fsub_rn(t, 12582912.0f);
    const int ni = __float_as_int(t) - 0x4B400000;
    float r = __fmaf_rn(n, -0.693359375f, y);
    r = __fmaf_rn(n, 2.12194440e-4f, r);
    float q = kExpC5;
    q = __fmaf_rn(q, r, kExpC4);
    q = __fmaf_rn(q, r, kExpC3);
    q = __fmaf_rn(q, r, kExpC2);
    q = __fmaf_rn(q, r, kExpC1);
    q = __fmaf_rn(q, r, 1.0f);
    return ok ? __uint_as_float(__float_as_uint(q) + ((uint32_t)ni << 23)) : 0.0f;
}
// The packed float32 pair operations (pk2, add2, sub2, mul2, fma2, dup2; common.cuh) round every lane like the
// scalar operation, so exp32_rule_x2 below returns, per lane, exactly exp32_rule's bits with half the
// floating-point instructions.
// exp32_rule((x0 - m) * c) and exp32_rule((x1 - m) * c), the operations of exp32_rule on both lanes at once (a lane
// whose argument is not above -87 is computed on and then replaced by 0, as exp32_rule returns).  UNIT: c is 1, so
// the product is the difference itself (multiplying by 1 is exact) and is not computed.
template <bool UNIT>
__device__ __forceinline__ void exp32_rule_x2(uint64_t x01, uint64_t m2, uint64_t c2, float& e0, float& e1) {
    const uint64_t y = UNIT ? sub2(x01, m2) : mul2(sub2(x01, m2), c2);
    const uint64_t t = add2(mul2(y, dup2(1.44269504088896341f)), dup2(12582912.0f));
    const uint64_t n = sub2(t, dup2(12582912.0f));
    uint64_t r = fma2(n, dup2(-0.693359375f), y);
    r = fma2(n, dup2(2.12194440e-4f), r);
    uint64_t q = dup2(kExpC5);
    q = fma2(q, r, dup2(kExpC4));
    q = fma2(q, r, dup2(kExpC3));
    q = fma2(q, r, dup2(kExpC2));
    q = fma2(q, r, dup2(kExpC1));
    q = fma2(q, r, dup2(1.0f));
    float y0, y1, t0, t1, q0, q1;
    upk2(y, y0, y1);
    upk2(t, t0, t1);
    upk2(q, q0, q1);
    // 2^n into the exponent field: (bits(t) - 0x4B400000) << 23 equals bits(t) << 23 modulo 2^32 (0x4B400000's
    // set bits all shift out), so one shift-add per lane gives exp32_rule's bits
    e0 = y0 > -87.0f ? __uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23)) : 0.0f;
    e1 = y1 > -87.0f ? __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23)) : 0.0f;
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
constexpr int kGreedyFlatKeys = 1024;  // part keys of one request staged by the one-ticket path
__global__ void __launch_bounds__(kGreedyThreads) greedy_kernel(Params p) {
    __shared__ uint64_t red[kGreedyThreads / 32];
    __shared__ uint64_t flat_keys[kGreedyFlatKeys];
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
    if (p.walk && p.parts > 1 && p.width * p.parts <= kGreedyFlatKeys) {
        // one ticket per request over all its rows' parts: the last CTA takes every row's maximum over its parts
        // (all keys staged in shared memory in one round of loads), writes the posterior and walks
        if (threadIdx.x == 0) {
            p.part_keys[row * p.parts + part] = best;
            __threadfence();
            const unsigned int t = atomicAdd(p.tickets + b, 1u);
            flag = (t == (unsigned int)(p.width * p.parts - 1));
        }
        __syncthreads();
        if (!flag) return;
        __threadfence();
        const int nkeys = (int)(p.width * p.parts);
        const uint64_t* keys = p.part_keys + b * p.width * p.parts;
        for (int e = threadIdx.x; e < nkeys; e += kGreedyThreads) flat_keys[e] = __ldcg(keys + e);
        __syncthreads();
        for (int r = threadIdx.x; r < (int)p.width; r += kGreedyThreads) {
            uint64_t k = 0;
            for (int i = 0; i < p.parts; ++i) {
                const uint64_t v = flat_keys[r * p.parts + i];
                k = v > k ? v : k;
            }
            p.posterior[b * p.width + r] = (int64_t)key_index(k);
        }
        __syncthreads();  // the posterior rows are visible to the walking warp
        if (threadIdx.x < 32) walk_request(p, b, &stage);
        if (threadIdx.x == 0) p.tickets[b] = 0u;
        return;
    }
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

constexpr int kSampleThreads = 256;
constexpr int kSampleCtasPerSm = 6;  // (40 registers a thread)
constexpr int kSampleWarps = kSampleThreads / 32;
constexpr int kMaxRounds = 192;  // rows up to 192 rounds x 256 threads x 8 logits = 393216 logits
constexpr int kUnroll = 4;      // rounds whose loads are in flight together

// the 8 logits of vector v (elements 8v .. 8v+7 of the row); absent elements read as -inf
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
__device__ __forceinline__ float vec_elem(const uint4& w, int j) {
    const uint32_t word = j < 2 ? w.x : (j < 4 ? w.y : (j < 6 ? w.z : w.w));
    return (j & 1) ? bf16hi(word) : bf16lo(word);
}
__device__ __forceinline__ double shfl_f64(double v, int src) {
    return __longlong_as_double((long long)shfl_u64((uint64_t)__double_as_longlong(v), src));
}

// stochastic: one 256-thread CTA per row (six resident per SM, so a CTA's serial search holds a sixth of an SM's
// warps; 512-thread CTAs, three per SM, measured 2% slower).  One pass over the logits: in round r warp w reduces
// block e = 8 r + w (vector 32 e + lane per lane, so every load is coalesced): the block maximum by warp
// shuffles, the lane sums of the weights against it, and their butterfly sum; lane 0 keeps (M_b, S_b) in shared
// memory.  A block's arithmetic does not depend on which warp reduces it, so the CTA size leaves the rule's bits
// unchanged.  Warp 0 then forms the block weights, the run sums and Z in the rule's order and locates the
// target run -> block -> lane -> logit (re-reading one block of 256 logits).
template <bool UNIT_T>  // temperature exactly 1 (then 1 / T is exactly 1)
__global__ void __launch_bounds__(kSampleThreads, kSampleCtasPerSm) sample_kernel(Params p) {
    __shared__ float blk_m[kMaxRounds * kSampleWarps];
    __shared__ float blk_s[kMaxRounds * kSampleWarps];
    __shared__ double blk_w[kMaxRounds * kSampleWarps];  // block weights, written by the search warp
    __shared__ WalkStage stage;
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
    const float inv_t = __frcp_rn(p.temperature);
    // ---- one pass: block maxima and block sums
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
            float mx = fmaxf(fmax3(vec_elem(w[u], 0), vec_elem(w[u], 1), vec_elem(w[u], 2)),
                             fmax3(vec_elem(w[u], 3), vec_elem(w[u], 4),
                                   fmaxf(vec_elem(w[u], 5), fmaxf(vec_elem(w[u], 6), vec_elem(w[u], 7)))));
            mx = warp_max_f32(mx);  // the block maximum (exact, so the reduction order does not matter)
            float sum = 0.0f;
            if (mx != -INFINITY) {
                const uint64_t m2 = dup2(mx), c2 = dup2(inv_t);
                const uint32_t ws[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {  // logits 2q, 2q + 1: the low and high bf16 of word q
                    float e0, e1;
                    exp32_rule_x2<UNIT_T>(pk2(bf16lo(ws[q]), bf16hi(ws[q])), m2, c2, e0, e1);
                    sum = __fadd_rn(sum, e0);
                    sum = __fadd_rn(sum, e1);
                }
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(MFD_FULL_MASK, sum, o));
            if (lane == 0) {
                blk_m[(r0 + u) * kSampleWarps + warp] = mx;
                blk_s[(r0 + u) * kSampleWarps + warp] = sum;
            }
        }
    }
    __syncthreads();
    if (warp == 0) {
        const int nb = (int)((V + 255) / 256);
        float m = -INFINITY;
        for (int e = lane; e < nb; e += 32) m = fmaxf(m, blk_m[e]);
        m = warp_max_f32(m);
        auto wblk = [&](int e) -> double {  // the block weight S_b * exp32((M_b - m) / T)
            const float mb = blk_m[e];
            if (mb == -INFINITY) return 0.0;
            return __dmul_rn((double)blk_s[e], (double)exp32_rule(__fmul_rn(__fsub_rn(mb, m), inv_t)));
        };
        auto weight = [&](int64_t i, float mb) -> float {  // e_i against its block's maximum
            return mb == -INFINITY ? 0.0f : exp32_rule(__fmul_rn(__fsub_rn(bf16_at(x + i), mb), inv_t));
        };
        // the last logit of positive weight in [lo, hi), or -1
        auto last_positive = [&](int64_t lo, int64_t hi) -> int64_t {
            hi = min(hi, V);
            for (int64_t top = hi; top > lo; top -= 32) {
                const int64_t i = top - 1 - lane;
                bool pos = false;
                if (i >= lo) pos = weight(i, blk_m[i >> 8]) > 0.0f;
                const uint32_t bal = __ballot_sync(MFD_FULL_MASK, pos);
                if (bal) return top - 1 - (__ffs(bal) - 1);  // the lowest lane holds the highest index
            }
            return -1;
        };
        const int per = (nb + 31) / 32;
        // the run sums; each block weight is kept (shared memory) for the walk below.  The unrolled loop lets the
        // exponentials of several blocks overlap while the sum keeps its left-to-right order.
        double run = 0.0;
#pragma unroll 4
        for (int e = lane * per; e < (lane + 1) * per && e < nb; ++e) {
            const double w = wblk(e);
            blk_w[e] = w;
            run = __dadd_rn(run, w);
        }
        // P_{L+1} = P_L + R_L in lane order (every lane computes the same sums); lane L keeps P_L
        double P = 0.0, myP = 0.0;
#pragma unroll
        for (int L = 0; L < 32; ++L) {
            const double r = shfl_f64(run, L);
            if (lane == L) myP = P;
            P = __dadd_rn(P, r);
        }
        const double Z = P;
        int64_t tok = V - 1;  // Z == 0: every logit -inf
        if (Z > 0.0) {
            const double t = __dmul_rn(p.uniforms[row], Z);
            const uint32_t cross = __ballot_sync(MFD_FULL_MASK, __dadd_rn(myP, run) > t);
            if (!cross) {
                tok = last_positive(0, 256 * (int64_t)nb);
            } else {
                const int Ls = __ffs(cross) - 1;
                const double t1 = __dsub_rn(t, shfl_f64(myP, Ls));
                // block of run Ls (lane Ls walks its run)
                int bs = -1;
                double t2 = 0.0;
                __syncwarp();  // the block weights of lane Ls's run are in shared memory
                if (lane == Ls) {
                    double Q = 0.0;
                    for (int e = Ls * per; e < (Ls + 1) * per && e < nb; ++e) {
                        const double Qn = __dadd_rn(Q, blk_w[e]);
                        if (Qn > t1) {
                            bs = e;
                            t2 = __dsub_rn(t1, Q);
                            break;
                        }
                        Q = Qn;
                    }
                }
                bs = __shfl_sync(MFD_FULL_MASK, bs, Ls);
                t2 = shfl_f64(t2, Ls);
                if (bs < 0) {
                    tok = last_positive(256 * (int64_t)(Ls * per), 256 * (int64_t)((Ls + 1) * per));
                } else {
                    const float mb = blk_m[bs];
                    const double sc = (double)exp32_rule(__fmul_rn(__fsub_rn(mb, m), inv_t));
                    const int64_t i0 = 256 * (int64_t)bs + 8 * lane;
                    double w8[8];  // this lane's 8 logit weights, each computed once
#pragma unroll
                    for (int j = 0; j < 8; ++j) w8[j] = i0 + j < V ? __dmul_rn((double)weight(i0 + j, mb), sc) : 0.0;
                    double cl = 0.0;
#pragma unroll
                    for (int j = 0; j < 8; ++j) cl = __dadd_rn(cl, w8[j]);
                    double B = 0.0, myB = 0.0;
#pragma unroll
                    for (int l = 0; l < 32; ++l) {
                        const double c = shfl_f64(cl, l);
                        if (lane == l) myB = B;
                        B = __dadd_rn(B, c);
                    }
                    const uint32_t lc = __ballot_sync(MFD_FULL_MASK, __dadd_rn(myB, cl) > t2);
                    if (!lc) {
                        tok = last_positive(256 * (int64_t)bs, 256 * (int64_t)bs + 256);
                    } else {
                        const int ls = __ffs(lc) - 1;
                        const double t3 = __dsub_rn(t2, shfl_f64(myB, ls));
                        int64_t hit = -1, lastpos = -1;
                        if (lane == ls) {
                            double a = 0.0;
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                const double wv = w8[j];
                                const double an = __dadd_rn(a, wv);
                                if (wv > 0.0) lastpos = i0 + j;
                                if (hit < 0 && an > t3 && wv > 0.0) hit = i0 + j;
                                a = an;
                            }
                            if (hit < 0) hit = lastpos;
                        }
                        tok = (int64_t)__shfl_sync(MFD_FULL_MASK, (long long)hit, ls);
                    }
                }
            }
            if (tok < 0) tok = V - 1;
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
    if (threadIdx.x < 32) walk_request(p, b, &stage);
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
        if (p.temperature == 1.0f)
            accept::sample_kernel<true><<<(unsigned)rows, accept::kSampleThreads, 0, stream>>>(p);
        else
            accept::sample_kernel<false><<<(unsigned)rows, accept::kSampleThreads, 0, stream>>>(p);
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
