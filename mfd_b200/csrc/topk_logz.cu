// topk_logz.cu -- the logits step of tree construction: per row of draft logits, the top-k candidates
// (value descending, equal values by lower index first) and log Z = logsumexp(row), in ONE pass over HBM.
//
// Reference: inference/hf/ddtree.py:240-244 (float32 topk + logsumexp, then top - log_z),
// inference/hf/tree_logits.py:16-46 (bf16 top-k + one-pass online logsumexp), SGLang
// DDTreeDraftTopK / _row_logsumexp_kernel (sglang-v0.5.22-mfd.patch:1451-1550).
//
// Work split: the R x V element space is cut into `grid` equal contiguous ranges, one per CTA, sized so the
// grid is a single wave (a multiple of the SM count).  A range may span a row boundary, so a CTA emits one
// partial record per row piece it covers: (max, sum exp) and its top-k list.  Inside a CTA each warp streams
// its share with 16-byte non-allocating loads, keeps an online (max, sum) per thread and a candidate buffer in
// shared memory filtered against a running threshold (the k-th best key seen so far; the per-element test is
// one float compare), compacting with a register bitonic sort when the buffer fills.  Warp lists merge into
// the CTA list by bitonic merges; the last CTA to finish a row (an atomic ticket per row, no waiting) merges
// that row's partial records and writes top_logp = top - logZ, ids, logZ.  The tickets reset themselves.
#include <cstdio>

#include "common.cuh"

namespace mfd {
namespace topk {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kUnroll = 4;

// Warp bitonic sort, descending, of CAP keys held as r[j] = element j*32 + lane.
template <int CAP>
__device__ __forceinline__ void warp_sort_desc(uint64_t (&r)[CAP / 32]) {
    constexpr int PER = CAP / 32;
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int size = 2; size <= CAP; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= 32) {
                const int js = stride >> 5;
#pragma unroll
                for (int j = 0; j < PER; ++j) {
                    if ((j & js) == 0) {
                        const int e = j * 32 + lane;
                        const bool desc = (e & size) == 0;  // descending block
                        uint64_t a = r[j], b = r[j | js];
                        const bool sw = desc ? (a < b) : (a > b);
                        r[j] = sw ? b : a;
                        r[j | js] = sw ? a : b;
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < PER; ++j) {
                    const int e = j * 32 + lane;
                    uint64_t o = shfl_xor_u64(r[j], stride);
                    const bool desc = (e & size) == 0;
                    const bool lower = (lane & stride) == 0;
                    // lower element keeps max in a descending block, min in an ascending one
                    const bool keep_max = (lower == desc);
                    r[j] = keep_max ? (r[j] > o ? r[j] : o) : (r[j] < o ? r[j] : o);
                }
            }
        }
    }
}

// Sort a bitonic sequence of KP keys (r[j] = element j*32 + lane when KP >= 32, else lane < KP holds r[0])
// into descending order.
template <int KP>
__device__ __forceinline__ void warp_bitonic_merge_desc(uint64_t (&r)[(KP + 31) / 32]) {
    constexpr int PER = (KP + 31) / 32;
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int stride = KP >> 1; stride > 0; stride >>= 1) {
        if (stride >= 32) {
            const int js = stride >> 5;
#pragma unroll
            for (int j = 0; j < PER; ++j) {
                if ((j & js) == 0) {
                    uint64_t a = r[j], b = r[j | js];
                    r[j] = a > b ? a : b;
                    r[j | js] = a > b ? b : a;
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < PER; ++j) {
                uint64_t o = shfl_xor_u64(r[j], stride);
                const bool lower = (lane & stride) == 0;
                r[j] = lower ? (r[j] > o ? r[j] : o) : (r[j] < o ? r[j] : o);
            }
        }
    }
}

// Merge two descending lists a[0..KP) and b[0..KP) (shared or global) into the descending top-KP, written to out.
template <int KP>
__device__ __forceinline__ void warp_merge_lists(const uint64_t* a, const uint64_t* b, uint64_t* out) {
    constexpr int PER = (KP + 31) / 32;
    const int lane = threadIdx.x & 31;
    uint64_t r[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int e = j * 32 + lane;
        if (e < KP) {
            uint64_t x = a[e], y = b[KP - 1 - e];
            r[j] = x > y ? x : y;  // the larger half of a bitonic concatenation
        } else {
            r[j] = 0;
        }
    }
    if (KP >= 2) warp_bitonic_merge_desc<KP>(r);
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int e = j * 32 + lane;
        if (e < KP) out[e] = r[j];
    }
}

struct Params {
    const void* x;
    int is_bf16;
    int64_t rows, vocab, row_stride;  // in elements
    int k;
    float* top_logp;      // [rows, k]
    void* top_ids;        // [rows, k] int32 or int64
    int ids_i64;
    float* logz;          // [rows] or null
    int64_t per_cta;      // elements per CTA (multiple of 8)
    int max_pieces;       // partial-record slots per row
    float2* part_ms;      // [rows, max_pieces]
    uint64_t* part_keys;  // [rows, max_pieces, KP]
    unsigned int* tickets;  // [rows], zero between launches
};

template <int CAP, int KP>
struct Smem {
    uint64_t buf[kWarps][CAP];
    uint64_t res[KP];  // running merge result of the last-CTA row merge
    float2 ms[kWarps];
    float logz;
    int flag;
};

template <int CAP, int KP>
struct WarpState {
    int cnt;          // buffered candidates (warp-uniform)
    uint64_t thr;     // a new element must beat this key
    float thr_v;      // value prefilter: x >= thr_v
};

template <int CAP, int KP>
__device__ __forceinline__ void compact(uint64_t* buf, WarpState<CAP, KP>& st, int k) {
    constexpr int PER = CAP / 32;
    const int lane = threadIdx.x & 31;
    __syncwarp();
    uint64_t r[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int e = j * 32 + lane;
        r[j] = (e < st.cnt) ? buf[e] : 0ull;
    }
    warp_sort_desc<CAP>(r);
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int e = j * 32 + lane;
        if (e < KP) buf[e] = (e < k) ? r[j] : 0ull;
    }
    // the k-th best key (element k-1) becomes the threshold once k candidates exist
    const int kk = k - 1;
    uint64_t mine = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j)
        if (j == (kk >> 5)) mine = r[j];
    uint64_t kth = shfl_u64(mine, kk & 31);
    __syncwarp();
    if (st.cnt >= k) {
        st.cnt = k;
        st.thr = kth;
        st.thr_v = key_value(kth);
    }
}

// Append the candidates among x[off..off+4) (element j has index idx0 + j) that beat the threshold.
template <int N, int CAP, int KP>
__device__ __forceinline__ void consume(uint64_t* buf, WarpState<CAP, KP>& st, int k, const float (&x)[N],
                                        uint32_t idx0, bool ok, int off) {
    bool any = false;
#pragma unroll
    for (int j = 0; j < 4 && off + j < N; ++j) any |= ok && (x[off + j] >= st.thr_v);
    if (!__any_sync(MFD_FULL_MASK, any)) return;
    if (st.cnt + 32 * 4 > CAP) compact<CAP, KP>(buf, st, k);
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < 4 && off + j < N; ++j) {
        const uint64_t key = ok ? topk_key(x[off + j], idx0 + (uint32_t)(off + j)) : 0ull;
        const bool take = ok && key > st.thr;
        uint32_t bal = __ballot_sync(MFD_FULL_MASK, take);
        if (take) buf[st.cnt + __popc(bal & ((1u << lane) - 1u))] = key;
        st.cnt += __popc(bal);
    }
}

template <int N>
__device__ __forceinline__ void online_lse(float& m, float& s, const float (&x)[N], bool ok) {
    if (!ok) return;
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < N; ++j) mx = fmaxf(mx, x[j]);
    const float mn = fmaxf(m, mx);
    if (mn == -INFINITY) return;
    // exponents as (x - mn) * log2(e): the difference is exact or nearly so, which keeps the large terms accurate
    float acc = s * fast_exp2((m - mn) * kLog2e);
#pragma unroll
    for (int j = 0; j < N; ++j) acc += fast_exp2((x[j] - mn) * kLog2e);
    s = acc;
    m = mn;
}

// Stream row `row` over columns [c0, c1) with the whole CTA; leaves each warp's sorted top list in
// sm.buf[warp][0..KP) and each warp's (m, s) in sm.ms[warp].
template <int CAP, int KP, bool BF16>
__device__ __forceinline__ void stream_piece(const Params p, Smem<CAP, KP>& sm, int64_t row, int64_t c0, int64_t c1) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t* buf = sm.buf[warp];
    WarpState<CAP, KP> st;
    st.cnt = 0;
    st.thr = 0;
    st.thr_v = -INFINITY;
    float m = -INFINITY, s = 0.f;
    constexpr int VE = BF16 ? 8 : 4;  // elements per 16-byte vector
    const char* base = (const char*)p.x + (size_t)row * p.row_stride * (BF16 ? 2 : 4);

    auto scalar_at = [&](int64_t c) -> float {
        return BF16 ? bf16_at((const uint16_t*)base + c) : ((const float*)base)[c];
    };

    // head: up to the first 16-byte boundary
    int64_t hb = c0;
    {
        const uintptr_t a = (uintptr_t)(base + c0 * (BF16 ? 2 : 4));
        const int64_t mis = (int64_t)((a & 15u) / (BF16 ? 2 : 4));
        if (mis) hb = c0 + (VE - mis);
        if (hb > c1) hb = c1;
        // the row pointer itself may be misaligned relative to elements (odd strides): then no vector body
        if (((uintptr_t)(base + hb * (BF16 ? 2 : 4)) & 15u) != 0) hb = c1;
    }
    for (int64_t c = c0; c < hb; c += kThreads) {
        const int64_t cc = c + threadIdx.x;
        const bool ok = cc < hb;
        float x[1] = {ok ? scalar_at(cc) : -INFINITY};
        online_lse<1>(m, s, x, ok);
        consume<1, CAP, KP>(buf, st, p.k, x, (uint32_t)cc, ok, 0);
    }
    // body: 16-byte vectors, kUnroll loads in flight per thread
    const int64_t nvec = (c1 - hb) / VE;
    const char* vbase = base + hb * (BF16 ? 2 : 4);
    const int64_t step = (int64_t)kThreads * kUnroll;
    for (int64_t v0 = 0; v0 < nvec; v0 += step) {
        uint4 raw[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t vi = v0 + (int64_t)u * kThreads + threadIdx.x;
            raw[u] = (vi < nvec) ? ldg_stream_u4(vbase + vi * 16) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t vi = v0 + (int64_t)u * kThreads + threadIdx.x;
            const bool ok = vi < nvec;
            float x[VE];
            if (BF16) {
                const uint32_t w[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    x[2 * q] = bf16lo(w[q]);
                    x[2 * q + 1] = bf16hi(w[q]);
                }
            } else {
                x[0] = __uint_as_float(raw[u].x);
                x[1] = __uint_as_float(raw[u].y);
                x[2] = __uint_as_float(raw[u].z);
                x[3] = __uint_as_float(raw[u].w);
            }
            const uint32_t i0 = (uint32_t)(hb + vi * VE);
            online_lse<VE>(m, s, x, ok);
            // at most 4 candidates per lane per append round keeps 32 * 4 + KP <= CAP
            consume<VE, CAP, KP>(buf, st, p.k, x, i0, ok, 0);
            if (BF16) consume<VE, CAP, KP>(buf, st, p.k, x, i0, ok, 4);
        }
    }
    // tail
    const int64_t tb = hb + nvec * VE;
    for (int64_t c = tb; c < c1; c += kThreads) {
        const int64_t cc = c + threadIdx.x;
        const bool ok = cc < c1;
        float x[1] = {ok ? scalar_at(cc) : -INFINITY};
        online_lse<1>(m, s, x, ok);
        consume<1, CAP, KP>(buf, st, p.k, x, (uint32_t)cc, ok, 0);
    }
    // final compaction: sorted, top-k kept, padded with zero keys to KP
    compact<CAP, KP>(buf, st, p.k);
    // warp (m, s)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float m2 = __shfl_xor_sync(MFD_FULL_MASK, m, o);
        float s2 = __shfl_xor_sync(MFD_FULL_MASK, s, o);
        lse_merge(m, s, m2, s2);
    }
    if (lane == 0) sm.ms[warp] = make_float2(m, s);
}

template <int CAP, int KP>
__device__ __forceinline__ void write_outputs(const Params p, int64_t row, const uint64_t* keys, float logz) {
    for (int e = threadIdx.x; e < p.k; e += blockDim.x) {
        const uint64_t key = keys[e];
        const float v = key_value(key);
        const uint32_t id = key_index(key);
        p.top_logp[row * p.k + e] = __fsub_rn(v, logz);
        if (p.ids_i64)
            ((int64_t*)p.top_ids)[row * p.k + e] = (int64_t)id;
        else
            ((int32_t*)p.top_ids)[row * p.k + e] = (int32_t)id;
    }
    if (threadIdx.x == 0 && p.logz) p.logz[row] = logz;
}

template <int CAP, int KP, bool BF16>
__global__ void __launch_bounds__(kThreads, 4) topk_logz_kernel(Params p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem<CAP, KP>& sm = *reinterpret_cast<Smem<CAP, KP>*>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t total = p.rows * p.vocab;
    const int64_t a = (int64_t)blockIdx.x * p.per_cta;
    const int64_t b = a + p.per_cta < total ? a + p.per_cta : total;
    if (a >= b) return;
    for (int64_t row = a / p.vocab; row * p.vocab < b; ++row) {
        const int64_t r0 = row * p.vocab;
        const int64_t c0 = a > r0 ? a - r0 : 0;
        const int64_t c1 = (b < r0 + p.vocab ? b : r0 + p.vocab) - r0;
        stream_piece<CAP, KP, BF16>(p, sm, row, c0, c1);
        __syncthreads();
        // CTA merge of the warp lists: 8 -> 4 -> 2 -> 1
#pragma unroll
        for (int span = 1; span < kWarps; span <<= 1) {
            if ((warp % (2 * span)) == 0) warp_merge_lists<KP>(sm.buf[warp], sm.buf[warp + span], sm.buf[warp]);
            __syncthreads();
        }
        // publish this piece
        const int64_t first_cta = r0 / p.per_cta;
        const int64_t last_cta = (r0 + p.vocab - 1) / p.per_cta;
        const int pieces = (int)(last_cta - first_cta + 1);
        const int slot = (int)(blockIdx.x - first_cta);
        uint64_t* dst = p.part_keys + ((size_t)row * p.max_pieces + slot) * KP;
        for (int e = threadIdx.x; e < KP; e += blockDim.x) dst[e] = sm.buf[0][e];
        if (threadIdx.x == 0) {
            float mm = -INFINITY, ss = 0.f;
            for (int w = 0; w < kWarps; ++w) lse_merge(mm, ss, sm.ms[w].x, sm.ms[w].y);
            p.part_ms[(size_t)row * p.max_pieces + slot] = make_float2(mm, ss);
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            const unsigned int t = atomicAdd(p.tickets + row, 1u);
            sm.flag = (t == (unsigned int)(pieces - 1));
        }
        __syncthreads();
        if (sm.flag) {
            // last piece of this row: merge every piece's list, then log Z in float64
            __threadfence();
            const uint64_t* src = p.part_keys + (size_t)row * p.max_pieces * KP;
            // fold the pieces in groups of kWarps: warp w loads piece base+w into sm.buf[w][0..KP), a tree merge
            // gathers the group in sm.buf[0], which then merges into the running result sm.res
            for (int base_i = 0; base_i < pieces; base_i += kWarps) {
                const int cnt = min(kWarps, pieces - base_i);
                if (warp < cnt) {
                    const uint64_t* sp = src + (size_t)(base_i + warp) * KP;
                    for (int e = lane; e < KP; e += 32) sm.buf[warp][e] = __ldcg(sp + e);
                }
                __syncthreads();
                for (int span = 1; span < cnt; span <<= 1) {
                    if ((warp % (2 * span)) == 0 && warp + span < cnt)
                        warp_merge_lists<KP>(sm.buf[warp], sm.buf[warp + span], sm.buf[warp]);
                    __syncthreads();
                }
                if (warp == 0) {
                    if (base_i == 0) {
                        for (int e = lane; e < KP; e += 32) sm.res[e] = sm.buf[0][e];
                    } else {
                        warp_merge_lists<KP>(sm.buf[0], sm.res, sm.res);
                    }
                }
                __syncthreads();
            }
            if (threadIdx.x == 0) {
                const float2* ms = p.part_ms + (size_t)row * p.max_pieces;
                double M = -INFINITY;
                for (int i = 0; i < pieces; ++i) {
                    const float2 v = __ldcg(ms + i);
                    if (v.y > 0.f) M = fmax(M, (double)v.x);
                }
                double S = 0.0;
                for (int i = 0; i < pieces; ++i) {
                    const float2 v = __ldcg(ms + i);
                    if (v.y > 0.f) S += (double)v.y * exp((double)v.x - M);
                }
                sm.logz = (M == -INFINITY) ? -INFINITY : (float)(M + log(S));
                p.tickets[row] = 0u;  // ready for the next launch
            }
            __syncthreads();
            write_outputs<CAP, KP>(p, row, sm.res, sm.logz);
        }
        __syncthreads();
    }
}

template <int CAP, int KP, bool BF16>
static int launch(const Params& p, int grid, cudaStream_t stream) {
    const size_t smem = sizeof(Smem<CAP, KP>);
    static_assert(KP + 128 <= CAP, "a compacted list plus one append round must fit in a warp buffer");
    auto kern = topk_logz_kernel<CAP, KP, BF16>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
        set_error("mfd_topk_logz: %s", cudaGetErrorString(e));
        return MFD_ERR_CUDA;
    }
    kern<<<grid, kThreads, smem, stream>>>(p);
    MFD_CHECK_LAUNCH("mfd_topk_logz");
    return MFD_OK;
}

static int sm_count() {
    int dev = 0, n = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

static int kp_for(int64_t k) {
    int kp = 1;
    while (kp < k) kp <<= 1;
    return kp < 32 ? 32 : kp;
}

struct Plan {
    int grid;
    int64_t per_cta;
    int max_pieces;
    int kp;
};

static Plan plan(int64_t rows, int64_t vocab, int64_t k) {
    Plan pl;
    const int64_t total = rows * vocab;
    const int ctas_per_sm = 4;
    int64_t grid = (int64_t)sm_count() * ctas_per_sm;
    const int64_t min_per = 8192;  // keep pieces long enough to amortise the merges
    if (grid * min_per > total) grid = (total + min_per - 1) / min_per;
    if (grid < 1) grid = 1;
    int64_t per = (total + grid - 1) / grid;
    per = (per + 7) / 8 * 8;
    grid = (total + per - 1) / per;
    pl.grid = (int)grid;
    pl.per_cta = per;
    pl.max_pieces = (int)((vocab + per - 1) / per + 1);
    pl.kp = kp_for(k);
    return pl;
}

}  // namespace topk
}  // namespace mfd

using namespace mfd;

extern "C" size_t mfd_topk_logz_workspace(int64_t rows, int64_t vocab, int64_t k) {
    if (rows <= 0 || vocab <= 0 || k <= 0) return 0;
    topk::Plan pl = topk::plan(rows, vocab, k);
    const size_t ms = (size_t)rows * pl.max_pieces * sizeof(float2);
    const size_t keys = (size_t)rows * pl.max_pieces * pl.kp * sizeof(uint64_t);
    const size_t tick = (size_t)rows * sizeof(unsigned int);
    return 256 + ((ms + 255) / 256) * 256 + ((keys + 255) / 256) * 256 + ((tick + 255) / 256) * 256;
}

extern "C" int mfd_topk_logz(const void* x, int x_dtype, int64_t rows, int64_t vocab, int64_t row_stride, int64_t k,
                             float* top_logp, void* top_ids, int ids_dtype, float* logz, void* workspace,
                             size_t workspace_bytes, void* stream) {
    if (rows < 0 || vocab <= 0 || k <= 0 || k > vocab || k > 256 || row_stride < vocab) {
        set_error("mfd_topk_logz: invalid sizes rows=%lld vocab=%lld k=%lld stride=%lld (need 0<k<=min(vocab,256))",
                  (long long)rows, (long long)vocab, (long long)k, (long long)row_stride);
        return MFD_ERR_INVALID;
    }
    if (x_dtype != MFD_F32 && x_dtype != MFD_BF16) {
        set_error("mfd_topk_logz: x_dtype must be MFD_F32 or MFD_BF16");
        return MFD_ERR_INVALID;
    }
    if (ids_dtype != MFD_I32 && ids_dtype != MFD_I64) {
        set_error("mfd_topk_logz: ids_dtype must be MFD_I32 or MFD_I64");
        return MFD_ERR_INVALID;
    }
    if (vocab >= (int64_t)0x7fffffff) {
        set_error("mfd_topk_logz: vocab must be < 2^31");
        return MFD_ERR_INVALID;
    }
    if (rows == 0) return MFD_OK;
    if (!x || !top_logp || !top_ids) {
        set_error("mfd_topk_logz: null pointer");
        return MFD_ERR_INVALID;
    }
    const size_t need = mfd_topk_logz_workspace(rows, vocab, k);
    if (!workspace || workspace_bytes < need) {
        set_error("mfd_topk_logz: workspace of %zu bytes needed (got %zu)", need, workspace_bytes);
        return MFD_ERR_INVALID;
    }
    topk::Plan pl = topk::plan(rows, vocab, k);
    char* ws = (char*)(((uintptr_t)workspace + 255) & ~(uintptr_t)255);
    topk::Params p;
    p.x = x;
    p.is_bf16 = x_dtype == MFD_BF16;
    p.rows = rows;
    p.vocab = vocab;
    p.row_stride = row_stride;
    p.k = (int)k;
    p.top_logp = top_logp;
    p.top_ids = top_ids;
    p.ids_i64 = ids_dtype == MFD_I64;
    p.logz = logz;
    p.per_cta = pl.per_cta;
    p.max_pieces = pl.max_pieces;
    const size_t ms = (size_t)rows * pl.max_pieces * sizeof(float2);
    const size_t keys = (size_t)rows * pl.max_pieces * pl.kp * sizeof(uint64_t);
    p.part_ms = (float2*)ws;
    ws += ((ms + 255) / 256) * 256;
    p.part_keys = (uint64_t*)ws;
    ws += ((keys + 255) / 256) * 256;
    p.tickets = (unsigned int*)ws;
    cudaStream_t st = (cudaStream_t)stream;
    const bool bf = p.is_bf16;
    switch (pl.kp) {
        case 32: return bf ? topk::launch<256, 32, true>(p, pl.grid, st) : topk::launch<256, 32, false>(p, pl.grid, st);
        case 64: return bf ? topk::launch<256, 64, true>(p, pl.grid, st) : topk::launch<256, 64, false>(p, pl.grid, st);
        case 128: return bf ? topk::launch<512, 128, true>(p, pl.grid, st) : topk::launch<512, 128, false>(p, pl.grid, st);
        case 256: return bf ? topk::launch<512, 256, true>(p, pl.grid, st) : topk::launch<512, 256, false>(p, pl.grid, st);
        default:
            set_error("mfd_topk_logz: unsupported k=%lld", (long long)k);
            return MFD_ERR_UNSUPPORTED;
    }
}
