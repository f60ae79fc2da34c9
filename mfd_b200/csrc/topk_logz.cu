// topk_logz.cu -- the logits step of tree construction: per row of draft logits, the top-k candidates
// (value descending, equal values by lower index first) and log Z = logsumexp(row), in ONE pass over HBM.
//
// Reference: inference/hf/ddtree.py:240-244 (float32 topk + logsumexp, then top - log_z),
// inference/hf/tree_logits.py:16-46 (bf16 top-k + one-pass online logsumexp), SGLang
// DDTreeDraftTopK / _row_logsumexp_kernel (sglang-v0.5.22-mfd.patch:1451-1550).
//
// Work split: the R x V element space is cut into equal contiguous ranges, 2 CTAs of 256 threads per SM (one
// wave).  A range may span a row boundary, so a CTA emits one partial record per row piece: (max, sum exp) and
// the piece's sorted top-k keys (64-bit: orderable value, then the complement of the index).
//
// Streaming (the hot loop) is register-only and software pipelined: every thread keeps eight 16-byte
// non-allocating loads in flight (each register slot is refilled from the next batch as soon as it is consumed), maintains an online (max, sum exp)
// with a lazy rescale, and tests each vector's maximum against ONE floor per piece (a compare and a warp vote);
// elements at or above the floor are appended, warp-aggregated, to a small per-warp buffer.  The floor comes
// from the piece's first batch: each warp sorts its 32 lane maxima, the CTA merges them, and the floor is the
// r-th largest lane maximum with r chosen so that about 2.5 k elements of the whole piece are expected to pass.
// That floor is speculative and is verified at the end of the piece: if at least k candidates were collected
// (and no buffer overflowed), every element of the piece's top k is among them -- an element below the floor has
// at least k collected elements above it.  Otherwise the piece is scanned again (an L2 hit) against a valid lower
// bound, the minimum over warps of each warp's ceil(k/8)-th largest lane maximum (the minimum of >= k distinct
// elements cannot exceed the k-th largest), so the result is exact either way.
// At the end of a piece the candidates are sorted by 8 warps in parallel and combined by bitonic merges.
#include "common.cuh"

namespace mfd {
namespace topk {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kCtasPerSm = 2;
constexpr int kLoads = 8;      // 16-byte loads per thread per batch (one batch in flight while one is processed)
constexpr int kCap = 2048;     // shared candidate buffer (keys)

// ------------------------------------------------------------------ warp sorting helpers

// Warp bitonic sort, descending, of 32*PER keys held as r[j] = element j*32 + lane.
template <int PER>
__device__ __forceinline__ void warp_sort_desc(uint64_t (&r)[PER]) {
    constexpr int N = PER * 32;
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int size = 2; size <= N; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= 32) {
                const int js = stride >> 5;
#pragma unroll
                for (int j = 0; j < PER; ++j) {
                    if ((j & js) == 0) {
                        const int e = j * 32 + lane;
                        const bool desc = (e & size) == 0;
                        const uint64_t a = r[j], b = r[j | js];
                        const bool sw = desc ? (a < b) : (a > b);
                        r[j] = sw ? b : a;
                        r[j | js] = sw ? a : b;
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < PER; ++j) {
                    const int e = j * 32 + lane;
                    const uint64_t o = shfl_xor_u64(r[j], stride);
                    const bool desc = (e & size) == 0;
                    const bool lower = (lane & stride) == 0;
                    const bool keep_max = (lower == desc);
                    r[j] = keep_max ? (r[j] > o ? r[j] : o) : (r[j] < o ? r[j] : o);
                }
            }
        }
    }
}

// Sort a bitonic sequence of 32*PER keys (layout as above) into descending order.
template <int PER>
__device__ __forceinline__ void warp_bitonic_merge_desc(uint64_t (&r)[PER]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int stride = PER * 16; stride > 0; stride >>= 1) {
        if (stride >= 32) {
            const int js = stride >> 5;
#pragma unroll
            for (int j = 0; j < PER; ++j) {
                if ((j & js) == 0) {
                    const uint64_t a = r[j], b = r[j | js];
                    r[j] = a > b ? a : b;
                    r[j | js] = a > b ? b : a;
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < PER; ++j) {
                const uint64_t o = shfl_xor_u64(r[j], stride);
                const bool lower = (lane & stride) == 0;
                r[j] = lower ? (r[j] > o ? r[j] : o) : (r[j] < o ? r[j] : o);
            }
        }
    }
}

// Merge two descending lists a, b of KP keys into the descending top KP (out may alias a or b).
template <int KP>
__device__ __forceinline__ void warp_merge_lists(const uint64_t* a, const uint64_t* b, uint64_t* out) {
    constexpr int PER = KP / 32;
    const int lane = threadIdx.x & 31;
    uint64_t r[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int e = j * 32 + lane;
        const uint64_t x = a[e], y = b[KP - 1 - e];
        r[j] = x > y ? x : y;  // the larger half of a bitonic concatenation
    }
    __syncwarp();
    warp_bitonic_merge_desc<PER>(r);
#pragma unroll
    for (int j = 0; j < PER; ++j) out[j * 32 + lane] = r[j];
    __syncwarp();
}

// ------------------------------------------------------------------ kernel state

struct Params {
    const void* x;
    int64_t rows, vocab, row_stride;  // in elements
    int k;
    float* top_logp;        // [rows, k]
    void* top_ids;          // [rows, k] int32 or int64
    int ids_i64;
    float* logz;            // [rows] or null
    int64_t per_cta;        // elements per CTA (multiple of 8)
    int max_pieces;         // partial-record slots per row
    float2* part_ms;        // [rows, max_pieces]
    uint64_t* part_keys;    // [rows, max_pieces, KP]
    unsigned int* tickets;  // [rows], zero between launches
};

constexpr int kWarpCap = 128;  // per-warp candidate buffer

template <int KP>
struct Smem {
    uint64_t cand[kCap];
    uint64_t wbuf[kWarps][kWarpCap];
    uint64_t lists[kWarps][KP];
    uint64_t res[KP];
    float2 ms[kWarps];
    float wthr[kWarps];
    int wcnt[kWarps];
    int count;
    int flag;
    int overflow;
    float floor_v;   // speculative floor (value)
    float bound_v;   // valid lower bound (value)
    float logz;
};

template <bool BF16>
__device__ __forceinline__ void unpack(const uint4& w, float (&x)[BF16 ? 8 : 4]) {
    if (BF16) {
        const uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            x[2 * q] = bf16lo(a[q]);
            x[2 * q + 1] = bf16hi(a[q]);
        }
    } else {
        x[0] = __uint_as_float(w.x);
        x[1] = __uint_as_float(w.y);
        x[2] = __uint_as_float(w.z);
        x[3] = __uint_as_float(w.w);
    }
}

// Online (max, sum) with a lazy rescale against the running maximum m (mL = m * log2 e).
template <int N>
__device__ __forceinline__ void lse_vec(float& m, float& mL, float& s, const float (&x)[N], float mx) {
    if (mx > m) {
        s = (m == -INFINITY) ? 0.f : s * fast_exp2((m - mx) * kLog2e);
        m = mx;
        mL = mx * kLog2e;
    }
    if (m == -INFINITY) return;
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) acc += fast_exp2(__fmaf_rn(x[j], kLog2e, -mL));
    s += acc;
}

// One pass over columns [c0, c1) of a row: thread t takes scalar head/tail element t and the 16-byte vectors
// t, t + 256, ... of the aligned body.  fn(x[VE], col0, live) per vector; scalars come as one live element.
template <bool BF16, class F>
__device__ __forceinline__ void scan_piece(const char* base, int64_t c0, int64_t c1, F&& fn) {
    constexpr int VE = BF16 ? 8 : 4;
    constexpr int ES = BF16 ? 2 : 4;
    int64_t hb = c0;
    {
        const uintptr_t ad = (uintptr_t)(base + c0 * ES);
        const int64_t mis = (int64_t)((ad & 15u) / ES);
        if (mis) hb = c0 + (VE - mis);
        if (hb > c1) hb = c1;
    }
    const int64_t nvec = (c1 - hb) / VE;
    const int64_t tb = hb + nvec * VE;
    {
        const int64_t nh = hb - c0, nt = c1 - tb, t = threadIdx.x;
        int64_t cs = -1;
        if (t < nh) cs = c0 + t;
        else if (t - nh < nt) cs = tb + (t - nh);
        if (cs >= 0) {
            float x[VE];
            x[0] = BF16 ? bf16_at((const uint16_t*)base + cs) : ((const float*)base)[cs];
#pragma unroll
            for (int e = 1; e < VE; ++e) x[e] = -INFINITY;
            fn(x, (uint32_t)cs, 1);
        }
    }
    const uint4* vb = (const uint4*)(base + hb * ES);
    for (int64_t v0 = 0; v0 < nvec; v0 += (int64_t)kThreads * kLoads) {
        uint4 w[kLoads];
#pragma unroll
        for (int u = 0; u < kLoads; ++u) {
            const int64_t vi = v0 + (int64_t)u * kThreads + threadIdx.x;
            if (vi < nvec) w[u] = ldg_stream_u4(vb + vi);
        }
#pragma unroll
        for (int u = 0; u < kLoads; ++u) {
            const int64_t vi = v0 + (int64_t)u * kThreads + threadIdx.x;
            if (vi < nvec) {
                float x[VE];
                unpack<BF16>(w[u], x);
                fn(x, (uint32_t)(hb + vi * VE), VE);
            }
        }
    }
}

// CTA: the descending top KP (zero-padded) of the n keys in sm.cand into sm.res.  Each warp sorts a chunk of
// 32*PER keys; the chunk lists combine by a tree of warp merges.
template <int KP, int PER>
__device__ __forceinline__ void select_chunks(Smem<KP>& sm, int n) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int CH = 32 * PER;
    uint64_t r[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int e = warp * CH + j * 32 + lane;
        r[j] = e < n ? sm.cand[e] : 0ull;
    }
    warp_sort_desc<PER>(r);
#pragma unroll
    for (int j = 0; j < KP / 32; ++j) sm.lists[warp][j * 32 + lane] = j < PER ? r[j < PER ? j : 0] : 0ull;
    __syncthreads();
#pragma unroll
    for (int span = 1; span < kWarps; span <<= 1) {
        if ((warp % (2 * span)) == 0) warp_merge_lists<KP>(sm.lists[warp], sm.lists[warp + span], sm.lists[warp]);
        __syncthreads();
    }
    for (int e = threadIdx.x; e < KP; e += kThreads) sm.res[e] = sm.lists[0][e];
    __syncthreads();
}

template <int KP>
__device__ __noinline__ void select_topk(Smem<KP>& sm, int n) {
    if (n <= kWarps * 32) {
        select_chunks<KP, 1>(sm, n);
    } else if (n <= kWarps * 64) {
        select_chunks<KP, 2>(sm, n);
    } else if (n <= kWarps * 128) {
        select_chunks<KP, 4>(sm, n);
    } else {
        select_chunks<KP, 8>(sm, n);  // n <= kCap = 2048
    }
}

// Append key if `take`; warp-aggregated slot, the caller guarantees room.
__device__ __forceinline__ void cta_append(int* count, uint64_t* cand, bool take, uint64_t key) {
    const int lane = threadIdx.x & 31;
    const uint32_t bal = __ballot_sync(MFD_FULL_MASK, take);
    if (!bal) return;
    const int leader = __ffs(bal) - 1;
    int base = 0;
    if (lane == leader) base = atomicAdd(count, __popc(bal));
    base = __shfl_sync(MFD_FULL_MASK, base, leader);
    if (take) cand[base + __popc(bal & ((1u << lane) - 1u))] = key;
}

template <int KP>
__device__ __forceinline__ void write_outputs(const Params& p, int64_t row, const uint64_t* keys, float logz) {
    for (int e = threadIdx.x; e < p.k; e += kThreads) {
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

// Rare: scan the piece for every element at or above the value floor `vf` (then every key above the running
// k-th best) into sm.cand and select; repeated with the improved k-th best while more than kCap keys qualify.
template <int KP, bool BF16>
__device__ __noinline__ void rescan_select(Smem<KP>& sm, const char* base, int64_t c0, int64_t c1, float vf,
                                           int k) {
    uint64_t thr = 0ull;
    constexpr int VE = BF16 ? 8 : 4;
    for (;;) {
        if (threadIdx.x == 0) sm.count = 0;
        __syncthreads();
        int overflow = 0;
        scan_piece<BF16>(base, c0, c1, [&](const float (&x)[VE], uint32_t col0, int live) {
#pragma unroll
            for (int e = 0; e < VE; ++e) {
                if (e < live && x[e] >= vf) {
                    const uint64_t key = topk_key(x[e], col0 + e);
                    if (key > thr) {
                        const int slot = atomicAdd(&sm.count, 1);
                        if (slot < kCap) sm.cand[slot] = key;
                        else overflow = 1;
                    }
                }
            }
        });
        __syncthreads();
        const int of = __syncthreads_or(overflow);
        const int n = of ? kCap : sm.count;
        select_topk<KP>(sm, n);
        if (!of) return;
        thr = sm.res[k - 1];  // the k-th best of kCap qualifying keys: a valid, higher threshold
    }
}

template <int KP, bool BF16>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) topk_logz_kernel(const Params p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem<KP>& sm = *reinterpret_cast<Smem<KP>*>(smem_raw);
    constexpr int VE = BF16 ? 8 : 4;
    constexpr int ES = BF16 ? 2 : 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int k = p.k;
    const int64_t total = p.rows * p.vocab;
    const int64_t a = (int64_t)blockIdx.x * p.per_cta;
    const int64_t b = a + p.per_cta < total ? a + p.per_cta : total;
    if (a >= b) return;
    for (int64_t row = a / p.vocab; row * p.vocab < b; ++row) {
        const int64_t r0 = row * p.vocab;
        const int64_t c0 = a > r0 ? a - r0 : 0;
        const int64_t c1 = (b < r0 + p.vocab ? b : r0 + p.vocab) - r0;
        const char* base = (const char*)p.x + (size_t)row * p.row_stride * ES;

        // ---- the streaming pass
        constexpr int kBatch = kThreads * kLoads;  // vectors per batch
        float m = -INFINITY, mL = -INFINITY, s = 0.f;
        float lmax = -INFINITY;  // lane maximum over the head/tail scalar and the first batch
        int wcnt = 0;            // this warp's buffered candidates (warp-uniform)
        bool wover = false;      // this warp's buffer overflowed
        uint64_t* wb = sm.wbuf[warp];
        int64_t hb = c0;
        {
            const uintptr_t ad = (uintptr_t)(base + c0 * ES);
            const int64_t mis = (int64_t)((ad & 15u) / ES);
            if (mis) hb = c0 + (VE - mis);
            if (hb > c1) hb = c1;
        }
        const int64_t nvec = (c1 - hb) / VE;
        const int64_t tb = hb + nvec * VE;
        const uint4* vb = (const uint4*)(base + hb * ES);
        const int64_t nbatch = (nvec + kBatch - 1) / kBatch;
        // warp-aggregated append of the elements of x[0..live) at or above fl
        auto offer = [&](const float (&x)[VE], uint32_t col0, int live, float fl) {
#pragma unroll
            for (int e = 0; e < VE; ++e) {
                const bool take = e < live && x[e] >= fl;
                const uint32_t bal = __ballot_sync(MFD_FULL_MASK, take);
                if (bal) {
                    const int slot = wcnt + __popc(bal & ((1u << lane) - 1u));
                    if (take && slot < kWarpCap) wb[slot] = topk_key(x[e], col0 + e);
                    wcnt += __popc(bal);
                }
            }
            if (wcnt > kWarpCap) wover = true;
        };
        // head/tail scalar of this thread
        float xs[VE];
        int64_t cs = -1;
        {
            const int64_t nh = hb - c0, nt = c1 - tb, t = threadIdx.x;
            if (t < nh) cs = c0 + t;
            else if (t - nh < nt) cs = tb + (t - nh);
#pragma unroll
            for (int e = 0; e < VE; ++e) xs[e] = -INFINITY;
            if (cs >= 0) xs[0] = BF16 ? bf16_at((const uint16_t*)base + cs) : ((const float*)base)[cs];
            lse_vec<VE>(m, mL, s, xs, xs[0]);
            lmax = xs[0];
        }
        // w[] holds one batch; after the floors, each slot is refilled with the next batch's vector as soon as it
        // has been consumed, so a batch of loads is always in flight
        uint4 w[kLoads];
#pragma unroll
        for (int u = 0; u < kLoads; ++u) {
            const int64_t vi = (int64_t)u * kThreads + threadIdx.x;
            if (vi < nvec) w[u] = ldg_stream_u4(vb + vi);
        }
        // first batch: (max, sum) and the lane maximum
        if (nbatch > 0) {
#pragma unroll
            for (int u = 0; u < kLoads; ++u) {
                const int64_t vi = (int64_t)u * kThreads + threadIdx.x;
                if (vi < nvec) {
                    float x[VE];
                    unpack<BF16>(w[u], x);
                    float mx = x[0];
#pragma unroll
                    for (int e = 1; e < VE; ++e) mx = fmaxf(mx, x[e]);
                    lse_vec<VE>(m, mL, s, x, mx);
                    lmax = fmaxf(lmax, mx);
                }
            }
        }
        // floors: each warp sorts its lane maxima; the speculative floor is the r-th largest over the CTA and the
        // valid bound the minimum over warps of each warp's ceil(k/8)-th largest
        {
            const int64_t sample = min(nvec, (int64_t)kBatch) * VE + (hb - c0) + (c1 - tb);
            const int64_t np = c1 - c0;
            int r = (int)((5LL * k * sample + 2 * np - 1) / (2 * np));
            r = max(r, 1);
            uint64_t r1[1] = {(uint64_t)ord_f32(lmax) << 32};
            warp_sort_desc<1>(r1);
            const int q = (k + kWarps - 1) / kWarps;
            const uint64_t qth = shfl_u64(r1[0], q - 1);
            if (lane == 0) sm.wthr[warp] = unord_f32((uint32_t)(qth >> 32));
            // the warp's sorted lane maxima as a list of KP (zero padded) for the CTA merge
#pragma unroll
            for (int j = 0; j < KP / 32; ++j) sm.lists[warp][j * 32 + lane] = j == 0 ? r1[0] : 0ull;
            __syncthreads();
#pragma unroll
            for (int span = 1; span < kWarps; span <<= 1) {
                if ((warp % (2 * span)) == 0) warp_merge_lists<KP>(sm.lists[warp], sm.lists[warp + span], sm.lists[warp]);
                __syncthreads();
            }
            if (threadIdx.x == 0) {
                float bv = INFINITY;
                for (int w = 0; w < kWarps; ++w) bv = fminf(bv, sm.wthr[w]);
                sm.bound_v = bv;
                // r-th largest lane maximum; r beyond the list (or beyond the lanes) -> no speculation
                sm.floor_v = (r <= KP && r <= kThreads && sm.lists[0][r - 1] != 0ull)
                                 ? fmaxf(bv, unord_f32((uint32_t)(sm.lists[0][r - 1] >> 32)))
                                 : bv;
                sm.overflow = 0;
            }
            __syncthreads();
        }
        const float fl = sm.floor_v;
        // the head/tail scalar and the first batch against the floor
        offer(xs, (uint32_t)(cs >= 0 ? cs : 0), cs >= 0 ? 1 : 0, fl);
        if (nbatch > 0) {
#pragma unroll
            for (int u = 0; u < kLoads; ++u) {
                const int64_t vi = (int64_t)u * kThreads + threadIdx.x;
                float x[VE];
                unpack<BF16>(w[u], x);
                float mx = x[0];
#pragma unroll
                for (int e = 1; e < VE; ++e) mx = fmaxf(mx, x[e]);
                if (__any_sync(MFD_FULL_MASK, vi < nvec && mx >= fl)) offer(x, (uint32_t)(hb + vi * VE), vi < nvec ? VE : 0, fl);
                const int64_t vn = vi + kBatch;  // the next batch's vector into the freed slot
                if (vn < nvec) w[u] = ldg_stream_u4(vb + vn);
            }
        }
        // the remaining batches, each slot refilled from two batches ahead as it is consumed
        for (int64_t bt = 1; bt < nbatch; ++bt) {
#pragma unroll
            for (int u = 0; u < kLoads; ++u) {
                const int64_t vi = bt * kBatch + (int64_t)u * kThreads + threadIdx.x;
                const bool ok = vi < nvec;
                float x[VE];
                unpack<BF16>(w[u], x);
                const int64_t vn = vi + kBatch;
                if (vn < nvec) w[u] = ldg_stream_u4(vb + vn);
                float mx = x[0];
#pragma unroll
                for (int e = 1; e < VE; ++e) mx = fmaxf(mx, x[e]);
                if (ok) lse_vec<VE>(m, mL, s, x, mx);
                if (__any_sync(MFD_FULL_MASK, ok && mx >= fl)) offer(x, (uint32_t)(hb + vi * VE), ok ? VE : 0, fl);
            }
        }

        // ---- the piece's (max, sum)
        {
            float mm = m, ss = s;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float m2 = __shfl_xor_sync(MFD_FULL_MASK, mm, o);
                const float s2 = __shfl_xor_sync(MFD_FULL_MASK, ss, o);
                lse_merge(mm, ss, m2, s2);
            }
            if (lane == 0) {
                sm.ms[warp] = make_float2(mm, ss);
                sm.wcnt[warp] = wcnt < kWarpCap ? wcnt : kWarpCap;
                if (wover) sm.overflow = 1;
            }
        }
        __syncthreads();

        // ---- gather the warp buffers; verify the speculative floor; select the top KP
        int n = 0, off = 0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            if (w < warp) off += sm.wcnt[w];
            n += sm.wcnt[w];
        }
        for (int i = lane; i < sm.wcnt[warp]; i += 32) sm.cand[off + i] = wb[i];
        __syncthreads();
        if (sm.overflow || n < k) {
            rescan_select<KP, BF16>(sm, base, c0, c1, sm.bound_v, k);
        } else {
            select_topk<KP>(sm, n);
        }

        // ---- publish this piece
        const int64_t first_cta = r0 / p.per_cta;
        const int64_t last_cta = (r0 + p.vocab - 1) / p.per_cta;
        const int pieces = (int)(last_cta - first_cta + 1);
        const int slot = (int)(blockIdx.x - first_cta);
        if (pieces == 1) {
            if (threadIdx.x == 0) {
                float mm = -INFINITY, ss = 0.f;
                for (int w = 0; w < kWarps; ++w) lse_merge(mm, ss, sm.ms[w].x, sm.ms[w].y);
                sm.logz = (mm == -INFINITY) ? -INFINITY : (float)((double)mm + log((double)ss));
            }
            __syncthreads();
            write_outputs<KP>(p, row, sm.res, sm.logz);
            __syncthreads();
            continue;
        }
        uint64_t* dst = p.part_keys + ((size_t)row * p.max_pieces + slot) * KP;
        for (int e = threadIdx.x; e < KP; e += kThreads) dst[e] = sm.res[e];
        if (threadIdx.x == 0) {
            float mm = -INFINITY, ss = 0.f;
            for (int w = 0; w < kWarps; ++w) lse_merge(mm, ss, sm.ms[w].x, sm.ms[w].y);
            p.part_ms[(size_t)row * p.max_pieces + slot] = make_float2(mm, ss);
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            const unsigned int tk = atomicAdd(p.tickets + row, 1u);
            sm.flag = (tk == (unsigned int)(pieces - 1));
        }
        __syncthreads();
        if (sm.flag) {
            // last piece of this row: merge every piece's list (in groups of kWarps), then log Z in float64
            __threadfence();
            const uint64_t* src = p.part_keys + (size_t)row * p.max_pieces * KP;
            for (int base_i = 0; base_i < pieces; base_i += kWarps) {
                const int cnt = min(kWarps, pieces - base_i);
                if (warp < cnt) {
                    const uint64_t* sp = src + (size_t)(base_i + warp) * KP;
                    for (int e = lane; e < KP; e += 32) sm.lists[warp][e] = __ldcg(sp + e);
                }
                __syncthreads();
                for (int span = 1; span < cnt; span <<= 1) {
                    if ((warp % (2 * span)) == 0 && warp + span < cnt)
                        warp_merge_lists<KP>(sm.lists[warp], sm.lists[warp + span], sm.lists[warp]);
                    __syncthreads();
                }
                if (warp == 0) {
                    if (base_i == 0) {
                        for (int e = lane; e < KP; e += 32) sm.res[e] = sm.lists[0][e];
                        __syncwarp();
                    } else {
                        warp_merge_lists<KP>(sm.lists[0], sm.res, sm.res);
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
            write_outputs<KP>(p, row, sm.res, sm.logz);
        }
        __syncthreads();
    }
}

template <int KP, bool BF16>
static int launch(const Params& p, int grid, cudaStream_t stream) {
    const size_t smem = sizeof(Smem<KP>);
    auto kern = topk_logz_kernel<KP, BF16>;
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
    int kp = 32;
    while (kp < k) kp <<= 1;
    return kp;
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
    int64_t grid = (int64_t)sm_count() * kCtasPerSm;
    const int64_t min_per = 8192;
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
    return 256 + ((ms + 255) / 256) * 256 + keys;
}

extern "C" int mfd_topk_logz(const void* x, int x_dtype, int64_t rows, int64_t vocab, int64_t row_stride, int64_t k,
                             float* top_logp, void* top_ids, int ids_dtype, float* logz, void* workspace,
                             size_t workspace_bytes, unsigned int* tickets, int64_t tickets_len, void* stream) {
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
    if (!tickets || tickets_len < rows) {
        set_error("mfd_topk_logz: a zeroed ticket buffer of %lld words is needed", (long long)rows);
        return MFD_ERR_INVALID;
    }
    topk::Plan pl = topk::plan(rows, vocab, k);
    char* ws = (char*)(((uintptr_t)workspace + 255) & ~(uintptr_t)255);
    topk::Params p;
    p.x = x;
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
    p.part_ms = (float2*)ws;
    ws += ((ms + 255) / 256) * 256;
    p.part_keys = (uint64_t*)ws;
    p.tickets = tickets;
    cudaStream_t st = (cudaStream_t)stream;
    const bool bf = x_dtype == MFD_BF16;
    switch (pl.kp) {
        case 32: return bf ? topk::launch<32, true>(p, pl.grid, st) : topk::launch<32, false>(p, pl.grid, st);
        case 64: return bf ? topk::launch<64, true>(p, pl.grid, st) : topk::launch<64, false>(p, pl.grid, st);
        case 128: return bf ? topk::launch<128, true>(p, pl.grid, st) : topk::launch<128, false>(p, pl.grid, st);
        case 256: return bf ? topk::launch<256, true>(p, pl.grid, st) : topk::launch<256, false>(p, pl.grid, st);
        default:
            set_error("mfd_topk_logz: unsupported k=%lld", (long long)k);
            return MFD_ERR_UNSUPPORTED;
    }
}
