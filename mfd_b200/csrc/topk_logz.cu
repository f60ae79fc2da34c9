// topk_logz.cu -- the logits step of tree construction: per row of draft logits, the top-k candidates
// (value descending, equal values by lower index first) and log Z = logsumexp(row), in ONE pass over HBM.
//
// Reference: inference/hf/ddtree.py:240-244 (float32 topk + logsumexp, then top - log_z),
// inference/hf/tree_logits.py:16-46 (bf16 top-k + one-pass online logsumexp), SGLang
// DDTreeDraftTopK / _row_logsumexp_kernel (sglang-v0.5.22-mfd.patch:1451-1550).
//
// Work split: 2 CTAs of 256 threads per SM (one wave), and no CTA's range crosses a row.  With at least as many
// rows as CTAs each CTA takes a balanced run of whole rows; with fewer, each row is cut into equal pieces, one per
// CTA, which emit partial records -- (max, sum exp) and the piece's sorted top-k keys (64-bit: orderable value,
// then the complement of the index) -- merged by the row's last CTA.
//
// Streaming (the hot loop) is register-only and software pipelined: every thread keeps eight 16-byte
// non-allocating loads in flight (the slots of a group are refilled from the next batch as soon as the group is
// unpacked).  Per group of 32 elements a thread takes ONE maximum, tests it against ONE floor per piece, makes ONE
// lazy-rescale check of its online (max, sum exp) and adds the 32 exponentials as a tree.  A thread whose group
// reaches the floor (rare) appends those elements with shared atomics to the CTA's candidate buffer.  The floor
// comes from the piece's first batch: each warp sorts its 32 lane maxima and the floor is the r-th largest over
// the CTA, found by rank, with r chosen so that about 3.5 k elements of the whole piece are expected to pass (a
// lower target sorts fewer candidates but fails the verification below more often, and a rescan costs more).  A
// second, upper floor (about 2 k expected) is found by the same rank search: when more candidates than one per
// thread were collected and at least k of them reach it, only those are sorted (one selection pass instead of two).
// That floor is speculative and is verified at the end of the piece: if at least k candidates were collected
// (and the buffer did not overflow), every element of the piece's top k is among them -- an element below the
// floor has at least k collected elements above it.  Otherwise the piece is scanned again (an L2 hit) against a
// valid lower bound, the minimum over warps of each warp's ceil(k/8)-th largest lane maximum (the minimum of >= k
// distinct elements cannot exceed the k-th largest), so the result is exact either way.
// At the end of a piece each warp sorts a chunk of the candidates and every key finds its rank by binary searches
// in the other chunks; the keys ranked below k are the piece's sorted top k.
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
    int pieces_per_row;     // P > 1: CTA c takes piece c % P of row c / P; P = 1: CTA c takes whole rows
    int64_t piece_len;      // elements per piece when P > 1 (a multiple of 8)
    int max_pieces;         // partial-record slots per row (= P)
    float2* part_ms;        // [rows, max_pieces]
    uint64_t* part_keys;    // [rows, max_pieces, KP]
    unsigned int* tickets;  // [rows], zero between launches
};


template <int KP>
struct Smem {
    uint64_t cand[kCap];
    uint64_t lists[kWarps][KP];
    uint64_t res[KP];
    float2 ms[kWarps];
    float wthr[kWarps];
    int count;
    int count_hi;
    int flag;
    int spec;        // a speculative floor was found
    float floor_v;   // speculative floor (value)
    int spec_hi;     // an upper speculative floor was found
    float floor_hi;  // upper speculative floor (value)
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

// Number of keys greater than `key` in the descending list c[0..CH) (binary search; CH a power of two).
template <int CH>
__device__ __forceinline__ int count_greater(const uint64_t* c, uint64_t key) {
    int pos = 0;
#pragma unroll
    for (int step = CH / 2; step > 0; step >>= 1)
        if (c[pos + step - 1] > key) pos += step;
    return pos + (c[pos] > key ? 1 : 0);
}

// CTA: the descending top KP (zero-padded) of the n distinct keys in sm.cand into sm.res.  Each warp sorts a
// chunk of 32*PER keys in registers and writes it back sorted; a key's rank is its position in its own chunk
// plus, for every other chunk, the number of keys there above it (a binary search).  Keys ranked below KP are
// stored at their rank.
template <int KP, int PER>
__device__ __forceinline__ void select_rank(Smem<KP>& sm, int n) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int CH = 32 * PER;
    uint64_t r[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int e = warp * CH + j * 32 + lane;
        r[j] = e < n ? sm.cand[e] : 0ull;
    }
    warp_sort_desc<PER>(r);
    __syncwarp();
#pragma unroll
    for (int j = 0; j < PER; ++j) sm.cand[warp * CH + j * 32 + lane] = r[j];
    for (int e = threadIdx.x; e < KP; e += kThreads)
        if (e >= n) sm.res[e] = 0ull;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        if (j * 32 >= KP) break;  // own position alone already >= KP
        const uint64_t key = r[j];
        if (key == 0ull) continue;
        int rank = j * 32 + lane;
#pragma unroll
        for (int w2 = 0; w2 < kWarps; ++w2)
            if (w2 != warp) rank += count_greater<CH>(sm.cand + w2 * CH, key);
        if (rank < KP) sm.res[rank] = key;
    }
    __syncthreads();
}

// inlined: the next row's first loads are in flight across it, and a call would have to save their registers
template <int KP>
__device__ __forceinline__ void select_topk(Smem<KP>& sm, int n) {
    if (n <= kWarps * 32) {
        select_rank<KP, 1>(sm, n);
    } else if (n <= kWarps * 64) {
        select_rank<KP, 2>(sm, n);
    } else if (n <= kWarps * 128) {
        select_rank<KP, 4>(sm, n);
    } else {
        select_rank<KP, 8>(sm, n);  // n <= kCap = 2048
    }
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

// Rare: scan the piece for every element at or above the value floor `vf` (then every key at or above the
// running k-th best) into sm.cand and select; repeated with the improved k-th best while more than kCap keys
// qualify.  The k-th best of kCap qualifying keys is itself a key of the piece, so at least k keys are at or above
// it; when every one of a full buffer's keys qualifies again, its k-th best is strictly higher, so the loop ends.
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
                    if (key >= thr) {
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
    // the CTA's pieces never cross a row: one piece of one row (P > 1), or a balanced run of whole rows
    const int P = p.pieces_per_row;
    int64_t row_begin, row_end, cc0 = 0, cc1 = p.vocab;
    int piece = 0;
    if (P > 1) {
        row_begin = blockIdx.x / P;
        row_end = row_begin + 1;
        piece = (int)(blockIdx.x % P);
        cc0 = (int64_t)piece * p.piece_len;
        cc1 = cc0 + p.piece_len < p.vocab ? cc0 + p.piece_len : p.vocab;
    } else {
        row_begin = (int64_t)blockIdx.x * p.rows / gridDim.x;
        row_end = (int64_t)(blockIdx.x + 1) * p.rows / gridDim.x;
    }
    if (row_begin >= p.rows || cc0 >= cc1) return;
    constexpr int kBatch = kThreads * kLoads;  // vectors per batch
    // the geometry of a row's piece: aligned body [hb, tb) as nvec 16-byte vectors, head / tail scalars outside it
    auto geometry = [&](int64_t row, const char*& base, int64_t& hb, int64_t& nvec, int64_t& tb) {
        base = (const char*)p.x + (size_t)row * p.row_stride * ES;
        hb = cc0;
        const uintptr_t ad = (uintptr_t)(base + cc0 * ES);
        const int64_t mis = (int64_t)((ad & 15u) / ES);
        if (mis) hb = cc0 + (VE - mis);
        if (hb > cc1) hb = cc1;
        nvec = (cc1 - hb) / VE;
        tb = hb + nvec * VE;
    };
    // the first batch and the head/tail scalar of a row, issued before the previous row's select when possible
    uint4 w[kLoads];
    float xs0 = -INFINITY;
    int64_t cs = -1;
    auto first_loads = [&](int64_t row) {
        const char* bse;
        int64_t hb_, nv_, tb_;
        geometry(row, bse, hb_, nv_, tb_);
        const uint4* vb_ = (const uint4*)(bse + hb_ * ES);
#pragma unroll
        for (int u = 0; u < kLoads; ++u) {
            const int64_t vi = (int64_t)u * kThreads + threadIdx.x;
            if (vi < nv_) w[u] = ldg_stream_u4(vb_ + vi);
        }
        const int64_t nh = hb_ - cc0, nt = cc1 - tb_, t = threadIdx.x;
        cs = -1;
        if (t < nh) cs = cc0 + t;
        else if (t - nh < nt) cs = tb_ + (t - nh);
        xs0 = -INFINITY;
        if (cs >= 0) xs0 = BF16 ? bf16_at((const uint16_t*)bse + cs) : ((const float*)bse)[cs];
    };
    first_loads(row_begin);
    for (int64_t row = row_begin; row < row_end; ++row) {
        const int64_t c0 = cc0, c1 = cc1;
        const char* base;

        // ---- the streaming pass
        float m = -INFINITY, mL = -INFINITY, s = 0.f;
        float lmax = -INFINITY;  // lane maximum over the head/tail scalar and the first batch
        int64_t hb, nvec, tb;
        geometry(row, base, hb, nvec, tb);
        const uint4* vb = (const uint4*)(base + hb * ES);
        const int64_t nbatch = (nvec + kBatch - 1) / kBatch;
        // append the elements of x[0..live) at or above fl to the CTA's candidates (a lane that has some works
        // alone: shared atomics, no warp collective; a count past kCap marks the overflow)
        auto offer = [&](const float (&x)[VE], uint32_t col0, int live, float fl) {
#pragma unroll
            for (int e = 0; e < VE; ++e) {
                if (e < live && x[e] >= fl) {
                    const int slot = atomicAdd(&sm.count, 1);
                    if (slot < kCap) sm.cand[slot] = topk_key(x[e], col0 + e);
                }
            }
        };
        // head/tail scalar of this thread (loaded with the first batch)
        float xs[VE];
        {
#pragma unroll
            for (int e = 0; e < VE; ++e) xs[e] = -INFINITY;
            xs[0] = xs0;
            lse_vec<VE>(m, mL, s, xs, xs[0]);
            lmax = xs[0];
        }
        // w[] holds one batch (the first one issued before the previous row's select); after the floors, each slot
        // is refilled with the next batch's vector as soon as it has been consumed
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
        float bv = -INFINITY, fl = -INFINITY;
        // floors: each warp sorts its lane maxima (made distinct by the thread index); the speculative floor is the
        // r-th largest over the CTA (found by rank, as in select_rank) and the valid bound the minimum over warps of
        // each warp's ceil(k/8)-th largest
        {
            const int64_t sample = min(nvec, (int64_t)kBatch) * VE + (hb - c0) + (c1 - tb);
            const int64_t np = c1 - c0;
            // two speculative floors: about 3.5 k and 2 k expected elements of the piece at or above them
            int r = (int)((7LL * k * sample + 2 * np - 1) / (2 * np));
            r = max(r, 1);
            const int r_hi = max((int)((2LL * k * sample + np - 1) / np), 1);
            uint64_t r1[1] = {((uint64_t)ord_f32(lmax) << 32) | (uint64_t)(~(uint32_t)threadIdx.x)};
            warp_sort_desc<1>(r1);
            const int q = (k + kWarps - 1) / kWarps;
            const uint64_t qth = shfl_u64(r1[0], q - 1);
            if (lane == 0) sm.wthr[warp] = unord_f32((uint32_t)(qth >> 32));
            sm.cand[threadIdx.x] = r1[0];  // (the candidate buffer is free until the floors are known)
            if (threadIdx.x == 0) {
                sm.spec = 0;
                sm.spec_hi = 0;
                sm.count = 0;
                sm.count_hi = 0;
            }
            __syncthreads();
            if (r <= kThreads) {
                int rank = lane;
#pragma unroll
                for (int w2 = 0; w2 < kWarps; ++w2)
                    if (w2 != warp) rank += count_greater<32>(sm.cand + w2 * 32, r1[0]);
                if (rank == r - 1) {
                    sm.floor_v = unord_f32((uint32_t)(r1[0] >> 32));
                    sm.spec = 1;
                }
                if (rank == r_hi - 1) {
                    sm.floor_hi = unord_f32((uint32_t)(r1[0] >> 32));
                    sm.spec_hi = 1;
                }
            }
            __syncthreads();
            bv = sm.wthr[0];
#pragma unroll
            for (int w2 = 1; w2 < kWarps; ++w2) bv = fminf(bv, sm.wthr[w2]);
            fl = sm.spec ? fmaxf(bv, sm.floor_v) : bv;
            __syncthreads();  // every thread has read the floors (and the buffer is free for candidates)
        }
        // the head/tail scalar and the first batch against the floor
        if (cs >= 0 && xs[0] >= fl) offer(xs, (uint32_t)cs, 1, fl);
        if (nbatch > 0) {
#pragma unroll
            for (int u = 0; u < kLoads; ++u) {
                const int64_t vi = (int64_t)u * kThreads + threadIdx.x;
                float x[VE];
                unpack<BF16>(w[u], x);
                float mx = x[0];
#pragma unroll
                for (int e = 1; e < VE; ++e) mx = fmaxf(mx, x[e]);
                if (vi < nvec && mx >= fl) offer(x, (uint32_t)(hb + vi * VE), VE, fl);
                const int64_t vn = vi + kBatch;  // the next batch's vector into the freed slot
                if (vn < nvec) w[u] = ldg_stream_u4(vb + vn);
            }
        }
        // the remaining batches, in groups of 32 elements per thread (the whole batch in float32, half of it in
        // bf16): a group's vectors are unpacked and their slots refilled with the next batch at once, then ONE
        // maximum, ONE floor test, ONE lazy-rescale check and a tree sum of the exponentials per group
        constexpr int kGroup = 32 / VE;  // vectors per group
        static_assert(kLoads % kGroup == 0, "whole groups per batch");
        const int64_t nfull = nvec / kBatch;
        const uint4* pb = vb + threadIdx.x;
        for (int64_t bt = 1; bt < nbatch; ++bt) {
            pb += kBatch;
            const bool full = bt < nfull, next_full = bt + 1 < nfull;
#pragma unroll
            for (int g0 = 0; g0 < kLoads; g0 += kGroup) {
                float x[kGroup][VE];
#pragma unroll
                for (int u = 0; u < kGroup; ++u) unpack<BF16>(w[g0 + u], x[u]);
#pragma unroll
                for (int u = 0; u < kGroup; ++u) {
                    const int uu = g0 + u;
                    if (next_full || (bt + 1) * kBatch + uu * kThreads + threadIdx.x < nvec)
                        w[uu] = ldg_stream_u4(pb + kBatch + uu * kThreads);
                }
                if (!full) {  // vectors past the piece read as -inf
#pragma unroll
                    for (int u = 0; u < kGroup; ++u)
                        if (bt * kBatch + (g0 + u) * kThreads + threadIdx.x >= nvec) {
#pragma unroll
                            for (int e = 0; e < VE; ++e) x[u][e] = -INFINITY;
                        }
                }
                float vm[kGroup];
#pragma unroll
                for (int u = 0; u < kGroup; ++u) {
                    float t[VE];
#pragma unroll
                    for (int e = 0; e < VE; ++e) t[e] = x[u][e];
#pragma unroll
                    for (int h = VE / 2; h > 0; h >>= 1)
#pragma unroll
                        for (int e = 0; e < h; ++e) t[e] = fmaxf(t[e], t[e + h]);
                    vm[u] = t[0];
                }
                float bmx = vm[0];
#pragma unroll
                for (int u = 1; u < kGroup; ++u) bmx = fmaxf(bmx, vm[u]);
                if (bmx >= fl) {  // rare; vectors past the piece are excluded explicitly (fl may be -inf)
#pragma unroll
                    for (int u = 0; u < kGroup; ++u) {
                        const int64_t vi = bt * kBatch + (int64_t)(g0 + u) * kThreads + threadIdx.x;
                        if (vi < nvec && vm[u] >= fl) offer(x[u], (uint32_t)(hb + vi * VE), VE, fl);
                    }
                }
                if (bmx > m) {
                    s = (m == -INFINITY) ? 0.f : s * fast_exp2((m - bmx) * kLog2e);
                    m = bmx;
                    mL = bmx * kLog2e;
                }
                if (m != -INFINITY) {
                    float acc[kGroup];
#pragma unroll
                    for (int u = 0; u < kGroup; ++u) {
                        float t[VE];
#pragma unroll
                        for (int e = 0; e < VE; ++e) t[e] = fast_exp2(__fmaf_rn(x[u][e], kLog2e, -mL));
#pragma unroll
                        for (int h = VE / 2; h > 0; h >>= 1)
#pragma unroll
                            for (int e = 0; e < h; ++e) t[e] += t[e + h];
                        acc[u] = t[0];
                    }
#pragma unroll
                    for (int h = kGroup / 2; h > 0; h >>= 1)
#pragma unroll
                        for (int u = 0; u < h; ++u) acc[u] += acc[u + h];
                    s += acc[0];
                }
            }
        }

        if (row + 1 < row_end) first_loads(row + 1);  // in flight during this row's select and publish
        // ---- the piece's (max, sum)
        {
            float mm = m, ss = s;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float m2 = __shfl_xor_sync(MFD_FULL_MASK, mm, o);
                const float s2 = __shfl_xor_sync(MFD_FULL_MASK, ss, o);
                lse_merge(mm, ss, m2, s2);
            }
            if (lane == 0) sm.ms[warp] = make_float2(mm, ss);
        }
        __syncthreads();

        // ---- verify the speculative floor; select the top KP
        int cnt = sm.count;
        const float fl_hi = sm.spec_hi ? fmaxf(fl, sm.floor_hi) : fl;
        __syncthreads();  // every thread has read the count before the selection may reset it
        if (cnt > kWarps * 32 && cnt <= kCap / 2) {
            // more candidates than one key per thread: when at least k of them reach the upper floor (about 2 k
            // expected), those alone hold the top k (any other has k collected keys above it), and sorting them
            // takes one pass of the selection instead of two.  They are compacted into the buffer's second half,
            // then moved to its front.
            for (int e = threadIdx.x; e < cnt; e += kThreads) {
                const uint64_t key = sm.cand[e];
                if (key_value(key) >= fl_hi) sm.cand[kCap / 2 + atomicAdd(&sm.count_hi, 1)] = key;
            }
            __syncthreads();
            const int nh = sm.count_hi;
            if (nh >= k && nh <= kWarps * 32) {
                for (int e = threadIdx.x; e < nh; e += kThreads) sm.cand[e] = sm.cand[kCap / 2 + e];
                cnt = nh;
            }
            __syncthreads();
        }
        const int n = cnt < kCap ? cnt : kCap;
        if (cnt > kCap || n < k) {
            rescan_select<KP, BF16>(sm, base, c0, c1, bv, k);
        } else {
            select_topk<KP>(sm, n);
        }

        // ---- publish this piece
        const int pieces = P, slot = piece;
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
    if (k > 256) return 256;  // (callers reject k > 256; this only keeps the doubling from overflowing)
    int kp = 32;
    while (kp < k) kp <<= 1;
    return kp;
}

struct Plan {
    int grid;
    int pieces_per_row;
    int64_t piece_len;
    int max_pieces;
    int kp;
};

// One wave of kCtasPerSm CTAs per SM.  With at least as many rows as CTA slots every CTA takes a balanced run of
// whole rows (no partial records); with fewer, each row is cut into P = slots / rows equal pieces of at least
// 8192 elements, one per CTA, so no CTA ever pays a piece's fixed costs (first-batch latency, floors, select)
// twice in a row.
static Plan plan(int64_t rows, int64_t vocab, int64_t k) {
    Plan pl;
    const int64_t slots = (int64_t)sm_count() * kCtasPerSm;
    const int64_t min_piece = 8192;
    if (rows >= slots) {
        pl.grid = (int)slots;
        pl.pieces_per_row = 1;
        pl.piece_len = vocab;
    } else {
        int64_t P = slots / rows;
        const int64_t cap = vocab / min_piece;
        if (P > cap) P = cap;
        if (P < 1) P = 1;
        int64_t len = (vocab + P - 1) / P;
        len = (len + 7) / 8 * 8;
        P = (vocab + len - 1) / len;
        pl.pieces_per_row = (int)P;
        pl.piece_len = len;
        pl.grid = (int)(rows * P);
    }
    pl.max_pieces = pl.pieces_per_row;
    pl.kp = kp_for(k);
    return pl;
}

}  // namespace topk
}  // namespace mfd

using namespace mfd;

extern "C" size_t mfd_topk_logz_workspace(int64_t rows, int64_t vocab, int64_t k) {
    if (rows <= 0 || vocab <= 0 || k <= 0 || k > vocab || k > 256 || vocab >= (int64_t)0x7fffffff) return 0;
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
    p.pieces_per_row = pl.pieces_per_row;
    p.piece_len = pl.piece_len;
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
