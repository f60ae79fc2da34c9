// tree_attention_tc.cu -- tree-masked GQA verify attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// softmax(q k^T * scale + mask) v for the tree rows of every request: row i sees every prefix key and, among the
// tree keys, exactly its ancestors and itself (the additive mask of inference/hf/ddtree.py:352-356, the flashinfer
// custom mask of sglang-v0.5.22-mfd.patch:1625-1703).  The mask is read from the builder's ancestor bitsets.
//
// Rows: the G query heads sharing a KV head are packed as r = node * G + g (260 rows for 65 nodes x 4 heads), so
// a key tile feeds G x n rows.  One CTA per (request, KV head, key split, 128-row M-tile); the M-tiles of one split
// are adjacent CTAs, so their shared K/V tiles come from L2 after the first read.  With per-request prefix lengths
// (up to 64 requests) the CTAs of the longest requests are launched first, so the short ones fill the tail.
//
// The kernel is a template over its tile configuration (Cfg below); the launched one has 128-key tiles, 3-stage K
// and V ring, 8 softmax warps and one CTA per SM.  Warp roles (320 threads):
//   warp 0       producer: Q once by TMA, then K and V tiles into their rings (128-byte swizzle, the canonical UMMA
//                K-major / MN-major layouts; no multicast) -- by TMA from dense [bs, Hkv, S, 128] caches (with an
//                L2 prefetch of the tiles kPrefetchAhead ahead), or, in paged mode (SGLang's paged mode attention),
//                gathered row by row with 16-byte cp.async through the request's req_to_token row into the same
//                swizzled layout
//   warp 1       MMA issuer: S[i%2] = Q K_i^T (M=128, N=tile keys, K=16 x 8) into TMEM, then O += P_{i-1} V_{i-1}
//                (M=128, N=128, A = P read from TMEM, V MN-major), so the scores of tile i are computed while the
//                softmax works on tile i-1
//   warps 2..    softmax: the PARTS warps of TMEM lane quarter q each take 128 / PARTS of a tile's key columns and
//                of O's columns (row max and, at the end, row sum exchanged through shared memory): tcgen05.ld of
//                S, mask (only tiles reaching the tree keys or the split end), exp2 (a third of them by a cubic on
//                the FMA pipe, the rest on the MUFU unit), bf16 P written back over S in TMEM; lazy O rescale in
//                TMEM only when a row's running max grows by more than 2^8.  A quarter whose 32 rows are all padding
//                (the last M-tile holds 4 of 128 rows for 65 x 4) keeps only the barrier protocol.  Epilogue
//                through a shared-memory stage so every store is coalesced.
// Splits: each CTA writes (O / l, log2 lse) partials; the splits of a (request, KV head, M-tile) then merge them
// together, 32 output columns at a time, claimed by an atomic counter: the last split to arrive always takes part,
// the others when they see every partial stored within a short bounded wait.  With one split the CTA writes out
// directly.
//
// TMEM: O at columns [0, 128), S[0] and S[1] after it (one column per tile key each): 512 columns allocated.
// Every mbarrier wait is bounded; when one gives up the CTA records a nonzero status, finishes without waiting
// further, and still releases its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tcgen05.cuh"
#include "tree_attention_tc.cuh"

namespace mfd {
namespace tca {

constexpr int D = 128;
constexpr int kSmemMax = 227 * 1024;  // the per-block opt-in maximum
constexpr int kSmemPerSm = 228 * 1024;  // per SM, of which 1 KB per resident block is reserved

// A kernel configuration: keys per tile, K/V ring depth, softmax warps per TMEM lane quarter (each takes
// KT / PARTS of a tile's key columns and D / PARTS of O's columns), resident CTAs per SM.  TMEM: O at columns
// [0, 128) and two S buffers after it (S of key tile i in buffer i % 2), so the scores of tile i are computed while
// the softmax works on tile i - 1.
// Launched: CfgRow = Cfg<128, 3, 2, 1>, one CTA per SM, 512 TMEM columns.  Measured alternatives (attention of the
// 256-request verify step, L2 flushed): four warps per row quarter (Cfg<128, 3, 4, 1>) 2127 us against 2030 us for
// two; one warp per row quarter (each thread a whole 128-key row) 2056 us; two M-tiles per CTA sharing each K / V
// tile with the MMA warp alternating between them (2 stages) 2221 to 2561 us; separate K and V rings (a K stage
// refilled as soon as its scores complete) 2146 us; Cfg<64, 2, 2, 2> (two CTAs per SM)
// was slower still at 32 requests (348 against 280 us).
template <int KT, int STAGES, int PARTS, int MINB, int TILES = 1>
struct Cfg {
    static constexpr int kKt = KT;
    static constexpr int kStages = STAGES;
    static constexpr int kParts = PARTS;
    static constexpr int kCtasPerSm = MINB;
    static constexpr int kTiles = TILES;
    static constexpr int kOCols = D / PARTS;  // O columns each part rescales and stores
    static constexpr int kGroupThreads = 128 * PARTS;  // the softmax warps of one M-tile
    static constexpr int kSoftmaxThreads = kGroupThreads * TILES;
    static constexpr int kThreads = 64 + kSoftmaxThreads;  // warp 0 producer, warp 1 MMA, then the softmax warps
    // Two parts per row (one M-tile): each part keeps its own O accumulator, running max and sum for its half of
    // every key tile's columns, so the parts never exchange maxima per tile; the epilogue merges the two.
    static constexpr bool kDualO = TILES == 1 && PARTS == 2;
    // O of M-tile t at column 128 t (dual: O of part p at 128 p); S buffer b at column kSCol + KT b (TILES = 1:
    // b = key tile parity; TILES = 2: b = M-tile); P (bf16 pairs) over its first KT / 2 columns (dual: each part's
    // P over the first half of its own KT / 2 columns)
    static constexpr int kSCol = kDualO ? 256 : 128 * TILES;
    static constexpr int kTmemCols = kSCol + 2 * KT <= 256 ? 256 : 512;
    static constexpr int kQBytes = kM * D * 2;    // 32 KB per M-tile: [2 d-halves][128 rows][128 B]
    static constexpr int kKVBytes = KT * D * 2;   // [2 d-halves][KT keys][128 B]
    static constexpr int kOffQ = 0;
    static constexpr int kOffK = kOffQ + TILES * kQBytes;
    static constexpr int kOffV = kOffK + STAGES * kKVBytes;
    static constexpr int kOffX = kOffV + STAGES * kKVBytes;  // row maxima / sums exchanged by the parts of a row
    static constexpr int kOffBar = kOffX + 2 * PARTS * kM * 4;  // (two tiles' exchanges)
    static constexpr int kBarArea = 256;
    static constexpr int kSmemUsed = kOffBar + kBarArea;  // + barriers, TMEM address, flags
    static constexpr int kSmemCap = MINB == 1 ? kSmemMax : kSmemPerSm / MINB - 1024;
    // the 128-byte-swizzled TMA destinations need a 1024-byte aligned base: the slack that fits is reserved and
    // the kernel checks at entry that the base's misalignment is within it
    static constexpr int kSmemSlack = kSmemCap - kSmemUsed < 1024 ? kSmemCap - kSmemUsed : 1024;
    static constexpr int kSmemBytes = kSmemUsed + kSmemSlack;
    // barrier slots
    static constexpr int kBarQ = 0;
    static constexpr int kBarKVFull = 1;                     // + stage
    static constexpr int kBarKVEmpty = kBarKVFull + STAGES;  // + stage
    static constexpr int kBarSFull = kBarKVEmpty + STAGES;   // + S buffer
    static constexpr int kBarPFull = kBarSFull + 2;  // + S buffer (P written into it; frees it for the next scores)
    static constexpr int kBarPV = kBarPFull + 2;     // + S buffer: the P V that read it completes
    static constexpr int kNumBars = kBarPV + 2;
    static_assert(KT % (32 * PARTS) == 0, "each softmax warp takes a multiple of 32 key columns");
    static_assert(TILES == 1 || (TILES == 2 && PARTS == 1 && kSCol + 2 * KT <= 512), "two M-tiles: one warp per row");
    static_assert(kOCols % 32 == 0, "O columns per part");
    static_assert(kSmemSlack >= 0 && kSmemBytes <= kSmemCap, "shared memory");
    static_assert(STAGES * kKVBytes >= TILES * kM * 256, "the epilogue stages 128 bf16 rows per M-tile in the K ring");
    static_assert(8 * kNumBars + 4 + 4 * TILES <= kBarArea, "barrier area");
    static_assert(MINB * kThreads <= 2048, "threads per SM");
};
using CfgRow = Cfg<128, 3, 2, 1>;
using CfgPair = Cfg<128, 2, 1, 1, 2>;
constexpr uint32_t kTries = 1u << 20;              // bounded mbarrier waits
// The split merge: output column slices of 32 that the splits of a unit claim, and the bounded wait of a split for
// the others' partials (32 polls, about 10-20 us; the splits of a unit normally run in one wave and arrive within a
// microsecond or two of each other).
constexpr int kMergeSlices = D / 32;
constexpr int kMergeSpins = 32;
__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int* ptr) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
    return v;
}
// K / V tiles are prefetched into L2 this many tiles before their load into the ring, so the ring's loads see L2
// latency instead of DRAM latency (a stage is refilled less than one tile period before its scores are needed)
constexpr int kPrefetchAhead = 4;

// ------------------------------------------------------------------ TMA (the tcgen05 wrappers are in tcgen05.cuh)
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(dst),
        "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(bar))
        : "memory");
}
// L2 prefetch of one tile of a tensor map (no shared-memory destination, no completion to wait for)
__device__ __forceinline__ void tma_prefetch_4d(const CUtensorMap* map, int c0, int c1, int c2, int c3) {
    asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(map), "r"(c0),
                 "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
}
// 2^x on the FMA pipe, both lanes of a packed pair, for a share of the softmax's exponentials (the MUFU unit's
// ex2 alone would bound the softmax).  x = n + f with n = round(x) (adding 1.5 * 2^23 rounds to an integer) and
// f in [-1/2, 1/2]; 2^f by the cubic p(f) = 1 + f (c1 + f (c2 + f c3)), coefficients fitted to 2^f on [-1/2, 1/2]
// for the least maximum relative error (iteratively reweighted least squares, Lawson's method, on 20001 points;
// the constant term fixed at 1): 1.02e-4, far below the bf16 rounding (2^-9) P gets next.  2^n enters as n << 23
// added to p's bits (the bits of the rounded sum are 0x4B400000 + n, and 0x4B400000 << 23 vanishes modulo 2^32).
// x is first clamped to -127: there f = 0 and p = 1 exactly, so the bits are those of +0 -- masked scores (-inf)
// and NaN give 0 as ex2.approx.ftz gives for -inf.  (Arguments stay at or below 8: the lazy rescale keeps every
// score within 2^8 of the running max.)
constexpr float kExpC1 = 0.6932827234268188f, kExpC2 = 0.24220797419548035f, kExpC3 = 0.055007610470056534f;
__device__ __forceinline__ uint64_t exp2_poly2(uint64_t x) {
    float x0, x1;
    upk2(x, x0, x1);
    const uint64_t xc = pk2(fmaxf(x0, -127.f), fmaxf(x1, -127.f));
    const uint64_t t = add2(xc, dup2(12582912.f));
    const uint64_t f = sub2(xc, sub2(t, dup2(12582912.f)));
    const uint64_t q = fma2(fma2(fma2(dup2(kExpC3), f, dup2(kExpC2)), f, dup2(kExpC1)), f, dup2(1.f));
    float q0, q1, t0, t1;
    upk2(q, q0, q1);
    upk2(t, t0, t1);
    return pk2(__uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23)),
               __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23)));
}
// every kPolyEvery-th exponential pair of a row's keys goes to exp2_poly2, the rest to ex2.approx
constexpr int kPolyEvery = 3;

// named barriers: 1 (and 6) = the softmax warps of M-tile 0 (and 1), 2 + q = the PARTS warps of TMEM lane quarter q
// (one warp: a warp sync)
template <int N>
__device__ __forceinline__ void group_sync(int g) {  // the softmax warps of M-tile g: barrier 1 or 6
    asm volatile("bar.sync %0, %1;" ::"r"(1 + 5 * g), "n"(N) : "memory");
}
template <int PARTS>
__device__ __forceinline__ void quarter_sync(int quarter) {
    if (PARTS == 1) __syncwarp();
    else asm volatile("bar.sync %0, %1;" ::"r"(2 + quarter), "n"(32 * PARTS) : "memory");
}
// the same barrier, returning the AND of v over the quarter's threads (so its warps leave a loop together)
template <int PARTS>
__device__ __forceinline__ bool quarter_sync_and(int quarter, bool v) {
    if (PARTS == 1) return __all_sync(MFD_FULL_MASK, v);
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\tsetp.ne.b32 pi, %1, 0;\n\tbar.red.and.pred po, %2, %3, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(2 + quarter), "n"(32 * PARTS)
        : "memory");
    return r != 0u;
}

// The request whose prefix is the z-th longest (ties by request index), so that the longest requests' CTAs are
// launched first and the shortest fill the tail.  Every warp computes it (lane j ranks requests j, j + 32, ...);
// used for up to kMaxOrdered requests with per-request prefix lengths, otherwise request z.
constexpr int kMaxOrdered = 64;
__device__ __forceinline__ int request_by_length_rank(const int32_t* prefix, int bs, int z) {
    const int lane = threadIdx.x & 31;
    int found = z;
    for (int c0 = 0; c0 < bs; c0 += 32) {
        const int me = c0 + lane;
        int rank = -1;
        if (me < bs) {
            const int lm = __ldg(prefix + me);
            rank = 0;
            for (int o = 0; o < bs; ++o) {
                const int lo = __ldg(prefix + o);
                rank += (lo > lm || (lo == lm && o < me)) ? 1 : 0;
            }
        }
        const uint32_t hit = __ballot_sync(MFD_FULL_MASK, rank == z);
        if (hit) found = c0 + __ffs(hit) - 1;
    }
    return found;
}

template <class C>
__global__ void __launch_bounds__(C::kThreads, C::kCtasPerSm)
    tree_attn_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                        const __grid_constant__ CUtensorMap tmv, const Params p) {
    constexpr int kKt = C::kKt, kStages = C::kStages, kParts = C::kParts, kOCols = C::kOCols, kTiles = C::kTiles;
    constexpr int kGroupThreads = C::kGroupThreads;
    constexpr bool kDualO = C::kDualO;
    constexpr int kSoftmaxThreads = C::kSoftmaxThreads, kTmemCols = C::kTmemCols, kSCol = C::kSCol;
    constexpr int kQBytes = C::kQBytes, kKVBytes = C::kKVBytes;
    constexpr int kOffQ = C::kOffQ, kOffK = C::kOffK, kOffV = C::kOffV, kOffX = C::kOffX, kOffBar = C::kOffBar;
    constexpr int kSmemSlack = C::kSmemSlack, kNumBars = C::kNumBars;
    constexpr int kBarQ = C::kBarQ, kBarKVFull = C::kBarKVFull, kBarKVEmpty = C::kBarKVEmpty;
    constexpr int kBarSFull = C::kBarSFull, kBarPFull = C::kBarPFull, kBarPV = C::kBarPV;
    constexpr int kKeyGroups = kKt / 32;  // the paged gather's 32-key groups per tile
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t pad = (1024u - (smem_addr(smem_raw) & 1023u)) & 1023u;
    if (pad > (uint32_t)kSmemSlack) {  // (uniform: before any barrier, copy or TMEM use)
        if (threadIdx.x == 0 && p.status) atomicExch(p.status, 2);
        return;
    }
    unsigned char* smem = smem_raw + pad;
    const uint32_t sbase = smem_addr(smem);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + 8 * kNumBars);
    int* shared_flags = reinterpret_cast<int*>(smem + kOffBar + 8 * kNumBars + 4);  // one per M-tile
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // CTA x = split * ctiles + c: the CTA takes M-tiles mt0 .. mt0 + ntl - 1 of its (request, KV head)
    const int ctiles = (p.mtiles + kTiles - 1) / kTiles;
    const int split = blockIdx.x / ctiles;
    const int mt0 = (blockIdx.x % ctiles) * kTiles;
    const int ntl = min(kTiles, p.mtiles - mt0);
    const int hk = blockIdx.y;
    const int b = (!p.paged && p.prefix && p.bs > 1 && p.bs <= kMaxOrdered)
                      ? request_by_length_rank(p.prefix, p.bs, (int)blockIdx.z)
                      : (int)blockIdx.z;
    const int nrows = p.n * p.G;
    // the phase of S buffer / P / P V barrier use i: one M-tile alternates two S buffers, two M-tiles have one each
    auto sph = [](int i) { return (uint32_t)(kTiles == 1 ? ((i >> 1) & 1) : (i & 1)); };
    // keys [0, prefix) are visible to every row; keys [prefix, prefix + n) are the tree (block) keys, visible by the
    // ancestor bitsets.  Paged mode: the prefix is the request's context length, read on the device.
    int prefix;
    const int32_t* r2t_row = nullptr;
    if (p.paged) {
        const int64_t c = __ldg(p.ctx + b);
        prefix = (int)(c < 0 ? 0 : (c > p.r2t_cols ? p.r2t_cols : c));
        int64_t pool_row = __ldg(p.rpi + b);
        pool_row = pool_row < 0 ? 0 : (pool_row >= p.r2t_rows ? p.r2t_rows - 1 : pool_row);
        r2t_row = p.r2t + pool_row * p.r2t_stride;
    } else {
        prefix = p.prefix ? p.prefix[b] : p.prefix_const;
    }
    const int total = prefix + p.n;
    int chunk = (total + p.splits - 1) / p.splits;
    chunk = (chunk + kKt - 1) / kKt * kKt;
    const int k_lo = split * chunk;
    const int k_hi = min(total, k_lo + chunk);
    const int ntiles = k_hi > k_lo ? (k_hi - k_lo + kKt - 1) / kKt : 0;

    // barriers and the first loads before anything else, so the TMA round trip overlaps the TMEM allocation
    if (threadIdx.x == 0) {
        for (int i = 0; i < kNumBars; ++i)
            mbar_init(&bars[i], (i >= kBarPFull && i < kBarPV) ? (uint32_t)(4 * kParts) : 1u);
        for (int t = 0; t < kTiles; ++t) shared_flags[t] = 0;
        mbar_fence_init();
    }
    auto prefetch_kv = [&](int i) {
        if (i >= ntiles) return;
        const int key0 = k_lo + i * kKt;
        for (int h = 0; h < 2; ++h) {
            tma_prefetch_4d(&tmk, h * 64, key0, hk, b);
            tma_prefetch_4d(&tmv, h * 64, key0, hk, b);
        }
    };
    auto load_kv = [&](int i) {
        const int st = i % kStages;
        const int key0 = k_lo + i * kKt;
        mbar_expect_tx(&bars[kBarKVFull + st], 2 * kKVBytes);
        for (int h = 0; h < 2; ++h) {
            tma_load_4d(sbase + kOffK + st * kKVBytes + h * (kKVBytes / 2), &tmk, &bars[kBarKVFull + st], h * 64,
                        key0, hk, b);
            tma_load_4d(sbase + kOffV + st * kKVBytes + h * (kKVBytes / 2), &tmv, &bars[kBarKVFull + st], h * 64,
                        key0, hk, b);
        }
    };
    // paged: warp 0 gathers each 128-key tile with 16-byte cp.async copies into the same 128-byte-swizzled layout the
    // tiled TMA load produces (granule c of key row r at r * 128 + ((c ^ (r & 7)) << 4) in each d-half).  Context
    // keys come from the caches through the request's req_to_token row, block keys from k_new / v_new (keys past
    // the end repeat the last block key and are masked).  One warp instruction moves 4 keys' half rows: lane l
    // takes key 32 t + 4 j + (l >> 3), granule l & 7.
    // slot ids of the next tile's keys key0 + lane + 32 t (context keys only), loaded one tile ahead so that the
    // req_to_token read is off the chain of the tile being issued
    int32_t next_slot[kKeyGroups];
    auto fetch_slots = [&](int i) {
        const int key0 = k_lo + i * kKt;
#pragma unroll
        for (int t = 0; t < kKeyGroups; ++t) {
            const int r = key0 + lane + 32 * t;
            next_slot[t] = (i < ntiles && r < prefix) ? __ldg(r2t_row + r) : 0;
        }
    };
    auto load_kv_paged = [&](int i) {
        const int st = i % kStages;
        const int key0 = k_lo + i * kKt;
        int64_t roff[kKeyGroups];  // element offsets of keys key0 + lane + 32 t (row start of this KV head)
        bool rcache[kKeyGroups];
#pragma unroll
        for (int t = 0; t < kKeyGroups; ++t) {
            const int r = key0 + lane + 32 * t;
            rcache[t] = r < prefix;
            roff[t] = rcache[t] ? (int64_t)min(max(next_slot[t], 0), (int)(p.slots - 1)) * p.skc_t + hk * D
                                : ((int64_t)b * p.n + min(r - prefix, p.n - 1)) * p.skn_t + hk * D;
        }
        fetch_slots(i + 1);
        const int c = lane & 7;
#pragma unroll
        for (int t = 0; t < kKeyGroups; ++t) {
#pragma unroll 2
            for (int j = 0; j < 8; ++j) {
                const int src = 4 * j + (lane >> 3);  // the lane holding this instruction's key
                const int key = 32 * t + src;          // key within the tile
                const int64_t off = (int64_t)__shfl_sync(MFD_FULL_MASK, (long long)roff[t], src);
                const bool cache = __shfl_sync(MFD_FULL_MASK, (int)rcache[t], src) != 0;
                const __nv_bfloat16* kr = (cache ? p.kc : p.kn) + off;
                const __nv_bfloat16* vr = (cache ? p.vc : p.vn) + off;
                const uint32_t sw = (uint32_t)(key * 128 + ((c ^ (key & 7)) << 4));
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t dk = sbase + kOffK + st * kKVBytes + h * (kKVBytes / 2) + sw;
                    const uint32_t dv = sbase + kOffV + st * kKVBytes + h * (kKVBytes / 2) + sw;
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dk), "l"(kr + h * 64 + c * 8)
                                 : "memory");
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dv), "l"(vr + h * 64 + c * 8)
                                 : "memory");
                }
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // the copies of tile j have landed: make them visible to the tensor cores (async proxy), then mark the stage full
    auto publish_paged = [&](int j, bool last) {
        if (last) asm volatile("cp.async.wait_group 0;" ::: "memory");
        else asm volatile("cp.async.wait_group 1;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[kBarKVFull + j % kStages]);
    };
    if (threadIdx.x == 0 && ntiles > 0) {  // (a split past the keys loads nothing: every issued copy is waited for)
        const int nodes_per_tile = kM / p.G;
        mbar_expect_tx(&bars[kBarQ], ntl * kQBytes);
        for (int t = 0; t < ntl; ++t)
            for (int h = 0; h < 2; ++h)
                tma_load_4d(sbase + kOffQ + t * kQBytes + h * (kQBytes / 2), &tmq, &bars[kBarQ], h * 64, hk * p.G,
                            (mt0 + t) * nodes_per_tile, b);
        if (!p.paged) {
            for (int i = 0; i < min(kStages, ntiles); ++i) load_kv(i);
            for (int i = kStages; i < kStages + kPrefetchAhead; ++i) prefetch_kv(i);
        }
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (p.paged) {
            // tile i's copies are issued, then tile i - 1 is published (two tiles' copies in flight); a stage is
            // refilled only after the MMA released it.  The release of stage i % kStages (the P V of tile
            // i - kStages) follows the scores of tile i - kStages + 1, so that tile must be published before the
            // wait: with a 2-stage ring that is tile i - 1, published as soon as its copies land.
            fetch_slots(0);
            int pub = 0;  // tiles published
            for (int i = 0; i < ntiles; ++i) {
                if (i >= kStages) {
                    if (pub < i - kStages + 2) {
                        publish_paged(i - 1, true);
                        pub = i;
                    }
                    bool w = true;
                    if (lane == 0) w = mbar_wait(&bars[kBarKVEmpty + i % kStages], ((i / kStages) - 1) & 1, kTries);
                    ok &= __shfl_sync(MFD_FULL_MASK, (int)w, 0) != 0;
                    if (!ok) break;
                }
                load_kv_paged(i);
                if (i >= 1 && pub < i) {
                    publish_paged(i - 1, false);
                    pub = i;
                }
            }
            if (ok && pub < ntiles) publish_paged(ntiles - 1, true);
            asm volatile("cp.async.wait_group 0;" ::: "memory");  // nothing in flight when the warp leaves
        } else if (lane == 0) {
            for (int i = kStages; i < ntiles && ok; ++i) {
                prefetch_kv(i + kPrefetchAhead);
                ok &= mbar_wait(&bars[kBarKVEmpty + i % kStages], ((i / kStages) - 1) & 1, kTries);
                if (ok) load_kv(i);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t kIdescS = idesc_bf16(kM, kKt, 0);
            constexpr uint32_t kIdescO = idesc_bf16(kM, D, 1);
            // S(t, i) = Q_t K_i^T into S buffer sb (key tile parity with one M-tile, the M-tile with two)
            auto issue_qk = [&](int t, int i, int sb) {
                const int st = i % kStages;
                const uint32_t kaddr = sbase + kOffK + st * kKVBytes;
                const uint32_t qaddr = sbase + kOffQ + t * kQBytes;
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks) {
                    const uint32_t qoff = (uint32_t)((ks >> 2) * (kQBytes / 2) + (ks & 3) * 32);
                    const uint32_t koff = (uint32_t)((ks >> 2) * (kKVBytes / 2) + (ks & 3) * 32);
                    umma(tmem + kSCol + sb * kKt, sdesc(qaddr + qoff, 16, 1024), sdesc(kaddr + koff, 16, 1024), kIdescS,
                         ks > 0);
                }
                umma_commit(&bars[kBarSFull + sb]);
            };
            // O_t += P(t, j) V_j once the softmax published P(t, j)
            auto issue_pv = [&](int t, int j, int sb) {
                const int st = j % kStages;
                ok &= mbar_wait(&bars[kBarPFull + sb], sph(j), kTries);
                tc_fence_after();
                const uint32_t vaddr = sbase + kOffV + st * kKVBytes;
#pragma unroll
                for (int ks = 0; ks < kKt / 16; ++ks) {  // P: 16 keys = 8 columns of bf16 pairs per step
                    if (kDualO) {  // keys of the first half into O_0, of the second into O_1
                        constexpr int kHalf = kKt / 32;  // steps per half
                        const int hf = ks / kHalf, kk = ks % kHalf;
                        umma_ts(tmem + hf * 128, tmem + kSCol + sb * kKt + hf * (kKt / 2) + kk * 8,
                                sdesc(vaddr + ks * 2048, kKVBytes / 2, 1024), kIdescO, (j > 0 || kk > 0) ? 1u : 0u);
                    } else {
                        umma_ts(tmem + t * 128, tmem + kSCol + sb * kKt + ks * 8,
                                sdesc(vaddr + ks * 2048, kKVBytes / 2, 1024), kIdescO, (j > 0 || ks > 0) ? 1u : 0u);
                    }
                }
                umma_commit(&bars[kBarPV + sb]);
            };
            auto wait_kv = [&](int i) {
                ok &= mbar_wait(&bars[kBarKVFull + i % kStages], (i / kStages) & 1, kTries);
                tc_fence_after();
            };
            if (ntiles > 0) ok &= mbar_wait(&bars[kBarQ], 0, kTries);
            if (kTiles == 1) {
                // scores of tile i while the softmax works on tile i - 1 (two S buffers); the stage of tile i - 1
                // is released when its P V completes.  S[i % 2] last held P(i - 2), which the P V issued in the
                // previous iteration consumed (tensor-core operations of this thread execute in order).
                for (int i = 0; i < ntiles && ok; ++i) {
                    wait_kv(i);
                    issue_qk(0, i, i & 1);
                    if (i >= 1 && ok) {
                        issue_pv(0, i - 1, (i - 1) & 1);
                        umma_commit(&bars[kBarKVEmpty + (i - 1) % kStages]);
                    }
                }
                if (ntiles > 0 && ok) {
                    issue_pv(0, ntiles - 1, (ntiles - 1) & 1);
                    umma_commit(&bars[kBarKVEmpty + (ntiles - 1) % kStages]);
                }
            } else {
                // two M-tiles, each with its own softmax warps and S buffer: P V of M-tile t for key tile i, then
                // its scores for key tile i + 1 (into the buffer the P V just read), while the other M-tile's
                // softmax runs; the stage of tile i is released after the last M-tile's P V
                if (ntiles > 0 && ok) {
                    wait_kv(0);
                    for (int t = 0; t < ntl; ++t) issue_qk(t, 0, t);
                }
                for (int i = 0; i < ntiles && ok; ++i) {
                    for (int t = 0; t < ntl && ok; ++t) {
                        issue_pv(t, i, t);
                        if (t == ntl - 1) umma_commit(&bars[kBarKVEmpty + i % kStages]);
                        if (i + 1 < ntiles && ok) {
                            if (t == 0) wait_kv(i + 1);
                            issue_qk(t, i + 1, t);
                        }
                    }
                }
            }
        }
    } else {
        // ---------------------------------------------------------------- softmax warps
        // warp w: M-tile t = (w - 2) / (4 kParts) of the CTA, TMEM lane quarter w % 4, key columns
        // [kCols part, kCols part + kCols) of each tile with part = ((w - 2) mod 4 kParts) / 4.  With two parts per
        // row (the launched single-M-tile configuration) each part keeps its own O accumulator, running max and
        // sum, merged with the other part's in the epilogue; with more parts they exchange their row maxima per
        // tile (and their row sums at the end) through shared memory.  With two M-tiles each has its own warps, so
        // one M-tile's softmax runs while the other's P V and scores do.
        const int wg = warp - 2;
        const int t = wg / (4 * kParts);
        const int quarter = warp & 3;
        const int part = (wg % (4 * kParts)) >> 2;
        const int gtid = threadIdx.x - 64 - t * kGroupThreads;  // thread index among this M-tile's warps
        const int row0 = (mt0 + t) * kM;
        const int mtile = mt0 + t;
        const int rt = quarter * 32 + lane;  // row within the M-tile (TMEM lane)
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        float* xmax = reinterpret_cast<float*>(smem + kOffX);  // [2][kParts][128 rows]
        constexpr int kCols = kKt / kParts, kChunks = kCols / 32;
        const int c_lo = part * kCols;   // this warp's kCols of the tile's kKt key columns
        const int o_lo = part * kOCols;  // and its kOCols of O's 128 columns
        const float sc = p.scale_log2;
        float m_run = -INFINITY, l_run = 0.f;
        // a quarter whose 32 rows are all padding keeps only the barrier protocol: it leaves its TMEM rows as they
        // are, and the P V rows they feed (rows are independent in the MMA) are never stored
        const bool quarter_live = row0 + quarter * 32 < nrows;
        const int loop_tiles = t < ntl ? ntiles : 0;  // (a CTA's last M-tile may have no second one)
        // with a per-tile max exchange the loop ends for all warps of a quarter together, at the exchange, where
        // their ok flags are AND-ed (a warp leaving alone would leave its partners waiting at a named barrier)
        for (int i = 0; i < loop_tiles; ++i) {
            const int key0 = k_lo + i * kKt;
            const int sb = kTiles == 1 ? (i & 1) : t;
            const uint32_t s_tm = tmem + lane_off + kSCol + sb * kKt;
            ok &= mbar_wait(&bars[kBarSFull + sb], sph(i), kTries);
            tc_fence_after();
            if (key0 + kKt > k_hi) {
                // the tile runs past this split's keys: its rows from k_hi on hold whatever the caller's buffer has
                // beyond the request's keys (any bits, NaN included).  Their P is 0, but 0 * NaN is NaN in the P V
                // product, so those V rows are cleared before P is published (the tile landed before S(i) was
                // computed, and an M-tile's P V (i) is issued only after all its softmax warps have arrived below;
                // with two M-tiles each clears every such row itself, the other's stores writing the same zeros).
                // Each key row is 128 contiguous bytes per d-half, whatever the swizzle order of its granules.
                const int r0 = k_hi > key0 ? k_hi - key0 : 0;
                unsigned char* vt = smem + kOffV + (i % kStages) * kKVBytes;
                for (int g = gtid; g < (kKt - r0) * 16; g += kGroupThreads) {
                    const int rr = r0 + (g >> 4), h = (g >> 3) & 1, c = g & 7;
                    *reinterpret_cast<uint4*>(vt + h * (kKVBytes / 2) + rr * 128 + c * 16) = make_uint4(0u, 0u, 0u, 0u);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor cores
            }
            if (!quarter_live) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars[kBarPFull + sb]);
                ok = __all_sync(MFD_FULL_MASK, ok);
                if (!ok) break;
                continue;
            }
            // this part's kCols scores of the row: kChunks TMEM loads in flight together
            uint32_t sraw[kChunks][32];
#pragma unroll
            for (int c = 0; c < kChunks; ++c) tmem_ld32_issue(s_tm + c_lo + 32 * c, sraw[c]);
            tmem_ld_wait(sraw);
            float s[kChunks][32];
#pragma unroll
            for (int c = 0; c < kChunks; ++c)
#pragma unroll
                for (int j = 0; j < 32; ++j) s[c][j] = __uint_as_float(sraw[c][j]);
            const bool fast = key0 + kKt <= prefix && key0 + kKt <= k_hi;
            if (!fast) {
                const int r = row0 + rt;  // packed row
                const int node = r < nrows ? r / p.G : 0;
                const uint64_t* anc_row = p.anc + ((size_t)(p.paged ? 0 : b) * p.n + node) * p.words;  // paged:
                                                                                                       // shared
#pragma unroll
                for (int c = 0; c < kChunks; ++c) {
                    // visibility of 32 keys as a bitmask: prefix keys, then the row's ancestor bits for the
                    // tree keys (two bitset words funnel-shifted into place), all cut at the split end
                    const int kb = key0 + c_lo + 32 * c;  // first key of this chunk
                    const int t0 = kb - prefix;             // its tree index (negative: prefix keys come first)
                    uint64_t vis;
                    if (t0 <= -64) {
                        vis = ~0ull;
                    } else {
                        const int w = t0 >> 6;  // floor division: word holding tree index t0 (t0 >= -63)
                        const int sh = t0 & 63;
                        const uint64_t lo = (w >= 0 && w < p.words) ? __ldg(anc_row + w) : 0ull;
                        const uint64_t hi = (w + 1 >= 0 && w + 1 < p.words) ? __ldg(anc_row + w + 1) : 0ull;
                        uint64_t tree = sh ? ((lo >> sh) | (hi << (64 - sh))) : lo;  // bit j: tree index t0 + j
                        if (t0 < 0) {  // the first -t0 keys are prefix keys
                            const int np = -t0;
                            tree = hi << np;
                            vis = tree | ((1ull << np) - 1ull);
                        } else {
                            vis = tree;
                        }
                    }
                    const int live_keys = k_hi - kb;  // keys of this chunk before the split end
                    if (live_keys < 32) vis &= live_keys <= 0 ? 0ull : ((1ull << live_keys) - 1ull);
#pragma unroll
                    for (int j = 0; j < 32; ++j) s[c][j] = ((vis >> j) & 1ull) ? s[c][j] : -INFINITY;
                }
            }
            float mx;
            {  // the raw scores' maximum as a tree of three-input maxima (scaling by sc > 0 keeps the order)
                float u[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) u[j] = fmaxf(s[0][j], s[0][j + 16]);
#pragma unroll
                for (int c = 1; c < kChunks; ++c)
#pragma unroll
                    for (int j = 0; j < 16; ++j) u[j] = fmax3(u[j], s[c][j], s[c][j + 16]);
#pragma unroll
                for (int j = 0; j < 5; ++j) u[j] = fmax3(u[3 * j], u[3 * j + 1], u[3 * j + 2]);
                mx = fmaxf(fmax3(u[0], u[1], u[2]), fmax3(u[3], u[4], u[15])) * sc;
            }
            if (kParts > 1 && !kDualO) {
                // the row's max over the parts, through a double-buffered exchange: after this barrier every part
                // has finished reading S (so P may overwrite it), and a part can run at most one tile ahead
                xmax[((i & 1) * kParts + part) * kM + rt] = mx;
                ok = quarter_sync_and<kParts>(quarter, ok);
#pragma unroll
                for (int q = 0; q < kParts; ++q) mx = fmaxf(mx, xmax[((i & 1) * kParts + q) * kM + rt]);
            } else {
                ok = __all_sync(MFD_FULL_MASK, ok);  // (dual: each part keeps its own running max)
            }
            if (!ok) break;
            float alpha = 1.f;
            bool rescale = false;
            if (mx > m_run + 8.f) {  // lazy: keep the running max unless the tile's exceeds it by over 2^8
                if (m_run != -INFINITY) {
                    alpha = fast_exp2(m_run - mx);
                    rescale = true;
                }
                m_run = mx;
            }
            const float mref = m_run == -INFINITY ? 0.f : m_run;  // nothing visible yet: every p is 0
            // p = 2^(s sc - mref) with the products and sums on packed pairs; every kPolyEvery-th pair's
            // exponentials on the FMA pipe (exp2_poly2), the others on the MUFU unit
            const uint64_t sc2 = dup2(sc), nm2 = dup2(-mref);
            uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};  // independent partial row sums (pairs)
#pragma unroll
            for (int c = 0; c < kChunks; ++c) {
                uint32_t pk[16];
#pragma unroll
                for (int jp = 0; jp < 16; ++jp) {
                    const uint64_t x = fma2(pk2(s[c][2 * jp], s[c][2 * jp + 1]), sc2, nm2);
                    uint64_t e;
                    if (jp % kPolyEvery == kPolyEvery - 1) {
                        e = exp2_poly2(x);
                    } else {
                        float x0, x1;
                        upk2(x, x0, x1);
                        e = pk2(fast_exp2(x0), fast_exp2(x1));
                    }
                    acc[jp & 3] = add2(acc[jp & 3], e);
                    float e0, e1;
                    upk2(e, e0, e1);
                    pk[jp] = pack_bf16(e0, e1);
                }
                // P as bf16 pairs over the first kKt / 2 columns of the S buffer (dual: of this part's own
                // columns): chunk c's 32 keys = 16 columns.  Every S value of the warp is in registers by now.
                tmem_st16u(s_tm + (kDualO ? c_lo : (c_lo >> 1)) + 16 * c, pk);
            }
            float l_add;
            {
                const uint64_t a2 = add2(add2(acc[0], acc[1]), add2(acc[2], acc[3]));
                float a0, a1;
                upk2(a2, a0, a1);
                l_add = a0 + a1;
            }
            l_run = l_run * alpha + l_add;
            if (__any_sync(MFD_FULL_MASK, rescale)) {  // O must hold the P V of key tile i - 1; this part
                                                       // rescales O's columns [o_lo, o_lo + kOCols)
                if (i >= 1) {
                    ok &= mbar_wait(&bars[kBarPV + (kTiles == 1 ? ((i - 1) & 1) : t)], sph(i - 1), kTries);
                    tc_fence_after();
                }
                // (dual: this part's own accumulator, all of its columns)
                constexpr int kRescaleCols = kDualO ? D : kOCols;
                const uint32_t obase = tmem + lane_off + (kDualO ? part * 128 : t * 128 + o_lo);
#pragma unroll
                for (int oc = 0; oc < kRescaleCols; oc += 32) {
                    float o[32];
                    tmem_ld32(obase + oc, o);
#pragma unroll
                    for (int j = 0; j < 32; ++j) o[j] *= alpha;
                    tmem_st32(obase + oc, o);
                }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[kBarPFull + sb]);
        }
        const size_t units = (size_t)p.bs * p.Hkv * p.mtiles;
        // staging of bf16 rows for coalesced stores: the K ring is free once the last P V completed
        unsigned char* stage = smem + kOffK + t * (kM * 256);  // [128 rows][256 B] per M-tile
        if (t < ntl) {
            if (ntiles > 0 && ok) {  // O's last P V (every earlier one completed before it)
                ok &= mbar_wait(&bars[kBarPV + (kTiles == 1 ? ((ntiles - 1) & 1) : t)], sph(ntiles - 1), kTries);
                tc_fence_after();
            }
            // ---- epilogue: the row sum over the parts, then this part's kOCols columns of O / l
            float l_row = l_run, m_fin = m_run;
            float fself = 1.f, fother = 0.f;  // dual: weights of this part's and the other part's accumulator
            if (kDualO) {
                // merge the two parts' (max, sum): each O_p holds its half's sum of 2^(s - m_p) v
                xmax[part * kM + rt] = m_run;
                xmax[(2 + part) * kM + rt] = l_run;
                quarter_sync<kParts>(quarter);
                const float mo = xmax[(1 - part) * kM + rt], lo = xmax[(3 - part) * kM + rt];
                m_fin = fmaxf(m_run, mo);
                fself = m_run == -INFINITY ? 0.f : fast_exp2(m_run - m_fin);
                fother = mo == -INFINITY ? 0.f : fast_exp2(mo - m_fin);
                l_row = l_run * fself + lo * fother;
            } else if (kParts > 1) {
                quarter_sync<kParts>(quarter);  // every part is past its last use of xmax
                xmax[part * kM + rt] = l_run;
                quarter_sync<kParts>(quarter);
                l_row = 0.f;
#pragma unroll
                for (int q = 0; q < kParts; ++q) l_row += xmax[q * kM + rt];
            }
            const float inv = l_row > 0.f ? 1.f / l_row : 0.f;
            const size_t unit = ((size_t)b * p.Hkv + hk) * p.mtiles + mtile;
#pragma unroll
            for (int oc = o_lo; oc < o_lo + kOCols; oc += 32) {
                float o[32];
                if (ntiles > 0 && quarter_live && kDualO) {
                    float o2[32];
                    tmem_ld32(tmem + lane_off + part * 128 + oc, o);
                    tmem_ld32(tmem + lane_off + (1 - part) * 128 + oc, o2);
#pragma unroll
                    for (int j = 0; j < 32; ++j) o[j] = o[j] * fself + o2[j] * fother;
                } else if (ntiles > 0 && quarter_live) {
                    tmem_ld32(tmem + lane_off + t * 128 + oc, o);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) o[j] = 0.f;
                }
                if (p.splits == 1) {
#pragma unroll
                    for (int j = 0; j < 32; j += 8)
                        *reinterpret_cast<uint4*>(stage + rt * 256 + (oc + j) * 2) = make_uint4(
                            pack_bf16(o[j] * inv, o[j + 1] * inv), pack_bf16(o[j + 2] * inv, o[j + 3] * inv),
                            pack_bf16(o[j + 4] * inv, o[j + 5] * inv), pack_bf16(o[j + 6] * inv, o[j + 7] * inv));
                } else {
                    // partials, chunk-major: float4 chunk c of row rt at [split][unit][c][rt] (a warp stores 512 B)
                    float4* dst = reinterpret_cast<float4*>(p.o_part) + ((size_t)split * units + unit) * (32 * kM);
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        dst[((oc + j) >> 2) * kM + rt] =
                            make_float4(o[j] * inv, o[j + 1] * inv, o[j + 2] * inv, o[j + 3] * inv);
                }
            }
            if (p.splits > 1) {
                if (part == 0)
                    p.lse_part[((size_t)split * units + unit) * kM + rt] =
                        l_row > 0.f ? m_fin + __log2f(l_row) : -INFINITY;
                // The splits of this (request, KV head, M-tile) merge their partials together: counters
                // [arrived, claimed, finished] per unit.  The last split to arrive knows every partial is stored; a
                // split that sees the arrival count complete within a short bounded wait joins it.  Each takes slices
                // of 32 output columns from the claim counter until none is left, so a split that gave up only
                // leaves its share to the others.  The last split to finish resets the counters.
                __threadfence();
                group_sync<kGroupThreads>(t);
                unsigned int* tk = p.tickets + 3 * unit;
                if (gtid == 0) {
                    const unsigned int tick = atomicAdd(tk, 1u);
                    int go = tick == (unsigned int)(p.splits - 1);
                    for (int it = 0; !go && it < kMergeSpins; ++it) {
                        __nanosleep(256);
                        go = ld_acquire_u32(tk) >= (unsigned int)p.splits;
                    }
                    shared_flags[t] = go;
                }
                group_sync<kGroupThreads>(t);
                const bool go = shared_flags[t] != 0;
                group_sync<kGroupThreads>(t);  // every thread has read the flag before the slot carries slices
                if (go) {
                    __threadfence();
                    const float* lse = p.lse_part + unit * kM + rt;  // split sp at lse[sp * units * kM]
                    float m = -INFINITY;
                    for (int sp0 = 0; sp0 < p.splits; sp0 += 8) {  // eight splits' values per L2 round trip
                        float l[8];
#pragma unroll
                        for (int u = 0; u < 8; ++u)
                            l[u] = sp0 + u < p.splits ? __ldcg(lse + (size_t)(sp0 + u) * units * kM) : -INFINITY;
#pragma unroll
                        for (int u = 0; u < 8; ++u) m = fmaxf(m, l[u]);
                    }
                    // a slice: this thread's row rt, columns [32 sl + kSliceCols part, + kSliceCols)
                    constexpr int kSliceCols = 32 / kParts, kSliceChunks = kSliceCols / 4;
                    constexpr int kFly = 16 / kSliceChunks;  // splits' loads in flight: 16 float4 a thread
                    for (;;) {
                        if (gtid == 0) shared_flags[t] = (int)atomicAdd(tk + 1, 1u);
                        group_sync<kGroupThreads>(t);
                        const int sl = shared_flags[t];
                        if (sl >= kMergeSlices) break;  // (the same value for the whole group)
                        const int c0 = 32 * sl + kSliceCols * part;
                        float acc[kSliceChunks][4];
#pragma unroll
                        for (int c = 0; c < kSliceChunks; ++c) acc[c][0] = acc[c][1] = acc[c][2] = acc[c][3] = 0.f;
                        float wsum = 0.f;
                        if (m != -INFINITY) {
                            for (int sp = 0; sp < p.splits; sp += kFly) {
                                float4 v[kFly][kSliceChunks];
                                float w[kFly];
#pragma unroll
                                for (int u = 0; u < kFly; ++u) {
                                    const int sq = sp + u < p.splits ? sp + u : sp;
                                    const float l = __ldcg(lse + (size_t)sq * units * kM);
                                    w[u] = (sp + u < p.splits && l != -INFINITY) ? fast_exp2(l - m) : 0.f;
                                    const float4* src = reinterpret_cast<const float4*>(p.o_part) +
                                                        ((size_t)sq * units + unit) * (32 * kM);
#pragma unroll
                                    for (int c = 0; c < kSliceChunks; ++c)
                                        v[u][c] = __ldcg(src + ((c0 >> 2) + c) * kM + rt);
                                }
#pragma unroll
                                for (int u = 0; u < kFly; ++u) {
                                    if (w[u] == 0.f) continue;  // (a split without visible keys holds zeros)
                                    wsum += w[u];
#pragma unroll
                                    for (int c = 0; c < kSliceChunks; ++c) {
                                        acc[c][0] += w[u] * v[u][c].x;
                                        acc[c][1] += w[u] * v[u][c].y;
                                        acc[c][2] += w[u] * v[u][c].z;
                                        acc[c][3] += w[u] * v[u][c].w;
                                    }
                                }
                            }
                        }
                        const float wi = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
                        for (int c = 0; c < kSliceChunks; c += 2)
                            *reinterpret_cast<uint4*>(stage + rt * 256 + (c0 + c * 4) * 2) = make_uint4(
                                pack_bf16(acc[c][0] * wi, acc[c][1] * wi), pack_bf16(acc[c][2] * wi, acc[c][3] * wi),
                                pack_bf16(acc[c + 1][0] * wi, acc[c + 1][1] * wi),
                                pack_bf16(acc[c + 1][2] * wi, acc[c + 1][3] * wi));
                        group_sync<kGroupThreads>(t);
                        // coalesced copy of the slice's 64 bytes of every row
                        for (int e = gtid; e < kM * 4; e += kGroupThreads) {
                            const int rr = e >> 2, c = 4 * sl + (e & 3);
                            const int pr = row0 + rr;
                            if (pr >= nrows) continue;
                            __nv_bfloat16* orow = p.out + (size_t)b * p.so_b + (size_t)(pr / p.G) * p.so_n +
                                                  (size_t)(hk * p.G + pr % p.G) * p.so_h;
                            *reinterpret_cast<uint4*>(orow + c * 8) =
                                *reinterpret_cast<const uint4*>(stage + rr * 256 + c * 16);
                        }
                    }
                }
                group_sync<kGroupThreads>(t);
                if (gtid == 0) {
                    __threadfence();  // this split's claims come before its finish
                    if (atomicAdd(tk + 2, 1u) == (unsigned int)(p.splits - 1)) {
                        tk[0] = 0u;  // every split is past its last use of the counters: ready for the next launch
                        tk[1] = 0u;
                        tk[2] = 0u;
                    }
                }
            }
            // coalesced copy of the staged bf16 rows to out (one split)
            group_sync<kGroupThreads>(t);
            if (p.splits == 1) {
                for (int e = gtid; e < kM * 16; e += kGroupThreads) {
                    const int rr = e >> 4, c = e & 15;
                    const int pr = row0 + rr;
                    if (pr >= nrows) continue;
                    __nv_bfloat16* orow = p.out + (size_t)b * p.so_b + (size_t)(pr / p.G) * p.so_n +
                                          (size_t)(hk * p.G + pr % p.G) * p.so_h;
                    *reinterpret_cast<uint4*>(orow + c * 8) =
                        *reinterpret_cast<const uint4*>(stage + rr * 256 + c * 16);
                }
            }
        }
    }
    if (!ok && p.status) atomicExch(p.status, 1);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// ------------------------------------------------------------------ host
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)ptr;
    }
    return fn;
}

// 4-D bf16 map: dims (x = head dim, d1, d2, d3), element strides of d1..d3, box (64, b1, b2, 1), 128-byte
// swizzle; boxes reaching past the dims read zeros
static bool make_map(CUtensorMap* m, const void* base, uint64_t d1, uint64_t d2, uint64_t d3, int64_t s1, int64_t s2,
                     int64_t s3, uint32_t b1, uint32_t b2) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[4] = {(cuuint64_t)D, d1, d2, d3};
    const cuuint64_t strides[3] = {(cuuint64_t)s1 * 2, (cuuint64_t)s2 * 2, (cuuint64_t)s3 * 2};
    const cuuint32_t box[4] = {64, b1, b2, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <class C>
static int launch_cfg(const Shape& sh, const Params& p, cudaStream_t stream) {
    const char* who = p.paged ? "mfd_paged_mode_attention" : "mfd_tree_attention";
    CUtensorMap tq, tk, tv;
    const uint32_t nodes_per_tile = (uint32_t)(kM / p.G);
    bool okm = make_map(&tq, sh.q, (uint64_t)p.H, (uint64_t)p.n, (uint64_t)p.bs, sh.sq_h, sh.sq_n, sh.sq_b,
                        (uint32_t)p.G, nodes_per_tile);
    if (p.paged) {  // K and V are gathered with cp.async; the maps are not read
        tk = tq;
        tv = tq;
    } else {
        okm = okm &&
              make_map(&tk, sh.k, (uint64_t)sh.max_keys, (uint64_t)p.Hkv, (uint64_t)p.bs, sh.sk_s, sh.sk_h, sh.sk_b,
                       C::kKt, 1) &&
              make_map(&tv, sh.v, (uint64_t)sh.max_keys, (uint64_t)p.Hkv, (uint64_t)p.bs, sh.sv_s, sh.sv_h, sh.sv_b,
                       C::kKt, 1);
    }
    if (!okm) {
        set_error("%s: could not encode the TMA tensor maps", who);
        return MFD_ERR_CUDA;
    }
    cudaError_t e =
        cudaFuncSetAttribute(tree_attn_tc_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) {
        set_error("%s: %s", who, cudaGetErrorString(e));
        return MFD_ERR_CUDA;
    }
    dim3 grid((unsigned)(p.splits * ((p.mtiles + C::kTiles - 1) / C::kTiles)), (unsigned)p.Hkv, (unsigned)p.bs);
    tree_attn_tc_kernel<C><<<grid, C::kThreads, C::kSmemBytes, stream>>>(tq, tk, tv, p);
    MFD_CHECK_LAUNCH(who);
    return MFD_OK;
}

// The paged gather (cp.async through req_to_token, issued by one warp) is the paged launch's bound, so pairs of its
// M-tiles share each gathered K/V tile (SGLang mode attention, 32 requests: 926 -> 716 us).  The dense TMA path keeps
// one M-tile per CTA: paired, its verify attention took 2324 against 2034 us at 256 requests.
int launch(const Shape& sh, const Params& p, cudaStream_t stream) {
    return (p.paged && p.mtiles >= 2) ? launch_cfg<CfgPair>(sh, p, stream) : launch_cfg<CfgRow>(sh, p, stream);
}

}  // namespace tca
}  // namespace mfd
