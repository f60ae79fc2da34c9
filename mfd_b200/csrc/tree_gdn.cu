// tree_gdn.cu -- tree verification of one gated-delta-rule (Gated DeltaNet) layer from the committed state, with
// the state contractions on the tcgen05 tensor cores.
//
// For the nodes of a draft tree in topological order (parents before children), value head h (key head
// hk = h / (H / HK)), G = log decay summed along the root path, anc(i) = ancestors of i and i itself:
//
//   u_i + sum_{j in anc(i), j != i} beta_i e^{G_i - G_j} (k_i . k_j) u_j = beta_i (v_i - e^{G_i} S0^T k_i)
//   o_i = e^{G_i} S0^T q_i + sum_{j in anc(i)} e^{G_i - G_j} (q_i . k_j) u_j
//   S_i = e^{G_i} S0 + sum_{j in anc(i)} e^{G_i - G_j} k_j u_j^T           (optional per-node states)
//
// which is inference/hf/tree_gdn_kernel.py:1-20 and 153-171 (tree_gdn: _tree_kkt + solve_tril + _tree_u), the
// state formula of inference/hf/qwen35_tree.py:12-27 and 134-137 applied to every node, and the math spec of
// tests/test_gdn_tree_math.py:29-60.
//
// tree_gdn_uo_kernel: one CTA per (value head, 32 value columns), 256 threads, 512 TMEM columns.
//   - K (all node tiles), Q (one 128-node tile at a time) and the S0 column slice, transposed and split into bf16
//     hi + lo (so the products keep fp32 accuracy), are staged in shared memory as 128-byte-swizzled K-major UMMA
//     operands;
//   - tcgen05.mma (M = 128 nodes, K = Dk): S0^T k_i and S0^T q_i of the slice (N = 32, hi and lo accumulated) and,
//     per pair of node tiles, the Gram products k_i . k_j and q_i . k_j (N = 128), accumulators in TMEM;
//   - the Gram tiles are read back with tcgen05.ld and only ancestor pairs are kept (one per node and depth);
//   - a tree's ancestor set is its root path, one node per depth, so the unit lower triangular system is solved
//     exactly by depth levels (every node of one depth at once, fp32 on the CUDA cores) instead of by inverting
//     dense diagonal blocks (fla solve_tril); o then sums the path terms.
// tree_gdn_states_kernel: one CTA per (value head, node residue), S0[h] kept in shared memory.  For
//   node i the path contraction sum_j (e^{G_i - G_j} u_j) k_j^T is one tcgen05.mma of M = 128 value rows, N = Dk key
//   columns and K = 64: the path's scaled u split into bf16 hi and lo against k twice, 32 path nodes per pass
//   (deeper paths accumulate more passes); the epilogue adds e^{G_i} S0 and streams the 64 KB state to memory with
//   coalesced stores (HBM-write bound: n H Dk Dv 4 bytes).
// Limits: n <= 384 (three 128-node tiles), Dk <= 128 and a multiple of 8, Dv a multiple of 4 (<= 128 with
// states); the ancestor pairs (sum over nodes of depth + 1) must fit the u/o kernel's shared memory (every tree of up
// to 128 nodes does; at 257 nodes about 6.8 thousand pairs, i.e. trees up to average depth 25).  Beyond that the
// status word receives MFD_ERR_CAPACITY.
#include "common.cuh"
#include "tcgen05.cuh"

namespace gdn {
using namespace mfd;

constexpr int kThreads = 256;
constexpr int kSlice = 32;         // value columns per u/o CTA
constexpr int kVs = kSlice + 2;    // row stride (bf16 elements) of the staged v slice: 17 words, odd
constexpr int kUs = kSlice + 1;    // row stride of the u rows in shared memory (odd: a warp reading one column of 32
                                   // different rows hits 32 different banks)
constexpr int kTile = 128;         // nodes per M-tile
constexpr int kMaxTiles = 3;
constexpr int kMaxNodes = kMaxTiles * kTile;
constexpr int kMaxDk = 128;
constexpr int kMaxDvStates = 128;
constexpr int kSmemCap = 227 * 1024;
constexpr int kSlack = 1024;              // the swizzled operands need a 1024-byte aligned base
constexpr int kTileBytes = kTile * 256;   // 128 rows x 128 K bf16 (two 64-element chunks)
constexpr int kSliceBytes = kSlice * 256; // the S0 slice operand: 32 rows x 128 K
constexpr int kColKS = 0, kColQS = 96, kColKK = 256, kColQK = 384;  // TMEM columns of the u/o kernel
constexpr uint32_t kTries = 1u << 22;     // bounded mbarrier polls

struct Params {
    const __nv_bfloat16* q;  // [n, HK, Dk], node stride sq
    const __nv_bfloat16* k;  // [n, HK, Dk], node stride sk
    const __nv_bfloat16* v;  // [n, H, Dv], node stride sv
    int64_t sq, sk, sv;
    const float* g;     // [n, H], node stride sg (G, the path sums)
    const float* beta;  // [n, H], node stride sb
    int64_t sg, sb;
    const float* s0;    // [H, Dk, Dv]
    const int8_t* anc;  // [n, n], row stride sa; anc[i][j] != 0 iff j is an ancestor of i or j == i
    int64_t sa;
    int n, H, HK, Dk, Dv;
    float* u;       // [n, H, Dv]
    float* o;       // [n, H, Dv]
    float* states;  // [n, H, Dk, Dv] or null
    int* status;    // optional: 0 ok, 1 not the ancestor matrix of a topologically ordered tree, MFD_ERR_CAPACITY
    int pair_cap;   // ancestor pairs the u/o kernel's shared memory holds
};

__host__ __device__ constexpr int a16(int x) { return (x + 15) & ~15; }

// u/o kernel shared memory, byte offsets from the 1024-aligned base
struct UoLayout {
    int kt, qt, sbh, sbl, bits, gg, eg, bb, depth, off, lvl, lstart, lcnt, vs, uu, node, mm, pq, bars, total;
    int words;
};
__host__ __device__ inline UoLayout uo_layout(int n, int mt, int pair_cap) {
    UoLayout L{};
    L.words = (n + 31) / 32;
    int off = 0;
    L.kt = off, off += mt * kTileBytes;
    L.qt = off, off += kTileBytes;
    L.sbh = off, off += kSliceBytes;
    L.sbl = off, off += kSliceBytes;
    L.bits = off, off += a16(n * L.words * 4);
    L.gg = off, off += a16(n * 4);
    L.eg = off, off += a16(n * 4);
    L.bb = off, off += a16(n * 4);
    L.depth = off, off += a16(n * 2);
    L.off = off, off += a16((n + 1) * 4);
    L.lvl = off, off += a16(n * 2);
    L.lstart = off, off += a16((n + 1) * 4);
    L.lcnt = off, off += a16((n + 1) * 4);
    L.vs = off, off += a16(n * kVs * 2);
    L.uu = L.kt;  // the right-hand side / u rows reuse the k tiles once every MMA has completed (n * 132 bytes)
    L.bars = off, off += 64;
    L.node = off, off += a16(pair_cap * 2);
    L.mm = off, off += a16(pair_cap * 4);
    L.pq = off, off += a16(pair_cap * 4);
    L.total = off;
    return L;
}
// the most ancestor pairs that fit next to everything else
inline int uo_pair_cap(int n, int mt) {
    const int fixed = uo_layout(n, mt, 0).total + kSlack + 64;
    const int cap = (kSmemCap - fixed) / 10;
    const int need = n * (n + 1) / 2;
    return cap < need ? cap : need;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void proxy_fence() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ uint32_t bf16_bits(float x) { return (uint32_t)__bfloat16_as_ushort(__float2bfloat16(x)); }
// x = hi + lo, both bf16: the pair carries x to about 2^-16 relative
__device__ __forceinline__ void split2(float x, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat16 h = __float2bfloat16(x);
    hi = (uint32_t)__bfloat16_as_ushort(h);
    lo = bf16_bits(x - __bfloat162float(h));
}

// Rows [row0, row0 + 128) of a [n, *, Dk] bf16 tensor (node stride `stride`, head offset `hoff` elements) into a
// 128-row swizzled K-major operand; rows past n and columns past Dk are zero.
__device__ __forceinline__ void stage_rows(uint32_t dst, const __nv_bfloat16* base, int64_t stride, int64_t hoff,
                                           int row0, int n, int Dk) {
    for (int e = threadIdx.x; e < kTile * 16; e += kThreads) {
        const int r = e >> 4, gr = e & 15;  // granule gr = elements 8 gr .. 8 gr + 7
        const int i = row0 + r;
        const bool live = i < n && gr * 8 < Dk;
        const __nv_bfloat16* src = live ? base + (int64_t)i * stride + hoff + gr * 8 : base;
        cp_async16(dst + sw128_offset(r, gr * 8, kTile), src, live ? 16 : 0);
    }
}

// The n x n ancestor matrix into shared memory (row stride rs bytes): a warp per row, each lane a column run,
// four rows' loads in flight per warp before their stores.
__device__ __forceinline__ void stage_anc(int8_t* dst, int64_t rs, const int8_t* anc, int64_t sa, int n) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r0 = warp * 4; r0 < n; r0 += (kThreads / 32) * 4) {
        for (int c0 = 0; c0 < n; c0 += 128) {
            int8_t v[4][4];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int x = 0; x < 4; ++x) {
                    const int row = r0 + r, col = c0 + 32 * x + lane;
                    v[r][x] = (row < n && col < n) ? anc[(int64_t)row * sa + col] : (int8_t)0;
                }
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int x = 0; x < 4; ++x) {
                    const int row = r0 + r, col = c0 + 32 * x + lane;
                    if (row < n && col < n) dst[(int64_t)row * rs + col] = v[r][x];
                }
        }
    }
}

// Ancestor bitsets of every node (one warp per row), then the checks that make the mask a topologically ordered
// tree, the depths, the pair offsets, the path lists (root first) and the nodes grouped by depth.  Returns false
// (uniformly) when the mask is not such a tree or the pairs exceed the capacity (*code: 1 or MFD_ERR_CAPACITY).
__device__ bool build_tree(const Params& p, unsigned char* sm, const UoLayout& L, const int8_t* rows, int64_t rs,
                           int* flags, int* code) {
    const int n = p.n, words = L.words;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t* bits = (uint32_t*)(sm + L.bits);
    uint16_t* depth = (uint16_t*)(sm + L.depth);
    int* off = (int*)(sm + L.off);
    uint16_t* lvl = (uint16_t*)(sm + L.lvl);
    int* lstart = (int*)(sm + L.lstart);
    int* lcnt = (int*)(sm + L.lcnt);
    uint16_t* node = (uint16_t*)(sm + L.node);
    for (int i = warp; i < n; i += kThreads / 32) {
        const int8_t* row = rows + (int64_t)i * rs;
        for (int w = 0; w < words; ++w) {
            const int c = w * 32 + lane;
            const uint32_t b = __ballot_sync(MFD_FULL_MASK, c < n && row[c] != 0);
            if (lane == 0) bits[i * words + w] = b;
        }
    }
    for (int d = threadIdx.x; d <= n; d += kThreads) lcnt[d] = 0;
    __syncthreads();
    // i in anc(i), nothing above i, and anc(i) = anc(parent) + {i} with parent = the largest strict ancestor
    for (int i = threadIdx.x; i < n; i += kThreads) {
        const uint32_t* bi = bits + i * words;
        bool ok = (bi[i >> 5] >> (i & 31)) & 1u;
        int cnt = 0, parent = -1;
        for (int w = 0; w < words; ++w) {
            const uint32_t b = bi[w];
            const int lo = w * 32;
            if (lo > i) {
                ok &= b == 0u;
                continue;
            }
            if (lo + 31 > i) ok &= (b >> (i - lo)) <= 1u;
            cnt += __popc(b);
            uint32_t strict = b;
            if (i < lo + 32) strict &= ~(1u << (i - lo));
            if (strict) parent = lo + 31 - __clz(strict);
        }
        if (ok && parent >= 0) {
            const uint32_t* bp = bits + parent * words;
            for (int w = 0; w < words; ++w) {
                uint32_t want = bp[w];
                if ((i >> 5) == w) want |= 1u << (i & 31);
                ok &= want == bi[w];
            }
        }
        if (!ok) atomicOr(&flags[0], 1);
        const int d = ok ? cnt - 1 : 0;
        depth[i] = (uint16_t)d;
        // one atomic per warp for the maximum and one per distinct depth for the level counts
        const uint32_t active = __activemask();
        const int dmax = __reduce_max_sync(active, d);
        if (lane == __ffs(active) - 1) atomicMax(&flags[1], dmax);
        const uint32_t same = __match_any_sync(active, d);
        if (lane == __ffs(same) - 1) atomicAdd(&lcnt[d], __popc(same));
    }
    __syncthreads();
    if (flags[0]) {
        *code = 1;
        return false;
    }
    if (warp == 0) {  // exclusive prefixes: pair offsets (depth + 1 per node) and level starts
        const int per = (n + 32) / 32;
        int s = 0, sl = 0;
        for (int t = 0; t < per; ++t) {
            const int i = lane * per + t;
            if (i < n) s += depth[i] + 1;
            if (i <= n) sl += lcnt[i];
        }
        int incl = s, incl_l = sl;
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(MFD_FULL_MASK, incl, o), yl = __shfl_up_sync(MFD_FULL_MASK, incl_l, o);
            if (lane >= o) incl += y, incl_l += yl;
        }
        int run = incl - s, run_l = incl_l - sl;
        for (int t = 0; t < per; ++t) {
            const int i = lane * per + t;
            if (i < n) off[i] = run, run += depth[i] + 1;
            if (i <= n) lstart[i] = run_l, run_l += lcnt[i];
        }
        if (lane == 31) {
            off[n] = incl;
            if (incl > p.pair_cap) flags[2] = 1;
        }
    }
    __syncthreads();
    if (flags[2]) {
        *code = MFD_ERR_CAPACITY;
        return false;
    }
    for (int d = threadIdx.x; d <= n; d += kThreads) lcnt[d] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += kThreads) {
        const int d = depth[i];
        const uint32_t active = __activemask();
        const uint32_t same = __match_any_sync(active, d);
        const int leader = __ffs(same) - 1;
        int base = 0;
        if (lane == leader) base = atomicAdd(&lcnt[d], __popc(same));
        base = __shfl_sync(same, base, leader);
        lvl[lstart[d] + base + __popc(same & ((1u << lane) - 1u))] = (uint16_t)i;
    }
    for (int i = warp; i < n; i += kThreads / 32) {  // the set bits of row i in ascending order (root first)
        int base = off[i];
        for (int w = 0; w < words; ++w) {
            const uint32_t b = bits[i * words + w];
            if ((b >> lane) & 1u) node[base + __popc(b & ((1u << lane) - 1u))] = (uint16_t)(w * 32 + lane);
            base += __popc(b);
        }
    }
    __syncthreads();
    return true;
}

template <int MT>
__global__ void __launch_bounds__(kThreads, 1) tree_gdn_uo_kernel(const Params p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t pad = (1024u - (smem_addr(smem_raw) & 1023u)) & 1023u;
    unsigned char* sm = smem_raw + pad;
    const uint32_t sb = smem_addr(sm);
    const int n = p.n, Dk = p.Dk, Dv = p.Dv;
    const UoLayout L = uo_layout(n, MT, p.pair_cap);
    const int h = blockIdx.x, c0 = blockIdx.y * kSlice;
    const int hk = h / (p.H / p.HK);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, quarter = warp & 3;
    const bool report = blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0 && p.status;
    uint64_t* bar = (uint64_t*)(sm + L.bars);
    uint32_t* tslot = (uint32_t*)(sm + L.bars + 8);
    int* flags = (int*)(sm + L.bars + 16);  // [0] not a tree, [1] max depth, [2] pair capacity, [3] a wait gave up
    float* gg = (float*)(sm + L.gg);
    float* eg = (float*)(sm + L.eg);
    float* bb = (float*)(sm + L.bb);
    const uint32_t* bits = (const uint32_t*)(sm + L.bits);
    const uint16_t* depth = (const uint16_t*)(sm + L.depth);
    const int* off = (const int*)(sm + L.off);
    const uint16_t* lvl = (const uint16_t*)(sm + L.lvl);
    const int* lstart = (const int*)(sm + L.lstart);
    const uint16_t* node = (const uint16_t*)(sm + L.node);
    float* uu = (float*)(sm + L.uu);  // [n][32]: right-hand side, then u
    float* mm = (float*)(sm + L.mm);  // [pairs]: beta_i e^{G_i - G_j} k_i . k_j (0 for j == i)
    float* pq = (float*)(sm + L.pq);  // [pairs]: e^{G_i - G_j} q_i . k_j

    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        for (int f = 0; f < 4; ++f) flags[f] = 0;
        mbar_fence_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_addr(tslot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    // ---- operands: every k tile, the first q tile, the S0 slice (transposed, split hi / lo); G, e^G, beta
    for (int t = 0; t < MT; ++t)
        stage_rows(sb + L.kt + t * kTileBytes, p.k, p.sk, (int64_t)hk * Dk, t * kTile, n, Dk);
    stage_rows(sb + L.qt, p.q, p.sq, (int64_t)hk * Dk, 0, n, Dk);
    const float* s0h = p.s0 + (int64_t)h * Dk * Dv;
    for (int e = threadIdx.x; e < kSlice * (kMaxDk / 8); e += kThreads) {
        const int c = e & (kSlice - 1), a8 = (e / kSlice) * 8;  // lanes: consecutive columns of the same 8 rows
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int x = 0; x < 4; ++x) {
            float v0 = 0.f, v1 = 0.f;
            if (c0 + c < Dv && a8 + 2 * x < Dk) v0 = s0h[(int64_t)(a8 + 2 * x) * Dv + c0 + c];
            if (c0 + c < Dv && a8 + 2 * x + 1 < Dk) v1 = s0h[(int64_t)(a8 + 2 * x + 1) * Dv + c0 + c];
            uint32_t h0, l0, h1, l1;
            split2(v0, h0, l0);
            split2(v1, h1, l1);
            hi[x] = h0 | (h1 << 16);
            lo[x] = l0 | (l1 << 16);
        }
        const uint32_t o = sw128_offset(c, a8, kSlice);
        *reinterpret_cast<uint4*>(sm + L.sbh + o) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(sm + L.sbl + o) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    for (int i0 = 0; i0 < n; i0 += 2 * kThreads) {  // both rows' loads in flight, then the stores
        float G[2], B[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int i = i0 + u * kThreads + threadIdx.x;
            G[u] = i < n ? p.g[(int64_t)i * p.sg + h] : 0.f;
            B[u] = i < n ? p.beta[(int64_t)i * p.sb + h] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int i = i0 + u * kThreads + threadIdx.x;
            if (i < n) {
                gg[i] = G[u];
                eg[i] = expf(G[u]);
                bb[i] = B[u];
            }
        }
    }
    // the ancestor matrix into the (still unused) pair area when it fits, else read in place
    const bool anc_smem = n * n <= L.total - L.node;
    if (anc_smem) stage_anc((int8_t*)(sm + L.node), n, p.anc, p.sa, n);
    // the v slice of every node (lanes along the columns: coalesced), for the right-hand side
    uint16_t* vs = (uint16_t*)(sm + L.vs);
    for (int e0 = 0; e0 < n * kSlice; e0 += 8 * kThreads) {  // eight loads in flight per thread, then the stores
        uint16_t x[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int e = e0 + u * kThreads + threadIdx.x, i = e / kSlice, c = e % kSlice;
            x[u] = (e < n * kSlice && c0 + c < Dv)
                       ? __bfloat16_as_ushort(p.v[(int64_t)i * p.sv + (int64_t)h * Dv + c0 + c]) : (uint16_t)0;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int e = e0 + u * kThreads + threadIdx.x;
            if (e < n * kSlice) vs[(e / kSlice) * kVs + e % kSlice] = x[u];
        }
    }
    cp_async_wait_all();
    proxy_fence();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    int code = 0;
    const bool tree_ok = anc_smem ? build_tree(p, sm, L, (const int8_t*)(sm + L.node), n, flags, &code)
                                  : build_tree(p, sm, L, p.anc, p.sa, flags, &code);
    if (!tree_ok) {
        if (report) *p.status = code;
    } else {
        if (report) *p.status = 0;
        const int ksteps = (Dk + 15) / 16;
        uint32_t phase = 0;
        for (int t = 0; t < MT; ++t) {
            if (t > 0) {  // the previous tile's MMAs have completed (waited below); reload q
                stage_rows(sb + L.qt, p.q, p.sq, (int64_t)hk * Dk, t * kTile, n, Dk);
                cp_async_wait_all();
                proxy_fence();
                __syncthreads();
            }
            if (threadIdx.x == 0) {
                tc_fence_after();
                constexpr uint32_t kIdS = idesc_bf16(kTile, kSlice, 0);
                constexpr uint32_t kIdG = idesc_bf16(kTile, kTile, 0);
                const uint32_t ka = sb + L.kt + t * kTileBytes;
                for (int ks = 0; ks < ksteps; ++ks) {  // S0^T k and S0^T q: hi then lo into one accumulator
                    umma(tmem + kColKS + 32 * t, sw128_desc(ka, ks, kTile), sw128_desc(sb + L.sbh, ks, kSlice), kIdS,
                         ks > 0);
                    umma(tmem + kColQS + 32 * t, sw128_desc(sb + L.qt, ks, kTile), sw128_desc(sb + L.sbh, ks, kSlice),
                         kIdS, ks > 0);
                }
                for (int ks = 0; ks < ksteps; ++ks) {
                    umma(tmem + kColKS + 32 * t, sw128_desc(ka, ks, kTile), sw128_desc(sb + L.sbl, ks, kSlice), kIdS, 1);
                    umma(tmem + kColQS + 32 * t, sw128_desc(sb + L.qt, ks, kTile), sw128_desc(sb + L.sbl, ks, kSlice),
                         kIdS, 1);
                }
                (void)kIdG;
            }
            for (int nj = 0; nj <= t; ++nj) {
                if (threadIdx.x == 0) {
                    constexpr uint32_t kIdG = idesc_bf16(kTile, kTile, 0);
                    const uint32_t ka = sb + L.kt + t * kTileBytes, kb = sb + L.kt + nj * kTileBytes;
                    for (int ks = 0; ks < ksteps; ++ks) {
                        umma(tmem + kColKK, sw128_desc(ka, ks, kTile), sw128_desc(kb, ks, kTile), kIdG, ks > 0);
                        umma(tmem + kColQK, sw128_desc(sb + L.qt, ks, kTile), sw128_desc(kb, ks, kTile), kIdG, ks > 0);
                    }
                    umma_commit(bar);
                }
                // one thread polls the barrier; the others sleep in bar.sync instead of spinning on it
                if (threadIdx.x == 0 && !mbar_wait(bar, phase, kTries)) flags[3] = 1;
                phase ^= 1u;
                __syncthreads();
                tc_fence_after();
                // ancestor pairs of this tile pair: warps 0-3 read k_i . k_j, warps 4-7 q_i . k_j
                const bool qk = warp >= 4;
                const int i = t * kTile + quarter * 32 + lane;
                const int imax = t * kTile + quarter * 32 + 31;
#pragma unroll 1
                for (int c4 = 0; c4 < 4; ++c4) {
                    const int jb = nj * kTile + c4 * 32;
                    if (jb > imax || jb >= n || t * kTile + quarter * 32 >= n) continue;  // warp-uniform
                    float val[32];
                    tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (qk ? kColQK : kColKK) + c4 * 32, val);
                    if (i < n) {
                        const uint32_t word = bits[i * L.words + (jb >> 5)];
                        const int o0 = off[i];
                        const float Gi = gg[i], bi = bb[i];
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj) {
                            if (!((word >> jj) & 1u)) continue;
                            const int j = jb + jj;
                            const int slot = o0 + depth[j];
                            const float gam = expf(Gi - gg[j]);
                            if (qk) pq[slot] = gam * val[jj];
                            else mm[slot] = j == i ? 0.f : bi * gam * val[jj];
                        }
                    }
                }
                tc_fence_before();
                __syncthreads();
            }
        }
        // ---- right-hand side beta_i (v_i - e^{G_i} S0^T k_i): thread = node (its TMEM lane), 32 columns
        for (int t = warp >> 2; t < MT; t += 2) {
            if (t * kTile + quarter * 32 >= n) continue;
            float ks_[32];
            tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + kColKS + 32 * t, ks_);
            const int i = t * kTile + quarter * 32 + lane;
            if (i >= n) continue;
#pragma unroll
            for (int c = 0; c < kSlice; ++c) {
                const float vv = __uint_as_float((uint32_t)vs[i * kVs + c] << 16);
                uu[i * kUs + c] = bb[i] * (vv - eg[i] * ks_[c]);
            }
        }
        __syncthreads();
        // ---- forward substitution by depth: every strict ancestor of a depth-d node has depth < d
        const int max_depth = flags[1];
        for (int d = 1; d <= max_depth; ++d) {
            const int l0 = lstart[d], items = (lstart[d + 1] - l0) * kSlice;
            for (int e = threadIdx.x; e < items; e += kThreads) {
                const int i = lvl[l0 + e / kSlice], c = e % kSlice;
                const int o0 = off[i];
                float acc = uu[i * kUs + c];
                for (int tt = 0; tt < d; ++tt) acc = fmaf(-mm[o0 + tt], uu[node[o0 + tt] * kUs + c], acc);
                uu[i * kUs + c] = acc;
            }
            __syncthreads();
        }
        // ---- outputs: o_i = e^{G_i} S0^T q_i + sum over the path of e^{G_i - G_j} (q_i . k_j) u_j, and u
        for (int t = warp >> 2; t < MT; t += 2) {
            if (t * kTile + quarter * 32 >= n) continue;
            float qs[32];
            tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + kColQS + 32 * t, qs);
            const int i = t * kTile + quarter * 32 + lane;
            if (i >= n) continue;
            const int o0 = off[i], d = depth[i];
            float acc[32];
#pragma unroll
            for (int c = 0; c < kSlice; ++c) acc[c] = eg[i] * qs[c];
            for (int tt = 0; tt <= d; ++tt) {
                const float w = pq[o0 + tt];
                const float* ur = uu + node[o0 + tt] * kUs;
#pragma unroll
                for (int c = 0; c < kSlice; ++c) acc[c] = fmaf(w, ur[c], acc[c]);
            }
            const int64_t at = ((int64_t)i * p.H + h) * Dv + c0;
            const float* ui = uu + i * kUs;
#pragma unroll
            for (int c = 0; c < kSlice; c += 4) {
                if (c0 + c >= Dv) break;
                *reinterpret_cast<float4*>(p.o + at + c) = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
                *reinterpret_cast<float4*>(p.u + at + c) = make_float4(ui[c], ui[c + 1], ui[c + 2], ui[c + 3]);
            }
        }
        if (flags[3] && report) *p.status = 3;  // a bounded wait gave up: outputs unspecified
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
}

// ---------------------------------------------------------------------------------------------- states
// CTAs of 128 threads (one warp per TMEM lane quarter), four per SM so that one CTA's stores overlap the others'
// operand builds and MMAs; CTA (h, s) takes the nodes i = s, s + S, ... of value head h.  Per node: its root path
// from the ancestor row; operand A (128 value rows x 64 K: e^{G_i - G_j} u_j split hi | lo) and B (key rows x 64 K:
// k_j twice), 32 path nodes per pass, 16 KB each, only the path's nodes loaded; one tcgen05.mma pass (M = 128 value
// rows, N = Dk) into 128 TMEM columns; the epilogue adds e^{G_i} S0 (read through L2) and the lanes of a warp write
// 128 contiguous bytes of a state row per store.
constexpr int kStThreads = 128;
constexpr int kStCtasPerSm = 4;
constexpr int kStOpBytes = 128 * 128;
constexpr int kStA = 0, kStB = kStOpBytes;
constexpr int kStPath = 2 * kStOpBytes;
constexpr int kStGam = kStPath + kMaxNodes * 2;
constexpr int kStG = kStGam + kMaxNodes * 4;
constexpr int kStBar = kStG + kMaxNodes * 4;
constexpr int kStTotal = kStBar + 64;

// FIXED: Dk = Dv = 128 known at compile time (the strides become immediate offsets); 0: runtime sizes.
template <int FIXED>
__global__ void __launch_bounds__(kStThreads, kStCtasPerSm) tree_gdn_states_kernel(const Params p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t pad = (1024u - (smem_addr(smem_raw) & 1023u)) & 1023u;
    unsigned char* sm = smem_raw + pad;
    const uint32_t sb = smem_addr(sm);
    const int n = p.n, H = p.H;
    const int Dk = FIXED ? FIXED : p.Dk, Dv = FIXED ? FIXED : p.Dv;
    const int nk = (Dk + 15) & ~15;  // N: key columns, a multiple of 16
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.x, hk = h / (H / p.HK);
    uint16_t* path = (uint16_t*)(sm + kStPath);
    float* gam = (float*)(sm + kStGam);
    float* gcol = (float*)(sm + kStG);
    uint64_t* bar = (uint64_t*)(sm + kStBar);
    uint32_t* tslot = (uint32_t*)(sm + kStBar + 8);
    int* scnt = (int*)(sm + kStBar + 16);  // [0] a wait gave up, [1..4] per-warp counts
    const int8_t* arows = p.anc;
    const int64_t ars = p.sa;
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        scnt[0] = 0;
        mbar_fence_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 128;" ::"r"(smem_addr(tslot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    for (int i0 = 0; i0 < n; i0 += 4 * kStThreads) {  // four loads in flight per thread
        float G[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int i = i0 + u * kStThreads + threadIdx.x;
            G[u] = i < n ? p.g[(int64_t)i * p.sg + h] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (i0 + u * kStThreads + threadIdx.x < n) gcol[i0 + u * kStThreads + threadIdx.x] = G[u];
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t idesc = idesc_bf16(128, nk, 0);
    const float* s0h = p.s0 + (int64_t)h * Dk * Dv;
    uint32_t phase = 0;
    const int words = (n + 31) / 32;
    const int row = threadIdx.x;  // operand row: value row c of A, key row a of B
    for (int i = blockIdx.y; i < n && !scnt[0]; i += gridDim.y) {
        // ---- the root path of node i, ascending: the set entries of its ancestor row (prefix sums over warps)
        const int8_t* arow = arows + (int64_t)i * ars;
        int total = 0;
        for (int w0 = 0; w0 < words; w0 += kStThreads / 32) {
            const int w = w0 + warp;
            const int c = w * 32 + lane;
            const uint32_t bm = __ballot_sync(MFD_FULL_MASK, w < words && c < n && c <= i && arow[c] != 0);
            if (lane == 0) scnt[1 + warp] = __popc(bm);
            __syncthreads();
            int before = total, all = total;
            for (int x = 0; x < kStThreads / 32; ++x) {
                if (x < warp) before += scnt[1 + x];
                all += scnt[1 + x];
            }
            if ((bm >> lane) & 1u) path[before + __popc(bm & ((1u << lane) - 1u))] = (uint16_t)c;
            total = all;
            __syncthreads();
        }
        const float Gi = gcol[i];
        for (int t = threadIdx.x; t < total; t += kStThreads) gam[t] = expf(Gi - gcol[path[t]]);
        __syncthreads();
        // ---- the contraction, 32 path nodes per pass: D[c][a] += sum_t (gam_t u_t[c]) k_t[a] (hi and lo parts)
        const int passes = (total + 31) / 32;
        for (int ps = 0; ps < passes; ++ps) {
#pragma unroll
            for (int grp = 0; grp < 2; ++grp) {
                const int t0 = ps * 32 + 16 * grp;
                uint32_t ah[8], al[8], kb[8];  // A: scaled u hi / lo (row = value index c); B: k (row = key index a)
#pragma unroll
                for (int x = 0; x < 8; ++x) ah[x] = al[x] = kb[x] = 0u;
                if (t0 < total) {  // (uniform) only the group's path nodes are loaded and converted
                    float uv[16];
                    uint32_t kv[16];
                    const float* ub = p.u + (int64_t)h * Dv + row;
                    const __nv_bfloat16* kbp = p.k + (int64_t)hk * Dk + row;
#pragma unroll
                    for (int x = 0; x < 16; ++x) {
                        uv[x] = 0.f;
                        kv[x] = 0u;
                        if (t0 + x >= total) break;
                        const int j = path[t0 + x];
                        if (row < Dv) uv[x] = gam[t0 + x] * ub[(int64_t)j * H * Dv];
                        if (row < Dk) kv[x] = (uint32_t)__bfloat16_as_ushort(kbp[(int64_t)j * p.sk]);
                    }
#pragma unroll
                    for (int x = 0; x < 8; ++x) {
                        if (t0 + 2 * x >= total) break;
                        uint32_t h0, l0, h1, l1;
                        split2(uv[2 * x], h0, l0);
                        split2(uv[2 * x + 1], h1, l1);
                        ah[x] = h0 | (h1 << 16);
                        al[x] = l0 | (l1 << 16);
                        kb[x] = kv[2 * x] | (kv[2 * x + 1] << 16);
                    }
                }
                // A[row][16 grp + ..] = hi, A[row][32 + 16 grp + ..] = lo; B[row][16 grp + ..] = B[row][32 + ..] = k
#pragma unroll
                for (int g8 = 0; g8 < 2; ++g8) {
                    const int kk = 16 * grp + 8 * g8;
                    const uint4 vh = make_uint4(ah[4 * g8], ah[4 * g8 + 1], ah[4 * g8 + 2], ah[4 * g8 + 3]);
                    const uint4 vl = make_uint4(al[4 * g8], al[4 * g8 + 1], al[4 * g8 + 2], al[4 * g8 + 3]);
                    const uint4 vk = make_uint4(kb[4 * g8], kb[4 * g8 + 1], kb[4 * g8 + 2], kb[4 * g8 + 3]);
                    *reinterpret_cast<uint4*>(sm + kStA + sw128_offset(row, kk, 128)) = vh;
                    *reinterpret_cast<uint4*>(sm + kStA + sw128_offset(row, 32 + kk, 128)) = vl;
                    *reinterpret_cast<uint4*>(sm + kStB + sw128_offset(row, kk, 128)) = vk;
                    *reinterpret_cast<uint4*>(sm + kStB + sw128_offset(row, 32 + kk, 128)) = vk;
                }
            }
            proxy_fence();
            tc_fence_before();
            __syncthreads();
            if (threadIdx.x == 0) {
                tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < 4; ++ks)
                    umma(tmem, sw128_desc(sb + kStA, ks, 128), sw128_desc(sb + kStB, ks, 128), idesc, (ps > 0 || ks > 0));
                umma_commit(bar);
            }
            // one thread polls the barrier; the others sleep in bar.sync (the operands may be rewritten only after
            // the MMAs that read them)
            if (threadIdx.x == 0 && !mbar_wait(bar, phase, kTries)) scnt[0] = 1;
            phase ^= 1u;
            __syncthreads();
            tc_fence_after();
        }
        if (scnt[0]) break;
        // ---- epilogue: this warp's TMEM lanes are value columns c; 32 key rows at a time, e^{G_i} S0 added; the
        // lanes of a warp write consecutive c of one state row (128 contiguous bytes per store)
        const int c = warp * 32 + lane;
        const float e = expf(Gi);
        const float* sp = s0h + c;
        float* op = p.states + ((int64_t)i * H + h) * Dk * Dv + c;
#pragma unroll 1
        for (int a0 = 0; a0 < Dk; a0 += 32) {
            if (warp * 32 >= Dv) break;  // warp-uniform
            const bool live = c < Dv;
            const int rows = Dk - a0 < 32 ? Dk - a0 : 32;
            float s0v[32];
            const float* sa = sp + (int64_t)a0 * Dv;
            if (live && rows == 32) {  // the common case: no per-row predicate, pointer steps only
#pragma unroll
                for (int x = 0; x < 32; ++x) {
                    s0v[x] = __ldg(sa);
                    sa += Dv;
                }
            } else {
#pragma unroll
                for (int x = 0; x < 32; ++x) {
                    s0v[x] = (live && x < rows) ? __ldg(sa) : 0.f;
                    sa += Dv;
                }
            }
            float acc[32];
            tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + a0, acc);
            float* oa = op + (int64_t)a0 * Dv;
            if (live && rows == 32) {
#pragma unroll
                for (int x = 0; x < 32; ++x) {
                    __stcs(oa, fmaf(e, s0v[x], acc[x]));
                    oa += Dv;
                }
            } else if (live) {
#pragma unroll
                for (int x = 0; x < 32; ++x) {
                    if (x < rows) __stcs(oa, fmaf(e, s0v[x], acc[x]));
                    oa += Dv;
                }
            }
        }
        tc_fence_before();
        __syncthreads();  // TMEM and the path are reused by the next node
    }
    if (scnt[0] && threadIdx.x == 0 && p.status) atomicExch(p.status, 3);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 128;" ::"r"(tmem));
    }
}

}  // namespace gdn

extern "C" int mfd_tree_gdn(const void* q, int64_t sq, const void* k, int64_t sk, const void* v, int64_t sv,
                            const float* g_cum, int64_t sg, const float* beta, int64_t sb, const float* s0,
                            const int8_t* anc, int64_t sa, int64_t n, int64_t num_heads, int64_t num_k_heads,
                            int64_t dk, int64_t dv, float* u, float* o, float* states, int* status, void* stream) {
    using namespace gdn;
    if (n < 0 || num_heads <= 0 || num_k_heads <= 0 || dk <= 0 || dv <= 0 || num_heads % num_k_heads) {
        mfd::set_error("mfd_tree_gdn: invalid sizes n=%lld H=%lld HK=%lld Dk=%lld Dv=%lld", (long long)n,
                       (long long)num_heads, (long long)num_k_heads, (long long)dk, (long long)dv);
        return MFD_ERR_INVALID;
    }
    if (n == 0) return MFD_OK;
    if (n > kMaxNodes || dk > kMaxDk || dk % 8 || dv % 4 || (states && dv > kMaxDvStates)) {
        mfd::set_error("mfd_tree_gdn: supports n <= %d nodes, Dk <= %d a multiple of 8 and Dv a multiple of 4 (<= %d "
                       "with states) (got n=%lld Dk=%lld Dv=%lld)", kMaxNodes, kMaxDk, kMaxDvStates, (long long)n,
                       (long long)dk, (long long)dv);
        return MFD_ERR_UNSUPPORTED;
    }
    if (!q || !k || !v || !g_cum || !beta || !s0 || !anc || !u || !o) {
        mfd::set_error("mfd_tree_gdn: null pointer");
        return MFD_ERR_INVALID;
    }
    if (((uintptr_t)q | (uintptr_t)k) % 16 || (sq | sk) % 8 || (uintptr_t)s0 % 16 || (uintptr_t)u % 16 ||
        (uintptr_t)o % 16 || (states && (uintptr_t)states % 16) || sa < n || sg < num_heads || sb < num_heads) {
        mfd::set_error("mfd_tree_gdn: q, k need 16-byte aligned rows (node strides multiples of 8); s0, u, o and "
                       "states 16-byte alignment; row strides of anc, g_cum and beta at least n, H, H");
        return MFD_ERR_INVALID;
    }
    Params p;
    p.q = (const __nv_bfloat16*)q;
    p.k = (const __nv_bfloat16*)k;
    p.v = (const __nv_bfloat16*)v;
    p.sq = sq;
    p.sk = sk;
    p.sv = sv;
    p.g = g_cum;
    p.beta = beta;
    p.sg = sg;
    p.sb = sb;
    p.s0 = s0;
    p.anc = anc;
    p.sa = sa;
    p.n = (int)n;
    p.H = (int)num_heads;
    p.HK = (int)num_k_heads;
    p.Dk = (int)dk;
    p.Dv = (int)dv;
    p.u = u;
    p.o = o;
    p.states = states;
    p.status = status;
    cudaStream_t st = (cudaStream_t)stream;
    const int mt = (int)((n + kTile - 1) / kTile);
    p.pair_cap = uo_pair_cap((int)n, mt);
    {
        const size_t smem = (size_t)uo_layout((int)n, mt, p.pair_cap).total + kSlack;
        auto kern = mt == 1 ? tree_gdn_uo_kernel<1> : (mt == 2 ? tree_gdn_uo_kernel<2> : tree_gdn_uo_kernel<3>);
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) {
            mfd::set_error("mfd_tree_gdn: %s", cudaGetErrorString(e));
            return MFD_ERR_CUDA;
        }
        dim3 grid((unsigned)num_heads, (unsigned)((dv + kSlice - 1) / kSlice));
        kern<<<grid, kThreads, smem, st>>>(p);
        MFD_CHECK_LAUNCH("mfd_tree_gdn");
    }
    if (states) {
        const size_t smem = (size_t)kStTotal + kSlack;
        const bool fixed = dk == 128 && dv == 128;
        auto kern = fixed ? tree_gdn_states_kernel<128> : tree_gdn_states_kernel<0>;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) {
            mfd::set_error("mfd_tree_gdn: %s", cudaGetErrorString(e));
            return MFD_ERR_CUDA;
        }
        // one wave of kStCtasPerSm CTAs per SM: num_heads x S CTAs, S node residues per head
        int64_t S = (int64_t)mfd::current_sm_count() * kStCtasPerSm / num_heads;
        if (S < 1) S = 1;
        if (S > n) S = n;
        kern<<<dim3((unsigned)num_heads, (unsigned)S), kStThreads, smem, st>>>(p);
        MFD_CHECK_LAUNCH("mfd_tree_gdn (states)");
    }
    return MFD_OK;
}
