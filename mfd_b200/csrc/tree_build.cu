// tree_build.cu -- exact best-first tree builders on the GPU, one CTA per request.
//
// Reproduces the pop order of the reference heaps bit for bit:
//   mixture (K modes): key = -(float(logw) + prior[mode]) in float32, ties by mode, parent, depth, rank
//     (inference/hf/tree_build_ext.py:48-62, 158-203; sglang-v0.5.22-mfd.patch:1330-1373);
//   single mode: key = -logw in float64, ties by the rank tuple (lexicographic), parent, depth, rank
//     (inference/hf/tree_build_ext.py:31-46, 118-156; patch:1295-1327; inference/hf/ddtree.py:161-192).
// logw is accumulated in float64 with the reference's operation order: a sibling is
// (logw - lp[rank]) + lp[rank+1], a child logw + lp[depth][0].  A prefix popped again by another mode
// reuses its node (dedup by (parent, token) in a shared-memory hash table).
//
// Heaps: the mixture heap (mixture_heap1_kernel) is a binary min-heap kept by one thread in shared memory; its
// comparator is one 64-bit key (orderable float32 key in the high word, mode|parent|depth|rank in the low word)
// that is unique per entry, so no further tie-break is ever reached and a pop is a sift-down, a push a sift-up.
// The single-mode heap (build_trees_kernel, also the fallback when the mixture tables do not fit shared memory)
// spreads the live entries over the lanes of a warp, each lane caching the minimum of its slots, and pops by a
// warp-wide min (two redux.sync); single-mode entries whose float64 keys tie exactly are ordered by rank tuple on
// a slow path that walks parent pointers.
//
// Outputs: the SGLang layout tree[bs, 3, B+1] (tokens, depths, parents; index 0 = root; tail entries
// tokens 0 / depths 0 / parents -1), counts[bs], and optionally each node's ancestor-or-self set as a
// bitset anc[bs, B+1, words] and/or a dense uint8 visibility matrix vis[bs, B+1, B+1]
// (inference/hf/tree_build_ext.py:92-114, ddtree.py:297-305).
#include "common.cuh"

namespace mfd {
namespace tree {

constexpr int kThreads = 128;
constexpr uint64_t kEmptyHash = ~0ull;

struct Params {
    const float* lp;      // [bs, K, L, k]
    const void* ids;      // [bs, K, L, k] int32 / int64
    int ids_i64;
    const float* prior;   // [bs, K] or null (zeros)
    int64_t bs;
    int K, L, k, B;
    int single;           // single-mode heap (K must be 1)
    int ks;               // ranks staged in shared memory per (mode, depth) row
    int S;                // entry slots per lane
    int hcap;             // hash capacity (power of two)
    int words;            // 64-bit words per ancestor row
    int64_t* tree;        // [bs, 3, B+1]
    int64_t* counts;      // [bs]
    uint64_t* anc;        // [bs, B+1, words] or null
    uint8_t* vis;         // [bs, B+1, B+1] or null
    int* status;          // device status word or null: set to MFD_ERR_CAPACITY on overflow
};

__device__ __forceinline__ uint32_t pack_aux(int mode, int parent, int depth, int rank) {
    return ((uint32_t)mode << 28) | ((uint32_t)parent << 16) | ((uint32_t)depth << 11) | (uint32_t)rank;
}

struct Smem {
    float* lp;        // [K][L][ks]
    int32_t* ids;     // [K][L][ks]
    uint64_t* comp;   // [32*S]
    double* logw;     // [32*S]
    uint32_t* aux;    // [32*S]
    int32_t* ntok;    // [B+1]
    int16_t* npar;    // [B+1]
    uint8_t* ndep;    // [B+1]
    int16_t* nrank;   // [B+1]
    uint64_t* hash;   // [hcap]
    float* prior;     // [K]
};

__device__ __forceinline__ float lp_at(const Params& p, const Smem& s, const float* glp, int m, int d, int r) {
    if (r < p.ks) return s.lp[(m * p.L + d) * p.ks + r];
    return glp[((size_t)m * p.L + d) * p.k + r];
}
__device__ __forceinline__ int64_t id_at(const Params& p, const Smem& s, const void* gids, int m, int d, int r) {
    if (r < p.ks) return s.ids[(m * p.L + d) * p.ks + r];
    const size_t o = ((size_t)m * p.L + d) * p.k + r;
    return p.ids_i64 ? ((const int64_t*)gids)[o] : (int64_t)((const int32_t*)gids)[o];
}

// rank tuple of a prospective node (parent `par`, own rank `rk`, depth `dep`), root-first, into t[0..dep)
__device__ __forceinline__ void rank_tuple(const Smem& s, int par, int rk, int dep, int16_t* t) {
    t[dep - 1] = (int16_t)rk;
    int node = par;
    for (int d = dep - 2; d >= 0; --d) {
        t[d] = s.nrank[node];
        node = s.npar[node];
    }
}
// lexicographic comparison of rank tuples (shorter first when one is a prefix), as Python tuples compare
__device__ __forceinline__ int tuple_cmp(const int16_t* a, int na, const int16_t* b, int nb) {
    const int n = na < nb ? na : nb;
    for (int i = 0; i < n; ++i)
        if (a[i] != b[i]) return a[i] < b[i] ? -1 : 1;
    return na == nb ? 0 : (na < nb ? -1 : 1);
}

// Tree outputs of request b from its node arrays: the SGLang layout, the count, ancestor bitsets, dense mask.
__device__ void write_tree_outputs(const Params& p, int b, int n, const int32_t* ntok, const int16_t* npar,
                                   const uint8_t* ndep) {
    const int W = p.B + 1;
    int64_t* t = p.tree + (size_t)b * 3 * W;
    int64_t* d = t + W;
    int64_t* pa = d + W;
    for (int i = threadIdx.x; i < W; i += kThreads) {
        const bool live_node = i <= n;
        t[i] = (live_node && i > 0) ? (int64_t)ntok[i] : 0;
        d[i] = live_node ? (int64_t)ndep[i] : 0;
        pa[i] = live_node ? (int64_t)npar[i] : -1;
    }
    if (threadIdx.x == 0) p.counts[b] = n;
    if (p.anc || p.vis) {
        const int words = p.words;
        for (int i = threadIdx.x; i < W; i += kThreads) {
            uint64_t bits[8];  // words <= 8 (B < 512)
#pragma unroll
            for (int w = 0; w < 8; ++w) bits[w] = 0;
            if (i <= n) {
                int node = i;
                while (node >= 0) {
                    bits[node >> 6] |= 1ull << (node & 63);
                    node = node == 0 ? -1 : npar[node];
                }
            }
            if (p.anc) {
                uint64_t* row = p.anc + ((size_t)b * W + i) * words;
#pragma unroll
                for (int w = 0; w < 8; ++w)
                    if (w < words) row[w] = bits[w];
            }
            if (p.vis) {
                uint8_t* row = p.vis + ((size_t)b * W + i) * W;
                for (int j = 0; j < W; ++j) row[j] = (uint8_t)((bits[j >> 6] >> (j & 63)) & 1ull);
            }
        }
    }
}

__global__ void __launch_bounds__(kThreads) build_trees_kernel(Params p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int b = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int K = p.K, L = p.L, k = p.k, B = p.B, S = p.S, W = B + 1;
    const int cap = 32 * S;

    // ---- carve shared memory
    Smem s;
    {
        unsigned char* q = smem_raw;
        auto take = [&](size_t bytes) {
            unsigned char* r = q;
            q += (bytes + 15) & ~(size_t)15;
            return r;
        };
        s.comp = (uint64_t*)take(sizeof(uint64_t) * cap);
        s.logw = (double*)take(sizeof(double) * cap);
        s.hash = (uint64_t*)take(sizeof(uint64_t) * p.hcap);
        s.aux = (uint32_t*)take(sizeof(uint32_t) * cap);
        s.lp = (float*)take(sizeof(float) * K * L * p.ks);
        s.ids = (int32_t*)take(sizeof(int32_t) * K * L * p.ks);
        s.ntok = (int32_t*)take(sizeof(int32_t) * W);
        s.npar = (int16_t*)take(sizeof(int16_t) * W);
        s.nrank = (int16_t*)take(sizeof(int16_t) * W);
        s.ndep = (uint8_t*)take(sizeof(uint8_t) * W);
        s.prior = (float*)take(sizeof(float) * (K > 0 ? K : 1));
    }
    const float* glp = p.lp + (size_t)b * K * L * k;
    const void* gids = p.ids_i64 ? (const void*)((const int64_t*)p.ids + (size_t)b * K * L * k)
                                 : (const void*)((const int32_t*)p.ids + (size_t)b * K * L * k);

    // ---- stage the candidate tables (all warps): 16-byte asynchronous copies when the tables are whole and
    // aligned, so every thread has many copies in flight; element copies otherwise
    const int rows = K * L;
    const int n_el = rows * p.ks;
    const bool whole = p.ks == k && (n_el % 4) == 0 && (((uintptr_t)glp) & 15u) == 0 &&
                       (((uintptr_t)gids) & 15u) == 0;
    if (whole) {
        for (int c = threadIdx.x; c < n_el / 4; c += kThreads) {
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(s.lp + 4 * c)),
                         "l"(glp + 4 * c));
            if (!p.ids_i64)
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(s.ids + 4 * c)),
                             "l"((const int32_t*)gids + 4 * c));
        }
        asm volatile("cp.async.commit_group;");
        if (p.ids_i64) {
            const longlong2* g2 = (const longlong2*)gids;
#pragma unroll 4
            for (int c = threadIdx.x; c < n_el / 2; c += kThreads) {
                const longlong2 v = __ldg(g2 + c);
                s.ids[2 * c] = (int32_t)v.x;
                s.ids[2 * c + 1] = (int32_t)v.y;
            }
        }
        asm volatile("cp.async.wait_all;");
    } else {
        for (int i = threadIdx.x; i < n_el; i += kThreads) {
            const int row = i / p.ks, r = i % p.ks;
            const size_t o = (size_t)row * k + r;
            s.lp[i] = glp[o];
            s.ids[i] = p.ids_i64 ? (int32_t)((const int64_t*)gids)[o] : ((const int32_t*)gids)[o];
        }
    }
    for (int i = threadIdx.x; i < p.hcap; i += kThreads) s.hash[i] = kEmptyHash;
    for (int i = threadIdx.x; i < cap; i += kThreads) {
        s.comp[i] = ~0ull;
        s.aux[i] = 0xffffffffu;
    }
    for (int i = threadIdx.x; i < K; i += kThreads) s.prior[i] = p.prior ? p.prior[(size_t)b * K + i] : 0.f;
    if (threadIdx.x == 0) {
        s.ntok[0] = 0;
        s.npar[0] = -1;
        s.ndep[0] = 0;
        s.nrank[0] = 0;
    }
    __syncthreads();

    __shared__ int sh_count, sh_fail;
    if (warp == 0) {
        int count = 0;
        int fail = 0;
        // lane-owned slot sets
        uint64_t occ = 0;             // occupied slots of this lane (bit j = slot lane + 32 j)
        uint64_t lmin = ~0ull;        // this lane's minimum key
        int lslot = -1;               // its slot
        int lcnt = 0;                 // how many of this lane's entries equal lmin (single-mode ties)
        int live = 0;                 // warp-uniform number of live entries
        int rr = 0;                   // round-robin insertion lane

        auto rescan = [&]() {
            lmin = ~0ull;
            lslot = -1;
            lcnt = 0;
            uint64_t o = occ;
            while (o) {
                const int j = __ffsll((long long)o) - 1;
                o &= o - 1;
                const int slot = lane + 32 * j;
                const uint64_t c = s.comp[slot];
                if (c < lmin) { lmin = c; lslot = slot; lcnt = 1; }
                else if (c == lmin) { ++lcnt; }
            }
        };
        // insert (comp, logw, aux) into lane `dst`'s free slot; warp-uniform call
        auto insert = [&](int dst, uint64_t c, double lw, uint32_t ax) {
            // pick a lane with room, preferring dst
            uint32_t room = __ballot_sync(MFD_FULL_MASK, (S >= 64) ? (occ != ~0ull) : (occ != ((1ull << S) - 1ull)));
            if (!room) { fail = 1; return; }
            if (!((room >> dst) & 1u)) dst = __ffs(room) - 1;
            if (lane == dst) {
                const int j = __ffsll((long long)~occ) - 1;
                const int slot = lane + 32 * j;
                occ |= 1ull << j;
                s.comp[slot] = c;
                s.logw[slot] = lw;
                s.aux[slot] = ax;
                if (c < lmin) { lmin = c; lslot = slot; lcnt = 1; }
                else if (c == lmin) { ++lcnt; }
            }
            ++live;
        };
        auto mix_comp = [&](double lw, int m, uint32_t ax) -> uint64_t {
            float key = -(__double2float_rn(lw) + s.prior[m]);
            key = key + 0.0f;  // -0.0 and +0.0 compare equal in the reference: fold them
            return ((uint64_t)ord_f32(key) << 32) | ax;
        };

        // initial entries: one per mode at (parent 0, depth 1, rank 0)
        if (B > 0 && L > 0) {
            if (p.single) {
                const double lw = (double)lp_at(p, s, glp, 0, 0, 0);
                insert(0, ord_f64(-lw), lw, pack_aux(0, 0, 1, 0));
            } else {
                for (int m = 0; m < K; ++m) {
                    const double lw = (double)lp_at(p, s, glp, m, 0, 0);
                    const uint32_t ax = pack_aux(m, 0, 1, 0);
                    insert(m & 31, mix_comp(lw, m, ax), lw, ax);
                }
            }
        }

        while (live > 0 && count < B && !fail) {
            // ---- pop the minimum
            const uint64_t M = warp_min_u64(lmin);
            const bool eq = (lmin == M) && lslot >= 0;
            int slot;
            const int tot = p.single ? __reduce_add_sync(MFD_FULL_MASK, eq ? lcnt : 0) : 1;
            if (tot == 1) {
                const int w = __ffs(__ballot_sync(MFD_FULL_MASK, eq)) - 1;
                slot = __shfl_sync(MFD_FULL_MASK, lslot, w);
            } else {
                // single-mode exact float64 tie: order the tied entries by rank tuple (lane 0, rare)
                __syncwarp();
                int best = -1;
                if (lane == 0) {
                    int16_t tb[32], tc[32];
                    int nb = 0;
                    for (int sl = 0; sl < cap; ++sl) {
                        if (!((s.comp[sl] == M) && (s.aux[sl] != 0xffffffffu))) continue;
                        const uint32_t ax = s.aux[sl];
                        const int par = (ax >> 16) & 0xfff, dep = (ax >> 11) & 31, rk = ax & 0x7ff;
                        if (best < 0) {
                            rank_tuple(s, par, rk, dep, tb);
                            nb = dep;
                            best = sl;
                        } else {
                            rank_tuple(s, par, rk, dep, tc);
                            if (tuple_cmp(tc, dep, tb, nb) < 0) {
                                for (int i = 0; i < dep; ++i) tb[i] = tc[i];
                                nb = dep;
                                best = sl;
                            }
                        }
                    }
                }
                slot = __shfl_sync(MFD_FULL_MASK, best, 0);
            }
            const double lw = s.logw[slot];
            const uint32_t ax = s.aux[slot];
            const int m = ax >> 28, par = (ax >> 16) & 0xfff, dep = (ax >> 11) & 31, rk = ax & 0x7ff;
            const int owner = slot & 31;
            const int64_t token = id_at(p, s, gids, m, dep - 1, rk);

            // ---- node: new, or an existing prefix reached by another mode
            int current;
            if (p.single) {
                current = count + 1;
            } else {
                const uint64_t want = ((uint64_t)(uint32_t)token << 32) | ((uint64_t)(uint32_t)par << 16);
                uint32_t h = (uint32_t)(((uint64_t)(uint32_t)token * 0x9E3779B1u) ^ ((uint32_t)par * 0x85EBCA77u));
                h &= (uint32_t)(p.hcap - 1);
                current = -1;
                for (int base = 0; base < p.hcap && current < 0; base += 32) {
                    const int hs = (int)((h + (uint32_t)base + (uint32_t)lane) & (uint32_t)(p.hcap - 1));
                    const uint64_t v = s.hash[hs];
                    const uint32_t hit = __ballot_sync(MFD_FULL_MASK, v != kEmptyHash && (v & ~0xffffull) == want);
                    const uint32_t emp = __ballot_sync(MFD_FULL_MASK, v == kEmptyHash);
                    // probe order = lane order; the first match before the first empty slot wins
                    const uint32_t before = emp ? ((emp & (0u - emp)) - 1u) : 0xffffffffu;
                    if (hit & before) {
                        const int hl = __ffs(hit & before) - 1;
                        current = (int)(__shfl_sync(MFD_FULL_MASK, (uint32_t)(v & 0xffffu), hl));
                    } else if (emp) {
                        const int el = __ffs(emp) - 1;
                        current = count + 1;
                        if (lane == el) s.hash[hs] = want | (uint64_t)(uint32_t)current;
                    }
                }
                __syncwarp();
                if (current < 0) { fail = 1; break; }
            }
            if (current == count + 1) {
                if (lane == 0) {
                    s.ntok[current] = (int32_t)token;
                    s.npar[current] = (int16_t)par;
                    s.ndep[current] = (uint8_t)dep;
                    s.nrank[current] = (int16_t)rk;
                }
                ++count;
            }

            // ---- successors: the sibling replaces the popped slot, the child takes a free slot
            const bool has_sib = rk + 1 < k;
            const bool has_child = dep < L;
            if (lane == owner) {
                if (has_sib) {
                    const double slw = (lw - (double)lp_at(p, s, glp, m, dep - 1, rk))
                                       + (double)lp_at(p, s, glp, m, dep - 1, rk + 1);
                    const uint32_t sax = pack_aux(m, par, dep, rk + 1);
                    s.comp[slot] = p.single ? ord_f64(-slw) : mix_comp(slw, m, sax);
                    s.logw[slot] = slw;
                    s.aux[slot] = sax;
                } else {
                    occ &= ~(1ull << (slot >> 5));
                    s.aux[slot] = 0xffffffffu;
                    s.comp[slot] = ~0ull;
                }
                rescan();
            }
            if (!has_sib) --live;
            if (has_child) {
                const double clw = lw + (double)lp_at(p, s, glp, m, dep, 0);
                const uint32_t cax = pack_aux(m, current, dep + 1, 0);
                const uint64_t cc = p.single ? ord_f64(-clw) : mix_comp(clw, m, cax);
                __syncwarp();
                insert(rr, cc, clw, cax);
                rr = (rr + 1) & 31;
            }
            __syncwarp();
        }
        if (lane == 0) {
            sh_count = count;
            sh_fail = fail;
        }
    }
    __syncthreads();
    const int n = sh_count;
    if (sh_fail && threadIdx.x == 0 && p.status) atomicExch(p.status, (int)MFD_ERR_CAPACITY);

    write_tree_outputs(p, b, n, s.ntok, s.npar, s.ndep);
}

// ------------------------------------------------------------------ mixture heap in one thread
// The same pop order from a 4-ary min-heap kept by one thread in shared memory (keys are unique, so any exact
// priority queue pops the same sequence): a pop is a sift-down of about log4(live) levels and a push a sift-up,
// with the (parent, token) dedup in a shared-memory hash -- no warp-wide collective on the critical path.
struct MixSmem {
    ulonglong2* he;   // [K (B + 1)] heap entries: (comparator key, logw bits)
    uint64_t* hash;   // [hcap] (token, parent) -> node
    float* lp;        // [K][L][k]
    int32_t* ids;     // [K][L][k]
    int32_t* ntok;    // [B + 1]
    int16_t* npar;    // [B + 1]
    uint8_t* ndep;    // [B + 1]
    float* prior;     // [K]
};

__device__ __forceinline__ unsigned char* smem_take(unsigned char*& q, size_t bytes) {
    unsigned char* r = q;
    q += (bytes + 15) & ~(size_t)15;
    return r;
}

__device__ MixSmem carve_mixture(const Params& p, unsigned char*& q) {
    const int K = p.K, L = p.L, k = p.k, W = p.B + 1;
    MixSmem s;
    s.he = (ulonglong2*)smem_take(q, 16 * (size_t)K * W);
    s.hash = (uint64_t*)smem_take(q, 8 * (size_t)p.hcap);
    s.lp = (float*)smem_take(q, 4 * (size_t)K * L * k);
    s.ids = (int32_t*)smem_take(q, 4 * (size_t)K * L * k);
    s.ntok = (int32_t*)smem_take(q, 4 * (size_t)W);
    s.npar = (int16_t*)smem_take(q, 2 * (size_t)W);
    s.ndep = (uint8_t*)smem_take(q, (size_t)W);
    s.prior = (float*)smem_take(q, 4 * (size_t)K);
    return s;
}
// host mirror of carve_mixture's size
static size_t mixture_smem_bytes(int K, int L, int k, int B, int hcap) {
    auto r16 = [](size_t v) { return (v + 15) & ~(size_t)15; };
    const size_t W = (size_t)B + 1;
    return r16(16 * (size_t)K * W) + r16(8 * (size_t)hcap) + 2 * r16(4 * (size_t)K * L * k) + r16(4 * W) +
           r16(2 * W) + r16(W) + r16(4 * (size_t)K);
}

// Stage tree b's candidate tables and prior in shared memory, clear the dedup hash, set the root node.  All
// threads of the CTA take part; the caller synchronises afterwards.
__device__ void stage_mixture(const Params& p, int b, const MixSmem& s) {
    const int K = p.K, L = p.L, k = p.k;
    const int nt = blockDim.x;
    const float* glp = p.lp + (size_t)b * K * L * k;
    const void* gids = p.ids_i64 ? (const void*)((const int64_t*)p.ids + (size_t)b * K * L * k)
                                 : (const void*)((const int32_t*)p.ids + (size_t)b * K * L * k);
    const int n_el = K * L * k;
    if ((n_el % 4) == 0 && (((uintptr_t)glp) & 15u) == 0 && (((uintptr_t)gids) & 15u) == 0) {
        for (int c = threadIdx.x; c < n_el / 4; c += nt) {
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(s.lp + 4 * c)), "l"(glp + 4 * c));
            if (!p.ids_i64)
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(s.ids + 4 * c)),
                             "l"((const int32_t*)gids + 4 * c));
        }
        asm volatile("cp.async.commit_group;");
        if (p.ids_i64) {
            const longlong2* g2 = (const longlong2*)gids;
#pragma unroll 4
            for (int c = threadIdx.x; c < n_el / 2; c += nt) {
                const longlong2 v = __ldg(g2 + c);
                s.ids[2 * c] = (int32_t)v.x;
                s.ids[2 * c + 1] = (int32_t)v.y;
            }
        }
        asm volatile("cp.async.wait_all;");
    } else {
        for (int i = threadIdx.x; i < n_el; i += nt) {
            s.lp[i] = glp[i];
            s.ids[i] = p.ids_i64 ? (int32_t)((const int64_t*)gids)[i] : ((const int32_t*)gids)[i];
        }
    }
    for (int i = threadIdx.x; i < p.hcap; i += nt) s.hash[i] = kEmptyHash;
    for (int i = threadIdx.x; i < K; i += nt) s.prior[i] = p.prior ? p.prior[(size_t)b * K + i] : 0.f;
    if (threadIdx.x == 0) {
        s.ntok[0] = 0;
        s.npar[0] = -1;
        s.ndep[0] = 0;
    }
}

// The mixture key of an entry: -(float(logw) + prior[mode]) (hf/tree_build_ext.py:167), -0.0 folded into +0.0
// (they compare equal in the reference), as an orderable uint32.
__device__ __forceinline__ uint32_t mix_key(double w, float prior_m) {
    float key = -(__double2float_rn(w) + prior_m);
    key = key + 0.0f;
    return ord_f32(key);
}

// The reference's mixture heap (hf/tree_build_ext.py:158-203), run by one thread over the staged tables.
// Returns the node count; *fail is set when the dedup hash overflows.
__device__ int serial_mixture(const Params& p, const MixSmem& s, int* fail) {
    const int K = p.K, L = p.L, k = p.k, B = p.B;
    ulonglong2* he = s.he;
    int n = 0;  // live entries
    auto comp = [&](double w, int m, uint32_t ax) -> uint64_t { return ((uint64_t)mix_key(w, s.prior[m]) << 32) | ax; };
    // a 4-ary min-heap of 16-byte entries: children of i are 4i+1 .. 4i+4, so about 3 levels for the at most
    // K (B + 1) live entries, and the four children of a level are loaded together
    auto push = [&](uint64_t c, double w) {
        int i = n++;
        while (i > 0) {
            const int par = (i - 1) >> 2;
            const ulonglong2 pe = he[par];
            if (pe.x <= c) break;
            he[i] = pe;
            i = par;
        }
        he[i] = make_ulonglong2(c, (unsigned long long)__double_as_longlong(w));
    };
    // replace the root by (c, w) and sift it down
    auto replace_top = [&](uint64_t c, double w) {
        int i = 0;
        for (;;) {
            const int l = 4 * i + 1;
            if (l >= n) break;
            ulonglong2 e[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) e[t] = l + t < n ? he[l + t] : make_ulonglong2(~0ull, 0ull);
            int j = l;
            ulonglong2 best = e[0];
#pragma unroll
            for (int t = 1; t < 4; ++t)
                if (e[t].x < best.x) {
                    best = e[t];
                    j = l + t;
                }
            if (c <= best.x) break;
            he[i] = best;
            i = j;
        }
        he[i] = make_ulonglong2(c, (unsigned long long)__double_as_longlong(w));
    };
    int count = 0;
    *fail = 0;
    if (B > 0 && L > 0)
        for (int m = 0; m < K; ++m) {
            const double w = (double)s.lp[(m * L) * k];
            push(comp(w, m, pack_aux(m, 0, 1, 0)), w);
        }
    while (n > 0 && count < B) {
        const ulonglong2 top = he[0];
        const uint64_t M = top.x;
        const double lwp = __longlong_as_double((long long)top.y);
        const uint32_t ax = (uint32_t)M;
        const int m = ax >> 28, par = (ax >> 16) & 0xfff, dep = (ax >> 11) & 31, rk = ax & 0x7ff;
        const int row = (m * L + dep - 1) * k;
        const int32_t token = s.ids[row + rk];
        const bool has_sib = rk + 1 < k, has_child = dep < L;
        const float lp_r = s.lp[row + rk];
        const float lp_r1 = has_sib ? s.lp[row + rk + 1] : 0.f;
        const float lp_c = has_child ? s.lp[row + k] : 0.f;
        // node: dedup by (parent, token)
        const uint64_t want = ((uint64_t)(uint32_t)token << 32) | ((uint64_t)(uint32_t)par << 16);
        uint32_t h = (uint32_t)(((uint64_t)(uint32_t)token * 0x9E3779B1u) ^ ((uint32_t)par * 0x85EBCA77u));
        int current = -1;
        for (int t = 0; t < p.hcap; ++t) {
            const uint32_t hs = (h + (uint32_t)t) & (uint32_t)(p.hcap - 1);
            const uint64_t v = s.hash[hs];
            if (v == kEmptyHash) {
                current = count + 1;
                s.hash[hs] = want | (uint64_t)(uint32_t)current;
                s.ntok[current] = token;
                s.npar[current] = (int16_t)par;
                s.ndep[current] = (uint8_t)dep;
                ++count;
                break;
            }
            if ((v & ~0xffffull) == want) {
                current = (int)(v & 0xffffu);
                break;
            }
        }
        if (current < 0) {
            *fail = 1;
            break;
        }
        // successors: the sibling replaces the popped root, the child is pushed
        if (has_sib) {
            const double slw = (lwp - (double)lp_r) + (double)lp_r1;
            replace_top(comp(slw, m, pack_aux(m, par, dep, rk + 1)), slw);
        } else {
            --n;
            if (n > 0) replace_top(he[n].x, __longlong_as_double((long long)he[n].y));
        }
        if (has_child) {
            const double clw = lwp + (double)lp_c;
            push(comp(clw, m, pack_aux(m, current, dep + 1, 0)), clw);
        }
    }
    return count;
}

__global__ void __launch_bounds__(kThreads) mixture_heap1_kernel(Params p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ int sh_count, sh_fail;
    const int b = blockIdx.x;
    unsigned char* q = smem_raw;
    const MixSmem s = carve_mixture(p, q);
    stage_mixture(p, b, s);
    __syncthreads();
    if (threadIdx.x == 0) {
        int fail = 0;
        sh_count = serial_mixture(p, s, &fail);
        sh_fail = fail;
    }
    __syncthreads();
    if (sh_fail && threadIdx.x == 0 && p.status) atomicExch(p.status, (int)MFD_ERR_CAPACITY);
    write_tree_outputs(p, b, sh_count, s.ntok, s.npar, s.ndep);
}

// ------------------------------------------------------------------ mixture tree, one warp per mode
// The heap pops entries in the order of the tuple (key, mode, parent, depth, rank).  An entry's successors (its
// sibling and its first child) never have a smaller key than the entry itself, so the pop order is that sorted
// order, and restricted to one mode it is the best-first enumeration of that mode alone -- except where two live
// entries of one mode have equal keys (their order then depends on global node ids).  This kernel therefore:
//   1. runs the K modes' enumerations at once, one warp per mode: the mode's live entries (one per open sibling
//      group, at most B + 1) sit in registers, three per lane, each with its two successors already computed, and a
//      pop is a warp-wide minimum (redux.sync), one ballot and a hand-over of the first child to the lane of its new
//      group; the successors of the two entries made live follow.  Round 1 pops B / 4 entries per mode and merges them
//      (steps 2-4); the B-th distinct prefix found bounds the tree's last node, so round 2 pops only the modes
//      whose next entry precedes that bound, up to it (or up to B entries when round 1 found fewer than B
//      prefixes -- B per mode always suffice, since the first B distinct nodes contain at most B entries of any
//      mode), and merges again;
//   2. ranks every popped entry in the merged order (key, then mode) by fixed-step searches in the other modes'
//      lists, run side by side;
//   3. merges equal prefixes: every popped entry gets a hash of its token path (summed up its parent chain by
//      pointer jumping), entries are grouped through a shared-memory hash table (atomicCAS / atomicMin give each
//      group its least merged position), and every grouped entry is compared token by token with that first
//      occurrence;
//   4. numbers the first occurrences in merged order by a block scan: the first B are the nodes, in the heap's
//      pop order.
// A mode whose warp minimum is not unique (an exact key tie), a successor with a smaller key than its generator
// (double rounding of equal log-probabilities), or two different paths with one hash sends the whole tree to
// serial_mixture, which replays the reference heap exactly.  Limits: K <= 16, B <= 95 (three groups per lane).
constexpr int kFastThreads = 512;
constexpr int kFastSlots = 3;
constexpr uint32_t kNoKey = 0xffffffffu;
constexpr int kFastMaxB = 32 * kFastSlots - 1;

struct FastSmem {
    uint32_t* ekey;   // [K][B] popped keys, in each mode's pop order (non-decreasing)
    int32_t* etok;    // [K][B] token (filled by the merge)
    int16_t* epl;     // [K][B] pop index of the parent entry in the same mode (-1: the root)
    uint8_t* edep;    // [K][B] depth
    int16_t* epos;    // [K][B] merged position
    int16_t* ecan;    // [K][B] merged position of the first occurrence of the entry's prefix
    int16_t* eslot;   // [K][B] dedup hash slot
    int16_t* pnid;    // [K B] node id by merged position (0: not a node)
    int16_t* pent;    // [K B] entry (mode * B + pop index) by merged position
    uint16_t* eidx;   // [K][B] index of the entry in its mode's [L][k] table
    uint64_t* ehash;  // [K][B] hash of the entry's token path (filled by the merge)
    int16_t* ejmp;    // [K][B] pointer-jumping ancestor (merge scratch)
    uint64_t* dkey;   // [dcap] dedup keys (path hashes)
    int32_t* dval;    // [dcap] least merged position holding the key
};

__device__ FastSmem carve_fast(const Params& p, unsigned char*& q, int dcap) {
    const size_t KB = (size_t)p.K * p.B;
    FastSmem f;
    f.dkey = (uint64_t*)smem_take(q, 8 * (size_t)dcap);
    f.dval = (int32_t*)smem_take(q, 4 * (size_t)dcap);
    f.ehash = (uint64_t*)smem_take(q, 8 * KB);
    f.pent = (int16_t*)smem_take(q, 2 * KB);
    f.eidx = (uint16_t*)smem_take(q, 2 * KB);
    f.ejmp = (int16_t*)smem_take(q, 2 * KB);
    f.ekey = (uint32_t*)smem_take(q, 4 * KB);
    f.etok = (int32_t*)smem_take(q, 4 * KB);
    f.epl = (int16_t*)smem_take(q, 2 * KB);
    f.epos = (int16_t*)smem_take(q, 2 * KB);
    f.ecan = (int16_t*)smem_take(q, 2 * KB);
    f.eslot = (int16_t*)smem_take(q, 2 * KB);
    f.pnid = (int16_t*)smem_take(q, 2 * KB);
    f.edep = (uint8_t*)smem_take(q, KB);
    return f;
}
static size_t fast_smem_bytes(int K, int B, int dcap) {
    auto r16 = [](size_t v) { return (v + 15) & ~(size_t)15; };
    const size_t KB = (size_t)K * B;
    return r16(8 * (size_t)dcap) + r16(4 * (size_t)dcap) + r16(8 * KB) + 3 * r16(2 * KB) + 2 * r16(4 * KB) +
           5 * r16(2 * KB) + r16(KB);
}
__host__ __device__ inline int fast_dcap(int K, int B) {
    int d = 64;
    while (d < 2 * K * B) d <<= 1;
    return d;
}

// Hash of a token path: the sum over its nodes of a splitmix64 finaliser of (token, depth), so that the merge can
// form every entry's hash at once by pointer jumping, off the pop loop.  It only groups candidate duplicates: every
// grouped pair is compared token by token before it is trusted.
__device__ __forceinline__ uint64_t path_term(int32_t token, int depth) {
    uint64_t z = (((uint64_t)(uint32_t)token << 5) | (uint64_t)depth) * 0x9E3779B97F4A7C15ull + 0x243F6A8885A308D3ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// The successors of a live entry of rank r at depth d (1 <= d <= L) with log-weight w, in double as the reference
// accumulates them (hf/tree_build_ext.py:190-199): the next sibling (w - lp[d][r]) + lp[d][r + 1] and the first
// child w + lp[d + 1][0], with their mixture keys (kNoKey where there is none).  lpm is the mode's [L][k] table.
// Indices are clamped, so lanes that evaluate it on state they then discard stay inside the table.
__device__ __forceinline__ void fast_successors(const float* lpm, int k, int L, float pr, double w, int r, int d,
                                                uint32_t& nk, double& nw, uint32_t& ck, double& cw) {
    const int dc = min(max(d, 1), L), rc = min(max(r, 0), k - 1);
    const float* row = lpm + (dc - 1) * k;
    const float lr = row[rc], lr1 = row[min(rc + 1, k - 1)];
    const float lc = lpm[min(dc, L - 1) * k];
    nw = (w - (double)lr) + (double)lr1;
    cw = w + (double)lc;
    const uint32_t kn = mix_key(nw, pr), kc = mix_key(cw, pr);
    nk = r + 1 < k ? kn : kNoKey;
    ck = d < L ? kc : kNoKey;
}

// KMAX: 8 or 16, a bound on K that sizes the rank searches of the merge
template <int KMAX>
__global__ void __launch_bounds__(kFastThreads) mixture_fast_kernel(Params p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ int sh_cnt[16], sh_done[16];
    __shared__ int sh_bad, sh_count, sh_total, sh_fail, sh_ntot, sh_wsum[kFastThreads / 32];
    __shared__ uint32_t sh_ukey;
    __shared__ int sh_umode;
    const int b = blockIdx.x;
    const int K = p.K, L = p.L, k = p.k, B = p.B;
    const int KB = K * B;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int dcap = fast_dcap(K, B);
    unsigned char* q = smem_raw;
    const MixSmem s = carve_mixture(p, q);
    const FastSmem f = carve_fast(p, q, dcap);
    stage_mixture(p, b, s);
    if (threadIdx.x == 0) sh_bad = 0;
    __syncthreads();

    // ---- 1. per-mode best-first enumeration, warp m = mode m.  Slot t of lane l holds group 32 t + l: the key of
    // its live entry, the entry's meta ((parent pop index + 1) << 16 | depth << 11 | rank), and the entry's two
    // successors, computed when it became live -- the next sibling (key n, log-weight v) and the first child (c, u).
    // A pop then only moves precomputed values; the double-precision successors of the two entries it makes live
    // come after.  The state persists across the two rounds.
    const int m = warp;
    const float pr = warp < K ? s.prior[m] : 0.f;
    const float* lpm = s.lp + (size_t)(warp < K ? m : 0) * L * k;
    uint32_t k0 = kNoKey, k1 = kNoKey, k2 = kNoKey, a0 = 0, a1 = 0, a2 = 0;
    uint32_t n0 = kNoKey, n1 = kNoKey, n2 = kNoKey, c0 = kNoKey, c1 = kNoKey, c2 = kNoKey;
    double v0 = 0.0, v1 = 0.0, v2 = 0.0, u0 = 0.0, u1 = 0.0, u2 = 0.0;
    if (warp < K && lane == 0) {  // group 0: the root's children, rank 0 first
        const double w = (double)lpm[0];
        k0 = mix_key(w, pr);
        a0 = 1u << 11;
        fast_successors(lpm, k, L, pr, w, 0, 1, n0, v0, c0, u0);
    }
    int groups = 1, npop = 0, bad = 0;
    // pop while fewer than `limit` entries are out and the next entry precedes (ukey, umode) in the merged order
    auto pop_run = [&](int limit, uint32_t ukey, int umode) {
        uint32_t* ekey = f.ekey + m * B;
        for (; npop < limit; ++npop) {
            const int i = npop;
            const uint32_t wmin = __reduce_min_sync(MFD_FULL_MASK, min(k0, min(k1, k2)));
            if (wmin == kNoKey || wmin > ukey || (wmin == ukey && m > umode)) break;
            const bool h0 = k0 == wmin, h1 = k1 == wmin, h2 = k2 == wmin;
            const uint32_t bal = __ballot_sync(MFD_FULL_MASK, h0 || h1 || h2);
            if (bal & (bal - 1)) {  // an exact tie inside the mode
                bad = 1;
                break;
            }
            const int owner = __ffs(bal) - 1;
            const bool own = lane == owner;
            // the popped entry, as the owner holds it
            const uint32_t a = h0 ? a0 : (h1 ? a1 : a2);
            const uint32_t sk = h0 ? n0 : (h1 ? n1 : n2);
            const double sw = h0 ? v0 : (h1 ? v1 : v2);
            const uint32_t ck = h0 ? c0 : (h1 ? c1 : c2);
            const double cw = h0 ? u0 : (h1 ? u1 : u2);
            const int r = (int)(a & 2047u), d = (int)((a >> 11) & 31u);
            // a second slot of the owner at the same key, or a successor that rounds below its generator
            if (own && ((int)h0 + (int)h1 + (int)h2 > 1 || sk < wmin || ck < wmin)) bad = 1;
            // the first child opens group `groups` (lane groups % 32, slot groups / 32)
            const uint32_t hk = __shfl_sync(MFD_FULL_MASK, ck, owner);
            const double hw = shfl_f64(cw, owner);
            const int hd = __shfl_sync(MFD_FULL_MASK, d, owner);
            if (own) {
                ekey[i] = wmin;
                f.eidx[m * B + i] = (uint16_t)((d - 1) * k + r);
                f.epl[m * B + i] = (int16_t)((int)(a >> 16) - 1);
                f.edep[m * B + i] = (uint8_t)d;
            }
            const int g = groups;
            const bool child = hd < L;
            groups += child ? 1 : 0;
            const bool recv = child && lane == (g & 31);
            const int rs = g >> 5;
            // successors of the owner's new live entry (the sibling) and of the new group's first entry
            uint32_t snk, sck, cnk, cck;
            double snw, scw, cnw, ccw;
            fast_successors(lpm, k, L, pr, sw, r + 1, d, snk, snw, sck, scw);
            fast_successors(lpm, k, L, pr, hw, 0, hd + 1, cnk, cnw, cck, ccw);
            const uint32_t sa = (a & ~2047u) | (uint32_t)(r + 1);
            const uint32_t ca = ((uint32_t)(i + 1) << 16) | ((uint32_t)(hd + 1) << 11);
#define MFD_SLOT_UPDATE(t, kt, at, nt, vt, ct, ut)                     \
    {                                                                  \
        const bool po = own && h##t, pr_ = recv && rs == t;            \
        kt = po ? sk : (pr_ ? hk : kt);                                \
        at = po ? sa : (pr_ ? ca : at);                                \
        nt = po ? snk : (pr_ ? cnk : nt);                              \
        vt = po ? snw : (pr_ ? cnw : vt);                              \
        ct = po ? sck : (pr_ ? cck : ct);                              \
        ut = po ? scw : (pr_ ? ccw : ut);                              \
    }
            MFD_SLOT_UPDATE(0, k0, a0, n0, v0, c0, u0)
            MFD_SLOT_UPDATE(1, k1, a1, n1, v1, c1, u1)
            MFD_SLOT_UPDATE(2, k2, a2, n2, v2, c2, u2)
#undef MFD_SLOT_UPDATE
        }
        bad = __any_sync(MFD_FULL_MASK, bad);
        if (lane == 0) {
            sh_cnt[m] = npop;
            if (bad) atomicOr(&sh_bad, 1);
        }
    };

    // ---- 2-4. merge the popped lists (all threads).  Sets sh_total (distinct prefixes), sh_count, pnid and, when
    // sh_total reaches B, (sh_ukey, sh_umode) = key and mode of the B-th distinct prefix's first occurrence.
    // Merged position of entry (mode mm, pop index i): i plus, in every other mode, the number of its entries that
    // precede (key, mm) -- keys below it, and equal keys of lower modes; the K searches run side by side
    auto merged_pos = [&](int mm, int i, uint32_t kv) {
        int pos = i;
#pragma unroll
        for (int m2 = 0; m2 < KMAX; ++m2) {
            const int cnt = (m2 < K && m2 != mm) ? sh_cnt[m2] : 0;
            const uint32_t* ek = f.ekey + m2 * B;
            const uint64_t lim = (uint64_t)kv + (m2 < mm ? 1u : 0u);  // count keys < lim
            int base = 0;
#pragma unroll
            for (int step = 64; step; step >>= 1)
                if (base + step <= cnt && (uint64_t)ek[base + step - 1] < lim) base += step;
            pos += base;
        }
        return pos;
    };
    // entry x's token path equals entry y's (same depth, the same tokens back to the root)
    auto same_path = [&](int x, int y) {
        if (f.edep[x] != f.edep[y]) return false;
        while (x >= 0 && y >= 0) {
            if (f.etok[x] != f.etok[y]) return false;
            const int px = f.epl[x], py = f.epl[y];
            x = px < 0 ? -1 : (x / B) * B + px;
            y = py < 0 ? -1 : (y / B) * B + py;
        }
        return x < 0 && y < 0;
    };
    auto merge = [&]() {
        for (int i = threadIdx.x; i < dcap; i += kFastThreads) {
            f.dkey[i] = kEmptyHash;
            f.dval[i] = 0x7fffffff;
        }
        if (threadIdx.x == 0) {
            int o = 0;
            for (int mm = 0; mm < K; ++mm) o += sh_cnt[mm];
            sh_ntot = o;
            sh_ukey = kNoKey;
            sh_umode = K;
        }
        // tokens, and the path hashes by pointer jumping: an entry's sum starts as its own term and its pointer as
        // its parent; each round adds the pointed-to entry's partial sum and moves the pointer to that entry's
        // pointer, so ceil(log2(depth)) rounds reach the root
        for (int x = threadIdx.x; x < KB; x += kFastThreads) {
            const int mm = x / B, i = x - mm * B;
            int jmp = -1;
            if (i < sh_cnt[mm]) {
                const int32_t tok = s.ids[(size_t)mm * L * k + f.eidx[x]];
                f.etok[x] = tok;
                f.ehash[x] = path_term(tok, f.edep[x]);
                const int pl = f.epl[x];
                jmp = pl < 0 ? -1 : mm * B + pl;
            }
            f.ejmp[x] = (int16_t)jmp;
        }
        __syncthreads();
        for (;;) {
            constexpr int kPer = (16 * kFastMaxB + kFastThreads - 1) / kFastThreads;
            uint64_t nh[kPer];
            int na[kPer];
            bool act[kPer];
            int any = 0;
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
                const int x = threadIdx.x + j * kFastThreads;
                const int a = x < KB ? f.ejmp[x] : -1;
                act[j] = a >= 0;
                if (act[j]) {
                    nh[j] = f.ehash[x] + f.ehash[a];
                    na[j] = f.ejmp[a];
                    any = 1;
                }
            }
            __syncthreads();
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
                const int x = threadIdx.x + j * kFastThreads;
                if (act[j]) {
                    f.ehash[x] = nh[j];
                    f.ejmp[x] = (int16_t)na[j];
                }
            }
            if (!__syncthreads_or(any)) break;
        }
        // positions, and each path's least position through the table of path hashes
        for (int x = threadIdx.x; x < KB; x += kFastThreads) {
            const int mm = x / B, i = x - mm * B;
            if (i >= sh_cnt[mm]) continue;
            const uint64_t hk = f.ehash[x] == kEmptyHash ? kEmptyHash - 1 : f.ehash[x];
            const int pos = merged_pos(mm, i, f.ekey[x]);
            f.epos[x] = (int16_t)pos;
            f.pent[pos] = (int16_t)x;
            uint32_t h = (uint32_t)(hk >> 32) & (uint32_t)(dcap - 1);
            for (int t = 0; t < dcap; ++t) {
                const unsigned long long prev =
                    atomicCAS((unsigned long long*)&f.dkey[h], (unsigned long long)kEmptyHash, (unsigned long long)hk);
                if (prev == kEmptyHash || prev == hk) break;
                h = (h + 1) & (uint32_t)(dcap - 1);
            }
            atomicMin(&f.dval[h], pos);
            f.eslot[x] = (int16_t)h;
        }
        __syncthreads();
        // each entry's first occurrence, checked token by token (a hash collision sends the tree to the serial
        // heap); first occurrences flagged by position
        for (int x = threadIdx.x; x < KB; x += kFastThreads) {
            const int mm = x / B, i = x - mm * B;
            if (i >= sh_cnt[mm]) continue;
            const int c = f.dval[f.eslot[x]];
            f.ecan[x] = (int16_t)c;
            const int pos = f.epos[x];
            if (c != pos && !same_path(x, f.pent[c])) sh_bad = 1;
            f.pnid[pos] = (int16_t)(c == pos ? 1 : 0);
        }
        __syncthreads();
        const int N = sh_ntot;
        {
            const int per = (N + kFastThreads - 1) / kFastThreads;
            const int p0 = min(N, (int)threadIdx.x * per), p1 = min(N, p0 + per);
            int local = 0;
            for (int x = p0; x < p1; ++x) local += f.pnid[x];
            int incl = local;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(MFD_FULL_MASK, incl, o);
                if (lane >= o) incl += y;
            }
            if (lane == 31) sh_wsum[warp] = incl;
            __syncthreads();
            int wv = lane < warp ? sh_wsum[lane] : 0;  // the totals of the warps before this one
#pragma unroll
            for (int o = 16; o; o >>= 1) wv += __shfl_xor_sync(MFD_FULL_MASK, wv, o);
            int run = wv + incl - local;
            for (int x = p0; x < p1; ++x) {
                const int fl = f.pnid[x];
                f.pnid[x] = (int16_t)(fl ? run + 1 : 0);
                if (fl && run + 1 == B) {  // the B-th distinct prefix's first occurrence
                    const int e = f.pent[x];
                    sh_ukey = f.ekey[e];
                    sh_umode = e / B;
                }
                run += fl;
            }
            if (threadIdx.x == kFastThreads - 1) {
                sh_total = run;
                sh_count = min(run, B);
            }
        }
        __syncthreads();
    };

    // round 1: every mode pops at most B / 4 (at least 8) entries; merge
    const int probe = min(B, max(8, B / 4));
    if (warp < K) pop_run(probe, kNoKey, K);
    __syncthreads();
    if (!sh_bad) merge();
    if (!sh_bad) {
        // a mode is complete once its next entry follows the bound (or it has none); the bound is the B-th
        // distinct prefix of round 1, so every entry the tree needs precedes it
        const bool bounded = sh_total >= B;
        const uint32_t ukey = bounded ? sh_ukey : kNoKey;
        const int umode = bounded ? sh_umode : K;
        if (warp < K) {
            const uint32_t nxt = __reduce_min_sync(MFD_FULL_MASK, min(k0, min(k1, k2)));
            const bool done = npop >= B || nxt == kNoKey || nxt > ukey || (nxt == ukey && m > umode);
            if (lane == 0) sh_done[m] = done ? 1 : 0;
        }
        __syncthreads();
        int all_done = 1;
        for (int mm = 0; mm < K; ++mm) all_done &= sh_done[mm];
        if (!all_done) {
            // round 2: the incomplete modes pop up to the bound (or to B entries when round 1 found fewer than B
            // distinct prefixes); merge again
            if (warp < K && !sh_done[m]) pop_run(B, ukey, umode);
            __syncthreads();
            if (!sh_bad) merge();
        }
    }
    if (sh_bad) {  // replay the reference heap in one thread
        if (threadIdx.x == 0) {
            int fail = 0;
            sh_count = serial_mixture(p, s, &fail);
            sh_fail = fail;
        }
        __syncthreads();
        if (sh_fail && threadIdx.x == 0 && p.status) atomicExch(p.status, (int)MFD_ERR_CAPACITY);
        if (threadIdx.x < kThreads) write_tree_outputs(p, b, sh_count, s.ntok, s.npar, s.ndep);
        return;
    }
    const int count = sh_count;
    for (int x = threadIdx.x; x < KB; x += kFastThreads) {
        const int mm = x / B, i = x - mm * B;
        if (i >= sh_cnt[mm]) continue;
        const int nid = f.pnid[f.epos[x]];
        if (nid == 0 || nid > count) continue;
        s.ntok[nid] = f.etok[x];
        s.ndep[nid] = f.edep[x];
        s.npar[nid] = (int16_t)(f.epl[x] < 0 ? 0 : f.pnid[f.ecan[mm * B + f.epl[x]]]);
    }
    __syncthreads();
    if (threadIdx.x < kThreads) write_tree_outputs(p, b, count, s.ntok, s.npar, s.ndep);
}

struct Plan {
    int ks, S, hcap, words;
    size_t smem;
};

static Plan plan(int K, int L, int k, int B) {
    Plan pl;
    const int W = B + 1;
    const int64_t live_max = (int64_t)K * (B + 1);  // K initial entries; pops <= K*B, each adds at most one
    pl.S = (int)((live_max + 31) / 32);
    if (pl.S < 2) pl.S = 2;
    pl.hcap = 64;
    while (pl.hcap < 4 * W) pl.hcap <<= 1;
    pl.words = (W + 63) / 64;
    const size_t fixed = (size_t)32 * pl.S * (8 + 8 + 4) + (size_t)pl.hcap * 8 + (size_t)W * (4 + 2 + 2 + 1) +
                         (size_t)K * 4 + 16 * 12;
    const size_t budget = 200 * 1024;
    const size_t per_rank = (size_t)K * L * 8;
    int ks = k;
    if (fixed + per_rank * ks > budget) ks = (int)((budget - fixed) / per_rank);
    if (ks < 1) ks = 1;
    pl.ks = ks;
    pl.smem = fixed + per_rank * ks + 64;
    return pl;
}

}  // namespace tree
}  // namespace mfd

using namespace mfd;

extern "C" int mfd_build_trees(const float* top_logp, const void* top_ids, int ids_dtype, const float* log_prior,
                               int64_t bs, int64_t num_modes, int64_t depth_limit, int64_t topk, int64_t budget,
                               int single, int64_t* tree, int64_t* counts, uint64_t* anc_bits, uint8_t* visibility,
                               int* status, void* stream) {
    if (bs < 0 || num_modes < 1 || depth_limit < 0 || topk < 1 || budget < 0) {
        set_error("mfd_build_trees: invalid sizes bs=%lld K=%lld L=%lld k=%lld B=%lld", (long long)bs,
                  (long long)num_modes, (long long)depth_limit, (long long)topk, (long long)budget);
        return MFD_ERR_INVALID;
    }
    if (num_modes > 16 || depth_limit > 31 || topk > 2047 || budget > 511) {
        set_error("mfd_build_trees: limits K<=16, L<=31, k<=2047, B<=511 (got K=%lld L=%lld k=%lld B=%lld)",
                  (long long)num_modes, (long long)depth_limit, (long long)topk, (long long)budget);
        return MFD_ERR_UNSUPPORTED;
    }
    if (single && num_modes != 1) {
        set_error("mfd_build_trees: the single-mode heap needs num_modes == 1");
        return MFD_ERR_INVALID;
    }
    if (ids_dtype != MFD_I32 && ids_dtype != MFD_I64) {
        set_error("mfd_build_trees: ids_dtype must be MFD_I32 or MFD_I64");
        return MFD_ERR_INVALID;
    }
    if (bs == 0) return MFD_OK;
    if (!tree || !counts || ((!top_logp || !top_ids) && depth_limit > 0 && budget > 0)) {
        set_error("mfd_build_trees: null pointer");
        return MFD_ERR_INVALID;
    }
    tree::Plan pl = tree::plan((int)num_modes, (int)depth_limit, (int)topk, (int)budget);
    if (num_modes * (budget + 1) > 32 * 64) {
        set_error("mfd_build_trees: K*(B+1) too large for the entry store (K=%lld B=%lld)", (long long)num_modes,
                  (long long)budget);
        return MFD_ERR_UNSUPPORTED;
    }
    const int64_t W = budget + 1;
    tree::Params p;
    p.lp = top_logp;
    p.ids = top_ids;
    p.ids_i64 = ids_dtype == MFD_I64;
    p.prior = log_prior;
    p.bs = bs;
    p.K = (int)num_modes;
    p.L = (int)depth_limit;
    p.k = (int)topk;
    p.B = (int)budget;
    p.single = single ? 1 : 0;
    p.ks = depth_limit > 0 ? pl.ks : 1;
    p.S = pl.S;
    p.hcap = pl.hcap;
    p.words = pl.words;
    p.tree = tree;
    p.counts = counts;
    p.anc = anc_bits;
    p.vis = visibility;
    p.status = status;
    const size_t h1_smem = tree::mixture_smem_bytes((int)num_modes, (int)depth_limit, (int)topk, (int)budget, pl.hcap) + 64;
    if (!single && depth_limit > 0 && budget > 0 && num_modes <= 16 && budget <= tree::kFastMaxB) {
        // one warp per mode, exact merge (the serial heap replays trees with exact key ties)
        const int dcap = tree::fast_dcap((int)num_modes, (int)budget);
        const size_t fsmem = h1_smem + tree::fast_smem_bytes((int)num_modes, (int)budget, dcap);
        if (fsmem <= 220 * 1024) {
            auto kern = num_modes <= 8 ? tree::mixture_fast_kernel<8> : tree::mixture_fast_kernel<16>;
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fsmem);
            if (e != cudaSuccess) {
                set_error("mfd_build_trees: %s", cudaGetErrorString(e));
                return MFD_ERR_CUDA;
            }
            kern<<<(unsigned)bs, tree::kFastThreads, fsmem, (cudaStream_t)stream>>>(p);
            MFD_CHECK_LAUNCH("mfd_build_trees");
            return MFD_OK;
        }
    }
    if (!single && depth_limit > 0 && budget > 0 && h1_smem <= 220 * 1024) {  // the mixture heap in one thread
        cudaError_t e = cudaFuncSetAttribute(tree::mixture_heap1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)h1_smem);
        if (e != cudaSuccess) {
            set_error("mfd_build_trees: %s", cudaGetErrorString(e));
            return MFD_ERR_CUDA;
        }
        tree::mixture_heap1_kernel<<<(unsigned)bs, tree::kThreads, h1_smem, (cudaStream_t)stream>>>(p);
        MFD_CHECK_LAUNCH("mfd_build_trees");
        return MFD_OK;
    }
    cudaError_t e = cudaFuncSetAttribute(tree::build_trees_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)pl.smem);
    if (e != cudaSuccess) {
        set_error("mfd_build_trees: %s", cudaGetErrorString(e));
        return MFD_ERR_CUDA;
    }
    tree::build_trees_kernel<<<(unsigned)bs, tree::kThreads, pl.smem, (cudaStream_t)stream>>>(p);
    MFD_CHECK_LAUNCH("mfd_build_trees");
    return MFD_OK;
}
