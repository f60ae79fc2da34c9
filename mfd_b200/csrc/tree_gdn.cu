// tree_gdn.cu -- tree verification of one gated-delta-rule (Gated DeltaNet) layer from the committed state.
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
// B200 design.  The ancestor set of a node in a tree is its root path, one node per depth, so the unit lower
// triangular system is solved exactly by depth levels (all nodes of one depth at once) instead of by inverting
// dense diagonal blocks; only ancestor pairs are ever formed (sum over nodes of depth+1 of them, a few hundred
// for a 65-node tree), not the dense n x n products.
//   tree_gdn_uo_kernel:     one CTA per (value head, 16-wide value slice); the value columns of u are
//                           independent, so 8 CTAs per head solve disjoint slices of the same system.  Latency
//                           bound (5.3 MB of traffic at the 65-node config).
//   tree_gdn_states_kernel: one CTA per (value head, 8 key rows) writes that band of every node's state, each
//                           warp a contiguous row of Dv floats; the 134 MB of states make it HBM-write bound.
// Arithmetic is fp32 throughout (bf16 q, k, v as given, fp32 S0, g, beta); the reference multiplies bf16-rounded
// S0 and bf16-rounded u, so this path is at least as close to the exact (float64) result.
#include "common.cuh"

namespace gdn {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxNodes = 128;
constexpr int kWords = kMaxNodes / 32;
constexpr int kMaxDk = 128;
constexpr int kMaxDv = 128;
constexpr int kBV = 16;                                 // value columns per CTA of the u/o kernel
constexpr int kBandA = 32;                              // key rows per CTA of the states kernel
constexpr int kNodeSplit = 2;                           // node ranges per (head, band) of the states kernel
constexpr int kMaxItems = kMaxNodes * kBV / kThreads;  // (node, column) items per thread of the u/o kernel

struct Params {
    const __nv_bfloat16* q;  // [n, HK, Dk], node stride sq
    const __nv_bfloat16* k;  // [n, HK, Dk], node stride sk
    const __nv_bfloat16* v;  // [n, H, Dv], node stride sv
    int64_t sq, sk, sv;
    const float* g;     // [n, H], node stride sg
    const float* beta;  // [n, H], node stride sb
    int64_t sg, sb;
    const float* s0;    // [H, Dk, Dv]
    const int8_t* anc;  // [n, n], row stride sa; anc[i][j] != 0 iff j is an ancestor of i or j == i
    int64_t sa;
    int n, H, HK, Dk, Dv;
    float* u;       // [n, H, Dv]
    float* o;       // [n, H, Dv]
    float* states;  // [n, H, Dk, Dv] or null
    int* status;    // optional: 0 ok, 1 the mask is not the ancestor matrix of a topologically ordered tree
};

__host__ __device__ constexpr int align16(int x) { return (x + 15) & ~15; }
__host__ __device__ constexpr int pair_cap(int n) { return n * (n + 1) / 2; }  // a chain of n nodes
__host__ __device__ constexpr int pad16(int n) { return (n + 15) & ~15; }

// Dynamic shared-memory layouts (byte offsets), sized for the call's n so small trees keep several CTAs per SM.
struct UoLayout {
    int kq, s, ks, qs, uu, m, pq, gg, bb, raw, node, row, total, kstride;
};
__host__ __device__ inline UoLayout uo_layout(int n, int dk) {
    UoLayout L{};
    int off = 0;
    const int pairs = pair_cap(n);
    L.kstride = dk + 8;  // bf16 elements per staged q / k row: rows land on different banks
    L.kq = off, off += align16(2 * pad16(n) * L.kstride * 2);
    L.s = off, off += align16(dk * kBV * 4);
    L.ks = off, off += align16(n * kBV * 4);
    L.qs = off, off += align16(n * kBV * 4);
    L.uu = off, off += align16(n * kBV * 4);
    L.m = off, off += align16(pairs * 4);
    L.pq = off, off += align16(pairs * 4);
    L.gg = off, off += align16(n * 4);
    L.bb = off, off += align16(n * 4);
    L.raw = off, off += align16(n * n);
    L.node = off, off += align16(pairs);
    L.row = off, off += align16(pairs);
    L.total = off;
    return L;
}
struct StLayout {
    int uu, kk, gamma, gg, raw, node, row, total;
};
__host__ __device__ inline StLayout st_layout(int n, int dv) {
    StLayout L{};
    int off = 0;
    const int pairs = pair_cap(n);
    L.uu = off, off += align16(n * dv * 4);
    L.kk = off, off += align16(n * kBandA * 4);
    L.gamma = off, off += align16(pairs * 4);
    L.gg = off, off += align16(2 * n * 4);  // G, then e^G
    L.raw = off, off += align16(n * n);
    L.node = off, off += align16(pairs);
    L.row = off, off += align16(pairs);
    L.total = off;
    return L;
}

// Root paths of all nodes, read from the ancestor mask.
struct PathsHdr {
    uint32_t bits[kMaxNodes][kWords];
    int off[kMaxNodes + 1];  // pair range of node i: [off[i], off[i] + depth[i] + 1); off[n] = pair count
    uint8_t depth[kMaxNodes];
    int max_depth;
    int bad;
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(mfd::smem_addr(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// mma.sync m16n8k16, bf16 operands, fp32 accumulators.  A fragment: a0 (row g, k 2t..2t+1), a1 (row g+8),
// a2 (row g, k 2t+8..), a3 (row g+8, k 2t+8..); B: b0 (k 2t..2t+1, col g), b1 (k 2t+8..); C: c0, c1 (row g,
// cols 2t, 2t+1), c2, c3 (row g+8) -- g = lane / 4, t = lane % 4.
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Four 8x8 bf16 matrices from shared memory; lane l supplies the address of row (l & 7) of matrix l / 8.
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(mfd::smem_addr(p)));
}
// x = hi + lo with hi, lo bfloat16: two bf16 products reproduce an fp32 operand to about 2^-16 relative.
__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
    hi = __float2bfloat16(x);
    lo = __float2bfloat16(x - __bfloat162float(hi));
}
__device__ __forceinline__ uint32_t pack2(__nv_bfloat16 a, __nv_bfloat16 b) {
    return (uint32_t)__bfloat16_as_ushort(a) | ((uint32_t)__bfloat16_as_ushort(b) << 16);
}

// Starts copying the n x n mask into raw (no barrier; complete after cp_async_wait_all + __syncthreads).
__device__ __forceinline__ void load_anc_raw(uint8_t* raw, const Params& p) {
    const int n = p.n, total = n * n;
    if (p.sa == n && ((uintptr_t)p.anc & 15u) == 0) {
        const int nv = total >> 4;
        for (int e = threadIdx.x; e < nv; e += kThreads) cp_async16(raw + e * 16, p.anc + e * 16, 16);
        for (int e = (nv << 4) + threadIdx.x; e < total; e += kThreads) raw[e] = (uint8_t)p.anc[e];
    } else {
        for (int e = threadIdx.x; e < total; e += kThreads) raw[e] = (uint8_t)p.anc[(int64_t)(e / n) * p.sa + e % n];
    }
}

// Fills ps, node[] and row[] from the staged mask (all threads call; ends with a barrier).  Invalid masks set
// ps.bad and leave the rest unspecified.
__device__ void build_paths(PathsHdr& ps, uint8_t* node, uint8_t* row, const uint8_t* raw, int n) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        ps.bad = 0;
        ps.max_depth = 0;
    }
    for (int i = warp; i < n; i += kWarps) {
#pragma unroll
        for (int w = 0; w < kWords; ++w) {
            const int c = w * 32 + lane;
            const uint32_t b = __ballot_sync(MFD_FULL_MASK, c < n && raw[i * n + c] != 0);
            if (lane == 0) ps.bits[i][w] = b;
        }
    }
    __syncthreads();
    // i in anc(i), nothing above i, and anc(i) = anc(parent) + {i} with parent = the largest strict ancestor
    for (int i = threadIdx.x; i < n; i += kThreads) {
        int cnt = 0, parent = -1;
        bool ok = (ps.bits[i][i >> 5] >> (i & 31)) & 1u;
#pragma unroll
        for (int w = 0; w < kWords; ++w) {
            const uint32_t b = ps.bits[i][w];
            const int lo = w * 32;
            if (lo > i) {
                ok &= (b == 0u);
                continue;
            }
            if (lo + 31 > i) ok &= (b >> (i - lo)) <= 1u;
            cnt += __popc(b);
            uint32_t strict = b;
            if (i < lo + 32) strict &= ~(1u << (i - lo));
            if (strict) parent = lo + 31 - __clz(strict);
        }
        if (ok && parent >= 0) {
#pragma unroll
            for (int w = 0; w < kWords; ++w) {
                uint32_t want = ps.bits[parent][w];
                if ((i >> 5) == w) want |= 1u << (i & 31);
                ok &= (want == ps.bits[i][w]);
            }
        }
        if (!ok) atomicOr(&ps.bad, 1);
        ps.depth[i] = (uint8_t)(cnt - 1);
        if (ok) atomicMax(&ps.max_depth, cnt - 1);
    }
    __syncthreads();
    if (ps.bad) return;
    if (warp == 0) {  // exclusive prefix of depth + 1 (4 nodes per lane)
        int v[4], s = 0;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int i = lane * 4 + t;
            v[t] = i < n ? (int)ps.depth[i] + 1 : 0;
            s += v[t];
        }
        int incl = s;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int y = __shfl_up_sync(MFD_FULL_MASK, incl, d);
            if (lane >= d) incl += y;
        }
        int run = incl - s;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int i = lane * 4 + t;
            if (i < n) ps.off[i] = run;
            run += v[t];
        }
        if (lane == 31) ps.off[n] = incl;
    }
    __syncthreads();
    for (int i = warp; i < n; i += kWarps) {  // the set bits of row i in ascending order (root first)
        int base = ps.off[i];
#pragma unroll
        for (int w = 0; w < kWords; ++w) {
            const uint32_t b = ps.bits[i][w];
            if ((b >> lane) & 1u) {
                const int t = base + __popc(b & ((1u << lane) - 1u));
                node[t] = (uint8_t)(w * 32 + lane);
                row[t] = (uint8_t)i;
            }
            base += __popc(b);
        }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kThreads) tree_gdn_uo_kernel(const Params p) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ PathsHdr ps;
    const int n = p.n, Dk = p.Dk, Dv = p.Dv;
    const UoLayout L = uo_layout(n, Dk);
    __nv_bfloat16* kq = (__nv_bfloat16*)(smem + L.kq);  // [2][pad16(n)][kstride]: k rows, then q rows
    float* s = (float*)(smem + L.s);                     // [Dk][kBV]: S0[h][:, slice]
    float* ks = (float*)(smem + L.ks);                   // [n][kBV]: S0^T k_i
    float* qs = (float*)(smem + L.qs);                   // [n][kBV]: S0^T q_i
    float* uu = (float*)(smem + L.uu);                   // [n][kBV]: right-hand side, then u
    float* mm = (float*)(smem + L.m);                    // [pairs]: beta_i e^{G_i-G_j} k_i.k_j (0 on the diagonal)
    float* pq = (float*)(smem + L.pq);                   // [pairs]: e^{G_i-G_j} q_i.k_j
    float* gg = (float*)(smem + L.gg);
    float* bb = (float*)(smem + L.bb);
    uint8_t* raw = smem + L.raw;
    uint8_t* node = smem + L.node;
    uint8_t* row = smem + L.row;
    const int ksd = L.kstride, np = pad16(n);
    const int h = blockIdx.x, c0 = blockIdx.y * kBV;
    const int hk = h / (p.H / p.HK);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // ---- every load issued up front: q / k rows and the S0 slice by cp.async, the mask, G, beta, v
    const int cpr = Dk >> 3;
    for (int e = threadIdx.x; e < 2 * n * cpr; e += kThreads) {
        const int which = e / (n * cpr), r = e - which * n * cpr, i = r / cpr, c = r - i * cpr;
        const __nv_bfloat16* src = (which ? p.q + (int64_t)i * p.sq : p.k + (int64_t)i * p.sk) + hk * Dk + c * 8;
        cp_async16(kq + (which * np + i) * ksd + c * 8, src, 16);
    }
    const float* s0h = p.s0 + (int64_t)h * Dk * Dv;
    for (int e = threadIdx.x; e < Dk * (kBV / 4); e += kThreads) {
        const int a = e >> 2, c = (e & 3) * 4;
        const bool ok = c0 + c < Dv;  // Dv % 4 == 0: 4-column chunks are whole or absent
        cp_async16(s + a * kBV + c, ok ? s0h + (int64_t)a * Dv + c0 + c : s0h, ok ? 16 : 0);
    }
    load_anc_raw(raw, p);
    for (int e = threadIdx.x; e < 2 * n; e += kThreads) {
        if (e < n) gg[e] = p.g[(int64_t)e * p.sg + h];
        else bb[e - n] = p.beta[(int64_t)(e - n) * p.sb + h];
    }
    float vreg[kMaxItems];
#pragma unroll
    for (int r = 0; r < kMaxItems; ++r) {
        const int it = threadIdx.x + r * kThreads, i = it / kBV, c = it % kBV;
        vreg[r] = (it < n * kBV && c0 + c < Dv) ? __bfloat162float(p.v[(int64_t)i * p.sv + (int64_t)h * Dv + c0 + c])
                                                : 0.f;
    }
    cp_async_wait_all();
    __syncthreads();
    build_paths(ps, node, row, raw, n);
    if (ps.bad) {
        if (p.status && h == 0 && blockIdx.y == 0 && threadIdx.x == 0) *p.status = 1;
        return;
    }
    if (p.status && h == 0 && blockIdx.y == 0 && threadIdx.x == 0) *p.status = 0;

    const int g = lane >> 2, tq = lane & 3;
    const int mt = np >> 4;  // 16-row tiles of nodes
    // ---- S0^T k_i and S0^T q_i over the slice on the tensor cores: task = (k or q, 16-node tile), S split into
    //      bf16 hi + lo so the product keeps fp32 accuracy; 2 column tiles of 8
    for (int task = warp; task < 2 * mt; task += kWarps) {
        const int which = task / mt, m0 = (task % mt) * 16;
        const __nv_bfloat16* arow = kq + (which * np + m0 + (lane & 15)) * ksd + (lane >> 4) * 8;
        float acc[2][4] = {};
        for (int k0 = 0; k0 < Dk; k0 += 16) {
            uint32_t a[4];
            ldsm_x4(a, arow + k0);
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                const int col = nt * 8 + g;
                __nv_bfloat16 h0, l0, h1, l1, h2, l2, h3, l3;
                split_bf16(s[(k0 + 2 * tq) * kBV + col], h0, l0);
                split_bf16(s[(k0 + 2 * tq + 1) * kBV + col], h1, l1);
                split_bf16(s[(k0 + 2 * tq + 8) * kBV + col], h2, l2);
                split_bf16(s[(k0 + 2 * tq + 9) * kBV + col], h3, l3);
                mma16816(acc[nt], a, pack2(h0, h1), pack2(h2, h3));
                mma16816(acc[nt], a, pack2(l0, l1), pack2(l2, l3));
            }
        }
        float* dst = which ? qs : ks;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            const int r0 = m0 + g, cc = nt * 8 + 2 * tq;
            if (r0 < n) *reinterpret_cast<float2*>(dst + r0 * kBV + cc) = make_float2(acc[nt][0], acc[nt][1]);
            if (r0 + 8 < n) *reinterpret_cast<float2*>(dst + (r0 + 8) * kBV + cc) = make_float2(acc[nt][2], acc[nt][3]);
        }
    }
    // ---- Gram products k_i.k_j and q_i.k_j on the tensor cores over the lower-triangular 16x16 tiles; only
    //      ancestor pairs (j in anc(i)) are kept, at pair slot off[i] + depth[j]
    for (int task = warp; task < mt * (mt + 1) / 2; task += kWarps) {
        int mi = 0;
        while ((mi + 1) * (mi + 2) / 2 <= task) ++mi;
        const int nj = task - mi * (mi + 1) / 2;
        const int m0 = mi * 16, j0 = nj * 16;
        const __nv_bfloat16* krow = kq + (m0 + (lane & 15)) * ksd + (lane >> 4) * 8;
        const __nv_bfloat16* qrow = kq + (np + m0 + (lane & 15)) * ksd + (lane >> 4) * 8;
        const __nv_bfloat16* brow = kq + (j0 + (lane & 7) + (lane >> 4) * 8) * ksd + ((lane >> 3) & 1) * 8;
        float ckk[2][4] = {}, cqk[2][4] = {};
        for (int k0 = 0; k0 < Dk; k0 += 16) {
            uint32_t ak[4], aq[4], b[4];
            ldsm_x4(ak, krow + k0);
            ldsm_x4(aq, qrow + k0);
            ldsm_x4(b, brow + k0);
            mma16816(ckk[0], ak, b[0], b[1]);
            mma16816(ckk[1], ak, b[2], b[3]);
            mma16816(cqk[0], aq, b[0], b[1]);
            mma16816(cqk[1], aq, b[2], b[3]);
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i = m0 + g + (e >> 1) * 8, j = j0 + nt * 8 + 2 * tq + (e & 1);
                if (i < n && j <= i && ((ps.bits[i][j >> 5] >> (j & 31)) & 1u)) {
                    const int t = ps.off[i] + ps.depth[j];
                    const float gamma = expf(gg[i] - gg[j]);
                    mm[t] = (i == j) ? 0.f : bb[i] * gamma * ckk[nt][e];
                    pq[t] = gamma * cqk[nt][e];
                }
            }
        }
    }
    __syncthreads();
    // ---- right-hand side beta_i (v_i - e^{G_i} S0^T k_i)
#pragma unroll
    for (int r = 0; r < kMaxItems; ++r) {
        const int it = threadIdx.x + r * kThreads;
        if (it < n * kBV) {
            const int i = it / kBV;
            uu[it] = bb[i] * (vreg[r] - expf(gg[i]) * ks[it]);
        }
    }
    __syncthreads();
    // ---- forward substitution by depth: every strict ancestor of a depth-d node has depth < d
    for (int d = 1; d <= ps.max_depth; ++d) {
        for (int it = threadIdx.x; it < n * kBV; it += kThreads) {
            const int i = it / kBV, c = it % kBV;
            if (ps.depth[i] != d) continue;
            const int o0 = ps.off[i];
            float acc = uu[it];
            for (int t = 0; t < d; ++t) acc = fmaf(-mm[o0 + t], uu[node[o0 + t] * kBV + c], acc);
            uu[it] = acc;
        }
        __syncthreads();
    }
    // ---- outputs
    for (int it = threadIdx.x; it < n * kBV; it += kThreads) {
        const int i = it / kBV, c = it % kBV;
        if (c0 + c >= Dv) continue;
        const int o0 = ps.off[i], d = ps.depth[i];
        float acc = expf(gg[i]) * qs[it];
        for (int t = 0; t <= d; ++t) acc = fmaf(pq[o0 + t], uu[node[o0 + t] * kBV + c], acc);
        const int64_t at = ((int64_t)i * p.H + h) * Dv + c0 + c;
        p.o[at] = acc;
        p.u[at] = uu[it];
    }
}

__global__ void __launch_bounds__(kThreads) tree_gdn_states_kernel(const Params p) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ PathsHdr ps;
    const int n = p.n, Dk = p.Dk, Dv = p.Dv;
    const StLayout L = st_layout(n, Dv);
    float* uu = (float*)(smem + L.uu);  // [n][Dv]
    float* kk = (float*)(smem + L.kk);  // [n][kBandA]: this band's key entries
    float* gamma = (float*)(smem + L.gamma);
    float* gg = (float*)(smem + L.gg);  // [n] G, then [n] e^G
    uint8_t* raw = smem + L.raw;
    uint8_t* node = smem + L.node;
    uint8_t* row = smem + L.row;
    const int h = blockIdx.x, a0 = blockIdx.y * kBandA;
    const int hk = h / (p.H / p.HK);
    const int dv4 = Dv >> 2;
    for (int e = threadIdx.x; e < n * dv4; e += kThreads) {
        const int i = e / dv4, c = e - i * dv4;
        cp_async16(uu + i * Dv + c * 4, p.u + ((int64_t)i * p.H + h) * Dv + c * 4, 16);
    }
    load_anc_raw(raw, p);
    for (int e = threadIdx.x; e < n * (kBandA / 8); e += kThreads) {  // 8 key entries per 16-byte load
        const int i = e / (kBandA / 8), c8 = (e % (kBandA / 8)) * 8;
        uint4 w = make_uint4(0u, 0u, 0u, 0u);
        if (a0 + c8 < Dk) w = *reinterpret_cast<const uint4*>(p.k + (int64_t)i * p.sk + (int64_t)hk * Dk + a0 + c8);
        float* d = kk + i * kBandA + c8;
        *reinterpret_cast<float4*>(d) = make_float4(mfd::bf16lo(w.x), mfd::bf16hi(w.x), mfd::bf16lo(w.y), mfd::bf16hi(w.y));
        *reinterpret_cast<float4*>(d + 4) =
            make_float4(mfd::bf16lo(w.z), mfd::bf16hi(w.z), mfd::bf16lo(w.w), mfd::bf16hi(w.w));
    }
    for (int i = threadIdx.x; i < n; i += kThreads) {
        const float G = p.g[(int64_t)i * p.sg + h];
        gg[i] = G;
        gg[n + i] = expf(G);
    }
    cp_async_wait_all();
    __syncthreads();
    build_paths(ps, node, row, raw, n);
    if (ps.bad) return;
    const int npairs = ps.off[n];
    for (int t = threadIdx.x; t < npairs; t += kThreads) gamma[t] = expf(gg[row[t]] - gg[node[t]]);
    __syncthreads();
    // thread -> (key rows a0 + 4w .. +3, value columns 4c .. 4c+3): 16 outputs per node from one float4 of this
    // band's key entries and one float4 of u per ancestor; each warp writes 4 contiguous rows per node
    const int w4 = (threadIdx.x >> 5) * 4, c = threadIdx.x & 31;
    if (c >= dv4 || a0 + w4 >= Dk) return;
    const int per = (n + kNodeSplit - 1) / kNodeSplit;
    const int i0 = blockIdx.z * per, i1 = min(n, i0 + per);
    float4 s4[4];
    float4* dst[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int a = a0 + w4 + r;
        const bool live = a < Dk;
        s4[r] = live ? *reinterpret_cast<const float4*>(p.s0 + ((int64_t)h * Dk + a) * Dv + c * 4)
                     : make_float4(0.f, 0.f, 0.f, 0.f);
        dst[r] = reinterpret_cast<float4*>(p.states + ((int64_t)h * Dk + (live ? a : a0)) * Dv + c * 4);
    }
    const int rows = min(4, Dk - a0 - w4);
    const int64_t node_stride4 = (int64_t)p.H * Dk * Dv / 4;
    for (int i = i0; i < i1; ++i) {
        const float e = gg[n + i];
        float4 acc[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[r] = make_float4(e * s4[r].x, e * s4[r].y, e * s4[r].z, e * s4[r].w);
        const int o0 = ps.off[i], d = ps.depth[i];
        for (int t = 0; t <= d; ++t) {
            const int j = node[o0 + t];
            const float gm = gamma[o0 + t];
            const float4 kj = *reinterpret_cast<const float4*>(kk + j * kBandA + w4);
            const float4 uj = *reinterpret_cast<const float4*>(uu + j * Dv + c * 4);
            const float wv[4] = {gm * kj.x, gm * kj.y, gm * kj.z, gm * kj.w};
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                acc[r].x = fmaf(wv[r], uj.x, acc[r].x);
                acc[r].y = fmaf(wv[r], uj.y, acc[r].y);
                acc[r].z = fmaf(wv[r], uj.z, acc[r].z);
                acc[r].w = fmaf(wv[r], uj.w, acc[r].w);
            }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
            if (r < rows) __stcs(dst[r] + i * node_stride4, acc[r]);
    }
}

// ---------------------------------------------------------------------------------------------- tree_prep
// Short causal convolution over each node's window (gathered through parent pointers; window entries below KC
// are the cached conv inputs), SiLU rounded to bf16, then l2 normalisation (and the q scale) per head of q and k,
// as inference/hf/tree_gdn_kernel.py:27-56 (_tree_prep) and 135-150 (tree_prep).  One CTA per (16 nodes, head
// group), one thread per channel of the head; head groups are q (HK), k (HK), v (H) in channel order.
constexpr int kPrepNodes = 16;
constexpr int kMaxConv = 8;

struct PrepParams {
    const __nv_bfloat16* x;           // [n, CD]
    const __nv_bfloat16* conv_state;  // [CD, KC]
    const int32_t* conv_index;        // [n, KC] into [conv state ; nodes]
    const __nv_bfloat16* conv_w;      // [CD, KC]
    __nv_bfloat16 *q, *k, *v;         // [n, HK, D], [n, HK, D], [n, H, D]
    int n, cd, kc, HK, H, D;
    float scale;
};

template <int KC>
__global__ void __launch_bounds__(kMaxDk) tree_prep_kernel(const PrepParams p) {
    __shared__ int sidx[kPrepNodes][KC];
    __shared__ float red[kMaxDk / 32][kPrepNodes];
    const int hg = blockIdx.y, d = threadIdx.x, warp = d >> 5, lane = d & 31;
    const int i0 = blockIdx.x * kPrepNodes;
    const bool live = d < p.D;
    const int ch = hg * p.D + (live ? d : 0);
    if (threadIdx.x < kPrepNodes * KC) {
        const int t = threadIdx.x / KC, j = threadIdx.x % KC, i = i0 + t;
        int idx = -1;
        if (i < p.n) {
            idx = p.conv_index[(int64_t)i * KC + j];
            if (idx < 0 || idx >= KC + p.n) idx = -1;  // not a window entry: contributes nothing
        }
        sidx[t][j] = idx;
    }
    float w[KC];
#pragma unroll
    for (int j = 0; j < KC; ++j) w[j] = __bfloat162float(p.conv_w[(int64_t)ch * KC + j]);
    __syncthreads();
    // every window load of the 16 nodes is independent and unconditional (absent entries read the first cached
    // input and weigh 0): issue them all, then accumulate oldest first
    float xv[kPrepNodes][KC];
#pragma unroll
    for (int t = 0; t < kPrepNodes; ++t) {
#pragma unroll
        for (int j = 0; j < KC; ++j) {
            const int idx = sidx[t][j];
            const __nv_bfloat16* src = idx < KC ? p.conv_state + (int64_t)ch * KC + (idx < 0 ? 0 : idx)
                                                : p.x + (int64_t)(idx - KC) * p.cd + ch;
            xv[t][j] = idx < 0 ? 0.f : __bfloat162float(*src);
        }
    }
    float y[kPrepNodes];
#pragma unroll
    for (int t = 0; t < kPrepNodes; ++t) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < KC; ++j) acc = fmaf(xv[t][j], w[j], acc);
        const float silu = acc / (1.f + expf(-acc));
        y[t] = live ? __bfloat162float(__float2bfloat16(silu)) : 0.f;
    }
    const bool norm = hg < 2 * p.HK;
    if (norm) {
#pragma unroll
        for (int t = 0; t < kPrepNodes; ++t) {
            float sq = y[t] * y[t];
#pragma unroll
            for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(MFD_FULL_MASK, sq, o);
            if (lane == 0) red[warp][t] = sq;
        }
        __syncthreads();
    }
    if (!live) return;
#pragma unroll
    for (int t = 0; t < kPrepNodes; ++t) {
        const int i = i0 + t;
        if (i >= p.n) break;
        float val = y[t];
        if (norm) {
            float ss = 0.f;
            for (int w2 = 0; w2 < (p.D + 31) / 32; ++w2) ss += red[w2][t];
            val = val * rsqrtf(ss + 1e-6f);
            if (hg < p.HK) {
                p.q[((int64_t)i * p.HK + hg) * p.D + d] = __float2bfloat16(val * p.scale);
            } else {
                p.k[((int64_t)i * p.HK + hg - p.HK) * p.D + d] = __float2bfloat16(val);
            }
        } else {
            p.v[((int64_t)i * p.H + hg - 2 * p.HK) * p.D + d] = __float2bfloat16(val);
        }
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
    if (n > kMaxNodes || dk > kMaxDk || dv > kMaxDv || dk % 8 || dv % 4) {
        mfd::set_error("mfd_tree_gdn: supports n <= %d nodes, Dk <= %d a multiple of 8 and Dv <= %d a multiple of 4 "
                       "(got n=%lld Dk=%lld Dv=%lld)", kMaxNodes, kMaxDk, kMaxDv, (long long)n, (long long)dk,
                       (long long)dv);
        return MFD_ERR_UNSUPPORTED;
    }
    if (!q || !k || !v || !g_cum || !beta || !s0 || !anc || !u || !o) {
        mfd::set_error("mfd_tree_gdn: null pointer");
        return MFD_ERR_INVALID;
    }
    if (((uintptr_t)q | (uintptr_t)k) % 16 || (sq | sk) % 8 || (uintptr_t)s0 % 16 || (uintptr_t)u % 16 ||
        (states && (uintptr_t)states % 16)) {
        mfd::set_error("mfd_tree_gdn: q, k need 16-byte aligned rows (node strides multiples of 8); s0, u and "
                       "states 16-byte alignment");
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
    {
        const size_t smem = (size_t)uo_layout((int)n, (int)dk).total;
        cudaError_t e = cudaFuncSetAttribute(tree_gdn_uo_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) {
            mfd::set_error("mfd_tree_gdn: %s", cudaGetErrorString(e));
            return MFD_ERR_CUDA;
        }
        dim3 grid((unsigned)num_heads, (unsigned)((dv + kBV - 1) / kBV));
        tree_gdn_uo_kernel<<<grid, kThreads, smem, st>>>(p);
        MFD_CHECK_LAUNCH("mfd_tree_gdn");
    }
    if (states) {
        const size_t smem = (size_t)st_layout((int)n, (int)dv).total;
        cudaError_t e =
            cudaFuncSetAttribute(tree_gdn_states_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) {
            mfd::set_error("mfd_tree_gdn: %s", cudaGetErrorString(e));
            return MFD_ERR_CUDA;
        }
        dim3 grid((unsigned)num_heads, (unsigned)((dk + kBandA - 1) / kBandA), (unsigned)kNodeSplit);
        tree_gdn_states_kernel<<<grid, kThreads, smem, st>>>(p);
        MFD_CHECK_LAUNCH("mfd_tree_gdn (states)");
    }
    return MFD_OK;
}

extern "C" int mfd_tree_prep(const void* x, const void* conv_state, const int32_t* conv_index, const void* conv_w,
                             int64_t n, int64_t conv_dim, int64_t kernel, int64_t num_k_heads, int64_t num_heads,
                             int64_t head_dim, float scale, void* q, void* k, void* v, void* stream) {
    using namespace gdn;
    if (n < 0 || kernel <= 0 || num_k_heads <= 0 || num_heads <= 0 || head_dim <= 0 ||
        conv_dim != (2 * num_k_heads + num_heads) * head_dim) {
        mfd::set_error("mfd_tree_prep: invalid sizes n=%lld conv_dim=%lld kernel=%lld HK=%lld H=%lld D=%lld",
                       (long long)n, (long long)conv_dim, (long long)kernel, (long long)num_k_heads,
                       (long long)num_heads, (long long)head_dim);
        return MFD_ERR_INVALID;
    }
    if (n == 0) return MFD_OK;
    if (head_dim > kMaxDk || kernel > kMaxConv) {
        mfd::set_error("mfd_tree_prep: head_dim <= %d and kernel <= %d supported (got %lld, %lld)", kMaxDk, kMaxConv,
                       (long long)head_dim, (long long)kernel);
        return MFD_ERR_UNSUPPORTED;
    }
    if (!x || !conv_state || !conv_index || !conv_w || !q || !k || !v) {
        mfd::set_error("mfd_tree_prep: null pointer");
        return MFD_ERR_INVALID;
    }
    PrepParams p;
    p.x = (const __nv_bfloat16*)x;
    p.conv_state = (const __nv_bfloat16*)conv_state;
    p.conv_index = conv_index;
    p.conv_w = (const __nv_bfloat16*)conv_w;
    p.q = (__nv_bfloat16*)q;
    p.k = (__nv_bfloat16*)k;
    p.v = (__nv_bfloat16*)v;
    p.n = (int)n;
    p.cd = (int)conv_dim;
    p.kc = (int)kernel;
    p.HK = (int)num_k_heads;
    p.H = (int)num_heads;
    p.D = (int)head_dim;
    p.scale = scale;
    dim3 grid((unsigned)((n + kPrepNodes - 1) / kPrepNodes), (unsigned)(2 * num_k_heads + num_heads));
    cudaStream_t st = (cudaStream_t)stream;
    switch (kernel) {
        case 1: tree_prep_kernel<1><<<grid, kMaxDk, 0, st>>>(p); break;
        case 2: tree_prep_kernel<2><<<grid, kMaxDk, 0, st>>>(p); break;
        case 3: tree_prep_kernel<3><<<grid, kMaxDk, 0, st>>>(p); break;
        case 4: tree_prep_kernel<4><<<grid, kMaxDk, 0, st>>>(p); break;
        case 5: tree_prep_kernel<5><<<grid, kMaxDk, 0, st>>>(p); break;
        case 6: tree_prep_kernel<6><<<grid, kMaxDk, 0, st>>>(p); break;
        case 7: tree_prep_kernel<7><<<grid, kMaxDk, 0, st>>>(p); break;
        default: tree_prep_kernel<8><<<grid, kMaxDk, 0, st>>>(p); break;
    }
    MFD_CHECK_LAUNCH("mfd_tree_prep");
    return MFD_OK;
}
