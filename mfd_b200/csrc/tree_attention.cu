// tree_attention.cu -- tree-masked GQA verify attention.
//
// softmax(q k^T * scale + mask) v for the B+1 tree rows of every request, where row i sees every
// prefix key and, among the tree keys, exactly its ancestors and itself (the additive mask of
// inference/hf/ddtree.py:352-356, the flashinfer custom mask of sglang-v0.5.22-mfd.patch:1625-1703).
// The mask comes from the builder's ancestor bitsets, never a dense [n, prefix + n] tensor.
//
// Layout: q, out [bs, n, H, D] (D = 128 contiguous); k, v [bs, Hkv, S, D] (HF cache layout: the prefix
// keys [0, prefix_b) followed by the n tree keys [prefix_b, prefix_b + n)); anc [bs, n, words].
// GQA packing: the G = H / Hkv query heads sharing a KV head are packed as rows r = node * G + g, so one
// key tile feeds G x n rows.  Each CTA takes 64 packed rows of one (request, KV head) over one split of the
// keys (flash-decoding); per-split (o, lse) partials are merged by a second kernel.
#include "common.cuh"

namespace mfd {
namespace attn {

constexpr int D = 128;
constexpr int kRows = 64;     // packed rows per CTA (4 warps x 16)
constexpr int kKeys = 64;     // keys per tile
constexpr int kThreads = 128;

struct Params {
    const __nv_bfloat16* q;   // [bs, n, H, D]
    int64_t sq_b, sq_n, sq_h;
    const __nv_bfloat16* k;   // [bs, Hkv, S, D]
    int64_t sk_b, sk_h, sk_s;
    const __nv_bfloat16* v;
    int64_t sv_b, sv_h, sv_s;
    const int32_t* prefix;    // [bs] prefix lengths (device)
    int prefix_const;         // used when prefix == null
    const uint64_t* anc;      // [bs, n, words]
    int words;
    int n, H, Hkv, G;
    float scale_log2;         // scale * log2(e)
    int splits;
    float* o_part;            // [splits, bs, Hkv, n*G, D]
    float* lse_part;          // [splits, bs, Hkv, n*G]
    __nv_bfloat16* out;       // [bs, n, H, D]
    int64_t so_b, so_n, so_h;
    int bs;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool ok) {
    const uint32_t d = smem_u32(dst);
    const int sz = ok ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(sz));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// 128-element (256-byte) rows, 16 chunks of 16 bytes, chunk c of row r stored at c ^ (r & 7)
__device__ __forceinline__ int swz(int row, int chunk) { return row * 16 + (chunk ^ (row & 7)); }

struct __align__(16) Smem {
    uint4 q[kRows * 16];
    uint4 k[2][kKeys * 16];
    uint4 v[2][kKeys * 16];
};

__global__ void __launch_bounds__(kThreads) tree_attn_kernel(Params p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
    const int split = blockIdx.z;
    const int b = blockIdx.y / p.Hkv, hk = blockIdx.y % p.Hkv;
    const int row0 = blockIdx.x * kRows;
    const int nrows = p.n * p.G;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int prefix = p.prefix ? p.prefix[b] : p.prefix_const;
    const int total = prefix + p.n;
    // this split's key range, in whole tiles
    int chunk = (total + p.splits - 1) / p.splits;
    chunk = (chunk + kKeys - 1) / kKeys * kKeys;
    const int k_lo = split * chunk;
    const int k_hi = min(total, k_lo + chunk);

    // ---- Q tile: packed row r -> node r / G, head hk * G + r % G
    for (int c = threadIdx.x; c < kRows * 16; c += kThreads) {
        const int r = c >> 4, ch = c & 15;
        const int pr = row0 + r;
        const bool ok = pr < nrows;
        const int node = ok ? pr / p.G : 0, head = hk * p.G + (ok ? pr % p.G : 0);
        const __nv_bfloat16* src = p.q + (size_t)b * p.sq_b + (size_t)node * p.sq_n + (size_t)head * p.sq_h + ch * 8;
        cp_async16(&sm.q[swz(r, ch)], src, ok);
    }
    cp_async_commit();

    const __nv_bfloat16* kbase = p.k + (size_t)b * p.sk_b + (size_t)hk * p.sk_h;
    const __nv_bfloat16* vbase = p.v + (size_t)b * p.sv_b + (size_t)hk * p.sv_h;
    auto load_tile = [&](int buf, int key0) {
        for (int c = threadIdx.x; c < kKeys * 16; c += kThreads) {
            const int r = c >> 4, ch = c & 15;
            const int key = key0 + r;
            const bool ok = key < k_hi;
            const int kk = ok ? key : 0;
            cp_async16(&sm.k[buf][swz(r, ch)], kbase + (size_t)kk * p.sk_s + ch * 8, ok);
            cp_async16(&sm.v[buf][swz(r, ch)], vbase + (size_t)kk * p.sv_s + ch * 8, ok);
        }
    };

    const int ntiles = k_hi > k_lo ? (k_hi - k_lo + kKeys - 1) / kKeys : 0;
    if (ntiles > 0) load_tile(0, k_lo);
    cp_async_commit();

    // rows of this thread: warp*16 + g and + 8
    const int g = lane >> 2, t = lane & 3;
    const int pr0 = row0 + warp * 16 + g, pr1 = pr0 + 8;
    const int node0 = pr0 < nrows ? pr0 / p.G : 0, node1 = pr1 < nrows ? pr1 / p.G : 0;
    const uint64_t* anc0 = p.anc + ((size_t)b * p.n + node0) * p.words;
    const uint64_t* anc1 = p.anc + ((size_t)b * p.n + node1) * p.words;

    float o[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    uint32_t qa[8][4];

    cp_async_wait<1>();
    __syncthreads();
    // Q fragments into registers
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
        const int r = warp * 16 + (lane & 15);
        const int ch = kk * 2 + (lane >> 4);
        ldsm_x4(qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], &sm.q[swz(r, ch)]);
    }

    for (int it = 0; it < ntiles; ++it) {
        const int buf = it & 1;
        const int key0 = k_lo + it * kKeys;
        if (it + 1 < ntiles) load_tile(buf ^ 1, key0 + kKeys);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();

        // S = Q K^T  (16 x 64 per warp)
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
            for (int jp = 0; jp < 4; ++jp) {
                // keys 16jp..16jp+15: matrices (keys lo8, d lo), (keys lo8, d hi), (keys hi8, d lo), (keys hi8, d hi)
                const int kr = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
                const int ch = kk * 2 + ((lane >> 3) & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(b0, b1, b2, b3, &sm.k[buf][swz(kr, ch)]);
                mma16816(s[2 * jp], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
                mma16816(s[2 * jp + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
            }
        }
        // mask + online softmax
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int key = key0 + j * 8 + 2 * t + e;
                bool vis0, vis1;
                if (key < prefix) {
                    vis0 = vis1 = true;
                } else if (key < k_hi) {
                    const int tj = key - prefix;
                    vis0 = (__ldg(anc0 + (tj >> 6)) >> (tj & 63)) & 1ull;
                    vis1 = (__ldg(anc1 + (tj >> 6)) >> (tj & 63)) & 1ull;
                } else {
                    vis0 = vis1 = false;
                }
                s[j][e] = vis0 ? s[j][e] * p.scale_log2 : -INFINITY;
                s[j][2 + e] = vis1 ? s[j][2 + e] * p.scale_log2 : -INFINITY;
                mx0 = fmaxf(mx0, s[j][e]);
                mx1 = fmaxf(mx1, s[j][2 + e]);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(MFD_FULL_MASK, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(MFD_FULL_MASK, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(MFD_FULL_MASK, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(MFD_FULL_MASK, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float a0 = mn0 == -INFINITY ? 1.f : fast_exp2(m0 - mn0);
        const float a1 = mn1 == -INFINITY ? 1.f : fast_exp2(m1 - mn1);
        float rs0 = 0.f, rs1 = 0.f;
        uint32_t pa[4][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float p0 = mn0 == -INFINITY ? 0.f : fast_exp2(s[j][0] - mn0);
            const float p1 = mn0 == -INFINITY ? 0.f : fast_exp2(s[j][1] - mn0);
            const float p2 = mn1 == -INFINITY ? 0.f : fast_exp2(s[j][2] - mn1);
            const float p3 = mn1 == -INFINITY ? 0.f : fast_exp2(s[j][3] - mn1);
            rs0 += p0 + p1;
            rs1 += p2 + p3;
            // A fragment of P for k-step j/2
            if ((j & 1) == 0) {
                pa[j >> 1][0] = pack_bf16(p0, p1);
                pa[j >> 1][1] = pack_bf16(p2, p3);
            } else {
                pa[j >> 1][2] = pack_bf16(p0, p1);
                pa[j >> 1][3] = pack_bf16(p2, p3);
            }
        }
        l0 = l0 * a0 + rs0;
        l1 = l1 * a1 + rs1;
        m0 = mn0;
        m1 = mn1;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            o[i][0] *= a0;
            o[i][1] *= a0;
            o[i][2] *= a1;
            o[i][3] *= a1;
        }
        // O += P V
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int dp = 0; dp < 8; ++dp) {
                // keys 16kk..+16, d 16dp..+16: matrices (keys lo, d lo), (keys hi, d lo), (keys lo, d hi), (keys hi, d hi)
                const int kr = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
                const int ch = dp * 2 + (lane >> 4);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(b0, b1, b2, b3, &sm.v[buf][swz(kr, ch)]);
                mma16816(o[2 * dp], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b0, b1);
                mma16816(o[2 * dp + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b2, b3);
            }
        }
        __syncthreads();
    }

    // row sums across the quad
    l0 += __shfl_xor_sync(MFD_FULL_MASK, l0, 1);
    l0 += __shfl_xor_sync(MFD_FULL_MASK, l0, 2);
    l1 += __shfl_xor_sync(MFD_FULL_MASK, l1, 1);
    l1 += __shfl_xor_sync(MFD_FULL_MASK, l1, 2);
    const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
    const size_t part_row = (((size_t)split * p.bs + b) * p.Hkv + hk) * (size_t)nrows;
    if (pr0 < nrows) {
        float* dst = p.o_part + (part_row + pr0) * D;
#pragma unroll
        for (int i = 0; i < 16; ++i)
            *reinterpret_cast<float2*>(dst + i * 8 + 2 * t) = make_float2(o[i][0] * inv0, o[i][1] * inv0);
        if (t == 0) p.lse_part[part_row + pr0] = l0 > 0.f ? m0 + __log2f(l0) : -INFINITY;
    }
    if (pr1 < nrows) {
        float* dst = p.o_part + (part_row + pr1) * D;
#pragma unroll
        for (int i = 0; i < 16; ++i)
            *reinterpret_cast<float2*>(dst + i * 8 + 2 * t) = make_float2(o[i][2] * inv1, o[i][3] * inv1);
        if (t == 0) p.lse_part[part_row + pr1] = l1 > 0.f ? m1 + __log2f(l1) : -INFINITY;
    }
}

// merge the split partials: one warp per packed row, 4 d-values per lane
__global__ void tree_attn_merge_kernel(Params p) {
    const int nrows = p.n * p.G;
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t total_rows = (int64_t)p.bs * p.Hkv * nrows;
    if (gw >= total_rows) return;
    const int pr = (int)(gw % nrows);
    const int hk = (int)((gw / nrows) % p.Hkv);
    const int b = (int)(gw / ((int64_t)nrows * p.Hkv));
    float m = -INFINITY;
    for (int s = 0; s < p.splits; ++s) {
        const size_t row = (((size_t)s * p.bs + b) * p.Hkv + hk) * (size_t)nrows + pr;
        m = fmaxf(m, p.lse_part[row]);
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    float wsum = 0.f;
    if (m != -INFINITY) {
        for (int s = 0; s < p.splits; ++s) {
            const size_t row = (((size_t)s * p.bs + b) * p.Hkv + hk) * (size_t)nrows + pr;
            const float l = p.lse_part[row];
            if (l == -INFINITY) continue;
            const float w = fast_exp2(l - m);
            wsum += w;
            const float4 v = *reinterpret_cast<const float4*>(p.o_part + row * D + lane * 4);
            acc[0] += w * v.x;
            acc[1] += w * v.y;
            acc[2] += w * v.z;
            acc[3] += w * v.w;
        }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    const int node = pr / p.G, head = hk * p.G + pr % p.G;
    __nv_bfloat16* dst = p.out + (size_t)b * p.so_b + (size_t)node * p.so_n + (size_t)head * p.so_h + lane * 4;
    __nv_bfloat162 v01 = __floats2bfloat162_rn(acc[0] * inv, acc[1] * inv);
    __nv_bfloat162 v23 = __floats2bfloat162_rn(acc[2] * inv, acc[3] * inv);
    reinterpret_cast<__nv_bfloat162*>(dst)[0] = v01;
    reinterpret_cast<__nv_bfloat162*>(dst)[1] = v23;
}

}  // namespace attn
}  // namespace mfd

using namespace mfd;

extern "C" size_t mfd_tree_attention_workspace(int64_t bs, int64_t n, int64_t num_heads, int64_t splits) {
    if (bs <= 0 || n <= 0 || num_heads <= 0 || splits <= 0) return 0;
    const size_t rows = (size_t)splits * bs * num_heads * n;
    return rows * attn::D * sizeof(float) + rows * sizeof(float) + 256;
}

extern "C" int mfd_tree_attention(const void* q, int64_t sq_b, int64_t sq_n, int64_t sq_h, const void* k,
                                  int64_t sk_b, int64_t sk_h, int64_t sk_s, const void* v, int64_t sv_b,
                                  int64_t sv_h, int64_t sv_s, const int32_t* prefix_lens, int64_t prefix_len,
                                  const uint64_t* anc_bits, int64_t anc_words, int64_t bs, int64_t n,
                                  int64_t num_heads, int64_t num_kv_heads, int64_t head_dim, float scale,
                                  int64_t splits, void* out, int64_t so_b, int64_t so_n, int64_t so_h,
                                  void* workspace, size_t workspace_bytes, void* stream) {
    if (bs < 0 || n < 1 || num_heads < 1 || num_kv_heads < 1 || num_heads % num_kv_heads || splits < 1 ||
        anc_words < (n + 63) / 64) {
        set_error("mfd_tree_attention: invalid sizes bs=%lld n=%lld H=%lld Hkv=%lld splits=%lld words=%lld",
                  (long long)bs, (long long)n, (long long)num_heads, (long long)num_kv_heads, (long long)splits,
                  (long long)anc_words);
        return MFD_ERR_INVALID;
    }
    if (head_dim != attn::D) {
        set_error("mfd_tree_attention: head_dim must be 128 (got %lld)", (long long)head_dim);
        return MFD_ERR_UNSUPPORTED;
    }
    if (bs == 0) return MFD_OK;
    if (!q || !k || !v || !anc_bits || !out) {
        set_error("mfd_tree_attention: null pointer");
        return MFD_ERR_INVALID;
    }
    const size_t need = mfd_tree_attention_workspace(bs, n, num_heads, splits);
    if (!workspace || workspace_bytes < need) {
        set_error("mfd_tree_attention: workspace of %zu bytes needed", need);
        return MFD_ERR_INVALID;
    }
    // 16-byte alignment of every row start (cp.async)
    const int64_t strides[] = {sq_b, sq_n, sq_h, sk_b, sk_h, sk_s, sv_b, sv_h, sv_s};
    for (int64_t s : strides)
        if (s % 8) {
            set_error("mfd_tree_attention: strides must be multiples of 8 elements");
            return MFD_ERR_INVALID;
        }
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) & 15u) {
        set_error("mfd_tree_attention: q, k, v must be 16-byte aligned");
        return MFD_ERR_INVALID;
    }
    attn::Params p;
    p.q = (const __nv_bfloat16*)q;
    p.sq_b = sq_b;
    p.sq_n = sq_n;
    p.sq_h = sq_h;
    p.k = (const __nv_bfloat16*)k;
    p.sk_b = sk_b;
    p.sk_h = sk_h;
    p.sk_s = sk_s;
    p.v = (const __nv_bfloat16*)v;
    p.sv_b = sv_b;
    p.sv_h = sv_h;
    p.sv_s = sv_s;
    p.prefix = prefix_lens;
    p.prefix_const = (int)prefix_len;
    p.anc = anc_bits;
    p.words = (int)anc_words;
    p.n = (int)n;
    p.H = (int)num_heads;
    p.Hkv = (int)num_kv_heads;
    p.G = (int)(num_heads / num_kv_heads);
    p.scale_log2 = scale * 1.4426950408889634f;
    p.splits = (int)splits;
    p.bs = (int)bs;
    const size_t rows = (size_t)splits * bs * num_heads * n;
    char* ws = (char*)(((uintptr_t)workspace + 255) & ~(uintptr_t)255);
    p.o_part = (float*)ws;
    p.lse_part = (float*)(ws + rows * attn::D * sizeof(float));
    p.out = (__nv_bfloat16*)out;
    p.so_b = so_b;
    p.so_n = so_n;
    p.so_h = so_h;
    const int nrows = (int)(n * p.G);
    dim3 grid((nrows + attn::kRows - 1) / attn::kRows, (unsigned)(bs * num_kv_heads), (unsigned)splits);
    const size_t smem = sizeof(attn::Smem);
    cudaError_t e = cudaFuncSetAttribute(attn::tree_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) {
        set_error("mfd_tree_attention: %s", cudaGetErrorString(e));
        return MFD_ERR_CUDA;
    }
    attn::tree_attn_kernel<<<grid, attn::kThreads, smem, (cudaStream_t)stream>>>(p);
    MFD_CHECK_LAUNCH("mfd_tree_attention");
    const int64_t warps = bs * num_kv_heads * nrows;
    attn::tree_attn_merge_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(p);
    MFD_CHECK_LAUNCH("mfd_tree_attention(merge)");
    return MFD_OK;
}
