// tree_prep.cu -- the input side of a Gated-DeltaNet layer over a draft tree: the short causal convolution of each
// node through its parent-pointer window, SiLU, and the l2 normalisation (and q scale) of q and k.
#include "common.cuh"

namespace gdn_prep {

constexpr int kMaxDk = 128;

// ---------------------------------------------------------------------------------------------- tree_prep
// Short causal convolution over each node's window (gathered through parent pointers; window entries below KC
// are the cached conv inputs), SiLU rounded to bf16, then l2 normalisation (and the q scale) per head of q and k,
// as inference/hf/tree_gdn_kernel.py:27-56 (_tree_prep) and 135-150 (tree_prep).  One CTA per (kPrepNodes nodes,
// head group), one thread per channel of the head; head groups are q (HK), k (HK), v (H) in channel order.  The
// work is a short chain of dependent loads per node, so the nodes are spread over many small CTAs (configs[2]: 16
// nodes per CTA 26.6 us, 4: 13.6 us, 2: 10.3 us, 1: 12.4 us).
constexpr int kPrepNodes = 2;
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
    __shared__ float red[kMaxDk / 32][kPrepNodes];
    const int hg = blockIdx.y, d = threadIdx.x, warp = d >> 5, lane = d & 31;
    const int i0 = blockIdx.x * kPrepNodes;
    const bool live = d < p.D;
    const int ch = hg * p.D + (live ? d : 0);
    // every thread reads its nodes' window indices itself (the same words for the whole CTA: broadcast loads), and
    // every window load is independent and unconditional (absent entries read the first cached input and weigh 0)
    int idx[kPrepNodes][KC];
#pragma unroll
    for (int t = 0; t < kPrepNodes; ++t)
#pragma unroll
        for (int j = 0; j < KC; ++j) {
            const int i = i0 + t;
            int e = i < p.n ? __ldg(p.conv_index + (int64_t)i * KC + j) : -1;
            idx[t][j] = (e < 0 || e >= KC + p.n) ? -1 : e;  // not a window entry: contributes nothing
        }
    float w[KC];
#pragma unroll
    for (int j = 0; j < KC; ++j) w[j] = __bfloat162float(p.conv_w[(int64_t)ch * KC + j]);
    float xv[kPrepNodes][KC];
#pragma unroll
    for (int t = 0; t < kPrepNodes; ++t) {
#pragma unroll
        for (int j = 0; j < KC; ++j) {
            const int e = idx[t][j];
            const __nv_bfloat16* src = e < KC ? p.conv_state + (int64_t)ch * KC + (e < 0 ? 0 : e)
                                              : p.x + (int64_t)(e - KC) * p.cd + ch;
            xv[t][j] = e < 0 ? 0.f : __bfloat162float(*src);
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

}  // namespace gdn_prep

extern "C" int mfd_tree_prep(const void* x, const void* conv_state, const int32_t* conv_index, const void* conv_w,
                             int64_t n, int64_t conv_dim, int64_t kernel, int64_t num_k_heads, int64_t num_heads,
                             int64_t head_dim, float scale, void* q, void* k, void* v, void* stream) {
    using namespace gdn_prep;
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
