// gdn_commit.cu -- the commit step of the Gated-DeltaNet layers: every layer's recurrent state advances to the
// deepest accepted node a, and its causal-conv window becomes a's window.
//
// Reference: inference/hf/qwen35_tree.py:122-148 (commit):
//   S_a = e^{G_a} S0 + sum_{j on the accepted path} e^{G_a - G_j} k_j u_j^T   (134-137; value head h reads key head
//   h / (H / HK), the repeat_interleave of 132-133), written back in the state's dtype;
//   conv window of a: column t = cached column window[t] (< kernel) or node input x[window[t] - kernel] (140-146),
//   built before the buffer is overwritten.
// All GDN layers in one launch each (device arrays of per-layer base addresses).  The state update is HBM-bound:
// one read and one write of H x Dk x Dv per layer; the path terms come from shared memory.
#include "common.cuh"

namespace mfd {
namespace gcm {

constexpr int kThreads = 256;
constexpr int kRows = 16;      // state rows (of Dk) per CTA
constexpr int kMaxPath = 128;  // accepted nodes

struct Params {
    const uint64_t* states;  // [layers] -> [H, Dk, Dv] (float32 or bf16), in place
    const uint64_t* u;       // [layers] -> [n, H, Dv] float32
    const uint64_t* k;       // [layers] -> [n, HK, Dk] bf16
    const uint64_t* g;       // [layers] -> [n, H] float32 (cumulative decay G)
    const int64_t* path;     // [p]
    int p, n, H, HK, Dk, Dv;
};

// CTA = (head, 16 state rows, layer).  Load phase: wk[j][r] = e^{G_a - G_j} k_j[r] and u_j for the path nodes into
// shared memory.  Then each thread owns float4 chunks of state rows: per path node one broadcast wk and one 16-byte
// u load feed four FMAs; the state is read and written as coalesced float4 (or 4 x bf16).
template <bool BF16>
__global__ void __launch_bounds__(kThreads) state_commit_kernel(Params prm) {
    extern __shared__ __align__(16) float sh[];
    const int h = blockIdx.x, r0 = blockIdx.y * kRows, layer = blockIdx.z;
    const int p = prm.p, Dk = prm.Dk, Dv = prm.Dv, H = prm.H;
    const int hk = h / (H / prm.HK);
    const int rows = min(kRows, Dk - r0);
    float* wk = sh;                // [p][kRows]
    float* uu = wk + p * kRows;    // [p][Dv] (16-byte aligned: p * kRows is a multiple of 4)
    __shared__ float ea;
    const float* g = reinterpret_cast<const float*>(prm.g[layer]);
    const float* u = reinterpret_cast<const float*>(prm.u[layer]);
    const __nv_bfloat16* k = reinterpret_cast<const __nv_bfloat16*>(prm.k[layer]);
    const int64_t last = prm.path[p - 1];
    const float Ga = g[last * H + h];
    if (threadIdx.x == 0) ea = expf(Ga);
    for (int e = threadIdx.x; e < p * kRows; e += kThreads) {
        const int j = e / kRows, r = e % kRows;
        const int64_t node = prm.path[j];
        const float w = expf(Ga - g[node * H + h]);
        wk[e] = r < rows ? w * __bfloat162float(k[(node * prm.HK + hk) * (int64_t)Dk + r0 + r]) : 0.f;
    }
    const int nch = Dv >> 2;  // float4 chunks per row
    for (int e = threadIdx.x; e < p * nch; e += kThreads) {
        const int j = e / nch, cc = e % nch;
        reinterpret_cast<float4*>(uu)[e] = reinterpret_cast<const float4*>(u + (prm.path[j] * H + h) * (int64_t)Dv)[cc];
    }
    __syncthreads();
    unsigned char* sbase = reinterpret_cast<unsigned char*>(prm.states[layer]);
    for (int e = threadIdx.x; e < rows * nch; e += kThreads) {
        const int r = e / nch, cc = e % nch;
        const int64_t idx = ((int64_t)h * Dk + r0 + r) * Dv + 4 * cc;
        float a[4];
        if (BF16) {
            const uint2 v = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(sbase) + idx);
            a[0] = bf16lo(v.x);
            a[1] = bf16hi(v.x);
            a[2] = bf16lo(v.y);
            a[3] = bf16hi(v.y);
        } else {
            const float4 v = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(sbase) + idx);
            a[0] = v.x;
            a[1] = v.y;
            a[2] = v.z;
            a[3] = v.w;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) a[q] *= ea;
        for (int j = 0; j < p; ++j) {
            const float c = wk[j * kRows + r];
            const float4 uv = reinterpret_cast<const float4*>(uu)[j * nch + cc];
            a[0] = __fmaf_rn(c, uv.x, a[0]);
            a[1] = __fmaf_rn(c, uv.y, a[1]);
            a[2] = __fmaf_rn(c, uv.z, a[2]);
            a[3] = __fmaf_rn(c, uv.w, a[3]);
        }
        if (BF16) {
            uint2 v;
            __nv_bfloat162 lo = __floats2bfloat162_rn(a[0], a[1]), hi = __floats2bfloat162_rn(a[2], a[3]);
            v.x = *reinterpret_cast<uint32_t*>(&lo);
            v.y = *reinterpret_cast<uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(sbase) + idx) = v;
        } else {
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(sbase) + idx) = make_float4(a[0], a[1], a[2], a[3]);
        }
    }
}

// conv window: thread = (layer, channel); reads the whole window, then writes it (in place)
template <typename T>
__global__ void conv_commit_kernel(const uint64_t* conv, const uint64_t* x, const int32_t* window, int64_t layers,
                                   int64_t conv_dim, int kernel) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= layers * conv_dim) return;
    const int64_t layer = t / conv_dim, c = t % conv_dim;
    T* cs = reinterpret_cast<T*>(conv[layer]) + c * kernel;
    const T* xs = reinterpret_cast<const T*>(x[layer]);
    T vals[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (i >= kernel) break;
        const int wi = window[i];
        vals[i] = wi < kernel ? cs[wi] : xs[(int64_t)(wi - kernel) * conv_dim + c];
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (i >= kernel) break;
        cs[i] = vals[i];
    }
}

}  // namespace gcm
}  // namespace mfd

using namespace mfd;

extern "C" int mfd_gdn_commit(const uint64_t* states, int state_dtype, const uint64_t* u, const uint64_t* k,
                              const uint64_t* g_cum, int64_t layers, const int64_t* path, int64_t path_len, int64_t n,
                              int64_t num_heads, int64_t num_k_heads, int64_t dk, int64_t dv, void* stream) {
    if (layers < 0 || path_len < 1 || path_len > gcm::kMaxPath || n < 1 || num_heads < 1 || num_k_heads < 1 ||
        num_heads % num_k_heads || dk < 1 || dv < 4 || dv > 256 || dv % 4 || dk > 65535 * gcm::kRows) {
        set_error("mfd_gdn_commit: invalid sizes layers=%lld path=%lld (1..%d) n=%lld H=%lld HK=%lld Dk=%lld "
                  "Dv=%lld (a multiple of 4, <= 256)",
                  (long long)layers, (long long)path_len, gcm::kMaxPath, (long long)n, (long long)num_heads,
                  (long long)num_k_heads, (long long)dk, (long long)dv);
        return MFD_ERR_INVALID;
    }
    if (state_dtype != MFD_F32 && state_dtype != MFD_BF16) {
        set_error("mfd_gdn_commit: state_dtype must be MFD_F32 or MFD_BF16");
        return MFD_ERR_INVALID;
    }
    if (layers == 0) return MFD_OK;
    if (!states || !u || !k || !g_cum || !path) {
        set_error("mfd_gdn_commit: null pointer");
        return MFD_ERR_INVALID;
    }
    if (layers > 65535 || num_heads > 0x7fffffffLL) {
        set_error("mfd_gdn_commit: too many layers or heads");
        return MFD_ERR_UNSUPPORTED;
    }
    gcm::Params p{states, u, k, g_cum, path, (int)path_len, (int)n, (int)num_heads, (int)num_k_heads, (int)dk,
                  (int)dv};
    const size_t smem = sizeof(float) * (size_t)(path_len * gcm::kRows + path_len * dv);
    dim3 grid((unsigned)num_heads, (unsigned)((dk + gcm::kRows - 1) / gcm::kRows), (unsigned)layers);
    cudaError_t e;
    if (state_dtype == MFD_BF16) {
        e = cudaFuncSetAttribute(gcm::state_commit_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
        if (e == cudaSuccess) gcm::state_commit_kernel<true><<<grid, gcm::kThreads, smem, (cudaStream_t)stream>>>(p);
    } else {
        e = cudaFuncSetAttribute(gcm::state_commit_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
        if (e == cudaSuccess) gcm::state_commit_kernel<false><<<grid, gcm::kThreads, smem, (cudaStream_t)stream>>>(p);
    }
    if (e != cudaSuccess) {
        set_error("mfd_gdn_commit: %s", cudaGetErrorString(e));
        return MFD_ERR_CUDA;
    }
    MFD_CHECK_LAUNCH("mfd_gdn_commit");
    return MFD_OK;
}

extern "C" int mfd_conv_commit(const uint64_t* conv_states, const uint64_t* x, int64_t elem_bytes, int64_t layers,
                               int64_t conv_dim, int64_t kernel, const int32_t* window, void* stream) {
    if (layers < 0 || conv_dim < 0 || kernel < 1 || kernel > 8 || (elem_bytes != 2 && elem_bytes != 4)) {
        set_error("mfd_conv_commit: invalid sizes layers=%lld conv_dim=%lld kernel=%lld (1..8) elem_bytes=%lld",
                  (long long)layers, (long long)conv_dim, (long long)kernel, (long long)elem_bytes);
        return MFD_ERR_INVALID;
    }
    if (layers == 0 || conv_dim == 0) return MFD_OK;
    if (!conv_states || !x || !window) {
        set_error("mfd_conv_commit: null pointer");
        return MFD_ERR_INVALID;
    }
    const int64_t total = layers * conv_dim;
    const unsigned blocks = (unsigned)((total + 255) / 256);
    if (elem_bytes == 2)
        gcm::conv_commit_kernel<uint16_t><<<blocks, 256, 0, (cudaStream_t)stream>>>(conv_states, x, window, layers,
                                                                                    conv_dim, (int)kernel);
    else
        gcm::conv_commit_kernel<uint32_t><<<blocks, 256, 0, (cudaStream_t)stream>>>(conv_states, x, window, layers,
                                                                                    conv_dim, (int)kernel);
    MFD_CHECK_LAUNCH("mfd_conv_commit");
    return MFD_OK;
}
