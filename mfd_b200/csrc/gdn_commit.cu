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

template <bool BF16>
__global__ void __launch_bounds__(kThreads) state_commit_kernel(Params prm) {
    extern __shared__ __align__(16) float sh[];
    const int h = blockIdx.x, r0 = blockIdx.y * kRows, layer = blockIdx.z;
    const int p = prm.p, Dk = prm.Dk, Dv = prm.Dv, H = prm.H;
    const int hk = h / (H / prm.HK);
    const int rows = min(kRows, Dk - r0);
    const int pp = (p + 3) & ~3;
    float* w = sh;              // [p]: e^{G_a - G_j}
    float* kk = w + pp;         // [p][kRows]
    float* uu = kk + pp * kRows;  // [p][Dv]
    __shared__ float ea;
    const float* g = reinterpret_cast<const float*>(prm.g[layer]);
    const float* u = reinterpret_cast<const float*>(prm.u[layer]);
    const __nv_bfloat16* k = reinterpret_cast<const __nv_bfloat16*>(prm.k[layer]);
    const int64_t last = prm.path[p - 1];
    const float Ga = g[last * H + h];
    if (threadIdx.x == 0) ea = expf(Ga);
    for (int j = threadIdx.x; j < p; j += kThreads) w[j] = expf(Ga - g[prm.path[j] * H + h]);
    for (int e = threadIdx.x; e < p * kRows; e += kThreads) {
        const int j = e / kRows, r = e % kRows;
        kk[e] = r < rows ? __bfloat162float(k[(prm.path[j] * prm.HK + hk) * (int64_t)Dk + r0 + r]) : 0.f;
    }
    for (int e = threadIdx.x; e < p * Dv; e += kThreads) {
        const int j = e / Dv, c = e % Dv;
        uu[e] = u[(prm.path[j] * H + h) * (int64_t)Dv + c];
    }
    __syncthreads();
    unsigned char* sbase = reinterpret_cast<unsigned char*>(prm.states[layer]);
    for (int e = threadIdx.x; e < rows * Dv; e += kThreads) {
        const int r = e / Dv, c = e % Dv;
        const int64_t idx = ((int64_t)h * Dk + r0 + r) * Dv + c;
        float s0;
        if (BF16) s0 = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(sbase)[idx]);
        else s0 = reinterpret_cast<const float*>(sbase)[idx];
        float acc = ea * s0;
        for (int j = 0; j < p; ++j) acc = __fmaf_rn(w[j] * kk[j * kRows + r], uu[j * Dv + c], acc);
        if (BF16) reinterpret_cast<__nv_bfloat16*>(sbase)[idx] = __float2bfloat16_rn(acc);
        else reinterpret_cast<float*>(sbase)[idx] = acc;
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
        num_heads % num_k_heads || dk < 1 || dv < 1 || dv > 256 || dk > 65535 * gcm::kRows) {
        set_error("mfd_gdn_commit: invalid sizes layers=%lld path=%lld (1..%d) n=%lld H=%lld HK=%lld Dk=%lld "
                  "Dv=%lld (<= 256)",
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
    const int64_t pp = (path_len + 3) & ~3LL;
    const size_t smem = sizeof(float) * (size_t)(pp + pp * gcm::kRows + path_len * dv);
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
