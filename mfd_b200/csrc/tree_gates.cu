// tree_gates.cu -- the gates of a Gated-DeltaNet layer over a draft tree, in one launch.
//
// Per node i and value head h, from the layer's projections a = in_proj_a(h), b = in_proj_b(h) and its
// parameters A_log, dt_bias:
//   beta[i, h] = sigmoid(b[i, h])
//   g[i, h]    = -exp(A_log[h]) * softplus(a[i, h] + dt_bias[h])          (the per-token log decay)
//   G[i, h]    = sum of g[j, h] over j on the root path of i, i included    (the log decay along the path)
// which is inference/hf/qwen35_tree.py:77-79 (beta, g, then G = anc_f @ g).  Here G is summed along the parent
// pointers (node first, then its ancestors) instead of as a dense [n, n] x [n, H] product: a path has one node per
// depth.  One CTA per value head: g of every node into shared memory, then each thread walks its nodes' paths.
// softplus follows torch's default (x for x > 20, else log1p(exp(x))).
#include "common.cuh"

namespace mfd {
namespace gates {

constexpr int kThreads = 256;
constexpr int kMaxNodes = 2048;

struct Params {
    const void* a;  // [n, H] rows of stride sa (elements); bf16 or fp32
    const void* b;  // [n, H] rows of stride sb
    int64_t sa, sb;
    int ab_bf16;
    const float* a_log;    // [H]
    const float* dt_bias;  // [H]
    const int64_t* parents;  // [n]; parents[i] < i, or -1 for a root
    int n, H;
    float* beta;  // [n, H]
    float* G;     // [n, H]
    int* status;  // optional: MFD_ERR_INVALID when a parent index is not an earlier node
};

__device__ __forceinline__ float load_val(const void* p, int64_t idx, int bf16) {
    return bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[idx]) : reinterpret_cast<const float*>(p)[idx];
}

__global__ void __launch_bounds__(kThreads) tree_gates_kernel(Params p) {
    __shared__ float g_s[kMaxNodes];
    __shared__ int par_s[kMaxNodes];
    const int h = blockIdx.x;
    const float decay = -expf(p.a_log[h]);
    const float bias = p.dt_bias[h];
    for (int i = threadIdx.x; i < p.n; i += kThreads) {
        const float x = load_val(p.a, (int64_t)i * p.sa + h, p.ab_bf16) + bias;
        const float sp = x > 20.f ? x : log1pf(expf(x));
        g_s[i] = decay * sp;
        const float bb = load_val(p.b, (int64_t)i * p.sb + h, p.ab_bf16);
        p.beta[(int64_t)i * p.H + h] = 1.f / (1.f + expf(-bb));
        int64_t par = p.parents[i];
        if (par >= i || par < -1) {  // not a topologically ordered tree: treat as a root and report it
            if (p.status) atomicExch(p.status, (int)MFD_ERR_INVALID);
            par = -1;
        }
        par_s[i] = (int)par;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < p.n; i += kThreads) {
        float acc = g_s[i];
        for (int j = par_s[i]; j >= 0; j = par_s[j]) acc += g_s[j];  // parents strictly decrease: at most i steps
        p.G[(int64_t)i * p.H + h] = acc;
    }
}

}  // namespace gates
}  // namespace mfd

using namespace mfd;

extern "C" int mfd_tree_gates(const void* a, int64_t sa, const void* b, int64_t sb, int ab_dtype, const float* a_log,
                              const float* dt_bias, const int64_t* parents, int64_t n, int64_t num_heads, float* beta,
                              float* G, int* status, void* stream) {
    if (n < 0 || num_heads < 1 || n > gates::kMaxNodes || sa < num_heads || sb < num_heads ||
        (ab_dtype != MFD_F32 && ab_dtype != MFD_BF16)) {
        set_error("mfd_tree_gates: invalid sizes n=%lld H=%lld (n <= %d) or dtype %d", (long long)n,
                  (long long)num_heads, gates::kMaxNodes, ab_dtype);
        return MFD_ERR_INVALID;
    }
    if (n == 0) return MFD_OK;
    if (!a || !b || !a_log || !dt_bias || !parents || !beta || !G) {
        set_error("mfd_tree_gates: null pointer");
        return MFD_ERR_INVALID;
    }
    gates::Params p;
    p.a = a;
    p.b = b;
    p.sa = sa;
    p.sb = sb;
    p.ab_bf16 = ab_dtype == MFD_BF16;
    p.a_log = a_log;
    p.dt_bias = dt_bias;
    p.parents = parents;
    p.n = (int)n;
    p.H = (int)num_heads;
    p.beta = beta;
    p.G = G;
    p.status = status;
    gates::tree_gates_kernel<<<(unsigned)num_heads, gates::kThreads, 0, (cudaStream_t)stream>>>(p);
    MFD_CHECK_LAUNCH("mfd_tree_gates");
    return MFD_OK;
}
