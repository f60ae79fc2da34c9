// tree_attention_tc.cuh -- parameters shared by the tcgen05 attention kernel (tree_attention_tc.cu) and its C ABI
// (tree_attention.cu): the dense verify / mode attention and the paged mode attention.
#pragma once

#include <stdint.h>

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace mfd {
namespace tca {

constexpr int kM = 128;  // rows per CTA (one M-tile)

struct Params {
    __nv_bfloat16* out;  // [bs, n, H, D] with strides so_b, so_n, so_h
    int64_t so_b, so_n, so_h;
    const int32_t* prefix;  // [bs] prefix lengths (device) or null (dense mode)
    int prefix_const;
    const uint64_t* anc;    // ancestor-or-self bitsets [bs, n, words] (paged mode: [n, words], shared by all requests)
    int words;
    int n, H, Hkv, G;
    int mtiles;        // M-tiles per (request, KV head) = ceil(n G / 128)
    float scale_log2;  // scale * log2(e)
    int splits;
    float* o_part;          // [splits, bs, Hkv, mtiles * 128, D]
    float* lse_part;        // [splits, bs, Hkv, mtiles * 128]
    unsigned int* tickets;  // [bs, Hkv, mtiles] in a ticket-only buffer, zero between launches
    int* status;            // sticky: 1 once a bounded wait gave up
    int bs;
    // paged mode: the context keys of request b are the cache rows r2t[rpi[b] * r2t_stride + j] for
    // j < ctx[b] (clamped to [0, r2t_cols]); its n block keys are rows b * n + j of k_new / v_new, gathered by the
    // kernel itself (the K / V tensor maps are not used)
    int paged;
    const int32_t* r2t;
    int64_t r2t_stride, r2t_rows, r2t_cols;
    const int64_t* rpi;
    const int64_t* ctx;
    const __nv_bfloat16* kc;  // caches [slots, Hkv, 128], token stride skc_t (K and V alike)
    const __nv_bfloat16* vc;
    const __nv_bfloat16* kn;  // this step's block keys / values [bs n, Hkv, 128], token stride skn_t (K and V alike)
    const __nv_bfloat16* vn;
    int64_t skc_t, skn_t;
    int64_t slots;  // cache rows: slot ids from req_to_token are clamped to [0, slots)
};

struct Shape {
    const void* q;
    int64_t sq_b, sq_n, sq_h;
    // dense: k, v [bs, Hkv, max_keys, 128] (paged mode: unused)
    const void* k;
    int64_t sk_b, sk_h, sk_s;
    const void* v;
    int64_t sv_b, sv_h, sv_s;
    int64_t max_keys;  // dense: stored keys
};

int launch(const Shape& sh, const Params& p, cudaStream_t stream);

}  // namespace tca
}  // namespace mfd
