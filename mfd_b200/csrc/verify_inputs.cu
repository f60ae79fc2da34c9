// verify_inputs.cu -- per (request, node): the verify token id, its position and its row of the flat
// int8 tree mask [W, prefix + W] (prefix fully visible, then the node's ancestors and itself).
// Reference: SGLang _ddtree_verify_inputs_kernel / ddtree_verify_inputs (sglang-v0.5.22-mfd.patch:1625-1703),
// including its bounded ancestor walk (max_depth + 1 steps) and root token at node 0.
#include "common.cuh"

namespace mfd {
namespace vin {

struct Params {
    const int64_t* root;      // [bs]
    const int64_t* prefix;    // [bs]
    const int64_t* tokens;    // [bs, *] stride tree_stride
    const int64_t* depths;
    const int64_t* parents;
    int64_t tree_stride;
    const int64_t* mask_off;  // [bs]
    int64_t* ids_out;         // [bs, W]
    int64_t* pos_out;         // [bs, W]
    int8_t* mask;
    int64_t W;
    int max_depth;
};

__global__ void verify_inputs_kernel(Params p) {
    const int64_t b = blockIdx.y, i = blockIdx.x;
    const int64_t prefix = p.prefix[b];
    const int64_t row_len = prefix + p.W;
    int8_t* row = p.mask + p.mask_off[b] + i * row_len;
    for (int64_t c = threadIdx.x; c < prefix; c += blockDim.x) row[c] = 1;
    const int64_t* par = p.parents + b * p.tree_stride;
    for (int64_t c = threadIdx.x; c < p.W; c += blockDim.x) {
        // is column c on node i's bounded ancestor walk?
        int64_t anc = i;
        bool vis = false;
        for (int s = 0; s <= p.max_depth; ++s) {
            if (anc == c && anc >= 0) vis = true;
            const int64_t nxt = par[anc > 0 ? anc : 0];
            anc = anc > 0 ? nxt : -1;
        }
        row[prefix + c] = vis ? 1 : 0;
    }
    if (threadIdx.x == 0) {
        const int64_t tok = p.tokens[b * p.tree_stride + i];
        p.ids_out[b * p.W + i] = i == 0 ? p.root[b] : tok;
        p.pos_out[b * p.W + i] = prefix + p.depths[b * p.tree_stride + i];
    }
}

}  // namespace vin
}  // namespace mfd

using namespace mfd;

extern "C" int mfd_verify_inputs(const int64_t* root_tokens, const int64_t* prefix_lens, const int64_t* tokens,
                                 const int64_t* depths, const int64_t* parents, int64_t tree_stride,
                                 const int64_t* mask_offsets, int64_t bs, int64_t width, int64_t max_depth,
                                 int64_t* ids_out, int64_t* positions_out, int8_t* mask_out, void* stream) {
    if (bs < 0 || width < 1 || max_depth < 0 || tree_stride < width) {
        set_error("mfd_verify_inputs: invalid sizes bs=%lld W=%lld max_depth=%lld", (long long)bs, (long long)width,
                  (long long)max_depth);
        return MFD_ERR_INVALID;
    }
    if (bs == 0) return MFD_OK;
    if (!root_tokens || !prefix_lens || !tokens || !depths || !parents || !mask_offsets || !ids_out ||
        !positions_out || !mask_out) {
        set_error("mfd_verify_inputs: null pointer");
        return MFD_ERR_INVALID;
    }
    vin::Params p;
    p.root = root_tokens;
    p.prefix = prefix_lens;
    p.tokens = tokens;
    p.depths = depths;
    p.parents = parents;
    p.tree_stride = tree_stride;
    p.mask_off = mask_offsets;
    p.ids_out = ids_out;
    p.pos_out = positions_out;
    p.mask = mask_out;
    p.W = width;
    p.max_depth = (int)max_depth;
    dim3 grid((unsigned)width, (unsigned)bs);
    vin::verify_inputs_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(p);
    MFD_CHECK_LAUNCH("mfd_verify_inputs");
    return MFD_OK;
}
