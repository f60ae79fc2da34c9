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

// ------------------------------------------------------------------------------------------------ HF compile
// The HF verify inputs of one tree (inference/hf/ddtree.py:317-357, compile_ddtree_tree) written straight from the
// device tree: the verify ids and positions, the tree's block of the additive mask and the bool visibility.  The
// reference first resets the previous round's block to 0 and then writes the new block; the two can overlap (the
// new prefix starts inside the old block), so each element takes the new block's value when it lies in the new
// block and 0 when it lies only in the old one, whatever order the threads run in.
namespace mfd {
namespace cmp {

struct Params {
    const int64_t* root;
    const int64_t* tokens;  // [n] (tokens[0], the root slot, unused)
    const int64_t* depths;  // [n] (depths[0] = 0)
    const uint8_t* vis;     // [n, vis_stride]: nonzero = column visible
    int64_t vis_stride;
    int64_t n, start, past, prev_start, prev_len;
    int64_t* ids;
    int64_t* pos;
    unsigned char* mask;
    int64_t mask_row_bytes;  // row stride in bytes
    int elem;                // 2 or 4
    uint32_t min_bits;
    bool* vis_out;
    int64_t vis_out_stride;
    int64_t c_lo, c_hi;      // columns touched: the union of the two blocks
};

__global__ void compile_tree_kernel(Params p) {
    const int64_t i = blockIdx.x;
    unsigned char* row = p.mask + i * p.mask_row_bytes;
    const bool in_new_row = i < p.n, in_old_row = i < p.prev_len;
    for (int64_t c = p.c_lo + threadIdx.x; c < p.c_hi; c += blockDim.x) {
        const bool in_new = in_new_row && c >= p.past && c < p.past + p.n;
        const bool in_old = in_old_row && c >= p.prev_start && c < p.prev_start + p.prev_len;
        if (!in_new && !in_old) continue;
        const uint32_t bits = in_new && !p.vis[i * p.vis_stride + (c - p.past)] ? p.min_bits : 0u;
        if (p.elem == 2)
            reinterpret_cast<uint16_t*>(row)[c] = (uint16_t)bits;
        else
            reinterpret_cast<uint32_t*>(row)[c] = bits;
    }
    if (!in_new_row) return;
    for (int64_t j = threadIdx.x; j < p.n; j += blockDim.x) p.vis_out[i * p.vis_out_stride + j] = p.vis[i * p.vis_stride + j] != 0;
    if (threadIdx.x == 0) {
        p.ids[i] = i == 0 ? *p.root : p.tokens[i];
        p.pos[i] = p.start + (i == 0 ? 0 : p.depths[i]);
    }
}

}  // namespace cmp
}  // namespace mfd

extern "C" int mfd_compile_tree(const int64_t* root_token, const int64_t* tokens, const int64_t* depths, int64_t n,
                                const uint8_t* vis, int64_t vis_stride, int64_t start, int64_t past_length,
                                int64_t prev_start, int64_t prev_length, int64_t* ids_out, int64_t* positions_out,
                                void* mask, int64_t mask_elem_bytes, int64_t mask_row_stride, int64_t mask_rows,
                                int64_t mask_cols, uint32_t min_bits, bool* vis_out, int64_t vis_out_stride,
                                void* stream) {
    if (n < 1 || vis_stride < n || past_length < 0 || prev_start < 0 || prev_length < 0 ||
        (mask_elem_bytes != 2 && mask_elem_bytes != 4) || mask_row_stride < mask_cols || vis_out_stride < n) {
        set_error("mfd_compile_tree: invalid sizes n=%lld past=%lld prev=(%lld, %lld) elem=%lld", (long long)n,
                  (long long)past_length, (long long)prev_start, (long long)prev_length, (long long)mask_elem_bytes);
        return MFD_ERR_INVALID;
    }
    if (n > mask_rows || past_length + n > mask_cols || prev_length > mask_rows ||
        prev_start + prev_length > mask_cols) {
        set_error("mfd_compile_tree: the tree block [%lld rows, columns %lld + %lld] or the previous one [%lld, %lld + "
                  "%lld] lies outside the %lld x %lld mask", (long long)n, (long long)past_length, (long long)n,
                  (long long)prev_length, (long long)prev_start, (long long)prev_length, (long long)mask_rows,
                  (long long)mask_cols);
        return MFD_ERR_INVALID;
    }
    if (!root_token || !tokens || !depths || !vis || !ids_out || !positions_out || !mask || !vis_out) {
        set_error("mfd_compile_tree: null pointer");
        return MFD_ERR_INVALID;
    }
    cmp::Params p;
    p.root = root_token;
    p.tokens = tokens;
    p.depths = depths;
    p.vis = vis;
    p.vis_stride = vis_stride;
    p.n = n;
    p.start = start;
    p.past = past_length;
    p.prev_start = prev_start;
    p.prev_len = prev_length;
    p.ids = ids_out;
    p.pos = positions_out;
    p.mask = (unsigned char*)mask;
    p.mask_row_bytes = mask_row_stride * mask_elem_bytes;
    p.elem = (int)mask_elem_bytes;
    p.min_bits = min_bits;
    p.vis_out = vis_out;
    p.vis_out_stride = vis_out_stride;
    p.c_lo = prev_length > 0 ? (past_length < prev_start ? past_length : prev_start) : past_length;
    const int64_t new_hi = past_length + n, old_hi = prev_start + prev_length;
    p.c_hi = prev_length > 0 && old_hi > new_hi ? old_hi : new_hi;
    const int64_t rows = n > prev_length ? n : prev_length;
    cmp::compile_tree_kernel<<<(unsigned)rows, 128, 0, (cudaStream_t)stream>>>(p);
    MFD_CHECK_LAUNCH("mfd_compile_tree");
    return MFD_OK;
}
