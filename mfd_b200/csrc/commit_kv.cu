// commit_kv.cu -- the commit step's KV moves: after acceptance, the K/V rows of the accepted tree nodes move into
// the positions the committed sequence occupies, in every attention layer's key and value buffer.
//
// SGLang (sglang-v0.5.22-mfd.patch:1769-1841, DDTreeKVCompactor / _ddtree_compact_kv_kernel): a token-major pool,
//   one slot per token and buffer; request b moves slot move_src[b, i] -> move_tgt[b, i] for every i whose source
//   and target differ (the no-ops of the move list, including the lanes past the path, are skipped), every source
//   read before any store, since a path slot can be another move's target.
// HF (inference/hf/ddtree.py:33-61 compact_tail_inplace, 385-403 _compact_appended_window, 406-436
//   compact_dynamic_cache): a cache tensor [..., S, D] whose rows [past, S) were appended for the tree; row
//   past + keep[i] moves to past + i for every outer index (batch x heads), nothing when keep is empty or keeps the
//   whole window (the reference returns early in both cases).
//
// One kernel serves both: a CTA owns one (group, buffer, tile of the slot) -- group = request (SGLang) or outer row
// block (HF) -- stages the tile of every moving source slot in shared memory, synchronizes, then stores, so each
// move reads the old contents whatever the other moves write.  Every buffer of a call (all layers' K and V) goes
// into one launch through a device array of base addresses.  HBM-bound: each moved row is read once and written
// once.
#include "common.cuh"

namespace mfd {
namespace ckv {

constexpr int kThreads = 128;
constexpr int kSmemCap = 96 * 1024;  // staging bytes per CTA (moves x tile)
constexpr int kMaxMoves = 1024;      // move-list width

struct Params {
    const uint64_t* bufs;    // [nbufs] base addresses
    int64_t group_stride;    // bytes between groups within a buffer (0: the slots are absolute)
    int64_t slot_stride;     // bytes between consecutive slots / rows
    int64_t slot_units;      // units per slot (unit = 16 or 8 bytes)
    const int64_t* src;      // [groups, L] (list_stride = L) or [L] (list_stride = 0); null: HF keep form
    const int64_t* tgt;
    const int64_t* keep;     // HF: rows past + keep[i] -> past + i
    int64_t past;
    int64_t rows;            // rows per group (HF) or slots of the pool (SGLang): bounds check; 0: unchecked
    int64_t list_stride;
    int L;
    int tile_units;          // units per CTA tile
    int* status;             // optional: MFD_ERR_INVALID when a row index / slot id is out of range
};

template <typename U>
__global__ void __launch_bounds__(kThreads) moves_kernel(Params p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    U* stage = reinterpret_cast<U*>(smem_raw);  // [L][tile_units]
    __shared__ int64_t mv_s[kMaxMoves], mv_t[kMaxMoves];  // the group's effective moves
    __shared__ int n_moves;
    const int64_t g = blockIdx.x;
    const int buf = blockIdx.y;
    const int64_t u0 = (int64_t)blockIdx.z * p.tile_units;
    const int64_t nu = min((int64_t)p.tile_units, p.slot_units - u0);
    unsigned char* base = reinterpret_cast<unsigned char*>(p.bufs[buf]) + g * p.group_stride;
    // the move list, read once in parallel and compacted to the moves that change a slot
    if (threadIdx.x == 0) n_moves = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < p.L; i += kThreads) {
        int64_t s, t;
        bool ok;
        if (p.keep) {
            const int64_t kp = p.keep[i];
            s = p.past + kp;
            t = p.past + i;
            ok = !(p.rows > 0 && (kp < 0 || s >= p.rows));
            if (!ok && p.status) atomicExch(p.status, (int)MFD_ERR_INVALID);
        } else {
            s = p.src[g * p.list_stride + i];
            t = p.tgt[g * p.list_stride + i];
            // a slot id beyond the pool is skipped and flagged, never dereferenced
            ok = !(p.rows > 0 && s != t && (s >= p.rows || t >= p.rows));
            if (!ok && p.status) atomicExch(p.status, (int)MFD_ERR_INVALID);
        }
        if (ok && s != t && s >= 0 && t >= 0) {
            const int slot = atomicAdd(&n_moves, 1);  // order within the list does not matter: sources are staged
            mv_s[slot] = s;
            mv_t[slot] = t;
        }
    }
    __syncthreads();
    const int nm = n_moves;
    // every source of the tile into shared memory (all loads of a thread issued before it waits on any), then
    // every target
    for (int64_t e = threadIdx.x; e < (int64_t)nm * nu; e += kThreads) {
        const int i = (int)(e / nu);
        const int64_t v = e - (int64_t)i * nu;
        stage[(size_t)i * p.tile_units + v] = reinterpret_cast<const U*>(base + mv_s[i] * p.slot_stride)[u0 + v];
    }
    __syncthreads();
    for (int64_t e = threadIdx.x; e < (int64_t)nm * nu; e += kThreads) {
        const int i = (int)(e / nu);
        const int64_t v = e - (int64_t)i * nu;
        reinterpret_cast<U*>(base + mv_t[i] * p.slot_stride)[u0 + v] = stage[(size_t)i * p.tile_units + v];
    }
}

static int launch(Params p, int64_t groups, int64_t nbufs, int64_t slot_bytes, bool aligned16, cudaStream_t stream,
                  const char* fn) {
    const int unit = aligned16 ? 16 : 8;
    p.slot_units = slot_bytes / unit;
    int64_t tile = kSmemCap / ((int64_t)max(p.L, 1) * unit);
    tile = min(tile, p.slot_units);
    tile = max(tile, (int64_t)1);
    p.tile_units = (int)tile;
    const int64_t tiles = (p.slot_units + tile - 1) / tile;
    if (groups > 0x7fffffffLL || nbufs > 65535 || tiles > 65535) {
        set_error("%s: grid too large (groups %lld, buffers %lld, tiles %lld)", fn, (long long)groups,
                  (long long)nbufs, (long long)tiles);
        return MFD_ERR_UNSUPPORTED;
    }
    const size_t smem = (size_t)p.L * tile * unit;
    dim3 grid((unsigned)groups, (unsigned)nbufs, (unsigned)tiles);
    // the staging buffer plus the static move lists can pass the 48 KB default: opt in (per device, cheap)
    cudaError_t e = aligned16
                        ? cudaFuncSetAttribute(moves_kernel<uint4>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap)
                        : cudaFuncSetAttribute(moves_kernel<uint2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap);
    if (e != cudaSuccess) {
        set_error("%s: cannot raise the shared-memory limit: %s", fn, cudaGetErrorString(e));
        return MFD_ERR_CUDA;
    }
    if (aligned16)
        moves_kernel<uint4><<<grid, kThreads, smem, stream>>>(p);
    else
        moves_kernel<uint2><<<grid, kThreads, smem, stream>>>(p);
    MFD_CHECK_LAUNCH(fn);
    return MFD_OK;
}

}  // namespace ckv
}  // namespace mfd

using namespace mfd;

extern "C" int mfd_commit_kv_moves(const uint64_t* buffers, int64_t num_buffers, int64_t slot_bytes,
                                   int64_t base_align, const int64_t* move_src, const int64_t* move_tgt, int64_t bs,
                                   int64_t width, int64_t pool_slots, int* status, void* stream) {
    if (bs < 0 || width < 0 || num_buffers < 0 || slot_bytes <= 0 || slot_bytes % 8 || width > ckv::kMaxMoves ||
        base_align <= 0 || base_align % 8 || pool_slots < 0) {
        set_error("mfd_commit_kv_moves: invalid sizes bs=%lld width=%lld buffers=%lld slot_bytes=%lld base_align=%lld "
                  "pool_slots=%lld (slot_bytes and base_align multiples of 8, width <= 1024)",
                  (long long)bs, (long long)width, (long long)num_buffers, (long long)slot_bytes,
                  (long long)base_align, (long long)pool_slots);
        return MFD_ERR_INVALID;
    }
    if (bs == 0 || width == 0 || num_buffers == 0) return MFD_OK;
    if (!buffers || !move_src || !move_tgt) {
        set_error("mfd_commit_kv_moves: null pointer");
        return MFD_ERR_INVALID;
    }
    ckv::Params p{};
    p.bufs = buffers;
    p.group_stride = 0;
    p.slot_stride = slot_bytes;
    p.src = move_src;
    p.tgt = move_tgt;
    p.list_stride = width;
    p.L = (int)width;
    p.rows = pool_slots;
    p.status = status;
    // 16-byte units need 16-byte slots and 16-byte aligned buffer bases
    return ckv::launch(p, bs, num_buffers, slot_bytes, slot_bytes % 16 == 0 && base_align % 16 == 0,
                       (cudaStream_t)stream, "mfd_commit_kv_moves");
}

extern "C" int mfd_compact_tail(const uint64_t* buffers, int64_t num_buffers, int64_t outer, int64_t outer_stride,
                                int64_t rows, int64_t row_stride, int64_t row_bytes, int64_t base_align,
                                int64_t past_length, const int64_t* keep, int64_t keep_count, int* status,
                                void* stream) {
    if (num_buffers < 0 || outer < 0 || rows < 0 || past_length < 0 || past_length > rows || keep_count < 0 ||
        row_bytes <= 0 || row_bytes % 8 || row_stride % 8 || outer_stride % 8 || keep_count > ckv::kMaxMoves ||
        base_align <= 0 || base_align % 8) {
        set_error("mfd_compact_tail: invalid sizes (buffers %lld, outer %lld, rows %lld, past %lld, keep %lld, row "
                  "bytes %lld)",
                  (long long)num_buffers, (long long)outer, (long long)rows, (long long)past_length,
                  (long long)keep_count, (long long)row_bytes);
        return MFD_ERR_INVALID;
    }
    const int64_t current = rows - past_length;
    if (keep_count > current) {
        set_error("mfd_compact_tail: keep_count %lld exceeds the appended window %lld", (long long)keep_count,
                  (long long)current);
        return MFD_ERR_INVALID;
    }
    // the reference returns early for an empty window, an empty keep list, or one keeping the whole window
    if (current <= 0 || keep_count == 0 || keep_count == current || num_buffers == 0 || outer == 0) return MFD_OK;
    if (!buffers || !keep) {
        set_error("mfd_compact_tail: null pointer");
        return MFD_ERR_INVALID;
    }
    ckv::Params p{};
    p.bufs = buffers;
    p.group_stride = outer_stride;
    p.slot_stride = row_stride;
    p.keep = keep;
    p.past = past_length;
    p.rows = rows;
    p.L = (int)keep_count;
    p.status = status;
    const bool a16 = row_bytes % 16 == 0 && row_stride % 16 == 0 && outer_stride % 16 == 0 && base_align % 16 == 0;
    return ckv::launch(p, outer, num_buffers, row_bytes, a16, (cudaStream_t)stream, "mfd_compact_tail");
}
