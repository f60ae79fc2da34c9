// topk_logz_static.cu -- the logits step without any caller-provided or library-allocated scratch.
//
// Some callers cannot allocate device memory when they call into this library: a host that owns every byte of
// the GPU through its own pool and forbids outside allocations, code on a latency-critical serving path where
// cudaMalloc (which may synchronise the device) is not acceptable, or plugins whose interface passes only the
// input and output pointers.  mfd_topk_logz_static serves them: its scratch (the per-piece partial records and
// the per-row tickets of mfd_topk_logz) lives in one file-scope device array that every GPU loading this
// library holds until the process exits.
//
// The array's name in host code is only a host-side stand-in for the device symbol, not a device address: a
// kernel given it would fault or, where the GPU can reach host memory, silently use the wrong memory.  So on the
// first call on each device, with that device current, cudaGetSymbolAddress() resolves the device address once
// and caches it per device; later calls reuse it.  Make that first call before capturing any stream.  The cached
// address belongs to the device context that was current then: after a cudaDeviceReset the module may load at
// another address, so resetting a device after its first call here is not supported.
//
// Every call shares the array and it keeps the previous call's contents: the ticket words, which must start at
// zero, are cleared on the call's stream before the kernel runs (cudaMemsetAsync, no allocation).  Calls whose
// work overlaps on the GPU (different streams, or different threads without ordering) race on the array.
// Nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include <atomic>
#include <mutex>

#include "common.cuh"

namespace {

// Capacity: partial records of up to kStaticPartBytes and tickets for up to kStaticRows rows.
constexpr size_t kStaticPartBytes = 4u << 20;  // 4 MiB
constexpr int64_t kStaticRows = 16384;
constexpr size_t kStaticTicketBytes = (size_t)kStaticRows * sizeof(unsigned int);

static __device__ __align__(256) unsigned char g_topk_static_scratch[kStaticTicketBytes + kStaticPartBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
std::atomic<unsigned char*> g_dev_scratch[kMaxDevices];

// Device address of the scratch array on the current device, resolved once per device.
int scratch_for_current_device(unsigned char** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        mfd::set_error("mfd_topk_logz_static: cudaGetDevice failed: %s", cudaGetErrorString(e));
        return MFD_ERR_CUDA;
    }
    if (dev < 0 || dev >= kMaxDevices) {
        mfd::set_error("mfd_topk_logz_static: device ordinal %d beyond the %d supported", dev, kMaxDevices);
        return MFD_ERR_UNSUPPORTED;
    }
    unsigned char* p = g_dev_scratch[dev].load(std::memory_order_acquire);
    if (!p) {
        std::lock_guard<std::mutex> lock(g_setup_mutex);
        p = g_dev_scratch[dev].load(std::memory_order_relaxed);
        if (!p) {
            void* addr = nullptr;
            e = cudaGetSymbolAddress(&addr, g_topk_static_scratch);
            if (e != cudaSuccess || !addr) {
                mfd::set_error("mfd_topk_logz_static: cudaGetSymbolAddress failed on device %d: %s", dev,
                               cudaGetErrorString(e));
                return MFD_ERR_CUDA;
            }
            p = (unsigned char*)addr;
            g_dev_scratch[dev].store(p, std::memory_order_release);
        }
    }
    *out = p;
    return MFD_OK;
}

}  // namespace

extern "C" int mfd_topk_logz_static(const void* x, int x_dtype, int64_t rows, int64_t vocab, int64_t row_stride,
                                    int64_t k, float* top_logp, void* top_ids, int ids_dtype, float* logz,
                                    void* stream) {
    // the argument checks of mfd_topk_logz, before any capacity check, so invalid calls report MFD_ERR_INVALID
    if (rows < 0 || vocab <= 0 || k <= 0 || k > vocab || k > 256 || row_stride < vocab) {
        mfd::set_error("mfd_topk_logz_static: invalid sizes rows=%lld vocab=%lld k=%lld stride=%lld (need "
                       "0<k<=min(vocab,256))", (long long)rows, (long long)vocab, (long long)k, (long long)row_stride);
        return MFD_ERR_INVALID;
    }
    if (x_dtype != MFD_F32 && x_dtype != MFD_BF16) {
        mfd::set_error("mfd_topk_logz_static: x_dtype must be MFD_F32 or MFD_BF16");
        return MFD_ERR_INVALID;
    }
    if (ids_dtype != MFD_I32 && ids_dtype != MFD_I64) {
        mfd::set_error("mfd_topk_logz_static: ids_dtype must be MFD_I32 or MFD_I64");
        return MFD_ERR_INVALID;
    }
    if (vocab >= (int64_t)0x7fffffff) {
        mfd::set_error("mfd_topk_logz_static: vocab must be < 2^31");
        return MFD_ERR_INVALID;
    }
    if (rows == 0) return MFD_OK;
    const size_t need = mfd_topk_logz_workspace(rows, vocab, k);
    if (rows > kStaticRows || need > kStaticPartBytes) {
        mfd::set_error(
            "mfd_topk_logz_static: rows=%lld vocab=%lld k=%lld need %zu bytes of scratch and %lld ticket rows; the "
            "static scratch holds %zu bytes and %lld rows (use mfd_topk_logz with a workspace instead)",
            (long long)rows, (long long)vocab, (long long)k, need, (long long)rows, kStaticPartBytes,
            (long long)kStaticRows);
        return MFD_ERR_UNSUPPORTED;
    }
    unsigned char* base = nullptr;
    int rc = scratch_for_current_device(&base);
    if (rc) return rc;
    unsigned int* tickets = (unsigned int*)base;
    cudaError_t e = cudaMemsetAsync(tickets, 0, (size_t)rows * sizeof(unsigned int), (cudaStream_t)stream);
    if (e != cudaSuccess) {
        mfd::set_error("mfd_topk_logz_static: clearing the tickets failed: %s", cudaGetErrorString(e));
        return MFD_ERR_CUDA;
    }
    return mfd_topk_logz(x, x_dtype, rows, vocab, row_stride, k, top_logp, top_ids, ids_dtype, logz,
                         base + kStaticTicketBytes, kStaticPartBytes, tickets, kStaticRows, stream);
}
