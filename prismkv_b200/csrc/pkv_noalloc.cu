// pkv_noalloc.cu -- pkv_attn_decode_noalloc: split-K decode attention whose
// scratch lives in a static device array instead of a caller workspace.
//
// Who needs it: a caller that cannot allocate device memory on its decode
// path -- a C or C++ host without a caching allocator, for which cudaMalloc
// and cudaFree would synchronise the device on every step, or an embedding
// runtime that hands the library only the KV buffers and a stream.  It has no
// counterpart in the reference, whose attention runs one query per call and
// keeps no workspace.
//
// Scratch layout (kNoallocBytes, 256-byte aligned, one copy per device):
//   [0, kCountOff)               split partials, placed so they END at kCountOff
//   [kCountOff, kNoallocBytes)   one int32 arrival counter per (batch, unit head)
// The counters are the only part that must be zero when a kernel starts.  The
// array is zero at module load, the first call on each device zeroes the
// counter region again, and every kernel leaves each counter it used at zero
// (the last CTA of a row resets it), so the region stays zero between calls.
// Partials are written before they are read and need no clearing.  Because
// the counters sit at a fixed offset, calls of different shapes never see a
// counter where an earlier call left partial sums.
//
// The array is shared by every call on a device: two calls that overlap in
// time (different streams, or threads without ordering) race on it.
#include <mutex>

#include "pkv_common.cuh"

namespace pkv {

size_t attn_counter_bytes(const pkv_codec* c, const pkv_attn_args* a);

constexpr size_t kNoallocBytes = PKV_NOALLOC_SCRATCH_BYTES;
constexpr size_t kCountOff = kNoallocBytes - (size_t)PKV_NOALLOC_MAX_KV_ROWS * sizeof(int32_t);
constexpr int kNoallocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocBytes];

static std::mutex g_noalloc_mu;
static void* g_noalloc_zeroed[kNoallocMaxDevices] = {};

// Address of the current context's copy of the scratch array, looked up on every call (cheap;
// a device reset or another context on the device gives another address).  The first call that
// sees an address on a device zeroes its counter region on `st`.
static int noalloc_scratch(cudaStream_t st, unsigned char** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return PKV_ERR_CUDA;
    if (dev < 0 || dev >= kNoallocMaxDevices) return PKV_ERR_UNSUPPORTED;
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) return PKV_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_zeroed[dev] != ptr) {
        if (cudaMemsetAsync(static_cast<unsigned char*>(ptr) + kCountOff, 0, kNoallocBytes - kCountOff, st) !=
            cudaSuccess)
            return PKV_ERR_CUDA;
        g_noalloc_zeroed[dev] = ptr;
    }
    *out = static_cast<unsigned char*>(ptr);
    return PKV_OK;
}

}  // namespace pkv

extern "C" int pkv_attn_decode_noalloc(const pkv_codec* c, const pkv_attn_args* a, void* stream) {
    const size_t need = pkv_attn_workspace_size(c, a);   // 0 for invalid arguments or one split
    if (need == 0) return pkv_attn_decode(c, a, nullptr, 0, stream);
    const size_t counters = pkv::attn_counter_bytes(c, a);
    const size_t part = need - counters;                  // partial bytes, a multiple of 256
    if (part > pkv::kCountOff || counters > pkv::kNoallocBytes - pkv::kCountOff) return PKV_ERR_SCRATCH_LIMIT;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned char* base = nullptr;
    const int rc = pkv::noalloc_scratch(st, &base);
    if (rc) return rc;
    // partials end where the counters begin: launch_attn puts the counters right after them
    return pkv_attn_decode(c, a, base + pkv::kCountOff - part, need, stream);
}
