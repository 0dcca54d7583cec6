// kb_flash_attn_ext_noalloc: attention for callers that cannot hand this library any device memory.
//
// kb_flash_attn_ext needs a scratch buffer for its split-KV partials, which the caller allocates. Some
// callers cannot: code that runs while a CUDA graph is being captured (cudaMalloc is not allowed there),
// hosts that reserve the whole GPU up front for their own pools and keep no headroom, and foreign-language
// bindings that only pass raw pointers and have no way to allocate on the device. This entry point keeps
// the partials in a fixed buffer compiled into the library instead.
//
// The buffer is a file-scope static __device__ array, so every GPU that loads this library holds
// KB_NOALLOC_SCRATCH_BYTES of device memory until the process exits. All calls on a device share it:
// calls that overlap on the GPU (different streams, or different host threads) race on it and must be
// serialised by the caller. Each call writes every partial it later reads, so nothing has to be cleared
// between calls; a call whose bounded wait ran out leaves its output undefined (see kb_device_error).
#include <cuda_runtime.h>

#include <atomic>

#include "../../include/klein_b200.h"
#include "kb_internal.h"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[KB_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch on the current device. In host code the array's name only stands for
// the symbol, so the address must come from cudaGetSymbolAddress, once per device, with that device current.
// The cache is keyed on the device ordinal: the library assumes each device's primary context for the life of
// the process (no cudaDeviceReset, no other current context). Threads that race on the first lookup store the
// same address; the atomics make that explicit.
void* scratch_address(kb_status* st) {
    static std::atomic<void*> addr[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        *st = KB_ERR_CUDA;
        return nullptr;
    }
    void* p = addr[dev].load(std::memory_order_acquire);
    if (!p) {
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
            *st = KB_ERR_CUDA;
            return nullptr;
        }
        addr[dev].store(p, std::memory_order_release);
    }
    *st = KB_OK;
    return p;
}

}  // namespace

extern "C" kb_status kb_flash_attn_ext_noalloc(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v,
                                               const kb_tensor* mask, const kb_fa_params* params, const kb_tensor* dst,
                                               void* stream) {
    // the address lookup runs on every call, so the first call on a device always does it, whatever its shape
    kb_status st = KB_OK;
    void* scratch = scratch_address(&st);
    if (st != KB_OK) return st;
    // the least scratch with which the call runs (the split partials of the streaming kernel); a larger
    // preferred size (the f16 view of a quantised cache for prefill) falls back to that kernel
    const size_t need = kb::flash_attn_min_scratch_bytes(q, k, v, params);
    if (need > KB_NOALLOC_SCRATCH_BYTES) return KB_ERR_SCRATCH;  // more partials than the built-in buffer holds
    return kb::flash_attn_with_scratch(q, k, v, mask, params, dst, scratch, KB_NOALLOC_SCRATCH_BYTES, stream);
}
