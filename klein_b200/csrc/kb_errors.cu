// The device error word: one int per device, set by kernels whose bounded waits run out.
#include <cuda_runtime.h>

#include <atomic>

#include "kb_internal.h"

namespace kb {

__device__ int g_kb_error_word;

// Keyed on the device ordinal (each device's primary context for the life of the process); threads racing on
// the first lookup store the same address.
int* device_error_word() {
    static std::atomic<int*> addr[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    int* a = addr[dev].load(std::memory_order_acquire);
    if (!a) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_kb_error_word) != cudaSuccess) return nullptr;
        a = static_cast<int*>(p);
        addr[dev].store(a, std::memory_order_release);
    }
    return a;
}

}  // namespace kb
