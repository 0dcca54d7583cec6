// The device error word: one int per device, set by kernels whose bounded waits run out.
#include <cuda_runtime.h>

#include "kb_internal.h"

namespace kb {

__device__ int g_kb_error_word;

int* device_error_word() {
    static int* addr[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (!addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_kb_error_word) != cudaSuccess) return nullptr;
        addr[dev] = static_cast<int*>(p);
    }
    return addr[dev];
}

}  // namespace kb
