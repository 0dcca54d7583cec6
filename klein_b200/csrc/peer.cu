// Exchange of split-KV partials between GPUs over NVLink without a collective library: every rank writes its
// packed partial (o, m, l) straight into the gather buffer of every rank (CUDA IPC peer mappings of plain device
// memory, ordinary stores), then counts its chunks in the destination's flag array (epoch x PUSH_CHUNKS once complete). The merge on each
// rank (lse_combine_kernel with flags) waits, bounded, for all epochs and reads its local buffer only. The epoch
// counter lives in device memory (flags[n_ranks]), so a captured CUDA graph replays correctly. This is
// the all-gather step of the KV-sequence split (the exchange that ops.cpp:9370-9438 does between CPU threads).
#include "kb_common.cuh"
#include "kb_internal.h"

namespace kb {

namespace {

constexpr int PUSH_THREADS = 256;

// Each destination's copy is spread over PUSH_CHUNKS CTAs (one SM alone pushes a few tens of GB/s over NVLink);
// every CTA adds 1 to the destination's flag for this source after its stores are visible system-wide, so a
// source's flag reads epoch * PUSH_CHUNKS once all of its chunks for that epoch have landed.
__global__ void __launch_bounds__(PUSH_THREADS) partials_push_kernel(const PeerPushParams p) {
    // this exchange's epoch: one past the last completed one (advanced by the merge, lse_combine_kernel)
    const int epoch = *reinterpret_cast<volatile const int*>(p.flags[p.rank] + p.n_ranks) + 1;
    const int dst = blockIdx.y;
    const float4* src = reinterpret_cast<const float4*>(p.part);
    float4* out = reinterpret_cast<float4*>(p.gather[dst] + (epoch & 1) * p.slot_set_floats + (int64_t) p.rank * p.part_floats);
    const int64_t n4 = p.part_floats / 4;
    const int64_t per = (n4 + PUSH_CHUNKS - 1) / PUSH_CHUNKS;
    const int64_t i0 = (int64_t) blockIdx.x * per, i1 = min(n4, i0 + per);
    for (int64_t i = i0 + threadIdx.x; i < i1; i += PUSH_THREADS) out[i] = src[i];
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) asm volatile("red.release.sys.global.add.s32 [%0], 1;" ::"l"(p.flags[dst] + p.rank) : "memory");
}

}  // namespace

cudaError_t launch_partials_push(const PeerPushParams& p, cudaStream_t stream) {
    partials_push_kernel<<<dim3(PUSH_CHUNKS, p.n_ranks), PUSH_THREADS, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace kb
