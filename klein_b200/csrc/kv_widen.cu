// Widening of a q8_0 / q4_0 KV-cache range to f16 for the tensor-core prefill (fa_prefill.cu).
//
// Prefill over a quantised cache is compute-bound: every 64-cell K/V block is read by the 6 query heads of its
// GQA group and by every 128-query tile that sees it, so widening it once per call into an f16 copy costs one
// HBM pass (read 1,088 or 576 B, write 2,048 B per cell and per K / V; 0.25 ms for 262,144 cells) where
// dequantising inside the attention kernel would repeat the work per tile and head on the CUDA cores that
// already bound the prefill's softmax. ggml-cuda does the same conversion before its MMA kernel
// (fattn-common.cuh:1031-1090). Values are f16(q * d) for q8_0 and f16((n - 8) * d) for q4_0
// (dequantize_row_q8_0 / dequantize_row_q4_0, ggml-quants.c:553-567, 459-477, rounded to f16 as the streaming
// kernel widens them).
//
// One warp per (cell, head) row: the raw row (272 or 144 B, 16-byte aligned) goes to shared memory by 32-bit
// loads, then lane l writes dims [8 l, 8 l + 8) as one 16-byte store, so a warp writes the row's 512 B contiguously.
#include "kb_common.cuh"
#include "kb_internal.h"

namespace kb {

namespace {

constexpr int WARPS = 8;
constexpr int MAX_WORDS = 68;  // a q8_0 head row of 256 values: 8 blocks x 34 B = 272 B

template <int KT>  // KB_TYPE_Q8_0 or KB_TYPE_Q4_0
__global__ void __launch_bounds__(WARPS * 32) kv_widen_kernel(const KvWidenParams p) {
    __shared__ uint32_t raw[WARPS][MAX_WORDS];
    constexpr int BLK = KT == KB_TYPE_Q8_0 ? 34 : 18;
    constexpr int WORDS = 8 * BLK / 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t n_cells = p.c1 - p.c0;
    const int64_t rows = n_cells * p.H_kv * p.ne3;
    const unsigned char* bytes = reinterpret_cast<const unsigned char*>(raw[warp]);
    for (int64_t row = (int64_t) blockIdx.x * WARPS + warp; row < rows; row += (int64_t) gridDim.x * WARPS) {
        const int hk = (int) (row % p.H_kv);
        const int64_t rest = row / p.H_kv;
        const int64_t cell = p.c0 + rest % n_cells;
        const int b = (int) (rest / n_cells);
        const char* sp = p.src + cell * p.s_nb1 + hk * p.s_nb2 + b * p.s_nb3;
        const uint32_t* src = reinterpret_cast<const uint32_t*>(sp);
        __syncwarp();
        for (int w = lane; w < WORDS; w += 32) raw[warp][w] = src[w];
        __syncwarp();
        const int blk = lane >> 2, part = lane & 3;
        const unsigned char* bp = bytes + BLK * blk;
        const float d = __half2float(*reinterpret_cast<const __half*>(bp));
        float x[8];
        if constexpr (KT == KB_TYPE_Q8_0) {
#pragma unroll
            for (int i = 0; i < 8; ++i) x[i] = (float) (signed char) bp[2 + 8 * part + i] * d;
        } else {
            // value j < 16: low nibble of byte j; value 16 + j: high nibble of byte j
            const int j0 = 8 * (part & 1), sh = 4 * (part >> 1);
#pragma unroll
            for (int i = 0; i < 8; ++i) x[i] = (float) (((bp[2 + j0 + i] >> sh) & 15) - 8) * d;
        }
        uint4 o;
        o.x = pack_half2(x[0], x[1]);
        o.y = pack_half2(x[2], x[3]);
        o.z = pack_half2(x[4], x[5]);
        o.w = pack_half2(x[6], x[7]);
        __half* dst = p.dst + ((b * p.n_kv + cell) * p.H_kv + hk) * (int64_t) FA_D;
        reinterpret_cast<uint4*>(dst)[lane] = o;
    }
}

}  // namespace

cudaError_t launch_kv_widen(const KvWidenParams& p, int kv_type, cudaStream_t stream) {
    const int64_t rows = (p.c1 - p.c0) * p.H_kv * p.ne3;
    if (rows <= 0) return cudaSuccess;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // up to 8 CTAs of 8 warps per SM, grid-stride beyond that
    const int64_t want = (rows + WARPS - 1) / WARPS;
    const int grid = (int) (want < (int64_t) sms * 8 ? want : (int64_t) sms * 8);
    if (kv_type == KB_TYPE_Q8_0)
        kv_widen_kernel<KB_TYPE_Q8_0><<<grid, WARPS * 32, 0, stream>>>(p);
    else if (kv_type == KB_TYPE_Q4_0)
        kv_widen_kernel<KB_TYPE_Q4_0><<<grid, WARPS * 32, 0, stream>>>(p);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

}  // namespace kb
