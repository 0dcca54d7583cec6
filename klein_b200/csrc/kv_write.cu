// KV-cache row write and DeltaNet rollback: the device-side copies around the attention ops.
//
// set_rows: ggml_set_rows (ggml-cpu/ops.cpp:5446-5500; ggml-cuda/set-rows.cu:8-110) — klein writes the new
// K and V rows of every pass into its cache with it (graph.cpp:111-112). f32 rows are converted to the
// cache type: f16/bf16 round to nearest even; q8_0 follows quantize_row_q8_0_ref (ggml-quants.c:276-299):
// per 32 elements d = amax / 127, id = d ? 1/d : 0, q = roundf(x * id), d stored as f16 — the same rule
// ggml-cuda's set_rows applies (cpy-utils.cuh:137-154), bit for bit; q4_0 follows quantize_row_q4_0_ref.
//
// rollback: State::rollback_recurrent (state.cpp:162-183) — after s rejected draft tokens every DeltaNet
// layer's conv slot s becomes slot 0 (byte copy) and snapshot row s-1 becomes the f32 state (exact
// widening from f16/bf16). All layers in one launch.
#include "kb_common.cuh"
#include "kb_gdn.h"

namespace kb {

namespace {

// one warp per 32-element block of one destination row
__global__ void __launch_bounds__(256) set_rows_kernel(const SetRowsParams p) {
    const int64_t blocks_per_row = p.ne0 / 32;
    const int64_t task = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const int64_t total = p.n_src * p.ne2 * p.ne3 * blocks_per_row;
    if (task >= total) return;
    const int64_t blk = task % blocks_per_row;
    int64_t rest = task / blocks_per_row;
    const int64_t r = rest % p.n_src;
    rest /= p.n_src;
    const int64_t i2 = rest % p.ne2, i3 = rest / p.ne2;
    const char* ip = p.idx + r * p.i_nb0 + (i2 % p.ne11) * p.i_nb1 + (i3 % p.ne12) * p.i_nb2;
    const int64_t row = p.idx_i32 ? (int64_t) * reinterpret_cast<const int32_t*>(ip) : *reinterpret_cast<const int64_t*>(ip);
    if (row < 0 || row >= p.n_rows) {
        if (lane == 0 && blk == 0) record_error(p.err, 1);
        return;
    }
    const float x = *reinterpret_cast<const float*>(p.src + r * p.s_nb1 + i2 * p.s_nb2 + i3 * p.s_nb3 + (blk * 32 + lane) * 4);
    char* drow = p.dst + row * p.d_nb1 + i2 * p.d_nb2 + i3 * p.d_nb3;
    switch (p.dst_type) {
        case 0: reinterpret_cast<float*>(drow)[blk * 32 + lane] = x; break;
        case 1: reinterpret_cast<__half*>(drow)[blk * 32 + lane] = __float2half_rn(x); break;
        case 30: reinterpret_cast<__nv_bfloat16*>(drow)[blk * 32 + lane] = __float2bfloat16_rn(x); break;
        case 2: store_block_q4_0(x, lane, reinterpret_cast<unsigned char*>(drow) + blk * 18); break;
        default: {  // q8_0
            float amax = fabsf(x);
#pragma unroll
            for (int off = 16; off; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
            const float d = amax / 127.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            char* b = drow + blk * 34;
            b[2 + lane] = (char) (int8_t) roundf(x * id);
            if (lane == 0) *reinterpret_cast<__half*>(b) = __float2half_rn(d);
        }
    }
}

__global__ void __launch_bounds__(256) rollback_kernel(const RollbackParams p) {
    const int layer = blockIdx.y;
    const int64_t stride = (int64_t) gridDim.x * blockDim.x;
    const int64_t i0 = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    // conv: slot s -> slot 0 (f32 byte copy), 4 floats per thread-step
    float* conv = p.conv[layer];
    const float4* csrc = reinterpret_cast<const float4*>(conv + (int64_t) p.s * p.conv_row);
    float4* cdst = reinterpret_cast<float4*>(conv);
    for (int64_t i = i0; i < p.conv_row / 4; i += stride) cdst[i] = csrc[i];
    // ssm: snapshot row s-1 -> f32 state
    float* ssm = p.ssm[layer];
    if (p.snap_type == 0) {
        const float4* src = reinterpret_cast<const float4*>(p.snap[layer] + (int64_t) (p.s - 1) * p.ssm_row * 4);
        for (int64_t i = i0; i < p.ssm_row / 4; i += stride) reinterpret_cast<float4*>(ssm)[i] = src[i];
    } else {
        const uint2* src = reinterpret_cast<const uint2*>(p.snap[layer] + (int64_t) (p.s - 1) * p.ssm_row * 2);
        for (int64_t i = i0; i < p.ssm_row / 4; i += stride) {
            uint2 u = src[i];
            float4 o;
            if (p.snap_type == 1) {
                const float2 a = __half22float2(*reinterpret_cast<__half2*>(&u.x));
                const float2 b = __half22float2(*reinterpret_cast<__half2*>(&u.y));
                o = make_float4(a.x, a.y, b.x, b.y);
            } else {
                const float2 a = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u.x));
                const float2 b = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u.y));
                o = make_float4(a.x, a.y, b.x, b.y);
            }
            reinterpret_cast<float4*>(ssm)[i] = o;
        }
    }
}

}  // namespace

cudaError_t launch_set_rows(const SetRowsParams& p, cudaStream_t stream) {
    const int64_t tasks = p.n_src * p.ne2 * p.ne3 * (p.ne0 / 32);
    if (tasks == 0) return cudaSuccess;
    const int64_t blocks = (tasks + 7) / 8;
    set_rows_kernel<<<(unsigned) blocks, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_rollback(const RollbackParams& p, cudaStream_t stream) {
    if (p.n_layers <= 0) return cudaSuccess;
    const int64_t work = (p.ssm_row / 4 + 255) / 256;
    dim3 grid((unsigned) (work < 64 ? work : 64), p.n_layers);
    rollback_kernel<<<grid, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace kb
