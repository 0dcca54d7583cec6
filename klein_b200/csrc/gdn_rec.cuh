// One token of the gated delta rule on 4 state columns per warp, shared by the recurrent kernel (gdn.cu) and the
// one-launch decode / verify layer (gdn_step.cu) so that both produce the same bits. ggml's semantics
// (ggml_compute_forward_gated_delta_net_one_chunk, ggml-cpu/ops.cpp:11227-11260), state stored transposed,
// M[j][i] = S[i][j]:
//   M[j][:] *= e               (scalar gate: e = exp(g); per-row gate: e[i] = exp(g[i]))
//   delta_j = (v_j - M[j] . k) * beta
//   M[j][:] += delta_j * k
//   o_j     = M[j] . q          (the caller applies 1 / sqrt(S))
// Layout: lane l holds 16 rows of column j0 + l / 8 as four float4, the d-th at rows gdn_row(l % 8, d) .. + 3
// = 4 (l % 8) + 32 d .. + 3, so that the column's 8 lanes cover 128 contiguous bytes per float4 (coalesced loads and
// whole-sector stores of the state). A dot product is the lane's four float4 partials (x, y, z, w in order) summed
// as (p0 + p1) + (p2 + p3), then the butterfly over the column's 8 lanes (xor 4, 2, 1): three shuffle levels per
// reduction, and 16 state values per lane.
#pragma once

#include <cuda_runtime.h>

namespace kb {

// first row of the lane's d-th float4 (r8 = lane % 8)
__device__ __forceinline__ int gdn_row(int r8, int d) { return 4 * r8 + 32 * d; }

__device__ __forceinline__ float gdn_dot4(const float4 a, const float4 b) {
    return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
}

__device__ __forceinline__ float gdn_col_sum8(float x) {
    x += __shfl_xor_sync(0xffffffffu, x, 4);
    x += __shfl_xor_sync(0xffffffffu, x, 2);
    x += __shfl_xor_sync(0xffffffffu, x, 1);
    return x;
}

// advances the lane's 16 state values by one token; returns o_j (equal in the column's 8 lanes)
__device__ __forceinline__ float gdn_token(float4 (&M)[4], const float4 (&k)[4], const float4 (&q)[4],
                                           const float4 (&e)[4], float v, float beta) {
#pragma unroll
    for (int d = 0; d < 4; ++d) {
        M[d].x *= e[d].x;
        M[d].y *= e[d].y;
        M[d].z *= e[d].z;
        M[d].w *= e[d].w;
    }
    float sk = (gdn_dot4(M[0], k[0]) + gdn_dot4(M[1], k[1])) + (gdn_dot4(M[2], k[2]) + gdn_dot4(M[3], k[3]));
    sk = gdn_col_sum8(sk);
    const float delta = (v - sk) * beta;
#pragma unroll
    for (int d = 0; d < 4; ++d) {
        M[d].x += delta * k[d].x;
        M[d].y += delta * k[d].y;
        M[d].z += delta * k[d].z;
        M[d].w += delta * k[d].w;
    }
    const float so = (gdn_dot4(M[0], q[0]) + gdn_dot4(M[1], q[1])) + (gdn_dot4(M[2], q[2]) + gdn_dot4(M[3], q[3]));
    return gdn_col_sum8(so);
}

__device__ __forceinline__ uint32_t gdn_pack2(int type, float a, float b) {
    if (type == 1) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// the lane's 16 values of a state column whose first element is `elem` (its row 0) in f32 / f16 / bf16 (type 0 / 1
// / 2; base 16-byte aligned): four 16- or 8-byte stores
__device__ __forceinline__ void gdn_store_col(char* base, int type, int64_t elem, int r8, const float4 (&M)[4]) {
#pragma unroll
    for (int d = 0; d < 4; ++d) {
        const int64_t e = elem + gdn_row(r8, d);
        if (type == 0)
            *reinterpret_cast<float4*>(base + e * 4) = M[d];
        else
            *reinterpret_cast<uint2*>(base + e * 2) =
                make_uint2(gdn_pack2(type, M[d].x, M[d].y), gdn_pack2(type, M[d].z, M[d].w));
    }
}

}  // namespace kb
