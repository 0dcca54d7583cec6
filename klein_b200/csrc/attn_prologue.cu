// Attention prologue: the ops between the Q/K/V projections and GGML_OP_FLASH_ATTN_EXT in klein's
// Builder::attention (graph.cpp:94-112), in one launch instead of a chain of ggml nodes:
//   q, gate  = the two halves of each head's slice of the interleaved projection [2 hd] (ggml_view_3d)
//   q, k     = ggml_rms_norm(x, eps) * weight per head row (ops.cpp:4107-4167: the sum of squares in double,
//              mean rounded to float, scale = 1 / sqrtf(mean + eps), y = x * scale * w)
//   q, k     = ggml_rope_multi, M-RoPE with interleaved sections for GGML_ROPE_TYPE_IMROPE (ops.cpp:6219-6306,
//              6376-6450): NeoX pairs (i, i + n_rot / 2) over the first n_rot dims, theta of pair i = the position
//              component its sector selects times theta_scale^i (the same running f32 product), no YaRN ramp
//   gate     = ggml_cont of the gate half
//   caches   = ggml_set_rows of the normed, roped K rows and the V rows at kv_idx, f32 -> f16 (round to
//              nearest), q8_0 (per 32 values: d = amax / 127, q = roundf(x / d)) or q4_0 (quantize_row_q4_0_ref),
//              as kb_set_rows
//
// Layout: one warp per (token, row), rows = the nh query heads, then the nkv K heads, then the nkv V heads.
// Lane l holds dims l, l + 32, ..., so a 32-dim q8_0 block is one register across the warp and a rope pair
// (i, i + n_rot / 2) sits in one lane whenever n_rot / 2 is a multiple of 32.
#include "kb_common.cuh"
#include "kb_internal.h"

namespace kb {

namespace {

// M-RoPE of one head row held as x[k] = dim lane + 32 k: pairs (i, i + n_rot / 2) for i = lane + 32 j, j < OFF
// (OFF = n_rot / 64), NeoX layout; theta of pair i = the position component its sector selects times theta_scale^i
// as ggml's running f32 product (ops.cpp:6219-6306)
template <int EPL, int OFF>
__device__ __forceinline__ void rope_pairs(float (&x)[EPL], const PrologueParams& p, int t, int lane) {
    static_assert(2 * OFF <= EPL, "n_rot <= head dim");
#pragma unroll
    for (int j = 0; j < OFF; ++j) {
        const int i = lane + 32 * j;
        const int sector = i % p.sect_dims;
        int comp;
        if (p.imrope) {
            if (sector % 3 == 1 && sector < 3 * p.sections[1]) comp = 1;
            else if (sector % 3 == 2 && sector < 3 * p.sections[2]) comp = 2;
            else if (sector % 3 == 0 && sector < 3 * p.sections[0]) comp = 0;
            else comp = 3;
        } else {
            const int sec_w = p.sections[0] + p.sections[1];
            if (sector >= p.sections[0] && sector < sec_w) comp = 1;
            else if (sector >= sec_w && sector < sec_w + p.sections[2]) comp = 2;
            else if (sector >= sec_w + p.sections[2]) comp = 3;
            else comp = 0;
        }
        float theta = (float) p.pos[(int64_t) comp * p.n + t];
        for (int s = 0; s < i; ++s) theta *= p.theta_scale;  // ggml's running product, pair by pair
        theta *= p.freq_scale;
        // cosf and sinf of one argument in one call (one range reduction: the slow path at long-context angles)
        float sv, cv;
        sincosf(theta, &sv, &cv);
        const float c = cv * p.attn_factor, sn = sv * p.attn_factor;
        const float x0 = x[j], x1 = x[j + OFF];
        x[j] = x0 * c - x1 * sn;
        x[j + OFF] = x0 * sn + x1 * c;
    }
}

template <int EPL>  // elements per lane: hd / 32
__global__ void __launch_bounds__(256) attn_prologue_kernel(const PrologueParams p) {
    constexpr int HD = 32 * EPL;
    const int lane = threadIdx.x & 31;
    const int64_t task = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int rows = p.nh + 2 * p.nkv;
    if (task >= (int64_t) p.n * rows) return;
    const int t = (int) (task / rows), r = (int) (task % rows);
    const bool is_q = r < p.nh, is_v = r >= p.nh + p.nkv;
    const int kh = is_q ? 0 : (r - p.nh) % p.nkv;

    const float* src = is_q ? reinterpret_cast<const float*>(p.qfull + t * p.q_nb1) + (int64_t) r * 2 * HD
                            : reinterpret_cast<const float*>(is_v ? p.vcur + t * p.v_nb1 : p.kcur + t * p.k_nb1) + (int64_t) kh * HD;
    float x[EPL];
#pragma unroll
    for (int k = 0; k < EPL; ++k) x[k] = src[lane + 32 * k];
    if (is_q) {
        // the gate half, copied as it is
        const float* gsrc = src + HD;
        float* gdst = p.gate_out + ((int64_t) t * p.nh + r) * HD;
        if (p.gate_vec) {
            // HD / 4 units of 16 bytes (offsets 2 hd * 4 r + hd * 4 and hd * 4 (t nh + r) keep them aligned)
#pragma unroll
            for (int u = lane; u < HD / 4; u += 32)
                reinterpret_cast<float4*>(gdst)[u] = reinterpret_cast<const float4*>(gsrc)[u];
        } else {
#pragma unroll
            for (int k = 0; k < EPL; ++k) gdst[lane + 32 * k] = gsrc[lane + 32 * k];
        }
    }
    if (!is_v) {
        // RMS norm: the sum of squares of float products, accumulated in double as ggml does
        double ss = 0.0;
#pragma unroll
        for (int k = 0; k < EPL; ++k) ss += (double) (x[k] * x[k]);
#pragma unroll
        for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        const float mean = (float) (ss / HD);
        const float scale = 1.0f / sqrtf(mean + p.eps);
        const float* w = is_q ? p.q_norm : p.k_norm;
#pragma unroll
        for (int k = 0; k < EPL; ++k) x[k] = x[k] * scale * w[lane + 32 * k];
        // M-RoPE over pairs (i, i + n_rot / 2), i = lane + 32 j: element j and its partner j + n_rot / 64, with
        // n_rot / 64 a template argument so every index is a constant and x stays in registers
        const int off = p.n_rot / 64;
        if (off == 1) rope_pairs<EPL, 1>(x, p, t, lane);
        if constexpr (EPL >= 4) {
            if (off == 2) rope_pairs<EPL, 2>(x, p, t, lane);
        }
        if constexpr (EPL >= 8) {
            if (off == 3) rope_pairs<EPL, 3>(x, p, t, lane);
            if (off == 4) rope_pairs<EPL, 4>(x, p, t, lane);
        }
    }
    if (is_q) {
        float* dst = p.q_out + ((int64_t) t * p.nh + r) * HD;
#pragma unroll
        for (int k = 0; k < EPL; ++k) dst[lane + 32 * k] = x[k];
        return;
    }
    // K / V row into the cache
    const int64_t cell = p.kv_idx[t];
    if (cell < 0 || cell >= p.n_cells) {
        if (lane == 0) record_error(p.err, 1);
        return;
    }
    char* row = (is_v ? p.v_cache : p.k_cache) + cell * (is_v ? p.vc_nb1 : p.kc_nb1);
    if (p.cache_type == 1) {
        __half* d = reinterpret_cast<__half*>(row) + (int64_t) kh * HD;
#pragma unroll
        for (int k = 0; k < EPL; ++k) d[lane + 32 * k] = __float2half_rn(x[k]);
    } else if (p.cache_type == 2) {  // q4_0: block k of this head = lanes 0-31 of register k
        unsigned char* hb = reinterpret_cast<unsigned char*>(row) + (int64_t) kh * (HD / 32) * 18;
#pragma unroll
        for (int k = 0; k < EPL; ++k) store_block_q4_0(x[k], lane, hb + k * 18);
    } else {  // q8_0: block k of this head = lanes 0-31 of register k
        char* hb = row + (int64_t) kh * (HD / 32) * 34;
#pragma unroll
        for (int k = 0; k < EPL; ++k) {
            float amax = fabsf(x[k]);
#pragma unroll
            for (int off = 16; off; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
            const float d = amax / 127.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            char* b = hb + k * 34;
            b[2 + lane] = (char) (int8_t) roundf(x[k] * id);
            if (lane == 0) *reinterpret_cast<__half*>(b) = __float2half_rn(d);
        }
    }
}

}  // namespace

cudaError_t launch_attn_prologue(const PrologueParams& p, int hd, cudaStream_t stream) {
    const int64_t tasks = (int64_t) p.n * (p.nh + 2 * p.nkv);
    if (tasks == 0) return cudaSuccess;
    const unsigned grid = (unsigned) ((tasks + 7) / 8);
    switch (hd) {
        case 64: attn_prologue_kernel<2><<<grid, 256, 0, stream>>>(p); break;
        case 128: attn_prologue_kernel<4><<<grid, 256, 0, stream>>>(p); break;
        default: attn_prologue_kernel<8><<<grid, 256, 0, stream>>>(p); break;
    }
    return cudaGetLastError();
}

}  // namespace kb
