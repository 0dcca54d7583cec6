// The ops on either side of GGML_OP_GATED_DELTA_NET in klein's Builder::deltanet, one launch each:
//
// input side (graph.cpp:136-165):
//   beta  = sigmoid(beta_raw)                      ggml_sigmoid: 1 / (1 + expf(-x))
//   g     = softplus(alpha + dt_bias) * a          ggml_softplus: x > 20 ? x : logf(1 + expf(x))
//   conv  = silu(ssm_conv([state | qkv], w))       per channel c and token t: sum_j in[t + j][c] * w[j][c] over the
//                                                  kernel width kc, in[] = the kc - 1 stored inputs then the batch
//                                                  (ops.cpp:9931-9982), silu = x / (1 + expf(-x))
//   q, k  = l2(conv[q], conv[k]) per head          rms_norm(x, eps / S) * (1 / sqrt(S)) (graph.cpp:41-44)
//   v     = conv[v]
//   state = conv-state snapshots: slot s <- the kc - 1 inputs before token n - s (clamped at 0), for s < K,
//           skipping slots s >= n other than 0 (graph.cpp:147-155)
// output side (graph.cpp:186-190): o = rms_norm(attn, eps) * w * silu(z) per head row.
//
// Layout of the input kernel: one warp per (chunk of 8 tokens, or 4 for the verify step; head slot of S channels:
// the H_k q heads, the H_k k heads, the H_v v heads); lane l holds channels l, l + 32, ... of the slot and keeps
// the chunk's inputs and the conv window in registers. The tokens of a chunk are computed without branches between
// them, so their chains interleave (a chunk of 8 at 2 CTAs per SM measured 115 us at 4,096 tokens, against 168 us
// for 16-token chunks computed one token after the other). Only the chunk-0 warps read the stored state, and
// they write the snapshots after reading it, so no warp reads a state slot another writes.
#include "kb_common.cuh"
#include "kb_internal.h"

namespace kb {

namespace {

constexpr int KC = 4;  // conv kernel width (qwen35's ssm_conv_kernel); others are rejected by the host

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

// CPL consecutive floats in one 16- (CPL 4) or 8-byte (CPL 2) access
template <int CPL>
__device__ __forceinline__ void ld_vec(const float* src, float* d) {
    static_assert(CPL == 2 || CPL == 4, "8- or 16-byte accesses");
    if constexpr (CPL == 4) {
        const float4 a = *reinterpret_cast<const float4*>(src);
        d[0] = a.x, d[1] = a.y, d[2] = a.z, d[3] = a.w;
    } else {
        const float2 a = *reinterpret_cast<const float2*>(src);
        d[0] = a.x, d[1] = a.y;
    }
}
template <int CPL>
__device__ __forceinline__ void st_vec(float* dst, const float* v) {
    if constexpr (CPL == 4) *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
    else *reinterpret_cast<float2*>(dst) = make_float2(v[0], v[1]);
}

// CPL: channels per lane (S / 32); CH: tokens per warp (8 for batches, 4 for the verify step); CONSEC: lane l holds
// channels c0 + CPL l .. + CPL - 1 with vector accesses (16-byte aligned buffers), else c0 + l, c0 + l + 32, ...
template <int CPL, int CH, bool CONSEC>
__global__ void __launch_bounds__(256, 2) gdn_input_kernel(const GdnInputParams p) {
    static_assert(CH > KC - 1, "only the first chunk reads the stored state");
    constexpr int S = 32 * CPL;
    constexpr int KM1 = KC - 1;
    const int lane = threadIdx.x & 31;
    const int slots = 2 * p.H_k + p.H_v;
    const int64_t task = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int n_chunks = (p.n + CH - 1) / CH;
    // the beta / g rows ride along: one warp per token after the conv tasks
    const int64_t conv_tasks = (int64_t) n_chunks * slots;
    if (task >= conv_tasks) {
        const int64_t t = task - conv_tasks;
        if (t >= p.n || !p.beta_raw) return;
        for (int h = lane; h < p.H_v; h += 32) {
            const float b = p.beta_raw[t * p.H_v + h];
            p.beta_out[t * p.H_v + h] = 1.0f / (1.0f + expf(-b));
            const float x = p.alpha[t * p.H_v + h] + p.dt_bias[h];
            const float sp = x > 20.0f ? x : logf(1.0f + expf(x));
            p.g_out[t * p.H_v + h] = sp * p.a[h];
        }
        return;
    }
    const int chunk = (int) (task / slots), slot = (int) (task % slots);
    const int c0 = slot * S;  // first channel of the slot
    const int t0 = chunk * CH, t1 = min(p.n, t0 + CH);
    // channel of this lane's element i
    auto chan = [&](int i) -> int64_t { return CONSEC ? c0 + CPL * lane + i : c0 + lane + 32 * i; };
    // win[i][j]: the KC - 1 inputs before token t0 of channel chan(i) (for chunk 0 the stored state)
    float win[CPL][KM1], w[CPL][KC];
    if constexpr (CONSEC) {
        // the lane's CPL channels are contiguous in conv_w ([ch][KC]) and in the state ([ch][KC - 1])
        const int64_t cl = chan(0);
#pragma unroll
        for (int q = 0; q < KC; ++q) ld_vec<CPL>(p.conv_w + cl * KC + q * CPL, &w[0][0] + q * CPL);
        if (t0 == 0) {
#pragma unroll
            for (int q = 0; q < KM1; ++q) ld_vec<CPL>(p.state + cl * KM1 + q * CPL, &win[0][0] + q * CPL);
        } else {
#pragma unroll
            for (int j = 0; j < KM1; ++j) {
                float v[CPL];
                ld_vec<CPL>(p.qkv + (int64_t) (t0 - KM1 + j) * p.qkv_ld + cl, v);
#pragma unroll
                for (int i = 0; i < CPL; ++i) win[i][j] = v[i];
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
            const int64_t c = chan(i);
#pragma unroll
            for (int j = 0; j < KC; ++j) w[i][j] = p.conv_w[c * KC + j];
#pragma unroll
            for (int j = 0; j < KM1; ++j)
                // only the first chunk's window reaches into the stored state (CH > KC - 1)
                win[i][j] = t0 == 0 ? p.state[c * KM1 + j] : p.qkv[(int64_t) (t0 - KM1 + j) * p.qkv_ld + c];
        }
    }
    // the chunk's inputs, all loads in flight together (zeros past the batch: computed, never stored)
    float xs[CH][CPL];
#pragma unroll
    for (int u = 0; u < CH; ++u) {
        if constexpr (CONSEC) {
            if (t0 + u < t1) {
                ld_vec<CPL>(p.qkv + (int64_t) (t0 + u) * p.qkv_ld + chan(0), xs[u]);
            } else {
#pragma unroll
                for (int i = 0; i < CPL; ++i) xs[u][i] = 0.0f;
            }
        } else {
#pragma unroll
            for (int i = 0; i < CPL; ++i)
                xs[u][i] = t0 + u < t1 ? p.qkv[(int64_t) (t0 + u) * p.qkv_ld + chan(i)] : 0.0f;
        }
    }
    if (chunk == 0) {
        // conv-state snapshots of this lane's channels: slot s <- in[n - s .. n - s + KC - 2] (in = stored state |
        // batch), the window after n - s tokens, clamped at the start of in[]. The stored state and the chunk's
        // inputs come from registers (read above, before any snapshot is written); later inputs from the batch.
        for (int s = 0; s < p.K; ++s) {
            if (s >= p.n && s > 0) continue;
            const int start = max(0, p.n - s);
            float* dst = p.state + (int64_t) s * p.state_ld;
            float sv[CPL][KM1];
#pragma unroll
            for (int i = 0; i < CPL; ++i) {
                const int64_t c = chan(i);
#pragma unroll
                for (int j = 0; j < KM1; ++j) {
                    const int ii = start + j;  // index into in[]
                    float v = 0.0f;
#pragma unroll
                    for (int jj = 0; jj < KM1; ++jj)
                        if (ii == jj) v = win[i][jj];
#pragma unroll
                    for (int u = 0; u < CH; ++u)
                        if (ii == KM1 + u) v = xs[u][i];
                    if (ii >= KM1 + CH) v = p.qkv[(int64_t) (ii - KM1) * p.qkv_ld + c];
                    sv[i][j] = v;
                    if constexpr (!CONSEC) dst[c * KM1 + j] = v;
                }
            }
            if constexpr (CONSEC) {
#pragma unroll
                for (int q = 0; q < KM1; ++q) st_vec<CPL>(dst + chan(0) * KM1 + q * CPL, &sv[0][0] + q * CPL);
            }
        }
    }
    // output row of this slot: q (slot < H_k), k, or v
    const bool is_q = slot < p.H_k, is_k = !is_q && slot < 2 * p.H_k;
    float* out = is_q ? p.q_out + (int64_t) slot * S : is_k ? p.k_out + (int64_t) (slot - p.H_k) * S
                                                               : p.v_out + (int64_t) (slot - 2 * p.H_k) * S;
    const int64_t out_ld = (int64_t) (is_q || is_k ? p.H_k : p.H_v) * S;
    // conv + SiLU of every token, newest first so xs[u] can take y[u] once no later token reads it; no branch
    // between tokens, so the per-token chains (and the norms' reductions below) interleave
#pragma unroll
    for (int u = CH - 1; u >= 0; --u) {
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
            // ggml's order: sum over the window oldest first, one multiply-add per tap
            float acc = 0.0f;
#pragma unroll
            for (int j = 0; j < KM1; ++j) acc += (u - KM1 + j >= 0 ? xs[u - KM1 + j < 0 ? 0 : u - KM1 + j][i]
                                                                   : win[i][u + j < KM1 ? u + j : 0]) * w[i][j];
            acc += xs[u][i] * w[i][KM1];
            xs[u][i] = silu_f(acc);
        }
    }
#pragma unroll
    for (int u = 0; u < CH; ++u) {
        if (is_q || is_k) {
            // l2: rms_norm with eps / S (sum of squares in double, as ggml), then * 1 / sqrt(S)
            double ss = 0.0;
#pragma unroll
            for (int i = 0; i < CPL; ++i) ss += (double) (xs[u][i] * xs[u][i]);
#pragma unroll
            for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
            const float mean = (float) (ss / S);
            const float scale = 1.0f / sqrtf(mean + p.l2_eps);
#pragma unroll
            for (int i = 0; i < CPL; ++i) xs[u][i] = xs[u][i] * scale * p.inv_sqrt_s;
        }
        if (t0 + u < t1) {
            if constexpr (CONSEC) {
                st_vec<CPL>(out + (int64_t) (t0 + u) * out_ld + CPL * lane, xs[u]);
            } else {
#pragma unroll
                for (int i = 0; i < CPL; ++i) out[(int64_t) (t0 + u) * out_ld + lane + 32 * i] = xs[u][i];
            }
        }
    }
}

template <int CPL>
__global__ void __launch_bounds__(256) gdn_gated_norm_kernel(const GdnNormParams p) {
    constexpr int S = 32 * CPL;
    const int lane = threadIdx.x & 31;
    const int64_t task = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (task >= (int64_t) p.n * p.H) return;
    const float* x = p.x + task * S;
    const float* z = p.z + task * S;
    float* o = p.dst + task * S;
    float v[CPL];
    double ss = 0.0;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
        v[i] = x[lane + 32 * i];
        ss += (double) (v[i] * v[i]);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float mean = (float) (ss / S);
    const float scale = 1.0f / sqrtf(mean + p.eps);
#pragma unroll
    for (int i = 0; i < CPL; ++i) o[lane + 32 * i] = v[i] * scale * p.w[lane + 32 * i] * silu_f(z[lane + 32 * i]);
}

// The same op with lane l holding the CPL consecutive channels l CPL .. l CPL + CPL - 1 (one 16- or 8-byte access
// per array) and RPW rows per warp, their reductions interleaved; for 16-byte aligned rows
template <int CPL, int RPW>
__global__ void __launch_bounds__(256) gdn_gated_norm_vec_kernel(const GdnNormParams p) {
    static_assert(CPL == 2 || CPL == 4, "8- or 16-byte accesses");
    constexpr int S = 32 * CPL;
    const int lane = threadIdx.x & 31;
    const int64_t rows = (int64_t) p.n * p.H;
    const int64_t r0 = ((int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW;
    if (r0 >= rows) return;
    auto load = [](const float* src, float (&v)[CPL]) {
        if constexpr (CPL == 4) {
            const float4 a = *reinterpret_cast<const float4*>(src);
            v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w;
        } else {
            const float2 a = *reinterpret_cast<const float2*>(src);
            v[0] = a.x, v[1] = a.y;
        }
    };
    float wv[CPL], xv[RPW][CPL], zv[RPW][CPL];
    load(p.w + lane * CPL, wv);
#pragma unroll
    for (int rr = 0; rr < RPW; ++rr) {
        const int64_t row = min(r0 + rr, rows - 1);  // a missing row repeats the last one and is not stored
        load(p.x + row * S + lane * CPL, xv[rr]);
        load(p.z + row * S + lane * CPL, zv[rr]);
    }
#pragma unroll
    for (int rr = 0; rr < RPW; ++rr) {
        double ss = 0.0;
#pragma unroll
        for (int i = 0; i < CPL; ++i) ss += (double) (xv[rr][i] * xv[rr][i]);
#pragma unroll
        for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        const float mean = (float) (ss / S);
        const float scale = 1.0f / sqrtf(mean + p.eps);
        float o[CPL];
#pragma unroll
        for (int i = 0; i < CPL; ++i) o[i] = xv[rr][i] * scale * wv[i] * silu_f(zv[rr][i]);
        if (r0 + rr < rows) {
            float* dst = p.dst + (r0 + rr) * S + lane * CPL;
            if constexpr (CPL == 4) *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
            else *reinterpret_cast<float2*>(dst) = make_float2(o[0], o[1]);
        }
    }
}

}  // namespace

cudaError_t launch_gdn_input(const GdnInputParams& p, int S, cudaStream_t stream) {
    // 4-token chunks for the verify step (one chunk, less dead work), 8 otherwise
    const int ch = p.n <= 4 ? 4 : 8;
    const int n_chunks = (p.n + ch - 1) / ch;
    const int64_t tasks = (int64_t) n_chunks * (2 * p.H_k + p.H_v) + p.n;
    if (tasks == 0) return cudaSuccess;
    const unsigned grid = (unsigned) ((tasks + 7) / 8);
    // vector accesses need 16-byte aligned buffers and row / slot strides of whole 16-byte units
    const auto a16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    const bool vec = a16(p.qkv) && a16(p.state) && a16(p.conv_w) && a16(p.q_out) && a16(p.k_out) && a16(p.v_out) &&
                     p.qkv_ld % 4 == 0 && p.state_ld % 4 == 0;
    if (vec) {
        if (ch == 4) {
            if (S == 64) gdn_input_kernel<2, 4, true><<<grid, 256, 0, stream>>>(p);
            else gdn_input_kernel<4, 4, true><<<grid, 256, 0, stream>>>(p);
        } else {
            if (S == 64) gdn_input_kernel<2, 8, true><<<grid, 256, 0, stream>>>(p);
            else gdn_input_kernel<4, 8, true><<<grid, 256, 0, stream>>>(p);
        }
    } else if (ch == 4) {
        if (S == 64) gdn_input_kernel<2, 4, false><<<grid, 256, 0, stream>>>(p);
        else gdn_input_kernel<4, 4, false><<<grid, 256, 0, stream>>>(p);
    } else {
        if (S == 64) gdn_input_kernel<2, 8, false><<<grid, 256, 0, stream>>>(p);
        else gdn_input_kernel<4, 8, false><<<grid, 256, 0, stream>>>(p);
    }
    return cudaGetLastError();
}

cudaError_t launch_gdn_gated_norm(const GdnNormParams& p, int S, cudaStream_t stream) {
    const int64_t tasks = (int64_t) p.n * p.H;
    if (tasks == 0) return cudaSuccess;
    const auto a16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    if (a16(p.x) && a16(p.z) && a16(p.w) && a16(p.dst)) {
        // rows of S floats stay 16-byte aligned; 2 rows per warp, 8 warps per CTA
        constexpr int RPW = 2;
        const unsigned vgrid = (unsigned) ((tasks + 8 * RPW - 1) / (8 * RPW));
        if (S == 64) gdn_gated_norm_vec_kernel<2, RPW><<<vgrid, 256, 0, stream>>>(p);
        else gdn_gated_norm_vec_kernel<4, RPW><<<vgrid, 256, 0, stream>>>(p);
        return cudaGetLastError();
    }
    const unsigned grid = (unsigned) ((tasks + 7) / 8);
    switch (S) {
        case 64: gdn_gated_norm_kernel<2><<<grid, 256, 0, stream>>>(p); break;
        default: gdn_gated_norm_kernel<4><<<grid, 256, 0, stream>>>(p); break;
    }
    return cudaGetLastError();
}

}  // namespace kb
