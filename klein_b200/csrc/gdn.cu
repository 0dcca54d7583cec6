// Gated DeltaNet, recurrent form: GGML_OP_GATED_DELTA_NET for decode and the MTP verify step (and, as a
// plain loop over tokens, any T). Semantics of ggml_compute_forward_gated_delta_net_one_chunk
// (ggml-cpu/ops.cpp:11123-11275):
//
//   value head h reads q/k head h % H_k (:11199); the state is stored transposed, M[j][i] = S[i][j] (:11227)
//   per token t:  M[j][:] *= exp(g)            (scalar gate; KDA: M[j][i] *= exp(g[i]))      (:11240)
//                 delta_j = (v_j - sum_i M[j][i] k_i) * beta                                  (:11243-11248)
//                 M[j][i] += delta_j * k_i                                                    (:11251-11253)
//                 o_j = (sum_i M[j][i] q_i) / sqrt(S)                                         (:11256-11260)
//                 if slot = T-1-t < K: state snapshot `slot` = M                              (:11265-11271)
//
// Every value column j of a head evolves independently, so a warp owns CPW columns of one (sequence, head):
// lane l holds M[j][4l..4l+3] as a float4 for each of them, the two dot products are warp reductions, and
// q/k rows are read as float4 per lane. The kernel streams the state once (read s0, write the slots),
// which makes it HBM-bound at decode/verify sizes.
//
// Where the slots go is the caller's choice: ggml's packed f32 output (attention, then K f32 slots), or
// klein's cache layout (graph.cpp:177-184, state.cpp:69-81): slot 0 back into the f32 state in place, slots
// 1..K-1 into the snapshot rows in f16 / bf16 / f32.
#include "kb_common.cuh"
#include "kb_gdn.h"

namespace kb {

namespace {

constexpr int CPW = 4;    // state columns per warp
constexpr int WARPS = 4;  // warps per CTA

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int off = 16; off; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
    return x;
}

__device__ __forceinline__ void store4(char* base, int type, int64_t elem, float4 v) {
    if (type == 0) {
        *reinterpret_cast<float4*>(base + elem * 4) = v;
    } else if (type == 1) {
        __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
        uint2 u = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
        *reinterpret_cast<uint2*>(base + elem * 2) = u;
    } else {
        __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
        uint2 u = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
        *reinterpret_cast<uint2*>(base + elem * 2) = u;
    }
}

template <bool KDA>
__global__ void __launch_bounds__(WARPS * 32) gdn_recurrent_kernel(const GdnParams p) {
    constexpr int S = 128;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sh = blockIdx.x;  // sequence * H_v + head
    const int seq = sh / p.H_v, h = sh % p.H_v;
    const int hk = h % p.H_k;
    const int sq_q = seq / p.rq3, sq_k = seq / p.rk3;
    const int j0 = (blockIdx.y * WARPS + warp) * CPW;
    const float scale = rsqrtf((float) S);

    float4 M[CPW];
    const float* s0 = p.s0 + (int64_t) seq * p.s0_seq_stride + (int64_t) h * S * S;
#pragma unroll
    for (int c = 0; c < CPW; ++c) M[c] = *reinterpret_cast<const float4*>(s0 + (int64_t) (j0 + c) * S + 4 * lane);

    // token inputs, loaded one token ahead of the math that uses them
    struct TokIn {
        float4 k4, q4, g4;
        float v[CPW];
        float beta;
    };
    auto load_tok = [&](int t, TokIn& in) {
        in.k4 = *reinterpret_cast<const float4*>(p.k + sq_k * p.k_nb3 + t * p.k_nb2 + hk * p.k_nb1 + lane * 16);
        in.q4 = *reinterpret_cast<const float4*>(p.q + sq_q * p.q_nb3 + t * p.q_nb2 + hk * p.q_nb1 + lane * 16);
        const char* vrow = p.v + seq * p.v_nb3 + t * p.v_nb2 + h * p.v_nb1;
#pragma unroll
        for (int c = 0; c < CPW; ++c) in.v[c] = *reinterpret_cast<const float*>(vrow + (int64_t) (j0 + c) * 4);
        in.beta = *reinterpret_cast<const float*>(p.beta + seq * p.b_nb3 + t * p.b_nb2 + h * p.b_nb1);
        const char* grow = p.g + seq * p.g_nb3 + t * p.g_nb2 + h * p.g_nb1;
        if (KDA) in.g4 = *reinterpret_cast<const float4*>(grow + lane * 16);
        else in.g4.x = *reinterpret_cast<const float*>(grow);
    };
    TokIn cur, nxt;
    load_tok(0, cur);
    for (int t = 0; t < p.T; ++t) {
        if (t + 1 < p.T) load_tok(t + 1, nxt);
        const float4 k4 = cur.k4, q4 = cur.q4;
        const float beta = cur.beta;
        float4 e;
        if (KDA) {
            e = make_float4(expf(cur.g4.x), expf(cur.g4.y), expf(cur.g4.z), expf(cur.g4.w));
        } else {
            const float eg = expf(cur.g4.x);
            e = make_float4(eg, eg, eg, eg);
        }
        float vj[CPW];
#pragma unroll
        for (int c = 0; c < CPW; ++c) vj[c] = cur.v[c];
        float sk[CPW];
#pragma unroll
        for (int c = 0; c < CPW; ++c) {
            M[c].x *= e.x;
            M[c].y *= e.y;
            M[c].z *= e.z;
            M[c].w *= e.w;
            sk[c] = M[c].x * k4.x + M[c].y * k4.y + M[c].z * k4.z + M[c].w * k4.w;
        }
#pragma unroll
        for (int c = 0; c < CPW; ++c) sk[c] = warp_sum(sk[c]);
        float so[CPW];
#pragma unroll
        for (int c = 0; c < CPW; ++c) {
            const float delta = (vj[c] - sk[c]) * beta;
            M[c].x += delta * k4.x;
            M[c].y += delta * k4.y;
            M[c].z += delta * k4.z;
            M[c].w += delta * k4.w;
            so[c] = M[c].x * q4.x + M[c].y * q4.y + M[c].z * q4.z + M[c].w * q4.w;
        }
#pragma unroll
        for (int c = 0; c < CPW; ++c) so[c] = warp_sum(so[c]);
        if (lane < CPW) {
            float o = so[0];
#pragma unroll
            for (int c = 1; c < CPW; ++c)
                if (lane == c) o = so[c];
            *reinterpret_cast<float*>(p.attn + seq * p.a_nb3 + t * p.a_nb2 + h * p.a_nb1 + (int64_t) (j0 + lane) * 4) =
                o * scale;
        }
        const int slot = p.T - 1 - t;
        if (slot < p.K) {
            char* base;
            int type;
            if (slot == 0) {
                base = p.slot0;
                type = 0;
            } else {
                base = p.slots + (int64_t) (slot - 1) * p.slots_stride;
                type = p.slots_type;
            }
            const int64_t e0 = ((int64_t) seq * p.H_v + h) * S * S;
#pragma unroll
            for (int c = 0; c < CPW; ++c) store4(base, type, e0 + (int64_t) (j0 + c) * S + 4 * lane, M[c]);
        }
        cur = nxt;
    }
}

}  // namespace

cudaError_t launch_gdn_recurrent(const GdnParams& p, cudaStream_t stream) {
    dim3 grid(p.n_seqs * p.H_v, 128 / (WARPS * CPW));
    if (p.kda) gdn_recurrent_kernel<true><<<grid, WARPS * 32, 0, stream>>>(p);
    else gdn_recurrent_kernel<false><<<grid, WARPS * 32, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace kb
