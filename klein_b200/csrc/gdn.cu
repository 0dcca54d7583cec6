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
// Every value column j of a head evolves independently, so a warp owns 4 columns with 8 lanes each: lane l holds
// 16 rows of column j0 + l / 8 (gdn_rec.cuh, the token step shared with the one-launch decode / verify layer), the two dot products per token are 3-level butterflies over the column's lanes, and the q / k rows
// are read as float4 per lane. The kernel streams the state once (read s0, write the slots), which makes it
// HBM-bound at decode/verify sizes.
//
// Where the slots go is the caller's choice: ggml's packed f32 output (attention, then K f32 slots), or
// klein's cache layout (graph.cpp:177-184, state.cpp:69-81): slot 0 back into the f32 state in place, slots
// 1..K-1 into the snapshot rows in f16 / bf16 / f32.
#include "kb_common.cuh"
#include "kb_gdn.h"
#include "gdn_rec.cuh"

namespace kb {

namespace {

constexpr int CPW = 4;    // state columns per warp
constexpr int WARPS = 4;  // warps per CTA

template <bool KDA>
__global__ void __launch_bounds__(WARPS * 32) gdn_recurrent_kernel(const GdnParams p) {
    constexpr int S = 128;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sh = blockIdx.x;  // sequence * H_v + head
    const int seq = sh / p.H_v, h = sh % p.H_v;
    const int hk = h % p.H_k;
    const int sq_q = seq / p.rq3, sq_k = seq / p.rk3;
    const int col = (blockIdx.y * WARPS + warp) * CPW + (lane >> 3);  // this lane's state column
    const int r8 = lane & 7;                                           // and its rows (gdn_row)
    const float scale = rsqrtf((float) S);

    float4 M[4];
    const float* s0 = p.s0 + (int64_t) seq * p.s0_seq_stride + (int64_t) h * S * S + (int64_t) col * S;
#pragma unroll
    for (int d = 0; d < 4; ++d) M[d] = *reinterpret_cast<const float4*>(s0 + gdn_row(r8, d));

    // token inputs, loaded one token ahead of the math that uses them
    struct TokIn {
        float4 k[4], q[4], e[4];
        float v, beta;
    };
    auto load_tok = [&](int t, TokIn& in) {
        const char* krow = p.k + sq_k * p.k_nb3 + t * p.k_nb2 + hk * p.k_nb1;
        const char* qrow = p.q + sq_q * p.q_nb3 + t * p.q_nb2 + hk * p.q_nb1;
#pragma unroll
        for (int d = 0; d < 4; ++d) {
            in.k[d] = *reinterpret_cast<const float4*>(krow + 4 * gdn_row(r8, d));
            in.q[d] = *reinterpret_cast<const float4*>(qrow + 4 * gdn_row(r8, d));
        }
        in.v = *reinterpret_cast<const float*>(p.v + seq * p.v_nb3 + t * p.v_nb2 + h * p.v_nb1 + (int64_t) col * 4);
        in.beta = *reinterpret_cast<const float*>(p.beta + seq * p.b_nb3 + t * p.b_nb2 + h * p.b_nb1);
        const char* grow = p.g + seq * p.g_nb3 + t * p.g_nb2 + h * p.g_nb1;
        if (KDA) {
#pragma unroll
            for (int d = 0; d < 4; ++d) in.e[d] = *reinterpret_cast<const float4*>(grow + 4 * gdn_row(r8, d));
        } else {
            const float g = *reinterpret_cast<const float*>(grow);
            in.e[0] = make_float4(g, g, g, g);
        }
    };
    TokIn cur, nxt;
    load_tok(0, cur);
    for (int t = 0; t < p.T; ++t) {
        if (t + 1 < p.T) load_tok(t + 1, nxt);
        float4 e[4];
        if (KDA) {
#pragma unroll
            for (int d = 0; d < 4; ++d)
                e[d] = make_float4(expf(cur.e[d].x), expf(cur.e[d].y), expf(cur.e[d].z), expf(cur.e[d].w));
        } else {
            const float eg = expf(cur.e[0].x);
#pragma unroll
            for (int d = 0; d < 4; ++d) e[d] = make_float4(eg, eg, eg, eg);
        }
        const float o = gdn_token(M, cur.k, cur.q, e, cur.v, cur.beta);
        if ((lane & 7) == 0)
            *reinterpret_cast<float*>(p.attn + seq * p.a_nb3 + t * p.a_nb2 + h * p.a_nb1 + (int64_t) col * 4) = o * scale;
        const int slot = p.T - 1 - t;
        if (slot < p.K) {
            char* base = slot == 0 ? p.slot0 : p.slots + (int64_t) (slot - 1) * p.slots_stride;
            const int type = slot == 0 ? 0 : p.slots_type;
            gdn_store_col(base, type, (((int64_t) seq * p.H_v + h) * S + col) * S, r8, M);
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
