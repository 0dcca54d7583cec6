// Internal parameter blocks of the DeltaNet, KV-write and rollback kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace kb {

// One recurrent gated-DeltaNet launch (S = 128). Byte strides follow ggml; row stride nb0 = 4 everywhere.
struct GdnParams {
    const char* q;                   // f32 [S, H_k, T, n_seqs_q]
    int64_t q_nb1, q_nb2, q_nb3;
    const char* k;                   // f32 [S, H_k, T, n_seqs_k]
    int64_t k_nb1, k_nb2, k_nb3;
    const char* v;                   // f32 [S, H_v, T, n_seqs]
    int64_t v_nb1, v_nb2, v_nb3;
    const char* g;                   // f32 [1 or S, H_v, T, n_seqs]
    int64_t g_nb1, g_nb2, g_nb3;
    int kda;                         // vector gate (g has S entries per head)
    const char* beta;                // f32 [1, H_v, T, n_seqs]
    int64_t b_nb1, b_nb2, b_nb3;
    const float* s0;                 // f32 [S, S, H_v, n_seqs] initial state (transposed), contiguous per sequence
    int64_t s0_seq_stride;           // floats
    int S, H_k, H_v, T, n_seqs, K, rq3, rk3;
    char* attn;                      // f32 attention output element (j, h, t, seq)
    int64_t a_nb1, a_nb2, a_nb3;
    char* slot0;                     // f32 state after the last token: element ((seq*H_v + h)*S + j)*S + i
    char* slots;                     // slots 1..K-1, same element indexing, type slots_type
    int64_t slots_stride;            // bytes between consecutive slots
    int slots_type;                  // 0 f32, 1 f16, 2 bf16
};

cudaError_t launch_gdn_recurrent(const GdnParams& p, cudaStream_t stream);

// Cache row write (ggml_set_rows): dst row idx[r] of every (i2, i3) <- src row r converted to dst_type.
struct SetRowsParams {
    const char* src;                 // f32 [ne0, n_src, ne2, ne3]
    int64_t s_nb1, s_nb2, s_nb3;
    const char* idx;                 // i64 or i32 [n_src, ne11, ne12]
    int64_t i_nb0, i_nb1, i_nb2;
    int idx_i32;
    int64_t ne11, ne12;
    char* dst;                       // [ne0, n_rows, ne2, ne3] of dst_type
    int64_t d_nb1, d_nb2, d_nb3;
    int dst_type;                    // 0 f32, 1 f16, 8 q8_0, 30 bf16
    int64_t ne0, n_src, ne2, ne3, n_rows;
    int* err;                        // set to 1 when an index is out of range (the row is skipped)
};

cudaError_t launch_set_rows(const SetRowsParams& p, cudaStream_t stream);

// Rollback of up to KB_MAX_ROLLBACK_LAYERS DeltaNet layers after s rejected tokens (state.cpp:162-183).
constexpr int MAX_ROLLBACK_LAYERS = 64;
struct RollbackParams {
    float* conv[MAX_ROLLBACK_LAYERS];       // [n_snapshots][conv_row] f32
    const char* snap[MAX_ROLLBACK_LAYERS];  // [n_snapshots - 1][ssm_row] of snap_type
    float* ssm[MAX_ROLLBACK_LAYERS];        // [ssm_row] f32
    int n_layers;
    int64_t conv_row, ssm_row;
    int snap_type;                          // 0 f32, 1 f16, 2 bf16
    int s;                                  // 1 <= s < n_snapshots
};

cudaError_t launch_rollback(const RollbackParams& p, cudaStream_t stream);

}  // namespace kb
