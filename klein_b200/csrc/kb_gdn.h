// Internal parameter blocks of the DeltaNet, KV-write and rollback kernels.
#pragma once

#include <cuda.h>
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

// Chunked form (scalar gate, S = 128): tokens [tok0, tok0 + n_tok) in chunks of GDN_CHUNK. The prep kernel writes
// one record per (sequence, value head, chunk) into caller scratch; the state kernel consumes them in order.
constexpr int GDN_CHUNK = 64;
constexpr int GDN_REC_W = 0;          // W = T^-1 diag(beta Gamma) K, f16 image [2][64 s][64 i], 128B-swizzled
constexpr int GDN_REC_AQ_HI = 16384;  // A_qk hi, f16 image [64 t][64 s]
constexpr int GDN_REC_AQ_LO = 24576;  // A_qk lo
constexpr int GDN_REC_U = 32768;      // U~ = T^-1 diag(beta) V, f32 [64 s][128 j]
constexpr int GDN_REC_G = 65536;      // G, f32 [64]: running sums of the log-gates within the chunk
constexpr int64_t GDN_REC_BYTES = 65536 + 256;

struct GdnChunkParams {
    GdnParams in;                     // inputs and the attention output (its slot fields are unused)
    int64_t tok0, n_tok;              // token range of this pass
    int n_chunks;                     // ceil(n_tok / GDN_CHUNK)
    char* rec;                        // [n_seqs][H_v][n_chunks] records of GDN_REC_BYTES, 16-byte aligned
    const float* s0;                  // state before tok0 (f32, transposed), per-sequence stride in floats
    int64_t s0_seq_stride;
    float* s_out;                     // state after the pass (may alias s0)
    int64_t s_out_seq_stride;
    char* snap;                       // optional copy of s_out in snap_type (0 f32, 1 f16, 2 bf16), element
    int snap_type;                    //   ((seq * H_v + h) * S + j) * S + i
    int* err;
    uint64_t wait_ns;
};

// tmO: 4-d f32 map over the attention output (value dim, head, token, sequence) with box {128, 1, 64, 1}, its
// token extent ending at tok0 + n_tok
cudaError_t launch_gdn_chunked(const GdnChunkParams& p, const CUtensorMap& tmO, cudaStream_t stream);
// the two halves of launch_gdn_chunked: the records of the pass's chunks, then the state chain over them
cudaError_t launch_gdn_prep(const GdnChunkParams& p, cudaStream_t stream);
cudaError_t launch_gdn_state(const GdnChunkParams& p, const CUtensorMap& tmO, cudaStream_t stream);

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
