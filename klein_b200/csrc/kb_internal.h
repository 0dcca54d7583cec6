// Internal interface between the C-ABI shim (kb_api.cpp) and the kernel launchers (*.cu).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/klein_b200.h"

namespace kb {

constexpr int FA_D = 256;            // head dimension of qwen35 full attention (K and V)
constexpr int FA_TILE = 64;          // keys per pipeline stage

// Parameters of one streaming (decode / verify) attention launch. Byte strides follow ggml.
struct FaStreamParams {
    const char* q;                   // f32 [D, n_q, H, ne3]
    int64_t q_nb1, q_nb2, q_nb3;
    int q_vec4;                      // q rows 16-byte aligned
    int n_q, n_head, n_head_kv, gqa, ne3, rk3;
    int R;                           // rows per KV head = n_q * gqa
    int64_t n_kv;
    // dense f16 mask [n_kv, n_q', ne32, ne33] or null
    const char* mask;
    int64_t m_nb1, m_nb2, m_nb3;
    int m_ne2, m_ne3;
    float scale_log2;                // scale * log2(e)          (no softcap)
    float scale_sc;                  // scale / softcap           (softcap)
    float softcap_log2;              // softcap * log2(e)         (softcap)
    int has_softcap;
    float max_bias, m0, m1;
    int n_head_log2;
    int causal;
    int64_t pos0, kv_lo, ring;
    // KV split
    int n_splits;                    // split s: 128-cell blocks [s base + min(s, extra), + base + (s < extra))
    int64_t blocks_base;
    int blocks_extra;
    int n_row_chunks;                // CTAs along the rows of one KV head (16 or 32 rows each at most)
    // outputs
    float* o_part;                   // scratch: [ne3][H_kv][chunk][split][RPC][D]
    float* ml_part;                  // scratch: [ne3][H_kv][chunk][split][RPC][2] (max in log2 units, sum)
    char* dst;                       // f32 [D, H, n_q, ne3]; with partial_out: unnormalised o, same layout
    int64_t d_nb1, d_nb2, d_nb3;
    int partial_out;                 // write (o, m, l) partials instead of the normalised output
    float* dst_ml;                   // partial_out: f32 [ne3][n_q][H][2] = (max in log2 units, sum)
    const char* gate;                // null, or f32 [D, H, n_q, ne3]: the output is o * sigmoid(gate) (not partials)
    int64_t g_nb1, g_nb2, g_nb3;
    // fused exchange (kb_flash_attn_ext_push): the split combine writes each merged partial row into slot `rank` of
    // every rank's gather buffer, and its last CTA counts the exchange in their flags (as kb_partials_push does)
    int push;
    int rank, n_ranks;
    int64_t slot_set_floats, part_floats;
    float* gather[16];
    int* flags[16];
    int* push_counter;               // in the scratch: combine CTAs done (zeroed by the attention kernel)
    // in-kernel exchange (kb_flash_attn_ext_exchange): after a grid barrier the kernel merges its splits, stores the
    // merged rows into every rank's gather buffer, flags each slot of rows in every rank's flag array, waits for the
    // same slot from every rank and writes the final output (gather / flags / rank / n_ranks / slot_set_floats /
    // part_floats as for push). Launched cooperatively: every CTA is resident at once.
    int xchg;
    int* err;                        // device error word
    uint64_t wait_ns;                // budget of every bounded wait
};

// the tcgen05 streaming kernel (kv_type: KB_TYPE_F16 = 1 or KB_TYPE_Q8_0 = 8): chunks of rpc = 16 or 32 rows, KV
// splits of whole 128-cell blocks (FA_TC_BLOCK)
constexpr int FA_TC_BLOCK = 128;
inline int fa_tc_rpc(int R) { return R <= 16 ? 16 : 32; }
size_t fa_stream_tc_smem_bytes(int rpc, int kv_type);
cudaError_t launch_fa_stream_tc(const FaStreamParams& p, int rpc, int kv_type, const CUtensorMap& tmK,
                                const CUtensorMap& tmV, cudaStream_t stream);

// Parameters of one causal-prefill launch (tcgen05 kernel): one CTA per 128-query tile of one head.
struct FaPrefillParams {
    const char* q;                   // f32 [D, n_q, H, ne3], rows 16-byte aligned
    int64_t q_nb1, q_nb2, q_nb3;
    int n_q, n_head, n_head_kv, gqa, ne3, rk3, n_qtiles;
    int64_t n_kv;
    const char* mask;                // f16 [n_kv, n_q', ne32, ne33] or null
    int64_t m_nb1, m_nb2, m_nb3;
    int m_ne2, m_ne3;
    float scale_log2, scale_sc, softcap_log2;
    int has_softcap;
    float max_bias, m0, m1;
    int n_head_log2;
    int causal;
    int64_t pos0, kv_lo;
    char* dst;                       // f32 [D, H, n_q, ne3]
    int64_t d_nb1, d_nb2, d_nb3;
    const char* gate;                // null, or f32 [D, H, n_q, ne3]: the output is o * sigmoid(gate)
    int64_t g_nb1, g_nb2, g_nb3;
    // a dense mask broadcast over the heads, classified per (128-query tile, 64-cell block) by
    // launch_fa_mask_classify: FA_MASK_MIXED, FA_MASK_ZERO (every value 0) or FA_MASK_HIDDEN (every value -inf); null
    // when not classified
    const uint8_t* mask_cls;
    int cls_ld;                      // blocks per tile row of the table
    int* err;
    uint64_t wait_ns;
};
constexpr uint8_t FA_MASK_MIXED = 0, FA_MASK_ZERO = 1, FA_MASK_HIDDEN = 2;

size_t fa_prefill_smem_bytes(bool pair);
// classes of mask rows [0, n_q) (row stride m_nb1) x cells [0, n_kv) into out[tile * n_blocks + block]
cudaError_t launch_fa_mask_classify(const char* mask, int64_t m_nb1, int n_q, int64_t n_kv, int n_blocks, uint8_t* out,
                                    cudaStream_t stream);
// fmt: 0 = f16 K/V, 1 = bf16 K/V, 2 = f16 K/V widened from q8_0 / q4_0 (Q rounded to q8_0 first). pair: clusters of 2
// CTAs sharing each MMA (n_head and gqa even; tmK's box 32 cells instead of 64)
cudaError_t launch_fa_prefill(const FaPrefillParams& p, int fmt, bool pair, const CUtensorMap& tmK, const CUtensorMap& tmV,
                              cudaStream_t stream);
constexpr int FA_PAIR_KROWS = 32;  // cells of a K tile each CTA of a pair loads

// Widening of cells [c0, c1) of a q8_0 / q4_0 cache view [D = 256, n_kv, H_kv, ne3] (kv_widen.cu) into a contiguous
// f16 copy [ne3][n_kv][H_kv][256] (cells outside [c0, c1) are not written).
struct KvWidenParams {
    const char* src;                 // raw rows; every head row 16-byte aligned
    int64_t s_nb1, s_nb2, s_nb3;
    __half* dst;
    int64_t n_kv, c0, c1;
    int H_kv, ne3;
};
cudaError_t launch_kv_widen(const KvWidenParams& p, int kv_type, cudaStream_t stream);

// merges n_parts partial results: o_p [rows][D] at o_parts + p*stride, ml_p [rows][2] at ml_parts + p*stride
// Plain merge: flags == nullptr. Exchange merge: flags = this rank's flag array [n_parts flags | epoch counter |
// done counter]; every CTA reads the counter, merges slot set (counter + 1) & 1 (parts at
// o_parts + set * slot_set_floats) after waiting, bounded by wait_ns, until flags[p] >= counter + 1 for all p; the
// last CTA to finish advances the counter.
cudaError_t launch_lse_combine(const float* o_parts, const float* ml_parts, int64_t stride, int n_parts, int64_t rows, int D,
                               float* dst, cudaStream_t stream, int* flags = nullptr, int64_t slot_set_floats = 0,
                               int* err = nullptr, uint64_t wait_ns = 0);

// Writes this rank's packed partial into slot `rank` of slot set (epoch & 1) of every rank's gather buffer
// (peer mappings), epoch = this rank's counter + 1, then releases epoch into flags[dst][rank] (system scope).
// One CTA per destination rank.
constexpr int MAX_PEERS = 16;
struct PeerPushParams {
    const float* part;
    int64_t part_floats;                 // multiple of 4
    int64_t slot_set_floats;             // floats between the two slot sets of a gather buffer
    float* gather[MAX_PEERS];            // each rank's gather buffer
    int* flags[MAX_PEERS];               // each rank's flag array [n_ranks flags | epoch counter | done counter]
    int rank, n_ranks;
};
constexpr int PUSH_CHUNKS = 32;  // CTAs per destination of a push; a complete push counts this many in its flag
// Flag array words of the in-kernel exchange: [n_ranks] epoch (shared with the push / wait exchange), [n_ranks + 2]
// grid-barrier arrivals, [n_ranks + 3] CTAs done, and from XCHG_FLAG_BASE one word per (source rank, output row)
// holding the last epoch that source has delivered for that row.
constexpr int XCHG_FLAG_BASE = 64;
constexpr int XCHG_MAX_SLOTS = 512;
cudaError_t launch_partials_push(const PeerPushParams& p, cudaStream_t stream);

// Parameters of the attention prologue (attn_prologue.cu): Q/gate split, RMS norms, M-RoPE, KV-cache writes.
struct PrologueParams {
    const char* qfull;               // f32 [n][nh][2 hd]: q then gate per head
    int64_t q_nb1;
    const char* kcur;                // f32 [n][nkv][hd]
    const char* vcur;
    int64_t k_nb1, v_nb1;
    const int32_t* pos;              // [4][n], section-major
    const int64_t* kv_idx;           // [n]
    const float* q_norm;             // [hd]
    const float* k_norm;
    float* q_out;                    // f32 [n][nh][hd]
    float* gate_out;                 // f32 [n][nh][hd]
    char* k_cache;                   // f16 / q8_0 rows of nkv * hd values
    char* v_cache;
    int64_t kc_nb1, vc_nb1, n_cells;
    int cache_type;                  // KB_TYPE_F16, KB_TYPE_Q8_0 or KB_TYPE_Q4_0
    int gate_vec;                    // qfull and gate_out 16-byte aligned (rows too): the gate is copied in 16 B units
    int n, nh, nkv;
    float eps;
    int n_rot, sect_dims, imrope;
    int sections[4];
    float theta_scale, freq_scale, attn_factor;
    int* err;
};
cudaError_t launch_attn_prologue(const PrologueParams& p, int hd, cudaStream_t stream);

// Parameters of the DeltaNet input side (gdn_io.cu): conv + SiLU + L2 norms + conv-state snapshots, beta and g.
struct GdnInputParams {
    const float* qkv;                // [n][qkv_ld]: channels 2 S H_k + S H_v (q heads, k heads, v heads)
    int64_t qkv_ld;
    float* state;                    // conv state slots [K][state_ld]: channel-major (kc - 1) inputs per channel
    int64_t state_ld;
    const float* conv_w;             // [ch][kc]
    const float* beta_raw;           // [n][H_v] or null (then alpha, dt_bias, a, beta_out, g_out are unused)
    const float* alpha;              // [n][H_v]
    const float* dt_bias;            // [H_v]
    const float* a;                  // [H_v]
    float* q_out;                    // [n][H_k][S]
    float* k_out;                    // [n][H_k][S]
    float* v_out;                    // [n][H_v][S]
    float* beta_out;                 // [n][H_v]
    float* g_out;                    // [n][H_v]
    int n, H_k, H_v, K;
    float l2_eps, inv_sqrt_s;
};
cudaError_t launch_gdn_input(const GdnInputParams& p, int S, cudaStream_t stream);

// Parameters of the DeltaNet gated RMS norm (gdn_io.cu): dst = rms_norm(x, eps) * w * silu(z) per [S] row.
struct GdnNormParams {
    const float* x;                  // [n][H][S]
    const float* z;                  // [n][H][S]
    const float* w;                  // [S]
    float* dst;                      // [n][H][S]
    int n, H;
    float eps;
};
cudaError_t launch_gdn_gated_norm(const GdnNormParams& p, int S, cudaStream_t stream);

// One DeltaNet layer of a decode / verify pass in one launch (gdn_step.cu): S = 128, conv width 4, 1 <= T <= 4;
// every buffer contiguous and 16-byte aligned.
struct GdnStepParams {
    const float* qkv;                // [T][qkv_ld]: q heads, k heads, v heads
    int64_t qkv_ld;
    float* conv_state;               // [K][conv_ld] conv state slots
    int64_t conv_ld;
    const float* conv_w;             // [ch][4]
    const float* beta_raw;           // [T][H_v]
    const float* alpha;              // [T][H_v]
    const float* dt_bias;            // [H_v]
    const float* a;                  // [H_v]
    float* state;                    // [H_v][S][S] f32, transposed; slot 0 in place
    char* snap;                      // slots 1..K-1 of snap_type (0 f32, 1 f16, 2 bf16)
    int64_t snap_stride;             // bytes
    int snap_type;
    const float* z;                  // [T][H_v][S]
    const float* norm_w;             // [S]
    float* out;                      // [T][H_v][S]
    int* sync;                       // [H_k] counters, zero between calls
    int T, H_k, H_v, K;
    float l2_eps, inv_sqrt_s, eps;
    int* err;                        // device error word
    uint64_t wait_ns;                // budget of the bounded wait for the cluster's partial sums
};
cudaError_t launch_gdn_step(const GdnStepParams& p, cudaStream_t stream);

int* device_error_word();  // address of the current device's error word (null on failure)

// kb_flash_attn_ext with caller-chosen scratch, and its scratch size (shared by the C-ABI entry points)
kb_status flash_attn_with_scratch(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* mask,
                                  const kb_fa_params* params, const kb_tensor* dst, void* scratch, size_t scratch_bytes,
                                  void* stream);
size_t flash_attn_scratch_bytes(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_fa_params* params);
// the least scratch with which kb_flash_attn_ext runs these operands (the streaming kernel's split partials); the
// preferred size above can be larger (the f16 view for prefill over a quantised cache)
size_t flash_attn_min_scratch_bytes(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v,
                                    const kb_fa_params* params);

}  // namespace kb
