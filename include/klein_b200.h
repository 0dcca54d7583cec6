/*
 * klein_b200 — B200 (sm_100a) kernels for klein's qwen35 attention hot path, behind a C ABI.
 *
 * The entry points keep the semantics of the ggml operator nodes klein's graph builds
 * (reference: src/graph.cpp:87-191), so a patched ggml-cuda backend can forward those nodes here
 * (the switch in third_party/ggml/src/ggml-cuda/ggml-cuda.cu:2488-2504). Tensors are described the
 * way ggml describes them: ne[0] is the innermost extent, nb[i] the byte stride of dimension i, data a
 * device pointer. All calls are asynchronous on the given CUDA stream, allocate nothing, do not
 * synchronise, and may be captured into a CUDA graph. Scratch memory, where a call needs it, comes from
 * the caller (as ggml-cuda's pool provides it, ggml-cuda.cu:925-926).
 *
 * Errors: ggml aborts (GGML_ASSERT); this library returns a kb_status instead and leaves the outputs
 * untouched when it rejects a call. A ggml-side shim turns a non-OK status into GGML_ABORT.
 */
#ifndef KLEIN_B200_H
#define KLEIN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum kb_status {
    KB_OK = 0,
    KB_ERR_ARG = 1,          /* null pointer or inconsistent argument */
    KB_ERR_BAD_SHAPE = 2,    /* shapes or strides that the op does not define */
    KB_ERR_UNSUPPORTED = 3,  /* a valid ggml configuration this library does not implement */
    KB_ERR_SCRATCH = 4,      /* scratch buffer missing or too small */
    KB_ERR_CUDA = 5,         /* a CUDA runtime/driver call failed */
    KB_ERR_TIMEOUT = 6       /* a bounded device-side wait ran out (see kb_device_error) */
} kb_status;

/* Element types, numbered as enum ggml_type (third_party/ggml/include/ggml.h:389-420). */
enum {
    KB_TYPE_F32 = 0,
    KB_TYPE_F16 = 1,
    KB_TYPE_Q4_0 = 2, /* blocks of 32: f16 scale d then 16 bytes of 4-bit values (ggml-common.h block_q4_0) */
    KB_TYPE_Q8_0 = 8, /* blocks of 32: f16 scale d then 32 int8 (ggml-common.h block_q8_0) */
    KB_TYPE_I32 = 26,
    KB_TYPE_I64 = 27,
    KB_TYPE_BF16 = 30
};

/* A strided device tensor in ggml's conventions (struct ggml_tensor's type/ne/nb/data, ggml.h). */
typedef struct kb_tensor {
    int32_t type;
    int64_t ne[4];
    size_t nb[4];
    void* data;
} kb_tensor;

/*
 * Parameters of GGML_OP_FLASH_ATTN_EXT. scale/max_bias/logit_softcap are the op_params set by
 * ggml_flash_attn_ext (third_party/ggml/src/ggml.c:5540-5541); prec is ggml_prec_set_acc's value
 * (this library always accumulates in f32, which satisfies every precision request).
 *
 * Analytic visibility (used only when the dense mask is NULL and causal != 0) states klein's mask rule
 * (src/engine.cpp:308-326) without materialising the n_kv x n_q f16 mask: query i sits at position
 * pos0 + i; with ring == 0 it sees cell j iff kv_lo <= j <= pos0 + i; with ring > 0 (the MTP head's
 * sliding-window ring buffer) slot j holds cell c = end - ((end - j) mod ring), end = pos0 + n_q - 1,
 * and is visible iff kv_lo <= c <= pos0 + i and c > pos0 + i - ring.
 */
typedef struct kb_fa_params {
    float scale;
    float max_bias;
    float logit_softcap;
    int32_t prec;
    int32_t causal;
    int64_t pos0;
    int64_t kv_lo;
    int64_t ring;
} kb_fa_params;

/*
 * GGML_OP_FLASH_ATTN_EXT (ggml_flash_attn_ext, ggml.h:2476-2495; CPU semantics ops.cpp:8842-9574;
 * replaces ggml_cuda_flash_attn_ext, ggml-cuda/fattn.cu:758-772).
 *   q    f32  [D, n_q, H, ne3]       any byte strides (klein passes a permuted view, graph.cpp:118)
 *   k, v f16/bf16/q8_0/q4_0 [D, n_kv, H_kv, ne3k]  nb[0] = element size (block size 34 for q8_0, 18 for q4_0);
 *                                    H % H_kv == 0,
 *                                    ne3 % ne3k == 0; base and nb[1..3] multiples of 16 bytes
 *   mask f16  [n_kv, >= n_q, ne32, ne33] contiguous, or NULL; broadcast over heads as in ggml
 *   dst  f32  [D, H, n_q, ne3]       ("permuted" result); nb[0] = 4
 * Head h reads KV head h / (H / H_kv). A row whose every cell is masked produces zeros.
 * scratch: device memory of at least kb_flash_attn_ext_scratch_bytes(...) bytes (may be NULL when that
 * is 0). Supported here: D = 256, K and V of the same type (f16, bf16, q8_0 or q4_0; bf16 for n_q >= 128 only).
 * Over a q8_0 or q4_0 cache Q is rounded to q8_0 first (the vec_dot type of both in ggml's CPU backend).
 * Kernels: n_q >= 128 (prompt chunks) runs the tensor-core prefill kernel. Over a q8_0 / q4_0 cache it first
 * widens the cells the queries can see into an f16 copy in the scratch (as ggml-cuda converts K and V to f16
 * for its MMA kernel, fattn-common.cuh:1031-1090); given less scratch than kb_flash_attn_ext_scratch_bytes
 * asks for but enough for the split partials, such a call runs on the streaming kernel instead (same result
 * within the parity bound, slower). Fewer query tokens (decode, the verify step), the MTP ring and
 * kb_flash_attn_ext_partial run the streaming kernel.
 */
kb_status kb_flash_attn_ext(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* mask,
                            const kb_fa_params* params, const kb_tensor* dst, void* scratch, size_t scratch_bytes,
                            void* stream);

/*
 * The same attention over one contiguous part of the KV sequence, leaving the result unnormalised so that
 * parts computed on different GPUs can be merged (the per-chunk partials of ggml's split-KV path,
 * ops.cpp:9489-9520, written out for a cross-device merge):
 *   o_part  f32 [D, H, n_q, ne3] (dst's layout): sum_j 2^(s_j - m) v_j over this part's visible cells
 *   ml_part f32 [ne3][n_q][H][2] contiguous: (m, l) with m the row maximum of s_j = score * log2(e) and
 *           l = sum_j 2^(s_j - m); l == 0 marks a row with no visible cell in this part
 * Causal/ring bounds in params are in the coordinates of this part's cells (cell 0 = its first cell).
 */
kb_status kb_flash_attn_ext_partial(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* mask,
                                    const kb_fa_params* params, const kb_tensor* o_part, float* ml_part, void* scratch,
                                    size_t scratch_bytes, void* stream);

/*
 * Log-sum-exp merge of n_parts partials (generalises flash_attn_combine_results, ggml-cuda/fattn-common.cuh:924-978,
 * and ggml_flash_attn_ext_reduce_partials, ggml-cpu/ops.cpp:9370-9438, to parts from several devices):
 *   part p's o at o_parts + p * part_stride: f32 [rows][head_dim]; its (m, l) at ml_parts + p * part_stride:
 *   f32 [rows][2] (as written by kb_flash_attn_ext_partial; rows = ne3 * n_q * H in dst order; part_stride in
 *   floats, so one all-gathered buffer of [o | ml] per part can be passed as is); dst f32 [rows][head_dim]
 *   dst[r] = sum_p 2^(m_p - M) o_p[r] / sum_p 2^(m_p - M) l_p[r], M = max over parts with l_p > 0; 0 if none.
 * Requires 1 <= n_parts <= 1024, head_dim % 8 == 0, part_stride % 4 == 0, o_parts 16-byte aligned.
 */
kb_status kb_lse_combine(const float* o_parts, const float* ml_parts, int64_t part_stride, int32_t n_parts, int64_t rows,
                         int32_t head_dim, float* dst, void* stream);

/*
 * Exchange of the split partials between GPUs over NVLink without a collective library (the all-gather step of
 * the KV-sequence split; ggml's split-KV exchanges them between CPU threads, ops.cpp:9489-9520, and has no
 * multi-GPU counterpart). One process per GPU; every rank holds
 *   a gather buffer  two slot sets of n_ranks packed partials (slot_set_floats >= n_ranks * part_floats each)
 *   a flag array     int32 [n_ranks + 2], zero at start: one arrival count per source rank, then this rank's
 *                    epoch counter and a completion counter used by the merge
 * both from kb_peer_alloc (zeroed device memory with a 64-byte CUDA IPC handle); kb_peer_open maps another
 * process's buffer from its handle (peer access over NVLink), kb_peer_close unmaps, kb_peer_free releases.
 *   kb_partials_push     writes `part` (this rank's packed partial, part_floats floats, 16-byte aligned) into slot
 *                        `rank` of slot set (e & 1) of every rank's gather buffer, e = this rank's counter + 1, in
 *                        32 chunks per destination; each chunk then adds 1 to flags[r][rank] of its destination r
 *                        with system-scope release, so a complete push of exchange e leaves 32 e there. gather /
 *                        flags: host arrays of n_ranks (<= KB_MAX_PEERS) device pointers, this rank's own buffers
 *                        included.
 *   kb_lse_combine_wait  waits until every source's count in this rank's flag array reaches 32 (counter + 1) (gives up
 *                        after 1 s and sets the device error word), merges that slot set of this rank's gather
 *                        buffer like kb_lse_combine (parts at gather + p * part_stride, (m, l) after the rows * D
 *                        output floats), and advances the counter.
 * The epochs live in device memory, so both calls can be captured in a CUDA graph and replayed. A rank runs at most
 * one exchange ahead of the slowest rank, so the two slot sets never hold data still being merged.
 */
#define KB_IPC_HANDLE_BYTES 64
#define KB_MAX_PEERS 16
kb_status kb_peer_alloc(size_t bytes, void** dev_ptr, void* ipc_handle);
kb_status kb_peer_open(const void* ipc_handle, void** dev_ptr);
kb_status kb_peer_close(void* dev_ptr);
kb_status kb_peer_free(void* dev_ptr);
kb_status kb_partials_push(const float* part, int64_t part_floats, float* const* gather, int64_t slot_set_floats,
                           int32_t* const* flags, int32_t rank, int32_t n_ranks, void* stream);
kb_status kb_lse_combine_wait(const float* gather, int64_t part_stride, int64_t slot_set_floats, int32_t n_parts,
                              int64_t rows, int32_t head_dim, int32_t* flags, float* dst, void* stream);

/*
 * kb_flash_attn_ext_partial and kb_partials_push in one call: the split combine of this rank's partial attention
 * writes every merged row (o unnormalised, m, l) straight into slot `rank` of every rank's gather buffer, in the
 * packed layout kb_partials_push uses (o [n_q * H][D], then (m, l) [n_q * H][2]; part_floats >= n_q * H * (D + 2),
 * a multiple of 4), and its last CTA counts the exchange in every rank's flags exactly as a push does; the next
 * call on this rank is kb_lse_combine_wait. Operands as kb_flash_attn_ext_partial (ne3 = 1, at least one cell);
 * scratch of kb_flash_attn_ext_push_scratch_bytes bytes.
 */
size_t kb_flash_attn_ext_push_scratch_bytes(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v,
                                            const kb_fa_params* params);
kb_status kb_flash_attn_ext_push(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* mask,
                                 const kb_fa_params* params, int64_t part_floats, float* const* gather,
                                 int64_t slot_set_floats, int32_t* const* flags, int32_t rank, int32_t n_ranks,
                                 void* scratch, size_t scratch_bytes, void* stream);

/*
 * The whole sequence-split attention of one layer on this rank in ONE launch: the partial attention over this
 * rank's cells, then, inside the same kernel (a cooperative launch, every CTA resident), the merge of its splits,
 * stores of the merged rows into slot `rank` of every rank's gather buffer over NVLink, a per-slot release flag in
 * every rank's flag array, a bounded wait for the same slots from every rank and the final log-sum-exp merge into
 * dst (with klein's output gate when gate != NULL, as kb_flash_attn_ext_gated). Replaces kb_flash_attn_ext_partial +
 * kb_partials_push + kb_lse_combine_wait (ggml's split-KV partials and reduce, ops.cpp:9489-9520, 9370-9438,
 * across devices).
 *   q, k, v, mask, params  as kb_flash_attn_ext_partial (causal / ring bounds in this rank's cell coordinates; ne3 = 1,
 *                          at least one cell); every rank passes the same n_q and heads
 *   gather, slot_set_floats, part_floats  as kb_partials_push (two slot sets of n_ranks packed partials per rank)
 *   flags   per rank an int32 array of kb_exchange_flag_bytes(n_ranks) bytes, zero at start (kb_peer_alloc); its
 *           first n_ranks + 2 words are the push / wait exchange's, so both can share one array
 *   dst     f32 [D, H, n_q, 1], rows 16-byte aligned; scratch of kb_flash_attn_ext_push_scratch_bytes bytes
 * Returns KB_ERR_UNSUPPORTED when the split plan needs more CTAs than the GPU has SMs or n_q * H exceeds 512
 * rows. A wait that runs out (a rank that never arrives) sets the device error word after
 * 1 s; the call returns without hanging. Captured in a CUDA graph, successive replays advance the device-side epoch.
 */
size_t kb_exchange_flag_bytes(int32_t n_ranks);
kb_status kb_flash_attn_ext_exchange(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* mask,
                                     const kb_fa_params* params, const kb_tensor* gate, int64_t part_floats,
                                     float* const* gather, int64_t slot_set_floats, int32_t* const* flags, int32_t rank,
                                     int32_t n_ranks, const kb_tensor* dst, void* scratch, size_t scratch_bytes,
                                     void* stream);

/* 1 when kb_flash_attn_ext accepts these operands (shapes, types, strides, params; data pointers may still be NULL,
 * as in ggml-cuda's supports_op, ggml-cuda.cu:5775-5776), 0 otherwise. Alignment of the data pointers themselves and
 * of dst are checked by the call. */
int32_t kb_flash_attn_ext_supported(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* mask,
                                    const kb_fa_params* params);

/* Scratch needed by kb_flash_attn_ext / kb_flash_attn_ext_partial for these operands on the current
 * device (the role of ggml_cuda_flash_attn_ext_get_alloc_size, fattn.cu:722-756): the split partials of the
 * streaming kernel (at most SM count x 32 rows x (256 + 2) x 4 bytes, ~4.9 MB on a 148-SM B200) and, for
 * n_q >= 128 over a q8_0 / q4_0 cache, the two f16 views (ne3 x n_kv x H_kv x 1,024 bytes). */
size_t kb_flash_attn_ext_scratch_bytes(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v,
                                       const kb_fa_params* params);

/*
 * GGML_OP_GATED_DELTA_NET (ggml_gated_delta_net, ggml.h:2639-2660; CPU semantics ops.cpp:11123-11275;
 * replaces ggml_cuda_op_gated_delta_net, ggml-cuda/gated_delta_net.cu:320-327), recurrent form.
 *   q, k  f32 [S, H_k, T, n_seqs_q/k]   rows contiguous (klein's L2-normalised views of the conv output)
 *   v     f32 [S, H_v, T, n_seqs]       value head h reads q/k head h % H_k
 *   g     f32 [1, H_v, T, n_seqs] (scalar log-decay) or [S, H_v, T, n_seqs] (per-channel, "KDA"), contiguous
 *   beta  f32 [1, H_v, T, n_seqs] contiguous
 *   state f32 [S, S, H_v, n_seqs] contiguous: s0, stored transposed (element (i, j) = S[j][i])
 *   dst   f32 [S*H_v, T*n_seqs + K*S*n_seqs] contiguous: attention output [S, H_v, T, n_seqs], then K state slots
 *         [S, S, H_v, n_seqs] most recent first (slot s = state s tokens before the end); only slots < min(T, K)
 *         are written.
 *   scratch  optional device memory (16-byte aligned). Calls with T - min(T, K) + 1 >= 64 tokens and the scalar
 *         gate run the chunked tensor-core form (64-token chunks) when scratch holds at least one chunk's records
 *         for every head (n_seqs * H_v * 65,792 bytes); kb_gated_delta_net_scratch_bytes gives the size for one
 *         pass, less runs several passes. Without scratch, or for the per-channel gate, the recurrent kernel
 *         processes every token (same results within the stated tolerance, slower for long prompts).
 * Supported here: S = 128; every pointer and row stride 16-byte aligned.
 */
kb_status kb_gated_delta_net(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* g,
                             const kb_tensor* beta, const kb_tensor* state, int32_t K, const kb_tensor* dst,
                             void* scratch, size_t scratch_bytes, void* stream);

/*
 * The same recurrence writing straight into klein's recurrent-state cache, i.e. ggml_gated_delta_net followed
 * by klein's two copies (graph.cpp:169-184) in one kernel:
 *   state  f32 [S, S, H_v, n_seqs]: read as s0, then overwritten with slot 0 (the state after the last token)
 *   snap   [S*S*H_v*n_seqs, >= min(T,K)-1] rows of f16, bf16 or f32 (klein's ssm_snap, state.cpp:74-78):
 *          slot s (1 <= s < min(T, K)) goes to row s-1, converted with round-to-nearest-even; may be NULL when
 *          min(T, K) == 1
 *   attn   f32 [S, H_v, T, n_seqs] attention output (any row strides)
 *   scratch as for kb_gated_delta_net
 */
kb_status kb_gated_delta_net_cache(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* g,
                                   const kb_tensor* beta, const kb_tensor* state, const kb_tensor* snap, int32_t K,
                                   const kb_tensor* attn, void* scratch, size_t scratch_bytes, void* stream);

/* Scratch for one pass of the chunked DeltaNet form over these operands (v: [S, H_v, T, n_seqs], g: the gate);
 * 0 when the call would not use it (short T, per-channel gate). A ggml-cuda shim takes it from the backend's
 * pool (ggml_cuda_pool_alloc), as launch_fattn does for its partials (fattn-common.cuh:1019-1021). */
size_t kb_gated_delta_net_scratch_bytes(const kb_tensor* v, const kb_tensor* g, int32_t K);

/*
 * State::rollback_recurrent (state.cpp:162-183): after s rejected draft tokens, for each of n_layers DeltaNet
 * layers, conv slot s -> conv slot 0 (f32, conv [n_snapshots][conv_row]) and snapshot row s-1 (snap_type f16,
 * bf16 or f32, snap [n_snapshots-1][ssm_row]) -> the f32 state ssm [ssm_row]; the restored state equals the
 * snapshot exactly. s == 0 is a no-op; 1 <= s < n_snapshots. The pointer arrays are host arrays of device
 * pointers (n_layers <= 64), replacing the per-layer ggml_cpy graph with one launch.
 */
kb_status kb_rollback_recurrent(int32_t n_layers, float* const* conv, int64_t conv_row, const void* const* snap,
                                int32_t snap_type, float* const* ssm, int64_t ssm_row, int32_t s, int32_t n_snapshots,
                                void* stream);

/*
 * ggml_set_rows (ops.cpp:5446-5500; replaces ggml-cuda/set-rows.cu:8-110), klein's KV-cache write
 * (graph.cpp:111-112): dst row idx[r] <- src row r for every (i2, i3), converted to dst's type.
 *   dst f32 / f16 / bf16 / q8_0 / q4_0 [ne0, n_rows, ne2, ne3]; src f32 [ne0, n_src, ne2, ne3] (rows
 *   contiguous); idx i64 or i32 [n_src, ne11, ne12] broadcast over ne2 % ne11, ne3 % ne12. ne0 % 32 == 0.
 *   q8_0 rounding is quantize_row_q8_0_ref's (ggml-quants.c:276-299), q4_0 quantize_row_q4_0_ref's
 *   (ggml-quants.c:113-148: the first value of largest magnitude sets d = max / -8), bit for bit.
 * An out-of-range index (ggml asserts) skips that row and sets the device error word (kb_device_error).
 */
kb_status kb_set_rows(const kb_tensor* dst, const kb_tensor* src, const kb_tensor* idx, void* stream);

/*
 * kb_flash_attn_ext followed by klein's output gate (graph.cpp:124: ggml_mul(o, ggml_sigmoid(gate))), fused into the
 * attention's final store: dst = o * 1 / (1 + expf(-gate)). gate f32 [D, H, n_q, ne3] (klein's contiguous gate
 * [D * H, n_q], e.g. kb_attn_prologue's gate_out), nb[0] = 4. Scratch as for kb_flash_attn_ext
 * (kb_flash_attn_ext_scratch_bytes).
 */
kb_status kb_flash_attn_ext_gated(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* mask,
                                  const kb_fa_params* params, const kb_tensor* gate, const kb_tensor* dst, void* scratch,
                                  size_t scratch_bytes, void* stream);

/*
 * The attention prologue of klein's Builder::attention (src/graph.cpp:94-112) in one launch: the q / gate split of
 * the interleaved query projection, ggml_rms_norm(eps) * q_norm / k_norm on every head row, ggml_rope_multi on q and
 * k, ggml_cont of the gate, and ggml_set_rows of the K and V rows into the caches. Operands (ggml ne / nb):
 *   qfull  f32 [2 hd nh, n] (per head: hd query values then hd gate values), rows of nb[1] bytes
 *   kcur, vcur  f32 [hd nkv, n]            pos  i32 [4 n] (section-major: t..., h..., w..., extra...)
 *   kv_idx i64 [n] (cache cell of each token)              q_norm, k_norm  f32 [hd]
 *   q_out  f32 [hd, nh, n] contiguous      gate_out  f32 [hd nh, n] contiguous
 *   k_cache, v_cache  f16, q8_0 or q4_0 [hd nkv, n_cells] (klein's cache rows)
 * hd is 64, 128 or 256; rope->n_rot a multiple of 64, at most hd. A kv_idx outside [0, n_cells) skips that row
 * and sets the device error word.
 */
typedef struct kb_rope_params {
    int32_t n_rot;       /* rotated dims (the first n_rot of each head) */
    int32_t sections[4]; /* M-RoPE sections: pairs per position component (t, h, w, extra) */
    int32_t mode;        /* 40 = GGML_ROPE_TYPE_IMROPE (interleaved sections, qwen35) or 8 = GGML_ROPE_TYPE_MROPE */
    float freq_base;     /* theta base */
    float freq_scale;    /* 1 for qwen35 */
    float attn_factor;   /* 1 for qwen35 (YaRN extrapolation is not supported: ext_factor 0) */
} kb_rope_params;
kb_status kb_attn_prologue(const kb_tensor* qfull, const kb_tensor* kcur, const kb_tensor* vcur, const kb_tensor* pos,
                           const kb_tensor* kv_idx, const kb_tensor* q_norm, const kb_tensor* k_norm, float rms_eps,
                           const kb_rope_params* rope, const kb_tensor* q_out, const kb_tensor* gate_out,
                           const kb_tensor* k_cache, const kb_tensor* v_cache, void* stream);

/*
 * The DeltaNet input side of klein's Builder::deltanet (src/graph.cpp:136-165) in one launch:
 *   beta = sigmoid(beta_raw), g = softplus(alpha + dt_bias) * a                     (the GDN gates)
 *   conv = silu(ggml_ssm_conv([conv state | qkv], conv_w))  over the kc = 4 wide window of each channel
 *   q, k = l2(conv[q heads]), l2(conv[k heads]) with l2(x) = rms_norm(x, eps / S) / sqrt(S); v = conv[v heads]
 *   conv state snapshots: slot s <- the kc - 1 inputs before token n - s (clamped at the stored state), for
 *   s < K, skipping slots s >= n other than 0 (the rollback slots of State::rollback_recurrent)
 * Operands (ggml ne): qkv f32 [ch, n], ch = 2 S H_k + S H_v (q heads, k heads, v heads); conv_state f32
 * [(kc - 1) ch, K] (slot 0 = the state, channel-major); conv_w f32 [kc, ch]; beta_raw, alpha f32 [H_v, n] or both
 * NULL (then dt_bias, a, beta_out, g_out are ignored); dt_bias, a f32 [H_v]; q_out, k_out f32 [S, H_k, n];
 * v_out f32 [S, H_v, n]; beta_out, g_out f32 [H_v, n] (the GDN op's shapes with their trailing 1s). All
 * contiguous; S is 64 or 128.
 */
kb_status kb_gdn_input(const kb_tensor* qkv, const kb_tensor* conv_state, const kb_tensor* conv_w,
                       const kb_tensor* beta_raw, const kb_tensor* alpha, const kb_tensor* dt_bias, const kb_tensor* a,
                       int32_t S, int32_t H_k, float rms_eps, const kb_tensor* q_out, const kb_tensor* k_out,
                       const kb_tensor* v_out, const kb_tensor* beta_out, const kb_tensor* g_out, void* stream);

/*
 * The DeltaNet output side (graph.cpp:186-190): dst = rms_norm(x, eps) * w * silu(z) on every [S] row.
 * x f32 [S, H, n] (GDN's attention output), z f32 [S H, n], w f32 [S], dst f32 [S H, n]; contiguous, S 64 or 128.
 */
kb_status kb_gdn_gated_norm(const kb_tensor* x, const kb_tensor* z, const kb_tensor* w, float rms_eps,
                            const kb_tensor* dst, void* stream);

/*
 * A whole DeltaNet layer of a decode / verify pass between its GEMMs (graph.cpp:136-190) in one launch, for n_tokens
 * 1..4: kb_gdn_input on the conv state slots, the recurrence into ssm (slot 0, in place) and ssm_snap (slots 1..,
 * kb_gated_delta_net_cache with K = n_snapshots) and kb_gdn_gated_norm, with bit-identical results.
 *   qkv, beta_raw, alpha, dt_bias, a, conv_w, conv_state  as kb_gdn_input (S = 128, conv width 4)
 *   ssm       f32 [S * S * H_v]; ssm_snap [S * S * H_v, n_snapshots - 1] of f32 / f16 / bf16, or null when
 *             n_snapshots is 1
 *   z, ssm_norm, out  as kb_gdn_gated_norm
 *   sync      device int32 [H_k] (kb_gdn_step_sync_bytes), zero before the first call; every call leaves it zero.
 *             Calls that share it must not run concurrently.
 * Every buffer contiguous and 16-byte aligned. KB_ERR_UNSUPPORTED for shapes outside this form
 * (the three calls above cover them).
 */
size_t kb_gdn_step_sync_bytes(int32_t H_k);
kb_status kb_gdn_step(const kb_tensor* qkv, const kb_tensor* conv_state, const kb_tensor* conv_w,
                      const kb_tensor* beta_raw, const kb_tensor* alpha, const kb_tensor* dt_bias, const kb_tensor* a,
                      const kb_tensor* ssm, const kb_tensor* ssm_snap, int32_t n_snapshots, const kb_tensor* z,
                      const kb_tensor* ssm_norm, float rms_eps, int32_t* sync, const kb_tensor* out, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * klein's per-sequence State, resident in HBM (replaces src/state.h / src/state.cpp's tensors; klein's mapped host
 * KV cache and its bulk host view, state.cpp:110-134, are not needed when the cache lives in device memory), the
 * per-pass indexing of Engine::run (engine.cpp:254-326), the accept / rollback of Engine::generate's verify step
 * (engine.cpp:584-590), and Builder::attention / Builder::deltanet (graph.cpp:87-191) bound to the state without
 * their weight GEMMs (the caller's projections feed them and consume their outputs).
 */

/* qwen35's shapes (src/model.h HParams). Layer il < n_layer is full attention iff (il + 1) % full_attn_interval
 * == 0, DeltaNet otherwise; with_mtp adds the MTP layer (index n_layer), full attention over a ring of cells. */
typedef struct kb_qwen35_dims {
    int32_t n_layer, full_attn_interval;
    int32_t n_head, n_head_kv, head_dim;
    int32_t ssm_conv_kernel, ssm_d_state, ssm_n_group, ssm_dt_rank;
    int32_t with_mtp;
} kb_qwen35_dims;

/* src/state.h StateConfig: cache types (f16, bf16, q8_0 or q4_0), recurrent slots (1 + max drafts) and their
 * snapshot type (f16, bf16 or f32), and the MTP ring's cells (min(n_ctx, mtp_window), state.cpp:17). */
typedef struct kb_state_config {
    int32_t n_ctx;
    int32_t type_k, type_v;
    int32_t n_snapshots;
    int32_t snap_type;
    int32_t mtp_window;
} kb_state_config;

typedef struct kb_state kb_state;

/* One layer's tensors (State::k / v / conv / ssm / ssm_snap): attention layers get k, v [kv_row, cells] (their
 * other fields are zero), DeltaNet layers conv [(kc - 1) * channels, n_snapshots] f32, ssm [d_state^2 * dt_rank, 1]
 * f32 and ssm_snap [d_state^2 * dt_rank, n_snapshots - 1] (data NULL when n_snapshots == 1). */
typedef struct kb_state_layer {
    kb_tensor k, v, conv, ssm, ssm_snap;
} kb_state_layer;

/* One forward pass over n_tokens cells from cell0 (Engine::run): ring (MTP only, 0 otherwise), the cells attended
 * n_kv (graph.cpp:16-19 padded_n_kv, at most the ring), and the visibility rule as analytic bounds (scale
 * 1 / sqrt(head_dim), causal, pos0 = cell0, kv_lo, ring), the same cells klein's dense mask admits. */
typedef struct kb_pass {
    int32_t n_tokens, mtp;
    int64_t cell0, kv_lo, ring, n_kv;
    kb_fa_params fa;
} kb_pass;

/* Byte counts of state_kv_bytes / state_mtp_kv_bytes / state_recurrent_bytes (state.cpp:20-35). */
kb_status kb_state_sizes(const kb_qwen35_dims* dims, const kb_state_config* cfg, size_t* kv_bytes,
                         size_t* mtp_kv_bytes, size_t* recurrent_bytes);
/* State::State: one device allocation on the current device, zeroed; kb_state_destroy frees it. */
kb_status kb_state_create(const kb_qwen35_dims* dims, const kb_state_config* cfg, kb_state** out);
/* The same inside the caller's device memory (e.g. a ggml backend buffer, as klein's State allocates its tensors),
 * at least kb_state_required_bytes bytes, 256-byte aligned, zeroed here; kb_state_destroy then frees nothing. */
size_t kb_state_required_bytes(const kb_qwen35_dims* dims, const kb_state_config* cfg);
kb_status kb_state_create_in(const kb_qwen35_dims* dims, const kb_state_config* cfg, void* base, size_t bytes,
                             kb_state** out);
kb_status kb_state_destroy(kb_state* state);
size_t kb_state_device_bytes(const kb_state* state);
kb_status kb_state_get_layer(const kb_state* state, int32_t il, kb_state_layer* out);
/* State::n_past / n_past_mtp (mtp != 0). */
int64_t kb_state_n_past(const kb_state* state, int32_t mtp);
kb_status kb_state_set_n_past(kb_state* state, int32_t mtp, int64_t n_past);
/* State::clear (state.cpp:148-160): recurrent states and snapshots to zero, n_past = n_past_mtp = 0. */
kb_status kb_state_clear(kb_state* state, void* stream);
/* State::rollback_recurrent (state.cpp:162-183): slot s -> current, every DeltaNet layer, one launch. */
kb_status kb_state_rollback(kb_state* state, int32_t s, void* stream);
/* Engine::run's pass indexing; kv_idx (host, n_tokens entries, may be NULL) receives each token's cache row
 * ((cell0 + i) mod ring for the MTP layer). Fails with KB_ERR_ARG when the pass does not fit the context. */
kb_status kb_plan_pass(const kb_qwen35_dims* dims, const kb_state_config* cfg, int32_t mtp, int32_t n_tokens,
                       int64_t cell0, int64_t kv_lo, kb_pass* out, int64_t* kv_idx);
/* the same from the state's n_past (or n_past_mtp) */
kb_status kb_state_plan_pass(const kb_state* state, int32_t mtp, int32_t n_tokens, int64_t kv_lo, kb_pass* out,
                             int64_t* kv_idx);
/* After a verify pass of n_batch cells from base: n_past = base + accepted + 1, and the DeltaNet states roll back
 * past the (n_batch - 1 - accepted) rejected drafts (Engine::generate, engine.cpp:584-590). */
kb_status kb_state_accept(kb_state* state, int64_t base, int32_t n_batch, int32_t accepted, void* stream);

/*
 * Builder::attention without its GEMMs (graph.cpp:94-124) for attention layer il (or the MTP layer, pass->mtp): the
 * prologue (q / gate split, Q / K RMS norms, M-RoPE, K and V rows written into the state's cache at kv_idx) and the
 * gated flash attention over pass->n_kv cells. qfull, kcur, vcur, pos, kv_idx, q_norm, k_norm and rope as
 * kb_attn_prologue (kv_idx: device copy of kb_plan_pass's); out f32 [head_dim * n_head, n_tokens] contiguous (the
 * input of wo). scratch: kb_layer_attention_scratch_bytes bytes, 256-byte aligned (the prologue's Q and gate, then the
 * attention's scratch).
 */
size_t kb_layer_attention_scratch_bytes(const kb_state* state, int32_t il, const kb_pass* pass);
kb_status kb_layer_attention(kb_state* state, int32_t il, const kb_pass* pass, const kb_tensor* qfull,
                             const kb_tensor* kcur, const kb_tensor* vcur, const kb_tensor* pos, const kb_tensor* kv_idx,
                             const kb_tensor* q_norm, const kb_tensor* k_norm, float rms_eps, const kb_rope_params* rope,
                             const kb_tensor* out, void* scratch, size_t scratch_bytes, void* stream);

/*
 * Builder::deltanet without its GEMMs (graph.cpp:134-190) for DeltaNet layer il: kb_gdn_input on the state's conv
 * slots, the recurrence into the state's ssm and snapshot rows (kb_gated_delta_net_cache with K = n_snapshots), and
 * the gated RMS norm. qkv, beta_raw, alpha, dt_bias, a, conv_w as kb_gdn_input; z and ssm_norm as kb_gdn_gated_norm;
 * out f32 [d_state * dt_rank, n_tokens] (the input of ssm_out). scratch: kb_layer_deltanet_scratch_bytes bytes,
 * 256-byte aligned (q, k, v, beta, g, the attention rows, then the chunked form's records for long passes).
 */
size_t kb_layer_deltanet_scratch_bytes(const kb_state* state, int32_t il, int32_t n_tokens);
kb_status kb_layer_deltanet(kb_state* state, int32_t il, int32_t n_tokens, const kb_tensor* qkv, const kb_tensor* z,
                            const kb_tensor* beta_raw, const kb_tensor* alpha, const kb_tensor* dt_bias,
                            const kb_tensor* a, const kb_tensor* conv_w, const kb_tensor* ssm_norm, float rms_eps,
                            const kb_tensor* out, void* scratch, size_t scratch_bytes, void* stream);

/*
 * Size of the device buffer built into the library for kb_flash_attn_ext_noalloc (per GPU, held from the
 * library's load until the process exits).
 */
#define KB_NOALLOC_SCRATCH_BYTES (8u << 20)

/*
 * kb_flash_attn_ext for callers that cannot allocate device memory: code running while a CUDA graph is
 * being captured (no cudaMalloc there), hosts that give the whole GPU to their own memory pools up front,
 * and foreign-language bindings that pass raw pointers but have no device allocator. Same operands,
 * semantics and errors as kb_flash_attn_ext, but the split-KV partials live in a fixed buffer of
 * KB_NOALLOC_SCRATCH_BYTES compiled into the library, so the call itself allocates nothing.
 *   - A call that would need more partials than the buffer holds returns KB_ERR_SCRATCH. The split
 *     partials never exceed SM count x 32 rows x (256 + 2) x 4 bytes (~4.9 MB on a 148-SM B200, e.g.
 *     262,144 cells x 4 tokens x 24/4 heads). Prompt-length calls over a q8_0 / q4_0 cache, whose f16
 *     views do not fit, run on the streaming kernel.
 *   - Every call looks up the buffer's device address (cudaGetSymbolAddress once per device, cached);
 *     make the first call on a device before any stream capture on that device. The cache assumes each
 *     device's primary context for the life of the process (no cudaDeviceReset in between).
 *   - All calls on a device share the buffer: calls that overlap on the GPU (other streams, other host
 *     threads) race on it and must be serialised by the caller. Nothing in it needs clearing between calls.
 * This entry point has no counterpart in the reference (ggml-cuda always draws scratch from its pool).
 */
kb_status kb_flash_attn_ext_noalloc(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* mask,
                                    const kb_fa_params* params, const kb_tensor* dst, void* stream);

/* Device-side error word of the current device: the code of the last bounded wait that ran out
 * (0 = none). clear != 0 resets it. Synchronous (reads device memory). */
kb_status kb_device_error(int32_t* code, int clear);

/* Library version string. */
const char* kb_version(void);

#ifdef __cplusplus
}
#endif

#endif /* KLEIN_B200_H */
