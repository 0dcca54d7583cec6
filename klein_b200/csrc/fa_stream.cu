// Split-KV streaming attention for decode (1 query token) and the MTP verify step (a few tokens):
// GGML_OP_FLASH_ATTN_EXT with few query rows over a long KV cache, on the 5th-generation tensor cores.
// HBM-bound: every K/V byte is read once, by TMA, and consumed by tcgen05 MMAs.
//
// Work split. One CTA per (KV split, KV head, row chunk). The rows of a KV head are its n_q * gqa query
// rows (query i, head-in-group g -> row i*gqa + g); a chunk of up to 16 or 32 of them forms the N columns of
// S^T = K Q^T over 128-cell blocks (M = 128), so each K/V byte reaches the tensor core once per CTA. Per-split
// partials (o, m, l) merge in a second kernel (the combine of ggml's ops.cpp:9370-9438 /
// fattn-common.cuh:924-978). The kernel, its roles and the softmax scheme are described at namespace tc.
//
// f16 cache: TMA writes K blocks and V tiles straight into the swizzled layouts the MMAs read.
// q8_0 / q4_0 cache: TMA brings the raw 34- or 18-byte blocks (ggml-common.h block_q8_0, block_q4_0),
// dequantisation warps widen K into TMEM and V into shared memory. Q is quantised to q8_0 as ggml quantises it for
// a q8_0 or q4_0 K (both have q8_0 as their vec_dot type; quantize_row_q8_0_ref, ggml-quants.c:276-299) and
// widened to f16(q * d).
//
// Semantics follow ggml_compute_forward_flash_attn_ext_f16_one_chunk (ops.cpp:8842-9078): Q is rounded to
// the K dot type (f16 for f16 K, q8_0 for q8_0 and q4_0 K, :8960), scores are scaled, soft-capped, masked (-inf
// cells skipped), and a row with no visible cell yields zeros (:9066). Accumulation is f32 throughout.
#include "kb_common.cuh"
#include "kb_internal.h"
#include "kb_tcgen05.cuh"

namespace kb {

namespace {

constexpr float LOG2E = 1.4426950408889634f;
constexpr int D = FA_D;
constexpr int TILE = FA_TILE;
constexpr int KTILE_F16 = TILE * D * 2;        // 32 KiB: 4 boxes of [64 cells][64 dims] f16, 128B-swizzled
constexpr int QROW = D / 32 * 34;              // bytes of one head's row in a q8_0 cache (272)
constexpr int Q4ROW = D / 32 * 18;             // bytes of one head's row in a q4_0 cache (144)

__device__ __forceinline__ float slope_of(const FaStreamParams& p, int h) {
    if (p.max_bias <= 0.0f) return 1.0f;
    return h < p.n_head_log2 ? powf(p.m0, (float) (h + 1)) : powf(p.m1, (float) (2 * (h - p.n_head_log2) + 1));
}

// score of one (key, row) pair in log2 units, or -inf when the cell is not visible
__device__ __forceinline__ float masked_score(const FaStreamParams& p, float x, int64_t key, int qi, int h, int b,
                                              float slope) {
    float v = p.has_softcap ? p.softcap_log2 * tanhf(x * p.scale_sc) : x * p.scale_log2;
    if (key >= p.n_kv || qi >= p.n_q) return -INFINITY;
    if (p.causal) {
        const int64_t pos = p.pos0 + qi;
        int64_t c = key;
        if (p.ring > 0) {
            const int64_t end = p.pos0 + p.n_q - 1;
            c = end - (((end - key) % p.ring) + p.ring) % p.ring;
            if (c <= pos - p.ring) return -INFINITY;
        }
        if (c < p.kv_lo || c > pos) return -INFINITY;
    }
    if (p.mask) {
        const __half mh = *reinterpret_cast<const __half*>(p.mask + key * 2 + qi * p.m_nb1 + (h % p.m_ne2) * p.m_nb2 +
                                                           (b % p.m_ne3) * p.m_nb3);
        const float mv = slope * __half2float(mh);
        if (mv == -INFINITY) return -INFINITY;
        v += mv * LOG2E;
    }
    return v;
}

// final store of one output element: normalised, or (o, m, l) partial for a cross-device combine
// klein's attention output gate (graph.cpp:124): o * sigmoid(gate), ggml_vec_sigmoid_f32's 1 / (1 + expf(-x))
__device__ __forceinline__ float gate_sigmoid(const char* g) {
    return 1.0f / (1.0f + expf(-*reinterpret_cast<const float*>(g)));
}

__device__ __forceinline__ void store_row(const FaStreamParams& p, int qi, int h, int b, int d, float O, float M, float L) {
    float* dst = reinterpret_cast<float*>(p.dst + (int64_t) d * 4 + h * p.d_nb1 + qi * p.d_nb2 + b * p.d_nb3);
    if (p.partial_out) {
        *dst = O;
        if (d == 0) {
            float* ml = p.dst_ml + (((int64_t) b * p.n_q + qi) * p.n_head + h) * 2;
            ml[0] = M;
            ml[1] = L;
        }
    } else {
        float o = L > 0.0f ? O / L : 0.0f;
        if (p.gate) o *= gate_sigmoid(p.gate + (int64_t) d * 4 + h * p.g_nb1 + qi * p.g_nb2 + b * p.g_nb3);
        *dst = o;
    }
}

// ------------------------------------------------------------------------------------------------ merges

// Merge of n partial results (o_s, m_s, l_s) of one row by one 256-thread block:
// out = sum_s 2^(m_s - M) o_s / sum_s 2^(m_s - M) l_s with M = max over parts with l_s > 0 (0 if none).
// The (m, l) pairs are reduced across the block, then warp w accumulates parts w, w+8, ... with every lane
// holding 8 consecutive dims (two float4 loads per part, all in flight), and the 8 warp sums meet in smem.
constexpr int MERGE_THREADS = 256;
constexpr int MERGE_MAX_PARTS = 1024;

__device__ void merge_row(const float* __restrict__ o, int64_t o_stride, const float* __restrict__ ml, int64_t ml_stride,
                          int n, int Dd, float* __restrict__ out_row, float* __restrict__ ml_out,
                          const char* __restrict__ gate_row = nullptr) {
    __shared__ float f[MERGE_MAX_PARTS];
    __shared__ float red[MERGE_THREADS / 32];
    __shared__ float acc_s[MERGE_THREADS / 32][256 + 4];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // block max of m over parts with l > 0
    float mx = -INFINITY;
    for (int s = tid; s < n; s += MERGE_THREADS) {
        const float l = ml[s * ml_stride + 1];
        if (l > 0.0f) mx = fmaxf(mx, ml[s * ml_stride]);
    }
    for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    float M = red[0];
    for (int wi = 1; wi < MERGE_THREADS / 32; ++wi) M = fmaxf(M, red[wi]);
    __syncthreads();
    // weights and the weighted sum of l
    float lsum = 0.0f;
    for (int s = tid; s < n; s += MERGE_THREADS) {
        const float l = ml[s * ml_stride + 1];
        const float wt = (l > 0.0f && M != -INFINITY) ? exp2f(ml[s * ml_stride] - M) : 0.0f;
        f[s] = wt;
        lsum += wt * l;
    }
    for (int off = 16; off; off >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
    if (lane == 0) red[warp] = lsum;
    __syncthreads();
    float L = 0.0f;
    for (int wi = 0; wi < MERGE_THREADS / 32; ++wi) L += red[wi];
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
    for (int d0 = 0; d0 < Dd; d0 += 256) {
        float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        const int d = d0 + lane * 8;
        if (d < Dd) {
#pragma unroll 4
            for (int s = warp; s < n; s += MERGE_THREADS / 32) {
                const float wt = f[s];
                const float4* src = reinterpret_cast<const float4*>(o + s * o_stride + d);
                const float4 x = src[0], y = src[1];
                a[0] += wt * x.x; a[1] += wt * x.y; a[2] += wt * x.z; a[3] += wt * x.w;
                a[4] += wt * y.x; a[5] += wt * y.y; a[6] += wt * y.z; a[7] += wt * y.w;
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) acc_s[warp][lane * 8 + e] = a[e];
        }
        __syncthreads();
        if (d0 + tid < Dd) {
            float t = 0.0f;
#pragma unroll
            for (int wi = 0; wi < MERGE_THREADS / 32; ++wi) t += acc_s[wi][tid];
            // a partial output stays unnormalised; a final one takes the output gate when there is one
            out_row[d0 + tid] = ml_out ? t : gate_row ? t * inv * gate_sigmoid(gate_row + (int64_t) (d0 + tid) * 4) : t * inv;
        }
        __syncthreads();
    }
    if (ml_out && tid == 0) {
        ml_out[0] = M;
        ml_out[1] = L;
    }
}

// Merges the per-split partials of one row of one KV head (grid: rows x KV heads x ne3).
template <int RPC>
__global__ void __launch_bounds__(MERGE_THREADS) fa_combine_kernel(const FaStreamParams p) {
    const int gr = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
    const int chunk = gr / RPC, r = gr % RPC;
    const int64_t base = (((int64_t) b * p.n_head_kv + hk) * p.n_row_chunks + chunk) * p.n_splits;
    const int qi = gr / p.gqa, h = hk * p.gqa + gr % p.gqa;
    float* out = reinterpret_cast<float*>(p.dst + h * p.d_nb1 + qi * p.d_nb2 + b * p.d_nb3);
    float* ml_out = p.partial_out ? p.dst_ml + (((int64_t) b * p.n_q + qi) * p.n_head + h) * 2 : nullptr;
    const char* gate_row = p.gate && !p.partial_out ? p.gate + h * p.g_nb1 + qi * p.g_nb2 + b * p.g_nb3 : nullptr;
    if (!p.push) {
        merge_row(p.o_part + (base * RPC + r) * D, (int64_t) RPC * D, p.ml_part + (base * RPC + r) * 2, (int64_t) RPC * 2,
                  p.n_splits, D, out, ml_out, gate_row);
        return;
    }
    // fused exchange: this rank's merged partial row (o unnormalised, m, l) into slot `rank` of the slot set of this
    // exchange's epoch in every rank's gather buffer (packed part: o [rows][D], then (m, l) [rows][2])
    const int epoch = *reinterpret_cast<volatile const int*>(p.flags[p.rank] + p.n_ranks) + 1;
    const int64_t rows = (int64_t) p.n_q * p.n_head, ro = (int64_t) qi * p.n_head + h;
    const int64_t off = (int64_t) (epoch & 1) * p.slot_set_floats + (int64_t) p.rank * p.part_floats;
    float* own = p.gather[p.rank] + off;
    merge_row(p.o_part + (base * RPC + r) * D, (int64_t) RPC * D, p.ml_part + (base * RPC + r) * 2, (int64_t) RPC * 2,
              p.n_splits, D, own + ro * D, own + rows * D + ro * 2);
    __syncthreads();
    for (int d = 0; d < p.n_ranks; ++d) {
        if (d == p.rank) continue;
        float* dst = p.gather[d] + off;
        for (int i = threadIdx.x; i < D; i += blockDim.x) dst[ro * D + i] = own[ro * D + i];
        if (threadIdx.x < 2) dst[rows * D + ro * 2 + threadIdx.x] = own[rows * D + ro * 2 + threadIdx.x];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int total = (int) (gridDim.x * gridDim.y * gridDim.z);
        if (atomicAdd(p.push_counter, 1) == total - 1) {
            // the last CTA: every row is in place on every rank (each CTA fenced before counting itself)
            *p.push_counter = 0;
            __threadfence_system();
            for (int d = 0; d < p.n_ranks; ++d)
                asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(p.flags[d] + p.rank), "r"(PUSH_CHUNKS)
                             : "memory");
        }
    }
}

// Merges partial results computed over disjoint KV ranges (e.g. one per GPU), one row per block.
// Optionally the merge of an exchange between GPUs (see peer.cu): flags = [n_parts flags | epoch counter | done
// counter] of this rank. One thread per CTA polls with system-scope acquire loads, bounded by wait_ns.
__global__ void __launch_bounds__(MERGE_THREADS) lse_combine_kernel(const float* __restrict__ o_parts,
                                                                    const float* __restrict__ ml_parts, int64_t stride,
                                                                    int n_parts, int64_t rows, int Dd,
                                                                    float* __restrict__ dst, int* flags,
                                                                    int64_t slot_set_floats, int* err, uint64_t wait_ns) {
    const int64_t r = blockIdx.x;
    if (flags) {
        __shared__ int ready, epoch;
        if (threadIdx.x == 0) {
            ready = 1;
            epoch = *reinterpret_cast<volatile int*>(flags + n_parts) + 1;
            const uint64_t t0 = globaltimer_ns();
            for (int p = 0; p < n_parts && ready; ++p) {
                // a source's flag counts its pushed chunks: epoch * PUSH_CHUNKS once this epoch's push is complete
                // (compared as a wrapping difference)
                const unsigned target = (unsigned) epoch * (unsigned) PUSH_CHUNKS;
                for (;;) {
                    unsigned v;
                    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + p) : "memory");
                    if ((int) (v - target) >= 0) break;
                    if (globaltimer_ns() - t0 > wait_ns) {
                        record_error(err, DEV_ERR_WAIT_PEER);
                        ready = 0;
                        break;
                    }
                    __nanosleep(64);
                }
            }
        }
        __syncthreads();
        if (ready) {
            const int64_t set = (int64_t) (epoch & 1) * slot_set_floats;
            merge_row(o_parts + set + r * Dd, stride, ml_parts + set + r * 2, stride, n_parts, Dd, dst + r * Dd, nullptr);
        }
        // the last CTA to finish advances the epoch counter (every CTA has read it before counting itself done)
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            if (atomicAdd(flags + n_parts + 1, 1) == (int) rows - 1) {
                flags[n_parts + 1] = 0;
                __threadfence();
                atomicAdd(flags + n_parts, 1);
            }
        }
        return;
    }
    merge_row(o_parts + r * Dd, stride, ml_parts + r * 2, stride, n_parts, Dd, dst + r * Dd, nullptr);
}

// ------------------------------------------------------------------------------------------------ in-kernel exchange
//
// The sequence-split exchange at the end of the attention kernel itself (kb_flash_attn_ext_exchange), so a layer is
// one launch on every rank. After its main loop each CTA has written its split's partials (o, m, l) to the scratch:
//   1. grid barrier (cooperative launch: all CTAs resident) so every split of every row is in place;
//   2. output row ro (of n_q * H, in dst order) belongs to CTAs ro, ro + G, ... (the same rows on every rank,
//      whatever its grid); the CTA merges the row over the splits (log-sum-exp, as fa_combine_kernel: each warp a
//      share of the splits, lanes 8 dims each, the warps' sums meeting in shared memory) and stores the merged
//      partial (o unnormalised, m, l) into slot `rank` of every rank's gather buffer (plain stores to peer memory over
//      NVLink); after one system-scope fence its thread 0 writes the epoch into flag word (rank, ro) of every rank;
//   3. the CTA waits (acquire polls, bounded) until every source's flag word for its row holds the epoch, then merges
//      the n_ranks partials of the row from its local gather buffer the same way and stores the normalised (gated)
//      output row;
//   4. the last CTA to finish resets the barrier counters and advances the epoch.
// Slot sets alternate by epoch parity; a rank cannot start epoch e + 2 before every rank has pushed epoch e + 1, which
// each does only in a launch after the one that consumed epoch e, so a slot set is never overwritten while read.
// Shared memory: the attention's buffers are free by then (every TMA and MMA has completed before the dealloc).

// Log-sum-exp merge of one row (D dims) over n partials by the whole CTA: part s has o at o + s * o_stride and
// (m, l) at ml + s * ml_stride. Leaves the weighted sum of o in sh_out[D] and returns (M, L) through sh_ml (the row
// max over parts with l > 0, and sum_s 2^(m_s - M) l_s). sh: >= 256 + 2 * WARPS + WARPS * D floats of shared memory.
// Loads go through L2 (ld.global.cg): the parts were written by other CTAs or GPUs during this kernel.
template <int WARPS>
__device__ void cta_merge_row(float* sh, const float* o, int64_t o_stride, const float* ml, int64_t ml_stride, int n,
                              float* sh_out, float* sh_ml) {
    float* f = sh;                     // [256] weights
    float* red = sh + 256;             // [2 WARPS]
    float* acc = sh + 256 + 2 * WARPS;  // [WARPS][D]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // the first PF parts of this warp (w, w + WARPS, ...) are loaded together with the (m, l) pairs, before the
    // weights are known: one round trip to L2 for up to PF * WARPS parts (48)
    constexpr int PF = WARPS <= 8 ? 6 : 3;
    float4 xa[PF], xb[PF];
#pragma unroll
    for (int k = 0; k < PF; ++k) {
        const int sp = warp + k * WARPS;
        xa[k] = xb[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (sp < n) {
            const float4* src = reinterpret_cast<const float4*>(o + (int64_t) sp * o_stride + lane * 8);
            xa[k] = __ldcg(src);
            xb[k] = __ldcg(src + 1);
        }
    }
    float mx = -INFINITY;
    float2 v0 = make_float2(-INFINITY, 0.0f);
    if (tid < n) {
        v0 = __ldcg(reinterpret_cast<const float2*>(ml + (int64_t) tid * ml_stride));
        if (v0.y > 0.0f) mx = v0.x;
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    float M = red[0];
#pragma unroll
    for (int w = 1; w < WARPS; ++w) M = fmaxf(M, red[w]);
    float lw = 0.0f;
    if (tid < n) {
        const float w = (v0.y > 0.0f && M != -INFINITY) ? exp2f(v0.x - M) : 0.0f;
        f[tid] = w;
        lw = w * v0.y;
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, off);
    if (lane == 0) red[WARPS + warp] = lw;
    __syncthreads();
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    auto fma8 = [&](float w, const float4& x, const float4& y) {
        a[0] = fmaf(w, x.x, a[0]), a[1] = fmaf(w, x.y, a[1]), a[2] = fmaf(w, x.z, a[2]), a[3] = fmaf(w, x.w, a[3]);
        a[4] = fmaf(w, y.x, a[4]), a[5] = fmaf(w, y.y, a[5]), a[6] = fmaf(w, y.z, a[6]), a[7] = fmaf(w, y.w, a[7]);
    };
#pragma unroll
    for (int k = 0; k < PF; ++k) {
        const int sp = warp + k * WARPS;
        if (sp < n) fma8(f[sp], xa[k], xb[k]);
    }
#pragma unroll 4
    for (int sp = warp + PF * WARPS; sp < n; sp += WARPS) {
        const float4* src = reinterpret_cast<const float4*>(o + (int64_t) sp * o_stride + lane * 8);
        fma8(f[sp], __ldcg(src), __ldcg(src + 1));
    }
    *reinterpret_cast<float4*>(acc + warp * D + lane * 8) = make_float4(a[0], a[1], a[2], a[3]);
    *reinterpret_cast<float4*>(acc + warp * D + lane * 8 + 4) = make_float4(a[4], a[5], a[6], a[7]);
    __syncthreads();
    for (int d = tid; d < D; d += WARPS * 32) {
        float t = 0.0f;
#pragma unroll
        for (int w = 0; w < WARPS; ++w) t += acc[w * D + d];
        sh_out[d] = t;
    }
    if (tid == 0) {
        float L = 0.0f;
#pragma unroll
        for (int w = 0; w < WARPS; ++w) L += red[WARPS + w];
        sh_ml[0] = M;
        sh_ml[1] = L;
    }
    __syncthreads();
}

template <int RPC, int WARPS>
__device__ void exchange_tail(const FaStreamParams& p, float* sh) {
    __shared__ int s_epoch;
    __shared__ volatile int s_ok;
    const int G = (int) (gridDim.x * gridDim.y * gridDim.z);
    const int cta = (int) (blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z));
    int* my = p.flags[p.rank];
    int* bar = my + p.n_ranks + 2;
    int* done = my + p.n_ranks + 3;
    float* sh_row = sh + 256 + 2 * WARPS + WARPS * D;  // [D] merged row, then (M, L)
    float* sh_ml = sh_row + D;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();  // the CTA's split partials (ordered before it by the barrier) are visible device-wide
        s_epoch = *reinterpret_cast<volatile int*>(my + p.n_ranks) + 1;
        s_ok = 1;
        atomicAdd(bar, 1);
        const uint64_t t0 = globaltimer_ns();
        while (ld_acquire_gpu(bar) < G) {
            if (globaltimer_ns() - t0 > p.wait_ns) {
                record_error(p.err, DEV_ERR_WAIT_GRID);
                s_ok = 0;
                break;
            }
        }
    }
    __syncthreads();
    const int e = s_epoch;
    const int rows = p.n_q * p.n_head;
    const int64_t set_off = (int64_t) (e & 1) * p.slot_set_floats;
    const int64_t own_off = set_off + (int64_t) p.rank * p.part_floats;
    if (s_ok) {
        for (int ro = cta; ro < rows; ro += G) {
            const int h = ro % p.n_head, qi = ro / p.n_head;
            const int hk = h / p.gqa, gr = qi * p.gqa + h % p.gqa, chunk = gr / RPC, r = gr % RPC;
            const int64_t base = ((int64_t) hk * p.n_row_chunks + chunk) * p.n_splits;
            cta_merge_row<WARPS>(sh, p.o_part + (base * RPC + r) * D, (int64_t) RPC * D, p.ml_part + base * RPC * 2 + r * 2,
                                 (int64_t) RPC * 2, p.n_splits, sh_row, sh_ml);
            // the merged partial of this rank into every rank's gather buffer: o row, then (m, l)
            for (int i = threadIdx.x; i < p.n_ranks * (D / 4 + 1); i += WARPS * 32) {
                const int d = i / (D / 4 + 1), k = i % (D / 4 + 1);
                float* g = p.gather[d] + own_off;
                if (k < D / 4)
                    *reinterpret_cast<float4*>(g + (int64_t) ro * D + 4 * k) = *reinterpret_cast<const float4*>(sh_row + 4 * k);
                else
                    *reinterpret_cast<float2*>(g + (int64_t) rows * D + (int64_t) ro * 2) = make_float2(sh_ml[0], sh_ml[1]);
            }
            // one system-scope fence per CTA: the barrier orders every thread's stores before thread 0's fence
            // (cumulativity), and the flag stores after it publish them
            __syncthreads();
            if (threadIdx.x == 0) {
                __threadfence_system();
                for (int d = 0; d < p.n_ranks; ++d)
                    st_relaxed_sys(p.flags[d] + XCHG_FLAG_BASE + p.rank * XCHG_MAX_SLOTS + ro, e);
            }
        }
        for (int ro = cta; ro < rows; ro += G) {
            if (threadIdx.x < p.n_ranks) {
                const int* f = my + XCHG_FLAG_BASE + threadIdx.x * XCHG_MAX_SLOTS + ro;
                const uint64_t t0 = globaltimer_ns();
                while ((int) ((unsigned) ld_acquire_sys(f) - (unsigned) e) < 0) {  // wrapping comparison
                    if (globaltimer_ns() - t0 > p.wait_ns) {
                        record_error(p.err, DEV_ERR_WAIT_PEER);
                        s_ok = 0;
                        break;
                    }
                    __nanosleep(20);
                }
            }
            __syncthreads();
            if (!s_ok) break;
            const float* g = p.gather[p.rank] + set_off;
            cta_merge_row<WARPS>(sh, g + (int64_t) ro * D, p.part_floats, g + (int64_t) rows * D + (int64_t) ro * 2,
                                 p.part_floats, p.n_ranks, sh_row, sh_ml);
            const int h = ro % p.n_head, qi = ro / p.n_head;
            const float L = sh_ml[1];
            const float inv = L > 0.0f ? 1.0f / L : 0.0f;
            float* out = reinterpret_cast<float*>(p.dst + h * p.d_nb1 + qi * p.d_nb2);
            for (int d = threadIdx.x; d < D; d += WARPS * 32) {
                float v = sh_row[d] * inv;
                if (p.gate) v *= gate_sigmoid(p.gate + h * p.g_nb1 + qi * p.g_nb2 + (int64_t) d * 4);
                out[d] = v;
            }
            __syncthreads();
        }
    }
    // the last CTA resets the counters and advances the epoch (every CTA has read the epoch before counting itself)
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(done, 1) == G - 1) {
            *reinterpret_cast<volatile int*>(bar) = 0;
            *reinterpret_cast<volatile int*>(done) = 0;
            __threadfence();
            atomicAdd(my + p.n_ranks, 1);
        }
    }
}

// ------------------------------------------------------------------------------------------------ tcgen05 kernel
//
// One CTA per (split, KV head, row chunk). The rows of a chunk are the N columns (16 or 32) of S^T = K Q^T,
// computed for 128 cells at a time (M = 128): every K and V byte is read by the tensor core once per CTA, and the
// softmax needs no per-row exchange within a thread. Roles (q8_0 / q4_0: 16 warps; f16: 8 warps, no
// dequantisation):
//   warps 0-3   softmax, thread = cell (TMEM lane) of the 128-cell block: x = score - row max against row maxima
//               kept in shared memory (+inf for a row that has seen nothing), one barrier reduction per block to
//               check max x <= 8 (log2 units, so P <= 2^8 in f16); when a row max rises the scores are re-read
//               from TMEM, the maxima recomputed, O^T and the partial sums rescaled. P^T as f16 into shared
//               memory; partial row sums per thread, summed once at the end
//   q8_0 / q4_0 only:
//   warps 4-7   K dequantisation, thread = cell: its raw row (aligned 16-byte loads: 272 B for q8_0, 144 B for
//               q4_0) -> 256 f16 values f16(q * d) (q4_0: (n - 8) * d) -> TMEM, the A operand of S^T (TS form)
//   warps 8-11  V dequantisation: raw tile -> f16 [64 cells][256 dims] swizzled tile, the A operand V^T of O^T
//               (bank-conflict-free assignment: 8 consecutive cells x 4 blocks per warp instruction)
//   then (quantised: warps 12-15, f16: warps 4-7):
//               TMA producers of K and V (quantised: raw tile rings of 4 and 3; f16: two 128-cell K blocks, the SS-form
//               A operand of S^T, and two 64-cell V tiles)
//               S issuer: S^T_j = K_j Q^T (16 MMAs of K 16) into buffer j % 2 once the softmax has read S_{j-2}
//               PV issuer: O^T += V^T P^T of block j (2 M-halves x 4 K-steps per 64-cell tile) once P_j is
//               written. Two issuers: the tensor core accepts only a few MMAs ahead, so one thread would hold
//               S_{j+2} back behind the 16 PV MMAs of block j.
// TMEM: S^T 2 x N columns at 0, O^T 2 x N at 64 (dims 0-127, 128-255 on the lanes), quantised: K f16 2 x 128 at
// 128. Numerics: f16 K: Q rounded to f16; q8_0 / q4_0 K: Q quantised to q8_0 and widened to f16(q * d), K and V
// widened to f16 of their dequantised values. f32 accumulation, P rounded to f16.
namespace tc {
constexpr int BLK = 128;  // cells per S^T block
constexpr int KRAW = 4, VRAW = 3;
// Each K-dequantisation warp pair waits on the slots of its own tiles (even or odd) only, so a slot must always
// carry tiles of one parity: with an odd depth a pair could wait for a phase two ahead of the slot's current one
// and pass it at once (a parity wait sees only the last two phases).
static_assert(KRAW % 2 == 0, "K ring slots carry tiles of one parity");
// cache kinds of the kernel (q8_0 and q4_0 add the 8 dequantisation warps 4-11)
constexpr int KT_F16 = 0, KT_Q8 = 1, KT_Q4 = 2;
template <int KT>
constexpr int raw_row() { return KT == KT_Q8 ? QROW : Q4ROW; }

template <bool Q8>  // Q8: a block-quantised cache (q8_0 or q4_0), with dequantisation warps
struct Roles {
    static constexpr int KDQ = 4, VDQ = 8;
    static constexpr int KTMA = Q8 ? 12 : 4, VTMA = Q8 ? 13 : 5, SMMA = Q8 ? 14 : 6, PVMMA = Q8 ? 15 : 7;
    static constexpr int THREADS = (Q8 ? 16 : 8) * 32;
    static constexpr uint32_t TMEM_COLS = Q8 ? 512 : 128;
    // quantised: registers per thread at launch (the whole register file over THREADS), and the shares the producer /
    // issuer warpgroup and each of the three compute warpgroups move to with setmaxnreg
    static constexpr uint32_t REG_LAUNCH = 65536 / THREADS, REG_PRODUCERS = 80, REG_COMPUTE = 144;
    static_assert(!Q8 || 3 * REG_COMPUTE + REG_PRODUCERS == 4 * REG_LAUNCH, "the shares add up to the launch's total");
};
constexpr uint32_t TM_S = 0, TM_O = 64, TM_K = 128;
constexpr float THRESH = 8.0f;  // log2 units

template <int N, int KT>
struct Smem {
    static constexpr int RAWT = TILE * raw_row<KT>();  // bytes of one raw tile (q8_0, q4_0)
    uint8_t v[2][KTILE_F16];        // f16 V tiles [4 dim chunks][64 cells][128 B], 128B-swizzled
    uint8_t q[D / 64][N * 128];     // Q f16, K-major swizzled: the B operand of S^T
    uint8_t p[2][2][N * 128];       // P^T [buffer][64-cell half][N rows][128 B]: the B operand of O^T
    // quantised: the raw K ring; f16: two K blocks [4 dim chunks][128 cells][128 B], the A operand of S^T
    uint8_t kbuf[KT != KT_F16 ? KRAW * RAWT : 2 * 2 * KTILE_F16];
    uint8_t vraw[KT != KT_F16 ? VRAW * RAWT : 16];  // quantised: the raw V ring
    float red[4][N];                // per-warp row maxima / sums
    float mrow[N];                  // running row maxima (log2 units), shared by all cells
    float nref[N];                  // -(row max) per row: +inf while the row has seen nothing, -inf past the rows
    float alpha[N];                 // rescale factors of the last raise
    int row_qi[N], row_h[N];
    float row_slope[N];
    const __half* row_mask[N];      // each row's mask row (dense mask), or null
    uint64_t kfull[KRAW], kempty[KRAW], vfull[VRAW], vempty[VRAW];
    uint64_t k_full[2], k_free[2], s_full[2], p_full[2], p_free[2], v_full[2], v_free[2], o_done, s_done;
    uint32_t tmem_base;
    int failed;
};

static_assert(sizeof(Smem<32, KT_Q8>) <= 232448 && sizeof(Smem<32, KT_Q4>) <= 232448 && sizeof(Smem<32, KT_F16>) <= 232448,
              "fits one SM's shared memory");

__device__ __forceinline__ bool wait_or_fail(uint64_t* bar, uint32_t parity, const FaStreamParams& p, volatile int* failed,
                                             int code) {
    if (*failed) return false;
    if (mbar_wait(bar, parity, p.wait_ns)) return true;
    record_error(p.err, code);
    *failed = 1;
    return false;
}

// OR of a predicate over the `count` threads that reach named barrier `id`
__device__ __forceinline__ bool bar_red_or(int id, int count, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t) pred), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}

// Reduces N per-row values over the 32 lanes of a warp; lane l ends with row (l % N). Each step halves the
// values a lane holds: it keeps one half, sends the other to its partner (31 shuffles for N = 32).
template <int N, bool MAX>
__device__ __forceinline__ float warp_rows_reduce(float (&v)[N], int lane) {
    auto op = [](float a, float b) { return MAX ? fmaxf(a, b) : a + b; };
    if constexpr (N == 16) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = op(v[i], __shfl_xor_sync(0xffffffffu, v[i], 16));
    }
#pragma unroll
    for (int off = N / 2, cnt = N / 2; off >= 1; off >>= 1, cnt >>= 1) {
        const bool upper = lane & off;
#pragma unroll
        for (int i = 0; i < cnt; ++i) {
            const float send = upper ? v[i] : v[i + cnt];
            const float keep = upper ? v[i + cnt] : v[i];
            v[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, off));
        }
    }
    return v[0];
}

// 4 q8_0 quants -> two f16 pairs q * d ((q ^ 0x80) in the low mantissa byte of 1024 is 1152 + q exactly)
__device__ __forceinline__ void q4_to_f16(uint32_t qw, __half2 d2, uint32_t& lo, uint32_t& hi) {
    const __half2 bias = __floats2half2_rn(1152.0f, 1152.0f);
    const uint32_t xw = qw ^ 0x80808080u;
    uint32_t a = __byte_perm(xw, 0x64646464u, 0x4140), c = __byte_perm(xw, 0x64646464u, 0x4342);
    __half2 l2 = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&a), bias), d2);
    __half2 h2 = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&c), bias), d2);
    lo = *reinterpret_cast<uint32_t*>(&l2);
    hi = *reinterpret_cast<uint32_t*>(&h2);
}

// 4 q4_0 bytes -> the f16 pairs of their low nibbles (values j .. j + 3 of the block) and of their high nibbles
// (values 16 + j .. 19 + j), (n - 8) * d ((n | 0x6400) is 1024 + n exactly; minus 1032)
__device__ __forceinline__ void n4_to_f16(uint32_t qw, __half2 d2, uint32_t& lo0, uint32_t& lo1, uint32_t& hi0,
                                          uint32_t& hi1) {
    const __half2 bias = __floats2half2_rn(1032.0f, 1032.0f);
    const uint32_t lo = qw & 0x0F0F0F0Fu, hi = (qw >> 4) & 0x0F0F0F0Fu;
    uint32_t a = __byte_perm(lo, 0x64646464u, 0x4140), b = __byte_perm(lo, 0x64646464u, 0x4342);
    uint32_t c = __byte_perm(hi, 0x64646464u, 0x4140), e = __byte_perm(hi, 0x64646464u, 0x4342);
    __half2 ra = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&a), bias), d2);
    __half2 rb = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&b), bias), d2);
    __half2 rc = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&c), bias), d2);
    __half2 re = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&e), bias), d2);
    lo0 = *reinterpret_cast<uint32_t*>(&ra);
    lo1 = *reinterpret_cast<uint32_t*>(&rb);
    hi0 = *reinterpret_cast<uint32_t*>(&rc);
    hi1 = *reinterpret_cast<uint32_t*>(&re);
}

// q4_0 V dequantisation slots: 2 sets of 4 blocks whose first nibble words are 0, 1, 2, 3 (mod 4) ({0, 1, 3, 5},
// {7, 2, 4, 6}), 3 bits each
constexpr uint32_t V4SLOTS = 0u | (1u << 3) | (3u << 6) | (5u << 9) | (7u << 12) | (2u << 15) | (4u << 18) | (6u << 21);

// V dequantisation slots: slot set ss (0-3) x slot (0-3) -> 2 * block + half, 4 bits each. In every set the
// first quant words of the 4 slots are 0, 1, 2, 3 (mod 4), so 8 consecutive cells x 4 slots hit 32 distinct banks:
//   {(0,0) (1,0) (3,0) (5,0)}  {(0,1) (1,1) (3,1) (5,1)}  {(7,0) (2,0) (4,0) (6,0)}  {(7,1) (2,1) (4,1) (6,1)}
constexpr uint64_t VSLOTS = 0x0ULL | (0ULL << 0) | (2ULL << 4) | (6ULL << 8) | (10ULL << 12) | (1ULL << 16) | (3ULL << 20) |
                            (7ULL << 24) | (11ULL << 28) | (14ULL << 32) | (4ULL << 36) | (8ULL << 40) | (12ULL << 44) |
                            (15ULL << 48) | (5ULL << 52) | (9ULL << 56) | (13ULL << 60);

template <int N, int KT>
__global__ void __launch_bounds__(Roles<KT != KT_F16>::THREADS, 1)
    fa_stream_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                        const FaStreamParams p) {
    constexpr bool Q8 = KT != KT_F16;  // a block-quantised cache: raw rings and dequantisation warps
    constexpr int RAWROW = raw_row<KT>(), RAWT = TILE * RAWROW;
    using R_ = Roles<Q8>;
    constexpr int THREADS = R_::THREADS;
    constexpr int W_KDQ = R_::KDQ, W_VDQ = R_::VDQ, W_KTMA = R_::KTMA, W_VTMA = R_::VTMA, W_SMMA = R_::SMMA,
                  W_PVMMA = R_::PVMMA;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    if (smem_u32(smem_raw) & 1023) {
        if (threadIdx.x == 0) record_error(p.err, DEV_ERR_ALIGN);
        return;
    }
    Smem<N, KT>& sm = *reinterpret_cast<Smem<N, KT>*>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x, hk = blockIdx.y;
    const int chunk = blockIdx.z % p.n_row_chunks, b = blockIdx.z / p.n_row_chunks;
    const int64_t key_begin = ((int64_t) split * p.blocks_base + min(split, p.blocks_extra)) * BLK;
    const int64_t key_end = min(p.n_kv, key_begin + (p.blocks_base + (split < p.blocks_extra ? 1 : 0)) * BLK);
    const int n_tiles = key_end > key_begin ? (int) ((key_end - key_begin + TILE - 1) / TILE) : 0;
    const int nblk = (n_tiles + 1) / 2;
    const int row0 = chunk * N;
    const int rows = min(N, p.R - row0);
    const int kb3 = b / p.rk3;

    if (p.push && threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) *p.push_counter = 0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < KRAW; ++s) {
            mbar_init(&sm.kfull[s], 1);
            mbar_init(&sm.kempty[s], 2);
        }
        for (int s = 0; s < VRAW; ++s) {
            mbar_init(&sm.vfull[s], 1);
            mbar_init(&sm.vempty[s], 4);
        }
        for (int s = 0; s < 2; ++s) {
            // quantised: the 4 dequantisation warps of each kind arrive; f16: the TMA transaction counts
            mbar_init(&sm.k_full[s], Q8 ? 4 : 1);
            mbar_init(&sm.k_free[s], 1);
            mbar_init(&sm.s_full[s], 1);
            mbar_init(&sm.p_full[s], 4);
            mbar_init(&sm.p_free[s], 1);
            mbar_init(&sm.v_full[s], Q8 ? 4 : 1);
            mbar_init(&sm.v_free[s], 1);
        }
        mbar_init(&sm.o_done, 1);
        mbar_init(&sm.s_done, 1);
        sm.failed = 0;
        fence_barrier_init();
    }
    if (warp == W_SMMA) {
        tmem_alloc(&sm.tmem_base, R_::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    volatile int* failed = &sm.failed;
    // Q staging by every warp but the TMA producers, which start streaming K and V once the Q loads are issued (so that
    // these are not queued behind the first K / V tiles). Q rounded to f16 (f16 K), or quantised like
    // quantize_row_q8_0_ref and widened to f16(q * d) (q8_0 / q4_0 K), into the swizzled K-major image; rows past the
    // chunk are zero. Thread t takes float4s t, t + QT, ... of the [N rows][64 float4] block, all loaded before any is
    // converted; a 32-dim q8_0 block is 8 consecutive threads (QT is a multiple of 8).
    constexpr int QT = THREADS - 64, NF = N * (D / 4), PER = (NF + QT - 1) / QT;
    const bool q_stager = warp != W_KTMA && warp != W_VTMA;
    const int tq = warp < W_KTMA ? (int) threadIdx.x : (int) threadIdx.x - 64;
    float4 qv[PER];
#pragma unroll
    for (int i = 0; i < PER && q_stager; ++i) {
        const int f = i * QT + tq, r = f / (D / 4);
        qv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (f < NF && r < rows) {
            const int gr = row0 + r;
            const int qi = gr / p.gqa, h = hk * p.gqa + gr % p.gqa;
            const char* src = p.q + (int64_t) (f % (D / 4)) * 16 + qi * p.q_nb1 + h * p.q_nb2 + b * p.q_nb3;
            if (p.q_vec4) {
                qv[i] = *reinterpret_cast<const float4*>(src);
            } else {
                const float* s4 = reinterpret_cast<const float*>(src);
                qv[i] = make_float4(s4[0], s4[1], s4[2], s4[3]);
            }
        }
    }
    named_bar_sync(3, THREADS);  // the Q loads are issued (their data may still be in flight)
    if (q_stager) {
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            const int f = i * QT + tq, r = f / (D / 4);
            float x0 = qv[i].x, x1 = qv[i].y, x2 = qv[i].z, x3 = qv[i].w;
            if constexpr (Q8) {
                // amax over the 8 threads of this 32-dim block (every thread of the warp takes part)
                float amax = fmaxf(fmaxf(fabsf(x0), fabsf(x1)), fmaxf(fabsf(x2), fabsf(x3)));
#pragma unroll
                for (int off = 1; off < 8; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
                const float d = amax / 127.0f;
                const float id = d != 0.0f ? 1.0f / d : 0.0f;
                const float dh = __half2float(__float2half_rn(d));
                x0 = roundf(x0 * id) * dh, x1 = roundf(x1 * id) * dh, x2 = roundf(x2 * id) * dh, x3 = roundf(x3 * id) * dh;
            }
            if (f < NF) {
                const int dim = (f % (D / 4)) * 4, e = dim & 63;
                *reinterpret_cast<uint2*>(sm.q[dim >> 6] + r * 128 + (((e >> 3) ^ (r & 7)) << 4) + (e & 7) * 2) =
                    make_uint2(pack_half2(x0, x1), pack_half2(x2, x3));
            }
        }
        if (threadIdx.x < N) {
            const int r = threadIdx.x;
            const int gr = row0 + min(r, max(rows - 1, 0));
            const int qi = gr / p.gqa, h = hk * p.gqa + gr % p.gqa;
            sm.row_qi[r] = qi;
            sm.row_h[r] = h;
            sm.row_slope[r] = slope_of(p, h);
            sm.row_mask[r] = p.mask ? reinterpret_cast<const __half*>(p.mask + qi * p.m_nb1 + (h % p.m_ne2) * p.m_nb2 +
                                                                        (b % p.m_ne3) * p.m_nb3)
                                    : nullptr;
        }
        fence_proxy_async_smem();
        named_bar_sync(2, THREADS - 64);
    }

    // Registers (quantised caches): the producer / issuer warpgroup (warps 12-15) gives 48 of its 128 per thread to
    // the three compute warpgroups (softmax, K and V dequantisation: 144 each); 3 x 144 + 80 = 4 x 128, the launch's
    // total. Both calls are made once per warp, by all 32 lanes together (every warp is converged after the Q-staging
    // barriers), and the counts are kept to the end: the common tail runs within the smaller share.
    if (warp >= W_KTMA) {
    if constexpr (Q8) {
        __syncwarp();
        reg_lower<R_::REG_PRODUCERS>();
    }
    if (warp == W_KTMA || warp == W_VTMA) {
        // ------------------------------------------------------------------------ TMA producers
        const bool is_v = warp == W_VTMA;
        if (lane == 0 && n_tiles > 0) {
            const CUtensorMap* map = is_v ? &tmV : &tmK;
            tma_prefetch_desc(map);
            const uint64_t pol = l2_policy_evict_first();
            if constexpr (Q8) {
                // raw tiles into rings of KRAW / VRAW tiles
                const int depth = is_v ? VRAW : KRAW;
                for (int t = 0; t < n_tiles; ++t) {
                    const int s = t % depth;
                    uint64_t* empty = is_v ? &sm.vempty[s] : &sm.kempty[s];
                    uint64_t* fullb = is_v ? &sm.vfull[s] : &sm.kfull[s];
                    uint8_t* dst = (is_v ? sm.vraw : sm.kbuf) + s * RAWT;
                    if (t >= depth && !wait_or_fail(empty, ((t / depth) - 1) & 1, p, failed, DEV_ERR_WAIT_EMPTY)) break;
                    mbar_arrive_expect_tx(fullb, RAWT);
                    tma_load_4d(dst, map, fullb, 0, hk, (int) (key_begin + (int64_t) t * TILE), kb3, pol);
                }
            } else if (!is_v) {
                // f16 K: 128-cell blocks as [4 dim chunks][128 cells][128 B] (two 64-cell boxes per chunk); a
                // block's second tile past the split is loaded too (finite cells of the next split, or zeros past
                // the cache) and masked by the softmax
                for (int j = 0; j < nblk; ++j) {
                    if (j >= 2 && !wait_or_fail(&sm.k_free[j & 1], ((j >> 1) - 1) & 1, p, failed, DEV_ERR_WAIT_EMPTY)) break;
                    mbar_arrive_expect_tx(&sm.k_full[j & 1], 2 * KTILE_F16);
                    uint8_t* dst = sm.kbuf + (j & 1) * 2 * KTILE_F16;
                    for (int c = 0; c < D / 64; ++c)
                        for (int h = 0; h < 2; ++h)
                            tma_load_4d(dst + c * (BLK * 128) + h * (TILE * 128), map, &sm.k_full[j & 1], 64 * c, hk,
                                        (int) (key_begin + (int64_t) j * BLK + h * TILE), kb3, pol);
                }
            } else {
                // f16 V: 64-cell tiles [4 dim chunks][64 cells][128 B], the A operand V^T as loaded
                for (int t = 0; t < n_tiles; ++t) {
                    if (t >= 2 && !wait_or_fail(&sm.v_free[t & 1], ((t >> 1) - 1) & 1, p, failed, DEV_ERR_WAIT_EMPTY)) break;
                    mbar_arrive_expect_tx(&sm.v_full[t & 1], KTILE_F16);
                    for (int c = 0; c < D / 64; ++c)
                        tma_load_4d(sm.v[t & 1] + c * (TILE * 128), map, &sm.v_full[t & 1], 64 * c, hk,
                                    (int) (key_begin + (int64_t) t * TILE), kb3, pol);
                }
            }
        }
    } else if (warp == W_SMMA) {
        // ------------------------------------------------------------------------ S issuer
        if (lane == 0) {
            constexpr uint32_t idS = umma_idesc_f16(0, BLK, N, false, false);
            const uint32_t q_addr = smem_u32(sm.q);
            for (int j = 0; j < nblk; ++j) {
                if (!wait_or_fail(&sm.k_full[j & 1], (j >> 1) & 1, p, failed, DEV_ERR_WAIT_FULL)) break;
                // the softmax has read S_{j-2} (it wrote P_{j-2} after its TMEM loads completed)
                if (j >= 2 && !wait_or_fail(&sm.p_full[j & 1], ((j >> 1) - 1) & 1, p, failed, DEV_ERR_WAIT_EMPTY)) break;
                tc_fence_after();
                const uint32_t k_addr = smem_u32(sm.kbuf + (j & 1) * 2 * KTILE_F16);
#pragma unroll
                for (int k = 0; k < D / 16; ++k) {
                    const uint64_t bdesc = smem_desc_sw128(q_addr + (k >> 2) * (N * 128) + (k & 3) * 32, 16, 1024);
                    if constexpr (Q8) {
                        // A = K f16 in TMEM (8 packed columns per K-step)
                        umma_ts(tmem + TM_S + (j & 1) * N, tmem + TM_K + (j & 1) * 128 + k * 8, bdesc, idS, k > 0);
                    } else {
                        // A = K block in shared memory, K-major
                        const uint64_t adesc = smem_desc_sw128(k_addr + (k >> 2) * (BLK * 128) + (k & 3) * 32, 16, 1024);
                        umma_ss(tmem + TM_S + (j & 1) * N, adesc, bdesc, idS, k > 0);
                    }
                }
                umma_commit(&sm.s_full[j & 1]);
                umma_commit(&sm.k_free[j & 1]);
            }
            umma_commit(&sm.s_done);  // on every path: the wait before the dealloc covers these MMAs
        }
    } else if (warp == W_PVMMA) {
        // ------------------------------------------------------------------------ PV issuer
        if (lane == 0) {
            constexpr uint32_t idO = umma_idesc_f16(0, BLK, N, true, false);
            for (int i = 0; i < nblk; ++i) {
                if (!wait_or_fail(&sm.p_full[i & 1], (i >> 1) & 1, p, failed, DEV_ERR_WAIT_FULL)) break;
                bool ok = true;
                for (int tt = 0; tt < 2 && ok; ++tt) {
                    const int t = 2 * i + tt;
                    if (t >= n_tiles) break;
                    ok = wait_or_fail(&sm.v_full[t & 1], (t >> 1) & 1, p, failed, DEV_ERR_WAIT_FULL);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t v_addr = smem_u32(sm.v[t & 1]), p_addr = smem_u32(sm.p[i & 1][tt]);
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
                        for (int ks = 0; ks < TILE / 16; ++ks) {
                            // A = V^T, MN-major: dims of 64-dim chunks 8 KiB apart (LBO), 8-cell groups 1 KiB
                            // apart (SBO); B = P^T, K-major
                            const uint64_t adesc = smem_desc_sw128(v_addr + hh * 2 * (TILE * 128) + ks * 16 * 128,
                                                                   TILE * 128, 1024);
                            const uint64_t bdesc = smem_desc_sw128(p_addr + ks * 32, 16, 1024);
                            umma_ss(tmem + TM_O + hh * N, adesc, bdesc, idO, i > 0 || tt > 0 || ks > 0);
                        }
                    }
                    umma_commit(&sm.v_free[t & 1]);
                }
                if (!ok) break;
                umma_commit(&sm.p_free[i & 1]);
            }
            umma_commit(&sm.o_done);  // on every path
        }
    }
    } else {
    if constexpr (Q8) {
        __syncwarp();
        reg_raise<R_::REG_COMPUTE>();
    }
    if (Q8 && warp >= W_KDQ && warp < W_VDQ) {
        // ------------------------------------------------------------------------ K dequantisation -> TMEM
        const int i = warp - W_KDQ;
        const int half = i >> 1, cell = 32 * (i & 1) + lane;
        const uint32_t lane_base = tmem + ((uint32_t) (32 * i) << 16);
        for (int j = 0; j < nblk; ++j) {
            const int t = 2 * j + half;
            bool ok = j < 2 || wait_or_fail(&sm.k_free[j & 1], ((j >> 1) - 1) & 1, p, failed, DEV_ERR_WAIT_EMPTY);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            if (t < n_tiles) {
                ok = wait_or_fail(&sm.kfull[t % KRAW], (t / KRAW) & 1, p, failed, DEV_ERR_WAIT_FULL);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
                const uint4* row = reinterpret_cast<const uint4*>(sm.kbuf + (t % KRAW) * RAWT + cell * RAWROW);
                tc_fence_after();
                if constexpr (KT == KT_Q4) {
                    // the 144-byte row by 9 aligned 16-byte loads; block b at byte 18 b (scale, then 16 bytes of
                    // nibbles: low nibbles values 0-15, high nibbles 16-31)
                    uint32_t w[36];
#pragma unroll
                    for (int b4 = 0; b4 < 8; ++b4) {
                        // two halves of registers: words 0-19 for blocks 0-3 (bytes 0-71), 16-35 for blocks 4-7
                        if (b4 == 0 || b4 == 4) {
#pragma unroll
                            for (int u = (b4 == 0 ? 0 : 4); u < (b4 == 0 ? 5 : 9); ++u) {
                                const uint4 x = row[u];
                                w[4 * u] = x.x, w[4 * u + 1] = x.y, w[4 * u + 2] = x.z, w[4 * u + 3] = x.w;
                            }
                        }
                        const uint32_t sw = w[(18 * b4) / 4];
                        const uint16_t dbits = (18 * b4) % 4 == 0 ? (uint16_t) (sw & 0xffffu) : (uint16_t) (sw >> 16);
                        const __half dh = __ushort_as_half(dbits);
                        const __half2 d2 = __halves2half2(dh, dh);
                        uint32_t out[16];
#pragma unroll
                        for (int g = 0; g < 4; ++g) {
                            const int byte = 18 * b4 + 2 + 4 * g;
                            const uint32_t qw =
                                byte % 4 == 0 ? w[byte / 4] : __funnelshift_r(w[byte / 4], w[byte / 4 + 1], 16);
                            n4_to_f16(qw, d2, out[2 * g], out[2 * g + 1], out[8 + 2 * g], out[8 + 2 * g + 1]);
                        }
                        tmem_st16(lane_base + TM_K + (j & 1) * 128 + 16 * b4, out);
                    }
                } else {
                // two halves of the row, one loop body: bytes [128 hb, 128 hb + 144) by 9 aligned 16-byte loads;
                // the half's 4 blocks start at byte 8 hb of that window, so the second half is shifted 2 words
#pragma unroll 1
                for (int hb = 0; hb < 2; ++hb) {
                    uint32_t w[36];
#pragma unroll
                    for (int u = 0; u < 9; ++u) {
                        const uint4 x = row[8 * hb + u];
                        w[4 * u] = x.x, w[4 * u + 1] = x.y, w[4 * u + 2] = x.z, w[4 * u + 3] = x.w;
                    }
#pragma unroll
                    for (int k = 0; k < 34; ++k) w[k] = hb ? w[k + 2] : w[k];
#pragma unroll
                    for (int bl = 0; bl < 4; ++bl) {
                        const uint32_t sw = w[(34 * bl) / 4];
                        const uint16_t dbits = (34 * bl) % 4 == 0 ? (uint16_t) (sw & 0xffffu) : (uint16_t) (sw >> 16);
                        const __half dh = __ushort_as_half(dbits);
                        const __half2 d2 = __halves2half2(dh, dh);
                        uint32_t out[16];
#pragma unroll
                        for (int g = 0; g < 8; ++g) {
                            const int byte = 34 * bl + 2 + 4 * g;
                            const uint32_t qw =
                                byte % 4 == 0 ? w[byte / 4] : __funnelshift_r(w[byte / 4], w[byte / 4 + 1], 16);
                            q4_to_f16(qw, d2, out[2 * g], out[2 * g + 1]);
                        }
                        tmem_st16(lane_base + TM_K + (j & 1) * 128 + 16 * (4 * hb + bl), out);
                    }
                }
                }
                tmem_wait_st();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.kempty[t % KRAW]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.k_full[j & 1]);
        }
    } else if (Q8 && warp >= W_VDQ && warp < W_KTMA) {
        // ------------------------------------------------------------------------ V dequantisation -> smem
        const int i = warp - W_VDQ;
        const int ci = lane & 7, slot = lane >> 3;
        int bh_of[4];  // 2 * block + half of this lane's slot in each slot set
#pragma unroll
        for (int ss = 0; ss < 4; ++ss) bh_of[ss] = (int) ((VSLOTS >> (4 * (4 * ss + slot))) & 15);
        for (int t = 0; t < n_tiles; ++t) {
            bool ok = wait_or_fail(&sm.vfull[t % VRAW], (t / VRAW) & 1, p, failed, DEV_ERR_WAIT_FULL);
            ok = ok && (t < 2 || wait_or_fail(&sm.v_free[t & 1], ((t >> 1) - 1) & 1, p, failed, DEV_ERR_WAIT_EMPTY));
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            const uint8_t* raw = sm.vraw + (t % VRAW) * RAWT;
            uint8_t* dst = sm.v[t & 1];
            if constexpr (KT == KT_Q4) {
                // 4 rounds of 8 consecutive cells x 4 whole blocks per warp (16 rounds per tile over the 4 warps);
                // round i + 4m: cells 8 (i + 4 (m % 2)) .. +7, block set m / 2 (first nibble words 0-3 mod 4);
                // two rounds at a time, their loads first
#pragma unroll 1
                for (int m0 = 0; m0 < 4; m0 += 2) {
                    uint32_t W[2][5];
                    __half dh[2];
                    const int blk = (int) ((V4SLOTS >> (3 * (4 * (m0 >> 1) + slot))) & 7);
                    const int qb = 18 * blk + 2, sh = (qb & 3) * 8;
#pragma unroll
                    for (int mm = 0; mm < 2; ++mm) {
                        const uint8_t* rowp = raw + (8 * (i + 4 * mm) + ci) * RAWROW;
                        const uint32_t* w32 = reinterpret_cast<const uint32_t*>(rowp + (qb & ~3));
#pragma unroll
                        for (int k = 0; k < 4; ++k) W[mm][k] = w32[k];
                        W[mm][4] = sh ? w32[4] : 0u;
                        dh[mm] = *reinterpret_cast<const __half*>(rowp + 18 * blk);
                    }
#pragma unroll
                    for (int mm = 0; mm < 2; ++mm) {
                        const int r = 8 * (i + 4 * mm) + ci;
                        const __half2 d2 = __halves2half2(dh[mm], dh[mm]);
                        uint32_t lo[8], hi[8];
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            n4_to_f16(__funnelshift_r(W[mm][k], W[mm][k + 1], sh), d2, lo[2 * k], lo[2 * k + 1],
                                      hi[2 * k], hi[2 * k + 1]);
                        // values 0-15 at dims 32 blk .. + 15 (units u0, u0 + 1), 16-31 at units u0 + 2, u0 + 3
                        const int u0 = ((32 * blk) & 63) >> 3;
                        uint8_t* rowd = dst + ((32 * blk) >> 6) * (TILE * 128) + r * 128;
                        *reinterpret_cast<uint4*>(rowd + ((u0 ^ (r & 7)) << 4)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                        *reinterpret_cast<uint4*>(rowd + (((u0 + 1) ^ (r & 7)) << 4)) =
                            make_uint4(lo[4], lo[5], lo[6], lo[7]);
                        *reinterpret_cast<uint4*>(rowd + (((u0 + 2) ^ (r & 7)) << 4)) =
                            make_uint4(hi[0], hi[1], hi[2], hi[3]);
                        *reinterpret_cast<uint4*>(rowd + (((u0 + 3) ^ (r & 7)) << 4)) =
                            make_uint4(hi[4], hi[5], hi[6], hi[7]);
                    }
                }
            } else {
            // all 8 rounds' loads first, then the conversions and stores (shared loads are not moved past
            // shared stores). Round i + 4m: cells 8 (i + 4 (m % 2)) .. +7, slot set m / 2.
#pragma unroll 1
            for (int m0 = 0; m0 < 8; m0 += 4) {
            uint32_t W[4][5];
            __half dh[4];
#pragma unroll
            for (int mm = 0; mm < 4; ++mm) {
                const int r = 8 * (i + 4 * (mm & 1)) + ci;
                const int bh = m0 ? bh_of[2 + (mm >> 1)] : bh_of[mm >> 1], blk = bh >> 1, hf = bh & 1;
                const uint8_t* rowp = raw + r * RAWROW;
                const int qb = 34 * blk + 2 + 16 * hf;  // first quant byte
                const uint32_t* w32 = reinterpret_cast<const uint32_t*>(rowp + (qb & ~3));
#pragma unroll
                for (int k = 0; k < 4; ++k) W[mm][k] = w32[k];
                W[mm][4] = (qb & 3) ? w32[4] : 0u;
                dh[mm] = *reinterpret_cast<const __half*>(rowp + 34 * blk);
            }
#pragma unroll
            for (int mm = 0; mm < 4; ++mm) {
                const int r = 8 * (i + 4 * (mm & 1)) + ci;
                const int bh = m0 ? bh_of[2 + (mm >> 1)] : bh_of[mm >> 1], blk = bh >> 1, hf = bh & 1;
                const int sh = ((34 * blk + 2 + 16 * hf) & 3) * 8;
                const __half2 d2 = __halves2half2(dh[mm], dh[mm]);
                uint32_t o8[8];
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    q4_to_f16(__funnelshift_r(W[mm][k], W[mm][k + 1], sh), d2, o8[2 * k], o8[2 * k + 1]);
                const int dim0 = 32 * blk + 16 * hf, u0 = (dim0 & 63) >> 3;
                uint8_t* d0 = dst + (dim0 >> 6) * (TILE * 128) + r * 128 + ((u0 ^ (r & 7)) << 4);
                *reinterpret_cast<uint4*>(d0) = make_uint4(o8[0], o8[1], o8[2], o8[3]);
                // unit u0 + 1 (u0 even): the swizzled address XOR 16
                *reinterpret_cast<uint4*>(reinterpret_cast<uintptr_t>(d0) ^ 16) = make_uint4(o8[4], o8[5], o8[6], o8[7]);
            }
            }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&sm.v_full[t & 1]);
                mbar_arrive(&sm.vempty[t % VRAW]);
            }
        }
    } else {
        // ------------------------------------------------------------------------ softmax (warps 0-3)
        const int c = 32 * warp + lane;  // cell of the block = TMEM lane
        const uint32_t lane_addr = tmem + ((uint32_t) (32 * warp) << 16);
        const float scl = p.scale_log2;
        // a dense mask broadcast over the heads whose rows for this chunk are <= 4 consecutive queries: each cell
        // loads those few values once per block (not one per row); the row addresses are formed in the branch that
        // reads them, so that they hold no registers across the loop
        const int q_first = sm.row_qi[0], q_last = sm.row_qi[max(rows - 1, 0)];
        const int dm_n = p.mask && p.m_ne2 == 1 && q_last - q_first < 4 ? q_last - q_first + 1 : 0;
        const int64_t min_pos = p.pos0 + sm.row_qi[0];
        float l[N];
#pragma unroll
        for (int r = 0; r < N; ++r) l[r] = 0.0f;
        if (threadIdx.x < N) {
            sm.mrow[threadIdx.x] = -INFINITY;
            sm.nref[threadIdx.x] = threadIdx.x < rows ? INFINITY : -INFINITY;
        }
        named_bar_sync(1, 128);
        bool ok = true;
        for (int j = 0; j < nblk; ++j) {
            ok = ok && wait_or_fail(&sm.s_full[j & 1], (j >> 1) & 1, p, failed, DEV_ERR_WAIT_FULL);
            // x = score (log2 units) - the row's max (+inf for a visible cell of a row that has seen nothing yet);
            // -inf where not visible and past the rows. With_ref false: the scores themselves.
            const int64_t key0 = key_begin + (int64_t) j * BLK, key = key0 + c;
            auto scores = [&](float (&x)[N], bool with_ref) {
                uint32_t sv[N];
                tmem_ld<N>(lane_addr + TM_S + (j & 1) * N, sv);
                tmem_wait_ld();
                const bool plain = !p.mask && !p.has_softcap && p.ring == 0 && key0 + BLK <= key_end &&
                                   (!p.causal || (key0 >= p.kv_lo && key0 + BLK - 1 <= min_pos));
                if (plain && with_ref) {
                    // pairs of rows on the packed f32x2 pipe: x = s * scale + nref
                    const uint64_t sc2 = f2pack(scl, scl);
#pragma unroll
                    for (int r = 0; r < N; r += 4) {
                        const float4 nr = *reinterpret_cast<const float4*>(sm.nref + r);
                        f2unpack(ffma2(f2pack(__uint_as_float(sv[r]), __uint_as_float(sv[r + 1])), sc2, f2pack(nr.x, nr.y)),
                                 x[r], x[r + 1]);
                        f2unpack(ffma2(f2pack(__uint_as_float(sv[r + 2]), __uint_as_float(sv[r + 3])), sc2,
                                       f2pack(nr.z, nr.w)),
                                 x[r + 2], x[r + 3]);
                    }
                } else if (!p.mask && !p.has_softcap) {
                    // causal bounds only: row r sees cells [kv_lo, pos0 + qi_r] below the split's end; with the MTP
                    // head's ring, slot `key` holds cell end - ((end - key) mod ring) (one mapping per slot, not per
                    // row) and row r also needs that cell inside its window (> pos0 + qi_r - ring)
                    int64_t cell = key;
                    if (p.causal && p.ring > 0) {
                        const int64_t end = p.pos0 + p.n_q - 1;
                        cell = end - (((end - key) % p.ring) + p.ring) % p.ring;
                    }
                    const bool in = key < key_end && (!p.causal || cell >= p.kv_lo);
#pragma unroll
                    for (int r = 0; r < N; ++r) {
                        const int64_t pos = p.pos0 + sm.row_qi[r];
                        const bool vis = r < rows && in && (!p.causal || (cell <= pos && (p.ring == 0 || cell > pos - p.ring)));
                        x[r] = vis ? fmaf(__uint_as_float(sv[r]), scl, with_ref ? sm.nref[r] : 0.0f) : -INFINITY;
                    }
                } else if (!p.has_softcap && p.ring == 0 && dm_n > 0) {
                    // a dense mask broadcast over the heads (klein's graph passes one): its values for this cell in
                    // the chunk's <= 4 query rows, 0 almost everywhere (then only the scale applies), plus the causal
                    // bounds when given; masked_score's arithmetic
                    const bool in = key < key_end && (!p.causal || key >= p.kv_lo);
                    const int dm_q0 = sm.row_qi[0];
                    const char* dm_cell = p.mask + (int64_t) dm_q0 * p.m_nb1 + (b % p.m_ne3) * p.m_nb3 + key * 2;
                    float mq[4];
                    bool zero = true;
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        mq[u] = (u < dm_n && in) ? __half2float(*reinterpret_cast<const __half*>(dm_cell + u * p.m_nb1))
                                                 : 0.0f;
                        zero = zero && mq[u] == 0.0f;
                    }
                    if (zero && in && with_ref && (!p.causal || key <= min_pos)) {
                        // visible to every row with nothing added: the unmasked form (rows past the chunk's end have
                        // a reference of -inf)
                        const uint64_t sc2 = f2pack(scl, scl);
#pragma unroll
                        for (int r = 0; r < N; r += 4) {
                            const float4 nr = *reinterpret_cast<const float4*>(sm.nref + r);
                            f2unpack(ffma2(f2pack(__uint_as_float(sv[r]), __uint_as_float(sv[r + 1])), sc2, f2pack(nr.x, nr.y)),
                                     x[r], x[r + 1]);
                            f2unpack(ffma2(f2pack(__uint_as_float(sv[r + 2]), __uint_as_float(sv[r + 3])), sc2,
                                           f2pack(nr.z, nr.w)),
                                     x[r + 2], x[r + 3]);
                        }
                        return;
                    }
#pragma unroll
                    for (int r = 0; r < N; ++r) {
                        float v = -INFINITY;
                        if (r < rows && in && (!p.causal || key <= p.pos0 + sm.row_qi[r])) {
                            v = __uint_as_float(sv[r]) * scl;
                            if (!zero) {
                                const int u = sm.row_qi[r] - dm_q0;
                                const float m = u == 0 ? mq[0] : u == 1 ? mq[1] : u == 2 ? mq[2] : mq[3];
                                const float mv = sm.row_slope[r] * m;
                                if (mv == -INFINITY) v = -INFINITY;
                                else v += mv * LOG2E;
                            }
                        }
                        x[r] = (v == -INFINITY || !with_ref) ? v : v + sm.nref[r];
                    }
                } else if (!p.has_softcap && p.ring == 0) {
                    // a dense mask of another shape: one f16 load per (cell, row) through the row's mask pointer
                    const bool in = key < key_end && (!p.causal || key >= p.kv_lo);
#pragma unroll
                    for (int r = 0; r < N; ++r) {
                        float v = -INFINITY;
                        if (r < rows && in && (!p.causal || key <= p.pos0 + sm.row_qi[r])) {
                            const float mv = sm.row_slope[r] * __half2float(sm.row_mask[r][key]);
                            if (mv != -INFINITY) {
                                v = __uint_as_float(sv[r]) * scl;
                                v += mv * LOG2E;
                            }
                        }
                        x[r] = (v == -INFINITY || !with_ref) ? v : v + sm.nref[r];
                    }
                } else {
                    const bool in = key < key_end;
#pragma unroll
                    for (int r = 0; r < N; ++r) {
                        const float ms = (r < rows && in) ? masked_score(p, __uint_as_float(sv[r]), key, sm.row_qi[r],
                                                                         sm.row_h[r], b, sm.row_slope[r])
                                                          : -INFINITY;
                        x[r] = (ms == -INFINITY || !with_ref) ? ms : ms + sm.nref[r];
                    }
                }
            };
            float x[N];
            if (ok) {
                tc_fence_after();
                scores(x, true);
            } else {
#pragma unroll
                for (int r = 0; r < N; ++r) x[r] = -INFINITY;
            }
            float xm = -INFINITY;
#pragma unroll
            for (int r = 0; r < N; r += 2) xm = max3f(xm, x[r], x[r + 1]);
            // one barrier reduction in the common case: does anyone leave, or see a cell more than 2^8 above its
            // row's reference? (P is computed against the reference, so values up to 2^8 are fine in f16)
            if (bar_red_or(1, 128, !ok || xm > THRESH)) {
                if (bar_red_or(1, 128, !ok)) {
                    ok = false;
                    break;
                }
                // raise: the block's scores again (S_j is still in TMEM), their maxima per row, 16 rows at a time
                scores(x, false);
#pragma unroll
                for (int h16 = 0; h16 < N / 16; ++h16) {
                    float v[16];
#pragma unroll
                    for (int r = 0; r < 16; ++r) v[r] = x[16 * h16 + r];
                    const float wm = warp_rows_reduce<16, true>(v, lane);
                    if (lane < 16) sm.red[warp][16 * h16 + lane] = wm;
                }
                named_bar_sync(1, 128);
                if (threadIdx.x < N) {
                    const int r = threadIdx.x;
                    const float bm = fmaxf(fmaxf(sm.red[0][r], sm.red[1][r]), fmaxf(sm.red[2][r], sm.red[3][r]));
                    const float mo = sm.mrow[r], mn = fmaxf(mo, bm);
                    sm.alpha[r] = mn == mo ? 1.0f : exp2f(mo - mn);
                    sm.mrow[r] = mn;
                    if (r < rows) sm.nref[r] = mn == -INFINITY ? INFINITY : -mn;
                }
                named_bar_sync(1, 128);  // new maxima visible; sm.red read before it is written again
                bool any_alpha = false;
#pragma unroll
                for (int r = 0; r < N; ++r) {
                    const float a = sm.alpha[r];
                    any_alpha |= a != 1.0f;
                    l[r] *= a;
                    x[r] = x[r] == -INFINITY ? -INFINITY : x[r] + sm.nref[r];
                }
                if (j > 0 && any_alpha) {
                    // O^T holds PV of blocks 0..j-1: rescale its columns once PV_{j-1} has completed
                    ok = wait_or_fail(&sm.p_free[(j - 1) & 1], ((j - 1) >> 1) & 1, p, failed, DEV_ERR_WAIT_FULL);
                    if (ok) {
                        tc_fence_after();
                        // 16 columns at a time: the scores and sums stay in registers meanwhile
#pragma unroll 1
                        for (int c16 = 0; c16 < 2 * N; c16 += 16) {
                            uint32_t ov[16];
                            tmem_ld16(lane_addr + TM_O + c16, ov);
                            tmem_wait_ld();
                            const float* al = sm.alpha + (c16 % N);
#pragma unroll
                            for (int e = 0; e < 16; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * al[e]);
                            tmem_st16(lane_addr + TM_O + c16, ov);
                        }
                        tmem_wait_st();
                    }
                }
            }
            // P^T into buffer j % 2 once PV_{j-2} has read it
            ok = ok && (j < 2 || wait_or_fail(&sm.p_free[j & 1], ((j >> 1) - 1) & 1, p, failed, DEV_ERR_WAIT_EMPTY));
            uint8_t* pb = sm.p[j & 1][c >> 6];
            const int cc = c & 63;
            if (ok) {
#pragma unroll
                for (int r = 0; r < N; ++r) {
                    x[r] = ex2_ftz(x[r]);
                    l[r] += x[r];
                }
#pragma unroll
                for (int r = 0; r < N; ++r)
                    if (r < rows)
                        *reinterpret_cast<__half*>(pb + r * 128 + (((cc >> 3) ^ (r & 7)) << 4) + (cc & 7) * 2) =
                            __float2half_rn(x[r]);
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.p_full[j & 1]);
        }
        // row sums over the block's cells, then over the 4 warps
        named_bar_sync(1, 128);
#pragma unroll
        for (int h16 = 0; h16 < N / 16; ++h16) {
            float v[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) v[r] = l[16 * h16 + r];
            const float wl = warp_rows_reduce<16, false>(v, lane);
            if (lane < 16) sm.red[warp][16 * h16 + lane] = wl;
        }
        named_bar_sync(1, 128);
        if (ok && nblk > 0) ok = wait_or_fail(&sm.o_done, 0, p, failed, DEV_ERR_WAIT_FULL);
        if (!*failed) {
            const int64_t part_row0 =
                ((((int64_t) b * p.n_head_kv + hk) * p.n_row_chunks + chunk) * p.n_splits + split) * N;
#pragma unroll 1
            for (int hh = 0; hh < 2; ++hh) {
                // dims [128 hh, 128 hh + 128) of O^T are on the lanes: this thread holds dim 128 hh + c
                uint32_t ov[N];
#pragma unroll
                for (int r = 0; r < N; ++r) ov[r] = 0u;
                if (ok && nblk > 0) {
                    tc_fence_after();
                    tmem_ld<N>(lane_addr + TM_O + hh * N, ov);
                    tmem_wait_ld();
                }
                const int d = 128 * hh + c;
#pragma unroll
                for (int r = 0; r < N; ++r) {
                    if (r >= rows) break;
                    const float L = (sm.red[0][r] + sm.red[1][r]) + (sm.red[2][r] + sm.red[3][r]);
                    const float M = nblk > 0 ? sm.mrow[r] : -INFINITY;
                    const float O = __uint_as_float(ov[r]);
                    if (p.n_splits == 1 && !p.push && !p.xchg) {
                        store_row(p, sm.row_qi[r], sm.row_h[r], b, d, O, M, L);
                    } else {
                        p.o_part[(part_row0 + r) * D + d] = O;
                        if (d == 0) {
                            p.ml_part[(part_row0 + r) * 2 + 0] = M;
                            p.ml_part[(part_row0 + r) * 2 + 1] = L;
                        }
                    }
                }
            }
        }
    }
    }
    // every MMA has completed before the columns are released (o_done is committed on every path)
    if (warp == W_SMMA) {
        mbar_wait(&sm.o_done, 0, p.wait_ns);
        mbar_wait(&sm.s_done, 0, p.wait_ns);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == W_SMMA) tmem_dealloc(tmem, R_::TMEM_COLS);
    if (p.xchg) exchange_tail<N, THREADS / 32>(p, reinterpret_cast<float*>(smem_raw));
}

}  // namespace tc

// ------------------------------------------------------------------------------------------------ launch

template <typename Kern>
cudaError_t set_smem_once(Kern kern, size_t smem, bool (&done)[64]) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64 && done[dev]) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e == cudaSuccess && dev >= 0 && dev < 64) done[dev] = true;
    return e;
}

template <int N, int KT>
cudaError_t launch_tc(const FaStreamParams& p, const CUtensorMap& tmK, const CUtensorMap& tmV, cudaStream_t stream) {
    static bool attr_done[64] = {};
    auto kern = tc::fa_stream_tc_kernel<N, KT>;
    const size_t smem = sizeof(tc::Smem<N, KT>);
    const bool first = [&] {
        int dev = 0;
        return cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || !attr_done[dev];
    }();
    if constexpr (KT != tc::KT_F16) {
        // the register split assumes the launch holds exactly REG_LAUNCH per thread: with fewer, a warpgroup's raise
        // would wait for registers that never come, so such a build is refused before its first launch
        if (first) {
            cudaFuncAttributes fa{};
            const cudaError_t ea = cudaFuncGetAttributes(&fa, kern);
            if (ea != cudaSuccess) return ea;
            if (fa.numRegs != (int) tc::Roles<true>::REG_LAUNCH) return cudaErrorInvalidConfiguration;
        }
    }
    cudaError_t e = set_smem_once(kern, smem, attr_done);
    if (e != cudaSuccess) return e;
    dim3 grid(p.n_splits, p.n_head_kv, p.n_row_chunks * p.ne3);
    if (p.xchg) {
        // the in-kernel exchange waits on a grid barrier: every CTA must be resident at once
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = grid;
        cfg.blockDim = dim3(tc::Roles<KT != tc::KT_F16>::THREADS);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, kern, tmK, tmV, p);
    }
    kern<<<grid, tc::Roles<KT != tc::KT_F16>::THREADS, smem, stream>>>(tmK, tmV, p);
    e = cudaGetLastError();
    if (e != cudaSuccess || (p.n_splits == 1 && !p.push)) return e;
    dim3 cgrid(p.R, p.n_head_kv, p.ne3);
    fa_combine_kernel<N><<<cgrid, MERGE_THREADS, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_fa_stream_tc(const FaStreamParams& p, int rpc, int kv_type, const CUtensorMap& tmK,
                                const CUtensorMap& tmV, cudaStream_t stream) {
    using namespace tc;
    if (kv_type == 8) return rpc <= 16 ? launch_tc<16, KT_Q8>(p, tmK, tmV, stream) : launch_tc<32, KT_Q8>(p, tmK, tmV, stream);
    if (kv_type == 2) return rpc <= 16 ? launch_tc<16, KT_Q4>(p, tmK, tmV, stream) : launch_tc<32, KT_Q4>(p, tmK, tmV, stream);
    return rpc <= 16 ? launch_tc<16, KT_F16>(p, tmK, tmV, stream) : launch_tc<32, KT_F16>(p, tmK, tmV, stream);
}

size_t fa_stream_tc_smem_bytes(int rpc, int kv_type) {
    using namespace tc;
    if (kv_type == 8) return rpc <= 16 ? sizeof(Smem<16, KT_Q8>) : sizeof(Smem<32, KT_Q8>);
    if (kv_type == 2) return rpc <= 16 ? sizeof(Smem<16, KT_Q4>) : sizeof(Smem<32, KT_Q4>);
    return rpc <= 16 ? sizeof(Smem<16, KT_F16>) : sizeof(Smem<32, KT_F16>);
}

cudaError_t launch_lse_combine(const float* o_parts, const float* ml_parts, int64_t stride, int n_parts, int64_t rows, int Dd,
                               float* dst, cudaStream_t stream, int* flags, int64_t slot_set_floats, int* err,
                               uint64_t wait_ns) {
    if (rows <= 0) return cudaSuccess;
    lse_combine_kernel<<<(unsigned) rows, MERGE_THREADS, 0, stream>>>(o_parts, ml_parts, stride, n_parts, rows, Dd, dst,
                                                                        flags, slot_set_floats, err, wait_ns);
    return cudaGetLastError();
}

}  // namespace kb
