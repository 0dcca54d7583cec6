// Gated DeltaNet, chunked form for prompt prefill: GGML_OP_GATED_DELTA_NET over many tokens with the scalar
// gate, on the 5th-generation tensor cores. Same result as the token-by-token recurrence of
// ggml_compute_forward_gated_delta_net_one_chunk (ggml-cpu/ops.cpp:11123-11275), reorganised per chunk of
// C = 64 tokens. With the state S[i][j] (= ggml's M[j][i]) at the start of a chunk, G_t = g_1 + ... + g_t and
// Gamma_t = exp(G_t) within the chunk, the delta written at token s is
//     u_s = beta_s (v_s - Gamma_s S^T k_s - sum_{r<s} e^{G_s - G_r} (k_s.k_r) u_r)
// so, for the whole chunk (the WY / UT form):
//     U  = U~ - W S,    U~ = T^-1 diag(beta) V,   W = T^-1 diag(beta Gamma) K,
//                       T  = I + A,  A[s][r] = beta_s e^{G_s - G_r} k_s.k_r  (r < s)
//     O  = diag(Gamma) Q S + A_qk U,               A_qk[t][s] = e^{G_t - G_s} q_t.k_s  (s <= t)
//     S' = Gamma_C S + K~^T U,                    K~[s] = e^{G_C - G_s} k_s
// and o_t is scaled by 1/sqrt(128) as in the recurrence. This is the recurrence unrolled exactly, not an
// approximation of it.
//
// Two kernels:
//   prep  (one CTA per value head, chunk and sequence; all in parallel): [K;Q] K^T, the unit-triangular inverse
//         T^-1 (CUDA cores, 16x16 blocks), then W and U~, written with A_qk and G as one record per chunk.
//   state (one CTA per value head and sequence; sequential over chunks): the f32 state lives in TMEM; per chunk
//         X = W S, U = U~ - X, dS = K~^T U, O = Q~ S + A_qk U, S <- Gamma_C S + dS. Warps: 8 epilogue (TMEM
//         lanes = value dims, two column halves), one MMA issuer, one bulk loader of the records, four
//         converters building the scaled Q~ / K~ operands from the f32 rows. Outputs leave by TMA stores.
// The transposed products put the 128 value (or key) columns on the 128 TMEM lanes: every product is M = 128.
//
// Precision: the reference computes in f32. Products whose rounding reaches the state or the output take their
// operands as f16 pairs x = hi + lo (hi = f16(x), lo = f16(x - hi)) and run three MMAs (hi.hi + hi.lo + lo.hi,
// f32 accumulation): [K;Q] K^T, U~, Q~ S, A_qk U and K~^T U. W S runs once in f16: its error is removed again
// by the same chunk's K~^T U (the delta rule rewrites what it reads). A numerical model of exactly this scheme
// against an f64 recurrence over 4096 tokens gave 1.3e-6 (state) and 1.8e-5 (output) max relative error; with
// plain f16 operands it was 7e-4 and 1.1e-3.
#include "kb_common.cuh"
#include "kb_gdn.h"
#include "kb_tcgen05.cuh"

namespace kb {

namespace {

constexpr int S = 128;        // key / value head dim
constexpr int C = GDN_CHUNK;  // tokens per chunk

// byte offset of the 16-byte unit u (elements [8u, 8u + 8)) of row `row` in a [rows][64] 16-bit tile with the
// 128-byte swizzle (the tile starts 1024-aligned)
__device__ __forceinline__ uint32_t sw_unit(int row, int u) { return (uint32_t) (row * 128 + ((u ^ (row & 7)) << 4)); }
// byte offset of the 16-bit element (row, col) of such a tile
__device__ __forceinline__ uint32_t sw_off(int row, int col) { return sw_unit(row, col >> 3) + ((col & 7) << 1); }

// f32 [64][64] row-major in shared memory with the float4 units of row r XOR-swizzled by r % 16: rows and
// columns both walk without bank conflicts
__device__ __forceinline__ float4& fm4(float* m, int r, int u4) {
    return reinterpret_cast<float4*>(m)[r * 16 + (u4 ^ (r & 15))];
}
__device__ __forceinline__ float& fm1(float* m, int r, int c) {
    return m[r * 64 + (((c >> 2) ^ (r & 15)) << 2) + (c & 3)];
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// x rounded to 11 significant bits (Veltkamp's splitting with the factor 2^13 + 1); exact in f16 for the
// magnitudes here. The intrinsics keep the compiler from contracting the three steps into an FMA.
__device__ __forceinline__ float hi11(float x) {
    const float t = __fmul_rn(x, 8193.0f);
    return __fsub_rn(t, __fsub_rn(t, x));
}

// x = hi + lo as two f16 values for two inputs packed as half2: hi = x to 11 bits, lo = f16(x - hi). One packed
// conversion per pair and part (conversions are the scarce pipe here, not FP32 arithmetic).
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const float h0 = hi11(x0), h1 = hi11(x1);
    hi = h2u(__floats2half2_rn(h0, h1));
    lo = h2u(__floats2half2_rn(__fsub_rn(x0, h0), __fsub_rn(x1, h1)));
}
__device__ __forceinline__ uint32_t split2_hi(float x0, float x1) { return h2u(__floats2half2_rn(hi11(x0), hi11(x1))); }
__device__ __forceinline__ uint32_t split2_lo(float x0, float x1) {
    return h2u(__floats2half2_rn(__fsub_rn(x0, hi11(x0)), __fsub_rn(x1, hi11(x1))));
}

__device__ __forceinline__ void split8(const float (&x)[8], uint4& hi, uint4& lo) {
    split2(x[0], x[1], hi.x, lo.x);
    split2(x[2], x[3], hi.y, lo.y);
    split2(x[4], x[5], hi.z, lo.z);
    split2(x[6], x[7], hi.w, lo.w);
}

__device__ __forceinline__ void load8(const char* src, float (&x)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(src), b = *reinterpret_cast<const float4*>(src + 16);
    x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
}

__device__ __forceinline__ bool wait_or_fail(uint64_t* bar, uint32_t parity, const GdnChunkParams& p, volatile int* failed,
                                             int code) {
    if (*failed) return false;
    if (mbar_wait(bar, parity, p.wait_ns)) return true;
    record_error(p.err, code);
    *failed = 1;
    return false;
}

// ================================================================================================ prep kernel

constexpr int PREP_THREADS = 160;                 // warps 0-3 compute (TMEM lanes 0-127), warp 4 issues the MMAs
constexpr uint32_t PT_KQ = 0, PT_W = 64, PT_U = 128;  // TMEM columns: [K;Q]K^T, W^T, U~^T (128 x 64 f32 each)
constexpr float LOG2E = 1.4426950408889634f;

// 96 KiB in three regions whose contents change between phases (two CTAs fit on an SM):
//   r0: [K;Q] hi, [2 key-dim chunks][128 rows: K 0-63, Q 64-127][64]. After [K;Q]K^T the Q rows (r0 + 8K and
//       r0 + 24K) hold the A_qk hi / lo images until they are stored; then r0 + 8K holds the inverse's block
//       products and after them T^-1 diag(beta) lo.
//   r1: [K;Q] lo. Then A f32 [64][64] at r1 and T^-1 f32 at r1 + 16K; once A is consumed, T^-1 diag(beta Gamma)
//       at r1 and T^-1 diag(beta) hi at r1 + 8K. Finally U~ [64 s][128 j] f32 for the record.
//   r2: V hi [2 value-dim chunks][64 rows][64] at r2, lo at r2 + 16K; then the W image for the record.
struct PrepSmem {
    uint8_t r0[32768];
    uint8_t r1[32768];
    uint8_t r2[32768];
    float G[C], beta[C];
    uint64_t bar;
    uint32_t tmem_base;
    int failed;
};

__device__ __forceinline__ void bulk_store(void* gdst, const void* ssrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(reinterpret_cast<uint64_t>(gdst)),
                 "r"(smem_u32(ssrc)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(PREP_THREADS, 2) gdn_chunk_prep_kernel(const GdnChunkParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    if (smem_u32(smem_raw) & 1023) {
        if (threadIdx.x == 0) record_error(p.err, DEV_ERR_ALIGN);
        return;
    }
    PrepSmem& sm = *reinterpret_cast<PrepSmem*>(smem_raw);
    const GdnParams& in = p.in;
    const int tid = threadIdx.x, warp = tid >> 5;
    // value heads vary fastest, the heads that share a key head next to each other: their K / Q rows come
    // from L2 after the first read
    const int R = in.H_v / in.H_k;
    const int cc = blockIdx.y, seq = blockIdx.z;
    const int hk = (int) blockIdx.x / R, h = hk + ((int) blockIdx.x % R) * in.H_k;
    const int64_t t_base = p.tok0 + (int64_t) cc * C;
    const int n_valid = (int) min((int64_t) C, p.tok0 + p.n_tok - t_base);
    char* rec = p.rec + (((int64_t) seq * in.H_v + h) * p.n_chunks + cc) * GDN_REC_BYTES;
    const char* kbase = in.k + (int64_t) (seq / in.rk3) * in.k_nb3 + (int64_t) hk * in.k_nb1;
    const char* qbase = in.q + (int64_t) (seq / in.rq3) * in.q_nb3 + (int64_t) hk * in.q_nb1;
    const char* vbase = in.v + (int64_t) seq * in.v_nb3 + (int64_t) h * in.v_nb1;

    uint8_t* kq_hi = sm.r0;
    uint8_t* kq_lo = sm.r1;
    uint8_t* v_hi = sm.r2;
    uint8_t* v_lo = sm.r2 + 16384;
    uint8_t* aq_hi = sm.r0 + 8192;
    uint8_t* aq_lo = sm.r0 + 24576;
    float* amat = reinterpret_cast<float*>(sm.r1);          // A, row-major (fm4 layout)
    float* tinv = reinterpret_cast<float*>(sm.r1 + 16384);  // T^-1, row-major (fm4 layout)
    float* ytmp = reinterpret_cast<float*>(sm.r0 + 8192);   // block products of the inverse
    uint8_t* tbg = sm.r1;
    uint8_t* tb_hi = sm.r1 + 8192;
    uint8_t* tb_lo = sm.r0 + 8192;
    float* ust = reinterpret_cast<float*>(sm.r1);
    uint8_t* wst = sm.r2;
    volatile int* failed = &sm.failed;

    if (tid == 0) {
        mbar_init(&sm.bar, 1);
        sm.failed = 0;
        fence_barrier_init();
    }
    if (warp == 4) {
        tmem_alloc(&sm.tmem_base, 256);
        tmem_relinquish();
    }
    if (tid < C) {
        float gv = 0.f, bv = 0.f;  // padding tokens: no decay, no write
        if (tid < n_valid) {
            const int64_t tok = t_base + tid;
            gv = *reinterpret_cast<const float*>(in.g + seq * in.g_nb3 + tok * in.g_nb2 + h * in.g_nb1);
            bv = *reinterpret_cast<const float*>(in.beta + seq * in.b_nb3 + tok * in.b_nb2 + h * in.b_nb1);
        }
        sm.G[tid] = gv;
        sm.beta[tid] = bv;
    }
    // K, Q and V rows as f16 hi/lo, 128B-swizzled; rows past the last token are zero. Each thread converts
    // the 16-byte unit u of rows tid/16 + 8m, with all eight rows' loads in flight at once.
    if (tid < 128) {
        const int u = tid & 15;
#pragma unroll 1
        for (int which = 0; which < 3; ++which) {  // 0 K, 1 Q, 2 V
            float x[8][8];
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                const int r = (tid >> 4) + 8 * m;
#pragma unroll
                for (int e = 0; e < 8; ++e) x[m][e] = 0.f;
                if (r < n_valid) {
                    const int64_t tok = t_base + r;
                    const char* row = which == 0 ? kbase + tok * in.k_nb2 : which == 1 ? qbase + tok * in.q_nb2 : vbase + tok * in.v_nb2;
                    load8(row + u * 32, x[m]);
                }
            }
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                const int r = (tid >> 4) + 8 * m;
                uint4 hi, lo;
                split8(x[m], hi, lo);
                if (which < 2) {
                    const uint32_t off = (u >> 3) * 16384 + sw_unit(r + which * C, u & 7);
                    *reinterpret_cast<uint4*>(kq_hi + off) = hi;
                    *reinterpret_cast<uint4*>(kq_lo + off) = lo;
                } else {
                    const uint32_t off = (u >> 3) * 8192 + sw_unit(r, u & 7);
                    *reinterpret_cast<uint4*>(v_hi + off) = hi;
                    *reinterpret_cast<uint4*>(v_lo + off) = lo;
                }
            }
        }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;

    if (tid == 128) {
        // [K;Q] K^T = (hi + lo)(hi + lo)^T without the lo.lo term: rows 0-63 K K^T, rows 64-127 Q K^T
        constexpr uint32_t id = umma_idesc_f16(0, 128, C, false, false);
        const uint32_t a_hi = smem_u32(kq_hi), a_lo = smem_u32(kq_lo);
        int n = 0;
#pragma unroll
        for (int pass = 0; pass < 3; ++pass) {
            const uint32_t a = pass == 2 ? a_lo : a_hi, b = pass == 1 ? a_lo : a_hi;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                umma_ss(tmem + PT_KQ, smem_desc_sw128(a + off, 16, 1024), smem_desc_sw128(b + off, 16, 1024), id, n++ > 0);
            }
        }
        umma_commit(&sm.bar);
    }
    // running log-decay within the chunk (inclusive prefix sums; warp 0, two tokens per lane)
    if (warp == 0) {
        const int lane = tid & 31;
        const float g0 = sm.G[2 * lane], g1 = sm.G[2 * lane + 1];
        float incl = g0 + g1;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += y;
        }
        sm.G[2 * lane + 1] = incl;
        sm.G[2 * lane] = incl - g1;
    }
    __syncthreads();
    if (tid < C) *reinterpret_cast<float*>(rec + GDN_REC_G + tid * 4) = sm.G[tid];
    // Loops below stay rolled over 8-column pieces: this code runs once per CTA.
    if (tid < 128) {
        wait_or_fail(&sm.bar, 0, p, failed, DEV_ERR_WAIT_FULL);  // on failure every thread still meets every barrier
        tc_fence_after();
        const uint32_t lane_addr = tmem + ((uint32_t) (warp * 32) << 16);
        const int row = tid & (C - 1);  // s for the K K^T rows (warps 0-1), t for the Q K^T rows (warps 2-3)
        const float Grow = sm.G[row], brow = sm.beta[row];
#pragma unroll 1
        for (int pc = 0; pc < C / 8; ++pc) {
            uint32_t v8[8];
            tmem_ld8(lane_addr + PT_KQ + pc * 8, v8);
            tmem_wait_ld();
            float x[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int c = pc * 8 + e;
                const float d = exp2f((Grow - sm.G[c]) * LOG2E) * __uint_as_float(v8[e]);
                x[e] = tid < C ? (c < row ? brow * d : 0.f) : (c <= row ? d : 0.f);
            }
            if (tid < C) {
                // A[s][r] = beta_s e^{G_s - G_r} k_s.k_r (r < s), row-major f32
                fm4(amat, row, 2 * pc) = make_float4(x[0], x[1], x[2], x[3]);
                fm4(amat, row, 2 * pc + 1) = make_float4(x[4], x[5], x[6], x[7]);
            } else {
                // A_qk[t][s] = e^{G_t - G_s} q_t.k_s (s <= t) as hi/lo images [64 t][64 s]
                uint4 hi, lo;
                split8(x, hi, lo);
                *reinterpret_cast<uint4*>(aq_hi + sw_unit(row, pc)) = hi;
                *reinterpret_cast<uint4*>(aq_lo + sw_unit(row, pc)) = lo;
            }
        }
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
        bulk_store(rec + GDN_REC_AQ_HI, aq_hi, 8192);
        bulk_store(rec + GDN_REC_AQ_LO, aq_lo, 8192);
        bulk_commit();
    }

    // T^-1 = (I + A)^-1 in 16 x 16 blocks. Diagonal blocks D_b = (I + A_bb)^-1 by forward substitution, one
    // column per thread ...
    if (tid < C) {
        const int o = (tid >> 4) * 16, c = tid & 15;
        float x[16];
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) {
            float acc = rr == c ? 1.f : 0.f;
#pragma unroll
            for (int q = 0; q < rr; ++q) acc = fmaf(-fm1(amat, o + rr, o + q), x[q], acc);
            x[rr] = acc;
        }
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) fm1(tinv, o + rr, o + c) = x[rr];
    }
    if (tid == 0) bulk_wait_read();  // the A_qk images have been read out: their space holds Y below
    __syncthreads();
    // ... then the blocks below the diagonal by distance l: T_{bi,bj} = -D_bi Y, Y = sum_{k=bj}^{bi-1} A_{bi,k} T_{k,bj}.
    // A task is one row segment (row rr, columns 4 c4 .. 4 c4 + 3) of one block.
#pragma unroll 1
    for (int l = 1; l < 4; ++l) {
        const int n_tasks = (4 - l) * 64;
#pragma unroll 1
        for (int task = tid; task < n_tasks && tid < 128; task += 128) {
            const int bj = task >> 6, bi = bj + l, rr = (task >> 2) & 15, c4 = task & 3;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
            for (int k = bj; k < bi; ++k) {
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                    const float a = fm1(amat, bi * 16 + rr, k * 16 + q);
                    const float4 t = fm4(tinv, k * 16 + q, bj * 4 + c4);
                    acc.x = fmaf(a, t.x, acc.x);
                    acc.y = fmaf(a, t.y, acc.y);
                    acc.z = fmaf(a, t.z, acc.z);
                    acc.w = fmaf(a, t.w, acc.w);
                }
            }
            reinterpret_cast<float4*>(ytmp)[task] = acc;  // Y of block bj, row rr, unit c4
        }
        __syncthreads();
#pragma unroll 1
        for (int task = tid; task < n_tasks && tid < 128; task += 128) {
            const int bj = task >> 6, bi = bj + l, rr = (task >> 2) & 15, c4 = task & 3;
            const float4* y = reinterpret_cast<const float4*>(ytmp) + bj * 64 + c4;  // row q at y[4 q]
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                if (q <= rr) {
                    const float d = fm1(tinv, bi * 16 + rr, bi * 16 + q);
                    const float4 yq = y[4 * q];
                    acc.x = fmaf(d, yq.x, acc.x);
                    acc.y = fmaf(d, yq.y, acc.y);
                    acc.z = fmaf(d, yq.z, acc.z);
                    acc.w = fmaf(d, yq.w, acc.w);
                }
            }
            fm4(tinv, bi * 16 + rr, bj * 4 + c4) = make_float4(-acc.x, -acc.y, -acc.z, -acc.w);
        }
        __syncthreads();
    }
    // B operands [s][64 r]: T^-1 diag(beta) as hi/lo and T^-1 diag(beta Gamma) in f16 (A is consumed: its space
    // takes them). Thread (s, half) writes row s, columns [32 half, 32 half + 32); T^-1 is zero above the diagonal.
    if (tid < 128) {
        const int sr = tid & (C - 1), half = tid >> 6;
#pragma unroll 1
        for (int u = half * 4; u < half * 4 + 4; ++u) {
            const float4 t0 = fm4(tinv, sr, 2 * u), t1 = fm4(tinv, sr, 2 * u + 1);
            const float tt[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
            float x[8], y[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int r = u * 8 + e;
                const float tv = r <= sr ? tt[e] : 0.f;
                x[e] = tv * sm.beta[r];
                y[e] = x[e] * exp2f(sm.G[r] * LOG2E);
            }
            uint4 hi, lo;
            split8(x, hi, lo);
            *reinterpret_cast<uint4*>(tb_hi + sw_unit(sr, u)) = hi;
            *reinterpret_cast<uint4*>(tb_lo + sw_unit(sr, u)) = lo;
            *reinterpret_cast<uint4*>(tbg + sw_unit(sr, u)) = make_uint4(pack_half2(y[0], y[1]), pack_half2(y[2], y[3]),
                                                                         pack_half2(y[4], y[5]), pack_half2(y[6], y[7]));
        }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 128 && !*failed) {
        // W^T = K^T (T^-1 diag(beta Gamma))^T: A = K read MN-major (key-dim chunks 16 KiB apart, 8-row groups
        // 1 KiB apart), B = tbg
        constexpr uint32_t idw = umma_idesc_f16(0, 128, C, true, false);
        const uint32_t k_addr = smem_u32(kq_hi);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
            umma_ss(tmem + PT_W, smem_desc_sw128(k_addr + ks * 2048, 16384, 1024),
                    smem_desc_sw128(smem_u32(tbg) + ks * 32, 16, 1024), idw, ks > 0);
        // U~^T = V^T (T^-1 diag(beta))^T in three passes; V chunks 8 KiB apart
        int n = 0;
#pragma unroll 1
        for (int pass = 0; pass < 3; ++pass) {
            const uint32_t a = smem_u32(pass == 2 ? v_lo : v_hi), b = smem_u32(pass == 1 ? tb_lo : tb_hi);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
                umma_ss(tmem + PT_U, smem_desc_sw128(a + ks * 2048, 8192, 1024), smem_desc_sw128(b + ks * 32, 16, 1024),
                        idw, n++ > 0);
        }
        umma_commit(&sm.bar);
    }
    if (tid < 128) {
        const bool ok = wait_or_fail(&sm.bar, 1, p, failed, DEV_ERR_WAIT_FULL);
        tc_fence_after();
        const uint32_t lane_addr = tmem + ((uint32_t) (warp * 32) << 16);
        // lane = key dim i for W^T: W image [i chunk][64 s][64 i] (B operand of the state kernel, K-major);
        // lane = value dim j for U~^T: U~[s][j] f32
        uint8_t* wdst = wst + (tid >> 6) * 8192;
#pragma unroll 1
        for (int pc = 0; pc < C / 8; ++pc) {
            uint32_t w8[8], u8[8];
            tmem_ld8(lane_addr + PT_W + pc * 8, w8);
            tmem_ld8(lane_addr + PT_U + pc * 8, u8);
            tmem_wait_ld();
            if (ok) {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int sr = pc * 8 + e;
                    *reinterpret_cast<__half*>(wdst + sw_off(sr, tid & 63)) = __float2half_rn(__uint_as_float(w8[e]));
                    ust[sr * S + tid] = __uint_as_float(u8[e]);
                }
            }
        }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        bulk_store(rec + GDN_REC_W, wst, 16384);
        bulk_store(rec + GDN_REC_U, ust, C * S * 4);
        bulk_commit();
        bulk_wait_all();  // shared memory must outlive the stores that read it
    }
    if (warp == 4) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

// ================================================================================================ state kernel

constexpr int EPI_WARPS = 8;  // two per TMEM lane quadrant: warp w owns lanes 32 (w % 4) .. + 31 and column half w / 4
constexpr int W_MMA = EPI_WARPS, W_LOAD = EPI_WARPS + 1, W_CONV = EPI_WARPS + 2;  // + 4 converter warps
constexpr int ST_THREADS = (EPI_WARPS + 6) * 32;
constexpr uint32_t TS_S = 0, TS_DS = 128, TS_X = 256, TS_O = 320, TS_UH = 384, TS_UL = 416, TS_X2 = 448;  // TMEM columns

struct StateSmem {
    uint8_t st_hi[2 * 128 * 128];    // S^T hi (A operand, K-major): [key-dim chunk][128 j][64 i]
    uint8_t st_lo[2 * 128 * 128];
    uint8_t w[2 * C * 128];          // W image [i chunk][64 s][64 i] (B, K-major)
    uint8_t aq[2 * C * 128];         // A_qk hi | lo images [64 t][64 s] (B, K-major)
    uint8_t kt_hi[2 * C * 128];      // K~ [i chunk][64 s][64 i] (B, MN-major)
    uint8_t kt_lo[2 * C * 128];
    uint8_t qt_hi[2 * C * 128];      // Q~ [i chunk][64 t][64 i] (B, K-major)
    uint8_t qt_lo[2 * C * 128];
    float u[C * S];                  // U~ [s][j]
    float ost[C * S];                // the chunk's outputs [t][j], written out by one TMA store
    uint64_t w_full, w_empty, aq_full, aq_empty, u_full, u_empty, kt_full, kt_empty, qt_full, qt_empty;
    uint64_t s_ready, s_lo_ready, x_full, u_ready, ds_full, o_full, o_free, mma_done, ost_free, ost_full;
    uint32_t tmem_base;
    int failed;
};

// 32 state values of row j (key dims [32q, 32q + 32)) into the S^T hi or lo image
template <bool LO>
__device__ __forceinline__ void put_state_row(StateSmem& sm, int j, int q, const float (&x)[32]) {
    uint8_t* img = (LO ? sm.st_lo : sm.st_hi) + (q >> 1) * 16384;
#pragma unroll
    for (int uu = 0; uu < 4; ++uu) {
        const float* y = x + uu * 8;
        const uint4 v = LO ? make_uint4(split2_lo(y[0], y[1]), split2_lo(y[2], y[3]), split2_lo(y[4], y[5]), split2_lo(y[6], y[7]))
                           : make_uint4(split2_hi(y[0], y[1]), split2_hi(y[2], y[3]), split2_hi(y[4], y[5]), split2_hi(y[6], y[7]));
        *reinterpret_cast<uint4*>(img + sw_unit(j, (q & 1) * 4 + uu)) = v;
    }
}

__device__ __forceinline__ void store_state_row(char* base, int type, int64_t elem, const float (&x)[32]) {
#pragma unroll
    for (int e = 0; e < 32; e += 4) {
        if (type == 0) {
            *reinterpret_cast<float4*>(base + (elem + e) * 4) = make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]);
        } else if (type == 1) {
            *reinterpret_cast<uint2*>(base + (elem + e) * 2) = make_uint2(pack_half2(x[e], x[e + 1]), pack_half2(x[e + 2], x[e + 3]));
        } else {
            *reinterpret_cast<uint2*>(base + (elem + e) * 2) = make_uint2(pack_bf162(x[e], x[e + 1]), pack_bf162(x[e + 2], x[e + 3]));
        }
    }
}

// 4-d tiled tensor store from shared memory (bulk group completion)
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* smem_src, int c0, int c1, int c2, int c3) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
}

__global__ void __launch_bounds__(ST_THREADS, 1)
    gdn_chunk_state_kernel(const __grid_constant__ CUtensorMap tmO, const GdnChunkParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    if (smem_u32(smem_raw) & 1023) {
        if (threadIdx.x == 0) record_error(p.err, DEV_ERR_ALIGN);
        return;
    }
    StateSmem& sm = *reinterpret_cast<StateSmem*>(smem_raw);
    const GdnParams& in = p.in;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.x, seq = blockIdx.y;
    const int hk = h % in.H_k;
    const int n_chunks = p.n_chunks;
    const char* rec0 = p.rec + ((int64_t) seq * in.H_v + h) * n_chunks * GDN_REC_BYTES;
    volatile int* failed = &sm.failed;

    if (tid == 0) {
        mbar_init(&sm.w_full, 1);
        mbar_init(&sm.w_empty, 1);
        mbar_init(&sm.aq_full, 1);
        mbar_init(&sm.aq_empty, 1);
        mbar_init(&sm.u_full, 1);
        mbar_init(&sm.u_empty, EPI_WARPS);
        mbar_init(&sm.kt_full, 4);
        mbar_init(&sm.kt_empty, 1);
        mbar_init(&sm.qt_full, 4);
        mbar_init(&sm.qt_empty, 1);
        mbar_init(&sm.s_ready, EPI_WARPS);
        mbar_init(&sm.s_lo_ready, EPI_WARPS);
        mbar_init(&sm.x_full, 1);
        mbar_init(&sm.u_ready, EPI_WARPS);
        mbar_init(&sm.ds_full, 1);
        mbar_init(&sm.o_full, 1);
        mbar_init(&sm.o_free, EPI_WARPS);
        mbar_init(&sm.mma_done, 1);
        mbar_init(&sm.ost_free, 1);
        mbar_init(&sm.ost_full, EPI_WARPS);
        sm.failed = 0;
        fence_barrier_init();
    }
    if (warp == W_MMA) {
        tmem_alloc(&sm.tmem_base, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;

    if (warp == W_LOAD) {
        // ------------------------------------------------------------------------------------ loader
        if (lane == 0) {
            int w_last = -1, u_last = -1, aq_last = -1;  // last chunk whose copy was issued, per buffer
            for (int c = 0; c < n_chunks; ++c) {
                const char* rec = rec0 + (int64_t) c * GDN_REC_BYTES;
                const uint32_t par = (c - 1) & 1;
                if (c > 0 && !wait_or_fail(&sm.w_empty, par, p, failed, DEV_ERR_WAIT_EMPTY)) break;
                mbar_arrive_expect_tx(&sm.w_full, 16384);
                bulk_load(sm.w, rec + GDN_REC_W, 16384, &sm.w_full);
                w_last = c;
                if (c > 0 && !wait_or_fail(&sm.u_empty, par, p, failed, DEV_ERR_WAIT_EMPTY)) break;
                mbar_arrive_expect_tx(&sm.u_full, C * S * 4);
                bulk_load(sm.u, rec + GDN_REC_U, C * S * 4, &sm.u_full);
                u_last = c;
                if (c > 0 && !wait_or_fail(&sm.aq_empty, par, p, failed, DEV_ERR_WAIT_EMPTY)) break;
                mbar_arrive_expect_tx(&sm.aq_full, 16384);
                bulk_load(sm.aq, rec + GDN_REC_AQ_HI, 16384, &sm.aq_full);
                aq_last = c;
            }
            // no copy may still be landing in shared memory when the CTA exits: wait (bounded) for the last ones
            if (w_last >= 0) mbar_wait(&sm.w_full, w_last & 1, p.wait_ns);
            if (u_last >= 0) mbar_wait(&sm.u_full, u_last & 1, p.wait_ns);
            if (aq_last >= 0) mbar_wait(&sm.aq_full, aq_last & 1, p.wait_ns);
        }
    } else if (warp == W_MMA) {
        // ------------------------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t id64 = umma_idesc_f16(0, 128, C, false, false);
            constexpr uint32_t id128 = umma_idesc_f16(0, 128, S, false, true);
            const uint32_t st_hi = smem_u32(sm.st_hi), st_lo = smem_u32(sm.st_lo), w = smem_u32(sm.w);
            const uint32_t qt_hi = smem_u32(sm.qt_hi), qt_lo = smem_u32(sm.qt_lo);
            const uint32_t kt_hi = smem_u32(sm.kt_hi), kt_lo = smem_u32(sm.kt_lo), aq = smem_u32(sm.aq);
            for (int c = 0; c < n_chunks; ++c) {
                const uint32_t par = c & 1;
                if (!wait_or_fail(&sm.s_ready, par, p, failed, DEV_ERR_WAIT_FULL)) break;
                if (!wait_or_fail(&sm.w_full, par, p, failed, DEV_ERR_WAIT_FULL)) break;
                tc_fence_after();
                // X = S^T W^T  (X[j][s] = (W S)[s][j]), the two key-dim halves in separate accumulators: two
                // chains of 4 MMAs complete sooner than one of 8
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    umma_ss(tmem + ((kk >> 2) ? TS_X2 : TS_X),
                            smem_desc_sw128(st_hi + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                            smem_desc_sw128(w + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024), id64, (kk & 3) > 0);
                umma_commit(&sm.x_full);
                umma_commit(&sm.w_empty);
                // O = S^T Q~^T, three passes (O of the previous chunk must have been read out)
                if (c > 0 && !wait_or_fail(&sm.o_free, (c - 1) & 1, p, failed, DEV_ERR_WAIT_EMPTY)) break;
                if (!wait_or_fail(&sm.s_lo_ready, par, p, failed, DEV_ERR_WAIT_FULL)) break;
                if (!wait_or_fail(&sm.qt_full, par, p, failed, DEV_ERR_WAIT_FULL)) break;
                tc_fence_after();
                int n = 0;
#pragma unroll 1
                for (int pass = 0; pass < 3; ++pass) {
                    const uint32_t a = pass == 2 ? st_lo : st_hi, b = pass == 1 ? qt_lo : qt_hi;
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        umma_ss(tmem + TS_O, smem_desc_sw128(a + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                                smem_desc_sw128(b + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024), id64, n++ > 0);
                }
                umma_commit(&sm.qt_empty);
                // dS^T = U^T K~, three passes; A = U from TMEM, B = K~ MN-major (key-dim chunks 8 KiB apart)
                if (!wait_or_fail(&sm.u_ready, par, p, failed, DEV_ERR_WAIT_FULL)) break;
                if (!wait_or_fail(&sm.kt_full, par, p, failed, DEV_ERR_WAIT_FULL)) break;
                tc_fence_after();
                n = 0;
#pragma unroll 1
                for (int pass = 0; pass < 3; ++pass) {
                    const uint32_t ua = pass == 2 ? TS_UL : TS_UH, b = pass == 1 ? kt_lo : kt_hi;
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        umma_ts(tmem + TS_DS, tmem + ua + ks * 8, smem_desc_sw128(b + ks * 2048, 8192, 1024), id128, n++ > 0);
                }
                umma_commit(&sm.ds_full);
                umma_commit(&sm.kt_empty);
                // O += U^T A_qk^T, three passes
                if (!wait_or_fail(&sm.aq_full, par, p, failed, DEV_ERR_WAIT_FULL)) break;
                tc_fence_after();
#pragma unroll 1
                for (int pass = 0; pass < 3; ++pass) {
                    const uint32_t ua = pass == 2 ? TS_UL : TS_UH, b = aq + (pass == 1 ? 8192 : 0);
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        umma_ts(tmem + TS_O, tmem + ua + ks * 8, smem_desc_sw128(b + ks * 32, 16, 1024), id64, true);
                }
                umma_commit(&sm.o_full);
                umma_commit(&sm.aq_empty);
            }
            // nothing may still run on the tensor core when TMEM is released
            umma_commit(&sm.mma_done);
            mbar_wait(&sm.mma_done, 0, p.wait_ns);
        }
    } else if (warp >= W_CONV) {
        // ------------------------------------------------------------------------------------ converters
        // Q~[t] = e^{G_t} q_t and K~[s] = e^{G_C - G_s} k_s as f16 hi/lo images, from the f32 rows
        const int ct = tid - W_CONV * 32;
        const char* kbase = in.k + (int64_t) (seq / in.rk3) * in.k_nb3 + (int64_t) hk * in.k_nb1;
        const char* qbase = in.q + (int64_t) (seq / in.rq3) * in.q_nb3 + (int64_t) hk * in.q_nb1;
        const int u = ct & 15;  // 16-byte unit of the rows this thread converts: rows ct/16 + 8m
        for (int c = 0; c < n_chunks; ++c) {
            const float* G = reinterpret_cast<const float*>(rec0 + (int64_t) c * GDN_REC_BYTES + GDN_REC_G);
            const int64_t t_base = p.tok0 + (int64_t) c * C;
            const int n_valid = (int) min((int64_t) C, p.tok0 + p.n_tok - t_base);
            const uint32_t par = (c - 1) & 1;
#pragma unroll 1
            for (int which = 0; which < 2; ++which) {  // 0: Q~, 1: K~
                float x[8][8];
#pragma unroll
                for (int m = 0; m < 8; ++m) {
                    const int r = (ct >> 4) + 8 * m;
#pragma unroll
                    for (int e = 0; e < 8; ++e) x[m][e] = 0.f;
                    if (r < n_valid) {
                        const int64_t tok = t_base + r;
                        load8((which == 0 ? qbase + tok * in.q_nb2 : kbase + tok * in.k_nb2) + u * 32, x[m]);
                    }
                }
                const float GC = G[C - 1];
                uint64_t* empty = which == 0 ? &sm.qt_empty : &sm.kt_empty;
                uint64_t* full = which == 0 ? &sm.qt_full : &sm.kt_full;
                if (c > 0 && !wait_or_fail(empty, par, p, failed, DEV_ERR_WAIT_EMPTY)) break;
                uint8_t* hi = which == 0 ? sm.qt_hi : sm.kt_hi;
                uint8_t* lo = which == 0 ? sm.qt_lo : sm.kt_lo;
#pragma unroll
                for (int m = 0; m < 8; ++m) {
                    const int r = (ct >> 4) + 8 * m;
                    const float f = which == 0 ? expf(G[r]) : expf(GC - G[r]);
#pragma unroll
                    for (int e = 0; e < 8; ++e) x[m][e] *= f;
                    uint4 vh, vl;
                    split8(x[m], vh, vl);
                    const uint32_t off = (u >> 3) * 8192 + sw_unit(r, u & 7);
                    *reinterpret_cast<uint4*>(hi + off) = vh;
                    *reinterpret_cast<uint4*>(lo + off) = vl;
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(full);
            }
            if (*failed) break;
        }
    } else {
        // ------------------------------------------------------------------------------------ epilogue
        // thread: value dim j = TMEM lane; column half hf: key dims [64 hf, 64 hf + 64) of the state, chunk
        // tokens [32 hf, 32 hf + 32) of U and O
        const int quad = warp & 3, hf = warp >> 2;
        const int j = quad * 32 + lane;
        const uint32_t lane_addr = tmem + ((uint32_t) (quad * 32) << 16);
        const int64_t row_elem = ((int64_t) h * S + j) * S;  // element (h, j, 0) within a sequence's state
        const bool leader = tid == 0;                         // issues the output stores
        {
            const float* s0 = p.s0 + seq * p.s0_seq_stride + row_elem;
#pragma unroll 1
            for (int qq = 0; qq < 2; ++qq) {
                const int q = 2 * hf + qq;
                float x[32];
                uint32_t r[32];
#pragma unroll
                for (int e = 0; e < 32; e += 4) {
                    const float4 v = *reinterpret_cast<const float4*>(s0 + q * 32 + e);
                    x[e] = v.x, x[e + 1] = v.y, x[e + 2] = v.z, x[e + 3] = v.w;
                }
#pragma unroll
                for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(x[e]);
                tmem_st32(lane_addr + TS_S + q * 32, r);
                put_state_row<false>(sm, j, q, x);
                put_state_row<true>(sm, j, q, x);
            }
            tmem_wait_st();
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&sm.s_ready);
                mbar_arrive(&sm.s_lo_ready);
            }
        }
        const float scale = rsqrtf((float) S);
        for (int c = 0; c < n_chunks; ++c) {
            const uint32_t par = c & 1;
            const char* rec = rec0 + (int64_t) c * GDN_REC_BYTES;
            const float gC = expf(reinterpret_cast<const float*>(rec + GDN_REC_G)[C - 1]);
            const int64_t t_base = p.tok0 + (int64_t) c * C;
            // U = U~ - W S for tokens [32 hf, 32 hf + 32) as hi/lo f16 in TMEM (A operand of the next products)
            if (!wait_or_fail(&sm.x_full, par, p, failed, DEV_ERR_WAIT_FULL)) break;
            tc_fence_after();
            uint32_t xs[32], xs2[32];
            tmem_ld32(lane_addr + TS_X + hf * 32, xs);
            tmem_ld32(lane_addr + TS_X2 + hf * 32, xs2);
            tmem_wait_ld();
            if (!wait_or_fail(&sm.u_full, par, p, failed, DEV_ERR_WAIT_FULL)) break;
            uint32_t uh[16], ul[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int s0i = hf * 32 + 2 * e;
                const float a = sm.u[s0i * S + j] - (__uint_as_float(xs[2 * e]) + __uint_as_float(xs2[2 * e]));
                const float b = sm.u[(s0i + 1) * S + j] - (__uint_as_float(xs[2 * e + 1]) + __uint_as_float(xs2[2 * e + 1]));
                split2(a, b, uh[e], ul[e]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.u_empty);
            tmem_st16(lane_addr + TS_UH + hf * 16, uh);
            tmem_st16(lane_addr + TS_UL + hf * 16, ul);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.u_ready);
            // S <- Gamma_C S + dS in TMEM (f32); the hi image releases the next chunk's X, the lo image follows
            if (!wait_or_fail(&sm.ds_full, par, p, failed, DEV_ERR_WAIT_FULL)) break;
            tc_fence_after();
            const bool last = c == n_chunks - 1;
#pragma unroll 1
            for (int qq = 0; qq < 2; ++qq) {
                const int q = 2 * hf + qq;
                uint32_t ms[32], ds[32];
                tmem_ld32(lane_addr + TS_S + q * 32, ms);
                tmem_ld32(lane_addr + TS_DS + q * 32, ds);
                tmem_wait_ld();
                float x[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    x[e] = fmaf(gC, __uint_as_float(ms[e]), __uint_as_float(ds[e]));
                    ms[e] = __float_as_uint(x[e]);
                }
                if (last) {
                    store_state_row(reinterpret_cast<char*>(p.s_out + seq * p.s_out_seq_stride), 0, row_elem + q * 32, x);
                    if (p.snap)
                        store_state_row(p.snap, p.snap_type, (int64_t) seq * in.H_v * S * S + row_elem + q * 32, x);
                } else {
                    tmem_st32(lane_addr + TS_S + q * 32, ms);
                    put_state_row<false>(sm, j, q, x);
                }
            }
            tmem_wait_st();
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.s_ready);
            if (!last) {
#pragma unroll 1
                for (int qq = 0; qq < 2; ++qq) {
                    const int q = 2 * hf + qq;
                    uint32_t ms[32];
                    tmem_ld32(lane_addr + TS_S + q * 32, ms);
                    tmem_wait_ld();
                    float x[32];
#pragma unroll
                    for (int e = 0; e < 32; ++e) x[e] = __uint_as_float(ms[e]);
                    put_state_row<true>(sm, j, q, x);
                }
                fence_proxy_async_smem();
                tc_fence_before();
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.s_lo_ready);
            // outputs of tokens [32 hf, 32 hf + 32): TMEM -> staging [t][j] -> one TMA store for the chunk
            if (!wait_or_fail(&sm.o_full, par, p, failed, DEV_ERR_WAIT_FULL)) break;
            tc_fence_after();
            uint32_t os[32];
            tmem_ld32(lane_addr + TS_O + hf * 32, os);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.o_free);
            if (leader) {
                bulk_wait_read();  // the previous chunk's store has read the staging buffer
                mbar_arrive(&sm.ost_free);
            }
            if (!wait_or_fail(&sm.ost_free, par, p, failed, DEV_ERR_WAIT_EMPTY)) break;
#pragma unroll
            for (int t = 0; t < 32; ++t) sm.ost[(hf * 32 + t) * S + j] = __uint_as_float(os[t]) * scale;
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.ost_full);
            if (leader) {
                if (!wait_or_fail(&sm.ost_full, par, p, failed, DEV_ERR_WAIT_FULL)) break;
                // rows past the end of this pass's tokens fall outside the map and are not written
                tma_store_4d(&tmO, sm.ost, 0, h, (int) t_base, seq);
                bulk_commit();
            }
        }
        if (leader) bulk_wait_all();  // the last chunk's output store has completed
    }
    tc_fence_before();
    __syncthreads();
    if (warp == W_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

template <typename Kern>
cudaError_t set_smem(Kern kern, size_t smem, bool (&done)[64]) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64 && done[dev]) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e == cudaSuccess && dev >= 0 && dev < 64) done[dev] = true;
    return e;
}

}  // namespace

cudaError_t launch_gdn_prep(const GdnChunkParams& p, cudaStream_t stream) {
    static bool prep_done[64] = {};
    cudaError_t e = set_smem(gdn_chunk_prep_kernel, sizeof(PrepSmem), prep_done);
    if (e != cudaSuccess) return e;
    gdn_chunk_prep_kernel<<<dim3(p.in.H_v, p.n_chunks, p.in.n_seqs), PREP_THREADS, sizeof(PrepSmem), stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_gdn_state(const GdnChunkParams& p, const CUtensorMap& tmO, cudaStream_t stream) {
    static bool state_done[64] = {};
    cudaError_t e = set_smem(gdn_chunk_state_kernel, sizeof(StateSmem), state_done);
    if (e != cudaSuccess) return e;
    gdn_chunk_state_kernel<<<dim3(p.in.H_v, p.in.n_seqs), ST_THREADS, sizeof(StateSmem), stream>>>(tmO, p);
    return cudaGetLastError();
}

cudaError_t launch_gdn_chunked(const GdnChunkParams& p, const CUtensorMap& tmO, cudaStream_t stream) {
    cudaError_t e = launch_gdn_prep(p, stream);
    if (e != cudaSuccess) return e;
    return launch_gdn_state(p, tmO, stream);
}

}  // namespace kb
