// Causal prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM): GGML_OP_FLASH_ATTN_EXT with
// many query tokens over an f16 or bf16 KV cache (klein's prompt chunks; config[2]'s 4,096-token prefill).
//
// One CTA computes a 128-query tile of one head. Roles:
//   warps 0-15 softmax, 4 warpgroups: query row r is TMEM lane r; warpgroup g handles cells [16g, 16g+16)
//              of each block and O dims [64g, 64g+64); they stage Q, run the online softmax, rescale O when
//              needed, and write the normalised output
//   warps 16-17 TMA producers for K and for V (independent chains): 64 cells x 256 dims, 2-deep rings,
//              128-byte swizzle
//   warp 18    MMA issuer (one thread): S_j = Q K_j^T (SS form, 16 MMAs of K=16) into a double-buffered TMEM
//              S, then O += P_{j-1} V_{j-1} (TS form: P from TMEM) — so the QK^T of block j overlaps the
//              softmax of block j-1
// TMEM (512 columns): O 128 x 256 f32 at [0, 256), S_0/S_1 128 x 64 f32 at [256, 384), P_0/P_1 128 x 64
// f16|bf16 (packed two per column) at [384, 448).
//
// Online softmax with a lazy rescale: a row's running max m is only raised (and O, l rescaled) when a block's
// max exceeds it by more than 8 (log2 units); otherwise exponents use the stale m, which O and l share, so the
// final O / l is unchanged. Semantics as ggml_compute_forward_flash_attn_ext_f16_one_chunk
// (ops.cpp:8842-9078): Q rounded to the K type (:8960), scale, softcap, additive mask with -inf skip, causal
// bounds, zero output for rows that see no cell (:9066). P is rounded to V's type for the PV product.
#include "kb_common.cuh"
#include "kb_internal.h"
#include "kb_tcgen05.cuh"

namespace kb {

namespace {

constexpr float LOG2E = 1.4426950408889634f;
constexpr int D = 256;
constexpr int BM = 128;                       // query rows per CTA
constexpr int BN = 64;                        // cells per K/V block
constexpr int QTILE = BM * D * 2;             // 64 KiB: 4 chunks of [128 rows][128 B]
constexpr int KVTILE = BN * D * 2;            // 32 KiB: 4 chunks of [64 cells][128 B]
constexpr int KSTAGE = 3;                     // K ring depth (the K chain is latency-bound: depth sets the rate)
constexpr int NSTAGE = 2;                     // V ring depth and the S / P / PV double buffers
constexpr int SOFTMAX_WGS = 4;                 // softmax warpgroups: each owns 64 / SOFTMAX_WGS cells of a row
constexpr int SOFTMAX_WARPS = 4 * SOFTMAX_WGS;
constexpr int CPT = BN / SOFTMAX_WGS;           // cells per softmax thread per block
constexpr int OPT = D / SOFTMAX_WGS;            // O columns per softmax thread (rescale / epilogue)
constexpr int THREADS = (SOFTMAX_WARPS + 3) * 32;  // + K producer, V producer, MMA issuer
constexpr uint32_t TM_O = 0, TM_S = 256, TM_P = 384;
constexpr float RESCALE_THRESHOLD = 8.0f;     // log2 units: rescale O only when the max grows by > 2^8

struct Smem {
    uint8_t q[QTILE];                          // 1024-aligned (offset 0)
    uint8_t k[KSTAGE][KVTILE];
    uint8_t v[NSTAGE][KVTILE];
    uint64_t k_full[KSTAGE], k_empty[KSTAGE], v_full[NSTAGE], v_empty[NSTAGE];
    uint64_t s_full[NSTAGE], s_free[NSTAGE], p_full[NSTAGE], o_done[NSTAGE];
    __half xmax[2][SOFTMAX_WGS][BM];           // [block parity][group][row]: partial row maxima exchanged per block
    uint32_t tmem_base;
    int failed;
};
// the epilogue's partial row sums [group][row] reuse the K ring, idle once the last PV has completed
static_assert(SOFTMAX_WGS * BM * sizeof(float) <= KVTILE, "row sums fit in a K stage");

__device__ __forceinline__ bool wait_or_fail(uint64_t* bar, uint32_t parity, const FaPrefillParams& p, volatile int* failed,
                                             int code) {
    if (*failed) return false;
    if (mbar_wait(bar, parity, p.wait_ns)) return true;
    record_error(p.err, code);
    *failed = 1;
    return false;
}

// score of one (cell, row) pair in log2 units, -inf when not visible
__device__ __forceinline__ float prefill_score(const FaPrefillParams& p, float x, int64_t key, int qi, const __half* mrow,
                                               float slope) {
    float v = p.has_softcap ? p.softcap_log2 * tanhf(x * p.scale_sc) : x * p.scale_log2;
    if (key >= p.n_kv || qi >= p.n_q) return -INFINITY;
    if (p.causal && (key < p.kv_lo || key > p.pos0 + qi)) return -INFINITY;
    if (mrow) {
        const float mv = slope * __half2float(mrow[key]);
        if (mv == -INFINITY) return -INFINITY;
        v += mv * LOG2E;
    }
    return v;
}

template <int FMT>  // 0 = f16, 1 = bf16 (K, V, and the rounding of Q and P)
__global__ void __launch_bounds__(THREADS, 1)
    fa_prefill_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                      const FaPrefillParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // the swizzled tiles need 1024-byte alignment; the dynamic window starts there (checked, not assumed)
    if (smem_u32(smem_raw) & 1023) {
        if (threadIdx.x == 0) record_error(p.err, DEV_ERR_ALIGN);
        return;
    }
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // heavy (late) query tiles first; consecutive CTAs share the tile and walk the heads (K/V reuse in L2)
    const int tile = p.n_qtiles - 1 - (int) (blockIdx.x / p.n_head);
    const int h = (int) (blockIdx.x % p.n_head), b = (int) blockIdx.y;
    const int hk = h / p.gqa, kb3 = b / p.rk3;
    const int q0 = tile * BM;
    // cells this tile can see: [c_lo, c_hi)
    int64_t c_hi = p.n_kv, c_lo = 0;
    if (p.causal) {
        c_hi = min(c_hi, p.pos0 + q0 + BM);
        c_lo = max((int64_t) 0, p.kv_lo) / BN * BN;
    }
    const int nb = c_hi > c_lo ? (int) ((c_hi - c_lo + BN - 1) / BN) : 0;
    // the heads of a GQA group walk the shared K/V blocks from different starting points, so that they do not
    // all request the same L2 lines at once; block order does not change the result of the online softmax
    const int rot = nb > 0 ? (int) (((int64_t) (h % p.gqa) * nb) / p.gqa) : 0;
    auto block_cell = [&](int j) -> int64_t { return c_lo + (int64_t) ((j + rot) % nb) * BN; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < KSTAGE; ++s) {
            mbar_init(&sm.k_full[s], 1);
            mbar_init(&sm.k_empty[s], 1);
        }
        for (int s = 0; s < NSTAGE; ++s) {
            mbar_init(&sm.v_full[s], 1);
            mbar_init(&sm.v_empty[s], 1);
            mbar_init(&sm.s_full[s], 1);
            mbar_init(&sm.s_free[s], SOFTMAX_WARPS);
            mbar_init(&sm.p_full[s], SOFTMAX_WARPS);
            mbar_init(&sm.o_done[s], 1);
        }
        sm.failed = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(&sm.tmem_base, 512);
        tmem_relinquish();
    }
    // stage Q (rounded to the K type) into the K-major 128B-swizzled layout: 4 chunks of [128 rows][128 B]
    for (int idx = threadIdx.x; idx < BM * (D / 8); idx += THREADS) {
        const int r = idx / (D / 8), u = idx % (D / 8);  // row, 16-byte unit of 8 dims
        const int qi = q0 + r;
        float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (qi < p.n_q) {
            const float4* src = reinterpret_cast<const float4*>(p.q + qi * p.q_nb1 + h * p.q_nb2 + b * p.q_nb3 + u * 32);
            const float4 a = src[0], c = src[1];
            x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = c.x, x[5] = c.y, x[6] = c.z, x[7] = c.w;
        }
        uint4 w;
        if (FMT == 0) {
            w = make_uint4(pack_half2(x[0], x[1]), pack_half2(x[2], x[3]), pack_half2(x[4], x[5]), pack_half2(x[6], x[7]));
        } else {
            w = make_uint4(pack_bf162(x[0], x[1]), pack_bf162(x[2], x[3]), pack_bf162(x[4], x[5]), pack_bf162(x[6], x[7]));
        }
        const int chunk = u >> 3, cu = u & 7;
        *reinterpret_cast<uint4*>(sm.q + chunk * (BM * 128) + r * 128 + ((cu ^ (r & 7)) << 4)) = w;
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    volatile int* failed = &sm.failed;

    if (warp == SOFTMAX_WARPS || warp == SOFTMAX_WARPS + 1) {
        // -------------------------------------------------------------------------------- TMA producers
        // K and V run independent chains: K_j waits only for S_{j-2}, V_j only for PV_{j-2}
        const bool is_v = warp == SOFTMAX_WARPS + 1;
        if (lane == 0 && nb > 0) {
            const CUtensorMap* map = is_v ? &tmV : &tmK;
            tma_prefetch_desc(map);
            const int depth = is_v ? NSTAGE : KSTAGE;
            for (int j = 0; j < nb; ++j) {
                const int s = j % depth;
                const int cell = (int) block_cell(j);
                uint64_t* empty = is_v ? &sm.v_empty[s] : &sm.k_empty[s];
                uint64_t* fullb = is_v ? &sm.v_full[s] : &sm.k_full[s];
                uint8_t* dst = is_v ? sm.v[s] : sm.k[s];
                if (j >= depth && !wait_or_fail(empty, ((j / depth) - 1) & 1, p, failed, DEV_ERR_WAIT_EMPTY)) break;
                mbar_arrive_expect_tx(fullb, KVTILE);
                for (int c = 0; c < D / 64; ++c) tma_load_4d(dst + c * (BN * 128), map, fullb, c * 64, hk, cell, kb3);
            }
        }
    } else if (warp == SOFTMAX_WARPS + 2) {
        // -------------------------------------------------------------------------------- MMA issuer
        if (lane == 0 && nb > 0) {
            constexpr uint32_t idS = umma_idesc_f16(FMT, BM, BN, false, false);
            constexpr uint32_t idO = umma_idesc_f16(FMT, BM, D, false, true);
            const uint32_t q_addr = smem_u32(sm.q);
            auto issue_pv = [&](int i) -> bool {
                const int s = i % NSTAGE;
                if (!wait_or_fail(&sm.p_full[s], (i / NSTAGE) & 1, p, failed, DEV_ERR_WAIT_FULL)) return false;
                if (!wait_or_fail(&sm.v_full[s], (i / NSTAGE) & 1, p, failed, DEV_ERR_WAIT_FULL)) return false;
                tc_fence_after();
                const uint32_t v_addr = smem_u32(sm.v[s]);
#pragma unroll
                for (int ks = 0; ks < BN / 16; ++ks) {
                    // B = V block, MN-major: 64-dim chunks 8 KiB apart (LBO), 8-cell groups 1 KiB apart (SBO)
                    const uint64_t bdesc = smem_desc_sw128(v_addr + ks * 16 * 128, BN * 128, 1024);
                    umma_ts(tmem + TM_O, tmem + TM_P + s * 32 + ks * 8, bdesc, idO, i > 0 || ks > 0);
                }
                umma_commit(&sm.o_done[s]);
                umma_commit(&sm.v_empty[s]);
                return true;
            };
            for (int j = 0; j < nb; ++j) {
                const int s = j % NSTAGE, ks_ = j % KSTAGE;
                if (!wait_or_fail(&sm.k_full[ks_], (j / KSTAGE) & 1, p, failed, DEV_ERR_WAIT_FULL)) break;
                if (j >= NSTAGE && !wait_or_fail(&sm.s_free[s], ((j / NSTAGE) - 1) & 1, p, failed, DEV_ERR_WAIT_EMPTY))
                    break;
                tc_fence_after();
                const uint32_t k_addr = smem_u32(sm.k[ks_]);
#pragma unroll
                for (int c = 0; c < D / 64; ++c) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t adesc = smem_desc_sw128(q_addr + c * (BM * 128) + kk * 32, 16, 1024);
                        const uint64_t bdesc = smem_desc_sw128(k_addr + c * (BN * 128) + kk * 32, 16, 1024);
                        umma_ss(tmem + TM_S + s * BN, adesc, bdesc, idS, (c | kk) != 0);
                    }
                }
                umma_commit(&sm.s_full[s]);
                umma_commit(&sm.k_empty[ks_]);
                if (j >= 1 && !issue_pv(j - 1)) break;
            }
            if (!*failed) issue_pv(nb - 1);
        }
    } else {
        // -------------------------------------------------------------------------------- softmax
        // row r = TMEM lane (warp % 4) * 32 + lane; group g = warp / 4 owns cells [CPT g, CPT g + CPT) of each
        // 64-cell block and dims [OPT g, OPT g + OPT) of O. The groups of a row agree on its max through shared
        // memory once per block. Every thread reaches every named barrier, failed or not.
        const int grp = warp >> 2;
        const int r = (warp & 3) * 32 + lane;
        const int qi = q0 + r;
        const uint32_t lane_addr = tmem + ((uint32_t) ((warp & 3) * 32) << 16);
        const __half* mrow = nullptr;
        float slope = 1.0f;
        if (p.mask && qi < p.n_q)
            mrow = reinterpret_cast<const __half*>(p.mask + qi * p.m_nb1 + (h % p.m_ne2) * p.m_nb2 + (b % p.m_ne3) * p.m_nb3);
        if (p.max_bias > 0.0f)
            slope = h < p.n_head_log2 ? powf(p.m0, (float) (h + 1)) : powf(p.m1, (float) (2 * (h - p.n_head_log2) + 1));
        const int64_t row_pos = p.pos0 + q0;  // position of the tile's first query
        const float scl = p.scale_log2;
        float m = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int j = 0; j < nb; ++j) {
            const int s = j % NSTAGE;
            ok = ok && wait_or_fail(&sm.s_full[s], (j / NSTAGE) & 1, p, failed, DEV_ERR_WAIT_FULL);
            ok = __all_sync(0xffffffffu, ok);
            uint32_t sv[CPT];
            float bm = -INFINITY;
            const int64_t blk0 = block_cell(j);
            const bool plain = !mrow && !p.has_softcap && blk0 + BN <= p.n_kv &&
                               (!p.causal || (blk0 >= p.kv_lo && blk0 + BN - 1 <= row_pos)) && q0 + BM <= p.n_q;
            if (ok) {
                tc_fence_after();
                tmem_ld<CPT>(lane_addr + TM_S + s * BN + grp * CPT, sv);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.s_free[s]);
                if (plain) {
                    // scale > 0: the max of the scaled scores is the scaled max of the raw ones
                    float a0 = -INFINITY, a1 = -INFINITY, a2 = -INFINITY, a3 = -INFINITY;
#pragma unroll
                    for (int e = 0; e < CPT; e += 4) {
                        a0 = fmaxf(a0, __uint_as_float(sv[e]));
                        a1 = fmaxf(a1, __uint_as_float(sv[e + 1]));
                        a2 = fmaxf(a2, __uint_as_float(sv[e + 2]));
                        a3 = fmaxf(a3, __uint_as_float(sv[e + 3]));
                    }
                    bm = fmaxf(fmaxf(a0, a1), fmaxf(a2, a3)) * scl;
                } else {
                    const int64_t cell0 = blk0 + grp * CPT;
#pragma unroll
                    for (int e = 0; e < CPT; ++e) {
                        const float sc = prefill_score(p, __uint_as_float(sv[e]), cell0 + e, qi, mrow, slope);
                        sv[e] = __float_as_uint(sc);
                        bm = fmaxf(bm, sc);
                    }
                }
                // exchanged as f16 rounded up (no cell exceeds the shared reference); scores are clamped to f16's
                // range first, a bound (6e4 in log2 units) no attention score reaches
                sm.xmax[j & 1][grp][r] = __float2half_ru(fminf(bm, 60000.0f));
            }
            named_bar_sync(1, SOFTMAX_WARPS * 32);
            if (!ok) continue;
            float bmax = -INFINITY;
#pragma unroll
            for (int g2 = 0; g2 < SOFTMAX_WGS; ++g2) bmax = fmaxf(bmax, __half2float(sm.xmax[j & 1][g2][r]));
            // lazy rescale
            float m_use = m;
            bool rescale = false;
            if ((bmax > m + RESCALE_THRESHOLD || m == -INFINITY) && bmax != -INFINITY) {
                m_use = bmax;
                rescale = m != -INFINITY;
            }
            const bool any_rescale = __any_sync(0xffffffffu, rescale);
            // O may only be rescaled once PV_{j-1} is complete
            if (any_rescale && j >= 1)
                ok = wait_or_fail(&sm.o_done[(j - 1) % NSTAGE], ((j - 1) / NSTAGE) & 1, p, failed, DEV_ERR_WAIT_FULL);
            // P_j reuses P_{j-2}'s buffer: PV_{j-2} must be complete
            if (j >= NSTAGE) ok = ok && wait_or_fail(&sm.o_done[s], ((j / NSTAGE) - 1) & 1, p, failed, DEV_ERR_WAIT_FULL);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) continue;
            tc_fence_after();
            if (any_rescale) {
                const float alpha = rescale ? exp2f(m - m_use) : 1.0f;
                l *= alpha;
#pragma unroll 1
                for (int c = 0; c < OPT / 32; ++c) {
                    uint32_t ov[32];
                    const uint32_t ta = lane_addr + TM_O + grp * OPT + c * 32;
                    tmem_ld32(ta, ov);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
                    tmem_st32(ta, ov);
                }
                tmem_wait_st();
            }
            m = m_use;
            const float mref = m == -INFINITY ? 0.0f : m;
            uint32_t pk[CPT / 2];
            float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
            if (plain) {
#pragma unroll
                for (int e = 0; e < CPT; e += 4) {
                    const float p0 = exp2f(fmaf(__uint_as_float(sv[e]), scl, -mref));
                    const float p1 = exp2f(fmaf(__uint_as_float(sv[e + 1]), scl, -mref));
                    const float p2 = exp2f(fmaf(__uint_as_float(sv[e + 2]), scl, -mref));
                    const float p3 = exp2f(fmaf(__uint_as_float(sv[e + 3]), scl, -mref));
                    s0 += p0, s1 += p1, s2 += p2, s3 += p3;
                    pk[e >> 1] = FMT == 0 ? pack_half2(p0, p1) : pack_bf162(p0, p1);
                    pk[(e >> 1) + 1] = FMT == 0 ? pack_half2(p2, p3) : pack_bf162(p2, p3);
                }
            } else {
#pragma unroll
                for (int e = 0; e < CPT; e += 4) {
                    const float p0 = exp2f(__uint_as_float(sv[e]) - mref), p1 = exp2f(__uint_as_float(sv[e + 1]) - mref);
                    const float p2 = exp2f(__uint_as_float(sv[e + 2]) - mref), p3 = exp2f(__uint_as_float(sv[e + 3]) - mref);
                    s0 += p0, s1 += p1, s2 += p2, s3 += p3;
                    pk[e >> 1] = FMT == 0 ? pack_half2(p0, p1) : pack_bf162(p0, p1);
                    pk[(e >> 1) + 1] = FMT == 0 ? pack_half2(p2, p3) : pack_bf162(p2, p3);
                }
            }
            l += (s0 + s1) + (s2 + s3);
            tmem_st<CPT / 2>(lane_addr + TM_P + s * 32 + grp * (CPT / 2), pk);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.p_full[s]);
        }
        // epilogue: O / sum of the groups' l for this row, each group writing its OPT dims. Once the last PV has
        // completed every MMA has, so the K ring is free to carry the partial row sums.
        if (nb > 0) {
            ok = ok && wait_or_fail(&sm.o_done[(nb - 1) % NSTAGE], ((nb - 1) / NSTAGE) & 1, p, failed, DEV_ERR_WAIT_FULL);
            ok = __all_sync(0xffffffffu, ok);
        }
        named_bar_sync(1, SOFTMAX_WARPS * 32);  // every group has waited: no K stage is still being read
        float* xl = reinterpret_cast<float*>(sm.k[0]);  // [group][row]
        xl[grp * BM + r] = l;
        named_bar_sync(1, SOFTMAX_WARPS * 32);
        float lt = 0.0f;
#pragma unroll
        for (int g2 = 0; g2 < SOFTMAX_WGS; ++g2) lt += xl[g2 * BM + r];
        float* out = reinterpret_cast<float*>(p.dst + h * p.d_nb1 + (int64_t) qi * p.d_nb2 + b * p.d_nb3) + grp * OPT;
        if (ok && nb > 0) {
            tc_fence_after();
            const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
#pragma unroll 1
            for (int c = 0; c < OPT / 32; ++c) {
                uint32_t ov[32];
                tmem_ld32(lane_addr + TM_O + grp * OPT + c * 32, ov);
                tmem_wait_ld();
                if (qi < p.n_q) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4)
                        *reinterpret_cast<float4*>(out + c * 32 + e) =
                            make_float4(__uint_as_float(ov[e]) * inv, __uint_as_float(ov[e + 1]) * inv,
                                        __uint_as_float(ov[e + 2]) * inv, __uint_as_float(ov[e + 3]) * inv);
                }
            }
        } else if (nb == 0 && qi < p.n_q) {
            for (int d = 0; d < OPT; d += 4) *reinterpret_cast<float4*>(out + d) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, 512);
}

}  // namespace

size_t fa_prefill_smem_bytes() { return sizeof(Smem); }

cudaError_t launch_fa_prefill(const FaPrefillParams& p, int fmt, const CUtensorMap& tmK, const CUtensorMap& tmV,
                              cudaStream_t stream) {
    static bool attr_done[2][64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    auto kern = fmt == 0 ? fa_prefill_kernel<0> : fa_prefill_kernel<1>;
    const size_t smem = fa_prefill_smem_bytes();
    if (dev < 0 || dev >= 64 || !attr_done[fmt][dev]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_done[fmt][dev] = true;
    }
    dim3 grid(p.n_qtiles * p.n_head, p.ne3);
    kern<<<grid, THREADS, smem, stream>>>(tmK, tmV, p);
    return cudaGetLastError();
}

}  // namespace kb
