// Causal prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM): GGML_OP_FLASH_ATTN_EXT with
// many query tokens over an f16 or bf16 KV cache (klein's prompt chunks; config[2]'s 4,096-token prefill), and over
// the f16 widening of a q8_0 / q4_0 cache (kv_widen.cu writes it; Q is then rounded to q8_0 first, as ggml's CPU op
// rounds it to the vec_dot type of a q8_0 or q4_0 K, ops.cpp:8960).
//
// One CTA computes a 128-query tile of one head. Roles (12 warps):
//   warps 0-7  softmax in two warpgroups that share every 64-cell block: group g takes cells [32 g, 32 g + 32) of
//              each row (row r = TMEM lane r, one thread per row and group) and dims [128 g, 128 g + 128) of O.
//              Stage Q, run the online softmax (unmasked blocks on the packed f32x2 pipe), rescale O when needed,
//              write the normalised output. The groups agree on each block's row max through shared memory (f32,
//              one named barrier per block); each keeps its part of the row sum. The block's softmax latency is the
//              S -> softmax -> PV -> S_{j+3} cycle's longest step: halving the cells per thread shortens it (one
//              thread per row over all 64 cells took 1.0 us of a 1.09 us block; groups taking alternate blocks
//              overlapped their work but left each block's latency, and so the cycle, unchanged).
//   warps 8-9  TMA producers for K and for V (independent chains): 64 cells x 256 dims, 128-byte swizzle, rings
//              of 3 tiles each
//   warp 10    S issuer (one thread): S_j = Q K_j^T, 16 MMAs of K = 16 into S buffer j % 3, once PV_{j-3} (the
//              last reader of that buffer) has completed
//   warp 11    PV issuer (one thread): O += P_j V_j (TS form: P from TMEM) as soon as the softmax has written P_j.
//              The tensor core accepts only a few MMAs ahead of the one executing, so one thread issuing both
//              would hold PV back behind the 16 S MMAs.
// TMEM (512 columns): O 128 x 256 f32 at [0, 256), S_0..S_2 128 x 64 f32 at [256, 448), Q dims 0-127 (f16|bf16
// packed two per column) at [448, 512); Q dims 128-255 sit in shared memory. P_j (32 columns) overwrites the first
// half of S_j once the softmax has read S_j. Three S / P buffers let S_{j+3} wait only for PV_j, so the loop
// S -> softmax -> PV spans three blocks; the split Q leaves shared memory to 3-deep K and V rings.
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
constexpr int KVTILE = BN * D * 2;            // 32 KiB: a whole K or V tile, 4 chunks of [64 cells][128 B]
constexpr int SOFTMAX_WGS = 2;                 // softmax warpgroups, sharing every block's cells
constexpr int SOFTMAX_WARPS = 4 * SOFTMAX_WGS;
constexpr int CPT = BN / SOFTMAX_WGS;           // cells per softmax thread per block
constexpr int OPT = D / SOFTMAX_WGS;            // O columns per softmax thread (rescale and epilogue)
constexpr int THREADS = (SOFTMAX_WARPS + 4) * 32;  // + K producer, V producer, S issuer, PV issuer
constexpr int W_KPROD = SOFTMAX_WARPS, W_VPROD = SOFTMAX_WARPS + 1, W_SMMA = SOFTMAX_WARPS + 2, W_PVMMA = SOFTMAX_WARPS + 3;
constexpr uint32_t TM_O = 0, TM_S = 256;              // O, then the S / P buffers (then Q's TMEM part, if any)
constexpr float RESCALE_THRESHOLD = 8.0f;     // log2 units: rescale O only when the max grows by > 2^8

// The K / V rings. One CTA holds whole tiles in 3-deep rings. A pair of CTAs (PAIR: two heads of a GQA group on the
// same query tile, M = 256 MMAs issued by CTA 0) splits every tile: each CTA holds 32 of a K tile's 64 cells and 2 of
// a V tile's 4 dim chunks, so the same shared memory carries 6-deep rings. The K ring's depth is what sets the
// steady state (K_{j+depth}'s load can start only when S_j's MMAs have freed its stage, and takes ~2.5 us).
//
// S / P buffers (NSTAGE): S_{j+NSTAGE} may start once PV_j has read P_j, so the loop S -> softmax -> PV spans NSTAGE
// blocks. O 256 + 3 x 64 S columns + Q dims 0-127 (64 packed columns) fill TMEM; Q dims 128-255 sit in shared memory.
// (A pair with all of Q in shared memory, 5-deep rings and a fourth S / P buffer measured slower: every S MMA then
// reads its A operand from shared memory as well, 3.4 us from issue to completion against 0.8.)
template <bool PAIR>
struct Ring {
    static constexpr int KROWS = PAIR ? BN / 2 : BN;     // cells of a K tile held here
    static constexpr int VCHUNKS = PAIR ? 2 : 4;         // 64-dim chunks of a V tile held here
    static constexpr int KST = KROWS * D * 2;            // bytes of a K stage
    static constexpr int VST = VCHUNKS * BN * 128;       // bytes of a V stage
    static constexpr int KSTAGE = PAIR ? 6 : 3, VSTAGE = PAIR ? 6 : 3;
    static constexpr int QT_DIMS = 128;                  // Q dims held in TMEM (the rest in shared memory)
    static constexpr int NSTAGE = 3;
    static constexpr uint32_t TM_Q = TM_S + NSTAGE * BN;
    static constexpr int OUT_V = (BM * D * 4 - KSTAGE * KST) / VST;  // V stages the output tile needs beyond the K ring
    static constexpr int QSTG = BM * QT_DIMS * 2 / VST;              // V stages (the last ones) of Q's staging image
    static_assert(TM_Q + QT_DIMS / 2 <= 512, "TMEM");
};

template <bool PAIR>
struct Smem {
    using R = Ring<PAIR>;
    uint8_t q[(D - R::QT_DIMS) / 64][BM * 128];  // Q's shared-memory dims: K-major, 128B-swizzled [chunk][128 rows][128 B]
    uint8_t k[R::KSTAGE][R::KST];              // (1024-aligned offsets)
    uint8_t v[R::VSTAGE][R::VST];
    uint64_t k_full[R::KSTAGE], k_empty[R::KSTAGE], v_full[R::VSTAGE], v_empty[R::VSTAGE];
    uint64_t s_full[R::NSTAGE], p_full[R::NSTAGE], o_done[R::NSTAGE];
    uint64_t q_staged;                         // the Q staging stages of the V ring are free again (softmax warps)
    uint64_t q_ready;                          // Q is in place (in both CTAs of a pair): the S issuer may start
    float xmax[2][SOFTMAX_WGS][BM];            // [block parity][group][row]: the groups' block maxima
    uint32_t tmem_base;
    int failed;
};
// the epilogue's output tile (128 rows x 1 KB) spans the K ring and the first OUT_V V stages and its partial row sums
// [group][row] the next V stage, all idle once the last PV has completed; Q's staging image (dims 0-127 as 16-bit
// pairs) uses the last QSTG V stages
template <bool PAIR>
constexpr bool ring_fits() {
    using R = Ring<PAIR>;
    return R::KSTAGE * R::KST + R::OUT_V * R::VST == BM * D * 4 && R::OUT_V + 1 <= R::VSTAGE - R::QSTG &&
           SOFTMAX_WGS * BM * (int) sizeof(float) <= R::VST && R::QSTG * R::VST == BM * R::QT_DIMS * 2 &&
           sizeof(Smem<PAIR>) <= 232448;
}
static_assert(ring_fits<false>() && ring_fits<true>(), "ring layout");


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

// FMT: 0 = f16 K/V, 1 = bf16 K/V (the type of K, V, and of the rounding of Q and P); 2 = f16 K/V widened from a
// q8_0 / q4_0 cache, with Q quantised to q8_0 (quantize_row_q8_0_ref's rule) and widened to f16(q * d)
//
// PAIR: launched in clusters of 2 (heads 2 i and 2 i + 1, same query tile, same KV head): the MMAs of both CTAs are one
// cta_group::2 MMA of M = 256 issued by CTA 0's issuers, which wait on CTA 0's barriers (each CTA's half-tile loads
// count there, and CTA 1's softmax warps arrive there) and commit to both CTAs' barriers.
template <int FMT, bool PAIR>
__global__ void __launch_bounds__(THREADS, 1)
    fa_prefill_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                      const FaPrefillParams p) {
    using R = Ring<PAIR>;
    constexpr int KSTAGE = R::KSTAGE, VSTAGE = R::VSTAGE, NSTAGE = R::NSTAGE, QT_DIMS = R::QT_DIMS;
    constexpr uint32_t TM_Q = R::TM_Q;
    constexpr int OPF = FMT == 1 ? 1 : 0;  // operand format of the MMAs: f16 or bf16
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // the swizzled tiles need 1024-byte alignment; the dynamic window starts there (checked, not assumed)
    if (smem_u32(smem_raw) & 1023) {
        if (threadIdx.x == 0) record_error(p.err, DEV_ERR_ALIGN);
        return;
    }
    Smem<PAIR>& sm = *reinterpret_cast<Smem<PAIR>*>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;  // CTA 0 of a pair issues the MMAs
    const bool issuer_cta = rank == 0;

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
    if (p.mask_cls) {
        // a classified mask: leading and trailing blocks hidden from the whole tile are not visited
        const uint8_t* cls = p.mask_cls + (int64_t) tile * p.cls_ld;
        int first = -1, last = -1;
        for (int bi = (int) (c_lo / BN); bi < p.cls_ld && (int64_t) bi * BN < c_hi; ++bi)
            if (cls[bi] != FA_MASK_HIDDEN) {
                if (first < 0) first = bi;
                last = bi;
            }
        if (first < 0) {
            c_hi = c_lo;
        } else {
            c_lo = max(c_lo, (int64_t) first * BN);
            c_hi = min(c_hi, (int64_t) (last + 1) * BN);
        }
    }
    const int nb = c_hi > c_lo ? (int) ((c_hi - c_lo + BN - 1) / BN) : 0;
    // the heads of a GQA group walk the shared K/V blocks from different starting points, so that they do not
    // all request the same L2 lines at once; block order does not change the result of the online softmax
    // (a pair walks as one: its two heads share every MMA)
    const int rot = nb > 0 ? (PAIR ? (int) (((int64_t) ((h % p.gqa) / 2) * nb) / (p.gqa / 2))
                                   : (int) (((int64_t) (h % p.gqa) * nb) / p.gqa))
                           : 0;
    auto block_cell = [&](int j) -> int64_t { return c_lo + (int64_t) ((j + rot) % nb) * BN; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < KSTAGE; ++s) {
            mbar_init(&sm.k_full[s], 1);
            mbar_init(&sm.k_empty[s], 1);
        }
        for (int s = 0; s < VSTAGE; ++s) {
            mbar_init(&sm.v_full[s], 1);
            mbar_init(&sm.v_empty[s], 1);
        }
        for (int s = 0; s < NSTAGE; ++s) {
            mbar_init(&sm.s_full[s], 1);
            mbar_init(&sm.p_full[s], (PAIR ? 2 : 1) * SOFTMAX_WARPS);
            mbar_init(&sm.o_done[s], 1);
        }
        mbar_init(&sm.q_staged, SOFTMAX_WARPS);
        mbar_init(&sm.q_ready, (PAIR ? 2 : 1) * SOFTMAX_WARPS);
        sm.failed = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        if constexpr (PAIR) {
            tmem_alloc_pair(&sm.tmem_base, 512);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(&sm.tmem_base, 512);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    volatile int* failed = &sm.failed;
    if (warp < SOFTMAX_WARPS) {
        // Q rounded to the K type, read with coalesced loads (a warp reads half a row, 512 contiguous bytes): dims
        // 128-255 go straight into their swizzled K-major image in shared memory (the A operand of QK^T); dims 0-127
        // into a row-major staging image in V stage 2 (16-byte units XOR-swizzled by row), from which each row's
        // thread moves them into TMEM. V stage 2 is first loaded for block 2, after this (the q_staged barrier).
        constexpr int NT = SOFTMAX_WARPS * 32;   // threads staging Q
        constexpr int F4 = D / 4;                // float4 per row
        const int tid = threadIdx.x;
        uint8_t* stage = sm.v[0] + (VSTAGE - R::QSTG) * R::VST;  // (unused when all of Q is in shared memory)
        constexpr int QB = 16;  // float4 loads in flight per thread
#pragma unroll 1
        for (int i0 = 0; i0 < BM * F4 / NT; i0 += QB) {
            float4 a[QB];
#pragma unroll
            for (int u = 0; u < QB; ++u) {
                const int f = tid + NT * (i0 + u), row = f / F4, c4 = f % F4, qi = q0 + row;
                a[u] = qi < p.n_q ? reinterpret_cast<const float4*>(p.q + qi * p.q_nb1 + h * p.q_nb2 + b * p.q_nb3)[c4]
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < QB; ++u) {
                const int f = tid + NT * (i0 + u), row = f / F4, c4 = f % F4;
                uint2 v2;
                if constexpr (FMT == 2) {
                    // q8_0 blocks of 32 dims = 8 float4 in 8 consecutive lanes: d = amax / 127, q = round(x / d),
                    // then f16(q * f16(d))
                    float amax = max3f(fabsf(a[u].x), fabsf(a[u].y), fmaxf(fabsf(a[u].z), fabsf(a[u].w)));
#pragma unroll
                    for (int off = 1; off < 8; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
                    const float d = amax / 127.0f;
                    const float id = d != 0.0f ? 1.0f / d : 0.0f;
                    const float dh = __half2float(__float2half_rn(d));
                    v2 = make_uint2(pack_half2(roundf(a[u].x * id) * dh, roundf(a[u].y * id) * dh),
                                    pack_half2(roundf(a[u].z * id) * dh, roundf(a[u].w * id) * dh));
                } else {
                    v2 = OPF == 0 ? make_uint2(pack_half2(a[u].x, a[u].y), pack_half2(a[u].z, a[u].w))
                                  : make_uint2(pack_bf162(a[u].x, a[u].y), pack_bf162(a[u].z, a[u].w));
                }
                if (c4 < QT_DIMS / 4) {
                    // staging row: 16 units of 16 bytes, unit c4 / 2 at position (c4 / 2) ^ (row % 16)
                    *reinterpret_cast<uint2*>(stage + row * 256 + (((c4 >> 1) ^ (row & 15)) << 4) + (c4 & 1) * 8) = v2;
                } else {
                    const int cc = c4 - QT_DIMS / 4;  // float4 index within Q's shared-memory dims
                    uint8_t* img = sm.q[cc / 16];
                    *reinterpret_cast<uint2*>(img + row * 128 + ((((cc % 16) >> 1) ^ (row & 7)) << 4) + (cc & 1) * 8) = v2;
                }
            }
        }
        named_bar_sync(1, NT);
        // TMEM row r = this thread's lane quadrant row; group g moves dims [64 g, 64 g + 64) (32 packed columns)
        if constexpr (QT_DIMS > 0) {
            const int grp = warp >> 2, r = (warp & 3) * 32 + lane;
            uint32_t qv[32];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const uint4 x = *reinterpret_cast<const uint4*>(stage + r * 256 + (((grp * 8 + u) ^ (r & 15)) << 4));
                qv[4 * u] = x.x, qv[4 * u + 1] = x.y, qv[4 * u + 2] = x.z, qv[4 * u + 3] = x.w;
            }
            tmem_st32(tmem + ((uint32_t) ((warp & 3) * 32) << 16) + TM_Q + grp * 32, qv);
        }
        tmem_wait_st();
        fence_proxy_async_smem();  // the generic writes of sm.q before the tensor core reads it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&sm.q_staged);
            if constexpr (PAIR)
                mbar_arrive_cluster(smem_rank(&sm.q_ready, 0));
            else
                mbar_arrive(&sm.q_ready);
        }
    }
    // the S issuer starts once Q is in place (q_ready); the producers and the PV issuer do not wait for it

    if (warp == W_KPROD || warp == W_VPROD) {
        // -------------------------------------------------------------------------------- TMA producers
        // K and V run independent chains: K_j waits only for S_{j-2}, V_j only for PV_{j-2}
        const bool is_v = warp == W_VPROD;
        if (lane == 0 && nb > 0) {
            const CUtensorMap* map = is_v ? &tmV : &tmK;
            tma_prefetch_desc(map);
            const int depth = is_v ? VSTAGE : KSTAGE;
            for (int j = 0; j < nb; ++j) {
                const int s = j % depth;
                const int cell = (int) block_cell(j);
                uint64_t* empty = is_v ? &sm.v_empty[s] : &sm.k_empty[s];
                uint64_t* fullb = is_v ? &sm.v_full[s] : &sm.k_full[s];
                uint8_t* dst = is_v ? sm.v[s] : sm.k[s];
                if (j >= depth && !wait_or_fail(empty, ((j / depth) - 1) & 1, p, failed, DEV_ERR_WAIT_EMPTY)) break;
                // V stage 2 carries the Q staging image until the softmax warps have moved it into TMEM
                if (R::QSTG > 0 && is_v && j == VSTAGE - R::QSTG &&
                    !wait_or_fail(&sm.q_staged, 0, p, failed, DEV_ERR_WAIT_EMPTY))
                    break;
                if constexpr (PAIR) {
                    // both halves complete on CTA 0's barrier, which expects the whole tile
                    if (issuer_cta) mbar_arrive_expect_tx(fullb, KVTILE);
                    const uint32_t bar0 = smem_rank(fullb, 0);
                    if (is_v) {
                        for (int cc = 0; cc < R::VCHUNKS; ++cc)
                            tma_load_4d_pair(dst + cc * (BN * 128), map, bar0, (int) (rank * R::VCHUNKS + cc) * 64, hk, cell,
                                             kb3);
                    } else {
                        for (int c = 0; c < D / 64; ++c)
                            tma_load_4d_pair(dst + c * (R::KROWS * 128), map, bar0, c * 64, hk, cell + (int) rank * R::KROWS,
                                             kb3);
                    }
                } else {
                    mbar_arrive_expect_tx(fullb, KVTILE);
                    for (int c = 0; c < D / 64; ++c) tma_load_4d(dst + c * (BN * 128), map, fullb, c * 64, hk, cell, kb3);
                }
            }
        }
    } else if (warp == W_SMMA) {
        // -------------------------------------------------------------------------------- S issuer
        // S_j = Q K_j^T into buffer j % 2, once PV_{j-2} (the last reader of that buffer, through P_{j-2}) has
        // completed. A separate PV issuer keeps PV from waiting behind these 16 MMAs: the tensor core accepts only
        // a few MMAs ahead of the one executing, so issuing them takes about as long as running them.
        if (lane == 0 && nb > 0 && issuer_cta) {
            constexpr uint32_t idS = umma_idesc_f16(OPF, PAIR ? 2 * BM : BM, BN, false, false);
            wait_or_fail(&sm.q_ready, 0, p, failed, DEV_ERR_WAIT_FULL);
            for (int j = 0; j < nb; ++j) {
                const int s = j % NSTAGE, ks_ = j % KSTAGE;
                if (!wait_or_fail(&sm.k_full[ks_], (j / KSTAGE) & 1, p, failed, DEV_ERR_WAIT_FULL)) break;
                if (j >= NSTAGE && !wait_or_fail(&sm.o_done[s], ((j / NSTAGE) - 1) & 1, p, failed, DEV_ERR_WAIT_EMPTY))
                    break;
                tc_fence_after();
                const uint32_t k_addr = smem_u32(sm.k[ks_]);
#pragma unroll
                for (int c = 0; c < D / 64; ++c) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        // A = Q (dims 0-127 from TMEM, 8 packed columns per step; dims 128-255 from shared
                        // memory), B = K block, K-major
                        const uint64_t bdesc = smem_desc_sw128(k_addr + c * (R::KROWS * 128) + kk * 32, 16, 1024);
                        if (c * 64 < QT_DIMS) {
                            if constexpr (PAIR)
                                umma_ts_pair(tmem + TM_S + s * BN, tmem + TM_Q + (c * 4 + kk) * 8, bdesc, idS, (c | kk) != 0);
                            else
                                umma_ts(tmem + TM_S + s * BN, tmem + TM_Q + (c * 4 + kk) * 8, bdesc, idS, (c | kk) != 0);
                        } else {
                            const uint64_t adesc =
                                smem_desc_sw128(smem_u32(sm.q[(c * 64 - QT_DIMS) / 64]) + kk * 32, 16, 1024);
                            if constexpr (PAIR)
                                umma_ss_pair(tmem + TM_S + s * BN, adesc, bdesc, idS, (c | kk) != 0);
                            else
                                umma_ss(tmem + TM_S + s * BN, adesc, bdesc, idS, (c | kk) != 0);
                        }
                    }
                }
                if constexpr (PAIR) {
                    for (uint32_t r2 = 0; r2 < 2; ++r2) {
                        umma_commit_pair(smem_rank(&sm.s_full[s], r2));
                        umma_commit_pair(smem_rank(&sm.k_empty[ks_], r2));
                    }
                } else {
                    umma_commit(&sm.s_full[s]);
                    umma_commit(&sm.k_empty[ks_]);
                }
            }
        }
    } else if (warp == W_PVMMA) {
        // -------------------------------------------------------------------------------- PV issuer
        // O += P_i V_i as soon as the softmax has written P_i (into the first half of S_i's columns)
        if (lane == 0 && nb > 0 && issuer_cta) {
            constexpr uint32_t idO = umma_idesc_f16(OPF, PAIR ? 2 * BM : BM, D, false, true);
            for (int i = 0; i < nb; ++i) {
                const int s = i % NSTAGE, vs = i % VSTAGE;
                if (!wait_or_fail(&sm.p_full[s], (i / NSTAGE) & 1, p, failed, DEV_ERR_WAIT_FULL)) break;
                if (!wait_or_fail(&sm.v_full[vs], (i / VSTAGE) & 1, p, failed, DEV_ERR_WAIT_FULL)) break;
                tc_fence_after();
                const uint32_t v_addr = smem_u32(sm.v[vs]);
#pragma unroll
                for (int ks = 0; ks < BN / 16; ++ks) {
                    // B = V block, MN-major: 64-dim chunks 8 KiB apart (LBO), 8-cell groups 1 KiB apart (SBO)
                    const uint64_t bdesc = smem_desc_sw128(v_addr + ks * 16 * 128, BN * 128, 1024);
                    if constexpr (PAIR)
                        umma_ts_pair(tmem + TM_O, tmem + TM_S + s * BN + ks * 8, bdesc, idO, i > 0 || ks > 0);
                    else
                        umma_ts(tmem + TM_O, tmem + TM_S + s * BN + ks * 8, bdesc, idO, i > 0 || ks > 0);
                }
                if constexpr (PAIR) {
                    for (uint32_t r2 = 0; r2 < 2; ++r2) {
                        umma_commit_pair(smem_rank(&sm.o_done[s], r2));
                        umma_commit_pair(smem_rank(&sm.v_empty[vs], r2));
                    }
                } else {
                    umma_commit(&sm.o_done[s]);
                    umma_commit(&sm.v_empty[vs]);
                }
            }
        }
    } else {
        // -------------------------------------------------------------------------------- softmax
        // row r = TMEM lane (warp % 4) * 32 + lane; group g = warp / 4 owns cells [CPT g, CPT g + CPT) of each
        // 64-cell block and dims [OPT g, OPT g + OPT) of O. Every thread reaches every named barrier, failed or not.
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
            const int64_t cell0 = blk0 + grp * CPT;
            // a block the mask leaves untouched (classified all 0) is computed as an unmasked one
            const bool mask_free = !mrow || (p.mask_cls && p.mask_cls[(int64_t) tile * p.cls_ld + blk0 / BN] == FA_MASK_ZERO);
            const bool plain = mask_free && !p.has_softcap && blk0 + BN <= p.n_kv &&
                               (!p.causal || (blk0 >= p.kv_lo && blk0 + BN - 1 <= row_pos)) && q0 + BM <= p.n_q;
            // without a mask tensor or softcap the visible cells of a row form one range [e_lo, e_hi) of the block
            const bool analytic = !mrow && !p.has_softcap;
            if (ok) {
                tc_fence_after();
                tmem_ld<CPT>(lane_addr + TM_S + s * BN + grp * CPT, sv);
                tmem_wait_ld();
                if (plain) {
                    // scale > 0: the max of the scaled scores is the scaled max of the raw ones (3-input max)
                    float a0 = -INFINITY, a1 = -INFINITY, a2 = -INFINITY, a3 = -INFINITY;
#pragma unroll
                    for (int e = 0; e < CPT; e += 8) {
                        a0 = max3f(a0, __uint_as_float(sv[e]), __uint_as_float(sv[e + 1]));
                        a1 = max3f(a1, __uint_as_float(sv[e + 2]), __uint_as_float(sv[e + 3]));
                        a2 = max3f(a2, __uint_as_float(sv[e + 4]), __uint_as_float(sv[e + 5]));
                        a3 = max3f(a3, __uint_as_float(sv[e + 6]), __uint_as_float(sv[e + 7]));
                    }
                    bm = fmaxf(fmaxf(a0, a1), fmaxf(a2, a3)) * scl;
                } else if (analytic) {
                    int64_t lo = 0, hi = min((int64_t) CPT, p.n_kv - cell0);
                    if (p.causal) {
                        lo = max(lo, p.kv_lo - cell0);
                        hi = min(hi, p.pos0 + qi + 1 - cell0);
                    }
                    if (qi >= p.n_q) hi = 0;
                    const int e_lo = (int) max((int64_t) 0, lo), e_hi = (int) max((int64_t) 0, hi);
#pragma unroll
                    for (int e = 0; e < CPT; ++e) {
                        const float sc = (e >= e_lo && e < e_hi) ? __uint_as_float(sv[e]) * scl : -INFINITY;
                        sv[e] = __float_as_uint(sc);
                        bm = fmaxf(bm, sc);
                    }
                } else if (mrow && !p.has_softcap && cell0 + CPT <= p.n_kv && qi < p.n_q &&
                           (reinterpret_cast<uintptr_t>(mrow + cell0) & 15) == 0) {
                    // the row's CPT mask values in 16-byte loads, then masked_score's arithmetic per cell
                    uint4 mw[CPT / 8];
#pragma unroll
                    for (int u = 0; u < CPT / 8; ++u) mw[u] = reinterpret_cast<const uint4*>(mrow + cell0)[u];
                    const __half* mh = reinterpret_cast<const __half*>(mw);
#pragma unroll
                    for (int e = 0; e < CPT; ++e) {
                        const int64_t key = cell0 + e;
                        float sc = -INFINITY;
                        if (!p.causal || (key >= p.kv_lo && key <= p.pos0 + qi)) {
                            const float mv = slope * __half2float(mh[e]);
                            if (mv != -INFINITY) sc = __uint_as_float(sv[e]) * scl + mv * LOG2E;
                        }
                        sv[e] = __float_as_uint(sc);
                        bm = fmaxf(bm, sc);
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < CPT; ++e) {
                        const float sc = prefill_score(p, __uint_as_float(sv[e]), cell0 + e, qi, mrow, slope);
                        sv[e] = __float_as_uint(sc);
                        bm = fmaxf(bm, sc);
                    }
                }
                sm.xmax[j & 1][grp][r] = bm;
            }
            // both groups have read their S_j (P_j overwrites its first half below) and published their maxima
            named_bar_sync(1, SOFTMAX_WARPS * 32);
            if (!ok) continue;
            float bmax = -INFINITY;
#pragma unroll
            for (int g2 = 0; g2 < SOFTMAX_WGS; ++g2) bmax = fmaxf(bmax, sm.xmax[j & 1][g2][r]);
            // lazy rescale: raise the reference only when the block max exceeds it by more than the threshold
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
            // (P_j reuses S_j's columns; PV_{j-3}, the last reader of this buffer, ran before S_j was written)
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
                // pairs of cells on the packed f32x2 pipe: x = score * scale - m, then ex2, then the row sums
                const uint64_t sc2 = f2pack(scl, scl), nm2 = f2pack(-mref, -mref);
                uint64_t acc0 = 0, acc1 = 0;  // (0.f, 0.f)
#pragma unroll
                for (int e = 0; e < CPT; e += 4) {
                    float x0, x1, x2, x3;
                    f2unpack(ffma2(f2pack(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])), sc2, nm2), x0, x1);
                    f2unpack(ffma2(f2pack(__uint_as_float(sv[e + 2]), __uint_as_float(sv[e + 3])), sc2, nm2), x2, x3);
                    const float p0 = ex2_ftz(x0), p1 = ex2_ftz(x1), p2 = ex2_ftz(x2), p3 = ex2_ftz(x3);
                    acc0 = fadd2(acc0, f2pack(p0, p1));
                    acc1 = fadd2(acc1, f2pack(p2, p3));
                    pk[e >> 1] = OPF == 0 ? pack_half2(p0, p1) : pack_bf162(p0, p1);
                    pk[(e >> 1) + 1] = OPF == 0 ? pack_half2(p2, p3) : pack_bf162(p2, p3);
                }
                f2unpack(fadd2(acc0, acc1), s0, s1);
            } else {
#pragma unroll
                for (int e = 0; e < CPT; e += 4) {
                    const float p0 = exp2f(__uint_as_float(sv[e]) - mref), p1 = exp2f(__uint_as_float(sv[e + 1]) - mref);
                    const float p2 = exp2f(__uint_as_float(sv[e + 2]) - mref), p3 = exp2f(__uint_as_float(sv[e + 3]) - mref);
                    s0 += p0, s1 += p1, s2 += p2, s3 += p3;
                    pk[e >> 1] = OPF == 0 ? pack_half2(p0, p1) : pack_bf162(p0, p1);
                    pk[(e >> 1) + 1] = OPF == 0 ? pack_half2(p2, p3) : pack_bf162(p2, p3);
                }
            }
            l += (s0 + s1) + (s2 + s3);
            // P_j into the first half of S_j's columns (every group has read its S_j: the named barrier above)
            tmem_st<CPT / 2>(lane_addr + TM_S + s * BN + grp * (CPT / 2), pk);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (PAIR)
                    mbar_arrive_cluster(smem_rank(&sm.p_full[s], 0));
                else
                    mbar_arrive(&sm.p_full[s]);
            }
        }
        // epilogue: O / sum of the groups' l for this row, each group writing its OPT dims. Once the last PV has
        // completed every MMA has, so the K and V rings are free to carry the row sums and the output tile.
        if (nb > 0) {
            ok = ok && wait_or_fail(&sm.o_done[(nb - 1) % NSTAGE], ((nb - 1) / NSTAGE) & 1, p, failed, DEV_ERR_WAIT_FULL);
            ok = __all_sync(0xffffffffu, ok);
        }
        named_bar_sync(1, SOFTMAX_WARPS * 32);  // every group has waited: no K / V stage is still being read
        float* xl = reinterpret_cast<float*>(sm.v[R::OUT_V]);  // [group][row]
        xl[grp * BM + r] = l;
        named_bar_sync(1, SOFTMAX_WARPS * 32);
        float lt = 0.0f;
#pragma unroll
        for (int g2 = 0; g2 < SOFTMAX_WGS; ++g2) lt += xl[g2 * BM + r];
        // the normalised rows into a [128 rows][1 KB] tile (16-byte units XOR-swizzled by row % 8), then written out
        // with coalesced stores (a warp writes half a row); rows that see no cell are zeros
        uint8_t* ost = sm.k[0];
        {
            const bool have = ok && nb > 0;
            const float inv = have && lt > 0.0f ? 1.0f / lt : 0.0f;
            if (have) tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < OPT / 32; ++c) {
                uint32_t ov[32];
                if (have) {
                    tmem_ld32(lane_addr + TM_O + grp * OPT + c * 32, ov);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) ov[e] = 0u;
                }
#pragma unroll
                for (int e = 0; e < 32; e += 4) {
                    const int unit = (grp * OPT + c * 32 + e) / 4;
                    *reinterpret_cast<float4*>(ost + r * 1024 + ((unit ^ (r & 7)) << 4)) =
                        make_float4(__uint_as_float(ov[e]) * inv, __uint_as_float(ov[e + 1]) * inv,
                                    __uint_as_float(ov[e + 2]) * inv, __uint_as_float(ov[e + 3]) * inv);
                }
            }
        }
        named_bar_sync(1, SOFTMAX_WARPS * 32);
        {
            constexpr int NT = SOFTMAX_WARPS * 32, F4 = D / 4;
            const int tid = threadIdx.x;
#pragma unroll 4
            for (int i = 0; i < BM * F4 / NT; ++i) {
                const int f = tid + NT * i, row = f / F4, c4 = f % F4, q = q0 + row;
                if (q >= p.n_q) continue;
                float4 o4 = *reinterpret_cast<const float4*>(ost + row * 1024 + ((c4 ^ (row & 7)) << 4));
                if (p.gate) {
                    // klein's output gate (graph.cpp:124): o * sigmoid(gate), ggml's 1 / (1 + expf(-x))
                    const float4 g4 = reinterpret_cast<const float4*>(p.gate + h * p.g_nb1 + (int64_t) q * p.g_nb2 +
                                                                      b * p.g_nb3)[c4];
                    o4.x *= 1.0f / (1.0f + expf(-g4.x));
                    o4.y *= 1.0f / (1.0f + expf(-g4.y));
                    o4.z *= 1.0f / (1.0f + expf(-g4.z));
                    o4.w *= 1.0f / (1.0f + expf(-g4.w));
                }
                reinterpret_cast<float4*>(p.dst + h * p.d_nb1 + (int64_t) q * p.d_nb2 + b * p.d_nb3)[c4] = o4;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    // a pair leaves together: CTA 0's MMAs read CTA 1's shared memory and TMEM, and CTA 1 arrives on CTA 0's barriers
    if constexpr (PAIR) cluster_sync_all();
    tc_fence_after();
    if (warp == 0) {
        if constexpr (PAIR)
            tmem_dealloc_pair(tmem, 512);
        else
            tmem_dealloc(tmem, 512);
    }
}

}  // namespace

namespace {

// One CTA of 128 threads per (128-query tile, 64-cell block), 128 bytes of each of the tile's rows. Aligned rows:
// thread t reads 16-byte unit t % 8 of rows t / 8 + 16 i (i < 8; a warp instruction covers 4 whole 128-byte row
// pieces, all 8 loads in flight); otherwise warp w reads rows 32 w .. + 31 in 4-byte or 2-byte pieces. Cells past
// n_kv count as -inf, rows past n_q are ignored.
__global__ void __launch_bounds__(128) fa_mask_classify_kernel(const char* mask, int64_t m_nb1, int n_q, int64_t n_kv,
                                                               int n_blocks, uint8_t* out) {
    const int blk = blockIdx.x, tile = blockIdx.y;
    const int64_t c0 = (int64_t) blk * BN;
    bool nonzero = false, visible = false;
    auto look = [&](uint16_t a) {
        nonzero = nonzero || (a & 0x7FFFu) != 0;  // +-0 is zero
        visible = visible || a != 0xFC00u;        // anything but -inf
    };
    if (((reinterpret_cast<uintptr_t>(mask) | (uintptr_t) m_nb1) & 15) == 0 && c0 + BN <= n_kv) {
        const int u = threadIdx.x & 7;
        uint4 w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int qi = tile * BM + (threadIdx.x >> 3) + 16 * i;
            w[i] = qi < n_q ? *reinterpret_cast<const uint4*>(mask + (int64_t) qi * m_nb1 + (c0 + 8 * u) * 2)
                            : make_uint4(0xFC00FC00u, 0xFC00FC00u, 0xFC00FC00u, 0xFC00FC00u);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t x[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int qi = tile * BM + (threadIdx.x >> 3) + 16 * i;
                if (qi < n_q) {
                    look((uint16_t) (x[e] & 0xFFFFu));
                    look((uint16_t) (x[e] >> 16));
                }
            }
        }
    } else {
        const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
        const int64_t cell = c0 + 2 * l;
        const bool pairs = ((reinterpret_cast<uintptr_t>(mask) | (uintptr_t) m_nb1) & 3) == 0 && cell + 1 < n_kv;
#pragma unroll 8
        for (int rr = 0; rr < 32; ++rr) {
            const int qi = tile * BM + w * 32 + rr;
            if (qi < n_q) {
                const uint16_t* row = reinterpret_cast<const uint16_t*>(mask + (int64_t) qi * m_nb1);
                uint16_t a, b;
                if (pairs) {
                    const uint32_t ab = *reinterpret_cast<const uint32_t*>(row + cell);
                    a = (uint16_t) (ab & 0xFFFFu), b = (uint16_t) (ab >> 16);
                } else {
                    a = cell < n_kv ? row[cell] : (uint16_t) 0xFC00u;
                    b = cell + 1 < n_kv ? row[cell + 1] : (uint16_t) 0xFC00u;
                }
                look(a);
                look(b);
            }
        }
    }
    const int nz = __syncthreads_or(nonzero), vis = __syncthreads_or(visible);
    if (threadIdx.x == 0) out[(int64_t) tile * n_blocks + blk] = !vis ? FA_MASK_HIDDEN : !nz ? FA_MASK_ZERO : FA_MASK_MIXED;
}

}  // namespace

cudaError_t launch_fa_mask_classify(const char* mask, int64_t m_nb1, int n_q, int64_t n_kv, int n_blocks, uint8_t* out,
                                    cudaStream_t stream) {
    if (n_q <= 0 || n_blocks <= 0) return cudaSuccess;
    fa_mask_classify_kernel<<<dim3(n_blocks, (n_q + BM - 1) / BM), 128, 0, stream>>>(mask, m_nb1, n_q, n_kv, n_blocks, out);
    return cudaGetLastError();
}

size_t fa_prefill_smem_bytes(bool pair) { return pair ? sizeof(Smem<true>) : sizeof(Smem<false>); }

cudaError_t launch_fa_prefill(const FaPrefillParams& p, int fmt, bool pair, const CUtensorMap& tmK, const CUtensorMap& tmV,
                              cudaStream_t stream) {
    static bool attr_done[2][3][64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (fmt < 0 || fmt > 2) return cudaErrorInvalidValue;
    if (pair && (p.n_head % 2 != 0 || p.gqa % 2 != 0)) return cudaErrorInvalidValue;
    using Kern = void (*)(CUtensorMap, CUtensorMap, FaPrefillParams);
    const Kern kern = pair ? (fmt == 0 ? fa_prefill_kernel<0, true> : fmt == 1 ? fa_prefill_kernel<1, true> : fa_prefill_kernel<2, true>)
                           : (fmt == 0 ? fa_prefill_kernel<0, false> : fmt == 1 ? fa_prefill_kernel<1, false>
                                                                                : fa_prefill_kernel<2, false>);
    const size_t smem = fa_prefill_smem_bytes(pair);
    if (dev < 0 || dev >= 64 || !attr_done[pair][fmt][dev]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_done[pair][fmt][dev] = true;
    }
    const dim3 grid(p.n_qtiles * p.n_head, p.ne3);
    if (!pair) {
        kern<<<grid, THREADS, smem, stream>>>(tmK, tmV, p);
        return cudaGetLastError();
    }
    // clusters of 2 consecutive CTAs: heads 2 i and 2 i + 1 of the same query tile
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2, attr[0].val.clusterDim.y = 1, attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, tmK, tmV, p);
}

}  // namespace kb
