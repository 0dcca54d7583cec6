// C-ABI shim: validates ggml-style tensor descriptors the way ggml's operator constructors and CPU ops do
// (ggml.c:5506-5548, ops.cpp:8865-8890), plans the kernel launch, builds the TMA descriptors and launches.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/klein_b200.h"
#include "kb_gdn.h"
#include "kb_internal.h"

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

struct DevInfo {
    int sm_count = 0;
};

DevInfo dev_info() {
    static DevInfo info[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DevInfo{};
    if (info[dev].sm_count == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        info[dev].sm_count = n;
    }
    return info[dev];
}

uint64_t g_wait_ns = 1000000000ull;  // 1 s budget for every bounded device wait
// Prefill on CTA pairs (cta_group::2, each CTA holding half of every K / V tile) where the head shape allows it,
// when KB_PREFILL_PAIR=1 (read per call). Off by default: correct, but 766 against 800 TFLOP/s for one CTA per tile
// at config[2] (deeper K / V rings moved the limit to the three S / P buffers).
bool prefill_pair_enabled() {
    const char* e = std::getenv("KB_PREFILL_PAIR");
    return e && e[0] == '1';
}

bool aligned16(size_t x) { return (x & 15) == 0; }

// The split-KV plan of one streaming attention call.
struct FaPlan {
    int rpc = 32, n_row_chunks = 1, n_splits = 1;
    int64_t blocks_base = 0;  // 128-cell blocks per split (the first blocks_extra splits take one more)
    int blocks_extra = 0;
    size_t scratch = 0;
};

struct FaShape {
    int D, n_q, H, ne3, H_kv, ne3k, gqa, R, kv_type;
    int64_t n_kv;
};

// Prefill (tcgen05) kernel: 128-query tiles of one head; f16 or bf16 K/V; whole-output calls only.
constexpr int PREFILL_MIN_Q = 128;
bool prefill_shape(const FaShape& s, const kb_fa_params* prm, bool partial) {
    return !partial && s.n_q >= PREFILL_MIN_Q && !(prm && prm->causal && prm->ring > 0);
}
// the class table of a dense mask for the prefill kernel: one byte per (128-query tile, 64-cell block)
size_t mask_cls_bytes(const FaShape& s) {
    const size_t n = (size_t) ((s.n_q + 127) / 128) * (size_t) ((s.n_kv + 63) / 64);
    return (n + 255) / 256 * 256;
}

bool use_prefill(const FaShape& s, const kb_fa_params* prm, bool partial) {
    return prefill_shape(s, prm, partial) && (s.kv_type == KB_TYPE_F16 || s.kv_type == KB_TYPE_BF16);
}
// Prefill over a q8_0 / q4_0 cache: the visible cells are widened to an f16 copy in the scratch (kv_widen.cu), then
// the f16 prefill kernel runs on it with Q rounded to q8_0. Without that much scratch the call runs on the streaming
// kernel instead (same results within the parity bound, slower for long prompts).
bool prefill_quant_shape(const FaShape& s, const kb_fa_params* prm, bool partial) {
    return prefill_shape(s, prm, partial) && (s.kv_type == KB_TYPE_Q8_0 || s.kv_type == KB_TYPE_Q4_0);
}
// bytes of one f16 view [ne3k][n_kv][H_kv][256] (K or V); the V view follows the K view
size_t widen_view_bytes(const FaShape& s) { return (size_t) s.ne3k * (size_t) s.n_kv * s.H_kv * kb::FA_D * 2; }

kb_status check_fa(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* mask, FaShape* s) {
    if (!q || !k || !v) return KB_ERR_ARG;
    if (q->type != KB_TYPE_F32) return KB_ERR_UNSUPPORTED;
    if (k->type != v->type) return KB_ERR_UNSUPPORTED;
    if (k->type != KB_TYPE_F16 && k->type != KB_TYPE_Q8_0 && k->type != KB_TYPE_Q4_0 && k->type != KB_TYPE_BF16)
        return KB_ERR_UNSUPPORTED;
    s->D = (int) q->ne[0];
    s->n_q = (int) q->ne[1];
    s->H = (int) q->ne[2];
    s->ne3 = (int) q->ne[3];
    s->n_kv = k->ne[1];
    s->H_kv = (int) k->ne[2];
    s->ne3k = (int) k->ne[3];
    // ggml_can_mul_mat(k, q) and the CPU op's shape asserts
    if (k->ne[0] != q->ne[0] || v->ne[0] != k->ne[0]) return KB_ERR_BAD_SHAPE;
    if (v->ne[1] != k->ne[1] || v->ne[2] != k->ne[2] || v->ne[3] != k->ne[3]) return KB_ERR_BAD_SHAPE;
    if (s->H_kv <= 0 || s->H % s->H_kv != 0 || s->ne3k <= 0 || s->ne3 % s->ne3k != 0) return KB_ERR_BAD_SHAPE;
    if (s->n_q <= 0 || s->H <= 0 || s->ne3 <= 0 || s->n_kv < 0) return KB_ERR_BAD_SHAPE;
    // nb[0]: element size, or the block size of a block-quantised type
    const size_t kv_es = k->type == KB_TYPE_Q8_0 ? 34 : k->type == KB_TYPE_Q4_0 ? 18 : 2;
    s->kv_type = k->type;
    if (q->nb[0] != 4 || k->nb[0] != kv_es || v->nb[0] != kv_es) return KB_ERR_BAD_SHAPE;
    if (s->D != kb::FA_D) return KB_ERR_UNSUPPORTED;
    if (mask) {
        if (mask->type != KB_TYPE_F16 || mask->nb[0] != 2) return KB_ERR_UNSUPPORTED;
        if (mask->ne[0] < s->n_kv || mask->ne[1] < s->n_q) return KB_ERR_BAD_SHAPE;
        if (mask->ne[2] <= 0 || mask->ne[3] <= 0 || s->H % mask->ne[2] != 0 || s->ne3 % mask->ne[3] != 0)
            return KB_ERR_BAD_SHAPE;
    }
    // TMA: 16-byte aligned base and strides
    for (const kb_tensor* t : {k, v}) {
        if (!aligned16(reinterpret_cast<uintptr_t>(t->data)) || !aligned16(t->nb[1]) || !aligned16(t->nb[2]) ||
            !aligned16(t->nb[3]))
            return KB_ERR_UNSUPPORTED;
    }
    s->gqa = s->H / s->H_kv;
    s->R = s->n_q * s->gqa;
    return KB_OK;
}

// push: the fused exchange (kb_flash_attn_ext_push) always runs the split combine and needs a counter
FaPlan plan_fa(const FaShape& s, bool push = false) {
    FaPlan pl;
    pl.rpc = kb::fa_tc_rpc(s.R);
    pl.n_row_chunks = (s.R + pl.rpc - 1) / pl.rpc;
    const int sms = dev_info().sm_count > 0 ? dev_info().sm_count : 148;
    const int64_t base = (int64_t) s.H_kv * pl.n_row_chunks * s.ne3;
    // split unit: a 128-cell block
    const int unit = kb::FA_TC_BLOCK;
    const int64_t tiles = (s.n_kv + unit - 1) / unit;
    int64_t target = sms / base;
    if (target < 1) target = 1;
    if (tiles == 0) {
        pl.n_splits = 1;
        pl.blocks_base = 1;
    } else {
        // as many splits as SMs allow, their block counts within one of each other (a CTA's time is its blocks)
        pl.n_splits = (int) std::min<int64_t>(target, tiles);
        pl.blocks_base = tiles / pl.n_splits;
        pl.blocks_extra = (int) (tiles % pl.n_splits);
    }
    if (pl.n_splits > 1 || push) {
        const size_t rows = (size_t) base * pl.n_splits * pl.rpc;
        pl.scratch = rows * kb::FA_D * 4 + 256 + rows * 2 * 4;
        if (push) pl.scratch = (pl.scratch + 255) / 256 * 256 + 256;  // the combine's CTA counter
    }
    return pl;
}

kb_status encode_kv_map(const kb_tensor* t, CUtensorMap* map, int box_cells = kb::FA_TILE) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return KB_ERR_CUDA;
    if (t->type == KB_TYPE_Q8_0 || t->type == KB_TYPE_Q4_0) {
        // raw blocks: one head's row is ne0/32 blocks of 34 (q8_0) or 18 (q4_0) bytes, read as 32-bit words without
        // swizzle; dims: words of a head row, KV head, cell, batch; box = a whole head row x 64 cells
        const cuuint64_t words = (cuuint64_t) t->ne[0] / 32 * (t->type == KB_TYPE_Q8_0 ? 34 : 18) / 4;
        const cuuint64_t dims[4] = {words, (cuuint64_t) t->ne[2], (cuuint64_t) t->ne[1], (cuuint64_t) t->ne[3]};
        const cuuint64_t strides[3] = {(cuuint64_t) t->nb[2], (cuuint64_t) t->nb[1], (cuuint64_t) t->nb[3]};
        const cuuint32_t box[4] = {(cuuint32_t) words, 1, (cuuint32_t) kb::FA_TILE, 1};
        const cuuint32_t estr[4] = {1, 1, 1, 1};
        CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, t->data, dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        return r == CUDA_SUCCESS ? KB_OK : KB_ERR_CUDA;
    }
    // dims (innermost first): head dim, KV head, cell, batch; box = 64 dims x 1 head x 64 cells
    const cuuint64_t dims[4] = {(cuuint64_t) t->ne[0], (cuuint64_t) t->ne[2], (cuuint64_t) t->ne[1], (cuuint64_t) t->ne[3]};
    const cuuint64_t strides[3] = {(cuuint64_t) t->nb[2], (cuuint64_t) t->nb[1], (cuuint64_t) t->nb[3]};
    const cuuint32_t box[4] = {64, 1, (cuuint32_t) box_cells, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUtensorMapDataType dt = t->type == KB_TYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUresult r = enc(map, dt, 4, t->data, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? KB_OK : KB_ERR_CUDA;
}

}  // namespace

extern "C" {

const char* kb_version(void) { return "klein_b200 0.1"; }

size_t kb_flash_attn_ext_scratch_bytes(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v,
                                       const kb_fa_params* params) {
    FaShape s;
    if (check_fa(q, k, v, nullptr, &s) != KB_OK) return 0;
    // the streaming kernel's split partials: what kb_flash_attn_ext_partial needs for any shape (the f16 / bf16
    // prefill kernel takes none), plus, for prefill shapes over a q8_0 / q4_0 cache, the two f16 views
    const size_t stream_need = plan_fa(s).scratch;
    if (prefill_quant_shape(s, params, false)) return std::max(2 * widen_view_bytes(s) + mask_cls_bytes(s), stream_need);
    if (use_prefill(s, params, false)) return std::max(mask_cls_bytes(s), stream_need);
    return stream_need;
}

}  // extern "C"

namespace {

// the destinations of the fused exchange
struct PushArgs {
    float* const* gather;
    int32_t* const* flags;
    int64_t slot_set_floats, part_floats;
    int rank, n_ranks;
};

// push: the fused push exchange (partials into the gather buffers); xchg: with push, the whole exchange in the
// attention kernel (kb_flash_attn_ext_exchange), dst the final output
kb_status fa_impl(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* mask,
                  const kb_fa_params* prm, const kb_tensor* dst, float* dst_ml, void* scratch, size_t scratch_bytes,
                  void* stream, const kb_tensor* gate = nullptr, const PushArgs* push = nullptr, bool xchg = false) {
    if (!prm || !dst) return KB_ERR_ARG;
    FaShape s;
    kb_status st = check_fa(q, k, v, mask, &s);
    if (st != KB_OK) return st;
    if (dst->type != KB_TYPE_F32 || dst->nb[0] != 4) return KB_ERR_BAD_SHAPE;
    if (dst->ne[0] != s.D || dst->ne[1] != s.H || dst->ne[2] != s.n_q || dst->ne[3] != s.ne3) return KB_ERR_BAD_SHAPE;
    if (gate && (gate->type != KB_TYPE_F32 || gate->nb[0] != 4 || gate->ne[0] != s.D || gate->ne[1] != s.H ||
                 gate->ne[2] != s.n_q || gate->ne[3] != s.ne3))
        return KB_ERR_BAD_SHAPE;
    if (gate && dst_ml) return KB_ERR_ARG;  // the gate applies to final outputs, not to partials
    if (push && ((gate && !xchg) || s.ne3 != 1)) return KB_ERR_ARG;
    if (prm->logit_softcap != 0.0f && !(std::isfinite(prm->logit_softcap))) return KB_ERR_ARG;
    if (prm->max_bias > 0.0f && !mask) return KB_ERR_ARG;  // ggml: ALiBi needs a mask
    if (prm->causal && prm->ring < 0) return KB_ERR_ARG;

    if (s.n_kv == 0 && push) return KB_ERR_UNSUPPORTED;  // nothing to attend: exchange l = 0 partials another way
    if (s.n_kv == 0) {
        // no cells: every row's softmax sum is 0, so the output is 0 (ops.cpp:9066); partials get l = 0
        const size_t row = (size_t) s.D * 4;
        if (dst->nb[1] != row || dst->nb[2] != row * s.H || dst->nb[3] != row * s.H * s.n_q) return KB_ERR_UNSUPPORTED;
        cudaStream_t cs = static_cast<cudaStream_t>(stream);
        if (cudaMemsetAsync(dst->data, 0, row * s.H * s.n_q * s.ne3, cs) != cudaSuccess) return KB_ERR_CUDA;
        if (dst_ml && cudaMemsetAsync(dst_ml, 0, (size_t) 2 * 4 * s.H * s.n_q * s.ne3, cs) != cudaSuccess)
            return KB_ERR_CUDA;
        return KB_OK;
    }
    const float log2e_ = 1.4426950408889634f;
    const bool partial = dst_ml != nullptr || push != nullptr;
    const bool quant_prefill =
        prefill_quant_shape(s, prm, partial) && scratch && scratch_bytes >= 2 * widen_view_bytes(s) &&
        aligned16(reinterpret_cast<uintptr_t>(scratch));
    if (use_prefill(s, prm, partial) || quant_prefill) {
        const bool qv4 = aligned16(reinterpret_cast<uintptr_t>(q->data)) && aligned16(q->nb[1]) && aligned16(q->nb[2]) &&
                         aligned16(q->nb[3]);
        if (!qv4 || !aligned16(dst->nb[1]) || !aligned16(dst->nb[2]) || !aligned16(dst->nb[3]) ||
            !aligned16(reinterpret_cast<uintptr_t>(dst->data)))
            return KB_ERR_UNSUPPORTED;
        kb::FaPrefillParams pp{};
        pp.q = static_cast<const char*>(q->data);
        pp.q_nb1 = (int64_t) q->nb[1], pp.q_nb2 = (int64_t) q->nb[2], pp.q_nb3 = (int64_t) q->nb[3];
        pp.n_q = s.n_q, pp.n_head = s.H, pp.n_head_kv = s.H_kv, pp.gqa = s.gqa, pp.ne3 = s.ne3, pp.rk3 = s.ne3 / s.ne3k;
        pp.n_qtiles = (s.n_q + 127) / 128;
        // CTA pairs share each MMA when the heads of a GQA group pair up (klein's 24 / 4 heads do)
        const bool pair = prefill_pair_enabled() && s.H % 2 == 0 && s.gqa % 2 == 0;
        pp.n_kv = s.n_kv;
        if (mask) {
            pp.mask = static_cast<const char*>(mask->data);
            pp.m_nb1 = (int64_t) mask->nb[1], pp.m_nb2 = (int64_t) mask->nb[2], pp.m_nb3 = (int64_t) mask->nb[3];
            pp.m_ne2 = (int) mask->ne[2], pp.m_ne3 = (int) mask->ne[3];
        }
        pp.scale_log2 = prm->scale * log2e_;
        pp.has_softcap = prm->logit_softcap != 0.0f;
        if (pp.has_softcap) {
            pp.scale_sc = prm->scale / prm->logit_softcap;
            pp.softcap_log2 = prm->logit_softcap * log2e_;
        }
        pp.max_bias = prm->max_bias;
        pp.n_head_log2 = 1 << (int) std::floor(std::log2((double) s.H));
        pp.m0 = std::pow(2.0f, -(prm->max_bias) / pp.n_head_log2);
        pp.m1 = std::pow(2.0f, -(prm->max_bias / 2.0f) / pp.n_head_log2);
        pp.causal = prm->causal, pp.pos0 = prm->pos0, pp.kv_lo = prm->kv_lo;
        pp.dst = static_cast<char*>(dst->data);
        pp.d_nb1 = (int64_t) dst->nb[1], pp.d_nb2 = (int64_t) dst->nb[2], pp.d_nb3 = (int64_t) dst->nb[3];
        if (gate) {
            pp.gate = static_cast<const char*>(gate->data);
            pp.g_nb1 = (int64_t) gate->nb[1], pp.g_nb2 = (int64_t) gate->nb[2], pp.g_nb3 = (int64_t) gate->nb[3];
        }
        pp.err = kb::device_error_word();
        pp.wait_ns = g_wait_ns;
        CUtensorMap tK, tV;
        cudaStream_t cs = static_cast<cudaStream_t>(stream);
        // a dense mask broadcast over the heads (klein's): classify its (query tile, 64-cell block) pieces first, so
        // that the kernel skips the hidden leading / trailing blocks and computes untouched blocks as unmasked ones
        const size_t cls_off = quant_prefill ? 2 * widen_view_bytes(s) : 0;
        if (mask && pp.m_ne2 == 1 && (pp.m_ne3 == 1 || s.ne3 == 1) && scratch &&
            scratch_bytes >= cls_off + mask_cls_bytes(s)) {
            uint8_t* cls = static_cast<uint8_t*>(scratch) + cls_off;
            const int n_blocks = (int) ((s.n_kv + 63) / 64);
            if (kb::launch_fa_mask_classify(pp.mask, pp.m_nb1, s.n_q, s.n_kv, n_blocks, cls, cs) != cudaSuccess)
                return KB_ERR_CUDA;
            pp.mask_cls = cls;
            pp.cls_ld = n_blocks;
        }
        if (quant_prefill) {
            // widen the cells the query tiles read (whole 64-cell blocks from kv_lo's block up to the last tile's
            // causal bound; every cell without causal bounds) into f16 views [ne3k][n_kv][H_kv][256] in the scratch
            int64_t c0 = 0, c1 = s.n_kv;
            if (prm->causal) {
                c0 = std::max<int64_t>(0, prm->kv_lo) / 64 * 64;
                const int64_t hi = std::min<int64_t>(s.n_kv, prm->pos0 + (int64_t) pp.n_qtiles * 128);
                c1 = hi > c0 ? std::min<int64_t>(s.n_kv, (hi + 63) / 64 * 64) : c0;
            }
            kb_tensor fv[2];
            const kb_tensor* src[2] = {k, v};
            for (int i = 0; i < 2; ++i) {
                kb_tensor& f = fv[i];
                f = kb_tensor{};
                f.type = KB_TYPE_F16;
                f.ne[0] = kb::FA_D, f.ne[1] = s.n_kv, f.ne[2] = s.H_kv, f.ne[3] = s.ne3k;
                f.nb[0] = 2, f.nb[2] = (size_t) kb::FA_D * 2, f.nb[1] = f.nb[2] * s.H_kv, f.nb[3] = f.nb[1] * s.n_kv;
                f.data = static_cast<char*>(scratch) + i * widen_view_bytes(s);
                if (c1 > c0) {
                    kb::KvWidenParams wp{};
                    wp.src = static_cast<const char*>(src[i]->data);
                    wp.s_nb1 = (int64_t) src[i]->nb[1], wp.s_nb2 = (int64_t) src[i]->nb[2], wp.s_nb3 = (int64_t) src[i]->nb[3];
                    wp.dst = static_cast<__half*>(f.data);
                    wp.n_kv = s.n_kv, wp.c0 = c0, wp.c1 = c1, wp.H_kv = s.H_kv, wp.ne3 = s.ne3k;
                    if (kb::launch_kv_widen(wp, s.kv_type, cs) != cudaSuccess) return KB_ERR_CUDA;
                }
            }
            if ((st = encode_kv_map(&fv[0], &tK, pair ? kb::FA_PAIR_KROWS : kb::FA_TILE)) != KB_OK) return st;
            if ((st = encode_kv_map(&fv[1], &tV)) != KB_OK) return st;
            return kb::launch_fa_prefill(pp, 2, pair, tK, tV, cs) == cudaSuccess ? KB_OK : KB_ERR_CUDA;
        }
        if ((st = encode_kv_map(k, &tK, pair ? kb::FA_PAIR_KROWS : kb::FA_TILE)) != KB_OK) return st;
        if ((st = encode_kv_map(v, &tV)) != KB_OK) return st;
        cudaError_t e = kb::launch_fa_prefill(pp, s.kv_type == KB_TYPE_BF16 ? 1 : 0, pair, tK, tV, cs);
        return e == cudaSuccess ? KB_OK : KB_ERR_CUDA;
    }
    if (s.kv_type == KB_TYPE_BF16) return KB_ERR_UNSUPPORTED;  // bf16 caches: prefill shapes only
    const FaPlan pl = plan_fa(s, push != nullptr);
    if (pl.scratch > 0 && (!scratch || scratch_bytes < pl.scratch)) return KB_ERR_SCRATCH;
    if (xchg) {
        // every CTA resident at once (one per SM), and the exchange's slots of rows within the flag array
        const int64_t slots = (int64_t) s.n_q * s.H;  // one flag word per output row and source rank
        const int64_t grid = (int64_t) pl.n_splits * s.H_kv * pl.n_row_chunks;
        const int sms = dev_info().sm_count > 0 ? dev_info().sm_count : 148;
        if (slots > kb::XCHG_MAX_SLOTS || grid > sms || (gate && !aligned16(gate->nb[1]))) return KB_ERR_UNSUPPORTED;
        if (!aligned16(dst->nb[1]) || !aligned16(dst->nb[2]) || (reinterpret_cast<uintptr_t>(dst->data) & 7) != 0)
            return KB_ERR_UNSUPPORTED;
    }

    kb::FaStreamParams p{};
    p.q = static_cast<const char*>(q->data);
    p.q_nb1 = (int64_t) q->nb[1];
    p.q_nb2 = (int64_t) q->nb[2];
    p.q_nb3 = (int64_t) q->nb[3];
    p.q_vec4 = aligned16(reinterpret_cast<uintptr_t>(q->data)) && aligned16(q->nb[1]) && aligned16(q->nb[2]) &&
               aligned16(q->nb[3]);
    p.n_q = s.n_q;
    p.n_head = s.H;
    p.n_head_kv = s.H_kv;
    p.gqa = s.gqa;
    p.ne3 = s.ne3;
    p.rk3 = s.ne3 / s.ne3k;
    p.R = s.R;
    p.n_kv = s.n_kv;
    if (mask) {
        p.mask = static_cast<const char*>(mask->data);
        p.m_nb1 = (int64_t) mask->nb[1];
        p.m_nb2 = (int64_t) mask->nb[2];
        p.m_nb3 = (int64_t) mask->nb[3];
        p.m_ne2 = (int) mask->ne[2];
        p.m_ne3 = (int) mask->ne[3];
    }
    const float log2e = 1.4426950408889634f;
    p.scale_log2 = prm->scale * log2e;
    p.has_softcap = prm->logit_softcap != 0.0f;
    if (p.has_softcap) {
        p.scale_sc = prm->scale / prm->logit_softcap;
        p.softcap_log2 = prm->logit_softcap * log2e;
    }
    p.max_bias = prm->max_bias;
    p.n_head_log2 = 1 << (int) std::floor(std::log2((double) s.H));
    p.m0 = std::pow(2.0f, -(prm->max_bias) / p.n_head_log2);
    p.m1 = std::pow(2.0f, -(prm->max_bias / 2.0f) / p.n_head_log2);
    p.causal = prm->causal;
    p.pos0 = prm->pos0;
    p.kv_lo = prm->kv_lo;
    p.ring = prm->causal ? prm->ring : 0;
    p.n_splits = pl.n_splits;
    p.blocks_base = pl.blocks_base;
    p.blocks_extra = pl.blocks_extra;
    p.n_row_chunks = pl.n_row_chunks;
    if (pl.scratch > 0) {
        const size_t rows = (size_t) s.H_kv * pl.n_row_chunks * s.ne3 * pl.n_splits * pl.rpc;
        p.o_part = static_cast<float*>(scratch);
        const uintptr_t ml = (reinterpret_cast<uintptr_t>(scratch) + rows * kb::FA_D * 4 + 255) & ~uintptr_t(255);
        p.ml_part = reinterpret_cast<float*>(ml);
    }
    p.dst = static_cast<char*>(dst->data);
    p.d_nb1 = (int64_t) dst->nb[1];
    p.d_nb2 = (int64_t) dst->nb[2];
    p.d_nb3 = (int64_t) dst->nb[3];
    if (gate) {
        p.gate = static_cast<const char*>(gate->data);
        p.g_nb1 = (int64_t) gate->nb[1], p.g_nb2 = (int64_t) gate->nb[2], p.g_nb3 = (int64_t) gate->nb[3];
    }
    p.partial_out = dst_ml != nullptr || (push != nullptr && !xchg);
    p.dst_ml = dst_ml;
    if (push) {
        p.push = xchg ? 0 : 1;
        p.xchg = xchg ? 1 : 0;
        p.rank = push->rank;
        p.n_ranks = push->n_ranks;
        p.slot_set_floats = push->slot_set_floats;
        p.part_floats = push->part_floats;
        for (int r = 0; r < push->n_ranks; ++r) {
            p.gather[r] = push->gather[r];
            p.flags[r] = push->flags[r];
        }
        p.push_counter = reinterpret_cast<int*>(static_cast<char*>(scratch) + pl.scratch - 256);
    }
    p.err = kb::device_error_word();
    p.wait_ns = g_wait_ns;

    CUtensorMap tmK, tmV;
    if ((st = encode_kv_map(k, &tmK)) != KB_OK) return st;
    if ((st = encode_kv_map(v, &tmV)) != KB_OK) return st;
    cudaError_t e = kb::launch_fa_stream_tc(p, pl.rpc, s.kv_type, tmK, tmV, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? KB_OK : KB_ERR_CUDA;
}

}  // namespace

namespace kb {

kb_status flash_attn_with_scratch(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* mask,
                                  const kb_fa_params* params, const kb_tensor* dst, void* scratch, size_t scratch_bytes,
                                  void* stream) {
    return fa_impl(q, k, v, mask, params, dst, nullptr, scratch, scratch_bytes, stream);
}

size_t flash_attn_scratch_bytes(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_fa_params* params) {
    return kb_flash_attn_ext_scratch_bytes(q, k, v, params);
}

size_t flash_attn_min_scratch_bytes(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v,
                                    const kb_fa_params* params) {
    FaShape s;
    if (check_fa(q, k, v, nullptr, &s) != KB_OK) return 0;
    if (use_prefill(s, params, false)) return 0;
    return plan_fa(s).scratch;
}

}  // namespace kb

extern "C" {

size_t kb_flash_attn_ext_push_scratch_bytes(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v,
                                            const kb_fa_params* params) {
    (void) params;
    FaShape s;
    if (check_fa(q, k, v, nullptr, &s) != KB_OK) return 0;
    return plan_fa(s, true).scratch;
}

kb_status kb_flash_attn_ext_push(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* mask,
                                 const kb_fa_params* params, int64_t part_floats, float* const* gather,
                                 int64_t slot_set_floats, int32_t* const* flags, int32_t rank, int32_t n_ranks,
                                 void* scratch, size_t scratch_bytes, void* stream) {
    if (!q || !gather || !flags || n_ranks < 1 || n_ranks > KB_MAX_PEERS || rank < 0 || rank >= n_ranks) return KB_ERR_ARG;
    // the packed partial of kb_partials_push: o [n_q * H][D], then (m, l) [n_q * H][2]
    const int64_t rows = q->ne[1] * q->ne[2], D = q->ne[0];
    if (part_floats < rows * D + rows * 2 || part_floats % 4 != 0 || slot_set_floats < n_ranks * part_floats)
        return KB_ERR_BAD_SHAPE;
    for (int r = 0; r < n_ranks; ++r)
        if (!gather[r] || !flags[r]) return KB_ERR_ARG;
    // a shape-only destination (nothing is stored through it in this mode)
    kb_tensor dst{};
    dst.type = KB_TYPE_F32;
    dst.ne[0] = D, dst.ne[1] = q->ne[2], dst.ne[2] = q->ne[1], dst.ne[3] = q->ne[3];
    dst.nb[0] = 4, dst.nb[1] = (size_t) D * 4, dst.nb[2] = dst.nb[1] * dst.ne[1], dst.nb[3] = dst.nb[2] * dst.ne[2];
    PushArgs pa{gather, flags, slot_set_floats, part_floats, rank, n_ranks};
    return fa_impl(q, k, v, mask, params, &dst, nullptr, scratch, scratch_bytes, stream, nullptr, &pa);
}

int32_t kb_flash_attn_ext_supported(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* mask,
                                    const kb_fa_params* params) {
    FaShape s;
    if (!params || check_fa(q, k, v, mask, &s) != KB_OK) return 0;
    if (params->logit_softcap != 0.0f && !std::isfinite(params->logit_softcap)) return 0;
    if (params->max_bias > 0.0f && !mask) return 0;
    if (params->causal && params->ring < 0) return 0;
    const bool prefill = use_prefill(s, params, false) || prefill_quant_shape(s, params, false);
    if (s.kv_type == KB_TYPE_BF16 && !prefill) return 0;  // bf16 caches: prefill shapes only
    // the prefill kernel loads Q rows and stores output rows in 16-byte units
    if (prefill && (!aligned16(q->nb[1]) || !aligned16(q->nb[2]) || !aligned16(q->nb[3]))) return 0;
    return 1;
}

size_t kb_exchange_flag_bytes(int32_t n_ranks) {
    if (n_ranks < 1 || n_ranks > KB_MAX_PEERS) return 0;
    return (size_t) (kb::XCHG_FLAG_BASE + n_ranks * kb::XCHG_MAX_SLOTS) * sizeof(int32_t);
}

kb_status kb_flash_attn_ext_exchange(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* mask,
                                     const kb_fa_params* params, const kb_tensor* gate, int64_t part_floats,
                                     float* const* gather, int64_t slot_set_floats, int32_t* const* flags, int32_t rank,
                                     int32_t n_ranks, const kb_tensor* dst, void* scratch, size_t scratch_bytes,
                                     void* stream) {
    if (!q || !dst || !gather || !flags || n_ranks < 1 || n_ranks > KB_MAX_PEERS || rank < 0 || rank >= n_ranks)
        return KB_ERR_ARG;
    const int64_t rows = q->ne[1] * q->ne[2], D = q->ne[0];
    if (part_floats < rows * D + rows * 2 || part_floats % 4 != 0 || slot_set_floats < n_ranks * part_floats ||
        slot_set_floats % 4 != 0)
        return KB_ERR_BAD_SHAPE;
    for (int r = 0; r < n_ranks; ++r) {
        if (!gather[r] || !flags[r]) return KB_ERR_ARG;
        if ((reinterpret_cast<uintptr_t>(gather[r]) & 15) != 0 || (reinterpret_cast<uintptr_t>(flags[r]) & 3) != 0)
            return KB_ERR_ARG;
    }
    PushArgs pa{gather, flags, slot_set_floats, part_floats, rank, n_ranks};
    return fa_impl(q, k, v, mask, params, dst, nullptr, scratch, scratch_bytes, stream, gate, &pa, true);
}

kb_status kb_flash_attn_ext_gated(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* mask,
                                  const kb_fa_params* params, const kb_tensor* gate, const kb_tensor* dst, void* scratch,
                                  size_t scratch_bytes, void* stream) {
    if (!gate) return KB_ERR_ARG;
    return fa_impl(q, k, v, mask, params, dst, nullptr, scratch, scratch_bytes, stream, gate);
}

kb_status kb_flash_attn_ext(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* mask,
                            const kb_fa_params* params, const kb_tensor* dst, void* scratch, size_t scratch_bytes,
                            void* stream) {
    return fa_impl(q, k, v, mask, params, dst, nullptr, scratch, scratch_bytes, stream);
}

kb_status kb_flash_attn_ext_partial(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* mask,
                                    const kb_fa_params* params, const kb_tensor* o_part, float* ml_part, void* scratch,
                                    size_t scratch_bytes, void* stream) {
    if (!ml_part) return KB_ERR_ARG;
    return fa_impl(q, k, v, mask, params, o_part, ml_part, scratch, scratch_bytes, stream);
}

kb_status kb_lse_combine(const float* o_parts, const float* ml_parts, int64_t part_stride, int32_t n_parts, int64_t rows,
                         int32_t head_dim, float* dst, void* stream) {
    if (!o_parts || !ml_parts || !dst || n_parts <= 0 || n_parts > 1024 || rows < 0 || head_dim <= 0) return KB_ERR_ARG;
    if (n_parts > 1 && part_stride < rows * head_dim) return KB_ERR_ARG;
    // vector loads: 16-byte aligned parts, head_dim a multiple of 8
    if (head_dim % 8 != 0 || part_stride % 4 != 0 || !aligned16(reinterpret_cast<uintptr_t>(o_parts)) ||
        (reinterpret_cast<uintptr_t>(ml_parts) & 7) != 0)
        return KB_ERR_ARG;
    return kb::launch_lse_combine(o_parts, ml_parts, part_stride, n_parts, rows, head_dim, dst,
                                  static_cast<cudaStream_t>(stream)) ==
                   cudaSuccess
               ? KB_OK
               : KB_ERR_CUDA;
}

kb_status kb_lse_combine_wait(const float* gather, int64_t part_stride, int64_t slot_set_floats, int32_t n_parts,
                              int64_t rows, int32_t head_dim, int32_t* flags, float* dst, void* stream) {
    if (!gather || !flags || !dst || n_parts <= 0 || n_parts > KB_MAX_PEERS || rows <= 0 || head_dim <= 0) return KB_ERR_ARG;
    if (part_stride < rows * head_dim + rows * 2 || slot_set_floats < part_stride * n_parts) return KB_ERR_ARG;
    if (head_dim % 8 != 0 || part_stride % 4 != 0 || slot_set_floats % 4 != 0 ||
        !aligned16(reinterpret_cast<uintptr_t>(gather)) || (reinterpret_cast<uintptr_t>(flags) & 3) != 0)
        return KB_ERR_ARG;
    return kb::launch_lse_combine(gather, gather + rows * head_dim, part_stride, n_parts, rows, head_dim, dst,
                                  static_cast<cudaStream_t>(stream), flags, slot_set_floats, kb::device_error_word(),
                                  g_wait_ns) == cudaSuccess
               ? KB_OK
               : KB_ERR_CUDA;
}

// ---------------------------------------------------------------------------------------------- peer exchange

kb_status kb_peer_alloc(size_t bytes, void** dev_ptr, void* ipc_handle) {
    if (!dev_ptr || !ipc_handle || bytes == 0) return KB_ERR_ARG;
    *dev_ptr = nullptr;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return KB_ERR_CUDA;
    cudaIpcMemHandle_t h;
    if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaFree(p);
        return KB_ERR_CUDA;
    }
    static_assert(sizeof(h) == KB_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(ipc_handle, &h, sizeof(h));
    *dev_ptr = p;
    return KB_OK;
}

kb_status kb_peer_open(const void* ipc_handle, void** dev_ptr) {
    if (!ipc_handle || !dev_ptr) return KB_ERR_ARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    return cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? KB_OK : KB_ERR_CUDA;
}

kb_status kb_peer_close(void* dev_ptr) {
    if (!dev_ptr) return KB_ERR_ARG;
    return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? KB_OK : KB_ERR_CUDA;
}

kb_status kb_peer_free(void* dev_ptr) {
    if (!dev_ptr) return KB_ERR_ARG;
    return cudaFree(dev_ptr) == cudaSuccess ? KB_OK : KB_ERR_CUDA;
}

kb_status kb_partials_push(const float* part, int64_t part_floats, float* const* gather, int64_t slot_set_floats,
                           int32_t* const* flags, int32_t rank, int32_t n_ranks, void* stream) {
    if (!part || !gather || !flags || n_ranks < 1 || n_ranks > KB_MAX_PEERS || rank < 0 || rank >= n_ranks ||
        part_floats <= 0 || part_floats % 4 != 0 || slot_set_floats < part_floats * n_ranks || slot_set_floats % 4 != 0)
        return KB_ERR_ARG;
    if (!aligned16(reinterpret_cast<uintptr_t>(part))) return KB_ERR_ARG;
    kb::PeerPushParams pp{};
    pp.part = part;
    pp.part_floats = part_floats;
    pp.slot_set_floats = slot_set_floats;
    for (int r = 0; r < n_ranks; ++r) {
        if (!gather[r] || !flags[r] || !aligned16(reinterpret_cast<uintptr_t>(gather[r]))) return KB_ERR_ARG;
        pp.gather[r] = gather[r];
        pp.flags[r] = flags[r];
    }
    pp.rank = rank;
    pp.n_ranks = n_ranks;
    return kb::launch_partials_push(pp, static_cast<cudaStream_t>(stream)) == cudaSuccess ? KB_OK : KB_ERR_CUDA;
}

// ---------------------------------------------------------------------------------------------- DeltaNet

}  // extern "C"

namespace {

bool rows_f32(const kb_tensor* t) { return t && t->type == KB_TYPE_F32 && t->nb[0] == 4; }

bool contiguous_f32(const kb_tensor* t) {
    return rows_f32(t) && t->nb[1] == (size_t) t->ne[0] * 4 && t->nb[2] == t->nb[1] * t->ne[1] &&
           t->nb[3] == t->nb[2] * t->ne[2];
}

int snap_code(int32_t type) { return type == KB_TYPE_F32 ? 0 : type == KB_TYPE_F16 ? 1 : type == KB_TYPE_BF16 ? 2 : -1; }

// checks the operands of GGML_OP_GATED_DELTA_NET (ggml.c:6375-6428) and fills the input half of the params
kb_status gdn_inputs(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* g,
                     const kb_tensor* beta, const kb_tensor* state, int32_t K, kb::GdnParams* p) {
    if (!q || !k || !v || !g || !beta || !state) return KB_ERR_ARG;
    if (!rows_f32(q) || !rows_f32(k) || !rows_f32(v) || !contiguous_f32(g) || !contiguous_f32(beta) ||
        !contiguous_f32(state))
        return KB_ERR_UNSUPPORTED;
    const int64_t S = v->ne[0], H = v->ne[1], T = v->ne[2], n_seqs = v->ne[3];
    if (K < 1 || T < 1 || n_seqs < 1) return KB_ERR_BAD_SHAPE;
    if (q->ne[0] != S || k->ne[0] != S || q->ne[1] != k->ne[1] || q->ne[2] != T || k->ne[2] != T) return KB_ERR_BAD_SHAPE;
    if (k->ne[1] <= 0 || H % k->ne[1] != 0 || n_seqs % q->ne[3] != 0 || n_seqs % k->ne[3] != 0) return KB_ERR_BAD_SHAPE;
    if (!(g->ne[0] == 1 || g->ne[0] == S) || g->ne[1] != H || g->ne[2] != T || g->ne[3] != n_seqs) return KB_ERR_BAD_SHAPE;
    if (beta->ne[0] != 1 || beta->ne[1] != H || beta->ne[2] != T || beta->ne[3] != n_seqs) return KB_ERR_BAD_SHAPE;
    if (state->ne[0] != S || state->ne[1] != S || state->ne[2] != H || state->ne[3] != n_seqs) return KB_ERR_BAD_SHAPE;
    if (S != 128) return KB_ERR_UNSUPPORTED;
    // float4 loads: q, k, state (and a per-channel gate) need 16-byte aligned rows
    for (const kb_tensor* t : {q, k, state, g}) {
        if (t == g && g->ne[0] != S) continue;
        if (!aligned16(reinterpret_cast<uintptr_t>(t->data)) || !aligned16(t->nb[1]) || !aligned16(t->nb[2]) ||
            !aligned16(t->nb[3]))
            return KB_ERR_UNSUPPORTED;
    }
    p->q = static_cast<const char*>(q->data);
    p->q_nb1 = q->nb[1], p->q_nb2 = q->nb[2], p->q_nb3 = q->nb[3];
    p->k = static_cast<const char*>(k->data);
    p->k_nb1 = k->nb[1], p->k_nb2 = k->nb[2], p->k_nb3 = k->nb[3];
    p->v = static_cast<const char*>(v->data);
    p->v_nb1 = v->nb[1], p->v_nb2 = v->nb[2], p->v_nb3 = v->nb[3];
    p->g = static_cast<const char*>(g->data);
    p->g_nb1 = g->nb[1], p->g_nb2 = g->nb[2], p->g_nb3 = g->nb[3];
    p->kda = g->ne[0] == S;
    p->beta = static_cast<const char*>(beta->data);
    p->b_nb1 = beta->nb[1], p->b_nb2 = beta->nb[2], p->b_nb3 = beta->nb[3];
    p->s0 = static_cast<const float*>(state->data);
    p->s0_seq_stride = (int64_t) (state->nb[3] / 4);
    p->S = (int) S, p->H_k = (int) k->ne[1], p->H_v = (int) H, p->T = (int) T, p->n_seqs = (int) n_seqs, p->K = K;
    p->rq3 = (int) (n_seqs / q->ne[3]);
    p->rk3 = (int) (n_seqs / k->ne[3]);
    return KB_OK;
}

// Prompt-length calls run the chunked tensor-core form over tokens [0, Tc), Tc = T - min(T, K) + 1: its final
// state is slot min(T, K) - 1. The remaining min(T, K) - 1 tokens, whose per-token states are the other slots,
// run through the recurrent kernel from there.
constexpr int64_t GDN_CHUNKED_MIN_TOKENS = 64;

int64_t gdn_chunked_tokens(int64_t T, int32_t K) { return T - std::min<int64_t>(T, K) + 1; }

size_t gdn_chunked_bytes(int64_t T, int32_t K, int64_t H_v, int64_t n_seqs, bool kda) {
    const int64_t Tc = gdn_chunked_tokens(T, K);
    if (kda || Tc < GDN_CHUNKED_MIN_TOKENS) return 0;
    return (size_t) (n_seqs * H_v * ((Tc + kb::GDN_CHUNK - 1) / kb::GDN_CHUNK) * kb::GDN_REC_BYTES);
}

// the chunked kernel writes its outputs by TMA: f32 (value dim, head, token, sequence), box 128 x 1 x 64 x 1,
// tokens clipped at tok_end
bool encode_attn_map(const kb::GdnParams& p, int64_t tok_end, CUtensorMap* map) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[4] = {(cuuint64_t) p.S, (cuuint64_t) p.H_v, (cuuint64_t) tok_end, (cuuint64_t) p.n_seqs};
    const cuuint64_t strides[3] = {(cuuint64_t) p.a_nb1, (cuuint64_t) p.a_nb2, (cuuint64_t) p.a_nb3};
    const cuuint32_t box[4] = {(cuuint32_t) p.S, 1, (cuuint32_t) kb::GDN_CHUNK, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.attn, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A side stream per device and a set of events for the overlapped chunked schedule below, created on first use
// and kept for the process (streams and events, no device memory). The mutex keeps two host threads from
// interleaving their records of the shared events.
constexpr int GDN_MAX_PARTS = 16;
constexpr int64_t GDN_PART_CHUNKS = 16;  // chunks per part (64 tokens each)
struct GdnOverlap {
    cudaStream_t side = nullptr;   // the records, lowest priority
    cudaStream_t chain = nullptr;  // the state chain, highest priority: a part's chain, once its records are ready,
                                   // takes SMs ahead of the next part's records
    cudaEvent_t fork = nullptr, join = nullptr;
    cudaEvent_t part[GDN_MAX_PARTS] = {};
    bool ok = false;
};
std::mutex g_overlap_mu;

GdnOverlap* gdn_overlap() {
    static GdnOverlap per_dev[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    GdnOverlap& o = per_dev[dev];
    if (!o.ok) {
        int lo = 0, hi = 0;
        if (cudaDeviceGetStreamPriorityRange(&lo, &hi) != cudaSuccess) return nullptr;
        if (cudaStreamCreateWithPriority(&o.side, cudaStreamNonBlocking, lo) != cudaSuccess) return nullptr;
        if (cudaStreamCreateWithPriority(&o.chain, cudaStreamNonBlocking, hi) != cudaSuccess) return nullptr;
        if (cudaEventCreateWithFlags(&o.fork, cudaEventDisableTiming) != cudaSuccess) return nullptr;
        if (cudaEventCreateWithFlags(&o.join, cudaEventDisableTiming) != cudaSuccess) return nullptr;
        for (cudaEvent_t& e : o.part)
            if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return nullptr;
        o.ok = true;
    }
    return &o;
}

kb_status gdn_run(const kb::GdnParams& p, bool packed, void* scratch, size_t scratch_bytes, cudaStream_t stream) {
    const int64_t S = p.S, T = p.T, n_w = std::min<int64_t>(T, p.K), Tc = gdn_chunked_tokens(T, p.K);
    const int64_t per_chunk = (int64_t) p.n_seqs * p.H_v * kb::GDN_REC_BYTES;
    const bool out_ok = aligned16(reinterpret_cast<uintptr_t>(p.attn)) && aligned16(p.a_nb1) && aligned16(p.a_nb2) &&
                        aligned16(p.a_nb3);
    const bool chunked = gdn_chunked_bytes(T, p.K, p.H_v, p.n_seqs, p.kda) > 0 && scratch && out_ok &&
                         (int64_t) scratch_bytes >= per_chunk && aligned16(reinterpret_cast<uintptr_t>(scratch));
    if (!chunked) return kb::launch_gdn_recurrent(p, stream) == cudaSuccess ? KB_OK : KB_ERR_CUDA;
    // the chunked part leaves slot n_w - 1: in the packed result, or in the f32 state (+ its snapshot row)
    float* s_out;
    char* snap = nullptr;
    if (packed) {
        s_out = reinterpret_cast<float*>(n_w == 1 ? p.slot0 : p.slots + (n_w - 2) * p.slots_stride);
    } else {
        s_out = reinterpret_cast<float*>(p.slot0);
        if (n_w >= 2) snap = p.slots + (n_w - 2) * p.slots_stride;
    }
    const int64_t state_stride = S * S * p.H_v;  // floats per sequence
    kb::GdnChunkParams c{};
    c.in = p;
    c.rec = static_cast<char*>(scratch);
    c.s_out = s_out;
    c.s_out_seq_stride = state_stride;
    c.snap_type = p.slots_type;
    c.err = kb::device_error_word();
    c.wait_ns = g_wait_ns;
    const int64_t n_chunks = (Tc + kb::GDN_CHUNK - 1) / kb::GDN_CHUNK;
    const int64_t per_pass = std::min<int64_t>(n_chunks, (int64_t) scratch_bytes / per_chunk);
    const int64_t n_parts = (n_chunks + GDN_PART_CHUNKS - 1) / GDN_PART_CHUNKS;
    GdnOverlap* ov = per_pass == n_chunks && n_parts >= 2 && n_parts <= GDN_MAX_PARTS ? gdn_overlap() : nullptr;
    if (ov) {
        // Overlapped schedule: the state chain runs on 48 SMs (one CTA per head) while the rest would idle, so the
        // records of part k + 1 are prepared on a side stream while part k's chain runs; part k's chain waits only
        // for part k's records (stream order and events; no kernel waits on another). Every part's records have
        // their own region of the scratch.
        std::lock_guard<std::mutex> lock(g_overlap_mu);
        if (cudaEventRecord(ov->fork, stream) != cudaSuccess || cudaStreamWaitEvent(ov->side, ov->fork, 0) != cudaSuccess ||
            cudaStreamWaitEvent(ov->chain, ov->fork, 0) != cudaSuccess)
            return KB_ERR_CUDA;
        std::vector<kb::GdnChunkParams> parts;
        for (int64_t k = 0; k < n_parts; ++k) {
            const int64_t c0 = k * GDN_PART_CHUNKS, nc = std::min(GDN_PART_CHUNKS, n_chunks - c0);
            kb::GdnChunkParams c2 = c;
            c2.rec = static_cast<char*>(scratch) + c0 * per_chunk;
            c2.tok0 = c0 * kb::GDN_CHUNK;
            c2.n_tok = std::min(nc * kb::GDN_CHUNK, Tc - c2.tok0);
            c2.n_chunks = (int) nc;
            c2.s0 = c0 == 0 ? p.s0 : s_out;
            c2.s0_seq_stride = c0 == 0 ? p.s0_seq_stride : state_stride;
            c2.snap = k == n_parts - 1 ? snap : nullptr;
            if (kb::launch_gdn_prep(c2, ov->side) != cudaSuccess) return KB_ERR_CUDA;
            if (cudaEventRecord(ov->part[k], ov->side) != cudaSuccess) return KB_ERR_CUDA;
            parts.push_back(c2);
        }
        for (int64_t k = 0; k < n_parts; ++k) {
            CUtensorMap tmO;
            if (!encode_attn_map(p, parts[k].tok0 + parts[k].n_tok, &tmO)) return KB_ERR_CUDA;
            if (cudaStreamWaitEvent(ov->chain, ov->part[k], 0) != cudaSuccess) return KB_ERR_CUDA;
            if (kb::launch_gdn_state(parts[k], tmO, ov->chain) != cudaSuccess) return KB_ERR_CUDA;
        }
        if (cudaEventRecord(ov->join, ov->chain) != cudaSuccess || cudaStreamWaitEvent(stream, ov->join, 0) != cudaSuccess)
            return KB_ERR_CUDA;
    }
    for (int64_t c0 = 0; !ov && c0 < n_chunks; c0 += per_pass) {
        const int64_t nc = std::min(per_pass, n_chunks - c0);
        c.tok0 = c0 * kb::GDN_CHUNK;
        c.n_tok = std::min(nc * kb::GDN_CHUNK, Tc - c.tok0);
        c.n_chunks = (int) nc;
        c.s0 = c0 == 0 ? p.s0 : s_out;
        c.s0_seq_stride = c0 == 0 ? p.s0_seq_stride : state_stride;
        c.snap = c0 + nc >= n_chunks ? snap : nullptr;
        CUtensorMap tmO;
        if (!encode_attn_map(p, c.tok0 + c.n_tok, &tmO)) return KB_ERR_CUDA;
        if (kb::launch_gdn_chunked(c, tmO, stream) != cudaSuccess) return KB_ERR_CUDA;
    }
    if (n_w == 1) return KB_OK;
    kb::GdnParams t = p;
    t.q += Tc * p.q_nb2;
    t.k += Tc * p.k_nb2;
    t.v += Tc * p.v_nb2;
    t.g += Tc * p.g_nb2;
    t.beta += Tc * p.b_nb2;
    t.attn += Tc * p.a_nb2;
    t.T = (int) (n_w - 1);
    t.s0 = s_out;
    t.s0_seq_stride = state_stride;
    return kb::launch_gdn_recurrent(t, stream) == cudaSuccess ? KB_OK : KB_ERR_CUDA;
}

}  // namespace

extern "C" {

kb_status kb_gated_delta_net(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* g,
                             const kb_tensor* beta, const kb_tensor* state, int32_t K, const kb_tensor* dst,
                             void* scratch, size_t scratch_bytes, void* stream) {
    kb::GdnParams p{};
    kb_status st = gdn_inputs(q, k, v, g, beta, state, K, &p);
    if (st != KB_OK) return st;
    if (!dst) return KB_ERR_ARG;
    const int64_t S = p.S, H = p.H_v, T = p.T, n_seqs = p.n_seqs;
    // ggml's packed result: [S*H, T*n_seqs + K*S*n_seqs] f32, contiguous
    if (!contiguous_f32(dst) || dst->ne[0] != S * H || dst->ne[1] != T * n_seqs + (int64_t) K * S * n_seqs ||
        dst->ne[2] != 1 || dst->ne[3] != 1)
        return KB_ERR_BAD_SHAPE;
    if (!aligned16(reinterpret_cast<uintptr_t>(dst->data))) return KB_ERR_UNSUPPORTED;
    char* base = static_cast<char*>(dst->data);
    p.attn = base;
    p.a_nb1 = S * 4, p.a_nb2 = S * H * 4, p.a_nb3 = S * H * T * 4;
    const int64_t attn_bytes = S * H * T * n_seqs * 4, slot_bytes = S * S * H * n_seqs * 4;
    p.slot0 = base + attn_bytes;
    p.slots = base + attn_bytes + slot_bytes;
    p.slots_stride = slot_bytes;
    p.slots_type = 0;
    return gdn_run(p, true, scratch, scratch_bytes, static_cast<cudaStream_t>(stream));
}

kb_status kb_gated_delta_net_cache(const kb_tensor* q, const kb_tensor* k, const kb_tensor* v, const kb_tensor* g,
                                   const kb_tensor* beta, const kb_tensor* state, const kb_tensor* snap, int32_t K,
                                   const kb_tensor* attn, void* scratch, size_t scratch_bytes, void* stream) {
    kb::GdnParams p{};
    kb_status st = gdn_inputs(q, k, v, g, beta, state, K, &p);
    if (st != KB_OK) return st;
    if (!attn || !rows_f32(attn)) return KB_ERR_ARG;
    if (attn->ne[0] != p.S || attn->ne[1] != p.H_v || attn->ne[2] != p.T || attn->ne[3] != p.n_seqs) return KB_ERR_BAD_SHAPE;
    const int n_written = p.T < K ? p.T : K;
    if (n_written > 1) {
        // snapshot rows: [S*S*H*n_seqs, >= n_written - 1], contiguous rows of f16 / bf16 / f32
        if (!snap) return KB_ERR_ARG;
        const int code = snap_code(snap->type);
        if (code < 0) return KB_ERR_UNSUPPORTED;
        const int64_t es = code == 0 ? 4 : 2;
        if (snap->ne[0] != (int64_t) p.S * p.S * p.H_v * p.n_seqs || snap->ne[1] < n_written - 1 ||
            snap->nb[0] != (size_t) es || !aligned16(reinterpret_cast<uintptr_t>(snap->data)) || !aligned16(snap->nb[1]))
            return KB_ERR_BAD_SHAPE;
        p.slots = static_cast<char*>(snap->data);
        p.slots_stride = (int64_t) snap->nb[1];
        p.slots_type = code;
    }
    p.attn = static_cast<char*>(attn->data);
    p.a_nb1 = attn->nb[1], p.a_nb2 = attn->nb[2], p.a_nb3 = attn->nb[3];
    p.slot0 = static_cast<char*>(state->data);  // slot 0 overwrites the state it was computed from
    return gdn_run(p, false, scratch, scratch_bytes, static_cast<cudaStream_t>(stream));
}

size_t kb_gated_delta_net_scratch_bytes(const kb_tensor* v, const kb_tensor* g, int32_t K) {
    if (!v || !g || K < 1 || v->ne[0] != 128) return 0;
    return gdn_chunked_bytes(v->ne[2], K, v->ne[1], v->ne[3], g->ne[0] != 1);
}

kb_status kb_set_rows(const kb_tensor* dst, const kb_tensor* src, const kb_tensor* idx, void* stream) {
    if (!dst || !src || !idx) return KB_ERR_ARG;
    if (!rows_f32(src)) return KB_ERR_UNSUPPORTED;
    if (idx->type != KB_TYPE_I64 && idx->type != KB_TYPE_I32) return KB_ERR_UNSUPPORTED;
    const int t = dst->type;
    if (t != KB_TYPE_F32 && t != KB_TYPE_F16 && t != KB_TYPE_BF16 && t != KB_TYPE_Q8_0 && t != KB_TYPE_Q4_0)
        return KB_ERR_UNSUPPORTED;
    const int64_t ne0 = src->ne[0];
    const bool quant = t == KB_TYPE_Q8_0 || t == KB_TYPE_Q4_0;
    if (dst->ne[0] != ne0 || ne0 % 32 != 0) return quant || dst->ne[0] != ne0 ? KB_ERR_BAD_SHAPE : KB_ERR_UNSUPPORTED;
    if (dst->ne[2] != src->ne[2] || dst->ne[3] != src->ne[3] || idx->ne[0] != src->ne[1]) return KB_ERR_BAD_SHAPE;
    if (idx->ne[1] <= 0 || idx->ne[2] <= 0 || src->ne[2] % idx->ne[1] != 0 || src->ne[3] % idx->ne[2] != 0)
        return KB_ERR_BAD_SHAPE;
    const size_t es = t == KB_TYPE_F32 ? 4 : t == KB_TYPE_Q8_0 ? 34 : t == KB_TYPE_Q4_0 ? 18 : 2;
    if (dst->nb[0] != es) return KB_ERR_BAD_SHAPE;
    kb::SetRowsParams p{};
    p.src = static_cast<const char*>(src->data);
    p.s_nb1 = src->nb[1], p.s_nb2 = src->nb[2], p.s_nb3 = src->nb[3];
    p.idx = static_cast<const char*>(idx->data);
    p.i_nb0 = idx->nb[0], p.i_nb1 = idx->nb[1], p.i_nb2 = idx->nb[2];
    p.idx_i32 = idx->type == KB_TYPE_I32;
    p.ne11 = idx->ne[1], p.ne12 = idx->ne[2];
    p.dst = static_cast<char*>(dst->data);
    p.d_nb1 = dst->nb[1], p.d_nb2 = dst->nb[2], p.d_nb3 = dst->nb[3];
    p.dst_type = t;
    p.ne0 = ne0, p.n_src = src->ne[1], p.ne2 = src->ne[2], p.ne3 = src->ne[3], p.n_rows = dst->ne[1];
    p.err = kb::device_error_word();
    return kb::launch_set_rows(p, static_cast<cudaStream_t>(stream)) == cudaSuccess ? KB_OK : KB_ERR_CUDA;
}

kb_status kb_attn_prologue(const kb_tensor* qfull, const kb_tensor* kcur, const kb_tensor* vcur, const kb_tensor* pos,
                           const kb_tensor* kv_idx, const kb_tensor* q_norm, const kb_tensor* k_norm, float rms_eps,
                           const kb_rope_params* rope, const kb_tensor* q_out, const kb_tensor* gate_out,
                           const kb_tensor* k_cache, const kb_tensor* v_cache, void* stream) {
    if (!qfull || !kcur || !vcur || !pos || !kv_idx || !q_norm || !k_norm || !rope || !q_out || !gate_out || !k_cache ||
        !v_cache)
        return KB_ERR_ARG;
    if (!rows_f32(qfull) || !rows_f32(kcur) || !rows_f32(vcur) || !contiguous_f32(q_norm) || !contiguous_f32(k_norm) ||
        !contiguous_f32(q_out) || !contiguous_f32(gate_out))
        return KB_ERR_UNSUPPORTED;
    if (pos->type != KB_TYPE_I32 || kv_idx->type != KB_TYPE_I64) return KB_ERR_UNSUPPORTED;
    const int64_t hd = q_norm->ne[0];
    if (hd != 64 && hd != 128 && hd != 256) return KB_ERR_UNSUPPORTED;
    const int64_t n = qfull->ne[1];
    if (qfull->ne[0] % (2 * hd) != 0 || kcur->ne[0] % hd != 0) return KB_ERR_BAD_SHAPE;
    const int64_t nh = qfull->ne[0] / (2 * hd), nkv = kcur->ne[0] / hd;
    if (nh <= 0 || nkv <= 0 || k_norm->ne[0] != hd || vcur->ne[0] != kcur->ne[0] || kcur->ne[1] != n ||
        vcur->ne[1] != n || pos->ne[0] < 4 * n || kv_idx->ne[0] != n)
        return KB_ERR_BAD_SHAPE;
    if (q_out->ne[0] != hd || q_out->ne[1] != nh || q_out->ne[2] != n || gate_out->ne[0] != hd * nh || gate_out->ne[1] != n)
        return KB_ERR_BAD_SHAPE;
    const int ct = k_cache->type;
    if ((ct != KB_TYPE_F16 && ct != KB_TYPE_Q8_0 && ct != KB_TYPE_Q4_0) || v_cache->type != ct) return KB_ERR_UNSUPPORTED;
    if (k_cache->ne[0] != hd * nkv || v_cache->ne[0] != hd * nkv || v_cache->ne[1] != k_cache->ne[1]) return KB_ERR_BAD_SHAPE;
    if (k_cache->nb[0] != (ct == KB_TYPE_F16 ? 2u : ct == KB_TYPE_Q8_0 ? 34u : 18u) || v_cache->nb[0] != k_cache->nb[0])
        return KB_ERR_BAD_SHAPE;
    if (rope->n_rot <= 0 || rope->n_rot % 64 != 0 || rope->n_rot > hd) return KB_ERR_UNSUPPORTED;
    if (rope->mode != 40 && rope->mode != 8) return KB_ERR_UNSUPPORTED;
    const int sect = rope->sections[0] + rope->sections[1] + rope->sections[2] + rope->sections[3];
    if (sect <= 0 || rope->sections[0] < 0 || rope->sections[1] < 0 || rope->sections[2] < 0 || rope->sections[3] < 0)
        return KB_ERR_BAD_SHAPE;
    if (n == 0) return KB_OK;
    kb::PrologueParams p{};
    p.qfull = static_cast<const char*>(qfull->data);
    p.q_nb1 = (int64_t) qfull->nb[1];
    p.kcur = static_cast<const char*>(kcur->data);
    p.vcur = static_cast<const char*>(vcur->data);
    p.k_nb1 = (int64_t) kcur->nb[1];
    p.v_nb1 = (int64_t) vcur->nb[1];
    p.pos = static_cast<const int32_t*>(pos->data);
    p.kv_idx = static_cast<const int64_t*>(kv_idx->data);
    p.q_norm = static_cast<const float*>(q_norm->data);
    p.k_norm = static_cast<const float*>(k_norm->data);
    p.q_out = static_cast<float*>(q_out->data);
    p.gate_out = static_cast<float*>(gate_out->data);
    p.gate_vec = aligned16(reinterpret_cast<uintptr_t>(qfull->data)) && aligned16(qfull->nb[1]) &&
                 aligned16(reinterpret_cast<uintptr_t>(gate_out->data));
    p.k_cache = static_cast<char*>(k_cache->data);
    p.v_cache = static_cast<char*>(v_cache->data);
    p.kc_nb1 = (int64_t) k_cache->nb[1];
    p.vc_nb1 = (int64_t) v_cache->nb[1];
    p.n_cells = k_cache->ne[1];
    p.cache_type = ct;
    p.n = (int) n;
    p.nh = (int) nh;
    p.nkv = (int) nkv;
    p.eps = rms_eps;
    p.n_rot = rope->n_rot;
    for (int i = 0; i < 4; ++i) p.sections[i] = rope->sections[i];
    p.sect_dims = sect;
    p.imrope = rope->mode == 40;
    // ggml: theta_scale = powf(freq_base, -2.0f / n_dims) (ops.cpp:6371)
    p.theta_scale = std::pow(rope->freq_base, -2.0f / (float) rope->n_rot);
    p.freq_scale = rope->freq_scale;
    p.attn_factor = rope->attn_factor;
    p.err = kb::device_error_word();
    return kb::launch_attn_prologue(p, (int) hd, static_cast<cudaStream_t>(stream)) == cudaSuccess ? KB_OK : KB_ERR_CUDA;
}

kb_status kb_gdn_input(const kb_tensor* qkv, const kb_tensor* conv_state, const kb_tensor* conv_w,
                       const kb_tensor* beta_raw, const kb_tensor* alpha, const kb_tensor* dt_bias, const kb_tensor* a,
                       int32_t S, int32_t H_k, float rms_eps, const kb_tensor* q_out, const kb_tensor* k_out,
                       const kb_tensor* v_out, const kb_tensor* beta_out, const kb_tensor* g_out, void* stream) {
    if (!qkv || !conv_state || !conv_w || !q_out || !k_out || !v_out) return KB_ERR_ARG;
    if (!!beta_raw != !!alpha) return KB_ERR_ARG;
    if (beta_raw && (!dt_bias || !a || !beta_out || !g_out)) return KB_ERR_ARG;
    if (S != 64 && S != 128) return KB_ERR_UNSUPPORTED;
    for (const kb_tensor* t : {qkv, conv_state, conv_w, q_out, k_out, v_out})
        if (!contiguous_f32(t)) return KB_ERR_UNSUPPORTED;
    const int64_t ch = qkv->ne[0], n = qkv->ne[1];
    if (H_k <= 0 || ch <= 2 * (int64_t) S * H_k || (ch - 2 * (int64_t) S * H_k) % S != 0) return KB_ERR_BAD_SHAPE;
    const int64_t H_v = (ch - 2 * (int64_t) S * H_k) / S;
    const int64_t kc = conv_w->ne[0];
    if (kc != 4) return KB_ERR_UNSUPPORTED;
    if (conv_w->ne[1] != ch || conv_state->ne[0] != (kc - 1) * ch || conv_state->ne[1] < 1) return KB_ERR_BAD_SHAPE;
    if (q_out->ne[0] != S || q_out->ne[1] != H_k || q_out->ne[2] != n || k_out->ne[0] != S || k_out->ne[1] != H_k ||
        k_out->ne[2] != n || v_out->ne[0] != S || v_out->ne[1] != H_v || v_out->ne[2] != n)
        return KB_ERR_BAD_SHAPE;
    if (beta_raw) {
        for (const kb_tensor* t : {beta_raw, alpha, dt_bias, a, beta_out, g_out})
            if (!contiguous_f32(t)) return KB_ERR_UNSUPPORTED;
        for (const kb_tensor* t : {beta_raw, alpha, beta_out, g_out})
            if (t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3] != H_v * n || (t->ne[0] != H_v && t->ne[1] != H_v))
                return KB_ERR_BAD_SHAPE;
        if (dt_bias->ne[0] * dt_bias->ne[1] != H_v || a->ne[0] * a->ne[1] != H_v) return KB_ERR_BAD_SHAPE;
    }
    if (n == 0) return KB_OK;
    kb::GdnInputParams p{};
    p.qkv = static_cast<const float*>(qkv->data);
    p.qkv_ld = ch;
    p.state = static_cast<float*>(conv_state->data);
    p.state_ld = conv_state->ne[0];
    p.conv_w = static_cast<const float*>(conv_w->data);
    if (beta_raw) {
        p.beta_raw = static_cast<const float*>(beta_raw->data);
        p.alpha = static_cast<const float*>(alpha->data);
        p.dt_bias = static_cast<const float*>(dt_bias->data);
        p.a = static_cast<const float*>(a->data);
        p.beta_out = static_cast<float*>(beta_out->data);
        p.g_out = static_cast<float*>(g_out->data);
    }
    p.q_out = static_cast<float*>(q_out->data);
    p.k_out = static_cast<float*>(k_out->data);
    p.v_out = static_cast<float*>(v_out->data);
    p.n = (int) n;
    p.H_k = H_k;
    p.H_v = (int) H_v;
    p.K = (int) conv_state->ne[1];
    // l2 (graph.cpp:41-44): rms_norm with eps / n, then a scale of 1 / sqrt(n), n = S (computed as klein does)
    p.l2_eps = rms_eps / (float) S;
    p.inv_sqrt_s = 1.0f / std::sqrt((float) S);
    return kb::launch_gdn_input(p, S, static_cast<cudaStream_t>(stream)) == cudaSuccess ? KB_OK : KB_ERR_CUDA;
}

kb_status kb_gdn_gated_norm(const kb_tensor* x, const kb_tensor* z, const kb_tensor* w, float rms_eps,
                            const kb_tensor* dst, void* stream) {
    if (!x || !z || !w || !dst) return KB_ERR_ARG;
    for (const kb_tensor* t : {x, z, w, dst})
        if (!contiguous_f32(t)) return KB_ERR_UNSUPPORTED;
    const int64_t S = w->ne[0];
    if (S != 64 && S != 128) return KB_ERR_UNSUPPORTED;
    const int64_t total = x->ne[0] * x->ne[1] * x->ne[2] * x->ne[3];
    if (x->ne[0] != S || total % S != 0 || z->ne[0] * z->ne[1] * z->ne[2] * z->ne[3] != total ||
        dst->ne[0] * dst->ne[1] * dst->ne[2] * dst->ne[3] != total)
        return KB_ERR_BAD_SHAPE;
    kb::GdnNormParams p{};
    p.x = static_cast<const float*>(x->data);
    p.z = static_cast<const float*>(z->data);
    p.w = static_cast<const float*>(w->data);
    p.dst = static_cast<float*>(dst->data);
    p.H = (int) x->ne[1];
    p.n = (int) (total / (S * x->ne[1]));
    p.eps = rms_eps;
    return kb::launch_gdn_gated_norm(p, (int) S, static_cast<cudaStream_t>(stream)) == cudaSuccess ? KB_OK : KB_ERR_CUDA;
}

size_t kb_gdn_step_sync_bytes(int32_t H_k) { return H_k > 0 ? (size_t) H_k * sizeof(int32_t) : 0; }

kb_status kb_gdn_step(const kb_tensor* qkv, const kb_tensor* conv_state, const kb_tensor* conv_w,
                      const kb_tensor* beta_raw, const kb_tensor* alpha, const kb_tensor* dt_bias, const kb_tensor* a,
                      const kb_tensor* ssm, const kb_tensor* ssm_snap, int32_t n_snapshots, const kb_tensor* z,
                      const kb_tensor* ssm_norm, float rms_eps, int32_t* sync, const kb_tensor* out, void* stream) {
    if (!qkv || !conv_state || !conv_w || !beta_raw || !alpha || !dt_bias || !a || !ssm || !z || !ssm_norm || !sync ||
        !out)
        return KB_ERR_ARG;
    if (n_snapshots < 1 || (n_snapshots > 1 && !ssm_snap)) return KB_ERR_ARG;
    constexpr int64_t S = 128;
    for (const kb_tensor* t : {qkv, conv_state, conv_w, beta_raw, alpha, dt_bias, a, ssm, z, ssm_norm, out})
        if (!contiguous_f32(t) || !aligned16(reinterpret_cast<uintptr_t>(t->data))) return KB_ERR_UNSUPPORTED;
    const int64_t n = qkv->ne[1], ch = qkv->ne[0];
    if (n < 1 || n > 4 || qkv->ne[2] * qkv->ne[3] != 1) return KB_ERR_UNSUPPORTED;
    if (ssm_norm->ne[0] * ssm_norm->ne[1] != S) return KB_ERR_UNSUPPORTED;
    const int64_t H_v = ssm->ne[0] * ssm->ne[1] * ssm->ne[2] * ssm->ne[3] / (S * S);
    if (H_v < 1 || H_v * S * S != ssm->ne[0] * ssm->ne[1] * ssm->ne[2] * ssm->ne[3]) return KB_ERR_BAD_SHAPE;
    const int64_t qk = ch - S * H_v;  // 2 S H_k
    if (qk <= 0 || qk % (2 * S)) return KB_ERR_BAD_SHAPE;
    const int64_t H_k = qk / (2 * S);
    if (H_v % H_k) return KB_ERR_UNSUPPORTED;
    if (conv_w->ne[0] != 4) return KB_ERR_UNSUPPORTED;
    if (conv_w->ne[1] != ch || conv_state->ne[0] != 3 * ch || conv_state->ne[1] != n_snapshots) return KB_ERR_BAD_SHAPE;
    for (const kb_tensor* t : {beta_raw, alpha})
        if (t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3] != H_v * n || (t->ne[0] != H_v && t->ne[1] != H_v))
            return KB_ERR_BAD_SHAPE;
    if (dt_bias->ne[0] * dt_bias->ne[1] != H_v || a->ne[0] * a->ne[1] != H_v) return KB_ERR_BAD_SHAPE;
    const int64_t rows = S * H_v * n;
    if (z->ne[0] * z->ne[1] * z->ne[2] * z->ne[3] != rows || out->ne[0] * out->ne[1] * out->ne[2] * out->ne[3] != rows)
        return KB_ERR_BAD_SHAPE;
    kb::GdnStepParams p{};
    const int64_t n_written = n < n_snapshots ? n : n_snapshots;
    if (n_written > 1) {
        const int code = snap_code(ssm_snap->type);
        if (code < 0) return KB_ERR_UNSUPPORTED;
        const size_t es = code == 0 ? 4 : 2;
        if (ssm_snap->ne[0] != S * S * H_v || ssm_snap->ne[1] < n_written - 1 || ssm_snap->nb[0] != es)
            return KB_ERR_BAD_SHAPE;
        if (!aligned16(reinterpret_cast<uintptr_t>(ssm_snap->data)) || !aligned16(ssm_snap->nb[1])) return KB_ERR_UNSUPPORTED;
        p.snap = static_cast<char*>(ssm_snap->data);
        p.snap_stride = (int64_t) ssm_snap->nb[1];
        p.snap_type = code;
    }
    if (reinterpret_cast<uintptr_t>(sync) & 3) return KB_ERR_ARG;
    p.qkv = static_cast<const float*>(qkv->data);
    p.qkv_ld = ch;
    p.conv_state = static_cast<float*>(conv_state->data);
    p.conv_ld = conv_state->ne[0];
    p.conv_w = static_cast<const float*>(conv_w->data);
    p.beta_raw = static_cast<const float*>(beta_raw->data);
    p.alpha = static_cast<const float*>(alpha->data);
    p.dt_bias = static_cast<const float*>(dt_bias->data);
    p.a = static_cast<const float*>(a->data);
    p.state = static_cast<float*>(ssm->data);
    p.z = static_cast<const float*>(z->data);
    p.norm_w = static_cast<const float*>(ssm_norm->data);
    p.out = static_cast<float*>(out->data);
    p.sync = sync;
    p.T = (int) n, p.H_k = (int) H_k, p.H_v = (int) H_v, p.K = n_snapshots;
    // as kb_gdn_input (graph.cpp:41-44) and kb_gdn_gated_norm
    p.l2_eps = rms_eps / (float) S;
    p.inv_sqrt_s = 1.0f / std::sqrt((float) S);
    p.eps = rms_eps;
    p.err = kb::device_error_word();
    p.wait_ns = g_wait_ns;
    return kb::launch_gdn_step(p, static_cast<cudaStream_t>(stream)) == cudaSuccess ? KB_OK : KB_ERR_CUDA;
}

kb_status kb_rollback_recurrent(int32_t n_layers, float* const* conv, int64_t conv_row, const void* const* snap,
                                int32_t snap_type, float* const* ssm, int64_t ssm_row, int32_t s, int32_t n_snapshots,
                                void* stream) {
    if (s <= 0) return KB_OK;  // nothing rejected (state.cpp:163)
    if (s >= n_snapshots) return KB_ERR_ARG;
    if (n_layers < 0 || n_layers > kb::MAX_ROLLBACK_LAYERS || !conv || !snap || !ssm) return KB_ERR_ARG;
    const int code = snap_code(snap_type);
    if (code < 0) return KB_ERR_UNSUPPORTED;
    if (conv_row % 4 != 0 || ssm_row % 4 != 0 || conv_row <= 0 || ssm_row <= 0) return KB_ERR_UNSUPPORTED;
    kb::RollbackParams p{};
    for (int l = 0; l < n_layers; ++l) {
        if (!conv[l] || !snap[l] || !ssm[l] || !aligned16(reinterpret_cast<uintptr_t>(conv[l])) ||
            !aligned16(reinterpret_cast<uintptr_t>(ssm[l])) || (reinterpret_cast<uintptr_t>(snap[l]) & 7) != 0)
            return KB_ERR_ARG;
        p.conv[l] = conv[l];
        p.snap[l] = static_cast<const char*>(snap[l]);
        p.ssm[l] = ssm[l];
    }
    p.n_layers = n_layers, p.conv_row = conv_row, p.ssm_row = ssm_row, p.snap_type = code, p.s = s;
    return kb::launch_rollback(p, static_cast<cudaStream_t>(stream)) == cudaSuccess ? KB_OK : KB_ERR_CUDA;
}

kb_status kb_device_error(int32_t* code, int clear) {
    if (!code) return KB_ERR_ARG;
    int* w = kb::device_error_word();
    if (!w) return KB_ERR_CUDA;
    int v = 0;
    if (cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return KB_ERR_CUDA;
    *code = v;
    if (clear && cudaMemset(w, 0, sizeof(int)) != cudaSuccess) return KB_ERR_CUDA;
    return KB_OK;
}

}  // extern "C"
