// klein's per-sequence State (src/state.h, src/state.cpp) kept resident in HBM, the per-pass indexing of
// Engine::run (src/engine.cpp:254-326), the accept / rollback bookkeeping of Engine::generate's verify step
// (engine.cpp:574-590), and Builder::attention / Builder::deltanet (src/graph.cpp:87-191) bound to that state
// without their weight GEMMs (those stay with the caller).
//
// Layout, as klein's (state.cpp:37-88): per full-attention layer a K and a V cache [kv_row, n_ctx] of type_k /
// type_v (token-major rows of n_head_kv * head_dim values); the MTP layer's caches are a ring of
// min(n_ctx, mtp_window) rows; per DeltaNet layer conv [(kc - 1) * channels, n_snapshots] f32 (slot 0 current),
// ssm [d_state^2 * dt_rank] f32 and ssm_snap [d_state^2 * dt_rank, n_snapshots - 1] of snap_type. Everything is one
// device allocation on the device current at creation; klein's pinned / mapped host KV and its bulk host view
// (state.cpp:110-134) are not needed when the cache is in HBM: the streaming kernels and the prefill kernel read the
// same device rows.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "../../include/klein_b200.h"

namespace {

constexpr size_t ALIGN = 256;

size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ggml_row_size for the cache and snapshot types this library stores
bool row_bytes(int32_t type, int64_t n, size_t* out) {
    switch (type) {
        case KB_TYPE_F32: *out = (size_t) n * 4; return true;
        case KB_TYPE_F16:
        case KB_TYPE_BF16: *out = (size_t) n * 2; return true;
        case KB_TYPE_Q8_0: if (n % 32) return false; *out = (size_t) n / 32 * 34; return true;
        case KB_TYPE_Q4_0: if (n % 32) return false; *out = (size_t) n / 32 * 18; return true;
        default: return false;
    }
}

// nb[0] of a cache view: the element size, or the block size of a block-quantised type
size_t elem_bytes(int32_t type) {
    return type == KB_TYPE_Q8_0 ? 34 : type == KB_TYPE_Q4_0 ? 18 : type == KB_TYPE_F32 ? 4 : 2;
}

bool valid_dims(const kb_qwen35_dims* d) {
    return d && d->n_layer > 0 && d->full_attn_interval > 0 && d->n_head > 0 && d->n_head_kv > 0 &&
           d->n_head % d->n_head_kv == 0 && d->head_dim > 0 && d->ssm_conv_kernel > 1 && d->ssm_d_state > 0 &&
           d->ssm_n_group > 0 && d->ssm_dt_rank > 0 && d->ssm_dt_rank % d->ssm_n_group == 0;
}

bool valid_cfg(const kb_state_config* c) {
    if (!c || c->n_ctx <= 0 || c->n_snapshots < 1 || c->mtp_window <= 0) return false;
    for (int32_t t : {c->type_k, c->type_v})
        if (t != KB_TYPE_F16 && t != KB_TYPE_Q8_0 && t != KB_TYPE_Q4_0 && t != KB_TYPE_BF16) return false;
    return c->snap_type == KB_TYPE_F16 || c->snap_type == KB_TYPE_BF16 || c->snap_type == KB_TYPE_F32;
}

bool is_recurrent(const kb_qwen35_dims* d, int il) { return il < d->n_layer && ((il + 1) % d->full_attn_interval) != 0; }
int n_attn_layers(const kb_qwen35_dims* d) { return d->n_layer / d->full_attn_interval; }
int64_t kv_row(const kb_qwen35_dims* d) { return (int64_t) d->n_head_kv * d->head_dim; }
int64_t conv_channels(const kb_qwen35_dims* d) {
    return (int64_t) d->ssm_dt_rank * d->ssm_d_state + 2 * (int64_t) d->ssm_n_group * d->ssm_d_state;
}
int64_t conv_row(const kb_qwen35_dims* d) { return (int64_t) (d->ssm_conv_kernel - 1) * conv_channels(d); }
int64_t ssm_row(const kb_qwen35_dims* d) { return (int64_t) d->ssm_d_state * d->ssm_d_state * d->ssm_dt_rank; }
int mtp_cells(const kb_state_config* c) { return std::min(c->n_ctx, c->mtp_window); }

// graph.cpp:16-19
int64_t padded_n_kv(int64_t n_past_after, int64_t n_ctx) { return std::min(n_ctx, (n_past_after + 255) / 256 * 256); }

kb_tensor tensor2d(int32_t type, int64_t ne0, int64_t ne1, size_t row, void* data) {
    kb_tensor t{};
    t.type = type;
    t.ne[0] = ne0, t.ne[1] = ne1, t.ne[2] = 1, t.ne[3] = 1;
    t.nb[0] = elem_bytes(type), t.nb[1] = row, t.nb[2] = row * (size_t) ne1, t.nb[3] = t.nb[2];
    t.data = data;
    return t;
}

kb_tensor f32_tensor(void* data, int64_t n0, int64_t n1, int64_t n2 = 1, int64_t n3 = 1) {
    kb_tensor t{};
    t.type = KB_TYPE_F32;
    t.ne[0] = n0, t.ne[1] = n1, t.ne[2] = n2, t.ne[3] = n3;
    t.nb[0] = 4, t.nb[1] = (size_t) n0 * 4, t.nb[2] = t.nb[1] * (size_t) n1, t.nb[3] = t.nb[2] * (size_t) n2;
    t.data = data;
    return t;
}

struct Layer {
    int64_t cells = 0;  // attention layers: cache rows (0 for a DeltaNet layer)
    size_t k_off = 0, v_off = 0, conv_off = 0, ssm_off = 0, snap_off = 0, sync_off = 0;
    bool has_snap = false;
    void *k = nullptr, *v = nullptr;                        // attention layers
    void *conv = nullptr, *ssm = nullptr, *snap = nullptr;  // DeltaNet layers
    int32_t* sync = nullptr;                                // DeltaNet layers: kb_gdn_step's counters (ssm_n_group)
};

}  // namespace

struct kb_state {
    kb_qwen35_dims dims;
    kb_state_config cfg;
    int device = 0;
    void* base = nullptr;
    size_t bytes = 0;
    bool owns = false;  // base from cudaMalloc (kb_state_create) or the caller's (kb_state_create_in)
    size_t row_k = 0, row_v = 0, snap_row = 0;
    std::vector<Layer> layers;  // n_layer decoder layers, then the MTP layer when there is one
    int64_t n_past = 0, n_past_mtp = 0;
};

namespace {

// the allocation of a state: (offset, bytes) of every tensor, laid out in one buffer
struct Plan {
    size_t total = 0, kv = 0, mtp_kv = 0, recurrent = 0;
};

bool plan_state(const kb_qwen35_dims* d, const kb_state_config* c, kb_state* st, Plan* pl) {
    size_t rk, rv, rs;
    if (!row_bytes(c->type_k, kv_row(d), &rk) || !row_bytes(c->type_v, kv_row(d), &rv) ||
        !row_bytes(c->snap_type, ssm_row(d), &rs))
        return false;
    if (rk % 16 || rv % 16) return false;  // TMA rows
    size_t off = 0;
    auto take = [&](size_t n) {
        const size_t at = off;
        off = round_up(off + n, ALIGN);
        return at;
    };
    std::vector<Layer> L(d->n_layer + (d->with_mtp ? 1 : 0));
    for (int il = 0; il < (int) L.size(); ++il) {
        const bool mtp = il >= d->n_layer;
        if (mtp || !is_recurrent(d, il)) {
            const int64_t cells = mtp ? mtp_cells(c) : c->n_ctx;
            L[il].cells = cells;
            L[il].k_off = take(rk * (size_t) cells);
            L[il].v_off = take(rv * (size_t) cells);
            (mtp ? pl->mtp_kv : pl->kv) += (rk + rv) * (size_t) cells;
        } else {
            L[il].conv_off = take((size_t) conv_row(d) * 4 * c->n_snapshots);
            L[il].ssm_off = take((size_t) ssm_row(d) * 4);
            L[il].has_snap = c->n_snapshots > 1;
            if (L[il].has_snap) L[il].snap_off = take(rs * (size_t) (c->n_snapshots - 1));
            pl->recurrent += (size_t) conv_row(d) * 4 * c->n_snapshots + (size_t) ssm_row(d) * 4 +
                             rs * (size_t) (c->n_snapshots - 1);
        }
    }
    // kb_gdn_step's counters, one set per DeltaNet layer (zero between calls)
    for (Layer& l : L)
        if (!l.cells) l.sync_off = take((size_t) d->ssm_n_group * sizeof(int32_t));
    pl->total = off;
    if (st) {
        st->row_k = rk, st->row_v = rv, st->snap_row = rs;
        st->layers = L;
    }
    return true;
}

}  // namespace

extern "C" {

kb_status kb_state_sizes(const kb_qwen35_dims* dims, const kb_state_config* cfg, size_t* kv_bytes, size_t* mtp_kv_bytes,
                         size_t* recurrent_bytes) {
    if (!valid_dims(dims) || !valid_cfg(cfg)) return KB_ERR_ARG;
    Plan pl;
    if (!plan_state(dims, cfg, nullptr, &pl)) return KB_ERR_UNSUPPORTED;
    if (kv_bytes) *kv_bytes = pl.kv;
    if (mtp_kv_bytes) *mtp_kv_bytes = pl.mtp_kv;
    if (recurrent_bytes) *recurrent_bytes = pl.recurrent;
    return KB_OK;
}

size_t kb_state_required_bytes(const kb_qwen35_dims* dims, const kb_state_config* cfg) {
    if (!valid_dims(dims) || !valid_cfg(cfg)) return 0;
    Plan pl;
    return plan_state(dims, cfg, nullptr, &pl) ? pl.total : 0;
}

namespace {

kb_status make_state(const kb_qwen35_dims* dims, const kb_state_config* cfg, void* base, size_t bytes, kb_state** out) {
    if (!out) return KB_ERR_ARG;
    *out = nullptr;
    if (!valid_dims(dims) || !valid_cfg(cfg)) return KB_ERR_ARG;
    if (dims->n_layer - n_attn_layers(dims) > 64) return KB_ERR_UNSUPPORTED;  // one rollback launch covers 64 layers
    kb_state* st = new kb_state();
    st->dims = *dims;
    st->cfg = *cfg;
    Plan pl;
    if (!plan_state(dims, cfg, st, &pl)) {
        delete st;
        return KB_ERR_UNSUPPORTED;
    }
    if (cudaGetDevice(&st->device) != cudaSuccess) {
        delete st;
        return KB_ERR_CUDA;
    }
    if (base) {
        if (bytes < pl.total || (reinterpret_cast<uintptr_t>(base) & (ALIGN - 1))) {
            delete st;
            return KB_ERR_SCRATCH;
        }
        st->base = base;
    } else {
        if (cudaMalloc(&st->base, pl.total) != cudaSuccess) {
            delete st;
            return KB_ERR_CUDA;
        }
        st->owns = true;
    }
    st->bytes = pl.total;
    char* b = static_cast<char*>(st->base);
    for (Layer& l : st->layers) {
        if (l.cells) {
            l.k = b + l.k_off;
            l.v = b + l.v_off;
        } else {
            l.conv = b + l.conv_off;
            l.ssm = b + l.ssm_off;
            l.snap = l.has_snap ? b + l.snap_off : nullptr;
            l.sync = reinterpret_cast<int32_t*>(b + l.sync_off);
        }
    }
    // State::State clears every buffer (state.cpp:140); the KV cells beyond n_past are masked anyway
    if (cudaMemset(st->base, 0, pl.total) != cudaSuccess) {
        if (st->owns) cudaFree(st->base);
        delete st;
        return KB_ERR_CUDA;
    }
    *out = st;
    return KB_OK;
}

}  // namespace

kb_status kb_state_create(const kb_qwen35_dims* dims, const kb_state_config* cfg, kb_state** out) {
    return make_state(dims, cfg, nullptr, 0, out);
}

kb_status kb_state_create_in(const kb_qwen35_dims* dims, const kb_state_config* cfg, void* base, size_t bytes,
                             kb_state** out) {
    if (!base) return KB_ERR_ARG;
    return make_state(dims, cfg, base, bytes, out);
}

kb_status kb_state_destroy(kb_state* st) {
    if (!st) return KB_OK;
    if (!st->owns) {
        delete st;
        return KB_OK;
    }
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != st->device) cudaSetDevice(st->device);
    const cudaError_t e = cudaFree(st->base);
    if (cur != st->device) cudaSetDevice(cur);
    delete st;
    return e == cudaSuccess ? KB_OK : KB_ERR_CUDA;
}

size_t kb_state_device_bytes(const kb_state* st) { return st ? st->bytes : 0; }

kb_status kb_state_get_layer(const kb_state* st, int32_t il, kb_state_layer* out) {
    if (!st || !out || il < 0 || il >= (int) st->layers.size()) return KB_ERR_ARG;
    *out = kb_state_layer{};
    const Layer& l = st->layers[il];
    const kb_qwen35_dims& d = st->dims;
    if (l.cells) {
        out->k = tensor2d(st->cfg.type_k, kv_row(&d), l.cells, st->row_k, l.k);
        out->v = tensor2d(st->cfg.type_v, kv_row(&d), l.cells, st->row_v, l.v);
    } else {
        out->conv = tensor2d(KB_TYPE_F32, conv_row(&d), st->cfg.n_snapshots, (size_t) conv_row(&d) * 4, l.conv);
        out->ssm = tensor2d(KB_TYPE_F32, ssm_row(&d), 1, (size_t) ssm_row(&d) * 4, l.ssm);
        if (l.snap) out->ssm_snap = tensor2d(st->cfg.snap_type, ssm_row(&d), st->cfg.n_snapshots - 1, st->snap_row, l.snap);
    }
    return KB_OK;
}

int64_t kb_state_n_past(const kb_state* st, int32_t mtp) { return !st ? -1 : mtp ? st->n_past_mtp : st->n_past; }

kb_status kb_state_set_n_past(kb_state* st, int32_t mtp, int64_t n_past) {
    if (!st || n_past < 0 || n_past > st->cfg.n_ctx) return KB_ERR_ARG;
    (mtp ? st->n_past_mtp : st->n_past) = n_past;
    return KB_OK;
}

// State::clear (state.cpp:148-160): the recurrent state and snapshots to zero, n_past to 0
kb_status kb_state_clear(kb_state* st, void* stream) {
    if (!st) return KB_ERR_ARG;
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    const kb_qwen35_dims& d = st->dims;
    for (const Layer& l : st->layers) {
        if (!l.conv) continue;
        if (cudaMemsetAsync(l.conv, 0, (size_t) conv_row(&d) * 4 * st->cfg.n_snapshots, cs) != cudaSuccess ||
            cudaMemsetAsync(l.ssm, 0, (size_t) ssm_row(&d) * 4, cs) != cudaSuccess ||
            (l.snap && cudaMemsetAsync(l.snap, 0, st->snap_row * (size_t) (st->cfg.n_snapshots - 1), cs) != cudaSuccess))
            return KB_ERR_CUDA;
    }
    st->n_past = 0;
    st->n_past_mtp = 0;
    return KB_OK;
}

// State::rollback_recurrent (state.cpp:162-183): slot s becomes the current state of every DeltaNet layer
kb_status kb_state_rollback(kb_state* st, int32_t s, void* stream) {
    if (!st) return KB_ERR_ARG;
    if (s <= 0) return KB_OK;
    if (s >= st->cfg.n_snapshots) return KB_ERR_ARG;
    std::vector<float*> conv, ssm;
    std::vector<const void*> snap;
    for (const Layer& l : st->layers) {
        if (!l.conv) continue;
        conv.push_back(static_cast<float*>(l.conv));
        ssm.push_back(static_cast<float*>(l.ssm));
        snap.push_back(l.snap);
    }
    if (conv.empty()) return KB_OK;
    return kb_rollback_recurrent((int32_t) conv.size(), conv.data(), conv_row(&st->dims), snap.data(), st->cfg.snap_type,
                                 ssm.data(), ssm_row(&st->dims), s, st->cfg.n_snapshots, stream);
}

// Engine::run's per-pass indexing (engine.cpp:254-326) for a pass of n_tokens cells from cell0: the ring of the MTP
// layer, the padded number of cells attended, each token's cache row, and the visibility rule as analytic bounds
// (kb_fa_params: the dense mask klein builds on the host is the same set of cells).
kb_status kb_plan_pass(const kb_qwen35_dims* dims, const kb_state_config* cfg, int32_t mtp, int32_t n_tokens,
                       int64_t cell0, int64_t kv_lo, kb_pass* out, int64_t* kv_idx) {
    if (!valid_dims(dims) || !valid_cfg(cfg) || !out || n_tokens <= 0 || cell0 < 0 || kv_lo < 0) return KB_ERR_ARG;
    if (mtp && !dims->with_mtp) return KB_ERR_ARG;
    if (cell0 + n_tokens > cfg->n_ctx) return KB_ERR_ARG;  // "context full" (engine.cpp:253)
    const int64_t ring = mtp && mtp_cells(cfg) < cfg->n_ctx ? mtp_cells(cfg) : 0;
    *out = kb_pass{};
    out->n_tokens = n_tokens;
    out->cell0 = cell0;
    out->kv_lo = kv_lo;
    out->mtp = mtp;
    out->ring = ring;
    out->n_kv = ring ? std::min<int64_t>(ring, padded_n_kv(cell0 + n_tokens, cfg->n_ctx))
                     : padded_n_kv(cell0 + n_tokens, cfg->n_ctx);
    out->fa.scale = 1.0f / std::sqrt((float) dims->head_dim);
    out->fa.prec = 10;  // GGML_PREC_F32 (graph.cpp:121); this library accumulates in f32 in any case
    out->fa.causal = 1;
    out->fa.pos0 = cell0;
    out->fa.kv_lo = kv_lo;
    out->fa.ring = ring;
    if (kv_idx)
        for (int i = 0; i < n_tokens; ++i) kv_idx[i] = ring > 0 ? (cell0 + i) % ring : cell0 + i;
    return KB_OK;
}

kb_status kb_state_plan_pass(const kb_state* st, int32_t mtp, int32_t n_tokens, int64_t kv_lo, kb_pass* out,
                             int64_t* kv_idx) {
    if (!st) return KB_ERR_ARG;
    return kb_plan_pass(&st->dims, &st->cfg, mtp, n_tokens, mtp ? st->n_past_mtp : st->n_past, kv_lo, out, kv_idx);
}

// Engine::generate after a verify pass of n_batch cells from `base` (engine.cpp:584-590): keep `next` and the
// accepted drafts, roll the DeltaNet states back past the rejected ones
kb_status kb_state_accept(kb_state* st, int64_t base, int32_t n_batch, int32_t accepted, void* stream) {
    if (!st || n_batch < 1 || accepted < 0 || accepted > n_batch - 1 || base < 0 || base + n_batch > st->cfg.n_ctx)
        return KB_ERR_ARG;
    const int rejected = (n_batch - 1) - accepted;
    if (rejected >= st->cfg.n_snapshots) return KB_ERR_ARG;
    st->n_past = base + accepted + 1;
    return rejected > 0 ? kb_state_rollback(st, rejected, stream) : KB_OK;
}

// ---------------------------------------------------------------------------------------------- layer composition

namespace {

bool attn_layer_of(const kb_state* st, int32_t il, const kb_pass* pass) {
    if (!st || !pass || il < 0 || il >= (int) st->layers.size() || !st->layers[il].cells) return false;
    return (il >= st->dims.n_layer) == (pass->mtp != 0);
}

// the prologue's outputs, then the attention's scratch
struct AttnScratch {
    size_t q_off, gate_off, fa_off, total, fa_bytes;
};

void attn_views(const kb_state* st, int32_t il, const kb_pass* pass, void* q_data, void* gate_data, void* out_data,
                kb_tensor* q, kb_tensor* k, kb_tensor* v, kb_tensor* gate, kb_tensor* out) {
    const kb_qwen35_dims& d = st->dims;
    const Layer& l = st->layers[il];
    const int64_t hd = d.head_dim, nh = d.n_head, nkv = d.n_head_kv, n = pass->n_tokens;
    // Q after the prologue: [hd, nh, n] contiguous, seen as klein's permuted view [hd, n, nh] (graph.cpp:118)
    *q = kb_tensor{};
    q->type = KB_TYPE_F32;
    q->ne[0] = hd, q->ne[1] = n, q->ne[2] = nh, q->ne[3] = 1;
    q->nb[0] = 4, q->nb[1] = (size_t) (hd * nh * 4), q->nb[2] = (size_t) (hd * 4), q->nb[3] = (size_t) (hd * nh * n * 4);
    q->data = q_data;
    // K / V: [hd, n_kv, nkv] views of the cache rows (graph.cpp:114-117)
    for (int i = 0; i < 2; ++i) {
        kb_tensor& t = i ? *v : *k;
        const int32_t type = i ? st->cfg.type_v : st->cfg.type_k;
        const size_t row = i ? st->row_v : st->row_k;
        size_t head;
        row_bytes(type, hd, &head);
        t = kb_tensor{};
        t.type = type;
        t.ne[0] = hd, t.ne[1] = pass->n_kv, t.ne[2] = nkv, t.ne[3] = 1;
        t.nb[0] = elem_bytes(type), t.nb[1] = row, t.nb[2] = head, t.nb[3] = row * (size_t) l.cells;
        t.data = i ? l.v : l.k;
    }
    // gate and output: [hd * nh, n] contiguous, seen as ggml's permuted result [hd, nh, n]
    *gate = f32_tensor(gate_data, hd, nh, n);
    *out = f32_tensor(out_data, hd, nh, n);
}

AttnScratch attn_scratch(const kb_state* st, int32_t il, const kb_pass* pass) {
    AttnScratch s{};
    const size_t t = round_up((size_t) st->dims.head_dim * st->dims.n_head * pass->n_tokens * 4, ALIGN);
    s.q_off = 0;
    s.gate_off = t;
    s.fa_off = 2 * t;
    kb_tensor q, k, v, g, o;
    attn_views(st, il, pass, reinterpret_cast<void*>(ALIGN), nullptr, nullptr, &q, &k, &v, &g, &o);
    s.fa_bytes = kb_flash_attn_ext_scratch_bytes(&q, &k, &v, &pass->fa);
    s.total = s.fa_off + round_up(s.fa_bytes, ALIGN);
    return s;
}

}  // namespace

size_t kb_layer_attention_scratch_bytes(const kb_state* st, int32_t il, const kb_pass* pass) {
    if (!attn_layer_of(st, il, pass)) return 0;
    return attn_scratch(st, il, pass).total;
}

kb_status kb_layer_attention(kb_state* st, int32_t il, const kb_pass* pass, const kb_tensor* qfull, const kb_tensor* kcur,
                             const kb_tensor* vcur, const kb_tensor* pos, const kb_tensor* kv_idx, const kb_tensor* q_norm,
                             const kb_tensor* k_norm, float rms_eps, const kb_rope_params* rope, const kb_tensor* out,
                             void* scratch, size_t scratch_bytes, void* stream) {
    if (!attn_layer_of(st, il, pass) || !out) return KB_ERR_ARG;
    const kb_qwen35_dims& d = st->dims;
    if (out->type != KB_TYPE_F32 || out->ne[0] != (int64_t) d.head_dim * d.n_head || out->ne[1] != pass->n_tokens ||
        out->nb[0] != 4 || out->nb[1] != (size_t) d.head_dim * d.n_head * 4)
        return KB_ERR_BAD_SHAPE;
    const AttnScratch sc = attn_scratch(st, il, pass);
    if (!scratch || scratch_bytes < sc.total || (reinterpret_cast<uintptr_t>(scratch) & (ALIGN - 1))) return KB_ERR_SCRATCH;
    char* base = static_cast<char*>(scratch);
    kb_tensor q, k, v, gate, o;
    attn_views(st, il, pass, base + sc.q_off, base + sc.gate_off, out->data, &q, &k, &v, &gate, &o);
    kb_state_layer lv;
    kb_state_get_layer(st, il, &lv);
    // Q / gate split, RMS norms, M-RoPE and the K / V cache writes at kv_idx (graph.cpp:94-112)
    const kb_tensor q_out = f32_tensor(base + sc.q_off, d.head_dim, d.n_head, pass->n_tokens);
    const kb_tensor gate_out = f32_tensor(base + sc.gate_off, (int64_t) d.head_dim * d.n_head, pass->n_tokens);
    kb_status s = kb_attn_prologue(qfull, kcur, vcur, pos, kv_idx, q_norm, k_norm, rms_eps, rope, &q_out, &gate_out,
                                   &lv.k, &lv.v, stream);
    if (s != KB_OK) return s;
    // attention over the padded cells with the output gate in its store (graph.cpp:113-124)
    return kb_flash_attn_ext_gated(&q, &k, &v, nullptr, &pass->fa, &gate, &o, base + sc.fa_off, sc.fa_bytes, stream);
}

namespace {

struct GdnScratch {
    size_t q, k, v, beta, g, attn, op, total, op_bytes;
};

GdnScratch gdn_scratch(const kb_state* st, int32_t n) {
    const kb_qwen35_dims& d = st->dims;
    const size_t S = d.ssm_d_state, Hk = d.ssm_n_group, Hv = d.ssm_dt_rank;
    GdnScratch s{};
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = round_up(off + bytes, ALIGN);
        return at;
    };
    s.q = take(S * Hk * n * 4);
    s.k = take(S * Hk * n * 4);
    s.v = take(S * Hv * n * 4);
    s.beta = take(Hv * n * 4);
    s.g = take(Hv * n * 4);
    s.attn = take(S * Hv * n * 4);
    s.op = off;
    const kb_tensor vt = f32_tensor(nullptr, (int64_t) S, (int64_t) Hv, n);
    const kb_tensor gt = f32_tensor(nullptr, 1, (int64_t) Hv, n);
    s.op_bytes = kb_gated_delta_net_scratch_bytes(&vt, &gt, st->cfg.n_snapshots);
    s.total = s.op + round_up(s.op_bytes, ALIGN);
    return s;
}

}  // namespace

size_t kb_layer_deltanet_scratch_bytes(const kb_state* st, int32_t il, int32_t n_tokens) {
    if (!st || il < 0 || il >= st->dims.n_layer || !st->layers[il].conv || n_tokens <= 0) return 0;
    return gdn_scratch(st, n_tokens).total;
}

kb_status kb_layer_deltanet(kb_state* st, int32_t il, int32_t n_tokens, const kb_tensor* qkv, const kb_tensor* z,
                            const kb_tensor* beta_raw, const kb_tensor* alpha, const kb_tensor* dt_bias, const kb_tensor* a,
                            const kb_tensor* conv_w, const kb_tensor* ssm_norm, float rms_eps, const kb_tensor* out,
                            void* scratch, size_t scratch_bytes, void* stream) {
    if (!st || il < 0 || il >= st->dims.n_layer || !st->layers[il].conv || n_tokens <= 0 || !out) return KB_ERR_ARG;
    const kb_qwen35_dims& d = st->dims;
    const int64_t S = d.ssm_d_state, Hk = d.ssm_n_group, Hv = d.ssm_dt_rank, n = n_tokens;
    if (!qkv || qkv->ne[1] != n) return KB_ERR_BAD_SHAPE;
    kb_state_layer lv;
    kb_state_get_layer(st, il, &lv);
    if (n <= 4) {
        // decode / verify passes: the whole layer in one launch (same results as the three calls below)
        const kb_status s = kb_gdn_step(qkv, &lv.conv, conv_w, beta_raw, alpha, dt_bias, a, &lv.ssm,
                                        lv.ssm_snap.data ? &lv.ssm_snap : nullptr, st->cfg.n_snapshots, z, ssm_norm,
                                        rms_eps, st->layers[il].sync, out, stream);
        if (s != KB_ERR_UNSUPPORTED) return s;
    }
    const GdnScratch sc = gdn_scratch(st, n_tokens);
    if (!scratch || scratch_bytes < sc.total || (reinterpret_cast<uintptr_t>(scratch) & (ALIGN - 1))) return KB_ERR_SCRATCH;
    char* b = static_cast<char*>(scratch);
    const kb_tensor q = f32_tensor(b + sc.q, S, Hk, n), k = f32_tensor(b + sc.k, S, Hk, n);
    const kb_tensor v = f32_tensor(b + sc.v, S, Hv, n);
    const kb_tensor beta = f32_tensor(b + sc.beta, Hv, n), g = f32_tensor(b + sc.g, Hv, n);
    // conv state slots and snapshots, conv + SiLU, L2 norms, beta and g (graph.cpp:136-165)
    kb_status s = kb_gdn_input(qkv, &lv.conv, conv_w, beta_raw, alpha, dt_bias, a, (int32_t) S, (int32_t) Hk, rms_eps, &q,
                               &k, &v, &beta, &g, stream);
    if (s != KB_OK) return s;
    // the recurrence into the state (slot 0) and the snapshot rows (graph.cpp:166-184)
    const kb_tensor g4 = f32_tensor(b + sc.g, 1, Hv, n), beta4 = f32_tensor(b + sc.beta, 1, Hv, n);
    const kb_tensor state = f32_tensor(lv.ssm.data, S, S, Hv);
    const kb_tensor attn = f32_tensor(b + sc.attn, S, Hv, n);
    s = kb_gated_delta_net_cache(&q, &k, &v, &g4, &beta4, &state, lv.ssm_snap.data ? &lv.ssm_snap : nullptr,
                                 st->cfg.n_snapshots, &attn, sc.op_bytes ? b + sc.op : nullptr, sc.op_bytes, stream);
    if (s != KB_OK) return s;
    // gated RMS norm (graph.cpp:186-190)
    return kb_gdn_gated_norm(&attn, z, ssm_norm, rms_eps, out, stream);
}

}  // extern "C"
