// Harness around the reference's own ggml CPU ops (TEST INFRASTRUCTURE: parity checker + timed CPU
// baseline; never linked into the klein_b200 product).
//
// Each entry point binds caller-owned host buffers to ggml tensors with exactly the views klein's graph
// builds, runs one node on ggml's CPU backend and returns. Nothing is copied into ggml-owned memory, so
// the 262,144-cell KV caches of the long-verify configuration are used in place.
//
//   kbref_flash_attn_ext   ggml_flash_attn_ext + ggml_prec_set_acc(F32) as in src/graph.cpp:113-121
//                          (q [hd, n, nh] permuted view, k/v [hd, n_kv, nkv] permuted cache views);
//                          CPU op third_party/ggml/src/ggml-cpu/ops.cpp:8842-9574
//   kbref_gated_delta_net  ggml_gated_delta_net as in src/graph.cpp:169; CPU op ops.cpp:11123-11316
//   kbref_quantize_q8_0    ggml_quantize_chunk(Q8_0) -> quantize_row_q8_0_ref (ggml-quants.c:276-299)
//   kbref_set_rows         ggml_set_rows as in src/graph.cpp:111-112; CPU op ops.cpp:5446-5530
//   kbref_cpy              ggml_cpy f32<->f16 (snapshot write graph.cpp:179-184, rollback state.cpp:162-183)
//   kbref_attn_prologue    the ops between the projections and the attention in Builder::attention
//                          (src/graph.cpp:94-112): q / gate views, ggml_rms_norm * weight, ggml_rope_multi,
//                          ggml_cont of the gate, ggml_set_rows of K and V into the caches
//   kbref_gdn_input        the DeltaNet input side of Builder::deltanet (src/graph.cpp:136-165): sigmoid,
//                          softplus gates, conv-state concat + snapshot copies, ggml_ssm_conv + silu, l2 norms
//   kbref_gdn_gated_norm   the DeltaNet output norm (src/graph.cpp:186-190): rms_norm * w * silu(z)
//
// use_ref = 1 selects ggml's vec-only reference path (no split-KV, no tiling; ops.cpp:9487-9550),
// which makes results independent of the thread count.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "ggml.h"
#include "ggml-cpu.h"

namespace {

struct Ctx {
    ggml_context* ctx = nullptr;
    explicit Ctx(size_t n_tensors) {
        ggml_init_params ip{ggml_tensor_overhead() * n_tensors + ggml_graph_overhead() + 4096, nullptr, true};
        ctx = ggml_init(ip);
    }
    ~Ctx() { if (ctx) ggml_free(ctx); }
};

int compute(ggml_context* ctx, ggml_tensor* out, int n_threads, int use_ref) {
    ggml_cgraph* gf = ggml_new_graph(ctx);
    ggml_build_forward_expand(gf, out);
    ggml_cplan plan = ggml_graph_plan(gf, n_threads > 0 ? n_threads : 1, nullptr);
    std::vector<uint8_t> work(plan.work_size + 64);
    plan.work_data = plan.work_size ? work.data() : nullptr;
    plan.use_ref = use_ref != 0;
    return ggml_graph_compute(gf, &plan) == GGML_STATUS_SUCCESS ? 0 : 1;
}

ggml_tensor* bind(ggml_context* ctx, ggml_type t, int64_t n0, int64_t n1, int64_t n2, int64_t n3, const void* data) {
    ggml_tensor* x = ggml_new_tensor_4d(ctx, t, n0, n1, n2, n3);
    x->data = const_cast<void*>(data);
    return x;
}

bool init_once() {
    static bool done = [] { ggml_cpu_init(); return true; }();
    return done;
}

}  // namespace

extern "C" {

// q    : f32 [n_q][n_head][D]            (token-major, as klein's q projection output)
// k, v : kv_type rows, row r at k + r*kv_row_bytes, head h at + h*row_size(D)   (klein's cache layout)
// mask : f16 [n_q][n_kv] or NULL          (klein's dense mask; -inf = not visible)
// out  : f32 [n_q][n_head][D]
int kbref_flash_attn_ext(const float* q, int n_q, int n_head, int D, const void* k, const void* v, int kv_type,
                         int64_t n_kv, int n_head_kv, size_t kv_row_bytes, const uint16_t* mask, float scale,
                         float max_bias, float softcap, float* out, int n_threads, int use_ref) {
    init_once();
    Ctx c(16);
    const ggml_type kt = (ggml_type) kv_type;
    ggml_tensor* qt = bind(c.ctx, GGML_TYPE_F32, D, n_head, n_q, 1, q);
    ggml_tensor* qp = ggml_permute(c.ctx, qt, 0, 2, 1, 3);  // [D, n_q, n_head]
    const size_t hs = ggml_row_size(kt, D);
    ggml_tensor* kb = ggml_new_tensor_2d(c.ctx, kt, (int64_t) D * n_head_kv, n_kv);
    ggml_tensor* vb = ggml_new_tensor_2d(c.ctx, kt, (int64_t) D * n_head_kv, n_kv);
    kb->data = const_cast<void*>(k);
    vb->data = const_cast<void*>(v);
    ggml_tensor* kv3 = ggml_view_3d(c.ctx, kb, D, n_head_kv, n_kv, hs, kv_row_bytes, 0);
    ggml_tensor* vv3 = ggml_view_3d(c.ctx, vb, D, n_head_kv, n_kv, hs, kv_row_bytes, 0);
    ggml_tensor* kp = ggml_permute(c.ctx, kv3, 0, 2, 1, 3);  // [D, n_kv, n_head_kv]
    ggml_tensor* vp = ggml_permute(c.ctx, vv3, 0, 2, 1, 3);
    ggml_tensor* mt = nullptr;
    if (mask) mt = bind(c.ctx, GGML_TYPE_F16, n_kv, n_q, 1, 1, mask);
    ggml_tensor* o = ggml_flash_attn_ext(c.ctx, qp, kp, vp, mt, scale, max_bias, softcap);
    ggml_prec_set_acc(o, GGML_PREC_F32);
    o->data = out;  // result [D, n_head, n_q] f32 contiguous == out[n_q][n_head][D]
    return compute(c.ctx, o, n_threads, use_ref);
}

// q, k : f32 [n_seqs][T][H_k][S]; v : f32 [n_seqs][T][H_v][S]; g : f32 [n_seqs][T][H_v][kda ? S : 1];
// beta : f32 [n_seqs][T][H_v]; s0 : f32 [n_seqs][H_v][S][S] (transposed state, row j = column j of S);
// out  : f32, ggml's packed layout: attn [n_seqs][T][H_v][S] then K slots of [n_seqs][H_v][S][S].
int kbref_gated_delta_net(const float* q, const float* k, const float* v, const float* g, const float* beta,
                          const float* s0, int S, int H_k, int H_v, int T, int n_seqs, int kda, int K, float* out,
                          int n_threads) {
    init_once();
    Ctx c(16);
    ggml_tensor* qt = bind(c.ctx, GGML_TYPE_F32, S, H_k, T, n_seqs, q);
    ggml_tensor* kt = bind(c.ctx, GGML_TYPE_F32, S, H_k, T, n_seqs, k);
    ggml_tensor* vt = bind(c.ctx, GGML_TYPE_F32, S, H_v, T, n_seqs, v);
    ggml_tensor* gt = bind(c.ctx, GGML_TYPE_F32, kda ? S : 1, H_v, T, n_seqs, g);
    ggml_tensor* bt = bind(c.ctx, GGML_TYPE_F32, 1, H_v, T, n_seqs, beta);
    ggml_tensor* st = bind(c.ctx, GGML_TYPE_F32, S, S, H_v, n_seqs, s0);
    ggml_tensor* r = ggml_gated_delta_net(c.ctx, qt, kt, vt, gt, bt, st, K);
    r->data = out;
    return compute(c.ctx, r, n_threads, 0);
}

// ggml_quantize_chunk(Q8_0, ...) -> quantize_row_q8_0_ref; n_per_row must be a multiple of 32.
size_t kbref_quantize_q8_0(const float* src, void* dst, int64_t nrows, int64_t n_per_row) {
    init_once();
    return ggml_quantize_chunk(GGML_TYPE_Q8_0, src, dst, 0, nrows, n_per_row, nullptr);
}

void kbref_dequantize(int type, const void* src, float* dst, int64_t n) {
    init_once();
    ggml_get_type_traits((ggml_type) type)->to_float(src, dst, n);
}

// ggml_set_rows(dst_cache [row_elems, n_rows] of dst_type, src f32 [row_elems, n_src], idx i64 [n_src])
int kbref_set_rows(void* dst, int dst_type, int64_t row_elems, int64_t n_rows, const float* src, int64_t n_src,
                   const int64_t* idx, int n_threads) {
    init_once();
    Ctx c(16);
    ggml_tensor* dt = bind(c.ctx, (ggml_type) dst_type, row_elems, n_rows, 1, 1, dst);
    ggml_tensor* st = bind(c.ctx, GGML_TYPE_F32, row_elems, n_src, 1, 1, src);
    ggml_tensor* it = bind(c.ctx, GGML_TYPE_I64, n_src, 1, 1, 1, idx);
    ggml_tensor* r = ggml_set_rows(c.ctx, dt, st, it);
    return compute(c.ctx, r, n_threads, 0);
}

// ggml_cpy of n elements between two contiguous 1-d tensors (f32 <-> f16 / bf16 / f32)
int kbref_cpy(const void* src, int src_type, void* dst, int dst_type, int64_t n) {
    init_once();
    Ctx c(8);
    ggml_tensor* s = bind(c.ctx, (ggml_type) src_type, n, 1, 1, 1, src);
    ggml_tensor* d = bind(c.ctx, (ggml_type) dst_type, n, 1, 1, 1, dst);
    ggml_tensor* r = ggml_cpy(c.ctx, s, d);
    return compute(c.ctx, r, 1, 0);
}

// Builder::attention's prologue for n tokens (graph.cpp:94-112). qfull f32 [n][nh][2 hd] (q then gate per head),
// kcur / vcur f32 [n][nkv][hd], pos i32 [4][n] (section-major), kv_idx i64 [n], q_norm / k_norm f32 [hd];
// outputs q_out f32 [n][nh][hd] (normed, roped), gate_out f32 [n][nh][hd], rows kv_idx of the caches
// (cache_type, [n_cells][nkv * hd]) written.
int kbref_attn_prologue(const float* qfull, const float* kcur, const float* vcur, const int32_t* pos,
                        const int64_t* kv_idx, const float* q_norm, const float* k_norm, int hd, int nh, int nkv, int n,
                        float eps, int n_rot, const int32_t* sections, int mode, float freq_base, int n_ctx_orig,
                        float* q_out, float* gate_out, void* k_cache, void* v_cache, int cache_type, int64_t n_cells,
                        int n_threads) {
    init_once();
    const size_t mem = (size_t) 16 * (2 * (size_t) hd * nh + 2 * (size_t) hd * nkv) * (size_t) n * 4 + ((size_t) 8 << 20);
    ggml_init_params ip{mem, nullptr, false};
    ggml_context* ctx = ggml_init(ip);
    if (!ctx) return 1;
    auto bindx = [&](ggml_type t, int64_t n0, int64_t n1, int64_t n2, const void* data) {
        ggml_tensor* x = ggml_new_tensor_3d(ctx, t, n0, n1, n2);
        x->data = const_cast<void*>(data);
        return x;
    };
    ggml_tensor* qf = bindx(GGML_TYPE_F32, (int64_t) 2 * hd * nh, n, 1, qfull);
    const size_t es = sizeof(float);
    ggml_tensor* q = ggml_view_3d(ctx, qf, hd, nh, n, es * hd * 2, es * hd * 2 * nh, 0);
    ggml_tensor* qn = bindx(GGML_TYPE_F32, hd, 1, 1, q_norm);
    ggml_tensor* kn = bindx(GGML_TYPE_F32, hd, 1, 1, k_norm);
    q = ggml_mul(ctx, ggml_rms_norm(ctx, q, eps), qn);
    ggml_tensor* gate = ggml_view_3d(ctx, qf, hd, nh, n, es * hd * 2, es * hd * 2 * nh, es * hd);
    gate = ggml_cont_2d(ctx, gate, (int64_t) hd * nh, n);
    ggml_tensor* k = bindx(GGML_TYPE_F32, hd, nkv, n, kcur);
    ggml_tensor* v = bindx(GGML_TYPE_F32, hd, nkv, n, vcur);
    k = ggml_mul(ctx, ggml_rms_norm(ctx, k, eps), kn);
    ggml_tensor* pt = bindx(GGML_TYPE_I32, (int64_t) 4 * n, 1, 1, pos);
    int sec[4] = {sections[0], sections[1], sections[2], sections[3]};
    q = ggml_rope_multi(ctx, q, pt, nullptr, n_rot, sec, mode, n_ctx_orig, freq_base, 1.0f, 0.0f, 1.0f, 32.0f, 1.0f);
    k = ggml_rope_multi(ctx, k, pt, nullptr, n_rot, sec, mode, n_ctx_orig, freq_base, 1.0f, 0.0f, 1.0f, 32.0f, 1.0f);
    ggml_tensor* ck = bindx((ggml_type) cache_type, (int64_t) hd * nkv, n_cells, 1, k_cache);
    ggml_tensor* cv = bindx((ggml_type) cache_type, (int64_t) hd * nkv, n_cells, 1, v_cache);
    ggml_tensor* it = bindx(GGML_TYPE_I64, n, 1, 1, kv_idx);
    ggml_cgraph* gf = ggml_new_graph(ctx);
    ggml_build_forward_expand(gf, ggml_set_rows(ctx, ck, ggml_reshape_2d(ctx, k, (int64_t) hd * nkv, n), it));
    ggml_build_forward_expand(gf, ggml_set_rows(ctx, cv, ggml_reshape_2d(ctx, v, (int64_t) hd * nkv, n), it));
    ggml_build_forward_expand(gf, ggml_cpy(ctx, q, bindx(GGML_TYPE_F32, hd, nh, n, q_out)));
    ggml_build_forward_expand(gf, ggml_cpy(ctx, gate, bindx(GGML_TYPE_F32, (int64_t) hd * nh, n, 1, gate_out)));
    ggml_cplan plan = ggml_graph_plan(gf, n_threads > 0 ? n_threads : 1, nullptr);
    std::vector<uint8_t> work(plan.work_size + 64);
    plan.work_data = plan.work_size ? work.data() : nullptr;
    const int rc = ggml_graph_compute(gf, &plan) == GGML_STATUS_SUCCESS ? 0 : 1;
    ggml_free(ctx);
    return rc;
}

// Builder::deltanet's input side for n tokens (graph.cpp:136-165). qkv f32 [n][ch] (ch = 2 S H_k + S H_v),
// conv_state f32 [K][(kc - 1) ch] (read and written), conv_w f32 [ch][kc], beta_raw / alpha f32 [n][H_v],
// dt_bias / a f32 [H_v]; outputs q_out, k_out f32 [n][H_k][S], v_out f32 [n][H_v][S], beta_out, g_out [n][H_v].
int kbref_gdn_input(const float* qkv, float* conv_state, const float* conv_w, const float* beta_raw, const float* alpha,
                    const float* dt_bias, const float* a, int S, int H_k, int H_v, int kc, int K, int n, float eps,
                    float* q_out, float* k_out, float* v_out, float* beta_out, float* g_out, int n_threads) {
    init_once();
    const int64_t ch = 2 * (int64_t) S * H_k + (int64_t) S * H_v;
    const size_t mem = (size_t) 16 * (size_t) (ch * (n + kc) + (int64_t) H_v * n) * 4 + ((size_t) 16 << 20);
    ggml_init_params ip{mem, nullptr, false};
    ggml_context* ctx = ggml_init(ip);
    if (!ctx) return 1;
    auto bindx = [&](ggml_type t, int64_t n0, int64_t n1, int64_t n2, const void* data) {
        ggml_tensor* x = ggml_new_tensor_3d(ctx, t, n0, n1, n2);
        x->data = const_cast<void*>(data);
        return x;
    };
    ggml_cgraph* gf = ggml_new_graph(ctx);
    ggml_tensor* qkv_t = bindx(GGML_TYPE_F32, ch, n, 1, qkv);
    ggml_tensor* beta = ggml_sigmoid(ctx, bindx(GGML_TYPE_F32, H_v, n, 1, beta_raw));
    ggml_tensor* g = ggml_mul(ctx, ggml_softplus(ctx, ggml_add(ctx, bindx(GGML_TYPE_F32, H_v, n, 1, alpha),
                                                                bindx(GGML_TYPE_F32, H_v, 1, 1, dt_bias))),
                              bindx(GGML_TYPE_F32, H_v, 1, 1, a));
    ggml_tensor* cs_all = bindx(GGML_TYPE_F32, (int64_t) (kc - 1) * ch, K, 1, conv_state);
    ggml_tensor* cs = ggml_view_1d(ctx, cs_all, cs_all->ne[0], 0);
    cs = ggml_reshape_3d(ctx, cs, kc - 1, ch, 1);
    ggml_tensor* xt = ggml_transpose(ctx, ggml_reshape_3d(ctx, qkv_t, ch, n, 1));
    ggml_tensor* conv_in = ggml_concat(ctx, cs, xt, 0);  // [kc - 1 + n, ch, 1]
    for (int t = 1; t <= K; ++t) {
        const int64_t s_idx = std::max<int64_t>(0, conv_in->ne[0] - (kc - 1) - K + t);
        const int slot = K - t;
        if (slot >= n && slot > 0) continue;
        ggml_tensor* src = ggml_view_3d(ctx, conv_in, kc - 1, ch, 1, conv_in->nb[1], conv_in->nb[2],
                                        ggml_row_size(conv_in->type, s_idx));
        ggml_tensor* dst = ggml_view_1d(ctx, cs_all, cs_all->ne[0], (size_t) slot * cs_all->nb[1]);
        ggml_build_forward_expand(gf, ggml_cpy(ctx, src, dst));
    }
    ggml_tensor* conv = ggml_silu(ctx, ggml_ssm_conv(ctx, conv_in, bindx(GGML_TYPE_F32, kc, ch, 1, conv_w)));
    const int64_t nb1 = ggml_row_size(conv->type, ch);
    ggml_tensor* q = ggml_view_4d(ctx, conv, S, H_k, n, 1, ggml_row_size(conv->type, S), nb1, nb1 * n, 0);
    ggml_tensor* k = ggml_view_4d(ctx, conv, S, H_k, n, 1, ggml_row_size(conv->type, S), nb1, nb1 * n,
                                  ggml_row_size(conv->type, (int64_t) S * H_k));
    ggml_tensor* v = ggml_view_4d(ctx, conv, S, H_v, n, 1, ggml_row_size(conv->type, S), nb1, nb1 * n,
                                  ggml_row_size(conv->type, 2 * (int64_t) S * H_k));
    auto l2 = [&](ggml_tensor* x) {
        const float nn = (float) x->ne[0];
        return ggml_scale(ctx, ggml_rms_norm(ctx, x, eps / nn), 1.0f / std::sqrt(nn));
    };
    q = l2(q);
    k = l2(k);
    ggml_build_forward_expand(gf, ggml_cpy(ctx, q, bindx(GGML_TYPE_F32, S, H_k, n, q_out)));
    ggml_build_forward_expand(gf, ggml_cpy(ctx, k, bindx(GGML_TYPE_F32, S, H_k, n, k_out)));
    ggml_build_forward_expand(gf, ggml_cpy(ctx, v, bindx(GGML_TYPE_F32, S, H_v, n, v_out)));
    ggml_build_forward_expand(gf, ggml_cpy(ctx, beta, bindx(GGML_TYPE_F32, H_v, n, 1, beta_out)));
    ggml_build_forward_expand(gf, ggml_cpy(ctx, g, bindx(GGML_TYPE_F32, H_v, n, 1, g_out)));
    ggml_cplan plan = ggml_graph_plan(gf, n_threads > 0 ? n_threads : 1, nullptr);
    std::vector<uint8_t> work(plan.work_size + 64);
    plan.work_data = plan.work_size ? work.data() : nullptr;
    const int rc = ggml_graph_compute(gf, &plan) == GGML_STATUS_SUCCESS ? 0 : 1;
    ggml_free(ctx);
    return rc;
}

// Builder::deltanet's output norm (graph.cpp:186-190): dst = rms_norm(x, eps) * w * silu(z); x, z, dst f32
// [n][H][S], w f32 [S].
int kbref_gdn_gated_norm(const float* x, const float* z, const float* w, int S, int H, int n, float eps, float* dst,
                         int n_threads) {
    init_once();
    const size_t mem = (size_t) 8 * (size_t) S * H * n * 4 + ((size_t) 4 << 20);
    ggml_init_params ip{mem, nullptr, false};
    ggml_context* ctx = ggml_init(ip);
    if (!ctx) return 1;
    ggml_tensor* xt = ggml_new_tensor_3d(ctx, GGML_TYPE_F32, S, H, n);
    xt->data = const_cast<float*>(x);
    ggml_tensor* zt = ggml_new_tensor_3d(ctx, GGML_TYPE_F32, S, H, n);
    zt->data = const_cast<float*>(z);
    ggml_tensor* wt = ggml_new_tensor_1d(ctx, GGML_TYPE_F32, S);
    wt->data = const_cast<float*>(w);
    ggml_tensor* dt = ggml_new_tensor_3d(ctx, GGML_TYPE_F32, S, H, n);
    dt->data = dst;
    ggml_tensor* o = ggml_mul(ctx, ggml_mul(ctx, ggml_rms_norm(ctx, xt, eps), wt), ggml_silu(ctx, zt));
    ggml_cgraph* gf = ggml_new_graph(ctx);
    ggml_build_forward_expand(gf, ggml_cpy(ctx, o, dt));
    ggml_cplan plan = ggml_graph_plan(gf, n_threads > 0 ? n_threads : 1, nullptr);
    std::vector<uint8_t> work(plan.work_size + 64);
    plan.work_data = plan.work_size ? work.data() : nullptr;
    const int rc = ggml_graph_compute(gf, &plan) == GGML_STATUS_SUCCESS ? 0 : 1;
    ggml_free(ctx);
    return rc;
}

}  // extern "C"
