// Test harness for the ggml-cuda integration (kb_ggml_cuda.cu): builds klein's own graph nodes through ggml's graph
// API and runs them on a backend, the CUDA backend (whose attention and DeltaNet cases now run on klein_b200) or
// ggml's CPU backend (the reference implementation), so the tests can compare the two.
//   kbggml_attention  Builder::attention's attention node (src/graph.cpp:113-121): Q [hd, nh, n] permuted, K / V
//                     views of a [kv_row, n_ctx] cache, the dense f16 mask, ggml_flash_attn_ext + ggml_prec_set_acc
//   kbggml_deltanet   Builder::deltanet's recurrence and its two copies (graph.cpp:166-184): ggml_gated_delta_net on
//                     the f32 state, slot 0 copied back into the state, slots 1.. into the snapshot rows
//   kbggml_rollback   State::rollback_recurrent's copies for one layer (src/state.cpp:162-183)
// Each entry point runs the graph `reps` times (the CUDA backend captures repeated graphs into CUDA graphs) and
// returns 0 on success.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "ggml-alloc.h"
#include "ggml-backend.h"
#include "ggml-cpu.h"
#include "ggml-cuda.h"
#include "ggml.h"

namespace {

struct Run {
    ggml_backend_t backend = nullptr;
    ggml_context* leaf = nullptr;   // inputs and state tensors (allocated in one backend buffer)
    ggml_context* ops = nullptr;    // the graph's nodes (allocated by the graph allocator)
    ggml_backend_buffer_t buf = nullptr;
    ggml_gallocr_t galloc = nullptr;
    ggml_cgraph* gf = nullptr;

    explicit Run(int use_cuda, int n_threads) {
        backend = use_cuda ? ggml_backend_cuda_init(0) : ggml_backend_cpu_init();
        if (!use_cuda && backend) ggml_backend_cpu_set_n_threads(backend, n_threads);
        ggml_init_params ip{ggml_tensor_overhead() * 64, nullptr, true};
        leaf = ggml_init(ip);
        ggml_init_params op{ggml_tensor_overhead() * 256 + ggml_graph_overhead(), nullptr, true};
        ops = ggml_init(op);
        gf = ggml_new_graph(ops);
    }
    bool alloc_leaves() {
        buf = ggml_backend_alloc_ctx_tensors(leaf, backend);
        return buf != nullptr;
    }
    bool compute(int reps) {
        galloc = ggml_gallocr_new(ggml_backend_get_default_buffer_type(backend));
        if (!ggml_gallocr_alloc_graph(galloc, gf)) return false;
        return true;
    }
    bool run(int reps) {
        for (int i = 0; i < reps; ++i)
            if (ggml_backend_graph_compute(backend, gf) != GGML_STATUS_SUCCESS) return false;
        ggml_backend_synchronize(backend);
        return true;
    }
    ~Run() {
        if (galloc) ggml_gallocr_free(galloc);
        if (buf) ggml_backend_buffer_free(buf);
        if (ops) ggml_free(ops);
        if (leaf) ggml_free(leaf);
        if (backend) ggml_backend_free(backend);
    }
};

}  // namespace

extern "C" {

int kbggml_attention(int use_cuda, int kv_type, int n_q, int n_ctx, int n_kv, int hd, int nh, int nkv, const float* q,
                     const void* k_cache, const void* v_cache, const uint16_t* mask, float* out, int reps, int n_threads) {
    Run r(use_cuda, n_threads);
    if (!r.backend) return 1;
    const ggml_type t = (ggml_type) kv_type;
    const int64_t kv_row = (int64_t) hd * nkv;
    ggml_tensor* tq = ggml_new_tensor_3d(r.leaf, GGML_TYPE_F32, hd, nh, n_q);
    ggml_tensor* ck = ggml_new_tensor_2d(r.leaf, t, kv_row, n_ctx);
    ggml_tensor* cv = ggml_new_tensor_2d(r.leaf, t, kv_row, n_ctx);
    ggml_tensor* tm = ggml_new_tensor_2d(r.leaf, GGML_TYPE_F16, n_kv, n_q);
    if (!r.alloc_leaves()) return 2;
    ggml_backend_tensor_set(tq, q, 0, ggml_nbytes(tq));
    ggml_backend_tensor_set(ck, k_cache, 0, ggml_nbytes(ck));
    ggml_backend_tensor_set(cv, v_cache, 0, ggml_nbytes(cv));
    ggml_backend_tensor_set(tm, mask, 0, ggml_nbytes(tm));
    // graph.cpp:113-121
    ggml_context* c = r.ops;
    ggml_tensor* k = ggml_view_3d(c, ck, hd, nkv, n_kv, ggml_row_size(t, hd), ggml_row_size(t, kv_row), 0);
    ggml_tensor* v = ggml_view_3d(c, cv, hd, nkv, n_kv, ggml_row_size(t, hd), ggml_row_size(t, kv_row), 0);
    k = ggml_permute(c, k, 0, 2, 1, 3);
    v = ggml_permute(c, v, 0, 2, 1, 3);
    ggml_tensor* qp = ggml_permute(c, tq, 0, 2, 1, 3);
    ggml_tensor* o = ggml_flash_attn_ext(c, qp, k, v, tm, 1.0f / std::sqrt((float) hd), 0.0f, 0.0f);
    ggml_prec_set_acc(o, GGML_PREC_F32);
    ggml_set_output(o);
    ggml_build_forward_expand(r.gf, o);
    if (!r.compute(reps)) return 3;
    if (!r.run(reps)) return 4;
    ggml_backend_tensor_get(o, out, 0, ggml_nbytes(o));
    return 0;
}

int kbggml_deltanet(int use_cuda, int S, int H_k, int H_v, int T, int K, int snap_type, const float* q, const float* k,
                    const float* v, const float* g, const float* beta, float* state, void* snap, float* attn, int reps,
                    int n_threads) {
    Run r(use_cuda, n_threads);
    if (!r.backend) return 1;
    const int64_t D = (int64_t) S * S * H_v;
    ggml_tensor* tq = ggml_new_tensor_4d(r.leaf, GGML_TYPE_F32, S, H_k, T, 1);
    ggml_tensor* tk = ggml_new_tensor_4d(r.leaf, GGML_TYPE_F32, S, H_k, T, 1);
    ggml_tensor* tv = ggml_new_tensor_4d(r.leaf, GGML_TYPE_F32, S, H_v, T, 1);
    ggml_tensor* tg = ggml_new_tensor_4d(r.leaf, GGML_TYPE_F32, 1, H_v, T, 1);
    ggml_tensor* tb = ggml_new_tensor_4d(r.leaf, GGML_TYPE_F32, 1, H_v, T, 1);
    ggml_tensor* ss = ggml_new_tensor_2d(r.leaf, GGML_TYPE_F32, D, 1);
    ggml_tensor* sn = K > 1 ? ggml_new_tensor_2d(r.leaf, (ggml_type) snap_type, D, K - 1) : nullptr;
    if (!r.alloc_leaves()) return 2;
    ggml_backend_tensor_set(tq, q, 0, ggml_nbytes(tq));
    ggml_backend_tensor_set(tk, k, 0, ggml_nbytes(tk));
    ggml_backend_tensor_set(tv, v, 0, ggml_nbytes(tv));
    ggml_backend_tensor_set(tg, g, 0, ggml_nbytes(tg));
    ggml_backend_tensor_set(tb, beta, 0, ggml_nbytes(tb));
    ggml_backend_tensor_set(ss, state, 0, ggml_nbytes(ss));
    if (sn) ggml_backend_tensor_set(sn, snap, 0, ggml_nbytes(sn));
    // graph.cpp:166-184
    ggml_context* c = r.ops;
    ggml_tensor* s0 = ggml_reshape_4d(c, ggml_view_1d(c, ss, D, 0), S, S, H_v, 1);
    ggml_tensor* res = ggml_gated_delta_net(c, tq, tk, tv, tg, tb, s0, K);
    const int64_t attn_elems = (int64_t) S * H_v * T;
    ggml_tensor* out = ggml_view_1d(c, res, attn_elems, 0);
    const int n_written = T < K ? T : K;
    ggml_tensor* cur = ggml_view_1d(c, res, D, ggml_row_size(res->type, attn_elems));
    ggml_build_forward_expand(r.gf, ggml_cpy(c, cur, ggml_view_1d(c, ss, D, 0)));
    if (n_written > 1 && sn) {
        ggml_tensor* src = ggml_view_2d(c, res, D, n_written - 1, ggml_row_size(res->type, D),
                                        ggml_row_size(res->type, attn_elems + D));
        ggml_build_forward_expand(r.gf, ggml_cpy(c, src, ggml_view_2d(c, sn, D, n_written - 1, sn->nb[1], 0)));
    }
    ggml_tensor* oc = ggml_cont(c, out);
    ggml_set_output(oc);
    ggml_build_forward_expand(r.gf, oc);
    if (!r.compute(reps)) return 3;
    if (!r.run(reps)) return 4;
    ggml_backend_tensor_get(oc, attn, 0, ggml_nbytes(oc));
    ggml_backend_tensor_get(ss, state, 0, ggml_nbytes(ss));
    if (sn) ggml_backend_tensor_get(sn, snap, 0, ggml_nbytes(sn));
    return 0;
}

int kbggml_rollback(int use_cuda, int s, int n_snapshots, int64_t conv_row, int64_t ssm_row, int snap_type, float* conv,
                    void* snap, float* ssm, int n_threads) {
    Run r(use_cuda, n_threads);
    if (!r.backend) return 1;
    ggml_tensor* tc = ggml_new_tensor_2d(r.leaf, GGML_TYPE_F32, conv_row, n_snapshots);
    ggml_tensor* ts = ggml_new_tensor_2d(r.leaf, GGML_TYPE_F32, ssm_row, 1);
    ggml_tensor* tn = ggml_new_tensor_2d(r.leaf, (ggml_type) snap_type, ssm_row, n_snapshots - 1);
    if (!r.alloc_leaves()) return 2;
    ggml_backend_tensor_set(tc, conv, 0, ggml_nbytes(tc));
    ggml_backend_tensor_set(ts, ssm, 0, ggml_nbytes(ts));
    ggml_backend_tensor_set(tn, snap, 0, ggml_nbytes(tn));
    // state.cpp:162-183 for one DeltaNet layer
    ggml_context* c = r.ops;
    auto copy = [&](ggml_tensor* from, size_t from_off, ggml_tensor* to, int64_t n) {
        ggml_tensor* src = ggml_view_1d(c, from, n, from_off);
        ggml_tensor* dst = ggml_view_1d(c, to, n, 0);
        ggml_build_forward_expand(r.gf, ggml_cpy(c, src, dst));
    };
    copy(tc, (size_t) s * tc->nb[1], tc, tc->ne[0]);
    copy(tn, (size_t) (s - 1) * tn->nb[1], ts, ts->ne[0]);
    if (!r.compute(1)) return 3;
    if (!r.run(1)) return 4;
    ggml_backend_tensor_get(tc, conv, 0, ggml_nbytes(tc));
    ggml_backend_tensor_get(ts, ssm, 0, ggml_nbytes(ts));
    return 0;
}

}  // extern "C"
