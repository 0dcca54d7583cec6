// ggml-cuda's attention and DeltaNet entry points implemented by klein_b200: a ggml CUDA backend built without its
// own fattn*.cu and gated_delta_net.cu translation units links this file instead, so that
// ggml_cuda_compute_forward's GGML_OP_FLASH_ATTN_EXT and GGML_OP_GATED_DELTA_NET cases (ggml-cuda.cu:2488-2504),
// its supports_op (ggml-cuda.cu:5775-5776), the buffer type's allocation size of an attention node
// (ggml-cuda.cu:925-926) and the DeltaNet snapshot-copy fusion (ggml-cuda.cu:3609-3620) all run on the library's
// C ABI. Nothing in klein's graph, ggml's scheduler or the rest of ggml-cuda changes.
//
// The functions keep the names and signatures ggml-cuda declares for them (fattn.cuh, gated_delta_net.cuh); this
// file is compiled against the ggml tree klein vendors (its include/, src/ and src/ggml-cuda/ directories).
//
// Scratch: like ggml-cuda's own attention (its f16 conversion buffers), the library's scratch lives right after the
// attention node's output in the compute buffer (ggml_cuda_flash_attn_ext_get_alloc_size adds it), so a call
// allocates nothing and can be captured in ggml-cuda's CUDA graphs. The chunked DeltaNet form (prompt lengths)
// draws its records from the backend's pool, as ggml-cuda's own kernels draw their temporaries.
#include "common.cuh"
#include "fattn.cuh"
#include "gated_delta_net.cuh"

#include "klein_b200.h"

#include <cstring>

namespace {

kb_tensor kb_view(const ggml_tensor* t) {
    kb_tensor d;
    d.type = (int32_t) t->type;  // the same numbering as enum ggml_type
    for (int i = 0; i < 4; ++i) {
        d.ne[i] = t->ne[i];
        d.nb[i] = t->nb[i];
    }
    d.data = t->data;
    return d;
}

void kb_check(kb_status st, const char* what) {
    if (st != KB_OK) GGML_ABORT("%s: klein_b200 returned status %d", what, (int) st);  // ggml's abort behaviour
}

kb_fa_params fa_params(const ggml_tensor* dst) {
    kb_fa_params p;
    std::memset(&p, 0, sizeof(p));
    std::memcpy(&p.scale, (const float*) dst->op_params + 0, sizeof(float));
    std::memcpy(&p.max_bias, (const float*) dst->op_params + 1, sizeof(float));
    std::memcpy(&p.logit_softcap, (const float*) dst->op_params + 2, sizeof(float));
    p.prec = dst->op_params[3];
    return p;
}

constexpr size_t SCRATCH_ALIGN = 256;

size_t fa_scratch_bytes(const ggml_tensor* dst) {
    const kb_tensor q = kb_view(dst->src[0]), k = kb_view(dst->src[1]), v = kb_view(dst->src[2]);
    const kb_fa_params p = fa_params(dst);
    return kb_flash_attn_ext_scratch_bytes(&q, &k, &v, &p);
}

void* fa_scratch(const ggml_tensor* dst) {
    const uintptr_t end = (uintptr_t) dst->data + ggml_nbytes(dst);
    return (void*) ((end + SCRATCH_ALIGN - 1) / SCRATCH_ALIGN * SCRATCH_ALIGN);
}

}  // namespace

bool ggml_cuda_flash_attn_ext_supported(int device, const ggml_tensor* dst) {
    (void) device;
    if (dst->src[4] != nullptr) return false;  // attention sinks: not part of klein's graph
    if (dst->src[0]->type != GGML_TYPE_F32 || dst->type != GGML_TYPE_F32) return false;
    const kb_tensor q = kb_view(dst->src[0]), k = kb_view(dst->src[1]), v = kb_view(dst->src[2]);
    kb_tensor m;
    const kb_tensor* mp = nullptr;
    if (dst->src[3]) {
        m = kb_view(dst->src[3]);
        mp = &m;
    }
    const kb_fa_params p = fa_params(dst);
    return kb_flash_attn_ext_supported(&q, &k, &v, mp, &p) != 0;
}

size_t ggml_cuda_flash_attn_ext_get_alloc_size(int device, const ggml_tensor* dst) {
    GGML_ASSERT(dst->op == GGML_OP_FLASH_ATTN_EXT);
    ggml_cuda_set_device(device);  // the split plan follows the device's SM count
    const size_t need = fa_scratch_bytes(dst);
    return need ? ggml_nbytes(dst) + SCRATCH_ALIGN + need : ggml_nbytes(dst);
}

void ggml_cuda_flash_attn_ext(ggml_backend_cuda_context& ctx, ggml_tensor* dst) {
    ggml_cuda_set_device(ctx.device);
    const kb_tensor q = kb_view(dst->src[0]), k = kb_view(dst->src[1]), v = kb_view(dst->src[2]);
    const kb_tensor out = kb_view(dst);
    kb_tensor m;
    const kb_tensor* mp = nullptr;
    if (dst->src[3]) {
        m = kb_view(dst->src[3]);
        mp = &m;
    }
    const kb_fa_params p = fa_params(dst);
    const size_t need = fa_scratch_bytes(dst);
    kb_check(kb_flash_attn_ext(&q, &k, &v, mp, &p, &out, need ? fa_scratch(dst) : nullptr, need, ctx.stream()),
             "flash_attn_ext");
}

namespace {

void gdn_call(ggml_backend_cuda_context& ctx, ggml_tensor* dst, const ggml_cuda_gated_delta_net_fused_cache* cache) {
    ggml_cuda_set_device(ctx.device);
    const kb_tensor q = kb_view(dst->src[0]), k = kb_view(dst->src[1]), v = kb_view(dst->src[2]);
    const kb_tensor g = kb_view(dst->src[3]), beta = kb_view(dst->src[4]), s0 = kb_view(dst->src[5]);
    const int32_t K = ggml_get_op_params_i32(dst, 0);
    const size_t need = kb_gated_delta_net_scratch_bytes(&v, &g, K);
    ggml_cuda_pool_alloc<uint8_t> scratch(ctx.pool());
    if (need) scratch.alloc(need);
    if (!cache) {
        const kb_tensor out = kb_view(dst);
        kb_check(kb_gated_delta_net(&q, &k, &v, &g, &beta, &s0, K, &out, need ? scratch.get() : nullptr, need, ctx.stream()),
                 "gated_delta_net");
        return;
    }
    // the snapshot-copy fusion: slot s of the state goes to cache->data + s * slot_stride (f32), the attention rows
    // stay at the start of dst. The library's cache form updates its state tensor in place with slot 0, so the slot-0
    // destination starts as a copy of s0 (it usually is s0 itself, klein's state tensor).
    const int64_t S = v.ne[0], H = v.ne[1], T = v.ne[2], n_seqs = v.ne[3];
    const int64_t D = S * S * H * n_seqs;
    if (cache->data != s0.data)
        CUDA_CHECK(cudaMemcpyAsync(cache->data, s0.data, (size_t) D * sizeof(float), cudaMemcpyDeviceToDevice, ctx.stream()));
    kb_tensor state = s0;
    state.data = cache->data;
    const int64_t n_written = T < K ? T : K;
    kb_tensor snap;
    const kb_tensor* sp = nullptr;
    if (n_written > 1) {
        std::memset(&snap, 0, sizeof(snap));
        snap.type = KB_TYPE_F32;
        snap.ne[0] = D, snap.ne[1] = K - 1, snap.ne[2] = 1, snap.ne[3] = 1;
        snap.nb[0] = sizeof(float), snap.nb[1] = (size_t) cache->slot_stride * sizeof(float);
        snap.nb[2] = snap.nb[1] * (size_t) (K - 1), snap.nb[3] = snap.nb[2];
        snap.data = cache->data + cache->slot_stride;
        sp = &snap;
    }
    kb_tensor attn;
    std::memset(&attn, 0, sizeof(attn));
    attn.type = KB_TYPE_F32;
    attn.ne[0] = S, attn.ne[1] = H, attn.ne[2] = T, attn.ne[3] = n_seqs;
    attn.nb[0] = sizeof(float), attn.nb[1] = (size_t) S * sizeof(float), attn.nb[2] = attn.nb[1] * H,
    attn.nb[3] = attn.nb[2] * T;
    attn.data = dst->data;
    kb_check(kb_gated_delta_net_cache(&q, &k, &v, &g, &beta, &state, sp, K, &attn, need ? scratch.get() : nullptr, need,
                                      ctx.stream()),
             "gated_delta_net (snapshot fusion)");
}

}  // namespace

void ggml_cuda_op_gated_delta_net(ggml_backend_cuda_context& ctx, ggml_tensor* dst) { gdn_call(ctx, dst, nullptr); }

void ggml_cuda_op_gated_delta_net_fused_cache(ggml_backend_cuda_context& ctx, ggml_tensor* dst,
                                              ggml_cuda_gated_delta_net_fused_cache cache) {
    gdn_call(ctx, dst, &cache);
}
