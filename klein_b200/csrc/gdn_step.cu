// One launch for a whole DeltaNet layer of the decode / verify step (T <= 4 tokens): klein's Builder::deltanet
// between its GEMMs (graph.cpp:136-190) — the conv input side (gdn_input_kernel), the recurrence with its state slot
// and snapshot rows (gdn_recurrent_kernel in klein's cache form) and the gated RMS norm (gdn_gated_norm_vec_kernel) —
// which otherwise take three launches whose cost at these sizes is mostly launch and load latency.
//
// The results are bit-identical to those three kernels: every value is computed by the same expression, and the two
// reductions (the L2 norms of q / k, the gated norm's sum of squares) keep their order — a lane's sum of its 4
// consecutive channels in double, then the xor butterfly over the 32 lanes of a 128-channel row.
//
// Grid: one cluster of 8 CTAs per value head h (thread block clusters, distributed shared memory); CTA r of the
// cluster owns value columns [16 r, 16 r + 16) of the head's 128 x 128 state (stored transposed, M[j][i]).
//   1. the CTA's state columns are loaded first (the longest loads), then the input side, warp-specialised:
//      warp 0 the q channels and warp 1 the k channels of key head h % H_k (lane l: channels 4 l .. 4 l + 3, conv +
//      SiLU + L2 norm), warp 2 lanes 0-3 the CTA's 16 v channels, warp 3 beta = sigmoid(beta_raw) and
//      exp(g), g = softplus(alpha + dt_bias) * a; all into shared memory.
//      Conv-state snapshots (slot s <- the 3 inputs before token T - s, clamped at the stored state, for s < K,
//      skipping s >= T other than 0): a CTA writes its own v channels; the q / k channels of a key head are read by
//      the 24 CTAs of its value heads, so the last of them to have read (a counter per key head in `sync`, zero
//      before the call and left at zero) writes them.
//   2. the recurrence, warp w on columns 16 r + 4 w .. + 3 (lane l: rows 4 l .. 4 l + 3 as float4): slot 0 back into
//      the f32 state in place, slots 1.. into the snapshot rows (f32 / f16 / bf16).
//   3. the gated norm: each CTA's 4 lane partial sums of squares per token are pushed into every CTA of the cluster
//      (st.async into distributed shared memory, completing on the receiver's mbarrier: no cluster-wide barrier,
//      whose release would wait for the state stores to drain), then the butterfly over the 32 partials and
//      out = o * (1 / sqrt(mean + eps)) * w * silu(z).
#include <cooperative_groups.h>

#include "kb_common.cuh"
#include "kb_internal.h"

namespace kb {

namespace {

namespace cg = cooperative_groups;

constexpr int S = 128, KC = 4, KM1 = KC - 1, CPL = 4, TMAX = 4, CLUSTER = 8, COLS = S / CLUSTER, THREADS = 128;
constexpr int LPC = COLS / CPL;  // lanes of a row's butterfly per CTA

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int off = 16; off; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
    return x;
}

__device__ __forceinline__ double warp_sum_d(double x) {
#pragma unroll
    for (int off = 16; off; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
    return x;
}

__device__ __forceinline__ int atom_add_acq_rel_gpu(int* addr, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
    return old;
}

// cluster barrier halves: arrive without release semantics (nothing but the barrier initialisation, made visible by its
// own fence, has to be ordered), wait with acquire
__device__ __forceinline__ void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait;" ::: "memory"); }

// address of the same shared variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_rank(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}

// an 8-byte store into another CTA's shared memory that completes on that CTA's mbarrier
__device__ __forceinline__ void st_async_b64(uint32_t remote, double v, uint32_t remote_bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b64 [%0], %1, [%2];" ::"r"(remote),
                 "l"(__double_as_longlong(v)), "r"(remote_bar)
                 : "memory");
}

__device__ __forceinline__ void ld4(const float* src, float* d) {
    const float4 a = *reinterpret_cast<const float4*>(src);
    d[0] = a.x, d[1] = a.y, d[2] = a.z, d[3] = a.w;
}

__device__ __forceinline__ void st4(float* dst, const float* v) {
    *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
}

__device__ __forceinline__ void store4(char* base, int type, int64_t elem, float4 v) {
    if (type == 0) {
        *reinterpret_cast<float4*>(base + elem * 4) = v;
    } else if (type == 1) {
        __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
        *reinterpret_cast<uint2*>(base + elem * 2) = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
    } else {
        __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
        *reinterpret_cast<uint2*>(base + elem * 2) = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
    }
}

// the conv-state snapshots of a lane's 4 channels from cl on: slot s <- in[start .. start + KM1), in = [stored window
// (KM1) | the T inputs], start = T - s clamped at 0
template <int T>
__device__ __forceinline__ void write_conv_slots(const GdnStepParams& p, int64_t cl, const float (&win)[CPL][KM1],
                                                 const float (&xs)[TMAX][CPL]) {
    for (int s = 0; s < p.K; ++s) {
        if (s >= T && s > 0) continue;
        const int start = max(0, T - s);
        float sv[CPL][KM1];
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
#pragma unroll
            for (int j = 0; j < KM1; ++j) {
                const int ii = start + j;
                float v = 0.0f;
#pragma unroll
                for (int jj = 0; jj < KM1; ++jj)
                    if (ii == jj) v = win[i][jj];
#pragma unroll
                for (int u = 0; u < T; ++u)
                    if (ii == KM1 + u) v = xs[u][i];
                sv[i][j] = v;
            }
        }
        float* dst = p.conv_state + (int64_t) s * p.conv_ld + cl * KM1;
#pragma unroll
        for (int q = 0; q < KM1; ++q) st4(dst + q * CPL, &sv[0][0] + q * CPL);
    }
}

template <int T>
__global__ void __cluster_dims__(CLUSTER, 1, 1) __launch_bounds__(THREADS) gdn_step_kernel(const GdnStepParams p) {
    __shared__ __align__(16) float qs[TMAX][S];
    __shared__ __align__(16) float ks[TMAX][S];
    __shared__ __align__(16) float vs[TMAX][COLS];
    __shared__ __align__(16) float os[TMAX][COLS];
    __shared__ float beta_s[TMAX], eg_s[TMAX];
    __shared__ double allp[TMAX][32];  // per token, the row's 32 lane partials, pushed by the cluster's 8 CTAs
    __shared__ __align__(8) uint64_t full;
    __shared__ int last;
    cg::cluster_group cluster = cg::this_cluster();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cr = (int) cluster.block_rank();
    const int h = blockIdx.y, hk = h % p.H_k;
    const int j_base = COLS * cr;
    const int j0 = j_base + 4 * warp;  // this warp's 4 state columns
    constexpr uint32_t PART_BYTES = CLUSTER * T * LPC * sizeof(double);
    if (tid == 0) {
        mbar_init(&full, 1);
        mbar_arrive_expect_tx(&full, PART_BYTES);
        fence_barrier_init();
    }
    cluster_arrive_relaxed();  // paired with the wait before the first push: every CTA's barrier is initialised

    float4 M[4];
    const float* s0 = p.state + (int64_t) h * S * S;
#pragma unroll
    for (int c = 0; c < 4; ++c) M[c] = *reinterpret_cast<const float4*>(s0 + (int64_t) (j0 + c) * S + 4 * lane);
    // the gated norm's operands, needed last: loaded now so their latency overlaps everything else
    float zv[CPL], wv[CPL];
    const bool norm_lane = warp < T && lane < LPC;
    if (norm_lane) {
        ld4(p.norm_w + j_base + CPL * lane, wv);
        ld4(p.z + (int64_t) warp * p.H_v * S + (int64_t) h * S + j_base + CPL * lane, zv);
    }

    // ------------------------------------------------------------------------------------ 1. input side
    // the lane's first channel: q / k of key head hk (warps 0 / 1), 4 of the CTA's v channels (warp 2, lanes 0-3)
    int64_t cl = -1;
    if (warp < 2) cl = (int64_t) (warp * p.H_k + hk) * S + CPL * lane;
    else if (warp == 2 && lane < LPC) cl = 2 * (int64_t) p.H_k * S + (int64_t) h * S + j_base + CPL * lane;
    float win[CPL][KM1], xs[TMAX][CPL];
    if (cl >= 0) {
        float w[CPL][KC], y[TMAX][CPL];
#pragma unroll
        for (int q = 0; q < KC; ++q) ld4(p.conv_w + cl * KC + q * CPL, &w[0][0] + q * CPL);
#pragma unroll
        for (int q = 0; q < KM1; ++q) ld4(p.conv_state + cl * KM1 + q * CPL, &win[0][0] + q * CPL);
#pragma unroll
        for (int u = 0; u < TMAX; ++u) {
            if (u < T) {
                ld4(p.qkv + (int64_t) u * p.qkv_ld + cl, xs[u]);
            } else {
#pragma unroll
                for (int i = 0; i < CPL; ++i) xs[u][i] = 0.0f;
            }
        }
        // conv + SiLU, ggml's order: the window oldest first, one multiply-add per tap
#pragma unroll
        for (int u = 0; u < T; ++u) {
#pragma unroll
            for (int i = 0; i < CPL; ++i) {
                float acc = 0.0f;
#pragma unroll
                for (int j = 0; j < KM1; ++j)
                    acc += (u - KM1 + j >= 0 ? xs[u - KM1 + j < 0 ? 0 : u - KM1 + j][i] : win[i][u + j < KM1 ? u + j : 0]) *
                           w[i][j];
                acc += xs[u][i] * w[i][KM1];
                y[u][i] = silu_f(acc);
            }
        }
        if (warp < 2) {
            // l2: rms_norm with eps / S (sum of squares in double), then * 1 / sqrt(S)
            float(*dst)[S] = warp == 0 ? qs : ks;
#pragma unroll
            for (int u = 0; u < T; ++u) {
                double ss = 0.0;
#pragma unroll
                for (int i = 0; i < CPL; ++i) ss += (double) (y[u][i] * y[u][i]);
                ss = warp_sum_d(ss);
                const float mean = (float) (ss / S);
                const float scale = 1.0f / sqrtf(mean + p.l2_eps);
#pragma unroll
                for (int i = 0; i < CPL; ++i) y[u][i] = y[u][i] * scale * p.inv_sqrt_s;
                st4(&dst[u][CPL * lane], y[u]);
            }
        } else {
#pragma unroll
            for (int u = 0; u < T; ++u) st4(&vs[u][CPL * lane], y[u]);
            write_conv_slots<T>(p, cl, win, xs);  // the CTA's own channels, read above by this thread only
        }
    } else if (warp == 3 && lane < T) {
        const float b = p.beta_raw[(int64_t) lane * p.H_v + h];
        beta_s[lane] = 1.0f / (1.0f + expf(-b));
        const float x = p.alpha[(int64_t) lane * p.H_v + h] + p.dt_bias[h];
        const float sp = x > 20.0f ? x : logf(1.0f + expf(x));
        const float g = __fmul_rn(sp, p.a[h]);  // rounded on its own, as when it is stored and read back
        eg_s[lane] = expf(g);
    }
    __syncthreads();
    // every read of the key head's stored window by this CTA is behind the barrier above: count this CTA among its
    // readers (release), and learn (acquire) whether it is the last one, which then writes the window's slots once
    // everything else is done. The atomic's result is consumed only after the recurrence.
    int prev = 0;
    if (tid == THREADS - 32) prev = atom_add_acq_rel_gpu(p.sync + hk, 1);

    // ------------------------------------------------------------------------------------ 2. recurrence
    {
        const float scale = rsqrtf((float) S);
        const int64_t e0 = (int64_t) h * S * S;
#pragma unroll
        for (int t = 0; t < T; ++t) {
            const float4 k4 = *reinterpret_cast<const float4*>(&ks[t][4 * lane]);
            const float4 q4 = *reinterpret_cast<const float4*>(&qs[t][4 * lane]);
            const float beta = beta_s[t];
            const float eg = eg_s[t];
            float vj[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) vj[c] = vs[t][4 * warp + c];
            float sk[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                M[c].x *= eg;
                M[c].y *= eg;
                M[c].z *= eg;
                M[c].w *= eg;
                sk[c] = M[c].x * k4.x + M[c].y * k4.y + M[c].z * k4.z + M[c].w * k4.w;
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) sk[c] = warp_sum(sk[c]);
            float so[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float delta = (vj[c] - sk[c]) * beta;
                M[c].x += delta * k4.x;
                M[c].y += delta * k4.y;
                M[c].z += delta * k4.z;
                M[c].w += delta * k4.w;
                so[c] = M[c].x * q4.x + M[c].y * q4.y + M[c].z * q4.z + M[c].w * q4.w;
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) so[c] = warp_sum(so[c]);
            if (lane < 4) {
                float o = so[0];
#pragma unroll
                for (int c = 1; c < 4; ++c)
                    if (lane == c) o = so[c];
                os[t][4 * warp + lane] = o * scale;
            }
            const int slot = T - 1 - t;
            if (slot < p.K) {
                char* base = slot == 0 ? reinterpret_cast<char*>(p.state) : p.snap + (int64_t) (slot - 1) * p.snap_stride;
                const int type = slot == 0 ? 0 : p.snap_type;
#pragma unroll
                for (int c = 0; c < 4; ++c) store4(base, type, e0 + (int64_t) (j0 + c) * S + 4 * lane, M[c]);
            }
        }
    }
    if (tid == THREADS - 32) {
        last = prev == (p.H_v / p.H_k) * CLUSTER - 1;
        if (last) p.sync[hk] = 0;  // all readers have counted: zero again for the next call
    }
    __syncthreads();

    // ------------------------------------------------------------------------------------ 3. gated norm
    cluster_wait();
    if (tid < T * LPC) {
        const int u = tid / LPC, i = tid % LPC;
        double ss = 0.0;
#pragma unroll
        for (int c = 0; c < CPL; ++c) ss += (double) (os[u][CPL * i + c] * os[u][CPL * i + c]);
        // lane cr * LPC + i of the row's butterfly (it holds channels 4 (cr LPC + i) .. + 3)
#pragma unroll
        for (int r = 0; r < CLUSTER; ++r)
            st_async_b64(map_rank(&allp[u][cr * LPC + i], (uint32_t) r), ss, map_rank(&full, (uint32_t) r));
    }
    if (warp < T) {
        const int u = warp;
        if (!mbar_wait(&full, 0, p.wait_ns)) {
            if (lane == 0) record_error(p.err, DEV_ERR_WAIT_PEER);
        } else {
            const double ss = warp_sum_d(allp[u][lane]);
            const float mean = (float) (ss / S);
            const float scale = 1.0f / sqrtf(mean + p.eps);
            if (norm_lane) {
                float o[CPL];
#pragma unroll
                for (int i = 0; i < CPL; ++i) o[i] = os[u][CPL * lane + i] * scale * wv[i] * silu_f(zv[i]);
                st4(p.out + (int64_t) u * p.H_v * S + (int64_t) h * S + j_base + CPL * lane, o);
            }
        }
    }
    if (last && warp < 2) write_conv_slots<T>(p, cl, win, xs);
    // no CTA of the cluster reads this one's shared memory, and every push into it has landed before its norm warps
    // finish: the CTA leaves without a cluster barrier
}

}  // namespace

cudaError_t launch_gdn_step(const GdnStepParams& p, cudaStream_t stream) {
    const dim3 grid(CLUSTER, p.H_v);
    switch (p.T) {
        case 1: gdn_step_kernel<1><<<grid, THREADS, 0, stream>>>(p); break;
        case 2: gdn_step_kernel<2><<<grid, THREADS, 0, stream>>>(p); break;
        case 3: gdn_step_kernel<3><<<grid, THREADS, 0, stream>>>(p); break;
        case 4: gdn_step_kernel<4><<<grid, THREADS, 0, stream>>>(p); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace kb
