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
//   1. the CTA's state columns are loaded first (the longest loads), then the input side, spread over all four
//      warps (so over the SM's four schedulers): thread t the conv + SiLU of q channel t and k channel t of key
//      head h % H_k, 16 threads the CTA's v channels, T threads beta = sigmoid(beta_raw) and exp(g),
//      g = softplus(alpha + dt_bias) * a; then the 2 T L2 norms of the q / k rows, one row per warp at a time (lane l:
//      channels 4 l .. 4 l + 3); all in shared memory.
//      Conv-state snapshots (slot s <- the 3 inputs before token T - s, clamped at the stored state, for s < K,
//      skipping s >= T other than 0): a CTA writes its own v channels; the q / k channels of a key head are read by
//      the 24 CTAs of its value heads, so the last of them to have read (a counter per key head in `sync`, zero
//      before the call and left at zero) writes them.
//   2. the recurrence (gdn_rec.cuh), warp w on columns 16 r + 4 w .. + 3 with 8 lanes per column: slot 0 back into
//      the f32 state in place, slots 1.. into the snapshot rows (f32 / f16 / bf16).
//   3. the gated norm: each CTA's 4 lane partial sums of squares per token are pushed into every CTA of the cluster
//      (st.async into distributed shared memory, completing on the receiver's mbarrier: no cluster-wide barrier,
//      whose release would wait for the state stores to drain), then the butterfly over the 32 partials and
//      out = o * (1 / sqrt(mean + eps)) * w * silu(z).
#include <cooperative_groups.h>

#include "kb_common.cuh"
#include "kb_internal.h"
#include "gdn_rec.cuh"

namespace kb {

namespace {

namespace cg = cooperative_groups;

constexpr int S = 128, KC = 4, KM1 = KC - 1, CPL = 4, TMAX = 4, CLUSTER = 8, COLS = S / CLUSTER, THREADS = 128;
constexpr int LPC = COLS / CPL;  // lanes of a row's butterfly per CTA

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

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

// conv + SiLU of one channel for tokens 0..T-1 over in[] = [stored window (KM1) | x (T)], ggml's order: the window
// oldest first, one multiply-add per tap
template <int T>
__device__ __forceinline__ void conv_silu(const float (&win)[KM1], const float (&x)[TMAX], const float (&w)[KC],
                                          float (&y)[TMAX]) {
#pragma unroll
    for (int u = 0; u < T; ++u) {
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < KM1; ++j)
            acc += (u - KM1 + j >= 0 ? x[u - KM1 + j < 0 ? 0 : u - KM1 + j] : win[u + j < KM1 ? u + j : 0]) * w[j];
        acc += x[u] * w[KM1];
        y[u] = silu_f(acc);
    }
}

// the conv-state snapshots of channel c: slot s <- in[start .. start + KM1), start = T - s clamped at 0
template <int T>
__device__ __forceinline__ void write_conv_slots(const GdnStepParams& p, int64_t c, const float (&win)[KM1],
                                                 const float (&x)[TMAX]) {
    for (int s = 0; s < p.K; ++s) {
        if (s >= T && s > 0) continue;
        const int start = max(0, T - s);
        float* dst = p.conv_state + (int64_t) s * p.conv_ld + c * KM1;
#pragma unroll
        for (int j = 0; j < KM1; ++j) {
            const int ii = start + j;
            float v = 0.0f;
#pragma unroll
            for (int jj = 0; jj < KM1; ++jj)
                if (ii == jj) v = win[jj];
#pragma unroll
            for (int u = 0; u < T; ++u)
                if (ii == KM1 + u) v = x[u];
            dst[j] = v;
        }
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

    // this lane's state column and first row (the token step's layout, gdn_rec.cuh)
    const int col = j0 + (lane >> 3), r8 = lane & 7;
    float4 M[4];
    const float* s0 = p.state + (int64_t) h * S * S + (int64_t) col * S;
#pragma unroll
    for (int d = 0; d < 4; ++d) M[d] = *reinterpret_cast<const float4*>(s0 + gdn_row(r8, d));
    // the gated norm's operands, needed last: loaded now so their latency overlaps everything else
    float zv[CPL], wv[CPL];
    const bool norm_lane = warp < T && lane < LPC;
    if (norm_lane) {
        ld4(p.norm_w + j_base + CPL * lane, wv);
        ld4(p.z + (int64_t) warp * p.H_v * S + (int64_t) h * S + j_base + CPL * lane, zv);
    }

    // ------------------------------------------------------------------------------------ 1. input side
    // conv + SiLU: thread t takes q channel t and k channel t of key head hk, warp 2's lanes 0-15 also the CTA's 16 v
    // channels, warp 3's lanes < T beta and exp(g) of token `lane`; the raw q / k rows go to shared memory
    const int64_t cq = (int64_t) hk * S + tid, ck = (int64_t) (p.H_k + hk) * S + tid;
    float winq[KM1], wink[KM1], xq[TMAX], xk[TMAX];
    {
        float wq[KC], wk[KC], yq[TMAX], yk[TMAX];
        ld4(p.conv_w + cq * KC, wq);
        ld4(p.conv_w + ck * KC, wk);
#pragma unroll
        for (int j = 0; j < KM1; ++j) winq[j] = p.conv_state[cq * KM1 + j], wink[j] = p.conv_state[ck * KM1 + j];
#pragma unroll
        for (int u = 0; u < TMAX; ++u) {
            xq[u] = u < T ? p.qkv[(int64_t) u * p.qkv_ld + cq] : 0.0f;
            xk[u] = u < T ? p.qkv[(int64_t) u * p.qkv_ld + ck] : 0.0f;
        }
        conv_silu<T>(winq, xq, wq, yq);
        conv_silu<T>(wink, xk, wk, yk);
#pragma unroll
        for (int u = 0; u < T; ++u) qs[u][tid] = yq[u], ks[u][tid] = yk[u];
    }
    if (warp == 2 && lane < COLS) {
        const int64_t cv = 2 * (int64_t) p.H_k * S + (int64_t) h * S + j_base + lane;
        float w[KC], win[KM1], x[TMAX], y[TMAX];
        ld4(p.conv_w + cv * KC, w);
#pragma unroll
        for (int j = 0; j < KM1; ++j) win[j] = p.conv_state[cv * KM1 + j];
#pragma unroll
        for (int u = 0; u < TMAX; ++u) x[u] = u < T ? p.qkv[(int64_t) u * p.qkv_ld + cv] : 0.0f;
        conv_silu<T>(win, x, w, y);
#pragma unroll
        for (int u = 0; u < T; ++u) vs[u][lane] = y[u];
        write_conv_slots<T>(p, cv, win, x);  // the CTA's own channel, read above by this thread only
    } else if (warp == 3 && lane < T) {
        const float b = p.beta_raw[(int64_t) lane * p.H_v + h];
        beta_s[lane] = 1.0f / (1.0f + expf(-b));
        const float x = p.alpha[(int64_t) lane * p.H_v + h] + p.dt_bias[h];
        const float sp = x > 20.0f ? x : logf(1.0f + expf(x));
        const float g = __fmul_rn(sp, p.a[h]);  // rounded on its own, as when it is stored and read back
        eg_s[lane] = expf(g);
    }
    __syncthreads();
    // l2 of the q and k rows of every token, one row per warp at a time: rms_norm with eps / S (lane l's 4 consecutive
    // channels summed in double, then the butterfly), then * 1 / sqrt(S)
#pragma unroll
    for (int task = warp; task < 2 * T; task += THREADS / 32) {
        float* row = task < T ? qs[task] : ks[task - T];
        float y[CPL];
        ld4(row + CPL * lane, y);
        double ss = 0.0;
#pragma unroll
        for (int i = 0; i < CPL; ++i) ss += (double) (y[i] * y[i]);
        ss = warp_sum_d(ss);
        const float mean = (float) (ss / S);
        const float scale = 1.0f / sqrtf(mean + p.l2_eps);
#pragma unroll
        for (int i = 0; i < CPL; ++i) y[i] = y[i] * scale * p.inv_sqrt_s;
        st4(row + CPL * lane, y);
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
        const int64_t elem = ((int64_t) h * S + col) * S;
#pragma unroll
        for (int t = 0; t < T; ++t) {
            float4 k[4], q[4], e[4];
#pragma unroll
            for (int d = 0; d < 4; ++d) {
                k[d] = *reinterpret_cast<const float4*>(&ks[t][gdn_row(r8, d)]);
                q[d] = *reinterpret_cast<const float4*>(&qs[t][gdn_row(r8, d)]);
                e[d] = make_float4(eg_s[t], eg_s[t], eg_s[t], eg_s[t]);
            }
            const float o = gdn_token(M, k, q, e, vs[t][col - j_base], beta_s[t]);
            if ((lane & 7) == 0) os[t][col - j_base] = o * scale;
            const int slot = T - 1 - t;
            if (slot < p.K) {
                char* base = slot == 0 ? reinterpret_cast<char*>(p.state) : p.snap + (int64_t) (slot - 1) * p.snap_stride;
                gdn_store_col(base, slot == 0 ? 0 : p.snap_type, elem, r8, M);
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
    if (last) {
        write_conv_slots<T>(p, cq, winq, xq);
        write_conv_slots<T>(p, ck, wink, xk);
    }
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
