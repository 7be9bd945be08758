// kernels_skyjepa.cu — SkyJEPA learned candidate scorer, fused with MPPI.
//
// Reference path (src/models/skyjepa/control.rs:246-317 -> model.rs:161-223
// -> tcn.rs, prober.rs:84-138, kinematics.rs:377-484 -> control.rs:430-452):
//   normalise actions; action TCN on every rolling window of
//   [history(H-1) ++ candidates]; state TCN + projection -> h0; T GRU steps;
//   prober MLP -> residual accel + angular map; explicit-Euler SO(3)
//   integrator; tracking cost averaged over the horizon.
//
// B200 mapping: one kernel per plan iteration, one 8-CTA thread-block
// cluster per M candidate rows (M = 8 x groups, chosen so that the whole grid
// is resident in one wave).  Each CTA runs 8 "GEMM" warps and 1 "prober" warp.
//  * Prologue (all warps): sampling of the CTA's M/8 own rows; the action TCN
//    of their rolling windows (one warp-local group of lanes per window), the
//    window embeddings broadcast to every CTA through distributed shared
//    memory (DSMEM); the state-history TCN + projection (h0), each CTA
//    computing 1/8 of the output channels of every convolution, k-sliced over
//    its threads and reduced in shared memory, broadcast through DSMEM.
//  * GRU loop (GEMM warps): CTA c owns hidden units [c*H/8, (c+1)*H/8); its
//    slice of W_hh (all three gates, all k) lives in REGISTERS for the whole
//    loop (96 floats a thread at H = 256), so the recurrent GEMM reads only h
//    from shared memory.  Each step the CTA computes its units' new hidden
//    values for all M rows and stores them into every CTA's next-h buffer
//    through DSMEM; a split cluster barrier (arrive.release / wait.acquire)
//    publishes them.
//  * Prober warp: while the GEMM warps compute step t+1, it runs the prober
//    MLP, the SO(3) integrator and the tracking cost of step t for the CTA's
//    own rows, so that work is off the critical path.
//  * Epilogue: the MPPI tuple of the own rows feeds the one-pass reduction
//    (lwm_mppi.cuh).
// No intermediate tensor ([B,S,T,latent], [B,S,T,18]) touches HBM.
//
// Numerics are f32 throughout.  Dot products use fused multiply-add
// explicitly; the file is compiled with -fmad=false so the element-wise math
// (normalisation, gates, integrator, cost) rounds every operation the way
// the reference's f32 kernels do.
#include <cooperative_groups.h>

#include <cstdint>

#include "lwm_device.cuh"
#include "lwm_kernels.hpp"
#include "lwm_mppi.cuh"
#include "lwm_skyjepa_dev.cuh"

namespace cg = cooperative_groups;

namespace lwm {

constexpr int kCluster = 8;
constexpr int kGemmWarps = 8;
constexpr int kGemmThreads = kGemmWarps * 32;
constexpr int kProberWarps = 4;               // one per SM sub-partition
constexpr int kProberThreads = kProberWarps * 32;
constexpr int kThreads = kGemmThreads + kProberThreads;
constexpr int kProberWarp0 = kGemmWarps;
constexpr int kProberBarrier = 1;             // named barrier of the prober warps
constexpr int kMaxTcnCh = 8;       // action-encoder channel bound
constexpr int kMaxHist = 16;
constexpr int kMaxRowsPerCta = 8;  // M <= 64 rows per cluster
constexpr int kMaxHid = 64;

template <int H>
struct Geom {
    static constexpr int U = H / kCluster;          // hidden units per CTA
    static constexpr int PAIRS = U / 2;             // unit pairs per CTA
    static constexpr int KG = kGemmThreads / PAIRS; // k-groups (lanes per pair)
    static constexpr int KPT = H / KG;              // k values per thread
    static constexpr int KQ = KPT / 4;              // float4 loads per row
    static constexpr int R = 4;                     // rows per GEMM group
    static constexpr int COMBOS = 2 * R;            // (unit-in-pair, row) combos
    static constexpr int PPW = 32 / KG;             // pairs per warp
    static constexpr int VEC = 2 * PPW;             // hidden units per warp
    static_assert(KPT % 4 == 0, "k interleave needs float4 granularity");
    static_assert(KG <= 32 && KG >= COMBOS, "k-groups must fit a warp and cover the combos");
    static_assert(32 / R == kCluster, "one destination CTA per lane in the store");
};

// Odd row strides put consecutive rows in different shared-memory banks.
__host__ __device__ inline uint32_t odd_stride(uint32_t n) { return n | 1u; }

__host__ __device__ inline uint32_t pow2_at_least(uint32_t v) {
    uint32_t p = 1;
    while (p < v) p <<= 1;
    return p;
}

struct SkySmem {
    // Offsets in floats inside the dynamic shared-memory block.
    uint32_t hA, hB, emb, cand, w1, wih, gb, pw2, pw3, pb, red1, a1, a2, pout, x, score, w, h0v, aw, sw, total;
    uint32_t w1_stride, pw_stride, sw_half;
};


// rows = M rows per cluster; Cs = widest state-TCN layer; Ca = action-TCN
// lanes per window (power of two).
__host__ __device__ inline SkySmem sky_smem_layout(uint32_t H, uint32_t rows, uint32_t T, uint32_t E, uint32_t A,
                                                   uint32_t hid, uint32_t layers, uint32_t Cs, uint32_t Ca,
                                                   uint32_t Hs, uint32_t aw_floats, uint32_t Ks, uint32_t Cl,
                                                   uint32_t Cs0, uint32_t levels) {
    SkySmem s;
    uint32_t off = 0;
    auto take = [&](uint32_t n) { uint32_t o = off; off += (n + 3u) & ~3u; return o; };
    const uint32_t rpc = rows / kCluster;
    // hA doubles as the state-TCN scratch, hB as the action-TCN scratch
    const uint32_t per = (Cs + kCluster - 1) / kCluster;
    const uint32_t ks = kThreads / per;
    const uint32_t state_scratch = 3 * Cs * Hs + ks * per * Hs + 8;
    const uint32_t action_scratch = (kThreads / Ca) * 3 * Ca * Hs;
    // the state-TCN weight slices (largest: conv2 + residual of level 0, or
    // the projection) stream through two halves overlaid on hB
    uint32_t wmax = (H / kCluster) * (Cl + 4);
    {
        uint32_t cin = Cs0;
        for (uint32_t l = 0; l < 8 && l < levels; ++l) {
            const uint32_t w1n = per * odd_stride(cin * Ks);
            const uint32_t w2n = per * odd_stride(Cs * Ks) + (cin != Cs ? per * cin : 0);
            wmax = w1n > wmax ? w1n : wmax;
            wmax = w2n > wmax ? w2n : wmax;
            cin = Cs;
        }
    }
    s.sw_half = (wmax + 3u) & ~3u;
    uint32_t hb_need = rows * H;
    hb_need = action_scratch > hb_need ? action_scratch : hb_need;
    hb_need = 2 * s.sw_half > hb_need ? 2 * s.sw_half : hb_need;
    s.hA = take(rows * H > state_scratch ? rows * H : state_scratch);
    s.hB = take(hb_need);
    s.sw = s.hB;
    s.emb = take(rows * T * E);
    s.cand = take(rpc * T * A);
    s.w1_stride = H + 4;
    s.w1 = take(hid * s.w1_stride);
    s.wih = take(3 * (H / kCluster) * E);
    s.gb = take(2 * 3 * (H / kCluster));
    s.pw_stride = hid + 1;
    s.pw2 = take((layers > 1 ? layers - 1 : 1) * hid * s.pw_stride);
    s.pw3 = take(15 * s.pw_stride);
    s.pb = take(hid * layers + 16);
    s.red1 = take(kProberWarps * rpc * hid);
    s.a1 = take(rpc * hid);
    s.a2 = take(rpc * hid);
    s.pout = take(rpc * 16);
    s.x = take(rpc * 20);
    s.score = take(rpc);
    s.w = take(rpc);
    s.h0v = take(H);
    s.aw = take(aw_floats);
    s.total = off;
    return s;
}

__host__ __device__ inline SkySmem layout_for(const SkyjepaArgs& a, uint32_t rows) {
    return sky_smem_layout(a.H, rows, a.T, a.E, a.A, a.hid, a.prober_layers, a.state_tcn.max_ch,
                           pow2_at_least(a.action_tcn.max_ch), a.Hs, tcn_weight_floats(a.action_tcn), a.state_tcn.k,
                           a.state_tcn.out_dim, a.state_tcn.input_dim, a.state_tcn.levels);
}

// acc[t] += sum_j w[j] * x[t - (K-1-j)*DIL] for t < HS (taps before the
// window start read the causal zero padding and are skipped).  HS == 0 is the
// runtime-shape fallback.
template <int HS, int K, int DIL>
__device__ __forceinline__ void conv_taps(float (&acc)[kMaxHist], const float* x, const float* w, uint32_t Hs,
                                          uint32_t Kr, uint32_t dil) {
    if constexpr (HS > 0) {
#pragma unroll
        for (int j = 0; j < K; ++j) {
            const float wv = w[j];
            const int sh = (K - 1 - j) * DIL;
#pragma unroll
            for (int t = sh; t < HS; ++t) acc[t] = fmaf(wv, x[t - sh], acc[t]);
        }
    } else {
        for (uint32_t j = 0; j < Kr; ++j) {
            const float wv = w[j];
            const int sh = static_cast<int>((Kr - 1 - j) * dil);
#pragma unroll
            for (int t = 0; t < kMaxHist; ++t)
                if (t < static_cast<int>(Hs) && t >= sh) acc[t] = fmaf(wv, x[t - sh], acc[t]);
        }
    }
}

// Dispatch on the dilation (1, 2, 4, 8 specialised) for one input channel.
template <int HS, int K>
__device__ __forceinline__ void conv_channel(float (&acc)[kMaxHist], const float* x, const float* w, uint32_t Hs,
                                             uint32_t Kr, uint32_t dil) {
    if constexpr (HS > 0) {
        switch (dil) {
            case 1: conv_taps<HS, K, 1>(acc, x, w, Hs, Kr, dil); return;
            case 2: conv_taps<HS, K, 2>(acc, x, w, Hs, Kr, dil); return;
            case 4: conv_taps<HS, K, 4>(acc, x, w, Hs, Kr, dil); return;
            case 8: conv_taps<HS, K, 8>(acc, x, w, Hs, Kr, dil); return;
            default: break;
        }
    }
    conv_taps<0, 0, 0>(acc, x, w, Hs, Kr, dil);
}

__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
__device__ __forceinline__ void prober_sync() { asm volatile("bar.sync %0, %1;" :: "n"(kProberBarrier), "n"(kProberThreads) : "memory"); }

// Asynchronous global->shared copy of n floats (4-byte granularity, any alignment).
__device__ __forceinline__ void async_copy(float* dst, const float* src, uint32_t n) {
    for (uint32_t i = threadIdx.x; i < n; i += kThreads) {
        const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst + i));
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" :: "r"(d), "l"(src + i) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void async_wait_all_but_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// --------------------------------------------------------------- prologue
//
// SkyJepaModel::encode_state_history (model.rs:57-61): normalised state
// history -> TemporalConvEncoder::forward_last (tcn.rs:138-160) ->
// state_projection.  CTA c computes output channels [c*per, (c+1)*per) of
// every convolution: thread (o, slice) sums its slice of input channels for
// all time steps, the slices are reduced in shared memory, and the result is
// broadcast to every CTA's activation buffer.
template <int HS, int KT>
__device__ void state_tcn_cluster(const SkyjepaArgs& a, cg::cluster_group& cluster, uint32_t c, uint32_t b,
                                  float* scratch, float* h0v, float* sw, uint32_t sw_half) {
    const TcnView& tcn = a.state_tcn;
    const uint32_t Hs = a.Hs, C = tcn.max_ch, tid = threadIdx.x, K = tcn.k;
    const uint32_t per = (C + kCluster - 1) / kCluster;
    const uint32_t KS = kThreads / per;
    const uint32_t o0 = c * per;
    const uint32_t hper = a.H / kCluster, Cl = tcn.out_dim;
    float* xa = scratch;
    float* xb = scratch + C * Hs;
    float* hb = scratch + 2 * C * Hs;
    float* red = scratch + 3 * C * Hs;  // [KS][per][Hs], local
    // Weight slices of the convolutions in order (conv1, conv2 + residual of
    // every level, then the projection) stream through two shared buffers.
    const uint32_t nstage = 2 * tcn.levels + 1;
    // rows of `row_len` floats land `dst_stride` apart (odd strides: no bank conflicts)
    auto copy_rows = [&](float* dst, const float* src, uint32_t rows_n, uint32_t row_len, uint32_t dst_stride) {
        for (uint32_t q = tid; q < rows_n * row_len; q += kThreads) {
            const uint32_t r = q / row_len, e = q - r * row_len;
            const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst + r * dst_stride + e));
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" :: "r"(d), "l"(src + q) : "memory");
        }
    };
    auto stage = [&](uint32_t n) {
        float* dst = sw + (n & 1) * sw_half;
        if (n < nstage) {
            if (n == nstage - 1) {
                copy_rows(dst, a.proj_w + static_cast<size_t>(c * hper) * Cl, hper, Cl, Cl + 4);
            } else {
                const TcnBlockView& bk = tcn.blocks[n / 2];
                const uint32_t cnt = min(per, bk.out > o0 ? bk.out - o0 : 0u);
                if (n % 2 == 0) {
                    copy_rows(dst, bk.w1 + static_cast<size_t>(o0) * bk.in * K, cnt, bk.in * K, odd_stride(bk.in * K));
                } else {
                    // conv2 slice, then the residual 1x1 slice after it
                    copy_rows(dst, bk.w2 + static_cast<size_t>(o0) * bk.out * K, cnt, bk.out * K, odd_stride(bk.out * K));
                    if (bk.wr)
                        copy_rows(dst + per * odd_stride(bk.out * K), bk.wr + static_cast<size_t>(o0) * bk.in, cnt, bk.in, bk.in);
                }
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    __syncthreads();  // the weight buffers overlay the action-TCN scratch
    stage(0);
    for (uint32_t q = tid; q < tcn.input_dim * Hs; q += kThreads) {
        const uint32_t i = q / Hs, t = q % Hs;
        const float v = a.state_hist[(static_cast<size_t>(b) * Hs + t) * 18 + i];
        xa[q] = (v - a.state_mean[i]) / a.state_std[i];
    }
    float* cur = xa;
    float* nxt = xb;
    const uint32_t o_local = tid % per, slice = tid / per;
    uint32_t n = 0;
    for (uint32_t l = 0; l < tcn.levels; ++l) {
        const TcnBlockView& bk = tcn.blocks[l];
        const uint32_t o = o0 + o_local;
        for (int conv = 0; conv < 2; ++conv, ++n) {
            stage(n + 1);
            async_wait_all_but_one();
            __syncthreads();
            const float* Ws = sw + (n & 1) * sw_half;
            const float* src = conv == 0 ? cur : hb;
            const uint32_t cin = conv == 0 ? bk.in : bk.out;
            const uint32_t wstride = odd_stride(cin * K);
            if (slice < KS && o < bk.out) {
                float acc[kMaxHist];
#pragma unroll
                for (int t = 0; t < kMaxHist; ++t) acc[t] = 0.0f;
                for (uint32_t i = slice; i < cin; i += KS)
                    conv_channel<HS, KT>(acc, src + i * Hs, Ws + o_local * wstride + i * K, Hs, K, bk.dil);
#pragma unroll
                for (int t = 0; t < kMaxHist; ++t)
                    if (t < static_cast<int>(Hs)) red[(slice * per + o_local) * Hs + t] = acc[t];
            }
            __syncthreads();
            for (uint32_t q = tid; q < per * Hs; q += kThreads) {
                const uint32_t ol = q / Hs, t = q % Hs, oo = o0 + ol;
                if (oo >= bk.out) continue;
                float s = 0.0f;
                for (uint32_t k = 0; k < KS; ++k) s += red[(k * per + ol) * Hs + t];
                float v;
                if (conv == 0) {
                    v = gelu_tanh(s + __ldg(bk.b1 + oo));
                } else {
                    const float h2 = gelu_tanh(s + __ldg(bk.b2 + oo));
                    float res;
                    if (bk.wr) {
                        const float* wrs = Ws + per * odd_stride(bk.out * K) + ol * bk.in;
                        float r0 = 0.0f, r1 = 0.0f;
                        uint32_t i = 0;
                        for (; i + 2 <= bk.in; i += 2) {
                            r0 = fmaf(wrs[i], cur[i * Hs + t], r0);
                            r1 = fmaf(wrs[i + 1], cur[(i + 1) * Hs + t], r1);
                        }
                        if (i < bk.in) r0 = fmaf(wrs[i], cur[i * Hs + t], r0);
                        res = (r0 + r1) + __ldg(bk.br + oo);
                    } else {
                        res = cur[oo * Hs + t];
                    }
                    v = gelu_tanh(h2 + res);
                }
                float* dst = conv == 0 ? hb : nxt;
                for (uint32_t d = 0; d < kCluster; ++d) cluster.map_shared_rank(dst, d)[oo * Hs + t] = v;
            }
            cluster.sync();
        }
        float* tmp = cur; cur = nxt; nxt = tmp;
    }
    // state_projection of the last time step: CTA c writes H/8 outputs to
    // every CTA; four lanes per output, reduced with shuffles.
    stage(n + 1);
    async_wait_all_but_one();
    __syncthreads();
    const float* Wp = sw + (n & 1) * sw_half;
    for (uint32_t q = tid; q < hper * 4; q += kThreads) {
        const uint32_t ol = q / 4, part = q % 4, oo = c * hper + ol;
        float s = 0.0f;
        for (uint32_t i = part; i < Cl; i += 4) s = fmaf(cur[i * Hs + Hs - 1], Wp[ol * (Cl + 4) + i], s);
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if (part == 0) {
            const float v = s + __ldg(a.proj_b + oo);
            for (uint32_t d = 0; d < kCluster; ++d) cluster.map_shared_rank(h0v, d)[oo] = v;
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// The history encoder alone: h0 of vehicle blockIdx.y by one 8-CTA cluster
// (state_tcn_cluster, the rollout kernel's prologue, as a kernel of its own)
// for the tensor-core rollouts of few vehicles with a wide state encoder.
__global__ void __launch_bounds__(kThreads, 1) skyjepa_h0_cluster_kernel(SkyjepaArgs a, float* h0,
                                                                         uint32_t scratch_floats, uint32_t sw_half) {
    extern __shared__ __align__(16) float smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t c = cluster.block_rank(), b = blockIdx.y;
    float* scratch = smem;
    float* sw = smem + scratch_floats;
    float* h0v = sw + 2 * sw_half;
    cluster.sync();  // every CTA of the cluster runs before any DSMEM access
    if (a.Hs == 10 && a.state_tcn.k == 3) state_tcn_cluster<10, 3>(a, cluster, c, b, scratch, h0v, sw, sw_half);
    else state_tcn_cluster<0, 0>(a, cluster, c, b, scratch, h0v, sw, sw_half);
    cluster.sync();  // h0 complete in every CTA
    if (c == 0)
        for (uint32_t u = threadIdx.x; u < a.H; u += kThreads) h0[static_cast<size_t>(b) * a.H + u] = h0v[u];
}

cudaError_t launch_skyjepa_h0_cluster(const SkyjepaArgs& a, float* h0, cudaStream_t stream) {
    const TcnView& tcn = a.state_tcn;
    const uint32_t C = tcn.max_ch, Hs = a.Hs, K = tcn.k;
    const uint32_t per = (C + kCluster - 1) / kCluster, ks = kThreads / per;
    const uint32_t scratch = ((3 * C * Hs + ks * per * Hs + 8) + 3u) & ~3u;
    uint32_t wmax = (a.H / kCluster) * (tcn.out_dim + 4);
    uint32_t cin = tcn.input_dim;
    for (uint32_t l = 0; l < tcn.levels; ++l) {
        const uint32_t w1n = per * odd_stride(cin * K);
        const uint32_t w2n = per * odd_stride(C * K) + (cin != C ? per * cin : 0);
        wmax = w1n > wmax ? w1n : wmax;
        wmax = w2n > wmax ? w2n : wmax;
        cin = C;
    }
    const uint32_t sw_half = (wmax + 3u) & ~3u;
    const size_t smem = (static_cast<size_t>(scratch) + 2 * sw_half + a.H) * sizeof(float);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(skyjepa_h0_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kCluster, a.B, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, skyjepa_h0_cluster_kernel, a, h0, scratch, sw_half);
}

// SkyJepaModel::rollout_candidates window encoding (model.rs:192-215) with
// TemporalConvEncoder::forward (tcn.rs:88-96, 138-160) over one window held
// in `cur` [Cm][Hs] (input channels normalised, zero elsewhere): `ca` lanes of
// one warp, lane o computing output channel o of every convolution at every
// position in registers, with warp-level syncs between the convolutions (every
// lane of the warp calls this, `active` or not).  On return cur holds the
// last block's output.  `aw` is where the encoder's weights (contiguous from
// tcn.blocks[0].w1) are read: a shared-memory copy or the blob itself.
template <int HS, int KT>
__device__ void action_tcn_window(const TcnView& tcn, const float* aw, float* cur, float* hb, uint32_t Hs, uint32_t o,
                                  bool active) {
    const float* wbase = tcn.blocks[0].w1;
    auto sm = [&](const float* p) { return aw + (p - wbase); };
    for (uint32_t l = 0; l < tcn.levels; ++l) {
        const TcnBlockView& bk = tcn.blocks[l];
        const bool mine = active && o < bk.out;
        float h2[kMaxHist];
        for (int conv = 0; conv < 2; ++conv) {
            const float* src = conv == 0 ? cur : hb;
            const uint32_t cin = conv == 0 ? bk.in : bk.out;
            const float* W = sm(conv == 0 ? bk.w1 : bk.w2);
            float acc[kMaxHist];
#pragma unroll
            for (int t = 0; t < kMaxHist; ++t) acc[t] = 0.0f;
            if (mine)
                for (uint32_t i = 0; i < cin; ++i)
                    conv_channel<HS, KT>(acc, src + i * Hs, W + (o * cin + i) * tcn.k, Hs, tcn.k, bk.dil);
            const float bias = mine ? sm(conv == 0 ? bk.b1 : bk.b2)[o] : 0.0f;
            if (conv == 0) {
                if (mine)
#pragma unroll
                    for (int t = 0; t < kMaxHist; ++t)
                        if (t < static_cast<int>(Hs)) hb[o * Hs + t] = gelu_tanh(acc[t] + bias);
            } else {
#pragma unroll
                for (int t = 0; t < kMaxHist; ++t) h2[t] = gelu_tanh(acc[t] + bias);
            }
            __syncwarp();
        }
        float res[kMaxHist];
#pragma unroll
        for (int t = 0; t < kMaxHist; ++t) res[t] = 0.0f;
        if (mine) {
            if (bk.wr) {
                const float br = sm(bk.br)[o];
                const float* wr = sm(bk.wr) + o * bk.in;
#pragma unroll
                for (int t = 0; t < kMaxHist; ++t) {
                    if (t >= static_cast<int>(Hs)) break;
                    float r = 0.0f;
                    for (uint32_t i = 0; i < bk.in; ++i) r = fmaf(wr[i], cur[i * Hs + t], r);
                    res[t] = r + br;
                }
            } else {
#pragma unroll
                for (int t = 0; t < kMaxHist; ++t)
                    if (t < static_cast<int>(Hs)) res[t] = cur[o * Hs + t];
            }
        }
        __syncwarp();
        if (mine)
#pragma unroll
            for (int t = 0; t < kMaxHist; ++t)
                if (t < static_cast<int>(Hs)) cur[o * Hs + t] = gelu_tanh(h2[t] + res[t]);
        __syncwarp();
    }
}

// The window of (row rr, step t0) is [history(Hs-1) ++ candidates][t0 .. t0+Hs),
// each window zero-padded on its own (TemporalBlock::forward, tcn.rs:88-96).
// The last position of every window of the CTA's own rows goes to every CTA
// of the cluster.
template <int HS, int KT>
__device__ void action_tcn_windows(const SkyjepaArgs& a, cg::cluster_group& cluster, uint32_t c, uint32_t b,
                                   uint32_t rpc, const float* s_cand, float* scratch, float* s_emb, const float* aw) {
    const TcnView& tcn = a.action_tcn;
    const uint32_t Hs = a.Hs, T = a.T, A = a.A, E = a.E, TA = T * A;
    const uint32_t ca = pow2_at_least(tcn.max_ch);
    const uint32_t wpp = kThreads / ca;
    const uint32_t slot = threadIdx.x / ca, o = threadIdx.x % ca;
    const uint32_t windows = rpc * T;
    const uint32_t Cm = ca;
    float* cur = scratch + slot * 3 * Cm * Hs;
    float* hb = cur + Cm * Hs;
    for (uint32_t w0 = 0; w0 < windows; w0 += wpp) {
        const uint32_t win = w0 + slot;
        const bool active = win < windows;
        const uint32_t rr = active ? win / T : 0, t0 = active ? win % T : 0;
        if (active && o < tcn.input_dim) {
            for (uint32_t w = 0; w < Hs; ++w) {
                const uint32_t pos = t0 + w;
                const float v = pos < Hs - 1 ? a.action_hist[(static_cast<size_t>(b) * (Hs - 1) + pos) * A + o]
                                             : s_cand[rr * TA + (pos - (Hs - 1)) * A + o];
                cur[o * Hs + w] = (v - a.action_mean[o]) / a.action_std[o];
            }
        }
        __syncwarp();
        action_tcn_window<HS, KT>(tcn, aw, cur, hb, Hs, o, active);
        if (active && o < E) {
            const float v = cur[o * Hs + Hs - 1];
            const uint32_t m = c * rpc + rr;
            for (uint32_t d = 0; d < kCluster; ++d) cluster.map_shared_rank(s_emb, d)[(m * T + t0) * E + o] = v;
        }
        __syncwarp();
    }
}

// ------------------------------------------------------- the prober warps
//
// SkyJepaProber::forward (prober.rs:84-102) for the CTA's own rows, then one
// step of lewm_skyjepa_integrate_f32 (kinematics.rs:377-484) and the tracking
// cost (control.rs:430-452) of that step.  Four warps: layer 1 is split over
// k (warp pw sums k in [pw*H/4, (pw+1)*H/4)), the later layers over
// (row, output) pairs; the integrator runs on lanes 0..rpc-1 of the first.
__device__ void prober_step(const SkyjepaArgs& a, const SkySmem& L, float* smem, const float* hn, uint32_t c,
                            uint32_t b, uint32_t rpc, uint32_t own0, uint32_t t, uint32_t H) {
    const uint32_t ptid = threadIdx.x - kGemmThreads;  // 0..127
    const uint32_t pw = ptid >> 5, lane = ptid & 31, hid = a.hid, T = a.T, A = a.A, TA = T * A;
    float* s_a1 = smem + L.a1;
    float* s_a2 = smem + L.a2;
    float* s_pout = smem + L.pout;
    float* red1 = smem + L.red1;  // [kProberWarps][rpc][hid]
    const float* w1 = smem + L.w1;
    const float* pb = smem + L.pb;
    // layer 1 partial sums: lane owns outputs lane and lane + 32
    {
        float acc[2][kMaxRowsPerCta];
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
            for (int r = 0; r < kMaxRowsPerCta; ++r) acc[q][r] = 0.0f;
        const bool has0 = lane < hid, has1 = lane + 32 < hid;
        const float* wr0 = w1 + lane * L.w1_stride;
        const float* wr1 = w1 + (lane + 32) * L.w1_stride;
        const uint32_t k0 = pw * (H / kProberWarps), k1 = k0 + H / kProberWarps;
        for (uint32_t k = k0; k < k1; k += 4) {
            const float4 w0 = has0 ? *reinterpret_cast<const float4*>(wr0 + k) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 w1v = has1 ? *reinterpret_cast<const float4*>(wr1 + k) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int r = 0; r < kMaxRowsPerCta; ++r) {
                if (static_cast<uint32_t>(r) >= rpc) break;
                const float4 hv = *reinterpret_cast<const float4*>(hn + (c * rpc + r) * H + k);
                float s = acc[0][r];
                s = fmaf(w0.x, hv.x, s); s = fmaf(w0.y, hv.y, s); s = fmaf(w0.z, hv.z, s); s = fmaf(w0.w, hv.w, s);
                acc[0][r] = s;
                if (has1) {
                    float u = acc[1][r];
                    u = fmaf(w1v.x, hv.x, u); u = fmaf(w1v.y, hv.y, u); u = fmaf(w1v.z, hv.z, u); u = fmaf(w1v.w, hv.w, u);
                    acc[1][r] = u;
                }
            }
        }
#pragma unroll
        for (int r = 0; r < kMaxRowsPerCta; ++r) {
            if (static_cast<uint32_t>(r) >= rpc) break;
            if (has0) red1[(pw * rpc + r) * hid + lane] = acc[0][r];
            if (has1) red1[(pw * rpc + r) * hid + lane + 32] = acc[1][r];
        }
    }
    prober_sync();
    for (uint32_t q = ptid; q < rpc * hid; q += kProberThreads) {
        const uint32_t r = q / hid, o = q % hid;
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < kProberWarps; ++w) s += red1[(w * rpc + r) * hid + o];
        s_a1[r * hid + o] = gelu_tanh(s + pb[o]);
    }
    prober_sync();
    // hidden layers: one (row, output) pair per thread
    float* pin = s_a1;
    float* pout = s_a2;
    for (uint32_t l = 0; l + 1 < a.prober_layers; ++l) {
        const float* W = smem + L.pw2 + l * hid * L.pw_stride;
        const float* bias = pb + (l + 1) * hid;
        for (uint32_t q = ptid; q < rpc * hid; q += kProberThreads) {
            const uint32_t r = q / hid, o = q % hid;
            const float* ar = pin + r * hid;
            const float* wr = W + o * L.pw_stride;
            float s0 = 0.0f, s1 = 0.0f;
            uint32_t i = 0;
            for (; i + 2 <= hid; i += 2) { s0 = fmaf(ar[i], wr[i], s0); s1 = fmaf(ar[i + 1], wr[i + 1], s1); }
            if (i < hid) s0 = fmaf(ar[i], wr[i], s0);
            pout[q] = gelu_tanh((s0 + s1) + bias[o]);
        }
        prober_sync();
        float* tmp = pin; pin = pout; pout = tmp;
    }
    // output layer: 15 values per row
    for (uint32_t q = ptid; q < rpc * 15; q += kProberThreads) {
        const uint32_t r = q / 15, o = q % 15;
        const float* ar = pin + r * hid;
        const float* wr = smem + L.pw3 + o * L.pw_stride;
        float s0 = 0.0f, s1 = 0.0f;
        uint32_t i = 0;
        for (; i + 2 <= hid; i += 2) { s0 = fmaf(ar[i], wr[i], s0); s1 = fmaf(ar[i + 1], wr[i + 1], s1); }
        if (i < hid) s0 = fmaf(ar[i], wr[i], s0);
        s_pout[r * 16 + o] = (s0 + s1) + pb[a.prober_layers * hid + o];
    }
    prober_sync();
    // integrator + cost: thread r of the first prober warp owns row r
    if (ptid < rpc) {
        float* xs = smem + L.x + ptid * 20;
        float x[18];
#pragma unroll
        for (int i = 0; i < 18; ++i) x[i] = xs[i];
        const float* act = smem + L.cand + ptid * TA + t * A;
        xs[18] += integrate_and_cost(a, b, own0 + ptid, t, x, act, s_pout + ptid * 16);
#pragma unroll
        for (int i = 0; i < 18; ++i) xs[i] = x[i];
    }
}

// ------------------------------------------------------------ rollout kernel

template <int H>
__global__ void __launch_bounds__(kThreads, 1) skyjepa_rollout_kernel(SkyjepaArgs a) {
    using G = Geom<H>;
    extern __shared__ __align__(16) float smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t c = cluster.block_rank();
    const uint32_t b = blockIdx.y;
    const uint32_t rb = blockIdx.x / kCluster;  // row block of this cluster
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t T = a.T, A = a.A, E = a.E, Hs = a.Hs, hid = a.hid;
    const uint32_t rows = a.rows, rpc = rows / kCluster, groups = rows / G::R;
    const SkySmem L = layout_for(a, rows);
    float* s_emb = smem + L.emb;     // [rows][T][E]
    float* s_cand = smem + L.cand;   // [rpc][T][A]
    float* s_wih = smem + L.wih;     // [3][U][E] for this CTA's units
    float* s_score = smem + L.score;
    float* s_w = smem + L.w;
    float* s_h0 = smem + L.h0v;
    const uint32_t own0 = rb * rows + c * rpc;  // first sample this CTA owns
    const uint32_t TA = T * A;

    // ---- shared copies of the small weights
    for (uint32_t q = tid; q < hid * H / 4; q += kThreads) {
        const uint32_t o = q / (H / 4), k4 = q % (H / 4);
        *reinterpret_cast<float4*>(smem + L.w1 + o * L.w1_stride + 4 * k4) =
            __ldg(reinterpret_cast<const float4*>(a.p_in_w) + q);
    }
    for (uint32_t q = tid; q < 3 * G::U * E; q += kThreads) {
        const uint32_t g = q / (G::U * E), rem = q % (G::U * E), u = rem / E, e = rem % E;
        s_wih[q] = __ldg(a.w_ih + (static_cast<size_t>(g) * H + c * G::U + u) * E + e);
    }
    for (uint32_t q = tid; q < 3 * G::U; q += kThreads) {
        const uint32_t g = q / G::U, u = q % G::U;
        smem[L.gb + q] = __ldg(a.b_ih + g * H + c * G::U + u);           // b_ih [3][U]
        smem[L.gb + 3 * G::U + q] = __ldg(a.b_hh + g * H + c * G::U + u);  // b_hh [3][U]
    }
    for (uint32_t l = 0; l + 1 < a.prober_layers; ++l)
        for (uint32_t q = tid; q < hid * hid; q += kThreads)
            smem[L.pw2 + l * hid * L.pw_stride + (q / hid) * L.pw_stride + q % hid] = __ldg(a.p_hid_w[l] + q);
    for (uint32_t q = tid; q < 15 * hid; q += kThreads)
        smem[L.pw3 + (q / hid) * L.pw_stride + q % hid] = __ldg(a.p_out_w + q);
    for (uint32_t q = tid; q < hid; q += kThreads) smem[L.pb + q] = __ldg(a.p_in_b + q);
    for (uint32_t l = 0; l + 1 < a.prober_layers; ++l)
        for (uint32_t q = tid; q < hid; q += kThreads) smem[L.pb + (l + 1) * hid + q] = __ldg(a.p_hid_b[l] + q);
    for (uint32_t q = tid; q < 15; q += kThreads) smem[L.pb + a.prober_layers * hid + q] = __ldg(a.p_out_b + q);
    {
        const uint32_t n = tcn_weight_floats(a.action_tcn);
        const float* src = a.action_tcn.blocks[0].w1;
        for (uint32_t q = tid; q < n; q += kThreads) smem[L.aw + q] = __ldg(src + q);
    }

    // ---- sampling of the CTA's own rows (as sample_kernel)
    for (uint32_t q = tid; q < rpc * TA; q += kThreads) {
        const uint32_t rr = q / TA, e = q % TA, act = e % A;
        const uint32_t s = own0 + rr;
        const uint64_t ci = (static_cast<uint64_t>(b) * a.S + s) * TA + e;
        float v;
        if (a.sample) {
            const size_t mi = static_cast<size_t>(b) * TA + e;
            if (a.sample_base + s == 0 || s >= a.S) {
                v = a.mean[mi];
            } else {
                const uint64_t gi = global_row(b, s, a.sample_base, a.sample_total, a.S) * TA + e;
                const float eps = a.noise ? a.noise[ci] : normal_at(a.seed, a.offset + gi);
                v = a.mean[mi] + eps * a.std[mi];
            }
            v = cmin(cmax(v, a.low[act]), a.high[act]);
            if (a.cand_out && s < a.S) a.cand_out[ci] = v;
        } else {
            v = s < a.S ? a.cand_in[ci] : a.low[act];
        }
        s_cand[q] = v;
    }
    for (uint32_t q = tid; q < rpc * 20; q += kThreads) {
        const uint32_t i = q % 20;
        smem[L.x + q] = i < 18 ? a.state_hist[(static_cast<size_t>(b) * Hs + Hs - 1) * 18 + i] : 0.0f;
    }
    // every CTA of the cluster must be running before any DSMEM access
    cluster.sync();

    // ---- window embeddings of the own rows -> every CTA; h0 -> every CTA
    if (Hs == 10 && a.action_tcn.k == 3) action_tcn_windows<10, 3>(a, cluster, c, b, rpc, s_cand, smem + L.hB, s_emb, smem + L.aw);
    else action_tcn_windows<0, 0>(a, cluster, c, b, rpc, s_cand, smem + L.hB, s_emb, smem + L.aw);
    if (Hs == 10 && a.state_tcn.k == 3) state_tcn_cluster<10, 3>(a, cluster, c, b, smem + L.hA, s_h0, smem + L.sw, L.sw_half);
    else state_tcn_cluster<0, 0>(a, cluster, c, b, smem + L.hA, s_h0, smem + L.sw, L.sw_half);
    cluster.sync();  // embeddings of all rows and h0 are complete everywhere
    {
        const float4* src = reinterpret_cast<const float4*>(s_h0);
        float4* dst = reinterpret_cast<float4*>(smem + L.hA);
        for (uint32_t q = tid; q < rows * H / 4; q += kThreads) dst[q] = src[q % (H / 4)];
    }
    __syncthreads();

    if (warp >= kProberWarp0) {
        // ---- prober warps: step t's prober / integrator / cost while the GEMM
        // warps compute step t+1.  Arrival at phase t means "done with h_t".
        for (uint32_t t = 0; t < T; ++t) {
            cluster_arrive();
            cluster_wait();
            const float* hn = smem + ((t & 1) ? L.hA : L.hB);
            prober_step(a, L, smem, hn, c, b, rpc, own0, t, H);
        }
    } else {
        // ---- GEMM warps: registers hold this thread's W_hh slice
        const uint32_t pl = lane / G::KG, kg = lane % G::KG;
        const uint32_t pair = warp * G::PPW + pl;
        // Accumulator slot s of this lane holds (unit-in-pair, row) combo
        // s ^ (kg % COMBOS): the lane's weights and h rows are taken in that
        // permuted order, so that every level of the reduce-scatter below
        // keeps slots [0, m) and sends slots [m, 2m) on every lane (the
        // partner's slot cc + m holds the combo of this lane's slot cc) and
        // needs no per-lane selects; the sums are the same, in the same order.
        const uint32_t xq = (kg % G::COMBOS) / G::R, xr = kg % G::R;
        float wr[2][3][G::KPT];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const uint32_t j = c * G::U + pair * 2 + (q ^ xq);
#pragma unroll
            for (int g = 0; g < 3; ++g) {
                const float* row = a.w_hh + (static_cast<size_t>(g) * H + j) * H;
#pragma unroll
                for (int i = 0; i < G::KQ; ++i) {
                    const float4 v = __ldg(reinterpret_cast<const float4*>(row + kg * 4 + 4 * G::KG * i));
                    wr[q][g][4 * i + 0] = v.x; wr[q][g][4 * i + 1] = v.y;
                    wr[q][g][4 * i + 2] = v.z; wr[q][g][4 * i + 3] = v.w;
                }
            }
        }
        const uint32_t combo = kg % G::COMBOS;
        const uint32_t my_q = combo / G::R, my_r = combo % G::R;
        const uint32_t my_local = pair * 2 + my_q;
        const uint32_t my_unit = c * G::U + my_local;
        const float* s_bih = smem + L.gb + my_local;             // stride U per gate
        const float* s_bhh = smem + L.gb + 3 * G::U + my_local;
        for (uint32_t t = 0; t < T; ++t) {
            const float* hc = smem + ((t & 1) ? L.hB : L.hA);
            float* hn = smem + ((t & 1) ? L.hA : L.hB);
#pragma unroll 1
            for (uint32_t grp = 0; grp < groups; ++grp) {
                // one group = 4 rows x this thread's 2 units x 3 gates
                float acc[2 * G::R][3];
#pragma unroll
                for (int q = 0; q < 2 * G::R; ++q) { acc[q][0] = 0.0f; acc[q][1] = 0.0f; acc[q][2] = 0.0f; }
#pragma unroll
                for (int i = 0; i < G::KQ; ++i) {
                    float4 hv[G::R];
#pragma unroll
                    for (int r = 0; r < G::R; ++r)
                        hv[r] = *reinterpret_cast<const float4*>(hc + (grp * G::R + (r ^ xr)) * H + kg * 4 +
                                                                 4 * G::KG * i);
#pragma unroll
                    for (int comp = 0; comp < 4; ++comp)
#pragma unroll
                        for (int r = 0; r < G::R; ++r) {
                            const float hcomp = comp == 0 ? hv[r].x : comp == 1 ? hv[r].y : comp == 2 ? hv[r].z : hv[r].w;
#pragma unroll
                            for (int q = 0; q < 2; ++q)
#pragma unroll
                                for (int g = 0; g < 3; ++g)
                                    acc[q * G::R + r][g] = fmaf(wr[q][g][4 * i + comp], hcomp, acc[q * G::R + r][g]);
                        }
                }
                // reduce-scatter over the low 3 lane bits (lane kg ends with
                // combo kg & 7 in slot 0), then all-reduce over the remaining
                // k-group bits
#pragma unroll
                for (int m = G::COMBOS / 2; m >= 1; m >>= 1)
#pragma unroll
                    for (int cc = 0; cc < m; ++cc)
#pragma unroll
                        for (int g = 0; g < 3; ++g)
                            acc[cc][g] = acc[cc][g] + __shfl_xor_sync(0xffffffffu, acc[cc + m][g], m);
#pragma unroll
                for (int m = G::COMBOS; m < G::KG; m <<= 1)
#pragma unroll
                    for (int g = 0; g < 3; ++g) acc[0][g] += __shfl_xor_sync(0xffffffffu, acc[0][g], m);
                // candle GRU step for (row mrow, unit my_unit)
                const uint32_t mrow = grp * G::R + my_r;
                const float* xe = s_emb + (mrow * T + t) * E;
                float gi[3];
                if (E == 4) {
                    // the common width: one 16-byte load per operand (the
                    // same fmas in the same order as the loop below)
                    const float4 x = *reinterpret_cast<const float4*>(xe);
#pragma unroll
                    for (int g = 0; g < 3; ++g) {
                        const float4 w = *reinterpret_cast<const float4*>(s_wih + (g * G::U + my_local) * 4);
                        float s = fmaf(x.x, w.x, 0.0f);
                        s = fmaf(x.y, w.y, s);
                        s = fmaf(x.z, w.z, s);
                        s = fmaf(x.w, w.w, s);
                        gi[g] = s + s_bih[g * G::U];
                    }
                } else {
#pragma unroll
                    for (int g = 0; g < 3; ++g) {
                        const float* wi = s_wih + (g * G::U + my_local) * E;
                        float s = 0.0f;
#pragma unroll
                        for (int e = 0; e < kMaxTcnCh; ++e)
                            if (static_cast<uint32_t>(e) < E) s = fmaf(xe[e], wi[e], s);
                        gi[g] = s + s_bih[g * G::U];
                    }
                }
                const float ghr = acc[0][0] + s_bhh[0], ghz = acc[0][1] + s_bhh[G::U], ghn = acc[0][2] + s_bhh[2 * G::U];
                const float rg = sigmoid(gi[0] + ghr);
                const float zg = sigmoid(gi[1] + ghz);
                const float ng = tanhf(gi[2] + rg * ghn);
                const float hp = hc[mrow * H + my_unit];
                const float hnew = zg * hp - (zg - 1.0f) * ng;
                // lane L stores row L & 3 (G::VEC consecutive units of this
                // warp) into CTA L >> 2
                const uint32_t srow_l = lane & (G::R - 1);
                float vals[G::VEC];
#pragma unroll
                for (int v = 0; v < G::VEC; ++v)
                    vals[v] = __shfl_sync(0xffffffffu, hnew, (v / 2) * G::KG + (v % 2) * G::R + srow_l);
                float* local = hn + (grp * G::R + srow_l) * H + c * G::U + warp * G::VEC;
                float* dst = cluster.map_shared_rank(local, lane / G::R);
                if constexpr (G::VEC == 4) {
                    *reinterpret_cast<float4*>(dst) = make_float4(vals[0], vals[1], vals[2], vals[3]);
                } else {
                    *reinterpret_cast<float2*>(dst) = make_float2(vals[0], vals[1]);
                }
            }
            cluster_arrive();  // h_{t+1} stored everywhere
            cluster_wait();
        }
    }
    __syncthreads();  // the prober warps have finished the last step

    // ---- scores of the own rows, then the MPPI tuple
    if (tid < rpc) {
        const float score = smem[L.x + tid * 20 + 18] * static_cast<float>(1.0 / static_cast<double>(T));
        s_score[tid] = score;
        const uint32_t s = own0 + tid;
        if (s < a.S) a.scores[static_cast<size_t>(b) * a.S + s] = score;
    }
    __syncthreads();
    if (a.mppi) {
        const uint32_t nvalid = own0 >= a.S ? 0u : min(rpc, a.S - own0);
        const uint32_t p = rb * kCluster + c;
        mppi_reduce_rows<kThreads>(a.m, b, p, nvalid, s_score, own0, s_cand, TA, s_w);
    }
}

// ------------------------------------------------------ small-latent path
//
// Models whose latent fits one or two registers per lane (latent <= 64, the
// paper-derived SkyJEPA: latent 24, TCN [8, 8, 16] / [4, 4, 8], prober 32 x 2)
// run a warp per candidate:
//   skyjepa_small_inputs_kernel  x_t of every (candidate, step): the action
//       encoder over its window (action_tcn_window), `ca` lanes per window;
//   skyjepa_small_kernel  the GRU rollout (lane j owns units j and j + 32;
//       h is broadcast by shuffles), the prober (lane o owns outputs o and
//       o + 32), then the integrator and the cost, computed by every lane
//       of the warp alike; the scores and the fused MPPI partial of the block.
// The initial latent per vehicle comes from skyjepa_h0_kernel.
constexpr uint32_t kSmallMaxH = 64, kSmallWarps = 8, kSmallThreads = kSmallWarps * 32;

struct SmallSmem {
    uint32_t whh, wih, bih, bhh, w1, b1, wh, bh, wo, bo, score, w, total;
    uint32_t hs, ps;  // row strides of W_hh and of the prober's hidden / output layers
};

__host__ __device__ inline SmallSmem small_layout(const SkyjepaArgs& a) {
    SmallSmem L{};
    const uint32_t H = a.H, E = a.E, hid = a.hid;
    L.hs = H + 1;
    L.ps = hid + 1;
    uint32_t o = 0;
    L.whh = o; o += 3 * H * L.hs;
    L.wih = o; o += 3 * H * E;
    L.bih = o; o += 3 * H;
    L.bhh = o; o += 3 * H;
    L.w1 = o; o += hid * L.hs;
    L.b1 = o; o += hid;
    L.wh = o; o += (a.prober_layers - 1) * hid * L.ps;
    L.bh = o; o += (a.prober_layers - 1) * hid;
    L.wo = o; o += 15 * L.ps;
    L.bo = o; o += 16;
    L.score = o; o += kSmallWarps;
    L.w = o; o += kSmallWarps;
    L.total = o;
    return L;
}

template <int HS, int KT>
__global__ void __launch_bounds__(256) skyjepa_small_inputs_kernel(SkyjepaArgs a, const float* cand, float* xout) {
    extern __shared__ float scratch[];
    const TcnView& tcn = a.action_tcn;
    const uint32_t Hs = a.Hs, T = a.T, A = a.A, E = a.E, TA = T * A;
    const uint32_t ca = pow2_at_least(tcn.max_ch), Cm = ca;
    const uint32_t wpb = blockDim.x / ca;
    const uint32_t slot = threadIdx.x / ca, o = threadIdx.x % ca;
    const uint64_t windows = static_cast<uint64_t>(a.B) * a.S * T;
    const uint64_t win = static_cast<uint64_t>(blockIdx.x) * wpb + slot;
    const bool active = win < windows;
    const uint64_t grow = active ? win / T : 0;  // b * S + s
    const uint32_t t0 = active ? static_cast<uint32_t>(win % T) : 0;
    const uint32_t b = static_cast<uint32_t>(grow / a.S);
    float* cur = scratch + slot * 3 * Cm * Hs;
    float* hb = cur + Cm * Hs;
    for (uint32_t q = o; q < Cm * Hs; q += ca) cur[q] = 0.0f;
    __syncwarp();
    if (active && o < tcn.input_dim) {
        for (uint32_t w = 0; w < Hs; ++w) {
            const uint32_t pos = t0 + w;
            const float v = pos < Hs - 1 ? a.action_hist[(static_cast<size_t>(b) * (Hs - 1) + pos) * A + o]
                                         : cand[grow * TA + (pos - (Hs - 1)) * A + o];
            cur[o * Hs + w] = (v - a.action_mean[o]) / a.action_std[o];
        }
    }
    __syncwarp();
    action_tcn_window<HS, KT>(tcn, tcn.blocks[0].w1, cur, hb, Hs, o, active);
    if (active && o < E) xout[win * E + o] = cur[o * Hs + Hs - 1];
}

__global__ void __launch_bounds__(kSmallThreads) skyjepa_small_kernel(SkyjepaArgs a, const float* h0, const float* xin,
                                                                    const float* cand) {
    extern __shared__ __align__(16) float smem[];
    const SmallSmem L = small_layout(a);
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t H = a.H, E = a.E, hid = a.hid, T = a.T, A = a.A, TA = T * A;
    const uint32_t b = blockIdx.y, s0 = blockIdx.x * kSmallWarps, s = s0 + warp;
    // ---- weights into shared memory (padded rows: lane j reads row j conflict-free)
    for (uint32_t q = tid; q < 3 * H * H; q += kSmallThreads) smem[L.whh + (q / H) * L.hs + q % H] = __ldg(a.w_hh + q);
    for (uint32_t q = tid; q < 3 * H * E; q += kSmallThreads) smem[L.wih + q] = __ldg(a.w_ih + q);
    for (uint32_t q = tid; q < 3 * H; q += kSmallThreads) {
        smem[L.bih + q] = __ldg(a.b_ih + q);
        smem[L.bhh + q] = __ldg(a.b_hh + q);
    }
    for (uint32_t q = tid; q < hid * H; q += kSmallThreads) smem[L.w1 + (q / H) * L.hs + q % H] = __ldg(a.p_in_w + q);
    for (uint32_t q = tid; q < hid; q += kSmallThreads) smem[L.b1 + q] = __ldg(a.p_in_b + q);
    for (uint32_t l = 0; l + 1 < a.prober_layers; ++l) {
        for (uint32_t q = tid; q < hid * hid; q += kSmallThreads)
            smem[L.wh + l * hid * L.ps + (q / hid) * L.ps + q % hid] = __ldg(a.p_hid_w[l] + q);
        for (uint32_t q = tid; q < hid; q += kSmallThreads) smem[L.bh + l * hid + q] = __ldg(a.p_hid_b[l] + q);
    }
    for (uint32_t q = tid; q < 15 * hid; q += kSmallThreads) smem[L.wo + (q / hid) * L.ps + q % hid] = __ldg(a.p_out_w + q);
    for (uint32_t q = tid; q < 15; q += kSmallThreads) smem[L.bo + q] = __ldg(a.p_out_b + q);
    __syncthreads();

    const bool active = s < a.S;
    if (active) {
        const size_t grow = static_cast<size_t>(b) * a.S + s;
        const uint32_t u0 = lane, u1 = lane + 32;
        const bool has0 = u0 < H, has1 = u1 < H;
        float hA = has0 ? h0[static_cast<size_t>(b) * H + u0] : 0.0f;
        float hB = has1 ? h0[static_cast<size_t>(b) * H + u1] : 0.0f;
        float x[18];
#pragma unroll
        for (int i = 0; i < 18; ++i) x[i] = a.state_hist[(static_cast<size_t>(b) * a.Hs + a.Hs - 1) * 18 + i];
        float cost = 0.0f;
        for (uint32_t t = 0; t < T; ++t) {
            float xe[kMaxTcnCh];
#pragma unroll
            for (int e = 0; e < kMaxTcnCh; ++e) xe[e] = static_cast<uint32_t>(e) < E ? xin[(grow * T + t) * E + e] : 0.0f;
            // candle GRU step (gates r, z, n; h' = z h + (1 - z) n) for units u0, u1
            float gh[2][3] = {{0.f, 0.f, 0.f}, {0.f, 0.f, 0.f}};
            const float* r0 = smem + L.whh + u0 * L.hs;
            const float* r1 = smem + L.whh + (has1 ? u1 : 0) * L.hs;
            for (uint32_t k = 0; k < H; ++k) {
                const float hk = __shfl_sync(0xffffffffu, k < 32 ? hA : hB, k & 31);
                if (has0) {
#pragma unroll
                    for (int g = 0; g < 3; ++g) gh[0][g] = fmaf(r0[g * H * L.hs + k], hk, gh[0][g]);
                }
                if (has1) {
#pragma unroll
                    for (int g = 0; g < 3; ++g) gh[1][g] = fmaf(r1[g * H * L.hs + k], hk, gh[1][g]);
                }
            }
            float hn[2] = {0.0f, 0.0f};
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const uint32_t u = q == 0 ? u0 : u1;
                if (u >= H) continue;
                float gi[3];
#pragma unroll
                for (int g = 0; g < 3; ++g) {
                    const float* wi = smem + L.wih + (g * H + u) * E;
                    float acc = 0.0f;
#pragma unroll
                    for (int e = 0; e < kMaxTcnCh; ++e)
                        if (static_cast<uint32_t>(e) < E) acc = fmaf(xe[e], wi[e], acc);
                    gi[g] = acc + smem[L.bih + g * H + u];
                }
                const float rg = sigmoid(gi[0] + (gh[q][0] + smem[L.bhh + u]));
                const float zg = sigmoid(gi[1] + (gh[q][1] + smem[L.bhh + H + u]));
                const float ng = tanhf(gi[2] + rg * (gh[q][2] + smem[L.bhh + 2 * H + u]));
                const float hp = q == 0 ? hA : hB;
                hn[q] = zg * hp - (zg - 1.0f) * ng;
            }
            hA = hn[0];
            hB = hn[1];
            // SkyJepaProber::forward (prober.rs:84-102): lane o owns outputs o, o + 32
            float p0 = 0.0f, p1 = 0.0f;
            {
                const bool o0 = lane < hid, o1 = lane + 32 < hid;
                const float* w0 = smem + L.w1 + lane * L.hs;
                const float* w1 = smem + L.w1 + (o1 ? lane + 32 : 0) * L.hs;
                float s0 = 0.0f, s1 = 0.0f;
                for (uint32_t k = 0; k < H; ++k) {
                    const float hk = __shfl_sync(0xffffffffu, k < 32 ? hA : hB, k & 31);
                    if (o0) s0 = fmaf(w0[k], hk, s0);
                    if (o1) s1 = fmaf(w1[k], hk, s1);
                }
                p0 = o0 ? gelu_tanh(s0 + smem[L.b1 + lane]) : 0.0f;
                p1 = o1 ? gelu_tanh(s1 + smem[L.b1 + lane + 32]) : 0.0f;
            }
            for (uint32_t l = 0; l + 1 < a.prober_layers; ++l) {
                const bool o0 = lane < hid, o1 = lane + 32 < hid;
                const float* w0 = smem + L.wh + l * hid * L.ps + lane * L.ps;
                const float* w1 = smem + L.wh + l * hid * L.ps + (o1 ? lane + 32 : 0) * L.ps;
                float s0 = 0.0f, s1 = 0.0f;
                for (uint32_t k = 0; k < hid; ++k) {
                    const float ak = __shfl_sync(0xffffffffu, k < 32 ? p0 : p1, k & 31);
                    if (o0) s0 = fmaf(w0[k], ak, s0);
                    if (o1) s1 = fmaf(w1[k], ak, s1);
                }
                p0 = o0 ? gelu_tanh(s0 + smem[L.bh + l * hid + lane]) : 0.0f;
                p1 = o1 ? gelu_tanh(s1 + smem[L.bh + l * hid + lane + 32]) : 0.0f;
            }
            float out = 0.0f;
            {
                const float* w0 = smem + L.wo + (lane < 15 ? lane : 0) * L.ps;
                float s0 = 0.0f;
                for (uint32_t k = 0; k < hid; ++k) {
                    const float ak = __shfl_sync(0xffffffffu, k < 32 ? p0 : p1, k & 31);
                    s0 = fmaf(w0[k], ak, s0);
                }
                out = s0 + smem[L.bo + (lane < 15 ? lane : 0)];
            }
            float po[16];
#pragma unroll
            for (int i = 0; i < 15; ++i) po[i] = __shfl_sync(0xffffffffu, out, i);
            float act[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) act[i] = cand[(grow * T + t) * A + i];
            // every lane integrates alike; lane 0 alone writes predicted states
            cost += integrate_and_cost(a, b, s, t, x, act, po, lane == 0);
        }
        const float score = cost * static_cast<float>(1.0 / static_cast<double>(T));
        if (lane == 0) {
            smem[L.score + warp] = score;
            a.scores[static_cast<size_t>(b) * a.S + s] = score;
        }
    }
    __syncthreads();
    if (a.mppi) {
        const uint32_t nvalid = s0 >= a.S ? 0u : min(kSmallWarps, a.S - s0);
        mppi_reduce_rows<kSmallThreads>(a.m, b, blockIdx.x, nvalid, smem + L.score, s0,
                                        cand + (static_cast<size_t>(b) * a.S + s0) * TA, TA, smem + L.w);
    }
}

// ------------------------------------------------------------------ host side


template <int H>
static int max_active_clusters(size_t smem) {
    static int cached[2] = {-1, -1};
    static size_t cached_smem[2] = {0, 0};
    const int slot = H == 256 ? 0 : 1;
    if (cached[slot] >= 0 && cached_smem[slot] == smem) return cached[slot];
    if (cudaFuncSetAttribute(skyjepa_rollout_kernel<H>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kCluster, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, skyjepa_rollout_kernel<H>, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        n = 0;
    }
    cached[slot] = n;
    cached_smem[slot] = smem;
    return n;
}

// Rows per cluster: the smallest multiple of 8 (>= 32) whose grid fits in one
// wave of co-resident clusters; 32 when even 64 rows would not fit (large
// fleets run as several waves).
uint32_t skyjepa_rows_per_cluster(const SkyjepaArgs& a) {
    const uint32_t R = a.H == 256 ? Geom<256>::R : Geom<128>::R;
    SkySmem big = layout_for(a, kMaxRowsPerCta * kCluster);
    const size_t smem = big.total * sizeof(float);
    const int maxc = a.H == 256 ? max_active_clusters<256>(smem) : max_active_clusters<128>(smem);
    for (uint32_t rows = 32; rows <= kMaxRowsPerCta * kCluster; rows += 8) {
        if (rows % R != 0) continue;
        const uint64_t clusters = static_cast<uint64_t>(a.B) * ((a.S + rows - 1) / rows);
        if (maxc > 0 && clusters <= static_cast<uint64_t>(maxc)) return rows;
    }
    return 32;
}

uint32_t skyjepa_partials_per_vehicle(uint32_t S, uint32_t rows) {
    return ((S + rows - 1) / rows) * kCluster;
}

bool skyjepa_supported(const SkyjepaArgs& a, const char** why) {
    if (a.H != 256 && a.H != 128) { *why = "latent_dim must be 128 or 256 on the fused path"; return false; }
    if (a.A != 4) { *why = "action_dim must be 4"; return false; }
    if (a.E > kMaxTcnCh || a.action_tcn.max_ch > kMaxTcnCh) { *why = "action encoder channels must be <= 8"; return false; }
    if (a.Hs > kMaxHist || a.Hs < 2) { *why = "history_steps must be in [2, 16]"; return false; }
    if (a.hid % 4 != 0 || a.hid > kMaxHid || a.hid == 0) { *why = "prober hidden_dim must be a multiple of 4 and <= 64"; return false; }
    if (a.prober_layers < 1 || a.prober_layers > 5) { *why = "prober hidden_layers must be in [1, 5]"; return false; }
    if (a.T == 0 || a.T > kMaxHorizon) { *why = "horizon must be in [1, 64]"; return false; }
    if (a.state_tcn.max_ch > 256) { *why = "state encoder channels must be <= 256"; return false; }
    const SkySmem L = layout_for(a, kMaxRowsPerCta * kCluster);
    if (L.total * sizeof(float) > 220 * 1024) { *why = "shared memory budget exceeded"; return false; }
    return true;
}

template <int H>
static cudaError_t launch_rollout(const SkyjepaArgs& a, cudaStream_t stream) {
    const SkySmem L = layout_for(a, a.rows);
    const size_t smem = L.total * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(skyjepa_rollout_kernel<H>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(((a.S + a.rows - 1) / a.rows) * kCluster, a.B, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attrs[1];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = kCluster;
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, skyjepa_rollout_kernel<H>, a);
}

bool skyjepa_small_supported(const SkyjepaArgs& a, const char** why) {
    if (a.H == 0 || a.H > kSmallMaxH) { *why = "latent_dim must be <= 64 on the small-latent path"; return false; }
    if (a.A != 4) { *why = "action_dim must be 4"; return false; }
    if (a.E > kMaxTcnCh || a.action_tcn.max_ch > kMaxTcnCh) { *why = "action encoder channels must be <= 8"; return false; }
    if (a.Hs > kMaxHist || a.Hs < 2) { *why = "history_steps must be in [2, 16]"; return false; }
    if (a.hid == 0 || a.hid > 64) { *why = "prober hidden_dim must be in [1, 64]"; return false; }
    if (a.prober_layers < 1 || a.prober_layers > 5) { *why = "prober hidden_layers must be in [1, 5]"; return false; }
    if (a.T == 0 || a.T > kMaxHorizon) { *why = "horizon must be in [1, 64]"; return false; }
    if (static_cast<size_t>(a.state_tcn.max_ch) * a.Hs * 3 * sizeof(float) > 48 * 1024) {
        *why = "state encoder too wide for the history kernel";
        return false;
    }
    if (small_layout(a).total * sizeof(float) > 200 * 1024) { *why = "shared memory budget exceeded"; return false; }
    return true;
}

uint32_t skyjepa_small_partials_per_vehicle(uint32_t S) { return (S + kSmallWarps - 1) / kSmallWarps; }

size_t skyjepa_small_x_bytes(const SkyjepaArgs& a, uint32_t B, uint32_t S, uint32_t T) {
    return static_cast<size_t>(B) * S * T * a.E * sizeof(float);
}

cudaError_t launch_skyjepa_small(const SkyjepaArgs& a, float* h0, float* x, cudaStream_t stream, int* launches,
                                 const SideStream* side) {
    int n = 0;
    cudaError_t e;
    // initial latent per vehicle, independent of the candidates (side stream when given)
    if ((e = fork_h0(a, h0, stream, side)) != cudaSuccess) return e;
    ++n;
    if (a.sample) {
        // candidates (sample_kernel: Philox or injected noise, mean slot, clamp)
        SampleArgs sa{};
        sa.B = a.B; sa.S = a.S; sa.T = a.T; sa.A = a.A;
        sa.mean = a.mean;
        sa.std = a.std;
        sa.low = a.low_dev;
        sa.high = a.high_dev;
        sa.noise = a.noise;
        sa.seed = a.seed;
        sa.offset = a.offset;
        sa.sample_base = a.sample_base;
        sa.sample_total = a.sample_total;
        sa.out = a.cand_out;
        if ((e = launch_sample(sa, stream)) != cudaSuccess) return e;
        ++n;
    }
    const float* cand = a.sample ? a.cand_out : a.cand_in;
    // per-step inputs of every candidate
    const uint32_t ca = pow2_at_least(a.action_tcn.max_ch), wpb = 256 / ca;
    const uint64_t windows = static_cast<uint64_t>(a.B) * a.S * a.T;
    const uint32_t blocks = static_cast<uint32_t>((windows + wpb - 1) / wpb);
    const size_t in_smem = static_cast<size_t>(wpb) * 3 * ca * a.Hs * sizeof(float);
    if (a.Hs == 10 && a.action_tcn.k == 3)
        skyjepa_small_inputs_kernel<10, 3><<<blocks, wpb * ca, in_smem, stream>>>(a, cand, x);
    else
        skyjepa_small_inputs_kernel<0, 0><<<blocks, wpb * ca, in_smem, stream>>>(a, cand, x);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    ++n;
    if ((e = join_h0(stream, side)) != cudaSuccess) return e;
    // rollout, cost, MPPI partials
    const size_t smem = small_layout(a).total * sizeof(float);
    if ((e = cudaFuncSetAttribute(skyjepa_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(smem))) != cudaSuccess)
        return e;
    skyjepa_small_kernel<<<dim3(skyjepa_small_partials_per_vehicle(a.S), a.B), kSmallThreads, smem, stream>>>(a, h0, x,
                                                                                                          cand);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    ++n;
    if (launches) *launches = n;
    return cudaSuccess;
}

cudaError_t launch_skyjepa(const SkyjepaArgs& a, cudaStream_t stream, int* launches) {
    if (a.rows % kCluster != 0 || a.rows < 32 || a.rows > kMaxRowsPerCta * kCluster) return cudaErrorInvalidValue;
    if (a.time_begin) cudaEventRecord(a.time_begin, stream);
    const cudaError_t e = (a.H == 256) ? launch_rollout<256>(a, stream) : launch_rollout<128>(a, stream);
    if (a.time_end) cudaEventRecord(a.time_end, stream);
    if (launches) *launches = 1;
    return e;
}

}  // namespace lwm
