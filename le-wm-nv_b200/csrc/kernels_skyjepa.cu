// kernels_skyjepa.cu — SkyJEPA learned candidate scorer, fused with MPPI.
//
// Reference path (src/models/skyjepa/control.rs:246-317 -> model.rs:161-223
// -> tcn.rs, prober.rs:84-138, kinematics.rs:377-484 -> control.rs:430-452):
//   normalise actions; action TCN on every rolling window of
//   [history(H-1) ++ candidates]; state TCN + projection -> h0; T GRU steps;
//   prober MLP -> residual accel + angular map; explicit-Euler SO(3)
//   integrator; tracking cost averaged over the horizon.
//
// B200 mapping.  Two kernels per plan:
//  * skyjepa_context_kernel — one 8-CTA cluster per vehicle computes the
//    state-history TCN and projection (h0).  It triggers programmatic launch
//    completion at entry so the rollout kernel's prologue overlaps it.
//  * skyjepa_rollout_kernel — one 8-CTA cluster per 32 candidates.  CTA c of
//    the cluster owns hidden units [c*H/8, (c+1)*H/8): its slice of W_hh (all
//    three gates, all k) lives in REGISTERS for the whole kernel (96 floats a
//    thread at H = 256), so the recurrent GEMM reads only h from shared
//    memory.  Every step each CTA computes its units' new hidden values for
//    all 32 rows and writes them into every CTA's next-h buffer through
//    distributed shared memory, then the cluster barrier publishes them.
//    Each CTA also owns 4 of the 32 rows for sampling, the action TCN, the
//    prober, the integrator and the cost; the MPPI tuple of its rows feeds
//    the one-pass reduction (lwm_mppi.cuh).
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

namespace cg = cooperative_groups;

namespace lwm {

constexpr int kCluster = 8;
constexpr int kRows = 32;          // candidate rows per cluster
constexpr int kThreads = 256;
constexpr int kRowsPerCta = kRows / kCluster;
constexpr int kMaxTcnCh = 8;       // action-encoder channel bound
constexpr int kMaxHist = 16;

template <int H>
struct Geom {
    static constexpr int U = H / kCluster;      // hidden units per CTA
    static constexpr int PAIRS = U / 2;         // unit pairs per CTA
    static constexpr int KG = kThreads / PAIRS; // k-groups (lanes per pair)
    static constexpr int KPT = H / KG;          // k values per thread
    static constexpr int KQ = KPT / 4;          // float4 loads per row
    static constexpr int R = KG / 2;            // rows per GEMM group
    static constexpr int GROUPS = kRows / R;
    static constexpr int PPW = 32 / KG;         // pairs per warp
    static constexpr int VEC = 2 * PPW;         // hidden units per warp
    static constexpr int LPR = 32 / R;          // lanes per row in the store
    static constexpr int DPL = kCluster / LPR;  // destination CTAs per lane
    static_assert(KPT % 4 == 0, "k interleave needs float4 granularity");
    static_assert(KG <= 32 && KG >= 2, "k-groups must fit a warp");
    static_assert(kRows % R == 0, "row groups");
};

struct SkySmem {
    // Offsets in floats inside the dynamic shared-memory block.
    uint32_t h0, h1, emb, cand, tcn, w1, wih, a1, a2, out, x, score, w, total;
};

__host__ __device__ inline SkySmem sky_smem_layout(uint32_t H, uint32_t T, uint32_t E, uint32_t A, uint32_t hid,
                                                   uint32_t tcn_ch, uint32_t Hs) {
    SkySmem s;
    uint32_t off = 0;
    auto take = [&](uint32_t n) { uint32_t o = off; off += (n + 3u) & ~3u; return o; };
    s.h0 = take(kRows * H);
    s.h1 = take(kRows * H);
    s.emb = take(kRows * T * E);
    s.cand = take(kRowsPerCta * T * A);
    const uint32_t windows = kRowsPerCta * T;
    s.tcn = take(windows * 3 * tcn_ch * Hs);
    s.w1 = take(hid * H);
    s.wih = take(3 * (H / kCluster) * E);
    s.a1 = take(kRowsPerCta * hid);
    s.a2 = take(kRowsPerCta * hid);
    s.out = take(kRowsPerCta * 16);
    s.x = take(kRowsPerCta * 20);
    s.score = take(kRowsPerCta);
    s.w = take(kRowsPerCta);
    s.total = off;
    return s;
}

// ------------------------------------------------------------ context kernel
//
// SkyJepaModel::encode_state_history (model.rs:57-61): normalised state
// history -> TemporalConvEncoder::forward_last (tcn.rs:155-160) ->
// state_projection.  Cluster of 8 CTAs per vehicle; CTA c computes output
// channels [c*C/8, (c+1)*C/8) of every convolution and broadcasts them.
__device__ __forceinline__ float conv_at(const float* x, uint32_t in, uint32_t Hs, const float* w,
                                         uint32_t o, uint32_t K, uint32_t dil, uint32_t t) {
    float acc = 0.0f;
    for (uint32_t i = 0; i < in; ++i) {
        const float* wr = w + (static_cast<size_t>(o) * in + i) * K;
        const float* xr = x + i * Hs;
        for (uint32_t j = 0; j < K; ++j) {
            const int src = static_cast<int>(t) - static_cast<int>((K - 1 - j) * dil);
            if (src >= 0) acc = fmaf(__ldg(wr + j), xr[src], acc);
        }
    }
    return acc;
}

__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads)
skyjepa_context_kernel(SkyjepaArgs a) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 900)
    cudaTriggerProgrammaticLaunchCompletion();
#endif
    extern __shared__ float smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t c = cluster.block_rank();
    const uint32_t b = blockIdx.y;
    const TcnView& tcn = a.state_tcn;
    const uint32_t Hs = a.Hs, C = tcn.max_ch;
    float* xa = smem;
    float* xb = smem + C * Hs;
    float* h1 = smem + 2 * C * Hs;
    // normalised state history, [channel][time]
    for (uint32_t q = threadIdx.x; q < tcn.input_dim * Hs; q += blockDim.x) {
        const uint32_t i = q / Hs, t = q % Hs;
        const float v = a.state_hist[(static_cast<size_t>(b) * Hs + t) * 18 + i];
        xa[q] = (v - a.state_mean[i]) / a.state_std[i];
    }
    cluster.sync();
    float* cur = xa;
    float* nxt = xb;
    for (uint32_t l = 0; l < tcn.levels; ++l) {
        const TcnBlockView& bk = tcn.blocks[l];
        const uint32_t per = (bk.out + kCluster - 1) / kCluster;
        const uint32_t o0 = c * per, o1 = min(bk.out, o0 + per);
        const uint32_t n_out = (o1 > o0 ? o1 - o0 : 0) * Hs;
        for (uint32_t q = threadIdx.x; q < n_out; q += blockDim.x) {
            const uint32_t o = o0 + q / Hs, t = q % Hs;
            const float v = gelu_tanh(conv_at(cur, bk.in, Hs, bk.w1, o, tcn.k, bk.dil, t) + __ldg(bk.b1 + o));
            for (uint32_t d = 0; d < kCluster; ++d) cluster.map_shared_rank(h1, d)[o * Hs + t] = v;
        }
        cluster.sync();
        for (uint32_t q = threadIdx.x; q < n_out; q += blockDim.x) {
            const uint32_t o = o0 + q / Hs, t = q % Hs;
            const float h2 = gelu_tanh(conv_at(h1, bk.out, Hs, bk.w2, o, tcn.k, bk.dil, t) + __ldg(bk.b2 + o));
            float res;
            if (bk.wr) res = conv_at(cur, bk.in, Hs, bk.wr, o, 1, 1, t) + __ldg(bk.br + o);
            else res = cur[o * Hs + t];
            const float v = gelu_tanh(h2 + res);
            for (uint32_t d = 0; d < kCluster; ++d) cluster.map_shared_rank(nxt, d)[o * Hs + t] = v;
        }
        cluster.sync();
        float* tmp = cur; cur = nxt; nxt = tmp;
    }
    // state_projection on the last time step: CTA c writes H/8 outputs.
    const uint32_t per = (a.H + kCluster - 1) / kCluster;
    const uint32_t Cl = tcn.out_dim;
    for (uint32_t q = threadIdx.x; q < per; q += blockDim.x) {
        const uint32_t o = c * per + q;
        if (o >= a.H) break;
        float acc = 0.0f;
        for (uint32_t i = 0; i < Cl; ++i) acc = fmaf(cur[i * Hs + Hs - 1], __ldg(a.proj_w + static_cast<size_t>(o) * Cl + i), acc);
        a.h0[static_cast<size_t>(b) * a.H + o] = acc + __ldg(a.proj_b + o);
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
    const SkySmem L = sky_smem_layout(H, T, E, A, hid, a.action_tcn.max_ch, Hs);
    float* s_emb = smem + L.emb;     // [kRows][T][E]
    float* s_cand = smem + L.cand;   // [kRowsPerCta][T][A]
    float* s_tcn = smem + L.tcn;
    float* s_w1 = smem + L.w1;       // [hid][H]
    float* s_wih = smem + L.wih;     // [3][U][E] for this CTA's units
    float* s_a1 = smem + L.a1;
    float* s_a2 = smem + L.a2;
    float* s_out = smem + L.out;     // [kRowsPerCta][16]
    float* s_x = smem + L.x;         // [kRowsPerCta][20]: state18, running cost
    float* s_score = smem + L.score;
    float* s_w = smem + L.w;
    const uint32_t row0 = rb * kRows;              // first sample of the cluster
    const uint32_t own0 = row0 + c * kRowsPerCta;  // first sample this CTA owns
    const uint32_t TA = T * A;

    // ---- registers: this thread's W_hh slice (independent of the context)
    const uint32_t pl = lane / G::KG, kg = lane % G::KG;
    const uint32_t pair = warp * G::PPW + pl;
    float wr[2][3][G::KPT];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const uint32_t j = c * G::U + pair * 2 + q;
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
    // gate epilogue of this lane: combo kg = (unit-in-pair, row-in-group)
    const uint32_t my_q = kg / G::R, my_r = kg % G::R;
    const uint32_t my_local = pair * 2 + my_q;
    const uint32_t my_unit = c * G::U + my_local;
    float bih[3], bhh[3];
#pragma unroll
    for (int g = 0; g < 3; ++g) {
        bih[g] = __ldg(a.b_ih + g * H + my_unit);
        bhh[g] = __ldg(a.b_hh + g * H + my_unit);
    }
    // shared copies: prober layer-1 weight, W_ih rows of this CTA's units
    for (uint32_t q = tid; q < hid * H / 4; q += kThreads)
        reinterpret_cast<float4*>(s_w1)[q] = __ldg(reinterpret_cast<const float4*>(a.p_in_w) + q);
    for (uint32_t q = tid; q < 3 * G::U * E; q += kThreads) {
        const uint32_t g = q / (G::U * E), rem = q % (G::U * E), u = rem / E, e = rem % E;
        s_wih[q] = __ldg(a.w_ih + (static_cast<size_t>(g) * H + c * G::U + u) * E + e);
    }

    // ---- sampling of the CTA's own rows (as sample_kernel)
    for (uint32_t q = tid; q < kRowsPerCta * TA; q += kThreads) {
        const uint32_t rr = q / TA, e = q % TA, act = e % A;
        const uint32_t s = own0 + rr;
        const uint64_t ci = (static_cast<uint64_t>(b) * a.S + s) * TA + e;
        float v;
        if (a.sample) {
            const size_t mi = static_cast<size_t>(b) * TA + e;
            if (s == 0 || s >= a.S) {
                v = a.mean[mi];
            } else {
                const float eps = a.noise ? a.noise[ci] : normal_at(a.seed, a.offset + ci);
                v = a.mean[mi] + eps * a.std[mi];
            }
            v = cmin(cmax(v, a.low[act]), a.high[act]);
            if (a.cand_out && s < a.S) a.cand_out[ci] = v;
        } else {
            v = s < a.S ? a.cand_in[ci] : a.low[act];
        }
        s_cand[q] = v;
    }
    if (tid < kRowsPerCta) {
        for (int i = 0; i < 18; ++i) s_x[tid * 20 + i] = a.state_hist[(static_cast<size_t>(b) * Hs + Hs - 1) * 18 + i];
        s_x[tid * 20 + 18] = 0.0f;
    }
    // every CTA of the cluster must be running before any DSMEM access
    cluster.sync();

    // ---- action TCN over the rolling windows of the own rows
    {
        const TcnView& tcn = a.action_tcn;
        const uint32_t Cm = tcn.max_ch;
        const uint32_t wpp = kThreads / Cm;           // windows per pass
        const uint32_t slot = tid / Cm, ch = tid % Cm;
        const uint32_t windows = kRowsPerCta * T;
        for (uint32_t w0 = 0; w0 < windows; w0 += wpp) {
            const uint32_t win = w0 + slot;
            const bool active = slot < wpp && win < windows;
            float* cur = s_tcn + (active ? slot : 0) * 3 * Cm * Hs;
            float* h1 = cur + Cm * Hs;
            float* h2 = h1 + Cm * Hs;
            const uint32_t rr = active ? win / T : 0, t0 = active ? win % T : 0;
            if (active && ch < tcn.input_dim) {
                for (uint32_t w = 0; w < Hs; ++w) {
                    const uint32_t pos = t0 + w;
                    float v;
                    if (pos < Hs - 1) v = a.action_hist[(static_cast<size_t>(b) * (Hs - 1) + pos) * A + ch];
                    else v = s_cand[rr * TA + (pos - (Hs - 1)) * A + ch];
                    cur[ch * Hs + w] = (v - a.action_mean[ch]) / a.action_std[ch];
                }
            }
            __syncthreads();
            for (uint32_t l = 0; l < tcn.levels; ++l) {
                const TcnBlockView& bk = tcn.blocks[l];
                const bool mine = active && ch < bk.out;
                if (mine)
                    for (uint32_t t = 0; t < Hs; ++t)
                        h1[ch * Hs + t] = gelu_tanh(conv_at(cur, bk.in, Hs, bk.w1, ch, tcn.k, bk.dil, t) + __ldg(bk.b1 + ch));
                __syncthreads();
                if (mine)
                    for (uint32_t t = 0; t < Hs; ++t)
                        h2[ch * Hs + t] = gelu_tanh(conv_at(h1, bk.out, Hs, bk.w2, ch, tcn.k, bk.dil, t) + __ldg(bk.b2 + ch));
                __syncthreads();
                if (mine)
                    for (uint32_t t = 0; t < Hs; ++t) {
                        float res;
                        if (bk.wr) res = conv_at(cur, bk.in, Hs, bk.wr, ch, 1, 1, t) + __ldg(bk.br + ch);
                        else res = cur[ch * Hs + t];
                        h1[ch * Hs + t] = gelu_tanh(h2[ch * Hs + t] + res);
                    }
                __syncthreads();
                if (mine)
                    for (uint32_t t = 0; t < Hs; ++t) cur[ch * Hs + t] = h1[ch * Hs + t];
                __syncthreads();
            }
            if (active && ch < E) {
                const float v = cur[ch * Hs + Hs - 1];
                const uint32_t m = c * kRowsPerCta + rr;
                for (uint32_t d = 0; d < kCluster; ++d)
                    cluster.map_shared_rank(s_emb, d)[(m * T + t0) * E + ch] = v;
            }
            __syncthreads();
        }
    }
    cluster.sync();  // every CTA now holds all 32 rows' window embeddings

    // ---- wait for h0 from the context kernel, broadcast it to all rows
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 900)
    if (a.use_pdl) cudaGridDependencySynchronize();
#endif
    {
        const float4* src = reinterpret_cast<const float4*>(a.h0 + static_cast<size_t>(b) * H);
        float4* dst = reinterpret_cast<float4*>(smem + L.h0);
        for (uint32_t q = tid; q < kRows * H / 4; q += kThreads) dst[q] = src[q % (H / 4)];
    }
    __syncthreads();

    constexpr int KR4 = H / 128;  // float4 per lane in prober layer 1
    const uint32_t opw = hid / 8;
    for (uint32_t t = 0; t < T; ++t) {
        const float* hc = smem + ((t & 1) ? L.h1 : L.h0);
        float* hn = smem + ((t & 1) ? L.h0 : L.h1);
        // ---- recurrent GEMM + GRU gates for this CTA's hidden units
#pragma unroll 1
        for (int grp = 0; grp < G::GROUPS; ++grp) {
            float acc[2 * G::R][3];
#pragma unroll
            for (int q = 0; q < 2 * G::R; ++q) { acc[q][0] = 0.0f; acc[q][1] = 0.0f; acc[q][2] = 0.0f; }
#pragma unroll
            for (int r = 0; r < G::R; ++r) {
                const float* hrow = hc + (grp * G::R + r) * H + kg * 4;
#pragma unroll
                for (int i = 0; i < G::KQ; ++i) {
                    const float4 hv = *reinterpret_cast<const float4*>(hrow + 4 * G::KG * i);
#pragma unroll
                    for (int q = 0; q < 2; ++q)
#pragma unroll
                        for (int g = 0; g < 3; ++g) {
                            float s = acc[q * G::R + r][g];
                            s = fmaf(wr[q][g][4 * i + 0], hv.x, s);
                            s = fmaf(wr[q][g][4 * i + 1], hv.y, s);
                            s = fmaf(wr[q][g][4 * i + 2], hv.z, s);
                            s = fmaf(wr[q][g][4 * i + 3], hv.w, s);
                            acc[q * G::R + r][g] = s;
                        }
                }
            }
            // reduce-scatter over the KG lanes of the pair: lane kg ends with combo kg
#pragma unroll
            for (int m = G::KG / 2; m >= 1; m >>= 1) {
                const bool upper = (kg & m) != 0;
#pragma unroll
                for (int cc = 0; cc < m; ++cc)
#pragma unroll
                    for (int g = 0; g < 3; ++g) {
                        const float send = upper ? acc[cc][g] : acc[cc + m][g];
                        const float keep = upper ? acc[cc + m][g] : acc[cc][g];
                        acc[cc][g] = keep + __shfl_xor_sync(0xffffffffu, send, m);
                    }
            }
            // candle GRU step for (row mrow, unit my_unit)
            const uint32_t mrow = grp * G::R + my_r;
            const float* xe = s_emb + (mrow * T + t) * E;
            float gi[3];
#pragma unroll
            for (int g = 0; g < 3; ++g) {
                const float* wi = s_wih + (g * G::U + my_local) * E;
                float s = 0.0f;
                for (uint32_t e = 0; e < E; ++e) s = fmaf(xe[e], wi[e], s);
                gi[g] = s + bih[g];
            }
            const float ghr = acc[0][0] + bhh[0], ghz = acc[0][1] + bhh[1], ghn = acc[0][2] + bhh[2];
            const float rg = sigmoid(gi[0] + ghr);
            const float zg = sigmoid(gi[1] + ghz);
            const float ng = tanhf(gi[2] + rg * ghn);
            const float hp = hc[mrow * H + my_unit];
            const float hnew = zg * hp - (zg - 1.0f) * ng;
            // gather G::VEC consecutive units of one row, store to every CTA
            float vals[G::VEC];
#pragma unroll
            for (int v = 0; v < G::VEC; ++v) vals[v] = __shfl_sync(0xffffffffu, hnew, v * G::R + (lane % G::R));
            const uint32_t srow = grp * G::R + (lane % G::R);
            const uint32_t slot = lane / G::R;
            float* local = hn + srow * H + c * G::U + warp * G::VEC;
#pragma unroll
            for (int dd = 0; dd < G::DPL; ++dd) {
                float* dst = cluster.map_shared_rank(local, slot * G::DPL + dd);
                if constexpr (G::VEC == 4) {
                    *reinterpret_cast<float4*>(dst) = make_float4(vals[0], vals[1], vals[2], vals[3]);
                } else {
                    *reinterpret_cast<float2*>(dst) = make_float2(vals[0], vals[1]);
                }
            }
        }
        cluster.sync();  // h_{t+1} complete in every CTA

        // ---- prober layer 1 for the own rows: lane = k slice, warp = output group.
        // 32 (output, row) combos are reduce-scattered over the 32 lanes.
        {
            float v[32];
#pragma unroll
            for (int q = 0; q < 32; ++q) v[q] = 0.0f;
#pragma unroll
            for (int k4 = 0; k4 < KR4; ++k4) {
                const uint32_t k = lane * 4 + 128 * k4;
                float4 wv[8];
#pragma unroll
                for (int o = 0; o < 8; ++o)
                    wv[o] = (static_cast<uint32_t>(o) < opw) ? *reinterpret_cast<const float4*>(s_w1 + (warp * opw + o) * H + k)
                                                             : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
                for (int rr = 0; rr < kRowsPerCta; ++rr) {
                    const float4 hv = *reinterpret_cast<const float4*>(hn + (c * kRowsPerCta + rr) * H + k);
#pragma unroll
                    for (int o = 0; o < 8; ++o) {
                        float s = v[o * kRowsPerCta + rr];
                        s = fmaf(wv[o].x, hv.x, s);
                        s = fmaf(wv[o].y, hv.y, s);
                        s = fmaf(wv[o].z, hv.z, s);
                        s = fmaf(wv[o].w, hv.w, s);
                        v[o * kRowsPerCta + rr] = s;
                    }
                }
            }
#pragma unroll
            for (int m = 16; m >= 1; m >>= 1) {
                const bool upper = (lane & m) != 0;
#pragma unroll
                for (int cc = 0; cc < m; ++cc) {
                    const float send = upper ? v[cc] : v[cc + m];
                    const float keep = upper ? v[cc + m] : v[cc];
                    v[cc] = keep + __shfl_xor_sync(0xffffffffu, send, m);
                }
            }
            const uint32_t o = lane / kRowsPerCta, rr = lane % kRowsPerCta;
            if (o < opw) {
                const uint32_t oo = warp * opw + o;
                s_a1[rr * hid + oo] = gelu_tanh(v[0] + __ldg(a.p_in_b + oo));
            }
        }
        __syncthreads();
        // ---- hidden prober layers and output layer (small)
        float* pin = s_a1;
        float* pout = s_a2;
        for (uint32_t l = 0; l + 1 < a.prober_layers; ++l) {
            for (uint32_t q = tid; q < kRowsPerCta * hid; q += kThreads) {
                const uint32_t rr = q / hid, o = q % hid;
                const float* wrow = a.p_hid_w[l] + static_cast<size_t>(o) * hid;
                float s = 0.0f;
                for (uint32_t i = 0; i < hid; ++i) s = fmaf(pin[rr * hid + i], __ldg(wrow + i), s);
                pout[q] = gelu_tanh(s + __ldg(a.p_hid_b[l] + o));
            }
            __syncthreads();
            float* tmp = pin; pin = pout; pout = tmp;
        }
        for (uint32_t q = tid; q < kRowsPerCta * 15; q += kThreads) {
            const uint32_t rr = q / 15, o = q % 15;
            const float* wrow = a.p_out_w + static_cast<size_t>(o) * hid;
            float s = 0.0f;
            for (uint32_t i = 0; i < hid; ++i) s = fmaf(pin[rr * hid + i], __ldg(wrow + i), s);
            s_out[rr * 16 + o] = s + __ldg(a.p_out_b + o);
        }
        __syncthreads();
        // ---- integrator step (lewm_skyjepa_integrate_f32) + tracking cost
        if (tid < kRowsPerCta) {
            float x[18];
#pragma unroll
            for (int i = 0; i < 18; ++i) x[i] = s_x[tid * 20 + i];
            const float* act = s_cand + tid * TA + t * A;
            const float* po = s_out + tid * 16;
            const float sdt = a.dt;
            float ta;
            if (a.rotor_forces) {
                ta = (act[0] + act[1] + act[2] + act[3]) / a.mass;
            } else {
                const float th = fminf(1.0f, fmaxf(0.0f, act[2]));
                ta = th * a.gravity / a.hover_throttle;
            }
            const float acc[3] = {x[8] * ta + po[0], x[11] * ta + po[1], x[14] * ta - a.gravity + po[2]};
            float ang[3];
#pragma unroll
            for (int row = 0; row < 3; ++row)
                ang[row] = po[3 + row * 4] * act[0] + po[4 + row * 4] * act[1] + po[5 + row * 4] * act[2] +
                           po[6 + row * 4] * act[3];
#pragma unroll
            for (int ax = 0; ax < 3; ++ax) { x[ax] += x[3 + ax] * sdt; x[3 + ax] += acc[ax] * sdt; }
            const float wx = x[15] * sdt, wy = x[16] * sdt, wz = x[17] * sdt;
            const float th2 = wx * wx + wy * wy + wz * wz;
            float ca, cb;
            if (th2 < 1.0e-6f) {
                const float th4 = th2 * th2;
                ca = 1.0f - th2 / 6.0f + th4 / 120.0f;
                cb = 0.5f - th2 / 24.0f + th4 / 720.0f;
            } else {
                const float th = sqrtf(th2);
                float sn, cs;
                sincosf(th, &sn, &cs);
                ca = sn / th;
                cb = (1.0f - cs) / th2;
            }
            const float dl[9] = {1.0f - cb * (wy * wy + wz * wz), cb * wx * wy - ca * wz, cb * wx * wz + ca * wy,
                                 cb * wy * wx + ca * wz, 1.0f - cb * (wx * wx + wz * wz), cb * wy * wz - ca * wx,
                                 cb * wz * wx - ca * wy, cb * wz * wy + ca * wx, 1.0f - cb * (wx * wx + wy * wy)};
            float nr[9];
#pragma unroll
            for (int row = 0; row < 3; ++row)
#pragma unroll
                for (int col = 0; col < 3; ++col)
                    nr[row * 3 + col] = x[6 + row * 3] * dl[col] + x[7 + row * 3] * dl[3 + col] + x[8 + row * 3] * dl[6 + col];
#pragma unroll
            for (int i = 0; i < 9; ++i) x[6 + i] = nr[i];
#pragma unroll
            for (int ax = 0; ax < 3; ++ax) x[15 + ax] += ang[ax] * sdt;
            const uint32_t s = own0 + tid;
            if (a.states && s < a.S) {
                float* o = a.states + ((static_cast<size_t>(b) * a.S + s) * T + t) * 18;
#pragma unroll
                for (int i = 0; i < 18; ++i) o[i] = x[i];
            }
            const float* ref = a.ref_states + (static_cast<size_t>(b) * T + t) * 18;
            float g0 = 0.0f, g1 = 0.0f, g2 = 0.0f, g3 = 0.0f;
#pragma unroll
            for (int i = 0; i < 3; ++i) { const float dd = x[i] - ref[i]; g0 += dd * dd; }
#pragma unroll
            for (int i = 3; i < 6; ++i) { const float dd = x[i] - ref[i]; g1 += dd * dd; }
#pragma unroll
            for (int i = 6; i < 15; ++i) { const float dd = x[i] - ref[i]; g2 += dd * dd; }
#pragma unroll
            for (int i = 15; i < 18; ++i) { const float dd = x[i] - ref[i]; g3 += dd * dd; }
            const float* ra = a.ref_actions + (static_cast<size_t>(b) * T + t) * 4;
            float ac = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i) { const float dd = act[i] - ra[i]; ac += (dd * dd) * a.cost.action[i]; }
            float st = g0 * a.cost.position + g1 * a.cost.velocity;
            st = st + g2 * a.cost.attitude;
            st = st + g3 * a.cost.angular_velocity;
#pragma unroll
            for (int i = 0; i < 18; ++i) s_x[tid * 20 + i] = x[i];
            s_x[tid * 20 + 18] += st + ac;
        }
    }

    // ---- scores of the own rows, then the MPPI tuple
    if (tid < kRowsPerCta) {
        const float score = s_x[tid * 20 + 18] * static_cast<float>(1.0 / static_cast<double>(T));
        s_score[tid] = score;
        const uint32_t s = own0 + tid;
        if (s < a.S) a.scores[static_cast<size_t>(b) * a.S + s] = score;
    }
    __syncthreads();
    if (a.mppi) {
        const uint32_t nvalid = own0 >= a.S ? 0u : min(static_cast<uint32_t>(kRowsPerCta), a.S - own0);
        const uint32_t p = rb * kCluster + c;
        mppi_reduce_rows<kThreads>(a.m, b, p, nvalid, s_score, own0, s_cand, TA, s_w);
    }
}

// ------------------------------------------------------------------ host side

uint32_t skyjepa_partials_per_vehicle(uint32_t S, uint32_t /*H*/) {
    return ((S + kRows - 1) / kRows) * kCluster;
}

bool skyjepa_supported(const SkyjepaArgs& a, const char** why) {
    if (a.H != 256 && a.H != 128) { *why = "latent_dim must be 128 or 256 on the fused path"; return false; }
    if (a.A != 4) { *why = "action_dim must be 4"; return false; }
    if (a.E > kMaxTcnCh || a.action_tcn.max_ch > kMaxTcnCh) { *why = "action encoder channels must be <= 8"; return false; }
    if (a.Hs > kMaxHist || a.Hs < 2) { *why = "history_steps must be in [2, 16]"; return false; }
    if (a.hid % 8 != 0 || a.hid > 64 || a.hid == 0) { *why = "prober hidden_dim must be a multiple of 8 and <= 64"; return false; }
    if (a.prober_layers < 1 || a.prober_layers > 5) { *why = "prober hidden_layers must be in [1, 5]"; return false; }
    if (a.T == 0 || a.T > kMaxHorizon) { *why = "horizon must be in [1, 64]"; return false; }
    if (a.state_tcn.max_ch > 256) { *why = "state encoder channels must be <= 256"; return false; }
    const SkySmem L = sky_smem_layout(a.H, a.T, a.E, a.A, a.hid, a.action_tcn.max_ch, a.Hs);
    if (L.total * sizeof(float) > 200 * 1024) { *why = "shared memory budget exceeded"; return false; }
    return true;
}

template <int H>
static cudaError_t launch_rollout(const SkyjepaArgs& a, cudaStream_t stream) {
    const SkySmem L = sky_smem_layout(H, a.T, a.E, a.A, a.hid, a.action_tcn.max_ch, a.Hs);
    const size_t smem = L.total * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(skyjepa_rollout_kernel<H>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(((a.S + kRows - 1) / kRows) * kCluster, a.B, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = kCluster;
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = a.use_pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, skyjepa_rollout_kernel<H>, a);
}

cudaError_t launch_skyjepa(const SkyjepaArgs& a, cudaStream_t stream, int* launches) {
    const size_t ctx_smem = static_cast<size_t>(3) * a.state_tcn.max_ch * a.Hs * sizeof(float);
    if (ctx_smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(skyjepa_context_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(ctx_smem));
        if (e != cudaSuccess) return e;
    }
    skyjepa_context_kernel<<<dim3(kCluster, a.B, 1), kThreads, ctx_smem, stream>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    e = (a.H == 256) ? launch_rollout<256>(a, stream) : launch_rollout<128>(a, stream);
    if (launches) *launches = 2;
    return e;
}

}  // namespace lwm
