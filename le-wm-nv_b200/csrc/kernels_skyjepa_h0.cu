// kernels_skyjepa_h0.cu — the history encoder of the SkyJEPA scorer,
//   h0 = state_projection(TemporalConvEncoder::forward_last(normalised history))
// (SkyJepaModel::encode_state_history, model.rs:57-61; tcn.rs:88-96,
// 138-160), for the shape the default model has: 10 history steps, kernel 3,
// three levels of 128 channels with dilations 1, 2, 4 (a 1x1 residual
// projection on level 1 only), latent 256.  One 16-CTA cluster per vehicle.
//
// Only the last position of the encoder's output is used, so each
// convolution is evaluated only where that output depends on it (causal zero
// padding inside the window):
//   level 1: conv1 at all 10 positions, block output at the odd ones;
//   level 2: conv1 at the odd positions, block output at 1, 5, 9;
//   level 3: conv1 at 1, 5, 9, block output at 9;
// 27 position-convolutions instead of 60.
//
// CTA c owns output channels [8c, 8c + 8) of every convolution and outputs
// [16c, 16c + 16) of the projection; its weight rows (72 KB) are copied into
// shared memory once, at the start, with 16-byte cp.async.  In a stage, warp
// w computes channel 8c + w at the stage's positions: the lanes split the
// input channels, a butterfly reduction gives every lane all sums, lane k
// finishes position k (bias, GELU, residual) and writes it into this CTA's
// activation; after one cluster barrier every CTA pulls the peers' channels
// of that activation from their shared memory (distributed shared memory).
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <type_traits>

#include "lwm_device.cuh"
#include "lwm_kernels.hpp"

namespace lwm {

namespace {

constexpr uint32_t kCl = 16;     // CTAs per vehicle
// (the stages' exchange and the projection's split are written for 16 CTAs
// of 8 channels: another cluster size measured wrong costs, 4e-4 relative)
static_assert(kCl == 16, "the pruned history encoder is written for 16-CTA clusters");
constexpr uint32_t kC = 128;     // channels
constexpr uint32_t kIn = 18;     // state features
constexpr uint32_t kHs = 10;     // history window
constexpr uint32_t kLat = 256;   // latent
constexpr uint32_t kPer = kC / kCl;       // 8 output channels per CTA
constexpr uint32_t kProjPer = kLat / kCl; // 16 projection outputs per CTA
constexpr uint32_t kThreads = 32 * kPer;  // one warp per owned channel
constexpr uint32_t kXLd = 32;             // row stride of the normalised input [pos][feature]

// shared memory, in floats
constexpr uint32_t kW1a = kPer * kIn * 3;  // level 1 conv1 rows
constexpr uint32_t kW2 = kPer * kC * 3;    // a 128-input conv's rows
constexpr uint32_t kWr = kPer * kIn;       // level 1 residual rows
constexpr uint32_t kWp = kProjPer * kC;    // projection rows
constexpr uint32_t kOffW1a = 0, kOffW2a = kOffW1a + kW1a, kOffWr = kOffW2a + kW2, kOffW1b = kOffWr + kWr,
                   kOffW2b = kOffW1b + kW2, kOffW1c = kOffW2b + kW2, kOffW2c = kOffW1c + kW2,
                   kOffWp = kOffW2c + kW2, kWFloats = kOffWp + kWp;
constexpr uint32_t kAct = kHs * kC;
constexpr uint32_t kOffX = kWFloats, kOffH1 = kOffX + kHs * kXLd, kOffY1 = kOffH1 + kAct, kOffH2 = kOffY1 + kAct,
                   kOffY2 = kOffH2 + kAct, kOffH3 = kOffY2 + kAct, kOffY3 = kOffH3 + kAct,
                   kSmemFloats = kOffY3 + kAct;
static_assert(kW1a % 4 == 0 && kW2 % 4 == 0 && kWr % 4 == 0 && kWp % 4 == 0, "16-byte weight chunks");

__device__ __forceinline__ uint32_t cta_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_barrier() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Every peer d's channels [8 d, 8 d + 8) of the activation at float offset
// `off` ([pos][128]), at positions P0 + k PSTEP (k < NP), into this CTA's
// copy: 16-byte loads from the peers' shared memory (each CTA writes only
// its own channels; after the cluster barrier every CTA pulls the rest).
template <int NP, int P0, int PSTEP>
__device__ __forceinline__ void pull(float* sm, uint32_t off, uint32_t c, uint32_t tid) {
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(sm));
    for (uint32_t q = tid; q < kCl * NP * 2; q += kThreads) {
        const uint32_t d = q / (NP * 2), k = (q / 2) % NP, h = q % 2;
        if (d == c) continue;
        const uint32_t e = off + (P0 + k * PSTEP) * kC + d * kPer + h * 4;
        uint32_t r;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(sbase + e * 4u), "r"(d));
        float4 v;
        asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                     : "r"(r)
                     : "memory");
        *reinterpret_cast<float4*>(sm + e) = v;
    }
}
// n floats (a multiple of 4, both addresses 16-byte aligned) global -> shared
__device__ __forceinline__ void copy16(float* dst, const float* src, uint32_t n) {
    for (uint32_t q = threadIdx.x * 4; q < n; q += kThreads * 4) {
        const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst + q));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src + q) : "memory");
    }
}

// Sums over input channels and taps of one output row `w` ([CIN][3]) at the
// positions P0 + k * PSTEP (k < NP) with dilation DIL, over the activation
// `in` ([pos][ld]); every lane returns all NP sums.
template <uint32_t CIN, int NP, int P0, int PSTEP, int DIL>
__device__ __forceinline__ void conv_sums(const float* w, const float* in, uint32_t ld, uint32_t lane,
                                          float (&acc)[NP]) {
#pragma unroll
    for (int k = 0; k < NP; ++k) acc[k] = 0.0f;
#pragma unroll
    for (uint32_t i0 = 0; i0 < CIN; i0 += 32) {
        const uint32_t i = i0 + lane;
        if (CIN % 32 == 0 || i < CIN) {
            const float w0 = w[i * 3], w1 = w[i * 3 + 1], w2 = w[i * 3 + 2];
#pragma unroll
            for (int k = 0; k < NP; ++k) {
                const int p = P0 + k * PSTEP;
                if (p - 2 * DIL >= 0) acc[k] = fmaf(w0, in[(p - 2 * DIL) * ld + i], acc[k]);
                if (p - DIL >= 0) acc[k] = fmaf(w1, in[(p - DIL) * ld + i], acc[k]);
                acc[k] = fmaf(w2, in[p * ld + i], acc[k]);
            }
        }
    }
#pragma unroll
    for (int k = 0; k < NP; ++k)
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], off);
}

template <int NP>
__device__ __forceinline__ float pick(const float (&acc)[NP], uint32_t lane) {
    float v = 0.0f;
#pragma unroll
    for (int k = 0; k < NP; ++k)
        if (lane == static_cast<uint32_t>(k)) v = acc[k];
    return v;
}

__global__ void __launch_bounds__(kThreads, 1) skyjepa_h0_pruned_kernel(SkyjepaArgs a, float* h0) {
    pdl_trigger();  // the input kernel after it in the stream needs nothing from it
    extern __shared__ __align__(16) float sm[];
    const uint32_t c = cta_rank(), b = blockIdx.x / kCl;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const TcnView& tcn = a.state_tcn;
    const TcnBlockView &L1 = tcn.blocks[0], &L2 = tcn.blocks[1], &L3 = tcn.blocks[2];
    const uint32_t o0 = c * kPer;
    // the CTA's weight rows, once, one copy group per stage: each stage waits
    // only for its own rows, the later ones land under the earlier stages
    auto commit = [] { asm volatile("cp.async.commit_group;" ::: "memory"); };
    copy16(sm + kOffW1a, L1.w1 + o0 * kIn * 3, kW1a);
    commit();
    copy16(sm + kOffW2a, L1.w2 + o0 * kC * 3, kW2);
    copy16(sm + kOffWr, L1.wr + o0 * kIn, kWr);
    commit();
    copy16(sm + kOffW1b, L2.w1 + o0 * kC * 3, kW2);
    commit();
    copy16(sm + kOffW2b, L2.w2 + o0 * kC * 3, kW2);
    commit();
    copy16(sm + kOffW1c, L3.w1 + o0 * kC * 3, kW2);
    commit();
    copy16(sm + kOffW2c, L3.w2 + o0 * kC * 3, kW2);
    commit();
    copy16(sm + kOffWp, a.proj_w + c * kProjPer * kC, kWp);
    commit();
    // groups still allowed in flight when a stage starts (its own and the earlier ones landed)
    auto landed = [](auto n) { asm volatile("cp.async.wait_group %0;" ::"n"(decltype(n)::value) : "memory"); };
    // the normalised history (every CTA its own copy)
    float* X = sm + kOffX;
    for (uint32_t q = tid; q < kHs * kIn; q += kThreads) {
        const uint32_t t = q / kIn, i = q % kIn;
        const float v = a.state_hist[(static_cast<size_t>(b) * kHs + t) * kIn + i];
        X[t * kXLd + i] = (v - a.state_mean[i]) / a.state_std[i];
    }
    landed(std::integral_constant<int, 6>{});
    __syncthreads();

    const uint32_t o = o0 + warp;
    auto out = [&](uint32_t off, int p) -> float& { return sm[off + p * kC + o]; };
    // ---- level 1, conv1 at all positions
    {
        float acc[10];
        conv_sums<kIn, 10, 0, 1, 1>(sm + kOffW1a + warp * kIn * 3, X, kXLd, lane, acc);
        if (lane < 10) out(kOffH1, lane) = gelu_tanh(pick(acc, lane) + __ldg(L1.b1 + o));
    }
    cluster_barrier();
    pull<10, 0, 1>(sm, kOffH1, c, tid);
    landed(std::integral_constant<int, 5>{});
    __syncthreads();
    // ---- level 1, conv2 + residual projection at the odd positions
    {
        float acc[5];
        conv_sums<kC, 5, 1, 2, 1>(sm + kOffW2a + warp * kC * 3, sm + kOffH1, kC, lane, acc);
        if (lane < 5) {
            const int p = 1 + 2 * static_cast<int>(lane);
            const float h2 = gelu_tanh(pick(acc, lane) + __ldg(L1.b2 + o));
            const float* wr = sm + kOffWr + warp * kIn;
            float r0 = 0.0f, r1 = 0.0f;
            for (uint32_t i = 0; i < kIn; i += 2) {
                r0 = fmaf(wr[i], X[p * kXLd + i], r0);
                r1 = fmaf(wr[i + 1], X[p * kXLd + i + 1], r1);
            }
            const float res = (r0 + r1) + __ldg(L1.br + o);
            out(kOffY1, p) = gelu_tanh(h2 + res);
        }
    }
    cluster_barrier();
    pull<5, 1, 2>(sm, kOffY1, c, tid);
    landed(std::integral_constant<int, 4>{});
    __syncthreads();
    // ---- level 2, conv1 at the odd positions
    {
        float acc[5];
        conv_sums<kC, 5, 1, 2, 2>(sm + kOffW1b + warp * kC * 3, sm + kOffY1, kC, lane, acc);
        if (lane < 5) out(kOffH2, 1 + 2 * lane) = gelu_tanh(pick(acc, lane) + __ldg(L2.b1 + o));
    }
    cluster_barrier();
    pull<5, 1, 2>(sm, kOffH2, c, tid);
    landed(std::integral_constant<int, 3>{});
    __syncthreads();
    // ---- level 2, conv2 + identity residual at 1, 5, 9
    {
        float acc[3];
        conv_sums<kC, 3, 1, 4, 2>(sm + kOffW2b + warp * kC * 3, sm + kOffH2, kC, lane, acc);
        if (lane < 3) {
            const int p = 1 + 4 * static_cast<int>(lane);
            const float h2 = gelu_tanh(pick(acc, lane) + __ldg(L2.b2 + o));
            out(kOffY2, p) = gelu_tanh(h2 + sm[kOffY1 + p * kC + o]);
        }
    }
    cluster_barrier();
    pull<3, 1, 4>(sm, kOffY2, c, tid);
    landed(std::integral_constant<int, 2>{});
    __syncthreads();
    // ---- level 3, conv1 at 1, 5, 9
    {
        float acc[3];
        conv_sums<kC, 3, 1, 4, 4>(sm + kOffW1c + warp * kC * 3, sm + kOffY2, kC, lane, acc);
        if (lane < 3) out(kOffH3, 1 + 4 * lane) = gelu_tanh(pick(acc, lane) + __ldg(L3.b1 + o));
    }
    cluster_barrier();
    pull<3, 1, 4>(sm, kOffH3, c, tid);
    landed(std::integral_constant<int, 1>{});
    __syncthreads();
    // ---- level 3, conv2 + identity residual at 9
    {
        float acc[1];
        conv_sums<kC, 1, 9, 1, 4>(sm + kOffW2c + warp * kC * 3, sm + kOffH3, kC, lane, acc);
        if (lane == 0) {
            const float h2 = gelu_tanh(acc[0] + __ldg(L3.b2 + o));
            out(kOffY3, 9) = gelu_tanh(h2 + sm[kOffY2 + 9 * kC + o]);
        }
    }
    cluster_barrier();
    pull<1, 9, 1>(sm, kOffY3, c, tid);
    landed(std::integral_constant<int, 0>{});
    __syncthreads();
    // ---- the projection of position 9: outputs 16c + 2w, 16c + 2w + 1
    const float* y = sm + kOffY3 + 9 * kC;
#pragma unroll
    for (uint32_t k = 0; k < 2; ++k) {
        const uint32_t ol = 2 * warp + k;
        const float* wp = sm + kOffWp + ol * kC;
        float s = 0.0f;
#pragma unroll
        for (uint32_t i = lane; i < kC; i += 32) s = fmaf(wp[i], y[i], s);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (lane == 0) {
            const uint32_t oo = c * kProjPer + ol;
            h0[static_cast<size_t>(b) * kLat + oo] = s + __ldg(a.proj_b + oo);
        }
    }
    cluster_barrier();  // no CTA leaves while a peer may still read its shared memory
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Shared-memory opt-in and non-portable cluster size, once per device; false
// when a 16-CTA cluster of the kernel cannot be resident.
bool h0_pruned_configure(int dev) {
    static std::mutex mu;
    static int state[64] = {};
    if (dev < 0 || dev >= 64) return false;
    std::lock_guard<std::mutex> lock(mu);
    if (state[dev] == 0) {
        const int smem = static_cast<int>(kSmemFloats * sizeof(float));
        cudaError_t e =
            cudaFuncSetAttribute(skyjepa_h0_pruned_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(skyjepa_h0_pruned_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        int n = 0;
        if (e == cudaSuccess) {
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(kCl, 1, 1);
            cfg.blockDim = dim3(kThreads, 1, 1);
            cfg.dynamicSmemBytes = static_cast<size_t>(smem);
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = kCl;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            e = cudaOccupancyMaxActiveClusters(&n, skyjepa_h0_pruned_kernel, &cfg);
        }
        (void)cudaGetLastError();
        state[dev] = (e == cudaSuccess && n >= 1) ? 1 : 2;
    }
    return state[dev] == 1;
}

}  // namespace

bool skyjepa_h0_pruned_supported(const SkyjepaArgs& a) {
    const TcnView& t = a.state_tcn;
    if (a.Hs != kHs || a.H != kLat || t.input_dim != kIn || t.k != 3 || t.levels != 3 || t.out_dim != kC ||
        t.max_ch != kC)
        return false;
    const uint32_t dil[3] = {1, 2, 4};
    for (uint32_t l = 0; l < 3; ++l) {
        const TcnBlockView& bk = t.blocks[l];
        if (bk.out != kC || bk.dil != dil[l] || bk.in != (l == 0 ? kIn : kC)) return false;
        if ((l == 0) != (bk.wr != nullptr)) return false;
        if (!aligned16(bk.w1) || !aligned16(bk.w2) || (bk.wr && !aligned16(bk.wr))) return false;
    }
    if (!aligned16(a.proj_w)) return false;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    return h0_pruned_configure(dev);
}

cudaError_t launch_skyjepa_h0_pruned(const SkyjepaArgs& a, float* h0, cudaStream_t stream) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(kCl * a.B, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemFloats * sizeof(float);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, skyjepa_h0_pruned_kernel, a, h0);
}

}  // namespace lwm
