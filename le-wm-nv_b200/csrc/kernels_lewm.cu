// kernels_lewm.cu — kernels of the LeWM / WorldModel scorer (f32).
//
// The scorer runs the reference's rollout (src/models/lewm/model.rs:94-147,
// modules.rs:9-399) as a short sequence of launches per predictor step over
// ALL candidates at once (rows = B*S*window tokens):
//   gemm_f32<EPI>   y = x W^T + b with a fused epilogue (GELU, SiLU, gated
//                   residual x += gate * y with the gate read from the
//                   precomputed AdaLN table through a row map)
//   ada_ln_kernel   LN_noaffine -> modulate(shift, scale) -> LN_affine, one
//                   warp per row (ConditionalBlock::forward, modules.rs:317-330)
//   attention_kernel causal softmax attention of a short window, one warp per
//                   (sequence, head, query); a one-token window needs no
//                   kernel at all (softmax over one key is exactly 1, so the
//                   attention output is V and only V is projected)
//   norm_act_kernel  BatchNorm(eval)/LayerNorm + GELU of the MLP hidden layer
//   + window assembly, goal cost, ViT patchify/assemble/attention.
// Everything stays in HBM-resident f32 buffers owned by the scorer.
#include <cuda_runtime.h>

#include <cstdint>

#include "lwm_device.cuh"
#include "lwm_lewm.hpp"
#include "lwm_lewm_epi.cuh"

namespace lwm {

// ------------------------------------------------------------------ GEMM
//
// C[M,N] = A[M,K] (row stride lda) . W[N,K]^T (+ bias), 64x64 tile per
// 256-thread block, 4x4 outputs per thread, K staged 32 at a time through
// shared memory (A transposed so a thread's 4 rows are one float4 read).  The
// next K tile is fetched into registers before the current one is multiplied,
// so its global-load latency overlaps the FMAs.  Each output's dot product
// runs in k order (as the reference's matmul).
constexpr int kBM = 64, kBN = 64, kBK = 32;

__global__ void __launch_bounds__(256) gemm_f32_kernel(GemmArgs g) {
    pdl_trigger();  // launched with programmatic serialization (launch_pdl): the next kernel may start
    pdl_wait();     // the kernels before this one are complete and their writes visible
    __shared__ __align__(16) float As[2][kBK][kBM + 4];
    __shared__ __align__(16) float Ws[2][kBK][kBN + 4];
    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;  // 16 x 16 threads, 4 x 4 outputs each
    const uint32_t m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
    float acc[4][4] = {};
    // this CTA's K range (split-K over blockIdx.z)
    const uint32_t kb = blockIdx.z * g.k_chunk;
    const uint32_t ke = min(g.K, kb + g.k_chunk);
    // loader mapping: 64 rows x 32 k = 2048 elements per tile, 8 per thread
    // (a lane reads 8 consecutive k of one row)
    const int lr = tid / 4, lk = (tid % 4) * 8;
    const uint32_t am = m0 + lr, wn = n0 + lr;
    const float* arow = g.A + static_cast<size_t>(am < g.M ? am : 0) * g.lda;
    const float* wrow = g.W + static_cast<size_t>(wn < g.N ? wn : 0) * g.ldw;
    float ra[8], rw[8];
    auto fetch = [&](uint32_t k0) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const uint32_t k = k0 + lk + q;
            ra[q] = (am < g.M && k < ke) ? __ldg(arow + k) : 0.0f;
            rw[q] = (wn < g.N && k < ke) ? __ldg(wrow + k) : 0.0f;
        }
    };
    auto stash = [&](int buf) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            As[buf][lk + q][lr] = ra[q];
            Ws[buf][lk + q][lr] = rw[q];
        }
    };
    fetch(kb);
    stash(0);
    __syncthreads();
    int buf = 0;
    for (uint32_t k0 = kb; k0 < ke; k0 += kBK) {
        const bool more = k0 + kBK < ke;
        if (more) fetch(k0 + kBK);  // in flight during the FMAs below
#pragma unroll
        for (int kk = 0; kk < kBK; ++kk) {
            const float4 a = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
            const float4 w = *reinterpret_cast<const float4*>(&Ws[buf][kk][tx * 4]);
            const float av[4] = {a.x, a.y, a.z, a.w}, wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], wv[j], acc[i][j]);
        }
        if (more) stash(buf ^ 1);
        __syncthreads();
        buf ^= 1;
    }
    // epilogue_value's arithmetic on the thread's 4 x 4 outputs, with every
    // bias / residual / gate operand loaded before the first store (loads
    // after a store to C would each wait for it: C might alias them)
    auto finish = [&](const float (&val)[4][4]) {
        float bv[4], cv[4][4], gv[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t n = n0 + tx * 4 + j;
            bv[j] = (g.bias && n < g.N) ? g.bias[n] : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t m = m0 + ty * 4 + i;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t n = n0 + tx * 4 + j;
                const bool in = g.residual && m < g.M && n < g.N;
                cv[i][j] = in ? g.C[static_cast<size_t>(m) * g.ldc + n] : 0.0f;
                gv[i][j] = (in && g.gate) ? g.gate[g.map.row(m) * g.ldg + n] : 0.0f;
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t m = m0 + ty * 4 + i;
            if (m >= g.M) continue;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t n = n0 + tx * 4 + j;
                if (n >= g.N) continue;
                float v = val[i][j];
                if (g.bias) v = v + bv[j];
                if (g.residual) {
                    if (g.gate) v = gv[i][j] * v;
                    v = cv[i][j] + v;
                } else {
                    v = apply_act(g.act, v);
                }
                g.C[static_cast<size_t>(m) * g.ldc + n] = v;
            }
        }
    };
    if (g.splits <= 1) {
        finish(acc);
        return;
    }
    // split-K: park this split's tile, the last split of the tile to arrive
    // adds the partial tiles in split order (deterministic) and runs the epilogue
    const size_t tile = static_cast<size_t>(blockIdx.y) * gridDim.x + blockIdx.x;
    float* mine = g.partial + (tile * g.splits + blockIdx.z) * (kBM * kBN);
#pragma unroll
    for (int i = 0; i < 4; ++i)
        *reinterpret_cast<float4*>(mine + (ty * 4 + i) * kBN + tx * 4) =
            make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    __threadfence();
    __syncthreads();
    __shared__ int s_last;
    if (tid == 0) s_last = atomicAdd(&g.counters[tile], 1u) == g.splits - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* parts = g.partial + tile * g.splits * (kBM * kBN);
    float sum[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) sum[i][j] = 0.0f;
    for (uint32_t z = 0; z < g.splits; ++z) {  // split order: sum += partial_z
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 p = __ldcg(reinterpret_cast<const float4*>(parts + z * (kBM * kBN) + (ty * 4 + i) * kBN + tx * 4));
            sum[i][0] += p.x;
            sum[i][1] += p.y;
            sum[i][2] += p.z;
            sum[i][3] += p.w;
        }
    }
    finish(sum);
    if (tid == 0) g.counters[tile] = 0u;
}

// Split K when the output tiles alone leave most SMs idle: aim for about two
// waves of CTAs, at least 64 K per split, at most 16 splits.
cudaError_t gemm_f32(const GemmArgs& in, cudaStream_t stream, const SplitScratch* sp) {
    if (in.M == 0 || in.N == 0) return cudaSuccess;
    if (sp && sp->tc_err && gemm_tc_eligible(in)) return gemm_tc(in, stream, sp, sp->tc_err);
    GemmArgs g = in;
    const uint32_t tx = (g.N + kBN - 1) / kBN, ty = (g.M + kBM - 1) / kBM;
    const size_t tiles = static_cast<size_t>(tx) * ty;
    uint32_t splits = 1;
    if (sp && sp->partial && tiles < 296 && g.K >= 128) {
        splits = static_cast<uint32_t>((296 + tiles - 1) / tiles);
        splits = min(splits, min(16u, g.K / 64));
        while (splits > 1 && tiles * splits * kBM * kBN > sp->floats) --splits;
        if (tiles > sp->n_counters) splits = 1;
    }
    g.splits = splits;
    g.k_chunk = splits > 1 ? ((g.K + splits - 1) / splits + kBK - 1) / kBK * kBK : g.K;
    if (splits > 1) {
        g.splits = (g.K + g.k_chunk - 1) / g.k_chunk;  // no empty split
        g.partial = sp->partial;
        g.counters = sp->counters;
    }
    dim3 grid(tx, ty, g.splits);
    if (cudaError_t e = launch_pdl(gemm_f32_kernel, grid, dim3(256), 0, stream, g); e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ------------------------------------------------------------ row kernels

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Per-row LayerNorm statistics over d elements held by one warp (x in global
// or shared memory): mean = sum / d, var = sum((x - mean)^2) / d.
__device__ __forceinline__ void row_stats(const float* x, uint32_t d, float& mean, float& den, float eps) {
    const int lane = threadIdx.x & 31;
    float s = 0.0f;
    for (uint32_t i = lane; i < d; i += 32) s += x[i];
    mean = warp_sum(s) / static_cast<float>(d);
    float v = 0.0f;
    for (uint32_t i = lane; i < d; i += 32) {
        const float c = x[i] - mean;
        v += c * c;
    }
    den = sqrtf(warp_sum(v) / static_cast<float>(d) + eps);
}

// y = LN_affine(LN_noaffine(x, 1e-6) * (scale + 1) + shift, 1e-5)
// shift/scale come from the AdaLN table row map.row(r) at column offsets
// shift_off / scale_off (modules.rs:317-330, 9-27).
// The row (d <= 1024) is held in registers, 32 values per lane at most;
// shift/scale are fetched together with it.
constexpr int kRowRegs = 32;
// NQ = values a lane holds: the row width over 32 rounded up (kRowRegs for
// any width up to 1024; the exact count for the common widths, so that no
// predicated-off loads or math are issued).
template <int NQ>
__global__ void ada_ln_kernel(const float* x, float* y, uint32_t rows, uint32_t d, const float* ada, uint32_t ld_ada,
                              uint32_t shift_off, uint32_t scale_off, RowMap map, const float* w, const float* b) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t r = blockIdx.x * (blockDim.x >> 5) + warp;
    if (r >= rows) return;
    const float* xr = x + static_cast<size_t>(r) * d;
    const float* a = ada + map.row(r) * ld_ada;
    // the affine weights too, so that no load waits behind the stores at the end
    float v[NQ], sh[NQ], sc[NQ], wv[NQ], bv[NQ];
    float s = 0.0f;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
        const uint32_t i = lane + 32 * q;
        const bool in = i < d;
        v[q] = in ? xr[i] : 0.0f;
        sh[q] = in ? a[shift_off + i] : 0.0f;
        sc[q] = in ? a[scale_off + i] : 0.0f;
        wv[q] = in ? w[i] : 0.0f;
        bv[q] = in ? b[i] : 0.0f;
        s += v[q];
    }
    float mean = warp_sum(s) / static_cast<float>(d);
    float var = 0.0f;
#pragma unroll
    for (int q = 0; q < NQ; ++q)
        if (lane + 32 * q < d) {
            const float c = v[q] - mean;
            var += c * c;
        }
    float den = sqrtf(warp_sum(var) / static_cast<float>(d) + 1e-6f);
    s = 0.0f;
#pragma unroll
    for (int q = 0; q < NQ; ++q)
        if (lane + 32 * q < d) {
            v[q] = (v[q] - mean) / den * (sc[q] + 1.0f) + sh[q];
            s += v[q];
        }
    mean = warp_sum(s) / static_cast<float>(d);
    var = 0.0f;
#pragma unroll
    for (int q = 0; q < NQ; ++q)
        if (lane + 32 * q < d) {
            const float c = v[q] - mean;
            var += c * c;
        }
    den = sqrtf(warp_sum(var) / static_cast<float>(d) + 1e-5f);
    float* yr = y + static_cast<size_t>(r) * d;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
        const uint32_t i = lane + 32 * q;
        if (i < d) yr[i] = (v[q] - mean) / den * wv[q] + bv[q];
    }
}

// LayerNorm (affine, eps) of rows gathered from src row (r * t_in + pick).
__global__ void layernorm_kernel(const float* x, float* y, uint32_t rows, uint32_t d, uint32_t t_in, uint32_t pick,
                                 const float* w, const float* b, float eps) {
    pdl_trigger();  // launched with programmatic serialization (launch_pdl): the next kernel may start
    pdl_wait();     // the kernels before this one are complete and their writes visible
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t r = blockIdx.x * (blockDim.x >> 5) + warp;
    if (r >= rows) return;
    const float* xr = x + (static_cast<size_t>(r) * t_in + pick) * d;
    float mean, den;
    row_stats(xr, d, mean, den, eps);
    float* yr = y + static_cast<size_t>(r) * d;
    for (uint32_t i = lane; i < d; i += 32) yr[i] = (xr[i] - mean) / den * w[i] + b[i];
}

// The same for rows of exactly NQ x 32 values (the ViT's 192: NQ = 6): the
// row is read once into registers; the sums run in row_stats' order, so the
// outputs are layernorm_kernel's.
template <int NQ>
__global__ void layernorm_reg_kernel(const float* x, float* y, uint32_t rows, uint32_t t_in, uint32_t pick,
                                     const float* w, const float* b, float eps) {
    pdl_trigger();  // launched with programmatic serialization (launch_pdl): the next kernel may start
    pdl_wait();     // the kernels before this one are complete and their writes visible
    constexpr uint32_t d = NQ * 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t r = blockIdx.x * (blockDim.x >> 5) + warp;
    if (r >= rows) return;
    const float* xr = x + (static_cast<size_t>(r) * t_in + pick) * d;
    float v[NQ];
#pragma unroll
    for (int q = 0; q < NQ; ++q) v[q] = xr[lane + 32 * q];
    float sum = 0.0f;
#pragma unroll
    for (int q = 0; q < NQ; ++q) sum += v[q];
    const float mean = warp_sum(sum) / static_cast<float>(d);
    float var = 0.0f;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
        const float c = v[q] - mean;
        var += c * c;
    }
    const float den = sqrtf(warp_sum(var) / static_cast<float>(d) + eps);
    float* yr = y + static_cast<size_t>(r) * d;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
        const uint32_t i = lane + 32 * q;
        yr[i] = (v[q] - mean) / den * w[i] + b[i];
    }
}

// In place: norm (BatchNorm eval / LayerNorm / none) then GELU (tanh) of an
// MLP hidden layer (Mlp::forward, modules.rs:108-115; VectorMlpEncoder).
__global__ void norm_act_kernel(float* x, uint32_t rows, uint32_t d, int kind, const float* w, const float* b,
                                const float* rm, const float* rv) {
    pdl_trigger();  // launched with programmatic serialization (launch_pdl): the next kernel may start
    pdl_wait();     // the kernels before this one are complete and their writes visible
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t r = blockIdx.x * (blockDim.x >> 5) + warp;
    if (r >= rows) return;
    float* xr = x + static_cast<size_t>(r) * d;
    float mean = 0.0f, den = 1.0f;
    if (kind == kNormLayer) row_stats(xr, d, mean, den, 1e-5f);
    __syncwarp();
    for (uint32_t i = lane; i < d; i += 32) {
        float v = xr[i];
        if (kind == kNormLayer) v = (v - mean) / den * w[i] + b[i];
        else if (kind == kNormBatch) v = (v - rm[i]) / sqrtf(rv[i] + 1e-5f) * w[i] + b[i];
        xr[i] = gelu_tanh(v);
    }
}

// The same for wide hidden layers (d up to 2048, e.g. the image model's
// pred_proj): a block per row, the row held in registers (kNaPer values a
// thread), one read and one write of it; the mean and the variance are
// block reductions (two passes over the registers, as row_stats does).
constexpr uint32_t kNaThreads = 256, kNaPer = 8;
__device__ __forceinline__ float block_sum(float v, float* red) {
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    v = warp_sum(v);
    __syncthreads();  // red is reused by consecutive reductions
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < (kNaThreads >> 5) ? red[lane] : 0.0f;
    return warp_sum(t);
}

__global__ void __launch_bounds__(kNaThreads) norm_act_row_kernel(float* x, uint32_t d, int kind, const float* w,
                                                                  const float* b, const float* rm, const float* rv) {
    pdl_trigger();  // launched with programmatic serialization (launch_pdl): the next kernel may start
    pdl_wait();     // the kernels before this one are complete and their writes visible
    __shared__ float red[kNaThreads >> 5];
    float* xr = x + static_cast<size_t>(blockIdx.x) * d;
    float v[kNaPer];
#pragma unroll
    for (uint32_t j = 0; j < kNaPer; ++j) {
        const uint32_t i = threadIdx.x + j * kNaThreads;
        v[j] = i < d ? xr[i] : 0.0f;
    }
    float mean = 0.0f, den = 1.0f;
    if (kind == kNormLayer) {
        float s = 0.0f;
#pragma unroll
        for (uint32_t j = 0; j < kNaPer; ++j) s += v[j];
        mean = block_sum(s, red) / static_cast<float>(d);
        float q = 0.0f;
#pragma unroll
        for (uint32_t j = 0; j < kNaPer; ++j) {
            const uint32_t i = threadIdx.x + j * kNaThreads;
            const float c = v[j] - mean;
            if (i < d) q += c * c;
        }
        den = sqrtf(block_sum(q, red) / static_cast<float>(d) + 1e-5f);
    }
#pragma unroll
    for (uint32_t j = 0; j < kNaPer; ++j) {
        const uint32_t i = threadIdx.x + j * kNaThreads;
        if (i >= d) break;
        float u = v[j];
        if (kind == kNormLayer) u = (u - mean) / den * w[i] + b[i];
        else if (kind == kNormBatch) u = (u - rm[i]) / sqrtf(rv[i] + 1e-5f) * w[i] + b[i];
        xr[i] = gelu_tanh(u);
    }
}

__global__ void silu_kernel(const float* x, float* y, size_t n) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) {
        const float v = x[i];
        y[i] = v / (1.0f + expf(-v));
    }
}

// Window tokens of one predictor step: X[(r, w)] = frames[r, lo + w] + pos[w]
// (rollout_embeddings_with_history, model.rs:128-141; Predictor::forward_last).
__global__ void window_kernel(const float* frames, uint32_t nframes, const float* pos, float* X, uint32_t rows,
                              uint32_t w_len, uint32_t lo, uint32_t d) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t total = static_cast<size_t>(rows) * w_len * d;
    if (i >= total) return;
    const uint32_t c = static_cast<uint32_t>(i % d);
    const size_t tok = i / d;
    const uint32_t w = static_cast<uint32_t>(tok % w_len);
    const size_t r = tok / w_len;
    X[i] = frames[(r * nframes + lo + w) * d + c] + pos[static_cast<size_t>(w) * d + c];
}

// frames[r, slot] = src[r]; frames[r, j] = hist[r / S, j] for j < h (init).
__global__ void frames_init_kernel(const float* hist, uint32_t h, uint32_t S, float* frames, uint32_t nframes,
                                   size_t rows, uint32_t d) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= rows * h * d) return;
    const uint32_t c = static_cast<uint32_t>(i % d);
    const size_t t = i / d;
    const uint32_t j = static_cast<uint32_t>(t % h);
    const size_t r = t / h;
    frames[(r * nframes + j) * d + c] = hist[((r / S) * h + j) * d + c];
}

__global__ void frames_put_kernel(const float* src, float* frames, uint32_t nframes, uint32_t slot, size_t rows,
                                  uint32_t d) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= rows * d) return;
    const size_t r = i / d;
    frames[(r * nframes + slot) * d + i % d] = src[i];
}

// Causal softmax attention of short windows (Attention::forward,
// modules.rs:245-275): qkv [seqs*t, 3*H*dh] -> out [seqs*t, H*dh]; one warp
// per (sequence, head, query); q scaled before the dot product as the
// reference does (q * scale).
__global__ void attention_kernel(const float* qkv, float* out, uint32_t seqs, uint32_t t, uint32_t H, uint32_t dh,
                                 float scale, int causal, int scale_q_first) {
    pdl_trigger();  // launched with programmatic serialization (launch_pdl): the next kernel may start
    pdl_wait();     // the kernels before this one are complete and their writes visible
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t gw = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + warp;
    const size_t total = static_cast<size_t>(seqs) * H * t;
    if (gw >= total) return;
    const uint32_t i = static_cast<uint32_t>(gw % t);
    const uint32_t h = static_cast<uint32_t>((gw / t) % H);
    const size_t s = gw / (static_cast<size_t>(t) * H);
    const uint32_t inner = H * dh;
    const float* base = qkv + s * t * 3 * inner;
    const float* q = base + static_cast<size_t>(i) * 3 * inner + h * dh;
    const uint32_t jmax = causal ? i + 1 : t;
    // pass 1: max score
    float mx = -INFINITY;
    for (uint32_t j = 0; j < jmax; ++j) {
        const float* k = base + static_cast<size_t>(j) * 3 * inner + inner + h * dh;
        float acc = 0.0f;
        for (uint32_t d = lane; d < dh; d += 32) acc += (scale_q_first ? q[d] * scale : q[d]) * k[d];
        acc = warp_sum(acc);
        if (!scale_q_first) acc *= scale;
        mx = fmaxf(mx, acc);
    }
    // pass 2: weights and output (dh <= 128: 4 accumulators per lane)
    float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float sum = 0.0f;
    for (uint32_t j = 0; j < jmax; ++j) {
        const float* k = base + static_cast<size_t>(j) * 3 * inner + inner + h * dh;
        float acc = 0.0f;
        for (uint32_t d = lane; d < dh; d += 32) acc += (scale_q_first ? q[d] * scale : q[d]) * k[d];
        acc = warp_sum(acc);
        if (!scale_q_first) acc *= scale;
        const float p = expf(acc - mx);
        sum += p;
        const float* v = base + static_cast<size_t>(j) * 3 * inner + 2 * inner + h * dh;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint32_t d = lane + 32 * u;
            if (d < dh) o[u] += p * v[d];
        }
    }
    float* orow = out + (s * t + i) * inner + h * dh;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const uint32_t d = lane + 32 * u;
        if (d < dh) orow[d] = o[u] / sum;
    }
}

// The same attention for long sequences (the ViT's 197 tokens): a block per
// (sequence, head, 32 queries) keeps the head's K (rows padded to dh + 1, so
// the lanes' different rows hit different banks) and V in shared memory; a
// warp takes one query at a time, its lanes score 32 keys in parallel, the
// softmax is a warp max / sum, and each lane then accumulates its own output
// dimensions over the keys.
constexpr uint32_t kAttnQ = 32, kAttnMaxT = 256;

__global__ void __launch_bounds__(256) attention_smem_kernel(const float* qkv, float* out, uint32_t t, uint32_t H,
                                                             uint32_t dh, float scale, int causal, int scale_q_first) {
    pdl_trigger();  // launched with programmatic serialization (launch_pdl): the next kernel may start
    pdl_wait();     // the kernels before this one are complete and their writes visible
    extern __shared__ float sm[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t h = blockIdx.y, q0 = blockIdx.x * kAttnQ;
    const size_t s = blockIdx.z;
    const uint32_t inner = H * dh, kld = dh + 1;
    float* Ks = sm;                  // [t][dh + 1]
    float* Vs = Ks + t * kld;        // [t][dh]
    float* Ps = Vs + t * dh;         // [8][t]
    float* Qs = Ps + 8 * t;          // [8][dh]
    const float* base = qkv + s * t * 3 * inner;
    for (uint32_t idx = threadIdx.x; idx < t * dh; idx += blockDim.x) {
        const uint32_t j = idx / dh, d = idx % dh;
        const float* row = base + static_cast<size_t>(j) * 3 * inner + h * dh + d;
        Ks[j * kld + d] = row[inner];
        Vs[j * dh + d] = row[2 * inner];
    }
    __syncthreads();
    float* p = Ps + warp * t;
    float* qv = Qs + warp * dh;
    for (uint32_t qi = warp; qi < kAttnQ; qi += 8) {
        const uint32_t i = q0 + qi;
        if (i >= t) break;
        const float* q = base + static_cast<size_t>(i) * 3 * inner + h * dh;
        for (uint32_t d = lane; d < dh; d += 32) qv[d] = scale_q_first ? q[d] * scale : q[d];
        __syncwarp();
        const uint32_t jmax = causal ? i + 1 : t;
        float sc[kAttnMaxT / 32];
        float mx = -INFINITY;
#pragma unroll
        for (uint32_t r = 0; r < kAttnMaxT / 32; ++r) {
            const uint32_t j = r * 32 + lane;
            float acc = -INFINITY;
            if (j < jmax) {
                const float* kr = Ks + j * kld;
                acc = 0.0f;
                for (uint32_t d = 0; d < dh; ++d) acc = fmaf(qv[d], kr[d], acc);
                if (!scale_q_first) acc *= scale;
            }
            sc[r] = acc;
            mx = fmaxf(mx, acc);
        }
        mx = warp_max(mx);
        float sum = 0.0f;
#pragma unroll
        for (uint32_t r = 0; r < kAttnMaxT / 32; ++r) {
            const uint32_t j = r * 32 + lane;
            if (j < jmax) {
                const float e = expf(sc[r] - mx);
                p[j] = e;
                sum += e;
            }
        }
        sum = warp_sum(sum);
        __syncwarp();
        float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (uint32_t j = 0; j < jmax; ++j) {
            const float w = p[j];
            const float* vr = Vs + j * dh;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t d = lane + 32 * u;
                if (d < dh) o[u] = fmaf(w, vr[d], o[u]);
            }
        }
        float* orow = out + (s * t + i) * inner + h * dh;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint32_t d = lane + 32 * u;
            if (d < dh) orow[d] = o[u] / sum;
        }
        __syncwarp();
    }
}

// The same attention for 64-wide heads, register-tiled: a block per
// (sequence, head, 8 QW queries), K (staged by cp.async; rows padded to 68 floats: 16-byte rows
// that eight lanes read from eight different bank quads), V and the block's
// queries in shared memory.  Warp w scores its QW (4, or 2 when the grid is
// small) queries against keys lane + 32 u (u < 8), QW x 8 accumulators a
// thread, 16-byte operand loads; the softmax weights go to a per-warp
// [key][4] table, and the lanes then accumulate output dimensions lane and
// lane + 32 of the QW queries over the keys.  Every dot product, the softmax and the weighted sums run in the
// same order as attention_smem_kernel's, so the outputs are identical.
constexpr uint32_t kAtQ = 32, kAtDh = 64, kAtKld = 68;

// 16 bytes global -> shared without a register round trip (zero-filled when
// `bytes` is 0); all of a thread's copies are in flight until the wait.
__device__ __forceinline__ void at_copy16(float* dst, const float* src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src), "r"(bytes)
                 : "memory");
}
__host__ __device__ inline uint32_t at_tpad(uint32_t t) { return (t + 31u) & ~31u; }
__host__ __device__ inline size_t at_smem_floats(uint32_t t) {
    const uint32_t tp = at_tpad(t);
    return static_cast<size_t>(tp) * kAtKld + static_cast<size_t>(tp) * kAtDh + kAtQ * kAtKld + 8u * tp * 4u;
}

template <uint32_t QW>
__global__ void __launch_bounds__(256) attention_tiled_kernel(const float* qkv, float* out, uint32_t t, uint32_t H,
                                                              float scale, int causal, int scale_q_first) {
    pdl_trigger();  // launched with programmatic serialization (launch_pdl): the next kernel may start
    pdl_wait();     // the kernels before this one are complete and their writes visible
    extern __shared__ __align__(16) float sm[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t h = blockIdx.y, q0 = blockIdx.x * (8u * QW), tp = at_tpad(t);
    const size_t s = blockIdx.z;
    const uint32_t inner = H * kAtDh;
    float* Ks = sm;                    // [tp][68]
    float* Vs = Ks + tp * kAtKld;      // [tp][64]
    float* Qs = Vs + tp * kAtDh;       // [32][68]
    float* Pt = Qs + kAtQ * kAtKld + warp * tp * 4u;  // this warp's [tp][4]
    const float* base = qkv + s * t * 3 * inner;
    // K and V rows by asynchronous copies (every row in flight at once; the
    // padding rows j >= t zero-filled)
    for (uint32_t idx = threadIdx.x; idx < tp * 16u; idx += blockDim.x) {
        const uint32_t j = idx >> 4, c = (idx & 15u) * 4u;
        const float* row = base + static_cast<size_t>(j < t ? j : 0u) * 3 * inner + h * kAtDh + c;
        const uint32_t bytes = j < t ? 16u : 0u;
        at_copy16(Ks + j * kAtKld + c, row + inner, bytes);
        at_copy16(Vs + j * kAtDh + c, row + 2 * inner, bytes);
    }
    for (uint32_t idx = threadIdx.x; idx < 8u * QW * 16u; idx += blockDim.x) {
        const uint32_t qi = idx >> 4, c = (idx & 15u) * 4u, i = q0 + qi;
        float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < t) {
            q = *reinterpret_cast<const float4*>(base + static_cast<size_t>(i) * 3 * inner + h * kAtDh + c);
            if (scale_q_first) { q.x *= scale; q.y *= scale; q.z *= scale; q.w *= scale; }
        }
        *reinterpret_cast<float4*>(Qs + qi * kAtKld + c) = q;
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    const uint32_t ql = warp * QW;  // the warp's first query, block-local
    if (q0 + ql >= t) return;
    float acc[QW][8];
#pragma unroll
    for (int a = 0; a < static_cast<int>(QW); ++a)
#pragma unroll
        for (int u = 0; u < 8; ++u) acc[a][u] = 0.0f;
    const uint32_t nu = tp / 32u;  // key rounds that hold real keys (the rest of the 8 stay unused)
#pragma unroll 1
    for (uint32_t d = 0; d < kAtDh; d += 4) {
        float4 q[QW];
#pragma unroll
        for (int a = 0; a < static_cast<int>(QW); ++a) q[a] = *reinterpret_cast<const float4*>(Qs + (ql + a) * kAtKld + d);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (static_cast<uint32_t>(u) >= nu) break;
            const float4 k = *reinterpret_cast<const float4*>(Ks + (u * 32u + lane) * kAtKld + d);
#pragma unroll
            for (int a = 0; a < static_cast<int>(QW); ++a) {
                acc[a][u] = fmaf(q[a].x, k.x, acc[a][u]);
                acc[a][u] = fmaf(q[a].y, k.y, acc[a][u]);
                acc[a][u] = fmaf(q[a].z, k.z, acc[a][u]);
                acc[a][u] = fmaf(q[a].w, k.w, acc[a][u]);
            }
        }
    }
    float inv[QW];
    uint32_t jend = 0;
#pragma unroll
    for (int a = 0; a < static_cast<int>(QW); ++a) {
        const uint32_t i = q0 + ql + a;
        const uint32_t jmax = i >= t ? 0u : (causal ? i + 1 : t);
        jend = jmax > jend ? jmax : jend;
        float mx = -INFINITY;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const uint32_t j = u * 32u + lane;
            float v = -INFINITY;
            if (static_cast<uint32_t>(u) < nu && j < jmax) v = scale_q_first ? acc[a][u] : acc[a][u] * scale;
            acc[a][u] = v;
            mx = fmaxf(mx, v);
        }
        mx = warp_max(mx);
        float sum = 0.0f;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const uint32_t j = u * 32u + lane;
            if (static_cast<uint32_t>(u) >= nu) break;
            float e = 0.0f;
            if (j < jmax) {
                e = expf(acc[a][u] - mx);
                sum += e;
            }
            Pt[j * 4u + a] = e;  // zero past the query's last key: adds nothing below
        }
        inv[a] = warp_sum(sum);
    }
    __syncwarp();
    float o[QW][2];
#pragma unroll
    for (int a = 0; a < static_cast<int>(QW); ++a) { o[a][0] = 0.0f; o[a][1] = 0.0f; }
    for (uint32_t j = 0; j < jend; ++j) {
        const float4 p = *reinterpret_cast<const float4*>(Pt + j * 4u);
        const float pw[4] = {p.x, p.y, p.z, p.w};
        const float v0 = Vs[j * kAtDh + lane], v1 = Vs[j * kAtDh + lane + 32u];
#pragma unroll
        for (int a = 0; a < static_cast<int>(QW); ++a) {
            o[a][0] = fmaf(pw[a], v0, o[a][0]);
            o[a][1] = fmaf(pw[a], v1, o[a][1]);
        }
    }
#pragma unroll
    for (int a = 0; a < static_cast<int>(QW); ++a) {
        const uint32_t i = q0 + ql + a;
        if (i >= t) break;
        float* orow = out + (s * t + i) * inner + h * kAtDh;
        orow[lane] = o[a][0] / inv[a];
        orow[lane + 32u] = o[a][1] / inv[a];
    }
}

// Goal cost (goal_cost, model.rs:149-165): sum_d (pred - goal[r / S])^2.
__global__ void goal_cost_kernel(const float* pred, const float* goal, uint32_t S, size_t rows, uint32_t d,
                                 float* scores) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t r = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + warp;
    if (r >= rows) return;
    const float* p = pred + r * d;
    const float* g = goal + (r / S) * d;
    float acc = 0.0f;
    for (uint32_t i = lane; i < d; i += 32) {
        const float e = p[i] - g[i];
        acc += e * e;
    }
    acc = warp_sum(acc);
    if (lane == 0) scores[r] = acc;
}

// ViT: patches [n, np, C*p*p] from pixels [n, C, img, img] (conv k = stride = p).
__global__ void patchify_kernel(const float* pix, float* patches, uint32_t n, uint32_t C, uint32_t img, uint32_t p) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint32_t side = img / p, kdim = C * p * p;
    const size_t total = static_cast<size_t>(n) * side * side * kdim;
    if (i >= total) return;
    const uint32_t k = static_cast<uint32_t>(i % kdim);
    const size_t pt = i / kdim;
    const uint32_t pidx = static_cast<uint32_t>(pt % (side * side));
    const size_t im = pt / (side * side);
    const uint32_t ch = k / (p * p), ky = (k / p) % p, kx = k % p;
    const uint32_t py = pidx / side, px = pidx % side;
    patches[i] = pix[((im * C + ch) * img + py * p + ky) * img + px * p + kx];
}

// tokens [n, 1 + np, vh] = [cls ; patch embeddings] + position embeddings.
__global__ void vit_assemble_kernel(const float* patch_out, const float* cls, const float* pos, float* x, uint32_t n,
                                    uint32_t np, uint32_t vh) {
    pdl_trigger();  // launched with programmatic serialization (launch_pdl): the next kernel may start
    pdl_wait();     // the kernels before this one are complete and their writes visible
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t total = static_cast<size_t>(n) * (np + 1) * vh;
    if (i >= total) return;
    const uint32_t c = static_cast<uint32_t>(i % vh);
    const size_t tok = i / vh;
    const uint32_t t = static_cast<uint32_t>(tok % (np + 1));
    const size_t im = tok / (np + 1);
    const float v = t == 0 ? cls[c] : patch_out[(im * np + t - 1) * vh + c];
    x[i] = v + pos[static_cast<size_t>(t) * vh + c];
}

// ------------------------------------------------------------- launchers

static inline uint32_t blocks_for(size_t n, uint32_t per) { return static_cast<uint32_t>((n + per - 1) / per); }

cudaError_t launch_ada_ln(const float* x, float* y, uint32_t rows, uint32_t d, const float* ada, uint32_t ld_ada,
                          uint32_t shift_off, uint32_t scale_off, RowMap map, const float* w, const float* b,
                          cudaStream_t s) {
    if (!rows) return cudaSuccess;
    constexpr int kWarps = 8;
    const dim3 grid(blocks_for(rows, kWarps)), block(kWarps * 32);
    switch (d) {
        case 192: ada_ln_kernel<6><<<grid, block, 0, s>>>(x, y, rows, d, ada, ld_ada, shift_off, scale_off, map, w, b); break;
        case 256: ada_ln_kernel<8><<<grid, block, 0, s>>>(x, y, rows, d, ada, ld_ada, shift_off, scale_off, map, w, b); break;
        case 384: ada_ln_kernel<12><<<grid, block, 0, s>>>(x, y, rows, d, ada, ld_ada, shift_off, scale_off, map, w, b); break;
        case 512: ada_ln_kernel<16><<<grid, block, 0, s>>>(x, y, rows, d, ada, ld_ada, shift_off, scale_off, map, w, b); break;
        default:
            ada_ln_kernel<kRowRegs><<<grid, block, 0, s>>>(x, y, rows, d, ada, ld_ada, shift_off, scale_off, map, w, b);
    }
    return cudaGetLastError();
}

cudaError_t launch_layernorm(const float* x, float* y, uint32_t rows, uint32_t d, uint32_t t_in, uint32_t pick,
                             const float* w, const float* b, float eps, cudaStream_t s) {
    if (!rows) return cudaSuccess;
    if (d == 192)
        return launch_pdl(layernorm_reg_kernel<6>, dim3(blocks_for(rows, 8)), dim3(256), 0, s, x, y, rows, t_in, pick, w,
                          b, eps);
    return launch_pdl(layernorm_kernel, dim3(blocks_for(rows, 8)), dim3(256), 0, s, x, y, rows, d, t_in, pick, w, b,
                      eps);
}

cudaError_t launch_norm_act(float* x, uint32_t rows, uint32_t d, int kind, const float* w, const float* b,
                            const float* rm, const float* rv, cudaStream_t s) {
    if (!rows) return cudaSuccess;
    if (d >= 512 && d <= kNaThreads * kNaPer)
        return launch_pdl(norm_act_row_kernel, dim3(rows), dim3(kNaThreads), 0, s, x, d, kind, w, b, rm, rv);
    else
        return launch_pdl(norm_act_kernel, dim3(blocks_for(rows, 8)), dim3(256), 0, s, x, rows, d, kind, w, b, rm, rv);
}

cudaError_t launch_silu(const float* x, float* y, size_t n, cudaStream_t s) {
    if (!n) return cudaSuccess;
    silu_kernel<<<blocks_for(n, 256), 256, 0, s>>>(x, y, n);
    return cudaGetLastError();
}

cudaError_t launch_window(const float* frames, uint32_t nframes, const float* pos, float* X, uint32_t rows,
                          uint32_t w_len, uint32_t lo, uint32_t d, cudaStream_t s) {
    const size_t n = static_cast<size_t>(rows) * w_len * d;
    if (!n) return cudaSuccess;
    window_kernel<<<blocks_for(n, 256), 256, 0, s>>>(frames, nframes, pos, X, rows, w_len, lo, d);
    return cudaGetLastError();
}

cudaError_t launch_frames_init(const float* hist, uint32_t h, uint32_t S, float* frames, uint32_t nframes,
                               size_t rows, uint32_t d, cudaStream_t s) {
    const size_t n = rows * h * d;
    if (!n) return cudaSuccess;
    frames_init_kernel<<<blocks_for(n, 256), 256, 0, s>>>(hist, h, S, frames, nframes, rows, d);
    return cudaGetLastError();
}

cudaError_t launch_frames_put(const float* src, float* frames, uint32_t nframes, uint32_t slot, size_t rows,
                              uint32_t d, cudaStream_t s) {
    const size_t n = rows * d;
    if (!n) return cudaSuccess;
    frames_put_kernel<<<blocks_for(n, 256), 256, 0, s>>>(src, frames, nframes, slot, rows, d);
    return cudaGetLastError();
}

cudaError_t launch_attention(const float* qkv, float* out, uint32_t seqs, uint32_t t, uint32_t H, uint32_t dh,
                             float scale, int causal, int scale_q_first, cudaStream_t s) {
    const size_t warps = static_cast<size_t>(seqs) * H * t;
    if (!warps) return cudaSuccess;
    const size_t tsmem = at_smem_floats(t) * sizeof(float);
    const bool aligned = (reinterpret_cast<uintptr_t>(qkv) & 15u) == 0 && (H * kAtDh * 3u) % 4u == 0;
    if (t > 32 && t <= kAttnMaxT && dh == kAtDh && aligned && tsmem <= 200 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(attention_tiled_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(tsmem));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(attention_tiled_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(tsmem));
        if (e != cudaSuccess) return e;
        // 4 queries a warp (32 a block); 2 (16 a block) when that leaves SMs
        // without a block (the ViT's 197 tokens x 3 heads x a few frames)
        const size_t blocks4 = static_cast<size_t>((t + kAtQ - 1) / kAtQ) * H * seqs;
        if (blocks4 < 148)
            return launch_pdl(attention_tiled_kernel<2>, dim3((t + 15) / 16, H, seqs), dim3(256), tsmem, s, qkv, out, t,
                              H, scale, causal, scale_q_first);
        return launch_pdl(attention_tiled_kernel<4>, dim3((t + kAtQ - 1) / kAtQ, H, seqs), dim3(256), tsmem, s, qkv, out, t,
                          H, scale, causal, scale_q_first);
    }
    const size_t smem = (static_cast<size_t>(t) * (2 * dh + 1) + 8 * t + 8 * dh) * sizeof(float);
    if (t > 32 && t <= kAttnMaxT && dh <= 128 && smem <= 200 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(attention_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        return launch_pdl(attention_smem_kernel, dim3((t + kAttnQ - 1) / kAttnQ, H, seqs), dim3(256), smem, s, qkv, out,
                          t, H, dh, scale, causal, scale_q_first);
    }
    return launch_pdl(attention_kernel, dim3(blocks_for(warps, 8)), dim3(256), 0, s, qkv, out, seqs, t, H, dh, scale,
                      causal, scale_q_first);
}

// The ActionEmbedder's first two layers for every (sample, time) token in
// one launch (modules.rs:150-158: patch_embed, a kernel-1 Conv1d over the
// action dim, then embed.0 with SiLU): y = silu(W1 (Wc a + bc) + b1).  Their
// K (the action dim, the smoothed dim) is too small for the tensor-core GEMM
// and the work is a few MFLOP, so two GEMM launches were all latency.  A
// block takes 4 tokens: the smoothed vectors go to shared memory, then each
// thread computes output columns tid, tid + 256, ... of the 4 tokens (sums in
// k order from 0, bias after, as the GEMM kernels do).
constexpr uint32_t kAeTok = 4, kAeMaxA = 8, kAeMaxSm = 64;
__global__ void __launch_bounds__(256) action_embed_kernel(const float* cand, uint32_t A, const float* wc,
                                                           const float* bc, uint32_t sm, const float* w1,
                                                           const float* b1, uint32_t ah, float* out, uint32_t rows) {
    __shared__ float s_sm[kAeTok][kAeMaxSm];
    const uint32_t r0 = blockIdx.x * kAeTok;
    {
        const uint32_t t = threadIdx.x / kAeMaxSm, k = threadIdx.x % kAeMaxSm;
        if (t < kAeTok && k < sm && r0 + t < rows) {
            const float* a = cand + static_cast<size_t>(r0 + t) * A;
            float acc = 0.0f;
            for (uint32_t i = 0; i < A; ++i) acc = fmaf(a[i], wc[static_cast<size_t>(k) * A + i], acc);
            s_sm[t][k] = bc ? acc + bc[k] : acc;
        }
    }
    __syncthreads();
    for (uint32_t j = threadIdx.x; j < ah; j += blockDim.x) {
        const float* wr = w1 + static_cast<size_t>(j) * sm;
        float acc[kAeTok] = {};
        for (uint32_t k = 0; k < sm; ++k) {
            const float wv = __ldg(wr + k);
#pragma unroll
            for (uint32_t t = 0; t < kAeTok; ++t) acc[t] = fmaf(s_sm[t][k], wv, acc[t]);
        }
        const float bias = b1 ? __ldg(b1 + j) : 0.0f;
#pragma unroll
        for (uint32_t t = 0; t < kAeTok; ++t)
            if (r0 + t < rows) out[static_cast<size_t>(r0 + t) * ah + j] = apply_act(kActSilu, b1 ? acc[t] + bias : acc[t]);
    }
}

bool action_embed_supported(uint32_t A, uint32_t sm) { return A >= 1 && A <= kAeMaxA && sm >= 1 && sm <= kAeMaxSm; }

cudaError_t launch_action_embed(const float* cand, uint32_t A, const float* wc, const float* bc, uint32_t sm,
                                const float* w1, const float* b1, uint32_t ah, float* out, uint32_t rows,
                                cudaStream_t s) {
    if (!rows) return cudaSuccess;
    if (!action_embed_supported(A, sm)) return cudaErrorInvalidValue;
    action_embed_kernel<<<(rows + kAeTok - 1) / kAeTok, 256, 0, s>>>(cand, A, wc, bc, sm, w1, b1, ah, out, rows);
    return cudaGetLastError();
}

cudaError_t launch_goal_cost(const float* pred, const float* goal, uint32_t S, size_t rows, uint32_t d,
                             float* scores, cudaStream_t s) {
    if (!rows) return cudaSuccess;
    goal_cost_kernel<<<blocks_for(rows, 8), 256, 0, s>>>(pred, goal, S, rows, d, scores);
    return cudaGetLastError();
}

cudaError_t launch_patchify(const float* pix, float* patches, uint32_t n, uint32_t C, uint32_t img, uint32_t p,
                            cudaStream_t s) {
    const size_t total = static_cast<size_t>(n) * (img / p) * (img / p) * C * p * p;
    if (!total) return cudaSuccess;
    patchify_kernel<<<blocks_for(total, 256), 256, 0, s>>>(pix, patches, n, C, img, p);
    return cudaGetLastError();
}

cudaError_t launch_vit_assemble(const float* patch_out, const float* cls, const float* pos, float* x, uint32_t n,
                                uint32_t np, uint32_t vh, cudaStream_t s) {
    const size_t total = static_cast<size_t>(n) * (np + 1) * vh;
    if (!total) return cudaSuccess;
    return launch_pdl(vit_assemble_kernel, dim3(blocks_for(total, 256)), dim3(256), 0, s, patch_out, cls, pos, x, n, np,
                      vh);
}

}  // namespace lwm
