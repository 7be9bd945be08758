// kernels_skyjepa_tc.cu — learned SkyJEPA MPPI on the 5th-generation tensor
// cores (tcgen05, bf16 operands, f32 accumulation in TMEM) for large
// candidate counts (the fleet: hundreds of vehicles x thousands of samples).
//
// Same computation as skyjepa_rollout_kernel (SkyJepaMppiScorer,
// src/models/skyjepa/control.rs:146-317; GRU rollout model.rs:105-223; TCN
// tcn.rs; prober prober.rs:84-138; integrator kinematics.rs:377-484; cost
// control.rs:430-452; MPPI src/planner.rs:1588-1602) with the recurrent GEMM
// on tensor cores:
//
//   per CTA, persistent over 128-candidate tiles of one vehicle; per step t
//   and per chunk of 32 hidden units (8 chunks):
//     D[128 x 128] = X_t[128 x 16] . Wx_c^T          (r | z | n_h | n_x cols)
//     D[:, 0:96]  += H_t[128 x 256] . Whh_c^T         (16 MMAs, K = 256)
//   then the GRU gates of those 32 units for the 128 rows (f32), with h_t in
//   TMEM twice: f32 (the recurrent state) and bf16 (the A operand of the
//   h-block MMAs, read by the tensor core straight from TMEM, so that shared
//   memory bandwidth goes to the weights alone).
//   The prober's first layer is one more MMA per step (A = h_{t+1}).
//
// Before it, the sampler draws the candidates and skyjepa_tc_inputs_seq_kernel
// computes every candidate's action-TCN input x_t for every step (one thread
// per candidate), written as bf16 K-major tiles with a constant 1 at k = E
// that carries the GRU biases through the x-block MMA.
//
// Roles (448 threads): warp 0 streams the weight chunks and the x tiles
// (bulk copies); warp 1 issues the MMAs and owns TMEM; warps 2-9 run the GRU
// epilogue (two warps per TMEM lane quadrant, 16 units each); warps 10-13
// (one thread per candidate) finish the prober, integrate, accumulate the
// cost and reduce the tile to an MPPI tuple.  All hand-offs are mbarriers
// with bounded waits; a wait that gives up records where and the kernel
// unwinds.
//
// TMEM (512 columns): one accumulator slot of 128 columns = [0,128); h_t as
// bf16 pairs = [128,256); h_t (f32) = [256,512).  The slot's consumers (GRU
// epilogue, prober) load it into registers and hand it back before their
// math, so the next chunk's MMAs overlap the gates of this one.  Weight
// chunks stream through a 3-deep shared-memory ring.  Weights are bf16
// (packed once per scorer by pack_tc_weights_kernel; the GRU biases ride in
// the x block); the prober's later layers, the TCN and the integrator stay f32.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "lwm_device.cuh"
#include "lwm_kernels.hpp"
#include "lwm_tc.cuh"
#include "lwm_skyjepa_tcn.cuh"

namespace lwm {

namespace {

constexpr uint32_t kRows = 128, kH = 256;
constexpr uint32_t kUnits = 32;                   // hidden units per chunk
constexpr uint32_t kChunks = kH / kUnits;         // 8 chunks per step
constexpr uint32_t kHRows = 3 * kUnits;           // B rows of the h part: r, z, n_h
constexpr uint32_t kXRows = 4 * kUnits;           // B rows of the x part: r, z, n_h, n_x
constexpr uint32_t kChunkHBytes = 4 * kHRows * 128;  // 4 K-blocks x 96 rows x 128 B (SW128)
constexpr uint32_t kChunkXBytes = kXRows * 32;       // 128 rows x 16 k (SW32)
constexpr uint32_t kChunkBytes = kChunkHBytes + kChunkXBytes;  // 52 KB, 1024-aligned
constexpr uint32_t kWStages = 3;                  // weight-chunk ring
constexpr uint32_t kSlots = 1, kSlotCols = kXRows; // accumulator: one slot of 128 TMEM columns
constexpr uint32_t kUPW = kUnits / 2;             // units per epilogue warp and chunk
constexpr uint32_t kACol = kSlots * kSlotCols;    // h_t as bf16 (the MMAs' A operand): TMEM columns [128, 256)
constexpr uint32_t kHCol = kACol + kH / 2;        // h (f32) lives in TMEM columns [256, 512)
static_assert(kHCol + kH == 512, "TMEM holds the slot, A and h");
constexpr uint32_t kEntries = kChunks + 1;        // accumulator-ring entries per step (chunks + prober)
constexpr uint32_t kXBytes = 128 * 32;
constexpr uint32_t kMaxHid = 32, kMaxLayers = 3;
constexpr uint32_t kP1Bytes = 4 * kMaxHid * 128;
constexpr uint32_t kPwFloats = kMaxHid + (kMaxLayers - 1) * (kMaxHid * kMaxHid + kMaxHid) + 16 * kMaxHid + 16;
constexpr uint32_t kTcnFloats = 1024;
constexpr uint32_t kTcnBlockFloats = 104, kTcnParamFloats = 3 * kTcnBlockFloats;  // the 4-channel, 3-level encoder
constexpr int kThreadsTc = 448;
constexpr uint32_t kAuxWarp0 = 10, kEpiWarp0 = 2;
constexpr uint32_t kAuxBarrier = 3, kAuxThreads = 128;
constexpr uint32_t kMaxHistTc = 16;

struct __align__(1024) TcSmem {
    uint8_t W[kWStages][kChunkBytes];
    uint8_t X[2][kXBytes];
    uint8_t P1[kP1Bytes];
    float pw[kPwFloats];  // prober: b1, hidden layers (W, b), output (W, b)
    float hst[kRows * (kMaxHid + 1)];  // prober hidden-layer outputs, one padded row per candidate
    float red_w[kRows];
    uint64_t red_key[4];
    float red_f[4];
    // accumulator slots are shared by two consumer groups (0: GRU epilogue,
    // 1: prober/aux); each group has its own full/empty barrier per slot so
    // every waiter sees every phase of the barriers it waits on
    uint64_t w_full[kWStages], w_empty[kWStages], full[2][kSlots], empty[2][kSlots], x_full[2], x_empty[2], h_full,
        a_read, done;
    uint32_t tmem;
    int last;
};

__device__ __forceinline__ void aux_sync() {
    asm volatile("bar.sync %0, %1;" ::"n"(kAuxBarrier), "n"(kAuxThreads) : "memory");
}

// True on every aux thread iff `v` is true on all of them (a barrier with an
// AND reduction).  The aux warps take every wait's outcome through it, so
// they leave their loop together and never meet aux_sync() short of a warp
// (a named barrier that a departed warp never reaches would not end).
__device__ __forceinline__ bool aux_all(bool v) {
    uint32_t out;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(out)
        : "r"(static_cast<uint32_t>(v)), "n"(kAuxBarrier), "n"(kAuxThreads)
        : "memory");
    return out != 0;
}

// The gates use the hardware tanh for sigmoid as well:
// sigmoid(v) = 0.5 + 0.5 tanh(v / 2).
__device__ __forceinline__ float sigmoid_f(float v) { return fmaf(0.5f, tanh_fast(0.5f * v), 0.5f); }

// Two f32 -> packed bf16x2 (the first value at the lower address).
__device__ __forceinline__ uint32_t bf2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}


// The element (row, k) of the prober / recurrent weights in the packed layouts.
__host__ __device__ inline uint32_t packed_h_offset(uint32_t j, uint32_t k, uint32_t rows) {
    return (k >> 6) * rows * 128u + tc::sw128_offset(j, k & 63u);
}

}  // namespace

// ------------------------------------------------------- weight packing
//
// Wc[chunk]: H part (rows r_u, z_u, n_u of the chunk's 16 units, K = 256 of
// weight_hh) in SW128 K-blocks, then the X part (rows r, z, n_h, n_x; k < E
// weight_ih (zero for n_h), k = E the biases) in SW32.  P1: prober input
// layer [hid x 256].
__global__ void pack_tc_weights_kernel(SkyjepaArgs a, uint8_t* wc, uint8_t* p1) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t n_h = static_cast<size_t>(kChunks) * kHRows * kH;
    const size_t n_x = static_cast<size_t>(kChunks) * kXRows * 16;
    const size_t n_p = static_cast<size_t>(a.hid) * kH;
    if (i < n_h) {
        const uint32_t c = static_cast<uint32_t>(i / (kHRows * kH)), rem = static_cast<uint32_t>(i % (kHRows * kH));
        const uint32_t j = rem / kH, k = rem % kH, g = j / kUnits, u = c * kUnits + j % kUnits;
        const float v = a.w_hh[static_cast<size_t>(g * kH + u) * kH + k];
        *reinterpret_cast<__nv_bfloat16*>(wc + static_cast<size_t>(c) * kChunkBytes + packed_h_offset(j, k, kHRows)) =
            __float2bfloat16_rn(v);
    } else if (i < n_h + n_x) {
        const size_t q = i - n_h;
        const uint32_t c = static_cast<uint32_t>(q / (kXRows * 16)), rem = static_cast<uint32_t>(q % (kXRows * 16));
        const uint32_t j = rem / 16, k = rem % 16, g = j / kUnits, u = c * kUnits + j % kUnits;
        float v = 0.0f;
        if (k < a.E && g != 2) {
            const uint32_t gate = g == 3 ? 2u : g;  // n_x uses weight_ih's n rows
            v = a.w_ih[static_cast<size_t>(gate * kH + u) * a.E + k];
        } else if (k == a.E) {
            // biases, multiplied by the constant 1 of the x tiles:
            // r: b_ir + b_hr, z: b_iz + b_hz, n_h: b_hn, n_x: b_in
            if (g == 0) v = a.b_ih[u] + a.b_hh[u];
            else if (g == 1) v = a.b_ih[kH + u] + a.b_hh[kH + u];
            else if (g == 2) v = a.b_hh[2 * kH + u];
            else v = a.b_ih[2 * kH + u];
        }
        *reinterpret_cast<__nv_bfloat16*>(wc + static_cast<size_t>(c) * kChunkBytes + kChunkHBytes +
                                          tc::sw32_offset(j, k)) = __float2bfloat16_rn(v);
    } else if (i < n_h + n_x + n_p) {
        const size_t q = i - n_h - n_x;
        const uint32_t j = static_cast<uint32_t>(q / kH), k = static_cast<uint32_t>(q % kH);
        *reinterpret_cast<__nv_bfloat16*>(p1 + packed_h_offset(j, k, a.hid)) =
            __float2bfloat16_rn(a.p_in_w[static_cast<size_t>(j) * kH + k]);
    }
}

// --------------------------------------------------- initial latent h0
//
// encode_state_history (model.rs:57-61): the state TCN over the normalised
// history, last step, state_projection.  One block per vehicle; one warp per
// output channel, its lanes striding the (input channel, tap) weights of that
// channel (contiguous in the blob) and a warp reduction per window position.
constexpr int kH0MaxHist = 16;

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Wide encoders (>= 64 channels): a warp per output channel, the lanes over
// the (input channel, tap) weights of that channel (coalesced weight rows).
__global__ void __launch_bounds__(256) skyjepa_h0_warp_kernel(SkyjepaArgs a, float* h0) {
    extern __shared__ float sh[];
    const uint32_t b = blockIdx.x, tid = threadIdx.x, Hs = a.Hs, warp = tid >> 5, lane = tid & 31;
    const uint32_t nwarps = blockDim.x >> 5;
    const TcnView& tcn = a.state_tcn;
    const uint32_t C = tcn.max_ch, K = tcn.k;
    float* cur = sh;                 // [C][Hs]
    float* h1 = cur + C * Hs;        // [C][Hs]
    float* h2 = h1 + C * Hs;         // [C][Hs]
    for (uint32_t q = tid; q < 18 * Hs; q += blockDim.x) {
        const uint32_t i = q / Hs, t = q % Hs;
        const float v = a.state_hist[(static_cast<size_t>(b) * Hs + t) * 18 + i];
        cur[i * Hs + t] = (v - a.state_mean[i]) / a.state_std[i];
    }
    __syncthreads();
    for (uint32_t l = 0; l < tcn.levels; ++l) {
        const TcnBlockView& bk = tcn.blocks[l];
        for (int conv = 0; conv < 2; ++conv) {
            const float* src = conv == 0 ? cur : h1;
            float* dst = conv == 0 ? h1 : h2;
            const uint32_t cin = conv == 0 ? bk.in : bk.out;
            const float* W = conv == 0 ? bk.w1 : bk.w2;
            const float* bias = conv == 0 ? bk.b1 : bk.b2;
            for (uint32_t o = warp; o < bk.out; o += nwarps) {
                float acc[kH0MaxHist];
#pragma unroll
                for (int t = 0; t < kH0MaxHist; ++t) acc[t] = 0.0f;
                const float* wo = W + static_cast<size_t>(o) * cin * K;
                for (uint32_t idx = lane; idx < cin * K; idx += 32) {
                    const uint32_t i = idx / K, jj = idx % K;
                    const float wv = __ldg(wo + idx);
                    const int shift = static_cast<int>((K - 1 - jj) * bk.dil);
                    const float* xi = src + i * Hs;
#pragma unroll
                    for (int t = 0; t < kH0MaxHist; ++t)
                        if (t < static_cast<int>(Hs) && t >= shift) acc[t] = fmaf(wv, xi[t - shift], acc[t]);
                }
#pragma unroll
                for (int t = 0; t < kH0MaxHist; ++t) {
                    const float v = warp_sum_f(acc[t]);
                    if (lane == 0 && t < static_cast<int>(Hs)) dst[o * Hs + t] = gelu_tanh(v + bias[o]);
                }
            }
            __syncthreads();
        }
        // residual (1x1 conv when the width changes) and the block output, into h1
        for (uint32_t o = warp; o < bk.out; o += nwarps) {
            float res[kH0MaxHist];
#pragma unroll
            for (int t = 0; t < kH0MaxHist; ++t) res[t] = 0.0f;
            if (bk.wr) {
                for (uint32_t i = lane; i < bk.in; i += 32) {
                    const float wv = __ldg(bk.wr + static_cast<size_t>(o) * bk.in + i);
#pragma unroll
                    for (int t = 0; t < kH0MaxHist; ++t)
                        if (t < static_cast<int>(Hs)) res[t] = fmaf(wv, cur[i * Hs + t], res[t]);
                }
#pragma unroll
                for (int t = 0; t < kH0MaxHist; ++t) res[t] = warp_sum_f(res[t]) + bk.br[o];
            } else {
#pragma unroll
                for (int t = 0; t < kH0MaxHist; ++t)
                    if (t < static_cast<int>(Hs)) res[t] = cur[o * Hs + t];
            }
            if (lane == 0)
                for (uint32_t t = 0; t < Hs; ++t) h1[o * Hs + t] = gelu_tanh(h2[o * Hs + t] + res[t]);
        }
        __syncthreads();
        for (uint32_t q = tid; q < bk.out * Hs; q += blockDim.x) cur[q] = h1[q];
        __syncthreads();
    }
    for (uint32_t u = warp; u < a.H; u += nwarps) {
        float acc = 0.0f;
        for (uint32_t c = lane; c < tcn.out_dim; c += 32)
            acc = fmaf(__ldg(a.proj_w + static_cast<size_t>(u) * tcn.out_dim + c), cur[c * Hs + Hs - 1], acc);
        acc = warp_sum_f(acc);
        if (lane == 0) h0[static_cast<size_t>(b) * a.H + u] = acc + a.proj_b[u];
    }
}

// Narrow encoders: one CTA per vehicle, every convolution a thread per (output channel,
// position) over the vehicle's [C][Hs] activations in shared memory; the
// threads of one channel read the same weights (L1 broadcast) and the
// taps run in (input channel, tap) order.
__global__ void __launch_bounds__(256) skyjepa_h0_kernel(SkyjepaArgs a, float* h0) {
    extern __shared__ float sh[];
    const uint32_t b = blockIdx.x, tid = threadIdx.x, Hs = a.Hs, nt = blockDim.x;
    const TcnView& tcn = a.state_tcn;
    const uint32_t C = tcn.max_ch, K = tcn.k;
    float* cur = sh;                 // [C][Hs]
    float* h1 = cur + C * Hs;        // [C][Hs]
    float* h2 = h1 + C * Hs;         // [C][Hs]
    for (uint32_t q = tid; q < 18 * Hs; q += nt) {
        const uint32_t i = q / Hs, t = q % Hs;
        const float v = a.state_hist[(static_cast<size_t>(b) * Hs + t) * 18 + i];
        cur[i * Hs + t] = (v - a.state_mean[i]) / a.state_std[i];
    }
    __syncthreads();
    for (uint32_t l = 0; l < tcn.levels; ++l) {
        const TcnBlockView& bk = tcn.blocks[l];
        for (int conv = 0; conv < 2; ++conv) {
            const float* src = conv == 0 ? cur : h1;
            float* dst = conv == 0 ? h1 : h2;
            const uint32_t cin = conv == 0 ? bk.in : bk.out;
            const float* W = conv == 0 ? bk.w1 : bk.w2;
            const float* bias = conv == 0 ? bk.b1 : bk.b2;
            for (uint32_t q = tid; q < bk.out * Hs; q += nt) {
                const uint32_t o = q / Hs, t = q % Hs;
                const float* wo = W + static_cast<size_t>(o) * cin * K;
                float acc = 0.0f;
                for (uint32_t i = 0; i < cin; ++i)
                    for (uint32_t j = 0; j < K; ++j) {
                        const uint32_t shift = (K - 1 - j) * bk.dil;
                        if (t >= shift) acc = fmaf(__ldg(wo + i * K + j), src[i * Hs + t - shift], acc);
                    }
                dst[o * Hs + t] = gelu_tanh(acc + __ldg(bias + o));
            }
            __syncthreads();
        }
        // residual (1x1 conv when the width changes) and the block output
        for (uint32_t q = tid; q < bk.out * Hs; q += nt) {
            const uint32_t o = q / Hs, t = q % Hs;
            float res;
            if (bk.wr) {
                float r = 0.0f;
                for (uint32_t i = 0; i < bk.in; ++i) r = fmaf(__ldg(bk.wr + static_cast<size_t>(o) * bk.in + i), cur[i * Hs + t], r);
                res = r + __ldg(bk.br + o);
            } else {
                res = cur[o * Hs + t];
            }
            h1[o * Hs + t] = gelu_tanh(h2[o * Hs + t] + res);
        }
        __syncthreads();
        for (uint32_t q = tid; q < bk.out * Hs; q += nt) cur[q] = h1[q];
        __syncthreads();
    }
    // state_projection of the last position
    for (uint32_t u = tid; u < a.H; u += nt) {
        const float* wu = a.proj_w + static_cast<size_t>(u) * tcn.out_dim;
        float acc = 0.0f;
        for (uint32_t c = 0; c < tcn.out_dim; ++c) acc = fmaf(__ldg(wu + c), cur[c * Hs + Hs - 1], acc);
        h0[static_cast<size_t>(b) * a.H + u] = acc + a.proj_b[u];
    }
}

// Many vehicles: the encoder runs layer by layer over the whole fleet, a
// thread per (vehicle, output channel) over all HS positions, activations in
// global scratch laid out [channel][vehicle][position] so that a warp's 32
// vehicles read one contiguous run per input channel (and share each weight:
// a broadcast load).  Same (input channel, tap) summation order as
// skyjepa_h0_kernel.  Launches: normalise, then per level conv1 and
// conv2 + residual + block output, then the projection.
template <int HS>
__global__ void __launch_bounds__(256) h0_normalise_kernel(SkyjepaArgs a, float* x /*[18][B][HS]*/) {
    const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;  // (b, t, i) in the history's order
    if (q >= a.B * HS * 18u) return;
    const uint32_t i = q % 18u, bt = q / 18u;
    x[static_cast<size_t>(i) * a.B * HS + bt] = (a.state_hist[q] - a.state_mean[i]) / a.state_std[i];
}

// conv == 1: out = gelu(conv1(in) + b1).  conv == 2: out = gelu(gelu(conv2(in)
// + b2) + res), res = wr . res_in + br (1x1, width change) or res_in itself.
template <int HS>
__global__ void __launch_bounds__(256) h0_conv_kernel(const float* __restrict__ in, const float* __restrict__ W,
                                                      const float* __restrict__ bias, uint32_t cin, uint32_t cout,
                                                      uint32_t B, uint32_t dil, int conv,
                                                      const float* __restrict__ res_in,
                                                      const float* __restrict__ wr, const float* __restrict__ br,
                                                      uint32_t cres, float* __restrict__ out) {
    constexpr int K = 3;
    const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= cout * B) return;
    const uint32_t o = q / B, b = q % B;
    const size_t plane = static_cast<size_t>(B) * HS;
    float acc[HS];
#pragma unroll
    for (int t = 0; t < HS; ++t) acc[t] = 0.0f;
    const float* wo = W + static_cast<size_t>(o) * cin * K;
    for (uint32_t i = 0; i < cin; ++i) {
        const float* xi = in + i * plane + static_cast<size_t>(b) * HS;
        float xv[HS];
#pragma unroll
        for (int t = 0; t < HS; ++t) xv[t] = xi[t];
#pragma unroll
        for (int j = 0; j < K; ++j) {
            const float wv = __ldg(wo + i * K + j);
            const uint32_t shift = static_cast<uint32_t>(K - 1 - j) * dil;
#pragma unroll
            for (int t = 0; t < HS; ++t)
                if (static_cast<uint32_t>(t) >= shift) acc[t] = fmaf(wv, xv[t - shift], acc[t]);
        }
    }
    const float bo = __ldg(bias + o);
    float* dst = out + o * plane + static_cast<size_t>(b) * HS;
    if (conv == 1) {
#pragma unroll
        for (int t = 0; t < HS; ++t) dst[t] = gelu_tanh(acc[t] + bo);
        return;
    }
    float res[HS];
    if (wr) {
#pragma unroll
        for (int t = 0; t < HS; ++t) res[t] = 0.0f;
        const float* wro = wr + static_cast<size_t>(o) * cres;
        for (uint32_t i = 0; i < cres; ++i) {
            const float wv = __ldg(wro + i);
            const float* xi = res_in + i * plane + static_cast<size_t>(b) * HS;
#pragma unroll
            for (int t = 0; t < HS; ++t) res[t] = fmaf(wv, xi[t], res[t]);
        }
        const float bro = __ldg(br + o);
#pragma unroll
        for (int t = 0; t < HS; ++t) res[t] = res[t] + bro;
    } else {
        const float* xo = res_in + o * plane + static_cast<size_t>(b) * HS;
#pragma unroll
        for (int t = 0; t < HS; ++t) res[t] = xo[t];
    }
#pragma unroll
    for (int t = 0; t < HS; ++t) dst[t] = gelu_tanh(gelu_tanh(acc[t] + bo) + res[t]);
}

// state_projection of the last position: a thread per (vehicle, latent unit).
template <int HS>
__global__ void __launch_bounds__(256) h0_project_kernel(SkyjepaArgs a, const float* __restrict__ cur, float* h0) {
    const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= a.H * a.B) return;
    const uint32_t u = q / a.B, b = q % a.B;
    const size_t plane = static_cast<size_t>(a.B) * HS;
    const float* wu = a.proj_w + static_cast<size_t>(u) * a.state_tcn.out_dim;
    float acc = 0.0f;
    for (uint32_t c = 0; c < a.state_tcn.out_dim; ++c)
        acc = fmaf(__ldg(wu + c), cur[c * plane + static_cast<size_t>(b) * HS + HS - 1], acc);
    h0[static_cast<size_t>(b) * a.H + u] = acc + a.proj_b[u];
}

constexpr uint32_t kH0BatchedMinVehicles = 32, kH0BatchedHist = 10;

size_t skyjepa_h0_work_bytes(const SkyjepaArgs& a, uint32_t B) {
    const uint32_t C = a.state_tcn.max_ch > 18u ? a.state_tcn.max_ch : 18u;
    return 3 * static_cast<size_t>(C) * B * kH0BatchedHist * sizeof(float);
}

namespace {

cudaError_t launch_h0_batched(const SkyjepaArgs& a, float* h0, cudaStream_t stream) {
    constexpr int HS = static_cast<int>(kH0BatchedHist);
    const uint32_t B = a.B, C = a.state_tcn.max_ch > 18u ? a.state_tcn.max_ch : 18u;
    const size_t buf = static_cast<size_t>(C) * B * HS;
    float* cur = a.h0_work;
    float* h1 = cur + buf;
    float* nxt = h1 + buf;
    const uint32_t n_in = B * HS * 18u;
    h0_normalise_kernel<HS><<<(n_in + 255) / 256, 256, 0, stream>>>(a, cur);
    for (uint32_t l = 0; l < a.state_tcn.levels; ++l) {
        const TcnBlockView& bk = a.state_tcn.blocks[l];
        const uint32_t n = bk.out * B;
        h0_conv_kernel<HS><<<(n + 255) / 256, 256, 0, stream>>>(cur, bk.w1, bk.b1, bk.in, bk.out, B, bk.dil, 1,
                                                                 nullptr, nullptr, nullptr, 0, h1);
        h0_conv_kernel<HS><<<(n + 255) / 256, 256, 0, stream>>>(h1, bk.w2, bk.b2, bk.out, bk.out, B, bk.dil, 2, cur,
                                                                 bk.wr, bk.br, bk.in, nxt);
        float* t = cur;
        cur = nxt;
        nxt = t;
    }
    const uint32_t n = a.H * B;
    h0_project_kernel<HS><<<(n + 255) / 256, 256, 0, stream>>>(a, cur, h0);
    return cudaGetLastError();
}

}  // namespace

// h0 of every vehicle: state_projection(TemporalConvEncoder(normalised state
// history))[last position] (SkyJepaModel::encode_history, model.rs:52-66).
cudaError_t launch_skyjepa_h0(const SkyjepaArgs& a, float* h0, cudaStream_t stream) {
    if (a.Hs > kH0MaxHist) return cudaErrorInvalidValue;
    // the default encoder: one 16-CTA cluster per vehicle, pruned to what the
    // last output depends on (one launch; 256 vehicles in 0.21 ms, against
    // 1.07 ms for the batched per-layer kernels below)
    if (skyjepa_h0_pruned_supported(a)) return launch_skyjepa_h0_pruned(a, h0, stream);
    if (a.h0_work && a.B >= kH0BatchedMinVehicles && a.Hs == kH0BatchedHist && a.state_tcn.k == 3)
        return launch_h0_batched(a, h0, stream);
    // few vehicles, wide encoder: one 8-CTA cluster per vehicle (weights
    // staged in shared memory, output channels split over the cluster)
    if (a.state_tcn.max_ch >= 64) return launch_skyjepa_h0_cluster(a, h0, stream);
    const size_t h0_smem = static_cast<size_t>(a.state_tcn.max_ch) * a.Hs * 3 * sizeof(float);
    if (a.state_tcn.max_ch >= 64)
        skyjepa_h0_warp_kernel<<<a.B, 256, h0_smem, stream>>>(a, h0);
    else
        skyjepa_h0_kernel<<<a.B, 256, h0_smem, stream>>>(a, h0);
    return cudaGetLastError();
}

namespace {

}  // namespace

// ------------------------------------------------------ per-step inputs
//
// x_t of every candidate and step (the action TCN over the window
// [history ++ candidate](t : t + 10), last position), one thread per
// (candidate, step), written as the bf16 x tile of (tile, step): rows = the
// tile's 128 candidates, k < 4 the encoder output, k = 4 the constant 1.
//
// The encoder's 312 weights come as a kernel parameter: with every index a
// compile-time constant after unrolling, the FMAs read them from the constant
// bank directly instead of through shared-memory loads.
struct TcnConst {
    float v[kTcnParamFloats];  // per level: conv1 weight [4][4][3], bias [4], conv2 weight, bias
};

// The same inputs, one thread per candidate walking its steps in order.
// The window of step t is the sequence positions t .. t + 9; a block-1
// value at window position p >= 2 (conv1) or p >= 4 (block output) reads no
// zero padding, so it is a function of its sequence position alone and is
// computed once, when it first enters a window (at p = 9), then slides down
// with the window.  Only the padded edge values (conv1 at p = 0, 1; block 1
// at p = 1, 3) and blocks 2 and 3 are evaluated per window.  Every
// convolution sums its taps in conv_at's order and the GELU is the fast
// GELU with its operations regrouped (gelu_fast5), so x_t is tcn_last's
// value for the window up to the last bits of each GELU.
// The fast GELU in five arithmetic operations and one MUFU: 0.5 v (1 + tanh(u))
// = h + h tanh(u) with h = v / 2 and u = v (c0 + c1 v^2), c0 = sqrt(2 / pi),
// c1 = 0.044715 c0 (gelu_fast's function, operations regrouped).
__device__ __forceinline__ float gelu_fast5(float v) {
    const float u = v * fmaf(0.7978845608028654f * 0.044715f, v * v, 0.7978845608028654f);
    const float h = 0.5f * v;
    return fmaf(h, tanh_fast(u), h);
}

template <bool kTap0, bool kTap1>
__device__ __forceinline__ void conv3(const float* W, const float* B, const float (&x0)[kTcnC], const float (&x1)[kTcnC],
                                      const float (&x2)[kTcnC], float (&out)[kTcnC]) {
#pragma unroll
    for (int o = 0; o < kTcnC; ++o) {
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < kTcnC; ++i) {
            if (kTap0) acc = fmaf(W[(o * kTcnC + i) * kTcnK + 0], x0[i], acc);
            if (kTap1) acc = fmaf(W[(o * kTcnC + i) * kTcnK + 1], x1[i], acc);
            acc = fmaf(W[(o * kTcnC + i) * kTcnK + 2], x2[i], acc);
        }
        out[o] = gelu_fast5(acc + B[o]);
    }
}

// gelu(conv2(taps) + residual): a block's output at one position
template <bool kTap0, bool kTap1>
__device__ __forceinline__ void block3(const TcnBlockW& w, const float (&h0)[kTcnC], const float (&h1)[kTcnC],
                                       const float (&h2)[kTcnC], const float (&res)[kTcnC], float (&out)[kTcnC]) {
    float c[kTcnC];
    conv3<kTap0, kTap1>(w.w2, w.b2, h0, h1, h2, c);
#pragma unroll
    for (int o = 0; o < kTcnC; ++o) out[o] = gelu_fast5(c[o] + res[o]);
}

__global__ void __launch_bounds__(128) skyjepa_tc_inputs_seq_kernel(SkyjepaArgs a, const __grid_constant__ TcnConst tw,
                                                                    uint8_t* xtiles) {
    const uint64_t grow = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // b * S + s
    if (grow >= static_cast<uint64_t>(a.B) * a.S) return;
    const uint32_t b = static_cast<uint32_t>(grow / a.S), T = a.T;
    TcnBlockW w[3];
#pragma unroll
    for (int l = 0; l < 3; ++l) {
        const float* blk = tw.v + l * kTcnBlockFloats;
        w[l] = {blk, blk + 48, blk + 52, blk + 100};
    }
    const float* cand = a.cand_out + grow * T * 4;
    const float* hist = a.action_hist + static_cast<size_t>(b) * (kTcnHs - 1) * 4;
    float mean[4], inv[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) { mean[c] = a.action_mean[c]; inv[c] = a.action_std[c]; }
    auto load = [&](uint32_t pos, float (&v)[kTcnC]) {
        const float4 f = *reinterpret_cast<const float4*>(pos < kTcnHs - 1 ? hist + pos * 4 : cand + (pos - (kTcnHs - 1)) * 4);
        v[0] = (f.x - mean[0]) / inv[0];
        v[1] = (f.y - mean[1]) / inv[1];
        v[2] = (f.z - mean[2]) / inv[2];
        v[3] = (f.w - mean[3]) / inv[3];
    };
    // window of step 0; block-1 values that read no padding: conv1 at 2..8, output at 4..8
    float x[kTcnHs][kTcnC], c1[kTcnHs][kTcnC], y1[kTcnHs][kTcnC];
#pragma unroll
    for (int q = 0; q < kTcnHs; ++q) load(q, x[q]);
#pragma unroll
    for (int q = 2; q < kTcnHs - 1; ++q) conv3<true, true>(w[0].w1, w[0].b1, x[q - 2], x[q - 1], x[q], c1[q]);
#pragma unroll
    for (int q = 4; q < kTcnHs - 1; ++q) block3<true, true>(w[0], c1[q - 2], c1[q - 1], c1[q], x[q], y1[q]);
    const uint64_t tile = grow / kRows;
    const uint32_t row = static_cast<uint32_t>(grow % kRows);
    for (uint32_t t = 0; t < T; ++t) {
        if (t > 0) {
#pragma unroll
            for (int q = 0; q + 1 < kTcnHs; ++q)
#pragma unroll
                for (int c = 0; c < kTcnC; ++c) x[q][c] = x[q + 1][c];
#pragma unroll
            for (int q = 2; q + 1 < kTcnHs; ++q)
#pragma unroll
                for (int c = 0; c < kTcnC; ++c) c1[q][c] = c1[q + 1][c];
#pragma unroll
            for (int q = 4; q + 1 < kTcnHs; ++q)
#pragma unroll
                for (int c = 0; c < kTcnC; ++c) y1[q][c] = y1[q + 1][c];
            load(t + kTcnHs - 1, x[kTcnHs - 1]);
        }
        // the window's new position 9
        conv3<true, true>(w[0].w1, w[0].b1, x[7], x[8], x[9], c1[9]);
        block3<true, true>(w[0], c1[7], c1[8], c1[9], x[9], y1[9]);
        // block 1 at the padded edge: conv1 at 0, 1; output at 1, 3
        float e0[kTcnC], e1[kTcnC], y1_1[kTcnC], y1_3[kTcnC];
        conv3<false, false>(w[0].w1, w[0].b1, x[0], x[0], x[0], e0);
        conv3<false, true>(w[0].w1, w[0].b1, x[0], x[0], x[1], e1);
        block3<false, true>(w[0], e0, e0, e1, x[1], y1_1);
        block3<true, true>(w[0], e1, c1[2], c1[3], x[3], y1_3);
        // block 2 (dilation 2): conv1 at odd positions, output at 1, 5, 9
        float h1[kTcnC], h3[kTcnC], h5[kTcnC], h7[kTcnC], h9[kTcnC];
        conv3<false, false>(w[1].w1, w[1].b1, y1_1, y1_1, y1_1, h1);
        conv3<false, true>(w[1].w1, w[1].b1, y1_1, y1_1, y1_3, h3);
        conv3<true, true>(w[1].w1, w[1].b1, y1_1, y1_3, y1[5], h5);
        conv3<true, true>(w[1].w1, w[1].b1, y1_3, y1[5], y1[7], h7);
        conv3<true, true>(w[1].w1, w[1].b1, y1[5], y1[7], y1[9], h9);
        float y2_1[kTcnC], y2_5[kTcnC], y2_9[kTcnC];
        block3<false, false>(w[1], h1, h1, h1, y1_1, y2_1);
        block3<true, true>(w[1], h1, h3, h5, y1[5], y2_5);
        block3<true, true>(w[1], h5, h7, h9, y1[9], y2_9);
        // block 3 (dilation 4): conv1 at 1, 5, 9, output at 9
        float g1[kTcnC], g5[kTcnC], g9[kTcnC], xo[kTcnC];
        conv3<false, false>(w[2].w1, w[2].b1, y2_1, y2_1, y2_1, g1);
        conv3<false, true>(w[2].w1, w[2].b1, y2_1, y2_1, y2_5, g5);
        conv3<true, true>(w[2].w1, w[2].b1, y2_1, y2_5, y2_9, g9);
        block3<true, true>(w[2], g1, g5, g9, y2_9, xo);
        uint8_t* xt = xtiles + (tile * T + t) * kXBytes;
        *reinterpret_cast<uint4*>(xt + tc::sw32_offset(row, 0)) =
            make_uint4(bf2(xo[0], xo[1]), bf2(xo[2], xo[3]), bf2(1.0f, 0.0f), 0u);
        *reinterpret_cast<uint4*>(xt + tc::sw32_offset(row, 8)) = make_uint4(0u, 0u, 0u, 0u);
    }
}

// ------------------------------------------------------------ main kernel

namespace {

struct TcArgs {
    SkyjepaArgs a;
    const uint8_t* wc;  // packed chunks
    const uint8_t* p1;  // packed prober layer 1
    const float* h0;    // [B, 256]
    const uint8_t* xt;  // x tiles [tiles][T][kXBytes]
    uint32_t tiles_per_vehicle, tiles;
    int* err;
    uint32_t wait_polls;     // polls before a pipeline wait gives up
    uint32_t skip_h_arrive;  // fault injection: CTA 0's first GRU-epilogue warp skips its first h_full arrival
};

}  // namespace

__global__ void __launch_bounds__(kThreadsTc, 1) skyjepa_tc_kernel(TcArgs p) {
    extern __shared__ uint8_t smem_raw[];
    TcSmem& s = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const SkyjepaArgs& a = p.a;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t T = a.T, hid = a.hid;
    volatile int* err = p.err;
    const uint32_t lim = p.wait_polls;

    // ---- setup: barriers, TMEM, resident weights
    if (tid == 0) {
        for (uint32_t i = 0; i < kWStages; ++i) {
            tc::mbar_init(&s.w_full[i], 1);
            tc::mbar_init(&s.w_empty[i], 1);
        }
        for (uint32_t i = 0; i < kSlots; ++i) {
            tc::mbar_init(&s.full[0][i], 1);
            tc::mbar_init(&s.full[1][i], 1);
            tc::mbar_init(&s.empty[0][i], 8);
            tc::mbar_init(&s.empty[1][i], 4);
        }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&s.x_full[i], 1);
            tc::mbar_init(&s.x_empty[i], 1);
        }
        tc::mbar_init(&s.h_full, 8);
        tc::mbar_init(&s.a_read, 1);
        tc::mbar_init(&s.done, 1);
        tc::mbar_fence_init();
    }
    if (warp == 1) tc::tmem_alloc(&s.tmem, 512);
    for (uint32_t q = tid; q < kP1Bytes / 16; q += kThreadsTc)
        reinterpret_cast<uint4*>(s.P1)[q] =
            q < hid * 4 * 128 / 16 ? reinterpret_cast<const uint4*>(p.p1)[q] : make_uint4(0, 0, 0, 0);
    {
        // prober: b1 [hid], hidden l: W [hid*hid], b [hid], output W [15*hid], b [15]
        float* pw = s.pw;
        for (uint32_t q = tid; q < hid; q += kThreadsTc) pw[q] = a.p_in_b[q];
        uint32_t off = hid;
        for (uint32_t l = 0; l + 1 < a.prober_layers; ++l) {
            for (uint32_t q = tid; q < hid * hid; q += kThreadsTc) pw[off + q] = a.p_hid_w[l][q];
            for (uint32_t q = tid; q < hid; q += kThreadsTc) pw[off + hid * hid + q] = a.p_hid_b[l][q];
            off += hid * hid + hid;
        }
        for (uint32_t q = tid; q < 15 * hid; q += kThreadsTc) pw[off + q] = a.p_out_w[q];
        for (uint32_t q = tid; q < 15; q += kThreadsTc) pw[off + 15 * hid + q] = a.p_out_b[q];
    }
    tc::fence_async_smem();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = s.tmem;
    const uint32_t entries = kEntries * T + 1;  // acc-ring entries per tile

    if (warp == 0) {
        // ================= producer: weight chunks (kWStages-deep ring), x tiles (2 slots)
        if (lane == 0) {
            uint32_t j = 0, xs = 0;
            for (uint32_t tile = blockIdx.x; tile < p.tiles && !err[0]; tile += gridDim.x)
                for (uint32_t t = 0; t < T && !err[0]; ++t, ++xs) {
                    const uint32_t xslot = xs & 1u;
                    if (!tc::mbar_wait(&s.x_empty[xslot], ((xs >> 1) & 1u) ^ 1u, err, 8, xs, lim)) break;
                    tc::mbar_expect_tx(&s.x_full[xslot], kXBytes);
                    tc::bulk_g2s(s.X[xslot], p.xt + (static_cast<size_t>(tile) * T + t) * kXBytes, kXBytes,
                                 &s.x_full[xslot]);
                    for (uint32_t c = 0; c < kChunks; ++c, ++j) {
                        const uint32_t slot = j % kWStages, n = j / kWStages;
                        if (!tc::mbar_wait(&s.w_empty[slot], (n & 1u) ^ 1u, err, 1, j, lim)) break;
                        tc::mbar_expect_tx(&s.w_full[slot], kChunkBytes);
                        tc::bulk_g2s(s.W[slot], p.wc + static_cast<size_t>(c) * kChunkBytes, kChunkBytes,
                                     &s.w_full[slot]);
                    }
                }
            // j weight chunks and xs x tiles were issued; when a wait gave up,
            // the last ones may not have been consumed: they land before the
            // CTA exits (each slot's last phase completes once its copy has)
            for (uint32_t sl = 0; sl < kWStages; ++sl)
                if (j > sl) {
                    const uint32_t last = sl + ((j - 1u - sl) / kWStages) * kWStages;
                    tc::mbar_wait_landing(&s.w_full[sl], (last / kWStages) & 1u, lim);
                }
            for (uint32_t sl = 0; sl < 2u; ++sl)
                if (xs > sl) {
                    const uint32_t last = sl + ((xs - 1u - sl) / 2u) * 2u;
                    tc::mbar_wait_landing(&s.x_full[sl], (last >> 1) & 1u, lim);
                }
        }
    } else if (warp == 1) {
        // ================= MMA issuer (the whole warp, converged; one elected lane issues)
        {
            const uint32_t id_gru_x = tc::idesc_bf16_f32(128, kXRows), id_gru_h = tc::idesc_bf16_f32(128, kHRows);
            const uint32_t id_prob = tc::idesc_bf16_f32(128, hid);
            const uint32_t a_tmem = tmem + kACol;
            // every lane waits; the outcome is the warp's (a diverged lane would leave elect.sync short)
            auto wwait = [&](uint64_t* bar, uint32_t parity, volatile int* e, int site, uint32_t detail,
                             uint32_t limit) -> bool {
                return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity, e, site, static_cast<int>(detail), limit));
            };
            // descriptors built once; a K step or a ring slot only adds to the start-address
            // field (address >> 4, every address of the ring stays below 2^18)
            const uint64_t p_desc = tc::smem_desc(tc::smem_u32(s.P1), 16, 1024, tc::kSwizzle128);
            const uint64_t wh_desc = tc::smem_desc(tc::smem_u32(s.W[0]), 16, 1024, tc::kSwizzle128);
            const uint64_t wx_desc = tc::smem_desc(tc::smem_u32(s.W[0]) + kChunkHBytes, 16, 256, tc::kSwizzle32);
            const uint64_t x_desc = tc::smem_desc(tc::smem_u32(s.X[0]), 16, 256, tc::kSwizzle32);
            uint32_t j = 0, K = 0, xs = 0, hq = 0, wslot = 0, wphase = 0;
            // per (group g, slot) the parity of its publications, bit 2 g + slot; per slot
            // whether it was published (bit slot of `used`) and to which group (bit slot of
            // `last_g`).  Bit masks rather than small arrays: a runtime index into an array
            // would place it in local memory.
            uint32_t uses = 0, used = 0, last_g = 0;
            // entry K goes to slot K % kSlots: wait until the slot's previous consumer group released it
            auto acc_slot = [&](uint32_t k, uint32_t& col) -> bool {
                const uint32_t slot = k % kSlots;
                col = slot * kSlotCols;
                if (!((used >> slot) & 1u)) return true;
                const uint32_t g = (last_g >> slot) & 1u;
                return wwait(&s.empty[g][slot], ((uses >> (2u * g + slot)) & 1u) ^ 1u, err, 5, k, lim);
            };
            auto publish = [&](uint32_t k, uint32_t g) {
                const uint32_t slot = k % kSlots;
                tc::commit_w(&s.full[g][slot]);
                uses ^= 1u << (2u * g + slot);
                used |= 1u << slot;
                last_g = (last_g & ~(1u << slot)) | (g << slot);
            };
            auto prober = [&](bool real) -> bool {
                uint32_t col;
                if (!acc_slot(K, col)) return false;
                tc::fence_after();
                if (real) {
#pragma unroll
                    for (uint32_t ks = 0; ks < 16; ++ks)
                        tc::mma_bf16_ta_w(tmem + col, a_tmem + ks * 8,
                                        p_desc + (((ks >> 2) * kMaxHid * 128 + (ks & 3u) * 32) >> 4), id_prob, ks > 0);
                }
                publish(K, 1u);
                ++K;
                return true;
            };
            bool ok = true;
            for (uint32_t tile = blockIdx.x; ok && tile < p.tiles; tile += gridDim.x) {
                for (uint32_t t = 0; ok && t < T; ++t) {
                    ok = wwait(&s.h_full, hq & 1u, err, 2, hq, lim);  // A holds h_t
                    ++hq;
                    const uint32_t xslot = xs & 1u;
                    if (ok) ok = wwait(&s.x_full[xslot], (xs >> 1) & 1u, err, 3, xs, lim);
                    for (uint32_t c = 0; ok && c < kChunks; ++c, ++j) {
                        if (c == 1 && !(ok = prober(t > 0))) break;  // prober of step t-1 (A = h_t)
                        if (!(ok = wwait(&s.w_full[wslot], wphase, err, 4, j, lim))) break;
                        uint32_t col;
                        if (!(ok = acc_slot(K, col))) break;
                        tc::fence_after();
                        const uint64_t wo = static_cast<uint64_t>(wslot * (kChunkBytes >> 4));
                        tc::mma_bf16_w(tmem + col, x_desc + xslot * (kXBytes >> 4), wx_desc + wo, id_gru_x, 0);
#pragma unroll
                        for (uint32_t ks = 0; ks < 16; ++ks)
                            tc::mma_bf16_ta_w(tmem + col, a_tmem + ks * 8,
                                            wh_desc + wo + (((ks >> 2) * kHRows * 128 + (ks & 3u) * 32) >> 4), id_gru_h, 1);
                        publish(K, 0u);
                        tc::commit_w(&s.w_empty[wslot]);
                        if (c == kChunks - 1) tc::commit_w(&s.x_empty[xslot]);
                        ++K;
                        if (++wslot == kWStages) { wslot = 0; wphase ^= 1u; }
                    }
                    ++xs;
                }
                if (ok) ok = wwait(&s.h_full, hq & 1u, err, 2, hq, lim);  // A holds h_T
                ++hq;
                if (ok) ok = prober(true);                           // prober of step T-1
                if (ok) tc::commit_w(&s.a_read);                       // A is no longer read in this tile
            }
            // every MMA issued has completed before TMEM is released
            tc::commit_w(&s.done);
            tc::mbar_wait_landing(&s.done, 0, lim);
        }
    } else if (warp < kAuxWarp0) {
        // ================= GRU epilogue: quadrant q, units [kUPW half, kUPW (half + 1)) of each chunk
        const uint32_t q = warp & 3u, half = (warp - kEpiWarp0) >> 2;
        const uint32_t lane_base = tmem + ((q * 32) << 16);
        uint32_t K0 = 0;  // acc-ring entry index of the tile's first entry
        uint32_t eu = 0, tiles_done = 0;  // bit slot: phase parity of full[0][slot]
        bool ok = true;
        for (uint32_t tile = blockIdx.x; ok && tile < p.tiles; tile += gridDim.x) {
            const uint32_t b = tile / p.tiles_per_vehicle;
            if (tiles_done > 0) {
                // the previous tile's last prober MMA read A: wait for it before overwriting
                if (!(ok = tc::mbar_wait(&s.a_read, (tiles_done - 1) & 1u, err, 7, tiles_done, lim))) break;
                tc::fence_after();
            }
            // h0 of the vehicle -> H (TMEM f32) and A (bf16), this warp's units
            // this warp's units: kUPW of every chunk, u = kUnits c + kUPW half + i
            for (uint32_t c = 0; c < kChunks; ++c)
                for (uint32_t g8 = 0; g8 < kUPW; g8 += 8) {
                    const uint32_t u0 = c * kUnits + half * kUPW + g8;
                    float hv[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) hv[i] = __ldg(p.h0 + static_cast<size_t>(b) * kH + u0 + i);
                    tc::tmem_st8(lane_base + kHCol + u0, hv);
                    const uint32_t hb[4] = {bf2(hv[0], hv[1]), bf2(hv[2], hv[3]), bf2(hv[4], hv[5]), bf2(hv[6], hv[7])};
                    tc::tmem_st4u(lane_base + kACol + u0 / 2, hb);
                }
            tc::tmem_st_wait();
            tc::fence_before();
            __syncwarp();
            const bool skip = p.skip_h_arrive && blockIdx.x == 0 && warp == kEpiWarp0 && tiles_done == 0;
            if (lane == 0 && !skip) tc::mbar_arrive(&s.h_full);
            for (uint32_t t = 0; ok && t < T; ++t) {
                for (uint32_t c = 0; c < kChunks; ++c) {
                    const uint32_t k = K0 + kEntries * t + (c == 0 ? 0u : c + 1u);
                    const uint32_t slot = k % kSlots;
                    if (!(ok = tc::mbar_wait(&s.full[0][slot], (eu >> slot) & 1u, err, 6, k, lim))) break;
                    eu ^= 1u << slot;
                    tc::fence_after();
                    static_assert(kUPW == 16, "the gate loop loads 16 units per warp");
                    {
                    const uint32_t u0 = c * kUnits + half * kUPW;
                    const uint32_t acol = lane_base + slot * kSlotCols + half * kUPW;
                    float r[16], z[16], nh[16], nx[16], hv[16];
                    tc::tmem_ld16(acol, r);
                    tc::tmem_ld16(acol + kUnits, z);
                    tc::tmem_ld16(acol + 2 * kUnits, nh);
                    tc::tmem_ld16(acol + 3 * kUnits, nx);
                    tc::tmem_ld16(lane_base + kHCol + u0, hv);
                    tc::tmem_ld_wait();
                    // the accumulator is in registers: the slot goes back to the MMA issuer
                    // before the gates are computed
                    tc::fence_before();
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&s.empty[0][slot]);
                    // A lane-divergent branch that is never taken (tiles_done never reaches
                    // 2^32 - 1, which the compiler cannot know): the divergent region it
                    // opens and closes keeps the gate arithmetic below from being scheduled
                    // ahead of the release above.  Measured on the 256-vehicle fleet: the
                    // rollout takes 15.5 ms with it and 18.9 ms without (written out here:
                    // the same test in a separate inline function did not keep the order).
                    if (lane == 0 && tiles_done == 0xFFFFFFFFu) p.err[3] = 0;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float rg = sigmoid_f(r[i]);
                        const float zg = sigmoid_f(z[i]);
                        const float ng = tanh_fast(fmaf(rg, nh[i], nx[i]));
                        hv[i] = zg * hv[i] - (zg - 1.0f) * ng;  // GRU::step, h' = z h - (z - 1) n
                    }
                    tc::tmem_st16(lane_base + kHCol + u0, hv);
                    }
                    tc::tmem_st_wait();
                }
                if (!ok) break;
                // all MMAs of step t are done (the last chunk's completed): h_{t+1} -> A,
                // four chunks' units per TMEM round trip
#pragma unroll
                for (uint32_t c0 = 0; c0 < kChunks; c0 += 4) {
                    float hv[4][16];
#pragma unroll
                    for (uint32_t i = 0; i < 4; ++i) tc::tmem_ld16(lane_base + kHCol + (c0 + i) * kUnits + half * kUPW, hv[i]);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (uint32_t i = 0; i < 4; ++i) {
                        uint32_t hb[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) hb[e] = bf2(hv[i][2 * e], hv[i][2 * e + 1]);
                        tc::tmem_st8u(lane_base + kACol + ((c0 + i) * kUnits + half * kUPW) / 2, hb);
                    }
                }
                tc::tmem_st_wait();
                tc::fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&s.h_full);
            }
            K0 += entries;
            ++tiles_done;
        }
    } else {
        // ================= aux: one thread per candidate row
        const uint32_t q = warp & 3u, row = q * 32 + lane, atid = tid - kAuxWarp0 * 32;
        const uint32_t lane_base = tmem + ((q * 32) << 16);
        const uint32_t TA = T * 4u;
        uint32_t K0 = 0, au = 0;  // bit slot: phase parity of full[1][slot]
        bool ok = true;
        for (uint32_t tile = blockIdx.x; ok && tile < p.tiles; tile += gridDim.x) {
            const uint32_t b = tile / p.tiles_per_vehicle, tv = tile % p.tiles_per_vehicle;
            const uint32_t srow = tv * kRows + row;  // sample index within the shard
            const size_t grow = static_cast<size_t>(b) * a.S + srow;
            const float* cand_row = a.cand_out + grow * TA;  // drawn by sample_kernel
            float x[18];
#pragma unroll
            for (int i = 0; i < 18; ++i) x[i] = a.state_hist[(static_cast<size_t>(b) * a.Hs + a.Hs - 1) * 18 + i];
            const float mass = a.masses ? __ldg(a.masses + b) : a.mass;
            float cost = 0.0f;
            for (uint32_t t = 0; ok && t <= T; ++t) {
                // prober of step t-1 (entry kEntries t + 1; at t = 0 an empty entry; the last at kEntries T)
                const uint32_t k = K0 + (t < T ? kEntries * t + 1 : kEntries * T);
                const uint32_t slot = k % kSlots;
                ok = aux_all(tc::mbar_wait(&s.full[1][slot], (au >> slot) & 1u, err, 9, k, lim));
                if (!ok) break;
                au ^= 1u << slot;
                tc::fence_after();
                if (t > 0) {
                    constexpr uint32_t hid = kMaxHid;  // the tensor-core path takes prober hidden_dim 32
                    float h1[kMaxHid];
                    const float* pw = s.pw;
                    {
                        float v0[16], v1[16];
                        tc::tmem_ld16(lane_base + slot * kSlotCols, v0);
                        tc::tmem_ld16(lane_base + slot * kSlotCols + 16, v1);
                        tc::tmem_ld_wait();
                        // the slot goes back to the MMA issuer before the prober's layers run
                        tc::fence_before();
                        __syncwarp();
                        if (lane == 0) tc::mbar_arrive(&s.empty[1][slot]);
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            h1[i] = gelu_fast(v0[i] + pw[i]);
                            h1[16 + i] = gelu_fast(v1[i] + pw[16 + i]);
                        }
                    }
                    uint32_t off = hid;
                    // a hidden layer's outputs go to this row's shared staging as they are
                    // produced and come back once the layer is done (h1 and the next h1
                    // are never held in registers together)
                    float* hrow = s.hst + row * (kMaxHid + 1);
                    for (uint32_t l = 0; l + 1 < a.prober_layers; ++l) {
                        const float* W = pw + off;
                        const float* bb = pw + off + hid * hid;
#pragma unroll 4
                        for (uint32_t o = 0; o < hid; ++o) {
                            float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
                            for (uint32_t i = 0; i < hid; i += 2) {
                                s0 = fmaf(h1[i], W[o * hid + i], s0);
                                s1 = fmaf(h1[i + 1], W[o * hid + i + 1], s1);
                            }
                            hrow[o] = gelu_fast((s0 + s1) + bb[o]);
                        }
#pragma unroll
                        for (uint32_t o = 0; o < hid; ++o) h1[o] = hrow[o];
                        off += hid * hid + hid;
                    }
#pragma unroll 4
                    for (uint32_t o = 0; o < 15; ++o) {
                        float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
                        for (uint32_t i = 0; i < hid; i += 2) {
                            s0 = fmaf(h1[i], pw[off + o * hid + i], s0);
                            s1 = fmaf(h1[i + 1], pw[off + o * hid + i + 1], s1);
                        }
                        hrow[o] = (s0 + s1) + pw[off + 15 * hid + o];
                    }
                    float po[15];
#pragma unroll
                    for (uint32_t o = 0; o < 15; ++o) po[o] = hrow[o];
                    // integrator step t-1 (lewm_skyjepa_integrate_f32, kinematics.rs:377-484) + cost
                    const uint32_t ts = t - 1;
                    const float* act = cand_row + ts * 4;
                    const float sdt = a.dt;
                    float ta;
                    if (a.rotor_forces) {
                        ta = (act[0] + act[1] + act[2] + act[3]) / mass;
                    } else {
                        const float th = fminf(1.0f, fmaxf(0.0f, act[2]));
                        ta = th * a.gravity / a.hover_throttle;
                    }
                    const float acc3[3] = {x[8] * ta + po[0], x[11] * ta + po[1], x[14] * ta - a.gravity + po[2]};
                    float ang[3];
#pragma unroll
                    for (int r3 = 0; r3 < 3; ++r3)
                        ang[r3] = po[3 + r3 * 4] * act[0] + po[4 + r3 * 4] * act[1] + po[5 + r3 * 4] * act[2] +
                                  po[6 + r3 * 4] * act[3];
#pragma unroll
                    for (int ax = 0; ax < 3; ++ax) {
                        x[ax] += x[3 + ax] * sdt;
                        x[3 + ax] += acc3[ax] * sdt;
                    }
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
                    const float dl[9] = {1.0f - cb * (wy * wy + wz * wz), cb * wx * wy - ca * wz,
                                         cb * wx * wz + ca * wy, cb * wy * wx + ca * wz,
                                         1.0f - cb * (wx * wx + wz * wz), cb * wy * wz - ca * wx,
                                         cb * wz * wx - ca * wy, cb * wz * wy + ca * wx,
                                         1.0f - cb * (wx * wx + wy * wy)};
                    float nr[9];
#pragma unroll
                    for (int r3 = 0; r3 < 3; ++r3)
#pragma unroll
                        for (int c3 = 0; c3 < 3; ++c3)
                            nr[r3 * 3 + c3] =
                                x[6 + r3 * 3] * dl[c3] + x[7 + r3 * 3] * dl[3 + c3] + x[8 + r3 * 3] * dl[6 + c3];
#pragma unroll
                    for (int i = 0; i < 9; ++i) x[6 + i] = nr[i];
#pragma unroll
                    for (int ax = 0; ax < 3; ++ax) x[15 + ax] += ang[ax] * sdt;
                    const float* ref = a.ref_states + (static_cast<size_t>(b) * T + ts) * 18;
                    float g0 = 0.0f, g1 = 0.0f, g2 = 0.0f, g3 = 0.0f;
#pragma unroll
                    for (int i = 0; i < 3; ++i) { const float dd = x[i] - ref[i]; g0 += dd * dd; }
#pragma unroll
                    for (int i = 3; i < 6; ++i) { const float dd = x[i] - ref[i]; g1 += dd * dd; }
#pragma unroll
                    for (int i = 6; i < 15; ++i) { const float dd = x[i] - ref[i]; g2 += dd * dd; }
#pragma unroll
                    for (int i = 15; i < 18; ++i) { const float dd = x[i] - ref[i]; g3 += dd * dd; }
                    const float* ra = a.ref_actions + (static_cast<size_t>(b) * T + ts) * 4;
                    float ac = 0.0f;
#pragma unroll
                    for (int i = 0; i < 4; ++i) { const float dd = act[i] - ra[i]; ac += (dd * dd) * a.cost.action[i]; }
                    float st = g0 * a.cost.position + g1 * a.cost.velocity;
                    st = st + g2 * a.cost.attitude;
                    st = st + g3 * a.cost.angular_velocity;
                    cost += st + ac;
                } else {
                    tc::fence_before();
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&s.empty[1][slot]);
                }
            }
            if (!ok) break;
            // score (mean over T) and the tile's MPPI tuple
            const float score = cost * static_cast<float>(1.0 / static_cast<double>(T));
            a.scores[grow] = score;
            uint64_t key = score_key(score, a.sample_base + srow);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const uint64_t other = __shfl_xor_sync(0xffffffffu, key, o);
                key = other < key ? other : key;
            }
            if (lane == 0) s.red_key[q] = key;
            aux_sync();
            uint64_t best = s.red_key[0];
            for (int w = 1; w < 4; ++w) best = s.red_key[w] < best ? s.red_key[w] : best;
            const float m = key_score(best);
            const float wgt = expf((score - m) * a.m.mul);
            s.red_w[row] = wgt;
            float wsum = wgt;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
            if (lane == 0) s.red_f[q] = wsum;
            aux_sync();
            wsum = s.red_f[0] + s.red_f[1] + s.red_f[2] + s.red_f[3];
            const MppiArgs& mm = a.m;
            float* part = mm.partials + (static_cast<size_t>(b) * mm.P + tv) * mm.pw;
            const float* cand_tile = a.cand_out + (static_cast<size_t>(b) * a.S + tv * kRows) * TA;
            for (uint32_t e = atid; e < TA; e += kAuxThreads) {
                float acc = 0.0f;
                for (uint32_t rr = 0; rr < kRows; ++rr) acc += s.red_w[rr] * cand_tile[rr * TA + e];
                part[4 + e] = acc;
            }
            if (atid == 0) {
                part[0] = m;
                part[1] = wsum;
                reinterpret_cast<uint64_t*>(part)[1] = best;
            }
            __threadfence();
            aux_sync();
            if (atid == 0) s.last = atomicAdd(&mm.counters[b], 1u) == mm.P - 1;
            aux_sync();
            if (s.last) {
                __threadfence();
                // combine the vehicle's tile tuples (mppi_finish with the aux group)
                const float* base = mm.partials + static_cast<size_t>(b) * mm.P * mm.pw;
                uint64_t gk = ~0ull;
                // (read at L2 with loads independent of one another, as mppi_finish)
                for (uint32_t i = atid; i < mm.P; i += kAuxThreads) {
                    const uint64_t kk =
                        __ldcg(reinterpret_cast<const unsigned long long*>(base + static_cast<size_t>(i) * mm.pw) + 1);
                    gk = kk < gk ? kk : gk;
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const uint64_t other = __shfl_xor_sync(0xffffffffu, gk, o);
                    gk = other < gk ? other : gk;
                }
                aux_sync();
                if (lane == 0) s.red_key[q] = gk;
                aux_sync();
                gk = s.red_key[0];
                for (int w = 1; w < 4; ++w) gk = s.red_key[w] < gk ? s.red_key[w] : gk;
                const float M = key_score(gk);
                float* tuple = mm.shard_tuple ? mm.shard_tuple + static_cast<size_t>(b) * mm.pw : nullptr;
                for (uint32_t e = atid; e < TA; e += kAuxThreads) {
                    float W = 0.0f, V = 0.0f;
#pragma unroll 4
                    for (uint32_t i = 0; i < mm.P; ++i) {
                        const float* pq = base + static_cast<size_t>(i) * mm.pw;
                        const uint64_t kk = __ldcg(reinterpret_cast<const unsigned long long*>(pq) + 1);
                        const float m = __ldcg(pq), w = __ldcg(pq + 1), v = __ldcg(pq + 4 + e);
                        if (kk == ~0ull) continue;
                        const float f = expf((m - M) * mm.mul);
                        W += w * f;
                        V += v * f;
                    }
                    if (tuple) {
                        tuple[4 + e] = V;
                        if (e == 0) { tuple[0] = M; tuple[1] = W; reinterpret_cast<uint64_t*>(tuple)[1] = gk; }
                        continue;
                    }
                    const float value = V / W;
                    const uint32_t t = e / 4u, act = e & 3u;
                    const size_t seq = static_cast<size_t>(b) * TA;
                    mm.sequence[seq + e] = value;
                    if (t == 0) mm.first_action[static_cast<size_t>(b) * 4 + act] = value;
                    if (t >= 1) mm.warm_start[seq + e - 4] = value;
                    if (t == T - 1) mm.warm_start[seq + e] = value;
                }
                if (atid == 0) {
                    if (!tuple) {
                        mm.best_index[b] = static_cast<uint32_t>(gk & 0xffffffffu);
                        mm.best_score[b] = M;
                    }
                    mm.counters[b] = 0u;
                }
            }
            aux_sync();
            K0 += entries;
        }
    }

    // ---- teardown
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (warp == 1) tc::tmem_free(tmem, 512);
}

// ------------------------------------------------------------ host side

bool skyjepa_tc_supported(const SkyjepaArgs& a, const char** why) {
    if (a.H != 256) { *why = "the tensor-core path needs latent_dim 256"; return false; }
    if (a.A != 4 || a.E != 4 || a.action_tcn.max_ch != 4 || a.action_tcn.input_dim != 4) {
        *why = "the tensor-core path needs 4 actions and a 4-channel action encoder";
        return false;
    }
    if (a.hid != kMaxHid) { *why = "the tensor-core path needs prober hidden_dim 32"; return false; }
    if (a.Hs != static_cast<uint32_t>(kTcnHs) || a.action_tcn.k != static_cast<uint32_t>(kTcnK) ||
        a.action_tcn.levels != 3 || a.action_tcn.blocks[0].dil != 1 || a.action_tcn.blocks[1].dil != 2 ||
        a.action_tcn.blocks[2].dil != 4) {
        *why = "the tensor-core path needs a 10-step history and a 3-level action encoder with kernel 3";
        return false;
    }
    if (a.prober_layers < 1 || a.prober_layers > kMaxLayers) { *why = "prober hidden_layers must be 1..3"; return false; }
    if (a.S % kRows != 0) { *why = "the tensor-core path needs samples divisible by 128"; return false; }
    if (a.Hs < 2 || a.Hs > kMaxHistTc || a.T == 0 || a.T > kMaxHorizon) { *why = "history/horizon out of range"; return false; }
    if (tcn_weight_floats(a.action_tcn) > kTcnFloats) { *why = "action encoder too large"; return false; }
    if (a.state_tcn.max_ch * a.Hs * 3 * sizeof(float) > 48 * 1024) { *why = "state encoder too wide"; return false; }
    if (a.states) { *why = "predicted states are produced by the f32 path"; return false; }
    if (!a.sample || !a.mppi) { *why = "the tensor-core path runs fused MPPI iterations"; return false; }
    return true;
}

size_t skyjepa_tc_packed_bytes() { return static_cast<size_t>(kChunks) * kChunkBytes + kP1Bytes; }

cudaError_t skyjepa_tc_pack(const SkyjepaArgs& a, uint8_t* packed, cudaStream_t stream) {
    cudaError_t e = cudaMemsetAsync(packed, 0, skyjepa_tc_packed_bytes(), stream);
    if (e != cudaSuccess) return e;
    const size_t n = static_cast<size_t>(kChunks) * kHRows * kH + static_cast<size_t>(kChunks) * kXRows * 16 +
                     static_cast<size_t>(a.hid) * kH;
    pack_tc_weights_kernel<<<static_cast<uint32_t>((n + 255) / 256), 256, 0, stream>>>(
        a, packed, packed + static_cast<size_t>(kChunks) * kChunkBytes);
    return cudaGetLastError();
}

uint32_t skyjepa_tc_partials_per_vehicle(uint32_t S) { return S / kRows; }

cudaError_t fork_h0(const SkyjepaArgs& a, float* h0, cudaStream_t stream, const SideStream* side) {
    if (!side || !side->stream) return launch_skyjepa_h0(a, h0, stream);
    cudaError_t e = cudaEventRecord(side->fork, stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(side->stream, side->fork, 0);
    if (e == cudaSuccess) e = launch_skyjepa_h0(a, h0, side->stream);
    if (e == cudaSuccess) e = cudaEventRecord(side->join, side->stream);
    return e;
}

cudaError_t join_h0(cudaStream_t stream, const SideStream* side) {
    if (!side || !side->stream) return cudaSuccess;
    return cudaStreamWaitEvent(stream, side->join, 0);
}

cudaError_t launch_skyjepa_tc(const SkyjepaArgs& a, const uint8_t* packed, float* h0, uint8_t* xtiles, int* err,
                              cudaStream_t stream, int* launches, const SideStream* side) {
    // 0. initial latent per vehicle (independent of the candidates: on the side stream when given)
    cudaError_t e = fork_h0(a, h0, stream, side);
    if (e != cudaSuccess) return e;
    // 1. candidates (sample_kernel: Philox or injected noise, mean slot, clamp)
    SampleArgs sa{};
    sa.B = a.B; sa.S = a.S; sa.T = a.T; sa.A = 4;
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
    e = launch_sample(sa, stream);
    if (e != cudaSuccess) return e;
    // 2. per-step inputs of every candidate; then the join with the latent
    if (!a.action_tcn_host || tcn_weight_floats(a.action_tcn) != kTcnParamFloats) return cudaErrorInvalidValue;
    TcnConst tw;
    for (uint32_t q = 0; q < kTcnParamFloats; ++q) tw.v[q] = a.action_tcn_host[q];
    const uint64_t rows = static_cast<uint64_t>(a.B) * a.S;
    skyjepa_tc_inputs_seq_kernel<<<static_cast<uint32_t>((rows + 127) / 128), 128, 0, stream>>>(a, tw, xtiles);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = join_h0(stream, side)) != cudaSuccess) return e;
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // 4. the rollout
    TcArgs p;
    p.a = a;
    p.wc = packed;
    p.p1 = packed + static_cast<size_t>(kChunks) * kChunkBytes;
    p.h0 = h0;
    p.xt = xtiles;
    p.tiles_per_vehicle = a.S / kRows;
    p.tiles = a.B * p.tiles_per_vehicle;
    p.err = err;
    p.wait_polls = a.test_wait_polls ? a.test_wait_polls : tc::kWaitLimit;
    p.skip_h_arrive = a.test_skip_h_arrive;
    const size_t smem = sizeof(TcSmem) + 1024;
    static bool attr = false;
    if (!attr) {
        e = cudaFuncSetAttribute(skyjepa_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        attr = true;
    }
    int sms = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t grid = static_cast<uint32_t>(sms) < p.tiles ? static_cast<uint32_t>(sms) : p.tiles;
    if (a.time_begin) cudaEventRecord(a.time_begin, stream);
    skyjepa_tc_kernel<<<grid, kThreadsTc, smem, stream>>>(p);
    if (a.time_end) cudaEventRecord(a.time_end, stream);
    if (launches) *launches = 4;
    return cudaGetLastError();
}

size_t skyjepa_tc_xtile_bytes(uint32_t B, uint32_t S, uint32_t T) {
    return static_cast<size_t>(B) * (S / kRows) * T * kXBytes;
}

}  // namespace lwm
