// kernels_skyjepa_mma.cu — the f32 learned SkyJEPA MPPI scorer with its
// recurrent GEMM on the 5th-generation tensor cores at f32-class accuracy.
//
// Same computation as skyjepa_rollout_kernel (SkyJepaMppiScorer,
// src/models/skyjepa/control.rs:146-317; GRU rollout model.rs:105-223; TCN
// tcn.rs; prober prober.rs:84-138; integrator kinematics.rs:377-484; cost
// control.rs:430-452; MPPI src/planner.rs:1588-1602), for the 4-action,
// latent-256, prober-32 model.
//
// Split fp16 operands.  Every GEMM operand v (the recurrent state h, the
// encoder outputs x, the weights and biases) is held as two fp16 numbers
// v = v0 + v1 with v0 = fp16(v) and v1 = fp16(v - v0), and every product is
// the sum of the three partial products v0 w0 + v0 w1 + v1 w0 (three
// tcgen05.mma kind::f16 with f32 accumulation in TMEM): about 22 significant
// bits per product — the accuracy class of an f32 multiply — instead of the
// 11 of one fp16 product.  The gates, the state h, the prober's later layers,
// the integrator and the cost stay f32 (this file is built with -fmad=false).
//
// Layout: one 16-CTA cluster per 128 candidate rows of a vehicle.  CTA c owns
// hidden units [16c, 16c + 16): its B operand holds their r, z and n rows of
// W_hh plus rows 2c, 2c+1 of the prober's first layer; one step is
//   D[128 x 80] = X_t . Bx^T                  (r | z | n_h | prober | n_x)
//   D[:, 0:64] += H_t . Bh^T                   (K = 256, 16 K-slices)
// then the GRU gates of the CTA's 16 units for the 128 rows; the new h slice
// (both fp16 halves) goes into the CTA's own A operand and to a per-cluster
// exchange buffer in global memory (L2), and every CTA bulk-loads the 15
// slices of its peers from there (the all-to-all goes through L2, whose
// bandwidth per SM is several times the SM-to-SM network's).
// The A operand is 16 K-slices of [128 rows x 16] (SW32), so CTA c's units
// are exactly one slice.  The prober's first layer for latent t comes out of
// step t + 1's MMA (its A operand is h_{t+1}); each CTA sends its two hidden
// units of every row to the CTA that owns the row (8 rows per CTA), which
// finishes the prober, integrates and accumulates the cost.
//
// Roles (448 threads): warp 0 loads the weights once and streams the x tiles;
// warp 1 allocates TMEM and issues the MMAs (the whole warp, one elected
// lane per instruction); warps 2-9 run the gates (two
// warps per TMEM lane quadrant, 8 units each); warps 10-13 read the prober
// columns, then finish the prober, the integrator, the cost and the MPPI
// partial of the CTA's 8 rows.  Every hand-off is an mbarrier with a bounded
// wait; a wait that gives up records its site and the kernel unwinds.
//
// Before it, per plan and in the same stream: the history encoder (h0 per
// vehicle) and skyjepa_mma_inputs_kernel (the candidates, sampled as
// sample_elem_kernel does, and the action encoder of every (candidate, step)
// as split-fp16 x tiles with a constant-1 column that carries the GRU
// biases), chained by programmatic dependent launch: the input kernel runs
// beside the encoder and the rollout's prologue beside the input kernel.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "lwm_device.cuh"
#include "lwm_mppi.cuh"
#include "lwm_kernels.hpp"
#include "lwm_skyjepa_dev.cuh"
#include "lwm_skyjepa_tcn.cuh"
#include "lwm_tc.cuh"

namespace lwm {

// The GRU gates from the hardware exponential and reciprocal (__expf and
// __fdividef, a few ulp over the gates' range): sigmoid(v) = 1 / (1 + e^-v),
// tanh(v) = 1 - 2 / (1 + e^2v).  Both saturate (a denominator past 2^126,
// e^x = inf included, gives 0); the absolute error is about 1e-7, far inside
// the scorer's 1e-4 cost tolerance, for a fraction of the instructions of
// expf / tanhf on the rollout's critical path (plan 0.118 -> 0.110 ms).
__device__ __forceinline__ float sigmoid_e(float v) { return __fdividef(1.0f, 1.0f + __expf(-v)); }
__device__ __forceinline__ float tanh_e(float v) { return 1.0f - __fdividef(2.0f, 1.0f + __expf(2.0f * v)); }
// Candle's tanh-form GELU (gelu_tanh's products and their order) with tanh_e.
__device__ __forceinline__ float gelu_e(float v) {
    const float k = 0.7978845608028654f;
    return __fmul_rn(__fmul_rn(0.5f, v),
                     1.0f + tanh_e(__fmul_rn(__fmul_rn(k, v), 1.0f + __fmul_rn(__fmul_rn(0.044715f, v), v))));
}

namespace {

constexpr uint32_t kCl = 16;                 // CTAs per cluster
constexpr uint32_t kRowsM = 128;             // candidate rows per cluster
constexpr uint32_t kH = 256;                 // latent
constexpr uint32_t kU = kH / kCl;            // 16 hidden units per CTA
constexpr uint32_t kOwnRows = kRowsM / kCl;  // 8 rows whose prober / cost a CTA finishes
constexpr uint32_t kHid = 32;                // prober hidden width
constexpr uint32_t kNh = 64;                 // gate columns: r, z, n_h (16 each), prober (2 used)
// TMEM accumulator slot: columns [0, 64) the products with the weights' high
// halves (and x1 w0, h1 w0), [64, 128) the products with their low halves
// (x0 w1, h0 w1), [128, 144) / [144, 160) the same two for n_x; a gate's
// pre-activation is the sum of its two columns
// K-slices of h in groups of 4: the MMAs of a group issue as soon as its
// peer slices have landed, while the next group's are still in flight
constexpr uint32_t kGroups = 4, kGroupSlices = kCl / kGroups;
constexpr uint32_t kColR = 0, kColZ = 16, kColNh = 32, kColP = 48, kColLo = 64, kColNx = 128, kColNxLo = 144;
constexpr uint32_t kSlotCols = 256;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSliceBytes = kRowsM * 32;        // one [128 x 16] fp16 K-slice, SW32: 4 KB
constexpr uint32_t kSlicePair = 2 * kSliceBytes;     // a slice's two halves, adjacent: 8 KB
constexpr uint32_t kABytes = kCl * kSlicePair;       // 16 slices x 2 halves: 128 KB
constexpr uint32_t kBhBlock = 2 * kNh * 128;         // one K-block: [w0 rows; w1 rows] of 64 elements, SW128: 16 KB
constexpr uint32_t kBhBytes = 4 * kBhBlock;          // K = 256: 64 KB
constexpr uint32_t kBxRows = 2 * kNh + 2 * 16;       // [w0 main; w1 main; w0 n_x; w1 n_x]
constexpr uint32_t kBxBytes = kBxRows * 32;          // SW32: 5 KB
constexpr uint32_t kWBytes = kBhBytes + kBxBytes;    // the CTA's packed weights
constexpr uint32_t kXTileBytes = 2 * kSliceBytes;    // one step's x tile, both halves: 8 KB
constexpr int kThreads = 448;
constexpr uint32_t kEpiWarp0 = 2, kAuxWarp0 = 10, kAuxBarrier = 3, kAuxThreads = 128;
constexpr uint32_t kMaxLayers = 3;
static_assert(kMaxHorizon * 4 <= 2 * kAuxThreads, "the last CTA's combine: two sequence elements per prober thread");
// The prober's hidden and output layers transposed ([in][out], the output
// layer padded to 16), after the CTAs' packed weights: a warp's lanes (one
// output each) read 32 consecutive floats per input.
constexpr uint32_t kProberTFloats = (kMaxLayers - 1) * kHid * kHid + kHid * 16;

struct __align__(1024) MmaSmem {
    uint8_t A[kABytes];            // h_t: [slice][half][128 x 16] fp16, SW32
    uint8_t W[kWBytes];            // Bh [4 K-blocks][128 x 64] SW128, then Bx [160 x 16] SW32
    uint8_t X[2][kXTileBytes];     // x tiles of step t (double buffer), [half][128 x 16] SW32
    float pre[2][kOwnRows][kHid];  // prober first-layer sums of the own rows, by step parity
    float a1[kOwnRows][kHid], a2[kOwnRows][kHid], pout[kOwnRows][16];
    float red_w[kOwnRows];
    uint64_t red_key[4];
    uint64_t w_full, x_full[2], x_empty[2], h_full, mma_done[2], empty[2], pro_full[2], g_ready[2], slice_ready,
        done;
    uint64_t h_grp[kGroups];  // the peer slices of K-slice group g of h_{t+1} have landed
    uint64_t staged;          // the last CTA's combine: a round of partial tuples has landed
    uint32_t tmem;
    int last;
};
static_assert(sizeof(MmaSmem) + 1024 <= 232448, "shared memory budget of one CTA");

__device__ __forceinline__ void aux_sync() {
    asm volatile("bar.sync %0, %1;" ::"n"(kAuxBarrier), "n"(kAuxThreads) : "memory");
}
// True on every prober thread iff `v` is true on all of them: the prober
// warps take every wait's outcome through it, so they leave their loop
// together and never meet aux_sync() short of a warp.
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

// kind::f16 instruction descriptor with fp16 A and B, f32 accumulation,
// K-major operands, shape M x N.
__host__ __device__ constexpr uint32_t idesc_f16_f32(uint32_t M, uint32_t N) {
    return (1u << 4) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// The shared-memory address of `local` in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_addr(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_peer_v2f(uint32_t addr, float a, float b) {
    asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}
// One arrival on the mbarrier at cluster-shared address `addr`, releasing
// this thread's earlier writes to the cluster.
__device__ __forceinline__ void arrive_peer(uint32_t addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}
// One arrival on the mbarrier at cluster-shared address `addr` without
// ordering of its own (a fence ahead of it releases what it publishes).
__device__ __forceinline__ void arrive_peer_relaxed(uint32_t addr) {
    asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}
// Bulk copy of `bytes` from this CTA's shared memory to global memory,
// waited for to completion (both addresses 16-byte aligned, bytes a
// multiple of 16); the writes are then ordered for the async proxy.
__device__ __forceinline__ void bulk_s2g_wait(void* dst, uint32_t src, uint32_t bytes) {
    asm volatile(
        "cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n\t"
        "cp.async.bulk.commit_group;\n\t"
        "cp.async.bulk.wait_group 0;\n\t"
        "fence.proxy.async.global;" ::"l"(dst),
        "r"(src), "r"(bytes)
        : "memory");
}
// Bounded wait with acquire at cluster scope, for barriers that other CTAs
// arrive on (the same give-up protocol as tc::mbar_wait).
__device__ __forceinline__ bool try_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(tc::smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool wait_cluster(uint64_t* bar, uint32_t parity, volatile int* err, int site,
                                             int detail, uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i) {
        if (try_cluster(bar, parity)) return true;
        if ((i & 1023u) == 1023u && err[0]) return false;
    }
    if (atomicCAS(const_cast<int*>(err), 0, site) == 0) {
        err[1] = static_cast<int>(blockIdx.x);
        err[2] = detail;
        err[3] = static_cast<int>(parity);
    }
    return false;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// (a, b) -> the packed fp16 pairs (fp16(a), fp16(b)) and (fp16(a - fp16(a)), fp16(b - fp16(b))).
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
    const __half la = __float2half_rn(a - __half2float(ha)), lb = __float2half_rn(b - __half2float(hb));
    const __half2 h2 = __halves2half2(ha, hb), l2 = __halves2half2(la, lb);
    hi = *reinterpret_cast<const uint32_t*>(&h2);
    lo = *reinterpret_cast<const uint32_t*>(&l2);
}

struct AccurateGelu {
    __device__ __forceinline__ float operator()(float v) const { return gelu_tanh(v); }
};

}  // namespace

// ------------------------------------------------------- weight packing
//
// Per CTA rank c: Bh — gate rows 0-15 W_hr, 16-31 W_hz, 32-47 W_hn of units
// 16c..16c+15, rows 48-49 the prober's first-layer rows 2c, 2c+1, rows 50-63
// zero; the high fp16 halves as operand rows 0-63 and the low halves as rows
// 64-127, K-major SW128 in 4 K-blocks.  Then Bx — gate rows 0-15 W_ir |
// b_ir + b_hr, 16-31 W_iz | b_iz + b_hz, 32-47 0 | b_hn, 48-63 zero, and the
// n_x rows W_in | b_in (k < E the weight, k = E the bias): high halves of the
// gate rows as operand rows 0-63, low halves 64-127, n_x high 128-143, low
// 144-159, SW32.
__global__ void pack_mma_weights_kernel(SkyjepaArgs a, uint8_t* packed) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t n_h = kCl * kNh * kH, n_x = kCl * (kNh + 16) * 16;
    uint32_t hi, lo;
    if (i >= n_h + n_x) {
        const uint32_t q = i - n_h - n_x;
        if (q >= kProberTFloats) return;
        float* wt = reinterpret_cast<float*>(packed + static_cast<size_t>(kCl) * kWBytes);
        const uint32_t n_hid = (kMaxLayers - 1) * kHid * kHid;
        if (q < n_hid) {
            const uint32_t l = q / (kHid * kHid), in = (q / kHid) % kHid, out = q % kHid;
            wt[q] = l + 1 < a.prober_layers ? a.p_hid_w[l][out * kHid + in] : 0.0f;
        } else {
            const uint32_t in = (q - n_hid) / 16, out = (q - n_hid) % 16;
            wt[q] = out < 15 ? a.p_out_w[out * kHid + in] : 0.0f;
        }
        return;
    }
    if (i < n_h) {
        const uint32_t c = i / (kNh * kH), rem = i % (kNh * kH), j = rem / kH, k = rem % kH;
        float v = 0.0f;
        if (j < 48) {
            const uint32_t g = j / kU, u = c * kU + j % kU;
            v = a.w_hh[static_cast<size_t>(g * kH + u) * kH + k];
        } else if (j < 50) {
            v = a.p_in_w[static_cast<size_t>(2 * c + (j - 48)) * kH + k];
        }
        split2(v, 0.0f, hi, lo);
        uint8_t* base = packed + static_cast<size_t>(c) * kWBytes + (k >> 6) * kBhBlock;
        *reinterpret_cast<uint16_t*>(base + tc::sw128_offset(j, k & 63u)) = static_cast<uint16_t>(hi & 0xffffu);
        *reinterpret_cast<uint16_t*>(base + tc::sw128_offset(kNh + j, k & 63u)) = static_cast<uint16_t>(lo & 0xffffu);
    } else if (i < n_h + n_x) {
        const uint32_t q = i - n_h, c = q / ((kNh + 16) * 16), rem = q % ((kNh + 16) * 16), j = rem / 16,
                       k = rem % 16;
        const uint32_t grp = j / kU, u = c * kU + j % kU;
        float v = 0.0f;
        if (k < a.E) {
            if (grp == 0 || grp == 1) v = a.w_ih[static_cast<size_t>(grp * kH + u) * a.E + k];
            else if (grp == 4) v = a.w_ih[static_cast<size_t>(2 * kH + u) * a.E + k];
        } else if (k == a.E) {
            if (grp == 0) v = a.b_ih[u] + a.b_hh[u];
            else if (grp == 1) v = a.b_ih[kH + u] + a.b_hh[kH + u];
            else if (grp == 2) v = a.b_hh[2 * kH + u];
            else if (grp == 4) v = a.b_ih[2 * kH + u];
        }
        split2(v, 0.0f, hi, lo);
        uint8_t* base = packed + static_cast<size_t>(c) * kWBytes + kBhBytes;
        const uint32_t rhi = j < kNh ? j : 2 * kNh + (j - kNh), rlo = rhi + (j < kNh ? kNh : 16u);
        *reinterpret_cast<uint16_t*>(base + tc::sw32_offset(rhi, k)) = static_cast<uint16_t>(hi & 0xffffu);
        *reinterpret_cast<uint16_t*>(base + tc::sw32_offset(rlo, k)) = static_cast<uint16_t>(lo & 0xffffu);
    }
}

// ------------------------------------------------------ per-step inputs
//
// x_t of every candidate and step (the action encoder over the window
// [history ++ candidate](t : t + 10), last position, f32 GELU), as the two
// fp16 halves of the tile of (128-row tile, step): k < 4 the encoder output,
// k = 4 the constant 1 that carries the biases, the rest 0.
struct MmaTcnConst {
    float v[3 * 104];  // per level: conv1 weight [4][4][3], bias [4], conv2 weight, bias
};

__global__ void __launch_bounds__(256) skyjepa_mma_inputs_kernel(SkyjepaArgs a, const __grid_constant__ MmaTcnConst tw,
                                                                 uint8_t* xtiles, int* err) {
    // one block per candidate: thread 4 t + o samples the candidate's action o
    // at step t (white noise, as sample_elem_kernel) and, with the other three
    // lanes of its group, encodes the window of step t (lane o: channel o)
    __shared__ float cand_s[kMaxHorizon][4];
    pdl_trigger();  // the rollout after it may start its prologue (it waits for this kernel before its inputs)
    if (blockIdx.x == 0 && threadIdx.x < 4) err[threadIdx.x] = 0;  // the rollout's error word starts clear
    const uint64_t grow = blockIdx.x;  // b * S + s
    const uint32_t b = static_cast<uint32_t>(grow / a.S), sidx = static_cast<uint32_t>(grow % a.S);
    const uint32_t o = threadIdx.x & 3u, base = threadIdx.x & 28u;
    const bool live = (threadIdx.x >> 2) < a.T;
    const uint32_t t = live ? (threadIdx.x >> 2) : a.T - 1;  // dead lanes still take part in the shuffles
    if (live) {
        const float v = sample_white(a.mean, a.std, a.low_dev, a.high_dev, a.noise, a.seed, a.offset, a.sample_base,
                                     a.sample_total, b, sidx, t, o, a.S, a.T, 4);
        a.cand_out[grow * a.T * 4 + t * 4 + o] = v;
        cand_s[t][o] = v;
    }
    __syncthreads();
    TcnChannelW w;
#pragma unroll
    for (int l = 0; l < 3; ++l) {
        const float* blk = tw.v + l * 104;
#pragma unroll
        for (int q = 0; q < kTcnC * kTcnK; ++q) {
            w.w[2 * l][q] = blk[o * kTcnC * kTcnK + q];
            w.w[2 * l + 1][q] = blk[52 + o * kTcnC * kTcnK + q];
        }
        w.b[2 * l] = blk[48 + o];
        w.b[2 * l + 1] = blk[100 + o];
    }
    float x0[kTcnC][kTcnHs];
#pragma unroll
    for (int q = 0; q < kTcnHs; ++q) {
        const uint32_t pos = t + q;
        float4 v;
        if (pos < kTcnHs - 1) {
            v = *reinterpret_cast<const float4*>(a.action_hist + (static_cast<size_t>(b) * (kTcnHs - 1) + pos) * 4);
        } else {
            const uint32_t k = pos - (kTcnHs - 1);
            v = make_float4(cand_s[k][0], cand_s[k][1], cand_s[k][2], cand_s[k][3]);
        }
        x0[0][q] = (v.x - a.action_mean[0]) / a.action_std[0];
        x0[1][q] = (v.y - a.action_mean[1]) / a.action_std[1];
        x0[2][q] = (v.z - a.action_mean[2]) / a.action_std[2];
        x0[3][q] = (v.w - a.action_mean[3]) / a.action_std[3];
    }
    const float mine = tcn_last_channel<AccurateGelu>(w, x0, o, base);
    float x[kTcnC];
#pragma unroll
    for (int q = 0; q < kTcnC; ++q) x[q] = __shfl_sync(0xffffffffu, mine, base + q);
    if (!live || o != 0) return;
    const uint64_t tile = grow / kRowsM;
    const uint32_t row = static_cast<uint32_t>(grow % kRowsM);
    uint8_t* xt = xtiles + (tile * a.T + t) * kXTileBytes;
    uint32_t h01, l01, h23, l23, h4, l4;
    split2(x[0], x[1], h01, l01);
    split2(x[2], x[3], h23, l23);
    split2(1.0f, 0.0f, h4, l4);
    *reinterpret_cast<uint4*>(xt + tc::sw32_offset(row, 0)) = make_uint4(h01, h23, h4, 0u);
    *reinterpret_cast<uint4*>(xt + tc::sw32_offset(row, 8)) = make_uint4(0u, 0u, 0u, 0u);
    *reinterpret_cast<uint4*>(xt + kSliceBytes + tc::sw32_offset(row, 0)) = make_uint4(l01, l23, l4, 0u);
    *reinterpret_cast<uint4*>(xt + kSliceBytes + tc::sw32_offset(row, 8)) = make_uint4(0u, 0u, 0u, 0u);
    // this kernel completes only after the history encoder before it: the
    // rollout's wait for this kernel then covers h0 as well
    pdl_wait();
}

// ------------------------------------------------------------ main kernel

namespace {

struct MmaArgs {
    SkyjepaArgs a;
    const uint8_t* w;    // packed weights [16][kWBytes]
    const float* h0;     // [B, 256]
    const uint8_t* xt;   // x tiles [tiles][T][kXTileBytes]
    uint8_t* xchg;       // h exchange [tiles][2 step parities][16 slices][kSlicePair]
    uint32_t tiles_per_vehicle, tiles;
    int* err;
    uint32_t wait_polls;
};

}  // namespace

__global__ void __launch_bounds__(kThreads, 1) skyjepa_mma_kernel(MmaArgs p) {
    extern __shared__ uint8_t smem_raw[];
    MmaSmem& s = *reinterpret_cast<MmaSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const SkyjepaArgs& a = p.a;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t T = a.T;
    const uint32_t c = cluster_rank();
    const uint32_t tile = blockIdx.x / kCl;  // this cluster's 128 rows
    const uint32_t b = tile / p.tiles_per_vehicle, tv = tile % p.tiles_per_vehicle;
    volatile int* err = p.err;
    const uint32_t lim = p.wait_polls;

    // ---- setup
    if (tid == 0) {
        tc::mbar_init(&s.w_full, 1);
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&s.x_full[i], 1);
            tc::mbar_init(&s.x_empty[i], 1);
            tc::mbar_init(&s.mma_done[i], 1);
            tc::mbar_init(&s.empty[i], 12);      // 8 gate warps + 4 prober warps release a slot
            tc::mbar_init(&s.pro_full[i], kRowsM);  // 8 own rows x 16 CTAs deliver per step
        }
        // h_t complete: the MMA issuer's arrival (with the 15 peer slices'
        // bytes expected) and the 8 gate warps' own-slice arrivals
        tc::mbar_init(&s.h_full, 8);  // the own slice of h_t (all of h_0) is in A
        for (uint32_t g = 0; g < kGroups; ++g) tc::mbar_init(&s.h_grp[g], 1);
        tc::mbar_init(&s.slice_ready, 8);  // the own slice of h is in the exchange buffer
        for (int i = 0; i < 2; ++i) tc::mbar_init(&s.g_ready[i], kCl - 1);  // the 15 peers' slices are, by step parity
        tc::mbar_init(&s.done, 1);
        tc::mbar_init(&s.staged, 1);
        tc::mbar_fence_init();
    }
    if (warp == 1) tc::tmem_alloc(&s.tmem, kTmemCols);
    tc::fence_before();
    __syncthreads();
    cluster_sync_all();  // every CTA's barriers exist before any remote arrival
    tc::fence_after();
    const uint32_t tmem = s.tmem;
    bool failed = false;
    // the weights do not come from the kernels before this one in the stream:
    // their copy starts before the wait for those kernels (h0, x tiles, the
    // cleared error word)
    if (warp == 0 && lane == 0) {
        tc::mbar_expect_tx(&s.w_full, kWBytes);
        tc::bulk_g2s(s.W, p.w + static_cast<size_t>(c) * kWBytes, kWBytes, &s.w_full);
    }
    pdl_wait();

    if (warp == 0) {
        // ================= producer: the CTA's weights once (issued above), then one x tile per step
        if (lane == 0) {
            const uint8_t* xg = p.xchg + static_cast<size_t>(tile) * 2 * kABytes;
            uint32_t t = 0;  // x tiles issued
            auto load_x = [&](uint32_t k) -> bool {
                const uint32_t xs = k & 1u;
                if (!tc::mbar_wait(&s.x_empty[xs], ((k >> 1) & 1u) ^ 1u, err, 1, k, lim)) return false;
                tc::mbar_expect_tx(&s.x_full[xs], kXTileBytes);
                tc::bulk_g2s(s.X[xs], p.xt + (static_cast<size_t>(tile) * T + k) * kXTileBytes, kXTileBytes,
                             &s.x_full[xs]);
                return true;
            };
            bool ok = load_x(0);
            t = ok ? 1u : 0u;
            for (uint32_t k = 0; ok && k < T; ++k) {
                // the next step's x tile ahead of the exchange
                if (k + 1 < T) {
                    if (!(ok = load_x(k + 1))) break;
                    t = k + 2;
                }
                // h_{k+1}: the 15 peer slices, once they are in the exchange buffer
                // and this CTA's MMAs of step k are done reading A
                if (!(ok = wait_cluster(&s.g_ready[k & 1u], (k >> 1) & 1u, err, 11, k, lim))) break;
                if (!(ok = tc::mbar_wait(&s.mma_done[k & 1u], (k >> 1) & 1u, err, 12, k, lim))) break;
                const uint8_t* src = xg + static_cast<size_t>((k + 1) & 1u) * kABytes;
                for (uint32_t g = 0; g < kGroups; ++g) {
                    const uint32_t n = (g == c / kGroupSlices) ? kGroupSlices - 1u : kGroupSlices;
                    tc::mbar_expect_tx(&s.h_grp[g], n * kSlicePair);
                    for (uint32_t j = g * kGroupSlices; j < (g + 1) * kGroupSlices; ++j)
                        if (j != c) tc::bulk_g2s(s.A + j * kSlicePair, src + j * kSlicePair, kSlicePair, &s.h_grp[g]);
                }
            }
            // copies issued and maybe not consumed land before the CTA exits
            tc::mbar_wait_landing(&s.w_full, 0, lim);
            for (uint32_t sl = 0; sl < 2u; ++sl)
                if (t > sl) {
                    const uint32_t last = sl + ((t - 1u - sl) / 2u) * 2u;
                    tc::mbar_wait_landing(&s.x_full[sl], (last >> 1) & 1u, lim);
                }
        }
    } else if (warp == 1) {
        // ================= MMA issuer (the whole warp, converged; one elected lane issues)
        {
            const uint32_t id128 = idesc_f16_f32(kRowsM, 2 * kNh), id64 = idesc_f16_f32(kRowsM, kNh);
            const uint32_t id32 = idesc_f16_f32(kRowsM, 32), id16 = idesc_f16_f32(kRowsM, 16);
            const uint32_t w_base = tc::smem_u32(s.W);
            // every lane waits; the outcome is the warp's (a diverged lane would leave elect.sync short)
            auto wwait = [&](uint64_t* bar, uint32_t parity, volatile int* e, int site, uint32_t detail,
                             uint32_t limit) -> bool {
                return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity, e, site, static_cast<int>(detail), limit));
            };
            // descriptors of the operand bases; an offset of n bytes adds n >> 4
            // to the start-address field (all addresses below 256 KB)
            const uint64_t da = tc::smem_desc(tc::smem_u32(s.A), 16, 256, tc::kSwizzle32);
            const uint64_t dbh = tc::smem_desc(w_base, 16, 1024, tc::kSwizzle128);
            const uint64_t dbx = tc::smem_desc(w_base + kBhBytes, 16, 256, tc::kSwizzle32);
            bool ok = wwait(&s.w_full, 0, err, 2, 0, lim);
            for (uint32_t t = 0; ok && t <= T; ++t) {
                const uint32_t slot = t & 1u;
                ok = wwait(&s.h_full, t & 1u, err, 3, t, lim);  // A holds the own slice of h_t
                if (ok && t >= 2) ok = wwait(&s.empty[slot], ((t >> 1) - 1u) & 1u, err, 4, t, lim);
                if (ok && t < T) ok = wwait(&s.x_full[slot], (t >> 1) & 1u, err, 5, t, lim);
                if (!ok) break;
                tc::fence_after();
                const uint32_t d = tmem + slot * kSlotCols;
                // split products: v0 [w0; w1] (both columns halves at once, N = 128)
                // and v1 w0 (N = 64), for x and for every K-slice of h
                uint32_t acc = 0;
                if (t < T) {
                    const uint64_t dx = tc::smem_desc(tc::smem_u32(s.X[slot]), 16, 256, tc::kSwizzle32);
                    constexpr uint64_t x1 = kSliceBytes >> 4, nx = (2 * kNh * 32) >> 4;
                    tc::mma_f16_w(d, dx, dbx, id128, 0);
                    tc::mma_f16_w(d, dx + x1, dbx, id64, 1);
                    tc::mma_f16_w(d + kColNx, dx, dbx + nx, id32, 0);
                    tc::mma_f16_w(d + kColNx, dx + x1, dbx + nx, id16, 1);
                    acc = 1;
                }
                auto slice = [&](uint32_t j) {
                    const uint64_t a0 = da + ((j * kSlicePair) >> 4), a1 = a0 + (kSliceBytes >> 4);
                    const uint64_t b = dbh + (((j >> 2) * kBhBlock + (j & 3u) * 32) >> 4);
                    tc::mma_f16_w(d, a0, b, id128, acc);
                    tc::mma_f16_w(d, a1, b, id64, 1);
                    acc = 1;
                };
                // the own slice first, then the peers' group by group as they land
                slice(c);
                for (uint32_t g = 0; ok && g < kGroups; ++g) {
                    if (t > 0) {
                        if (!(ok = wwait(&s.h_grp[g], (t - 1u) & 1u, err, 13, t, lim))) break;
                        tc::fence_after();
                    }
#pragma unroll
                    for (uint32_t i = 0; i < kGroupSlices; ++i) {
                        const uint32_t j = g * kGroupSlices + i;
                        if (j != c) slice(j);
                    }
                }
                if (!ok) break;
                tc::commit_w(&s.mma_done[slot]);
                if (t < T) tc::commit_w(&s.x_empty[slot]);
            }
            failed = !ok;
            // every MMA issued has completed before TMEM is released
            tc::commit_w(&s.done);
            tc::mbar_wait_landing(&s.done, 0, lim);
        }
    } else if (warp < kAuxWarp0) {
        // ================= GRU gates: quadrant q (rows 32q..32q+31), units 8 half .. 8 half + 7 of the slice
        const uint32_t q = warp & 3u, half = (warp - kEpiWarp0) >> 2, row = q * 32 + lane;
        const uint32_t lane_base = tmem + ((q * 32) << 16);
        const float* h0 = p.h0 + static_cast<size_t>(b) * kH;
        // h_0 into the whole A operand (every unit, both halves); this thread
        // writes the slices of its parity for its row
        for (uint32_t j = half; j < kCl; j += 2)
            for (uint32_t k8 = 0; k8 < 16; k8 += 8) {
                float v[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = __ldg(h0 + j * kU + k8 + i);
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) split2(v[2 * i], v[2 * i + 1], hi[i], lo[i]);
                const uint32_t off = j * kSlicePair + tc::sw32_offset(row, k8);
                *reinterpret_cast<uint4*>(s.A + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4*>(s.A + kSliceBytes + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
        float hprev[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) hprev[i] = __ldg(h0 + c * kU + half * 8 + i);
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&s.h_full);  // phase 0: h_0 written locally
        const uint32_t slice_off = c * kSlicePair + tc::sw32_offset(row, half * 8);
        const uint32_t gready_local = tc::smem_u32(&s.g_ready[0]);
        const uint32_t a_slice = tc::smem_u32(s.A) + c * kSlicePair;
        uint8_t* xg = p.xchg + static_cast<size_t>(tile) * 2 * kABytes + c * kSlicePair;
        // the first gate warp publishes the CTA's slice and tells the peers
        const uint32_t wi = warp - kEpiWarp0;
        bool ok = true;
        for (uint32_t t = 0; ok && t < T; ++t) {
            const uint32_t slot = t & 1u;
            if (!(ok = tc::mbar_wait(&s.mma_done[slot], (t >> 1) & 1u, err, 6, t, lim))) break;
            tc::fence_after();
            const uint32_t col = lane_base + slot * kSlotCols + half * 8;
            float r[8], z[8], nh[8], nx[8], r1[8], z1[8], nh1[8], nx1[8];
            tc::tmem_ld8(col + kColR, r);
            tc::tmem_ld8(col + kColZ, z);
            tc::tmem_ld8(col + kColNh, nh);
            tc::tmem_ld8(col + kColNx, nx);
            tc::tmem_ld8(col + kColLo + kColR, r1);
            tc::tmem_ld8(col + kColLo + kColZ, z1);
            tc::tmem_ld8(col + kColLo + kColNh, nh1);
            tc::tmem_ld8(col + kColNxLo, nx1);
            tc::tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                r[i] += r1[i];
                z[i] += z1[i];
                nh[i] += nh1[i];
                nx[i] += nx1[i];
            }
            tc::fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&s.empty[slot]);
            // candle GRU::step: r, z = sigmoid(.), n = tanh(x_n + r * h_n), h' = z h - (z - 1) n
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float rg = sigmoid_e(r[i]);
                const float zg = sigmoid_e(z[i]);
                const float ng = tanh_e(nx[i] + rg * nh[i]);
                hprev[i] = zg * hprev[i] - (zg - 1.0f) * ng;
            }
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) split2(hprev[2 * i], hprev[2 * i + 1], hi[i], lo[i]);
            // the own slice of h_{t+1} into the local A operand (this CTA's MMA
            // of step t is done reading it: mma_done above), for the tensor
            // core and the bulk store below
            *reinterpret_cast<uint4*>(s.A + slice_off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4*>(s.A + kSliceBytes + slice_off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            tc::fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                tc::mbar_arrive(&s.slice_ready);
                tc::mbar_arrive(&s.h_full);
                if (wi == 0) {
                    // once the whole slice is in A: its 8 KB to the exchange buffer
                    // of parity (t + 1) & 1 (whose readers of h_{t-1} are done: they
                    // passed their MMA of step t - 1 before this CTA's MMA of step
                    // t could run), then one release for the 15 peers' arrivals
                    ok = tc::mbar_wait(&s.slice_ready, t & 1u, err, 10, t, lim);
                    if (ok) {
                        bulk_s2g_wait(xg + static_cast<size_t>((t + 1) & 1u) * kABytes, a_slice, kSlicePair);
                        asm volatile("fence.release.cluster;" ::: "memory");
                        for (uint32_t d = 1; d < kCl; ++d)
                            arrive_peer_relaxed(peer_addr(gready_local + (t & 1u) * 8u, (c + d) & (kCl - 1u)));
                    }
                }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        }
        failed = !ok;
    } else {
        // ================= prober, integrator, cost and MPPI partial of the own rows
        const uint32_t q = warp & 3u, row = q * 32 + lane, atid = tid - kAuxWarp0 * 32;
        const uint32_t lane_base = tmem + ((q * 32) << 16);
        const uint32_t TA = T * 4u;
        const float* wt = reinterpret_cast<const float*>(p.w + static_cast<size_t>(kCl) * kWBytes);
        const uint32_t own0 = tv * kRowsM + c * kOwnRows;  // first sample of this CTA's own rows
        const size_t grow0 = static_cast<size_t>(b) * a.S + own0;
        // the slot of MMA(0) has no prober columns to read
        if (lane == 0) tc::mbar_arrive(&s.empty[0]);
        float x[18], cost = 0.0f;
        if (atid < kOwnRows)
#pragma unroll
            for (int i = 0; i < 18; ++i) x[i] = a.state_hist[(static_cast<size_t>(b) * a.Hs + a.Hs - 1) * 18 + i];
        const uint32_t pre_local = tc::smem_u32(&s.pre[0][0][0]);
        const uint32_t owner = row / kOwnRows;
        bool ok = true;
        for (uint32_t t = 0; t < T; ++t) {
            // prober layer 1 of latent t = h_{t+1}: columns kColP, kColP + 1 of MMA(t + 1)
            const uint32_t m = t + 1, slot = m & 1u, par = t & 1u;
            ok = aux_all(tc::mbar_wait(&s.mma_done[slot], (m >> 1) & 1u, err, 8, m, lim));
            if (!ok) break;
            tc::fence_after();
            float v[8], v1[8];
            tc::tmem_ld8(lane_base + slot * kSlotCols + kColP, v);
            tc::tmem_ld8(lane_base + slot * kSlotCols + kColLo + kColP, v1);
            tc::tmem_ld_wait();
            v[0] += v1[0];
            v[1] += v1[1];
            tc::fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&s.empty[slot]);
            // to the CTA that owns this row: its pre[t & 1][row % 8][2c, 2c + 1]
            const uint32_t dst =
                peer_addr(pre_local, owner) + ((par * kOwnRows + row % kOwnRows) * kHid + 2 * c) * 4u;
            st_peer_v2f(dst, v[0], v[1]);
            arrive_peer(peer_addr(tc::smem_u32(&s.pro_full[par]), owner));
            ok = aux_all(wait_cluster(&s.pro_full[par], (t >> 1) & 1u, err, 9, t, lim));
            if (!ok) break;
            // layer 1 activation, hidden layers, output (SkyJepaProber::forward, prober.rs:84-102)
            for (uint32_t e = atid; e < kOwnRows * kHid; e += kAuxThreads) {
                const uint32_t rr = e / kHid, o = e % kHid;
                s.a1[rr][o] = gelu_e(s.pre[par][rr][o] + __ldg(a.p_in_b + o));
            }
            aux_sync();
            float(*pin)[kHid] = s.a1;
            float(*pout)[kHid] = s.a2;
            // lane = output unit, rows q and q + 4 (the weights' transposed copy:
            // coalesced reads shared by both rows)
            const uint32_t ra = q, rb = q + 4;
            for (uint32_t l = 0; l + 1 < a.prober_layers; ++l) {
                const float* W = wt + l * kHid * kHid + lane;
                float s0a = 0.0f, s1a = 0.0f, s0b = 0.0f, s1b = 0.0f;
#pragma unroll
                for (uint32_t i = 0; i < kHid; i += 2) {
                    const float w0 = __ldg(W + i * kHid), w1 = __ldg(W + (i + 1) * kHid);
                    s0a = fmaf(pin[ra][i], w0, s0a);
                    s1a = fmaf(pin[ra][i + 1], w1, s1a);
                    s0b = fmaf(pin[rb][i], w0, s0b);
                    s1b = fmaf(pin[rb][i + 1], w1, s1b);
                }
                const float bias = __ldg(a.p_hid_b[l] + lane);
                pout[ra][lane] = gelu_e((s0a + s1a) + bias);
                pout[rb][lane] = gelu_e((s0b + s1b) + bias);
                aux_sync();
                float(*tmp)[kHid] = pin;
                pin = pout;
                pout = tmp;
            }
            if (lane < 16) {
                const float* W = wt + (kMaxLayers - 1) * kHid * kHid + lane;
                float s0a = 0.0f, s1a = 0.0f, s0b = 0.0f, s1b = 0.0f;
#pragma unroll
                for (uint32_t i = 0; i < kHid; i += 2) {
                    const float w0 = __ldg(W + i * 16), w1 = __ldg(W + (i + 1) * 16);
                    s0a = fmaf(pin[ra][i], w0, s0a);
                    s1a = fmaf(pin[ra][i + 1], w1, s1a);
                    s0b = fmaf(pin[rb][i], w0, s0b);
                    s1b = fmaf(pin[rb][i + 1], w1, s1b);
                }
                if (lane < 15) {
                    const float bias = __ldg(a.p_out_b + lane);
                    s.pout[ra][lane] = (s0a + s1a) + bias;
                    s.pout[rb][lane] = (s0b + s1b) + bias;
                }
            }
            aux_sync();
            if (atid < kOwnRows) {
                const float* act = a.cand_out + (grow0 + atid) * TA + t * 4;
                cost += integrate_and_cost(a, b, own0 + atid, t, x, act, s.pout[atid], false);
            }
        }
        failed = !ok;
        if (ok) {
            // scores of the own rows (mean over T) and the CTA's MPPI tuple
            float score = 0.0f;
            uint64_t key = ~0ull;
            if (atid < kOwnRows) {
                score = cost * static_cast<float>(1.0 / static_cast<double>(T));
                a.scores[grow0 + atid] = score;
                key = score_key(score, a.sample_base + own0 + atid);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const uint64_t other = __shfl_xor_sync(0xffffffffu, key, o);
                key = other < key ? other : key;
            }
            if (lane == 0) s.red_key[q] = key;
            aux_sync();
            uint64_t best = s.red_key[0];
            for (int w = 1; w < 4; ++w) best = s.red_key[w] < best ? s.red_key[w] : best;
            const float mval = key_score(best);
            if (atid < kOwnRows) s.red_w[atid] = expf((score - mval) * a.m.mul);
            aux_sync();
            float wsum = 0.0f;
            for (uint32_t rr = 0; rr < kOwnRows; ++rr) wsum += s.red_w[rr];
            const MppiArgs& mm = a.m;
            const uint32_t pidx = tv * kCl + c;
            float* part = mm.partials + (static_cast<size_t>(b) * mm.P + pidx) * mm.pw;
            const float* cand_rows = a.cand_out + grow0 * TA;
            for (uint32_t e = atid; e < TA; e += kAuxThreads) {
                float acc = 0.0f;
                for (uint32_t rr = 0; rr < kOwnRows; ++rr) acc += s.red_w[rr] * cand_rows[rr * TA + e];
                part[4 + e] = acc;
            }
            if (atid == 0) {
                part[0] = mval;
                part[1] = wsum;
                reinterpret_cast<uint64_t*>(part)[1] = best;
            }
            __threadfence();
            aux_sync();
            if (atid == 0) s.last = atomicAdd(&mm.counters[b], 1u) == mm.P - 1;
            aux_sync();
            if (s.last) {
                __threadfence();
                // the last CTA of the vehicle combines its partial tuples
                const float* base = mm.partials + static_cast<size_t>(b) * mm.P * mm.pw;
                uint64_t gk = ~0ull;
                for (uint32_t i = atid; i < mm.P; i += kAuxThreads) {
                    const uint64_t kk =
                        reinterpret_cast<const volatile uint64_t*>(base + static_cast<size_t>(i) * mm.pw)[1];
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
                // W = sum_i w_i f_i and V[e] = sum_i v_i[e] f_i, f_i = exp((m_i - M) mul),
                // over the non-empty partials in ascending order.  The partials
                // are staged into shared memory (the h operand, idle now) by one
                // bulk copy per round, as many as fit; each f_i is computed once,
                // by one thread.
                tc::fence_async_smem();
                float* stage = reinterpret_cast<float*>(s.A);
                const uint32_t cap = kABytes / (mm.pw * 4u + 4u);
                constexpr uint32_t kMaxE = 2;  // TA <= 2 x 128
                float W[kMaxE] = {0.0f, 0.0f}, V[kMaxE] = {0.0f, 0.0f};
                bool staged_ok = true;
                for (uint32_t i0 = 0, round = 0; i0 < mm.P; i0 += cap, ++round) {
                    const uint32_t n = mm.P - i0 < cap ? mm.P - i0 : cap;
                    if (atid == 0) {
                        // (tuples are 16-byte multiples: pw is a multiple of 4)
                        const uint32_t bytes = n * mm.pw * 4u;
                        tc::mbar_expect_tx(&s.staged, bytes);
                        tc::bulk_g2s(stage, base + static_cast<size_t>(i0) * mm.pw, bytes, &s.staged);
                        staged_ok = tc::mbar_wait(&s.staged, round & 1u, err, 14, static_cast<int>(round), lim);
                    }
                    if (!aux_all(staged_ok)) break;
                    float* fac = stage + static_cast<size_t>(n) * mm.pw;
                    for (uint32_t j = atid; j < n; j += kAuxThreads) {
                        const float* pq = stage + static_cast<size_t>(j) * mm.pw;
                        fac[j] = expf((pq[0] - M) * mm.mul);
                    }
                    aux_sync();
#pragma unroll
                    for (uint32_t k = 0; k < kMaxE; ++k) {
                        const uint32_t e = atid + k * kAuxThreads;
                        if (e >= TA) continue;
#pragma unroll 8
                        for (uint32_t j = 0; j < n; ++j) {
                            const float* pq = stage + static_cast<size_t>(j) * mm.pw;
                            const bool rows = reinterpret_cast<const uint64_t*>(pq)[1] != ~0ull;  // else no rows
                            const float w = pq[1] * fac[j], v = pq[4 + e] * fac[j];
                            W[k] = rows ? W[k] + w : W[k];
                            V[k] = rows ? V[k] + v : V[k];
                        }
                    }
                    aux_sync();
                }
                for (uint32_t k = 0; k < kMaxE; ++k) {
                    const uint32_t e = atid + k * kAuxThreads;
                    if (e >= TA) continue;
                    if (tuple) {
                        tuple[4 + e] = V[k];
                        if (e == 0) {
                            tuple[0] = M;
                            tuple[1] = W[k];
                            reinterpret_cast<uint64_t*>(tuple)[1] = gk;
                        }
                        continue;
                    }
                    const float value = V[k] / W[k];
                    const uint32_t tt = e / 4u, act = e & 3u;
                    const size_t seq = static_cast<size_t>(b) * TA;
                    mm.sequence[seq + e] = value;
                    if (tt == 0) mm.first_action[static_cast<size_t>(b) * 4 + act] = value;
                    if (tt >= 1) mm.warm_start[seq + e - 4] = value;
                    if (tt == T - 1) mm.warm_start[seq + e] = value;
                }
                if (atid == 0) {
                    if (!tuple) {
                        mm.best_index[b] = static_cast<uint32_t>(gk & 0xffffffffu);
                        mm.best_score[b] = M;
                    }
                    mm.counters[b] = 0u;
                }
            }
        }
    }

    // ---- teardown: TMEM back, then no CTA leaves while a peer may still write to it
    tc::fence_before();
    const int any_failed = __syncthreads_or(failed || err[0]);  // block-uniform
    tc::fence_after();
    if (warp == 1) tc::tmem_free(tmem, kTmemCols);
    if (any_failed) {
        // a wait gave up somewhere: let remote stores already issued in the
        // cluster land (a fixed, bounded grace period) before the barrier
        uint64_t t0;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
        for (uint32_t i = 0; i < (1u << 20); ++i) {
            uint64_t t1;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
            if (t1 - t0 > 200000ull) break;
        }
    }
    __syncwarp();
    cluster_sync_all();
}

// ------------------------------------------------------------ host side

bool skyjepa_mma_supported(const SkyjepaArgs& a, const char** why) {
    if (a.H != kH) { *why = "the split-fp16 path needs latent_dim 256"; return false; }
    if (a.A != 4 || a.E != 4 || a.action_tcn.max_ch != 4 || a.action_tcn.input_dim != 4) {
        *why = "the split-fp16 path needs 4 actions and a 4-channel action encoder";
        return false;
    }
    if (a.hid != kHid) { *why = "the split-fp16 path needs prober hidden_dim 32"; return false; }
    if (a.Hs != static_cast<uint32_t>(kTcnHs) || a.action_tcn.k != static_cast<uint32_t>(kTcnK) ||
        a.action_tcn.levels != 3 || a.action_tcn.blocks[0].dil != 1 || a.action_tcn.blocks[1].dil != 2 ||
        a.action_tcn.blocks[2].dil != 4) {
        *why = "the split-fp16 path needs a 10-step history and a 3-level action encoder with kernel 3";
        return false;
    }
    if (a.prober_layers < 1 || a.prober_layers > kMaxLayers) { *why = "prober hidden_layers must be 1..3"; return false; }
    if (a.S % kRowsM != 0) { *why = "the split-fp16 path needs samples divisible by 128"; return false; }
    if (a.T == 0 || a.T > kMaxHorizon) { *why = "horizon out of range"; return false; }
    if (tcn_weight_floats(a.action_tcn) != 3 * 104) { *why = "action encoder size"; return false; }
    if (a.states) { *why = "predicted states are produced by the f32 CUDA-core path"; return false; }
    if (!a.sample || !a.mppi) { *why = "the split-fp16 path runs fused MPPI iterations"; return false; }
    return true;
}

size_t skyjepa_mma_packed_bytes() { return static_cast<size_t>(kCl) * kWBytes + kProberTFloats * sizeof(float); }

cudaError_t skyjepa_mma_pack(const SkyjepaArgs& a, uint8_t* packed, cudaStream_t stream) {
    const uint32_t n = kCl * kNh * kH + kCl * (kNh + 16) * 16 + kProberTFloats;
    pack_mma_weights_kernel<<<(n + 255) / 256, 256, 0, stream>>>(a, packed);
    return cudaGetLastError();
}

uint32_t skyjepa_mma_partials_per_vehicle(uint32_t S) { return (S / kRowsM) * kCl; }

size_t skyjepa_mma_xtile_bytes(uint32_t B, uint32_t S, uint32_t T) {
    return static_cast<size_t>(B) * (S / kRowsM) * T * kXTileBytes;
}

namespace {

// Shared-memory opt-in and non-portable cluster size, once per device; false
// when a 16-CTA cluster of this kernel cannot be resident on the device.
bool mma_configure(int dev) {
    static std::mutex mu;
    static int state[64] = {};  // 0 unknown, 1 fits, 2 does not
    if (dev < 0 || dev >= 64) return false;
    std::lock_guard<std::mutex> lock(mu);
    if (state[dev] == 0) {
        const size_t smem = sizeof(MmaSmem) + 1024;
        cudaError_t e = cudaFuncSetAttribute(skyjepa_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(skyjepa_mma_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        int n = 0;
        if (e == cudaSuccess) {
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(kCl, 1, 1);
            cfg.blockDim = dim3(kThreads, 1, 1);
            cfg.dynamicSmemBytes = smem;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = kCl;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            e = cudaOccupancyMaxActiveClusters(&n, skyjepa_mma_kernel, &cfg);
        }
        (void)cudaGetLastError();
        state[dev] = (e == cudaSuccess && n >= 1) ? 1 : 2;
    }
    return state[dev] == 1;
}

}  // namespace

bool skyjepa_mma_fits_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    return mma_configure(dev);
}

size_t skyjepa_mma_exchange_bytes(uint32_t B, uint32_t S) {
    return static_cast<size_t>(B) * (S / kRowsM) * 2 * kABytes;
}

cudaError_t launch_skyjepa_mma(const SkyjepaArgs& a, const uint8_t* packed, float* h0, uint8_t* xtiles,
                               uint8_t* xchg, int* err, cudaStream_t stream, int* launches, const SideStream* side) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (!mma_configure(dev)) return cudaErrorNotSupported;
    if (!a.action_tcn_host) return cudaErrorInvalidValue;
    (void)side;
    // 0. initial latent per vehicle; 1. the candidates (white noise) and the
    // action encoder of every (candidate, step) as split-fp16 x tiles, one
    // block per candidate; 2. the rollout.  One stream with programmatic
    // dependent launch: the input kernel runs beside the history encoder
    // (which triggers at its start) and finishes after it; the rollout starts
    // its prologue (barriers, TMEM, the weight copy) beside the input kernel
    // and waits for it before touching h0 and the x tiles.
    if ((e = launch_skyjepa_h0(a, h0, stream)) != cudaSuccess) return e;
    MmaTcnConst tw;
    for (uint32_t q = 0; q < 3 * 104; ++q) tw.v[q] = a.action_tcn_host[q];
    const uint32_t threads = (4 * a.T + 31) / 32 * 32;
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    {
        cudaLaunchConfig_t ic{};
        ic.gridDim = dim3(a.B * a.S, 1, 1);
        ic.blockDim = dim3(threads, 1, 1);
        ic.stream = stream;
        ic.attrs = pdl;
        ic.numAttrs = 1;
        if ((e = cudaLaunchKernelEx(&ic, skyjepa_mma_inputs_kernel, a, tw, xtiles, err)) != cudaSuccess) return e;
    }
    // 3. the rollout: one 16-CTA cluster per 128 rows
    MmaArgs p;
    p.a = a;
    p.w = packed;
    p.h0 = h0;
    p.xt = xtiles;
    p.xchg = xchg;
    p.tiles_per_vehicle = a.S / kRowsM;
    p.tiles = a.B * p.tiles_per_vehicle;
    p.err = err;
    p.wait_polls = a.test_wait_polls ? a.test_wait_polls : tc::kWaitLimit;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(p.tiles * kCl, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = sizeof(MmaSmem) + 1024;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1] = pdl[0];
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (a.time_begin) cudaEventRecord(a.time_begin, stream);
    e = cudaLaunchKernelEx(&cfg, skyjepa_mma_kernel, p);
    if (a.time_end) cudaEventRecord(a.time_end, stream);
    if (launches) *launches = 3;
    return e;
}

}  // namespace lwm
