// kernels_lewm_pred.cu — the LeWM predictor's whole autoregressive rollout in
// one launch (bf16 tcgen05, f32 residual stream), for the image model's shape:
// residual width 192 (no input/output projection), V width 1024, MLP 2048,
// pred_proj 2048 with BatchNorm (or none), a one-frame window (history 1, so
// the attention of a token is its V: softmax over one key is exactly 1).
//
// Computation (the reference's rollout_embeddings_with_history, model.rs:94-147;
// ConditionalBlock::forward, modules.rs:232-300, 317-330; Transformer::
// forward_last and pred_proj, modules.rs:349-359, 369-380, 389-398): per step
//   x = frame + pos[0]
//   per layer l:  x += g1 * (V(AdaLN(x; ada_l[0:2])) Wo^T + bo)
//                 x += g2 * (GELU(AdaLN(x; ada_l[3:5]) W1^T + b1) W2^T + b2)
//   frame' = pred_proj(LN(x))   (fc1 -> BatchNorm -> GELU -> fc2)
// with the AdaLN table ada_l of every (token, time) precomputed by the caller
// (it depends on the candidate's action only).
//
// Layout: one cluster of 8 CTAs per 128 tokens (the MMA's M).  Every GEMM
// pair of a half-layer is split tensor-parallel over the cluster: CTA j
// computes columns [N1 j / 8, N1 (j+1) / 8) of the first GEMM (V, fc1) and,
// with those as its K slice, a partial sum of the second (out-projection,
// fc2) over all 192 outputs.  CTA j owns tokens [16 j, 16 j + 16): it holds
// their residual stream in registers, sums the 8 partials of its tokens (in
// CTA order), applies bias, gate and residual, runs the next LayerNorm /
// AdaLN, and publishes its 16 rows of the next bf16 A operand.  Partials and
// A rows go through per-cluster exchange buffers in global memory (L2); each
// publish ends with one cluster-scope release and a remote mbarrier arrival
// on every CTA of the cluster.
//
// Roles (320 threads): warp 0 lane 0 streams this CTA's weight blocks through
// a 3-stage ring (one 1-D bulk copy each), lane 1 gathers the 8 owners' A
// rows; warp 1 issues the MMAs (TMEM: first GEMM at columns [0, 256), second
// at [256, 448)); warps 2-9 drain the accumulators (bias, activation, bf16 or
// f32 partials) and do the owner work.  Every wait is bounded and records
// its site in the error word on giving up; the kernel then unwinds.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "lwm_device.cuh"
#include "lwm_lewm.hpp"
#include "lwm_tc.cuh"

namespace lwm {

namespace {

constexpr uint32_t kTP = 8;                 // CTAs per cluster
constexpr uint32_t kM = 128;                // tokens per cluster
constexpr uint32_t kOwn = kM / kTP;         // 16 tokens a CTA owns
constexpr uint32_t kD = 192;                // residual width
constexpr uint32_t kKB = 64;                // K block (SW128: 128-byte rows)
constexpr uint32_t kDKB = kD / kKB;         // 3
constexpr uint32_t kBlk = kM * 128;         // one [128 x 64] bf16 A block: 16 KB
constexpr uint32_t kHBlks = 4;              // H: up to 256 columns
constexpr uint32_t kN1Max = 256;            // first GEMM columns per CTA
constexpr uint32_t kPartRow = kD * 4;       // a partial row: 768 bytes
constexpr uint32_t kPartChunk = kOwn * kPartRow;  // an owner's 16 partial rows: 12 KB
constexpr uint32_t kStage = 32 * 1024;      // weight ring stage (a [256 x 64] block)
constexpr uint32_t kStages = 3;
constexpr uint32_t kColD2 = 256;            // TMEM column of the second GEMM's accumulator
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kCompWarp0 = 2, kCompWarps = 16, kCompThreads = kCompWarps * 32, kCompBarrier = 1;
constexpr uint32_t kThreads = (kCompWarp0 + kCompWarps) * 32;  // 576
constexpr uint32_t kColSplit = kCompWarps / 4;  // compute warps per TMEM lane quadrant
constexpr uint32_t kRowsPerWarp = kOwn / kCompWarps;
constexpr uint32_t kOwnChunk = kOwn * 128;  // an owner's 16 rows of one A block: 2 KB
constexpr uint32_t kPerLane = kD / 32;      // 6 residual columns a lane holds

// half-layer kinds
constexpr int kAttn = 0, kMlp = 1, kPred = 2;

struct __align__(1024) PredSmem {
    uint8_t X[kDKB][kBlk];         // the gathered A operand (AdaLN / LN output), bf16 SW128
    uint8_t H[kHBlks][kBlk];       // the first GEMM's output slice, bf16 SW128 (A of the second)
    uint8_t W[kStages][kStage];    // weight blocks
    uint8_t own[kDKB][kOwnChunk];  // this CTA's 16 rows of the next A, before the bulk store
    float b1s[kN1Max];             // the first GEMM's bias of this CTA's columns
    float bns[4][kN1Max];          // and pred_proj's BatchNorm weight, bias, mean, variance
    uint64_t w_full[kStages], w_empty[kStages];
    uint64_t a_full, x_free, d1_full, d2_full, h_free, d1_drained, d2_drained, done;
    uint64_t h_ready[kHBlks];      // K block kb of H is written (every compute warp arrives once)
    uint64_t a_ready[2], p_ready[2];  // remote: the 8 owners' A rows / the 8 CTAs' partials, by parity
    uint32_t tmem;
};
static_assert(sizeof(PredSmem) + 1024 <= 232448, "shared memory budget of one CTA");

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t peer_addr(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
__device__ __forceinline__ void arrive_peer_relaxed(uint32_t addr) {
    asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void comp_sync() {
    asm volatile("bar.sync %0, %1;" ::"n"(kCompBarrier), "n"(kCompThreads) : "memory");
}
// True on every compute thread iff `v` is true on all of them: the compute
// warps take every wait's outcome through it, so they leave their loop
// together and never meet comp_sync() short of a warp.
__device__ __forceinline__ bool comp_all(bool v) {
    uint32_t out;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(out)
        : "r"(static_cast<uint32_t>(v)), "n"(kCompBarrier), "n"(kCompThreads)
        : "memory");
    return out != 0;
}
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
__device__ __forceinline__ void record_error(volatile int* err, int site, int detail, uint32_t parity) {
    if (atomicCAS(const_cast<int*>(err), 0, site) == 0) {
        err[1] = static_cast<int>(blockIdx.x);
        err[2] = detail;
        err[3] = static_cast<int>(parity);
    }
}
__device__ __forceinline__ bool wait_cluster(uint64_t* bar, uint32_t parity, volatile int* err, int site, int detail,
                                             uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i) {
        if (try_cluster(bar, parity)) return true;
        if ((i & 1023u) == 1023u && err[0]) return false;
    }
    record_error(err, site, detail, parity);
    return false;
}
// Bulk copy shared -> global, waited for to completion and ordered for the
// async proxy (the peers read it with bulk copies).
__device__ __forceinline__ void bulk_s2g_wait(void* dst, uint32_t src, uint32_t bytes) {
    asm volatile(
        "cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n\t"
        "cp.async.bulk.commit_group;\n\t"
        "cp.async.bulk.wait_group 0;\n\t"
        "fence.proxy.async.global;" ::"l"(dst),
        "r"(src), "r"(bytes)
        : "memory");
}
__device__ __forceinline__ uint16_t bf16_bits(float v) {
    const __nv_bfloat16 b = __float2bfloat16_rn(v);
    return *reinterpret_cast<const uint16_t*>(&b);
}
__device__ __forceinline__ float warp_sum32(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// LayerNorm statistics of a row of 192 held as 6 values per lane, as
// row_stats / ada_ln_kernel form them: mean = sum / d, den = sqrt(sum((x -
// mean)^2) / d + eps).
__device__ __forceinline__ void row_norm(const float (&v)[kPerLane], float eps, float& mean, float& den) {
    float s = 0.0f;
#pragma unroll
    for (uint32_t i = 0; i < kPerLane; ++i) s += v[i];
    mean = warp_sum32(s) / static_cast<float>(kD);
    float q = 0.0f;
#pragma unroll
    for (uint32_t i = 0; i < kPerLane; ++i) {
        const float c = v[i] - mean;
        q += c * c;
    }
    den = sqrtf(warp_sum32(q) / static_cast<float>(kD) + eps);
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1) lewm_pred_kernel(const __grid_constant__ PredArgs p) {
    extern __shared__ uint8_t smem_raw[];
    PredSmem& s = *reinterpret_cast<PredSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t c = cluster_rank();
    const uint32_t tile = blockIdx.x / kTP;
    volatile int* err = p.err;
    const uint32_t lim = p.wait_polls ? p.wait_polls : tc::kWaitLimit;
    const uint32_t G = p.steps * p.halves;  // half-layers of the whole rollout

    // ---- setup
    if (warp == 1) tc::tmem_alloc(&s.tmem, kTmemCols);
    if (tid == 0) {
        for (uint32_t i = 0; i < kStages; ++i) {
            tc::mbar_init(&s.w_full[i], 1);
            tc::mbar_init(&s.w_empty[i], 1);
        }
        tc::mbar_init(&s.a_full, 1);
        tc::mbar_init(&s.x_free, 1);
        tc::mbar_init(&s.d1_full, 1);
        tc::mbar_init(&s.d2_full, 1);
        for (uint32_t kb = 0; kb < kHBlks; ++kb) tc::mbar_init(&s.h_ready[kb], kCompWarps);
        tc::mbar_init(&s.h_free, 1);
        tc::mbar_init(&s.d1_drained, kCompWarps);
        tc::mbar_init(&s.d2_drained, kCompWarps);
        tc::mbar_init(&s.done, 1);
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&s.a_ready[i], kTP);
            tc::mbar_init(&s.p_ready[i], kTP);
        }
        tc::mbar_fence_init();
    }
    tc::fence_before();
    __syncthreads();
    cluster_sync_all();  // every CTA's barriers exist before any remote arrival
    tc::fence_after();
    const uint32_t tmem = s.tmem;
    bool failed = false;
    uint8_t* xa_tile = p.xa + static_cast<size_t>(tile) * 2 * kTP * kDKB * kOwnChunk;
    float* xp_tile = p.xp + static_cast<size_t>(tile) * 2 * kTP * kTP * kOwn * kD;

    if (warp == 0) {
        if (lane == 0) {
            // ================= weight blocks, in the order the MMAs consume them
            uint32_t n = 0;  // blocks issued
            bool ok = true;
            for (uint32_t g = 0; ok && g < G; ++g) {
                const PredHalf& hf = p.half[g % p.halves];
                const uint8_t* src = hf.w + static_cast<size_t>(c) * hf.bytes;
                const uint32_t b1 = hf.n1 * 128, nb = kDKB + hf.n1 / kKB;
                for (uint32_t k = 0; k < nb; ++k, ++n) {
                    const uint32_t slot = n % kStages, use = n / kStages;
                    if (!(ok = tc::mbar_wait(&s.w_empty[slot], (use & 1u) ^ 1u, err, 1, n, lim))) break;
                    const uint32_t bytes = k < kDKB ? b1 : kD * 128;
                    tc::mbar_expect_tx(&s.w_full[slot], bytes);
                    tc::bulk_g2s(s.W[slot], src, bytes, &s.w_full[slot]);
                    src += bytes;
                }
            }
            // copies issued and maybe not consumed land before the CTA exits
            for (uint32_t slot = 0; slot < kStages && slot < n; ++slot) {
                const uint32_t last = slot + ((n - 1 - slot) / kStages) * kStages;
                tc::mbar_wait_landing(&s.w_full[slot], (last / kStages) & 1u, lim);
            }
        } else if (lane == 1) {
            // ================= the A operand of every half-layer: 8 owners x 3 blocks of 2 KB
            bool ok = true;
            uint32_t g = 0;
            for (; ok && g < G; ++g) {
                if (g > 0 && !(ok = tc::mbar_wait(&s.x_free, (g - 1) & 1u, err, 2, g, lim))) break;
                if (!(ok = wait_cluster(&s.a_ready[g & 1u], (g >> 1) & 1u, err, 3, g, lim))) break;
                tc::mbar_expect_tx(&s.a_full, kDKB * kM * 128);
                const uint8_t* src = xa_tile + static_cast<size_t>(g & 1u) * kTP * kDKB * kOwnChunk;
                for (uint32_t o = 0; o < kTP; ++o)
                    for (uint32_t kb = 0; kb < kDKB; ++kb)
                        tc::bulk_g2s(s.X[kb] + o * kOwnChunk, src + (o * kDKB + kb) * kOwnChunk, kOwnChunk,
                                     &s.a_full);
            }
            if (g > 0) tc::mbar_wait_landing(&s.a_full, (g - 1) & 1u, lim);
        }
    } else if (warp == 1) {
        // ================= MMA issuer (the whole warp, converged; one elected lane issues)
        {
            const uint32_t xb = tc::smem_u32(s.X[0]), hb = tc::smem_u32(s.H[0]), wb = tc::smem_u32(s.W[0]);
            // every lane waits; the outcome is the warp's (a diverged lane would leave elect.sync short)
            auto wwait = [&](uint64_t* bar, uint32_t parity, volatile int* e, int site, uint32_t detail,
                             uint32_t limit) -> bool {
                return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity, e, site, static_cast<int>(detail), limit));
            };
            uint32_t n = 0;
            bool ok = true;
            for (uint32_t g = 0; ok && g < G; ++g) {
                const PredHalf& hf = p.half[g % p.halves];
                const uint32_t ph = g & 1u, nkb2 = hf.n1 / kKB;
                // first GEMM: D1 = X W1^T ([128 x 192] x [192 x n1])
                if (g > 0 && !(ok = wwait(&s.d1_drained, (g - 1) & 1u, err, 4, g, lim))) break;
                if (!(ok = wwait(&s.a_full, ph, err, 5, g, lim))) break;
                tc::fence_after();
                const uint32_t id1 = tc::idesc_bf16_f32(kM, hf.n1);
                for (uint32_t kb = 0; ok && kb < kDKB; ++kb, ++n) {
                    const uint32_t slot = n % kStages;
                    if (!(ok = wwait(&s.w_full[slot], (n / kStages) & 1u, err, 6, n, lim))) break;
                    tc::fence_after();
                    const uint64_t da = tc::smem_desc(xb + kb * kBlk, 16, 1024, tc::kSwizzle128);
                    const uint64_t db = tc::smem_desc(wb + slot * kStage, 16, 1024, tc::kSwizzle128);
#pragma unroll
                    for (uint32_t k = 0; k < kKB / 16; ++k)
                        tc::mma_bf16_w(tmem, da + 2 * k, db + 2 * k, id1, (kb | k) ? 1u : 0u);
                    tc::commit_w(&s.w_empty[slot]);
                }
                if (!ok) break;
                tc::commit_w(&s.x_free);
                tc::commit_w(&s.d1_full);
                // second GEMM: D2 = H W2^T ([128 x n1] x [n1 x 192]), this CTA's K slice
                if (g > 0 && !(ok = wwait(&s.d2_drained, (g - 1) & 1u, err, 7, g, lim))) break;
                const uint32_t id2 = tc::idesc_bf16_f32(kM, kD);
                for (uint32_t kb = 0; ok && kb < nkb2; ++kb, ++n) {
                    // each K block as soon as the drains have written it
                    if (!(ok = wwait(&s.h_ready[kb], ph, err, 8, g, lim))) break;
                    tc::fence_after();
                    const uint32_t slot = n % kStages;
                    if (!(ok = wwait(&s.w_full[slot], (n / kStages) & 1u, err, 9, n, lim))) break;
                    tc::fence_after();
                    const uint64_t da = tc::smem_desc(hb + kb * kBlk, 16, 1024, tc::kSwizzle128);
                    const uint64_t db = tc::smem_desc(wb + slot * kStage, 16, 1024, tc::kSwizzle128);
#pragma unroll
                    for (uint32_t k = 0; k < kKB / 16; ++k)
                        tc::mma_bf16_w(tmem + kColD2, da + 2 * k, db + 2 * k, id2, (kb | k) ? 1u : 0u);
                    tc::commit_w(&s.w_empty[slot]);
                }
                if (!ok) break;
                tc::commit_w(&s.h_free);
                tc::commit_w(&s.d2_full);
            }
            failed = !ok;
            // every MMA issued has completed before TMEM is released
            tc::commit_w(&s.done);
            tc::mbar_wait_landing(&s.done, 0, lim);
        }
    } else {
        // ================= accumulator drains and the owner work
        const uint32_t cw = warp - kCompWarp0;          // 0..7
        const uint32_t q = warp & 3u, part = cw >> 2;   // TMEM lane quadrant, column part
        const uint32_t row = q * 32 + lane;             // accumulator row = token of the tile
        const uint32_t lane_base = tmem + ((q * 32) << 16);
        // the owned tokens of this warp: rows 2 cw, 2 cw + 1 of the CTA's 16
        const uint32_t tok0 = tile * kM + c * kOwn + kRowsPerWarp * cw;
        bool live[kRowsPerWarp];
#pragma unroll
        for (uint32_t r = 0; r < kRowsPerWarp; ++r) live[r] = tok0 + r < p.tokens;
        float x[kRowsPerWarp][kPerLane];
        uint8_t* own_base = s.own[0];
        const uint32_t own_s = tc::smem_u32(own_base);

        // The next half-layer's AdaLN inputs of the owned rows (shift and
        // scale of this lane's columns, and the LayerNorm affine), fetched
        // ahead of the wait that precedes their use.
        struct Next {
            float sh[kRowsPerWarp][kPerLane], sc[kRowsPerWarp][kPerLane], lw[kPerLane], lb[kPerLane];
            int kind;
        };
        auto fetch_next = [&](uint32_t g_next, Next& nx) {
            const PredHalf& hn = p.half[g_next % p.halves];
            nx.kind = hn.kind;
            const uint32_t step = g_next / p.halves;
#pragma unroll
            for (uint32_t i = 0; i < kPerLane; ++i) {
                nx.lw[i] = __ldg(hn.ln_w + lane + 32 * i);
                nx.lb[i] = __ldg(hn.ln_b + lane + 32 * i);
            }
            if (hn.kind == kPred) return;
            const uint32_t sh_off = hn.kind == kAttn ? 0 : 3 * kD, sc_off = sh_off + kD;
#pragma unroll
            for (uint32_t r = 0; r < kRowsPerWarp; ++r) {
                const uint32_t tok = live[r] ? tok0 + r : 0;
                const size_t arow = static_cast<size_t>(tok) * p.T + (p.h - 1 + step);
                const float* a = p.ada + (static_cast<size_t>(hn.layer) * p.tokens * p.T + arow) * 6 * kD;
#pragma unroll
                for (uint32_t i = 0; i < kPerLane; ++i) {
                    nx.sh[r][i] = __ldg(a + sh_off + lane + 32 * i);
                    nx.sc[r][i] = __ldg(a + sc_off + lane + 32 * i);
                }
            }
        };
        // the A rows of the next half-layer from the owned residual rows
        auto publish_a = [&](uint32_t g_next, const Next& nx) {
#pragma unroll
            for (uint32_t r = 0; r < kRowsPerWarp; ++r) {
                float v[kPerLane];
#pragma unroll
                for (uint32_t i = 0; i < kPerLane; ++i) v[i] = x[r][i];
                float mean, den;
                if (nx.kind == kPred) {
                    // Transformer::forward_last's final LayerNorm (eps 1e-5)
                    row_norm(v, 1e-5f, mean, den);
#pragma unroll
                    for (uint32_t i = 0; i < kPerLane; ++i) v[i] = (v[i] - mean) / den * nx.lw[i] + nx.lb[i];
                } else {
                    // AdaLN: LN(1e-6) -> * (scale + 1) + shift -> LN(1e-5) affine
                    row_norm(v, 1e-6f, mean, den);
#pragma unroll
                    for (uint32_t i = 0; i < kPerLane; ++i) v[i] = (v[i] - mean) / den * (nx.sc[r][i] + 1.0f) + nx.sh[r][i];
                    row_norm(v, 1e-5f, mean, den);
#pragma unroll
                    for (uint32_t i = 0; i < kPerLane; ++i) v[i] = (v[i] - mean) / den * nx.lw[i] + nx.lb[i];
                }
                // bf16, SW128 K-major: row 2 cw + r of the owner's 16, column col
                const uint32_t orow = kRowsPerWarp * cw + r;
#pragma unroll
                for (uint32_t i = 0; i < kPerLane; ++i) {
                    const uint32_t col = lane + 32 * i, kb = col / kKB;
                    *reinterpret_cast<uint16_t*>(own_base + kb * kOwnChunk + tc::sw128_offset(orow, col % kKB)) =
                        bf16_bits(live[r] ? v[i] : 0.0f);
                }
            }
            tc::fence_async_smem();
            comp_sync();
            if (cw == 0 && lane == 0) {
                uint8_t* dst = xa_tile + static_cast<size_t>(g_next & 1u) * kTP * kDKB * kOwnChunk +
                               static_cast<size_t>(c) * kDKB * kOwnChunk;
                bulk_s2g_wait(dst, own_s, kDKB * kOwnChunk);
                asm volatile("fence.release.cluster;" ::: "memory");
                const uint32_t bar = tc::smem_u32(&s.a_ready[g_next & 1u]);
                for (uint32_t d = 0; d < kTP; ++d) arrive_peer_relaxed(peer_addr(bar, d));
            }
        };

        // the first step's input: x = frame + pos[0], the frame the last context embedding
        for (uint32_t r = 0; r < kRowsPerWarp; ++r) {
            const uint32_t tok = live[r] ? tok0 + r : 0;
            const float* e = p.emb + (static_cast<size_t>(tok / p.S) * p.h + (p.h - 1)) * kD;
#pragma unroll
            for (uint32_t i = 0; i < kPerLane; ++i) {
                const uint32_t col = lane + 32 * i;
                x[r][i] = __ldg(e + col) + __ldg(p.pos + col);
            }
        }
        Next nx;
        fetch_next(0, nx);
        publish_a(0, nx);
        bool ok = true;
        for (uint32_t g = 0; ok && g < G; ++g) {
            const uint32_t hi = g % p.halves;
            const int kind = p.half[hi].kind;
            const uint32_t n1 = p.half[hi].n1, layer = p.half[hi].layer;
            const float* b1 = p.half[hi].b1;
            const float* b2 = p.half[hi].b2;
            const float *bn_w = p.half[hi].bn_w, *bn_b = p.half[hi].bn_b, *bn_rm = p.half[hi].bn_rm,
                        *bn_rv = p.half[hi].bn_rv;
            const uint32_t ph = g & 1u, step = g / p.halves;
            // ---- first GEMM's slice -> bias, activation -> bf16 H (this warp's column half);
            // the per-column parameters staged once, while the MMA runs
            {
                const uint32_t t = cw * 32 + lane, gc = c * n1 + t;
                if (t < n1) {
                    s.b1s[t] = b1 ? __ldg(b1 + gc) : 0.0f;
                    if (kind == kPred && bn_w) {
                        s.bns[0][t] = __ldg(bn_w + gc);
                        s.bns[1][t] = __ldg(bn_b + gc);
                        s.bns[2][t] = __ldg(bn_rm + gc);
                        s.bns[3][t] = __ldg(bn_rv + gc);
                    }
                }
            }
            ok = tc::mbar_wait(&s.d1_full, ph, err, 10, g, lim);
            if (ok && g > 0) ok = tc::mbar_wait(&s.h_free, (g - 1) & 1u, err, 11, g, lim);
            if (!(ok = comp_all(ok))) break;
            tc::fence_after();
            {
                // K block by K block: warp part p takes columns [16 p, 16 p + 16)
                // of every block, so all warps finish block 0 first and the
                // second GEMM starts on it while the later blocks drain
                const uint32_t nkb = n1 / kKB;
                for (uint32_t kb = 0; kb < kHBlks; ++kb) {
                    if (kb < nkb) {
                        const uint32_t c0 = kb * kKB + part * 16;
                        float v[16];
                        tc::tmem_ld16(lane_base + c0, v);
                        tc::tmem_ld_wait();
                        if (kind == kAttn) {
#pragma unroll
                            for (uint32_t i = 0; i < 16; ++i) v[i] = v[i] + s.b1s[c0 + i];
                        } else if (kind == kMlp) {
#pragma unroll
                            for (uint32_t i = 0; i < 16; ++i) v[i] = gelu_fast(v[i] + s.b1s[c0 + i]);
                        } else {
                            // BatchNorm (eval, with the reciprocal square root), then GELU
#pragma unroll
                            for (uint32_t i = 0; i < 16; ++i) {
                                const uint32_t lc = c0 + i;
                                float t = v[i] + s.b1s[lc];
                                if (bn_w)
                                    t = (t - s.bns[2][lc]) * rsqrtf(s.bns[3][lc] + 1e-5f) * s.bns[0][lc] + s.bns[1][lc];
                                v[i] = gelu_fast(t);
                            }
                        }
                        // 16 columns = 32 bytes of the row, two 16-byte pieces
                        uint8_t* blk = s.H[kb];
#pragma unroll
                        for (uint32_t q8 = 0; q8 < 2; ++q8) {
                            uint32_t pk[4];
#pragma unroll
                            for (uint32_t k = 0; k < 4; ++k)
                                pk[k] = static_cast<uint32_t>(bf16_bits(v[8 * q8 + 2 * k])) |
                                        (static_cast<uint32_t>(bf16_bits(v[8 * q8 + 2 * k + 1])) << 16);
                            *reinterpret_cast<uint4*>(blk + tc::sw128_offset(row, part * 16 + 8 * q8)) =
                                make_uint4(pk[0], pk[1], pk[2], pk[3]);
                        }
                        tc::fence_async_smem();
                    }
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&s.h_ready[kb]);  // (blocks past n1: no data, phase kept in step)
                }
            }
            tc::fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&s.d1_drained);
            // ---- second GEMM's partial -> the exchange, rows grouped by owner
            if (!(ok = comp_all(tc::mbar_wait(&s.d2_full, ph, err, 12, g, lim)))) break;
            tc::fence_after();
            {
                // staged in shared memory (X and H are idle now: the next A
                // gather waits for this CTA's partials, the MMAs of this
                // half-layer are done), one 12 KB chunk per owner, each row's
                // 16-byte units XOR-permuted by row so a warp's stores spread
                // over the banks; the owners undo the permutation
                const uint32_t o = row / kOwn, rr = row % kOwn;
                uint8_t* chunk = (o < 4 ? s.X[0] : s.H[0]) + (o & 3u) * kPartChunk + rr * kPartRow;
                constexpr uint32_t kCols2 = kD / kColSplit;  // 48
                const uint32_t c0 = part * kCols2;
#pragma unroll
                for (uint32_t cc = 0; cc < kCols2; cc += 16) {
                    float v[16];
                    tc::tmem_ld16(lane_base + kColD2 + c0 + cc, v);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (uint32_t i = 0; i < 16; i += 4) {
                        const uint32_t u = ((c0 + cc + i) >> 2) ^ (rr & 7u);
                        *reinterpret_cast<float4*>(chunk + u * 16) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
                    }
                }
            }
            tc::fence_async_smem();
            tc::fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&s.d2_drained);
            comp_sync();  // every row of the partial is staged
            if (cw == 0 && lane == 0) {
                float* dst = xp_tile + (static_cast<size_t>(ph) * kTP + c) * kTP * kOwn * kD;
                for (uint32_t o = 0; o < kTP; ++o)
                    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                                     reinterpret_cast<uint8_t*>(dst) + o * kPartChunk),
                                 "r"(tc::smem_u32((o < 4 ? s.X[0] : s.H[0]) + (o & 3u) * kPartChunk)), "r"(kPartChunk)
                                 : "memory");
                asm volatile("cp.async.bulk.commit_group;\n\tcp.async.bulk.wait_group 0;\n\tfence.proxy.async.global;"
                             ::: "memory");
                asm volatile("fence.release.cluster;" ::: "memory");
                const uint32_t bar = tc::smem_u32(&s.p_ready[ph]);
                for (uint32_t d = 0; d < kTP; ++d) arrive_peer_relaxed(peer_addr(bar, d));
            }
            // ---- owner: this half-layer's gates and the next one's AdaLN inputs, fetched
            // while the partials arrive; then the 8 partials of the owned rows in CTA order
            float gate[kRowsPerWarp][kPerLane], bias2[kPerLane];
            if (kind != kPred) {
                const uint32_t gate_off = kind == kAttn ? 2 * kD : 5 * kD;
#pragma unroll
                for (uint32_t r = 0; r < kRowsPerWarp; ++r) {
                    const uint32_t tok = live[r] ? tok0 + r : 0;
                    const size_t arow = static_cast<size_t>(tok) * p.T + (p.h - 1 + step);
                    const float* gt = p.ada + (static_cast<size_t>(layer) * p.tokens * p.T + arow) * 6 * kD + gate_off;
#pragma unroll
                    for (uint32_t i = 0; i < kPerLane; ++i) gate[r][i] = __ldg(gt + lane + 32 * i);
                }
            }
#pragma unroll
            for (uint32_t i = 0; i < kPerLane; ++i) bias2[i] = b2 ? __ldg(b2 + lane + 32 * i) : 0.0f;
            if (g + 1 < G) fetch_next(g + 1, nx);
            if (!(ok = comp_all(wait_cluster(&s.p_ready[ph], (g >> 1) & 1u, err, 13, g, lim)))) break;
            {
                const float* src = xp_tile + static_cast<size_t>(ph) * kTP * kTP * kOwn * kD;
                float sum[kRowsPerWarp][kPerLane];
#pragma unroll
                for (uint32_t r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
                    for (uint32_t i = 0; i < kPerLane; ++i) sum[r][i] = 0.0f;
#pragma unroll
                for (uint32_t j = 0; j < kTP; ++j)
#pragma unroll
                    for (uint32_t r = 0; r < kRowsPerWarp; ++r) {
                        const uint32_t orow = kRowsPerWarp * cw + r;
                        const float* pr = src + ((static_cast<size_t>(j) * kTP + c) * kOwn + orow) * kD;
#pragma unroll
                        for (uint32_t i = 0; i < kPerLane; ++i) {
                            const uint32_t col = lane + 32 * i, u = (col >> 2) ^ (orow & 7u);
                            sum[r][i] += __ldcg(pr + u * 4 + (col & 3u));
                        }
                    }
#pragma unroll
                for (uint32_t r = 0; r < kRowsPerWarp; ++r) {
#pragma unroll
                    for (uint32_t i = 0; i < kPerLane; ++i) {
                        const uint32_t col = lane + 32 * i;
                        float t = sum[r][i];
                        if (b2) t = t + bias2[i];
                        if (kind == kPred) {
                            // the predicted frame; the next step's input adds pos[0]
                            if (g + 1 == G) {
                                if (live[r]) p.pred[static_cast<size_t>(tok0 + r) * kD + col] = t;
                            } else {
                                x[r][i] = t + __ldg(p.pos + col);
                            }
                        } else {
                            t = gate[r][i] * t;
                            x[r][i] = x[r][i] + t;
                        }
                    }
                }
            }
            if (g + 1 < G) publish_a(g + 1, nx);
        }
        failed = !ok;
    }

    // ---- teardown: TMEM back, then no CTA leaves while a peer may still write to it
    tc::fence_before();
    const int any_failed = __syncthreads_or(failed || err[0]);
    tc::fence_after();
    if (warp == 1) tc::tmem_free(tmem, kTmemCols);
    if (any_failed) {
        // a wait gave up somewhere: let remote arrivals and copies already
        // issued land (a fixed, bounded grace period) before the barrier
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

// ------------------------------------------------------------ packing
//
// Per half-layer and CTA rank j: the first GEMM's rows [n1 j, n1 (j+1)) as
// 3 K blocks of [n1 x 64], then the second GEMM's columns [n1 j, n1 (j+1))
// as n1/64 K blocks of [192 x 64]; bf16, SW128 K-major (each block the exact
// shared-memory image of one MMA operand).
__global__ void pack_pred_kernel(const float* w1, uint32_t w1_row0, uint32_t w1_ld, const float* w2, uint32_t w2_ld,
                                 uint32_t n1, uint8_t* out, uint32_t bytes_per_rank) {
    const uint32_t j = blockIdx.y;  // rank
    const uint32_t n_w1 = n1 * kD, n_w2 = kD * n1;
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_w1 + n_w2) return;
    uint8_t* base = out + static_cast<size_t>(j) * bytes_per_rank;
    if (i < n_w1) {
        const uint32_t r = i / kD, k = i % kD;  // row of the rank's slice, input column
        const float v = w1[static_cast<size_t>(w1_row0 + j * n1 + r) * w1_ld + k];
        uint8_t* blk = base + (k / kKB) * (n1 * 128);
        *reinterpret_cast<uint16_t*>(blk + tc::sw128_offset(r, k % kKB)) = bf16_bits(v);
    } else {
        const uint32_t q = i - n_w1, r = q / n1, k = q % n1;  // output row (of 192), K within the slice
        const float v = w2[static_cast<size_t>(r) * w2_ld + j * n1 + k];
        uint8_t* blk = base + kDKB * (n1 * 128) + (k / kKB) * (kD * 128);
        *reinterpret_cast<uint16_t*>(blk + tc::sw128_offset(r, k % kKB)) = bf16_bits(v);
    }
}

namespace {

bool pred_configure(int dev) {
    static std::mutex mu;
    static int state[64] = {};
    if (dev < 0 || dev >= 64) return false;
    std::lock_guard<std::mutex> lock(mu);
    if (state[dev] == 0) {
        const size_t smem = sizeof(PredSmem) + 1024;
        cudaError_t e = cudaFuncSetAttribute(lewm_pred_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        int n = 0;
        if (e == cudaSuccess) {
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(kTP, 1, 1);
            cfg.blockDim = dim3(kThreads, 1, 1);
            cfg.dynamicSmemBytes = smem;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = kTP;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            e = cudaOccupancyMaxActiveClusters(&n, lewm_pred_kernel, &cfg);
        }
        (void)cudaGetLastError();
        state[dev] = (e == cudaSuccess && n >= 1) ? 1 : 2;
    }
    return state[dev] == 1;
}

}  // namespace

bool lewm_pred_supported(const lwm_lewm_config& c, uint32_t history, const char** why) {
    const uint32_t inner = c.heads * c.dim_head;
    if (history != 1) { *why = "the fused predictor takes one-frame windows"; return false; }
    if (c.embed_dim != kD || c.pred_hidden_dim != kD) { *why = "the fused predictor takes width 192"; return false; }
    auto slice_ok = [](uint32_t n) { return n % (kTP * kKB) == 0 && n / kTP <= 256; };
    if (!slice_ok(inner) || !slice_ok(c.mlp_dim) || !slice_ok(c.pred_proj_hidden)) {
        *why = "the fused predictor's GEMM widths must be multiples of 512 up to 2048";
        return false;
    }
    if (c.pred_proj_norm == LWM_NORM_LAYER) { *why = "the fused predictor's pred_proj norm is BatchNorm or none"; return false; }
    if (c.depth == 0 || 2 * c.depth + 1 > kPredMaxHalves) { *why = "the fused predictor takes depth 1..8"; return false; }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || !pred_configure(dev)) { *why = "no resident 8-CTA cluster"; return false; }
    return true;
}

size_t lewm_pred_half_bytes(uint32_t n1_total) {
    const uint32_t n1 = n1_total / kTP;
    return static_cast<size_t>(kDKB) * n1 * 128 + static_cast<size_t>(n1 / kKB) * kD * 128;
}

cudaError_t lewm_pred_pack(const float* w1, uint32_t w1_row0, uint32_t w1_ld, const float* w2, uint32_t w2_ld,
                           uint32_t n1_total, uint8_t* out, cudaStream_t s) {
    const uint32_t n1 = n1_total / kTP;
    const uint32_t n = 2 * n1 * kD;
    const uint32_t bytes = static_cast<uint32_t>(lewm_pred_half_bytes(n1_total));
    pack_pred_kernel<<<dim3((n + 255) / 256, kTP), 256, 0, s>>>(w1, w1_row0, w1_ld, w2, w2_ld, n1, out, bytes);
    return cudaGetLastError();
}

size_t lewm_pred_exchange_bytes(uint32_t tokens) {
    const size_t tiles = (tokens + kM - 1) / kM;
    return tiles * (2 * kTP * kDKB * kOwnChunk + 2 * kTP * kTP * kOwn * kD * sizeof(float));
}

cudaError_t launch_lewm_pred(const PredArgs& a, cudaStream_t s) {
    const uint32_t tiles = (a.tokens + kM - 1) / kM;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(tiles * kTP, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = sizeof(PredSmem) + 1024;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kTP;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, lewm_pred_kernel, a);
}

}  // namespace lwm
