// kernels_lewm_tc.cu — bf16 tensor-core GEMM of the LeWM scorer (tcgen05).
//
// C[M,N] = A[M,K] . W[N,K]^T with the scorer's fused epilogue (bias, GELU /
// SiLU, gated residual), for the bf16 predictor / encoder of the LeWM image
// workload.  One 128 x 128 (or 128 x 64) output tile per CTA (N tiles
// narrower at the edge), K in 64-element blocks through two shared-memory
// stages:
//   A  f32 activations from HBM/L2, rounded to bf16 by the loading threads
//      and stored in the SW128 K-major layout (the residual stream and every
//      other activation stay f32);
//   W  bf16 weights [N, K] (converted once per scorer), 16-byte cp.async
//      copies into the same layout;
//   warp 0 (converged, one elected lane) issues tcgen05.mma (M 128, N <= 128,
//   K 16) into a TMEM accumulator and commits each stage to an mbarrier that
//   releases it; the next block's loads run while the tensor core works on
//   this one.  Launched with programmatic dependent launch inside the ViT
//   encoder: the weights of the first block load before the wait for the
//   kernel that wrote the activations.
// The epilogue reads the accumulator with tcgen05.ld (warp w owns TMEM lanes
// 32 (w % 4) .. +31 = rows, w / 4 picks the column half) into a shared-memory
// tile, then writes it a warp per row so that C, the gate table and the
// output move in whole cache lines.  Split-K writes each split's tile to a
// [splits][M][N] partial buffer and splitk_reduce_kernel adds them in split
// order (deterministic) with the epilogue.  Every mbarrier wait is bounded
// and reports through err.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>

#include "lwm_device.cuh"
#include "lwm_lewm.hpp"
#include "lwm_lewm_epi.cuh"
#include "lwm_tc.cuh"

namespace lwm {
namespace {

constexpr uint32_t kTM = 128, kTN = 128, kTK = 64;
constexpr uint32_t kStageA = kTM * kTK * 2, kStageB = kTN * kTK * 2;  // 16 KB each
constexpr uint32_t kTileLd = 132;  // f32 row stride of the staged output tile (float4-aligned, fewer bank conflicts)
constexpr uint32_t kStageBytes = 2 * (kStageA + kStageB) > kTM * kTileLd * 4 ? 2 * (kStageA + kStageB) : kTM * kTileLd * 4;
constexpr uint32_t kTcSmem = kStageBytes + 1024 + 64;
constexpr int kSiteStage = 21, kSiteFinal = 22;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__global__ void __launch_bounds__(256, 1) gemm_tc_kernel(GemmArgs g, int* err, uint32_t tn) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;                    // [2][128 rows x 128 B]
    uint8_t* sB = smem + 2 * kStageA;      // [2][128 rows x 128 B]
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStageBytes);  // stage[2], final
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t m0 = blockIdx.y * kTM, n0 = blockIdx.x * tn;
    const uint32_t n_tile = min(tn, g.N - n0), n_mma = (n_tile + 15u) & ~15u;
    const uint32_t kb = blockIdx.z * g.k_chunk, ke = min(g.K, kb + g.k_chunk);
    const uint32_t nblk = (ke - kb + kTK - 1) / kTK;
    if (tid == 0) {
        tc::mbar_init(&bars[0], 1);
        tc::mbar_init(&bars[1], 1);
        tc::mbar_init(&bars[2], 1);
        tc::mbar_fence_init();
    }
    if (warp == 0) tc::tmem_alloc(tmem_slot, 128);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = *tmem_slot;

    // A: 128 rows x 64 k f32 = 2048 float4, 8 per thread; lanes of a warp read
    // two rows' 256 contiguous bytes each.
    float4 ra[8];
    auto load_a = [&](uint32_t k0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t e = static_cast<uint32_t>(i) * 256u + tid;
            const uint32_t row = e >> 4, kq = (e & 15u) * 4u;
            const uint32_t m = m0 + row, k = k0 + kq;
            ra[i] = (m < g.M && k < ke) ? __ldg(reinterpret_cast<const float4*>(g.A + static_cast<size_t>(m) * g.lda + k))
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    auto store_a = [&](uint32_t s) {
        uint8_t* base = sA + s * kStageA;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t e = static_cast<uint32_t>(i) * 256u + tid;
            const uint32_t row = e >> 4, kq = (e & 15u) * 4u;
            const __nv_bfloat162 lo = __floats2bfloat162_rn(ra[i].x, ra[i].y);
            const __nv_bfloat162 hi = __floats2bfloat162_rn(ra[i].z, ra[i].w);
            uint2 v;
            v.x = *reinterpret_cast<const uint32_t*>(&lo);
            v.y = *reinterpret_cast<const uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(base + tc::sw128_offset(row, kq)) = v;
        }
    };
    // W: the tile's rows x 8 chunks of 16 B, up to 4 per thread; rows past N
    // read nothing (zero-filled); rows past the MMA's N are not copied.
    auto load_b = [&](uint32_t s, uint32_t k0) {
        const uint32_t base = tc::smem_u32(sB + s * kStageB);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t c = static_cast<uint32_t>(i) * 256u + tid;
            const uint32_t row = c >> 3, j = c & 7u;
            if (row >= n_mma) break;
            const uint32_t n = n0 + row, k = k0 + j * 8u;
            const bool ok = n < g.N && k < ke;
            const uint16_t* src = ok ? g.Wb + static_cast<size_t>(n) * g.ldw + k : g.Wb;
            cp_async16(base + tc::sw128_offset(row, j * 8u), src, ok ? 16u : 0u);
        }
    };

    pdl_trigger();  // launched with programmatic serialization (launch_pdl): the next kernel may start
    load_b(0, kb);  // the weights are not written by the kernels before this one
    pdl_wait();     // the activations are: they are complete and visible from here
    load_a(kb);
    store_a(0);
    cp_async_wait_all();
    tc::fence_async_smem();
    __syncthreads();
    const uint32_t idesc = tc::idesc_bf16_f32(kTM, n_mma);
    for (uint32_t i = 0; i < nblk; ++i) {
        const uint32_t s = i & 1u, k0 = kb + i * kTK;
        if (warp == 0) {  // the whole warp, converged; one elected lane issues
            tc::fence_after();
            const uint32_t a0 = tc::smem_u32(sA + s * kStageA), b0 = tc::smem_u32(sB + s * kStageB);
            const uint32_t steps = min(4u, (ke - k0) / 16u);
            for (uint32_t j = 0; j < steps; ++j)
                tc::mma_bf16_w(tmem, tc::smem_desc(a0 + j * 32u, 16, 1024, tc::kSwizzle128),
                               tc::smem_desc(b0 + j * 32u, 16, 1024, tc::kSwizzle128), idesc, (i | j) != 0u);
            tc::commit_w(&bars[s]);
        }
        if (i + 1 < nblk) {
            const uint32_t s2 = s ^ 1u, k1 = k0 + kTK;
            load_a(k1);  // global loads in flight while the MMAs run
            if (i >= 1) tc::mbar_wait(&bars[s2], ((i - 1) >> 1) & 1u, err, kSiteStage, static_cast<int>(i));
            load_b(s2, k1);
            store_a(s2);
            cp_async_wait_all();
            tc::fence_async_smem();
            __syncthreads();
        }
    }
    if (warp == 0) tc::commit_w(&bars[2]);
    tc::mbar_wait(&bars[2], 0, err, kSiteFinal, static_cast<int>(nblk));
    tc::fence_after();

    // accumulator -> shared-memory tile (the stage buffers are free now)
    const uint32_t q = warp & 3u, half = warp >> 2;
    const uint32_t row = q * 32u + lane;
    const uint32_t lane_addr = tmem + ((q * 32u) << 16);
    float* stile = reinterpret_cast<float*>(smem);  // [128][kTileLd]
#pragma unroll 1
    for (uint32_t c = 0; c < 4; ++c) {
        const uint32_t col0 = half * 64u + c * 16u;
        if (col0 >= n_mma) break;
        float v[16];
        tc::tmem_ld16(lane_addr + col0, v);
        tc::tmem_ld_wait();
        float4* dst = reinterpret_cast<float4*>(stile + row * kTileLd + col0);
#pragma unroll
        for (int e = 0; e < 4; ++e) dst[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
    }
    tc::fence_before();
    __syncthreads();
    if (warp == 0) tc::tmem_free(tmem, 128);
    // tile -> global, a warp per row, consecutive columns per lane: the
    // epilogue (or the split's partial) is written, and C / the gate read,
    // in whole cache lines; each lane takes 4 rows (8 apart) at a time and
    // issues their loads before it uses them
    const bool split = g.splits > 1;
    float* part = split ? g.partial + static_cast<size_t>(blockIdx.z) * g.M * g.N : nullptr;
    for (uint32_t r0 = warp; r0 < kTM; r0 += 32u) {
        if (m0 + r0 >= g.M) break;
        for (uint32_t col = lane; col < n_tile; col += 32u) {
            const uint32_t n = n0 + col;
            float v[4], cv[4], gv[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t r = r0 + 8u * q, m = m0 + r;
                v[q] = stile[r * kTileLd + col];
                cv[q] = 0.0f;
                gv[q] = 0.0f;
                if (!split && g.residual && m < g.M) {
                    cv[q] = g.C[static_cast<size_t>(m) * g.ldc + n];
                    if (g.gate) gv[q] = g.gate[g.map.row(m) * g.ldg + n];
                }
            }
            const float bias = (!split && g.bias) ? g.bias[n] : 0.0f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t m = m0 + r0 + 8u * q;
                if (m >= g.M) break;
                if (split) {
                    part[static_cast<size_t>(m) * g.N + n] = v[q];
                    continue;
                }
                // epilogue_value's arithmetic: bias, then the gated residual or the activation
                float x = v[q];
                if (g.bias) x = x + bias;
                if (g.residual) {
                    if (g.gate) x = gv[q] * x;
                    x = cv[q] + x;
                } else {
                    x = apply_act(g.act, x);
                }
                g.C[static_cast<size_t>(m) * g.ldc + n] = x;
            }
        }
    }
}

// Split-K: C = epilogue(sum over the splits' partials [splits][M][N], in
// split order), one thread per output (coalesced; every SM takes part).
// The partials of an output are all loaded before they are added (in split
// order); indices are 32-bit (the partial buffer holds under 2^32 floats).
__global__ void __launch_bounds__(256) splitk_reduce_kernel(GemmArgs g) {
    pdl_trigger();  // launched with programmatic serialization (launch_pdl): the next kernel may start
    pdl_wait();     // the kernels before this one are complete and their writes visible
    constexpr uint32_t kMaxSplits = 16;
    const uint32_t total = g.M * g.N, plane = total;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const uint32_t m = i / g.N, n = i - m * g.N;
        float p[kMaxSplits];
#pragma unroll
        for (uint32_t z = 0; z < kMaxSplits; ++z)
            p[z] = z < g.splits ? __ldcg(g.partial + static_cast<size_t>(z) * plane + i) : 0.0f;
        float v = 0.0f;
#pragma unroll
        for (uint32_t z = 0; z < kMaxSplits; ++z)
            if (z < g.splits) v += p[z];
        float* cp = g.C + static_cast<size_t>(m) * g.ldc + n;
        *cp = epilogue_value(g, m, n, v, cp);
    }
}

}  // namespace

bool gemm_tc_eligible(const GemmArgs& g) {
    return g.Wb && g.K >= 16 && g.K % 16 == 0 && g.lda % 4 == 0 && g.ldw % 8 == 0 &&
           (reinterpret_cast<uintptr_t>(g.A) & 15u) == 0 && (reinterpret_cast<uintptr_t>(g.Wb) & 15u) == 0;
}

// Output tiles are 128 x 128, or 128 x 64 when the 128-wide tiles would not
// give every SM a CTA (two CTAs fit an SM, so one's epilogue overlaps the
// other's loads); then K is split when the tiles alone still leave SMs idle:
// about one wave of CTAs, at least two 64-wide K blocks per split, at most 16
// splits.
cudaError_t gemm_tc(const GemmArgs& in, cudaStream_t stream, const SplitScratch* sp, int* err) {
    static std::atomic<bool> configured[64] = {};  // the attribute is per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64 || !configured[dev]) {
        e = cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kTcSmem));
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    GemmArgs g = in;
    const uint32_t ty = (g.M + kTM - 1) / kTM;
    const uint32_t tn = (static_cast<size_t>((g.N + kTN - 1) / kTN) * ty < 148 && g.N > 64) ? 64u : kTN;
    const uint32_t tx = (g.N + tn - 1) / tn;
    const size_t tiles = static_cast<size_t>(tx) * ty;
    uint32_t splits = 1;
    if (sp && sp->partial && tiles < 148 && g.K >= 2 * 2 * kTK && static_cast<uint64_t>(g.M) * g.N < (1ull << 31)) {
        splits = static_cast<uint32_t>((148 + tiles - 1) / tiles);
        splits = min(splits, min(16u, g.K / (2 * kTK)));
        while (splits > 1 && static_cast<size_t>(splits) * g.M * g.N > sp->floats) --splits;
    }
    g.splits = splits;
    g.k_chunk = splits > 1 ? ((g.K + splits - 1) / splits + kTK - 1) / kTK * kTK : g.K;
    if (splits > 1) {
        g.splits = (g.K + g.k_chunk - 1) / g.k_chunk;  // no empty split
        g.partial = sp->partial;
    }
    dim3 grid(tx, ty, g.splits);
    if ((e = launch_pdl(gemm_tc_kernel, grid, dim3(256), kTcSmem, stream, g, err, tn)) != cudaSuccess || g.splits <= 1)
        return e;
    const uint64_t total = static_cast<uint64_t>(g.M) * g.N;
    e = launch_pdl(splitk_reduce_kernel, dim3(static_cast<uint32_t>(std::min<uint64_t>((total + 255) / 256, 148 * 8))),
                   dim3(256), 0, stream, g);
    if (e != cudaSuccess) return e;
    if (sp->extra_launches) ++*sp->extra_launches;
    return cudaGetLastError();
}

__global__ void f32_to_bf16_kernel(const float* src, __nv_bfloat16* dst, size_t n) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        dst[i] = __float2bfloat16_rn(src[i]);
}

cudaError_t launch_f32_to_bf16(const float* src, uint16_t* dst, size_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const unsigned blocks = static_cast<unsigned>(std::min<size_t>((n + 255) / 256, 148 * 8));
    f32_to_bf16_kernel<<<blocks, 256, 0, s>>>(src, reinterpret_cast<__nv_bfloat16*>(dst), n);
    return cudaGetLastError();
}

}  // namespace lwm
