// lwm_device.cuh — device helpers shared by the planner kernels (sm_100a).
//
// Sampler: Philox4x32-10 (Salmon et al., SC 2011) + Box-Muller.  Draw i of the
// stream for `seed` uses block i>>2; words (0,1) and (2,3) are Box-Muller
// pairs; even lanes take the cosine, odd lanes the sine.  Uniforms are
// (2k+1)*2^-24 from the top 23 bits of a word.  This is the planners' seeded
// sampler (it replaces the cuRAND fill of src/planner.rs:1452-1486; the
// draw-count reservation of :1488-1514 is kept).
#pragma once

#include <cstdint>
#include <utility>

#include "lwm_pdl.hpp"
#include <cuda_runtime.h>

namespace lwm {

__device__ __forceinline__ uint4 philox4x32_10(uint64_t counter, uint64_t key) {
    uint32_t c0 = static_cast<uint32_t>(counter), c1 = static_cast<uint32_t>(counter >> 32);
    uint32_t c2 = 0u, c3 = 0u;
    uint32_t k0 = static_cast<uint32_t>(key), k1 = static_cast<uint32_t>(key >> 32);
#pragma unroll
    for (int round = 0; round < 10; ++round) {
        const uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
        const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
        const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return make_uint4(c0, c1, c2, c3);
}

__device__ __forceinline__ float unit_open(uint32_t word) {
    return static_cast<float>(2u * (word >> 9) + 1u) * 5.9604644775390625e-8f;  // * 2^-24
}

__device__ __forceinline__ float normal_at(uint64_t seed, uint64_t index) {
    const uint4 w = philox4x32_10(index >> 2, seed);
    const uint32_t lane = static_cast<uint32_t>(index & 3u);
    const uint32_t a = (lane & 2u) ? w.z : w.x;
    const uint32_t b = (lane & 2u) ? w.w : w.y;
    const float r = sqrtf(-2.0f * logf(unit_open(a)));
    float s, c;
    sincospif(2.0f * unit_open(b), &s, &c);
    return (lane & 1u) ? r * s : r * c;
}

// Draws 4i .. 4i + 3 of the stream (one Philox block, both Box-Muller pairs):
// the values normal_at gives for those indices.
__device__ __forceinline__ float4 normal_quad(uint64_t seed, uint64_t block) {
    const uint4 w = philox4x32_10(block, seed);
    const float r0 = sqrtf(-2.0f * logf(unit_open(w.x)));
    const float r1 = sqrtf(-2.0f * logf(unit_open(w.z)));
    float s0, c0, s1, c1;
    sincospif(2.0f * unit_open(w.y), &s0, &c0);
    sincospif(2.0f * unit_open(w.w), &s1, &c1);
    return make_float4(r0 * c0, r0 * s0, r1 * c1, r1 * s1);
}

// Programmatic dependent launch (griddepcontrol): a kernel launched with
// cudaLaunchAttributeProgrammaticStreamSerialization may start once every
// CTA of the kernel before it in the stream has called pdl_trigger (or
// exited); pdl_wait returns once that kernel has completed and its writes
// are visible.  Both are no-ops in a kernel launched without the attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launches `kernel`, with programmatic stream serialization while a PdlScope
// is open on the launching thread (the kernel calls pdl_wait before it reads
// what the kernels before it wrote, and before it completes; without the
// attribute both are no-ops).  The ViT encoder's chain of short launches
// gains from it; a chain that interleaves with launches made without it
// (the vector model's predictor) measured slower, so it stays off there.
template <typename... Params, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g_pdl_launch ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Candle's f32 maximum / minimum: (a < b) ? b : a and (a > b) ? b : a.
__device__ __forceinline__ float cmax(float a, float b) { return a < b ? b : a; }
__device__ __forceinline__ float cmin(float a, float b) { return a > b ? b : a; }

// Candle Tensor::gelu (tanh approximation).
__device__ __forceinline__ float gelu_tanh(float v) {
    const float k = 0.7978845608028654f;
    return __fmul_rn(__fmul_rn(0.5f, v),
                     1.0f + tanhf(__fmul_rn(__fmul_rn(k, v),
                                            1.0f + __fmul_rn(__fmul_rn(0.044715f, v), v))));
}

// Hardware tanh (MUFU.TANH, tanh.approx.f32): relative error about 2^-11,
// inside the bf16 paths' tolerance, where its result is rounded to bf16.
__device__ __forceinline__ float tanh_fast(float v) {
    float r;
    asm("tanh.approx.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}
// Candle's tanh-approximation GELU with the hardware tanh (bf16 paths).
__device__ __forceinline__ float gelu_fast(float v) {
    const float u = 0.7978845608028654f * v * fmaf(0.044715f * v, v, 1.0f);
    return 0.5f * v * (1.0f + tanh_fast(u));
}

// 1 / (1 + exp(-v)); the correctly rounded reciprocal equals IEEE 1/x exactly.
__device__ __forceinline__ float sigmoid(float v) { return __frcp_rn(1.0f + expf(-v)); }

// Orderable key of a score: NaN ranks as +inf, -0 as +0; ascending keys give
// ascending scores.  Low word = sample index, so ties resolve to the lower
// index (src/planner.rs:1811, 1830-1833).
__device__ __forceinline__ uint64_t score_key(float v, uint32_t index) {
    if (v != v) v = __int_as_float(0x7f800000);
    if (v == 0.0f) v = 0.0f;
    uint32_t bits = __float_as_uint(v);
    bits = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
    return (static_cast<uint64_t>(bits) << 32) | index;
}

__device__ __forceinline__ float key_score(uint64_t key) {
    uint32_t bits = static_cast<uint32_t>(key >> 32);
    bits = (bits & 0x80000000u) ? (bits & 0x7fffffffu) : ~bits;
    return __uint_as_float(bits);
}

}  // namespace lwm
