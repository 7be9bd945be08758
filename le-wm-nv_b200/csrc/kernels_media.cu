// kernels_media.cu — image preprocessing for the ViT encoder: packed
// RGB/BGR(A) or NV12 u8 frames -> bilinear resize (half-pixel centres) ->
// [0,1] -> (x - mean) / std -> NCHW (or one slot of an [B, history, 3, H, W]
// buffer), f32 or bf16.
//
// Reference kernels: swm_packed_u8_to_nchw_f32 and swm_nv12_to_nchw_f32
// (src/media/mod.rs:1113-1194, 1196-1333).  Here one thread produces all
// three channels of an output pixel (the reference's packed kernel runs one
// thread per output element and repeats the coordinate math and the four
// taps per channel), so every source byte is read once per pixel; the
// row-staged kernels go further (below).  The output can also be the ViT's
// patch matrix, so the patch-embedding GEMM reads the preprocessed frames
// directly.  Compiled with -fmad=false: every product and sum is rounded on
// its own.
#include <cuda_bf16.h>

#include <cmath>
#include <cstdint>
#include <mutex>
#include <type_traits>

#include "lwm_kernels.hpp"
#include "lwm_tc.cuh"

namespace lwm {


__device__ __forceinline__ float clampf(float v, float lo, float hi) { return fminf(fmaxf(v, lo), hi); }

// ------------------------------------------------------------ output maps
//
// Where element (frame b, channel c, row y, column x) of the normalised
// image goes: NCHW (or one slot of an [B, history, 3, H, W] buffer), or —
// with a.patch = p > 0 — the ViT's patch matrix [B, (H/p)(W/p), 3 p p]
// (the patch-embedding convolution's input, vit.rs:32-52), at patch
// (y / p, x / p), column c p p + (y % p) p + x % p.  An offset is
// row_base(b, y) + col(x) + c * plane; four columns 4j .. 4j+3 are
// contiguous in both layouts (p a multiple of 4).
__device__ __forceinline__ size_t out_row_base(const MediaArgs& a, uint32_t b, uint32_t y) {
    if (a.patch) {
        const uint32_t p = a.patch, side = a.out_w / p;
        return (static_cast<size_t>(b) * (a.out_h / p) * side + static_cast<size_t>(y / p) * side) * (3u * p * p) +
               static_cast<size_t>(y % p) * p;
    }
    const uint32_t frames = a.history_len ? a.history_len : 1u, slot = a.history_len ? a.history_slot : 0u;
    return ((static_cast<size_t>(b) * frames + slot) * 3u * a.out_h + y) * a.out_w;
}
__device__ __forceinline__ size_t out_col(const MediaArgs& a, uint32_t x) {
    return a.patch ? static_cast<size_t>(x / a.patch) * (3u * a.patch * a.patch) + x % a.patch : x;
}
__device__ __forceinline__ size_t out_plane(const MediaArgs& a) {
    return a.patch ? static_cast<size_t>(a.patch) * a.patch : static_cast<size_t>(a.out_h) * a.out_w;
}

// ------------------------------------------------------ per-pixel kernels
//
// For the shapes the row-staged kernels below do not take.  One thread per
// output pixel makes all three channels: the source coordinates and the
// bilinear neighbours are found once per axis, the taps of every channel
// come from the same neighbours, the result is normalised and stored.

// One resampling axis: the neighbours of a source coordinate clamped to
// [0, n - 1] and the weight of the upper one.
struct Axis {
    uint32_t i0, i1;
    float w;
};
__device__ __forceinline__ Axis axis_of(float s, uint32_t n) {
    s = clampf(s, 0.0f, static_cast<float>(n - 1u));
    const float f = floorf(s);
    const uint32_t i0 = static_cast<uint32_t>(f);
    return {i0, i0 + 1u < n ? i0 + 1u : i0, s - f};
}

// Four taps blended along x within each row, then along y (the order the
// reference rounds in: swm_sample_plane, src/media/mod.rs:1201-1230).
__device__ __forceinline__ float blend(float v00, float v01, float v10, float v11, float wx, float wy) {
    const float top = v00 + (v01 - v00) * wx;
    const float bottom = v10 + (v11 - v10) * wx;
    return top + (bottom - top) * wy;
}

__device__ __forceinline__ void store_pixel(const MediaArgs& a, uint32_t b, uint32_t y, uint32_t x,
                                            const float (&v)[3]) {
    const size_t base = out_row_base(a, b, y) + out_col(a, x), plane = out_plane(a);
#pragma unroll
    for (uint32_t c = 0; c < 3; ++c) {
        const float normalized = (v[c] - a.mean[c]) / a.std[c];
        if (a.bf16) static_cast<__nv_bfloat16*>(a.out)[base + c * plane] = __float2bfloat16_rn(normalized);
        else static_cast<float*>(a.out)[base + c * plane] = normalized;
    }
}

// (b, y, x) of output pixel `idx`.
__device__ __forceinline__ void pixel_of(const MediaArgs& a, uint64_t idx, uint32_t& b, uint32_t& y, uint32_t& x) {
    x = static_cast<uint32_t>(idx % a.out_w);
    const uint64_t q = idx / a.out_w;
    y = static_cast<uint32_t>(q % a.out_h);
    b = static_cast<uint32_t>(q / a.out_h);
}

// Packed RGB / BGR / RGBA / BGRA (swm_packed_u8_to_nchw_f32, src/media/
// mod.rs:1113-1194): half-pixel source coordinates clamped below at 0.
__global__ void __launch_bounds__(256) packed_pixel_kernel(MediaArgs a) {
    const uint64_t idx = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<uint64_t>(a.batch) * a.out_h * a.out_w) return;
    uint32_t b, y, x;
    pixel_of(a, idx, b, y, x);
    const Axis ay = axis_of(fmaxf((static_cast<float>(y) + 0.5f) * (static_cast<float>(a.in_h) / static_cast<float>(a.out_h)) - 0.5f, 0.0f), a.in_h);
    const Axis ax = axis_of(fmaxf((static_cast<float>(x) + 0.5f) * (static_cast<float>(a.in_w) / static_cast<float>(a.out_w)) - 0.5f, 0.0f), a.in_w);
    const uint32_t C = a.channels;
    const uint8_t* r0 = a.a + (static_cast<size_t>(b) * a.in_h + ay.i0) * a.in_w * C;
    const uint8_t* r1 = a.a + (static_cast<size_t>(b) * a.in_h + ay.i1) * a.in_w * C;
    const bool swap = a.format == 1u || a.format == 3u;  // BGR, BGRA
    float v[3];
#pragma unroll
    for (uint32_t c = 0; c < 3; ++c) {
        const uint32_t k = swap ? 2u - c : c;
        v[c] = blend(__ldg(r0 + ax.i0 * C + k), __ldg(r0 + ax.i1 * C + k), __ldg(r1 + ax.i0 * C + k),
                     __ldg(r1 + ax.i1 * C + k), ax.w, ay.w) * 0.00392156862745098f;
    }
    store_pixel(a, b, y, x, v);
}

// YUV -> RGB of the four NV12 colour spaces (src/media/mod.rs:1298-1318):
// limited range scales (Y - 16)+ by 255/219 first; then R = Y + rv V,
// G = Y - gu U - gv V, B = Y + bu U.
struct ColourSpace {
    int limited;
    float rv, gu, gv, bu;
};
__constant__ ColourSpace kColourSpaces[4] = {
    {1, 1.59602678f, 0.39176229f, 0.81296765f, 2.01723214f},  // BT.601, video range
    {1, 1.79274107f, 0.21324861f, 0.53290933f, 2.11240179f},  // BT.709, video range
    {0, 1.402f, 0.344136f, 0.714136f, 1.772f},                 // BT.601, full range
    {0, 1.5748f, 0.187324f, 0.468124f, 1.8556f},               // BT.709, full range
};

// NV12 (swm_nv12_to_nchw_f32, src/media/mod.rs:1232-1333): luma at the
// half-pixel source coordinate, chroma at half of it on the half-size
// interleaved UV plane, both clamped to their planes.
__global__ void __launch_bounds__(256) nv12_pixel_kernel(MediaArgs a) {
    const uint64_t idx = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<uint64_t>(a.batch) * a.out_h * a.out_w) return;
    uint32_t b, y, x;
    pixel_of(a, idx, b, y, x);
    const float sy = (static_cast<float>(y) + 0.5f) * (static_cast<float>(a.in_h) / static_cast<float>(a.out_h)) - 0.5f;
    const float sx = (static_cast<float>(x) + 0.5f) * (static_cast<float>(a.in_w) / static_cast<float>(a.out_w)) - 0.5f;
    const Axis ly = axis_of(sy, a.in_h), lx = axis_of(sx, a.in_w);
    const uint32_t ch = a.in_h / 2u, cw = a.in_w / 2u;
    const Axis cy = axis_of(sy * 0.5f, ch), cx = axis_of(sx * 0.5f, cw);
    const uint8_t* l0 = a.a + (static_cast<size_t>(b) * a.in_h + ly.i0) * a.in_w;
    const uint8_t* l1 = a.a + (static_cast<size_t>(b) * a.in_h + ly.i1) * a.in_w;
    const float Y = blend(__ldg(l0 + lx.i0), __ldg(l0 + lx.i1), __ldg(l1 + lx.i0), __ldg(l1 + lx.i1), lx.w, ly.w);
    const uint8_t* c0 = a.uv + (static_cast<size_t>(b) * ch + cy.i0) * cw * 2u;
    const uint8_t* c1 = a.uv + (static_cast<size_t>(b) * ch + cy.i1) * cw * 2u;
    float uvv[2];
#pragma unroll
    for (uint32_t k = 0; k < 2; ++k)  // U at even bytes, V at odd bytes
        uvv[k] = blend(__ldg(c0 + 2u * cx.i0 + k), __ldg(c0 + 2u * cx.i1 + k), __ldg(c1 + 2u * cx.i0 + k),
                       __ldg(c1 + 2u * cx.i1 + k), cx.w, cy.w) - 128.0f;
    const ColourSpace cs = kColourSpaces[a.format & 3u];
    const float yy = cs.limited ? fmaxf(Y - 16.0f, 0.0f) * 1.16438356f : Y;
    const float r = yy + cs.rv * uvv[1];
    const float g = yy - cs.gu * uvv[0] - cs.gv * uvv[1];
    const float bl = yy + cs.bu * uvv[0];
    const float v[3] = {clampf(r, 0.0f, 255.0f) * 0.00392156862745098f, clampf(g, 0.0f, 255.0f) * 0.00392156862745098f,
                        clampf(bl, 0.0f, 255.0f) * 0.00392156862745098f};
    store_pixel(a, b, y, x, v);
}

// ------------------------------------------------------------------------
// NV12, row-staged.  The generic kernel above spends most of its issue slots
// on index and conversion arithmetic (64-bit div/mod per pixel, I2F/F2I at
// the conversion rate, a library division per channel); at full HD it runs
// at a sixth of the HBM roofline.  This one keeps the arithmetic of
// swm_nv12_to_nchw_f32 exactly, and removes the rest:
//   * warp-specialised blocks, grid-stride over batch x output rows: one
//     producer thread copies, kStages rows ahead, the two luma rows and two
//     chroma rows each output row taps into shared memory with the
//     bulk-copy engine (cp.async.bulk, one instruction per row, completion
//     on an mbarrier) and writes the row's weights and output offset beside
//     them; the consumer warps take one output row at a time and hand the
//     stage back through a second mbarrier (no block-wide barrier);
//   * a thread owns four adjacent output columns for the whole kernel: their
//     source columns and bilinear weights are computed once, in registers;
//   * taps are u8 loads from shared memory turned into floats with the 2^23
//     bit trick (bits 0x4B0000bb are the float 2^23 + b, exact), and the
//     difference of two taps is taken before the 2^23 is removed (exact);
//   * all per-pixel float arithmetic runs as Blackwell packed f32x2
//     instructions (two pixels per instruction, each lane rounded as its own
//     f32 op, subnormals kept); products that feed an add are written so
//     that ptxas cannot fuse them (see Prod), and the clamp to [0, 255]
//     with the scale by 1/255 is one saturating multiply per value (see
//     unit_clamp);
//   * the division by std is a product with the correctly rounded
//     reciprocal r = 1/std (computed on the host) followed by two
//     remainder corrections q += (a - std q) r; the second starts from a
//     quotient within an ulp, so by Markstein's theorem (Markstein 1990;
//     Cornea, Harrison, Tang 2002) it returns the correctly rounded a / std.
// Taps, weights, products and sums are the same f32 operations, in the same
// order, as the generic kernel's, so its outputs are bit-identical.
namespace staged {

constexpr uint32_t kStages = 4;
constexpr uint32_t kMagic = 0x4B000000u;  // the float 2^23
constexpr uint32_t kMaxConsumers = 512;   // 4 columns each: output rows up to 2048
constexpr uint32_t kMaxThreads = kMaxConsumers + 32;  // + the producer warp
constexpr uint32_t kWaitLimit = 1u << 26;

struct f2 {
    unsigned long long v;
};
__device__ __forceinline__ f2 mk(float a, float b) {
    f2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r.v) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ f2 splat(float a) { return mk(a, a); }
__device__ __forceinline__ float lo(f2 a) {
    float x;
    asm("{\n\t.reg .f32 t;\n\tmov.b64 {%0, t}, %1;\n\t}" : "=f"(x) : "l"(a.v));
    return x;
}
__device__ __forceinline__ float hi(f2 a) {
    float y;
    asm("{\n\t.reg .f32 t;\n\tmov.b64 {t, %0}, %1;\n\t}" : "=f"(y) : "l"(a.v));
    return y;
}
__device__ __forceinline__ f2 add(f2 a, f2 b) {
    f2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
    return r;
}
__device__ __forceinline__ f2 sub(f2 a, f2 b) {
    f2 r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
    return r;
}
__device__ __forceinline__ f2 mul(f2 a, f2 b) {
    f2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
    return r;
}
// A product that feeds an add or a subtract.  ptxas contracts a packed
// f32x2 multiply whose only use is an add into one fused multiply-add (the
// .rn qualifier and -fmad=false notwithstanding), which rounds once where
// swm_nv12_to_nchw_f32 rounds twice.  So the product is written as an fma
// whose addend is -0 read from the kernel parameters: RN(a b + -0) is
// RN(a b) for every a, b (signed zeros included), and with the addend
// unknown at compile time the fma is neither simplified to a multiply nor
// fused with the add that follows.
__device__ __forceinline__ f2 fma(f2 a, f2 b, f2 c);
struct Prod {
    f2 nz;  // (-0, -0), from the kernel parameters
    __device__ __forceinline__ f2 operator()(f2 a, f2 b) const { return fma(a, b, nz); }
    __device__ __forceinline__ f2 operator()(f2 a, float k) const { return fma(a, splat(k), nz); }
};
__device__ __forceinline__ f2 fma(f2 a, f2 b, f2 c) {
    f2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r.v) : "l"(a.v), "l"(b.v), "l"(c.v));
    return r;
}
// clamp(v, 0, 255) / 255 as RN(v RN(1/255)) saturated to [0, 1]: the
// product is monotonic in v and RN(255 RN(1/255)) = 1, so the saturated
// product equals the product of the clamped value (mul.sat: saturation after
// rounding; the clamp of a negative v gives +0, as does the saturation).
// Packed f32x2 multiplies take no .sat, so this one is scalar.
__device__ __forceinline__ float unit_clamp(float a) {
    float r;
    asm("mul.rn.sat.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(0.00392156862745098f));
    return r;
}
__device__ __forceinline__ f2 unit_clamp(f2 a) { return mk(unit_clamp(lo(a)), unit_clamp(hi(a))); }
__device__ __forceinline__ f2 relu(f2 a) { return mk(fmaxf(lo(a), 0.0f), fmaxf(hi(a), 0.0f)); }

// u8 tap -> float with 2^23 added (exact): byte b of `word` under the magic.
__device__ __forceinline__ float magic_byte(uint32_t word, uint32_t sel) {
    return __uint_as_float(__byte_perm(word, kMagic, sel));
}
__device__ __forceinline__ float magic_u8(uint32_t byte) { return __uint_as_float(byte | kMagic); }

// floor of v in [0, 2^23) as an integer and as a float, without conversion
// instructions: v + 2^23 rounded toward zero keeps floor(v) in its low bits.
__device__ __forceinline__ uint32_t floor_u(float v, float& f) {
    const float t = __fadd_rz(v, 8388608.0f);
    f = t - 8388608.0f;
    return __float_as_uint(t) - kMagic;
}

// Bilinear lerp of two pixels' taps held with 2^23 added; weights wx per
// pixel, wy shared (the arithmetic of blend above).
__device__ __forceinline__ f2 bilerp(const Prod& mul, f2 t00, f2 t01, f2 t10, f2 t11, f2 wx, f2 wy) {
    const f2 m = splat(8388608.0f);
    const f2 top = add(sub(t00, m), mul(sub(t01, t00), wx));
    const f2 bottom = add(sub(t10, m), mul(sub(t11, t10), wx));
    return add(top, mul(sub(bottom, top), wy));
}

struct Row {
    uint32_t y0, y1, c0, c1;  // luma and chroma source rows
    float wy, cwy;
};
__device__ __forceinline__ Row row_taps(float sy, uint32_t in_h) {
    Row r;
    float f;
    const float s = clampf(sy, 0.0f, static_cast<float>(in_h - 1u));
    r.y0 = floor_u(s, f);
    r.y1 = r.y0 + 1u < in_h ? r.y0 + 1u : r.y0;
    r.wy = s - f;
    const uint32_t ch = in_h / 2u;
    const float cs = clampf(sy * 0.5f, 0.0f, static_cast<float>(ch - 1u));
    r.c0 = floor_u(cs, f);
    r.c1 = r.c0 + 1u < ch ? r.c0 + 1u : r.c0;
    r.cwy = cs - f;
    return r;
}

__device__ __forceinline__ bool wait_stage(uint64_t* bar, uint32_t parity, uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i)
        if (tc::mbar_try(bar, parity)) return true;
    return false;
}

template <uint32_t CS>
__device__ __forceinline__ void to_rgb(const Prod& mul_sep, f2 Y, f2 U, f2 V, f2& r, f2& g, f2& b) {
    // colour matrices of src/media/mod.rs:1298-1318
    if constexpr (CS == 0u || CS == 1u) {
        const f2 yy = mul_sep(relu(sub(Y, splat(16.0f))), 1.16438356f);
        if constexpr (CS == 0u) {
            r = add(yy, mul_sep(V, 1.59602678f));
            g = sub(sub(yy, mul_sep(U, 0.39176229f)), mul_sep(V, 0.81296765f));
            b = add(yy, mul_sep(U, 2.01723214f));
        } else {
            r = add(yy, mul_sep(V, 1.79274107f));
            g = sub(sub(yy, mul_sep(U, 0.21324861f)), mul_sep(V, 0.53290933f));
            b = add(yy, mul_sep(U, 2.11240179f));
        }
    } else if constexpr (CS == 2u) {
        r = add(Y, mul_sep(V, 1.402f));
        g = sub(sub(Y, mul_sep(U, 0.344136f)), mul_sep(V, 0.714136f));
        b = add(Y, mul_sep(U, 1.772f));
    } else {
        r = add(Y, mul_sep(V, 1.5748f));
        g = sub(sub(Y, mul_sep(U, 0.187324f)), mul_sep(V, 0.468124f));
        b = add(Y, mul_sep(U, 1.8556f));
    }
}

// a / sd with rcp = RN(1 / sd), the division as described above.
__device__ __forceinline__ f2 divide(f2 a, float sd, float rcp) {
    const f2 r = splat(rcp), nsd = splat(-sd);
    f2 q = mul(a, r);
    q = fma(fma(nsd, q, a), r, q);
    return fma(fma(nsd, q, a), r, q);
}

// (clamp(v) / 255 - mean) / std.
__device__ __forceinline__ f2 normalize(f2 v, float mean, float sd, float rcp) {
    return divide(sub(unit_clamp(v), splat(mean)), sd, rcp);
}

// The three channel planes of four adjacent output pixels: one 16-byte
// (f32) or 8-byte (bf16) store per channel.
template <bool BF16>
__device__ __forceinline__ void store4(const MediaArgs& a, size_t base, size_t plane, const f2 (&out)[3][2]) {
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        if constexpr (BF16) {
            const __nv_bfloat162 p0 = __floats2bfloat162_rn(lo(out[c][0]), hi(out[c][0]));
            const __nv_bfloat162 p1 = __floats2bfloat162_rn(lo(out[c][1]), hi(out[c][1]));
            uint2 w;
            w.x = *reinterpret_cast<const uint32_t*>(&p0);
            w.y = *reinterpret_cast<const uint32_t*>(&p1);
            *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a.out) + base + c * plane) = w;
        } else {
            *reinterpret_cast<float4*>(static_cast<float*>(a.out) + base + c * plane) =
                make_float4(lo(out[c][0]), hi(out[c][0]), lo(out[c][1]), hi(out[c][1]));
        }
    }
}

// Per staged row: the row weights and the output offset, written by the
// producer next to the row's copies.
struct RowSlot {
    float wy, cwy;
    unsigned long long base;  // element offset of (frame, channel 0, row y, column 0): out_row_base
};

// Warp-specialised: the last warp's lane 0 is the producer (row weights and
// the four bulk copies of each row, kStages rows ahead); the other warps are
// consumers.  full[s] completes when stage s's bytes have landed, empty[s]
// when every consumer warp is done with it; no block-wide barrier in the
// row loop.
template <uint32_t CS, bool BF16, uint32_t ROWCAP>
__global__ void __launch_bounds__(kMaxThreads, 1) nv12_staged_kernel(MediaArgs a, StagedMedia m) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr uint32_t kStageBytes = 4u * ROWCAP;  // luma y0, luma y1, chroma c0, chroma c1
    RowSlot* slots = reinterpret_cast<RowSlot*>(smem + kStages * kStageBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(slots + kStages);
    uint64_t* empty = full + kStages;
    const uint32_t tid = threadIdx.x, in_w = a.in_w, rows = a.batch * a.out_h;
    const uint32_t consumers = blockDim.x - 32u;
    if (tid == 0) {
        for (uint32_t s = 0; s < kStages; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], consumers / 32u);
        }
        tc::mbar_fence_init();
    }
    __syncthreads();

    if (tid >= consumers) {
        if (tid != consumers) return;
        // producer
        uint32_t k = 0;
        for (;; ++k) {
            const uint32_t r = blockIdx.x + k * gridDim.x;
            if (r >= rows) break;
            const uint32_t s = k % kStages;
            if (k >= kStages && !wait_stage(&empty[s], (k / kStages - 1u) & 1u, m.wait_polls)) {
                m.err[1] = static_cast<int>(blockIdx.x);
                m.err[2] = static_cast<int>(k);
                m.err[3] = 2;
                m.err[0] = 1;
                break;
            }
            const uint32_t b = r / a.out_h, y = r - b * a.out_h;
            const Row t = row_taps((static_cast<float>(y) + 0.5f) * m.ratio_h - 0.5f, a.in_h);
            slots[s].wy = t.wy;
            slots[s].cwy = t.cwy;
            slots[s].base = out_row_base(a, b, y);
            uint8_t* st = smem + s * kStageBytes;
            const size_t frame = static_cast<size_t>(b) * a.in_h;
            if (r == m.skip_row) continue;  // fault injection: this stage never fills
            tc::mbar_expect_tx(&full[s], 4u * in_w);
            tc::bulk_g2s(st, a.a + (frame + t.y0) * in_w, in_w, &full[s]);
            tc::bulk_g2s(st + ROWCAP, a.a + (frame + t.y1) * in_w, in_w, &full[s]);
            tc::bulk_g2s(st + 2u * ROWCAP, a.uv + (frame / 2u + t.c0) * in_w, in_w, &full[s]);
            tc::bulk_g2s(st + 3u * ROWCAP, a.uv + (frame / 2u + t.c1) * in_w, in_w, &full[s]);
        }
        // the copies still in flight land before the block's shared memory
        // can be released
        for (uint32_t j = k > kStages ? k - kStages : 0u; j < k; ++j)
            wait_stage(&full[j % kStages], (j / kStages) & 1u, m.wait_polls);
        return;
    }

    // consumers: the four output columns of this thread, their source
    // columns and weights
    const uint32_t x4 = tid * 4u, lane = tid & 31u;
    const bool active = x4 < a.out_w;
    uint32_t l0[4], l1[4], u0[4], u1[4];
    float wx[4], cwx[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t x = active ? x4 + i : 0u;
        const float sx = (static_cast<float>(x) + 0.5f) * m.ratio_w - 0.5f;
        float f;
        const float s = clampf(sx, 0.0f, static_cast<float>(in_w - 1u));
        l0[i] = floor_u(s, f);
        l1[i] = l0[i] + 1u < in_w ? l0[i] + 1u : l0[i];
        wx[i] = s - f;
        const uint32_t cw = in_w / 2u;
        const float cs = clampf(sx * 0.5f, 0.0f, static_cast<float>(cw - 1u));
        const uint32_t c0 = floor_u(cs, f);
        u0[i] = 2u * c0;
        u1[i] = 2u * (c0 + 1u < cw ? c0 + 1u : c0);
        cwx[i] = cs - f;
    }
    const Prod prod{splat(m.neg_zero)};
    const f2 wxa = mk(wx[0], wx[1]), wxb = mk(wx[2], wx[3]);
    const f2 cwxa = mk(cwx[0], cwx[1]), cwxb = mk(cwx[2], cwx[3]);
    const bool csh[2] = {u0[0] == u0[1] && u1[0] == u1[1], u0[2] == u0[3] && u1[2] == u1[3]};
    const size_t plane = out_plane(a), col = out_col(a, active ? x4 : 0u);

    // one output row from stage S (a compile-time shared-memory offset);
    // returns false once the block's rows are done or a copy never landed
    auto step = [&](uint32_t k, auto stage) -> bool {
        constexpr uint32_t S = decltype(stage)::value;
        if (blockIdx.x + k * gridDim.x >= rows) return false;
        if (!wait_stage(&full[S], (k / kStages) & 1u, m.wait_polls)) {
            if (lane == 0) {
                m.err[1] = static_cast<int>(blockIdx.x);
                m.err[2] = static_cast<int>(k);
                m.err[3] = 1;
                m.err[0] = 1;
            }
            return false;
        }
        if (active) {
            const RowSlot rs = slots[S];
            const uint8_t* ly0 = smem + S * kStageBytes;
            const uint8_t* ly1 = ly0 + ROWCAP;
            const uint8_t* cr0 = ly0 + 2u * ROWCAP;
            const uint8_t* cr1 = ly0 + 3u * ROWCAP;
            const f2 wy = splat(rs.wy), cwy = splat(rs.cwy);
            f2 out[3][2];
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                const int i = 2 * p, j = 2 * p + 1;
                const f2 wxp = p ? wxb : wxa, cwxp = p ? cwxb : cwxa;
                const f2 Y = bilerp(prod, mk(magic_u8(ly0[l0[i]]), magic_u8(ly0[l0[j]])),
                                    mk(magic_u8(ly0[l1[i]]), magic_u8(ly0[l1[j]])),
                                    mk(magic_u8(ly1[l0[i]]), magic_u8(ly1[l0[j]])),
                                    mk(magic_u8(ly1[l1[i]]), magic_u8(ly1[l1[j]])), wxp, wy);
                constexpr uint32_t kU = 0x7540u, kV = 0x7541u;
                const f2 c128 = splat(128.0f);
                f2 U, V;
                if (csh[p]) {
                    // both pixels tap the same chroma columns (native size,
                    // upscaling, downscaling under 2x): one load per tap
                    const uint32_t a00 = *reinterpret_cast<const uint16_t*>(cr0 + u0[i]);
                    const uint32_t a01 = *reinterpret_cast<const uint16_t*>(cr0 + u1[i]);
                    const uint32_t a10 = *reinterpret_cast<const uint16_t*>(cr1 + u0[i]);
                    const uint32_t a11 = *reinterpret_cast<const uint16_t*>(cr1 + u1[i]);
                    U = sub(bilerp(prod, splat(magic_byte(a00, kU)), splat(magic_byte(a01, kU)),
                                   splat(magic_byte(a10, kU)), splat(magic_byte(a11, kU)), cwxp, cwy),
                            c128);
                    V = sub(bilerp(prod, splat(magic_byte(a00, kV)), splat(magic_byte(a01, kV)),
                                   splat(magic_byte(a10, kV)), splat(magic_byte(a11, kV)), cwxp, cwy),
                            c128);
                } else {
                    const uint32_t a00 = *reinterpret_cast<const uint16_t*>(cr0 + u0[i]);
                    const uint32_t b00 = *reinterpret_cast<const uint16_t*>(cr0 + u0[j]);
                    const uint32_t a01 = *reinterpret_cast<const uint16_t*>(cr0 + u1[i]);
                    const uint32_t b01 = *reinterpret_cast<const uint16_t*>(cr0 + u1[j]);
                    const uint32_t a10 = *reinterpret_cast<const uint16_t*>(cr1 + u0[i]);
                    const uint32_t b10 = *reinterpret_cast<const uint16_t*>(cr1 + u0[j]);
                    const uint32_t a11 = *reinterpret_cast<const uint16_t*>(cr1 + u1[i]);
                    const uint32_t b11 = *reinterpret_cast<const uint16_t*>(cr1 + u1[j]);
                    U = sub(bilerp(prod, mk(magic_byte(a00, kU), magic_byte(b00, kU)),
                                   mk(magic_byte(a01, kU), magic_byte(b01, kU)),
                                   mk(magic_byte(a10, kU), magic_byte(b10, kU)),
                                   mk(magic_byte(a11, kU), magic_byte(b11, kU)), cwxp, cwy),
                            c128);
                    V = sub(bilerp(prod, mk(magic_byte(a00, kV), magic_byte(b00, kV)),
                                   mk(magic_byte(a01, kV), magic_byte(b01, kV)),
                                   mk(magic_byte(a10, kV), magic_byte(b10, kV)),
                                   mk(magic_byte(a11, kV), magic_byte(b11, kV)), cwxp, cwy),
                            c128);
                }
                f2 R, G, B;
                to_rgb<CS>(prod, Y, U, V, R, G, B);
                out[0][p] = normalize(R, a.mean[0], a.std[0], m.rcp_std[0]);
                out[1][p] = normalize(G, a.mean[1], a.std[1], m.rcp_std[1]);
                out[2][p] = normalize(B, a.mean[2], a.std[2], m.rcp_std[2]);
            }
            store4<BF16>(a, rs.base + col, plane, out);
        }
        // the warp is done with stage S
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&empty[S]);
        return true;
    };
    static_assert(kStages == 4, "the row loop below is unrolled over four stages");
    for (uint32_t k = 0;; k += kStages) {
        if (!step(k, std::integral_constant<uint32_t, 0>{})) break;
        if (!step(k + 1, std::integral_constant<uint32_t, 1>{})) break;
        if (!step(k + 2, std::integral_constant<uint32_t, 2>{})) break;
        if (!step(k + 3, std::integral_constant<uint32_t, 3>{})) break;
    }
}

// Launches a staged kernel with one consumer thread per 4 output columns
// plus the producer warp, as many blocks as fit on the device at once (or
// one per output row when there are fewer rows).
template <auto Kern>
cudaError_t launch_grid(uint32_t smem, const MediaArgs& a, const StagedMedia& m, cudaStream_t stream) {
    const uint32_t threads = ((a.out_w / 4u + 31u) / 32u) * 32u + 32u;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    // per device: the shared-memory opt-in, the SM count and the resident
    // blocks per SM of the last block size; guarded, since contexts on other
    // threads may launch at the same time
    static std::mutex mu;
    static int configured[64] = {}, per_sm[64] = {}, sms[64] = {};
    static uint32_t per_sm_threads[64] = {};
    int blocks_per_sm = 1, sm_count = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!configured[dev]) {
            e = cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
            if (e != cudaSuccess) return e;
            e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
            if (e != cudaSuccess) return e;
            configured[dev] = 1;
        }
        if (per_sm_threads[dev] != threads) {
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm[dev], Kern, static_cast<int>(threads), smem);
            if (e != cudaSuccess) return e;
            per_sm_threads[dev] = threads;
        }
        blocks_per_sm = per_sm[dev] > 0 ? per_sm[dev] : 1;
        sm_count = sms[dev];
    }
    const uint64_t rows = static_cast<uint64_t>(a.batch) * a.out_h;
    const uint64_t resident = static_cast<uint64_t>(blocks_per_sm) * sm_count;
    const uint32_t grid = static_cast<uint32_t>(rows < resident ? rows : resident);
    Kern<<<grid, threads, smem, stream>>>(a, m);
    return cudaGetLastError();
}

template <uint32_t CS, bool BF16, uint32_t ROWCAP>
cudaError_t launch_one(const MediaArgs& a, const StagedMedia& m, cudaStream_t stream) {
    const uint32_t smem = kStages * (4u * ROWCAP + sizeof(RowSlot) + 2u * sizeof(uint64_t));
    return launch_grid<nv12_staged_kernel<CS, BF16, ROWCAP>>(smem, a, m, stream);
}

template <uint32_t CS>
cudaError_t launch_cs(const MediaArgs& a, const StagedMedia& m, cudaStream_t stream) {
    const bool small = a.in_w <= 2048u;
    if (a.bf16) return small ? launch_one<CS, true, 2048>(a, m, stream) : launch_one<CS, true, 4096>(a, m, stream);
    return small ? launch_one<CS, false, 2048>(a, m, stream) : launch_one<CS, false, 4096>(a, m, stream);
}

// ------------------------------------------------------------------------
// Packed RGB / BGR / RGBA / BGRA frames, row-staged the same way
// (swm_packed_u8_to_nchw_f32, src/media/mod.rs:1113-1194): the producer
// bulk-copies the two source rows each output row taps; each consumer
// thread keeps its four columns' byte offsets and weights in registers and
// makes all three channels of its pixels.  The source coordinates are
// clamped below at 0 only, as the reference does (the upper neighbour is
// clamped to the last row / column, where the weight no longer matters:
// both taps are the same byte).
template <uint32_t C, bool SWAP, bool BF16, uint32_t ROWCAP>
__global__ void __launch_bounds__(kMaxThreads, 2) packed_staged_kernel(MediaArgs a, StagedMedia m) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr uint32_t kStageBytes = 2u * ROWCAP;  // source rows y0, y1
    RowSlot* slots = reinterpret_cast<RowSlot*>(smem + kStages * kStageBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(slots + kStages);
    uint64_t* empty = full + kStages;
    const uint32_t tid = threadIdx.x, in_w = a.in_w, rows = a.batch * a.out_h, row_bytes = a.in_w * C;
    const uint32_t consumers = blockDim.x - 32u;
    if (tid == 0) {
        for (uint32_t s = 0; s < kStages; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], consumers / 32u);
        }
        tc::mbar_fence_init();
    }
    __syncthreads();

    if (tid >= consumers) {
        if (tid != consumers) return;
        // producer
        uint32_t k = 0;
        for (;; ++k) {
            const uint32_t r = blockIdx.x + k * gridDim.x;
            if (r >= rows) break;
            const uint32_t s = k % kStages;
            if (k >= kStages && !wait_stage(&empty[s], (k / kStages - 1u) & 1u, m.wait_polls)) {
                m.err[1] = static_cast<int>(blockIdx.x);
                m.err[2] = static_cast<int>(k);
                m.err[3] = 2;
                m.err[0] = 1;
                break;
            }
            const uint32_t b = r / a.out_h, y = r - b * a.out_h;
            float f;
            const float sy = fmaxf((static_cast<float>(y) + 0.5f) * m.ratio_h - 0.5f, 0.0f);
            const uint32_t y0 = floor_u(sy, f), y1 = y0 + 1u < a.in_h ? y0 + 1u : y0;
            slots[s].wy = sy - f;
            slots[s].base = out_row_base(a, b, y);
            uint8_t* st = smem + s * kStageBytes;
            const size_t frame = static_cast<size_t>(b) * a.in_h;
            if (r == m.skip_row) continue;  // fault injection: this stage never fills
            tc::mbar_expect_tx(&full[s], 2u * row_bytes);
            tc::bulk_g2s(st, a.a + (frame + y0) * row_bytes, row_bytes, &full[s]);
            tc::bulk_g2s(st + ROWCAP, a.a + (frame + y1) * row_bytes, row_bytes, &full[s]);
        }
        for (uint32_t j = k > kStages ? k - kStages : 0u; j < k; ++j)
            wait_stage(&full[j % kStages], (j / kStages) & 1u, m.wait_polls);
        return;
    }

    // consumers: byte offsets of the two source columns of each of this
    // thread's four output columns, and their weights
    const uint32_t x4 = tid * 4u, lane = tid & 31u;
    const bool active = x4 < a.out_w;
    uint32_t o0[4], o1[4];
    float wx[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t x = active ? x4 + i : 0u;
        float f;
        const float sx = fmaxf((static_cast<float>(x) + 0.5f) * m.ratio_w - 0.5f, 0.0f);
        const uint32_t x0 = floor_u(sx, f);
        o0[i] = C * x0;
        o1[i] = C * (x0 + 1u < in_w ? x0 + 1u : x0);
        wx[i] = sx - f;
    }
    const Prod prod{splat(m.neg_zero)};
    const f2 wxa = mk(wx[0], wx[1]), wxb = mk(wx[2], wx[3]);
    const size_t plane = out_plane(a), col = out_col(a, active ? x4 : 0u);

    auto step = [&](uint32_t k, auto stage) -> bool {
        constexpr uint32_t S = decltype(stage)::value;
        if (blockIdx.x + k * gridDim.x >= rows) return false;
        if (!wait_stage(&full[S], (k / kStages) & 1u, m.wait_polls)) {
            if (lane == 0) {
                m.err[1] = static_cast<int>(blockIdx.x);
                m.err[2] = static_cast<int>(k);
                m.err[3] = 1;
                m.err[0] = 1;
            }
            return false;
        }
        if (active) {
            const RowSlot rs = slots[S];
            const uint8_t* r0 = smem + S * kStageBytes;
            const uint8_t* r1 = r0 + ROWCAP;
            const f2 wy = splat(rs.wy);
            f2 out[3][2];
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                const int i = 2 * p, j = 2 * p + 1;
                const f2 wxp = p ? wxb : wxa;
                f2 t00[3], t01[3], t10[3], t11[3];
                if constexpr (C == 4) {
                    // one 32-bit load per tap, the channels picked by byte permutes
                    const uint32_t w00i = *reinterpret_cast<const uint32_t*>(r0 + o0[i]);
                    const uint32_t w00j = *reinterpret_cast<const uint32_t*>(r0 + o0[j]);
                    const uint32_t w01i = *reinterpret_cast<const uint32_t*>(r0 + o1[i]);
                    const uint32_t w01j = *reinterpret_cast<const uint32_t*>(r0 + o1[j]);
                    const uint32_t w10i = *reinterpret_cast<const uint32_t*>(r1 + o0[i]);
                    const uint32_t w10j = *reinterpret_cast<const uint32_t*>(r1 + o0[j]);
                    const uint32_t w11i = *reinterpret_cast<const uint32_t*>(r1 + o1[i]);
                    const uint32_t w11j = *reinterpret_cast<const uint32_t*>(r1 + o1[j]);
#pragma unroll
                    for (uint32_t c = 0; c < 3; ++c) {
                        const uint32_t sel = 0x7540u | (SWAP ? 2u - c : c);
                        t00[c] = mk(magic_byte(w00i, sel), magic_byte(w00j, sel));
                        t01[c] = mk(magic_byte(w01i, sel), magic_byte(w01j, sel));
                        t10[c] = mk(magic_byte(w10i, sel), magic_byte(w10j, sel));
                        t11[c] = mk(magic_byte(w11i, sel), magic_byte(w11j, sel));
                    }
                } else {
#pragma unroll
                    for (uint32_t c = 0; c < 3; ++c) {
                        const uint32_t sc = SWAP ? 2u - c : c;
                        t00[c] = mk(magic_u8(r0[o0[i] + sc]), magic_u8(r0[o0[j] + sc]));
                        t01[c] = mk(magic_u8(r0[o1[i] + sc]), magic_u8(r0[o1[j] + sc]));
                        t10[c] = mk(magic_u8(r1[o0[i] + sc]), magic_u8(r1[o0[j] + sc]));
                        t11[c] = mk(magic_u8(r1[o1[i] + sc]), magic_u8(r1[o1[j] + sc]));
                    }
                }
#pragma unroll
                for (int c = 0; c < 3; ++c) {
                    const f2 v = prod(bilerp(prod, t00[c], t01[c], t10[c], t11[c], wxp, wy), 0.00392156862745098f);
                    out[c][p] = divide(sub(v, splat(a.mean[c])), a.std[c], m.rcp_std[c]);
                }
            }
            store4<BF16>(a, rs.base + col, plane, out);
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&empty[S]);
        return true;
    };
    static_assert(kStages == 4, "the row loop below is unrolled over four stages");
    for (uint32_t k = 0;; k += kStages) {
        if (!step(k, std::integral_constant<uint32_t, 0>{})) break;
        if (!step(k + 1, std::integral_constant<uint32_t, 1>{})) break;
        if (!step(k + 2, std::integral_constant<uint32_t, 2>{})) break;
        if (!step(k + 3, std::integral_constant<uint32_t, 3>{})) break;
    }
}

template <uint32_t C, bool SWAP, bool BF16>
cudaError_t launch_packed_rc(const MediaArgs& a, const StagedMedia& m, cudaStream_t stream) {
    if (a.in_w * C <= 4096u) {
        constexpr uint32_t R = 4096;
        return launch_grid<packed_staged_kernel<C, SWAP, BF16, R>>(
            kStages * (2u * R + sizeof(RowSlot) + 2u * sizeof(uint64_t)), a, m, stream);
    }
    constexpr uint32_t R = 8192;
    return launch_grid<packed_staged_kernel<C, SWAP, BF16, R>>(
        kStages * (2u * R + sizeof(RowSlot) + 2u * sizeof(uint64_t)), a, m, stream);
}

template <uint32_t C, bool SWAP>
cudaError_t launch_packed(const MediaArgs& a, const StagedMedia& m, cudaStream_t stream) {
    return a.bf16 ? launch_packed_rc<C, SWAP, true>(a, m, stream) : launch_packed_rc<C, SWAP, false>(a, m, stream);
}

}  // namespace staged

namespace {
bool aligned(const void* p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

// What both staged kernels need of the output and the normalisation.
bool staged_common_ok(const MediaArgs& a) {
    if (a.out_w % 4u != 0 || a.out_w > 4u * staged::kMaxConsumers || a.out_h == 0) return false;
    if (a.patch % 4u != 0) return false;  // four-column stores stay inside one patch row
    if (!aligned(a.out, a.bf16 ? 8 : 16)) return false;
    if (static_cast<uint64_t>(a.batch) * a.out_h >= (1ull << 31) ||
        static_cast<uint64_t>(a.batch) * a.in_h >= (1ull << 31))
        return false;
    for (int c = 0; c < 3; ++c) {
        // The corrected quotient is exact while the quotient and the
        // remainder stay normal: with values in [0, 1], std in [2^-40, 2^40]
        // and mean 0 or of magnitude in [2^-40, 2^40] they do.
        const float s = a.std[c], mu = std::fabs(a.mean[c]);
        if (!(s >= 0x1p-40f && s <= 0x1p40f)) return false;
        if (!(mu == 0.0f || (mu >= 0x1p-40f && mu <= 0x1p40f))) return false;
    }
    return true;
}

StagedMedia staged_params(const MediaArgs& a, int* err) {
    StagedMedia m{};
    m.ratio_h = static_cast<float>(a.in_h) / static_cast<float>(a.out_h);
    m.ratio_w = static_cast<float>(a.in_w) / static_cast<float>(a.out_w);
    for (int c = 0; c < 3; ++c) m.rcp_std[c] = 1.0f / a.std[c];
    m.err = err;
    m.neg_zero = -0.0f;
    m.skip_row = a.test_skip_row_plus1 ? a.test_skip_row_plus1 - 1u : ~0u;
    m.wait_polls = a.test_wait_polls ? a.test_wait_polls : staged::kWaitLimit;
    return m;
}
}  // namespace

bool nv12_staged_eligible(const MediaArgs& a) {
    if (a.in_w % 16u != 0 || a.in_w > 4096u || a.in_h < 2u) return false;
    if (!aligned(a.a, 16) || !aligned(a.uv, 16)) return false;
    return staged_common_ok(a);
}

bool packed_staged_eligible(const MediaArgs& a) {
    const uint64_t row_bytes = static_cast<uint64_t>(a.in_w) * a.channels;
    if (a.format > 3u || (a.channels != 3u && a.channels != 4u)) return false;
    if (row_bytes % 16u != 0 || row_bytes > 8192u || a.in_h == 0 || !aligned(a.a, 16)) return false;
    return staged_common_ok(a);
}

cudaError_t launch_packed_staged(const MediaArgs& a, int* err, cudaStream_t stream) {
    const StagedMedia m = staged_params(a, err);
    switch (a.format) {
        case 0: return staged::launch_packed<3, false>(a, m, stream);
        case 1: return staged::launch_packed<3, true>(a, m, stream);
        case 2: return staged::launch_packed<4, false>(a, m, stream);
        default: return staged::launch_packed<4, true>(a, m, stream);
    }
}

cudaError_t launch_nv12_staged(const MediaArgs& a, int* err, cudaStream_t stream) {
    const StagedMedia m = staged_params(a, err);
    switch (a.format) {
        case 0: return staged::launch_cs<0>(a, m, stream);
        case 1: return staged::launch_cs<1>(a, m, stream);
        case 2: return staged::launch_cs<2>(a, m, stream);
        default: return staged::launch_cs<3>(a, m, stream);
    }
}

cudaError_t launch_media(const MediaArgs& a, bool nv12, cudaStream_t stream) {
    const uint64_t pixels = static_cast<uint64_t>(a.batch) * a.out_h * a.out_w;
    const uint32_t blocks = static_cast<uint32_t>((pixels + 255) / 256);
    if (nv12) nv12_pixel_kernel<<<blocks, 256, 0, stream>>>(a);
    else packed_pixel_kernel<<<blocks, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace lwm
