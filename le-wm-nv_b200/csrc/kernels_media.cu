// kernels_media.cu — image preprocessing for the ViT encoder: packed
// RGB/BGR(A) or NV12 u8 frames -> bilinear resize (half-pixel centres) ->
// [0,1] -> (x - mean) / std -> NCHW (or one slot of an [B, history, 3, H, W]
// buffer), f32 or bf16.
//
// Reference kernels: swm_packed_u8_to_nchw_f32 and swm_nv12_to_nchw_f32
// (src/media/mod.rs:1113-1194, 1196-1333).  Here one thread produces all
// three channels of an output pixel (the reference's packed kernel runs one
// thread per output element and repeats the coordinate math and the four
// taps per channel), so every source byte is read once per pixel.  Compiled
// with -fmad=false: every product and sum is rounded on its own.
#include <cuda_bf16.h>

#include <cstdint>

#include "lwm_kernels.hpp"

namespace lwm {


__device__ __forceinline__ float clampf(float v, float lo, float hi) { return fminf(fmaxf(v, lo), hi); }

// Bilinear tap of channel `ch` of an interleaved plane; coordinates clamped
// to the plane (swm_sample_plane, src/media/mod.rs:1201-1230).
__device__ __forceinline__ float sample_plane(const uint8_t* plane, uint32_t b, uint32_t h, uint32_t w, uint32_t channels,
                                              uint32_t ch, float sy, float sx) {
    sy = clampf(sy, 0.0f, static_cast<float>(h - 1u));
    sx = clampf(sx, 0.0f, static_cast<float>(w - 1u));
    const uint32_t y0 = static_cast<uint32_t>(floorf(sy)), x0 = static_cast<uint32_t>(floorf(sx));
    const uint32_t y1 = y0 + 1u < h ? y0 + 1u : y0, x1 = x0 + 1u < w ? x0 + 1u : x0;
    const float wy = sy - static_cast<float>(y0), wx = sx - static_cast<float>(x0);
    const size_t row0 = (static_cast<size_t>(b) * h + y0) * w, row1 = (static_cast<size_t>(b) * h + y1) * w;
    const float v00 = __ldg(plane + (row0 + x0) * channels + ch), v01 = __ldg(plane + (row0 + x1) * channels + ch);
    const float v10 = __ldg(plane + (row1 + x0) * channels + ch), v11 = __ldg(plane + (row1 + x1) * channels + ch);
    const float top = v00 + (v01 - v00) * wx;
    const float bottom = v10 + (v11 - v10) * wx;
    return top + (bottom - top) * wy;
}

__device__ __forceinline__ void store3(const MediaArgs& a, uint32_t b, uint32_t y, uint32_t x, const float (&v)[3]) {
    for (uint32_t c = 0; c < 3; ++c) {
        const float normalized = (v[c] - a.mean[c]) / a.std[c];
        size_t idx;
        if (a.history_len == 0)
            idx = ((static_cast<size_t>(b) * 3 + c) * a.out_h + y) * a.out_w + x;
        else
            idx = (((static_cast<size_t>(b) * a.history_len + a.history_slot) * 3 + c) * a.out_h + y) * a.out_w + x;
        if (a.bf16) static_cast<__nv_bfloat16*>(a.out)[idx] = __float2bfloat16_rn(normalized);
        else static_cast<float*>(a.out)[idx] = normalized;
    }
}

__global__ void __launch_bounds__(256) packed_to_nchw_kernel(MediaArgs a) {
    const uint64_t idx = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint64_t pixels = static_cast<uint64_t>(a.batch) * a.out_h * a.out_w;
    if (idx >= pixels) return;
    const uint32_t x = static_cast<uint32_t>(idx % a.out_w);
    const uint64_t tmp = idx / a.out_w;
    const uint32_t y = static_cast<uint32_t>(tmp % a.out_h), b = static_cast<uint32_t>(tmp / a.out_h);
    // swm_packed_u8_to_nchw_f32: half-pixel source coordinate, clamped below at 0
    float sy = (static_cast<float>(y) + 0.5f) * (static_cast<float>(a.in_h) / static_cast<float>(a.out_h)) - 0.5f;
    float sx = (static_cast<float>(x) + 0.5f) * (static_cast<float>(a.in_w) / static_cast<float>(a.out_w)) - 0.5f;
    if (sy < 0.0f) sy = 0.0f;
    if (sx < 0.0f) sx = 0.0f;
    const bool swap = a.format == 1u || a.format == 3u;
    float v[3];
    for (uint32_t c = 0; c < 3; ++c)
        v[c] = sample_plane(a.a, b, a.in_h, a.in_w, a.channels, swap ? 2u - c : c, sy, sx) * 0.00392156862745098f;
    store3(a, b, y, x, v);
}

__global__ void __launch_bounds__(256) nv12_to_nchw_kernel(MediaArgs a) {
    const uint64_t idx = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint64_t pixels = static_cast<uint64_t>(a.batch) * a.out_h * a.out_w;
    if (idx >= pixels) return;
    const uint32_t x = static_cast<uint32_t>(idx % a.out_w);
    const uint64_t tmp = idx / a.out_w;
    const uint32_t y = static_cast<uint32_t>(tmp % a.out_h), b = static_cast<uint32_t>(tmp / a.out_h);
    const float sy = (static_cast<float>(y) + 0.5f) * (static_cast<float>(a.in_h) / static_cast<float>(a.out_h)) - 0.5f;
    const float sx = (static_cast<float>(x) + 0.5f) * (static_cast<float>(a.in_w) / static_cast<float>(a.out_w)) - 0.5f;
    const float yv = sample_plane(a.a, b, a.in_h, a.in_w, 1u, 0u, sy, sx);
    const float u = sample_plane(a.uv, b, a.in_h / 2u, a.in_w / 2u, 2u, 0u, sy * 0.5f, sx * 0.5f) - 128.0f;
    const float vv = sample_plane(a.uv, b, a.in_h / 2u, a.in_w / 2u, 2u, 1u, sy * 0.5f, sx * 0.5f) - 128.0f;
    float r, g, bl;
    // colour matrices of src/media/mod.rs:1298-1318
    if (a.format == 0u) {
        const float yy = fmaxf(yv - 16.0f, 0.0f) * 1.16438356f;
        r = yy + 1.59602678f * vv;
        g = yy - 0.39176229f * u - 0.81296765f * vv;
        bl = yy + 2.01723214f * u;
    } else if (a.format == 1u) {
        const float yy = fmaxf(yv - 16.0f, 0.0f) * 1.16438356f;
        r = yy + 1.79274107f * vv;
        g = yy - 0.21324861f * u - 0.53290933f * vv;
        bl = yy + 2.11240179f * u;
    } else if (a.format == 2u) {
        r = yv + 1.402f * vv;
        g = yv - 0.344136f * u - 0.714136f * vv;
        bl = yv + 1.772f * u;
    } else {
        r = yv + 1.5748f * vv;
        g = yv - 0.187324f * u - 0.468124f * vv;
        bl = yv + 1.8556f * u;
    }
    const float v[3] = {clampf(r, 0.0f, 255.0f) * 0.00392156862745098f, clampf(g, 0.0f, 255.0f) * 0.00392156862745098f,
                        clampf(bl, 0.0f, 255.0f) * 0.00392156862745098f};
    store3(a, b, y, x, v);
}

cudaError_t launch_media(const MediaArgs& a, bool nv12, cudaStream_t stream) {
    const uint64_t pixels = static_cast<uint64_t>(a.batch) * a.out_h * a.out_w;
    const uint32_t blocks = static_cast<uint32_t>((pixels + 255) / 256);
    if (nv12) nv12_to_nchw_kernel<<<blocks, 256, 0, stream>>>(a);
    else packed_to_nchw_kernel<<<blocks, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace lwm
