// lwm_skyjepa_tcn.cuh — the action encoder of one candidate window in
// registers (TemporalConvEncoder::forward_last over [history ++ candidate]
// (t : t + 10), src/models/skyjepa/tcn.rs:88-96, 138-160; model.rs:192-215),
// for the 4-channel, 3-level, kernel-3 encoder the tensor-core rollouts take.
// Gelu is the activation functor: the reference's tanh-form GELU at f32
// accuracy, or a faster approximation where the tolerance allows it.
#pragma once

#include <cstdint>

namespace lwm {

// Action-TCN input of step t for one candidate (TemporalConvEncoder over the
// window [history ++ candidate](t : t + 10), last position), written as bf16
// into the X tile.  One thread per candidate, in registers.
//
// Only the last output position of the window is used, so each block is
// evaluated where that output depends on it (kernel 3, dilations 1, 2, 4,
// causal zero padding inside the window):
//   block 1: conv1 at all 10 positions, output at odd positions 1..9
//   block 2: conv1 at odd positions, output at 1, 5, 9
//   block 3: conv1 at 1, 5, 9, output at 9
// (27 position-convolutions instead of 60; the values computed are the
// reference's, tcn.rs:88-96 / 138-160).
constexpr int kTcnHs = 10, kTcnK = 3, kTcnC = 4;

// The 4 channels at window position P of conv(in) with dilation DIL (+ bias, GELU).
template <int P, int DIL, typename Gelu>
__device__ __forceinline__ void conv_at(const float (&in)[kTcnC][kTcnHs], const float* W, const float* B,
                                        float (&out)[kTcnC][kTcnHs]) {
#pragma unroll
    for (int o = 0; o < kTcnC; ++o) {
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < kTcnC; ++i)
#pragma unroll
            for (int j = 0; j < kTcnK; ++j) {
                const int src = P - (kTcnK - 1 - j) * DIL;
                if (src >= 0) acc = fmaf(W[(o * kTcnC + i) * kTcnK + j], in[i][src], acc);
            }
        out[o][P] = Gelu()(acc + B[o]);
    }
}

// out[P] = gelu(gelu(conv2(h)[P]) + res[P])
template <int P, int DIL, typename Gelu>
__device__ __forceinline__ void block_out_at(const float (&h)[kTcnC][kTcnHs], const float (&res)[kTcnC][kTcnHs],
                                             const float* W2, const float* B2, float (&out)[kTcnC][kTcnHs]) {
    float c2[kTcnC][kTcnHs];
    conv_at<P, DIL, Gelu>(h, W2, B2, c2);
#pragma unroll
    for (int o = 0; o < kTcnC; ++o) out[o][P] = Gelu()(c2[o][P] + res[o][P]);
}

struct TcnBlockW {
    const float *w1, *b1, *w2, *b2;
};

// x_t of one candidate: `win` holds the normalised window (4 channels x 10).
template <typename Gelu>
__device__ __forceinline__ void tcn_last(const TcnBlockW (&w)[3], const float (&x0)[kTcnC][kTcnHs], float (&x)[kTcnC]) {
    // block 1 (dilation 1)
    float h[kTcnC][kTcnHs], y1[kTcnC][kTcnHs];
    conv_at<0, 1, Gelu>(x0, w[0].w1, w[0].b1, h);
    conv_at<1, 1, Gelu>(x0, w[0].w1, w[0].b1, h);
    conv_at<2, 1, Gelu>(x0, w[0].w1, w[0].b1, h);
    conv_at<3, 1, Gelu>(x0, w[0].w1, w[0].b1, h);
    conv_at<4, 1, Gelu>(x0, w[0].w1, w[0].b1, h);
    conv_at<5, 1, Gelu>(x0, w[0].w1, w[0].b1, h);
    conv_at<6, 1, Gelu>(x0, w[0].w1, w[0].b1, h);
    conv_at<7, 1, Gelu>(x0, w[0].w1, w[0].b1, h);
    conv_at<8, 1, Gelu>(x0, w[0].w1, w[0].b1, h);
    conv_at<9, 1, Gelu>(x0, w[0].w1, w[0].b1, h);
    block_out_at<1, 1, Gelu>(h, x0, w[0].w2, w[0].b2, y1);
    block_out_at<3, 1, Gelu>(h, x0, w[0].w2, w[0].b2, y1);
    block_out_at<5, 1, Gelu>(h, x0, w[0].w2, w[0].b2, y1);
    block_out_at<7, 1, Gelu>(h, x0, w[0].w2, w[0].b2, y1);
    block_out_at<9, 1, Gelu>(h, x0, w[0].w2, w[0].b2, y1);
    // block 2 (dilation 2): reads y1 at odd positions only
    float y2[kTcnC][kTcnHs];
    conv_at<1, 2, Gelu>(y1, w[1].w1, w[1].b1, h);
    conv_at<3, 2, Gelu>(y1, w[1].w1, w[1].b1, h);
    conv_at<5, 2, Gelu>(y1, w[1].w1, w[1].b1, h);
    conv_at<7, 2, Gelu>(y1, w[1].w1, w[1].b1, h);
    conv_at<9, 2, Gelu>(y1, w[1].w1, w[1].b1, h);
    block_out_at<1, 2, Gelu>(h, y1, w[1].w2, w[1].b2, y2);
    block_out_at<5, 2, Gelu>(h, y1, w[1].w2, w[1].b2, y2);
    block_out_at<9, 2, Gelu>(h, y1, w[1].w2, w[1].b2, y2);
    // block 3 (dilation 4): reads y2 at 1, 5, 9
    float y3[kTcnC][kTcnHs];
    conv_at<1, 4, Gelu>(y2, w[2].w1, w[2].b1, h);
    conv_at<5, 4, Gelu>(y2, w[2].w1, w[2].b1, h);
    conv_at<9, 4, Gelu>(y2, w[2].w1, w[2].b1, h);
    block_out_at<9, 4, Gelu>(h, y2, w[2].w2, w[2].b2, y3);
#pragma unroll
    for (int o = 0; o < kTcnC; ++o) x[o] = y3[o][kTcnHs - 1];
}

// The same encoder split over the 4 lanes of a window (lane `o` computes
// output channel o of every convolution; the lanes of one window are
// consecutive, starting at lane `base` of the warp).  Each convolution's
// outputs are gathered back to all 4 lanes with shuffles.  Every sum is
// formed in the order conv_at forms it, so the values are tcn_last's.
struct TcnChannelW {
    float w[6][kTcnC * kTcnK];  // convolution 2l + k (level l; k = 0 conv1, 1 conv2): row o
    float b[6];
};

// Output channel o at position P of conv(in) with dilation `dil`, + bias, GELU.
template <typename Gelu>
__device__ __forceinline__ float conv_ch(const float (&in)[kTcnC][kTcnHs], const float (&W)[kTcnC * kTcnK],
                                         float B, int P, int dil) {
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < kTcnC; ++i)
#pragma unroll
        for (int j = 0; j < kTcnK; ++j) {
            const int src = P - (kTcnK - 1 - j) * dil;
            if (src >= 0) acc = fmaf(W[i * kTcnK + j], in[i][src], acc);
        }
    return Gelu()(acc + B);
}

__device__ __forceinline__ void gather_ch(float (&dst)[kTcnC][kTcnHs], int P, float mine, uint32_t base) {
#pragma unroll
    for (int i = 0; i < kTcnC; ++i) dst[i][P] = __shfl_sync(0xffffffffu, mine, base + i);
}

// Channel o of x_t; the return value is the lane's own channel.  (Arrays
// are indexed with compile-time positions only, so they stay in registers;
// the lane's own channel of a block output is kept beside it.)
template <typename Gelu>
__device__ __forceinline__ float tcn_last_channel(const TcnChannelW& w, const float (&x0)[kTcnC][kTcnHs], uint32_t o,
                                                  uint32_t base) {
    float h1[kTcnC][kTcnHs], y1[kTcnC][kTcnHs], h2[kTcnC][kTcnHs], y2[kTcnC][kTcnHs], h3[kTcnC][kTcnHs];
    float y1o[kTcnHs], y2o[kTcnHs];
    // block 1 (dilation 1): conv1 everywhere, output at odd positions
#pragma unroll
    for (int P = 0; P < kTcnHs; ++P) gather_ch(h1, P, conv_ch<Gelu>(x0, w.w[0], w.b[0], P, 1), base);
#pragma unroll
    for (int P = 1; P < kTcnHs; P += 2) {
        const float res = o == 0 ? x0[0][P] : o == 1 ? x0[1][P] : o == 2 ? x0[2][P] : x0[3][P];
        y1o[P] = Gelu()(conv_ch<Gelu>(h1, w.w[1], w.b[1], P, 1) + res);
        gather_ch(y1, P, y1o[P], base);
    }
    // block 2 (dilation 2): conv1 at odd positions, output at 1, 5, 9
#pragma unroll
    for (int P = 1; P < kTcnHs; P += 2) gather_ch(h2, P, conv_ch<Gelu>(y1, w.w[2], w.b[2], P, 2), base);
#pragma unroll
    for (int P = 1; P < kTcnHs; P += 4) {
        y2o[P] = Gelu()(conv_ch<Gelu>(h2, w.w[3], w.b[3], P, 2) + y1o[P]);
        gather_ch(y2, P, y2o[P], base);
    }
    // block 3 (dilation 4): conv1 at 1, 5, 9, output at 9
#pragma unroll
    for (int P = 1; P < kTcnHs; P += 4) gather_ch(h3, P, conv_ch<Gelu>(y2, w.w[4], w.b[4], P, 4), base);
    return Gelu()(conv_ch<Gelu>(h3, w.w[5], w.b[5], kTcnHs - 1, 4) + y2o[kTcnHs - 1]);
}

}  // namespace lwm
