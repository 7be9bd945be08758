// lwm_lewm_epi.cuh — the fused GEMM epilogue of the LeWM scorer (bias,
// activation, gated residual), shared by the f32 and the tensor-core GEMMs.
#pragma once

#include <cuda_runtime.h>

#include "lwm_device.cuh"
#include "lwm_lewm.hpp"

namespace lwm {

__device__ __forceinline__ float apply_act(int act, float v) {
    switch (act) {
        case kActGeluTanh: return gelu_tanh(v);
        case kActGeluErf: return (0.5f * v) * (1.0f + erff(v * 0.7071067811865476f));
        case kActSilu: return v / (1.0f + expf(-v));
        default: return v;
    }
}

__device__ __forceinline__ float epilogue_value(const GemmArgs& g, uint32_t m, uint32_t n, float v, float* c) {
    if (g.bias) v = v + g.bias[n];
    if (g.residual) {
        // x = x + gate * y (ConditionalBlock) or x = y + x (ViT layer)
        if (g.gate) v = g.gate[g.map.row(m) * g.ldg + n] * v;
        return *c + v;
    }
    return apply_act(g.act, v);
}

}  // namespace lwm
