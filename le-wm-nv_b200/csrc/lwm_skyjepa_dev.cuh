// lwm_skyjepa_dev.cuh — device code shared by the f32 SkyJEPA rollout
// kernels: one explicit-Euler step of the learned integrator from the prober
// outputs, with that step's tracking cost.  Include it from translation units
// built with -fmad=false, so every product and sum rounds on its own as in the
// reference's f32 kernels.
#pragma once

#include <cstdint>

#include "lwm_kernels.hpp"

namespace lwm {

// One step of lewm_skyjepa_integrate_f32 (kinematics.rs:377-484) from the
// prober outputs po[15] and the candidate's action, and the tracking cost
// (control.rs:430-452) of that step, returned.  x[18] is updated in place;
// the state is written to a.states (row s of vehicle b, step t) when asked
// and `store` is set.
__device__ __forceinline__ float integrate_and_cost(const SkyjepaArgs& a, uint32_t b, uint32_t s, uint32_t t,
                                                    float (&x)[18], const float* act, const float* po,
                                                    bool store = true) {
    const uint32_t T = a.T;
    const float sdt = a.dt;
    float ta;
    if (a.rotor_forces) {
        ta = (act[0] + act[1] + act[2] + act[3]) / (a.masses ? __ldg(a.masses + b) : a.mass);
    } else {
        const float th = fminf(1.0f, fmaxf(0.0f, act[2]));
        ta = th * a.gravity / a.hover_throttle;
    }
    const float acc[3] = {x[8] * ta + po[0], x[11] * ta + po[1], x[14] * ta - a.gravity + po[2]};
    float ang[3];
#pragma unroll
    for (int row = 0; row < 3; ++row)
        ang[row] = po[3 + row * 4] * act[0] + po[4 + row * 4] * act[1] + po[5 + row * 4] * act[2] +
                   po[6 + row * 4] * act[3];
#pragma unroll
    for (int ax = 0; ax < 3; ++ax) { x[ax] += x[3 + ax] * sdt; x[3 + ax] += acc[ax] * sdt; }
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
    const float dl[9] = {1.0f - cb * (wy * wy + wz * wz), cb * wx * wy - ca * wz, cb * wx * wz + ca * wy,
                         cb * wy * wx + ca * wz, 1.0f - cb * (wx * wx + wz * wz), cb * wy * wz - ca * wx,
                         cb * wz * wx - ca * wy, cb * wz * wy + ca * wx, 1.0f - cb * (wx * wx + wy * wy)};
    float nr[9];
#pragma unroll
    for (int row = 0; row < 3; ++row)
#pragma unroll
        for (int col = 0; col < 3; ++col)
            nr[row * 3 + col] = x[6 + row * 3] * dl[col] + x[7 + row * 3] * dl[3 + col] + x[8 + row * 3] * dl[6 + col];
#pragma unroll
    for (int i = 0; i < 9; ++i) x[6 + i] = nr[i];
#pragma unroll
    for (int ax = 0; ax < 3; ++ax) x[15 + ax] += ang[ax] * sdt;
    if (store && a.states && s < a.S) {
        float* o = a.states + ((static_cast<size_t>(b) * a.S + s) * T + t) * 18;
#pragma unroll
        for (int i = 0; i < 18; ++i) o[i] = x[i];
    }
    const float* ref = a.ref_states + (static_cast<size_t>(b) * T + t) * 18;
    float g0 = 0.0f, g1 = 0.0f, g2 = 0.0f, g3 = 0.0f;
#pragma unroll
    for (int i = 0; i < 3; ++i) { const float dd = x[i] - ref[i]; g0 += dd * dd; }
#pragma unroll
    for (int i = 3; i < 6; ++i) { const float dd = x[i] - ref[i]; g1 += dd * dd; }
#pragma unroll
    for (int i = 6; i < 15; ++i) { const float dd = x[i] - ref[i]; g2 += dd * dd; }
#pragma unroll
    for (int i = 15; i < 18; ++i) { const float dd = x[i] - ref[i]; g3 += dd * dd; }
    const float* ra = a.ref_actions + (static_cast<size_t>(b) * T + t) * 4;
    float ac = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) { const float dd = act[i] - ra[i]; ac += (dd * dd) * a.cost.action[i]; }
    float st = g0 * a.cost.position + g1 * a.cost.velocity;
    st = st + g2 * a.cost.attitude;
    st = st + g3 * a.cost.angular_velocity;
    return st + ac;
}

}  // namespace lwm
