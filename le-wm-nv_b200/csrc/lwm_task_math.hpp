// lwm_task_math.hpp — the task side of closed-loop control, written once for
// the host (the controller session, g++) and the device (the fleet loop,
// nvcc): reference trajectories, the geometric action prior and one step of
// the rotor plant.  Both builds keep every operation separately rounded
// (-ffp-contract=off / -fmad=false).
//
// Reference: skyjepa_reference_state (src/skyjepa_task.rs:57-110),
// skyjepa_geometric_action_prior (:118-240), SkyJepaRotorPlant::step
// (src/skyjepa_sim.rs:206-281).
#pragma once

#include <cmath>
#include <cstdint>

#include "../../include/lewm_b200.h"

#ifdef __CUDACC__
#define LWM_HD __host__ __device__ inline
#else
#define LWM_HD inline
#endif

namespace lwm {
namespace task {

LWM_HD float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

LWM_HD void cross3(const float* l, const float* r, float* o) {
    o[0] = l[1] * r[2] - l[2] * r[1];
    o[1] = l[2] * r[0] - l[0] * r[2];
    o[2] = l[0] * r[1] - l[1] * r[0];
}

LWM_HD float dot3(const float* a, const float* b) { return a[0] * b[0] + a[1] * b[1] + a[2] * b[2]; }

LWM_HD void normalize_or(const float* v, const float* fallback, float* out) {
    const float n = sqrtf(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
    if (n > 1e-6f) {
        out[0] = v[0] / n; out[1] = v[1] / n; out[2] = v[2] / n;
    } else {
        out[0] = fallback[0]; out[1] = fallback[1]; out[2] = fallback[2];
    }
}

// Columns (x, y, up) of a rotation whose third column is `up`, x from `heading`.
LWM_HD void frame_from_up(const float* up, const float* heading, float* R) {
    const float fy[3] = {0.0f, 1.0f, 0.0f};
    float c[3], by[3], bx[3];
    cross3(up, heading, c);
    normalize_or(c, fy, by);
    cross3(by, up, c);
    normalize_or(c, heading, bx);
    R[0] = bx[0]; R[1] = by[0]; R[2] = up[0];
    R[3] = bx[1]; R[4] = by[1]; R[5] = up[1];
    R[6] = bx[2]; R[7] = by[2]; R[8] = up[2];
}

// skyjepa_reference_state: kind 0 hover, 1 circle, 2 figure-eight.
LWM_HD void reference_state(int kind, float time, float radius, float period, float* s) {
    for (int i = 0; i < 18; ++i) s[i] = 0.0f;
    s[2] = 1.0f;
    const float omega = 2.0f * static_cast<float>(M_PI) / period;
    const float angle = omega * time;
    float acc[3] = {0.0f, 0.0f, 0.0f};
    if (kind == 1) {
        acc[0] = -radius * omega * omega * cosf(angle);
        acc[1] = -radius * omega * omega * sinf(angle);
        s[0] = radius * (cosf(angle) - 1.0f);
        s[1] = radius * sinf(angle);
        s[3] = -radius * omega * sinf(angle);
        s[4] = radius * omega * cosf(angle);
    } else if (kind == 2) {
        acc[0] = -radius * omega * omega * sinf(angle);
        acc[1] = -2.0f * radius * omega * omega * sinf(2.0f * angle);
        acc[2] = -0.0625f * omega * omega * sinf(0.5f * angle);
        s[0] = radius * sinf(angle);
        s[1] = radius * 0.5f * sinf(2.0f * angle);
        s[2] = 1.2f + 0.25f * sinf(0.5f * angle);
        s[3] = radius * omega * cosf(angle);
        s[4] = radius * omega * cosf(2.0f * angle);
        s[5] = 0.125f * omega * cosf(0.5f * angle);
    }
    const float fz[3] = {0.0f, 0.0f, 1.0f};
    const float a[3] = {acc[0], acc[1], acc[2] + 9.81f};
    float up[3];
    normalize_or(a, fz, up);
    float heading[3] = {1.0f, 0.0f, 0.0f};
    if (!(fabsf(up[0]) < 0.95f)) { heading[0] = 0.0f; heading[1] = 1.0f; }
    frame_from_up(up, heading, s + 6);
}

// Rotor forces of the geometric prior at step `index` of `T` references
// (refs [T][18]) from the current state `cur` [18].
LWM_HD void geometric_prior_step(const float* cur, const float* refs, uint32_t index, uint32_t T, float dt,
                                 const lwm_domain& d, float* out4) {
    const float fz[3] = {0.0f, 0.0f, 1.0f}, fx[3] = {1.0f, 0.0f, 0.0f};
    const float* ref = refs + static_cast<size_t>(index) * 18;
    float accel[3] = {0.0f, 0.0f, 0.0f};
    const float* before = nullptr;
    const float* after = nullptr;
    if (index + 1 < T) { before = ref; after = refs + static_cast<size_t>(index + 1) * 18; }
    else if (index > 0) { before = refs + static_cast<size_t>(index - 1) * 18; after = ref; }
    if (before) for (int a = 0; a < 3; ++a) accel[a] = (after[3 + a] - before[3 + a]) / dt;
    const float fb = index == 0 ? 1.0f : 0.0f;
    float des[3];
    for (int a = 0; a < 3; ++a)
        des[a] = accel[a] + fb * (3.5f * (ref[a] - cur[a]) + 2.6f * (ref[3 + a] - cur[3 + a])) +
                 (a == 2 ? d.gravity : 0.0f);
    float up[3], hd[3];
    const float hraw[3] = {ref[6], ref[9], 0.0f};
    normalize_or(des, fz, up);
    normalize_or(hraw, fx, hd);
    if (fabsf(dot3(up, hd)) > 0.95f) { const float h0 = hd[0]; hd[0] = -hd[1]; hd[1] = h0; hd[2] = 0.0f; }
    float D[9];
    frame_from_up(up, hd, D);
    const float* R = index == 0 ? cur + 6 : ref + 6;
    const float* om = index == 0 ? cur + 15 : ref + 15;
    // attitude_error_body: vee of the skew part of D^T R
    float P[9];
    for (int col = 0; col < 3; ++col) {
        const float v[3] = {R[col], R[3 + col], R[6 + col]};
        P[0 * 3 + col] = D[0] * v[0] + D[3] * v[1] + D[6] * v[2];
        P[1 * 3 + col] = D[1] * v[0] + D[4] * v[1] + D[7] * v[2];
        P[2 * 3 + col] = D[2] * v[0] + D[5] * v[1] + D[8] * v[2];
    }
    const float err[3] = {0.5f * (P[7] - P[5]), 0.5f * (P[2] - P[6]), 0.5f * (P[3] - P[1])};
    float torque[3];
    for (int a = 0; a < 3; ++a) torque[a] = -d.inertia[a] * (25.0f * err[a] + 8.0f * om[a]);
    const float cup[3] = {R[2], R[5], R[8]};
    float proj = dot3(des, cup);
    if (proj < 0.0f) proj = 0.0f;
    const float total = clampf(d.mass * proj / d.thrust_scale, 0.0f, d.mass * d.gravity * d.max_thrust_weight);
    const float arm = d.arm_length * d.thrust_scale;
    const float yaw = 0.025f * d.torque_scale * d.thrust_scale;
    const float base = total / 4.0f;
    const float f[4] = {base - torque[1] / (2.0f * arm) + torque[2] / (4.0f * yaw),
                        base + torque[0] / (2.0f * arm) - torque[2] / (4.0f * yaw),
                        base + torque[1] / (2.0f * arm) + torque[2] / (4.0f * yaw),
                        base - torque[0] / (2.0f * arm) - torque[2] / (4.0f * yaw)};
    const float maximum = d.mass * d.gravity * d.max_thrust_weight / 4.0f;
    for (int r = 0; r < 4; ++r) out4[r] = clampf(f[r], 0.0f, maximum);
}

// One plant step of dt: first-order motors toward the clamped command,
// rigid-body attitude / rate update with gyroscopic and drag terms, ground
// contact at 5 cm.  x [18] and motors [4] in place.
LWM_HD void plant_step(const lwm_domain& d, float* x, float* motors, const float* cmd, float dt) {
    const float max_force = d.mass * d.gravity * d.max_thrust_weight / 4.0f;
    const float response = 1.0f - expf(-dt / d.motor_time_constant);
    for (int r = 0; r < 4; ++r) motors[r] += (clampf(cmd[r], 0.0f, max_force) - motors[r]) * response;
    float f[4];
    for (int r = 0; r < 4; ++r) f[r] = motors[r] * d.thrust_scale;
    const float total = ((f[0] + f[1]) + f[2]) + f[3];
    const float yaw = 0.025f * d.torque_scale;
    const float torque[3] = {d.arm_length * (f[1] - f[3]), d.arm_length * (f[2] - f[0]),
                             yaw * (f[0] - f[1] + f[2] - f[3])};
    float* w = x + 15;
    const float iw[3] = {d.inertia[0] * w[0], d.inertia[1] * w[1], d.inertia[2] * w[2]};
    float gyro[3];
    cross3(w, iw, gyro);
    for (int a = 0; a < 3; ++a) w[a] += ((torque[a] - gyro[a] - 0.015f * w[a]) / d.inertia[a]) * dt;
    const float v3[3] = {w[0] * dt, w[1] * dt, w[2] * dt};
    const float theta = sqrtf(v3[0] * v3[0] + v3[1] * v3[1] + v3[2] * v3[2]);
    float dr[9];
    if (theta < 1e-6f) {
        dr[0] = 1.0f; dr[1] = -v3[2]; dr[2] = v3[1];
        dr[3] = v3[2]; dr[4] = 1.0f; dr[5] = -v3[0];
        dr[6] = -v3[1]; dr[7] = v3[0]; dr[8] = 1.0f;
    } else {
        const float inv = 1.0f / theta;
        const float ax = v3[0] * inv, ay = v3[1] * inv, az = v3[2] * inv;
        const float c = cosf(theta), s = sinf(theta), oc = 1.0f - c;
        dr[0] = c + ax * ax * oc; dr[1] = ax * ay * oc - az * s; dr[2] = ax * az * oc + ay * s;
        dr[3] = ay * ax * oc + az * s; dr[4] = c + ay * ay * oc; dr[5] = ay * az * oc - ax * s;
        dr[6] = az * ax * oc - ay * s; dr[7] = az * ay * oc + ax * s; dr[8] = c + az * az * oc;
    }
    float* R = x + 6;
    float r[9];
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) r[i * 3 + j] = R[i * 3] * dr[j] + R[i * 3 + 1] * dr[3 + j] + R[i * 3 + 2] * dr[6 + j];
    const float fx[3] = {1.0f, 0.0f, 0.0f}, fy[3] = {0.0f, 1.0f, 0.0f};
    const float c0[3] = {r[0], r[3], r[6]};
    float cx[3], cy[3], cz[3];
    normalize_or(c0, fx, cx);
    const float dot = cx[0] * r[1] + cx[1] * r[4] + cx[2] * r[7];
    const float y0[3] = {r[1] - dot * cx[0], r[4] - dot * cx[1], r[7] - dot * cx[2]};
    normalize_or(y0, fy, cy);
    cross3(cx, cy, cz);
    R[0] = cx[0]; R[1] = cy[0]; R[2] = cz[0];
    R[3] = cx[1]; R[4] = cy[1]; R[5] = cz[1];
    R[6] = cx[2]; R[7] = cy[2]; R[8] = cz[2];
    float* v = x + 3;
    const float bv[3] = {R[0] * v[0] + R[3] * v[1] + R[6] * v[2], R[1] * v[0] + R[4] * v[1] + R[7] * v[2],
                         R[2] * v[0] + R[5] * v[1] + R[8] * v[2]};
    const float bd[3] = {d.drag[0] * bv[0], d.drag[1] * bv[1], d.drag[2] * bv[2]};
    const float dw[3] = {R[0] * bd[0] + R[1] * bd[1] + R[2] * bd[2], R[3] * bd[0] + R[4] * bd[1] + R[5] * bd[2],
                         R[6] * bd[0] + R[7] * bd[1] + R[8] * bd[2]};
    const float acc[3] = {R[2] * total / d.mass - dw[0] / d.mass, R[5] * total / d.mass - dw[1] / d.mass,
                          R[8] * total / d.mass - d.gravity - dw[2] / d.mass};
    for (int a = 0; a < 3; ++a) {
        v[a] += acc[a] * dt;
        x[a] += v[a] * dt;
    }
    if (x[2] < 0.05f) {
        x[2] = 0.05f;
        v[2] = fmaxf(v[2], 0.0f);
    }
}

}  // namespace task
}  // namespace lwm
