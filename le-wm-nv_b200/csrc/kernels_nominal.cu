// kernels_nominal.cu — fused nominal-physics MPPI: sample -> trim-calibrated
// rigid-body rollout -> tracking cost -> MPPI reduction, one launch per
// planner iteration.  One thread per candidate (the physics is a sequential
// chain of substeps); candidate actions live in shared memory for the
// weighted action sum.
//
// Physics: SkyJepaRotorPlant::step (src/skyjepa_sim.rs:206-270) with
// orthonormalize (:272-281), as the reference's CPU branch of
// nominal_physics_rollout runs it (src/models/skyjepa/nominal.rs:50-71);
// the reference's CUDA branch (nominal.cu:7-65) computes the same model.
// Cost: tracking_scores (src/models/skyjepa/control.rs:430-452).
// This file is compiled with -fmad=false so that every product and sum is
// rounded separately, as in the reference's f32 CPU plant.
#include <cstdint>
#include <mutex>

#include "lwm_device.cuh"
#include "lwm_kernels.hpp"
#include "lwm_mppi.cuh"

namespace lwm {

constexpr int kNominalThreads = 64;

__device__ __forceinline__ void normalize_div(float& x, float& y, float& z, float fx, float fy, float fz) {
    const float n = sqrtf(x * x + y * y + z * z);
    if (n > 1e-6f) {
        x = x / n; y = y / n; z = z / n;
    } else {
        x = fx; y = fy; z = fz;
    }
}

// One SkyJepaRotorPlant::step; x = p(3) v(3) R(9, row-major) w(3).
__device__ __forceinline__ void plant_step(float* x, float* motors, const float* cmd, float dt,
                                           const DomainParams& d, float response, float max_force) {
    #pragma unroll
    for (int r = 0; r < 4; ++r) {
        float target = cmd[r];
        target = target < 0.0f ? 0.0f : target;
        target = target > max_force ? max_force : target;
        motors[r] += (target - motors[r]) * response;
    }
    float f[4];
    #pragma unroll
    for (int r = 0; r < 4; ++r) f[r] = motors[r] * d.thrust_scale;
    const float total = ((f[0] + f[1]) + f[2]) + f[3];
    const float yaw = 0.025f * d.torque_scale;
    const float torque[3] = {d.arm * (f[1] - f[3]), d.arm * (f[2] - f[0]), yaw * (f[0] - f[1] + f[2] - f[3])};
    float* w = x + 15;
    const float iw[3] = {d.inertia[0] * w[0], d.inertia[1] * w[1], d.inertia[2] * w[2]};
    const float gyro[3] = {w[1] * iw[2] - w[2] * iw[1], w[2] * iw[0] - w[0] * iw[2], w[0] * iw[1] - w[1] * iw[0]};
    #pragma unroll
    for (int a = 0; a < 3; ++a) w[a] += ((torque[a] - gyro[a] - 0.015f * w[a]) / d.inertia[a]) * dt;
    // mat3_from_rotvec (src/data/drone_racing.rs:901-921)
    const float vx = w[0] * dt, vy = w[1] * dt, vz = w[2] * dt;
    const float theta = sqrtf(vx * vx + vy * vy + vz * vz);
    float dr[9];
    if (theta < 1e-6f) {
        dr[0] = 1.0f; dr[1] = -vz; dr[2] = vy;
        dr[3] = vz; dr[4] = 1.0f; dr[5] = -vx;
        dr[6] = -vy; dr[7] = vx; dr[8] = 1.0f;
    } else {
        const float inv = 1.0f / theta;
        const float ax = vx * inv, ay = vy * inv, az = vz * inv;
        float s, c;
        sincosf(theta, &s, &c);
        const float oc = 1.0f - c;
        dr[0] = c + ax * ax * oc; dr[1] = ax * ay * oc - az * s; dr[2] = ax * az * oc + ay * s;
        dr[3] = ay * ax * oc + az * s; dr[4] = c + ay * ay * oc; dr[5] = ay * az * oc - ax * s;
        dr[6] = az * ax * oc - ay * s; dr[7] = az * ay * oc + ax * s; dr[8] = c + az * az * oc;
    }
    float* R = x + 6;
    float r[9];
    #pragma unroll
    for (int i = 0; i < 3; ++i)
        #pragma unroll
        for (int j = 0; j < 3; ++j)
            r[i * 3 + j] = R[i * 3] * dr[j] + R[i * 3 + 1] * dr[3 + j] + R[i * 3 + 2] * dr[6 + j];
    float cx0 = r[0], cx1 = r[3], cx2 = r[6];
    normalize_div(cx0, cx1, cx2, 1.0f, 0.0f, 0.0f);
    const float dot = cx0 * r[1] + cx1 * r[4] + cx2 * r[7];
    float cy0 = r[1] - dot * cx0, cy1 = r[4] - dot * cx1, cy2 = r[7] - dot * cx2;
    normalize_div(cy0, cy1, cy2, 0.0f, 1.0f, 0.0f);
    const float cz0 = cx1 * cy2 - cx2 * cy1, cz1 = cx2 * cy0 - cx0 * cy2, cz2 = cx0 * cy1 - cx1 * cy0;
    R[0] = cx0; R[1] = cy0; R[2] = cz0;
    R[3] = cx1; R[4] = cy1; R[5] = cz1;
    R[6] = cx2; R[7] = cy2; R[8] = cz2;
    float* v = x + 3;
    const float bv[3] = {R[0] * v[0] + R[3] * v[1] + R[6] * v[2], R[1] * v[0] + R[4] * v[1] + R[7] * v[2],
                         R[2] * v[0] + R[5] * v[1] + R[8] * v[2]};
    const float bd[3] = {d.drag[0] * bv[0], d.drag[1] * bv[1], d.drag[2] * bv[2]};
    const float dw[3] = {R[0] * bd[0] + R[1] * bd[1] + R[2] * bd[2], R[3] * bd[0] + R[4] * bd[1] + R[5] * bd[2],
                         R[6] * bd[0] + R[7] * bd[1] + R[8] * bd[2]};
    // body_up = R * e_z: exactly the third column.
    const float acc[3] = {R[2] * total / d.mass - dw[0] / d.mass, R[5] * total / d.mass - dw[1] / d.mass,
                          R[8] * total / d.mass - d.gravity - dw[2] / d.mass};
    #pragma unroll
    for (int a = 0; a < 3; ++a) {
        v[a] += acc[a] * dt;
        x[a] += v[a] * dt;
    }
    if (x[2] < 0.05f) {
        x[2] = 0.05f;
        v[2] = fmaxf(v[2], 0.0f);
    }
}

__global__ void __launch_bounds__(kNominalThreads) nominal_mppi_kernel(NominalArgs a) {
    extern __shared__ float s_dyn[];
    __shared__ float s_score[kNominalThreads];
    __shared__ float s_w[kNominalThreads];
    const uint32_t TA = a.T * 4;
    const uint32_t stride = TA + 1;  // odd stride: rows land in different banks
    float* s_cand = s_dyn;           // [kNominalThreads][stride]
    const uint32_t b = blockIdx.y;
    const uint32_t first = blockIdx.x * kNominalThreads;
    const uint32_t r = threadIdx.x;
    const uint32_t s = first + r;
    const bool valid = s < a.S;
    const uint32_t nrows = min(static_cast<uint32_t>(kNominalThreads), a.S - first);
    const uint64_t row = static_cast<uint64_t>(b) * a.S + s;
    float* my = s_cand + r * stride;

    if (valid) {
        for (uint32_t e = 0; e < TA; ++e) {
            const uint64_t ci = row * TA + e;
            float v;
            if (a.sample) {
                const uint32_t act = e & 3u;
                const size_t mi = static_cast<size_t>(b) * TA + e;
                if (a.sample_base + s == 0) {
                    v = a.mean[mi];
                } else {
                    const uint64_t gi = global_row(b, s, a.sample_base, a.sample_total, a.S) * TA + e;
                    const float eps = a.noise ? a.noise[ci] : normal_at(a.seed, a.offset + gi);
                    v = a.mean[mi] + eps * a.std[mi];
                }
                v = cmin(cmax(v, a.low[act]), a.high[act]);
                if (a.cand_out) a.cand_out[ci] = v;
            } else {
                v = a.cand_in[ci];
            }
            my[e] = v;
        }
    }

    float score = 0.0f;
    if (valid) {
        const DomainParams d = a.domains[b];
        const float response = 1.0f - expf(-a.h / d.tau);
        const float max_force = d.mass * d.gravity * d.max_tw / 4.0f;
        float x[18], motors[4];
        #pragma unroll
        for (int i = 0; i < 18; ++i) x[i] = a.initial[static_cast<size_t>(b) * 18 + i];
        #pragma unroll
        for (int i = 0; i < 4; ++i) motors[i] = a.motors[static_cast<size_t>(b) * 4 + i];
        float total = 0.0f;
        for (uint32_t t = 0; t < a.T; ++t) {
            float cmd[4];
            #pragma unroll
            for (int i = 0; i < 4; ++i) cmd[i] = my[t * 4 + i] * a.inv_trim;
            for (uint32_t k = 0; k < a.substeps; ++k) plant_step(x, motors, cmd, a.h, d, response, max_force);
            if (a.states) {
                float* o = a.states + (row * a.T + t) * 18;
                #pragma unroll
                for (int i = 0; i < 18; ++i) o[i] = x[i];
            }
            const float* ref = a.ref_states + (static_cast<size_t>(b) * a.T + t) * 18;
            float g0 = 0.0f, g1 = 0.0f, g2 = 0.0f, g3 = 0.0f;
            #pragma unroll
            for (int i = 0; i < 3; ++i) { const float dd = x[i] - ref[i]; g0 += dd * dd; }
            #pragma unroll
            for (int i = 3; i < 6; ++i) { const float dd = x[i] - ref[i]; g1 += dd * dd; }
            #pragma unroll
            for (int i = 6; i < 15; ++i) { const float dd = x[i] - ref[i]; g2 += dd * dd; }
            #pragma unroll
            for (int i = 15; i < 18; ++i) { const float dd = x[i] - ref[i]; g3 += dd * dd; }
            const float* ra = a.ref_actions + (static_cast<size_t>(b) * a.T + t) * 4;
            float act = 0.0f;
            #pragma unroll
            for (int i = 0; i < 4; ++i) { const float dd = my[t * 4 + i] - ra[i]; act += (dd * dd) * a.cost.action[i]; }
            float st = g0 * a.cost.position + g1 * a.cost.velocity;
            st = st + g2 * a.cost.attitude;
            st = st + g3 * a.cost.angular_velocity;
            total += st + act;
        }
        score = total * static_cast<float>(1.0 / static_cast<double>(a.T));  // Candle mean
        a.scores[row] = score;
    }
    s_score[r] = score;
    __syncthreads();
    if (a.mppi) mppi_reduce_rows<kNominalThreads>(a.m, b, blockIdx.x, nrows, s_score, first, s_cand, stride, s_w);
}

uint32_t nominal_blocks_per_vehicle(uint32_t S) { return (S + kNominalThreads - 1) / kNominalThreads; }

cudaError_t launch_nominal(const NominalArgs& a, cudaStream_t stream) {
    if (a.T == 0 || a.T > kMaxHorizon) return cudaErrorInvalidValue;
    const size_t smem = static_cast<size_t>(kNominalThreads) * (a.T * 4 + 1) * sizeof(float);
    if (smem > 48 * 1024) {
        // the opt-in for the longest horizon, once per device (not a driver
        // call on every plan of a real-time loop)
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
        static std::mutex mu;
        static bool configured[64] = {};
        std::lock_guard<std::mutex> lock(mu);
        if (!configured[dev]) {
            const size_t max_smem = static_cast<size_t>(kNominalThreads) * (kMaxHorizon * 4 + 1) * sizeof(float);
            e = cudaFuncSetAttribute(nominal_mppi_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(max_smem));
            if (e != cudaSuccess) return e;
            configured[dev] = true;
        }
    }
    dim3 grid(nominal_blocks_per_vehicle(a.S), a.B);
    nominal_mppi_kernel<<<grid, kNominalThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace lwm
