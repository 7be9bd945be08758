// kernels_fleet_loop.cu — the control loop of a fleet kept on the device.
//
// Between two MPPI plans of a fleet, the controller of every vehicle commits
// the state its plant reached and the action it executed, builds the next
// reference window and the geometric action prior (SkyJepaControllerSession::
// commit_observation / plan_internal, src/models/skyjepa/session.rs:301-400),
// and the plant advances.  Here all of that runs on the device, so a fleet
// loop needs no host round trip per control step:
//   fleet_control_kernel  a block per vehicle: history shift, reference
//                         states (skyjepa_reference_horizon), the prior times
//                         the vehicle's trim, clamped to the rotor bound,
//                         written straight into the scorer's context
//   plant_kernel          a thread per vehicle: `substeps` plant steps with
//                         the vehicle's own domain (SkyJepaRotorPlant::step)
// The task math is lwm_task_math.hpp, shared with the host session.
#include <cuda_runtime.h>

#include <cstdint>

#include "lwm_kernels.hpp"
#include "lwm_task_math.hpp"

namespace lwm {
namespace {

__global__ void __launch_bounds__(128) plant_kernel(const lwm_domain* domains, float* states, float* motors,
                                                    const float* commands, uint32_t stride, uint32_t B, float dt,
                                                    uint32_t substeps) {
    const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const lwm_domain d = domains[b];
    float x[18], m[4], c[4];
    for (int i = 0; i < 18; ++i) x[i] = states[static_cast<size_t>(b) * 18 + i];
    for (int i = 0; i < 4; ++i) {
        m[i] = motors[static_cast<size_t>(b) * 4 + i];
        c[i] = commands[static_cast<size_t>(b) * stride + i];
    }
    for (uint32_t s = 0; s < substeps; ++s) task::plant_step(d, x, m, c, dt);
    for (int i = 0; i < 18; ++i) states[static_cast<size_t>(b) * 18 + i] = x[i];
    for (int i = 0; i < 4; ++i) motors[static_cast<size_t>(b) * 4 + i] = m[i];
}

__global__ void __launch_bounds__(64) fleet_control_kernel(lwm_fleet_step a) {
    __shared__ float s_cur[18];
    __shared__ float s_refs[kMaxHorizon * 18];
    const uint32_t b = blockIdx.x, t = threadIdx.x, T = a.horizon, H = a.history;
    float* sh = a.state_history + static_cast<size_t>(b) * H * 18;
    float* ah = a.action_history + static_cast<size_t>(b) * (H - 1) * 4;
    // commit_observation: drop the oldest state / action, append the new ones
    if (a.last_action) {
        for (uint32_t i = t; i < 18; i += blockDim.x) {
            for (uint32_t h = 0; h + 1 < H; ++h) sh[h * 18 + i] = sh[(h + 1) * 18 + i];
            sh[(H - 1) * 18 + i] = a.state[static_cast<size_t>(b) * 18 + i];
        }
        for (uint32_t i = t; i < 4; i += blockDim.x) {
            for (uint32_t h = 0; h + 2 < H; ++h) ah[h * 4 + i] = ah[(h + 1) * 4 + i];
            ah[(H - 2) * 4 + i] = a.last_action[static_cast<size_t>(b) * a.last_action_stride + i];
        }
    }
    for (uint32_t i = t; i < 18; i += blockDim.x) s_cur[i] = a.state[static_cast<size_t>(b) * 18 + i];
    // skyjepa_reference_horizon: states at time + k dt, k = 1..T
    for (uint32_t k = t; k < T; k += blockDim.x) {
        float* r = s_refs + k * 18;
        task::reference_state(a.reference_kind, a.time + static_cast<float>(k + 1) * a.dt, a.radius, a.period, r);
        for (int i = 0; i < 18; ++i) a.reference_states[(static_cast<size_t>(b) * T + k) * 18 + i] = r[i];
    }
    __syncthreads();
    // prior_action_sequence (session.rs:497-511): the geometric prior of the
    // nominal domain, times the vehicle's trim, clamped to the rotor bound
    const float trim = a.trim ? a.trim[b] : 1.0f;
    const lwm_domain& d = a.prior_domain;
    const float high = d.mass * d.gravity * d.max_thrust_weight / 4.0f;
    for (uint32_t k = t; k < T; k += blockDim.x) {
        float f[4];
        task::geometric_prior_step(s_cur, s_refs, k, T, a.dt, d, f);
        for (int i = 0; i < 4; ++i)
            a.reference_actions[(static_cast<size_t>(b) * T + k) * 4 + i] = task::clampf(f[i] * trim, 0.0f, high);
    }
}

}  // namespace

cudaError_t launch_fleet_control(const lwm_fleet_step& a, cudaStream_t stream) {
    if (a.batch == 0) return cudaSuccess;
    fleet_control_kernel<<<a.batch, 64, 0, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_plant(const lwm_domain* domains, float* states, float* motors, const float* commands,
                         uint32_t stride, uint32_t B, float dt, uint32_t substeps, cudaStream_t stream) {
    if (B == 0) return cudaSuccess;
    plant_kernel<<<(B + 127) / 128, 128, 0, stream>>>(domains, states, motors, commands, stride, B, dt, substeps);
    return cudaGetLastError();
}

}  // namespace lwm
