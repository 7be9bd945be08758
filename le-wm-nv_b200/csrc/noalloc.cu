// noalloc.cu — one fused nominal-physics MPPI iteration on caller-owned
// device buffers, with its scratch in a static device array instead of
// memory the library allocates.
//
// Who needs this: callers that must not allocate device memory while they
// run — a flight controller's real-time loop after start-up, or a host
// runtime that pre-allocates everything and forbids cudaMalloc/cudaFree on
// its control thread (an allocation can synchronise the device and take an
// unbounded time).  They pass every input and output; the only extra memory
// the iteration needs (the per-block MPPI tuples, the per-vehicle arrival
// counters and best scores) lives in `g_noalloc_scratch` below, which every
// GPU that loads this library holds until the process exits.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/lewm_b200.h"
#include "lwm_kernels.hpp"

namespace lwm {
lwm_status set_last_error(lwm_status status, const std::string& message);
}

namespace {

constexpr size_t kScratchBytes = size_t(1) << 20;  // 1 MiB per device
constexpr size_t kCounterBytes = 4096;             // arrival counters: <= 1024 vehicles
constexpr size_t kBestScoreBytes = 4096;           // best score per vehicle
constexpr size_t kPartialBytes = kScratchBytes - kCounterBytes - kBestScoreBytes;
constexpr uint32_t kMaxVehicles = kCounterBytes / sizeof(uint32_t);
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_addr[kMaxDevices] = {};

static_assert(sizeof(lwm_domain) == sizeof(lwm::DomainParams), "domain layouts must agree");

lwm_status fail(lwm_status s, const std::string& m) { return lwm::set_last_error(s, m); }

// Device address of the scratch array on `device` (current), resolved once.
lwm_status scratch_address(int device, unsigned char** out) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_addr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr)
            return fail(LWM_CUDA_ERROR, std::string("cudaGetSymbolAddress(scratch) failed: ") + cudaGetErrorString(e));
        g_scratch_addr[device] = p;
    }
    *out = static_cast<unsigned char*>(g_scratch_addr[device]);
    return LWM_OK;
}

bool finite(float v) { return v == v && v - v == 0.0f; }

// Puts the caller's current device back when the entry point returns.
struct CurrentDevice {
    int device;
    explicit CurrentDevice(int d) : device(d) {}
    ~CurrentDevice() { cudaSetDevice(device); }
    CurrentDevice(const CurrentDevice&) = delete;
    CurrentDevice& operator=(const CurrentDevice&) = delete;
};

}  // namespace

extern "C" lwm_status lwm_nominal_mppi_noalloc(int device, void* stream, const lwm_nominal_scorer_config* cfg,
                                               uint32_t batch, uint32_t samples, uint32_t horizon,
                                               const float* bounds_low, const float* bounds_high, float temperature,
                                               uint64_t seed, uint64_t offset, const lwm_nominal_mppi_io* io) {
    if (!cfg || !bounds_low || !bounds_high || !io) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (!io->initial || !io->motors || !io->reference_states || !io->reference_actions || !io->domains || !io->mean ||
        !io->std || !io->scores || !io->sequence || !io->first_action || !io->warm_start || !io->best_indices)
        return fail(LWM_INVALID_ARGUMENT, "a required device buffer is null");
    if (batch == 0 || samples == 0 || horizon == 0)
        return fail(LWM_INVALID_ARGUMENT, "batch, samples and horizon must be greater than zero");
    if (horizon > lwm::kMaxHorizon) return fail(LWM_INVALID_ARGUMENT, "horizon must be at most 64");
    if (batch > kMaxVehicles)
        return fail(LWM_INVALID_ARGUMENT, "batch " + std::to_string(batch) + " exceeds the no-alloc limit of " +
                                              std::to_string(kMaxVehicles) + " vehicles");
    const uint32_t blocks = lwm::nominal_blocks_per_vehicle(samples);
    const uint32_t pw = (4 + 4 * horizon + 3) & ~3u;
    const size_t need = static_cast<size_t>(batch) * blocks * pw * sizeof(float);
    if (need > kPartialBytes)
        return fail(LWM_INVALID_ARGUMENT, "batch x samples x horizon needs " + std::to_string(need) +
                                              " bytes of MPPI scratch; the no-alloc limit is " +
                                              std::to_string(kPartialBytes) + " bytes");
    if (!finite(cfg->dt) || cfg->dt <= 0.0f || cfg->substeps == 0 || !finite(cfg->trim_scale) || cfg->trim_scale <= 0.0f)
        return fail(LWM_INVALID_ARGUMENT, "invalid nominal physics rollout shape or timestep");
    if (!finite(temperature) || temperature <= 0.0f)
        return fail(LWM_INVALID_ARGUMENT, "MPPI temperature must be finite and greater than zero");
    for (int i = 0; i < 4; ++i) {
        if (!finite(bounds_low[i]) || !finite(bounds_high[i]))
            return fail(LWM_INVALID_ARGUMENT, "action bound " + std::to_string(i) + " is not finite");
        if (bounds_low[i] > bounds_high[i])
            return fail(LWM_INVALID_ARGUMENT, "action bound " + std::to_string(i) + " has low greater than high");
    }
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count || device >= kMaxDevices)
        return fail(LWM_INVALID_ARGUMENT, "CUDA device " + std::to_string(device) + " does not exist");
    int caller_device = 0;
    cudaError_t e = cudaGetDevice(&caller_device);
    if (e != cudaSuccess) return fail(LWM_CUDA_ERROR, std::string("cudaGetDevice failed: ") + cudaGetErrorString(e));
    const CurrentDevice keep(caller_device);  // the caller's current device is back on every return
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return fail(LWM_CUDA_ERROR, std::string("cudaSetDevice failed: ") + cudaGetErrorString(e));
    unsigned char* base = nullptr;
    const lwm_status st = scratch_address(device, &base);
    if (st != LWM_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    lwm::NominalArgs a{};
    a.B = batch;
    a.S = samples;
    a.T = horizon;
    a.substeps = cfg->substeps;
    a.h = cfg->dt / static_cast<float>(cfg->substeps);
    a.inv_trim = static_cast<float>(1.0 / static_cast<double>(cfg->trim_scale));
    a.domains = reinterpret_cast<const lwm::DomainParams*>(io->domains);
    a.initial = io->initial;
    a.motors = io->motors;
    a.ref_states = io->reference_states;
    a.ref_actions = io->reference_actions;
    a.cost.position = cfg->cost.position;
    a.cost.velocity = cfg->cost.velocity;
    a.cost.attitude = cfg->cost.attitude;
    a.cost.angular_velocity = cfg->cost.angular_velocity;
    for (int i = 0; i < 4; ++i) {
        a.cost.action[i] = cfg->cost.action[i];
        a.low[i] = bounds_low[i];
        a.high[i] = bounds_high[i];
    }
    a.sample = 1;
    a.mean = io->mean;
    a.std = io->std;
    a.noise = io->injected_noise;
    a.seed = seed;
    a.offset = offset;
    a.cand_out = nullptr;
    a.scores = io->scores;
    a.states = nullptr;
    a.mppi = 1;
    a.m.counters = reinterpret_cast<unsigned int*>(base);
    a.m.best_score = reinterpret_cast<float*>(base + kCounterBytes);
    a.m.partials = reinterpret_cast<float*>(base + kCounterBytes + kBestScoreBytes);
    a.m.sequence = io->sequence;
    a.m.first_action = io->first_action;
    a.m.warm_start = io->warm_start;
    a.m.best_index = io->best_indices;
    a.m.T = horizon;
    a.m.A = 4;
    a.m.P = blocks;
    a.m.pw = pw;
    a.m.mul = static_cast<float>(-(1.0 / static_cast<double>(temperature)));
    // The arrival counters must start at zero; the kernel leaves them at zero
    // after a completed call, but a call that failed part-way would not.
    e = cudaMemsetAsync(a.m.counters, 0, static_cast<size_t>(batch) * sizeof(uint32_t), s);
    if (e != cudaSuccess) return fail(LWM_CUDA_ERROR, std::string("clearing the scratch counters failed: ") + cudaGetErrorString(e));
    e = lwm::launch_nominal(a, s);
    if (e != cudaSuccess) return fail(LWM_CUDA_ERROR, std::string("nominal MPPI launch failed: ") + cudaGetErrorString(e));
    return LWM_OK;
}
