// api.cpp — the C ABI (include/lewm_b200.h): contexts, planners (MPPI, CEM,
// iCEM) and candidate scorers, written as C++ objects that mirror the
// reference's Rust types (src/planner.rs, src/models/skyjepa/control.rs).
//
// Nothing here computes on the host except validation and bookkeeping; every
// numeric step is a kernel launch on the context's stream, and the only
// device synchronisation is in lwm_plan (the result copy to host memory).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <charconv>
#include <chrono>
#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <random>
#include <string>
#include <vector>

#include "../../include/lewm_b200.h"
#include "lwm_kernels.hpp"
#include "lwm_host.hpp"
#include "lwm_lewm.hpp"

using lwm::MppiArgs;

namespace {

thread_local std::string g_last_error;

lwm_status fail(lwm_status s, const std::string& msg) {
    g_last_error = msg;
    return s;
}

// Rust's `{}` formatting of an f32: shortest round-trip digits, no exponent.
std::string fmt(float v) {
    if (std::isnan(v)) return "NaN";
    if (std::isinf(v)) return v > 0 ? "inf" : "-inf";
    char buf[64];
    auto r = std::to_chars(buf, buf + sizeof buf, v, std::chars_format::fixed);
    return std::string(buf, r.ptr);
}

bool finite(float v) { return std::isfinite(v); }

#define LWM_CUDA(expr)                                                                      \
    do {                                                                                    \
        cudaError_t e_ = (expr);                                                            \
        if (e_ != cudaSuccess)                                                              \
            return fail(LWM_CUDA_ERROR, std::string(#expr) + " failed: " + cudaGetErrorString(e_)); \
    } while (0)

#define LWM_TRY(expr)                       \
    do {                                    \
        lwm_status s_ = (expr);             \
        if (s_ != LWM_OK) return s_;        \
    } while (0)

// Device allocation that only grows.
struct DevBuf {
    void* ptr = nullptr;
    size_t bytes = 0;
    bool view = false;  // a part of another DevBuf's allocation (not freed here)
    lwm_status ensure(size_t need) {
        if (need <= bytes) return LWM_OK;
        if (view) return fail(LWM_CUDA_ERROR, "internal: a buffer view cannot grow");
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
        cudaError_t e = cudaMalloc(&ptr, need);
        if (e != cudaSuccess) return fail(LWM_CUDA_ERROR, std::string("cudaMalloc failed: ") + cudaGetErrorString(e));
        bytes = need;
        return LWM_OK;
    }
    template <class T> T* as() const { return static_cast<T*>(ptr); }
    void release() {
        if (ptr && !view) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
        view = false;
    }
    void set_view(void* base, size_t off, size_t n) {
        ptr = static_cast<char*>(base) + off;
        bytes = n;
        view = true;
    }
};

// A plan's outputs (first action, sequence, scores, best indices) share one
// device allocation laid out like the pinned staging they are copied to, so
// that lwm_plan reads all of them back with one copy.
struct ResultLayout {
    size_t fa, seq, sc, best, err, total;
};
inline size_t round256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }
// first action, sequence, scores, best indices, then the tensor-core
// rollouts' error word (4 ints: site, block, detail, parity), so that one
// device-to-host copy brings back the results and the error word together
inline ResultLayout result_layout(size_t B, size_t T, size_t A, size_t S) {
    ResultLayout l;
    l.fa = 0;
    l.seq = round256(B * A * 4);
    l.sc = round256(l.seq + B * T * A * 4);
    l.best = round256(l.sc + B * S * 4);
    l.err = (l.best + B * 4 + 15) & ~static_cast<size_t>(15);
    l.total = l.err + 4 * sizeof(int);
    return l;
}

// Pinned host staging that only grows.
struct HostBuf {
    void* ptr = nullptr;
    size_t bytes = 0;
    lwm_status ensure(size_t need) {
        if (need <= bytes) return LWM_OK;
        if (ptr) cudaFreeHost(ptr);
        ptr = nullptr;
        bytes = 0;
        cudaError_t e = cudaMallocHost(&ptr, need);
        if (e != cudaSuccess) return fail(LWM_CUDA_ERROR, std::string("cudaMallocHost failed: ") + cudaGetErrorString(e));
        bytes = need;
        return LWM_OK;
    }
    template <class T> T* as() const { return static_cast<T*>(ptr); }
    void release() {
        if (ptr) cudaFreeHost(ptr);
        ptr = nullptr;
        bytes = 0;
    }
};

uint64_t round_even(uint64_t n) { return (n % 2 == 0) ? n : n + 1; }

}  // namespace

namespace lwm {
// Records the thread's last error for entry points defined in other files.
lwm_status set_last_error(lwm_status status, const std::string& message) { return fail(status, message); }
}  // namespace lwm

struct lwm_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::atomic<uint64_t> launches{0};
    uint64_t unseeded_seed = 0;
    std::atomic<uint64_t> unseeded_offset{0};
    // error word of the row-staged NV12 kernel: mapped pinned host memory,
    // read after every stream synchronisation (allocated on first use)
    int* media_err = nullptr;
    int* media_err_dev = nullptr;
    lwm_test_faults faults{};  // fault injection for tests (lwm_ctx_set_test_faults)
    // kernel timing (lwm_ctx_set_kernel_timing): events around the last
    // SkyJEPA rollout launch
    cudaEvent_t kt_begin = nullptr, kt_end = nullptr;
    bool kt_on = false, kt_valid = false;
    void kernel_timing(lwm::SkyjepaArgs& a) {
        if (!kt_on) return;
        a.time_begin = kt_begin;
        a.time_end = kt_end;
        kt_valid = true;
    }
};

enum class PlannerKind { Mppi, Cem, Icem };
enum class ScorerKind { Nominal, Skyjepa, Callback, Lewm };

struct lwm_scorer {
    lwm_ctx* ctx = nullptr;
    ScorerKind kind = ScorerKind::Callback;
    std::mutex mu;
    uint32_t batch = 0, horizon = 0;
    bool has_context = false;
    // nominal
    lwm_nominal_scorer_config nominal{};
    // skyjepa
    lwm_skyjepa_config sky{};
    lwm::SkyjepaArgs sky_args{};  // weight views + constants, context pointers set per plan
    DevBuf weights;
    lwm_tracking_cost cost{};
    float dt = 0.05f;
    // context (device) and its pinned staging
    DevBuf ctx_dev;
    HostBuf ctx_host;
    cudaEvent_t staged = nullptr;
    size_t off_initial = 0, off_motors = 0, off_ref_states = 0, off_ref_actions = 0, off_domains = 0;
    size_t off_state_hist = 0, off_action_hist = 0, off_masses = 0;
    bool has_masses = false;
    // callback
    lwm_score_fn fn = nullptr;
    void* user = nullptr;
    // LeWM world model
    std::unique_ptr<lwm::LewmModel> lewm;
    // learned scorer on tensor cores (bf16): packed weights, per-vehicle h0, wait-timeout flag
    int32_t precision = LWM_PRECISION_F32;
    DevBuf tc_packed, tc_h0, tc_x, h0_work;
    bool sky_small = false;  // latent <= 64: the warp-per-candidate path (h0 in tc_h0, inputs in small_x)
    DevBuf small_x;
    lwm::SideStream side;    // the history encoding runs here, beside sampling and the inputs
    lwm::SideStream enc_side;  // LeWM: the frame encoder of lwm_lewm_plan_nv12_device (high priority)
    std::vector<float> action_tcn_host;  // the action encoder's weights, for kernel-parameter packing
    bool tc_ready = false;
    DevBuf mma_packed;       // split-fp16 weights of the f32 tensor-core path (per CTA rank)
    DevBuf mma_xchg;         // its per-step h exchange between the CTAs of a cluster
    bool mma_ready = false;
};

struct lwm_planner {
    lwm_ctx* ctx = nullptr;
    PlannerKind kind = PlannerKind::Mppi;
    std::mutex mu;
    lwm_mppi_config mppi{};
    lwm_cem_config cem{};
    lwm_icem_config icem{};
    uint32_t T = 0, S = 0, A = 0, iterations = 0;
    std::atomic<uint64_t> rng_offset{0};
    bool has_warm = false;
    uint32_t warm_batch = 0;
    // device state, sized for `cap_b` vehicles
    uint32_t cap_b = 0;
    DevBuf bounds, zeros, std_init, mean, stdv, cand, scores, partials, counters, sequence, first_action, warm,
        best, best_score, carried, noise_tmp;
    DevBuf results;  // holds first_action, sequence, scores, best (views into it) and the error word
    uint32_t results_batch = 0;  // the batch the views were laid out for
    HostBuf staging;
    uint32_t last_batch = 0, last_cols = 0;
    // iCEM trace: [iterations][4][B] scores and the elite mean of an iteration
    DevBuf trace, trace_elite;
    // candidate-range shard (shard_total 0: unsharded) and its combined tuples
    uint32_t shard_base = 0, shard_total = 0;
    DevBuf shard_tuples;
    // CEM / iCEM shards: the elite exchange and its buffers
    lwm_exchange_fn exchange = nullptr;
    void* exchange_user = nullptr;
    uint32_t exchange_shards = 0;
    DevBuf elite_local, elite_gathered, merged_scores, merged_cand, merged_index;
    // CEM / iCEM: the elite indices every iteration of the last plan selected [iterations][B][K]
    DevBuf elite_idx;
    uint32_t elite_iterations = 0;
    bool has_result = false;
};

// The tensor-core rollouts' error word in the planner's result block.
static int* result_err(lwm_planner* p, uint32_t B) {
    return reinterpret_cast<int*>(static_cast<char*>(p->results.ptr) + result_layout(B, p->T, p->A, p->S).err);
}

namespace {

const char* planner_name(PlannerKind k) {
    return k == PlannerKind::Mppi ? "MPPI" : (k == PlannerKind::Cem ? "CEM" : "iCEM");
}

// ActionBounds::validate (src/planner.rs:85-103).
lwm_status validate_bounds(const float* low, const float* high, uint32_t action_dim) {
    for (uint32_t i = 0; i < action_dim; ++i) {
        if (!finite(low[i]) || !finite(high[i])) return fail(LWM_INVALID_ARGUMENT, "action bound " + std::to_string(i) + " is not finite");
        if (low[i] > high[i])
            return fail(LWM_INVALID_ARGUMENT, "action bound " + std::to_string(i) + " has low " + fmt(low[i]) +
                                                  " greater than high " + fmt(high[i]));
    }
    return LWM_OK;
}

// validate_deadline_action (src/planner.rs:1060-1089).
lwm_status validate_deadline(int32_t has, const float* action, uint32_t action_dim, const float* low, const float* high,
                             const char* name) {
    if (!has) return LWM_OK;
    for (uint32_t i = 0; i < action_dim; ++i) {
        if (!finite(action[i]))
            return fail(LWM_INVALID_ARGUMENT, std::string(name) + " deadline_action[" + std::to_string(i) + "] is not finite");
        if (action[i] < low[i] || action[i] > high[i])
            return fail(LWM_INVALID_ARGUMENT, std::string(name) + " deadline_action[" + std::to_string(i) + "]=" + fmt(action[i]) +
                                                  " is outside [" + fmt(low[i]) + ", " + fmt(high[i]) + "]");
    }
    return LWM_OK;
}

lwm_status check_dims(uint32_t horizon, uint32_t action_dim) {
    if (action_dim > LWM_MAX_ACTION_DIM)
        return fail(LWM_UNSUPPORTED, "action_dim " + std::to_string(action_dim) + " exceeds the supported maximum of 16");
    if (horizon > lwm::kMaxHorizon)
        return fail(LWM_UNSUPPORTED, "horizon " + std::to_string(horizon) + " exceeds the supported maximum of 64");
    return LWM_OK;
}

// MppiConfig::validate (src/planner.rs:210-253).
lwm_status validate_mppi(const lwm_mppi_config& c) {
    if (c.horizon == 0) return fail(LWM_INVALID_ARGUMENT, "MPPI horizon must be greater than zero");
    if (c.samples == 0) return fail(LWM_INVALID_ARGUMENT, "MPPI samples must be greater than zero");
    if (c.iterations == 0) return fail(LWM_INVALID_ARGUMENT, "MPPI iterations must be greater than zero");
    if (c.action_dim == 0) return fail(LWM_INVALID_ARGUMENT, "MPPI action_dim must be greater than zero");
    LWM_TRY(check_dims(c.horizon, c.action_dim));
    if (!finite(c.noise_std) || c.noise_std <= 0.0f)
        return fail(LWM_INVALID_ARGUMENT, "MPPI noise_std must be finite and greater than zero");
    if (c.has_noise_std_per_action)
        for (uint32_t i = 0; i < c.action_dim; ++i)
            if (!finite(c.noise_std_per_action[i]) || c.noise_std_per_action[i] <= 0.0f)
                return fail(LWM_INVALID_ARGUMENT, "MPPI per-action noise values must be finite and greater than zero");
    if (!finite(c.temperature) || c.temperature <= 0.0f)
        return fail(LWM_INVALID_ARGUMENT, "MPPI temperature must be finite and greater than zero");
    LWM_TRY(validate_bounds(c.bounds_low, c.bounds_high, c.action_dim));
    return validate_deadline(c.has_deadline_action, c.deadline_action, c.action_dim, c.bounds_low, c.bounds_high, "MPPI");
}

// CemConfig::validate (src/planner.rs:139-175).
lwm_status validate_cem(const lwm_cem_config& c) {
    if (c.horizon == 0) return fail(LWM_INVALID_ARGUMENT, "CEM horizon must be greater than zero");
    if (c.samples == 0) return fail(LWM_INVALID_ARGUMENT, "CEM samples must be greater than zero");
    if (c.elites < 2) return fail(LWM_INVALID_ARGUMENT, "CEM elites must be at least two");
    if (c.elites > c.samples)
        return fail(LWM_INVALID_ARGUMENT, "CEM elites " + std::to_string(c.elites) + " cannot exceed samples " + std::to_string(c.samples));
    if (c.iterations == 0) return fail(LWM_INVALID_ARGUMENT, "CEM iterations must be greater than zero");
    if (c.action_dim == 0) return fail(LWM_INVALID_ARGUMENT, "CEM action_dim must be greater than zero");
    LWM_TRY(check_dims(c.horizon, c.action_dim));
    if (!finite(c.init_std) || c.init_std <= 0.0f) return fail(LWM_INVALID_ARGUMENT, "CEM init_std must be finite and greater than zero");
    if (!finite(c.min_std) || c.min_std < 0.0f) return fail(LWM_INVALID_ARGUMENT, "CEM min_std must be finite and non-negative");
    LWM_TRY(validate_bounds(c.bounds_low, c.bounds_high, c.action_dim));
    return validate_deadline(c.has_deadline_action, c.deadline_action, c.action_dim, c.bounds_low, c.bounds_high, "CEM");
}

// IcemConfig::validate (src/planner.rs:296-345).
lwm_status validate_icem(const lwm_icem_config& c) {
    if (c.horizon == 0) return fail(LWM_INVALID_ARGUMENT, "iCEM horizon must be greater than zero");
    if (c.samples == 0) return fail(LWM_INVALID_ARGUMENT, "iCEM samples must be greater than zero");
    if (c.elites < 2) return fail(LWM_INVALID_ARGUMENT, "iCEM elites must be at least two");
    if (c.elites > c.samples)
        return fail(LWM_INVALID_ARGUMENT, "iCEM elites " + std::to_string(c.elites) + " cannot exceed samples " +
                                              std::to_string(c.samples) + " on the first iteration");
    if (c.keep_elites > c.elites)
        return fail(LWM_INVALID_ARGUMENT, "iCEM keep_elites " + std::to_string(c.keep_elites) + " cannot exceed elites " +
                                              std::to_string(c.elites));
    if (c.iterations == 0) return fail(LWM_INVALID_ARGUMENT, "iCEM iterations must be greater than zero");
    if (!finite(c.noise_beta) || c.noise_beta < 0.0f) return fail(LWM_INVALID_ARGUMENT, "iCEM noise_beta must be finite and non-negative");
    if (!finite(c.alpha) || c.alpha < 0.0f || c.alpha > 1.0f) return fail(LWM_INVALID_ARGUMENT, "iCEM alpha must be finite and in [0, 1]");
    if (c.action_dim == 0) return fail(LWM_INVALID_ARGUMENT, "iCEM action_dim must be greater than zero");
    LWM_TRY(check_dims(c.horizon, c.action_dim));
    if (!finite(c.init_std) || c.init_std <= 0.0f) return fail(LWM_INVALID_ARGUMENT, "iCEM init_std must be finite and greater than zero");
    if (!finite(c.min_std) || c.min_std < 0.0f) return fail(LWM_INVALID_ARGUMENT, "iCEM min_std must be finite and non-negative");
    LWM_TRY(validate_bounds(c.bounds_low, c.bounds_high, c.action_dim));
    return validate_deadline(c.has_deadline_action, c.deadline_action, c.action_dim, c.bounds_low, c.bounds_high, "iCEM");
}

lwm_status validate_planner(const lwm_planner* p) {
    switch (p->kind) {
        case PlannerKind::Mppi: return validate_mppi(p->mppi);
        case PlannerKind::Cem: return validate_cem(p->cem);
        default: return validate_icem(p->icem);
    }
}

const float* planner_low(const lwm_planner* p) {
    return p->kind == PlannerKind::Mppi ? p->mppi.bounds_low : (p->kind == PlannerKind::Cem ? p->cem.bounds_low : p->icem.bounds_low);
}
const float* planner_high(const lwm_planner* p) {
    return p->kind == PlannerKind::Mppi ? p->mppi.bounds_high : (p->kind == PlannerKind::Cem ? p->cem.bounds_high : p->icem.bounds_high);
}

lwm::CostParams cost_params(const lwm_tracking_cost& c) {
    lwm::CostParams p;
    p.position = c.position;
    p.velocity = c.velocity;
    p.attitude = c.attitude;
    p.angular_velocity = c.angular_velocity;
    for (int i = 0; i < 4; ++i) p.action[i] = c.action[i];
    return p;
}

// SkyJepaTrackingCost::validate (src/models/skyjepa/control.rs:40-63).
lwm_status validate_cost(const lwm_tracking_cost& c) {
    const char* names[4] = {"position", "velocity", "attitude", "angular_velocity"};
    const float vals[4] = {c.position, c.velocity, c.attitude, c.angular_velocity};
    for (int i = 0; i < 4; ++i)
        if (!finite(vals[i]) || vals[i] < 0.0f)
            return fail(LWM_INVALID_ARGUMENT, std::string("SkyJEPA ") + names[i] + " cost must be finite and non-negative");
    for (int i = 0; i < 4; ++i)
        if (!finite(c.action[i]) || c.action[i] < 0.0f)
            return fail(LWM_INVALID_ARGUMENT, "SkyJEPA action costs must be finite and non-negative");
    return LWM_OK;
}

// SkyJepaDomain::validate (src/skyjepa_sim.rs:88-123).
lwm_status validate_domain(const lwm_domain& d) {
    if (!finite(d.mass) || d.mass <= 0.0f) return fail(LWM_INVALID_ARGUMENT, "mass must be positive");
    for (int i = 0; i < 3; ++i)
        if (!finite(d.inertia[i]) || d.inertia[i] <= 0.0f) return fail(LWM_INVALID_ARGUMENT, "inertia must be positive");
    if (!finite(d.motor_time_constant) || d.motor_time_constant <= 0.0f)
        return fail(LWM_INVALID_ARGUMENT, "motor time constant must be positive");
    for (int i = 0; i < 3; ++i)
        if (!finite(d.drag[i]) || d.drag[i] < 0.0f) return fail(LWM_INVALID_ARGUMENT, "drag must be non-negative");
    if (!finite(d.thrust_scale) || d.thrust_scale <= 0.0f) return fail(LWM_INVALID_ARGUMENT, "thrust scale must be positive");
    if (!finite(d.torque_scale) || d.torque_scale <= 0.0f) return fail(LWM_INVALID_ARGUMENT, "torque scale must be positive");
    if (!finite(d.arm_length) || d.arm_length <= 0.0f) return fail(LWM_INVALID_ARGUMENT, "arm length must be positive");
    return LWM_OK;
}

lwm::DomainParams domain_params(const lwm_domain& d) {
    lwm::DomainParams p;
    p.mass = d.mass;
    for (int i = 0; i < 3; ++i) { p.inertia[i] = d.inertia[i]; p.drag[i] = d.drag[i]; }
    p.tau = d.motor_time_constant;
    p.thrust_scale = d.thrust_scale;
    p.torque_scale = d.torque_scale;
    p.arm = d.arm_length;
    p.gravity = d.gravity;
    p.max_tw = d.max_thrust_weight;
    return p;
}

// ------------------------------------------------------------- planner state

lwm_status ensure_planner_buffers(lwm_planner* p, uint32_t B) {
    if (B <= p->cap_b && p->cap_b != 0) return LWM_OK;
    const size_t seq = static_cast<size_t>(B) * p->T * p->A;
    const size_t n = seq * p->S;
    uint32_t P = std::max<uint32_t>(lwm::nominal_blocks_per_vehicle(p->S),
                                    lwm::skyjepa_partials_per_vehicle(p->S, 32));
    P = std::max<uint32_t>(P, (p->S + 255) / 256);
    P = std::max<uint32_t>(P, lwm::skyjepa_small_partials_per_vehicle(p->S));
    const size_t pw = (4 + static_cast<size_t>(p->T) * p->A + 3) & ~static_cast<size_t>(3);
    LWM_TRY(p->zeros.ensure(seq * 4));
    LWM_TRY(p->std_init.ensure(seq * 4));
    LWM_TRY(p->mean.ensure(seq * 4));
    LWM_TRY(p->stdv.ensure(seq * 4));
    LWM_TRY(p->cand.ensure(n * 4));
    const ResultLayout rl = result_layout(B, p->T, p->A, p->S);
    if (p->results.bytes < rl.total) {
        LWM_TRY(p->results.ensure(rl.total));
        LWM_CUDA(cudaMemset(p->results.ptr, 0, rl.total));  // the error word starts clear
    }
    if (p->results_batch != B) {
        // the views move with the batch (the error word is zero wherever it lands:
        // every plan that can set it clears it first, and a reported error clears it)
        LWM_CUDA(cudaMemset(static_cast<char*>(p->results.ptr) + rl.err, 0, 4 * sizeof(int)));
        p->results_batch = B;
    }
    p->first_action.set_view(p->results.ptr, rl.fa, static_cast<size_t>(B) * p->A * 4);
    p->sequence.set_view(p->results.ptr, rl.seq, seq * 4);
    p->scores.set_view(p->results.ptr, rl.sc, static_cast<size_t>(B) * p->S * 4);
    p->best.set_view(p->results.ptr, rl.best, static_cast<size_t>(B) * 4);
    LWM_TRY(p->partials.ensure(static_cast<size_t>(B) * P * pw * 4));
    LWM_TRY(p->counters.ensure(static_cast<size_t>(B) * 4));

    // the warm start is kept across plans: preserve it when growing
    if (p->warm.bytes < seq * 4) {
        DevBuf grown;
        LWM_TRY(grown.ensure(seq * 4));
        if (p->warm.ptr) LWM_CUDA(cudaMemcpyAsync(grown.ptr, p->warm.ptr, p->warm.bytes, cudaMemcpyDeviceToDevice, p->ctx->stream));
        LWM_CUDA(cudaStreamSynchronize(p->ctx->stream));
        p->warm.release();
        p->warm = grown;
    }
    LWM_TRY(p->best_score.ensure(static_cast<size_t>(B) * 4));
    LWM_TRY(p->shard_tuples.ensure(static_cast<size_t>(B) * pw * 4));
    const uint32_t keep = p->kind == PlannerKind::Icem ? std::max<uint32_t>(p->icem.keep_elites, 1) : 1;
    LWM_TRY(p->carried.ensure(static_cast<size_t>(B) * keep * p->T * p->A * 4));
    if (p->kind != PlannerKind::Mppi) {
        const uint32_t K = p->kind == PlannerKind::Cem ? p->cem.elites : p->icem.elites;
        LWM_TRY(p->elite_idx.ensure(static_cast<size_t>(p->iterations) * B * K * 4));
    }
    LWM_TRY(p->bounds.ensure(2 * LWM_MAX_ACTION_DIM * 4));
    // staging carries the bounds (2 x 16 floats), the initial std, deadline
    // sequences and the result burst of lwm_plan
    const size_t staging = std::max<size_t>(seq * 4 * 3 + static_cast<size_t>(B) * p->S * 4 + static_cast<size_t>(B) * 8 + 1024,
                                            2 * LWM_MAX_ACTION_DIM * 4);
    LWM_TRY(p->staging.ensure(staging));
    LWM_CUDA(cudaMemsetAsync(p->zeros.ptr, 0, seq * 4, p->ctx->stream));
    LWM_CUDA(cudaMemsetAsync(p->counters.ptr, 0, static_cast<size_t>(B) * 4, p->ctx->stream));
    // bounds [low(16), high(16)] and the per-plan initial std, both constant per planner
    float* h = p->staging.as<float>();
    std::memcpy(h, planner_low(p), LWM_MAX_ACTION_DIM * 4);
    std::memcpy(h + LWM_MAX_ACTION_DIM, planner_high(p), LWM_MAX_ACTION_DIM * 4);
    LWM_CUDA(cudaMemcpyAsync(p->bounds.ptr, h, 2 * LWM_MAX_ACTION_DIM * 4, cudaMemcpyHostToDevice, p->ctx->stream));
    LWM_CUDA(cudaStreamSynchronize(p->ctx->stream));
    for (size_t i = 0; i < seq; ++i) {
        const uint32_t a = static_cast<uint32_t>(i % p->A);
        float v;
        if (p->kind == PlannerKind::Mppi) v = p->mppi.has_noise_std_per_action ? p->mppi.noise_std_per_action[a] : p->mppi.noise_std;
        else if (p->kind == PlannerKind::Cem) v = p->cem.init_std;
        else v = p->icem.init_std;
        h[i] = v;
    }
    LWM_CUDA(cudaMemcpyAsync(p->std_init.ptr, h, seq * 4, cudaMemcpyHostToDevice, p->ctx->stream));
    LWM_CUDA(cudaStreamSynchronize(p->ctx->stream));
    p->cap_b = B;
    return LWM_OK;
}

MppiArgs mppi_args(lwm_planner* p, float temperature) {
    MppiArgs m{};
    m.partials = p->partials.as<float>();
    m.counters = p->counters.as<unsigned int>();
    m.sequence = p->sequence.as<float>();
    m.first_action = p->first_action.as<float>();
    m.warm_start = p->warm.as<float>();
    m.best_index = p->best.as<uint32_t>();
    m.best_score = p->best_score.as<float>();
    m.T = p->T;
    m.A = p->A;
    m.pw = static_cast<uint32_t>((4 + static_cast<size_t>(p->T) * p->A + 3) & ~static_cast<size_t>(3));
    m.mul = static_cast<float>(-(1.0 / static_cast<double>(temperature)));
    return m;
}

// -------------------------------------------------------------- scorer calls

lwm::NominalArgs nominal_args(lwm_scorer* sc, uint32_t S) {
    lwm::NominalArgs a{};
    a.B = sc->batch;
    a.S = S;
    a.T = sc->horizon;
    a.substeps = sc->nominal.substeps;
    a.h = sc->nominal.dt / static_cast<float>(sc->nominal.substeps);
    a.inv_trim = static_cast<float>(1.0 / static_cast<double>(sc->nominal.trim_scale));
    const char* base = sc->ctx_dev.as<char>();
    a.domains = reinterpret_cast<const lwm::DomainParams*>(base + sc->off_domains);
    a.initial = reinterpret_cast<const float*>(base + sc->off_initial);
    a.motors = reinterpret_cast<const float*>(base + sc->off_motors);
    a.ref_states = reinterpret_cast<const float*>(base + sc->off_ref_states);
    a.ref_actions = reinterpret_cast<const float*>(base + sc->off_ref_actions);
    a.cost = cost_params(sc->nominal.cost);
    return a;
}

// Packed bf16 weights (once per scorer), per-vehicle h0 and the error flag.
lwm_status ensure_side(lwm_scorer* sc);

lwm_status ensure_tc(lwm_scorer* sc, const lwm::SkyjepaArgs& a, uint32_t B, uint32_t S, uint32_t T) {
    LWM_TRY(ensure_side(sc));
    if (!sc->tc_ready) {
        LWM_TRY(sc->tc_packed.ensure(lwm::skyjepa_tc_packed_bytes()));
        LWM_CUDA(lwm::skyjepa_tc_pack(a, sc->tc_packed.as<uint8_t>(), sc->ctx->stream));
        sc->tc_ready = true;
    }
    LWM_TRY(sc->tc_h0.ensure(static_cast<size_t>(B) * a.H * sizeof(float)));
    LWM_TRY(sc->h0_work.ensure(lwm::skyjepa_h0_work_bytes(a, B)));
    LWM_TRY(sc->tc_x.ensure(lwm::skyjepa_tc_xtile_bytes(B, S, T)));
    return LWM_OK;
}

lwm_status ensure_mma(lwm_scorer* sc, const lwm::SkyjepaArgs& a, uint32_t B, uint32_t S, uint32_t T) {
    LWM_TRY(ensure_side(sc));
    if (!sc->mma_ready) {
        LWM_TRY(sc->mma_packed.ensure(lwm::skyjepa_mma_packed_bytes()));
        LWM_CUDA(lwm::skyjepa_mma_pack(a, sc->mma_packed.as<uint8_t>(), sc->ctx->stream));
        sc->mma_ready = true;
    }
    LWM_TRY(sc->tc_h0.ensure(static_cast<size_t>(B) * a.H * sizeof(float)));
    LWM_TRY(sc->h0_work.ensure(lwm::skyjepa_h0_work_bytes(a, B)));
    LWM_TRY(sc->tc_x.ensure(lwm::skyjepa_mma_xtile_bytes(B, S, T)));
    LWM_TRY(sc->mma_xchg.ensure(lwm::skyjepa_mma_exchange_bytes(B, S)));
    return LWM_OK;
}

lwm_status ensure_side(lwm_scorer* sc) {
    if (sc->side.stream) return LWM_OK;
    LWM_CUDA(cudaStreamCreateWithFlags(&sc->side.stream, cudaStreamNonBlocking));
    LWM_CUDA(cudaEventCreateWithFlags(&sc->side.fork, cudaEventDisableTiming));
    LWM_CUDA(cudaEventCreateWithFlags(&sc->side.join, cudaEventDisableTiming));
    return LWM_OK;
}

lwm_status ensure_small(lwm_scorer* sc, const lwm::SkyjepaArgs& a, uint32_t B, uint32_t S, uint32_t T) {
    LWM_TRY(ensure_side(sc));
    LWM_TRY(sc->tc_h0.ensure(static_cast<size_t>(B) * a.H * sizeof(float)));
    LWM_TRY(sc->h0_work.ensure(lwm::skyjepa_h0_work_bytes(a, B)));
    LWM_TRY(sc->small_x.ensure(std::max<size_t>(lwm::skyjepa_small_x_bytes(a, B, S, T), 4)));
    return LWM_OK;
}

lwm::SkyjepaArgs skyjepa_args(lwm_scorer* sc, uint32_t S) {
    lwm::SkyjepaArgs a = sc->sky_args;
    a.action_tcn_host = sc->action_tcn_host.empty() ? nullptr : sc->action_tcn_host.data();
    a.B = sc->batch;
    a.S = S;
    a.T = sc->horizon;
    const char* base = sc->ctx_dev.as<char>();
    a.state_hist = reinterpret_cast<const float*>(base + sc->off_state_hist);
    a.action_hist = reinterpret_cast<const float*>(base + sc->off_action_hist);
    a.ref_states = reinterpret_cast<const float*>(base + sc->off_ref_states);
    a.ref_actions = reinterpret_cast<const float*>(base + sc->off_ref_actions);
    a.masses = sc->has_masses ? reinterpret_cast<const float*>(base + sc->off_masses) : nullptr;
    a.rows = lwm::skyjepa_rows_per_cluster(a);
    return a;
}

lwm_status check_scorer_shape(lwm_scorer* sc, uint32_t B, uint32_t T, uint32_t A) {
    if (!sc->has_context && sc->kind != ScorerKind::Callback)
        return fail(LWM_INVALID_ARGUMENT, "scorer context has not been set");
    if (sc->kind == ScorerKind::Nominal) {
        if (B != sc->batch || T != sc->horizon || A != 4) return fail(LWM_INVALID_ARGUMENT, "nominal candidate shape mismatch");
    } else if (sc->kind == ScorerKind::Lewm) {
        if (B != sc->batch || A != sc->lewm->c.action_dim)
            return fail(LWM_INVALID_ARGUMENT, "LeWM candidate actions [" + std::to_string(B) + ", S, T, " + std::to_string(A) +
                                                  "] do not match batch=" + std::to_string(sc->batch) +
                                                  ", action_dim=" + std::to_string(sc->lewm->c.action_dim));
        if (T < sc->lewm->h)
            return fail(LWM_INVALID_ARGUMENT, "action horizon " + std::to_string(T) + " is shorter than history " +
                                                  std::to_string(sc->lewm->h));
    } else if (sc->kind == ScorerKind::Skyjepa) {
        if (B != sc->batch || T != sc->horizon || A != 4)
            return fail(LWM_INVALID_ARGUMENT, "SkyJEPA candidate actions [" + std::to_string(B) + ", S, " + std::to_string(T) + ", " +
                                                  std::to_string(A) + "] do not match batch=" + std::to_string(sc->batch) +
                                                  ", horizon=" + std::to_string(sc->horizon) + ", action_dim=4");
    } else if (B != sc->batch) {
        return fail(LWM_INVALID_ARGUMENT, "callback scorer batch mismatch");
    }
    return LWM_OK;
}

// CandidateScorer::score_candidates on device buffers (no sampling, no MPPI).
lwm_status score_device(lwm_scorer* sc, const float* cand, uint32_t B, uint32_t S, uint32_t T, uint32_t A, float* scores,
                        float* states) {
    LWM_TRY(check_scorer_shape(sc, B, T, A));
    cudaStream_t stream = sc->ctx->stream;
    if (sc->kind == ScorerKind::Nominal) {
        lwm::NominalArgs a = nominal_args(sc, S);
        a.sample = 0;
        a.cand_in = cand;
        a.scores = scores;
        a.states = states;
        a.mppi = 0;
        LWM_CUDA(lwm::launch_nominal(a, stream));
        sc->ctx->launches += 1;
    } else if (sc->kind == ScorerKind::Skyjepa) {
        lwm::SkyjepaArgs a = skyjepa_args(sc, S);
        a.sample = 0;
        a.cand_in = cand;
        a.scores = scores;
        a.states = states;
        a.mppi = 0;
        int n = 0;
        if (sc->sky_small) {
            LWM_TRY(ensure_small(sc, a, B, S, a.T));
            a.h0_work = sc->h0_work.as<float>();
            LWM_CUDA(lwm::launch_skyjepa_small(a, sc->tc_h0.as<float>(), sc->small_x.as<float>(), stream, &n,
                                               &sc->side));
        } else {
            LWM_CUDA(lwm::launch_skyjepa(a, stream, &n));
        }
        sc->ctx->launches += static_cast<uint64_t>(n);
    } else if (sc->kind == ScorerKind::Lewm) {
        LWM_CUDA(sc->lewm->score(cand, S, T, scores, states, stream));
        sc->ctx->launches += static_cast<uint64_t>(sc->lewm->launches);
    } else {
        if (states) return fail(LWM_UNSUPPORTED, "callback scorers do not predict states");
        const int rc = sc->fn(sc->user, cand, B, S, T, A, scores, stream);
        if (rc != 0) return fail(LWM_INVALID_ARGUMENT, "candidate scorer callback failed with code " + std::to_string(rc));
    }
    return LWM_OK;
}

// ------------------------------------------------------------------ planning

lwm_status deadline_result(lwm_planner* p, uint32_t B, bool use_warm, const char* name, lwm_plan_device_result* out,
                           std::chrono::steady_clock::time_point start) {
    const size_t seq = static_cast<size_t>(B) * p->T * p->A;
    cudaStream_t stream = p->ctx->stream;
    p->elite_iterations = 0;
    int outcome;
    if (use_warm) {
        LWM_CUDA(cudaMemcpyAsync(p->sequence.ptr, p->warm.ptr, seq * 4, cudaMemcpyDeviceToDevice, stream));
        outcome = LWM_DEADLINE_WARM_START;
    } else {
        const float* action = p->kind == PlannerKind::Mppi ? p->mppi.deadline_action
                              : (p->kind == PlannerKind::Cem ? p->cem.deadline_action : p->icem.deadline_action);
        const int32_t has = p->kind == PlannerKind::Mppi ? p->mppi.has_deadline_action
                            : (p->kind == PlannerKind::Cem ? p->cem.has_deadline_action : p->icem.has_deadline_action);
        if (!has)
            return fail(LWM_DEADLINE, std::string(name) +
                                          " deadline reached before any iteration completed and no deadline_action is configured");
        LWM_CUDA(cudaStreamSynchronize(stream));
        float* h = p->staging.as<float>();
        for (size_t i = 0; i < seq; ++i) h[i] = action[i % p->A];
        LWM_CUDA(cudaMemcpyAsync(p->sequence.ptr, h, seq * 4, cudaMemcpyHostToDevice, stream));
        outcome = LWM_DEADLINE_CONFIGURED_ACTION;
    }
    // first_action = sequence[:, 0, :]; scores and indices [B, 1] of zeros
    LWM_CUDA(cudaMemcpy2DAsync(p->first_action.ptr, p->A * 4, p->sequence.ptr, static_cast<size_t>(p->T) * p->A * 4, p->A * 4, B,
                               cudaMemcpyDeviceToDevice, stream));
    LWM_CUDA(cudaMemsetAsync(p->scores.ptr, 0, static_cast<size_t>(B) * 4, stream));
    LWM_CUDA(cudaMemsetAsync(p->best.ptr, 0, static_cast<size_t>(B) * 4, stream));
    LWM_CUDA(cudaStreamSynchronize(stream));  // the staging buffer is reused by the next call
    out->first_action = p->first_action.as<float>();
    out->sequence = p->sequence.as<float>();
    out->scores = p->scores.as<float>();
    out->best_indices = p->best.as<uint32_t>();
    out->batch = B;
    out->scores_cols = 1;
    out->iterations_completed = 0;
    out->deadline_reached = 1;
    out->deadline_outcome = outcome;
    out->elapsed_ns = static_cast<uint64_t>(
        std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - start).count());
    p->last_batch = B;
    p->last_cols = 1;
    p->has_result = true;
    return LWM_OK;
}

// `trace` (iCEM only): IcemPlanner::trace_device (src/planner.rs:900-1010) —
// no deadlines; per iteration the scores of the mean, the best candidate, the
// elite mean and the updated mean go to p->trace ([iterations][4][B]).
lwm_status plan_device_locked(lwm_planner* p, lwm_scorer* sc, const float* injected, lwm_plan_device_result* out,
                              bool trace = false) {
    const auto start = std::chrono::steady_clock::now();
    (void)cudaGetLastError();  // drop a stale non-sticky error of an earlier failed call
    LWM_TRY(validate_planner(p));
    const uint32_t B = sc->batch;
    if (B == 0) return fail(LWM_INVALID_ARGUMENT, "scorer batch is zero (set its context first)");
    LWM_TRY(check_scorer_shape(sc, B, p->T, p->A));
    LWM_TRY(ensure_planner_buffers(p, B));
    cudaStream_t stream = p->ctx->stream;
    const char* name = planner_name(p->kind);
    if (p->kind != PlannerKind::Cem && p->has_warm && p->warm_batch != B)
        return fail(LWM_INVALID_ARGUMENT, std::string(name) + " warm-start shape [" + std::to_string(p->warm_batch) + ", " +
                                              std::to_string(p->T) + ", " + std::to_string(p->A) + "] does not match expected [" +
                                              std::to_string(B) + ", " + std::to_string(p->T) + ", " + std::to_string(p->A) + "]");
    const size_t n = static_cast<size_t>(B) * p->S * p->T * p->A;
    const bool sharded = p->shard_total != 0;
    // a shard reserves the draws of the whole (unsharded) plan, so every
    // shard's Philox indices line up with the single-GPU stream
    const uint64_t per_iter = round_even(sharded ? static_cast<size_t>(B) * p->shard_total * p->T * p->A : n);
    const bool seeded = p->kind == PlannerKind::Mppi ? p->mppi.has_seed
                        : (p->kind == PlannerKind::Cem ? p->cem.has_seed : p->icem.has_seed);
    const uint64_t seed = seeded ? (p->kind == PlannerKind::Mppi ? p->mppi.seed : (p->kind == PlannerKind::Cem ? p->cem.seed : p->icem.seed))
                                 : p->ctx->unseeded_seed;
    const uint64_t reserve = std::max<uint64_t>(per_iter * p->iterations, 1);
    // PlannerRng::reserve_offset (src/planner.rs:1415-1422)
    uint64_t offset;
    if (seeded) {
        uint64_t cur = p->rng_offset.load();
        do {
            if (cur > UINT64_MAX - reserve) return fail(LWM_INVALID_ARGUMENT, "planner CUDA RNG offset overflowed");
        } while (!p->rng_offset.compare_exchange_weak(cur, cur + reserve));
        offset = cur;
    } else {
        offset = p->ctx->unseeded_offset.fetch_add(reserve);
    }
    const int64_t deadline_ns = p->kind == PlannerKind::Mppi ? p->mppi.deadline_ns
                                : (p->kind == PlannerKind::Cem ? p->cem.deadline_ns : p->icem.deadline_ns);
    const float* low = p->bounds.as<float>();
    const float* high = low + LWM_MAX_ACTION_DIM;
    const size_t seq = static_cast<size_t>(B) * p->T * p->A;
    // initial mean and std
    const float* mean_in = (p->kind != PlannerKind::Cem && p->has_warm) ? p->warm.as<float>() : p->zeros.as<float>();
    if (p->kind != PlannerKind::Mppi) {
        LWM_CUDA(cudaMemcpyAsync(p->mean.ptr, mean_in, seq * 4, cudaMemcpyDeviceToDevice, stream));
        LWM_CUDA(cudaMemcpyAsync(p->stdv.ptr, p->std_init.ptr, seq * 4, cudaMemcpyDeviceToDevice, stream));
    }
    uint32_t completed = 0;
    bool deadline_hit = false;
    MppiArgs m = mppi_args(p, p->kind == PlannerKind::Mppi ? p->mppi.temperature : 1.0f);
    if (sharded) {
        m.sample_base = p->shard_base;
        m.shard_tuple = p->shard_tuples.as<float>();
    }
    const uint32_t carried_keep = p->kind == PlannerKind::Icem ? p->icem.keep_elites : 0;
    for (uint32_t it = 0; it < p->iterations; ++it) {
        if (deadline_ns >= 0 && !trace && !sharded) {  // every shard takes the same iterations
            const auto el = std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - start).count();
            if (el >= deadline_ns) {
                deadline_hit = true;
                if (it == 0) return deadline_result(p, B, p->kind != PlannerKind::Cem && p->has_warm, name, out, start);
                break;
            }
        }
        const float* noise = injected ? injected + static_cast<size_t>(it) * n : nullptr;
        const uint64_t it_offset = offset + static_cast<uint64_t>(it) * per_iter;
        if (p->kind == PlannerKind::Mppi && (sc->kind == ScorerKind::Nominal || sc->kind == ScorerKind::Skyjepa)) {
            const float* mean_it = (it == 0) ? mean_in : p->sequence.as<float>();
            if (sc->kind == ScorerKind::Nominal) {
                lwm::NominalArgs a = nominal_args(sc, p->S);
                a.sample = 1;
                a.mean = mean_it;
                a.std = p->std_init.as<float>();
                for (int i = 0; i < 4; ++i) { a.low[i] = planner_low(p)[i]; a.high[i] = planner_high(p)[i]; }
                a.noise = noise;
                a.seed = seed;
                a.offset = it_offset;
                a.sample_base = p->shard_base;
                a.sample_total = p->shard_total;
                a.cand_out = p->cand.as<float>();
                a.scores = p->scores.as<float>();
                a.mppi = 1;
                a.m = m;
                a.m.P = lwm::nominal_blocks_per_vehicle(p->S);
                LWM_CUDA(lwm::launch_nominal(a, stream));
                p->ctx->launches += 1;
            } else {
                lwm::SkyjepaArgs a = skyjepa_args(sc, p->S);
                a.sample = 1;
                a.mean = mean_it;
                a.std = p->std_init.as<float>();
                for (int i = 0; i < 4; ++i) { a.low[i] = planner_low(p)[i]; a.high[i] = planner_high(p)[i]; }
                a.noise = noise;
                a.seed = seed;
                a.offset = it_offset;
                a.sample_base = p->shard_base;
                a.sample_total = p->shard_total;
                a.cand_out = p->cand.as<float>();
                a.scores = p->scores.as<float>();
                a.mppi = 1;
                a.m = m;
                a.m.P = lwm::skyjepa_partials_per_vehicle(p->S, a.rows);
                int launched = 0;
                const char* why = nullptr;
                if (sc->sky_small) {
                    LWM_TRY(ensure_small(sc, a, B, p->S, p->T));
                    a.h0_work = sc->h0_work.as<float>();
                    a.m.P = lwm::skyjepa_small_partials_per_vehicle(p->S);
                    a.low_dev = low;
                    a.high_dev = high;
                    LWM_CUDA(lwm::launch_skyjepa_small(a, sc->tc_h0.as<float>(), sc->small_x.as<float>(), stream,
                                                       &launched, &sc->side));
                } else if (sc->precision == LWM_PRECISION_BF16 && lwm::skyjepa_tc_supported(a, &why)) {
                    LWM_TRY(ensure_tc(sc, a, B, p->S, p->T));
                    a.h0_work = sc->h0_work.as<float>();
                    a.test_wait_polls = p->ctx->faults.wait_polls;
                    a.test_skip_h_arrive = p->ctx->faults.tc_skip_h_arrive;
                    a.m.P = lwm::skyjepa_tc_partials_per_vehicle(p->S);
                    a.low_dev = low;
                    a.high_dev = high;
                    int* err_word = result_err(p, B);
                    LWM_CUDA(cudaMemsetAsync(err_word, 0, 4 * sizeof(int), stream));
                    p->ctx->kernel_timing(a);
                    LWM_CUDA(lwm::launch_skyjepa_tc(a, sc->tc_packed.as<uint8_t>(), sc->tc_h0.as<float>(),
                                                    sc->tc_x.as<uint8_t>(), err_word, stream, &launched, &sc->side));
                } else if (sc->precision == LWM_PRECISION_F32 && lwm::skyjepa_mma_supported(a, &why) &&
                           lwm::skyjepa_mma_fits_device()) {
                    // f32-class accuracy on the tensor cores (split-fp16 operands)
                    LWM_TRY(ensure_mma(sc, a, B, p->S, p->T));
                    a.h0_work = sc->h0_work.as<float>();
                    a.test_wait_polls = p->ctx->faults.wait_polls;
                    a.m.P = lwm::skyjepa_mma_partials_per_vehicle(p->S);
                    a.low_dev = low;
                    a.high_dev = high;
                    // (the input kernel ahead of the rollout clears the error word)
                    p->ctx->kernel_timing(a);
                    LWM_CUDA(lwm::launch_skyjepa_mma(a, sc->mma_packed.as<uint8_t>(), sc->tc_h0.as<float>(),
                                                     sc->tc_x.as<uint8_t>(), sc->mma_xchg.as<uint8_t>(),
                                                     result_err(p, B), stream, &launched, &sc->side));
                } else {
                    p->ctx->kernel_timing(a);
                    LWM_CUDA(lwm::launch_skyjepa(a, stream, &launched));
                }
                p->ctx->launches += static_cast<uint64_t>(launched);
            }
        } else {
            // sample -> score -> reduce (MPPI) / top-k refit (CEM, iCEM)
            lwm::SampleArgs s{};
            s.B = B; s.S = p->S; s.T = p->T; s.A = p->A;
            s.mean = (p->kind == PlannerKind::Mppi) ? ((it == 0) ? mean_in : p->sequence.as<float>()) : p->mean.as<float>();
            s.std = (p->kind == PlannerKind::Mppi) ? p->std_init.as<float>() : p->stdv.as<float>();
            s.low = low;
            s.high = high;
            s.noise = noise;
            s.seed = seed;
            s.offset = it_offset;
            s.sample_base = p->shard_base;
            s.sample_total = p->shard_total;
            s.smooth = 0.0f;
            if (p->kind == PlannerKind::Icem && p->icem.noise_beta != 0.0f) {
                float smooth = p->icem.noise_beta / (p->icem.noise_beta + 1.0f);
                smooth = std::min(std::max(smooth, 0.0f), 0.98f);
                s.smooth = smooth;
            }
            if (p->kind == PlannerKind::Icem && it > 0 && carried_keep > 0) {
                s.carried = p->carried.as<float>();
                s.carried_count = carried_keep;
                s.inject = std::min(carried_keep, (sharded ? p->shard_total : p->S) - 1);
            }
            s.out = p->cand.as<float>();
            float* tr = trace ? p->trace.as<float>() + static_cast<size_t>(it) * 4 * B : nullptr;
            if (tr) LWM_TRY(score_device(sc, p->mean.as<float>(), B, 1, p->T, p->A, tr, nullptr));  // mean_score
            LWM_CUDA(lwm::launch_sample(s, stream));
            p->ctx->launches += 1;
            LWM_TRY(score_device(sc, p->cand.as<float>(), B, p->S, p->T, p->A, p->scores.as<float>(), nullptr));
            if (p->kind == PlannerKind::Mppi) {
                MppiArgs mm = m;
                mm.P = (p->S + 255) / 256;
                LWM_CUDA(lwm::launch_mppi_reduce(mm, p->cand.as<float>(), p->scores.as<float>(), B, p->S, stream));
                p->ctx->launches += 1;
            } else {
                lwm::RefitArgs r{};
                r.S = p->S; r.T = p->T; r.A = p->A;
                r.K = p->kind == PlannerKind::Cem ? p->cem.elites : p->icem.elites;
                r.keep = carried_keep;
                if (!lwm::topk_layout(p->S, r.K, &r.sort_len, &r.select))
                    return fail(LWM_UNSUPPORTED, "elite selection supports at most " + std::to_string(lwm::kMaxElites) +
                                                     " elites");
                r.elite_index = p->elite_idx.as<uint32_t>() + static_cast<size_t>(it) * B * r.K;
                r.scores = p->scores.as<float>();
                r.cand = p->cand.as<float>();
                r.mean = p->mean.as<float>();
                r.std = p->stdv.as<float>();
                r.carried = p->carried.as<float>();
                r.icem = p->kind == PlannerKind::Icem;
                r.return_best = p->kind == PlannerKind::Icem && !p->icem.return_mean;
                r.alpha = p->kind == PlannerKind::Icem ? p->icem.alpha : 0.0f;
                r.min_std = p->kind == PlannerKind::Cem ? p->cem.min_std : p->icem.min_std;
                r.inv_k = static_cast<float>(1.0 / static_cast<double>(r.K));
                r.inv_km1 = static_cast<float>(1.0 / static_cast<double>(r.K - 1));
                r.sequence = p->sequence.as<float>();
                r.first_action = p->first_action.as<float>();
                r.warm_start = p->kind == PlannerKind::Icem ? p->warm.as<float>() : nullptr;
                r.best_index = p->best.as<uint32_t>();
                r.best_score = p->best_score.as<float>();
                r.elite_mean_out = tr ? p->trace_elite.as<float>() : nullptr;
                if (sharded) {
                    // this shard's elites -> every shard's (exchange) -> the merged set, refit as one
                    const uint32_t K = r.K, TA = p->T * p->A, G = p->exchange_shards, W = 2 + TA;
                    const size_t local = static_cast<size_t>(B) * K * W;
                    LWM_TRY(p->elite_local.ensure(local * 4));
                    LWM_TRY(p->elite_gathered.ensure(local * G * 4));
                    LWM_TRY(p->merged_scores.ensure(static_cast<size_t>(B) * G * K * 4));
                    LWM_TRY(p->merged_cand.ensure(static_cast<size_t>(B) * G * K * TA * 4));
                    LWM_TRY(p->merged_index.ensure(static_cast<size_t>(B) * G * K * 4));
                    LWM_CUDA(lwm::launch_elite_tuples(p->scores.as<float>(), p->cand.as<float>(), B, p->S, K, TA,
                                                      p->shard_base, p->elite_local.as<float>(), stream));
                    const int rc = p->exchange(p->exchange_user, p->elite_local.as<float>(), local,
                                               p->elite_gathered.as<float>(), stream);
                    if (rc != 0) return fail(LWM_NCCL_ERROR, "elite exchange callback failed with code " + std::to_string(rc));
                    LWM_CUDA(lwm::launch_elite_merge(p->elite_gathered.as<float>(), G, B, K, TA,
                                                     p->merged_scores.as<float>(), p->merged_cand.as<float>(),
                                                     p->merged_index.as<uint32_t>(), stream));
                    r.S = G * K;
                    if (!lwm::topk_layout(r.S, K, &r.sort_len, &r.select))
                        return fail(LWM_UNSUPPORTED, "elite selection supports at most " +
                                                         std::to_string(lwm::kMaxElites) + " elites");
                    r.scores = p->merged_scores.as<float>();
                    r.cand = p->merged_cand.as<float>();
                    r.index_map = p->merged_index.as<uint32_t>();
                    p->ctx->launches += 2;
                }
                LWM_CUDA(lwm::launch_topk_refit(r, B, stream));
                p->ctx->launches += 1;
                if (tr) {
                    // best_candidate_score, elite_mean_score, updated_mean_score
                    LWM_CUDA(cudaMemcpyAsync(tr + B, p->best_score.ptr, static_cast<size_t>(B) * 4,
                                             cudaMemcpyDeviceToDevice, stream));
                    LWM_TRY(score_device(sc, p->trace_elite.as<float>(), B, 1, p->T, p->A, tr + 2 * B, nullptr));
                    LWM_TRY(score_device(sc, p->mean.as<float>(), B, 1, p->T, p->A, tr + 3 * B, nullptr));
                }
            }
        }
        ++completed;
    }
    p->elite_iterations = p->kind == PlannerKind::Mppi ? 0u : completed;
    if (sharded && p->kind == PlannerKind::Mppi) {
        // the outputs (and the warm start) come from lwm_mppi_combine_device
        out->first_action = nullptr;
        out->sequence = nullptr;
        out->best_indices = nullptr;
        out->scores = p->scores.as<float>();
        out->batch = B;
        out->scores_cols = p->S;
        out->iterations_completed = completed;
        out->deadline_reached = 0;
        out->deadline_outcome = LWM_DEADLINE_NONE;
        out->elapsed_ns = static_cast<uint64_t>(
            std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - start).count());
        p->last_batch = B;
        p->last_cols = p->S;
        return LWM_OK;
    }
    if (p->kind != PlannerKind::Cem) {
        p->has_warm = true;
        p->warm_batch = B;
    }
    out->first_action = p->first_action.as<float>();
    out->sequence = p->sequence.as<float>();
    out->scores = p->scores.as<float>();
    out->best_indices = p->best.as<uint32_t>();
    out->batch = B;
    out->scores_cols = p->S;
    out->iterations_completed = completed;
    out->deadline_reached = deadline_hit ? 1 : 0;
    out->deadline_outcome = LWM_DEADLINE_NONE;
    out->elapsed_ns = static_cast<uint64_t>(
        std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - start).count());
    p->last_batch = B;
    p->last_cols = p->S;
    p->has_result = true;
    return LWM_OK;
}

lwm_status stage_context(lwm_scorer* sc, size_t bytes) {
    if (sc->staged) LWM_CUDA(cudaEventSynchronize(sc->staged));
    LWM_TRY(sc->ctx_host.ensure(bytes));
    LWM_TRY(sc->ctx_dev.ensure(bytes));
    return LWM_OK;
}

lwm_status upload_context(lwm_scorer* sc, size_t bytes) {
    LWM_CUDA(cudaMemcpyAsync(sc->ctx_dev.ptr, sc->ctx_host.ptr, bytes, cudaMemcpyHostToDevice, sc->ctx->stream));
    if (!sc->staged) LWM_CUDA(cudaEventCreateWithFlags(&sc->staged, cudaEventDisableTiming));
    LWM_CUDA(cudaEventRecord(sc->staged, sc->ctx->stream));
    return LWM_OK;
}

size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

void build_tcn_view(const lwm_tcn_config& t, const float* base, size_t& off, lwm::TcnView& v) {
    std::memset(&v, 0, sizeof v);
    v.input_dim = t.input_dim;
    v.levels = t.levels;
    v.k = t.kernel_size;
    uint32_t in = t.input_dim, mx = t.input_dim;
    for (uint32_t l = 0; l < t.levels; ++l) {
        const uint32_t o = t.channels[l];
        lwm::TcnBlockView& b = v.blocks[l];
        b.in = in; b.out = o; b.dil = 1u << l;
        b.w1 = base + off; off += static_cast<size_t>(o) * in * t.kernel_size;
        b.b1 = base + off; off += o;
        b.w2 = base + off; off += static_cast<size_t>(o) * o * t.kernel_size;
        b.b2 = base + off; off += o;
        if (in != o) {
            b.wr = base + off; off += static_cast<size_t>(o) * in;
            b.br = base + off; off += o;
        }
        in = o;
        mx = std::max(mx, o);
    }
    v.out_dim = in;
    v.max_ch = mx;
}

}  // namespace

// ======================================================================= ABI

extern "C" {

const char* lwm_last_error(void) { return g_last_error.c_str(); }
const char* lwm_version(void) { return "lewm-b200 0.1.0 (sm_100a)"; }
int lwm_abi_version(void) { return LWM_ABI_VERSION; }

lwm_status lwm_ctx_create(int device, lwm_ctx** out) {
    if (!out) return fail(LWM_INVALID_ARGUMENT, "output pointer is null");
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) return fail(LWM_CUDA_ERROR, std::string("no CUDA device: ") + cudaGetErrorString(e));
    if (device < 0 || device >= count)
        return fail(LWM_INVALID_ARGUMENT, "CUDA device " + std::to_string(device) + " does not exist (" + std::to_string(count) + " visible)");
    LWM_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop{};
    LWM_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(LWM_UNSUPPORTED, std::string("this library is built for sm_100a (B200); device is ") + prop.name);
    auto* ctx = new lwm_ctx();
    ctx->device = device;
    e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete ctx;
        return fail(LWM_CUDA_ERROR, std::string("cudaStreamCreate failed: ") + cudaGetErrorString(e));
    }
    std::random_device rd;
    ctx->unseeded_seed = (static_cast<uint64_t>(rd()) << 32) ^ rd();
    *out = ctx;
    return LWM_OK;
}

lwm_status lwm_ctx_destroy(lwm_ctx* ctx) {
    if (!ctx) return LWM_OK;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    cudaStreamDestroy(ctx->stream);
    if (ctx->media_err) cudaFreeHost(ctx->media_err);
    if (ctx->kt_begin) cudaEventDestroy(ctx->kt_begin);
    if (ctx->kt_end) cudaEventDestroy(ctx->kt_end);
    delete ctx;
    return LWM_OK;
}

lwm_status lwm_ctx_stream(lwm_ctx* ctx, void** stream_out) {
    if (!ctx || !stream_out) return fail(LWM_INVALID_ARGUMENT, "null argument");
    *stream_out = ctx->stream;
    return LWM_OK;
}

lwm_status lwm_ctx_synchronize(lwm_ctx* ctx) {
    if (!ctx) return fail(LWM_INVALID_ARGUMENT, "null context");
    LWM_CUDA(cudaSetDevice(ctx->device));
    LWM_CUDA(cudaStreamSynchronize(ctx->stream));
    if (ctx->media_err && ctx->media_err[0]) {
        const std::string where = "block " + std::to_string(ctx->media_err[1]) + ", row step " +
                                  std::to_string(ctx->media_err[2]);
        for (int i = 0; i < 4; ++i) ctx->media_err[i] = 0;
        return fail(LWM_CUDA_ERROR, "image preprocessing: a source-row copy never completed (" + where +
                                        "); that launch's output is incomplete");
    }
    return LWM_OK;
}

lwm_status lwm_ctx_set_test_faults(lwm_ctx* ctx, const lwm_test_faults* faults) {
    if (!ctx) return fail(LWM_INVALID_ARGUMENT, "null context");
    if (faults) ctx->faults = *faults;
    else ctx->faults = lwm_test_faults{};
    return LWM_OK;
}

lwm_status lwm_ctx_launch_count(lwm_ctx* ctx, uint64_t* out) {
    if (!ctx || !out) return fail(LWM_INVALID_ARGUMENT, "null argument");
    *out = ctx->launches.load();
    return LWM_OK;
}

lwm_status lwm_ctx_set_kernel_timing(lwm_ctx* ctx, int on) {
    if (!ctx) return fail(LWM_INVALID_ARGUMENT, "null argument");
    LWM_CUDA(cudaSetDevice(ctx->device));
    if (on && !ctx->kt_begin) {
        LWM_CUDA(cudaEventCreate(&ctx->kt_begin));
        LWM_CUDA(cudaEventCreate(&ctx->kt_end));
    }
    ctx->kt_on = on != 0;
    ctx->kt_valid = false;
    return LWM_OK;
}

lwm_status lwm_ctx_kernel_time_ms(lwm_ctx* ctx, float* ms_out) {
    if (!ctx || !ms_out) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (!ctx->kt_on || !ctx->kt_valid) return fail(LWM_INVALID_ARGUMENT, "no rollout launch timed");
    LWM_CUDA(cudaSetDevice(ctx->device));
    LWM_CUDA(cudaEventSynchronize(ctx->kt_end));
    LWM_CUDA(cudaEventElapsedTime(ms_out, ctx->kt_begin, ctx->kt_end));
    return LWM_OK;
}

void lwm_mppi_config_default(uint32_t horizon, uint32_t samples, uint32_t action_dim, lwm_mppi_config* c) {
    std::memset(c, 0, sizeof(*c));
    c->horizon = horizon;
    c->samples = samples;
    c->iterations = 1;
    c->action_dim = action_dim;
    for (int i = 0; i < LWM_MAX_ACTION_DIM; ++i) { c->bounds_low[i] = -1.0f; c->bounds_high[i] = 1.0f; }
    c->noise_std = 1.0f;
    c->temperature = 1.0f;
    c->deadline_ns = -1;
}

void lwm_cem_config_default(uint32_t horizon, uint32_t samples, uint32_t elites, uint32_t action_dim, lwm_cem_config* c) {
    std::memset(c, 0, sizeof(*c));
    c->horizon = horizon;
    c->samples = samples;
    c->elites = elites;
    c->iterations = 4;
    c->action_dim = action_dim;
    for (int i = 0; i < LWM_MAX_ACTION_DIM; ++i) { c->bounds_low[i] = -1.0f; c->bounds_high[i] = 1.0f; }
    c->init_std = 1.0f;
    c->min_std = 1e-3f;
    c->deadline_ns = -1;
}

void lwm_icem_config_default(uint32_t horizon, uint32_t samples, uint32_t elites, uint32_t action_dim, lwm_icem_config* c) {
    std::memset(c, 0, sizeof(*c));
    c->horizon = horizon;
    c->samples = samples;
    c->elites = elites;
    c->keep_elites = elites;
    c->iterations = 4;
    c->noise_beta = 2.0f;
    c->alpha = 0.1f;
    c->action_dim = action_dim;
    for (int i = 0; i < LWM_MAX_ACTION_DIM; ++i) { c->bounds_low[i] = -1.0f; c->bounds_high[i] = 1.0f; }
    c->init_std = 1.0f;
    c->min_std = 1e-3f;
    c->return_mean = 1;
    c->deadline_ns = -1;
}

static lwm_status make_planner(lwm_ctx* ctx, PlannerKind kind, lwm_planner** out) {
    if (!ctx || !out) return fail(LWM_INVALID_ARGUMENT, "null argument");
    auto* p = new lwm_planner();
    p->ctx = ctx;
    p->kind = kind;
    *out = p;
    return LWM_OK;
}

lwm_status lwm_mppi_create(lwm_ctx* ctx, const lwm_mppi_config* cfg, lwm_planner** out) {
    if (!cfg) return fail(LWM_INVALID_ARGUMENT, "null config");
    LWM_TRY(validate_mppi(*cfg));
    LWM_TRY(make_planner(ctx, PlannerKind::Mppi, out));
    (*out)->mppi = *cfg;
    (*out)->T = cfg->horizon; (*out)->S = cfg->samples; (*out)->A = cfg->action_dim; (*out)->iterations = cfg->iterations;
    return LWM_OK;
}

lwm_status lwm_cem_create(lwm_ctx* ctx, const lwm_cem_config* cfg, lwm_planner** out) {
    if (!cfg) return fail(LWM_INVALID_ARGUMENT, "null config");
    LWM_TRY(validate_cem(*cfg));
    LWM_TRY(make_planner(ctx, PlannerKind::Cem, out));
    (*out)->cem = *cfg;
    (*out)->T = cfg->horizon; (*out)->S = cfg->samples; (*out)->A = cfg->action_dim; (*out)->iterations = cfg->iterations;
    return LWM_OK;
}

lwm_status lwm_icem_create(lwm_ctx* ctx, const lwm_icem_config* cfg, lwm_planner** out) {
    if (!cfg) return fail(LWM_INVALID_ARGUMENT, "null config");
    LWM_TRY(validate_icem(*cfg));
    LWM_TRY(make_planner(ctx, PlannerKind::Icem, out));
    (*out)->icem = *cfg;
    (*out)->T = cfg->horizon; (*out)->S = cfg->samples; (*out)->A = cfg->action_dim; (*out)->iterations = cfg->iterations;
    return LWM_OK;
}

lwm_status lwm_planner_destroy(lwm_planner* p) {
    if (!p) return LWM_OK;
    cudaSetDevice(p->ctx->device);
    cudaStreamSynchronize(p->ctx->stream);
    for (DevBuf* b : {&p->bounds, &p->zeros, &p->std_init, &p->mean, &p->stdv, &p->cand, &p->scores, &p->partials, &p->counters,
                      &p->sequence, &p->first_action, &p->warm, &p->best, &p->best_score, &p->carried, &p->noise_tmp,
                      &p->shard_tuples, &p->trace, &p->trace_elite, &p->elite_local, &p->elite_gathered,
                      &p->merged_scores, &p->merged_cand, &p->merged_index, &p->elite_idx, &p->results})
        b->release();
    p->staging.release();
    delete p;
    return LWM_OK;
}

lwm_status lwm_planner_set_warm_start(lwm_planner* p, const float* sequence, uint32_t batch, uint32_t horizon,
                                      uint32_t action_dim) {
    if (!p || !sequence) return fail(LWM_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> lock(p->mu);
    if (p->kind == PlannerKind::Cem) return fail(LWM_INVALID_ARGUMENT, "CEM planners have no warm start");
    if (horizon != p->T || action_dim != p->A || batch == 0)
        return fail(LWM_INVALID_ARGUMENT, std::string(planner_name(p->kind)) + " warm-start shape [" + std::to_string(batch) + ", " +
                                              std::to_string(horizon) + ", " + std::to_string(action_dim) + "] does not match expected [B, " +
                                              std::to_string(p->T) + ", " + std::to_string(p->A) + "]");
    LWM_CUDA(cudaSetDevice(p->ctx->device));
    LWM_TRY(ensure_planner_buffers(p, batch));
    const size_t bytes = static_cast<size_t>(batch) * horizon * action_dim * 4;
    LWM_CUDA(cudaMemcpyAsync(p->warm.ptr, sequence, bytes, cudaMemcpyHostToDevice, p->ctx->stream));
    LWM_CUDA(cudaStreamSynchronize(p->ctx->stream));
    p->has_warm = true;
    p->warm_batch = batch;
    return LWM_OK;
}

lwm_status lwm_planner_set_warm_start_device(lwm_planner* p, const float* sequence, uint32_t batch, uint32_t horizon,
                                             uint32_t action_dim) {
    if (!p || !sequence) return fail(LWM_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> lock(p->mu);
    if (p->kind == PlannerKind::Cem) return fail(LWM_INVALID_ARGUMENT, "CEM planners have no warm start");
    if (horizon != p->T || action_dim != p->A || batch == 0)
        return fail(LWM_INVALID_ARGUMENT, std::string(planner_name(p->kind)) + " warm-start shape [" + std::to_string(batch) + ", " +
                                              std::to_string(horizon) + ", " + std::to_string(action_dim) + "] does not match expected [B, " +
                                              std::to_string(p->T) + ", " + std::to_string(p->A) + "]");
    LWM_CUDA(cudaSetDevice(p->ctx->device));
    LWM_TRY(ensure_planner_buffers(p, batch));
    const size_t bytes = static_cast<size_t>(batch) * horizon * action_dim * 4;
    LWM_CUDA(cudaMemcpyAsync(p->warm.ptr, sequence, bytes, cudaMemcpyDeviceToDevice, p->ctx->stream));
    p->has_warm = true;
    p->warm_batch = batch;
    return LWM_OK;
}

lwm_status lwm_fleet_control_step_device(lwm_ctx* ctx, const lwm_fleet_step* st) {
    if (!ctx || !st) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (!st->state || !st->state_history || !st->action_history || !st->reference_states || !st->reference_actions)
        return fail(LWM_INVALID_ARGUMENT, "fleet step buffers must be device pointers, not null");
    if (st->history < 2 || st->horizon == 0 || st->horizon > lwm::kMaxHorizon)
        return fail(LWM_INVALID_ARGUMENT, "fleet step needs history >= 2 and horizon in [1, 64]");
    if (st->reference_kind < 0 || st->reference_kind > 2) return fail(LWM_INVALID_ARGUMENT, "unknown reference kind");
    if (!std::isfinite(st->dt) || st->dt <= 0.0f || !(st->period > 0.0f))
        return fail(LWM_INVALID_ARGUMENT, "fleet step dt and period must be positive");
    if (st->last_action && st->last_action_stride < 4) return fail(LWM_INVALID_ARGUMENT, "last_action_stride must be >= 4");
    LWM_CUDA(cudaSetDevice(ctx->device));
    LWM_CUDA(lwm::launch_fleet_control(*st, ctx->stream));
    ctx->launches += st->batch ? 1 : 0;
    return LWM_OK;
}

lwm_status lwm_rotor_plant_step_device(lwm_ctx* ctx, const lwm_domain* domains, float* states, float* motors,
                                       const float* commands, uint32_t stride, uint32_t batch, float dt,
                                       uint32_t substeps) {
    if (!ctx || !domains || !states || !motors || !commands) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (stride < 4) return fail(LWM_INVALID_ARGUMENT, "command_stride must be >= 4");
    if (!std::isfinite(dt) || dt <= 0.0f) return fail(LWM_INVALID_ARGUMENT, "plant dt must be finite and positive");
    LWM_CUDA(cudaSetDevice(ctx->device));
    LWM_CUDA(lwm::launch_plant(domains, states, motors, commands, stride, batch, dt, substeps, ctx->stream));
    ctx->launches += batch ? 1 : 0;
    return LWM_OK;
}

lwm_status lwm_scorer_skyjepa_context_device(lwm_scorer* s, float** state_history, float** action_history,
                                             float** reference_states, float** reference_actions) {
    if (!s || s->kind != ScorerKind::Skyjepa) return fail(LWM_INVALID_ARGUMENT, "not a SkyJEPA scorer");
    if (!s->batch || !s->ctx_dev.ptr) return fail(LWM_INVALID_ARGUMENT, "set the scorer's context first");
    char* base = s->ctx_dev.as<char>();
    if (state_history) *state_history = reinterpret_cast<float*>(base + s->off_state_hist);
    if (action_history) *action_history = reinterpret_cast<float*>(base + s->off_action_hist);
    if (reference_states) *reference_states = reinterpret_cast<float*>(base + s->off_ref_states);
    if (reference_actions) *reference_actions = reinterpret_cast<float*>(base + s->off_ref_actions);
    return LWM_OK;
}

lwm_status lwm_planner_clear_warm_start(lwm_planner* p) {
    if (!p) return fail(LWM_INVALID_ARGUMENT, "null planner");
    std::lock_guard<std::mutex> lock(p->mu);
    p->has_warm = false;
    p->warm_batch = 0;
    return LWM_OK;
}

lwm_status lwm_planner_warm_start(lwm_planner* p, float* out, size_t capacity, uint32_t* batch_out) {
    if (!p || !batch_out) return fail(LWM_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> lock(p->mu);
    *batch_out = 0;
    if (!p->has_warm) return LWM_OK;
    const size_t n = static_cast<size_t>(p->warm_batch) * p->T * p->A;
    if (!out || capacity < n) return fail(LWM_INVALID_ARGUMENT, "warm-start output buffer too small");
    LWM_CUDA(cudaSetDevice(p->ctx->device));
    LWM_CUDA(cudaMemcpyAsync(out, p->warm.ptr, n * 4, cudaMemcpyDeviceToHost, p->ctx->stream));
    LWM_CUDA(cudaStreamSynchronize(p->ctx->stream));
    *batch_out = p->warm_batch;
    return LWM_OK;
}

lwm_status lwm_planner_reset_rng(lwm_planner* p) {
    if (!p) return fail(LWM_INVALID_ARGUMENT, "null planner");
    p->rng_offset.store(0);
    return LWM_OK;
}

lwm_status lwm_planner_rng_offset(lwm_planner* p, uint64_t* out) {
    if (!p || !out) return fail(LWM_INVALID_ARGUMENT, "null argument");
    *out = p->rng_offset.load();
    return LWM_OK;
}

lwm_status lwm_planner_elite_indices(lwm_planner* p, uint32_t* out, size_t capacity, uint32_t* iterations_out,
                                     uint32_t* batch_out, uint32_t* elites_out) {
    if (!p || !iterations_out || !batch_out || !elites_out) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (p->kind == PlannerKind::Mppi) return fail(LWM_INVALID_ARGUMENT, "MPPI selects no elites");
    std::lock_guard<std::mutex> lock(p->mu);
    const uint32_t K = p->kind == PlannerKind::Cem ? p->cem.elites : p->icem.elites;
    const uint32_t its = p->has_result ? p->elite_iterations : 0u, B = p->has_result ? p->last_batch : 0u;
    *iterations_out = its;
    *batch_out = B;
    *elites_out = K;
    const size_t n = static_cast<size_t>(its) * B * K;
    if (n == 0) return LWM_OK;
    if (!out || capacity < n) return fail(LWM_INVALID_ARGUMENT, "elite index output buffer too small");
    LWM_CUDA(cudaSetDevice(p->ctx->device));
    LWM_CUDA(cudaMemcpyAsync(out, p->elite_idx.ptr, n * 4, cudaMemcpyDeviceToHost, p->ctx->stream));
    LWM_CUDA(cudaStreamSynchronize(p->ctx->stream));
    return LWM_OK;
}

lwm_status lwm_planner_last_candidates(lwm_planner* p, const float** cand, uint32_t* samples_out) {
    if (!p || !cand || !samples_out) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (!p->has_result) return fail(LWM_INVALID_ARGUMENT, "planner has not planned yet");
    *cand = p->cand.as<float>();
    *samples_out = p->S;
    return LWM_OK;
}

// ----------------------------------------------------------------- scorers

static lwm_scorer* new_scorer(lwm_ctx* ctx, ScorerKind kind) {
    auto* s = new lwm_scorer();
    s->ctx = ctx;
    s->kind = kind;
    return s;
}

lwm_status lwm_scorer_nominal_create(lwm_ctx* ctx, const lwm_nominal_scorer_config* cfg, lwm_scorer** out) {
    if (!ctx || !cfg || !out) return fail(LWM_INVALID_ARGUMENT, "null argument");
    LWM_TRY(validate_cost(cfg->cost));
    if (!finite(cfg->trim_scale) || cfg->trim_scale <= 0.0f) return fail(LWM_INVALID_ARGUMENT, "invalid nominal scorer context");
    if (!finite(cfg->dt) || cfg->dt <= 0.0f || cfg->substeps == 0)
        return fail(LWM_INVALID_ARGUMENT, "invalid nominal physics rollout shape or timestep");
    LWM_TRY(validate_domain(cfg->domain));
    lwm_scorer* s = new_scorer(ctx, ScorerKind::Nominal);
    s->nominal = *cfg;
    *out = s;
    return LWM_OK;
}

lwm_status lwm_scorer_nominal_set_context(lwm_scorer* s, uint32_t B, uint32_t T, const float* initial, const float* motors,
                                          const float* ref_states, const float* ref_actions, const lwm_domain* domains) {
    if (!s || s->kind != ScorerKind::Nominal) return fail(LWM_INVALID_ARGUMENT, "not a nominal scorer");
    if (!initial || !motors || !ref_states || !ref_actions || B == 0 || T == 0)
        return fail(LWM_INVALID_ARGUMENT, "invalid nominal scorer context");
    if (T > lwm::kMaxHorizon) return fail(LWM_UNSUPPORTED, "horizon exceeds the supported maximum of 64");
    if (domains)
        for (uint32_t b = 0; b < B; ++b) LWM_TRY(validate_domain(domains[b]));
    std::lock_guard<std::mutex> lock(s->mu);
    LWM_CUDA(cudaSetDevice(s->ctx->device));
    size_t off = 0;
    s->off_initial = off; off = align256(off + static_cast<size_t>(B) * 18 * 4);
    s->off_motors = off; off = align256(off + static_cast<size_t>(B) * 4 * 4);
    s->off_ref_states = off; off = align256(off + static_cast<size_t>(B) * T * 18 * 4);
    s->off_ref_actions = off; off = align256(off + static_cast<size_t>(B) * T * 4 * 4);
    s->off_domains = off; off = align256(off + static_cast<size_t>(B) * sizeof(lwm::DomainParams));
    LWM_TRY(stage_context(s, off));
    char* h = s->ctx_host.as<char>();
    std::memcpy(h + s->off_initial, initial, static_cast<size_t>(B) * 18 * 4);
    std::memcpy(h + s->off_motors, motors, static_cast<size_t>(B) * 4 * 4);
    std::memcpy(h + s->off_ref_states, ref_states, static_cast<size_t>(B) * T * 18 * 4);
    std::memcpy(h + s->off_ref_actions, ref_actions, static_cast<size_t>(B) * T * 4 * 4);
    auto* dp = reinterpret_cast<lwm::DomainParams*>(h + s->off_domains);
    for (uint32_t b = 0; b < B; ++b) dp[b] = domain_params(domains ? domains[b] : s->nominal.domain);
    LWM_TRY(upload_context(s, off));
    s->batch = B;
    s->horizon = T;
    s->has_context = true;
    return LWM_OK;
}

lwm_status lwm_scorer_skyjepa_create(lwm_ctx* ctx, const lwm_skyjepa_config* cfg, const float* weights, size_t count,
                                     const float* state_mean, const float* state_std, const float* action_mean,
                                     const float* action_std, const lwm_tracking_cost* cost, float dt, lwm_scorer** out) {
    if (!ctx || !cfg || !weights || !state_mean || !state_std || !action_mean || !action_std || !cost || !out)
        return fail(LWM_INVALID_ARGUMENT, "null argument");
    const size_t need = lwm_skyjepa_weight_count(cfg);
    if (need == 0) return fail(LWM_INVALID_ARGUMENT, "invalid SkyJEPA configuration");
    if (count != need)
        return fail(LWM_INVALID_ARGUMENT, "SkyJEPA weight blob has " + std::to_string(count) + " values, expected " + std::to_string(need));
    LWM_TRY(validate_cost(*cost));
    if (!finite(dt) || dt <= 0.0f) return fail(LWM_INVALID_ARGUMENT, "SkyJEPA control dt must be finite and positive");
    // validate_stats (src/models/skyjepa/control.rs:454-472)
    for (int i = 0; i < 18; ++i)
        if (!finite(state_mean[i]) || !finite(state_std[i]) || state_std[i] <= 0.0f)
            return fail(LWM_INVALID_ARGUMENT, "SkyJEPA state normalization is non-finite or has non-positive std");
    for (int i = 0; i < 4; ++i)
        if (!finite(action_mean[i]) || !finite(action_std[i]) || action_std[i] <= 0.0f)
            return fail(LWM_INVALID_ARGUMENT, "SkyJEPA action normalization is non-finite or has non-positive std");
    if (cfg->prober_hidden_layers > 5) return fail(LWM_UNSUPPORTED, "prober hidden_layers must be at most 5");
    LWM_CUDA(cudaSetDevice(ctx->device));
    lwm_scorer* s = new_scorer(ctx, ScorerKind::Skyjepa);
    s->sky = *cfg;
    s->cost = *cost;
    s->dt = dt;
    lwm_status st = s->weights.ensure(need * 4);
    if (st != LWM_OK) { delete s; return st; }
    cudaError_t e = cudaMemcpy(s->weights.ptr, weights, need * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) { s->weights.release(); delete s; return fail(LWM_CUDA_ERROR, cudaGetErrorString(e)); }
    lwm::SkyjepaArgs& a = s->sky_args;
    std::memset(&a, 0, sizeof a);
    const float* base = s->weights.as<float>();
    size_t off = 0;
    build_tcn_view(cfg->state_encoder, base, off, a.state_tcn);
    const uint32_t H = cfg->latent_dim;
    a.proj_w = base + off; off += static_cast<size_t>(H) * a.state_tcn.out_dim;
    a.proj_b = base + off; off += H;
    const size_t tcn_off = off;
    build_tcn_view(cfg->action_encoder, base, off, a.action_tcn);
    s->action_tcn_host.assign(weights + tcn_off, weights + off);
    const uint32_t E = a.action_tcn.out_dim;
    a.w_ih = base + off; off += static_cast<size_t>(3) * H * E;
    a.w_hh = base + off; off += static_cast<size_t>(3) * H * H;
    a.b_ih = base + off; off += static_cast<size_t>(3) * H;
    a.b_hh = base + off; off += static_cast<size_t>(3) * H;
    const uint32_t hid = cfg->prober_hidden_dim;
    a.p_in_w = base + off; off += static_cast<size_t>(hid) * H;
    a.p_in_b = base + off; off += hid;
    for (uint32_t i = 0; i + 1 < cfg->prober_hidden_layers; ++i) {
        a.p_hid_w[i] = base + off; off += static_cast<size_t>(hid) * hid;
        a.p_hid_b[i] = base + off; off += hid;
    }
    a.p_out_w = base + off; off += static_cast<size_t>(15) * hid;
    a.p_out_b = base + off; off += 15;
    a.A = cfg->action_dim;
    a.Hs = cfg->history_steps;
    a.H = H;
    a.E = E;
    a.hid = hid;
    a.prober_layers = cfg->prober_hidden_layers;
    for (int i = 0; i < 18; ++i) { a.state_mean[i] = state_mean[i]; a.state_std[i] = state_std[i]; }
    for (int i = 0; i < 4; ++i) { a.action_mean[i] = action_mean[i]; a.action_std[i] = action_std[i]; }
    a.mass = static_cast<float>(cfg->kinematics.mass);
    a.gravity = static_cast<float>(cfg->kinematics.gravity);
    a.hover_throttle = static_cast<float>(cfg->kinematics.hover_throttle);
    a.rotor_forces = cfg->kinematics.action_space == LWM_ACTION_SPACE_ROTOR_FORCES;
    a.dt = dt;
    a.cost = cost_params(*cost);
    a.T = 1;
    const char* why = nullptr;
    const char* why_small = nullptr;
    if (!lwm::skyjepa_supported(a, &why)) {
        if (!lwm::skyjepa_small_supported(a, &why_small)) {
            s->weights.release();
            delete s;
            return fail(LWM_UNSUPPORTED, std::string("SkyJEPA configuration not supported: ") + why + "; " + why_small);
        }
        s->sky_small = true;
    }
    *out = s;
    return LWM_OK;
}

lwm_status lwm_scorer_skyjepa_set_context(lwm_scorer* s, uint32_t B, uint32_t T, const float* state_hist,
                                          const float* action_hist, const float* ref_states, const float* ref_actions) {
    return lwm_scorer_skyjepa_set_context_ex(s, B, T, state_hist, action_hist, ref_states, ref_actions, nullptr);
}

lwm_status lwm_scorer_skyjepa_set_context_ex(lwm_scorer* s, uint32_t B, uint32_t T, const float* state_hist,
                                             const float* action_hist, const float* ref_states,
                                             const float* ref_actions, const float* masses) {
    if (!s || s->kind != ScorerKind::Skyjepa) return fail(LWM_INVALID_ARGUMENT, "not a SkyJEPA scorer");
    if (!state_hist || !action_hist || !ref_states || !ref_actions || B == 0 || T == 0)
        return fail(LWM_INVALID_ARGUMENT, "invalid SkyJEPA control shapes");
    if (masses)
        for (uint32_t b = 0; b < B; ++b)
            if (!(masses[b] > 0.0f) || !std::isfinite(masses[b]))
                return fail(LWM_INVALID_ARGUMENT, "vehicle mass " + std::to_string(b) + " must be finite and positive");
    lwm::SkyjepaArgs probe = s->sky_args;
    probe.T = T;
    const char* why = nullptr;
    if (!(s->sky_small ? lwm::skyjepa_small_supported(probe, &why) : lwm::skyjepa_supported(probe, &why)))
        return fail(LWM_UNSUPPORTED, why);
    std::lock_guard<std::mutex> lock(s->mu);
    LWM_CUDA(cudaSetDevice(s->ctx->device));
    const uint32_t Hs = s->sky.history_steps;
    size_t off = 0;
    s->off_state_hist = off; off = align256(off + static_cast<size_t>(B) * Hs * 18 * 4);
    s->off_action_hist = off; off = align256(off + static_cast<size_t>(B) * (Hs - 1) * 4 * 4);
    s->off_ref_states = off; off = align256(off + static_cast<size_t>(B) * T * 18 * 4);
    s->off_ref_actions = off; off = align256(off + static_cast<size_t>(B) * T * 4 * 4);
    s->off_masses = off; off = align256(off + (masses ? static_cast<size_t>(B) * 4 : 0));
    LWM_TRY(stage_context(s, off));
    char* h = s->ctx_host.as<char>();
    if (masses) std::memcpy(h + s->off_masses, masses, static_cast<size_t>(B) * 4);
    std::memcpy(h + s->off_state_hist, state_hist, static_cast<size_t>(B) * Hs * 18 * 4);
    std::memcpy(h + s->off_action_hist, action_hist, static_cast<size_t>(B) * (Hs - 1) * 4 * 4);
    std::memcpy(h + s->off_ref_states, ref_states, static_cast<size_t>(B) * T * 18 * 4);
    std::memcpy(h + s->off_ref_actions, ref_actions, static_cast<size_t>(B) * T * 4 * 4);
    LWM_TRY(upload_context(s, off));
    s->batch = B;
    s->horizon = T;
    s->has_masses = masses != nullptr;
    s->has_context = true;
    return LWM_OK;
}

lwm_status lwm_scorer_lewm_create(lwm_ctx* ctx, const lwm_lewm_config* cfg, const float* weights, size_t count,
                                  lwm_scorer** out) {
    if (!ctx || !cfg || !weights || !out) return fail(LWM_INVALID_ARGUMENT, "null argument");
    const char* why = nullptr;
    if (!lwm::lewm_config_valid(*cfg, &why)) return fail(LWM_INVALID_ARGUMENT, why);
    const size_t n = lwm::lewm_walk(*cfg, nullptr, nullptr);
    if (count != n)
        return fail(LWM_INVALID_ARGUMENT, "LeWM weight blob has " + std::to_string(count) + " floats, expected " +
                                              std::to_string(n));
    LWM_CUDA(cudaSetDevice(ctx->device));
    auto model = std::make_unique<lwm::LewmModel>();
    model->c = *cfg;
    LWM_CUDA(cudaMalloc(&model->blob, n * sizeof(float)));
    LWM_CUDA(cudaMemcpy(model->blob, weights, n * sizeof(float), cudaMemcpyHostToDevice));
    lwm::lewm_walk(*cfg, model->blob, &model->w);
    LWM_CUDA(model->fuse_vit_qkv());
    LWM_CUDA(model->fold_v_out());
    lwm_scorer* s = new_scorer(ctx, ScorerKind::Lewm);
    s->lewm = std::move(model);
    *out = s;
    return LWM_OK;
}

static lwm_status lewm_set_context(lwm_scorer* s, uint32_t B, uint32_t h, uint32_t history, const float* emb,
                                   const float* goal, cudaMemcpyKind kind) {
    if (!s || s->kind != ScorerKind::Lewm) return fail(LWM_INVALID_ARGUMENT, "not a LeWM scorer");
    if (!emb || !goal || B == 0 || h == 0) return fail(LWM_INVALID_ARGUMENT, "invalid LeWM context shapes");
    lwm::LewmModel& m = *s->lewm;
    const uint32_t window = history ? history : h;
    if (window > m.c.num_frames)
        return fail(LWM_INVALID_ARGUMENT, "rollout window " + std::to_string(window) + " exceeds predictor.num_frames " +
                                              std::to_string(m.c.num_frames));
    std::lock_guard<std::mutex> lock(s->mu);
    LWM_CUDA(cudaSetDevice(s->ctx->device));
    const size_t D = m.c.embed_dim;
    const size_t need = static_cast<size_t>(B) * h * D;
    LWM_CUDA(m.ensure_context(B, h, false, s->ctx->stream));
    LWM_CUDA(cudaMemcpyAsync(m.emb, emb, need * sizeof(float), kind, s->ctx->stream));
    LWM_CUDA(cudaMemcpyAsync(m.goal, goal, static_cast<size_t>(B) * D * sizeof(float), kind, s->ctx->stream));
    if (kind == cudaMemcpyHostToDevice) LWM_CUDA(cudaStreamSynchronize(s->ctx->stream));  // host arrays may go away
    m.B = B;
    m.h = h;
    m.history = window;
    s->batch = B;
    s->has_context = true;
    return LWM_OK;
}

lwm_status lwm_scorer_lewm_set_context(lwm_scorer* s, uint32_t B, uint32_t h, uint32_t history, const float* emb,
                                       const float* goal) {
    return lewm_set_context(s, B, h, history, emb, goal, cudaMemcpyHostToDevice);
}

lwm_status lwm_scorer_lewm_set_context_device(lwm_scorer* s, uint32_t B, uint32_t h, uint32_t history,
                                              const float* emb, const float* goal) {
    return lewm_set_context(s, B, h, history, emb, goal, cudaMemcpyDeviceToDevice);
}

lwm_status lwm_lewm_encode_vector_device(lwm_scorer* s, const float* obs, uint32_t n, float* out) {
    if (!s || s->kind != ScorerKind::Lewm || !obs || !out || n == 0) return fail(LWM_INVALID_ARGUMENT, "invalid encode arguments");
    if (s->lewm->c.encoder != LWM_ENCODER_VECTOR_MLP)
        return fail(LWM_INVALID_ARGUMENT, "encode_vector called on non-vector observation encoder");
    std::lock_guard<std::mutex> lock(s->mu);
    LWM_CUDA(cudaSetDevice(s->ctx->device));
    LWM_CUDA(s->lewm->encode_vector(obs, n, out, s->ctx->stream));
    s->ctx->launches += static_cast<uint64_t>(s->lewm->launches);
    return LWM_OK;
}

lwm_status lwm_lewm_encode_pixels_device(lwm_scorer* s, const float* pixels, uint32_t n, float* out) {
    if (!s || s->kind != ScorerKind::Lewm || !pixels || !out || n == 0)
        return fail(LWM_INVALID_ARGUMENT, "invalid encode arguments");
    if (s->lewm->c.encoder != LWM_ENCODER_VIT)
        return fail(LWM_INVALID_ARGUMENT, "encode_pixels called on non-image observation encoder");
    std::lock_guard<std::mutex> lock(s->mu);
    LWM_CUDA(cudaSetDevice(s->ctx->device));
    LWM_CUDA(s->lewm->encode_pixels(pixels, n, out, s->ctx->stream));
    s->ctx->launches += static_cast<uint64_t>(s->lewm->launches);
    return LWM_OK;
}

lwm_status lwm_scorer_skyjepa_set_precision(lwm_scorer* s, int32_t precision) {
    if (!s || s->kind != ScorerKind::Skyjepa) return fail(LWM_INVALID_ARGUMENT, "not a SkyJEPA scorer");
    if (precision != LWM_PRECISION_F32 && precision != LWM_PRECISION_BF16 && precision != LWM_PRECISION_F32_CUDA_CORE)
        return fail(LWM_INVALID_ARGUMENT, "unknown precision " + std::to_string(precision));
    std::lock_guard<std::mutex> lock(s->mu);
    s->precision = precision;
    return LWM_OK;
}

lwm_status lwm_scorer_lewm_set_precision(lwm_scorer* s, int32_t precision) {
    if (!s || s->kind != ScorerKind::Lewm) return fail(LWM_INVALID_ARGUMENT, "not a LeWM scorer");
    if (precision != LWM_PRECISION_F32 && precision != LWM_PRECISION_BF16)
        return fail(LWM_INVALID_ARGUMENT, "unknown precision " + std::to_string(precision));
    std::lock_guard<std::mutex> lock(s->mu);
    LWM_CUDA(cudaSetDevice(s->ctx->device));
    LWM_CUDA(s->lewm->set_precision(precision, s->ctx->stream));
    s->precision = precision;
    return LWM_OK;
}

lwm_status lwm_scorer_callback_create(lwm_ctx* ctx, uint32_t batch, lwm_score_fn fn, void* user, lwm_scorer** out) {
    if (!ctx || !fn || !out || batch == 0) return fail(LWM_INVALID_ARGUMENT, "invalid callback scorer arguments");
    lwm_scorer* s = new_scorer(ctx, ScorerKind::Callback);
    s->batch = batch;
    s->fn = fn;
    s->user = user;
    *out = s;
    return LWM_OK;
}

lwm_status lwm_scorer_score_device(lwm_scorer* s, const float* cand, uint32_t B, uint32_t S, uint32_t T, uint32_t A,
                                   float* scores) {
    if (!s || !cand || !scores || S == 0) return fail(LWM_INVALID_ARGUMENT, "invalid score arguments");
    std::lock_guard<std::mutex> lock(s->mu);
    LWM_CUDA(cudaSetDevice(s->ctx->device));
    return score_device(s, cand, B, S, T, A, scores, nullptr);
}

lwm_status lwm_scorer_predict_device(lwm_scorer* s, const float* cand, uint32_t B, uint32_t S, uint32_t T, float* states) {
    if (!s || !cand || !states || S == 0) return fail(LWM_INVALID_ARGUMENT, "invalid predict arguments");
    if (s->kind == ScorerKind::Callback) return fail(LWM_UNSUPPORTED, "callback scorers do not predict states");
    std::lock_guard<std::mutex> lock(s->mu);
    LWM_CUDA(cudaSetDevice(s->ctx->device));
    DevBuf tmp;
    LWM_TRY(tmp.ensure(static_cast<size_t>(B) * S * 4));
    const uint32_t A = s->kind == ScorerKind::Lewm ? s->lewm->c.action_dim : 4;
    lwm_status st = score_device(s, cand, B, S, T, A, tmp.as<float>(), states);
    cudaStreamSynchronize(s->ctx->stream);
    tmp.release();
    return st;
}

lwm_status lwm_scorer_destroy(lwm_scorer* s) {
    if (!s) return LWM_OK;
    cudaSetDevice(s->ctx->device);
    cudaStreamSynchronize(s->ctx->stream);
    s->lewm.reset();
    if (s->staged) cudaEventDestroy(s->staged);
    s->weights.release();
    s->tc_packed.release();
    s->mma_packed.release();
    s->mma_xchg.release();
    s->tc_h0.release();
    s->h0_work.release();
    s->tc_x.release();
    s->small_x.release();
    if (s->side.stream) cudaStreamDestroy(s->side.stream);
    if (s->side.fork) cudaEventDestroy(s->side.fork);
    if (s->side.join) cudaEventDestroy(s->side.join);
    if (s->enc_side.stream) cudaStreamDestroy(s->enc_side.stream);
    if (s->enc_side.fork) cudaEventDestroy(s->enc_side.fork);
    if (s->enc_side.join) cudaEventDestroy(s->enc_side.join);
    s->ctx_dev.release();
    s->ctx_host.release();
    delete s;
    return LWM_OK;
}

// ------------------------------------------------------------------ planning

lwm_status lwm_plan_device(lwm_planner* p, lwm_scorer* sc, const float* injected, lwm_plan_device_result* out) {
    if (!p || !sc || !out) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (sc->ctx != p->ctx) return fail(LWM_INVALID_ARGUMENT, "planner and scorer belong to different contexts");
    if (p->shard_total && p->kind == PlannerKind::Mppi)
        return fail(LWM_INVALID_ARGUMENT, "planner is a candidate shard: use lwm_plan_device_shard");
    if (p->shard_total && !p->exchange)
        return fail(LWM_INVALID_ARGUMENT, "CEM / iCEM candidate shards need an elite exchange (lwm_planner_set_shard_exchange)");
    std::lock_guard<std::mutex> lock(p->mu);
    std::lock_guard<std::mutex> lock2(sc->mu);
    LWM_CUDA(cudaSetDevice(p->ctx->device));
    return plan_device_locked(p, sc, injected, out);
}

lwm_status lwm_icem_trace_device(lwm_planner* p, lwm_scorer* sc, const float* injected, lwm_plan_device_result* out,
                                 const float** trace) {
    if (!p || !sc || !out || !trace) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (p->kind != PlannerKind::Icem) return fail(LWM_INVALID_ARGUMENT, "trace_device is an iCEM planner call");
    if (sc->ctx != p->ctx) return fail(LWM_INVALID_ARGUMENT, "planner and scorer belong to different contexts");
    std::lock_guard<std::mutex> lock(p->mu);
    std::lock_guard<std::mutex> lock2(sc->mu);
    LWM_CUDA(cudaSetDevice(p->ctx->device));
    const uint32_t B = sc->batch;
    LWM_TRY(p->trace.ensure(static_cast<size_t>(p->iterations) * 4 * std::max<uint32_t>(B, 1) * 4));
    LWM_TRY(p->trace_elite.ensure(static_cast<size_t>(std::max<uint32_t>(B, 1)) * p->T * p->A * 4));
    LWM_TRY(plan_device_locked(p, sc, injected, out, true));
    *trace = p->trace.as<float>();
    return LWM_OK;
}

lwm_status lwm_planner_set_shard(lwm_planner* p, uint32_t sample_base, uint32_t sample_total) {
    if (!p) return fail(LWM_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> lock(p->mu);
    if (sample_total == 0) {
        p->shard_base = 0;
        p->shard_total = 0;
        return LWM_OK;
    }
    if (p->kind == PlannerKind::Mppi && p->iterations != 1)
        return fail(LWM_UNSUPPORTED, "candidate sharding supports MPPI planners with one iteration");
    if (p->kind != PlannerKind::Mppi) {
        const uint32_t K = p->kind == PlannerKind::Cem ? p->cem.elites : p->icem.elites;
        if (K > p->S)
            return fail(LWM_INVALID_ARGUMENT, "every shard needs at least `elites` (" + std::to_string(K) +
                                                  ") candidates, this one has " + std::to_string(p->S));
    }
    if (static_cast<uint64_t>(sample_base) + p->S > sample_total)
        return fail(LWM_INVALID_ARGUMENT, "shard samples [" + std::to_string(sample_base) + ", " +
                                              std::to_string(static_cast<uint64_t>(sample_base) + p->S) +
                                              ") exceed sample_total " + std::to_string(sample_total));
    p->shard_base = sample_base;
    p->shard_total = sample_total;
    return LWM_OK;
}

lwm_status lwm_planner_set_shard_exchange(lwm_planner* p, uint32_t shards, lwm_exchange_fn fn, void* user) {
    if (!p) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (p->kind == PlannerKind::Mppi)
        return fail(LWM_INVALID_ARGUMENT, "MPPI shards exchange tuples through lwm_mppi_combine_device");
    if ((fn == nullptr) != (shards == 0)) return fail(LWM_INVALID_ARGUMENT, "exchange and shard count go together");
    std::lock_guard<std::mutex> lock(p->mu);
    p->exchange = fn;
    p->exchange_user = user;
    p->exchange_shards = shards;
    return LWM_OK;
}

lwm_status lwm_plan_device_shard(lwm_planner* p, lwm_scorer* sc, const float* injected, const float** tuples,
                                 uint32_t* tuple_width) {
    if (!p || !sc || !tuples || !tuple_width) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (sc->ctx != p->ctx) return fail(LWM_INVALID_ARGUMENT, "planner and scorer belong to different contexts");
    if (!p->shard_total) return fail(LWM_INVALID_ARGUMENT, "planner is not a candidate shard (lwm_planner_set_shard)");
    std::lock_guard<std::mutex> lock(p->mu);
    std::lock_guard<std::mutex> lock2(sc->mu);
    LWM_CUDA(cudaSetDevice(p->ctx->device));
    lwm_plan_device_result r{};
    LWM_TRY(plan_device_locked(p, sc, injected, &r));
    *tuples = p->shard_tuples.as<float>();
    *tuple_width = mppi_args(p, p->mppi.temperature).pw;
    return LWM_OK;
}

lwm_status lwm_mppi_combine_device(lwm_planner* p, const float* tuples, uint32_t shards, lwm_plan_device_result* out) {
    if (!p || !tuples || !out || shards == 0) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (p->kind != PlannerKind::Mppi) return fail(LWM_UNSUPPORTED, "only MPPI tuples can be combined");
    std::lock_guard<std::mutex> lock(p->mu);
    const uint32_t B = p->last_batch;
    if (B == 0) return fail(LWM_INVALID_ARGUMENT, "no shard plan to combine");
    LWM_CUDA(cudaSetDevice(p->ctx->device));
    MppiArgs m = mppi_args(p, p->mppi.temperature);
    LWM_CUDA(lwm::launch_mppi_combine(m, tuples, B, shards, p->ctx->stream));
    p->ctx->launches += 1;
    p->has_warm = true;
    p->warm_batch = B;
    out->first_action = p->first_action.as<float>();
    out->sequence = p->sequence.as<float>();
    out->scores = p->scores.as<float>();
    out->best_indices = p->best.as<uint32_t>();
    out->batch = B;
    out->scores_cols = p->S;
    out->iterations_completed = 1;
    out->elapsed_ns = 0;
    out->deadline_reached = 0;
    out->deadline_outcome = LWM_DEADLINE_NONE;
    p->has_result = true;
    return LWM_OK;
}

lwm_status lwm_plan(lwm_planner* p, lwm_scorer* sc, const float* injected, lwm_plan_result* out) {
    if (!p || !sc || !out) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (sc->ctx != p->ctx) return fail(LWM_INVALID_ARGUMENT, "planner and scorer belong to different contexts");
    if (p->shard_total && p->kind == PlannerKind::Mppi)
        return fail(LWM_INVALID_ARGUMENT, "planner is a candidate shard: use lwm_plan_device_shard");
    if (p->shard_total && !p->exchange)
        return fail(LWM_INVALID_ARGUMENT, "CEM / iCEM candidate shards need an elite exchange (lwm_planner_set_shard_exchange)");
    const auto start = std::chrono::steady_clock::now();
    std::lock_guard<std::mutex> lock(p->mu);
    std::lock_guard<std::mutex> lock2(sc->mu);
    LWM_CUDA(cudaSetDevice(p->ctx->device));
    const float* dev_noise = nullptr;
    if (injected) {
        const size_t n = static_cast<size_t>(sc->batch) * p->S * p->T * p->A * p->iterations;
        LWM_TRY(p->noise_tmp.ensure(n * 4));
        LWM_CUDA(cudaMemcpyAsync(p->noise_tmp.ptr, injected, n * 4, cudaMemcpyHostToDevice, p->ctx->stream));
        dev_noise = p->noise_tmp.as<float>();
    }
    lwm_plan_device_result d{};
    LWM_TRY(plan_device_locked(p, sc, dev_noise, &d));
    const size_t B = d.batch;
    const size_t seq = B * p->T * p->A;
    const size_t nsc = B * d.scores_cols;
    // the results through the planner's pinned staging, laid out as the
    // planner's device result block: one copy when every output is wanted
    // and comes from that block
    const ResultLayout rl = result_layout(B, p->T, p->A, p->S);
    const size_t off_fa = rl.fa, off_seq = rl.seq, off_sc = rl.sc, off_best = rl.best;
    if (out->scores && out->scores_capacity < nsc) return fail(LWM_INVALID_ARGUMENT, "scores buffer too small");
    LWM_TRY(p->staging.ensure(rl.total));
    char* h = p->staging.as<char>();
    cudaStream_t stream = p->ctx->stream;
    const char* blk = p->results.as<char>();
    const bool one_copy = out->first_action && out->sequence && out->scores && out->best_indices &&
                          d.first_action == reinterpret_cast<const float*>(blk + rl.fa) &&
                          d.sequence == reinterpret_cast<const float*>(blk + rl.seq) &&
                          d.scores == reinterpret_cast<const float*>(blk + rl.sc) &&
                          d.best_indices == reinterpret_cast<const uint32_t*>(blk + rl.best);
    if (one_copy) {
        LWM_CUDA(cudaMemcpyAsync(h, blk, rl.total, cudaMemcpyDeviceToHost, stream));
    } else {
        if (out->first_action) LWM_CUDA(cudaMemcpyAsync(h + off_fa, d.first_action, B * p->A * 4, cudaMemcpyDeviceToHost, stream));
        if (out->sequence) LWM_CUDA(cudaMemcpyAsync(h + off_seq, d.sequence, seq * 4, cudaMemcpyDeviceToHost, stream));
        if (out->scores) LWM_CUDA(cudaMemcpyAsync(h + off_sc, d.scores, nsc * 4, cudaMemcpyDeviceToHost, stream));
        if (out->best_indices) LWM_CUDA(cudaMemcpyAsync(h + off_best, d.best_indices, B * 4, cudaMemcpyDeviceToHost, stream));
    }
    // the error word: the SkyJEPA tensor-core rollouts write theirs into the
    // result block (in the copy above when it is one copy); the LeWM GEMMs
    // keep theirs with the model
    int tc_err[4] = {0, 0, 0, 0};
    int* err_dev = sc->kind == ScorerKind::Lewm ? sc->lewm->split.tc_err : result_err(p, static_cast<uint32_t>(B));
    const bool err_in_copy = one_copy && sc->kind != ScorerKind::Lewm;
    if (err_dev && !err_in_copy)
        LWM_CUDA(cudaMemcpyAsync(tc_err, err_dev, sizeof tc_err, cudaMemcpyDeviceToHost, stream));
    LWM_CUDA(cudaStreamSynchronize(stream));
    if (err_in_copy) std::memcpy(tc_err, h + rl.err, sizeof tc_err);
    if (tc_err[0]) LWM_CUDA(cudaMemset(err_dev, 0, sizeof tc_err));
    if (tc_err[0] && p->counters.ptr) {
        // the blocks that gave up never arrived: clear the per-vehicle
        // arrival counters so the planner's next plan starts clean
        LWM_CUDA(cudaMemsetAsync(p->counters.ptr, 0, p->counters.bytes, stream));
        LWM_CUDA(cudaStreamSynchronize(stream));
    }
    if (tc_err[0])
        return fail(LWM_TIMEOUT, "a tensor-core pipeline wait timed out on the device (site " + std::to_string(tc_err[0]) +
                                     ", block " + std::to_string(tc_err[1]) + ", index " + std::to_string(tc_err[2]) +
                                     ", parity " + std::to_string(tc_err[3]) + ")");
    if (out->first_action) std::memcpy(out->first_action, h + off_fa, B * p->A * 4);
    if (out->sequence) std::memcpy(out->sequence, h + off_seq, seq * 4);
    if (out->scores) std::memcpy(out->scores, h + off_sc, nsc * 4);
    if (out->best_indices) std::memcpy(out->best_indices, h + off_best, B * 4);
    out->batch = d.batch;
    out->scores_cols = d.scores_cols;
    out->iterations_completed = d.iterations_completed;
    out->deadline_reached = d.deadline_reached;
    out->deadline_outcome = d.deadline_outcome;
    out->elapsed_ns = static_cast<uint64_t>(
        std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - start).count());
    return LWM_OK;
}

// --------------------------------------------------------- planner pieces

lwm_status lwm_lowest_k_device(lwm_ctx* ctx, const float* scores, uint32_t B, uint32_t S, uint32_t K, uint32_t* out) {
    if (!ctx || !scores || !out) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (K == 0) return fail(LWM_INVALID_ARGUMENT, "top-k count must be greater than zero");
    if (S == 0) return fail(LWM_INVALID_ARGUMENT, "score tensor must contain at least one sample");
    if (K > S) return fail(LWM_INVALID_ARGUMENT, "top-k count " + std::to_string(K) + " cannot exceed samples " + std::to_string(S));
    if (K > lwm::kMaxElites)
        return fail(LWM_UNSUPPORTED, "lowest-k supports at most " + std::to_string(lwm::kMaxElites) + " selected indices");
    LWM_CUDA(cudaSetDevice(ctx->device));
    LWM_CUDA(lwm::launch_lowest_k(scores, out, B, S, K, ctx->stream));
    ctx->launches += 1;
    return LWM_OK;
}

lwm_status lwm_color_noise_device(lwm_ctx* ctx, const float* noise, float* out, uint32_t B, uint32_t S, uint32_t T, uint32_t A,
                                  float beta) {
    if (!ctx || !noise || !out) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (!finite(beta) || beta < 0.0f) return fail(LWM_INVALID_ARGUMENT, "iCEM noise_beta must be finite and non-negative");
    LWM_CUDA(cudaSetDevice(ctx->device));
    const size_t n = static_cast<size_t>(B) * S * T * A;
    if (beta == 0.0f || T <= 1) {
        if (out != noise) LWM_CUDA(cudaMemcpyAsync(out, noise, n * 4, cudaMemcpyDeviceToDevice, ctx->stream));
        return LWM_OK;
    }
    float smooth = std::min(std::max(beta / (beta + 1.0f), 0.0f), 0.98f);
    LWM_CUDA(lwm::launch_color_noise(noise, out, B, S, T, A, smooth, ctx->stream));
    ctx->launches += 1;
    return LWM_OK;
}

void lwm_image_preprocess_imagenet_224(lwm_image_preprocess* out) {
    out->output_height = 224;
    out->output_width = 224;
    out->mean[0] = 0.485f; out->mean[1] = 0.456f; out->mean[2] = 0.406f;
    out->std[0] = 0.229f; out->std[1] = 0.224f; out->std[2] = 0.225f;
}

// ImagePreprocess::validate (src/media/mod.rs:185-193) and the history-slot check.
static lwm_status validate_preprocess(const lwm_image_preprocess* cfg, uint32_t history_len, uint32_t slot,
                                      const char* kind) {
    if (cfg->output_height == 0 || cfg->output_width == 0)
        return fail(LWM_INVALID_ARGUMENT, "CUDA preprocess output dimensions must be greater than zero");
    for (int i = 0; i < 3; ++i)
        if (cfg->std[i] == 0.0f) return fail(LWM_INVALID_ARGUMENT, "CUDA preprocess std values must be non-zero");
    if (history_len > 0 && slot >= history_len)
        return fail(LWM_INVALID_ARGUMENT, std::string("CUDA ") + kind + " history slot " + std::to_string(slot) +
                                              " is outside history_len " + std::to_string(history_len));
    return LWM_OK;
}

// The error word of the row-staged preprocessing kernels (mapped pinned
// host memory, read by lwm_ctx_synchronize), allocated on first use.
static lwm_status ensure_media_err(lwm_ctx* ctx) {
    if (ctx->media_err) return LWM_OK;
    void* dev = nullptr;
    int* host = nullptr;
    LWM_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&host), 4 * sizeof(int), cudaHostAllocMapped));
    for (int i = 0; i < 4; ++i) host[i] = 0;
    const cudaError_t e = cudaHostGetDevicePointer(&dev, host, 0);
    if (e != cudaSuccess) {
        cudaFreeHost(host);
        return fail(LWM_CUDA_ERROR, std::string("cudaHostGetDevicePointer: ") + cudaGetErrorString(e));
    }
    ctx->media_err = host;
    ctx->media_err_dev = static_cast<int*>(dev);
    return LWM_OK;
}

static lwm::MediaArgs media_args(const lwm_image_preprocess* cfg, uint32_t B, uint32_t H, uint32_t W,
                                 uint32_t history_len, uint32_t slot, int32_t bf16, void* out) {
    lwm::MediaArgs a{};
    a.out = out;
    a.batch = B; a.in_h = H; a.in_w = W;
    a.out_h = cfg->output_height; a.out_w = cfg->output_width;
    a.history_len = history_len; a.history_slot = slot;
    a.bf16 = bf16 ? 1 : 0;
    for (int i = 0; i < 3; ++i) { a.mean[i] = cfg->mean[i]; a.std[i] = cfg->std[i]; }
    return a;
}

}  // extern "C"

namespace {

// Argument checks and the launch of packed / NV12 preprocessing into any
// output layout (`patch` > 0: the ViT patch matrix).
lwm_status preprocess_packed(lwm_ctx* ctx, const uint8_t* input, uint32_t B, uint32_t H, uint32_t W, int32_t format,
                             const lwm_image_preprocess* cfg, uint32_t history_len, uint32_t slot, uint32_t patch,
                             int32_t out_bf16, void* output) {
    if (!cfg) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (format < 0 || format > 3)
        return fail(LWM_INVALID_ARGUMENT, "unknown packed image format " + std::to_string(format) +
                                              "; expected 0=RGB, 1=BGR, 2=RGBA, or 3=BGRA");
    if (B == 0 || H == 0 || W == 0) return fail(LWM_INVALID_ARGUMENT, "packed CUDA image dimensions must be greater than zero");
    LWM_TRY(validate_preprocess(cfg, history_len, slot, "image"));
    if (!ctx || !input || !output) return fail(LWM_INVALID_ARGUMENT, "null argument");
    LWM_CUDA(cudaSetDevice(ctx->device));
    lwm::MediaArgs a = media_args(cfg, B, H, W, history_len, slot, out_bf16, output);
    a.a = input;
    a.channels = format >= 2 ? 4 : 3;
    a.format = static_cast<uint32_t>(format);
    a.patch = patch;
    a.test_skip_row_plus1 = ctx->faults.media_skip_row_plus1;
    a.test_wait_polls = ctx->faults.wait_polls;
    if (lwm::packed_staged_eligible(a)) {
        LWM_TRY(ensure_media_err(ctx));
        LWM_CUDA(lwm::launch_packed_staged(a, ctx->media_err_dev, ctx->stream));
    } else {
        LWM_CUDA(lwm::launch_media(a, false, ctx->stream));
    }
    ctx->launches += 1;
    return LWM_OK;
}

lwm_status preprocess_nv12(lwm_ctx* ctx, const uint8_t* y_plane, const uint8_t* uv_plane, uint32_t B, uint32_t H,
                           uint32_t W, int32_t color_space, const lwm_image_preprocess* cfg, uint32_t history_len,
                           uint32_t slot, uint32_t patch, int32_t out_bf16, void* output,
                           cudaStream_t stream = nullptr) {
    if (!cfg) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (color_space < 0 || color_space > 3)
        return fail(LWM_INVALID_ARGUMENT, "unknown NV12 color space " + std::to_string(color_space) +
                                              "; expected 0=BT.601 video, 1=BT.709 video, 2=BT.601 full, or 3=BT.709 full");
    if (B == 0 || H == 0 || W == 0) return fail(LWM_INVALID_ARGUMENT, "NV12 CUDA image dimensions must be greater than zero");
    if (H % 2 != 0 || W % 2 != 0)
        return fail(LWM_INVALID_ARGUMENT, "NV12 CUDA image dimensions must be even, got " + std::to_string(H) + "x" +
                                              std::to_string(W));
    LWM_TRY(validate_preprocess(cfg, history_len, slot, "NV12"));
    if (!ctx || !y_plane || !uv_plane || !output) return fail(LWM_INVALID_ARGUMENT, "null argument");
    LWM_CUDA(cudaSetDevice(ctx->device));
    lwm::MediaArgs a = media_args(cfg, B, H, W, history_len, slot, out_bf16, output);
    a.a = y_plane;
    a.uv = uv_plane;
    a.channels = 1;
    a.format = static_cast<uint32_t>(color_space);
    a.patch = patch;
    a.test_skip_row_plus1 = ctx->faults.media_skip_row_plus1;
    a.test_wait_polls = ctx->faults.wait_polls;
    if (lwm::nv12_staged_eligible(a)) {
        LWM_TRY(ensure_media_err(ctx));
        LWM_CUDA(lwm::launch_nv12_staged(a, ctx->media_err_dev, stream ? stream : ctx->stream));
    } else {
        LWM_CUDA(lwm::launch_media(a, true, stream ? stream : ctx->stream));
    }
    ctx->launches += 1;
    return LWM_OK;
}

lwm_status check_patch(const lwm_image_preprocess* cfg, uint32_t patch) {
    if (!cfg) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (patch == 0 || cfg->output_height % patch != 0 || cfg->output_width % patch != 0)
        return fail(LWM_INVALID_ARGUMENT, "patch size " + std::to_string(patch) + " must divide the output size " +
                                              std::to_string(cfg->output_height) + "x" +
                                              std::to_string(cfg->output_width));
    return LWM_OK;
}

// The image encoder's patch size and frame size must be the output's.
lwm_status check_vit_encoder(lwm_scorer* s, const lwm_image_preprocess* cfg) {
    const lwm_lewm_config& c = s->lewm->c;
    if (c.encoder != LWM_ENCODER_VIT) return fail(LWM_INVALID_ARGUMENT, "encode_pixels called on non-image observation encoder");
    if (c.channels != 3) return fail(LWM_INVALID_ARGUMENT, "frame encoding needs a 3-channel image encoder");
    if (cfg->output_height != c.image_size || cfg->output_width != c.image_size)
        return fail(LWM_INVALID_ARGUMENT, "preprocess output " + std::to_string(cfg->output_height) + "x" +
                                              std::to_string(cfg->output_width) + " does not match the encoder's image size " +
                                              std::to_string(c.image_size));
    return LWM_OK;
}

lwm_status check_vit_frames(lwm_scorer* s, const lwm_image_preprocess* cfg, uint32_t n, float* out) {
    if (!s || s->kind != ScorerKind::Lewm || !cfg || !out || n == 0)
        return fail(LWM_INVALID_ARGUMENT, "invalid encode arguments");
    return check_vit_encoder(s, cfg);
}

}  // namespace

extern "C" {

lwm_status lwm_preprocess_packed_device(lwm_ctx* ctx, const uint8_t* input, uint32_t B, uint32_t H, uint32_t W,
                                        int32_t format, const lwm_image_preprocess* cfg, uint32_t history_len,
                                        uint32_t slot, int32_t out_bf16, void* output) {
    return preprocess_packed(ctx, input, B, H, W, format, cfg, history_len, slot, 0, out_bf16, output);
}

lwm_status lwm_preprocess_nv12_device(lwm_ctx* ctx, const uint8_t* y_plane, const uint8_t* uv_plane, uint32_t B,
                                      uint32_t H, uint32_t W, int32_t color_space, const lwm_image_preprocess* cfg,
                                      uint32_t history_len, uint32_t slot, int32_t out_bf16, void* output) {
    return preprocess_nv12(ctx, y_plane, uv_plane, B, H, W, color_space, cfg, history_len, slot, 0, out_bf16, output);
}

lwm_status lwm_preprocess_packed_patches_device(lwm_ctx* ctx, const uint8_t* input, uint32_t B, uint32_t H, uint32_t W,
                                                int32_t format, const lwm_image_preprocess* cfg, uint32_t patch,
                                                int32_t out_bf16, void* output) {
    LWM_TRY(check_patch(cfg, patch));
    return preprocess_packed(ctx, input, B, H, W, format, cfg, 0, 0, patch, out_bf16, output);
}

lwm_status lwm_preprocess_nv12_patches_device(lwm_ctx* ctx, const uint8_t* y_plane, const uint8_t* uv_plane,
                                              uint32_t B, uint32_t H, uint32_t W, int32_t color_space,
                                              const lwm_image_preprocess* cfg, uint32_t patch, int32_t out_bf16,
                                              void* output) {
    LWM_TRY(check_patch(cfg, patch));
    return preprocess_nv12(ctx, y_plane, uv_plane, B, H, W, color_space, cfg, 0, 0, patch, out_bf16, output);
}

lwm_status lwm_lewm_encode_nv12_device(lwm_scorer* s, const uint8_t* y_plane, const uint8_t* uv_plane, uint32_t n,
                                       uint32_t H, uint32_t W, int32_t color_space, const lwm_image_preprocess* cfg,
                                       float* out) {
    LWM_TRY(check_vit_frames(s, cfg, n, out));
    std::lock_guard<std::mutex> lock(s->mu);
    LWM_CUDA(cudaSetDevice(s->ctx->device));
    float* patches = nullptr;
    LWM_CUDA(s->lewm->patch_buffer(n, &patches));
    LWM_TRY(preprocess_nv12(s->ctx, y_plane, uv_plane, n, H, W, color_space, cfg, 0, 0, s->lewm->c.patch_size, 0,
                            patches));
    LWM_CUDA(s->lewm->encode_patches(n, out, s->ctx->stream));
    s->ctx->launches += static_cast<uint64_t>(s->lewm->launches);
    return LWM_OK;
}

lwm_status lwm_lewm_encode_packed_device(lwm_scorer* s, const uint8_t* input, uint32_t n, uint32_t H, uint32_t W,
                                         int32_t format, const lwm_image_preprocess* cfg, float* out) {
    LWM_TRY(check_vit_frames(s, cfg, n, out));
    std::lock_guard<std::mutex> lock(s->mu);
    LWM_CUDA(cudaSetDevice(s->ctx->device));
    float* patches = nullptr;
    LWM_CUDA(s->lewm->patch_buffer(n, &patches));
    LWM_TRY(preprocess_packed(s->ctx, input, n, H, W, format, cfg, 0, 0, s->lewm->c.patch_size, 0, patches));
    LWM_CUDA(s->lewm->encode_patches(n, out, s->ctx->stream));
    s->ctx->launches += static_cast<uint64_t>(s->lewm->launches);
    return LWM_OK;
}

// LeWmSession::reset_pixels + encode_pixels of the goal + plan
// (src/session.rs:31-40, 46-65; planner.rs:450): the frames' encoder runs on
// the scorer's high-priority encoder stream, beside the planner's sampling and
// the candidate-only part of scoring on the context stream; the rollout waits
// for it.  The context stream is ordered after the encoder on every return.
lwm_status lwm_lewm_plan_nv12_device(lwm_planner* p, lwm_scorer* s, const uint8_t* y_plane, const uint8_t* uv_plane,
                                     uint32_t B, uint32_t h, uint32_t H, uint32_t W, int32_t color_space,
                                     const lwm_image_preprocess* cfg, const float* injected,
                                     lwm_plan_device_result* out) {
    if (!p || !s || !out || !y_plane || !uv_plane || !cfg) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (s->kind != ScorerKind::Lewm) return fail(LWM_INVALID_ARGUMENT, "not a LeWM scorer");
    if (s->ctx != p->ctx) return fail(LWM_INVALID_ARGUMENT, "planner and scorer belong to different contexts");
    if (p->shard_total) return fail(LWM_INVALID_ARGUMENT, "planner is a candidate shard: encode, set the context and plan");
    if (B == 0 || h == 0) return fail(LWM_INVALID_ARGUMENT, "invalid LeWM context shapes");
    lwm::LewmModel& m = *s->lewm;
    if (h > m.c.num_frames)
        return fail(LWM_INVALID_ARGUMENT, "rollout window " + std::to_string(h) + " exceeds predictor.num_frames " +
                                              std::to_string(m.c.num_frames));
    const uint64_t frames = static_cast<uint64_t>(B) * (static_cast<uint64_t>(h) + 1);
    if (frames > 65536) return fail(LWM_INVALID_ARGUMENT, "too many frames: " + std::to_string(frames));
    const uint32_t n = static_cast<uint32_t>(frames);
    LWM_TRY(check_vit_encoder(s, cfg));
    std::lock_guard<std::mutex> lock(p->mu);
    std::lock_guard<std::mutex> lock2(s->mu);
    LWM_CUDA(cudaSetDevice(p->ctx->device));
    cudaStream_t stream = p->ctx->stream;
    lwm::SideStream& side = s->enc_side;
    if (!side.stream) {
        int least = 0, greatest = 0;
        LWM_CUDA(cudaDeviceGetStreamPriorityRange(&least, &greatest));
        LWM_CUDA(cudaStreamCreateWithPriority(&side.stream, cudaStreamNonBlocking, greatest));
        LWM_CUDA(cudaEventCreateWithFlags(&side.fork, cudaEventDisableTiming));
        LWM_CUDA(cudaEventCreateWithFlags(&side.join, cudaEventDisableTiming));
    }
    // observation frames [B, h] then the B goals: one encoder output fills emb and goal
    LWM_CUDA(m.ensure_context(B, h, true, stream));
    float* patches = nullptr;
    LWM_CUDA(m.patch_buffer(n, &patches));
    // the frames and the context buffers were last touched in stream order
    LWM_CUDA(cudaEventRecord(side.fork, stream));
    LWM_CUDA(cudaStreamWaitEvent(side.stream, side.fork, 0));
    struct Join {  // on every return: the context stream waits for the encoder stream
        lwm::LewmModel& m;
        lwm::SideStream& side;
        cudaStream_t stream;
        ~Join() {
            m.join_ev = nullptr;
            if (cudaEventRecord(side.join, side.stream) == cudaSuccess) cudaStreamWaitEvent(stream, side.join, 0);
        }
    } join{m, side, stream};
    LWM_TRY(preprocess_nv12(s->ctx, y_plane, uv_plane, n, H, W, color_space, cfg, 0, 0, m.c.patch_size, 0, patches,
                            side.stream));
    LWM_CUDA(m.encode_patches(n, m.emb, side.stream));
    s->ctx->launches += static_cast<uint64_t>(m.launches);
    LWM_CUDA(cudaEventRecord(side.join, side.stream));
    m.B = B;
    m.h = h;
    m.history = h;
    s->batch = B;
    s->has_context = true;
    m.join_ev = side.join;
    return plan_device_locked(p, s, injected, out);
}

lwm_status lwm_normal_device(lwm_ctx* ctx, uint64_t seed, uint64_t offset, size_t count, float* out) {
    if (!ctx || !out) return fail(LWM_INVALID_ARGUMENT, "null argument");
    if (count == 0) return LWM_OK;
    LWM_CUDA(cudaSetDevice(ctx->device));
    LWM_CUDA(lwm::launch_normal_fill(seed, offset, count, out, ctx->stream));
    ctx->launches += 1;
    return LWM_OK;
}

}  // extern "C"
