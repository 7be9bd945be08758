// host_task.cpp — host-side inputs of the planner: the rotor domain, the
// reference trajectories, the geometric action prior, one plant step and
// seeded random model weights.  These are host code in the reference too
// (src/skyjepa_sim.rs, src/skyjepa_task.rs, candle_nn init); they build the
// context a plan consumes.
#include <cmath>
#include <cstdint>
#include <cstring>

#include "../../include/lewm_b200.h"
#include "lwm_task_math.hpp"

using lwm::task::clampf;

namespace {

// SplitMix64 (src/skyjepa_sim.rs:294-318): the reference's domain sampler.
struct SplitMix64 {
    uint64_t state;
    uint64_t next() {
        state += 0x9E3779B97F4A7C15ull;
        uint64_t v = state;
        v = (v ^ (v >> 30)) * 0xBF58476D1CE4E5B9ull;
        v = (v ^ (v >> 27)) * 0x94D049BB133111EBull;
        return v ^ (v >> 31);
    }
    float unit() { return (static_cast<float>(next() >> 40) + 0.5f) / static_cast<float>(1u << 24); }
    float range(float lo, float hi) { return lo + (hi - lo) * unit(); }
    double unit53() { return (static_cast<double>(next() >> 11) + 0.5) * (1.0 / 9007199254740992.0); }
    double normal() {
        const double u1 = unit53(), u2 = unit53();
        return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
    }
};

}  // namespace

extern "C" {

void lwm_domain_default(lwm_domain* d) {
    d->mass = 1.3f;
    d->inertia[0] = 0.021f; d->inertia[1] = 0.023f; d->inertia[2] = 0.040f;
    d->motor_time_constant = 0.04f;
    d->drag[0] = 0.25f; d->drag[1] = 0.25f; d->drag[2] = 0.30f;
    d->thrust_scale = 1.0f;
    d->torque_scale = 1.0f;
    d->arm_length = 0.17f;
    d->gravity = 9.81f;
    d->max_thrust_weight = 4.0f;
}

// SkyJepaDomain::sample (src/skyjepa_sim.rs:61-86), training ranges.
void lwm_domain_sample(uint64_t seed, lwm_domain* d) {
    lwm_domain nominal;
    lwm_domain_default(&nominal);
    SplitMix64 rng{seed};
    *d = nominal;
    d->mass = nominal.mass * rng.range(0.5f, 1.5f);
    for (int i = 0; i < 3; ++i) d->inertia[i] = nominal.inertia[i] * rng.range(0.7f, 1.3f);
    d->motor_time_constant = rng.range(0.01f, 0.1f);
    for (int i = 0; i < 3; ++i) d->drag[i] = rng.range(0.1f, 0.5f);
    d->thrust_scale = rng.range(0.5f, 1.5f);
    d->torque_scale = rng.range(0.5f, 1.5f);
    d->arm_length = nominal.arm_length * rng.range(0.8f, 1.2f);
}

void lwm_tracking_cost_paper(lwm_tracking_cost* c) {
    c->position = 400.0f;
    c->velocity = 40.0f;
    c->attitude = 20.0f;
    c->angular_velocity = 20.0f;
    c->action[0] = 0.01f; c->action[1] = 0.05f; c->action[2] = 0.05f; c->action[3] = 0.10f;
}

static void tcn_cfg(lwm_tcn_config* t, uint32_t in, uint32_t levels, const uint32_t* ch, uint32_t k) {
    std::memset(t, 0, sizeof(*t));
    t->input_dim = in;
    t->levels = levels;
    for (uint32_t i = 0; i < levels; ++i) t->channels[i] = ch[i];
    t->kernel_size = k;
}

void lwm_skyjepa_config_paper(lwm_skyjepa_config* c) {
    std::memset(c, 0, sizeof(*c));
    c->state_dim = 18; c->action_dim = 4; c->history_steps = 10; c->rollout_steps = 20; c->latent_dim = 24;
    const uint32_t s[3] = {8, 8, 16}, a[3] = {4, 4, 8};
    tcn_cfg(&c->state_encoder, 18, 3, s, 3);
    tcn_cfg(&c->action_encoder, 4, 3, a, 3);
    c->prober_hidden_dim = 32;
    c->prober_hidden_layers = 2;
    c->kinematics.mass = 1.3; c->kinematics.gravity = 9.81; c->kinematics.hover_throttle = 0.2;
    c->kinematics.action_space = LWM_ACTION_SPACE_ROTOR_FORCES;
}

void lwm_skyjepa_config_wide(lwm_skyjepa_config* c) {
    lwm_skyjepa_config_paper(c);
    c->latent_dim = 256;
    const uint32_t s[3] = {128, 128, 128}, a[3] = {4, 4, 4};
    tcn_cfg(&c->state_encoder, 18, 3, s, 3);
    tcn_cfg(&c->action_encoder, 4, 3, a, 3);
}

// Tensor order of the weight blob (include/lewm_b200.h).  kind: 0 Kaiming
// normal (fan_in), 1 U(+-1/sqrt(fan_in)), 2 Kaiming uniform (fan_in),
// 3 zeros, 4 N(0, 1e-3).
struct TensorSpec { size_t n; size_t fan_in; int kind; };

static size_t visit_tcn(const lwm_tcn_config& t, TensorSpec* out, size_t idx) {
    uint32_t in = t.input_dim;
    for (uint32_t l = 0; l < t.levels; ++l) {
        const uint32_t o = t.channels[l];
        const size_t k = t.kernel_size;
        if (out) {
            out[idx + 0] = {static_cast<size_t>(o) * in * k, in * k, 0};
            out[idx + 1] = {o, in * k, 1};
            out[idx + 2] = {static_cast<size_t>(o) * o * k, o * k, 0};
            out[idx + 3] = {o, o * k, 1};
        }
        idx += 4;
        if (in != o) {
            if (out) {
                out[idx + 0] = {static_cast<size_t>(o) * in, in, 0};
                out[idx + 1] = {o, in, 1};
            }
            idx += 2;
        }
        in = o;
    }
    return idx;
}

static bool valid_tcn(const lwm_tcn_config& t) {
    if (t.input_dim == 0 || t.levels == 0 || t.levels > LWM_TCN_MAX_LEVELS || t.kernel_size == 0) return false;
    for (uint32_t l = 0; l < t.levels; ++l) if (t.channels[l] == 0) return false;
    return true;
}

static size_t weight_specs(const lwm_skyjepa_config* c, TensorSpec* out) {
    size_t idx = 0;
    idx = visit_tcn(c->state_encoder, out, idx);
    const uint32_t H = c->latent_dim;
    const uint32_t so = c->state_encoder.channels[c->state_encoder.levels - 1];
    if (out) { out[idx] = {static_cast<size_t>(H) * so, so, 0}; out[idx + 1] = {H, so, 1}; }
    idx += 2;
    idx = visit_tcn(c->action_encoder, out, idx);
    const uint32_t E = c->action_encoder.channels[c->action_encoder.levels - 1];
    if (out) {
        out[idx + 0] = {static_cast<size_t>(3) * H * E, E, 2};
        out[idx + 1] = {static_cast<size_t>(3) * H * H, H, 2};
        out[idx + 2] = {static_cast<size_t>(3) * H, H, 3};
        out[idx + 3] = {static_cast<size_t>(3) * H, H, 3};
    }
    idx += 4;
    const uint32_t hid = c->prober_hidden_dim;
    if (out) { out[idx] = {static_cast<size_t>(hid) * H, H, 0}; out[idx + 1] = {hid, H, 1}; }
    idx += 2;
    for (uint32_t i = 0; i + 1 < c->prober_hidden_layers; ++i) {
        if (out) { out[idx] = {static_cast<size_t>(hid) * hid, hid, 0}; out[idx + 1] = {hid, hid, 1}; }
        idx += 2;
    }
    if (out) { out[idx] = {static_cast<size_t>(15) * hid, hid, 4}; out[idx + 1] = {15, hid, 3}; }
    idx += 2;
    return idx;
}

static bool valid_config(const lwm_skyjepa_config* c) {
    return c && c->state_dim == 18 && c->action_dim == 4 && c->history_steps >= 2 && c->latent_dim > 0 &&
           valid_tcn(c->state_encoder) && valid_tcn(c->action_encoder) && c->state_encoder.input_dim == 18 &&
           c->action_encoder.input_dim == 4 && c->prober_hidden_dim > 0 && c->prober_hidden_layers > 0;
}

size_t lwm_skyjepa_weight_count(const lwm_skyjepa_config* c) {
    if (!valid_config(c)) return 0;
    const size_t n = weight_specs(c, nullptr);
    TensorSpec* specs = new TensorSpec[n];
    weight_specs(c, specs);
    size_t total = 0;
    for (size_t i = 0; i < n; ++i) total += specs[i].n;
    delete[] specs;
    return total;
}

lwm_status lwm_skyjepa_random_weights(const lwm_skyjepa_config* c, uint64_t seed, float* out, size_t count) {
    if (!valid_config(c) || !out || count != lwm_skyjepa_weight_count(c)) return LWM_INVALID_ARGUMENT;
    const size_t n = weight_specs(c, nullptr);
    TensorSpec* specs = new TensorSpec[n];
    weight_specs(c, specs);
    SplitMix64 rng{seed ^ 0x6C65776D62323030ull};
    size_t off = 0;
    for (size_t i = 0; i < n; ++i) {
        const double fan = static_cast<double>(specs[i].fan_in);
        for (size_t j = 0; j < specs[i].n; ++j) {
            double v = 0.0;
            switch (specs[i].kind) {
                case 0: v = rng.normal() * std::sqrt(2.0 / fan); break;
                case 1: { const double bound = 1.0 / std::sqrt(fan); v = (2.0 * rng.unit53() - 1.0) * bound; break; }
                case 2: { const double bound = std::sqrt(6.0 / fan); v = (2.0 * rng.unit53() - 1.0) * bound; break; }
                case 3: v = 0.0; break;
                default: v = rng.normal() * 1e-3; break;
            }
            out[off + j] = static_cast<float>(v);
        }
        off += specs[i].n;
    }
    delete[] specs;
    return LWM_OK;
}

lwm_status lwm_skyjepa_reference_horizon(int32_t kind, float time, float dt, uint32_t horizon, float radius,
                                         float period, float* out) {
    if (!out || kind < 0 || kind > 2) return LWM_INVALID_ARGUMENT;
    for (uint32_t i = 1; i <= horizon; ++i)
        lwm::task::reference_state(kind, time + static_cast<float>(i) * dt, radius, period,
                                   out + static_cast<size_t>(i - 1) * 18);
    return LWM_OK;
}

// skyjepa_geometric_action_prior (src/skyjepa_task.rs:118-240).
lwm_status lwm_skyjepa_geometric_prior(const float* cur, const float* refs, uint32_t T, float dt,
                                       const lwm_domain* d, float* out) {
    if (!cur || !refs || !d || !out) return LWM_INVALID_ARGUMENT;
    for (uint32_t index = 0; index < T; ++index)
        lwm::task::geometric_prior_step(cur, refs, index, T, dt, *d, out + static_cast<size_t>(index) * 4);
    return LWM_OK;
}

// SkyJepaRotorPlant::step (src/skyjepa_sim.rs:206-281).
lwm_status lwm_rotor_plant_step(const lwm_domain* d, float* x, float* motors, const float* cmd, float dt) {
    if (!d || !x || !motors || !cmd) return LWM_INVALID_ARGUMENT;
    if (!std::isfinite(dt) || dt <= 0.0f) return LWM_OK;
    lwm::task::plant_step(*d, x, motors, cmd, dt);
    return LWM_OK;
}

}  // extern "C"
