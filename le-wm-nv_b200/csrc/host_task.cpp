// host_task.cpp — host-side inputs of the planner: the rotor domain, the
// reference trajectories, the geometric action prior, one plant step and
// seeded random model weights.  These are host code in the reference too
// (src/skyjepa_sim.rs, src/skyjepa_task.rs, candle_nn init); they build the
// context a plan consumes.
#include <cmath>
#include <cstdint>
#include <cstring>

#include "../../include/lewm_b200.h"

namespace {

float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

void cross3(const float* l, const float* r, float* o) {
    o[0] = l[1] * r[2] - l[2] * r[1];
    o[1] = l[2] * r[0] - l[0] * r[2];
    o[2] = l[0] * r[1] - l[1] * r[0];
}

float dot3(const float* a, const float* b) { return a[0] * b[0] + a[1] * b[1] + a[2] * b[2]; }

void normalize_or(const float* v, const float* fallback, float* out) {
    const float n = std::sqrt(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
    if (n > 1e-6f) {
        out[0] = v[0] / n; out[1] = v[1] / n; out[2] = v[2] / n;
    } else {
        out[0] = fallback[0]; out[1] = fallback[1]; out[2] = fallback[2];
    }
}

// Columns (x, y, up) of a rotation whose third column is `up`, x from `heading`.
void frame_from_up(const float* up, const float* heading, float* R) {
    static const float fy[3] = {0.0f, 1.0f, 0.0f};
    float c[3], by[3], bx[3];
    cross3(up, heading, c);
    normalize_or(c, fy, by);
    cross3(by, up, c);
    normalize_or(c, heading, bx);
    R[0] = bx[0]; R[1] = by[0]; R[2] = up[0];
    R[3] = bx[1]; R[4] = by[1]; R[5] = up[1];
    R[6] = bx[2]; R[7] = by[2]; R[8] = up[2];
}

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

// skyjepa_reference_state (src/skyjepa_task.rs:57-110).
static void reference_state(int kind, float time, float radius, float period, float* s) {
    std::memset(s, 0, 18 * sizeof(float));
    s[2] = 1.0f;
    const float omega = 2.0f * static_cast<float>(M_PI) / period;
    const float angle = omega * time;
    float acc[3] = {0.0f, 0.0f, 0.0f};
    if (kind == 1) {
        acc[0] = -radius * omega * omega * std::cos(angle);
        acc[1] = -radius * omega * omega * std::sin(angle);
        s[0] = radius * (std::cos(angle) - 1.0f);
        s[1] = radius * std::sin(angle);
        s[3] = -radius * omega * std::sin(angle);
        s[4] = radius * omega * std::cos(angle);
    } else if (kind == 2) {
        acc[0] = -radius * omega * omega * std::sin(angle);
        acc[1] = -2.0f * radius * omega * omega * std::sin(2.0f * angle);
        acc[2] = -0.0625f * omega * omega * std::sin(0.5f * angle);
        s[0] = radius * std::sin(angle);
        s[1] = radius * 0.5f * std::sin(2.0f * angle);
        s[2] = 1.2f + 0.25f * std::sin(0.5f * angle);
        s[3] = radius * omega * std::cos(angle);
        s[4] = radius * omega * std::cos(2.0f * angle);
        s[5] = 0.125f * omega * std::cos(0.5f * angle);
    }
    static const float fz[3] = {0.0f, 0.0f, 1.0f};
    const float a[3] = {acc[0], acc[1], acc[2] + 9.81f};
    float up[3];
    normalize_or(a, fz, up);
    float heading[3] = {1.0f, 0.0f, 0.0f};
    if (!(std::fabs(up[0]) < 0.95f)) { heading[0] = 0.0f; heading[1] = 1.0f; }
    frame_from_up(up, heading, s + 6);
}

lwm_status lwm_skyjepa_reference_horizon(int32_t kind, float time, float dt, uint32_t horizon, float radius,
                                         float period, float* out) {
    if (!out || kind < 0 || kind > 2) return LWM_INVALID_ARGUMENT;
    for (uint32_t i = 1; i <= horizon; ++i)
        reference_state(kind, time + static_cast<float>(i) * dt, radius, period, out + static_cast<size_t>(i - 1) * 18);
    return LWM_OK;
}

// skyjepa_geometric_action_prior (src/skyjepa_task.rs:118-240).
lwm_status lwm_skyjepa_geometric_prior(const float* cur, const float* refs, uint32_t T, float dt,
                                       const lwm_domain* d, float* out) {
    if (!cur || !refs || !d || !out) return LWM_INVALID_ARGUMENT;
    static const float fz[3] = {0.0f, 0.0f, 1.0f}, fx[3] = {1.0f, 0.0f, 0.0f};
    for (uint32_t index = 0; index < T; ++index) {
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
                     (a == 2 ? d->gravity : 0.0f);
        float up[3], hd[3];
        const float hraw[3] = {ref[6], ref[9], 0.0f};
        normalize_or(des, fz, up);
        normalize_or(hraw, fx, hd);
        if (std::fabs(dot3(up, hd)) > 0.95f) { const float h0 = hd[0]; hd[0] = -hd[1]; hd[1] = h0; hd[2] = 0.0f; }
        float D[9];
        frame_from_up(up, hd, D);
        const float* R = index == 0 ? cur + 6 : ref + 6;
        const float* om = index == 0 ? cur + 15 : ref + 15;
        // attitude_error_body: vee of the skew part of D^T R
        float P[9];
        for (int col = 0; col < 3; ++col) {
            const float v[3] = {R[col], R[3 + col], R[6 + col]};
            const float dx = D[0] * v[0] + D[3] * v[1] + D[6] * v[2];
            const float dy = D[1] * v[0] + D[4] * v[1] + D[7] * v[2];
            const float dz = D[2] * v[0] + D[5] * v[1] + D[8] * v[2];
            P[0 * 3 + col] = dx; P[1 * 3 + col] = dy; P[2 * 3 + col] = dz;
        }
        const float err[3] = {0.5f * (P[7] - P[5]), 0.5f * (P[2] - P[6]), 0.5f * (P[3] - P[1])};
        float torque[3];
        for (int a = 0; a < 3; ++a) torque[a] = -d->inertia[a] * (25.0f * err[a] + 8.0f * om[a]);
        const float cup[3] = {R[2], R[5], R[8]};
        float proj = dot3(des, cup);
        if (proj < 0.0f) proj = 0.0f;
        const float total = clampf(d->mass * proj / d->thrust_scale, 0.0f, d->mass * d->gravity * d->max_thrust_weight);
        const float arm = d->arm_length * d->thrust_scale;
        const float yaw = 0.025f * d->torque_scale * d->thrust_scale;
        const float base = total / 4.0f;
        const float f[4] = {base - torque[1] / (2.0f * arm) + torque[2] / (4.0f * yaw),
                            base + torque[0] / (2.0f * arm) - torque[2] / (4.0f * yaw),
                            base + torque[1] / (2.0f * arm) + torque[2] / (4.0f * yaw),
                            base - torque[0] / (2.0f * arm) - torque[2] / (4.0f * yaw)};
        const float maximum = d->mass * d->gravity * d->max_thrust_weight / 4.0f;
        for (int r = 0; r < 4; ++r) out[static_cast<size_t>(index) * 4 + r] = clampf(f[r], 0.0f, maximum);
    }
    return LWM_OK;
}

// SkyJepaRotorPlant::step (src/skyjepa_sim.rs:206-281).
lwm_status lwm_rotor_plant_step(const lwm_domain* d, float* x, float* motors, const float* cmd, float dt) {
    if (!d || !x || !motors || !cmd) return LWM_INVALID_ARGUMENT;
    if (!std::isfinite(dt) || dt <= 0.0f) return LWM_OK;
    const float max_force = d->mass * d->gravity * d->max_thrust_weight / 4.0f;
    const float response = 1.0f - std::exp(-dt / d->motor_time_constant);
    for (int r = 0; r < 4; ++r) motors[r] += (clampf(cmd[r], 0.0f, max_force) - motors[r]) * response;
    float f[4];
    for (int r = 0; r < 4; ++r) f[r] = motors[r] * d->thrust_scale;
    const float total = ((f[0] + f[1]) + f[2]) + f[3];
    const float yaw = 0.025f * d->torque_scale;
    const float torque[3] = {d->arm_length * (f[1] - f[3]), d->arm_length * (f[2] - f[0]),
                             yaw * (f[0] - f[1] + f[2] - f[3])};
    float* w = x + 15;
    const float iw[3] = {d->inertia[0] * w[0], d->inertia[1] * w[1], d->inertia[2] * w[2]};
    float gyro[3];
    cross3(w, iw, gyro);
    for (int a = 0; a < 3; ++a) w[a] += ((torque[a] - gyro[a] - 0.015f * w[a]) / d->inertia[a]) * dt;
    const float v3[3] = {w[0] * dt, w[1] * dt, w[2] * dt};
    const float theta = std::sqrt(v3[0] * v3[0] + v3[1] * v3[1] + v3[2] * v3[2]);
    float dr[9];
    if (theta < 1e-6f) {
        const float m[9] = {1.0f, -v3[2], v3[1], v3[2], 1.0f, -v3[0], -v3[1], v3[0], 1.0f};
        std::memcpy(dr, m, sizeof m);
    } else {
        const float inv = 1.0f / theta;
        const float ax = v3[0] * inv, ay = v3[1] * inv, az = v3[2] * inv;
        const float c = std::cos(theta), s = std::sin(theta), oc = 1.0f - c;
        const float m[9] = {c + ax * ax * oc, ax * ay * oc - az * s, ax * az * oc + ay * s,
                            ay * ax * oc + az * s, c + ay * ay * oc, ay * az * oc - ax * s,
                            az * ax * oc - ay * s, az * ay * oc + ax * s, c + az * az * oc};
        std::memcpy(dr, m, sizeof m);
    }
    float* R = x + 6;
    float r[9];
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) r[i * 3 + j] = R[i * 3] * dr[j] + R[i * 3 + 1] * dr[3 + j] + R[i * 3 + 2] * dr[6 + j];
    static const float fx[3] = {1.0f, 0.0f, 0.0f}, fy[3] = {0.0f, 1.0f, 0.0f};
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
    const float bd[3] = {d->drag[0] * bv[0], d->drag[1] * bv[1], d->drag[2] * bv[2]};
    const float dw[3] = {R[0] * bd[0] + R[1] * bd[1] + R[2] * bd[2], R[3] * bd[0] + R[4] * bd[1] + R[5] * bd[2],
                         R[6] * bd[0] + R[7] * bd[1] + R[8] * bd[2]};
    const float acc[3] = {R[2] * total / d->mass - dw[0] / d->mass, R[5] * total / d->mass - dw[1] / d->mass,
                          R[8] * total / d->mass - d->gravity - dw[2] / d->mass};
    for (int a = 0; a < 3; ++a) {
        v[a] += acc[a] * dt;
        x[a] += v[a] * dt;
    }
    if (x[2] < 0.05f) {
        x[2] = 0.05f;
        v[2] = std::fmax(v[2], 0.0f);
    }
    return LWM_OK;
}

}  // extern "C"
