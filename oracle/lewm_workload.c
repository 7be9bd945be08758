/* lewm_workload.c — synthetic inputs of the benchmark workloads, for the CPU
 * reference arm and the tests (TEST INFRASTRUCTURE ONLY).
 *
 * The reference's default vehicle domain, tracking cost and model
 * configurations, reference-trajectory horizons, and seeded random weights in
 * the SkyJEPA weight blob's tensor order, so that the CPU arm builds the
 * benchmark workload from this library alone.  The random weights follow the
 * generator the benchmark's synthetic workload is defined with (SplitMix64;
 * per tensor Kaiming normal, U(+-1/sqrt(fan_in)), Kaiming uniform, zeros or
 * N(0, 1e-3)), so both arms plan with identical weights for a seed. */
#include "lewm_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* SkyJepaDomain::default (src/skyjepa_sim.rs:42-55). */
void orc_domain_default(lwm_domain* d) {
    d->mass = 1.3f;
    d->inertia[0] = 0.021f;
    d->inertia[1] = 0.023f;
    d->inertia[2] = 0.040f;
    d->motor_time_constant = 0.04f;
    d->drag[0] = 0.25f;
    d->drag[1] = 0.25f;
    d->drag[2] = 0.30f;
    d->thrust_scale = 1.0f;
    d->torque_scale = 1.0f;
    d->arm_length = 0.17f;
    d->gravity = 9.81f;
    d->max_thrust_weight = 4.0f;
}

/* SkyJepaTrackingCost::paper_derived (src/models/skyjepa/control.rs:28-37). */
void orc_tracking_cost_paper(lwm_tracking_cost* c) {
    c->position = 400.0f;
    c->velocity = 40.0f;
    c->attitude = 20.0f;
    c->angular_velocity = 20.0f;
    c->action[0] = 0.01f;
    c->action[1] = 0.05f;
    c->action[2] = 0.05f;
    c->action[3] = 0.10f;
}

static void tcn(lwm_tcn_config* t, uint32_t in, uint32_t c0, uint32_t c1, uint32_t c2) {
    memset(t, 0, sizeof(*t));
    t->input_dim = in;
    t->levels = 3;
    t->channels[0] = c0;
    t->channels[1] = c1;
    t->channels[2] = c2;
    t->kernel_size = 3;
}

/* SkyJepaConfig::paper_derived (src/models/skyjepa/config.rs:59-78), the
 * prober's default (prober.rs:19-25) and the kinematics' (kinematics.rs:44-52);
 * `wide` is the benchmark model: latent 256, state TCN [128,128,128], action
 * TCN [4,4,4]. */
void orc_skyjepa_config(int wide, lwm_skyjepa_config* c) {
    memset(c, 0, sizeof(*c));
    c->state_dim = 18;
    c->action_dim = 4;
    c->history_steps = 10;
    c->rollout_steps = 20;
    c->latent_dim = wide ? 256 : 24;
    if (wide) {
        tcn(&c->state_encoder, 18, 128, 128, 128);
        tcn(&c->action_encoder, 4, 4, 4, 4);
    } else {
        tcn(&c->state_encoder, 18, 8, 8, 16);
        tcn(&c->action_encoder, 4, 4, 4, 8);
    }
    c->prober_hidden_dim = 32;
    c->prober_hidden_layers = 2;
    c->kinematics.mass = 1.3;
    c->kinematics.gravity = 9.81;
    c->kinematics.hover_throttle = 0.2;
    c->kinematics.action_space = LWM_ACTION_SPACE_ROTOR_FORCES;
}

/* skyjepa_reference_horizon (src/skyjepa_task.rs:44-55): the reference
 * states at time + i dt, i = 1..horizon. */
void orc_reference_horizon(int kind, float time, float dt, uint32_t horizon, float radius, float period,
                           float* out) {
    for (uint32_t i = 1; i <= horizon; ++i)
        orc_reference_state(kind, time + (float)i * dt, radius, period, out + (size_t)(i - 1) * 18);
}

/* ---- seeded weights */

typedef struct {
    uint64_t state;
} mix64;

static uint64_t mix_next(mix64* m) {
    m->state += 0x9E3779B97F4A7C15ull;
    uint64_t v = m->state;
    v = (v ^ (v >> 30)) * 0xBF58476D1CE4E5B9ull;
    v = (v ^ (v >> 27)) * 0x94D049BB133111EBull;
    return v ^ (v >> 31);
}
static double mix_unit53(mix64* m) { return ((double)(mix_next(m) >> 11) + 0.5) * (1.0 / 9007199254740992.0); }
static double mix_normal(mix64* m) {
    const double u1 = mix_unit53(m), u2 = mix_unit53(m);
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

typedef struct {
    size_t n, fan_in;
    int kind; /* 0 Kaiming normal, 1 U(+-1/sqrt(fan_in)), 2 Kaiming uniform, 3 zeros, 4 N(0, 1e-3) */
} wspec;

static void put(wspec* out, size_t* idx, size_t n, size_t fan_in, int kind) {
    if (out) {
        out[*idx].n = n;
        out[*idx].fan_in = fan_in;
        out[*idx].kind = kind;
    }
    ++*idx;
}

/* The tensors of the weight blob in order (TemporalConvEncoder blocks:
 * conv1 weight/bias, conv2 weight/bias, a 1x1 residual weight/bias when the
 * width changes; the state projection; the action encoder; GRU weight_ih,
 * weight_hh, bias_ih, bias_hh; the prober's layers). */
static void tcn_specs(const lwm_tcn_config* t, wspec* out, size_t* idx) {
    uint32_t in = t->input_dim;
    for (uint32_t l = 0; l < t->levels; ++l) {
        const uint32_t o = t->channels[l];
        const size_t k = t->kernel_size;
        put(out, idx, (size_t)o * in * k, in * k, 0);
        put(out, idx, o, in * k, 1);
        put(out, idx, (size_t)o * o * k, o * k, 0);
        put(out, idx, o, o * k, 1);
        if (in != o) {
            put(out, idx, (size_t)o * in, in, 0);
            put(out, idx, o, in, 1);
        }
        in = o;
    }
}

static size_t skyjepa_specs(const lwm_skyjepa_config* c, wspec* out) {
    size_t idx = 0;
    tcn_specs(&c->state_encoder, out, &idx);
    const uint32_t H = c->latent_dim;
    const uint32_t so = c->state_encoder.channels[c->state_encoder.levels - 1];
    put(out, &idx, (size_t)H * so, so, 0);
    put(out, &idx, H, so, 1);
    tcn_specs(&c->action_encoder, out, &idx);
    const uint32_t E = c->action_encoder.channels[c->action_encoder.levels - 1];
    put(out, &idx, (size_t)3 * H * E, E, 2);
    put(out, &idx, (size_t)3 * H * H, H, 2);
    put(out, &idx, (size_t)3 * H, H, 3);
    put(out, &idx, (size_t)3 * H, H, 3);
    const uint32_t hid = c->prober_hidden_dim;
    put(out, &idx, (size_t)hid * H, H, 0);
    put(out, &idx, hid, H, 1);
    for (uint32_t i = 0; i + 1 < c->prober_hidden_layers; ++i) {
        put(out, &idx, (size_t)hid * hid, hid, 0);
        put(out, &idx, hid, hid, 1);
    }
    put(out, &idx, (size_t)15 * hid, hid, 4);
    put(out, &idx, 15, hid, 3);
    return idx;
}

/* Fills the count floats of the blob; 0 on success, -1 when count does not
 * match the configuration. */
int orc_skyjepa_random_weights(const lwm_skyjepa_config* c, uint64_t seed, float* out, size_t count) {
    const size_t n = skyjepa_specs(c, NULL);
    wspec* specs = (wspec*)malloc(n * sizeof(wspec));
    if (!specs) return -1;
    skyjepa_specs(c, specs);
    size_t total = 0;
    for (size_t i = 0; i < n; ++i) total += specs[i].n;
    if (total != count) {
        free(specs);
        return -1;
    }
    mix64 rng = {seed ^ 0x6C65776D62323030ull};
    size_t off = 0;
    for (size_t i = 0; i < n; ++i) {
        const double fan = (double)specs[i].fan_in;
        for (size_t j = 0; j < specs[i].n; ++j) {
            double v = 0.0;
            switch (specs[i].kind) {
                case 0: v = mix_normal(&rng) * sqrt(2.0 / fan); break;
                case 1: v = (2.0 * mix_unit53(&rng) - 1.0) * (1.0 / sqrt(fan)); break;
                case 2: v = (2.0 * mix_unit53(&rng) - 1.0) * sqrt(6.0 / fan); break;
                case 3: v = 0.0; break;
                default: v = mix_normal(&rng) * 1e-3; break;
            }
            out[off + j] = (float)v;
        }
        off += specs[i].n;
    }
    free(specs);
    return 0;
}
