/*
 * lewm_oracle.c — CPU oracle (TEST INFRASTRUCTURE ONLY; see lewm_oracle.h).
 *
 * Restates le-wm-nv's planner hot path in C, function by function, citing
 * the reference path:line each one follows.  f32 arithmetic in the
 * reference's operation order; OpenMP over candidate rows where the
 * reference batches candidates.
 */
#include "lewm_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 1;

void orc_set_threads(int threads) { g_threads = threads < 1 ? 1 : threads; }
int orc_get_threads(void) { return g_threads; }

/* ------------------------------------------------------------------ RNG */

/* Philox4x32-10 counter-based generator, as published by Salmon, Moraes,
 * Dror and Shaw ("Parallel random numbers: as easy as 1, 2, 3", SC 2011):
 * ten rounds of two 32x32->64 multiplies with key schedule bumps between
 * rounds.  Counter words = (lo, hi) of the 64-bit block index, 0, 0. */
void orc_philox4x32_10(uint64_t counter, uint64_t key, uint32_t out[4]) {
    uint32_t c0 = (uint32_t)counter, c1 = (uint32_t)(counter >> 32), c2 = 0u, c3 = 0u;
    uint32_t k0 = (uint32_t)key, k1 = (uint32_t)(key >> 32);
    for (int round = 0; round < 10; ++round) {
        uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        uint32_t n1 = (uint32_t)p1;
        uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        uint32_t n3 = (uint32_t)p0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* Draw `index` of the stream for `seed`: block index>>2 of Philox gives four
 * words; words (0,1) and (2,3) are Box-Muller pairs; even lanes take the
 * cosine branch, odd lanes the sine branch.  Uniforms are (2k+1) * 2^-24
 * with k the top 23 bits of a word, so they lie strictly inside (0, 1). */
float orc_normal_at(uint64_t seed, uint64_t index) {
    uint32_t w[4];
    orc_philox4x32_10(index >> 2, seed, w);
    unsigned lane = (unsigned)(index & 3u);
    unsigned pair = lane >> 1;
    double u1 = (double)(2u * (w[2 * pair] >> 9) + 1u) * (1.0 / 16777216.0);
    double u2 = (double)(2u * (w[2 * pair + 1] >> 9) + 1u) * (1.0 / 16777216.0);
    double r = sqrt(-2.0 * log(u1));
    double angle = 2.0 * M_PI * u2;
    return (float)((lane & 1u) ? r * sin(angle) : r * cos(angle));
}

void orc_normals(uint64_t seed, uint64_t offset, size_t count, float* out) {
    for (size_t i = 0; i < count; ++i) out[i] = orc_normal_at(seed, offset + i);
}

/* --------------------------------------------------------- planner pieces */

/* Candle's f32 maximum / minimum: (a < b) ? b : a and (a > b) ? b : a. */
static inline float fmax_candle(float a, float b) { return a < b ? b : a; }
static inline float fmin_candle(float a, float b) { return a > b ? b : a; }

/* sample_candidates + inject_mean_candidate + clamp_actions
 * (src/planner.rs:1152-1172, 1198-1208, 1614-1616):
 * cand = mean + noise * std; slot 0 = mean; clamp to [low, high]. */
void orc_sample(const float* mean, const float* std, const float* noise, const float* low,
                const float* high, uint32_t B, uint32_t S, uint32_t T, uint32_t A, float* out) {
    for (uint32_t b = 0; b < B; ++b)
        for (uint32_t s = 0; s < S; ++s)
            for (uint32_t t = 0; t < T; ++t)
                for (uint32_t a = 0; a < A; ++a) {
                    size_t ms = ((size_t)b * T + t) * A + a;
                    size_t ci = (((size_t)b * S + s) * T + t) * A + a;
                    float v;
                    if (s == 0) {
                        v = mean[ms];
                    } else {
                        float scaled = noise[ci] * std[ms];
                        v = mean[ms] + scaled;
                    }
                    v = fmax_candle(v, low[a]);
                    v = fmin_candle(v, high[a]);
                    out[ci] = v;
                }
}

/* color_temporal_noise + swm_temporal_color_noise_f32
 * (src/planner.rs:1516-1586, 1852-1896): per (batch, sample, action) lane an
 * EMA with smooth = clamp(beta/(beta+1), 0, 0.98), then centre and scale by
 * 1/sqrt(var/T + 1e-6).  Identity when beta == 0 or T <= 1. */
void orc_color_noise(const float* in, float* out, uint32_t B, uint32_t S, uint32_t T, uint32_t A,
                     float beta) {
    size_t n = (size_t)B * S * T * A;
    if (beta == 0.0f || T <= 1) {
        if (out != in) memcpy(out, in, n * sizeof(float));
        return;
    }
    float smooth = beta / (beta + 1.0f);
    if (smooth < 0.0f) smooth = 0.0f;
    if (smooth > 0.98f) smooth = 0.98f;
    float keep = 1.0f - smooth;
    size_t sequences = (size_t)B * S * A;
    for (size_t idx = 0; idx < sequences; ++idx) {
        size_t action = idx % A;
        size_t sample = idx / A;
        size_t base = sample * T * A + action;
        float prev = in[base];
        float mean = 0.0f;
        for (uint32_t t = 0; t < T; ++t) {
            size_t off = base + (size_t)t * A;
            float raw = in[off];
            prev = (t == 0) ? raw : fmaf(smooth, prev, keep * raw);
            out[off] = prev;
            mean += prev;
        }
        mean /= (float)T;
        float var = 0.0f;
        for (uint32_t t = 0; t < T; ++t) {
            size_t off = base + (size_t)t * A;
            float c = out[off] - mean;
            out[off] = c;
            var += c * c;
        }
        float inv_std = 1.0f / sqrtf(var / (float)T + 1.0e-6f);
        for (uint32_t t = 0; t < T; ++t) out[base + (size_t)t * A] *= inv_std;
    }
}

/* inject_carried_elites (src/planner.rs:1210-1235): slots 1..1+inject take
 * the carried elites, inject = min(keep, carried, S-1). */
void orc_inject_carried(float* cand, const float* carried, uint32_t carried_count, uint32_t keep,
                        uint32_t B, uint32_t S, uint32_t T, uint32_t A) {
    if (keep == 0 || S <= 1) return;
    uint32_t inject = keep;
    if (carried_count < inject) inject = carried_count;
    if (S - 1 < inject) inject = S - 1;
    size_t seq = (size_t)T * A;
    for (uint32_t b = 0; b < B; ++b)
        for (uint32_t e = 0; e < inject; ++e)
            memcpy(cand + ((size_t)b * S + 1 + e) * seq, carried + ((size_t)b * carried_count + e) * seq,
                   seq * sizeof(float));
}

/* mppi_weighted_sequence (src/planner.rs:1588-1602): logits =
 * (s - min s) * (-1/lambda); softmax over samples; weighted candidate sum. */
void orc_mppi_weighted(const float* cand, const float* scores, uint32_t B, uint32_t S, uint32_t T,
                       uint32_t A, float temperature, float* out) {
    float mul = (float)(-(1.0 / (double)temperature));
    float* w = (float*)malloc(sizeof(float) * S);
    for (uint32_t b = 0; b < B; ++b) {
        const float* sc = scores + (size_t)b * S;
        float mn = sc[0];
        for (uint32_t s = 1; s < S; ++s) if (sc[s] < mn) mn = sc[s];
        float mx = -INFINITY;
        for (uint32_t s = 0; s < S; ++s) {
            w[s] = (sc[s] - mn) * mul + 0.0f;
            mx = fmax_candle(mx, w[s]);
        }
        float sum = 0.0f;
        for (uint32_t s = 0; s < S; ++s) { w[s] = expf(w[s] - mx); sum += w[s]; }
        for (uint32_t s = 0; s < S; ++s) w[s] = w[s] / sum;
        for (uint32_t t = 0; t < T; ++t)
            for (uint32_t a = 0; a < A; ++a) {
                float acc = 0.0f;
                for (uint32_t s = 0; s < S; ++s)
                    acc += cand[(((size_t)b * S + s) * T + t) * A + a] * w[s];
                out[((size_t)b * T + t) * A + a] = acc;
            }
    }
    free(w);
}

/* lowest_score_indices / swm_lowest_k_indices_f32 (src/planner.rs:1647-1659,
 * 1793-1850): ascending order, NaN ranks as +inf, ties to the lower index. */
typedef struct { float v; uint32_t i; } orc_vi;
static int orc_vi_cmp(const void* pa, const void* pb) {
    const orc_vi* a = (const orc_vi*)pa;
    const orc_vi* b = (const orc_vi*)pb;
    if (a->v < b->v) return -1;
    if (a->v > b->v) return 1;
    return a->i < b->i ? -1 : (a->i > b->i ? 1 : 0);
}
void orc_lowest_k(const float* scores, uint32_t B, uint32_t S, uint32_t k, uint32_t* out) {
    orc_vi* buf = (orc_vi*)malloc(sizeof(orc_vi) * S);
    for (uint32_t b = 0; b < B; ++b) {
        for (uint32_t s = 0; s < S; ++s) {
            float v = scores[(size_t)b * S + s];
            buf[s].v = (v == v) ? v : INFINITY;
            buf[s].i = s;
        }
        qsort(buf, S, sizeof(orc_vi), orc_vi_cmp);
        for (uint32_t j = 0; j < k; ++j) out[(size_t)b * k + j] = buf[j].i;
    }
    free(buf);
}

/* gather_candidate_sequences (src/planner.rs:1740-1754). */
void orc_gather(const float* cand, const uint32_t* idx, uint32_t B, uint32_t S, uint32_t k,
                uint32_t T, uint32_t A, float* out) {
    size_t seq = (size_t)T * A;
    for (uint32_t b = 0; b < B; ++b)
        for (uint32_t j = 0; j < k; ++j)
            memcpy(out + ((size_t)b * k + j) * seq, cand + ((size_t)b * S + idx[(size_t)b * k + j]) * seq,
                   seq * sizeof(float));
}

/* elites.mean(1), elites.var(1) (unbiased), sqrt, enforce_min_std
 * (src/planner.rs:516-517, 1618-1626). */
void orc_refit(const float* elites, uint32_t B, uint32_t k, uint32_t T, uint32_t A,
               float min_std, float* mean, float* std) {
    float inv_k = (float)(1.0 / (double)k);
    float inv_km1 = (float)(1.0 / (double)(k - 1));
    for (uint32_t b = 0; b < B; ++b)
        for (uint32_t t = 0; t < T; ++t)
            for (uint32_t a = 0; a < A; ++a) {
                float sum = 0.0f;
                for (uint32_t j = 0; j < k; ++j) sum += elites[(((size_t)b * k + j) * T + t) * A + a];
                float m = sum * inv_k;
                float sq = 0.0f;
                for (uint32_t j = 0; j < k; ++j) {
                    float d = elites[(((size_t)b * k + j) * T + t) * A + a] - m;
                    sq += d * d;
                }
                float var = sq * inv_km1;
                float sd = sqrtf(var);
                if (min_std != 0.0f) sd = fmax_candle(sd, min_std);
                mean[((size_t)b * T + t) * A + a] = m;
                std[((size_t)b * T + t) * A + a] = sd;
            }
}

/* momentum_update (src/planner.rs:1628-1636). */
void orc_momentum(const float* prev, const float* cur, size_t n, float alpha, float* out) {
    if (alpha == 0.0f) { memmove(out, cur, n * sizeof(float)); return; }
    if (alpha == 1.0f) { memmove(out, prev, n * sizeof(float)); return; }
    float beta = 1.0f - alpha;
    for (size_t i = 0; i < n; ++i) out[i] = prev[i] * alpha + cur[i] * beta;
}

/* enforce_min_std (src/planner.rs:1618-1626). */
void orc_min_std(float* std, size_t n, float min_std) {
    if (min_std == 0.0f) return;
    for (size_t i = 0; i < n; ++i) std[i] = fmax_candle(std[i], min_std);
}

/* shift_sequence_for_warm_start (src/planner.rs:1604-1612). */
void orc_shift(const float* seq, uint32_t B, uint32_t T, uint32_t A, float* out) {
    for (uint32_t b = 0; b < B; ++b)
        for (uint32_t t = 0; t < T; ++t) {
            uint32_t src = (t + 1 < T) ? t + 1 : T - 1;
            memcpy(out + ((size_t)b * T + t) * A, seq + ((size_t)b * T + src) * A, A * sizeof(float));
        }
}

/* ---------------------------------------------------------- rotor physics */

static void cross3(const float* l, const float* r, float* o) {
    o[0] = l[1] * r[2] - l[2] * r[1];
    o[1] = l[2] * r[0] - l[0] * r[2];
    o[2] = l[0] * r[1] - l[1] * r[0];
}

/* mat3_from_rotvec (src/data/drone_racing.rs:901-921). */
static void mat3_from_rotvec(const float* v, float* m) {
    float theta = sqrtf(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
    if (theta < 1e-6f) {
        m[0] = 1.0f; m[1] = -v[2]; m[2] = v[1];
        m[3] = v[2]; m[4] = 1.0f; m[5] = -v[0];
        m[6] = -v[1]; m[7] = v[0]; m[8] = 1.0f;
        return;
    }
    float inv = 1.0f / theta;
    float x = v[0] * inv, y = v[1] * inv, z = v[2] * inv;
    float c = cosf(theta), s = sinf(theta), oc = 1.0f - c;
    m[0] = c + x * x * oc; m[1] = x * y * oc - z * s; m[2] = x * z * oc + y * s;
    m[3] = y * x * oc + z * s; m[4] = c + y * y * oc; m[5] = y * z * oc - x * s;
    m[6] = z * x * oc - y * s; m[7] = z * y * oc + x * s; m[8] = c + z * z * oc;
}

/* normalize (src/skyjepa_sim.rs:283-291): division by the norm. */
static void normalize_div(float* v, const float* fallback) {
    float n = sqrtf(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
    if (n > 1e-6f) { v[0] /= n; v[1] /= n; v[2] /= n; }
    else { v[0] = fallback[0]; v[1] = fallback[1]; v[2] = fallback[2]; }
}

/* SkyJepaRotorPlant::step (src/skyjepa_sim.rs:206-270) with orthonormalize
 * (:272-281).  state18 = p, v, R (row-major, world_from_body), omega. */
void orc_plant_step(const lwm_domain* d, float* x, float* motors, const float* cmd, float dt) {
    if (!(dt == dt) || isinf(dt) || dt <= 0.0f) return;
    float max_force = d->mass * d->gravity * d->max_thrust_weight / 4.0f;
    float response = 1.0f - expf(-dt / d->motor_time_constant);
    for (int r = 0; r < 4; ++r) {
        float target = cmd[r];
        if (target < 0.0f) target = 0.0f;
        if (target > max_force) target = max_force;
        motors[r] += (target - motors[r]) * response;
    }
    float f[4];
    for (int r = 0; r < 4; ++r) f[r] = motors[r] * d->thrust_scale;
    float total = 0.0f;
    for (int r = 0; r < 4; ++r) total += f[r];
    float arm = d->arm_length;
    float yaw = 0.025f * d->torque_scale;
    float torque[3] = {arm * (f[1] - f[3]), arm * (f[2] - f[0]), yaw * (f[0] - f[1] + f[2] - f[3])};
    float* w = x + 15;
    float iw[3] = {d->inertia[0] * w[0], d->inertia[1] * w[1], d->inertia[2] * w[2]};
    float gyro[3];
    cross3(w, iw, gyro);
    for (int a = 0; a < 3; ++a) {
        float acc = (torque[a] - gyro[a] - 0.015f * w[a]) / d->inertia[a];
        w[a] += acc * dt;
    }
    float rv[3] = {w[0] * dt, w[1] * dt, w[2] * dt};
    float dr[9], r[9];
    mat3_from_rotvec(rv, dr);
    const float* R = x + 6;
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j)
            r[i * 3 + j] = R[i * 3] * dr[j] + R[i * 3 + 1] * dr[3 + j] + R[i * 3 + 2] * dr[6 + j];
    static const float fx[3] = {1.0f, 0.0f, 0.0f};
    static const float fy[3] = {0.0f, 1.0f, 0.0f};
    float cx[3] = {r[0], r[3], r[6]};
    normalize_div(cx, fx);
    float y0[3] = {r[1], r[4], r[7]};
    float dot = cx[0] * y0[0] + cx[1] * y0[1] + cx[2] * y0[2];
    float cy[3] = {y0[0] - dot * cx[0], y0[1] - dot * cx[1], y0[2] - dot * cx[2]};
    normalize_div(cy, fy);
    float cz[3];
    cross3(cx, cy, cz);
    float* Rn = x + 6;
    Rn[0] = cx[0]; Rn[1] = cy[0]; Rn[2] = cz[0];
    Rn[3] = cx[1]; Rn[4] = cy[1]; Rn[5] = cz[1];
    Rn[6] = cx[2]; Rn[7] = cy[2]; Rn[8] = cz[2];
    float* v = x + 3;
    /* mat3_t_mul_vec3 / mat3_mul_vec3 (src/data/drone_racing.rs:876-890) */
    float bv[3] = {Rn[0] * v[0] + Rn[3] * v[1] + Rn[6] * v[2],
                   Rn[1] * v[0] + Rn[4] * v[1] + Rn[7] * v[2],
                   Rn[2] * v[0] + Rn[5] * v[1] + Rn[8] * v[2]};
    float bd[3] = {d->drag[0] * bv[0], d->drag[1] * bv[1], d->drag[2] * bv[2]};
    float dw[3] = {Rn[0] * bd[0] + Rn[1] * bd[1] + Rn[2] * bd[2],
                   Rn[3] * bd[0] + Rn[4] * bd[1] + Rn[5] * bd[2],
                   Rn[6] * bd[0] + Rn[7] * bd[1] + Rn[8] * bd[2]};
    float up[3] = {Rn[0] * 0.0f + Rn[1] * 0.0f + Rn[2] * 1.0f,
                   Rn[3] * 0.0f + Rn[4] * 0.0f + Rn[5] * 1.0f,
                   Rn[6] * 0.0f + Rn[7] * 0.0f + Rn[8] * 1.0f};
    float acc[3] = {up[0] * total / d->mass - dw[0] / d->mass,
                    up[1] * total / d->mass - dw[1] / d->mass,
                    up[2] * total / d->mass - d->gravity - dw[2] / d->mass};
    float* p = x;
    for (int a = 0; a < 3; ++a) {
        v[a] += acc[a] * dt;
        p[a] += v[a] * dt;
    }
    if (p[2] < 0.05f) {
        p[2] = 0.05f;
        v[2] = fmax_candle(v[2], 0.0f);
    }
}

/* nominal_physics_rollout, CPU branch (src/models/skyjepa/nominal.rs:50-71):
 * each candidate's plant stepped `substeps` times per action with
 * dt / substeps, state written after every action. */
void orc_nominal_rollout(const float* initial, const float* actions, const float* motors,
                         uint32_t N, uint32_t T, float dt, uint32_t substeps,
                         const lwm_domain* d, float* out) {
    float h = dt / (float)substeps;
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (long long n = 0; n < (long long)N; ++n) {
        float x[18], m[4];
        memcpy(x, initial + (size_t)n * 18, sizeof x);
        memcpy(m, motors + (size_t)n * 4, sizeof m);
        for (uint32_t t = 0; t < T; ++t) {
            const float* a = actions + ((size_t)n * T + t) * 4;
            for (uint32_t s = 0; s < substeps; ++s) orc_plant_step(d, x, m, a, h);
            memcpy(out + ((size_t)n * T + t) * 18, x, sizeof x);
        }
    }
}

/* skyjepa_nominal_f32 (src/models/skyjepa/nominal.cu:7-65): the CUDA
 * branch's restatement; same physics, division-by-theta axis and in-loop
 * Gram-Schmidt.  Kept to show the two reference branches agree. */
static void normalize3_k4(float* v, int fallback) {
    float n = sqrtf(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
    for (int i = 0; i < 3; ++i) v[i] = n > 1e-6f ? v[i] / n : (i == fallback ? 1.0f : 0.0f);
}
void orc_nominal_rollout_k4(const float* initial, const float* actions, const float* initial_motors,
                            uint32_t N, uint32_t T, float dt, uint32_t substeps,
                            const lwm_domain* d, float* out) {
    for (uint32_t c = 0; c < N; ++c) {
        float x[18], motors[4];
        for (int i = 0; i < 18; ++i) x[i] = initial[(size_t)c * 18 + i];
        for (int i = 0; i < 4; ++i) motors[i] = initial_motors[(size_t)c * 4 + i];
        float inertia[3] = {d->inertia[0], d->inertia[1], d->inertia[2]};
        float drag[3] = {d->drag[0], d->drag[1], d->drag[2]};
        float h = dt / substeps, response = 1.0f - expf(-h / d->motor_time_constant);
        float maximum = d->mass * d->gravity * d->max_thrust_weight / 4.0f;
        for (uint32_t t = 0; t < T; ++t) {
            const float* action = actions + ((size_t)c * T + t) * 4;
            for (uint32_t sub = 0; sub < substeps; ++sub) {
                float force[4], total = 0.0f;
                for (int i = 0; i < 4; ++i) {
                    motors[i] += (fminf(maximum, fmaxf(0.0f, action[i])) - motors[i]) * response;
                    force[i] = motors[i] * d->thrust_scale;
                    total += force[i];
                }
                float torque[3] = {d->arm_length * (force[1] - force[3]),
                                   d->arm_length * (force[2] - force[0]),
                                   0.025f * d->torque_scale * (force[0] - force[1] + force[2] - force[3])};
                float iw[3] = {inertia[0] * x[15], inertia[1] * x[16], inertia[2] * x[17]};
                float gyro[3] = {x[16] * iw[2] - x[17] * iw[1], x[17] * iw[0] - x[15] * iw[2],
                                 x[15] * iw[1] - x[16] * iw[0]};
                for (int i = 0; i < 3; ++i)
                    x[15 + i] += ((torque[i] - gyro[i] - 0.015f * x[15 + i]) / inertia[i]) * h;
                float a = x[15] * h, b = x[16] * h, cc = x[17] * h;
                float theta = sqrtf(a * a + b * b + cc * cc), dr[9];
                if (theta < 1e-6f) {
                    float small[9] = {1, -cc, b, cc, 1, -a, -b, a, 1};
                    for (int i = 0; i < 9; ++i) dr[i] = small[i];
                } else {
                    a /= theta; b /= theta; cc /= theta;
                    float co = cosf(theta), si = sinf(theta), q = 1.0f - co;
                    float rot[9] = {co + a * a * q, a * b * q - cc * si, a * cc * q + b * si,
                                    b * a * q + cc * si, co + b * b * q, b * cc * q - a * si,
                                    cc * a * q - b * si, cc * b * q + a * si, co + cc * cc * q};
                    for (int i = 0; i < 9; ++i) dr[i] = rot[i];
                }
                float r[9];
                for (int row = 0; row < 3; ++row)
                    for (int col = 0; col < 3; ++col)
                        r[row * 3 + col] = x[6 + row * 3] * dr[col] + x[7 + row * 3] * dr[3 + col] +
                                           x[8 + row * 3] * dr[6 + col];
                float cx[3] = {r[0], r[3], r[6]}, cy[3] = {r[1], r[4], r[7]};
                normalize3_k4(cx, 0);
                float dot = cx[0] * cy[0] + cx[1] * cy[1] + cx[2] * cy[2];
                for (int i = 0; i < 3; ++i) cy[i] -= dot * cx[i];
                normalize3_k4(cy, 1);
                float cz[3] = {cx[1] * cy[2] - cx[2] * cy[1], cx[2] * cy[0] - cx[0] * cy[2],
                               cx[0] * cy[1] - cx[1] * cy[0]};
                for (int i = 0; i < 3; ++i) { x[6 + i * 3] = cx[i]; x[7 + i * 3] = cy[i]; x[8 + i * 3] = cz[i]; }
                float body_drag[3];
                for (int i = 0; i < 3; ++i)
                    body_drag[i] = (x[6 + i] * x[3] + x[9 + i] * x[4] + x[12 + i] * x[5]) * drag[i];
                for (int i = 0; i < 3; ++i) {
                    float dw = x[6 + i * 3] * body_drag[0] + x[7 + i * 3] * body_drag[1] +
                               x[8 + i * 3] * body_drag[2];
                    float accel = x[8 + i * 3] * total / d->mass - (i == 2 ? d->gravity : 0.0f) - dw / d->mass;
                    x[3 + i] += accel * h;
                    x[i] += x[3 + i] * h;
                }
                if (x[2] < 0.05f) { x[2] = 0.05f; x[5] = fmaxf(x[5], 0.0f); }
            }
            for (int i = 0; i < 18; ++i) out[((size_t)c * T + t) * 18 + i] = x[i];
        }
    }
}

/* tracking_scores + grouped_squared_error
 * (src/models/skyjepa/control.rs:430-452, 485-496). */
void orc_tracking_scores(const float* pred, const float* actions, const float* ref_states,
                         const float* ref_actions, const lwm_tracking_cost* cost, uint32_t B,
                         uint32_t S, uint32_t T, float* out) {
    float inv_t = (float)(1.0 / (double)T);
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (long long row = 0; row < (long long)B * S; ++row) {
        uint32_t b = (uint32_t)(row / S);
        float total = 0.0f;
        for (uint32_t t = 0; t < T; ++t) {
            const float* p = pred + ((size_t)row * T + t) * 18;
            const float* r = ref_states + ((size_t)b * T + t) * 18;
            float g[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            static const int start[4] = {0, 3, 6, 15}, len[4] = {3, 3, 9, 3};
            for (int k = 0; k < 4; ++k)
                for (int i = 0; i < len[k]; ++i) {
                    float dd = p[start[k] + i] - r[start[k] + i];
                    g[k] += dd * dd;
                }
            const float* a = actions + ((size_t)row * T + t) * 4;
            const float* ra = ref_actions + ((size_t)b * T + t) * 4;
            float act = 0.0f;
            for (int i = 0; i < 4; ++i) {
                float dd = a[i] - ra[i];
                act += (dd * dd) * cost->action[i];
            }
            float state = g[0] * cost->position + g[1] * cost->velocity;
            state = state + g[2] * cost->attitude;
            state = state + g[3] * cost->angular_velocity;
            total += state + act;
        }
        out[row] = total * inv_t;
    }
}

/* SkyJepaNominalScorer::{predict_metric_candidates, score_candidates}
 * (src/models/skyjepa/control.rs:377-427): actions * (1/trim) into the plant,
 * tracking cost on the metric candidates. */
void orc_nominal_scores(const float* initial, const float* motors, const float* ref_states,
                        const float* ref_actions, const lwm_tracking_cost* cost, float dt,
                        float trim_scale, uint32_t substeps, const lwm_domain* domain,
                        const lwm_domain* domains, const float* cand, uint32_t B, uint32_t S,
                        uint32_t T, float* scores, float* states_out) {
    size_t rows = (size_t)B * S;
    float* states = states_out ? states_out : (float*)malloc(sizeof(float) * rows * T * 18);
    float* calibrated = (float*)malloc(sizeof(float) * rows * T * 4);
    float mul = (float)(1.0 / (double)trim_scale);
    for (size_t i = 0; i < rows * T * 4; ++i) calibrated[i] = cand[i] * mul;
    float* init_b = (float*)malloc(sizeof(float) * S * 18);
    float* mot_b = (float*)malloc(sizeof(float) * S * 4);
    for (uint32_t b = 0; b < B; ++b) {
        for (uint32_t s = 0; s < S; ++s) {
            memcpy(init_b + (size_t)s * 18, initial + (size_t)b * 18, 18 * sizeof(float));
            memcpy(mot_b + (size_t)s * 4, motors + (size_t)b * 4, 4 * sizeof(float));
        }
        const lwm_domain* d = domains ? &domains[b] : domain;
        orc_nominal_rollout(init_b, calibrated + (size_t)b * S * T * 4, mot_b, S, T, dt, substeps, d,
                            states + (size_t)b * S * T * 18);
    }
    orc_tracking_scores(states, cand, ref_states, ref_actions, cost, B, S, T, scores);
    free(init_b);
    free(mot_b);
    free(calibrated);
    if (!states_out) free(states);
}

void orc_nominal_score_fn(void* user, const float* cand, uint32_t B, uint32_t S, uint32_t T,
                          uint32_t A, float* scores) {
    (void)A;
    const orc_nominal_ctx* c = (const orc_nominal_ctx*)user;
    orc_nominal_scores(c->initial, c->motors, c->ref_states, c->ref_actions, &c->cost, c->dt,
                       c->trim_scale, c->substeps, &c->domain, c->domains, cand, B, S, T, scores,
                       NULL);
}

/* ------------------------------------------------------- SkyJEPA model */

typedef struct {
    const float *w1, *b1, *w2, *b2, *wr, *br;
    uint32_t in, out, dil;
} orc_block;

typedef struct {
    uint32_t input_dim, levels, k, out_dim;
    orc_block blocks[LWM_TCN_MAX_LEVELS];
} orc_tcn;

struct orc_skyjepa {
    lwm_skyjepa_config cfg;
    orc_tcn tcn[2];
    const float *proj_w, *proj_b;
    const float *w_ih, *w_hh, *b_ih, *b_hh;
    const float *p_in_w, *p_in_b;
    const float *p_hid_w[16], *p_hid_b[16];
    const float *p_out_w, *p_out_b;
    float* storage;
    /* 1: round where the bf16 tensor-core rollout rounds (see
     * orc_skyjepa_set_tensor_core_rounding) */
    int tc_rounding;
};

static size_t tcn_layout(const lwm_tcn_config* c, orc_tcn* t, const float* base, size_t off) {
    uint32_t in = c->input_dim;
    if (t) { t->input_dim = c->input_dim; t->levels = c->levels; t->k = c->kernel_size; }
    for (uint32_t l = 0; l < c->levels; ++l) {
        uint32_t out = c->channels[l];
        size_t k = c->kernel_size;
        orc_block blk;
        memset(&blk, 0, sizeof blk);
        blk.in = in; blk.out = out; blk.dil = 1u << l;
        blk.w1 = base ? base + off : NULL; off += (size_t)out * in * k;
        blk.b1 = base ? base + off : NULL; off += out;
        blk.w2 = base ? base + off : NULL; off += (size_t)out * out * k;
        blk.b2 = base ? base + off : NULL; off += out;
        if (in != out) {
            blk.wr = base ? base + off : NULL; off += (size_t)out * in;
            blk.br = base ? base + off : NULL; off += out;
        }
        if (t) t->blocks[l] = blk;
        in = out;
    }
    if (t) t->out_dim = in;
    return off;
}

static size_t model_layout(const lwm_skyjepa_config* c, struct orc_skyjepa* m, const float* base) {
    size_t off = 0;
    uint32_t H = c->latent_dim;
    off = tcn_layout(&c->state_encoder, m ? &m->tcn[0] : NULL, base, off);
    uint32_t s_out = c->state_encoder.channels[c->state_encoder.levels - 1];
    if (m) { m->proj_w = base + off; }
    off += (size_t)H * s_out;
    if (m) { m->proj_b = base + off; }
    off += H;
    off = tcn_layout(&c->action_encoder, m ? &m->tcn[1] : NULL, base, off);
    uint32_t E = c->action_encoder.channels[c->action_encoder.levels - 1];
    if (m) m->w_ih = base + off;
    off += (size_t)3 * H * E;
    if (m) m->w_hh = base + off;
    off += (size_t)3 * H * H;
    if (m) m->b_ih = base + off;
    off += (size_t)3 * H;
    if (m) m->b_hh = base + off;
    off += (size_t)3 * H;
    uint32_t hid = c->prober_hidden_dim;
    if (m) m->p_in_w = base + off;
    off += (size_t)hid * H;
    if (m) m->p_in_b = base + off;
    off += hid;
    for (uint32_t i = 0; i + 1 < c->prober_hidden_layers; ++i) {
        if (m) m->p_hid_w[i] = base + off;
        off += (size_t)hid * hid;
        if (m) m->p_hid_b[i] = base + off;
        off += hid;
    }
    if (m) m->p_out_w = base + off;
    off += (size_t)15 * hid;
    if (m) m->p_out_b = base + off;
    off += 15;
    return off;
}

size_t orc_skyjepa_weight_count(const lwm_skyjepa_config* cfg) { return model_layout(cfg, NULL, NULL); }

orc_skyjepa* orc_skyjepa_new(const lwm_skyjepa_config* cfg, const float* weights, size_t count) {
    size_t need = model_layout(cfg, NULL, NULL);
    if (count != need || cfg->prober_hidden_layers > 16) return NULL;
    orc_skyjepa* m = (orc_skyjepa*)calloc(1, sizeof(orc_skyjepa));
    m->cfg = *cfg;
    m->storage = (float*)malloc(sizeof(float) * count);
    memcpy(m->storage, weights, sizeof(float) * count);
    model_layout(cfg, m, m->storage);
    return m;
}

/* f32 -> bf16 -> f32, round to nearest even (the rounding of
 * __float2bfloat16_rn; NaN stays NaN). */
static float round_bf16(float v) {
    uint32_t u;
    memcpy(&u, &v, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return v;
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
    memcpy(&v, &u, 4);
    return v;
}

/* The tensor-core rollout's numerics (bf16 operands, f32 accumulation and
 * state), not a reference behaviour: the recurrent and input weights and the
 * prober's first-layer weights are bf16; the GRU biases enter the GEMM as one
 * bf16 value per gate row (r: b_ir + b_hr, z: b_iz + b_hz, n: b_in and b_hn
 * apart); the action-encoder output and the copy of h that the GEMMs read are
 * rounded to bf16 every step while h itself stays f32.  It lets the bf16
 * path be checked against a model of its own rounding instead of only the
 * f32 tolerance.  The weights of `m` are re-rounded in place: make a fresh
 * model to go back to f32. */
void orc_skyjepa_set_tensor_core_rounding(orc_skyjepa* m) {
    uint32_t H = m->cfg.latent_dim, E = m->tcn[1].out_dim, hid = m->cfg.prober_hidden_dim;
    float* w_ih = (float*)m->w_ih;
    float* w_hh = (float*)m->w_hh;
    float* b_ih = (float*)m->b_ih;
    float* b_hh = (float*)m->b_hh;
    float* p_in = (float*)m->p_in_w;
    for (size_t i = 0; i < (size_t)3 * H * E; ++i) w_ih[i] = round_bf16(w_ih[i]);
    for (size_t i = 0; i < (size_t)3 * H * H; ++i) w_hh[i] = round_bf16(w_hh[i]);
    for (size_t i = 0; i < (size_t)hid * H; ++i) p_in[i] = round_bf16(p_in[i]);
    for (uint32_t u = 0; u < 2 * H; ++u) {  /* r and z rows: one combined bias */
        b_ih[u] = round_bf16(b_ih[u] + b_hh[u]);
        b_hh[u] = 0.0f;
    }
    for (uint32_t u = 2 * H; u < 3 * H; ++u) {
        b_ih[u] = round_bf16(b_ih[u]);
        b_hh[u] = round_bf16(b_hh[u]);
    }
    m->tc_rounding = 1;
}

void orc_skyjepa_free(orc_skyjepa* m) {
    if (!m) return;
    free(m->storage);
    free(m);
}

/* Candle Tensor::gelu: tanh approximation
 * 0.5 * x * (1 + tanh(sqrt(2/pi) * x * (1 + 0.044715 * x * x))). */
static inline float gelu_tanh(float v) {
    const float k = 0.7978845608028654f;
    return 0.5f * v * (1.0f + tanhf(k * v * (1.0f + 0.044715f * v * v)));
}

static inline float sigmoidf(float v) { return 1.0f / (1.0f + expf(-v)); }

/* CausalConv1d::forward (src/models/skyjepa/tcn.rs:36-43): left zero padding
 * of dilation*(k-1), then Candle conv1d (weight [out,in,k], bias added after
 * the sum). x, y: [channels, time]. */
static void causal_conv(const float* x, uint32_t in, uint32_t time, const float* w, const float* b,
                        uint32_t out, uint32_t k, uint32_t dil, float* y) {
    for (uint32_t o = 0; o < out; ++o)
        for (uint32_t t = 0; t < time; ++t) {
            float acc = 0.0f;
            for (uint32_t i = 0; i < in; ++i)
                for (uint32_t j = 0; j < k; ++j) {
                    long long src = (long long)t - (long long)(k - 1 - j) * dil;
                    if (src < 0) continue;
                    acc += w[((size_t)o * in + i) * k + j] * x[(size_t)i * time + (size_t)src];
                }
            y[(size_t)o * time + t] = acc + b[o];
        }
}

/* TemporalBlock::forward (tcn.rs:88-96) over TemporalConvEncoder
 * (tcn.rs:138-160): h = gelu(conv1 x); h = gelu(conv2 h); out = gelu(h + res). */
static void tcn_sequence(const orc_tcn* tcn, const float* x_tf, uint32_t time, float* work,
                         float* last) {
    uint32_t maxc = tcn->input_dim;
    for (uint32_t l = 0; l < tcn->levels; ++l) if (tcn->blocks[l].out > maxc) maxc = tcn->blocks[l].out;
    float* cur = work;
    float* h1 = work + (size_t)maxc * time;
    float* h2 = h1 + (size_t)maxc * time;
    float* res = h2 + (size_t)maxc * time;
    for (uint32_t i = 0; i < tcn->input_dim; ++i)
        for (uint32_t t = 0; t < time; ++t) cur[(size_t)i * time + t] = x_tf[(size_t)t * tcn->input_dim + i];
    for (uint32_t l = 0; l < tcn->levels; ++l) {
        const orc_block* bk = &tcn->blocks[l];
        causal_conv(cur, bk->in, time, bk->w1, bk->b1, bk->out, tcn->k, bk->dil, h1);
        for (size_t q = 0; q < (size_t)bk->out * time; ++q) h1[q] = gelu_tanh(h1[q]);
        causal_conv(h1, bk->out, time, bk->w2, bk->b2, bk->out, tcn->k, bk->dil, h2);
        for (size_t q = 0; q < (size_t)bk->out * time; ++q) h2[q] = gelu_tanh(h2[q]);
        if (bk->wr) {
            causal_conv(cur, bk->in, time, bk->wr, bk->br, bk->out, 1, 1, res);
        } else {
            memcpy(res, cur, sizeof(float) * bk->out * time);
        }
        for (size_t q = 0; q < (size_t)bk->out * time; ++q) cur[q] = gelu_tanh(h2[q] + res[q]);
    }
    uint32_t C = tcn->out_dim;
    for (uint32_t c = 0; c < C; ++c) last[c] = cur[(size_t)c * time + time - 1];
}

static size_t tcn_work_floats(const orc_tcn* tcn, uint32_t time) {
    uint32_t maxc = tcn->input_dim;
    for (uint32_t l = 0; l < tcn->levels; ++l) if (tcn->blocks[l].out > maxc) maxc = tcn->blocks[l].out;
    return (size_t)4 * maxc * time;
}

/* TemporalConvEncoder::forward_last (tcn.rs:155-160). */
void orc_tcn_forward_last(const orc_skyjepa* m, int which, const float* x, uint32_t N,
                          uint32_t time, float* out) {
    const orc_tcn* tcn = &m->tcn[which ? 1 : 0];
#pragma omp parallel num_threads(g_threads)
    {
        float* work = (float*)malloc(sizeof(float) * tcn_work_floats(tcn, time));
#pragma omp for schedule(static)
        for (long long n = 0; n < (long long)N; ++n)
            tcn_sequence(tcn, x + (size_t)n * time * tcn->input_dim, time, work, out + (size_t)n * tcn->out_dim);
        free(work);
    }
}

/* Linear::forward: y = x W^T + b (sum first, bias after). */
static void linear(const float* x, uint32_t in, const float* w, const float* b, uint32_t out, float* y) {
    for (uint32_t o = 0; o < out; ++o) {
        float acc = 0.0f;
        for (uint32_t i = 0; i < in; ++i) acc += x[i] * w[(size_t)o * in + i];
        y[o] = acc + b[o];
    }
}

/* SkyJepaModel::encode_state_history (model.rs:57-61): state TCN last step,
 * then state_projection. */
void orc_initial_latent(const orc_skyjepa* m, const float* norm_state_hist, uint32_t B, float* out) {
    uint32_t Hs = m->cfg.history_steps;
    const orc_tcn* tcn = &m->tcn[0];
    float* work = (float*)malloc(sizeof(float) * tcn_work_floats(tcn, Hs));
    float* last = (float*)malloc(sizeof(float) * tcn->out_dim);
    for (uint32_t b = 0; b < B; ++b) {
        tcn_sequence(tcn, norm_state_hist + (size_t)b * Hs * tcn->input_dim, Hs, work, last);
        linear(last, tcn->out_dim, m->proj_w, m->proj_b, m->cfg.latent_dim, out + (size_t)b * m->cfg.latent_dim);
    }
    free(last);
    free(work);
}

/* candle_nn GRU::step (gate order r, z, n; PyTorch convention):
 * r = sigmoid(Wir x + bir + Whr h + bhr), z = sigmoid(...),
 * n = tanh(Win x + bin + r * (Whn h + bhn)), h' = z*h - (z-1)*n. */
static void gru_row(const orc_skyjepa* m, const float* x, const float* h, float* gi, float* gh, float* out) {
    uint32_t H = m->cfg.latent_dim;
    uint32_t E = m->tcn[1].out_dim;
    if (m->tc_rounding) {  /* the GEMMs read bf16 copies of x and h */
        float* xq = (float*)malloc(sizeof(float) * (E + H));
        float* hq = xq + E;
        for (uint32_t i = 0; i < E; ++i) xq[i] = round_bf16(x[i]);
        for (uint32_t i = 0; i < H; ++i) hq[i] = round_bf16(h[i]);
        linear(xq, E, m->w_ih, m->b_ih, 3 * H, gi);
        linear(hq, H, m->w_hh, m->b_hh, 3 * H, gh);
        free(xq);
    } else {
        linear(x, E, m->w_ih, m->b_ih, 3 * H, gi);
        linear(h, H, m->w_hh, m->b_hh, 3 * H, gh);
    }
    for (uint32_t j = 0; j < H; ++j) {
        float r = sigmoidf(gi[j] + gh[j]);
        float z = sigmoidf(gi[H + j] + gh[H + j]);
        float n = tanhf(gi[2 * H + j] + r * gh[2 * H + j]);
        out[j] = z * h[j] - (z - 1.0f) * n;
    }
}

void orc_gru_step(const orc_skyjepa* m, const float* x, const float* h, uint32_t N, float* out) {
    uint32_t H = m->cfg.latent_dim;
    uint32_t E = m->tcn[1].out_dim;
    float* gi = (float*)malloc(sizeof(float) * 3 * H);
    float* gh = (float*)malloc(sizeof(float) * 3 * H);
    for (uint32_t n = 0; n < N; ++n) gru_row(m, x + (size_t)n * E, h + (size_t)n * H, gi, gh, out + (size_t)n * H);
    free(gi);
    free(gh);
}

/* Eight rows at once: every row keeps its own sequential sum order (lanes are
 * rows, never reassociated), so results equal gru_row's; the row-interleaved
 * layout lets the compiler vectorise across rows. */
#define ORC_LANES 8
static void gru_rows8(const orc_skyjepa* m, const float* x8 /*[E][8]*/, const float* hT /*[H][8]*/,
                      const float* hqT /*[H][8]: the h the GEMM reads*/, float* gi /*[3H][8]*/,
                      float* gh /*[3H][8]*/, float* outT /*[H][8]*/) {
    uint32_t H = m->cfg.latent_dim;
    uint32_t E = m->tcn[1].out_dim;
    for (uint32_t g = 0; g < 3 * H; ++g) {
        float acc[ORC_LANES] = {0};
        const float* w = m->w_ih + (size_t)g * E;
        for (uint32_t i = 0; i < E; ++i)
            for (int l = 0; l < ORC_LANES; ++l) acc[l] += x8[i * ORC_LANES + l] * w[i];
        for (int l = 0; l < ORC_LANES; ++l) gi[g * ORC_LANES + l] = acc[l] + m->b_ih[g];
    }
    for (uint32_t g = 0; g < 3 * H; ++g) {
        float acc[ORC_LANES] = {0};
        const float* w = m->w_hh + (size_t)g * H;
        for (uint32_t k = 0; k < H; ++k) {
            float wk = w[k];
            const float* hk = hqT + (size_t)k * ORC_LANES;
            for (int l = 0; l < ORC_LANES; ++l) acc[l] += hk[l] * wk;
        }
        for (int l = 0; l < ORC_LANES; ++l) gh[g * ORC_LANES + l] = acc[l] + m->b_hh[g];
    }
    for (uint32_t j = 0; j < H; ++j)
        for (int l = 0; l < ORC_LANES; ++l) {
            float r = sigmoidf(gi[j * ORC_LANES + l] + gh[j * ORC_LANES + l]);
            float z = sigmoidf(gi[(H + j) * ORC_LANES + l] + gh[(H + j) * ORC_LANES + l]);
            float n = tanhf(gi[(2 * H + j) * ORC_LANES + l] + r * gh[(2 * H + j) * ORC_LANES + l]);
            float hv = hT[(size_t)j * ORC_LANES + l];
            outT[(size_t)j * ORC_LANES + l] = z * hv - (z - 1.0f) * n;
        }
}

/* SkyJepaModel::rollout_candidates (model.rs:161-223): windows of
 * [history(H-1) ++ candidates(T)] at offsets t..t+H through the action TCN
 * (each window zero-padded independently), state history once through the
 * state TCN + projection, then T GRU steps; latents[t] = h_{t+1}. */
void orc_rollout_latents(const orc_skyjepa* m, const float* norm_state_hist,
                         const float* norm_action_hist, const float* norm_cand, uint32_t B,
                         uint32_t S, uint32_t T, float* out) {
    uint32_t Hs = m->cfg.history_steps;
    uint32_t A = m->cfg.action_dim;
    uint32_t H = m->cfg.latent_dim;
    uint32_t E = m->tcn[1].out_dim;
    float* h0 = (float*)malloc(sizeof(float) * (size_t)B * H);
    orc_initial_latent(m, norm_state_hist, B, h0);
    uint32_t groups_per_b = (S + ORC_LANES - 1) / ORC_LANES;
#pragma omp parallel num_threads(g_threads)
    {
        const orc_tcn* tcn = &m->tcn[1];
        float* work = (float*)malloc(sizeof(float) * tcn_work_floats(tcn, Hs));
        float* window = (float*)malloc(sizeof(float) * (size_t)Hs * A);
        float* emb = (float*)malloc(sizeof(float) * (size_t)T * E * ORC_LANES);
        float* hT = (float*)malloc(sizeof(float) * (size_t)H * ORC_LANES);
        float* nT = (float*)malloc(sizeof(float) * (size_t)H * ORC_LANES);
        float* qT = m->tc_rounding ? (float*)malloc(sizeof(float) * (size_t)H * ORC_LANES) : NULL;
        float* gi = (float*)malloc(sizeof(float) * (size_t)3 * H * ORC_LANES);
        float* gh = (float*)malloc(sizeof(float) * (size_t)3 * H * ORC_LANES);
        float* last = (float*)malloc(sizeof(float) * E);
#pragma omp for schedule(dynamic, 1)
        for (long long grp = 0; grp < (long long)B * groups_per_b; ++grp) {
            uint32_t b = (uint32_t)(grp / groups_per_b);
            uint32_t s0 = (uint32_t)(grp % groups_per_b) * ORC_LANES;
            for (int l = 0; l < ORC_LANES; ++l) {
                uint32_t s = s0 + (uint32_t)l;
                if (s >= S) s = S - 1; /* padding lane recomputes the last row */
                const float* cand = norm_cand + ((size_t)b * S + s) * T * A;
                for (uint32_t t = 0; t < T; ++t) {
                    for (uint32_t w = 0; w < Hs; ++w) {
                        uint32_t pos = t + w; /* position in history ++ candidates */
                        const float* src = pos < Hs - 1 ? norm_action_hist + ((size_t)b * (Hs - 1) + pos) * A
                                                        : cand + (size_t)(pos - (Hs - 1)) * A;
                        memcpy(window + (size_t)w * A, src, A * sizeof(float));
                    }
                    tcn_sequence(tcn, window, Hs, work, last);
                    for (uint32_t e = 0; e < E; ++e)
                        emb[((size_t)t * E + e) * ORC_LANES + l] = m->tc_rounding ? round_bf16(last[e]) : last[e];
                }
                for (uint32_t j = 0; j < H; ++j) hT[(size_t)j * ORC_LANES + l] = h0[(size_t)b * H + j];
            }
            for (uint32_t t = 0; t < T; ++t) {
                if (qT)
                    for (size_t q = 0; q < (size_t)H * ORC_LANES; ++q) qT[q] = round_bf16(hT[q]);
                gru_rows8(m, emb + (size_t)t * E * ORC_LANES, hT, qT ? qT : hT, gi, gh, nT);
                float* tmp = hT; hT = nT; nT = tmp;
                for (int l = 0; l < ORC_LANES; ++l) {
                    uint32_t s = s0 + (uint32_t)l;
                    if (s >= S) break;
                    float* dst = out + (((size_t)b * S + s) * T + t) * H;
                    for (uint32_t j = 0; j < H; ++j) dst[j] = hT[(size_t)j * ORC_LANES + l];
                }
            }
        }
        free(work); free(window); free(emb); free(hT); free(nT); free(qT); free(gi); free(gh); free(last);
    }
    free(h0);
}

/* SkyJepaProber::forward (prober.rs:84-102): Linear+gelu, hidden
 * Linear+gelu layers, output Linear -> 15 (residual[3], map[3x4]). */
void orc_prober(const orc_skyjepa* m, const float* latents, uint32_t N, float* out15) {
    uint32_t H = m->cfg.latent_dim, hid = m->cfg.prober_hidden_dim;
#pragma omp parallel num_threads(g_threads)
    {
        float* a = (float*)malloc(sizeof(float) * hid);
        float* b = (float*)malloc(sizeof(float) * hid);
        float* q = m->tc_rounding ? (float*)malloc(sizeof(float) * H) : NULL;
#pragma omp for schedule(static)
        for (long long n = 0; n < (long long)N; ++n) {
            const float* in = latents + (size_t)n * H;
            if (q) {  /* the prober's first GEMM reads the bf16 copy of h */
                for (uint32_t i = 0; i < H; ++i) q[i] = round_bf16(in[i]);
                in = q;
            }
            linear(in, H, m->p_in_w, m->p_in_b, hid, a);
            for (uint32_t i = 0; i < hid; ++i) a[i] = gelu_tanh(a[i]);
            for (uint32_t l = 0; l + 1 < m->cfg.prober_hidden_layers; ++l) {
                linear(a, hid, m->p_hid_w[l], m->p_hid_b[l], hid, b);
                for (uint32_t i = 0; i < hid; ++i) a[i] = gelu_tanh(b[i]);
            }
            linear(a, hid, m->p_out_w, m->p_out_b, 15, out15 + (size_t)n * 15);
        }
        free(a);
        free(b);
        free(q);
    }
}

/* lewm_skyjepa_integrate_f32 (src/models/skyjepa/kinematics.rs:377-484):
 * explicit Euler with the pre-step rotation; Rodrigues coefficients by
 * series when theta^2 < 1e-6. */
void orc_integrate_k3(const float* initial, const float* actions, const float* dt,
                      const float* residual, const float* maps, uint32_t N, uint32_t T,
                      const lwm_kinematic_config* kin, float* output) {
    float mass = (float)kin->mass, gravity = (float)kin->gravity, hover = (float)kin->hover_throttle;
    int rotor = kin->action_space == LWM_ACTION_SPACE_ROTOR_FORCES;
    for (uint32_t n = 0; n < N; ++n) {
        const float* x0 = initial + (size_t)n * 18;
        float p[3] = {x0[0], x0[1], x0[2]}, v[3] = {x0[3], x0[4], x0[5]}, r[9];
        for (int i = 0; i < 9; ++i) r[i] = x0[6 + i];
        float om[3] = {x0[15], x0[16], x0[17]};
        for (uint32_t step = 0; step < T; ++step) {
            size_t ao = ((size_t)n * T + step) * 4, vo = ((size_t)n * T + step) * 3;
            const float* a = actions + ao;
            float sdt = dt[(size_t)n * T + step];
            float ta;
            if (rotor) ta = (a[0] + a[1] + a[2] + a[3]) / mass;
            else {
                float th = fminf(1.0f, fmaxf(0.0f, a[2]));
                ta = th * gravity / hover;
            }
            float acc[3] = {r[2] * ta + residual[vo], r[5] * ta + residual[vo + 1],
                            r[8] * ta - gravity + residual[vo + 2]};
            const float* mp = maps + ao * 3;
            float ang[3];
            for (int row = 0; row < 3; ++row)
                ang[row] = mp[row * 4] * a[0] + mp[row * 4 + 1] * a[1] + mp[row * 4 + 2] * a[2] +
                           mp[row * 4 + 3] * a[3];
            for (int ax = 0; ax < 3; ++ax) { p[ax] += v[ax] * sdt; v[ax] += acc[ax] * sdt; }
            float wx = om[0] * sdt, wy = om[1] * sdt, wz = om[2] * sdt;
            float th2 = wx * wx + wy * wy + wz * wz, ca, cb;
            if (th2 < 1.0e-6f) {
                float th4 = th2 * th2;
                ca = 1.0f - th2 / 6.0f + th4 / 120.0f;
                cb = 0.5f - th2 / 24.0f + th4 / 720.0f;
            } else {
                float th = sqrtf(th2);
                ca = sinf(th) / th;
                cb = (1.0f - cosf(th)) / th2;
            }
            float dl[9] = {1.0f - cb * (wy * wy + wz * wz), cb * wx * wy - ca * wz, cb * wx * wz + ca * wy,
                           cb * wy * wx + ca * wz, 1.0f - cb * (wx * wx + wz * wz), cb * wy * wz - ca * wx,
                           cb * wz * wx - ca * wy, cb * wz * wy + ca * wx, 1.0f - cb * (wx * wx + wy * wy)};
            float nr[9];
            for (int row = 0; row < 3; ++row)
                for (int col = 0; col < 3; ++col)
                    nr[row * 3 + col] = r[row * 3] * dl[col] + r[row * 3 + 1] * dl[3 + col] + r[row * 3 + 2] * dl[6 + col];
            memcpy(r, nr, sizeof r);
            for (int ax = 0; ax < 3; ++ax) om[ax] += ang[ax] * sdt;
            float* o = output + ((size_t)n * T + step) * 18;
            o[0] = p[0]; o[1] = p[1]; o[2] = p[2];
            o[3] = v[0]; o[4] = v[1]; o[5] = v[2];
            for (int i = 0; i < 9; ++i) o[6 + i] = r[i];
            o[15] = om[0]; o[16] = om[1]; o[17] = om[2];
        }
    }
}

/* so3_exp (kinematics.rs:336-375): I + K a + K^2 b with
 * theta_safe = sqrt(theta^2 + 1e-12) and series below theta^2 < 1e-6. */
void orc_so3_exp(const float* w, float* out) {
    float x = w[0], y = w[1], z = w[2];
    float K[9] = {0.0f, -z, y, z, 0.0f, -x, -y, x, 0.0f};
    float K2[9];
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j)
            K2[i * 3 + j] = K[i * 3] * K[j] + K[i * 3 + 1] * K[3 + j] + K[i * 3 + 2] * K[6 + j];
    float th2 = x * x + y * y + z * z;
    float th4 = th2 * th2;
    float ths = sqrtf(th2 + 1e-12f);
    float ra = sinf(ths) / ths;
    float rb = (-cosf(ths) + 1.0f) / (th2 + 1e-12f);
    float sa = (th2 * (float)(-1.0 / 6.0) + 1.0f) + th4 * (float)(1.0 / 120.0);
    float sb = (th2 * (float)(-1.0 / 24.0) + 0.5f) + th4 * (float)(1.0 / 720.0);
    int small = th2 < 1e-6f;
    float a = small ? sa : ra, b = small ? sb : rb;
    for (int i = 0; i < 9; ++i) out[i] = ((i % 4 == 0) ? 1.0f : 0.0f) + K[i] * a + K2[i] * b;
}

/* integrate_metric_rollout (kinematics.rs:57-147): the differentiable
 * Candle integrator, step order p, v, R <- R exp(w dt), w. */
void orc_integrate_reference(const float* initial, const float* actions, const float* dt,
                             const float* residual, const float* maps, uint32_t N, uint32_t T,
                             const lwm_kinematic_config* kin, float* output) {
    for (uint32_t n = 0; n < N; ++n) {
        const float* x0 = initial + (size_t)n * 18;
        float p[3], v[3], r[9], om[3];
        memcpy(p, x0, sizeof p); memcpy(v, x0 + 3, sizeof v); memcpy(r, x0 + 6, sizeof r); memcpy(om, x0 + 15, sizeof om);
        for (uint32_t step = 0; step < T; ++step) {
            size_t ao = ((size_t)n * T + step) * 4, vo = ((size_t)n * T + step) * 3;
            const float* a = actions + ao;
            float sdt = dt[(size_t)n * T + step];
            float ta;
            if (kin->action_space == LWM_ACTION_SPACE_ROTOR_FORCES) {
                float sum = ((a[0] + a[1]) + a[2]) + a[3];
                ta = sum * (float)(1.0 / kin->mass);
            } else {
                float th = fminf(1.0f, fmaxf(0.0f, a[2]));
                ta = th * (float)(kin->gravity / kin->hover_throttle);
            }
            float g[3] = {0.0f, 0.0f, (float)kin->gravity};
            float up[3] = {r[2], r[5], r[8]};
            float acc[3];
            for (int i = 0; i < 3; ++i) acc[i] = (up[i] * ta - g[i]) + residual[vo + i];
            const float* mp = maps + ao * 3;
            float ang[3];
            for (int row = 0; row < 3; ++row)
                ang[row] = mp[row * 4] * a[0] + mp[row * 4 + 1] * a[1] + mp[row * 4 + 2] * a[2] + mp[row * 4 + 3] * a[3];
            float w[3];
            for (int i = 0; i < 3; ++i) { p[i] = p[i] + v[i] * sdt; }
            for (int i = 0; i < 3; ++i) { v[i] = v[i] + acc[i] * sdt; }
            for (int i = 0; i < 3; ++i) w[i] = om[i] * sdt;
            float dl[9], nr[9];
            orc_so3_exp(w, dl);
            for (int row = 0; row < 3; ++row)
                for (int col = 0; col < 3; ++col)
                    nr[row * 3 + col] = r[row * 3] * dl[col] + r[row * 3 + 1] * dl[3 + col] + r[row * 3 + 2] * dl[6 + col];
            memcpy(r, nr, sizeof r);
            for (int i = 0; i < 3; ++i) om[i] = om[i] + ang[i] * sdt;
            float* o = output + ((size_t)n * T + step) * 18;
            memcpy(o, p, sizeof p); memcpy(o + 3, v, sizeof v); memcpy(o + 6, r, sizeof r); memcpy(o + 15, om, sizeof om);
        }
    }
}

/* SkyJepaMppiScorer::{new, predict_candidates, score_candidates}
 * (src/models/skyjepa/control.rs:163-317). */
void orc_skyjepa_scores(const orc_skyjepa* m, const float* state_mean, const float* state_std,
                        const float* action_mean, const float* action_std,
                        const float* state_hist, const float* action_hist,
                        const float* ref_states, const float* ref_actions,
                        const lwm_tracking_cost* cost, float dt, const float* cand, uint32_t B,
                        uint32_t S, uint32_t T, const float* masses, float* scores, float* states_out) {
    uint32_t Hs = m->cfg.history_steps, A = m->cfg.action_dim, D = m->cfg.state_dim, H = m->cfg.latent_dim;
    size_t rows = (size_t)B * S;
    float* nsh = (float*)malloc(sizeof(float) * (size_t)B * Hs * D);
    float* nah = (float*)malloc(sizeof(float) * (size_t)B * (Hs - 1) * A);
    float* nc = (float*)malloc(sizeof(float) * rows * T * A);
    for (size_t i = 0; i < (size_t)B * Hs * D; ++i) nsh[i] = (state_hist[i] - state_mean[i % D]) / state_std[i % D];
    for (size_t i = 0; i < (size_t)B * (Hs - 1) * A; ++i) nah[i] = (action_hist[i] - action_mean[i % A]) / action_std[i % A];
    for (size_t i = 0; i < rows * T * A; ++i) nc[i] = (cand[i] - action_mean[i % A]) / action_std[i % A];
    float* lat = (float*)malloc(sizeof(float) * rows * T * H);
    orc_rollout_latents(m, nsh, nah, nc, B, S, T, lat);
    float* pr = (float*)malloc(sizeof(float) * rows * T * 15);
    orc_prober(m, lat, (uint32_t)(rows * T), pr);
    float* res = (float*)malloc(sizeof(float) * rows * T * 3);
    float* mp = (float*)malloc(sizeof(float) * rows * T * 12);
    for (size_t i = 0; i < rows * T; ++i) {
        memcpy(res + i * 3, pr + i * 15, 3 * sizeof(float));
        memcpy(mp + i * 12, pr + i * 15 + 3, 12 * sizeof(float));
    }
    float* init = (float*)malloc(sizeof(float) * rows * 18);
    for (size_t r = 0; r < rows; ++r) memcpy(init + r * 18, state_hist + ((r / S) * Hs + Hs - 1) * 18, 18 * sizeof(float));
    float* dts = (float*)malloc(sizeof(float) * rows * T);
    for (size_t i = 0; i < rows * T; ++i) dts[i] = dt;
    float* states = states_out ? states_out : (float*)malloc(sizeof(float) * rows * T * 18);
    /* one integrator call per vehicle: the reference runs one scorer (one
     * kinematics config) per vehicle when vehicles differ in mass */
    for (uint32_t b = 0; b < B; ++b) {
        lwm_kinematic_config kin = m->cfg.kinematics;
        if (masses) kin.mass = masses[b];
        size_t r0 = (size_t)b * S;
        orc_integrate_k3(init + r0 * 18, cand + r0 * T * A, dts + r0 * T, res + r0 * T * 3, mp + r0 * T * 12, S, T,
                         &kin, states + r0 * T * 18);
    }
    orc_tracking_scores(states, cand, ref_states, ref_actions, cost, B, S, T, scores);
    if (!states_out) free(states);
    free(dts); free(init); free(mp); free(res); free(pr); free(lat); free(nc); free(nah); free(nsh);
}

void orc_skyjepa_score_fn(void* user, const float* cand, uint32_t B, uint32_t S, uint32_t T,
                          uint32_t A, float* scores) {
    (void)A;
    const orc_skyjepa_ctx* c = (const orc_skyjepa_ctx*)user;
    orc_skyjepa_scores(c->model, c->state_mean, c->state_std, c->action_mean, c->action_std, c->state_hist,
                       c->action_hist, c->ref_states, c->ref_actions, &c->cost, c->dt, cand, B, S, T,
                       c->masses, scores, NULL);
}

/* ---------------------------------------------------------------- planners */

static uint64_t round_even(uint64_t n) { return (n % 2 == 0) ? n : n + 1; }

static void draw(const float* noise, uint64_t seed, uint64_t offset, uint32_t iter, size_t per_iter,
                 size_t n, float* out) {
    if (noise) memcpy(out, noise + (size_t)iter * n, n * sizeof(float));
    else orc_normals(seed, offset + (uint64_t)iter * per_iter, n, out);
}

/* MppiPlanner::plan_device (src/planner.rs:590-692). */
int orc_mppi_plan(const lwm_mppi_config* cfg, const float* warm_start, uint32_t B,
                  const float* noise, uint64_t seed, uint64_t offset, orc_score_fn fn,
                  void* user, float* sequence, float* scores, uint32_t* best, float* warm_out,
                  float* last_cand) {
    uint32_t S = cfg->samples, T = cfg->horizon, A = cfg->action_dim;
    size_t seq_n = (size_t)B * T * A, n = (size_t)B * S * T * A;
    size_t per_iter = round_even(n);
    float* mean = (float*)calloc(seq_n, sizeof(float));
    float* std = (float*)malloc(sizeof(float) * seq_n);
    float* eps = (float*)malloc(sizeof(float) * n);
    float* cand = (float*)malloc(sizeof(float) * n);
    float* sc = (float*)malloc(sizeof(float) * (size_t)B * S);
    if (warm_start) memcpy(mean, warm_start, seq_n * sizeof(float));
    for (size_t i = 0; i < seq_n; ++i)
        std[i] = cfg->has_noise_std_per_action ? cfg->noise_std_per_action[i % A] : cfg->noise_std;
    for (uint32_t it = 0; it < cfg->iterations; ++it) {
        draw(noise, seed, offset, it, per_iter, n, eps);
        orc_sample(mean, std, eps, cfg->bounds_low, cfg->bounds_high, B, S, T, A, cand);
        fn(user, cand, B, S, T, A, sc);
        orc_mppi_weighted(cand, sc, B, S, T, A, cfg->temperature, mean);
    }
    memcpy(sequence, mean, seq_n * sizeof(float));
    if (scores) memcpy(scores, sc, sizeof(float) * B * S);
    if (best) orc_lowest_k(sc, B, S, 1, best);
    if (warm_out) orc_shift(mean, B, T, A, warm_out);
    if (last_cand) memcpy(last_cand, cand, n * sizeof(float));
    free(mean); free(std); free(eps); free(cand); free(sc);
    return 0;
}

/* CemPlanner::plan_device (src/planner.rs:450-541). */
int orc_cem_plan(const lwm_cem_config* cfg, uint32_t B, const float* noise, uint64_t seed,
                 uint64_t offset, orc_score_fn fn, void* user, float* sequence, float* scores,
                 uint32_t* best, float* last_cand, uint32_t* elites_out, float* iter_scores_out) {
    uint32_t S = cfg->samples, T = cfg->horizon, A = cfg->action_dim, K = cfg->elites;
    size_t seq_n = (size_t)B * T * A, n = (size_t)B * S * T * A;
    size_t per_iter = round_even(n);
    float* mean = (float*)calloc(seq_n, sizeof(float));
    float* std = (float*)malloc(sizeof(float) * seq_n);
    float* eps = (float*)malloc(sizeof(float) * n);
    float* cand = (float*)malloc(sizeof(float) * n);
    float* sc = (float*)malloc(sizeof(float) * (size_t)B * S);
    uint32_t* idx = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)B * K);
    float* el = (float*)malloc(sizeof(float) * (size_t)B * K * T * A);
    for (size_t i = 0; i < seq_n; ++i) std[i] = cfg->init_std;
    for (uint32_t it = 0; it < cfg->iterations; ++it) {
        draw(noise, seed, offset, it, per_iter, n, eps);
        orc_sample(mean, std, eps, cfg->bounds_low, cfg->bounds_high, B, S, T, A, cand);
        fn(user, cand, B, S, T, A, sc);
        orc_lowest_k(sc, B, S, K, idx);
        if (elites_out) memcpy(elites_out + (size_t)it * B * K, idx, sizeof(uint32_t) * B * K);
        if (iter_scores_out) memcpy(iter_scores_out + (size_t)it * B * S, sc, sizeof(float) * B * S);
        orc_gather(cand, idx, B, S, K, T, A, el);
        orc_refit(el, B, K, T, A, cfg->min_std, mean, std);
    }
    memcpy(sequence, mean, seq_n * sizeof(float));
    if (scores) memcpy(scores, sc, sizeof(float) * B * S);
    if (best) orc_lowest_k(sc, B, S, 1, best);
    if (last_cand) memcpy(last_cand, cand, n * sizeof(float));
    free(mean); free(std); free(eps); free(cand); free(sc); free(idx); free(el);
    return 0;
}

/* IcemPlanner::plan_device (src/planner.rs:778-898). */
/* IcemPlanner::plan_device (src/planner.rs:778-898); with `trace`, also
 * IcemPlanner::trace_device (:900-1010): per iteration the scores of the
 * mean, the best candidate, the elite mean and the updated mean
 * ([iterations][4][B]). */
static int icem_core(const lwm_icem_config* cfg, const float* warm_start, uint32_t B, const float* noise,
                     uint64_t seed, uint64_t offset, orc_score_fn fn, void* user, float* sequence, float* scores,
                     uint32_t* best, float* warm_out, float* last_cand, float* trace, uint32_t* elites_out,
                     float* iter_scores_out) {
    uint32_t S = cfg->samples, T = cfg->horizon, A = cfg->action_dim, K = cfg->elites, keep = cfg->keep_elites;
    size_t seq_n = (size_t)B * T * A, n = (size_t)B * S * T * A;
    size_t per_iter = round_even(n);
    float* mean = (float*)calloc(seq_n, sizeof(float));
    float* std = (float*)malloc(sizeof(float) * seq_n);
    float* em = (float*)malloc(sizeof(float) * seq_n);
    float* es = (float*)malloc(sizeof(float) * seq_n);
    float* eps = (float*)malloc(sizeof(float) * n);
    float* cand = (float*)malloc(sizeof(float) * n);
    float* sc = (float*)malloc(sizeof(float) * (size_t)B * S);
    uint32_t* idx = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)B * K);
    float* el = (float*)malloc(sizeof(float) * (size_t)B * K * T * A);
    float* carried = (float*)malloc(sizeof(float) * (size_t)B * (keep ? keep : 1) * T * A);
    int have_carried = 0;
    if (warm_start) memcpy(mean, warm_start, seq_n * sizeof(float));
    for (size_t i = 0; i < seq_n; ++i) std[i] = cfg->init_std;
    for (uint32_t it = 0; it < cfg->iterations; ++it) {
        float* tr = trace ? trace + (size_t)it * 4 * B : NULL;
        if (tr) fn(user, mean, B, 1, T, A, tr);
        draw(noise, seed, offset, it, per_iter, n, eps);
        orc_color_noise(eps, eps, B, S, T, A, cfg->noise_beta);
        orc_sample(mean, std, eps, cfg->bounds_low, cfg->bounds_high, B, S, T, A, cand);
        if (have_carried) orc_inject_carried(cand, carried, keep, keep, B, S, T, A);
        fn(user, cand, B, S, T, A, sc);
        orc_lowest_k(sc, B, S, K, idx);
        if (elites_out) memcpy(elites_out + (size_t)it * B * K, idx, sizeof(uint32_t) * B * K);
        if (iter_scores_out) memcpy(iter_scores_out + (size_t)it * B * S, sc, sizeof(float) * B * S);
        orc_gather(cand, idx, B, S, K, T, A, el);
        orc_refit(el, B, K, T, A, cfg->min_std, em, es);
        if (tr) {
            for (uint32_t b = 0; b < B; ++b) tr[B + b] = sc[(size_t)b * S + idx[(size_t)b * K]];
            fn(user, em, B, 1, T, A, tr + 2 * B);
        }
        orc_momentum(mean, em, seq_n, cfg->alpha, mean);
        orc_momentum(std, es, seq_n, cfg->alpha, std);
        orc_min_std(std, seq_n, cfg->min_std);
        if (tr) fn(user, mean, B, 1, T, A, tr + 3 * B);
        if (keep > 0) {
            for (uint32_t b = 0; b < B; ++b)
                memcpy(carried + (size_t)b * keep * T * A, el + (size_t)b * K * T * A, sizeof(float) * keep * T * A);
            have_carried = 1;
        }
    }
    uint32_t* b1 = (uint32_t*)malloc(sizeof(uint32_t) * B);
    orc_lowest_k(sc, B, S, 1, b1);
    if (cfg->return_mean) memcpy(sequence, mean, seq_n * sizeof(float));
    else for (uint32_t b = 0; b < B; ++b)
        memcpy(sequence + (size_t)b * T * A, cand + ((size_t)b * S + b1[b]) * T * A, sizeof(float) * T * A);
    if (scores) memcpy(scores, sc, sizeof(float) * B * S);
    if (best) memcpy(best, b1, sizeof(uint32_t) * B);
    if (warm_out) orc_shift(sequence, B, T, A, warm_out);
    if (last_cand) memcpy(last_cand, cand, n * sizeof(float));
    free(b1); free(mean); free(std); free(em); free(es); free(eps); free(cand); free(sc); free(idx); free(el); free(carried);
    return 0;
}

int orc_icem_plan(const lwm_icem_config* cfg, const float* warm_start, uint32_t B, const float* noise, uint64_t seed,
                  uint64_t offset, orc_score_fn fn, void* user, float* sequence, float* scores, uint32_t* best,
                  float* warm_out, float* last_cand, uint32_t* elites_out, float* iter_scores_out) {
    return icem_core(cfg, warm_start, B, noise, seed, offset, fn, user, sequence, scores, best, warm_out, last_cand,
                     NULL, elites_out, iter_scores_out);
}

int orc_icem_trace(const lwm_icem_config* cfg, const float* warm_start, uint32_t B, const float* noise, uint64_t seed,
                   uint64_t offset, orc_score_fn fn, void* user, float* sequence, float* scores, uint32_t* best,
                   float* warm_out, float* trace) {
    return icem_core(cfg, warm_start, B, noise, seed, offset, fn, user, sequence, scores, best, warm_out, NULL,
                     trace, NULL, NULL);
}

/* ---------------------------------------------------------------- task */

static void normalize3_fb(const float* v, const float* fb, float* o) {
    float n = sqrtf(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
    if (n > 1e-6f) { o[0] = v[0] / n; o[1] = v[1] / n; o[2] = v[2] / n; }
    else { o[0] = fb[0]; o[1] = fb[1]; o[2] = fb[2]; }
}

static float dot3f(const float* a, const float* b) { return a[0] * b[0] + a[1] * b[1] + a[2] * b[2]; }

/* desired_rotation (src/skyjepa_task.rs:190-203). */
static void desired_rotation(const float* up, float* R) {
    float heading[3] = {1.0f, 0.0f, 0.0f};
    if (!(fabsf(up[0]) < 0.95f)) { heading[0] = 0.0f; heading[1] = 1.0f; }
    float c[3], by[3], bx[3];
    static const float fy[3] = {0.0f, 1.0f, 0.0f};
    cross3(up, heading, c);
    normalize3_fb(c, fy, by);
    cross3(by, up, c);
    normalize3_fb(c, heading, bx);
    R[0] = bx[0]; R[1] = by[0]; R[2] = up[0];
    R[3] = bx[1]; R[4] = by[1]; R[5] = up[1];
    R[6] = bx[2]; R[7] = by[2]; R[8] = up[2];
}

/* skyjepa_reference_state (src/skyjepa_task.rs:57-110). */
void orc_reference_state(int kind, float time, float radius, float period, float* s) {
    memset(s, 0, 18 * sizeof(float));
    s[2] = 1.0f;
    float omega = 2.0f * (float)M_PI / period;
    float acc[3] = {0.0f, 0.0f, 0.0f};
    float angle = omega * time;
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
    float a[3] = {acc[0], acc[1], acc[2] + 9.81f}, up[3];
    static const float fz[3] = {0.0f, 0.0f, 1.0f};
    normalize3_fb(a, fz, up);
    desired_rotation(up, s + 6);
}

/* skyjepa_geometric_action_prior (src/skyjepa_task.rs:118-162) with
 * reference_acceleration (:164-178), allocate_rotor_forces (:180-188),
 * desired_rotation_with_heading (:205-217), attitude_error_body (:219-240). */
void orc_geometric_prior(const float* cur, const float* refs, uint32_t T, float dt,
                         const lwm_domain* d, float* out) {
    for (uint32_t index = 0; index < T; ++index) {
        const float* ref = refs + (size_t)index * 18;
        float accel[3] = {0.0f, 0.0f, 0.0f};
        const float *before = NULL, *after = NULL;
        if (index + 1 < T) { before = ref; after = refs + (size_t)(index + 1) * 18; }
        else if (index > 0) { before = refs + (size_t)(index - 1) * 18; after = ref; }
        if (before) for (int a = 0; a < 3; ++a) accel[a] = (after[3 + a] - before[3 + a]) / dt;
        float fb = index == 0 ? 1.0f : 0.0f;
        float des[3];
        for (int a = 0; a < 3; ++a)
            des[a] = accel[a] + fb * (3.5f * (ref[a] - cur[a]) + 2.6f * (ref[3 + a] - cur[3 + a])) +
                     (a == 2 ? d->gravity : 0.0f);
        static const float fz[3] = {0.0f, 0.0f, 1.0f}, fxh[3] = {1.0f, 0.0f, 0.0f}, fy[3] = {0.0f, 1.0f, 0.0f};
        float up[3], hd[3], hraw[3] = {ref[6], ref[9], 0.0f};
        normalize3_fb(des, fz, up);
        normalize3_fb(hraw, fxh, hd);
        if (fabsf(dot3f(up, hd)) > 0.95f) { float h0 = hd[0]; hd[0] = -hd[1]; hd[1] = h0; hd[2] = 0.0f; }
        float c[3], by[3], bx[3], D[9];
        cross3(up, hd, c);
        normalize3_fb(c, fy, by);
        cross3(by, up, c);
        normalize3_fb(c, hd, bx);
        D[0] = bx[0]; D[1] = by[0]; D[2] = up[0];
        D[3] = bx[1]; D[4] = by[1]; D[5] = up[1];
        D[6] = bx[2]; D[7] = by[2]; D[8] = up[2];
        const float* R = index == 0 ? cur + 6 : ref + 6;
        const float* om = index == 0 ? cur + 15 : ref + 15;
        float dxc[3][3];
        for (int col = 0; col < 3; ++col) {
            float v[3] = {R[col], R[3 + col], R[6 + col]};
            dxc[col][0] = D[0] * v[0] + D[3] * v[1] + D[6] * v[2];
            dxc[col][1] = D[1] * v[0] + D[4] * v[1] + D[7] * v[2];
            dxc[col][2] = D[2] * v[0] + D[5] * v[1] + D[8] * v[2];
        }
        float P[9] = {dxc[0][0], dxc[1][0], dxc[2][0], dxc[0][1], dxc[1][1], dxc[2][1], dxc[0][2], dxc[1][2], dxc[2][2]};
        float err[3] = {0.5f * (P[7] - P[5]), 0.5f * (P[2] - P[6]), 0.5f * (P[3] - P[1])};
        float torque[3];
        for (int a = 0; a < 3; ++a) torque[a] = -d->inertia[a] * (25.0f * err[a] + 8.0f * om[a]);
        float cup[3] = {R[0] * 0.0f + R[1] * 0.0f + R[2] * 1.0f, R[3] * 0.0f + R[4] * 0.0f + R[5] * 1.0f,
                        R[6] * 0.0f + R[7] * 0.0f + R[8] * 1.0f};
        float proj = dot3f(des, cup);
        if (proj < 0.0f) proj = 0.0f;
        float total = d->mass * proj / d->thrust_scale;
        float tmax = d->mass * d->gravity * d->max_thrust_weight;
        if (total < 0.0f) total = 0.0f;
        if (total > tmax) total = tmax;
        float arm = d->arm_length * d->thrust_scale;
        float yaw = 0.025f * d->torque_scale * d->thrust_scale;
        float base = total / 4.0f;
        float f[4] = {base - torque[1] / (2.0f * arm) + torque[2] / (4.0f * yaw),
                      base + torque[0] / (2.0f * arm) - torque[2] / (4.0f * yaw),
                      base + torque[1] / (2.0f * arm) + torque[2] / (4.0f * yaw),
                      base - torque[0] / (2.0f * arm) - torque[2] / (4.0f * yaw)};
        float maximum = d->mass * d->gravity * d->max_thrust_weight / 4.0f;
        for (int r = 0; r < 4; ++r) {
            float v = f[r];
            if (v < 0.0f) v = 0.0f;
            if (v > maximum) v = maximum;
            out[(size_t)index * 4 + r] = v;
        }
    }
}

/* ------------------------------------------------------------------ image preprocessing */

static float orc_clampf(float v, float lo, float hi) { return fminf(fmaxf(v, lo), hi); }

/* swm_sample_plane (src/media/mod.rs:1201-1230): clamped bilinear tap. */
static float orc_sample_plane(const uint8_t* plane, size_t b, uint32_t h, uint32_t w, uint32_t channels,
                              uint32_t channel, float sy, float sx) {
    sy = orc_clampf(sy, 0.0f, (float)(h - 1u));
    sx = orc_clampf(sx, 0.0f, (float)(w - 1u));
    uint32_t y0 = (uint32_t)floorf(sy), x0 = (uint32_t)floorf(sx);
    uint32_t y1 = y0 + 1u < h ? y0 + 1u : y0, x1 = x0 + 1u < w ? x0 + 1u : x0;
    float wy = sy - (float)y0, wx = sx - (float)x0;
    float v00 = (float)plane[((b * h + y0) * w + x0) * channels + channel];
    float v01 = (float)plane[((b * h + y0) * w + x1) * channels + channel];
    float v10 = (float)plane[((b * h + y1) * w + x0) * channels + channel];
    float v11 = (float)plane[((b * h + y1) * w + x1) * channels + channel];
    float top = v00 + (v01 - v00) * wx;
    float bottom = v10 + (v11 - v10) * wx;
    return top + (bottom - top) * wy;
}

static size_t orc_media_index(size_t b, uint32_t c, uint32_t y, uint32_t x, uint32_t oh, uint32_t ow,
                              uint32_t history_len, uint32_t slot) {
    if (history_len == 0u) return ((b * 3u + c) * oh + y) * ow + x;
    return (((b * history_len + slot) * 3u + c) * oh + y) * ow + x;
}

/* One output element (b, c, y, x) at a time, in the kernel's order
 * (src/media/mod.rs:1134-1193). */
void orc_preprocess_packed(const uint8_t* input, uint32_t B, uint32_t H, uint32_t W, uint32_t format,
                           uint32_t oh, uint32_t ow, const float* mean, const float* stdv, uint32_t history_len,
                           uint32_t slot, float* out) {
    const uint32_t channels = format >= 2u ? 4u : 3u;
    for (size_t b = 0; b < B; ++b)
        for (uint32_t c = 0; c < 3u; ++c)
            for (uint32_t y = 0; y < oh; ++y)
                for (uint32_t x = 0; x < ow; ++x) {
                    float sy = ((float)y + 0.5f) * ((float)H / (float)oh) - 0.5f;
                    float sx = ((float)x + 0.5f) * ((float)W / (float)ow) - 0.5f;
                    if (sy < 0.0f) sy = 0.0f;
                    if (sx < 0.0f) sx = 0.0f;
                    uint32_t y0 = (uint32_t)floorf(sy), x0 = (uint32_t)floorf(sx);
                    uint32_t y1 = y0 + 1u < H ? y0 + 1u : y0, x1 = x0 + 1u < W ? x0 + 1u : x0;
                    float wy = sy - (float)y0, wx = sx - (float)x0;
                    uint32_t sc = (format == 1u || format == 3u) ? 2u - c : c;
                    float v00 = (float)input[((b * H + y0) * W + x0) * channels + sc];
                    float v01 = (float)input[((b * H + y0) * W + x1) * channels + sc];
                    float v10 = (float)input[((b * H + y1) * W + x0) * channels + sc];
                    float v11 = (float)input[((b * H + y1) * W + x1) * channels + sc];
                    float top = v00 + (v01 - v00) * wx;
                    float bottom = v10 + (v11 - v10) * wx;
                    float value = (top + (bottom - top) * wy) * 0.00392156862745098f;
                    out[orc_media_index(b, c, y, x, oh, ow, history_len, slot)] = (value - mean[c]) / stdv[c];
                }
}

/* src/media/mod.rs:1232-1332; colour matrices :1298-1318. */
void orc_preprocess_nv12(const uint8_t* yp, const uint8_t* uvp, uint32_t B, uint32_t H, uint32_t W,
                         uint32_t cs, uint32_t oh, uint32_t ow, const float* mean, const float* stdv,
                         uint32_t history_len, uint32_t slot, float* out) {
    for (size_t b = 0; b < B; ++b)
        for (uint32_t y = 0; y < oh; ++y)
            for (uint32_t x = 0; x < ow; ++x) {
                float sy = ((float)y + 0.5f) * ((float)H / (float)oh) - 0.5f;
                float sx = ((float)x + 0.5f) * ((float)W / (float)ow) - 0.5f;
                float yv = orc_sample_plane(yp, b, H, W, 1u, 0u, sy, sx);
                float u = orc_sample_plane(uvp, b, H / 2u, W / 2u, 2u, 0u, sy * 0.5f, sx * 0.5f) - 128.0f;
                float v = orc_sample_plane(uvp, b, H / 2u, W / 2u, 2u, 1u, sy * 0.5f, sx * 0.5f) - 128.0f;
                float r, g, bl;
                if (cs == 0u) {
                    float yy = fmaxf(yv - 16.0f, 0.0f) * 1.16438356f;
                    r = yy + 1.59602678f * v;
                    g = yy - 0.39176229f * u - 0.81296765f * v;
                    bl = yy + 2.01723214f * u;
                } else if (cs == 1u) {
                    float yy = fmaxf(yv - 16.0f, 0.0f) * 1.16438356f;
                    r = yy + 1.79274107f * v;
                    g = yy - 0.21324861f * u - 0.53290933f * v;
                    bl = yy + 2.11240179f * u;
                } else if (cs == 2u) {
                    r = yv + 1.402f * v;
                    g = yv - 0.344136f * u - 0.714136f * v;
                    bl = yv + 1.772f * u;
                } else {
                    r = yv + 1.5748f * v;
                    g = yv - 0.187324f * u - 0.468124f * v;
                    bl = yv + 1.8556f * u;
                }
                const float vals[3] = {orc_clampf(r, 0.0f, 255.0f) * 0.00392156862745098f,
                                       orc_clampf(g, 0.0f, 255.0f) * 0.00392156862745098f,
                                       orc_clampf(bl, 0.0f, 255.0f) * 0.00392156862745098f};
                for (uint32_t c = 0; c < 3u; ++c)
                    out[orc_media_index(b, c, y, x, oh, ow, history_len, slot)] = (vals[c] - mean[c]) / stdv[c];
            }
}
