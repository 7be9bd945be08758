/*
 * lewm_oracle.h — CPU oracle for the planner hot path.  TEST INFRASTRUCTURE:
 * only the tests, the smoke check and the CPU-baseline leg of the benchmark
 * use this library, and only as the checker / timed CPU reference.  The
 * product library never links or calls it.
 *
 * A plain-C restatement of le-wm-nv's planner math (Rust, not buildable here:
 * no Rust toolchain in this image).  Each function cites the reference
 * path:line it follows.  Arithmetic is f32 in the reference's operation order
 * (Candle's CPU kernels compute element-wise in f32); the library is compiled
 * with -ffp-contract=off so no multiply-add is fused behind our back.
 *
 * Third-party numerics the reference delegates to Candle 0.10.2 (not vendored
 * in the reference tree, so restated from their published definitions and
 * recorded as assumptions): Conv1d (cross-correlation, weight [out,in,k]),
 * Linear (x W^T + b), GRU step (PyTorch gate order r,z,n;
 * h' = z*h - (z-1)*n), gelu = tanh approximation, sigmoid = 1/(1+exp(-x)),
 * softmax = exp(x-max)/sum, var = unbiased, mean = sum * (1/n).
 */
#ifndef LEWM_ORACLE_H
#define LEWM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#include "../include/lewm_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

void orc_set_threads(int threads);
int orc_get_threads(void);

/* ---- RNG: Philox4x32-10 (Salmon et al., SC'11) + Box-Muller normals ---- */
void orc_philox4x32_10(uint64_t counter, uint64_t key, uint32_t out[4]);
float orc_normal_at(uint64_t seed, uint64_t index);
void orc_normals(uint64_t seed, uint64_t offset, size_t count, float* out);

/* ---- planner pieces (src/planner.rs) ---- */
void orc_sample(const float* mean, const float* std, const float* noise, const float* low,
                const float* high, uint32_t B, uint32_t S, uint32_t T, uint32_t A, float* out);
void orc_color_noise(const float* in, float* out, uint32_t B, uint32_t S, uint32_t T, uint32_t A,
                     float beta);
void orc_inject_carried(float* cand, const float* carried, uint32_t carried_count, uint32_t keep,
                        uint32_t B, uint32_t S, uint32_t T, uint32_t A);
void orc_mppi_weighted(const float* cand, const float* scores, uint32_t B, uint32_t S, uint32_t T,
                       uint32_t A, float temperature, float* out);
void orc_lowest_k(const float* scores, uint32_t B, uint32_t S, uint32_t k, uint32_t* out);
void orc_gather(const float* cand, const uint32_t* idx, uint32_t B, uint32_t S, uint32_t k,
                uint32_t T, uint32_t A, float* out);
void orc_refit(const float* elites, uint32_t B, uint32_t k, uint32_t T, uint32_t A,
               float min_std, float* mean, float* std);
void orc_momentum(const float* prev, const float* cur, size_t n, float alpha, float* out);
void orc_min_std(float* std, size_t n, float min_std);
void orc_shift(const float* seq, uint32_t B, uint32_t T, uint32_t A, float* out);

/* ---- rotor physics ---- */
void orc_plant_step(const lwm_domain* d, float* state18, float* motors4, const float* cmd4,
                    float dt);
void orc_nominal_rollout(const float* initial, const float* actions, const float* motors,
                         uint32_t N, uint32_t T, float dt, uint32_t substeps,
                         const lwm_domain* d, float* out);
void orc_nominal_rollout_k4(const float* initial, const float* actions, const float* motors,
                            uint32_t N, uint32_t T, float dt, uint32_t substeps,
                            const lwm_domain* d, float* out);
void orc_tracking_scores(const float* pred, const float* actions, const float* ref_states,
                         const float* ref_actions, const lwm_tracking_cost* cost, uint32_t B,
                         uint32_t S, uint32_t T, float* out);
/* SkyJepaNominalScorer::score_candidates; domains: B entries or NULL. */
void orc_nominal_scores(const float* initial, const float* motors, const float* ref_states,
                        const float* ref_actions, const lwm_tracking_cost* cost, float dt,
                        float trim_scale, uint32_t substeps, const lwm_domain* domain,
                        const lwm_domain* domains, const float* cand, uint32_t B, uint32_t S,
                        uint32_t T, float* scores, float* states_out);

/* ---- SkyJEPA learned model ---- */
typedef struct orc_skyjepa orc_skyjepa;
orc_skyjepa* orc_skyjepa_new(const lwm_skyjepa_config* cfg, const float* weights, size_t count);
/* Switch a model to the bf16 tensor-core rollout's rounding (weights
 * re-rounded in place; not reversible). */
void orc_skyjepa_set_tensor_core_rounding(orc_skyjepa* m);
void orc_skyjepa_free(orc_skyjepa* m);
size_t orc_skyjepa_weight_count(const lwm_skyjepa_config* cfg);
/* which = 0 state encoder, 1 action encoder; x [N, time, in] -> out [N, C_last] */
void orc_tcn_forward_last(const orc_skyjepa* m, int which, const float* x, uint32_t N,
                          uint32_t time, float* out);
void orc_initial_latent(const orc_skyjepa* m, const float* norm_state_hist, uint32_t B,
                        float* out);
void orc_gru_step(const orc_skyjepa* m, const float* x, const float* h, uint32_t N, float* out);
void orc_rollout_latents(const orc_skyjepa* m, const float* norm_state_hist,
                         const float* norm_action_hist, const float* norm_cand, uint32_t B,
                         uint32_t S, uint32_t T, float* out);
void orc_prober(const orc_skyjepa* m, const float* latents, uint32_t N, float* out15);
void orc_integrate_k3(const float* initial, const float* actions, const float* dt,
                      const float* residual, const float* map, uint32_t N, uint32_t T,
                      const lwm_kinematic_config* kin, float* out);
void orc_integrate_reference(const float* initial, const float* actions, const float* dt,
                             const float* residual, const float* map, uint32_t N, uint32_t T,
                             const lwm_kinematic_config* kin, float* out);
void orc_so3_exp(const float* w3, float* out9);
/* SkyJepaMppiScorer::score_candidates with its context. */
void orc_skyjepa_scores(const orc_skyjepa* m, const float* state_mean, const float* state_std,
                        const float* action_mean, const float* action_std,
                        const float* state_hist, const float* action_hist,
                        const float* ref_states, const float* ref_actions,
                        const lwm_tracking_cost* cost, float dt, const float* cand, uint32_t B,
                        uint32_t S, uint32_t T, const float* masses, float* scores, float* states_out);

/* ---- planners ---- */
typedef void (*orc_score_fn)(void* user, const float* cand, uint32_t B, uint32_t S, uint32_t T,
                             uint32_t A, float* scores);

/* Outputs (nullable unless noted): sequence [B,T,A] (required), scores
 * [B,S], best [B], warm_out [B,T,A], last_cand [B,S,T,A].  noise: injected
 * draws [iterations,B,S,T,A] or NULL for Philox(seed, offset). */
int orc_mppi_plan(const lwm_mppi_config* cfg, const float* warm_start, uint32_t B,
                  const float* noise, uint64_t seed, uint64_t offset, orc_score_fn fn,
                  void* user, float* sequence, float* scores, uint32_t* best, float* warm_out,
                  float* last_cand);
/* elites_out (nullable): every iteration's lowest_score_indices
 * [iterations][B][elites]; iter_scores_out (nullable): every iteration's
 * candidate scores [iterations][B][S]. */
int orc_cem_plan(const lwm_cem_config* cfg, uint32_t B, const float* noise, uint64_t seed,
                 uint64_t offset, orc_score_fn fn, void* user, float* sequence, float* scores,
                 uint32_t* best, float* last_cand, uint32_t* elites_out, float* iter_scores_out);
int orc_icem_plan(const lwm_icem_config* cfg, const float* warm_start, uint32_t B,
                  const float* noise, uint64_t seed, uint64_t offset, orc_score_fn fn,
                  void* user, float* sequence, float* scores, uint32_t* best, float* warm_out,
                  float* last_cand, uint32_t* elites_out, float* iter_scores_out);
/* IcemPlanner::trace_device (src/planner.rs:900-1010): as orc_icem_plan plus
 * trace [iterations][4][B] = mean, best-candidate, elite-mean and
 * updated-mean scores of every iteration. */
int orc_icem_trace(const lwm_icem_config* cfg, const float* warm_start, uint32_t B, const float* noise,
                   uint64_t seed, uint64_t offset, orc_score_fn fn, void* user, float* sequence, float* scores,
                   uint32_t* best, float* warm_out, float* trace);

/* Scorer adapters usable as orc_score_fn (user = the matching struct). */
typedef struct orc_nominal_ctx {
    const float* initial;
    const float* motors;
    const float* ref_states;
    const float* ref_actions;
    lwm_tracking_cost cost;
    float dt;
    float trim_scale;
    uint32_t substeps;
    lwm_domain domain;
    const lwm_domain* domains;
} orc_nominal_ctx;
void orc_nominal_score_fn(void* user, const float* cand, uint32_t B, uint32_t S, uint32_t T,
                          uint32_t A, float* scores);

typedef struct orc_skyjepa_ctx {
    const orc_skyjepa* model;
    const float* state_mean;
    const float* state_std;
    const float* action_mean;
    const float* action_std;
    const float* state_hist;
    const float* action_hist;
    const float* ref_states;
    const float* ref_actions;
    lwm_tracking_cost cost;
    float dt;
    const float* masses; /* [B] per-vehicle mass or NULL */
} orc_skyjepa_ctx;
void orc_skyjepa_score_fn(void* user, const float* cand, uint32_t B, uint32_t S, uint32_t T,
                          uint32_t A, float* scores);

/* ---- task inputs (src/skyjepa_task.rs) ---- */
void orc_reference_state(int kind, float time, float radius, float period, float* out18);
void orc_geometric_prior(const float* current, const float* refs, uint32_t T, float dt,
                         const lwm_domain* d, float* out);

/* ---- synthetic workload inputs (lewm_workload.c) ---- */
void orc_domain_default(lwm_domain* d);
void orc_tracking_cost_paper(lwm_tracking_cost* c);
void orc_skyjepa_config(int wide, lwm_skyjepa_config* c);
void orc_reference_horizon(int kind, float time, float dt, uint32_t horizon, float radius, float period,
                           float* out);
int orc_skyjepa_random_weights(const lwm_skyjepa_config* c, uint64_t seed, float* out, size_t count);

/* ---- LeWM / WorldModel scorer (lewm_world.c) ---- */
typedef struct orc_lewm orc_lewm;
size_t orc_lewm_weight_count(const lwm_lewm_config* cfg);
orc_lewm* orc_lewm_new(const lwm_lewm_config* cfg, const float* weights, size_t count);
void orc_lewm_free(orc_lewm* m);
void orc_lewm_action_embed(const orc_lewm* m, const float* act, uint32_t n, float* out);
void orc_lewm_predict_last(const orc_lewm* m, const float* frames, const float* act_emb, uint32_t seqs, uint32_t t,
                           float* out);
void orc_lewm_scores(const orc_lewm* m, const float* emb, uint32_t h, const float* goal, const float* cand,
                     uint32_t B, uint32_t S, uint32_t T, uint32_t history, float* scores, float* last_out);
void orc_lewm_encode_vector(const orc_lewm* m, const float* obs, uint32_t n, float* out);
void orc_lewm_encode_pixels(const orc_lewm* m, const float* pixels, uint32_t n, float* out);
typedef struct orc_lewm_ctx {
    const orc_lewm* model;
    const float* emb;  /* [B, h, D] */
    const float* goal; /* [B, D] */
    uint32_t h;
    uint32_t history;
} orc_lewm_ctx;
void orc_lewm_score_fn(void* user, const float* cand, uint32_t B, uint32_t S, uint32_t T, uint32_t A,
                       float* scores);

/* ---- image preprocessing (src/media/mod.rs) ---- */
/* swm_packed_u8_to_nchw_f32 (src/media/mod.rs:1113-1194): format 0 RGB,
 * 1 BGR, 2 RGBA, 3 BGRA; history_len 0 writes [B,3,oh,ow], otherwise slot
 * `history_slot` of [B,history_len,3,oh,ow]. */
void orc_preprocess_packed(const uint8_t* input, uint32_t B, uint32_t H, uint32_t W, uint32_t format,
                           uint32_t out_h, uint32_t out_w, const float* mean3, const float* std3,
                           uint32_t history_len, uint32_t history_slot, float* out);
/* swm_nv12_to_nchw_f32 (src/media/mod.rs:1196-1333): colour space 0
 * BT.601 video, 1 BT.709 video, 2 BT.601 full, 3 BT.709 full. */
void orc_preprocess_nv12(const uint8_t* y_plane, const uint8_t* uv_plane, uint32_t B, uint32_t H, uint32_t W,
                         uint32_t color_space, uint32_t out_h, uint32_t out_w, const float* mean3,
                         const float* std3, uint32_t history_len, uint32_t history_slot, float* out);

#ifdef __cplusplus
}
#endif

#endif
