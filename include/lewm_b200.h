/*
 * lewm_b200.h — C ABI of the B200-native sampling planner (MPPI / CEM / iCEM)
 * and its candidate scorers.
 *
 * Every entry point replaces one piece of le-wm-nv's Rust planner API; the
 * comment above each declaration names the reference item (path:line inside
 * the le-wm-nv project) it stands in for.  Plain pointers and sizes only: no
 * torch, no Candle, no Rust types.  All host pointers are read during the call
 * and never retained.  Device pointers (the *_device entry points) refer to
 * memory on the context's device and are used on the context's stream.
 *
 * Threading: every handle serialises its calls with an internal mutex.  A
 * context owns one CUDA stream; work issued through handles created from the
 * same context is ordered on that stream.
 *
 * Errors: every call returns an lwm_status.  On failure a human-readable
 * message (matching the reference's bail! texts where one exists) is stored in
 * thread-local storage and returned by lwm_last_error().
 */
#ifndef LEWM_B200_H
#define LEWM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LWM_ABI_VERSION 1
#define LWM_MAX_ACTION_DIM 16
#define LWM_TCN_MAX_LEVELS 8
#define LWM_STATE_DIM 18
#define LWM_ROTOR_COUNT 4

typedef enum lwm_status {
    LWM_OK = 0,
    LWM_INVALID_ARGUMENT = 1,
    LWM_CUDA_ERROR = 2,
    LWM_DEADLINE = 3,
    LWM_NCCL_ERROR = 4,
    LWM_TIMEOUT = 5,
    LWM_UNSUPPORTED = 6,
} lwm_status;

typedef struct lwm_ctx lwm_ctx;
typedef struct lwm_planner lwm_planner;
typedef struct lwm_scorer lwm_scorer;

/* Thread-local message of the last failing call on this thread ("" if none). */
const char* lwm_last_error(void);
/* Library version string and ABI version number. */
const char* lwm_version(void);
int lwm_abi_version(void);

/* ---------------------------------------------------------------- context */

/* Device selection: replaces DeviceSpec::Cuda(index) / Device::new_cuda
 * (src/runtime.rs:7-18).  Creates a non-blocking stream on `device`. */
lwm_status lwm_ctx_create(int device, lwm_ctx** out);
lwm_status lwm_ctx_destroy(lwm_ctx* ctx);
/* The context's cudaStream_t, for callers that interleave their own work. */
lwm_status lwm_ctx_stream(lwm_ctx* ctx, void** stream_out);
/* Waits for the context's stream.  Also reports (LWM_CUDA_ERROR, once) an
 * NV12 preprocessing launch whose source-row copies never completed since
 * the previous call; that launch's output is then incomplete. */
lwm_status lwm_ctx_synchronize(lwm_ctx* ctx);
/* Number of kernels this library has launched on the context so far. */
lwm_status lwm_ctx_launch_count(lwm_ctx* ctx, uint64_t* out);
/* Device time of the rollout kernel (the dominant kernel of a SkyJEPA plan),
 * for measurement; no counterpart in the reference.  While on, every
 * SkyJEPA plan on the context records two CUDA events on its stream around
 * the rollout launch; lwm_ctx_kernel_time_ms waits for the later one and
 * returns the milliseconds between them for the most recent plan
 * (LWM_INVALID_ARGUMENT while off or before the first timed launch). */
lwm_status lwm_ctx_set_kernel_timing(lwm_ctx* ctx, int on);
lwm_status lwm_ctx_kernel_time_ms(lwm_ctx* ctx, float* ms_out);

/* Fault injection for tests of the failure paths (no counterpart in the
 * reference, whose only failure path is the planning deadline,
 * src/planner.rs:1055-1150).  Every pipeline wait in this library's kernels
 * is bounded: a wait that gives up records where in an error word and the
 * kernel unwinds and returns (nothing traps or hangs).  These knobs make
 * such a wait run out on purpose, from the host, on a context's later
 * launches; all zero = off (the default).
 *   wait_polls            pipeline waits give up after this many polls
 *                         (0: the built-in limit);
 *   tc_skip_h_arrive      1: in the bf16 tensor-core rollout, the first GRU
 *                         epilogue warp of block 0 skips its first hand-off
 *                         of h to the MMA issuer, whose wait then runs out:
 *                         the plan returns LWM_TIMEOUT naming the site;
 *   media_skip_row_plus1  r + 1: the row-staged preprocessing producer
 *                         skips the source-row copies of output row r;
 *                         the consumers' wait runs out and
 *                         lwm_ctx_synchronize reports LWM_CUDA_ERROR.
 * NULL clears every knob. */
typedef struct lwm_test_faults {
    uint32_t wait_polls;
    uint32_t tc_skip_h_arrive;
    uint32_t media_skip_row_plus1;
} lwm_test_faults;
lwm_status lwm_ctx_set_test_faults(lwm_ctx* ctx, const lwm_test_faults* faults);

/* ---------------------------------------------------------------- planners */

/* ActionBounds + MppiConfig (src/planner.rs:67-103, 178-254).
 * deadline_ns < 0 means "no deadline" (Option<Duration>::None). */
typedef struct lwm_mppi_config {
    uint32_t horizon;
    uint32_t samples;
    uint32_t iterations;
    uint32_t action_dim;
    float bounds_low[LWM_MAX_ACTION_DIM];
    float bounds_high[LWM_MAX_ACTION_DIM];
    float noise_std;
    int32_t has_noise_std_per_action;
    float noise_std_per_action[LWM_MAX_ACTION_DIM];
    float temperature;
    int64_t deadline_ns;
    int32_t has_deadline_action;
    float deadline_action[LWM_MAX_ACTION_DIM];
    int32_t has_seed;
    uint64_t seed;
} lwm_mppi_config;

/* CemConfig (src/planner.rs:107-176). */
typedef struct lwm_cem_config {
    uint32_t horizon;
    uint32_t samples;
    uint32_t elites;
    uint32_t iterations;
    uint32_t action_dim;
    float bounds_low[LWM_MAX_ACTION_DIM];
    float bounds_high[LWM_MAX_ACTION_DIM];
    float init_std;
    float min_std;
    int64_t deadline_ns;
    int32_t has_deadline_action;
    float deadline_action[LWM_MAX_ACTION_DIM];
    int32_t has_seed;
    uint64_t seed;
} lwm_cem_config;

/* IcemConfig (src/planner.rs:256-346). */
typedef struct lwm_icem_config {
    uint32_t horizon;
    uint32_t samples;
    uint32_t elites;
    uint32_t keep_elites;
    uint32_t iterations;
    float noise_beta;
    float alpha;
    uint32_t action_dim;
    float bounds_low[LWM_MAX_ACTION_DIM];
    float bounds_high[LWM_MAX_ACTION_DIM];
    float init_std;
    float min_std;
    int32_t return_mean;
    int64_t deadline_ns;
    int32_t has_deadline_action;
    float deadline_action[LWM_MAX_ACTION_DIM];
    int32_t has_seed;
    uint64_t seed;
} lwm_icem_config;

/* Defaults of MppiConfig::new / CemConfig::new / IcemConfig::new
 * (src/planner.rs:193-208, 122-137, 275-295). */
void lwm_mppi_config_default(uint32_t horizon, uint32_t samples, uint32_t action_dim,
                             lwm_mppi_config* out);
void lwm_cem_config_default(uint32_t horizon, uint32_t samples, uint32_t elites,
                            uint32_t action_dim, lwm_cem_config* out);
void lwm_icem_config_default(uint32_t horizon, uint32_t samples, uint32_t elites,
                             uint32_t action_dim, lwm_icem_config* out);

/* MppiPlanner::new / CemPlanner::new / IcemPlanner::new
 * (src/planner.rs:553-561, 426-433, 741-749).  The configuration is validated
 * here and again on every plan (the reference validates inside plan_device,
 * src/planner.rs:451,591,779); the messages are the reference's. */
lwm_status lwm_mppi_create(lwm_ctx* ctx, const lwm_mppi_config* cfg, lwm_planner** out);
lwm_status lwm_cem_create(lwm_ctx* ctx, const lwm_cem_config* cfg, lwm_planner** out);
lwm_status lwm_icem_create(lwm_ctx* ctx, const lwm_icem_config* cfg, lwm_planner** out);
lwm_status lwm_planner_destroy(lwm_planner* planner);

/* set_warm_start_sequence / clear_warm_start / warm_start_sequence
 * (src/planner.rs:571-581, 759-769).  `sequence` is host [batch, horizon,
 * action_dim] f32.  lwm_planner_warm_start writes *batch_out = 0 when no warm
 * start is set.  CEM has no warm start (LWM_INVALID_ARGUMENT). */
lwm_status lwm_planner_set_warm_start(lwm_planner* planner, const float* sequence,
                                      uint32_t batch, uint32_t horizon, uint32_t action_dim);
lwm_status lwm_planner_clear_warm_start(lwm_planner* planner);
lwm_status lwm_planner_warm_start(lwm_planner* planner, float* sequence_out, size_t capacity,
                                  uint32_t* batch_out);
/* reset_rng_sequence / rng_offset (src/planner.rs:442-448, 583-589). */
lwm_status lwm_planner_reset_rng(lwm_planner* planner);
lwm_status lwm_planner_rng_offset(lwm_planner* planner, uint64_t* out);
/* The elite indices each iteration of the last CEM / iCEM plan selected,
 * as select_elites / lowest_score_indices return them (src/planner.rs:
 * 1647-1659, 1730-1754; ascending score, ties to the lower index), copied to
 * `out` as [iterations][batch][elites]; a sharded plan reports the global
 * candidate indices.  The reference keeps them inside plan_device; they are
 * exposed here so callers (and parity tests) can check the selection.  Sets
 * *iterations_out to the iterations the plan completed (0 before the first
 * plan or after a deadline fallback).  MPPI planners: LWM_INVALID_ARGUMENT. */
lwm_status lwm_planner_elite_indices(lwm_planner* planner, uint32_t* out, size_t capacity,
                                     uint32_t* iterations_out, uint32_t* batch_out, uint32_t* elites_out);

/* ---------------------------------------------------------------- scorers */

/* SkyJepaDomain (src/skyjepa_sim.rs:28-56). */
typedef struct lwm_domain {
    float mass;
    float inertia[3];
    float motor_time_constant;
    float drag[3];
    float thrust_scale;
    float torque_scale;
    float arm_length;
    float gravity;
    float max_thrust_weight;
} lwm_domain;
void lwm_domain_default(lwm_domain* out);
/* SkyJepaDomain::sample (src/skyjepa_sim.rs:61-86), SplitMix64 stream. */
void lwm_domain_sample(uint64_t seed, lwm_domain* out);

/* SkyJepaTrackingCost (src/models/skyjepa/control.rs:19-37). */
typedef struct lwm_tracking_cost {
    float position;
    float velocity;
    float attitude;
    float angular_velocity;
    float action[LWM_ROTOR_COUNT];
} lwm_tracking_cost;
void lwm_tracking_cost_paper(lwm_tracking_cost* out);

/* SkyJepaNominalScorer::new (src/models/skyjepa/control.rs:344-375) with the
 * rollout of nominal_physics_rollout (src/models/skyjepa/nominal.rs:17-72).
 * `substeps` is 10 in the reference scorer (control.rs:401); the domain is
 * SkyJepaDomain::default() there.  `domains` (nullable) gives one domain per
 * vehicle for fleets; NULL = `domain` for every vehicle. */
typedef struct lwm_nominal_scorer_config {
    float dt;
    float trim_scale;
    uint32_t substeps;
    lwm_tracking_cost cost;
    lwm_domain domain;
} lwm_nominal_scorer_config;
lwm_status lwm_scorer_nominal_create(lwm_ctx* ctx, const lwm_nominal_scorer_config* cfg,
                                     lwm_scorer** out);
/* Context of one plan: host arrays initial [B,18], motors [B,4],
 * reference_states [B,T,18], reference_actions [B,T,4]; domains [B] or NULL. */
lwm_status lwm_scorer_nominal_set_context(lwm_scorer* scorer, uint32_t batch, uint32_t horizon,
                                          const float* initial, const float* motors,
                                          const float* reference_states,
                                          const float* reference_actions,
                                          const lwm_domain* domains);

/* TemporalConvConfig (src/models/skyjepa/config.rs:9-14). */
typedef struct lwm_tcn_config {
    uint32_t input_dim;
    uint32_t levels;
    uint32_t channels[LWM_TCN_MAX_LEVELS];
    uint32_t kernel_size;
} lwm_tcn_config;

typedef enum lwm_action_space {
    LWM_ACTION_SPACE_BODY_RATES_THROTTLE = 0,
    LWM_ACTION_SPACE_ROTOR_FORCES = 1,
} lwm_action_space;

/* KinematicConfig (src/models/skyjepa/kinematics.rs:18-47). */
typedef struct lwm_kinematic_config {
    double mass;
    double gravity;
    double hover_throttle;
    int32_t action_space;
} lwm_kinematic_config;

/* SkyJepaConfig (src/models/skyjepa/config.rs:45-55) + SkyJepaProberConfig
 * (src/models/skyjepa/prober.rs:10-16). */
typedef struct lwm_skyjepa_config {
    uint32_t state_dim;
    uint32_t action_dim;
    uint32_t history_steps;
    uint32_t rollout_steps;
    uint32_t latent_dim;
    lwm_tcn_config state_encoder;
    lwm_tcn_config action_encoder;
    uint32_t prober_hidden_dim;
    uint32_t prober_hidden_layers;
    lwm_kinematic_config kinematics;
} lwm_skyjepa_config;

/* SkyJepaConfig::paper_derived (config.rs:59-77) with a rotor-force prober. */
void lwm_skyjepa_config_paper(lwm_skyjepa_config* out);
/* The 512-candidate learned-MPPI workload's model: latent/GRU 256, state TCN
 * [128,128,128], action TCN [4,4,4], prober 32 x 2, rotor forces. */
void lwm_skyjepa_config_wide(lwm_skyjepa_config* out);

/* Weight blob: one f32 array, tensors concatenated in this order, each
 * row-major with the shape of its VarBuilder path (model.rs:25-38, tcn.rs,
 * prober.rs:54-80):
 *   state_encoder.blocks.{l}.conv1.weight [C_l, C_{l-1}, K] .conv1.bias [C_l]
 *   state_encoder.blocks.{l}.conv2.weight [C_l, C_l, K]     .conv2.bias [C_l]
 *   state_encoder.blocks.{l}.residual.weight [C_l, C_{l-1}, 1] .residual.bias
 *       (only when C_{l-1} != C_l)
 *   state_projection.weight [latent, C_last] .bias [latent]
 *   action_encoder.blocks.{l}.*  (as above)
 *   predictor.weight_ih_l0 [3*latent, E] .weight_hh_l0 [3*latent, latent]
 *   predictor.bias_ih_l0 [3*latent] .bias_hh_l0 [3*latent]
 *   prober.input.weight [hid, latent] .bias [hid]
 *   prober.hidden.{i}.weight [hid, hid] .bias [hid]   (hidden_layers - 1 times)
 *   prober.output.weight [15, hid] .bias [15]
 * Returns the element count, or 0 for an invalid configuration. */
size_t lwm_skyjepa_weight_count(const lwm_skyjepa_config* cfg);
/* Seeded random initialisation with Candle's default init families:
 * Kaiming-normal conv/linear weights, U(+-1/sqrt(fan_in)) biases,
 * Kaiming-uniform GRU weights with zero biases, N(0, 1e-3) prober output
 * weight with zero bias.  Deterministic for (cfg, seed). */
lwm_status lwm_skyjepa_random_weights(const lwm_skyjepa_config* cfg, uint64_t seed,
                                      float* out, size_t count);

/* SkyJepaMppiScorer::new (src/models/skyjepa/control.rs:163-240).  Copies
 * the weights to the device once.  Normalisation stats are mean/std of length
 * state_dim and action_dim (SkyJepaNormalization, data/skyjepa.rs:175-178). */
lwm_status lwm_scorer_skyjepa_create(lwm_ctx* ctx, const lwm_skyjepa_config* cfg,
                                     const float* weights, size_t weight_count,
                                     const float* state_mean, const float* state_std,
                                     const float* action_mean, const float* action_std,
                                     const lwm_tracking_cost* cost, float dt,
                                     lwm_scorer** out);
/* Per-plan context (control.rs:163-240 arguments): host arrays
 * state_history [B,H,18], action_history [B,H-1,4], reference_states [B,T,18],
 * reference_actions [B,T,4].  Uploaded with one H2D copy. */
lwm_status lwm_scorer_skyjepa_set_context(lwm_scorer* scorer, uint32_t batch, uint32_t horizon,
                                          const float* state_history,
                                          const float* action_history,
                                          const float* reference_states,
                                          const float* reference_actions);
/* As lwm_scorer_skyjepa_set_context, plus an optional per-vehicle mass [B]
 * (NULL: the model's kinematics.mass for every vehicle).  The mass enters
 * the rotor-forces integrator (src/models/skyjepa/kinematics.rs:411-413);
 * the reference needs one scorer per vehicle for a fleet whose vehicles
 * differ in mass. */
lwm_status lwm_scorer_skyjepa_set_context_ex(lwm_scorer* scorer, uint32_t batch, uint32_t horizon,
                                             const float* state_history,
                                             const float* action_history,
                                             const float* reference_states,
                                             const float* reference_actions,
                                             const float* vehicle_mass);

/* Arithmetic of the learned scorer's fused MPPI iterations.
 * LWM_PRECISION_F32 (default): f32-class results.  For the model shape the
 * tensor-core rollouts take (latent 256, 4 actions, 4-channel action encoder
 * with kernel 3 over a 10-step history, prober hidden 32) and sample counts
 * that are multiples of 128, the recurrent and prober-input GEMMs run on the
 * tcgen05 tensor cores with every operand split into two fp16 halves and
 * three partial products per product (about 22 significant bits, f32
 * accumulation), gates / state / prober tail / integrator / cost in f32;
 * other shapes run the f32 CUDA-core rollout.  Both match the f32 reference
 * within 1e-4 relative.
 * LWM_PRECISION_BF16: bf16 weights and recurrent state on the tensor cores
 * with f32 accumulation, for the same shapes; costs agree with f32 within
 * about 2e-2 relative (other shapes keep the f32 rollout).
 * LWM_PRECISION_F32_CUDA_CORE: always the f32 CUDA-core rollout. */
typedef enum lwm_precision {
    LWM_PRECISION_F32 = 0,
    LWM_PRECISION_BF16 = 1,
    LWM_PRECISION_F32_CUDA_CORE = 2,
} lwm_precision;
lwm_status lwm_scorer_skyjepa_set_precision(lwm_scorer* scorer, int32_t precision);
/* Precision of the LeWM scorer's GEMMs (predictor, action embedder, pred_proj,
 * encoders).  LWM_PRECISION_F32 (default): f32 CUDA-core GEMMs.
 * LWM_PRECISION_BF16: bf16 weights (converted once) and bf16-rounded GEMM
 * inputs on the tcgen05 tensor cores with f32 accumulation; the residual
 * stream, norms, attention and the goal cost stay f32.  GEMMs whose K is not
 * a multiple of 16 (the action embedder's input) stay f32. */
lwm_status lwm_scorer_lewm_set_precision(lwm_scorer* scorer, int32_t precision);

/* A scorer supplied by the caller: the CandidateScorer trait
 * (src/planner.rs:25-32).  The callback receives device pointers on the
 * context's stream: candidates [B,S,T,A] f32 and scores [B,S] f32 to fill,
 * and returns 0 on success. */
typedef int (*lwm_score_fn)(void* user, const float* candidates, uint32_t batch,
                            uint32_t samples, uint32_t horizon, uint32_t action_dim,
                            float* scores, void* stream);
lwm_status lwm_scorer_callback_create(lwm_ctx* ctx, uint32_t batch, lwm_score_fn fn, void* user,
                                      lwm_scorer** out);

/* CandidateScorer::score_candidates (src/planner.rs:31) on device buffers:
 * candidates [B,S,T,A], scores [B,S].  Asynchronous on the context stream. */
lwm_status lwm_scorer_score_device(lwm_scorer* scorer, const float* candidates, uint32_t batch,
                                   uint32_t samples, uint32_t horizon, uint32_t action_dim,
                                   float* scores);
/* SkyJepaMppiScorer::predict_candidates / SkyJepaNominalScorer::
 * predict_metric_candidates (control.rs:246-290, 377-406): device candidates
 * [B,S,T,4] -> device states [B,S,T,18]. */
lwm_status lwm_scorer_predict_device(lwm_scorer* scorer, const float* candidates, uint32_t batch,
                                     uint32_t samples, uint32_t horizon, float* states);
lwm_status lwm_scorer_destroy(lwm_scorer* scorer);

/* ---------------------------------------------------------------- planning */

/* PlanDeadlineOutcome (src/planner.rs:348-353). */
typedef enum lwm_deadline_outcome {
    LWM_DEADLINE_NONE = 0,
    LWM_DEADLINE_WARM_START = 1,
    LWM_DEADLINE_CONFIGURED_ACTION = 2,
} lwm_deadline_outcome;

/* PlanResult (src/planner.rs:355-366) in caller-owned host buffers:
 * first_action [B*A], sequence [B*T*A], scores [B*scores_cols],
 * best_indices [B].  Any pointer may be NULL to skip that copy.
 * `scores_capacity` is the element capacity of `scores`. */
typedef struct lwm_plan_result {
    float* first_action;
    float* sequence;
    float* scores;
    size_t scores_capacity;
    uint32_t* best_indices;
    uint32_t batch;
    uint32_t scores_cols;
    uint32_t iterations_completed;
    uint64_t elapsed_ns;
    int32_t deadline_reached;
    int32_t deadline_outcome;
} lwm_plan_result;

/* PlanDeviceResult (src/planner.rs:368-379): device pointers owned by the
 * planner, valid until its next plan call. */
typedef struct lwm_plan_device_result {
    const float* first_action;
    const float* sequence;
    const float* scores;
    const uint32_t* best_indices;
    uint32_t batch;
    uint32_t scores_cols;
    uint32_t iterations_completed;
    uint64_t elapsed_ns;
    int32_t deadline_reached;
    int32_t deadline_outcome;
} lwm_plan_device_result;

/* plan (src/planner.rs:446-448, 586-588, 774-776): runs every iteration and
 * copies the result to host buffers (the only device synchronisation).
 * `injected_noise` (host, nullable) replaces the seeded sampler with fixed
 * standard-normal draws [iterations, B, S, T, A] — the parity hook. */
lwm_status lwm_plan(lwm_planner* planner, lwm_scorer* scorer, const float* injected_noise,
                    lwm_plan_result* out);
/* plan_device (src/planner.rs:450, 590, 778): asynchronous; results stay on
 * the device.  `injected_noise` is a device pointer or NULL. */
lwm_status lwm_plan_device(lwm_planner* planner, lwm_scorer* scorer,
                           const float* injected_noise, lwm_plan_device_result* out);

/* Device copy of the candidates of the last iteration [B,S,T,A] (a debugging
 * and parity hook with no reference counterpart in the public API). */
lwm_status lwm_planner_last_candidates(lwm_planner* planner, const float** candidates_device,
                                       uint32_t* samples_out);

/* ---------------------------------------------------------------- planner pieces
 * Device-buffer entry points for the building blocks the planners use; each
 * mirrors one private function of src/planner.rs and exists so that callers
 * with their own loop (and the parity tests) can run them alone. */

/* lowest_score_indices (src/planner.rs:1647-1659 and kernel :1793-1850):
 * ascending, NaN ranks as +inf, ties to the lower index; any sample count. */
lwm_status lwm_lowest_k_device(lwm_ctx* ctx, const float* scores, uint32_t batch,
                               uint32_t samples, uint32_t count, uint32_t* indices);
/* color_temporal_noise (src/planner.rs:1516-1586, kernel :1852-1896). */
lwm_status lwm_color_noise_device(lwm_ctx* ctx, const float* noise, float* out, uint32_t batch,
                                  uint32_t samples, uint32_t horizon, uint32_t action_dim,
                                  float noise_beta);
/* Seeded standard normals: draw i of stream (seed) is element i - offset of
 * `out`; the sampler the planners use. */
lwm_status lwm_normal_device(lwm_ctx* ctx, uint64_t seed, uint64_t offset, size_t count,
                             float* out);

/* ---------------------------------------------------------------- LeWM world-model scorer */

/* LeWM / WorldModel (src/models/lewm/{config,model,modules,vit}.rs,
 * src/models/world_model/{config,model}.rs): an observation encoder (vector
 * MLP or ViT + projector MLP), an action embedder, an AdaLN-conditioned
 * causal transformer predictor and a pred_proj MLP; candidates are scored by
 * the squared L2 distance of the last predicted embedding to a goal
 * embedding (LeWmSession::score_candidates, src/session.rs:46-66). */
typedef enum lwm_norm_kind {
    LWM_NORM_BATCH = 0, /* BatchNorm1d in eval mode (running statistics), eps 1e-5 */
    LWM_NORM_LAYER = 1, /* LayerNorm, eps 1e-5 */
    LWM_NORM_NONE = 2,
} lwm_norm_kind;
typedef enum lwm_encoder_kind {
    LWM_ENCODER_VECTOR_MLP = 0,
    LWM_ENCODER_VIT = 1,
} lwm_encoder_kind;
typedef struct lwm_lewm_config {
    uint32_t embed_dim;        /* D: encoder output = predictor input/output */
    uint32_t action_dim;       /* ActionEmbedderConfig (src/models/lewm/config.rs:69-88) */
    uint32_t smoothed_dim;
    uint32_t action_mlp_scale;
    uint32_t history_size;     /* rollout window (LeWmConfig::history_size) */
    uint32_t num_frames;       /* PredictorConfig (config.rs:42-67) */
    uint32_t pred_hidden_dim;
    uint32_t depth;
    uint32_t heads;
    uint32_t dim_head;
    uint32_t mlp_dim;
    uint32_t pred_proj_hidden; /* pred_proj MlpConfig (config.rs:90-107) */
    int32_t pred_proj_norm;    /* lwm_norm_kind */
    int32_t encoder;           /* lwm_encoder_kind */
    /* VectorMlpConfig (src/models/world_model/config.rs:22-44) */
    uint32_t obs_dim;
    uint32_t obs_hidden_dim;
    uint32_t obs_depth;
    int32_t obs_norm;          /* LayerNorm or None (BatchNorm maps to LayerNorm, model.rs:297-305) */
    /* VitEncoderConfig (src/models/lewm/config.rs:14-40) + projector MLP */
    uint32_t image_size;
    uint32_t patch_size;
    uint32_t vit_hidden;
    uint32_t vit_layers;
    uint32_t vit_heads;
    uint32_t vit_mlp;
    float vit_eps;
    uint32_t channels;
    int32_t qkv_bias;
    uint32_t projector_hidden;
    int32_t projector_norm;
} lwm_lewm_config;

/* The vector-observation CEM workload's model: VectorMlp 16 -> 512 (depth 3,
 * LayerNorm) -> 192, ActionEmbedder(2 -> 192), predictor depth 4, 8 heads x
 * 32, MLP 768, one frame, pred_proj 192 -> 512 -> 192 LayerNorm. */
void lwm_lewm_config_vector(lwm_lewm_config* out);
/* The image MPPI workload's model: ViT-Tiny (224, patch 16, 12 layers, 192,
 * 3 heads, MLP 768, eps 1e-12) + projector 192 -> 2048 -> 192 BatchNorm,
 * ActionEmbedder(2 -> 192), predictor depth 6, 16 heads x 64, MLP 2048
 * (PredictorConfig::lewm_tiny), one frame, pred_proj as the projector. */
void lwm_lewm_config_image(lwm_lewm_config* out);
/* Weight blob: one f32 array in this order (VarBuilder paths; Linear weights
 * [out, in], then bias):
 *   action_encoder.patch_embed.weight [sm, A, 1] .bias [sm]
 *   action_encoder.embed.0 [scale*D, sm] + bias, .embed.2 [D, scale*D] + bias
 *   predictor.pos_embedding [1, num_frames, D]
 *   predictor.transformer.input_proj [hid, D] + bias   (only when hid != D)
 *   predictor.transformer.cond_proj [hid, D] + bias    (only when hid != D)
 *   predictor.transformer.layers.{i}:
 *     attn.norm.weight [hid] .bias [hid], attn.to_qkv.weight [3*heads*dh, hid],
 *     attn.to_out.0.weight [hid, heads*dh] .bias [hid],
 *     mlp.net.0.weight [hid] .bias [hid], mlp.net.1 [mlp, hid] + bias,
 *     mlp.net.4 [hid, mlp] + bias, adaLN_modulation.1 [6*hid, hid] + bias
 *   predictor.transformer.norm.weight [hid] .bias [hid]
 *   predictor.transformer.output_proj [D, hid] + bias   (only when hid != D)
 *   pred_proj: net.0 [ph, D] + bias, net.1 (BatchNorm: weight, bias,
 *     running_mean, running_var [ph]; LayerNorm: weight, bias; None: nothing),
 *     net.3 [D, ph] + bias
 *   observation encoder, vector: layers.0 [oh, obs] + bias, norms.0 (LayerNorm
 *     weight, bias when obs_norm != None), layers.{j} [oh, oh] + bias and
 *     norms.{j} for j = 1 .. depth-2, layers.{depth-1} [D, oh] + bias
 *   observation encoder, ViT: embeddings.cls_token [1,1,vh],
 *     embeddings.position_embeddings [1, 1 + (img/p)^2, vh],
 *     embeddings.patch_embeddings.projection.weight [vh, C, p, p] .bias [vh],
 *     per layer: layernorm_before (w, b), attention.query/key/value [vh, vh]
 *     (+ bias when qkv_bias), attention.output.dense [vh, vh] + bias,
 *     layernorm_after (w, b), intermediate.dense [vmlp, vh] + bias,
 *     output.dense [vh, vmlp] + bias; then layernorm (w, b); then the
 *     projector MLP laid out as pred_proj (input vh, hidden projector_hidden). */
size_t lwm_lewm_weight_count(const lwm_lewm_config* cfg);
/* Seeded random init: Linear weights N(0, 2/fan_in) (Kaiming normal, candle's
 * linear default), biases U(+-1/sqrt(fan_in)), norm weights 1 / biases 0,
 * BatchNorm running mean 0 / var 1, position embeddings and CLS N(0, 0.02^2). */
lwm_status lwm_lewm_random_weights(const lwm_lewm_config* cfg, uint64_t seed, float* out, size_t count);

/* LeWmSession / WorldModel scorer (src/session.rs:46-66): weights in the
 * blob order above.  Fails with the reference's validation texts. */
lwm_status lwm_scorer_lewm_create(lwm_ctx* ctx, const lwm_lewm_config* cfg, const float* weights, size_t count,
                                  lwm_scorer** out);
/* Per-plan context: history embeddings [B, h, D] (LeWmSession::reset_pixels
 * caches them) shared by every sample of a vehicle, and the goal embedding
 * [B, D] (goal_cost, src/models/lewm/model.rs:149-165).  `history` is the
 * rollout window (rollout_embeddings_with_history); 0 uses h, as the session
 * does.  Host arrays, or device arrays with the _device variant. */
lwm_status lwm_scorer_lewm_set_context(lwm_scorer* scorer, uint32_t batch, uint32_t h, uint32_t history,
                                       const float* emb, const float* goal);
lwm_status lwm_scorer_lewm_set_context_device(lwm_scorer* scorer, uint32_t batch, uint32_t h, uint32_t history,
                                              const float* emb, const float* goal);
/* WorldModel::encode_vector (src/models/world_model/model.rs:48-50):
 * device obs [n, obs_dim] -> device embeddings [n, D]. */
lwm_status lwm_lewm_encode_vector_device(lwm_scorer* scorer, const float* obs, uint32_t n, float* out);
/* LeWm::encode_pixels (src/models/lewm/model.rs:41-55): device normalised
 * pixels [n, C, image, image] -> device embeddings [n, D]. */
lwm_status lwm_lewm_encode_pixels_device(lwm_scorer* scorer, const float* pixels, uint32_t n, float* out);

/* IcemPlanner::trace_device (src/planner.rs:900-1010): plan without
 * deadlines and record, per iteration, the scores of the mean before
 * sampling, the best candidate, the elite mean and the updated mean:
 * *trace -> device [iterations][4][B] f32 (IcemTraceDeviceStep's
 * mean_score, best_candidate_score, elite_mean_score, updated_mean_score),
 * valid until the planner's next call. */
lwm_status lwm_icem_trace_device(lwm_planner* planner, lwm_scorer* scorer, const float* injected_noise,
                                 lwm_plan_device_result* out, const float** trace);

/* ---------------------------------------------------------------- candidate-range sharding */

/* Multi-GPU MPPI over one vehicle batch: each GPU's planner owns samples
 * [sample_base, sample_base + samples) of sample_total.  It draws the same
 * Philox noise as an unsharded planner of sample_total samples and only the
 * shard holding sample 0 carries the mean candidate.  lwm_plan_device_shard
 * scores the shard and reduces it to one tuple per vehicle, [B][tuple_width]
 * floats on the device: (min score, sum of weights, best (score, global index)
 * key as 8 bytes, weighted action sums [T*A]).  The caller gathers the tuples
 * of all shards ([shards][B][tuple_width], e.g. one NCCL all-gather) and
 * lwm_mppi_combine_device rescales them to the global minimum and finishes
 * the plan as mppi_weighted_sequence (src/planner.rs:1588-1602) would over
 * all samples, warm start included.  MPPI with one iteration only.
 * sample_total 0 makes the planner unsharded again.  No reference
 * counterpart: the reference plans on one device. */
lwm_status lwm_planner_set_shard(lwm_planner* planner, uint32_t sample_base, uint32_t sample_total);
lwm_status lwm_plan_device_shard(lwm_planner* planner, lwm_scorer* scorer, const float* injected_noise,
                                 const float** tuples, uint32_t* tuple_width);
lwm_status lwm_mppi_combine_device(lwm_planner* planner, const float* tuples, uint32_t shards,
                                   lwm_plan_device_result* out);
/* Candidate shards of a CEM / iCEM plan (any iteration count; set the range
 * with lwm_planner_set_shard).  Every iteration each shard reduces its
 * candidates to its lowest `elites` as tuples (score, global candidate index
 * as uint32 bits, the T*A actions), `exchange` all-gathers the tuples of
 * every shard in sample-range order, and every shard refits from the merged
 * set: its lowest `elites` by (score, global index) are exactly the
 * unsharded plan's elites, so all shards continue from the same mean, std
 * and carried elites.  lwm_plan / lwm_plan_device then return the whole
 * plan's sequence, first action, best (global) index and warm start; the
 * scores are this shard's [B, samples].  `exchange(user, local, count,
 * gathered, stream)` runs on the planning thread with device buffers (count
 * floats of this shard; shards * count floats to fill) and the context's
 * stream, and returns 0 on success.  Shards ignore the deadline (every
 * shard must take the same iterations). */
typedef int (*lwm_exchange_fn)(void* user, const float* local, size_t count, float* gathered, void* stream);
lwm_status lwm_planner_set_shard_exchange(lwm_planner* planner, uint32_t shards, lwm_exchange_fn exchange,
                                          void* user);

/* ---------------------------------------------------------------- image preprocessing */

/* PackedImageFormat (src/media/mod.rs:59-83) and Nv12ColorSpace (:131-148). */
typedef enum lwm_packed_format {
    LWM_PACKED_RGB = 0,
    LWM_PACKED_BGR = 1,
    LWM_PACKED_RGBA = 2,
    LWM_PACKED_BGRA = 3,
} lwm_packed_format;
typedef enum lwm_nv12_color_space {
    LWM_NV12_BT601_VIDEO = 0,
    LWM_NV12_BT709_VIDEO = 1,
    LWM_NV12_BT601_FULL = 2,
    LWM_NV12_BT709_FULL = 3,
} lwm_nv12_color_space;

/* ImagePreprocess (src/media/mod.rs:168-193). */
typedef struct lwm_image_preprocess {
    uint32_t output_height;
    uint32_t output_width;
    float mean[3];
    float std[3];
} lwm_image_preprocess;
/* ImagePreprocess::imagenet_224 (src/media/mod.rs:175-183). */
void lwm_image_preprocess_imagenet_224(lwm_image_preprocess* out);

/* ImagePreprocessor::preprocess_packed_u8 and
 * ImageHistoryPreprocessor::preprocess_packed_u8_into_slot
 * (src/media/mod.rs:275-343, 470-543; kernel :1113-1194).  `input` is a
 * device [B,H,W,C] u8 frame batch (C = 3 or 4 by `format`); `output` is a
 * device [B,3,oh,ow] buffer (history_len == 0) or [B,history_len,3,oh,ow]
 * with slot `history_slot` written; out_bf16 selects bf16 instead of f32.
 * With W x channels a multiple of 16 up to 8192 bytes and the output /
 * normalisation conditions of lwm_preprocess_nv12_device below, a
 * row-staged kernel runs; otherwise a per-pixel kernel.  Both write the same
 * values. */
lwm_status lwm_preprocess_packed_device(lwm_ctx* ctx, const uint8_t* input, uint32_t batch, uint32_t height,
                                        uint32_t width, int32_t format, const lwm_image_preprocess* cfg,
                                        uint32_t history_len, uint32_t history_slot, int32_t out_bf16,
                                        void* output);
/* Nv12Preprocessor::preprocess_nv12 and Nv12HistoryPreprocessor::
 * preprocess_nv12_into_slot (src/media/mod.rs:196-273, 345-468; kernel
 * :1196-1333).  Device Y plane [B,H,W] and interleaved UV plane
 * [B,H/2,W/2,2]; H and W must be even.  With W a multiple of 16 up to 4096,
 * the output width a multiple of 4 up to 2048, 16-byte aligned planes and
 * output (8 bytes for bf16), std in [2^-40, 2^40] and mean 0 or of magnitude
 * in [2^-40, 2^40], a row-staged kernel runs (source rows bulk-copied into
 * shared memory); otherwise a per-pixel kernel.  Both write the same values. */
lwm_status lwm_preprocess_nv12_device(lwm_ctx* ctx, const uint8_t* y_plane, const uint8_t* uv_plane,
                                      uint32_t batch, uint32_t height, uint32_t width, int32_t color_space,
                                      const lwm_image_preprocess* cfg, uint32_t history_len,
                                      uint32_t history_slot, int32_t out_bf16, void* output);
/* The same preprocessing written as the ViT patch-embedding input instead of
 * an NCHW image: output [B, (oh/p)(ow/p), 3 p p] where element (b, c, y, x)
 * of the normalised image sits at patch (y/p) (ow/p) + x/p, column
 * c p p + (y%p) p + x%p — the layout Embeddings' stride-p convolution reads
 * (src/models/lewm/vit.rs:32-52, fed by src/media/mod.rs:1113-1333).  The
 * values equal the NCHW call's, permuted; `patch` must divide oh and ow (the
 * row-staged kernels take patch sizes that are multiples of 4). */
lwm_status lwm_preprocess_packed_patches_device(lwm_ctx* ctx, const uint8_t* input, uint32_t batch,
                                                uint32_t height, uint32_t width, int32_t format,
                                                const lwm_image_preprocess* cfg, uint32_t patch,
                                                int32_t out_bf16, void* output);
lwm_status lwm_preprocess_nv12_patches_device(lwm_ctx* ctx, const uint8_t* y_plane, const uint8_t* uv_plane,
                                              uint32_t batch, uint32_t height, uint32_t width,
                                              int32_t color_space, const lwm_image_preprocess* cfg,
                                              uint32_t patch, int32_t out_bf16, void* output);
/* LeWm::encode_pixels (src/models/lewm/model.rs:41-55) of device NV12 /
 * packed frames with the preprocessing fused into the encoder's input: the
 * frames are preprocessed (as above, f32) straight into the encoder's patch
 * matrix, then the ViT and projector run from it — no NCHW image and no
 * patchify pass.  cfg's output size must be the encoder's image size; out
 * [n, D] device embeddings. */
lwm_status lwm_lewm_encode_nv12_device(lwm_scorer* scorer, const uint8_t* y_plane, const uint8_t* uv_plane,
                                       uint32_t n, uint32_t height, uint32_t width, int32_t color_space,
                                       const lwm_image_preprocess* cfg, float* out);
lwm_status lwm_lewm_encode_packed_device(lwm_scorer* scorer, const uint8_t* input, uint32_t n, uint32_t height,
                                         uint32_t width, int32_t format, const lwm_image_preprocess* cfg,
                                         float* out);
/* One control step of LeWmSession (src/session.rs:31-40 reset_pixels and
 * encode_pixels, :46-65 score_candidates) under a planner (plan_device,
 * src/planner.rs:450): device NV12 frames -> embeddings -> scorer context ->
 * plan.  Frames [0, batch*history) are the observation history (batch-major,
 * `history` frames a row; the rollout window is `history`), frames
 * [batch*history, batch*(history+1)) the goals.  Results equal
 * lwm_lewm_encode_nv12_device + lwm_scorer_lewm_set_context_device (window
 * = history) + lwm_plan_device.  The encoder runs on a high-priority stream of
 * the scorer, beside the planner's sampling and the candidate-only part of
 * scoring (action embedding, AdaLN tables) on the context stream; the rollout
 * waits for it, and the context stream is ordered after it on return.
 * Asynchronous like lwm_plan_device; whole planners only (no shards). */
lwm_status lwm_lewm_plan_nv12_device(lwm_planner* planner, lwm_scorer* scorer, const uint8_t* y_plane,
                                     const uint8_t* uv_plane, uint32_t batch, uint32_t history, uint32_t height,
                                     uint32_t width, int32_t color_space, const lwm_image_preprocess* cfg,
                                     const float* injected_noise, lwm_plan_device_result* out);

/* ---------------------------------------------------------------- allocation-free iteration */

/* Device buffers of lwm_nominal_mppi_noalloc, all owned by the caller. */
typedef struct lwm_nominal_mppi_io {
    const float* initial;            /* [B,18] */
    const float* motors;             /* [B,4] */
    const float* reference_states;   /* [B,T,18] */
    const float* reference_actions;  /* [B,T,4] */
    const lwm_domain* domains;       /* [B] */
    const float* mean;               /* [B,T,4] sampling mean (e.g. the warm start) */
    const float* std;                /* [B,T,4] sampling std */
    const float* injected_noise;     /* [B,S,T,4] standard normals, or NULL for Philox(seed, offset) */
    float* scores;                   /* [B,S] */
    float* sequence;                 /* [B,T,4] MPPI-weighted sequence */
    float* first_action;             /* [B,4] */
    float* warm_start;               /* [B,T,4] sequence shifted by one step */
    uint32_t* best_indices;          /* [B] */
} lwm_nominal_mppi_io;

/* One fused nominal-physics MPPI iteration (sample, rotor rollout, tracking
 * cost, weighted sequence, best index) that allocates no memory: no
 * cudaMalloc, no cudaFree, no allocating library call.  No counterpart in the
 * reference; it exists for callers that cannot allocate device memory once
 * they run — real-time control loops and runtimes that reserve all memory up
 * front, where an allocation may synchronise the device or block.
 *
 * The caller owns every input and output (`io`, device pointers on `device`)
 * and the stream (NULL = the default stream).  The iteration's scratch — the
 * per-block MPPI tuples, per-vehicle arrival counters and best scores — is a
 * 1 MiB array in device memory that every GPU loading this library keeps
 * until the process exits.  Limits: batch <= 1024 vehicles and
 * batch * ceil(samples / 64) * (4 + 4 * horizon, rounded up to 4) * 4 bytes
 * <= 1,040,384 bytes; larger requests fail with LWM_INVALID_ARGUMENT and do
 * no GPU work.  The first call on a device loads this library's device code
 * on that device (CUDA loads modules lazily; loading them takes device
 * memory for the code and for the array) and looks up the array's device
 * address (cudaGetSymbolAddress), so make one call at start-up, before the
 * loop that may not allocate and before any stream capture.  The address is
 * kept for the life of the process: a cudaDeviceReset (or any teardown of
 * the device's primary context) invalidates it, and this entry point must
 * not be called on that device afterwards.  The call makes `device` current
 * while it runs and gives the caller's current device back before it
 * returns.  All calls share the one array and each call clears its counters
 * first, so two calls whose work overlaps on the GPU (different streams, or
 * different threads) race on it: serialise them.  Results equal
 * lwm_plan_device's for an MPPI planner with the nominal scorer given the
 * same mean, std, noise (or seed and offset) and context. */
lwm_status lwm_nominal_mppi_noalloc(int device, void* stream, const lwm_nominal_scorer_config* cfg,
                                    uint32_t batch, uint32_t samples, uint32_t horizon,
                                    const float* bounds_low, const float* bounds_high, float temperature,
                                    uint64_t seed, uint64_t offset, const lwm_nominal_mppi_io* io);

/* ---------------------------------------------------------------- task inputs */

/* skyjepa_reference_horizon (src/skyjepa_task.rs:44-55): kind 0 hover,
 * 1 circle, 2 figure-eight; out [horizon, 18]. */
lwm_status lwm_skyjepa_reference_horizon(int32_t kind, float time, float dt, uint32_t horizon,
                                         float radius, float period, float* out);
/* skyjepa_geometric_action_prior (src/skyjepa_task.rs:118-162):
 * current_state [18], references [horizon, 18] -> out [horizon, 4]. */
lwm_status lwm_skyjepa_geometric_prior(const float* current_state, const float* references,
                                       uint32_t horizon, float dt, const lwm_domain* domain,
                                       float* out);
/* One SkyJepaRotorPlant::step (src/skyjepa_sim.rs:206-270) on the host:
 * state [18] and motors [4] are updated in place. */
lwm_status lwm_rotor_plant_step(const lwm_domain* domain, float* state, float* motors,
                                const float* commanded_forces, float dt);

/* ---------------------------------------------------------------- control session */

/* SkyJepaControllerSession (src/models/skyjepa/session.rs:110-470): the
 * closed-loop controller around one vehicle's MPPI planner.  It keeps the
 * state/action histories, calibrates the trim from the holding action, builds
 * the geometric prior and the warm start (fresh prior or prior + the shifted,
 * clamped residual of the previous plan), and plans with the learned or the
 * nominal-physics scorer.  Per plan: one upload of the context, one upload of
 * the warm start, one synchronising read of the results. */
typedef struct lwm_skyjepa_session lwm_skyjepa_session;

typedef enum lwm_warm_start {
    LWM_WARM_START_FRESH_PRIOR = 0,
    LWM_WARM_START_SHIFTED_RESIDUAL = 1,
} lwm_warm_start;

typedef enum lwm_dynamics {
    LWM_DYNAMICS_LEARNED = 0,         /* SkyJepaDynamics::Trained / Untrained: the given weights */
    LWM_DYNAMICS_NOMINAL_PHYSICS = 1, /* SkyJepaDynamics::NominalPhysics */
} lwm_dynamics;

/* SkyJepaSessionConfig (session.rs:40-87) + the control settings the session
 * derives (SkyJepaControlConfig::paper_derived, control.rs:83-94, with dt =
 * 1 / model rate). */
typedef struct lwm_skyjepa_session_config {
    uint32_t samples;
    uint32_t horizon;
    uint64_t planner_seed;
    int32_t warm_start;       /* lwm_warm_start */
    float residual_limit_n;
    int32_t dynamics;         /* lwm_dynamics */
    float trim_multiplier;
    float dt;
    uint32_t iterations;
    float temperature;
    float action_noise[LWM_ROTOR_COUNT];
    lwm_tracking_cost cost;
} lwm_skyjepa_session_config;
void lwm_skyjepa_session_config_paper(lwm_skyjepa_session_config* out);

/* SkyJepaControllerPlan (session.rs:89-100).  action_sequence [horizon*4]
 * and predicted_states [horizon*18] are caller buffers (predicted_states may
 * be NULL when no prediction is asked for). */
typedef struct lwm_skyjepa_controller_plan {
    float action[LWM_ROTOR_COUNT];
    float prior_action[LWM_ROTOR_COUNT];
    float action_correction[LWM_ROTOR_COUNT];
    float* action_sequence;
    float* predicted_states;
    float best_candidate_score;
    double plan_ms;
    int32_t deadline_reached;
} lwm_skyjepa_controller_plan;

/* Creates the session and resets it to `initial_state` [18] with the hover
 * action.  The learned dynamics need the model, its weight blob and the
 * normalisation; NULLs are accepted for the nominal physics. */
lwm_status lwm_skyjepa_session_create(lwm_ctx* ctx, const lwm_skyjepa_session_config* cfg,
                                      const lwm_skyjepa_config* model, const float* weights,
                                      size_t weight_count, const float* state_mean,
                                      const float* state_std, const float* action_mean,
                                      const float* action_std, const float* initial_state,
                                      lwm_skyjepa_session** out);
void lwm_skyjepa_session_destroy(lwm_skyjepa_session* session);
/* reset / reset_with_action (session.rs:241-299). */
lwm_status lwm_skyjepa_session_reset(lwm_skyjepa_session* session, const float* state);
lwm_status lwm_skyjepa_session_reset_with_action(lwm_skyjepa_session* session, const float* state,
                                                 const float* action);
/* commit_observation (session.rs:301-320): the state reached after `action`. */
lwm_status lwm_skyjepa_session_commit_observation(lwm_skyjepa_session* session, const float* state,
                                                  const float* action);
/* plan / plan_with_prediction (session.rs:322-445): reference_states
 * [horizon*18]. */
lwm_status lwm_skyjepa_session_plan(lwm_skyjepa_session* session, const float* reference_states,
                                    int32_t include_prediction, lwm_skyjepa_controller_plan* out);
/* The session's scorer (for lwm_scorer_skyjepa_set_precision) and its
 * calibrated trim scale. */
lwm_scorer* lwm_skyjepa_session_scorer(lwm_skyjepa_session* session);
float lwm_skyjepa_session_trim_scale(const lwm_skyjepa_session* session);
/* shifted_residual (session.rs:534-543): clamp(sequence - prior, +-limit)
 * shifted one step earlier with a zero last step; [horizon*action_dim]. */
lwm_status lwm_skyjepa_shifted_residual(const float* sequence, const float* prior, uint32_t horizon,
                                        uint32_t action_dim, float limit, float* out);

/* ---------------------------------------------------------------- fleet loop */

/* The control loop of a fleet on the device, without host round trips per
 * control step.  Per step: lwm_fleet_control_step_device writes the scorer
 * context (commit_observation's history shift, the reference window, the
 * geometric prior as reference actions) into the learned scorer's context
 * buffers (lwm_scorer_skyjepa_context_device) and the prior into the
 * planner's warm start (lwm_planner_set_warm_start_device, a fresh-prior
 * warm start as SkyJepaControllerSession::plan_internal uses,
 * src/models/skyjepa/session.rs:322-400), lwm_plan_device plans, and
 * lwm_rotor_plant_step_device advances every vehicle's plant with the plan's
 * first action.  All calls are asynchronous on the context's stream. */
typedef struct lwm_fleet_step {
    uint32_t batch;
    uint32_t horizon;
    uint32_t history;            /* state history steps (>= 2) */
    float time;                  /* time of the current state */
    float dt;
    int32_t reference_kind;      /* 0 hover, 1 circle, 2 figure-eight */
    float radius;
    float period;
    lwm_domain prior_domain;     /* the controller's nominal domain (SkyJepaDomain::default) */
    const float* trim;           /* device [B] trim scale per vehicle, or NULL (1) */
    const float* state;          /* device [B,18]: the state each plant reached */
    const float* last_action;    /* device, the executed action per vehicle (row stride below),
                                    or NULL on the first step (no history shift) */
    uint32_t last_action_stride;
    float* state_history;        /* device [B,history,18], in/out */
    float* action_history;       /* device [B,history-1,4], in/out */
    float* reference_states;     /* device [B,horizon,18], out */
    float* reference_actions;    /* device [B,horizon,4], out: the prior (trim-scaled, clamped) */
} lwm_fleet_step;
lwm_status lwm_fleet_control_step_device(lwm_ctx* ctx, const lwm_fleet_step* step);
/* SkyJepaRotorPlant::step (src/skyjepa_sim.rs:206-281) for every vehicle:
 * `substeps` steps of dt with its own domain (device [B] lwm_domain), state
 * [B,18] and motors [B,4] in place (device), commands read with the given
 * row stride (device; e.g. a plan's first_action, stride 4). */
lwm_status lwm_rotor_plant_step_device(lwm_ctx* ctx, const lwm_domain* domains, float* states, float* motors,
                                       const float* commands, uint32_t command_stride, uint32_t batch,
                                       float dt, uint32_t substeps);
/* Device addresses of a learned scorer's context sections (after
 * lwm_scorer_skyjepa_set_context sized them): state_history [B,H,18],
 * action_history [B,H-1,4], reference_states [B,T,18], reference_actions
 * [B,T,4]; valid until the next set_context. */
lwm_status lwm_scorer_skyjepa_context_device(lwm_scorer* scorer, float** state_history, float** action_history,
                                             float** reference_states, float** reference_actions);
/* The warm start from device memory [batch, horizon, action_dim]
 * (asynchronous on the context's stream). */
lwm_status lwm_planner_set_warm_start_device(lwm_planner* planner, const float* sequence, uint32_t batch,
                                             uint32_t horizon, uint32_t action_dim);

/* ---------------------------------------------------------------- checkpoints */

/* Trained weights from safetensors files (the format candle's
 * VarBuilder::from_mmaped_safetensors reads, src/checkpoint.rs:6-17), looked
 * up by their VarBuilder names and written into the weight blob order above.
 * F32, F64, F16 and BF16 tensors are converted to f32 (the sessions build
 * their VarBuilders in F32).  Errors: LWM_INVALID_ARGUMENT with
 * "cannot find tensor <name>" for a missing tensor, "shape mismatch for
 * <name>, expected [..], got [..]", or the file/header problem. */
typedef struct lwm_tensor_info {
    char name[160];      /* VarBuilder path, e.g. "predictor.weight_hh_l0" */
    uint32_t rank;
    uint32_t shape[4];
    size_t offset;       /* first element in the weight blob */
    size_t numel;
    int32_t file;        /* SkyJEPA: 0 latent model file, 1 prober file; LeWM: 0 */
} lwm_tensor_info;

/* Naming of a LeWM-family checkpoint: LeWm (src/models/lewm/model.rs:20-31:
 * encoder.*, projector.*, predictor.*, action_encoder.*, pred_proj.*; ViT
 * encoders only) or WorldModel (src/models/world_model/model.rs:19-33,
 * 166-180: observation_encoder.{encoder,projector,vector_mlp}.*). */
typedef enum lwm_lewm_names {
    LWM_LEWM_NAMES_LEWM = 0,
    LWM_LEWM_NAMES_WORLD_MODEL = 1,
} lwm_lewm_names;

/* The tensors of the blob in order: returns their count (0 for an invalid
 * configuration) and fills *out for index < count. */
size_t lwm_skyjepa_tensor_info(const lwm_skyjepa_config* cfg, size_t index, lwm_tensor_info* out);
size_t lwm_lewm_tensor_info(const lwm_lewm_config* cfg, int32_t names, size_t index, lwm_tensor_info* out);

/* SkyJEPA: the latent model (SkyJepaModel::new, src/models/skyjepa/model.rs:
 * 22-39) from latent_path, the prober (SkyJepaProber::new, prober.rs:54-80)
 * from prober_path, as SkyJepaSession::open loads them
 * (src/models/skyjepa/session.rs:183-199). */
lwm_status lwm_skyjepa_weights_from_safetensors(const lwm_skyjepa_config* cfg, const char* latent_path,
                                                const char* prober_path, float* out, size_t count);
/* LeWm / WorldModel weights from one safetensors file. */
lwm_status lwm_lewm_weights_from_safetensors(const lwm_lewm_config* cfg, int32_t names, const char* path,
                                             float* out, size_t count);

#ifdef __cplusplus
}
#endif

#endif /* LEWM_B200_H */
