// session.cpp — the SkyJEPA closed-loop controller session on top of the
// planner and scorer entry points (SkyJepaControllerSession,
// src/models/skyjepa/session.rs:110-470).
//
// Host state per session: the state / action history windows, the trim
// calibration and the first-order motor model of the nominal dynamics, the
// warm-start residual of the last plan.  One plan = the geometric prior on
// the host (skyjepa_geometric_action_prior, src/skyjepa_task.rs:118-162,
// scaled by the trim and clamped to the bounds), the warm start, the scorer
// context, one MPPI plan with the results read back once, and the next
// residual (shifted_residual, session.rs:534-543).
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <chrono>
#include <cmath>
#include <cstring>
#include <deque>
#include <memory>
#include <string>
#include <vector>

#include "lwm_host.hpp"

namespace {

lwm_status bad(const std::string& m) { return lwm::set_last_error(LWM_INVALID_ARGUMENT, m); }

bool finite(float v) { return std::isfinite(v); }

}  // namespace

struct lwm_skyjepa_session {
    lwm_ctx* ctx = nullptr;
    lwm_skyjepa_session_config cfg{};
    bool learned = true;
    uint32_t H = 10;  // history steps
    lwm_domain dom{};
    float high = 0.0f;  // rotor force bound
    float hover[4] = {};
    float trim_scale = 1.0f;
    float nominal_motor[4] = {};
    lwm_scorer* scorer = nullptr;
    lwm_planner* planner = nullptr;
    std::deque<std::array<float, 18>> states;
    std::deque<std::array<float, 4>> actions;
    bool has_active = false, has_pending = false;
    std::vector<float> active, pending;  // [T*4]
    std::vector<float> prior, warm, seq, scores, hist_s, hist_a;
    float* d_cand = nullptr;    // [T*4] device (prediction)
    float* d_states = nullptr;  // [T*18] device (prediction)

    ~lwm_skyjepa_session() {
        if (planner) lwm_planner_destroy(planner);
        if (scorer) lwm_scorer_destroy(scorer);
        if (d_cand) cudaFree(d_cand);
        if (d_states) cudaFree(d_states);
    }

    lwm_status make_planner() {
        if (planner) lwm_planner_destroy(planner);
        planner = nullptr;
        lwm_mppi_config m;
        lwm_mppi_config_default(cfg.horizon, cfg.samples, 4, &m);
        m.iterations = cfg.iterations;
        for (int i = 0; i < 4; ++i) {
            m.bounds_low[i] = 0.0f;
            m.bounds_high[i] = high;
            m.noise_std_per_action[i] = cfg.action_noise[i];
            m.deadline_action[i] = hover[i];
        }
        m.has_noise_std_per_action = 1;
        m.temperature = cfg.temperature;
        m.has_deadline_action = 1;
        m.has_seed = 1;
        m.seed = cfg.planner_seed;
        return lwm_mppi_create(ctx, &m, &planner);
    }

    // The nominal scorer carries the trim scale: rebuilt when the trim changes.
    lwm_status make_nominal_scorer() {
        if (scorer) lwm_scorer_destroy(scorer);
        scorer = nullptr;
        lwm_nominal_scorer_config n{};
        n.dt = cfg.dt;
        n.trim_scale = trim_scale;
        n.substeps = 10;
        n.cost = cfg.cost;
        n.domain = dom;
        return lwm_scorer_nominal_create(ctx, &n, &scorer);
    }

    lwm_status reset_with_action(const float* state, const float* action) {
        for (int i = 0; i < 4; ++i)
            if (!finite(action[i]) || action[i] < 0.0f) return bad("SkyJEPA initial action must be finite and non-negative");
        for (int i = 0; i < 18; ++i)
            if (!finite(state[i])) return bad("SkyJEPA initial state must be finite");
        const float nominal_collective = hover[0] + hover[1] + hover[2] + hover[3];
        const float collective = action[0] + action[1] + action[2] + action[3];
        if (!(collective > 0.0f)) return bad("initial trim must have positive collective force");
        const float ts = collective / nominal_collective * cfg.trim_multiplier;
        if (!finite(ts) || ts <= 0.0f) return bad("invalid calibrated trim");
        trim_scale = ts;
        for (int i = 0; i < 4; ++i) nominal_motor[i] = action[i] / trim_scale;
        has_active = has_pending = false;
        std::array<float, 18> s;
        std::memcpy(s.data(), state, sizeof s);
        std::array<float, 4> a;
        std::memcpy(a.data(), action, sizeof a);
        states.assign(H, s);
        actions.assign(H - 1, a);
        lwm_status st = make_planner();
        if (st != LWM_OK) return st;
        if (!learned) {
            st = make_nominal_scorer();
            if (st != LWM_OK) return st;
        }
        std::vector<float> w(static_cast<size_t>(cfg.horizon) * 4);
        for (uint32_t t = 0; t < cfg.horizon; ++t) std::memcpy(&w[t * 4], action, 16);
        return lwm_planner_set_warm_start(planner, w.data(), 1, cfg.horizon, 4);
    }
};

extern "C" {

void lwm_skyjepa_session_config_paper(lwm_skyjepa_session_config* out) {
    if (!out) return;
    std::memset(out, 0, sizeof *out);
    // SkyJepaSessionConfig::paper_derived (session.rs:52-64) and
    // SkyJepaControlConfig::paper_derived (control.rs:84-94)
    out->samples = 512;
    out->horizon = 15;
    out->planner_seed = 7;
    out->warm_start = LWM_WARM_START_FRESH_PRIOR;
    out->residual_limit_n = 2.0f;
    out->dynamics = LWM_DYNAMICS_LEARNED;
    out->trim_multiplier = 1.0f;
    out->dt = 0.05f;
    out->iterations = 1;
    out->temperature = 1e-4f;
    const float noise[4] = {0.60f, 0.15f, 0.15f, 0.05f};
    std::memcpy(out->action_noise, noise, sizeof noise);
    lwm_tracking_cost_paper(&out->cost);
}

lwm_status lwm_skyjepa_session_create(lwm_ctx* ctx, const lwm_skyjepa_session_config* cfg,
                                      const lwm_skyjepa_config* model, const float* weights, size_t weight_count,
                                      const float* state_mean, const float* state_std, const float* action_mean,
                                      const float* action_std, const float* initial_state,
                                      lwm_skyjepa_session** out) {
    if (!ctx || !cfg || !initial_state || !out) return bad("null argument");
    // SkyJepaSessionConfig::validate (session.rs:66-80), SkyJepaControlConfig::validate (control.rs:96-122)
    if (cfg->samples == 0) return bad("SkyJEPA session samples must be positive");
    if (cfg->horizon == 0) return bad("SkyJEPA session horizon must be positive");
    if (!finite(cfg->residual_limit_n) || cfg->residual_limit_n <= 0.0f)
        return bad("warm-start residual limit must be finite and positive");
    if (!finite(cfg->trim_multiplier) || cfg->trim_multiplier <= 0.0f)
        return bad("trim multiplier must be finite and positive");
    if (cfg->iterations == 0) return bad("SkyJEPA MPPI iterations must be positive");
    if (!finite(cfg->dt) || cfg->dt <= 0.0f) return bad("SkyJEPA control dt must be finite and positive");
    if (!finite(cfg->temperature) || cfg->temperature <= 0.0f)
        return bad("SkyJEPA MPPI temperature must be finite and positive");
    for (int i = 0; i < 4; ++i)
        if (!finite(cfg->action_noise[i]) || cfg->action_noise[i] <= 0.0f)
            return bad("SkyJEPA action noise values must be finite and positive");
    if (cfg->warm_start != LWM_WARM_START_FRESH_PRIOR && cfg->warm_start != LWM_WARM_START_SHIFTED_RESIDUAL)
        return bad("unknown warm start " + std::to_string(cfg->warm_start));
    if (cfg->dynamics != LWM_DYNAMICS_LEARNED && cfg->dynamics != LWM_DYNAMICS_NOMINAL_PHYSICS)
        return bad("unknown dynamics " + std::to_string(cfg->dynamics));
    auto s = std::make_unique<lwm_skyjepa_session>();
    s->ctx = ctx;
    s->cfg = *cfg;
    s->learned = cfg->dynamics == LWM_DYNAMICS_LEARNED;
    lwm_domain_default(&s->dom);
    s->high = s->dom.mass * s->dom.gravity * s->dom.max_thrust_weight / 4.0f;
    for (int i = 0; i < 4; ++i) s->hover[i] = s->dom.mass * s->dom.gravity / 4.0f;
    if (s->learned) {
        if (!model || !weights || !state_mean || !state_std || !action_mean || !action_std)
            return bad("learned dynamics need the model, its weights and the normalisation");
        s->H = model->history_steps;
        lwm_status st = lwm_scorer_skyjepa_create(ctx, model, weights, weight_count, state_mean, state_std,
                                                  action_mean, action_std, &cfg->cost, cfg->dt, &s->scorer);
        if (st != LWM_OK) return st;
    } else if (model) {
        s->H = model->history_steps;
    }
    if (s->H < 2) return bad("SkyJEPA history must hold at least two steps");
    const size_t T = cfg->horizon;
    s->prior.resize(T * 4);
    s->warm.resize(T * 4);
    s->seq.resize(T * 4);
    s->scores.resize(cfg->samples);
    s->active.assign(T * 4, 0.0f);
    s->pending.assign(T * 4, 0.0f);
    s->hist_s.resize(static_cast<size_t>(s->H) * 18);
    s->hist_a.resize(static_cast<size_t>(s->H - 1) * 4);
    const float hover[4] = {s->hover[0], s->hover[1], s->hover[2], s->hover[3]};
    lwm_status st = s->reset_with_action(initial_state, hover);
    if (st != LWM_OK) return st;
    *out = s.release();
    return LWM_OK;
}

void lwm_skyjepa_session_destroy(lwm_skyjepa_session* s) { delete s; }

lwm_status lwm_skyjepa_session_reset(lwm_skyjepa_session* s, const float* state) {
    if (!s || !state) return bad("null argument");
    const float hover[4] = {s->hover[0], s->hover[1], s->hover[2], s->hover[3]};
    return s->reset_with_action(state, hover);
}

lwm_status lwm_skyjepa_session_reset_with_action(lwm_skyjepa_session* s, const float* state, const float* action) {
    if (!s || !state || !action) return bad("null argument");
    return s->reset_with_action(state, action);
}

lwm_status lwm_skyjepa_session_commit_observation(lwm_skyjepa_session* s, const float* state, const float* action) {
    if (!s || !state || !action) return bad("null argument");
    // the residual of the plan whose action was executed becomes active
    s->has_active = s->has_pending;
    if (s->has_pending) s->active = s->pending;
    s->has_pending = false;
    const float response = 1.0f - std::exp(-s->cfg.dt / s->dom.motor_time_constant);
    for (int i = 0; i < 4; ++i) {
        const float target = std::min(std::max(action[i] / s->trim_scale, 0.0f), s->high);
        s->nominal_motor[i] += (target - s->nominal_motor[i]) * response;
    }
    std::array<float, 18> st;
    std::memcpy(st.data(), state, sizeof st);
    std::array<float, 4> a;
    std::memcpy(a.data(), action, sizeof a);
    s->states.pop_front();
    s->states.push_back(st);
    s->actions.pop_front();
    s->actions.push_back(a);
    return LWM_OK;
}

lwm_status lwm_skyjepa_shifted_residual(const float* sequence, const float* prior, uint32_t horizon,
                                        uint32_t action_dim, float limit, float* out) {
    if (!sequence || !prior || !out || horizon == 0 || action_dim == 0) return bad("invalid shifted residual arguments");
    for (uint32_t t = 0; t + 1 < horizon; ++t)
        for (uint32_t a = 0; a < action_dim; ++a) {
            const size_t i = static_cast<size_t>(t + 1) * action_dim + a;
            out[static_cast<size_t>(t) * action_dim + a] = std::min(std::max(sequence[i] - prior[i], -limit), limit);
        }
    for (uint32_t a = 0; a < action_dim; ++a) out[static_cast<size_t>(horizon - 1) * action_dim + a] = 0.0f;
    return LWM_OK;
}

lwm_status lwm_skyjepa_session_plan(lwm_skyjepa_session* s, const float* refs, int32_t include_prediction,
                                    lwm_skyjepa_controller_plan* out) {
    if (!s || !refs || !out || !out->action_sequence) return bad("null argument");
    if (include_prediction && !out->predicted_states) return bad("predicted_states buffer is required for a prediction");
    const auto started = std::chrono::steady_clock::now();
    s->has_pending = false;
    const uint32_t T = s->cfg.horizon;
    // prior_action_sequence (session.rs:497-511)
    const std::array<float, 18>& last = s->states.back();
    lwm_status st = lwm_skyjepa_geometric_prior(last.data(), refs, T, s->cfg.dt, &s->dom, s->prior.data());
    if (st != LWM_OK) return st;
    for (float& f : s->prior) f = std::min(std::max(f * s->trim_scale, 0.0f), s->high);
    for (size_t i = 0; i < s->warm.size(); ++i) {
        float w = s->prior[i];
        if (s->cfg.warm_start == LWM_WARM_START_SHIFTED_RESIDUAL && s->has_active) w = w + s->active[i];
        s->warm[i] = std::min(std::max(w, 0.0f), s->high);
    }
    st = lwm_planner_set_warm_start(s->planner, s->warm.data(), 1, T, 4);
    if (st != LWM_OK) return st;
    if (s->learned) {
        for (uint32_t h = 0; h < s->H; ++h) std::memcpy(&s->hist_s[h * 18], s->states[h].data(), 18 * 4);
        for (uint32_t h = 0; h + 1 < s->H; ++h) std::memcpy(&s->hist_a[h * 4], s->actions[h].data(), 16);
        st = lwm_scorer_skyjepa_set_context(s->scorer, 1, T, s->hist_s.data(), s->hist_a.data(), refs, s->prior.data());
    } else {
        st = lwm_scorer_nominal_set_context(s->scorer, 1, T, last.data(), s->nominal_motor, refs, s->prior.data(),
                                            nullptr);
    }
    if (st != LWM_OK) return st;
    lwm_plan_result r{};
    float first[4];
    uint32_t best = 0;
    r.first_action = first;
    r.sequence = s->seq.data();
    r.scores = s->scores.data();
    r.scores_capacity = s->scores.size();
    r.best_indices = &best;
    st = lwm_plan(s->planner, s->scorer, nullptr, &r);
    if (st != LWM_OK) return st;
    float best_score = INFINITY;
    bool nan = false;
    for (uint32_t i = 0; i < r.scores_cols; ++i) {
        nan = nan || std::isnan(s->scores[i]);
        best_score = std::min(best_score, s->scores[i]);
    }
    if (nan) best_score = NAN;
    for (int i = 0; i < 4; ++i)
        if (!finite(first[i])) return bad("SkyJEPA planner produced a non-finite action or score");
    if (!finite(best_score)) return bad("SkyJEPA planner produced a non-finite action or score");
    if (include_prediction) {
        const size_t T4 = static_cast<size_t>(T) * 4, T18 = static_cast<size_t>(T) * 18;
        if (!s->d_cand) {
            if (cudaMalloc(&s->d_cand, T4 * 4) != cudaSuccess || cudaMalloc(&s->d_states, T18 * 4) != cudaSuccess)
                return lwm::set_last_error(LWM_CUDA_ERROR, "cannot allocate the prediction buffers");
        }
        if (cudaMemcpy(s->d_cand, s->seq.data(), T4 * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return lwm::set_last_error(LWM_CUDA_ERROR, "prediction upload failed");
        st = lwm_scorer_predict_device(s->scorer, s->d_cand, 1, 1, T, s->d_states);
        if (st != LWM_OK) return st;
        st = lwm_ctx_synchronize(s->ctx);
        if (st != LWM_OK) return st;
        if (cudaMemcpy(out->predicted_states, s->d_states, T18 * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
            return lwm::set_last_error(LWM_CUDA_ERROR, "prediction download failed");
    }
    if (s->cfg.warm_start == LWM_WARM_START_SHIFTED_RESIDUAL) {
        lwm_skyjepa_shifted_residual(s->seq.data(), s->prior.data(), T, 4, s->cfg.residual_limit_n, s->pending.data());
        s->has_pending = true;
    }
    for (int i = 0; i < 4; ++i) {
        out->action[i] = first[i];
        out->prior_action[i] = s->prior[i];
        out->action_correction[i] = first[i] - s->prior[i];
    }
    std::memcpy(out->action_sequence, s->seq.data(), s->seq.size() * 4);
    out->best_candidate_score = best_score;
    out->deadline_reached = r.deadline_reached;
    out->plan_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - started).count();
    return LWM_OK;
}

lwm_scorer* lwm_skyjepa_session_scorer(lwm_skyjepa_session* s) { return s ? s->scorer : nullptr; }

float lwm_skyjepa_session_trim_scale(const lwm_skyjepa_session* s) { return s ? s->trim_scale : 0.0f; }

}  // extern "C"
