// lwm_kernels.hpp — argument blocks and launchers of the library's kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/lewm_b200.h"


namespace lwm {

// Output and scratch of the one-pass MPPI reduction (lwm_mppi.cuh).
struct MppiArgs {
    float* partials;          // [B][P][pw]
    unsigned int* counters;   // [B], zero between launches
    float* sequence;          // [B][T][A]; also the next iteration's mean
    float* first_action;      // [B][A]
    float* warm_start;        // [B][T][A], shifted sequence
    uint32_t* best_index;     // [B]
    float* best_score;        // [B]
    uint32_t T, A, P, pw;     // pw = partial row width in floats (4 + T*A, padded)
    float mul;                // -1 / temperature
    uint32_t sample_base;     // global index of this shard's first sample (best-index keys)
    float* shard_tuple;       // [B][pw]: when set, the vehicle's combined tuple is written
                              // here (for a cross-GPU combine) instead of the final outputs
};

// Candidate-range shards: a planner that owns samples [sample_base,
// sample_base + S) of sample_total draws the same noise as an unsharded
// planner of sample_total samples (Philox index of the global sample) and
// only the shard holding sample 0 carries the mean candidate.
__host__ __device__ inline uint64_t global_row(uint32_t b, uint32_t s, uint32_t sample_base, uint32_t sample_total,
                                               uint32_t S) {
    const uint32_t total = sample_total ? sample_total : S;
    return static_cast<uint64_t>(b) * total + sample_base + s;
}

constexpr uint32_t kMaxHorizon = 64;
constexpr uint32_t kMaxActionDim = 16;

struct SampleArgs {
    uint32_t B, S, T, A;
    const float* mean;     // [B,T,A]
    const float* std;      // [B,T,A]
    const float* low;      // [A] (device)
    const float* high;     // [A] (device)
    const float* noise;    // injected [B,S,T,A] or nullptr
    uint64_t seed, offset;
    float smooth;          // colored-noise EMA factor; 0 = white noise
    uint32_t sample_base, sample_total;  // candidate-range shard (sample_total 0: unsharded)
    const float* carried;  // [B,carried_count,T,A] or nullptr
    uint32_t carried_count, inject;
    float* out;            // [B,S,T,A]
};

struct RefitArgs {
    uint32_t S, T, A, K, keep, sort_len, select;  // sort_len, select: from topk_layout
    const float* scores;   // [B,S]
    const float* cand;     // [B,S,T,A]
    float* mean;           // [B,T,A] in/out
    float* std;            // [B,T,A] in/out
    float* carried;        // [B,keep,T,A]
    uint32_t* elite_index; // [B,K] or nullptr
    int icem, return_best;
    float alpha, min_std, inv_k, inv_km1;
    float* sequence;       // [B,T,A]
    float* first_action;   // [B,A]
    float* warm_start;     // [B,T,A] or nullptr
    uint32_t* best_index;  // [B]
    float* best_score;     // [B]
    float* elite_mean_out; // [B,T,A] elite mean before the momentum update, or nullptr
    const uint32_t* index_map;  // [B,S] candidate -> reported index (merged shard elites), or nullptr
};

// SkyJepaDomain (src/skyjepa_sim.rs:28-40) as laid out on the device.
struct DomainParams {
    float mass, inertia[3], tau, drag[3], thrust_scale, torque_scale, arm, gravity, max_tw;
};

struct CostParams {
    float position, velocity, attitude, angular_velocity, action[4];
};

struct NominalArgs {
    uint32_t B, S, T, substeps;
    float h;          // dt / substeps
    float inv_trim;   // (float)(1 / trim_scale)
    const DomainParams* domains;  // [B]
    const float* initial;         // [B,18]
    const float* motors;          // [B,4]
    const float* ref_states;      // [B,T,18]
    const float* ref_actions;     // [B,T,4]
    CostParams cost;
    int sample;                   // 1: sample candidates in-kernel; 0: read cand_in
    const float* mean;            // [B,T,4]
    const float* std;             // [B,T,4]
    float low[4], high[4];
    const float* noise;           // injected [B,S,T,4] or nullptr
    uint64_t seed, offset;
    uint32_t sample_base, sample_total;  // candidate-range shard (sample_total 0: unsharded)
    const float* cand_in;         // [B,S,T,4] when sample == 0
    float* cand_out;              // [B,S,T,4] or nullptr
    float* scores;                // [B,S]
    float* states;                // [B,S,T,18] or nullptr
    int mppi;                     // 1: fused MPPI reduction
    MppiArgs m;
};

// SkyJEPA learned scorer: device weight views (see the weight-blob layout in
// include/lewm_b200.h) and per-plan context.
struct TcnBlockView {
    const float *w1, *b1, *w2, *b2, *wr, *br;
    uint32_t in, out, dil;
};
struct TcnView {
    uint32_t input_dim, levels, k, out_dim, max_ch;
    TcnBlockView blocks[8];
};

// Floats of an encoder's weights (contiguous in the blob).
__host__ __device__ inline uint32_t tcn_weight_floats(const TcnView& t) {
    uint32_t n = 0;
    for (uint32_t l = 0; l < t.levels; ++l) {
        const TcnBlockView& b = t.blocks[l];
        n += b.out * b.in * t.k + b.out + b.out * b.out * t.k + b.out;
        if (b.in != b.out) n += b.out * b.in + b.out;
    }
    return n;
}

struct SkyjepaArgs {
    uint32_t B, S, T, A, Hs, H, E, hid, prober_layers;
    TcnView state_tcn, action_tcn;
    const float *proj_w, *proj_b;
    const float *w_ih, *w_hh, *b_ih, *b_hh;
    const float *p_in_w, *p_in_b, *p_hid_w[4], *p_hid_b[4], *p_out_w, *p_out_b;
    float state_mean[18], state_std[18], action_mean[4], action_std[4];
    float mass, gravity, hover_throttle;
    int rotor_forces;
    float dt;
    CostParams cost;
    const float* state_hist;      // [B,Hs,18] raw
    const float* action_hist;     // [B,Hs-1,4] raw
    const float* ref_states;      // [B,T,18]
    const float* ref_actions;     // [B,T,4]
    const float* masses;          // [B] per-vehicle mass, or nullptr (use `mass`)
    uint32_t sample_base, sample_total;  // candidate-range shard (sample_total 0: unsharded)
    uint32_t rows;                // candidate rows per cluster (multiple of 8, 32..64)
    int sample;
    const float* mean;            // [B,T,4]
    const float* std;             // [B,T,4]
    float low[4], high[4];
    const float* low_dev;         // the same bounds in device memory ([16] each)
    const float* high_dev;
    const float* noise;
    uint64_t seed, offset;
    const float* cand_in;
    float* cand_out;
    float* scores;
    float* states;
    int mppi;
    MppiArgs m;
    const float* action_tcn_host;  // host copy of the action encoder's weights (kernel-parameter packing), or nullptr
    float* h0_work;                // scratch of the batched history encoder (skyjepa_h0_work_bytes), or nullptr
    // fault injection for tests (lwm_ctx_set_test_faults): 0 = off
    uint32_t test_wait_polls;      // tensor-core pipeline waits give up after this many polls
    uint32_t test_skip_h_arrive;   // the tensor-core rollout's first h hand-off of CTA 0 misses one arrival
    // CUDA events recorded on the stream around the rollout kernel's launch
    // (kernel timing, lwm_ctx_set_kernel_timing), or nullptr
    cudaEvent_t time_begin, time_end;
};

cudaError_t launch_sample(const SampleArgs& a, cudaStream_t stream);
// Tensor-core (tcgen05, bf16) learned-MPPI path for large candidate counts.
bool skyjepa_tc_supported(const SkyjepaArgs& a, const char** why);
size_t skyjepa_tc_packed_bytes();
cudaError_t skyjepa_tc_pack(const SkyjepaArgs& a, uint8_t* packed, cudaStream_t stream);
uint32_t skyjepa_tc_partials_per_vehicle(uint32_t S);
// A second stream of a scorer: work that does not depend on the main chain
// (the history encoding) runs there between a fork and a join event.
struct SideStream {
    cudaStream_t stream = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};
cudaError_t launch_skyjepa_tc(const SkyjepaArgs& a, const uint8_t* packed, float* h0, uint8_t* xtiles, int* err,
                              cudaStream_t stream, int* launches, const SideStream* side = nullptr);
size_t skyjepa_tc_xtile_bytes(uint32_t B, uint32_t S, uint32_t T);
// Initial latent of every vehicle (state encoder + projection) into h0 [B, H].
// Split-fp16 tensor-core path of the f32 learned scorer (kernels_skyjepa_mma.cu):
// every GEMM operand as two fp16 halves and three partial products per
// product, f32 gates / state / prober tail; one 16-CTA cluster per 128 rows.
bool skyjepa_mma_supported(const SkyjepaArgs& a, const char** why);
bool skyjepa_mma_fits_device();
size_t skyjepa_mma_packed_bytes();
cudaError_t skyjepa_mma_pack(const SkyjepaArgs& a, uint8_t* packed, cudaStream_t stream);
uint32_t skyjepa_mma_partials_per_vehicle(uint32_t S);
size_t skyjepa_mma_xtile_bytes(uint32_t B, uint32_t S, uint32_t T);
// The history encoder for the default shape (10 steps, kernel 3, three
// 128-channel levels with dilations 1, 2, 4, latent 256): one 16-CTA cluster
// per vehicle, only the positions the last output depends on.
bool skyjepa_h0_pruned_supported(const SkyjepaArgs& a);
cudaError_t launch_skyjepa_h0_pruned(const SkyjepaArgs& a, float* h0, cudaStream_t stream);
// Global buffer of the per-step h exchange between a cluster's CTAs.
size_t skyjepa_mma_exchange_bytes(uint32_t B, uint32_t S);
cudaError_t launch_skyjepa_mma(const SkyjepaArgs& a, const uint8_t* packed, float* h0, uint8_t* xtiles,
                               uint8_t* xchg, int* err, cudaStream_t stream, int* launches, const SideStream* side);
cudaError_t launch_skyjepa_h0(const SkyjepaArgs& a, float* h0, cudaStream_t stream);
// h0 of every vehicle by one 8-CTA cluster each (kernels_skyjepa.cu).
cudaError_t launch_skyjepa_h0_cluster(const SkyjepaArgs& a, float* h0, cudaStream_t stream);
// Scratch for the history encoder run over many vehicles at once (used when
// SkyjepaArgs::h0_work is set, B >= 32 and the history has 10 steps).
size_t skyjepa_h0_work_bytes(const SkyjepaArgs& a, uint32_t B);
// Small-latent (<= 64) learned path: a warp per candidate (sampling, action
// encoder inputs x [B,S,T,E], h0, rollout + cost + MPPI partials).
bool skyjepa_small_supported(const SkyjepaArgs& a, const char** why);
uint32_t skyjepa_small_partials_per_vehicle(uint32_t S);
size_t skyjepa_small_x_bytes(const SkyjepaArgs& a, uint32_t B, uint32_t S, uint32_t T);
cudaError_t launch_skyjepa_small(const SkyjepaArgs& a, float* h0, float* x, cudaStream_t stream, int* launches,
                                 const SideStream* side = nullptr);
// h0 on `side` (forked from `stream`) when given, else on `stream`; the
// caller joins with join_h0 before the rollout.
cudaError_t fork_h0(const SkyjepaArgs& a, float* h0, cudaStream_t stream, const SideStream* side);
cudaError_t join_h0(cudaStream_t stream, const SideStream* side);

cudaError_t launch_mppi_reduce(const MppiArgs& m, const float* cand, const float* scores, uint32_t B,
                               uint32_t S, cudaStream_t stream);
// Combine `shards` per-vehicle tuples [shards][B][pw] into the final outputs.
cudaError_t launch_mppi_combine(const MppiArgs& m, const float* tuples, uint32_t B, uint32_t shards,
                                cudaStream_t stream);
uint32_t sort_length(uint32_t S);
// Lowest-K selection limits: rows of up to kSortWholeRow scores are sorted
// whole; longer rows (any length) are radix-selected down to their K lowest
// keys first.  K is at most kMaxElites (its keys are sorted in shared memory).
constexpr uint32_t kSortWholeRow = 4096, kMaxElites = 16384;
// The shared-memory key count (`len`) and mode of a lowest-K selection over
// S scores; false when K is 0, above S or above kMaxElites.
bool topk_layout(uint32_t S, uint32_t K, uint32_t* len, uint32_t* select);
cudaError_t launch_topk_refit(const RefitArgs& a, uint32_t B, cudaStream_t stream);
// A CEM / iCEM shard's lowest K candidates as tuples [B][K][2 + TA] (score,
// global index bits, actions), and the merge of every shard's tuples.
cudaError_t launch_elite_tuples(const float* scores, const float* cand, uint32_t B, uint32_t S, uint32_t K,
                                uint32_t TA, uint32_t base, float* out, cudaStream_t stream);
cudaError_t launch_elite_merge(const float* gathered, uint32_t G, uint32_t B, uint32_t K, uint32_t TA, float* scores,
                               float* cand, uint32_t* index, cudaStream_t stream);
cudaError_t launch_lowest_k(const float* scores, uint32_t* out, uint32_t B, uint32_t S, uint32_t K,
                            cudaStream_t stream);
cudaError_t launch_color_noise(const float* in, float* out, uint32_t B, uint32_t S, uint32_t T, uint32_t A,
                               float smooth, cudaStream_t stream);
cudaError_t launch_normal_fill(uint64_t seed, uint64_t offset, uint64_t count, float* out, cudaStream_t stream);

// The fleet loop on the device (kernels_fleet_loop.cu).
cudaError_t launch_fleet_control(const lwm_fleet_step& a, cudaStream_t stream);
cudaError_t launch_plant(const lwm_domain* domains, float* states, float* motors, const float* commands,
                         uint32_t stride, uint32_t B, float dt, uint32_t substeps, cudaStream_t stream);

// Number of blocks (MPPI partials per vehicle) the nominal kernel uses.
uint32_t nominal_blocks_per_vehicle(uint32_t S);
cudaError_t launch_nominal(const NominalArgs& a, cudaStream_t stream);

struct MediaArgs {
    const uint8_t* a;   // packed pixels, or the Y plane
    const uint8_t* uv;  // NV12 interleaved UV plane (nullptr for packed input)
    void* out;
    uint32_t batch, in_h, in_w, channels, out_h, out_w;
    uint32_t format;    // packed: 0 RGB, 1 BGR, 2 RGBA, 3 BGRA; NV12: colour space 0..3
    uint32_t history_len, history_slot;
    int bf16;
    float mean[3], std[3];
    uint32_t patch;     // 0: NCHW / history slot; p > 0: ViT patch matrix [B, (H/p)(W/p), 3 p p]
    // fault injection for tests (lwm_ctx_set_test_faults), 0 = off: the
    // row-staged producer skips output row test_skip_row_plus1 - 1; waits
    // give up after test_wait_polls polls
    uint32_t test_skip_row_plus1, test_wait_polls;
};
cudaError_t launch_media(const MediaArgs& a, bool nv12, cudaStream_t stream);
// The row-staged NV12 kernel (bulk-copied source rows, packed f32x2 math):
// bit-identical to launch_media's NV12 kernel where eligible (row bytes a
// multiple of 16 up to 4096, output width a multiple of 4 up to 2048,
// aligned planes and output, std in [2^-40, 2^40], mean 0 or
// of magnitude in [2^-40, 2^40]).  `err` (4 ints, device-
// visible) gets 1 in err[0] when a row copy never completed.
struct StagedMedia {
    // fault injection for tests (lwm_ctx_set_test_faults): the producer skips
    // the copies of output row `skip_row` (~0u: none); waits give up after
    // `wait_polls` polls
    uint32_t skip_row, wait_polls;
    float ratio_h, ratio_w;
    float rcp_std[3];
    float neg_zero;  // -0.0f
    int* err;
};
bool nv12_staged_eligible(const MediaArgs& a);
cudaError_t launch_nv12_staged(const MediaArgs& a, int* err, cudaStream_t stream);
// The row-staged packed RGB / BGR / RGBA / BGRA kernel, bit-identical with
// launch_media's packed kernel where eligible (row bytes W x channels a
// multiple of 16 up to 8192, the output and normalisation conditions as
// above).
bool packed_staged_eligible(const MediaArgs& a);
cudaError_t launch_packed_staged(const MediaArgs& a, int* err, cudaStream_t stream);

// Rows per cluster (one wave of co-resident clusters when possible) and MPPI
// partials per vehicle of the fused SkyJEPA kernel.
uint32_t skyjepa_rows_per_cluster(const SkyjepaArgs& a);
uint32_t skyjepa_partials_per_vehicle(uint32_t S, uint32_t rows);
bool skyjepa_supported(const SkyjepaArgs& a, const char** why);
// Launches the fused rollout kernel (a.rows must be set).
cudaError_t launch_skyjepa(const SkyjepaArgs& a, cudaStream_t stream, int* launches);

}  // namespace lwm
