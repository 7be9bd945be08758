// lwm_lewm.hpp — the LeWM / WorldModel scorer: kernel interfaces and the
// host-side model (device weight views, workspaces, the launch sequence).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <vector>

#include "../../include/lewm_b200.h"

namespace lwm {

constexpr int kActNone = 0, kActGeluTanh = 1, kActGeluErf = 2, kActSilu = 3;
constexpr int kNormBatch = LWM_NORM_BATCH, kNormLayer = LWM_NORM_LAYER, kNormNone = LWM_NORM_NONE;

// Row r of a window batch ([seqs, t] tokens) -> row of a per-(sample, time)
// table ([seqs, T] rows): (r / t) * T + lo + r % t.  t == 0: identity.
struct RowMap {
    uint32_t t = 0, T = 0, lo = 0;
    __host__ __device__ size_t row(size_t r) const {
        return t == 0 ? r : (r / t) * T + lo + r % t;
    }
};

struct GemmArgs {
    const float* A;       // [M, K], row stride lda
    const float* W;       // [N, K], row stride ldw
    const float* bias;    // [N] or nullptr
    float* C;             // [M, N], row stride ldc
    uint32_t M, N, K, lda, ldw, ldc;
    int act;              // kAct* (ignored with residual)
    int residual;         // C += (gate ?) * (A W^T + b)
    const float* gate;    // gate table, row map.row(m), stride ldg, or nullptr
    uint32_t ldg;
    RowMap map;
    const uint16_t* Wb;   // bf16 copy of W (same [N, K] layout, row stride ldw): tensor-core path, or nullptr
    // split-K (set by gemm_f32): partial tiles and per-tile arrival counters
    uint32_t splits, k_chunk;
    float* partial;
    unsigned int* counters;
};

// Split-K scratch shared by the GEMMs of one stream (they run in order).
struct SplitScratch {
    float* partial = nullptr;
    size_t floats = 0;
    unsigned int* counters = nullptr;  // zero between GEMMs (the last CTA of a tile resets its counter)
    size_t n_counters = 0;
    int* tc_err = nullptr;             // error word of the tensor-core GEMM's bounded waits (4 ints)
    int* extra_launches = nullptr;     // counts the split-K reduce launches of the tensor-core GEMM
};

// Launches C = A W^T (+ epilogue); splits K over CTAs (deterministically) when
// `split` is given and the output tiles alone would leave most SMs idle.  With
// g.Wb set (and K a multiple of 16, A and Wb 16-byte aligned) the product runs
// on the tensor cores in bf16 with f32 accumulation (gemm_tc); otherwise f32.
cudaError_t gemm_f32(const GemmArgs& g, cudaStream_t s, const SplitScratch* split);
bool gemm_tc_eligible(const GemmArgs& g);
cudaError_t gemm_tc(const GemmArgs& g, cudaStream_t s, const SplitScratch* split, int* err);
cudaError_t launch_f32_to_bf16(const float* src, uint16_t* dst, size_t n, cudaStream_t s);
cudaError_t launch_ada_ln(const float* x, float* y, uint32_t rows, uint32_t d, const float* ada, uint32_t ld_ada,
                          uint32_t shift_off, uint32_t scale_off, RowMap map, const float* w, const float* b,
                          cudaStream_t s);
cudaError_t launch_layernorm(const float* x, float* y, uint32_t rows, uint32_t d, uint32_t t_in, uint32_t pick,
                             const float* w, const float* b, float eps, cudaStream_t s);
cudaError_t launch_norm_act(float* x, uint32_t rows, uint32_t d, int kind, const float* w, const float* b,
                            const float* rm, const float* rv, cudaStream_t s);
cudaError_t launch_silu(const float* x, float* y, size_t n, cudaStream_t s);
cudaError_t launch_window(const float* frames, uint32_t nframes, const float* pos, float* X, uint32_t rows,
                          uint32_t w_len, uint32_t lo, uint32_t d, cudaStream_t s);
cudaError_t launch_frames_init(const float* hist, uint32_t h, uint32_t S, float* frames, uint32_t nframes,
                               size_t rows, uint32_t d, cudaStream_t s);
cudaError_t launch_frames_put(const float* src, float* frames, uint32_t nframes, uint32_t slot, size_t rows,
                              uint32_t d, cudaStream_t s);
cudaError_t launch_attention(const float* qkv, float* out, uint32_t seqs, uint32_t t, uint32_t H, uint32_t dh,
                             float scale, int causal, int scale_q_first, cudaStream_t s);
// silu(W1 (Wc a + bc) + b1) for every row of `cand` [rows, A] (the action
// embedder's first two layers); A <= 8, sm <= 64 (action_embed_supported).
bool action_embed_supported(uint32_t A, uint32_t sm);
cudaError_t launch_action_embed(const float* cand, uint32_t A, const float* wc, const float* bc, uint32_t sm,
                                const float* w1, const float* b1, uint32_t ah, float* out, uint32_t rows,
                                cudaStream_t s);
cudaError_t launch_goal_cost(const float* pred, const float* goal, uint32_t S, size_t rows, uint32_t d,
                             float* scores, cudaStream_t s);
cudaError_t launch_patchify(const float* pix, float* patches, uint32_t n, uint32_t C, uint32_t img, uint32_t p,
                            cudaStream_t s);
cudaError_t launch_vit_assemble(const float* patch_out, const float* cls, const float* pos, float* x, uint32_t n,
                                uint32_t np, uint32_t vh, cudaStream_t s);

// ------------------------------------------------- fused predictor rollout
//
// The predictor's whole rollout in one launch for the image model's shape
// (width 192, one-frame windows), bf16 on the tensor cores:
// kernels_lewm_pred.cu.  Half-layers in order: attention and MLP halves of
// every layer, then pred_proj; each a pair of GEMMs split over the 8 CTAs of
// a cluster.
constexpr uint32_t kPredMaxHalves = 2 * 8 + 1;

// One half-layer's device views (the caller's f32 blob and the packed bf16 weights).
struct PredHalf {
    const uint8_t* w;   // this half-layer's packed weights of CTA rank 0 (rank j at + j * bytes)
    uint32_t bytes;     // per rank: W1 blocks, then W2 blocks
    uint32_t n1;        // first GEMM's columns per rank (64..256)
    const float* b1;    // first GEMM's bias (full width) or nullptr
    const float* b2;    // second GEMM's bias [192] or nullptr
    const float *bn_w, *bn_b, *bn_rm, *bn_rv;  // pred_proj BatchNorm (eval) or nullptr
    const float *ln_w, *ln_b;  // the LayerNorm that produces this half-layer's A (AdaLN's affine / final)
    int kind;
    uint32_t layer;     // transformer layer (AdaLN table slice)
};

struct PredArgs {
    PredHalf half[kPredMaxHalves];
    uint32_t halves;          // 2 depth + 1
    uint32_t tokens;          // B S
    uint32_t S, T, h, steps;  // samples per vehicle, horizon, context frames, steps = T - h + 1
    const float* emb;         // [B, h, 192] context embeddings
    const float* pos;         // [192] position embedding 0
    const float* ada;         // [depth][tokens * T][6 * 192]
    float* pred;              // [tokens, 192] the last step's frame
    uint8_t* xa;              // A exchange [tiles][2][8 owners][3][2 KB]
    float* xp;                // partial exchange [tiles][2][8 src][8 owners][16][192]
    int* err;
    uint32_t wait_polls;
};

bool lewm_pred_supported(const lwm_lewm_config& c, uint32_t history, const char** why);
// Bytes of one half-layer's packed weights per CTA rank (first GEMM width n1_total).
size_t lewm_pred_half_bytes(uint32_t n1_total);
// Packs rows [w1_row0, w1_row0 + n1_total) of w1 ([., 192], row stride w1_ld)
// and the matching n1_total columns of w2 ([192, w2_ld]) for the 8 ranks.
cudaError_t lewm_pred_pack(const float* w1, uint32_t w1_row0, uint32_t w1_ld, const float* w2, uint32_t w2_ld,
                           uint32_t n1_total, uint8_t* out, cudaStream_t s);
size_t lewm_pred_exchange_bytes(uint32_t tokens);
cudaError_t launch_lewm_pred(const PredArgs& a, cudaStream_t s);

// ------------------------------------------------------------ host model

struct Lin {
    const float* w = nullptr;
    const float* b = nullptr;
    uint32_t out = 0, in = 0;
    const uint16_t* wb = nullptr;  // bf16 copy of w (bf16 precision only)
};
struct Norm {
    int kind = kNormNone;
    const float *w = nullptr, *b = nullptr, *rm = nullptr, *rv = nullptr;
};
struct MlpW {
    Lin fc1;
    Norm norm;
    Lin fc2;
};
struct BlockW {
    Norm attn_norm, mlp_norm;
    Lin qkv, to_out, fc1, fc2, ada;
    Lin vo;  // V rows of qkv folded into to_out (LewmModel::fold_v_out; f32 path, one-token windows)
};
struct VitBlockW {
    Norm ln1, ln2;
    Lin q, k, v, o, fc1, fc2;
    Lin qkv;  // q, k and v as one Linear of 3 x vit_hidden outputs (LewmModel::fuse_vit_qkv)
};

// Tensor views into one weight blob (host walk of the documented order); with
// base == nullptr only the float count is computed.
struct LewmWeights {
    Lin act_conv, act_fc1, act_fc2;
    const float* pos = nullptr;
    bool has_proj = false;
    Lin input_proj, cond_proj, output_proj;
    std::vector<BlockW> blocks;
    Norm final_norm;
    MlpW pred_proj;
    std::vector<Lin> enc_lin;
    std::vector<Norm> enc_norm;
    const float *cls = nullptr, *vpos = nullptr;
    Lin patch;
    std::vector<VitBlockW> vit;
    Norm vit_norm;
    MlpW projector;
    size_t count = 0;
};
size_t lewm_walk(const lwm_lewm_config& c, const float* base, LewmWeights* out);
bool lewm_config_valid(const lwm_lewm_config& c, const char** why);

// Grow-only device workspace.
struct Arena {
    float* ptr = nullptr;
    size_t floats = 0;
    cudaError_t ensure(size_t n);
    void release();
};

// One captured launch sequence, replayed while its key (shapes and every
// buffer address it touches) stays the same.
struct GraphCache {
    static constexpr int kKey = 14;
    cudaGraphExec_t exec = nullptr;
    uint64_t key[kKey] = {};
    bool seen = false;  // the key ran once uncaptured (workspaces allocated)
    int launches = 0;
    void reset();
};

// Float offsets of the encoder workspace's regions (the patch matrix at 0).
struct EncoderOffsets {
    size_t patch, pe, x, y, qkv, att, f, cls, ph;
};

struct LewmModel {
    lwm_lewm_config c{};
    LewmWeights w;
    float* blob = nullptr;  // device weights
    uint16_t* blob_bf16 = nullptr;  // bf16 copies of the GEMM weights, each 256-byte aligned
    float* vit_qkv = nullptr;       // the ViT layers' fused query/key/value weights and biases
    float* vo_blob = nullptr;       // the predictor layers' folded V / out-projection maps
    int precision = LWM_PRECISION_F32;
    // bf16 with the image model's predictor shape: the whole rollout in one
    // launch (lewm_pred_kernel) with its weights packed per CTA rank
    uint8_t* pred_w = nullptr;
    PredArgs pred{};
    bool pred_ready = false;
    // per-plan context
    uint32_t B = 0, h = 0, history = 0;
    float* emb = nullptr;   // [B, h, D], at the start of one allocation
    float* goal = nullptr;  // [B, D], ctx_cap floats after emb (same allocation)
    size_t ctx_cap = 0;
    // Set while an observation encoding that writes emb / goal runs on
    // another stream: scoring then builds the candidate-only part (action
    // embedding, AdaLN tables) first, waits for this event, then rolls out.
    cudaEvent_t join_ev = nullptr;
    Arena ws;               // rollout workspace
    Arena enc;              // encoder workspace
    SplitScratch split;     // split-K partial tiles
    SplitScratch split_cand;  // the candidate-only part's own, while an encoder uses `split`
    GraphCache g_score, g_enc, g_score_cand, g_score_roll;
    int launches = 0;
    int split_launches = 0;  // split-K reduce kernels of the current launch sequence
    ~LewmModel();
    // part 0: all of scoring; 1: the candidate-only part (on split_cand, so
    // it may run beside an encoder that uses `split`); 2: the rest
    cudaError_t score_body(const float* cand, uint32_t S, uint32_t T, float* scores, float* last_emb, cudaStream_t s,
                           int part = 0);
    // emb and goal for [B, h] observation embeddings and B goals; `packed`:
    // goal directly behind emb's B h D floats (one encoder output fills both)
    cudaError_t ensure_context(uint32_t B, uint32_t h, bool packed, cudaStream_t s);
    cudaError_t encode_pixels_body(const float* pixels, uint32_t n, float* out, cudaStream_t s);
    cudaError_t encode_patches_body(uint32_t n, float* out, cudaStream_t s);
    size_t encoder_layout(uint32_t n, EncoderOffsets* o) const;
    cudaError_t ensure_split();
    cudaError_t ensure_split_cand();
    cudaError_t fuse_vit_qkv();
    cudaError_t fold_v_out();
    // LWM_PRECISION_F32: f32 GEMMs; LWM_PRECISION_BF16: bf16 weights and
    // GEMM inputs on the tensor cores, f32 accumulation and activations.
    cudaError_t set_precision(int p, cudaStream_t s);
    cudaError_t build_pred(cudaStream_t s);
    // scores [B,S] of candidates [B,S,T,A] (all device)
    cudaError_t score(const float* cand, uint32_t S, uint32_t T, float* scores, float* last_emb, cudaStream_t s);
    cudaError_t encode_vector(const float* obs, uint32_t n, float* out, cudaStream_t s);
    cudaError_t encode_pixels(const float* pixels, uint32_t n, float* out, cudaStream_t s);
    // The ViT patch matrix [n, (image/p)^2, C p p] of the encoder workspace,
    // for preprocessing to write directly; then encode_patches runs the
    // encoder from it (no NCHW image, no patchify pass).
    cudaError_t patch_buffer(uint32_t n, float** patches);
    cudaError_t encode_patches(uint32_t n, float* out, cudaStream_t s);
};

}  // namespace lwm
