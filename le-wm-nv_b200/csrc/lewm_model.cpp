// lewm_model.cpp — host side of the LeWM / WorldModel scorer: model presets,
// the weight-blob layout and seeded init, and the launch sequence of one
// scoring call (every candidate of every vehicle in each launch).
//
// Reference: LeWm / WorldModel (src/models/lewm/model.rs:20-165,
// src/models/world_model/model.rs:19-160), LeWmSession::score_candidates
// (src/session.rs:46-66), modules.rs:9-399, vit.rs:7-57.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "lwm_host.hpp"
#include "lwm_pdl.hpp"
#include "lwm_lewm.hpp"

namespace lwm {

namespace {

struct Spec {
    size_t off, n;
    int kind;      // 0 Linear weight (Kaiming normal), 1 bias U(+-1/sqrt(fan)), 2 ones, 3 zeros, 4 N(0, 0.02^2)
    uint32_t fan;
};

struct Walker {
    const float* base;
    size_t off = 0;
    std::vector<Spec>* specs;
    std::vector<NamedTensor>* named = nullptr;  // VarBuilder path and shape of each tensor
    const float* take(size_t n, int kind, uint32_t fan, const std::string& name, std::vector<uint32_t> shape) {
        if (specs) specs->push_back({off, n, kind, fan});
        if (named) named->push_back({name, std::move(shape), off, n, 0});
        const float* p = base ? base + off : nullptr;
        off += n;
        return p;
    }
    // Linear (or convolution, with its weight shape given) at VarBuilder path `name`.
    Lin lin(uint32_t out, uint32_t in, bool bias, const std::string& name, std::vector<uint32_t> wshape = {}) {
        Lin l;
        l.out = out;
        l.in = in;
        if (wshape.empty()) wshape = {out, in};
        l.w = take(static_cast<size_t>(out) * in, 0, in, name + ".weight", std::move(wshape));
        l.b = bias ? take(out, 1, in, name + ".bias", {out}) : nullptr;
        return l;
    }
    Norm norm(int kind, uint32_t d, const std::string& name) {
        Norm n;
        n.kind = kind;
        if (kind == kNormBatch) {
            n.w = take(d, 2, 0, name + ".weight", {d});
            n.b = take(d, 3, 0, name + ".bias", {d});
            n.rm = take(d, 3, 0, name + ".running_mean", {d});
            n.rv = take(d, 2, 0, name + ".running_var", {d});
        } else if (kind == kNormLayer) {
            n.w = take(d, 2, 0, name + ".weight", {d});
            n.b = take(d, 3, 0, name + ".bias", {d});
        }
        return n;
    }
    // Mlp (modules.rs:90-101): net.0 Linear, net.1 norm, net.3 Linear.
    MlpW mlp(uint32_t in, uint32_t hid, uint32_t out, int norm_kind, const std::string& name) {
        MlpW m;
        m.fc1 = lin(hid, in, true, name + ".net.0");
        m.norm = norm(norm_kind, hid, name + ".net.1");
        m.fc2 = lin(out, hid, true, name + ".net.3");
        return m;
    }
};

// Walks the blob in its documented order.  `names` picks the checkpoint
// naming of the observation encoder (LeWm: encoder / projector; WorldModel:
// observation_encoder.{encoder, projector, vector_mlp}).
size_t walk(const lwm_lewm_config& c, const float* base, LewmWeights* out, std::vector<Spec>* specs,
            std::vector<NamedTensor>* named = nullptr, int names = LWM_LEWM_NAMES_WORLD_MODEL) {
    LewmWeights w;
    Walker k{base, 0, specs, named};
    const uint32_t D = c.embed_dim, hid = c.pred_hidden_dim, inner = c.heads * c.dim_head;
    // ActionEmbedder (modules.rs:120-145): Conv1d(A -> smoothed, k=1), embed.0, embed.2
    w.act_conv = k.lin(c.smoothed_dim, c.action_dim, true, "action_encoder.patch_embed", {c.smoothed_dim, c.action_dim, 1});
    w.act_fc1 = k.lin(c.action_mlp_scale * D, c.smoothed_dim, true, "action_encoder.embed.0");
    w.act_fc2 = k.lin(D, c.action_mlp_scale * D, true, "action_encoder.embed.2");
    // Predictor (modules.rs:360-372) and its Transformer (modules.rs:305-330)
    w.pos = k.take(static_cast<size_t>(c.num_frames) * D, 4, 0, "predictor.pos_embedding", {1, c.num_frames, D});
    const std::string tr = "predictor.transformer";
    w.has_proj = hid != D;
    if (w.has_proj) {
        w.input_proj = k.lin(hid, D, true, tr + ".input_proj");
        w.cond_proj = k.lin(hid, D, true, tr + ".cond_proj");
    }
    w.blocks.resize(c.depth);
    for (uint32_t l = 0; l < c.depth; ++l) {
        // ConditionalBlock (modules.rs:275-290): attn, mlp, adaLN_modulation.1
        const std::string p = tr + ".layers." + std::to_string(l);
        BlockW& b = w.blocks[l];
        b.attn_norm = k.norm(kNormLayer, hid, p + ".attn.norm");
        b.qkv = k.lin(3 * inner, hid, false, p + ".attn.to_qkv");
        b.to_out = k.lin(hid, inner, true, p + ".attn.to_out.0");
        b.mlp_norm = k.norm(kNormLayer, hid, p + ".mlp.net.0");
        b.fc1 = k.lin(c.mlp_dim, hid, true, p + ".mlp.net.1");
        b.fc2 = k.lin(hid, c.mlp_dim, true, p + ".mlp.net.4");
        b.ada = k.lin(6 * hid, hid, true, p + ".adaLN_modulation.1");
    }
    w.final_norm = k.norm(kNormLayer, hid, tr + ".norm");
    if (w.has_proj) w.output_proj = k.lin(D, hid, true, tr + ".output_proj");
    w.pred_proj = k.mlp(D, c.pred_proj_hidden, D, c.pred_proj_norm, "pred_proj");
    const bool lewm = names == LWM_LEWM_NAMES_LEWM;
    if (c.encoder == LWM_ENCODER_VECTOR_MLP) {
        // VectorMlpEncoder (world_model/model.rs:215-250): layers.{j}, norms.{j}
        const std::string p = "observation_encoder.vector_mlp";
        const int nk = c.obs_norm == LWM_NORM_NONE ? kNormNone : kNormLayer;
        w.enc_lin.resize(c.obs_depth);
        w.enc_norm.resize(c.obs_depth);
        for (uint32_t j = 0; j < c.obs_depth; ++j) {
            const uint32_t in = j == 0 ? c.obs_dim : c.obs_hidden_dim;
            const uint32_t o = j + 1 == c.obs_depth ? D : c.obs_hidden_dim;
            w.enc_lin[j] = k.lin(o, in, true, p + ".layers." + std::to_string(j));
            if (j + 1 < c.obs_depth) w.enc_norm[j] = k.norm(nk, c.obs_hidden_dim, p + ".norms." + std::to_string(j));
        }
    } else {
        // HfVitEncoder (vit.rs:30-45) with the Hugging Face ViT paths
        const std::string e = lewm ? "encoder" : "observation_encoder.encoder";
        const uint32_t vh = c.vit_hidden, p = c.patch_size, side = c.image_size / p;
        w.cls = k.take(vh, 4, 0, e + ".embeddings.cls_token", {1, 1, vh});
        w.vpos = k.take(static_cast<size_t>(side * side + 1) * vh, 4, 0, e + ".embeddings.position_embeddings",
                        {1, side * side + 1, vh});
        w.patch = k.lin(vh, c.channels * p * p, true, e + ".embeddings.patch_embeddings.projection",
                        {vh, c.channels, p, p});
        w.vit.resize(c.vit_layers);
        for (uint32_t l = 0; l < c.vit_layers; ++l) {
            const std::string q = e + ".encoder.layer." + std::to_string(l);
            VitBlockW& b = w.vit[l];
            b.ln1 = k.norm(kNormLayer, vh, q + ".layernorm_before");
            b.q = k.lin(vh, vh, c.qkv_bias != 0, q + ".attention.attention.query");
            b.k = k.lin(vh, vh, c.qkv_bias != 0, q + ".attention.attention.key");
            b.v = k.lin(vh, vh, c.qkv_bias != 0, q + ".attention.attention.value");
            b.o = k.lin(vh, vh, true, q + ".attention.output.dense");
            b.ln2 = k.norm(kNormLayer, vh, q + ".layernorm_after");
            b.fc1 = k.lin(c.vit_mlp, vh, true, q + ".intermediate.dense");
            b.fc2 = k.lin(vh, c.vit_mlp, true, q + ".output.dense");
        }
        w.vit_norm = k.norm(kNormLayer, vh, e + ".layernorm");
        w.projector = k.mlp(vh, c.projector_hidden, D, c.projector_norm, lewm ? "projector" : "observation_encoder.projector");
    }
    w.count = k.off;
    if (out) *out = w;
    return k.off;
}

// SplitMix64 stream and Box-Muller normals for the seeded init.
struct Mix {
    uint64_t s;
    uint64_t next() {
        s += 0x9E3779B97F4A7C15ull;
        uint64_t v = s;
        v = (v ^ (v >> 30)) * 0xBF58476D1CE4E5B9ull;
        v = (v ^ (v >> 27)) * 0x94D049BB133111EBull;
        return v ^ (v >> 31);
    }
    double unit() { return (static_cast<double>(next() >> 11) + 0.5) * (1.0 / 9007199254740992.0); }
    double normal() { return std::sqrt(-2.0 * std::log(unit())) * std::cos(6.283185307179586 * unit()); }
};

}  // namespace

size_t lewm_walk(const lwm_lewm_config& c, const float* base, LewmWeights* out) { return walk(c, base, out, nullptr); }

size_t lewm_named_tensors(const lwm_lewm_config& c, int names, std::vector<NamedTensor>* out) {
    const char* why = nullptr;
    if (!lewm_config_valid(c, &why)) return 0;
    return walk(c, nullptr, nullptr, nullptr, out, names);
}

bool lewm_config_valid(const lwm_lewm_config& c, const char** why) {
    auto bad = [&](const char* m) { *why = m; return false; };
    if (!c.embed_dim || !c.action_dim || !c.smoothed_dim || !c.action_mlp_scale) return bad("LeWM dims must be > 0");
    if (!c.history_size || c.num_frames < c.history_size)
        return bad("predictor.num_frames must be >= history_size > 0");
    if (!c.pred_hidden_dim || !c.depth || !c.heads || !c.dim_head || !c.mlp_dim || !c.pred_proj_hidden)
        return bad("LeWM predictor dims must be > 0");
    if (c.dim_head > 128) return bad("dim_head must be <= 128");
    if (c.pred_hidden_dim > 1024 || c.embed_dim > 2048) return bad("pred_hidden_dim must be <= 1024 and embed_dim <= 2048");
    if (c.pred_proj_norm < 0 || c.pred_proj_norm > 2) return bad("unknown pred_proj norm");
    if (c.encoder == LWM_ENCODER_VECTOR_MLP) {
        if (c.obs_depth < 2) return bad("VectorMlp depth must be at least 2");
        if (!c.obs_dim || !c.obs_hidden_dim) return bad("VectorMlp dims must be > 0");
    } else if (c.encoder == LWM_ENCODER_VIT) {
        if (!c.patch_size || c.image_size % c.patch_size) return bad("image_size must be a multiple of patch_size");
        if (!c.vit_heads || c.vit_hidden % c.vit_heads) return bad("vit_hidden must be a multiple of vit_heads");
        if (c.vit_hidden / c.vit_heads > 128) return bad("ViT head dim must be <= 128");
        if (!c.channels || !c.vit_layers || !c.vit_mlp || !c.projector_hidden) return bad("ViT dims must be > 0");
        if (c.projector_norm < 0 || c.projector_norm > 2) return bad("unknown projector norm");
    } else {
        return bad("unknown observation encoder");
    }
    return true;
}

cudaError_t Arena::ensure(size_t n) {
    if (n <= floats) return cudaSuccess;
    release();
    cudaError_t e = cudaMalloc(&ptr, n * sizeof(float));
    if (e == cudaSuccess) floats = n;
    return e;
}

void Arena::release() {
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    floats = 0;
}

LewmModel::~LewmModel() {
    g_score.reset();
    g_enc.reset();
    g_score_cand.reset();
    g_score_roll.reset();
    if (blob_bf16) cudaFree(blob_bf16);
    if (vit_qkv) cudaFree(vit_qkv);
    if (vo_blob) cudaFree(vo_blob);
    if (pred_w) cudaFree(pred_w);
    if (split.tc_err) cudaFree(split.tc_err);
    if (split.partial) cudaFree(split.partial);
    if (split.counters) cudaFree(split.counters);
    if (split_cand.partial) cudaFree(split_cand.partial);
    if (split_cand.counters) cudaFree(split_cand.counters);
    ws.release();
    enc.release();
    if (blob) cudaFree(blob);
    if (emb) cudaFree(emb);  // goal lives in the same allocation
}

namespace {

#define LWM_CU(x)                              \
    do {                                       \
        const cudaError_t e_ = (x);            \
        if (e_ != cudaSuccess) return e_;      \
    } while (0)

cudaError_t gemm_f32(const SplitScratch* sp, const GemmArgs& g, cudaStream_t s) { return lwm::gemm_f32(g, s, sp); }

GemmArgs gemm(const float* A, uint32_t lda, const Lin& l, float* C, uint32_t ldc, uint32_t M, int act = kActNone) {
    GemmArgs g{};
    g.A = A;
    g.W = l.w;
    g.bias = l.b;
    g.C = C;
    g.M = M;
    g.N = l.out;
    g.K = l.in;
    g.lda = lda;
    g.ldw = l.in;
    g.Wb = l.wb;
    g.ldc = ldc;
    g.act = act;
    return g;
}

// Mlp::forward on the device: fc1 -> norm + GELU -> fc2.
cudaError_t mlp(const SplitScratch* sp, const MlpW& m, const float* x, uint32_t n, float* hid, float* out,
                cudaStream_t s, int& launches) {
    LWM_CU(gemm_f32(sp, gemm(x, m.fc1.in, m.fc1, hid, m.fc1.out, n), s));
    LWM_CU(launch_norm_act(hid, n, m.fc1.out, m.norm.kind, m.norm.w, m.norm.b, m.norm.rm, m.norm.rv, s));
    LWM_CU(gemm_f32(sp, gemm(hid, m.fc1.out, m.fc2, out, m.fc2.out, n), s));
    launches += 3;
    return cudaSuccess;
}

}  // namespace

cudaError_t LewmModel::score_body(const float* cand, uint32_t S, uint32_t T, float* scores, float* last_emb,
                                  cudaStream_t s, int part) {
    const SplitScratch* sp = part == 1 ? &split_cand : &split;
    const uint32_t D = c.embed_dim, hid = c.pred_hidden_dim, inner = c.heads * c.dim_head, A = c.action_dim;
    const uint32_t sm = c.smoothed_dim, ah = c.action_mlp_scale * D, ph = c.pred_proj_hidden;
    const size_t bs = static_cast<size_t>(B) * S, all = bs * T;
    const uint32_t W = history;  // window tokens per sequence (at most)
    const uint32_t nframes = T + 1;
    // workspace layout (floats)
    size_t off = 0;
    auto take = [&](size_t n) { const size_t o = off; off += (n + 63) & ~static_cast<size_t>(63); return o; };
    const size_t o_sm = take(all * sm), o_ah = take(all * ah), o_act = take(all * D), o_cond = take(all * hid);
    const size_t o_ada = take(static_cast<size_t>(c.depth) * all * 6 * hid);
    const size_t o_frames = take(bs * nframes * D), o_X = take(bs * W * D), o_x = take(bs * W * hid);
    const size_t o_y = take(bs * W * hid), o_qkv = take(bs * W * 3 * inner), o_att = take(bs * W * inner);
    const size_t o_f = take(bs * W * c.mlp_dim), o_last = take(bs * hid), o_po = take(bs * D);
    const size_t o_p1 = take(bs * ph), o_pred = take(bs * D);
    // the fused rollout (bf16, the image model's predictor shape) and its exchange buffers
    const bool fused = pred_ready && precision == LWM_PRECISION_BF16 && history == 1 && T >= h && !w.has_proj;
    const size_t xa_bytes = static_cast<size_t>((bs + 127) / 128) * 2 * 8 * 3 * 2048;
    const size_t o_xch = fused ? take((lewm_pred_exchange_bytes(static_cast<uint32_t>(bs)) + 3) / 4) : 0;
    LWM_CU(ws.ensure(off));
    float* base = ws.ptr;
    float *f_sm = base + o_sm, *f_ah = base + o_ah, *f_act = base + o_act, *f_cond = base + o_cond;
    float *f_ada = base + o_ada, *f_frames = base + o_frames, *f_X = base + o_X, *f_x = base + o_x;
    float *f_y = base + o_y, *f_qkv = base + o_qkv, *f_att = base + o_att, *f_f = base + o_f;
    float *f_last = base + o_last, *f_po = base + o_po, *f_p1 = base + o_p1, *f_pred = base + o_pred;
    int n = 0;
    split_launches = 0;
    const uint32_t rows_all = static_cast<uint32_t>(all);
    if (part != 2) {
        // ActionEmbedder over every (sample, time) token (modules.rs:150-158): the
        // small-K first two layers in one kernel, the last as a GEMM
        if (action_embed_supported(A, sm) && w.act_conv.in == A && w.act_fc1.in == sm) {
            LWM_CU(launch_action_embed(cand, A, w.act_conv.w, w.act_conv.b, sm, w.act_fc1.w, w.act_fc1.b, ah, f_ah,
                                       rows_all, s));
            n += 1;
        } else {
            LWM_CU(gemm_f32(sp, gemm(cand, A, w.act_conv, f_sm, sm, rows_all), s));
            LWM_CU(gemm_f32(sp, gemm(f_sm, sm, w.act_fc1, f_ah, ah, rows_all, kActSilu), s));
            n += 2;
        }
        LWM_CU(gemm_f32(sp, gemm(f_ah, ah, w.act_fc2, f_act, D, rows_all), s));
        n += 1;
        // cond -> SiLU -> AdaLN table of every layer (ConditionalBlock::forward, modules.rs:317-320);
        // the condition of a token depends only on its action, so the table is
        // built once per scoring call for all (sample, time) tokens.
        const float* cond = f_act;
        if (w.has_proj) {
            LWM_CU(gemm_f32(sp, gemm(f_act, D, w.cond_proj, f_cond, hid, rows_all), s));
            ++n;
            cond = f_cond;
        }
        LWM_CU(launch_silu(cond, f_cond, all * hid, s));
        ++n;
        for (uint32_t l = 0; l < c.depth; ++l) {
            float* table = f_ada + static_cast<size_t>(l) * all * 6 * hid;
            LWM_CU(gemm_f32(sp, gemm(f_cond, hid, w.blocks[l].ada, table, 6 * hid, rows_all), s));
            ++n;
        }
        if (part == 1) {
            launches = n + split_launches;
            return cudaSuccess;
        }
    }
    if (fused) {
        // the whole rollout in one launch
        PredArgs a = pred;
        a.tokens = static_cast<uint32_t>(bs);
        a.S = S;
        a.T = T;
        a.h = h;
        a.steps = T - h + 1;
        a.emb = emb;
        a.pos = w.pos;
        a.ada = base + o_ada;
        a.pred = f_pred;
        a.xa = reinterpret_cast<uint8_t*>(base + o_xch);
        a.xp = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(base + o_xch) + xa_bytes);
        a.err = split.tc_err;
        a.wait_polls = 0;
        LWM_CU(launch_lewm_pred(a, s));
        ++n;
        LWM_CU(launch_goal_cost(f_pred, goal, S, bs, D, scores, s));
        ++n;
        if (last_emb) LWM_CU(cudaMemcpyAsync(last_emb, f_pred, bs * D * sizeof(float), cudaMemcpyDeviceToDevice, s));
        launches = n + split_launches;
        return cudaSuccess;
    }
    LWM_CU(launch_frames_init(emb, h, S, f_frames, nframes, bs, D, s));
    ++n;
    const float scale = static_cast<float>(std::pow(static_cast<double>(c.dim_head), -0.5));
    uint32_t count = h;
    for (uint32_t step = 0; step + h <= T; ++step) {
        const uint32_t upper = h + step, lo = upper > history ? upper - history : 0, wl = upper - lo;
        const uint32_t rows = static_cast<uint32_t>(bs * wl);
        RowMap map;
        map.t = wl;
        map.T = T;
        map.lo = lo;
        LWM_CU(launch_window(f_frames, nframes, w.pos, f_X, static_cast<uint32_t>(bs), wl, lo, D, s));
        ++n;
        float* x = f_X;
        if (w.has_proj) {
            LWM_CU(gemm_f32(sp, gemm(f_X, D, w.input_proj, f_x, hid, rows), s));
            ++n;
            x = f_x;
        }
        for (uint32_t l = 0; l < c.depth; ++l) {
            const BlockW& b = w.blocks[l];
            const float* ada = f_ada + static_cast<size_t>(l) * all * 6 * hid;
            LWM_CU(launch_ada_ln(x, f_y, rows, hid, ada, 6 * hid, 0, hid, map, b.attn_norm.w, b.attn_norm.b, s));
            const float* att = f_att;
            uint32_t ld_att = inner;
            const bool folded = wl == 1 && b.vo.w && !b.qkv.wb;
            if (folded) {
                // one-token window, f32 weights: V and the out-projection as
                // the one folded map vo (x += g1 * (y Wvo^T + bvo))
                GemmArgs gv = gemm(f_y, hid, b.vo, x, hid, rows);
                gv.residual = 1;
                gv.gate = ada + 2 * hid;
                gv.ldg = 6 * hid;
                gv.map = map;
                LWM_CU(gemm_f32(sp, gv, s));
                n += 2;
            } else if (wl == 1) {
                // softmax over a single key is exactly 1: the attention output is V
                Lin v = b.qkv;
                v.w = b.qkv.w + static_cast<size_t>(2) * inner * hid;
                if (b.qkv.wb) v.wb = b.qkv.wb + static_cast<size_t>(2) * inner * hid;
                v.out = inner;
                LWM_CU(gemm_f32(sp, gemm(f_y, hid, v, f_att, inner, rows), s));
                n += 2;
            } else {
                LWM_CU(gemm_f32(sp, gemm(f_y, hid, b.qkv, f_qkv, 3 * inner, rows), s));
                LWM_CU(launch_attention(f_qkv, f_att, static_cast<uint32_t>(bs), wl, c.heads, c.dim_head, scale, 1, 1,
                                        s));
                n += 3;
            }
            if (!folded) {
                GemmArgs go = gemm(att, ld_att, b.to_out, x, hid, rows);
                go.residual = 1;
                go.gate = ada + 2 * hid;
                go.ldg = 6 * hid;
                go.map = map;
                LWM_CU(gemm_f32(sp, go, s));
                ++n;
            }
            LWM_CU(launch_ada_ln(x, f_y, rows, hid, ada, 6 * hid, 3 * hid, 4 * hid, map, b.mlp_norm.w, b.mlp_norm.b,
                                 s));
            LWM_CU(gemm_f32(sp, gemm(f_y, hid, b.fc1, f_f, c.mlp_dim, rows, kActGeluTanh), s));
            GemmArgs g2 = gemm(f_f, c.mlp_dim, b.fc2, x, hid, rows);
            g2.residual = 1;
            g2.gate = ada + 5 * hid;
            g2.ldg = 6 * hid;
            g2.map = map;
            LWM_CU(gemm_f32(sp, g2, s));
            n += 3;
        }
        // last token -> norm -> output_proj -> pred_proj (Transformer::forward_last, modules.rs:369-380)
        LWM_CU(launch_layernorm(x, f_last, static_cast<uint32_t>(bs), hid, wl, wl - 1, w.final_norm.w, w.final_norm.b,
                                1e-5f, s));
        ++n;
        const float* pin = f_last;
        if (w.has_proj) {
            LWM_CU(gemm_f32(sp, gemm(f_last, hid, w.output_proj, f_po, D, static_cast<uint32_t>(bs)), s));
            ++n;
            pin = f_po;
        }
        LWM_CU(mlp(sp, w.pred_proj, pin, static_cast<uint32_t>(bs), f_p1, f_pred, s, n));
        LWM_CU(launch_frames_put(f_pred, f_frames, nframes, count, bs, D, s));
        ++n;
        ++count;
    }
    LWM_CU(launch_goal_cost(f_pred, goal, S, bs, D, scores, s));
    ++n;
    if (last_emb) LWM_CU(cudaMemcpyAsync(last_emb, f_pred, bs * D * sizeof(float), cudaMemcpyDeviceToDevice, s));
    launches = n + split_launches;
    return cudaSuccess;
}

cudaError_t LewmModel::encode_vector(const float* obs, uint32_t n, float* out, cudaStream_t s) {
    LWM_CU(ensure_split());
    const SplitScratch* sp = &split;
    const uint32_t oh = c.obs_hidden_dim;
    LWM_CU(enc.ensure(static_cast<size_t>(2) * n * oh));
    float *a = enc.ptr, *b = enc.ptr + static_cast<size_t>(n) * oh;
    int k = 0;
    split_launches = 0;
    LWM_CU(gemm_f32(sp, gemm(obs, c.obs_dim, w.enc_lin[0], a, oh, n), s));
    ++k;
    for (uint32_t j = 0; j + 1 < c.obs_depth; ++j) {
        const Norm& nm = w.enc_norm[j];
        LWM_CU(launch_norm_act(a, n, oh, nm.kind, nm.w, nm.b, nullptr, nullptr, s));
        ++k;
        if (j + 2 < c.obs_depth) {
            LWM_CU(gemm_f32(sp, gemm(a, oh, w.enc_lin[j + 1], b, oh, n), s));
            ++k;
            float* t = a;
            a = b;
            b = t;
        }
    }
    LWM_CU(gemm_f32(sp, gemm(a, oh, w.enc_lin[c.obs_depth - 1], out, c.embed_dim, n), s));
    launches = k + 1 + split_launches;
    return cudaSuccess;
}

// The encoder workspace of n frames: the patch matrix first (offset 0), so
// that preprocessing can write it directly (patch_buffer).
size_t LewmModel::encoder_layout(uint32_t n, EncoderOffsets* o) const {
    const uint32_t vh = c.vit_hidden, p = c.patch_size, side = c.image_size / p, np = side * side, t = np + 1;
    const uint32_t kdim = c.channels * p * p;
    size_t off = 0;
    auto take = [&](size_t k) { const size_t q = off; off += (k + 63) & ~static_cast<size_t>(63); return q; };
    EncoderOffsets e;
    e.patch = take(static_cast<size_t>(n) * np * kdim);
    e.pe = take(static_cast<size_t>(n) * np * vh);
    e.x = take(static_cast<size_t>(n) * t * vh);
    e.y = take(static_cast<size_t>(n) * t * vh);
    e.qkv = take(static_cast<size_t>(n) * t * 3 * vh);
    e.att = take(static_cast<size_t>(n) * t * vh);
    e.f = take(static_cast<size_t>(n) * t * c.vit_mlp);
    e.cls = take(static_cast<size_t>(n) * vh);
    e.ph = take(static_cast<size_t>(n) * c.projector_hidden);
    if (o) *o = e;
    return off;
}

cudaError_t LewmModel::patch_buffer(uint32_t n, float** patches) {
    LWM_CU(enc.ensure(encoder_layout(n, nullptr)));
    *patches = enc.ptr;  // EncoderOffsets::patch == 0
    return cudaSuccess;
}

cudaError_t LewmModel::encode_pixels_body(const float* pix, uint32_t n, float* out, cudaStream_t s) {
    LWM_CU(enc.ensure(encoder_layout(n, nullptr)));
    LWM_CU(launch_patchify(pix, enc.ptr, n, c.channels, c.image_size, c.patch_size, s));
    LWM_CU(encode_patches_body(n, out, s));
    launches += 1;
    return cudaSuccess;
}

// HfVitEncoder::forward from the patch matrix in the workspace: patch
// embedding GEMM, [CLS] + position embeddings, the encoder layers, the final
// norm of the CLS token, then the projector.
cudaError_t LewmModel::encode_patches_body(uint32_t n, float* out, cudaStream_t s) {
    const PdlScope pdl;  // the encoder's launches overlap each other's prologues
    const SplitScratch* sp = &split;
    const uint32_t vh = c.vit_hidden, p = c.patch_size, side = c.image_size / p, np = side * side, t = np + 1;
    const uint32_t kdim = c.channels * p * p, H = c.vit_heads, dh = vh / H;
    EncoderOffsets o;
    LWM_CU(enc.ensure(encoder_layout(n, &o)));
    float* e = enc.ptr;
    float *f_patch = e + o.patch, *f_pe = e + o.pe, *f_x = e + o.x, *f_y = e + o.y, *f_qkv = e + o.qkv;
    float *f_att = e + o.att, *f_f = e + o.f, *f_cls = e + o.cls, *f_ph = e + o.ph;
    const uint32_t rows = n * t;
    int k = 0;
    split_launches = 0;
    LWM_CU(gemm_f32(sp, gemm(f_patch, kdim, w.patch, f_pe, vh, n * np), s));
    LWM_CU(launch_vit_assemble(f_pe, w.cls, w.vpos, f_x, n, np, vh, s));
    k += 2;
    const float scale = 1.0f / std::sqrt(static_cast<float>(dh));
    for (uint32_t l = 0; l < c.vit_layers; ++l) {
        const VitBlockW& b = w.vit[l];
        LWM_CU(launch_layernorm(f_x, f_y, rows, vh, 1, 0, b.ln1.w, b.ln1.b, c.vit_eps, s));
        LWM_CU(gemm_f32(sp, gemm(f_y, vh, b.qkv, f_qkv, 3 * vh, rows), s));
        LWM_CU(launch_attention(f_qkv, f_att, n, t, H, dh, scale, 0, 0, s));
        GemmArgs go = gemm(f_att, vh, b.o, f_x, vh, rows);
        go.residual = 1;
        LWM_CU(gemm_f32(sp, go, s));
        LWM_CU(launch_layernorm(f_x, f_y, rows, vh, 1, 0, b.ln2.w, b.ln2.b, c.vit_eps, s));
        LWM_CU(gemm_f32(sp, gemm(f_y, vh, b.fc1, f_f, c.vit_mlp, rows, kActGeluErf), s));
        GemmArgs g2 = gemm(f_f, c.vit_mlp, b.fc2, f_x, vh, rows);
        g2.residual = 1;
        LWM_CU(gemm_f32(sp, g2, s));
        k += 7;
    }
    LWM_CU(launch_layernorm(f_x, f_cls, n, vh, t, 0, w.vit_norm.w, w.vit_norm.b, c.vit_eps, s));
    ++k;
    LWM_CU(mlp(sp, w.projector, f_cls, n, f_ph, out, s, k));
    launches = k + split_launches;
    return cudaSuccess;
}

void GraphCache::reset() {
    if (exec) cudaGraphExecDestroy(exec);
    exec = nullptr;
    seen = false;
}

// The ViT's query, key and value projections as one Linear of 3 x vit_hidden
// outputs (weight rows q, then k, then v; the biases alike), so each layer
// runs one GEMM into the [rows, 3 vit_hidden] buffer that the three filled
// column range by column range (HfVitEncoder's SelfAttention: three Linears
// of the same input).
// One-token windows make the attention output V itself, so the attention
// half-layer is two chained linear maps: y -> V = y Wv^T + bv -> V Wo^T + bo.
// Their product, Wvo = Wo Wv and bvo = Wo bv + bo, is formed once here (in
// double, rounded to f32) and replaces both GEMMs on the f32 path; results
// differ from the two-GEMM order by f32 rounding only.
cudaError_t LewmModel::fold_v_out() {
    if (vo_blob || w.blocks.empty()) return cudaSuccess;
    const size_t hid = c.pred_hidden_dim, inner = static_cast<size_t>(c.heads) * c.dim_head;
    const size_t per = hid * hid + hid;
    std::vector<float> wv(inner * hid), bv(inner), wo(hid * inner), bo(hid), out(per * w.blocks.size());
    std::vector<double> acc(hid);
    for (size_t l = 0; l < w.blocks.size(); ++l) {
        const BlockW& b = w.blocks[l];
        if (b.qkv.in != hid || b.qkv.out != 3 * inner || b.to_out.in != inner || b.to_out.out != hid) return cudaSuccess;
        LWM_CU(cudaMemcpy(wv.data(), b.qkv.w + 2 * inner * hid, wv.size() * sizeof(float), cudaMemcpyDeviceToHost));
        LWM_CU(cudaMemcpy(wo.data(), b.to_out.w, wo.size() * sizeof(float), cudaMemcpyDeviceToHost));
        std::fill(bv.begin(), bv.end(), 0.0f);
        std::fill(bo.begin(), bo.end(), 0.0f);
        if (b.qkv.b) LWM_CU(cudaMemcpy(bv.data(), b.qkv.b + 2 * inner, inner * sizeof(float), cudaMemcpyDeviceToHost));
        if (b.to_out.b) LWM_CU(cudaMemcpy(bo.data(), b.to_out.b, hid * sizeof(float), cudaMemcpyDeviceToHost));
        float* dst = out.data() + l * per;
        for (size_t o = 0; o < hid; ++o) {
            std::fill(acc.begin(), acc.end(), 0.0);
            double bias = bo[o];
            for (size_t k = 0; k < inner; ++k) {
                const double a = wo[o * inner + k];
                const float* row = wv.data() + k * hid;
                for (size_t i = 0; i < hid; ++i) acc[i] += a * row[i];
                bias += a * bv[k];
            }
            for (size_t i = 0; i < hid; ++i) dst[o * hid + i] = static_cast<float>(acc[i]);
            dst[hid * hid + o] = static_cast<float>(bias);
        }
    }
    LWM_CU(cudaMalloc(&vo_blob, out.size() * sizeof(float)));
    LWM_CU(cudaMemcpy(vo_blob, out.data(), out.size() * sizeof(float), cudaMemcpyHostToDevice));
    for (size_t l = 0; l < w.blocks.size(); ++l) {
        Lin& vo = w.blocks[l].vo;
        vo.w = vo_blob + l * per;
        vo.b = vo_blob + l * per + hid * hid;
        vo.in = vo.out = static_cast<uint32_t>(hid);
        vo.wb = nullptr;
    }
    return cudaSuccess;
}

cudaError_t LewmModel::fuse_vit_qkv() {
    if (c.encoder != LWM_ENCODER_VIT || w.vit.empty() || vit_qkv) return cudaSuccess;
    const size_t vh = c.vit_hidden, per = 3 * vh * vh + 3 * vh;
    LWM_CU(cudaMalloc(&vit_qkv, per * w.vit.size() * sizeof(float)));
    for (size_t l = 0; l < w.vit.size(); ++l) {
        VitBlockW& b = w.vit[l];
        float* dst = vit_qkv + l * per;
        const Lin* src[3] = {&b.q, &b.k, &b.v};
        for (int i = 0; i < 3; ++i) {
            LWM_CU(cudaMemcpy(dst + i * vh * vh, src[i]->w, vh * vh * sizeof(float), cudaMemcpyDeviceToDevice));
            if (src[i]->b)
                LWM_CU(cudaMemcpy(dst + 3 * vh * vh + i * vh, src[i]->b, vh * sizeof(float), cudaMemcpyDeviceToDevice));
        }
        b.qkv.w = dst;
        b.qkv.b = b.q.b ? dst + 3 * vh * vh : nullptr;
        b.qkv.out = static_cast<uint32_t>(3 * vh);
        b.qkv.in = static_cast<uint32_t>(vh);
        b.qkv.wb = nullptr;
    }
    return cudaSuccess;
}

namespace {

// 4 M floats of partial tiles (16 splits of 64 tiles) and 64 K tile counters
cudaError_t alloc_split(SplitScratch& sp, int* extra_launches) {
    if (sp.partial) return cudaSuccess;
    constexpr size_t kPartial = static_cast<size_t>(4) << 20, kCounters = 65536;
    LWM_CU(cudaMalloc(&sp.partial, kPartial * sizeof(float)));
    LWM_CU(cudaMalloc(&sp.counters, kCounters * sizeof(unsigned int)));
    LWM_CU(cudaMemset(sp.counters, 0, kCounters * sizeof(unsigned int)));
    sp.floats = kPartial;
    sp.n_counters = kCounters;
    sp.extra_launches = extra_launches;
    return cudaSuccess;
}

}  // namespace

cudaError_t LewmModel::ensure_split() { return alloc_split(split, &split_launches); }

// Same sizes as `split`, the same tensor-core error word: the candidate-only
// part of scoring sums its split-K partials in the same order as on `split`.
cudaError_t LewmModel::ensure_split_cand() {
    LWM_CU(alloc_split(split_cand, &split_launches));
    split_cand.tc_err = split.tc_err;
    return cudaSuccess;
}

namespace {

// Every Linear of the model (the GEMM weights).
template <class F>
void for_each_lin(LewmWeights& w, F f) {
    for (Lin* l : {&w.act_conv, &w.act_fc1, &w.act_fc2, &w.input_proj, &w.cond_proj, &w.output_proj,
                   &w.pred_proj.fc1, &w.pred_proj.fc2, &w.patch, &w.projector.fc1, &w.projector.fc2})
        f(*l);
    for (BlockW& b : w.blocks)
        for (Lin* l : {&b.qkv, &b.to_out, &b.fc1, &b.fc2, &b.ada}) f(*l);
    for (Lin& l : w.enc_lin) f(l);
    for (VitBlockW& b : w.vit)
        for (Lin* l : {&b.qkv, &b.o, &b.fc1, &b.fc2}) f(*l);
}

}  // namespace

cudaError_t LewmModel::set_precision(int p, cudaStream_t s) {
    if (p == precision) return cudaSuccess;
    LWM_CU(cudaStreamSynchronize(s));
    g_score.reset();  // captured launches hold the old weight pointers
    g_enc.reset();
    if (p == LWM_PRECISION_F32) {
        for_each_lin(w, [](Lin& l) { l.wb = nullptr; });
        if (blob_bf16) cudaFree(blob_bf16);
        blob_bf16 = nullptr;
        if (pred_w) cudaFree(pred_w);
        pred_w = nullptr;
        pred_ready = false;
        if (split.tc_err) cudaFree(split.tc_err);
        split.tc_err = nullptr;
        precision = p;
        return cudaSuccess;
    }
    // one bf16 slot per weight matrix, each 256-byte aligned
    size_t total = 0;
    for_each_lin(w, [&](Lin& l) {
        if (l.w) total += (static_cast<size_t>(l.out) * l.in + 127) & ~static_cast<size_t>(127);
    });
    LWM_CU(ensure_split());
    if (!split.tc_err) {
        LWM_CU(cudaMalloc(&split.tc_err, 4 * sizeof(int)));
        LWM_CU(cudaMemset(split.tc_err, 0, 4 * sizeof(int)));
    }
    LWM_CU(cudaMalloc(&blob_bf16, std::max<size_t>(total, 1) * sizeof(uint16_t)));
    size_t off = 0;
    cudaError_t err = cudaSuccess;
    for_each_lin(w, [&](Lin& l) {
        if (!l.w || err != cudaSuccess) return;
        const size_t n = static_cast<size_t>(l.out) * l.in;
        err = launch_f32_to_bf16(l.w, blob_bf16 + off, n, s);
        l.wb = blob_bf16 + off;
        off += (n + 127) & ~static_cast<size_t>(127);
    });
    LWM_CU(err);
    LWM_CU(build_pred(s));
    LWM_CU(cudaStreamSynchronize(s));
    precision = p;
    return cudaSuccess;
}

// The fused predictor's packed weights and its per-half-layer views, when the
// model has the shape lewm_pred_kernel takes; otherwise the rollout keeps its
// per-GEMM launch sequence.
cudaError_t LewmModel::build_pred(cudaStream_t s) {
    pred_ready = false;
    const char* why = nullptr;
    if (!lewm_pred_supported(c, c.history_size, &why)) return cudaSuccess;
    const uint32_t inner = c.heads * c.dim_head, L = c.depth;
    size_t total = 0;
    for (uint32_t l = 0; l < L; ++l) total += 8 * (lewm_pred_half_bytes(inner) + lewm_pred_half_bytes(c.mlp_dim));
    total += 8 * lewm_pred_half_bytes(c.pred_proj_hidden);
    if (!pred_w) LWM_CU(cudaMalloc(&pred_w, total));
    PredArgs a{};
    size_t off = 0;
    auto half = [&](uint32_t i, int kind, uint32_t layer, const float* w1, uint32_t row0, uint32_t ld1,
                    const float* w2, uint32_t ld2, uint32_t n1_total) -> cudaError_t {
        PredHalf& h = a.half[i];
        h.w = pred_w + off;
        h.bytes = static_cast<uint32_t>(lewm_pred_half_bytes(n1_total));
        h.n1 = n1_total / 8;
        h.kind = kind;
        h.layer = layer;
        const cudaError_t e = lewm_pred_pack(w1, row0, ld1, w2, ld2, n1_total, pred_w + off, s);
        off += static_cast<size_t>(8) * h.bytes;
        return e;
    };
    for (uint32_t l = 0; l < L; ++l) {
        const BlockW& b = w.blocks[l];
        // attention half: V = rows [2 inner, 3 inner) of the qkv projection, then the out-projection
        LWM_CU(half(2 * l, 0, l, b.qkv.w, 2 * inner, b.qkv.in, b.to_out.w, b.to_out.in, inner));
        PredHalf& ha = a.half[2 * l];
        ha.b1 = b.qkv.b ? b.qkv.b + static_cast<size_t>(2) * inner : nullptr;
        ha.b2 = b.to_out.b;
        ha.ln_w = b.attn_norm.w;
        ha.ln_b = b.attn_norm.b;
        LWM_CU(half(2 * l + 1, 1, l, b.fc1.w, 0, b.fc1.in, b.fc2.w, b.fc2.in, c.mlp_dim));
        PredHalf& hm = a.half[2 * l + 1];
        hm.b1 = b.fc1.b;
        hm.b2 = b.fc2.b;
        hm.ln_w = b.mlp_norm.w;
        hm.ln_b = b.mlp_norm.b;
    }
    const MlpW& pp = w.pred_proj;
    LWM_CU(half(2 * L, 2, 0, pp.fc1.w, 0, pp.fc1.in, pp.fc2.w, pp.fc2.in, c.pred_proj_hidden));
    PredHalf& hp = a.half[2 * L];
    hp.b1 = pp.fc1.b;
    hp.b2 = pp.fc2.b;
    if (pp.norm.kind == kNormBatch) {
        hp.bn_w = pp.norm.w;
        hp.bn_b = pp.norm.b;
        hp.bn_rm = pp.norm.rm;
        hp.bn_rv = pp.norm.rv;
    }
    hp.ln_w = w.final_norm.w;
    hp.ln_b = w.final_norm.b;
    a.halves = 2 * L + 1;
    pred = a;
    pred_ready = true;
    return cudaSuccess;
}

namespace {

// Runs `body` through `cache`: the first call of a key runs it directly (so
// its workspaces get allocated), the second captures it into a CUDA graph,
// later calls replay the graph.
template <class F>
cudaError_t run_graphed(GraphCache& cache, const uint64_t (&key)[GraphCache::kKey], cudaStream_t s, int& launches,
                        F&& body) {
    const bool same = cache.seen && std::memcmp(cache.key, key, sizeof key) == 0;
    if (same && cache.exec) {
        launches = cache.launches;
        return cudaGraphLaunch(cache.exec, s);
    }
    if (!same) {
        cache.reset();
        std::memcpy(cache.key, key, sizeof key);
        LWM_CU(body());
        cache.seen = true;
        return cudaSuccess;
    }
    cudaGraph_t graph = nullptr;
    LWM_CU(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    const cudaError_t e = body();
    const cudaError_t e2 = cudaStreamEndCapture(s, &graph);
    if (e != cudaSuccess || e2 != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        return e != cudaSuccess ? e : e2;
    }
    const cudaError_t e3 = cudaGraphInstantiate(&cache.exec, graph, 0);
    cudaGraphDestroy(graph);
    LWM_CU(e3);
    cache.launches = launches;
    return cudaGraphLaunch(cache.exec, s);
}

inline uint64_t u(const void* p) { return reinterpret_cast<uint64_t>(p); }

}  // namespace

cudaError_t LewmModel::score(const float* cand, uint32_t S, uint32_t T, float* scores, float* last_emb,
                             cudaStream_t s) {
    LWM_CU(ensure_split());
    const uint64_t key[GraphCache::kKey] = {u(cand), u(scores), u(last_emb), S, T, B, u(emb), u(goal), h, history,
                                            u(ws.ptr), ws.floats, u(s), 1};
    if (!join_ev)
        return run_graphed(g_score, key, s, launches, [&] { return score_body(cand, S, T, scores, last_emb, s); });
    // the encoder that writes emb / goal runs on another stream until join_ev
    LWM_CU(ensure_split_cand());
    uint64_t key1[GraphCache::kKey], key2[GraphCache::kKey];
    std::memcpy(key1, key, sizeof key);
    std::memcpy(key2, key, sizeof key);
    key1[GraphCache::kKey - 1] = 4;
    key2[GraphCache::kKey - 1] = 5;
    LWM_CU(run_graphed(g_score_cand, key1, s, launches,
                       [&] { return score_body(cand, S, T, scores, last_emb, s, 1); }));
    const int n1 = launches;
    LWM_CU(cudaStreamWaitEvent(s, join_ev, 0));
    LWM_CU(run_graphed(g_score_roll, key2, s, launches,
                       [&] { return score_body(cand, S, T, scores, last_emb, s, 2); }));
    launches += n1;
    return cudaSuccess;
}

cudaError_t LewmModel::ensure_context(uint32_t B_, uint32_t h_, bool packed, cudaStream_t s) {
    const size_t D = c.embed_dim;
    const size_t need = static_cast<size_t>(B_) * h_ * D, need_goal = static_cast<size_t>(B_) * D;
    const size_t cap = std::max(need, need_goal);
    if (emb && (packed ? ctx_cap == need && need >= need_goal : ctx_cap >= cap)) return cudaSuccess;
    LWM_CU(cudaStreamSynchronize(s));
    if (emb) cudaFree(emb);
    emb = goal = nullptr;
    ctx_cap = 0;
    LWM_CU(cudaMalloc(&emb, 2 * cap * sizeof(float)));
    goal = emb + cap;
    ctx_cap = cap;
    return cudaSuccess;
}

cudaError_t LewmModel::encode_pixels(const float* pix, uint32_t n, float* out, cudaStream_t s) {
    LWM_CU(ensure_split());
    const uint64_t key[GraphCache::kKey] = {u(pix), n, u(out), u(enc.ptr), enc.floats, u(s), 2};
    return run_graphed(g_enc, key, s, launches, [&] { return encode_pixels_body(pix, n, out, s); });
}

cudaError_t LewmModel::encode_patches(uint32_t n, float* out, cudaStream_t s) {
    LWM_CU(ensure_split());
    const uint64_t key[GraphCache::kKey] = {n, u(out), u(enc.ptr), enc.floats, u(s), 3};
    return run_graphed(g_enc, key, s, launches, [&] { return encode_patches_body(n, out, s); });
}

}  // namespace lwm

// ----------------------------------------------------------------- C ABI

extern "C" {

void lwm_lewm_config_vector(lwm_lewm_config* o) {
    std::memset(o, 0, sizeof *o);
    o->embed_dim = 192;
    o->action_dim = 2;
    o->smoothed_dim = 2;
    o->action_mlp_scale = 4;
    o->history_size = 1;
    o->num_frames = 1;
    o->pred_hidden_dim = 192;
    o->depth = 4;
    o->heads = 8;
    o->dim_head = 32;
    o->mlp_dim = 768;
    o->pred_proj_hidden = 512;
    o->pred_proj_norm = LWM_NORM_LAYER;
    o->encoder = LWM_ENCODER_VECTOR_MLP;
    o->obs_dim = 16;
    o->obs_hidden_dim = 512;
    o->obs_depth = 3;
    o->obs_norm = LWM_NORM_LAYER;
}

void lwm_lewm_config_image(lwm_lewm_config* o) {
    std::memset(o, 0, sizeof *o);
    o->embed_dim = 192;
    o->action_dim = 2;
    o->smoothed_dim = 2;
    o->action_mlp_scale = 4;
    o->history_size = 1;
    o->num_frames = 1;
    o->pred_hidden_dim = 192;
    o->depth = 6;
    o->heads = 16;
    o->dim_head = 64;
    o->mlp_dim = 2048;
    o->pred_proj_hidden = 2048;
    o->pred_proj_norm = LWM_NORM_BATCH;
    o->encoder = LWM_ENCODER_VIT;
    o->image_size = 224;
    o->patch_size = 16;
    o->vit_hidden = 192;
    o->vit_layers = 12;
    o->vit_heads = 3;
    o->vit_mlp = 768;
    o->vit_eps = 1e-12f;
    o->channels = 3;
    o->qkv_bias = 1;
    o->projector_hidden = 2048;
    o->projector_norm = LWM_NORM_BATCH;
}

size_t lwm_lewm_weight_count(const lwm_lewm_config* c) {
    const char* why = nullptr;
    if (!c || !lwm::lewm_config_valid(*c, &why)) return 0;
    return lwm::lewm_walk(*c, nullptr, nullptr);
}

lwm_status lwm_lewm_random_weights(const lwm_lewm_config* c, uint64_t seed, float* out, size_t count) {
    const char* why = nullptr;
    if (!c || !out || !lwm::lewm_config_valid(*c, &why)) return LWM_INVALID_ARGUMENT;
    std::vector<lwm::Spec> specs;
    const size_t n = lwm::walk(*c, nullptr, nullptr, &specs);
    if (count != n) return LWM_INVALID_ARGUMENT;
    lwm::Mix rng{seed ^ 0x6C65776D2D776D31ull};
    for (const lwm::Spec& sp : specs) {
        for (size_t j = 0; j < sp.n; ++j) {
            double v = 0.0;
            switch (sp.kind) {
                case 0: v = rng.normal() * std::sqrt(2.0 / sp.fan); break;
                case 1: v = (2.0 * rng.unit() - 1.0) / std::sqrt(static_cast<double>(sp.fan)); break;
                case 2: v = 1.0; break;
                case 3: v = 0.0; break;
                default: v = rng.normal() * 0.02; break;
            }
            out[sp.off + j] = static_cast<float>(v);
        }
    }
    return LWM_OK;
}

}  // extern "C"
