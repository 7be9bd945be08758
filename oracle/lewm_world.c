/*
 * lewm_world.c — CPU oracle of the LeWM / WorldModel scorer (TEST
 * INFRASTRUCTURE ONLY: the tests, the smoke check and the benchmark's CPU leg
 * use it; the product never links it).
 *
 * Restates, in f32 and in the reference's operation order:
 *   ActionEmbedder, Mlp, FeedForward, Attention, ConditionalBlock,
 *   Transformer::forward_last, Predictor::forward_last
 *       (src/models/lewm/modules.rs:9-399)
 *   LeWm::rollout_embeddings_with_history, goal_cost
 *       (src/models/lewm/model.rs:94-165; world_model/model.rs:84-160)
 *   VectorMlpEncoder (src/models/world_model/model.rs:207-274)
 *   HfVitEncoder::{forward, cls} (src/models/lewm/vit.rs:7-57) over the
 *   candle-transformers ViT (not in the reference tree; restated from the
 *   published ViT definition: conv patch embedding, CLS token, learned
 *   positions, pre-LayerNorm encoder blocks with exact-erf GELU, final
 *   LayerNorm) — parity of that third-party code is unpinned.
 * Candle semantics followed: Tensor::gelu is the tanh approximation, SiLU is
 * x / (1 + exp(-x)), LayerNorm divides by sqrt(var + eps) with the biased
 * variance, BatchNorm1d in eval mode uses the running statistics.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "lewm_oracle.h"

typedef struct {
    const float *w, *b;
} lin_t;
typedef struct {
    const float *w, *b, *rm, *rv; /* rm/rv only for BatchNorm */
    int kind;
} norm_t;
typedef struct {
    lin_t fc1;
    norm_t norm;
    lin_t fc2;
    uint32_t in, hid, out;
} mlp_t;
typedef struct {
    norm_t attn_norm;
    const float* qkv_w;
    lin_t to_out;
    norm_t mlp_norm;
    lin_t fc1, fc2, ada;
} block_t;
typedef struct {
    norm_t ln1, ln2;
    lin_t q, k, v, o, fc1, fc2;
} vit_block_t;

struct orc_lewm {
    lwm_lewm_config c;
    lin_t act_conv, act_fc1, act_fc2;
    const float* pos;
    lin_t input_proj, cond_proj, output_proj;
    int has_in_proj, has_out_proj;
    block_t* blocks;
    norm_t final_norm;
    mlp_t pred_proj;
    /* vector encoder */
    lin_t* enc_lin;
    norm_t* enc_norm;
    /* vit */
    const float *cls, *vpos;
    lin_t patch;
    vit_block_t* vit;
    norm_t vit_norm;
    mlp_t projector;
    float* blob;
};

/* ---------------------------------------------------------------- layout */

typedef struct {
    const float* base;
    size_t off;
    int count_only;
} cursor_t;

static const float* take(cursor_t* c, size_t n) {
    const float* p = c->count_only ? NULL : c->base + c->off;
    c->off += n;
    return p;
}

static lin_t take_lin(cursor_t* c, uint32_t out, uint32_t in, int bias) {
    lin_t l;
    l.w = take(c, (size_t)out * in);
    l.b = bias ? take(c, out) : NULL;
    return l;
}

static norm_t take_norm(cursor_t* c, int kind, uint32_t dim) {
    norm_t n = {0};
    n.kind = kind;
    if (kind == LWM_NORM_BATCH) {
        n.w = take(c, dim);
        n.b = take(c, dim);
        n.rm = take(c, dim);
        n.rv = take(c, dim);
    } else if (kind == LWM_NORM_LAYER) {
        n.w = take(c, dim);
        n.b = take(c, dim);
    }
    return n;
}

static mlp_t take_mlp(cursor_t* c, uint32_t in, uint32_t hid, uint32_t out, int norm) {
    mlp_t m;
    m.fc1 = take_lin(c, hid, in, 1);
    m.norm = take_norm(c, norm, hid);
    m.fc2 = take_lin(c, out, hid, 1);
    m.in = in;
    m.hid = hid;
    m.out = out;
    return m;
}

/* Walks the blob in the order documented with lwm_lewm_config; fills m when
 * it is non-NULL and returns the float count. */
static size_t walk(const lwm_lewm_config* cfg, const float* base, struct orc_lewm* m) {
    cursor_t c = {base, 0, base == NULL};
    const uint32_t D = cfg->embed_dim, A = cfg->action_dim, sm = cfg->smoothed_dim;
    const uint32_t hid = cfg->pred_hidden_dim, inner = cfg->heads * cfg->dim_head;
    lin_t act_conv = take_lin(&c, sm, A, 1);
    lin_t act_fc1 = take_lin(&c, cfg->action_mlp_scale * D, sm, 1);
    lin_t act_fc2 = take_lin(&c, D, cfg->action_mlp_scale * D, 1);
    const float* pos = take(&c, (size_t)cfg->num_frames * D);
    lin_t in_proj = {0}, cond_proj = {0}, out_proj = {0};
    if (hid != D) {
        in_proj = take_lin(&c, hid, D, 1);
        cond_proj = take_lin(&c, hid, D, 1);
    }
    if (m) m->blocks = (block_t*)calloc(cfg->depth, sizeof(block_t));
    for (uint32_t l = 0; l < cfg->depth; ++l) {
        block_t b;
        b.attn_norm = take_norm(&c, LWM_NORM_LAYER, hid);
        b.qkv_w = take(&c, (size_t)3 * inner * hid);
        b.to_out = take_lin(&c, hid, inner, 1);
        b.mlp_norm = take_norm(&c, LWM_NORM_LAYER, hid);
        b.fc1 = take_lin(&c, cfg->mlp_dim, hid, 1);
        b.fc2 = take_lin(&c, hid, cfg->mlp_dim, 1);
        b.ada = take_lin(&c, 6 * hid, hid, 1);
        if (m) m->blocks[l] = b;
    }
    norm_t final_norm = take_norm(&c, LWM_NORM_LAYER, hid);
    if (hid != D) out_proj = take_lin(&c, D, hid, 1);
    mlp_t pred_proj = take_mlp(&c, D, cfg->pred_proj_hidden, D, cfg->pred_proj_norm);
    if (m) {
        m->act_conv = act_conv;
        m->act_fc1 = act_fc1;
        m->act_fc2 = act_fc2;
        m->pos = pos;
        m->input_proj = in_proj;
        m->cond_proj = cond_proj;
        m->output_proj = out_proj;
        m->has_in_proj = hid != D;
        m->has_out_proj = hid != D;
        m->final_norm = final_norm;
        m->pred_proj = pred_proj;
    }
    if (cfg->encoder == LWM_ENCODER_VECTOR_MLP) {
        const uint32_t depth = cfg->obs_depth, oh = cfg->obs_hidden_dim;
        const int nk = cfg->obs_norm == LWM_NORM_NONE ? LWM_NORM_NONE : LWM_NORM_LAYER;
        if (m) {
            m->enc_lin = (lin_t*)calloc(depth, sizeof(lin_t));
            m->enc_norm = (norm_t*)calloc(depth, sizeof(norm_t));
        }
        for (uint32_t j = 0; j < depth; ++j) {
            const uint32_t in = j == 0 ? cfg->obs_dim : oh, out = j == depth - 1 ? D : oh;
            lin_t l = take_lin(&c, out, in, 1);
            norm_t n = {0};
            n.kind = LWM_NORM_NONE;
            if (j + 1 < depth) n = take_norm(&c, nk, oh);
            if (m) {
                m->enc_lin[j] = l;
                m->enc_norm[j] = n;
            }
        }
    } else {
        const uint32_t vh = cfg->vit_hidden, p = cfg->patch_size, np = (cfg->image_size / p) * (cfg->image_size / p);
        const float* cls = take(&c, vh);
        const float* vpos = take(&c, (size_t)(np + 1) * vh);
        lin_t patch = take_lin(&c, vh, cfg->channels * p * p, 1);
        if (m) m->vit = (vit_block_t*)calloc(cfg->vit_layers, sizeof(vit_block_t));
        for (uint32_t l = 0; l < cfg->vit_layers; ++l) {
            vit_block_t b;
            b.ln1 = take_norm(&c, LWM_NORM_LAYER, vh);
            b.q = take_lin(&c, vh, vh, cfg->qkv_bias);
            b.k = take_lin(&c, vh, vh, cfg->qkv_bias);
            b.v = take_lin(&c, vh, vh, cfg->qkv_bias);
            b.o = take_lin(&c, vh, vh, 1);
            b.ln2 = take_norm(&c, LWM_NORM_LAYER, vh);
            b.fc1 = take_lin(&c, cfg->vit_mlp, vh, 1);
            b.fc2 = take_lin(&c, vh, cfg->vit_mlp, 1);
            if (m) m->vit[l] = b;
        }
        norm_t vn = take_norm(&c, LWM_NORM_LAYER, vh);
        mlp_t proj = take_mlp(&c, vh, cfg->projector_hidden, D, cfg->projector_norm);
        if (m) {
            m->cls = cls;
            m->vpos = vpos;
            m->patch = patch;
            m->vit_norm = vn;
            m->projector = proj;
        }
    }
    return c.off;
}

size_t orc_lewm_weight_count(const lwm_lewm_config* cfg) { return walk(cfg, NULL, NULL); }

orc_lewm* orc_lewm_new(const lwm_lewm_config* cfg, const float* weights, size_t count) {
    if (count != orc_lewm_weight_count(cfg)) return NULL;
    orc_lewm* m = (orc_lewm*)calloc(1, sizeof(orc_lewm));
    m->c = *cfg;
    m->blob = (float*)malloc(count * sizeof(float));
    memcpy(m->blob, weights, count * sizeof(float));
    walk(cfg, m->blob, m);
    return m;
}

void orc_lewm_free(orc_lewm* m) {
    if (!m) return;
    free(m->blocks);
    free(m->enc_lin);
    free(m->enc_norm);
    free(m->vit);
    free(m->blob);
    free(m);
}

/* ---------------------------------------------------------------- ops */

/* y[n, out] = x[n, in] W^T + b (candle Linear), sums in k order. */
static void linear(const float* x, uint32_t n, uint32_t in, uint32_t out, lin_t l, float* y) {
#pragma omp parallel for schedule(static) if ((size_t)n * out * in > 200000)
    for (long r = 0; r < (long)n; ++r) {
        const float* xr = x + (size_t)r * in;
        for (uint32_t o = 0; o < out; ++o) {
            const float* w = l.w + (size_t)o * in;
            float acc = 0.0f;
            for (uint32_t k = 0; k < in; ++k) acc += xr[k] * w[k];
            y[(size_t)r * out + o] = l.b ? acc + l.b[o] : acc;
        }
    }
}

static float gelu_tanh(float v) {
    const float k = 0.7978845608028654f;
    return (0.5f * v) * (1.0f + tanhf((k * v) * (1.0f + (0.044715f * v) * v)));
}
static float gelu_erf(float v) { return (0.5f * v) * (1.0f + erff(v * 0.7071067811865476f)); }
static float silu(float v) { return v / (1.0f + expf(-v)); }

/* LayerNorm over the last dim (biased variance), optionally affine. */
static void layer_norm_row(const float* x, uint32_t d, const float* w, const float* b, float eps, float* y) {
    float s = 0.0f;
    for (uint32_t i = 0; i < d; ++i) s += x[i];
    const float mean = s / (float)d;
    float v = 0.0f;
    for (uint32_t i = 0; i < d; ++i) {
        const float c = x[i] - mean;
        v += c * c;
    }
    const float den = sqrtf(v / (float)d + eps);
    for (uint32_t i = 0; i < d; ++i) {
        const float c = (x[i] - mean) / den;
        y[i] = w ? c * w[i] + b[i] : c;
    }
}

static void apply_norm(norm_t n, float* x, uint32_t rows, uint32_t d) {
    if (n.kind == LWM_NORM_NONE) return;
    for (uint32_t r = 0; r < rows; ++r) {
        float* xr = x + (size_t)r * d;
        if (n.kind == LWM_NORM_LAYER) {
            layer_norm_row(xr, d, n.w, n.b, 1e-5f, xr);
        } else {
            for (uint32_t i = 0; i < d; ++i) xr[i] = (xr[i] - n.rm[i]) / sqrtf(n.rv[i] + 1e-5f) * n.w[i] + n.b[i];
        }
    }
}

/* Mlp::forward (modules.rs:108-115): fc1 -> norm -> gelu -> fc2. */
static void mlp_forward(const mlp_t* m, const float* x, uint32_t n, float* y) {
    float* h = (float*)malloc(sizeof(float) * (size_t)n * m->hid);
    linear(x, n, m->in, m->hid, m->fc1, h);
    apply_norm(m->norm, h, n, m->hid);
    for (size_t i = 0; i < (size_t)n * m->hid; ++i) h[i] = gelu_tanh(h[i]);
    linear(h, n, m->hid, m->out, m->fc2, y);
    free(h);
}

/* Softmax attention of one sequence of t tokens: qkv [t, 3*H*dh] laid out
 * (3, H, dh) per token; out [t, H*dh].  causal adds -inf above the diagonal. */
static void attention(const float* qkv, uint32_t t, uint32_t H, uint32_t dh, float scale, int causal,
                      int scale_q_first, float* out) {
    const uint32_t inner = H * dh;
    float* p = (float*)malloc(sizeof(float) * t);
    for (uint32_t h = 0; h < H; ++h)
        for (uint32_t i = 0; i < t; ++i) {
            const float* q = qkv + (size_t)i * 3 * inner + h * dh;
            float mx = -INFINITY;
            for (uint32_t j = 0; j < t; ++j) {
                float s;
                if (causal && j > i) {
                    s = -INFINITY;
                } else {
                    const float* k = qkv + (size_t)j * 3 * inner + inner + h * dh;
                    float acc = 0.0f;
                    if (scale_q_first)
                        for (uint32_t d = 0; d < dh; ++d) acc += (q[d] * scale) * k[d];
                    else
                        for (uint32_t d = 0; d < dh; ++d) acc += q[d] * k[d];
                    s = scale_q_first ? acc : acc * scale;
                }
                p[j] = s;
                if (s > mx) mx = s;
            }
            float sum = 0.0f;
            for (uint32_t j = 0; j < t; ++j) {
                p[j] = expf(p[j] - mx);
                sum += p[j];
            }
            float* o = out + (size_t)i * inner + h * dh;
            for (uint32_t d = 0; d < dh; ++d) o[d] = 0.0f;
            for (uint32_t j = 0; j < t; ++j) {
                const float w = p[j] / sum;
                const float* v = qkv + (size_t)j * 3 * inner + 2 * inner + h * dh;
                for (uint32_t d = 0; d < dh; ++d) o[d] += w * v[d];
            }
        }
    free(p);
}

/* ActionEmbedder::forward (modules.rs:150-158) for n tokens [n, A]. */
void orc_lewm_action_embed(const orc_lewm* m, const float* act, uint32_t n, float* out) {
    const lwm_lewm_config* c = &m->c;
    const uint32_t sm = c->smoothed_dim, hid = c->action_mlp_scale * c->embed_dim;
    float* s = (float*)malloc(sizeof(float) * (size_t)n * sm);
    float* h = (float*)malloc(sizeof(float) * (size_t)n * hid);
    linear(act, n, c->action_dim, sm, m->act_conv, s); /* kernel-1 conv = per-token linear */
    linear(s, n, sm, hid, m->act_fc1, h);
    for (size_t i = 0; i < (size_t)n * hid; ++i) h[i] = silu(h[i]);
    linear(h, n, hid, c->embed_dim, m->act_fc2, out);
    free(h);
    free(s);
}

/* Predictor::forward_last + pred_proj (model.rs:74-86) for `seqs` sequences
 * of t tokens: frames [seqs, t, D], act_emb [seqs, t, D] -> out [seqs, D]. */
void orc_lewm_predict_last(const orc_lewm* m, const float* frames, const float* act_emb, uint32_t seqs, uint32_t t,
                           float* out) {
    const lwm_lewm_config* c = &m->c;
    const uint32_t D = c->embed_dim, hid = c->pred_hidden_dim, inner = c->heads * c->dim_head;
    const size_t rows = (size_t)seqs * t;
    float* x = (float*)malloc(sizeof(float) * rows * hid);
    float* cond = (float*)malloc(sizeof(float) * rows * hid);
    float* tmp = (float*)malloc(sizeof(float) * rows * (D > hid ? D : hid));
    for (size_t r = 0; r < rows; ++r)
        for (uint32_t i = 0; i < D; ++i) tmp[r * D + i] = frames[r * D + i] + m->pos[(r % t) * D + i];
    if (m->has_in_proj) {
        linear(tmp, (uint32_t)rows, D, hid, m->input_proj, x);
        linear(act_emb, (uint32_t)rows, D, hid, m->cond_proj, cond);
    } else {
        memcpy(x, tmp, sizeof(float) * rows * D);
        memcpy(cond, act_emb, sizeof(float) * rows * D);
    }
    float* sc = (float*)malloc(sizeof(float) * rows * hid);
    float* ada = (float*)malloc(sizeof(float) * rows * 6 * hid);
    float* y = (float*)malloc(sizeof(float) * rows * hid);
    float* qkv = (float*)malloc(sizeof(float) * rows * 3 * inner);
    float* att = (float*)malloc(sizeof(float) * rows * inner);
    float* o = (float*)malloc(sizeof(float) * rows * hid);
    float* f1 = (float*)malloc(sizeof(float) * rows * c->mlp_dim);
    for (size_t i = 0; i < rows * hid; ++i) sc[i] = silu(cond[i]);
    const float scale = (float)pow((double)c->dim_head, -0.5);
    for (uint32_t l = 0; l < c->depth; ++l) {
        const block_t* b = &m->blocks[l];
        linear(sc, (uint32_t)rows, hid, 6 * hid, b->ada, ada); /* chunks: shift/scale/gate msa, mlp */
        for (size_t r = 0; r < rows; ++r) {
            const float* a = ada + r * 6 * hid;
            float* yr = y + r * hid;
            layer_norm_row(x + r * hid, hid, NULL, NULL, 1e-6f, yr);
            for (uint32_t i = 0; i < hid; ++i) yr[i] = yr[i] * (a[hid + i] + 1.0f) + a[i];
            layer_norm_row(yr, hid, b->attn_norm.w, b->attn_norm.b, 1e-5f, yr);
        }
        lin_t qkvl = {b->qkv_w, NULL};
        linear(y, (uint32_t)rows, hid, 3 * inner, qkvl, qkv);
        for (uint32_t s = 0; s < seqs; ++s)
            attention(qkv + (size_t)s * t * 3 * inner, t, c->heads, c->dim_head, scale, 1, 1,
                      att + (size_t)s * t * inner);
        linear(att, (uint32_t)rows, inner, hid, b->to_out, o);
        for (size_t r = 0; r < rows; ++r) {
            const float* a = ada + r * 6 * hid;
            for (uint32_t i = 0; i < hid; ++i) x[r * hid + i] = x[r * hid + i] + a[2 * hid + i] * o[r * hid + i];
        }
        for (size_t r = 0; r < rows; ++r) {
            const float* a = ada + r * 6 * hid;
            float* yr = y + r * hid;
            layer_norm_row(x + r * hid, hid, NULL, NULL, 1e-6f, yr);
            for (uint32_t i = 0; i < hid; ++i) yr[i] = yr[i] * (a[4 * hid + i] + 1.0f) + a[3 * hid + i];
            layer_norm_row(yr, hid, b->mlp_norm.w, b->mlp_norm.b, 1e-5f, yr);
        }
        linear(y, (uint32_t)rows, hid, c->mlp_dim, b->fc1, f1);
        for (size_t i = 0; i < rows * c->mlp_dim; ++i) f1[i] = gelu_tanh(f1[i]);
        linear(f1, (uint32_t)rows, c->mlp_dim, hid, b->fc2, o);
        for (size_t r = 0; r < rows; ++r) {
            const float* a = ada + r * 6 * hid;
            for (uint32_t i = 0; i < hid; ++i) x[r * hid + i] = x[r * hid + i] + a[5 * hid + i] * o[r * hid + i];
        }
    }
    /* last token -> norm -> output_proj -> pred_proj */
    float* last = (float*)malloc(sizeof(float) * seqs * hid);
    for (uint32_t s = 0; s < seqs; ++s)
        layer_norm_row(x + ((size_t)s * t + t - 1) * hid, hid, m->final_norm.w, m->final_norm.b, 1e-5f,
                       last + (size_t)s * hid);
    float* proj_in = last;
    float* po = NULL;
    if (m->has_out_proj) {
        po = (float*)malloc(sizeof(float) * seqs * D);
        linear(last, seqs, hid, D, m->output_proj, po);
        proj_in = po;
    }
    mlp_forward(&m->pred_proj, proj_in, seqs, out);
    free(po);
    free(last);
    free(f1);
    free(o);
    free(att);
    free(qkv);
    free(y);
    free(ada);
    free(sc);
    free(tmp);
    free(cond);
    free(x);
}

/* LeWmSession::score_candidates (src/session.rs:46-66): history embeddings
 * emb [B, h, D] shared by every sample, candidates [B,S,T,A], window
 * `history` (rollout_embeddings_with_history, model.rs:94-147), goal_cost
 * against goal [B, D] (model.rs:149-165). */
void orc_lewm_scores(const orc_lewm* m, const float* emb, uint32_t h, const float* goal, const float* cand,
                     uint32_t B, uint32_t S, uint32_t T, uint32_t history, float* scores, float* last_out) {
    const lwm_lewm_config* c = &m->c;
    const uint32_t D = c->embed_dim, A = c->action_dim;
    const size_t bs = (size_t)B * S;
    float* act = (float*)malloc(sizeof(float) * bs * T * D);
    orc_lewm_action_embed(m, cand, (uint32_t)(bs * T), act);
    const uint32_t nframes = T + 1;
    float* frames = (float*)malloc(sizeof(float) * bs * nframes * D);
    for (size_t r = 0; r < bs; ++r)
        for (uint32_t j = 0; j < h; ++j) memcpy(frames + (r * nframes + j) * D, emb + ((r / S) * h + j) * D, D * 4);
    float* win = (float*)malloc(sizeof(float) * bs * history * D);
    float* wact = (float*)malloc(sizeof(float) * bs * history * D);
    float* pred = (float*)malloc(sizeof(float) * bs * D);
    uint32_t count = h;
    for (uint32_t step = 0; step + h <= T; ++step) {
        const uint32_t upper = h + step;
        const uint32_t lo = upper > history ? upper - history : 0;
        const uint32_t w = upper - lo;
        for (size_t r = 0; r < bs; ++r) {
            memcpy(win + r * w * D, frames + (r * nframes + lo) * D, (size_t)w * D * 4);
            memcpy(wact + r * w * D, act + (r * T + lo) * D, (size_t)w * D * 4);
        }
        orc_lewm_predict_last(m, win, wact, (uint32_t)bs, w, pred);
        for (size_t r = 0; r < bs; ++r) memcpy(frames + (r * nframes + count) * D, pred + r * D, D * 4);
        ++count;
    }
    for (size_t r = 0; r < bs; ++r) {
        const float* p = frames + (r * nframes + count - 1) * D;
        const float* g = goal + (r / S) * D;
        float acc = 0.0f;
        for (uint32_t i = 0; i < D; ++i) {
            const float d = p[i] - g[i];
            acc += d * d;
        }
        scores[r] = acc;
        if (last_out) memcpy(last_out + r * D, p, D * 4);
    }
    (void)A;
    free(pred);
    free(wact);
    free(win);
    free(frames);
    free(act);
}

/* VectorMlpEncoder::forward (world_model/model.rs:256-273): [n, obs] -> [n, D]. */
void orc_lewm_encode_vector(const orc_lewm* m, const float* obs, uint32_t n, float* out) {
    const lwm_lewm_config* c = &m->c;
    const uint32_t oh = c->obs_hidden_dim;
    float* a = (float*)malloc(sizeof(float) * (size_t)n * oh);
    float* b = (float*)malloc(sizeof(float) * (size_t)n * oh);
    linear(obs, n, c->obs_dim, oh, m->enc_lin[0], a);
    for (uint32_t j = 0; j + 1 < c->obs_depth; ++j) {
        apply_norm(m->enc_norm[j], a, n, oh);
        for (size_t i = 0; i < (size_t)n * oh; ++i) a[i] = gelu_tanh(a[i]);
        if (j + 2 < c->obs_depth) {
            linear(a, n, oh, oh, m->enc_lin[j + 1], b);
            float* t = a;
            a = b;
            b = t;
        }
    }
    linear(a, n, oh, c->embed_dim, m->enc_lin[c->obs_depth - 1], out);
    free(a);
    free(b);
}

/* HfVitEncoder::cls + projector (LeWm::encode_pixels, model.rs:41-55):
 * pixels [n, C, H, W] (normalised) -> [n, D]. */
void orc_lewm_encode_pixels(const orc_lewm* m, const float* pix, uint32_t n, float* out) {
    const lwm_lewm_config* c = &m->c;
    const uint32_t vh = c->vit_hidden, p = c->patch_size, side = c->image_size / p, np = side * side;
    const uint32_t t = np + 1, C = c->channels, img = c->image_size, kdim = C * p * p;
    const uint32_t H = c->vit_heads, dh = vh / H;
    float* cls_all = (float*)malloc(sizeof(float) * (size_t)n * vh);
    float* patches = (float*)malloc(sizeof(float) * (size_t)np * kdim);
    float* x = (float*)malloc(sizeof(float) * (size_t)t * vh);
    float* y = (float*)malloc(sizeof(float) * (size_t)t * vh);
    float* qkv = (float*)malloc(sizeof(float) * (size_t)t * 3 * vh);
    float* tq = (float*)malloc(sizeof(float) * (size_t)t * vh);
    float* att = (float*)malloc(sizeof(float) * (size_t)t * vh);
    float* f1 = (float*)malloc(sizeof(float) * (size_t)t * c->vit_mlp);
    const float scale = 1.0f / sqrtf((float)dh);
    for (uint32_t im = 0; im < n; ++im) {
        const float* px = pix + (size_t)im * C * img * img;
        for (uint32_t py = 0; py < side; ++py)
            for (uint32_t pxi = 0; pxi < side; ++pxi) {
                float* row = patches + ((size_t)py * side + pxi) * kdim;
                for (uint32_t ch = 0; ch < C; ++ch)
                    for (uint32_t ky = 0; ky < p; ++ky)
                        for (uint32_t kx = 0; kx < p; ++kx)
                            row[(ch * p + ky) * p + kx] = px[((size_t)ch * img + py * p + ky) * img + pxi * p + kx];
            }
        linear(patches, np, kdim, vh, m->patch, x + vh);
        memcpy(x, m->cls, vh * 4);
        for (size_t i = 0; i < (size_t)t * vh; ++i) x[i] += m->vpos[i];
        for (uint32_t l = 0; l < c->vit_layers; ++l) {
            const vit_block_t* b = &m->vit[l];
            for (uint32_t r = 0; r < t; ++r) layer_norm_row(x + r * vh, vh, b->ln1.w, b->ln1.b, c->vit_eps, y + r * vh);
            linear(y, t, vh, vh, b->q, tq);
            for (uint32_t r = 0; r < t; ++r) memcpy(qkv + (size_t)r * 3 * vh, tq + r * vh, vh * 4);
            linear(y, t, vh, vh, b->k, tq);
            for (uint32_t r = 0; r < t; ++r) memcpy(qkv + (size_t)r * 3 * vh + vh, tq + r * vh, vh * 4);
            linear(y, t, vh, vh, b->v, tq);
            for (uint32_t r = 0; r < t; ++r) memcpy(qkv + (size_t)r * 3 * vh + 2 * vh, tq + r * vh, vh * 4);
            attention(qkv, t, H, dh, scale, 0, 0, att);
            linear(att, t, vh, vh, b->o, y);
            for (size_t i = 0; i < (size_t)t * vh; ++i) x[i] = y[i] + x[i];
            for (uint32_t r = 0; r < t; ++r) layer_norm_row(x + r * vh, vh, b->ln2.w, b->ln2.b, c->vit_eps, y + r * vh);
            linear(y, t, vh, c->vit_mlp, b->fc1, f1);
            for (size_t i = 0; i < (size_t)t * c->vit_mlp; ++i) f1[i] = gelu_erf(f1[i]);
            linear(f1, t, c->vit_mlp, vh, b->fc2, y);
            for (size_t i = 0; i < (size_t)t * vh; ++i) x[i] = y[i] + x[i];
        }
        layer_norm_row(x, vh, m->vit_norm.w, m->vit_norm.b, c->vit_eps, cls_all + (size_t)im * vh);
    }
    mlp_forward(&m->projector, cls_all, n, out);
    free(f1);
    free(att);
    free(tq);
    free(qkv);
    free(y);
    free(x);
    free(patches);
    free(cls_all);
}

void orc_lewm_score_fn(void* user, const float* cand, uint32_t B, uint32_t S, uint32_t T, uint32_t A,
                       float* scores) {
    (void)A;
    const orc_lewm_ctx* c = (const orc_lewm_ctx*)user;
    orc_lewm_scores(c->model, c->emb, c->h, c->goal, cand, B, S, T, c->history, scores, NULL);
}
