/* CPU restatement of the reference's fp32 Qwen3.5 forward pass -- TEST INFRASTRUCTURE.
 * See qwen_oracle.h for what this file is for and how it is pinned. Every function
 * names the reference lines (paths inside the reference project) whose arithmetic it
 * restates. Plain C11 + OpenMP over GEMV rows; no product code links this file. */
#include "qwen_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define MAXT 4096

static float bf16f(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* include/forward_pass.h:21-24 */
static float o_silu(float x) { return x / (1.0f + expf(-x)); }
static float o_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }
static float o_softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

/* src/forward_pass.cpp:44-75: y[o] = sum_i bf16(W[o,i]) * x[i], fp32 accumulation in
 * 8 interleaved lanes (the reference uses 4 x 8-lane AVX2 accumulators). */
void orc_matmul_bf16(const uint16_t* W, const float* x, float* y, int out_dim, int in_dim) {
    #pragma omp parallel for schedule(static)
    for (int o = 0; o < out_dim; ++o) {
        const uint16_t* w = W + (size_t)o * in_dim;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        int i = 0;
        for (; i + 8 <= in_dim; i += 8)
            for (int l = 0; l < 8; ++l) acc[l] += bf16f(w[i + l]) * x[i + l];
        float r = ((acc[0] + acc[4]) + (acc[1] + acc[5])) + ((acc[2] + acc[6]) + (acc[3] + acc[7]));
        for (; i < in_dim; ++i) r += bf16f(w[i]) * x[i];
        y[o] = r;
    }
}

/* src/forward_pass.cpp:77-84: y = x * rsqrt(mean(x^2) + eps) * (1 + w), sum in double */
void orc_rmsnorm(const float* x, const float* w, float* y, int n, float eps) {
    double s = 0.0;
    for (int i = 0; i < n; ++i) s += (double)x[i] * x[i];
    float inv = 1.0f / sqrtf((float)(s / n) + eps);
    for (int i = 0; i < n; ++i) y[i] = x[i] * inv * (1.0f + w[i]);
}

/* src/forward_pass.cpp:86-93: y = w * (x * rsqrt(mean(x^2) + eps)) * silu(g) */
void orc_rmsnorm_gated(const float* x, const float* w, const float* g, float* y, int n, float eps) {
    double s = 0.0;
    for (int i = 0; i < n; ++i) s += (double)x[i] * x[i];
    float inv = 1.0f / sqrtf((float)(s / n) + eps);
    for (int i = 0; i < n; ++i) y[i] = w[i] * (x[i] * inv) * o_silu(g[i]);
}

/* src/forward_pass.cpp:95-100: x /= sqrt(sum(x^2) + eps) */
void orc_l2norm(float* x, int n, float eps) {
    double s = 0.0;
    for (int i = 0; i < n; ++i) s += (double)x[i] * x[i];
    float inv = 1.0f / sqrtf((float)s + eps);
    for (int i = 0; i < n; ++i) x[i] *= inv;
}

/* src/forward_pass.cpp:102-112: rotate_half on the first rot dims, pairs (i, i+rot/2),
 * inv_freq = theta^(-2i/rot), angle and cos/sin in double, rounded to float. */
void orc_apply_rope(float* v, int rot, int pos, double theta) {
    int half = rot / 2;
    for (int i = 0; i < half; ++i) {
        double inv_freq = pow(theta, -(double)(2 * i) / rot);
        double ang = (double)pos * inv_freq;
        float c = (float)cos(ang), s = (float)sin(ang);
        float x1 = v[i], x2 = v[i + half];
        v[i] = x1 * c - x2 * s;
        v[i + half] = x2 * c + x1 * s;
    }
}

/* ------------------------------------------------------------------------- */
typedef struct { const void* p; int dtype; int64_t n; } orc_raw;

typedef struct {
    int is_attn, idx;
    float *in_ln, *post_ln;
    const uint16_t *gate, *up, *down;
    const uint16_t *q, *k, *v, *o;
    float *q_norm, *k_norm;
    const uint16_t *in_qkv, *in_z, *in_b, *in_a, *out;
    float *conv, *dt_bias, *A_log, *gdn_norm;
} orc_layer;

typedef struct { char* name; orc_raw t; } orc_entry;

struct orc_model {
    orc_config c;
    int max_ctx, pos;
    orc_entry* ents;
    int n_ents, cap_ents;
    float** owned;
    int n_owned;
    orc_layer* lw;
    const uint16_t *embed, *head;
    float* final_norm;
    float **kc, **vc, **S, **cs; /* per attention layer / per GDN layer state */
    int n_attn, n_gdn;
    float *hidden, *normed, *mix, *ff, *scratch;
    size_t scratch_n;
};

orc_model* orc_create(const orc_config* cfg, int max_context) {
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    m->c = *cfg;
    m->max_ctx = max_context;
    return m;
}

static void* xalloc(orc_model* m, size_t nfloat) {
    float* p = (float*)calloc(nfloat ? nfloat : 1, sizeof(float));
    m->owned = (float**)realloc(m->owned, sizeof(float*) * (m->n_owned + 1));
    m->owned[m->n_owned++] = p;
    return p;
}

void orc_destroy(orc_model* m) {
    if (!m) return;
    for (int i = 0; i < m->n_owned; ++i) free(m->owned[i]);
    for (int i = 0; i < m->n_ents; ++i) free(m->ents[i].name);
    free(m->owned); free(m->ents); free(m->lw);
    free(m->kc); free(m->vc); free(m->S); free(m->cs);
    free(m);
}

int orc_set_tensor(orc_model* m, const char* name, int dtype, const void* data, int64_t numel) {
    if (m->n_ents == m->cap_ents) {
        m->cap_ents = m->cap_ents ? 2 * m->cap_ents : 256;
        m->ents = (orc_entry*)realloc(m->ents, sizeof(orc_entry) * m->cap_ents);
    }
    m->ents[m->n_ents].name = strdup(name);
    m->ents[m->n_ents].t.p = data;
    m->ents[m->n_ents].t.dtype = dtype;
    m->ents[m->n_ents].t.n = numel;
    m->n_ents++;
    return 0;
}

static const orc_raw* find(orc_model* m, const char* name) {
    for (int i = 0; i < m->n_ents; ++i)
        if (!strcmp(m->ents[i].name, name)) return &m->ents[i].t;
    return NULL;
}

static char g_missing[512];

/* get_f32 (src/safetensors_loader.cpp:252-278): widen a small tensor to fp32 once */
static float* get_f32(orc_model* m, const char* name, int* ok) {
    const orc_raw* r = find(m, name);
    if (!r) { if (*ok) snprintf(g_missing, sizeof g_missing, "%s", name); *ok = 0; return NULL; }
    float* f = (float*)xalloc(m, (size_t)r->n);
    if (r->dtype == 0) memcpy(f, r->p, (size_t)r->n * 4);
    else for (int64_t i = 0; i < r->n; ++i) f[i] = bf16f(((const uint16_t*)r->p)[i]);
    return f;
}

/* view (src/safetensors_loader.cpp:241-250): matrices stay bf16 in place */
static const uint16_t* get_bf16(orc_model* m, const char* name, int* ok) {
    const orc_raw* r = find(m, name);
    if (!r || r->dtype != 1) { if (*ok) snprintf(g_missing, sizeof g_missing, "%s", name); *ok = 0; return NULL; }
    return (const uint16_t*)r->p;
}

/* QwenModel::QwenModel (src/qwen_model.cpp:12-96): resolve weights, allocate state */
int orc_finalize(orc_model* m, char* missing, int missing_len) {
    const orc_config* c = &m->c;
    int ok = 1;
    char nm[256];
    const char* LM = "model.language_model.";
    m->lw = (orc_layer*)calloc(c->layers, sizeof(orc_layer));
    m->kc = (float**)calloc(c->layers, sizeof(float*));
    m->vc = (float**)calloc(c->layers, sizeof(float*));
    m->S = (float**)calloc(c->layers, sizeof(float*));
    m->cs = (float**)calloc(c->layers, sizeof(float*));
    int KD = c->k_heads * c->k_dim, VD = c->v_heads * c->v_dim, CONV = 2 * KD + VD;
#define NM(fmt, ...) (snprintf(nm, sizeof nm, fmt, __VA_ARGS__), nm)
    for (int L = 0; L < c->layers; ++L) {
        orc_layer* lw = &m->lw[L];
        lw->in_ln = get_f32(m, NM("%slayers.%d.input_layernorm.weight", LM, L), &ok);
        lw->post_ln = get_f32(m, NM("%slayers.%d.post_attention_layernorm.weight", LM, L), &ok);
        lw->gate = get_bf16(m, NM("%slayers.%d.mlp.gate_proj.weight", LM, L), &ok);
        lw->up = get_bf16(m, NM("%slayers.%d.mlp.up_proj.weight", LM, L), &ok);
        lw->down = get_bf16(m, NM("%slayers.%d.mlp.down_proj.weight", LM, L), &ok);
        if ((L + 1) % c->interval == 0) {
            lw->is_attn = 1; lw->idx = m->n_attn++;
            lw->q = get_bf16(m, NM("%slayers.%d.self_attn.q_proj.weight", LM, L), &ok);
            lw->k = get_bf16(m, NM("%slayers.%d.self_attn.k_proj.weight", LM, L), &ok);
            lw->v = get_bf16(m, NM("%slayers.%d.self_attn.v_proj.weight", LM, L), &ok);
            lw->o = get_bf16(m, NM("%slayers.%d.self_attn.o_proj.weight", LM, L), &ok);
            lw->q_norm = get_f32(m, NM("%slayers.%d.self_attn.q_norm.weight", LM, L), &ok);
            lw->k_norm = get_f32(m, NM("%slayers.%d.self_attn.k_norm.weight", LM, L), &ok);
            m->kc[lw->idx] = (float*)xalloc(m, (size_t)m->max_ctx * c->kv_heads * c->head_dim);
            m->vc[lw->idx] = (float*)xalloc(m, (size_t)m->max_ctx * c->kv_heads * c->head_dim);
        } else {
            lw->is_attn = 0; lw->idx = m->n_gdn++;
            lw->in_qkv = get_bf16(m, NM("%slayers.%d.linear_attn.in_proj_qkv.weight", LM, L), &ok);
            lw->in_z = get_bf16(m, NM("%slayers.%d.linear_attn.in_proj_z.weight", LM, L), &ok);
            lw->in_b = get_bf16(m, NM("%slayers.%d.linear_attn.in_proj_b.weight", LM, L), &ok);
            lw->in_a = get_bf16(m, NM("%slayers.%d.linear_attn.in_proj_a.weight", LM, L), &ok);
            lw->out = get_bf16(m, NM("%slayers.%d.linear_attn.out_proj.weight", LM, L), &ok);
            lw->conv = get_f32(m, NM("%slayers.%d.linear_attn.conv1d.weight", LM, L), &ok);
            lw->dt_bias = get_f32(m, NM("%slayers.%d.linear_attn.dt_bias", LM, L), &ok);
            lw->A_log = get_f32(m, NM("%slayers.%d.linear_attn.A_log", LM, L), &ok);
            lw->gdn_norm = get_f32(m, NM("%slayers.%d.linear_attn.norm.weight", LM, L), &ok);
            m->S[lw->idx] = (float*)xalloc(m, (size_t)c->v_heads * c->k_dim * c->v_dim);
            m->cs[lw->idx] = (float*)xalloc(m, (size_t)CONV * (c->conv_k - 1));
        }
    }
    m->embed = get_bf16(m, NM("%sembed_tokens.weight", LM, 0), &ok);
    m->final_norm = get_f32(m, NM("%snorm.weight", LM, 0), &ok);
    /* lm_head if present, else tied embedding (src/qwen_model.cpp:67-69) */
    int ok2 = 1;
    m->head = get_bf16(m, "lm_head.weight", &ok2);
    if (!ok2) { ok2 = 1; m->head = get_bf16(m, NM("%slm_head.weight", LM, 0), &ok2); }
    if (!ok2) m->head = m->embed;
#undef NM
    m->hidden = (float*)xalloc(m, c->hidden);
    m->normed = (float*)xalloc(m, c->hidden);
    m->mix = (float*)xalloc(m, c->hidden);
    m->ff = (float*)xalloc(m, c->hidden);
    size_t attn_ws = (size_t)c->q_heads * c->head_dim * 5 + (size_t)c->kv_heads * c->head_dim + m->max_ctx;
    size_t gdn_ws = (size_t)CONV * 2 + (size_t)VD * 4 + 2 * c->v_heads + 2 * KD + 2 * c->v_dim;
    size_t ffn_ws = (size_t)c->ffn * 3;
    m->scratch_n = attn_ws > gdn_ws ? attn_ws : gdn_ws;
    if (ffn_ws > m->scratch_n) m->scratch_n = ffn_ws;
    m->scratch = (float*)xalloc(m, m->scratch_n + 64);
    if (!ok && missing) snprintf(missing, missing_len, "%s", g_missing);
    return ok ? 0 : -1;
}

/* QwenModel::reset (src/qwen_model.cpp:98-104) */
void orc_reset(orc_model* m) {
    const orc_config* c = &m->c;
    int KD = c->k_heads * c->k_dim, VD = c->v_heads * c->v_dim, CONV = 2 * KD + VD;
    m->pos = 0;
    for (int i = 0; i < m->n_attn; ++i) {
        memset(m->kc[i], 0, sizeof(float) * (size_t)m->max_ctx * c->kv_heads * c->head_dim);
        memset(m->vc[i], 0, sizeof(float) * (size_t)m->max_ctx * c->kv_heads * c->head_dim);
    }
    for (int i = 0; i < m->n_gdn; ++i) {
        memset(m->S[i], 0, sizeof(float) * (size_t)c->v_heads * c->k_dim * c->v_dim);
        memset(m->cs[i], 0, sizeof(float) * (size_t)CONV * (c->conv_k - 1));
    }
}

int orc_position(const orc_model* m) { return m->pos; }

/* The attention of one query row over cached positions 0..n_ctx-1
 * (src/qwen_model.cpp:134-150, src/qwen_forward.cpp:58-79). */
void orc_attention(int NQ, int NKV, int HD, int n_ctx, const float* q_all, const float* gate,
                   const float* kc, const float* vc, float* out) {
    int GRP = NQ / NKV;
    float sc = 1.0f / sqrtf((float)HD);
    float* sco = (float*)malloc(sizeof(float) * (n_ctx > 0 ? n_ctx : 1));
    for (int h = 0; h < NQ; ++h) {
        int kh = h / GRP;
        const float* q = q_all + (size_t)h * HD;
        float mx = -1e30f;
        for (int j = 0; j < n_ctx; ++j) {
            const float* k = kc + ((size_t)j * NKV + kh) * HD;
            float s = 0;
            for (int d = 0; d < HD; ++d) s += q[d] * k[d];
            s *= sc;
            sco[j] = s;
            if (s > mx) mx = s;
        }
        float sm = 0;
        for (int j = 0; j < n_ctx; ++j) { sco[j] = expf(sco[j] - mx); sm += sco[j]; }
        float* oh = out + (size_t)h * HD;
        for (int d = 0; d < HD; ++d) oh[d] = 0;
        for (int j = 0; j < n_ctx; ++j) {
            float p = sco[j] / sm;
            const float* v = vc + ((size_t)j * NKV + kh) * HD;
            for (int d = 0; d < HD; ++d) oh[d] += p * v[d];
        }
    }
    for (int i = 0; i < NQ * HD; ++i) out[i] *= o_sigmoid(gate[i]);
    free(sco);
}

/* QwenModel::attn_step (src/qwen_model.cpp:106-152) */
static void attn_step(orc_model* m, const orc_layer* lw, const float* in, float* out) {
    const orc_config* c = &m->c;
    int H = c->hidden, HD = c->head_dim, NQ = c->q_heads, NKV = c->kv_heads;
    float* qkv = m->scratch;
    float* Q = qkv + (size_t)NQ * HD * 2;
    float* gate = Q + (size_t)NQ * HD;
    float* kv = gate + (size_t)NQ * HD;
    float* ac = kv + (size_t)NKV * HD;
    orc_matmul_bf16(lw->q, in, qkv, NQ * HD * 2, H);
    for (int h = 0; h < NQ; ++h) {
        const float* qg = qkv + (size_t)h * HD * 2; /* per head [q | gate] */
        orc_rmsnorm(qg, lw->q_norm, Q + (size_t)h * HD, HD, c->eps);
        orc_apply_rope(Q + (size_t)h * HD, c->rot_dim, m->pos, c->theta);
        memcpy(gate + (size_t)h * HD, qg + HD, sizeof(float) * HD);
    }
    float* kslot = m->kc[lw->idx] + (size_t)m->pos * NKV * HD;
    float* vslot = m->vc[lw->idx] + (size_t)m->pos * NKV * HD;
    orc_matmul_bf16(lw->k, in, kv, NKV * HD, H);
    for (int kh = 0; kh < NKV; ++kh) {
        orc_rmsnorm(kv + (size_t)kh * HD, lw->k_norm, kslot + (size_t)kh * HD, HD, c->eps);
        orc_apply_rope(kslot + (size_t)kh * HD, c->rot_dim, m->pos, c->theta);
    }
    orc_matmul_bf16(lw->v, in, vslot, NKV * HD, H);
    orc_attention(NQ, NKV, HD, m->pos + 1, Q, gate, m->kc[lw->idx], m->vc[lw->idx], ac);
    orc_matmul_bf16(lw->o, ac, out, H, NQ * HD);
}

/* The GDN mixer between projections and gated norm, for T tokens in order
 * (src/qwen_model.cpp:173-207; per token identical to qwen_forward.cpp:109-142). */
void orc_gdn_core(int T, int KH, int VH, int DK, int DV, int K,
                  const float* mixed, const float* conv_w, const float* a, const float* b,
                  const float* A_log, const float* dt_bias, float* state, float* conv_state,
                  float* out) {
    int KD = KH * DK, VD = VH * DV, C = 2 * KD + VD, rep = VH / KH;
    float qs = 1.0f / sqrtf((float)DK);
    float* conv = (float*)malloc(sizeof(float) * C);
    float* Q = (float*)malloc(sizeof(float) * KD);
    float* Kx = (float*)malloc(sizeof(float) * KD);
    float* km = (float*)malloc(sizeof(float) * DV);
    float* dl = (float*)malloc(sizeof(float) * DV);
    for (int t = 0; t < T; ++t) {
        const float* x = mixed + (size_t)t * C;
        /* causal depthwise conv over the rolling state, then SiLU; shift the state */
        for (int ch = 0; ch < C; ++ch) {
            const float* w = conv_w + (size_t)ch * K;
            float* st = conv_state + (size_t)ch * (K - 1);
            float acc = 0;
            for (int k = 0; k < K - 1; ++k) acc += w[k] * st[k];
            acc += w[K - 1] * x[ch];
            conv[ch] = o_silu(acc);
            for (int k = 0; k < K - 2; ++k) st[k] = st[k + 1];
            st[K - 2] = x[ch];
        }
        for (int h = 0; h < KH; ++h) {
            float* q = Q + (size_t)h * DK;
            float* k = Kx + (size_t)h * DK;
            for (int d = 0; d < DK; ++d) { q[d] = conv[h * DK + d]; k[d] = conv[KD + h * DK + d]; }
            orc_l2norm(q, DK, 1e-6f);
            orc_l2norm(k, DK, 1e-6f);
            for (int d = 0; d < DK; ++d) q[d] *= qs;
        }
        const float* V = conv + 2 * KD;
        for (int vh = 0; vh < VH; ++vh) {
            int kh = vh / rep;
            float g = -expf(A_log[vh]) * o_softplus(a[(size_t)t * VH + vh] + dt_bias[vh]);
            float gt = expf(g), bb = o_sigmoid(b[(size_t)t * VH + vh]);
            const float* q = Q + (size_t)kh * DK;
            const float* k = Kx + (size_t)kh * DK;
            const float* v = V + (size_t)vh * DV;
            float* S = state + (size_t)vh * DK * DV; /* [DK][DV] */
            for (size_t i = 0; i < (size_t)DK * DV; ++i) S[i] *= gt;
            for (int vv = 0; vv < DV; ++vv) {
                float s = 0;
                for (int kk = 0; kk < DK; ++kk) s += S[(size_t)kk * DV + vv] * k[kk];
                km[vv] = s;
            }
            for (int vv = 0; vv < DV; ++vv) dl[vv] = (v[vv] - km[vv]) * bb;
            for (int kk = 0; kk < DK; ++kk) {
                float kv = k[kk];
                float* Sr = S + (size_t)kk * DV;
                for (int vv = 0; vv < DV; ++vv) Sr[vv] += kv * dl[vv];
            }
            float* o = out + ((size_t)t * VH + vh) * DV;
            for (int vv = 0; vv < DV; ++vv) {
                float s = 0;
                for (int kk = 0; kk < DK; ++kk) s += S[(size_t)kk * DV + vv] * q[kk];
                o[vv] = s;
            }
        }
    }
    free(conv); free(Q); free(Kx); free(km); free(dl);
}

/* QwenModel::gdn_step (src/qwen_model.cpp:154-209) */
static void gdn_step(orc_model* m, const orc_layer* lw, const float* in, float* out) {
    const orc_config* c = &m->c;
    int H = c->hidden, VH = c->v_heads, DV = c->v_dim;
    int KD = c->k_heads * c->k_dim, VD = VH * DV, CONV = 2 * KD + VD;
    float* qkv = m->scratch;
    float* z = qkv + CONV;
    float* bt = z + VD;
    float* at = bt + VH;
    float* o = at + VH;
    orc_matmul_bf16(lw->in_qkv, in, qkv, CONV, H);
    orc_matmul_bf16(lw->in_z, in, z, VD, H);
    orc_matmul_bf16(lw->in_b, in, bt, VH, H);
    orc_matmul_bf16(lw->in_a, in, at, VH, H);
    orc_gdn_core(1, c->k_heads, VH, c->k_dim, DV, c->conv_k, qkv, lw->conv, at, bt, lw->A_log,
                 lw->dt_bias, m->S[lw->idx], m->cs[lw->idx], o);
    for (int vh = 0; vh < VH; ++vh)
        orc_rmsnorm_gated(o + (size_t)vh * DV, lw->gdn_norm, z + (size_t)vh * DV,
                          o + (size_t)vh * DV, DV, c->eps);
    orc_matmul_bf16(lw->out, o, out, H, VD);
}

/* FFN block of QwenModel::step (src/qwen_model.cpp:225-232) */
static void ffn(orc_model* m, const orc_layer* lw, const float* x, float* out) {
    const orc_config* c = &m->c;
    int H = c->hidden, I = c->ffn;
    float* g = m->scratch;
    float* u = g + I;
    float* hh = u + I;
    orc_matmul_bf16(lw->gate, x, g, I, H);
    orc_matmul_bf16(lw->up, x, u, I, H);
    for (int i = 0; i < I; ++i) hh[i] = o_silu(g[i]) * u[i];
    orc_matmul_bf16(lw->down, hh, out, H, I);
}

/* QwenModel::step (src/qwen_model.cpp:211-239) */
int orc_step(orc_model* m, int token, float* logits, float* layer_hidden) {
    const orc_config* c = &m->c;
    int H = c->hidden;
    if (token < 0 || token >= c->vocab || m->pos >= m->max_ctx) return -1;
    const uint16_t* row = m->embed + (size_t)token * H;
    for (int i = 0; i < H; ++i) m->hidden[i] = bf16f(row[i]);
    if (layer_hidden) memcpy(layer_hidden, m->hidden, sizeof(float) * H);
    for (int L = 0; L < c->layers; ++L) {
        const orc_layer* lw = &m->lw[L];
        orc_rmsnorm(m->hidden, lw->in_ln, m->normed, H, c->eps);
        if (lw->is_attn) attn_step(m, lw, m->normed, m->mix);
        else gdn_step(m, lw, m->normed, m->mix);
        for (int i = 0; i < H; ++i) m->hidden[i] += m->mix[i];
        orc_rmsnorm(m->hidden, lw->post_ln, m->normed, H, c->eps);
        ffn(m, lw, m->normed, m->ff);
        for (int i = 0; i < H; ++i) m->hidden[i] += m->ff[i];
        if (layer_hidden) memcpy(layer_hidden + (size_t)(L + 1) * H, m->hidden, sizeof(float) * H);
    }
    if (logits) {
        orc_rmsnorm(m->hidden, m->final_norm, m->normed, H, c->eps);
        orc_matmul_bf16(m->head, m->normed, logits, c->vocab, H);
    }
    m->pos++;
    return 0;
}

/* QwenModel::generate_greedy (src/qwen_model.cpp:241-255): argmax where a later
 * index must be strictly greater to win, so the lowest index wins ties. */
int orc_generate_greedy(orc_model* m, const int* prompt, int n_prompt, int n_new, int* out) {
    float* lg = (float*)malloc(sizeof(float) * m->c.vocab);
    orc_reset(m);
    int have = 0;
    for (int i = 0; i < n_prompt; ++i) {
        if (orc_step(m, prompt[i], lg, NULL)) { free(lg); return -1; }
        have = 1;
    }
    int n = 0;
    for (int i = 0; i < n_new && have; ++i) {
        int am = 0;
        for (int v = 1; v < m->c.vocab; ++v) if (lg[v] > lg[am]) am = v;
        out[n++] = am;
        if (orc_step(m, am, lg, NULL)) break;
    }
    free(lg);
    return n;
}

/* QwenForward::prefill (src/qwen_forward.cpp:154-206): layer-major over the whole
 * sequence from a zero state; the arithmetic per token equals the step path
 * (per-token GEMVs, zero-padded causal conv, causal attention over j <= t). It leaves
 * the decode state untouched. */
int orc_prefill(orc_model* m, const int* ids, int T, float* logits, float* layer_hidden,
                int last_only) {
    const orc_config* c = &m->c;
    int H = c->hidden, HD = c->head_dim, NQ = c->q_heads, NKV = c->kv_heads;
    int VH = c->v_heads, DV = c->v_dim, KD = c->k_heads * c->k_dim, VD = VH * DV;
    int CONV = 2 * KD + VD;
    for (int t = 0; t < T; ++t) if (ids[t] < 0 || ids[t] >= c->vocab) return -1;
    float* hid = (float*)malloc(sizeof(float) * (size_t)T * H);
    float* nrm = (float*)malloc(sizeof(float) * (size_t)T * H);
    float* mix = (float*)malloc(sizeof(float) * (size_t)T * H);
    for (int t = 0; t < T; ++t)
        for (int i = 0; i < H; ++i) hid[(size_t)t * H + i] = bf16f(m->embed[(size_t)ids[t] * H + i]);
    if (layer_hidden) memcpy(layer_hidden, hid, sizeof(float) * (size_t)T * H);
    for (int L = 0; L < c->layers; ++L) {
        const orc_layer* lw = &m->lw[L];
        for (int t = 0; t < T; ++t) orc_rmsnorm(hid + (size_t)t * H, lw->in_ln, nrm + (size_t)t * H, H, c->eps);
        if (lw->is_attn) {
            /* mix_attention (src/qwen_forward.cpp:20-80) */
            float* qkv = (float*)malloc(sizeof(float) * NQ * HD * 2);
            float* Q = (float*)malloc(sizeof(float) * (size_t)T * NQ * HD);
            float* G = (float*)malloc(sizeof(float) * (size_t)T * NQ * HD);
            float* Kc = (float*)malloc(sizeof(float) * (size_t)T * NKV * HD);
            float* Vc = (float*)malloc(sizeof(float) * (size_t)T * NKV * HD);
            float* kv = (float*)malloc(sizeof(float) * NKV * HD);
            float* ac = (float*)malloc(sizeof(float) * NQ * HD);
            for (int t = 0; t < T; ++t) {
                const float* x = nrm + (size_t)t * H;
                orc_matmul_bf16(lw->q, x, qkv, NQ * HD * 2, H);
                for (int h = 0; h < NQ; ++h) {
                    float* qd = Q + ((size_t)t * NQ + h) * HD;
                    orc_rmsnorm(qkv + (size_t)h * HD * 2, lw->q_norm, qd, HD, c->eps);
                    orc_apply_rope(qd, c->rot_dim, t, c->theta);
                    memcpy(G + ((size_t)t * NQ + h) * HD, qkv + (size_t)h * HD * 2 + HD, sizeof(float) * HD);
                }
                orc_matmul_bf16(lw->k, x, kv, NKV * HD, H);
                for (int kh = 0; kh < NKV; ++kh) {
                    float* kd = Kc + ((size_t)t * NKV + kh) * HD;
                    orc_rmsnorm(kv + (size_t)kh * HD, lw->k_norm, kd, HD, c->eps);
                    orc_apply_rope(kd, c->rot_dim, t, c->theta);
                }
                orc_matmul_bf16(lw->v, x, Vc + (size_t)t * NKV * HD, NKV * HD, H);
            }
            for (int t = 0; t < T; ++t) {
                orc_attention(NQ, NKV, HD, t + 1, Q + (size_t)t * NQ * HD, G + (size_t)t * NQ * HD,
                              Kc, Vc, ac);
                orc_matmul_bf16(lw->o, ac, mix + (size_t)t * H, H, NQ * HD);
            }
            free(qkv); free(Q); free(G); free(Kc); free(Vc); free(kv); free(ac);
        } else {
            /* mix_gdn (src/qwen_forward.cpp:83-152) */
            float* mixed = (float*)malloc(sizeof(float) * (size_t)T * CONV);
            float* z = (float*)malloc(sizeof(float) * (size_t)T * VD);
            float* a = (float*)malloc(sizeof(float) * (size_t)T * VH);
            float* b = (float*)malloc(sizeof(float) * (size_t)T * VH);
            float* o = (float*)malloc(sizeof(float) * (size_t)T * VD);
            float* S = (float*)calloc((size_t)VH * c->k_dim * DV, sizeof(float));
            float* cs = (float*)calloc((size_t)CONV * (c->conv_k - 1), sizeof(float));
            for (int t = 0; t < T; ++t) {
                const float* x = nrm + (size_t)t * H;
                orc_matmul_bf16(lw->in_qkv, x, mixed + (size_t)t * CONV, CONV, H);
                orc_matmul_bf16(lw->in_z, x, z + (size_t)t * VD, VD, H);
                orc_matmul_bf16(lw->in_b, x, b + (size_t)t * VH, VH, H);
                orc_matmul_bf16(lw->in_a, x, a + (size_t)t * VH, VH, H);
            }
            orc_gdn_core(T, c->k_heads, VH, c->k_dim, DV, c->conv_k, mixed, lw->conv, a, b,
                         lw->A_log, lw->dt_bias, S, cs, o);
            for (int t = 0; t < T; ++t) {
                for (int vh = 0; vh < VH; ++vh) {
                    float* oh = o + ((size_t)t * VH + vh) * DV;
                    orc_rmsnorm_gated(oh, lw->gdn_norm, z + ((size_t)t * VH + vh) * DV, oh, DV, c->eps);
                }
                orc_matmul_bf16(lw->out, o + (size_t)t * VD, mix + (size_t)t * H, H, VD);
            }
            free(mixed); free(z); free(a); free(b); free(o); free(S); free(cs);
        }
        for (size_t i = 0; i < (size_t)T * H; ++i) hid[i] += mix[i];
        /* FFN per token (src/qwen_forward.cpp:183-192) */
        for (int t = 0; t < T; ++t) {
            orc_rmsnorm(hid + (size_t)t * H, lw->post_ln, nrm + (size_t)t * H, H, c->eps);
            ffn(m, lw, nrm + (size_t)t * H, mix + (size_t)t * H);
        }
        for (size_t i = 0; i < (size_t)T * H; ++i) hid[i] += mix[i];
        if (layer_hidden) memcpy(layer_hidden + (size_t)(L + 1) * T * H, hid, sizeof(float) * (size_t)T * H);
    }
    if (logits) {
        float* fno = (float*)malloc(sizeof(float) * H);
        int t0 = last_only ? T - 1 : 0;
        for (int t = t0; t < T; ++t) {
            orc_rmsnorm(hid + (size_t)t * H, m->final_norm, fno, H, c->eps);
            orc_matmul_bf16(m->head, fno, logits + (size_t)(last_only ? 0 : t) * c->vocab, c->vocab, H);
        }
        free(fno);
    }
    free(hid); free(nrm); free(mix);
    return 0;
}
