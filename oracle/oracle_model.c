/*
 * oracle_model.c - CPU restatement of rembed's per-architecture forward
 * passes (internal/model) and its batch fan-out (rembed.go).
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA path and the
 * CPU baseline in bench.py.  The product never links or loads it.
 *
 * Weights are borrowed float32 tensors named as in the Hugging Face
 * checkpoints the reference loads (bert.go:338-518).  Dense projections
 * follow newDense/applyDense (bert.go:263-301): fp32 (k-ordered FMA),
 * weight-only int8 (PackB8) or full int8 (PackB8VNNI + per-row u8
 * activations), each followed by a separate bias add.
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define MAXW 4096
#define NAMELEN 160

typedef struct {
    char name[NAMELEN];
    const float *data;
    int64_t numel;
} wentry;

/* denseWeight (bert.go:32-39) after newDense. */
typedef struct {
    int in, out;
    const float *w;   /* fp32 [out x in] (borrowed or owned via own) */
    float *own;       /* owned fused buffer, if any */
    int8_t *q;        /* int8 [out x in] */
    float *scales;
    int32_t *colsum;
    const float *bias;
    float *own_bias;
} dense;

typedef struct {
    dense qkv, attn_out, ffn1, ffn2;
    const float *attn_ln_g, *attn_ln_b, *out_ln_g, *out_ln_b;
} bert_layer;

/* One decoder-style layer (qwen3.go:20-34, modernbert.go:20-28,
 * gemma3.go:20-38, nomic.go:12-20); unused fields stay NULL. */
typedef struct {
    dense q, k, v, qkv, o, gate, up, down, wi, fc11, fc12;
    const float *in_norm, *q_norm, *k_norm, *post_attn, *pre_ffn, *post_ffn, *mlp_norm;
    float *own[6]; /* unit-offset copies (Gemma) */
    const float *n1g, *n1b, *n2g, *n2b;
    int global;
} dec_layer;

struct or_model {
    or_config cfg;
    int quant;
    wentry w[MAXW];
    int nw;
    int finalized;
    int pos_off;
    const float *word_emb, *pos_emb, *type_emb, *emb_ln_g, *emb_ln_b, *rel_bias;
    bert_layer *layers;
    dec_layer *dl;
    const float *final_norm;
    float *final_norm_own, *zero_beta;
    const float *dense1, *dense2; /* Gemma Dense head [D x H], [H x D] */
};

static void seterr(char *err, const char *fmt, ...) {
    if (!err) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, 256, fmt, ap);
    va_end(ap);
}

or_model *or_model_new(const or_config *cfg, int quant) {
    or_model *m = (or_model *)calloc(1, sizeof(or_model));
    m->cfg = *cfg;
    m->quant = quant;
    if (m->cfg.eps == 0.0f) m->cfg.eps = 1e-12f; /* config.go:228-230 */
    /* PositionOffset, config.go:84-89 */
    m->pos_off = (cfg->arch == OR_ARCH_MPNET || cfg->arch == OR_ARCH_ROBERTA) ? cfg->pad_token_id + 1 : 0;
    return m;
}

int or_model_set(or_model *m, const char *name, const float *data, int64_t numel) {
    if (m->nw >= MAXW || strlen(name) >= NAMELEN) return -1;
    for (int i = 0; i < m->nw; i++)
        if (strcmp(m->w[i].name, name) == 0) {
            m->w[i].data = data;
            m->w[i].numel = numel;
            return 0;
        }
    snprintf(m->w[m->nw].name, NAMELEN, "%s", name);
    m->w[m->nw].data = data;
    m->w[m->nw].numel = numel;
    m->nw++;
    return 0;
}

/* Look up name with any of the reference's prefixes (bert.go:338-343). */
static const float *get_tensor(or_model *m, const char *name, int64_t numel, char *err) {
    static const char *prefixes[] = {"", "bert.", "roberta.", "mpnet.", "distilbert.", "model."};
    char full[NAMELEN * 2];
    for (size_t p = 0; p < sizeof(prefixes) / sizeof(prefixes[0]); p++) {
        snprintf(full, sizeof(full), "%s%s", prefixes[p], name);
        for (int i = 0; i < m->nw; i++)
            if (strcmp(m->w[i].name, full) == 0) {
                if (numel >= 0 && m->w[i].numel != numel) {
                    seterr(err, "tensor %s has %lld elements, want %lld", full, (long long)m->w[i].numel,
                           (long long)numel);
                    return NULL;
                }
                return m->w[i].data;
            }
    }
    seterr(err, "missing tensor %s", name);
    return NULL;
}

/* newDense, bert.go:263-278 (quantisation at load, never a silent
 * fallback here: a non-finite weight under int8 is an error). */
static int make_dense(dense *d, const float *w, const float *bias, int in, int out, int quant, char *err) {
    d->in = in;
    d->out = out;
    d->w = w;
    d->bias = bias;
    if (quant == OR_QUANT_FULL) {
        d->q = (int8_t *)malloc((size_t)in * out);
        d->colsum = (int32_t *)malloc(sizeof(int32_t) * out);
        d->scales = (float *)malloc(sizeof(float) * out);
        if (or_packb8vnni(w, in, out, d->q, d->colsum, d->scales) != 0) {
            seterr(err, "PackB8VNNI rejected a [%d x %d] weight (non-finite value or out %% 16 != 0)", out, in);
            return -1;
        }
    } else if (quant == OR_QUANT_WEIGHTS) {
        d->q = (int8_t *)malloc((size_t)in * out);
        d->scales = (float *)malloc(sizeof(float) * out);
        if (or_packb8(w, in, out, d->q, d->scales) != 0) {
            seterr(err, "PackB8 rejected a [%d x %d] weight (non-finite value or out %% 16 != 0)", out, in);
            return -1;
        }
    }
    return 0;
}

static void free_dense(dense *d) {
    free(d->own);
    free(d->own_bias);
    free(d->q);
    free(d->scales);
    free(d->colsum);
}

/* applyDense, bert.go:282-301 */
static void apply_dense(const dense *d, float *dst, const float *x, int seq, int quant) {
    if (quant == OR_QUANT_FULL)
        or_matmul_vnni(dst, x, d->q, d->colsum, d->scales, seq, d->in, d->out);
    else if (quant == OR_QUANT_WEIGHTS)
        or_matmul_packed8(dst, x, d->q, d->scales, seq, d->in, d->out);
    else
        or_matmul_packed(dst, x, d->w, seq, d->in, d->out);
    if (d->bias) or_add_bias(dst, d->bias, seq, d->out);
}

/* BERT / DistilBERT / RoBERTa / MPNet weight binding, bert.go:338-518. */
static int finalize_bert(or_model *m, char *err) {
    const or_config *c = &m->cfg;
    int H = c->hidden, I = c->inter, arch = c->arch;
    int distil = arch == OR_ARCH_DISTILBERT, mpnet = arch == OR_ARCH_MPNET;
    if (c->heads <= 0 || H % c->heads != 0) {
        seterr(err, "hidden_size %d not divisible by num_attention_heads %d", H, c->heads);
        return -1;
    }
    if (!(m->word_emb = get_tensor(m, "embeddings.word_embeddings.weight", (int64_t)c->vocab * H, err))) return -1;
    if (!(m->pos_emb = get_tensor(m, "embeddings.position_embeddings.weight", (int64_t)c->max_pos * H, err))) return -1;
    if (!(m->emb_ln_g = get_tensor(m, "embeddings.LayerNorm.weight", H, err))) return -1;
    if (!(m->emb_ln_b = get_tensor(m, "embeddings.LayerNorm.bias", H, err))) return -1;
    m->layers = (bert_layer *)calloc(c->layers, sizeof(bert_layer));
    char nm[NAMELEN];
#define GET(dst, fmt, n)                                   \
    do {                                                   \
        snprintf(nm, sizeof nm, fmt, li);                  \
        if (!((dst) = get_tensor(m, nm, (n), err))) return -1;   \
    } while (0)
    for (int li = 0; li < c->layers; li++) {
        bert_layer *l = &m->layers[li];
        const float *qW, *qB, *kW, *kB, *vW, *vB, *oW, *oB, *f1W, *f1B, *f2W, *f2B;
        if (distil) {
            GET(qW, "transformer.layer.%d.attention.q_lin.weight", (int64_t)H * H);
            GET(qB, "transformer.layer.%d.attention.q_lin.bias", H);
            GET(kW, "transformer.layer.%d.attention.k_lin.weight", (int64_t)H * H);
            GET(kB, "transformer.layer.%d.attention.k_lin.bias", H);
            GET(vW, "transformer.layer.%d.attention.v_lin.weight", (int64_t)H * H);
            GET(vB, "transformer.layer.%d.attention.v_lin.bias", H);
            GET(oW, "transformer.layer.%d.attention.out_lin.weight", (int64_t)H * H);
            GET(oB, "transformer.layer.%d.attention.out_lin.bias", H);
            GET(l->attn_ln_g, "transformer.layer.%d.sa_layer_norm.weight", H);
            GET(l->attn_ln_b, "transformer.layer.%d.sa_layer_norm.bias", H);
            GET(f1W, "transformer.layer.%d.ffn.lin1.weight", (int64_t)I * H);
            GET(f1B, "transformer.layer.%d.ffn.lin1.bias", I);
            GET(f2W, "transformer.layer.%d.ffn.lin2.weight", (int64_t)H * I);
            GET(f2B, "transformer.layer.%d.ffn.lin2.bias", H);
            GET(l->out_ln_g, "transformer.layer.%d.output_layer_norm.weight", H);
            GET(l->out_ln_b, "transformer.layer.%d.output_layer_norm.bias", H);
        } else {
            if (mpnet) {
                GET(qW, "encoder.layer.%d.attention.attn.q.weight", (int64_t)H * H);
                GET(qB, "encoder.layer.%d.attention.attn.q.bias", H);
                GET(kW, "encoder.layer.%d.attention.attn.k.weight", (int64_t)H * H);
                GET(kB, "encoder.layer.%d.attention.attn.k.bias", H);
                GET(vW, "encoder.layer.%d.attention.attn.v.weight", (int64_t)H * H);
                GET(vB, "encoder.layer.%d.attention.attn.v.bias", H);
                GET(oW, "encoder.layer.%d.attention.attn.o.weight", (int64_t)H * H);
                GET(oB, "encoder.layer.%d.attention.attn.o.bias", H);
                GET(l->attn_ln_g, "encoder.layer.%d.attention.LayerNorm.weight", H);
                GET(l->attn_ln_b, "encoder.layer.%d.attention.LayerNorm.bias", H);
            } else {
                GET(qW, "encoder.layer.%d.attention.self.query.weight", (int64_t)H * H);
                GET(qB, "encoder.layer.%d.attention.self.query.bias", H);
                GET(kW, "encoder.layer.%d.attention.self.key.weight", (int64_t)H * H);
                GET(kB, "encoder.layer.%d.attention.self.key.bias", H);
                GET(vW, "encoder.layer.%d.attention.self.value.weight", (int64_t)H * H);
                GET(vB, "encoder.layer.%d.attention.self.value.bias", H);
                GET(oW, "encoder.layer.%d.attention.output.dense.weight", (int64_t)H * H);
                GET(oB, "encoder.layer.%d.attention.output.dense.bias", H);
                GET(l->attn_ln_g, "encoder.layer.%d.attention.output.LayerNorm.weight", H);
                GET(l->attn_ln_b, "encoder.layer.%d.attention.output.LayerNorm.bias", H);
            }
            GET(f1W, "encoder.layer.%d.intermediate.dense.weight", (int64_t)I * H);
            GET(f1B, "encoder.layer.%d.intermediate.dense.bias", I);
            GET(f2W, "encoder.layer.%d.output.dense.weight", (int64_t)H * I);
            GET(f2B, "encoder.layer.%d.output.dense.bias", H);
            GET(l->out_ln_g, "encoder.layer.%d.output.LayerNorm.weight", H);
            GET(l->out_ln_b, "encoder.layer.%d.output.LayerNorm.bias", H);
        }
        /* Fused Q||K||V [3H x H], bert.go:479-485 */
        float *qkvW = (float *)malloc(sizeof(float) * 3 * (size_t)H * H);
        float *qkvB = (float *)malloc(sizeof(float) * 3 * (size_t)H);
        memcpy(qkvW, qW, sizeof(float) * (size_t)H * H);
        memcpy(qkvW + (size_t)H * H, kW, sizeof(float) * (size_t)H * H);
        memcpy(qkvW + 2 * (size_t)H * H, vW, sizeof(float) * (size_t)H * H);
        memcpy(qkvB, qB, sizeof(float) * H);
        memcpy(qkvB + H, kB, sizeof(float) * H);
        memcpy(qkvB + 2 * H, vB, sizeof(float) * H);
        l->qkv.own = qkvW;
        l->qkv.own_bias = qkvB;
        if (make_dense(&l->qkv, qkvW, qkvB, H, 3 * H, m->quant, err)) return -1;
        if (make_dense(&l->attn_out, oW, oB, H, H, m->quant, err)) return -1;
        if (make_dense(&l->ffn1, f1W, f1B, H, I, m->quant, err)) return -1;
        if (make_dense(&l->ffn2, f2W, f2B, I, H, m->quant, err)) return -1;
    }
#undef GET
    if (distil) return 0;
    if (mpnet) {
        if (!(m->rel_bias = get_tensor(m, "encoder.relative_attention_bias.weight", (int64_t)c->rel_buckets * c->heads, err)))
            return -1;
        return 0;
    }
    /* token_type_embeddings: any first dimension, row 0 used (bert.go:507-515) */
    for (int i = 0; i < m->nw; i++) {
        const char *n = m->w[i].name;
        const char *s = strstr(n, "embeddings.token_type_embeddings.weight");
        if (s && m->w[i].numel >= H && m->w[i].numel % H == 0) {
            m->type_emb = m->w[i].data;
            return 0;
        }
    }
    seterr(err, "missing tensor embeddings.token_type_embeddings.weight");
    return -1;
}

static float *unit_offset(const float *v, int n) { /* gemma3.go:44-50 */
    float *o = (float *)malloc(sizeof(float) * n);
    for (int i = 0; i < n; i++) o[i] = v[i] + 1.0f;
    return o;
}

/* qwen3.go:114-183, modernbert.go:33-106, gemma3.go:57-170, nomic.go:22-111 */
static int finalize_decoder(or_model *m, char *err) {
    const or_config *c = &m->cfg;
    int arch = c->arch, H = c->hidden, I = c->inter, q = m->quant;
    int dh = c->head_dim ? c->head_dim : H / c->heads;
    int nq = c->heads, nkv = c->kv_heads ? c->kv_heads : c->heads;
    int qd = nq * dh, kvd = nkv * dh;
    char nm[NAMELEN];
    m->dl = (dec_layer *)calloc(c->layers, sizeof(dec_layer));
    if (arch == OR_ARCH_QWEN3) {
        if (!(m->word_emb = get_tensor(m, "embed_tokens.weight", (int64_t)c->vocab * H, err))) return -1;
        if (!(m->final_norm = get_tensor(m, "norm.weight", H, err))) return -1;
    } else if (arch == OR_ARCH_GEMMA3) {
        const float *fn;
        if (!(m->word_emb = get_tensor(m, "embed_tokens.weight", (int64_t)c->vocab * H, err))) return -1;
        if (!(fn = get_tensor(m, "norm.weight", H, err))) return -1;
        m->final_norm = m->final_norm_own = unit_offset(fn, H);
        if (!(m->dense1 = get_tensor(m, "2_Dense.linear.weight", (int64_t)c->dense_hidden * H, err))) return -1;
        if (!(m->dense2 = get_tensor(m, "3_Dense.linear.weight", (int64_t)H * c->dense_hidden, err))) return -1;
    } else if (arch == OR_ARCH_MODERNBERT) {
        if (!(m->word_emb = get_tensor(m, "embeddings.tok_embeddings.weight", (int64_t)c->vocab * H, err))) return -1;
        if (!(m->emb_ln_g = get_tensor(m, "embeddings.norm.weight", H, err))) return -1;
        if (!(m->final_norm = get_tensor(m, "final_norm.weight", H, err))) return -1;
        m->zero_beta = (float *)calloc(H, sizeof(float));
    } else { /* nomic */
        if (!(m->word_emb = get_tensor(m, "embeddings.word_embeddings.weight", (int64_t)c->vocab * H, err))) return -1;
        if (!(m->type_emb = get_tensor(m, "embeddings.token_type_embeddings.weight", 2 * (int64_t)H, err))) return -1;
        if (!(m->emb_ln_g = get_tensor(m, "emb_ln.weight", H, err))) return -1;
        if (!(m->emb_ln_b = get_tensor(m, "emb_ln.bias", H, err))) return -1;
    }
#define GETL(dst, name, n)                                        \
    do {                                                          \
        snprintf(nm, sizeof nm, "%s%d.%s", pre, li, name);        \
        if (!((dst) = get_tensor(m, nm, (n), err))) return -1;    \
    } while (0)
    for (int li = 0; li < c->layers; li++) {
        dec_layer *l = &m->dl[li];
        const float *w1, *w2, *w3, *w4;
        if (arch == OR_ARCH_QWEN3 || arch == OR_ARCH_GEMMA3) {
            const char *pre = "layers.";
            const float *in, *qn, *kn, *pa = NULL, *pf = NULL, *pff = NULL, *post = NULL;
            GETL(in, "input_layernorm.weight", H);
            GETL(qn, "self_attn.q_norm.weight", dh);
            GETL(kn, "self_attn.k_norm.weight", dh);
            if (arch == OR_ARCH_QWEN3) {
                GETL(post, "post_attention_layernorm.weight", H);
                l->in_norm = in;
                l->q_norm = qn;
                l->k_norm = kn;
                l->post_attn = post;
            } else {
                GETL(pa, "post_attention_layernorm.weight", H);
                GETL(pf, "pre_feedforward_layernorm.weight", H);
                GETL(pff, "post_feedforward_layernorm.weight", H);
                l->in_norm = l->own[0] = unit_offset(in, H);
                l->q_norm = l->own[1] = unit_offset(qn, dh);
                l->k_norm = l->own[2] = unit_offset(kn, dh);
                l->post_attn = l->own[3] = unit_offset(pa, H);
                l->pre_ffn = l->own[4] = unit_offset(pf, H);
                l->post_ffn = l->own[5] = unit_offset(pff, H);
                l->global = (li + 1) % c->sliding_pattern == 0; /* gemma3.go:91 */
            }
            GETL(w1, "self_attn.q_proj.weight", (int64_t)qd * H);
            if (make_dense(&l->q, w1, NULL, H, qd, q, err)) return -1;
            GETL(w1, "self_attn.k_proj.weight", (int64_t)kvd * H);
            if (make_dense(&l->k, w1, NULL, H, kvd, q, err)) return -1;
            GETL(w1, "self_attn.v_proj.weight", (int64_t)kvd * H);
            if (make_dense(&l->v, w1, NULL, H, kvd, q, err)) return -1;
            GETL(w1, "self_attn.o_proj.weight", (int64_t)H * qd);
            if (make_dense(&l->o, w1, NULL, qd, H, q, err)) return -1;
            GETL(w1, "mlp.gate_proj.weight", (int64_t)I * H);
            if (make_dense(&l->gate, w1, NULL, H, I, q, err)) return -1;
            GETL(w1, "mlp.up_proj.weight", (int64_t)I * H);
            if (make_dense(&l->up, w1, NULL, H, I, q, err)) return -1;
            GETL(w1, "mlp.down_proj.weight", (int64_t)H * I);
            if (make_dense(&l->down, w1, NULL, I, H, q, err)) return -1;
        } else if (arch == OR_ARCH_MODERNBERT) {
            const char *pre = "layers.";
            l->global = li % c->global_every == 0; /* modernbert.go:73 */
            if (li != 0) GETL(l->in_norm, "attn_norm.weight", H);
            GETL(l->mlp_norm, "mlp_norm.weight", H);
            GETL(w1, "attn.Wqkv.weight", 3 * (int64_t)H * H);
            GETL(w2, "attn.Wo.weight", (int64_t)H * H);
            GETL(w3, "mlp.Wi.weight", 2 * (int64_t)I * H);
            GETL(w4, "mlp.Wo.weight", (int64_t)H * I);
            if (make_dense(&l->qkv, w1, NULL, H, 3 * H, q, err)) return -1;
            if (make_dense(&l->o, w2, NULL, H, H, q, err)) return -1;
            if (make_dense(&l->wi, w3, NULL, H, 2 * I, q, err)) return -1;
            if (make_dense(&l->down, w4, NULL, I, H, q, err)) return -1;
        } else { /* nomic */
            const char *pre = "encoder.layers.";
            GETL(l->n1g, "norm1.weight", H);
            GETL(l->n1b, "norm1.bias", H);
            GETL(l->n2g, "norm2.weight", H);
            GETL(l->n2b, "norm2.bias", H);
            GETL(w1, "attn.Wqkv.weight", 3 * (int64_t)H * H);
            GETL(w2, "attn.out_proj.weight", (int64_t)H * H);
            if (make_dense(&l->qkv, w1, NULL, H, 3 * H, q, err)) return -1;
            if (make_dense(&l->o, w2, NULL, H, H, q, err)) return -1;
            GETL(w1, "mlp.fc11.weight", (int64_t)I * H);
            if (make_dense(&l->fc11, w1, NULL, H, I, q, err)) return -1;
            GETL(w1, "mlp.fc12.weight", (int64_t)I * H);
            if (make_dense(&l->fc12, w1, NULL, H, I, q, err)) return -1;
            GETL(w1, "mlp.fc2.weight", (int64_t)H * I);
            if (make_dense(&l->down, w1, NULL, I, H, q, err)) return -1;
        }
    }
#undef GETL
    return 0;
}

int or_model_finalize(or_model *m, char *err) {
    int rc;
    switch (m->cfg.arch) {
    case OR_ARCH_BERT:
    case OR_ARCH_DISTILBERT:
    case OR_ARCH_ROBERTA:
    case OR_ARCH_MPNET:
        rc = finalize_bert(m, err);
        break;
    case OR_ARCH_QWEN3:
    case OR_ARCH_MODERNBERT:
    case OR_ARCH_GEMMA3:
    case OR_ARCH_NOMIC:
        rc = finalize_decoder(m, err);
        break;
    default:
        seterr(err, "oracle: architecture %d not restated", m->cfg.arch);
        return -1;
    }
    if (rc == 0) m->finalized = 1;
    return rc;
}

void or_model_free(or_model *m) {
    if (!m) return;
    if (m->dl) {
        for (int i = 0; i < m->cfg.layers; i++) {
            dec_layer *l = &m->dl[i];
            dense *ds[] = {&l->q, &l->k, &l->v, &l->qkv, &l->o, &l->gate, &l->up, &l->down, &l->wi, &l->fc11, &l->fc12};
            for (size_t j = 0; j < sizeof ds / sizeof ds[0]; j++) free_dense(ds[j]);
            for (int j = 0; j < 6; j++) free(l->own[j]);
        }
        free(m->dl);
    }
    free(m->final_norm_own);
    free(m->zero_beta);
    if (m->layers) {
        for (int i = 0; i < m->cfg.layers; i++) {
            free_dense(&m->layers[i].qkv);
            free_dense(&m->layers[i].attn_out);
            free_dense(&m->layers[i].ffn1);
            free_dense(&m->layers[i].ffn2);
        }
        free(m->layers);
    }
    free(m);
}

static int max_seq_len(const or_model *m) { return m->cfg.max_pos - m->pos_off; } /* config.go:93-95 */

/* encodeWorkers BERT body, bert.go:740-923 (serial: workers = 1). */
static int encode_bert(or_model *m, const int64_t *ids, int seq, float *x, char *err) {
    const or_config *c = &m->cfg;
    int H = c->hidden, heads = c->heads, dh = H / heads, I = c->inter, q = m->quant;
    float eps = c->eps;
    for (int i = 0; i < seq; i++) {
        if (ids[i] < 0 || ids[i] >= c->vocab) {
            seterr(err, "token id %lld out of vocab range %d", (long long)ids[i], c->vocab);
            return -1;
        }
    }
    /* Embeddings, bert.go:795-814 */
    for (int i = 0; i < seq; i++) {
        float *row = x + (int64_t)i * H;
        const float *w = m->word_emb + ids[i] * H;
        const float *p = m->pos_emb + (int64_t)(i + m->pos_off) * H;
        if (m->type_emb) {
            for (int j = 0; j < H; j++) row[j] = w[j] + p[j] + m->type_emb[j];
        } else {
            for (int j = 0; j < H; j++) row[j] = w[j] + p[j];
        }
    }
    or_layernorm(x, m->emb_ln_g, m->emb_ln_b, seq, H, eps);

    float *bias_delta = NULL;
    int ndelta = 2 * seq - 1;
    if (m->rel_bias) { /* bert.go:820-830 */
        bias_delta = (float *)malloc(sizeof(float) * heads * ndelta);
        for (int d = -(seq - 1); d <= seq - 1; d++) {
            int b = or_relpos_bucket(d, c->rel_buckets);
            for (int h = 0; h < heads; h++) bias_delta[h * ndelta + d + seq - 1] = m->rel_bias[b * heads + h];
        }
    }
    float *qkv = (float *)malloc(sizeof(float) * (size_t)seq * 3 * H);
    float *ctx = (float *)malloc(sizeof(float) * (size_t)seq * H);
    float *tmp = (float *)malloc(sizeof(float) * (size_t)seq * H);
    float *ffh = (float *)malloc(sizeof(float) * (size_t)seq * I);
    float *sc = (float *)malloc(sizeof(float) * (size_t)seq * seq);
    float *qh = (float *)malloc(sizeof(float) * (size_t)seq * dh);
    float *kh = (float *)malloc(sizeof(float) * (size_t)seq * dh);
    float *vt = (float *)malloc(sizeof(float) * (size_t)seq * dh);
    float *ch = (float *)malloc(sizeof(float) * (size_t)seq * dh);
    float scale = (float)(1.0 / sqrt((double)dh));

    for (int li = 0; li < c->layers; li++) {
        bert_layer *l = &m->layers[li];
        apply_dense(&l->qkv, qkv, x, seq, q);
        for (int h = 0; h < heads; h++) { /* bert.go:853-902 */
            int off = h * dh;
            for (int i = 0; i < seq; i++) {
                const float *row = qkv + (int64_t)i * 3 * H;
                memcpy(qh + (int64_t)i * dh, row + off, sizeof(float) * dh);
                memcpy(kh + (int64_t)i * dh, row + H + off, sizeof(float) * dh);
                for (int d = 0; d < dh; d++) vt[(int64_t)d * seq + i] = row[2 * H + off + d];
            }
            or_matmul_serial(sc, qh, kh, seq, dh, seq);
            if (bias_delta) {
                const float *bd = bias_delta + h * ndelta;
                for (int i = 0; i < seq; i++) {
                    float *row = sc + (int64_t)i * seq;
                    const float *bdi = bd + (seq - 1 - i);
                    for (int j = 0; j < seq; j++) row[j] = (float)(row[j] * scale) + bdi[j];
                }
            } else {
                for (int i = 0; i < seq * seq; i++) sc[i] *= scale;
            }
            or_softmax(sc, seq, seq);
            or_matmul_serial(ch, sc, vt, seq, seq, dh);
            for (int i = 0; i < seq; i++) memcpy(ctx + (int64_t)i * H + off, ch + (int64_t)i * dh, sizeof(float) * dh);
        }
        apply_dense(&l->attn_out, tmp, ctx, seq, q);
        or_add(x, tmp, seq * H);
        or_layernorm(x, l->attn_ln_g, l->attn_ln_b, seq, H, eps);
        apply_dense(&l->ffn1, ffh, x, seq, q);
        or_gelu(ffh, seq * I);
        apply_dense(&l->ffn2, tmp, ffh, seq, q);
        or_add(x, tmp, seq * H);
        or_layernorm(x, l->out_ln_g, l->out_ln_b, seq, H, eps);
    }
    free(bias_delta);
    free(qkv);
    free(ctx);
    free(tmp);
    free(ffh);
    free(sc);
    free(qh);
    free(kh);
    free(vt);
    free(ch);
    return 0;
}

/* ropeTable, modernbert.go:108-123: float64 inverse frequencies and trig,
 * rounded to float32; cos/sin [seq x dh/2]. */
static void rope_table(float *cs, float *sn, int seq, int dh, double theta) {
    int half = dh / 2;
    for (int d = 0; d < half; d++) {
        double inv = pow(theta, -2.0 * (double)d / (double)dh);
        for (int p = 0; p < seq; p++) {
            double ang = (double)p * inv;
            cs[p * half + d] = (float)cos(ang);
            sn[p * half + d] = (float)sin(ang);
        }
    }
}

/* applyRoPE, modernbert.go:125-143: rotate_half, products rounded before
 * the add. x is [seq x dh]. */
static void apply_rope(float *x, int seq, int dh, const float *cs, const float *sn) {
    int half = dh / 2;
    for (int p = 0; p < seq; p++) {
        float *row = x + (int64_t)p * dh;
        const float *c = cs + (int64_t)p * half, *s = sn + (int64_t)p * half;
        for (int d = 0; d < half; d++) {
            float x1 = row[d], x2 = row[d + half], cc = c[d], ss = s[d];
            row[d] = (x1 * cc) - (x2 * ss);
            row[d + half] = (x2 * cc) + (x1 * ss);
        }
    }
}

/* flashAttnCausalHead, qwen3.go:307-390 (block 64, online softmax,
 * future key blocks skipped). */
#define FLASH_BLK 64
static void flash_attn_causal_head(const float *qH, const float *kH, const float *vH, float *out, int seq, int dh,
                                   float scale, float *sblk, float *acc, float *mrow, float *lrow) {
    const float neg = -1e30f;
    for (int q0 = 0; q0 < seq; q0 += FLASH_BLK) {
        int q1 = q0 + FLASH_BLK < seq ? q0 + FLASH_BLK : seq;
        int nq = q1 - q0;
        for (int r = 0; r < nq; r++) {
            mrow[r] = neg;
            lrow[r] = 0;
        }
        memset(acc, 0, sizeof(float) * (size_t)nq * dh);
        for (int k0 = 0; k0 < q1; k0 += FLASH_BLK) {
            int k1 = k0 + FLASH_BLK < q1 ? k0 + FLASH_BLK : q1;
            int nk = k1 - k0;
            or_matmul_serial(sblk, qH + (int64_t)q0 * dh, kH + (int64_t)k0 * dh, nq, dh, nk);
            for (int r = 0; r < nq; r++) {
                int i = q0 + r;
                float *srow = sblk + (int64_t)r * nk;
                float rmax = neg;
                for (int c = 0; c < nk; c++) {
                    if (k0 + c > i) {
                        srow[c] = neg;
                    } else {
                        srow[c] *= scale;
                        if (srow[c] > rmax) rmax = srow[c];
                    }
                }
                if (rmax == neg) continue;
                float mprev = mrow[r], mnew = mprev;
                if (rmax > mnew) mnew = rmax;
                float *ar = acc + (int64_t)r * dh;
                if (mprev != neg && mnew != mprev) {
                    float corr = or_expnonpos(mprev - mnew);
                    lrow[r] *= corr;
                    for (int d = 0; d < dh; d++) ar[d] *= corr;
                }
                float lr = lrow[r];
                for (int c = 0; c < nk; c++) {
                    if (k0 + c > i) continue;
                    float pp = or_expnonpos(srow[c] - mnew);
                    lr += pp;
                    const float *vk = vH + (int64_t)(k0 + c) * dh;
                    for (int d = 0; d < dh; d++) ar[d] += pp * vk[d];
                }
                lrow[r] = lr;
                mrow[r] = mnew;
            }
        }
        for (int r = 0; r < nq; r++) {
            float inv = 1.0f / lrow[r];
            for (int d = 0; d < dh; d++) out[(int64_t)(q0 + r) * dh + d] = acc[(int64_t)r * dh + d] * inv;
        }
    }
}

/* Exported form of flash_attn_causal_head with its own scratch, so the
 * reference's TestFlashAttnCausalHead (qwen3_test.go:15-80) can pin it
 * against a naive softmax.  Returns 0, or -1 if scratch cannot be had. */
int or_flash_attn_causal_head(const float *qH, const float *kH, const float *vH, float *out, int seq, int dh,
                              float scale) {
    int bq = seq < FLASH_BLK ? seq : FLASH_BLK;
    float *sblk = malloc(sizeof(float) * (size_t)bq * bq);
    float *acc = malloc(sizeof(float) * (size_t)bq * dh);
    float *mrow = malloc(sizeof(float) * (size_t)bq);
    float *lrow = malloc(sizeof(float) * (size_t)bq);
    int rc = -1;
    if (sblk && acc && mrow && lrow) {
        flash_attn_causal_head(qH, kH, vH, out, seq, dh, scale, sblk, acc, mrow, lrow);
        rc = 0;
    }
    free(sblk);
    free(acc);
    free(mrow);
    free(lrow);
    return rc;
}

/* Full-score attention of one head with a bidirectional window (the
 * ModernBERT / Gemma / nomic pattern: MatMulSerial, scale, mask, Softmax,
 * MatMulSerial). window_kind: 0 none; 1 |i-j| <= w (modernbert.go:268-274);
 * 2 |i-j| < w (gemma3.go:339-346).  vT is [dh x seq]. */
static void full_attn_head(const float *qH, const float *kH, const float *vT, float *out, int seq, int dh,
                           float scale, int window_kind, int w, float *sc) {
    or_matmul_serial(sc, qH, kH, seq, dh, seq);
    for (int i = 0; i < seq; i++) {
        float *row = sc + (int64_t)i * seq;
        for (int j = 0; j < seq; j++) row[j] *= scale;
        if (window_kind == 1) {
            for (int j = 0; j < seq; j++)
                if (j < i - w || j > i + w) row[j] = -1e30f;
        } else if (window_kind == 2) {
            for (int j = 0; j < seq; j++)
                if (j <= i - w || j >= i + w) row[j] = -1e30f;
        }
    }
    or_softmax(sc, seq, seq);
    or_matmul_serial(out, sc, vT, seq, seq, dh);
}

/* encodeQwen3 / encodeModernBERT / encodeGemma3 / encodeNomic
 * (qwen3.go:395-548, modernbert.go:148-311, gemma3.go:206-384,
 * nomic.go:113-250). */
static int encode_decoder(or_model *m, const int64_t *ids, int seq, float *x, char *err) {
    const or_config *c = &m->cfg;
    int arch = c->arch, H = c->hidden, I = c->inter, qt = m->quant;
    int dh = c->head_dim ? c->head_dim : H / c->heads;
    int nq = c->heads, nkv = c->kv_heads ? c->kv_heads : c->heads, group = nq / nkv, half = dh / 2;
    int qd = nq * dh, kvd = nkv * dh;
    float eps = c->eps;
    for (int i = 0; i < seq; i++)
        if (ids[i] < 0 || ids[i] >= c->vocab) {
            seterr(err, "token id %lld out of vocab range %d", (long long)ids[i], c->vocab);
            return -1;
        }
    float *cosG = malloc(sizeof(float) * (size_t)seq * half), *sinG = malloc(sizeof(float) * (size_t)seq * half);
    float *cosL = malloc(sizeof(float) * (size_t)seq * half), *sinL = malloc(sizeof(float) * (size_t)seq * half);
    if (arch == OR_ARCH_QWEN3 || arch == OR_ARCH_NOMIC) {
        rope_table(cosG, sinG, seq, dh, c->rope_theta);
    } else {
        rope_table(cosG, sinG, seq, dh, c->global_theta);
        rope_table(cosL, sinL, seq, dh, c->local_theta);
    }
    /* embeddings */
    if (arch == OR_ARCH_GEMMA3) {
        float es = (float)sqrt((double)H); /* gemma3.go:264-275 */
        for (int i = 0; i < seq; i++)
            for (int j = 0; j < H; j++) x[(int64_t)i * H + j] = m->word_emb[ids[i] * H + j] * es;
    } else if (arch == OR_ARCH_NOMIC) {
        for (int i = 0; i < seq; i++)
            for (int j = 0; j < H; j++) x[(int64_t)i * H + j] = m->word_emb[ids[i] * H + j] + m->type_emb[j];
        or_layernorm(x, m->emb_ln_g, m->emb_ln_b, seq, H, eps);
    } else {
        for (int i = 0; i < seq; i++) memcpy(x + (int64_t)i * H, m->word_emb + ids[i] * H, sizeof(float) * H);
        if (arch == OR_ARCH_MODERNBERT) or_layernorm(x, m->emb_ln_g, m->zero_beta, seq, H, eps);
    }
    size_t S = (size_t)seq;
    float *normed = malloc(sizeof(float) * S * H);
    float *qkv = malloc(sizeof(float) * S * (qd + 2 * kvd));
    float *qb = malloc(sizeof(float) * S * qd), *kb = malloc(sizeof(float) * S * kvd), *vb = malloc(sizeof(float) * S * kvd);
    float *kHead = malloc(sizeof(float) * (size_t)nkv * S * dh), *vHead = malloc(sizeof(float) * (size_t)nkv * S * dh);
    float *qH = malloc(sizeof(float) * S * dh), *cH = malloc(sizeof(float) * S * dh);
    float *ctx = malloc(sizeof(float) * S * qd), *tmp = malloc(sizeof(float) * S * H);
    float *gb = malloc(sizeof(float) * S * 2 * I), *ub = malloc(sizeof(float) * S * I), *act = malloc(sizeof(float) * S * I);
    float *sc = malloc(sizeof(float) * S * S);
    int bq = seq < FLASH_BLK ? seq : FLASH_BLK;
    float *sblk = malloc(sizeof(float) * bq * bq), *facc = malloc(sizeof(float) * bq * dh);
    float *mrow = malloc(sizeof(float) * bq), *lrow = malloc(sizeof(float) * bq);
    float qscale = (float)(1.0 / sqrt((double)dh));
    if (arch == OR_ARCH_GEMMA3) qscale = (float)(1.0 / sqrt((double)c->query_pre_attn_scalar));

    for (int li = 0; li < c->layers; li++) {
        dec_layer *l = &m->dl[li];
        const float *cs = cosG, *sn = sinG;
        if ((arch == OR_ARCH_MODERNBERT || arch == OR_ARCH_GEMMA3) && !l->global) {
            cs = cosL;
            sn = sinL;
        }
        if (arch == OR_ARCH_QWEN3 || arch == OR_ARCH_GEMMA3) {
            memcpy(normed, x, sizeof(float) * S * H);
            or_rmsnorm(normed, l->in_norm, seq, H, eps);
            apply_dense(&l->q, qb, normed, seq, qt);
            apply_dense(&l->k, kb, normed, seq, qt);
            apply_dense(&l->v, vb, normed, seq, qt);
            for (int kv = 0; kv < nkv; kv++) {
                float *kH = kHead + (size_t)kv * S * dh, *vH = vHead + (size_t)kv * S * dh;
                for (int i = 0; i < seq; i++) {
                    memcpy(kH + (size_t)i * dh, kb + (size_t)i * kvd + kv * dh, sizeof(float) * dh);
                    if (arch == OR_ARCH_QWEN3) {
                        memcpy(vH + (size_t)i * dh, vb + (size_t)i * kvd + kv * dh, sizeof(float) * dh);
                    } else { /* transposed V [dh x seq] (gemma3.go:292-301) */
                        for (int d = 0; d < dh; d++) vH[(size_t)d * S + i] = vb[(size_t)i * kvd + kv * dh + d];
                    }
                }
                or_rmsnorm(kH, l->k_norm, seq, dh, eps);
                apply_rope(kH, seq, dh, cs, sn);
            }
            for (int hh = 0; hh < nq; hh++) {
                for (int i = 0; i < seq; i++) memcpy(qH + (size_t)i * dh, qb + (size_t)i * qd + hh * dh, sizeof(float) * dh);
                or_rmsnorm(qH, l->q_norm, seq, dh, eps);
                apply_rope(qH, seq, dh, cs, sn);
                int kv = hh / group;
                float *kH = kHead + (size_t)kv * S * dh, *vH = vHead + (size_t)kv * S * dh;
                if (arch == OR_ARCH_QWEN3)
                    flash_attn_causal_head(qH, kH, vH, cH, seq, dh, qscale, sblk, facc, mrow, lrow);
                else
                    full_attn_head(qH, kH, vH, cH, seq, dh, qscale, l->global ? 0 : 2, c->sliding_window, sc);
                for (int i = 0; i < seq; i++) memcpy(ctx + (size_t)i * qd + hh * dh, cH + (size_t)i * dh, sizeof(float) * dh);
            }
            apply_dense(&l->o, tmp, ctx, seq, qt);
            if (arch == OR_ARCH_GEMMA3) or_rmsnorm(tmp, l->post_attn, seq, H, eps); /* gemma3.go:357-358 */
            or_add(x, tmp, seq * H);
            memcpy(normed, x, sizeof(float) * S * H);
            or_rmsnorm(normed, arch == OR_ARCH_QWEN3 ? l->post_attn : l->pre_ffn, seq, H, eps);
            apply_dense(&l->gate, gb, normed, seq, qt);
            apply_dense(&l->up, ub, normed, seq, qt);
            for (size_t i = 0; i < S * I; i++) act[i] = gb[i];
            if (arch == OR_ARCH_QWEN3)
                or_silu(act, seq * I); /* qwen3.go:530-539 */
            else
                or_gelu_tanh(act, seq * I); /* gemma3.go:365-374 */
            for (size_t i = 0; i < S * I; i++) act[i] *= ub[i];
            apply_dense(&l->down, tmp, act, seq, qt);
            if (arch == OR_ARCH_GEMMA3) or_rmsnorm(tmp, l->post_ffn, seq, H, eps);
            or_add(x, tmp, seq * H);
        } else { /* ModernBERT (pre-norm) and nomic (post-norm): fused Wqkv */
            const float *xin = x;
            if (arch == OR_ARCH_MODERNBERT) {
                memcpy(normed, x, sizeof(float) * S * H);
                if (l->in_norm) or_layernorm(normed, l->in_norm, m->zero_beta, seq, H, eps);
                xin = normed;
            }
            apply_dense(&l->qkv, qkv, xin, seq, qt);
            for (int hh = 0; hh < nq; hh++) {
                int off = hh * dh;
                float *kH = kHead, *vT = vHead;
                for (int i = 0; i < seq; i++) {
                    const float *row = qkv + (size_t)i * 3 * H;
                    memcpy(qH + (size_t)i * dh, row + off, sizeof(float) * dh);
                    memcpy(kH + (size_t)i * dh, row + H + off, sizeof(float) * dh);
                    for (int d = 0; d < dh; d++) vT[(size_t)d * S + i] = row[2 * H + off + d];
                }
                apply_rope(qH, seq, dh, cs, sn);
                apply_rope(kH, seq, dh, cs, sn);
                int wk = (arch == OR_ARCH_MODERNBERT && !l->global) ? 1 : 0;
                full_attn_head(qH, kH, vT, cH, seq, dh, qscale, wk, c->local_attention / 2, sc);
                for (int i = 0; i < seq; i++) memcpy(ctx + (size_t)i * H + off, cH + (size_t)i * dh, sizeof(float) * dh);
            }
            apply_dense(&l->o, tmp, ctx, seq, qt);
            or_add(x, tmp, seq * H);
            if (arch == OR_ARCH_NOMIC) {
                or_layernorm(x, l->n1g, l->n1b, seq, H, eps);
                apply_dense(&l->fc11, gb, x, seq, qt);
                apply_dense(&l->fc12, ub, x, seq, qt);
                for (size_t i = 0; i < S * I; i++) act[i] = ub[i];
                or_silu(act, seq * I); /* nomic.go:232-242: fc11 * silu(fc12) */
                for (size_t i = 0; i < S * I; i++) act[i] *= gb[i];
                apply_dense(&l->down, tmp, act, seq, qt);
                or_add(x, tmp, seq * H);
                or_layernorm(x, l->n2g, l->n2b, seq, H, eps);
            } else {
                memcpy(normed, x, sizeof(float) * S * H);
                or_layernorm(normed, l->mlp_norm, m->zero_beta, seq, H, eps);
                apply_dense(&l->wi, gb, normed, seq, qt);
                for (int i = 0; i < seq; i++) { /* gelu(value) * gate, modernbert.go:292-301 */
                    float *dst = act + (size_t)i * I;
                    memcpy(dst, gb + (size_t)i * 2 * I, sizeof(float) * I);
                    or_gelu(dst, I);
                    for (int d = 0; d < I; d++) dst[d] *= gb[(size_t)i * 2 * I + I + d];
                }
                apply_dense(&l->down, tmp, act, seq, qt);
                or_add(x, tmp, seq * H);
            }
        }
    }
    if (arch == OR_ARCH_QWEN3 || arch == OR_ARCH_GEMMA3)
        or_rmsnorm(x, m->final_norm, seq, H, eps);
    else if (arch == OR_ARCH_MODERNBERT)
        or_layernorm(x, m->final_norm, m->zero_beta, seq, H, eps);
    free(cosG); free(sinG); free(cosL); free(sinL);
    free(normed); free(qkv); free(qb); free(kb); free(vb); free(kHead); free(vHead); free(qH); free(cH);
    free(ctx); free(tmp); free(gb); free(ub); free(act); free(sc); free(sblk); free(facc); free(mrow); free(lrow);
    return 0;
}

/* applyGemmaDenseHead, gemma3.go:177-198: two bias-free float32 mat-vecs
 * with a plain sequential float32 sum. */
static void gemma_dense_head(const or_model *m, float *pooled) {
    int H = m->cfg.hidden, D = m->cfg.dense_hidden;
    float *hid = malloc(sizeof(float) * D);
    for (int o = 0; o < D; o++) {
        const float *row = m->dense1 + (size_t)o * H;
        float acc = 0.0f;
        for (int i = 0; i < H; i++) acc += row[i] * pooled[i];
        hid[o] = acc;
    }
    for (int o = 0; o < H; o++) {
        const float *row = m->dense2 + (size_t)o * D;
        float acc = 0.0f;
        for (int i = 0; i < D; i++) acc += row[i] * hid[i];
        pooled[o] = acc;
    }
    free(hid);
}

/* ForwardWorkers, bert.go:657-703 */
int or_forward(or_model *m, const int64_t *ids, int seq, float *pooled, float *tokens, char *err) {
    const or_config *c = &m->cfg;
    int H = c->hidden;
    if (!m->finalized) {
        seterr(err, "model not finalized");
        return -1;
    }
    if (seq == 0) { /* bert.go:742-747 */
        seterr(err, "empty token sequence");
        return -1;
    }
    if (seq > max_seq_len(m)) {
        seterr(err, "sequence length %d exceeds the model's maximum %d", seq, max_seq_len(m));
        return -1;
    }
    float *x = (float *)malloc(sizeof(float) * (size_t)seq * H);
    int rc;
    switch (c->arch) {
    case OR_ARCH_BERT:
    case OR_ARCH_DISTILBERT:
    case OR_ARCH_ROBERTA:
    case OR_ARCH_MPNET:
        rc = encode_bert(m, ids, seq, x, err);
        break;
    case OR_ARCH_QWEN3:
    case OR_ARCH_MODERNBERT:
    case OR_ARCH_GEMMA3:
    case OR_ARCH_NOMIC:
        rc = encode_decoder(m, ids, seq, x, err);
        break;
    default:
        seterr(err, "oracle: architecture %d not restated", c->arch);
        rc = -1;
    }
    if (rc == 0) {
        if (tokens) memcpy(tokens, x, sizeof(float) * (size_t)seq * H);
        if (pooled) {
            switch (c->pooling) {
            case OR_POOL_CLS:
                memcpy(pooled, x, sizeof(float) * H);
                break;
            case OR_POOL_LAST:
                memcpy(pooled, x + (int64_t)(seq - 1) * H, sizeof(float) * H);
                break;
            default: /* poolMean, bert.go:692-703 */
                for (int j = 0; j < H; j++) pooled[j] = 0.0f;
                for (int i = 0; i < seq; i++)
                    for (int j = 0; j < H; j++) pooled[j] += x[(int64_t)i * H + j];
                {
                    float inv = 1.0f / (float)seq;
                    for (int j = 0; j < H; j++) pooled[j] *= inv;
                }
            }
            if (m->dense1) gemma_dense_head(m, pooled); /* bert.go:682-684 */
            if (c->normalize) or_l2normalize(pooled, H);
        }
    }
    free(x);
    return rc;
}

/* ---- batch fan-out, rembed.go:309-331 -------------------------------- */
typedef struct {
    or_model *m;
    const int64_t *ids;
    const int32_t *cu;
    int nseq, out_kind, dim;
    float *out;
    int next; /* atomic work counter, like ParallelForCap (tensor.go:177-229) */
    int failed_index;
    char err[320];
    pthread_mutex_t mu;
} batch_job;

static void *batch_worker(void *arg) {
    batch_job *j = (batch_job *)arg;
    int H = j->m->cfg.hidden;
    float *pooled = (float *)malloc(sizeof(float) * H);
    char err[256];
    for (;;) {
        int i = __atomic_fetch_add(&j->next, 1, __ATOMIC_RELAXED);
        if (i >= j->nseq) break;
        int s0 = j->cu[i], seq = j->cu[i + 1] - j->cu[i];
        int rc;
        if (j->out_kind == 1) {
            rc = or_forward(j->m, j->ids + s0, seq, NULL, j->out + (int64_t)s0 * H, err);
        } else {
            rc = or_forward(j->m, j->ids + s0, seq, pooled, NULL, err);
            if (rc == 0) {
                /* truncate, rembed.go:441-448 */
                if (j->dim < H) or_l2normalize(pooled, j->dim);
                memcpy(j->out + (int64_t)i * j->dim, pooled, sizeof(float) * j->dim);
            }
        }
        if (rc != 0) {
            pthread_mutex_lock(&j->mu);
            if (j->failed_index < 0 || i < j->failed_index) { /* firstError: lowest index */
                j->failed_index = i;
                snprintf(j->err, sizeof j->err, "text %d: %.255s", i, err);
            }
            pthread_mutex_unlock(&j->mu);
        }
    }
    free(pooled);
    return NULL;
}

int or_embed_batch(or_model *m, const int64_t *ids, const int32_t *cu_seqlens, int nseq, int nthreads,
                   int out_kind, int dim, float *out, char *err) {
    if (nseq <= 0) return 0;
    if (dim <= 0 || dim > m->cfg.hidden) dim = m->cfg.hidden;
    batch_job j;
    memset(&j, 0, sizeof j);
    j.m = m;
    j.ids = ids;
    j.cu = cu_seqlens;
    j.nseq = nseq;
    j.out_kind = out_kind;
    j.dim = dim;
    j.out = out;
    j.failed_index = -1;
    pthread_mutex_init(&j.mu, NULL);
    int across = nthreads < nseq ? nthreads : nseq;
    if (across < 1) across = 1;
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * across);
    for (int t = 0; t < across; t++) pthread_create(&th[t], NULL, batch_worker, &j);
    for (int t = 0; t < across; t++) pthread_join(th[t], NULL);
    free(th);
    pthread_mutex_destroy(&j.mu);
    if (j.failed_index >= 0) {
        seterr(err, "%.255s", j.err);
        return -1;
    }
    return 0;
}
