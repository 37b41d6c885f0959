/* draft.c — CPU restatement of the DSpark draft executor.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h). Follows tools/dspark/src/draft.rs:
 * dot (74-92, = orc_dot), mm (94-101), rms_mul (103-110, = orc_rms_norm),
 * sigmoid (122-125), rope_head (129-143), rope_for/rope_vec (548-565),
 * encode_features (567-628), decode_block (641-901), gelu_tanh (905-911),
 * silu (913-916), argmax (917-928), mm_embed (931-940).
 *
 * The reference re-encodes every committed position each round; the encoding of a
 * position depends only on that position's captures, so encoding [p0, p1) once and
 * keeping the result is the same computation. The shared-KV form (a layer without
 * attn_v) has no encode path in the reference and is not restated.
 */
#include "oracle_draft.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

struct orc_draft {
    orc_draft_cfg c;
    orc_draft_layer *L;
    orc_draft_globals g;
    int *swa;
    int max_ctx, threads;
    float *inj_k, *inj_v;   /* [layers][max_ctx][kv_dim], roped K and V of encoded positions */
    int enc_lo, enc_hi;     /* positions [enc_lo, enc_hi) hold encodings */
};

static void *xcalloc(size_t n, size_t s) { return calloc(n ? n : 1, s); }

static float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

/* draft.rs:905-911 */
static float gelu_tanh(float x) {
    const float A = 0.044715f, S = 0.7978846f;
    return 0.5f * x * (1.0f + tanhf(S * x * (1.0f + A * x * x)));
}

/* draft.rs:913-916 */
static float silu(float x) { return x * sigmoidf_(x); }

/* draft.rs:917-928: first maximum, strict > from -inf */
static uint32_t argmax_(const float *x, size_t n) {
    size_t best = 0;
    float bv = -INFINITY;
    for (size_t i = 0; i < n; i++)
        if (x[i] > bv) {
            bv = x[i];
            best = i;
        }
    return (uint32_t)best;
}

/* draft.rs:129-143 */
static void rope_head(float *x, int pos, float theta, int dim) {
    const int half = dim / 2;
    for (int i = 0; i < half; i++) {
        const float freq = 1.0f / powf(theta, (float)(2 * i) / (float)dim);
        const float a = (float)pos * freq;
        const float c = cosf(a), s = sinf(a);
        const float lo = x[i], hi = x[i + half];
        const float t0 = lo * c, t1 = hi * s, t2 = hi * c, t3 = lo * s;
        x[i] = t0 - t1;
        x[i + half] = t2 + t3;
    }
}

/* draft.rs:548-565 */
static void rope_for(const orc_draft *d, int layer, int *nrot, float *theta) {
    if (d->swa[layer]) {
        *nrot = d->c.rope_swa_dims;
        *theta = d->c.rope_swa_theta;
    } else {
        *nrot = d->c.rope_full_dims;
        *theta = d->c.rope_full_theta;
    }
}

static void rope_vec(float *v, int heads, int hd, int pos, int nrot, float theta) {
    const int dim = nrot < hd ? nrot : hd;
    for (int h = 0; h < heads; h++) rope_head(v + (size_t)h * hd, pos, theta, dim);
}

int orc_draft_block_rows(const orc_draft_cfg *c, int has_markov, int n_draft) {
    if (has_markov) return c->sample_from_anchor ? n_draft : n_draft + 1;
    return n_draft + 1;
}

orc_draft *orc_draft_new(const orc_draft_cfg *c, const orc_draft_layer *layers, const orc_draft_globals *g,
                         int max_ctx, int threads) {
    if (!c || !layers || !g || c->layers < 1 || max_ctx < 1) return NULL;
    orc_draft *d = (orc_draft *)xcalloc(1, sizeof *d);
    if (!d) return NULL;
    d->c = *c;
    d->L = (orc_draft_layer *)xcalloc((size_t)c->layers, sizeof(orc_draft_layer));
    d->swa = (int *)xcalloc((size_t)c->layers, sizeof(int));
    memcpy(d->L, layers, (size_t)c->layers * sizeof(orc_draft_layer));
    for (int l = 0; l < c->layers; l++) d->swa[l] = c->swa_pattern ? c->swa_pattern[l] : 0;
    d->c.swa_pattern = d->swa;
    d->g = *g;
    d->max_ctx = max_ctx;
    d->threads = threads > 0 ? threads : 1;
    const size_t kvd = (size_t)c->kv_heads * c->head_dim;
    d->inj_k = (float *)xcalloc((size_t)c->layers * (size_t)max_ctx * kvd, sizeof(float));
    d->inj_v = (float *)xcalloc((size_t)c->layers * (size_t)max_ctx * kvd, sizeof(float));
    if (!d->inj_k || !d->inj_v) {
        orc_draft_free(d);
        return NULL;
    }
    return d;
}

void orc_draft_free(orc_draft *d) {
    if (!d) return;
    free(d->L);
    free(d->swa);
    free(d->inj_k);
    free(d->inj_v);
    free(d);
}

/* draft.rs:567-628 */
int orc_draft_encode(orc_draft *d, const float *caps, size_t slot_stride, int p0, int p1) {
    const orc_draft_cfg *c = &d->c;
    if (p0 < 0 || p1 < p0 || p1 > d->max_ctx) return -1;
    if (p1 == p0) return 0;
    const int h = c->hidden, nt = c->n_target, hd = c->head_dim;
    const size_t kvd = (size_t)c->kv_heads * hd;
    float *concat = (float *)xcalloc((size_t)nt * h, sizeof(float));
    float *fused = (float *)xcalloc((size_t)h, sizeof(float));
    float *gp = (float *)xcalloc((size_t)h, sizeof(float));
    float *tmp = (float *)xcalloc((size_t)hd, sizeof(float));
    for (int p = p0; p < p1; p++) {
        for (int k = 0; k < nt; k++)
            orc_rms_norm(caps + (size_t)k * slot_stride + (size_t)p * h, d->g.fc_norm + (size_t)k * h, c->eps,
                         (size_t)h, concat + (size_t)k * h);
        orc_matvec(d->g.fc, (size_t)h, (size_t)nt * h, concat, fused, d->threads);
        orc_rms_norm(fused, d->g.enc_norm, c->eps, (size_t)h, gp);
        for (int li = 0; li < c->layers; li++) {
            const orc_draft_layer *L = &d->L[li];
            int nrot;
            float theta;
            rope_for(d, li, &nrot, &theta);
            float *kv = d->inj_k + ((size_t)li * d->max_ctx + p) * kvd;
            float *vv = d->inj_v + ((size_t)li * d->max_ctx + p) * kvd;
            orc_matvec(L->k, kvd, (size_t)h, gp, kv, d->threads);
            orc_matvec(L->v, kvd, (size_t)h, gp, vv, d->threads);
            if (L->k_norm)
                for (int cc = 0; cc < c->kv_heads; cc++) {
                    orc_rms_norm(kv + (size_t)cc * hd, L->k_norm, c->eps, (size_t)hd, tmp);
                    memcpy(kv + (size_t)cc * hd, tmp, (size_t)hd * sizeof(float));
                }
            rope_vec(kv, c->kv_heads, hd, p, nrot, theta);
        }
    }
    free(concat);
    free(fused);
    free(gp);
    free(tmp);
    /* valid range: [p0, p1) joined to the earlier one when they touch; positions past p1
     * were encoded before a rollback and are stale */
    if (d->enc_hi <= d->enc_lo || p0 > d->enc_hi || p1 < d->enc_lo) d->enc_lo = p0;
    else if (p0 < d->enc_lo) d->enc_lo = p0;
    d->enc_hi = p1;
    return 0;
}

/* draft.rs:641-901 */
int orc_draft_decode_block(orc_draft *d, const float *embed, int vocab, uint32_t anchor, int pos0, int n_draft,
                           float *logits, float *conf, uint32_t *amax) {
    const orc_draft_cfg *c = &d->c;
    const int is_dspark = d->g.markov_w1 != NULL && d->g.markov_w2 != NULL;
    const int anchor_mode = c->sample_from_anchor;
    const int n_block = orc_draft_block_rows(c, is_dspark, n_draft);
    if (n_draft == 0 || n_draft > c->block_size) return -1;
    if (n_block > c->block_size + 1) return -1;
    if (vocab < c->vocab) return -1;
    if (pos0 < 0 || pos0 + n_block > d->max_ctx) return -1;
    const int h = c->hidden, hd = c->head_dim, heads = c->heads, kvh = c->kv_heads;
    const size_t qdim = (size_t)heads * hd, kvd = (size_t)kvh * hd;
    const float scale = 1.0f / sqrtf((float)hd);
    const long nswa = is_dspark ? (long)c->swa_window + 1 : (long)c->swa_window;
    /* the keys the reference keeps from its injection (positions 0..pos0-1) must be encoded */
    const long inj_lo = (long)pos0 - nswa + 1 > 0 ? (long)pos0 - nswa + 1 : 0;
    if (inj_lo < pos0 && (inj_lo < d->enc_lo || pos0 > d->enc_hi)) return -1;

    uint32_t *tokens = (uint32_t *)xcalloc((size_t)n_block, sizeof(uint32_t));
    for (int i = 0; i < n_block; i++) tokens[i] = i == 0 ? anchor : (uint32_t)c->mask_token;
    for (int i = 0; i < n_block; i++)
        if ((int)tokens[i] >= vocab) {
            free(tokens);
            return -1;
        }
    const size_t nb = (size_t)n_block;
    float *x = (float *)xcalloc(nb * h, sizeof(float));
    float *nx = (float *)xcalloc(nb * h, sizeof(float));
    float *q = (float *)xcalloc(nb * qdim, sizeof(float));
    float *ok = (float *)xcalloc(nb * kvd, sizeof(float));
    float *ov = (float *)xcalloc(nb * kvd, sizeof(float));
    float *xn = (float *)xcalloc((size_t)h, sizeof(float));
    float *tmp = (float *)xcalloc((size_t)(h > hd ? h : hd), sizeof(float));
    float *gate_row = (float *)xcalloc((size_t)heads, sizeof(float));
    float *attn = (float *)xcalloc(qdim, sizeof(float));
    float *out = (float *)xcalloc((size_t)h, sizeof(float));
    float *up = (float *)xcalloc((size_t)c->ffn, sizeof(float));
    float *gt = (float *)xcalloc((size_t)c->ffn, sizeof(float));
    float *act = (float *)xcalloc((size_t)c->ffn, sizeof(float));
    float *down = (float *)xcalloc((size_t)h, sizeof(float));
    const size_t maxkeys = (size_t)(pos0 - inj_lo) + nb;
    const float **kk = (const float **)xcalloc(maxkeys, sizeof(float *));
    const float **vk = (const float **)xcalloc(maxkeys, sizeof(float *));
    float *sc = (float *)xcalloc(maxkeys, sizeof(float));
    float *o = (float *)xcalloc((size_t)hd, sizeof(float));
    int rc = n_block;

    for (int i = 0; i < n_block; i++) memcpy(x + (size_t)i * h, embed + (size_t)tokens[i] * h, (size_t)h * sizeof(float));
    for (int li = 0; li < c->layers && rc > 0; li++) {
        const orc_draft_layer *L = &d->L[li];
        int nrot;
        float theta;
        rope_for(d, li, &nrot, &theta);
        for (int i = 0; i < n_block; i++) {
            float *qi = q + (size_t)i * qdim, *ki = ok + (size_t)i * kvd, *vi = ov + (size_t)i * kvd;
            orc_rms_norm(x + (size_t)i * h, L->norm, c->eps, (size_t)h, xn);
            orc_matvec(L->q, qdim, (size_t)h, xn, qi, d->threads);
            orc_matvec(L->k, kvd, (size_t)h, xn, ki, d->threads);
            orc_matvec(L->v, kvd, (size_t)h, xn, vi, d->threads);
            if (L->q_norm && L->k_norm) {
                for (int cc = 0; cc < heads; cc++) {
                    orc_rms_norm(qi + (size_t)cc * hd, L->q_norm, c->eps, (size_t)hd, tmp);
                    memcpy(qi + (size_t)cc * hd, tmp, (size_t)hd * sizeof(float));
                }
                for (int cc = 0; cc < kvh; cc++) {
                    orc_rms_norm(ki + (size_t)cc * hd, L->k_norm, c->eps, (size_t)hd, tmp);
                    memcpy(ki + (size_t)cc * hd, tmp, (size_t)hd * sizeof(float));
                }
            }
            rope_vec(qi, heads, hd, pos0 + i, nrot, theta);
            rope_vec(ki, kvh, hd, pos0 + i, nrot, theta);
        }
        /* every query uses the anchor row's mask (draft.rs:772-795): injected keys first,
         * in position order, then the block's own rows */
        const long p1 = pos0;
        size_t nk = 0;
        for (long p = inj_lo; p < pos0; p++) {
            const int keep = (!c->causal || p <= p1) && (p1 - p < nswa);
            if (keep) {
                kk[nk] = d->inj_k + ((size_t)li * d->max_ctx + (size_t)p) * kvd;
                vk[nk] = d->inj_v + ((size_t)li * d->max_ctx + (size_t)p) * kvd;
                nk++;
            }
        }
        for (int i = 0; i < n_block; i++) {
            const long p = pos0 + i;
            const int keep = (!c->causal || p <= p1) && (p1 - p < nswa);
            if (keep) {
                kk[nk] = ok + (size_t)i * kvd;
                vk[nk] = ov + (size_t)i * kvd;
                nk++;
            }
        }
        if (nk == 0) {
            rc = -1;
            break;
        }
        for (int i = 0; i < n_block; i++) {
            orc_rms_norm(x + (size_t)i * h, L->norm, c->eps, (size_t)h, xn);
            if (L->gate) orc_matvec(L->gate, (size_t)heads, (size_t)h, xn, gate_row, d->threads);
            const float *qi = q + (size_t)i * qdim;
            for (int hh = 0; hh < heads; hh++) {
                const int group = hh * kvh / heads;
                const float *qh = qi + (size_t)hh * hd;
                float mx = -INFINITY;
                for (size_t j = 0; j < nk; j++) {
                    sc[j] = orc_dot(qh, kk[j] + (size_t)group * hd, (size_t)hd) * scale;
                    mx = fmaxf(mx, sc[j]);
                }
                float sum = 0.0f;
                for (size_t j = 0; j < nk; j++) {
                    sc[j] = expf(sc[j] - mx);
                    sum += sc[j];
                }
                const float inv = 1.0f / sum;
                memset(o, 0, (size_t)hd * sizeof(float));
                for (size_t j = 0; j < nk; j++) {
                    const float p = sc[j] * inv;
                    const float *vh = vk[j] + (size_t)group * hd;
                    for (int e = 0; e < hd; e++) {
                        const float t = p * vh[e];
                        o[e] += t;
                    }
                }
                if (L->gate) {
                    const float g = sigmoidf_(gate_row[hh]);
                    for (int e = 0; e < hd; e++) o[e] *= g;
                }
                memcpy(attn + (size_t)hh * hd, o, (size_t)hd * sizeof(float));
            }
            orc_matvec(L->out, (size_t)h, qdim, attn, out, d->threads);
            if (L->attn_post) {
                orc_rms_norm(out, L->attn_post, c->eps, (size_t)h, tmp);
                memcpy(out, tmp, (size_t)h * sizeof(float));
            }
            float *res = nx + (size_t)i * h;
            for (int k2 = 0; k2 < h; k2++) res[k2] = x[(size_t)i * h + k2] + out[k2];
            orc_rms_norm(res, L->ffn_norm, c->eps, (size_t)h, xn);
            orc_matvec(L->ffn_up, (size_t)c->ffn, (size_t)h, xn, up, d->threads);
            orc_matvec(L->ffn_gate, (size_t)c->ffn, (size_t)h, xn, gt, d->threads);
            for (int k2 = 0; k2 < c->ffn; k2++) act[k2] = (c->act == 1 ? silu(gt[k2]) : gelu_tanh(gt[k2])) * up[k2];
            orc_matvec(L->ffn_down, (size_t)h, (size_t)c->ffn, act, down, d->threads);
            for (int k2 = 0; k2 < h; k2++) res[k2] += down[k2];
            if (L->ffn_post) {
                orc_rms_norm(res, L->ffn_post, c->eps, (size_t)h, tmp);
                memcpy(res, tmp, (size_t)h * sizeof(float));
            }
            if (L->out_scale != 0.0f)
                for (int k2 = 0; k2 < h; k2++) res[k2] *= L->out_scale;
        }
        memcpy(x, nx, nb * h * sizeof(float));
    }

    if (rc > 0) {
        float *hid = nx;   /* reuse: hid[i] = rms_mul(x[i], out_norm) */
        for (int i = 0; i < n_block; i++) orc_rms_norm(x + (size_t)i * h, d->g.out_norm, c->eps, (size_t)h, hid + (size_t)i * h);
        for (int i = 0; i < n_block; i++) {
            orc_matvec(embed, (size_t)vocab, (size_t)h, hid + (size_t)i * h, logits + (size_t)i * vocab, d->threads);
            conf[i] = NAN;
        }
        if (is_dspark) {
            const int rank = d->g.rank;
            const int i_beg = anchor_mode ? 0 : 1;
            uint32_t prev = anchor;
            float *bias = (float *)xcalloc((size_t)vocab, sizeof(float));
            float *feat = (float *)xcalloc((size_t)(h + rank), sizeof(float));
            if (!anchor_mode) conf[0] = d->g.conf_proj ? sigmoidf_(logits[0]) : NAN;
            const int vmax = vocab < c->vocab ? vocab : c->vocab;
            for (int i = i_beg; i < n_block; i++) {
                const float *w1p = d->g.markov_w1 + (size_t)prev * rank;
                orc_matvec(d->g.markov_w2, (size_t)c->vocab, (size_t)rank, w1p, bias, d->threads);
                float *li = logits + (size_t)i * vocab;
                for (int t = 0; t < vmax; t++) li[t] += bias[t];
                if (d->g.conf_proj) {
                    memcpy(feat, hid + (size_t)i * h, (size_t)h * sizeof(float));
                    memcpy(feat + h, w1p, (size_t)rank * sizeof(float));
                    float cv = orc_dot(d->g.conf_proj, feat, (size_t)(h + rank));
                    cv += d->g.conf_bias;
                    conf[i] = sigmoidf_(cv);
                }
                if (i + 1 < n_block) prev = argmax_(li, (size_t)vocab);
            }
            free(bias);
            free(feat);
        }
        for (int i = 0; i < n_block; i++) amax[i] = argmax_(logits + (size_t)i * vocab, (size_t)vocab);
    }
    free(tokens);
    free(x);
    free(nx);
    free(q);
    free(ok);
    free(ov);
    free(xn);
    free(tmp);
    free(gate_row);
    free(attn);
    free(out);
    free(up);
    free(gt);
    free(act);
    free(down);
    free(kk);
    free(vk);
    free(sc);
    free(o);
    return rc;
}
