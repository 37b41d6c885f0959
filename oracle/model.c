/* model.c — CPU restatement of the reference's f32 decode step.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h). Follows
 * tools/vq-runtime/src/model.rs:442-591 (Model::forward) line for line:
 * f64 RMSNorm sums, f32 powf rope table (model.rs:416-429), NeoX rotate-half
 * (431-439), f32 KV cache position-major [layer][pos][kv_dim] (499-506),
 * sliding start pos+1-window (508-512), per-head softmax attention with the
 * sigmoid gate (519-553), erf-GELU(gate) * up (570-574), tied head (585-589).
 * Weights are f32 row-major out x in, as Weights::from_vq expands them.
 */
#include "oracle_model.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

struct orc_model {
    orc_cfg c;
    orc_layer *L;
    const float *embed, *norm;
    int max_ctx, threads;
    float *kv_k, *kv_v;   /* [layers][max_ctx][kv_dim] */
    float *h, *xn, *qkv, *gate, *attn, *o, *g, *u, *act, *cos, *sin;
    int *full;
    int *cap_slot;   /* per layer: capture slot or -1 (model.rs:322-343) */
    float *cap;      /* [slots][max_ctx][hidden] */
};

static void *xcalloc(size_t n, size_t s) { return calloc(n ? n : 1, s); }

orc_model *orc_model_new(const orc_cfg *c, const orc_layer *layers, const float *embed, const float *norm,
                         int max_ctx, int threads) {
    orc_model *m = (orc_model *)xcalloc(1, sizeof *m);
    if (!m) return NULL;
    m->c = *c;
    m->L = (orc_layer *)xcalloc((size_t)c->layers, sizeof(orc_layer));
    m->full = (int *)xcalloc((size_t)c->layers, sizeof(int));
    memcpy(m->L, layers, (size_t)c->layers * sizeof(orc_layer));
    memcpy(m->full, c->full, (size_t)c->layers * sizeof(int));
    m->c.full = m->full;
    m->cap_slot = (int *)xcalloc((size_t)c->layers, sizeof(int));
    for (int l = 0; l < c->layers; l++) m->cap_slot[l] = -1;
    m->embed = embed;
    m->norm = norm;
    m->max_ctx = max_ctx;
    m->threads = threads > 0 ? threads : 1;
    const size_t qd = (size_t)c->heads * c->head_dim, kvd = (size_t)c->kv_heads * c->head_dim;
    m->kv_k = (float *)xcalloc((size_t)c->layers * (size_t)max_ctx * kvd, sizeof(float));
    m->kv_v = (float *)xcalloc((size_t)c->layers * (size_t)max_ctx * kvd, sizeof(float));
    m->h = (float *)xcalloc((size_t)c->hidden, sizeof(float));
    m->xn = (float *)xcalloc((size_t)c->hidden, sizeof(float));
    m->qkv = (float *)xcalloc(qd + 2 * kvd, sizeof(float));
    m->gate = (float *)xcalloc((size_t)c->heads, sizeof(float));
    m->attn = (float *)xcalloc(qd, sizeof(float));
    m->o = (float *)xcalloc((size_t)c->hidden, sizeof(float));
    m->g = (float *)xcalloc((size_t)c->inter, sizeof(float));
    m->u = (float *)xcalloc((size_t)c->inter, sizeof(float));
    m->act = (float *)xcalloc((size_t)c->inter, sizeof(float));
    m->cos = (float *)xcalloc((size_t)c->head_dim, sizeof(float));
    m->sin = (float *)xcalloc((size_t)c->head_dim, sizeof(float));
    if (!m->kv_k || !m->kv_v) {
        orc_model_free(m);
        return NULL;
    }
    return m;
}

void orc_model_free(orc_model *m) {
    if (!m) return;
    free(m->L);
    free(m->full);
    free(m->cap_slot);
    free(m->kv_k);
    free(m->kv_v);
    free(m->h);
    free(m->xn);
    free(m->qkv);
    free(m->gate);
    free(m->attn);
    free(m->o);
    free(m->g);
    free(m->u);
    free(m->act);
    free(m->cos);
    free(m->sin);
    free(m);
}

int orc_rope_dim(const orc_cfg *c, int layer) {
    const float partial = c->full[layer] ? c->rope_partial_full : c->rope_partial_slide;
    int dim = (int)((float)c->head_dim * partial);
    return dim < c->head_dim ? dim : c->head_dim;
}

/* model.rs:416-429 */
static void rope_table(orc_model *m, int pos, int layer) {
    const orc_cfg *c = &m->c;
    const float theta = c->full[layer] ? c->rope_theta_full : c->rope_theta_slide;
    const int dim = orc_rope_dim(c, layer), half = dim / 2;
    for (int i = 0; i < half; i++) {
        const float freq = 1.0f / powf(theta, (float)(2 * i) / (float)dim);
        const float a = (float)pos * freq;
        m->cos[i] = cosf(a);
        m->cos[i + half] = cosf(a);
        m->sin[i] = sinf(a);
        m->sin[i + half] = sinf(a);
    }
}

/* model.rs:431-439 */
static void apply_rope(float *x, const float *cs, const float *sn, int dim) {
    const int half = dim / 2;
    for (int i = 0; i < half; i++) {
        const float a = x[i], b = x[i + half];
        const float t0 = a * cs[i], t1 = b * sn[i];
        const float t2 = b * cs[i + half], t3 = a * sn[i + half];
        x[i] = t0 - t1;
        x[i + half] = t2 + t3;
    }
}

int orc_model_forward(orc_model *m, uint32_t token, int pos, float *logits) {
    const orc_cfg *c = &m->c;
    if ((int)token >= c->vocab || pos < 0 || pos >= m->max_ctx) return -1;
    const int hidden = c->hidden, hd = c->head_dim;
    const size_t qd = (size_t)c->heads * hd, kvd = (size_t)c->kv_heads * hd;
    const float scale = 1.0f / sqrtf((float)hd);
    const int threads = m->threads;

    memcpy(m->h, m->embed + (size_t)token * hidden, (size_t)hidden * sizeof(float));
    for (int li = 0; li < c->layers; li++) {
        const orc_layer *L = &m->L[li];
        /* the residual entering the layer (model.rs:466-472) */
        if (m->cap && m->cap_slot[li] >= 0)
            memcpy(m->cap + ((size_t)m->cap_slot[li] * m->max_ctx + (size_t)pos) * hidden, m->h,
                   (size_t)hidden * sizeof(float));
        rope_table(m, pos, li);
        orc_rms_norm(m->h, L->in_norm, c->eps, (size_t)hidden, m->xn);
        orc_matvec(L->qkv, qd + 2 * kvd, (size_t)hidden, m->xn, m->qkv, threads);
        orc_matvec(L->attn_gate, (size_t)c->heads, (size_t)hidden, m->xn, m->gate, threads);
        const int dim = orc_rope_dim(c, li);
        for (int h = 0; h < c->heads; h++) apply_rope(m->qkv + (size_t)h * hd, m->cos, m->sin, dim);
        for (int h = 0; h < c->kv_heads; h++) apply_rope(m->qkv + qd + (size_t)h * hd, m->cos, m->sin, dim);

        float *kc = m->kv_k + (size_t)li * m->max_ctx * kvd, *vc = m->kv_v + (size_t)li * m->max_ctx * kvd;
        memcpy(kc + (size_t)pos * kvd, m->qkv + qd, kvd * sizeof(float));
        memcpy(vc + (size_t)pos * kvd, m->qkv + qd + kvd, kvd * sizeof(float));

        const int start = c->full[li] ? 0 : (pos + 1 > c->window ? pos + 1 - c->window : 0);
        const int n = pos + 1 - start;
        int h;
#pragma omp parallel for schedule(static) num_threads(threads)
        for (h = 0; h < c->heads; h++) {
            const int kvh = h * c->kv_heads / c->heads;
            const float *q = m->qkv + (size_t)h * hd;
            float *sc = (float *)malloc((size_t)n * sizeof(float));
            for (int j = 0; j < n; j++) {
                const size_t o = (size_t)(start + j) * kvd + (size_t)kvh * hd;
                sc[j] = orc_dot(q, kc + o, (size_t)hd) * scale;
            }
            float mx = -INFINITY;
            for (int j = 0; j < n; j++) mx = fmaxf(mx, sc[j]);
            float sum = 0.0f;
            for (int j = 0; j < n; j++) {
                sc[j] = expf(sc[j] - mx);
                sum += sc[j];
            }
            const float inv = 1.0f / sum;
            float *o = m->attn + (size_t)h * hd;
            for (int d = 0; d < hd; d++) o[d] = 0.0f;
            for (int j = 0; j < n; j++) {
                const float p = sc[j] * inv;
                const float *vb = vc + (size_t)(start + j) * kvd + (size_t)kvh * hd;
                for (int d = 0; d < hd; d++) {
                    const float t = p * vb[d];
                    o[d] += t;
                }
            }
            const float g = orc_sigmoid(m->gate[h]);
            for (int d = 0; d < hd; d++) o[d] *= g;
            free(sc);
        }
        orc_matvec(L->out, (size_t)hidden, qd, m->attn, m->o, threads);
        for (int i = 0; i < hidden; i++) m->h[i] += m->o[i];

        orc_rms_norm(m->h, L->post_norm, c->eps, (size_t)hidden, m->xn);
        orc_matvec(L->gate, (size_t)c->inter, (size_t)hidden, m->xn, m->g, threads);
        orc_matvec(L->up, (size_t)c->inter, (size_t)hidden, m->xn, m->u, threads);
        for (int i = 0; i < c->inter; i++) m->act[i] = orc_gelu(m->g[i]) * m->u[i];
        orc_matvec(L->down, (size_t)hidden, (size_t)c->inter, m->act, m->o, threads);
        for (int i = 0; i < hidden; i++) m->h[i] += m->o[i];
    }
    orc_rms_norm(m->h, m->norm, c->eps, (size_t)hidden, m->xn);
    orc_matvec(m->embed, (size_t)c->vocab, (size_t)hidden, m->xn, logits, threads);
    return 0;
}

/* model.rs:361-382 — positions >= pos are simply overwritten later. */
/* model.rs:322-343: layer-input capture for the listed layers into dst [n][max_ctx][hidden]
 * (caller-owned); -1 on a layer outside the model or listed twice. */
int orc_model_capture(orc_model *m, const int *layers, int n, float *dst) {
    for (int l = 0; l < m->c.layers; l++) m->cap_slot[l] = -1;
    m->cap = NULL;
    for (int k = 0; k < n; k++) {
        if (layers[k] < 0 || layers[k] >= m->c.layers || m->cap_slot[layers[k]] >= 0) {
            for (int l = 0; l < m->c.layers; l++) m->cap_slot[l] = -1;
            return -1;
        }
        m->cap_slot[layers[k]] = k;
    }
    m->cap = n > 0 ? dst : NULL;
    return 0;
}

int orc_model_rollback(orc_model *m, int pos) { return (pos < 0 || pos > m->max_ctx) ? -1 : 0; }

/* The K and V caches of one layer, [max_ctx][kv_dim] f32 each (position-major, as
 * model.rs:398-412 keeps them), for tests that give a device cache the same rows. */
int orc_model_kv(orc_model *m, int layer, float **k, float **v) {
    if (layer < 0 || layer >= m->c.layers) return -1;
    const size_t kvd = (size_t)m->c.kv_heads * m->c.head_dim;
    *k = m->kv_k + (size_t)layer * m->max_ctx * kvd;
    *v = m->kv_v + (size_t)layer * m->max_ctx * kvd;
    return 0;
}

/* The hidden state entering the final norm, for debugging parity. */
const float *orc_model_hidden(const orc_model *m) { return m->h; }

/* Fill the first n positions of every layer's K/V cache with seeded values
 * (splitmix-style hash -> uniform [-1, 1)), so a CPU-baseline sample can time a
 * step at a long context without first running the whole prompt on the CPU. */
void orc_model_fill_kv(orc_model *m, int n, uint64_t seed) {
    const orc_cfg *c = &m->c;
    const size_t kvd = (size_t)c->kv_heads * c->head_dim;
    if (n > m->max_ctx) n = m->max_ctx;
    for (int li = 0; li < c->layers; li++) {
        float *kc = m->kv_k + (size_t)li * m->max_ctx * kvd, *vc = m->kv_v + (size_t)li * m->max_ctx * kvd;
        for (size_t i = 0; i < (size_t)n * kvd; i++) {
            uint64_t z = seed + (uint64_t)li * 0x9E3779B97F4A7C15ull + i * 0xBF58476D1CE4E5B9ull;
            z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
            z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
            z ^= z >> 31;
            kc[i] = (float)((double)(z >> 11) * (1.0 / 4503599627370496.0)) - 1.0f;
            vc[i] = (float)((double)((z * 0x2545F4914F6CDD1Dull) >> 11) * (1.0 / 4503599627370496.0)) - 1.0f;
        }
    }
}
