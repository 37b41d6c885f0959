/* oracle.c — CPU restatement of the reference's decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h). Compiled with -ffp-contract=off so
 * every f32 product and sum rounds separately, as the Rust reference does.
 */
#include "oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static uint16_t u16le(const uint8_t *b, size_t o) { return (uint16_t)(b[o] | (b[o + 1] << 8)); }
static uint32_t u32le(const uint8_t *b, size_t o) {
    return (uint32_t)b[o] | ((uint32_t)b[o + 1] << 8) | ((uint32_t)b[o + 2] << 16) | ((uint32_t)b[o + 3] << 24);
}
static uint64_t u64le(const uint8_t *b, size_t o) {
    uint64_t v = 0;
    for (int k = 7; k >= 0; k--) v = (v << 8) | b[o + (size_t)k];
    return v;
}

static int fail(char *err, int errn, const char *msg) {
    if (err && errn > 0) snprintf(err, (size_t)errn, "%s", msg);
    return -1;
}

/* lib.rs:50-73: subnormals start at exponent 113 = 127 - 15 + 1. */
float orc_f16(uint16_t h) {
    const uint32_t s = ((uint32_t)h & 0x8000u) << 16;
    const uint32_t e = ((uint32_t)h >> 10) & 0x1fu;
    uint32_t m = (uint32_t)h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = s;
        } else {
            uint32_t ee = 113u;
            while ((m & 0x400u) == 0) {
                m <<= 1;
                ee -= 1;
            }
            bits = s | (ee << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (e == 31) {
        bits = s | 0x7f800000u | (m << 13);
    } else {
        bits = s | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint32_t index_bits(size_t nc) {
    uint32_t nbit = 1;
    while (((size_t)1 << nbit) < nc) nbit++;
    return nbit;
}

/* lib.rs:94-159 */
int orc_stage_open(const uint8_t *p, size_t n, orc_stage *st, char *err, int errn) {
    memset(st, 0, sizeof *st);
    const int v3 = n >= 4 && !memcmp(p, "DQV3", 4);
    if (n < 16 || (!v3 && memcmp(p, "DQVQ", 4))) return fail(err, errn, "stage payload magic is neither DQVQ nor DQV3");
    const size_t hdr = v3 ? 24 : 16;
    const size_t dim = u16le(p, 4), nc = u16le(p, 6), rows = u32le(p, 8), cols = u32le(p, 12);
    if (!dim || !nc || !rows || !cols || cols % dim) return fail(err, errn, "stage header is inconsistent");
    const size_t cb_len = nc * dim * 2, gain_len = rows * 2;
    if (n < hdr + cb_len + gain_len) return fail(err, errn, "stage payload is truncated");
    const uint32_t nbit = index_bits(nc);
    if (v3 && nbit > 13) return fail(err, errn, "DQV3 carries 13 index bits; rewrite with --format v2");
    const size_t nidx_row = cols / dim;
    size_t mrow = 0, prow = 0, idx_bytes;
    if (v3) {
        const size_t mb = nbit < 12 ? nbit : 12;
        mrow = (nidx_row * mb + 7) / 8;
        prow = nbit > 12 ? (nidx_row + 7) / 8 : 0;
        idx_bytes = rows * (mrow + prow);
    } else {
        const size_t nidx = rows * nidx_row;
        idx_bytes = nbit == 8 ? nidx : (nidx * nbit + 7) / 8 + 1;
    }
    if (n < hdr + cb_len + gain_len + idx_bytes) return fail(err, errn, "stage index stream is truncated");
    st->dim = (int)dim;
    st->nc = (int)nc;
    st->rows = (int)rows;
    st->cols = (int)cols;
    st->nbit = (int)nbit;
    st->v3 = v3;
    st->mrow = mrow;
    st->prow = prow;
    st->gains = p + hdr + cb_len;
    st->stream = p + hdr + cb_len + gain_len;
    st->stream_len = n - (hdr + cb_len + gain_len);
    st->cb32 = (float *)malloc(nc * dim * sizeof(float));
    if (!st->cb32) return fail(err, errn, "out of memory");
    for (size_t i = 0; i < nc * dim; i++) st->cb32[i] = orc_f16(u16le(p + hdr, i * 2));
    return 0;
}

void orc_stage_close(orc_stage *st) {
    free(st->cb32);
    st->cb32 = NULL;
}

static uint32_t sbyte(const orc_stage *st, size_t k) { return k < st->stream_len ? st->stream[k] : 0u; }

/* lib.rs:162-190 */
uint32_t orc_stage_index(const orc_stage *st, size_t row, size_t i) {
    if (st->v3) {
        const uint32_t mb = st->nbit < 12 ? (uint32_t)st->nbit : 12u;
        const size_t bit = i * mb;
        const size_t q = row * st->mrow + (bit >> 3);
        const uint32_t w = sbyte(st, q) | sbyte(st, q + 1) << 8 | sbyte(st, q + 2) << 16 | sbyte(st, q + 3) << 24;
        uint32_t v = (w >> (bit & 7)) & ((1u << mb) - 1u);
        if (st->prow > 0) {
            const size_t p = st->mrow * (size_t)st->rows + row * st->prow + (i >> 3);
            v |= ((sbyte(st, p) >> (i & 7)) & 1u) << 12;
        }
        return v;
    }
    const size_t gi = row * (size_t)(st->cols / st->dim) + i;
    if (st->nbit == 8) return st->stream[gi];
    const size_t bit = gi * (size_t)st->nbit;
    const uint32_t w = (uint32_t)st->stream[bit >> 3] | (uint32_t)st->stream[(bit >> 3) + 1] << 8 |
                       (uint32_t)st->stream[(bit >> 3) + 2] << 16;
    return (w >> (bit & 7)) & ((1u << st->nbit) - 1u);
}

float orc_stage_gain(const orc_stage *st, size_t row) { return orc_f16(u16le(st->gains, row * 2)); }

/* lib.rs:197-212 (rows are independent: spread over the host threads, same arithmetic per element) */
void orc_stage_add_into(const orc_stage *st, float *out) {
    const size_t nidx_row = (size_t)(st->cols / st->dim);
    long rr;
#pragma omp parallel for schedule(static)
    for (rr = 0; rr < (long)st->rows; rr++) {
        const size_t r = (size_t)rr;
        const float g = orc_stage_gain(st, r);
        float *o = out + r * (size_t)st->cols;
        for (size_t i = 0; i < nidx_row; i++) {
            const size_t v = orc_stage_index(st, r, i);
            const float *cb = st->cb32 + v * (size_t)st->dim;
            for (int d = 0; d < st->dim; d++) {
                const float t = cb[d] * g;
                o[i * (size_t)st->dim + (size_t)d] += t;
            }
        }
    }
}

/* lib.rs:215-228 */
void orc_stage_dot_row(const orc_stage *st, size_t r, const float *x, float *acc) {
    const size_t nidx_row = (size_t)(st->cols / st->dim);
    const float g = orc_stage_gain(st, r);
    float s = 0.0f;
    for (size_t i = 0; i < nidx_row; i++) {
        const size_t v = orc_stage_index(st, r, i);
        const float *cb = st->cb32 + v * (size_t)st->dim;
        for (int d = 0; d < st->dim; d++) {
            const float t = cb[d] * x[i * (size_t)st->dim + (size_t)d];
            s += t;
        }
    }
    const float t = s * g;
    acc[r] += t;
}

typedef struct {
    int dim, nc, nstages, rows, cols, v3;
    size_t per;
} orc_cont;

/* lib.rs:240-289 */
static int cont_parse(const uint8_t *buf, size_t n, orc_cont *c, char *err, int errn) {
    if (n < 32 || memcmp(buf, "RQVQ", 4)) return fail(err, errn, "not an RQVQ container");
    const size_t dim = u16le(buf, 4), nc = u16le(buf, 6), nst = u16le(buf, 8);
    const size_t rows = u32le(buf, 12), cols = u32le(buf, 16);
    const uint64_t payload = u64le(buf, 24);
    if (!dim || !nc || !nst || !rows || !cols) return fail(err, errn, "container header is inconsistent");
    const uint32_t nbit = index_bits(nc);
    const int v3 = n >= 36 && !memcmp(buf + 32, "DQV3", 4);
    if (v3 && nbit > 13) return fail(err, errn, "DQV3 carries 13 index bits; rewrite with --format v2");
    const size_t nidx_row = cols / dim;
    size_t per;
    if (v3) {
        const size_t mb = nbit < 12 ? nbit : 12;
        const size_t mrow = (nidx_row * mb + 7) / 8, prow = nbit > 12 ? (nidx_row + 7) / 8 : 0;
        per = 24 + nc * dim * 2 + rows * 2 + rows * (mrow + prow);
    } else {
        const size_t nidx = rows * nidx_row;
        per = 16 + nc * dim * 2 + rows * 2 + (nbit == 8 ? nidx : (nidx * nbit + 7) / 8 + 1);
    }
    if (payload != (uint64_t)(nst * per)) return fail(err, errn, "payload byte count disagrees with the layout");
    if (n != 32 + payload) return fail(err, errn, "file size disagrees with header and payload");
    c->dim = (int)dim;
    c->nc = (int)nc;
    c->nstages = (int)nst;
    c->rows = (int)rows;
    c->cols = (int)cols;
    c->v3 = v3;
    c->per = per;
    return 0;
}

static int cont_stage(const uint8_t *buf, const orc_cont *c, int s, orc_stage *st, char *err, int errn) {
    if (orc_stage_open(buf + 32 + (size_t)s * c->per, c->per, st, err, errn)) return -1;
    if (st->rows != c->rows || st->cols != c->cols || st->dim != c->dim || st->nc != c->nc) {
        orc_stage_close(st);
        return fail(err, errn, "stage disagrees with the container header");
    }
    return 0;
}

int orc_container_info(const uint8_t *buf, size_t n, int *dim, int *nc, int *stages, int *rows, int *cols,
                       int *v3, char *err, int errn) {
    orc_cont c;
    if (cont_parse(buf, n, &c, err, errn)) return -1;
    *dim = c.dim;
    *nc = c.nc;
    *stages = c.nstages;
    *rows = c.rows;
    *cols = c.cols;
    *v3 = c.v3;
    return 0;
}

/* lib.rs:309-316 */
int orc_container_decode(const uint8_t *buf, size_t n, float *out, char *err, int errn) {
    orc_cont c;
    if (cont_parse(buf, n, &c, err, errn)) return -1;
    long rr;
#pragma omp parallel for schedule(static)
    for (rr = 0; rr < (long)c.rows; rr++) memset(out + (size_t)rr * c.cols, 0, (size_t)c.cols * sizeof(float));
    for (int s = 0; s < c.nstages; s++) {
        orc_stage st;
        if (cont_stage(buf, &c, s, &st, err, errn)) return -1;
        orc_stage_add_into(&st, out);
        orc_stage_close(&st);
    }
    return 0;
}

/* tools/dqvq/src/main.rs:131-143 */
int orc_container_gemv_fused(const uint8_t *buf, size_t n, const float *x, float *y, int threads, char *err,
                             int errn) {
    orc_cont c;
    if (cont_parse(buf, n, &c, err, errn)) return -1;
    memset(y, 0, (size_t)c.rows * sizeof(float));
    for (int s = 0; s < c.nstages; s++) {
        orc_stage st;
        if (cont_stage(buf, &c, s, &st, err, errn)) return -1;
        long r;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
        for (r = 0; r < (long)c.rows; r++) orc_stage_dot_row(&st, (size_t)r, x, y);
        orc_stage_close(&st);
    }
    return 0;
}

/* model.rs:209-226 */
float orc_dot(const float *a, const float *b, size_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    size_t i = 0;
    while (i + 8 <= n) {
        for (int k = 0; k < 8; k++) {
            const float t = a[i + (size_t)k] * b[i + (size_t)k];
            acc[k] += t;
        }
        i += 8;
    }
    float s = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
    while (i < n) {
        const float t = a[i] * b[i];
        s += t;
        i++;
    }
    return s;
}

/* model.rs:229-234 */
void orc_matvec(const float *W, size_t rows, size_t cols, const float *x, float *y, int threads) {
    long r;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
    for (r = 0; r < (long)rows; r++) y[r] = orc_dot(W + (size_t)r * cols, x, cols);
}

/* ggml dequantize_row_q6_K: 256-weight super-block = ql[128] (low 4 bits),
 * qh[64] (high 2 bits), int8 scales[16] (one per 16 weights), f16 d.
 * Weight w = d * scale * (q - 32), evaluated as (d * scale) * q in f32. */
void orc_q6k_dequant(const uint8_t *blocks, size_t nblocks, float *out) {
    for (size_t b = 0; b < nblocks; b++) {
        const uint8_t *blk = blocks + b * 210;
        const uint8_t *ql = blk;
        const uint8_t *qh = blk + 128;
        const int8_t *sc = (const int8_t *)(blk + 192);
        const float d = orc_f16(u16le(blk, 208));
        float *y = out + b * 256;
        for (int n = 0; n < 256; n += 128) {
            for (int l = 0; l < 32; l++) {
                const int is = l / 16;
                const int q1 = (int)((ql[l + 0] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                const int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                const int q3 = (int)((ql[l + 0] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                const int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                y[l + 0] = d * (float)sc[is + 0] * (float)q1;
                y[l + 32] = d * (float)sc[is + 2] * (float)q2;
                y[l + 64] = d * (float)sc[is + 4] * (float)q3;
                y[l + 96] = d * (float)sc[is + 6] * (float)q4;
            }
            y += 128;
            ql += 64;
            qh += 32;
            sc += 8;
        }
    }
}

/* ggml dequantize_row_q8_0: 32-weight block = f16 d + int8 qs[32]; w = q * d. */
void orc_q80_dequant(const uint8_t *blocks, size_t nblocks, float *out) {
    for (size_t b = 0; b < nblocks; b++) {
        const uint8_t *blk = blocks + b * 34;
        const float d = orc_f16(u16le(blk, 0));
        const int8_t *qs = (const int8_t *)(blk + 2);
        for (int j = 0; j < 32; j++) out[b * 32 + (size_t)j] = (float)qs[j] * d;
    }
}

static void block_gemv(const uint8_t *w, size_t rows, size_t cols, const float *x, float *y, int threads,
                       int q6k) {
    const size_t per_blk = q6k ? 210 : 34, wpb = q6k ? 256 : 32;
    const size_t nb = cols / wpb, row_bytes = nb * per_blk;
    long r;
#pragma omp parallel num_threads(threads > 0 ? threads : 1)
    {
        float *tmp = (float *)malloc(cols * sizeof(float));
#pragma omp for schedule(static)
        for (r = 0; r < (long)rows; r++) {
            if (q6k)
                orc_q6k_dequant(w + (size_t)r * row_bytes, nb, tmp);
            else
                orc_q80_dequant(w + (size_t)r * row_bytes, nb, tmp);
            y[r] = orc_dot(tmp, x, cols);
        }
        free(tmp);
    }
}

void orc_q6k_gemv(const uint8_t *w, size_t rows, size_t cols, const float *x, float *y, int threads) {
    block_gemv(w, rows, cols, x, y, threads, 1);
}

void orc_q80_gemv(const uint8_t *w, size_t rows, size_t cols, const float *x, float *y, int threads) {
    block_gemv(w, rows, cols, x, y, threads, 0);
}

/* model.rs:236-245 */
void orc_rms_norm(const float *x, const float *w, float eps, size_t n, float *out) {
    double ss = 0.0;
    for (size_t i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
    const float inv = (float)(1.0 / sqrt(ss / (double)n + (double)eps));
    for (size_t i = 0; i < n; i++) {
        const float t = x[i] * inv;
        out[i] = t * w[i];
    }
}

/* model.rs:253-258 */
float orc_gelu(float x) {
    const double e = erf((double)x * 0.70710678118654752440);
    const float h = 0.5f * x;
    const float one = 1.0f + (float)e;
    return h * one;
}

/* model.rs:247-250 */
float orc_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

/* model.rs:594-604 */
uint32_t orc_argmax(const float *v, size_t n) {
    size_t best = 0;
    float bv = -INFINITY;
    for (size_t i = 0; i < n; i++)
        if (v[i] > bv) {
            bv = v[i];
            best = i;
        }
    return (uint32_t)best;
}
