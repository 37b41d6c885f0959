/* oracle_draft.h — CPU restatement of the DSpark draft executor
 * (tools/dspark/src/draft.rs: encode_features 567-628, decode_block 641-901).
 * TEST INFRASTRUCTURE ONLY (see oracle.h). */
#ifndef SPK_ORACLE_DRAFT_H
#define SPK_ORACLE_DRAFT_H
#include "oracle.h"

#ifdef __cplusplus
extern "C" {
#endif

/* The manifest header fields the executor reads (tools/dspark/src/manifest.rs:84-110). */
typedef struct {
    int hidden, layers, heads, kv_heads, head_dim, ffn, vocab, mask_token;
    int rope_full_dims, rope_swa_dims;
    float rope_full_theta, rope_swa_theta, eps;
    int act;                 /* 0: gelu (ggml's tanh form), 1: silu */
    int swa_window, causal, block_size, sample_from_anchor;
    int n_target;            /* number of target capture layers (fc input = n_target * hidden) */
    const int *swa_pattern;  /* per layer: 1 = sliding window */
} orc_draft_cfg;

/* draft.rs:243-259 (DraftLayer), f32 weights row-major out x in (as Mat holds them).
 * Optional tensors are NULL; out_scale 0 means none (draft.rs:368-373). */
typedef struct {
    const float *norm, *q, *k, *v, *gate, *out, *q_norm, *k_norm;
    const float *ffn_norm, *ffn_gate, *ffn_up, *ffn_down, *attn_post, *ffn_post;
    float out_scale;
} orc_draft_layer;

/* draft.rs:261-272 (Draft globals). markov_w1/w2 are [vocab][rank]; conf_proj is
 * [hidden + rank]. */
typedef struct {
    const float *fc, *fc_norm, *enc_norm, *out_norm;
    const float *markov_w1, *markov_w2, *conf_proj;
    float conf_bias;
    int rank;
} orc_draft_globals;

typedef struct orc_draft orc_draft;

orc_draft *orc_draft_new(const orc_draft_cfg *c, const orc_draft_layer *layers, const orc_draft_globals *g,
                         int max_ctx, int threads);
void orc_draft_free(orc_draft *d);

/* encode_features (draft.rs:567-628) for the positions [p0, p1): caps holds the target's
 * layer-input rows, slot k of position p at caps[k * slot_stride + p * hidden]. The injected
 * K/V of those positions replace whatever was stored there. 0, or -1 on a bad range. */
int orc_draft_encode(orc_draft *d, const float *caps, size_t slot_stride, int p0, int p1);

/* decode_block (draft.rs:641-901) over the f32 target embedding [vocab][hidden]. Writes
 * n_block rows of logits [n_block][vocab], conf [n_block] and argmax [n_block]; returns
 * n_block, or -1 on an argument the reference refuses (its error cases). */
int orc_draft_decode_block(orc_draft *d, const float *embed, int vocab, uint32_t anchor, int pos0, int n_draft,
                           float *logits, float *conf, uint32_t *argmax);

/* The block row count decode_block uses for n_draft (draft.rs:652-660). */
int orc_draft_block_rows(const orc_draft_cfg *c, int has_markov, int n_draft);

#ifdef __cplusplus
}
#endif
#endif
