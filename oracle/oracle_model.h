/* oracle_model.h — CPU restatement of tools/vq-runtime/src/model.rs forward.
 * TEST INFRASTRUCTURE ONLY (see oracle.h). */
#ifndef SPK_ORACLE_MODEL_H
#define SPK_ORACLE_MODEL_H
#include "oracle.h"

#ifdef __cplusplus
extern "C" {
#endif

/* tools/vq-runtime/src/config.rs:16-30 */
typedef struct {
    int hidden, layers, heads, kv_heads, head_dim, inter, vocab, window;
    float eps;
    float rope_theta_full, rope_partial_full, rope_theta_slide, rope_partial_slide;
    const int *full;   /* per layer: 1 = full attention, 0 = sliding window */
} orc_cfg;

/* tools/vq-runtime/src/model.rs:44-55 (borrowed f32 weights, out x in) */
typedef struct {
    const float *in_norm, *post_norm;
    const float *qkv, *attn_gate, *out, *gate, *up, *down;
} orc_layer;

typedef struct orc_model orc_model;

orc_model *orc_model_new(const orc_cfg *c, const orc_layer *layers, const float *embed, const float *norm,
                         int max_ctx, int threads);
void orc_model_free(orc_model *m);
/* model.rs:442-591: logits (vocab f32) of the token at pos. */
int orc_model_forward(orc_model *m, uint32_t token, int pos, float *logits);
int orc_model_rollback(orc_model *m, int pos);
int orc_model_capture(orc_model *m, const int *layers, int n, float *dst);
int orc_rope_dim(const orc_cfg *c, int layer);
const float *orc_model_hidden(const orc_model *m);
void orc_model_fill_kv(orc_model *m, int n, uint64_t seed);
int orc_model_kv(orc_model *m, int layer, float **k, float **v);

#ifdef __cplusplus
}
#endif
#endif
