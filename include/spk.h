/* spk.h — C-ABI of libspk, the B200 (sm_100a) decode hot path.
 *
 * Two families of entry points:
 *
 *  vqg_*  Drop-in for the reference's kernel ABI, tools/vq/gpu/decode-gpu.cu:765-1140,
 *         same names, argument meaning and error convention: 0 = ok, -1 = error with
 *         the message in vqg_decode_error(). `payload` is a DEVICE pointer to ONE stage
 *         (starting at its 'DQV3'/'DQVQ' magic) followed by >= 8 zeroed slack bytes;
 *         host code never dereferences it. y / out ACCUMULATE (+=). Default stream,
 *         asynchronous; the *_launch* forms never synchronize, the timed forms do.
 *         `variant` values are the reference's (0 auto, 1 generic warp, 2 dim-4 warp,
 *         3 DQV3 block) with the reference's legality rules; they select between this
 *         build's kernels, which all compute the same sum.
 *
 *  spk_*  New entry points for the rest of the path (multi-stage fused VQ GEMV,
 *         Q6_K / Q8_0 dequant-GEMV, tied head with argmax, the decode step). Same
 *         error convention; every one takes a cudaStream_t as `void *stream`
 *         (NULL = legacy default stream). All data pointers are device pointers
 *         unless a comment says otherwise.
 *
 * Errors are kept per host thread. Kernels never trap: a bounded wait that runs
 * out records an error that spk_check_device_error() reports.
 */
#ifndef SPK_H
#define SPK_H
#include <stddef.h>

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif
#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ errors, device */
/* decode-gpu.cu:23 */
const char *vqg_decode_error(void);
/* Same string as vqg_decode_error, for the spk_* entry points. */
const char *spk_last_error(void);
/* 0, or -1 if a kernel recorded a device-side error (a wait that ran out). */
int spk_check_device_error(void);
/* decode-gpu.cu:769-776 (current device instead of device 0) */
int vqg_device_name(char *out, int n);
/* decode-gpu.cu:780-784 */
int vqg_driver_version(void);

/* ----------------------------------------------- reference kernel ABI (vqg_*) */
/* decode-gpu.cu:789-798 */
int vqg_gemv_ready(int dim, int nc, int rows, int cols, int v3, int variant);
/* decode-gpu.cu:864-901 (timed: best of `iters` launches into *ms) */
int vqg_gemv_t(const void *payload, int dim, int nc, int rows, int cols, int v3, const float *x, float *y,
               int variant, int threads, int iters, double *ms);
/* decode-gpu.cu:903-906 */
int vqg_gemv(const void *payload, int dim, int nc, int rows, int cols, int v3, const float *x, float *y, int variant,
             int iters, double *ms);
/* decode-gpu.cu:911-916 (one launch, no sync) */
int vqg_gemv_launch_t(const void *payload, int dim, int nc, int rows, int cols, int v3, const float *x, float *y,
                      int variant, int threads);
/* decode-gpu.cu:918-922 */
int vqg_gemv_launch(const void *payload, int dim, int nc, int rows, int cols, int v3, const float *x, float *y,
                    int variant);
/* decode-gpu.cu:834-858 (bit-exact: out += decoded stage) */
int vqg_dequant(const void *payload, int dim, int nc, int rows, int cols, int v3, float *out, int iters, double *ms);
/* decode-gpu.cu:947-956 (bit-exact: out[cols] += decoded row) */
int vqg_row_dequant(const void *payload, int dim, int nc, int rows, int cols, int v3, int row, float *out);
/* decode-gpu.cu:1120-1138 (y += W x over an expanded f32 matrix) */
int vqg_gemv_f32(const float *w, const float *x, float *y, int rows, int cols, int iters, double *ms);

/* Prefill / verify (xT is [cols][ntok], y is [ntok][rows], y accumulates).
 * decode-gpu.cu:998-1008 */
int vqg_prefill_ready(int dim, int nc, int rows, int cols, int v3, int variant);
/* decode-gpu.cu:1012 */
int vqg_prefill_cfg_count(void);
/* decode-gpu.cu:1014-1019 */
int vqg_prefill_cfg(int idx, int *bn, int *bk);
/* decode-gpu.cu:1024-1029 */
int vqg_prefill_cfg_ready(int dim, int nc, int rows, int cols, int v3, int bn, int bk, int variant);
/* decode-gpu.cu:1034-1048 */
int vqg_prefill(const void *payload, int dim, int nc, int rows, int cols, int v3, const float *xT, int ntok, float *y,
                int iters, double *ms, int variant);
/* decode-gpu.cu:1051-1065 */
int vqg_prefill_tile(const void *payload, int dim, int nc, int rows, int cols, int v3, const float *xT, int ntok,
                     float *y, int iters, double *ms, int bn, int bk, int variant);
/* decode-gpu.cu:1071-1094 */
int vqg_prefill_launch(const void *payload, int dim, int nc, int rows, int cols, int v3, const float *xT, int ntok,
                       float *y, int variant);
/* decode-gpu.cu:1099-1118 */
int vqg_prefill_launch_tile(const void *payload, int dim, int nc, int rows, int cols, int v3, const float *xT,
                            int ntok, float *y, int bn, int bk, int variant);

/* ------------------------------------------------------------- new (spk_*) */
/* All stages of a VQ container in one pass (replaces the per-stage loop of
 * vq-model-gpu.cu:651-660 `gemv()` plus its memset).
 *   ngroups 1: y = (accumulate ? y : 0) + sum_s gain_s * W_s x
 *   ngroups 2: y = gelu_erf(W_gate x) * (W_up x), stages = {gate stages..., up stages...}
 *              (replaces the gate GEMV, up GEMV and gelu_mul_kernel, vq-model-gpu.cu:464-469, 822-826)
 * norm_w (may be NULL) folds RMSNorm(x; norm_w, eps) into the load of x
 * (replaces rmsnorm_kernel, vq-model-gpu.cu:364-377). */
int spk_vq_gemv(const void *const *stages, int nstages, int ngroups, int dim, int nc, int rows, int cols, int v3,
                const float *x, const float *norm_w, float eps, float *y, int accumulate, void *stream);
/* The same GEMV as shared-memory table look-ups (the decode step's kernel for DQV3 dim 4,
 * 4096 codes, 12-bit indices; replaces the same per-stage loop as spk_vq_gemv). Each stage is
 * re-laid once into self-contained words (spk_vq_lut_pack into spk_vq_lut_bytes device bytes,
 * 16-byte aligned; 0 = geometry not taken): its code words, its gains, and its index stream
 * slice-major, the same bytes as the payload's. spk_vq_lut_gemv then takes spk_vq_gemv's
 * arguments plus the re-laid words (group-major like stages; stages themselves may be NULL)
 * and spk_vq_lut_scratch_bytes of device scratch, zeroed before its first use (its first
 * 256 bytes are a grid barrier the kernel leaves as it found them; calls sharing a scratch
 * must not overlap on the GPU). One launch, no sync. */
size_t spk_vq_lut_bytes(int dim, int nc, int rows, int cols, int v3);
int spk_vq_lut_pack(const void *stage, int dim, int nc, int rows, int cols, int v3, void *dst, void *stream);
size_t spk_vq_lut_scratch_bytes(int ngroups, int dim, int nc, int rows, int cols, int v3);
int spk_vq_lut_gemv(const void *const *stages, const void *const *luts, int nstages, int ngroups, int dim, int nc,
                    int rows, int cols, int v3, const float *x, const float *norm_w, float eps, float *y,
                    int accumulate, void *scratch, void *stream);
/* The same with the table kernel's consumer thread count stated (0 = default; the kernel runs
 * 512 consumer threads and a producer warp), as vqg_gemv_t takes one (decode-gpu.cu:800-807). */
int spk_vq_lut_gemv_t(const void *const *stages, const void *const *luts, int nstages, int ngroups, int dim, int nc,
                      int rows, int cols, int v3, const float *x, const float *norm_w, float eps, float *y,
                      int accumulate, void *scratch, int threads, void *stream);
/* The decode step's VQ GEMV (the same contract as spk_vq_gemv, replacing the same per-stage
 * loop, vq-model-gpu.cu:651-660 over decode-gpu.cu:267-301) as shared-memory table look-ups
 * over index words whose look-up order is scheduled for the shared-memory banks: DQV3, dim 4,
 * 4096 codes, 12-bit, 1-2 stages, 1-2 groups, rows a multiple of 32 up to 10240, cols a
 * multiple of 32. Re-lay each stage once with spk_vq_tab_pack into spk_vq_tab_bytes device
 * bytes (16-byte aligned; 0 = geometry not taken): per (8-group slice, row) one 16-byte word of
 * 8 u16 table offsets. spk_vq_tab_gemv reads the code words and gains from the payloads and
 * takes spk_vq_tab_scratch_bytes of device scratch (for the device current at the call),
 * zeroed before its first use and kept for later calls: its first 256 bytes hold a grid
 * barrier's count, which every call advances; calls sharing a scratch must not overlap on the
 * GPU. One launch (the cross-CTA sums and the epilogue inside it), no sync. */
size_t spk_vq_tab_bytes(int dim, int nc, int rows, int cols, int v3);
int spk_vq_tab_pack(const void *stage, int dim, int nc, int rows, int cols, int v3, void *dst, void *stream);
size_t spk_vq_tab_scratch_bytes(int ngroups, int dim, int nc, int rows, int cols, int v3);
int spk_vq_tab_gemv(const void *const *stages, const void *const *words, int nstages, int ngroups, int dim, int nc,
                    int rows, int cols, int v3, const float *x, const float *norm_w, float eps, float *y,
                    int accumulate, void *scratch, void *stream);
/* The VQ GEMM of a token batch on the tcgen05 tensor cores, from spk_vq_lut_pack's words:
 * for n < ntok <= 128, Y[n] (=|+=) sum_s gain_s W_s RMSNorm?(X[n]) (DQV3 dim 4, 4096 codes,
 * 12-bit, 1-2 stages, cols a multiple of 32; replaces forward_batch's gemm_tiled_kernel
 * launches, vq-model-gpu.cu:858-943, decode-gpu.cu:359-501, and the verify batch's GEMMs).
 * X rows stride ldx floats, Y rows ldy; scratch: spk_vq_lut_gemm_scratch_bytes device bytes,
 * zeroed before the first call (calls leave it reusable; calls sharing one must not overlap
 * on the GPU). Two launches, no sync. */
size_t spk_vq_lut_gemm_scratch_bytes(int rows, int cols, int ntok);
int spk_vq_lut_gemm(const void *const *luts, int nstages, int dim, int nc, int rows, int cols, int v3, int ntok,
                    const float *x, int ldx, const float *norm_w, float eps, float *y, int ldy, int accumulate,
                    void *scratch, void *stream);
/* 1 if spk_vq_gemv runs the persistent TMA kernel for this geometry, 0 if the generic one. */
int spk_vq_gemv_fast_ok(int nstages, int ngroups, int dim, int nc, int rows, int cols, int v3);
/* Bit-exact stage decode on a stream: out += decoded stage (vqg_dequant without timing). */
int spk_vq_dequant(const void *payload, int dim, int nc, int rows, int cols, int v3, float *out, void *stream);

/* Q6_K / Q8_0 dequant-GEMV over raw ggml blocks (row-major, cols a multiple of the
 * block width). No reference GPU implementation: the reference serves these
 * formats through llama.cpp (tools/runtime/build-runtime.sh:181-246); the block
 * rules are ggml's, called at tools/vq/quant_err.c:35-42.
 *   y = (accumulate ? y : 0) + W RMSNorm?(x) */
int spk_q6k_gemv(const void *w, int rows, int cols, const float *x, const float *norm_w, float eps, float *y,
                 int accumulate, void *stream);
int spk_q80_gemv(const void *w, int rows, int cols, const float *x, const float *norm_w, float eps, float *y,
                 int accumulate, void *stream);
/* Tied Q8_0 head: logits = W RMSNorm(x) and the first index of the maximum into
 * *argmax_out (replaces the head GEMV + argmax_kernel, vq-model-gpu.cu:471-488, 831-833;
 * argmax rule model.rs:594-604). Allocates a small per-device workspace on first use. */
int spk_q80_head(const void *w, int rows, int cols, const float *x, const float *norm_w, float eps, float *logits,
                 int *argmax_out, void *stream);
/* The head for a verify batch: ntok <= 8 rows of x (stride ldx) in one pass over W;
 * logits [ntok][ldl], amax[ntok] the first-max index per row (model.rs:594-604; the
 * reference runs its head GEMV once per row, vq-model-gpu.cu:957-966). Allocates a small
 * per-device workspace on first use. */
int spk_q80_head_batch(const void *w, int rows, int cols, int ntok, const float *x, int ldx, const float *norm_w,
                       float eps, float *logits, int ldl, int *amax, void *stream);
/* The same head without any allocation. No counterpart in the reference. For callers
 * that cannot call cudaMalloc: code inside a CUDA-graph capture, real-time loops that
 * must not stall on an allocation, and host frameworks that own all device memory.
 * Its scratch is a fixed 8,448-byte array inside libspk (held by every GPU that loads
 * the library until exit); a launch needing more than 1024 CTAs is rejected. The first
 * call on a device looks up that array (make it before any stream capture); calls on a
 * device share the array, so calls that overlap on the GPU race: serialize them. */
int spk_q80_head_noalloc(const void *w, int rows, int cols, const float *x, const float *norm_w, float eps,
                         float *logits, int *argmax_out, void *stream);
/* Bit-exact block decode (ggml dequantize_row_q6_K / dequantize_row_q8_0). */
int spk_q6k_dequant(const void *w, size_t nblocks, float *out, void *stream);
int spk_q80_dequant(const void *w, size_t nblocks, float *out, void *stream);
/* One decoded Q8_0 row into out[cols]; row index from `row`, or from the device
 * int *token when token != NULL (replaces the embedding row of vq-model-gpu.cu:783-788). */
int spk_q80_row(const void *w, int rows, int cols, int row, const int *token, float *out, void *stream);

/* --------------------------------------------------- verify batch (M <= 8) ---
 * The speculative verify's GEMM: one pass over a VQ matrix for up to 8 tokens
 * (replaces the tiled prefill GEMM the reference runs for a draft block,
 * gemm_tiled_kernel decode-gpu.cu:359-501 via forward_batch vq-model-gpu.cu:858-943).
 * x: ntok rows of cols floats, stride ldx; y: ntok rows of rows floats, stride ldy;
 * norm_w (optional) applies RMSNorm to every x row first. */
int spk_verify_gemm(const void *const *stages, int nstages, int dim, int nc, int rows, int cols, int v3, int ntok,
                    const float *x, int ldx, const float *norm_w, float eps, float *y, int ldy, int accumulate,
                    void *stream);

/* ------------------------------------------------------- GQA attention ---
 * Decode attention over a KV cache (model.rs:508-557; the reference's attn_kernel,
 * vq-model-gpu.cu:408-461), for one token or a batch of up to 8 consecutive tokens.
 * Per token t (position *pos_dev + t): rope q and k (NeoX on the first pdim dims,
 * freq[pdim/2] = 1/theta^(2i/pdim)), and — when store is 1 (ntok 1) — write k, v into
 * the cache at slot pos % slots; with store 0 the rows must already be there (see
 * spk_attn_store). Then out[t][h] = sigmoid(gate[t][h]) * softmax(q_h K^T / sqrt(hd)) V
 * over positions [0, pos] (full) or [pos+1-window, pos] (sliding), GQA group
 * heads/kv_heads <= 4. The workspace (spk_attn_workspace_bytes, zeroed once before
 * first use) holds the split partials and merge tickets; it is left zeroed after each
 * call. */
typedef struct {
    const float *qkv;           /* [ntok][ldqkv]: q (heads*hd) | k (kv_heads*hd) | v */
    int ldqkv;
    void *k_cache, *v_cache;    /* [kv_heads][slots] rows: kv_type 0 hd f32, 1 hd f16, 2 q8_0 */
    int kv_type, slots, full, window; /* q8_0 rows: [hd int8][hd/32 f16 scales], ggml's q8_0 rule */
    const float *freq;          /* device [pdim/2] */
    int pdim, heads, kv_heads, head_dim;
    const int *pos_dev;         /* device int: position of token 0 */
    int ntok, store, nsplit;    /* nsplit 1..256 sequence splits per KV head */
    const float *gate;          /* [ntok][ldgate] pre-sigmoid */
    int ldgate;
    float *out;                 /* [ntok][ldout] */
    int ldout;
    void *workspace;
} spk_attn_args;
size_t spk_attn_workspace_bytes(int ntok, int heads, int kv_heads, int head_dim, int nsplit);
int spk_attn_decode(const spk_attn_args *a, void *stream);
int spk_attn_store(const spk_attn_args *a, void *stream);

/* --------------------------------------------------- decode step (model) ---
 * The model-level ABI the Rust host side (tools/vq-runtime/src/model.rs Model)
 * needs: forward(token, pos) -> logits / next id, rollback, reset. Weights are
 * borrowed device pointers (the caller keeps them alive); the model owns its
 * KV cache and scratch. */

/* tools/vq-runtime/src/config.rs:16-30, plus the cache capacity and dtype. */
typedef struct {
    int hidden, layers, heads, kv_heads, head_dim, inter, vocab, window;
    float eps;
    float rope_theta_full, rope_partial_full, rope_theta_slide, rope_partial_slide;
    const int *full;   /* host array [layers]: 1 = full attention, 0 = sliding window */
    int max_ctx;       /* cache capacity in positions */
    int kv_type;       /* 0: f32 K/V (the reference runtimes' cache), 1: f16, 2: q8_0 (ggml's
                        * rule per 32 values, d f16; stored planar [hd int8][hd/32 d]) */
    /* Tensor parallelism (no counterpart in the reference, which runs one GPU): this
     * model is rank tp_rank of tp_world (0 or 1: a single GPU). A rank holds q heads
     * [r*heads/t, (r+1)*heads/t), the KV heads they read (KV heads are replicated when
     * t > kv_heads), intermediate rows [r*inter/t, (r+1)*inter/t) of gate/up and the
     * matching input columns of down, and vocabulary rows [r*vocab/t, (r+1)*vocab/t)
     * of the head; the embedding table stays whole on every rank. */
    int tp_rank, tp_world;
} spk_model_config;

/* One VQ matrix: the device pointers of its stage payloads (each with >= 8 zeroed
 * slack bytes) and their geometry, as load_mat parses it (vq-model-gpu.cu:230-328). */
typedef struct {
    const void *stages[4];
    int nstages, dim, nc, rows, cols, v3;
} spk_vq_matrix;

typedef struct spk_model spk_model;
struct spk_vqprof;   /* a tuning profile, defined with its entry points below */

/* Model::new (model.rs:294-320). stream: the cudaStream_t every launch goes to. */
spk_model *spk_model_create(const spk_model_config *cfg, void *stream);
void spk_model_destroy(spk_model *m);
/* Weights::load per layer (model.rs:130-187): q_k_v_proj, g_proj, out_proj,
 * gate_proj, up_proj, down_proj and the two norms (device f32 [hidden]). */
int spk_model_set_layer(spk_model *m, int layer, const spk_vq_matrix *qkv, const spk_vq_matrix *attn_gate,
                        const spk_vq_matrix *out, const spk_vq_matrix *gate, const spk_vq_matrix *up,
                        const spk_vq_matrix *down, const float *in_norm, const float *post_norm);
/* Tied embedding / LM head as Q8_0 blocks [vocab][hidden] and model.norm.weight. */
int spk_model_set_head(spk_model *m, const void *embed_q80, const float *final_norm);
/* Model::forward (model.rs:442-591) + Model::argmax (594-604) through HOST buffers:
 * logits_host (may be NULL) receives vocab f32, *next_host the greedy id. Synchronizes. */
int spk_model_forward(spk_model *m, int token, int pos, float *logits_host, int *next_host);
/* The speculative verify (vq-model-gpu.cu:947-969 verify_logits, tools/dspark/src/
 * spec.rs:197-205): tokens[0..ntok) (ntok <= 8: the anchor and 7 proposals) at
 * positions pos..pos+ntok-1 in one batched forward; next_host[t] = greedy id after
 * tokens[t]; logits_host (may be NULL) receives [ntok][vocab]. Leaves len = pos + ntok:
 * keep the accepted prefix with spk_model_rollback(m, pos + k + 1) as spec.rs:241 does.
 * Synchronizes. */
int spk_model_verify(spk_model *m, const int *tokens, int ntok, int pos, int *next_host, float *logits_host);
/* The prompt in chunks of up to 128 tokens on the tensor cores (forward_batch + its chunk loop,
 * vq-model-gpu.cu:858-943, 1164-1168): tokens[0..n) at positions pos.., every K/V row stored;
 * the last token's greedy next id and logits (vocab floats, may be NULL) come back as
 * spk_model_forward's would. Synchronizes. */
int spk_model_prefill(spk_model *m, const int *tokens, int n, int pos, int *next_host, float *logits_host);
/* Device-resident greedy loop: set the start (token, pos) and a device int buffer
 * for the generated ids; spk_model_run then replays the captured step `steps` times
 * with no host round trip (asynchronous on the model's stream). */
int spk_model_begin(spk_model *m, int token, int pos, int *ids_dev, int ids_cap);
int spk_model_run(spk_model *m, int steps);
/* Device pointer to the last step's logits [vocab]. */
const float *spk_model_logits(spk_model *m);
/* Model::rollback (model.rs:361-382) and Model::reset (384-396). */
int spk_model_rollback(spk_model *m, int pos);
int spk_model_reset(spk_model *m);
/* Positions cached; and the host-side length bump after spk_model_run. */
int spk_model_len(spk_model *m);
int spk_model_advance_len(spk_model *m, int n);
/* Cache rows given as values (no counterpart in the reference, whose Model fills its cache
 * only through forward): positions pos0 .. pos0 + n - 1 of `layer` from device f32 rows
 * k, v [n][kv_heads * head_dim] (keys already roped), stored in the cache's type; a
 * tensor-parallel rank keeps its own KV heads. Asynchronous; record the positions with
 * spk_model_advance_len. */
int spk_model_write_kv(spk_model *m, int layer, int pos0, int n, const float *k, const float *v);

/* Per-launch device times of one decode step (no counterpart in the reference): runs
 * one step from the device state, as spk_model_run does, from a second captured graph
 * with a timing event after every launch; us[i] receives launch i's microseconds in
 * enqueue order: embedding row; per layer QKV+g_proj, attention, out_proj,
 * [tp_sum], gate+up, down, [tp_sum]; head; [tp_argmax]; advance. Returns the launch
 * count or -1. Needs one step run before; with tp_world > 1 every rank traces together. */
int spk_model_trace(spk_model *m, float *us, int cap);
/* Apply a tuning profile the caller has trusted (spk_vqprof_trust == 0), per matrix
 * geometry, as vq-model-gpu.cu:301-324 does: a gemv entry naming SPK_VARIANT_TABLE puts
 * that geometry's matrices on the table kernel (the gate/up pair only both together), any
 * other variant on the code-word kernel; an entry the kernel cannot run keeps the heuristic
 * (a line on stderr says so); geometries without an entry keep it too. NULL restores the
 * heuristic. Layers already set are re-laid and the captured step graphs are dropped (the
 * next step captures again). The profile is copied. */
int spk_model_use_profile(spk_model *m, const struct spk_vqprof *pf);
/* Which kernel the decode step runs for a layer's matrix (0 q_k_v_proj, 1 g_proj, 2 out_proj,
 * 3 gate_proj, 4 up_proj, 5 down_proj): SPK_VARIANT_TABLE for the table kernel, 3 for the
 * code-word kernel (g_proj rides with q_k_v_proj), -1 on error. */
int spk_model_kernel_of(spk_model *m, int layer, int matrix);

/* Tensor-parallel wiring (no counterpart in the reference). Each rank's model owns a
 * mailbox in device memory; the residual reductions and the head's argmax store rows
 * into every rank's mailbox over NVLink as (value, sequence) pairs and wait until every
 * rank's pairs carry the exchange's sequence, bounded by wait_ms (a wait that runs out
 * sets a device error that spk_model_forward reports).
 * spk_model_tp_handle writes the mailbox's cudaIpcMemHandle_t (n >= 64 bytes);
 * spk_model_tp_attach takes every rank's handle in rank order (n = 64 * tp_world);
 * spk_model_tp_attach_ptrs takes the mailboxes as pointers valid in this process (one
 * process driving several GPUs with peer access enabled). Attach before the first step.
 * With tp_world > 1, spk_model_logits is this rank's vocabulary shard; spk_model_forward
 * gathers the whole vocabulary when logits_host is not NULL. */
int spk_model_tp_handle(spk_model *m, void *handle_out, int n);
int spk_model_tp_attach(spk_model *m, const void *handles, int n, int wait_ms);
int spk_model_tp_attach_ptrs(spk_model *m, void *const *mailboxes, int world, int wait_ms);
/* This rank's mailbox pointer (for spk_model_tp_attach_ptrs). */
void *spk_model_tp_mailbox(spk_model *m);

/* Model::enable_capture / captured (model.rs:322-348): from the next step on, the residual
 * entering each listed layer is written at every position the decode step and the verify
 * batch visit, into device memory [n][max_ctx][hidden] (slot k of position p at
 * spk_model_captures(m, &stride)[k * stride + p * hidden]). At most 8 layers; n = 0 turns
 * capture off. Rollback needs no action: later positions are rewritten when revisited. */
int spk_model_enable_capture(spk_model *m, const int *layers, int n);
const float *spk_model_captures(spk_model *m, size_t *slot_stride);
/* The head's table re-laid for the tensor-core head (spk_q80_tile layout; this rank's
 * vocabulary rows), made by spk_model_set_head; NULL when the geometry is not tiled. */
const void *spk_model_head_tiled(spk_model *m);
/* Kernels one decode step launches (known after the first spk_model_forward / run step;
 * 0 before it). */
int spk_model_step_launches(const spk_model *m);

/* ------------------------------------------------ DSpark draft (row D) ---
 * The draft executor of tools/dspark/src/draft.rs (encode_features 567-628,
 * decode_block 641-901), replacing the reference's GPU executor (dspark-gpu.h:914-1152:
 * cuBLAS SGEMM on f32-expanded weights, a host sync per Markov row). BF16 weights are
 * borrowed device pointers, row-major out x in (the manifest's GGUF shapes read as
 * [ne1][ne0]); f32 vectors; NULL marks an absent optional tensor. */
#define SPK_DRAFT_MAX_LAYERS 32

/* The manifest header (tools/dspark/src/manifest.rs:84-110) plus the cache capacity. */
typedef struct {
    int hidden, layers, heads, kv_heads, head_dim, ffn, vocab, mask_token;
    int rope_full_dims, rope_swa_dims;
    float rope_full_theta, rope_swa_theta, eps;
    int act;          /* 0: gelu (ggml's tanh form), 1: silu */
    int swa_window, causal, block_size, sample_from_anchor;
    int n_target;     /* target capture layers the encoder concatenates (fc: [hidden][n_target*hidden]) */
    int rank;         /* Markov rank (markov_w1/w2 [vocab][rank]); 0 = no Markov head */
    int max_ctx;      /* draft cache positions */
    int swa_pattern[SPK_DRAFT_MAX_LAYERS];   /* per layer: 1 = sliding-window rope */
} spk_draft_config;

/* draft.rs:243-259 DraftLayer. Optional: gate, q_norm/k_norm (used together, as the
 * reference does), attn_post, ffn_post; out_scale 0 = none. */
typedef struct {
    const void *q, *k, *v, *gate, *out, *ffn_gate, *ffn_up, *ffn_down;   /* bf16 */
    const float *norm, *q_norm, *k_norm, *ffn_norm, *attn_post, *ffn_post;
    float out_scale;
} spk_draft_layer;

/* draft.rs:261-272 globals. conf_proj is f32 [hidden + rank], or NULL. */
typedef struct {
    const void *fc;                      /* bf16 [hidden][n_target * hidden] */
    const float *fc_norm;                /* [n_target][hidden] */
    const float *enc_norm, *out_norm;
    const void *markov_w1, *markov_w2;   /* bf16 [vocab][rank] */
    const float *conf_proj;
    float conf_bias;
} spk_draft_globals;

typedef struct spk_draft spk_draft;

/* Draft::open's device state: the injected K/V cache and scratch, on the current device. */
spk_draft *spk_draft_create(const spk_draft_config *cfg, void *stream);
void spk_draft_destroy(spk_draft *d);
int spk_draft_set_layer(spk_draft *d, int layer, const spk_draft_layer *w);
int spk_draft_set_globals(spk_draft *d, const spk_draft_globals *g);
/* encode_features for the committed positions [p0, p1) from the target's layer-input
 * captures (device; slot k of position p at caps[k * slot_stride + p * hidden]). */
int spk_draft_encode(spk_draft *d, const float *caps, size_t slot_stride, int p0, int p1);
/* decode_block over the target's Q8_0 embedding [vocab][hidden] (device): ids (host,
 * n_block) get the greedy argmax of every block row after the Markov bias, conf (host,
 * optional) the confidence head (NaN where the reference leaves it). Returns n_block
 * (n_draft with sample_from_anchor and a Markov head, else n_draft + 1) or -1.
 * The injected window before pos0 must be encoded. Synchronizes the draft's stream. */
int spk_draft_block(spk_draft *d, const void *embed, int vocab, int anchor, int pos0, int n_draft, int *ids,
                    float *conf);
/* The block's head from the target's tiled table (spk_model_head_tiled, all vocabulary rows)
 * instead of the ggml blocks; NULL reverts. */
int spk_draft_set_head_tiled(spk_draft *d, const void *tiled);
/* The last block's biased logits, [n_block][vocab] f32 on device. */
const float *spk_draft_logits(const spk_draft *d);

/* The tied Q8_0 head in a tensor-core tile layout (no counterpart in the reference; it
 * replaces the reference's per-row head GEMV over the same ggml blocks). spk_q80_tile
 * re-lays a ggml Q8_0 matrix into [rows/16][cols/32] tile-blocks of 544 bytes (the 16 rows'
 * 32 int8 in mma.sync fragment order, then their 16 f16 scales) in spk_q80_tile_bytes bytes;
 * spk_q80_tile_head computes logits[n*ldl + r] = (W RMSNorm?(x[n*ldx ..]))[r] for ntok <= 8
 * rows and, when amax is not NULL, the first-max argmax per row. rows % 16 == 0, cols a
 * multiple of 32 in [256, 4096]; scratch is spk_q80_tile_scratch_bytes() device bytes, zeroed
 * once and left zeroed; calls sharing a scratch must not overlap on the GPU. */
size_t spk_q80_tile_bytes(int rows, int cols);
int spk_q80_tile(const void *w, int rows, int cols, void *dst, void *stream);
size_t spk_q80_tile_scratch_bytes(void);
int spk_q80_tile_head(const void *wt, int rows, int cols, int ntok, const float *x, int ldx, const float *norm_w,
                      float eps, float *logits, int ldl, int *amax, void *scratch, void *stream);

/* The draft's skinny BF16 GEMM (dspark-gpu.h:897-907 draft_gemm): y[n*ldy + r] (=, or +=)
 * (W x[n*ldx ..])[r] for n < ntok <= 8; W bf16 [rows][cols], 16-byte aligned, cols % 32 == 0. */
int spk_bf16_gemm(const void *w, int rows, int cols, int ntok, const float *x, int ldx, float *y, int ldy,
                  int accumulate, void *stream);
/* The FFN pair y = act(G x) * (U x), act 0 = gelu (tanh form), 1 = silu (draft.rs:838-855). */
int spk_bf16_gemm_pair(const void *gate, const void *up, int rows, int cols, int ntok, const float *x, int ldx,
                       float *y, int ldy, int act, void *stream);

/* ------------------------------------------------------- tuning profiles */
/* VQPROF 1 per-artifact tuning profiles (tools/vq/gpu/vq-profile.h:1-40, the format;
 * tools/vq-tune/src/profile.rs, the writer; vq-model-gpu.cu:1094-1122 and :301-324, how the
 * reference runtime trusts and applies one). Host memory throughout; no device work.
 *
 * GEMV variants a profile entry can name for this build's kernels: 0-3 as vqg_gemv takes
 * them (the model runs them all as the code-word kernel, vq.cu, which falls back to the
 * generic kernel where its geometry rules fail), and SPK_VARIANT_TABLE, the shared-memory
 * table kernel over re-laid words (vq_tab.cu). `threads` and the prefill tile (bn, bk) are
 * recorded and written back but this build's kernels fix their own launch shapes. */
#define SPK_VQPROF_VERSION 1
#define SPK_VQPROF_MAX 512
#define SPK_VARIANT_TABLE 4
typedef struct {
    int kind;                   /* 0 = gemv, 1 = prefill */
    int dim, nc, rows, cols, v3;
    int variant;
    int threads;                /* gemv */
    int bn, bk;                 /* prefill */
    double rate;                /* the trailing measured rate: GB/s (gemv), tok/s (prefill) */
} spk_vqprof_entry;
typedef struct spk_vqprof {
    unsigned long long artifact;   /* the fingerprint the profile was tuned on */
    char gpu[128];                 /* device name, matched literally */
    char driver[64];
    int version;                   /* the VQPROF line's number */
    int n;
    spk_vqprof_entry e[SPK_VQPROF_MAX];
} spk_vqprof;
/* vq-profile.h:114-140 (vqprof_artifact): FNV-1a 64 over dir/manifest.txt, then per matrix
 * line `name rows cols stages bytes relL2` with stages > 0, in file order: the name, the size
 * of dir/name.bin as 8 LE bytes, its first and last min(4096, size) bytes. */
int spk_vqprof_fingerprint(const char *dir, unsigned long long *out);
/* vq-profile.h:152-187 (vqprof_load): 0 when the file parsed and says VQPROF 1 (pf holds
 * what was read either way), -1 otherwise. Unknown lines are skipped; at most
 * SPK_VQPROF_MAX entries are kept. */
int spk_vqprof_load(const char *path, spk_vqprof *pf);
/* vq-profile.h:189-197 (vqprof_find): the index of the first entry of that kind and
 * geometry, or -1. */
int spk_vqprof_find(const spk_vqprof *pf, int kind, int dim, int nc, int rows, int cols, int v3);
/* The runtime's gate (vq-model-gpu.cu:1101-1121): 0 = trusted; 1 = tuned on another
 * artifact; 2 = tuned on another device (names compared literally); 3 = not version 1. */
int spk_vqprof_trust(const spk_vqprof *pf, unsigned long long artifact, const char *device);
/* profile.rs render + write_atomic: the text through path.tmp and a rename. */
int spk_vqprof_write(const char *path, const spk_vqprof *pf);

#ifdef __cplusplus
}
#endif
#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#endif
