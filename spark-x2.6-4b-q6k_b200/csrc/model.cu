// model.cu — the batch-1 decode step of the Spark2_5 decoder on B200, and its C-ABI.
//
// What it computes is tools/vq-runtime/src/model.rs:442-591 (Model::forward):
//   h = embed[token]
//   per layer:  xn = rmsnorm(h); qkv = W_qkv xn; g = W_g xn; rope(q, k); kv[pos] = (k, v)
//               a_h = softmax(q_h K^T / sqrt(hd)) V * sigmoid(g_h)   (GQA, sliding or full)
//               h += W_out a;  xn = rmsnorm(h);  h += W_down (gelu_erf(W_gate xn) * W_up xn)
//   logits = W_embed rmsnorm(h); next = argmax(logits)
// The launches per layer (the reference issues ~218 launches and one host sync
// per token, vq-model-gpu.cu:776-835):
//   1. QKV and g_proj GEMVs in one launch, RMSNorm prologue (vq.cu, persistent TMA kernel)
//   2. attention: rope, KV store, split-K flash-decode over the cache, the splits
//      merged and the sigmoid gate applied by the last CTA (attn.cu)
//   3. out_proj GEMV accumulating into h
//   4. gate+up GEMV pair with RMSNorm prologue and erf-GELU(gate)*up epilogue
//   5. down GEMV accumulating into h
// then the tied Q8_0 head with fused argmax (ggml.cu) and a one-thread advance
// kernel (pos += 1, token = argmax). Token and position live in device memory,
// so the whole step is captured once in a CUDA graph and replayed per token.
//
// Tensor parallel (tp_world t > 1): a rank runs the same launches over its shards
// (q heads / KV heads, intermediate rows, vocabulary rows); out_proj and down_proj
// write a partial residual that tp_sum (tp.cu) reduces over all ranks into the
// replicated h, and tp_argmax picks the greedy id over the vocabulary shards.
#include <math.h>
#include <stdio.h>
#include <stdlib.h>

#include <vector>

#include "attn.cuh"
#include "common.cuh"
#include "spk.h"
#include "tp.cuh"
#include "vq_mma.cuh"

using namespace spk;

namespace {

// With SPK_TRACE_ERRORS set, the first model entry point that finds a CUDA error pending
// (one an earlier call left behind without reporting it) says where; a diagnostic only.
void trace_pending(const char *where, int arg = -1) {
    static const bool on = getenv("SPK_TRACE_ERRORS") != nullptr;
    static int said = 0;
    if (!on || said >= 3) return;
    const cudaError_t e = cudaPeekAtLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "[spk] CUDA error pending at %s (%d): %s\n", where, arg, cudaGetErrorString(e));
        said++;
    }
}

// End of a step: record the generated id, feed it back as the next token, advance.
struct DevCtl {
    int *ids;   // where spk_model_run records generated ids (may be null)
    int cap;
};

// The residual rows entering a layer (ntok rows of h) into its capture slot at positions
// *pos + t (model.rs:466-472, the layer-input rows the draft encoder reads).
__global__ void capture_kernel(const float *h, int H, int ntok, const int *pos, float *dst) {
    pdl_trigger();
    pdl_wait();
    const size_t p = (size_t)*pos;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ntok * H; i += gridDim.x * blockDim.x) {
        const int t = i / H;
        dst[(p + t) * H + (i - t * H)] = h[i];
    }
}

__global__ void advance_kernel(int *pos, int *token, const int *argmax, const DevCtl *ctl, int *step) {
    pdl_trigger();
    pdl_wait();
    const int s = *step;
    if (ctl->ids && s < ctl->cap) ctl->ids[s] = *argmax;
    *token = *argmax;
    *pos = *pos + 1;
    *step = s + 1;
}

__global__ void set_state_kernel(int *pos, int *token, int p, int t) {
    *pos = p;
    *token = t;
}

}  // namespace

// ================================================================ host ===
struct spk_model {
    spk_model_config cfg;
    std::vector<int> full;
    struct Layer {
        spk_vq_matrix m[6];   // qkv, attn_gate, out, gate, up, down
        const float *in_norm = nullptr, *post_norm = nullptr;
        bool set = false;
        // the stages' index streams re-laid for the decode step's table kernel (vq_lut.cu),
        // one allocation per matrix; null: the matrix runs the code-word kernel (vq.cu)
        void *lut_mem[6] = {};
        const void *lut[6][4] = {};
        bool dec[6] = {};     // the decode step runs this matrix through the table kernel
        void *tab_mem[6] = {};   // its index streams re-laid for that kernel (vq_tab.cu)
        const void *tab[6][4] = {};
    };
    std::vector<Layer> layers;
    const void *embed = nullptr;
    const float *final_norm = nullptr;
    int q_dim = 0, kv_dim = 0, G = 0, pdim_full = 0, pdim_slide = 0, nsplit_full = 1, nsplit_slide = 1;
    // tensor parallel: local head counts, intermediate rows, vocabulary shard
    int tp_rank = 0, tp_world = 1, hl = 0, kvl = 0, inter_l = 0, vocab_l = 0, row0 = 0;
    void *mailbox = nullptr;      // this rank's exchange mailbox (+ flags + logits shard when t > 1)
    size_t mail_flags_off = 0, mail_logits_off = 0;
    int mail_stride = 0;
    void *peer_open[TP_MAX] = {};   // IPC mappings to close
    const float *peer_logits[TP_MAX] = {};
    float *pbuf = nullptr, *logits_full = nullptr, *gbuf = nullptr;
    int *vtok = nullptr;                 // verify batch tokens (device)
    cudaGraphExec_t vexec[ATT_MAX_TOK + 1] = {};   // captured verify steps, by batch size
    cudaGraph_t vgraph[ATT_MAX_TOK + 1] = {};
    int veager[ATT_MAX_TOK + 1] = {};
    unsigned int *att_count = nullptr;   // attention merge tickets [ATT_MAX_TOK][kv heads]
    unsigned int *tp_seq = nullptr;
    TpView tpv = {};
    bool tp_ready = false;
    float *h = nullptr, *qkv = nullptr, *gate = nullptr, *attn = nullptr, *act = nullptr, *logits = nullptr,
          *part = nullptr, *freq_full = nullptr, *freq_slide = nullptr;
    void *kc = nullptr, *vc = nullptr;
    std::vector<size_t> kv_off;   // per layer byte offset into kc / vc
    std::vector<int> kv_slots;
    int *state = nullptr;         // device: pos, token, argmax, step, local argmax; [8..16) verify ids, [16..24) local
    DevCtl *ctl = nullptr;        // device: id buffer of spk_model_run
    DevCtl *host_ctl = nullptr;   // pinned staging for it
    unsigned long long *head_partial = nullptr;
    unsigned int *head_counter = nullptr;
    int step_launches = 0;        // kernels one decode step launches (counted while enqueuing it)
    void *tab_scr = nullptr;      // the decode table kernel's grid-barrier count and per-CTA partials (vq_tab.cu)
    size_t tab_scr_size = 0;
    void *tc_scr = nullptr;       // the batched tensor-core GEMM's scratch (vq_tc.cu), zeroed once
    size_t tc_scr_size = 0;
    // the prompt path (spk_model_prefill): rows for a chunk of up to PF_MAX tokens, made on first use
    float *pf_h = nullptr, *pf_qkv = nullptr, *pf_gate = nullptr, *pf_attn = nullptr, *pf_act = nullptr,
          *pf_g = nullptr;
    int *pf_tok = nullptr, *pf_pos = nullptr, *pf_host = nullptr;
    void *pf_scr = nullptr;
    void *head_tiled = nullptr;   // this rank's head rows re-laid for the tensor-core head (q8t.cu)
    void *head_tiled_scratch = nullptr;
    unsigned long long *vhead_partial = nullptr;   // the verify batch's head
    unsigned int *vhead_counter = nullptr;
    int *host_io = nullptr;       // pinned: pos, token, argmax; [8..16) verify tokens, [16..24) verify ids
    cudaStream_t stream = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    // spk_model_trace: a second capture of the step with a timing event after every launch
    std::vector<cudaEvent_t> tev;
    int tracing = 0, nmark = 0;
    int nmark_all = 0, step_marks = 0;   // marks an enqueued step makes (counted traced or not)
    int capturing = 0;            // enqueue_step is being captured into a step graph
    cudaGraph_t tgraph = nullptr;
    cudaGraphExec_t texec = nullptr;
    int eager_steps = 0;
    int len = 0;                  // positions cached (host view, for rollback checks)
    std::vector<int> cap_slot;    // per layer: capture slot or -1
    std::vector<spk_vqprof_entry> prof;   // spk_model_use_profile's gemv entries (empty: heuristics)
    float *cap = nullptr;         // [ncap][max_ctx][hidden]
    int ncap = 0;
};

namespace {

int vq_call(const spk_vq_matrix &M, int ngroups, const spk_vq_matrix *M2, const float *x, const float *norm_w,
            float eps, float *y, int accumulate, cudaStream_t s) {
    const void *st[8];
    for (int i = 0; i < M.nstages; i++) st[i] = M.stages[i];
    if (M2)
        for (int i = 0; i < M2->nstages; i++) st[M.nstages + i] = M2->stages[i];
    return spk_vq_gemv(st, M.nstages, ngroups, M.dim, M.nc, M.rows, M.cols, M.v3, x, norm_w, eps, y, accumulate, s);
}

// q_k_v_proj and g_proj (same input, same encoding) as one launch when the
// encodings agree, else two.
int qkv_gate(const spk_model::Layer &L, const float *h, float eps, float *qkv, float *gate, cudaStream_t s) {
    const spk_vq_matrix &Q = L.m[0], &G = L.m[1];
    if (Q.nstages == G.nstages && Q.nstages <= 2) {
        const Layout LQ = make_layout(Q.dim, Q.nc, Q.rows, Q.cols, Q.v3), LG = make_layout(G.dim, G.nc, G.rows, G.cols, G.v3);
        const int rc = vq_gemv_with_extra(Q.stages, Q.nstages, LQ, G.stages, LG, h, L.in_norm, eps, qkv, gate, 0, s);
        if (rc <= 0) return rc;
    }
    if (vq_call(Q, 1, nullptr, h, L.in_norm, eps, qkv, 0, s)) return -1;
    return vq_call(G, 1, nullptr, h, L.in_norm, eps, gate, 0, s);
}


// Layer matrix mi (with mi2, the up_proj of a pair) through the table kernel when it
// was re-laid for it: 0 launched, 1 not taken, -1 error. For q_k_v_proj, g_proj rides
// along (the kernel's last CTAs).
int lut_call(spk_model *m, const spk_model::Layer &L, int mi, int mi2, const float *x, const float *norm_w, float eps,
             float *y, int accumulate, float *xy, cudaStream_t s) {
    const spk_vq_matrix &M = L.m[mi];
    if (!L.dec[mi] || (mi2 >= 0 && !L.dec[mi2])) return 1;
    const void *st[8], *lt[8];
    for (int q = 0; q < M.nstages; q++) st[q] = M.stages[q], lt[q] = L.tab[mi][q];
    if (mi2 >= 0)
        for (int q = 0; q < M.nstages; q++) st[M.nstages + q] = L.m[mi2].stages[q], lt[M.nstages + q] = L.tab[mi2][q];
    const Layout LM = make_layout(M.dim, M.nc, M.rows, M.cols, M.v3);
    const spk_vq_matrix &G = L.m[1];
    Layout LG;
    const bool extra = xy && G.nstages == M.nstages && G.dim == M.dim && G.nc == M.nc && G.v3 == M.v3 && G.rows <= 64;
    if (xy && !extra) return 1;
    if (extra) LG = make_layout(G.dim, G.nc, G.rows, G.cols, G.v3);
    return tab::gemv(st, lt, M.nstages, mi2 >= 0 ? 2 : 1, LM, x, norm_w, eps, y, accumulate, m->tab_scr,
                    extra ? G.stages : nullptr, extra ? &LG : nullptr, extra ? xy : nullptr, s) ? -1 : 0;
}

// The attention arguments of layer li for a batch of ntok tokens starting at the
// device position (buffers [ntok][...]: qkv, gate, attn).
AttnArgs attn_args(spk_model *m, int li, int ntok) {
    const spk_model_config &c = m->cfg;
    AttnArgs a;
    memset(&a, 0, sizeof a);
    a.qkv = m->qkv;
    a.ldqkv = m->q_dim + 2 * m->kv_dim;
    a.kc = (uint8_t *)m->kc + m->kv_off[li];
    a.vc = (uint8_t *)m->vc + m->kv_off[li];
    a.kv_type = c.kv_type;
    a.slots = m->kv_slots[li];
    a.full = m->full[li];
    a.window = c.window;
    a.freq = a.full ? m->freq_full : m->freq_slide;
    a.pdim = a.full ? m->pdim_full : m->pdim_slide;
    a.heads = m->hl;
    a.kv_heads = m->kvl;
    a.hd = c.head_dim;
    a.pos = m->state;
    a.ntok = ntok;
    a.nsplit = a.full ? m->nsplit_full : m->nsplit_slide;
    a.part = m->part;
    a.count = m->att_count;
    a.gate = m->gate;
    a.ldgate = m->hl;
    a.out = m->attn;
    a.ldout = m->q_dim;
    a.err = device_error_ptr();
    return a;
}

// Layer li's input rows into its capture slot, when capture is on (no trace mark: the
// copy is counted with the launch after it).
int capture_rows(spk_model *m, int li, int ntok, cudaStream_t s, const float *h = nullptr, const int *pos = nullptr) {
    if (!m->ncap || m->cap_slot[li] < 0) return 0;
    const int H = m->cfg.hidden;
    float *dst = m->cap + (size_t)m->cap_slot[li] * m->cfg.max_ctx * H;
    cudaError_t e = launch_pdl(capture_kernel, dim3((ntok * H + 255) / 256), dim3(256), 0, s, h ? h : (const float *)m->h,
                               H, ntok, pos ? pos : (const int *)m->state, dst);
    return e == cudaSuccess ? 0 : cuda_fail("layer capture launch", e);
}

// Under spk_model_trace's capture: an event after the launch just enqueued.
int mark(spk_model *m) {
    m->nmark_all++;
    if (!m->tracing) return 0;
    if (m->nmark >= (int)m->tev.size()) return set_error("trace: more launches than events");
    cudaError_t e = cudaEventRecordWithFlags(m->tev[m->nmark++], m->stream, cudaEventRecordExternal);
    return e == cudaSuccess ? 0 : cuda_fail("trace event", e);
}

// out_proj / down_proj (matrix mi) into the residual: at N = 1 accumulated into h; under
// tensor parallelism the code-word kernel with the residual exchange fused in (one launch,
// vq_gemv_tp), else this rank's partial into pbuf and tp_sum. *nl counts the launches.
int residual_gemv(spk_model *m, const spk_model::Layer &L, int mi, const float *x, cudaStream_t s, int *nl) {
    const spk_model_config &c = m->cfg;
    const bool tp = m->tp_world > 1;
    if (tp && !L.dec[mi]) {   // (a profile that puts this matrix on the table kernel: lut_call + tp_sum)
        const spk_vq_matrix &M = L.m[mi];
        const Layout LM = make_layout(M.dim, M.nc, M.rows, M.cols, M.v3);
        const int rc = vq_gemv_tp(M.stages, M.nstages, LM, x, m->h, m->tpv, s);
        if (rc < 0) return -1;
        if (rc == 0) {
            *nl += 1;
            return mark(m);
        }
    }
    float *const ro = tp ? m->pbuf : m->h;   // rank partial, or the residual
    const int lr = lut_call(m, L, mi, -1, x, nullptr, 0.f, ro, tp ? 0 : 1, nullptr, s);
    if (lr < 0 || (lr == 1 && vq_call(L.m[mi], 1, nullptr, x, nullptr, 0.f, ro, tp ? 0 : 1, s)) || mark(m))
        return -1;
    *nl += 1;
    if (tp) {
        if (tp_sum(m->tpv, m->pbuf, m->h, c.hidden, s) || mark(m)) return -1;
        *nl += 1;
    }
    return 0;
}

// Enqueue one decode step on m->stream: reads pos/token from m->state.
int enqueue_step(spk_model *m) {
    const spk_model_config &c = m->cfg;
    cudaStream_t s = m->stream;
    int *pos = m->state, *token = m->state + 1, *amax = m->state + 2, *amax_l = m->state + 4;
    const bool tp = m->tp_world > 1;
    m->nmark_all = 0;
    if (mark(m) || spk_q80_row(m->embed, c.vocab, c.hidden, 0, token, m->h, s) || mark(m)) return -1;
    // embedding row, head, advance; per layer attention plus one launch per GEMV (and a
    // tensor-parallel exchange launch where it is not fused into the GEMV), plus the
    // vocabulary argmax
    int nl = 3 + (tp ? 1 : 0);
    for (int li = 0; li < c.layers; li++) {
        const spk_model::Layer &L = m->layers[li];
        if (capture_rows(m, li, 1, s)) return -1;
        nl += (m->ncap && m->cap_slot[li] >= 0) + 1;
        int lr = lut_call(m, L, 0, -1, m->h, L.in_norm, c.eps, m->qkv, 0, m->gate, s);
        if (lr < 0 || (lr == 1 && qkv_gate(L, m->h, c.eps, m->qkv, m->gate, s)) || mark(m)) return -1;
        nl += 1;
        AttnArgs a = attn_args(m, li, 1);
        a.store = 1;
        a.cached_before = m->capturing;   // a graph replay: every earlier step has completed
        if (attn_decode(a, s) || mark(m)) return -1;
        if (residual_gemv(m, L, 2, m->attn, s, &nl)) return -1;
        lr = lut_call(m, L, 3, 4, m->h, L.post_norm, c.eps, m->act, 0, nullptr, s);
        if (lr < 0 || (lr == 1 && vq_call(L.m[3], 2, &L.m[4], m->h, L.post_norm, c.eps, m->act, 0, s)) || mark(m))
            return -1;
        nl += 1;
        if (residual_gemv(m, L, 5, m->act, s, &nl)) return -1;
    }
    const uint8_t *head_rows = (const uint8_t *)m->embed + (size_t)m->row0 * (c.hidden / 32) * 34;
    const int ht = m->head_tiled ? q8t_head_launch(m->head_tiled, m->vocab_l, c.hidden, 1, m->h, c.hidden,
                                                   m->final_norm, c.eps, m->logits, m->vocab_l, tp ? amax_l : amax,
                                                   m->head_tiled_scratch, s)
                                 : 0;
    if (ht < 0) return -1;
    if (ht == 0 && q80_head_launch(head_rows, m->vocab_l, c.hidden, m->h, m->final_norm, c.eps, m->logits,
                                   tp ? amax_l : amax, m->head_partial, m->head_counter, s))
        return -1;
    if (mark(m)) return -1;
    if (tp && (tp_argmax(m->tpv, m->logits, m->vocab_l, amax_l, m->row0, amax, 1, s) || mark(m))) return -1;
    cudaError_t e = launch_pdl(advance_kernel, dim3(1), dim3(1), 0, s, pos, token, (const int *)amax,
                               (const DevCtl *)m->ctl, m->state + 3);
    if (e != cudaSuccess) return cuda_fail("decode step launch", e);
    m->step_launches = nl;
    if (mark(m)) return -1;
    m->step_marks = m->nmark_all;
    return 0;
}

// ---------------------------------------------------------- verify batch ---
// Layer matrix mi for a batch of ntok token rows on the tcgen05 GEMM over its re-laid words
// (vq_tc.cu): 0 launched, 1 not taken, -1 error.
int tc_call(spk_model *m, const spk_model::Layer &L, int mi, int ntok, const float *x, int ldx, const float *norm_w,
            float eps, float *y, int ldy, int accumulate, int mode, const float *aux, cudaStream_t s) {
    const spk_vq_matrix &M = L.m[mi];
    if (!L.lut[mi][0] || !m->tc_scr) return 1;
    const Layout LM = make_layout(M.dim, M.nc, M.rows, M.cols, M.v3);
    const int rc = tc_gemm(L.lut[mi], M.nstages, LM, ntok, x, ldx, norm_w, eps, y, ldy, accumulate, mode, aux,
                           m->tc_scr, s);
    return rc < 0 ? -1 : rc == 1 ? 0 : 1;
}

// y[n] (=|+=) W RMSNorm?(x[n]) for a batch of ntok token rows: the tcgen05 GEMM, else the
// mma.sync kernel (vq_mma.cu) through spk_verify_gemm.
// (The verify batch, ntok <= 8, is bound by the code-word gathers either way; the tcgen05 GEMM
// is the faster of the two for rows of 8192 columns and more, measured at 58 vs 72 us for
// down_proj 2560 x 10240 at 8 tokens, and slower for the shorter rows.)
int vq_batch(spk_model *m, const spk_model::Layer &L, int mi, int ntok, const float *x, int ldx, const float *norm_w,
             float eps, float *y, int ldy, int accumulate, cudaStream_t s) {
    if (L.m[mi].cols >= 8192) {
        const int rc = tc_call(m, L, mi, ntok, x, ldx, norm_w, eps, y, ldy, accumulate, 0, nullptr, s);
        if (rc <= 0) return rc;
    }
    const spk_vq_matrix &M = L.m[mi];
    return spk_verify_gemm(M.stages, M.nstages, M.dim, M.nc, M.rows, M.cols, M.v3, ntok, x, ldx, norm_w, eps, y, ldy,
                           accumulate, s);
}

// act[n] = gelu_erf(W_gate xn) * (W_up xn) for the batch: gate into g, then up with the
// GELU epilogue on a tensor-core kernel; else the SIMT pair token by token.
int ffn_batch(spk_model *m, const spk_model::Layer &L, int ntok, const float *h, int ldh, float eps, float *g,
              float *act, int ld, cudaStream_t s) {
    if (L.lut[3][0] && L.lut[4][0] && m->tc_scr && L.m[3].cols >= 8192) {
        int rc = tc_call(m, L, 3, ntok, h, ldh, L.post_norm, eps, g, ld, 0, 0, nullptr, s);
        if (rc < 0) return -1;
        if (rc == 0) {
            rc = tc_call(m, L, 4, ntok, h, ldh, L.post_norm, eps, act, ld, 0, 1, g, s);
            if (rc <= 0) return rc;
        }
    }
    const spk_vq_matrix &Gm = L.m[3], &U = L.m[4];
    if (Gm.nstages <= 2 && Gm.nstages == U.nstages) {
        const Layout LG = make_layout(Gm.dim, Gm.nc, Gm.rows, Gm.cols, Gm.v3);
        const Layout LU = make_layout(U.dim, U.nc, U.rows, U.cols, U.v3);
        int rc = vq_mma_batch(Gm.stages, Gm.nstages, LG, ntok, h, ldh, L.post_norm, eps, g, ld, 0, 0, nullptr, s);
        if (rc < 0) return -1;
        if (rc == 1) {
            rc = vq_mma_batch(U.stages, U.nstages, LU, ntok, h, ldh, L.post_norm, eps, act, ld, 0, 1, g, s);
            if (rc != 0) return rc < 0 ? -1 : 0;
        }
    }
    for (int t = 0; t < ntok; t++)
        if (vq_call(Gm, 2, &U, h + (size_t)t * ldh, L.post_norm, eps, act + (size_t)t * ld, 0, s)) return -1;
    return 0;
}

// The verify forward of ntok tokens (device m->vtok) at positions state[0] + t:
// per-row greedy ids into state[8 + t]. Same math as ntok decode steps: every
// token's K/V row is stored before any token attends, and each token sees the
// positions up to its own.
int enqueue_verify(spk_model *m, int ntok) {
    const spk_model_config &c = m->cfg;
    cudaStream_t s = m->stream;
    const bool tp = m->tp_world > 1;
    int *vam = m->state + 8, *vam_l = m->state + 16;
    const int H = c.hidden, ldqkv = m->q_dim + 2 * m->kv_dim;
    for (int t = 0; t < ntok; t++)
        if (spk_q80_row(m->embed, c.vocab, H, 0, m->vtok + t, m->h + (size_t)t * H, s)) return -1;
    for (int li = 0; li < c.layers; li++) {
        const spk_model::Layer &L = m->layers[li];
        if (capture_rows(m, li, ntok, s)) return -1;
        if (vq_batch(m, L, 0, ntok, m->h, H, L.in_norm, c.eps, m->qkv, ldqkv, 0, s) ||
            vq_batch(m, L, 1, ntok, m->h, H, L.in_norm, c.eps, m->gate, m->hl, 0, s))
            return -1;
        AttnArgs a = attn_args(m, li, ntok);
        a.store = 0;
        // ntok times a decode step's CTAs: fewer splits keep the grid near one wave
        a.nsplit = std::max(1, std::min(a.nsplit, (sm_count() + m->kvl * ntok - 1) / (m->kvl * ntok)));
        if (attn_store_batch(a, s) || attn_decode(a, s)) return -1;
        if (vq_batch(m, L, 2, ntok, m->attn, m->q_dim, nullptr, 0.f, tp ? m->pbuf : m->h, H, tp ? 0 : 1, s))
            return -1;
        if (tp && tp_sum(m->tpv, m->pbuf, m->h, ntok * H, s)) return -1;
        if (ffn_batch(m, L, ntok, m->h, H, c.eps, m->gbuf, m->act, m->inter_l, s)) return -1;
        if (vq_batch(m, L, 5, ntok, m->act, m->inter_l, nullptr, 0.f, tp ? m->pbuf : m->h, H, tp ? 0 : 1, s))
            return -1;
        if (tp && tp_sum(m->tpv, m->pbuf, m->h, ntok * H, s)) return -1;
    }
    const uint8_t *head_rows = (const uint8_t *)m->embed + (size_t)m->row0 * (H / 32) * 34;
    // all rows in one pass over the table: the tiled head (q8t.cu), else head_batch.cu, else row by row
    int hb = m->head_tiled ? q8t_head_launch(m->head_tiled, m->vocab_l, H, ntok, m->h, H, m->final_norm, c.eps,
                                             m->logits, m->vocab_l, tp ? vam_l : vam, m->head_tiled_scratch, s)
                           : 0;
    if (hb == 0)
        hb = q80_head_batch_launch(head_rows, m->vocab_l, H, ntok, m->h, H, m->final_norm, c.eps, m->logits,
                                   m->vocab_l, tp ? vam_l : vam, m->vhead_partial, m->vhead_counter, s);
    if (hb < 0) return -1;
    for (int t = 0; hb == 0 && t < ntok; t++)
        if (q80_head_launch(head_rows, m->vocab_l, H, m->h + (size_t)t * H, m->final_norm, c.eps,
                            m->logits + (size_t)t * m->vocab_l, (tp ? vam_l : vam) + t, m->head_partial,
                            m->head_counter, s))
            return -1;
    if (tp && tp_argmax(m->tpv, m->logits, m->vocab_l, vam_l, m->row0, vam, ntok, s)) return -1;
    return 0;
}

// ------------------------------------------------------------- prompt path ---
int alloc(void **p, size_t bytes, const char *what);
constexpr int PF_MAX = 128;   // tokens per prompt chunk (the batched GEMM's widest batch)

// The forward of n <= PF_MAX prompt tokens (device m->pf_tok) at positions pf_pos[0] + t
// (pf_pos[b] = pf_pos[0] + 8 b): every token's K/V row is stored, each token attends the
// positions up to its own (8 tokens per attention launch, in order), and the last token's
// logits and greedy id come out (forward_batch + tail_logits, vq-model-gpu.cu:858-949).
// All GEMMs run on the tensor-core kernel over the re-laid words (vq_tc.cu).
int enqueue_prefill(spk_model *m, int n) {
    const spk_model_config &c = m->cfg;
    cudaStream_t s = m->stream;
    const int H = c.hidden, ldqkv = m->q_dim + 2 * m->kv_dim;
    auto gemm = [&](const spk_model::Layer &L, int mi, const float *x, int ldx, const float *nw, float *y, int ldy,
                    int acc, int mode, const float *aux) -> int {
        const spk_vq_matrix &M = L.m[mi];
        if (!L.lut[mi][0]) return set_error("prompt path: matrix %d was not re-laid (geometry not taken)", mi);
        const Layout LM = make_layout(M.dim, M.nc, M.rows, M.cols, M.v3);
        const int rc = tc_gemm(L.lut[mi], M.nstages, LM, n, x, ldx, nw, c.eps, y, ldy, acc, mode, aux, m->pf_scr, s);
        return rc == 1 ? 0 : rc < 0 ? -1 : set_error("prompt path: the batched GEMM does not take matrix %d", mi);
    };
    for (int t = 0; t < n; t++)
        if (spk_q80_row(m->embed, c.vocab, H, 0, m->pf_tok + t, m->pf_h + (size_t)t * H, s)) return -1;
    for (int li = 0; li < c.layers; li++) {
        const spk_model::Layer &L = m->layers[li];
        if (capture_rows(m, li, n, s, m->pf_h, m->pf_pos)) return -1;
        if (gemm(L, 0, m->pf_h, H, L.in_norm, m->pf_qkv, ldqkv, 0, 0, nullptr) ||
            gemm(L, 1, m->pf_h, H, L.in_norm, m->pf_gate, m->hl, 0, 0, nullptr))
            return -1;
        for (int b = 0; 8 * b < n; b++) {
            const int nb = std::min(8, n - 8 * b);
            AttnArgs a = attn_args(m, li, nb);
            a.qkv = m->pf_qkv + (size_t)8 * b * ldqkv;
            a.gate = m->pf_gate + (size_t)8 * b * m->hl;
            a.out = m->pf_attn + (size_t)8 * b * m->q_dim;
            a.pos = m->pf_pos + b;
            a.store = 0;
            a.nsplit = std::max(1, std::min(a.nsplit, (sm_count() + m->kvl * nb - 1) / (m->kvl * nb)));
            if (attn_store_batch(a, s) || attn_decode(a, s)) return -1;
        }
        if (gemm(L, 2, m->pf_attn, m->q_dim, nullptr, m->pf_h, H, 1, 0, nullptr) ||
            gemm(L, 3, m->pf_h, H, L.post_norm, m->pf_g, m->inter_l, 0, 0, nullptr) ||
            gemm(L, 4, m->pf_h, H, L.post_norm, m->pf_act, m->inter_l, 0, 1, m->pf_g) ||
            gemm(L, 5, m->pf_act, m->inter_l, nullptr, m->pf_h, H, 1, 0, nullptr))
            return -1;
    }
    const float *last = m->pf_h + (size_t)(n - 1) * H;
    int *amax = m->state + 2;
    const int ht = m->head_tiled ? q8t_head_launch(m->head_tiled, m->vocab_l, H, 1, last, H, m->final_norm, c.eps,
                                                   m->logits, m->vocab_l, amax, m->head_tiled_scratch, s)
                                 : 0;
    if (ht < 0) return -1;
    if (ht == 0 && q80_head_launch(m->embed, m->vocab_l, H, last, m->final_norm, c.eps, m->logits, amax,
                                   m->head_partial, m->head_counter, s))
        return -1;
    return 0;
}

// The prompt buffers and the batched GEMM's scratch for PF_MAX tokens, on first use.
int prefill_buffers(spk_model *m) {
    if (m->pf_h) return 0;
    const spk_model_config &c = m->cfg;
    const size_t R = PF_MAX;
    size_t scr = 0;
    for (const auto &L : m->layers)
        for (int mi = 0; mi < 6; mi++)
            if (L.lut[mi][0]) scr = std::max(scr, tc_scratch_bytes(L.m[mi].rows, L.m[mi].cols, PF_MAX));
    if (!scr) return set_error("prompt path: no matrix was re-laid for the batched GEMM");
    if (alloc((void **)&m->pf_h, R * c.hidden * 4, "alloc prompt rows") ||
        alloc((void **)&m->pf_qkv, R * (m->q_dim + 2 * m->kv_dim) * 4, "alloc prompt qkv") ||
        alloc((void **)&m->pf_gate, R * m->hl * 4, "alloc prompt gate") ||
        alloc((void **)&m->pf_attn, R * m->q_dim * 4, "alloc prompt attention") ||
        alloc((void **)&m->pf_act, R * m->inter_l * 4, "alloc prompt act") ||
        alloc((void **)&m->pf_g, R * m->inter_l * 4, "alloc prompt gate act") ||
        alloc((void **)&m->pf_tok, R * sizeof(int), "alloc prompt tokens") ||
        alloc((void **)&m->pf_pos, R / 8 * sizeof(int), "alloc prompt positions") || alloc(&m->pf_scr, scr, "alloc prompt scratch"))
        return -1;
    if (cudaMallocHost((void **)&m->pf_host, (R + R / 8) * sizeof(int)) != cudaSuccess)
        return set_error("prompt staging allocation failed");
    cudaError_t e = cudaMemset(m->pf_scr, 0, scr);   // the batched GEMM's tile tickets start at zero
    return e == cudaSuccess ? 0 : cuda_fail("zero the prompt scratch", e);
}

bool ready(const spk_model *m) {
    if (!m->embed || !m->final_norm) return false;
    if (m->tp_world > 1 && !m->tp_ready) return false;
    for (const auto &L : m->layers)
        if (!L.set) return false;
    return true;
}

// One step: eager for the first one (it also performs every one-time kernel
// set-up), then from a CUDA graph captured once.
int run_step(spk_model *m) {
    if (!ready(m)) return set_error("model weights are not all set");
    if (m->eager_steps == 0) {
        m->eager_steps++;
        return enqueue_step(m);
    }
    if (!m->exec) {
        cudaError_t e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) return cuda_fail("begin step capture", e);
        m->capturing = 1;
        const int rc = enqueue_step(m);
        m->capturing = 0;
        cudaGraph_t g = nullptr;
        e = cudaStreamEndCapture(m->stream, &g);
        if (rc) {
            if (g) cudaGraphDestroy(g);
            return -1;
        }
        if (e != cudaSuccess) return cuda_fail("end step capture", e);
        m->graph = g;
        e = cudaGraphInstantiate(&m->exec, g, 0);
        if (e != cudaSuccess) return cuda_fail("instantiate step graph", e);
    }
    cudaError_t e = cudaGraphLaunch(m->exec, m->stream);
    return e == cudaSuccess ? 0 : cuda_fail("step graph launch", e);
}

// One verify batch: eager the first time for a batch size, then from a graph captured
// for that size.
int run_verify(spk_model *m, int ntok) {
    if (!m->veager[ntok]) {
        m->veager[ntok] = 1;
        return enqueue_verify(m, ntok);
    }
    if (!m->vexec[ntok]) {
        cudaError_t e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) return cuda_fail("begin verify capture", e);
        const int rc = enqueue_verify(m, ntok);
        cudaGraph_t g = nullptr;
        e = cudaStreamEndCapture(m->stream, &g);
        if (rc) {
            if (g) cudaGraphDestroy(g);
            return -1;
        }
        if (e != cudaSuccess) return cuda_fail("end verify capture", e);
        m->vgraph[ntok] = g;
        e = cudaGraphInstantiate(&m->vexec[ntok], g, 0);
        if (e != cudaSuccess) return cuda_fail("instantiate verify graph", e);
    }
    cudaError_t e = cudaGraphLaunch(m->vexec[ntok], m->stream);
    return e == cudaSuccess ? 0 : cuda_fail("verify graph launch", e);
}

int alloc(void **p, size_t bytes, const char *what) {
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
    if (e != cudaSuccess) return cuda_fail(what, e);
    return 0;
}

}  // namespace

extern "C" {

/* vq_runtime::model::Model::new (model.rs:294-320) plus the device state the
 * reference GPU runtime allocates in alloc_model (vq-model-gpu.cu:662-705). */
spk_model *spk_model_create(const spk_model_config *cfg, void *stream) {
    trace_pending("spk_model_create (entry)");
    if (!cfg || !cfg->full) {
        set_error("model config is missing");
        return nullptr;
    }
    const spk_model_config &c = *cfg;
    if (c.hidden <= 0 || c.layers <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.heads % c.kv_heads ||
        c.heads / c.kv_heads > ATT_MAX_GROUP || (c.head_dim != 128 && c.head_dim != 256) || c.inter <= 0 ||
        c.vocab <= 0 || c.window <= 0 || c.max_ctx <= 0 || c.hidden % 32 || c.hidden > 65536) {
        set_error("unsupported model geometry (head_dim 128/256, GQA group <= 4, hidden a multiple of 32)");
        return nullptr;
    }
    const int t = c.tp_world > 1 ? c.tp_world : 1, r = t > 1 ? c.tp_rank : 0;
    if (t > TP_MAX || r < 0 || r >= t || c.heads % t || (c.kv_heads % t && t % c.kv_heads) || c.inter % t ||
        c.vocab % t) {
        set_error("tensor parallel %d of %d: heads, inter and vocab must divide by the world size, and kv_heads "
                  "must divide it or be divisible by it (at most %d ranks)", r, t, TP_MAX);
        return nullptr;
    }
    spk_model *m = new spk_model();
    m->tp_rank = r;
    m->tp_world = t;
    m->hl = c.heads / t;
    m->kvl = c.kv_heads >= t ? c.kv_heads / t : 1;
    m->inter_l = c.inter / t;
    m->vocab_l = c.vocab / t;
    m->row0 = r * m->vocab_l;
    m->cfg = c;
    m->full.assign(c.full, c.full + c.layers);
    m->cfg.full = m->full.data();
    m->layers.resize(c.layers);
    m->cap_slot.assign(c.layers, -1);
    m->stream = (cudaStream_t)stream;
    m->q_dim = m->hl * c.head_dim;
    m->kv_dim = m->kvl * c.head_dim;
    m->G = m->hl / m->kvl;
    auto pdim = [&](float partial) {
        int d = (int)((float)c.head_dim * partial);
        return d < c.head_dim ? d : c.head_dim;
    };
    m->pdim_full = pdim(c.rope_partial_full);
    m->pdim_slide = pdim(c.rope_partial_slide);
    // as many splits as SMs per KV head (the attention is latency-bound: every CTA's
    // row loads in flight at once), with at least 64 positions (one tensor-core stage) per
    // split: a 512-position window measured 11.9 us at 8 splits, 12.8 us at 32
    const int per_head = std::min(ATT_MAX_SPLIT, sm_count() / m->kvl > 0 ? sm_count() / m->kvl : 1);
    m->nsplit_full = std::max(1, std::min(per_head, (c.max_ctx + 63) / 64));
    m->nsplit_slide = std::max(1, std::min(per_head, (std::min(c.window, c.max_ctx) + 63) / 64));
    if (c.kv_type < KV_F32 || c.kv_type > KV_Q8) {
        set_error("KV cache type %d (0 f32, 1 f16, 2 q8_0)", c.kv_type);
        delete m;
        return nullptr;
    }
    size_t kv_bytes = 0;
    for (int li = 0; li < c.layers; li++) {
        // Sliding layers keep their whole history too (not a window-sized ring), as
        // model.rs:398-412 does: Model::rollback to any earlier position stays exact,
        // which a speculative verify that rejects rows relies on. 27 sliding layers
        // at 131072 positions are 14.5 GB in f16: HBM affords it.
        const int slots = c.max_ctx;
        m->kv_off.push_back(kv_bytes);
        m->kv_slots.push_back(slots);
        kv_bytes += (size_t)m->kvl * slots * kv_row_bytes(c.kv_type, c.head_dim);
    }
    const int nsplit = std::max(m->nsplit_full, m->nsplit_slide);
    // activations hold up to ATT_MAX_TOK rows (a verify batch); the decode step uses row 0
    const size_t R = ATT_MAX_TOK;
    bool ok = !alloc((void **)&m->h, R * c.hidden * 4, "alloc h") &&
              !alloc((void **)&m->qkv, R * (m->q_dim + 2 * m->kv_dim) * 4, "alloc qkv") &&
              !alloc((void **)&m->gate, R * m->hl * 4, "alloc gate") && !alloc((void **)&m->attn, R * m->q_dim * 4, "alloc attn") &&
              !alloc((void **)&m->act, R * m->inter_l * 4, "alloc act") && !alloc((void **)&m->gbuf, R * m->inter_l * 4, "alloc g") &&
              !alloc((void **)&m->vtok, R * sizeof(int), "alloc verify tokens") &&
              !alloc((void **)&m->part, (size_t)ATT_MAX_TOK * m->kvl * nsplit * m->G * (c.head_dim + 4) * 4, "alloc attention partials") &&
              !alloc((void **)&m->att_count, (size_t)ATT_MAX_TOK * m->kvl * sizeof(unsigned int), "alloc attention tickets") &&
              !alloc((void **)&m->freq_full, c.head_dim * 4, "alloc rope") && !alloc((void **)&m->freq_slide, c.head_dim * 4, "alloc rope") &&
              !alloc(&m->kc, kv_bytes, "alloc K cache") && !alloc(&m->vc, kv_bytes, "alloc V cache") &&
              !alloc((void **)&m->state, 32 * sizeof(int), "alloc state") &&
              !alloc((void **)&m->ctl, sizeof(DevCtl), "alloc control") &&
              !alloc((void **)&m->head_partial, 1024 * sizeof(unsigned long long), "alloc head partials") &&
              !alloc((void **)&m->head_counter, sizeof(unsigned int), "alloc head counter") &&
              !alloc((void **)&m->vhead_partial, q80_head_batch_scratch(), "alloc batched head partials") &&
              !alloc((void **)&m->vhead_counter, sizeof(unsigned int), "alloc batched head counter");
    if (ok && t == 1) {
        ok = !alloc((void **)&m->logits, R * c.vocab * 4, "alloc logits");
    } else if (ok) {
        // one mailbox holds the exchange rows, the flags and this rank's logits shard
        // (peers read the shard when a host forward asks for the whole vocabulary)
        // rows of (value, sequence) pairs: two floats' room per exchanged value
        const size_t mb = tp_mailbox_bytes(t, 2 * (int)R * c.hidden, &m->mail_flags_off, &m->mail_stride);
        m->mail_logits_off = (mb + 255) / 256 * 256;
        const size_t total = m->mail_logits_off + R * m->vocab_l * 4;
        ok = !alloc(&m->mailbox, total, "alloc tensor-parallel mailbox") &&
             cudaMemset(m->mailbox, 0, total) == cudaSuccess && !alloc((void **)&m->pbuf, R * c.hidden * 4, "alloc partial") &&
             !alloc((void **)&m->logits_full, R * c.vocab * 4, "alloc gathered logits") &&
             !alloc((void **)&m->tp_seq, 2 * sizeof(unsigned int), "alloc exchange counter") &&
             cudaMemset(m->tp_seq, 0, 2 * sizeof(unsigned int)) == cudaSuccess;
        if (ok) m->logits = (float *)((uint8_t *)m->mailbox + m->mail_logits_off);
        else set_error("tensor-parallel allocation failed");
    }
    if (ok && (cudaMallocHost((void **)&m->host_io, 32 * sizeof(int)) != cudaSuccess ||
               cudaMallocHost((void **)&m->host_ctl, sizeof(DevCtl)) != cudaSuccess))
        ok = !set_error("pinned staging allocation failed");
    if (ok) {
        // rope frequencies in f32 exactly as model.rs:416-429 forms them
        std::vector<float> ff(c.head_dim, 0.f), fs(c.head_dim, 0.f);
        for (int i = 0; i < m->pdim_full / 2; i++) ff[i] = 1.0f / powf(c.rope_theta_full, (float)(2 * i) / (float)m->pdim_full);
        for (int i = 0; i < m->pdim_slide / 2; i++) fs[i] = 1.0f / powf(c.rope_theta_slide, (float)(2 * i) / (float)m->pdim_slide);
        ok = cudaMemcpy(m->freq_full, ff.data(), c.head_dim * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemcpy(m->freq_slide, fs.data(), c.head_dim * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemset(m->kc, 0, kv_bytes) == cudaSuccess && cudaMemset(m->vc, 0, kv_bytes) == cudaSuccess &&
             cudaMemset(m->state, 0, 32 * sizeof(int)) == cudaSuccess && cudaMemset(m->ctl, 0, sizeof(DevCtl)) == cudaSuccess &&
             cudaMemset(m->head_counter, 0, sizeof(unsigned int)) == cudaSuccess &&
             cudaMemset(m->vhead_counter, 0, sizeof(unsigned int)) == cudaSuccess &&
             cudaMemset(m->att_count, 0, (size_t)ATT_MAX_TOK * m->kvl * sizeof(unsigned int)) == cudaSuccess;
        if (!ok) set_error("model initialisation copies failed");
    }
    if (!ok) {
        spk_model_destroy(m);
        return nullptr;
    }
    return m;
}

void spk_model_destroy(spk_model *m) {
    trace_pending("spk_model_destroy (entry)");
    if (!m) return;
    if (m->cap) cudaFree(m->cap);
    if (m->head_tiled) cudaFree(m->head_tiled);
    if (m->head_tiled_scratch) cudaFree(m->head_tiled_scratch);
    for (auto &L : m->layers) {
        for (void *p : L.lut_mem)
            if (p) cudaFree(p);
        for (void *p : L.tab_mem)
            if (p) cudaFree(p);
    }
    if (m->tab_scr) cudaFree(m->tab_scr);
    if (m->tc_scr) cudaFree(m->tc_scr);
    for (void *p : {(void *)m->pf_h, (void *)m->pf_qkv, (void *)m->pf_gate, (void *)m->pf_attn, (void *)m->pf_act,
                    (void *)m->pf_g, (void *)m->pf_tok, (void *)m->pf_pos, m->pf_scr})
        if (p) cudaFree(p);
    if (m->pf_host) cudaFreeHost(m->pf_host);
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    if (m->texec) cudaGraphExecDestroy(m->texec);
    if (m->tgraph) cudaGraphDestroy(m->tgraph);
    for (cudaEvent_t e : m->tev) cudaEventDestroy(e);
    for (int k = 0; k <= ATT_MAX_TOK; k++) {
        if (m->vexec[k]) cudaGraphExecDestroy(m->vexec[k]);
        if (m->vgraph[k]) cudaGraphDestroy(m->vgraph[k]);
    }
    for (int r = 0; r < TP_MAX; r++)
        if (m->peer_open[r]) cudaIpcCloseMemHandle(m->peer_open[r]);
    void *ps[] = {m->h, m->qkv, m->gate, m->attn, m->act, m->tp_world > 1 ? nullptr : m->logits, m->part,
                  m->freq_full, m->freq_slide, m->kc, m->vc, m->state, m->ctl, m->head_partial, m->head_counter,
                  m->mailbox, m->pbuf, m->logits_full, m->tp_seq, m->att_count, m->gbuf, m->vtok, m->vhead_partial, m->vhead_counter};
    for (void *p : ps)
        if (p) cudaFree(p);
    if (m->host_io) cudaFreeHost(m->host_io);
    if (m->host_ctl) cudaFreeHost(m->host_ctl);
    delete m;
    trace_pending("spk_model_destroy (exit)");
}

// Every layer matrix the table layout takes (DQV3 dim 4, 4096 codes, 12-bit) is re-laid once
// here (vq_lut.cu's words: code words, gains, slice-major index records): the batched GEMM of
// the verify batch runs on those words (vq_tc.cu). The decode step runs the gate/up pair through
// the bank-scheduled table kernel (vq_tab.cu) when its shard has at least PAIR_TAB_MIN_ROWS rows
// (measured on B200: 35 vs 43 us at 5120 rows, even at 2560, slower below: a table of 4096 x 8
// entries pays back only over many rows, and the kernel has a fixed cost of its own); every
// other matrix through the code-word kernel (vq.cu) over the payloads, which stay (g_proj reads
// them too), and which measured faster for q_k_v_proj, out_proj and down_proj at every shard.
constexpr int PAIR_TAB_MIN_ROWS = 4096;

static int relay_layer(spk_model *m, spk_model::Layer &L) {
    auto release = [](void *&p, const char *what) -> int {
        if (!p) return 0;
        const cudaError_t e = cudaFree(p);
        p = nullptr;
        return e == cudaSuccess ? 0 : cuda_fail(what, e);
    };
    for (int mi = 0; mi < 6; mi++) {
        if (release(L.lut_mem[mi], "free vq table words") || release(L.tab_mem[mi], "free vq table words")) return -1;
        L.dec[mi] = false;
        for (int q = 0; q < 4; q++) L.lut[mi][q] = L.tab[mi][q] = nullptr;
    }
    const int ng_of[6] = {1, 1, 1, 2, 2, 1};
    size_t part_need = 0, tc_need = 0;
    for (int mi = 0; mi < 6; mi++) {
        const spk_vq_matrix &M = L.m[mi];
        const Layout LM = make_layout(M.dim, M.nc, M.rows, M.cols, M.v3);
        if (!lut_ok(LM, M.nstages, 1)) continue;
        const size_t per = lut_bytes(LM);
        if (alloc(&L.lut_mem[mi], per * M.nstages, "alloc vq table words")) return -1;
        for (int q = 0; q < M.nstages; q++) {
            L.lut[mi][q] = (const uint8_t *)L.lut_mem[mi] + per * q;
            if (lut_pack(M.stages[q], LM, (void *)L.lut[mi][q], m->stream)) return -1;
        }
        bool want = (mi == 3 || mi == 4) && M.rows >= PAIR_TAB_MIN_ROWS;   // the heuristic
        bool runs = tab::ok(LM, M.nstages, ng_of[mi]);
        for (int q = 0; runs && q < M.nstages; q++)
            if (((uintptr_t)M.stages[q] + LM.cb_off) & 7) runs = false;
        // a profile entry for this geometry replaces the heuristic where its kernel can run
        // (vq-model-gpu.cu:301-324); g_proj rides with q_k_v_proj and takes no entry
        for (const spk_vqprof_entry &e : m->prof) {
            if (mi == 1 || e.kind != 0 || e.dim != M.dim || e.nc != M.nc || e.rows != M.rows || e.cols != M.cols ||
                e.v3 != M.v3)
                continue;
            if (e.variant == SPK_VARIANT_TABLE && !runs)
                fprintf(stderr, "profile: gemv entry for %dx%d is not runnable here; heuristic kept\n", M.rows, M.cols);
            else if (e.variant < 0 || e.variant > SPK_VARIANT_TABLE)
                fprintf(stderr, "profile: gemv entry for %dx%d names variant %d; heuristic kept\n", M.rows, M.cols,
                        e.variant);
            else
                want = e.variant == SPK_VARIANT_TABLE;
            break;
        }
        L.dec[mi] = want && runs;
        if (L.dec[mi]) {
            const size_t pw = tab::bytes(LM);
            if (alloc(&L.tab_mem[mi], pw * M.nstages, "alloc vq table words")) return -1;
            for (int q = 0; q < M.nstages; q++) {
                L.tab[mi][q] = (const uint8_t *)L.tab_mem[mi] + pw * q;
                if (tab::pack(M.stages[q], LM, (void *)L.tab[mi][q], m->stream)) return -1;
            }
            part_need = std::max(part_need, tab::scratch_bytes(LM, ng_of[mi]));
        }
        if (M.cols % 32 == 0) tc_need = std::max(tc_need, tc_scratch_bytes(M.rows, M.cols, ATT_MAX_TOK));
    }
    if (!(L.dec[3] && L.dec[4]))   // the pair only together
        for (int mi : {3, 4}) {
            if (release(L.tab_mem[mi], "free vq table words")) return -1;
            L.dec[mi] = false;
        }
    // the scratches, grown (once) to the largest need of any layer
    if (part_need > m->tab_scr_size) {
        if (release(m->tab_scr, "free vq table scratch")) return -1;
        m->tab_scr_size = 0;
        if (alloc(&m->tab_scr, part_need, "alloc vq table scratch")) return -1;
        m->tab_scr_size = part_need;
        cudaError_t e = cudaMemset(m->tab_scr, 0, part_need);   // the grid barrier's count starts at zero
        if (e != cudaSuccess) return cuda_fail("zero the vq table scratch", e);
    }
    if (tc_need > m->tc_scr_size) {
        if (release(m->tc_scr, "free batched gemm scratch")) return -1;
        m->tc_scr_size = 0;
        if (alloc(&m->tc_scr, tc_need, "alloc batched gemm scratch")) return -1;
        m->tc_scr_size = tc_need;
        cudaError_t e = cudaMemset(m->tc_scr, 0, tc_need);   // the tile tickets start at zero
        if (e != cudaSuccess) return cuda_fail("zero the batched gemm scratch", e);
    }
    trace_pending("relay: exit");
    cudaError_t e = cudaStreamSynchronize(m->stream);
    return e == cudaSuccess ? 0 : cuda_fail("re-lay the index streams", e);
}

static int check_mat(const spk_vq_matrix *M, int rows, int cols, const char *name) {
    if (!M) return set_error("%s: matrix is missing", name);
    if (M->rows != rows || M->cols != cols)
        return set_error("%s: is %dx%d, the architecture needs %dx%d", name, M->rows, M->cols, rows, cols);
    if (M->nstages < 1 || M->nstages > 4) return set_error("%s: %d stages (1..4 supported)", name, M->nstages);
    for (int s = 0; s < M->nstages; s++)
        if (!M->stages[s]) return set_error("%s: stage %d is null", name, s);
    return 0;
}

/* Weights::load per layer (model.rs:130-187): shapes checked as the reference checks them. */
int spk_model_set_layer(spk_model *m, int layer, const spk_vq_matrix *qkv, const spk_vq_matrix *attn_gate,
                        const spk_vq_matrix *out, const spk_vq_matrix *gate, const spk_vq_matrix *up,
                        const spk_vq_matrix *down, const float *in_norm, const float *post_norm) {
    trace_pending("spk_model_set_layer (entry)");
    if (!m) return set_error("model is null");
    if (layer < 0 || layer >= m->cfg.layers) return set_error("layer %d is outside the %d layers", layer, m->cfg.layers);
    const spk_model_config &c = m->cfg;
    if (check_mat(qkv, m->q_dim + 2 * m->kv_dim, c.hidden, "q_k_v_proj") || check_mat(attn_gate, m->hl, c.hidden, "g_proj") ||
        check_mat(out, c.hidden, m->q_dim, "out_proj") || check_mat(gate, m->inter_l, c.hidden, "gate_proj") ||
        check_mat(up, m->inter_l, c.hidden, "up_proj") || check_mat(down, c.hidden, m->inter_l, "down_proj"))
        return -1;
    if (gate->nstages != up->nstages || gate->dim != up->dim || gate->nc != up->nc || gate->v3 != up->v3)
        return set_error("gate_proj and up_proj must share one encoding to run as a pair");
    if (!in_norm || !post_norm) return set_error("layer %d: a norm is missing", layer);
    spk_model::Layer &L = m->layers[layer];
    L.m[0] = *qkv;
    L.m[1] = *attn_gate;
    L.m[2] = *out;
    L.m[3] = *gate;
    L.m[4] = *up;
    L.m[5] = *down;
    L.in_norm = in_norm;
    L.post_norm = post_norm;
    if (relay_layer(m, L)) return -1;
    L.set = true;
    return 0;
}

// Drop every captured graph: the next step (and verify batch) captures again.
static void drop_graphs(spk_model *m) {
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    if (m->texec) cudaGraphExecDestroy(m->texec);
    if (m->tgraph) cudaGraphDestroy(m->tgraph);
    m->exec = nullptr;
    m->graph = nullptr;
    m->texec = nullptr;
    m->tgraph = nullptr;
    for (int k = 0; k <= ATT_MAX_TOK; k++) {
        if (m->vexec[k]) cudaGraphExecDestroy(m->vexec[k]);
        if (m->vgraph[k]) cudaGraphDestroy(m->vgraph[k]);
        m->vexec[k] = nullptr;
        m->vgraph[k] = nullptr;
    }
}

int spk_model_use_profile(spk_model *m, const spk_vqprof *pf) {
    if (!m) return set_error("use_profile: model is null");
    m->prof.clear();
    if (pf) {
        if (pf->n < 0 || pf->n > SPK_VQPROF_MAX) return set_error("use_profile: %d entries (0..%d)", pf->n, SPK_VQPROF_MAX);
        for (int i = 0; i < pf->n; i++)
            if (pf->e[i].kind == 0) m->prof.push_back(pf->e[i]);
    }
    cudaError_t e = cudaStreamSynchronize(m->stream);   // no step in flight reads what is re-laid
    if (e != cudaSuccess) return cuda_fail("use_profile: synchronize", e);
    drop_graphs(m);
    for (spk_model::Layer &L : m->layers)
        if (L.set && relay_layer(m, L)) return -1;
    return 0;
}

int spk_model_kernel_of(spk_model *m, int layer, int matrix) {
    if (!m || layer < 0 || layer >= (int)m->layers.size() || matrix < 0 || matrix > 5)
        return set_error("kernel_of: layer %d / matrix %d out of range", layer, matrix);
    const spk_model::Layer &L = m->layers[layer];
    if (!L.set) return set_error("kernel_of: layer %d is not set", layer);
    return L.dec[matrix] ? SPK_VARIANT_TABLE : 3;
}

/* The tied embedding / LM head as Q8_0 blocks [vocab][hidden] and the final norm. */
int spk_model_set_head(spk_model *m, const void *embed_q80, const float *final_norm) {
    trace_pending("spk_model_set_head (entry)");
    if (!m || !embed_q80 || !final_norm) return set_error("head weights are missing");
    m->embed = embed_q80;
    m->final_norm = final_norm;
    // the head's rows (this rank's vocabulary shard) re-laid once for the tensor-core head;
    // the embedding row gather keeps reading the ggml blocks
    const int H = m->cfg.hidden;
    if (!m->head_tiled && m->vocab_l % 16 == 0 && H % 32 == 0 && H >= 256 && H <= 4096) {
        if (alloc(&m->head_tiled, q8t_bytes(m->vocab_l, H), "alloc tiled head") ||
            alloc(&m->head_tiled_scratch, q8t_scratch(), "alloc tiled head scratch"))
            return -1;
        if (cudaMemset(m->head_tiled_scratch, 0, q8t_scratch()) != cudaSuccess)
            return cuda_fail("clear tiled head scratch", cudaGetLastError());
    }
    if (m->head_tiled) {
        const uint8_t *rows = (const uint8_t *)embed_q80 + (size_t)m->row0 * (H / 32) * 34;
        if (q8t_pack(rows, m->vocab_l, H, m->head_tiled, m->stream)) return -1;
        cudaError_t e = cudaStreamSynchronize(m->stream);
        if (e != cudaSuccess) return cuda_fail("tile the head", e);
    }
    return 0;
}

/* Model::forward(token, pos) (model.rs:442-591) through host buffers: the token
 * goes up, the greedy next id (and, if logits_host is not NULL, the vocab-wide
 * logits) come back; synchronizes the model's stream. */
int spk_model_forward(spk_model *m, int token, int pos, float *logits_host, int *next_host) {
    trace_pending("spk_model_forward (entry)");
    if (!m) return set_error("model is null");
    if (token < 0 || token >= m->cfg.vocab) return set_error("token %d is outside the vocabulary", token);
    if (pos < 0 || pos >= m->cfg.max_ctx) return set_error("position %d exceeds the %d-token cache", pos, m->cfg.max_ctx);
    if (pos > m->len) return set_error("position %d skips cached positions (%d cached)", pos, m->len);
    m->host_io[0] = pos;
    m->host_io[1] = token;
    cudaError_t e = cudaMemcpyAsync(m->state, m->host_io, 2 * sizeof(int), cudaMemcpyHostToDevice, m->stream);
    if (e != cudaSuccess) return cuda_fail("state upload", e);
    if (run_step(m)) return -1;
    e = cudaMemcpyAsync(m->host_io + 2, m->state + 2, sizeof(int), cudaMemcpyDeviceToHost, m->stream);
    const float *full = m->logits;
    if (e == cudaSuccess && logits_host && m->tp_world > 1) {
        // every rank's shard is final once this rank's argmax exchange has completed,
        // and no rank can overwrite it before this rank joins the next step
        for (int r = 0; r < m->tp_world && e == cudaSuccess; r++)
            e = cudaMemcpyAsync(m->logits_full + (size_t)r * m->vocab_l, m->peer_logits[r], (size_t)m->vocab_l * 4,
                                cudaMemcpyDefault, m->stream);
        full = m->logits_full;
    }
    if (e == cudaSuccess && logits_host)
        e = cudaMemcpyAsync(logits_host, full, (size_t)m->cfg.vocab * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) return cuda_fail("forward", e);
    if (check_device_error("forward")) return -1;
    if (next_host) *next_host = m->host_io[2];
    m->len = pos + 1;
    return 0;
}

/* The speculative verify (vq-model-gpu.cu:947-969 verify_logits, spec.rs:197-205):
 * tokens[0..ntok) at positions pos..pos+ntok-1 in one batched forward; next_host[t]
 * receives the greedy id after tokens[t] (Model::argmax of that row), logits_host
 * (optional) the [ntok][vocab] logits. Afterwards len = pos + ntok; the caller keeps
 * the accepted prefix with spk_model_rollback, as spec.rs:241 does. Synchronizes. */
int spk_model_verify(spk_model *m, const int *tokens, int ntok, int pos, int *next_host, float *logits_host) {
    trace_pending("spk_model_verify (entry)");
    if (!m) return set_error("model is null");
    if (!ready(m)) return set_error("model weights are not all set");
    if (!tokens || ntok < 1 || ntok > ATT_MAX_TOK) return set_error("verify takes 1..%d tokens, not %d", ATT_MAX_TOK, ntok);
    for (int t = 0; t < ntok; t++)
        if (tokens[t] < 0 || tokens[t] >= m->cfg.vocab) return set_error("token %d is outside the vocabulary", tokens[t]);
    if (pos < 0 || pos + ntok > m->cfg.max_ctx) return set_error("positions %d..%d exceed the %d-token cache", pos, pos + ntok - 1, m->cfg.max_ctx);
    if (pos > m->len) return set_error("position %d skips cached positions (%d cached)", pos, m->len);
    m->host_io[0] = pos;
    for (int t = 0; t < ntok; t++) m->host_io[8 + t] = tokens[t];
    cudaError_t e = cudaMemcpyAsync(m->state, m->host_io, sizeof(int), cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->vtok, m->host_io + 8, ntok * sizeof(int), cudaMemcpyHostToDevice, m->stream);
    if (e != cudaSuccess) return cuda_fail("verify upload", e);
    if (run_verify(m, ntok)) return -1;
    e = cudaMemcpyAsync(m->host_io + 16, m->state + 8, ntok * sizeof(int), cudaMemcpyDeviceToHost, m->stream);
    const float *full = m->logits;
    if (e == cudaSuccess && logits_host && m->tp_world > 1) {
        for (int t = 0; t < ntok && e == cudaSuccess; t++)
            for (int r = 0; r < m->tp_world && e == cudaSuccess; r++)
                e = cudaMemcpyAsync(m->logits_full + (size_t)t * m->cfg.vocab + (size_t)r * m->vocab_l,
                                    m->peer_logits[r] + (size_t)t * m->vocab_l, (size_t)m->vocab_l * 4,
                                    cudaMemcpyDefault, m->stream);
        full = m->logits_full;
    }
    if (e == cudaSuccess && logits_host)
        e = cudaMemcpyAsync(logits_host, full, (size_t)ntok * m->cfg.vocab * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) return cuda_fail("verify", e);
    if (check_device_error("verify")) return -1;
    if (next_host)
        for (int t = 0; t < ntok; t++) next_host[t] = m->host_io[16 + t];
    m->len = pos + ntok;
    return 0;
}

/* The prompt: tokens[0..n) at positions pos .. pos + n - 1 through the model in chunks of up to
 * 128 tokens (the reference's chunked prefill, forward_batch, vq-model-gpu.cu:858-943, and its
 * loop at :1164-1168), every GEMM on the tensor cores (tcgen05); every position's K/V row is
 * stored, and the last token's greedy next id (*next_host) and logits (logits_host, vocab
 * floats) come back as spk_model_forward's would. Tensor-parallel models take the prompt in
 * verify batches of 8. Synchronizes. */
int spk_model_prefill(spk_model *m, const int *tokens, int n, int pos, int *next_host, float *logits_host) {
    trace_pending("spk_model_prefill (entry)");
    if (!m) return set_error("model is null");
    if (!ready(m)) return set_error("model weights are not all set");
    if (!tokens || n < 1) return set_error("prefill needs at least one token");
    for (int t = 0; t < n; t++)
        if (tokens[t] < 0 || tokens[t] >= m->cfg.vocab) return set_error("token %d is outside the vocabulary", tokens[t]);
    if (pos < 0 || (long long)pos + n > m->cfg.max_ctx)
        return set_error("positions %d..%d exceed the %d-token cache", pos, pos + n - 1, m->cfg.max_ctx);
    if (pos > m->len) return set_error("position %d skips cached positions (%d cached)", pos, m->len);
    if (m->tp_world > 1) {   // verify batches: the exchanges hold 8 rows
        for (int t0 = 0; t0 < n; t0 += ATT_MAX_TOK) {
            const int nb = std::min(ATT_MAX_TOK, n - t0);
            int ids[ATT_MAX_TOK];
            const bool last = t0 + nb == n;
            if (spk_model_verify(m, tokens + t0, nb, pos + t0, ids, nullptr)) return -1;
            if (last) {
                if (next_host) *next_host = ids[nb - 1];
                if (logits_host) {   // the verify batch left every row's logits; the last is wanted
                    std::vector<float> all((size_t)nb * m->cfg.vocab);
                    if (spk_model_verify(m, tokens + t0, nb, pos + t0, ids, all.data())) return -1;
                    memcpy(logits_host, all.data() + (size_t)(nb - 1) * m->cfg.vocab, (size_t)m->cfg.vocab * 4);
                }
            }
        }
        return 0;
    }
    if (prefill_buffers(m)) return -1;
    cudaError_t e = cudaSuccess;
    for (int t0 = 0; t0 < n; t0 += PF_MAX) {
        const int nb = std::min(PF_MAX, n - t0);
        for (int t = 0; t < nb; t++) m->pf_host[t] = tokens[t0 + t];
        for (int b = 0; b < PF_MAX / 8; b++) m->pf_host[PF_MAX + b] = pos + t0 + 8 * b;
        e = cudaMemcpyAsync(m->pf_tok, m->pf_host, nb * sizeof(int), cudaMemcpyHostToDevice, m->stream);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(m->pf_pos, m->pf_host + PF_MAX, PF_MAX / 8 * sizeof(int), cudaMemcpyHostToDevice, m->stream);
        if (e != cudaSuccess) return cuda_fail("prefill upload", e);
        if (enqueue_prefill(m, nb)) return -1;
        // the staging is rewritten for the next chunk: its copies must have left
        e = cudaStreamSynchronize(m->stream);
        if (e != cudaSuccess) return cuda_fail("prefill", e);
    }
    m->host_io[0] = pos + n;
    e = cudaMemcpyAsync(m->state, m->host_io, sizeof(int), cudaMemcpyHostToDevice, m->stream);   // the next position
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->host_io + 2, m->state + 2, sizeof(int), cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess && logits_host)
        e = cudaMemcpyAsync(logits_host, m->logits, (size_t)m->cfg.vocab * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) return cuda_fail("prefill", e);
    if (check_device_error("prefill")) return -1;
    if (next_host) *next_host = m->host_io[2];
    m->len = pos + n;
    return 0;
}

/* Device-resident greedy decoding: set (pos, token) and the device id buffer
 * that spk_model_run fills, one id per step. */
int spk_model_begin(spk_model *m, int token, int pos, int *ids_dev, int ids_cap) {
    trace_pending("spk_model_begin (entry)");
    if (!m) return set_error("model is null");
    if (token < 0 || token >= m->cfg.vocab || pos < 0 || pos > m->len) return set_error("bad start token/position");
    cudaError_t e = cudaStreamSynchronize(m->stream);   // the pinned staging may still be in flight
    if (e != cudaSuccess) return cuda_fail("begin", e);
    m->host_ctl->ids = ids_dev;
    m->host_ctl->cap = ids_dev ? ids_cap : 0;
    e = cudaMemcpyAsync(m->ctl, m->host_ctl, sizeof(DevCtl), cudaMemcpyHostToDevice, m->stream);
    if (e != cudaSuccess) return cuda_fail("begin", e);
    set_state_kernel<<<1, 1, 0, m->stream>>>(m->state, m->state + 1, pos, token);
    e = cudaMemsetAsync(m->state + 3, 0, sizeof(int), m->stream);
    return e == cudaSuccess ? 0 : cuda_fail("begin", e);
}

/* Run `steps` greedy decode steps from the device state, no host round trip. */
int spk_model_run(spk_model *m, int steps) {
    trace_pending("spk_model_run (entry)");
    if (!m) return set_error("model is null");
    for (int i = 0; i < steps; i++)
        if (run_step(m)) return -1;
    return 0;
}

/* Device pointer of the last step's logits [vocab]. */
const float *spk_model_logits(spk_model *m) { return m ? m->logits : nullptr; }

/* Model::enable_capture (model.rs:322-343). The captured graphs are dropped so the next
 * step and verify batch are captured again with the copies in them. */
int spk_model_enable_capture(spk_model *m, const int *layers, int n) {
    if (!m) return set_error("model is null");
    if (n < 0 || n > 8 || (n && !layers)) return set_error("capture takes 0..8 layers, not %d", n);
    std::vector<int> slot(m->cfg.layers, -1);
    for (int k = 0; k < n; k++) {
        if (layers[k] < 0 || layers[k] >= m->cfg.layers) return set_error("capture layer %d is outside the %d layers", layers[k], m->cfg.layers);
        if (slot[layers[k]] >= 0) return set_error("capture layer %d is listed twice", layers[k]);
        slot[layers[k]] = k;
    }
    cudaError_t e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) return cuda_fail("capture set-up", e);
    if (m->cap) cudaFree(m->cap);
    m->cap = nullptr;
    m->ncap = 0;
    if (n) {
        const size_t bytes = (size_t)n * m->cfg.max_ctx * m->cfg.hidden * sizeof(float);
        if (alloc((void **)&m->cap, bytes, "alloc layer captures")) return -1;
        if (cudaMemset(m->cap, 0, bytes) != cudaSuccess) return cuda_fail("clear layer captures", cudaGetLastError());
    }
    m->cap_slot = slot;
    m->ncap = n;
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    m->exec = nullptr;
    m->graph = nullptr;
    if (m->texec) cudaGraphExecDestroy(m->texec);
    if (m->tgraph) cudaGraphDestroy(m->tgraph);
    m->texec = nullptr;
    m->tgraph = nullptr;
    for (int k = 0; k <= ATT_MAX_TOK; k++) {
        if (m->vexec[k]) cudaGraphExecDestroy(m->vexec[k]);
        if (m->vgraph[k]) cudaGraphDestroy(m->vgraph[k]);
        m->vexec[k] = nullptr;
        m->vgraph[k] = nullptr;
    }
    return 0;
}

/* Model::captured (model.rs:345-348): the capture rows on device, slot k of position p at
 * [k * *slot_stride + p * hidden]. NULL while capture is off. */
int spk_model_step_launches(const spk_model *m) { return m ? m->step_launches : -1; }

const void *spk_model_head_tiled(spk_model *m) { return m ? m->head_tiled : nullptr; }

const float *spk_model_captures(spk_model *m, size_t *slot_stride) {
    if (!m || !m->ncap) return nullptr;
    if (slot_stride) *slot_stride = (size_t)m->cfg.max_ctx * m->cfg.hidden;
    return m->cap;
}

/* Model::rollback (model.rs:361-382): keep the first `pos` cached positions. */
int spk_model_rollback(spk_model *m, int pos) {
    trace_pending("spk_model_rollback (entry)");
    if (!m) return set_error("model is null");
    if (pos < 0 || pos > m->len) return set_error("rollback to %d exceeds the %d cached positions", pos, m->len);
    m->len = pos;
    return 0;
}

/* Model::reset (model.rs:384-396) */
int spk_model_reset(spk_model *m) { return spk_model_rollback(m, 0); }

/* Positions cached (Model::len). */
int spk_model_len(spk_model *m) { return m ? m->len : -1; }

/* Cache rows given as values: positions pos0 .. pos0 + n - 1 of `layer` take K and V from
 * device f32 rows k, v [n][kv_heads * head_dim] (every KV head of the model, keys already
 * roped, as the attention stores them; a tensor-parallel rank keeps its own heads), stored
 * in the cache's type. Asynchronous on the model's stream; the host length is not changed
 * (spk_model_advance_len records the positions). */
int spk_model_write_kv(spk_model *m, int layer, int pos0, int n, const float *k, const float *v) {
    if (!m) return set_error("model is null");
    const spk_model_config &c = m->cfg;
    if (layer < 0 || layer >= c.layers || pos0 < 0 || n < 0 || (long long)pos0 + n > c.max_ctx)
        return set_error("cache write: layer %d, positions %d + %d outside the model", layer, pos0, n);
    if (n > 0 && (!k || !v)) return set_error("cache write: null rows");
    const int head0 = m->tp_rank * m->hl * c.kv_heads / c.heads;
    return kv_write((uint8_t *)m->kc + m->kv_off[layer], (uint8_t *)m->vc + m->kv_off[layer], c.kv_type,
                    m->kv_slots[layer], m->kvl, head0, c.head_dim, pos0, n, k, v, c.kv_heads * c.head_dim,
                    m->stream);
}

/* Record that `n` device-run steps extended the cache (spk_model_run does not
 * sync, so the host view is advanced explicitly). */
int spk_model_advance_len(spk_model *m, int n) {
    if (!m || n < 0 || m->len + n > m->cfg.max_ctx) return set_error("bad length advance");
    m->len += n;
    return 0;
}

/* One decode step from the device state (as spk_model_run does) with the device time
 * of every launch: us[i] = microseconds of launch i in enqueue order (embedding row;
 * per layer QKV+g_proj, attention, out_proj, [tp_sum], gate+up, down,
 * [tp_sum]; head; [tp_argmax]; advance). Returns the number of launches, or -1.
 * Needs one step run before (it reuses the kernels' one-time set-up); with
 * tensor parallelism every rank traces the same step. */
int spk_model_trace(spk_model *m, float *us, int cap) {
    if (!m) return set_error("model is null");
    if (!ready(m)) return set_error("model weights are not all set");
    if (!m->eager_steps) return set_error("trace needs one step run first");
    const int n = m->step_marks;   // marks of a step (the first one before any launch), as the last enqueue made
    if (!us || cap < n - 1) return set_error("trace needs room for %d launches", n - 1);
    if (!m->texec) {
        for (int i = 0; i < n; i++) {
            cudaEvent_t e;
            if (cudaEventCreate(&e) != cudaSuccess) return cuda_fail("trace events", cudaGetLastError());
            m->tev.push_back(e);
        }
        cudaError_t e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) return cuda_fail("begin trace capture", e);
        m->tracing = 1;
        m->capturing = 1;
        m->nmark = 0;
        const int rc = enqueue_step(m);
        m->tracing = 0;
        m->capturing = 0;
        cudaGraph_t g = nullptr;
        e = cudaStreamEndCapture(m->stream, &g);
        if (rc || e != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            return rc ? -1 : cuda_fail("end trace capture", e);
        }
        if (m->nmark != n) {
            cudaGraphDestroy(g);
            return set_error("trace: %d marks, expected %d", m->nmark, n);
        }
        m->tgraph = g;
        e = cudaGraphInstantiate(&m->texec, g, 0);
        if (e != cudaSuccess) return cuda_fail("instantiate trace graph", e);
    }
    cudaError_t e = cudaGraphLaunch(m->texec, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) return cuda_fail("trace step", e);
    if (check_device_error("trace step")) return -1;
    for (int i = 0; i + 1 < n; i++) {
        float ms = 0.f;
        e = cudaEventElapsedTime(&ms, m->tev[i], m->tev[i + 1]);
        if (e != cudaSuccess) return cuda_fail("trace elapsed", e);
        us[i] = ms * 1000.f;
    }
    return n - 1;
}

/* The mailbox's IPC handle, for the other ranks' spk_model_tp_attach. */
int spk_model_tp_handle(spk_model *m, void *handle_out, int n) {
    if (!m || m->tp_world < 2 || !m->mailbox) return set_error("the model is not tensor-parallel");
    if (!handle_out || n < (int)sizeof(cudaIpcMemHandle_t)) return set_error("the handle buffer needs %d bytes", (int)sizeof(cudaIpcMemHandle_t));
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, m->mailbox);
    if (e != cudaSuccess) return cuda_fail("export the mailbox", e);
    memcpy(handle_out, &h, sizeof h);
    return 0;
}

static int tp_wire(spk_model *m, void *const *bases, int wait_ms) {
    if (wait_ms <= 0) return set_error("the exchange wait limit must be positive");
    TpView &v = m->tpv;
    v = TpView{};
    for (int r = 0; r < m->tp_world; r++) {
        v.mail[r] = (float *)bases[r];
        v.flags[r] = (unsigned int *)((uint8_t *)bases[r] + m->mail_flags_off);
        m->peer_logits[r] = (const float *)((const uint8_t *)bases[r] + m->mail_logits_off);
    }
    v.rank = m->tp_rank;
    v.world = m->tp_world;
    v.stride = m->mail_stride;
    v.seq = m->tp_seq;
    v.wait_ns = (unsigned long long)wait_ms * 1000000ull;
    v.err = device_error_ptr();
    m->tp_ready = true;
    return 0;
}

/* Every rank's mailbox handle in rank order (this rank's own entry is ignored). */
int spk_model_tp_attach(spk_model *m, const void *handles, int n, int wait_ms) {
    if (!m || m->tp_world < 2) return set_error("the model is not tensor-parallel");
    if (m->exec || m->eager_steps || m->tp_ready) return set_error("attach before the first step, once");
    const int hs = (int)sizeof(cudaIpcMemHandle_t);
    if (!handles || n != hs * m->tp_world) return set_error("expected %d handles of %d bytes", m->tp_world, hs);
    void *bases[TP_MAX] = {};
    for (int r = 0; r < m->tp_world; r++) {
        if (r == m->tp_rank) {
            bases[r] = m->mailbox;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, (const uint8_t *)handles + (size_t)r * hs, hs);
        cudaError_t e = cudaIpcOpenMemHandle(&bases[r], h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return cuda_fail("open a peer mailbox", e);
        m->peer_open[r] = bases[r];
    }
    return tp_wire(m, bases, wait_ms);
}

/* Mailboxes as pointers valid in this process, rank order; mailboxes[tp_rank] must be
 * this model's own (pass NULL there to have it filled in). */
int spk_model_tp_attach_ptrs(spk_model *m, void *const *mailboxes, int world, int wait_ms) {
    if (!m || m->tp_world < 2) return set_error("the model is not tensor-parallel");
    if (m->exec || m->eager_steps || m->tp_ready) return set_error("attach before the first step, once");
    if (!mailboxes || world != m->tp_world) return set_error("expected %d mailboxes", m->tp_world);
    void *bases[TP_MAX] = {};
    for (int r = 0; r < world; r++) {
        bases[r] = r == m->tp_rank ? m->mailbox : mailboxes[r];
        if (!bases[r]) return set_error("mailbox %d is null", r);
        if (r == m->tp_rank && mailboxes[r] && mailboxes[r] != m->mailbox) return set_error("mailbox %d is not this model's", r);
    }
    return tp_wire(m, bases, wait_ms);
}

/* This model's mailbox (for spk_model_tp_attach_ptrs in a single-process setup). */
void *spk_model_tp_mailbox(spk_model *m) { return m ? m->mailbox : nullptr; }

}  // extern "C"
