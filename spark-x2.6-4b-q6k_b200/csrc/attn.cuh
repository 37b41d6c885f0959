// attn.cuh — GQA decode attention over the KV cache (model.rs:508-557), for one
// token or a verify batch of up to 8 consecutive tokens.
#pragma once
#include "common.cuh"

namespace spk {

constexpr int ATT_MAX_GROUP = 4;     // q heads per KV head
constexpr int ATT_MAX_SPLIT = 256;   // sequence splits per KV head
constexpr int ATT_MAX_TOK = 8;

// KV cache row of head_dim values, by cache type:
//   KV_F32  hd f32   (the reference runtimes' cache)
//   KV_F16  hd f16
//   KV_Q8   ggml's q8_0 rule per 32 values (d = max|x| / 127 stored as f16, q = round(x / d)),
//           stored planar so every lane's quants load aligned: [hd int8 q][hd/32 f16 d]
enum : int { KV_F32 = 0, KV_F16 = 1, KV_Q8 = 2 };
__host__ __device__ constexpr size_t kv_row_bytes(int type, int hd) {
    return type == KV_F32 ? (size_t)hd * 4 : type == KV_F16 ? (size_t)hd * 2 : (size_t)hd + (size_t)hd / 16;
}

struct AttnArgs {
    const float *qkv;          // [ntok][ldqkv]: q (heads*hd) | k (kv_heads*hd) | v, pre-rope
    int ldqkv;
    void *kc, *vc;             // this layer's caches: [kv_heads][slots] rows of kv_row_bytes(kv_type, hd)
    int kv_type;
    int slots;                 // cache positions
    int full, window;
    const float *freq;         // [pdim/2] rope frequencies of this layer type (model.rs:416-429)
    int pdim;
    int heads, kv_heads, hd;   // this rank's heads
    const int *pos;            // device position of token 0; token t sits at pos + t
    int ntok;                  // grid.z
    int store;                 // 1: the kernel writes each token's K/V row itself (ntok 1)
    int span;                  // 0: causal rows; > 0: every row reads [pos0 + 1 - window, pos0 + span - 1]
    int cached_before;         // 1: every cache row but the own one was written by an earlier graph launch
                               // (a non-causal draft block whose rows sit at pos0 .. pos0 + span - 1)
    int nsplit;                // grid.y: sequence splits
    float *part;               // [ntok][kv_heads][nsplit][group][hd + 4]: o, m, l (+2 pad) per split
    unsigned int *count;       // [ntok][kv_heads], zero; the last split of each resets its own
    const float *gate;         // [ntok][ldgate] g_proj output (pre-sigmoid)
    int ldgate;
    float *out;                // [ntok][ldout] sigmoid(g_h) * softmax(q_h K^T / sqrt(hd)) V
    int ldout;
    int *err;
};

// Split-K flash-decode with the merge in the last CTA of every (token, KV head).
int attn_decode(const AttnArgs &a, cudaStream_t s);

// Rope K and store K/V rows of a batch of ntok tokens (before attn_decode with store 0).
int attn_store_batch(const AttnArgs &a, cudaStream_t s);

// Store the rows of positions pos0 .. pos0 + n - 1 for cache heads 0 .. kv_heads - 1, read
// from f32 rows k / v [n][ld] at head offsets (head0 + h) * hd (already roped keys), by
// the cache type's rule.
int kv_write(void *kc, void *vc, int kv_type, int slots, int kv_heads, int head0, int hd, int pos0, int n,
             const float *k, const float *v, int ld, cudaStream_t s);

}  // namespace spk
