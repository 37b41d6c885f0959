// attn.cu — GQA decode attention (model.rs:508-557) on B200.
//
// One CTA = one (token, KV head, sequence split). It ropes the token's q heads of
// the KV head's group and its k (model.rs:431-439), and — for a single token —
// the CTA whose split holds the token's own position writes the new K/V row. Its
// 8 warps walk the split's positions 4 at a time (4 independent K/V row loads
// per warp in flight: the loop is latency-bound, not compute-bound), form the
// group's scores with butterfly sums and keep an online softmax per q head. The
// warps merge in shared memory into the split's (o, m, l), and the last split of
// each (token, KV head) to finish — an atomic ticket — merges all splits in a
// fixed order and applies the per-head sigmoid gate (model.rs:538-550). The
// ticket is reset by that CTA, so a captured graph replays without a memset.
#include <cooperative_groups.h>

#include "attn.cuh"
#include "spk.h"

namespace spk {
namespace {

constexpr int ATT_THREADS = 256;
constexpr int ATT_WARPS = ATT_THREADS / 32;

// NeoX rotate-half on the first pdim elements of x (shared memory), model.rs:431-439:
//   x[i] = a cos - b sin ; x[i+half] = b cos + a sin, each product rounded.
__device__ void rope_smem(float *x, const float *freq, int pdim, int pos) {
    const int half = pdim / 2;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float ang = __fmul_rn((float)pos, freq[i]);
        const float c = cosf(ang), s = sinf(ang);
        const float a = x[i], b = x[i + half];
        x[i] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        x[i + half] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
    }
}

// The same rotation on the G query heads and the key of one token at once: the angle of a
// dims pair depends only on the pair, so its cosine and sine are computed once for all G + 1
// vectors (each element's arithmetic is rope_smem's). fi: freq[threadIdx.x], loaded by the
// caller together with the vectors (its first pair), so its latency overlaps theirs.
__device__ void rope_group(float (*q)[256], int G, float *k, const float *freq, float fi, int pdim, int pos) {
    const int half = pdim / 2;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float ang = __fmul_rn((float)pos, i == (int)threadIdx.x ? fi : freq[i]);
        const float c = cosf(ang), s = sinf(ang);
        for (int h = 0; h <= G; h++) {
            float *x = h < G ? q[h] : k;
            const float a = x[i], b = x[i + half];
            x[i] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
            x[i + half] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
        }
    }
}

// This lane's DPL dims (lane*DPL ..) of one cache row of HD values, as f32.
template <int HD, int DPL, int KT>
__device__ __forceinline__ void load_row(const uint8_t *row, int lane, float (&r)[DPL]) {
    if constexpr (KT == KV_F16) {
        const __half *p = reinterpret_cast<const __half *>(row) + lane * DPL;
        if constexpr (DPL == 8) {
            const uint4 w = *reinterpret_cast<const uint4 *>(p);
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&ws[i]));
                r[2 * i] = f.x;
                r[2 * i + 1] = f.y;
            }
        } else {
            const uint2 w = *reinterpret_cast<const uint2 *>(p);
            const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&w.x));
            const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&w.y));
            r[0] = f0.x;
            r[1] = f0.y;
            r[2] = f1.x;
            r[3] = f1.y;
        }
    } else if constexpr (KT == KV_Q8) {
        // quants at row[0 .. HD), the f16 scale of 32-value block b at row[HD + 2b]
        const float d = __half2float(reinterpret_cast<const __half *>(row + HD)[(lane * DPL) / 32]);
        uint32_t w[DPL / 4];
        if constexpr (DPL == 8) {
            const uint2 v = *reinterpret_cast<const uint2 *>(row + lane * DPL);
            w[0] = v.x;
            w[1] = v.y;
        } else {
            w[0] = *reinterpret_cast<const uint32_t *>(row + lane * DPL);
        }
#pragma unroll
        for (int i = 0; i < DPL; i++) r[i] = (float)(int8_t)(w[i >> 2] >> (8 * (i & 3))) * d;
    } else {
        const float4 *p = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(row) + lane * DPL);
#pragma unroll
        for (int i = 0; i < DPL / 4; i++) {
            const float4 f = p[i];
            r[4 * i] = f.x;
            r[4 * i + 1] = f.y;
            r[4 * i + 2] = f.z;
            r[4 * i + 3] = f.w;
        }
    }
}

// Store one row of hd values from shared memory into the cache, by all threads of
// the block. q8_0 follows ggml's quantize_row_q8_0 rule: per 32 values
// d = max|x| / 127, q = roundf(x * (1/d)) (0 when d is 0), d kept as f16.
template <int KT>
__device__ void store_row(const float *src, uint8_t *row, int hd) {
    if constexpr (KT == KV_Q8) {
        for (int b = threadIdx.x; b < hd / 32; b += blockDim.x) {
            float amax = 0.f;
            for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(src[32 * b + j]));
            const float d = amax / 127.0f, id = d != 0.f ? 1.0f / d : 0.0f;
            reinterpret_cast<__half *>(row + hd)[b] = __float2half_rn(d);
            for (int j = 0; j < 32; j++) row[32 * b + j] = (uint8_t)(int8_t)roundf(src[32 * b + j] * id);
        }
    } else {
        for (int i = threadIdx.x; i < hd; i += blockDim.x) {
            if (KT == KV_F16)
                reinterpret_cast<__half *>(row)[i] = __float2half_rn(src[i]);
            else
                reinterpret_cast<float *>(row)[i] = src[i];
        }
    }
}

// The split's partial is written; the last split of this (token, KV head) to finish
// (an atomic ticket, reset by it) merges all splits in a fixed order and applies the
// per-head sigmoid gate (model.rs:538-550).
template <int HD>
__device__ void finish_splits(const AttnArgs &a, int kvh, int tok, int G, size_t pbase, size_t pstride,
                              float (*cw)[ATT_MAX_SPLIT], float *cl, int *is_last_p) {
    constexpr int PR = HD + 4;
    int &is_last = *is_last_p;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __threadfence();
    __syncthreads();
    unsigned int *ticket = a.count + (size_t)tok * a.kv_heads + kvh;
    if (threadIdx.x == 0) is_last = atomicAdd(ticket, 1u) == (unsigned int)(a.nsplit - 1);
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const float *p0 = a.part + pbase * pstride;
    for (int i = threadIdx.x; i < G * a.nsplit; i += blockDim.x) {
        const int h = i / a.nsplit, c = i - h * a.nsplit;
        cw[h][c] = __ldcg(p0 + c * pstride + h * PR + HD);
    }
    __syncthreads();
    if (warp < G) {   // warp h: the split weights e^{m_c - M} and the total L of head h
        const int h = warp;
        float M = -INFINITY;
        for (int c = lane; c < a.nsplit; c += 32) M = fmaxf(M, cw[h][c]);
        for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
        float L = 0.f;
        for (int c = lane; c < a.nsplit; c += 32) {
            const float mc = cw[h][c];
            const float e = mc == -INFINITY ? 0.f : expf(mc - M);
            L += __ldcg(p0 + c * pstride + h * PR + HD + 1) * e;
            cw[h][c] = e;
        }
        L = warp_sum(L);
        if (lane == 0) cl[h] = L;
    }
    __syncthreads();
    // one thread per 4 output dims, 8 float4 loads in flight per thread
    for (int i = threadIdx.x; i < G * (HD / 4); i += blockDim.x) {
        const int h = i / (HD / 4), d4 = i - h * (HD / 4);
        const float *ph = p0 + h * PR + 4 * d4;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
        for (int c = 0; c < a.nsplit; c++) {
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(ph + c * pstride));
            const float w = cw[h][c];
            O.x = fmaf(v.x, w, O.x);
            O.y = fmaf(v.y, w, O.y);
            O.z = fmaf(v.z, w, O.z);
            O.w = fmaf(v.w, w, O.w);
        }
        const int qh = kvh * G + h;
        const float gsig = 1.0f / (1.0f + expf(-a.gate[(size_t)tok * a.ldgate + qh]));
        float *dst = a.out + (size_t)tok * a.ldout + (size_t)qh * HD + 4 * d4;
        dst[0] = (O.x / cl[h]) * gsig;
        dst[1] = (O.y / cl[h]) * gsig;
        dst[2] = (O.z / cl[h]) * gsig;
        dst[3] = (O.w / cl[h]) * gsig;
    }
    if (threadIdx.x == 0) *ticket = 0u;
}

// ATT_U: positions per warp per iteration (4 for long splits, 2 for short ones so
// that all 8 warps have a position).
template <int HD, int KT, int ATT_U>
__global__ void __launch_bounds__(ATT_THREADS) attn_kernel(const AttnArgs a) {
    constexpr int DPL = HD / 32;   // dims per lane
    constexpr size_t RB = kv_row_bytes(KT, HD);
    constexpr int MG = ATT_MAX_GROUP;
    __shared__ float qs[MG][HD];
    __shared__ float kn[HD], vn[HD];
    __shared__ float wm[ATT_WARPS][MG], wl[ATT_WARPS][MG];
    __shared__ float wo[ATT_WARPS][MG][HD];
    __shared__ float cw[MG][ATT_MAX_SPLIT];
    __shared__ float cl[MG];
    __shared__ int is_last;
    pdl_trigger();
    pdl_wait();
    const int kvh = blockIdx.x, split = blockIdx.y, tok = blockIdx.z;
    const int G = a.heads / a.kv_heads;
    const int qd = a.heads * HD, kvd = a.kv_heads * HD;
    const int pos = *a.pos + tok;
    // causal: token t reads [start, pos]; a block (span > 0) reads the anchor row's keys,
    // the window before pos0 and the block's span rows, whatever its own row
    const int last = a.span > 0 ? *a.pos + a.span - 1 : pos;
    const int start = a.full ? 0 : max(0, (a.span > 0 ? *a.pos : pos) + 1 - a.window);
    const int n = last + 1 - start;
    const int csz = max((n + a.nsplit - 1) / a.nsplit, 16);
    const int c0 = start + split * csz, c1 = min(last + 1, c0 + csz);
    const float *qrow = a.qkv + (size_t)tok * a.ldqkv;
    const size_t pbase = ((size_t)tok * a.kv_heads + kvh) * a.nsplit;   // this (token, KV head)'s splits
    constexpr int PR = HD + 4;   // a partial row: o[HD], m, l, 2 pad (16-byte rows)
    const size_t pstride = (size_t)G * PR;
    float *out = a.part + (pbase + split) * pstride;

    for (int i = threadIdx.x; i < G * HD; i += blockDim.x) qs[i / HD][i % HD] = qrow[(size_t)(kvh * G + i / HD) * HD + i % HD];
    for (int i = threadIdx.x; i < HD; i += blockDim.x) {
        kn[i] = qrow[qd + (size_t)kvh * HD + i];
        vn[i] = qrow[qd + kvd + (size_t)kvh * HD + i];
    }
    __syncthreads();
    for (int h = 0; h < G; h++) rope_smem(qs[h], a.freq, a.pdim, pos);
    rope_smem(kn, a.freq, a.pdim, pos);
    __syncthreads();
    // a single token's own K/V row: written by the split that owns `pos`; nobody reads that slot now
    if (a.store && c0 <= pos && pos < c1) {
        const size_t o = ((size_t)kvh * a.slots + pos % a.slots) * RB;
        store_row<KT>(kn, reinterpret_cast<uint8_t *>(a.kc) + o, HD);
        store_row<KT>(vn, reinterpret_cast<uint8_t *>(a.vc) + o, HD);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (c0 < c1) {
        float q[MG][DPL], o[MG][DPL], m[MG], l[MG];
        const float scale = 1.0f / sqrtf((float)HD);
#pragma unroll
        for (int h = 0; h < MG; h++) {
            m[h] = -INFINITY;
            l[h] = 0.f;
#pragma unroll
            for (int d = 0; d < DPL; d++) {
                q[h][d] = h < G ? qs[h][lane * DPL + d] : 0.f;
                o[h][d] = 0.f;
            }
        }
        for (int j0 = c0 + warp * ATT_U; j0 < c1; j0 += ATT_WARPS * ATT_U) {
            float kr[ATT_U][DPL], vr[ATT_U][DPL];
#pragma unroll
            for (int u = 0; u < ATT_U; u++) {
                const int j = j0 + u;
                if (j >= c1) {
#pragma unroll
                    for (int d = 0; d < DPL; d++) kr[u][d] = vr[u][d] = 0.f;
                } else if (j == pos && a.span == 0) {   // this token's own row: f32, before the cache's rounding
#pragma unroll
                    for (int d = 0; d < DPL; d++) {
                        kr[u][d] = kn[lane * DPL + d];
                        vr[u][d] = vn[lane * DPL + d];
                    }
                } else {
                    const size_t o = ((size_t)kvh * a.slots + j % a.slots) * RB;
                    load_row<HD, DPL, KT>(reinterpret_cast<const uint8_t *>(a.kc) + o, lane, kr[u]);
                    load_row<HD, DPL, KT>(reinterpret_cast<const uint8_t *>(a.vc) + o, lane, vr[u]);
                }
            }
            float s[ATT_U][MG];
#pragma unroll
            for (int u = 0; u < ATT_U; u++)
#pragma unroll
                for (int h = 0; h < MG; h++) {
                    float t = 0.f;
#pragma unroll
                    for (int d = 0; d < DPL; d++) t = fmaf(q[h][d], kr[u][d], t);
                    s[u][h] = t;
                }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                for (int u = 0; u < ATT_U; u++)
#pragma unroll
                    for (int h = 0; h < MG; h++) s[u][h] += __shfl_xor_sync(0xffffffffu, s[u][h], off);
#pragma unroll
            for (int h = 0; h < MG; h++) {
                if (h >= G) break;
                float mx = -INFINITY;
#pragma unroll
                for (int u = 0; u < ATT_U; u++)
                    if (j0 + u < c1) mx = fmaxf(mx, s[u][h] * scale);
                const float mn = fmaxf(m[h], mx);
                const float corr = expf(m[h] - mn);
                float p[ATT_U], ps = 0.f;
#pragma unroll
                for (int u = 0; u < ATT_U; u++) {
                    p[u] = j0 + u < c1 ? expf(s[u][h] * scale - mn) : 0.f;
                    ps += p[u];
                }
                l[h] = l[h] * corr + ps;
#pragma unroll
                for (int d = 0; d < DPL; d++) {
                    float v = o[h][d] * corr;
#pragma unroll
                    for (int u = 0; u < ATT_U; u++) v = fmaf(p[u], vr[u][d], v);
                    o[h][d] = v;
                }
                m[h] = mn;
            }
        }
        // merge the warps into this split's (o, m, l)
        if (lane == 0)
            for (int h = 0; h < G; h++) {
                wm[warp][h] = m[h];
                wl[warp][h] = l[h];
            }
        for (int h = 0; h < G; h++)
#pragma unroll
            for (int d = 0; d < DPL; d++) wo[warp][h][lane * DPL + d] = o[h][d];
        __syncthreads();
        for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
            const int h = i / HD, d = i % HD;
            float M = -INFINITY;
            for (int w = 0; w < ATT_WARPS; w++) M = fmaxf(M, wm[w][h]);
            float L = 0.f, O = 0.f;
            for (int w = 0; w < ATT_WARPS; w++) {
                if (wm[w][h] == -INFINITY) continue;
                const float e = expf(wm[w][h] - M);
                L += wl[w][h] * e;
                O += wo[w][h][d] * e;
            }
            out[h * PR + d] = O;
            if (d == 0) {
                out[h * PR + HD] = M;
                out[h * PR + HD + 1] = L;
            }
        }
    } else {   // an empty split: weight 0 in the merge
        for (int i = threadIdx.x; i < G * PR; i += blockDim.x) out[i] = (i % PR) == HD ? -INFINITY : 0.f;
    }
    finish_splits<HD>(a, kvh, tok, G, pbase, pstride, cw, cl, &is_last);
}

// Rope K and store the K/V rows of ntok consecutive tokens: block t = token t.
template <int KT>
__global__ void attn_store_kernel(const AttnArgs a) {
    extern __shared__ float ks[];   // [2][kv_heads * hd]: roped k, then v
    pdl_trigger();
    pdl_wait();
    const int tok = blockIdx.x, pos = *a.pos + tok;
    const int qd = a.heads * a.hd, kvd = a.kv_heads * a.hd;
    const float *row = a.qkv + (size_t)tok * a.ldqkv;
    for (int i = threadIdx.x; i < 2 * kvd; i += blockDim.x) ks[i] = row[qd + i];
    __syncthreads();
    for (int h = 0; h < a.kv_heads; h++) rope_smem(ks + (size_t)h * a.hd, a.freq, a.pdim, pos);
    __syncthreads();
    const size_t RB = kv_row_bytes(KT, a.hd);
    for (int h = 0; h < a.kv_heads; h++) {
        const size_t o = ((size_t)h * a.slots + pos % a.slots) * RB;
        store_row<KT>(ks + (size_t)h * a.hd, reinterpret_cast<uint8_t *>(a.kc) + o, a.hd);
        store_row<KT>(ks + kvd + (size_t)h * a.hd, reinterpret_cast<uint8_t *>(a.vc) + o, a.hd);
    }
}


// ===================================================== tensor-core decode ===
// The same (token, KV head, split) grid for head_dim 256 over an f16 cache, with the
// contractions on the tensor cores (mma.sync m16n8k16 f16 -> f32):
//  * K and V rows of 64 positions per stage arrive by cp.async (16 bytes a thread,
//    zero-filled past the split) into two slots of 544-byte rows (padded: no bank
//    conflicts); each 16-position tile of a stage goes to a pair of warps, which both
//    form its scores and softmax and split the PV product's 256 dims (8 warps a CTA).
//  * S^T = K q^T: K rows are the A operand (positions as rows; a thread's four k-slots
//    are four consecutive dims, one 8-byte load), B holds the group's q heads as an
//    f16 pair, hi in columns 0..3 and lo in 4..7, so one MMA per 16 dims gives ~22-bit
//    scores; hi and lo meet by one shuffle.
//  * the online softmax per head (model.rs:519-553 order of terms: s * scale, exp(s - m)),
//    the lanes holding a head's scores also holding its O^T columns;
//  * O^T += V^T P^T: V^T by ldmatrix.trans, P as an f16 pair again (hi / lo columns).
// The token's own row (the SIMT kernel's exact f32 row) is masked in the tiles and
// enters the CTA merge as a fifth, exact f32 term.
// q8_0 cache: K quants convert to f16 exactly at use, each 32-dim block's two k-steps
// into a fresh accumulator scaled by that row's d; V quants are converted once per stage
// into the padded f16 tile, and V's per-block scale multiplies P instead (one B operand
// per 32-dim block), so every product stays exact.
constexpr int TC_WARPS = 8, TC_THREADS = TC_WARPS * 32;
constexpr int TC_POS = 64;                       // positions per stage
constexpr int TC_TILES = TC_POS / 16;            // 16-position tiles per stage, two warps each
constexpr int TC_RS = 256 * 2 + 32;              // shared-memory bytes of an f16 K or V row (padded)
constexpr int TC_RS8 = 256 + 16;                 // a q8_0 row as cached (272 bytes: conflict-free as is)
template <int KT>
struct TcLayout {
    static constexpr int KRS = KT == KV_Q8 ? TC_RS8 : TC_RS;   // K row stride in a slot
    static constexpr int CH = KT == KV_Q8 ? TC_RS8 / 16 : 32;  // 16-byte chunks per cached row
    static constexpr int SLOT = 2 * TC_POS * KRS;               // K then V rows as loaded
    static constexpr size_t SMEM = (size_t)2 * SLOT + (KT == KV_Q8 ? (size_t)TC_POS * TC_RS : 0);   // + f16 V
};

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma_f16_tc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four int8 of w as two exact f16 pairs (bytes 0,1 | bytes 2,3), low half first:
// byte ^ 0x80 under the exponent of 1024 (0x64bb == 1024 + bb), minus 1152.
__device__ __forceinline__ void s8x4_to_f16_exact(uint32_t w, uint32_t &lo, uint32_t &hi) {
    const uint32_t b = w ^ 0x80808080u;
    uint32_t l = __byte_perm(b, 0x64646464u, 0x5140u), h = __byte_perm(b, 0x64646464u, 0x7362u);
    const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6480u));
    const __half2 lv = __hsub2(*reinterpret_cast<__half2 *>(&l), bias);
    const __half2 hv = __hsub2(*reinterpret_cast<__half2 *>(&h), bias);
    lo = *reinterpret_cast<const uint32_t *>(&lv);
    hi = *reinterpret_cast<const uint32_t *>(&hv);
}

// (x, y) as an f16 pair: the hi parts rn(x), rn(y), or the lo parts rn(x - hi), rn(y - hi).
__device__ __forceinline__ uint32_t f16_pair(float x, float y, bool lo) {
    const __half hx = __float2half_rn(x), hy = __float2half_rn(y);
    const __half ox = lo ? __float2half_rn(x - __half2float(hx)) : hx;
    const __half oy = lo ? __float2half_rn(y - __half2float(hy)) : hy;
    return (uint32_t)__half_as_ushort(ox) | ((uint32_t)__half_as_ushort(oy) << 16);
}

// CL: the splits of a (token, KV head) run as one thread-block cluster (grid.y = nsplit <= 8 =
// the cluster's size) and CTA r owns output dims r * dpc .. (dpc = HD / nsplit): each split
// stores its (o, m, l) for those dims straight into CTA r's shared memory (distributed shared
// memory stores, which do not wait for an answer) and, after one cluster barrier, every CTA
// merges its own dims from its own shared memory: no global round trip, no ticket, no remote
// load.
template <int KT, bool CL>
__global__ void __launch_bounds__(TC_THREADS, 1) attn_tc_kernel(const AttnArgs a) {
    constexpr int HD = 256, MG = ATT_MAX_GROUP, PR = HD + 4, NW = TC_TILES + 1;
    constexpr size_t RB = kv_row_bytes(KT, HD);
    using TL = TcLayout<KT>;
    constexpr bool Q8 = KT == KV_Q8;
    extern __shared__ __align__(16) uint8_t tsm[];
    __shared__ float qs[MG][HD];
    __shared__ float kn[HD], vn[HD];
    __shared__ float wm[NW][MG], wl[NW][MG];
    __shared__ float wo[NW][MG][HD];
    __shared__ float pt[TC_WARPS][16][MG];   // each warp's P, transposed for the B operand
    __shared__ float cw[MG][CL ? 1 : ATT_MAX_SPLIT];
    __shared__ float cl[MG];
    __shared__ int is_last;
    // CL: every split's (o for this CTA's dims, m, l) per head, [split][head][dpc + 2]
    __shared__ float mrg[CL ? MG * (HD + 2 * 8) : 1];
    __shared__ float gs[MG];                          // CL: the heads' sigmoid gates
    __shared__ float we[NW][MG], wml[MG][2];          // the merge's per-(tile, head) weights, per-head (M, L)
    __shared__ float cwt[CL ? 8 : 1][MG];             // CL: the splits' per-head weights
    pdl_trigger();
    if constexpr (CL)   // first half of the barrier that shows every CTA of the cluster runs
        asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    // The model's decode step (one token storing its own row, cached_before set) reads only
    // cache rows written by earlier graph launches, which run one after another, plus its own
    // row, which the score masks: its first K/V stages are issued before the wait for the
    // previous kernel. Every other caller (the verify batch reads rows its preceding kernel
    // stored) waits first.
    const bool early = a.cached_before && a.store && a.span == 0 && a.ntok == 1;
    if (!early) pdl_wait();
    const int kvh = blockIdx.x, split = blockIdx.y, tok = blockIdx.z;
    const int G = a.heads / a.kv_heads;
    const int qd = a.heads * HD, kvd = a.kv_heads * HD;
    const int pos = *a.pos + tok;
    const int last = a.span > 0 ? *a.pos + a.span - 1 : pos;
    const int start = a.full ? 0 : max(0, (a.span > 0 ? *a.pos : pos) + 1 - a.window);
    const int n = last + 1 - start;
    const int csz = max((n + a.nsplit - 1) / a.nsplit, 16);
    const int c0 = start + split * csz, c1 = min(last + 1, c0 + csz);
    const float *qrow = a.qkv + (size_t)tok * a.ldqkv;
    const size_t pbase = ((size_t)tok * a.kv_heads + kvh) * a.nsplit;
    const size_t pstride = (size_t)G * PR;
    float *out = a.part + (pbase + split) * pstride;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int tw = warp % TC_TILES, dh = warp / TC_TILES;   // the warp's tile of a stage and its PV dims half

    const uint8_t *kbase = reinterpret_cast<const uint8_t *>(a.kc) + (size_t)kvh * a.slots * RB;
    const uint8_t *vbase = reinterpret_cast<const uint8_t *>(a.vc) + (size_t)kvh * a.slots * RB;
    const int nstage = c0 < c1 ? (c1 - c0 + TC_POS - 1) / TC_POS : 0;
    auto issue = [&](int st, int slot) {
        uint8_t *kd = tsm + (size_t)slot * TL::SLOT, *vd = kd + TC_POS * TL::KRS;
        const int js = c0 + st * TC_POS;
        for (int i = threadIdx.x; i < TC_POS * TL::CH; i += TC_THREADS) {   // 16-byte chunks of the rows
            const int r = i / TL::CH, c = i - r * TL::CH, j = js + r;
            const bool v = j < c1;
            const size_t off = (size_t)((v ? j : c0) % a.slots) * RB + 16 * c;
            cp_async16(kd + r * TL::KRS + 16 * c, kbase + off, v);
            cp_async16(vd + r * TL::KRS + 16 * c, vbase + off, v);
        }
        cp_async_commit();
    };
    if (early) {
        if (nstage > 0) issue(0, 0);
        else cp_async_commit();
        if (nstage > 1) issue(1, 1);
        else cp_async_commit();
        pdl_wait();
    }

    const float fi = (int)threadIdx.x < a.pdim / 2 ? a.freq[threadIdx.x] : 0.f;
    for (int i = threadIdx.x; i < MG * HD; i += blockDim.x)
        qs[i / HD][i % HD] = i / HD < G ? qrow[(size_t)(kvh * G + i / HD) * HD + i % HD] : 0.f;
    for (int i = threadIdx.x; i < HD; i += blockDim.x) {
        kn[i] = qrow[qd + (size_t)kvh * HD + i];
        vn[i] = qrow[qd + kvd + (size_t)kvh * HD + i];
    }
    if (CL && threadIdx.x < G)   // the heads' gates (model.rs:538-550), loaded with q
        gs[threadIdx.x] = 1.0f / (1.0f + expf(-a.gate[(size_t)tok * a.ldgate + kvh * G + threadIdx.x]));
    __syncthreads();
    rope_group(qs, G, kn, a.freq, fi, a.pdim, pos);
    __syncthreads();
    if (a.store && c0 <= pos && pos < c1) {   // a single token's own row; nobody reads that slot now
        const size_t o = ((size_t)kvh * a.slots + pos % a.slots) * RB;
        store_row<KT>(kn, reinterpret_cast<uint8_t *>(a.kc) + o, HD);
        store_row<KT>(vn, reinterpret_cast<uint8_t *>(a.vc) + o, HD);
    }
    const bool own = a.span == 0 && c0 <= pos && pos < c1;   // exact f32 own row: masked below
    const float scale = 1.0f / sqrtf((float)HD);

    // B fragments of q for the 16 k-steps: column g = head g & 3, hi (g < 4) or lo part
    uint32_t qb[16][2];
#pragma unroll
    for (int ks = 0; ks < 16; ks++) {
        const float *qh = qs[g & 3] + 16 * ks + 4 * t;
        qb[ks][0] = f16_pair(qh[0], qh[1], g >= 4);
        qb[ks][1] = f16_pair(qh[2], qh[3], g >= 4);
    }
    float o[8][4];   // O^T for dims 128 dh .. 128 dh + 127: m-tiles 8 dh + i
#pragma unroll
    for (int i = 0; i < 8; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;   // heads 2(t&1), 2(t&1)+1

    if (!early) {
        if (nstage > 0) issue(0, 0);
        else cp_async_commit();
        if (nstage > 1) issue(1, 1);
        else cp_async_commit();
    }
    const int vpos = (lane & 7) + ((lane >> 4) << 3), vdim = ((lane >> 3) & 1) * 8;   // ldmatrix.trans rows
    for (int st = 0; st < nstage; st++) {
        cp_async_wait<1>();
        __syncthreads();   // stage st landed for every thread
        uint8_t *kt = tsm + (size_t)(st & 1) * TL::SLOT, *vraw = kt + TC_POS * TL::KRS;
        const uint8_t *vt = vraw;   // the f16 V tile ldmatrix reads
        // The token's own row enters the merge exactly (below) and its score is masked, but the
        // tile may hold what the slot held before this step's store (a row from before a rollback,
        // possibly an overflowed f16): its V values (f16) or V scales (q8_0) are zeroed here so
        // the masked P = 0 never meets an Inf or NaN in the PV product.
        const int jo = own ? pos - (c0 + st * TC_POS) : -1;
        const bool zown = jo >= 0 && jo < TC_POS;   // the same for every thread of the CTA
        if constexpr (Q8) {   // V quants -> the f16 tile (exact); the scales stay in the raw rows
            uint8_t *v16 = tsm + (size_t)2 * TL::SLOT;
            for (int i = threadIdx.x; i < TC_POS * (HD / 4); i += TC_THREADS) {
                const int r = i / (HD / 4), w = i - r * (HD / 4);
                uint32_t lo, hi;
                s8x4_to_f16_exact(*reinterpret_cast<const uint32_t *>(vraw + (size_t)r * TL::KRS + 4 * w), lo, hi);
                *reinterpret_cast<uint2 *>(v16 + (size_t)r * TC_RS + 8 * w) = make_uint2(lo, hi);
            }
            if (zown && threadIdx.x < HD / 32)
                reinterpret_cast<__half *>(vraw + (size_t)jo * TL::KRS + HD)[threadIdx.x] = __ushort_as_half(0);
            __syncthreads();
            vt = v16;
        } else if (zown) {
            if (threadIdx.x < HD / 8)
                *reinterpret_cast<uint4 *>(vraw + (size_t)jo * TL::KRS + 16 * threadIdx.x) = make_uint4(0, 0, 0, 0);
            __syncthreads();
        }
        const int jw = c0 + st * TC_POS + 16 * tw;   // this warp's first position
        if (jw < c1) {
            float sc[4] = {0.f, 0.f, 0.f, 0.f};
            if constexpr (Q8) {
                const uint8_t *ra = kt + (size_t)(16 * tw + g) * TL::KRS, *rb8 = ra + (size_t)8 * TL::KRS;
#pragma unroll
                for (int b = 0; b < HD / 32; b++) {
                    float sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int kk = 0; kk < 2; kk++) {
                        const int ks = 2 * b + kk;
                        uint32_t a0, a1, a2, a3;
                        s8x4_to_f16_exact(*reinterpret_cast<const uint32_t *>(ra + 16 * ks + 4 * t), a0, a2);
                        s8x4_to_f16_exact(*reinterpret_cast<const uint32_t *>(rb8 + 16 * ks + 4 * t), a1, a3);
                        mma_f16_tc(sb, a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
                    }
                    const float da = __half2float(reinterpret_cast<const __half *>(ra + HD)[b]);
                    const float db = __half2float(reinterpret_cast<const __half *>(rb8 + HD)[b]);
                    sc[0] = fmaf(da, sb[0], sc[0]);
                    sc[1] = fmaf(da, sb[1], sc[1]);
                    sc[2] = fmaf(db, sb[2], sc[2]);
                    sc[3] = fmaf(db, sb[3], sc[3]);
                }
            } else {
                const uint8_t *ra = kt + (size_t)(16 * tw + g) * TC_RS + 8 * t, *rb8 = ra + (size_t)8 * TC_RS;
#pragma unroll
                for (int ks = 0; ks < 16; ks++) {
                    const uint2 ka = *reinterpret_cast<const uint2 *>(ra + 32 * ks);
                    const uint2 kb = *reinterpret_cast<const uint2 *>(rb8 + 32 * ks);
                    mma_f16_tc(sc, ka.x, kb.x, ka.y, kb.y, qb[ks][0], qb[ks][1]);
                }
            }
#pragma unroll
            for (int e = 0; e < 4; e++) sc[e] += __shfl_xor_sync(0xffffffffu, sc[e], 2);   // hi + lo
            const int p0 = jw + g, p1 = jw + g + 8;
            const bool v0 = p0 < c1 && !(own && p0 == pos), v1 = p1 < c1 && !(own && p1 == pos);
            const float s0 = v0 ? sc[0] * scale : -INFINITY, s1 = v0 ? sc[1] * scale : -INFINITY;
            const float s2 = v1 ? sc[2] * scale : -INFINITY, s3 = v1 ? sc[3] * scale : -INFINITY;
            float xA = fmaxf(s0, s2), xB = fmaxf(s1, s3);
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                xA = fmaxf(xA, __shfl_xor_sync(0xffffffffu, xA, off));
                xB = fmaxf(xB, __shfl_xor_sync(0xffffffffu, xB, off));
            }
            const float nA = fmaxf(mA, xA), nB = fmaxf(mB, xB);
            const float cA = nA == -INFINITY ? 1.f : expf(mA - nA), cB = nB == -INFINITY ? 1.f : expf(mB - nB);
            const float pA0 = v0 ? expf(s0 - nA) : 0.f, pB0 = v0 ? expf(s1 - nB) : 0.f;
            const float pA1 = v1 ? expf(s2 - nA) : 0.f, pB1 = v1 ? expf(s3 - nB) : 0.f;
            float sA = pA0 + pA1, sB = pB0 + pB1;
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                sA += __shfl_xor_sync(0xffffffffu, sA, off);
                sB += __shfl_xor_sync(0xffffffffu, sB, off);
            }
            lA = lA * cA + sA;
            lB = lB * cB + sB;
            mA = nA;
            mB = nB;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                o[i][0] *= cA;
                o[i][1] *= cB;
                o[i][2] *= cA;
                o[i][3] *= cB;
            }
            // P^T as the B operand: row pos, column g (head g & 3, hi / lo), via shared memory
            if (t < 2) {
                pt[warp][g][2 * t] = pA0;
                pt[warp][g][2 * t + 1] = pB0;
                pt[warp][g + 8][2 * t] = pA1;
                pt[warp][g + 8][2 * t + 1] = pB1;
            }
            __syncwarp();
            const int hh = g & 3;
            const float q0 = pt[warp][2 * t][hh], q1 = pt[warp][2 * t + 1][hh];
            const float q2 = pt[warp][2 * t + 8][hh], q3 = pt[warp][2 * t + 9][hh];
            __syncwarp();
            const uint8_t *vr = vt + (size_t)(16 * tw + vpos) * TC_RS + 2 * vdim + 256 * dh;
            if constexpr (Q8) {   // per 32-dim block b: B = (P * d_b) as an f16 pair
                const __half *dr = reinterpret_cast<const __half *>(vraw + (size_t)(16 * tw + 2 * t) * TL::KRS + HD);
                const size_t rs = TL::KRS / 2;   // row stride in halves
#pragma unroll
                for (int bb = 0; bb < 4; bb++) {
                    const int b = 4 * dh + bb;
                    const float d0 = __half2float(dr[b]), d1 = __half2float(dr[rs + b]);
                    const float d8 = __half2float(dr[8 * rs + b]), d9 = __half2float(dr[9 * rs + b]);
                    const uint32_t pb0 = f16_pair(q0 * d0, q1 * d1, g >= 4);
                    const uint32_t pb1 = f16_pair(q2 * d8, q3 * d9, g >= 4);
#pragma unroll
                    for (int i = 2 * bb; i < 2 * bb + 2; i++) {
                        uint32_t av[4];
                        ldsm_x4_trans(av, vr + 32 * i);
                        mma_f16_tc(o[i], av[0], av[1], av[2], av[3], pb0, pb1);
                    }
                }
            } else {
                const uint32_t pb0 = f16_pair(q0, q1, g >= 4), pb1 = f16_pair(q2, q3, g >= 4);
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    uint32_t av[4];
                    ldsm_x4_trans(av, vr + 32 * i);
                    mma_f16_tc(o[i], av[0], av[1], av[2], av[3], pb0, pb1);
                }
            }
        }
        __syncthreads();   // every warp is done with this slot
        if (st + 2 < nstage) issue(st + 2, st & 1);
        else cp_async_commit();
    }
    cp_async_wait<0>();

    // this warp's (o, m, l) for the merge: O[h][dim] = O^T[dim][h] + O^T[dim][h + 4]
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int e = 0; e < 4; e++) o[i][e] += __shfl_xor_sync(0xffffffffu, o[i][e], 2);
    const int hA = 2 * (t & 1), hB = hA + 1;
    if (t < 2) {   // the pair's m, l agree (same scores, same code); each writes its dims half
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int d0 = 128 * dh + 16 * i + g;
            wo[tw][hA][d0] = o[i][0];
            wo[tw][hB][d0] = o[i][1];
            wo[tw][hA][d0 + 8] = o[i][2];
            wo[tw][hB][d0 + 8] = o[i][3];
        }
        if (g == 0 && dh == 0) {
            wm[tw][hA] = mA;
            wm[tw][hB] = mB;
            wl[tw][hA] = lA;
            wl[tw][hB] = lB;
        }
    }
    // the own row, exact in f32 (warp h: head h's score)
    if (warp < MG) {
        const int h = warp;
        float sv = 0.f;
        if (own && h < G)
            for (int d = lane; d < HD; d += 32) sv = fmaf(qs[h][d], kn[d], sv);
        sv = warp_sum(sv);
        if (lane == 0) {
            wm[TC_TILES][h] = own && h < G ? sv * scale : -INFINITY;
            wl[TC_TILES][h] = own && h < G ? 1.f : 0.f;
        }
        for (int d = lane; d < HD; d += 32) wo[TC_TILES][h][d] = own ? vn[d] : 0.f;
    }
    __syncthreads();
    if (threadIdx.x < G) {   // per head: the running max, the tiles' weights e^{m_w - M}, the sum L
        const int h = threadIdx.x;
        float M = -INFINITY;
        for (int w = 0; w < NW; w++) M = fmaxf(M, wm[w][h]);
        float L = 0.f;
        for (int w = 0; w < NW; w++) {
            const float e = wm[w][h] == -INFINITY ? 0.f : expf(wm[w][h] - M);
            if (wm[w][h] != -INFINITY) L += wl[w][h] * e;
            we[w][h] = e;
        }
        wml[h][0] = M;
        wml[h][1] = L;
    }
    __syncthreads();
    if constexpr (CL)   // the other half of the first barrier: every CTA of the cluster runs
        asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
        const int h = i / HD, d = i % HD;
        const float M = wml[h][0], L = wml[h][1];
        float O = 0.f;
        for (int w = 0; w < NW; w++) {
            if (wm[w][h] == -INFINITY) continue;
            O += wo[w][h][d] * we[w][h];
        }
        if constexpr (CL) {   // dim d goes to the CTA that owns it; m, l to every CTA (d < ns)
            namespace cg = cooperative_groups;
            cg::cluster_group cluster = cg::this_cluster();
            const int ns = a.nsplit, dpc = HD / ns, me = (int)cluster.block_rank(), rr = d / dpc;
            cluster.map_shared_rank(mrg, rr)[(me * G + h) * (dpc + 2) + d - rr * dpc] = O;
            if (d < ns) {
                float *dm = cluster.map_shared_rank(mrg, d) + (me * G + h) * (dpc + 2) + dpc;
                dm[0] = M;
                dm[1] = L;
            }
        } else {
            float *dst = out + h * PR;
            dst[d] = O;
            if (d == 0) {
                dst[HD] = M;
                dst[HD + 1] = L;
            }
        }
    }
    if constexpr (CL) {
        namespace cg = cooperative_groups;
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();   // every split's stores are in; nothing touches another CTA's memory after it
        const int ns = a.nsplit, r = (int)cluster.block_rank(), dpc = HD / ns;
        if (threadIdx.x < G) {   // per head: the splits' weights e^{m_c - M} and the sum L, once
            const int h = threadIdx.x;
            float M = -INFINITY;
            for (int c = 0; c < ns; c++) M = fmaxf(M, mrg[(c * G + h) * (dpc + 2) + dpc]);
            float L = 0.f;
            for (int c = 0; c < ns; c++) {   // the same order as the ticket merge: split 0 first
                const float mc = mrg[(c * G + h) * (dpc + 2) + dpc];
                const float e = mc == -INFINITY ? 0.f : expf(mc - M);
                L += mrg[(c * G + h) * (dpc + 2) + dpc + 1] * e;
                cwt[c][h] = e;
            }
            wml[h][1] = L;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < G * dpc; i += blockDim.x) {   // this CTA's dims, every head
            const int h = i / dpc, dd = i - h * dpc;
            float O = 0.f;
            for (int c = 0; c < ns; c++) O = fmaf(mrg[(c * G + h) * (dpc + 2) + dd], cwt[c][h], O);
            a.out[(size_t)tok * a.ldout + (size_t)(kvh * G + h) * HD + r * dpc + dd] = (O / wml[h][1]) * gs[h];
        }
    } else {
        finish_splits<HD>(a, kvh, tok, G, pbase, pstride, cw, cl, &is_last);
    }
}

}  // namespace

int attn_decode(const AttnArgs &a, cudaStream_t s) {
    if (a.heads % a.kv_heads || a.heads / a.kv_heads > ATT_MAX_GROUP) return set_error("attention: GQA group above %d", ATT_MAX_GROUP);
    if (a.nsplit < 1 || a.nsplit > ATT_MAX_SPLIT || a.ntok < 1 || a.ntok > ATT_MAX_TOK)
        return set_error("attention: %d splits x %d tokens out of range", a.nsplit, a.ntok);
    if (a.store && a.ntok != 1) return set_error("attention: in-kernel K/V store takes one token");
    const dim3 grid(a.kv_heads, a.nsplit, a.ntok);
    // the longest split this layer can see: the cache span over the splits
    const int span = a.full ? a.slots : (a.window < a.slots ? a.window : a.slots);
    const bool longs = (span + a.nsplit - 1) / a.nsplit >= 64;
    if (a.hd != 256 && a.hd != 128) return set_error("attention: head_dim %d (128 or 256)", a.hd);
    if (a.kv_type < KV_F32 || a.kv_type > KV_Q8) return set_error("attention: cache type %d", a.kv_type);
    if (a.hd == 256 && (a.kv_type == KV_F16 || a.kv_type == KV_Q8)) {   // the tensor-core kernel
        static int opted[4][64];
        int dev = 0;
        cudaGetDevice(&dev);
        const int q8 = a.kv_type == KV_Q8;
        // up to 8 splits: one cluster per (token, KV head), the merge in distributed shared memory
        const bool cl = a.nsplit <= 8 && (a.hd % a.nsplit) == 0;
        auto k = q8 ? (cl ? attn_tc_kernel<KV_Q8, true> : attn_tc_kernel<KV_Q8, false>)
                    : (cl ? attn_tc_kernel<KV_F16, true> : attn_tc_kernel<KV_F16, false>);
        const size_t sm = q8 ? TcLayout<KV_Q8>::SMEM : TcLayout<KV_F16>::SMEM;
        if (!opted[q8 * 2 + cl][dev & 63]) {
            cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
            if (e != cudaSuccess) return cuda_fail("attention shared-memory opt-in", e);
            opted[q8 * 2 + cl][dev & 63] = 1;
        }
        cudaError_t e;
        if (cl) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = grid;
            cfg.blockDim = dim3(TC_THREADS);
            cfg.dynamicSmemBytes = sm;
            cfg.stream = s;
            cudaLaunchAttribute at[2];
            at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            at[0].val.programmaticStreamSerializationAllowed = 1;
            at[1].id = cudaLaunchAttributeClusterDimension;
            at[1].val.clusterDim.x = 1;
            at[1].val.clusterDim.y = a.nsplit;
            at[1].val.clusterDim.z = 1;
            cfg.attrs = at;
            cfg.numAttrs = 2;
            e = cudaLaunchKernelEx(&cfg, k, a);
        } else {
            e = launch_pdl(k, grid, dim3(TC_THREADS), sm, s, a);
        }
        return e == cudaSuccess ? 0 : cuda_fail("attention launch", e);
    }
    const int sel = (a.hd == 256 ? 0 : 6) + a.kv_type * 2 + (longs ? 1 : 0);
    void (*const ks[12])(const AttnArgs) = {
        attn_kernel<256, 0, 2>, attn_kernel<256, 0, 4>, attn_kernel<256, 1, 2>, attn_kernel<256, 1, 4>,
        attn_kernel<256, 2, 2>, attn_kernel<256, 2, 4>, attn_kernel<128, 0, 2>, attn_kernel<128, 0, 4>,
        attn_kernel<128, 1, 2>, attn_kernel<128, 1, 4>, attn_kernel<128, 2, 2>, attn_kernel<128, 2, 4>};
    const cudaError_t e = launch_pdl(ks[sel], grid, dim3(ATT_THREADS), 0, s, a);
    return e == cudaSuccess ? 0 : cuda_fail("attention launch", e);
}

int attn_store_batch(const AttnArgs &a, cudaStream_t s) {
    const size_t sm = 2 * (size_t)a.kv_heads * a.hd * sizeof(float);
    if (a.kv_type < KV_F32 || a.kv_type > KV_Q8) return set_error("attention store: cache type %d", a.kv_type);
    void (*const ks[3])(const AttnArgs) = {attn_store_kernel<0>, attn_store_kernel<1>, attn_store_kernel<2>};
    cudaError_t e = launch_pdl(ks[a.kv_type], dim3(a.ntok), dim3(256), sm, s, a);
    return e == cudaSuccess ? 0 : cuda_fail("attention K/V store launch", e);
}

// Cache rows written from given f32 values: CTA (position, head) stores K and V of that head.
template <int KT>
__global__ void kv_write_kernel(uint8_t *kc, uint8_t *vc, int slots, int hd, int pos0, int head0, const float *k,
                                const float *v, int ld) {
    const int t = blockIdx.x, h = blockIdx.y;
    const size_t o = ((size_t)h * slots + (size_t)(pos0 + t) % slots) * kv_row_bytes(KT, hd);
    const size_t src = (size_t)t * ld + (size_t)(head0 + h) * hd;
    store_row<KT>(k + src, kc + o, hd);
    store_row<KT>(v + src, vc + o, hd);
}

int kv_write(void *kc, void *vc, int kv_type, int slots, int kv_heads, int head0, int hd, int pos0, int n,
             const float *k, const float *v, int ld, cudaStream_t s) {
    if (kv_type < KV_F32 || kv_type > KV_Q8) return set_error("cache write: cache type %d", kv_type);
    if (n <= 0) return 0;
    void (*const ks[3])(uint8_t *, uint8_t *, int, int, int, int, const float *, const float *, int) = {
        kv_write_kernel<0>, kv_write_kernel<1>, kv_write_kernel<2>};
    ks[kv_type]<<<dim3(n, kv_heads), dim3(128), 0, s>>>((uint8_t *)kc, (uint8_t *)vc, slots, hd, pos0, head0, k, v, ld);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail("cache write launch", e);
}

}  // namespace spk

using namespace spk;

namespace {
bool to_args(const spk_attn_args *u, AttnArgs *a) {
    if (!u || !u->qkv || !u->k_cache || !u->v_cache || !u->freq || !u->pos_dev || !u->gate || !u->out || !u->workspace) {
        set_error("attention: a buffer is missing");
        return false;
    }
    if (u->kv_heads <= 0 || u->heads <= 0 || u->slots <= 0 || u->window <= 0 || u->pdim < 2 || u->pdim > u->head_dim) {
        set_error("attention: bad geometry");
        return false;
    }
    memset(a, 0, sizeof *a);
    a->qkv = u->qkv;
    a->ldqkv = u->ldqkv;
    a->kc = u->k_cache;
    a->vc = u->v_cache;
    a->kv_type = u->kv_type;
    a->slots = u->slots;
    a->full = u->full;
    a->window = u->window;
    a->freq = u->freq;
    a->pdim = u->pdim;
    a->heads = u->heads;
    a->kv_heads = u->kv_heads;
    a->hd = u->head_dim;
    a->pos = u->pos_dev;
    a->ntok = u->ntok;
    a->store = u->store;
    a->nsplit = u->nsplit;
    a->gate = u->gate;
    a->ldgate = u->ldgate;
    a->out = u->out;
    a->ldout = u->ldout;
    a->count = reinterpret_cast<unsigned int *>(u->workspace);
    a->part = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(u->workspace) + 256 * sizeof(unsigned int));
    a->err = device_error_ptr();
    return true;
}
}  // namespace

extern "C" {

size_t spk_attn_workspace_bytes(int ntok, int heads, int kv_heads, int head_dim, int nsplit) {
    if (ntok < 1 || kv_heads < 1 || heads < kv_heads || nsplit < 1) return 0;
    return 256 * sizeof(unsigned int) +
           (size_t)ntok * kv_heads * nsplit * (heads / kv_heads) * (head_dim + 4) * sizeof(float);
}

int spk_attn_decode(const spk_attn_args *u, void *stream) {
    AttnArgs a;
    if (!to_args(u, &a)) return -1;
    if ((size_t)a.ntok * a.kv_heads > 256) return set_error("attention: %d token x KV-head tickets exceed 256", a.ntok * a.kv_heads);
    return attn_decode(a, (cudaStream_t)stream);
}

int spk_attn_store(const spk_attn_args *u, void *stream) {
    AttnArgs a;
    if (!to_args(u, &a)) return -1;
    if (a.ntok < 1 || a.ntok > ATT_MAX_TOK) return set_error("attention store: %d tokens", a.ntok);
    return attn_store_batch(a, (cudaStream_t)stream);
}

}  // extern "C"
