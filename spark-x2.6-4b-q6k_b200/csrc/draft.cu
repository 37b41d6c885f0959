// draft.cu — the DSpark draft executor on device (tools/dspark/src/draft.rs
// encode_features 567-628, decode_block 641-901; the reference's GPU executor is
// dspark-gpu.h:914-1152, which runs cuBLAS SGEMMs on f32-expanded weights and
// syncs the host once per Markov row).
//
// Kernels:
//  * bf16_gemm_kernel: Y[n][r] (=, +=, or act(G x) * (U x)) for n < ntok <= 8 over
//    row-major BF16 weights, streamed once from HBM with 16-byte non-allocating
//    loads. A 16-row tile per CTA, its K range cut over 8 warps; the weights are the
//    A fragment of mma.sync m16n8k16 bf16 straight from registers, the tokens the 8
//    B columns (x as bf16 hi + lo, ~16 bits), partials reduced in a fixed order.
//  * rms_rows_kernel: rms_mul (draft.rs:103-110) over row segments, f64 sum.
//  * q80_rows_kernel: the block's token embeddings from the target's Q8_0 table.
//  * markov_kernel: one block row of the Markov head, logits += w2 . w1[prev] with
//    prev read on device (the previous row's argmax), fused first-max argmax and the
//    confidence head, so the chain of rows needs no host round trip.
#include <cuda_bf16.h>
#include <math.h>

#include <vector>

#include "attn.cuh"
#include "common.cuh"
#include "spk.h"

namespace spk {

namespace {

constexpr int BW = 8;          // warps per CTA of the GEMM
constexpr int BT = BW * 32;
constexpr int BU = 4;          // 32-wide K steps per batch of loads
constexpr int BF_MAXSEG = 4;

enum { BF_STORE = 0, BF_ACC = 1, BF_GELU = 2, BF_SILU = 3 };

struct BfSeg {
    const uint16_t *w;   // [rows][cols] bf16
    int rows;
};

struct BfArgs {
    BfSeg seg[BF_MAXSEG];   // stacked along the output rows (pair modes: seg[0] gate, seg[1] up)
    int nseg, rows, cols;
    const float *x;
    int ldx, ntok;
    float *y;
    int ldy, mode;
};

__device__ __forceinline__ uint4 ld_stream16(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t *>(&v); }

// (a, b) as bf16 pairs: hi = rn(x), lo = rn(x - hi); the low half holds a.
__device__ __forceinline__ void split_bf16x2(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const float2 hf = __bfloat1622float2(h);
    hi = bf2_bits(h);
    lo = bf2_bits(__floats2bfloat162_rn(__fsub_rn(a, hf.x), __fsub_rn(b, hf.y)));
}

// draft.rs:905-911 (ggml's tanh form) and 913-916, in the same f32 operation order
__device__ __forceinline__ float gelu_tanh_f(float x) {
    const float A = 0.044715f, S = 0.7978846f;
    const float in = __fmul_rn(__fmul_rn(S, x), __fadd_rn(1.0f, __fmul_rn(__fmul_rn(A, x), x)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(in)));
}
__device__ __forceinline__ float sigmoid_f(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }
__device__ __forceinline__ float silu_f(float x) { return __fmul_rn(x, sigmoid_f(x)); }

// Physical K order of one 32-wide step: thread t holds columns k0 + 8t .. k0 + 8t + 7 of
// its rows (one 16-byte load each) and of its token; MMA 0 takes words 0-1 (logical k
// 2t, 2t+1 | 2t+8, 2t+9), MMA 1 words 2-3. A and B use the same map, so every column
// meets its own x exactly once.
template <int PAIR>
__global__ void __launch_bounds__(BT) bf16_gemm_kernel(const BfArgs a) {
    __shared__ float part[PAIR + 1][BW][16 * 8];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int r0 = blockIdx.x * 16;
    const uint16_t *w0 = nullptr, *w1 = nullptr;
    int nr;
    if (PAIR) {
        w0 = a.seg[0].w + (size_t)r0 * a.cols;
        w1 = a.seg[1].w + (size_t)r0 * a.cols;
        nr = min(16, a.rows - r0);
    } else {
        const uint16_t *ws = a.seg[0].w;
        int off = 0, rs = a.seg[0].rows;
#pragma unroll
        for (int i = 1; i < BF_MAXSEG; i++)   // constant indices: the arguments stay in the constant bank
            if (i < a.nseg && r0 >= off + rs) {
                off += rs;
                ws = a.seg[i].w;
                rs = a.seg[i].rows;
            }
        w0 = ws + (size_t)(r0 - off) * a.cols;
        nr = min(16, off + rs - r0);
    }
    const bool va = g < nr, vb = g + 8 < nr, live = g < a.ntok;
    const int nk = a.cols / 32;
    const int kb = warp * nk / BW, ke = (warp + 1) * nk / BW;
    const uint8_t *pa0 = reinterpret_cast<const uint8_t *>(w0 + (size_t)g * a.cols) + 16 * t;
    const uint8_t *pb0 = reinterpret_cast<const uint8_t *>(w0 + (size_t)(g + 8) * a.cols) + 16 * t;
    const uint8_t *pa1 = PAIR ? reinterpret_cast<const uint8_t *>(w1 + (size_t)g * a.cols) + 16 * t : nullptr;
    const uint8_t *pb1 = PAIR ? reinterpret_cast<const uint8_t *>(w1 + (size_t)(g + 8) * a.cols) + 16 * t : nullptr;
    const float *xr = a.x + (size_t)(live ? g : 0) * a.ldx + 8 * t;

    float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
    uint4 A0[BU], B0[BU], A1[BU], B1[BU];
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    auto load_w = [&](int k) {
#pragma unroll
        for (int u = 0; u < BU; u++) {
            const bool in = k + u < ke;
            const size_t o = (size_t)(k + u) * 64;   // 32 bf16 per step
            A0[u] = in && va ? ld_stream16(pa0 + o) : z;
            B0[u] = in && vb ? ld_stream16(pb0 + o) : z;
            if (PAIR) {
                A1[u] = in && va ? ld_stream16(pa1 + o) : z;
                B1[u] = in && vb ? ld_stream16(pb1 + o) : z;
            }
        }
    };
    pdl_trigger();
    load_w(kb);   // weights only: issued while the producer of x drains
    pdl_wait();
    for (int k = kb; k < ke; k += BU) {
        uint32_t bh[BU][4], bl[BU][4];
#pragma unroll
        for (int u = 0; u < BU; u++) {
            float4 xa = make_float4(0.f, 0.f, 0.f, 0.f), xb = xa;
            if (live && k + u < ke) {
                xa = __ldg(reinterpret_cast<const float4 *>(xr + (size_t)(k + u) * 32));
                xb = __ldg(reinterpret_cast<const float4 *>(xr + (size_t)(k + u) * 32 + 4));
            }
            split_bf16x2(xa.x, xa.y, bh[u][0], bl[u][0]);
            split_bf16x2(xa.z, xa.w, bh[u][1], bl[u][1]);
            split_bf16x2(xb.x, xb.y, bh[u][2], bl[u][2]);
            split_bf16x2(xb.z, xb.w, bh[u][3], bl[u][3]);
        }
#pragma unroll
        for (int u = 0; u < BU; u++) {
            mma_bf16(d0, A0[u].x, B0[u].x, A0[u].y, B0[u].y, bh[u][0], bh[u][1]);
            mma_bf16(d0, A0[u].x, B0[u].x, A0[u].y, B0[u].y, bl[u][0], bl[u][1]);
            mma_bf16(d0, A0[u].z, B0[u].z, A0[u].w, B0[u].w, bh[u][2], bh[u][3]);
            mma_bf16(d0, A0[u].z, B0[u].z, A0[u].w, B0[u].w, bl[u][2], bl[u][3]);
            if (PAIR) {
                mma_bf16(d1, A1[u].x, B1[u].x, A1[u].y, B1[u].y, bh[u][0], bh[u][1]);
                mma_bf16(d1, A1[u].x, B1[u].x, A1[u].y, B1[u].y, bl[u][0], bl[u][1]);
                mma_bf16(d1, A1[u].z, B1[u].z, A1[u].w, B1[u].w, bh[u][2], bh[u][3]);
                mma_bf16(d1, A1[u].z, B1[u].z, A1[u].w, B1[u].w, bl[u][2], bl[u][3]);
            }
        }
        if (k + BU < ke) load_w(k + BU);
    }
    float *p0 = part[0][warp];
    p0[g * 8 + 2 * t] = d0[0];
    p0[g * 8 + 2 * t + 1] = d0[1];
    p0[(g + 8) * 8 + 2 * t] = d0[2];
    p0[(g + 8) * 8 + 2 * t + 1] = d0[3];
    if (PAIR) {
        float *p1 = part[PAIR][warp];
        p1[g * 8 + 2 * t] = d1[0];
        p1[g * 8 + 2 * t + 1] = d1[1];
        p1[(g + 8) * 8 + 2 * t] = d1[2];
        p1[(g + 8) * 8 + 2 * t + 1] = d1[3];
    }
    __syncthreads();
    if (tid < 128) {
        const int row = tid >> 3, col = tid & 7;
        if (row < nr && col < a.ntok) {
            float v = 0.f, u = 0.f;
#pragma unroll
            for (int w = 0; w < BW; w++) v += part[0][w][tid];
            if (PAIR)
#pragma unroll
                for (int w = 0; w < BW; w++) u += part[PAIR][w][tid];
            float *o = a.y + (size_t)col * a.ldy + r0 + row;
            if (a.mode == BF_STORE) *o = v;
            else if (a.mode == BF_ACC) *o = __fadd_rn(*o, v);
            else if (a.mode == BF_GELU) *o = __fmul_rn(gelu_tanh_f(v), u);
            else *o = __fmul_rn(silu_f(v), u);
        }
    }
}

// y[row][seg] = (acc ? y : 0) + rms_mul(x[row][seg], w[seg]) (or rms_only when w is
// null), then * scale when scale != 0. grid (nseg, rows); x == y is allowed.
__global__ void rms_rows_kernel(const float *x, size_t ldx, size_t sx, const float *w, size_t sw, float *y, size_t ldy,
                                size_t sy, int n, float eps, int acc, float scale) {
    __shared__ double red[32];
    __shared__ float s_inv;
    pdl_trigger();
    pdl_wait();
    const float *xr = x + (size_t)blockIdx.y * ldx + (size_t)blockIdx.x * sx;
    float *yr = y + (size_t)blockIdx.y * ldy + (size_t)blockIdx.x * sy;
    const float *wr = w ? w + (size_t)blockIdx.x * sw : nullptr;
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss += (double)xr[i] * (double)xr[i];
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += red[i];
        s_inv = (float)(1.0 / sqrt(t / (double)n + (double)eps));
    }
    __syncthreads();
    const float inv = s_inv;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = __fmul_rn(xr[i], inv);
        if (wr) v = __fmul_rn(v, wr[i]);
        if (scale != 0.0f) v = __fmul_rn(v, scale);
        yr[i] = acc ? __fadd_rn(yr[i], v) : v;
    }
}

// y[row] *= s (layer_out_scale without an ffn_post norm)
__global__ void scale_rows_kernel(float *y, size_t ldy, int n, float s) {
    pdl_trigger();
    pdl_wait();
    float *yr = y + (size_t)blockIdx.y * ldy;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) yr[i] = __fmul_rn(yr[i], s);
}

// The block's token embeddings from a Q8_0 table, grid (cols/256, n): row 0 is the
// anchor (*anchor_dev, or anchor), rows 1.. the mask token (draft.rs:698-713).
__global__ void q80_rows_kernel(const uint8_t *w, int rows, int cols, const int *anchor_dev, int anchor, int mask,
                                float *out, int ldo, int *err) {
    pdl_trigger();
    pdl_wait();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    int r = blockIdx.y ? mask : (anchor_dev ? *anchor_dev : anchor);
    if (r < 0 || r >= rows) {
        if (c == 0) atomicExch(err, DEV_BAD_INDEX);
        r = 0;
    }
    const uint8_t *blk = w + ((size_t)r * (cols / 32) + (c >> 5)) * 34;
    const float d = __half2float(__ushort_as_half((uint16_t)(blk[0] | (blk[1] << 8))));
    out[(size_t)blockIdx.y * ldo + c] = __fmul_rn((float)(int8_t)blk[2 + (c & 31)], d);
}

// conf[0] of a non-anchor block: sigmoid(logits[0][0]) (draft.rs:864-868)
__global__ void conf0_kernel(const float *logits, float *conf) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) *conf = sigmoid_f(logits[0]);
}

// Order-preserving (value, index) key: larger value wins, then the smaller index
// (draft.rs:917-928's strict > from -inf); NaN never wins, -0 ties +0.
__device__ __forceinline__ unsigned long long vi_key(float v, int i) {
    uint32_t u = __float_as_uint(v);
    if (u == 0x80000000u) u = 0u;
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    if (v != v) u = 0u;
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)i);
}

constexpr int MK_THREADS = 256;
constexpr int MK_MAXRANK = 1024;
constexpr int MK_MAXCTA = 1024;

struct MkArgs {
    const uint16_t *w1, *w2;   // [vocab_m][rank] bf16
    int rank, vocab_m, vocab;
    const int *prev;           // device: the row's previous token (null: prev_host)
    int prev_host;
    float *logits;             // this row [vocab]
    int *amax;                 // this row's argmax
    const float *conf_proj;    // [hidden + rank] f32, or null
    float conf_bias;
    const float *hid;          // this row's normed hidden [hidden]
    int hidden;
    float *conf;               // this row's confidence
    unsigned long long *partial;   // [gridDim.x]
    unsigned int *counter;         // zero; the last CTA resets it
    int *err;
};

// draft.rs:869-891 for one block row: logits[t] += w2[t] . w1[prev] (t < vocab_m), the
// argmax over all vocab logits, and conf = sigmoid(conf_proj . [hid; w1[prev]] + bias).
__global__ void __launch_bounds__(MK_THREADS) markov_kernel(const MkArgs a) {
    __shared__ float w1s[MK_MAXRANK];
    __shared__ unsigned long long best_w[MK_THREADS / 32];
    __shared__ bool last;
    __shared__ double cred[MK_THREADS / 32];
    pdl_trigger();
    pdl_wait();   // prev and the logits row come from the preceding kernels
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int prev = a.prev ? *a.prev : a.prev_host;
    if (prev < 0 || prev >= a.vocab_m) {
        if (tid == 0) atomicExch(a.err, DEV_BAD_INDEX);
        prev = 0;
    }
    for (int i = tid; i < a.rank; i += MK_THREADS) w1s[i] = __bfloat162float(__ushort_as_bfloat16(a.w1[(size_t)prev * a.rank + i]));
    __syncthreads();
    unsigned long long best = 0ull;
    const int nw = gridDim.x * (MK_THREADS / 32);
    for (int t = blockIdx.x * (MK_THREADS / 32) + warp; t < a.vocab; t += nw) {
        float v = a.logits[t];
        if (t < a.vocab_m) {
            const uint16_t *wr = a.w2 + (size_t)t * a.rank;
            float s = 0.f;
            for (int c = lane * 8; c < a.rank; c += 256) {
                const uint4 q = *reinterpret_cast<const uint4 *>(wr + c);
                const uint32_t qq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&qq[j]));
                    s = fmaf(f.x, w1s[c + 2 * j], s);
                    s = fmaf(f.y, w1s[c + 2 * j + 1], s);
                }
            }
            for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            v = __fadd_rn(v, s);
            if (lane == 0) a.logits[t] = v;
        }
        const unsigned long long k = vi_key(v, t);
        best = k > best ? k : best;
    }
    if (lane == 0) best_w[warp] = best;
    __syncthreads();
    if (tid == 0) {
        unsigned long long b = 0ull;
        for (int w = 0; w < MK_THREADS / 32; w++) b = best_w[w] > b ? best_w[w] : b;
        a.partial[blockIdx.x] = b;
        __threadfence();
        last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (tid == 0) {
        unsigned long long b = 0ull;
        for (int i = 0; i < (int)gridDim.x; i++) {
            const unsigned long long p = *reinterpret_cast<volatile unsigned long long *>(a.partial + i);
            b = p > b ? p : b;
        }
        *a.amax = (int)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull));
        *a.counter = 0u;
    }
    if (a.conf_proj) {   // one CTA: the dot over [hid; w1[prev]]
        double s = 0.0;
        for (int i = tid; i < a.hidden + a.rank; i += MK_THREADS)
            s += (double)a.conf_proj[i] * (double)(i < a.hidden ? a.hid[i] : w1s[i - a.hidden]);
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) cred[warp] = s;
        __syncthreads();
        if (tid == 0) {
            double tt = 0.0;
            for (int w = 0; w < MK_THREADS / 32; w++) tt += cred[w];
            *a.conf = sigmoid_f(__fadd_rn((float)tt, a.conf_bias));
        }
    }
}

}  // namespace

// ------------------------------------------------------------------ launchers ---
int bf16_gemm(const BfSeg *seg, int nseg, int cols, int ntok, const float *x, int ldx, float *y, int ldy, int mode,
              cudaStream_t s) {
    if (nseg < 1 || nseg > BF_MAXSEG || ntok < 1 || ntok > 8 || cols < 32 || cols % 32)
        return set_error("bf16 gemm: %d segments, %d tokens, %d columns", nseg, ntok, cols);
    if (((uintptr_t)x & 15) || (ldx & 3)) return set_error("bf16 gemm: x must be 16-byte aligned rows");
    const bool pair = mode == BF_GELU || mode == BF_SILU;
    if (pair && (nseg != 2 || seg[0].rows != seg[1].rows)) return set_error("bf16 gemm: a pair takes two equal matrices");
    BfArgs A;
    memset(&A, 0, sizeof A);
    int rows = 0;
    for (int i = 0; i < nseg; i++) {
        if (!seg[i].w || seg[i].rows < 1 || ((uintptr_t)seg[i].w & 15)) return set_error("bf16 gemm: segment %d", i);
        if (!pair && i < nseg - 1 && seg[i].rows % 16) return set_error("bf16 gemm: stacked segments need 16-row multiples");
        A.seg[i] = seg[i];
        rows += seg[i].rows;
    }
    A.nseg = nseg;
    A.rows = pair ? seg[0].rows : rows;
    A.cols = cols;
    A.x = x;
    A.ldx = ldx;
    A.ntok = ntok;
    A.y = y;
    A.ldy = ldy;
    A.mode = mode;
    const dim3 grid((A.rows + 15) / 16);
    cudaError_t e = pair ? launch_pdl(bf16_gemm_kernel<1>, grid, dim3(BT), 0, s, A)
                         : launch_pdl(bf16_gemm_kernel<0>, grid, dim3(BT), 0, s, A);
    return e == cudaSuccess ? 0 : cuda_fail("bf16 gemm launch", e);
}

int rms_rows(const float *x, size_t ldx, size_t sx, const float *w, size_t sw, float *y, size_t ldy, size_t sy, int n,
             int nseg, int rows, float eps, int acc, float scale, cudaStream_t s) {
    if (n < 1 || nseg < 1 || rows < 1) return set_error("rms rows: %d x %d x %d", rows, nseg, n);
    cudaError_t e = launch_pdl(rms_rows_kernel, dim3(nseg, rows), dim3(256), 0, s, x, ldx, sx, w, sw, y, ldy, sy, n, eps,
                               acc, scale);
    return e == cudaSuccess ? 0 : cuda_fail("rms rows launch", e);
}

}  // namespace spk

using namespace spk;

extern "C" {

/* The draft's skinny BF16 GEMM (replaces draft_gemm's cublasSgemm, dspark-gpu.h:897-907):
 * y[n*ldy + r] (=, or += when accumulate) (W x[n*ldx ..])[r] for n < ntok <= 8, W a
 * row-major bf16 [rows][cols] device matrix (16-byte aligned, cols % 32 == 0). */
int spk_bf16_gemm(const void *w, int rows, int cols, int ntok, const float *x, int ldx, float *y, int ldy,
                  int accumulate, void *stream) {
    if (!w || !x || !y || rows < 1 || ldx < cols || ldy < rows) return set_error("bf16 gemm: bad arguments");
    const BfSeg sg = {(const uint16_t *)w, rows};
    return bf16_gemm(&sg, 1, cols, ntok, x, ldx, y, ldy, accumulate ? BF_ACC : BF_STORE, (cudaStream_t)stream);
}

/* The FFN pair: y[n][r] = act(G x)[r] * (U x)[r], act 0 = gelu (ggml's tanh form), 1 = silu
 * (draft.rs:838-855). */
int spk_bf16_gemm_pair(const void *gate, const void *up, int rows, int cols, int ntok, const float *x, int ldx,
                       float *y, int ldy, int act, void *stream) {
    if (!gate || !up || !x || !y || rows < 1 || ldx < cols || ldy < rows) return set_error("bf16 pair: bad arguments");
    const BfSeg sg[2] = {{(const uint16_t *)gate, rows}, {(const uint16_t *)up, rows}};
    return bf16_gemm(sg, 2, cols, ntok, x, ldx, y, ldy, act == 1 ? BF_SILU : BF_GELU, (cudaStream_t)stream);
}

}  // extern "C"

// ============================================================ the executor ===
struct spk_draft {
    spk_draft_config cfg;
    struct Layer {
        spk_draft_layer p;
        bool set = false;
    };
    std::vector<Layer> layers;
    spk_draft_globals g = {};
    bool gset = false;
    int max_ctx = 0, q_dim = 0, kv_dim = 0, ldq = 0, nsplit = 16;
    long nswa = 0;
    int enc_lo = 0, enc_hi = 0;   // positions [enc_lo, enc_hi) hold encodings
    float *kc = nullptr, *vc = nullptr;   // [layers][kv_heads][max_ctx][hd] f32
    float *freq_swa = nullptr, *freq_full = nullptr;
    int *iota = nullptr;                  // iota[p] = p: device positions for the kernels
    float *x = nullptr, *xn = nullptr, *qkvg = nullptr, *attn = nullptr, *act = nullptr, *tmp = nullptr,
          *hid = nullptr, *logits = nullptr, *conf = nullptr, *concat = nullptr, *genc = nullptr, *noattn_gate = nullptr;
    int *amax = nullptr;
    unsigned int *att_count = nullptr;
    float *att_part = nullptr;
    unsigned long long *head_partial = nullptr, *mk_partial = nullptr;
    unsigned int *head_counter = nullptr, *mk_counter = nullptr;
    int *host_ids = nullptr;
    float *host_conf = nullptr;
    cudaStream_t stream = nullptr;
    int vocab_target = 0;
    const void *head_tiled = nullptr;   // optional: the target head's tiled table (q8t.cu)
    void *qt_scratch = nullptr;
};

namespace {

constexpr int DR_ROWS = 8;   // block rows and encode chunk

int dalloc(void **p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
    if (e != cudaSuccess) {
        *p = nullptr;
        return cuda_fail("draft allocation", e);
    }
    return 0;
}

int mk_grid() { return sm_count() * 2 < MK_MAXCTA ? sm_count() * 2 : MK_MAXCTA; }

AttnArgs draft_attn(spk_draft *d, int li, int p, int ntok, const float *qkv) {
    const spk_draft_config &c = d->cfg;
    AttnArgs a;
    memset(&a, 0, sizeof a);
    a.qkv = qkv;
    a.ldqkv = d->ldq;
    const size_t lay = (size_t)c.kv_heads * d->max_ctx * c.head_dim;
    a.kc = d->kc + (size_t)li * lay;
    a.vc = d->vc + (size_t)li * lay;
    a.kv_type = KV_F32;
    a.slots = d->max_ctx;
    a.full = 0;   // the keep rule applies the window to every layer (draft.rs:772-795)
    a.window = (int)d->nswa;
    const bool swa = c.swa_pattern[li] != 0;
    const int nrot = swa ? c.rope_swa_dims : c.rope_full_dims;
    a.freq = swa ? d->freq_swa : d->freq_full;
    a.pdim = nrot < c.head_dim ? nrot : c.head_dim;
    a.heads = c.heads;
    a.kv_heads = c.kv_heads;
    a.hd = c.head_dim;
    a.pos = d->iota + p;
    a.ntok = ntok;
    a.nsplit = d->nsplit;
    a.part = d->att_part;
    a.count = d->att_count;
    a.err = device_error_ptr();
    return a;
}

// q|k|v|g of ntok rows of xn into qkvg [ntok][ldq]
int draft_qkvg(spk_draft *d, const spk_draft::Layer &L, int ntok, cudaStream_t s) {
    const spk_draft_config &c = d->cfg;
    BfSeg sg[4] = {{(const uint16_t *)L.p.q, d->q_dim}, {(const uint16_t *)L.p.k, d->kv_dim},
                   {(const uint16_t *)L.p.v, d->kv_dim}, {(const uint16_t *)L.p.gate, c.heads}};
    return bf16_gemm(sg, L.p.gate ? 4 : 3, c.hidden, ntok, d->xn, c.hidden, d->qkvg, d->ldq, BF_STORE, s);
}

}  // namespace

extern "C" {

spk_draft *spk_draft_create(const spk_draft_config *cfg, void *stream) {
    if (!cfg) {
        set_error("draft config is missing");
        return nullptr;
    }
    const spk_draft_config &c = *cfg;
    if (c.hidden <= 0 || c.hidden % 512 || c.layers < 1 || c.layers > SPK_DRAFT_MAX_LAYERS || c.heads <= 0 ||
        c.kv_heads <= 0 || c.heads % c.kv_heads || c.heads / c.kv_heads > ATT_MAX_GROUP ||
        (c.head_dim != 128 && c.head_dim != 256) || c.ffn <= 0 || c.ffn % 32 || c.vocab <= 0 || c.max_ctx <= 0 ||
        c.block_size < 1 || c.block_size + 1 > DR_ROWS + 1 || c.n_target < 1 || c.swa_window < 1 ||
        (c.rank && (c.rank % 8 || c.rank > MK_MAXRANK)) || c.act < 0 || c.act > 1 || c.mask_token < 0 ||
        c.mask_token >= c.vocab) {
        set_error("unsupported draft geometry (hidden a multiple of 512, head_dim 128/256, GQA group <= 4, "
                  "block_size <= 8, rank a multiple of 8 up to 1024)");
        return nullptr;
    }
    spk_draft *d = new spk_draft();
    d->cfg = c;
    d->layers.resize(c.layers);
    d->max_ctx = c.max_ctx;
    d->q_dim = c.heads * c.head_dim;
    d->kv_dim = c.kv_heads * c.head_dim;
    d->ldq = d->q_dim + 2 * d->kv_dim + c.heads;
    d->ldq = (d->ldq + 3) / 4 * 4;
    d->nswa = c.rank ? (long)c.swa_window + 1 : (long)c.swa_window;   // draft.rs:685-692
    d->stream = (cudaStream_t)stream;
    const int R = DR_ROWS, H = c.hidden;
    const size_t kvl = (size_t)c.layers * c.kv_heads * c.max_ctx * c.head_dim;
    bool ok = !dalloc((void **)&d->kc, kvl * 4) && !dalloc((void **)&d->vc, kvl * 4) &&
              !dalloc((void **)&d->freq_swa, c.head_dim * 4) && !dalloc((void **)&d->freq_full, c.head_dim * 4) &&
              !dalloc((void **)&d->iota, ((size_t)c.max_ctx + R) * 4) &&
              !dalloc((void **)&d->x, (size_t)R * H * 4) && !dalloc((void **)&d->xn, (size_t)R * H * 4) &&
              !dalloc((void **)&d->qkvg, (size_t)R * d->ldq * 4) && !dalloc((void **)&d->attn, (size_t)R * d->q_dim * 4) &&
              !dalloc((void **)&d->act, (size_t)R * c.ffn * 4) && !dalloc((void **)&d->tmp, (size_t)R * H * 4) &&
              !dalloc((void **)&d->hid, (size_t)R * H * 4) && !dalloc((void **)&d->conf, R * 4) &&
              !dalloc((void **)&d->concat, (size_t)R * c.n_target * H * 4) && !dalloc((void **)&d->genc, (size_t)R * H * 4) &&
              !dalloc((void **)&d->noattn_gate, (size_t)R * d->ldq * 4) && !dalloc((void **)&d->amax, R * 4) &&
              !dalloc((void **)&d->att_count, 256 * 4) &&
              !dalloc((void **)&d->att_part, (size_t)R * c.kv_heads * d->nsplit * (c.heads / c.kv_heads) *
                                                 (c.head_dim + 4) * 4) &&
              !dalloc((void **)&d->head_partial, q80_head_batch_scratch() > 8192 ? q80_head_batch_scratch() : 8192) &&
              !dalloc((void **)&d->head_counter, 64) && !dalloc((void **)&d->mk_partial, MK_MAXCTA * 8) &&
              !dalloc((void **)&d->mk_counter, 64);
    if (ok && (cudaMallocHost((void **)&d->host_ids, R * 4) != cudaSuccess ||
               cudaMallocHost((void **)&d->host_conf, R * 4) != cudaSuccess))
        ok = !set_error("draft pinned staging allocation failed");
    if (ok) {
        // rope frequencies in f32 as draft.rs:129-143 forms them
        std::vector<float> fs(c.head_dim, 0.f), ff(c.head_dim, 0.f);
        const int ds = c.rope_swa_dims < c.head_dim ? c.rope_swa_dims : c.head_dim;
        const int df = c.rope_full_dims < c.head_dim ? c.rope_full_dims : c.head_dim;
        for (int i = 0; i < ds / 2; i++) fs[i] = 1.0f / powf(c.rope_swa_theta, (float)(2 * i) / (float)ds);
        for (int i = 0; i < df / 2; i++) ff[i] = 1.0f / powf(c.rope_full_theta, (float)(2 * i) / (float)df);
        std::vector<int> io(c.max_ctx + R);
        for (int i = 0; i < c.max_ctx + R; i++) io[i] = i;
        // a layer without attn_gate multiplies by sigmoid(+inf) = 1 exactly
        std::vector<float> inf((size_t)R * d->ldq, INFINITY);
        ok = cudaMemcpy(d->freq_swa, fs.data(), c.head_dim * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemcpy(d->freq_full, ff.data(), c.head_dim * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemcpy(d->iota, io.data(), io.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemcpy(d->noattn_gate, inf.data(), inf.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemset(d->kc, 0, kvl * 4) == cudaSuccess && cudaMemset(d->vc, 0, kvl * 4) == cudaSuccess &&
             cudaMemset(d->att_count, 0, 256 * 4) == cudaSuccess && cudaMemset(d->head_counter, 0, 64) == cudaSuccess &&
             cudaMemset(d->mk_counter, 0, 64) == cudaSuccess && cudaMemset(d->conf, 0, R * 4) == cudaSuccess;
        if (!ok) set_error("draft initialisation failed");
    }
    if (!ok) {
        spk_draft_destroy(d);
        return nullptr;
    }
    return d;
}

void spk_draft_destroy(spk_draft *d) {
    if (!d) return;
    void *bufs[] = {d->kc, d->vc, d->freq_swa, d->freq_full, d->iota, d->x, d->xn, d->qkvg, d->attn, d->act,
                    d->tmp, d->hid, d->conf, d->concat, d->genc, d->noattn_gate, d->amax, d->att_count, d->att_part,
                    d->head_partial, d->head_counter, d->mk_partial, d->mk_counter};
    for (void *b : bufs)
        if (b) cudaFree(b);
    if (d->qt_scratch) cudaFree(d->qt_scratch);
    if (d->host_ids) cudaFreeHost(d->host_ids);
    if (d->host_conf) cudaFreeHost(d->host_conf);
    delete d;
}

int spk_draft_set_layer(spk_draft *d, int li, const spk_draft_layer *p) {
    if (!d || !p || li < 0 || li >= d->cfg.layers) return set_error("draft layer %d: bad arguments", li);
    if (!p->q || !p->k || !p->v || !p->out || !p->ffn_gate || !p->ffn_up || !p->ffn_down || !p->norm || !p->ffn_norm)
        return set_error("draft layer %d: a required tensor is missing", li);
    const void *m[] = {p->q, p->k, p->v, p->gate, p->out, p->ffn_gate, p->ffn_up, p->ffn_down};
    for (const void *w : m)
        if (w && ((uintptr_t)w & 15)) return set_error("draft layer %d: weights must be 16-byte aligned", li);
    d->layers[li].p = *p;
    d->layers[li].set = true;
    return 0;
}

int spk_draft_set_globals(spk_draft *d, const spk_draft_globals *g) {
    if (!d || !g || !g->fc || !g->fc_norm || !g->enc_norm || !g->out_norm) return set_error("draft globals: a tensor is missing");
    if (d->cfg.rank && (!g->markov_w1 || !g->markov_w2)) return set_error("draft globals: rank %d without Markov weights", d->cfg.rank);
    if (((uintptr_t)g->fc & 15) || ((uintptr_t)g->markov_w1 & 15) || ((uintptr_t)g->markov_w2 & 15))
        return set_error("draft globals: weights must be 16-byte aligned");
    d->g = *g;
    d->gset = true;
    return 0;
}

/* encode_features (draft.rs:567-628) for the committed positions [p0, p1): caps holds
 * the target's layer-input rows, slot k of position p at caps[k*slot_stride + p*hidden]
 * (device). The injected K/V of those positions go to the draft cache. */
int spk_draft_encode(spk_draft *d, const float *caps, size_t slot_stride, int p0, int p1) {
    if (!d || !caps || p0 < 0 || p1 < p0 || p1 > d->max_ctx) return set_error("draft encode: bad range [%d, %d)", p0, p1);
    for (int li = 0; li < d->cfg.layers; li++)
        if (!d->layers[li].set) return set_error("draft layer %d is not set", li);
    if (!d->gset) return set_error("draft globals are not set");
    const spk_draft_config &c = d->cfg;
    const int H = c.hidden, nt = c.n_target;
    if ((size_t)p1 * H > slot_stride) return set_error("draft encode: position %d lies outside a capture slot", p1 - 1);
    cudaStream_t s = d->stream;
    for (int p = p0; p < p1; p += DR_ROWS) {
        const int n = p1 - p < DR_ROWS ? p1 - p : DR_ROWS;
        if (rms_rows(caps + (size_t)p * H, H, slot_stride, d->g.fc_norm, H, d->concat, (size_t)nt * H, H, H, nt, n, c.eps,
                     0, 0.f, s))
            return -1;
        const BfSeg fc = {(const uint16_t *)d->g.fc, H};
        if (bf16_gemm(&fc, 1, nt * H, n, d->concat, nt * H, d->genc, H, BF_STORE, s)) return -1;
        if (rms_rows(d->genc, H, 0, d->g.enc_norm, 0, d->genc, H, 0, H, 1, n, c.eps, 0, 0.f, s)) return -1;
        for (int li = 0; li < c.layers; li++) {
            const spk_draft::Layer &L = d->layers[li];
            const BfSeg kv[2] = {{(const uint16_t *)L.p.k, d->kv_dim}, {(const uint16_t *)L.p.v, d->kv_dim}};
            if (bf16_gemm(kv, 2, H, n, d->genc, H, d->qkvg + d->q_dim, d->ldq, BF_STORE, s)) return -1;
            if (L.p.k_norm && rms_rows(d->qkvg + d->q_dim, d->ldq, c.head_dim, L.p.k_norm, 0, d->qkvg + d->q_dim,
                                       d->ldq, c.head_dim, c.head_dim, c.kv_heads, n, c.eps, 0, 0.f, s))
                return -1;
            if (attn_store_batch(draft_attn(d, li, p, n, d->qkvg), s)) return -1;
        }
    }
    if (p1 > p0) {
        if (d->enc_hi <= d->enc_lo || p0 > d->enc_hi || p1 < d->enc_lo) d->enc_lo = p0;
        else if (p0 < d->enc_lo) d->enc_lo = p0;
        d->enc_hi = p1;
    }
    return 0;
}

/* decode_block (draft.rs:641-901) over the target's Q8_0 embedding [vocab][hidden]
 * (device). ids (host, n_block) receive the greedy argmax per block row, conf (host,
 * optional) the confidence; the biased logits stay on device (spk_draft_logits).
 * Returns n_block, or -1. Synchronizes the draft's stream. */
int spk_draft_block(spk_draft *d, const void *embed, int vocab, int anchor, int pos0, int n_draft, int *ids,
                    float *conf) {
    if (!d || !embed || !ids) return set_error("draft block: bad arguments");
    const spk_draft_config &c = d->cfg;
    for (int li = 0; li < c.layers; li++)
        if (!d->layers[li].set) return set_error("draft layer %d is not set", li);
    if (!d->gset) return set_error("draft globals are not set");
    const bool markov = c.rank > 0;
    const int nb = markov ? (c.sample_from_anchor ? n_draft : n_draft + 1) : n_draft + 1;
    if (n_draft < 1 || n_draft > c.block_size) return set_error("n_draft %d is outside the trained block_size %d", n_draft, c.block_size);
    if (nb > DR_ROWS) return set_error("block row count %d exceeds %d", nb, DR_ROWS);
    if (vocab < c.vocab || vocab % 32) return set_error("target embedding of %d rows does not cover the draft vocab %d", vocab, c.vocab);
    if (anchor < 0 || anchor >= vocab) return set_error("token %d is outside the target embedding", anchor);
    if (pos0 < 0 || pos0 + nb > d->max_ctx) return set_error("block at %d exceeds the %d-position cache", pos0, d->max_ctx);
    const long lo = pos0 - d->nswa + 1 > 0 ? pos0 - d->nswa + 1 : 0;
    if (lo < pos0 && (lo < d->enc_lo || pos0 > d->enc_hi))
        return set_error("draft block at %d: positions [%ld, %d) are not encoded", pos0, lo, pos0);
    if (!d->logits || d->vocab_target != vocab) {
        if (d->logits) cudaFree(d->logits);
        d->logits = nullptr;
        if (dalloc((void **)&d->logits, (size_t)DR_ROWS * vocab * 4)) return -1;
        d->vocab_target = vocab;
    }
    const int H = c.hidden;
    cudaStream_t s = d->stream;
    cudaError_t e = launch_pdl(q80_rows_kernel, dim3((H + 255) / 256, nb), dim3(256), 0, s, (const uint8_t *)embed, vocab,
                               H, (const int *)nullptr, anchor, c.mask_token, d->x, H, device_error_ptr());
    if (e != cudaSuccess) return cuda_fail("draft embedding launch", e);
    for (int li = 0; li < c.layers; li++) {
        const spk_draft::Layer &L = d->layers[li];
        if (rms_rows(d->x, H, 0, L.p.norm, 0, d->xn, H, 0, H, 1, nb, c.eps, 0, 0.f, s)) return -1;
        if (draft_qkvg(d, L, nb, s)) return -1;
        if (L.p.q_norm && L.p.k_norm &&
            (rms_rows(d->qkvg, d->ldq, c.head_dim, L.p.q_norm, 0, d->qkvg, d->ldq, c.head_dim, c.head_dim, c.heads, nb,
                      c.eps, 0, 0.f, s) ||
             rms_rows(d->qkvg + d->q_dim, d->ldq, c.head_dim, L.p.k_norm, 0, d->qkvg + d->q_dim, d->ldq, c.head_dim,
                      c.head_dim, c.kv_heads, nb, c.eps, 0, 0.f, s)))
            return -1;
        AttnArgs a = draft_attn(d, li, pos0, nb, d->qkvg);
        if (attn_store_batch(a, s)) return -1;
        a.span = c.causal ? 1 : nb;
        a.gate = L.p.gate ? d->qkvg + d->q_dim + 2 * d->kv_dim : d->noattn_gate;
        a.ldgate = d->ldq;
        a.out = d->attn;
        a.ldout = d->q_dim;
        if (attn_decode(a, s)) return -1;
        const BfSeg out = {(const uint16_t *)L.p.out, H};
        if (L.p.attn_post) {
            if (bf16_gemm(&out, 1, d->q_dim, nb, d->attn, d->q_dim, d->tmp, H, BF_STORE, s) ||
                rms_rows(d->tmp, H, 0, L.p.attn_post, 0, d->x, H, 0, H, 1, nb, c.eps, 1, 0.f, s))
                return -1;
        } else if (bf16_gemm(&out, 1, d->q_dim, nb, d->attn, d->q_dim, d->x, H, BF_ACC, s)) {
            return -1;
        }
        if (rms_rows(d->x, H, 0, L.p.ffn_norm, 0, d->xn, H, 0, H, 1, nb, c.eps, 0, 0.f, s)) return -1;
        const BfSeg gu[2] = {{(const uint16_t *)L.p.ffn_gate, c.ffn}, {(const uint16_t *)L.p.ffn_up, c.ffn}};
        if (bf16_gemm(gu, 2, H, nb, d->xn, H, d->act, c.ffn, c.act == 1 ? BF_SILU : BF_GELU, s)) return -1;
        const BfSeg dn = {(const uint16_t *)L.p.ffn_down, H};
        if (bf16_gemm(&dn, 1, c.ffn, nb, d->act, c.ffn, d->x, H, BF_ACC, s)) return -1;
        if (L.p.ffn_post) {
            if (rms_rows(d->x, H, 0, L.p.ffn_post, 0, d->x, H, 0, H, 1, nb, c.eps, 0, L.p.out_scale, s)) return -1;
        } else if (L.p.out_scale != 0.0f) {
            e = launch_pdl(scale_rows_kernel, dim3((H + 255) / 256, nb), dim3(256), 0, s, d->x, (size_t)H, H, L.p.out_scale);
            if (e != cudaSuccess) return cuda_fail("draft scale launch", e);
        }
    }
    if (rms_rows(d->x, H, 0, d->g.out_norm, 0, d->hid, H, 0, H, 1, nb, c.eps, 0, 0.f, s)) return -1;
    // the target's tied head over all rows in one pass (its tiled table when the target shares
    // it, else the ggml blocks), else row by row
    int hb = d->head_tiled ? q8t_head_launch(d->head_tiled, vocab, H, nb, d->hid, H, nullptr, c.eps, d->logits, vocab,
                                             d->amax, d->qt_scratch, s)
                           : 0;
    if (hb == 0)
        hb = q80_head_batch_launch(embed, vocab, H, nb, d->hid, H, nullptr, c.eps, d->logits, vocab, d->amax,
                                   d->head_partial, d->head_counter, s);
    if (hb < 0) return -1;
    if (hb == 0)
        for (int i = 0; i < nb; i++)
            if (q80_head_launch(embed, vocab, H, d->hid + (size_t)i * H, nullptr, c.eps, d->logits + (size_t)i * vocab,
                                d->amax + i, d->head_partial, d->head_counter, s))
                return -1;
    if (markov) {
        const int i_beg = c.sample_from_anchor ? 0 : 1;
        if (!c.sample_from_anchor && d->g.conf_proj) {
            e = launch_pdl(conf0_kernel, dim3(1), dim3(32), 0, s, (const float *)d->logits, d->conf);
            if (e != cudaSuccess) return cuda_fail("draft conf launch", e);
        }
        for (int i = i_beg; i < nb; i++) {
            MkArgs m;
            memset(&m, 0, sizeof m);
            m.w1 = (const uint16_t *)d->g.markov_w1;
            m.w2 = (const uint16_t *)d->g.markov_w2;
            m.rank = c.rank;
            m.vocab_m = c.vocab;
            m.vocab = vocab;
            m.prev = i == i_beg ? nullptr : d->amax + i - 1;   // the chain starts at the anchor (draft.rs:862)
            m.prev_host = anchor;
            m.logits = d->logits + (size_t)i * vocab;
            m.amax = d->amax + i;
            m.conf_proj = d->g.conf_proj;
            m.conf_bias = d->g.conf_bias;
            m.hid = d->hid + (size_t)i * H;
            m.hidden = H;
            m.conf = d->conf + i;
            m.partial = d->mk_partial;
            m.counter = d->mk_counter;
            m.err = device_error_ptr();
            e = launch_pdl(markov_kernel, dim3(mk_grid()), dim3(MK_THREADS), 0, s, m);
            if (e != cudaSuccess) return cuda_fail("draft Markov head launch", e);
        }
    }
    if (cudaMemcpyAsync(d->host_ids, d->amax, nb * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyAsync(d->host_conf, d->conf, nb * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return cuda_fail("draft result copy", cudaGetLastError());
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail("draft block", e);
    if (check_device_error("draft block")) return -1;
    for (int i = 0; i < nb; i++) ids[i] = d->host_ids[i];
    if (conf)   // NaN where the reference leaves it (no Markov or no confidence head)
        for (int i = 0; i < nb; i++) conf[i] = markov && d->g.conf_proj ? d->host_conf[i] : NAN;
    return nb;
}

/* Read the block's logits from the target head's tiled table (spk_model_head_tiled: the same
 * embedding in the q8t layout, all vocabulary rows) instead of the ggml blocks; NULL reverts. */
int spk_draft_set_head_tiled(spk_draft *d, const void *tiled) {
    if (!d) return set_error("draft is null");
    if (tiled && !d->qt_scratch) {
        if (dalloc(&d->qt_scratch, q8t_scratch())) return -1;
        if (cudaMemset(d->qt_scratch, 0, q8t_scratch()) != cudaSuccess)
            return cuda_fail("clear draft head scratch", cudaGetLastError());
    }
    d->head_tiled = tiled;
    return 0;
}

/* The last block's biased logits, [n_block][vocab] f32 on device. */
const float *spk_draft_logits(const spk_draft *d) { return d ? d->logits : nullptr; }

}  // extern "C"
