// ggml.cu — Q6_K / Q8_0 block decode kernels for B200 (raw ggml block layout).
//
// Block formats (ggml, sizes as tools/kquant/stubs.c:23-52 price them):
//   Q6_K: 256 weights in 210 bytes: ql[128] low 4 bits, qh[64] high 2 bits,
//         int8 scales[16] (one per 16 weights), f16 d; w = (d * scale) * (q - 32).
//         Weight n = 128h + 32j + l (h half, j quadrant, l lane 0..31):
//         low nibble of ql[64h + l + 32(j&1)] (j<2) or its high nibble (j>=2),
//         high bits (qh[32h + l] >> 2j) & 3, scale scales[8h + 2j + l/16].
//   Q8_0: 32 weights in 34 bytes: f16 d, int8 qs[32]; w = q * d.
//
// The GEMVs accumulate sum (q - 32) * x per 16-weight sub-block and apply the
// block scale once per sub-block. The integer-to-float step uses the bit
// pattern 0x3F000000 | q << 16 == 0.5 + q/256 (q < 64), so a 6-bit value
// becomes a float with one byte permute: sum (q-32) x = 256 (sum f x - 0.625 sum x).
// Dequant kernels are bit-exact with ggml's CPU decode (one rounded f32 multiply
// per operand, in ggml's order).
#include "common.cuh"
#include "spk.h"
#include "stream.cuh"

using namespace spk;

namespace {

__device__ __forceinline__ float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ uint32_t ld_u32_unaligned(const uint8_t *p) {
    // p is at least 2-byte aligned (ggml blocks are 210 / 34 bytes); a 2-aligned
    // word is read as two halves so no byte outside the field is touched.
    if (((uintptr_t)p & 3) == 0) return __ldg((const uint32_t *)p);
    const uint32_t lo = __ldg((const unsigned short *)p), hi = __ldg((const unsigned short *)(p + 2));
    return lo | (hi << 16);
}

__device__ float block_rms_inv(const float *x, int n, float eps, double *red) {
    double s = 0.0;
    for (int i0 = threadIdx.x; i0 < n; i0 += 8 * blockDim.x) {   // 8 loads in flight, summed in index order
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = i0 + j * (int)blockDim.x < n ? x[i0 + j * blockDim.x] : 0.f;
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (i0 + j * (int)blockDim.x < n) s += (double)v[j] * (double)v[j];
    }
    s = warp_sum_d(s);
    const int w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    if ((threadIdx.x & 31) == 0) red[w] = s;
    __syncthreads();
    double t = 0.0;
    for (int k = 0; k < nw; k++) t += red[k];
    __syncthreads();
    return (float)(1.0 / sqrt(t / (double)n + (double)eps));
}

__device__ __forceinline__ float xval(const float *x, const float *nw, float inv, int c) {
    float v = x[c];
    if (nw) v = __fmul_rn(__fmul_rn(v, inv), nw[c]);
    return v;
}

// One unit = 16 weights of one row: half h, lane-quad m (l = 4m..4m+3), all
// four quadrants j. Returns sum over the unit of w * x.
__device__ __forceinline__ float q6k_unit(const uint8_t *blk, int h, int m, const float *x, const float *nw,
                                          float inv, int col0) {
    const uint32_t qa = ld_u32_unaligned(blk + 64 * h + 4 * m);
    const uint32_t qb = ld_u32_unaligned(blk + 64 * h + 32 + 4 * m);
    const uint32_t qh = ld_u32_unaligned(blk + 128 + 32 * h + 4 * m);
    const float d = h2f_bits(*(const uint16_t *)(blk + 208));
    const int8_t *sc = (const int8_t *)(blk + 192 + 8 * h + (m >> 2));
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t lo = ((j & 1) ? qb : qa) >> ((j & 2) ? 4 : 0);
        const uint32_t q = (lo & 0x0F0F0F0Fu) | (((qh >> (2 * j)) & 0x03030303u) << 4);
        float s = 0.f, xs = 0.f;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float xv = xval(x, nw, inv, col0 + 128 * h + 32 * j + 4 * m + e);
            const float f = __uint_as_float(__byte_perm(q, 0x3F000000u, 0x7044u | ((uint32_t)e << 8)));
            s = fmaf(f, xv, s);
            xs += xv;
        }
        s = fmaf(-0.625f, xs, s);
        acc = fmaf(__fmul_rn(d, (float)sc[2 * j]) * 256.0f, s, acc);
    }
    return acc;
}

struct BlkArgs {
    const uint8_t *w;   // row-major blocks
    int rows, cols;
    const float *x;
    const float *norm_w;
    float eps;
    float *y;
    int accumulate;
};

// Warp per row, lanes stride over the row's 16-weight units.
__global__ void q6k_gemv_kernel(const BlkArgs a) {
    __shared__ double red[32];
    float inv = 1.0f;
    if (a.norm_w) inv = block_rms_inv(a.x, a.cols, a.eps, red);
    const int warp = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (warp >= a.rows) return;
    const int nb = a.cols / 256;
    const uint8_t *row = a.w + (size_t)warp * nb * 210;
    float acc = 0.f;
    for (int u = lane; u < nb * 16; u += 32) {
        const int b = u >> 4, h = (u >> 3) & 1, m = u & 7;
        acc += q6k_unit(row + (size_t)b * 210, h, m, a.x, a.norm_w, inv, b * 256);
    }
    acc = warp_sum(acc);
    if (lane == 0) a.y[warp] = (a.accumulate ? a.y[warp] : 0.0f) + acc;
}

// 8 weights of a Q8_0 block (quarter k of block blk).
__device__ __forceinline__ float q80_quarter(const uint8_t *blk, int k, const float *x, const float *nw, float inv,
                                             int col0) {
    const float d = h2f_bits(*(const uint16_t *)blk);
    const uint32_t w0 = ld_u32_unaligned(blk + 2 + 8 * k) ^ 0x80808080u;
    const uint32_t w1 = ld_u32_unaligned(blk + 6 + 8 * k) ^ 0x80808080u;
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        const uint32_t w = e < 4 ? w0 : w1;
        // 0x4B0000bb = 2^23 + bb; bb = q + 128
        const float f = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | (uint32_t)(e & 3))) - 8388736.0f;
        s = fmaf(f, xval(x, nw, inv, col0 + 8 * k + e), s);
    }
    return d * s;
}

__global__ void q80_gemv_kernel(const BlkArgs a) {
    __shared__ double red[32];
    float inv = 1.0f;
    if (a.norm_w) inv = block_rms_inv(a.x, a.cols, a.eps, red);
    const int warp = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (warp >= a.rows) return;
    const int nb = a.cols / 32;
    const uint8_t *row = a.w + (size_t)warp * nb * 34;
    float acc = 0.f;
    for (int u = lane; u < nb * 4; u += 32) acc += q80_quarter(row + (size_t)(u >> 2) * 34, u & 3, a.x, a.norm_w, inv, (u >> 2) * 32);
    acc = warp_sum(acc);
    if (lane == 0) a.y[warp] = (a.accumulate ? a.y[warp] : 0.0f) + acc;
}

// Q8_0 head: logits plus the first index of the maximum (model.rs:594-604),
// reduced per block and then by the last block to finish (a counter that the
// last block resets, so the kernel replays in a graph).
struct HeadArgs {
    BlkArgs b;
    unsigned long long *partial;   // per block: (ordered value << 32) | ~index
    unsigned int *counter;
    int *argmax_out;
};

__device__ __forceinline__ unsigned long long pack_vi(float v, int i) {
    // Larger value wins; for equal values the smaller index wins. NaN never wins.
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    if (v == 0.0f) u = 0x80000000u;   // -0 ties +0, as the CPU's strict > does
    if (v != v) u = 0;
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)i);
}

__global__ void q80_head_kernel(const HeadArgs a) {
    __shared__ double red[32];
    __shared__ unsigned long long best_w[32];
    __shared__ bool last;
    const BlkArgs &b = a.b;
    pdl_trigger();
    pdl_wait();
    float inv = 1.0f;
    if (b.norm_w) inv = block_rms_inv(b.x, b.cols, b.eps, red);
    const int wib = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarp = blockDim.x >> 5;
    const int nb = b.cols / 32;
    unsigned long long best = pack_vi(-INFINITY, 0);
    for (int r = blockIdx.x * nwarp + wib; r < b.rows; r += gridDim.x * nwarp) {
        const uint8_t *row = b.w + (size_t)r * nb * 34;
        float acc = 0.f;
        for (int u = lane; u < nb * 4; u += 32) acc += q80_quarter(row + (size_t)(u >> 2) * 34, u & 3, b.x, b.norm_w, inv, (u >> 2) * 32);
        acc = warp_sum(acc);
        if (lane == 0) {
            b.y[r] = acc;
            const unsigned long long c = pack_vi(acc, r);
            if (c > best) best = c;
        }
    }
    if (lane == 0) best_w[wib] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long m = best_w[0];
        for (int k = 1; k < nwarp; k++) m = best_w[k] > m ? best_w[k] : m;
        a.partial[blockIdx.x] = m;
        __threadfence();
        last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        __threadfence();
        unsigned long long m = 0;
        for (int k = 0; k < (int)gridDim.x; k++) {
            const unsigned long long v = ((volatile unsigned long long *)a.partial)[k];
            m = v > m ? v : m;
        }
        *a.argmax_out = (int)(0xFFFFFFFFu - (uint32_t)(m & 0xFFFFFFFFull));
        *a.counter = 0;
    }
}

// ggml dequantize_row_q6_K, bit-exact: (d * (float)sc) * (float)(q - 32).
__global__ void q6k_dequant_kernel(const uint8_t *w, size_t nblk, float *out) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;   // weight index
    if (i >= nblk * 256) return;
    const size_t b = i >> 8;
    const int n = (int)(i & 255), h = n >> 7, j = (n >> 5) & 3, l = n & 31;
    const uint8_t *blk = w + b * 210;
    const uint8_t qlb = blk[64 * h + l + 32 * (j & 1)];
    const int lo = (j & 2) ? (qlb >> 4) : (qlb & 0xF);
    const int hi = (blk[128 + 32 * h + l] >> (2 * j)) & 3;
    const int q = (lo | (hi << 4)) - 32;
    const int8_t sc = (int8_t)blk[192 + 8 * h + 2 * j + l / 16];
    const float d = h2f_bits((uint16_t)(blk[208] | (blk[209] << 8)));
    out[i] = __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
}

// ggml dequantize_row_q8_0, bit-exact: (float)q * d.
__global__ void q80_dequant_kernel(const uint8_t *w, size_t nblk, float *out) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nblk * 32) return;
    const uint8_t *blk = w + (i >> 5) * 34;
    const float d = h2f_bits((uint16_t)(blk[0] | (blk[1] << 8)));
    out[i] = __fmul_rn((float)(int8_t)blk[2 + (i & 31)], d);
}

// One row of a Q8_0 matrix (the token embedding of the tied head).
__global__ void q80_row_kernel(const uint8_t *w, int rows, int cols, const int *tok, int row, float *out, int *err) {
    pdl_trigger();
    pdl_wait();   // *tok and out belong to the preceding kernels
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    int r = tok ? *tok : row;
    if (r < 0 || r >= rows) {   // a device-side token id out of range: report, read row 0
        if (c == 0) atomicExch(err, DEV_BAD_INDEX);
        r = 0;
    }
    const uint8_t *blk = w + ((size_t)r * (cols / 32) + (c >> 5)) * 34;
    const float d = h2f_bits((uint16_t)(blk[0] | (blk[1] << 8)));
    out[c] = __fmul_rn((float)(int8_t)blk[2 + (c & 31)], d);
}

// ============================================================ fast path ===
// Persistent CTAs (one per SM), each owning a contiguous row range. Tiles of
// block rows arrive by TMA (stream.cuh) in a 3-deep ring. A unit is 16
// weights (Q6_K: one half-block lane quad) or 8 weights (Q8_0: a quarter
// block); lane l of a warp takes units chunk + l + 32k, so the 32 lanes of one
// shared-memory load read neighbouring bytes, and every lane's columns are the
// same for every row: its activations live in registers.
constexpr int GF_WARPS = 16;
constexpr int GF_THREADS = GF_WARPS * 32;
constexpr int GF_NBUF = 3;

template <int FMT>
struct GFmt;
template <>
struct GFmt<0> {   // Q6_K
    static constexpr int BB = 210, WPB = 256, UPB = 16, WPU = 16, UMAX = 5;
};
template <>
struct GFmt<1> {   // Q8_0
    static constexpr int BB = 34, WPB = 32, UPB = 4, WPU = 8, UMAX = 10;
};

struct GFArgs {
    const uint8_t *w;
    int rows, cols;
    const float *x;
    const float *norm_w;
    float eps;
    float *y;
    int accumulate;
    int ks, tr;
    uint32_t rb_bytes, slot_bytes;
    unsigned long long *partial;   // head only
    unsigned int *counter;
    int *argmax_out;
    int *err;
};

// A 32-bit little-endian word at a 2-byte aligned shared-memory address.
__device__ __forceinline__ uint32_t lds_a2(const uint8_t *p) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>((uintptr_t)p & ~(uintptr_t)3);
    return __funnelshift_r(w[0], w[1], (uint32_t)((uintptr_t)p & 2) * 8u);
}

// Exact integer value of byte e of v minus `bias`, via 0x4B0000bb == 2^23 + bb.
__device__ __forceinline__ float byte_val(uint32_t v, int e, float bias) {
    return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | (uint32_t)e)) - bias;
}

template <int FMT>
__device__ __forceinline__ int unit_col(int u, int i) {
    if constexpr (FMT == 0) {
        const int b = u >> 4, h = (u >> 3) & 1, m = u & 7, j = i >> 2, e = i & 3;
        return 256 * b + 128 * h + 32 * j + 4 * m + e;
    }
    return 8 * u + i;
}

// Q6_K unit: half h, lane quad m (l = 4m..4m+3), quadrants j = 0..3.
__device__ __forceinline__ float q6k_unit_s(const uint8_t *row, int u, const float (&xu)[16]) {
    const int b = u >> 4, h = (u >> 3) & 1, m = u & 7;
    const uint8_t *blk = row + 210 * b;
    const uint32_t qa = lds_a2(blk + 64 * h + 4 * m);
    const uint32_t qb = lds_a2(blk + 64 * h + 32 + 4 * m);
    const uint32_t qh = lds_a2(blk + 128 + 32 * h + 4 * m);
    const uint8_t *S = blk + 192 + 8 * h + (m >> 2);
    const uint8_t *S2 = reinterpret_cast<const uint8_t *>((uintptr_t)S & ~(uintptr_t)1);
    const int o = (int)((uintptr_t)S & 1);
    const uint32_t slo = lds_a2(S2) ^ 0x80808080u, shi = lds_a2(S2 + 4) ^ 0x80808080u;
    const float d = h2f_bits(*reinterpret_cast<const uint16_t *>(blk + 208));
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t lo = ((j & 1) ? qb : qa) >> ((j & 2) ? 4 : 0);
        const uint32_t q = (lo & 0x0F0F0F0Fu) | (((qh >> (2 * j)) & 0x03030303u) << 4);
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < 4; e++) s = fmaf(byte_val(q, e, 8388640.0f), xu[4 * j + e], s);   // q - 32
        const int sb = o + 2 * j;                                   // scale byte in the window
        const uint32_t sw = sb < 4 ? slo : shi;
        const float sc = __uint_as_float(__byte_perm(sw, 0x4B000000u, 0x7440u | (uint32_t)(sb & 3))) - 8388736.0f;
        acc = fmaf(d * sc, s, acc);
    }
    return acc;
}

// Q8_0 unit: quarter k of block b.
__device__ __forceinline__ float q80_unit_s(const uint8_t *row, int u, const float (&xu)[8]) {
    const uint8_t *blk = row + 34 * (u >> 2);
    const int k = u & 3;
    const float d = h2f_bits(*reinterpret_cast<const uint16_t *>(blk));
    const uint32_t w0 = lds_a2(blk + 2 + 8 * k) ^ 0x80808080u, w1 = lds_a2(blk + 6 + 8 * k) ^ 0x80808080u;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int e = 0; e < 4; e++) {
        s0 = fmaf(byte_val(w0, e, 8388736.0f), xu[e], s0);
        s1 = fmaf(byte_val(w1, e, 8388736.0f), xu[4 + e], s1);
    }
    return d * (s0 + s1);
}

__device__ __forceinline__ void gf_issue(const GFArgs &a, uint8_t *slot, uint64_t *bar, int r0, int nr) {
    BulkList<1> bl;
    bl.tx = 0;
    const uintptr_t A = (uintptr_t)(a.w + (size_t)r0 * a.rb_bytes);
    const uintptr_t limit = (uintptr_t)(a.w + (size_t)a.rows * a.rb_bytes);   // no slack promised
    bulk_plan(bl, 0, slot, A, A + (size_t)nr * a.rb_bytes, limit);
    bulk_issue(bl, bar);
}

template <int FMT, int U, int HEAD>
__global__ void __launch_bounds__(GF_THREADS, 1) blk_fast_kernel(const GFArgs a) {
    using Fm = GFmt<FMT>;
    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t *ring = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(ring + (size_t)GF_NBUF * a.slot_bytes);
    float *part = reinterpret_cast<float *>(full + GF_NBUF);   // [2][tr][ks]
    double *red = reinterpret_cast<double *>(part + 2 * a.tr * a.ks);
    unsigned long long *bw = reinterpret_cast<unsigned long long *>(red + 32);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ks_n = a.ks, tr = a.tr, ks = warp % ks_n, rw = warp / ks_n;
    const int G = gridDim.x;
    const int rb = (int)(((long long)blockIdx.x * a.rows) / G), re = (int)(((long long)(blockIdx.x + 1) * a.rows) / G);
    const int ntile = (re - rb + tr - 1) / tr;

    pdl_trigger();
    if (tid == 0) {
        for (int b = 0; b < GF_NBUF; b++) mbar_init(&full[b], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0)
        for (int t = 0; t < GF_NBUF - 1 && t < ntile; t++) {
            const int r0 = rb + t * tr;
            gf_issue(a, ring + (size_t)t * a.slot_bytes, &full[t], r0, min(tr, re - r0));
        }
    pdl_wait();   // the weight tiles above are immutable; x, y and the scratch are not
    float inv = 1.0f;
    if (a.norm_w) inv = block_rms_inv(a.x, a.cols, a.eps, red);
    float xr[U][Fm::WPU];
    const int u0 = ks * 32 * U + lane;
#pragma unroll
    for (int k = 0; k < U; k++)
#pragma unroll
        for (int i = 0; i < Fm::WPU; i++) {
            const int c = unit_col<FMT>(u0 + 32 * k, i);
            float v = a.x[c];
            if (a.norm_w) v = __fmul_rn(__fmul_rn(v, inv), a.norm_w[c]);
            xr[k][i] = v;
        }
    unsigned long long best = pack_vi(-INFINITY, 0);

    for (int t = 0; t < ntile; t++) {
        const int slot = t % GF_NBUF;
        if (tid == 0 && t + GF_NBUF - 1 < ntile) {
            const int tn = t + GF_NBUF - 1, r0n = rb + tn * tr;
            gf_issue(a, ring + (size_t)(tn % GF_NBUF) * a.slot_bytes, &full[tn % GF_NBUF], r0n, min(tr, re - r0n));
        }
        const int r0 = rb + t * tr, nr = min(tr, re - r0);
        // a wait that runs out records the error and skips the tile; every thread
        // still reaches the barrier below
        const bool have = mbar_wait(&full[slot], (uint32_t)((t / GF_NBUF) & 1), a.err);
        float *pt = part + (size_t)(t & 1) * tr * ks_n;
        if (rw < nr) {
            const uintptr_t A = (uintptr_t)(a.w + (size_t)r0 * a.rb_bytes);
            const uint8_t *row = ring + (size_t)slot * a.slot_bytes + (A & 15) + (size_t)rw * a.rb_bytes;
            float acc = 0.f;
#pragma unroll
            for (int k = 0; k < U; k++) {
                if (!have) break;
                if constexpr (FMT == 0)
                    acc += q6k_unit_s(row, u0 + 32 * k, reinterpret_cast<const float(&)[16]>(xr[k]));
                else
                    acc += q80_unit_s(row, u0 + 32 * k, reinterpret_cast<const float(&)[8]>(xr[k]));
            }
            acc = warp_sum(acc);
            if (lane == 0) pt[rw * ks_n + ks] = acc;
        }
        __syncthreads();
        if (tid < nr) {
            const int r = r0 + tid;
            float v = 0.f;
            for (int k = 0; k < ks_n; k++) v += pt[tid * ks_n + k];
            const float o = (a.accumulate ? a.y[r] : 0.0f) + v;
            a.y[r] = o;
            if (HEAD) {
                const unsigned long long c = pack_vi(o, r);
                best = c > best ? c : best;
            }
        }
    }
    if (HEAD) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
            best = o > best ? o : best;
        }
        if (lane == 0) bw[warp] = best;
        __syncthreads();
        if (tid == 0) {
            unsigned long long m = bw[0];
            for (int k = 1; k < GF_WARPS; k++) m = bw[k] > m ? bw[k] : m;
            a.partial[blockIdx.x] = m;
            __threadfence();
            const bool last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
            if (last) {
                __threadfence();
                unsigned long long mm = 0;
                for (int k = 0; k < (int)gridDim.x; k++) {
                    const unsigned long long v = ((volatile unsigned long long *)a.partial)[k];
                    mm = v > mm ? v : mm;
                }
                *a.argmax_out = (int)(0xFFFFFFFFu - (uint32_t)(mm & 0xFFFFFFFFull));
                *a.counter = 0;
            }
        }
    }
}

struct GFPlan {
    int U;
    size_t smem;
    GFArgs a;
};

// The fast path needs whole lane runs of units: units per row divisible by 32*ks
// with U = units/(32 ks) one of the instantiated widths.
bool gf_plan(int fmt, const void *w, int rows, int cols, GFPlan *P) {
    const int wpb = fmt == 0 ? 256 : 32, upb = fmt == 0 ? 16 : 4, bb = fmt == 0 ? 210 : 34;
    const int umax = fmt == 0 ? 5 : 10;
    const long nu = (long)(cols / wpb) * upb;
    int ks = 0, U = 0;
    for (int k = 1; k <= 16; k *= 2) {
        if (nu % (32 * k)) continue;
        const int u = (int)(nu / (32 * k));
        const bool ok = fmt == 0 ? (u == 1 || u == 2 || u == 4 || u == 5)
                                 : (u == 1 || u == 2 || u == 4 || u == 5 || u == 8 || u == 10);
        if (ok && u <= umax) {
            ks = k;
            U = u;
            break;
        }
    }
    if (!ks) return false;
    GFArgs &a = P->a;
    memset(&a, 0, sizeof a);
    a.w = (const uint8_t *)w;
    a.rows = rows;
    a.cols = cols;
    a.ks = ks;
    a.tr = GF_WARPS / ks;
    a.rb_bytes = (uint32_t)((cols / wpb) * bb);
    a.slot_bytes = (uint32_t)(((size_t)a.tr * a.rb_bytes + 32 + 15) & ~(size_t)15);
    P->U = U;
    P->smem = (size_t)GF_NBUF * a.slot_bytes + GF_NBUF * 8 + (size_t)2 * a.tr * ks * 4 + 32 * 8 + GF_WARPS * 8;
    return P->smem <= smem_optin_max();
}

template <int FMT, int U, int HEAD>
int gf_launch_t(const GFPlan &P, cudaStream_t s) {
    auto k = blk_fast_kernel<FMT, U, HEAD>;
    static size_t opted[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (P.smem > opted[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P.smem);
        if (e != cudaSuccess) return cuda_fail("ggml fast kernel shared-memory opt-in", e);
        opted[dev & 63] = P.smem;
    }
    const int ntr = (P.a.rows + P.a.tr - 1) / P.a.tr;
    const int grid = ntr < sm_count() ? ntr : sm_count();
    cudaError_t e = launch_pdl(k, dim3(grid), dim3(GF_THREADS), P.smem, s, P.a);
    return e == cudaSuccess ? 0 : cuda_fail("ggml fast kernel launch", e);
}

template <int HEAD>
int gf_launch(int fmt, const GFPlan &P, cudaStream_t s) {
    if (fmt == 0) {
        switch (P.U) {
            case 1: return gf_launch_t<0, 1, HEAD>(P, s);
            case 2: return gf_launch_t<0, 2, HEAD>(P, s);
            case 4: return gf_launch_t<0, 4, HEAD>(P, s);
            case 5: return gf_launch_t<0, 5, HEAD>(P, s);
        }
    } else {
        switch (P.U) {
            case 1: return gf_launch_t<1, 1, HEAD>(P, s);
            case 2: return gf_launch_t<1, 2, HEAD>(P, s);
            case 4: return gf_launch_t<1, 4, HEAD>(P, s);
            case 5: return gf_launch_t<1, 5, HEAD>(P, s);
            case 8: return gf_launch_t<1, 8, HEAD>(P, s);
            case 10: return gf_launch_t<1, 10, HEAD>(P, s);
        }
    }
    return set_error("ggml fast kernel: no instantiation for U=%d", P.U);
}

int check_blocks(const void *w, int rows, int cols, int wpb) {
    if (!w) return set_error("weight pointer is null");
    if (rows <= 0 || cols <= 0) return set_error("gemv needs a non-empty matrix");
    if (cols % wpb) return set_error("cols %d is not a multiple of the %d-weight block", cols, wpb);
    if ((uintptr_t)w & 1) return set_error("block pointer must be 2-byte aligned");
    return 0;
}

int launch_blk(bool q6k, const BlkArgs &a, cudaStream_t s) {
    const int threads = 256;
    const int blocks = (int)(((size_t)a.rows * 32 + threads - 1) / threads);
    if (q6k)
        q6k_gemv_kernel<<<blocks, threads, 0, s>>>(a);
    else
        q80_gemv_kernel<<<blocks, threads, 0, s>>>(a);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail(q6k ? "q6_k gemv launch" : "q8_0 gemv launch", e);
}

unsigned int *g_head_counter[64];
unsigned long long *g_head_partial[64];

}  // namespace

extern "C" {

/* Q6_K dequant-GEMV over raw ggml blocks: y = (accumulate ? y : 0) + W x, with
 * an optional RMSNorm(x; norm_w, eps) prologue. All pointers are device pointers. */
int spk_q6k_gemv(const void *w, int rows, int cols, const float *x, const float *norm_w, float eps, float *y,
                 int accumulate, void *stream) {
    if (check_blocks(w, rows, cols, 256)) return -1;
    GFPlan P;
    if (gf_plan(0, w, rows, cols, &P)) {
        P.a.x = x;
        P.a.norm_w = norm_w;
        P.a.eps = eps;
        P.a.y = y;
        P.a.accumulate = accumulate;
        P.a.err = device_error_ptr();
        return gf_launch<0>(0, P, (cudaStream_t)stream);
    }
    BlkArgs a = {(const uint8_t *)w, rows, cols, x, norm_w, eps, y, accumulate};
    return launch_blk(true, a, (cudaStream_t)stream);
}

/* Q8_0 dequant-GEMV over raw ggml blocks (same contract as spk_q6k_gemv). */
int spk_q80_gemv(const void *w, int rows, int cols, const float *x, const float *norm_w, float eps, float *y,
                 int accumulate, void *stream) {
    if (check_blocks(w, rows, cols, 32)) return -1;
    GFPlan P;
    if (gf_plan(1, w, rows, cols, &P)) {
        P.a.x = x;
        P.a.norm_w = norm_w;
        P.a.eps = eps;
        P.a.y = y;
        P.a.accumulate = accumulate;
        P.a.err = device_error_ptr();
        return gf_launch<0>(1, P, (cudaStream_t)stream);
    }
    BlkArgs a = {(const uint8_t *)w, rows, cols, x, norm_w, eps, y, accumulate};
    return launch_blk(false, a, (cudaStream_t)stream);
}

/* Tied Q8_0 head: logits = W RMSNorm(x) and the first index of the maximum
 * logit into *argmax_out (device int). Logits are written, not accumulated. */
int spk_q80_head(const void *w, int rows, int cols, const float *x, const float *norm_w, float eps, float *logits,
                 int *argmax_out, void *stream) {
    if (check_blocks(w, rows, cols, 32)) return -1;
    if (!argmax_out) return set_error("argmax output pointer is null");
    int dev = 0;
    cudaGetDevice(&dev);
    const int grid = 2 * sm_count() < 1024 ? 2 * sm_count() : 1024;   // the partial buffer holds 1024 slots
    if (!g_head_counter[dev & 63]) {
        void *c = nullptr, *p = nullptr;
        cudaError_t e = cudaMalloc(&c, sizeof(unsigned int));
        if (e == cudaSuccess) e = cudaMalloc(&p, sizeof(unsigned long long) * 1024);
        if (e == cudaSuccess) e = cudaMemset(c, 0, sizeof(unsigned int));
        if (e != cudaSuccess) return cuda_fail("head scratch allocation", e);
        g_head_counter[dev & 63] = (unsigned int *)c;
        g_head_partial[dev & 63] = (unsigned long long *)p;
    }
    GFPlan P;
    if (gf_plan(1, w, rows, cols, &P)) {
        P.a.x = x;
        P.a.norm_w = norm_w;
        P.a.eps = eps;
        P.a.y = logits;
        P.a.accumulate = 0;
        P.a.partial = g_head_partial[dev & 63];
        P.a.counter = g_head_counter[dev & 63];
        P.a.argmax_out = argmax_out;
        P.a.err = device_error_ptr();
        return gf_launch<1>(1, P, (cudaStream_t)stream);
    }
    HeadArgs a;
    a.b = {(const uint8_t *)w, rows, cols, x, norm_w, eps, logits, 0};
    a.partial = g_head_partial[dev & 63];
    a.counter = g_head_counter[dev & 63];
    a.argmax_out = argmax_out;
    q80_head_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(a);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail("q8_0 head launch", e);
}

}  // extern "C"

namespace spk {
// The head with caller-owned scratch (partial: >= sm_count() entries, counter
// zeroed once), for callers that capture it in a graph.
int q80_head_launch(const void *w, int rows, int cols, const float *x, const float *norm_w, float eps, float *logits,
                    int *argmax_out, unsigned long long *partial, unsigned int *counter, cudaStream_t s) {
    if (check_blocks(w, rows, cols, 32)) return -1;
    GFPlan P;
    if (gf_plan(1, w, rows, cols, &P)) {
        P.a.x = x;
        P.a.norm_w = norm_w;
        P.a.eps = eps;
        P.a.y = logits;
        P.a.accumulate = 0;
        P.a.partial = partial;
        P.a.counter = counter;
        P.a.argmax_out = argmax_out;
        P.a.err = device_error_ptr();
        return gf_launch<1>(1, P, s);
    }
    HeadArgs a;
    a.b = {(const uint8_t *)w, rows, cols, x, norm_w, eps, logits, 0};
    a.partial = partial;
    a.counter = counter;
    a.argmax_out = argmax_out;
    cudaError_t e = launch_pdl(q80_head_kernel, dim3(2 * sm_count() < 1024 ? 2 * sm_count() : 1024), dim3(256), 0, s, a);
    return e == cudaSuccess ? 0 : cuda_fail("q8_0 head launch", e);
}
}  // namespace spk

extern "C" {

/* Bit-exact block decode into f32 (nblocks * 256 or * 32 values). */
int spk_q6k_dequant(const void *w, size_t nblocks, float *out, void *stream) {
    if (!w || !out) return set_error("dequant needs input and output");
    const size_t n = nblocks * 256;
    q6k_dequant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>((const uint8_t *)w, nblocks, out);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail("q6_k dequant launch", e);
}

int spk_q80_dequant(const void *w, size_t nblocks, float *out, void *stream) {
    if (!w || !out) return set_error("dequant needs input and output");
    const size_t n = nblocks * 32;
    q80_dequant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>((const uint8_t *)w, nblocks, out);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail("q8_0 dequant launch", e);
}

/* One decoded row of a Q8_0 matrix into out[cols]: row `row`, or *token when
 * token (device int) is not null — the token-embedding gather of a tied head. */
int spk_q80_row(const void *w, int rows, int cols, int row, const int *token, float *out, void *stream) {
    if (check_blocks(w, rows, cols, 32)) return -1;
    if (!token && (row < 0 || row >= rows)) return set_error("row %d is outside %d", row, rows);
    cudaError_t e = launch_pdl(q80_row_kernel, dim3((cols + 255) / 256), dim3(256), 0, (cudaStream_t)stream,
                               (const uint8_t *)w, rows, cols, token, row, out, device_error_ptr());
    return e == cudaSuccess ? 0 : cuda_fail("q8_0 row launch", e);
}

}  // extern "C"

// ================================================ head with no allocation ===
// spk_q80_head keeps its scratch (one 8-byte partial per CTA plus a finishing
// counter) in memory it allocates with cudaMalloc on first use. Some callers
// cannot allow that: code running while a stream is being captured into a CUDA
// graph (cudaMalloc is not permitted there), real-time decode loops that must
// not stall on the implicit device synchronization an allocation can cause,
// and host frameworks that own every device byte through their own pool and
// forbid a library from allocating behind them. For them the same head runs
// with its scratch in the fixed array below, which lives in the library's
// device image: every GPU that loads libspk holds these 8,448 bytes until the
// process exits.
namespace {
constexpr int NOALLOC_HEAD_MAX_CTAS = 1024;   // partial slots: the largest grid this head may launch
constexpr int NOALLOC_HEAD_PARTIAL0 = 32;     // the counter sits in slot 0; partials start 256 bytes in
static __device__ __align__(256) unsigned long long g_head_noalloc_scratch[NOALLOC_HEAD_PARTIAL0 + NOALLOC_HEAD_MAX_CTAS];
// Device address of the array per device. In host code the array's name is
// only a host-side stand-in, never a device address, so it is looked up with
// cudaGetSymbolAddress once per device, with that device current.
static unsigned long long *g_head_noalloc_dev[64];
}  // namespace

extern "C" {

/* Tied Q8_0 head without any allocation (no counterpart in the reference): the
 * same contract as spk_q80_head — logits = W RMSNorm(x) and the first index of the
 * maximum into *argmax_out — but its scratch is a fixed array inside libspk.
 * Limits and rules:
 *  - the launch may use at most 1024 CTAs (at most sm_count CTAs are used on the
 *    fast path, 2 x sm_count capped at 1024 otherwise); a launch needing more is
 *    rejected with an error;
 *  - the first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress) — make that first call before any stream capture;
 *  - every call on a device shares the one array and leaves its contents behind;
 *    each call clears the counter it needs at zero (an asynchronous memset on
 *    `stream`, not an allocation), and calls that overlap on the GPU (different
 *    streams, or graphs replayed concurrently) race on it: serialize them. */
int spk_q80_head_noalloc(const void *w, int rows, int cols, const float *x, const float *norm_w, float eps,
                         float *logits, int *argmax_out, void *stream) {
    if (check_blocks(w, rows, cols, 32)) return -1;
    if (!argmax_out || !x || !logits) return set_error("head needs x, logits and argmax_out");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail("no-alloc head: current device", e);
    if (dev < 0 || dev >= 64) return set_error("no-alloc head: device %d is outside the 64 this build tracks", dev);
    if (!g_head_noalloc_dev[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_head_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail("no-alloc head: scratch address", e);
        g_head_noalloc_dev[dev] = (unsigned long long *)p;
    }
    GFPlan P;
    int grid;
    if (gf_plan(1, w, rows, cols, &P)) {
        const int ntr = (rows + P.a.tr - 1) / P.a.tr;
        grid = ntr < sm_count() ? ntr : sm_count();
    } else {
        grid = 2 * sm_count() < 1024 ? 2 * sm_count() : 1024;
    }
    if (grid > NOALLOC_HEAD_MAX_CTAS)
        return set_error("no-alloc head: this launch needs %d CTAs, the built-in scratch holds %d", grid,
                         NOALLOC_HEAD_MAX_CTAS);
    unsigned long long *base = g_head_noalloc_dev[dev];
    unsigned int *counter = reinterpret_cast<unsigned int *>(base);
    e = cudaMemsetAsync(counter, 0, sizeof(unsigned int), (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail("no-alloc head: clear counter", e);
    return q80_head_launch(w, rows, cols, x, norm_w, eps, logits, argmax_out, base + NOALLOC_HEAD_PARTIAL0, counter,
                           (cudaStream_t)stream);
}

}  // extern "C"
