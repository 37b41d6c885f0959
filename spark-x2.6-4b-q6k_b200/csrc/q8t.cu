// q8t.cu — the tied Q8_0 head in a tensor-core tile layout.
//
// ggml's Q8_0 rows (34-byte blocks: f16 d, 32 int8) are re-laid once, at load, into
// tile-blocks of 16 rows x 32 columns, 544 bytes each (the bytes of the 16 blocks they
// replace), a row tile's blocks consecutive:
//   [rows/16][cols/32] tile-blocks of { 512 B quants, 32 B the 16 rows' d (f16) }
// with the quants in mma.sync fragment order: lane L = 4g + t of a warp reads bytes
// [16L, 16L + 16) = row g cols 4t..4t+3 | row g+8 cols 4t..4t+3 | row g cols 16+4t..
// | row g+8 cols 16+4t.. — its A fragments for both k16 halves of the block (inside a
// half the K order is permuted: thread t's four k-slots are four consecutive columns,
// and B uses the same map). One aligned, conflict-free 16-byte load per lane per block.
//
// The GEMV: persistent CTA per SM over a contiguous range of row tiles; a row tile
// (contiguous, cols/32 x 544 bytes) arrives by one TMA bulk copy into a 3-slot ring
// (stream.cuh); 8 warps split its K range. int8 -> f16 exactly (byte ^ 0x80 under the
// exponent of 1024, minus 1152), x as an f16 pair hi + lo staged in shared memory, one
// block's two halves into a fresh accumulator, then y += d * (that sum) in f32; the
// warps' partials meet in shared memory in a fixed order, and the first-max argmax
// over the rows is fused (per-CTA key, the last CTA reduces).
#include "common.cuh"
#include "spk.h"
#include "stream.cuh"

namespace spk {

namespace {

constexpr int QT_WARPS = 8, QT_THREADS = QT_WARPS * 32;
constexpr int QT_MAXT = 8;
constexpr int QT_MAXCOLS = 4096;
constexpr int QT_BB = 544;                     // bytes per tile-block
constexpr int QT_NBUF = 3;
constexpr int QT_MAXCTA = 1024;

struct QtArgs {
    const uint8_t *w;          // tiled
    int rows, cols, ntok;      // rows a multiple of 16
    const float *x;
    int ldx;
    const float *norm_w;
    float eps;
    float *logits;
    int ldl;
    int *amax;                 // [ntok] or null
    unsigned long long *partial;   // [gridDim.x][QT_MAXT]
    unsigned int *counter;         // zero; the last CTA resets it
    uint32_t tile_bytes;
    int *err;
};

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four int8 of w as two exact f16 pairs (bytes 0,1 | bytes 2,3), low half first.
__device__ __forceinline__ void s8x4_to_f16(uint32_t w, uint32_t &lo, uint32_t &hi) {
    const uint32_t b = w ^ 0x80808080u;   // q + 128, as unsigned bytes
    uint32_t l = __byte_perm(b, 0x64646464u, 0x5140u), h = __byte_perm(b, 0x64646464u, 0x7362u);
    const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6480u));   // 1152
    const __half2 lv = __hsub2(*reinterpret_cast<__half2 *>(&l), bias);
    const __half2 hv = __hsub2(*reinterpret_cast<__half2 *>(&h), bias);
    lo = *reinterpret_cast<const uint32_t *>(&lv);
    hi = *reinterpret_cast<const uint32_t *>(&hv);
}

__device__ __forceinline__ unsigned long long qt_key(float v, int i) {
    uint32_t u = __float_as_uint(v);
    if (u == 0x80000000u) u = 0u;
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    if (v != v) u = 0u;
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)i);
}

// ggml Q8_0 rows -> tile-blocks: one thread per 16-byte unit (32 lane chunks + 2 of d).
__global__ void q8t_pack_kernel(const uint8_t *src, int rows, int cols, uint8_t *dst) {
    const int nb = cols / 32;
    const size_t total = (size_t)((rows + 15) / 16) * nb * 34;
    for (size_t u = blockIdx.x * (size_t)blockDim.x + threadIdx.x; u < total; u += (size_t)gridDim.x * blockDim.x) {
        const size_t tb = u / 34;
        const int k = (int)(u % 34);
        const int R = (int)(tb / nb), B = (int)(tb % nb);
        uint8_t out[16];
        if (k < 32) {   // lane k: rows g, g+8 at cols 4t.., 16+4t..
            const int g = k >> 2, t = k & 3;
#pragma unroll
            for (int part = 0; part < 4; part++) {
                const int row = 16 * R + g + 8 * (part & 1), col = 16 * (part >> 1) + 4 * t;
                const uint8_t *blk = src + ((size_t)row * nb + B) * 34;
#pragma unroll
                for (int e = 0; e < 4; e++) out[4 * part + e] = row < rows ? blk[2 + col + e] : 0;
            }
        } else {        // d of rows 8(k-32) .. +7
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int row = 16 * R + 8 * (k - 32) + j;
                const uint8_t *blk = src + ((size_t)row * nb + B) * 34;
                out[2 * j] = row < rows ? blk[0] : 0;
                out[2 * j + 1] = row < rows ? blk[1] : 0;
            }
        }
        uint4 v;
        memcpy(&v, out, 16);
        *reinterpret_cast<uint4 *>(dst + tb * QT_BB + 16 * (size_t)k) = v;
    }
}

// TWO = 0: one token, B columns 0 / 1 = x hi / lo (one MMA per half);
// TWO = 1: up to 8 tokens as B columns, hi then lo (two MMAs per half).
template <int TWO>
__global__ void __launch_bounds__(QT_THREADS, 1) q8t_head_kernel(const QtArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float red[2][QT_WARPS][16][8];   // by tile parity
    __shared__ float inv[QT_MAXT];
    __shared__ unsigned long long bw[16][QT_MAXT];
    __shared__ bool last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int nt = TWO ? a.ntok : 1;
    const int hc = a.cols / 2 + 8;   // words per staged x row, padded: the 8 token rows in different banks
    const int nb = a.cols / 32, ntiles = a.rows / 16;
    uint8_t *ring = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(ring + (size_t)QT_NBUF * a.tile_bytes);
    uint64_t *empty = full + QT_NBUF;
    uint32_t *xs = reinterpret_cast<uint32_t *>(empty + QT_NBUF);   // [2 nt][hc] f16 pairs: hi rows, lo rows

    const int G = gridDim.x;
    const int tb0 = (int)((long long)blockIdx.x * ntiles / G), tb1 = (int)((long long)(blockIdx.x + 1) * ntiles / G);
    const int ntile = tb1 - tb0;
    pdl_trigger();
    if (tid == 0) {
        for (int b = 0; b < QT_NBUF; b++) {
            mbar_init(&full[b], 1);
            mbar_init(&empty[b], QT_WARPS);
        }
        fence_mbar_init();
    }
    __syncthreads();
    auto issue = [&](int k, int slot) {
        const uint8_t *src = a.w + (size_t)(tb0 + k) * a.tile_bytes;
        mbar_arrive_expect_tx(&full[slot], a.tile_bytes);
        fence_proxy_async();
        bulk_g2s(ring + (size_t)slot * a.tile_bytes, src, a.tile_bytes, &full[slot]);
    };
    if (tid == 0)
        for (int k = 0; k < QT_NBUF - 1 && k < ntile; k++) issue(k, k);   // weights only, before the wait
    pdl_wait();
    // per-token RMSNorm scale (f64 sum of squares, model.rs:236-245), then x -> f16 hi/lo
    if (warp < nt) {
        float iv = 1.0f;
        if (a.norm_w) {
            const float *xr = a.x + (size_t)warp * a.ldx;
            double sq = 0.0;
            for (int i = lane; i < a.cols; i += 32) sq += (double)xr[i] * (double)xr[i];
            sq = warp_sum_d(sq);
            iv = (float)(1.0 / sqrt(sq / (double)a.cols + (double)a.eps));
        }
        if (lane == 0) inv[warp] = iv;
    }
    __syncthreads();
    for (int i = tid; i < nt * (a.cols / 2); i += QT_THREADS) {
        const int n = i / (a.cols / 2), c = 2 * (i - n * (a.cols / 2));
        float v0 = a.x[(size_t)n * a.ldx + c], v1 = a.x[(size_t)n * a.ldx + c + 1];
        if (a.norm_w) {
            v0 = __fmul_rn(__fmul_rn(v0, inv[n]), a.norm_w[c]);
            v1 = __fmul_rn(__fmul_rn(v1, inv[n]), a.norm_w[c + 1]);
        }
        const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
        const __half l0 = __float2half_rn(v0 - __half2float(h0)), l1 = __float2half_rn(v1 - __half2float(h1));
        xs[(size_t)n * hc + (c >> 1)] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
        xs[(size_t)(nt + n) * hc + (c >> 1)] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
    }
    __syncthreads();

    const int b0 = warp * nb / QT_WARPS, b1 = (warp + 1) * nb / QT_WARPS;   // this warp's blocks of a tile
    // B column of this thread: token g (TWO), or g = 0 hi / g = 1 lo (one token)
    const bool bl = TWO ? g < nt : g < 2;
    const uint32_t *xb = TWO ? xs + (size_t)g * hc : xs + (size_t)(g == 1 ? nt : 0) * hc;
    const uint32_t *xl = xs + (size_t)(nt + (g < nt ? g : 0)) * hc;   // TWO: this token's lo
    const int er = tid >> 3, en = tid & 7;   // epilogue thread: tile row er (< 16), token en
    unsigned long long best = qt_key(-INFINITY, 0);

    for (int k = 0; k < ntile; k++) {
        const int slot = k % QT_NBUF;
        if (tid == 0 && k + QT_NBUF - 1 < ntile) {
            const int kn = k + QT_NBUF - 1, sn = kn % QT_NBUF;
            if (kn < QT_NBUF || mbar_wait(&empty[sn], (uint32_t)(((kn / QT_NBUF) - 1) & 1), a.err)) issue(kn, sn);
        }
        // a wait that runs out records the error and skips the tile; no thread leaves the loop
        const bool have = mbar_wait(&full[slot], (uint32_t)((k / QT_NBUF) & 1), a.err);
        const uint8_t *tile = ring + (size_t)slot * a.tile_bytes;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        if (have) {
#pragma unroll 2
            for (int b = b0; b < b1; b++) {
                const uint8_t *blk = tile + (size_t)b * QT_BB;
                const uint4 q = *reinterpret_cast<const uint4 *>(blk + 16 * lane);
                const uint16_t *dp = reinterpret_cast<const uint16_t *>(blk + 512);
                const float da = __half2float(__ushort_as_half(dp[g])), db = __half2float(__ushort_as_half(dp[g + 8]));
                uint32_t a00, a02, a01, a03, a10, a12, a11, a13;
                s8x4_to_f16(q.x, a00, a02);   // row g, half 0
                s8x4_to_f16(q.y, a01, a03);   // row g+8, half 0
                s8x4_to_f16(q.z, a10, a12);   // row g, half 1
                s8x4_to_f16(q.w, a11, a13);   // row g+8, half 1
                const int c0 = b * 16 + 2 * t;   // f16-pair index of cols 32 b + 4t
                float s[4] = {0.f, 0.f, 0.f, 0.f};
                mma_f16(s, a00, a01, a02, a03, bl ? xb[c0] : 0u, bl ? xb[c0 + 1] : 0u);
                mma_f16(s, a10, a11, a12, a13, bl ? xb[c0 + 8] : 0u, bl ? xb[c0 + 9] : 0u);
                if (TWO) {
                    mma_f16(s, a00, a01, a02, a03, bl ? xl[c0] : 0u, bl ? xl[c0 + 1] : 0u);
                    mma_f16(s, a10, a11, a12, a13, bl ? xl[c0 + 8] : 0u, bl ? xl[c0 + 9] : 0u);
                }
                acc[0] = fmaf(da, s[0], acc[0]);
                acc[1] = fmaf(da, s[1], acc[1]);
                acc[2] = fmaf(db, s[2], acc[2]);
                acc[3] = fmaf(db, s[3], acc[3]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        float(*rw)[8] = red[k & 1][warp];
        rw[g][2 * t] = acc[0];
        rw[g][2 * t + 1] = acc[1];
        rw[g + 8][2 * t] = acc[2];
        rw[g + 8][2 * t + 1] = acc[3];
        __syncthreads();
        // no second barrier: tile k + 2 rewrites red[k & 1] only after every thread has passed
        // tile k + 1's barrier, which follows this reduction
        if (tid < 16 * 8 && en < nt) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < QT_WARPS; w++) v += TWO ? red[k & 1][w][er][en] : red[k & 1][w][er][0] + red[k & 1][w][er][1];
            const int row = (tb0 + k) * 16 + er;
            a.logits[(size_t)en * a.ldl + row] = v;
            const unsigned long long c = qt_key(v, row);
            best = c > best ? c : best;
        }
    }
    if (!a.amax) return;
    // per token: the CTA's best over its rows, then over CTAs by the last CTA
    if (tid < 16 * 8) bw[er][en] = best;
    __syncthreads();
    if (tid < nt) {
        unsigned long long b = 0ull;
        for (int r = 0; r < 16; r++) b = bw[r][tid] > b ? bw[r][tid] : b;
        a.partial[(size_t)blockIdx.x * QT_MAXT + tid] = b;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (tid < nt) {
        unsigned long long b = 0ull;
        for (int c = 0; c < (int)gridDim.x; c++) {
            const unsigned long long p = __ldcg(a.partial + (size_t)c * QT_MAXT + tid);
            b = p > b ? p : b;
        }
        a.amax[tid] = (int)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull));
    }
    if (tid == 0) *a.counter = 0u;
}

}  // namespace

size_t q8t_bytes(int rows, int cols) { return (size_t)((rows + 15) / 16) * (cols / 32) * QT_BB; }

size_t q8t_scratch() { return (size_t)QT_MAXCTA * QT_MAXT * sizeof(unsigned long long) + 256; }

int q8t_pack(const void *w, int rows, int cols, void *dst, cudaStream_t s) {
    if (!w || !dst || rows < 1 || cols < 32 || cols % 32) return set_error("q8t pack: bad arguments");
    q8t_pack_kernel<<<sm_count() * 4, 256, 0, s>>>((const uint8_t *)w, rows, cols, (uint8_t *)dst);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail("q8t pack launch", e);
}

// 1 launched, 0 geometry not taken, -1 error.
int q8t_head_launch(const void *wt, int rows, int cols, int ntok, const float *x, int ldx, const float *norm_w,
                    float eps, float *logits, int ldl, int *amax, void *scratch, cudaStream_t s) {
    if (rows % 16 || cols % 32 || cols < 32 * QT_WARPS || cols > QT_MAXCOLS || ntok < 1 || ntok > QT_MAXT) return 0;
    if (((uintptr_t)wt & 15) || ((uintptr_t)x & 3)) return 0;
    QtArgs A;
    memset(&A, 0, sizeof A);
    A.w = (const uint8_t *)wt;
    A.rows = rows;
    A.cols = cols;
    A.ntok = ntok;
    A.x = x;
    A.ldx = ldx;
    A.norm_w = norm_w;
    A.eps = eps;
    A.logits = logits;
    A.ldl = ldl;
    A.amax = amax;
    A.counter = reinterpret_cast<unsigned int *>(scratch);
    A.partial = reinterpret_cast<unsigned long long *>((uint8_t *)scratch + 256);
    A.tile_bytes = (uint32_t)((cols / 32) * QT_BB);
    A.err = device_error_ptr();
    const int two = ntok > 1;
    const size_t smem = (size_t)QT_NBUF * A.tile_bytes + 2 * QT_NBUF * 8 +
                        (size_t)2 * (two ? ntok : 1) * (cols / 2 + 8) * 4;
    if (smem + 10 * 1024 > smem_optin_max()) return 0;   // + the kernel's static shared memory
    const int ntiles = rows / 16;
    int grid = sm_count() < QT_MAXCTA ? sm_count() : QT_MAXCTA;
    if (grid > ntiles) grid = ntiles;
    static size_t opted[2][64];
    int dev = 0;
    cudaGetDevice(&dev);
    auto k = two ? q8t_head_kernel<1> : q8t_head_kernel<0>;
    if (smem > opted[two][dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_fail("q8t head shared-memory opt-in", e);
        opted[two][dev & 63] = smem;
    }
    const cudaError_t e = launch_pdl(k, dim3(grid), dim3(QT_THREADS), smem, s, A);
    return e == cudaSuccess ? 1 : cuda_fail("q8t head launch", e);
}

}  // namespace spk

using namespace spk;

extern "C" {

size_t spk_q80_tile_bytes(int rows, int cols) { return (rows < 1 || cols < 32 || cols % 32) ? 0 : q8t_bytes(rows, cols); }

int spk_q80_tile(const void *w, int rows, int cols, void *dst, void *stream) {
    return q8t_pack(w, rows, cols, dst, (cudaStream_t)stream);
}

size_t spk_q80_tile_scratch_bytes(void) { return q8t_scratch(); }

int spk_q80_tile_head(const void *wt, int rows, int cols, int ntok, const float *x, int ldx, const float *norm_w,
                      float eps, float *logits, int ldl, int *amax, void *scratch, void *stream) {
    if (!wt || !x || !logits || !scratch || ldx < cols || ldl < rows) return set_error("q8t head: bad arguments");
    const int rc = q8t_head_launch(wt, rows, cols, ntok, x, ldx, norm_w, eps, logits, ldl, amax, scratch,
                                   (cudaStream_t)stream);
    if (rc == 0) return set_error("q8t head: %d x %d x %d tokens is not a tiled geometry", rows, cols, ntok);
    return rc < 0 ? -1 : 0;
}

}  // extern "C"
