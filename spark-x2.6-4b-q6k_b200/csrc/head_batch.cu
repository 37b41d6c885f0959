// head_batch.cu — the tied Q8_0 head for a verify batch (up to 8 token rows) in
// one pass over the 357 MB table, with each row's greedy id.
//
// logits[n][r] = sum_b d[r][b] * sum_{j<32} q[r][b][j] * xn[n][32b + j],  xn = RMSNorm(x[n]) * w
// (the reference runs the head once per row, vq-model-gpu.cu:957-966). Persistent CTAs
// stream 16-row tiles of blocks by TMA. The int8 weights are exact in f16 and form
// the A fragment of mma.sync m16n8k16 (K permuted so a thread's four k-slots are
// four consecutive weights); the 8 tokens' activations, split into f16 hi + lo
// (~22 bits), are the B columns and stay in registers: warp w owns a fixed range
// of blocks. Each 32-weight block's partial is scaled by its f16 d into the f32
// accumulator. Warp partials are summed in a fixed order; the argmax per token is
// reduced per CTA and then by the last CTA (a ticket the last CTA resets).
#include "common.cuh"
#include "spk.h"
#include "stream.cuh"
#include "vq_mma.cuh"

namespace spk {
namespace {

constexpr int HB_WARPS = 16, HB_THREADS = HB_WARPS * 32, HB_ROWS = 16, HB_MAXT = 8, HB_NBUF = 3;

__device__ __forceinline__ float h2f_u16_hb(uint16_t h) { return __half2float(__ushort_as_half(h)); }

struct HBArgs {
    const uint8_t *w;
    int rows, cols, nblk, bpw;   // blocks per row, blocks per warp
    const float *x;
    int ldx, ntok;
    const float *norm_w;
    float eps;
    float *logits;
    int ldl;
    int *amax;
    unsigned long long *partial;   // [gridDim.x][HB_MAXT]
    unsigned int *counter;
    uint32_t rb_bytes, slot_bytes;
    int *err;
};

__device__ __forceinline__ unsigned long long hb_key(float v, int i) {
    // larger value wins, then the smaller index; NaN never wins, -0 ties +0
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    if (v == 0.0f) u = 0x80000000u;
    if (v != v) u = 0;
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)i);
}

// four int8 weights (2-byte aligned) -> two f16x2 registers, exactly
__device__ __forceinline__ uint2 q4_to_f16(const uint8_t *p) {
    const uint32_t lo = *reinterpret_cast<const uint16_t *>(p), hi = *reinterpret_cast<const uint16_t *>(p + 2);
    const uint32_t w = lo | (hi << 16);
    uint2 r;
    const __half h0 = __int2half_rn((int)(int8_t)(w & 0xFF)), h1 = __int2half_rn((int)(int8_t)((w >> 8) & 0xFF));
    const __half h2 = __int2half_rn((int)(int8_t)((w >> 16) & 0xFF)), h3 = __int2half_rn((int)(int8_t)(w >> 24));
    r.x = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
    r.y = (uint32_t)__half_as_ushort(h2) | ((uint32_t)__half_as_ushort(h3) << 16);
    return r;
}

__device__ __forceinline__ void hb_issue(const HBArgs &a, uint8_t *slot, uint64_t *bar, int r0, int nr) {
    BulkList<1> bl;
    bl.tx = 0;
    const uintptr_t A = (uintptr_t)(a.w + (size_t)r0 * a.rb_bytes);
    bulk_plan(bl, 0, slot, A, A + (size_t)nr * a.rb_bytes, (uintptr_t)(a.w + (size_t)a.rows * a.rb_bytes));
    bulk_issue(bl, bar);
}

template <int BPW>
__global__ void __launch_bounds__(HB_THREADS, 1) head_batch_kernel(const HBArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t *ring = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(ring + (size_t)HB_NBUF * a.slot_bytes);
    uint64_t *empty = full + HB_NBUF;
    float *part = reinterpret_cast<float *>(empty + HB_NBUF);             // [HB_WARPS][16][8]
    float *inv = part + HB_WARPS * HB_ROWS * HB_MAXT;                      // [8]
    unsigned long long *bw = reinterpret_cast<unsigned long long *>(inv + HB_MAXT);   // [16 rows][8]
    __shared__ int is_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int G = gridDim.x;
    const int rb = (int)(((long long)blockIdx.x * a.rows) / G), re = (int)(((long long)(blockIdx.x + 1) * a.rows) / G);
    const int ntile = (re - rb + HB_ROWS - 1) / HB_ROWS;

    pdl_trigger();
    if (tid == 0) {
        for (int b = 0; b < HB_NBUF; b++) {
            mbar_init(&full[b], 1);
            mbar_init(&empty[b], HB_WARPS);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0)
        for (int k = 0; k < HB_NBUF - 1 && k < ntile; k++) {
            const int r0 = rb + k * HB_ROWS;
            hb_issue(a, ring + (size_t)k * a.slot_bytes, &full[k], r0, min(HB_ROWS, re - r0));
        }
    pdl_wait();   // the weight tiles above are immutable; x and the outputs are not
    if (warp < HB_MAXT) {   // per-token RMSNorm scale, f64 sum of squares (model.rs:236-245)
        float iv = 1.0f;
        if (a.norm_w && warp < a.ntok) {
            const float *xr = a.x + (size_t)warp * a.ldx;
            double sq = 0.0;
            for (int i = lane; i < a.cols; i += 32) sq += (double)xr[i] * (double)xr[i];
            sq = warp_sum_d(sq);
            iv = (float)(1.0 / sqrt(sq / (double)a.cols + (double)a.eps));
        }
        if (lane == 0) inv[warp] = iv;
    }
    __syncthreads();
    // B fragments of this warp's blocks: token g, columns 32b + 16j + 4t .. +3, hi and lo
    uint32_t bh[BPW][2][2], bl[BPW][2][2];
    {
        const bool live = g < a.ntok;
#pragma unroll
        for (int b = 0; b < BPW; b++)
#pragma unroll
            for (int j = 0; j < 2; j++) {
                bh[b][j][0] = bh[b][j][1] = bl[b][j][0] = bl[b][j][1] = 0u;
                if (!live) continue;
                const int c = 32 * (warp * BPW + b) + 16 * j + 4 * t;
                float4 v = *reinterpret_cast<const float4 *>(a.x + (size_t)g * a.ldx + c);
                if (a.norm_w) {
                    const float4 w = *reinterpret_cast<const float4 *>(a.norm_w + c);
                    const float iv = inv[g];
                    v.x = __fmul_rn(__fmul_rn(v.x, iv), w.x);
                    v.y = __fmul_rn(__fmul_rn(v.y, iv), w.y);
                    v.z = __fmul_rn(__fmul_rn(v.z, iv), w.z);
                    v.w = __fmul_rn(__fmul_rn(v.w, iv), w.w);
                }
                uint2 hi, lo;
                split_f16x4(v, hi, lo);
                bh[b][j][0] = hi.x;
                bh[b][j][1] = hi.y;
                bl[b][j][0] = lo.x;
                bl[b][j][1] = lo.y;
            }
    }
    // epilogue mapping: thread e < 128 owns tile row e / 8, token e % 8
    const int er = tid >> 3, en = tid & 7;
    unsigned long long best = hb_key(-INFINITY, 0);

    for (int k = 0; k < ntile; k++) {
        const int slot = k % HB_NBUF;
        if (tid == 0 && k + HB_NBUF - 1 < ntile) {
            const int kn = k + HB_NBUF - 1, r0n = rb + kn * HB_ROWS, sn = kn % HB_NBUF;
            if (kn < HB_NBUF || mbar_wait(&empty[sn], (uint32_t)(((kn / HB_NBUF) - 1) & 1), a.err))
                hb_issue(a, ring + (size_t)sn * a.slot_bytes, &full[sn], r0n, min(HB_ROWS, re - r0n));
        }
        const int r0 = rb + k * HB_ROWS, nr = min(HB_ROWS, re - r0);
        const bool have = mbar_wait(&full[slot], (uint32_t)((k / HB_NBUF) & 1), a.err);
        const uint8_t *tile = ring + (size_t)slot * a.slot_bytes + ((uintptr_t)(a.w + (size_t)r0 * a.rb_bytes) & 15);
        const bool v0 = have && g < nr, v1 = have && g + 8 < nr;
        const uint8_t *ra = tile + (size_t)g * a.rb_bytes, *rbp = tile + (size_t)(g + 8) * a.rb_bytes;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int b = 0; b < BPW; b++) {
            const size_t bo = (size_t)(warp * BPW + b) * 34;   // this block's offset in a row
            float d4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const size_t wo = bo + 2 + 16 * j + 4 * t;
                uint2 qa = make_uint2(0u, 0u), qb = make_uint2(0u, 0u);
                if (v0) qa = q4_to_f16(ra + wo);
                if (v1) qb = q4_to_f16(rbp + wo);
                mma_16816(d4, qa.x, qb.x, qa.y, qb.y, bh[b][j][0], bh[b][j][1]);
                mma_16816(d4, qa.x, qb.x, qa.y, qb.y, bl[b][j][0], bl[b][j][1]);
            }
            const float da = v0 ? h2f_u16_hb(*reinterpret_cast<const uint16_t *>(ra + bo)) : 0.f;
            const float db = v1 ? h2f_u16_hb(*reinterpret_cast<const uint16_t *>(rbp + bo)) : 0.f;
            acc[0] = fmaf(da, d4[0], acc[0]);
            acc[1] = fmaf(da, d4[1], acc[1]);
            acc[2] = fmaf(db, d4[2], acc[2]);
            acc[3] = fmaf(db, d4[3], acc[3]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        float *pw = part + (size_t)warp * HB_ROWS * HB_MAXT;
        pw[g * 8 + 2 * t] = acc[0];
        pw[g * 8 + 2 * t + 1] = acc[1];
        pw[(g + 8) * 8 + 2 * t] = acc[2];
        pw[(g + 8) * 8 + 2 * t + 1] = acc[3];
        __syncthreads();
        if (tid < HB_ROWS * HB_MAXT && er < nr && en < a.ntok) {
            float v = 0.f;
            for (int w = 0; w < HB_WARPS; w++) v += part[((size_t)w * HB_ROWS + er) * HB_MAXT + en];
            const int r = r0 + er;
            a.logits[(size_t)en * a.ldl + r] = v;
            const unsigned long long c = hb_key(v, r);
            best = c > best ? c : best;
        }
        __syncthreads();   // the partials are reused by the next tile
    }
    // per token: the CTA's best over its rows, then over CTAs by the last CTA
    if (tid < HB_ROWS * HB_MAXT) bw[tid] = best;
    __syncthreads();
    if (tid < HB_MAXT) {
        unsigned long long m = bw[tid];
        for (int e = 1; e < HB_ROWS; e++) m = bw[e * HB_MAXT + tid] > m ? bw[e * HB_MAXT + tid] : m;
        a.partial[(size_t)blockIdx.x * HB_MAXT + tid] = m;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (is_last && tid < a.ntok) {
        __threadfence();
        unsigned long long m = 0;
        for (int c = 0; c < (int)gridDim.x; c++) {
            const unsigned long long v = __ldcg(a.partial + (size_t)c * HB_MAXT + tid);
            m = v > m ? v : m;
        }
        a.amax[tid] = (int)(0xFFFFFFFFu - (uint32_t)(m & 0xFFFFFFFFull));
    }
    __syncthreads();
    if (is_last && tid == 0) *a.counter = 0u;
}

template <int BPW>
int hb_launch_t(const HBArgs &a, size_t smem, int grid, cudaStream_t s) {
    auto k = head_batch_kernel<BPW>;
    static size_t opted[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem > opted[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_fail("batched head shared-memory opt-in", e);
        opted[dev & 63] = smem;
    }
    cudaError_t e = launch_pdl(k, dim3(grid), dim3(HB_THREADS), smem, s, a);
    return e == cudaSuccess ? 0 : cuda_fail("batched head launch", e);
}

}  // namespace

size_t q80_head_batch_scratch() { return (size_t)1024 * HB_MAXT * sizeof(unsigned long long); }

// 1 launched, 0 geometry not taken (cols not a multiple of 512 up to 2560), -1 error.
int q80_head_batch_launch(const void *w, int rows, int cols, int ntok, const float *x, int ldx, const float *norm_w,
                          float eps, float *logits, int ldl, int *amax, unsigned long long *partial,
                          unsigned int *counter, cudaStream_t s) {
    if (ntok < 1 || ntok > HB_MAXT || cols % 512 || cols > 2560 || rows < 1) return 0;
    if (((uintptr_t)w & 15) || ((uintptr_t)x & 15) || (ldx & 3) || (norm_w && ((uintptr_t)norm_w & 15))) return 0;
    HBArgs a;
    memset(&a, 0, sizeof a);
    a.w = (const uint8_t *)w;
    a.rows = rows;
    a.cols = cols;
    a.nblk = cols / 32;
    a.bpw = a.nblk / HB_WARPS;
    a.x = x;
    a.ldx = ldx;
    a.ntok = ntok;
    a.norm_w = norm_w;
    a.eps = eps;
    a.logits = logits;
    a.ldl = ldl;
    a.amax = amax;
    a.partial = partial;
    a.counter = counter;
    a.rb_bytes = (uint32_t)(a.nblk * 34);
    a.slot_bytes = (uint32_t)(((size_t)HB_ROWS * a.rb_bytes + 32 + 15) & ~(size_t)15);
    a.err = device_error_ptr();
    const size_t smem = (size_t)HB_NBUF * a.slot_bytes + 2 * HB_NBUF * 8 + (size_t)HB_WARPS * HB_ROWS * HB_MAXT * 4 +
                        HB_MAXT * 4 + (size_t)HB_ROWS * HB_MAXT * 8;
    if (smem > smem_optin_max()) return 0;
    const int ntr = (rows + HB_ROWS - 1) / HB_ROWS;
    const int grid = ntr < sm_count() ? ntr : sm_count();
    if (grid > 1024) return set_error("batched head: grid %d above the scratch", grid);
    int rc;
    switch (a.bpw) {
        case 1: rc = hb_launch_t<1>(a, smem, grid, s); break;
        case 2: rc = hb_launch_t<2>(a, smem, grid, s); break;
        case 3: rc = hb_launch_t<3>(a, smem, grid, s); break;
        case 4: rc = hb_launch_t<4>(a, smem, grid, s); break;
        default: rc = hb_launch_t<5>(a, smem, grid, s); break;
    }
    return rc ? -1 : 1;
}

}  // namespace spk

using namespace spk;

extern "C" {

/* The tied Q8_0 head for a verify batch (replaces the reference's per-row head GEMV,
 * vq-model-gpu.cu:957-966): logits[n*ldl + r] = (W RMSNorm(x[n*ldx ..]))[r] for n < ntok <= 8
 * in one pass over W, and amax[n] = first index of row n's maximum (model.rs:594-604).
 * Allocates a small per-device workspace on first use. Geometries the tensor-core kernel
 * does not take (cols not a multiple of 512 up to 2560) run spk_q80_head per row. */
int spk_q80_head_batch(const void *w, int rows, int cols, int ntok, const float *x, int ldx, const float *norm_w,
                       float eps, float *logits, int ldl, int *amax, void *stream) {
    if (!w || !x || !logits || !amax || ntok < 1 || ntok > HB_MAXT || ldx < cols || ldl < rows || cols % 32)
        return set_error("batched head: bad arguments");
    static unsigned long long *part[64];
    static unsigned int *cnt[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return set_error("device %d out of range", dev);
    if (!part[dev]) {
        cudaError_t e = cudaMalloc((void **)&part[dev], q80_head_batch_scratch());
        if (e == cudaSuccess) e = cudaMalloc((void **)&cnt[dev], sizeof(unsigned int));
        if (e == cudaSuccess) e = cudaMemset(cnt[dev], 0, sizeof(unsigned int));
        if (e != cudaSuccess) return cuda_fail("batched head workspace", e);
    }
    cudaStream_t s = (cudaStream_t)stream;
    const int rc = q80_head_batch_launch(w, rows, cols, ntok, x, ldx, norm_w, eps, logits, ldl, amax, part[dev],
                                         cnt[dev], s);
    if (rc != 0) return rc < 0 ? -1 : 0;
    for (int n = 0; n < ntok; n++)
        if (spk_q80_head(w, rows, cols, x + (size_t)n * ldx, norm_w, eps, logits + (size_t)n * ldl, amax + n, stream))
            return -1;
    return 0;
}

}  // extern "C"
