// vq_mma.cu — the tensor-core VQ decode-GEMV (see vq_mma.cuh for the fragment map).
//
// Persistent CTA per SM, 32 warps, over a contiguous row range. Row tiles of
// TRR (16 or 8) rows of every stage's index stream arrive by TMA bulk copy into
// a ring of shared-memory slots (mbarrier full/empty pairs). Every warp owns a
// fixed K range of 4S groups of each row (so its B fragments — x as f16 hi/lo —
// are computed once and stay in registers) and, per tile, runs S mma steps per
// stage over the tile's 16 rows. Warp partials are summed in a fixed order, so
// results are deterministic.
#include "common.cuh"
#include "spk.h"
#include "stream.cuh"
#include "vq_mma.cuh"

namespace spk {

namespace {

constexpr int MW = 32;           // warps per CTA
constexpr int MTHREADS = MW * 32;

struct MmaArgs {
    const uint8_t *st[2];
    Layout L;
    const float *x, *norm_w, *aux;
    float eps;
    float *y;
    int accumulate, mode;   // mode 0: y = (acc ? y : 0) + W x;  mode 1: y = gelu_erf(aux) * (W x)
    int trr, nbuf;
    uint32_t main_slot, plane_slot, slot_bytes;
    int *err;
};

__device__ __forceinline__ float h2f_u16(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ float rms_inv_block(const float *x, int n, float eps, double *red) {
    double s = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += (double)x[i] * (double)x[i];
    s = warp_sum_d(s);
    const int w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    if ((threadIdx.x & 31) == 0) red[w] = s;
    __syncthreads();
    double t = 0.0;
    for (int k = 0; k < nw; k++) t += red[k];
    __syncthreads();
    return (float)(1.0 / sqrt(t / (double)n + (double)eps));
}

__device__ __forceinline__ void mma_issue(const MmaArgs &a, int nq, uint8_t *slot, uint64_t *bar, int r0, int nr) {
    const Layout &L = a.L;
    const size_t payload = L.stream_off + (size_t)L.rows * (L.mrow + L.prow);
    BulkList bl;
    bl.n = 0;
    bl.tx = 0;
    for (int q = 0; q < nq; q++) {
        const uintptr_t limit = (uintptr_t)(a.st[q] + payload + 8);
        const uint8_t *m = a.st[q] + L.stream_off + (size_t)r0 * L.mrow;
        bulk_plan(bl, slot + q * a.main_slot, (uintptr_t)m, (uintptr_t)m + (size_t)nr * L.mrow, limit);
        if (L.prow) {
            const uint8_t *p = a.st[q] + L.stream_off + (size_t)L.rows * L.mrow + (size_t)r0 * L.prow;
            bulk_plan(bl, slot + nq * a.main_slot + q * a.plane_slot, (uintptr_t)p, (uintptr_t)p + (size_t)nr * L.prow,
                      limit);
        }
    }
    bulk_issue(bl, bar);
}

template <int NSTG, int S, int EXT>
__global__ void __launch_bounds__(MTHREADS, 1) vq_mma_kernel(const MmaArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    const Layout &L = a.L;
    const int nc = L.nc, TRR = a.trr, NB = a.nbuf;
    uint8_t *cbb = smem;
    uint8_t *ring = smem + (((size_t)NSTG * nc * 8 + 15) & ~(size_t)15);
    uint64_t *full = reinterpret_cast<uint64_t *>(ring + (size_t)NB * a.slot_bytes);
    uint64_t *empty = full + NB;
    float *part = reinterpret_cast<float *>(empty + NB);   // [2][NSTG][MW][16]
    double *red = reinterpret_cast<double *>(part + 2 * NSTG * MW * 16);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int G = gridDim.x;
    const int rb = (int)(((long long)blockIdx.x * L.rows) / G), re = (int)(((long long)(blockIdx.x + 1) * L.rows) / G);
    const int ntile = (re - rb + TRR - 1) / TRR;

    if (tid == 0) {
        for (int b = 0; b < NB; b++) {
            mbar_init(&full[b], 1);
            mbar_init(&empty[b], MW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0)
        for (int k = 0; k < NB - 1 && k < ntile; k++) {
            const int r0 = rb + k * TRR;
            mma_issue(a, NSTG, ring + (size_t)k * a.slot_bytes, &full[k], r0, min(TRR, re - r0));
        }
    for (int q = 0; q < NSTG; q++) {
        const uint2 *src = reinterpret_cast<const uint2 *>(a.st[q] + L.cb_off);
        uint2 *dst = reinterpret_cast<uint2 *>(cbb + (size_t)q * nc * 8);
        for (int v = tid; v < nc; v += MTHREADS) dst[v] = __ldg(src + v);
    }
    float inv = 1.0f;
    if (a.norm_w) inv = rms_inv_block(a.x, L.cols, a.eps, red);
    // B fragments: this warp's K range is groups [warp*4S, (warp+1)*4S); thread t
    // walks [warp*4S + t*S, +S). Column g=0 holds x_hi, g=1 x_lo, others zero.
    const int c0 = warp * 4 * S + t * S;
    uint32_t bx[S], by[S];
#pragma unroll
    for (int s = 0; s < S; s++) {
        bx[s] = 0u;
        by[s] = 0u;
        if (g < 2) {
            const int c = c0 + s;
            float4 v = *reinterpret_cast<const float4 *>(a.x + 4 * c);
            if (a.norm_w) {
                const float4 w = *reinterpret_cast<const float4 *>(a.norm_w + 4 * c);
                v.x = __fmul_rn(__fmul_rn(v.x, inv), w.x);
                v.y = __fmul_rn(__fmul_rn(v.y, inv), w.y);
                v.z = __fmul_rn(__fmul_rn(v.z, inv), w.z);
                v.w = __fmul_rn(__fmul_rn(v.w, inv), w.w);
            }
            uint2 hi, lo;
            split_f16x4(v, hi, lo);
            bx[s] = g == 0 ? hi.x : lo.x;
            by[s] = g == 0 ? hi.y : lo.y;
        }
    }
    __syncthreads();
    const uint32_t bit0 = 12u * (uint32_t)c0, pbit0 = (uint32_t)c0;

    for (int k = 0; k < ntile; k++) {
        const int slot = k % NB;
        if (tid == 0 && k + NB - 1 < ntile) {
            const int kn = k + NB - 1, r0n = rb + kn * TRR, sn = kn % NB;
            if (kn >= NB && !mbar_wait(&empty[sn], (uint32_t)(((kn / NB) - 1) & 1), a.err)) return;
            mma_issue(a, NSTG, ring + (size_t)sn * a.slot_bytes, &full[sn], r0n, min(TRR, re - r0n));
        }
        const int r0 = rb + k * TRR, nr = min(TRR, re - r0);
        if (!mbar_wait(&full[slot], (uint32_t)((k / NB) & 1), a.err)) return;
        const uint8_t *sb = ring + (size_t)slot * a.slot_bytes;
        const bool v0 = g < nr, v1 = g + 8 < nr;
        float d[NSTG][4];
#pragma unroll
        for (int q = 0; q < NSTG; q++) {
            d[q][0] = d[q][1] = d[q][2] = d[q][3] = 0.f;
            const uintptr_t A = (uintptr_t)(a.st[q] + L.stream_off + (size_t)r0 * L.mrow);
            const uint8_t *rowA = sb + q * a.main_slot + (A & 15) + (size_t)g * L.mrow;
            const uint8_t *rowB = rowA + (size_t)8 * L.mrow;
            Run<S> ra, rbn;
            ra.load(rowA, bit0, v0);
            rbn.load(rowB, bit0, v1);
            uint32_t pa = 0, pb = 0;
            if (EXT) {
                const uintptr_t P = (uintptr_t)(a.st[q] + L.stream_off + (size_t)L.rows * L.mrow + (size_t)r0 * L.prow);
                const uint8_t *plA = sb + NSTG * a.main_slot + q * a.plane_slot + (P & 15) + (size_t)g * L.prow;
                const uint32_t *ppA = reinterpret_cast<const uint32_t *>(plA) + (pbit0 >> 5);
                const uint32_t *ppB = reinterpret_cast<const uint32_t *>(plA + (size_t)8 * L.prow) + (pbit0 >> 5);
                if (v0) pa = __funnelshift_r(ppA[0], ppA[1], pbit0 & 31u);
                if (v1) pb = __funnelshift_r(ppB[0], ppB[1], pbit0 & 31u);
            }
            const uint8_t *cq = cbb + (size_t)q * nc * 8;
#pragma unroll
            for (int s = 0; s < S; s++) {
                uint32_t oa = ra.off(s), ob = rbn.off(s);
                if (EXT) {
                    oa |= ((pa >> s) & 1u) << 15;
                    ob |= ((pb >> s) & 1u) << 15;
                }
                uint2 ca = make_uint2(0u, 0u), cbw = make_uint2(0u, 0u);
                if (v0) ca = *reinterpret_cast<const uint2 *>(cq + oa);
                if (v1) cbw = *reinterpret_cast<const uint2 *>(cq + ob);
                mma_16816(d[q], ca.x, cbw.x, ca.y, cbw.y, bx[s], by[s]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        float *pt = part + (size_t)(k & 1) * NSTG * MW * 16;
        if (t == 0) {
#pragma unroll
            for (int q = 0; q < NSTG; q++) {
                pt[(q * MW + warp) * 16 + g] = d[q][0] + d[q][1];
                pt[(q * MW + warp) * 16 + g + 8] = d[q][2] + d[q][3];
            }
        }
        __syncthreads();
        if (tid < nr) {
            const int r = r0 + tid;
            float o = (a.mode == 0 && a.accumulate) ? a.y[r] : 0.0f;
#pragma unroll
            for (int q = 0; q < NSTG; q++) {
                float v = 0.f;
                for (int w = 0; w < MW; w++) v += pt[(q * MW + w) * 16 + tid];
                const float gq = h2f_u16(*reinterpret_cast<const uint16_t *>(a.st[q] + L.gain_off + 2 * (size_t)r));
                o = __fadd_rn(o, __fmul_rn(v, gq));
            }
            if (a.mode == 1) {
                const float gv = a.aux[r];
                const double e = erf((double)gv * 0.70710678118654752440);
                o = __fmul_rn(__fmul_rn(__fmul_rn(0.5f, gv), __fadd_rn(1.0f, (float)e)), o);
            }
            a.y[r] = o;
        }
    }
}

template <int NSTG, int S, int EXT>
int mma_launch_t(const MmaArgs &A, size_t smem, cudaStream_t s) {
    auto k = vq_mma_kernel<NSTG, S, EXT>;
    static size_t opted[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem > opted[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_fail("vq mma kernel shared-memory opt-in", e);
        opted[dev & 63] = smem;
    }
    const int ntr = (A.L.rows + A.trr - 1) / A.trr;
    const int grid = ntr < sm_count() ? ntr : sm_count();
    k<<<grid, MTHREADS, smem, s>>>(A);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail("vq mma kernel launch", e);
}

template <int NSTG, int S>
int mma_launch_e(const MmaArgs &A, size_t smem, cudaStream_t s) {
    return A.L.prow ? mma_launch_t<NSTG, S, 1>(A, smem, s) : mma_launch_t<NSTG, S, 0>(A, smem, s);
}

template <int NSTG>
int mma_launch_s(int S, const MmaArgs &A, size_t smem, cudaStream_t s) {
    switch (S) {
        case 1: return mma_launch_e<NSTG, 1>(A, smem, s);
        case 2: return mma_launch_e<NSTG, 2>(A, smem, s);
        case 4: return mma_launch_e<NSTG, 4>(A, smem, s);
        case 5: return mma_launch_e<NSTG, 5>(A, smem, s);
        case 8: return mma_launch_e<NSTG, 8>(A, smem, s);
    }
    return set_error("vq mma kernel: no instantiation for S=%d", S);
}

}  // namespace

// The tensor-core path for a single matrix of 1-2 stages (dim 4, 12/13-bit DQV3,
// whole 128-index lane runs): 1 = launched, 0 = geometry not taken (the caller
// uses another kernel), -1 = error. mode 1 computes gelu_erf(aux) * (W x).
int vq_mma_gemv(const void *const *stages, int nstg, const Layout &L, const float *x, const float *norm_w, float eps,
                float *y, int accumulate, int mode, const float *aux, cudaStream_t s) {
    if (L.dim != 4 || !L.v3 || L.nbit < 12 || nstg < 1 || nstg > 2) return 0;
    if (L.nidx_row % (4 * MW) || L.mrow % 4 || L.stream_off % 4 || (L.prow && L.prow % 4)) return 0;
    const int S = (int)(L.nidx_row / (4 * MW));
    // S 10 and 20 would hold 20-40 B-fragment registers per lane and spill at 64 registers
    if (!(S == 1 || S == 2 || S == 4 || S == 5 || S == 8)) return 0;
    for (int q = 0; q < nstg; q++)
        if (((uintptr_t)stages[q] & 7) != 0) return 0;
    if (((uintptr_t)x & 15) || (norm_w && ((uintptr_t)norm_w & 15))) return 0;
    const size_t cb = (((size_t)nstg * L.nc * 8 + 15) & ~(size_t)15);
    const size_t fixed = cb + (size_t)2 * nstg * MW * 16 * 4 + 32 * 8;
    for (int trr = 16; trr >= 8; trr /= 2) {
        const uint32_t main_slot = (uint32_t)(((size_t)trr * L.mrow + 32 + 15) & ~(size_t)15);
        const uint32_t plane_slot = L.prow ? (uint32_t)(((size_t)trr * L.prow + 32 + 15) & ~(size_t)15) : 0u;
        const uint32_t slot = nstg * (main_slot + plane_slot);
        for (int nb = 4; nb >= 2; nb--) {
            const size_t smem = fixed + (size_t)nb * slot + 2 * (size_t)nb * 8;
            if (smem > smem_optin_max()) continue;
            MmaArgs A;
            memset(&A, 0, sizeof A);
            for (int q = 0; q < nstg; q++) A.st[q] = (const uint8_t *)stages[q];
            A.L = L;
            A.x = x;
            A.norm_w = norm_w;
            A.aux = aux;
            A.eps = eps;
            A.y = y;
            A.accumulate = accumulate;
            A.mode = mode;
            A.trr = trr;
            A.nbuf = nb;
            A.main_slot = main_slot;
            A.plane_slot = plane_slot;
            A.slot_bytes = slot;
            A.err = device_error_ptr();
            const int rc = nstg == 1 ? mma_launch_s<1>(S, A, smem, s) : mma_launch_s<2>(S, A, smem, s);
            return rc ? -1 : 1;
        }
    }
    return 0;
}

}  // namespace spk
