// vq_mma.cu — the batched (M <= 8) VQ decode-GEMM of the speculative verify
// (see vq_mma.cuh for the fragment map).
//
// Persistent CTA per SM, 16 or 32 warps, over a contiguous row range. Tiles of 16 rows
// of every stage's index stream arrive by TMA bulk copy into a ring of shared-
// memory slots (mbarrier full/empty pairs); the stages' codebooks sit in shared
// memory. A row's K range is cut into `passes` passes of MW warps x 4 threads x
// S groups; per pass every thread builds its B fragments (its token column of X,
// RMSNorm folded in, split hi/lo) from L2-resident X, then runs S MMA steps per
// stage. Warp partials are summed in a fixed order, so results are deterministic.
#include "common.cuh"
#include "spk.h"
#include "stream.cuh"
#include "vq_mma.cuh"

namespace spk {

namespace {

// Warps per CTA, by S: 16 (512 threads, 128 registers a thread) for S = 10, the single
// pass over a 2560-wide row; 32 otherwise, where more warps split a long row into fewer
// passes (a pass rebuilds the B fragments) at 64 registers a thread.
__host__ __device__ constexpr int warps_for(int S) { return S == 10 ? 16 : 32; }
constexpr int MW_MAX = 32;
constexpr int MAXT = 8;          // tokens per batch (the 8 columns of B)
constexpr int TRR_MAX = 16;      // rows per tile: the 16 rows of A, or 8 (rows g+8 empty) for long rows

struct MmaArgs {
    const uint8_t *st[2];
    Layout L;
    const float *x, *norm_w, *aux;
    float eps;
    float *y;
    int ldx, ldy, ntok;
    int accumulate, mode;   // mode 0: y = (acc ? y : 0) + W x;  mode 1: y = gelu_erf(aux) * (W x)
    int nbuf, passes, trr;
    uint32_t main_slot, plane_slot, slot_bytes;
    int *err;
};

__device__ __forceinline__ float h2f_u16(uint16_t h) { return __half2float(__ushort_as_half(h)); }

template <int NQ>
__device__ __forceinline__ void mma_issue(const MmaArgs &a, uint8_t *slot, uint64_t *bar, int r0, int nr) {
    const Layout &L = a.L;
    const size_t payload = L.stream_off + (size_t)L.rows * (L.mrow + L.prow);
    BulkList<2 * NQ> bl;
    bl.tx = 0;
#pragma unroll
    for (int q = 0; q < NQ; q++) {
        const uintptr_t limit = (uintptr_t)(a.st[q] + payload + 8);
        const uint8_t *m = a.st[q] + L.stream_off + (size_t)r0 * L.mrow;
        bulk_plan(bl, 2 * q, slot + q * a.main_slot, (uintptr_t)m, (uintptr_t)m + (size_t)nr * L.mrow, limit);
        const uint8_t *p = a.st[q] + L.stream_off + (size_t)L.rows * L.mrow + (size_t)r0 * L.prow;
        bulk_plan(bl, 2 * q + 1, slot + NQ * a.main_slot + q * a.plane_slot, (uintptr_t)p,
                  (uintptr_t)p + (size_t)nr * L.prow, limit);   // empty without a plane (prow 0)
    }
    bulk_issue(bl, bar);
}

// This thread's B fragments for one pass: column n = g of B is token n (TWO) or,
// packed, token g (hi) for g < 4 and token g - 4 (lo) for g >= 4.
template <int S, int TWO>
__device__ __forceinline__ void load_b(const MmaArgs &a, const float *inv, int g, int cg0, uint32_t (&b0)[S],
                                       uint32_t (&b1)[S], uint32_t (&l0)[S], uint32_t (&l1)[S]) {
    const int tok = TWO ? g : (g & 3);
    const bool lo_col = !TWO && g >= 4;
    const bool live = tok < a.ntok;
#pragma unroll
    for (int s = 0; s < S; s++) {
        b0[s] = b1[s] = l0[s] = l1[s] = 0u;
        if (!live) continue;
        const int c = cg0 + s;
        float4 v = *reinterpret_cast<const float4 *>(a.x + (size_t)tok * a.ldx + 4 * c);
        if (a.norm_w) {
            const float4 w = *reinterpret_cast<const float4 *>(a.norm_w + 4 * c);
            const float iv = inv[tok];
            v.x = __fmul_rn(__fmul_rn(v.x, iv), w.x);
            v.y = __fmul_rn(__fmul_rn(v.y, iv), w.y);
            v.z = __fmul_rn(__fmul_rn(v.z, iv), w.z);
            v.w = __fmul_rn(__fmul_rn(v.w, iv), w.w);
        }
        uint2 hi, lo;
        split_f16x4(v, hi, lo);
        if (TWO) {
            b0[s] = hi.x;
            b1[s] = hi.y;
            l0[s] = lo.x;
            l1[s] = lo.y;
        } else {
            b0[s] = lo_col ? lo.x : hi.x;
            b1[s] = lo_col ? lo.y : hi.y;
        }
    }
}

template <int NSTG, int S, int EXT, int TWO>
__global__ void __launch_bounds__(warps_for(S) * 32, 1) vq_mma_kernel(const MmaArgs a) {
    constexpr int MW = warps_for(S), MTHREADS = MW * 32;
    constexpr int NG = MTHREADS / 128;   // epilogue warp groups: thread e of group k sums WPG warps' element e
    constexpr int WPG = MW / NG;
    extern __shared__ __align__(16) uint8_t smem[];
    const Layout &L = a.L;
    const int nc = L.nc, NB = a.nbuf;
    uint8_t *cbb = smem;
    uint8_t *ring = smem + (((size_t)NSTG * nc * 8 + 15) & ~(size_t)15);
    uint64_t *full = reinterpret_cast<uint64_t *>(ring + (size_t)NB * a.slot_bytes);
    uint64_t *empty = full + NB;
    float *part = reinterpret_cast<float *>(empty + NB);   // [NSTG][MW][16 rows x 8 columns]
    float *red = part + NSTG * MW * 16 * 8;                // [NSTG][NG warp groups][16 x 8]
    float *inv = red + NSTG * NG * 16 * 8;                 // [MAXT]

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int G = gridDim.x;
    const int rb = (int)(((long long)blockIdx.x * L.rows) / G), re = (int)(((long long)(blockIdx.x + 1) * L.rows) / G);
    const int TRR = a.trr;
    const int ntile = (re - rb + TRR - 1) / TRR;

    pdl_trigger();
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
            mma_issue<NSTG>(a, ring + (size_t)k * a.slot_bytes, &full[k], r0, min(TRR, re - r0));
        }
    for (int q = 0; q < NSTG; q++) {
        const uint2 *src = reinterpret_cast<const uint2 *>(a.st[q] + L.cb_off);
        uint2 *dst = reinterpret_cast<uint2 *>(cbb + (size_t)q * nc * 8);
        for (int v = tid; v < nc; v += MTHREADS) dst[v] = __ldg(src + v);
    }
    pdl_wait();   // weights above; X, Y and AUX come from the preceding kernels
    // per-token RMSNorm scale (f64 sum of squares, model.rs:236-245): warp n does token n
    if (warp < MAXT) {
        float iv = 1.0f;
        if (a.norm_w && warp < a.ntok) {
            const float *xr = a.x + (size_t)warp * a.ldx;
            double sq = 0.0;
            for (int i = lane; i < L.cols; i += 32) sq += (double)xr[i] * (double)xr[i];
            sq = warp_sum_d(sq);
            iv = (float)(1.0 / sqrt(sq / (double)L.cols + (double)a.eps));
        }
        if (lane == 0) inv[warp] = iv;
    }
    __syncthreads();

    const int per_pass = MW * 4 * S;   // groups per pass
    uint32_t b0[S], b1[S], l0[S], l1[S];
    if (a.passes == 1) load_b<S, TWO>(a, inv, g, warp * 4 * S + t * S, b0, b1, l0, l1);

    for (int k = 0; k < ntile; k++) {
        const int slot = k % NB;
        // A wait that runs out records the error and skips the work it guarded; no
        // thread leaves the loop, so the CTA barriers below are always complete.
        if (tid == 0 && k + NB - 1 < ntile) {
            const int kn = k + NB - 1, r0n = rb + kn * TRR, sn = kn % NB;
            if (kn < NB || mbar_wait(&empty[sn], (uint32_t)(((kn / NB) - 1) & 1), a.err))
                mma_issue<NSTG>(a, ring + (size_t)sn * a.slot_bytes, &full[sn], r0n, min(TRR, re - r0n));
        }
        const int r0 = rb + k * TRR, nr = min(TRR, re - r0);
        const bool have = mbar_wait(&full[slot], (uint32_t)((k / NB) & 1), a.err);
        const uint8_t *sb = ring + (size_t)slot * a.slot_bytes;
        const bool v0 = have && g < nr, v1 = have && g + 8 < nr;   // nr <= TRR: rows g+8 exist only at 16
        float d[NSTG][4];
#pragma unroll
        for (int q = 0; q < NSTG; q++) d[q][0] = d[q][1] = d[q][2] = d[q][3] = 0.f;
        for (int p = 0; p < a.passes; p++) {
            const int cg0 = p * per_pass + warp * 4 * S + t * S;   // this thread's first group
            if (a.passes > 1) load_b<S, TWO>(a, inv, g, cg0, b0, b1, l0, l1);
            const uint32_t bit0 = 12u * (uint32_t)cg0, pbit0 = (uint32_t)cg0;
#pragma unroll
            for (int q = 0; q < NSTG; q++) {
                const uintptr_t A = (uintptr_t)(a.st[q] + L.stream_off + (size_t)r0 * L.mrow);
                const uint8_t *rowA = sb + q * a.main_slot + (A & 15) + (size_t)g * L.mrow;
                const uint8_t *rowB = rowA + (size_t)8 * L.mrow;
                Run<S> ra, rbn;
                ra.load(rowA, bit0, v0);
                rbn.load(rowB, bit0, v1);
                uint32_t pa = 0, pb = 0;
                if (EXT) {
                    const uintptr_t P =
                        (uintptr_t)(a.st[q] + L.stream_off + (size_t)L.rows * L.mrow + (size_t)r0 * L.prow);
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
                    mma_16816(d[q], ca.x, cbw.x, ca.y, cbw.y, b0[s], b1[s]);
                    if (TWO) mma_16816(d[q], ca.x, cbw.x, ca.y, cbw.y, l0[s], l1[s]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        // the epilogue's per-row operands, fetched after the main loop (not live across it)
        // and before the partials' barrier, which hides their latency
        const int orl = tid >> 3, on_ = tid & 7;   // output (row orl, column on_) for tid < 128
        const bool oown = tid < 128 && orl < nr && (TWO ? on_ : (on_ & 3)) < a.ntok && (TWO || on_ < 4);
        float og[NSTG], oy = 0.f;
        if (oown) {
#pragma unroll
            for (int q = 0; q < NSTG; q++)
                og[q] = h2f_u16(*reinterpret_cast<const uint16_t *>(a.st[q] + L.gain_off + 2 * (size_t)(r0 + orl)));
            if (a.mode == 1) oy = a.aux[(size_t)on_ * a.ldy + r0 + orl];
            else if (a.accumulate) oy = a.y[(size_t)on_ * a.ldy + r0 + orl];
        }
#pragma unroll
        for (int q = 0; q < NSTG; q++) {
            float *pw = part + ((size_t)q * MW + warp) * 16 * 8;
            pw[g * 8 + 2 * t] = d[q][0];
            pw[g * 8 + 2 * t + 1] = d[q][1];
            pw[(g + 8) * 8 + 2 * t] = d[q][2];
            pw[(g + 8) * 8 + 2 * t + 1] = d[q][3];
        }
        __syncthreads();
        // Phase 1, every thread: element e = tid & 127 of the 16 x 8 tile, summed over the
        // WPG warps of group tid >> 7 per stage (a warp reads 32 consecutive floats: no bank
        // conflict). Phase 2, thread e < 128: the 8 groups in order, gains, epilogue.
        {
            const int e = tid & 127, wg = tid >> 7;
#pragma unroll
            for (int q = 0; q < NSTG; q++) {
                const float *pq = part + ((size_t)q * MW + wg * WPG) * 16 * 8 + e;
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < WPG; w++) v += pq[(size_t)w * 16 * 8];
                red[((size_t)q * NG + wg) * 16 * 8 + e] = v;
            }
        }
        __syncthreads();
        if (oown) {
            float o = (a.mode == 0 && a.accumulate) ? oy : 0.0f;
#pragma unroll
            for (int q = 0; q < NSTG; q++) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < NG; w++) {
                    const float *rw = red + ((size_t)q * NG + w) * 16 * 8 + orl * 8;
                    v += TWO ? rw[on_] : (rw[on_] + rw[on_ + 4]);
                }
                o = __fadd_rn(o, __fmul_rn(v, og[q]));
            }
            if (a.mode == 1) {
                const double e = erf((double)oy * 0.70710678118654752440);
                o = __fmul_rn(__fmul_rn(__fmul_rn(0.5f, oy), __fadd_rn(1.0f, (float)e)), o);
            }
            a.y[(size_t)on_ * a.ldy + r0 + orl] = o;
        }
        // no third barrier: the next tile writes the partials only after every warp has
        // passed the barrier above (phase 1 done), and phase 2 reads only `red`, which the
        // next tile rewrites after its own first barrier
    }
}

template <int NSTG, int S, int EXT, int TWO>
int mma_launch_t(const MmaArgs &A, size_t smem, cudaStream_t s) {
    auto k = vq_mma_kernel<NSTG, S, EXT, TWO>;
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
    cudaError_t e = launch_pdl(k, dim3(grid), dim3(warps_for(S) * 32), smem, s, A);
    return e == cudaSuccess ? 0 : cuda_fail("vq mma kernel launch", e);
}

template <int NSTG, int S, int EXT>
int mma_launch_w(const MmaArgs &A, size_t smem, cudaStream_t s) {
    return A.ntok > 4 ? mma_launch_t<NSTG, S, EXT, 1>(A, smem, s) : mma_launch_t<NSTG, S, EXT, 0>(A, smem, s);
}

template <int NSTG, int S>
int mma_launch_e(const MmaArgs &A, size_t smem, cudaStream_t s) {
    return A.L.prow ? mma_launch_w<NSTG, S, 1>(A, smem, s) : mma_launch_w<NSTG, S, 0>(A, smem, s);
}

template <int NSTG>
int mma_launch_s(int S, const MmaArgs &A, size_t smem, cudaStream_t s) {
    switch (S) {
        case 1: return mma_launch_e<NSTG, 1>(A, smem, s);
        case 2: return mma_launch_e<NSTG, 2>(A, smem, s);
        case 4: return mma_launch_e<NSTG, 4>(A, smem, s);
        case 5: return mma_launch_e<NSTG, 5>(A, smem, s);
        case 8: return mma_launch_e<NSTG, 8>(A, smem, s);
        case 10: return mma_launch_e<NSTG, 10>(A, smem, s);
    }
    return set_error("vq mma kernel: no instantiation for S=%d", S);
}

}  // namespace

int vq_mma_batch(const void *const *stages, int nstg, const Layout &L, int ntok, const float *x, int ldx,
                 const float *norm_w, float eps, float *y, int ldy, int accumulate, int mode, const float *aux,
                 cudaStream_t s) {
    if (ntok < 1 || ntok > MAXT) return 0;
    if (L.dim != 4 || !L.v3 || L.nbit < 12 || nstg < 1 || nstg > 2) return 0;
    if (L.nidx_row % (4 * MW_MAX) || L.mrow % 4 || L.stream_off % 4 || (L.prow && L.prow % 4)) return 0;
    // S groups per thread per pass: 10 with 16 warps when that is the whole row in one pass,
    // else the largest of 8, 5, 4, 2, 1 that divides the row's share of 32 warps
    int S = 0;
    if (L.nidx_row == 4 * warps_for(10) * 10) {
        S = 10;
    } else {
        const int per32 = (int)(L.nidx_row / (4 * MW_MAX));
        for (int c : {8, 5, 4, 2, 1})
            if (per32 % c == 0) {
                S = c;
                break;
            }
    }
    const int MW = warps_for(S), NG = MW * 32 / 128;
    const int per = (int)(L.nidx_row / (4 * MW));
    for (int q = 0; q < nstg; q++)
        if (((uintptr_t)stages[q] & 7) != 0) return 0;
    if (((uintptr_t)x & 15) || (ldx & 3) || (norm_w && ((uintptr_t)norm_w & 15))) return 0;
    const size_t cb = (((size_t)nstg * L.nc * 8 + 15) & ~(size_t)15);
    const size_t fixed = cb + (size_t)nstg * MW * 16 * 8 * 4 + (size_t)nstg * NG * 16 * 8 * 4 + MAXT * 4;
    // 16-row tiles, else 8-row tiles (half the A rows empty: the gathers, not the MMAs, bound
    // the kernel) where a 16-row ring does not fit shared memory (long rows: down_proj)
    for (int c = 0; c < 4; c++) {
    const int trr = c < 2 ? TRR_MAX : TRR_MAX / 2, nb = 3 - (c & 1);
    const uint32_t main_slot = (uint32_t)(((size_t)trr * L.mrow + 32 + 15) & ~(size_t)15);
    const uint32_t plane_slot = L.prow ? (uint32_t)(((size_t)trr * L.prow + 32 + 15) & ~(size_t)15) : 0u;
    const uint32_t slot = nstg * (main_slot + plane_slot);
    {
        const size_t smem = ((fixed + 15) & ~(size_t)15) + (size_t)nb * slot + 2 * (size_t)nb * 8;
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
        A.ldx = ldx;
        A.ldy = ldy;
        A.ntok = ntok;
        A.accumulate = accumulate;
        A.mode = mode;
        A.nbuf = nb;
        A.trr = trr;
        A.passes = per / S;
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

using namespace spk;

extern "C" {

/* The verify-batch GEMM (replaces the reference's tiled prefill GEMM for a draft
 * block, gemm_tiled_kernel decode-gpu.cu:359-501, at M = 1 + 7): for every token n
 * of ntok <= 8, y[n*ldy + r] = (accumulate ? y : 0) + (W RMSNorm?(x[n*ldx ..]))[r]
 * with W the sum of the stages. Geometries the tensor-core kernel does not take
 * run token by token on the GEMV path. */
int spk_verify_gemm(const void *const *stages, int nstages, int dim, int nc, int rows, int cols, int v3, int ntok,
                    const float *x, int ldx, const float *norm_w, float eps, float *y, int ldy, int accumulate,
                    void *stream) {
    if (!stages || nstages < 1 || nstages > 4) return set_error("verify gemm needs 1..4 stages");
    if (ntok < 1 || ntok > 8) return set_error("verify gemm takes 1..8 tokens, not %d", ntok);
    if (!x || !y || ldx < cols || ldy < rows) return set_error("verify gemm: bad activation buffers");
    if (v3 && !v3_width_ok(nc)) return set_error("DQV3 carries 13 index bits, nc %d is too wide", nc);
    if (rows <= 0 || cols <= 0 || dim <= 0 || cols % dim) return set_error("verify gemm: bad geometry");
    for (int q = 0; q < nstages; q++)
        if (!stages[q]) return set_error("stage %d payload pointer is null", q);
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    cudaStream_t s = (cudaStream_t)stream;
    if (nstages <= 2) {
        const int rc = vq_mma_batch(stages, nstages, L, ntok, x, ldx, norm_w, eps, y, ldy, accumulate, 0, nullptr, s);
        if (rc != 0) return rc < 0 ? -1 : 0;
    }
    for (int n = 0; n < ntok; n++)
        if (spk_vq_gemv(stages, nstages, 1, dim, nc, rows, cols, v3, x + (size_t)n * ldx, norm_w, eps,
                        y + (size_t)n * ldy, accumulate, stream))
            return -1;
    return 0;
}

}  // extern "C"
