// vq_tc.cu — the VQ decode-GEMM for a batch of token rows on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in tensor memory): the speculative verify batch (M = 1 + 7 tokens)
// and prompt chunks.
//
// What it computes is vq_mma.cu's (forward_batch / verify_logits, vq-model-gpu.cu:858-969, with
// gemm_tiled_kernel's role, decode-gpu.cu:359-501, and every row's GEMV as Stage::dot_row,
// tools/vq-format/src/lib.rs:215-228, summed over stages):
//   Y[n][r] (=|+=) sum_s gain_s[r] * sum_k W_s[r][k] * X[n][k]       (mode 0)
//   Y[n][r] = gelu_erf(AUX[n][r]) * sum_s gain_s[r] * (W_s X[n])[r]   (mode 1)
// for DQV3 stages of dim 4 with 4096 codes (12-bit indices), read from the table kernel's
// re-laid stage words (vq_lut.cu: code words, gains, slice-major 12-byte index records).
//
// The B200 design:
//   * a unit is (row tile of 128 rows, slice of 32 columns); the units, tile-major, are cut
//     evenly over one persistent CTA per SM; a CTA's range is a few segments (one tile's run of
//     slices), each accumulated in tensor memory: D_s [128 lanes][N columns] per stage;
//   * the operands: A_s = the tile's gathered code words (f16, exact) for the slice, 128 x 32,
//     built in shared memory by 8 gather warps in the canonical K-major layout (8-row x 16-byte
//     core matrices); B = the tokens' activations, N = 2 x ntok8 columns (each token as an f16
//     pair hi = rn(x), lo = rn(x - hi): ~22 bits), made once per launch by a small kernel in
//     the same core-matrix layout, one 16-byte-aligned block per slice, brought in by TMA
//     (1-D bulk copies, no multicast) with the index records;
//   * one thread issues tcgen05.mma (kind::f16, M = 128, N, K = 16: two per slice and stage)
//     and tcgen05.commit to release the operand slots; the epilogue warps read D by
//     tcgen05.ld and form g0 (D0[n] + D0[n + ntok8]) + g1 (D1[n] + ...);
//   * a tile covered by more than one CTA: each writes its segment's partial to scratch, and
//     the last to finish (an atomic ticket it resets) sums them in CTA order (the same order on
//     every run) and applies the epilogue; a tile one CTA covers is finished in place.
// Every mbarrier wait is bounded (a lost copy records a device error; the work it guarded is
// skipped, never the loop), and the tensor memory is freed on every path.
#include "common.cuh"
#include "spk.h"

namespace spk {

namespace {

constexpr int TC_M = 128;          // rows per tile (tensor-memory lanes)
constexpr int TC_KB = 32;          // columns per slice (one k-block: two K = 16 MMAs)
constexpr int TC_NAMAX = 3;        // operand slots (A tiles of both stages + B block + records): more measured slower
constexpr int TC_GW = 8;           // gather warps
constexpr int TC_THREADS = (2 + TC_GW) * 32;   // producer, MMA issuer, gather / epilogue warps
constexpr int TC_MAXSEG = 8;       // segments a CTA may walk
constexpr int TC_MAXTOK = 128;     // tokens per launch (N = 256)
constexpr int LUT_CB = 4096 * 8;   // a re-laid stage's fragment-order code words (vq_lut.cu)
constexpr int A_BYTES = TC_M * TC_KB * 2;   // one stage's A tile for a slice (8 KB)

struct TcArgs {
    const uint8_t *lut[2];          // re-laid stage words (vq_lut.cu layout) of the stages
    int ns, rows, rows8, nsl, cols, ntok, ntok8, N;
    size_t cbn_off, gain_off, rec_off;   // byte offsets of the natural-order code words, gains, records
    const uint8_t *xb;              // the tokens' f16 pairs, [nsl][N x 64 bytes] in core-matrix order
    float *y;                       // [ntok][ldy]
    int ldy;
    int mode, accumulate;
    const float *aux;               // mode 1: [ntok][ldy]
    float *scratch;                 // [tiles][TC_MAXSEG... contributors][ntok][128] partials
    unsigned int *tickets;          // [tiles], zero at rest
    int maxc;                       // contributor slots per tile in scratch
    int na;                         // operand slots (as many as shared memory holds, <= TC_NAMAX)
    int *err;
};

__device__ __forceinline__ float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ float gelu_erf(float g) {
    // model.rs:253-258: 0.5*x*(1 + erf(x/sqrt2)), erf in f64
    const double e = erf((double)g * 0.70710678118654752440);
    return __fmul_rn(__fmul_rn(0.5f, g), __fadd_rn(1.0f, (float)e));
}

// Shared-memory matrix descriptor (tcgen05, K-major, no swizzle): start, leading-dimension
// byte offset (between the two 16-byte K chunks of an MMA), stride byte offset (between
// 8-row groups), version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor, kind::f16: f32 accumulate, f16 A and B, both K-major, N, M = 128.
__device__ __forceinline__ uint32_t instr_desc(int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(TC_M >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 8 consecutive f32 columns of this thread's tensor-memory lane (the warp's lane quarter).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}

struct Seg {
    int tile, kb0, kb1, cidx, ncontrib;
};

// The CTA's segments: units (tile, slice) tile-major, range [u0, u1) of U = tiles x nsl.
__device__ int tc_segs(int nsl, int tiles, int G, int c, Seg *sg) {
    const long long U = (long long)tiles * nsl;
    const long long u0 = U * c / G, u1 = U * (c + 1) / G;
    int n = 0;
    for (long long u = u0; u < u1 && n < TC_MAXSEG;) {
        const int t = (int)(u / nsl), k0 = (int)(u - (long long)t * nsl);
        const int k1 = (int)min((long long)nsl, k0 + (u1 - u));
        // contributors of tile t: the CTAs whose ranges meet [t nsl, (t + 1) nsl)
        const long long ta = (long long)t * nsl, tb = ta + nsl;
        const int cfirst = (int)((ta * G) / U);   // first CTA with u1 > ta
        int cf = cfirst;
        while (cf > 0 && U * cf / G > ta) cf--;
        while (U * (cf + 1) / G <= ta) cf++;
        int cl = cf;
        while (cl + 1 < G && U * (cl + 1) / G < tb) cl++;
        sg[n++] = {t, k0, k1, c - cf, cl - cf + 1};
        u += k1 - k0;
    }
    return n;
}

__global__ void __launch_bounds__(TC_THREADS, 1) vq_tc_kernel(const TcArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    // [cb natural, 2 stages x 32 KB][A: na x 2 stages x 8 KB][B: na x N*64][rec: na x 2 x 128 x 12]
    // [gains 2 x 128 f16][barriers][tmem address]
    const int N = a.N, TC_NA = a.na;
    uint8_t *cbn = smem;
    uint8_t *As = cbn + 2 * LUT_CB;
    uint8_t *Bs = As + (size_t)TC_NA * 2 * A_BYTES;
    uint8_t *Rs = Bs + (size_t)TC_NA * N * 64;
    uint16_t *gs = reinterpret_cast<uint16_t *>(Rs + (size_t)TC_NA * 2 * TC_M * 12);
    uint64_t *bars = reinterpret_cast<uint64_t *>(gs + 2 * TC_M);
    uint64_t *in_full = bars, *a_full = bars + TC_NA, *slot_free = bars + 2 * TC_NA;
    uint64_t *cb_full = bars + 3 * TC_NA, *d_full = cb_full + 1, *g_full = cb_full + 2;
    uint32_t *tmem_s = reinterpret_cast<uint32_t *>(bars + 3 * TC_NA + 3);
    Seg *segs = reinterpret_cast<Seg *>(tmem_s + 2);
    __shared__ int nseg_s;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tiles = (a.rows + TC_M - 1) / TC_M;
    const int tcols = 2 * N <= 32 ? 32 : 2 * N <= 64 ? 64 : 2 * N <= 128 ? 128 : 2 * N <= 256 ? 256 : 512;

    if (tid == 0) {
        for (int i = 0; i < TC_NA; i++) {
            mbar_init(in_full + i, 1);
            mbar_init(a_full + i, TC_GW);
            mbar_init(slot_free + i, 1);
        }
        mbar_init(cb_full, 1);
        mbar_init(d_full, 1);
        mbar_init(g_full, 1);
        fence_mbar_init();
        nseg_s = tc_segs(a.nsl, tiles, gridDim.x, blockIdx.x, segs);
    }
    if (warp == 1) {   // this warp owns the tensor memory: 2 stages x N f32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_s)),
                     "r"(tcols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    pdl_trigger();
    const uint32_t tmem = *tmem_s;
    const int nseg = nseg_s;
    const uint32_t idesc = instr_desc(N);

    if (warp == 0) {   // ------------------------------------------------------ producer
        if (lane == 0) {
            // the stages' natural-order code words, once (weights: before the wait)
            mbar_arrive_expect_tx(cb_full, a.ns * LUT_CB);
            for (int s = 0; s < a.ns; s++) bulk_g2s(cbn + s * LUT_CB, a.lut[s] + a.cbn_off, LUT_CB, cb_full);
            pdl_wait();   // the activation blocks are the previous kernel's output
            int k = 0;
            for (int j = 0; j < nseg; j++) {
                const Seg sg = segs[j];
                const int r0 = sg.tile * TC_M, nr = min(TC_M, a.rows8 - r0);
                for (int kb = sg.kb0; kb < sg.kb1; kb++, k++) {
                    const int slot = k % TC_NA;
                    if (k >= TC_NA && !mbar_wait(slot_free + slot, ((k / TC_NA) - 1) & 1, a.err)) break;
                    mbar_arrive_expect_tx(in_full + slot, (uint32_t)(N * 64 + a.ns * nr * 12));
                    bulk_g2s(Bs + (size_t)slot * N * 64, a.xb + (size_t)kb * N * 64, N * 64, in_full + slot);
                    for (int s = 0; s < a.ns; s++)
                        bulk_g2s(Rs + (size_t)(slot * 2 + s) * TC_M * 12,
                                 a.lut[s] + a.rec_off + ((size_t)kb * a.rows8 + r0) * 12, nr * 12, in_full + slot);
                }
            }
        }
    } else if (warp == 1) {   // -------------------------------------------------- MMA issuer
        if (lane == 0) {
            int k = 0;
            const uint32_t lboA = 16 * 128, lboB = (uint32_t)(N / 8) * 128;
            for (int j = 0; j < nseg; j++) {
                const Seg sg = segs[j];
                for (int kb = sg.kb0; kb < sg.kb1; kb++, k++) {
                    const int slot = k % TC_NA;
                    const bool ok = mbar_wait(a_full + slot, (k / TC_NA) & 1, a.err) &&
                                    mbar_wait(in_full + slot, (k / TC_NA) & 1, a.err);
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    if (ok) {
                        const uint32_t bb = smem_u32(Bs + (size_t)slot * N * 64);
                        for (int s = 0; s < a.ns; s++) {
                            const uint32_t ab = smem_u32(As + (size_t)(slot * 2 + s) * A_BYTES);
                            for (int h = 0; h < 2; h++)
                                mma_f16(tmem + (uint32_t)(s * N), smem_desc(ab + h * 2 * lboA, lboA, 128),
                                        smem_desc(bb + h * 2 * lboB, lboB, 128), idesc,
                                        (kb > sg.kb0 || h > 0) ? 1u : 0u);
                        }
                    }
                    mma_commit(slot_free + slot);   // the slot is free once these MMAs have read it
                }
                mma_commit(d_full);   // the segment's accumulators are complete
                // the epilogue reads them before the next segment's first MMA overwrites them
                if (j + 1 < nseg && !mbar_wait(g_full, j & 1, a.err)) break;
            }
        }
    } else {   // --------------------------------------------------- gather / epilogue warps
        const int gw = warp - 2;   // 0 .. TC_GW - 1
        const bool cb_ok = mbar_wait(cb_full, 0, a.err);
        int k = 0;
        for (int j = 0; j < nseg; j++) {
            const Seg sg = segs[j];
            const int r0 = sg.tile * TC_M;
            for (int kb = sg.kb0; kb < sg.kb1; kb++, k++) {
                const int slot = k % TC_NA;
                bool ok = cb_ok && mbar_wait(in_full + slot, (k / TC_NA) & 1, a.err);
                // the slot's A tiles are free again once the MMAs of k - TC_NA completed; the
                // producer waited for that commit before refilling in_full, so in_full implies it
                // item = (stage, row, pair of groups): 2 x 128 x 4 over 256 threads
#pragma unroll
                for (int it = 0; it < 4; it++) {
                    const int e = gw * 32 + lane + it * TC_GW * 32;   // 0 .. 1023
                    const int s = e >> 9, rr = (e >> 2) & 127, pr = e & 3;
                    if (s < a.ns) {
                        uint32_t i0 = 0, i1 = 0;
                        if (ok && r0 + rr < a.rows8) {
                            const uint8_t *rec = Rs + (size_t)(slot * 2 + s) * TC_M * 12 + rr * 12;
                            // indices 2 pr, 2 pr + 1: bits [24 pr, 24 pr + 24) of the record
                            const uint8_t *q = rec + 3 * pr;
                            const uint32_t b = (uint32_t)q[0] | ((uint32_t)q[1] << 8) | ((uint32_t)q[2] << 16);
                            i0 = b & 0xFFFu;
                            i1 = b >> 12;
                        }
                        const uint2 *cb = reinterpret_cast<const uint2 *>(cbn + s * LUT_CB);
                        const uint2 c0 = cb[i0], c1 = cb[i1];
                        // A core matrix: K chunk pr (columns 8 pr .. 8 pr + 7), 8-row group rr / 8
                        uint8_t *dst = As + (size_t)(slot * 2 + s) * A_BYTES + pr * 2048 + (rr >> 3) * 128 + (rr & 7) * 16;
                        *reinterpret_cast<uint4 *>(dst) = make_uint4(c0.x, c0.y, c1.x, c1.y);
                    }
                }
                fence_proxy_async();   // the tensor cores read what these generic stores wrote
                __syncwarp();
                if (lane == 0) mbar_arrive(a_full + slot);
            }
            // ---- epilogue of segment j: warps gw 0..3 read D (tensor-memory lane quarter = warp % 4)
            if (gw < 4) {
                const int q4 = warp & 3;   // this warp's lane quarter
                const int r = r0 + 32 * q4 + lane;
                const bool dok = mbar_wait(d_full, j & 1, a.err);
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                if (j == 0) pdl_wait();   // y and aux are earlier kernels' output
                float g[2] = {0.f, 0.f};
                if (r < a.rows)
                    for (int s = 0; s < a.ns; s++)
                        g[s] = h2f_bits(reinterpret_cast<const uint16_t *>(a.lut[s] + a.gain_off)[r]);
                const bool alone = sg.ncontrib == 1;
                float *part = a.scratch + ((size_t)sg.tile * a.maxc + sg.cidx) * a.ntok * TC_M;
                for (int n0 = 0; n0 < a.ntok; n0 += 8) {
                    float yv[8];
#pragma unroll
                    for (int i = 0; i < 8; i++) yv[i] = 0.f;
                    for (int s = 0; s < a.ns; s++) {
                        float hi[8], lo[8];
                        tmem_ld8(tmem + ((uint32_t)(32 * q4) << 16) + (uint32_t)(s * N + n0), hi);
                        tmem_ld8(tmem + ((uint32_t)(32 * q4) << 16) + (uint32_t)(s * N + a.ntok8 + n0), lo);
#pragma unroll
                        for (int i = 0; i < 8; i++) yv[i] = __fadd_rn(yv[i], __fmul_rn(__fadd_rn(hi[i], lo[i]), g[s]));
                    }
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int n = n0 + i;
                        if (n >= a.ntok || r >= a.rows || !dok) continue;
                        if (alone) {
                            float *yp = a.y + (size_t)n * a.ldy + r;
                            if (a.mode == 1) *yp = __fmul_rn(gelu_erf(a.aux[(size_t)n * a.ldy + r]), yv[i]);
                            else *yp = a.accumulate ? __fadd_rn(*yp, yv[i]) : yv[i];
                        } else {
                            part[(size_t)n * TC_M + 32 * q4 + lane] = yv[i];
                        }
                    }
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                // all four epilogue warps done: the issuer may overwrite D
                asm volatile("bar.sync 2, 128;" ::: "memory");
                if (gw == 0 && lane == 0) mbar_arrive(g_full);
                if (!alone) {   // the last contributor of this tile sums all partials in order
                    __threadfence();
                    asm volatile("bar.sync 2, 128;" ::: "memory");
                    __shared__ int last_s;
                    if (gw == 0 && lane == 0) {
                        const unsigned int t = atomicAdd(a.tickets + sg.tile, 1u);
                        last_s = t == (unsigned)(sg.ncontrib - 1);
                        if (last_s) a.tickets[sg.tile] = 0;   // at rest again for the next launch
                    }
                    asm volatile("bar.sync 2, 128;" ::: "memory");
                    if (last_s) {
                        __threadfence();
                        const float *base = a.scratch + (size_t)sg.tile * a.maxc * a.ntok * TC_M;
                        for (int n = 0; n < a.ntok && r < a.rows; n++) {
                            float v = 0.f;
                            for (int c = 0; c < sg.ncontrib; c++)
                                v = __fadd_rn(v, __ldcg(base + ((size_t)c * a.ntok + n) * TC_M + 32 * q4 + lane));
                            float *yp = a.y + (size_t)n * a.ldy + r;
                            if (a.mode == 1) *yp = __fmul_rn(gelu_erf(a.aux[(size_t)n * a.ldy + r]), v);
                            else *yp = a.accumulate ? __fadd_rn(*yp, v) : v;
                        }
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols) : "memory");
    }
}

// The tokens' activations as f16 pairs in the B core-matrix layout: block kb (32 columns) is
// [chunk (4 x 8 columns)][column group (N / 8)][8 columns n][8 halves], column n < ntok8 = hi of
// token n, n >= ntok8 = lo of token n - ntok8 (zero past ntok). RMSNorm per token (f64 sum of
// squares, model.rs:236-245) when norm_w is given. One CTA per token column pair.
__global__ void vq_tc_xprep_kernel(const float *x, int ldx, const float *norm_w, float eps, int cols, int ntok,
                                   int ntok8, int N, uint8_t *xb) {
    pdl_trigger();
    pdl_wait();
    __shared__ double red[8];
    const int n = blockIdx.x;   // token 0 .. ntok8 - 1
    const float *xr = x + (size_t)n * ldx;
    float inv = 1.0f;
    if (norm_w && n < ntok) {
        double s = 0.0;
        for (int i = threadIdx.x; i < cols; i += blockDim.x) s += (double)xr[i] * (double)xr[i];
        s = warp_sum_d(s);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
        __syncthreads();
        double t = 0.0;
        for (int k = 0; k < (int)(blockDim.x >> 5); k++) t += red[k];
        inv = (float)(1.0 / sqrt(t / (double)cols + (double)eps));
    }
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        float v = 0.f;
        if (n < ntok) {
            v = xr[c];
            if (norm_w) v = __fmul_rn(__fmul_rn(v, inv), norm_w[c]);
        }
        const __half h = __float2half_rn(v), l = __float2half_rn(v - __half2float(h));
        const int kb = c / TC_KB, kk = c % TC_KB, ch = kk >> 3, e = kk & 7;
        __half *blk = reinterpret_cast<__half *>(xb + (size_t)kb * N * 64);
        const int nh = n, nl = ntok8 + n;
        blk[((size_t)ch * (N / 8) + (nh >> 3)) * 64 + (nh & 7) * 8 + e] = h;
        blk[((size_t)ch * (N / 8) + (nl >> 3)) * 64 + (nl & 7) * 8 + e] = l;
    }
}

size_t tc_smem(int N, int na) {
    return (size_t)2 * LUT_CB + (size_t)na * 2 * A_BYTES + (size_t)na * N * 64 + (size_t)na * 2 * TC_M * 12 +
           2 * TC_M * 2 + (3 * TC_NAMAX + 3) * 8 + 8 + TC_MAXSEG * sizeof(Seg) + 64;
}

}  // namespace

// Scratch bytes the batched GEMM needs for a geometry and batch: the activation blocks, the
// contributors' partials and the tile tickets (the tickets, first, must start at zero).
size_t tc_scratch_bytes(int rows, int cols, int ntok) {
    const int ntok8 = (ntok + 7) & ~7, N = 2 * ntok8, nsl = cols / TC_KB, tiles = (rows + TC_M - 1) / TC_M;
    const long long U = (long long)tiles * nsl;
    const int G = (int)(U < sm_count() ? U : sm_count());
    const int maxc = (int)((nsl * (long long)G + U - 1) / U) + 2;
    return 4096 + (size_t)nsl * N * 64 + (size_t)tiles * maxc * ntok * TC_M * 4;
}

// 1 launched, 0 geometry not taken, -1 error. luts: the stages' re-laid words (vq_lut.cu).
int tc_gemm(const void *const *luts, int ns, const Layout &L, int ntok, const float *x, int ldx, const float *norm_w,
            float eps, float *y, int ldy, int accumulate, int mode, const float *aux, void *scratch, cudaStream_t s) {
    if (ntok < 1 || ntok > TC_MAXTOK || ns < 1 || ns > 2) return 0;
    if (!(L.v3 && L.dim == 4 && L.nc == 4096 && L.nbit == 12 && L.prow == 0 && L.cols % TC_KB == 0)) return 0;
    for (int q = 0; q < ns; q++)
        if (!luts[q] || ((uintptr_t)luts[q] & 15)) return 0;
    const int ntok8 = (ntok + 7) & ~7, N = 2 * ntok8, nsl = L.cols / TC_KB, tiles = (L.rows + TC_M - 1) / TC_M;
    // the kernel's static shared memory (2 ints, padded by the compiler) counts against the same limit
    const size_t limit = smem_optin_max() > 2048 ? smem_optin_max() - 2048 : 0;
    int na = TC_NAMAX;
    while (na > 2 && tc_smem(N, na) > limit) na--;
    const size_t smem = tc_smem(N, na);
    if (smem > limit) return 0;
    const long long U = (long long)tiles * nsl;
    const int G = (int)(U < sm_count() ? U : sm_count());   // every CTA has work
    if ((U + G - 1) / G / nsl + 2 > TC_MAXSEG) return 0;
    TcArgs a;
    memset(&a, 0, sizeof a);
    for (int q = 0; q < ns; q++) a.lut[q] = (const uint8_t *)luts[q];
    a.ns = ns;
    a.rows = L.rows;
    a.rows8 = (L.rows + 7) & ~7;
    a.nsl = nsl;
    a.cols = L.cols;
    a.ntok = ntok;
    a.ntok8 = ntok8;
    a.N = N;
    const size_t gain_bytes = ((size_t)a.rows8 * 2 + 15) & ~(size_t)15;
    a.cbn_off = LUT_CB;            // after the fragment-order code words (vq_lut.cu's layout)
    a.gain_off = 2 * (size_t)LUT_CB;
    a.rec_off = a.gain_off + gain_bytes;
    uint8_t *scr = (uint8_t *)scratch;
    a.tickets = (unsigned int *)scr;
    a.xb = scr + 4096;
    a.scratch = (float *)(scr + 4096 + (size_t)nsl * N * 64);
    a.maxc = (int)((nsl * (long long)G + U - 1) / U) + 2;
    a.na = na;
    if (tiles > 1024) return 0;
    a.y = y;
    a.ldy = ldy;
    a.mode = mode;
    a.accumulate = accumulate;
    a.aux = aux;
    a.err = device_error_ptr();
    cudaError_t e = launch_pdl(vq_tc_xprep_kernel, dim3(ntok8), dim3(256), 0, s, x, ldx, norm_w, eps, L.cols, ntok,
                               ntok8, N, (uint8_t *)a.xb);
    if (e != cudaSuccess) return cuda_fail("verify gemm activation launch", e);
    static size_t opted[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem > opted[dev & 63]) {
        e = cudaFuncSetAttribute(vq_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_fail("verify gemm shared-memory opt-in", e);
        opted[dev & 63] = smem;
    }
    e = launch_pdl(vq_tc_kernel, dim3(G), dim3(TC_THREADS), smem, s, a);
    if (e != cudaSuccess) return cuda_fail("verify gemm launch", e);
    return 1;
}

}  // namespace spk

using namespace spk;

extern "C" {

/* Device scratch bytes spk_vq_lut_gemm needs for a geometry and batch size (its first 4 KB
 * are tile tickets that must be zero before the first call; every call leaves them zero). */
size_t spk_vq_lut_gemm_scratch_bytes(int rows, int cols, int ntok) {
    if (rows <= 0 || cols <= 0 || cols % TC_KB || ntok < 1 || ntok > TC_MAXTOK) return 0;
    return tc_scratch_bytes(rows, cols, ntok);
}

/* The VQ GEMM of a token batch on the tensor cores (tcgen05): for n < ntok <= 128,
 *   Y[n] (=|+=) sum_s gain_s W_s RMSNorm?(X[n])
 * from the stages' spk_vq_lut_pack words (DQV3 dim 4, 4096 codes, 12-bit indices, 1-2 stages;
 * replaces forward_batch's per-matrix gemm_tiled_kernel launches, vq-model-gpu.cu:858-943,
 * decode-gpu.cu:359-501). X rows stride ldx floats, Y rows ldy. Two launches, no sync; calls
 * that share a scratch must not overlap on the GPU. */
int spk_vq_lut_gemm(const void *const *luts, int nstages, int dim, int nc, int rows, int cols, int v3, int ntok,
                    const float *x, int ldx, const float *norm_w, float eps, float *y, int ldy, int accumulate,
                    void *scratch, void *stream) {
    if (!luts || !x || !y || !scratch) return set_error("batched vq gemm: null pointer");
    if (ntok < 1 || ntok > TC_MAXTOK) return set_error("batched vq gemm takes 1..%d tokens, not %d", TC_MAXTOK, ntok);
    if (ldx < cols || ldy < rows) return set_error("batched vq gemm: row strides below the matrix");
    if (dim <= 0 || nc <= 0 || rows <= 0 || cols <= 0 || cols % dim) return set_error("batched vq gemm: bad geometry");
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    const int rc = tc_gemm(luts, nstages, L, ntok, x, ldx, norm_w, eps, y, ldy, accumulate, 0, nullptr, scratch,
                           (cudaStream_t)stream);
    if (rc == 0) return set_error("batched vq gemm: geometry not taken (DQV3 dim 4, 4096 codes, 12-bit, 1-2 stages, "
                                  "whole 32-column slices, 16-byte aligned words)");
    return rc < 0 ? -1 : 0;
}

}  // extern "C"
