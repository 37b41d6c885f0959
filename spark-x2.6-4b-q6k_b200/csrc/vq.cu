// vq.cu — residual-VQ (DQV3 / DQVQ) decode kernels for B200, and the vqg_* C-ABI.
//
// What the reference computes (tools/vq-format/src/lib.rs:162-228,
// tools/vq/gpu/decode-gpu.cu:103-301): for every stage s of a container,
//   y[r] += gain_s[r] * sum_i sum_d cb_s[idx_s(r,i)][d] * x[i*dim + d]
// with idx_s read from the stage's packed stream.
//
// The B200 design (fast path, DQV3 dim 4 with a 12-bit main stream):
//   * persistent CTAs, one per SM, each owning a contiguous row range;
//   * every stage's f16 codebook staged once per CTA in shared memory;
//   * the row index streams of a tile of rows pulled by the TMA engine
//     (cp.async.bulk, 1-D, no tensor map, no multicast) into a 3-deep ring of
//     shared-memory slots completed by mbarriers, so HBM reads run ahead of the math;
//   * every lane owns a fixed contiguous run of F indices of the row, so its
//     4F activations live in registers for the whole kernel and only the
//     codebook gathers touch shared memory;
//   * all stages (and, for the FFN, the gate and up matrices) of a row are
//     reduced in one pass, with an optional RMSNorm prologue and either a
//     store / residual-accumulate or an erf-GELU(gate)*up epilogue.
// Every other legal geometry (any dim, DQVQ v2 global streams, narrow or
// unaligned streams) runs a generic warp-per-row kernel with the reference's
// exact index semantics. Dequant kernels are bit-exact: one f32 multiply and
// one f32 add per element, no contraction.
#include "common.cuh"
#include "tp.cuh"
#include "spk.h"
#include "stream.cuh"

using namespace spk;

namespace {

__device__ __forceinline__ float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ float gelu_erf(float g) {
    // model.rs:253-258: 0.5*x*(1 + erf(x/sqrt2)) with erf evaluated in f64.
    const double e = erf((double)g * 0.70710678118654752440);
    return __fmul_rn(__fmul_rn(0.5f, g), __fadd_rn(1.0f, (float)e));
}

// Block-wide RMSNorm scale from each thread's partial sum s of x[i]^2 over i = threadIdx.x,
// threadIdx.x + blockDim.x, ... (in that order), the total in f64 (model.rs:236-245). Every
// CTA sums in the same order, so every CTA gets the same scale.
__device__ float block_rms_inv_from(double s, int n, float eps, double *red) {
    s = warp_sum_d(s);
    const int w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    if ((threadIdx.x & 31) == 0) red[w] = s;
    __syncthreads();
    double t = 0.0;
    for (int k = 0; k < nw; k++) t += red[k];
    __syncthreads();
    return (float)(1.0 / sqrt(t / (double)n + (double)eps));
}

// The same scale over the `nt` threads (whole warps, starting at warp w0) that meet on named
// barrier `id`: each passes its partial sum over its own strided share of x in index order.
__device__ float group_rms_inv_from(double s, int n, float eps, double *red, int id, int nt, int w0) {
    s = warp_sum_d(s);
    const int w = (int)(threadIdx.x >> 5) - w0, nw = nt >> 5;
    if ((threadIdx.x & 31) == 0) red[w] = s;
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nt) : "memory");
    double t = 0.0;
    for (int k = 0; k < nw; k++) t += red[k];
    return (float)(1.0 / sqrt(t / (double)n + (double)eps));
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
    return block_rms_inv_from(s, n, eps, red);
}

// ============================================================ fast path ===
// 16 warps per CTA at every F: a lane's 4F activations live in registers
// (512 threads, up to 128 registers each). 24 warps at F <= 10 measured slower
// on the model's shapes than 16 warps at F 16/20.
template <int F>
struct Warps {
    static constexpr int W = 16;
};
constexpr int FAST_NBUF = 3;
constexpr int CB_PIECES = 8;   // bulk copies per stage codebook
constexpr int X_BATCH = 22;    // activations a staging thread loads in one round trip
constexpr int X_BAR = 15;      // named barrier of the staging warps (row barriers use 1 .. 8)

// Shared-memory bytes of one stage's codebook region: nc 8-byte code words copied from the
// 16-byte boundary at or below the codebook (the payload keeps it 8-byte aligned), so up to 8
// leading and 15 trailing bytes ride along.
__host__ __device__ constexpr size_t cb_region(int nc) { return ((size_t)nc * 8 + 16 + 15) & ~(size_t)15; }
constexpr int MAXQ = 4;   // streams: groups x stages

struct FastArgs {
    const uint8_t *st[MAXQ];   // stage payloads, group-major
    Layout L;
    const float *x;
    const float *norm_w;       // optional RMSNorm weight (nullptr: none)
    float eps;
    float *y;                  // NG 1: y[rows]; NG 2: act[rows]
    int accumulate;            // NG 1: y += result instead of y = result
    int ks;                    // warps per row chunk split
    int tr;                    // rows per tile
    uint32_t main_slot, plane_slot, slot_bytes;
    int nbuf;                  // ring depth (2 or 3, whatever fits shared memory)
    int *err;
    // Optional second matrix of the same encoding and input (NG 1): the last CTA
    // computes all of it (xy = X RMSNorm?(x)) while the others share the main rows.
    int has_x;
    const uint8_t *xst[MAXQ];
    Layout XL;
    float *xy;
    // Tensor parallel (NG 1, no second matrix): the rows are this rank's partial of a residual
    // update; a CTA sends its rows to every rank's mailbox as (value, sequence) pairs instead
    // of writing y, then adds the rank-ordered sum of every rank's rows into h (tp.cuh).
    int tp;
    TpView tpv;
    float *h;
};

template <int F>
struct Chunk {
    // largest bit offset a lane's run can start at inside a 32-bit word
    static constexpr int G = ((12 * F) % 32 == 0) ? 32 : ((12 * F) % 32 % 16 == 0 ? 16 : ((12 * F) % 32 % 8 == 0 ? 8 : 4));
    static constexpr int MAXSH = 32 - G == 0 ? 0 : 32 - G;
    static constexpr int NWR = (MAXSH + 12 * F + 31) / 32;   // words read
    static constexpr int NWU = (12 * F + 31) / 32;           // words used after the shift
};

// One lane's partial dot over its F indices of one row of one stage.
template <int F, int EXT>
__device__ __forceinline__ float row_chunk(const uint8_t *row, const uint8_t *plane, const uint2 *cb,
                                           const float (&xr)[4 * F], uint32_t bit0, uint32_t pbit0) {
    using C = Chunk<F>;
    const uint32_t *wp = reinterpret_cast<const uint32_t *>(row) + (bit0 >> 5);
    const uint32_t sh = bit0 & 31u;
    uint32_t w[C::NWR];
#pragma unroll
    for (int j = 0; j < C::NWR; j++) w[j] = wp[j];
    uint32_t u[C::NWU];
#pragma unroll
    for (int j = 0; j < C::NWU; j++) u[j] = __funnelshift_r(w[j], (j + 1 < C::NWR) ? w[j + 1] : 0u, sh);
    uint32_t pb = 0;
    if (EXT) {
        const uint32_t *pp = reinterpret_cast<const uint32_t *>(plane) + (pbit0 >> 5);
        pb = __funnelshift_r(pp[0], pp[1], pbit0 & 31u);
    }
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int j = 0; j < F; j++) {
        const int b = 12 * j, wi = b >> 5, s = b & 31;
        uint32_t v;
        if (s + 12 <= 32)
            v = (u[wi] >> s) & 0xFFFu;
        else
            v = __funnelshift_r(u[wi], u[wi + 1], s) & 0xFFFu;
        if (EXT) v |= ((pb >> j) & 1u) << 12;
        const uint2 c = cb[v];
        const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&c.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&c.y));
        a0 = fmaf(lo.x, xr[4 * j + 0], a0);
        a1 = fmaf(lo.y, xr[4 * j + 1], a1);
        a0 = fmaf(hi.x, xr[4 * j + 2], a0);
        a1 = fmaf(hi.y, xr[4 * j + 3], a1);
    }
    return a0 + a1;
}

// Producer: thread 0 fills one ring slot with the index streams of rows
// [r0, r0+nr) of every stream (stream.cuh). The contract gives every stage
// payload 8 zeroed slack bytes, so a copy may round up to at most 8 bytes past
// the payload end.
template <int NQ, int EXT>
__device__ __forceinline__ void issue_tile(const FastArgs &a, const uint8_t *const (&stp)[NQ], const Layout &L,
                                           uint8_t *slot, uint64_t *bar, int r0, int nr) {
    const size_t payload = L.stream_off + (size_t)L.rows * (L.mrow + L.prow);
    BulkList<NQ * (1 + EXT)> bl;
    bl.tx = 0;
#pragma unroll
    for (int q = 0; q < NQ; q++) {
        const uintptr_t limit = (uintptr_t)(stp[q] + payload + 8);
#pragma unroll
        for (int part = 0; part < 1 + EXT; part++) {
            const uint8_t *base = stp[q] + L.stream_off +
                                  (part ? (size_t)L.rows * L.mrow + (size_t)r0 * L.prow : (size_t)r0 * L.mrow);
            const size_t bytes = (size_t)nr * (part ? L.prow : L.mrow);
            uint8_t *d = slot + (part ? (NQ * a.main_slot + q * a.plane_slot) : q * a.main_slot);
            bulk_plan(bl, q * (1 + EXT) + part, d, (uintptr_t)base, (uintptr_t)base + bytes, limit);
        }
    }
    bulk_issue(bl, bar);
}

template <int NSTG, int NG, int F, int EXT>
__global__ void __launch_bounds__(Warps<F>::W * 32, 1) vq_fast_kernel(const FastArgs a) {
    constexpr int FAST_WARPS = Warps<F>::W, FAST_THREADS = FAST_WARPS * 32;
    constexpr int NQ = NSTG * NG;
    // padded per-lane stride of the staged activations (floats): an odd number of
    // 16-byte chunks, so 8 lanes' float4 reads hit 8 distinct bank quads
    constexpr int XS = 4 * (F + 1 + (F & 1));
    extern __shared__ __align__(16) uint8_t smem[];
    const bool xt = NG == 1 && a.has_x && blockIdx.x == gridDim.x - 1;   // this CTA runs the second matrix
    const Layout &L = xt ? a.XL : a.L;
    const uint8_t *stp[NQ];   // this CTA's stage payloads, in registers
#pragma unroll
    for (int q = 0; q < NQ; q++) stp[q] = xt ? a.xst[q] : a.st[q];
    float *const yout = xt ? a.xy : a.y;
    const int nc = L.nc;
    const int ks_n = a.ks, tr = a.tr, NB = a.nbuf;
    const size_t CBR = cb_region(nc);
    float *xs = reinterpret_cast<float *>(smem + NQ * CBR);
    uint8_t *ring = reinterpret_cast<uint8_t *>(xs + (size_t)ks_n * 32 * XS);
    uint64_t *full = reinterpret_cast<uint64_t *>(ring + (size_t)NB * a.slot_bytes);
    uint64_t *empty = full + NB;
    uint64_t *cbar = empty + NB;                            // the codebooks' copy
    float *part = reinterpret_cast<float *>(cbar + 2);   // [2][tr][NG][ks][NSTG]
    double *red = reinterpret_cast<double *>(part + 2 * tr * NG * ks_n * NSTG);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // warp -> (row in tile, group, k chunk)
    const int ks = warp % ks_n, g = (warp / ks_n) % NG, rw = warp / (ks_n * NG);
    const bool direct = (NG == 1) && (ks_n == 1);   // the row's warp finishes the row itself

    const int G = gridDim.x - (NG == 1 && a.has_x ? 1 : 0);
    const int rb = xt ? 0 : (int)(((long long)blockIdx.x * L.rows) / G);
    const int re = xt ? L.rows : (int)(((long long)(blockIdx.x + 1) * L.rows) / G);
    const int ntile = (re - rb + tr - 1) / tr;

    pdl_trigger();
    if (tid == 0) {
        for (int b = 0; b < NB; b++) {
            mbar_init(&full[b], 1);
            mbar_init(&empty[b], FAST_WARPS);
        }
        mbar_init(cbar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    // Warp 0: lane 0 issues the first tile; then every lane takes codebook pieces (NQ x nc code
    // words of 8 bytes as CB_PIECES bulk copies per stage), issued side by side rather than one
    // after another; then lane 0 issues the other ring tiles. Every CTA reads the same codebook
    // lines: each starts at its own piece (rotated by CTA), so at any moment the CTAs'
    // requests spread over the L2 slices instead of queueing on the same lines.
    if (warp == 0) {
        if (lane == 0 && ntile > 0) issue_tile<NQ, EXT>(a, stp, L, ring, &full[0], rb, min(tr, re - rb));
        uint32_t tx = 0;
        uintptr_t cba[NQ];
        uint32_t cbn[NQ];
#pragma unroll
        for (int q = 0; q < NQ; q++) {
            const uintptr_t A = (uintptr_t)(stp[q] + L.cb_off);
            cba[q] = A & ~(uintptr_t)15;
            cbn[q] = (uint32_t)((((A + (size_t)nc * 8) + 15) & ~(uintptr_t)15) - cba[q]);
            tx += cbn[q];
        }
        if (lane == 0) mbar_arrive_expect_tx(cbar, tx);   // before any piece can complete
        __syncwarp();
#pragma unroll
        for (int q = 0; q < NQ; q++) {
            const uint32_t piece = ((cbn[q] / CB_PIECES) + 15) & ~15u;   // a multiple of 16 bytes
            for (int k = lane; k < CB_PIECES; k += 32) {
                const uint32_t o = (uint32_t)((k + blockIdx.x) % CB_PIECES) * piece;
                if (o < cbn[q]) bulk_g2s(smem + q * CBR + o, (const void *)(cba[q] + o), min(piece, cbn[q] - o), cbar);
            }
        }
        if (lane == 0) {
            for (int t = 1; t < NB - 1 && t < ntile; t++) {
                const int r0 = rb + t * tr;
                issue_tile<NQ, EXT>(a, stp, L, ring + (size_t)t * a.slot_bytes, &full[t], r0, min(tr, re - r0));
            }
        }
    }
    // Warps 1 .. 15 stage the activations while warp 0 issues the copies above: coalesced loads
    // (one read of x; the optional RMSNorm's sum of squares taken on the way, the scale applied
    // in registers) into a per-lane padded layout, from which each lane later takes its 4F values
    // with 16-byte shared loads that hit distinct banks. Up to X_BATCH values per staging thread
    // are in flight at once (the RMSNorm weights, being weights, before the dependency wait).
    constexpr int XT = FAST_THREADS - 32;   // staging threads
    if (warp > 0) {
        const int xt0 = tid - 32;
        const bool xone = L.cols <= X_BATCH * XT;
        float nwv[X_BATCH];
        if (xone && a.norm_w) {
#pragma unroll
            for (int j = 0; j < X_BATCH; j++) {
                const int c = xt0 + j * XT;
                nwv[j] = c < L.cols ? a.norm_w[c] : 0.f;
            }
        }
        pdl_wait();   // everything above read weights only; x comes from the preceding kernels
        if (xone) {
            float v[X_BATCH];
#pragma unroll
            for (int j = 0; j < X_BATCH; j++) {
                const int c = xt0 + j * XT;
                v[j] = c < L.cols ? a.x[c] : 0.f;
            }
            if (a.norm_w) {   // the staging warps' common branch
                double ss = 0.0;   // this thread's values in index order
#pragma unroll
                for (int j = 0; j < X_BATCH; j++)
                    if (xt0 + j * XT < L.cols) ss += (double)v[j] * (double)v[j];
                const float inv = group_rms_inv_from(ss, L.cols, a.eps, red, X_BAR, XT, 1);
#pragma unroll
                for (int j = 0; j < X_BATCH; j++) v[j] = __fmul_rn(__fmul_rn(v[j], inv), nwv[j]);
            }
#pragma unroll
            for (int j = 0; j < X_BATCH; j++) {
                const int c = xt0 + j * XT;
                const int ln = c / (4 * F);   // global lane index = ks * 32 + lane
                if (c < L.cols) xs[(size_t)ln * XS + (c - ln * 4 * F)] = v[j];
            }
        } else {
            double ss = 0.0;
#pragma unroll 4
            for (int c = xt0; c < L.cols; c += XT) {
                const float v = a.x[c];
                ss += (double)v * (double)v;
                const int ln = c / (4 * F);
                xs[(size_t)ln * XS + (c - ln * 4 * F)] = v;
            }
            if (a.norm_w) {
                const float inv = group_rms_inv_from(ss, L.cols, a.eps, red, X_BAR, XT, 1);
#pragma unroll 4
                for (int c = xt0; c < L.cols; c += XT) {
                    const int ln = c / (4 * F);
                    float &v = xs[(size_t)ln * XS + (c - ln * 4 * F)];
                    v = __fmul_rn(__fmul_rn(v, inv), a.norm_w[c]);
                }
            }
        }
    } else {
        pdl_wait();   // warp 0 reads and writes y (and the exchange counters) after the wait too
    }
    __shared__ unsigned int s_tp_seq;
    __shared__ int s_tp_last;
    if (NG == 1 && a.tp && tid == 0) s_tp_seq = a.tpv.seq[0] + 1u;   // this exchange's number
    __syncthreads();
    // A finished row: y, or under tensor parallelism this rank's pair in every rank's mailbox.
    auto emit = [&](int rr, float o) {
        if (NG == 1 && a.tp) {
            const unsigned int seq = s_tp_seq;
            const size_t prow = (size_t)a.tpv.stride / 2;
            const size_t mine = ((size_t)(seq & 1u) * a.tpv.world + a.tpv.rank) * prow + rr;
            for (int q = 0; q < a.tpv.world; q++)
                tp_st_pair(reinterpret_cast<uint2 *>(a.tpv.mail[q]) + mine, __float_as_uint(o), seq);
        } else {
            yout[rr] = o;
        }
    };
    float xr[4 * F];
    {
        const float4 *xp = reinterpret_cast<const float4 *>(xs + (size_t)(ks * 32 + lane) * XS);
#pragma unroll
        for (int j = 0; j < F; j++) {
            const float4 v = xp[j];
            xr[4 * j] = v.x;
            xr[4 * j + 1] = v.y;
            xr[4 * j + 2] = v.z;
            xr[4 * j + 3] = v.w;
        }
    }
    const int i0 = ks * 32 * F + lane * F;
    const uint32_t bit0 = 12u * (uint32_t)i0, pbit0 = (uint32_t)i0;
    const uint2 *cbq[NQ];   // each stage's code words in shared memory
#pragma unroll
    for (int q = 0; q < NQ; q++)
        cbq[q] = reinterpret_cast<const uint2 *>(smem + q * CBR + ((uintptr_t)(stp[q] + L.cb_off) & 15));
    // this warp's group's stages (selected once: a register array indexed by the warp's group
    // inside the loop would go to local memory)
    const uint8_t *wst[NSTG];
    const uint2 *wcb[NSTG];
#pragma unroll
    for (int s = 0; s < NSTG; s++) {
        wst[s] = (NG == 2 && g) ? stp[NSTG + s] : stp[s];
        wcb[s] = (NG == 2 && g) ? cbq[NSTG + s] : cbq[s];
    }
    const bool cb_in = mbar_wait(cbar, 0u, a.err);   // a lost copy: the error is set, no look-ups

    for (int t = 0; t < ntile; t++) {
        const int slot = t % NB;
        // A wait that runs out records the error and skips the work it guarded, but no
        // thread leaves the loop: every warp still reaches its row's barrier below.
        if (tid == 0 && t + NB - 1 < ntile) {
            const int tn = t + NB - 1, r0n = rb + tn * tr, sn = tn % NB;
            // the slot last held tile tn - NBUF: wait until every warp released it
            if (tn < NB || mbar_wait(&empty[sn], (uint32_t)(((tn / NB) - 1) & 1), a.err))
                issue_tile<NQ, EXT>(a, stp, L, ring + (size_t)sn * a.slot_bytes, &full[sn], r0n, min(tr, re - r0n));
        }
        const int r0 = rb + t * tr, nr = min(tr, re - r0);
        const int r = r0 + rw;
        float gain[NSTG], yold = 0.f;
        if (direct && lane == 0 && rw < nr) {   // issued before the gathers, consumed after
#pragma unroll
            for (int s = 0; s < NSTG; s++)
                gain[s] = h2f_bits(*reinterpret_cast<const uint16_t *>(stp[s] + L.gain_off + 2 * (size_t)r));
            if (a.accumulate) yold = yout[r];
        }
        const bool have = mbar_wait(&full[slot], (uint32_t)((t / NB) & 1), a.err);
        float *pt = part + (size_t)(t & 1) * tr * NG * ks_n * NSTG;
        float acc[NSTG];
#pragma unroll
        for (int s = 0; s < NSTG; s++) acc[s] = 0.f;
        if (rw < nr && have && cb_in) {
            const uint8_t *sb = ring + (size_t)slot * a.slot_bytes;
#pragma unroll
            for (int s = 0; s < NSTG; s++) {
                const int q = g * NSTG + s;
                const uintptr_t A = (uintptr_t)(wst[s] + L.stream_off + (size_t)r0 * L.mrow);
                const uint8_t *row = sb + q * a.main_slot + (A & 15) + (size_t)rw * L.mrow;
                const uint8_t *pl = nullptr;
                if (EXT) {
                    const uintptr_t P = (uintptr_t)(wst[s] + L.stream_off + (size_t)L.rows * L.mrow +
                                                    (size_t)r0 * L.prow);
                    pl = sb + NQ * a.main_slot + q * a.plane_slot + (P & 15) + (size_t)rw * L.prow;
                }
                acc[s] = row_chunk<F, EXT>(row, pl, wcb[s], xr, bit0, pbit0);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);   // this warp is done reading the slot
        if (rw < nr) {
#pragma unroll
            for (int s = 0; s < NSTG; s++) acc[s] = warp_sum(acc[s]);
            if (lane == 0) {
                if (direct) {
                    float o = yold;
#pragma unroll
                    for (int s = 0; s < NSTG; s++) o = __fadd_rn(o, __fmul_rn(acc[s], gain[s]));
                    emit(r, o);
                } else {
#pragma unroll
                    for (int s = 0; s < NSTG; s++) pt[((rw * NG + g) * ks_n + ks) * NSTG + s] = acc[s];
                }
            }
        }
        if (direct) continue;
        // The row's ks_n x NG warps meet on a named barrier (id 1 + rw; tr <= 8 here)
        // and the first of them finishes the row; the other rows' warps run on.
        // pt is double-buffered by tile parity, and a warp can only reach tile t+2
        // after passing tile t+1's barrier, so the reader is done with tile t by then.
        asm volatile("bar.sync %0, %1;" ::"r"(1 + rw), "r"(32 * ks_n * NG) : "memory");
        if (ks == 0 && g == 0 && lane == 0 && rw < nr) {
            const int rr = r0 + rw;
            float outv[NG];
#pragma unroll
            for (int gg = 0; gg < NG; gg++) {
                float o = (NG == 1 && a.accumulate) ? yout[rr] : 0.0f;
#pragma unroll
                for (int s = 0; s < NSTG; s++) {
                    float v = 0.f;
                    for (int k = 0; k < ks_n; k++) v += pt[((rw * NG + gg) * ks_n + k) * NSTG + s];
                    const uint16_t gh =
                        *reinterpret_cast<const uint16_t *>(stp[gg * NSTG + s] + L.gain_off + 2 * (size_t)rr);
                    o = __fadd_rn(o, __fmul_rn(v, h2f_bits(gh)));
                }
                outv[gg] = o;
            }
            if (NG == 1)
                emit(rr, outv[0]);
            else
                yout[rr] = __fmul_rn(gelu_erf(outv[0]), outv[NG - 1]);
        }
    }
    if (NG == 1 && a.tp) {
        // every row of this CTA is sent; add every rank's rows, in rank order, into h
        __syncthreads();
        const unsigned int seq = s_tp_seq;
        tp_reduce_rows(a.tpv, seq, rb, re, a.h);
        // the last CTA to finish advances the exchange counter (every CTA has read it by then)
        __syncthreads();
        if (tid == 0) s_tp_last = atomicAdd(&a.tpv.seq[1], 1u) == gridDim.x - 1;
        __syncthreads();
        if (s_tp_last && tid == 0) {
            a.tpv.seq[1] = 0u;
            a.tpv.seq[0] = seq;
        }
    }
}

// ========================================================= generic path ===
// One warp per row, codebook read through L1. Any dim, DQVQ or DQV3, any width.
struct GenArgs {
    const uint8_t *st[MAXQ];
    int nstg, ng;
    Layout L;
    const float *x;
    const float *norm_w;
    float eps;
    float *y;
    int accumulate;
};

__global__ void vq_generic_kernel(const GenArgs a) {
    __shared__ double red[32];
    const Layout &L = a.L;
    pdl_trigger();
    pdl_wait();
    float inv = 1.0f;
    if (a.norm_w) inv = block_rms_inv(a.x, L.cols, a.eps, red);
    const int warp = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (warp >= L.rows) return;
    const int r = warp;
    float outv[2] = {0.f, 0.f};
    for (int g = 0; g < a.ng; g++) {
        float o = (a.ng == 1 && a.accumulate) ? a.y[r] : 0.0f;
        for (int s = 0; s < a.nstg; s++) {
            const uint8_t *p = a.st[g * a.nstg + s];
            const __half *cb = reinterpret_cast<const __half *>(p + L.cb_off);
            const uint8_t *st = p + L.stream_off;
            float acc = 0.f;
            for (size_t i = lane; i < L.nidx_row; i += 32) {
                const uint32_t v = min(rd_idx(st, L, (size_t)r, i), (uint32_t)L.nc - 1u);   // malformed stream: stay in the codebook
                const __half *c = cb + (size_t)v * L.dim;
                for (int d = 0; d < L.dim; d++) {
                    const size_t col = i * (size_t)L.dim + (size_t)d;
                    float xv = a.x[col];
                    if (a.norm_w) xv = __fmul_rn(__fmul_rn(xv, inv), a.norm_w[col]);
                    acc = fmaf(__half2float(c[d]), xv, acc);
                }
            }
            acc = warp_sum(acc);
            const uint16_t gh = *reinterpret_cast<const uint16_t *>(p + L.gain_off + 2 * (size_t)r);
            o = __fadd_rn(o, __fmul_rn(acc, h2f_bits(gh)));
        }
        outv[g] = o;
    }
    if (lane == 0) a.y[r] = a.ng == 1 ? outv[0] : __fmul_rn(gelu_erf(outv[0]), outv[1]);
}

// lib.rs:197-212 / decode-gpu.cu:124-150: out[r][i*dim+d] += cb[v][d] * gain[r],
// one rounded multiply and one rounded add, bit-exact with the CPU decode.
__global__ void vq_dequant_kernel(const uint8_t *p, const Layout L, float *out, int *err) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= L.nidx) return;
    const size_t r = i / L.nidx_row, k = i - r * L.nidx_row;
    const uint32_t v = rd_idx(p + L.stream_off, L, r, k);
    if (v >= (uint32_t)L.nc) {
        atomicExch(err, DEV_BAD_INDEX);
        return;
    }
    const float g = h2f_bits(*reinterpret_cast<const uint16_t *>(p + L.gain_off + 2 * r));
    const __half *c = reinterpret_cast<const __half *>(p + L.cb_off) + (size_t)v * L.dim;
    float *o = out + i * (size_t)L.dim;
    for (int d = 0; d < L.dim; d++) o[d] = __fadd_rn(o[d], __fmul_rn(__half2float(c[d]), g));
}

// decode-gpu.cu:934-945: one row of one stage accumulated into out (the
// embedding row of a VQ embedding matrix).
__global__ void vq_row_dequant_kernel(const uint8_t *p, const Layout L, int row, float *out) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= L.nidx_row) return;
    const uint32_t v = min(rd_idx(p + L.stream_off, L, (size_t)row, i), (uint32_t)L.nc - 1u);
    const float g = h2f_bits(*reinterpret_cast<const uint16_t *>(p + L.gain_off + 2 * (size_t)row));
    const __half *c = reinterpret_cast<const __half *>(p + L.cb_off) + (size_t)v * L.dim;
    float *o = out + i * (size_t)L.dim;
    for (int d = 0; d < L.dim; d++) o[d] = __fadd_rn(o[d], __fmul_rn(__half2float(c[d]), g));
}

// Plain f32 GEMV, the "already expanded" bandwidth baseline (decode-gpu.cu:662-677).
__global__ void gemv_f32_kernel(const float *w, const float *x, float *y, int rows, int cols) {
    const int warp = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float *wr = w + (size_t)warp * cols;
    float acc = 0.f;
    if ((cols & 3) == 0 && ((uintptr_t)wr & 15) == 0 && ((uintptr_t)x & 15) == 0) {
        const float4 *w4 = reinterpret_cast<const float4 *>(wr), *x4 = reinterpret_cast<const float4 *>(x);
        for (int c = lane; c < cols / 4; c += 32) {
            const float4 a = __ldg(w4 + c), b = x4[c];
            acc = fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, fmaf(a.w, b.w, acc))));
        }
    } else {
        for (int c = lane; c < cols; c += 32) acc = fmaf(wr[c], x[c], acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) y[warp] += acc;
}

// ----------------------------------------------------------- dispatch ---
// Preconditions of the fast path (same contract as v3_blk_ok, decode-gpu.cu:62-64,
// plus dim 4 and this kernel's lane split): a DQV3 payload with a 12-bit main
// stream, whole 32-index groups, word-aligned row streams, an 8-byte aligned
// codebook.
bool blk_ok(const Layout &L) {
    return L.v3 && L.nbit >= 12 && L.nidx_row % 32 == 0 && L.mrow % 4 == 0 && L.stream_off % 4 == 0;
}

int pick_split(const Layout &L, int *F) {
    // smallest k (warps per row) giving F = nidx_row/(32k) of 20 or 16 (fewest
    // warps per row, least partial-sum traffic); else the smallest k giving one
    // of the other instantiated F
    for (int pass = 0; pass < 2; pass++)
        for (int k = 1; k <= 16; k *= 2) {
            if (L.nidx_row % (32 * (size_t)k)) continue;
            const int f = (int)(L.nidx_row / (32 * (size_t)k));
            if ((pass == 0 && (f == 20 || f == 16)) || (pass == 1 && (f == 10 || f == 8 || f == 5 || f == 4))) {
                *F = f;
                return k;
            }
        }
    return 0;
}

struct FastPlan {
    int ks, F, tr;
    size_t smem;
    FastArgs args;
};

bool fast_plan(const uint8_t *const *st, int nstg, int ng, const Layout &L, FastPlan *P) {
    if (L.dim != 4 || !blk_ok(L) || nstg < 1 || nstg > 2 || ng < 1 || ng > 2) return false;
    for (int q = 0; q < nstg * ng; q++)
        if (((uintptr_t)st[q] & 7) != 0) return false;
    int F = 0;
    const int ks = pick_split(L, &F);
    const int W = Warps<20>::W;
    if (!ks || ks * ng > W || W % (ks * ng)) return false;
    const int tr = W / (ks * ng);
    const int nq = nstg * ng, ext = L.prow ? 1 : 0;
    const uint32_t main_slot = (uint32_t)(((size_t)tr * L.mrow + 32 + 15) & ~(size_t)15);
    const uint32_t plane_slot = ext ? (uint32_t)(((size_t)tr * L.prow + 32 + 15) & ~(size_t)15) : 0u;
    const uint32_t slot = nq * (main_slot + plane_slot);
    int nbuf = FAST_NBUF;
    size_t smem = 0;
    for (; nbuf >= 2; nbuf--) {
        smem = (size_t)nq * cb_region(L.nc) + (size_t)ks * 32 * (4 * (F + 1 + (F & 1))) * 4 + (size_t)nbuf * slot +
               (2 * (size_t)nbuf + 2) * 8 + (size_t)2 * tr * ng * ks * nstg * 4 + 32 * 8;
        if (smem <= smem_optin_max()) break;
    }
    if (nbuf < 2) return false;
    FastArgs &a = P->args;
    memset(&a, 0, sizeof a);
    for (int q = 0; q < nq; q++) a.st[q] = st[q];
    a.L = L;
    a.ks = ks;
    a.tr = tr;
    a.main_slot = main_slot;
    a.plane_slot = plane_slot;
    a.slot_bytes = slot;
    a.nbuf = nbuf;
    P->ks = ks;
    P->F = F;
    P->tr = tr;
    P->smem = smem;
    return true;
}

template <int NSTG, int NG, int F, int EXT>
int launch_fast_t(const FastPlan &P, cudaStream_t s) {
    auto k = vq_fast_kernel<NSTG, NG, F, EXT>;
    static size_t opted[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (P.smem > opted[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P.smem);
        if (e != cudaSuccess) return cuda_fail("vq fast kernel shared-memory opt-in", e);
        opted[dev & 63] = P.smem;
    }
    const int ntr = (P.args.L.rows + P.tr - 1) / P.tr;
    const int cap = sm_count() - (P.args.has_x ? 1 : 0);
    const int grid = (ntr < cap ? ntr : cap) + (P.args.has_x ? 1 : 0);
    cudaError_t e = launch_pdl(k, dim3(grid), dim3(Warps<F>::W * 32), P.smem, s, P.args);
    return e == cudaSuccess ? 0 : cuda_fail("vq fast kernel launch", e);
}

template <int NSTG, int NG, int F>
int launch_fast_e(const FastPlan &P, cudaStream_t s) {
    return P.args.L.prow ? launch_fast_t<NSTG, NG, F, 1>(P, s) : launch_fast_t<NSTG, NG, F, 0>(P, s);
}

template <int NSTG, int NG>
int launch_fast_f(const FastPlan &P, cudaStream_t s) {
    switch (P.F) {
        case 20: return launch_fast_e<NSTG, NG, 20>(P, s);
        case 16: return launch_fast_e<NSTG, NG, 16>(P, s);
        case 10: return launch_fast_e<NSTG, NG, 10>(P, s);
        case 8: return launch_fast_e<NSTG, NG, 8>(P, s);
        case 5: return launch_fast_e<NSTG, NG, 5>(P, s);
        case 4: return launch_fast_e<NSTG, NG, 4>(P, s);
    }
    return set_error("vq fast kernel: no instantiation for F=%d", P.F);
}

int launch_fast(const FastPlan &P, int nstg, int ng, cudaStream_t s) {
    if (nstg == 1 && ng == 1) return launch_fast_f<1, 1>(P, s);
    if (nstg == 2 && ng == 1) return launch_fast_f<2, 1>(P, s);
    if (nstg == 1 && ng == 2) return launch_fast_f<1, 2>(P, s);
    if (nstg == 2 && ng == 2) return launch_fast_f<2, 2>(P, s);
    return set_error("vq fast kernel: %d stages x %d groups not instantiated", nstg, ng);
}

int launch_generic(const uint8_t *const *st, int nstg, int ng, const Layout &L, const float *x,
                   const float *norm_w, float eps, float *y, int accumulate, int threads, cudaStream_t s) {
    GenArgs a;
    memset(&a, 0, sizeof a);
    for (int q = 0; q < nstg * ng; q++) a.st[q] = st[q];
    a.nstg = nstg;
    a.ng = ng;
    a.L = L;
    a.x = x;
    a.norm_w = norm_w;
    a.eps = eps;
    a.y = y;
    a.accumulate = accumulate;
    const int blocks = (int)(((size_t)L.rows * 32 + threads - 1) / threads);
    cudaError_t e = launch_pdl(vq_generic_kernel, dim3(blocks), dim3(threads), 0, s, a);
    return e == cudaSuccess ? 0 : cuda_fail("vq generic kernel launch", e);
}

int check_geometry(int dim, int nc, int rows, int cols, int v3) {
    if (v3 && !v3_width_ok(nc)) {
        int b = 1;
        while ((1 << b) < nc) b++;
        return set_error("DQV3 carries 13 index bits, nc %d needs %d", nc, b);
    }
    if (rows <= 0 || cols <= 0) return set_error("gemv needs a non-empty matrix");
    if (dim <= 0 || nc <= 0 || cols % dim) return set_error("geometry dim %d nc %d cols %d is inconsistent", dim, nc, cols);
    if (nc > 65535) return set_error("nc %d does not fit the u16 header field", nc);
    return 0;
}

// Multi-stage, optionally paired (gate/up) GEMV on a stream.
int vq_gemv_impl(const void *const *stages, int nstg, int ng, const Layout &L, const float *x,
                 const float *norm_w, float eps, float *y, int accumulate, int variant, int threads,
                 cudaStream_t s) {
    const uint8_t *st[MAXQ];
    if (nstg < 1 || ng < 1 || nstg * ng > MAXQ) return set_error("%d stages x %d groups exceeds %d streams", nstg, ng, MAXQ);
    for (int q = 0; q < nstg * ng; q++) {
        if (!stages[q]) return set_error("stage %d payload pointer is null", q);
        st[q] = (const uint8_t *)stages[q];
    }
    if (!x || !y) return set_error("gemv needs x and y");
    FastPlan P;
    if ((variant == 0 || variant == 3) && fast_plan(st, nstg, ng, L, &P)) {
        P.args.x = x;
        P.args.norm_w = norm_w;
        P.args.eps = eps;
        P.args.y = y;
        P.args.accumulate = accumulate;
        P.args.err = device_error_ptr();
        return launch_fast(P, nstg, ng, s);
    }
    if (variant == 3) return set_error("the DQV3 block kernel does not take this geometry");
    return launch_generic(st, nstg, ng, L, x, norm_w, eps, y, accumulate, threads, s);
}

}  // namespace

// y = W RMSNorm?(x) and xy = X RMSNorm?(x) for two matrices of one encoding and
// input width (QKV and g_proj) in one launch, the last CTA taking all of X.
// Returns 0 launched, 1 not taken (the fast kernel does not take the pair), -1 error.
int spk::vq_gemv_with_extra(const void *const *stages, int nstg, const Layout &L, const void *const *xstages,
                       const Layout &XL, const float *x, const float *norm_w, float eps, float *y, float *xy,
                       int accumulate, cudaStream_t s) {
    const uint8_t *st[MAXQ], *xst[MAXQ];
    if (nstg < 1 || nstg > 2) return set_error("%d stages: the paired launch takes 1 or 2", nstg);
    for (int q = 0; q < nstg; q++) {
        if (!stages[q] || !xstages[q]) return set_error("stage %d payload pointer is null", q);
        st[q] = (const uint8_t *)stages[q];
        xst[q] = (const uint8_t *)xstages[q];
    }
    if (check_geometry(L.dim, L.nc, L.rows, L.cols, L.v3) || check_geometry(XL.dim, XL.nc, XL.rows, XL.cols, XL.v3))
        return -1;
    FastPlan P, PX;
    const bool same = XL.dim == L.dim && XL.nc == L.nc && XL.cols == L.cols && XL.v3 == L.v3 && XL.rows <= 64;
    if (same && fast_plan(st, nstg, 1, L, &P) && fast_plan(xst, nstg, 1, XL, &PX) && PX.F == P.F && PX.tr == P.tr) {
        P.args.x = x;
        P.args.norm_w = norm_w;
        P.args.eps = eps;
        P.args.y = y;
        P.args.accumulate = accumulate;
        P.args.err = device_error_ptr();
        P.args.has_x = 1;
        for (int q = 0; q < nstg; q++) P.args.xst[q] = xst[q];
        P.args.XL = XL;
        P.args.xy = xy;
        return launch_fast(P, nstg, 1, s);
    }
    return 1;
}

int spk::vq_gemv_tp(const void *const *stages, int nstg, const Layout &L, const float *x, float *h, const TpView &v,
                    cudaStream_t s) {
    const uint8_t *st[MAXQ];
    if (nstg < 1 || nstg > 2) return 1;
    for (int q = 0; q < nstg; q++) {
        if (!stages[q]) return set_error("stage %d payload pointer is null", q);
        st[q] = (const uint8_t *)stages[q];
    }
    if (!x || !h) return set_error("gemv needs x and h");
    if (check_geometry(L.dim, L.nc, L.rows, L.cols, L.v3)) return -1;
    FastPlan P;
    if (!fast_plan(st, nstg, 1, L, &P)) return 1;
    if ((size_t)v.stride < 2 * (size_t)L.rows) return set_error("tensor-parallel mailbox rows hold %d floats, %d needed", v.stride, 2 * L.rows);
    P.args.x = x;
    P.args.y = h;   // not written: the rows travel as pairs
    P.args.accumulate = 0;
    P.args.err = device_error_ptr();
    P.args.tp = 1;
    P.args.tpv = v;
    P.args.h = h;
    return launch_fast(P, nstg, 1, s) ? -1 : 0;
}

namespace {

int timed(int iters, double *ms, int (*fn)(void *), void *ctx) {
    cudaEvent_t a, b;
    if (cudaEventCreate(&a) != cudaSuccess || cudaEventCreate(&b) != cudaSuccess)
        return cuda_fail("event create", cudaGetLastError());
    float best = 1e30f;
    int rc = 0;
    for (int it = 0; it < iters && !rc; it++) {
        cudaEventRecord(a);
        rc = fn(ctx);
        cudaEventRecord(b);
        cudaError_t e = cudaEventSynchronize(b);
        if (!rc && e != cudaSuccess) rc = cuda_fail("timed launch", e);
        float t = 0;
        cudaEventElapsedTime(&t, a, b);
        if (t < best) best = t;
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    if (!rc) rc = check_device_error("timed launch");
    if (ms) *ms = iters > 0 ? best : 0.0;
    return rc;
}

}  // namespace

// =================================================================== ABI ===
extern "C" {

/* decode-gpu.cu:789-798. Legality is the reference's, variant by variant; the
 * variants are accepted aliases of this build's kernels. */
int vqg_gemv_ready(int dim, int nc, int rows, int cols, int v3, int variant) {
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    switch (variant) {
        case 3: return blk_ok(L) ? 1 : 0;
        case 2: return L.dim == 4;
        case 1: return 1;
        case 0: return (size_t)L.nc * L.dim * 2 <= smem_optin_max();
        default: return 0;
    }
}

struct GemvCtx {
    const void *p;
    Layout L;
    const float *x;
    float *y;
    int variant, threads;
};

static int gemv_once(void *c) {
    GemvCtx *g = (GemvCtx *)c;
    const void *st[1] = {g->p};
    return vq_gemv_impl(st, 1, 1, g->L, g->x, nullptr, 0.f, g->y, 1, g->variant == 0 ? 0 : g->variant, g->threads,
                        0);
}

/* decode-gpu.cu:864-901: timed fused GEMV of one stage, y += W_s x (device pointers). */
int vqg_gemv_t(const void *payload, int dim, int nc, int rows, int cols, int v3, const float *x, float *y,
               int variant, int threads, int iters, double *ms) {
    if (check_geometry(dim, nc, rows, cols, v3)) return -1;
    if (variant < 0 || variant > 3) return set_error("unknown gemv variant %d", variant);
    if (variant != 0 && (threads < 32 || threads > 1024 || threads % 32))
        return set_error("gemv launch width %d is not a warp multiple up to 1024", threads);
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    if (variant == 3 && !blk_ok(L)) return set_error("the DQV3 block kernel does not take this geometry");
    GemvCtx c = {payload, L, x, y, variant, variant == 0 ? 256 : threads};
    return timed(iters, ms, gemv_once, &c);
}

/* decode-gpu.cu:903-906 */
int vqg_gemv(const void *payload, int dim, int nc, int rows, int cols, int v3, const float *x, float *y, int variant,
             int iters, double *ms) {
    return vqg_gemv_t(payload, dim, nc, rows, cols, v3, x, y, variant, 256, iters, ms);
}

/* decode-gpu.cu:911-916: one launch, no timing, no synchronization. */
int vqg_gemv_launch_t(const void *payload, int dim, int nc, int rows, int cols, int v3, const float *x, float *y,
                      int variant, int threads) {
    if (check_geometry(dim, nc, rows, cols, v3)) return -1;
    if (threads < 32 || threads > 1024 || threads % 32)
        return set_error("gemv launch width %d is not a warp multiple up to 1024", threads);
    if (variant < 0 || variant > 3) return set_error("unknown gemv variant %d", variant);
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    const void *st[1] = {payload};
    return vq_gemv_impl(st, 1, 1, L, x, nullptr, 0.f, y, 1, variant, threads, 0);
}

/* decode-gpu.cu:918-922 */
int vqg_gemv_launch(const void *payload, int dim, int nc, int rows, int cols, int v3, const float *x, float *y,
                    int variant) {
    return vqg_gemv_launch_t(payload, dim, nc, rows, cols, v3, x, y, variant, 256);
}

struct DqCtx {
    const void *p;
    Layout L;
    float *out;
};

static int dequant_once(void *c) {
    DqCtx *d = (DqCtx *)c;
    const int threads = 256;
    const int blocks = (int)((d->L.nidx + threads - 1) / threads);
    vq_dequant_kernel<<<blocks, threads>>>((const uint8_t *)d->p, d->L, d->out, device_error_ptr());
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail("dequant launch", e);
}

/* decode-gpu.cu:834-858: out += decoded stage (bit-exact), optionally timed. */
int vqg_dequant(const void *payload, int dim, int nc, int rows, int cols, int v3, float *out, int iters, double *ms) {
    if (check_geometry(dim, nc, rows, cols, v3)) return -1;
    DqCtx c = {payload, make_layout(dim, nc, rows, cols, v3), out};
    return timed(iters, ms, dequant_once, &c);
}

/* decode-gpu.cu:947-956 */
int vqg_row_dequant(const void *payload, int dim, int nc, int rows, int cols, int v3, int row, float *out) {
    if (check_geometry(dim, nc, rows, cols, v3)) return -1;
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    if (row < 0 || row >= L.rows) return set_error("row %d is outside %d", row, L.rows);
    const int threads = 256;
    const int blocks = (int)((L.nidx_row + threads - 1) / threads);
    vq_row_dequant_kernel<<<blocks, threads>>>((const uint8_t *)payload, L, row, out);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail("row dequant launch", e);
}

struct F32Ctx {
    const float *w, *x;
    float *y;
    int rows, cols;
};

static int f32_once(void *c) {
    F32Ctx *f = (F32Ctx *)c;
    const int threads = 256;
    gemv_f32_kernel<<<(f->rows * 32 + threads - 1) / threads, threads>>>(f->w, f->x, f->y, f->rows, f->cols);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail("gemv f32 launch", e);
}

/* decode-gpu.cu:1120-1138: y += W x for an expanded f32 matrix, timed. */
int vqg_gemv_f32(const float *w, const float *x, float *y, int rows, int cols, int iters, double *ms) {
    if (rows <= 0 || cols <= 0) return set_error("gemv f32 needs a non-empty matrix");
    F32Ctx c = {w, x, y, rows, cols};
    return timed(iters, ms, f32_once, &c);
}

/* New: all stages of a container (and optionally a second, paired container)
 * in one pass, on a caller stream.
 *   ng 1: y = (accumulate ? y : 0) + sum_s gain_s * W_s x
 *   ng 2: y = gelu_erf(W_gate x) * (W_up x); stages = {gate_0..gate_n, up_0..up_n}
 * norm_w (optional) folds RMSNorm(x) with eps into the load of x. */
int spk_vq_gemv(const void *const *stages, int nstages, int ngroups, int dim, int nc, int rows, int cols, int v3,
                const float *x, const float *norm_w, float eps, float *y, int accumulate, void *stream) {
    if (check_geometry(dim, nc, rows, cols, v3)) return -1;
    if (ngroups == 2 && accumulate) return set_error("the paired gate/up form writes its output, it cannot accumulate");
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    return vq_gemv_impl(stages, nstages, ngroups, L, x, norm_w, eps, y, accumulate, 0, 256, (cudaStream_t)stream);
}

/* Which kernel spk_vq_gemv would run: 1 = the persistent TMA kernel, 0 = generic. */
int spk_vq_gemv_fast_ok(int nstages, int ngroups, int dim, int nc, int rows, int cols, int v3) {
    if (dim <= 0 || nc <= 0 || rows <= 0 || cols <= 0) return 0;
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    const uint8_t *st[MAXQ] = {nullptr};
    for (int q = 0; q < MAXQ; q++) st[q] = (const uint8_t *)(uintptr_t)256;
    FastPlan P;
    return fast_plan(st, nstages, ngroups, L, &P) ? 1 : 0;
}

/* Bit-exact stage decode on a stream: out += decoded stage. */
int spk_vq_dequant(const void *payload, int dim, int nc, int rows, int cols, int v3, float *out, void *stream) {
    if (check_geometry(dim, nc, rows, cols, v3)) return -1;
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    const int threads = 256;
    const int blocks = (int)((L.nidx + threads - 1) / threads);
    vq_dequant_kernel<<<blocks, threads, 0, (cudaStream_t)stream>>>((const uint8_t *)payload, L, out,
                                                                   device_error_ptr());
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail("dequant launch", e);
}

}  // extern "C"
