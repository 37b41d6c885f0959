// vq_tab.cu — the decode step's VQ GEMVs as shared-memory table look-ups over index words
// whose look-up order is scheduled at load for the shared-memory banks, with the cross-CTA
// sums and the epilogue in the same launch.
//
// What it computes is spk_vq_gemv's (tools/vq-format/src/lib.rs:215-228 Stage::dot_row,
// decode-gpu.cu:267-301 gemv_v3blk_kernel, summed over stages as vq-model-gpu.cu:651-660):
//   y[r] (+)= sum_s gain_s[r] * sum_i sum_d cb_s[idx_s(r,i)][d] * xn[4i+d]
// for DQV3 stages of dim 4 with 4096 codes (12-bit row-local indices, no 13th-bit plane),
// xn = RMSNorm(x) when a norm weight is given (model.rs:236-245, f64 sum of squares), and the
// paired form y = gelu_erf(W_gate xn) * (W_up xn) (model.rs:253-258).
//
// The B200 design. A VQ index is a random look-up, so the GEMV is bound by the SM (shared-
// memory wavefronts, issue slots, latency), not by HBM. Per slice of 8 column groups (32
// columns) and stage a CTA builds the table T[jj][c] = cb_s[c] . xn[4(8 sl + jj) .. +4] for
// all 4096 codes (128 KB of f32, two 64 KB halves: jj 0-3 and jj 4-7), after which an index
// costs one shared load at a register offset and one add:
//   * the index streams are re-laid once at load: per (slice, row) one 16-byte word of 8 u16
//     byte offsets into a half table (16384 (jj mod 4) + 4 idx), u16 0-3 for jj 0-3 and 4-7
//     for jj 4-7, slice-major [sl][row]. Each offset names its own sub-table, so a row's four
//     look-ups of a half may run in any order; the re-lay orders them, for every warp of 32
//     rows, so that the warp's load steps spread over the 32 banks (a greedy assignment step
//     by step, then pairwise swaps within a row while the two steps' summed maximum bank
//     load drops): ~2.2 wavefronts per warp load instead of ~3.5 for 32 random words;
//   * the work, (group, slice, 32-row chunk) in that order, is cut evenly over one CTA per
//     SM; a CTA walks its contiguous range segment by segment (one slice's run of chunks),
//     and per segment stage by stage (a phase) builds the table and runs its look-ups. A warp
//     owns chunks c = warp + 16 j, a lane row 32 c + lane: the row's running sum stays in
//     shared memory (a conflict-free slot per thread and chunk) across every phase of the
//     CTA's range, so a CTA writes one partial per row it touched. The words of a phase's first 8 chunks are loaded before its table build (which
//     hides their latency), each later one 8 chunks ahead; the next phase's code words come
//     into shared memory by cp.async while this phase's look-ups run;
//   * the table build runs on paired f32 FMAs (two codes per instruction, the same rounding
//     as one FMA chain per entry), one conflict-free 8-byte store per entry pair;
//   * then a grid barrier (one CTA per SM, all resident: each triggers its dependents only
//     after starting), after which each CTA gathers the partials of its share of the rows
//     into shared memory by cp.async (one round trip), sums them over the CTAs that wrote
//     them in CTA order (the same order on every run) and applies the epilogue: store,
//     residual accumulate, or gelu_erf(gate) * up; for q_k_v_proj the last CTAs also compute
//     g_proj's rows.
#include "common.cuh"
#include "spk.h"

namespace spk {
namespace tab {

namespace {

constexpr int GC = 8;            // column groups per slice
constexpr int NC = 4096;         // codes
constexpr int NT = 512;          // threads of the kernel
constexpr int NW = NT / 32;      // warps
constexpr int MAXS = 20;         // 32-row chunks a warp owns: rows <= 32 * NW * MAXS
constexpr int D = 8;             // word prefetch depth (chunks)
constexpr int MAXSEG = 8;        // segments a CTA may walk
constexpr int MAXG = 2, MAXST = 2;
constexpr int MAXCH = 4;         // 32-row chunks a CTA's finishing rows span
constexpr int GX_MAX = 64;       // g_proj rows the kernel takes
constexpr int MAXCTA = 192;       // grid size the unit boundaries hold
constexpr int BUILD_COST = 96;    // a segment's table builds, in 32-row chunks of look-ups (for the split)
constexpr size_t SYNC_BYTES = 256;   // the scratch's grid-barrier count, ahead of the partials
constexpr size_t T_BYTES = (size_t)GC * NC * 4;
constexpr size_t HALF = T_BYTES / 2;
constexpr size_t CB_BYTES = (size_t)NC * 8;
// shared-memory plan (bytes)
constexpr size_t SM_T = 0, SM_CB = SM_T + T_BYTES, SM_ACC = SM_CB + CB_BYTES;
constexpr size_t SM_X = SM_ACC + (size_t)MAXS * NT * 4;
constexpr size_t SM_RED = SM_X + (size_t)MAXSEG * GC * 4 * 8, SM_FRED = SM_RED + NW * 8;
constexpr size_t SM_BND = SM_FRED + MAXST * NW * 4;
constexpr size_t SM_Y = SM_BND + (MAXCTA + 1) * 4;   // the finishing rows' residual (accumulate)
constexpr size_t SM_END = SM_Y + 128 * 4;

struct TabArgs {
    const uint4 *w[MAXG][MAXST];        // re-laid words [nsl][rows]
    const uint2 *cb[MAXG][MAXST];       // code words, 4 x f16 (8-byte aligned)
    const uint16_t *gain[MAXG][MAXST];  // f16 row gains
    int ng, ns, rows, nsl, cols;
    const float *x;
    const float *norm_w;                // optional RMSNorm weight
    float eps;
    float *part;                        // [ng][grid][rows]
    unsigned long long *bar;            // grid barrier count
    int mode;                           // 0 store, 1 accumulate, 2 gelu_erf(group 0) * group 1
    float *y;
    // g_proj (optional): rows of a second small matrix of the same input
    int xrows, xns;
    const uint8_t *xst[MAXST];
    Layout XL;
    float *xy;
    int *err;
    int bnd[MAXCTA + 1];                // CTA k walks units [bnd[k], bnd[k + 1])
};

__device__ __forceinline__ float h2f_bits(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }

__device__ __forceinline__ float gelu_erf(float g) {
    // model.rs:253-258: 0.5*x*(1 + erf(x/sqrt2)), erf in f64
    const double e = erf((double)g * 0.70710678118654752440);
    return __fmul_rn(__fmul_rn(0.5f, g), __fadd_rn(1.0f, (float)e));
}

// RMSNorm scale with the sum of squares in f64 (model.rs:236-245); every CTA sums in the
// same order and gets the same scale.
__device__ float rms_inv(const float *x, int n, float eps, double *red) {
    double s = 0.0;
    for (int i0 = threadIdx.x; i0 < n; i0 += 8 * NT) {   // 8 loads in flight, summed in index order
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = i0 + j * NT < n ? x[i0 + j * NT] : 0.f;
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (i0 + j * NT < n) s += (double)v[j] * (double)v[j];
    }
    s = warp_sum_d(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    double t = 0.0;
    for (int k = 0; k < NW; k++) t += red[k];
    __syncthreads();
    return (float)(1.0 / sqrt(t / (double)n + (double)eps));
}

__device__ __forceinline__ uint4 ldg_nc4(const uint4 *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t ldg_nc16(const uint16_t *p) {
    uint16_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned long long ld_relaxed(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// A hint to bring [p, p + bytes) into L2 by the TMA engine (16-byte granules inside the range).
__device__ __forceinline__ void l2_prefetch(const void *p, size_t bytes) {
    uintptr_t b = ((uintptr_t)p + 15) & ~(uintptr_t)15;
    const uintptr_t e = ((uintptr_t)p + bytes) & ~(uintptr_t)15;
    while (b < e) {
        const uint32_t n = (uint32_t)min((uintptr_t)65536, e - b);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(b), "r"(n) : "memory");
        b += n;
    }
}

__device__ __forceinline__ void cp_async8(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// A stage's 4096 code words into shared memory (8 per thread).
__device__ __forceinline__ void fetch_cb(uint2 *dst, const uint2 *src) {
#pragma unroll
    for (int c = threadIdx.x; c < NC; c += NT) cp_async8(dst + c, src + c);
    cp_async_commit();
}

// f32 pairs: two codes' products in one instruction, each half rounded as a scalar FMA.
__device__ __forceinline__ unsigned long long f2(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ unsigned long long mul2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// T[jj][c] = cb[c] . xs[jj][0..4] for the 4096 codes: thread t takes the code pairs
// (2p, 2p + 1), p = t + NT i; per pair and jj four paired FMAs (cb[c][0] x0 first, then
// + cb[c][1] x1, ..., as one FMA chain per entry) and one 8-byte store. xs2 holds each
// activation twice, (x, x), the pairs' second operand.
__device__ __forceinline__ void build_table(uint8_t *smem, const unsigned long long *xs2) {
    float *T = reinterpret_cast<float *>(smem + SM_T);
    const uint4 *cb4 = reinterpret_cast<const uint4 *>(smem + SM_CB);
    unsigned long long P[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint4 q = cb4[threadIdx.x + NT * i];
        const float2 a0 = __half22float2(*reinterpret_cast<const __half2 *>(&q.x));
        const float2 a1 = __half22float2(*reinterpret_cast<const __half2 *>(&q.y));
        const float2 b0 = __half22float2(*reinterpret_cast<const __half2 *>(&q.z));
        const float2 b1 = __half22float2(*reinterpret_cast<const __half2 *>(&q.w));
        P[i][0] = f2(a0.x, b0.x);
        P[i][1] = f2(a0.y, b0.y);
        P[i][2] = f2(a1.x, b1.x);
        P[i][3] = f2(a1.y, b1.y);
    }
#pragma unroll 2
    for (int jj = 0; jj < GC; jj++) {
        const ulonglong2 xa = reinterpret_cast<const ulonglong2 *>(xs2)[2 * jj];
        const ulonglong2 xb = reinterpret_cast<const ulonglong2 *>(xs2)[2 * jj + 1];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            unsigned long long e = mul2(P[i][0], xa.x);
            e = fma2(P[i][1], xa.y, e);
            e = fma2(P[i][2], xb.x, e);
            e = fma2(P[i][3], xb.y, e);
            *reinterpret_cast<unsigned long long *>(T + jj * NC + 2 * (threadIdx.x + NT * i)) = e;
        }
    }
}

// The 8 look-ups of one word: u16 0-3 are byte offsets into the low half table (jj 0-3),
// u16 4-7 into the high half (jj 4-7).
__device__ __forceinline__ float look8(const uint8_t *smem, const uint4 &w) {
    const uint8_t *ta = smem + SM_T, *tb = smem + SM_T + HALF;
    const float p0 = *reinterpret_cast<const float *>(ta + (w.x & 0xFFFFu));
    const float p1 = *reinterpret_cast<const float *>(ta + (w.x >> 16));
    const float p2 = *reinterpret_cast<const float *>(ta + (w.y & 0xFFFFu));
    const float p3 = *reinterpret_cast<const float *>(ta + (w.y >> 16));
    const float p4 = *reinterpret_cast<const float *>(tb + (w.z & 0xFFFFu));
    const float p5 = *reinterpret_cast<const float *>(tb + (w.z >> 16));
    const float p6 = *reinterpret_cast<const float *>(tb + (w.w & 0xFFFFu));
    const float p7 = *reinterpret_cast<const float *>(tb + (w.w >> 16));
    return ((p0 + p1) + (p2 + p3)) + ((p4 + p5) + (p6 + p7));
}

// Every CTA of the grid arrives once per launch, so the count is a multiple of the grid size
// whenever no launch is in flight; a CTA reads it after its wait for the previous kernel
// (`seen`: that launch has completed, and at most grid - 1 CTAs of this one have arrived), so
// this launch's target is the next multiple. Arrival is a release add with no reply; the CTA
// then polls with acquire loads, and returns when all have arrived or after a second with the
// error recorded. The grid is one CTA per SM and every CTA is resident before any dependent
// kernel may launch (each triggers dependents right after it starts), so all CTAs meet here.
__device__ void grid_barrier(unsigned long long *bar, unsigned long long seen, int *err) {
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned long long G = gridDim.x, target = (seen / G + 1) * G;
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(bar) : "memory");
        const unsigned long long t0 = globaltimer_ns();
        for (;;) {
            unsigned long long v;
            asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(bar) : "memory");
            if (v >= target) break;
            if (globaltimer_ns() - t0 > 1000000000ull) {
                if (err) atomicExch(err, DEV_WAIT_TIMEOUT);
                break;
            }
            __nanosleep(32);
        }
    }
    __syncthreads();
}

// One g_proj row (the stage payloads, read through L1): sum_s gain_s[row] * W_s[row] . xn,
// a CTA's threads over the row's indices, warp sums in a fixed order.
__device__ void gproj_row(const TabArgs &a, int row, float inv, float *fred) {
    const Layout &L = a.XL;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int s = 0; s < a.xns; s++) {
        const uint8_t *rowp = a.xst[s] + L.stream_off + (size_t)row * L.mrow;
        const uint2 *cb = reinterpret_cast<const uint2 *>(a.xst[s] + L.cb_off);
        float t = 0.f;
        for (int i = threadIdx.x; i < (int)L.nidx_row; i += NT) {
            const uint8_t *q = rowp + ((12 * i) >> 3);
            const uint32_t v = (((uint32_t)q[0] | ((uint32_t)q[1] << 8)) >> ((12 * i) & 7)) & 0xFFFu;
            const uint2 c = __ldg(cb + v);
            const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&c.x));
            const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&c.y));
            float xv[4];
#pragma unroll
            for (int d = 0; d < 4; d++) {
                xv[d] = a.x[4 * i + d];
                if (a.norm_w) xv[d] = __fmul_rn(__fmul_rn(xv[d], inv), a.norm_w[4 * i + d]);
            }
            t = fmaf(hi.y, xv[3], fmaf(hi.x, xv[2], fmaf(lo.y, xv[1], fmaf(lo.x, xv[0], t))));
        }
        t = warp_sum(t);
        if (lane == 0) fred[s * NW + warp] = t;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float o = 0.f;
        for (int s = 0; s < a.xns; s++) {
            float t = 0.f;
            for (int k = 0; k < NW; k++) t += fred[s * NW + k];
            const uint16_t gh = *reinterpret_cast<const uint16_t *>(a.xst[s] + L.gain_off + 2 * (size_t)row);
            o = __fadd_rn(o, __fmul_rn(t, h2f_bits(gh)));
        }
        a.xy[row] = o;
    }
    __syncthreads();
}

__global__ void __launch_bounds__(NT, 1) vq_tab_kernel(const TabArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint2 *cbs = reinterpret_cast<uint2 *>(smem + SM_CB);
    unsigned long long *xs2 = reinterpret_cast<unsigned long long *>(smem + SM_X);   // [MAXSEG][GC][4] (x, x)
    double *red = reinterpret_cast<double *>(smem + SM_RED);
    float *fred = reinterpret_cast<float *>(smem + SM_FRED);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, k = blockIdx.x;
    const int R = a.rows, nch = R >> 5, nsl = a.nsl;
    const int per_g = nsl * nch, W = per_g * a.ng;
    const int u0 = a.bnd[k], u1 = a.bnd[k + 1];
    int *bs = reinterpret_cast<int *>(smem + SM_BND);   // every CTA's unit boundaries, for the finishing sums
    for (int i = tid; i <= G; i += NT) bs[i] = a.bnd[i];
    pdl_trigger();
    // The index words and gains of phase (segment at unit u, stage st) into L2, a phase ahead.
    auto prefetch_phase = [&](int u, int st) {
        const int g = u / per_g, rem = u - g * per_g, sl = rem / nch, ca = rem - sl * nch;
        const int ce = min(nch, ca + (u1 - u));
        l2_prefetch(a.w[g][st] + (size_t)sl * R + 32 * ca, (size_t)(ce - ca) * 32 * 16);
        l2_prefetch(a.gain[g][st] + 32 * ca, (size_t)(ce - ca) * 32 * 2);
    };
    if (u0 < u1) {   // weights: before the wait
        fetch_cb(cbs, a.cb[u0 / per_g][0]);
        if (tid == 0) prefetch_phase(u0, 0);
    }
    // this thread's slice activation (segment tid / 32) and its norm weight (a weight: early)
    const int xv0 = u0 / nch, xnseg = min((u1 - 1) / nch - xv0 + 1, MAXSEG);
    const bool xmine = u0 < u1 && tid < xnseg * 32;
    const int xc = 32 * ((xv0 + tid / 32) % nsl) + (tid & 31);
    const float wv = xmine && a.norm_w ? a.norm_w[xc] : 1.f;

    float *acc = reinterpret_cast<float *>(smem + SM_ACC) + tid;   // [MAXS][NT]: this thread's rows' running sums
    uint32_t touched = 0;
    int cur_g = u0 < u1 ? u0 / per_g : 0;
    bool have_x = false;
    float inv = 1.0f;
    unsigned long long seen = 0;   // the barrier count after the wait (thread 0)
    const int r0 = R * k / G, r1 = R * (k + 1) / G, nr = r1 - r0;   // this CTA's finishing rows
    float *ys = reinterpret_cast<float *>(smem + SM_Y);

    int seg = 0;
    for (int u = u0; u < u1; seg++) {
        const int g = u / per_g, rem = u - g * per_g, sl = rem / nch, ca = rem - sl * nch;
        const int ce = min(nch, ca + (u1 - u));
        if (g != cur_g) {   // the pair's CTA that spans both groups: the gate rows' partials out
            float *pp = a.part + ((size_t)cur_g * G + k) * R + tid;
#pragma unroll
            for (int j = 0; j < MAXS; j++)
                if ((touched >> j) & 1u) pp[(size_t)j * NT] = acc[j * NT];
            touched = 0;
            cur_g = g;
        }
        // this warp's chunks warp + NW j in [ca, ce)
        const int ja = ca > warp ? (ca - warp + NW - 1) / NW : 0;
        const int jb = ce > warp ? (ce - warp + NW - 1) / NW : 0;
        const uint32_t fresh = jb > ja ? ((1u << jb) - 1u) & ~((1u << ja) - 1u) & ~touched : 0u;
        touched |= fresh;
        for (int s = 0; s < a.ns; s++) {
            const uint4 *wp = a.w[g][s] + (size_t)sl * R + tid;   // chunk j: + j * NT
            const uint16_t *gp = a.gain[g][s] + tid;
            uint4 wr[D];
            uint32_t gr[D];
#pragma unroll
            for (int j = 0; j < D; j++)
                if (j >= ja && j < jb) {
                    wr[j] = ldg_nc4(wp + (size_t)j * NT);
                    gr[j] = ldg_nc16(gp + (size_t)j * NT);
                }
            if (!have_x) {   // weights only so far: the activations after the wait
                pdl_wait();
                if (tid == 0) seen = ld_relaxed(a.bar);
                if (a.mode == 1 && tid < nr) ys[tid] = a.y[r0 + tid];   // the residual they add to, early
                // this thread's slice activation, loaded with the norm's
                float xv = xmine ? a.x[xc] : 0.f;
                if (a.norm_w) inv = rms_inv(a.x, a.cols, a.eps, red);
                if (xmine) {
                    if (a.norm_w) xv = __fmul_rn(__fmul_rn(xv, inv), wv);
                    xs2[tid] = f2(xv, xv);
                }
                have_x = true;
            }
            cp_async_wait_all();
            __syncthreads();   // the code words and xs2 are in; the previous look-ups are done with T
            build_table(smem, xs2 + 32 * seg);
            __syncthreads();
            // the next phase's code words, while these look-ups run
            if (s + 1 < a.ns) {
                fetch_cb(cbs, a.cb[g][s + 1]);
                if (tid == 0) prefetch_phase(u, s + 1);
            } else if (u + (ce - ca) < u1) {
                fetch_cb(cbs, a.cb[(u + (ce - ca)) / per_g][0]);
                if (tid == 0) prefetch_phase(u + (ce - ca), 0);
            }
            const uint4 *wq = wp + (size_t)D * NT;
            const uint16_t *gq = gp + (size_t)D * NT;
#pragma unroll 1
            for (int j0 = 0; j0 < jb; j0 += D) {
#pragma unroll
                for (int i = 0; i < D; i++) {
                    const int j = j0 + i;
                    if (j >= ja && j < jb) {
                        const float prev = (s == 0 && ((fresh >> j) & 1u)) ? 0.f : acc[j * NT];
                        acc[j * NT] = fmaf(look8(smem, wr[i]), h2f_bits(gr[i]), prev);
                    }
                    if (j + D >= ja && j + D < jb) {
                        wr[i] = ldg_nc4(wq);
                        gr[i] = ldg_nc16(gq);
                    }
                    wq += NT;
                    gq += NT;
                }
            }
        }
        u += ce - ca;
    }
    if (!have_x) {   // a CTA with no units still meets the barrier (and may take a g_proj row)
        pdl_wait();
        if (tid == 0) seen = ld_relaxed(a.bar);
        if (a.mode == 1 && tid < nr) ys[tid] = a.y[r0 + tid];
        if (a.norm_w) inv = rms_inv(a.x, a.cols, a.eps, red);
    }
    if (u0 < u1) {
        float *pp = a.part + ((size_t)cur_g * G + k) * R + tid;
#pragma unroll
        for (int j = 0; j < MAXS; j++)
            if ((touched >> j) & 1u) pp[(size_t)j * NT] = acc[j * NT];
    }
    grid_barrier(a.bar, seen, a.err);

    // ---- the finishing share: rows [r0, r1), summed over the CTAs that wrote them. A CTA that
    // holds unit (g, sl, c) for any slice sl wrote a partial for every row of chunk c of group
    // g; the rows' sums run over those CTAs in CTA order.
    if (nr > 0) {
        const int c0 = r0 >> 5, nck = ((r1 - 1) >> 5) - c0 + 1, ntask = a.ng * nck;   // task: (group, chunk)
        uint8_t *flag = smem;                                              // [ntask][G]
        int *lst = reinterpret_cast<int *>(smem + MAXG * MAXCH * MAXCTA);  // [ntask][G] covering CTAs, in order
        int *len = lst + MAXG * MAXCH * MAXCTA;                            // [ntask]
        float *Q = reinterpret_cast<float *>(len + MAXG * MAXCH);          // [parts][32]
        for (int e = tid; e < ntask * G; e += NT) {
            const int task = e / G, kk = e - task * G;
            const int base = (task / nck) * per_g + c0 + task % nck;   // unit (g, sl = 0, c)
            const int v0 = bs[kk], v1 = bs[kk + 1], lo = max(v0, base);
            const int sl0 = (lo - base + nch - 1) / nch;   // the first unit of chunk c at or after the range start
            flag[e] = sl0 < nsl && base + sl0 * nch < v1;
        }
        __syncthreads();
        const uint32_t lt = (1u << lane) - 1u;
        for (int task = warp; task < ntask; task += NW) {
            int n = 0;
            for (int k0 = 0; k0 < G; k0 += 32) {
                const int kk = k0 + lane;
                const bool f = kk < G && flag[task * G + kk];
                const uint32_t m = __ballot_sync(0xffffffffu, f);
                if (f) lst[task * G + n + __popc(m & lt)] = kk;
                n += __popc(m);
            }
            if (lane == 0) len[task] = n;
        }
        __syncthreads();
        // P warps per task split its list; each sums its share in list order, 16 loads in flight
        const int P = max(1, NW / ntask);
        for (int w2 = warp; w2 < ntask * P; w2 += NW) {
            const int task = w2 / P, pp = w2 % P, g = task / nck;
            const int row = 32 * (c0 + task % nck) + lane, n = len[task];
            const int i0 = n * pp / P, i1 = n * (pp + 1) / P;
            float t = 0.f;
            if (row >= r0 && row < r1) {
                const float *src = a.part + (size_t)g * G * R + row;
                const int *l = lst + task * G;
                int i = i0;
                for (; i + 16 <= i1; i += 16) {
                    float v[16];
#pragma unroll
                    for (int q = 0; q < 16; q++) v[q] = __ldcg(src + (size_t)l[i + q] * R);
#pragma unroll
                    for (int q = 0; q < 16; q++) t += v[q];
                }
                for (; i < i1; i++) t += __ldcg(src + (size_t)l[i] * R);
            }
            Q[(task * P + pp) * 32 + lane] = t;
        }
        __syncthreads();
        for (int ri = tid; ri < nr; ri += NT) {
            const int r = r0 + ri, cc = (r >> 5) - c0;
            float sg[MAXG];
#pragma unroll
            for (int g = 0; g < MAXG; g++) {
                float t = 0.f;
                if (g < a.ng)
                    for (int pp = 0; pp < P; pp++) t += Q[((g * nck + cc) * P + pp) * 32 + (r & 31)];
                sg[g] = t;
            }
            if (a.mode == 2)
                a.y[r] = __fmul_rn(gelu_erf(sg[0]), sg[1]);
            else if (a.mode == 1)
                a.y[r] = __fadd_rn(ys[ri], sg[0]);
            else
                a.y[r] = sg[0];
        }
    }
    // g_proj's rows: the last xrows CTAs, one row each
    if (a.xrows > 0 && k >= G - a.xrows) {
        __syncthreads();
        gproj_row(a, k - (G - a.xrows), inv, fred);
    }
}

// --------------------------------------------------------------- re-lay ---
// One thread per (slice, 32-row chunk): the chunk's rows' 8 indices of the slice (bytes
// [12 sl, 12 sl + 12) of each DQV3 row stream), as u16 byte offsets 16384 (jj mod 4) + 4 idx
// into their half table, u16 0-3 holding jj 0-3 and 4-7 holding jj 4-7, each half's four
// ordered per row so that the warp's load steps spread over the banks (bank = idx mod 32):
//   greedy: step by step, each row (in a rotating order) takes its remaining look-up whose
//   bank is least used in this step so far, ties to the bank with the most look-ups left;
//   then two passes of pairwise swaps within a row that lower the two steps' summed maximum
//   bank load (or keep it and lower the sum of squared loads).
constexpr int PK_T = 64;   // threads per block of the re-lay

struct PackScratch {
    uint8_t cnt[GC][32];   // per step, per bank
    uint8_t ord[GC][32];   // per step, per row: which of its 8 look-ups
    uint8_t mx[GC], nmx[GC];
    uint16_t dem[32];
    uint8_t used[32];
};

__global__ void __launch_bounds__(PK_T) tab_pack_kernel(const uint8_t *st, Layout L, uint4 *dst) {
    __shared__ PackScratch ps[PK_T];
    PackScratch &P = ps[threadIdx.x];
    const int nch = L.rows >> 5, nsl = (int)(L.nidx_row / GC);
    const long long n = (long long)nsl * nch;
    for (long long e = blockIdx.x * (long long)PK_T + threadIdx.x; e < n; e += (long long)gridDim.x * PK_T) {
        const int sl = (int)(e / nch), c = (int)(e % nch);
        uint16_t idx[32][GC];
        for (int l = 0; l < 32; l++) {
            const uint8_t *q = st + L.stream_off + (size_t)(32 * c + l) * L.mrow + 12 * (size_t)sl;
#pragma unroll
            for (int h = 0; h < 4; h++) {
                const uint32_t b = (uint32_t)q[3 * h] | ((uint32_t)q[3 * h + 1] << 8) | ((uint32_t)q[3 * h + 2] << 16);
                idx[l][2 * h] = (uint16_t)(b & 0xFFFu);
                idx[l][2 * h + 1] = (uint16_t)((b >> 12) & 0xFFFu);
            }
        }
        auto remax = [&](int t) {
            int m = 0, nm = 0;
            for (int b = 0; b < 32; b++) {
                const int v = P.cnt[t][b];
                if (v > m) m = v, nm = 1;
                else if (v == m) nm++;
            }
            P.mx[t] = (uint8_t)m;
            P.nmx[t] = (uint8_t)nm;
        };
        for (int hf = 0; hf < 2; hf++) {   // look-ups jj 4 hf .. 4 hf + 3 into steps 4 hf .. 4 hf + 3
            const int q0 = 4 * hf;
            for (int b = 0; b < 32; b++) P.dem[b] = 0;
            for (int l = 0; l < 32; l++) {
                P.used[l] = 0;
                for (int q = q0; q < q0 + 4; q++) P.dem[idx[l][q] & 31]++;
            }
            for (int t = q0; t < q0 + 4; t++) {
                for (int b = 0; b < 32; b++) P.cnt[t][b] = 0;
                for (int i = 0; i < 32; i++) {
                    const int l = (t * 7 + i) & 31;
                    int best = q0, bk = 1 << 30;
                    for (int q = q0; q < q0 + 4; q++) {
                        if ((P.used[l] >> q) & 1) continue;
                        const int b = idx[l][q] & 31;
                        const int key = (int)P.cnt[t][b] * 1024 - (int)P.dem[b];
                        if (key < bk) bk = key, best = q;
                    }
                    const int b = idx[l][best] & 31;
                    P.used[l] |= (uint8_t)(1u << best);
                    P.cnt[t][b]++;
                    P.dem[b]--;
                    P.ord[t][l] = (uint8_t)best;
                }
                remax(t);
            }
            for (int pass = 0; pass < 2; pass++)
                for (int l = 0; l < 32; l++)
                    for (int t1 = q0; t1 < q0 + 3; t1++)
                        for (int t2 = t1 + 1; t2 < q0 + 4; t2++) {
                            const int b1 = idx[l][P.ord[t1][l]] & 31, b2 = idx[l][P.ord[t2][l]] & 31;
                            if (b1 == b2) continue;
                            int m1 = (P.cnt[t1][b1] == P.mx[t1] && P.nmx[t1] == 1) ? P.mx[t1] - 1 : P.mx[t1];
                            m1 = max(m1, P.cnt[t1][b2] + 1);
                            int m2 = (P.cnt[t2][b2] == P.mx[t2] && P.nmx[t2] == 1) ? P.mx[t2] - 1 : P.mx[t2];
                            m2 = max(m2, P.cnt[t2][b1] + 1);
                            const int was = P.mx[t1] + P.mx[t2], now = m1 + m2;
                            const int s0 = P.cnt[t1][b1] + P.cnt[t2][b2], s1 = P.cnt[t1][b2] + P.cnt[t2][b1] + 2;
                            if (now < was || (now == was && s1 < s0)) {
                                P.cnt[t1][b1]--, P.cnt[t1][b2]++, P.cnt[t2][b2]--, P.cnt[t2][b1]++;
                                const uint8_t o = P.ord[t1][l];
                                P.ord[t1][l] = P.ord[t2][l];
                                P.ord[t2][l] = o;
                                remax(t1);
                                remax(t2);
                            }
                        }
        }
        for (int l = 0; l < 32; l++) {
            uint32_t o[4];
#pragma unroll
            for (int h = 0; h < 4; h++) {
                const int qa = P.ord[2 * h][l], qb = P.ord[2 * h + 1][l];
                o[h] = (16384u * (qa & 3) + 4u * idx[l][qa]) | ((16384u * (qb & 3) + 4u * idx[l][qb]) << 16);
            }
            dst[(size_t)sl * L.rows + 32 * c + l] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

// The CTAs' unit ranges: contiguous, in order, each costing its chunks plus BUILD_COST per
// segment it touches (its table builds), the largest cost as small as a greedy cut allows
// (binary search on the bound; trailing CTAs may be empty).
int greedy_cut(int W, int nch, long long C, int *bnd, int G) {
    int u = 0, n = 0;
    while (u < W) {
        if (bnd && n < G) bnd[n] = u;
        n++;
        long long c = 0;
        const int start = u;
        while (u < W) {
            const int se = min(W, (u / nch + 1) * nch);
            if (c + BUILD_COST + (se - u) <= C) {
                c += BUILD_COST + (se - u);
                u = se;
            } else {
                const long long take = C - c - BUILD_COST;
                if (take > 0) u += (int)take;
                else if (u == start) u++;   // cannot happen for C >= BUILD_COST + 1
                break;
            }
        }
    }
    return n;
}

void split_units_now(int W, int nch, int G, int *bnd) {
    long long lo = (W + G - 1) / G + BUILD_COST, hi = (long long)W + (long long)BUILD_COST * (W / nch + 2);
    while (lo < hi) {
        const long long mid = (lo + hi) / 2;
        if (greedy_cut(W, nch, mid, nullptr, G) <= G) hi = mid;
        else lo = mid + 1;
    }
    const int n = greedy_cut(W, nch, lo, bnd, G);
    for (int k = n; k <= G; k++) bnd[k] = W;
}

// The same, remembered per geometry (a launch must not pay the search): a small per-thread cache.
void split_units(int W, int nch, int G, int *bnd) {
    struct Entry {
        int W, nch, G;
        int bnd[MAXCTA + 1];
    };
    static thread_local Entry cache[16];
    static thread_local int used = 0, next = 0;
    for (int i = 0; i < used; i++)
        if (cache[i].W == W && cache[i].nch == nch && cache[i].G == G) {
            memcpy(bnd, cache[i].bnd, sizeof(int) * (G + 1));
            return;
        }
    Entry &e = cache[next];
    next = (next + 1) % 16;
    if (used < 16) used++;
    e.W = W, e.nch = nch, e.G = G;
    split_units_now(W, nch, G, e.bnd);
    memcpy(bnd, e.bnd, sizeof(int) * (G + 1));
}

}  // namespace

bool ok(const Layout &L, int ns, int ng) {
    if (!(L.v3 && L.dim == 4 && L.nc == NC && L.nbit == 12 && L.prow == 0 && L.nidx_row % GC == 0)) return false;
    if (ns < 1 || ns > MAXST || ng < 1 || ng > MAXG || L.mrow * 2 != L.nidx_row * 3) return false;
    if (L.rows % 32 || L.rows > 32 * NW * MAXS) return false;
    const long long G = sm_count(), nch = L.rows / 32, nsl = (long long)L.nidx_row / GC;
    if (G > MAXCTA) return false;
    const long long W = (long long)ng * nsl * nch;
    if ((W + 1) * (G + 1) >= (1LL << 31) || (long long)L.rows * (G + 1) >= (1LL << 31)) return false;   // 32-bit
    int bnd[MAXCTA + 1];
    split_units((int)W, (int)nch, (int)G, bnd);
    for (int k = 0; k < G; k++)
        if (bnd[k + 1] > bnd[k] && (bnd[k + 1] - 1) / nch - bnd[k] / nch + 1 > MAXSEG) return false;
    const long long nr = (L.rows + G - 1) / G;
    if ((nr + 31) / 32 + 1 > MAXCH) return false;
    // the finishing stage: partials [ng][G][nrp] and covering flags [ng][G][chunks] in the table's space
    if ((size_t)MAXG * MAXCH * MAXCTA * 5 + MAXG * MAXCH * 4 + (size_t)MAXG * MAXCH * ((G + 31) / 32) * 32 * 4 > SM_X)
        return false;
    if (nr > 128) return false;   // the residual rows held for the epilogue
    return SM_END <= smem_optin_max();
}

size_t bytes(const Layout &L) { return (L.nidx_row / GC) * (size_t)L.rows * 16; }

size_t scratch_bytes(const Layout &L, int ng) { return SYNC_BYTES + (size_t)ng * sm_count() * L.rows * 4; }

int pack(const void *stage, const Layout &L, void *dst, cudaStream_t s) {
    if (!stage || !dst) return set_error("vq table re-lay: null pointer");
    if (((uintptr_t)dst & 15) != 0) return set_error("vq table re-lay: the destination must be 16-byte aligned");
    const long long n = (long long)(L.nidx_row / GC) * (L.rows / 32);
    const long long nb = (n + PK_T - 1) / PK_T;
    const int blocks = (int)(nb < 65535 ? nb : 65535);
    tab_pack_kernel<<<blocks, PK_T, 0, s>>>((const uint8_t *)stage, L, (uint4 *)dst);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail("vq table re-lay launch", e);
}

// y (=|+=) W RMSNorm?(x) (ng 1) or y = gelu_erf(W_gate xn) * (W_up xn) (ng 2); stages / words
// group-major; scratch >= scratch_bytes(L, ng), zeroed before its first use. xst / XL / xy: an
// optional g_proj of the same input (xrows <= 64), computed by the last CTAs.
int gemv(const void *const *stages, const void *const *words, int ns, int ng, const Layout &L, const float *x,
         const float *norm_w, float eps, float *y, int accumulate, void *scratch, const void *const *xst,
         const Layout *XL, float *xy, cudaStream_t s) {
    if (!ok(L, ns, ng)) return set_error("vq table kernel: geometry not taken");
    if (ng == 2 && accumulate) return set_error("the paired gate/up form writes its output, it cannot accumulate");
    if (!x || !y || !scratch) return set_error("vq table kernel: null pointer");
    if ((uintptr_t)scratch & 15) return set_error("vq table kernel: scratch must be 16-byte aligned");
    TabArgs a;
    memset(&a, 0, sizeof a);
    for (int g = 0; g < ng; g++)
        for (int q = 0; q < ns; q++) {
            const uint8_t *st = (const uint8_t *)stages[g * ns + q];
            if (!st || !words[g * ns + q]) return set_error("stage %d payload or table words are null", g * ns + q);
            if (((uintptr_t)st + L.cb_off) & 7) return set_error("stage codebook is not 8-byte aligned");
            if ((uintptr_t)words[g * ns + q] & 15) return set_error("vq table words must be 16-byte aligned");
            a.w[g][q] = (const uint4 *)words[g * ns + q];
            a.cb[g][q] = (const uint2 *)(st + L.cb_off);
            a.gain[g][q] = (const uint16_t *)(st + L.gain_off);
        }
    a.ng = ng;
    a.ns = ns;
    a.rows = L.rows;
    a.nsl = (int)(L.nidx_row / GC);
    a.cols = L.cols;
    a.x = x;
    a.norm_w = norm_w;
    a.eps = eps;
    a.bar = (unsigned long long *)scratch;
    a.part = (float *)((uint8_t *)scratch + SYNC_BYTES);
    a.mode = ng == 2 ? 2 : (accumulate ? 1 : 0);
    a.y = y;
    a.err = device_error_ptr();
    split_units(ng * a.nsl * (L.rows / 32), L.rows / 32, sm_count(), a.bnd);
    if (xst && XL && xy) {
        if (XL->rows > GX_MAX || XL->rows > sm_count() || XL->cols != L.cols || !XL->v3 || XL->dim != 4 ||
            XL->nbit != 12 || XL->prow)
            return set_error("vq table kernel: the extra matrix is not a small DQV3 matrix of the same input");
        a.xrows = XL->rows;
        a.xns = ns;
        for (int q = 0; q < ns; q++) a.xst[q] = (const uint8_t *)xst[q];
        a.XL = *XL;
        a.xy = xy;
    }
    static size_t opted[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (SM_END > opted[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(vq_tab_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SM_END);
        if (e != cudaSuccess) return cuda_fail("vq table kernel shared-memory opt-in", e);
        opted[dev & 63] = SM_END;
    }
    cudaError_t e = launch_pdl(vq_tab_kernel, dim3(sm_count()), dim3(NT), SM_END, s, a);
    return e == cudaSuccess ? 0 : cuda_fail("vq table kernel launch", e);
}

}  // namespace tab
}  // namespace spk

using namespace spk;

extern "C" {

size_t spk_vq_tab_bytes(int dim, int nc, int rows, int cols, int v3) {
    if (dim <= 0 || nc <= 0 || rows <= 0 || cols <= 0 || cols % dim) return 0;
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    return tab::ok(L, 1, 1) ? tab::bytes(L) : 0;
}

int spk_vq_tab_pack(const void *stage, int dim, int nc, int rows, int cols, int v3, void *dst, void *stream) {
    if (!spk_vq_tab_bytes(dim, nc, rows, cols, v3)) return set_error("vq table kernel: geometry not taken");
    return tab::pack(stage, make_layout(dim, nc, rows, cols, v3), dst, (cudaStream_t)stream);
}

size_t spk_vq_tab_scratch_bytes(int ngroups, int dim, int nc, int rows, int cols, int v3) {
    if (!spk_vq_tab_bytes(dim, nc, rows, cols, v3) || ngroups < 1 || ngroups > 2) return 0;
    return tab::scratch_bytes(make_layout(dim, nc, rows, cols, v3), ngroups);
}

int spk_vq_tab_gemv(const void *const *stages, const void *const *words, int nstages, int ngroups, int dim, int nc,
                    int rows, int cols, int v3, const float *x, const float *norm_w, float eps, float *y,
                    int accumulate, void *scratch, void *stream) {
    if (!stages || !words) return set_error("vq table kernel: null stage list");
    if (!spk_vq_tab_bytes(dim, nc, rows, cols, v3)) return set_error("vq table kernel: geometry not taken");
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    return tab::gemv(stages, words, nstages, ngroups, L, x, norm_w, eps, y, accumulate, scratch, nullptr, nullptr,
                     nullptr, (cudaStream_t)stream);
}

}  // extern "C"
