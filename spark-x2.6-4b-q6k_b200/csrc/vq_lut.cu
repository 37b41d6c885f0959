// vq_lut.cu — the decode GEMV over residual-VQ stages as shared-memory table look-ups.
//
// What it computes is spk_vq_gemv's (tools/vq-format/src/lib.rs:215-228 Stage::dot_row,
// decode-gpu.cu:267-301 gemv_v3blk_kernel, summed over stages as vq-model-gpu.cu:651-660):
//   y[r] (+)= sum_s gain_s[r] * sum_i sum_d cb_s[idx_s(r,i)][d] * x[4i+d]
// for DQV3 stages of dim 4 with 4096 codes (12-bit row-local indices, no 13th-bit plane).
//
// The B200 design. The VQ GEMV is bound by shared memory, not by HBM: every index is a random
// look-up. Gathering 8-byte code words costs ~7 shared wavefronts per 32 indices plus two
// conversions and four FMAs each; here an index costs one 4-byte look-up (~3.5 wavefronts
// per 32 random lanes) and one add:
//   * the column groups i (4 columns each) are cut into slices of 8; for one slice and one
//     stage the CTA builds the table T[jj][c] = cb_s[c] . (w . x)[4(8 sl + jj) .. +4] for all
//     4096 codes c and the slice's 8 groups jj (128 KB of f32 in shared memory);
//   * each stage is re-laid once at load into self-contained words: the code words, the row
//     gains, then the index stream slice-major, [sl][row] 12-byte records holding the row's 8
//     indices of the slice exactly as the DQV3 row stream holds them (bytes [12 sl, 12 sl + 12)
//     of the row): the same bytes as the payload, so the kernel reads 1.0x the container;
//   * the work, (group, slice, row octet) in that order, is cut evenly over one CTA per SM; a
//     CTA's range is a run of segments (one slice's rows of one group), walked in phases
//     (segment, stage) ordered group, stage, segment, building the table once per phase;
//   * warp specialization: one producer warp streams the records and gains of every phase,
//     512 rows per tile, with the TMA engine (1-D bulk copies, no multicast) into a 12-slot
//     mbarrier ring, after an L2 prefetch of all the CTA's records at launch; sixteen consumer
//     warps build each table on the tensor cores (mma tf32, code-word fragments loaded into
//     registers during the previous phase) and do the look-ups, a lane per row, four rows at a
//     time;
//   * a row's value for the slice (gains applied, stages summed, times the RMSNorm scale, which
//     the table leaves out: T is linear in x) goes to a partial buffer [group][slice][row]
//     (the stage-0 value waits there for stage 1);
//   * then a grid barrier (one CTA per SM, all resident), after which every warp of the grid
//     sums rows' partials in slice order (the same order on every run) and applies the
//     epilogue: store, residual accumulate, or gelu_erf(gate) * up; for q_k_v_proj the producer
//     warps of the first CTAs compute g_proj's rows from the stage payloads meanwhile.
#include "common.cuh"
#include "spk.h"

namespace spk {

namespace {

constexpr int LGC = 8;           // column groups per slice
constexpr int LNC = 4096;        // codes
constexpr int LMAXS = 2;         // stages
constexpr int TPAD = LNC + 4;    // floats per jj table: the +4 makes the builder's stores conflict-free
constexpr int CW = 16;           // warps of the table kernel
constexpr int CT = CW * 32;      // its threads
constexpr int NT = CT;
constexpr int TR = CT;           // rows per tile (a thread per row)
constexpr int IT = 4;            // tiles per iteration (rows per thread), the next iteration's loads in flight
constexpr int CB_BYTES = LNC * 8;
constexpr int GX_MAX = 64;       // g_proj rows the finishing kernel takes
constexpr int LMAXSEG = 8;       // segments a CTA of the table kernel may walk
constexpr size_t LUT_SYNC_BYTES = 256;   // the scratch's grid-barrier words, ahead of the partials

constexpr int CBW = LNC / 16 / CW;   // code-word fragments a thread holds per table build
// Shared-memory plan of the table kernel (bytes): table, then the rest.
constexpr size_t SM_T = 0, SM_REST = SM_T + (size_t)LGC * TPAD * 4;

// A re-laid stage: [code words 32 KB, in the table builder's fragment order][code words 32 KB,
// natural order (the batched GEMM's gathers, vq_tc.cu)][gains, rows8 f16, padded to 16 B]
// [records nsl x rows8 x 12]. rows8: rows rounded up to a multiple of 8 (padding rows are
// zero), so every tile's records and gains start on a 16-byte boundary.
__host__ __device__ constexpr size_t lut_gain_bytes(int rows8) { return ((size_t)rows8 * 2 + 15) & ~(size_t)15; }

struct LutArgs {
    const uint8_t *lut[2][LMAXS];     // re-laid stage words, group-major
    int ng, ns, rows, rows8, nsl, cols;
    size_t rec_off;                   // byte offset of the records in a stage's words
    const float *x;
    const float *norm_w;              // optional RMSNorm weight
    float eps;
    float *part;                      // [ng][nsl][rows]
    unsigned int *sync;               // grid barrier: [0] arrivals, [8] generation (zeroed once)
    int mode;                         // 0 store, 1 accumulate, 2 gelu_erf(group 0) * group 1
    float *y;
    // g_proj (optional): rows of a second matrix of the same input, one producer warp each
    int xrows, xns;
    const uint8_t *xst[LMAXS];
    Layout XL;
    float *xy;
    int *err;
};

__device__ __forceinline__ float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ float gelu_erf(float g) {
    // model.rs:253-258: 0.5*x*(1 + erf(x/sqrt2)), erf in f64
    const double e = erf((double)g * 0.70710678118654752440);
    return __fmul_rn(__fmul_rn(0.5f, g), __fadd_rn(1.0f, (float)e));
}

// A hint to bring [p, p + bytes) into L2 by the TMA engine (16-byte granules inside the range:
// the start rounded up, the end down, so nothing outside it is touched).
__device__ __forceinline__ void l2_prefetch(const void *p, size_t bytes) {
    uintptr_t b = ((uintptr_t)p + 15) & ~(uintptr_t)15;
    const uintptr_t e = ((uintptr_t)p + bytes) & ~(uintptr_t)15;
    while (b < e) {
        const uint32_t n = (uint32_t)min((uintptr_t)32768, e - b);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(b), "r"(n) : "memory");
        b += n;
    }
}

// A CTA's unit range [u0, u1) (units: row octets) is a run of segments, each one slice's
// contiguous rows of one group: (g, sl, [ra, rb)). The CTA walks them in phases (segment,
// stage) ordered by group, then stage, then segment, so the code words change only with the
// (group, stage) block: at most 2 x ns code-word loads per CTA.
struct Seg {
    int g, sl, ra, rb;
};

__device__ int make_segs(const LutArgs &a, int u0, int u1, Seg *segs) {
    const int Q = a.rows8 >> 3, per_g = a.nsl * Q;
    int u = u0, n = 0;
    while (u < u1 && n < LMAXSEG) {
        const int g = u / per_g, rem = u - g * per_g, sl = rem / Q, qa = rem - sl * Q;
        const int qb = min(Q, qa + (u1 - u));
        segs[n++] = {g, sl, 8 * qa, 8 * qb};
        u += qb - qa;
    }
    return n;
}

// Phase k: segment j at stage s, in block b (its code words); first / last phase of its block.
struct Phase {
    int j, s, b;
    bool first, last;
};

__device__ __forceinline__ bool phase_of(const Seg *segs, int nseg, int ns, int k, Phase &p) {
    int b = 0;
    for (int i0 = 0; i0 < nseg;) {
        int i1 = i0 + 1;
        while (i1 < nseg && segs[i1].g == segs[i0].g) i1++;
        const int cnt = i1 - i0;
        for (int s = 0; s < ns; s++, b++) {
            if (k < cnt) {
                p.j = i0 + k;
                p.s = s;
                p.b = b;
                p.first = k == 0;
                p.last = k == cnt - 1;
                return true;
            }
            k -= cnt;
        }
        i0 = i1;
    }
    return false;
}

// Byte offsets 4 * idx_jj of a record's 8 indices (bits [12 jj, 12 jj + 12) of the record's
// little-endian 96 bits w0 | w1 << 32 | w2 << 64), summed from the table.
__device__ __forceinline__ float lookup8(const char *t, uint32_t w0, uint32_t w1, uint32_t w2) {
    constexpr int S = TPAD * 4;   // bytes per jj table
    const uint32_t o0 = (w0 << 2) & 0x3FFCu;
    const uint32_t o1 = (w0 >> 10) & 0x3FFCu;
    const uint32_t o2 = __funnelshift_r(w0, w1, 22) & 0x3FFCu;
    const uint32_t o3 = (w1 >> 2) & 0x3FFCu;
    const uint32_t o4 = (w1 >> 14) & 0x3FFCu;
    const uint32_t o5 = __funnelshift_r(w1, w2, 26) & 0x3FFCu;
    const uint32_t o6 = (w2 >> 6) & 0x3FFCu;
    const uint32_t o7 = (w2 >> 18) & 0x3FFCu;
    const float p0 = *reinterpret_cast<const float *>(t + o0);
    const float p1 = *reinterpret_cast<const float *>(t + S + o1);
    const float p2 = *reinterpret_cast<const float *>(t + 2 * S + o2);
    const float p3 = *reinterpret_cast<const float *>(t + 3 * S + o3);
    const float p4 = *reinterpret_cast<const float *>(t + 4 * S + o4);
    const float p5 = *reinterpret_cast<const float *>(t + 5 * S + o5);
    const float p6 = *reinterpret_cast<const float *>(t + 6 * S + o6);
    const float p7 = *reinterpret_cast<const float *>(t + 7 * S + o7);
    return ((p0 + p1) + (p2 + p3)) + ((p4 + p5) + (p6 + p7));
}

__device__ __forceinline__ uint32_t tf32_rna(float v) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
    return r;
}

// T[jj][c] = cb[c] . xv[jj] for the slice's 8 groups and all 4096 codes on the tensor cores:
// mma m16n8k8 tf32 with the 16 codes of a block as M, the 8 groups as N and K = (4 dims of
// x_hi, 4 dims of x_lo), x = x_hi + x_lo split in tf32 (~22 bits; the code words, f16, are
// exact in tf32). Code words come in fragment order: word (block, t, g) holds codes
// 16 block + g and 16 block + g + 8 of dim t as an f16 pair; warp w builds blocks w, w + CW, ...
// from the CBW words its lane loaded (cb_load) ahead of time.
__device__ __forceinline__ void cb_load(uint32_t (&w)[CBW], const uint8_t *words) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const uint32_t *cw = reinterpret_cast<const uint32_t *>(words);
#pragma unroll
    for (int i = 0; i < CBW; i++) w[i] = __ldg(cw + ((warp + CW * i) * 4 + t) * 8 + g);
}

__device__ __forceinline__ void build_table(float *T, const uint32_t (&w)[CBW], const float *xs32) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const float xv = xs32[4 * g + t];   // group g, dim t
    const uint32_t bh = tf32_rna(xv);
    const uint32_t bl = tf32_rna(xv - __uint_as_float(bh));
#pragma unroll
    for (int i = 0; i < CBW; i++) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
        const uint32_t a0 = __float_as_uint(f.x), a1 = __float_as_uint(f.y);
        float d0, d1, d2, d3;
        asm volatile(
            "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%10,%10,%10,%10};"
            : "=f"(d0), "=f"(d1), "=f"(d2), "=f"(d3)
            : "r"(a0), "r"(a1), "r"(a0), "r"(a1), "r"(bh), "r"(bl), "f"(0.0f));
        const int c = 16 * (warp + CW * i) + g;
        T[(2 * t) * TPAD + c] = d0;
        T[(2 * t + 1) * TPAD + c] = d1;
        T[(2 * t) * TPAD + c + 8] = d2;
        T[(2 * t + 1) * TPAD + c + 8] = d3;
    }
}

// One g_proj row by one warp (the stage payloads, read through L1): sum_s gain_s[row] *
// W_s[row] . xn, the RMSNorm scale from the warp's own f64 sum of squares.
__device__ void gproj_warp(const LutArgs &a, int row) {
    const int lane = threadIdx.x & 31;
    const Layout &L = a.XL;
    float inv = 1.0f;
    if (a.norm_w) {
        double ss = 0.0;
        for (int i = lane; i < L.cols; i += 32) ss += (double)a.x[i] * (double)a.x[i];
        ss = warp_sum_d(ss);
        inv = (float)(1.0 / sqrt(ss / (double)L.cols + (double)a.eps));
    }
    float o = 0.f;
    for (int s = 0; s < a.xns; s++) {
        const uint8_t *rowp = a.xst[s] + L.stream_off + (size_t)row * L.mrow;
        const uint2 *cb = reinterpret_cast<const uint2 *>(a.xst[s] + L.cb_off);
        float t = 0.f;
        for (int i = lane; i < (int)L.nidx_row; i += 32) {
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
        const uint16_t gh = *reinterpret_cast<const uint16_t *>(a.xst[s] + L.gain_off + 2 * (size_t)row);
        o = __fadd_rn(o, __fmul_rn(t, h2f_bits(gh)));
    }
    if (lane == 0) a.xy[row] = o;
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Every CTA of the grid arrives; returns when all have (generation flip), or after a second
// with the error recorded. The grid is one CTA per SM and every CTA is resident before any
// dependent kernel may launch (each triggers it only after starting), so all CTAs meet here.
__device__ void grid_barrier(unsigned int *sync, int *err) {
    if (threadIdx.x == 0) {
        volatile unsigned int *gen = sync + 8;
        const unsigned int g0 = *gen;
        __threadfence();
        if (atomicAdd(sync, 1u) == gridDim.x - 1) {
            sync[0] = 0;
            __threadfence();
            atomicAdd(sync + 8, 1u);
        } else {
            const unsigned long long t0 = globaltimer_ns();
            while (*gen == g0)
                if (globaltimer_ns() - t0 > 1000000000ull) {
                    atomicExch(err, DEV_WAIT_TIMEOUT);
                    break;
                }
        }
        __threadfence();
    }
    __syncthreads();
}

// A thread's records and gains for IT rows of a phase (rows ra + (t0 + i) TR + tid), read-only
// loads straight to registers.
struct Rows {
    uint32_t w0[IT], w1[IT], w2[IT];
    float gn[IT];
};

__device__ __forceinline__ void load_rows(Rows &q, const uint32_t *rec, const uint16_t *gai, int t0, int nr) {
#pragma unroll
    for (int i = 0; i < IT; i++) {
        const int ir = (t0 + i) * TR + (int)threadIdx.x;
        if (ir < nr) {
            q.w0[i] = __ldg(rec + 3 * ir);
            q.w1[i] = __ldg(rec + 3 * ir + 1);
            q.w2[i] = __ldg(rec + 3 * ir + 2);
            q.gn[i] = h2f_bits(__ldg(gai + ir));
        } else {
            q.w0[i] = q.w1[i] = q.w2[i] = 0;
            q.gn[i] = 0.f;
        }
    }
}

__global__ void __launch_bounds__(NT, 1) vq_lut_kernel(const LutArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    float *T = reinterpret_cast<float *>(smem + SM_T);                    // [LGC][TPAD]
    float *xs = reinterpret_cast<float *>(smem + SM_REST);                 // [LMAXSEG][32] (w . x) per segment
    double *red = reinterpret_cast<double *>(xs + LMAXSEG * 32);           // [CW]
    Seg *segs = reinterpret_cast<Seg *>(red + CW);                         // [LMAXSEG]
    int *nseg_s = reinterpret_cast<int *>(segs + LMAXSEG);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int W = a.ng * a.nsl * (a.rows8 >> 3);   // the host checks it fits in 32 bits
    const int u0 = (int)((long long)W * blockIdx.x / gridDim.x), u1 = (int)((long long)W * (blockIdx.x + 1) / gridDim.x);
    if (tid == 0) *nseg_s = make_segs(a, u0, u1, segs);
    __syncthreads();
    pdl_trigger();
    const int nseg = *nseg_s;
    Phase p;
    if (tid == 0)   // weights only: everything this CTA reads, into L2
        for (int k = 0; phase_of(segs, nseg, a.ns, k, p); k++) {
            const Seg &sg = segs[p.j];
            l2_prefetch(a.lut[sg.g][p.s] + a.rec_off + ((size_t)sg.sl * a.rows8 + sg.ra) * 12, (size_t)(sg.rb - sg.ra) * 12);
            l2_prefetch(a.lut[sg.g][p.s] + 2 * CB_BYTES + (size_t)sg.ra * 2, (size_t)(sg.rb - sg.ra) * 2);
        }
    uint32_t cbf[CBW];   // the next table's code-word fragments
    Rows cur;            // the first rows of the first phase: weights, loaded before the wait
    if (phase_of(segs, nseg, a.ns, 0, p)) {
        const Seg &sg = segs[p.j];
        cb_load(cbf, a.lut[sg.g][p.s]);
        load_rows(cur, reinterpret_cast<const uint32_t *>(a.lut[sg.g][p.s] + a.rec_off) + ((size_t)sg.sl * a.rows8 + sg.ra) * 3,
                  reinterpret_cast<const uint16_t *>(a.lut[sg.g][p.s] + 2 * CB_BYTES) + sg.ra, 0, sg.rb - sg.ra);
    }
    pdl_wait();
    // the RMSNorm sum of squares (f64, model.rs:236-245): loads now, reduced at the first table's barrier
    double ss = 0.0;
    if (a.norm_w)
        for (int i = tid; i < a.cols; i += CT) ss += (double)a.x[i] * (double)a.x[i];
    for (int j = warp; j < nseg; j += CW) {   // each segment's 32 activations (norm weight applied;
        const int c = 32 * segs[j].sl + lane; // the scale multiplies the result)
        xs[32 * j + lane] = a.norm_w ? __fmul_rn(a.x[c], a.norm_w[c]) : a.x[c];
    }
    float inv = 1.0f;
    for (int k = 0; phase_of(segs, nseg, a.ns, k, p); k++) {
        __syncthreads();   // every thread is done with the previous table; xs is written
        const Seg sg = segs[p.j];
        build_table(T, cbf, xs + 32 * p.j);
        if (k == 0 && a.norm_w) {
            ss = warp_sum_d(ss);
            if (lane == 0) red[warp] = ss;
        }
        __syncthreads();   // the table is complete
        if (k == 0 && a.norm_w) {   // every thread sums the warps in the same order
            double t = 0.0;
            for (int i = 0; i < CW; i++) t += red[i];
            inv = (float)(1.0 / sqrt(t / (double)a.cols + (double)a.eps));
        }
        Phase q;
        const bool more = phase_of(segs, nseg, a.ns, k + 1, q);
        if (more) cb_load(cbf, a.lut[segs[q.j].g][q.s]);   // the next table's code words
        const uint32_t *rec = reinterpret_cast<const uint32_t *>(a.lut[sg.g][p.s] + a.rec_off) + ((size_t)sg.sl * a.rows8 + sg.ra) * 3;
        const uint16_t *gai = reinterpret_cast<const uint16_t *>(a.lut[sg.g][p.s] + 2 * CB_BYTES) + sg.ra;
        float *pout = a.part + (size_t)(sg.g * a.nsl + sg.sl) * a.rows;
        const bool first = p.s == 0, last = p.s + 1 == a.ns;
        const char *tb = reinterpret_cast<const char *>(T);
        const int nr = sg.rb - sg.ra;
        const int ntile = (nr + TR - 1) / TR;
        for (int t0 = 0; t0 < ntile; t0 += IT) {
            Rows nxt;
            if (t0 + IT < ntile) load_rows(nxt, rec, gai, t0 + IT, nr);   // the next rows in flight
            else if (more) {   // the next phase's first rows
                const Seg &s2 = segs[q.j];
                load_rows(nxt, reinterpret_cast<const uint32_t *>(a.lut[s2.g][q.s] + a.rec_off) + ((size_t)s2.sl * a.rows8 + s2.ra) * 3,
                          reinterpret_cast<const uint16_t *>(a.lut[s2.g][q.s] + 2 * CB_BYTES) + s2.ra, 0, s2.rb - s2.ra);
            }
            float prev[IT];
#pragma unroll
            for (int i = 0; i < IT; i++) {   // the stage-0 values of these rows, written by this same thread
                const int ir = (t0 + i) * TR + tid;
                prev[i] = (!first && ir < nr && sg.ra + ir < a.rows) ? pout[sg.ra + ir] : 0.f;
            }
            float sum[IT];
#pragma unroll
            for (int i = 0; i < IT; i++) sum[i] = lookup8(tb, cur.w0[i], cur.w1[i], cur.w2[i]);
#pragma unroll
            for (int i = 0; i < IT; i++) {
                const int ir = (t0 + i) * TR + tid;
                if (ir >= nr || sg.ra + ir >= a.rows) continue;
                float v = __fmul_rn(sum[i], cur.gn[i]);
                if (!first) v = __fadd_rn(prev[i], v);
                pout[sg.ra + ir] = last ? __fmul_rn(v, inv) : v;
            }
            cur = nxt;
        }
    }
    // -------------------------------------------------- every row's partials, once all CTAs wrote them
    __threadfence();
    __syncthreads();
    grid_barrier(a.sync, a.err);
    const int q8 = lane & 7, ri = lane >> 3;
    const int gw = (int)blockIdx.x * CW + warp, nw = (int)gridDim.x * CW;
    if (gw >= nw - a.xrows) gproj_warp(a, gw - (nw - a.xrows));   // the last warps: g_proj's rows
    const size_t gs = (size_t)a.nsl * a.rows;
    for (int r0 = 4 * gw; r0 < a.rows; r0 += 4 * nw) {   // 4 rows per warp, 8 lanes per row
        const int r = r0 + ri;
        float s0 = 0.f, s1 = 0.f;
        if (r < a.rows) {
            const float *pp = a.part + r;
            // lane q sums slices q, q + 8, ... in order: loads first (in flight together), then the adds
            constexpr int U = 8;
            for (int sl0 = q8; sl0 < a.nsl; sl0 += 8 * U) {
                float v0[U], v1[U];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int sl = sl0 + 8 * u;
                    v0[u] = sl < a.nsl ? __ldcg(pp + (size_t)sl * a.rows) : 0.f;
                    v1[u] = sl < a.nsl && a.ng == 2 ? __ldcg(pp + gs + (size_t)sl * a.rows) : 0.f;
                }
#pragma unroll
                for (int u = 0; u < U; u++) {
                    s0 += v0[u];
                    s1 += v1[u];
                }
            }
        }
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) {   // the 8 lanes of a row by a fixed butterfly
            s0 += __shfl_xor_sync(0xffffffffu, s0, o);
            s1 += __shfl_xor_sync(0xffffffffu, s1, o);
        }
        if (q8 == 0 && r < a.rows) {
            if (a.mode == 2)
                a.y[r] = __fmul_rn(gelu_erf(s0), s1);
            else if (a.mode == 1)
                a.y[r] = __fadd_rn(a.y[r], s0);
            else
                a.y[r] = s0;
        }
    }
}

// The stage re-laid for the table kernel: code words in the builder's fragment order (word
// (block, t, g) = codes 16 block + g and 16 block + g + 8 of dim t), the code words in natural
// order, gains (rows padded to a multiple of 8 with zeros), then record [sl][row] = bytes
// [12 sl, 12 sl + 12) of the row's DQV3 stream (padding rows zero).
__global__ void vq_lut_pack_kernel(const uint8_t *st, Layout L, int rows8, size_t rec_off, uint8_t *dst) {
    const int nsl = (int)(L.nidx_row / LGC);
    const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, nth = (size_t)gridDim.x * blockDim.x;
    const uint16_t *cb = reinterpret_cast<const uint16_t *>(st + L.cb_off);   // [code][4] f16
    uint32_t *cw = reinterpret_cast<uint32_t *>(dst);
    for (size_t e = tid; e < (size_t)LNC * 2; e += nth) {
        const int g = (int)(e & 7), t = (int)((e >> 3) & 3), blk = (int)(e >> 5);
        const int c = 16 * blk + g;
        cw[e] = (uint32_t)cb[(size_t)c * 4 + t] | ((uint32_t)cb[(size_t)(c + 8) * 4 + t] << 16);
    }
    for (size_t e = tid; e < (size_t)CB_BYTES; e += nth) dst[CB_BYTES + e] = st[L.cb_off + e];
    for (size_t e = tid; e < lut_gain_bytes(rows8); e += nth) dst[2 * CB_BYTES + e] = e < (size_t)L.rows * 2 ? st[L.gain_off + e] : 0;
    const size_t n = (size_t)nsl * rows8;
    for (size_t e = tid; e < n; e += nth) {
        const int r = (int)(e % rows8), sl = (int)(e / rows8);
        uint8_t *o = dst + rec_off + e * 12;
        if (r < L.rows) {
            const uint8_t *q = st + L.stream_off + (size_t)r * L.mrow + 12 * (size_t)sl;
#pragma unroll
            for (int j = 0; j < 12; j++) o[j] = q[j];
        } else {
#pragma unroll
            for (int j = 0; j < 12; j++) o[j] = 0;
        }
    }
}

int rows8_of(const Layout &L) { return (L.rows + 7) & ~7; }
size_t rec_off_of(const Layout &L) { return 2 * CB_BYTES + lut_gain_bytes(rows8_of(L)); }

size_t lut_smem() { return SM_REST + LMAXSEG * 32 * 4 + CW * 8 + LMAXSEG * sizeof(Seg) + 16; }

long long units_per_cta(const Layout &L, int ng) {
    const long long W = (long long)ng * (L.nidx_row / LGC) * (rows8_of(L) / 8);
    return (W + sm_count() - 1) / sm_count();
}

// segments a CTA walks at most: its units span ceil(per / Q) + 1 slices
bool lut_segments_ok(const Layout &L, int ng) {
    const long long Q = rows8_of(L) / 8;
    return (units_per_cta(L, ng) + Q - 1) / Q + 1 <= LMAXSEG;
}

}  // namespace

bool lut_ok(const Layout &L, int ns, int ng) {
    if ((long long)ng * (L.nidx_row / LGC) * (rows8_of(L) / 8) >= (1LL << 31)) return false;   // 32-bit units
    if (!(L.v3 && L.dim == 4 && L.nc == LNC && L.nbit == 12 && L.prow == 0 && L.nidx_row % LGC == 0)) return false;
    if (ns < 1 || ns > LMAXS || ng < 1 || ng > 2 || L.mrow * 2 != L.nidx_row * 3) return false;
    return lut_segments_ok(L, ng) && lut_smem() <= smem_optin_max();
}

size_t lut_bytes(const Layout &L) { return rec_off_of(L) + (L.nidx_row / LGC) * (size_t)rows8_of(L) * 12; }

size_t lut_part_bytes(const Layout &L, int ng) { return LUT_SYNC_BYTES + (size_t)ng * (L.nidx_row / LGC) * L.rows * 4; }

int lut_pack(const void *stage, const Layout &L, void *dst, cudaStream_t s) {
    if (!stage || !dst) return set_error("vq table pack: null pointer");
    if (((uintptr_t)dst & 15) != 0) return set_error("vq table pack: the destination must be 16-byte aligned");
    const size_t n = (L.nidx_row / LGC) * (size_t)rows8_of(L);
    const int blocks = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    const cudaError_t before = cudaGetLastError();   // an earlier call's error: not this launch's
    if (before != cudaSuccess) return cuda_fail("vq table pack: an earlier CUDA call had failed", before);
    vq_lut_pack_kernel<<<blocks > 128 ? blocks : 128, 256, 0, s>>>((const uint8_t *)stage, L, rows8_of(L),
                                                                  rec_off_of(L), (uint8_t *)dst);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail("vq table pack launch", e);
}

// y (=|+=) W RMSNorm?(x) (ng 1) or y = gelu_erf(W_gate xn) * (W_up xn) (ng 2); luts group-major
// (stages: the DQV3 payloads, read only for the optional g_proj); part >= lut_part_bytes(L, ng).
// xst / XL / xy: an optional g_proj computed by the finishing kernel (xrows <= 64, same input
// and norm).
int lut_gemv(const void *const *stages, const void *const *luts, int ns, int ng, const Layout &L, const float *x,
             const float *norm_w, float eps, float *y, int accumulate, float *part, const void *const *xst,
             const Layout *XL, float *xy, cudaStream_t s, int threads) {
    (void)stages;
    if (!lut_ok(L, ns, ng)) return set_error("vq table kernel: geometry not taken");
    if (ng == 2 && accumulate) return set_error("the paired gate/up form writes its output, it cannot accumulate");
    if (!x || !y || !part) return set_error("vq table kernel: null pointer");
    if (threads != 0 && threads != CT) return set_error("vq table kernel: %d consumer threads (0 or %d)", threads, CT);
    LutArgs a;
    memset(&a, 0, sizeof a);
    for (int g = 0; g < ng; g++)
        for (int q = 0; q < ns; q++) {
            const void *lt = luts[g * ns + q];
            if (!lt) return set_error("stage %d table words are null", g * ns + q);
            if ((uintptr_t)lt & 15) return set_error("vq table words must be 16-byte aligned");
            a.lut[g][q] = (const uint8_t *)lt;
        }
    a.ng = ng;
    a.ns = ns;
    a.rows = L.rows;
    a.rows8 = rows8_of(L);
    a.nsl = (int)(L.nidx_row / LGC);
    a.cols = L.cols;
    a.rec_off = rec_off_of(L);
    a.x = x;
    a.norm_w = norm_w;
    a.eps = eps;
    a.sync = reinterpret_cast<unsigned int *>(part);
    a.part = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(part) + LUT_SYNC_BYTES);
    a.mode = ng == 2 ? 2 : (accumulate ? 1 : 0);
    a.y = y;
    if (xst && XL && xy) {
        if (XL->rows > GX_MAX || XL->cols != L.cols || !XL->v3 || XL->dim != 4 ||
            XL->nbit != 12 || XL->prow)
            return set_error("vq table kernel: the extra matrix is not a small DQV3 matrix of the same input");
        a.xrows = XL->rows;
        a.xns = ns;
        for (int q = 0; q < ns; q++) a.xst[q] = (const uint8_t *)xst[q];
        a.XL = *XL;
        a.xy = xy;
    }
    a.err = device_error_ptr();
    const size_t smem = lut_smem();
    static size_t opted[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem > opted[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(vq_lut_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_fail("vq table kernel shared-memory opt-in", e);
        opted[dev & 63] = smem;
    }
    cudaError_t e = launch_pdl(vq_lut_kernel, dim3(sm_count()), dim3(NT), smem, s, a);
    return e == cudaSuccess ? 0 : cuda_fail("vq table kernel launch", e);
}

}  // namespace spk

using namespace spk;

extern "C" {

/* Bytes of one stage re-laid for spk_vq_lut_gemv (its code words, gains and index stream
 * slice-major); 0 when that kernel does not take the geometry (DQV3, dim 4, 4096 codes,
 * whole slices of 8 index groups). */
size_t spk_vq_lut_bytes(int dim, int nc, int rows, int cols, int v3) {
    if (dim <= 0 || nc <= 0 || rows <= 0 || cols <= 0 || cols % dim) return 0;
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    return lut_ok(L, 1, 1) ? lut_bytes(L) : 0;
}

/* Re-lay one stage (device DQV3 payload) into dst (device, 16-byte aligned, spk_vq_lut_bytes). */
int spk_vq_lut_pack(const void *stage, int dim, int nc, int rows, int cols, int v3, void *dst, void *stream) {
    if (!spk_vq_lut_bytes(dim, nc, rows, cols, v3)) return set_error("vq table kernel: geometry not taken");
    return lut_pack(stage, make_layout(dim, nc, rows, cols, v3), dst, (cudaStream_t)stream);
}

/* Device scratch spk_vq_lut_gemv needs for the per-slice partial sums. */
size_t spk_vq_lut_scratch_bytes(int ngroups, int dim, int nc, int rows, int cols, int v3) {
    if (!spk_vq_lut_bytes(dim, nc, rows, cols, v3) || ngroups < 1 || ngroups > 2) return 0;
    return lut_part_bytes(make_layout(dim, nc, rows, cols, v3), ngroups);
}

/* spk_vq_gemv's contract (ngroups 1: y (=|+=) sum_s gain_s W_s RMSNorm?(x); ngroups 2:
 * y = gelu_erf(W_gate xn) * (W_up xn)) through the table kernel: luts are the stages'
 * spk_vq_lut_pack words, group-major (they carry the code words and gains; stages, the DQV3
 * payloads, may be null); scratch is spk_vq_lut_scratch_bytes device bytes. Two launches,
 * no sync. */
int spk_vq_lut_gemv(const void *const *stages, const void *const *luts, int nstages, int ngroups, int dim, int nc,
                    int rows, int cols, int v3, const float *x, const float *norm_w, float eps, float *y,
                    int accumulate, void *scratch, void *stream) {
    if (!luts) return set_error("vq table kernel: null stage list");
    if (!spk_vq_lut_bytes(dim, nc, rows, cols, v3)) return set_error("vq table kernel: geometry not taken");
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    return lut_gemv(stages, luts, nstages, ngroups, L, x, norm_w, eps, y, accumulate, (float *)scratch, nullptr,
                    nullptr, nullptr, (cudaStream_t)stream, 0);
}

/* spk_vq_lut_gemv with the table kernel's consumer thread count stated (0: the default; the
 * kernel runs 512 consumer threads plus one producer warp), as vqg_gemv_t takes one for the
 * reference's kernels. */
int spk_vq_lut_gemv_t(const void *const *stages, const void *const *luts, int nstages, int ngroups, int dim, int nc,
                      int rows, int cols, int v3, const float *x, const float *norm_w, float eps, float *y,
                      int accumulate, void *scratch, int threads, void *stream) {
    if (!luts) return set_error("vq table kernel: null stage list");
    if (threads != 0 && threads != CT) return set_error("vq table kernel: threads 0 or %d", CT);
    if (!spk_vq_lut_bytes(dim, nc, rows, cols, v3)) return set_error("vq table kernel: geometry not taken");
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    return lut_gemv(stages, luts, nstages, ngroups, L, x, norm_w, eps, y, accumulate, (float *)scratch, nullptr,
                    nullptr, nullptr, (cudaStream_t)stream, threads);
}

}  // extern "C"
