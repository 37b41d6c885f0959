// vq_lut16.cu — the decode step's gate/up pair as shared-memory table look-ups over index
// streams re-laid as 16-byte words of u16 table offsets (internal to the model, no C-ABI entry;
// the C-ABI's table kernel and the tensor-core GEMM share vq_lut.cu's 12-byte records). It is
// kept for the pair because it measures faster there (35-38 us against 43 us for vq_lut.cu's
// kernel, 2 x 10240 x 2560, 2 stages).
//
// The GEMV over residual-VQ stages as shared-memory table look-ups.
//
// What it computes is spk_vq_gemv's (tools/vq-format/src/lib.rs:215-228 Stage::dot_row,
// decode-gpu.cu:267-301 gemv_v3blk_kernel, summed over stages as vq-model-gpu.cu:651-660):
//   y[r] (+)= sum_s gain_s[r] * sum_i sum_d cb_s[idx_s(r,i)][d] * x[4i+d]
// for DQV3 stages of dim 4 with 4096 codes (12-bit row-local indices, no 13th-bit plane).
//
// The B200 design. The VQ GEMV is bound by random code-word gathers from shared memory,
// not by HBM. With the activations of a fixed column run in each lane's registers (vq.cu)
// every index costs an 8-byte random gather (~5 shared wavefronts per 32 lanes), two
// conversions and four dependent FMAs, and the registers the activations hold cap the
// warps an SM can keep gathering. Here:
//   * the column groups i (4 columns each) are cut into slices of 8; for one slice and one
//     stage a CTA builds the table T[jj][c] = cb_s[c] . x[4(8*sl + jj) .. +4] for all 4096
//     codes c and the slice's 8 groups jj (128 KB of f32 in shared memory). An index then
//     costs one 4-byte shared load (~3.5 wavefronts per 32 random lanes) and one add, and
//     no activation lives in a register;
//   * the index streams are re-laid once at load, slice-major: a row's 8 indices of slice sl
//     (bytes [12 sl, 12 sl + 12) of its DQV3 row stream) become one 16-byte word at [sl][row]
//     of 8 u16 byte offsets into the table (4 * idx), so a look-up is one mask or shift, a
//     shared load at an immediate table offset and an add, and 32 lanes on 32 consecutive
//     rows load 512 coalesced bytes straight into registers, a chunk of rows ahead;
//   * the work, (group, slice, row) in that order, is cut evenly over one CTA per SM; a CTA
//     walks its contiguous range segment by segment (a segment: one slice's run of rows),
//     building the table once per segment and stage; a row's value for the slice (gains
//     applied, stages summed) goes to a partial buffer [group][slice][row];
//   * a second kernel sums each row's partials in slice order (the same order on every
//     run) and applies the epilogue: store, residual accumulate, or gelu_erf(gate) * up;
//     for q_k_v_proj its extra CTAs also compute g_proj's rows from the stage payloads.
#include "common.cuh"
#include "spk.h"

namespace spk {
namespace w16 {

namespace {

constexpr int LGC = 8;           // column groups per slice
constexpr int LNC = 4096;        // codes
constexpr int LMAXS = 2;         // stages
constexpr int FR = 32;           // rows per CTA of the finishing kernel
constexpr int FT = 512;          // threads of the finishing kernel
constexpr int FQ = FT / FR;      // slice lanes per row there
constexpr int GX_MAX = 64;       // g_proj rows the finishing kernel takes
constexpr int LMAXSEG = 8;       // segments a CTA of the table kernel may walk

struct LutArgs {
    const uint4 *idx[2][LMAXS];      // re-laid index words [nsl][rows], 8 u16 table offsets each
    const uint2 *cb[2][LMAXS];        // code words, 4 x f16
    const uint16_t *gain[2][LMAXS];   // f16 row gains
    int ng, ns, rows, nsl, cols;
    const float *x;
    const float *norm_w;              // optional RMSNorm weight
    float eps;
    float *part;                      // [ng][nsl][rows]
    int srow_cap;                     // floats of the stage-0 row buffer
};

struct FinArgs {
    const float *part;
    int ng, nsl, rows;
    int mode;                         // 0 store, 1 accumulate, 2 gelu_erf(group 0) * group 1
    float *y;
    // g_proj (optional): rows of a second matrix of the same input, one CTA per row
    int xrows, xns;
    const uint8_t *xst[LMAXS];
    Layout XL;
    const float *x;
    const float *norm_w;
    float eps;
    float *xy;
};

__device__ __forceinline__ float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ float gelu_erf(float g) {
    // model.rs:253-258: 0.5*x*(1 + erf(x/sqrt2)), erf in f64
    const double e = erf((double)g * 0.70710678118654752440);
    return __fmul_rn(__fmul_rn(0.5f, g), __fadd_rn(1.0f, (float)e));
}

// RMSNorm scale with the sum of squares in f64 (model.rs:236-245); every CTA sums in the
// same order and gets the same scale.
__device__ float rms_inv(const float *x, int n, float eps, double *red) {
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

__device__ __forceinline__ uint4 ldg_nc4(const uint4 *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint16_t ldg_nc16(const uint16_t *p) {
    uint16_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

// The words and gains of rows r0 + (k0 + c) * NT, c < CH, of one slice and stage.
template <int NT, int CH>
__device__ __forceinline__ void load_chunk(uint4 (&w)[CH], uint16_t (&gn)[CH], const uint4 *ip, const uint16_t *gp,
                                           int r0, int k0, int nk) {
#pragma unroll
    for (int c = 0; c < CH; c++) {
        if (k0 + c < nk) {
            const int r = r0 + (k0 + c) * NT;
            w[c] = ldg_nc4(ip + r);
            gn[c] = ldg_nc16(gp + r);
        }
    }
}

// A stage's 4096 code words (8-byte aligned in the payload) into shared memory by cp.async.
template <int NT>
__device__ __forceinline__ void prefetch_cb(uint2 *dst, const uint2 *src) {
#pragma unroll
    for (int c = threadIdx.x; c < LNC; c += NT)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst + c)), "l"(src + c) : "memory");
    asm volatile("cp.async.commit_group;" ::: "memory");
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

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

// The index words and gains one phase (group g, stage s, slice sl, rows [ra, rb)) reads.
__device__ __forceinline__ void prefetch_phase(const LutArgs &a, int g, int s, int sl, int ra, int rb) {
    l2_prefetch(a.idx[g][s] + (size_t)sl * a.rows + ra, (size_t)(rb - ra) * 16);
    l2_prefetch(a.gain[g][s] + ra, (size_t)(rb - ra) * 2);
}

// Sum over a row's 8 indices of one slice: T[jj][idx_jj], the word holding 4 * idx_jj in
// u16 jj (little-endian).
__device__ __forceinline__ float lookup8(const float *T, const uint4 &w) {
    const char *t = reinterpret_cast<const char *>(T);
    constexpr int S = LNC * 4;   // bytes per jj table
    const float p0 = *reinterpret_cast<const float *>(t + (w.x & 0xFFFFu));
    const float p1 = *reinterpret_cast<const float *>(t + S + (w.x >> 16));
    const float p2 = *reinterpret_cast<const float *>(t + 2 * S + (w.y & 0xFFFFu));
    const float p3 = *reinterpret_cast<const float *>(t + 3 * S + (w.y >> 16));
    const float p4 = *reinterpret_cast<const float *>(t + 4 * S + (w.z & 0xFFFFu));
    const float p5 = *reinterpret_cast<const float *>(t + 5 * S + (w.z >> 16));
    const float p6 = *reinterpret_cast<const float *>(t + 6 * S + (w.w & 0xFFFFu));
    const float p7 = *reinterpret_cast<const float *>(t + 7 * S + (w.w >> 16));
    return ((p0 + p1) + (p2 + p3)) + ((p4 + p5) + (p6 + p7));
}

template <int NT, int CH>
__global__ void __launch_bounds__(NT, 1) vq_lut_kernel(const LutArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    float *T = reinterpret_cast<float *>(smem);         // [LGC][LNC]
    uint2 *cbs = reinterpret_cast<uint2 *>(T + LGC * LNC);   // [LNC] the stage's code words
    float *srow = reinterpret_cast<float *>(cbs + LNC);      // [srow_cap]
    float *xs = srow + a.srow_cap;                       // [LMAXSEG][32] each segment's activations
    double *red = reinterpret_cast<double *>(xs + LMAXSEG * 32);   // [NT / 32]
    const int tid = threadIdx.x;
    // unit indices (group, slice, row) fit in 32 bits (the host checks), so no 64-bit division
    const int R = a.rows, nsl = a.nsl;
    const int per_g = nsl * R, W = per_g * a.ng;
    const int u0 = (int)((long long)W * blockIdx.x / gridDim.x), u1 = (int)((long long)W * (blockIdx.x + 1) / gridDim.x);
    pdl_trigger();
    if (u0 < u1) {   // weights: before the wait
        prefetch_cb<NT>(cbs, a.cb[u0 / per_g][0]);
        if (tid == 0) {
            const int r0 = u0 % per_g;
            const int sl0 = r0 / R, ra0 = r0 % R;
            prefetch_phase(a, u0 / per_g, 0, sl0, ra0, min(R, ra0 + (u1 - u0)));
        }
    }
    bool have_x = false;
    float inv = 1.0f;
    for (int u = u0, seg = 0; u < u1; seg++) {
        const int g = u / per_g;
        const int rem = u - g * per_g;
        const int sl = rem / R, ra = rem - sl * R;
        const int rb = min(R, ra + (u1 - u));
        const int nr = rb - ra;
        const int nk = nr > tid ? (nr - tid + NT - 1) / NT : 0;   // this thread's rows ra + tid + k NT
        for (int s = 0; s < a.ns; s++) {
            const uint4 *ip = a.idx[g][s] + (size_t)sl * R;
            const uint16_t *gp = a.gain[g][s];
            uint4 w[CH];
            uint16_t gn[CH];
            load_chunk<NT, CH>(w, gn, ip, gp, ra + tid, 0, nk);   // weights: before the wait
            if (!have_x) {
                // every segment's 32 activations at once: thread t takes segment t / 32
                pdl_wait();
                if (a.norm_w) inv = rms_inv(a.x, a.cols, a.eps, red);
                if (tid < LMAXSEG * 32) {
                    int v = u0;
                    for (int k = 0; v < u1 && k < tid / 32; k++) v += min(R - v % per_g % R, u1 - v);
                    if (v < u1) {
                        const int c = 32 * (v % per_g / R) + (tid & 31);
                        float xv = a.x[c];
                        if (a.norm_w) xv = __fmul_rn(__fmul_rn(xv, inv), a.norm_w[c]);
                        xs[tid] = xv;
                    }
                }
                have_x = true;
            }
            cp_async_wait_all();
            __syncthreads();   // the previous table's readers are done; xs and the code words are in
            {
                const float4 *x4 = reinterpret_cast<const float4 *>(xs + 32 * seg);
                float4 xv[LGC];
#pragma unroll
                for (int jj = 0; jj < LGC; jj++) xv[jj] = x4[jj];
#pragma unroll 2
                for (int c = tid; c < LNC; c += NT) {
                    const uint2 q = cbs[c];
                    const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&q.x));
                    const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&q.y));
#pragma unroll
                    for (int jj = 0; jj < LGC; jj++)
                        T[jj * LNC + c] = fmaf(hi.y, xv[jj].w, fmaf(hi.x, xv[jj].z, fmaf(lo.y, xv[jj].y, lo.x * xv[jj].x)));
                }
            }
            __syncthreads();
            // the next stage's (or segment's) code words, while this one's look-ups run
            if (s + 1 < a.ns) {
                prefetch_cb<NT>(cbs, a.cb[g][s + 1]);
                if (tid == 0) prefetch_phase(a, g, s + 1, sl, ra, rb);
            } else if (u + nr < u1) {
                const int un = u + nr, rn = un % per_g;
                const int gn2 = un / per_g, sln = rn / R, ran = rn % R;
                prefetch_cb<NT>(cbs, a.cb[gn2][0]);
                if (tid == 0) prefetch_phase(a, gn2, 0, sln, ran, min(R, ran + (u1 - un)));
            }
            float *pout = a.part + (size_t)(g * nsl + sl) * R;
            const bool last = s + 1 == a.ns;
            for (int k0 = 0; k0 < nk; k0 += CH) {
                uint4 wn[CH];
                uint16_t gnn[CH];
                if (k0 + CH < nk) load_chunk<NT, CH>(wn, gnn, ip, gp, ra + tid, k0 + CH, nk);
#pragma unroll
                for (int c = 0; c < CH; c++) {
                    const int k = k0 + c;
                    if (k < nk) {
                        const int i = tid + k * NT;   // row ra + i
                        const float v = __fmul_rn(lookup8(T, w[c]), h2f_bits(gn[c]));
                        if (!last)
                            srow[i] = s == 0 ? v : __fadd_rn(srow[i], v);
                        else
                            pout[ra + i] = s == 0 ? v : __fadd_rn(srow[i], v);
                    }
                }
#pragma unroll
                for (int c = 0; c < CH; c++) {
                    w[c] = wn[c];
                    gn[c] = gnn[c];
                }
            }
        }
        u += nr;
    }
    cp_async_wait_all();
    if (!have_x) pdl_wait();
}

// One g_proj row (the stage payloads, read through L1): sum_s gain_s[row] * W_s[row] . xn.
__device__ void gproj_row(const FinArgs &a, int row) {
    __shared__ double dred[FT / 32];
    __shared__ float fred[LMAXS][FT / 32];
    const Layout &L = a.XL;
    float inv = 1.0f;
    if (a.norm_w) inv = rms_inv(a.x, L.cols, a.eps, dred);
    for (int s = 0; s < a.xns; s++) {
        const uint8_t *rowp = a.xst[s] + L.stream_off + (size_t)row * L.mrow;
        const uint2 *cb = reinterpret_cast<const uint2 *>(a.xst[s] + L.cb_off);
        float t = 0.f;
        for (int i = threadIdx.x; i < (int)L.nidx_row; i += FT) {
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
        if ((threadIdx.x & 31) == 0) fred[s][threadIdx.x >> 5] = t;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float o = 0.f;
        for (int s = 0; s < a.xns; s++) {
            float t = 0.f;
            for (int k = 0; k < FT / 32; k++) t += fred[s][k];
            const uint16_t gh = *reinterpret_cast<const uint16_t *>(a.xst[s] + L.gain_off + 2 * (size_t)row);
            o = __fadd_rn(o, __fmul_rn(t, h2f_bits(gh)));
        }
        a.xy[row] = o;
    }
}

__global__ void __launch_bounds__(FT) vq_lut_finish_kernel(const FinArgs a) {
    __shared__ float red[2][FQ][FR + 1];
    pdl_trigger();
    pdl_wait();
    const int nrb = (a.rows + FR - 1) / FR;
    if ((int)blockIdx.x >= nrb) {
        gproj_row(a, blockIdx.x - nrb);
        return;
    }
    const int ri = threadIdx.x % FR, q = threadIdx.x / FR;
    const int r = blockIdx.x * FR + ri;
    float s0 = 0.f, s1 = 0.f;   // both groups' loads in flight together
    if (r < a.rows) {
        const float *p = a.part + r;
        const size_t gs = (size_t)a.nsl * a.rows;
#pragma unroll 4
        for (int sl = q; sl < a.nsl; sl += FQ) {
            s0 += p[(size_t)sl * a.rows];
            if (a.ng == 2) s1 += p[gs + (size_t)sl * a.rows];
        }
    }
    red[0][q][ri] = s0;
    red[1][q][ri] = s1;
    __syncthreads();
    if (q == 0 && r < a.rows) {
        float t[2] = {0.f, 0.f};
        for (int g = 0; g < a.ng; g++)
            for (int k = 0; k < FQ; k++) t[g] += red[g][k][ri];
        if (a.mode == 2)
            a.y[r] = __fmul_rn(gelu_erf(t[0]), t[1]);
        else if (a.mode == 1)
            a.y[r] = __fadd_rn(a.y[r], t[0]);
        else
            a.y[r] = t[0];
    }
}

// word [sl][row] = the 8 indices at bytes [12 sl, 12 sl + 12) of row's DQV3 stream, each
// as the u16 byte offset 4 * idx into its table
__global__ void vq_lut_pack_kernel(const uint8_t *st, Layout L, uint4 *dst) {
    const int nsl = (int)(L.nidx_row / LGC);
    const size_t n = (size_t)nsl * L.rows;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(e % L.rows), sl = (int)(e / L.rows);
        const uint8_t *q = st + L.stream_off + (size_t)r * L.mrow + 12 * (size_t)sl;
        uint32_t o[4];
#pragma unroll
        for (int h = 0; h < 4; h++) {   // indices 2h, 2h + 1: bytes 3h .. 3h + 2
            const uint32_t b = (uint32_t)q[3 * h] | ((uint32_t)q[3 * h + 1] << 8) | ((uint32_t)q[3 * h + 2] << 16);
            o[h] = ((b & 0xFFFu) << 2) | (((b >> 12) & 0xFFFu) << 18);
        }
        dst[e] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

size_t lut_smem(int srow_cap) {
    return (size_t)LGC * LNC * 4 + (size_t)LNC * 8 + (size_t)srow_cap * 4 + LMAXSEG * 32 * 4 + (1024 / 32) * 8;
}

// segments a CTA walks at most: its units span ceil(per / rows) + 1 slices
bool lut_segments_ok(const Layout &L, int ng) {
    const long long W = (long long)ng * (L.nidx_row / LGC) * L.rows;
    const long long per = (W + sm_count() - 1) / sm_count();
    return (per + L.rows - 1) / L.rows + 1 <= LMAXSEG;
}

int lut_srow_cap(const Layout &L, int ns, int ng) {
    if (ns < 2) return 0;
    const long long W = (long long)ng * (L.nidx_row / LGC) * L.rows;
    const long long per = (W + sm_count() - 1) / sm_count();
    const long long cap = per < L.rows ? per : L.rows;
    return (int)((cap + 3) & ~3LL);
}

}  // namespace

bool ok(const Layout &L, int ns, int ng) {
    if ((long long)ng * (long long)L.nidx_row * L.rows >= (1LL << 31)) return false;   // 32-bit unit indices
    if (!(L.v3 && L.dim == 4 && L.nc == LNC && L.nbit == 12 && L.prow == 0 && L.nidx_row % LGC == 0)) return false;
    if (ns < 1 || ns > LMAXS || ng < 1 || ng > 2 || L.mrow * 2 != L.nidx_row * 3) return false;
    return lut_segments_ok(L, ng) && lut_smem(lut_srow_cap(L, ns, ng)) <= smem_optin_max();
}

size_t bytes(const Layout &L) { return (L.nidx_row / LGC) * (size_t)L.rows * 16; }

size_t part_bytes(const Layout &L, int ng) { return (size_t)ng * (L.nidx_row / LGC) * L.rows * 4; }

int pack(const void *stage, const Layout &L, void *dst, cudaStream_t s) {
    if (!stage || !dst) return set_error("vq table pack: null pointer");
    if (((uintptr_t)dst & 15) != 0) return set_error("vq table pack: the destination must be 16-byte aligned");
    const size_t n = bytes(L) / 16;
    const int blocks = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    vq_lut_pack_kernel<<<blocks, 256, 0, s>>>((const uint8_t *)stage, L, (uint4 *)dst);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail("vq table pack launch", e);
}

// y (=|+=) W RMSNorm?(x) (ng 1) or y = gelu_erf(W_gate xn) * (W_up xn) (ng 2); stages /
// luts group-major; part >= lut_part_bytes(L, ng). xst / XL / xy: an optional g_proj
// computed by the finishing kernel (xrows <= 64, same input and norm).
int gemv(const void *const *stages, const void *const *luts, int ns, int ng, const Layout &L, const float *x,
             const float *norm_w, float eps, float *y, int accumulate, float *part, const void *const *xst,
             const Layout *XL, float *xy, cudaStream_t s, int threads) {
    if (!ok(L, ns, ng)) return set_error("vq table kernel: geometry not taken");
    if (ng == 2 && accumulate) return set_error("the paired gate/up form writes its output, it cannot accumulate");
    if (!x || !y || !part) return set_error("vq table kernel: null pointer");
    LutArgs a;
    memset(&a, 0, sizeof a);
    for (int g = 0; g < ng; g++)
        for (int q = 0; q < ns; q++) {
            const uint8_t *st = (const uint8_t *)stages[g * ns + q];
            if (!st || !luts[g * ns + q]) return set_error("stage %d payload or table words are null", g * ns + q);
            if (((uintptr_t)st + L.cb_off) & 7) return set_error("stage codebook is not 8-byte aligned");
            if ((uintptr_t)luts[g * ns + q] & 15) return set_error("vq table words must be 16-byte aligned");
            a.idx[g][q] = (const uint4 *)luts[g * ns + q];
            a.cb[g][q] = (const uint2 *)(st + L.cb_off);
            a.gain[g][q] = (const uint16_t *)(st + L.gain_off);
        }
    a.ng = ng;
    a.ns = ns;
    a.rows = L.rows;
    a.nsl = (int)(L.nidx_row / LGC);
    a.cols = L.cols;
    a.x = x;
    a.norm_w = norm_w;
    a.eps = eps;
    a.part = part;
    a.srow_cap = lut_srow_cap(L, ns, ng);
    const size_t smem = lut_smem(a.srow_cap);
    const int nt = threads == 1024 ? 1024 : 512;
    auto k = nt == 1024 ? vq_lut_kernel<1024, 2> : vq_lut_kernel<512, 4>;
    static size_t opted[2][64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem > opted[nt == 1024][dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_fail("vq table kernel shared-memory opt-in", e);
        opted[nt == 1024][dev & 63] = smem;
    }
    cudaError_t e = launch_pdl(k, dim3(sm_count()), dim3(nt), smem, s, a);
    if (e != cudaSuccess) return cuda_fail("vq table kernel launch", e);

    FinArgs f;
    memset(&f, 0, sizeof f);
    f.part = part;
    f.ng = ng;
    f.nsl = a.nsl;
    f.rows = L.rows;
    f.mode = ng == 2 ? 2 : (accumulate ? 1 : 0);
    f.y = y;
    if (xst && XL && xy) {
        if (XL->rows > GX_MAX || XL->cols != L.cols || !XL->v3 || XL->dim != 4 || XL->nbit != 12 || XL->prow)
            return set_error("vq table kernel: the extra matrix is not a small DQV3 matrix of the same input");
        f.xrows = XL->rows;
        f.xns = ns;
        for (int q = 0; q < ns; q++) f.xst[q] = (const uint8_t *)xst[q];
        f.XL = *XL;
        f.x = x;
        f.norm_w = norm_w;
        f.eps = eps;
        f.xy = xy;
    }
    const int grid = (L.rows + FR - 1) / FR + f.xrows;
    e = launch_pdl(vq_lut_finish_kernel, dim3(grid), dim3(FT), 0, s, f);
    return e == cudaSuccess ? 0 : cuda_fail("vq table finish launch", e);
}

}  // namespace w16
}  // namespace spk

using namespace spk;

extern "C" {

/* Bytes of one stage's index stream re-laid for spk_vq_lut16_gemv (16-byte words of u16 table
 * offsets, one per row and slice of 8 index groups); 0 when the kernel does not take the
 * geometry (DQV3, dim 4, 4096 codes, 12-bit, whole slices). */
size_t spk_vq_lut16_bytes(int dim, int nc, int rows, int cols, int v3) {
    if (dim <= 0 || nc <= 0 || rows <= 0 || cols <= 0 || cols % dim) return 0;
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    return w16::ok(L, 1, 1) ? w16::bytes(L) : 0;
}

/* Re-lay one stage's index stream (device DQV3 payload) into dst (device, 16-byte aligned). */
int spk_vq_lut16_pack(const void *stage, int dim, int nc, int rows, int cols, int v3, void *dst, void *stream) {
    if (!spk_vq_lut16_bytes(dim, nc, rows, cols, v3)) return set_error("vq table kernel: geometry not taken");
    return w16::pack(stage, make_layout(dim, nc, rows, cols, v3), dst, (cudaStream_t)stream);
}

/* Device scratch spk_vq_lut16_gemv needs for the per-slice partial sums. */
size_t spk_vq_lut16_scratch_bytes(int ngroups, int dim, int nc, int rows, int cols, int v3) {
    if (!spk_vq_lut16_bytes(dim, nc, rows, cols, v3) || ngroups < 1 || ngroups > 2) return 0;
    return w16::part_bytes(make_layout(dim, nc, rows, cols, v3), ngroups);
}

/* spk_vq_gemv's contract through the decode step's gate/up-pair table kernel: stages are the
 * DQV3 payloads (code words and gains are read there), luts their spk_vq_lut16_pack words, both
 * group-major; scratch is spk_vq_lut16_scratch_bytes device bytes. Two launches, no sync. */
int spk_vq_lut16_gemv(const void *const *stages, const void *const *luts, int nstages, int ngroups, int dim, int nc,
                      int rows, int cols, int v3, const float *x, const float *norm_w, float eps, float *y,
                      int accumulate, void *scratch, void *stream) {
    if (!stages || !luts) return set_error("vq table kernel: null stage list");
    if (!spk_vq_lut16_bytes(dim, nc, rows, cols, v3)) return set_error("vq table kernel: geometry not taken");
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    return w16::gemv(stages, luts, nstages, ngroups, L, x, norm_w, eps, y, accumulate, (float *)scratch, nullptr,
                     nullptr, nullptr, (cudaStream_t)stream, 0);
}

}  // extern "C"
