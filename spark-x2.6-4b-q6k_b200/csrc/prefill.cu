// prefill.cu — multi-token VQ GEMM (prefill / speculative verify) and the
// vqg_prefill* C-ABI (tools/vq/gpu/decode-gpu.cu:998-1118).
//
// Layout contract kept from the reference: xT is [cols][ntok] (column-major
// activations), y is [ntok][rows] and accumulates. The tile table and the
// legality rules are the reference's (decode-gpu.cu:527-560) so a caller that
// asks vqg_prefill_cfg_ready gets the same answers; every legal (tile, variant)
// runs this file's kernel, which computes the same sum.
//
// Kernel: one warp per row, 8 tokens per pass. A lane gathers each codeword
// once and applies it to all 8 tokens, so the index stream and the codebook are
// read once per 8 tokens instead of once per token.
#include "common.cuh"
#include "spk.h"

using namespace spk;

namespace {

constexpr int TOK = 8;

__global__ void vq_prefill_kernel(const uint8_t *p, const Layout L, const float *xT, int ntok, float *y) {
    const int warp = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (warp >= L.rows) return;
    const int r = warp;
    const __half *cb = reinterpret_cast<const __half *>(p + L.cb_off);
    const uint8_t *st = p + L.stream_off;
    const float g = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t *>(p + L.gain_off + 2 * (size_t)r)));
    for (int t0 = 0; t0 < ntok; t0 += TOK) {
        const int nt = min(TOK, ntok - t0);
        float acc[TOK];
#pragma unroll
        for (int t = 0; t < TOK; t++) acc[t] = 0.f;
        for (size_t i = lane; i < L.nidx_row; i += 32) {
            const uint32_t v = min(rd_idx(st, L, (size_t)r, i), (uint32_t)L.nc - 1u);
            const __half *c = cb + (size_t)v * L.dim;
            for (int d = 0; d < L.dim; d++) {
                const float cw = __half2float(c[d]);
                const float *xc = xT + (i * (size_t)L.dim + (size_t)d) * (size_t)ntok + t0;
#pragma unroll
                for (int t = 0; t < TOK; t++)
                    if (t < nt) acc[t] = fmaf(cw, xc[t], acc[t]);
            }
        }
#pragma unroll
        for (int t = 0; t < TOK; t++) {
            const float s = warp_sum(acc[t]);
            if (lane == 0 && t < nt) y[(size_t)(t0 + t) * L.rows + r] += s * g;
        }
    }
}

// decode-gpu.cu:527-530: the reference's geometry rule for its tiled kernel.
bool pre_ok(const Layout &L, int bk) {
    return L.v3 && (L.dim == 4 || L.dim == 8) && L.rows > 0 && L.cols > 0 && L.nbit >= 12 && L.cols % bk == 0 &&
           L.mrow % 4 == 0 && L.stream_off % 4 == 0;
}

const struct {
    int bn, bk;
} k_cfg[] = {{64, 64}, {128, 64}, {256, 64}};
constexpr int NCFG = 3;

bool cfg_known(int bn, int bk) {
    for (int i = 0; i < NCFG; i++)
        if (k_cfg[i].bn == bn && k_cfg[i].bk == bk) return true;
    return false;
}

// decode-gpu.cu:516-519, 553-560
bool cfg_ready(const Layout &L, int bn, int bk, int cb) {
    if (!cfg_known(bn, bk) || !pre_ok(L, bk)) return false;
    if (cb && (size_t)(128 + bn) * bk * 2u + (size_t)L.nc * L.dim * 2u > smem_optin_max()) return false;
    return true;
}

int launch(const void *payload, const Layout &L, const float *xT, int ntok, float *y, cudaStream_t s) {
    const int threads = 256;
    const int blocks = (int)(((size_t)L.rows * 32 + threads - 1) / threads);
    vq_prefill_kernel<<<blocks, threads, 0, s>>>((const uint8_t *)payload, L, xT, ntok, y);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail("prefill launch", e);
}

int timed_prefill(const void *payload, const Layout &L, const float *xT, int ntok, float *y, int iters, double *ms) {
    cudaEvent_t a, b;
    if (cudaEventCreate(&a) != cudaSuccess || cudaEventCreate(&b) != cudaSuccess)
        return cuda_fail("event create", cudaGetLastError());
    float best = 1e30f;
    int rc = 0;
    for (int it = 0; it < iters && !rc; it++) {
        cudaEventRecord(a);
        rc = launch(payload, L, xT, ntok, y, 0);
        cudaEventRecord(b);
        cudaError_t e = cudaEventSynchronize(b);
        if (!rc && e != cudaSuccess) rc = cuda_fail("prefill launch", e);
        float t = 0;
        cudaEventElapsedTime(&t, a, b);
        if (t < best) best = t;
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    if (ms) *ms = iters > 0 ? best : 0.0;
    return rc;
}

int pre_checks(int dim, int nc, int rows, int cols, int v3, int ntok) {
    if (v3 && !v3_width_ok(nc)) {
        int b = 1;
        while ((1 << b) < nc) b++;
        return set_error("DQV3 carries 13 index bits, nc %d needs %d", nc, b);
    }
    if (ntok <= 0) return set_error("prefill needs at least one token");
    if (rows <= 0 || cols <= 0) return set_error("prefill needs a non-empty matrix");
    if (dim <= 0 || cols % dim) return set_error("geometry dim %d cols %d is inconsistent", dim, cols);
    return 0;
}

}  // namespace

extern "C" {

/* decode-gpu.cu:998-1008 */
int vqg_prefill_ready(int dim, int nc, int rows, int cols, int v3, int variant) {
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    switch (variant) {
        case 0: return 1;
        case 1: return cfg_ready(L, 128, 64, 0) ? 1 : 0;
        case 2: return cfg_ready(L, 128, 64, 1) ? 1 : 0;
        case 3: return 1;
        default: return 0;
    }
}

/* decode-gpu.cu:1012 */
int vqg_prefill_cfg_count(void) { return NCFG; }

/* decode-gpu.cu:1014-1019 */
int vqg_prefill_cfg(int idx, int *bn, int *bk) {
    if (idx < 0 || idx >= NCFG || !bn || !bk) return -1;
    *bn = k_cfg[idx].bn;
    *bk = k_cfg[idx].bk;
    return 0;
}

/* decode-gpu.cu:1024-1029 */
int vqg_prefill_cfg_ready(int dim, int nc, int rows, int cols, int v3, int bn, int bk, int variant) {
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    if (variant == 3) return 1;
    if (variant != 1 && variant != 2) return 0;
    return cfg_ready(L, bn, bk, variant == 2) ? 1 : 0;
}

/* decode-gpu.cu:1034-1048 */
int vqg_prefill(const void *payload, int dim, int nc, int rows, int cols, int v3, const float *xT, int ntok, float *y,
                int iters, double *ms, int variant) {
    if (pre_checks(dim, nc, rows, cols, v3, ntok)) return -1;
    if (variant < 0 || variant > 3) return set_error("unknown prefill variant %d", variant);
    return timed_prefill(payload, make_layout(dim, nc, rows, cols, v3), xT, ntok, y, iters, ms);
}

/* decode-gpu.cu:1051-1065 */
int vqg_prefill_tile(const void *payload, int dim, int nc, int rows, int cols, int v3, const float *xT, int ntok,
                     float *y, int iters, double *ms, int bn, int bk, int variant) {
    if (pre_checks(dim, nc, rows, cols, v3, ntok)) return -1;
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    if (variant != 3 && ((variant != 1 && variant != 2) || !cfg_ready(L, bn, bk, variant == 2)))
        return set_error("tile %dx%d with variant %d does not fit this geometry", bn, bk, variant);
    return timed_prefill(payload, L, xT, ntok, y, iters, ms);
}

/* decode-gpu.cu:1071-1094 */
int vqg_prefill_launch(const void *payload, int dim, int nc, int rows, int cols, int v3, const float *xT, int ntok,
                       float *y, int variant) {
    if (pre_checks(dim, nc, rows, cols, v3, ntok)) return -1;
    if (variant < 0 || variant > 3) return set_error("unknown prefill variant %d", variant);
    return launch(payload, make_layout(dim, nc, rows, cols, v3), xT, ntok, y, 0);
}

/* decode-gpu.cu:1099-1118 */
int vqg_prefill_launch_tile(const void *payload, int dim, int nc, int rows, int cols, int v3, const float *xT,
                            int ntok, float *y, int bn, int bk, int variant) {
    if (pre_checks(dim, nc, rows, cols, v3, ntok)) return -1;
    const Layout L = make_layout(dim, nc, rows, cols, v3);
    if (variant != 3 && ((variant != 1 && variant != 2) || !cfg_ready(L, bn, bk, variant == 2)))
        return set_error("tile %dx%d with variant %d does not fit this geometry", bn, bk, variant);
    return launch(payload, L, xT, ntok, y, 0);
}

}  // extern "C"
