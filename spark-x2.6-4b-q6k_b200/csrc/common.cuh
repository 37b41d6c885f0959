// common.cuh — shared host/device helpers for libspk (sm_100a only).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libspk is built for sm_100a only"
#endif

namespace spk {

// ---------------------------------------------------------------- errors ---
// Thread-local last-error string. The reference keeps one process-global
// buffer (decode-gpu.cu:21-28); a thread-local one gives the same answer to a
// single-threaded caller and does not race for a multi-threaded one.
const char *last_error();
int set_error(const char *fmt, ...);
int cuda_fail(const char *what, cudaError_t e);

// Device-side error word. Kernels never trap: a bounded wait that runs out
// sets a code here and the kernel returns; the host reads it with check_device_error().
enum : int { DEV_OK = 0, DEV_WAIT_TIMEOUT = 1, DEV_BAD_INDEX = 2, DEV_PEER_TIMEOUT = 3 };
int check_device_error(const char *where);
int *device_error_ptr();   // address of the word on the current device

// ------------------------------------------------------- stage geometry ---
// One stage payload as the host parses it; the payload itself is a device
// pointer that host code never dereferences (decode-gpu.cu:30-56).
struct Layout {
    int dim, nc, rows, cols, nbit, v3;
    uint32_t mask;
    size_t cb_off, gain_off, stream_off, nidx, nidx_row, mrow, prow;
};

inline Layout make_layout(int dim, int nc, int rows, int cols, int v3) {
    Layout L;
    L.dim = dim;
    L.nc = nc;
    L.rows = rows;
    L.cols = cols;
    L.v3 = v3 ? 1 : 0;
    L.nbit = 1;
    while ((1u << L.nbit) < (unsigned)nc) L.nbit++;
    L.mask = (1u << L.nbit) - 1u;
    const size_t nidx_row = dim > 0 ? (size_t)cols / (size_t)dim : 0;
    const int mb = L.nbit > 12 ? 12 : L.nbit;
    L.cb_off = v3 ? 24 : 16;
    L.gain_off = L.cb_off + (size_t)nc * dim * 2;
    L.stream_off = L.gain_off + (size_t)rows * 2;
    L.nidx = (size_t)rows * nidx_row;
    L.nidx_row = nidx_row;
    L.mrow = v3 ? (nidx_row * (size_t)mb + 7) / 8 : 0;
    L.prow = (v3 && L.nbit > 12) ? (nidx_row + 7) / 8 : 0;
    return L;
}

inline size_t stage_bytes(const Layout &L) {
    if (L.v3) return L.stream_off + (size_t)L.rows * (L.mrow + L.prow);
    const size_t idx = L.nbit == 8 ? L.nidx : (L.nidx * (size_t)L.nbit + 7) / 8 + 1;
    return L.stream_off + idx;
}

// ----------------------------------------------------------- index read ---
// lib.rs:162-190 / decode-gpu.cu:82-121. Byte reads: a payload's row stream
// need not be word aligned for the generic path. The 4-byte window may read
// up to 3 bytes past the last index, inside the caller's 8 zeroed slack bytes.
__device__ __forceinline__ uint32_t rd_idx(const uint8_t *st, const Layout &L, size_t r, size_t i) {
    if (!L.v3) {
        const size_t gi = r * L.nidx_row + i;
        if (L.nbit == 8) return st[gi];
        const size_t bit = gi * (size_t)L.nbit;
        const uint8_t *q = st + (bit >> 3);
        const uint32_t w = (uint32_t)q[0] | ((uint32_t)q[1] << 8) | ((uint32_t)q[2] << 16);
        return (w >> (bit & 7)) & L.mask;
    }
    const uint32_t mb = L.nbit > 12 ? 12u : (uint32_t)L.nbit;
    const size_t bit = i * mb;
    const uint8_t *q = st + r * L.mrow + (bit >> 3);
    const uint32_t w = (uint32_t)q[0] | ((uint32_t)q[1] << 8) | ((uint32_t)q[2] << 16) | ((uint32_t)q[3] << 24);
    uint32_t v = (w >> (bit & 7)) & ((1u << mb) - 1u);
    if (L.prow) {
        const uint8_t *pl = st + L.mrow * (size_t)L.rows + r * L.prow;
        v |= (uint32_t)((pl[i >> 3] >> (i & 7)) & 1u) << 12;
    }
    return v;
}

// A DQV3 width above 13 bits would decode truncated indices silently
// (decode-gpu.cu:66-80), so every entry point refuses it.
inline bool v3_width_ok(int nc) {
    int b = 1;
    while ((1 << b) < nc) b++;
    return b <= 13;
}

int sm_count();
size_t smem_optin_max();

// QKV and g_proj in one launch (vq.cu): y = W RMSNorm?(x), xy = X RMSNorm?(x).
// 0 launched, 1 geometry not taken, -1 error.
int vq_gemv_with_extra(const void *const *stages, int nstg, const Layout &L, const void *const *xstages,
                       const Layout &XL, const float *x, const float *norm_w, float eps, float *y, float *xy,
                       int accumulate, cudaStream_t s);

// The Q8_0 head for up to 8 token rows in one pass (head_batch.cu), caller scratch:
// partial >= q80_head_batch_scratch() bytes, counter zeroed once. 1 launched, 0 not taken, -1 error.
size_t q80_head_batch_scratch();
int q80_head_batch_launch(const void *w, int rows, int cols, int ntok, const float *x, int ldx, const float *norm_w,
                          float eps, float *logits, int ldl, int *amax, unsigned long long *partial,
                          unsigned int *counter, cudaStream_t s);

// The decode GEMV as shared-memory table look-ups (vq_lut.cu): DQV3 dim 4, 4096 codes.
// lut_ok: the kernel takes the geometry; lut_bytes: one stage's re-laid index words;
// lut_part_bytes: the partial-sum scratch; lut_gemv: spk_vq_gemv's contract (plus an
// optional small extra matrix of the same input, g_proj) in two launches.
bool lut_ok(const Layout &L, int ns, int ng);
size_t lut_bytes(const Layout &L);
size_t lut_part_bytes(const Layout &L, int ng);
int lut_pack(const void *stage, const Layout &L, void *dst, cudaStream_t s);
int lut_gemv(const void *const *stages, const void *const *luts, int ns, int ng, const Layout &L, const float *x,
             const float *norm_w, float eps, float *y, int accumulate, float *part, const void *const *xst,
             const Layout *XL, float *xy, cudaStream_t s, int threads = 0);

// The decode step's VQ GEMVs as table look-ups over bank-scheduled u16-offset words, the
// cross-CTA sums and the epilogue in the same launch (vq_tab.cu). scratch: scratch_bytes,
// zeroed once (a grid barrier's count, then the per-CTA partials). An optional small matrix of
// the same input (g_proj, <= 64 rows) rides along.
namespace tab {
bool ok(const Layout &L, int ns, int ng);
size_t bytes(const Layout &L);
size_t scratch_bytes(const Layout &L, int ng);
int pack(const void *stage, const Layout &L, void *dst, cudaStream_t s);
int gemv(const void *const *stages, const void *const *words, int ns, int ng, const Layout &L, const float *x,
         const float *norm_w, float eps, float *y, int accumulate, void *scratch, const void *const *xst,
         const Layout *XL, float *xy, cudaStream_t s);
}  // namespace tab

// The VQ GEMM of a token batch on the tcgen05 tensor cores (vq_tc.cu), over the table
// kernel's re-laid stage words: 1 launched, 0 geometry not taken, -1 error.
//   mode 0: Y[n][r] = (accumulate ? Y[n][r] : 0) + (W RMSNorm?(X[n]))[r]
//   mode 1: Y[n][r] = gelu_erf(AUX[n][r]) * (W RMSNorm?(X[n]))[r]
size_t tc_scratch_bytes(int rows, int cols, int ntok);
int tc_gemm(const void *const *luts, int ns, const Layout &L, int ntok, const float *x, int ldx, const float *norm_w,
            float eps, float *y, int ldy, int accumulate, int mode, const float *aux, void *scratch, cudaStream_t s);

// The tied Q8_0 head in the tensor-core tile layout (q8t.cu): bytes of the tiled table,
// the re-lay from ggml blocks, its scratch (zeroed once), and the head for ntok <= 8 rows
// (1 launched, 0 geometry not taken, -1 error).
size_t q8t_bytes(int rows, int cols);
size_t q8t_scratch();
int q8t_pack(const void *w, int rows, int cols, void *dst, cudaStream_t s);
int q8t_head_launch(const void *wt, int rows, int cols, int ntok, const float *x, int ldx, const float *norm_w,
                    float eps, float *logits, int ldl, int *amax, void *scratch, cudaStream_t s);

// Q8_0 head (logits + argmax) with caller-owned scratch (ggml.cu).
int q80_head_launch(const void *w, int rows, int cols, const float *x, const float *norm_w, float eps, float *logits,
                    int *argmax_out, unsigned long long *partial, unsigned int *counter, cudaStream_t s);

// ------------------------------------------- programmatic dependent launch ---
// Every kernel of the decode path is launched with programmatic stream
// serialization: it may become resident (on SMs its predecessor has left) before
// the predecessor finishes, and do work that reads only immutable data (weights:
// codebooks, index streams, scales) until pdl_wait(). pdl_wait() returns when the
// preceding kernel has completed and its writes are visible; since every such
// kernel calls it on every path before it finishes, all earlier kernels of the
// stream have completed too. Without the launch attribute pdl_wait() returns at
// once. pdl_trigger() lets the next kernel start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, args...);
}

// ------------------------------------------------------ device helpers ---
#define SPK_WAIT_LIMIT (1u << 26)

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait: returns false (and records DEV_WAIT_TIMEOUT) if the phase never
// completes, so a lost copy ends the kernel with an error instead of a hang.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err) {
    for (uint32_t i = 0; i < SPK_WAIT_LIMIT; i++)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicExch(err, DEV_WAIT_TIMEOUT);
    return false;
}

// 1-D bulk copy global -> shared (TMA engine, no tensor map, no multicast).
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace spk
