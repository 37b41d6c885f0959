// tp.cu — the two exchange kernels of the tensor-parallel decode step.
//
// Megatron-style sharding (attention by head, FFN by intermediate column) leaves
// two reductions of the 2560-wide residual per layer (after out_proj and after
// down_proj) and one argmax over the vocabulary shards of the head. Each is one
// single-CTA launch here: the rank's row goes to every peer's mailbox with
// NVLink stores, a release flag follows, and the reduction runs on the rows
// received. There is no library collective on this path.
#include "spk.h"
#include "tp.cuh"

namespace spk {
namespace {

constexpr int TP_THREADS = 512;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int *p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(unsigned int *p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Threads 0..world-1 publish this rank's flag for `seq` to every rank (after the
// CTA's mailbox stores, which the barrier orders before the release).
__device__ __forceinline__ void publish(const TpView &v, int slot, unsigned int seq) {
    __syncthreads();
    if ((int)threadIdx.x < v.world) {
        __threadfence_system();
        st_release_sys(v.flags[threadIdx.x] + slot * TP_MAX + v.rank, seq);
    }
}

// Wait until every sender's flag in this rank's mailbox has reached `seq`. The
// wait gives up after v.wait_ns (or 2^30 polls), records DEV_PEER_TIMEOUT and
// returns false; the kernel then finishes on whatever rows are present, and once
// the error is recorded later exchanges do not wait at all (the step's results
// are already invalid and the host reports the error).
__device__ bool wait_all(const TpView &v, int slot, unsigned int seq) {
    __shared__ int ok;
    if (threadIdx.x == 0) ok = 1;
    __syncthreads();
    if ((int)threadIdx.x < v.world) {
        const unsigned int *f = v.flags[v.rank] + slot * TP_MAX + threadIdx.x;
        const unsigned long long t0 = globaltimer_ns();
        bool give_up = *reinterpret_cast<volatile int *>(v.err) == DEV_PEER_TIMEOUT;
        for (unsigned int it = 0; !give_up; it++) {
            if ((int)(ld_acquire_sys(f) - seq) >= 0) break;
            give_up = it > (1u << 30) || globaltimer_ns() - t0 > v.wait_ns;
            if (give_up) atomicExch(v.err, DEV_PEER_TIMEOUT);
        }
        if (give_up) ok = 0;
    }
    __syncthreads();
    return ok != 0;
}

__global__ void __launch_bounds__(TP_THREADS) tp_sum_kernel(const TpView v, const float *__restrict__ part,
                                                            float *__restrict__ h, int n) {
    __shared__ unsigned int s_seq;
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) s_seq = *v.seq + 1u;
    __syncthreads();
    const unsigned int seq = s_seq;
    const int slot = (int)(seq & 1u);
    const size_t row = ((size_t)slot * v.world + v.rank) * v.stride;
    const float4 *p4 = reinterpret_cast<const float4 *>(part);
    for (int i = threadIdx.x; i < n / 4; i += blockDim.x) {
        const float4 x = p4[i];
        for (int q = 0; q < v.world; q++) reinterpret_cast<float4 *>(v.mail[q] + row)[i] = x;
    }
    publish(v, slot, seq);
    wait_all(v, slot, seq);
    const float *mine = v.mail[v.rank] + (size_t)slot * v.world * v.stride;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float s = __ldcg(mine + i);
        for (int r = 1; r < v.world; r++) s += __ldcg(mine + (size_t)r * v.stride + i);
        h[i] = h[i] + s;
    }
    __syncthreads();
    if (threadIdx.x == 0) *v.seq = seq;
}

// Order-preserving key of (value, index): larger value wins, then the smaller
// index; NaN ranks below every number, -0 equals +0.
__device__ __forceinline__ unsigned long long argmax_key(float x, int idx) {
    unsigned int b = __float_as_uint(x);
    if (b == 0x80000000u) b = 0u;
    unsigned int k = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    if (x != x) k = 0u;
    return ((unsigned long long)k << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned int)idx);
}

__global__ void tp_argmax_kernel(const TpView v, const float *__restrict__ logits, int ldl,
                                 const int *__restrict__ amax_local, int row0, int *__restrict__ amax, int ntok) {
    __shared__ unsigned int s_seq;
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) s_seq = *v.seq + 1u;
    __syncthreads();
    const unsigned int seq = s_seq;
    const int slot = (int)(seq & 1u);
    const size_t row = ((size_t)slot * v.world + v.rank) * v.stride;
    const int t = threadIdx.x;   // token row t of the batch
    if (t < ntok) {
        const int li = amax_local[t];
        const unsigned long long key = argmax_key(logits[(size_t)t * ldl + li], row0 + li);
        for (int q = 0; q < v.world; q++) reinterpret_cast<unsigned long long *>(v.mail[q] + row)[t] = key;
    }
    publish(v, slot, seq);
    wait_all(v, slot, seq);
    if (t < ntok) {
        const float *mine = v.mail[v.rank] + (size_t)slot * v.world * v.stride;
        unsigned long long best = 0ull;
        for (int r = 0; r < v.world; r++) {
            const unsigned long long k =
                __ldcg(reinterpret_cast<const unsigned long long *>(mine + (size_t)r * v.stride) + t);
            best = k > best ? k : best;
        }
        amax[t] = (int)(0xFFFFFFFFu - (unsigned int)(best & 0xFFFFFFFFull));
    }
    __syncthreads();
    if (t == 0) *v.seq = seq;
}

}  // namespace

size_t tp_mailbox_bytes(int world, int n, size_t *flags_off, int *stride) {
    const int st = (n + 63) / 64 * 64;
    const size_t mail = (size_t)2 * world * st * sizeof(float);
    const size_t off = (mail + 255) / 256 * 256;
    if (flags_off) *flags_off = off;
    if (stride) *stride = st;
    return off + (size_t)2 * TP_MAX * sizeof(unsigned int);
}

int tp_sum(const TpView &v, const float *part, float *h, int n, cudaStream_t s) {
    if (n % 4 || n > v.stride) return set_error("tp_sum: %d floats do not fit the %d-float mailbox rows", n, v.stride);
    cudaError_t e = launch_pdl(tp_sum_kernel, dim3(1), dim3(TP_THREADS), 0, s, v, part, h, n);
    return e == cudaSuccess ? 0 : cuda_fail("tp_sum launch", e);
}

int tp_argmax(const TpView &v, const float *logits, int ldl, const int *amax_local, int row0, int *amax, int ntok,
              cudaStream_t s) {
    if (ntok < 1 || ntok > 32 || 2 * ntok > v.stride) return set_error("tp_argmax: %d rows", ntok);
    cudaError_t e = launch_pdl(tp_argmax_kernel, dim3(1), dim3(32), 0, s, v, logits, ldl, amax_local, row0, amax, ntok);
    return e == cudaSuccess ? 0 : cuda_fail("tp_argmax launch", e);
}

}  // namespace spk
