// tp.cu — the two exchange kernels of the tensor-parallel decode step.
//
// Megatron-style sharding (attention by head, FFN by intermediate column) leaves
// two reductions of the 2560-wide residual per layer (after out_proj and after
// down_proj) and one argmax over the vocabulary shards of the head. Each is one
// launch here: every CTA sends its chunk of the rank's row to every peer's mailbox
// with NVLink stores, a release flag follows, and the CTA reduces the chunk once
// every rank's has arrived. There is no library collective on this path.
#include "spk.h"
#include "tp.cuh"

namespace spk {
namespace {

constexpr int TP_THREADS = 128;

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

__device__ __forceinline__ unsigned int *flag_at(const TpView &v, int owner, int slot, int chunk, int sender) {
    return v.flags[owner] + ((size_t)slot * TP_CHUNKS + chunk) * TP_MAX + sender;
}

// Threads 0..world-1 publish this rank's flag of `chunk` for `seq` to every rank
// (after the CTA's mailbox stores, which the barrier orders before the release).
__device__ __forceinline__ void publish(const TpView &v, int slot, int chunk, unsigned int seq) {
    __syncthreads();
    if ((int)threadIdx.x < v.world) {
        __threadfence_system();
        st_release_sys(flag_at(v, threadIdx.x, slot, chunk, v.rank), seq);
    }
}

// Wait until every sender's flag in this rank's mailbox has reached `seq`. The
// wait gives up after v.wait_ns (or 2^30 polls), records DEV_PEER_TIMEOUT and
// returns false; the kernel then finishes on whatever rows are present, and once
// the error is recorded later exchanges do not wait at all (the step's results
// are already invalid and the host reports the error).
__device__ bool wait_all(const TpView &v, int slot, int chunk, unsigned int seq) {
    __shared__ int ok;
    if (threadIdx.x == 0) ok = 1;
    __syncthreads();
    if ((int)threadIdx.x < v.world) {
        const unsigned int *f = flag_at(v, v.rank, slot, chunk, threadIdx.x);
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

// CTA c owns floats [c*chunk, min(n, (c+1)*chunk)), chunk a multiple of 4.
__global__ void __launch_bounds__(TP_THREADS) tp_sum_kernel(const TpView v, const float *__restrict__ part,
                                                            float *__restrict__ h, int n, int chunk) {
    __shared__ unsigned int s_seq;
    __shared__ int s_last;
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) s_seq = v.seq[0] + 1u;
    __syncthreads();
    const unsigned int seq = s_seq;
    const int slot = (int)(seq & 1u), c = blockIdx.x;
    const int i0 = c * chunk / 4, i1 = min((c + 1) * chunk, n) / 4;   // this CTA's float4 range
    const size_t row = ((size_t)slot * v.world + v.rank) * v.stride;
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const float4 x = reinterpret_cast<const float4 *>(part)[i];
        for (int q = 0; q < v.world; q++) reinterpret_cast<float4 *>(v.mail[q] + row)[i] = x;
    }
    publish(v, slot, c, seq);
    wait_all(v, slot, c, seq);
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const float4 *mail = reinterpret_cast<const float4 *>(v.mail[v.rank] + (size_t)slot * v.world * v.stride);
        float4 acc = __ldcg(mail + i);
        for (int r = 1; r < v.world; r++) {
            const float4 t = __ldcg(mail + (size_t)r * (v.stride / 4) + i);
            acc.x += t.x;
            acc.y += t.y;
            acc.z += t.z;
            acc.w += t.w;
        }
        float4 hv = reinterpret_cast<float4 *>(h)[i];
        hv.x = hv.x + acc.x;
        hv.y = hv.y + acc.y;
        hv.z = hv.z + acc.z;
        hv.w = hv.w + acc.w;
        reinterpret_cast<float4 *>(h)[i] = hv;
    }
    // the last CTA to finish advances the counter (every CTA has read it by then)
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&v.seq[1], 1u) == gridDim.x - 1;
    __syncthreads();
    if (s_last && threadIdx.x == 0) {
        v.seq[1] = 0u;
        v.seq[0] = seq;
    }
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
    if (threadIdx.x == 0) s_seq = v.seq[0] + 1u;
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
    publish(v, slot, 0, seq);
    wait_all(v, slot, 0, seq);
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
    if (t == 0) v.seq[0] = seq;
}

}  // namespace

size_t tp_mailbox_bytes(int world, int n, size_t *flags_off, int *stride) {
    const int st = (n + 63) / 64 * 64;
    const size_t mail = (size_t)2 * world * st * sizeof(float);
    const size_t off = (mail + 255) / 256 * 256;
    if (flags_off) *flags_off = off;
    if (stride) *stride = st;
    return off + (size_t)2 * TP_CHUNKS * TP_MAX * sizeof(unsigned int);
}

int tp_sum(const TpView &v, const float *part, float *h, int n, cudaStream_t s) {
    if (n % 4 || n > v.stride) return set_error("tp_sum: %d floats do not fit the %d-float mailbox rows", n, v.stride);
    // chunks of 256 floats (10 CTAs for the 2560-wide residual), at most TP_CHUNKS
    int chunk = 256, nb = (n + chunk - 1) / chunk;
    if (nb > TP_CHUNKS) {
        nb = TP_CHUNKS;
        chunk = ((n + nb - 1) / nb + 3) / 4 * 4;
        nb = (n + chunk - 1) / chunk;
    }
    cudaError_t e = launch_pdl(tp_sum_kernel, dim3(nb), dim3(TP_THREADS), 0, s, v, part, h, n, chunk);
    return e == cudaSuccess ? 0 : cuda_fail("tp_sum launch", e);
}

int tp_argmax(const TpView &v, const float *logits, int ldl, const int *amax_local, int row0, int *amax, int ntok,
              cudaStream_t s) {
    if (ntok < 1 || ntok > 32 || 2 * ntok > v.stride) return set_error("tp_argmax: %d rows", ntok);
    cudaError_t e = launch_pdl(tp_argmax_kernel, dim3(1), dim3(32), 0, s, v, logits, ldl, amax_local, row0, amax, ntok);
    return e == cudaSuccess ? 0 : cuda_fail("tp_argmax launch", e);
}

}  // namespace spk
