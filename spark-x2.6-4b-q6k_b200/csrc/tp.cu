// tp.cu — the two exchange kernels of the tensor-parallel decode step.
//
// Megatron-style sharding (attention by head, FFN by intermediate column) leaves
// two reductions of the 2560-wide residual per layer (after out_proj and after
// down_proj) and one argmax over the vocabulary shards of the head. Each is one
// launch here: every CTA sends its chunk of the rank's row to every peer's mailbox
// with NVLink stores and reduces the chunk once every rank's has arrived: every
// value travels as a (value, sequence number) pair in one 8-byte store.
// There is no library collective on this path.
#include "spk.h"
#include "tp.cuh"

namespace spk {
namespace {

constexpr int TP_THREADS = 128;

__device__ __forceinline__ unsigned long long globaltimer_ns() { return tp_time_ns(); }
__device__ __forceinline__ void st_pair(uint2 *p, uint32_t value, uint32_t seq) { tp_st_pair(p, value, seq); }
__device__ __forceinline__ uint2 ld_pair(const uint2 *p) { return tp_ld_pair(p); }

// The residual reduction, low-latency form: every value travels as an 8-byte
// (value, sequence number) pair — one single-copy-atomic store — so a receiver
// knows a value has arrived when its pair carries this exchange's number, and no
// fence or separate flag is needed. The pair rows live in the mailbox's float area
// (stride floats per sender row = stride/2 pairs). CTA c owns values
// [c*chunk, min(n, (c+1)*chunk)). Each thread polls the pairs it reduces, bounded
// in time; a wait that runs out records DEV_PEER_TIMEOUT and later waits skip.
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
    const int i0 = c * chunk, i1 = min((c + 1) * chunk, n);
    const size_t prow = (size_t)v.stride / 2;   // pairs per sender row
    const size_t mine_row = ((size_t)slot * v.world + v.rank) * prow;
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const uint32_t x = __float_as_uint(part[i]);
        for (int q = 0; q < v.world; q++) st_pair(reinterpret_cast<uint2 *>(v.mail[q]) + mine_row + i, x, seq);
    }
    tp_reduce_rows(v, seq, i0, i1, h);
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

// The vocabulary-shard argmax: token t's 64-bit key travels as two (half, sequence)
// pairs at pair positions 2t, 2t+1 of the sender's row, like the residual's values.
__global__ void tp_argmax_kernel(const TpView v, const float *__restrict__ logits, int ldl,
                                 const int *__restrict__ amax_local, int row0, int *__restrict__ amax, int ntok) {
    __shared__ unsigned int s_seq;
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) s_seq = v.seq[0] + 1u;
    __syncthreads();
    const unsigned int seq = s_seq;
    const int slot = (int)(seq & 1u);
    const size_t prow = (size_t)v.stride / 2;
    const int t = threadIdx.x;   // token row t of the batch
    if (t < ntok) {
        const int li = amax_local[t];
        const unsigned long long key = argmax_key(logits[(size_t)t * ldl + li], row0 + li);
        for (int q = 0; q < v.world; q++) {
            uint2 *dst = reinterpret_cast<uint2 *>(v.mail[q]) + ((size_t)slot * v.world + v.rank) * prow + 2 * t;
            st_pair(dst, (uint32_t)key, seq);
            st_pair(dst + 1, (uint32_t)(key >> 32), seq);
        }
    }
    if (t < ntok) {
        const uint2 *mail = reinterpret_cast<const uint2 *>(v.mail[v.rank]) + (size_t)slot * v.world * prow;
        bool give_up = *reinterpret_cast<volatile int *>(v.err) == DEV_PEER_TIMEOUT;
        const unsigned long long t0 = globaltimer_ns();
        unsigned long long best = 0ull;
        for (int r = 0; r < v.world; r++) {
            uint32_t half[2];
            for (int k = 0; k < 2; k++) {
                uint2 pr = ld_pair(mail + (size_t)r * prow + 2 * t + k);
                for (unsigned int it = 0; pr.y != seq && !give_up; it++) {
                    if (it > (1u << 30) || globaltimer_ns() - t0 > v.wait_ns) {
                        give_up = true;
                        atomicExch(v.err, DEV_PEER_TIMEOUT);
                        break;
                    }
                    pr = ld_pair(mail + (size_t)r * prow + 2 * t + k);
                }
                half[k] = pr.x;
            }
            const unsigned long long kr = ((unsigned long long)half[1] << 32) | half[0];
            best = kr > best ? kr : best;
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
    if (n % 4 || 2 * n > v.stride) return set_error("tp_sum: %d values do not fit the %d-float mailbox rows as pairs", n, v.stride);
    // chunks of 256 values (10 CTAs for the 2560-wide residual), at most TP_CHUNKS
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
