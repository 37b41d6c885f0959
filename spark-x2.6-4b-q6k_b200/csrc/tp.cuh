// tp.cuh — tensor-parallel exchanges of the decode step over peer memory.
//
// Every rank owns one device allocation (its "mailbox"), exported to the other
// ranks with CUDA IPC (or passed as plain pointers by a single process that
// drives several GPUs with peer access):
//   mail[2][world][stride / 2] 8-byte (value, sequence) pairs, slot-major, one row per sender
// An exchange with sequence number s uses slot s & 1. The row is cut into chunks,
// one CTA each: a CTA stores its chunk into every rank's mailbox (NVLink stores,
// each value paired with s in one single-copy-atomic 8-byte store), waits, bounded
// in time, until every sender's pairs for its chunk carry s, and reduces the chunk
// in rank order 0..world-1, so all ranks end with bit-identical results. Sequence
// numbers are unique, so a stale pair never passes for a new one. Two slots
// suffice: a rank can only start exchange s+2 after every rank has stored its row
// of s+1, which each does only after it has finished reading s.
#pragma once
#include "common.cuh"

namespace spk {

constexpr int TP_MAX = 8;
constexpr int TP_CHUNKS = 32;   // CTAs (row chunks) per exchange, at most

struct TpView {
    float *mail[TP_MAX];            // every rank's mailbox, as mapped in this process
    unsigned int *flags[TP_MAX];    // every rank's area past the pair rows (unused by the exchanges)
    int rank, world;
    int stride;                     // floats per mailbox row (>= the exchanged length, a multiple of 64)
    unsigned int *seq;              // this rank's [exchange counter, finished-CTA ticket] (device, zero)
    unsigned long long wait_ns;     // give-up time of a wait
    int *err;                       // device error word
};

// Device helpers of the exchanges: the global nanosecond timer of the bounded waits, and one
// (value, sequence) pair stored or loaded as a single 8-byte access.
__device__ __forceinline__ unsigned long long tp_time_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void tp_st_pair(uint2 *p, uint32_t value, uint32_t seq) {
    asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(value), "r"(seq) : "memory");
}
__device__ __forceinline__ uint2 tp_ld_pair(const uint2 *p) {
    uint2 v;
    asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
    return v;
}

// The residual reduction of rows [r0, r1) after this rank stored its (value, seq) pairs for
// them into every rank's mailbox (slot seq & 1, this rank's sender row): h[r] += the rows of
// every rank summed in rank order 0..world-1 (each pair waited for, bounded in time; a wait
// that runs out records DEV_PEER_TIMEOUT and later waits skip), by the calling CTA's threads.
__device__ __forceinline__ void tp_reduce_rows(const TpView &v, unsigned int seq, int r0, int r1, float *h) {
    const size_t prow = (size_t)v.stride / 2;
    const uint2 *mail = reinterpret_cast<const uint2 *>(v.mail[v.rank]) + (size_t)(seq & 1u) * v.world * prow;
    bool give_up = *reinterpret_cast<volatile int *>(v.err) == DEV_PEER_TIMEOUT;
    const unsigned long long t0 = tp_time_ns();
    for (int i = r0 + (int)threadIdx.x; i < r1; i += blockDim.x) {
        float acc = 0.f;
        for (int r = 0; r < v.world; r++) {
            uint2 pr = tp_ld_pair(mail + (size_t)r * prow + i);
            for (unsigned int it = 0; pr.y != seq && !give_up; it++) {
                if (it > (1u << 30) || tp_time_ns() - t0 > v.wait_ns) {
                    give_up = true;
                    atomicExch(v.err, DEV_PEER_TIMEOUT);
                    break;
                }
                pr = tp_ld_pair(mail + (size_t)r * prow + i);
            }
            const float x = __uint_as_float(pr.x);
            acc = r == 0 ? x : acc + x;
        }
        h[i] = h[i] + acc;
    }
}

// Bytes of one mailbox for `world` ranks and rows of up to n floats (n/2 pairs);
// *flags_off receives the byte offset just past the rows.
size_t tp_mailbox_bytes(int world, int n, size_t *flags_off, int *stride);

// h[i] += sum over ranks r (in rank order) of part_r[i], i < n (n a multiple of 4, the
// mailbox rows at least 2n floats: the values travel as (value, sequence) pairs).
int tp_sum(const TpView &v, const float *part, float *h, int n, cudaStream_t s);

// Global greedy ids over vocabulary shards, for ntok token rows: rank r holds
// vocabulary rows [row0_r, row0_r + n_r), token t's logits at logits[t*ldl ..] and
// its local first-max index amax_local[t]; amax[t] receives the first index of the
// global maximum (NaN never wins, -0 equals +0).
int tp_argmax(const TpView &v, const float *logits, int ldl, const int *amax_local, int row0, int *amax, int ntok,
              cudaStream_t s);

// out_proj / down_proj of the tensor-parallel decode step with the residual exchange fused in
// (vq.cu): the code-word GEMV's CTA k computes this rank's partial of rows [rb_k, re_k) of
// W x, sends them to every rank's mailbox, waits for every rank's rows [rb_k, re_k) (the
// peers' CTA k, the same row split) and adds their rank-ordered sum into h, tp_sum's exact
// arithmetic in the same launch. 0 launched, 1 not taken (the fast kernel does not take the
// geometry), -1 error.
int vq_gemv_tp(const void *const *stages, int nstg, const Layout &L, const float *x, float *h, const TpView &v,
               cudaStream_t s);

}  // namespace spk
