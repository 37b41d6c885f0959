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

}  // namespace spk
