// stream.cuh — TMA row-tile streamer shared by the VQ and ggml GEMV kernels.
//
// A tile is one or more byte ranges [A, B) of global memory (the index stream or
// block rows of a tile of matrix rows). Each range lands in its own 16-byte
// aligned shared-memory region, byte A at offset (A & 15). The aligned interior
// moves by cp.async.bulk (TMA, 1-D, no multicast); the copy is rounded up to a
// 16-byte end only when that stays below `limit` (the last readable byte + 1:
// the payload end plus the caller's guaranteed slack), otherwise the ragged
// tail (< 16 bytes, 2-byte aligned) goes through registers: all its loads are
// issued before any store, so it costs one memory round trip.
#pragma once
#include "common.cuh"

namespace spk {

// The copies of one tile: range k of the tile in entry k (len 0: nothing to copy). Every
// caller plans with compile-time k, so after unrolling the list lives in registers; a list
// indexed by a running count would sit in local memory, and the producer's loads and stores
// to it would queue behind the consumers' shared- and global-memory traffic.
template <int N>
struct BulkList {
    const void *src[N];
    void *dst[N];
    uint32_t len[N];
    uint32_t tx;
};

template <int N>
__device__ __forceinline__ void bulk_plan(BulkList<N> &bl, int k, uint8_t *d, uintptr_t A, uintptr_t B, uintptr_t limit) {
    bl.len[k] = 0;
    const uintptr_t Aal = A & ~(uintptr_t)15, Bup = (B + 15) & ~(uintptr_t)15;
    if (B <= A) return;
    bl.src[k] = (const void *)Aal;
    bl.dst[k] = d;
    if (Bup <= limit) {
        bl.len[k] = (uint32_t)(Bup - Aal);
        bl.tx += bl.len[k];
        return;
    }
    const uintptr_t Bfl = B & ~(uintptr_t)15;
    if (Bfl > Aal) {
        bl.len[k] = (uint32_t)(Bfl - Aal);
        bl.tx += bl.len[k];
    }
    const uintptr_t t0 = Bfl > Aal ? Bfl : Aal;   // 2-byte aligned, B - t0 < 16
    const int nt = (int)((B - t0 + 1) >> 1);
    uint16_t tv[8];
#pragma unroll
    for (int j = 0; j < 8; j++)
        if (j < nt) tv[j] = reinterpret_cast<const uint16_t *>(t0)[j];
    uint16_t *dt = reinterpret_cast<uint16_t *>(d + (t0 - Aal));
#pragma unroll
    for (int j = 0; j < 8; j++)
        if (j < nt) dt[j] = tv[j];
}

// Called by one thread after every bulk_plan of the tile: arrive on the
// tile's mbarrier with its byte count (release: orders the register-tail stores
// before the consumers' acquire), then start the copies.
template <int N>
__device__ __forceinline__ void bulk_issue(const BulkList<N> &bl, uint64_t *bar) {
    mbar_arrive_expect_tx(bar, bl.tx);
    fence_proxy_async();
#pragma unroll
    for (int k = 0; k < N; k++)
        if (bl.len[k]) bulk_g2s(bl.dst[k], bl.src[k], bl.len[k], bar);
}

}  // namespace spk
