// vq_mma.cuh — VQ decode-GEMM for a small token batch (the speculative verify,
// M = 1 + 7 tokens) with the tensor cores as the contraction engine.
//
// Y[n][r] = sum_s gain_s[r] * sum_i cb_s[idx_s(r,i)] . X[n][4i..4i+3]   (dim 4, 12/13-bit DQV3)
//
// The weights' cost is the random 8-byte code-word gather from shared memory;
// with M tokens every gathered code word feeds M dot products, which SIMT lanes
// cannot hold activations for (4F values x M tokens per lane), so the gathered
// words go straight from registers into mma.sync m16n8k16 (f16 x f16 -> f32) as
// the A fragment, and the tokens are the 8 columns of B.
//
// Fragment mapping (PTX ISA, mma.m16n8k16 .row.col f16): thread (g = lane/4,
// t = lane%4) holds A rows g and g+8 at k-slots {2t, 2t+1, 2t+8, 2t+9}. K is
// permuted so that those four k-slots are the four dims of ONE code word, of
// group c_t: A regs {0, 2} = code word of row g (halves .x, .y), regs {1, 3} =
// code word of row g+8. B column n of thread (g, t) holds the same four k-slots
// of group c_t for column n = g. X is carried to ~22 bits as an f16 pair
// hi = rn(x), lo = rn(x - hi); products of f16 values are exact in f32:
//   M <= 4: one MMA, columns 0..3 = tokens' hi, 4..7 = tokens' lo (Y = D[n] + D[n+4]);
//   M 5..8: two MMAs into one accumulator, B_hi then B_lo (Y = D[n]).
// D (16x8 f32) of thread (g, t) is rows g, g+8 x columns 2t, 2t+1.
#pragma once
#include "common.cuh"

namespace spk {

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// x as an f16 pair: hi = rn(x), lo = rn(x - hi).
__device__ __forceinline__ void split_f16x4(float4 v, uint2 &hi, uint2 &lo) {
    const __half h0 = __float2half_rn(v.x), h1 = __float2half_rn(v.y), h2 = __float2half_rn(v.z),
                 h3 = __float2half_rn(v.w);
    const __half l0 = __float2half_rn(v.x - __half2float(h0)), l1 = __float2half_rn(v.y - __half2float(h1)),
                 l2 = __float2half_rn(v.z - __half2float(h2)), l3 = __float2half_rn(v.w - __half2float(h3));
    hi.x = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
    hi.y = (uint32_t)__half_as_ushort(h2) | ((uint32_t)__half_as_ushort(h3) << 16);
    lo.x = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
    lo.y = (uint32_t)__half_as_ushort(l2) | ((uint32_t)__half_as_ushort(l3) << 16);
}

// A run of S 12-bit fields starting at bit `bit0` of a row in shared memory
// (4-byte aligned row), returned as byte offsets v*8 into the code-word table.
template <int S>
struct Run {
    static constexpr int NW = (62 + 12 * S) / 32;   // words read: ceil((31 + 12S) / 32), any start shift
    static constexpr int NU = (31 + 12 * S) / 32;   // words after alignment: ceil(12S / 32)
    uint32_t u[NU];
    __device__ __forceinline__ void load(const uint8_t *row, uint32_t bit0, bool valid) {
        const uint32_t *wp = reinterpret_cast<const uint32_t *>(row) + (bit0 >> 5);
        const uint32_t sh = bit0 & 31u;
        uint32_t w[NW];
#pragma unroll
        for (int j = 0; j < NW; j++) w[j] = valid ? wp[j] : 0u;
#pragma unroll
        for (int j = 0; j < NU; j++) u[j] = __funnelshift_r(w[j], j + 1 < NW ? w[j + 1] : 0u, sh);
    }
    // byte offset (index * 8) of field s
    __device__ __forceinline__ uint32_t off(int s) const {
        const int b = 12 * s, wi = b >> 5, sh = b & 31;
        uint32_t v;
        if (sh + 12 <= 32 || wi + 1 >= NU)
            v = u[wi] >> sh;
        else
            v = __funnelshift_r(u[wi], u[wi + 1], sh);
        return (v & 0xFFFu) << 3;
    }
};

// The batched GEMM (vq_mma.cu): 1 launched, 0 geometry not taken, -1 error.
//   mode 0: Y[n][r] = (accumulate ? Y[n][r] : 0) + (W RMSNorm?(X[n]))[r]
//   mode 1: Y[n][r] = gelu_erf(AUX[n][r]) * (W RMSNorm?(X[n]))[r]
// X rows have stride ldx floats, Y / AUX rows stride ldy.
int vq_mma_batch(const void *const *stages, int nstg, const Layout &L, int ntok, const float *x, int ldx,
                 const float *norm_w, float eps, float *y, int ldy, int accumulate, int mode, const float *aux,
                 cudaStream_t s);

}  // namespace spk
