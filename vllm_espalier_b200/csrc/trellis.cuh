// Trellis decode core: 16-bit trellis states -> codebook values, as mma.sync fragments.
//
// Format (the reference's experts_grouped.cuh:83-154, 330-339): a 16x16 tile of weights is a circular MSB-first
// bitstream of 256*K bits (K = bits a weight) stored as 8*K uint32 words (int16 pairs, little-endian). The state of
// value p (0..255) is the 16 bits ending just before stream bit (p + 1) * K. Value p = 8 * lane + j sits at row
// (input k) 2t + 8((j >> 1) & 1) + (j & 1) and column (output n) g + 8(j >> 2) of the tile, lane = 4g + t.
//
// Design (B200): a lane reads the 2-3 words that hold its eight windows straight from shared memory (the tile was
// staged there by the producer warps' asynchronous copies), aligns them once with a funnel shift and cuts the eight states with constant shifts.
// The eight values are exactly the lane's A fragment of an m16n8k16 MMA whose M dimension is the tile's 16 output
// columns and whose N dimension is 8 tokens (weights as A: one MMA per tile per 8 tokens, no register shuffles).
//
// Codebooks (kernel ids of the reference, experts_grouped.cuh:23-80): 1 mcg, 3 E2M1, 6 int5, 7 int6.
//   exact form  (cb_exact): the reference's fp16 values bit for bit (dequant, tests).
//   kernel form (cb_gemv):  what the GEMVs multiply by. mcg, int5 and int6: the exact values themselves, so every
//                           product uses a weight bit-identical to the reference's decode; E2M1: the exact values
//                           divided by C = 0.75 (hardware e2m1 conversion; multiples of C are exact in fp16, so the
//                           sum times C equals the sum of the exact products). The GEMV epilogue multiplies its fp32
//                           sums by cb_step: C for E2M1, 1 otherwise.
#pragma once

#include "common.cuh"

namespace esp {

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// mcg pair (experts_grouped.cuh:64-79): x = s * 0xCBAC1FED; x = (x & 0x8FFF8FFF) ^ 0x3B603B60; v = fp16 lo + fp16 hi.
// Each sum is one fp16 add of the word's two halves broadcast (v in both halves), and one permute packs v0, v1: a
// permute fewer than gathering the low and the high halves first, on the ALU pipe that bounds the decode.
__device__ __forceinline__ uint32_t mcg2(uint32_t s0, uint32_t s1) {
    uint32_t x0 = s0 * 0xCBAC1FEDu, x1 = s1 * 0xCBAC1FEDu;
    x0 = (x0 & 0x8FFF8FFFu) ^ 0x3B603B60u;
    x1 = (x1 & 0x8FFF8FFFu) ^ 0x3B603B60u;
    const __half2 h0 = u2h(x0), h1 = u2h(x1);
    const __half2 v0 = __hadd2(__low2half2(h0), __high2half2(h0));
    const __half2 v1 = __hadd2(__low2half2(h1), __high2half2(h1));
    return h2u(__lows2half2(v0, v1));
}

// E2M1 in units of C = 0.75. The reference thresholds |v| at C * {.25, .75, 1.25, 1.75, 2.5, 3.5, 5} with strict '>'
// (ties go down). Here u = v * fl32(fl32(1/C) * (1 - 2^-20)) in fp32 and the hardware's round-to-nearest-even e2m1
// conversion: the factor sits just below 1/C, so an exact tie lands below its midpoint and every other fp16 v stays on
// its side (checked for all 65536 states against the reference's rule). Saturates at 6, keeps the sign of zero.
constexpr float E2M1_C = 0.75f;
constexpr float E2M1_INV_C = 0x1.55554p+0f;   // fl32(fl32(1 / 0.75) * fl32(1 - 2^-20))

// Two fp32 lanes in one 64-bit register for the sm_100 packed fp32 instructions (each lane an IEEE round-to-nearest
// operation of its own, the same results as two scalar instructions in half the issue slots).
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2unpack(uint64_t r, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t f2splat(float a) { return f2pack(a, a); }

__device__ __forceinline__ uint32_t e2m1_units2(uint32_t v) {
    const float2 f = __half22float2(u2h(v));
    float a, b;
    f2unpack(mul_f32x2(f2pack(f.x, f.y), f2splat(E2M1_INV_C)), a, b);
    uint32_t h;
    // a -> low half, b -> high half: the packing puts the first source in the upper nibble
    asm("{ .reg .b8 t; cvt.rn.satfinite.e2m1x2.f32 t, %1, %2; cvt.rn.f16x2.e2m1x2 %0, t; }" : "=r"(h) : "f"(b), "f"(a));
    return h;
}

// int5 / int6 grid index q = rintf(fl32(v * k)) (experts_grouped.cuh:39-55). rintf through a magic add:
// fl32(p + M) with M = 1.5 * 2^23 + 0x6420 rounds p to an integer (ties to even, M even) and leaves the fp16 bits of
// 1056 + q in the low half-word; one fp16 subtraction of 1056 gives q exactly (|q| <= 31).
constexpr float INT5_K = 0x1.e62c10p+1f;
constexpr float INT6_K = 0x1.f660bap+2f;
constexpr float INT_MAGIC = 12608544.0f;   // 1.5 * 2^23 + 0x6420

// int6 admits a single fused multiply-add: with k' = k + 1 ulp the exactly rounded fl32(v k' + M) equals
// rintf(fl32(v k)) + M for every one of the 65536 states (an interval of 332 such fp32 k' exists; checked exhaustively).
// int5 has no such k' (the feasible interval of k is a single point), so it keeps the product's own rounding.
constexpr float INT6_K_FMA = 0x1.f660bcp+2f;   // INT6_K + 1 ulp

// int6 uses one packed fp32x2 FMA. int5 keeps scalar multiply and add: the packed multiply followed by the packed add
// decoded 19 of the 65536 states one index off on a B200 (the result of a single rounding of v k + M, which int5
// cannot tolerate), the scalar pair none (all states checked on the GPU).
template <int CB>
__device__ __forceinline__ uint32_t int_index2(uint32_t v) {
    const float2 f = __half22float2(u2h(v));
    uint32_t a, b;
    if constexpr (CB == 7) {
        float fa, fb;
        f2unpack(fma_f32x2(f2pack(f.x, f.y), f2splat(INT6_K_FMA), f2splat(INT_MAGIC)), fa, fb);
        a = __float_as_uint(fa);
        b = __float_as_uint(fb);
    } else {
        a = __float_as_uint(__fadd_rn(__fmul_rn(f.x, INT5_K), INT_MAGIC));
        b = __float_as_uint(__fadd_rn(__fmul_rn(f.y, INT5_K), INT_MAGIC));
    }
    const __half2 q = u2h(__byte_perm(a, b, 0x5410));
    return h2u(__hsub2(q, __float2half2_rn(1056.0f)));
}

// int5 / int6 weights w = fl16(fl32(q * c)), c = fl32(3.94921875 / 15 or / 31) (experts_grouped.cuh:39-55), from the
// grid index q in fp16 by two fp16 operations: w = fl16(q * c_hi + fl16(q * c_lo)) with c_hi = fl16(c) and
// c_lo = fl16(c - c_hi). For every index |q| <= 31 this is the reference's value bit for bit (checked exhaustively;
// no single fp16 factor reproduces all of them). int6's c_lo is an fp16 subnormal, which fp16 arithmetic keeps.
constexpr uint32_t INT5_C_HI2 = 0x34363436u, INT5_C_LO2 = 0x06660666u;
constexpr uint32_t INT6_C_HI2 = 0x30143014u, INT6_C_LO2 = 0x83198319u;

template <int CB>
__device__ __forceinline__ uint32_t int_weight2(uint32_t v) {
    const __half2 q = u2h(int_index2<CB>(v));
    const __half2 hi = u2h(CB == 6 ? INT5_C_HI2 : INT6_C_HI2), lo = u2h(CB == 6 ? INT5_C_LO2 : INT6_C_LO2);
    return h2u(__hfma2(q, hi, __hmul2(q, lo)));
}

// factor the fp32 sums of kernel-form products are multiplied by: C for E2M1 (values in units of C), 1 otherwise
__host__ __device__ __forceinline__ float cb_step(int cb) { return cb == 3 ? E2M1_C : 1.0f; }

template <int CB>
__device__ __forceinline__ uint32_t cb_gemv(uint32_t s0, uint32_t s1) {
    const uint32_t m = mcg2(s0, s1);
    if constexpr (CB == 1) return m;
    else if constexpr (CB == 3) return e2m1_units2(m);
    else return int_weight2<CB>(m);
}

// the reference's fp16 values bit for bit. int5 / int6 through rintf, which keeps the sign of a zero index (the
// magic add of int_index2 gives +0 where rintf gives -0; the sign of a zero weight changes no GEMV sum)
template <int CB>
__device__ __forceinline__ uint32_t cb_exact(uint32_t s0, uint32_t s1) {
    const uint32_t m = mcg2(s0, s1);
    if constexpr (CB == 1) {
        return m;
    } else if constexpr (CB == 3) {
        return h2u(__hmul2(u2h(e2m1_units2(m)), __float2half2_rn(E2M1_C)));
    } else {
        constexpr float k = CB == 6 ? INT5_K : INT6_K;
        constexpr float c = 3.94921875f / (CB == 6 ? 15.0f : 31.0f);
        const float2 v = __half22float2(u2h(m));
        return h2u(__floats2half2_rn(rintf(__fmul_rn(v.x, k)) * c, rintf(__fmul_rn(v.y, k)) * c));
    }
}

// The (codebook, bits) pairs this library instantiates: the reference's set (experts_grouped.cuh:227-229).
#define ESP_FOR_EACH_CASE(X) \
    X(1, 1) X(1, 2) X(1, 3) X(1, 4) X(1, 5) X(1, 6) X(1, 7) X(1, 8) \
    X(3, 1) X(3, 2) X(3, 3) X(6, 2) X(6, 3) X(6, 4) X(7, 3) X(7, 4) X(7, 5)

__host__ __device__ constexpr bool case_supported(int cb, int K) {
    return (cb == 1 && K >= 1 && K <= 8) || (cb == 3 && K >= 1 && K <= 3) || (cb == 6 && K >= 2 && K <= 4) ||
           (cb == 7 && K >= 3 && K <= 5);
}

// ---------------------------------------------------------------------------------------------------------------
// A lane's eight states of one tile. `tile` points at the tile's 8K words (shared or global memory).
// ---------------------------------------------------------------------------------------------------------------
template <int K>
__device__ __forceinline__ void tile_states(const uint32_t* tile, int lane, uint32_t (&st)[8]) {
    constexpr int NB = 256 * K, TW = 8 * K;
    // the lane's window: stream bits [a, a + 7K + 16), a = 8 lane K + K - 16 (circular)
    int w0, sh;
    if constexpr (K == 4) {
        w0 = (lane + 31) & 31;   // a = 32 lane - 12: word lane - 1, bit 20
        sh = 20;
    } else if constexpr (K == 8) {
        w0 = (2 * lane + 63) & 63;   // a = 64 lane - 8: word 2 lane - 1, bit 24
        sh = 24;
    } else {
        const int a = (8 * lane * K + K - 16 + NB) % NB;
        w0 = a >> 5;
        sh = a & 31;
    }
    const uint32_t wa = tile[w0];
    const uint32_t wb = tile[(w0 + 1) % TW];
    // (hi : lo) = the 64 stream bits from a on, MSB first; state j is bits [jK, jK + 16) of it
    uint32_t hi, lo, lo2 = 0;
    if constexpr (K <= 4) {
        hi = __funnelshift_l(wb, wa, sh);
        lo = wb << sh;
    } else {
        const uint32_t wc = tile[(w0 + 2) % TW];
        hi = __funnelshift_l(wb, wa, sh);
        lo = __funnelshift_l(wc, wb, sh);
        lo2 = wc << sh;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int o = j * K;   // offset of state j from the window's first bit
        uint32_t s;
        if (o == 0) s = hi >> 16;
        else if (o == 8) s = __byte_perm(hi, 0u, 0x4421);
        else if (o == 16) s = hi & 0xffffu;
        else if (o < 16) s = (hi >> (16 - o)) & 0xffffu;
        else if (o == 32) s = lo >> 16;
        else if (o == 40) s = __byte_perm(lo, 0u, 0x4421);
        else if (o == 48) s = lo & 0xffffu;
        else if (o < 48) s = __funnelshift_r(lo, hi, 48 - o) & 0xffffu;
        else s = __funnelshift_r(lo2, lo, 80 - o) & 0xffffu;
        st[j] = s;
    }
}

// A fragment of m16n8k16 (row-major A = W^T: rows = 16 output columns, cols = 16 inputs) from the eight values:
// a0 = values 0,1 (col g, k 2t..2t+1); a1 = 4,5 (col g+8); a2 = 2,3 (k 2t+8..); a3 = 6,7.
template <int CB, int K>
__device__ __forceinline__ void decode_a(const uint32_t* tile, int lane, uint32_t (&a)[4]) {
    uint32_t st[8];
    tile_states<K>(tile, lane, st);
    a[0] = cb_gemv<CB>(st[0], st[1]);
    a[1] = cb_gemv<CB>(st[4], st[5]);
    a[2] = cb_gemv<CB>(st[2], st[3]);
    a[3] = cb_gemv<CB>(st[6], st[7]);
}

// D (16 columns x 8 tokens, fp32) += A (16 x 16 fp16) * B (16 x 8 fp16)
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

}  // namespace esp
