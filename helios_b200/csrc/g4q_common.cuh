// g4q_common.cuh -- shared device helpers for the g4q kernels (sm_100a only).
//
// Kernel layout v1 of a 4-bit, group-64 affine matrix W[N, K] (N % 16 == 0, K % 64 == 0):
//   packed: (K/64) x (N/16) blocks of 128 uint32; block (g, r) starts at word (g*(N/16)+r)*128.
//           In a block, lane l = 4*gi + t owns words l*4 + j (j = 0..3, one 16-byte load);
//           word j covers k0 = 64*g + 16*j for rows n0 = 16*r + gi and n1 = n0 + 8. Its nibble
//           slots hold exactly the mma.m16n8k16 A fragment of that lane:
//             slot 0:(n0,k0+2t) 4:(n0,k0+2t+1)  1:(n1,k0+2t) 5:(n1,k0+2t+1)
//             slot 2:(n0,k0+2t+8) 6:(n0,k0+2t+9) 3:(n1,k0+2t+8) 7:(n1,k0+2t+9)
//           so (word >> 4p) & 0x000F000F yields the bf16x2 register p of the fragment.
//   sb:     (K/64) x N uint32, word (g, n) = scale_bits | bias_bits << 16.
// A 256-row tile at group g is 8 KB of contiguous packed words plus 1 KB of sb, which is
// what the prefill GEMM copies with one bulk copy each.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace g4q {

constexpr uint32_t kMagic128 = 0x43004300u;   // bf16x2 (128, 128)
constexpr uint32_t kNibbleMask = 0x000F000Fu;
constexpr uint32_t kNeg128x2 = 0xC300C300u;   // bf16x2 (-128, -128)

__device__ __forceinline__ uint32_t lop_nibbles(uint32_t w) {
    // ((w & 0x000F000F) | 0x43004300): bf16x2 (128 + q_lo, 128 + q_hi), exact
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(w), "r"(kNibbleMask), "r"(kMagic128));
    return r;
}

__device__ __forceinline__ uint32_t fma_bf16x2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t sub_bf16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// (lo, lo) and (hi, hi) of a pair of 16-bit halves, written as packed-half moves: ptxas folds such a
// broadcast into the operand of the bf16x2 instruction that reads it (a byte permute would cost an
// ALU instruction of its own; measured 404 -> 378 instructions per streamed unit of the decode loop).
__device__ __forceinline__ uint32_t bcast_lo(uint32_t w) {
    uint32_t d;
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %1;\n\tmov.b32 %0, {l, l};\n\t}" : "=r"(d) : "r"(w));
    return d;
}

__device__ __forceinline__ uint32_t bcast_hi(uint32_t w) {
    uint32_t d;
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %1;\n\tmov.b32 %0, {h, h};\n\t}" : "=r"(d) : "r"(w));
    return d;
}

// Per-row constants of one group for the fast dequant: s2 = (s, s), n2 = (-128 s, -128 s),
// b2 = (b, b) as bf16x2 from an sb word (s | b << 16).
struct RowConsts {
    uint32_t s2, n2, b2;
};

__device__ __forceinline__ RowConsts row_consts(uint32_t sbw) {
    RowConsts c;
    c.s2 = bcast_lo(sbw);
    c.b2 = bcast_hi(sbw);
    c.n2 = mul_bf16x2(c.s2, kNeg128x2);   // exact scaling by -2^7 (|s| < 2^120 checked at load)
    return c;
}

// s * 2^129 for both halves of (s, s) by adding 129 to the exponent fields: exact for |s| < 2^-1
// (exponent <= 125, so no carry into the sign) unless s is subnormal; a zero s gives 4.0, and the
// odd-row dequant RN(RN(q * 2^-129 * 4) + b) then still returns b for any bias of magnitude above
// 2^-115 (and 0 for q = 0), so weights with subnormal scales are the only ones excluded.
constexpr uint32_t kExp129x2 = 0x40804080u;

// Chain R2 on a bf16x2 pair of (128 + q): bf16(bf16(s*q) + b).
//   fma.rn((128+q), s, -128 s) = RN(q*s) exactly (one rounding of the exact value);
//   add.rn(., b) = RN(RN(q*s) + b).
__device__ __forceinline__ uint32_t deq_r2_fast(uint32_t qp, const RowConsts& c) {
    return add_bf16x2(fma_bf16x2(qp, c.s2, c.n2), c.b2);
}

// General chains for any finite scale (used by the bit-exact dequantize kernels):
//   q = (128+q) - 128 exactly; R2 = RN(RN(q*s) + b); R1 = RN(q*s + b).
__device__ __forceinline__ uint32_t deq_general(uint32_t qp, uint32_t s2, uint32_t b2, int chain) {
    const uint32_t q = sub_bf16x2(qp, kMagic128);
    if (chain == 1) return fma_bf16x2(q, s2, b2);
    return add_bf16x2(mul_bf16x2(q, s2), b2);
}

__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

__device__ __forceinline__ uint32_t ldg_u32(const uint32_t* p) {
    uint32_t r;
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}

// D (f32 16x8) += A (bf16 16x16) * B (bf16 16x8)
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// geglu (native_model.cc:378-386) of one bf16 pair (g, u), each of the reference's nine bf16 ops
// rounded to bf16: cubic = bf16(0.044715), tanh_approx = bf16(0.7978845608028654) as model_scalar
// rounds them; g^3 = g*g*g is exact in fp32 for a bf16 g. Returns the bf16 bits.
__device__ __forceinline__ uint16_t geglu_bf16(float g, float u, float cubic, float tanh_approx) {
    const auto rb = [](float f) { return __bfloat162float(__float2bfloat16_rn(f)); };
    const float g3 = rb(g * g * g);              // power(gate, 3)
    const float t1 = rb(cubic * g3);             // 0.044715 * gate^3
    const float t2 = rb(g + t1);                 // gate + ...
    const float t3 = rb(tanh_approx * t2);       // sqrt(2/pi) * (...)
    const float t4 = rb(tanhf(t3));              // tanh
    const float t5 = rb(1.0f + t4);              // 1 + tanh
    const float t6 = rb(0.5f * g);               // 0.5 * gate
    const float t7 = rb(t6 * t5);                // gelu
    return f32_to_bf16_bits(t7 * u);             // gelu * up
}

// Order-preserving key of (value, index): max key = max value, ties -> smallest index.
// NaN maps to 0 so it is never selected over a number.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t index) {
    if (v != v) return 0ull;
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - index);
}

__device__ __forceinline__ float key_value(unsigned long long key) {
    uint32_t u = (uint32_t)(key >> 32);
    u = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
    return __uint_as_float(u);
}

__device__ __forceinline__ uint32_t key_index(unsigned long long key) {
    return 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull);
}

// ---- deterministic fp32 tanh from +,-,*,/ only (twin of the CPU oracle's g4o_tanh) -----
// Cody-Waite range reduction with ln2 split into a 15-bit head and a tail, Taylor series of
// expm1 to r^9/9!, tanh(a) = expm1(2a) / (expm1(2a) + 2). Every operation is an explicit
// round-to-nearest intrinsic so nothing is contracted into an FMA.
__device__ __forceinline__ float expm1_pos(float y) {
    const float LN2_HI = 0.693145751953125f;
    const float LN2_LO = 1.42860677e-06f;
    const int k = (int)__fadd_rn(__fmul_rn(y, 1.44269504f), 0.5f);
    const float kf = (float)k;
    const float r = __fsub_rn(__fsub_rn(y, __fmul_rn(kf, LN2_HI)), __fmul_rn(kf, LN2_LO));
    float p = 2.75573192e-06f;
    p = __fadd_rn(__fmul_rn(p, r), 2.48015873e-05f);
    p = __fadd_rn(__fmul_rn(p, r), 1.98412698e-04f);
    p = __fadd_rn(__fmul_rn(p, r), 1.38888889e-03f);
    p = __fadd_rn(__fmul_rn(p, r), 8.33333333e-03f);
    p = __fadd_rn(__fmul_rn(p, r), 4.16666667e-02f);
    p = __fadd_rn(__fmul_rn(p, r), 1.66666667e-01f);
    p = __fadd_rn(__fmul_rn(p, r), 0.5f);
    p = __fadd_rn(__fmul_rn(p, r), 1.0f);
    p = __fmul_rn(p, r);
    if (k == 0) return p;
    const float pow2 = __uint_as_float((uint32_t)(127 + k) << 23);
    return __fsub_rn(__fmul_rn(__fadd_rn(p, 1.0f), pow2), 1.0f);
}

__device__ __forceinline__ float tanh_det(float x) {
    if (x != x) return x;
    const uint32_t u = __float_as_uint(x);
    const float a = __uint_as_float(u & 0x7fffffffu);
    float t;
    if (a >= 9.0f) {
        t = 1.0f;
    } else if (a == 0.0f) {
        t = 0.0f;
    } else {
        const float e = expm1_pos(__fadd_rn(a, a));
        t = __fdiv_rn(e, __fadd_rn(e, 2.0f));
    }
    return __uint_as_float(__float_as_uint(t) | (u & 0x80000000u));
}

// MLX bf16 softcap: bf16(bf16(tanh(bf16(l / cap))) * cap), each step fp32 then RN to bf16.
__device__ __forceinline__ float softcap_bf16(float logit_bf16_value, float cap) {
    const float d = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(logit_bf16_value, cap)));
    const float t = __bfloat162float(__float2bfloat16_rn(tanh_det(d)));
    return __bfloat162float(__float2bfloat16_rn(__fmul_rn(t, cap)));
}

}  // namespace g4q
