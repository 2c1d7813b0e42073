// g4q_mlp.cu -- the elementwise neighbours of the quantized MLP linears (sm_100a).
//
// layer_forward (native/gemma4_mlx/src/native_model.cc:899-970) runs, around gate/up/down:
//   h = bf16(fast::rms_norm(h, pre_feedforward_layernorm.weight, 1e-6))     (:929-932)
//   act = geglu(gate, up)                                                   (:378-386, :945)
// MLX evaluates geglu as nine separate bf16 ops (power, two scalar products, an add, tanh, an add,
// two products and the final product with up), each rounding its fp32 result to bf16. geglu_kernel
// performs the same nine roundings in registers in one pass over gate and up: one launch instead
// of nine, and 3 x 2 bytes of HBM per element instead of ~27 x 2. g^3 is computed as g*g*g, which
// is exact in fp32 for a bf16 g (8-bit significands), so it equals the correctly rounded power.
//
// rms_norm_kernel: one CTA per row; fp32 sum of squares, inv = the correctly rounded 1/sqrt of the
// fp32 mean + eps; the normalized value x * inv is rounded to bf16 (the input dtype) and then
// multiplied by the bf16 weight with one more rounding, out = bf16(w * bf16(x * inv)), as MLX's
// fast::rms_norm orders its roundings; the weight may be absent (values norm, :844).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "g4q_common.cuh"
#include "g4q_internal.h"

namespace g4q {
namespace {

__device__ __forceinline__ float bf(uint32_t h) { return __uint_as_float(h << 16); }

// f32 -> bf16 (round to nearest even) -> f32
__device__ __forceinline__ float rb(float f) { return __bfloat162float(__float2bfloat16_rn(f)); }

__device__ __forceinline__ uint32_t bits(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }

struct GegluConsts {
    float cubic, tanh_approx;   // bf16(0.044715), bf16(0.7978845608028654)
};

// out[m, i] for i in [0, I); 8 elements per thread, 16-byte loads and stores (I % 8 == 0).
__global__ void __launch_bounds__(256) geglu_kernel(const uint16_t* __restrict__ gate, int64_t ldg,
                                                    const uint16_t* __restrict__ up, int64_t ldu,
                                                    uint16_t* __restrict__ out, int64_t ldo, int64_t M, int64_t I,
                                                    GegluConsts c) {
    const int64_t per_row = I / 8;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= M * per_row) return;
    const int64_t m = idx / per_row, i = (idx - m * per_row) * 8;
    const uint4 gv = *reinterpret_cast<const uint4*>(gate + m * ldg + i);
    const uint4 uv = *reinterpret_cast<const uint4*>(up + m * ldu + i);
    const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
    uint32_t ow[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t lo = geglu_bf16(bf(gw[j] & 0xFFFFu), bf(uw[j] & 0xFFFFu), c.cubic, c.tanh_approx);
        const uint32_t hi = geglu_bf16(bf(gw[j] >> 16), bf(uw[j] >> 16), c.cubic, c.tanh_approx);
        ow[j] = lo | (hi << 16);
    }
    *reinterpret_cast<uint4*>(out + m * ldo + i) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
}

constexpr int kNormThreads = 256;

// res / scale (optional): the tail of a layer's sub-block, out = bf16(bf16(res + norm) * scale)
// (native_model.cc:954-968: post_feedforward_layernorm, the residual add, layer_scalar; :920-926:
// post_attention_layernorm and its residual add, no scale). scale is a bf16 scalar in device memory.
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const uint16_t* x, int64_t ldx,
                                                                const uint16_t* __restrict__ w, int64_t K, float eps,
                                                                uint16_t* out, int64_t ldo,
                                                                const uint16_t* res, int64_t ldr,
                                                                const uint16_t* __restrict__ scale) {
    __shared__ float part[kNormThreads / 32];
    __shared__ float inv_s;
    const uint16_t* xr = x + (int64_t)blockIdx.x * ldx;
    uint16_t* orow = out + (int64_t)blockIdx.x * ldo;
    float ss = 0.0f;
    for (int64_t k = (int64_t)threadIdx.x * 8; k < K; k += kNormThreads * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
        const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float a = bf(vw[j] & 0xFFFFu), b = bf(vw[j] >> 16);
            ss = fmaf(a, a, ss);
            ss = fmaf(b, b, ss);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int i = 0; i < kNormThreads / 32; ++i) s += part[i];
        inv_s = __frsqrt_rn(s / (float)K + eps);
    }
    __syncthreads();
    const float inv = inv_s;
    const uint16_t* rrow = res != nullptr ? res + (int64_t)blockIdx.x * ldr : nullptr;
    const float sc = scale != nullptr ? bf(*scale) : 1.0f;
    for (int64_t k = (int64_t)threadIdx.x * 8; k < K; k += kNormThreads * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
        uint4 wv = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);   // bf16 1.0 pairs
        if (w != nullptr) wv = *reinterpret_cast<const uint4*>(w + k);
        uint4 rv = make_uint4(0u, 0u, 0u, 0u);
        if (rrow != nullptr) rv = *reinterpret_cast<const uint4*>(rrow + k);
        const uint32_t vw[4] = {v.x, v.y, v.z, v.w}, ww[4] = {wv.x, wv.y, wv.z, wv.w}, rw[4] = {rv.x, rv.y, rv.z, rv.w};
        uint32_t ow[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float lo = rb(bf(ww[j] & 0xFFFFu) * rb(bf(vw[j] & 0xFFFFu) * inv));
            float hi = rb(bf(ww[j] >> 16) * rb(bf(vw[j] >> 16) * inv));
            if (rrow != nullptr) {   // the residual add, then the layer scalar, each rounded to bf16
                lo = rb(bf(rw[j] & 0xFFFFu) + lo);
                hi = rb(bf(rw[j] >> 16) + hi);
                if (scale != nullptr) {
                    lo = lo * sc;
                    hi = hi * sc;
                }
            }
            ow[j] = bits(lo) | (bits(hi) << 16);
        }
        *reinterpret_cast<uint4*>(orow + k) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
}

}  // namespace

float bf16_round_host(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
    memcpy(&f, &u, 4);
    return f;
}

void launch_geglu(const uint16_t* gate, int64_t ldg, const uint16_t* up, int64_t ldu, uint16_t* out, int64_t ldo,
                  int64_t M, int64_t I, cudaStream_t st) {
    const int64_t total = M * (I / 8);
    if (total == 0) return;
    GegluConsts c;
    c.cubic = bf16_round_host(0.044715f);               // model_scalar(kGeluCubic)
    c.tanh_approx = bf16_round_host(0.7978845608028654f);   // model_scalar(kTanhApprox)
    geglu_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(gate, ldg, up, ldu, out, ldo, M, I, c);
    check_cuda(cudaGetLastError(), "geglu_kernel launch");
}

void launch_rms_norm(const uint16_t* x, int64_t ldx, const uint16_t* w, int64_t M, int64_t K, float eps,
                     uint16_t* out, int64_t ldo, cudaStream_t st, const uint16_t* res, int64_t ldr,
                     const uint16_t* scale) {
    if (M == 0) return;
    rms_norm_kernel<<<(unsigned)M, kNormThreads, 0, st>>>(x, ldx, w, K, eps, out, ldo, res, ldr, scale);
    check_cuda(cudaGetLastError(), "rms_norm_kernel launch");
}

}  // namespace g4q
