// g4q_lora.cu -- the LoRA delta added to a quantized linear's output (sm_100a).
//
// Restates add_lora_delta_if_active (native/gemma4_mlx/src/native_model.cc:316-328):
//   low   = matmul(f32(x), a_transposed)                 fp32 [M, rank]
//   delta = matmul(low, b_transposed) * bf16(scale)      fp32 [M, N] (fp32 x bf16 scalar -> fp32)
//   y     = bf16(y_base + bf16(delta))                   the bf16 add of two bf16 arrays
// with scale = alpha / rank (native_model.cc:3378) and the adapter matrices converted to fp32 at
// load (:3419-3420). The base output y is the bf16 result of the quantized matmul; the delta is
// added in place.
//
// Two launches per chunk of tokens: lora_down (one warp per rank row, the x row read with
// 16-byte loads, four tokens per CTA so each A row is read once per four tokens) writes the fp32
// low-rank activations to the handle's scratch; lora_up (one thread per output feature, eight
// tokens per CTA, the low-rank rows staged in shared memory, B kept transposed [rank][N] so a
// warp's loads are coalesced) forms the delta and applies the two bf16 roundings. Both are
// CUDA-core fp32 work: rank <= 256 makes the delta ~rank/2 FLOP per output element, far below
// what the quantized matmul itself costs.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "g4q_internal.h"

namespace g4q {
namespace {

constexpr int kDownTokens = 4;    // tokens per lora_down CTA
constexpr int kDownWarps = 8;     // rank rows per lora_down CTA
constexpr int kUpTokens = 8;      // tokens per lora_up CTA
constexpr int kUpThreads = 256;   // output features per lora_up CTA

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// low[m, j] = sum_k f32(x[m, k]) * a[j, k]; K % 8 == 0, x rows 16-byte aligned (checked by the host).
__global__ void __launch_bounds__(kDownWarps * 32) lora_down_kernel(const uint16_t* __restrict__ x, int64_t ldx,
                                                                  int M, int64_t K, const float* __restrict__ a,
                                                                  int rank, float* __restrict__ low) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j = blockIdx.x * kDownWarps + warp;
    const int m0 = blockIdx.y * kDownTokens;
    if (j >= rank) return;
    const float* arow = a + (int64_t)j * K;
    float acc[kDownTokens];
#pragma unroll
    for (int t = 0; t < kDownTokens; ++t) acc[t] = 0.f;
    for (int64_t k = (int64_t)lane * 8; k < K; k += 256) {
        const float4 a0 = __ldg(reinterpret_cast<const float4*>(arow + k));
        const float4 a1 = __ldg(reinterpret_cast<const float4*>(arow + k + 4));
#pragma unroll
        for (int t = 0; t < kDownTokens; ++t) {
            if (m0 + t < M) {
                const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + (int64_t)(m0 + t) * ldx + k));
                float s = acc[t];
                s = fmaf(bf16_bits_to_f32(xv.x & 0xFFFFu), a0.x, s);
                s = fmaf(bf16_bits_to_f32(xv.x >> 16), a0.y, s);
                s = fmaf(bf16_bits_to_f32(xv.y & 0xFFFFu), a0.z, s);
                s = fmaf(bf16_bits_to_f32(xv.y >> 16), a0.w, s);
                s = fmaf(bf16_bits_to_f32(xv.z & 0xFFFFu), a1.x, s);
                s = fmaf(bf16_bits_to_f32(xv.z >> 16), a1.y, s);
                s = fmaf(bf16_bits_to_f32(xv.w & 0xFFFFu), a1.z, s);
                s = fmaf(bf16_bits_to_f32(xv.w >> 16), a1.w, s);
                acc[t] = s;
            }
        }
    }
#pragma unroll
    for (int t = 0; t < kDownTokens; ++t) {
        float s = acc[t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
        if (lane == 0 && m0 + t < M) low[(int64_t)(m0 + t) * rank + j] = s;
    }
}

// y[m, n] = bf16(f32(y[m, n]) + f32(bf16(f32(sum_j low[m, j] * bt[j, n]) * scale))).
__global__ void __launch_bounds__(kUpThreads) lora_up_kernel(const float* __restrict__ low, int M, int rank,
                                                            const float* __restrict__ bt, int64_t N, float scale,
                                                            uint16_t* __restrict__ y, int64_t ldy) {
    extern __shared__ float low_s[];   // [kUpTokens][rank]
    const int m0 = blockIdx.y * kUpTokens;
    const int tokens = min(kUpTokens, M - m0);
    for (int i = threadIdx.x; i < tokens * rank; i += kUpThreads) low_s[i] = low[(int64_t)m0 * rank + i];
    __syncthreads();
    const int64_t n = (int64_t)blockIdx.x * kUpThreads + threadIdx.x;
    if (n >= N) return;
    float acc[kUpTokens];
#pragma unroll
    for (int t = 0; t < kUpTokens; ++t) acc[t] = 0.f;
    for (int j = 0; j < rank; ++j) {
        const float b = __ldg(bt + (int64_t)j * N + n);
#pragma unroll
        for (int t = 0; t < kUpTokens; ++t) acc[t] = fmaf(low_s[t * rank + j], b, acc[t]);
    }
#pragma unroll
    for (int t = 0; t < kUpTokens; ++t) {
        if (t < tokens) {
            uint16_t* p = y + (int64_t)(m0 + t) * ldy + n;
            const float delta = bf16_bits_to_f32(f32_to_bf16_bits(acc[t] * scale));
            *p = f32_to_bf16_bits(bf16_bits_to_f32(*p) + delta);
        }
    }
}

// bt[j, n] = b[n, j]: the load-time transpose of lora_B [N][rank] into [rank][N].
__global__ void lora_transpose_kernel(const float* __restrict__ b, int64_t N, int rank, float* __restrict__ bt) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N * rank) return;
    const int64_t j = i / N, n = i - j * N;
    bt[i] = b[n * rank + j];
}

}  // namespace

void launch_lora_transpose(const float* b, int64_t N, int rank, float* bt, cudaStream_t st) {
    const int64_t total = N * rank;
    if (total == 0) return;
    lora_transpose_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(b, N, rank, bt);
    check_cuda(cudaGetLastError(), "lora_transpose_kernel launch");
}

void launch_lora_apply(const Lora& l, const uint16_t* x, int64_t M, int64_t ldx, uint16_t* y, int64_t ldy,
                       cudaStream_t st) {
    const size_t smem = (size_t)kUpTokens * l.rank * sizeof(float);
    for (int64_t m0 = 0; m0 < M; m0 += l.max_tokens) {
        const int mc = (int)((M - m0) < l.max_tokens ? (M - m0) : l.max_tokens);
        dim3 gd((unsigned)((l.rank + kDownWarps - 1) / kDownWarps), (unsigned)((mc + kDownTokens - 1) / kDownTokens));
        lora_down_kernel<<<gd, kDownWarps * 32, 0, st>>>(x + m0 * ldx, ldx, mc, l.K, l.a, l.rank, l.low);
        check_cuda(cudaGetLastError(), "lora_down_kernel launch");
        dim3 gu((unsigned)((l.N + kUpThreads - 1) / kUpThreads), (unsigned)((mc + kUpTokens - 1) / kUpTokens));
        lora_up_kernel<<<gu, kUpThreads, smem, st>>>(l.low, mc, l.rank, l.bt, l.N, l.scale_bf16, y + m0 * ldy, ldy);
        check_cuda(cudaGetLastError(), "lora_up_kernel launch");
    }
}

}  // namespace g4q
