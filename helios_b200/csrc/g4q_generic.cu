// g4q_generic.cu -- quantized matmul and dequantize for weights kept in MLX's own layout: the
// 8-bit group-64 per-module override the reference's manifest allows (model_manifest.cc:146-152,
// looked up by quantization_for, native_model.cc:208-215), plus groups 32 and 128, which
// mlx::core::quantized_matmul / dequantize accept in general. Such modules are rare, so this path
// favours plain, exact code over speed: CUDA-core fp32 FMA over the bit-exact bf16 weights, one
// warp per output row.
//
// MLX layout: packed uint32 [N, K*bits/32] (element k of a row at bits*(k mod (32/bits)) of word
// k/(32/bits), little-endian), scales and biases bf16 [N, K/group]. Dequantized weight = chain
// R2 bf16(bf16(s*q) + b) (or R1 bf16(s*q + b)), the same arithmetic as g4q_dequantize_mlx.
#include "g4q_common.cuh"
#include "g4q_internal.h"

namespace g4q {
namespace {

constexpr int kGenThreads = 256;   // 8 warps, one output row each
constexpr int kGenTok = 8;         // tokens per pass over a row

__device__ __forceinline__ uint32_t deq_pair_mlx(uint32_t word, int e, int bits, uint32_t mask, uint32_t s2,
                                                 uint32_t b2, int chain) {
    const float qa = (float)((word >> (bits * e)) & mask);
    const float qb = (float)((word >> (bits * (e + 1))) & mask);
    const uint32_t q2 = (uint32_t)f32_to_bf16_bits(qa) | ((uint32_t)f32_to_bf16_bits(qb) << 16);
    return chain == 1 ? fma_bf16x2(q2, s2, b2) : add_bf16x2(mul_bf16x2(q2, s2), b2);
}

// y[m, n] = rs[m] * sum_k x[m, k] * deq(W)[n, k] for tokens m0 .. m0+7 (blockIdx.y picks m0)
__global__ void __launch_bounds__(kGenThreads) qmm_mlx_kernel(const uint32_t* __restrict__ w,
                                                              const uint16_t* __restrict__ s,
                                                              const uint16_t* __restrict__ b, int64_t N, int64_t K,
                                                              int bits, int gs, const uint16_t* __restrict__ x,
                                                              int64_t M, int64_t ldx, const float* __restrict__ rs,
                                                              void* y, int64_t ldy, uint32_t flags) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int per = 32 / bits;
    const int64_t wpr = K / per, G = K / gs;
    const uint32_t mask = (1u << bits) - 1u;
    const int64_t m0 = (int64_t)blockIdx.y * kGenTok;
    const int mt = (int)(M - m0 < kGenTok ? M - m0 : kGenTok);
    for (int64_t n = (int64_t)blockIdx.x * (kGenThreads / 32) + warp; n < N;
         n += (int64_t)gridDim.x * (kGenThreads / 32)) {
        float acc[kGenTok];
#pragma unroll
        for (int m = 0; m < kGenTok; ++m) acc[m] = 0.0f;
        const uint32_t* wr = w + n * wpr;
        for (int64_t kw = lane; kw < wpr; kw += 32) {
            const int64_t k0 = kw * per;
            const int64_t g = k0 / gs;   // one word never straddles a group (per divides gs)
            const uint32_t sv = s[n * G + g], bv = b[n * G + g];
            const uint32_t s2 = sv | (sv << 16), b2 = bv | (bv << 16);
            const uint32_t word = wr[kw];
            for (int e = 0; e < per; e += 2) {
                const uint32_t d = deq_pair_mlx(word, e, bits, mask, s2, b2, 2);
                const float w0 = bf16_bits_to_f32(d & 0xffffu), w1 = bf16_bits_to_f32(d >> 16);
#pragma unroll
                for (int m = 0; m < kGenTok; ++m)
                    if (m < mt) {
                        const uint32_t xv = *reinterpret_cast<const uint32_t*>(x + (m0 + m) * ldx + k0 + e);
                        acc[m] = fmaf(w0, bf16_bits_to_f32(xv & 0xffffu), acc[m]);
                        acc[m] = fmaf(w1, bf16_bits_to_f32(xv >> 16), acc[m]);
                    }
            }
        }
#pragma unroll
        for (int m = 0; m < kGenTok; ++m)
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], off);
        if (lane < mt) {
            float v = 0.0f;
#pragma unroll
            for (int m = 0; m < kGenTok; ++m)
                if (m == lane) v = acc[m];
            const int64_t row = m0 + lane;
            if (rs) v = __fmul_rn(v, rs[row]);
            if (flags & G4Q_QMM_OUT_F32)
                reinterpret_cast<float*>(y)[row * ldy + n] = v;
            else
                reinterpret_cast<uint16_t*>(y)[row * ldy + n] = f32_to_bf16_bits(v);
        }
    }
}

// 1/sqrt(mean(x[m]^2) + eps) per token row, one warp per row
__global__ void rms_rows_generic_kernel(const uint16_t* __restrict__ x, int64_t M, int64_t K, int64_t ldx, float eps,
                                        float* __restrict__ out) {
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= M) return;
    float ss = 0.0f;
    for (int64_t k = lane; k < K; k += 32) {
        const float v = bf16_bits_to_f32(x[row * ldx + k]);
        ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
    if (lane == 0) out[row] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
}

// gathered rows of the dequantized table (embedding lookup); ids outside [0, N) give a zero row
// and set bit 1 of the handle's flag word
__global__ void dequant_mlx_rows_kernel(const uint32_t* __restrict__ w, const uint16_t* __restrict__ s,
                                        const uint16_t* __restrict__ b, int64_t N, int64_t K, int bits, int gs,
                                        int chain, const int32_t* __restrict__ ids, int64_t n_ids,
                                        uint16_t* __restrict__ out, int* flags) {
    const int per = 32 / bits;
    const int64_t wpr = K / per, G = K / gs, words = n_ids * wpr;
    const uint32_t mask = (1u << bits) - 1u;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < words;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = idx / wpr, kw = idx - i * wpr;
        const int64_t k0 = kw * per;
        uint32_t* o = reinterpret_cast<uint32_t*>(out + i * K + k0);
        const int64_t n = ids[i];
        if (n < 0 || n >= N) {
            for (int e = 0; e < per / 2; ++e) o[e] = 0u;
            if (kw == 0) atomicOr(flags, 2);
            continue;
        }
        const int64_t g = k0 / gs;
        const uint32_t sv = s[n * G + g], bv = b[n * G + g];
        const uint32_t s2 = sv | (sv << 16), b2 = bv | (bv << 16);
        const uint32_t word = w[n * wpr + kw];
        for (int e = 0; e < per; e += 2) o[e >> 1] = deq_pair_mlx(word, e, bits, mask, s2, b2, chain);
    }
}

int grid_of(int64_t work, int per_block) {
    const int64_t g = (work + per_block - 1) / per_block;
    return (int)(g < 4 * 148 * 8 ? (g > 0 ? g : 1) : 4 * 148 * 8);
}

}  // namespace

void launch_qmm_mlx(const QmmCall& c, cudaStream_t st) {
    const Weight& w = *c.w;
    const float* rs = nullptr;
    if (c.flags & G4Q_QMM_RMS_SCALE) {
        DeviceScratch& ds = device_scratch();
        if (c.M > ds.rms_rows)
            throw Error(G4Q_ERR_UNSUPPORTED_CONFIG,
                        "RMS_SCALE supports at most " + std::to_string(ds.rms_rows) + " rows per call");
        rms_rows_generic_kernel<<<grid_of(c.M * 32, 256), 256, 0, st>>>(c.x, c.M, w.K, c.ldx, c.eps, ds.rms);
        check_cuda(cudaGetLastError(), "rms launch");
        rs = ds.rms;
    }
    const dim3 grid((unsigned)grid_of(w.N, kGenThreads / 32), (unsigned)((c.M + kGenTok - 1) / kGenTok));
    qmm_mlx_kernel<<<grid, kGenThreads, 0, st>>>(w.packed, w.mlx_scales, w.mlx_biases, w.N, w.K, w.bits,
                                                 w.group_size, c.x, c.M, c.ldx, rs, c.y, c.ldy, c.flags);
    check_cuda(cudaGetLastError(), "qmm (MLX layout) launch");
}

void launch_dequantize_mlx_rows(const Weight& w, const int32_t* ids, int64_t n_ids, uint16_t* out, int chain,
                                cudaStream_t st) {
    if (n_ids == 0) return;
    const int64_t words = n_ids * (w.K * w.bits / 32);
    dequant_mlx_rows_kernel<<<grid_of(words, 256), 256, 0, st>>>(w.packed, w.mlx_scales, w.mlx_biases, w.N, w.K,
                                                                 w.bits, w.group_size, chain, ids, n_ids, out,
                                                                 w.d_flags);
    check_cuda(cudaGetLastError(), "dequantize rows (MLX layout) launch");
}

}  // namespace g4q
