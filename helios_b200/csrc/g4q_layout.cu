// g4q_layout.cu -- loader repack (MLX layout -> kernel layout v1), its inverse, the bit-exact
// dequantize kernels and the seeded synthetic-data generator.
//
// Repack: the reference keeps MLX's `{prefix}.weight` uint32 [N, K/8] plus bf16 `.scales` /
// `.biases` [N, K/64] as loaded by NativeTextModel::load (native_model.cc:3506-3590). Here the
// load path rewrites them once into the layout described in g4q_common.cuh: the nibbles each
// tensor-core lane needs sit in one 16-byte word, and scale/bias of a row share one 32-bit word.
// Only the placement of nibbles changes; every q, scale and bias bit is kept (export inverts it).
#include "g4q_common.cuh"
#include "g4q_internal.h"

namespace g4q {
namespace {

__device__ __forceinline__ uint64_t rand64(uint64_t seed, uint64_t i) {
    uint64_t z = seed + (i + 1ull) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Irwin-Hall(12) normal, identical to the CPU oracle's normal_at: exact integer sum of twelve
// 16-bit uniforms, centred, times 2^-16.
__device__ __forceinline__ float normal_at(uint64_t seed, uint64_t i) {
    int64_t sum = 0;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        const uint64_t r = rand64(seed, 3ull * i + (uint64_t)j);
        sum += (int64_t)(r & 0xffffull) + (int64_t)((r >> 16) & 0xffffull) + (int64_t)((r >> 32) & 0xffffull) +
               (int64_t)(r >> 48);
    }
    return __fmul_rn((float)(sum - 393216), 1.0f / 65536.0f);
}

__global__ void synth_words_kernel(uint64_t seed, int64_t words, uint32_t* w) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < words; i += (int64_t)gridDim.x * blockDim.x)
        w[i] = (uint32_t)(rand64(seed, (uint64_t)i) >> 32);
}

__global__ void synth_groups_kernel(uint64_t seed_s, uint64_t seed_b, int64_t groups, uint16_t* s, uint16_t* b) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < groups; i += (int64_t)gridDim.x * blockDim.x) {
        const float u = __fmul_rn((float)(rand64(seed_s, (uint64_t)i) >> 40), 5.9604644775390625e-8f);
        const float sv = __fadd_rn(0.002f, __fmul_rn(u, 0.018f));
        const uint16_t sbits = f32_to_bf16_bits(sv);
        if (s) s[i] = sbits;
        if (b) {
            const float t1 = __fmul_rn(-8.0f, bf16_bits_to_f32(sbits));
            const float t2 = __fmul_rn(1e-3f, normal_at(seed_b, (uint64_t)i));
            b[i] = f32_to_bf16_bits(__fadd_rn(t1, t2));
        }
    }
}

__global__ void synth_normal_kernel(uint64_t seed, int64_t count, uint16_t* out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = f32_to_bf16_bits(normal_at(seed, (uint64_t)i));
}

// (lane, word j, slot) -> (row offset in tile, k offset in group); see g4q_common.cuh.
__device__ __forceinline__ void slot_coords(int lane, int j, int slot, int& dn, int& dk) {
    const int gi = lane >> 2, t = lane & 3, pair = slot & 3, hi = slot >> 2;
    dn = gi + ((pair & 1) ? 8 : 0);
    dk = 16 * j + 2 * t + hi + ((pair & 2) ? 8 : 0);
}

__global__ void repack_words_kernel(const uint32_t* __restrict__ src, int64_t src_ld_words, int64_t src_row0,
                                    int64_t src_k0, int64_t n_tiles, int64_t G, int64_t R, int64_t dst_tile0,
                                    uint32_t* __restrict__ packed) {
    const int64_t total = G * n_tiles * 128;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t g = idx / (n_tiles * 128);
        const int64_t rem = idx - g * n_tiles * 128;
        const int64_t rl = rem >> 7;
        const int lw = (int)(rem & 127), lane = lw >> 2, j = lw & 3;
        uint32_t word = 0;
#pragma unroll
        for (int slot = 0; slot < 8; ++slot) {
            int dn, dk;
            slot_coords(lane, j, slot, dn, dk);
            const int64_t srow = src_row0 + rl * 16 + dn;
            const int64_t sk = src_k0 + 64 * g + dk;
            const uint32_t sw = src[srow * src_ld_words + (sk >> 3)];
            word |= ((sw >> (4 * (sk & 7))) & 15u) << (4 * slot);
        }
        packed[(g * R + dst_tile0 + rl) * 128 + lw] = word;
    }
}

__global__ void repack_sb_kernel(const uint16_t* __restrict__ s, const uint16_t* __restrict__ b,
                                 int64_t src_ld_groups, int64_t src_row0, int64_t src_g0, int64_t n_rows, int64_t G,
                                 int64_t N, int64_t dst_row0, uint32_t* __restrict__ sb, int* flags) {
    const int64_t total = G * n_rows;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t g = idx / n_rows, n = idx - g * n_rows;
        const int64_t src = (src_row0 + n) * src_ld_groups + src_g0 + g;
        const uint32_t sv = s[src], bv = b[src];
        sb[g * N + dst_row0 + n] = sv | (bv << 16);
        // fast dequant path needs -128*s exact: |s| < 2^120 and finite (exponent field < 247);
        // the decode plan also scales s by 2^129 exactly: |s| < 2^-1 (exponent field < 126)
        const uint32_t e = (sv >> 7) & 0xFFu;
        if (e >= 126u) atomicOr(flags, e >= 247u ? 5 : 4);
        if (e == 0u && (sv & 0x7Fu) != 0u) atomicOr(flags, 8);   // subnormal: the plan scales s by an exponent add
    }
}

// The scale flags of repack_sb_kernel, recomputed over a whole sb array (weights opened from a
// cache file skip the repack).
__global__ void sb_flags_kernel(const uint32_t* __restrict__ sb, int64_t count, int* flags) {
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < count;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t e = (sb[idx] >> 7) & 0xFFu;
        if (e >= 126u) atomicOr(flags, e >= 247u ? 5 : 4);
        if (e == 0u && (sb[idx] & 0x7Fu) != 0u) atomicOr(flags, 8);
    }
}

__global__ void export_words_kernel(const uint32_t* __restrict__ packed, int64_t N, int64_t K,
                                    uint32_t* __restrict__ dst) {
    const int64_t R = N / 16, words = N * (K / 8);
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < words;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = idx / (K / 8), kw = idx - n * (K / 8);
        const int64_t r = n >> 4;
        const int rn = (int)(n & 15), gi = rn & 7, hrow = rn >> 3;
        uint32_t out = 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int64_t k = kw * 8 + e;
            const int64_t g = k >> 6;
            const int dk = (int)(k & 63), j = dk >> 4, kk = dk & 15;
            const int khalf = kk >> 3, t = (kk & 7) >> 1, hi = kk & 1;
            const int pair = (khalf << 1) | hrow, slot = pair + 4 * hi, lane = 4 * gi + t;
            const uint32_t w = packed[(g * R + r) * 128 + lane * 4 + j];
            out |= ((w >> (4 * slot)) & 15u) << (4 * e);
        }
        dst[idx] = out;
    }
}

__global__ void export_sb_kernel(const uint32_t* __restrict__ sb, int64_t N, int64_t G, uint16_t* s, uint16_t* b) {
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < N * G;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = idx / G, g = idx - n * G;
        const uint32_t w = sb[g * N + n];
        s[idx] = (uint16_t)(w & 0xffffu);
        b[idx] = (uint16_t)(w >> 16);
    }
}

// Whole-matrix dequantize from layout v1: one thread per (group g, row tile r, gi) unit,
// i.e. rows n0 = 16r+gi and n1 = n0+8 over the 64 columns of group g (64 packed bytes in,
// 256 bytes of bf16 out).
__global__ void dequant_layout_kernel(const uint32_t* __restrict__ packed, const uint32_t* __restrict__ sb,
                                      int64_t N, int64_t K, int chain, uint16_t* __restrict__ out) {
    const int64_t R = N / 16, G = K / 64, units = G * R * 8;
    for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units; u += (int64_t)gridDim.x * blockDim.x) {
        const int gi = (int)(u & 7);
        const int64_t r = (u >> 3) % R, g = (u >> 3) / R;
        const uint4* src = reinterpret_cast<const uint4*>(packed + (g * R + r) * 128) + 4 * gi;
        uint4 wv[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) wv[t] = src[t];
        const int64_t n0 = 16 * r + gi, n1 = n0 + 8;
        const uint32_t sb0 = sb[g * N + n0], sb1 = sb[g * N + n1];
        const uint32_t s0 = prmt(sb0, 0u, 0x1010u), b0 = prmt(sb0, 0u, 0x3232u);
        const uint32_t s1 = prmt(sb1, 0u, 0x1010u), b1 = prmt(sb1, 0u, 0x3232u);
        uint4* o0 = reinterpret_cast<uint4*>(out + n0 * K + 64 * g);
        uint4* o1 = reinterpret_cast<uint4*>(out + n1 * K + 64 * g);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t p[4][4];  // [t][pair]
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const uint32_t w = j == 0 ? wv[t].x : j == 1 ? wv[t].y : j == 2 ? wv[t].z : wv[t].w;
#pragma unroll
                for (int pr = 0; pr < 4; ++pr) {
                    const uint32_t qp = lop_nibbles(w >> (4 * pr));
                    p[t][pr] = (pr & 1) ? deq_general(qp, s1, b1, chain) : deq_general(qp, s0, b0, chain);
                }
            }
            o0[2 * j] = make_uint4(p[0][0], p[1][0], p[2][0], p[3][0]);
            o0[2 * j + 1] = make_uint4(p[0][2], p[1][2], p[2][2], p[3][2]);
            o1[2 * j] = make_uint4(p[0][1], p[1][1], p[2][1], p[3][1]);
            o1[2 * j + 1] = make_uint4(p[0][3], p[1][3], p[2][3], p[3][3]);
        }
    }
}

// Gathered rows (embedding lookup): one thread per (id index, group).
__global__ void dequant_rows_kernel(const uint32_t* __restrict__ packed, const uint32_t* __restrict__ sb,
                                    int64_t N, int64_t K, const int32_t* __restrict__ ids, int64_t n_ids,
                                    int chain, uint16_t* __restrict__ out, int* flags) {
    const int64_t R = N / 16, G = K / 64;
    for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < n_ids * G;
         u += (int64_t)gridDim.x * blockDim.x) {
        const int64_t ti = u / G, g = u - ti * G;
        const int64_t n = ids[ti];
        uint4* o = reinterpret_cast<uint4*>(out + ti * K + 64 * g);
        if (n < 0 || n >= N) {
            atomicOr(flags, 2);
#pragma unroll
            for (int c = 0; c < 8; ++c) o[c] = make_uint4(0, 0, 0, 0);
            continue;
        }
        const int64_t r = n >> 4;
        const int rn = (int)(n & 15), gi = rn & 7, hrow = rn >> 3;
        const uint4* src = reinterpret_cast<const uint4*>(packed + (g * R + r) * 128) + 4 * gi;
        const uint32_t sbw = sb[g * N + n];
        const uint32_t s2 = prmt(sbw, 0u, 0x1010u), b2 = prmt(sbw, 0u, 0x3232u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t lo[4], hi[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const uint4 wv = src[t];
                const uint32_t w = j == 0 ? wv.x : j == 1 ? wv.y : j == 2 ? wv.z : wv.w;
                lo[t] = deq_general(lop_nibbles(w >> (4 * hrow)), s2, b2, chain);
                hi[t] = deq_general(lop_nibbles(w >> (4 * (hrow + 2))), s2, b2, chain);
            }
            o[2 * j] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            o[2 * j + 1] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        }
    }
}

// MLX-layout dequantize (bits 4 or 8). q values become exact bf16 through fp32 (integers
// <= 255 are exact in bf16), then the chain runs in bf16x2 arithmetic.
__global__ void dequant_mlx_kernel(const uint32_t* __restrict__ w, const uint16_t* __restrict__ s,
                                   const uint16_t* __restrict__ b, int64_t N, int64_t K, int bits, int gs,
                                   int chain, uint16_t* __restrict__ out) {
    const int per = 32 / bits;
    const int64_t wpr = K / per, G = K / gs, words = N * wpr;
    const uint32_t mask = (1u << bits) - 1u;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < words;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = idx / wpr, kw = idx - n * wpr;
        const int64_t k0 = kw * per;
        const int64_t g = k0 / gs;
        const uint32_t sv = s[n * G + g], bv = b[n * G + g];
        const uint32_t s2 = sv | (sv << 16), b2 = bv | (bv << 16);
        const uint32_t word = w[idx];
        uint32_t res[4];
        for (int e = 0; e < per; e += 2) {
            const float qa = (float)((word >> (bits * e)) & mask);
            const float qb = (float)((word >> (bits * (e + 1))) & mask);
            const uint32_t q2 = (uint32_t)f32_to_bf16_bits(qa) | ((uint32_t)f32_to_bf16_bits(qb) << 16);
            res[e >> 1] = chain == 1 ? fma_bf16x2(q2, s2, b2) : add_bf16x2(mul_bf16x2(q2, s2), b2);
        }
        uint32_t* o = reinterpret_cast<uint32_t*>(out + n * K + k0);
        for (int e = 0; e < per / 2; ++e) o[e] = res[e];
    }
}

inline int grid_for(int64_t work, int threads = 256) {
    int64_t blocks = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)device_sm_count() * 32;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (int)blocks;
}

}  // namespace

void launch_synth_matrix(uint64_t seed, int64_t N, int64_t K, int bits, int group_size, uint32_t* w, uint16_t* s,
                         uint16_t* b, cudaStream_t st) {
    // sub-stream seeds: element 1, 2, 3 of the matrix seed's own stream (as the oracle)
    auto host_rand = [](uint64_t sd, uint64_t i) {
        uint64_t z = sd + (i + 1ull) * 0x9E3779B97F4A7C15ull;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    const uint64_t sw = host_rand(seed, 1), ss = host_rand(seed, 2), sbs = host_rand(seed, 3);
    const int64_t words = N * K * bits / 32, groups = N * (K / group_size);
    if (w) synth_words_kernel<<<grid_for(words), 256, 0, st>>>(sw, words, w);
    synth_groups_kernel<<<grid_for(groups), 256, 0, st>>>(ss, sbs, groups, s, b);
    check_cuda(cudaGetLastError(), "synth_matrix launch");
}

void launch_synth_normal(uint64_t seed, int64_t count, uint16_t* out, cudaStream_t st) {
    synth_normal_kernel<<<grid_for(count), 256, 0, st>>>(seed, count, out);
    check_cuda(cudaGetLastError(), "synth_normal launch");
}

void launch_repack(const uint32_t* src_w, const uint16_t* src_s, const uint16_t* src_b, int64_t src_ld_words,
                   int64_t src_ld_groups, int64_t src_row0, int64_t src_k0, int64_t n_rows, Weight& w,
                   int64_t dst_row0, cudaStream_t st) {
    const int64_t G = w.K / 64, R = w.N / 16, n_tiles = n_rows / 16;
    repack_words_kernel<<<grid_for(G * n_tiles * 128), 256, 0, st>>>(src_w, src_ld_words, src_row0, src_k0, n_tiles,
                                                                      G, R, dst_row0 / 16, w.packed);
    repack_sb_kernel<<<grid_for(G * n_rows), 256, 0, st>>>(src_s, src_b, src_ld_groups, src_row0, src_k0 / 64, n_rows,
                                                           G, w.N, dst_row0, w.sb, w.d_flags);
    check_cuda(cudaGetLastError(), "repack launch");
}

void launch_sb_flags(const Weight& w, cudaStream_t st) {
    const int64_t count = (w.K / 64) * w.N;
    sb_flags_kernel<<<grid_for(count), 256, 0, st>>>(w.sb, count, w.d_flags);
    check_cuda(cudaGetLastError(), "sb flags launch");
}

void launch_export(const Weight& w, uint32_t* dst_w, uint16_t* dst_s, uint16_t* dst_b, cudaStream_t st) {
    export_words_kernel<<<grid_for(w.N * w.K / 8), 256, 0, st>>>(w.packed, w.N, w.K, dst_w);
    export_sb_kernel<<<grid_for(w.N * w.K / 64), 256, 0, st>>>(w.sb, w.N, w.K / 64, dst_s, dst_b);
    check_cuda(cudaGetLastError(), "export launch");
}

void launch_dequantize(const Weight& w, const int32_t* ids, int64_t n_ids, uint16_t* out, int chain, int* d_err,
                       cudaStream_t st) {
    if (ids == nullptr) {
        dequant_layout_kernel<<<grid_for(w.K / 64 * (w.N / 16) * 8), 256, 0, st>>>(w.packed, w.sb, w.N, w.K, chain,
                                                                                   out);
    } else if (n_ids > 0) {
        dequant_rows_kernel<<<grid_for(n_ids * (w.K / 64)), 256, 0, st>>>(w.packed, w.sb, w.N, w.K, ids, n_ids, chain,
                                                                          out, d_err);
    }
    check_cuda(cudaGetLastError(), "dequantize launch");
}

void launch_dequantize_mlx(const uint32_t* wp, const uint16_t* s, const uint16_t* b, int64_t N, int64_t K, int bits,
                           int group_size, int chain, uint16_t* out, cudaStream_t st) {
    const int64_t words = N * K * bits / 32;
    dequant_mlx_kernel<<<grid_for(words), 256, 0, st>>>(wp, s, b, N, K, bits, group_size, chain, out);
    check_cuda(cudaGetLastError(), "dequantize_mlx launch");
}

}  // namespace g4q
