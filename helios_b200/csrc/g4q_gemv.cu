// g4q_gemv.cu -- K1: decode quantized GEMV for M <= 16 (M = 1 decode, M <= 15 MTP verify), and
// K4: the tied LM head with fused bf16 softcap + greedy argmax.
//
// Replaces mlx::core::quantized_matmul(x, W, s, b, transpose=true, 64, 4, "affine") at the
// decode/verify call sites (native_model.cc:993-1128, 1158-1281, 1318-1321, 1366-1369) and the
// LM head + argmax (native_model.cc:1782-1795, 3825).
//
// Design (B200):
//  * Weight streaming is the bound (0.5625 B per weight). Each warp owns one 16-row tile and a
//    range of 64-wide groups; per group one 16-byte streaming load per lane brings the whole
//    mma.m16n8k16 A fragment for 4 k16-steps (layout v1), plus one 32-bit scale|bias word per row.
//  * Dequantisation happens in registers and is bit-exact with chain R2:
//    (128+q) via one LOP3, RN(q*s) via fma.rn.bf16x2((128+q), s, -128*s), + bias via add.rn.bf16x2.
//    The bf16 weights then feed mma.sync with fp32 accumulation; tokens are the MMA's n dimension
//    (n = 8 per MMA, two MMAs for 9..16 tokens), so M <= 8 costs the same instructions as M = 1.
//  * x (the activations) is staged once per CTA into shared memory in B-fragment order.
//  * Split-K without global scratch: the S CTAs that share a 64-row chunk form one thread-block
//    cluster (1 x S x 1); partial sums (and partial sums of squares for the fused RMS scale) are
//    combined through distributed shared memory by cluster rank 0, in a fixed order.
#include <cooperative_groups.h>

#include <mutex>
#include <string>

#include "g4q_common.cuh"
#include "g4q_internal.h"

namespace cg = cooperative_groups;

namespace g4q {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxTokens = 16;
constexpr int kPrefetch = 4;  // groups of weights in flight per warp
constexpr uint32_t kFastScaleLimit = 247u << 7;   // bf16 |scale| >= 2^120 (exponent 127 + 120), inf, NaN

struct GemvArgs {
    const uint4* packed;
    const uint32_t* sb;
    int N, K, R, G, M;
    const uint16_t* x;
    int64_t ldx;
    void* y;
    int64_t ldy;
    uint32_t flags;
    float eps;
    int gps;  // groups per K-split
};

__host__ __device__ inline size_t xf_bytes(int gps, int M) { return (size_t)gps * M * 128; }
__host__ __device__ inline size_t gemv_smem_bytes(int gps, int M, int MT) {
    return xf_bytes(gps, M) + (size_t)kThreads * 4 * MT * 4 + (size_t)kThreads * kMaxTokens * 4 + kMaxTokens * 4;
}

// Stage x[:, 64*g0 .. 64*g1) into B-fragment order: entry (kk, m, t) holds the two bf16 pairs
// {x[m][16kk+2t..+1], x[m][16kk+2t+8..+9]} of lane (gi = m mod 8, t). Also per-thread partial
// sums of squares per token (deterministic reduction afterwards).
__device__ __forceinline__ void stage_x(const GemvArgs& a, int g0, int ng, uint2* xf, float* ssp, float* ssum) {
    const int tid = threadIdx.x;
    const bool rms = (a.flags & G4Q_QMM_RMS_SCALE) != 0;
    const int units = ng * 8;
#pragma unroll 1
    for (int m = 0; m < a.M; ++m) {
        float ss = 0.0f;
        const uint16_t* xr = a.x + (int64_t)m * a.ldx + (int64_t)g0 * 64;
        for (int u = tid; u < units; u += kThreads) {
            const uint4 v = *reinterpret_cast<const uint4*>(xr + u * 8);
            const int kk = u >> 1, h = u & 1;
            uint32_t* e = reinterpret_cast<uint32_t*>(xf + (kk * a.M + m) * 4);
            e[0 * 2 + h] = v.x;
            e[1 * 2 + h] = v.y;
            e[2 * 2 + h] = v.z;
            e[3 * 2 + h] = v.w;
            if (rms) {
                const uint32_t p[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float lo = bf16_bits_to_f32(p[q] & 0xffffu), hi = bf16_bits_to_f32(p[q] >> 16);
                    ss = __fadd_rn(ss, __fmul_rn(lo, lo));
                    ss = __fadd_rn(ss, __fmul_rn(hi, hi));
                }
            }
        }
        if (rms) ssp[m * kThreads + tid] = ss;
    }
    __syncthreads();
    if (rms && tid < a.M) {
        float s = 0.0f;
        for (int i = 0; i < kThreads; ++i) s = __fadd_rn(s, ssp[tid * kThreads + i]);
        ssum[tid] = s;
    }
    __syncthreads();
}

// One warp: acc += W[16r.., 64*g0 .. 64*(g0+ng)) . x^T for its 16-row tile r. kScan: also keep in
// scale_max the largest exponent-and-mantissa field (bits 7..14 | 0..6) of the scales it reads, so a
// caller whose weight has not been scanned at load time can tell whether every |scale| < 2^120.
template <int MT, bool kScan = false>
__device__ __forceinline__ void warp_tile(const GemvArgs& a, int r, int g0, int ng, const uint2* xf,
                                          float (&out)[MT][4], uint32_t* scale_max = nullptr) {
    const int lane = threadIdx.x & 31, gi = lane >> 2, t = lane & 3;
    float acc[2][MT][4];
#pragma unroll
    for (int s = 0; s < 2; ++s)
#pragma unroll
        for (int nt = 0; nt < MT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[s][nt][i] = 0.0f;

    const size_t wstride = (size_t)a.R * 32;
    const uint4* wp = a.packed + ((size_t)g0 * a.R + r) * 32 + lane;
    const uint32_t* sp = a.sb + (size_t)g0 * a.N + (size_t)r * 16 + gi;
    const size_t sstride = (size_t)a.N;

    uint4 wq[kPrefetch];
    uint32_t s0[kPrefetch], s1[kPrefetch];
#pragma unroll
    for (int i = 0; i < kPrefetch; ++i) {
        if (i < ng) {
            wq[i] = ldg_stream(wp + i * wstride);
            s0[i] = ldg_u32(sp + i * sstride);
            s1[i] = ldg_u32(sp + i * sstride + 8);
        }
    }
#pragma unroll 1
    for (int gb = 0; gb < ng; gb += kPrefetch) {
#pragma unroll
        for (int i = 0; i < kPrefetch; ++i) {
            const int gl = gb + i;
            if (gl < ng) {
                const uint4 w = wq[i];
                const RowConsts c0 = row_consts(s0[i]), c1 = row_consts(s1[i]);
                if constexpr (kScan) *scale_max = max(*scale_max, max(s0[i] & 0x7FFFu, s1[i] & 0x7FFFu));
                if (gl + kPrefetch < ng) {
                    wq[i] = ldg_stream(wp + (gl + kPrefetch) * wstride);
                    s0[i] = ldg_u32(sp + (gl + kPrefetch) * sstride);
                    s1[i] = ldg_u32(sp + (gl + kPrefetch) * sstride + 8);
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t word = j == 0 ? w.x : j == 1 ? w.y : j == 2 ? w.z : w.w;
                    const uint32_t a0 = deq_r2_fast(lop_nibbles(word), c0);
                    const uint32_t a1 = deq_r2_fast(lop_nibbles(word >> 4), c1);
                    const uint32_t a2 = deq_r2_fast(lop_nibbles(word >> 8), c0);
                    const uint32_t a3 = deq_r2_fast(lop_nibbles(word >> 12), c1);
                    const int kk = gl * 4 + j;
#pragma unroll
                    for (int nt = 0; nt < MT; ++nt) {
                        const int tok = nt * 8 + gi;
                        uint2 bf = make_uint2(0u, 0u);
                        if (tok < a.M) bf = xf[(kk * a.M + tok) * 4 + t];
                        mma_bf16_16816(acc[j & 1][nt], a0, a1, a2, a3, bf.x, bf.y);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int nt = 0; nt < MT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) out[nt][i] = acc[0][nt][i] + acc[1][nt][i];
}

__device__ __forceinline__ float rms_factor(const float* ssum, int tok, int K, float eps) {
    const float mean = __fdiv_rn(ssum[tok], (float)K);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

template <int MT>
__device__ __forceinline__ void store_tile(const GemvArgs& a, int r, const float (&out)[MT][4], const float* ssum) {
    const int lane = threadIdx.x & 31, gi = lane >> 2, t = lane & 3;
    const bool rms = (a.flags & G4Q_QMM_RMS_SCALE) != 0;
    const bool f32 = (a.flags & G4Q_QMM_OUT_F32) != 0;
#pragma unroll
    for (int nt = 0; nt < MT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int tok = nt * 8 + 2 * t + (i & 1);
            const int row = r * 16 + gi + ((i & 2) ? 8 : 0);
            if (tok < a.M) {
                float v = out[nt][i];
                if (rms) v = __fmul_rn(v, rms_factor(ssum, tok, a.K, a.eps));
                if (f32)
                    reinterpret_cast<float*>(a.y)[(int64_t)tok * a.ldy + row] = v;
                else
                    reinterpret_cast<uint16_t*>(a.y)[(int64_t)tok * a.ldy + row] = f32_to_bf16_bits(v);
            }
        }
}

template <int MT, bool kCluster>
__global__ void __launch_bounds__(kThreads) gemv_kernel(GemvArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int warp = threadIdx.x >> 5;
    const int split = blockIdx.y;
    const int g0 = split * a.gps;
    const int ng = min(a.G, g0 + a.gps) - g0;
    uint2* xf = reinterpret_cast<uint2*>(smem);
    float* red = reinterpret_cast<float*>(smem + xf_bytes(a.gps, a.M));
    float* ssp = red + kThreads * 4 * MT;
    float* ssum = ssp + kThreads * kMaxTokens;

    stage_x(a, g0, ng, xf, ssp, ssum);

    const int r = blockIdx.x * kWarps + warp;
    float out[MT][4];
    if (r < a.R) {
        warp_tile<MT>(a, r, g0, ng, xf, out);
    } else {
#pragma unroll
        for (int nt = 0; nt < MT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) out[nt][i] = 0.0f;
    }

    if constexpr (!kCluster) {
        if (r < a.R) store_tile<MT>(a, r, out, ssum);
    } else {
        cg::cluster_group cluster = cg::this_cluster();
#pragma unroll
        for (int nt = 0; nt < MT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) red[(nt * 4 + i) * kThreads + threadIdx.x] = out[nt][i];
        cluster.sync();
        if (cluster.block_rank() == 0) {
            const int S = (int)cluster.num_blocks();
            for (int q = 1; q < S; ++q) {
                const float* rr = cluster.map_shared_rank(red, q);
#pragma unroll
                for (int nt = 0; nt < MT; ++nt)
#pragma unroll
                    for (int i = 0; i < 4; ++i) out[nt][i] += rr[(nt * 4 + i) * kThreads + threadIdx.x];
            }
            if ((a.flags & G4Q_QMM_RMS_SCALE) && threadIdx.x < a.M) {
                float s = ssum[threadIdx.x];
                for (int q = 1; q < S; ++q) s = __fadd_rn(s, cluster.map_shared_rank(ssum, q)[threadIdx.x]);
                ssp[threadIdx.x] = s;  // reuse: cluster-wide sum of squares per token
            }
            __syncthreads();
            if (r < a.R) store_tile<MT>(a, r, out, ssp);
        }
        cluster.sync();
    }
}

// LM head: persistent over 16-row tiles, full K staged once, fused bf16 logits -> softcap ->
// argmax key; CTA-level reduction, one 64-bit atomicMax per token into the handle's scratch,
// and the last CTA to finish (ticket counter) publishes tokens/values/keys and resets the
// scratch to zero for the next call.
// kScan (the allocation-free entry point, whose caller-owned weight was never scanned at load):
// any scale that is non-finite or has |scale| >= 2^120 -- outside what the fast dequantisation
// handles -- records code 50 in the device error word (the results are then invalid).
template <int MT, bool kScan = false>
__global__ void __launch_bounds__(kThreads) lm_head_kernel(GemvArgs a, float cap, int64_t row_offset,
                                                           uint16_t* logits, int64_t ldl,
                                                           unsigned long long* scratch, int32_t* tokens,
                                                           float* values, unsigned long long* keys_out,
                                                           int* err) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ unsigned long long wbest[kWarps][kMaxTokens];
    __shared__ int is_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gi = lane >> 2, t = lane & 3;
    uint2* xf = reinterpret_cast<uint2*>(smem);
    float* ssp = reinterpret_cast<float*>(smem + xf_bytes(a.gps, a.M) + (size_t)kThreads * 4 * MT * 4);
    float* ssum = ssp + kThreads * kMaxTokens;
    stage_x(a, 0, a.G, xf, ssp, ssum);
    const bool rms = (a.flags & G4Q_QMM_RMS_SCALE) != 0;

    unsigned long long best[MT][2];
#pragma unroll
    for (int nt = 0; nt < MT; ++nt) best[nt][0] = best[nt][1] = 0ull;

    uint32_t scale_max = 0u;
    for (int r = blockIdx.x * kWarps + warp; r < a.R; r += gridDim.x * kWarps) {
        float out[MT][4];
        warp_tile<MT, kScan>(a, r, 0, a.G, xf, out, &scale_max);
#pragma unroll
        for (int nt = 0; nt < MT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int tok = nt * 8 + 2 * t + (i & 1);
                const int row = r * 16 + gi + ((i & 2) ? 8 : 0);
                if (tok < a.M) {
                    float v = out[nt][i];
                    if (rms) v = __fmul_rn(v, rms_factor(ssum, tok, a.K, a.eps));
                    const uint16_t lb = f32_to_bf16_bits(v);
                    if (logits) logits[(int64_t)tok * ldl + row] = lb;
                    const float lv = bf16_bits_to_f32(lb);
                    const float sv = cap > 0.0f ? softcap_bf16(lv, cap) : lv;
                    const unsigned long long key = argmax_key(sv, (uint32_t)(row_offset + row));
                    if (key > best[nt][i & 1]) best[nt][i & 1] = key;
                }
            }
    }
    if constexpr (kScan) {
        if (__any_sync(0xffffffffu, scale_max >= kFastScaleLimit) && lane == 0) atomicCAS(err, 0, 50);
    }
    // lanes sharing t hold the same tokens: reduce over gi (lane bits 2..4)
#pragma unroll
    for (int nt = 0; nt < MT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            unsigned long long k = best[nt][e];
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, off);
                k = o > k ? o : k;
            }
            best[nt][e] = k;
        }
    if (gi == 0) {
#pragma unroll
        for (int nt = 0; nt < MT; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int tok = nt * 8 + 2 * t + e;
                if (tok < kMaxTokens) wbest[warp][tok] = best[nt][e];
            }
    }
    __syncthreads();
    if (threadIdx.x < a.M) {
        unsigned long long k = 0ull;
        for (int w = 0; w < kWarps; ++w) k = wbest[w][threadIdx.x] > k ? wbest[w][threadIdx.x] : k;
        atomicMax(scratch + threadIdx.x, k);
        __threadfence();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned long long ticket = atomicAdd(scratch + kMaxTokens, 1ull);
        is_last = ticket == (unsigned long long)(gridDim.x - 1);
    }
    __syncthreads();
    if (is_last) {
        __threadfence();
        if (threadIdx.x < a.M) {
            const unsigned long long k = atomicExch(scratch + threadIdx.x, 0ull);
            if (tokens) tokens[threadIdx.x] = (int32_t)key_index(k);
            if (values) values[threadIdx.x] = key_value(k);
            if (keys_out) keys_out[threadIdx.x] = k;
        }
        __syncthreads();
        if (threadIdx.x == 0) atomicExch(scratch + kMaxTokens, 0ull);
    }
}

template <typename Kern>
void set_max_smem(Kern kern) {
    // once per process and kernel instance: opt in to the full 227 KB of dynamic shared memory
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)max_dynamic_smem(reinterpret_cast<const void*>(kern))),
               "cudaFuncSetAttribute(smem)");
}

template <typename Kern>
int occupancy(Kern kern, size_t smem) {
    int blocks = 0;
    check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kern, kThreads, smem), "occupancy");
    return blocks;
}

GemvArgs make_args(const Weight& w, const uint16_t* x, int64_t M, int64_t ldx, void* y, int64_t ldy, uint32_t flags,
                   float eps) {
    GemvArgs a;
    a.packed = reinterpret_cast<const uint4*>(w.packed);
    a.sb = w.sb;
    a.N = (int)w.N;
    a.K = (int)w.K;
    a.R = (int)(w.N / 16);
    a.G = (int)(w.K / 64);
    a.M = (int)M;
    a.x = x;
    a.ldx = ldx;
    a.y = y;
    a.ldy = ldy;
    a.flags = flags;
    a.eps = eps;
    a.gps = a.G;
    return a;
}

template <int MT>
void launch_gemv_t(GemvArgs a, cudaStream_t st) {
    static bool attr_set[64] = {false};
    const int dev = current_device();
    if (!attr_set[dev & 63]) {
        set_max_smem(gemv_kernel<MT, false>);
        set_max_smem(gemv_kernel<MT, true>);
        attr_set[dev & 63] = true;
    }
    const int sms = device_sm_count();
    const int chunks = (a.R + kWarps - 1) / kWarps;
    // K-split S (cluster size): the largest S <= 8 that keeps the launch in one wave of resident
    // CTAs with >= 4 groups per warp; S = 1 when the row chunks alone fill the GPU.
    int best_S = 1, best_gps = a.G;
    for (int S = 2; S <= 8 && S <= a.G; ++S) {
        const int gps = (a.G + S - 1) / S;
        const int S_eff = (a.G + gps - 1) / gps;
        if (S_eff != S || gps < 4) continue;
        const size_t smem = gemv_smem_bytes(gps, a.M, MT);
        if (smem > max_dynamic_smem(reinterpret_cast<const void*>(gemv_kernel<MT, true>))) continue;
        const int cap = occupancy(gemv_kernel<MT, true>, smem) * sms;
        if (chunks * S <= cap) {
            best_S = S;
            best_gps = gps;
        }
    }
    a.gps = best_gps;
    const size_t smem = gemv_smem_bytes(a.gps, a.M, MT);
    if (smem > max_dynamic_smem(reinterpret_cast<const void*>(gemv_kernel<MT, false>)))
        throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, "qmm: activation slice does not fit in shared memory");
    if (best_S == 1) {
        gemv_kernel<MT, false><<<dim3(chunks, 1), kThreads, smem, st>>>(a);
    } else {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(chunks, best_S, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = best_S;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        check_cuda(cudaLaunchKernelEx(&cfg, gemv_kernel<MT, true>, a), "cudaLaunchKernelEx(gemv)");
    }
    check_cuda(cudaGetLastError(), "gemv launch");
}

template <int MT, bool kScan = false>
void launch_lm_t(GemvArgs a, float cap, int64_t row_offset, uint16_t* logits, int64_t ldl,
                 unsigned long long* scratch, int32_t* tokens, float* values, unsigned long long* keys, int* err,
                 cudaStream_t st) {
    static bool attr_set[64] = {false};
    const int dev = current_device();
    if (!attr_set[dev & 63]) {
        set_max_smem(lm_head_kernel<MT, kScan>);
        attr_set[dev & 63] = true;
    }
    a.gps = a.G;
    const size_t smem = gemv_smem_bytes(a.G, a.M, MT);
    if (smem > max_dynamic_smem(reinterpret_cast<const void*>(lm_head_kernel<MT, kScan>)))
        throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, "lm_head: activations do not fit in shared memory");
    const int chunks = (a.R + kWarps - 1) / kWarps;
    int grid = occupancy(lm_head_kernel<MT, kScan>, smem) * device_sm_count();
    if (grid < 1) grid = 1;
    if (grid > chunks) grid = chunks;
    lm_head_kernel<MT, kScan><<<grid, kThreads, smem, st>>>(a, cap, row_offset, logits, ldl, scratch, tokens, values,
                                                           keys, err);
    check_cuda(cudaGetLastError(), "lm_head launch");
}

}  // namespace

void launch_gemv(const QmmCall& c, cudaStream_t st) {
    if (gemv2_supported(c)) {
        launch_gemv2(c, st);
        return;
    }
    GemvArgs a = make_args(*c.w, c.x, c.M, c.ldx, c.y, c.ldy, c.flags, c.eps);
    if (c.M <= 8)
        launch_gemv_t<1>(a, st);
    else
        launch_gemv_t<2>(a, st);
}

// ---- allocation-free LM head (g4q_lm_head_argmax_noalloc) --------------------------------------
// For callers that cannot allocate device memory at call time: code running inside a CUDA stream
// capture (cudaMalloc is not allowed there) and host runtimes that own every device byte through a
// pre-sized arena and forbid driver allocations once serving starts. The argmax scratch (16
// running keys + a ticket counter) lives in this static array instead of handle-owned memory.
// Every GPU that loads the library holds these 136 bytes until the process exits; all calls on a
// device share them, so calls that overlap on the GPU race and must be serialised by the caller.
// Word kMaxTokens + 1 is this entry point's own error word: the scale check below records code 50
// there (g4q_device_error reads it beside the library's error word), and the per-call clearing of
// the keys and the ticket leaves it alone.
constexpr int kNoAllocScratchWords = kMaxTokens + 1;
static __device__ __align__(256) unsigned long long g_noalloc_scratch[kNoAllocScratchWords + 1];

static unsigned long long* noalloc_scratch_ptr() {
    // The symbol's host-side name is only a stand-in: its device address is looked up once per
    // device (with that device current) on the first call, which must therefore precede any capture.
    static unsigned long long* ptrs[64] = {nullptr};
    static std::mutex mu;
    const int dev = current_device();
    std::lock_guard<std::mutex> lock(mu);
    if (ptrs[dev & 63] == nullptr) {
        void* p = nullptr;
        check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(noalloc scratch)");
        ptrs[dev & 63] = static_cast<unsigned long long*>(p);
    }
    return ptrs[dev & 63];
}

void launch_lm_head_noalloc(const uint32_t* packed, const uint32_t* sb, int64_t N, int64_t K, const uint16_t* x,
                            int64_t M, int64_t ldx, float softcap, uint32_t flags, float eps, int64_t row_offset,
                            uint16_t* logits, int64_t ld_logits, int32_t* tokens, float* values,
                            unsigned long long* keys, cudaStream_t st) {
    if (M < 1 || M > kMaxTokens)
        throw Error(G4Q_ERR_INVALID_ARGUMENT, "M must be in [1, " + std::to_string(kMaxTokens) +
                                                  "]: the static scratch holds " + std::to_string(kMaxTokens) + " keys");
    unsigned long long* scratch = noalloc_scratch_ptr();
    // the scratch keeps the previous call's contents: start from zero keys and a zero ticket
    check_cuda(cudaMemsetAsync(scratch, 0, sizeof(unsigned long long) * kNoAllocScratchWords, st),
               "cudaMemsetAsync(noalloc scratch)");
    Weight w;   // a view of caller memory: nothing is allocated
    w.N = N;
    w.K = K;
    w.packed = const_cast<uint32_t*>(packed);
    w.sb = const_cast<uint32_t*>(sb);
    GemvArgs a = make_args(w, x, M, ldx, nullptr, 0, flags, eps);
    // the caller's weight was never scanned at load time: the kernel checks the scales it reads
    int* err = reinterpret_cast<int*>(scratch + kNoAllocScratchWords);
    if (M <= 8)
        launch_lm_t<1, true>(a, softcap, row_offset, logits, ld_logits, scratch, tokens, values, keys, err, st);
    else
        launch_lm_t<2, true>(a, softcap, row_offset, logits, ld_logits, scratch, tokens, values, keys, err, st);
}

int noalloc_error(bool reset) {
    int v = 0;
    check_cuda(cudaMemcpyFromSymbol(&v, g_noalloc_scratch, sizeof(int), sizeof(unsigned long long) * kNoAllocScratchWords),
               "read the allocation-free LM head's error word");
    if (reset && v != 0) {
        const unsigned long long zero = 0ull;
        check_cuda(cudaMemcpyToSymbol(g_noalloc_scratch, &zero, sizeof(zero),
                                      sizeof(unsigned long long) * kNoAllocScratchWords),
                   "reset the allocation-free LM head's error word");
    }
    return v;
}

void launch_lm_head(const Weight& w, const uint16_t* x, int64_t M, int64_t ldx, float softcap, uint32_t flags,
                    float eps, int64_t row_offset, uint16_t* logits, int64_t ld_logits, int32_t* tokens,
                    float* values, unsigned long long* keys, cudaStream_t st) {
    GemvArgs a = make_args(w, x, M, ldx, nullptr, 0, flags, eps);
    if (M <= 8)
        launch_lm_t<1>(a, softcap, row_offset, logits, ld_logits, w.argmax_scratch, tokens, values, keys, nullptr, st);
    else
        launch_lm_t<2>(a, softcap, row_offset, logits, ld_logits, w.argmax_scratch, tokens, values, keys, nullptr, st);
}

}  // namespace g4q
