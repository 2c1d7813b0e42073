// g4q_gemm.cu -- K2: chunked-prefill quantized matmul (M > 16) on the 5th-generation tensor cores.
//
// Replaces mlx::core::quantized_matmul at the prefill call sites (native_model.cc:802-949 via
// forward_hidden / decode_block_hidden, :1682-1780; chunk loop :1819-1841).
//
// One CTA computes a 256-token x 256-row tile of y = x . deq(W)^T (cta_group::1, no clusters,
// every copy private to its CTA), warp-specialised over a 3-stage mbarrier pipeline with one 64-wide
// quantization group per k-step. Every dequantized weight tile feeds two M=128 MMAs (the two token
// halves), so the CUDA-core dequant work per tensor-core FLOP is half that of a 128-token tile:
//   warp 0      TMA producer: x tile [256 x 64] bf16 (tensor map, SWIZZLE_128B), the 8 KB packed
//               tile of 16 layout-v1 blocks (tensor map over 128-byte rows, SWIZZLE_128B so the
//               dequant reads are bank-conflict free) and the 1 KB scale|bias words.
//   warps 2..9  dequant, one weight row per thread: packed nibbles -> bit-exact bf16 (chain R2, two
//               bf16x2 ops per pair) written straight into the canonical K-major SWIZZLE_128B
//               layout of the B operand, then a generic->async proxy fence and an mbarrier arrive.
//   warp 1      allocates all 512 TMEM columns (two 128 x 256 fp32 accumulators); one thread
//               issues 2 x 4 tcgen05.mma (M=128, N=256, K=16, bf16 x bf16 -> fp32) per k-step and
//               tcgen05.commit frees the stage.
//   warps 2..9  epilogue: tcgen05.ld 32x32b.x32 -> optional RMS row scale -> bf16/fp32 -> global.
// Every mbarrier wait is bounded (clock64 limit); a timeout records an error code in a device word
// (read with g4q_device_error) and the CTA still runs to its end and frees its TMEM.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "g4q_common.cuh"
#include "g4q_internal.h"

namespace g4q {
namespace {

constexpr int BM = 256;                       // two M=128 MMA halves
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 3;
constexpr int kDequantWarps = 8;
constexpr int kGemmThreads = (2 + kDequantWarps) * 32;
constexpr uint32_t kXBytes = BM * BK * 2;     // 32 KB (two 16 KB halves of 128 rows)
constexpr uint32_t kBBytes = BN * BK * 2;     // 32 KB
constexpr uint32_t kPBytes = BN * BK / 2;     // 8 KB
constexpr uint32_t kSBBytes = BN * 4;         // 1 KB
constexpr uint32_t kStageBytes = kXBytes + kBBytes + kPBytes + kSBBytes;
constexpr uint32_t kSmemBytes = STAGES * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kXHalf = 128 * BK * 2;      // bytes of one 128-row half of the x tile
constexpr long long kWaitLimitCycles = 4000000000ll;   // ~2 s at 2 GHz

struct GemmParams {
    int M, N, K, R, KB;
    void* y;
    int64_t ldy;
    uint32_t flags;
    const float* rms;     // per-row scale or nullptr
    int vec_ok;
    int* err;
    int splits;           // > 1: split-K; blockIdx.z takes k-blocks [KB*z/splits, KB*(z+1)/splits) and
    float* part;          //      writes its unscaled fp32 tile to part + z*M*N (row stride N)
    int geglu;            // paired gate|up weight: y = geglu(gate, up), bf16 [M, N/2] (row stride ldy)
    float gk_cubic, gk_tanh;   // the GeGLU constants rounded to bf16
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Bounded wait on an mbarrier phase; returns false (and records `code`) after ~2 s. Once any
// wait on the device has given up (error word nonzero) every other wait returns at once, so a
// broken pipeline drains in one timeout instead of one per wait.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code) {
    const long long t0 = clock64();
    for (uint32_t it = 0;; ++it) {
        if ((it & 1023u) == 1023u && *reinterpret_cast<volatile int*>(err) != 0) return false;
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
        if (clock64() - t0 > kWaitLimitCycles) {
            atomicCAS(err, 0, code);
            return false;
        }
    }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// K-major SWIZZLE_128B UMMA shared-memory descriptor (tile base 1024-byte aligned):
// start address >> 4, LBO = 1 (unused for swizzled K-major), SBO = 1024 B between 8-row groups,
// version 1 (sm_100), layout type 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// kind::f16 instruction descriptor: D f32, A bf16, B bf16, both K-major, N = 256, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_p,
                 const __grid_constant__ CUtensorMap tm_sb, GemmParams p) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled tiles
    const uint32_t base_u32 = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t* base = smem_raw + (base_u32 - smem_u32(smem_raw));
    const uint32_t sX = base_u32;
    const uint32_t sB = sX + STAGES * kXBytes;
    const uint32_t sP = sB + STAGES * kBBytes;
    const uint32_t sSB = sP + STAGES * kPBytes;
    const uint32_t sBar = sSB + STAGES * kSBBytes;
    const uint32_t* sbw = reinterpret_cast<const uint32_t*>(base + (sSB - base_u32));
    auto full = [&](int s) { return sBar + 8u * s; };
    auto bfull = [&](int s) { return sBar + 8u * (STAGES + s); };
    auto empty = [&](int s) { return sBar + 8u * (2 * STAGES + s); };
    const uint32_t accum = sBar + 8u * (3 * STAGES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + (sBar - base_u32) + 8u * (3 * STAGES + 1));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    // this CTA's k-blocks (all of them unless split-K); i counts k-steps from kb_begin
    const int kb_begin = (int)((int64_t)p.KB * blockIdx.z / p.splits);
    const int nkb = (int)((int64_t)p.KB * (blockIdx.z + 1) / p.splits) - kb_begin;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full(s), 1);
            mbar_init(bfull(s), kDequantWarps);
            mbar_init(empty(s), 1);
        }
        mbar_init(accum, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer
        if (lane == 0) {
            for (int i = 0; i < nkb; ++i) {
                const int kb = kb_begin + i, s = i % STAGES;
                if (i >= STAGES) mbar_wait(empty(s), ((i / STAGES) - 1) & 1, p.err, 1);
                mbar_expect_tx(full(s), kXBytes + kPBytes + kSBBytes);
                tma_load_2d(sX + s * kXBytes, &tm_x, kb * BK, m0, full(s));
                tma_load_2d(sP + s * kPBytes, &tm_p, 0, (kb * p.R + n0 / 16) * 4, full(s));
                tma_load_2d(sSB + s * kSBBytes, &tm_sb, n0, kb, full(s));
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        for (int i = 0; i < nkb; ++i) {
            const int s = i % STAGES;
            const uint32_t ph = (i / STAGES) & 1;
            mbar_wait(full(s), ph, p.err, 2);
            mbar_wait(bfull(s), ph, p.err, 3);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (lane == 0) {
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    const uint64_t bd = umma_desc_sw128(sB + s * kBBytes + kk * 32);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {   // token rows 0-127 -> columns 0-255, 128-255 -> 256-511
                        const uint64_t ad = umma_desc_sw128(sX + s * kXBytes + h * kXHalf + kk * 32);
                        umma_bf16(tmem + (uint32_t)(h * BN), ad, bd, (i | kk) != 0);
                    }
                }
                umma_commit(empty(s));
            }
            __syncwarp();
        }
        if (lane == 0) umma_commit(accum);
        __syncwarp();
    } else {
        // ---------------- dequant warps (threads 64..319), one weight row each, then epilogue
        const int d = threadIdx.x - 64;
        const int rl = (d & 127) >> 3, gi = d & 7, half = d >> 7;   // 16-row tile, row pair, row of the pair
        const int nl = 16 * rl + gi + 8 * half;
        for (int i = 0; i < nkb; ++i) {
            const int s = i % STAGES;
            mbar_wait(full(s), (i / STAGES) & 1, p.err, 4);
            // packed words of lanes 4gi..4gi+3 of block rl: 64 logical bytes at rl*512 + gi*64,
            // stored by the 128B-swizzled TMA as chunk c of row rho at chunk c ^ (rho & 7)
            uint4 wv[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const uint32_t off = rl * 512 + gi * 64 + t * 16;
                const uint32_t rho = off >> 7, ch = (off >> 4) & 7;
                wv[t] = lds128(sP + s * kPBytes + rho * 128 + ((ch ^ (rho & 7)) << 4));
            }
            const uint32_t* sbs = sbw + s * (kSBBytes / 4);
            const RowConsts c = row_consts(sbs[nl]);
            const uint32_t bbase = sB + s * kBBytes + nl * 128;
            const int sh0 = 4 * half;   // row n0 uses nibble slots 0/2, row n1 slots 1/3
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t q[4][2];   // [t][lo/hi eight of the k16 step]
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const uint32_t w = (j == 0 ? wv[t].x : j == 1 ? wv[t].y : j == 2 ? wv[t].z : wv[t].w) >> sh0;
                    q[t][0] = deq_r2_fast(lop_nibbles(w), c);
                    q[t][1] = deq_r2_fast(lop_nibbles(w >> 8), c);
                }
                // row n: chunk (2j) holds k 16j..16j+7, chunk (2j+1) holds k 16j+8..16j+15
                const uint32_t c_lo = 2 * j, c_hi = 2 * j + 1;
                sts128(bbase + ((c_lo ^ (nl & 7)) << 4), make_uint4(q[0][0], q[1][0], q[2][0], q[3][0]));
                sts128(bbase + ((c_hi ^ (nl & 7)) << 4), make_uint4(q[0][1], q[1][1], q[2][1], q[3][1]));
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(bfull(s));
        }
        // ---------------- epilogue: TMEM lane quarter = warp % 4; warps 2..5 read the accumulator of
        //                  token rows 0-127, warps 6..9 that of rows 128-255 (columns 256..511)
        mbar_wait(accum, 0, p.err, 5);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int quarter = warp & 3, hm = (warp - 2) >> 2;
        const int row = m0 + hm * 128 + quarter * 32 + lane;
        const bool f32 = (p.flags & G4Q_QMM_OUT_F32) != 0;
        const float scale = (p.rms != nullptr && row < p.M) ? p.rms[row] : 1.0f;
        if (p.geglu && p.splits == 1) {
            // paired gate|up tile: quad j of the tile holds 32 gate rows (columns 64j..64j+31) and the
            // same 32 up rows (64j+32..64j+63); each output is geglu of the two bf16 matmul outputs,
            // rounded exactly as the unfused matmul followed by g4q_geglu rounds them
#pragma unroll 1
            for (int j = 0; j < BN / 64; ++j) {
#pragma unroll 1
                for (int h = 0; h < 2; ++h) {
                    uint32_t g[16], u[16];
                    const uint32_t col = (uint32_t)(hm * BN + 64 * j + 16 * h);
                    tmem_ld_32x32b_x16(tmem + ((uint32_t)(quarter * 32) << 16) + col, g);
                    tmem_ld_32x32b_x16(tmem + ((uint32_t)(quarter * 32) << 16) + col + 32, u);
                    if (row >= p.M || n0 + 64 * j >= p.N) continue;
                    uint32_t pk[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        uint32_t o2[2];
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const float gv = bf16_bits_to_f32(f32_to_bf16_bits(__fmul_rn(__uint_as_float(g[2 * i + e]), scale)));
                            const float uv = bf16_bits_to_f32(f32_to_bf16_bits(__fmul_rn(__uint_as_float(u[2 * i + e]), scale)));
                            o2[e] = geglu_bf16(gv, uv, p.gk_cubic, p.gk_tanh);
                        }
                        pk[i] = o2[0] | (o2[1] << 16);
                    }
                    uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.y) + (int64_t)row * p.ldy +
                                                        (n0 / 2 + 32 * j + 16 * h));
                    o[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    o[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                }
            }
        } else
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(hm * BN + c * 32), v);
            const int ncol = n0 + c * 32;
            if (row >= p.M || ncol >= p.N) continue;
            if (p.splits > 1) {   // unscaled fp32 partial; the reduction applies the epilogue
                float* pr = p.part + (int64_t)blockIdx.z * p.M * p.N + (int64_t)row * p.N + ncol;
                if (ncol + 32 <= p.N) {   // N % 16 == 0 keeps these 16-byte aligned
                    float4* o = reinterpret_cast<float4*>(pr);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        o[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                           __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
                } else {
                    for (int i = 0; i < 32; ++i)
                        if (ncol + i < p.N) pr[i] = __uint_as_float(v[i]);
                }
            } else if (f32) {
                float* yr = reinterpret_cast<float*>(p.y) + (int64_t)row * p.ldy + ncol;
                for (int i = 0; i < 32; ++i)
                    if (ncol + i < p.N) yr[i] = __fmul_rn(__uint_as_float(v[i]), scale);
            } else {
                uint16_t* yr = reinterpret_cast<uint16_t*>(p.y) + (int64_t)row * p.ldy + ncol;
                if (p.vec_ok && ncol + 32 <= p.N) {
                    uint32_t pk[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        pk[i] = (uint32_t)f32_to_bf16_bits(__fmul_rn(__uint_as_float(v[2 * i]), scale)) |
                                ((uint32_t)f32_to_bf16_bits(__fmul_rn(__uint_as_float(v[2 * i + 1]), scale)) << 16);
                    uint4* o = reinterpret_cast<uint4*>(yr);
#pragma unroll
                    for (int i = 0; i < 4; ++i) o[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
                } else {
                    for (int i = 0; i < 32; ++i)
                        if (ncol + i < p.N) yr[i] = f32_to_bf16_bits(__fmul_rn(__uint_as_float(v[i]), scale));
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// 1/sqrt(mean(x[m]^2) + eps) per row, one warp per row.
__global__ void rms_rows_kernel(const uint16_t* __restrict__ x, int M, int K, int64_t ldx, float eps,
                                float* __restrict__ out) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= M) return;
    const uint16_t* xr = x + (int64_t)warp * ldx;
    float ss = 0.0f;
    for (int k = lane * 8; k < K; k += 256) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float lo = bf16_bits_to_f32(w[i] & 0xffffu), hi = bf16_bits_to_f32(w[i] >> 16);
            ss = __fadd_rn(ss, __fmul_rn(lo, lo));
            ss = __fadd_rn(ss, __fmul_rn(hi, hi));
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
    if (lane == 0) out[warp] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
}

// Split-K reduction of a paired gate|up weight with the GeGLU epilogue: output o = 32j + i of row m is
// geglu(bf16(gate), bf16(up)) of columns 64j + i and 64j + 32 + i, each summed in split order and
// scaled by rms[m] exactly as the unsplit epilogue does. Four outputs per thread.
__global__ void splitk_reduce_geglu_kernel(const float* __restrict__ part, int splits, int M, int N, const float* rms,
                                           uint16_t* y, int64_t ldy, float cubic, float tanh_c) {
    const int m = blockIdx.y;
    const int o = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (o >= N / 2) return;
    const int j = o >> 5, i = o & 31;
    const int64_t total = (int64_t)M * N, ig = (int64_t)m * N + 64 * j + i, iu = ig + 32;
    float4 g = __ldcs(reinterpret_cast<const float4*>(part + ig)), u = __ldcs(reinterpret_cast<const float4*>(part + iu));
    for (int z = 1; z < splits; ++z) {
        const float4 tg = __ldcs(reinterpret_cast<const float4*>(part + (int64_t)z * total + ig));
        const float4 tu = __ldcs(reinterpret_cast<const float4*>(part + (int64_t)z * total + iu));
        g.x += tg.x;
        g.y += tg.y;
        g.z += tg.z;
        g.w += tg.w;
        u.x += tu.x;
        u.y += tu.y;
        u.z += tu.z;
        u.w += tu.w;
    }
    const float r = rms ? rms[m] : 1.0f;
    const float gs[4] = {g.x, g.y, g.z, g.w}, us[4] = {u.x, u.y, u.z, u.w};
    uint16_t* yr = y + (int64_t)m * ldy + o;
    for (int e = 0; e < 4; ++e) {
        const float gv = bf16_bits_to_f32(f32_to_bf16_bits(__fmul_rn(gs[e], r)));
        const float uv = bf16_bits_to_f32(f32_to_bf16_bits(__fmul_rn(us[e], r)));
        yr[e] = geglu_bf16(gv, uv, cubic, tanh_c);
    }
}

// Split-K reduction: y[m, n] = (sum over splits, in split order, of part[z][m][n]) * rms[m].
// One CTA row per output row (blockIdx.y), four columns per thread.
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int M, int N, const float* rms,
                                     void* y, int64_t ldy, int f32) {
    const int m = blockIdx.y;
    const int n = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (n >= N) return;
    const int64_t total = (int64_t)M * N, i = (int64_t)m * N + n;
    float4 s = __ldcs(reinterpret_cast<const float4*>(part + i));
    for (int z = 1; z < splits; ++z) {
        const float4 t = __ldcs(reinterpret_cast<const float4*>(part + (int64_t)z * total + i));
        s.x += t.x;
        s.y += t.y;
        s.z += t.z;
        s.w += t.w;
    }
    const float r = rms ? rms[m] : 1.0f;
    const float o[4] = {__fmul_rn(s.x, r), __fmul_rn(s.y, r), __fmul_rn(s.z, r), __fmul_rn(s.w, r)};
    if (f32) {
        float* yr = reinterpret_cast<float*>(y) + (int64_t)m * ldy + n;
        for (int e = 0; e < 4; ++e) yr[e] = o[e];
    } else {
        uint16_t* yr = reinterpret_cast<uint16_t*>(y) + (int64_t)m * ldy + n;
        for (int e = 0; e < 4; ++e) yr[e] = f32_to_bf16_bits(o[e]);
    }
}

struct SplitScratch {
    float* part = nullptr;
    size_t bytes = 0;
};
SplitScratch g_split[64];
std::mutex g_split_mu;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    if (!fn) throw Error(G4Q_ERR_RUNTIME, "cuTensorMapEncodeTiled is unavailable");
    return fn;
}

void make_map(CUtensorMap* m, CUtensorMapDataType dt, void* base, uint64_t d0, uint64_t d1, uint64_t stride1_bytes,
              uint32_t b0, uint32_t b1, CUtensorMapSwizzle sw) {
    const cuuint64_t dims[2] = {d0, d1};
    const cuuint64_t strides[1] = {stride1_bytes};
    const cuuint32_t box[2] = {b0, b1};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = encode_fn()(m, dt, 2, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw Error(G4Q_ERR_RUNTIME, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
}

}  // namespace

bool gemm_supported(const QmmCall& c) { return c.w->K % BK == 0; }

// Split-K when the tiles fill less than half of the SMs (small N, e.g. q|k|v or k/v shards under
// tensor parallelism): up to 8 splits of at least 4 k-blocks, so that tiles x splits <= SMs.
int gemm_splits(int64_t M, int64_t N, int64_t K) {
    const int tiles = (int)(((M + BM - 1) / BM) * ((N + BN - 1) / BN));
    const int sms = device_sm_count();
    int splits = 1;
    if (2 * tiles <= sms) {
        splits = sms / tiles;
        if (splits > 8) splits = 8;
        if (splits > (int)(K / BK) / 4) splits = (int)(K / BK) / 4;
        if (splits < 1) splits = 1;
    }
    return splits;
}

void launch_gemm(const QmmCall& c, cudaStream_t st) {
    static bool attr_set[64] = {false};
    const int dev = current_device();
    if (!attr_set[dev & 63]) {
        check_cuda(cudaFuncSetAttribute(qgemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes),
                   "cudaFuncSetAttribute(qgemm)");
        attr_set[dev & 63] = true;
    }
    const Weight& w = *c.w;
    DeviceScratch& ds = device_scratch();
    CUtensorMap tm_x, tm_p, tm_sb;
    make_map(&tm_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, const_cast<uint16_t*>(c.x), (uint64_t)w.K, (uint64_t)c.M,
             (uint64_t)c.ldx * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
    make_map(&tm_p, CU_TENSOR_MAP_DATA_TYPE_UINT32, w.packed, 32, (uint64_t)w.N * w.K / 256, 128, 32, BN * BK / 256,
             CU_TENSOR_MAP_SWIZZLE_128B);
    make_map(&tm_sb, CU_TENSOR_MAP_DATA_TYPE_UINT32, w.sb, (uint64_t)w.N, (uint64_t)(w.K / 64), (uint64_t)w.N * 4, BN,
             1, CU_TENSOR_MAP_SWIZZLE_NONE);
    GemmParams p;
    p.M = (int)c.M;
    p.N = (int)w.N;
    p.K = (int)w.K;
    p.R = (int)(w.N / 16);
    p.KB = (int)(w.K / BK);
    p.y = c.y;
    p.ldy = c.ldy;
    p.flags = c.flags;
    p.rms = nullptr;
    p.err = ds.err;
    const bool f32 = (c.flags & G4Q_QMM_OUT_F32) != 0;
    p.vec_ok = (!f32 && (reinterpret_cast<uintptr_t>(c.y) & 15u) == 0 && c.ldy % 8 == 0) ? 1 : 0;
    if (c.flags & G4Q_QMM_RMS_SCALE) {
        if (c.M > ds.rms_rows)
            throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, "RMS_SCALE supports at most " + std::to_string(ds.rms_rows) +
                                                        " rows per call");
        rms_rows_kernel<<<(int)((c.M * 32 + 255) / 256), 256, 0, st>>>(c.x, (int)c.M, (int)w.K, c.ldx, c.eps, ds.rms);
        check_cuda(cudaGetLastError(), "rms launch");
        p.rms = ds.rms;
    }
    const int splits = gemm_splits(c.M, w.N, w.K);
    p.splits = 1;
    p.part = nullptr;
    p.geglu = c.geglu ? 1 : 0;
    p.gk_cubic = bf16_round_host(0.044715f);
    p.gk_tanh = bf16_round_host(0.7978845608028654f);
    if (c.geglu && (w.N % 64 != 0 || (c.flags & G4Q_QMM_OUT_F32) || (reinterpret_cast<uintptr_t>(c.y) & 15u) ||
                    c.ldy % 8 != 0))
        throw Error(G4Q_ERR_INVALID_ARGUMENT, "GeGLU epilogue: rows % 64, bf16 out, 16-byte aligned rows");
    if (splits > 1) {
        const size_t need = (size_t)splits * c.M * w.N * sizeof(float);
        std::lock_guard<std::mutex> lock(g_split_mu);
        SplitScratch& ss = g_split[dev & 63];
        if (need > ss.bytes) {
            // grow only outside a stream capture (no allocation may be captured); else stay unsplit
            cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
            check_cuda(cudaStreamIsCapturing(st, &cap), "cudaStreamIsCapturing");
            if (cap == cudaStreamCaptureStatusNone) {
                // the smaller buffer is retired, not freed: a graph captured earlier may still
                // replay a split-K launch that writes it (it stays allocated until exit)
                float* grown = nullptr;
                check_cuda(cudaMalloc(&grown, need), "split-K scratch");
                ss.part = grown;
                ss.bytes = need;
            }
        }
        if (need <= ss.bytes) {
            p.splits = splits;
            p.part = ss.part;
        }
    }
    const dim3 grid((unsigned)((c.M + BM - 1) / BM), (unsigned)((w.N + BN - 1) / BN), (unsigned)p.splits);
    qgemm_kernel<<<grid, kGemmThreads, kSmemBytes, st>>>(tm_x, tm_p, tm_sb, p);
    check_cuda(cudaGetLastError(), "qgemm launch");
    if (p.splits > 1 && p.geglu) {
        const dim3 rgrid((unsigned)((w.N / 8 + 255) / 256), (unsigned)c.M);
        splitk_reduce_geglu_kernel<<<rgrid, 256, 0, st>>>(p.part, p.splits, (int)c.M, (int)w.N, p.rms,
                                                          static_cast<uint16_t*>(c.y), c.ldy, p.gk_cubic, p.gk_tanh);
        check_cuda(cudaGetLastError(), "split-K GeGLU reduction launch");
    } else if (p.splits > 1) {
        const dim3 rgrid((unsigned)((w.N / 4 + 255) / 256), (unsigned)c.M);
        splitk_reduce_kernel<<<rgrid, 256, 0, st>>>(p.part, p.splits, (int)c.M, (int)w.N, p.rms, c.y, c.ldy,
                                                    (c.flags & G4Q_QMM_OUT_F32) ? 1 : 0);
        check_cuda(cudaGetLastError(), "split-K reduction launch");
    }
}

}  // namespace g4q
