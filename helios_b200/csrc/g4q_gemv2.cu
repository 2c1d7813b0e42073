// g4q_gemv2.cu -- K1 v2: persistent stream-K decode GEMV (M <= 8) fed by per-warp TMA bulk rings.
//
// Same product as g4q_gemv.cu (bit-exact R2 dequant in registers, mma.sync bf16 -> fp32), organised
// for HBM streaming on B200:
//  * Work unit = one 64-wide quantization group of a "quad" of four 16-row tiles (64 rows): 2 KB of
//    packed words (contiguous in layout v1) + 256 B of scale|bias words.
//  * Persistent grid, one 16-warp CTA per SM. The (quad, group) unit space, quad-major, is cut into
//    equal contiguous CTA ranges, so every SM streams the same number of bytes whatever N and K are.
//    Inside a CTA the units of each quad go round-robin to the 16 warps.
//  * Each warp owns a private ring of kStages unit buffers in shared memory. Lane 0 refills a buffer
//    with two cp.async.bulk copies (mbarrier completion) as soon as the warp has the unit in
//    registers, running kStages units ahead through the warp's sequence, across quad boundaries.
//  * x (M <= 8 tokens, full K) is staged once per CTA in B-fragment order while the first weight
//    copies are in flight; the RMS scale (sum of squares over K) is reduced there too.
//  * Per quad the 16 warps' fp32 partials are summed in shared memory in warp order. A quad cut by
//    a CTA-range boundary (2-3 CTAs) is finished through global slots: each CTA stores its partial
//    in its own slot and bumps the quad's counter; the last arriver sums the slots in CTA order,
//    applies the epilogue and resets the counter to zero. Results are bit-reproducible.
#include "g4q_common.cuh"
#include "g4q_internal.h"

namespace g4q {
namespace {

constexpr int kWarpsV2 = 16;
constexpr int kThreadsV2 = kWarpsV2 * 32;
constexpr int kStages = 3;
constexpr uint32_t kUnitPacked = 4 * 512;     // four 16-row tiles x one group
constexpr uint32_t kUnitSb = 64 * 4;
constexpr uint32_t kUnitBytes = kUnitPacked + kUnitSb;
constexpr uint32_t kRingBytes = kStages * kUnitBytes;
constexpr uint32_t kRedBytesPerTok = kWarpsV2 * 64 * 4;
constexpr long long kWaitLimitCycles2 = 4000000000ll;

struct Gemv2Args {
    const uint32_t* packed;
    const uint32_t* sb;
    int N, K, R, G, M, Q;   // Q = R / 4 quads
    int U;                  // Q * G units
    const uint16_t* x;
    int64_t ldx;
    void* y;
    int64_t ldy;
    uint32_t flags;
    float eps;
    float* slots;           // [Q][maxc][64 rows][8 tokens]
    int maxc;
    int* counters;          // [Q], zero between launches
    int* err;
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void wait_parity(uint32_t bar, uint32_t parity, int* err) {
    const long long t0 = clock64();
    for (uint32_t it = 0;; ++it) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return;
        if ((it & 1023u) == 1023u && *reinterpret_cast<volatile int*>(err) != 0) return;
        if (clock64() - t0 > kWaitLimitCycles2) {
            atomicCAS(err, 0, 16);
            return;
        }
    }
}

__device__ __forceinline__ void issue_unit(const Gemv2Args& a, int q, int g, uint32_t dst, uint32_t bar) {
    const uint32_t* src_p = a.packed + ((size_t)g * a.R + (size_t)q * 4) * 128;
    const uint32_t* src_s = a.sb + (size_t)g * a.N + (size_t)q * 64;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(kUnitBytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src_p), "r"(kUnitPacked), "r"(bar)
                 : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     dst + kUnitPacked),
                 "l"(src_s), "r"(kUnitSb), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ int range_start(int c, int U, int C) { return (int)(((long long)c * U) / C); }

__device__ __forceinline__ int cta_of_unit(int u, int U, int C) {
    int c = (int)(((long long)u * C) / U);
    while (c + 1 < C && range_start(c + 1, U, C) <= u) ++c;
    while (c > 0 && range_start(c, U, C) > u) --c;
    return c;
}

// A warp's walk over its units: quads [q, q_last] of the CTA range [cs, ce), and inside each quad
// every kWarpsV2-th unit starting at the warp index.
struct Walk {
    int q, u, hi;
    bool done;
    __device__ __forceinline__ void settle(int G, int ce, int q_last, int w) {
        while (!done && u >= hi) {
            ++q;
            if (q > q_last) {
                done = true;
                break;
            }
            hi = min(ce, (q + 1) * G);
            u = q * G + w;
        }
    }
    __device__ __forceinline__ void init(int cs, int ce, int G, int q_first, int q_last, int w) {
        done = cs >= ce;
        q = q_first;
        hi = min(ce, (q + 1) * G);
        u = cs + w;
        settle(G, ce, q_last, w);
    }
    __device__ __forceinline__ void next(int G, int ce, int q_last, int w) {
        u += kWarpsV2;
        settle(G, ce, q_last, w);
    }
};

__global__ void __launch_bounds__(kThreadsV2, 1) gemv2_kernel(Gemv2Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) unsigned long long bars[kWarpsV2][kStages];
    __shared__ float wss[kWarpsV2][8];
    __shared__ float rs[8];
    __shared__ int last_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gi = lane >> 2, t = lane & 3;
    const int C = gridDim.x, cta = blockIdx.x;
    const int cs = range_start(cta, a.U, C), ce = range_start(cta + 1, a.U, C);
    const int G = a.G;
    const int q_first = cs / G, q_last = (ce - 1) / G;
    uint8_t* ring = smem + (size_t)warp * kRingBytes;
    const uint32_t ring_s = smem_addr(ring);
    float* red = reinterpret_cast<float*>(smem + (size_t)kWarpsV2 * kRingBytes);
    uint2* xf = reinterpret_cast<uint2*>(smem + (size_t)kWarpsV2 * kRingBytes + (size_t)kRedBytesPerTok * a.M);

    Walk pre;
    pre.init(cs, ce, G, q_first, q_last, warp);
    if (lane == 0) {
        for (int s = 0; s < kStages; ++s)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&bars[warp][s])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int s = 0; s < kStages && !pre.done; ++s) {
            issue_unit(a, pre.q, pre.u - pre.q * G, ring_s + s * kUnitBytes, smem_addr(&bars[warp][s]));
            pre.next(G, ce, q_last, warp);
        }
    } else {
        for (int s = 0; s < kStages && !pre.done; ++s) pre.next(G, ce, q_last, warp);
    }
    __syncwarp();

    // stage x (full K, M <= 8 tokens) into B-fragment order; sums of squares per token
    const bool rms = (a.flags & G4Q_QMM_RMS_SCALE) != 0;
    const int units8 = a.K / 8;
    for (int m = 0; m < a.M; ++m) {
        float ss = 0.0f;
        const uint16_t* xr = a.x + (int64_t)m * a.ldx;
        for (int u = threadIdx.x; u < units8; u += kThreadsV2) {
            const uint4 v = *reinterpret_cast<const uint4*>(xr + u * 8);
            const int kk = u >> 1, h = u & 1;
            uint32_t* e = reinterpret_cast<uint32_t*>(xf + (kk * a.M + m) * 4);
            e[0 + h] = v.x;
            e[2 + h] = v.y;
            e[4 + h] = v.z;
            e[6 + h] = v.w;
            if (rms) {
                const uint32_t pv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float lo = bf16_bits_to_f32(pv[i] & 0xffffu), hi = bf16_bits_to_f32(pv[i] >> 16);
                    ss = __fadd_rn(ss, __fmul_rn(lo, lo));
                    ss = __fadd_rn(ss, __fmul_rn(hi, hi));
                }
            }
        }
        if (rms) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
            if (lane == 0) wss[warp][m] = ss;
        }
    }
    __syncthreads();
    if (threadIdx.x < 8) {
        float r = 1.0f;
        if (rms && threadIdx.x < a.M) {
            float s = 0.0f;
            for (int w = 0; w < kWarpsV2; ++w) s = __fadd_rn(s, wss[w][threadIdx.x]);
            r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)a.K), a.eps)));
        }
        rs[threadIdx.x] = r;
    }
    __syncthreads();

    const bool tok_ok = gi < a.M;
    const bool f32 = (a.flags & G4Q_QMM_OUT_F32) != 0;
    Walk cur;
    cur.init(cs, ce, G, q_first, q_last, warp);
    int stage = 0;
    uint32_t phase = 0;
    for (int q = q_first; q <= q_last; ++q) {
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[i][e] = 0.0f;
        while (!cur.done && cur.q == q) {
            const int g = cur.u - q * G;
            wait_parity(smem_addr(&bars[warp][stage]), phase, a.err);
            const uint8_t* st = ring + stage * kUnitBytes;
            uint4 wv[4];
            uint32_t sb0[4], sb1[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                wv[i] = reinterpret_cast<const uint4*>(st + i * 512)[lane];
                const uint32_t* sbw = reinterpret_cast<const uint32_t*>(st + kUnitPacked) + i * 16 + gi;
                sb0[i] = sbw[0];
                sb1[i] = sbw[8];
            }
            // the unit is in registers: lane 0 refills this buffer with the warp's next-but-(kStages-1) unit
            __syncwarp();
            if (lane == 0 && !pre.done) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue_unit(a, pre.q, pre.u - pre.q * G, ring_s + stage * kUnitBytes, smem_addr(&bars[warp][stage]));
            }
            pre.next(G, ce, q_last, warp);
            if (++stage == kStages) {
                stage = 0;
                phase ^= 1u;
            }
            uint2 bf[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) bf[j] = tok_ok ? xf[((g * 4 + j) * a.M + gi) * 4 + t] : make_uint2(0u, 0u);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const RowConsts c0 = row_consts(sb0[i]), c1 = row_consts(sb1[i]);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t w = j == 0 ? wv[i].x : j == 1 ? wv[i].y : j == 2 ? wv[i].z : wv[i].w;
                    const uint32_t a0 = deq_r2_fast(lop_nibbles(w), c0);
                    const uint32_t a1 = deq_r2_fast(lop_nibbles(w >> 4), c1);
                    const uint32_t a2 = deq_r2_fast(lop_nibbles(w >> 8), c0);
                    const uint32_t a3 = deq_r2_fast(lop_nibbles(w >> 12), c1);
                    mma_bf16_16816(acc[i], a0, a1, a2, a3, bf[j].x, bf[j].y);
                }
            }
            cur.next(G, ce, q_last, warp);
        }
        // ---- reduce quad q over the 16 warps: red[tok][warp][row]
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int tok = 2 * t + (e & 1);
                const int row = i * 16 + gi + ((e & 2) ? 8 : 0);
                if (tok < a.M) red[(tok * kWarpsV2 + warp) * 64 + row] = acc[i][e];
            }
        __syncthreads();
        const int lo = max(cs, q * G), hi = min(ce, (q + 1) * G);
        const bool whole = lo == q * G && hi == (q + 1) * G;
        const int nout = 64 * a.M;
        float v = 0.0f;
        const int row = threadIdx.x & 63, tok = threadIdx.x >> 6;
        if (threadIdx.x < nout) {
            for (int w = 0; w < kWarpsV2; ++w) v += red[(tok * kWarpsV2 + w) * 64 + row];
        }
        if (whole) {
            if (threadIdx.x < nout) {
                const float o = __fmul_rn(v, rs[tok]);
                const int64_t idx = (int64_t)tok * a.ldy + q * 64 + row;
                if (f32)
                    reinterpret_cast<float*>(a.y)[idx] = o;
                else
                    reinterpret_cast<uint16_t*>(a.y)[idx] = f32_to_bf16_bits(o);
            }
        } else {
            const int cf = cta_of_unit(q * G, a.U, C), cl = cta_of_unit((q + 1) * G - 1, a.U, C);
            const int nc = cl - cf + 1;
            float* base = a.slots + (size_t)q * a.maxc * 64 * 8;
            if (threadIdx.x < nout) base[(size_t)(cta - cf) * 512 + row * 8 + tok] = v;
            __threadfence();
            __syncthreads();
            if (threadIdx.x == 0) last_flag = (atomicAdd(a.counters + q, 1) == nc - 1);
            __syncthreads();
            if (last_flag) {
                __threadfence();
                if (threadIdx.x < nout) {
                    float s = 0.0f;
                    for (int c = 0; c < nc; ++c) s += __ldcg(base + (size_t)c * 512 + row * 8 + tok);
                    const float o = __fmul_rn(s, rs[tok]);
                    const int64_t idx = (int64_t)tok * a.ldy + q * 64 + row;
                    if (f32)
                        reinterpret_cast<float*>(a.y)[idx] = o;
                    else
                        reinterpret_cast<uint16_t*>(a.y)[idx] = f32_to_bf16_bits(o);
                }
                if (threadIdx.x == 0) atomicExch(a.counters + q, 0);
            }
        }
        __syncthreads();   // red is rewritten by the next quad
    }
}

}  // namespace

size_t gemv2_slots_bytes(int64_t N, int64_t K, int sms) {
    (void)K;
    (void)sms;
    // 8 slots of 64 rows x 8 tokens fp32 per 64-row quad (launch_gemv2 keeps contributors <= 8)
    return (size_t)(N / 64) * 8 * 64 * 8 * sizeof(float);
}

bool gemv2_supported(const QmmCall& c) {
    const size_t xbytes = (size_t)c.w->K * c.M * 2;
    const long long units = (c.w->N / 64) * (c.w->K / 64);
    return c.M >= 1 && c.M <= 8 && c.w->N % 64 == 0 && units >= 1 && units < (1ll << 31) &&
           (size_t)kWarpsV2 * kRingBytes + (size_t)kRedBytesPerTok * c.M + xbytes <= 220 * 1024;
}

void launch_gemv2(const QmmCall& c, cudaStream_t st) {
    static bool attr_set[64] = {false};
    const int dev = current_device();
    if (!attr_set[dev & 63]) {
        check_cuda(cudaFuncSetAttribute(gemv2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)max_dynamic_smem(reinterpret_cast<const void*>(gemv2_kernel))),
                   "cudaFuncSetAttribute(gemv2)");
        attr_set[dev & 63] = true;
    }
    const Weight& w = *c.w;
    DeviceScratch& ds = device_scratch();
    const int sms = device_sm_count();
    Gemv2Args a;
    a.packed = w.packed;
    a.sb = w.sb;
    a.N = (int)w.N;
    a.K = (int)w.K;
    a.R = (int)(w.N / 16);
    a.G = (int)(w.K / 64);
    a.M = (int)c.M;
    a.Q = a.R / 4;
    a.U = a.Q * a.G;
    // every CTA owns at least one unit, and a quad (G units) meets at most (G-1)/min_range + 2 CTA
    // ranges: shrink the grid until that is within the 8 slots reserved per quad
    int grid = sms < a.U ? sms : a.U;
    while (grid > 1 && (a.G - 1) / (a.U / grid) + 2 > 8) --grid;
    if ((size_t)a.Q * 8 * 64 * 8 * sizeof(float) > ds.slots_bytes)
        throw Error(G4Q_ERR_RUNTIME, "gemv scratch too small for this shape (create the weight before capture)");
    a.x = c.x;
    a.ldx = c.ldx;
    a.y = c.y;
    a.ldy = c.ldy;
    a.flags = c.flags;
    a.eps = c.eps;
    a.slots = ds.slots;
    a.maxc = 8;
    a.counters = ds.counters;
    a.err = ds.err;
    const size_t smem = (size_t)kWarpsV2 * kRingBytes + (size_t)kRedBytesPerTok * a.M + (size_t)a.K * a.M * 2;
    gemv2_kernel<<<grid, kThreadsV2, smem, st>>>(a);
    check_cuda(cudaGetLastError(), "gemv2 launch");
}

}  // namespace g4q
