// g4q_gemv2.cu -- K1 v2: persistent stream-K decode GEMV (M <= 8) fed by per-warp TMA bulk rings.
//
// Same product as g4q_gemv.cu (bit-exact R2 dequant in registers, mma.sync bf16 -> fp32), organised
// for HBM streaming on B200:
//  * Work unit = one 64-wide quantization group of a "quad" of four 16-row tiles (64 rows): 2 KB of
//    packed words (contiguous in layout v1) + 256 B of scale|bias words.
//  * Persistent grid (one 12-warp CTA per SM). The (quad, group) space, quad-major, is cut into equal
//    contiguous ranges, one per warp: every SM streams the same number of bytes whatever N and K are.
//  * Each warp owns a private ring of kStages unit buffers in shared memory; lane 0 refills a buffer
//    with two cp.async.bulk copies on an mbarrier as soon as the warp has read it, so up to
//    kStages * 2.3 KB per warp (~110 KB per SM) are in flight without holding registers.
//  * x (M <= 8 tokens, full K) is staged once per CTA in B-fragment order while the first weight
//    copies are in flight; the RMS scale (sum of squares over K) is computed there too.
//  * A quad whose groups are split over several warps is reduced deterministically: each contributor
//    stores its fp32 partial in its own slot, bumps the quad's counter, and the last arriver sums the
//    slots in contributor order, applies the epilogue and resets the counter to zero.
#include "g4q_common.cuh"
#include "g4q_internal.h"

namespace g4q {
namespace {

constexpr int kWarpsV2 = 12;
constexpr int kThreadsV2 = kWarpsV2 * 32;
constexpr int kStages = 4;
constexpr uint32_t kUnitPacked = 4 * 512;     // four 16-row tiles x one group
constexpr uint32_t kUnitSb = 64 * 4;
constexpr uint32_t kUnitBytes = kUnitPacked + kUnitSb;
constexpr uint32_t kRingBytes = kStages * kUnitBytes;
constexpr long long kWaitLimitCycles2 = 4000000000ll;

struct Gemv2Args {
    const uint32_t* packed;
    const uint32_t* sb;
    int N, K, R, G, M, Q;   // Q = R / 4 quads
    long long U;            // Q * G units
    int TW;                 // total warps
    int maxc;               // slots per quad
    const uint16_t* x;
    int64_t ldx;
    void* y;
    int64_t ldy;
    uint32_t flags;
    float eps;
    float* slots;           // [Q][maxc][64 rows][M]
    int* counters;          // [Q], zero between launches
    int* err;
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool wait_parity(uint32_t bar, uint32_t parity, int* err) {
    const long long t0 = clock64();
    for (uint32_t it = 0;; ++it) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
        if ((it & 1023u) == 1023u && *reinterpret_cast<volatile int*>(err) != 0) return false;
        if (clock64() - t0 > kWaitLimitCycles2) {
            atomicCAS(err, 0, 16);
            return false;
        }
    }
}

__device__ __forceinline__ void issue_unit(const Gemv2Args& a, long long u, uint32_t dst, uint32_t bar) {
    const long long q = u / a.G;
    const long long g = u - q * a.G;
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

__device__ __forceinline__ long long range_start(long long w, long long U, int TW) { return (w * U) / TW; }

// warp index whose range contains unit u
__device__ __forceinline__ int warp_of_unit(long long u, long long U, int TW) {
    long long w = (u * TW) / U;
    while (w + 1 < TW && range_start(w + 1, U, TW) <= u) ++w;
    while (w > 0 && range_start(w, U, TW) > u) --w;
    return (int)w;
}

__device__ __forceinline__ void store_quad(const Gemv2Args& a, int q, const float (&acc)[4][4], const float* rs) {
    const int lane = threadIdx.x & 31, gi = lane >> 2, t = lane & 3;
    const bool f32 = (a.flags & G4Q_QMM_OUT_F32) != 0;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int tok = 2 * t + (e & 1);
            const int row = q * 64 + i * 16 + gi + ((e & 2) ? 8 : 0);
            if (tok < a.M) {
                const float v = __fmul_rn(acc[i][e], rs[tok]);
                if (f32)
                    reinterpret_cast<float*>(a.y)[(int64_t)tok * a.ldy + row] = v;
                else
                    reinterpret_cast<uint16_t*>(a.y)[(int64_t)tok * a.ldy + row] = f32_to_bf16_bits(v);
            }
        }
}

// A quad's partial from one warp: written to its slot; the last of the quad's contributors sums
// the slots in order and stores the result.
__device__ __forceinline__ void flush_quad(const Gemv2Args& a, int q, long long my_w, float (&acc)[4][4],
                                           const float* rs) {
    const int lane = threadIdx.x & 31, gi = lane >> 2, t = lane & 3;
    const long long u0 = (long long)q * a.G, u1 = u0 + a.G - 1;
    const long long ws = range_start(my_w, a.U, a.TW), we = range_start(my_w + 1, a.U, a.TW);
    if (ws <= u0 && we > u1) {   // this warp covered every group of the quad
        store_quad(a, q, acc, rs);
        return;
    }
    const int wf = warp_of_unit(u0, a.U, a.TW), wl = warp_of_unit(u1, a.U, a.TW);
    const int slot = (int)my_w - wf, nc = wl - wf + 1;
    float* base = a.slots + (size_t)q * a.maxc * 64 * 8;
    float* mine = base + (size_t)slot * 64 * 8;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int tok = 2 * t + (e & 1);
            const int row = i * 16 + gi + ((e & 2) ? 8 : 0);
            if (tok < a.M) mine[row * 8 + tok] = acc[i][e];
        }
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = (atomicAdd(a.counters + q, 1) == nc - 1);
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence();
    float sum[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) sum[i][e] = 0.0f;
    for (int s = 0; s < nc; ++s) {
        const float* src = base + (size_t)s * 64 * 8;
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int tok = 2 * t + (e & 1);
                const int row = i * 16 + gi + ((e & 2) ? 8 : 0);
                if (tok < a.M) sum[i][e] += __ldcg(src + row * 8 + tok);
            }
    }
    store_quad(a, q, sum, rs);
    __syncwarp();
    if (lane == 0) atomicExch(a.counters + q, 0);
}

__global__ void __launch_bounds__(kThreadsV2, 1) gemv2_kernel(Gemv2Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) unsigned long long bars[kWarpsV2][kStages];
    __shared__ float wss[kWarpsV2][8];
    __shared__ float rs[8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gi = lane >> 2, t = lane & 3;
    const long long my_w = (long long)blockIdx.x * kWarpsV2 + warp;
    const long long ub = range_start(my_w, a.U, a.TW), ue = range_start(my_w + 1, a.U, a.TW);
    uint8_t* ring = smem + (size_t)warp * kRingBytes;
    const uint32_t ring_s = smem_addr(ring);
    uint2* xf = reinterpret_cast<uint2*>(smem + (size_t)kWarpsV2 * kRingBytes);

    if (lane == 0) {
        for (int s = 0; s < kStages; ++s)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&bars[warp][s])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int s = 0; s < kStages && ub + s < ue; ++s)
            issue_unit(a, ub + s, ring_s + s * kUnitBytes, smem_addr(&bars[warp][s]));
    }
    __syncwarp();

    // stage x (full K, M <= 8 tokens) into B-fragment order and reduce sums of squares per token
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

    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][e] = 0.0f;
    int cur_q = ub < ue ? (int)(ub / a.G) : -1;
    const bool tok_ok = gi < a.M;

    for (long long u = ub; u < ue; ++u) {
        const int s = (int)((u - ub) % kStages);
        const uint32_t parity = (uint32_t)(((u - ub) / kStages) & 1);
        wait_parity(smem_addr(&bars[warp][s]), parity, a.err);
        const int q = (int)(u / a.G);
        const int g = (int)(u - (long long)q * a.G);
        if (q != cur_q) {
            flush_quad(a, cur_q, my_w, acc, rs);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[i][e] = 0.0f;
            cur_q = q;
        }
        const uint8_t* st = ring + s * kUnitBytes;
        uint4 wv[4];
        RowConsts c0[4], c1[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            wv[i] = reinterpret_cast<const uint4*>(st + i * 512)[lane];
            const uint32_t* sbw = reinterpret_cast<const uint32_t*>(st + kUnitPacked) + i * 16 + gi;
            c0[i] = row_consts(sbw[0]);
            c1[i] = row_consts(sbw[8]);
        }
        // every lane has its words in registers: lane 0 may refill this buffer
        __syncwarp();
        if (lane == 0 && u + kStages < ue) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue_unit(a, u + kStages, ring_s + s * kUnitBytes, smem_addr(&bars[warp][s]));
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint2 bf = make_uint2(0u, 0u);
            if (tok_ok) bf = xf[((g * 4 + j) * a.M + gi) * 4 + t];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t w = j == 0 ? wv[i].x : j == 1 ? wv[i].y : j == 2 ? wv[i].z : wv[i].w;
                const uint32_t a0 = deq_r2_fast(lop_nibbles(w), c0[i]);
                const uint32_t a1 = deq_r2_fast(lop_nibbles(w >> 4), c1[i]);
                const uint32_t a2 = deq_r2_fast(lop_nibbles(w >> 8), c0[i]);
                const uint32_t a3 = deq_r2_fast(lop_nibbles(w >> 12), c1[i]);
                mma_bf16_16816(acc[i], a0, a1, a2, a3, bf.x, bf.y);
            }
        }
    }
    if (cur_q >= 0) flush_quad(a, cur_q, my_w, acc, rs);
}

}  // namespace

size_t gemv2_slots_bytes(int64_t N, int64_t K, int sms) {
    const int64_t Q = N / 64, G = K / 64;
    const int64_t TW = (int64_t)sms * kWarpsV2;
    const int64_t per = (Q * G) / TW;
    const int64_t maxc = per >= 1 ? (G + per - 1) / per + 1 : G;
    return (size_t)Q * (size_t)(maxc < G ? maxc : G) * 64 * 8 * sizeof(float);
}

bool gemv2_supported(const QmmCall& c) {
    const size_t xbytes = (size_t)c.w->K * c.M * 2;
    const long long units = (c.w->N / 64) * (c.w->K / 64);
    // every warp of the grid must own at least one unit (empty ranges would stall a quad's reduction)
    return c.M >= 1 && c.M <= 8 && c.w->N % 64 == 0 && units >= kWarpsV2 &&
           (size_t)kWarpsV2 * kRingBytes + xbytes <= 200 * 1024;
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
    a.U = (long long)a.Q * a.G;
    int grid = sms;
    if ((long long)grid * kWarpsV2 > a.U) grid = (int)(a.U / kWarpsV2);   // >= 1 by gemv2_supported
    a.TW = grid * kWarpsV2;
    const long long per = a.U / a.TW;
    a.maxc = (int)(per >= 1 ? (a.G + per - 1) / per + 1 : a.G);
    if (a.maxc > a.G) a.maxc = a.G;
    const size_t need = (size_t)a.Q * a.maxc * 64 * 8 * sizeof(float);
    if (need > ds.slots_bytes)
        throw Error(G4Q_ERR_RUNTIME, "gemv scratch too small for this shape (allocate the weight before capture)");
    a.x = c.x;
    a.ldx = c.ldx;
    a.y = c.y;
    a.ldy = c.ldy;
    a.flags = c.flags;
    a.eps = c.eps;
    a.slots = ds.slots;
    a.counters = ds.counters;
    a.err = ds.err;
    const size_t smem = (size_t)kWarpsV2 * kRingBytes + (size_t)a.K * a.M * 2;
    gemv2_kernel<<<grid, kThreadsV2, smem, st>>>(a);
    check_cuda(cudaGetLastError(), "gemv2 launch");
}

}  // namespace g4q
