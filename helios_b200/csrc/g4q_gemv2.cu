// g4q_gemv2.cu -- K1 v2: persistent stream-K decode GEMV (M <= 8) fed by per-warp TMA bulk rings.
//
// Same product as g4q_gemv.cu (bit-exact R2 dequant in registers, mma.sync bf16 -> fp32 with the
// tokens as the n dimension), organised for HBM streaming on B200:
//  * Work unit = one 64-wide quantization group of a "quad" of four 16-row tiles (64 rows): 2 KB of
//    packed words (contiguous in layout v1) + 256 B of scale|bias words.
//  * Persistent grid, one 16-warp CTA per SM. The (quad, group) unit space, quad-major, is cut into
//    equal contiguous CTA ranges, so every SM streams the same number of bytes whatever N and K are;
//    inside a CTA each warp owns a contiguous run of units (counts differ by at most one), so a
//    warp meets at most two quads that other warps share.
//  * Each warp owns a private ring of 3 unit buffers in shared memory (2 when the tokens' x would not
//    fit beside 3). Lane 0 refills a buffer with two cp.async.bulk copies (mbarrier completion) as
//    soon as the warp has read the unit.
//  * x (M <= 8 tokens) is staged once per CTA, per token in B-fragment order (two 16-byte loads per
//    lane and unit), while the first weight copies land: all of K, or only the window of groups the
//    CTA's range reads when every range is shorter than a quad row (long K, e.g. down_proj), which
//    lets more tokens fit; the per-token RMS scale (sum of squares over K) is reduced there too.
//  * Weights whose |scales| are all < 2^-1 take the raw odd-nibble dequant (the masked bits read as
//    bf16 are q * 2^-129, times s * 2^129): two operations fewer per packed word.
//  * A warp parks its fp32 partial of a quad in shared memory when it leaves the quad; the last warp
//    of a shared quad sums the partials in warp order, so no warp ever waits. A quad cut by a
//    CTA-range boundary is finished through global slots: each CTA stores its partial in its own
//    slot and bumps the quad's counter; the last arriver sums the slots in CTA order, applies the
//    epilogue and resets the counter to zero. Results are bit-reproducible.
#include "g4q_common.cuh"
#include "g4q_internal.h"

namespace g4q {
namespace {

constexpr int kWarpsV2 = 16;                  // warps per CTA (12 when the tokens' x needs the room)
constexpr int kStages = 3;                    // the most ring stages (the launch may use 2)
constexpr uint32_t kUnitPacked = 4 * 512;     // four 16-row tiles x one group
constexpr uint32_t kUnitSb = 64 * 4;
constexpr uint32_t kUnitBytes = kUnitPacked + kUnitSb;
// partial-sum bytes per token of a CTA of w warps: [quad parity][tok][warp][row]
constexpr uint32_t red_bytes_per_tok(int w) { return 2u * (uint32_t)w * 64u * 4u; }
constexpr long long kWaitLimitCycles2 = 4000000000ll;
constexpr uint32_t kOddNibbleMask = 0x00F000F0u;  // q at bits 4-7 of each half: bf16 value q * 2^-129

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
    float* slots;           // [Q][8][64 rows][8 tokens]
    int* counters;          // [Q], zero between launches
    int* err;
    int stages;             // ring stages per warp (2 or 3)
    int xg;                 // 64-wide groups of x staged per token: G, or fewer when every CTA's
                            // range is shorter than a quad row (the window its units read)
    const uint16_t* norm_w; // non-null: fused RMSNorm of x with this bf16 [K] weight (no output scale)
    uint16_t* xn;           // non-null (norm only): CTA 0 also writes the normalized rows here
    int64_t ldxn;
    int geglu;              // 1: paired gate|up quads, y = geglu(gate, up) bf16 [M, N/2]
    float gk_cubic, gk_tanh;   // the GeGLU constants rounded to bf16
};

// One bf16 pair of the fused RMSNorm: bf16(w * bf16(x * inv)) per half, the rounding order of
// fast::rms_norm (the normalized value in the input dtype, then the weight product).
__device__ __forceinline__ uint32_t norm_pair(uint32_t xv, uint32_t wv, float inv) {
    const float lo = __fmul_rn(bf16_bits_to_f32(wv & 0xffffu),
                               bf16_bits_to_f32(f32_to_bf16_bits(__fmul_rn(bf16_bits_to_f32(xv & 0xffffu), inv))));
    const float hi = __fmul_rn(bf16_bits_to_f32(wv >> 16),
                               bf16_bits_to_f32(f32_to_bf16_bits(__fmul_rn(bf16_bits_to_f32(xv >> 16), inv))));
    return (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
}

__device__ __forceinline__ uint4 norm_vec(uint4 v, uint4 w, float inv) {
    return make_uint4(norm_pair(v.x, w.x, inv), norm_pair(v.y, w.y, inv), norm_pair(v.z, w.z, inv),
                      norm_pair(v.w, w.w, inv));
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __noinline__ void wait_slow(uint32_t bar, uint32_t parity, int* err) {
    const long long t0 = clock64();
    for (uint32_t it = 0;; ++it) {
        if (try_wait(bar, parity)) return;
        if ((it & 1023u) == 1023u && *reinterpret_cast<volatile int*>(err) != 0) return;
        if (clock64() - t0 > kWaitLimitCycles2) {
            atomicCAS(err, 0, 16);
            return;
        }
    }
}

__device__ __forceinline__ void wait_parity(uint32_t bar, uint32_t parity, int* err) {
    if (!try_wait(bar, parity)) wait_slow(bar, parity, err);
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

// Warp w owns the contiguous units [wstart(w), wstart(w + 1)) of its CTA's n units (relative
// numbering): the first n % kW warps take one unit more, warps past n own none.
template <int kW>
__device__ __forceinline__ int wstart(int w, int n) {
    const int b = n / kW, r = n - b * kW;
    return w * b + min(w, r);
}

template <int kW>
__device__ __forceinline__ int warp_of(int u, int n) {   // owner of relative unit u, 0 <= u < n
    const int b = n / kW, r = n - b * kW, big = r * (b + 1);
    return u < big ? u / (b + 1) : r + (u - big) / b;
}

// next unit in (quad, group) order
__device__ __forceinline__ void step1(int& q, int& g, int G) {
    if (++g == G) {
        g = 0;
        ++q;
    }
}

__device__ __forceinline__ void store_out(const Gemv2Args& a, int q, int row, int tok, float v, float r) {
    const float o = __fmul_rn(v, r);
    const int64_t idx = (int64_t)tok * a.ldy + q * 64 + row;
    if (a.flags & G4Q_QMM_OUT_F32)
        reinterpret_cast<float*>(a.y)[idx] = o;
    else
        reinterpret_cast<uint16_t*>(a.y)[idx] = f32_to_bf16_bits(o);
}

// GeGLU epilogue of a paired quad q: rows r and r + 32 are gate and up of output feature 32q + r;
// each is scaled and rounded to bf16 as the matmul's own output would be, then geglu'd.
__device__ __forceinline__ void store_act(const Gemv2Args& a, int q, int r, int tok, float vg, float vu, float rs) {
    const float g = bf16_bits_to_f32(f32_to_bf16_bits(__fmul_rn(vg, rs)));
    const float u = bf16_bits_to_f32(f32_to_bf16_bits(__fmul_rn(vu, rs)));
    reinterpret_cast<uint16_t*>(a.y)[(int64_t)tok * a.ldy + q * 32 + r] = geglu_bf16(g, u, a.gk_cubic, a.gk_tanh);
}

// Shared-memory order of x: inside each 64-wide group, lane t's B-fragment words for the four k16
// steps (j) sit together: word w = 8j + t + 4hi of the group goes to slot 8t + 2j + hi, so a lane
// fetches the group's fragments of its token with two 16-byte loads.
__device__ __forceinline__ int xperm(int w) {
    const int r = w & 7;
    return (w & ~31) | ((r & 3) << 3) | (((w >> 3) & 3) << 1) | (r >> 2);
}

// Park this warp's partial of quad q (the M token columns of its 64 rows). A warp keeps the partial
// of the first quad of its run in red[warp][0] (earlier warps may share that quad) and any other in
// red[warp][1] (only its last quad is shared, with later warps, and it comes last), so no warp ever
// waits. The last contributing warp (arrival counter of the quad's first warp) sums the partials in
// warp order, then stores a quad whole in this CTA or leaves the CTA's partial in its global slot;
// the last CTA to arrive at a cut quad sums the slots in CTA order. Results are bit-reproducible.
template <int kW>
__device__ __forceinline__ void park_quad(const Gemv2Args& a, int* qcnt, float* red, int q, int first_q, int cs,
                                          int ce, int cta, int C, const float (&acc)[4][4], const float* rs) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gi = lane >> 2, t = lane & 3;
    const int M = a.M, G = a.G, n = ce - cs;
    float* rb = red + (size_t)(warp * 2 + (q == first_q ? 0 : 1)) * M * 64;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int tok = 2 * t + (e & 1);
            if (tok < M) rb[tok * 64 + i * 16 + gi + ((e & 2) ? 8 : 0)] = acc[i][e];
        }
    __threadfence_block();
    __syncwarp();
    const int lo = max(cs, q * G), hi = min(ce, (q + 1) * G);
    const int wa = warp_of<kW>(lo - cs, n), wb = warp_of<kW>(hi - 1 - cs, n);
    if (wb > wa) {   // shared with other warps: only the last of them goes on
        int last = 0;
        if (lane == 0) last = atomicAdd(&qcnt[wa], 1) == wb - wa;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) return;
        __threadfence_block();
        if (lane == 0) qcnt[wa] = 0;
    }
    // warp wa holds q in slot 0 only if q is also its first quad; the others hold it as their first
    const int slot_a = (cs + wstart<kW>(wa, n)) / G == q ? 0 : 1;
    const bool whole = cs <= q * G && ce >= (q + 1) * G;
    const int nout = 64 * M;
    float* base = a.slots + (size_t)q * 8 * 512;
    int cf = 0, nc = 1;
    if (!whole) {
        cf = cta_of_unit(q * G, a.U, C);
        nc = cta_of_unit((q + 1) * G - 1, a.U, C) - cf + 1;
    }
    if (whole && a.geglu) {   // both rows of each gate/up pair, summed exactly as below
        for (int o2 = lane; o2 < 32 * M; o2 += 32) {
            const int tok = o2 >> 5, r = o2 & 31, og = tok * 64 + r, ou = og + 32;
            float vg = red[(size_t)(wa * 2 + slot_a) * M * 64 + og];
            float vu = red[(size_t)(wa * 2 + slot_a) * M * 64 + ou];
            for (int w = wa + 1; w <= wb; ++w) {
                vg += red[(size_t)w * 2 * M * 64 + og];
                vu += red[(size_t)w * 2 * M * 64 + ou];
            }
            store_act(a, q, r, tok, vg, vu, rs[tok]);
        }
    } else {
        for (int o = lane; o < nout; o += 32) {
            const int tok = o >> 6, row = o & 63;
            float v = red[(size_t)(wa * 2 + slot_a) * M * 64 + o];
            for (int w = wa + 1; w <= wb; ++w) v += red[(size_t)w * 2 * M * 64 + o];
            if (whole)
                store_out(a, q, row, tok, v, rs[tok]);
            else
                base[(size_t)(cta - cf) * 512 + row * 8 + tok] = v;
        }
    }
    if (!whole) {
        // arrival: the warp barrier orders the lanes' slot stores before lane 0's gpu-scope release
        // on the counter, and the last arriver's acquire makes every CTA's slots visible to its lanes
        // (one acq_rel atomic instead of a fence on each side of a relaxed one: measured 14.9 -> 14.1 us
        // for up_proj at M = 1, together with the plain-store reset below)
        __syncwarp();
        int lastc = 0;
        if (lane == 0) {
            unsigned int old;
            asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(a.counters + q) : "memory");
            lastc = old == (unsigned)(nc - 1);
        }
        lastc = __shfl_sync(0xffffffffu, lastc, 0);
        __syncwarp();
        if (lastc) {
            if (a.geglu) {
                for (int o2 = lane; o2 < 32 * M; o2 += 32) {
                    const int tok = o2 >> 5, r = o2 & 31;
                    float sg = 0.0f, su = 0.0f;
                    for (int c = 0; c < nc; ++c) {
                        sg += __ldcg(base + (size_t)c * 512 + r * 8 + tok);
                        su += __ldcg(base + (size_t)c * 512 + (r + 32) * 8 + tok);
                    }
                    store_act(a, q, r, tok, sg, su, rs[tok]);
                }
            } else {
                for (int o = lane; o < nout; o += 32) {
                    const int tok = o >> 6, row = o & 63;
                    float s = 0.0f;
                    for (int c = 0; c < nc; ++c) s += __ldcg(base + (size_t)c * 512 + row * 8 + tok);
                    store_out(a, q, row, tok, s, rs[tok]);
                }
            }
            __syncwarp();
            // nothing else touches this counter in this launch and the next launch reads it only after
            // this grid completes, so a plain store resets it (no round trip on the kernel's tail)
            if (lane == 0) asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(a.counters + q), "r"(0u) : "memory");
        }
    }
    __syncwarp();
}

// kRaw: every |scale| < 2^-1 and none subnormal, so the odd-nibble rows dequantize from the raw masked bits (q * 2^-129
// read as bf16, times s * 2^129); otherwise all four rows go through the (128 + q) magic.
template <bool kRaw, int kW>
__global__ void __launch_bounds__(kW * 32, 1) gemv2_kernel(Gemv2Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) unsigned long long bars[kW][kStages];
    __shared__ float wss[kW][8];
    __shared__ float rs[8];
    __shared__ float ninv[8];   // fused RMSNorm: per-token inverse RMS
    __shared__ int qcnt[kW];
    // the warp index through a shuffle from lane 0: provably warp-uniform, so the compiler keeps it
    // and everything derived from it (ring and barrier addresses, unit cursors) in uniform registers
    const int warp = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0), lane = threadIdx.x & 31, gi = lane >> 2,
              t = lane & 3;
    const int C = gridDim.x, cta = blockIdx.x;
    const int cs = range_start(cta, a.U, C), ce = range_start(cta + 1, a.U, C);
    const int G = a.G, M = a.M;
    const int stages = a.stages;
    const size_t ring_bytes = (size_t)stages * kUnitBytes;
    uint8_t* ring = smem + (size_t)warp * ring_bytes;
    const uint32_t ring_s = smem_addr(ring);
    const uint32_t bar0 = smem_addr(&bars[warp][0]);
    float* red = reinterpret_cast<float*>(smem + (size_t)kW * ring_bytes);
    uint32_t* xs = reinterpret_cast<uint32_t*>(smem + (size_t)kW * ring_bytes + (size_t)red_bytes_per_tok(kW) * M);

    // this warp's run of units
    const int n = ce - cs;
    const int u0 = wstart<kW>(warp, n);
    const int n_units = wstart<kW>(warp + 1, n) - u0;
    int pq = (cs + u0) / G, pg = (cs + u0) - pq * G;   // producer position
    if (lane == 0) {
        for (int s = 0; s < stages; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8 * s));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x < kW) qcnt[threadIdx.x] = 0;
    __syncwarp();
    for (int s = 0; s < stages && s < n_units; ++s) {
        if (lane == 0) issue_unit(a, pq, pg, ring_s + s * kUnitBytes, bar0 + 8 * s);
        step1(pq, pg, G);
    }
    // Launched as a programmatic dependent of the previous kernel in the stream: everything above
    // touches only this launch's shared memory and the weights (written before any compute call
    // returns), so it overlaps the previous kernel's tail. x, y and the shared scratch wait for that
    // kernel to complete; the next launch may start its own prologue as this grid's SMs free up.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    // stage x (M <= 8 tokens) into B-fragment order per token: all K, or, when the CTA's range is
    // shorter than a quad row, the window of a.xg groups starting at its first unit's group (slot j
    // holds group (cs + j) mod G, so relative unit u reads slot u); sums of squares per token over K
    const bool rms = (a.flags & G4Q_QMM_RMS_SCALE) != 0;
    const bool win = a.xg < G;
    const int words = a.xg * 32;   // bf16 pairs staged per token
    const int g0 = win ? cs % G : 0;
    const bool norm = a.norm_w != nullptr;
    if (norm) {
        // fused RMSNorm: the per-token inverse RMS over all of K first (every CTA reduces in the same
        // order, so every CTA stages the same bits), then x is normalized as it is staged
        for (int m = 0; m < M; ++m) {
            float ss = 0.0f;
            const uint4* xr = reinterpret_cast<const uint4*>(a.x + (int64_t)m * a.ldx);
            for (int u = threadIdx.x; u < a.K / 8; u += (kW * 32)) {
                const uint4 v = xr[u];
                const uint32_t pv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float lo = bf16_bits_to_f32(pv[i] & 0xffffu), hi = bf16_bits_to_f32(pv[i] >> 16);
                    ss = __fadd_rn(ss, __fmul_rn(lo, lo));
                    ss = __fadd_rn(ss, __fmul_rn(hi, hi));
                }
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
            if (lane == 0) wss[warp][m] = ss;
        }
        __syncthreads();
        if (threadIdx.x < M) {
            float s = 0.0f;
            for (int w = 0; w < kW; ++w) s = __fadd_rn(s, wss[w][threadIdx.x]);
            ninv[threadIdx.x] = __frsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)a.K), a.eps));
        }
        __syncthreads();
        if (a.xn != nullptr && cta == 0) {   // the normalized rows, for callers that need them too
            for (int m = 0; m < M; ++m) {
                const uint4* xr = reinterpret_cast<const uint4*>(a.x + (int64_t)m * a.ldx);
                const uint4* wr = reinterpret_cast<const uint4*>(a.norm_w);
                uint4* outr = reinterpret_cast<uint4*>(a.xn + (int64_t)m * a.ldxn);
                for (int u = threadIdx.x; u < a.K / 8; u += (kW * 32)) outr[u] = norm_vec(xr[u], wr[u], ninv[m]);
            }
        }
    }
    for (int m = 0; m < M; ++m) {
        float ss = 0.0f;
        const uint4* xr = reinterpret_cast<const uint4*>(a.x + (int64_t)m * a.ldx);
        uint32_t* xm = xs + (size_t)m * words;
        for (int u = threadIdx.x; u < a.xg * 8; u += (kW * 32)) {
            int g = g0 + (u >> 3);
            if (g >= G) g -= G;
            uint4 v = xr[g * 8 + (u & 7)];
            if (norm) v = norm_vec(v, reinterpret_cast<const uint4*>(a.norm_w)[g * 8 + (u & 7)], ninv[m]);
            xm[xperm(4 * u)] = v.x;
            xm[xperm(4 * u + 1)] = v.y;
            xm[xperm(4 * u + 2)] = v.z;
            xm[xperm(4 * u + 3)] = v.w;
            if (rms && !win) {
                const uint32_t pv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float lo = bf16_bits_to_f32(pv[i] & 0xffffu), hi = bf16_bits_to_f32(pv[i] >> 16);
                    ss = __fadd_rn(ss, __fmul_rn(lo, lo));
                    ss = __fadd_rn(ss, __fmul_rn(hi, hi));
                }
            }
        }
        if (rms && win) {   // the RMS scale needs all of x
            for (int u = threadIdx.x; u < a.K / 8; u += (kW * 32)) {
                const uint4 v = xr[u];
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
        if (rms && threadIdx.x < M) {
            float s = 0.0f;
            for (int w = 0; w < kW; ++w) s = __fadd_rn(s, wss[w][threadIdx.x]);
            r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)a.K), a.eps)));
        }
        rs[threadIdx.x] = r;
    }
    __syncthreads();

    // B fragments: lane (gi, t) reads token gi (token 0 for the columns past M; those outputs are
    // never stored)
    const uint4* xt = reinterpret_cast<const uint4*>(xs + (size_t)(gi < M ? gi : 0) * words) + 2 * t;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][e] = 0.0f;
    int cq = (cs + u0) / G, cg = (cs + u0) - cq * G;   // consumer position
    const int first_q = cq;
    int stage = 0;
    uint32_t phase = 0;
    // the run as segments of whole quads: one park per segment, no per-unit quad bookkeeping
    for (int k = 0; k < n_units;) {
        const int seg = min(n_units - k, G - cg);
        const uint4* xp = xt + (size_t)(win ? u0 + k : cg) * 8;   // staged slot of the segment's first group
        for (int j = 0; j < seg; ++j, xp += 8) {
            wait_parity(bar0 + 8 * stage, phase, a.err);
            const uint8_t* st = ring + stage * kUnitBytes;
            const uint4 xa = xp[0], xb = xp[1];
            const uint32_t b0[4] = {xa.x, xa.z, xb.x, xb.z}, b1[4] = {xa.y, xa.w, xb.y, xb.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint4 wv = reinterpret_cast<const uint4*>(st + i * 512)[lane];
                const uint32_t* sbw = reinterpret_cast<const uint32_t*>(st + kUnitPacked) + i * 16 + gi;
                const RowConsts c0 = row_consts(sbw[0]);
                if constexpr (kRaw) {
                    const uint32_t b1s = bcast_hi(sbw[8]);
                    const uint32_t s1h = bcast_lo(sbw[8]) + kExp129x2;   // s * 2^129 (no subnormal scales)
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        const uint32_t w = jj == 0 ? wv.x : jj == 1 ? wv.y : jj == 2 ? wv.z : wv.w;
                        const uint32_t w8 = w >> 8;
                        const uint32_t a0 = deq_r2_fast(lop_nibbles(w), c0);
                        const uint32_t a1 = add_bf16x2(mul_bf16x2(w & kOddNibbleMask, s1h), b1s);
                        const uint32_t a2 = deq_r2_fast(lop_nibbles(w8), c0);
                        const uint32_t a3 = add_bf16x2(mul_bf16x2(w8 & kOddNibbleMask, s1h), b1s);
                        mma_bf16_16816(acc[i], a0, a1, a2, a3, b0[jj], b1[jj]);
                    }
                } else {
                    const RowConsts c1 = row_consts(sbw[8]);
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        const uint32_t w = jj == 0 ? wv.x : jj == 1 ? wv.y : jj == 2 ? wv.z : wv.w;
                        const uint32_t a0 = deq_r2_fast(lop_nibbles(w), c0);
                        const uint32_t a1 = deq_r2_fast(lop_nibbles(w >> 4), c1);
                        const uint32_t a2 = deq_r2_fast(lop_nibbles(w >> 8), c0);
                        const uint32_t a3 = deq_r2_fast(lop_nibbles(w >> 12), c1);
                        mma_bf16_16816(acc[i], a0, a1, a2, a3, b0[jj], b1[jj]);
                    }
                }
            }
            // the unit has been read: refill this buffer `stages` units ahead
            __syncwarp();
            if (k + j + stages < n_units) {
                if (lane == 0) issue_unit(a, pq, pg, ring_s + stage * kUnitBytes, bar0 + 8 * stage);
                step1(pq, pg, G);
            }
            if (++stage == stages) {
                stage = 0;
                phase ^= 1u;
            }
        }
        park_quad<kW>(a, qcnt, red, cq, first_q, cs, ce, cta, C, acc, rs);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[i][e] = 0.0f;
        k += seg;
        ++cq;
        cg = 0;
    }
}

}  // namespace

size_t gemv2_slots_bytes(int64_t N, int64_t K, int sms) {
    (void)K;
    (void)sms;
    // 8 slots of 64 rows x 8 tokens fp32 per 64-row quad (launch_gemv2 keeps contributors <= 8)
    return (size_t)(N / 64) * 8 * 64 * 8 * sizeof(float);
}

// grid for a U-unit, G-group problem: every CTA owns >= 1 unit and a quad meets <= 8 CTA ranges
static int gemv2_grid(int U, int G, int sms) {
    int grid = sms < U ? sms : U;
    while (grid > 1 && (G - 1) / (U / grid) + 2 > 8) --grid;
    return grid;
}

static size_t gemv2_smem(int warps, int stages, int64_t M, int64_t xg) {
    return (size_t)warps * stages * kUnitBytes + (size_t)red_bytes_per_tok(warps) * M + (size_t)xg * 64 * M * 2;
}

// groups of x each CTA stages: all G, or the window of its range when every range is shorter
static int gemv2_xgroups(int U, int G, int grid) {
    const int nmax = (U + grid - 1) / grid;
    return nmax < G ? nmax : G;
}

// Warps per CTA and ring stages: 16 warps of 3 stages when they fit beside the tokens' x, else 16 of
// 2, else 12 warps of 2 (e.g. down_proj's 15360-wide x at 8 tokens, whose window per CTA takes 100 KB);
// warps 0: does not fit at all.
struct Gemv2Shape {
    int warps, stages;
};
static Gemv2Shape gemv2_shape(int64_t M, int64_t xg) {
    const Gemv2Shape tries[] = {{kWarpsV2, 3}, {kWarpsV2, 2}, {12, 2}};
    for (const Gemv2Shape& t : tries)
        if (gemv2_smem(t.warps, t.stages, M, xg) <= 220 * 1024) return t;
    return {0, 0};
}

bool gemv2_supported(const QmmCall& c) {
    if (c.M < 1 || c.M > 8 || c.w->N % 64 != 0) return false;
    const long long units = (c.w->N / 64) * (c.w->K / 64);
    if (units < 1 || units >= (1ll << 31)) return false;
    const int G = (int)(c.w->K / 64);
    const int grid = gemv2_grid((int)units, G, device_sm_count());
    if (grid <= 0) return false;
    return gemv2_shape(c.M, gemv2_xgroups((int)units, G, grid)).warps != 0;
}

void launch_gemv2(const QmmCall& c, cudaStream_t st) {
    static bool attr_set[64] = {false};
    const int dev = current_device();
    const void* kernels[2][2] = {{reinterpret_cast<const void*>(gemv2_kernel<false, kWarpsV2>),
                                  reinterpret_cast<const void*>(gemv2_kernel<false, 12>)},
                                 {reinterpret_cast<const void*>(gemv2_kernel<true, kWarpsV2>),
                                  reinterpret_cast<const void*>(gemv2_kernel<true, 12>)}};
    if (!attr_set[dev & 63]) {
        for (auto& row : kernels)
            for (const void* k : row)
                check_cuda(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)max_dynamic_smem(k)),
                           "cudaFuncSetAttribute(gemv2)");
        attr_set[dev & 63] = true;
    }
    const Weight& w = *c.w;
    DeviceScratch& ds = device_scratch();
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
    const int grid = gemv2_grid(a.U, a.G, device_sm_count());
    if (grid <= 0) throw Error(G4Q_ERR_RUNTIME, "gemv2: no valid grid for this shape");
    if ((size_t)a.Q * 8 * 64 * 8 * sizeof(float) > ds.slots_bytes)
        throw Error(G4Q_ERR_RUNTIME, "gemv scratch too small for this shape (create the weight before capture)");
    a.x = c.x;
    a.ldx = c.ldx;
    a.y = c.y;
    a.ldy = c.ldy;
    a.flags = c.flags;
    a.eps = c.eps;
    a.slots = ds.slots;
    a.counters = ds.counters;
    a.err = ds.err;
    a.geglu = c.geglu ? 1 : 0;
    a.gk_cubic = bf16_round_host(0.044715f);
    a.gk_tanh = bf16_round_host(0.7978845608028654f);
    a.norm_w = c.norm_w;
    a.xn = c.norm_w != nullptr ? c.xn : nullptr;
    a.ldxn = c.ldxn;
    a.xg = gemv2_xgroups(a.U, a.G, grid);
    const Gemv2Shape shape = gemv2_shape(a.M, a.xg);
    if (shape.warps == 0) throw Error(G4Q_ERR_RUNTIME, "gemv2: x does not fit in shared memory");
    a.stages = shape.stages;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(shape.warps * 32);
    cfg.dynamicSmemBytes = gemv2_smem(shape.warps, a.stages, a.M, a.xg);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {&a};
    const void* k = kernels[w.small_scales && !w.subnormal_scales ? 1 : 0][shape.warps == kWarpsV2 ? 0 : 1];
    check_cuda(cudaLaunchKernelExC(&cfg, k, args), "gemv2 launch");
}

}  // namespace g4q
