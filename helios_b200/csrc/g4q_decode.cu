// g4q_decode.cu -- the whole quantized-linear part of a decode step in ONE persistent kernel.
//
// Replaces the per-token sequence of quantized_matmul calls that the reference's decode drivers
// issue (native_model.cc:1843-1911 decode_last_logits, 48 x target_layer_decode_forward at
// :1284-1328, then the tied LM head :1782-1795 and argmax :3825): a "plan" lists the phases
// (one quantized matmul each, e.g. q|k|v, o, gate|up, down per layer, then the LM head with the
// fused softcap + argmax); each phase reads the previous phase's output.
//
// Why one kernel: at batch 1 every phase is a few microseconds of HBM streaming, so separate
// launches spend a large share of the step in prologues (staging x) and epilogues (reductions,
// tails). Here one cooperative grid (one 16-warp CTA per SM) stays resident for the whole step:
//  * every warp streams its weight units through a private ring of cp.async.bulk buffers that
//    runs ahead ACROSS phase boundaries, so the next phase's weights are already landing while the
//    grid waits for the current phase to finish;
//  * phase p+1 starts in a CTA once the per-phase completion counter says all CTAs have stored
//    phase p (bounded spin), then x is re-staged in shared memory (with the RMS scale if asked);
//  * inside a phase the units are split exactly as in the stream-K GEMV (g4q_gemv2.cu): equal
//    contiguous CTA ranges over (64-row quad, 64-wide group) units, warp w takes every 16th unit,
//    deterministic per-quad reductions in shared memory and through global slots for quads cut by a
//    CTA-range boundary;
//  * the argmax phase keeps per-token 64-bit keys (order-preserving logit bits | ~row) and the last
//    CTA publishes tokens/values/keys; the last CTA to leave resets every counter, so the plan is
//    ready for the next launch (and for CUDA-graph replay) without a memset.
#include <string>
#include <vector>

#include "g4q_common.cuh"
#include "g4q_internal.h"

namespace g4q {
namespace {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 4;
constexpr uint32_t kUnitPacked = 4 * 512;
constexpr uint32_t kUnitSb = 64 * 4;
constexpr uint32_t kUnitBytes = kUnitPacked + kUnitSb;
constexpr uint32_t kRingBytes = kStages * kUnitBytes;
constexpr int kMaxTok = 2;
constexpr int kSlots = 16;   // CTA ranges one 64-row quad may be cut into
constexpr long long kSpinLimit = 4000000000ll;   // ~2 s of SM clocks

struct PhaseDev {
    const uint32_t* packed;
    const uint32_t* sb;
    const uint16_t* x;
    void* y;
    int64_t ldx, ldy;
    int N, K, R, G, Q, U;
    uint32_t flags;
};

struct DecodeArgs {
    const PhaseDev* ph;
    int n_phases;
    int M;
    float eps, softcap;
    int64_t row_offset;          // global index of the argmax phase's row 0 (vocabulary shard)
    unsigned int* done;          // [n_phases] CTAs that finished each phase
    unsigned int* exit_count;    // [1]
    unsigned long long* keys;    // [kMaxTok] running argmax keys
    float* slots;                // [max quads][kSlots][64][kMaxTok], shared by the phases (they run one at a time)
    int* qcount;                 // [max quads], zero between phases
    int32_t* tokens;
    float* values;
    unsigned long long* keys_out;
    uint16_t* logits;            // optional bf16 logits of the argmax phase
    int64_t ld_logits;
    int* err;
};

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

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
        if (clock64() - t0 > kSpinLimit) {
            atomicCAS(err, 0, 32);
            return;
        }
    }
}

__device__ __forceinline__ void wait_parity(uint32_t bar, uint32_t parity, int* err) {
    if (!try_wait(bar, parity)) wait_slow(bar, parity, err);
}

__device__ __forceinline__ int range_start(int c, int U, int C) { return (int)(((long long)c * U) / C); }

__device__ __forceinline__ int cta_of_unit(int u, int U, int C) {
    int c = (int)(((long long)u * C) / U);
    while (c + 1 < C && range_start(c + 1, U, C) <= u) ++c;
    while (c > 0 && range_start(c, U, C) > u) --c;
    return c;
}

// Position of one warp in its unit sequence across all phases.
struct Cursor {
    int p;      // phase
    int k, n;   // unit k of n in this phase
    int q, g;   // current (quad, group)
    __device__ __forceinline__ void enter(const DecodeArgs& a, int cta, int C, int w) {
        while (p < a.n_phases) {
            const PhaseDev& P = a.ph[p];
            const int cs = range_start(cta, P.U, C), ce = range_start(cta + 1, P.U, C);
            n = ce - cs > w ? (ce - cs - w + kWarps - 1) / kWarps : 0;
            k = 0;
            if (n > 0) {
                q = (cs + w) / P.G;
                g = (cs + w) - q * P.G;
                return;
            }
            ++p;
        }
    }
    __device__ __forceinline__ void next(const DecodeArgs& a, int cta, int C, int w) {
        if (++k < n) {
            const int G = a.ph[p].G;
            g += kWarps;
            while (g >= G) {
                g -= G;
                ++q;
            }
            return;
        }
        ++p;
        enter(a, cta, C, w);
    }
};

__device__ __forceinline__ void issue_unit(const PhaseDev& P, int q, int g, uint32_t dst, uint32_t bar) {
    const uint32_t* src_p = P.packed + ((size_t)g * P.R + (size_t)q * 4) * 128;
    const uint32_t* src_s = P.sb + (size_t)g * P.N + (size_t)q * 64;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(kUnitBytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src_p), "r"(kUnitPacked), "r"(bar)
                 : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     dst + kUnitPacked),
                 "l"(src_s), "r"(kUnitSb), "r"(bar)
                 : "memory");
}

struct CtaShared {
    unsigned long long bars[kWarps][kStages];
    float wss[kWarps][kMaxTok];
    float rs[kMaxTok];
    int cnt[2];
    int seq_done[2];
    int warps_finished;
    unsigned long long best[kMaxTok];
    int last_cta;
    uint2 zero;
};

// Final value of one output element of phase P: store, or (argmax phase) fold into the running key.
__device__ __forceinline__ void emit(const DecodeArgs& a, const PhaseDev& P, int q, int row, int tok, float v,
                                     const float* rs, unsigned long long& best) {
    const float o = __fmul_rn(v, rs[tok]);
    const int n = q * 64 + row;
    if (P.flags & G4Q_PHASE_ARGMAX) {
        const uint16_t lb = f32_to_bf16_bits(o);
        if (a.logits) a.logits[(int64_t)tok * a.ld_logits + n] = lb;
        const float lv = bf16_bits_to_f32(lb);
        const float sv = a.softcap > 0.0f ? softcap_bf16(lv, a.softcap) : lv;
        const unsigned long long key = argmax_key(sv, (uint32_t)(a.row_offset + n));
        if (key > best) best = key;
        return;
    }
    const int64_t idx = (int64_t)tok * P.ldy + n;
    if (P.flags & G4Q_QMM_OUT_F32)
        reinterpret_cast<float*>(P.y)[idx] = o;
    else
        reinterpret_cast<uint16_t*>(P.y)[idx] = f32_to_bf16_bits(o);
}

__device__ void park(const DecodeArgs& a, const PhaseDev& P, CtaShared& sh, float* red, int seq, int q, int cs,
                     int ce, int cta, int C, const float (&acc)[4][4], unsigned long long (&best)[kMaxTok]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gi = lane >> 2, t = lane & 3;
    const int M = a.M, G = P.G;
    const int b = seq & 1;
    if (*reinterpret_cast<volatile int*>(&sh.seq_done[b]) < seq - 2) {
        const long long t0 = clock64();
        while (*reinterpret_cast<volatile int*>(&sh.seq_done[b]) < seq - 2) {
            if (clock64() - t0 > kSpinLimit) {
                atomicCAS(a.err, 0, 33);
                break;
            }
        }
    }
    float* rb = red + (size_t)b * kMaxTok * kWarps * 64;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int tok = 2 * t + (e & 1);
            if (tok < M) rb[(tok * kWarps + warp) * 64 + i * 16 + gi + ((e & 2) ? 8 : 0)] = acc[i][e];
        }
    __threadfence_block();
    __syncwarp();
    const int lo = max(cs, q * G), hi = min(ce, (q + 1) * G);
    const int nw = min(kWarps, hi - lo);
    const int w0 = (lo - cs) % kWarps;
    int last = 0;
    if (lane == 0) last = atomicAdd(&sh.cnt[b], 1) == nw - 1;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence_block();
    const bool whole = cs <= q * G && ce >= (q + 1) * G;
    const int nout = 64 * M;
    float* base = a.slots + ((size_t)q * kSlots) * 64 * kMaxTok;
    int cf = 0, nc = 1;
    if (!whole) {
        cf = cta_of_unit(q * G, P.U, C);
        nc = cta_of_unit((q + 1) * G - 1, P.U, C) - cf + 1;
    }
    for (int o = lane; o < nout; o += 32) {
        const int tok = o >> 6, row = o & 63;
        float v = 0.0f;
        for (int w = 0; w < kWarps; ++w) {
            const int d = (w - w0 + kWarps) % kWarps;
            if (d < nw) v += rb[(tok * kWarps + w) * 64 + row];
        }
        if (whole)
            emit(a, P, q, row, tok, v, sh.rs, best[tok]);
        else
            base[((size_t)(cta - cf) * 64 + row) * kMaxTok + tok] = v;
    }
    __syncwarp();
    if (lane == 0) sh.cnt[b] = 0;
    if (whole) __threadfence();   // outputs visible GPU-wide before the phase counter moves
    if (!whole) {
        __threadfence();
        __syncwarp();
        int lastc = 0;
        if (lane == 0) lastc = atomicAdd(a.qcount + q, 1) == nc - 1;
        lastc = __shfl_sync(0xffffffffu, lastc, 0);
        if (lastc) {
            __threadfence();
            for (int o = lane; o < nout; o += 32) {
                const int tok = o >> 6, row = o & 63;
                float s = 0.0f;
                for (int c = 0; c < nc; ++c) s += __ldcg(base + ((size_t)c * 64 + row) * kMaxTok + tok);
                emit(a, P, q, row, tok, s, sh.rs, best[tok]);
            }
            __threadfence();
            __syncwarp();
            if (lane == 0) atomicExch(a.qcount + q, 0);
        }
    }
    __threadfence_block();
    __syncwarp();
    if (lane == 0) *reinterpret_cast<volatile int*>(&sh.seq_done[b]) = seq;
}

__device__ __forceinline__ void spin_until(const unsigned int* ctr, unsigned int target, int* err) {
    if (*reinterpret_cast<const volatile unsigned int*>(ctr) >= target) return;
    const long long t0 = clock64();
    while (*reinterpret_cast<const volatile unsigned int*>(ctr) < target) {
        if (*reinterpret_cast<volatile int*>(err) != 0) return;
        if (clock64() - t0 > kSpinLimit) {
            atomicCAS(err, 0, 34);
            return;
        }
    }
}

__global__ void __launch_bounds__(kThreads, 1) decode_kernel(DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ CtaShared sh;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gi = lane >> 2, t = lane & 3;
    const int C = gridDim.x, cta = blockIdx.x;
    const int M = a.M;
    uint8_t* ring = smem + (size_t)warp * kRingBytes;
    const uint32_t ring_s = saddr(ring);
    float* red = reinterpret_cast<float*>(smem + (size_t)kWarps * kRingBytes);
    uint32_t* xs = reinterpret_cast<uint32_t*>(smem + (size_t)kWarps * kRingBytes + 2 * kMaxTok * kWarps * 64 * 4);
    const uint32_t bar0 = saddr(&sh.bars[warp][0]);

    if (lane == 0) {
        for (int s = 0; s < kStages; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8 * s));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x == 0) {
        sh.cnt[0] = sh.cnt[1] = 0;
        sh.seq_done[0] = -2;
        sh.seq_done[1] = -1;
        sh.warps_finished = 0;
        for (int m = 0; m < kMaxTok; ++m) sh.best[m] = 0ull;
        sh.zero = make_uint2(0u, 0u);
    }
    __syncwarp();
    Cursor pre;
    pre.p = 0;
    pre.enter(a, cta, C, warp);
    for (int s = 0; s < kStages && pre.p < a.n_phases; ++s) {
        if (lane == 0) issue_unit(a.ph[pre.p], pre.q, pre.g, ring_s + s * kUnitBytes, bar0 + 8 * s);
        pre.next(a, cta, C, warp);
    }

    int stage = 0;
    uint32_t phase_bit = 0;
    int seq_base = 0;   // CTA-wide ordinal of the first quad of the current phase (parity picks the red buffer)
    unsigned long long best[kMaxTok];
#pragma unroll
    for (int m = 0; m < kMaxTok; ++m) best[m] = 0ull;

    for (int p = 0; p < a.n_phases; ++p) {
        const PhaseDev& P = a.ph[p];
        const int cs = range_start(cta, P.U, C), ce = range_start(cta + 1, P.U, C);
        const int G = P.G;
        const int q_first = cs / G;
        // ---- phase entry: wait for the producing phase everywhere, then stage x (row stride K+8)
        __syncthreads();
        if (p > 0 && threadIdx.x == 0) spin_until(a.done + (p - 1), (unsigned)C, a.err);
        __syncthreads();
        const int xstride = P.K + 8;   // bf16 elements; +16 bytes keeps the B-fragment reads conflict-free
        const bool rms = (P.flags & G4Q_QMM_RMS_SCALE) != 0;
        for (int m = 0; m < M; ++m) {
            float ss = 0.0f;
            const uint16_t* xr = P.x + (int64_t)m * P.ldx;
            for (int u = threadIdx.x; u < P.K / 8; u += kThreads) {
                const uint4 v = __ldcg(reinterpret_cast<const uint4*>(xr + u * 8));
                *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(xs) + m * xstride + u * 8) = v;
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
                if (lane == 0) sh.wss[warp][m] = ss;
            }
        }
        __syncthreads();
        if (threadIdx.x < kMaxTok) {
            float r = 1.0f;
            if (rms && threadIdx.x < M) {
                float s = 0.0f;
                for (int w = 0; w < kWarps; ++w) s = __fadd_rn(s, sh.wss[w][threadIdx.x]);
                r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)P.K), a.eps)));
            }
            sh.rs[threadIdx.x] = r;
        }
        __syncthreads();

        // ---- this warp's units of phase p
        const int n_units = ce - cs > warp ? (ce - cs - warp + kWarps - 1) / kWarps : 0;
        const bool tok_ok = gi < M;
        const uint32_t* xw = tok_ok ? xs + gi * (xstride / 2) + t : reinterpret_cast<const uint32_t*>(&sh.zero);
        const int kst = tok_ok ? 8 : 0;   // 32-bit words per k16 step
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[i][e] = 0.0f;
        int cq = (cs + warp) / G, cg = (cs + warp) - cq * G, acc_q = cq;
        for (int k = 0; k < n_units; ++k) {
            if (cq != acc_q) {
                park(a, P, sh, red, seq_base + (acc_q - q_first), acc_q, cs, ce, cta, C, acc, best);
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[i][e] = 0.0f;
                acc_q = cq;
            }
            wait_parity(bar0 + 8 * stage, phase_bit, a.err);
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
            const uint32_t* xg = xw + cg * 4 * kst;
            uint32_t b0[4], b1[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                b0[j] = xg[j * kst];
                b1[j] = xg[j * kst + (tok_ok ? 4 : 1)];
            }
            __syncwarp();
            if (pre.p < a.n_phases) {
                if (lane == 0) issue_unit(a.ph[pre.p], pre.q, pre.g, ring_s + stage * kUnitBytes, bar0 + 8 * stage);
                pre.next(a, cta, C, warp);
            }
            if (++stage == kStages) {
                stage = 0;
                phase_bit ^= 1u;
            }
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
                    mma_bf16_16816(acc[i], a0, a1, a2, a3, b0[j], b1[j]);
                }
            }
            cg += kWarps;
            while (cg >= G) {
                cg -= G;
                ++cq;
            }
        }
        if (n_units > 0) park(a, P, sh, red, seq_base + (acc_q - q_first), acc_q, cs, ce, cta, C, acc, best);
        seq_base += (ce - 1) / G - q_first + 1;
        // ---- argmax phase: fold the warp's best keys into the CTA's
        if (P.flags & G4Q_PHASE_ARGMAX) {
            for (int m = 0; m < M; ++m) {
                unsigned long long k = best[m];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, off);
                    k = o > k ? o : k;
                }
                if (lane == 0) atomicMax(&sh.best[m], k);
            }
        }
        // ---- the CTA has stored everything it owes for phase p
        __threadfence_block();
        __syncwarp();
        int last_warp = 0;
        if (lane == 0) last_warp = atomicAdd(&sh.warps_finished, 1) == kWarps - 1;
        last_warp = __shfl_sync(0xffffffffu, last_warp, 0);
        if (last_warp) {
            if (lane == 0) {
                sh.warps_finished = 0;
                if (P.flags & G4Q_PHASE_ARGMAX)
                    for (int m = 0; m < M; ++m) atomicMax(a.keys + m, sh.best[m]);
                __threadfence();
                const unsigned int prev = atomicAdd(a.done + p, 1u);
                sh.last_cta = (P.flags & G4Q_PHASE_ARGMAX) && prev == (unsigned)C - 1;
            }
            __syncwarp();
            if ((P.flags & G4Q_PHASE_ARGMAX) && sh.last_cta && lane < M) {
                __threadfence();
                const unsigned long long k = atomicExch(a.keys + lane, 0ull);
                if (a.tokens) a.tokens[lane] = (int32_t)key_index(k);
                if (a.values) a.values[lane] = key_value(k);
                if (a.keys_out) a.keys_out[lane] = k;
            }
        }
    }
    // ---- the last CTA out resets the phase counters for the next launch
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned int prev = atomicAdd(a.exit_count, 1u);
        if (prev == (unsigned)C - 1) {
            for (int p = 0; p < a.n_phases; ++p) a.done[p] = 0u;
            __threadfence();
            atomicExch(a.exit_count, 0u);
        }
    }
}

}  // namespace

struct DecodePlan {
    uint64_t magic = 0;
    int device = -1;
    int n_phases = 0, max_tokens = 0, grid = 0, argmax_phase = -1;
    size_t smem = 0;
    PhaseDev* d_ph = nullptr;
    unsigned int* d_done = nullptr;   // n_phases + 1 (exit counter last)
    unsigned long long* d_keys = nullptr;
    float* d_slots = nullptr;
    int* d_qcount = nullptr;
};

constexpr uint64_t kPlanMagic = 0x4734514445434f44ull;

void* decode_plan_create(const G4qDecodePhase* phases, int n, int max_tokens) {
    if (n <= 0 || phases == nullptr) throw Error(G4Q_ERR_INVALID_ARGUMENT, "a plan needs at least one phase");
    if (max_tokens < 1 || max_tokens > kMaxTok)
        throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, "the decode plan supports 1.." + std::to_string(kMaxTok) + " tokens");
    const int dev = current_device();
    const int sms = device_sm_count();
    std::vector<PhaseDev> ph(n);
    int total_quads = 0, kmax = 0, argmax = -1;
    for (int i = 0; i < n; ++i) {
        const Weight* w = reinterpret_cast<const Weight*>(phases[i].weight);
        if (!w || w->magic != kWeightMagic) throw Error(G4Q_ERR_INVALID_ARGUMENT, "phase " + std::to_string(i) + ": invalid weight");
        if (w->device != dev) throw Error(G4Q_ERR_INVALID_ARGUMENT, "phase weight lives on another device");
        if (!w->fast_ok) throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, "phase weight has scales outside |s| < 2^120");
        if (w->N % 64 != 0) throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, "decode plan phases need rows % 64 == 0");
        const uint32_t fl = phases[i].flags;
        if (fl & ~(G4Q_QMM_RMS_SCALE | G4Q_QMM_OUT_F32 | G4Q_PHASE_ARGMAX))
            throw Error(G4Q_ERR_INVALID_ARGUMENT, "unknown phase flag bits");
        if (fl & G4Q_PHASE_ARGMAX) {
            if (i != n - 1) throw Error(G4Q_ERR_INVALID_ARGUMENT, "the argmax phase must be the last phase");
            argmax = i;
        } else if (!phases[i].y) {
            throw Error(G4Q_ERR_INVALID_ARGUMENT, "phase " + std::to_string(i) + " needs an output");
        }
        if (!phases[i].x || (reinterpret_cast<uintptr_t>(phases[i].x) & 15u) || phases[i].ldx % 8 || phases[i].ldx < w->K)
            throw Error(G4Q_ERR_INVALID_ARGUMENT, "phase x must be 16-byte aligned with ldx % 8 == 0, ldx >= K");
        PhaseDev& d = ph[i];
        d.packed = w->packed;
        d.sb = w->sb;
        d.x = phases[i].x;
        d.y = phases[i].y;
        d.ldx = phases[i].ldx;
        d.ldy = phases[i].ldy;
        d.N = (int)w->N;
        d.K = (int)w->K;
        d.R = (int)(w->N / 16);
        d.G = (int)(w->K / 64);
        d.Q = d.R / 4;
        d.U = d.Q * d.G;
        d.flags = fl;
        if (d.Q > total_quads) total_quads = d.Q;   // slots are shared: size them for the largest phase
        if (d.K > kmax) kmax = d.K;
        if (d.U < sms) throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, "phase too small for a full-grid decode plan");
        // a quad (G units) meets at most (G-1)/min_range + 2 CTA ranges
        if ((d.G - 1) / (d.U / sms) + 2 > kSlots)
            throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, "phase " + std::to_string(i) + " is split too finely for the grid");
    }
    auto* plan = new DecodePlan();
    plan->device = dev;
    plan->n_phases = n;
    plan->max_tokens = max_tokens;
    plan->grid = sms;
    plan->argmax_phase = argmax;
    plan->smem = (size_t)kWarps * kRingBytes + 2 * kMaxTok * kWarps * 64 * 4 + (size_t)kMaxTok * (kmax + 8) * 2;
    if (plan->smem > max_dynamic_smem(reinterpret_cast<const void*>(decode_kernel))) {
        delete plan;
        throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, "decode plan: K too large for shared memory");
    }
    cudaError_t e = cudaMalloc(&plan->d_ph, sizeof(PhaseDev) * n);
    if (e == cudaSuccess) e = cudaMalloc(&plan->d_done, sizeof(unsigned int) * (n + 1));
    if (e == cudaSuccess) e = cudaMalloc(&plan->d_keys, sizeof(unsigned long long) * kMaxTok);
    if (e == cudaSuccess) e = cudaMalloc(&plan->d_slots, sizeof(float) * (size_t)total_quads * kSlots * 64 * kMaxTok);
    if (e == cudaSuccess) e = cudaMalloc(&plan->d_qcount, sizeof(int) * (size_t)total_quads);
    if (e == cudaSuccess) e = cudaMemcpy(plan->d_ph, ph.data(), sizeof(PhaseDev) * n, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(plan->d_done, 0, sizeof(unsigned int) * (n + 1));
    if (e == cudaSuccess) e = cudaMemset(plan->d_keys, 0, sizeof(unsigned long long) * kMaxTok);
    if (e == cudaSuccess) e = cudaMemset(plan->d_qcount, 0, sizeof(int) * (size_t)total_quads);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(plan->d_ph);
        cudaFree(plan->d_done);
        cudaFree(plan->d_keys);
        cudaFree(plan->d_slots);
        cudaFree(plan->d_qcount);
        delete plan;
        check_cuda(e, "decode plan allocation");
    }
    check_cuda(cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan->smem),
               "cudaFuncSetAttribute(decode)");
    int per_sm = 0;
    check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_kernel, kThreads, plan->smem),
               "occupancy(decode)");
    if (per_sm < 1) throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, "decode kernel does not fit on an SM");
    plan->magic = kPlanMagic;
    return plan;
}

void decode_plan_free(void* h) {
    auto* plan = static_cast<DecodePlan*>(h);
    if (!plan || plan->magic != kPlanMagic) throw Error(G4Q_ERR_INVALID_ARGUMENT, "invalid decode plan handle");
    plan->magic = 0;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(plan->device);
    cudaFree(plan->d_ph);
    cudaFree(plan->d_done);
    cudaFree(plan->d_keys);
    cudaFree(plan->d_slots);
    cudaFree(plan->d_qcount);
    cudaSetDevice(prev);
    delete plan;
}

void decode_plan_run(void* h, int M, float eps, float softcap, int64_t row_offset, int32_t* tokens, float* values,
                     uint64_t* keys, uint16_t* logits, int64_t ld_logits, cudaStream_t st) {
    auto* plan = static_cast<DecodePlan*>(h);
    if (!plan || plan->magic != kPlanMagic) throw Error(G4Q_ERR_INVALID_ARGUMENT, "invalid decode plan handle");
    if (plan->device != current_device()) throw Error(G4Q_ERR_INVALID_ARGUMENT, "plan belongs to another device");
    if (M < 1 || M > plan->max_tokens) throw Error(G4Q_ERR_INVALID_ARGUMENT, "M outside the plan's token range");
    DecodeArgs a;
    a.ph = plan->d_ph;
    a.n_phases = plan->n_phases;
    a.M = M;
    a.eps = eps;
    a.softcap = softcap;
    a.row_offset = row_offset;
    a.done = plan->d_done;
    a.exit_count = plan->d_done + plan->n_phases;
    a.keys = plan->d_keys;
    a.slots = plan->d_slots;
    a.qcount = plan->d_qcount;
    a.tokens = tokens;
    a.values = values;
    a.keys_out = reinterpret_cast<unsigned long long*>(keys);
    a.logits = logits;
    a.ld_logits = ld_logits;
    a.err = device_scratch().err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan->grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = plan->smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;   // every CTA resident: CTAs wait on each other's phases
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    check_cuda(cudaLaunchKernelEx(&cfg, decode_kernel, a), "cudaLaunchKernelEx(decode)");
}

}  // namespace g4q
