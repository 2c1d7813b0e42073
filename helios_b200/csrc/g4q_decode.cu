// g4q_decode.cu -- the whole quantized-linear part of a decode step in ONE persistent kernel.
//
// Replaces the per-token sequence of quantized_matmul calls that the reference's decode drivers
// issue (native_model.cc:1843-1911 decode_last_logits, 48 x target_layer_decode_forward at
// :1284-1328, then the tied LM head :1782-1795 and argmax :3825): a "plan" lists the phases
// (one quantized matmul each, e.g. q|k|v, o, gate|up, down per layer, then the LM head with the
// fused softcap + argmax); each phase may read (a column window of) the previous phase's output.
//
// Why one kernel: at batch 1 every phase is a few microseconds of HBM streaming, so separate
// launches spend a large share of the step in prologues (staging x) and epilogues (reductions,
// tails). Here one cooperative grid (one 16-warp CTA per SM) stays resident for the whole step:
//  * every warp streams its weight units (64 rows x one 64-wide group: 2 KB of packed words +
//    256 B of scale|bias) through a private ring of cp.async.bulk buffers that runs ahead ACROSS
//    phase boundaries, so the next phase's weights land while the grid finishes the current one;
//  * the units of a phase are cut into equal contiguous CTA ranges (quad-major) and each CTA range
//    into contiguous warp runs; a quad's warp partials are reduced in shared memory, wait-free;
//  * dataflow instead of grid barriers or arrival counters: every output quad has ONE finisher. A
//    quad whole in one CTA is finished by that CTA; a quad cut between CTA ranges is finished by the
//    first of its CTAs (whose part of the quad comes last in its range), which polls the others'
//    fp32 partials -- stored as 64-bit words (value | phase tag) -- and sums them in CTA order. The
//    finisher writes y and, for the phase that reads it, the final bf16 values as tagged words of an
//    exchange buffer; a consumer CTA polls those words while it stages its x. So a phase starts on an
//    SM as soon as its inputs exist, and no store needs a fence: each word carries its own tag. Tags
//    are unique per (launch, phase); exchange and slot buffers rotate over three phases, which the
//    host proves safe when the plan is made (or places a grid barrier);
//  * tensor parallel plans (one process per GPU): after a row-parallel phase (G4Q_PHASE_ALLREDUCE)
//    each CTA stores its tagged partial of every quad it touched into the rank-partial buffer of
//    every rank over NVLink (peer stores); the finisher of the quad on each rank polls all ranks'
//    partials and adds them in rank-then-CTA order, so the allreduce after o/down needs no separate
//    collective and every rank sees the same bits. The LM-head keys are exchanged the same way at
//    the end of the step;
//  * the argmax phase keeps 64-bit keys (order-preserving logit bits | ~row); its cut quads are
//    finished like any other, and the last CTA to finish publishes tokens/values/keys. The last CTA
//    to leave resets the counters and advances the launch counter (the tag base), so a plan is ready
//    for the next launch and for CUDA-graph replay without a memset.
// Every wait is bounded (about two seconds of clocks); a wait that gives up records an error code
// in the per-device error word and the kernel runs to its end.
#include <algorithm>
#include <cmath>
#include <mutex>
#include <string>
#include <vector>

#include "g4q_common.cuh"
#include "g4q_internal.h"

namespace g4q {
namespace {

constexpr int kWarps = 16;                        // warps per CTA at M = 1, 2, 4 (the most at any M)
constexpr int kThreads = kWarps * 32;
constexpr int kMaxStages = 3;
constexpr uint32_t kUnitPacked = 4 * 512;
constexpr uint32_t kUnitSb = 64 * 4;
constexpr uint32_t kUnitBytes = kUnitPacked + kUnitSb;
constexpr int kMaxPlanTokens = 8;                 // tokens per step (M): 1, 2, 4 or 8
constexpr int kXKeyStride = 16;                   // key-exchange words per rank: keys[0..M), tag at [15]

// Warps per CTA and ring stages per warp at M tokens: 16 warps of three stages at M <= 4; at M = 8
// the partial-sum buffers (2 x 64 rows x 8 tokens of fp32 per warp) and the tokens' x need the room,
// so 12 warps of two stages (55 KB of weights in flight per SM, still above what HBM latency needs).
template <int kM>
constexpr int warps_of() { return kM == 8 ? 12 : kWarps; }
template <int kM>
constexpr int ring_stages() { return kM == 8 ? 2 : 3; }
int warps_for(int tokens) { return tokens == 8 ? 12 : kWarps; }
int stages_for(int tokens) { return tokens == 8 ? 2 : 3; }
constexpr uint32_t kFlagPrologue = 0x100u;           // PhaseDev::flags: the phase has a prologue
constexpr int kSlots = 16;                        // CTA ranges one 64-row quad may be cut into
constexpr int kBufs = 3;                          // exchange / slot buffers rotate over three phases
constexpr int kMaxCtaQuads = 64;                  // quads one CTA range may touch in a phase
constexpr int kMaxRanks = 8;
constexpr int kMaxXQuads = 256;                   // 64-wide groups of x a phase may read (K <= 16384)
constexpr long long kSpinLimit = 4000000000ll;    // ~2 s of SM clocks
constexpr uint32_t kOddNibbleMask = 0x00F000F0u;  // q at bits 4-7 of each half: bf16 value q * 2^-129

struct PhaseDev {
    const uint32_t* packed;
    const uint32_t* sb;
    const uint16_t* x;
    void* y;
    int N, K, R, G, Q, U;
    uint32_t flags;
    int src;          // phase whose output x is (-1: external input or an older output)
    int src_col;      // first column of x inside that phase's output (multiple of 64)
    int src_ranks;    // ranks whose partials each quad of this phase sums (1, or n_ranks if ALLREDUCE)
    int ar;           // ordinal of this allreduce phase among the plan's allreduce phases (-1: none)
    int ks;           // slot rows per (quad, rank): the most CTA ranges one quad meets
    int sync_before;  // wait for every CTA to finish the previous phase before staging x
    int need_done;    // count finished CTAs of this phase (a later barrier or the argmax publish)
    int xout;         // the next phase stages this phase's output from the exchange buffer
    int64_t ldx, ldy; // row strides of x and y (elements), one row per token
    int xwin;         // 0: every CTA stages all of x (slot = group); 1: only the groups of its own range
                      // (slot = unit index relative to the range start; the range is shorter than G)
    int xslots;       // 64-wide slots of x staged per token
    int nout;         // output features: N, or N / 2 for a GeGLU phase
    // prologue (G4qPhasePrologue): elementwise work on the staged x before the matmul
    const uint16_t* post_w;   // post-norm weight of the staged values (bf16 [K]) or null
    const uint16_t* norm_w;   // input-norm weight (bf16 [K]) or null
    const uint16_t* scalar;   // layer scalar (one bf16) or null
    uint16_t* res_user;       // copy of the updated residual stream [M, ld_res_user] or null
    int64_t ld_res_user;
    int res_mode;             // 0 none, 1 the staged values start the residual stream, 2 added to it
    int res_in, res_out;      // residual-stream buffers read (mode 2) and written (modes 1 and 2); res_out
                              // -1: the stream lives in each CTA's shared memory, res_in words after x
    float peps;               // eps of the prologue norms
};

struct DecodeArgs {
    const PhaseDev* ph;
    int n_phases;
    float eps, softcap;
    int64_t row_offset;                       // global index of the argmax phase's row 0
    unsigned int* done;                       // [n_phases] CTAs that finished each phase
    unsigned int* exit_count;                 // [1]
    unsigned int* run;                        // [1] launches so far (tag base)
    unsigned long long* key;                  // [M] running argmax keys of this rank
    unsigned long long* slots;                // [kBufs][buf_words] tagged fp32 partials of cut quads
    unsigned long long* xbuf;                 // [kBufs][xbuf_words] tagged bf16 pairs of finished outputs
    unsigned long long* rp;                   // this rank's rank-partial buffers (tagged, written by all ranks)
    unsigned long long* const* peer_rp;       // [n_ranks] rank-partial buffers of every rank (device array)
    unsigned long long* const* peer_xkeys;    // [n_ranks] key exchange arrays ([n_ranks][8]) of every rank
    int rank, n_ranks;
    int64_t buf_words;                        // words per slot buffer
    int64_t xbuf_words;                       // words per exchange buffer
    int64_t xbuf_tok;                         // words per token inside an exchange buffer
    int64_t ld_logits;                        // row stride of the optional logits (elements)
    uint16_t* resbuf;                         // [2][M][res_ld] residual stream of plans with prologues
    int64_t res_ld;                           // elements per token of a residual buffer
    float gk_cubic, gk_tanh;                  // GeGLU constants rounded to bf16
    int64_t rp_words;                         // words per rank-partial buffer
    int32_t* tokens;
    float* values;
    unsigned long long* keys_out;
    uint16_t* logits;                         // optional bf16 logits of the argmax phase
    int* err;
    unsigned long long* trace;                // kTrace: [C][n_phases][kTraceWords] globaltimer stamps
};

// Per-phase timeline of one CTA (tracing instantiation only): word 0 phase entry, 1 producers of x
// done (every wait before staging met), 2 x staged and its RMS scale known, 3 + w the end of warp w's
// units (after its last park).
constexpr int kTraceWords = 3 + kWarps;

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

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

// CTA c of C owns units [range_start(c), range_start(c + 1)) of a phase with U units. The owner of
// unit u is the largest c with floor(c*U/C) <= u, i.e. c*U < (u+1)*C: c = ((u+1)*C - 1) / U.
// (U*C < 2^32 is checked when the plan is made.)
__device__ __forceinline__ int range_start(int c, int U, int C) { return (int)(((uint32_t)c * (uint32_t)U) / (uint32_t)C); }

__device__ __forceinline__ int cta_of_unit(int u, int U, int C) {
    return (int)(((uint32_t)(u + 1) * (uint32_t)C - 1u) / (uint32_t)U);
}

// CTA range [cf, cl] covering quad q of a phase (cf == cl: the quad is whole in one CTA).
__device__ __forceinline__ void quad_ctas(const PhaseDev& P, int q, int C, int& cf, int& cl) {
    cf = cta_of_unit(q * P.G, P.U, C);
    cl = cta_of_unit((q + 1) * P.G - 1, P.U, C);
}

// Tag of phase p given the launch's tag base: unique per (launch, phase) over 2^32 - 1 phases,
// never 0 (the value slot buffers start with).
__device__ __forceinline__ uint32_t phase_tag(uint32_t tag0, int p) {
    uint32_t t = tag0 + (uint32_t)p;   // tag0 < 2^32 - 1, p < 2^16
    if (t < tag0 || t >= 0xFFFFFFFFu) t -= 0xFFFFFFFFu;
    return t + 1u;
}

// Slots of a phase live in buffer p mod 3: tagged fp32 partials, word index of (quad q, source CTA
// offset c = cta - cf, token tok, row 0).
template <int kM>
__device__ __forceinline__ int64_t slot_w(const DecodeArgs& a, const PhaseDev& P, int p, int q, int c, int tok) {
    return (int64_t)(p % kBufs) * a.buf_words + (((int64_t)q * P.ks + c) * kM + tok) * 64;
}

// Finished bf16 outputs of phase p in exchange buffer p mod 3: word of (token, output pair n/2).
__device__ __forceinline__ int64_t xbuf_w(const DecodeArgs& a, int p, int tok, int n) {
    return (int64_t)(p % kBufs) * a.xbuf_words + (int64_t)tok * a.xbuf_tok + (n >> 1);
}

// Rank partials of the allreduce phase with ordinal ar: word index of (quad q, slot, token tok, row 0),
// where the partial of rank r's c-th CTA of a quad cut into nc CTA ranges takes slot r * nc + c, so a
// quad's n_ranks * nc partials are contiguous in rank-major, CTA order (one flattened poll sums them);
// at 4 and 8 tokens per step, and at 2 on more than two ranks, rank r's summed partial takes slot r.
// The buffers rotate over allreduce ordinals: a rank writes buffer j mod 3 again only after every
// rank has sent allreduce j+2, i.e. after every rank has finished reading allreduce j.
template <int kM>
__device__ __forceinline__ int64_t rp_word(const DecodeArgs& a, const PhaseDev& P, int ar, int q, int slot, int tok) {
    return (int64_t)(ar % kBufs) * a.rp_words + (((((int64_t)q * a.n_ranks * P.ks) + slot) * kM + tok) * 64);
}

// Warp w owns the contiguous units [wstart(w), wstart(w + 1)) of its CTA's n units of a phase
// (relative numbering): the first n % kW warps take one unit more, warps past n own none.
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

// The prefetching position of one warp, across phases: the next unit to issue is group g of the
// current quad of phase p, at byte offsets off_p / off_s of that phase's packed words / sb.
template <int kW>
struct Pre {
    int p, left, g, G;
    uint32_t off_p, off_s, step_p, step_s;
    const char* base_p;
    const char* base_s;
    __device__ __forceinline__ void enter(const DecodeArgs& a, int cta, int C, int w) {
        while (p < a.n_phases) {
            const PhaseDev& P = a.ph[p];
            const int cs = range_start(cta, P.U, C), n = range_start(cta + 1, P.U, C) - cs;
            const int u0 = wstart<kW>(w, n);
            left = wstart<kW>(w + 1, n) - u0;
            if (left > 0) {
                G = P.G;
                const int u = cs + u0, q = u / G;
                g = u - q * G;
                step_p = (uint32_t)P.R * 512u;
                step_s = (uint32_t)P.N * 4u;
                off_p = (uint32_t)g * step_p + (uint32_t)q * 2048u;
                off_s = (uint32_t)g * step_s + (uint32_t)q * 256u;
                base_p = reinterpret_cast<const char*>(P.packed);
                base_s = reinterpret_cast<const char*>(P.sb);
                return;
            }
            ++p;
        }
    }
    __device__ __forceinline__ void next(const DecodeArgs& a, int cta, int C, int w) {
        if (--left > 0) {
            if (++g == G) {   // next quad: group 0, four row tiles further
                g = 0;
                off_p += 2048u - (uint32_t)(G - 1) * step_p;
                off_s += 256u - (uint32_t)(G - 1) * step_s;
            } else {
                off_p += step_p;
                off_s += step_s;
            }
            return;
        }
        ++p;
        enter(a, cta, C, w);
    }
    __device__ __forceinline__ void issue(uint32_t dst, uint32_t bar) const {
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(kUnitBytes) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         dst),
                     "l"(base_p + off_p), "r"(kUnitPacked), "r"(bar)
                     : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         dst + kUnitPacked),
                     "l"(base_s + off_s), "r"(kUnitSb), "r"(bar)
                     : "memory");
    }
};

template <int kM>
struct CtaShared {
    unsigned long long bars[kWarps][kMaxStages];
    float wss[kWarps][kM];
    float rs[kM];
    uint32_t tag0;
    int qcnt[kMaxCtaQuads];   // arrivals per quad of the CTA's range (reset by the last arriver)
    int warps_finished;
    unsigned long long best[kM];
};

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned int atom_add_acq_rel(unsigned int* p, unsigned int v) {
    unsigned int old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ void spin_until(const unsigned int* ctr, unsigned int target, int* err) {
    if (ld_acquire(ctr) >= target) return;
    const long long t0 = clock64();
    while (ld_acquire(ctr) < target) {
        if (*reinterpret_cast<volatile int*>(err) != 0) return;
        if (clock64() - t0 > kSpinLimit) {
            atomicCAS(err, 0, 34);
            return;
        }
    }
}

__device__ __forceinline__ void ld_relaxed2(const unsigned long long* p, unsigned long long& a, unsigned long long& b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long tagged(float v, uint32_t tag) {
    return (unsigned long long)__float_as_uint(v) | ((unsigned long long)tag << 32);
}

// The finisher's sum over n tagged source rows of a quad (rows lane and lane + 32 of each, source
// stride `stride` words), in source order after `init` (when has_init), polling until every word
// carries `tag`: the sources are other CTAs' (and ranks') partials, stored on their own schedule; a
// short sleep between polls leaves the issue slots to the warps still streaming. Bounded: a wait that
// gives up records code 35 and returns what it has.
__device__ __noinline__ float2 poll_sum(const unsigned long long* base, int n, int stride, uint32_t tag, float2 init,
                                        bool has_init, int* err) {
    const int lane = threadIdx.x & 31;
    float2 s = init;
    bool have = has_init;
    const long long t0 = clock64();
    for (int i0 = 0; i0 < n; i0 += 4) {
        unsigned long long w[4][2];
        for (;;) {
            bool ok = true;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (i0 + e < n) {
                    const unsigned long long* src = base + (int64_t)(i0 + e) * stride;
                    w[e][0] = ld_relaxed(src + lane);
                    w[e][1] = ld_relaxed(src + lane + 32);
                    ok &= (uint32_t)(w[e][0] >> 32) == tag && (uint32_t)(w[e][1] >> 32) == tag;
                }
            }
            if (__all_sync(0xffffffffu, ok)) break;
            if (*reinterpret_cast<volatile int*>(err) != 0) return s;
            if (clock64() - t0 > kSpinLimit) {
                atomicCAS(err, 0, 35);
                return s;
            }
            __nanosleep(20);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            if (i0 + e < n) {
                const float v0 = __uint_as_float((uint32_t)w[e][0]), v1 = __uint_as_float((uint32_t)w[e][1]);
                if (have) {
                    s.x += v0;
                    s.y += v1;
                } else {
                    s = make_float2(v0, v1);
                    have = true;
                }
            }
        }
    }
    return s;
}

// A CTA's partial of a quad of an allreduce phase, tagged, into its slot row of every rank's
// rank-partial buffer (NVLink peer stores for the other ranks).
__device__ __forceinline__ void send_partial(unsigned long long* const* peers, int n_ranks, int64_t w0, float v0,
                                             float v1, uint32_t tag) {
    const int lane = threadIdx.x & 31;
    const unsigned long long e0 = tagged(v0, tag), e1 = tagged(v1, tag);
    for (int r = 0; r < n_ranks; ++r) {
        unsigned long long* dst = peers[r] + w0;
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst + lane), "l"(e0) : "memory");
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst + lane + 32), "l"(e1) : "memory");
    }
}

// GeGLU phase: the paired quad's row lane is gate feature 32q + lane, row lane + 32 the matching up
// feature; both are rounded to bf16 as the matmul output would be, then the GeGLU.
__device__ __forceinline__ void publish_geglu(const DecodeArgs& a, const PhaseDev& P, int p, int q, int tok, float f0,
                                           float f1, uint32_t tag) {
    const int lane = threadIdx.x & 31;
    const uint32_t o = geglu_bf16(bf16_bits_to_f32(f32_to_bf16_bits(f0)), bf16_bits_to_f32(f32_to_bf16_bits(f1)),
                                  a.gk_cubic, a.gk_tanh);
    reinterpret_cast<uint16_t*>(P.y)[(int64_t)tok * P.ldy + (int64_t)q * 32 + lane] = (uint16_t)o;
    if (P.xout) {
        const uint32_t n = __shfl_down_sync(0xffffffffu, o, 1);
        if ((lane & 1) == 0)
            st_relaxed(a.xbuf + xbuf_w(a, p, tok, q * 32 + lane),
                       (unsigned long long)(o | (n << 16)) | ((unsigned long long)tag << 32));
    }
}

// Finished rows lane and lane + 32 of quad q of phase p for one token (unscaled sums v0, v1):
// y = v * rs, and for a phase the next one reads, the bf16 values as tagged pairs in the exchange
// buffer (even lanes store the pairs (lane, lane + 1) and (lane + 32, lane + 33)).
// kPro: the plan has prologue or GeGLU phases (plans without them run kernels without that code,
// whose finishers and register allocation stay those of the plain matmul chain).
template <bool kPro>
__device__ __forceinline__ void publish(const DecodeArgs& a, const PhaseDev& P, int p, int q, int tok, float v0,
                                        float v1, float rs, uint32_t tag) {
    const int lane = threadIdx.x & 31;
    const float f0 = __fmul_rn(v0, rs), f1 = __fmul_rn(v1, rs);
    if constexpr (kPro) {
        if (P.flags & G4Q_PHASE_GEGLU) {
            publish_geglu(a, P, p, q, tok, f0, f1, tag);
            return;
        }
    }
    const int64_t yo = (int64_t)tok * P.ldy + (int64_t)q * 64;
    if (P.flags & G4Q_QMM_OUT_F32) {
        float* y = reinterpret_cast<float*>(P.y) + yo;
        y[lane] = f0;
        y[lane + 32] = f1;
        return;
    }
    const uint32_t b0 = f32_to_bf16_bits(f0), b1 = f32_to_bf16_bits(f1);
    uint16_t* y = reinterpret_cast<uint16_t*>(P.y) + yo;
    y[lane] = (uint16_t)b0;
    y[lane + 32] = (uint16_t)b1;
    if (P.xout) {
        const uint32_t n0 = __shfl_down_sync(0xffffffffu, b0, 1), n1 = __shfl_down_sync(0xffffffffu, b1, 1);
        if ((lane & 1) == 0) {
            const unsigned long long t = (unsigned long long)tag << 32;
            unsigned long long* xw = a.xbuf + xbuf_w(a, p, tok, q * 64);
            st_relaxed(xw + (lane >> 1), (unsigned long long)(b0 | (n0 << 16)) | t);
            st_relaxed(xw + 16 + (lane >> 1), (unsigned long long)(b1 | (n1 << 16)) | t);
        }
    }
}

// argmax phase: fold one finished output into the running key
__device__ __forceinline__ unsigned long long fold_logit(uint16_t* logits, float softcap, int64_t row_offset, int n,
                                                         float o, unsigned long long best) {
    const uint16_t lb = f32_to_bf16_bits(o);
    if (logits) logits[n] = lb;
    const float lv = bf16_bits_to_f32(lb);
    const float sv = softcap > 0.0f ? softcap_bf16(lv, softcap) : lv;
    const unsigned long long key = argmax_key(sv, (uint32_t)(row_offset + n));
    return key > best ? key : best;
}

// Park this warp's partial of quad q (its 64 rows for each of the M tokens). A warp keeps the partial
// of the first quad of its range in red[warp][0] (the previous warp may need it) and everything else
// in red[warp][1] (only the last quad of the range is read by another warp, and it comes last). The
// last contributing warp sums the partials in warp order, which gives the CTA's partial of the quad,
// and then, per token:
//  * allreduce phase: stores it, tagged, into every rank's rank-partial buffer; the quad's finisher
//    CTA (the first CTA of the quad) then sums all ranks' partials and publishes the quad;
//  * a quad whole in this CTA: publishes it (argmax phase: folds the logits into the running key);
//  * a cut quad: a CTA other than the quad's first stores its tagged partial in its slot; the first
//    CTA, whose share of the quad is the last of its range, polls the others' slots, sums them in CTA
//    order after its own and publishes (or folds) the quad.
// No warp waits here except a finisher, for partials that are (or are about to be) stored.
template <bool kTP, int kM, bool kPro>
__device__ __forceinline__ void park(const DecodeArgs& a, const PhaseDev& P, int p, CtaShared<kM>& sh, float* red,
                                     int q, int first_q, int cs, int ce, int cta, int C, const float (&acc)[4][4],
                                     unsigned long long (&best)[kM]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gi = lane >> 2, t = lane & 3;
    const int G = P.G, n = ce - cs;
    float* rb = red + (size_t)(warp * 2 + (q == first_q ? 0 : 1)) * kM * 64;
    // C fragment: lane (gi, t) holds rows gi, gi + 8 of each tile for tokens 2t, 2t + 1
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int tok = 2 * t + (e & 1);
            if (tok < kM) rb[tok * 64 + i * 16 + gi + ((e & 2) ? 8 : 0)] = acc[i][e];
        }
    __threadfence_block();
    __syncwarp();
    const int lo = max(cs, q * G), hi = min(ce, (q + 1) * G);
    constexpr int kW = warps_of<kM>();
    const int wa = warp_of<kW>(lo - cs, n), wb = warp_of<kW>(hi - 1 - cs, n);
    const int qi = q - cs / G;
    if (wb > wa) {
        int last = 0;
        if (lane == 0) last = atomicAdd(&sh.qcnt[qi], 1) == wb - wa;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) return;
        __threadfence_block();
        if (lane == 0) sh.qcnt[qi] = 0;
    }
    // warp wa holds q in slot 0 only if q is also its first quad; the others hold it as their first
    const int slot_a = (cs + wstart<kW>(wa, n)) / G == q ? 0 : 1;
    float2 f[kM];
#pragma unroll
    for (int tok = 0; tok < kM; ++tok) {
        float v[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int row = tok * 64 + lane + 32 * h;
            float s = red[(wa * 2 + slot_a) * kM * 64 + row];
            for (int w = wa + 1; w <= wb; ++w) s += red[w * 2 * kM * 64 + row];
            v[h] = s;
        }
        f[tok] = make_float2(v[0], v[1]);
    }
    const bool whole = cs <= q * G && ce >= (q + 1) * G;
    const bool argmax = (P.flags & G4Q_PHASE_ARGMAX) != 0;
    const uint32_t tag = phase_tag(sh.tag0, p);
    int cf, cl;
    quad_ctas(P, q, C, cf, cl);
    bool two_level = false;
    if constexpr (kM >= 4) two_level = true;
    if constexpr (kM == 2) two_level = a.n_ranks > 2;
    if (kTP && P.src_ranks > 1) {
        if (two_level) {
            // two levels: the finisher polls each token's partials one token after another, so at 4 and
            // 8 tokens (and at 2 on more than two ranks) the quad's first CTA sums this rank's CTA
            // partials first (local slots, CTA order), then sends one rank partial (slot = rank) to
            // every rank and sums the ranks' in rank order -- n_ranks sources per token to poll
            // instead of n_ranks x (CTAs of the quad)
            if (!whole) {
                if (cta != cf) {
#pragma unroll
                    for (int tok = 0; tok < kM; ++tok) {
                        unsigned long long* sl = a.slots + slot_w<kM>(a, P, p, q, cta - cf, tok);
                        st_relaxed(sl + lane, tagged(f[tok].x, tag));
                        st_relaxed(sl + lane + 32, tagged(f[tok].y, tag));
                    }
                    return;
                }
#pragma unroll
                for (int tok = 0; tok < kM; ++tok)
                    f[tok] = poll_sum(a.slots + slot_w<kM>(a, P, p, q, 1, tok), cl - cf, kM * 64, tag, f[tok], true,
                                      a.err);
            }
#pragma unroll
            for (int tok = 0; tok < kM; ++tok)
                send_partial(a.peer_rp, a.n_ranks, rp_word<kM>(a, P, P.ar, q, a.rank, tok), f[tok].x, f[tok].y, tag);
#pragma unroll
            for (int tok = 0; tok < kM; ++tok)
                f[tok] = poll_sum(a.rp + rp_word<kM>(a, P, P.ar, q, 0, tok), a.n_ranks, kM * 64, tag, f[tok], false,
                                  a.err);
        } else {
#pragma unroll
            for (int tok = 0; tok < kM; ++tok)
                send_partial(a.peer_rp, a.n_ranks, rp_word<kM>(a, P, P.ar, q, a.rank * (cl - cf + 1) + cta - cf, tok),
                             f[tok].x, f[tok].y, tag);
            if (cta != cf) return;
            const int nc = cl - cf + 1;
#pragma unroll
            for (int tok = 0; tok < kM; ++tok)   // rank-major, then CTA order: the same bits on every rank
                f[tok] = poll_sum(a.rp + rp_word<kM>(a, P, P.ar, q, 0, tok), a.n_ranks * nc, kM * 64, tag, f[tok],
                                  false, a.err);
        }
    } else if (!whole) {
        if (cta != cf) {
#pragma unroll
            for (int tok = 0; tok < kM; ++tok) {
                unsigned long long* sl = a.slots + slot_w<kM>(a, P, p, q, cta - cf, tok);
                st_relaxed(sl + lane, tagged(f[tok].x, tag));
                st_relaxed(sl + lane + 32, tagged(f[tok].y, tag));
            }
            return;
        }
#pragma unroll
        for (int tok = 0; tok < kM; ++tok)
            f[tok] = poll_sum(a.slots + slot_w<kM>(a, P, p, q, 1, tok), cl - cf, kM * 64, tag, f[tok], true, a.err);
    }
#pragma unroll
    for (int tok = 0; tok < kM; ++tok) {
        if (argmax) {
            uint16_t* lg = a.logits ? a.logits + (int64_t)tok * a.ld_logits : nullptr;
            best[tok] = fold_logit(lg, a.softcap, a.row_offset, q * 64 + lane, __fmul_rn(f[tok].x, sh.rs[tok]), best[tok]);
            best[tok] = fold_logit(lg, a.softcap, a.row_offset, q * 64 + lane + 32, __fmul_rn(f[tok].y, sh.rs[tok]),
                                   best[tok]);
        } else {
            publish<kPro>(a, P, p, q, tok, f[tok].x, f[tok].y, sh.rs[tok], tag);
        }
    }
}

// Shared-memory order of x: inside each 64-wide group, lane t's B-fragment words for the four k16
// steps (j) sit together: word w = 8j + t + 4hi of the group goes to slot 8t + 2j + hi, so a lane
// fetches the whole group's fragments with two 16-byte loads.
__device__ __forceinline__ int xperm(int w) {
    const int r = w & 7;
    return (w & ~31) | ((r & 3) << 3) | (((w >> 3) & 3) << 1) | (r >> 2);
}

// The 64-wide group of x that staging slot j of a CTA range starting at unit cs holds.
__device__ __forceinline__ int slot_group(const PhaseDev& P, int cs, int j) {
    return P.xwin ? (cs + j) % P.G : j;
}

constexpr int kMaxStageLoads = 8;   // 16-byte exchange loads per thread and token (four values each)
// 16 warps stage the widest x in one pass; with 12 warps (M = 8) the host refuses a phase whose
// staged x from the exchange buffer exceeds kMaxStageLoads loads per thread
static_assert(kMaxStageLoads * kThreads * 4 >= kMaxXQuads * 64, "staging must cover the widest x");

// Staging of one token's x from the exchange buffer (out of line: its loads in flight need registers
// the streaming loop does not have to keep free): the finished bf16 pairs of the producer phase,
// polled until they carry that phase's tag; every load of a thread is in flight at once, and only
// words still missing are loaded again. src points at the token's word of x's first column.
// kWin: the CTA's window (slot j holds group (cs + j) mod G); otherwise slot j holds group j. The
// phase's numbers come by value: loads through the phase record would be repeated after every
// polling load (each is a memory clobber).
template <bool kWin, int kT>
__device__ __noinline__ float stage_xbuf(const unsigned long long* src, int nslots, int cs, int G, uint32_t tag,
                                         uint32_t* xs, bool rms, int* err) {
    float ss = 0.0f;
    auto acc_sq = [&](uint32_t w) {
        const float lo = bf16_bits_to_f32(w & 0xffffu), hi = bf16_bits_to_f32(w >> 16);
        ss = __fadd_rn(ss, __fmul_rn(lo, lo));
        ss = __fadd_rn(ss, __fmul_rn(hi, hi));
    };
    const int nl = nslots * 16;   // 16-byte loads: two tagged words, four values; 16 per slot
    auto word_of = [&](int i) -> int64_t {
        if constexpr (kWin)
            return (int64_t)((cs + (i >> 4)) % G) * 32 + 2 * (i & 15);
        else
            return (int64_t)2 * i;
    };
    uint32_t w[kMaxStageLoads][2];   // the value halves of the words (the tags are checked on arrival)
    uint32_t missing = 0;
#pragma unroll
    for (int j = 0; j < kMaxStageLoads; ++j) {
        const int i = threadIdx.x + j * kT;
        if (i < nl) {
            unsigned long long u0, u1;
            ld_relaxed2(src + word_of(i), u0, u1);
            w[j][0] = (uint32_t)u0;
            w[j][1] = (uint32_t)u1;
            if ((uint32_t)(u0 >> 32) != tag || (uint32_t)(u1 >> 32) != tag) missing |= 1u << j;
        }
    }
    if (missing) {
        const long long t0 = clock64();
        while (missing) {
#pragma unroll
            for (int j = 0; j < kMaxStageLoads; ++j) {
                if (missing & (1u << j)) {
                    const int i = threadIdx.x + j * kT;
                    unsigned long long u0, u1;
                    ld_relaxed2(src + word_of(i), u0, u1);
                    w[j][0] = (uint32_t)u0;
                    w[j][1] = (uint32_t)u1;
                    if ((uint32_t)(u0 >> 32) == tag && (uint32_t)(u1 >> 32) == tag) missing &= ~(1u << j);
                }
            }
            if (missing && (*reinterpret_cast<volatile int*>(err) != 0 || clock64() - t0 > kSpinLimit)) {
                atomicCAS(err, 0, 37);
                break;
            }
        }
    }
#pragma unroll
    for (int j = 0; j < kMaxStageLoads; ++j) {
        const int i = threadIdx.x + j * kT;
        if (i < nl) {
            const uint32_t lo = w[j][0], hi = w[j][1];
            xs[xperm(2 * i)] = lo;
            xs[xperm(2 * i + 1)] = hi;
            if (rms) {
                acc_sq(lo);
                acc_sq(hi);
            }
        }
    }
    return ss;
}

// Stage the x of phase P (per token: K bf16 values, or the CTA's window of groups) into shared memory,
// token tok at xs + tok * xslots * 32 words; ss[tok] receives this thread's sum of squares (every CTA
// maps values to threads the same way, so every CTA derives the same RMS scale). From an external
// input: plain 16-byte copies; from the previous phase's output: its exchange words.
template <int kM>
__device__ __forceinline__ void stage_x(const DecodeArgs& a, const PhaseDev& P, uint32_t* xs, int cs, uint32_t tag0,
                                        bool rms, float (&ss)[kM]) {
#pragma unroll
    for (int tok = 0; tok < kM; ++tok) {
        uint32_t* xt = xs + (size_t)tok * P.xslots * 32;
        float s = 0.0f;
        if (P.src < 0) {
            for (int u = threadIdx.x; u < P.xslots * 8; u += warps_of<kM>() * 32) {
                const int g = slot_group(P, cs, u >> 3);
                const uint4 v = __ldcg(reinterpret_cast<const uint4*>(P.x + (int64_t)tok * P.ldx + (int64_t)g * 64) + (u & 7));
                xt[xperm(4 * u)] = v.x;
                xt[xperm(4 * u + 1)] = v.y;
                xt[xperm(4 * u + 2)] = v.z;
                xt[xperm(4 * u + 3)] = v.w;
                if (rms) {
                    const uint32_t pv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float lo = bf16_bits_to_f32(pv[e] & 0xffffu), hi = bf16_bits_to_f32(pv[e] >> 16);
                        s = __fadd_rn(s, __fmul_rn(lo, lo));
                        s = __fadd_rn(s, __fmul_rn(hi, hi));
                    }
                }
            }
        } else {
            const unsigned long long* src = a.xbuf + xbuf_w(a, P.src, tok, P.src_col);
            if (kM > 1 && P.xwin)
                s = stage_xbuf<kM != 1, warps_of<kM>() * 32>(src, P.xslots, cs, P.G, phase_tag(tag0, P.src), xt, rms,
                                                             a.err);
            else
                s = stage_xbuf<false, warps_of<kM>() * 32>(src, P.xslots, cs, P.G, phase_tag(tag0, P.src), xt, rms,
                                                           a.err);
        }
        ss[tok] = s;
    }
}

// Per token, 1/sqrt(mean(v^2) + eps) from every thread's partial sum of squares: warp sums, then
// every thread adds the warps in warp order, so every thread (and every CTA) gets the same bits;
// the rounding of g4q_rms_norm (fp32 fma accumulation, correctly rounded reciprocal square root).
template <int kM>
__device__ __forceinline__ void cta_inv_rms(CtaShared<kM>& sh, float (&ss)[kM], int K, float eps, float (&inv)[kM]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int tok = 0; tok < kM; ++tok) {
        float v = ss[tok];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0) sh.wss[warp][tok] = v;
    }
    __syncthreads();
#pragma unroll
    for (int tok = 0; tok < kM; ++tok) {
        float s = 0.0f;
        for (int w = 0; w < warps_of<kM>(); ++w) s += sh.wss[w][tok];
        inv[tok] = __frsqrt_rn(s / (float)K + eps);
    }
    __syncthreads();   // sh.wss is written again by the next reduction
}

// The phase's prologue, in place on the staged x of every token (all K columns staged: a prologue
// phase is never windowed). Thread t owns the pair words t, t + kT, ... (columns 2w, 2w + 1)
// in every pass, so no pass needs a barrier of its own beyond the norms' reductions.
template <int kM>
__device__ __noinline__ void prologue(const DecodeArgs& a, const PhaseDev& P, uint32_t* xs, CtaShared<kM>& sh,
                                      int cta) {
    constexpr int kT = warps_of<kM>() * 32;
    const int K = P.K, words = K / 2, tstride = P.xslots * 32;
    auto bfv = [](uint32_t h) { return bf16_bits_to_f32(h & 0xffffu); };
    auto rb = [](float f) { return bf16_bits_to_f32(f32_to_bf16_bits(f)); };
    float ss[kM], inv[kM];
    if (P.post_w != nullptr) {
#pragma unroll
        for (int tok = 0; tok < kM; ++tok) {
            float s = 0.0f;
            for (int w = threadIdx.x; w < words; w += kT) {
                const uint32_t v = xs[tok * tstride + xperm(w)];
                const float lo = bfv(v), hi = bfv(v >> 16);
                s = fmaf(lo, lo, s);
                s = fmaf(hi, hi, s);
            }
            ss[tok] = s;
        }
        cta_inv_rms<kM>(sh, ss, K, P.peps, inv);
#pragma unroll
        for (int tok = 0; tok < kM; ++tok)
            for (int w = threadIdx.x; w < words; w += kT) {
                uint32_t* e = xs + tok * tstride + xperm(w);
                const uint32_t v = *e, wv = __ldg(reinterpret_cast<const uint32_t*>(P.post_w) + w);
                const float lo = rb(bfv(wv) * rb(bfv(v) * inv[tok]));
                const float hi = rb(bfv(wv >> 16) * rb(bfv(v >> 16) * inv[tok]));
                *e = (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
            }
    }
    if (P.res_mode != 0 || P.norm_w != nullptr) {
        // Where the stream lives: in this CTA's shared memory when it fits (every CTA stages all of x
        // in every prologue phase and computes the same bits, so each keeps its own copy, and thread t
        // always owns the same words: no memory traffic, no fence); otherwise in the plan's global
        // double buffer, written by CTA 0, which fenced before publishing that phase's first quad --
        // this CTA has polled that quad's words, so a fence orders its reads.
        const bool sm = P.res_out < 0;
        if (P.res_mode == 2 && !sm) __threadfence();
        const float sc = P.scalar != nullptr ? bf16_bits_to_f32(*P.scalar) : 1.0f;
#pragma unroll
        for (int tok = 0; tok < kM; ++tok) {
            uint32_t* rsm = sm ? xs + P.res_in + tok * (int)(a.res_ld / 2) : nullptr;
            const uint32_t* rin =
                sm ? nullptr : reinterpret_cast<const uint32_t*>(a.resbuf + (P.res_in * kM + tok) * a.res_ld);
            uint32_t* rout = sm ? nullptr : reinterpret_cast<uint32_t*>(a.resbuf + (P.res_out * kM + tok) * a.res_ld);
            uint32_t* ruser =
                P.res_user != nullptr ? reinterpret_cast<uint32_t*>(P.res_user + (int64_t)tok * P.ld_res_user) : nullptr;
            float s = 0.0f;
            for (int w = threadIdx.x; w < words; w += kT) {
                uint32_t* e = xs + tok * tstride + xperm(w);
                uint32_t v = *e;
                if (P.res_mode == 2) {   // residual add, then the layer scalar, each rounded to bf16
                    const uint32_t r = sm ? rsm[w] : __ldcg(rin + w);
                    float lo = rb(bfv(r) + bfv(v)), hi = rb(bfv(r >> 16) + bfv(v >> 16));
                    if (P.scalar != nullptr) {
                        lo = lo * sc;
                        hi = hi * sc;
                    }
                    v = (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
                    *e = v;
                }
                if (P.res_mode != 0) {
                    if (sm)
                        rsm[w] = v;
                    else if (cta == 0)
                        rout[w] = v;
                    if (ruser && cta == 0) ruser[w] = v;
                }
                const float lo = bfv(v), hi = bfv(v >> 16);
                s = fmaf(lo, lo, s);
                s = fmaf(hi, hi, s);
            }
            ss[tok] = s;
        }
        if (P.res_mode != 0 && cta == 0 && !sm) __threadfence();   // before this CTA publishes anything later
        if (P.norm_w != nullptr) {
            cta_inv_rms<kM>(sh, ss, K, P.peps, inv);
#pragma unroll
            for (int tok = 0; tok < kM; ++tok)
                for (int w = threadIdx.x; w < words; w += kT) {
                    uint32_t* e = xs + tok * tstride + xperm(w);
                    const uint32_t v = *e, wv = __ldg(reinterpret_cast<const uint32_t*>(P.norm_w) + w);
                    const float lo = rb(bfv(wv) * rb(bfv(v) * inv[tok]));
                    const float hi = rb(bfv(wv >> 16) * rb(bfv(v >> 16) * inv[tok]));
                    *e = (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
                }
        }
    }
}

// End of a step on a tensor-parallel plan: every rank's last CTA posts its argmax keys to every rank
// (key words, then the tag with release semantics) and waits for all of them; the maximum per token
// is the step's key on every rank. Also keeps the ranks within one step of each other.
template <int kM>
__device__ __forceinline__ void exchange_keys(const DecodeArgs& a, unsigned long long (&key)[kM], uint32_t tag) {
    for (int r = 0; r < a.n_ranks; ++r) {
        unsigned long long* dst = a.peer_xkeys[r] + kXKeyStride * a.rank;
#pragma unroll
        for (int tok = 0; tok < kM; ++tok)
            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst + tok), "l"(key[tok]) : "memory");
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(dst + kXKeyStride - 1), "l"((unsigned long long)tag)
                     : "memory");
    }
    unsigned long long best[kM];
#pragma unroll
    for (int tok = 0; tok < kM; ++tok) best[tok] = 0ull;
    const long long t0 = clock64();
    for (int r = 0; r < a.n_ranks; ++r) {
        const unsigned long long* src = a.peer_xkeys[a.rank] + kXKeyStride * r;
        for (;;) {
            unsigned long long t;
            asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(t) : "l"(src + kXKeyStride - 1) : "memory");
            if ((uint32_t)t == tag) break;
            if (clock64() - t0 > kSpinLimit) {
                atomicCAS(a.err, 0, 36);
                return;
            }
        }
#pragma unroll
        for (int tok = 0; tok < kM; ++tok) {
            unsigned long long k;
            asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(k) : "l"(src + tok) : "memory");
            best[tok] = k > best[tok] ? k : best[tok];
        }
    }
#pragma unroll
    for (int tok = 0; tok < kM; ++tok) key[tok] = best[tok];
}

// kTP: tensor-parallel instantiation (allreduce phases, key exchange); the single-GPU one has none
// of that code. kM: tokens per step (the MMA's n dimension holds them). kTrace: also stamps each
// CTA's per-phase timeline into a.trace (a profiling build selected at run time; the default
// instantiations have no trace code).
template <bool kTP, int kM, bool kTrace = false, bool kPro = false>
__global__ void __launch_bounds__(warps_of<kM>() * 32, 1) decode_kernel(DecodeArgs a) {
    constexpr int kS = ring_stages<kM>();
    constexpr int kW = warps_of<kM>();
    constexpr uint32_t kRing = kS * kUnitBytes;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ CtaShared<kM> sh;
    // the warp index through a shuffle from lane 0: provably warp-uniform, so the compiler keeps it
    // and everything derived from it (ring and barrier addresses, unit cursors) in uniform registers
    const int warp = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0), lane = threadIdx.x & 31, gi = lane >> 2,
              t = lane & 3;
    const int C = gridDim.x, cta = blockIdx.x;
    uint8_t* ring = smem + (size_t)warp * kRing;
    const uint32_t ring_s = saddr(ring);
    float* red = reinterpret_cast<float*>(smem + (size_t)kW * kRing);
    uint32_t* xs = reinterpret_cast<uint32_t*>(smem + (size_t)kW * kRing + (size_t)2 * kW * kM * 64 * 4);
    const uint32_t bar0 = saddr(&sh.bars[warp][0]);

    if (lane == 0) {
        for (int s = 0; s < kS; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8 * s));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < kMaxCtaQuads; ++i) sh.qcnt[i] = 0;
        sh.warps_finished = 0;
#pragma unroll
        for (int tok = 0; tok < kM; ++tok) {
            sh.best[tok] = 0ull;
            sh.rs[tok] = 1.0f;
        }
        const unsigned long long e = (unsigned long long)*reinterpret_cast<volatile unsigned int*>(a.run) *
                                     (unsigned)(a.n_phases + 1);
        sh.tag0 = (uint32_t)(e % 0xFFFFFFFFull);
    }
    __syncwarp();
    Pre<kW> pre;
    pre.p = 0;
    pre.enter(a, cta, C, warp);

    int stage = 0;
    uint32_t phase_bit = 0;
    unsigned long long best[kM];
#pragma unroll
    for (int tok = 0; tok < kM; ++tok) best[tok] = 0ull;
    // the token whose x this lane's B fragment carries (column gi of the MMA's n dimension); columns
    // past the M tokens repeat token 0 and their accumulators are never read
    const int xtok = gi < kM ? gi : 0;

    for (int p = 0; p < a.n_phases; ++p) {
        const PhaseDev& P = a.ph[p];
        const int cs = range_start(cta, P.U, C), ce = range_start(cta + 1, P.U, C);
        const int G = P.G;
        // ---- phase entry: the CTA's warps are done with the previous phase (x buffer reuse)
        __syncthreads();
        unsigned long long* tr = nullptr;
        if constexpr (kTrace) {
            tr = a.trace + ((size_t)cta * a.n_phases + p) * kTraceWords;
            if (threadIdx.x == 0) tr[0] = global_ns();
        }
        if (P.sync_before) {   // x is not the previous phase's output: a grid barrier first
            if (threadIdx.x == 0) spin_until(a.done + (p - 1), (unsigned)C, a.err);
            __syncthreads();
        }
        if constexpr (kTrace) {
            if (threadIdx.x == 0) tr[1] = global_ns();
        }
        const uint32_t tag0 = sh.tag0;
        // ---- stage x (polls the producer's exchange words) and its RMS scale per token
        const bool rms = (P.flags & G4Q_QMM_RMS_SCALE) != 0;
        float ss[kM];
        stage_x<kM>(a, P, xs, cs, tag0, rms, ss);
        if (p == 0) {   // first weight loads only now: the x loads above are not queued behind them
            for (int s = 0; s < kS && pre.p < a.n_phases; ++s) {
                if (lane == 0) pre.issue(ring_s + s * kUnitBytes, bar0 + 8 * s);
                pre.next(a, cta, C, warp);
            }
        }
        if (rms) {
#pragma unroll
            for (int tok = 0; tok < kM; ++tok) {
                float v = ss[tok];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
                if (lane == 0) sh.wss[warp][tok] = v;
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) {
#pragma unroll
            for (int tok = 0; tok < kM; ++tok) {
                float r = 1.0f;
                if (rms) {
                    float s = 0.0f;
                    for (int w = 0; w < kW; ++w) s = __fadd_rn(s, sh.wss[w][tok]);
                    r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)P.K), a.eps)));
                }
                sh.rs[tok] = r;
            }
            if constexpr (kTrace) tr[2] = global_ns();
        }
        __syncthreads();
        if constexpr (kPro) {
            if (P.flags & kFlagPrologue) {
                prologue<kM>(a, P, xs, sh, cta);
                __syncthreads();
            }
        }

        // ---- this warp's units of phase p
        const int u0 = wstart<kW>(warp, ce - cs);
        const int n_units = wstart<kW>(warp + 1, ce - cs) - u0;
        // B fragments: this lane's token, two 16-byte loads per unit from the unit's x slot
        const uint4* xt = reinterpret_cast<const uint4*>(xs) + (size_t)xtok * P.xslots * 8 + 2 * t;
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[i][e] = 0.0f;
        // the run as segments of whole quads: one park per segment, no per-unit quad bookkeeping
        int cq = (cs + u0) / G, cg = (cs + u0) - cq * G;
        const int first_q = cq;
        for (int k = 0; k < n_units;) {
            const int seg = min(n_units - k, G - cg);
            // x slot of the segment's first unit: its group, or (windowed) its index in the range
            int xslot = cg;
            if constexpr (kM > 1) {
                if (P.xwin) xslot = u0 + k;
            }
            const uint4* xp = xt + (size_t)xslot * 8;
            for (int j = 0; j < seg; ++j, xp += 8) {
                wait_parity(bar0 + 8 * stage, phase_bit, a.err);
                const uint8_t* st = ring + stage * kUnitBytes;
                const uint4 xa = xp[0], xb = xp[1];
                const uint32_t b0[4] = {xa.x, xa.z, xb.x, xb.z}, b1[4] = {xa.y, xa.w, xb.y, xb.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint4 wv = reinterpret_cast<const uint4*>(st + i * 512)[lane];
                    const uint32_t* sbw = reinterpret_cast<const uint32_t*>(st + kUnitPacked) + i * 16 + gi;
                    // row n0 (nibbles at bits 0-3 / 8-11): (128 + q) magic, RN(q*s) = fma((128+q), s, -128 s);
                    // row n1 (bits 4-7 / 12-15): the masked bits read as bf16 are exactly q * 2^-129, so
                    // RN(q*s) = RN((q * 2^-129) * (s * 2^129)) with s * 2^129 exact for |s| < 2^-1
                    // s * 2^129 is an exponent add (the host refuses weights with subnormal scales)
                    const RowConsts c0 = row_consts(sbw[0]);
                    const uint32_t b1s = bcast_hi(sbw[8]);
                    const uint32_t s1h = bcast_lo(sbw[8]) + kExp129x2;
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
                }
                // the unit has been read: refill the buffer with the warp's next unit (maybe of a later phase)
                __syncwarp();
                if (pre.p < a.n_phases) {
                    if (lane == 0) pre.issue(ring_s + stage * kUnitBytes, bar0 + 8 * stage);
                    pre.next(a, cta, C, warp);
                }
                if (++stage == kS) {
                    stage = 0;
                    phase_bit ^= 1u;
                }
            }
            park<kTP, kM, kPro>(a, P, p, sh, red, cq, first_q, cs, ce, cta, C, acc, best);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[i][e] = 0.0f;
            k += seg;
            ++cq;
            cg = 0;
        }
        if constexpr (kTrace) {
            if (lane == 0) tr[3 + warp] = global_ns();
        }
        const bool argmax = (P.flags & G4Q_PHASE_ARGMAX) != 0;
        if (argmax) {
#pragma unroll
            for (int tok = 0; tok < kM; ++tok) {
                unsigned long long kk = best[tok];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    const unsigned long long o = __shfl_xor_sync(0xffffffffu, kk, off);
                    kk = o > kk ? o : kk;
                }
                if (lane == 0) atomicMax(&sh.best[tok], kk);
            }
        }
        // ---- completion count, only where a later barrier or the argmax publish needs it: the warps
        //      meet on a shared counter (CTA scope), the last one publishes with a gpu-scope release
        if (P.need_done) {
            __syncwarp();
            int last_warp = 0;
            if (lane == 0) {
                __threadfence_block();
                last_warp = atomicAdd(&sh.warps_finished, 1) == kW - 1;
            }
            last_warp = __shfl_sync(0xffffffffu, last_warp, 0);
            if (last_warp && lane == 0) {
                __threadfence_block();
                sh.warps_finished = 0;
                if (argmax) {
#pragma unroll
                    for (int tok = 0; tok < kM; ++tok) atomicMax(a.key + tok, sh.best[tok]);
                }
                // a reduction, not an atomic with a result: the warp does not wait for the round
                // trip to L2 before the next phase's CTA barrier (measured: step 2.70 -> 2.62 ms)
                asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.done + p) : "memory");
            }
        }
    }
    // ---- the last CTA out publishes the step's keys, resets the counters and advances the tag base
    const int last = a.n_phases - 1;
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int prev = atom_add_acq_rel(a.exit_count, 1u);
        if (prev == (unsigned)C - 1) {
            unsigned long long k[kM];
#pragma unroll
            for (int tok = 0; tok < kM; ++tok) k[tok] = atomicExch(a.key + tok, 0ull);
            if constexpr (kTP) exchange_keys<kM>(a, k, phase_tag(sh.tag0, a.n_phases));
            if (a.ph[last].flags & G4Q_PHASE_ARGMAX) {
#pragma unroll
                for (int tok = 0; tok < kM; ++tok) {
                    if (a.tokens) a.tokens[tok] = (int32_t)key_index(k[tok]);
                    if (a.values) a.values[tok] = key_value(k[tok]);
                    if (a.keys_out) a.keys_out[tok] = k[tok];
                }
            }
            for (int p = 0; p < a.n_phases; ++p) a.done[p] = 0u;
            atomicAdd(a.run, 1u);
            __threadfence();
            atomicExch(a.exit_count, 0u);
        }
    }
}

// The instantiation a plan launches: tensor parallel or not, tokens per step, tracing (M = 1 only),
// prologue / GeGLU phases present or not.
template <bool kPro>
const void* decode_kernel_pick(bool tp, int tokens, bool trace) {
    if (trace) return tp ? reinterpret_cast<const void*>(decode_kernel<true, 1, true, kPro>)
                         : reinterpret_cast<const void*>(decode_kernel<false, 1, true, kPro>);
    switch (tokens) {
        case 2:
            return tp ? reinterpret_cast<const void*>(decode_kernel<true, 2, false, kPro>)
                      : reinterpret_cast<const void*>(decode_kernel<false, 2, false, kPro>);
        case 4:
            return tp ? reinterpret_cast<const void*>(decode_kernel<true, 4, false, kPro>)
                      : reinterpret_cast<const void*>(decode_kernel<false, 4, false, kPro>);
        case 8:
            return tp ? reinterpret_cast<const void*>(decode_kernel<true, 8, false, kPro>)
                      : reinterpret_cast<const void*>(decode_kernel<false, 8, false, kPro>);
        default:
            return tp ? reinterpret_cast<const void*>(decode_kernel<true, 1, false, kPro>)
                      : reinterpret_cast<const void*>(decode_kernel<false, 1, false, kPro>);
    }
}

const void* decode_kernel_for(bool tp, int tokens, bool trace, bool pro) {
    return pro ? decode_kernel_pick<true>(tp, tokens, trace) : decode_kernel_pick<false>(tp, tokens, trace);
}

size_t ring_bytes_for(int tokens) {
    return (size_t)warps_for(tokens) * stages_for(tokens) * kUnitBytes;
}

}  // namespace

struct DecodePlan {
    uint64_t magic = 0;
    int device = -1;
    int n_phases = 0, grid = 0;
    int tokens = 1;                    // M per step
    int rank = 0, n_ranks = 1;
    size_t smem = 0;
    int64_t buf_words = 0;
    PhaseDev* d_ph = nullptr;
    unsigned int* d_done = nullptr;   // n_phases + 2 (exit counter, launch counter)
    unsigned long long* d_key = nullptr;
    unsigned long long* d_slots = nullptr;
    unsigned long long* d_rp = nullptr;      // rank partials (tensor parallel), written by every rank
    int64_t rp_words = 0;
    unsigned long long* d_xkeys = nullptr;   // [kMaxRanks][kXKeyStride]
    unsigned long long* d_xbuf = nullptr;    // [kBufs][xbuf_words] exchange buffers
    int64_t xbuf_words = 0, xbuf_tok = 0;
    unsigned long long** d_peers = nullptr;   // [2][kMaxRanks]: slot buffers, key arrays of every rank
    unsigned long long* peer_rp[kMaxRanks] = {};
    unsigned long long* peer_xkeys[kMaxRanks] = {};
    unsigned long long* trace = nullptr;      // caller's buffer: runs use the tracing kernel while set
    uint16_t* d_res = nullptr;                // [2][M][res_ld] residual stream of the prologues
    int64_t res_ld = 8;
    bool pro = false;                         // prologue or GeGLU phases: the kernels that carry them
};

constexpr uint64_t kPlanMagic = 0x4734514445434f44ull;

static void free_plan_memory(DecodePlan* plan) {
    cudaFree(plan->d_ph);
    cudaFree(plan->d_done);
    cudaFree(plan->d_key);
    cudaFree(plan->d_slots);
    cudaFree(plan->d_rp);
    cudaFree(plan->d_xkeys);
    cudaFree(plan->d_xbuf);
    cudaFree(plan->d_peers);
    cudaFree(plan->d_res);
}

static void upload_peers(DecodePlan* plan) {
    unsigned long long* table[2 * kMaxRanks];
    for (int r = 0; r < kMaxRanks; ++r) {
        table[r] = plan->peer_rp[r];
        table[kMaxRanks + r] = plan->peer_xkeys[r];
    }
    check_cuda(cudaMemcpy(plan->d_peers, table, sizeof(table), cudaMemcpyHostToDevice), "upload peer pointers");
}

void* decode_plan_create(const G4qDecodePhase* phases, int n, int max_tokens, int rank, int n_ranks,
                         const G4qPhasePrologue* prologues) {
    if (n <= 0 || phases == nullptr) throw Error(G4Q_ERR_INVALID_ARGUMENT, "a plan needs at least one phase");
    if (max_tokens != 1 && max_tokens != 2 && max_tokens != 4 && max_tokens != 8)
        throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, "the decode plan runs 1, 2, 4 or 8 tokens per step (max_tokens)");
    const int kM = max_tokens;
    if (n_ranks < 1 || n_ranks > kMaxRanks || rank < 0 || rank >= n_ranks)
        throw Error(G4Q_ERR_INVALID_ARGUMENT, "rank must be in [0, n_ranks) with 1 <= n_ranks <= 8");
    if (n > 60000) throw Error(G4Q_ERR_INVALID_ARGUMENT, "too many phases");
    const int dev = current_device();
    const int sms = device_sm_count();
    std::vector<PhaseDev> ph(n);
    std::vector<std::vector<char>> producers(n);   // which producer CTAs each phase's x window needs
    int kmax = 0;
    for (int i = 0; i < n; ++i) {
        const Weight* w = reinterpret_cast<const Weight*>(phases[i].weight);
        const std::string tag = "phase " + std::to_string(i) + ": ";
        if (!w || w->magic != kWeightMagic) throw Error(G4Q_ERR_INVALID_ARGUMENT, tag + "invalid weight");
        if (w->device != dev) throw Error(G4Q_ERR_INVALID_ARGUMENT, tag + "weight lives on another device");
        if (w->mlx) throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, tag + "the decode plan takes 4-bit group-64 weights");
        if (!w->fast_ok || !w->small_scales || w->subnormal_scales)
            throw Error(G4Q_ERR_UNSUPPORTED_CONFIG,
                        tag + "the decode plan needs every |scale| < 2^-1 and no subnormal (nonzero, < 2^-126) scale");
        if (w->N % 64 != 0) throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, tag + "rows must be a multiple of 64");
        const uint32_t fl = phases[i].flags;
        if (fl & ~(G4Q_QMM_RMS_SCALE | G4Q_QMM_OUT_F32 | G4Q_PHASE_ARGMAX | G4Q_PHASE_ALLREDUCE | G4Q_PHASE_GEGLU))
            throw Error(G4Q_ERR_INVALID_ARGUMENT, tag + "unknown flag bits");
        if ((fl & G4Q_PHASE_GEGLU) && (fl & (G4Q_PHASE_ARGMAX | G4Q_PHASE_ALLREDUCE | G4Q_QMM_OUT_F32)))
            throw Error(G4Q_ERR_INVALID_ARGUMENT, tag + "a GeGLU phase writes bf16 and is neither argmax nor allreduce");
        if ((fl & G4Q_PHASE_ARGMAX) && i != n - 1)
            throw Error(G4Q_ERR_INVALID_ARGUMENT, tag + "the argmax phase must be the last phase");
        if ((fl & G4Q_PHASE_ARGMAX) && (fl & G4Q_PHASE_ALLREDUCE))
            throw Error(G4Q_ERR_INVALID_ARGUMENT, tag + "the argmax phase cannot be an allreduce phase");
        if ((fl & G4Q_PHASE_ALLREDUCE) && (fl & G4Q_QMM_RMS_SCALE))
            throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, tag + "an allreduce phase takes no RMS scale");
        if (!(fl & G4Q_PHASE_ARGMAX) && !phases[i].y) throw Error(G4Q_ERR_INVALID_ARGUMENT, tag + "needs an output");
        if (!phases[i].x || (reinterpret_cast<uintptr_t>(phases[i].x) & 15u))
            throw Error(G4Q_ERR_INVALID_ARGUMENT, tag + "x must be 16-byte aligned");
        PhaseDev& d = ph[i];
        d.packed = w->packed;
        d.sb = w->sb;
        d.x = phases[i].x;
        d.y = phases[i].y;
        d.N = (int)w->N;
        d.K = (int)w->K;
        d.R = (int)(w->N / 16);
        d.G = (int)(w->K / 64);
        d.Q = d.R / 4;
        d.U = d.Q * d.G;
        d.flags = fl;
        d.src = -1;
        d.src_col = 0;
        d.ldx = phases[i].ldx;
        d.ldy = phases[i].ldy;
        d.xwin = 0;
        d.xslots = d.G;
        d.nout = (fl & G4Q_PHASE_GEGLU) ? d.N / 2 : d.N;
        if (kM > 1 && (d.ldx < d.K || d.ldx % 8 != 0 || (!(fl & G4Q_PHASE_ARGMAX) && d.ldy < d.nout)))
            throw Error(G4Q_ERR_INVALID_ARGUMENT, tag + "ldx >= K (a multiple of 8) and ldy >= the outputs are required");
        d.post_w = d.norm_w = d.scalar = nullptr;
        d.res_user = nullptr;
        d.ld_res_user = 0;
        d.res_mode = 0;
        d.res_in = d.res_out = 0;
        d.peps = 1e-6f;
        if (prologues != nullptr) {
            const G4qPhasePrologue& pr = prologues[i];
            if (pr.residual < 0 || pr.residual > 2) throw Error(G4Q_ERR_INVALID_ARGUMENT, tag + "residual must be 0, 1 or 2");
            if (pr.layer_scalar && pr.residual != 2)
                throw Error(G4Q_ERR_INVALID_ARGUMENT, tag + "a layer scalar scales a residual add (residual = 2)");
            if (pr.residual_out && (pr.residual == 0 || pr.ld_residual_out < d.K))
                throw Error(G4Q_ERR_INVALID_ARGUMENT, tag + "residual_out needs a residual op and ld >= K");
            if (!(pr.eps >= 0.0f) || !std::isfinite(pr.eps)) throw Error(G4Q_ERR_INVALID_ARGUMENT, tag + "eps");
            for (const void* q : {(const void*)pr.post_norm_weight, (const void*)pr.norm_weight})
                if (q && (reinterpret_cast<uintptr_t>(q) & 3u))
                    throw Error(G4Q_ERR_INVALID_ARGUMENT, tag + "norm weights must be 4-byte aligned");
            d.post_w = pr.post_norm_weight;
            d.norm_w = pr.norm_weight;
            d.scalar = pr.layer_scalar;
            d.res_user = pr.residual_out;
            d.ld_res_user = pr.ld_residual_out;
            d.res_mode = pr.residual;
            d.peps = pr.eps;
            if ((d.post_w || d.norm_w || d.res_mode) && (fl & G4Q_QMM_RMS_SCALE))
                throw Error(G4Q_ERR_INVALID_ARGUMENT, tag + "a phase with a prologue takes no RMS scale");
            if (d.post_w || d.norm_w || d.res_mode) d.flags |= kFlagPrologue;
        }
        d.src_ranks = (fl & G4Q_PHASE_ALLREDUCE) ? n_ranks : 1;
        d.ar = -1;
        d.sync_before = 0;
        d.need_done = (fl & G4Q_PHASE_ARGMAX) ? 1 : 0;
        d.xout = 0;
        if (d.U < sms) throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, tag + "too small for a full-grid decode plan");
        if (d.G > kMaxXQuads) throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, tag + "K above 16384");
        if ((uint64_t)(d.U + 1) * (uint64_t)sms >= (1ull << 32) || (uint64_t)w->N * (uint64_t)w->K / 2 >= (1ull << 32))
            throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, tag + "too many units for 32-bit partition arithmetic");
        // a CTA range (at most ceil(U/C) units) touches at most (ceil(U/C) + G - 2) / G + 1 quads
        if ((d.U + sms - 1) / sms + d.G - 2 >= (kMaxCtaQuads - 1) * d.G)
            throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, tag + "too many quads per CTA range");
        // the most CTA ranges one quad meets, from the partition itself
        int ks = 1;
        for (int q = 0; q < d.Q; ++q) {
            const int64_t cf = ((int64_t)q * d.G + 1) * sms - 1, cl = ((int64_t)(q + 1) * d.G) * sms - 1;
            ks = std::max<int>(ks, (int)(cl / d.U - cf / d.U + 1));
        }
        if (ks > kSlots) throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, tag + "split too finely");
        d.ks = ks;
        // x inside the previous phase's (bf16) output row: consume it from the slots (dataflow)
        if (i > 0 && !(ph[i - 1].flags & (G4Q_PHASE_ARGMAX | G4Q_QMM_OUT_F32))) {
            const uint16_t* y0 = static_cast<const uint16_t*>(ph[i - 1].y);
            if (phases[i].x >= y0 && phases[i].x < y0 + ph[i - 1].nout) {
                const int64_t col = phases[i].x - y0;
                if (col % 64 != 0 || col + d.K > ph[i - 1].nout)
                    throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, tag + "x must be a 64-aligned column window of phase " +
                                                                std::to_string(i - 1) + "'s output");
                d.src = i - 1;
                d.src_col = (int)col;
            }
        }
        // producer CTAs this phase's x depends on (all of them for an external or older input)
        producers[i].assign(sms, d.src < 0 ? 1 : 0);
        if (d.src >= 0) {
            const PhaseDev& S = ph[d.src];
            const int per_q = (S.flags & G4Q_PHASE_GEGLU) ? 32 : 64;   // outputs per producer quad
            const int qa = d.src_col / per_q, qb = (d.src_col + d.K) / per_q;
            const int64_t cf = (((int64_t)qa * S.G + 1) * sms - 1) / S.U, cl = (((int64_t)qb * S.G) * sms - 1) / S.U;
            for (int64_t c = cf; c <= cl && c < sms; ++c) producers[i][c] = 1;
        }
        if (d.K > kmax) kmax = d.K;
    }
    // Staging of x per token: all K when the tokens' x fits beside the rings and the partial-sum
    // buffers; otherwise (M = 4 on a long K without an RMS scale, e.g. down_proj) each CTA stages only
    // the groups of its own range, which is then shorter than a quad row.
    bool pro = false;
    for (int i = 0; i < n; ++i) pro |= (ph[i].flags & (kFlagPrologue | G4Q_PHASE_GEGLU)) != 0;
    const void* kfn = decode_kernel_for(n_ranks > 1, kM, false, pro);
    const size_t red_bytes = (size_t)2 * warps_for(kM) * kM * 64 * 4;
    const size_t fixed = ring_bytes_for(kM) + red_bytes + 16;
    const size_t smem_max = max_dynamic_smem(kfn);
    if (fixed >= smem_max) throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, "decode plan: shared memory");
    const size_t x_budget = smem_max - fixed;
    int max_slots = 1;
    for (int i = 0; i < n; ++i) {
        PhaseDev& d = ph[i];
        const std::string tag = "phase " + std::to_string(i) + ": ";
        if ((size_t)kM * d.G * 128 > x_budget) {
            const int nmax = (d.U + sms - 1) / sms;
            if ((d.flags & G4Q_QMM_RMS_SCALE) || nmax >= d.G || (size_t)kM * nmax * 128 > x_budget)
                throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, tag + "the tokens' x does not fit in shared memory");
            d.xwin = 1;
            d.xslots = nmax;
        }
        // staging from the exchange buffer: sixteen 16-byte loads per slot and token, at most
        // kMaxStageLoads per thread in one pass (a limit only with the 12 warps of M = 8)
        if (d.src >= 0 && d.xslots * 16 > kMaxStageLoads * warps_for(kM) * 32)
            throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, tag + "x too wide to stage at this token count");
        max_slots = std::max(max_slots, d.xslots);
    }
    // Prologues: the staged x must be the whole input (phase 0's external x, or all of the previous
    // phase's output, staged by every CTA whole), which also makes the residual stream's double
    // buffer safe: when CTA 0 writes update k + 1, every CTA has finished the phase of update k.
    int res_cur = -1, res_k = 0;
    for (int i = 0; i < n; ++i) {
        PhaseDev& d = ph[i];
        const bool pro = d.post_w || d.norm_w || d.res_mode;
        if (!pro) continue;
        const std::string tag = "phase " + std::to_string(i) + ": ";
        if (d.xwin) throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, tag + "a prologue needs all of x staged");
        if (i > 0 && d.src != i - 1)
            throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, tag + "a prologue phase reads the previous phase's output");
        if (i > 0) {
            const PhaseDev& S = ph[i - 1];
            if (d.src_col != 0 || d.K != S.nout)
                throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, tag + "a prologue phase reads all of the previous phase's output");
        }
        if (d.res_mode != 0) {
            if (res_k != 0 && res_k != d.K)
                throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, tag + "the residual stream keeps one width");
            res_k = d.K;
            if (d.res_mode == 2 && res_cur < 0)
                throw Error(G4Q_ERR_INVALID_ARGUMENT, tag + "residual = 2 needs an earlier phase with a residual op");
            d.res_in = res_cur < 0 ? 0 : res_cur;
            d.res_out = res_cur < 0 ? 0 : 1 - res_cur;
            res_cur = d.res_out;
        }
    }
    // Dataflow: a phase that reads the previous phase's output polls that phase's exchange words (its
    // finished, tagged bf16 values) and needs no barrier. A phase whose x is anything else (an external
    // input or an older output) waits for every CTA of this rank to finish the previous phase first.
    // A phase "reads all" of its predecessor when its x window covers every producer CTA's quads and
    // every CTA stages all of it (no per-CTA windows).
    auto full = [&](int i) {
        if (ph[i].xwin) return false;
        for (int c = 0; c < sms; ++c)
            if (!producers[i][c]) return false;
        return true;
    };
    int n_ar = 0;
    for (int i = 0; i < n; ++i)
        if (ph[i].src_ranks > 1) ph[i].ar = n_ar++;
    for (int i = 1; i < n; ++i) {
        if (ph[i].src >= 0)
            ph[i - 1].xout = 1;
        else
            ph[i].sync_before = 1;
    }
    // Buffer rotation: phase i's slots and exchange words (buffer i mod 3) are read during phase i (by
    // finishers) and while phase i+1 stages x; phase i+3 writes the same buffer. A CTA can only stage
    // x of a phase j that reads ALL of phase j-1's output after every CTA has finished its share of
    // phase j-1 (every CTA owns units in every phase), and so after every CTA has staged phase j-1.
    // So the buffer is free once such a phase j <= i+3 (with j >= i+2) has been staged, or a barrier
    // sits at i+2 or i+3; otherwise a barrier is placed at phase i+3.
    for (int i = 0; i + 3 < n; ++i) {
        bool safe = false;
        for (int j = i + 2; j <= i + 3; ++j)
            safe |= ph[j].sync_before || (ph[j].src == j - 1 && full(j));
        if (!safe) ph[i + 3].sync_before = 1;
    }
    // Across ranks there is no barrier at all: a rank can only run ahead into the next phase that
    // reads an allreduce phase's output, which needs every rank's partials. So every allreduce phase
    // must feed the phase after it whole, and the step ends with the key exchange.
    if (n_ranks > 1)
        for (int i = 0; i < n; ++i)
            if ((ph[i].flags & G4Q_PHASE_ALLREDUCE) && (i + 1 >= n || ph[i + 1].src != i || !full(i + 1)))
                throw Error(G4Q_ERR_UNSUPPORTED_CONFIG,
                            "phase " + std::to_string(i) + ": the next phase must read all of an allreduce output");
    for (int i = 1; i < n; ++i)
        if (ph[i].sync_before) ph[i - 1].need_done = 1;
    ph[n - 1].need_done = 1;   // the argmax publish (or the plan's end) counts the last phase
    int64_t buf_words = 64, xbuf_tok = 32, rp_words = 64;
    for (int i = 0; i < n; ++i) {
        buf_words = std::max<int64_t>(buf_words, (int64_t)ph[i].Q * ph[i].ks * kM * 64);
        if (ph[i].xout) xbuf_tok = std::max<int64_t>(xbuf_tok, (int64_t)ph[i].nout / 2);
        if (ph[i].src_ranks > 1)
            rp_words = std::max<int64_t>(rp_words, (int64_t)ph[i].Q * n_ranks * ph[i].ks * kM * 64);
    }
    const int64_t xbuf_words = xbuf_tok * kM;
    if ((int64_t)kBufs * std::max(buf_words, rp_words) >= (1ll << 31))
        throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, "decode plan: slot buffers above 2^31 words");
    auto* plan = new DecodePlan();
    plan->device = dev;
    plan->n_phases = n;
    plan->grid = sms;
    plan->rank = rank;
    plan->n_ranks = n_ranks;
    plan->buf_words = buf_words;
    plan->rp_words = rp_words;
    plan->xbuf_words = xbuf_words;
    plan->xbuf_tok = xbuf_tok;
    plan->tokens = kM;
    plan->pro = pro;
    plan->res_ld = std::max(res_k, 8);
    plan->smem = fixed + (size_t)kM * max_slots * 128;
    // the residual stream in every CTA's shared memory, after the x region, when it fits: its phases
    // carry res_out = -1 and the stream's word offset from x in res_in
    if (res_k > 0 && plan->smem + (size_t)kM * plan->res_ld * 2 <= smem_max) {
        for (int i = 0; i < n; ++i)
            if (ph[i].res_mode != 0) {
                ph[i].res_out = -1;
                ph[i].res_in = (int)(kM * max_slots * 32);
            }
        plan->smem += (size_t)kM * plan->res_ld * 2;
    }
    const void* kfn_trace = decode_kernel_for(n_ranks > 1, 1, true, pro);
    if (plan->smem > smem_max) {
        delete plan;
        throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, "decode plan: K too large for shared memory");
    }
    const size_t slot_bytes = sizeof(unsigned long long) * kBufs * (size_t)buf_words;
    cudaError_t e = cudaMalloc(&plan->d_ph, sizeof(PhaseDev) * n);
    if (e == cudaSuccess) e = cudaMalloc(&plan->d_done, sizeof(unsigned int) * (n + 2));
    if (e == cudaSuccess) e = cudaMalloc(&plan->d_key, sizeof(unsigned long long) * kMaxPlanTokens);
    if (e == cudaSuccess) e = cudaMalloc(&plan->d_slots, slot_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&plan->d_rp, sizeof(unsigned long long) * kBufs * (size_t)rp_words);
    if (e == cudaSuccess) e = cudaMemset(plan->d_rp, 0, sizeof(unsigned long long) * kBufs * (size_t)rp_words);
    if (e == cudaSuccess) e = cudaMalloc(&plan->d_xkeys, sizeof(unsigned long long) * kXKeyStride * kMaxRanks);
    if (e == cudaSuccess) e = cudaMalloc(&plan->d_xbuf, sizeof(unsigned long long) * kBufs * (size_t)xbuf_words);
    if (e == cudaSuccess) e = cudaMalloc(&plan->d_peers, sizeof(void*) * 2 * kMaxRanks);
    if (e == cudaSuccess) e = cudaMalloc(&plan->d_res, sizeof(uint16_t) * 2 * kM * (size_t)plan->res_ld);
    if (e == cudaSuccess) e = cudaMemcpy(plan->d_ph, ph.data(), sizeof(PhaseDev) * n, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(plan->d_done, 0, sizeof(unsigned int) * (n + 2));
    if (e == cudaSuccess) e = cudaMemset(plan->d_key, 0, sizeof(unsigned long long) * kMaxPlanTokens);
    if (e == cudaSuccess) e = cudaMemset(plan->d_slots, 0, slot_bytes);
    if (e == cudaSuccess) e = cudaMemset(plan->d_xkeys, 0, sizeof(unsigned long long) * kXKeyStride * kMaxRanks);
    if (e == cudaSuccess) e = cudaMemset(plan->d_xbuf, 0, sizeof(unsigned long long) * kBufs * (size_t)xbuf_words);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        free_plan_memory(plan);
        delete plan;
        check_cuda(e, "decode plan allocation");
    }
    plan->peer_rp[rank] = plan->d_rp;
    plan->peer_xkeys[rank] = plan->d_xkeys;
    upload_peers(plan);
    check_cuda(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)max_dynamic_smem(kfn)),
               "cudaFuncSetAttribute(decode)");
    check_cuda(cudaFuncSetAttribute(kfn_trace, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)max_dynamic_smem(kfn_trace)),
               "cudaFuncSetAttribute(decode, tracing)");
    int per_sm = 0;
    check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, warps_for(kM) * 32, plan->smem),
               "occupancy(decode)");
    if (per_sm < 1) throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, "decode kernel does not fit on an SM");
    plan->magic = kPlanMagic;
    return plan;
}

static DecodePlan* checked_plan(void* h) {
    auto* plan = static_cast<DecodePlan*>(h);
    if (!plan || plan->magic != kPlanMagic) throw Error(G4Q_ERR_INVALID_ARGUMENT, "invalid decode plan handle");
    return plan;
}

void decode_plan_buffers(void* h, void** slots, uint64_t* slot_bytes, void** xkeys, uint64_t* xkey_bytes) {
    DecodePlan* plan = checked_plan(h);
    if (slots) *slots = plan->d_rp;
    if (slot_bytes) *slot_bytes = sizeof(unsigned long long) * kBufs * (uint64_t)plan->rp_words;
    if (xkeys) *xkeys = plan->d_xkeys;
    if (xkey_bytes) *xkey_bytes = sizeof(unsigned long long) * kXKeyStride * kMaxRanks;
}

void decode_plan_set_peers(void* h, void* const* slots, void* const* xkeys) {
    DecodePlan* plan = checked_plan(h);
    if (!slots || !xkeys) throw Error(G4Q_ERR_INVALID_ARGUMENT, "peer pointer arrays must be non-null");
    for (int r = 0; r < plan->n_ranks; ++r) {
        if (r == plan->rank) continue;
        if (!slots[r] || !xkeys[r]) throw Error(G4Q_ERR_INVALID_ARGUMENT, "missing peer buffer of rank " + std::to_string(r));
        plan->peer_rp[r] = static_cast<unsigned long long*>(slots[r]);
        plan->peer_xkeys[r] = static_cast<unsigned long long*>(xkeys[r]);
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(plan->device);
    upload_peers(plan);
    cudaSetDevice(prev);
}

void decode_plan_free(void* h) {
    DecodePlan* plan = checked_plan(h);
    plan->magic = 0;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(plan->device);
    free_plan_memory(plan);
    cudaSetDevice(prev);
    delete plan;
}

void decode_plan_run(void* h, int M, float eps, float softcap, int64_t row_offset, int32_t* tokens, float* values,
                     uint64_t* keys, uint16_t* logits, int64_t ld_logits, cudaStream_t st) {
    DecodePlan* plan = checked_plan(h);
    if (plan->device != current_device()) throw Error(G4Q_ERR_INVALID_ARGUMENT, "plan belongs to another device");
    if (M != plan->tokens)
        throw Error(G4Q_ERR_INVALID_ARGUMENT, "the plan was made for " + std::to_string(plan->tokens) +
                                                  " tokens per step (M = max_tokens)");
    if (logits != nullptr && M > 1 && ld_logits < 1)
        throw Error(G4Q_ERR_INVALID_ARGUMENT, "ld_logits must be the logits' row stride");
    if (plan->trace != nullptr && M != 1)
        throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, "the tracing build runs one token per step");
    for (int r = 0; r < plan->n_ranks; ++r)
        if (!plan->peer_rp[r] || !plan->peer_xkeys[r])
            throw Error(G4Q_ERR_INVALID_ARGUMENT, "tensor-parallel plan: peer buffers not set");
    DecodeArgs a{};
    a.ph = plan->d_ph;
    a.n_phases = plan->n_phases;
    a.eps = eps;
    a.softcap = softcap;
    a.row_offset = row_offset;
    a.done = plan->d_done;
    a.exit_count = plan->d_done + plan->n_phases;
    a.run = plan->d_done + plan->n_phases + 1;
    a.key = plan->d_key;
    a.slots = plan->d_slots;
    a.rp = plan->d_rp;
    a.rp_words = plan->rp_words;
    a.peer_rp = plan->d_peers;
    a.peer_xkeys = plan->d_peers + kMaxRanks;
    a.rank = plan->rank;
    a.n_ranks = plan->n_ranks;
    a.buf_words = plan->buf_words;
    a.xbuf = plan->d_xbuf;
    a.xbuf_words = plan->xbuf_words;
    a.xbuf_tok = plan->xbuf_tok;
    a.ld_logits = ld_logits;
    a.resbuf = plan->d_res;
    a.res_ld = plan->res_ld;
    a.gk_cubic = bf16_round_host(0.044715f);
    a.gk_tanh = bf16_round_host(0.7978845608028654f);
    a.tokens = tokens;
    a.values = values;
    a.keys_out = reinterpret_cast<unsigned long long*>(keys);
    a.logits = logits;
    a.err = device_scratch().err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan->grid);
    cfg.blockDim = dim3(warps_for(plan->tokens) * 32);
    cfg.dynamicSmemBytes = plan->smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;   // every CTA resident: CTAs wait on each other's data
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    a.trace = plan->trace;
    void* args[] = {&a};
    check_cuda(cudaLaunchKernelExC(&cfg, decode_kernel_for(plan->n_ranks > 1, plan->tokens, plan->trace != nullptr, plan->pro),
                                   args),
               "cudaLaunchKernelEx(decode)");
}

int64_t decode_plan_trace_words(void* h) {
    DecodePlan* plan = checked_plan(h);
    return (int64_t)plan->grid * plan->n_phases * kTraceWords;
}

void decode_plan_set_trace(void* h, uint64_t* buffer, int64_t words) {
    DecodePlan* plan = checked_plan(h);
    if (buffer != nullptr && plan->tokens != 1)
        throw Error(G4Q_ERR_UNSUPPORTED_CONFIG, "the tracing build runs plans of one token per step");
    if (buffer != nullptr && words < decode_plan_trace_words(h))
        throw Error(G4Q_ERR_INVALID_ARGUMENT, "trace buffer needs " + std::to_string(decode_plan_trace_words(h)) +
                                                  " 64-bit words");
    plan->trace = reinterpret_cast<unsigned long long*>(buffer);
}

}  // namespace g4q
