/*
 * g4q_oracle.c -- CPU restatement of MLX's affine quantized format for the Helios
 * quantized-linear hot path. TEST INFRASTRUCTURE ONLY (see g4q_oracle.h for the
 * reference call sites restated here and the parity status).
 *
 * Build: oracle/Makefile (-O3 -fopenmp -ffp-contract=off). -ffp-contract=off matters:
 * the synthetic generator and the tanh below must evaluate each fp32 operation with its
 * own rounding so that the CUDA twin (which uses __fmul_rn/__fadd_rn) matches bit for bit.
 */
#include "g4q_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- bf16 helpers -- */
static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float g4o_bf16_to_f32(uint16_t h) { return bits_f32((uint32_t)h << 16); }

uint16_t g4o_f32_to_bf16(float f) {
    uint32_t u = f32_bits(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);  /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* Round the exact real value v + err to bf16 (nearest, ties to even), where
 * v = RN_double(v + err) and err is the exact remainder (TwoSum). Handles normal,
 * subnormal and overflowing results. */
static uint16_t round_bf16_exact(double v, double err) {
    if (isnan(v)) return 0x7fc0;
    if (isinf(v)) return v > 0 ? 0x7f80 : 0xff80;
    if (v == 0.0) return signbit(v) ? 0x8000 : 0x0000;
    const int neg = v < 0.0;
    const double a = neg ? -v : v;
    const double e = neg ? -err : err;
    int ex;
    (void)frexp(a, &ex);                 /* a = m * 2^ex, m in [0.5, 1) */
    int qexp = ex - 8;                   /* bf16 keeps 8 significant bits */
    if (qexp < -133) qexp = -133;        /* subnormal quantum 2^-133 */
    const double t = ldexp(a, -qexp);    /* exact */
    double n = floor(t);
    const double frac = t - n;           /* exact */
    if (frac > 0.5 || (frac == 0.5 && (e > 0.0 || (e == 0.0 && fmod(n, 2.0) != 0.0)))) n += 1.0;
    const double r = ldexp(n, qexp);
    uint16_t h;
    if (r >= 0x1p128) h = 0x7f80;
    else h = (uint16_t)(f32_bits((float)r) >> 16);   /* exact: r has <= 9 bits */
    return (uint16_t)(h | (neg ? 0x8000u : 0u));
}

static inline void two_sum(double a, double b, double* s, double* err) {
    const double sum = a + b;
    const double bb = sum - a;
    *err = (a - (sum - bb)) + (b - bb);
    *s = sum;
}

/* ---------------------------------------------------------------- generator -- */
uint64_t g4o_rand(uint64_t seed, uint64_t index) {
    uint64_t z = seed + (index + 1u) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t g4o_matrix_seed(int layer, int proj) {
    return 0x48454C494F53ull ^ (uint64_t)(layer * 16 + proj);
}

uint64_t g4o_activation_seed(int chunk) {
    return 0x48454C494F53ull ^ 0xF00ull ^ (uint64_t)chunk;
}

/* Irwin-Hall(12) normal: twelve 16-bit uniforms summed exactly in integers, centred and
 * scaled by 2^-16 (exact in fp32). Mean ~0, variance ~1, support (-6, 6). */
static inline float normal_at(uint64_t seed, uint64_t i) {
    int64_t sum = 0;
    for (int j = 0; j < 3; ++j) {
        const uint64_t r = g4o_rand(seed, 3u * i + (uint64_t)j);
        sum += (int64_t)(r & 0xffffu) + (int64_t)((r >> 16) & 0xffffu) +
               (int64_t)((r >> 32) & 0xffffu) + (int64_t)(r >> 48);
    }
    return (float)(sum - 393216) * (1.0f / 65536.0f);
}

void g4o_synth_normal_bf16(uint64_t seed, int64_t count, uint16_t* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < count; ++i) out[i] = g4o_f32_to_bf16(normal_at(seed, (uint64_t)i));
}

void g4o_synth_matrix(uint64_t seed, int64_t N, int64_t K, int bits, int group_size,
                      uint32_t* w, uint16_t* scales, uint16_t* biases) {
    const uint64_t seed_w = g4o_rand(seed, 1), seed_s = g4o_rand(seed, 2), seed_b = g4o_rand(seed, 3);
    const int64_t words = N * K * bits / 32;
    const int64_t groups = N * (K / group_size);
    if (w) {
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < words; ++i) w[i] = (uint32_t)(g4o_rand(seed_w, (uint64_t)i) >> 32);
    }
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < groups; ++i) {
        /* scale = bf16(0.002 + u * 0.018), u uniform on [0,1) with 24 bits */
        const float u = (float)(g4o_rand(seed_s, (uint64_t)i) >> 40) * 5.9604644775390625e-8f;
        const float prod = u * 0.018f;
        const float sv = 0.002f + prod;
        const uint16_t s = g4o_f32_to_bf16(sv);
        if (scales) scales[i] = s;
        if (biases) {
            /* bias = bf16(-8 * scale + 1e-3 * z), z ~ N(0, 1) */
            const float t1 = -8.0f * g4o_bf16_to_f32(s);
            const float t2 = 1e-3f * normal_at(seed_b, (uint64_t)i);
            biases[i] = g4o_f32_to_bf16(t1 + t2);
        }
    }
}

/* ---------------------------------------------------------------- the format -- */
uint16_t g4o_deq1(uint16_t scale, uint32_t q, uint16_t bias, int chain) {
    const double s = (double)g4o_bf16_to_f32(scale);
    const double b = (double)g4o_bf16_to_f32(bias);
    const double p = s * (double)q;                      /* exact: <= 8 + 8 bits */
    double sum, err;
    if (chain == G4O_CHAIN_R1) {
        two_sum(p, b, &sum, &err);
        return round_bf16_exact(sum, err);
    }
    const double p1 = (double)g4o_bf16_to_f32(round_bf16_exact(p, 0.0));
    two_sum(p1, b, &sum, &err);
    return round_bf16_exact(sum, err);
}

static int check_format(int64_t N, int64_t K, int bits, int group_size, int chain) {
    if (N < 0 || K <= 0) return G4O_ERR_ARG;
    if (bits != 4 && bits != 8) return G4O_ERR_ARG;
    if (group_size != 64 && group_size != 32 && group_size != 128) return G4O_ERR_ARG;
    if (K % group_size != 0) return G4O_ERR_ARG;
    if (chain != G4O_CHAIN_R1 && chain != G4O_CHAIN_R2) return G4O_ERR_ARG;
    return G4O_OK;
}

static inline uint32_t q_at(const uint32_t* wrow, int64_t k, int bits) {
    const int per = 32 / bits;
    return (wrow[k / per] >> (bits * (int)(k % per))) & ((1u << bits) - 1u);
}

/* One row of deq(W) as bf16 bits, through a per-group table of all q values. */
static void dequant_row(const uint32_t* wrow, const uint16_t* srow, const uint16_t* brow,
                        int64_t K, int bits, int group_size, int chain, uint16_t* out) {
    uint16_t lut[256];
    const int nq = 1 << bits;
    for (int64_t g = 0; g < K / group_size; ++g) {
        for (int q = 0; q < nq; ++q) lut[q] = g4o_deq1(srow[g], (uint32_t)q, brow[g], chain);
        for (int64_t k = g * group_size; k < (g + 1) * group_size; ++k) out[k] = lut[q_at(wrow, k, bits)];
    }
}

int g4o_dequantize(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                   int64_t N, int64_t K, int bits, int group_size, int chain, uint16_t* out) {
    if (check_format(N, K, bits, group_size, chain) != G4O_OK) return G4O_ERR_ARG;
    const int64_t wpr = K * bits / 32, G = K / group_size;
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n)
        dequant_row(w + n * wpr, scales + n * G, biases + n * G, K, bits, group_size, chain, out + n * K);
    return G4O_OK;
}

int g4o_dequantize_rows(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                        int64_t N, int64_t K, int bits, int group_size, int chain,
                        const int32_t* ids, int64_t T, uint16_t* out) {
    if (check_format(N, K, bits, group_size, chain) != G4O_OK || T < 0) return G4O_ERR_ARG;
    for (int64_t t = 0; t < T; ++t)
        if (ids[t] < 0 || ids[t] >= N) return G4O_ERR_ARG;
    const int64_t wpr = K * bits / 32, G = K / group_size;
    for (int64_t t = 0; t < T; ++t) {
        const int64_t n = ids[t];
        dequant_row(w + n * wpr, scales + n * G, biases + n * G, K, bits, group_size, chain, out + t * K);
    }
    return G4O_OK;
}

int g4o_qmm(const uint16_t* x, int64_t M, const uint32_t* w, const uint16_t* scales,
            const uint16_t* biases, int64_t N, int64_t K, int bits, int group_size, int chain,
            const float* row_scale, double* y_exact, uint16_t* y_bf16) {
    if (check_format(N, K, bits, group_size, chain) != G4O_OK || M < 0) return G4O_ERR_ARG;
    const int64_t wpr = K * bits / 32, G = K / group_size;
    double* xd = (double*)malloc(sizeof(double) * (size_t)(M * K + 1));
    if (!xd) return G4O_ERR_ARG;
    for (int64_t i = 0; i < M * K; ++i) xd[i] = (double)g4o_bf16_to_f32(x[i]);
#pragma omp parallel
    {
        uint16_t* row = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)K);
        double* rowd = (double*)malloc(sizeof(double) * (size_t)K);
#pragma omp for schedule(static)
        for (int64_t n = 0; n < N; ++n) {
            dequant_row(w + n * wpr, scales + n * G, biases + n * G, K, bits, group_size, chain, row);
            for (int64_t k = 0; k < K; ++k) rowd[k] = (double)g4o_bf16_to_f32(row[k]);
            for (int64_t m = 0; m < M; ++m) {
                const double* xr = xd + m * K;
                double acc = 0.0;
                for (int64_t k = 0; k < K; ++k) acc += xr[k] * rowd[k];
                if (row_scale) acc *= (double)row_scale[m];
                if (y_exact) y_exact[m * N + n] = acc;
                if (y_bf16) y_bf16[m * N + n] = round_bf16_exact(acc, 0.0);
            }
        }
        free(row);
        free(rowd);
    }
    free(xd);
    return G4O_OK;
}

/* Threads of the OpenMP loops below (the checker's own setting; a launcher such as torchrun may
 * have set OMP_NUM_THREADS=1 for the process). n <= 0 keeps the runtime's default. */
void g4o_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int g4o_qmm_f32(const uint16_t* x, int64_t M, const uint32_t* w, const uint16_t* scales,
                const uint16_t* biases, int64_t N, int64_t K, int group_size, int chain,
                int threads, uint16_t* y_bf16) {
    if (check_format(N, K, 4, group_size, chain) != G4O_OK || M < 0) return G4O_ERR_ARG;
    const int64_t wpr = K / 8, G = K / group_size;
    float* xf = (float*)malloc(sizeof(float) * (size_t)(M * K + 1));
    if (!xf) return G4O_ERR_ARG;
    for (int64_t i = 0; i < M * K; ++i) xf[i] = g4o_bf16_to_f32(x[i]);
#ifdef _OPENMP
    const int nt = threads > 0 ? threads : omp_get_max_threads();
#else
    const int nt = 1;
    (void)threads;
#endif
#pragma omp parallel num_threads(nt)
    {
        float* wf = (float*)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(static)
        for (int64_t n = 0; n < N; ++n) {
            const uint32_t* wr = w + n * wpr;
            for (int64_t g = 0; g < G; ++g) {
                float lut[16];
                if (chain == G4O_CHAIN_R2) {
                    /* R2 in fp32: s*q is exact in fp32 (<= 12 significant bits); the fp32 sum of two
                     * bf16 values rounds to the same bf16 as the exact sum, so this table equals
                     * g4o_deq1(..., R2) bit for bit (checked by the tests) at a fraction of the cost. */
                    const float s = g4o_bf16_to_f32(scales[n * G + g]), b = g4o_bf16_to_f32(biases[n * G + g]);
                    for (int q = 0; q < 16; ++q) {
                        const float p = g4o_bf16_to_f32(g4o_f32_to_bf16(s * (float)q));
                        lut[q] = g4o_bf16_to_f32(g4o_f32_to_bf16(p + b));
                    }
                } else {
                    for (int q = 0; q < 16; ++q)
                        lut[q] = g4o_bf16_to_f32(g4o_deq1(scales[n * G + g], (uint32_t)q, biases[n * G + g], chain));
                }
                for (int64_t k = g * group_size; k < (g + 1) * group_size; k += 8) {
                    const uint32_t word = wr[k / 8];
                    for (int j = 0; j < 8; ++j) wf[k + j] = lut[(word >> (4 * j)) & 15u];
                }
            }
            for (int64_t m = 0; m < M; ++m) {
                const float* xr = xf + m * K;
                float acc[16] = {0};
                for (int64_t k = 0; k < K; k += 16)
                    for (int j = 0; j < 16; ++j) acc[j] = fmaf(xr[k + j], wf[k + j], acc[j]);
                float s = 0.0f;
                for (int j = 0; j < 16; ++j) s += acc[j];
                y_bf16[m * N + n] = g4o_f32_to_bf16(s);
            }
        }
        free(wf);
    }
    free(xf);
    return G4O_OK;
}

float g4o_rms_scale(const uint16_t* x, int64_t K, float eps) {
    float ss = 0.0f;
    for (int64_t k = 0; k < K; ++k) {
        const float v = g4o_bf16_to_f32(x[k]);
        const float sq = v * v;
        ss = ss + sq;
    }
    const float mean = ss / (float)K;
    return 1.0f / sqrtf(mean + eps);
}

/* ---------------------------------------------------------------- softcap -- */
/* expm1 on [0, 18): y = k*ln2 + r with ln2 split into a 15-bit head (k*LN2_HI exact) and
 * a tail (Cody-Waite), expm1(r) by its Taylor series to r^9/9! (|r| <= ln2/2, truncation
 * < 1e-11), then 2^k * (1 + expm1(r)) - 1. */
static float expm1_pos(float y) {
    const float LN2_HI = 0.693145751953125f;
    const float LN2_LO = 1.42860677e-06f;
    const int k = (int)(y * 1.44269504f + 0.5f);
    const float kf = (float)k;
    const float t1 = kf * LN2_HI;
    const float t2 = y - t1;
    const float t3 = kf * LN2_LO;
    const float r = t2 - t3;
    float p = 2.75573192e-06f;           /* 1/9! */
    p = p * r; p = p + 2.48015873e-05f;  /* 1/8! */
    p = p * r; p = p + 1.98412698e-04f;  /* 1/7! */
    p = p * r; p = p + 1.38888889e-03f;  /* 1/6! */
    p = p * r; p = p + 8.33333333e-03f;  /* 1/5! */
    p = p * r; p = p + 4.16666667e-02f;  /* 1/4! */
    p = p * r; p = p + 1.66666667e-01f;  /* 1/3! */
    p = p * r; p = p + 0.5f;             /* 1/2! */
    p = p * r; p = p + 1.0f;
    p = p * r;                            /* expm1(r) */
    if (k == 0) return p;
    const float pow2 = bits_f32((uint32_t)(127 + k) << 23);
    const float e = p + 1.0f;
    const float scaled = e * pow2;
    return scaled - 1.0f;
}

float g4o_tanh(float x) {
    if (x != x) return x;
    const uint32_t u = f32_bits(x);
    const float a = bits_f32(u & 0x7fffffffu);
    float t;
    if (a >= 9.0f) {
        t = 1.0f;        /* 1 - tanh(a) < 3.1e-8 here: below half an fp32 ulp of 1 */
    } else if (a == 0.0f) {
        t = 0.0f;
    } else {
        const float y = a + a;
        const float e = expm1_pos(y);
        const float d = e + 2.0f;
        t = e / d;
    }
    return bits_f32(f32_bits(t) | (u & 0x80000000u));
}

uint16_t g4o_softcap(uint16_t logit, float cap) {
    const float l = g4o_bf16_to_f32(logit);
    const float d = l / cap;
    const float db = g4o_bf16_to_f32(g4o_f32_to_bf16(d));
    const float t = g4o_tanh(db);
    const float tb = g4o_bf16_to_f32(g4o_f32_to_bf16(t));
    const float r = tb * cap;
    return g4o_f32_to_bf16(r);
}

int g4o_softcap_argmax(const uint16_t* logits, int64_t V, float cap, int32_t* token, float* value) {
    if (V <= 0 || !logits) return G4O_ERR_ARG;
    float best = -INFINITY;
    int64_t arg = 0;
    for (int64_t i = 0; i < V; ++i) {
        const uint16_t h = cap > 0.0f ? g4o_softcap(logits[i], cap) : logits[i];
        const float v = g4o_bf16_to_f32(h);
        if (v > best) { best = v; arg = i; }
    }
    if (token) *token = (int32_t)arg;
    if (value) *value = best;
    return G4O_OK;
}

/* ---------------------------------------------------------------- layout v1 -- */
static inline void slot_coords(int lane, int j, int slot, int* dn, int* dk) {
    const int gi = lane >> 2, t = lane & 3;
    const int pair = slot & 3, hi = slot >> 2;      /* slot p -> pair p low half, p+4 high */
    *dn = gi + ((pair & 1) ? 8 : 0);
    *dk = 16 * j + 2 * t + hi + ((pair & 2) ? 8 : 0);
}

int g4o_repack(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
               int64_t N, int64_t K, uint32_t* packed, uint32_t* sb) {
    if (N % 16 != 0 || K % 64 != 0 || N <= 0) return G4O_ERR_ARG;
    const int64_t R = N / 16, G = K / 64, wpr = K / 8;
#pragma omp parallel for schedule(static)
    for (int64_t g = 0; g < G; ++g) {
        for (int64_t r = 0; r < R; ++r) {
            uint32_t* blk = packed + (g * R + r) * 128;
            for (int lane = 0; lane < 32; ++lane)
                for (int j = 0; j < 4; ++j) {
                    uint32_t word = 0;
                    for (int slot = 0; slot < 8; ++slot) {
                        int dn, dk;
                        slot_coords(lane, j, slot, &dn, &dk);
                        const int64_t n = 16 * r + dn, k = 64 * g + dk;
                        word |= q_at(w + n * wpr, k, 4) << (4 * slot);
                    }
                    blk[lane * 4 + j] = word;
                }
        }
        for (int64_t n = 0; n < N; ++n)
            sb[g * N + n] = (uint32_t)scales[n * G + g] | ((uint32_t)biases[n * G + g] << 16);
    }
    return G4O_OK;
}

int g4o_unpack(const uint32_t* packed, const uint32_t* sb, int64_t N, int64_t K,
               uint32_t* w, uint16_t* scales, uint16_t* biases) {
    if (N % 16 != 0 || K % 64 != 0 || N <= 0) return G4O_ERR_ARG;
    const int64_t R = N / 16, G = K / 64, wpr = K / 8;
    memset(w, 0, sizeof(uint32_t) * (size_t)(N * wpr));
    for (int64_t g = 0; g < G; ++g)
        for (int64_t r = 0; r < R; ++r) {
            const uint32_t* blk = packed + (g * R + r) * 128;
            for (int lane = 0; lane < 32; ++lane)
                for (int j = 0; j < 4; ++j)
                    for (int slot = 0; slot < 8; ++slot) {
                        int dn, dk;
                        slot_coords(lane, j, slot, &dn, &dk);
                        const int64_t n = 16 * r + dn, k = 64 * g + dk;
                        const uint32_t q = (blk[lane * 4 + j] >> (4 * slot)) & 15u;
                        w[n * wpr + k / 8] |= q << (4 * (k % 8));
                    }
        }
    for (int64_t g = 0; g < G; ++g)
        for (int64_t n = 0; n < N; ++n) {
            scales[n * G + g] = (uint16_t)(sb[g * N + n] & 0xffffu);
            biases[n * G + g] = (uint16_t)(sb[g * N + n] >> 16);
        }
    return G4O_OK;
}
