/*
 * g4q_oracle.h -- CPU restatement of the MLX affine quantized-linear format used by
 * Helios/gemma4d's native graph. TEST INFRASTRUCTURE ONLY: the product path
 * (libg4q.so) never links, loads or calls anything declared here. Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm use it, as the
 * checker or as the timed CPU stand-in for MLX's CPU quantized_matmul.
 *
 * What it restates (reference call sites, paths relative to the reference project):
 *   - quantized_linear(): mlx::core::quantized_matmul(x, W, scales, biases,
 *     transpose=true, group_size, bits, "affine") then cast to bf16
 *     (native/gemma4_mlx/src/native_model.cc:349-362, model_dtype at :335-340).
 *   - quantized_embedding(): take rows, then mlx::core::dequantize(..., "affine")
 *     (native/gemma4_mlx/src/native_model.cc:364-376).
 *   - target_logits_for_hidden(): tied LM head quantized_matmul, bf16 cast, then
 *     tanh(l / 30) * 30 in bf16 (native/gemma4_mlx/src/native_model.cc:1782-1795);
 *     callers take argmax with the first index winning ties
 *     (native/gemma4_mlx/src/native_model.cc:3825, 3934).
 *   - The packed shape rule K = cols * 32 / bits
 *     (native/gemma4_mlx/src/native_model.cc:281-287) and the per-module
 *     {bits in {4,8}, group_size 64} contract (native/gemma4_mlx/src/model_manifest.cc:146-152).
 *
 * The arithmetic itself lives in MLX 0.31.2 (third-party, pinned in the reference's
 * BENCHMARKS.md:682), which is not vendored in the reference and not installable here.
 * This file restates the published format: W is uint32 [N, K*bits/32], element k of a
 * row sits in word k/(32/bits) at bit offset bits*(k mod (32/bits)) (little-endian
 * nibbles/bytes); scales and biases are bf16 [N, K/group_size];
 * w = scale * q + bias.
 *
 * PARITY STATUS: unpinned against MLX itself (MLX is absent and the reference holds no
 * golden vectors for this path). The restatement is pinned instead to known-answer
 * vectors computed with exact rational arithmetic from the format definition
 * (tests/golden/make_golden.py) and cross-checked against an independent numpy
 * restatement (oracle/affine.py).
 *
 * The rounding chain of the bf16 "scale*q + bias" is a parameter because MLX's cannot
 * be observed here:
 *   G4O_CHAIN_R1: bf16_rn(scale*q + bias) with one rounding of the exact value;
 *   G4O_CHAIN_R2: bf16_rn(bf16_rn(scale*q) + bias), one rounding per bf16 operation
 *                 (a generic bf16 CPU path). R2 is the default.
 */
#ifndef G4Q_ORACLE_H
#define G4Q_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { G4O_CHAIN_R1 = 1, G4O_CHAIN_R2 = 2 };
enum { G4O_OK = 0, G4O_ERR_ARG = 1 };

/* ---- bf16 helpers ---------------------------------------------------------------- */
float g4o_bf16_to_f32(uint16_t h);
uint16_t g4o_f32_to_bf16(float f);                  /* round to nearest even */

/* ---- seeded synthetic data (counter-based splitmix64; identical on CPU and GPU) ---- */
uint64_t g4o_rand(uint64_t seed, uint64_t index);
uint64_t g4o_matrix_seed(int layer, int proj);      /* 0x48454C494F53 ^ (layer*16+proj) */
uint64_t g4o_activation_seed(int chunk);            /* 0x48454C494F53 ^ 0xF00 ^ chunk  */
void g4o_synth_matrix(uint64_t seed, int64_t N, int64_t K, int bits, int group_size,
                      uint32_t* w, uint16_t* scales, uint16_t* biases);
void g4o_synth_normal_bf16(uint64_t seed, int64_t count, uint16_t* out);

/* ---- the format ------------------------------------------------------------------ */
uint16_t g4o_deq1(uint16_t scale, uint32_t q, uint16_t bias, int chain);
int g4o_dequantize(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                   int64_t N, int64_t K, int bits, int group_size, int chain, uint16_t* out);
int g4o_dequantize_rows(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                        int64_t N, int64_t K, int bits, int group_size, int chain,
                        const int32_t* ids, int64_t T, uint16_t* out);

/* y[m,n] = row_scale[m] * sum_k x[m,k] * deq(W)[n,k], accumulated in double.
 * row_scale may be NULL (1.0). y_exact (may be NULL) gets the unrounded value,
 * y_bf16 (may be NULL) the bf16 round-to-nearest-even of it. OpenMP over n. */
int g4o_qmm(const uint16_t* x, int64_t M, const uint32_t* w, const uint16_t* scales,
            const uint16_t* biases, int64_t N, int64_t K, int bits, int group_size, int chain,
            const float* row_scale, double* y_exact, uint16_t* y_bf16);

/* CPU baseline: the same product with fp32 accumulation (vectorisable), bf16 out,
 * `threads` OpenMP threads (<=0: all). This is the timed stand-in for MLX's CPU path. */
void g4o_set_threads(int n);                     /* OpenMP threads of the oracle's loops */
int g4o_qmm_f32(const uint16_t* x, int64_t M, const uint32_t* w, const uint16_t* scales,
                const uint16_t* biases, int64_t N, int64_t K, int group_size, int chain,
                int threads, uint16_t* y_bf16);

/* 1/sqrt(mean(x^2) + eps) of one bf16 row, fp32, sequential sum. */
float g4o_rms_scale(const uint16_t* x, int64_t K, float eps);

/* tanh from IEEE +,-,*,/ only (Cody-Waite reduction + Taylor expm1), so the CUDA twin
 * in the product library returns the same fp32 bits. */
float g4o_tanh(float x);
/* bf16( bf16(tanh(bf16(l / cap))) * cap ), each step in fp32 then rounded. */
uint16_t g4o_softcap(uint16_t logit, float cap);
/* argmax over softcap(logits) (cap <= 0: no softcap); first index wins ties. */
int g4o_softcap_argmax(const uint16_t* logits, int64_t V, float cap,
                       int32_t* token, float* value);

/* ---- kernel layout v1 (what libg4q's upload produces) ------------------------------
 * packed: (K/64) x (N/16) blocks of 128 uint32; block (g, r) at word (g*(N/16)+r)*128;
 * lane l = 4*gi + t, word j (0..3) at l*4 + j covers k0 = 64*g + 16*j, rows
 * n0 = 16*r + gi and n1 = n0 + 8, nibble slots:
 *   0:(n0,k0+2t) 4:(n0,k0+2t+1) 1:(n1,k0+2t) 5:(n1,k0+2t+1)
 *   2:(n0,k0+2t+8) 6:(n0,k0+2t+9) 3:(n1,k0+2t+8) 7:(n1,k0+2t+9)
 * sb: (K/64) x N uint32, word (g, n) = scale_bits | bias_bits << 16.
 * Requires bits == 4, group_size == 64, N % 16 == 0, K % 64 == 0. */
int g4o_repack(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
               int64_t N, int64_t K, uint32_t* packed, uint32_t* sb);
int g4o_unpack(const uint32_t* packed, const uint32_t* sb, int64_t N, int64_t K,
               uint32_t* w, uint16_t* scales, uint16_t* biases);

#ifdef __cplusplus
}
#endif
#endif
