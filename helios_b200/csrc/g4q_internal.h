// g4q_internal.h -- host-side internals shared by the g4q translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "g4q.h"

namespace g4q {

constexpr uint64_t kWeightMagic = 0x4734515745494748ull;  // "G4QWEIGH"

struct Weight {
    uint64_t magic = 0;
    int64_t N = 0, K = 0;        // logical shape of this handle (after any TP split)
    int bits = 4, group_size = 64;
    int device = -1;
    uint32_t* packed = nullptr;  // layout v1 (4-bit, group 64) or, for other specs, MLX's layout
    uint32_t* sb = nullptr;
    bool mlx = false;            // kept in MLX's layout (bits 8, or groups 32 / 128): generic kernels
    uint16_t* mlx_scales = nullptr;   // [N][K/group] bf16 (MLX layout only)
    uint16_t* mlx_biases = nullptr;
    size_t bytes = 0;
    int* d_flags = nullptr;      // device word: bit0 = a scale outside |s| < 2^120 or non-finite,
                                 // bit1 = a gathered row id was out of range, bit2 = |s| >= 2^-1,
                                 // bit3 = a subnormal nonzero scale
    bool fast_ok = true;         // host copy of !(bit0), refreshed by every load
    bool small_scales = true;    // host copy of !(bit2): every |scale| < 2^-1
    bool subnormal_scales = false;   // host copy of bit3: some scale is subnormal (exponent 0, nonzero)
    // lazily created scratch for the LM-head argmax (keys[16] + counter), zeroed once
    unsigned long long* argmax_scratch = nullptr;
};

constexpr uint64_t kLoraMagic = 0x47345141524F4C47ull;    // "G4QLORAG"

// One LoRA adapter module (the reference's NativeLoraAdapter::Impl::Module, native_model.cc:66-73):
// lora_A kept as [rank][K] fp32, lora_B transposed to [rank][N] fp32, the scale already rounded to
// bf16 as model_scalar does, and a [max_tokens][rank] fp32 scratch for the low-rank activations.
struct Lora {
    uint64_t magic = 0;
    int64_t N = 0, K = 0;
    int rank = 0;
    int max_tokens = 0;
    float alpha = 0.f;
    float scale_bf16 = 0.f;     // float value of bf16(alpha / rank)
    int device = -1;
    float* a = nullptr;
    float* bt = nullptr;
    float* low = nullptr;
};

// kernels (g4q_lora.cu)
void launch_lora_transpose(const float* b, int64_t N, int rank, float* bt, cudaStream_t st);
void launch_lora_apply(const Lora& l, const uint16_t* x, int64_t M, int64_t ldx, uint16_t* y, int64_t ldy,
                       cudaStream_t st);

// round-to-nearest-even of a float to bf16, as a float (host side)
float bf16_round_host(float f);

// kernels (g4q_mlp.cu): the MLP's elementwise neighbours
void launch_geglu(const uint16_t* gate, int64_t ldg, const uint16_t* up, int64_t ldu, uint16_t* out, int64_t ldo,
                  int64_t M, int64_t I, cudaStream_t st);
void launch_rms_norm(const uint16_t* x, int64_t ldx, const uint16_t* w, int64_t M, int64_t K, float eps,
                     uint16_t* out, int64_t ldo, cudaStream_t st, const uint16_t* res = nullptr, int64_t ldr = 0,
                     const uint16_t* scale = nullptr);

// tensor-parallel allreduce over NVLink peer memory (g4q_comm.cu)
void* comm_create(int rank, int n_ranks, int64_t max_elems);
void comm_buffer(const void* h, void** buf, uint64_t* bytes);
void comm_set_peers(void* h, void* const* peer_bufs);
void comm_allreduce(void* h, void* data, int64_t count, int dtype, cudaStream_t st);
void comm_free(void* h);

// Raised inside entry points; converted to a status + last-error message at the C-ABI edge.
struct Error : std::runtime_error {
    G4qStatus status;
    Error(G4qStatus s, const std::string& m) : std::runtime_error(m), status(s) {}
};

inline void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();   // do not leave a non-sticky error behind for the next launch check
        throw Error(G4Q_ERR_RUNTIME, std::string(what) + ": " + cudaGetErrorString(e));
    }
}

int device_sm_count();
int current_device();
// Largest dynamic shared memory a kernel may opt in to, given its static shared memory.
size_t max_dynamic_smem(const void* kernel);

// Per-device library state, created by the first g4q_weight_create on that device (never
// inside a stream capture): a device error word written by bounded waits that gave up, and the
// per-row RMS scales of the prefill GEMM.
struct DeviceScratch {
    int* err = nullptr;
    float* rms = nullptr;
    int64_t rms_rows = 0;
    float* slots = nullptr;      // stream-K GEMV partial sums
    size_t slots_bytes = 0;
    int* counters = nullptr;     // stream-K GEMV per-quad arrival counters, zero between launches
    int64_t counters_n = 0;
};
DeviceScratch& device_scratch();
// the current device's scratch if a call has created it already, else nullptr (allocates nothing)
DeviceScratch* device_scratch_if_created();
// Grows the GEMV partial-sum slots to cover an N x K weight (called by g4q_weight_create).
void reserve_gemv_scratch(int64_t N, int64_t K);

// kernels (g4q_gemv2.cu): persistent stream-K GEMV for M <= 8
size_t gemv2_slots_bytes(int64_t N, int64_t K, int sms);

// kernels (g4q_layout.cu)
void launch_synth_matrix(uint64_t seed, int64_t N, int64_t K, int bits, int group_size, uint32_t* w,
                         uint16_t* s, uint16_t* b, cudaStream_t st);
void launch_synth_normal(uint64_t seed, int64_t count, uint16_t* out, cudaStream_t st);
void launch_repack(const uint32_t* src_w, const uint16_t* src_s, const uint16_t* src_b, int64_t src_ld_words,
                   int64_t src_ld_groups, int64_t src_row0, int64_t src_k0, int64_t n_rows, Weight& w,
                   int64_t dst_row0, cudaStream_t st);
void launch_export(const Weight& w, uint32_t* dst_w, uint16_t* dst_s, uint16_t* dst_b, cudaStream_t st);
void launch_sb_flags(const Weight& w, cudaStream_t st);
// kernels (g4q_generic.cu): weights kept in MLX's layout (specs other than 4-bit / group 64)
void launch_dequantize_mlx_rows(const Weight& w, const int32_t* ids, int64_t n_ids, uint16_t* out, int chain,
                                cudaStream_t st);
void launch_dequantize(const Weight& w, const int32_t* ids, int64_t n_ids, uint16_t* out, int chain,
                       int* d_err, cudaStream_t st);
void launch_dequantize_mlx(const uint32_t* w, const uint16_t* s, const uint16_t* b, int64_t N, int64_t K,
                           int bits, int group_size, int chain, uint16_t* out, cudaStream_t st);

// kernels (g4q_gemv.cu)
struct QmmCall {
    const Weight* w;
    const uint16_t* x;
    int64_t M, ldx;
    void* y;
    int64_t ldy;
    uint32_t flags;
    float eps;
    // fused RMSNorm prologue (stream-K GEMV only): x is replaced by bf16(norm_w * bf16(x * inv)),
    // inv = 1/sqrt(mean(x^2) + eps); the normalized rows also go to xn when it is non-null
    const uint16_t* norm_w = nullptr;
    uint16_t* xn = nullptr;
    int64_t ldxn = 0;
    // fused GeGLU epilogue (stream-K GEMV only): the weight's 64-row quads pair 32 gate rows with the
    // matching 32 up rows; y receives geglu(gate, up) = bf16 [M, N/2] with row stride ldy
    bool geglu = false;
};
void launch_qmm_mlx(const QmmCall& c, cudaStream_t st);

void launch_gemv(const QmmCall& c, cudaStream_t st);
bool gemv2_supported(const QmmCall& c);
void launch_gemv2(const QmmCall& c, cudaStream_t st);
void launch_lm_head_noalloc(const uint32_t* packed, const uint32_t* sb, int64_t N, int64_t K, const uint16_t* x,
                            int64_t M, int64_t ldx, float softcap, uint32_t flags, float eps, int64_t row_offset,
                            uint16_t* logits, int64_t ld_logits, int32_t* tokens, float* values,
                            unsigned long long* keys, cudaStream_t st);
// the allocation-free LM head's own error word (code 50: a scale outside the fast dequantisation's
// range); read, and optionally cleared, without allocating
int noalloc_error(bool reset);
void launch_lm_head(const Weight& w, const uint16_t* x, int64_t M, int64_t ldx, float softcap, uint32_t flags,
                    float eps, int64_t row_offset, uint16_t* logits, int64_t ld_logits, int32_t* tokens,
                    float* values, unsigned long long* keys, cudaStream_t st);

// kernels (g4q_decode.cu): persistent decode-step kernel
void* decode_plan_create(const G4qDecodePhase* phases, int n, int max_tokens, int rank, int n_ranks,
                         const G4qPhasePrologue* prologues = nullptr);
void decode_plan_buffers(void* plan, void** slots, uint64_t* slot_bytes, void** xkeys, uint64_t* xkey_bytes);
void decode_plan_set_peers(void* plan, void* const* slots, void* const* xkeys);
void decode_plan_free(void* plan);
int64_t decode_plan_trace_words(void* plan);
void decode_plan_set_trace(void* plan, uint64_t* buffer, int64_t words);
void decode_plan_run(void* plan, int M, float eps, float softcap, int64_t row_offset, int32_t* tokens, float* values,
                     uint64_t* keys, uint16_t* logits, int64_t ld_logits, cudaStream_t st);

// kernels (g4q_gemm.cu): tcgen05 dequant-GEMM for M > 16
void launch_gemm(const QmmCall& c, cudaStream_t st);
bool gemm_supported(const QmmCall& c);
// k-block splits the GEMM uses for an M x N x K call (1: unsplit; a larger count also needs the
// split-K scratch, which is grown outside stream captures only)
int gemm_splits(int64_t M, int64_t N, int64_t K);

}  // namespace g4q
