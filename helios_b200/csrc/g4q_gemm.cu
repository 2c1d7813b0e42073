// g4q_gemm.cu -- K2: chunked-prefill quantized matmul for M > 16.
//
// Interim implementation: the M > 16 product runs the decode GEMV kernel over 16-token slices
// (same bit-exact R2 dequant, fp32 accumulation). The tcgen05/TMEM dequant-GEMM replaces it.
#include "g4q_internal.h"

namespace g4q {

bool gemm_supported(const QmmCall&) { return true; }

void launch_gemm(const QmmCall& c, cudaStream_t st) {
    const size_t esize = (c.flags & G4Q_QMM_OUT_F32) ? 4 : 2;
    for (int64_t m0 = 0; m0 < c.M; m0 += 16) {
        QmmCall s = c;
        s.M = c.M - m0 < 16 ? c.M - m0 : 16;
        s.x = c.x + m0 * c.ldx;
        s.y = static_cast<char*>(c.y) + m0 * c.ldy * esize;
        launch_gemv(s, st);
    }
}

}  // namespace g4q
