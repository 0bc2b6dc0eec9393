/*
 * cpu_proj.h — CPU oracle for the fused decode projections. TEST INFRASTRUCTURE ONLY.
 *
 * Restates alpaca.swift's CPU operations that the fused single-token projection kernels (dec_f16 / dec_q8_0 /
 * dec_q4_0, Sources/AlpacaMetal/Kernels/decode_fused.metal:32-122) compose:
 *   CPUOps.rmsNorm   Sources/AlpacaCore/Operations/CPUOps.swift:144-158
 *   CPUOps.linear    CPUOps.swift:77-105, with CPUOps.dot (:107-141) for f32 / f16 / q8_0 / q4_0 weight rows
 *   CPUOps.silu      CPUOps.swift:49-53, CPUOps.mul / add (:30-37)
 *   dequantize / quantize (GGUF q8_0, q4_0)  Sources/AlpacaCore/Operations/Quantization.swift:9-73
 * Pinned by the reference's own fixtures Tests/AlpacaCoreTests/Fixtures/ops.json ["linear"], ["rmsnorm"],
 * ["silu"], ["q8_0"], ["q4_0"] (tests/golden/proj_kat.json). Only tests/ and bench.py's CPU leg load it.
 */
#ifndef ALPACA_ORACLE_CPU_PROJ_H
#define ALPACA_ORACLE_CPU_PROJ_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Weight formats: 0 f16, 1 q8_0 (34-byte blocks: f16 scale + 32 int8), 2 q4_0 (18-byte blocks: f16 scale + 16
 * bytes of nibbles, element j in the low nibble of byte j, element j + 16 in its high nibble), 3 f32. */
int64_t oracle_row_bytes(int format, int k);

/* CPUOps.dot: one weight row with an f32 vector, f32 accumulation in index order (per-block partial sums times the
 * block scale for the quantised formats). */
float oracle_row_dot(int format, const void* row, const float* x, int k);

/* CPUOps.rmsNorm over rows of d: out = x * (1 / sqrt(mean(x^2) + eps)) * w. */
void oracle_rmsnorm(const float* x, const float* w, int64_t rows, int d, float eps, float* out);

/* CPUOps.silu: x / (1 + exp(-x)). */
float oracle_silu(float x);

/* dequantize(): `elements` values of `format` blocks into f32. */
void oracle_dequantize(int format, const void* src, int64_t elements, float* dst);

/* quantize(): ggml's reference quantiser as Quantization.swift:39-73 states it (q8_0 or q4_0); n % 32 == 0. */
void oracle_quantize(int format, const float* values, int64_t n, void* dst);

/* The fused projection of dec_*: for each token t (x row t), xn = rmsNorm(x_t) when flags & 1 (NORM) else x_t;
 * SILU (flags & 2): y0[t][r] = silu(W0[r]·xn) * (W1[r]·xn) for r < rows[0]; otherwise y_i[t][r] = W_i[r]·xn for
 * each matrix i with rows[i] > 0, plus the previous y_i[t][r] when flags & 4 (ADD). */
void oracle_decode_project(int format, int k, const int rows[3], unsigned flags, float eps, const void* const w[3],
                           const float* x, int n_tokens, int64_t x_stride, const float* norm_weight, float* const y[3],
                           const int64_t y_stride[3]);

#ifdef __cplusplus
}
#endif

#endif
