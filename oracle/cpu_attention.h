/*
 * cpu_attention.h — CPU oracle for the attention hot path. TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of alpaca.swift's CPU reference attention (Sources/AlpacaCore/Operations/CPUOps.swift)
 * used as the checker for the CUDA library. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * load it; the product library never links or calls it.
 *
 * Parity pinned by: the reference's own known-answer case Tests/AlpacaCoreTests/Fixtures/ops.json["attention"]
 * (and ["softmax"]), checked at the reference's tolerances (OperationTests.swift:72-86), plus a float64
 * torch SDPA cross-check on larger shapes (tests/test_oracle.py).
 */
#ifndef ALPACA_ORACLE_CPU_ATTENTION_H
#define ALPACA_ORACLE_CPU_ATTENTION_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* f32 -> binary16 -> f32, round to nearest even (Tensor.converted(to: .float16), Tensor.swift:234). */
float oracle_f16_round(float x);
void oracle_f16_round_array(const float* in, float* out, int64_t n);
/* binary16 bit patterns <-> f32 */
uint16_t oracle_f32_to_f16_bits(float x);
float oracle_f16_bits_to_f32(uint16_t h);

/* CPUOps.attentionScores (CPUOps.swift:222-249): scores[H][T][length], masked entries -inf. */
void oracle_attention_scores(const float* q, const float* keys, int tokens, int n_heads, int n_kv, int head_dim,
                             int length, int start, float* scores);
/* CPUOps.softmax (CPUOps.swift:162-175), in place over rows of n. */
void oracle_softmax(float* x, int64_t rows, int n);
/* CPUOps.attentionApply (CPUOps.swift:252-274): out[T][H][d] from probs[H][T][length]. */
void oracle_attention_apply(const float* probs, const float* values, int n_heads, int tokens, int length, int n_kv,
                            int head_dim, float* out);

/* The three steps fused row by row (one (head, token) row at a time, same per-element operation order, so the
 * result is bit-identical to scores -> softmax -> apply without materialising [H,T,length]). `scale` <= 0
 * selects the reference's 1/sqrt(head_dim). Rows are split over `threads` POSIX threads (1 = the reference's
 * single-threaded loops). `row_begin/row_end` select a subset of the H*T rows (row = h*T + t) for sampled
 * parity checks and bounded CPU timing; pass 0 and H*T for all. Rows outside the range are left untouched. */
void oracle_attention(const float* q, const float* keys, const float* values, int tokens, int n_heads, int n_kv,
                      int head_dim, int length, int start, float scale, float* out, int threads, int64_t row_begin,
                      int64_t row_end);

/* Strided variant of oracle_attention over one sequence: q token stride, kv row stride, out token stride (in
 * elements), so batched caches with capacity > length can be checked in place. */
void oracle_attention_strided(const float* q, int64_t q_token_stride, const float* keys, const float* values,
                              int64_t kv_row_stride, int tokens, int n_heads, int n_kv, int head_dim, int length,
                              int start, float scale, float* out, int64_t out_token_stride, int threads,
                              int64_t row_begin, int64_t row_end);

/* Like oracle_attention_strided but over an explicit list of rows (row = h*tokens + t), split over `threads`
 * POSIX threads: exact sampled parity checks and bounded CPU timing without per-row call overhead. */
void oracle_attention_rows(const float* q, int64_t q_token_stride, const float* keys, const float* values,
                           int64_t kv_row_stride, int tokens, int n_heads, int n_kv, int head_dim, int length,
                           int start, float scale, float* out, int64_t out_token_stride, const int64_t* rows,
                           int64_t n_rows, int threads);

/* ErrorMetrics (Sources/AlpacaCore/Runtime/ErrorMetrics.swift:15-27):
 * out[0]=maxAbs, out[1]=meanAbs, out[2]=rms, out[3]=maxRelativeToPeak. */
void oracle_error_metrics(const float* actual, const double* expected, int64_t n, double out[4]);
void oracle_error_metrics_f32(const float* actual, const float* expected, int64_t n, double out[4]);

/* SplitMix64 of Tests/AlpacaMetalTests/KernelTests.swift:102-114; nextFloat() uniform in [-1,1), times `scale`. */
void oracle_splitmix_uniform(uint64_t seed, float scale, float* out, int64_t n);
/* SplitMix64 + Box-Muller standard normal draws (pairs, double precision, rounded to f32). */
void oracle_splitmix_normal(uint64_t seed, float* out, int64_t n);

#ifdef __cplusplus
}
#endif

#endif
