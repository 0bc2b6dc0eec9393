/*
 * cpu_rope.h — CPU oracle for the RoPE + KV-cache append step that produces the attention hand-off.
 * TEST INFRASTRUCTURE ONLY (loaded by tests/, __graft_entry__.smoke() and bench.py's CPU leg as the checker).
 *
 * Restates alpaca.swift's CPUOps.rope (Sources/AlpacaCore/Operations/CPUOps.swift:184-210) and composes it into
 * the per-token work of the Metal kernel rope_qkv_impl (Sources/AlpacaMetal/Kernels/decode_fused.metal:126-154):
 * q rotated in place, k rotated and v copied into cache rows start .. start + tokens - 1, each cache value
 * rounded to binary16 when the cache is f16 (KVPrecision.float16).
 *
 * Parity pinned by the reference's own known-answer case Tests/AlpacaCoreTests/Fixtures/ops.json["rope"] (both
 * pair conventions, tolerance 2e-6 of OperationTests.swift:63-70), committed as tests/golden/rope_kat.json.
 */
#ifndef ALPACA_ORACLE_CPU_ROPE_H
#define ALPACA_ORACLE_CPU_ROPE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* CPUOps.rope: x[tokens][heads][head_dim] rotated in place, token t at position start + t. interleaved != 0
 * rotates adjacent pairs (x[2i], x[2i+1]); otherwise split halves (x[i], x[i + head_dim/2]). */
void oracle_rope(float* x, int tokens, int heads, int head_dim, int start, double theta, int interleaved);

/* One sequence of the fused step. q[tokens][heads][head_dim] is rotated in place; k, v [tokens][kv_heads][head_dim]
 * are read; k_cache / v_cache [rows][kv_heads][head_dim] (f32 arrays, rows >= start + tokens) receive the rotated
 * k and the raw v at rows start + t, rounded to binary16 when cache_f16. */
void oracle_rope_kv_append(float* q, const float* k, const float* v, float* k_cache, float* v_cache, int tokens,
                           int heads, int kv_heads, int head_dim, int start, double theta, int interleaved,
                           int cache_f16);

#ifdef __cplusplus
}
#endif

#endif
