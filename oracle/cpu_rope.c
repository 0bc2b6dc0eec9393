/*
 * cpu_rope.c — CPU oracle for RoPE + KV-cache append. TEST INFRASTRUCTURE ONLY (see cpu_rope.h).
 * Built with -ffp-contract=off: every product and sum is a separately rounded float operation, as in Swift.
 */
#include "cpu_rope.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "cpu_attention.h"

/* CPUOps.swift:184-210. For pair i: freq = theta^(-2i/head_dim) and angle = position * freq in double, cos and
 * sin rounded once to float; a' = a*c - b*s, b' = a*s + b*c in float. */
void oracle_rope(float* x, int tokens, int heads, int head_dim, int start, double theta, int interleaved) {
    const int half = head_dim / 2;
    for (int t = 0; t < tokens; t++) {
        const double pos = (double)(start + t);
        for (int i = 0; i < half; i++) {
            const double freq = pow(theta, -2.0 * (double)i / (double)head_dim);
            const double angle = pos * freq;
            const float c = (float)cos(angle), s = (float)sin(angle);
            for (int h = 0; h < heads; h++) {
                const int64_t base = ((int64_t)t * heads + h) * head_dim;
                const int64_t ia = interleaved ? base + 2 * i : base + i;
                const int64_t ib = interleaved ? base + 2 * i + 1 : base + i + half;
                const float a = x[ia], b = x[ib];
                x[ia] = a * c - b * s;
                x[ib] = a * s + b * c;
            }
        }
    }
}

/* decode_fused.metal:126-154 on the CPU path: q in place; cache row start + t gets KV(rotated k) and KV(v). */
void oracle_rope_kv_append(float* q, const float* k, const float* v, float* k_cache, float* v_cache, int tokens,
                           int heads, int kv_heads, int head_dim, int start, double theta, int interleaved,
                           int cache_f16) {
    oracle_rope(q, tokens, heads, head_dim, start, theta, interleaved);
    const int64_t n = (int64_t)tokens * kv_heads * head_dim;
    float* kr = (float*)malloc(sizeof(float) * (size_t)n);
    if (!kr) return;
    memcpy(kr, k, sizeof(float) * (size_t)n);
    oracle_rope(kr, tokens, kv_heads, head_dim, start, theta, interleaved);
    const int64_t row = (int64_t)kv_heads * head_dim;
    for (int t = 0; t < tokens; t++) {
        float* kd = k_cache + (int64_t)(start + t) * row;
        float* vd = v_cache + (int64_t)(start + t) * row;
        for (int64_t e = 0; e < row; e++) {
            const float kv = kr[(int64_t)t * row + e], vv = v[(int64_t)t * row + e];
            kd[e] = cache_f16 ? oracle_f16_round(kv) : kv;
            vd[e] = cache_f16 ? oracle_f16_round(vv) : vv;
        }
    }
    free(kr);
}
