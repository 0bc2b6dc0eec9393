/*
 * cpu_proj.c — CPU oracle for the fused decode projections. TEST INFRASTRUCTURE ONLY: loaded by tests/ and the
 * CPU leg of bench.py as the checker; never by the product library.
 *
 * Restates CPUOps.rmsNorm / linear / dot / silu and the GGUF q8_0 / q4_0 (de)quantisers of alpaca.swift
 * (Sources/AlpacaCore/Operations/CPUOps.swift:49-158, Quantization.swift:9-73) with the same per-element
 * arithmetic: f32 operands and accumulators, sums in index order, no fused multiply-add (-ffp-contract=off).
 */
#include "cpu_proj.h"

#include <math.h>
#include <string.h>

#include "cpu_attention.h"

int64_t oracle_row_bytes(int format, int k) {
    switch (format) {
        case 0: return 2 * (int64_t)k;
        case 1: return (int64_t)(k / 32) * 34;
        case 2: return (int64_t)(k / 32) * 18;
        default: return 4 * (int64_t)k;
    }
}

static float half_at(const uint8_t* p) {
    uint16_t h;
    memcpy(&h, p, 2); /* loadUnaligned(as: Float16.self) */
    return oracle_f16_bits_to_f32(h);
}

/* CPUOps.dot (CPUOps.swift:107-141). */
float oracle_row_dot(int format, const void* row, const float* x, int k) {
    const uint8_t* p = (const uint8_t*)row;
    float acc = 0.0f;
    switch (format) {
        case 0:
            for (int i = 0; i < k; i++) acc += half_at(p + 2 * i) * x[i];
            break;
        case 1:
            for (int b = 0; b < k / 32; b++) {
                const uint8_t* blk = p + (int64_t)b * 34;
                const float d = half_at(blk);
                float s = 0.0f;
                for (int j = 0; j < 32; j++) s += (float)(int8_t)blk[2 + j] * x[b * 32 + j];
                acc += d * s;
            }
            break;
        case 2:
            for (int b = 0; b < k / 32; b++) {
                const uint8_t* blk = p + (int64_t)b * 18;
                const float d = half_at(blk);
                float s = 0.0f;
                for (int j = 0; j < 16; j++) {
                    s += (float)((int)(blk[2 + j] & 0x0F) - 8) * x[b * 32 + j];
                    s += (float)((int)(blk[2 + j] >> 4) - 8) * x[b * 32 + j + 16];
                }
                acc += d * s;
            }
            break;
        default: {
            const float* w = (const float*)row;
            for (int i = 0; i < k; i++) acc += w[i] * x[i];
        }
    }
    return acc;
}

/* CPUOps.rmsNorm (CPUOps.swift:144-158). */
void oracle_rmsnorm(const float* x, const float* w, int64_t rows, int d, float eps, float* out) {
    for (int64_t r = 0; r < rows; r++) {
        const float* xr = x + r * d;
        float ss = 0.0f;
        for (int i = 0; i < d; i++) ss += xr[i] * xr[i];
        const float scale = 1.0f / sqrtf(ss / (float)d + eps);
        for (int i = 0; i < d; i++) out[r * d + i] = xr[i] * scale * w[i];
    }
}

/* CPUOps.silu (CPUOps.swift:49-53). */
float oracle_silu(float x) { return x / (1.0f + expf(-x)); }

/* dequantize (Quantization.swift:9-35). */
void oracle_dequantize(int format, const void* src, int64_t elements, float* dst) {
    const uint8_t* p = (const uint8_t*)src;
    const int64_t blocks = elements / 32;
    if (format == 1) {
        for (int64_t b = 0; b < blocks; b++) {
            const float d = half_at(p + b * 34);
            for (int j = 0; j < 32; j++) dst[b * 32 + j] = d * (float)(int8_t)p[b * 34 + 2 + j];
        }
    } else if (format == 2) {
        for (int64_t b = 0; b < blocks; b++) {
            const float d = half_at(p + b * 18);
            for (int j = 0; j < 16; j++) {
                dst[b * 32 + j] = d * (float)((int)(p[b * 18 + 2 + j] & 0x0F) - 8);
                dst[b * 32 + j + 16] = d * (float)((int)(p[b * 18 + 2 + j] >> 4) - 8);
            }
        }
    } else if (format == 0) {
        for (int64_t i = 0; i < elements; i++) dst[i] = half_at(p + 2 * i);
    } else {
        memcpy(dst, src, (size_t)elements * 4);
    }
}

/* quantize (Quantization.swift:39-73): ggml's quantize_row_q8_0_ref / quantize_row_q4_0_ref as restated there. */
void oracle_quantize(int format, const float* values, int64_t n, void* dst) {
    uint8_t* out = (uint8_t*)dst;
    for (int64_t b = 0; b < n / 32; b++) {
        const float* x = values + b * 32;
        if (format == 1) {
            float amax = 0.0f;
            for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(x[j]));
            const float d = amax / 127.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            uint8_t* p = out + b * 34;
            const uint16_t dh = oracle_f32_to_f16_bits(d);
            memcpy(p, &dh, 2);
            for (int j = 0; j < 32; j++) p[2 + j] = (uint8_t)(int8_t)roundf(x[j] * id); /* to nearest, ties away */
        } else {
            float maxv = 0.0f, amax = 0.0f;
            for (int j = 0; j < 32; j++)
                if (fabsf(x[j]) > amax) {
                    amax = fabsf(x[j]);
                    maxv = x[j];
                }
            const float d = maxv / -8.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            uint8_t* p = out + b * 18;
            const uint16_t dh = oracle_f32_to_f16_bits(d);
            memcpy(p, &dh, 2);
            for (int j = 0; j < 16; j++) {
                int lo = (int)(x[j] * id + 8.5f), hi = (int)(x[j + 16] * id + 8.5f); /* Int() truncates */
                if (lo > 15) lo = 15;
                if (hi > 15) hi = 15;
                p[2 + j] = (uint8_t)(lo | (hi << 4));
            }
        }
    }
}

void oracle_decode_project(int format, int k, const int rows[3], unsigned flags, float eps, const void* const w[3],
                           const float* x, int n_tokens, int64_t x_stride, const float* norm_weight, float* const y[3],
                           const int64_t y_stride[3]) {
    const int64_t rb = oracle_row_bytes(format, k);
    float xn[16384];
    for (int t = 0; t < n_tokens; t++) {
        const float* xt = x + t * x_stride;
        if (flags & 1u) oracle_rmsnorm(xt, norm_weight, 1, k, eps, xn);
        else memcpy(xn, xt, (size_t)k * 4);
        if (flags & 2u) {
            for (int r = 0; r < rows[0]; r++) {
                const float g = oracle_row_dot(format, (const uint8_t*)w[0] + r * rb, xn, k);
                const float u = oracle_row_dot(format, (const uint8_t*)w[1] + r * rb, xn, k);
                y[0][t * y_stride[0] + r] = oracle_silu(g) * u;
            }
            continue;
        }
        for (int m = 0; m < 3; m++)
            for (int r = 0; r < rows[m]; r++) {
                const float s = oracle_row_dot(format, (const uint8_t*)w[m] + r * rb, xn, k);
                float* yp = y[m] + t * y_stride[m] + r;
                *yp = ((flags & 4u) ? *yp : 0.0f) + s;
            }
    }
}
