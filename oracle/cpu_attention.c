/*
 * cpu_attention.c — CPU oracle for the attention hot path. TEST INFRASTRUCTURE ONLY: loaded by tests/,
 * __graft_entry__.smoke() and the CPU-baseline leg of bench.py as the checker; never by the product library.
 *
 * Restates Sources/AlpacaCore/Operations/CPUOps.swift of alpaca.swift with the same per-element arithmetic:
 * float32 operands, float32 accumulators, the dot product summed over i = 0..d-1 in order, the 1/sqrt(d)
 * scale applied after the dot, libm expf, sums in position order, and the w == 0 skip of attentionApply.
 * Built with -ffp-contract=off so no multiply-add is fused (Swift does not contract a*b+c).
 */
#include "cpu_attention.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- binary16 rounding (round to nearest even) */

uint16_t oracle_f32_to_f16_bits(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    uint32_t sign = (u >> 16) & 0x8000u;
    uint32_t exp = (u >> 23) & 0xffu;
    uint32_t man = u & 0x7fffffu;
    if (exp == 0xffu) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u | (man >> 13) : 0u)); /* inf / nan */
    int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u); /* overflow -> inf */
    if (e <= 0) {
        /* subnormal half (or zero): value = man_full * 2^(exp-150); half ulp = 2^-24 */
        if (e < -10) return (uint16_t)sign; /* below half of the smallest subnormal: rounds to zero */
        uint32_t full = man | 0x800000u;   /* 24-bit significand */
        uint32_t shift = (uint32_t)(14 - e); /* bits to drop so the unit is 2^-24 */
        uint32_t q = full >> shift;
        uint32_t rem = full & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q); /* q may carry into the exponent field: that is the correct encoding */
    }
    uint32_t q = ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++; /* carry may reach inf: correct */
    return (uint16_t)(sign | q);
}

float oracle_f16_bits_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = ((uint32_t)h >> 10) & 0x1fu;
    uint32_t man = (uint32_t)h & 0x3ffu;
    uint32_t u;
    if (exp == 0) {
        if (man == 0) {
            u = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do { e++; man <<= 1; } while (!(man & 0x400u));
            u = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
        }
    } else if (exp == 31) {
        u = sign | 0x7f800000u | (man << 13);
    } else {
        u = sign | ((exp - 15 + 127) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

float oracle_f16_round(float x) { return oracle_f16_bits_to_f32(oracle_f32_to_f16_bits(x)); }

void oracle_f16_round_array(const float* in, float* out, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = oracle_f16_round(in[i]);
}

/* ---------------------------------------------------------------- the three reference steps */

static float ref_scale(int head_dim) { return 1.0f / sqrtf((float)head_dim); } /* CPUOps.swift:234 */

/* CPUOps.swift:222-249 */
void oracle_attention_scores(const float* q, const float* keys, int tokens, int n_heads, int n_kv, int hd,
                             int length, int start, float* s) {
    const int group = n_heads / n_kv;
    const float scale = ref_scale(hd);
    for (int64_t i = 0; i < (int64_t)n_heads * tokens * length; i++) s[i] = -INFINITY;
    for (int h = 0; h < n_heads; h++) {
        for (int t = 0; t < tokens; t++) {
            for (int p = 0; p <= start + t; p++) {
                float acc = 0.0f;
                const int64_t qb = ((int64_t)t * n_heads + h) * hd, kb = ((int64_t)p * n_kv + h / group) * hd;
                for (int i = 0; i < hd; i++) acc += q[qb + i] * keys[kb + i];
                s[((int64_t)h * tokens + t) * length + p] = acc * scale;
            }
        }
    }
}

/* CPUOps.swift:162-175 */
void oracle_softmax(float* v, int64_t rows, int d) {
    for (int64_t r = 0; r < rows; r++) {
        float* row = v + r * d;
        float mx = -INFINITY;
        for (int i = 0; i < d; i++) mx = row[i] > mx ? row[i] : mx; /* Swift max(mx, x) */
        float sum = 0.0f;
        for (int i = 0; i < d; i++) {
            row[i] = expf(row[i] - mx);
            sum += row[i];
        }
        for (int i = 0; i < d; i++) row[i] /= sum;
    }
}

/* CPUOps.swift:252-274 */
void oracle_attention_apply(const float* probs, const float* values, int n_heads, int tokens, int length, int n_kv,
                            int hd, float* out) {
    const int group = n_heads / n_kv;
    memset(out, 0, sizeof(float) * (size_t)tokens * n_heads * hd);
    for (int h = 0; h < n_heads; h++) {
        for (int t = 0; t < tokens; t++) {
            for (int p = 0; p < length; p++) {
                const float w = probs[((int64_t)h * tokens + t) * length + p];
                if (w == 0.0f) continue;
                const int64_t vb = ((int64_t)p * n_kv + h / group) * hd, ob = ((int64_t)t * n_heads + h) * hd;
                for (int i = 0; i < hd; i++) out[ob + i] += w * values[vb + i];
            }
        }
    }
}

/* ---------------------------------------------------------------- fused row-by-row form */

typedef struct {
    const float *q, *k, *v;
    int64_t q_ts, kv_rs, o_ts;
    int tokens, n_heads, n_kv, hd, length, start;
    float scale;
    float* out;
    int64_t row_begin, row_end;
    int tid, nthreads;
    const int64_t* rows; /* optional explicit row list of length row_end (row_begin unused) */
} row_job;

/* One (h, t) row: scores over the whole `length` (masked = -inf), softmax, apply; identical operation order to
 * the three-step form, whose loops visit each row's elements in the same sequence. */
static void attention_row(const row_job* j, int h, int t, float* srow) {
    const int group = j->n_heads / j->n_kv, hd = j->hd, length = j->length;
    const float* qrow = j->q + (int64_t)t * j->q_ts + (int64_t)h * hd;
    for (int p = 0; p < length; p++) srow[p] = -INFINITY;
    for (int p = 0; p <= j->start + t; p++) {
        const float* krow = j->k + (int64_t)p * j->kv_rs + (int64_t)(h / group) * hd;
        float acc = 0.0f;
        for (int i = 0; i < hd; i++) acc += qrow[i] * krow[i];
        srow[p] = acc * j->scale;
    }
    float mx = -INFINITY;
    for (int p = 0; p < length; p++) mx = srow[p] > mx ? srow[p] : mx;
    float sum = 0.0f;
    for (int p = 0; p < length; p++) {
        srow[p] = expf(srow[p] - mx);
        sum += srow[p];
    }
    for (int p = 0; p < length; p++) srow[p] /= sum;
    float* orow = j->out + (int64_t)t * j->o_ts + (int64_t)h * hd;
    for (int i = 0; i < hd; i++) orow[i] = 0.0f;
    for (int p = 0; p < length; p++) {
        const float w = srow[p];
        if (w == 0.0f) continue;
        const float* vrow = j->v + (int64_t)p * j->kv_rs + (int64_t)(h / group) * hd;
        for (int i = 0; i < hd; i++) orow[i] += w * vrow[i];
    }
}

static void* list_worker(void* arg);

static void* row_worker(void* arg) {
    const row_job* j = (const row_job*)arg;
    float* srow = (float*)malloc(sizeof(float) * (size_t)(j->length > 0 ? j->length : 1));
    if (!srow) return NULL;
    /* row = h * tokens + t; interleave rows over threads so causal work is balanced */
    for (int64_t r = j->row_begin + j->tid; r < j->row_end; r += j->nthreads) {
        const int h = (int)(r / j->tokens), t = (int)(r % j->tokens);
        attention_row(j, h, t, srow);
    }
    free(srow);
    return NULL;
}

void oracle_attention_strided(const float* q, int64_t q_ts, const float* keys, const float* values, int64_t kv_rs,
                              int tokens, int n_heads, int n_kv, int hd, int length, int start, float scale,
                              float* out, int64_t o_ts, int threads, int64_t row_begin, int64_t row_end) {
    if (tokens <= 0 || n_heads <= 0) return;
    const int64_t nrows = (int64_t)n_heads * tokens;
    if (row_begin < 0) row_begin = 0;
    if (row_end > nrows) row_end = nrows;
    if (row_end <= row_begin) return;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    row_job base = {q, keys, values, q_ts, kv_rs, o_ts, tokens, n_heads, n_kv, hd, length, start,
                    scale > 0.0f ? scale : ref_scale(hd), out, row_begin, row_end, 0, threads, NULL};
    if (threads == 1) {
        row_worker(&base);
        return;
    }
    pthread_t tids[256];
    row_job jobs[256];
    int started = 0;
    for (int i = 0; i < threads; i++) {
        jobs[i] = base;
        jobs[i].tid = i;
        if (pthread_create(&tids[i], NULL, row_worker, &jobs[i]) == 0) {
            started++;
        } else {
            /* could not start a thread: run its share here */
            row_worker(&jobs[i]);
            tids[i] = 0;
        }
    }
    for (int i = 0; i < threads; i++)
        if (tids[i]) pthread_join(tids[i], NULL);
    (void)started;
}

static void* list_worker(void* arg) {
    const row_job* j = (const row_job*)arg;
    float* srow = (float*)malloc(sizeof(float) * (size_t)(j->length > 0 ? j->length : 1));
    if (!srow) return NULL;
    const int64_t nrows = (int64_t)j->n_heads * j->tokens;
    for (int64_t i = j->tid; i < j->row_end; i += j->nthreads) {
        const int64_t r = j->rows[i];
        if (r < 0 || r >= nrows) continue;
        attention_row(j, (int)(r / j->tokens), (int)(r % j->tokens), srow);
    }
    free(srow);
    return NULL;
}

void oracle_attention_rows(const float* q, int64_t q_ts, const float* keys, const float* values, int64_t kv_rs,
                           int tokens, int n_heads, int n_kv, int hd, int length, int start, float scale, float* out,
                           int64_t o_ts, const int64_t* rows, int64_t n_rows, int threads) {
    if (tokens <= 0 || n_heads <= 0 || n_rows <= 0) return;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    row_job base = {q, keys, values, q_ts, kv_rs, o_ts, tokens, n_heads, n_kv, hd, length, start,
                    scale > 0.0f ? scale : ref_scale(hd), out, 0, n_rows, 0, threads, rows};
    if (threads == 1) {
        list_worker(&base);
        return;
    }
    pthread_t tids[256];
    row_job jobs[256];
    for (int i = 0; i < threads; i++) {
        jobs[i] = base;
        jobs[i].tid = i;
        if (pthread_create(&tids[i], NULL, list_worker, &jobs[i]) != 0) {
            list_worker(&jobs[i]);
            tids[i] = 0;
        }
    }
    for (int i = 0; i < threads; i++)
        if (tids[i]) pthread_join(tids[i], NULL);
}

void oracle_attention(const float* q, const float* keys, const float* values, int tokens, int n_heads, int n_kv,
                      int hd, int length, int start, float scale, float* out, int threads, int64_t row_begin,
                      int64_t row_end) {
    oracle_attention_strided(q, (int64_t)n_heads * hd, keys, values, (int64_t)n_kv * hd, tokens, n_heads, n_kv, hd,
                             length, start, scale, out, (int64_t)n_heads * hd, threads, row_begin, row_end);
}

/* ---------------------------------------------------------------- ErrorMetrics.swift:15-27 */

void oracle_error_metrics(const float* a, const double* e, int64_t n, double out[4]) {
    double mx = 0.0, sum = 0.0, sq = 0.0, peak = 0.0;
    for (int64_t i = 0; i < n; i++) {
        const double d = fabs((double)a[i] - e[i]);
        mx = d > mx ? d : mx;
        sum += d;
        sq += d * d;
        const double ae = fabs(e[i]);
        peak = ae > peak ? ae : peak;
    }
    out[0] = mx;
    out[1] = n > 0 ? sum / (double)n : 0.0;
    out[2] = n > 0 ? sqrt(sq / (double)n) : 0.0;
    out[3] = peak > 0.0 ? mx / peak : mx;
}

void oracle_error_metrics_f32(const float* a, const float* e, int64_t n, double out[4]) {
    double mx = 0.0, sum = 0.0, sq = 0.0, peak = 0.0;
    for (int64_t i = 0; i < n; i++) {
        const double d = fabs((double)a[i] - (double)e[i]);
        mx = d > mx ? d : mx;
        sum += d;
        sq += d * d;
        const double ae = fabs((double)e[i]);
        peak = ae > peak ? ae : peak;
    }
    out[0] = mx;
    out[1] = n > 0 ? sum / (double)n : 0.0;
    out[2] = n > 0 ? sqrt(sq / (double)n) : 0.0;
    out[3] = peak > 0.0 ? mx / peak : mx;
}

/* ---------------------------------------------------------------- seeded generators */

/* KernelTests.swift:102-111 */
static uint64_t splitmix_next(uint64_t* state) {
    *state += 0x9E3779B97F4A7C15ull;
    uint64_t z = *state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* KernelTests.swift:113: Float(Double(next() >> 11) / Double(1 << 53)) * 2 - 1 (float ops after the cast) */
void oracle_splitmix_uniform(uint64_t seed, float scale, float* out, int64_t n) {
    uint64_t st = seed;
    for (int64_t i = 0; i < n; i++) {
        const float u = (float)((double)(splitmix_next(&st) >> 11) / 9007199254740992.0);
        out[i] = (u * 2.0f - 1.0f) * scale;
    }
}

void oracle_splitmix_normal(uint64_t seed, float* out, int64_t n) {
    uint64_t st = seed;
    const double two_pi = 6.283185307179586476925286766559;
    for (int64_t i = 0; i < n; i += 2) {
        const double u1 = ((double)(splitmix_next(&st) >> 11) + 1.0) / 9007199254740992.0; /* (0, 1] */
        const double u2 = (double)(splitmix_next(&st) >> 11) / 9007199254740992.0;         /* [0, 1) */
        const double r = sqrt(-2.0 * log(u1));
        out[i] = (float)(r * cos(two_pi * u2));
        if (i + 1 < n) out[i + 1] = (float)(r * sin(two_pi * u2));
    }
}
