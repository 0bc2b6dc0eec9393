/*
 * abi_client.c — a plain C caller of the attention library, as a Swift, Go or C host would bind it: only
 * include/alpaca_cuda.h, libalpaca_cuda.so and the CUDA runtime, no Python, no torch.
 *
 *   abi_client          host-only entry points (version, status strings, dispatch policy, workspace sizing,
 *                       argument validation); runs without a GPU
 *   abi_client gpu      also a prefill (tcgen05 kernel, f16 Q/K/V, f32 out, 300 tokens after a 40-row prefix) and
 *                       a ragged split decode through alpaca_attention on cudaMalloc'd buffers, each checked against
 *                       the C oracle (oracle/liboracle.so) at the f16 bound 2e-3
 *
 * Exit status 0 when every check passes. Test infrastructure: the oracle is linked only as the checker.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "alpaca_cuda.h"
#include "cpu_attention.h"

#define CHECK(cond, ...)                                  \
    do {                                                  \
        if (!(cond)) {                                    \
            fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__); \
            fprintf(stderr, __VA_ARGS__);                 \
            fprintf(stderr, "\n");                        \
            exit(1);                                      \
        }                                                 \
    } while (0)

/* IEEE binary16 bits of x, round to nearest even. */
static uint16_t f16_bits(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int32_t e8 = (int32_t)((x >> 23) & 0xffu);
    uint32_t mant = x & 0x7fffffu;
    if (e8 == 0xff) return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0u));
    const int32_t e = e8 - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        const int shift = 14 - e;
        uint32_t h = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

static uint64_t lcg = 20260101u;
static float uniform_pm2(void) { /* deterministic values in [-2, 2) */
    lcg = lcg * 6364136223846793005ull + 1442695040888963407ull;
    return (float)((lcg >> 40) & 0xffffffu) / 16777216.0f * 4.0f - 2.0f;
}

/* n f16-rounded values: bits for the device, the same values as floats for the oracle. */
static void fill(uint16_t* bits, float* vals, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        const float x = uniform_pm2();
        bits[i] = f16_bits(x);
        vals[i] = oracle_f16_bits_to_f32(bits[i]);
        CHECK(vals[i] == oracle_f16_round(x), "f16 rounding disagrees with the oracle at %g", x);
    }
}

static void host_checks(void) {
    CHECK(alpaca_cuda_version() > 0, "version");
    CHECK(strcmp(alpaca_cuda_status_string(ALPACA_CUDA_OK), "") != 0, "status string");
    alpaca_attn_desc d;
    memset(&d, 0, sizeof d);
    static uint16_t dummy[16] __attribute__((aligned(16)));
    d.n_seqs = 1; d.n_heads = 9; d.n_kv_heads = 3; d.head_dim = 64; d.tokens = 300; d.start_position = 40;
    d.q_dtype = d.kv_dtype = ALPACA_F16; d.out_dtype = ALPACA_F32;
    d.q = d.k = d.v = d.out = dummy;
    d.q_token_stride = d.out_token_stride = 9 * 64; d.kv_row_stride = 3 * 64;
    alpaca_attn_kernel kind = ALPACA_ATTN_AUTO;
    CHECK(alpaca_attention_select(&d, &kind) == ALPACA_CUDA_OK && kind == ALPACA_ATTN_PREFILL_TC, "prefill policy");
    size_t ws = 1;
    CHECK(alpaca_attention_workspace_bytes(&d, ALPACA_ATTN_PREFILL_TC, &ws) == ALPACA_CUDA_OK && ws == 0,
          "f16 prefill needs no workspace");
    d.tokens = 1; d.start_position = 300;
    CHECK(alpaca_attention_select(&d, &kind) == ALPACA_CUDA_OK && kind == ALPACA_ATTN_DECODE_SPLIT, "decode policy");
    CHECK(alpaca_attention_workspace_bytes(&d, ALPACA_ATTN_DECODE_SPLIT, &ws) == ALPACA_CUDA_OK && ws > 0,
          "multi-split decode needs a workspace");
    d.n_heads = 10; /* not a multiple of the KV heads */
    CHECK(alpaca_attention_select(&d, &kind) == ALPACA_CUDA_ERR_INVALID_ARGUMENT, "invalid heads rejected");
    CHECK(strlen(alpaca_cuda_last_error()) > 0, "detail message");
    printf("host entry points ok (version %d)\n", alpaca_cuda_version());
}

static double max_abs(const float* a, const float* b, int64_t n) {
    double m = 0;
    for (int64_t i = 0; i < n; i++) {
        const double e = fabs((double)a[i] - (double)b[i]);
        if (!(e <= m)) m = e; /* NaN propagates */
    }
    return m;
}

static void gpu_prefill(void) {
    const int T = 300, start = 40, H = 9, KVH = 3, D = 64, L = start + T;
    const int64_t nq = (int64_t)T * H * D, nkv = (int64_t)L * KVH * D;
    uint16_t *hq = malloc(nq * 2), *hk = malloc(nkv * 2), *hv = malloc(nkv * 2);
    float *fq = malloc(nq * 4), *fk = malloc(nkv * 4), *fv = malloc(nkv * 4), *out = malloc(nq * 4), *ref = malloc(nq * 4);
    fill(hq, fq, nq);
    fill(hk, fk, nkv);
    fill(hv, fv, nkv);
    void *dq, *dk, *dv, *dout;
    CHECK(cudaMalloc(&dq, nq * 2) == cudaSuccess && cudaMalloc(&dk, nkv * 2) == cudaSuccess &&
              cudaMalloc(&dv, nkv * 2) == cudaSuccess && cudaMalloc(&dout, nq * 4) == cudaSuccess, "cudaMalloc");
    CHECK(cudaMemcpy(dq, hq, nq * 2, cudaMemcpyHostToDevice) == cudaSuccess, "copy q");
    CHECK(cudaMemcpy(dk, hk, nkv * 2, cudaMemcpyHostToDevice) == cudaSuccess, "copy k");
    CHECK(cudaMemcpy(dv, hv, nkv * 2, cudaMemcpyHostToDevice) == cudaSuccess, "copy v");
    alpaca_attn_desc d;
    memset(&d, 0, sizeof d);
    d.n_seqs = 1; d.n_heads = H; d.n_kv_heads = KVH; d.head_dim = D; d.tokens = T; d.start_position = start;
    d.q_dtype = d.kv_dtype = ALPACA_F16; d.out_dtype = ALPACA_F32;
    d.q = dq; d.k = dk; d.v = dv; d.out = dout;
    d.q_token_stride = d.out_token_stride = H * D; d.kv_row_stride = KVH * D;
    CHECK(alpaca_attention(&d, ALPACA_ATTN_PREFILL_TC, NULL, 0, NULL) == ALPACA_CUDA_OK, "prefill: %s",
          alpaca_cuda_last_error());
    CHECK(alpaca_cuda_device_status(NULL, 1) == ALPACA_CUDA_OK, "prefill device status");
    CHECK(cudaMemcpy(out, dout, nq * 4, cudaMemcpyDeviceToHost) == cudaSuccess, "copy out");
    oracle_attention(fq, fk, fv, T, H, KVH, D, L, start, 0.f, ref, 4, 0, (int64_t)H * T);
    const double err = max_abs(out, ref, nq);
    printf("prefill through the C ABI: max-abs %.3e against the oracle\n", err);
    CHECK(err <= 2e-3, "prefill max-abs %.3e", err);
    cudaFree(dq); cudaFree(dk); cudaFree(dv); cudaFree(dout);
    free(hq); free(hk); free(hv); free(fq); free(fk); free(fv); free(out); free(ref);
}

static void gpu_decode(void) {
    const int S = 4, H = 9, KVH = 3, D = 64, CAP = 700;
    const int32_t lens[4] = {1, 129, 300, 700};
    const int64_t nq = (int64_t)S * H * D, nkv = (int64_t)S * CAP * KVH * D;
    uint16_t *hk = malloc(nkv * 2), *hv = malloc(nkv * 2), *hqb = malloc(nq * 2);
    float *fq = malloc(nq * 4), *fk = malloc(nkv * 4), *fv = malloc(nkv * 4), *out = malloc(nq * 4), *ref = malloc(nq * 4);
    fill(hqb, fq, nq); /* f32 queries: the rounded values are exact in f32 too */
    fill(hk, fk, nkv);
    fill(hv, fv, nkv);
    void *dq, *dk, *dv, *dout, *dl, *ws;
    size_t wsb = 0;
    CHECK(cudaMalloc(&dq, nq * 4) == cudaSuccess && cudaMalloc(&dk, nkv * 2) == cudaSuccess &&
              cudaMalloc(&dv, nkv * 2) == cudaSuccess && cudaMalloc(&dout, nq * 4) == cudaSuccess &&
              cudaMalloc(&dl, sizeof lens) == cudaSuccess, "cudaMalloc");
    CHECK(cudaMemcpy(dq, fq, nq * 4, cudaMemcpyHostToDevice) == cudaSuccess, "copy q");
    CHECK(cudaMemcpy(dk, hk, nkv * 2, cudaMemcpyHostToDevice) == cudaSuccess, "copy k");
    CHECK(cudaMemcpy(dv, hv, nkv * 2, cudaMemcpyHostToDevice) == cudaSuccess, "copy v");
    CHECK(cudaMemcpy(dl, lens, sizeof lens, cudaMemcpyHostToDevice) == cudaSuccess, "copy lens");
    alpaca_attn_desc d;
    memset(&d, 0, sizeof d);
    d.n_seqs = S; d.n_heads = H; d.n_kv_heads = KVH; d.head_dim = D; d.tokens = 1;
    d.ctx_lens = dl; d.max_ctx_len = CAP;
    d.q_dtype = ALPACA_F32; d.kv_dtype = ALPACA_F16; d.out_dtype = ALPACA_F32;
    d.q = dq; d.k = dk; d.v = dv; d.out = dout;
    d.q_token_stride = d.out_token_stride = H * D; d.q_seq_stride = d.out_seq_stride = H * D;
    d.kv_row_stride = KVH * D; d.kv_seq_stride = (int64_t)CAP * KVH * D;
    CHECK(alpaca_attention_workspace_bytes(&d, ALPACA_ATTN_DECODE_SPLIT, &wsb) == ALPACA_CUDA_OK, "workspace query");
    CHECK(cudaMalloc(&ws, wsb) == cudaSuccess, "cudaMalloc workspace");
    CHECK(alpaca_attention(&d, ALPACA_ATTN_DECODE_SPLIT, ws, 0, NULL) == ALPACA_CUDA_ERR_WORKSPACE_TOO_SMALL,
          "a short workspace is reported");
    CHECK(alpaca_attention(&d, ALPACA_ATTN_DECODE_SPLIT, ws, wsb, NULL) == ALPACA_CUDA_OK, "decode: %s",
          alpaca_cuda_last_error());
    CHECK(alpaca_cuda_device_status(NULL, 1) == ALPACA_CUDA_OK, "decode device status");
    CHECK(cudaMemcpy(out, dout, nq * 4, cudaMemcpyDeviceToHost) == cudaSuccess, "copy out");
    double worst = 0;
    for (int s = 0; s < S; s++) {
        oracle_attention(fq + (int64_t)s * H * D, fk + (int64_t)s * CAP * KVH * D, fv + (int64_t)s * CAP * KVH * D, 1, H,
                         KVH, D, lens[s], lens[s] - 1, 0.f, ref + (int64_t)s * H * D, 1, 0, H);
        const double e = max_abs(out + (int64_t)s * H * D, ref + (int64_t)s * H * D, H * D);
        if (e > worst) worst = e;
    }
    printf("ragged decode through the C ABI: max-abs %.3e against the oracle\n", worst);
    CHECK(worst <= 2e-3, "decode max-abs %.3e", worst);
    cudaFree(dq); cudaFree(dk); cudaFree(dv); cudaFree(dout); cudaFree(dl); cudaFree(ws);
    free(hk); free(hv); free(hqb); free(fq); free(fk); free(fv); free(out); free(ref);
}

int main(int argc, char** argv) {
    host_checks();
    if (argc > 1 && strcmp(argv[1], "gpu") == 0) {
        gpu_prefill();
        gpu_decode();
    }
    printf("ok\n");
    return 0;
}
