// attn_general.cu — general causal GQA attention with fp32 arithmetic (SIMT, no tensor cores).
//
// Same role as alpaca.swift's attention_kv16 / attention_kv32 kernels (Sources/AlpacaMetal/Kernels/
// attention.metal:34-87): any head_dim that is a multiple of 32 up to 256, f16 or f32 Q / KV / output, any
// token count and start position. It is the exact path (f32 KV is bit-faithful to the CPU reference cache) and
// the fallback the dispatch policy uses for short prefills (< 8 tokens) and short decode contexts.
//
// One warp per (sequence, token, head) row, four rows per CTA. The warp walks the visible positions 32 at a time:
// lane j scores position c*32+j against the query (held in shared memory) with a sequential fp32 dot product
// scaled after the sum, as CPUOps.attentionScores does (CPUOps.swift:238-245); the chunk updates a running
// max / denominator (accurate expf); then the weighted values are accumulated with lanes spread over the head
// dimension so value reads are coalesced.
#include "common.cuh"
#include "internal.h"

namespace alpaca {
namespace {

constexpr int kWarps = 4;

struct GeneralArgs {
    const void* q;
    int64_t q_token_stride, q_seq_stride;
    int q_f16;
    const void* k;
    const void* v;
    int64_t kv_row_stride, kv_seq_stride;
    void* out;
    int64_t out_token_stride, out_seq_stride;
    int out_f16;
    const int* ctx_lens;
    int n_seqs, n_heads, n_kv_heads, tokens, start;
    float scale;
};

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }

// Dot of the shared-memory query with one cache row, summed in index order.
template <typename KT, int D>
__device__ __forceinline__ float row_dot(const float* qs, const KT* krow);

template <int D>
__device__ __forceinline__ float row_dot_impl_f32(const float* qs, const float* krow) {
    float acc = 0.f;
#pragma unroll 4
    for (int i = 0; i < D; i += 4) {
        const float4 k4 = *reinterpret_cast<const float4*>(krow + i);
        acc = fmaf(qs[i], k4.x, acc);
        acc = fmaf(qs[i + 1], k4.y, acc);
        acc = fmaf(qs[i + 2], k4.z, acc);
        acc = fmaf(qs[i + 3], k4.w, acc);
    }
    return acc;
}

template <int D>
__device__ __forceinline__ float row_dot_impl_f16(const float* qs, const __half* krow) {
    float acc = 0.f;
#pragma unroll 2
    for (int i = 0; i < D; i += 8) {
        const uint4 u = *reinterpret_cast<const uint4*>(krow + i);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float2 f = __half22float2(h[j]);
            acc = fmaf(qs[i + 2 * j], f.x, acc);
            acc = fmaf(qs[i + 2 * j + 1], f.y, acc);
        }
    }
    return acc;
}

template <typename KT, int D>
__global__ void __launch_bounds__(kWarps * 32) general_kernel(const GeneralArgs a) {
    constexpr int EPL = D / 32;
    __shared__ __align__(16) float q_s[kWarps][D];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
    const int64_t total = static_cast<int64_t>(a.n_seqs) * a.tokens * a.n_heads;
    if (row >= total) return;  // whole warp
    const int h = static_cast<int>(row % a.n_heads);
    const int t = static_cast<int>((row / a.n_heads) % a.tokens);
    const int seq = static_cast<int>(row / (static_cast<int64_t>(a.n_heads) * a.tokens));
    const int G = a.n_heads / a.n_kv_heads, kvh = h / G;
    const int start = a.ctx_lens ? a.ctx_lens[seq] - 1 : a.start;
    const int last = start + t;  // inclusive causal limit

    const int64_t qoff = seq * a.q_seq_stride + t * a.q_token_stride + static_cast<int64_t>(h) * D;
#pragma unroll
    for (int e = 0; e < EPL; e++) {
        const int i = lane + 32 * e;
        q_s[warp][i] = a.q_f16 ? __half2float(static_cast<const __half*>(a.q)[qoff + i])
                               : static_cast<const float*>(a.q)[qoff + i];
    }
    __syncwarp();

    const KT* kb = static_cast<const KT*>(a.k) + seq * a.kv_seq_stride + static_cast<int64_t>(kvh) * D;
    const KT* vb = static_cast<const KT*>(a.v) + seq * a.kv_seq_stride + static_cast<int64_t>(kvh) * D;
    float m = -INFINITY, l = 0.f, acc[EPL];
#pragma unroll
    for (int e = 0; e < EPL; e++) acc[e] = 0.f;

    for (int c0 = 0; c0 <= last; c0 += 32) {
        const int p = c0 + lane;
        float s = -INFINITY;
        if (p <= last) {
            float dot;
            if constexpr (sizeof(KT) == 4)
                dot = row_dot_impl_f32<D>(q_s[warp], reinterpret_cast<const float*>(kb) + p * a.kv_row_stride);
            else
                dot = row_dot_impl_f16<D>(q_s[warp], reinterpret_cast<const __half*>(kb) + p * a.kv_row_stride);
            s = dot * a.scale;
        }
        float cm = s;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
        const float m_new = fmaxf(m, cm);
        const float corr = expf(m - m_new);  // m = -inf on the first chunk -> 0
        const float w = (p <= last) ? expf(s - m_new) : 0.f;
        float ws = w;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) ws += __shfl_xor_sync(0xffffffffu, ws, o);
        l = l * corr + ws;
#pragma unroll
        for (int e = 0; e < EPL; e++) acc[e] *= corr;
        const int n = min(32, last - c0 + 1);
        for (int j = 0; j < n; j++) {
            const float wj = __shfl_sync(0xffffffffu, w, j);
            const KT* vrow = vb + static_cast<int64_t>(c0 + j) * a.kv_row_stride;
#pragma unroll
            for (int e = 0; e < EPL; e++) acc[e] = fmaf(wj, to_f(vrow[lane + 32 * e]), acc[e]);
        }
        m = m_new;
    }
    const float inv = 1.f / l;
    const int64_t ooff = seq * a.out_seq_stride + t * a.out_token_stride + static_cast<int64_t>(h) * D;
#pragma unroll
    for (int e = 0; e < EPL; e++) {
        const float val = acc[e] * inv;
        if (a.out_f16) static_cast<__half*>(a.out)[ooff + lane + 32 * e] = __float2half_rn(val);
        else static_cast<float*>(a.out)[ooff + lane + 32 * e] = val;
    }
}

template <typename KT>
cudaError_t launch_kt(const GeneralArgs& a, int D, cudaStream_t s) {
    const int64_t total = static_cast<int64_t>(a.n_seqs) * a.tokens * a.n_heads;
    const int64_t blocks = (total + kWarps - 1) / kWarps;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
    const dim3 grid(static_cast<unsigned>(blocks)), block(kWarps * 32);
    switch (D) {
        case 32: general_kernel<KT, 32><<<grid, block, 0, s>>>(a); break;
        case 64: general_kernel<KT, 64><<<grid, block, 0, s>>>(a); break;
        case 96: general_kernel<KT, 96><<<grid, block, 0, s>>>(a); break;
        case 128: general_kernel<KT, 128><<<grid, block, 0, s>>>(a); break;
        case 160: general_kernel<KT, 160><<<grid, block, 0, s>>>(a); break;
        case 192: general_kernel<KT, 192><<<grid, block, 0, s>>>(a); break;
        case 224: general_kernel<KT, 224><<<grid, block, 0, s>>>(a); break;
        case 256: general_kernel<KT, 256><<<grid, block, 0, s>>>(a); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_general(const Call& c, cudaStream_t s) {
    const alpaca_attn_desc& d = *c.d;
    GeneralArgs a;
    a.q = d.q;
    a.q_token_stride = d.q_token_stride;
    a.q_seq_stride = d.q_seq_stride;
    a.q_f16 = d.q_dtype == ALPACA_F16;
    a.k = d.k;
    a.v = d.v;
    a.kv_row_stride = d.kv_row_stride;
    a.kv_seq_stride = d.kv_seq_stride;
    a.out = d.out;
    a.out_token_stride = d.out_token_stride;
    a.out_seq_stride = d.out_seq_stride;
    a.out_f16 = d.out_dtype == ALPACA_F16;
    a.ctx_lens = d.tokens == 1 ? d.ctx_lens : nullptr;
    a.n_seqs = d.n_seqs;
    a.n_heads = d.n_heads;
    a.n_kv_heads = d.n_kv_heads;
    a.tokens = d.tokens;
    a.start = d.start_position;
    a.scale = c.scale;
    return d.kv_dtype == ALPACA_F32 ? launch_kt<float>(a, d.head_dim, s) : launch_kt<__half>(a, d.head_dim, s);
}

}  // namespace alpaca
