// rope_kv.cu — fused RoPE of the new queries and keys plus the KV-cache append, the step upstream of attention.
//
// Same job as alpaca.swift's rope_qkv_store_kv16 / _kv32 (Sources/AlpacaMetal/Kernels/decode_fused.metal:126-154,
// encoded by KernelEncoder.ropeQKVStore, KernelEncoder.swift:401-411): q rotated in place, k rotated and v copied
// into cache row `position`, each cache value converted to the cache type. The angle arithmetic follows the CPU
// reference CPUOps.rope (Sources/AlpacaCore/Operations/CPUOps.swift:184-210) rather than the Metal kernel's f32
// angle: frequencies theta^(-2i/d) are computed on the host in double (the caller's ropeFrequencies,
// KernelEncoder.swift:413-415, without the rounding to f32), the angle position * freq in double, cos and sin in
// double rounded once to f32, and the rotation a*c - b*s, a*s + b*c as separately rounded f32 operations.
//
// One CTA per (token, sequence): its first d/2 threads compute the token's (cos, sin) pairs into shared memory,
// then all threads rotate / copy the pairs of the token's H query rows and Hkv key and value rows. The step is a
// few bytes per element and HBM-bound; accesses are per pair (8 bytes f32), coalesced along head_dim.
#include <cuda_fp16.h>

#include <cmath>

#include "common.cuh"
#include "internal.h"

namespace alpaca {
namespace {

constexpr int kRopeThreads = 128;
constexpr int kRopeMaxPairs = 128;  // head_dim <= 256

struct RopeArgs {
    void* q;
    int64_t q_token_stride, q_seq_stride;
    const float* k;
    const float* v;
    int64_t kv_token_stride, kv_seq_stride;
    void* k_cache;
    void* v_cache;
    int64_t cache_row_stride, cache_seq_stride;
    const int* positions;
    int start, n_heads, n_kv_heads, half;
    double freq[kRopeMaxPairs];  // theta^(-2i/d), host-computed in double
};

template <typename T>
__device__ __forceinline__ float ld(const T* p);
template <>
__device__ __forceinline__ float ld<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld<__half>(const __half* p) { return __half2float(*p); }

template <typename T>
__device__ __forceinline__ void st(T* p, float x);
template <>
__device__ __forceinline__ void st<float>(float* p, float x) { *p = x; }
template <>
__device__ __forceinline__ void st<__half>(__half* p, float x) { *p = __float2half_rn(x); }

// Element offsets of pair i within a head row.
template <bool kInterleaved>
__device__ __forceinline__ void pair_index(int i, int half, int& ia, int& ib) {
    ia = kInterleaved ? 2 * i : i;
    ib = kInterleaved ? 2 * i + 1 : i + half;
}

template <bool kInterleaved, typename QT, typename CT>
__global__ void __launch_bounds__(kRopeThreads) rope_kv_kernel(const __grid_constant__ RopeArgs a) {
    __shared__ float2 cs[kRopeMaxPairs];
    const int t = blockIdx.x, seq = blockIdx.y, tid = threadIdx.x;
    const int pos = (a.positions ? a.positions[seq] : a.start) + t;
    for (int i = tid; i < a.half; i += kRopeThreads) {
        double s, c;
        sincos(static_cast<double>(pos) * a.freq[i], &s, &c);
        cs[i] = make_float2(static_cast<float>(c), static_cast<float>(s));
    }
    __syncthreads();

    const int d = 2 * a.half;
    const int rows = a.n_heads + 2 * a.n_kv_heads;
    QT* q = static_cast<QT*>(a.q) + seq * a.q_seq_stride + static_cast<int64_t>(t) * a.q_token_stride;
    const int64_t kv_off = seq * a.kv_seq_stride + static_cast<int64_t>(t) * a.kv_token_stride;
    const int64_t cache_off = seq * a.cache_seq_stride + static_cast<int64_t>(pos) * a.cache_row_stride;
    CT* kc = static_cast<CT*>(a.k_cache) + cache_off;
    CT* vc = static_cast<CT*>(a.v_cache) + cache_off;
    for (int idx = tid; idx < rows * a.half; idx += kRopeThreads) {
        const int r = idx / a.half, i = idx - r * a.half;
        int ia, ib;
        pair_index<kInterleaved>(i, a.half, ia, ib);
        const float2 w = cs[i];
        if (r < a.n_heads) {  // query head r, in place
            QT* p = q + r * d;
            const float x0 = ld(p + ia), x1 = ld(p + ib);
            st(p + ia, __fsub_rn(__fmul_rn(x0, w.x), __fmul_rn(x1, w.y)));
            st(p + ib, __fadd_rn(__fmul_rn(x0, w.y), __fmul_rn(x1, w.x)));
        } else if (r < a.n_heads + a.n_kv_heads) {  // key head: rotate into the cache
            const int h = r - a.n_heads;
            const float* p = a.k + kv_off + h * d;
            const float x0 = p[ia], x1 = p[ib];
            st(kc + h * d + ia, __fsub_rn(__fmul_rn(x0, w.x), __fmul_rn(x1, w.y)));
            st(kc + h * d + ib, __fadd_rn(__fmul_rn(x0, w.y), __fmul_rn(x1, w.x)));
        } else {  // value head: copy into the cache
            const int h = r - a.n_heads - a.n_kv_heads;
            const float* p = a.v + kv_off + h * d;
            st(vc + h * d + ia, p[ia]);
            st(vc + h * d + ib, p[ib]);
        }
    }
}

template <bool kInterleaved, typename QT>
cudaError_t launch_q(const RopeArgs& a, const alpaca_rope_desc& d, cudaStream_t s) {
    const dim3 grid(d.tokens, d.n_seqs, 1);
    if (d.cache_dtype == ALPACA_F16) rope_kv_kernel<kInterleaved, QT, __half><<<grid, kRopeThreads, 0, s>>>(a);
    else rope_kv_kernel<kInterleaved, QT, float><<<grid, kRopeThreads, 0, s>>>(a);
    return cudaGetLastError();
}

template <bool kInterleaved>
cudaError_t launch_i(const RopeArgs& a, const alpaca_rope_desc& d, cudaStream_t s) {
    return d.q_dtype == ALPACA_F16 ? launch_q<kInterleaved, __half>(a, d, s) : launch_q<kInterleaved, float>(a, d, s);
}

}  // namespace

int rope_max_head_dim() { return 2 * kRopeMaxPairs; }

cudaError_t launch_rope_kv(const alpaca_rope_desc& d, cudaStream_t s) {
    RopeArgs a;
    a.q = d.q;
    a.q_token_stride = d.q_token_stride;
    a.q_seq_stride = d.q_seq_stride;
    a.k = d.k;
    a.v = d.v;
    a.kv_token_stride = d.kv_token_stride;
    a.kv_seq_stride = d.kv_seq_stride;
    a.k_cache = d.k_cache;
    a.v_cache = d.v_cache;
    a.cache_row_stride = d.cache_row_stride;
    a.cache_seq_stride = d.cache_seq_stride;
    a.positions = d.positions;
    a.start = d.start_position;
    a.n_heads = d.n_heads;
    a.n_kv_heads = d.n_kv_heads;
    a.half = d.head_dim / 2;
    const double theta = static_cast<double>(d.theta);
    for (int i = 0; i < kRopeMaxPairs; i++)
        a.freq[i] = i < a.half ? std::pow(theta, -2.0 * static_cast<double>(i) / static_cast<double>(d.head_dim)) : 0.0;
    return d.interleaved ? launch_i<true>(a, d, s) : launch_i<false>(a, d, s);
}

}  // namespace alpaca
