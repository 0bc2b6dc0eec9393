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
// Vector kernel (head_dim % 8 == 0, 16-byte aligned tensors, the usual case): one CTA per 8 tokens of a sequence.
// Every thread issues its first batch of 16-byte loads (groups of 4 pairs of the tokens' H query rows and Hkv key
// and value rows), then the CTA computes the tokens' (cos, sin) table into shared memory while those loads are in
// flight, and the threads rotate / copy and store. Scalar kernel otherwise: one CTA per token, one pair per thread
// step. The step moves ~20 bytes per f32 element pair and is HBM-bound.
#include <cuda_fp16.h>

#include <cmath>
#include <cstdlib>

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
    int start, n_heads, n_kv_heads, half, tokens;
    int tpc;  // tokens per CTA of the vector kernel (1 .. kVecTokens)
    const int* block_table;  // paged cache: [seq][max_blocks] (null: contiguous caches)
    int block_rows, max_blocks, pool_blocks;
    int64_t block_stride;
    int cache_rows;  // contiguous caches: rows per sequence, or 0 (unchecked)
    unsigned* err;
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

// Element offset of cache row `pos` of sequence `seq`; a position outside the cache (negative, past cache_rows, or
// past the block table) or a table entry outside the pool clears `ok` — nothing is written there — and raises the
// device error word.
__device__ __forceinline__ int64_t cache_row_offset(const RopeArgs& a, int seq, int pos, bool& ok) {
    ok = true;
    if (!a.block_table) {
        if (pos < 0 || (a.cache_rows > 0 && pos >= a.cache_rows)) {  // past the cache: write nothing, report it
            ok = false;
            atomicOr(a.err, kDevErrBadIndex);
            return 0;
        }
        return seq * a.cache_seq_stride + static_cast<int64_t>(pos) * a.cache_row_stride;
    }
    const int b = pos / a.block_rows;
    const int blk = (pos >= 0 && b < a.max_blocks) ? a.block_table[static_cast<int64_t>(seq) * a.max_blocks + b] : -1;
    if (blk < 0 || blk >= a.pool_blocks) {
        ok = false;
        atomicOr(a.err, kDevErrBadIndex);
        return 0;
    }
    return static_cast<int64_t>(blk) * a.block_stride + static_cast<int64_t>(pos % a.block_rows) * a.cache_row_stride;
}

template <bool kInterleaved, typename QT, typename CT>
__global__ void __launch_bounds__(kRopeThreads) rope_kv_kernel(const __grid_constant__ RopeArgs a) {
    // The attention call that follows may launch now; it waits for this grid to finish before reading.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // Launched with programmatic dependent launch: no global access before the previous kernel's writes are
    // complete and visible.
    asm volatile("griddepcontrol.wait;" ::: "memory");
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
    bool row_ok = true;
    const int64_t cache_off = a.n_kv_heads > 0 ? cache_row_offset(a, seq, pos, row_ok) : 0;
    CT* kc = static_cast<CT*>(a.k_cache) + cache_off;
    CT* vc = static_cast<CT*>(a.v_cache) + cache_off;
    for (int idx = tid; idx < rows * a.half; idx += kRopeThreads) {
        const int r = idx / a.half, i = idx - r * a.half;
        if (r >= a.n_heads && !row_ok) break;  // k / v rows of an unwritable cache row
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

constexpr int kVecThreads = 256;
constexpr int kVecTokens = 32;  // most tokens per CTA of the vector kernel
constexpr int kVecTokensDefault = 8;  // measured best at the config-2 shape (4, 16 and 32 are slower)
constexpr int kVecBatch = 4;   // groups of 4 pairs a thread loads before it rotates / stores them

// Four pairs i0..i0+3 of one head row: a[j] = x[ia(i0+j)], b[j] = x[ib(i0+j)].
template <bool kInterleaved>
__device__ __forceinline__ void load4(const float* p, int i0, int half, float (&a)[4], float (&b)[4]) {
    if (kInterleaved) {
        const float4 u = *reinterpret_cast<const float4*>(p + 2 * i0), w = *reinterpret_cast<const float4*>(p + 2 * i0 + 4);
        a[0] = u.x; b[0] = u.y; a[1] = u.z; b[1] = u.w; a[2] = w.x; b[2] = w.y; a[3] = w.z; b[3] = w.w;
    } else {
        const float4 u = *reinterpret_cast<const float4*>(p + i0), w = *reinterpret_cast<const float4*>(p + half + i0);
        a[0] = u.x; a[1] = u.y; a[2] = u.z; a[3] = u.w; b[0] = w.x; b[1] = w.y; b[2] = w.z; b[3] = w.w;
    }
}
template <bool kInterleaved>
__device__ __forceinline__ void load4(const __half* p, int i0, int half, float (&a)[4], float (&b)[4]) {
    if (kInterleaved) {
        const uint4 u = *reinterpret_cast<const uint4*>(p + 2 * i0);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float2 f = __half22float2(h[j]);
            a[j] = f.x;
            b[j] = f.y;
        }
    } else {
        const uint2 u = *reinterpret_cast<const uint2*>(p + i0), w = *reinterpret_cast<const uint2*>(p + half + i0);
        const __half2* hu = reinterpret_cast<const __half2*>(&u);
        const __half2* hw = reinterpret_cast<const __half2*>(&w);
        const float2 u0 = __half22float2(hu[0]), u1 = __half22float2(hu[1]);
        const float2 w0 = __half22float2(hw[0]), w1 = __half22float2(hw[1]);
        a[0] = u0.x; a[1] = u0.y; a[2] = u1.x; a[3] = u1.y; b[0] = w0.x; b[1] = w0.y; b[2] = w1.x; b[3] = w1.y;
    }
}
template <bool kInterleaved>
__device__ __forceinline__ void store4(float* p, int i0, int half, const float (&a)[4], const float (&b)[4]) {
    if (kInterleaved) {
        *reinterpret_cast<float4*>(p + 2 * i0) = make_float4(a[0], b[0], a[1], b[1]);
        *reinterpret_cast<float4*>(p + 2 * i0 + 4) = make_float4(a[2], b[2], a[3], b[3]);
    } else {
        *reinterpret_cast<float4*>(p + i0) = make_float4(a[0], a[1], a[2], a[3]);
        *reinterpret_cast<float4*>(p + half + i0) = make_float4(b[0], b[1], b[2], b[3]);
    }
}
template <bool kInterleaved>
__device__ __forceinline__ void store4(__half* p, int i0, int half, const float (&a)[4], const float (&b)[4]) {
    if (kInterleaved) {
        __half2 h[4];
#pragma unroll
        for (int j = 0; j < 4; j++) h[j] = __floats2half2_rn(a[j], b[j]);
        *reinterpret_cast<uint4*>(p + 2 * i0) = *reinterpret_cast<const uint4*>(h);
    } else {
        __half2 u[2] = {__floats2half2_rn(a[0], a[1]), __floats2half2_rn(a[2], a[3])};
        __half2 w[2] = {__floats2half2_rn(b[0], b[1]), __floats2half2_rn(b[2], b[3])};
        *reinterpret_cast<uint2*>(p + i0) = *reinterpret_cast<const uint2*>(u);
        *reinterpret_cast<uint2*>(p + half + i0) = *reinterpret_cast<const uint2*>(w);
    }
}

// Group `idx` (4 pairs) of the CTA's tokens: which token, row and pairs, and where that row lives.
template <typename QT, typename CT>
struct VecItem {
    bool valid, is_q, is_k, dst_ok;
    int tt, i0;
    const float* src;  // k or v row (f32)
    QT* qrow;          // query row (rotated in place)
    CT* dst;           // cache row
};

template <bool kDst, typename QT, typename CT>
__device__ __forceinline__ VecItem<QT, CT> vec_item(const RopeArgs& a, int seq, int t0, int pos0, int ntok, int idx) {
    VecItem<QT, CT> it;
    const int d = 2 * a.half, quads = a.half / 4;
    const int per_tok = (a.n_heads + 2 * a.n_kv_heads) * quads;
    it.valid = idx < ntok * per_tok;
    const int tt = it.valid ? idx / per_tok : 0, rem = it.valid ? idx - tt * per_tok : 0;
    const int r = rem / quads;
    it.tt = tt;
    it.i0 = 4 * (rem - r * quads);
    const int t = t0 + tt;
    it.is_q = r < a.n_heads;
    it.is_k = !it.is_q && r < a.n_heads + a.n_kv_heads;
    const int h = it.is_q ? 0 : (it.is_k ? r - a.n_heads : r - a.n_heads - a.n_kv_heads);
    it.qrow = static_cast<QT*>(a.q) + seq * a.q_seq_stride + static_cast<int64_t>(t) * a.q_token_stride + r * d;
    it.src = (it.is_k ? a.k : a.v) + seq * a.kv_seq_stride + static_cast<int64_t>(t) * a.kv_token_stride + h * d;
    it.dst_ok = true;
    it.dst = static_cast<CT*>(it.is_k ? a.k_cache : a.v_cache) + h * d;
    if (kDst && it.valid && !it.is_q) it.dst += cache_row_offset(a, seq, pos0 + tt, it.dst_ok);
    return it;
}

template <bool kInterleaved, typename QT, typename CT>
__device__ __forceinline__ void vec_load(const RopeArgs& a, int seq, int t0, int pos0, int ntok, int idx,
                                         float (&x0)[4], float (&x1)[4]) {
    const VecItem<QT, CT> it = vec_item<false, QT, CT>(a, seq, t0, pos0, ntok, idx);
    if (!it.valid) return;
    if (it.is_q) load4<kInterleaved>(it.qrow, it.i0, a.half, x0, x1);
    else load4<kInterleaved>(it.src, it.i0, a.half, x0, x1);
}

template <bool kInterleaved, typename QT, typename CT>
__device__ __forceinline__ void vec_store(const RopeArgs& a, int seq, int t0, int pos0, int ntok, int idx,
                                          const float2* cs, float (&x0)[4], float (&x1)[4]) {
    const VecItem<QT, CT> it = vec_item<true, QT, CT>(a, seq, t0, pos0, ntok, idx);
    if (!it.valid) return;
    if (it.is_q || it.is_k) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float2 w = cs[it.tt * a.half + it.i0 + j];
            const float y0 = __fsub_rn(__fmul_rn(x0[j], w.x), __fmul_rn(x1[j], w.y));
            x1[j] = __fadd_rn(__fmul_rn(x0[j], w.y), __fmul_rn(x1[j], w.x));
            x0[j] = y0;
        }
    }
    if (it.is_q) store4<kInterleaved>(it.qrow, it.i0, a.half, x0, x1);
    else if (it.dst_ok) store4<kInterleaved>(it.dst, it.i0, a.half, x0, x1);
}

template <bool kInterleaved, typename QT, typename CT>
__global__ void __launch_bounds__(kVecThreads, 4) rope_kv_vec_kernel(const __grid_constant__ RopeArgs a) {
    // The attention call that follows may launch now; it waits for this grid to finish before reading.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    extern __shared__ float2 cs[];  // [tpc][half] (cos, sin)
    const int t0 = blockIdx.x * a.tpc, seq = blockIdx.y, tid = threadIdx.x;
    const int ntok = min(a.tpc, a.tokens - t0);
    const int total = ntok * (a.n_heads + 2 * a.n_kv_heads) * (a.half / 4);
    constexpr int kStride = kVecThreads * kVecBatch;
    const auto table = [&](int pos0) {
        for (int j = tid; j < ntok * a.half; j += kVecThreads) {
            const int tt = j / a.half, i = j - tt * a.half;
            double s, c;
            sincos(static_cast<double>(pos0 + tt) * a.freq[i], &s, &c);
            cs[j] = make_float2(static_cast<float>(c), static_cast<float>(s));
        }
    };
    // A uniform start position needs no global data: the (cos, sin) table is computed while the previous kernel
    // drains. Launched with programmatic dependent launch, the CTA then waits for that kernel's writes before its
    // first global access.
    const bool uniform = a.positions == nullptr;
    if (uniform) table(a.start + t0);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int pos0 = (uniform ? a.start : a.positions[seq]) + t0;

    // every thread's first batch of loads is in flight while a per-sequence (cos, sin) table is computed
    float x0[kVecBatch][4], x1[kVecBatch][4];
#pragma unroll
    for (int b = 0; b < kVecBatch; b++)
        vec_load<kInterleaved, QT, CT>(a, seq, t0, pos0, ntok, tid + b * kVecThreads, x0[b], x1[b]);
    if (!uniform) table(pos0);
    __syncthreads();  // every thread of the CTA reaches this once
#pragma unroll
    for (int b = 0; b < kVecBatch; b++)
        vec_store<kInterleaved, QT, CT>(a, seq, t0, pos0, ntok, tid + b * kVecThreads, cs, x0[b], x1[b]);
    for (int base = tid + kStride; base < total; base += kStride) {
#pragma unroll
        for (int b = 0; b < kVecBatch; b++)
            vec_load<kInterleaved, QT, CT>(a, seq, t0, pos0, ntok, base + b * kVecThreads, x0[b], x1[b]);
#pragma unroll
        for (int b = 0; b < kVecBatch; b++)
            vec_store<kInterleaved, QT, CT>(a, seq, t0, pos0, ntok, base + b * kVecThreads, cs, x0[b], x1[b]);
    }
}

// 16-byte vectors: head_dim % 8 == 0, tensor pointers 16-byte aligned, every stride a multiple of 8 elements.
bool vector_ok(const alpaca_rope_desc& d) {
    auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    if (d.head_dim % 8) return false;
    if (d.n_heads > 0 && (!al16(d.q) || d.q_token_stride % 8 || d.q_seq_stride % 8)) return false;
    if (d.n_kv_heads > 0 && (!al16(d.k) || !al16(d.v) || !al16(d.k_cache) || !al16(d.v_cache) ||
                             d.kv_token_stride % 8 || d.kv_seq_stride % 8 || d.cache_row_stride % 8 ||
                             d.cache_seq_stride % 8 || (d.block_table && d.block_stride % 8)))
        return false;
    return true;
}

template <bool kInterleaved, typename QT, typename CT>
cudaError_t launch_qc(const RopeArgs& a, const alpaca_rope_desc& d, cudaStream_t s) {
    // Programmatic dependent launch: the CTAs may become resident while the previous kernel on the stream drains
    // (both kernels wait in griddepcontrol.wait before touching global memory).
    cudaLaunchConfig_t cfg = {};
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    if (vector_ok(d)) {
        cfg.gridDim = dim3((d.tokens + a.tpc - 1) / a.tpc, d.n_seqs, 1);
        cfg.blockDim = dim3(kVecThreads, 1, 1);
        cfg.dynamicSmemBytes = sizeof(float2) * a.tpc * a.half;  // <= 32 KB
        return cudaLaunchKernelEx(&cfg, rope_kv_vec_kernel<kInterleaved, QT, CT>, a);
    }
    cfg.gridDim = dim3(d.tokens, d.n_seqs, 1);
    cfg.blockDim = dim3(kRopeThreads, 1, 1);
    return cudaLaunchKernelEx(&cfg, rope_kv_kernel<kInterleaved, QT, CT>, a);
}

template <bool kInterleaved, typename QT>
cudaError_t launch_q(const RopeArgs& a, const alpaca_rope_desc& d, cudaStream_t s) {
    return d.cache_dtype == ALPACA_F16 ? launch_qc<kInterleaved, QT, __half>(a, d, s)
                                       : launch_qc<kInterleaved, QT, float>(a, d, s);
}

template <bool kInterleaved>
cudaError_t launch_i(const RopeArgs& a, const alpaca_rope_desc& d, cudaStream_t s) {
    return d.q_dtype == ALPACA_F16 ? launch_q<kInterleaved, __half>(a, d, s) : launch_q<kInterleaved, float>(a, d, s);
}

// Tokens per CTA of the vector kernel: ALPACA_ROPE_TPC (1 .. 32), default 8.
int rope_tokens_per_cta() {
    static const int v = [] {
        const char* e = std::getenv("ALPACA_ROPE_TPC");
        const int x = e ? std::atoi(e) : 0;
        return (x >= 1 && x <= kVecTokens) ? x : kVecTokensDefault;
    }();
    return v;
}

}  // namespace

int rope_max_head_dim() { return 2 * kRopeMaxPairs; }

cudaError_t launch_rope_kv(const alpaca_rope_desc& d, unsigned* err, cudaStream_t s) {
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
    a.tokens = d.tokens;
    a.tpc = rope_tokens_per_cta();
    a.block_table = d.block_table;
    a.block_rows = d.block_rows;
    a.max_blocks = d.max_blocks;
    a.pool_blocks = d.pool_blocks;
    a.block_stride = d.block_stride;
    a.cache_rows = d.cache_rows;
    a.err = err;
    const double theta = static_cast<double>(d.theta);
    for (int i = 0; i < kRopeMaxPairs; i++)
        a.freq[i] = i < a.half ? std::pow(theta, -2.0 * static_cast<double>(i) / static_cast<double>(d.head_dim)) : 0.0;
    return d.interleaved ? launch_i<true>(a, d, s) : launch_i<false>(a, d, s);
}

}  // namespace alpaca
