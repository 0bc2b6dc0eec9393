// decode_proj.cu — fused single-token projections of a decode step: optional RMSNorm of the input row, then up to
// three weight matrices applied to it (Q / K / V in one launch), or the SwiGLU gate + up pair, or one matrix with the
// result added to the output (the out- and down-projections with their residual). Same job as alpaca.swift's
// dec_f16 / dec_q8_0 / dec_q4_0 (Sources/AlpacaMetal/Kernels/decode_fused.metal:32-122), dispatched by
// KernelEncoder.decodeQKV / decodeProjection / decodeGateUp (Sources/AlpacaMetal/Backend/KernelEncoder.swift:
// 386-400); weights f16 or GGUF q8_0 / q4_0.
//
// HBM-bound (every weight byte is read once per launch; the input rows are a few KB), so the design is about bytes in
// flight and cheap decoding:
//   * each CTA (8 warps) stages the call's input rows, RMS-normalised when asked, in shared memory once; one warp
//     computes one output row at a time, lanes striding over the row's 16-byte f16 chunks or GGUF blocks;
//   * quantised blocks (34 / 18 bytes, 2-byte aligned) are read with aligned 4-byte loads and realigned with funnel
//     shifts; int8 and 4-bit values become floats through a byte permute into 2^23 + v (no conversion instructions);
//   * for quantised formats the staged row is stored transposed per block (element j of block b at
//     j * (blocks + 1) + b), so the 32 lanes of a warp, which work on 32 consecutive blocks, read 32 consecutive words
//     of shared memory, and the staging writes (consecutive elements, one block apart) fall in 32 different banks
//     (without the pad word the stride is a multiple of 32 words: a 32-way conflict on every staging store, which
//     held q8_0 projections near 0.4 TB/s);
//   * up to 4 input rows (tokens of a batched decode step) share every weight load; more rows take more passes;
//   * single-token q8_0 / q4_0 calls run on the tensor cores instead (proj_mma_kernel): the input row as exact int8
//     digit planes against the weight quants in mma.sync m16n8k32 (s8), the block scales applied to the exact int32
//     sums.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace alpaca {
namespace {

constexpr int kProjThreads = 256;
constexpr int kProjWarps = kProjThreads / 32;
constexpr int kProjMaxTokens = 4;
constexpr size_t kProjSmemBudget = 160 * 1024;  // staged input rows per CTA

struct ProjArgs {
    const uint8_t* w[3];
    const uint8_t* w_end[3];  // one past each matrix (bounds of the 4-byte loads at its end)
    int rows[3];
    int total_rows;          // rows the warps iterate over (SiLU: rows[0])
    int k, units;            // input width; 16-byte chunks (f16) or blocks (quantised) per row
    int64_t row_bytes;
    unsigned flags;
    float eps;
    const float* x;
    int64_t x_stride;
    const float* g;
    float* y[3];
    int64_t y_stride[3];
    int n_tokens;
    int wpr;       // warps per row (1, 2, 4 or 8): each takes every wpr-th group of 32 units of the row
    int prefetch;  // bulk L2 prefetch of the CTA's weight rows at the start
};

__device__ __forceinline__ uint32_t ldg32(const uint8_t* p) { return __ldg(reinterpret_cast<const unsigned int*>(p)); }
__device__ __forceinline__ uint32_t ldg16(const uint8_t* p) {
    return __ldg(reinterpret_cast<const unsigned short*>(p));
}

// Four signed bytes -> floats: byte v + 128 placed in the low mantissa bits of 2^23, minus 2^23 + 128.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float (&f)[4]) {
    const uint32_t u = w ^ 0x80808080u;
#pragma unroll
    for (int e = 0; e < 4; e++) f[e] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540u + e)) - 8388736.0f;
}
// Four bytes holding 4-bit values n -> floats n - 8.
__device__ __forceinline__ void n4x4_to_f32(uint32_t w, float (&f)[4]) {
#pragma unroll
    for (int e = 0; e < 4; e++) f[e] = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u + e)) - 8388616.0f;
}

// The 32 bytes after the 2-byte scale of a q8_0 block at p (2-byte aligned), as 8 words, and the scale.
__device__ __forceinline__ float q8_block(const uint8_t* p, const uint8_t* end, uint32_t (&q)[8]) {
    if (reinterpret_cast<uintptr_t>(p) & 2u) {  // scale in the high half of the word before p + 2
        const uint8_t* b = p - 2;
        const uint32_t w0 = ldg32(b);
#pragma unroll
        for (int i = 0; i < 8; i++) q[i] = ldg32(b + 4 + 4 * i);
        return __half2float(__ushort_as_half(static_cast<unsigned short>(w0 >> 16)));
    }
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 8; i++) w[i] = ldg32(p + 4 * i);
    w[8] = (p + 36 <= end) ? ldg32(p + 32) : ldg16(p + 32);  // the block may end the matrix
#pragma unroll
    for (int i = 0; i < 8; i++) q[i] = __funnelshift_r(w[i], w[i + 1], 16);
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w[0] & 0xFFFFu)));
}

// The 16 bytes of nibbles after the scale of a q4_0 block at p (2-byte aligned), as 4 words, and the scale.
__device__ __forceinline__ float q4_block(const uint8_t* p, const uint8_t* end, uint32_t (&q)[4]) {
    if (reinterpret_cast<uintptr_t>(p) & 2u) {
        const uint8_t* b = p - 2;
        const uint32_t w0 = ldg32(b);
#pragma unroll
        for (int i = 0; i < 4; i++) q[i] = ldg32(b + 4 + 4 * i);
        return __half2float(__ushort_as_half(static_cast<unsigned short>(w0 >> 16)));
    }
    uint32_t w[5];
#pragma unroll
    for (int i = 0; i < 4; i++) w[i] = ldg32(p + 4 * i);
    w[4] = (p + 20 <= end) ? ldg32(p + 16) : ldg16(p + 16);
#pragma unroll
    for (int i = 0; i < 4; i++) q[i] = __funnelshift_r(w[i], w[i + 1], 16);
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w[0] & 0xFFFFu)));
}

// Shared-memory index of element i of a staged row: plain for f16, transposed per 32-element block otherwise, each
// of the 32 element planes padded by one word.
template <int F>
__device__ __forceinline__ int xs_index(int i, int units) {
    if constexpr (F == 0) return i;
    return (i & 31) * (units + 1) + (i >> 5);
}
// Floats of one staged row.
template <int F>
__host__ __device__ __forceinline__ int xs_row(int k, int units) {
    return F == 0 ? k : 32 * (units + 1);
}

// One unit of a weight row in registers: a 16-byte f16 chunk, or a q8_0 / q4_0 block's scale and quant words.
template <int F>
struct UnitRegs {
    uint32_t q[F == 0 ? 4 : (F == 1 ? 8 : 4)];
    float d;
};

template <int F>
__device__ __forceinline__ void load_unit(const uint8_t* rowp, const uint8_t* end, int u, UnitRegs<F>& r) {
    if constexpr (F == 0) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(rowp) + u);
        r.q[0] = w.x;
        r.q[1] = w.y;
        r.q[2] = w.z;
        r.q[3] = w.w;
        r.d = 1.f;
    } else if constexpr (F == 1) {
        r.d = q8_block(rowp + static_cast<int64_t>(u) * 34, end, r.q);
    } else {
        r.d = q4_block(rowp + static_cast<int64_t>(u) * 18, end, r.q);
    }
}

// acc[t] += unit u of the row . xn_t
template <int F, int TP>
__device__ __forceinline__ void dot_unit(const UnitRegs<F>& r, int u, const float* xs, int XR, int P, float (&acc)[TP]) {
    if constexpr (F == 0) {
        float wf[8];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&r.q[i]));
            wf[2 * i] = f.x;
            wf[2 * i + 1] = f.y;
        }
#pragma unroll
        for (int t = 0; t < TP; t++) {
            const float4 x0 = *reinterpret_cast<const float4*>(xs + t * XR + 8 * u);
            const float4 x1 = *reinterpret_cast<const float4*>(xs + t * XR + 8 * u + 4);
            float s = acc[t];
            s = fmaf(wf[0], x0.x, s);
            s = fmaf(wf[1], x0.y, s);
            s = fmaf(wf[2], x0.z, s);
            s = fmaf(wf[3], x0.w, s);
            s = fmaf(wf[4], x1.x, s);
            s = fmaf(wf[5], x1.y, s);
            s = fmaf(wf[6], x1.z, s);
            s = fmaf(wf[7], x1.w, s);
            acc[t] = s;
        }
    } else {
        float s[TP];
#pragma unroll
        for (int t = 0; t < TP; t++) s[t] = 0.f;
        const float* xb = xs + u;  // element j of this block at xb[j * P] (+ t * XR)
        if constexpr (F == 1) {
#pragma unroll
            for (int i = 0; i < 8; i++) {
                float f[4];
                i8x4_to_f32(r.q[i], f);
#pragma unroll
                for (int e = 0; e < 4; e++)
#pragma unroll
                    for (int t = 0; t < TP; t++) s[t] = fmaf(f[e], xb[t * XR + (4 * i + e) * P], s[t]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                float lo[4], hi[4];
                n4x4_to_f32(r.q[i] & 0x0F0F0F0Fu, lo);
                n4x4_to_f32((r.q[i] >> 4) & 0x0F0F0F0Fu, hi);
#pragma unroll
                for (int e = 0; e < 4; e++)
#pragma unroll
                    for (int t = 0; t < TP; t++) {
                        s[t] = fmaf(lo[e], xb[t * XR + (4 * i + e) * P], s[t]);
                        s[t] = fmaf(hi[e], xb[t * XR + (4 * i + e + 16) * P], s[t]);
                    }
            }
        }
#pragma unroll
        for (int t = 0; t < TP; t++) acc[t] = fmaf(r.d, s[t], acc[t]);
    }
}

// This warp's share of NR rows at once (row n's bytes at rowp[n]; a null rowp skips it) against the TP staged rows:
// acc[n][t] = the sum over units u = base, base + S, ... of W[row n] . xn_t. Every lane ends with the warp's sums.
// Two units of each row per lane are loaded before any is used, so a warp keeps 2 NR loads (or blocks) in flight.
template <int F, int TP, int NR>
__device__ __forceinline__ void rows_dot(const ProjArgs& a, const uint8_t* const (&rowp)[NR],
                                         const uint8_t* const (&end)[NR], const float* xs, int base, int S,
                                         float (&acc)[NR][TP]) {
#pragma unroll
    for (int n = 0; n < NR; n++)
#pragma unroll
        for (int t = 0; t < TP; t++) acc[n][t] = 0.f;
    const int U = a.units, XR = xs_row<F>(a.k, U), P = U + 1;
    for (int u0 = base; u0 < U; u0 += 2 * S) {
        UnitRegs<F> r[NR][2];
#pragma unroll
        for (int n = 0; n < NR; n++)
#pragma unroll
            for (int h = 0; h < 2; h++)
                if (rowp[n] && u0 + h * S < U) load_unit<F>(rowp[n], end[n], u0 + h * S, r[n][h]);
#pragma unroll
        for (int n = 0; n < NR; n++)
#pragma unroll
            for (int h = 0; h < 2; h++)
                if (rowp[n] && u0 + h * S < U) dot_unit<F, TP>(r[n][h], u0 + h * S, xs, XR, P, acc[n]);
    }
#pragma unroll
    for (int n = 0; n < NR; n++)
#pragma unroll
        for (int t = 0; t < TP; t++)
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) acc[n][t] += __shfl_xor_sync(0xffffffffu, acc[n][t], o);
}

// L2 prefetch of bytes [p, p + n) of a matrix (16-byte aligned start, whole 16-byte units inside [p, end)).
__device__ __forceinline__ void prefetch_l2(const uint8_t* p, int64_t n, const uint8_t* end) {
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(p) & ~uintptr_t(15);
    const uintptr_t a1 = std::min(reinterpret_cast<uintptr_t>(p + n) + 15, reinterpret_cast<uintptr_t>(end)) &
                         ~uintptr_t(15);
    for (uintptr_t a = a0; a < a1; a += (1u << 20)) {
        const uint32_t len = static_cast<uint32_t>(std::min<uintptr_t>(a1 - a, 1u << 20));
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(len) : "memory");
    }
}

// grid (row CTAs, token passes), 256 threads; dynamic shared memory TP staged rows. One staged row: 64 registers per
// thread, 4 CTAs (32 warps) per SM, so each SM keeps enough weight bytes in flight (at 110 registers only 2 CTAs fit
// and a q8_0 gate + up launch ran at 1.2 TB/s); more staged rows need the registers of their accumulators.
template <int F, int TP>
__global__ void __launch_bounds__(kProjThreads, TP == 1 ? 4 : 2) proj_kernel(const ProjArgs a) {
    extern __shared__ __align__(16) float xs[];
    __shared__ float red[kProjWarps][TP];
    __shared__ float scale[TP];
    // The next stream-ordered kernel may launch now; it waits for this grid before touching memory.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const bool silu = (a.flags & ALPACA_PROJ_SILU) != 0;
    const int RPC = (kProjWarps / a.wpr) * (silu ? 1 : 2);  // output rows per CTA pass
    if (a.prefetch && threadIdx.x == 0 && blockIdx.y == 0) {
        // Start the DRAM reads of this CTA's weight rows into L2 at once, while the previous kernel drains and the
        // input rows are staged (a prefetch changes no memory, so it may precede the dependency wait).
        for (int r0 = blockIdx.x * RPC; r0 < a.total_rows; r0 += gridDim.x * RPC) {
            const int r1 = min(r0 + RPC, a.total_rows);
            if (silu) {
                for (int m = 0; m < 2; m++) prefetch_l2(a.w[m] + r0 * a.row_bytes, (r1 - r0) * a.row_bytes, a.w_end[m]);
                continue;
            }
            for (int m = 0, base = 0; m < 3; base += a.rows[m], m++) {
                const int lo = max(r0, base), hi = min(r1, base + a.rows[m]);
                if (lo < hi) prefetch_l2(a.w[m] + (lo - base) * a.row_bytes, (hi - lo) * a.row_bytes, a.w_end[m]);
            }
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");  // x (and y when adding) come from the previous kernel
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.y * TP;
    const int nt = min(TP, a.n_tokens - t0);
    const int k = a.k, XR = xs_row<F>(k, a.units);

    // Stage the input rows (and their sums of squares).
    float ss[TP];
#pragma unroll
    for (int t = 0; t < TP; t++) ss[t] = 0.f;
    for (int i = tid; i < k; i += kProjThreads) {
#pragma unroll
        for (int t = 0; t < TP; t++) {
            const float v = t < nt ? a.x[(t0 + t) * a.x_stride + i] : 0.f;
            xs[t * XR + xs_index<F>(i, a.units)] = v;
            ss[t] = fmaf(v, v, ss[t]);
        }
    }
    if (a.flags & ALPACA_PROJ_NORM) {
#pragma unroll
        for (int t = 0; t < TP; t++) {
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) ss[t] += __shfl_xor_sync(0xffffffffu, ss[t], o);
            if (lane == 0) red[warp][t] = ss[t];
        }
        __syncthreads();
        if (tid < TP) {
            float tot = 0.f;
#pragma unroll
            for (int w = 0; w < kProjWarps; w++) tot += red[w][tid];
            scale[tid] = 1.0f / sqrtf(tot / static_cast<float>(k) + a.eps);  // CPUOps.rmsNorm's scale
        }
        __syncthreads();
        for (int i = tid; i < k; i += kProjThreads) {
            const float gi = a.g[i];
#pragma unroll
            for (int t = 0; t < TP; t++) {
                float* p = xs + t * XR + xs_index<F>(i, a.units);
                *p = (*p * scale[t]) * gi;  // x * scale * w, in that order
            }
        }
    }
    __syncthreads();

    // Warps [slot * wpr, slot * wpr + wpr) share their rows: each takes every wpr-th group of 32 units, and the first
    // of them adds the others' sums from shared memory (double-buffered by pass, one barrier per pass). A warp works
    // on two rows at once: the gate and up rows of one output (SiLU), or two consecutive output rows.
    __shared__ float part[2][kProjWarps][2][TP];
    const int WPR = a.wpr, slot = warp / WPR, piece = warp - slot * WPR;
    const int RPW = silu ? 1 : 2;  // output rows per warp slot
    int buf = 0;
    for (int r0 = blockIdx.x * RPC; r0 < a.total_rows; r0 += gridDim.x * RPC, buf ^= 1) {  // uniform per CTA
        int m[2] = {0, 0}, lr[2];
        const uint8_t* rp[2] = {nullptr, nullptr};
        const uint8_t* re[2] = {nullptr, nullptr};
#pragma unroll
        for (int n = 0; n < 2; n++) {
            const int r = r0 + slot * RPW + (silu ? 0 : n);
            lr[n] = r;
            if (r >= a.total_rows) continue;
            if (silu) {
                m[n] = n;  // gate (W0) and up (W1) rows of output r
            } else if (lr[n] >= a.rows[0]) {
                lr[n] -= a.rows[0];
                m[n] = 1;
                if (lr[n] >= a.rows[1]) {
                    lr[n] -= a.rows[1];
                    m[n] = 2;
                }
            }
            rp[n] = a.w[m[n]] + lr[n] * a.row_bytes;
            re[n] = a.w_end[m[n]];
        }
        float acc[2][TP];
        rows_dot<F, TP, 2>(a, rp, re, xs, 32 * piece + lane, 32 * WPR, acc);
        if (WPR > 1) {
            if (lane == 0)
#pragma unroll
                for (int n = 0; n < 2; n++)
#pragma unroll
                    for (int t = 0; t < TP; t++) part[buf][warp][n][t] = acc[n][t];
            __syncthreads();
            if (piece == 0)
#pragma unroll
                for (int n = 0; n < 2; n++)
#pragma unroll
                    for (int t = 0; t < TP; t++) {
                        float sum = 0.f;
                        for (int p = 0; p < WPR; p++) sum += part[buf][warp + p][n][t];
                        acc[n][t] = sum;
                    }
        }
        if (piece != 0 || lane != 0) continue;
        if (silu) {
            if (!rp[0]) continue;
#pragma unroll
            for (int t = 0; t < TP; t++)
                if (t < nt) {
                    const float gt = acc[0][t];
                    a.y[0][(t0 + t) * a.y_stride[0] + lr[0]] = (gt / (1.0f + expf(-gt))) * acc[1][t];
                }
            continue;
        }
#pragma unroll
        for (int n = 0; n < 2; n++) {
            if (!rp[n]) continue;
#pragma unroll
            for (int t = 0; t < TP; t++)
                if (t < nt) {
                    float* yp = a.y[m[n]] + (t0 + t) * a.y_stride[m[n]] + lr[n];
                    *yp = ((a.flags & ALPACA_PROJ_ADD) ? *yp : 0.f) + acc[n][t];
                }
        }
    }
}

// ---- single-token path: the input slice each lane needs lives in registers.
// A lane always multiplies the same units of every row (units piece*32 + lane + j*32*wpr), so after the CTA has
// staged (and normalised) the input row once, each lane copies its UPL units' elements into registers and the row loop
// is weight loads and FMAs only: no shared-memory reads in the inner loop. Each warp slot works on RR rows per pass, all
// their loads issued before any is used; partial sums of a row's wpr pieces meet in shared memory once per pass.
constexpr int kRegRows = 2;  // rows per warp slot per pass (SiLU: 1 output, its gate and up rows)

template <int F>
struct RegGeo {
    static constexpr int E = F == 0 ? 8 : 32;   // elements per unit (16-byte chunk or block)
    static constexpr int UPL = F == 0 ? 4 : 1;  // units per lane
};

template <int F>
__global__ void __launch_bounds__(kProjThreads, 3) proj_reg_kernel(const ProjArgs a) {
    using G = RegGeo<F>;
    constexpr int E = G::E, UPL = G::UPL;
    extern __shared__ __align__(16) float xs[];  // the staged input row [k]
    __shared__ float red[kProjWarps];
    __shared__ float scale;
    __shared__ float part[2][kProjWarps][kRegRows];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const bool silu = (a.flags & ALPACA_PROJ_SILU) != 0;
    const int WPR = a.wpr, SLOTS = kProjWarps / WPR;
    const int RPC = SLOTS * (silu ? kRegRows / 2 : kRegRows);  // output rows per CTA pass
    if (a.prefetch && threadIdx.x == 0) {
        for (int r0 = blockIdx.x * RPC; r0 < a.total_rows; r0 += gridDim.x * RPC) {
            const int r1 = min(r0 + RPC, a.total_rows);
            if (silu) {
                for (int m = 0; m < 2; m++) prefetch_l2(a.w[m] + r0 * a.row_bytes, (r1 - r0) * a.row_bytes, a.w_end[m]);
                continue;
            }
            for (int m = 0, base = 0; m < 3; base += a.rows[m], m++) {
                const int lo = max(r0, base), hi = min(r1, base + a.rows[m]);
                if (lo < hi) prefetch_l2(a.w[m] + (lo - base) * a.row_bytes, (hi - lo) * a.row_bytes, a.w_end[m]);
            }
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, k = a.k, U = a.units;

    // stage the row (sum of squares alongside), normalise in place when asked
    float ss = 0.f;
    for (int i = tid; i < k; i += kProjThreads) {
        const float v = a.x[i];
        xs[i] = v;
        ss = fmaf(v, v, ss);
    }
    if (a.flags & ALPACA_PROJ_NORM) {
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (tid == 0) {
            float tot = 0.f;
#pragma unroll
            for (int w = 0; w < kProjWarps; w++) tot += red[w];
            scale = 1.0f / sqrtf(tot / static_cast<float>(k) + a.eps);  // CPUOps.rmsNorm's scale
        }
        __syncthreads();
        for (int i = tid; i < k; i += kProjThreads) xs[i] = (xs[i] * scale) * a.g[i];  // x * scale * w
    }
    __syncthreads();

    // this lane's units and their input elements
    const int slot = warp / WPR, piece = warp - slot * WPR;
    int uidx[UPL];
    float xr[UPL][E];
#pragma unroll
    for (int j = 0; j < UPL; j++) {
        uidx[j] = piece * 32 + lane + j * 32 * WPR;
        const bool in = uidx[j] < U;
#pragma unroll
        for (int e = 0; e < E; e += 4) {
            const float4 v = in ? *reinterpret_cast<const float4*>(xs + uidx[j] * E + e) : make_float4(0.f, 0.f, 0.f, 0.f);
            xr[j][e] = v.x;
            xr[j][e + 1] = v.y;
            xr[j][e + 2] = v.z;
            xr[j][e + 3] = v.w;
        }
    }

    int buf = 0;
    for (int r0 = blockIdx.x * RPC; r0 < a.total_rows; r0 += gridDim.x * RPC, buf ^= 1) {  // uniform per CTA
        // the slot's rows: SiLU: gate / up of outputs o0, o0 + 1; otherwise kRegRows consecutive outputs
        const uint8_t* rp[kRegRows];
        const uint8_t* re[kRegRows];
#pragma unroll
        for (int n = 0; n < kRegRows; n++) {
            int r, m = 0;
            if (silu) {
                r = r0 + slot * (kRegRows / 2) + n / 2;
                m = n & 1;
            } else {
                r = r0 + slot * kRegRows + n;
            }
            rp[n] = nullptr;
            re[n] = nullptr;
            if (r >= a.total_rows) continue;
            int lr = r;
            if (!silu && lr >= a.rows[0]) {
                lr -= a.rows[0];
                m = 1;
                if (lr >= a.rows[1]) {
                    lr -= a.rows[1];
                    m = 2;
                }
            }
            rp[n] = a.w[m] + lr * a.row_bytes;
            re[n] = a.w_end[m];
        }
        UnitRegs<F> w[kRegRows][UPL];
#pragma unroll
        for (int n = 0; n < kRegRows; n++)
#pragma unroll
            for (int j = 0; j < UPL; j++)
                if (rp[n] && uidx[j] < U) load_unit<F>(rp[n], re[n], uidx[j], w[n][j]);
        float acc[kRegRows];
#pragma unroll
        for (int n = 0; n < kRegRows; n++) {
            float sacc = 0.f;
#pragma unroll
            for (int j = 0; j < UPL; j++) {
                if (!rp[n] || uidx[j] >= U) continue;
                if constexpr (F == 0) {
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[n][j].q[i]));
                        sacc = fmaf(f.x, xr[j][2 * i], sacc);
                        sacc = fmaf(f.y, xr[j][2 * i + 1], sacc);
                    }
                } else if constexpr (F == 1) {
                    float sb = 0.f;
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        float f[4];
                        i8x4_to_f32(w[n][j].q[i], f);
#pragma unroll
                        for (int e = 0; e < 4; e++) sb = fmaf(f[e], xr[j][4 * i + e], sb);
                    }
                    sacc = fmaf(w[n][j].d, sb, sacc);
                } else {
                    float sb = 0.f;
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        float lo[4], hi[4];
                        n4x4_to_f32(w[n][j].q[i] & 0x0F0F0F0Fu, lo);
                        n4x4_to_f32((w[n][j].q[i] >> 4) & 0x0F0F0F0Fu, hi);
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            sb = fmaf(lo[e], xr[j][4 * i + e], sb);
                            sb = fmaf(hi[e], xr[j][4 * i + e + 16], sb);
                        }
                    }
                    sacc = fmaf(w[n][j].d, sb, sacc);
                }
            }
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) sacc += __shfl_xor_sync(0xffffffffu, sacc, o);
            acc[n] = sacc;
        }
        if (WPR > 1) {
            if (lane == 0)
#pragma unroll
                for (int n = 0; n < kRegRows; n++) part[buf][warp][n] = acc[n];
            __syncthreads();
            if (piece == 0)
#pragma unroll
                for (int n = 0; n < kRegRows; n++) {
                    float sum = 0.f;
                    for (int p = 0; p < WPR; p++) sum += part[buf][warp + p][n];
                    acc[n] = sum;
                }
        }
        if (piece != 0 || lane != 0) continue;
        if (silu) {
#pragma unroll
            for (int o = 0; o < kRegRows / 2; o++) {
                if (!rp[2 * o]) continue;
                const int out = r0 + slot * (kRegRows / 2) + o;
                const float gt = acc[2 * o];
                a.y[0][out] = (gt / (1.0f + expf(-gt))) * acc[2 * o + 1];
            }
            continue;
        }
#pragma unroll
        for (int n = 0; n < kRegRows; n++) {
            if (!rp[n]) continue;
            int lr = r0 + slot * kRegRows + n, m = 0;
            if (lr >= a.rows[0]) {
                lr -= a.rows[0];
                m = 1;
                if (lr >= a.rows[1]) {
                    lr -= a.rows[1];
                    m = 2;
                }
            }
            float* yp = a.y[m] + lr;
            *yp = ((a.flags & ALPACA_PROJ_ADD) ? *yp : 0.f) + acc[n];
        }
    }
}

// ---- single-token path for GGUF blocks: coalesced staging of each warp's span of 32 blocks.
// A warp piece covers 32 consecutive blocks of a row (1088 bytes of q8_0, 576 of q4_0), contiguous in memory: the warp
// copies the span into its own shared-memory buffer with 16-byte cp.async (one copy per lane and 16 bytes instead of
// nine 4-byte loads per lane and block), double-buffered across passes so the next rows' copies are in flight while
// the current ones are used. Two lanes share a block (16 quants, or 8 bytes of nibble pairs, each), so a lane always
// meets the same elements of every row and keeps those 32 input values in registers; each lane scales its partial dot
// by its block's scale, so blocks need no cross-lane reduction. Quants are read as aligned words and funnel-shifted by
// the block's 2-byte phase (no branch: neighbouring blocks alternate phase) and multiplied as f32 pairs.
constexpr int kQRows = 2;  // rows per warp slot per pass (SiLU: one output, its gate and up rows)

template <int F>
struct QGeo {
    static constexpr int BB = F == 1 ? 34 : 18;             // bytes per block
    static constexpr int QB = F == 1 ? 16 : 8;              // quant bytes per lane (half of the block's)
    static constexpr int SPAN = 32 * BB;                    // bytes of a warp's 32 blocks
    static constexpr int BUF = (SPAN + 32 + 15) / 16 * 16;  // the span's 16-byte-aligned cover (+ the funnel word)
};

__device__ __forceinline__ void cp_async16_zfill(void* smem_dst, const void* gsrc, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(src_bytes)
                 : "memory");
}

// Copy the 16-byte cover of [p, p + n) (n <= SPAN) into buf; bytes at or past `end` are zero-filled, never read.
// Returns the offset of p inside buf.
template <int F>
__device__ __forceinline__ int stage_span(uint8_t* buf, const uint8_t* p, int n, const uint8_t* end, int lane) {
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(p) & ~uintptr_t(15);
    const uintptr_t a1 = reinterpret_cast<uintptr_t>(p + n);
    const uintptr_t lim = reinterpret_cast<uintptr_t>(end);
    for (uintptr_t a = a0 + 16 * lane; a < a1; a += 16 * 32) {
        const uint32_t src = a >= lim ? 0u : static_cast<uint32_t>(std::min<uintptr_t>(16, lim - a));
        cp_async16_zfill(buf + (a - a0), reinterpret_cast<const void*>(src ? a : a0), src);
    }
    return static_cast<int>(reinterpret_cast<uintptr_t>(p) - a0);
}

template <int F>
__global__ void __launch_bounds__(kProjThreads, 3) proj_q_kernel(const ProjArgs a) {
    using G = QGeo<F>;
    constexpr int BB = G::BB, BUF = G::BUF;
    extern __shared__ __align__(16) uint8_t smem[];
    float* xs = reinterpret_cast<float*>(smem);                                    // the staged row [k]
    uint8_t* spans = smem + ((sizeof(float) * a.k + 15) / 16) * 16;               // [warp][2 passes][kQRows][BUF]
    __shared__ float red[kProjWarps];
    __shared__ float scale;
    __shared__ float part[2][kProjWarps][kQRows];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const bool silu = (a.flags & ALPACA_PROJ_SILU) != 0;
    const int WPR = a.wpr, SLOTS = kProjWarps / WPR;
    const int RPC = SLOTS * (silu ? kQRows / 2 : kQRows);
    if (a.prefetch && threadIdx.x == 0) {
        for (int r0 = blockIdx.x * RPC; r0 < a.total_rows; r0 += gridDim.x * RPC) {
            const int r1 = min(r0 + RPC, a.total_rows);
            if (silu) {
                for (int m = 0; m < 2; m++) prefetch_l2(a.w[m] + r0 * a.row_bytes, (r1 - r0) * a.row_bytes, a.w_end[m]);
                continue;
            }
            for (int m = 0, base = 0; m < 3; base += a.rows[m], m++) {
                const int lo = max(r0, base), hi = min(r1, base + a.rows[m]);
                if (lo < hi) prefetch_l2(a.w[m] + (lo - base) * a.row_bytes, (hi - lo) * a.row_bytes, a.w_end[m]);
            }
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, k = a.k, U = a.units;
    const int slot = warp / WPR, piece = warp - slot * WPR;
    uint8_t* wbuf = spans + warp * (2 * kQRows * BUF);

    // The rows of pass (r0): row n of the slot, its matrix row pointer (null past the end).
    auto rows_of = [&](int r0, const uint8_t* (&rp)[kQRows], const uint8_t* (&re)[kQRows]) {
#pragma unroll
        for (int n = 0; n < kQRows; n++) {
            int r, m = 0;
            if (silu) {
                r = r0 + slot * (kQRows / 2) + n / 2;
                m = n & 1;
            } else {
                r = r0 + slot * kQRows + n;
            }
            rp[n] = nullptr;
            re[n] = nullptr;
            if (r >= a.total_rows) continue;
            int lr = r;
            if (!silu && lr >= a.rows[0]) {
                lr -= a.rows[0];
                m = 1;
                if (lr >= a.rows[1]) {
                    lr -= a.rows[1];
                    m = 2;
                }
            }
            rp[n] = a.w[m] + lr * a.row_bytes;
            re[n] = a.w_end[m];
        }
    };
    const int nblk = min(32, U - piece * 32);  // blocks of this piece (may be < 32 at the row's end, or <= 0)
    auto stage_pass = [&](int r0, int buf, int (&off)[kQRows]) {
        const uint8_t* rp[kQRows];
        const uint8_t* re[kQRows];
        rows_of(r0, rp, re);
#pragma unroll
        for (int n = 0; n < kQRows; n++)
            off[n] = (rp[n] && nblk > 0)
                         ? stage_span<F>(wbuf + (buf * kQRows + n) * BUF, rp[n] + piece * 32 * BB, nblk * BB, re[n], lane)
                         : 0;
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    // first pass's copies go out before the input row is staged
    int off[2][kQRows];
    const int first = blockIdx.x * RPC;
    if (first < a.total_rows) stage_pass(first, 0, off[0]);

    float ss = 0.f;
    for (int i = tid; i < k; i += kProjThreads) {
        const float v = a.x[i];
        xs[i] = v;
        ss = fmaf(v, v, ss);
    }
    if (a.flags & ALPACA_PROJ_NORM) {
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (tid == 0) {
            float tot = 0.f;
#pragma unroll
            for (int w = 0; w < kProjWarps; w++) tot += red[w];
            scale = 1.0f / sqrtf(tot / static_cast<float>(k) + a.eps);  // CPUOps.rmsNorm's scale
        }
        __syncthreads();
        for (int i = tid; i < k; i += kProjThreads) xs[i] = (xs[i] * scale) * a.g[i];  // x * scale * w
    }
    __syncthreads();

    // the lane's elements: half h of blocks bq and bq + 16 of the piece (q8_0: quants 16h..16h+15; q4_0: bytes
    // 8h..8h+7, whose low nibbles are elements 8h + j and high nibbles 16 + 8h + j), as f32 pairs
    const int h = lane & 1, bq = lane >> 1;
    constexpr int QB = G::QB, NW = QB / 4;  // quant words per lane and block
    float2 xr[2][8];
#pragma unroll
    for (int st = 0; st < 2; st++) {
        const int bl = bq + 16 * st;
        const bool in = bl < nblk;
        const float* xb = xs + (piece * 32 + bl) * 32;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            int c0;
            if constexpr (F == 1) c0 = 16 * h + 2 * j;
            else c0 = (j < 4 ? 8 * h : 16 + 8 * h) + 2 * (j & 3);
            xr[st][j] = in ? make_float2(xb[c0], xb[c0 + 1]) : make_float2(0.f, 0.f);
        }
    }
    const float2 bias = F == 1 ? make_float2(-8388736.0f, -8388736.0f) : make_float2(-8388616.0f, -8388616.0f);

    int pb = 0;
    for (int r0 = first; r0 < a.total_rows; r0 += gridDim.x * RPC, pb ^= 1) {  // uniform per CTA
        const int r0n = r0 + gridDim.x * RPC;
        if (r0n < a.total_rows) {
            stage_pass(r0n, pb ^ 1, off[pb ^ 1]);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncwarp();
        const uint8_t* rp[kQRows];
        const uint8_t* re[kQRows];
        rows_of(r0, rp, re);
        float acc[kQRows];
#pragma unroll
        for (int n = 0; n < kQRows; n++) {
            float2 acc2 = make_float2(0.f, 0.f);
            if (rp[n]) {
                const uint8_t* sb = wbuf + (pb * kQRows + n) * BUF + off[pb][n];
#pragma unroll
                for (int st = 0; st < 2; st++) {
                    const int bl = bq + 16 * st;
                    if (bl >= nblk) continue;
                    const uint8_t* blk = sb + bl * BB;
                    const float d = __half2float(*reinterpret_cast<const __half*>(blk));
                    // the lane's quant bytes at blk + 2 + QB h: aligned words from floor4, shifted by the phase
                    const uintptr_t qa = reinterpret_cast<uintptr_t>(blk + 2 + QB * h);
                    const uint32_t* wp = reinterpret_cast<const uint32_t*>(qa & ~uintptr_t(3));
                    const uint32_t sh = static_cast<uint32_t>(qa & 3u) * 8u;
                    uint32_t wv[NW + 1];
#pragma unroll
                    for (int i = 0; i <= NW; i++) wv[i] = wp[i];
                    float2 sp = make_float2(0.f, 0.f);
#pragma unroll
                    for (int i = 0; i < NW; i++) {
                        const uint32_t w = __funnelshift_r(wv[i], wv[i + 1], sh);
                        if constexpr (F == 1) {
                            const uint32_t u = w ^ 0x80808080u;
                            const float2 f0 = __fadd2_rn(
                                make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540u)),
                                            __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541u))), bias);
                            const float2 f1 = __fadd2_rn(
                                make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542u)),
                                            __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543u))), bias);
                            sp = __ffma2_rn(f0, xr[st][2 * i], sp);
                            sp = __ffma2_rn(f1, xr[st][2 * i + 1], sp);
                        } else {
                            const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
                            const float2 l0 = __fadd2_rn(
                                make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7540u)),
                                            __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7541u))), bias);
                            const float2 l1 = __fadd2_rn(
                                make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7542u)),
                                            __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7543u))), bias);
                            const float2 h0 = __fadd2_rn(
                                make_float2(__uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7540u)),
                                            __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7541u))), bias);
                            const float2 h1 = __fadd2_rn(
                                make_float2(__uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7542u)),
                                            __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7543u))), bias);
                            sp = __ffma2_rn(l0, xr[st][2 * i], sp);
                            sp = __ffma2_rn(l1, xr[st][2 * i + 1], sp);
                            sp = __ffma2_rn(h0, xr[st][4 + 2 * i], sp);
                            sp = __ffma2_rn(h1, xr[st][4 + 2 * i + 1], sp);
                        }
                    }
                    acc2 = __ffma2_rn(make_float2(d, d), sp, acc2);
                }
            }
            float sacc = acc2.x + acc2.y;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) sacc += __shfl_xor_sync(0xffffffffu, sacc, o);
            acc[n] = sacc;
        }
        __syncwarp();  // the buffer of this pass is free for the pass after next
        if (WPR > 1) {
            if (lane == 0)
#pragma unroll
                for (int n = 0; n < kQRows; n++) part[pb][warp][n] = acc[n];
            __syncthreads();
            if (piece == 0)
#pragma unroll
                for (int n = 0; n < kQRows; n++) {
                    float sum = 0.f;
                    for (int p = 0; p < WPR; p++) sum += part[pb][warp + p][n];
                    acc[n] = sum;
                }
        }
        if (piece != 0 || lane != 0) continue;
        if (silu) {
            if (!rp[0]) continue;
            const int out = r0 + slot * (kQRows / 2);
            const float gt = acc[0];
            a.y[0][out] = (gt / (1.0f + expf(-gt))) * acc[1];
            continue;
        }
#pragma unroll
        for (int n = 0; n < kQRows; n++) {
            if (!rp[n]) continue;
            int lr = r0 + slot * kQRows + n, m = 0;
            if (lr >= a.rows[0]) {
                lr -= a.rows[0];
                m = 1;
                if (lr >= a.rows[1]) {
                    lr -= a.rows[1];
                    m = 2;
                }
            }
            float* yp = a.y[m] + lr;
            *yp = ((a.flags & ALPACA_PROJ_ADD) ? *yp : 0.f) + acc[n];
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// ---- single-token quantised form on the tensor cores: int8 mma.sync against exact digit planes of the input.
//
// The input row (normalised when asked) is rewritten once per CTA as signed base-128 digits: with E the exponent of
// the row's largest |x|, F = rint(x * 2^(26 - E)) (|F| < 2^27; exact to 2^-27 of that largest value) = d0 * 2^21 +
// d1 * 2^14 + d2 * 2^7 + d3 with d1..d3 in [-64, 63] and d0 in [-65, 65]: four int8 planes per 32-element block.
// One mma.sync m16n8k32 (s8 x s8 -> s32) per block takes the planes (rows 0-3 of A) against the block's 32 quants
// of 8 weight rows (B; q4_0 nibbles as unsigned 0..15, 8 x the digit sums subtracted after). The int32 sums are
// exact; each is multiplied by its row's f16 block scale and accumulated in f32 per plane, and the planes meet,
// weighted by 2^(7 (3 - plane) + E - 26), at the end of the row. Per block and row that is ~2.5 warp instructions,
// against ~13 for the float dot product.
// Each warp owns a tile of 8 weight rows (SiLU: 8 gate + 8 up rows for 8 outputs) and a strided share of the row's
// blocks (wpr warps per tile); a job = its KB blocks of the 8 (16) rows, staged with 16-byte cp.async into a
// two-stage ring (row slots 16 mod 128 bytes apart, so the 8 rows' words fall in different banks).
template <int F, int S, int H>
struct MmaGeo {
    static constexpr int BB = F == 1 ? 34 : 18;                 // bytes per block
    static constexpr int NR = S ? 16 : 8;                       // weight rows per warp tile
    static constexpr int KB = 16 / (S ? 2 : 1) / (H ? 2 : 1);   // blocks per job (H: half jobs)
    static constexpr int SPAN = KB * BB;
    static constexpr int CH = (SPAN + 30 + 15) / 16;            // 16-byte chunks of a span's cover at any 2-byte phase
    static constexpr int RS = 16 + 128 * ((CH * 16 + 4 - 16 + 127) / 128);  // row slot: >= cover + 4, 16 mod 128
    static constexpr int STAGE = NR * RS;
};

__device__ __forceinline__ void mma_s8_16832(int (&c)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1), "r"(0));
}

template <int F, int S, int H>
__global__ void __launch_bounds__(kProjThreads, 2) proj_mma_kernel(const ProjArgs a) {
    using Gm = MmaGeo<F, S, H>;
    constexpr int BB = Gm::BB, KB = Gm::KB, CH = Gm::CH, RS = Gm::RS, STAGE = Gm::STAGE;
    extern __shared__ __align__(16) uint8_t smem[];
    const int U = a.units;
    uint8_t* xq = smem;                                              // [U][4 planes][32] int8 digits
    int* xsum = reinterpret_cast<int*>(smem + U * 128);              // [U][4] digit sums (q4_0)
    uint8_t* stg = smem + U * 128 + (F == 2 ? U * 16 : 0);           // [8 warps][2][STAGE], 16-byte aligned
    __shared__ float red[kProjWarps];
    __shared__ float scale;
    __shared__ float part[2][kProjWarps][16];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int WPR = a.wpr, SLOTS = kProjWarps / WPR, RPC = SLOTS * 8;  // output rows per CTA pass
    const int total = a.total_rows;
    if (a.prefetch && threadIdx.x == 0) {
        for (int r0 = blockIdx.x * RPC; r0 < total; r0 += gridDim.x * RPC) {
            const int r1 = min(r0 + RPC, total);
            if constexpr (S) {
                for (int m = 0; m < 2; m++) prefetch_l2(a.w[m] + r0 * a.row_bytes, (r1 - r0) * a.row_bytes, a.w_end[m]);
            } else {
                for (int m = 0, base = 0; m < 3; base += a.rows[m], m++) {
                    const int lo = max(r0, base), hi = min(r1, base + a.rows[m]);
                    if (lo < hi) prefetch_l2(a.w[m] + (lo - base) * a.row_bytes, (hi - lo) * a.row_bytes, a.w_end[m]);
                }
            }
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int slot = warp / WPR, piece = warp - slot * WPR;
    const int NCH = (U + KB - 1) / KB;                              // jobs per row tile
    const int nj = piece < NCH ? (NCH - piece + WPR - 1) / WPR : 0;  // this warp's jobs per pass
    uint8_t* wst = stg + warp * 2 * STAGE;

    // Weight row i of the tile whose first output row is o0 (SiLU: rows 0-7 gate, 8-15 up): its start, or null.
    auto row_ptr = [&](int o0, int i, const uint8_t*& end) -> const uint8_t* {
        int r, m = 0;
        if (S) {
            r = o0 + (i & 7);
            m = i >> 3;
        } else {
            r = o0 + i;
        }
        end = nullptr;
        if (r >= total) return nullptr;
        if (!S && r >= a.rows[0]) {
            r -= a.rows[0];
            m = 1;
            if (r >= a.rows[1]) {
                r -= a.rows[1];
                m = 2;
            }
        }
        end = a.w_end[m];
        return a.w[m] + static_cast<int64_t>(r) * a.row_bytes;
    };
    // Staging: lane l copies for weight row (S ? l / 2 : l / 4) of the tile, every (S ? 2 : 4)-th 16-byte chunk of
    // the cover of the row's KB blocks of the job; bytes past a matrix are zero-filled. The row's start is looked up
    // once per pass.
    constexpr int CSUB = S ? 2 : 4;
    const int crow = lane / CSUB, csub = lane % CSUB;
    int c_o0 = -1;                 // pass whose copy row is cached
    const uint8_t* c_rp = nullptr;
    const uint8_t* c_end = nullptr;
    auto issue = [&](int o0, int c, int st) {
        if (o0 != c_o0) {
            c_rp = row_ptr(o0, crow, c_end);
            c_o0 = o0;
        }
        if (c_rp) {
            uint8_t* dst = wst + st * STAGE + crow * RS;
            const uint8_t* p = c_rp + static_cast<int64_t>(c) * KB * BB;
            const uintptr_t a0 = reinterpret_cast<uintptr_t>(p) & ~uintptr_t(15);
            const uintptr_t stop = reinterpret_cast<uintptr_t>(p + min(KB, U - c * KB) * BB);
            const uintptr_t lim = reinterpret_cast<uintptr_t>(c_end);
#pragma unroll
            for (int ch = csub; ch < CH; ch += CSUB) {
                const uintptr_t ad = a0 + 16 * ch;
                if (ad >= stop) break;
                const uint32_t src = ad >= lim ? 0u : static_cast<uint32_t>(lim - ad >= 16 ? 16 : lim - ad);
                cp_async16_zfill(dst + 16 * ch, reinterpret_cast<const void*>(src ? ad : a0), src);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    const int first = blockIdx.x * RPC;
    if (nj > 0 && first < total) issue(first + slot * 8, piece, 0);  // in flight while the input is prepared

    // ---- the input row as digit planes: staged as floats in the planes' own bytes (one batch of loads), normalised
    // in place when asked, then each warp rewrites its blocks in place (a block's 32 floats and its four 32-byte
    // planes take the same 128 bytes). One exponent for the whole row (that of its largest |value|), so the digit
    // sums of every block carry the same scale and it is applied once, after the row's sum.
    float* xs = reinterpret_cast<float*>(xq);
    __shared__ int s_exp;
    {
        float ss = 0.f;
        for (int i = tid; i < a.k; i += kProjThreads) {
            const float v = a.x[i];
            xs[i] = v;
            ss = fmaf(v, v, ss);
        }
        if (a.flags & ALPACA_PROJ_NORM) {
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) red[warp] = ss;
            __syncthreads();
            if (tid == 0) {
                float tot = 0.f;
#pragma unroll
                for (int w = 0; w < kProjWarps; w++) tot += red[w];
                scale = 1.0f / sqrtf(tot / static_cast<float>(a.k) + a.eps);  // CPUOps.rmsNorm's scale
            }
        }
        __syncthreads();
        uint32_t mx = 0u;
        for (int i = tid; i < a.k; i += kProjThreads) {
            float v = xs[i];
            if (a.flags & ALPACA_PROJ_NORM) {
                v = (v * scale) * a.g[i];  // x * scale * w
                xs[i] = v;
            }
            mx = max(mx, __float_as_uint(v) & 0x7fffffffu);
        }
        mx = __reduce_max_sync(0xffffffffu, mx);
        if (lane == 0) red[warp] = __uint_as_float(mx);
        __syncthreads();
        if (tid == 0) {
            uint32_t m = 0u;
#pragma unroll
            for (int w = 0; w < kProjWarps; w++) m = max(m, __float_as_uint(red[w]));
            s_exp = static_cast<int>(m >> 23) - 127;  // exponent of the row's largest |value|
        }
        __syncthreads();
    }
    const int E = s_exp;
    // F = rint(x * 2^(26 - E)), |F| < 2^27; a row whose largest |value| is below 2^-100 counts as zero
    const float fscale = E >= -100 ? __int_as_float((127 + 26 - E) << 23) : 0.f;
    for (int b = warp; b < U; b += kProjWarps) {
        const float v = xs[b * 32 + lane];
        __syncwarp();  // every lane holds its float before the block's bytes are rewritten
        const int Fx = __float2int_rn(v * fscale);
        const int d3 = (Fx << 25) >> 25;
        const int f1 = (Fx - d3) >> 7;
        const int d2 = (f1 << 25) >> 25;
        const int f2 = (f1 - d2) >> 7;
        const int d1 = (f2 << 25) >> 25;
        const int d0 = (f2 - d1) >> 7;
        int8_t* xb = reinterpret_cast<int8_t*>(xq + b * 128);
        xb[lane] = static_cast<int8_t>(d0);
        xb[32 + lane] = static_cast<int8_t>(d1);
        xb[64 + lane] = static_cast<int8_t>(d2);
        xb[96 + lane] = static_cast<int8_t>(d3);
        if constexpr (F == 2) {
            const int s0 = __reduce_add_sync(0xffffffffu, d0), s1 = __reduce_add_sync(0xffffffffu, d1);
            const int s2 = __reduce_add_sync(0xffffffffu, d2), s3 = __reduce_add_sync(0xffffffffu, d3);
            if (lane == 0) *reinterpret_cast<int4*>(xsum + 4 * b) = make_int4(s0, s1, s2, s3);
        }
    }
    __syncthreads();

    // ---- lane roles: B column n = weight row n (and 8 + n), k group t; A row g = digit plane g (lanes g < 4);
    // C: plane g, columns 2t / 2t + 1 = weight rows 2t / 2t + 1
    const int n = lane >> 2, t = lane & 3, g = lane >> 2;
    // plane g's weight in the row: 2^(7 (3 - g)) x 2^(E - 26) (exact; 0 for the zero rows of A, or a zero row)
    const float psc = (g < 4 && E >= -100) ? __int_as_float((127 + 7 * (3 - g) + E - 26) << 23) : 0.f;
    const uint32_t amask = g < 4 ? 0xFFFFFFFFu : 0u;  // A rows 4-7 (and 8-15) are zero
    auto row_phase = [&](int o0, int i) -> int {  // the row start's offset in its 16-byte line
        const uint8_t* end;
        const uint8_t* rp = row_ptr(o0, i, end);
        return rp ? static_cast<int>(reinterpret_cast<uintptr_t>(rp) & 15u) : 0;
    };

    int pb = 0, st = 0;
    for (int r0 = first; r0 < total; r0 += gridDim.x * RPC, pb ^= 1) {  // uniform per CTA
        const int o0 = r0 + slot * 8;
        const int r0n = r0 + gridDim.x * RPC;
        // per pass: the phases of the lane's B row and scale rows (the span of chunk c starts at phase + c KB BB)
        int ph_b[2], ph_d[2][2];
#pragma unroll
        for (int h = 0; h < (S ? 2 : 1); h++) {
            ph_b[h] = row_phase(o0, 8 * h + n);
            ph_d[h][0] = row_phase(o0, 8 * h + 2 * t);
            ph_d[h][1] = row_phase(o0, 8 * h + 2 * t + 1);
        }
        float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};  // [gate / only, up][row 2t, 2t + 1]
        for (int j = 0; j < nj; j++) {
            const int c = piece + j * WPR;
            // the next job: this tile's next chunk, else the first chunk of the next pass
            __syncwarp();  // every lane is done with the stage the next job goes into
            if (j + 1 < nj) issue(o0, c + WPR, st ^ 1);
            else if (r0n < total) issue(r0n + slot * 8, piece, st ^ 1);
            else asm volatile("cp.async.commit_group;" ::: "memory");
            asm volatile("cp.async.wait_group 1;" ::: "memory");
            __syncwarp();
            const uint8_t* sbp = wst + st * STAGE;
            const int cb = c * KB * BB;
            // per-job lane pointers; BB = 2 mod 4, so the blocks' quants alternate between two phases: even blocks
            // at the first word phase, odd ones at the other, each from its own aligned base (immediate offsets)
            const uint8_t* qe[2];
            const uint8_t* qo[2];
            const uint8_t* dp[2][2];
            uint32_t she = 0, sho = 0;
#pragma unroll
            for (int h = 0; h < (S ? 2 : 1); h++) {
                const uintptr_t q0 = reinterpret_cast<uintptr_t>(sbp + (8 * h + n) * RS + ((ph_b[h] + cb) & 15) + 2 + 4 * t);
                const uint32_t ph = static_cast<uint32_t>(q0 & 3u);  // 0 or 2
                qe[h] = reinterpret_cast<const uint8_t*>(q0 - ph);
                qo[h] = reinterpret_cast<const uint8_t*>(q0 - ph + (ph ? 2 : -2));
                she = ph * 8u;
                sho = 16u - she;
                dp[h][0] = sbp + (8 * h + 2 * t) * RS + ((ph_d[h][0] + cb) & 15);
                dp[h][1] = sbp + (8 * h + 2 * t + 1) * RS + ((ph_d[h][1] + cb) & 15);
            }
            const uint8_t* xa = xq + (c * KB) * 128 + (g & 3) * 32 + 4 * t;  // plane g & 3 of the job's first block
            const int* xsm = xsum + 4 * (c * KB) + (g & 3);
            auto block = [&](int bl) {
                const uint32_t a0 = *reinterpret_cast<const uint32_t*>(xa + bl * 128) & amask;
                const uint32_t a2 = *reinterpret_cast<const uint32_t*>(xa + bl * 128 + 16) & amask;
                int corr = 0;
                if constexpr (F == 2) corr = 8 * static_cast<int>(static_cast<uint32_t>(xsm[4 * bl]) & amask);
#pragma unroll
                for (int h = 0; h < (S ? 2 : 1); h++) {
                    const uint8_t* w = ((bl & 1) ? qo[h] : qe[h]) + bl * BB;
                    const uint32_t sh = (bl & 1) ? sho : she;
                    uint32_t b0, b1;
                    if constexpr (F == 1) {
                        b0 = __funnelshift_r(*reinterpret_cast<const uint32_t*>(w), *reinterpret_cast<const uint32_t*>(w + 4), sh);
                        b1 = __funnelshift_r(*reinterpret_cast<const uint32_t*>(w + 16), *reinterpret_cast<const uint32_t*>(w + 20), sh);
                    } else {  // byte j holds element j (low nibble) and element 16 + j (high nibble)
                        const uint32_t x = __funnelshift_r(*reinterpret_cast<const uint32_t*>(w), *reinterpret_cast<const uint32_t*>(w + 4), sh);
                        b0 = x & 0x0F0F0F0Fu;
                        b1 = (x >> 4) & 0x0F0F0F0Fu;
                    }
                    int cc[4];
                    mma_s8_16832(cc, a0, a2, b0, b1);
                    const float w0 = __half2float(*reinterpret_cast<const __half*>(dp[h][0] + bl * BB));
                    const float w1 = __half2float(*reinterpret_cast<const __half*>(dp[h][1] + bl * BB));
                    acc[h][0] = fmaf(w0, static_cast<float>(cc[0] - corr), acc[h][0]);
                    acc[h][1] = fmaf(w1, static_cast<float>(cc[1] - corr), acc[h][1]);
                }
            };
            const int nb = min(KB, U - c * KB);
            if (nb == KB) {
#pragma unroll
                for (int bl = 0; bl < KB; bl++) block(bl);
            } else {
                for (int bl = 0; bl < nb; bl++) block(bl);
            }
            st ^= 1;
        }
        // planes 0-3 (lanes t, 4 + t, 8 + t, 12 + t), each scaled by its weight, meet in lanes 0-3; then the wpr
        // warps of the tile
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
            for (int x = 0; x < 2; x++) {
                acc[h][x] *= psc;
                acc[h][x] += __shfl_down_sync(0xffffffffu, acc[h][x], 8);
                acc[h][x] += __shfl_down_sync(0xffffffffu, acc[h][x], 4);
            }
        if (lane < 4) {
            part[pb][warp][2 * lane] = acc[0][0];
            part[pb][warp][2 * lane + 1] = acc[0][1];
            if (S) {
                part[pb][warp][8 + 2 * lane] = acc[1][0];
                part[pb][warp][8 + 2 * lane + 1] = acc[1][1];
            }
        }
        __syncthreads();
        if (tid < RPC) {
            const int s = tid >> 3, i = tid & 7, out = r0 + tid;
            if (out < total) {
                float v0 = 0.f, v1 = 0.f;
                for (int p = 0; p < WPR; p++) {
                    v0 += part[pb][s * WPR + p][i];
                    if (S) v1 += part[pb][s * WPR + p][8 + i];
                }
                if (S) {
                    a.y[0][out] = (v0 / (1.0f + expf(-v0))) * v1;
                } else {
                    int lr = out, m = 0;
                    if (lr >= a.rows[0]) {
                        lr -= a.rows[0];
                        m = 1;
                        if (lr >= a.rows[1]) {
                            lr -= a.rows[1];
                            m = 2;
                        }
                    }
                    float* yp = a.y[m] + lr;
                    *yp = ((a.flags & ALPACA_PROJ_ADD) ? *yp : 0.f) + v0;
                }
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

int proj_env(const char* name, int fallback) {
    const char* e = std::getenv(name);
    return (e && *e) ? std::atoi(e) : fallback;
}
int proj_ctas_per_sm(int fallback) {
    static const int v = proj_env("ALPACA_PROJ_CTAS", 0);
    return v > 0 ? v : fallback;
}

// Single-token launch of the register form: wpr from the lane's unit count, the row staged in shared memory.
template <int F>
cudaError_t launch_reg(ProjArgs a, int num_sms, cudaStream_t s) {
    constexpr int per_warp = 32 * RegGeo<F>::UPL;  // units one warp covers
    const int want = (a.units + per_warp - 1) / per_warp;
    a.wpr = want >= 8 ? 8 : (want >= 4 ? 4 : (want >= 2 ? 2 : 1));
    const size_t smem = sizeof(float) * static_cast<size_t>(a.k);
    const auto fn = proj_reg_kernel<F>;
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    const bool silu = (a.flags & ALPACA_PROJ_SILU) != 0;
    const int rpc = (kProjWarps / a.wpr) * (silu ? kRegRows / 2 : kRegRows);
    const int row_ctas = (a.total_rows + rpc - 1) / rpc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::max(1, std::min(row_ctas, num_sms * proj_ctas_per_sm(3))), 1, 1);
    cfg.blockDim = dim3(kProjThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, a);
}

// Single-token launch of the staged-block form (quantised weights): one warp per 32 blocks of a row.
template <int F>
cudaError_t launch_q(ProjArgs a, int num_sms, cudaStream_t s) {
    const int want = (a.units + 31) / 32;
    a.wpr = want >= 8 ? 8 : (want >= 4 ? 4 : (want >= 2 ? 2 : 1));
    const size_t smem = (sizeof(float) * a.k + 15) / 16 * 16 + static_cast<size_t>(kProjWarps) * 2 * kQRows * QGeo<F>::BUF;
    const auto fn = proj_q_kernel<F>;
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    const bool silu = (a.flags & ALPACA_PROJ_SILU) != 0;
    const int rpc = (kProjWarps / a.wpr) * (silu ? kQRows / 2 : kQRows);
    const int row_ctas = (a.total_rows + rpc - 1) / rpc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::max(1, std::min(row_ctas, num_sms * proj_ctas_per_sm(3))), 1, 1);
    cfg.blockDim = dim3(kProjThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, a);
}

// Single-token launch of the int8 tensor-core form: wpr = the smallest power of two >= the row's jobs (at most 8).
template <int F, int S, int H>
size_t mma_smem(int units) {
    return static_cast<size_t>(units) * (128 + (F == 2 ? 16 : 0)) + 2 * kProjWarps * MmaGeo<F, S, H>::STAGE;
}
template <int F, int S, int H>
int mma_wpr(int units) {
    const int nch = (units + MmaGeo<F, S, H>::KB - 1) / MmaGeo<F, S, H>::KB;
    return nch > 4 ? 8 : (nch > 2 ? 4 : nch);
}
template <int F, int S, int H>
cudaError_t launch_mma_fsh(ProjArgs a, int num_sms, cudaStream_t s) {
    a.wpr = mma_wpr<F, S, H>(a.units);
    const size_t smem = mma_smem<F, S, H>(a.units);
    const auto fn = proj_mma_kernel<F, S, H>;
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    static std::mutex mu;
    static size_t last_smem = 0;
    static int last_occ = 1;
    int occ;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (last_smem != smem) {
            int o = 0;
            const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, fn, kProjThreads, smem);
            if (e != cudaSuccess) return e;
            last_occ = std::max(1, o);
            last_smem = smem;
        }
        occ = last_occ;
    }
    const int rpc = (kProjWarps / a.wpr) * 8;
    const int row_ctas = (a.total_rows + rpc - 1) / rpc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::max(1, std::min(row_ctas, num_sms * proj_ctas_per_sm(occ))), 1, 1);
    cfg.blockDim = dim3(kProjThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, a);
}
// Full jobs unless they leave fewer than two CTAs per SM of row tiles (small matrices: more warps per row) or two
// CTAs of them do not fit an SM (long rows: the staged input takes the room).
template <int F, int S>
cudaError_t launch_mma_fs(ProjArgs a, int num_sms, cudaStream_t s) {
    const int rpc = (kProjWarps / mma_wpr<F, S, 0>(a.units)) * 8;
    const int row_ctas = (a.total_rows + rpc - 1) / rpc;
    const bool half = row_ctas < 2 * num_sms || mma_smem<F, S, 0>(a.units) > 113 * 1024;
    return half ? launch_mma_fsh<F, S, 1>(a, num_sms, s) : launch_mma_fsh<F, S, 0>(a, num_sms, s);
}
template <int F>
cudaError_t launch_mma(ProjArgs a, int num_sms, cudaStream_t s) {
    return (a.flags & ALPACA_PROJ_SILU) ? launch_mma_fs<F, 1>(a, num_sms, s) : launch_mma_fs<F, 0>(a, num_sms, s);
}

// Whether the register form covers k: at most 8 warps of 32 lanes x UPL units per row.
bool reg_form_fits(int format, int k) {
    return format == ALPACA_W_F16 ? k <= 8 * 32 * 4 * 8 : k <= 8 * 32 * 32;
}

template <int F>
cudaError_t launch_f(const ProjArgs& a, int tp, int num_sms, cudaStream_t s) {
    using Fn = void (*)(ProjArgs);
    Fn fn = tp == 1 ? proj_kernel<F, 1> : (tp == 2 ? proj_kernel<F, 2> : proj_kernel<F, 4>);
    const int tpk = tp;  // 1, 2 or 4 rows staged per pass
    const size_t smem = sizeof(float) * static_cast<size_t>(tpk) * xs_row<F>(a.k, a.units);
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    const int rpc = (kProjWarps / a.wpr) * ((a.flags & ALPACA_PROJ_SILU) ? 1 : 2);
    const int row_ctas = (a.total_rows + rpc - 1) / rpc;
    const int resident = proj_ctas_per_sm(tpk == 1 ? 4 : 2);  // CTAs per SM under the launch bounds
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::max(1, std::min(row_ctas, num_sms * resident)), (a.n_tokens + tpk - 1) / tpk, 1);
    cfg.blockDim = dim3(kProjThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, a);
}

}  // namespace

int64_t proj_row_bytes(int format, int k) {
    switch (format) {
        case ALPACA_W_F16: return 2 * static_cast<int64_t>(k);
        case ALPACA_W_Q8_0: return static_cast<int64_t>(k / 32) * 34;
        case ALPACA_W_Q4_0: return static_cast<int64_t>(k / 32) * 18;
        default: return 0;
    }
}

// Input rows staged per pass: 4, 2 or 1, as the shared-memory budget allows for rows of k (+ 32 pad) floats.
int proj_max_tokens_per_pass(int k) {
    const size_t by_smem = kProjSmemBudget / (sizeof(float) * static_cast<size_t>(k + 32));
    return by_smem >= kProjMaxTokens ? kProjMaxTokens : (by_smem >= 2 ? 2 : 1);
}

cudaError_t launch_proj(const alpaca_proj_desc& d, int num_sms, cudaStream_t s) {
    ProjArgs a;
    const bool silu = (d.flags & ALPACA_PROJ_SILU) != 0;
    a.row_bytes = proj_row_bytes(d.format, d.k);
    for (int i = 0; i < 3; i++) {
        const int mi = silu ? (i < 2 ? i : 1) : i;
        const int rows = silu ? d.rows[0] : d.rows[i];
        a.w[i] = static_cast<const uint8_t*>(d.w[mi] ? d.w[mi] : d.w[0]);
        a.w_end[i] = a.w[i] + static_cast<int64_t>(rows) * a.row_bytes;
        a.rows[i] = silu ? (i == 0 ? d.rows[0] : 0) : d.rows[i];
        a.y[i] = d.y[i] ? d.y[i] : d.y[0];
        a.y_stride[i] = d.y[i] ? d.y_stride[i] : d.y_stride[0];
    }
    a.total_rows = silu ? d.rows[0] : d.rows[0] + d.rows[1] + d.rows[2];
    a.k = d.k;
    a.units = d.format == ALPACA_W_F16 ? d.k / 8 : d.k / 32;
    a.flags = d.flags;
    a.eps = d.eps;
    a.x = d.x;
    a.x_stride = d.x_stride;
    a.g = d.norm_weight;
    a.n_tokens = d.n_tokens;
    // warps per row: about two units (16-byte chunks or blocks) per lane per row, up to the CTA's 8 warps
    const int want = (a.units + 63) / 64;
    a.wpr = want >= 8 ? 8 : (want >= 4 ? 4 : (want >= 2 ? 2 : 1));
    static const int wpr_cap = proj_env("ALPACA_PROJ_WPR", 8);
    a.wpr = std::min(a.wpr, std::max(1, wpr_cap));
    static const int prefetch = proj_env("ALPACA_PROJ_PREFETCH", 1);
    a.prefetch = prefetch;
    const int cap = proj_max_tokens_per_pass(d.k);
    const int tp = d.n_tokens >= cap ? cap : (d.n_tokens == 1 ? 1 : (d.n_tokens == 2 ? 2 : std::min(cap, 4)));
    static const int reg_form = proj_env("ALPACA_PROJ_REG", 1);
    static const int mma_form = proj_env("ALPACA_PROJ_MMA", 1);
    if (d.n_tokens == 1 && mma_form && d.format != ALPACA_W_F16)
        return d.format == ALPACA_W_Q8_0 ? launch_mma<1>(a, num_sms, s) : launch_mma<2>(a, num_sms, s);
    if (d.n_tokens == 1 && reg_form && reg_form_fits(d.format, d.k)) {
        switch (d.format) {
            case ALPACA_W_F16: return launch_reg<0>(a, num_sms, s);
            case ALPACA_W_Q8_0: return reg_form == 2 ? launch_reg<1>(a, num_sms, s) : launch_q<1>(a, num_sms, s);
            default: return reg_form == 2 ? launch_reg<2>(a, num_sms, s) : launch_q<2>(a, num_sms, s);
        }
    }
    switch (d.format) {
        case ALPACA_W_F16: return launch_f<0>(a, tp, num_sms, s);
        case ALPACA_W_Q8_0: return launch_f<1>(a, tp, num_sms, s);
        default: return launch_f<2>(a, tp, num_sms, s);
    }
}

}  // namespace alpaca
