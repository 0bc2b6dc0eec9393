// attn_decode.cu — split-KV single-token decode attention over the f16 KV cache, plus the combine kernel.
//
// Same job as alpaca.swift's attn_decode_split_* / attn_decode_merge (Sources/AlpacaMetal/Kernels/
// attention_decode.metal:28-133, dispatched by KernelEncoder.swift:309-326), designed for B200 HBM3e:
//
//   split kernel  grid (splits x kv_heads, seqs), 128 threads, KV heads fastest. One CTA owns SL consecutive cache rows of one KV
//                 head of one sequence and serves all G query heads of that KV head, so every K/V byte is read
//                 from HBM exactly once. Each cache row (d halves) is copied by d/8 lanes with 16-byte cp.async
//                 into shared memory (rows past the context are zero-filled), K first then V, so registers stay
//                 low (six CTAs per SM keep ~190 KB in flight per SM) and the V copy overlaps the score math.
//                 head_dim 64: each warp takes a quarter of the rows on mma.sync m16n8k16 with split-precision
//                 f16 operands (hi / remainder rows of Q and of P in the two halves of the 16-row tile, ~2^-22
//                 relative error), K and V read with ldmatrix from XOR-swizzled tiles, P kept in registers.
//                 head_dim 128: packed f32x2 FMAs; scores reduced across a row's lanes with a transposing
//                 butterfly (7 shuffles for 8 rows instead of 24), softmax once per (row, head) from shared
//                 memory, P·V partial sums reduced across rows through shared memory.
//   combine       grid (kv_heads, seqs), 256 threads: rescales the per-split (m, l, acc) states of the G heads to
//                 the global max and normalises. Launched with programmatic dependent launch so its launch
//                 overlaps the split tail. Sequences with one split are finished by the split kernel itself.
//
// Scores are kept in log2 units (q pre-scaled by scale*log2(e)), so every exponential is one ex2.approx.
// Partial-state layout: [seq][kv_head][split][g][d + 2] f32 = accumulators, then m (log2 units), then l.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace alpaca {
namespace {

constexpr int kThreads = 128;
constexpr int kSlots = 8;     // cache rows per thread per split
constexpr int kMaxGroup = 8;  // query heads per KV head (attention_decode.metal:25)
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct Geo {
    static constexpr int LPR = D / 8;                    // lanes per cache row (16 B each)
    static constexpr int RPW = 32 / LPR;                 // rows per warp per slot
    static constexpr int RPS = RPW * (kThreads / 32);    // rows per CTA per slot
    static constexpr int SL = RPS * kSlots;              // rows per split: 128 (d=64), 64 (d=128)
};

struct DecodeArgs {
    const void* q;
    int64_t q_seq_stride;
    int q_f16;
    const __half* k;
    const __half* v;
    int64_t kv_row_stride, kv_seq_stride;
    void* out;
    int64_t out_seq_stride;
    int out_f16;
    float* partial;
    const int* ctx_lens;
    int uniform_len;
    int max_len;  // upper bound of every context length (desc.max_ctx_len, or uniform_len)
    int n_heads, n_kv_heads, max_splits;
    float scale_log2;
    const int* block_table;  // paged cache: [seq][max_blocks] block indices (null: contiguous caches)
    int block_rows, max_blocks, pool_blocks;
    int64_t block_stride;
    unsigned* err;
    // Fused RoPE + KV append (alpaca_attn_decode_rope): each sequence's new token sits at row ctx_len - 1; its
    // k / v rows (f32 [seq][kv_head][d]) are rotated / copied into the cache there, and q is rotated as it is read.
    int rope, interleaved;
    const float* k_new;
    const float* v_new;
    int64_t new_seq_stride;
    int early_release;  // split CTAs release the combine launch at their start (else at their end)
    double freq[128];  // theta^(-2i/d), host-computed in double as for alpaca_rope_kv_append
};

// Element offset of cache row `row0` of KV head `kvh` of sequence `seq` (contiguous, or through the block table;
// a unit's SL rows never cross a block because block_rows is a multiple of 128). A table entry outside the pool
// clears `valid` (the unit's rows are then zero-filled, not read) and raises the device error word.
__device__ __forceinline__ int64_t unit_offset(const DecodeArgs& a, int seq, int kvh, int row0, int D, bool& valid) {
    valid = true;
    if (a.block_table) {
        const int blk = a.block_table[static_cast<int64_t>(seq) * a.max_blocks + row0 / a.block_rows];
        if (blk < 0 || blk >= a.pool_blocks) {
            valid = false;
            atomicOr(a.err, kDevErrBadIndex);
            return 0;
        }
        return static_cast<int64_t>(blk) * a.block_stride + static_cast<int64_t>(row0 % a.block_rows) * a.kv_row_stride +
               static_cast<int64_t>(kvh) * D;
    }
    return static_cast<int64_t>(seq) * a.kv_seq_stride + static_cast<int64_t>(row0) * a.kv_row_stride +
           static_cast<int64_t>(kvh) * D;
}

// Context length of sequence s. A device entry outside [1, max_len] breaks the caller's contract (the grid and the
// workspace were sized for max_len): it is clamped, so no CTA reads or writes past the sequence's records, and the
// device error word reports it (INVALID_ARGUMENT from alpaca_cuda_device_status).
__device__ __forceinline__ int ctx_len_of(const DecodeArgs& a, int s) {
    if (!a.ctx_lens) return a.uniform_len;
    const int L = a.ctx_lens[s];
    if (L < 1 || L > a.max_len) {
        atomicOr(a.err, kDevErrBadIndex);
        return L < 1 ? 0 : a.max_len;
    }
    return L;
}

__device__ __forceinline__ void half8_to_float(const uint4& u, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

// Transposing butterfly: on entry every lane of a row group holds partial sums for kSlots rows; on exit lane
// holds the full sum of one row (slot index returned). LPR lanes form a row group.
template <int LPR>
__device__ __forceinline__ float reduce_rows(float (&v)[kSlots], int lane, int& slot) {
    float w[kSlots];
#pragma unroll
    for (int i = 0; i < kSlots; i++) w[i] = v[i];
    int n = kSlots;
    int off = LPR / 2;
    slot = 0;
#pragma unroll
    for (int step = 0; step < 3; step++) {  // kSlots = 8 -> 3 halvings
        const bool up = (lane & off) != 0;
        const int half = n / 2;
#pragma unroll
        for (int i = 0; i < kSlots / 2; i++) {
            if (i < half) {
                const float send = up ? w[i] : w[i + half];
                const float keep = up ? w[i + half] : w[i];
                w[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
            }
        }
        if (up) slot += half;
        n = half;
        off >>= 1;
    }
    float r = w[0];
#pragma unroll
    for (int o = off; o >= 1; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    return r;
}

// 16-byte async copy global -> shared (L2 only); src_bytes = 0 fills the 16 bytes with zeros.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gsrc),
                 "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Issue the async copies of one unit's K rows (one commit group) and V rows (a second group) into shared memory.
// Rows past the context are zero-filled and never read. Each thread later reads back only the chunks it copied.
// kSwz: 16-byte chunk c of row r is stored at chunk c ^ (r & 7), so the eight rows an ldmatrix reads at one chunk
// index fall in eight different bank groups.
// kSkip: row skip_row (absolute) is not copied at all because the CTA writes it into the tiles itself.
template <int D, bool kSwz = false, bool kSkip = false>
__device__ __forceinline__ void stage_unit(const DecodeArgs& a, int seq, int kvh, int row0, int row_end,
                                           __half* s_k, __half* s_v, int lr, int rowlane, int skip_row = -1) {
    constexpr int RPS = Geo<D>::RPS;
    bool valid;
    const int64_t base = unit_offset(a, seq, kvh, row0, D, valid) + lr * 8;
#pragma unroll
    for (int i = 0; i < kSlots; i++) {
        const int rl = i * RPS + rowlane, r = row0 + rl;
        const bool in = valid && r < row_end;
        const int c = kSwz ? (lr ^ (rl & 7)) : lr;
        if (!kSkip || r != skip_row)
            cp_async16(s_k + rl * D + c * 8, a.k + base + (in ? static_cast<int64_t>(rl) * a.kv_row_stride : 0),
                       in ? 16u : 0u);
    }
    cp_async_commit();
#pragma unroll
    for (int i = 0; i < kSlots; i++) {
        const int rl = i * RPS + rowlane, r = row0 + rl;
        const bool in = valid && r < row_end;
        const int c = kSwz ? (lr ^ (rl & 7)) : lr;
        if (!kSkip || r != skip_row)
            cp_async16(s_v + rl * D + c * 8, a.v + base + (in ? static_cast<int64_t>(rl) * a.kv_row_stride : 0),
                       in ? 16u : 0u);
    }
    cp_async_commit();
}

// ---- fused RoPE + KV append: the same arithmetic as alpaca_rope_kv_append (rope_kv.cu), so the fused call gives
// the results of the two calls bit for bit: angle position * freq and cos / sin in double, rounded once to f32,
// rotation as separately rounded f32 products, f16 values rounded once.

// (cos, sin) of position pos for the D/2 pairs.
template <int D>
__device__ __forceinline__ void rope_table(const DecodeArgs& a, int pos, float2* s_cs, int tid) {
    for (int i = tid; i < D / 2; i += kThreads) {
        double sn, cs;
        sincos(static_cast<double>(pos) * a.freq[i], &sn, &cs);
        s_cs[i] = make_float2(static_cast<float>(cs), static_cast<float>(sn));
    }
}

// Pair partner of element dim (D elements per row) and whether dim is the pair's first element.
__device__ __forceinline__ int rope_partner(int dim, int D, int interleaved, bool& first) {
    const int h = D / 2;
    first = interleaved ? (dim & 1) == 0 : dim < h;
    return interleaved ? dim ^ 1 : (first ? dim + h : dim - h);
}
// Rotated element from the element x and its partner xp: a' = a c - b s for the first, b' = a s + b c for the
// second element of a pair (a, b), as separately rounded f32 operations.
__device__ __forceinline__ float rope_rotate(float x, float xp, int dim, int D, int interleaved, const float2* cs) {
    const int h = D / 2;
    const bool first = interleaved ? (dim & 1) == 0 : dim < h;
    const float2 w = cs[interleaved ? dim >> 1 : (first ? dim : dim - h)];
    const float a0 = first ? x : xp, b0 = first ? xp : x;
    return first ? __fsub_rn(__fmul_rn(a0, w.x), __fmul_rn(b0, w.y)) : __fadd_rn(__fmul_rn(a0, w.y), __fmul_rn(b0, w.x));
}

// Fused-call prologue, part 1 (before the (cos, sin) table): this thread's query elements of the G heads and their
// partners, and for the CTA holding the new row its k / v elements, loaded while the table is computed.
template <int D, int G>
struct RopeRegs {
    static constexpr int QE = (G * D + kThreads - 1) / kThreads;  // query elements per thread
    float qx[QE], qp[QE];
    float nx[8], np[8];  // new row: 8 elements of one 16-byte chunk of k or v, and (k) their partners
};

template <int D, int G>
__device__ __forceinline__ void rope_load(const DecodeArgs& a, int seq, int kvh, bool has_new_row, int tid,
                                          RopeRegs<D, G>& r) {
    const int64_t qbase = static_cast<int64_t>(seq) * a.q_seq_stride + static_cast<int64_t>(kvh * G) * D;
#pragma unroll
    for (int k = 0; k < RopeRegs<D, G>::QE; k++) {
        const int i = tid + k * kThreads;
        r.qx[k] = r.qp[k] = 0.f;
        if (i < G * D) {
            const int g = i / D, dim = i - g * D;
            bool first;
            const int pd = rope_partner(dim, D, a.interleaved, first);
            const int64_t o = qbase + static_cast<int64_t>(g) * D;
            if (a.q_f16) {
                r.qx[k] = __half2float(static_cast<const __half*>(a.q)[o + dim]);
                r.qp[k] = __half2float(static_cast<const __half*>(a.q)[o + pd]);
            } else {
                r.qx[k] = static_cast<const float*>(a.q)[o + dim];
                r.qp[k] = static_cast<const float*>(a.q)[o + pd];
            }
        }
    }
    constexpr int CH = D / 8;
    if (has_new_row && tid < 2 * CH) {
        const bool is_k = tid < CH;
        const int c = is_k ? tid : tid - CH;
        const float* src = (is_k ? a.k_new : a.v_new) + static_cast<int64_t>(seq) * a.new_seq_stride +
                           static_cast<int64_t>(kvh) * D;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const int dim = c * 8 + e;
            bool first;
            r.nx[e] = src[dim];
            r.np[e] = is_k ? src[rope_partner(dim, D, a.interleaved, first)] : 0.f;
        }
    }
}

// Part 2 (after the table): the rotated queries into s_q [G][D] (rounded to f16 when q is f16, as the in-place
// rotation stores them), and the new row — rotated k and raw v rounded to f16 — into the cache in global memory and
// straight into the unit's tiles (local row row - row0; swizzled chunks when kSwz).
template <int D, int G, bool kSwz>
__device__ __forceinline__ void rope_store(const DecodeArgs& a, int seq, int kvh, int row, int row0, __half* s_k,
                                           __half* s_v, float* s_q, const float2* cs, int tid,
                                           const RopeRegs<D, G>& r) {
#pragma unroll
    for (int k = 0; k < RopeRegs<D, G>::QE; k++) {
        const int i = tid + k * kThreads;
        if (i < G * D) {
            const int dim = i % D;
            float x = rope_rotate(r.qx[k], r.qp[k], dim, D, a.interleaved, cs);
            if (a.q_f16) x = __half2float(__float2half_rn(x));
            s_q[i] = x;
        }
    }
    constexpr int CH = D / 8;
    if (row < 0 || tid >= 2 * CH) return;
    const bool is_k = tid < CH;
    const int c = is_k ? tid : tid - CH;
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
        const int dim = c * 8 + e;
        const float x0 = is_k ? rope_rotate(r.nx[e], r.np[e], dim, D, a.interleaved, cs) : r.nx[e];
        const float x1 = is_k ? rope_rotate(r.nx[e + 1], r.np[e + 1], dim + 1, D, a.interleaved, cs) : r.nx[e + 1];
        const __half2 h = __floats2half2_rn(x0, x1);
        w[e / 2] = *reinterpret_cast<const uint32_t*>(&h);
    }
    const uint4 u = make_uint4(w[0], w[1], w[2], w[3]);
    const int rl = row - row0;
    const int cc = kSwz ? (c ^ (rl & 7)) : c;
    *reinterpret_cast<uint4*>((is_k ? s_k : s_v) + rl * D + cc * 8) = u;
    bool valid;
    const int64_t off = unit_offset(a, seq, kvh, row, D, valid);
    if (valid) *reinterpret_cast<uint4*>(const_cast<__half*>(is_k ? a.k : a.v) + off + c * 8) = u;
}

// ---- tensor-core form of a unit: mma.sync m16n8k16 (f16 operands, f32 accumulators) with split-precision A
// operands. Q·Kᵀ: A rows 0..7 hold f16(q) of the G heads and rows 8..15 the f16 remainder q - f16(q), so the two
// accumulator halves a lane holds (rows g and g+8) add up to the f32 score to ~2^-22 relative; K is f16 already.
// P·V: the same split of P (rows g / g+8), built straight from the score accumulators. Each warp owns SL/4 rows.

__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// (x0, x1) -> f16 pair hi and the f16 pair of the remainders lo.
__device__ __forceinline__ void split_f16x2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(x0 - hf.x, x1 - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// At head_dim 128 the four warps' P·V rows [4][G][D] are reduced in the K|V tiles (after one more barrier) rather
// than in a buffer of their own, which would cost a CTA per SM.
__host__ __device__ constexpr bool tc_red_aliases_kv(int D) { return D == 128; }

// kRope: the rotated queries of the G heads are in shared memory (s_q [G][D] f32) instead of global memory.
template <int D, int G, int kAfter, bool kRope = false>
__device__ __forceinline__ void compute_unit_tc(const DecodeArgs& a, int seq, int kvh, int split, int row0,
                                                int row_end, int nsplits, const __half* s_k, const __half* s_v,
                                                float* s_red, float* s_stat, const float* s_q, int tid, int warp,
                                                int lane) {
    constexpr int SL = Geo<D>::SL, RW = SL / 4, NT = RW / 8, KS = D / 16, DT = D / 8;
    static_assert(NT % 2 == 0 && KS % 2 == 0 && DT % 2 == 0, "tile shape");
    const int g = lane >> 2, t4 = lane & 3;
    const bool act = g < G;
    const int rbase = warp * RW;

    // A fragments of the scaled query (log2 units): hi rows 0..7, remainder rows 8..15; rows of absent heads are 0.
    uint32_t qa[KS][4];
    {
        const int64_t qoff = static_cast<int64_t>(seq) * a.q_seq_stride + static_cast<int64_t>(kvh * G + (act ? g : 0)) * D;
#pragma unroll
        for (int kk = 0; kk < KS; kk++) {
            float x[4];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int col = kk * 16 + h * 8 + t4 * 2;
                float2 v;
                if (kRope) v = *reinterpret_cast<const float2*>(s_q + (act ? g : 0) * D + col);
                else if (a.q_f16) v = __half22float2(*reinterpret_cast<const __half2*>(static_cast<const __half*>(a.q) + qoff + col));
                else v = *reinterpret_cast<const float2*>(static_cast<const float*>(a.q) + qoff + col);
                x[2 * h] = act ? v.x * a.scale_log2 : 0.f;
                x[2 * h + 1] = act ? v.y * a.scale_log2 : 0.f;
            }
            split_f16x2(x[0], x[1], qa[kk][0], qa[kk][1]);
            split_f16x2(x[2], x[3], qa[kk][2], qa[kk][3]);
        }
    }

    // S = Q·Kᵀ over this warp's RW rows.
    cp_async_wait<kAfter + 1>();
    __syncthreads();  // every thread's K chunks have landed
    float sc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
#pragma unroll
        for (int j = 0; j < 4; j++) sc[nt][j] = 0.f;
        const int row = rbase + nt * 8 + (lane & 7);
#pragma unroll
        for (int q2 = 0; q2 < KS / 2; q2++) {
            const int chunk = q2 * 4 + (lane >> 3);
            uint32_t b0, b1, b2, b3;
            ldsm_x4(s_k + row * D + ((chunk ^ (row & 7)) * 8), b0, b1, b2, b3);
            mma16816(sc[nt], qa[2 * q2], b0, b1);
            mma16816(sc[nt], qa[2 * q2 + 1], b2, b3);
        }
    }
    // scores of head g at rows rbase + nt*8 + t4*2 + {0, 1}: hi + remainder halves; rows past the context -> -inf
    float mloc = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const int r = row0 + rbase + nt * 8 + t4 * 2 + j;
            const float v = (r < row_end) ? sc[nt][j] + sc[nt][j + 2] : -INFINITY;
            sc[nt][j] = v;
            mloc = fmaxf(mloc, v);
        }
    mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 1));
    mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 2));
    float* s_mx = s_stat;          // [4][G] warp maxima
    float* s_sum = s_stat + 4 * G; // [4][G] warp sums
    if (act && t4 == 0) s_mx[warp * G + g] = mloc;
    __syncthreads();
    float m = -INFINITY;
    if (act) {
#pragma unroll
        for (int w = 0; w < 4; w++) m = fmaxf(m, s_mx[w * G + g]);
    }
    float lsum = 0.f;
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const float p = act ? ex2_approx(sc[nt][j] - m) : 0.f;  // masked rows: 2^-inf = 0
            sc[nt][j] = p;
            lsum += p;
        }
    lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
    lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
    if (act && t4 == 0) s_sum[warp * G + g] = lsum;

    // O += P·V over this warp's rows, all D columns.
    cp_async_wait<kAfter>();
    __syncthreads();  // every thread's V chunks have landed (and s_sum is written)
    float o[DT][4];
#pragma unroll
    for (int dt = 0; dt < DT; dt++)
#pragma unroll
        for (int j = 0; j < 4; j++) o[dt][j] = 0.f;
#pragma unroll
    for (int kk = 0; kk < NT / 2; kk++) {
        uint32_t pa[4];
        split_f16x2(sc[2 * kk][0], sc[2 * kk][1], pa[0], pa[1]);
        split_f16x2(sc[2 * kk + 1][0], sc[2 * kk + 1][1], pa[2], pa[3]);
        const int row = rbase + kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
        for (int d2 = 0; d2 < DT / 2; d2++) {
            const int chunk = d2 * 2 + (lane >> 4);
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(s_v + row * D + ((chunk ^ (row & 7)) * 8), b0, b1, b2, b3);
            mma16816(o[2 * d2], pa, b0, b1);
            mma16816(o[2 * d2 + 1], pa, b2, b3);
        }
    }
    if (tc_red_aliases_kv(D)) __syncthreads();  // s_red lies over the K|V tiles: every warp is done with V
    if (act) {
#pragma unroll
        for (int dt = 0; dt < DT; dt++)
            *reinterpret_cast<float2*>(s_red + (warp * G + g) * D + dt * 8 + t4 * 2) =
                make_float2(o[dt][0] + o[dt][2], o[dt][1] + o[dt][3]);
    }
    __syncthreads();

    // Sum the four warps' rows; finish single-split sequences, else store the partial state.
    const int64_t part_base = ((static_cast<int64_t>(seq) * a.n_kv_heads + kvh) * a.max_splits + split) * G;
    for (int o2 = tid; o2 < G * D; o2 += kThreads) {
        const int gg = o2 / D, col = o2 - gg * D;
        const float sacc = s_red[gg * D + col] + s_red[(G + gg) * D + col] + s_red[(2 * G + gg) * D + col] +
                           s_red[(3 * G + gg) * D + col];
        const float l = s_sum[gg] + s_sum[G + gg] + s_sum[2 * G + gg] + s_sum[3 * G + gg];
        if (nsplits == 1) {
            store_out_dec(a, seq, kvh * G + gg, D, col, sacc / l);
        } else {
            float* pp = a.partial + (part_base + gg) * (D + 2);
            pp[col] = sacc;
            if (col == 0) {
                pp[D] = fmaxf(fmaxf(s_mx[gg], s_mx[G + gg]), fmaxf(s_mx[2 * G + gg], s_mx[3 * G + gg]));
                pp[D + 1] = l;
            }
        }
    }
}

__device__ __forceinline__ void store_out_dec(const DecodeArgs& a, int seq, int head, int D, int col, float val) {
    const int64_t oo = static_cast<int64_t>(seq) * a.out_seq_stride + static_cast<int64_t>(head) * D + col;
    if (a.out_f16) static_cast<__half*>(a.out)[oo] = __float2half_rn(val);
    else static_cast<float*>(a.out)[oo] = val;
}

// One unit = SL cache rows of one KV head of one sequence, for its G query heads. kAfter = commit groups issued
// after this unit's two (the next unit's prefetch), so the waits below release exactly this unit's K, then V.
// s_red reuses this unit's K|V buffers after the last read of them.
template <int D, int G, int kAfter, bool kRope = false>
__device__ __forceinline__ void compute_unit(const DecodeArgs& a, int seq, int kvh, int split, int row0, int row_end,
                                             int nsplits, const __half* s_k, const __half* s_v, float* s_p,
                                             float* s_ml, const float* s_q, int tid, int warp, int lane, int lr,
                                             int rowlane) {
    using Gm = Geo<D>;
    constexpr int SL = Gm::SL, RPS = Gm::RPS, LPR = Gm::LPR;
    float* s_red = reinterpret_cast<float*>(const_cast<__half*>(s_k));  // [RPS][G][D] (K|V are contiguous)

    // Queries of the G heads (this lane's 8 dims), pre-scaled into log2 units.
    float qv[G][8];
#pragma unroll
    for (int g = 0; g < G; g++) {
        const int64_t qoff = static_cast<int64_t>(seq) * a.q_seq_stride + static_cast<int64_t>(kvh * G + g) * D + lr * 8;
        if (kRope) {
#pragma unroll
            for (int e = 0; e < 8; e++) qv[g][e] = s_q[g * D + lr * 8 + e];
        } else if (a.q_f16) {
            const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const __half*>(a.q) + qoff);
            half8_to_float(u, qv[g]);
        } else {
            const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(a.q) + qoff);
            const float4 x0 = p[0], x1 = p[1];
            qv[g][0] = x0.x; qv[g][1] = x0.y; qv[g][2] = x0.z; qv[g][3] = x0.w;
            qv[g][4] = x1.x; qv[g][5] = x1.y; qv[g][6] = x1.z; qv[g][7] = x1.w;
        }
#pragma unroll
        for (int e = 0; e < 8; e++) qv[g][e] *= a.scale_log2;
    }

    // Scores: partial dots, then the transposing row reduction; one lane per (row, head) stores it.
    cp_async_wait<kAfter + 1>();  // this thread's K chunks have landed
    float part[G][kSlots];
#pragma unroll
    for (int i = 0; i < kSlots; i++) {
        float kf[8];
        half8_to_float(*reinterpret_cast<const uint4*>(s_k + (i * RPS + rowlane) * D + lr * 8), kf);
#pragma unroll
        for (int g = 0; g < G; g++) {  // packed f32x2 FMAs: two dims per instruction
            float2 sc = make_float2(0.f, 0.f);
#pragma unroll
            for (int e = 0; e < 8; e += 2)
                sc = __ffma2_rn(make_float2(qv[g][e], qv[g][e + 1]), make_float2(kf[e], kf[e + 1]), sc);
            part[g][i] = sc.x + sc.y;
        }
    }
#pragma unroll
    for (int g = 0; g < G; g++) {
        int slot;
        const float sc = reduce_rows<LPR>(part[g], lane, slot);
        // lanes that share a slot after the plain-reduce tail hold equal values; the lowest one stores
        const bool writer = (LPR <= 8) || ((lr & (LPR / 8 - 1)) == 0);
        if (writer) {
            const int rl = slot * RPS + rowlane;
            s_p[g * SL + rl] = (row0 + rl < row_end) ? sc : -INFINITY;
        }
    }
    __syncthreads();

    // Softmax statistics per head over this unit (one warp per head).
    for (int g = warp; g < G; g += kThreads / 32) {
        float mx = -INFINITY;
        for (int r = lane; r < SL; r += 32) mx = fmaxf(mx, s_p[g * SL + r]);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.f;
        for (int r = lane; r < SL; r += 32) {
            const float p = ex2_approx(s_p[g * SL + r] - mx);  // masked rows: 2^-inf = 0
            s_p[g * SL + r] = p;
            sum += p;
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) {
            s_ml[2 * g] = mx;
            s_ml[2 * g + 1] = sum;
        }
    }
    cp_async_wait<kAfter>();  // this thread's V chunks have landed
    __syncthreads();

    // P·V over this thread's rows and dims.
    float2 acc2[G][4];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < 4; e++) acc2[g][e] = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < kSlots; i++) {
        float vf[8];
        const int rl = i * RPS + rowlane;
        half8_to_float(*reinterpret_cast<const uint4*>(s_v + rl * D + lr * 8), vf);
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float p = s_p[g * SL + rl];
            const float2 p2 = make_float2(p, p);
#pragma unroll
            for (int e = 0; e < 4; e++) acc2[g][e] = __ffma2_rn(p2, make_float2(vf[2 * e], vf[2 * e + 1]), acc2[g][e]);
        }
    }
    __syncthreads();  // every thread is done with K|V: the reduction buffer reuses them
#pragma unroll
    for (int g = 0; g < G; g++) {
        float4* dst = reinterpret_cast<float4*>(s_red + (rowlane * G + g) * D + lr * 8);
        dst[0] = make_float4(acc2[g][0].x, acc2[g][0].y, acc2[g][1].x, acc2[g][1].y);
        dst[1] = make_float4(acc2[g][2].x, acc2[g][2].y, acc2[g][3].x, acc2[g][3].y);
    }
    __syncthreads();

    // Reduce across row lanes; finish single-split sequences, else store the partial state.
    const int64_t part_base =
        ((static_cast<int64_t>(seq) * a.n_kv_heads + kvh) * a.max_splits + split) * G;
    for (int o = tid; o < G * D; o += kThreads) {
        const int g = o / D, col = o - g * D;
        float sacc = 0.f;
#pragma unroll
        for (int rl = 0; rl < RPS; rl++) sacc += s_red[(rl * G + g) * D + col];
        if (nsplits == 1) {
            const float val = sacc / s_ml[2 * g + 1];
            const int64_t oo = static_cast<int64_t>(seq) * a.out_seq_stride + static_cast<int64_t>(kvh * G + g) * D + col;
            if (a.out_f16) static_cast<__half*>(a.out)[oo] = __float2half_rn(val);
            else static_cast<float*>(a.out)[oo] = val;
        } else {
            float* pp = a.partial + (part_base + g) * (D + 2);
            pp[col] = sacc;
            if (col == 0) {
                pp[D] = s_ml[2 * g];
                pp[D + 1] = s_ml[2 * g + 1];
            }
        }
    }
}

// One CTA per (KV head x split, sequence) grid cell; CTAs past a sequence's context exit at once.
template <int D, int G, bool kTc, bool kRope>
__global__ void __launch_bounds__(kThreads, (G <= 4 ? 6 : 3)) decode_split_kernel(const DecodeArgs a) {
    using Gm = Geo<D>;
    constexpr int SL = Gm::SL, LPR = Gm::LPR, RPW = Gm::RPW;
    // KV heads vary fastest across the grid, so the CTAs reading the parts of the same cache rows run together
    // and DRAM sees whole rows streamed in order.
    const int split = blockIdx.x / a.n_kv_heads, kvh = blockIdx.x - split * a.n_kv_heads, seq = blockIdx.y;
    // Launched with programmatic dependent launch: the CTA may be resident before the previous kernel on the
    // stream has finished, so it touches no global memory before that kernel's writes are complete and visible.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // When the whole grid is resident at once, the combine kernel may launch as soon as every CTA has started: its
    // CTAs then wait in griddepcontrol.wait for this grid's memory, already resident when the last split ends
    // (two-split batches: 8.7 -> 7.6 us per layer). With several waves the release stays at the CTAs' end (early
    // release measured 23.5 against 22.7 us per config-3 layer).
    if (a.early_release) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int L = ctx_len_of(a, seq);
    const int row0 = split * SL;
    if (row0 >= L) return;  // uniform for the whole CTA
    const int row_end = min(L, row0 + SL);
    const int nsplits = (L + SL - 1) / SL;

    extern __shared__ __align__(16) uint8_t smem_b[];
    __half* s_k = reinterpret_cast<__half*>(smem_b);       // [SL][D] this unit's K rows
    __half* s_v = s_k + SL * D;                            // [SL][D] V rows
    float* s_p = reinterpret_cast<float*>(s_v + SL * D);   // [G][SL] scores, then probabilities
    float* s_ml = s_p + G * SL;                            // [G][2] unit max (log2 units), denominator

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int lr = lane % LPR, rowlane = warp * RPW + lane / LPR;
    float* s_red = tc_red_aliases_kv(D) ? reinterpret_cast<float*>(s_k) : s_p;  // tensor-core form
    float* s_stat = tc_red_aliases_kv(D) ? s_p : s_p + 4 * G * D;
    // Fused RoPE + append (kRope): [D/2] (cos, sin) after the statistics, and the G rotated query rows [G][D] f32 —
    // over the P·V reduction rows in the tensor-core form at head_dim 64 (read into registers before those are
    // written), after the table otherwise.
    float2* s_cs = reinterpret_cast<float2*>(kTc ? s_stat + 8 * G : s_ml + 2 * G);
    float* s_q = (kTc && !tc_red_aliases_kv(D)) ? s_red : reinterpret_cast<float*>(s_cs + D / 2);
    if constexpr (kRope) {
        // The sequence's new token is row L - 1; the CTA whose unit holds it writes that row itself.
        const int new_row = row_end == L ? L - 1 : -1;
        stage_unit<D, kTc, true>(a, seq, kvh, row0, row_end, s_k, s_v, lr, rowlane, new_row);
        RopeRegs<D, G> rr;
        rope_load<D, G>(a, seq, kvh, new_row >= 0, tid, rr);  // loads in flight with the unit's copies
        rope_table<D>(a, L - 1, s_cs, tid);
        __syncthreads();
        rope_store<D, G, kTc>(a, seq, kvh, new_row, row0, s_k, s_v, s_q, s_cs, tid, rr);
        __syncthreads();  // rotated queries and the new row are in shared memory before any thread reads them
    } else {
        stage_unit<D, kTc>(a, seq, kvh, row0, row_end, s_k, s_v, lr, rowlane);
    }
    if (kTc)
        compute_unit_tc<D, G, 0, kRope>(a, seq, kvh, split, row0, row_end, nsplits, s_k, s_v, s_red, s_stat, s_q, tid,
                                        warp, lane);
    else
        compute_unit<D, G, 0, kRope>(a, seq, kvh, split, row0, row_end, nsplits, s_k, s_v, s_p, s_ml, s_q, tid, warp,
                                     lane, lr, rowlane);
    // The combine kernel may start launching now; it waits for this grid's memory before reading.
    if (!a.early_release) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

constexpr int kCombineThreads = 256;
constexpr int kCombineSmem = 48 * 1024;  // staging budget per CTA (no opt-in attribute needed)

// Splits staged per round of the combine: [chunk][G][d + 2] records + [chunk][G] weights in kCombineSmem.
__host__ __device__ constexpr int combine_chunk(int G, int D) {
    return (kCombineSmem / 4 - G) / (G * (D + 2) + G);
}

// 8-byte async copy global -> shared.
__device__ __forceinline__ void cp_async8(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}

// One CTA per (KV head, sequence): the global max per head, then the split states staged into shared memory a
// chunk of splits at a time (every copy of a chunk in flight at once), weights 2^(m_s - M) once per (split, head),
// and every output column summed over the staged splits.
template <int D>
__global__ void __launch_bounds__(kCombineThreads) decode_combine_kernel(const DecodeArgs a) {
    const int kvh = blockIdx.x, seq = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = a.n_heads / a.n_kv_heads;
    // The context lengths are read before the wait for the split kernel: that kernel does not write them, and this
    // grid launches only once every split CTA has passed its own griddepcontrol.wait, so whatever wrote them
    // before the split kernel is complete and visible. The length read then overlaps the split grid's drain.
    const int L = ctx_len_of(a, seq);
    const int nsp = (L + Geo<D>::SL - 1) / Geo<D>::SL;
    // Every CTA waits for the split grid, single-split units included (they only return afterwards): this grid then
    // completes after the split kernel, so a later launch on the stream that reads `out` sees the split kernel's
    // writes even when no CTA has records to combine.
    asm volatile("griddepcontrol.wait;" ::: "memory");  // split kernel's writes are visible after this
    if (nsp <= 1) return;
    // The next stream-ordered kernel may launch now (it waits for this grid to finish before touching memory).
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int rec = G * (D + 2);                 // floats per split
    const int chunk = combine_chunk(G, D);
    extern __shared__ __align__(16) float cs[];
    float* s_rec = cs;                           // [chunk][G][D + 2]
    float* s_w = cs + chunk * rec;               // [chunk][G]
    float* s_max = s_w + chunk * G;              // [G]
    const float* base = a.partial + (static_cast<int64_t>(seq) * a.n_kv_heads + kvh) * a.max_splits * rec;
    const bool one_chunk = nsp <= chunk;
    if (one_chunk) {  // every split state staged in one round trip; the global max is then read from shared memory
        for (int i = tid; i < nsp * rec / 2; i += kCombineThreads) cp_async8(s_rec + 2 * i, base + 2 * i);
        asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
        __syncthreads();
    }
    for (int g = warp; g < G; g += kCombineThreads / 32) {
        float M = -INFINITY;
        for (int sp = lane; sp < nsp; sp += 32)
            M = fmaxf(M, one_chunk ? s_rec[sp * rec + g * (D + 2) + D] : __ldcg(base + sp * rec + g * (D + 2) + D));
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        if (lane == 0) s_max[g] = M;
    }
    constexpr int kMaxCols = (8 * D + kCombineThreads - 1) / kCombineThreads;  // G <= 8
    float num[kMaxCols], den[kMaxCols];
#pragma unroll
    for (int c = 0; c < kMaxCols; c++) num[c] = den[c] = 0.f;
    for (int c0 = 0; c0 < nsp; c0 += chunk) {
        const int nc = min(chunk, nsp - c0);
        if (!one_chunk) {
            const float* src = base + static_cast<int64_t>(c0) * rec;
            for (int i = tid; i < nc * rec / 2; i += kCombineThreads) cp_async8(s_rec + 2 * i, src + 2 * i);
            asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();  // staged records (and, first time round, s_max) visible
        for (int i = tid; i < nc * G; i += kCombineThreads) {
            const int sp = i / G, g = i - sp * G;
            s_w[i] = ex2_approx(s_rec[sp * rec + g * (D + 2) + D] - s_max[g]);
        }
        __syncthreads();
#pragma unroll
        for (int c = 0; c < kMaxCols; c++) {
            const int o = tid + c * kCombineThreads;
            if (o < G * D) {
                const int g = o / D, col = o - g * D;
                const float* r = s_rec + g * (D + 2);
                for (int sp = 0; sp < nc; sp++) {
                    const float w = s_w[sp * G + g];
                    num[c] = fmaf(r[sp * rec + col], w, num[c]);
                    den[c] = fmaf(r[sp * rec + D + 1], w, den[c]);
                }
            }
        }
        __syncthreads();  // chunk consumed before the next one is staged
    }
#pragma unroll
    for (int c = 0; c < kMaxCols; c++) {
        const int o = tid + c * kCombineThreads;
        if (o < G * D) {
            const int g = o / D, col = o - g * D;
            const float val = num[c] / den[c];
            const int64_t oo = static_cast<int64_t>(seq) * a.out_seq_stride + static_cast<int64_t>(kvh * G + g) * D + col;
            if (a.out_f16) static_cast<__half*>(a.out)[oo] = __float2half_rn(val);
            else static_cast<float*>(a.out)[oo] = val;
        }
    }
}

// Tensor-core unit compute at head_dim 64 (config-3 layer 26.2 -> 22.4 us); at head_dim 128 the packed-FMA form
// measured faster (51.1 against 54.0 us on the same batch) and stays. ALPACA_DECODE_MMA=0 / 1 forces either form.
bool decode_tensor_cores(int head_dim) {
    static const int v = [] {
        const char* e = std::getenv("ALPACA_DECODE_MMA");
        return e ? (e[0] == '0' ? 0 : 1) : -1;
    }();
    return v < 0 ? head_dim == 64 : v == 1;
}

template <int D, int G>
cudaError_t launch_split(const DecodeArgs& a, int n_seqs, int num_sms, cudaStream_t s) {
    using Gm = Geo<D>;
    static_assert(Gm::RPS * G * D * sizeof(float) <= sizeof(__half) * 2 * Gm::SL * D, "reduction buffer too big");
    const bool tc = decode_tensor_cores(D);
    // K and V tiles (2 * SL * D halves; the reduction buffer RPS*G*D floats fits inside them), scores, (m, l);
    // tensor-core form: K and V tiles, the four warps' P·V rows [4][G][D] and their (max, sum) [2][4][G]
    const size_t smem =
        (tc ? sizeof(__half) * 2 * Gm::SL * D + sizeof(float) * ((tc_red_aliases_kv(D) ? 0 : 4 * G * D) + 8 * G)
            : sizeof(__half) * 2 * Gm::SL * D + sizeof(float) * (G * Gm::SL + 2 * G)) +
        (a.rope ? sizeof(float2) * (D / 2) + ((tc && !tc_red_aliases_kv(D)) ? 0 : sizeof(float) * G * D) : 0);
    static_assert(4 * G * D * sizeof(float) <= sizeof(__half) * 2 * Gm::SL * D, "P·V rows must fit the K|V tiles");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.max_splits * a.n_kv_heads, n_seqs, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    const auto fn = tc ? (a.rope ? decode_split_kernel<D, G, true, true> : decode_split_kernel<D, G, true, false>)
                       : (a.rope ? decode_split_kernel<D, G, false, true> : decode_split_kernel<D, G, false, false>);
    // CTAs of this kernel form one SM holds (depends only on the form and its shared memory): one query per form.
    const int fidx = (tc ? 2 : 0) + (a.rope ? 1 : 0);
    static int occ[4] = {0, 0, 0, 0};
    static std::once_flag occ_once[4];
    std::call_once(occ_once[fidx], [&] {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kThreads, smem) == cudaSuccess) occ[fidx] = n;
    });
    DecodeArgs la = a;
    la.early_release = static_cast<int64_t>(a.max_splits) * a.n_kv_heads * n_seqs <=
                       static_cast<int64_t>(occ[fidx]) * num_sms;
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    // Six CTAs of ~37 KB per SM need the whole shared-memory carve-out; without a preference the driver may pick a
    // smaller one (more L1) for a kernel with a stack frame, and fewer CTAs fit.
    const cudaError_t ce = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                                cudaFuncAttributePreferredSharedMemoryCarveout,
                                                static_cast<int>(cudaSharedmemCarveoutMaxShared));
    if (ce != cudaSuccess) return ce;
    return cudaLaunchKernelEx(&cfg, fn, la);
}

template <int D>
cudaError_t launch_d(const DecodeArgs& a, int n_seqs, int num_sms, cudaStream_t s) {
    cudaError_t e;
    switch (a.n_heads / a.n_kv_heads) {
        case 1: e = launch_split<D, 1>(a, n_seqs, num_sms, s); break;
        case 2: e = launch_split<D, 2>(a, n_seqs, num_sms, s); break;
        case 3: e = launch_split<D, 3>(a, n_seqs, num_sms, s); break;
        case 4: e = launch_split<D, 4>(a, n_seqs, num_sms, s); break;
        case 5: e = launch_split<D, 5>(a, n_seqs, num_sms, s); break;
        case 6: e = launch_split<D, 6>(a, n_seqs, num_sms, s); break;
        case 7: e = launch_split<D, 7>(a, n_seqs, num_sms, s); break;
        case 8: e = launch_split<D, 8>(a, n_seqs, num_sms, s); break;
        default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    if (a.max_splits <= 1) return cudaSuccess;  // every sequence finished in the split kernel
    const int G = a.n_heads / a.n_kv_heads;
    const int chunk = combine_chunk(G, D);
    const size_t csmem = sizeof(float) * (static_cast<size_t>(chunk) * (G * (D + 2) + G) + G);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_kv_heads, n_seqs, 1);
    cfg.blockDim = dim3(kCombineThreads, 1, 1);
    cfg.dynamicSmemBytes = csmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_combine_kernel<D>, a);
}

// Built-in decode scratch for alpaca_attn_decode_noalloc: a file-scope device array, so that entry point never
// asks for device memory. Every device that loads the library holds these bytes until the process exits; all
// calls on a device share them.
static __device__ __align__(256) float g_decode_scratch[kDecodeBuiltinScratchBytes / sizeof(float)];

constexpr int kMaxScratchDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxScratchDevices] = {};

}  // namespace

// Device address of the built-in scratch on the current device. The first call on a device looks it up with
// cudaGetSymbolAddress (with that device current) and caches it; later calls only read the cache.
cudaError_t decode_builtin_scratch(void** ptr) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxScratchDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[dev] = p;
    }
    *ptr = g_scratch_ptr[dev];
    return cudaSuccess;
}

int decode_split_len(int head_dim) { return head_dim == 128 ? Geo<128>::SL : Geo<64>::SL; }

int decode_max_splits(const alpaca_attn_desc& d) {
    const int L = d.ctx_lens ? d.max_ctx_len : d.start_position + 1;
    const int sl = decode_split_len(d.head_dim);
    return (L + sl - 1) / sl;
}

size_t decode_workspace_bytes(const alpaca_attn_desc& d) {
    const int ms = decode_max_splits(d);
    if (ms <= 1) return 0;
    return sizeof(float) * static_cast<size_t>(d.n_seqs) * d.n_heads * ms * (d.head_dim + 2);
}

bool decode_supported(const alpaca_attn_desc& d) {
    if (d.head_dim != 64 && d.head_dim != 128) return false;
    if (d.n_kv_heads <= 0 || d.n_heads % d.n_kv_heads != 0) return false;
    const int G = d.n_heads / d.n_kv_heads;
    return G >= 1 && G <= kMaxGroup && d.kv_dtype == ALPACA_F16 && d.tokens == 1;
}

cudaError_t launch_decode(const Call& c, cudaStream_t s) {
    const alpaca_attn_desc& d = *c.d;
    DecodeArgs a;
    a.q = d.q;
    a.q_seq_stride = d.q_seq_stride;
    a.q_f16 = d.q_dtype == ALPACA_F16;
    a.k = static_cast<const __half*>(d.k);
    a.v = static_cast<const __half*>(d.v);
    a.kv_row_stride = d.kv_row_stride;
    a.kv_seq_stride = d.kv_seq_stride;
    a.out = d.out;
    a.out_seq_stride = d.out_seq_stride;
    a.out_f16 = d.out_dtype == ALPACA_F16;
    a.partial = static_cast<float*>(c.ws);
    a.ctx_lens = d.ctx_lens;
    a.uniform_len = d.start_position + 1;
    a.max_len = d.ctx_lens ? d.max_ctx_len : a.uniform_len;
    a.n_heads = d.n_heads;
    a.n_kv_heads = d.n_kv_heads;
    a.max_splits = decode_max_splits(d);
    a.scale_log2 = c.scale * kLog2e;
    a.block_table = d.block_table;
    a.block_rows = d.block_rows;
    a.max_blocks = d.max_blocks;
    a.pool_blocks = d.pool_blocks;
    a.block_stride = d.block_stride;
    a.err = c.err;
    a.early_release = 0;  // set per launch in launch_split
    a.rope = c.rope ? 1 : 0;
    a.interleaved = 0;
    a.k_new = a.v_new = nullptr;
    a.new_seq_stride = 0;
    for (int i = 0; i < 128; i++) a.freq[i] = 0.0;
    if (c.rope) {  // frequencies exactly as alpaca_rope_kv_append computes them
        const alpaca_rope_desc& r = *c.rope;
        a.interleaved = r.interleaved;
        a.k_new = r.k;
        a.v_new = r.v;
        a.new_seq_stride = r.kv_seq_stride;
        const double theta = static_cast<double>(r.theta);
        for (int i = 0; i < d.head_dim / 2; i++)
            a.freq[i] = std::pow(theta, -2.0 * static_cast<double>(i) / static_cast<double>(d.head_dim));
    }
    if (a.max_splits < 1) return cudaSuccess;
    return d.head_dim == 128 ? launch_d<128>(a, d.n_seqs, c.num_sms, s) : launch_d<64>(a, d.n_seqs, c.num_sms, s);
}

}  // namespace alpaca
