// attn_prefill_sm100.cu — causal grouped-query flash attention for prefill on B200 tensor cores (tcgen05).
//
// Same computation as alpaca.swift's attn_tensor_* / attn_prefill_* kernels (Sources/AlpacaMetal/Kernels/
// tensor_attention.metal:29-117, attention_prefill.metal:31-182): f16 Q/K/V, S = Q·Kᵀ with f32 accumulation,
// online softmax, P rounded to f16, O += P·V with f32 accumulation, causal block skip, mask only on diagonal
// blocks, final 1/l. The structure is B200-native:
//
//   * persistent kernel, one CTA per SM, work items = (sequence, head, pair of 128-row query tiles A and B)
//     ordered heaviest first (items with more visible KV blocks come first) and dealt to the CTAs in serpentine
//     rounds, so the causal triangle is balanced over the 148 SMs even when there are few items per SM;
//   * head_dim 64 (128-row KV blocks) and 128 (64-row KV blocks, so S, O and P of both tiles fit TMEM); rows of Q,
//     K and V are stored as head_dim/64 column blocks of 128 bytes;
//   * warp 0: TMA producer. Q tiles and a 3-stage ring of K/V blocks land in shared memory with 128-byte swizzle,
//     no multicast;
//   * warps 1 and 2: one thread each issues tcgen05.mma for tile A / B: S = Q·Kᵀ (A and B from shared memory)
//     into TMEM, and O += P·V with P read from TMEM (A operand in tensor memory, B = V from shared memory), so
//     P never touches shared memory and the tensor core's shared-memory reads stay within bandwidth. Each issuer
//     queues S(j+1) before PV(j), so the next S block is ready when the softmax finishes the current one;
//   * head_dim 64: warps 4-11 and 12-19: softmax for tile A and B, two threads per query row (one per half of the
//     S block row). head_dim 128: warps 4-7 and 8-11, one thread per query row (the same steps without the
//     exchange of partial row maxima and sums; 384 threads, registers from the launch bound). They read S from TMEM, mask diagonal blocks and keep the running max in log2 units
//     (it only moves when it grows by more than 8, so O rarely needs rescaling). Each half computes its P
//     against its own candidate max and only then reads the other half's candidate (shared memory, a
//     two-arrival mbarrier per pair of warps that share TMEM lanes), so the exchange is off the critical path;
//     the half with the lower candidate scales its f16 P pairs down. P = 2^(s*c - m) — most exponentials on
//     MUFU, a fixed share on the FMA pipe with a polynomial — is summed per row in f32, stored to TMEM as f16
//     pairs, and each tile ends with O / l, written into a shared-memory staging tile (128-byte swizzle) and sent
//     to global memory by one thread's TMA stores (mbarrier hand-offs with bounded waits; rows past the tokens are
//     clipped by the tensor map);
//   * registers (two-thread form): the control warpgroup drops to 56 per thread (setmaxnreg) so the softmax warps
//     get 104; the one-thread form takes up to 168 per thread from its launch bound.
//   * an alternative head_dim-64 form (template parameter NT = 3, switch ALPACA_PREFILL_TILES=3): work items of
//     three query tiles with 64-row KV blocks and one softmax thread per row (warps 4-15, issuers in warps 1-3),
//     so each SMSP holds three independent softmax phase groups; 2 of 8 exponential pairs on the FMA pipe.
//   TMEM (see PG): d=64: S_A 0-127, S_B 128-255, O_A 256-319, O_B 320-383, P_A 384-447, P_B 448-511;
//                  d=128: S_A 0-63, S_B 64-127, O_A 128-255, O_B 256-383, P_A 384-415, P_B 416-447.
//
// Every mbarrier wait is bounded (2 s; 2 ms under ALPACA_ATTN_FLAG_DEBUG_FORCE_TIMEOUT). On a timeout the CTA
// raises its abort flag and the device error word, waits (bounded) for its own TMA loads and MMAs in flight,
// frees TMEM and returns.
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace alpaca {
namespace {

constexpr int kBM = 128;        // query rows per tile
// K/V ring depth: 3 (as fast as 4 at head_dim 64, and it leaves room for the output staging tiles).
template <int D, int NT>
__host__ __device__ constexpr int stages_for() { return NT == 3 ? 4 : 3; }
// The default forms (head_dim 64 with two softmax threads per row, head_dim 128 with one) write the output through
// shared-memory staging tiles and TMA stores.
template <int D, int R, int NT>
__host__ __device__ constexpr bool tma_out() { return (D == 64 && R == 2) || (D == 128 && R == 1) || NT == 3; }
// Threads per CTA: warps 0-3 are the TMA producer, the MMA issuers of the NT query tiles (warp 2 also allocates
// TMEM) and, with two tiles, an idle warp; then 4 R softmax warps per tile (R threads per query row).
template <int R, int NT>
__host__ __device__ constexpr int threads_for() { return 32 * (4 + 4 * R * NT); }
constexpr int kThreads = threads_for<2, 2>();
constexpr int kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;      // log2 units
constexpr int kMaxKvSplits = 8;                // split-KV parts of a work item at most

// Geometry per head dim and number of query tiles per work item (NT). Rows of Q, K and V live in shared memory as
// D/64 column blocks [rows][64] (128 bytes per row, 128-byte swizzle), the layout a 64 x 1 x rows x 1 TMA box
// writes. d = 64 with two tiles: 128-row KV blocks; d = 128, and d = 64 with three tiles: 64-row KV blocks, so that
// S, O and P of every tile fit the 512 TMEM columns.
//   TMEM: S_t at t BN, O_t (D columns) at NT BN + t D, P_t (BN/2 columns of f16 pairs) at NT (BN + D) + t BN/2:
//   d = 64, two tiles: S 0 / 128, O 256 / 320, P 384 / 448;  d = 128: S 0 / 64, O 128 / 256, P 384 / 416;
//   d = 64, three tiles: S 0 / 64 / 128, O 192 / 256 / 320, P 384 / 416 / 448.
template <int D, int NT = 2>
struct PG {
    static_assert(D == 64 || D == 128, "head_dim 64 or 128");
    static_assert(NT == 2 || (NT == 3 && D == 64), "three query tiles at head_dim 64 only");
    static constexpr int BN = (D == 64 && NT == 2) ? 128 : 64;  // KV rows per block
    static constexpr int CB = D / 64;              // 64-column blocks per row
    static constexpr int SC = BN / 2;              // S columns per softmax thread (half a block row)
    static constexpr int OC = D / 2;               // O columns per softmax thread
    static constexpr uint32_t kQBytes = kBM * D * 2;
    static constexpr uint32_t kKVBytes = BN * D * 2;
    __host__ __device__ static constexpr uint32_t col_s(int tile) { return tile * BN; }
    __host__ __device__ static constexpr uint32_t col_o(int tile) { return NT * BN + tile * D; }
    __host__ __device__ static constexpr uint32_t col_p(int tile) { return NT * (BN + D) + tile * (BN / 2); }
    static_assert(NT * (BN + D + BN / 2) <= kTmemCols, "TMEM map exceeds 512 columns");
};
// Register split after the role dispatch (setmaxnreg): the control warpgroup (warps 0-3) gives registers to
// the four softmax warpgroups (128 * 56 + 512 * 104 of the 640 x 96 registers the CTA is launched with).
constexpr uint32_t kRegsControl = 56, kRegsSoftmax = 104;
static_assert(128 * kRegsControl + 512 * kRegsSoftmax <= kThreads * 96, "register split exceeds the launch budget");
// Three-tile form: 512 threads launched at 128 registers; the three softmax warpgroups take 152.
constexpr uint32_t kRegsSoftmax3 = 152;
static_assert(128 * kRegsControl + 384 * kRegsSoftmax3 <= 512 * 128, "register split exceeds the launch budget");
constexpr float kLog2e = 1.4426950408889634f;

struct PrefillArgs {
    void* out;
    int64_t out_token_stride, out_seq_stride;
    int out_f16;
    int n_seqs, n_heads, n_kv_heads, tokens, start, kv_len;
    int n_groups, total_items;  // groups of NT query tiles per (sequence, head); work items
    float scale_log2;
    unsigned* err;
    unsigned flags;
    // Split KV (calls with fewer work items than SMs): each item's KV blocks are cut into kv_splits parts (a ragged
    // unit into as many as its own blocks allow, unit_parts), each part an item of its own that leaves its
    // unnormalised rows and their (max, sum) in `part` ([item][tile][row][D + 2] f32), and prefill_merge_kernel
    // writes the output; a ragged unit left whole writes its output itself. kv_splits = 1 otherwise.
    int kv_splits;
    float* part;
    const int* block_table;  // paged cache: [seq][max_blocks] (null: contiguous caches)
    int block_rows, max_blocks, pool_blocks, last_block;  // last_block: block (of a sequence) holding row kv_len - 1
    // Ragged form: the work list the plan kernel wrote into the workspace. plan[0].x = units; unit u is
    // plan[1 + 2u] = {sequence, packed row of its first query, absolute position of that query, query rows} and
    // plan[2 + 2u].x = the sequence's context end (start + tokens). Sequences heaviest first, each one's units
    // together and heaviest first.
    const int4* plan;
};

template <int D, int NT = 2>
struct SmemLayout {
    static constexpr int kStages = stages_for<D, NT>();
    __half q[NT][kBM * D];                // [tile][column block][row][64]
    // per tile, 64 columns of the normalised output [128 rows][64] as TMA store boxes of 128-byte rows with the
    // 128-byte swizzle (f32: two boxes of 32 columns; f16: one box of 64); head_dim 128 stages it in two rounds
    float o_stage[NT * kBM * 64];
    __half k[kStages][PG<D, NT>::BN * D];  // [stage][column block][row][64]
    __half v[kStages][PG<D, NT>::BN * D];
    uint64_t q_full[NT], q_empty[NT];
    uint64_t k_full[kStages], k_empty[kStages], v_full[kStages], v_empty[kStages];
    uint64_t v_ready[kStages];  // ragged form: V rows past the sequence's context zeroed (warp 3), P·V may read
    uint64_t s_full[NT], s_empty[NT], p_full[NT], o_done[NT];
    uint64_t xbar[2][4];       // per (tile, lane quarter): the two half-row warps exchange partial row state
    uint64_t dbg, fin[NT], retire;
    uint64_t o_staged[NT], o_free[NT];  // output: rows staged (the tile's softmax warps), staging free again (issuer)
    // two-thread form (head_dim 64 only): exchanged partial row maxima and sums
    static constexpr int kXR = (D == 64 && NT == 2) ? kBM : 1;
    float xmax[2][2][2][kXR];  // [tile][exchange parity][half][row]
    float xl[2][2][kXR];       // [tile][half][row] (epilogue)
    uint32_t tmem_base;
    int abort_flag;
};

template <int D, int NT = 2>
constexpr size_t smem_bytes() { return sizeof(SmemLayout<D, NT>) + 1024; }  // + alignment slack
static_assert(smem_bytes<64>() <= 232448 && smem_bytes<128>() <= 232448 && smem_bytes<64, 3>() <= 232448,
              "shared memory exceeds 227 KB per CTA");

// One work item: NT query tiles of 128 rows of one (sequence, head). First NT entries of the arrays used.
struct Item {
    int seq, head;  // sequence (cache / block-table index) and query head
    int cseq;       // sequence coordinate of the Q and output tensor maps (0 in the packed ragged layout)
    int row0[3];    // Q / output map row of each tile's first query
    int pos0[3];    // absolute position of each tile's first query
    int nrows[3];   // query rows of each tile that exist (ragged form; the uniform form clips through the maps)
    int nblk[3];    // KV blocks each tile attends to
    int ctx_end;    // ragged form: the sequence's context end; rows at or past it are never used
    int jb0, jb1;   // KV blocks [jb0, jb1) of this item (of its part, with split KV; else 0 .. the most of any tile)
};

// Split-KV parts a ragged unit of `nmax` KV blocks uses out of the call's `splits`: at least 4 blocks per part (the
// host sizes `splits` from the call's bounds, and a unit near the start of its sequence has few blocks).
__host__ __device__ __forceinline__ int unit_parts(int splits, int nmax) { return max(1, min(splits, nmax / 4)); }

template <int BN>
__device__ __forceinline__ int tile_blocks(const PrefillArgs& a, int row0) {
    if (row0 >= a.tokens) return 0;
    const int last_row = min(row0 + kBM, a.tokens);  // exclusive
    const int visible = a.start + last_row;          // KV rows visible to the tile's last row
    return (visible + BN - 1) / BN;
}

template <int BN, int NT, bool VL, bool KS = false>
__device__ __forceinline__ Item decode_item(const PrefillArgs& a, int it) {
    Item x;
    if constexpr (VL) {
        // unit-major (then, split KV, its parts), head-minor: consecutive items share the unit's queries and (within
        // a KV head) its K/V
        const int slot = it / a.n_heads;
        const int unit = KS ? slot / a.kv_splits : slot;
        const int part = KS ? slot - unit * a.kv_splits : 0;
        x.head = it - slot * a.n_heads;
        const int4 r = __ldg(a.plan + 1 + 2 * unit);
        x.seq = r.x;
        x.cseq = 0;
        x.ctx_end = __ldg(a.plan + 2 + 2 * unit).x;
#pragma unroll
        for (int t = 0; t < NT; t++) {
            x.row0[t] = r.y + t * kBM;
            x.pos0[t] = r.z + t * kBM;
            x.nrows[t] = max(0, min(kBM, r.w - t * kBM));
            x.nblk[t] = x.nrows[t] > 0 ? (x.pos0[t] + x.nrows[t] + BN - 1) / BN : 0;
        }
        int nmax = x.nblk[0];
#pragma unroll
        for (int t = 1; t < NT; t++) nmax = max(nmax, x.nblk[t]);
        if constexpr (KS) {
            const int up = unit_parts(a.kv_splits, nmax);  // parts at or past `up` hold no block
            x.jb0 = part < up ? part * nmax / up : nmax;
            x.jb1 = part < up ? (part + 1) * nmax / up : nmax;
        } else {
            x.jb0 = 0;
            x.jb1 = nmax;
        }
        return x;
    }
    const int per_rank = a.n_seqs * a.n_heads;
    const int slot = it / per_rank, rem = it - slot * per_rank;
    // heaviest groups first, then (split KV) their parts; without the split the part range is the whole, as constants
    const int splits = KS ? a.kv_splits : 1;
    const int group = a.n_groups - 1 - (KS ? slot / splits : slot);
    const int part = KS ? slot - (slot / splits) * splits : 0;
    x.seq = rem / a.n_heads;
    x.head = rem - x.seq * a.n_heads;
    x.cseq = x.seq;
    x.ctx_end = a.kv_len;
    int nmax = 0;
#pragma unroll
    for (int t = 0; t < NT; t++) {
        x.row0[t] = (group * NT + t) * kBM;
        x.pos0[t] = a.start + x.row0[t];
        x.nrows[t] = kBM;
        x.nblk[t] = tile_blocks<BN>(a, x.row0[t]);
        nmax = max(nmax, x.nblk[t]);
    }
    x.jb0 = KS ? part * nmax / splits : 0;
    x.jb1 = KS ? (part + 1) * nmax / splits : nmax;
    return x;
}

// One tile of work item `it`, as the softmax warps of tile `t` (a run-time, warp-uniform index) need it: scalar
// fields, so they live in registers (an Item indexed by a run-time tile would sit in local memory).
struct TileWork {
    int seq, head, cseq, row0, pos0, nrows, nblk;
    int jb0, jb1;  // this tile's KV blocks [jb0, jb1) in the item (its part; empty when jb1 <= jb0)
    bool rec;      // split KV: the item is one of several parts and writes a record, not the output
};

template <int BN, int NT, bool VL, bool KS = false>
__device__ __forceinline__ TileWork tile_work(const PrefillArgs& a, int it, int t) {
    TileWork w;
    if constexpr (VL) {
        const int slot = it / a.n_heads;  // as decode_item
        const int unit = KS ? slot / a.kv_splits : slot;
        const int part = KS ? slot - unit * a.kv_splits : 0;
        w.head = it - slot * a.n_heads;
        const int4 r = __ldg(a.plan + 1 + 2 * unit);
        w.seq = r.x;
        w.cseq = 0;
        w.row0 = r.y + t * kBM;
        w.pos0 = r.z + t * kBM;
        w.nrows = max(0, min(kBM, r.w - t * kBM));
        w.nblk = w.nrows > 0 ? (w.pos0 + w.nrows + BN - 1) / BN : 0;
        if constexpr (KS) {
            int nmax = 0;
#pragma unroll
            for (int u = 0; u < NT; u++) {
                const int rows = max(0, min(kBM, r.w - u * kBM));
                nmax = max(nmax, rows > 0 ? (r.z + u * kBM + rows + BN - 1) / BN : 0);
            }
            const int up = unit_parts(a.kv_splits, nmax);
            w.jb0 = part < up ? part * nmax / up : nmax;
            w.jb1 = part < up ? min(w.nblk, (part + 1) * nmax / up) : nmax;
            w.rec = up > 1;  // a unit left whole writes its output as the unsplit form does
        } else {
            w.jb0 = 0;
            w.jb1 = w.nblk;
            w.rec = false;
        }
        return w;
    }
    const int per_rank = a.n_seqs * a.n_heads;
    const int slot = it / per_rank, rem = it - slot * per_rank;
    const int splits = KS ? a.kv_splits : 1;  // as decode_item
    const int group = a.n_groups - 1 - (KS ? slot / splits : slot);
    const int part = KS ? slot - (slot / splits) * splits : 0;
    w.seq = rem / a.n_heads;
    w.head = rem - w.seq * a.n_heads;
    w.cseq = w.seq;
    w.row0 = (group * NT + t) * kBM;
    w.pos0 = a.start + w.row0;
    w.nrows = kBM;
    w.nblk = tile_blocks<BN>(a, w.row0);
    if constexpr (KS) {
        // the item's block count is its last existing tile's (later tiles see more positions)
        int nmax = 0;
#pragma unroll
        for (int u = 0; u < NT; u++) nmax = max(nmax, tile_blocks<BN>(a, (group * NT + u) * kBM));
        w.jb0 = part * nmax / splits;
        w.jb1 = min(w.nblk, (part + 1) * nmax / splits);
    } else {
        w.jb0 = 0;
        w.jb1 = w.nblk;
    }
    w.rec = KS;  // a uniform split call cuts every item into its `splits` parts
    return w;
}

// ---------------------------------------------------------------------------------------------- MMA helpers

// S_t = Q_t · K_stageᵀ: M=128, N=BN, K=D (D/16 steps of 16); both operands K-major, 128-byte swizzle. K step kk
// lies in column block kk/4 at byte offset (kk%4)*32 of each 128-byte row.
template <int D, int NT>
__device__ __forceinline__ void mma_s(const SmemLayout<D, NT>* sm, int tile, int stage, uint32_t tmem_base) {
    using G = PG<D, NT>;
    constexpr uint32_t idesc = idesc_f16_f32(kBM, G::BN, false, false);
    const uint32_t qa = smem_u32(sm->q[tile]), ka = smem_u32(sm->k[stage]);
#pragma unroll
    for (int kk = 0; kk < D / 16; kk++) {
        const uint64_t ad = smem_desc_sw128(qa + (kk >> 2) * (kBM * 128) + (kk & 3) * 32, 16, 1024);
        const uint64_t bd = smem_desc_sw128(ka + (kk >> 2) * (G::BN * 128) + (kk & 3) * 32, 16, 1024);
        tc_mma_ss(tmem_base + G::col_s(tile), ad, bd, idesc, kk > 0 ? 1u : 0u);
    }
}

// O_t (+)= P_t · V_stage: M=128, N=D, K=BN (BN/16 steps of 16). P in TMEM (8 columns of f16 pairs per step), V
// MN-major in shared memory: 16 KV rows = 2 KB per step, the next 64-column block BN*128 bytes further (LBO).
template <int D, int NT>
__device__ __forceinline__ void mma_pv(const SmemLayout<D, NT>* sm, int tile, int stage, uint32_t tmem_base,
                                       bool accumulate) {
    using G = PG<D, NT>;
    constexpr uint32_t idesc = idesc_f16_f32(kBM, D, false, true);
    const uint32_t va = smem_u32(sm->v[stage]);
#pragma unroll
    for (int kk = 0; kk < G::BN / 16; kk++) {
        const uint64_t bd = smem_desc_sw128(va + kk * 16 * 128, G::BN * 128, 1024);
        tc_mma_ts(tmem_base + G::col_o(tile), tmem_base + G::col_p(tile) + kk * 8, bd, idesc,
                  (accumulate || kk > 0) ? 1u : 0u);
    }
}

// ---------------------------------------------------------------------------------------------- kernel

template <int D, int kEmuPairs, int R, int NT, bool VL = false, bool KS = false>
__global__ void __launch_bounds__(threads_for<R, NT>(), 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_kt,
                   const __grid_constant__ CUtensorMap tm_vt, const __grid_constant__ CUtensorMap tm_o,
                   const PrefillArgs a) {
    using G = PG<D, NT>;
    constexpr int kStages = stages_for<D, NT>();
    constexpr bool kTmaOut = tma_out<D, R, NT>();
    static_assert(D == 64 || R == 1, "head_dim 128 is built in the one-thread-per-row form only");
    static_assert(!KS || NT == 2, "split KV in the two-tile forms only");
    static_assert(NT == 2 || R == 1, "three query tiles in the one-thread-per-row form only");
    constexpr int kBN = G::BN, SC = G::SC, OC = G::OC;
    extern __shared__ uint8_t smem_raw[];
    auto* sm = reinterpret_cast<SmemLayout<D, NT>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // The next stream-ordered kernel may launch now; it waits for this grid to finish before touching memory.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const bool debug_timeout = (a.flags & ALPACA_ATTN_FLAG_DEBUG_FORCE_TIMEOUT) != 0;
    AbortState ab{&sm->abort_flag, a.err, debug_timeout ? kDebugWaitLimitNs : kWaitLimitNs};
    // Items are dealt in serpentine rounds (CTA c takes item c of even rounds and item gridDim.x-1-c of odd ones),
    // so the CTA that draws the heaviest item of one round draws the lightest of the next. Every role of the CTA
    // walks the same sequence.
    const auto item_of = [&](int r) {
        return r * static_cast<int>(gridDim.x) + ((r & 1) ? static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x)
                                                          : static_cast<int>(blockIdx.x));
    };

    if (tid == 0) {
        sm->abort_flag = 0;
        for (int i = 0; i < NT; i++) {
            mbar_init(&sm->q_full[i], 1);
            mbar_init(&sm->q_empty[i], 1);
            mbar_init(&sm->s_full[i], 1);
            mbar_init(&sm->s_empty[i], 4 * R);  // one arrival per softmax warp of the tile
            mbar_init(&sm->p_full[i], 4 * R);
            mbar_init(&sm->o_done[i], 1);
            mbar_init(&sm->fin[i], 1);
            mbar_init(&sm->o_staged[i], 4 * R);  // the tile's softmax warps
            mbar_init(&sm->o_free[i], 1);
        }
        for (int i = 0; i < 2; i++)
            for (int qq = 0; qq < 4; qq++) mbar_init(&sm->xbar[i][qq], 2);  // one arrival per warp of the pair
        for (int i = 0; i < kStages; i++) {
            mbar_init(&sm->k_full[i], 1);
            mbar_init(&sm->k_empty[i], NT);  // released by every tile's MMA issuer
            mbar_init(&sm->v_full[i], 1);
            mbar_init(&sm->v_empty[i], NT);
            mbar_init(&sm->v_ready[i], 1);
        }
        mbar_init(&sm->dbg, 1);
        mbar_init(&sm->retire, 4 * R * NT + 2);  // the softmax warps, the producer and tile 0's issuer
        fence_barrier_init();
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_k);
        tma_prefetch_desc(&tm_v);
        if (kTmaOut) tma_prefetch_desc(&tm_o);
        if (a.block_table) {
            tma_prefetch_desc(&tm_kt);
            tma_prefetch_desc(&tm_vt);
        }
    }
    if (warp == 2) {
        tmem_alloc(&sm->tmem_base, kTmemCols);
        tmem_relinquish();
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    // Launched with programmatic dependent launch: barriers, TMEM and tensor maps are set up while the previous
    // kernel on the stream drains; no global memory is touched before its writes are complete and visible.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t tmem_base = sm->tmem_base;
    // Work items: fixed by the call's shape, or (ragged form) units of the plan the previous launch wrote x heads.
    const int total_items = VL ? __ldg(&a.plan[0].x) * a.n_heads * (KS ? a.kv_splits : 1) : a.total_items;
    if (warp == 0) {
        if constexpr (R == 2 || NT == 3) setmaxnreg_dec<kRegsControl>();
        if (lane != 0) return;
        // ------------------------------------------------------------------ TMA producer
        uint32_t kv_it = 0, k_issued = 0, v_issued = 0, q_uses[NT] = {};
        bool ok = true;
        for (int r = 0, it = item_of(0); ok && it < total_items; it = item_of(++r)) {
            const Item x = decode_item<kBN, NT, VL, KS>(a, it);
            const int kvh = x.head / (a.n_heads / a.n_kv_heads);
#pragma unroll
            for (int t = 0; t < NT; t++) {  // unrolled: the Item and q_uses stay in registers
                if (!ok || min(x.nblk[t], x.jb1) <= x.jb0) continue;  // no KV block of this tile in the item
                ok = mbar_wait(&sm->q_empty[t], (q_uses[t] & 1) ^ 1, ab);
                if (!ok) continue;
                mbar_arrive_expect_tx(&sm->q_full[t], G::kQBytes);
#pragma unroll
                for (int cb = 0; cb < G::CB; cb++)
                    tma_load_4d(sm->q[t] + cb * kBM * 64, &tm_q, 64 * cb, x.head, x.row0[t], x.cseq, &sm->q_full[t]);
                q_uses[t]++;
            }
            for (int j = x.jb0; ok && j < x.jb1; j++, kv_it++) {
                const int st = kv_it % kStages;
                const uint32_t ph = (kv_it / kStages) & 1;
                // Contiguous caches: coordinates (row, sequence) of the per-sequence map. Paged: (row within the
                // block, pool block); blocks holding the last visible row use the tail maps, whose row extent ends
                // at that row, so rows past the context are zero-filled rather than read from the pool.
                int crow = j * kBN, cseq = x.seq;
                const CUtensorMap* mk = &tm_k;
                const CUtensorMap* mv = &tm_v;
                if (a.block_table) {
                    const int blk = crow / a.block_rows;
                    cseq = a.block_table[static_cast<int64_t>(x.seq) * a.max_blocks + blk];
                    crow -= blk * a.block_rows;
                    if (cseq < 0 || cseq >= a.pool_blocks) {  // outside the pool: the TMA zero-fills the rows
                        atomicOr(a.err, kDevErrBadIndex);
                        cseq = a.pool_blocks;
                    }
                    if (blk == a.last_block) {
                        mk = &tm_kt;
                        mv = &tm_vt;
                    }
                }
                ok = mbar_wait(&sm->k_empty[st], ph ^ 1, ab);
                if (!ok) break;
                mbar_arrive_expect_tx(&sm->k_full[st], G::kKVBytes);
#pragma unroll
                for (int cb = 0; cb < G::CB; cb++)
                    tma_load_4d(sm->k[st] + cb * kBN * 64, mk, 64 * cb, kvh, crow, cseq, &sm->k_full[st]);
                k_issued = kv_it + 1;
                ok = mbar_wait(&sm->v_empty[st], ph ^ 1, ab);
                if (!ok) break;
                mbar_arrive_expect_tx(&sm->v_full[st], G::kKVBytes);
#pragma unroll
                for (int cb = 0; cb < G::CB; cb++)
                    tma_load_4d(sm->v[st] + cb * kBN * 64, mv, 64 * cb, kvh, crow, cseq, &sm->v_full[st]);
                v_issued = kv_it + 1;
            }
        }
        if (!ok) {
            // Drain our own loads still in flight before the CTA retires.
            int dummy = 0;
            AbortState drain{&dummy, a.err, kWaitLimitNs};
            for (uint32_t i = (k_issued > kStages ? k_issued - kStages : 0); i < k_issued; i++)
                mbar_wait(&sm->k_full[i % kStages], (i / kStages) & 1, drain);
            for (uint32_t i = (v_issued > kStages ? v_issued - kStages : 0); i < v_issued; i++)
                mbar_wait(&sm->v_full[i % kStages], (i / kStages) & 1, drain);
            for (int t = 0; t < NT; t++)
                if (q_uses[t] > 0) mbar_wait(&sm->q_full[t], (q_uses[t] - 1) & 1, drain);
        }
        mbar_arrive(&sm->retire);
    } else if (warp >= 1 && warp <= NT) {
        if constexpr (R == 2 || NT == 3) setmaxnreg_dec<kRegsControl>();
        if (lane == 0) {
            // ------------------------------------------------------------------ MMA issuers, one thread per tile
            // Every issuer walks every KV block of every item: a tile with fewer blocks than the others still
            // releases the K/V stages it does not use (after they land), so each stage's empty barrier (count NT)
            // completes once per use.
            const int t = warp - 1;
            uint32_t kv_it = 0, q_uses = 0, s_uses = 0, p_uses = 0;
            bool ok = true;
            if (debug_timeout && t == 0) ok = mbar_wait(&sm->dbg, 0, ab);  // nothing arrives: exercises the give-up path
            for (int r = 0, it = item_of(0); ok && it < total_items; it = item_of(++r)) {
                const TileWork tw = tile_work<kBN, NT, VL, KS>(a, it, t);  // this issuer's tile
                const int n = tw.jb1;                                    // its blocks are [j0, n)
                const Item xi = decode_item<kBN, NT, VL, KS>(a, it);
                const int j0 = xi.jb0, j1 = xi.jb1;                      // the item's blocks
                const bool has = n > j0;
                if (has) {
                    ok = mbar_wait(&sm->q_full[t], q_uses & 1, ab);
                    if (!ok) break;
                }
                // Iteration j consumes K(j) (S of block j) and then V(j-1) (P·V of block j-1): the producer's load
                // order, so every wait here depends only on releases made kStages iterations earlier.
                for (int j = j0; ok && j <= j1; j++) {
                    if (j < j1) {
                        const uint32_t cur = kv_it + (j - j0);
                        const int st = cur % kStages;
                        ok = mbar_wait(&sm->k_full[st], (cur / kStages) & 1, ab);
                        if (!ok) break;
                        if (j < n) {
                            ok = mbar_wait(&sm->s_empty[t], (s_uses & 1) ^ 1, ab);
                            if (!ok) break;
                            tc_fence_after();
                            mma_s<D, NT>(sm, t, st, tmem_base);
                            tc_commit(&sm->s_full[t]);
                            s_uses++;
                            if (j + 1 == n) tc_commit(&sm->q_empty[t]);
                            tc_commit(&sm->k_empty[st]);
                        } else {
                            mbar_arrive(&sm->k_empty[st]);  // block this tile does not use
                        }
                    }
                    if (j > j0) {
                        const int b = j - 1;
                        const uint32_t prv = kv_it + (b - j0);
                        const int sp = prv % kStages;
                        // ragged form: warp 3 has zeroed the V rows past the context (and is done with the stage).
                        // Every block waits for it, not only the blocks that reach the context end: the stage's
                        // next load follows this P.V, and warp 3 must have seen this load's barrier phase before the
                        // next one completes (a version that sent inner blocks straight to the MMA let warp 3 fall
                        // a phase behind and zero the wrong block).
                        ok = mbar_wait(VL ? &sm->v_ready[sp] : &sm->v_full[sp], (prv / kStages) & 1, ab);
                        if (!ok) break;
                        if (b < n) {
                            ok = mbar_wait(&sm->p_full[t], p_uses & 1, ab);
                            if (!ok) break;
                            tc_fence_after();
                            mma_pv<D, NT>(sm, t, sp, tmem_base, b > j0);  // the part's first block starts O
                            tc_commit(&sm->o_done[t]);
                            tc_commit(&sm->v_empty[sp]);
                            p_uses++;
                        } else {
                            mbar_arrive(&sm->v_empty[sp]);
                        }
                    }
                }
                if (!ok) break;
                kv_it += j1 - j0;
                if (has) q_uses++;
            }
            // Retire every MMA this thread issued before TMEM is freed.
            int dummy = 0;
            AbortState drain{&dummy, a.err, kWaitLimitNs};
            tc_commit(&sm->fin[t]);
            mbar_wait(&sm->fin[t], 0, drain);
            if (t == 0) mbar_arrive(&sm->retire);
        }
        // Warp 2 frees TMEM once every role has retired (no block-wide barrier after the register split).
        __syncwarp();
        if (warp == 2) {
            int dummy = 0;
            AbortState drain{&dummy, a.err, 2 * kWaitLimitNs};
            mbar_wait(&sm->retire, 0, drain);
            tc_fence_after();
            tmem_dealloc(tmem_base, kTmemCols);
        }
    } else if (warp == 3) {
        if constexpr (R == 2 || NT == 3) setmaxnreg_dec<kRegsControl>();
        if constexpr (VL) {
            // ------------------------------------------------------------------ ragged form: V tail fix-up
            // A sequence's cache rows at or past its context end (start + tokens) may hold anything, and the
            // tensor maps only bound the rows at max_ctx_len. P is 0 in those columns for every query that exists,
            // but 0 x NaN is NaN in the P·V MMA, so the warp zeroes those rows of each landed V block before
            // releasing it to the MMA issuers (v_ready); K needs nothing (the causal mask replaces those scores).
            uint32_t kv_it = 0;
            bool ok = true;
            for (int r = 0, it = item_of(0); ok && it < total_items; it = item_of(++r)) {
                const Item x = decode_item<kBN, NT, VL, KS>(a, it);
                for (int j = x.jb0; j < x.jb1; j++, kv_it++) {
                    const int st = kv_it % kStages;
                    ok = __all_sync(0xffffffffu, mbar_wait(&sm->v_full[st], (kv_it / kStages) & 1, ab));
                    if (!ok) break;
                    const int keep = max(0, x.ctx_end - j * kBN);  // rows of this block inside the context
                    if (keep < kBN) {
#pragma unroll
                        for (int cb = 0; cb < G::CB; cb++) {
                            uint4* blk = reinterpret_cast<uint4*>(sm->v[st] + cb * kBN * 64);  // 8 x 16 B per row
                            for (int i = keep * 8 + lane; i < kBN * 8; i += 32) blk[i] = make_uint4(0u, 0u, 0u, 0u);
                        }
                        fence_proxy_async_smem();  // the zeros are visible to the tensor core's reads
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sm->v_ready[st]);
                }
            }
        }
    } else if constexpr (R == 1) {
        if constexpr (NT == 3) setmaxnreg_inc<kRegsSoftmax3>();
        // ------------------------------------------------------------------ softmax warps, one thread per row
        // Warp 4 + 4*tile + quarter owns TMEM lane quarter `quarter` of tile `tile`: each thread a whole query row,
        // so the row max and the row sum need no exchange. Registers come from the launch bound (no split).
        const int tile = (warp - 4) >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        const uint32_t s_addr = lane_addr + G::col_s(tile);
        const uint32_t o_addr = lane_addr + G::col_o(tile);
        const uint32_t p_addr = lane_addr + G::col_p(tile);
        uint32_t s_uses = 0, o_uses = 0, ep_uses = 0;
        const bool issuer = kTmaOut && ((warp - 4) & 3) == 0 && lane == 0;  // the tile's output TMA thread
        bool ok = true;
        for (int r = 0, it = item_of(0); ok && it < total_items; it = item_of(++r)) {
            const TileWork x = tile_work<kBN, NT, VL, KS>(a, it, tile);
            const int jb0 = x.jb0;  // this tile's KV blocks [jb0, jb1) in the item
            if (x.jb1 <= jb0) continue;
            const int row0 = x.row0;
            const int pos0 = x.pos0;     // absolute position of the tile's first query
            const int qpos = pos0 + row;  // and of this thread's
            float m_used = -INFINITY;
            float2 lsum = make_float2(0.f, 0.f);
            for (int j = jb0; j < x.jb1; j++) {
                ok = __all_sync(0xffffffffu, mbar_wait(&sm->s_full[tile], s_uses & 1, ab));
                if (!ok) break;
                s_uses++;
                tc_fence_after();
                float s[kBN];
#pragma unroll
                for (int c = 0; c < kBN; c += 32) tmem_ld32(s_addr + c, s + c);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm->s_empty[tile]);

                const int kv0 = j * kBN;
                if (kv0 + kBN - 1 > pos0) {  // the block reaches past the tile's first query: mask
#pragma unroll
                    for (int c = 0; c < kBN; c++)
                        if (kv0 + c > qpos) s[c] = -INFINITY;
                }
                float mv[8];
#pragma unroll
                for (int i = 0; i < 8; i++) mv[i] = s[i];
#pragma unroll
                for (int c = 8; c + 16 <= kBN; c += 16)
#pragma unroll
                    for (int i = 0; i < 8; i++) mv[i] = fmax3(mv[i], s[c + i], s[c + 8 + i]);
#pragma unroll
                for (int i = 0; i < 8; i++) mv[i] = fmaxf(mv[i], s[kBN - 8 + i]);
                const float pmax = fmaxf(fmax3(mv[0], mv[1], mv[2]), fmax3(fmax3(mv[3], mv[4], mv[5]), mv[6], mv[7]));
                // running max in log2 units; it moves only when the block exceeds it by more than the threshold
                const float pms = pmax * a.scale_log2;
                const float m_new = (j == jb0 || pms > m_used + kRescaleThreshold) ? pms : m_used;
                const float m_sub = (m_new == -INFINITY) ? 0.f : m_new;
                const float2 c2 = make_float2(a.scale_log2, a.scale_log2), nm2 = make_float2(-m_sub, -m_sub);
                uint32_t pk[kBN / 2];
                float2 ls[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                                make_float2(0.f, 0.f)};
#pragma unroll
                for (int pr = 0; pr < kBN / 2; pr++) {
                    const float2 xx = __ffma2_rn(make_float2(s[2 * pr], s[2 * pr + 1]), c2, nm2);
                    float2 e;
                    if ((pr & 7) < kEmuPairs) e = exp2_poly2(make_float2(fmaxf(xx.x, -125.f), fmaxf(xx.y, -125.f)));
                    else e = make_float2(ex2_approx(xx.x), ex2_approx(xx.y));
                    ls[pr & 3] = __fadd2_rn(ls[pr & 3], e);
                    pk[pr] = pack_half2(e.x, e.y);
                }
                const float2 lb = __fadd2_rn(__fadd2_rn(ls[0], ls[1]), __fadd2_rn(ls[2], ls[3]));
                bool rescale = false;
                float alpha = 1.f;
                if (j > jb0 && m_new > m_used) {
                    alpha = ex2_approx(m_used - m_new);
                    rescale = true;
                    lsum.x *= alpha;
                    lsum.y *= alpha;
                }
                m_used = m_new;
                lsum = __fadd2_rn(lsum, lb);
                if (j > jb0) {  // PV(j-1) must be done before P is overwritten or O is rescaled
                    ok = __all_sync(0xffffffffu, mbar_wait(&sm->o_done[tile], o_uses & 1, ab));
                    if (!ok) break;
                    o_uses++;
                    tc_fence_after();
                }
                if (__any_sync(0xffffffffu, rescale)) {  // warp-collective TMEM access: alpha is 1 for other rows
#pragma unroll
                    for (int c0 = 0; c0 < D; c0 += 32) {
                        float o[32];
                        tmem_ld32(o_addr + c0, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int c = 0; c < 32; c++) o[c] *= alpha;
                        tmem_st32(o_addr + c0, o);
                    }
                }
#pragma unroll
                for (int c = 0; c < kBN / 2; c += 32) tmem_st32(p_addr + c, reinterpret_cast<const float*>(pk + c));
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm->p_full[tile]);
            }
            if (!ok) break;
            // epilogue: O / l
            ok = __all_sync(0xffffffffu, mbar_wait(&sm->o_done[tile], o_uses & 1, ab));
            if (!ok) break;
            o_uses++;
            tc_fence_after();
            if (KS && x.rec) {  // split KV: this part's rows unnormalised, with their max (log2 units) and sum
                float* rec = a.part + ((static_cast<int64_t>(it) * NT + tile) * kBM + row) * (D + 2);
#pragma unroll
                for (int c0 = 0; c0 < D; c0 += 32) {
                    float o[32];
                    tmem_ld32(o_addr + c0, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 32; c += 2)  // records are 8-byte aligned ((D + 2) x 4 bytes each)
                        *reinterpret_cast<float2*>(rec + c0 + c) = make_float2(o[c], o[c + 1]);
                }
                *reinterpret_cast<float2*>(rec + D) = make_float2(m_used, lsum.x + lsum.y);
                tc_fence_before();
                continue;
            }
            const float inv = 1.f / (lsum.x + lsum.y);
            // whole tiles leave through the staging box and TMA stores; in the ragged form a sequence's last,
            // partial tile is stored row by row (its map rows past the tile belong to the next sequence)
            const bool tma_tile = kTmaOut && (!VL || x.nrows == kBM);
            if (tma_tile) {
                // Two rounds of 64 columns through the tile's staging boxes and one thread's TMA stores, with the
                // same o_free / o_staged hand-offs as the two-thread form.
                float* stage = sm->o_stage + tile * (kBM * 64);
#pragma unroll 1
                for (int r64 = 0; r64 < D / 64; r64++) {
                    float o[64];
                    tmem_ld32(o_addr + r64 * 64, o);
                    tmem_ld32(o_addr + r64 * 64 + 32, o + 32);
                    tmem_wait_ld();
                    if (ep_uses > 0) {
                        if (issuer) {
                            bulk_wait_read_all();
                            mbar_arrive(&sm->o_free[tile]);
                        }
                        ok = __all_sync(0xffffffffu, mbar_wait(&sm->o_free[tile], (ep_uses - 1) & 1, ab));
                        if (!ok) break;
                    }
                    if (a.out_f16) {
                        __half* rowp = reinterpret_cast<__half*>(stage) + row * 64;
#pragma unroll
                        for (int c = 0; c < 8; c++) {
                            const int ch = c ^ (row & 7);
                            const float* v = o + 8 * c;
                            *reinterpret_cast<uint4*>(rowp + ch * 8) =
                                make_uint4(pack_half2(v[0] * inv, v[1] * inv), pack_half2(v[2] * inv, v[3] * inv),
                                           pack_half2(v[4] * inv, v[5] * inv), pack_half2(v[6] * inv, v[7] * inv));
                        }
                    } else {
#pragma unroll
                        for (int b = 0; b < 2; b++) {
                            float* rowp = stage + b * (kBM * 32) + row * 32;
#pragma unroll
                            for (int c = 0; c < 8; c++) {
                                const int ch = c ^ (row & 7);
                                const float* v = o + 32 * b + 4 * c;
                                *reinterpret_cast<float4*>(rowp + ch * 4) =
                                    make_float4(v[0] * inv, v[1] * inv, v[2] * inv, v[3] * inv);
                            }
                        }
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sm->o_staged[tile]);
                    bool sent = true;
                    if (issuer) {
                        sent = mbar_wait(&sm->o_staged[tile], ep_uses & 1, ab);
                        if (sent) {
                            if (a.out_f16) {
                                tma_store_4d(&tm_o, stage, r64 * 64, x.head, row0, x.cseq);
                            } else {
                                tma_store_4d(&tm_o, stage, r64 * 64, x.head, row0, x.cseq);
                                tma_store_4d(&tm_o, stage + kBM * 32, r64 * 64 + 32, x.head, row0, x.cseq);
                            }
                            bulk_commit();
                        }
                    }
                    ok = __all_sync(0xffffffffu, sent);
                    if (!ok) break;
                    ep_uses++;
                }
                if (!ok) break;
                tc_fence_before();
                continue;
            }
            const int t = row0 + row;  // row of the output map
            const bool have = VL ? row < x.nrows : t < a.tokens;
            const int64_t off = x.cseq * a.out_seq_stride + static_cast<int64_t>(t) * a.out_token_stride +
                                static_cast<int64_t>(x.head) * D;
#pragma unroll
            for (int c0 = 0; c0 < D; c0 += 32) {
                float o[32];
                tmem_ld32(o_addr + c0, o);
                tmem_wait_ld();
                if (have) {
                    if (a.out_f16) {
                        uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(a.out) + off + c0);
#pragma unroll
                        for (int c = 0; c < 32; c += 8)
                            dst[c / 8] = make_uint4(pack_half2(o[c] * inv, o[c + 1] * inv),
                                                    pack_half2(o[c + 2] * inv, o[c + 3] * inv),
                                                    pack_half2(o[c + 4] * inv, o[c + 5] * inv),
                                                    pack_half2(o[c + 6] * inv, o[c + 7] * inv));
                    } else {
                        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + off + c0);
#pragma unroll
                        for (int c = 0; c < 32; c += 4)
                            dst[c / 4] = make_float4(o[c] * inv, o[c + 1] * inv, o[c + 2] * inv, o[c + 3] * inv);
                    }
                }
            }
            tc_fence_before();
        }
        if (issuer) bulk_wait_all();  // the tile's last output stores are done before the CTA retires
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm->retire);
    } else {
        setmaxnreg_inc<kRegsSoftmax>();
        // ------------------------------------------------------------------ softmax warps
        const int sw = warp - 4;
        const int tile = sw >> 3;                   // query tile A (0) or B (1)
        const int half = (sw >> 2) & 1;             // S columns [half*SC, half*SC + SC) of each block
        const int quarter = warp & 3;               // TMEM lane quarter this warp may access
        const int row = quarter * 32 + lane;        // query row within the tile = TMEM lane
        const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        const uint32_t s_addr = lane_addr + G::col_s(tile) + half * SC;
        const uint32_t o_addr = lane_addr + G::col_o(tile) + half * OC;      // this thread's OC context columns
        const uint32_t p_addr = lane_addr + G::col_p(tile) + half * (SC / 2); // its SC/2 columns of P pairs
        uint64_t* xbar = &sm->xbar[tile][quarter];
        uint32_t s_uses = 0, o_uses = 0, x_uses = 0, ep_uses = 0;
        const bool issuer = kTmaOut && ((warp - 4) & 7) == 0 && lane == 0;  // the tile's output TMA thread
        bool ok = true;
        for (int r = 0, it = item_of(0); ok && it < total_items; it = item_of(++r)) {
            const TileWork x = tile_work<kBN, NT, VL, KS>(a, it, tile);
            const int jb0 = x.jb0;  // this tile's KV blocks [jb0, jb1) in the item
            if (x.jb1 <= jb0) continue;
            const int row0 = x.row0;
            const int pos0 = x.pos0;     // absolute position of the tile's first query
            const int qpos = pos0 + row;  // and of this thread's
            float m_used = -INFINITY;
            float2 lsum = make_float2(0.f, 0.f);    // this thread's half of the row sum (two lanes of a pair)
            for (int j = jb0; j < x.jb1; j++) {
                ok = __all_sync(0xffffffffu, mbar_wait(&sm->s_full[tile], s_uses & 1, ab));
                if (!ok) break;
                s_uses++;
                tc_fence_after();
                float s[SC];
#pragma unroll
                for (int c = 0; c < SC; c += 32) tmem_ld32(s_addr + c, s + c);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm->s_empty[tile]);

                const int kv0 = j * kBN + half * SC;
                if (kv0 + SC - 1 > pos0) {  // these columns reach past the tile's first query: mask
#pragma unroll
                    for (int c = 0; c < SC; c++)
                        if (kv0 + c > qpos) s[c] = -INFINITY;
                }
                // partial row max over SC columns: 8 independent 3-input max chains, then a small tree
                static_assert(SC % 16 == 0, "max tree expects SC = 8 + 16k + 8");
                float mv[8];
#pragma unroll
                for (int i = 0; i < 8; i++) mv[i] = s[i];
#pragma unroll
                for (int c = 8; c + 16 <= SC; c += 16)
#pragma unroll
                    for (int i = 0; i < 8; i++) mv[i] = fmax3(mv[i], s[c + i], s[c + 8 + i]);
#pragma unroll
                for (int i = 0; i < 8; i++) mv[i] = fmaxf(mv[i], s[SC - 8 + i]);
                const float pmax = fmaxf(fmax3(mv[0], mv[1], mv[2]), fmax3(fmax3(mv[3], mv[4], mv[5]), mv[6], mv[7]));
                // This half's candidate max (log2 units): the running max unless these columns exceed it by more
                // than the threshold. The two halves publish their candidates and compute P against their own
                // without waiting; the row max is the larger candidate, and a half whose candidate was lower
                // scales its P pairs down afterwards (rare: first block of a tile, or a max that jumped).
                const float pms = pmax * a.scale_log2;
                const float m_mine = (j == jb0 || pms > m_used + kRescaleThreshold) ? pms : m_used;
                const int par = x_uses & 1;
                sm->xmax[tile][par][half][row] = m_mine;
                __threadfence_block();
                __syncwarp();
                if (lane == 0) mbar_arrive(xbar);
                // P = 2^(s*c - m) per column pair: kEmuPairs of every 8 pairs on the FMA pipe, the rest on MUFU;
                // the f32 values feed the row sum, the f16 pairs the P·V MMA. A fully masked half (m_mine = -inf)
                // subtracts 0 instead, giving P = 0.
                const float m_sub = (m_mine == -INFINITY) ? 0.f : m_mine;
                const float2 c2 = make_float2(a.scale_log2, a.scale_log2), nm2 = make_float2(-m_sub, -m_sub);
                uint32_t pk[SC / 2];
                float2 ls[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                                make_float2(0.f, 0.f)};  // four independent partial sums (no serial chain)
#pragma unroll
                for (int pr = 0; pr < SC / 2; pr++) {
                    const float2 xx = __ffma2_rn(make_float2(s[2 * pr], s[2 * pr + 1]), c2, nm2);
                    float2 e;
                    if ((pr & 7) < kEmuPairs) e = exp2_poly2(make_float2(fmaxf(xx.x, -125.f), fmaxf(xx.y, -125.f)));
                    else e = make_float2(ex2_approx(xx.x), ex2_approx(xx.y));
                    ls[pr & 3] = __fadd2_rn(ls[pr & 3], e);
                    pk[pr] = pack_half2(e.x, e.y);
                }
                float2 lb = __fadd2_rn(__fadd2_rn(ls[0], ls[1]), __fadd2_rn(ls[2], ls[3]));
                // the partner's candidate (published before its exponentials, so normally already there)
                ok = __all_sync(0xffffffffu, mbar_wait(xbar, par, ab));
                if (!ok) break;
                x_uses++;
                const float m_row = fmaxf(m_mine, sm->xmax[tile][par][half ^ 1][row]);
                if (__any_sync(0xffffffffu, m_mine < m_row)) {
                    // f16 factor, applied identically to the P pairs and to this half's row sum: 1 where m_mine ==
                    // m_row, including a row that sees no key of this block range (both -inf, whose difference is
                    // NaN: a split-KV part that starts past the row's position)
                    const __half2 f2 = __float2half2_rn(m_mine == m_row ? 1.f : ex2_approx(m_mine - m_row));
                    const float f = __low2float(f2);
#pragma unroll
                    for (int pr = 0; pr < SC / 2; pr++) {
                        __half2 h = *reinterpret_cast<__half2*>(&pk[pr]);
                        h = __hmul2(h, f2);
                        pk[pr] = *reinterpret_cast<uint32_t*>(&h);
                    }
                    lb.x *= f;
                    lb.y *= f;
                }
                bool rescale = false;
                float alpha = 1.f;
                if (j > jb0 && m_row > m_used) {
                    alpha = ex2_approx(m_used - m_row);
                    rescale = true;
                    lsum.x *= alpha;
                    lsum.y *= alpha;
                }
                m_used = m_row;
                lsum = __fadd2_rn(lsum, lb);
                if (j > jb0) {  // PV(j-1) must be done before P is overwritten or O is rescaled
                    ok = __all_sync(0xffffffffu, mbar_wait(&sm->o_done[tile], o_uses & 1, ab));
                    if (!ok) break;
                    o_uses++;
                    tc_fence_after();
                }
                // tcgen05.ld/st are warp-collective: the whole warp rescales when any of its rows must (alpha
                // stays 1 for the others)
                if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
                    for (int c0 = 0; c0 < OC; c0 += 32) {
                        float o[32];
                        tmem_ld32(o_addr + c0, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int c = 0; c < 32; c++) o[c] *= alpha;
                        tmem_st32(o_addr + c0, o);
                    }
                }
                if constexpr (SC / 2 == 32) tmem_st32(p_addr, reinterpret_cast<const float*>(pk));
                else tmem_st16(p_addr, reinterpret_cast<const float*>(pk));
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm->p_full[tile]);
            }
            if (!ok) break;
            // epilogue: O / l; the two halves of the row sum meet through shared memory
            ok = __all_sync(0xffffffffu, mbar_wait(&sm->o_done[tile], o_uses & 1, ab));
            if (!ok) break;
            o_uses++;
            tc_fence_after();
            float o[OC];
#pragma unroll
            for (int c0 = 0; c0 < OC; c0 += 32) tmem_ld32(o_addr + c0, o + c0);
            const float lpart = lsum.x + lsum.y;
            sm->xl[tile][half][row] = lpart;
            __threadfence_block();
            __syncwarp();
            if (lane == 0) mbar_arrive(xbar);
            tmem_wait_ld();
            tc_fence_before();
            ok = __all_sync(0xffffffffu, mbar_wait(xbar, x_uses & 1, ab));
            if (!ok) break;
            x_uses++;
            const float l = lpart + sm->xl[tile][half ^ 1][row];
            if (KS && x.rec) {  // split KV: this part's rows unnormalised, with their max (log2 units) and sum
                float* rec = a.part + ((static_cast<int64_t>(it) * NT + tile) * kBM + row) * (D + 2);
#pragma unroll
                for (int c = 0; c < OC; c += 2)  // records are 8-byte aligned ((D + 2) x 4 bytes each)
                    *reinterpret_cast<float2*>(rec + half * OC + c) = make_float2(o[c], o[c + 1]);
                if (half == 0) *reinterpret_cast<float2*>(rec + D) = make_float2(m_used, l);
                continue;
            }
            const int t = row0 + row;  // row of the output map
            // whole tiles leave through the staging box and TMA stores; in the ragged form a sequence's last,
            // partial tile is stored row by row (its map rows past the tile belong to the next sequence)
            const bool tma_tile = kTmaOut && (!VL || x.nrows == kBM);
            if (tma_tile) {
                // The rows go through the tile's staging box and one thread's TMA stores (rows past the tokens are
                // clipped by the tensor map). Hand-offs on mbarriers with bounded waits: o_free (the previous
                // store has read the box) and o_staged (all 8 warps have written their rows).
                const float inv = 1.f / l;
                if (ep_uses > 0) {
                    if (issuer) {
                        bulk_wait_read_all();
                        mbar_arrive(&sm->o_free[tile]);
                    }
                    ok = __all_sync(0xffffffffu, mbar_wait(&sm->o_free[tile], (ep_uses - 1) & 1, ab));
                    if (!ok) break;
                }
                float* stage = sm->o_stage + tile * (kBM * 64);
                if (a.out_f16) {
                    __half* rowp = reinterpret_cast<__half*>(stage) + row * 64;  // one box, 128-byte rows of 64
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        const int ch = (half * 4 + c) ^ (row & 7);
                        const float* v = o + 8 * c;
                        *reinterpret_cast<uint4*>(rowp + ch * 8) =
                            make_uint4(pack_half2(v[0] * inv, v[1] * inv), pack_half2(v[2] * inv, v[3] * inv),
                                       pack_half2(v[4] * inv, v[5] * inv), pack_half2(v[6] * inv, v[7] * inv));
                    }
                } else {
                    float* rowp = stage + half * (kBM * 32) + row * 32;  // this half's box, 128-byte rows of 32
#pragma unroll
                    for (int c = 0; c < 8; c++) {
                        const int ch = c ^ (row & 7);
                        *reinterpret_cast<float4*>(rowp + ch * 4) =
                            make_float4(o[4 * c] * inv, o[4 * c + 1] * inv, o[4 * c + 2] * inv, o[4 * c + 3] * inv);
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm->o_staged[tile]);
                bool sent = true;
                if (issuer) {
                    sent = mbar_wait(&sm->o_staged[tile], ep_uses & 1, ab);
                    if (sent) {
                        if (a.out_f16) {
                            tma_store_4d(&tm_o, stage, 0, x.head, row0, x.cseq);
                        } else {
                            tma_store_4d(&tm_o, stage, 0, x.head, row0, x.cseq);
                            tma_store_4d(&tm_o, stage + kBM * 32, 32, x.head, row0, x.cseq);
                        }
                        bulk_commit();
                    }
                }
                ok = __all_sync(0xffffffffu, sent);
                if (!ok) break;
                ep_uses++;
            } else if (VL ? row < x.nrows : t < a.tokens) {
                const float inv = 1.f / l;
                const int64_t off = x.cseq * a.out_seq_stride + static_cast<int64_t>(t) * a.out_token_stride +
                                    static_cast<int64_t>(x.head) * D + half * OC;
                if (a.out_f16) {
                    uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(a.out) + off);
#pragma unroll
                    for (int c = 0; c < OC; c += 8)
                        dst[c / 8] = make_uint4(pack_half2(o[c] * inv, o[c + 1] * inv),
                                                pack_half2(o[c + 2] * inv, o[c + 3] * inv),
                                                pack_half2(o[c + 4] * inv, o[c + 5] * inv),
                                                pack_half2(o[c + 6] * inv, o[c + 7] * inv));
                } else {
                    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + off);
#pragma unroll
                    for (int c = 0; c < OC; c += 4)
                        dst[c / 4] = make_float4(o[c] * inv, o[c + 1] * inv, o[c + 2] * inv, o[c + 3] * inv);
                }
            }
        }
        if (issuer) bulk_wait_all();  // the tile's last output stores are done before the CTA retires
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm->retire);
    }

}

// Split KV: one warp per output row (item of the unsplit call, tile, row) merges the row's parts. With m_p the part's
// running max (log2 units, -inf where the part saw no visible key), l_p its sum and O_p its unnormalised context,
// out = sum_p 2^(m_p - M) O_p / sum_p 2^(m_p - M) l_p, M = max_p m_p. A part that holds no KV block of the tile wrote
// nothing and is skipped (the block ranges are recomputed as the prefill kernel cut them). A ragged unit that ran
// whole (one part) wrote its output itself and is skipped too.
template <int D, int BN, bool VL>
__global__ void __launch_bounds__(256) prefill_merge_kernel(const PrefillArgs a) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");  // every part of the prefill launch has been written
    constexpr int NT = 2, CPL = D / 32;                  // columns per lane
    const int w = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    const int row = w % kBM, tile = (w / kBM) % NT, base = w / (kBM * NT);
    const int S = a.kv_splits;
    int nblk, nmax, up;      // the tile's KV blocks, the item's, and the parts the item was cut into
    int64_t item0, pstep;    // record item of part p: item0 + p * pstep
    int64_t off;             // output element of the row's first column
    if constexpr (VL) {
        // base = (unit, head) of the ragged work list (unit-major, head-minor, as the prefill kernel deals it)
        const int unit = base / a.n_heads, head = base - unit * a.n_heads;
        if (unit >= __ldg(&a.plan[0].x)) return;
        const int4 r = __ldg(a.plan + 1 + 2 * unit);
        const int rows_t = max(0, min(kBM, r.w - tile * kBM));
        if (row >= rows_t) return;
        nblk = (r.z + tile * kBM + rows_t + BN - 1) / BN;
        nmax = 0;
#pragma unroll
        for (int u = 0; u < NT; u++) {
            const int rows = max(0, min(kBM, r.w - u * kBM));
            nmax = max(nmax, rows > 0 ? (r.z + u * kBM + rows + BN - 1) / BN : 0);
        }
        up = unit_parts(S, nmax);
        if (up <= 1) return;  // the unit ran whole and wrote its output itself
        item0 = static_cast<int64_t>(unit) * S * a.n_heads + head;
        pstep = a.n_heads;
        off = static_cast<int64_t>(r.y + tile * kBM + row) * a.out_token_stride + static_cast<int64_t>(head) * D;
    } else {
        const int per_rank = a.n_seqs * a.n_heads;
        const int gr = base / per_rank, rem = base - gr * per_rank;  // group rank (heaviest first) and (seq, head)
        if (gr >= a.n_groups) return;
        const int group = a.n_groups - 1 - gr;
        const int seq = rem / a.n_heads, head = rem - seq * a.n_heads;
        const int row0 = (group * NT + tile) * kBM;
        const int t = row0 + row;
        if (t >= a.tokens) return;
        nblk = tile_blocks<BN>(a, row0);
        nmax = 0;
#pragma unroll
        for (int u = 0; u < NT; u++) nmax = max(nmax, tile_blocks<BN>(a, (group * NT + u) * kBM));
        up = S;
        item0 = static_cast<int64_t>(gr) * S * per_rank + rem;
        pstep = per_rank;
        off = static_cast<int64_t>(seq) * a.out_seq_stride + static_cast<int64_t>(t) * a.out_token_stride +
              static_cast<int64_t>(head) * D;
    }
    // every part's loads first (up to kMaxKvSplits parts, unrolled), then the sums
    float mp[kMaxKvSplits], lp[kMaxKvSplits], op[kMaxKvSplits][CPL];
#pragma unroll
    for (int p = 0; p < kMaxKvSplits; p++) {
        const bool use = p < up && min(nblk, (p + 1) * nmax / up) > p * nmax / up;
        mp[p] = -INFINITY;
        lp[p] = 0.f;
#pragma unroll
        for (int c = 0; c < CPL; c++) op[p][c] = 0.f;
        if (use) {
            const float* rec = a.part + ((item0 + p * pstep) * NT + tile) * kBM * (D + 2) + row * (D + 2);
            const float2 ml = __ldg(reinterpret_cast<const float2*>(rec + D));
            mp[p] = ml.x;
            lp[p] = ml.y;
#pragma unroll
            for (int c = 0; c < CPL; c++) op[p][c] = __ldg(rec + lane + 32 * c);
        }
    }
    float M = -INFINITY;
#pragma unroll
    for (int p = 0; p < kMaxKvSplits; p++) M = fmaxf(M, mp[p]);
    float acc[CPL] = {};
    float L = 0.f;
#pragma unroll
    for (int p = 0; p < kMaxKvSplits; p++) {
        const float wgt = mp[p] == -INFINITY ? 0.f : exp2f(mp[p] - M);  // a part that saw no visible key: 0
        L = fmaf(wgt, lp[p], L);
#pragma unroll
        for (int c = 0; c < CPL; c++) acc[c] = fmaf(wgt, op[p][c], acc[c]);
    }
    const float inv = 1.f / L;
#pragma unroll
    for (int c = 0; c < CPL; c++) {
        if (a.out_f16) static_cast<__half*>(a.out)[off + lane + 32 * c] = __float2half_rn(acc[c] * inv);
        else static_cast<float*>(a.out)[off + lane + 32 * c] = acc[c] * inv;
    }
}

// f32 -> f16 copy of Q into the workspace ([seq][token][head][d], dense), for f32 callers.
__global__ void q_to_half_kernel(const float* __restrict__ q, int64_t token_stride, int64_t seq_stride,
                                 __half* __restrict__ dst, int n_seqs, int tokens, int hd_total) {
    const int64_t n = static_cast<int64_t>(n_seqs) * tokens * hd_total;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t c = i % hd_total, r = i / hd_total;
        const int64_t t = r % tokens, sq = r / tokens;
        dst[i] = __float2half_rn(q[sq * seq_stride + t * token_stride + c]);
    }
}

// ---------------------------------------------------------------------------------------------- ragged plan

// Work list of a ragged call. A unit is one group of kUnitTiles query tiles of one sequence (all heads: the prefill
// kernel takes unit-major, head-minor items). Sequences come heaviest first (by the KV blocks their last query
// attends to) and each sequence's units stay together, heaviest first: the items a persistent kernel runs at the
// same time then share the K/V rows of a few sequences, so the re-reads of those rows by the sequence's other query
// tiles hit L2 (ordering units by cost across sequences spread each sequence's re-reads over the whole launch and
// sent them to DRAM), while the lightest sequences still fill the tail. One CTA counts the units per cost bucket of
// their sequence, turns the counts into write positions in descending order, and each sequence claims a contiguous
// range of its bucket.
constexpr int kPlanThreads = 1024;
constexpr int kPlanBuckets = 2 * kPlanThreads;  // costs above kPlanBuckets - 1 blocks share the first bucket
constexpr int kUnitTiles = 2;                   // query tiles per unit (the two-tile forms)

struct PlanArgs {
    const int* q_offsets;
    const int* start_positions;
    int4* plan;
    int n_seqs, max_tokens, max_ctx, total_tokens, bn;
    unsigned* err;
};

// Sequence s's packed offset, query count and start position. False for an empty sequence and for one that breaks
// the call's bounds (reported through the error word; its queries are not computed).
__device__ __forceinline__ bool plan_span(const PlanArgs& p, int s, int& off, int& len, int& start) {
    off = p.q_offsets[s];
    const int end = p.q_offsets[s + 1];
    start = p.start_positions[s];
    len = end - off;
    const bool in_range = off >= 0 && end >= off && end <= p.total_tokens;
    if (in_range && len == 0) return false;
    if (!in_range || len > p.max_tokens || start < 0 || static_cast<int64_t>(start) + len > p.max_ctx) {
        atomicOr(p.err, kDevErrBadIndex);
        return false;
    }
    return true;
}

// Bucket of a sequence: the KV blocks its last query attends to, heaviest first.
__device__ __forceinline__ int plan_bucket(const PlanArgs& p, int start, int len) {
    const int cost = (start + len + p.bn - 1) / p.bn;
    return kPlanBuckets - 1 - min(cost, kPlanBuckets - 1);
}

__device__ __forceinline__ int plan_units_of(int len) { return (len + kUnitTiles * kBM - 1) / (kUnitTiles * kBM); }

__global__ void __launch_bounds__(kPlanThreads) prefill_plan_kernel(const PlanArgs p) {
    __shared__ int cnt[kPlanBuckets];  // units per bucket, then the buckets' write cursors
    __shared__ int warp_tot[kPlanThreads / 32];
    // The prefill kernel may launch now; it waits for this grid's memory before reading the plan.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < kPlanBuckets; i += kPlanThreads) cnt[i] = 0;
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the offsets may come from the previous kernel
    __syncthreads();
    for (int s = tid; s < p.n_seqs; s += kPlanThreads) {
        int off, len, start;
        if (!plan_span(p, s, off, len, start)) continue;
        atomicAdd(&cnt[plan_bucket(p, start, len)], plan_units_of(len));
    }
    __syncthreads();
    // exclusive prefix sum of the counts: thread i owns buckets 2i and 2i + 1
    const int c0 = cnt[2 * tid], c1 = cnt[2 * tid + 1];
    int incl = c0 + c1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = warp_tot[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += n;
        }
        warp_tot[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int before = (warp > 0 ? warp_tot[warp - 1] : 0) + incl - c0 - c1;
    cnt[2 * tid] = before;
    cnt[2 * tid + 1] = before + c0;
    if (tid == kPlanThreads - 1) p.plan[0] = make_int4(before + c0 + c1, 0, 0, 0);
    __syncthreads();
    for (int s = tid; s < p.n_seqs; s += kPlanThreads) {
        int off, len, start;
        if (!plan_span(p, s, off, len, start)) continue;
        const int n = plan_units_of(len);
        const int base = atomicAdd(&cnt[plan_bucket(p, start, len)], n);
        for (int i = 0; i < n; i++) {  // the sequence's units, last (heaviest) group first
            const int g = n - 1 - i, r0 = g * kUnitTiles * kBM;
            p.plan[1 + 2 * (base + i)] = make_int4(s, off + r0, start + r0, min(kUnitTiles * kBM, len - r0));
            p.plan[2 + 2 * (base + i)] = make_int4(start + len, 0, 0, 0);
        }
    }
}

// ---------------------------------------------------------------------------------------------- host side

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 4-D f16 map over [seqs][rows][heads][d] with a 64 x 1 x box_rows x 1 box (one 128-byte column block of
// box_rows rows), 128-byte swizzle, zero fill.
bool make_map(CUtensorMap* map, const void* base, int d, int heads, int rows, int seqs, int64_t row_stride,
              int64_t seq_stride, int box_rows) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    if (seqs == 1 || seq_stride == 0) seq_stride = static_cast<int64_t>(rows) * row_stride;
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(rows),
                          static_cast<cuuint64_t>(seqs)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(d) * 2, static_cast<cuuint64_t>(row_stride) * 2,
                             static_cast<cuuint64_t>(seq_stride) * 2};
    cuuint32_t box[4] = {64, 1, static_cast<cuuint32_t>(box_rows), 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Share of exponentials computed on the FMA pipe: ALPACA_PREFILL_EMU column pairs of every 8 (0, 2, 3 or 4).
// MUFU gives 16 exp2 per clock per SM. Defaults, measured on 30 layers x 4096 tokens: the two-tile forms keep every
// exponential on MUFU (0.806 against 0.820 ms with 2 of 8 pairs on the FMA pipe, now that the output leaves through
// TMA stores); the three-tile form, whose three softmax phase groups keep MUFU busier, moves 2 of 8 (0.831 against
// 0.924 ms; 3 of 8: 0.839, 4 of 8: 0.951).
int prefill_emu_pairs(int tiles) {
    static const int v = [] {
        const char* e = std::getenv("ALPACA_PREFILL_EMU");
        if (!e || !*e) return -1;
        const int x = std::atoi(e);
        return (x == 0 || x == 2 || x == 3 || x == 4) ? x : -1;
    }();
    return v >= 0 ? v : (tiles == 3 ? 2 : 0);
}

using PrefillFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, PrefillArgs);

// 4-D map of the output [seqs][tokens][heads][d] (f32 or f16) for TMA stores: boxes of one 128-byte row segment
// (32 f32 or 64 f16 columns) x 128 tokens, 128-byte swizzle; rows past `tokens` are clipped.
bool make_out_map(CUtensorMap* map, void* base, bool f16, int d, int heads, int tokens, int seqs, int64_t token_stride,
                  int64_t seq_stride) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    const int es = f16 ? 2 : 4;
    if (seqs == 1 || seq_stride == 0) seq_stride = static_cast<int64_t>(tokens) * token_stride;
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(tokens),
                          static_cast<cuuint64_t>(seqs)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(d) * es, static_cast<cuuint64_t>(token_stride) * es,
                             static_cast<cuuint64_t>(seq_stride) * es};
    cuuint32_t box[4] = {static_cast<cuuint32_t>(128 / es), 1, static_cast<cuuint32_t>(kBM), 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Softmax threads per query row: one at head_dim 128 (822 against 747 TFLOP/s on 30 layers x 4096 tokens), two at
// head_dim 64 (637 against 612-617: with a whole 128-column row per thread two softmax warps per SMSP hide less
// latency than four). ALPACA_PREFILL_ROWS = 1 or 2 forces a form at head_dim 64; head_dim 128 has only the
// one-thread form.
int prefill_row_threads(int head_dim) {
    static const int v = [] {
        const char* e = std::getenv("ALPACA_PREFILL_ROWS");
        return e ? (e[0] == '1' ? 1 : 2) : 0;
    }();
    return v ? v : (head_dim == 128 ? 1 : 2);
}

// Query tiles per work item at head_dim 64: 2 (128-row KV blocks; default) or 3 (64-row KV blocks, one softmax
// thread per row, three softmax phase groups per SMSP instead of two): 0.831 against 0.807 ms on 30 layers x 4096
// tokens. ALPACA_PREFILL_TILES = 3 selects the three-tile form.
int prefill_tiles(int head_dim) {
    static const int v = [] {
        const char* e = std::getenv("ALPACA_PREFILL_TILES");
        return e ? (e[0] == '3' ? 3 : 2) : 0;
    }();
    return head_dim != 64 ? 2 : (v ? v : 2);
}

template <int D>
PrefillFn prefill_variant(int emu, int rows, int tiles) {
    if constexpr (D == 64) {  // head_dim 128 is built in the one-thread two-tile form only
        if (tiles == 3) {
            switch (emu) {
                case 0: return prefill_kernel<D, 0, 1, 3>;
                case 3: return prefill_kernel<D, 3, 1, 3>;
                case 4: return prefill_kernel<D, 4, 1, 3>;
                default: return prefill_kernel<D, 2, 1, 3>;
            }
        }
        if (rows != 1) {
            switch (emu) {
                case 0: return prefill_kernel<D, 0, 2, 2>;
                case 3: return prefill_kernel<D, 3, 2, 2>;
                case 4: return prefill_kernel<D, 4, 2, 2>;
                default: return prefill_kernel<D, 2, 2, 2>;
            }
        }
    }
    switch (emu) {
        case 0: return prefill_kernel<D, 0, 1, 2>;
        case 3: return prefill_kernel<D, 3, 1, 2>;
        case 4: return prefill_kernel<D, 4, 1, 2>;
        default: return prefill_kernel<D, 2, 1, 2>;
    }
}

}  // namespace

bool prefill_supported(const alpaca_attn_desc& d) {
    return (d.head_dim == 64 || d.head_dim == 128) && d.kv_dtype == ALPACA_F16 && d.n_kv_heads > 0 && d.n_heads % d.n_kv_heads == 0 &&
           d.ctx_lens == nullptr;
}

namespace {
bool is_varlen(const alpaca_attn_desc& d) { return (d.flags & ALPACA_ATTN_FLAG_VARLEN) != 0; }

// Bytes of f16 queries staged for an f32-Q call, rounded up to 16 so the ragged work list after them is aligned.
size_t q_stage_bytes(const alpaca_attn_desc& d) {
    if (d.q_dtype != ALPACA_F32) return 0;
    const size_t rows = is_varlen(d) ? static_cast<size_t>(d.total_tokens) : static_cast<size_t>(d.n_seqs) * d.tokens;
    return (sizeof(__half) * rows * d.n_heads * d.head_dim + 15) / 16 * 16;
}

// Units of a ragged call at most: every sequence's token bound split into groups of kUnitTiles tiles.
size_t plan_units(const alpaca_attn_desc& d) {
    const int group = kUnitTiles * kBM;
    return static_cast<size_t>(d.n_seqs) * ((d.tokens + group - 1) / group);
}
// Split KV for calls with fewer work items than one per SM of a B200 (148): each item's KV blocks are cut into up to
// 8 parts of at least 4 blocks of its heaviest group, as many as keep the call in one wave of items, so the call fills
// the SMs (a smaller call does not repay the merge: a 512-token chunk at position 0 measured 12.2 us per layer
// unsplit against 18.7 in two parts). This is the case of alpaca.swift's prefill loop, one session's 512-token chunk
// per call at a moving start position (MetalLlamaModel.swift:293-298): 18 items at SmolLM2-135M's 9 heads. A ragged
// call is sized from its bounds (units x heads, max_ctx_len); each unit then uses the parts its own blocks allow.
// ALPACA_PREFILL_SPLITS caps the parts (1 turns the split off).
constexpr int kSplitTargetItems = 148;
int prefill_kv_splits(const alpaca_attn_desc& d) {
    static const int cap = [] {
        const char* e = std::getenv("ALPACA_PREFILL_SPLITS");
        const int v = (e && *e) ? std::atoi(e) : kMaxKvSplits;
        return std::max(1, std::min(kMaxKvSplits, v));
    }();
    const bool vl = is_varlen(d);  // the ragged form runs the two-tile forms whatever the switches say
    if ((!vl && prefill_tiles(d.head_dim) != 2) || d.tokens <= 0) return 1;
    const int bn = d.head_dim == 128 ? PG<128>::BN : PG<64>::BN;
    // items and KV blocks of the heaviest tile: exact for a uniform call, the host bounds for a ragged one (whose
    // units then each use as many of the parts as their own blocks allow, unit_parts)
    const int64_t items = vl ? static_cast<int64_t>(plan_units(d)) * d.n_heads
                             : static_cast<int64_t>((d.tokens + 2 * kBM - 1) / (2 * kBM)) * d.n_seqs * d.n_heads;
    if (items >= kSplitTargetItems) return 1;
    const int nmax = ((vl ? d.max_ctx_len : d.start_position + d.tokens) + bn - 1) / bn;
    // the most parts that keep every item in one wave: a second wave puts two parts on some SMs
    const int want = static_cast<int>(kSplitTargetItems / items);
    return std::max(1, std::min(std::min(cap, want), nmax / 4));  // at least 4 blocks per part
}
// Partial records of a split call: [item][part][tile][row][head_dim + 2] f32.
size_t split_bytes(const alpaca_attn_desc& d) {
    const int splits = prefill_kv_splits(d);
    if (splits <= 1) return 0;
    const size_t items = is_varlen(d) ? plan_units(d) * d.n_heads
                                      : static_cast<size_t>((d.tokens + 2 * kBM - 1) / (2 * kBM)) * d.n_seqs * d.n_heads;
    return items * splits * 2 * kBM * (d.head_dim + 2) * sizeof(float);
}
}  // namespace

size_t prefill_workspace_min_bytes(const alpaca_attn_desc& d) {
    return q_stage_bytes(d) + (is_varlen(d) ? sizeof(int4) * (1 + 2 * plan_units(d)) : 0);
}

size_t prefill_workspace_bytes(const alpaca_attn_desc& d) {
    return prefill_workspace_min_bytes(d) + split_bytes(d);
}

cudaError_t launch_prefill(const Call& c, cudaStream_t s) {
    const alpaca_attn_desc& d = *c.d;
    const bool d128 = d.head_dim == 128;
    const bool vl = is_varlen(d);
    // The ragged form is built in the default two-tile forms only (the switches select among the uniform forms).
    const int tiles = vl ? kUnitTiles : prefill_tiles(d.head_dim);
    const int emu = vl ? 0 : prefill_emu_pairs(tiles);
    // split KV when the call is short of work items and the caller's workspace holds the partial records (a
    // workspace of the minimum size runs the call unsplit); split calls take the default two-tile forms
    int splits = prefill_kv_splits(d);
    if (splits > 1 && (c.ws_bytes < prefill_workspace_bytes(d) || !c.ws || (reinterpret_cast<uintptr_t>(c.ws) & 15u)))
        splits = 1;
    // softmax threads per query row of the form launched (its thread count and output path follow from it)
    const int rows = (d128 || tiles == 3) ? 1 : ((vl || splits > 1) ? 2 : prefill_row_threads(d.head_dim));
    const PrefillFn fn =
        vl ? (splits > 1 ? (d128 ? prefill_kernel<128, 0, 1, 2, true, true> : prefill_kernel<64, 0, 2, 2, true, true>)
                         : (d128 ? prefill_kernel<128, 0, 1, 2, true> : prefill_kernel<64, 0, 2, 2, true>))
           : splits > 1 ? (d128 ? prefill_kernel<128, 0, 1, 2, false, true> : prefill_kernel<64, 0, 2, 2, false, true>)
                        : (d128 ? prefill_variant<128>(emu, rows, tiles) : prefill_variant<64>(emu, rows, tiles));
    const size_t smem = d128 ? smem_bytes<128>() : (tiles == 3 ? smem_bytes<64, 3>() : smem_bytes<64>());
    const int bn = d128 ? PG<128>::BN : (tiles == 3 ? PG<64, 3>::BN : PG<64>::BN);
    // per-device function attribute (host-side, cheap next to the launch itself)
    cudaError_t attr_err = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (attr_err != cudaSuccess) return attr_err;

    // Queries (and outputs) as maps over [seqs][tokens]; the packed ragged layout is one sequence of total_tokens.
    const int q_seqs = vl ? 1 : d.n_seqs, q_rows = vl ? d.total_tokens : d.tokens;
    const void* qh = d.q;
    int64_t q_ts = d.q_token_stride, q_ss = vl ? 0 : d.q_seq_stride;
    if (d.q_dtype == ALPACA_F32) {
        __half* dst = static_cast<__half*>(c.ws);
        const int hd_total = d.n_heads * d.head_dim;
        const int64_t n = static_cast<int64_t>(q_seqs) * q_rows * hd_total;
        const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 4096));
        q_to_half_kernel<<<blocks, 256, 0, s>>>(static_cast<const float*>(d.q), d.q_token_stride, q_ss, dst, q_seqs,
                                                q_rows, hd_total);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        qh = dst;
        q_ts = hd_total;
        q_ss = static_cast<int64_t>(q_rows) * hd_total;
    }
    int4* plan = nullptr;
    if (vl) {
        plan = reinterpret_cast<int4*>(static_cast<uint8_t*>(c.ws) + q_stage_bytes(d));
        PlanArgs pa{d.q_offsets, d.start_positions, plan, d.n_seqs, d.tokens, d.max_ctx_len, d.total_tokens, bn, c.err};
        cudaLaunchConfig_t pcfg = {};
        pcfg.gridDim = dim3(1, 1, 1);
        pcfg.blockDim = dim3(kPlanThreads, 1, 1);
        pcfg.stream = s;
        cudaLaunchAttribute pattr[1];
        pattr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        pattr[0].val.programmaticStreamSerializationAllowed = 1;
        pcfg.attrs = pattr;
        pcfg.numAttrs = pdl_enabled() ? 1 : 0;
        const cudaError_t e = cudaLaunchKernelEx(&pcfg, prefill_plan_kernel, pa);
        if (e != cudaSuccess) return e;
    }
    // KV rows each sequence's map covers: the uniform call's visible rows, or the ragged call's bound.
    const int kv_len = vl ? d.max_ctx_len : d.start_position + d.tokens;
    CUtensorMap tq, tk, tv, tkt, tvt;
    if (!make_map(&tq, qh, d.head_dim, d.n_heads, q_rows, q_seqs, q_ts, q_ss, kBM)) return cudaErrorInvalidValue;
    int last_block = -1;
    if (d.block_table && vl) {
        // pool maps only: warp 3 zeroes the V rows past each sequence's context in its last block
        if (!make_map(&tk, d.k, d.head_dim, d.n_kv_heads, d.block_rows, d.pool_blocks, d.kv_row_stride, d.block_stride, bn) ||
            !make_map(&tv, d.v, d.head_dim, d.n_kv_heads, d.block_rows, d.pool_blocks, d.kv_row_stride, d.block_stride, bn))
            return cudaErrorInvalidValue;
        tkt = tk;
        tvt = tv;
    } else if (d.block_table) {
        // pool maps: [pool_blocks][block_rows] rows; tail maps end at the last visible row of its block
        last_block = (kv_len - 1) / d.block_rows;
        const int tail_rows = kv_len - last_block * d.block_rows;
        if (!make_map(&tk, d.k, d.head_dim, d.n_kv_heads, d.block_rows, d.pool_blocks, d.kv_row_stride, d.block_stride, bn) ||
            !make_map(&tv, d.v, d.head_dim, d.n_kv_heads, d.block_rows, d.pool_blocks, d.kv_row_stride, d.block_stride, bn) ||
            !make_map(&tkt, d.k, d.head_dim, d.n_kv_heads, tail_rows, d.pool_blocks, d.kv_row_stride, d.block_stride, bn) ||
            !make_map(&tvt, d.v, d.head_dim, d.n_kv_heads, tail_rows, d.pool_blocks, d.kv_row_stride, d.block_stride, bn))
            return cudaErrorInvalidValue;
    } else {
        if (!make_map(&tk, d.k, d.head_dim, d.n_kv_heads, kv_len, d.n_seqs, d.kv_row_stride, d.kv_seq_stride, bn) ||
            !make_map(&tv, d.v, d.head_dim, d.n_kv_heads, kv_len, d.n_seqs, d.kv_row_stride, d.kv_seq_stride, bn))
            return cudaErrorInvalidValue;
        tkt = tk;
        tvt = tv;
    }

    CUtensorMap to = tq;  // unused by the forms that store the output directly
    if ((d128 || rows != 1 || tiles == 3) &&
        !make_out_map(&to, d.out, d.out_dtype == ALPACA_F16, d.head_dim, d.n_heads, q_rows, q_seqs,
                      d.out_token_stride, vl ? 0 : d.out_seq_stride))
        return cudaErrorInvalidValue;

    PrefillArgs a;
    a.out = d.out;
    a.out_token_stride = d.out_token_stride;
    a.out_seq_stride = d.out_seq_stride;
    a.out_f16 = d.out_dtype == ALPACA_F16;
    a.n_seqs = d.n_seqs;
    a.n_heads = d.n_heads;
    a.n_kv_heads = d.n_kv_heads;
    a.tokens = d.tokens;
    a.start = d.start_position;
    a.kv_len = kv_len;
    a.n_groups = (d.tokens + tiles * kBM - 1) / (tiles * kBM);
    a.kv_splits = splits;
    // the parts' records follow the f32 queries' staging and the ragged work list
    a.part = splits > 1 ? reinterpret_cast<float*>(static_cast<uint8_t*>(c.ws) + prefill_workspace_min_bytes(d))
                        : nullptr;
    // ragged form: the plan's unit count, read by the kernel; the grid is sized for the bound
    a.total_items = vl ? static_cast<int>(plan_units(d)) * d.n_heads * splits : a.n_groups * d.n_seqs * d.n_heads * splits;
    a.scale_log2 = c.scale * kLog2e;
    a.err = c.err;
    a.flags = d.flags;
    a.block_table = d.block_table;
    a.block_rows = d.block_rows;
    a.max_blocks = d.max_blocks;
    a.pool_blocks = d.pool_blocks;
    a.last_block = last_block;
    a.plan = plan;
    const int grid = std::max(1, std::min(a.total_items, c.num_sms));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(32 * (4 + 4 * rows * tiles), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, fn, tq, tk, tv, tkt, tvt, to, a);
    if (e != cudaSuccess || splits <= 1) return e;
    // the merge: one warp per output row of the unsplit items (8 rows per CTA)
    // (ragged: for the bound of units; the units past the plan's count return at once)
    const int64_t out_rows = (vl ? static_cast<int64_t>(plan_units(d)) : static_cast<int64_t>(a.n_groups) * d.n_seqs) *
                             d.n_heads * 2 * kBM;
    cudaLaunchConfig_t mcfg = cfg;
    mcfg.gridDim = dim3(static_cast<unsigned>((out_rows + 7) / 8), 1, 1);
    mcfg.blockDim = dim3(256, 1, 1);
    mcfg.dynamicSmemBytes = 0;
    if (vl)
        return d128 ? cudaLaunchKernelEx(&mcfg, prefill_merge_kernel<128, PG<128>::BN, true>, a)
                    : cudaLaunchKernelEx(&mcfg, prefill_merge_kernel<64, PG<64>::BN, true>, a);
    return d128 ? cudaLaunchKernelEx(&mcfg, prefill_merge_kernel<128, PG<128>::BN, false>, a)
                : cudaLaunchKernelEx(&mcfg, prefill_merge_kernel<64, PG<64>::BN, false>, a);
}

}  // namespace alpaca
