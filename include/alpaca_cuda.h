/*
 * alpaca_cuda.h — C ABI of the B200 (sm_100a) attention library for alpaca.swift.
 *
 * This library is a drop-in for the attention hot path of alpaca.swift's Metal backend. Each entry point
 * below names the reference interface it replaces (paths are relative to the alpaca.swift repository):
 *
 *   KernelEncoder.attention(q:kCache:vCache:out:heads:kvHeads:headDim:startPosition:tokens:kv:decodeScratch:outputHalf:)
 *       Sources/AlpacaMetal/Backend/KernelEncoder.swift:306-343        -> alpaca_attention (ALPACA_ATTN_AUTO)
 *   KernelEncoder.attentionTensor(qHalf:kCache:vCache:out:outputHalf:...)
 *       Sources/AlpacaMetal/Backend/KernelEncoder.swift:284-292        -> alpaca_attn_prefill
 *   the split-K decode branch of KernelEncoder.attention (attn_decode_split_* + attn_decode_merge)
 *       Sources/AlpacaMetal/Backend/KernelEncoder.swift:309-326        -> alpaca_attn_decode
 *   KernelEncoder.decodeScratchBytes(heads:kvHeads:headDim:capacity:)
 *       Sources/AlpacaMetal/Backend/KernelEncoder.swift:88-92          -> alpaca_attention_workspace_bytes
 *   MetalError.invalidArgument / .unsupported / .commandFailed
 *       Sources/AlpacaMetal/Backend/MetalContext.swift:7-31            -> alpaca_cuda_status + alpaca_cuda_status_string
 *   KernelEncoder.ropeQKVStore(q:k:v:kCache:vCache:freqs:heads:kvHeads:headDim:startPosition:tokens:kv:)
 *       Sources/AlpacaMetal/Backend/KernelEncoder.swift:401-411        -> alpaca_rope_kv_append
 *       (kernels rope_qkv_store_kv16 / _kv32, Sources/AlpacaMetal/Kernels/decode_fused.metal:126-154; with no K/V
 *       it is MetalOps.rope, Sources/AlpacaMetal/Backend/MetalOps.swift:165-171)
 *
 * Data layout (the hand-off of Sources/AlpacaMetal/Backend/MetalLlamaModel.swift:189-191, 322-337):
 *   q    [n_seqs][tokens][n_heads][head_dim]     post-RoPE queries (f16 or f32); token t of a sequence sits at
 *                                                 absolute position start_position + t.
 *   k, v [n_seqs][rows][n_kv_heads][head_dim]    KV cache rows, row index = absolute position (f16 or f32).
 *                                                 K holds post-RoPE keys, V raw values. Query head h reads KV
 *                                                 head h / (n_heads / n_kv_heads).
 *   out  [n_seqs][tokens][n_heads][head_dim]     context vectors (f32 or f16).
 * Strides are in elements. The innermost [heads][head_dim] block of one token / row is contiguous.
 *
 * Ownership and threading: every pointer in a descriptor is a caller-owned device pointer. Calls only
 * enqueue work on `stream` and return; the library never allocates device memory on the attention path.
 * Scratch space is passed in by the caller and sized by alpaca_attention_workspace_bytes. Calls on different
 * streams may run concurrently; descriptors are read only during the call.
 */
#ifndef ALPACA_CUDA_H
#define ALPACA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ALPACA_CUDA_VERSION 10100 /* 1.1.0 */

/* Same object as cudaStream_t; NULL is the legacy default stream. */
typedef struct CUstream_st* alpaca_stream_t;

/* Status codes. Mirrors MetalError (MetalContext.swift:7-16): INVALID_ARGUMENT ~ .invalidArgument,
 * UNSUPPORTED ~ .unsupported, LAUNCH_FAILED / CUDA_ERROR / DEVICE_TIMEOUT ~ .commandFailed. */
typedef enum alpaca_cuda_status {
    ALPACA_CUDA_OK = 0,
    ALPACA_CUDA_ERR_INVALID_ARGUMENT = 1,    /* bad shape, stride, pointer, alignment or G above the limit */
    ALPACA_CUDA_ERR_UNSUPPORTED = 2,         /* valid request this build has no kernel for (dtype, head_dim) */
    ALPACA_CUDA_ERR_WORKSPACE_TOO_SMALL = 3, /* workspace_bytes below alpaca_attention_workspace_bytes() */
    ALPACA_CUDA_ERR_LAUNCH_FAILED = 4,       /* the kernel launch itself failed */
    ALPACA_CUDA_ERR_DEVICE_TIMEOUT = 5,      /* a bounded device-side wait gave up (see alpaca_cuda_device_status) */
    ALPACA_CUDA_ERR_CUDA = 6                 /* any other CUDA runtime / driver error */
} alpaca_cuda_status;

typedef enum alpaca_dtype {
    ALPACA_F32 = 0,
    ALPACA_F16 = 1 /* IEEE binary16 */
} alpaca_dtype;

/* Kernel selection. ALPACA_ATTN_AUTO applies the dispatch policy of KernelEncoder.attention
 * (KernelEncoder.swift:306-343): split decode for one f16-KV token with context >= ALPACA_DECODE_MINCTX,
 * the tensor-core prefill for f16 KV and >= 8 tokens, and the general fp32 kernel otherwise. */
typedef enum alpaca_attn_kernel {
    ALPACA_ATTN_AUTO = 0,
    ALPACA_ATTN_DECODE_SPLIT = 1, /* split-KV decode + combine (attention_decode.metal) */
    ALPACA_ATTN_PREFILL_TC = 2,   /* tcgen05 causal flash prefill (tensor_attention.metal, attention_prefill.metal) */
    ALPACA_ATTN_GENERAL = 3       /* fp32 SIMT online-softmax attention, f16 or f32 KV (attention.metal) */
} alpaca_attn_kernel;

/* Descriptor flags. */
#define ALPACA_ATTN_FLAG_NONE 0u
/* Ragged (varlen) prefill: the call's sequences have their own query counts and start positions, given by the
 * q_offsets / start_positions / total_tokens fields below (read only with this flag). Served by the tensor-core
 * prefill (ALPACA_ATTN_PREFILL_TC, or AUTO). */
#define ALPACA_ATTN_FLAG_VARLEN (1u << 0)
/* Fault-injection hook for tests: the tensor-core prefill kernel waits on a barrier nothing arrives at, with a
 * ~2 ms limit, so its bounded-wait give-up path runs. The call still returns OK (it only enqueues);
 * alpaca_cuda_device_status then reports ALPACA_CUDA_ERR_DEVICE_TIMEOUT. The output is unspecified. */
#define ALPACA_ATTN_FLAG_DEBUG_FORCE_TIMEOUT (1u << 31)

typedef struct alpaca_attn_desc {
    int32_t n_seqs;          /* independent sequences (or layers) in this call, >= 1 */
    int32_t n_heads;         /* query heads H */
    int32_t n_kv_heads;      /* KV heads Hkv; H % Hkv == 0 */
    int32_t head_dim;        /* d: multiple of 32, <= 256 (64 and 128 have fast kernels) */
    int32_t tokens;          /* query tokens per sequence, >= 1 */
    int32_t start_position;  /* absolute position of query token 0; visible KV rows = start_position + tokens */
    const int32_t* ctx_lens; /* decode only (tokens == 1): optional DEVICE array [n_seqs] of visible KV rows per
                                sequence (>= 1). When set it overrides start_position (start = ctx_len - 1). */
    int32_t max_ctx_len;     /* required with ctx_lens: an upper bound of every ctx_lens entry */
    int32_t q_dtype;         /* alpaca_dtype */
    int32_t kv_dtype;        /* alpaca_dtype (K and V share it) */
    int32_t out_dtype;       /* alpaca_dtype */
    int32_t reserved0;
    const void* q;
    int64_t q_token_stride;  /* elements between consecutive tokens (usually n_heads*head_dim) */
    int64_t q_seq_stride;    /* elements between sequences */
    const void* k;
    const void* v;
    int64_t kv_row_stride;   /* elements between cache rows (usually n_kv_heads*head_dim) */
    int64_t kv_seq_stride;   /* elements between sequences' caches */
    void* out;
    int64_t out_token_stride;
    int64_t out_seq_stride;
    float scale;             /* softmax scale; 0 selects 1/sqrt(head_dim) as CPUOps.attentionScores does */
    uint32_t flags;          /* ALPACA_ATTN_FLAG_* */
    /* Paged KV cache (optional; block_table == NULL means one contiguous cache per sequence). k and v then point
     * at pools of pool_blocks blocks, block_stride elements apart, each holding block_rows consecutive cache rows
     * (kv_row_stride apart); row r of sequence s lives in block block_table[s * max_blocks + r / block_rows] at
     * row r % block_rows, and kv_seq_stride is ignored. block_rows is a multiple of 128. Served by the split
     * decode and the tensor-core prefill kernels (f16 cache); alpaca.swift has no paged cache (README.md:257), so
     * this extends the layout of KernelEncoder.swift:9-17 for batched serving. */
    const int32_t* block_table; /* DEVICE array [n_seqs][max_blocks] of block indices into the pools */
    int32_t block_rows;
    int32_t max_blocks;
    int64_t block_stride;       /* elements between blocks of the pool */
    int32_t pool_blocks;        /* blocks in each pool (bounds of the TMA maps) */
    int32_t reserved1;
    /* Ragged prefill (flags & ALPACA_ATTN_FLAG_VARLEN; ignored otherwise): several sequences' query chunks in one
     * call, as a serving loop prefills the 512-token chunks of several sessions at their own positions
     * (MetalLlamaModel.swift:293-298 runs one session's chunk per call at a moving startPosition). q and out are
     * packed: sequence s owns token rows q_offsets[s] .. q_offsets[s+1]-1 of them (q_token_stride /
     * out_token_stride apart; q_seq_stride, out_seq_stride and start_position are ignored), and its query token t
     * sits at absolute position start_positions[s] + t of its own cache (kv_seq_stride apart, or through
     * block_table), whose first start_positions[s] + t + 1 rows it attends to. A sequence with no tokens is
     * skipped. Host-side bounds: `tokens` >= every sequence's token count (it sizes the workspace), max_ctx_len >=
     * every start_positions[s] + token count (each contiguous cache must hold max_ctx_len rows; a block table must
     * cover them), total_tokens = the rows of q and out. Rows of a cache past its sequence's context are never
     * used. Device arrays that break these bounds are reported by alpaca_cuda_device_status (INVALID_ARGUMENT) and
     * that sequence's output is not written. */
    const int32_t* q_offsets;       /* DEVICE [n_seqs + 1], non-decreasing, from >= 0 to <= total_tokens */
    const int32_t* start_positions; /* DEVICE [n_seqs], >= 0 */
    int32_t total_tokens;           /* rows of the packed q and out */
    int32_t reserved2;
} alpaca_attn_desc;

/* Enqueue attention described by `desc` with the kernel `kind` on `stream`.
 * Replaces KernelEncoder.attention (KernelEncoder.swift:306-343) when kind == ALPACA_ATTN_AUTO. */
alpaca_cuda_status alpaca_attention(const alpaca_attn_desc* desc, alpaca_attn_kernel kind, void* workspace,
                                    size_t workspace_bytes, alpaca_stream_t stream);

/* Tensor-core causal prefill (tcgen05 + TMEM + TMA). f16 KV; f16 or f32 Q (f32 Q is converted into the
 * workspace first, as MetalLlamaModel.swift:327 converts Q to half). Replaces KernelEncoder.attentionTensor
 * (KernelEncoder.swift:284-292) and the tiled attn_prefill branch (KernelEncoder.swift:328-335). With
 * ALPACA_ATTN_FLAG_VARLEN it prefills sequences of different lengths and start positions in one launch, their work
 * dealt to the SMs heaviest first across all sequences (the workspace then also holds that work list).
 * A call with fewer work items (sequences x heads x pairs of 128-query tiles; ragged: its bound, n_seqs x
 * ceil(tokens / 256) x heads) than SMs, such as one session's 512-token chunk at a moving start position
 * (MetalLlamaModel.swift:293-298) or a ragged step of a few sessions' chunks, splits each item's KV range into parts
 * that run on their own SMs and merges them in a second kernel, when the workspace is at least
 * alpaca_attention_workspace_bytes (the parts' records live there). Parts per item: min(8, floor(148 / items),
 * KV blocks / 4), so all parts fit one wave and each holds at least 4 KV blocks. A ragged unit uses as many of the
 * parts as its own KV blocks allow; a unit left whole writes its output directly. Given only the minimum (0 bytes for f16 queries, the f32
 * queries' staging otherwise, plus the ragged work list) the call runs unsplit. The results of the two agree to f32
 * rounding, but are not bit for bit equal. ALPACA_PREFILL_SPLITS=1 in the environment turns the split off. */
alpaca_cuda_status alpaca_attn_prefill(const alpaca_attn_desc* desc, void* workspace, size_t workspace_bytes,
                                       alpaca_stream_t stream);

/* Split-KV single-token decode over the f16 KV cache plus the combine kernel. Replaces the decode-split branch
 * of KernelEncoder.attention (KernelEncoder.swift:309-326). tokens must be 1. */
alpaca_cuda_status alpaca_attn_decode(const alpaca_attn_desc* desc, void* workspace, size_t workspace_bytes,
                                      alpaca_stream_t stream);

/* Split-KV decode that allocates nothing and takes no workspace. No counterpart in alpaca.swift: it is an
 * addition of this library for callers that cannot call cudaMalloc or hand over a scratch buffer, such as a host
 * runtime that owns every device allocation through its own fixed memory plan, or code running where allocation is
 * forbidden. Same computation, kernels and results as alpaca_attn_decode; the caller still passes every input and
 * output pointer in `desc`.
 *   - Split scratch lives in a file-scope device array of 8 MiB (8388608 bytes). Every GPU that loads the library
 *     holds it until the process exits. A call whose split state needs more (n_seqs * n_heads * splits *
 *     (head_dim + 2) * 4 bytes, see alpaca_attention_workspace_bytes) is rejected with
 *     ALPACA_CUDA_ERR_WORKSPACE_TOO_SMALL before anything is enqueued.
 *   - The first call on a device looks up the array's device address (cudaGetSymbolAddress, with that device
 *     current) and caches it; make that first call before any stream capture. The cached address is that of the
 *     runtime's primary context: the entry point is not meant for a caller's own driver-API context or for use
 *     across cudaDeviceReset (which unloads the array).
 *   - All calls on a device share the array, which keeps the last call's contents. Nothing in it needs to start at
 *     zero: every split state the combine step reads is written earlier in the same call. Calls that overlap on
 *     the GPU (different streams without ordering) race on the array; order them on one stream or with events.
 *   - No cudaMalloc, cudaFree or allocating library routine is called. */
alpaca_cuda_status alpaca_attn_decode_noalloc(const alpaca_attn_desc* desc, alpaca_stream_t stream);

/* Bytes of workspace `kind` needs for `desc` (0 when none). Replaces KernelEncoder.decodeScratchBytes
 * (KernelEncoder.swift:88-92). Host-only; enqueues nothing. For the tensor-core prefill this includes the split-KV
 * records of a call short of work items (see alpaca_attn_prefill), which a call may go without. */
alpaca_cuda_status alpaca_attention_workspace_bytes(const alpaca_attn_desc* desc, alpaca_attn_kernel kind,
                                                    size_t* bytes);

/* Which kernel ALPACA_ATTN_AUTO would run for `desc` (host-only policy query, KernelEncoder.swift:306-343);
 * ALPACA_CUDA_ERR_UNSUPPORTED when none can (a paged cache of f32 rows, for instance). */
alpaca_cuda_status alpaca_attention_select(const alpaca_attn_desc* desc, alpaca_attn_kernel* kind);

/* ---- RoPE + KV-cache append: the step that produces the attention hand-off (the next row upstream of it). */

/* Rotates q in place and appends rotated k and raw v to the KV cache, for `tokens` new tokens of each of n_seqs
 * sequences: token t of sequence s sits at absolute position pos = (positions ? positions[s] : start_position) + t;
 * its cache row is pos. Pair i of head_dim rotates by angle pos * theta^(-2i/head_dim), computed in double with
 * cos / sin rounded once to f32 and the rotation in f32, as CPUOps.rope (Sources/AlpacaCore/Operations/
 * CPUOps.swift:184-210) does; cache values are rounded to the cache type (f16: round to nearest even).
 *   q        [n_seqs][tokens][n_heads][head_dim]   f32 or f16, rotated in place (n_heads == 0: no queries)
 *   k, v     [n_seqs][tokens][n_kv_heads][head_dim] f32 projections (n_kv_heads == 0: no append)
 *   k_cache, v_cache [n_seqs][rows][n_kv_heads][head_dim] f16 or f32; rows > every written position
 * Pointers 8-byte aligned, strides in elements and even. The caller guarantees every written row exists. */
typedef struct alpaca_rope_desc {
    int32_t n_seqs;           /* >= 1 */
    int32_t n_heads;          /* query heads (0: rotate no queries) */
    int32_t n_kv_heads;       /* KV heads (0: append nothing) */
    int32_t head_dim;         /* even, 2 .. 256 */
    int32_t tokens;           /* new tokens per sequence, >= 1 */
    int32_t start_position;   /* position of token 0 when positions is NULL, >= 0 */
    const int32_t* positions; /* optional DEVICE array [n_seqs] of the position of each sequence's token 0 */
    float theta;              /* RoPE base (LlamaConfig.ropeTheta), > 0 */
    int32_t interleaved;      /* 1: adjacent pairs (x[2i], x[2i+1]), the layout of GGUF Llama files and of the
                                 Metal kernel; 0: split halves (x[i], x[i + head_dim/2]), "rotate_half" */
    int32_t q_dtype;          /* alpaca_dtype of q */
    int32_t cache_dtype;      /* alpaca_dtype of k_cache / v_cache */
    void* q;
    int64_t q_token_stride;
    int64_t q_seq_stride;
    const float* k;
    const float* v;
    int64_t kv_token_stride;  /* elements between tokens of k / v */
    int64_t kv_seq_stride;
    void* k_cache;
    void* v_cache;
    int64_t cache_row_stride; /* elements between cache rows */
    int64_t cache_seq_stride;
    uint32_t flags;           /* 0 */
    /* Paged cache (optional, the layout of alpaca_attn_desc's block_table): k_cache / v_cache are pools of
     * pool_blocks blocks of block_rows rows (a multiple of 128), block_stride elements apart; cache row pos of
     * sequence s is row pos % block_rows of block block_table[s * max_blocks + pos / block_rows];
     * cache_seq_stride is ignored. An entry outside the pool writes nothing and is reported by
     * alpaca_cuda_device_status. */
    const int32_t* block_table;
    int32_t block_rows;
    int32_t max_blocks;
    int64_t block_stride;
    int32_t pool_blocks;
    int32_t cache_rows;       /* rows of each contiguous cache, or 0 (unchecked); a token whose position is outside
                                 [0, cache_rows) writes no cache row and is reported by alpaca_cuda_device_status */
} alpaca_rope_desc;

/* Enqueue the fused RoPE + KV append on `stream`. Replaces KernelEncoder.ropeQKVStore (KernelEncoder.swift:
 * 401-411) and its rope_qkv_store_kv16 / _kv32 kernels (decode_fused.metal:126-154). */
alpaca_cuda_status alpaca_rope_kv_append(const alpaca_rope_desc* desc, alpaca_stream_t stream);

/* One decode step with the RoPE + KV append fused into the split-KV attention launch: the results of
 * alpaca_rope_kv_append(rope) followed by alpaca_attention(attn, ALPACA_ATTN_DECODE_SPLIT, ...) bit for bit, with
 * one kernel launch fewer (the pair MetalLlamaSession.encodeChunk issues per layer for a one-token chunk,
 * MetalLlamaModel.swift:347-351). Each sequence's new token is at position ctx_lens[s] - 1 (start_position when
 * ctx_lens is NULL): rope->positions must be NULL and rope->start_position equal attn->start_position. The RoPE
 * descriptor must describe that one token (tokens 1) of the same sequences, heads, q and f16 caches (same layout,
 * block table included). q is read and rotated as it is read, not rotated in place. Workspace as for the decode
 * call (alpaca_attention_workspace_bytes with ALPACA_ATTN_DECODE_SPLIT). */
alpaca_cuda_status alpaca_attn_decode_rope(const alpaca_attn_desc* attn, const alpaca_rope_desc* rope,
                                           void* workspace, size_t workspace_bytes, alpaca_stream_t stream);

/* ---- Fused decode projections: the mat-vec steps around the attention in a single-token decode step. */

/* Weight formats of alpaca_proj_desc: f16 rows, or GGUF blocks of 32 weights (q8_0: f16 scale + 32 int8, 34 bytes;
 * q4_0: f16 scale + 16 bytes whose low / high nibbles hold weights j / j + 16 as value + 8, 18 bytes). */
typedef enum alpaca_weight_format {
    ALPACA_W_F16 = 0,
    ALPACA_W_Q8_0 = 1,
    ALPACA_W_Q4_0 = 2
} alpaca_weight_format;

#define ALPACA_PROJ_NORM 1u /* RMS-normalise each input row first: x * (1 / sqrt(mean(x^2) + eps)) * norm_weight */
#define ALPACA_PROJ_SILU 2u /* y[0] = silu(W0 . xn) * (W1 . xn): the SwiGLU gate + up pair (rows[0] rows each) */
#define ALPACA_PROJ_ADD 4u  /* y_i += W_i . xn instead of y_i = W_i . xn: the projection with its residual */

/* y_i[t] = W_i . xn_t for the n_tokens input rows x_t (xn_t = x_t, or RMS-normalised with ALPACA_PROJ_NORM), up to
 * three matrices in one launch (Q, K and V: rows[0..2]), all in one format, f32 accumulation, f32 outputs. */
typedef struct alpaca_proj_desc {
    int32_t n_tokens;         /* input rows (one token, or one per sequence of a batched decode step), >= 1 */
    int32_t k;                /* input width: a multiple of 32, <= 16384 */
    int32_t rows[3];          /* output rows of W0, W1, W2 (0 for an absent matrix); ALPACA_PROJ_SILU: rows[0] rows
                                 in both W0 and W1, rows[1] = rows[2] = 0 */
    int32_t format;           /* alpaca_weight_format of every matrix */
    uint32_t flags;           /* ALPACA_PROJ_* */
    float eps;                /* RMSNorm epsilon (> 0) with ALPACA_PROJ_NORM */
    const void* w[3];         /* DEVICE weight matrices [rows_i][k] in `format`, 16-byte aligned */
    const float* x;           /* DEVICE input rows [n_tokens][x_stride] */
    int64_t x_stride;         /* elements between input rows, >= k */
    const float* norm_weight; /* DEVICE RMSNorm weight [k] (ALPACA_PROJ_NORM) */
    float* y[3];              /* DEVICE outputs [n_tokens][y_stride[i]] of matrix i (SILU: y[0] only) */
    int64_t y_stride[3];      /* elements between output rows, >= rows[i] */
} alpaca_proj_desc;

/* Enqueue the fused projection on `stream`. Replaces KernelEncoder.decodeQKV (norm + Q / K / V),
 * decodeProjection (optional norm, optional residual add: the out- and down-projections and the final logits) and
 * decodeGateUp (norm + SwiGLU gate and up) (Sources/AlpacaMetal/Backend/KernelEncoder.swift:386-400) and their
 * kernels dec_f16 / dec_q8_0 / dec_q4_0 (Sources/AlpacaMetal/Kernels/decode_fused.metal:32-122). alpaca.swift
 * runs these for one token (KernelEncoder.canFuseDecode, :362-366); n_tokens > 1 serves a batched decode step, every
 * weight read once per pass of up to 4 rows (larger batches belong to a GEMM). */
alpaca_cuda_status alpaca_decode_project(const alpaca_proj_desc* desc, alpaca_stream_t stream);

/* Synchronises `stream`, then reports and (when `clear` != 0) resets the device-side error word of that stream on the
 * current device: ALPACA_CUDA_ERR_DEVICE_TIMEOUT when a bounded wait gave up, ALPACA_CUDA_ERR_INVALID_ARGUMENT when
 * a device-side contract check failed (a block-table entry outside the pool, a ctx_lens entry outside
 * [1, max_ctx_len], a RoPE position outside the cache), ALPACA_CUDA_OK otherwise.
 * Each stream gets its own word on its first call on a device, so calls on other streams do not show here (the
 * streams beyond the first 1023 on a device share one word). Kernels captured into a CUDA graph report into the word
 * of the stream they were captured on, wherever the graph is replayed. The word addresses are looked up once per
 * device in the runtime's primary context: the library is not meant for other contexts or for use across
 * cudaDeviceReset. */
alpaca_cuda_status alpaca_cuda_device_status(alpaca_stream_t stream, int clear);

/* Static description of a status code. */
const char* alpaca_cuda_status_string(alpaca_cuda_status status);

/* Detail message of the last failing call on this host thread ("" when none). */
const char* alpaca_cuda_last_error(void);

/* ALPACA_CUDA_VERSION of the loaded library. */
int alpaca_cuda_version(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* ALPACA_CUDA_H */
