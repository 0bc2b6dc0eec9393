// api.cu — the C ABI (include/alpaca_cuda.h): argument validation, the kernel dispatch policy of alpaca.swift's
// KernelEncoder.attention (Sources/AlpacaMetal/Backend/KernelEncoder.swift:306-343), workspace sizing
// (KernelEncoder.decodeScratchBytes, :88-92), status codes mirroring MetalError (MetalContext.swift:7-31) and
// the per-stream device error words that bounded device-side waits and contract checks report into.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "common.cuh"
#include "internal.h"

namespace alpaca {

bool pdl_enabled() {
    static const bool v = [] {
        const char* e = std::getenv("ALPACA_PDL");
        return !(e && e[0] == '0');
    }();
    return v;
}

// Device error words. Each stream that calls into the library on a device gets its own word (a slot of this
// array), so a bounded wait that gives up or a bad index met by one call is reported to the caller that synchronises
// that stream, not to whichever caller reads first. Slot 0 is shared by the streams beyond the first
// kErrorSlots - 1 on a device. Kernels receive the address of their call's slot; host code reads it through
// alpaca_cuda_device_status.
constexpr int kErrorSlots = 1024;
__device__ unsigned g_error_slots[kErrorSlots];

namespace {

thread_local std::string t_last_error;

alpaca_cuda_status fail(alpaca_cuda_status st, const std::string& msg) {
    t_last_error = msg;
    return st;
}

alpaca_cuda_status ok() {
    t_last_error.clear();
    return ALPACA_CUDA_OK;
}

constexpr int kMaxDevices = 64;

struct DeviceState {
    unsigned* slots = nullptr;  // device address of g_error_slots on this device
    int num_sms = 0;
    bool ready = false;
    std::unordered_map<uintptr_t, int> slot_of;  // stream handle -> error slot
    int next_slot = 1;
};
DeviceState g_devices[kMaxDevices];
std::mutex g_devices_mu;

// What a launch needs from the current device: its SM count and the error word of `stream`.
struct DeviceInfo {
    unsigned* err = nullptr;
    int num_sms = 0;
};

// Per-device set-up, done once with that device current (address of the error slots, SM count), then the slot of
// `stream` (assigned on the stream's first call). The addresses are those of the context current at set-up, the
// runtime's primary context, and stay valid until the process exits or the device is reset.
cudaError_t device_info(cudaStream_t stream, DeviceInfo* out, bool assign = true, int* slot_out = nullptr) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_devices_mu);
    DeviceState& ds = g_devices[dev];
    if (!ds.ready) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_error_slots);
        if (e != cudaSuccess) return e;
        e = cudaDeviceGetAttribute(&ds.num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        ds.slots = static_cast<unsigned*>(p);
        ds.ready = true;
    }
    const uintptr_t key = reinterpret_cast<uintptr_t>(stream);
    int slot = -1;
    auto it = ds.slot_of.find(key);
    if (it != ds.slot_of.end()) {
        slot = it->second;
    } else if (assign) {
        slot = ds.next_slot < kErrorSlots ? ds.next_slot++ : 0;
        ds.slot_of.emplace(key, slot);
    }
    if (slot_out) *slot_out = slot;
    out->err = slot >= 0 ? ds.slots + slot : nullptr;
    out->num_sms = ds.num_sms;
    return cudaSuccess;
}

int env_int(const char* name, int fallback) {
    const char* v = std::getenv(name);
    if (!v || !*v) return fallback;
    char* end = nullptr;
    long x = std::strtol(v, &end, 10);
    return (end && *end == '\0') ? static_cast<int>(x) : fallback;
}

// Tuning knobs with the reference's names and defaults (KernelEncoder.swift:69-85).
int decode_min_ctx() {
    static const int v = env_int("ALPACA_DECODE_MINCTX", 64);
    return v;
}
constexpr int kPrefillMinTokens = 8;  // KernelEncoder.prefillAttentionMinTokens (:70)

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
size_t dtype_size(int dt) { return dt == ALPACA_F16 ? 2 : 4; }

std::string shape_str(const alpaca_attn_desc& d) {
    char buf[256];
    std::snprintf(buf, sizeof(buf), "seqs=%d T=%d start=%d H=%d/%d d=%d q=%s kv=%s out=%s", d.n_seqs, d.tokens,
                  d.start_position, d.n_heads, d.n_kv_heads, d.head_dim, d.q_dtype == ALPACA_F16 ? "f16" : "f32",
                  d.kv_dtype == ALPACA_F16 ? "f16" : "f32", d.out_dtype == ALPACA_F16 ? "f16" : "f32");
    return buf;
}

// Shape / pointer / stride checks (MetalOps.swift:179-181 plus what a raw-pointer ABI needs).
alpaca_cuda_status validate(const alpaca_attn_desc* dp) {
    if (!dp) return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: null descriptor");
    const alpaca_attn_desc& d = *dp;
    const std::string sh = shape_str(d);
    if (d.n_seqs < 1 || d.n_heads < 1 || d.n_kv_heads < 1 || d.tokens < 1 || d.start_position < 0)
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention shapes: " + sh);
    if (d.n_heads % d.n_kv_heads != 0)
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: heads not a multiple of kvHeads: " + sh);
    if (d.head_dim < 32 || d.head_dim > 256 || d.head_dim % 32 != 0)
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: headDim must be a multiple of 32 up to 256: " + sh);
    for (int dt : {d.q_dtype, d.kv_dtype, d.out_dtype})
        if (dt != ALPACA_F32 && dt != ALPACA_F16)
            return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: unknown dtype: " + sh);
    if (!d.q || !d.k || !d.v || !d.out) return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: null tensor pointer");
    if (!aligned16(d.q) || !aligned16(d.k) || !aligned16(d.v) || !aligned16(d.out))
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: tensor pointers must be 16-byte aligned");
    const int64_t hq = static_cast<int64_t>(d.n_heads) * d.head_dim, hk = static_cast<int64_t>(d.n_kv_heads) * d.head_dim;
    if (d.q_token_stride < hq || d.out_token_stride < hq || d.kv_row_stride < hk)
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: row strides smaller than a row: " + sh);
    if (d.q_seq_stride < 0 || d.kv_seq_stride < 0 || d.out_seq_stride < 0)
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: negative sequence stride");
    const bool varlen = (d.flags & ALPACA_ATTN_FLAG_VARLEN) != 0;
    if (d.n_seqs > 1 && ((!varlen && (d.q_seq_stride == 0 || d.out_seq_stride == 0)) ||
                         (!d.block_table && d.kv_seq_stride == 0)))
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: zero sequence stride with several sequences");
    if (varlen) {  // ragged prefill: packed queries, per-sequence offsets and start positions on the device
        if (d.ctx_lens)
            return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: ctx_lens and the ragged prefill flag together");
        if (!d.q_offsets || !d.start_positions)
            return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: ragged prefill needs q_offsets and start_positions");
        if (d.total_tokens < 1 || d.max_ctx_len < 1)
            return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT,
                        "attention: ragged prefill needs total_tokens >= 1 and max_ctx_len >= 1: " + sh);
        if (d.n_seqs > (1 << 24) || static_cast<int64_t>(d.n_seqs) * ((d.tokens + 255) / 256) > (1 << 26))
            return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: ragged prefill has too many sequences: " + sh);
    }
    const int64_t qs = static_cast<int64_t>(dtype_size(d.q_dtype)), ks = dtype_size(d.kv_dtype), os = dtype_size(d.out_dtype);
    if ((d.q_token_stride * qs) % 16 || (d.q_seq_stride * qs) % 16 || (d.kv_row_stride * ks) % 16 ||
        (d.kv_seq_stride * ks) % 16 || (d.out_token_stride * os) % 16 || (d.out_seq_stride * os) % 16)
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: strides must be multiples of 16 bytes");
    if (d.ctx_lens) {
        if (d.tokens != 1)
            return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: ctx_lens is only valid for one-token decode");
        if (d.max_ctx_len < 1)
            return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: max_ctx_len must bound ctx_lens (>= 1)");
    }
    if (d.start_position > (1 << 30) || d.tokens > (1 << 30) - d.start_position)
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: positions out of range: " + sh);
    if (!(d.scale >= 0.f) || !std::isfinite(d.scale))
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: scale must be finite and >= 0");
    if (d.block_table) {  // paged cache
        const int64_t rows_needed =
            (d.ctx_lens || varlen) ? d.max_ctx_len : static_cast<int64_t>(d.start_position) + d.tokens;
        if (d.block_rows < 128 || d.block_rows % 128 != 0)
            return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: block_rows must be a positive multiple of 128");
        if (d.max_blocks < 1 || d.pool_blocks < 1 ||
            rows_needed > static_cast<int64_t>(d.max_blocks) * d.block_rows)
            return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: block table too short for the context: " + sh);
        if (d.block_stride < static_cast<int64_t>(d.block_rows) * d.kv_row_stride || (d.block_stride * ks) % 16)
            return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT,
                        "attention: block_stride must cover block_rows rows and be a multiple of 16 bytes");
    }
    return ok();
}

// RoPE + KV append checks (CPUOps.rope's guards, CPUOps.swift:188-191, plus what a raw-pointer ABI needs).
alpaca_cuda_status validate_rope(const alpaca_rope_desc* dp) {
    if (!dp) return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "rope: null descriptor");
    const alpaca_rope_desc& d = *dp;
    char sh[200];
    std::snprintf(sh, sizeof(sh), "seqs=%d T=%d start=%d H=%d/%d d=%d", d.n_seqs, d.tokens, d.start_position,
                  d.n_heads, d.n_kv_heads, d.head_dim);
    if (d.n_seqs < 1 || d.n_seqs > 65535 || d.tokens < 1 || d.n_heads < 0 || d.n_kv_heads < 0 ||
        d.n_heads + d.n_kv_heads < 1 || d.start_position < 0)
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, std::string("rope shapes: ") + sh);
    if (d.head_dim < 2 || d.head_dim % 2 != 0 || d.head_dim > rope_max_head_dim())
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, std::string("rope: headDim must be even, 2..256: ") + sh);
    if (!(d.theta > 0.f) || !std::isfinite(d.theta))
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "rope: theta must be finite and > 0");
    if (d.interleaved != 0 && d.interleaved != 1)
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "rope: interleaved must be 0 or 1");
    if (d.flags != 0) return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "rope: unknown flags");
    if (d.start_position > (1 << 30) || d.tokens > (1 << 30) - d.start_position)
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, std::string("rope: positions out of range: ") + sh);
    auto al8 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; };
    if (d.n_heads > 0) {
        if (d.q_dtype != ALPACA_F32 && d.q_dtype != ALPACA_F16)
            return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "rope: unknown q dtype");
        if (!d.q || !al8(d.q)) return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "rope: q null or not 8-byte aligned");
        if (d.q_token_stride < static_cast<int64_t>(d.n_heads) * d.head_dim || d.q_seq_stride < 0 ||
            (d.n_seqs > 1 && d.q_seq_stride == 0) || d.q_token_stride % 2 || d.q_seq_stride % 2)
            return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, std::string("rope: q strides: ") + sh);
    }
    if (d.n_kv_heads > 0) {
        if (d.cache_dtype != ALPACA_F32 && d.cache_dtype != ALPACA_F16)
            return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "rope: unknown cache dtype");
        if (!d.k || !d.v || !d.k_cache || !d.v_cache)
            return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "rope: null k / v / cache pointer");
        if (!al8(d.k) || !al8(d.v) || !al8(d.k_cache) || !al8(d.v_cache))
            return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "rope: k / v / cache pointers must be 8-byte aligned");
        const int64_t hk = static_cast<int64_t>(d.n_kv_heads) * d.head_dim;
        if (d.kv_token_stride < hk || d.cache_row_stride < hk || d.kv_seq_stride < 0 || d.cache_seq_stride < 0 ||
            (d.n_seqs > 1 && (d.kv_seq_stride == 0 || (d.cache_seq_stride == 0 && !d.block_table))) ||
            d.kv_token_stride % 2 ||
            d.kv_seq_stride % 2 || d.cache_row_stride % 2 || d.cache_seq_stride % 2)
            return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, std::string("rope: k / v / cache strides: ") + sh);
        if (d.cache_rows < 0) return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, std::string("rope: cache_rows < 0: ") + sh);
        if (!d.block_table && d.cache_rows > 0 && !d.positions &&
            static_cast<int64_t>(d.start_position) + d.tokens > d.cache_rows)
            return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, std::string("rope: rows past cache_rows: ") + sh);
        if (d.block_table) {
            if (d.block_rows < 128 || d.block_rows % 128 || d.max_blocks < 1 || d.pool_blocks < 1 ||
                d.block_stride < static_cast<int64_t>(d.block_rows) * d.cache_row_stride || d.block_stride % 2)
                return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT,
                            std::string("rope: paged cache needs block_rows a multiple of 128, max_blocks and pool_blocks "
                                        ">= 1, block_stride covering a block and even: ") + sh);
            if (!d.positions && static_cast<int64_t>(d.start_position) + d.tokens >
                                    static_cast<int64_t>(d.max_blocks) * d.block_rows)
                return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, std::string("rope: block table too short: ") + sh);
        }
    }
    return ok();
}

// KernelEncoder.attention's policy (KernelEncoder.swift:309-343).
alpaca_attn_kernel select_kernel(const alpaca_attn_desc& d) {
    if (d.flags & ALPACA_ATTN_FLAG_VARLEN) return ALPACA_ATTN_PREFILL_TC;  // the only kernel with the ragged form
    if (d.block_table)  // a paged cache is read by the split decode (any context) and the tensor-core prefill only
        return (d.tokens == 1 && decode_supported(d)) ? ALPACA_ATTN_DECODE_SPLIT : ALPACA_ATTN_PREFILL_TC;
    const int ctx = d.ctx_lens ? d.max_ctx_len : d.start_position + 1;
    if (d.tokens == 1 && decode_supported(d) && (d.ctx_lens || ctx >= decode_min_ctx())) return ALPACA_ATTN_DECODE_SPLIT;
    if (d.tokens >= kPrefillMinTokens && prefill_supported(d)) return ALPACA_ATTN_PREFILL_TC;
    return ALPACA_ATTN_GENERAL;
}

size_t workspace_for(const alpaca_attn_desc& d, alpaca_attn_kernel k) {
    switch (k) {
        case ALPACA_ATTN_DECODE_SPLIT: return decode_workspace_bytes(d);
        case ALPACA_ATTN_PREFILL_TC: return prefill_workspace_bytes(d);
        default: return 0;
    }
}

alpaca_cuda_status check_kind(const alpaca_attn_desc& d, alpaca_attn_kernel k) {
    if ((d.flags & ALPACA_ATTN_FLAG_VARLEN) && k != ALPACA_ATTN_PREFILL_TC && k != ALPACA_ATTN_AUTO)
        return fail(ALPACA_CUDA_ERR_UNSUPPORTED, "the ragged prefill form is served by the tensor-core prefill only");
    switch (k) {
        case ALPACA_ATTN_DECODE_SPLIT:
            if (!decode_supported(d))
                return fail(ALPACA_CUDA_ERR_UNSUPPORTED,
                            "split decode needs tokens=1, f16 KV, headDim 64/128 and heads/kvHeads <= 8: " + shape_str(d));
            return ok();
        case ALPACA_ATTN_PREFILL_TC:
            if (!prefill_supported(d))
                return fail(ALPACA_CUDA_ERR_UNSUPPORTED,
                            "tensor-core prefill needs f16 KV and headDim 64/128: " + shape_str(d));
            return ok();
        case ALPACA_ATTN_GENERAL:
            if (d.block_table)
                return fail(ALPACA_CUDA_ERR_UNSUPPORTED, "the general kernel reads contiguous caches only (paged cache given)");
            return ok();
        default: return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "attention: unknown kernel kind");
    }
}

float call_scale(const alpaca_attn_desc& d) {
    return d.scale > 0.f ? d.scale : 1.0f / std::sqrt(static_cast<float>(d.head_dim));
}

// The host-side checks every attention entry point shares: the descriptor, then the kernel choice
// (ALPACA_ATTN_AUTO resolved) and its limits.
alpaca_cuda_status prepare(const alpaca_attn_desc* dp, alpaca_attn_kernel& kind) {
    alpaca_cuda_status st = validate(dp);
    if (st != ALPACA_CUDA_OK) return st;
    if (kind == ALPACA_ATTN_AUTO) kind = select_kernel(*dp);
    return check_kind(*dp, kind);
}

// The device set-up every launch shares (SM count, this stream's error word); `who` prefixes the message.
alpaca_cuda_status device_for(cudaStream_t stream, const char* who, DeviceInfo* di) {
    const cudaError_t e = device_info(stream, di);
    if (e != cudaSuccess) return fail(ALPACA_CUDA_ERR_CUDA, std::string(who) + ": device query: " + cudaGetErrorString(e));
    return ok();
}

// Caller workspace against what `kind` needs for `d`.
alpaca_cuda_status check_workspace(const alpaca_attn_desc& d, alpaca_attn_kernel kind, const void* ws, size_t ws_bytes,
                                   const char* who) {
    // the tensor-core prefill runs unsplit when given less than its query size, so only its minimum is required
    const size_t need = kind == ALPACA_ATTN_PREFILL_TC ? prefill_workspace_min_bytes(d) : workspace_for(d, kind);
    if (need > 0 && (ws_bytes < need || !ws))
        return fail(ALPACA_CUDA_ERR_WORKSPACE_TOO_SMALL, std::string(who) + ": workspace of " + std::to_string(ws_bytes) +
                                                             " bytes, " + std::to_string(need) + " needed");
    if (need > 0 && !aligned16(ws))
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, std::string(who) + ": workspace must be 16-byte aligned");
    return ok();
}

alpaca_cuda_status launched(cudaError_t e, const char* who) {
    if (e != cudaSuccess)
        return fail(ALPACA_CUDA_ERR_LAUNCH_FAILED, std::string(who) + " launch failed: " + cudaGetErrorString(e));
    return ok();
}

alpaca_cuda_status run(const alpaca_attn_desc* dp, alpaca_attn_kernel kind, void* ws, size_t ws_bytes,
                       cudaStream_t stream) {
    alpaca_cuda_status st = prepare(dp, kind);
    if (st != ALPACA_CUDA_OK) return st;
    const alpaca_attn_desc& d = *dp;
    st = check_workspace(d, kind, ws, ws_bytes, "attention");
    if (st != ALPACA_CUDA_OK) return st;
    DeviceInfo di;
    st = device_for(stream, "attention", &di);
    if (st != ALPACA_CUDA_OK) return st;
    Call c{&d, call_scale(d), di.err, ws, ws_bytes, di.num_sms};
    cudaError_t e;
    switch (kind) {
        case ALPACA_ATTN_DECODE_SPLIT: e = launch_decode(c, stream); break;
        case ALPACA_ATTN_PREFILL_TC: e = launch_prefill(c, stream); break;
        default: e = launch_general(c, stream); break;
    }
    return launched(e, "attention");
}

}  // namespace
}  // namespace alpaca

using namespace alpaca;

extern "C" {

alpaca_cuda_status alpaca_attention(const alpaca_attn_desc* desc, alpaca_attn_kernel kind, void* workspace,
                                    size_t workspace_bytes, alpaca_stream_t stream) {
    return run(desc, kind, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

alpaca_cuda_status alpaca_attn_prefill(const alpaca_attn_desc* desc, void* workspace, size_t workspace_bytes,
                                       alpaca_stream_t stream) {
    return run(desc, ALPACA_ATTN_PREFILL_TC, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

alpaca_cuda_status alpaca_attn_decode(const alpaca_attn_desc* desc, void* workspace, size_t workspace_bytes,
                                      alpaca_stream_t stream) {
    return run(desc, ALPACA_ATTN_DECODE_SPLIT, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

alpaca_cuda_status alpaca_attn_decode_noalloc(const alpaca_attn_desc* desc, alpaca_stream_t stream) {
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    alpaca_attn_kernel kind = ALPACA_ATTN_DECODE_SPLIT;
    alpaca_cuda_status st = prepare(desc, kind);
    if (st != ALPACA_CUDA_OK) return st;
    const size_t need = decode_workspace_bytes(*desc);
    if (need > kDecodeBuiltinScratchBytes)
        return fail(ALPACA_CUDA_ERR_WORKSPACE_TOO_SMALL,
                    "decode_noalloc: this call needs " + std::to_string(need) + " bytes of split scratch; the built-in " +
                        "scratch holds " + std::to_string(kDecodeBuiltinScratchBytes) +
                        " bytes (use alpaca_attn_decode with a workspace)");
    DeviceInfo di;
    st = device_for(s, "decode_noalloc", &di);
    if (st != ALPACA_CUDA_OK) return st;
    void* scratch = nullptr;
    const cudaError_t e = decode_builtin_scratch(&scratch);
    if (e != cudaSuccess)
        return fail(ALPACA_CUDA_ERR_CUDA, std::string("decode_noalloc: scratch address: ") + cudaGetErrorString(e));
    Call c{desc, call_scale(*desc), di.err, scratch, kDecodeBuiltinScratchBytes, di.num_sms};
    return launched(launch_decode(c, s), "decode_noalloc");
}

alpaca_cuda_status alpaca_attn_decode_rope(const alpaca_attn_desc* attn, const alpaca_rope_desc* rope,
                                           void* workspace, size_t workspace_bytes, alpaca_stream_t stream) {
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    alpaca_attn_kernel kind = ALPACA_ATTN_DECODE_SPLIT;
    alpaca_cuda_status st = prepare(attn, kind);
    if (st != ALPACA_CUDA_OK) return st;
    st = validate_rope(rope);
    if (st != ALPACA_CUDA_OK) return st;
    const alpaca_attn_desc& d = *attn;
    const alpaca_rope_desc& r = *rope;
    auto bad = [](const char* what) { return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, std::string("decode_rope: ") + what); };
    if (r.n_seqs != d.n_seqs || r.tokens != 1 || r.n_heads != d.n_heads || r.n_kv_heads != d.n_kv_heads ||
        r.head_dim != d.head_dim)
        return bad("the RoPE descriptor must describe one new token of the attention call's sequences and heads");
    if (r.q != d.q || r.q_dtype != d.q_dtype || (d.n_seqs > 1 && r.q_seq_stride != d.q_seq_stride))
        return bad("the RoPE descriptor's q must be the attention call's q");
    if (r.cache_dtype != ALPACA_F16 || r.k_cache != d.k || r.v_cache != d.v || r.cache_row_stride != d.kv_row_stride)
        return bad("the RoPE descriptor's caches must be the attention call's f16 K / V caches");
    if (r.block_table != d.block_table ||
        (d.block_table ? (r.block_rows != d.block_rows || r.max_blocks != d.max_blocks ||
                          r.block_stride != d.block_stride || r.pool_blocks != d.pool_blocks)
                       : (d.n_seqs > 1 && r.cache_seq_stride != d.kv_seq_stride)))
        return bad("the RoPE descriptor's cache layout must be the attention call's");
    if (r.positions || (!d.ctx_lens && r.start_position != d.start_position))
        return bad("the new token's position is the attention call's (ctx_lens - 1, or start_position): positions "
                   "must be NULL and start_position equal to the attention descriptor's");
    st = check_workspace(d, kind, workspace, workspace_bytes, "decode_rope");
    if (st != ALPACA_CUDA_OK) return st;
    DeviceInfo di;
    st = device_for(s, "decode_rope", &di);
    if (st != ALPACA_CUDA_OK) return st;
    Call c{attn, call_scale(d), di.err, workspace, workspace_bytes, di.num_sms};
    c.rope = rope;
    return launched(launch_decode(c, s), "decode_rope");
}

alpaca_cuda_status alpaca_rope_kv_append(const alpaca_rope_desc* desc, alpaca_stream_t stream) {
    alpaca_cuda_status st = validate_rope(desc);
    if (st != ALPACA_CUDA_OK) return st;
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    DeviceInfo di;
    st = device_for(s, "rope", &di);
    if (st != ALPACA_CUDA_OK) return st;
    return launched(launch_rope_kv(*desc, di.err, s), "rope");
}

alpaca_cuda_status alpaca_decode_project(const alpaca_proj_desc* dp, alpaca_stream_t stream) {
    if (!dp) return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "project: null descriptor");
    const alpaca_proj_desc& d = *dp;
    char sh[160];
    std::snprintf(sh, sizeof(sh), "tokens=%d k=%d rows=%d/%d/%d format=%d flags=%u", d.n_tokens, d.k, d.rows[0],
                  d.rows[1], d.rows[2], d.format, d.flags);
    auto bad = [&](const char* what) {
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, std::string("project: ") + what + ": " + sh);
    };
    if (d.format != ALPACA_W_F16 && d.format != ALPACA_W_Q8_0 && d.format != ALPACA_W_Q4_0)
        return fail(ALPACA_CUDA_ERR_UNSUPPORTED, std::string("project: unknown weight format: ") + sh);
    if (d.flags & ~(ALPACA_PROJ_NORM | ALPACA_PROJ_SILU | ALPACA_PROJ_ADD)) return bad("unknown flags");
    if (d.n_tokens < 1 || d.k < 32 || d.k % 32 || d.k > 16384) return bad("n_tokens >= 1 and k a multiple of 32 up to 16384");
    const bool silu = (d.flags & ALPACA_PROJ_SILU) != 0;
    if (silu && (d.flags & ALPACA_PROJ_ADD)) return bad("SILU and ADD together");
    if (silu ? (d.rows[0] < 1 || d.rows[1] != 0 || d.rows[2] != 0)
             : (d.rows[0] < 0 || d.rows[1] < 0 || d.rows[2] < 0 || d.rows[0] + d.rows[1] + d.rows[2] < 1))
        return bad("row counts");
    const int used = silu ? 2 : 3;
    for (int i = 0; i < used; i++) {
        const bool present = silu || d.rows[i] > 0;
        if (!present) continue;
        if (!d.w[i] || !aligned16(d.w[i])) return bad("weights null or not 16-byte aligned");
        if (i == 0 || !silu) {
            if (!d.y[i] || (reinterpret_cast<uintptr_t>(d.y[i]) & 3u)) return bad("outputs null or not 4-byte aligned");
            const int r = d.rows[i];
            if (d.n_tokens > 1 && d.y_stride[i] < r) return bad("output stride smaller than its rows");
        }
    }
    if (!d.x || (reinterpret_cast<uintptr_t>(d.x) & 3u)) return bad("input null or not 4-byte aligned");
    if (d.n_tokens > 1 && d.x_stride < d.k) return bad("input stride smaller than k");
    if (d.flags & ALPACA_PROJ_NORM) {
        if (!d.norm_weight || (reinterpret_cast<uintptr_t>(d.norm_weight) & 3u)) return bad("norm weight null or unaligned");
        if (!(d.eps > 0.f) || !std::isfinite(d.eps)) return bad("eps must be finite and > 0");
    }
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    DeviceInfo di;
    const alpaca_cuda_status st = device_for(s, "project", &di);
    if (st != ALPACA_CUDA_OK) return st;
    return launched(launch_proj(d, di.num_sms, s), "project");
}

alpaca_cuda_status alpaca_attention_workspace_bytes(const alpaca_attn_desc* desc, alpaca_attn_kernel kind,
                                                    size_t* bytes) {
    if (!bytes) return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "workspace_bytes: null output");
    alpaca_cuda_status st = validate(desc);
    if (st != ALPACA_CUDA_OK) return st;
    if (kind == ALPACA_ATTN_AUTO) kind = select_kernel(*desc);
    st = check_kind(*desc, kind);
    if (st != ALPACA_CUDA_OK) return st;
    *bytes = workspace_for(*desc, kind);
    return ok();
}

alpaca_cuda_status alpaca_attention_select(const alpaca_attn_desc* desc, alpaca_attn_kernel* kind) {
    if (!kind) return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT, "select: null output");
    alpaca_cuda_status st = validate(desc);
    if (st != ALPACA_CUDA_OK) return st;
    *kind = select_kernel(*desc);
    return check_kind(*desc, *kind);  // UNSUPPORTED when no kernel can serve it (only possible with a paged cache)
}

alpaca_cuda_status alpaca_cuda_device_status(alpaca_stream_t stream, int clear) {
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail(ALPACA_CUDA_ERR_CUDA, std::string("device status: ") + cudaGetErrorString(e));
    DeviceInfo di;
    int slot = -1;
    e = device_info(s, &di, /*assign=*/false, &slot);
    if (e != cudaSuccess) return fail(ALPACA_CUDA_ERR_CUDA, std::string("device status: ") + cudaGetErrorString(e));
    if (slot < 0) return ok();  // this stream has made no call on the current device
    unsigned word = 0;
    const size_t off = sizeof(unsigned) * static_cast<size_t>(slot);
    e = cudaMemcpyFromSymbol(&word, g_error_slots, sizeof(word), off);
    if (e != cudaSuccess) return fail(ALPACA_CUDA_ERR_CUDA, std::string("device status: ") + cudaGetErrorString(e));
    if (clear && word) {
        const unsigned zero = 0;
        e = cudaMemcpyToSymbol(g_error_slots, &zero, sizeof(zero), off);
        if (e != cudaSuccess) return fail(ALPACA_CUDA_ERR_CUDA, std::string("device status: ") + cudaGetErrorString(e));
    }
    if (word & kDevErrTimeout) return fail(ALPACA_CUDA_ERR_DEVICE_TIMEOUT, "a bounded device-side wait gave up");
    if (word & kDevErrBadIndex)
        return fail(ALPACA_CUDA_ERR_INVALID_ARGUMENT,
                    "a device-side contract check failed: a block table entry outside the KV pool (rows read as zero), "
                    "a context length outside [1, max_ctx_len], or a position outside the cache");
    if (word) return fail(ALPACA_CUDA_ERR_CUDA, "device error word " + std::to_string(word));
    return ok();
}

const char* alpaca_cuda_status_string(alpaca_cuda_status status) {
    switch (status) {
        case ALPACA_CUDA_OK: return "ok";
        case ALPACA_CUDA_ERR_INVALID_ARGUMENT: return "invalid argument";
        case ALPACA_CUDA_ERR_UNSUPPORTED: return "unsupported";
        case ALPACA_CUDA_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
        case ALPACA_CUDA_ERR_LAUNCH_FAILED: return "kernel launch failed";
        case ALPACA_CUDA_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
        case ALPACA_CUDA_ERR_CUDA: return "CUDA error";
    }
    return "unknown status";
}

const char* alpaca_cuda_last_error(void) { return t_last_error.c_str(); }

int alpaca_cuda_version(void) { return ALPACA_CUDA_VERSION; }

}  // extern "C"
