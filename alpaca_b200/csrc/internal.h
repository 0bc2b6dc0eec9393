// internal.h — launchers shared between the C-ABI front end (api.cu) and the kernel translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/alpaca_cuda.h"

namespace alpaca {

// A validated call: the caller's descriptor plus the values the front end resolved for it.
struct Call {
    const alpaca_attn_desc* d;
    float scale;        // softmax scale (desc.scale or 1/sqrt(d))
    unsigned* err;      // device error word of the current device
    void* ws;           // caller workspace (may be null when the kernel needs none)
    size_t ws_bytes;
    int num_sms;        // multiprocessors of the current device
    const alpaca_rope_desc* rope = nullptr;  // decode with the RoPE + KV append fused in (alpaca_attn_decode_rope)
};

// ---- split-KV decode (attn_decode.cu)
int decode_split_len(int head_dim);                          // KV rows per split CTA
int decode_max_splits(const alpaca_attn_desc& d);            // splits of the longest sequence
size_t decode_workspace_bytes(const alpaca_attn_desc& d);    // partial-state bytes
bool decode_supported(const alpaca_attn_desc& d);            // head_dim / group limits of the kernel
cudaError_t launch_decode(const Call& c, cudaStream_t s);
// Programmatic dependent launch of the attention kernels (ALPACA_PDL=0 turns it off).
bool pdl_enabled();
// Built-in scratch of alpaca_attn_decode_noalloc (file-scope device array in attn_decode.cu).
constexpr size_t kDecodeBuiltinScratchBytes = size_t(8) << 20;  // 8 MiB
cudaError_t decode_builtin_scratch(void** ptr);

// ---- general fp32 SIMT attention (attn_general.cu)
cudaError_t launch_general(const Call& c, cudaStream_t s);

// ---- RoPE + KV-cache append (rope_kv.cu)
int rope_max_head_dim();
cudaError_t launch_rope_kv(const alpaca_rope_desc& d, unsigned* err, cudaStream_t s);

// ---- fused decode projections (decode_proj.cu)
int64_t proj_row_bytes(int format, int k);  // bytes of one weight row (0 for an unknown format)
cudaError_t launch_proj(const alpaca_proj_desc& d, int num_sms, cudaStream_t s);

// ---- tcgen05 prefill (attn_prefill_sm100.cu)
bool prefill_supported(const alpaca_attn_desc& d);
// f32 -> f16 Q staging when q_dtype is f32, the ragged work list, and the split-KV records of a call with fewer
// work items than SMs (the query size; a call given only the minimum runs unsplit)
size_t prefill_workspace_bytes(const alpaca_attn_desc& d);
size_t prefill_workspace_min_bytes(const alpaca_attn_desc& d);
cudaError_t launch_prefill(const Call& c, cudaStream_t s);

}  // namespace alpaca
