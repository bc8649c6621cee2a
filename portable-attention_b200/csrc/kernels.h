// Internal launcher declarations shared by the C-ABI entry points.
#pragma once

#include <functional>

#include "common.cuh"

namespace pa {

// Structural checks of a descriptor shared by every entry point.
pa_status check_desc(const pa_sdpa_desc* d);

pa_status launch_fwd_exact(const pa_sdpa_desc& d, const void* q, const void* k, const void* v,
                           const void* mask, void* out, float* lse, cudaStream_t st);

// Dense (B, H, L, D) fp16/bf16 operands, D in {64, 128}.
bool fwd_tc_eligible(const pa_sdpa_desc& d, std::string* why);
pa_status launch_fwd_tc(const pa_sdpa_desc& d, const void* q, const void* k, const void* v,
                        const void* mask, void* out, float* lse, cudaStream_t st);

// Fill out with zeros and lse with -inf (S == 0: every row fully masked).
pa_status launch_fill_dead(const pa_sdpa_desc& d, void* out, float* lse, cudaStream_t st);

// True when q/k/v are dense (B..., H, rows, D) with grouped heads on the last
// leading axis; reports the flattened slice count and head counts.
bool dense_bhsd(const pa_sdpa_desc& d, int64_t* slices, int64_t* heads, int64_t* kv_heads);

// Split-KV decode (query length 1) on dense operands: workspace size, and a
// run with a caller-provided workspace (csrc/decode.cu).
pa_status decode_ws_bytes(const pa_sdpa_desc& d, size_t* bytes);
pa_status run_decode(const pa_sdpa_desc& d, const void* q, const void* k, const void* v, void* out,
                     float* lse, void* ws, size_t ws_bytes, cudaStream_t st);

// Backward of one dense call whose dQ, dK, dV are added in fp32 into the given
// accumulators (dense layouts of dq / dk / dv) instead of being stored (csrc/bwd.cu).
// `before_dkdv` runs on the host after the dQ kernel is enqueued and before the
// dK/dV kernel (e.g. a stream wait for accumulators that are still arriving).
pa_status bwd_accumulate(const pa_sdpa_desc& d, const void* q, const void* k, const void* v,
                         const void* out, const void* dout, const float* lse, float* dq_acc,
                         float* dk_acc, float* dv_acc, cudaStream_t st,
                         const std::function<void()>& before_dkdv);

// Reads and clears the status word pa_decode_fwd_static uses when its caller
// passes none (0 on a device where that entry point never ran).
pa_status take_static_decode_status(int* code);

}  // namespace pa
