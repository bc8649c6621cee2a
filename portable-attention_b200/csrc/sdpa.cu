// pa_sdpa_fwd: descriptor validation and kernel choice for the forward pass.
#include <math.h>

#include <cstdio>

#include "common.cuh"
#include "kernels.h"

namespace pa {
namespace {

__global__ void fill_dead_kernel(uint8_t* out, size_t out_bytes, float* lse, int64_t rows) {
  const size_t tid = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = tid; i < out_bytes; i += stride) out[i] = 0;
  if (lse)
    for (size_t i = tid; i < static_cast<size_t>(rows); i += stride) lse[i] = -INFINITY;
}

size_t elem_size(int32_t dt) {
  switch (dt) {
    case PA_F16:
    case PA_BF16: return 2;
    case PA_F32: return 4;
    case PA_F64: return 8;
    case PA_BOOL: return 1;
    default: return 0;
  }
}

}  // namespace

pa_status launch_fill_dead(const pa_sdpa_desc& d, void* out, float* lse, cudaStream_t st) {
  const int64_t rows = lead_count(d) * d.L;
  const size_t bytes = static_cast<size_t>(rows) * d.Ev * elem_size(d.dtype);
  if (rows == 0) return PA_OK;
  fill_dead_kernel<<<sm_count() * 4, 256, 0, st>>>(static_cast<uint8_t*>(out), bytes, lse, rows);
  PA_CUDA(cudaGetLastError());
  return PA_OK;
}

// Structural checks shared by every entry point. Shape errors that the
// reference reports (reference.py:110-128) are caught by the Python host
// first; these guard the C ABI against inconsistent descriptors.
pa_status check_desc(const pa_sdpa_desc* d) {
  if (!d) return fail(PA_ERR_INVALID, "null descriptor");
  if (!elem_size(d->dtype) || d->dtype == PA_BOOL) return fail(PA_ERR_INVALID, "unknown dtype");
  if (d->nlead < 0 || d->nlead > PA_MAX_LEAD) return fail(PA_ERR_INVALID, "nlead out of range");
  if (d->L < 0 || d->S < 0 || d->E < 0 || d->Ev < 0) return fail(PA_ERR_INVALID, "negative extent");
  for (int i = 0; i < d->nlead; ++i)
    if (d->lead[i] < 0) return fail(PA_ERR_INVALID, "negative leading extent");
  if (d->gqa_group < 1) return fail(PA_ERR_INVALID, "gqa_group must be >= 1");
  if (d->gqa_group > 1) {
    if (d->gqa_axis < 0 || d->gqa_axis >= d->nlead)
      return fail(PA_ERR_INVALID, "gqa_axis must index a leading dim");
    if (d->lead[d->gqa_axis] % d->gqa_group)
      return fail(PA_ERR_INVALID, "query head count must be a multiple of gqa_group");
  }
  if (d->is_causal && d->mask_kind != PA_MASK_NONE)
    return fail(PA_ERR_INVALID, "Pass either is_causal=True or attn_mask, not both.");
  if (d->mask_kind == PA_MASK_BOOL && d->mask_dtype != PA_BOOL)
    return fail(PA_ERR_INVALID, "boolean mask must have mask_dtype PA_BOOL");
  if (d->mask_kind == PA_MASK_ADD &&
      d->mask_dtype != PA_F16 && d->mask_dtype != PA_BF16 && d->mask_dtype != PA_F32 &&
      d->mask_dtype != PA_F64)
    return fail(PA_ERR_INVALID, "additive mask must be a float type");
  if (d->mask_kind < 0 || d->mask_kind > PA_MASK_ADD) return fail(PA_ERR_INVALID, "unknown mask kind");
  if (!(d->scale == d->scale)) return fail(PA_ERR_INVALID, "scale is NaN");
  return PA_OK;
}

}  // namespace pa

using namespace pa;

extern "C" pa_status pa_sdpa_fwd(const pa_sdpa_desc* desc, const void* q, const void* k,
                                 const void* v, const void* mask, void* out, float* lse,
                                 void* stream) {
  clear_error();
  PA_TRY(check_desc(desc));
  const pa_sdpa_desc& d = *desc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (lead_count(d) == 0 || d.L == 0) return PA_OK;
  if (d.mask_kind != PA_MASK_NONE && !mask) return fail(PA_ERR_INVALID, "mask kind set but mask is null");
  if (d.S == 0) return launch_fill_dead(d, out, lse, st);
  if (fwd_tc_eligible(d, nullptr)) return launch_fwd_tc(d, q, k, v, mask, out, lse, st);
  return launch_fwd_exact(d, q, k, v, mask, out, lse, st);
}
