// Exact CUDA-core SDPA forward: any leading shape, any L/S/E/Ev, broadcast
// masks, grouped-query heads; fp64 math for fp64 operands, fp32 math (FFMA,
// no TF32) for fp32/fp16/bf16 operands.
//
// One warp owns one query row. Keys stream in chunks of 32 (one key per
// lane): the lane forms its score, the warp reduces the chunk max and sum,
// and the running output row (lanes own value columns) is rescaled and
// accumulated -- an online softmax whose result equals the two-pass
// max-shifted softmax of src/portable_attention/reference.py:151-162, with
// fully-masked rows exactly zero (l == 0 -> 0) and their lse -inf.
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace pa {
namespace {

constexpr int kWarps = 4;
constexpr int kEvPerLane = 8;  // value columns per lane per pass (256 per pass)

struct ExactArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* mask;
  void* out;
  float* lse;
  LeadTable lt;
  int64_t L, S, E, Ev;
  int64_t q_rs, k_rs, v_rs, m_rs, m_cs;
  int64_t nslices;
  int32_t causal;
  double scale;
};

template <typename T>
__device__ __forceinline__ float to_f(T x) { return static_cast<float>(x); }
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename Acc, typename T>
__device__ __forceinline__ Acc load_as(const T* p) {
  return static_cast<Acc>(to_f(*p));
}
template <>
__device__ __forceinline__ double load_as<double, double>(const double* p) { return *p; }

template <typename T>
__device__ __forceinline__ T from_acc(double x) { return static_cast<T>(x); }
template <>
__device__ __forceinline__ __half from_acc<__half>(double x) { return __float2half_rn(static_cast<float>(x)); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_acc<__nv_bfloat16>(double x) {
  return __float2bfloat16_rn(static_cast<float>(x));
}

__device__ __forceinline__ float exp_acc(float x) { return expf(x); }
__device__ __forceinline__ double exp_acc(double x) { return exp(x); }
__device__ __forceinline__ float log_acc(float x) { return logf(x); }
__device__ __forceinline__ double log_acc(double x) { return log(x); }

template <typename Acc>
__device__ __forceinline__ Acc warp_max(Acc x) {
  for (int o = 16; o; o >>= 1) x = fmax(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}
template <typename Acc>
__device__ __forceinline__ Acc warp_sum(Acc x) {
  for (int o = 16; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

template <typename T, typename Acc, int MASK, typename MaskT>
__global__ void __launch_bounds__(kWarps * 32) sdpa_exact_kernel(ExactArgs a) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t groups = (a.L + kWarps - 1) / kWarps;
  const int64_t slice = blockIdx.x / groups;
  const int64_t i = (blockIdx.x % groups) * kWarps + warp;
  if (slice >= a.nslices || i >= a.L) return;

  const SliceOffsets off = slice_offsets(a.lt, slice);
  const T* qrow = static_cast<const T*>(a.q) + off.q + i * a.q_rs;
  const T* kb = static_cast<const T*>(a.k) + off.k;
  const T* vb = static_cast<const T*>(a.v) + off.v;
  T* orow = static_cast<T*>(a.out) + (slice * a.L + i) * a.Ev;
  const Acc scale = static_cast<Acc>(a.scale);
  const Acc neg_inf = -static_cast<Acc>(INFINITY);
  // Keys past this bound are causally invisible to row i (top-left aligned).
  const int64_t s_end = a.causal ? (i + 1 < a.S ? i + 1 : a.S) : a.S;

  for (int64_t ev0 = 0; ev0 < a.Ev || (ev0 == 0 && a.Ev == 0); ev0 += 32 * kEvPerLane) {
    Acc acc[kEvPerLane];
#pragma unroll
    for (int c = 0; c < kEvPerLane; ++c) acc[c] = 0;
    Acc m = neg_inf, l = 0;

    for (int64_t j0 = 0; j0 < s_end; j0 += 32) {
      const int64_t j = j0 + lane;
      Acc s = neg_inf;
      if (j < s_end) {
        const T* krow = kb + j * a.k_rs;
        Acc dot = 0;
        for (int64_t e = 0; e < a.E; ++e) dot = fma(load_as<Acc>(qrow + e), load_as<Acc>(krow + e), dot);
        s = dot * scale;
        if (MASK == PA_MASK_BOOL) {
          const uint8_t keep = static_cast<const uint8_t*>(a.mask)[off.m + i * a.m_rs + j * a.m_cs];
          if (!keep) s = neg_inf;
        } else if (MASK == PA_MASK_ADD) {
          s += load_as<Acc>(static_cast<const MaskT*>(a.mask) + off.m + i * a.m_rs + j * a.m_cs);
        }
      }
      const Acc m_new = fmax(m, warp_max(s));
      if (m_new == neg_inf) continue;  // every key so far masked: nothing accumulates
      const Acc alpha = (m == neg_inf) ? Acc(0) : exp_acc(m - m_new);
      const Acc p = (s == neg_inf) ? Acc(0) : exp_acc(s - m_new);
      l = l * alpha + warp_sum(p);
#pragma unroll
      for (int c = 0; c < kEvPerLane; ++c) acc[c] *= alpha;
      const int nk = static_cast<int>(s_end - j0 < 32 ? s_end - j0 : 32);
      for (int t = 0; t < nk; ++t) {
        const Acc pt = __shfl_sync(0xffffffffu, p, t);
        const T* vrow = vb + (j0 + t) * a.v_rs + ev0;
#pragma unroll
        for (int c = 0; c < kEvPerLane; ++c) {
          const int64_t col = lane + 32 * c;
          if (ev0 + col < a.Ev) acc[c] = fma(pt, load_as<Acc>(vrow + col), acc[c]);
        }
      }
      m = m_new;
    }

#pragma unroll
    for (int c = 0; c < kEvPerLane; ++c) {
      const int64_t col = ev0 + lane + 32 * c;
      if (col < a.Ev) orow[col] = from_acc<T>(l > 0 ? static_cast<double>(acc[c] / l) : 0.0);
    }
    if (ev0 == 0 && a.lse && lane == 0)
      a.lse[slice * a.L + i] = l > 0 ? static_cast<float>(m + log_acc(l)) : -INFINITY;
    if (a.Ev == 0) break;
  }
}

template <typename T, typename Acc>
pa_status launch_typed(const ExactArgs& a, const pa_sdpa_desc& d, cudaStream_t st) {
  const int64_t blocks = a.nslices * ((a.L + kWarps - 1) / kWarps);
  if (blocks > 0x7fffffffLL) return fail(PA_ERR_UNSUPPORTED, "problem too large for the exact kernel");
  dim3 grid(static_cast<unsigned>(blocks)), block(kWarps * 32);
  if (d.mask_kind == PA_MASK_NONE || d.is_causal) {
    sdpa_exact_kernel<T, Acc, PA_MASK_NONE, float><<<grid, block, 0, st>>>(a);
  } else if (d.mask_kind == PA_MASK_BOOL) {
    sdpa_exact_kernel<T, Acc, PA_MASK_BOOL, uint8_t><<<grid, block, 0, st>>>(a);
  } else {
    switch (d.mask_dtype) {
      case PA_F16: sdpa_exact_kernel<T, Acc, PA_MASK_ADD, __half><<<grid, block, 0, st>>>(a); break;
      case PA_BF16: sdpa_exact_kernel<T, Acc, PA_MASK_ADD, __nv_bfloat16><<<grid, block, 0, st>>>(a); break;
      case PA_F32: sdpa_exact_kernel<T, Acc, PA_MASK_ADD, float><<<grid, block, 0, st>>>(a); break;
      case PA_F64: sdpa_exact_kernel<T, Acc, PA_MASK_ADD, double><<<grid, block, 0, st>>>(a); break;
      default: return fail(PA_ERR_INVALID, "unsupported additive mask dtype");
    }
  }
  PA_CUDA(cudaGetLastError());
  return PA_OK;
}

}  // namespace

pa_status launch_fwd_exact(const pa_sdpa_desc& d, const void* q, const void* k, const void* v,
                           const void* mask, void* out, float* lse, cudaStream_t st) {
  ExactArgs a{};
  a.q = q; a.k = k; a.v = v; a.mask = mask; a.out = out; a.lse = lse;
  a.lt = make_lead_table(d);
  a.L = d.L; a.S = d.S; a.E = d.E; a.Ev = d.Ev;
  a.q_rs = d.q_row_stride; a.k_rs = d.k_row_stride; a.v_rs = d.v_row_stride;
  a.m_rs = d.m_row_stride; a.m_cs = d.m_col_stride;
  a.nslices = lead_count(d);
  a.causal = d.is_causal;
  a.scale = d.scale;
  switch (d.dtype) {
    case PA_F64: return launch_typed<double, double>(a, d, st);
    case PA_F32: return launch_typed<float, float>(a, d, st);
    case PA_F16: return launch_typed<__half, float>(a, d, st);
    case PA_BF16: return launch_typed<__nv_bfloat16, float>(a, d, st);
    default: return fail(PA_ERR_INVALID, "unsupported dtype for the exact kernel");
  }
}

}  // namespace pa
