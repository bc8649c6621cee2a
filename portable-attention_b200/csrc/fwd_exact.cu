// Exact CUDA-core SDPA forward: any leading shape, any L/S/E/Ev, broadcast
// masks, grouped-query heads; fp64 math for fp64 operands, fp32 math (FFMA,
// no TF32) for fp32/fp16/bf16 operands.
//
// One warp owns one query row (when E, Ev <= 256: two rows per warp, 32 rows
// per CTA sharing 32-key K/V tiles in shared memory). Keys stream in chunks of 32 (one key per
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

// ---------------------------------------------------------------------------
// Tiled variant for E, Ev <= 256: a CTA of 16 warps owns 16 consecutive query
// rows of one slice (one row per warp, as above) and streams 32-key K and V
// tiles through shared memory, so each key and value row is read from memory
// once per 16 query rows instead of once per row. K rows are padded by four
// elements so that lane j's 16-byte loads of key row j hit distinct banks; q
// rows sit in shared memory and are read as broadcasts.
constexpr int kTWarps = 16;             // warps per CTA
constexpr int kTRows = 2 * kTWarps;     // query rows per CTA: two per warp
constexpr int kTKeys = 32;              // keys per tile
constexpr int kTMaxDim = 256;

__host__ __device__ constexpr int tiled_pitch(int e) { return ((e + 3) & ~3) + 4; }

template <typename Acc>
__host__ __device__ constexpr size_t tiled_smem(int e, int ev) {
  return static_cast<size_t>(kTKeys * tiled_pitch(e) + kTKeys * ev + kTRows * tiled_pitch(e)) * sizeof(Acc);
}

// Online-softmax step of one row over one tile: returns this lane's p.
template <typename Acc, int NC>
__device__ __forceinline__ Acc row_step(Acc s, Acc& m, Acc& l, Acc (&acc)[NC]) {
  const Acc neg_inf = -static_cast<Acc>(INFINITY);
  const Acc m_new = fmax(m, warp_max(s));
  if (m_new == neg_inf) return Acc(0);  // every key so far masked: nothing accumulates
  const Acc alpha = (m == neg_inf) ? Acc(0) : exp_acc(m - m_new);
  const Acc p = (s == neg_inf) ? Acc(0) : exp_acc(s - m_new);
  l = l * alpha + warp_sum(p);
#pragma unroll
  for (int c = 0; c < NC; ++c) acc[c] *= alpha;
  m = m_new;
  return p;
}

template <typename T, typename Acc, int MASK, typename MaskT, int NC>
__global__ void __launch_bounds__(kTWarps * 32, 2) sdpa_exact_tiled_kernel(ExactArgs a) {
  extern __shared__ __align__(16) uint8_t smem_t[];
  const int E = static_cast<int>(a.E), Ev = static_cast<int>(a.Ev);
  const int KP = tiled_pitch(E);
  Acc* sK = reinterpret_cast<Acc*>(smem_t);   // [kTKeys][KP]
  Acc* sV = sK + kTKeys * KP;                  // [kTKeys][Ev]
  Acc* sQ = sV + kTKeys * Ev;                  // [kTRows][KP]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t groups = (a.L + kTRows - 1) / kTRows;
  const int64_t slice = blockIdx.x / groups;
  const int64_t i0 = (blockIdx.x % groups) * kTRows;
  const int64_t ia = i0 + 2 * warp, ib = ia + 1;  // this warp's two query rows
  const SliceOffsets off = slice_offsets(a.lt, slice);
  const T* qb = static_cast<const T*>(a.q) + off.q;
  const T* kb = static_cast<const T*>(a.k) + off.k;
  const T* vb = static_cast<const T*>(a.v) + off.v;
  const Acc scale = static_cast<Acc>(a.scale);
  const Acc neg_inf = -static_cast<Acc>(INFINITY);

#pragma unroll
  for (int h = 0; h < 2; ++h) {  // warp w stages query rows 2w, 2w + 1 (zero-padded to KP)
    const int64_t r = ia + h;
    const T* src = qb + r * a.q_rs;
    for (int e = lane; e < KP; e += 32)
      sQ[(2 * warp + h) * KP + e] = (e < E && r < a.L) ? load_as<Acc>(src + e) : Acc(0);
  }
  auto row_end = [&](int64_t r) -> int64_t {
    if (r >= a.L) return 0;
    return a.causal ? (r + 1 < a.S ? r + 1 : a.S) : a.S;
  };
  const int64_t end_a = row_end(ia), end_b = row_end(ib);
  const int64_t end_w = end_a > end_b ? end_a : end_b;
  const int64_t last_row = (i0 + kTRows < a.L ? i0 + kTRows : a.L) - 1;
  const int64_t cta_end = a.causal ? (last_row + 1 < a.S ? last_row + 1 : a.S) : a.S;

  Acc acc_a[NC], acc_b[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) acc_a[c] = acc_b[c] = 0;
  Acc m_a = neg_inf, l_a = 0, m_b = neg_inf, l_b = 0;
  const Acc* qa = sQ + (2 * warp) * KP;
  const Acc* qbr = qa + KP;

  auto masked = [&](Acc s, int64_t r, int64_t j) -> Acc {
    if (MASK == PA_MASK_BOOL) {
      if (!static_cast<const uint8_t*>(a.mask)[off.m + r * a.m_rs + j * a.m_cs]) return neg_inf;
    } else if (MASK == PA_MASK_ADD) {
      s += load_as<Acc>(static_cast<const MaskT*>(a.mask) + off.m + r * a.m_rs + j * a.m_cs);
    }
    return s;
  };

  for (int64_t j0 = 0; j0 < cta_end; j0 += kTKeys) {
    __syncthreads();  // the previous tile is consumed (and, first time, sQ is written)
    // warp w stages key/value rows 2w and 2w + 1 of the tile (lanes over columns)
#pragma unroll
    for (int h = 0; h < kTKeys / kTWarps; ++h) {
      const int t = warp * (kTKeys / kTWarps) + h;
      const int64_t key = j0 + t;
      const bool in = key < a.S;
      const T* kr = kb + (in ? key : 0) * a.k_rs;
      const T* vr = vb + (in ? key : 0) * a.v_rs;
      for (int e = lane; e < KP; e += 32) sK[t * KP + e] = (in && e < E) ? load_as<Acc>(kr + e) : Acc(0);
      for (int e = lane; e < Ev; e += 32) sV[t * Ev + e] = in ? load_as<Acc>(vr + e) : Acc(0);
    }
    __syncthreads();
    if (j0 >= end_w) continue;  // warp-uniform: both rows are past their last key
    const int64_t j = j0 + lane;
    Acc sa = neg_inf, sb = neg_inf;
    if (j < end_w) {
      const Acc* kr = sK + lane * KP;
      Acc a0 = 0, a1 = 0, b0 = 0, b1 = 0;
      for (int e = 0; e < E; e += 4) {  // E is padded with zeros to a multiple of 4
        if (sizeof(Acc) == 4) {         // 16-byte loads: lane j's key row hits its own banks
          const float4 kv = *reinterpret_cast<const float4*>(kr + e);
          const float4 xa = *reinterpret_cast<const float4*>(qa + e);
          const float4 xb = *reinterpret_cast<const float4*>(qbr + e);
          a0 = fma(static_cast<Acc>(xa.x), static_cast<Acc>(kv.x), a0);
          a1 = fma(static_cast<Acc>(xa.y), static_cast<Acc>(kv.y), a1);
          a0 = fma(static_cast<Acc>(xa.z), static_cast<Acc>(kv.z), a0);
          a1 = fma(static_cast<Acc>(xa.w), static_cast<Acc>(kv.w), a1);
          b0 = fma(static_cast<Acc>(xb.x), static_cast<Acc>(kv.x), b0);
          b1 = fma(static_cast<Acc>(xb.y), static_cast<Acc>(kv.y), b1);
          b0 = fma(static_cast<Acc>(xb.z), static_cast<Acc>(kv.z), b0);
          b1 = fma(static_cast<Acc>(xb.w), static_cast<Acc>(kv.w), b1);
        } else {
#pragma unroll
          for (int u = 0; u < 4; u += 2) {
            a0 = fma(qa[e + u], kr[e + u], a0);
            a1 = fma(qa[e + u + 1], kr[e + u + 1], a1);
            b0 = fma(qbr[e + u], kr[e + u], b0);
            b1 = fma(qbr[e + u + 1], kr[e + u + 1], b1);
          }
        }
      }
      if (j < end_a) sa = masked((a0 + a1) * scale, ia, j);
      if (j < end_b) sb = masked((b0 + b1) * scale, ib, j);
    }
    const Acc pa = row_step<Acc, NC>(sa, m_a, l_a, acc_a);
    const Acc pb = row_step<Acc, NC>(sb, m_b, l_b, acc_b);
    const int nk = static_cast<int>(end_w - j0 < kTKeys ? end_w - j0 : kTKeys);
    for (int t = 0; t < nk; ++t) {
      const Acc pta = __shfl_sync(0xffffffffu, pa, t);
      const Acc ptb = __shfl_sync(0xffffffffu, pb, t);
      const Acc* vr = sV + t * Ev;
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int col = lane + 32 * c;
        if (col < Ev) {
          const Acc x = vr[col];
          acc_a[c] = fma(pta, x, acc_a[c]);
          acc_b[c] = fma(ptb, x, acc_b[c]);
        }
      }
    }
  }
  auto store_row = [&](int64_t r, const Acc (&acc)[NC], Acc m, Acc l) {
    if (r >= a.L) return;
    T* orow = static_cast<T*>(a.out) + (slice * a.L + r) * a.Ev;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int col = lane + 32 * c;
      if (col < Ev) orow[col] = from_acc<T>(l > 0 ? static_cast<double>(acc[c] / l) : 0.0);
    }
    if (a.lse && lane == 0) a.lse[slice * a.L + r] = l > 0 ? static_cast<float>(m + log_acc(l)) : -INFINITY;
  };
  store_row(ia, acc_a, m_a, l_a);
  store_row(ib, acc_b, m_b, l_b);
}

template <typename T, typename Acc, int MASK, typename MaskT, int NC>
pa_status launch_tiled_nc(const ExactArgs& a, cudaStream_t st) {
  auto kern = sdpa_exact_tiled_kernel<T, Acc, MASK, MaskT, NC>;
  static uint64_t attr_set = 0;
  PA_TRY(set_smem_attr_once(reinterpret_cast<const void*>(kern), static_cast<int>(tiled_smem<Acc>(kTMaxDim, kTMaxDim)),
                            &attr_set));
  const int64_t blocks = a.nslices * ((a.L + kTRows - 1) / kTRows);
  if (blocks > 0x7fffffffLL) return fail(PA_ERR_UNSUPPORTED, "problem too large for the exact kernel");
  const size_t smem = tiled_smem<Acc>(static_cast<int>(a.E), static_cast<int>(a.Ev));
  kern<<<static_cast<unsigned>(blocks), kTWarps * 32, smem, st>>>(a);
  PA_CUDA(cudaGetLastError());
  return PA_OK;
}

// NC value columns per lane: Ev <= 64, <= 128 or <= 256.
template <typename T, typename Acc, int MASK, typename MaskT>
pa_status launch_tiled(const ExactArgs& a, cudaStream_t st) {
  if (a.Ev <= 64) return launch_tiled_nc<T, Acc, MASK, MaskT, 2>(a, st);
  if (a.Ev <= 128) return launch_tiled_nc<T, Acc, MASK, MaskT, 4>(a, st);
  return launch_tiled_nc<T, Acc, MASK, MaskT, 8>(a, st);
}

template <typename T, typename Acc>
pa_status launch_typed(const ExactArgs& a, const pa_sdpa_desc& d, cudaStream_t st) {
  const int64_t blocks = a.nslices * ((a.L + kWarps - 1) / kWarps);
  if (blocks > 0x7fffffffLL) return fail(PA_ERR_UNSUPPORTED, "problem too large for the exact kernel");
  dim3 grid(static_cast<unsigned>(blocks)), block(kWarps * 32);
  if (a.E <= kTMaxDim && a.Ev <= kTMaxDim && a.L > 0) {
    if (d.mask_kind == PA_MASK_NONE || d.is_causal) return launch_tiled<T, Acc, PA_MASK_NONE, float>(a, st);
    if (d.mask_kind == PA_MASK_BOOL) return launch_tiled<T, Acc, PA_MASK_BOOL, uint8_t>(a, st);
    switch (d.mask_dtype) {
      case PA_F16: return launch_tiled<T, Acc, PA_MASK_ADD, __half>(a, st);
      case PA_BF16: return launch_tiled<T, Acc, PA_MASK_ADD, __nv_bfloat16>(a, st);
      case PA_F32: return launch_tiled<T, Acc, PA_MASK_ADD, float>(a, st);
      case PA_F64: return launch_tiled<T, Acc, PA_MASK_ADD, double>(a, st);
      default: return fail(PA_ERR_INVALID, "unsupported additive mask dtype");
    }
  }
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
