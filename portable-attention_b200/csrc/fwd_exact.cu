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
  int32_t lt_kv_aligned;  // every k/v slice offset is a multiple of 4 elements
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

// ---------------------------------------------------------------------------
// Register-tiled fp32 variant for E, Ev <= 128 (fp32, fp16 and bf16 operands;
// fp64 keeps the kernels above). A CTA of 256 threads owns 64 query rows of
// one slice and streams 64-key K/V tiles through shared memory (cp.async,
// double-buffered, when the operands are fp32 with 16-byte rows; converting
// loads otherwise). Thread (ty, tx) = (tid / 16, tid % 16) computes a 4 x 4
// block of scores (rows ty + 16a, keys tx + 16b: each warp reads two q rows
// as broadcasts and sixteen key rows without bank conflicts) and a 4 x NCO
// block of the output (rows ty + 16a, columns 4tx.. and 64 + 4tx..), so every
// value read from shared memory feeds four to eight FMAs. The softmax runs in
// log2 units (q pre-scaled by scale * log2 e, library exp2f); a row's running
// max is reduced over its 16 threads with shuffles, and its running sum stays
// split over them until the end (the rescale factor is common to the row).
// Same semantics as the kernels above: fully-masked rows exactly zero with
// lse -inf, top-left causal, broadcast boolean / additive masks.
constexpr int kRBM = 64;       // query rows per CTA
constexpr int kRBN = 64;       // keys per tile
constexpr int kRThreads = 256;
constexpr int kRMaxDim = 128;
constexpr float kLog2e = 1.4426950408889634f;

__host__ __device__ constexpr int rt_qpitch(int e) { return ((e + 3) & ~3) + 4; }
__host__ __device__ constexpr int rt_vpitch(int ev) { return ev <= 64 ? 64 : 128; }
constexpr int kRPPitch = kRBM + 4;

__host__ __device__ constexpr size_t rt_smem(int e, int ev) {
  // sQ + 2 x (sK + sV) + sP, in floats
  return static_cast<size_t>(kRBM * rt_qpitch(e) + 2 * (kRBN * rt_qpitch(e) + kRBN * rt_vpitch(ev)) +
                             kRBN * kRPPitch) * sizeof(float);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const uint32_t d = smem_u32(dst);
  const uint32_t n = valid ? 16u : 0u;  // 0: fill the 16 bytes with zeros, read nothing
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <typename T, int MASK, typename MaskT, int NCO, bool ASYNC, int EPT>
__global__ void __launch_bounds__(kRThreads, 2) sdpa_exact_rt_kernel(ExactArgs a) {
  extern __shared__ __align__(16) uint8_t smem_r[];
  // EPT != 0: the head dimension is EPT (a multiple of 4), known at compile time
  // so the score loop unrolls completely.
  const int E = EPT ? EPT : static_cast<int>(a.E), Ev = static_cast<int>(a.Ev);
  const int QP = EPT ? EPT + 4 : rt_qpitch(E), EP = QP - 4;
  constexpr int VP = NCO == 4 ? 64 : 128;
  float* sQ = reinterpret_cast<float*>(smem_r);        // [kRBM][QP]
  float* sK0 = sQ + kRBM * QP;                          // [2][kRBN][QP]
  float* sV0 = sK0 + 2 * kRBN * QP;                     // [2][kRBN][VP]
  float* sP = sV0 + 2 * kRBN * VP;                      // [kRBN][kRPPitch], P^T with rows permuted
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t groups = (a.L + kRBM - 1) / kRBM;
  const int64_t slice = blockIdx.x / groups;
  const int64_t i0 = (blockIdx.x % groups) * kRBM;
  const SliceOffsets off = slice_offsets(a.lt, slice);
  const T* qb = static_cast<const T*>(a.q) + off.q;
  const T* kb = static_cast<const T*>(a.k) + off.k;
  const T* vb = static_cast<const T*>(a.v) + off.v;
  const float qscale = static_cast<float>(a.scale) * kLog2e;
  const float neg_inf = -INFINITY;
  const int64_t last_row = (i0 + kRBM < a.L ? i0 + kRBM : a.L) - 1;
  const int64_t cta_end = a.causal ? (last_row + 1 < a.S ? last_row + 1 : a.S) : a.S;
  const int ntiles = static_cast<int>((cta_end + kRBN - 1) / kRBN);

  // Q rows, pre-scaled, zero-padded; V padding columns zeroed once (never stored,
  // but they must be finite).
  for (int idx = tid; idx < kRBM * QP; idx += kRThreads) {
    const int r = idx / QP, e = idx % QP;
    const int64_t row = i0 + r;
    sQ[idx] = (e < E && row < a.L) ? load_as<float>(qb + row * a.q_rs + e) * qscale : 0.f;
  }
  if (Ev < VP)
    for (int idx = tid; idx < 2 * kRBN * VP; idx += kRThreads)
      if (idx % VP >= Ev) sV0[idx] = 0.f;

  auto load_tile = [&](int t, int buf) {
    float* sK = sK0 + buf * kRBN * QP;
    float* sV = sV0 + buf * kRBN * VP;
    const int64_t j0 = static_cast<int64_t>(t) * kRBN;
    if (ASYNC) {
      const int kc = E / 4, vc = Ev / 4;  // 16-byte chunks per row (E, Ev multiples of 4 here)
      for (int idx = tid; idx < kRBN * kc; idx += kRThreads) {
        const int r = idx / kc, c = idx % kc;
        const int64_t key = j0 + r;
        const bool ok = key < a.S;
        cp_async16(sK + r * QP + 4 * c, kb + (ok ? key : 0) * a.k_rs + 4 * c, ok);
      }
      for (int idx = tid; idx < kRBN * vc; idx += kRThreads) {
        const int r = idx / vc, c = idx % vc;
        const int64_t key = j0 + r;
        const bool ok = key < a.S;
        cp_async16(sV + r * VP + 4 * c, vb + (ok ? key : 0) * a.v_rs + 4 * c, ok);
      }
    } else {
      for (int idx = tid; idx < kRBN * EP; idx += kRThreads) {
        const int r = idx / EP, e = idx % EP;
        const int64_t key = j0 + r;
        sK[r * QP + e] = (key < a.S && e < E) ? load_as<float>(kb + key * a.k_rs + e) : 0.f;
      }
      for (int idx = tid; idx < kRBN * Ev; idx += kRThreads) {
        const int r = idx / Ev, c = idx % Ev;
        const int64_t key = j0 + r;
        sV[r * VP + c] = key < a.S ? load_as<float>(vb + key * a.v_rs + c) : 0.f;
      }
    }
  };

  // Output accumulators as packed pairs of adjacent columns (f32x2 FMAs).
  uint64_t o2[4][NCO / 2];
  float m[4], l[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    m[r] = neg_inf;
    l[r] = 0.f;
#pragma unroll
    for (int c = 0; c < NCO / 2; ++c) o2[r][c] = 0ull;
  }

  if (ASYNC && ntiles > 0) {
    load_tile(0, 0);
    cp_async_commit();
  }
  for (int t = 0; t < ntiles; ++t) {
    const int buf = t & 1;
    __syncthreads();  // the previous tile's P and V reads are done (and sQ is written)
    if (ASYNC) {
      if (t + 1 < ntiles) load_tile(t + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();  // this thread's copies of tile t have landed
    } else {
      load_tile(t, buf);
    }
    __syncthreads();
    const float* sK = sK0 + buf * kRBN * QP;
    const float* sV = sV0 + buf * kRBN * VP;
    const int64_t j0 = static_cast<int64_t>(t) * kRBN;

    // Scores: each (row, key) keeps two partial sums (even / odd head-dim
    // terms) in one packed pair, so a 16-byte q and k load feed two f32x2 FMAs.
    uint64_t s2[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int b = 0; b < 4; ++b) s2[r][b] = 0ull;
#pragma unroll
    for (int e = 0; e < EP; e += 4) {
      float4 qv[4], kv[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) qv[r] = *reinterpret_cast<const float4*>(sQ + (ty + 16 * r) * QP + e);
#pragma unroll
      for (int b = 0; b < 4; ++b) kv[b] = *reinterpret_cast<const float4*>(sK + (tx + 16 * b) * QP + e);
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          s2[r][b] = fma2(f2(qv[r].x, qv[r].y), f2(kv[b].x, kv[b].y), s2[r][b]);
          s2[r][b] = fma2(f2(qv[r].z, qv[r].w), f2(kv[b].z, kv[b].w), s2[r][b]);
        }
    }
    float s[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int b = 0; b < 4; ++b) s[r][b] = f2_lo(s2[r][b]) + f2_hi(s2[r][b]);

    // Mask, online softmax (log2 units), P^T into shared memory.
    float alpha[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int64_t row = i0 + ty + 16 * r;
      const int64_t vis = a.causal ? (row + 1 < a.S ? row + 1 : a.S) : a.S;
      float mt = neg_inf;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int64_t key = j0 + tx + 16 * b;
        float x = (key < vis && row < a.L) ? s[r][b] : neg_inf;
        if (MASK != PA_MASK_NONE && x != neg_inf) {
          const int64_t mo = off.m + row * a.m_rs + key * a.m_cs;
          if (MASK == PA_MASK_BOOL) {
            if (!static_cast<const uint8_t*>(a.mask)[mo]) x = neg_inf;
          } else {
            x = fmaf(load_as<float>(static_cast<const MaskT*>(a.mask) + mo), kLog2e, x);
          }
        }
        s[r][b] = x;
        mt = fmaxf(mt, x);
      }
#pragma unroll
      for (int sh = 8; sh; sh >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, sh));
      const float m_new = fmaxf(m[r], mt);
      if (m_new == neg_inf) {  // every key so far masked: nothing accumulates
        alpha[r] = 1.f;
#pragma unroll
        for (int b = 0; b < 4; ++b) s[r][b] = 0.f;
      } else {
        alpha[r] = exp2f(m[r] - m_new);  // 0 when m[r] is -inf
        float ps = 0.f;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          s[r][b] = exp2f(s[r][b] - m_new);
          ps += s[r][b];
        }
        l[r] = l[r] * alpha[r] + ps;
        m[r] = m_new;
      }
    }
#pragma unroll
    for (int b = 0; b < 4; ++b)
      *reinterpret_cast<float4*>(sP + (tx + 16 * b) * kRPPitch + 4 * ty) =
          make_float4(s[0][b], s[1][b], s[2][b], s[3][b]);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint64_t al2 = f2(alpha[r], alpha[r]);
#pragma unroll
      for (int c = 0; c < NCO / 2; ++c) o2[r][c] = mul2(o2[r][c], al2);
    }
    __syncthreads();

    const int nk = static_cast<int>(cta_end - j0 < kRBN ? cta_end - j0 : kRBN);
#pragma unroll 4
    for (int k = 0; k < nk; ++k) {
      const float4 pv = *reinterpret_cast<const float4*>(sP + k * kRPPitch + 4 * ty);
      const uint64_t pd[4] = {f2(pv.x, pv.x), f2(pv.y, pv.y), f2(pv.z, pv.z), f2(pv.w, pv.w)};
#pragma unroll
      for (int g = 0; g < NCO / 4; ++g) {
        const float4 vv = *reinterpret_cast<const float4*>(sV + k * VP + 64 * g + 4 * tx);
        const uint64_t v01 = f2(vv.x, vv.y), v23 = f2(vv.z, vv.w);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          o2[r][2 * g] = fma2(pd[r], v01, o2[r][2 * g]);
          o2[r][2 * g + 1] = fma2(pd[r], v23, o2[r][2 * g + 1]);
        }
      }
    }
  }

  // Row sums over the row's 16 threads, then normalise and store.
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    float lr = l[r];
#pragma unroll
    for (int sh = 8; sh; sh >>= 1) lr += __shfl_xor_sync(0xffffffffu, lr, sh);
    const int64_t row = i0 + ty + 16 * r;
    if (row >= a.L) continue;
    const float inv = lr > 0.f ? 1.f / lr : 0.f;
    T* orow = static_cast<T*>(a.out) + (slice * a.L + row) * a.Ev;
#pragma unroll
    for (int g = 0; g < NCO / 4; ++g)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int col = 64 * g + 4 * tx + c;
        const uint64_t pr = o2[r][2 * g + c / 2];
        const float ov = (c & 1) ? f2_hi(pr) : f2_lo(pr);
        if (col < Ev) orow[col] = from_acc<T>(static_cast<double>(lr > 0.f ? ov * inv : 0.f));
      }
    if (a.lse && tx == 0)
      a.lse[slice * a.L + row] = lr > 0.f ? (m[r] + log2f(lr)) * 0.6931471805599453f : -INFINITY;
  }
}

template <typename T, int MASK, typename MaskT, int NCO, bool ASYNC, int EPT = 0>
pa_status launch_rt_v(const ExactArgs& a, cudaStream_t st) {
  auto kern = sdpa_exact_rt_kernel<T, MASK, MaskT, NCO, ASYNC, EPT>;
  static uint64_t attr_set = 0;
  PA_TRY(set_smem_attr_once(reinterpret_cast<const void*>(kern),
                            static_cast<int>(rt_smem(kRMaxDim, NCO == 4 ? 64 : 128)), &attr_set));
  const int64_t blocks = a.nslices * ((a.L + kRBM - 1) / kRBM);
  if (blocks > 0x7fffffffLL) return fail(PA_ERR_UNSUPPORTED, "problem too large for the exact kernel");
  const size_t smem = rt_smem(static_cast<int>(a.E), NCO == 4 ? 64 : 128);
  kern<<<static_cast<unsigned>(blocks), kRThreads, smem, st>>>(a);
  PA_CUDA(cudaGetLastError());
  return PA_OK;
}

template <typename T, int MASK, typename MaskT>
pa_status launch_rt(const ExactArgs& a, cudaStream_t st) {
  // cp.async needs fp32 rows of whole 16-byte chunks at 16-byte aligned addresses.
  const bool async = sizeof(T) == 4 && a.E % 4 == 0 && a.Ev % 4 == 0 && a.k_rs % 4 == 0 &&
                     a.v_rs % 4 == 0 && (reinterpret_cast<uintptr_t>(a.k) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(a.v) & 15) == 0 && a.lt_kv_aligned;
  if (MASK == PA_MASK_NONE && async && a.Ev <= 64 && a.E == 64) return launch_rt_v<T, MASK, MaskT, 4, true, 64>(a, st);
  if (MASK == PA_MASK_NONE && async && a.Ev > 64 && a.E == 128) return launch_rt_v<T, MASK, MaskT, 8, true, 128>(a, st);
  if (a.Ev <= 64)
    return async ? launch_rt_v<T, MASK, MaskT, 4, true>(a, st) : launch_rt_v<T, MASK, MaskT, 4, false>(a, st);
  return async ? launch_rt_v<T, MASK, MaskT, 8, true>(a, st) : launch_rt_v<T, MASK, MaskT, 8, false>(a, st);
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
  if (sizeof(Acc) == 4 && a.E <= kRMaxDim && a.Ev <= kRMaxDim && a.L > 0) {
    if (d.mask_kind == PA_MASK_NONE || d.is_causal) return launch_rt<T, PA_MASK_NONE, float>(a, st);
    if (d.mask_kind == PA_MASK_BOOL) return launch_rt<T, PA_MASK_BOOL, uint8_t>(a, st);
    switch (d.mask_dtype) {
      case PA_F16: return launch_rt<T, PA_MASK_ADD, __half>(a, st);
      case PA_BF16: return launch_rt<T, PA_MASK_ADD, __nv_bfloat16>(a, st);
      case PA_F32: return launch_rt<T, PA_MASK_ADD, float>(a, st);
      case PA_F64: return launch_rt<T, PA_MASK_ADD, double>(a, st);
      default: return fail(PA_ERR_INVALID, "unsupported additive mask dtype");
    }
  }
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
  a.lt_kv_aligned = 1;
  for (int i = 0; i < d.nlead; ++i)
    if (d.k_lead_stride[i] % 4 || d.v_lead_stride[i] % 4) a.lt_kv_aligned = 0;
  switch (d.dtype) {
    case PA_F64: return launch_typed<double, double>(a, d, st);
    case PA_F32: return launch_typed<float, float>(a, d, st);
    case PA_F16: return launch_typed<__half, float>(a, d, st);
    case PA_BF16: return launch_typed<__nv_bfloat16, float>(a, d, st);
    default: return fail(PA_ERR_INVALID, "unsupported dtype for the exact kernel");
  }
}

}  // namespace pa
