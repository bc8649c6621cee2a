// Split-KV decode forward (query length 1), HBM-bound, on CUDA cores.
//
// Work unit: (batch b, key/value head kh, split s) -> one CTA that reads keys
// [s*chunk, min(S, (s+1)*chunk)) of K[b, kh] and V[b, kh] exactly once and
// serves all G = Hq / Hkv query heads that share that key/value head, so
// grouped-query K/V is never repeated.
//
// CTA = 1 producer warp + 8 compute warps.
//   producer  TMA-loads 32-key K and V tiles (128-byte swizzle, 64-column
//             boxes) into a ring of shared-memory stages; keeps ~190 KB in
//             flight per SM so HBM stays busy.
//   compute   warp w consumes tiles w, w+8, w+16, ... on its own:
//               scores   lane j <-> key j of the tile; q (fp32, G heads) is
//                        read from shared memory as broadcasts, the key row
//                        with conflict-free 16-byte loads (swizzled);
//               softmax  per-head running max / sum in log2 units;
//               P V      lane l <-> value columns [l*D/32, (l+1)*D/32), the
//                        probabilities of the 32 keys broadcast by shuffles.
//             The 8 warps' partial states merge in shared memory at the end
//             and the CTA writes one partial (m, l, acc[D]) per query head
//             into the workspace.
// combine     one CTA per (b, query head) merges the splits by log-sum-exp
//             and writes the fp16/bf16 output and, optionally, the lse.
//
// The math is reference.py:139-162 for L == 1 (no mask, not causal).
#include <math.h>

#include <cmath>
#include <cstdio>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace pa {
namespace {

constexpr int kWarpsC = 8;                 // compute warps
constexpr int kThreadsDec = 32 * (kWarpsC + 1);
constexpr int kTileKeys = 32;
constexpr float kLn2f = 0.6931471805599453f;

template <int D>
struct DecCfg {
  static constexpr int kBoxes = D / 64;
  static constexpr int kTileBytes = kTileKeys * D * 2;        // one K (or V) tile
  static constexpr int kStageBytes = 2 * kTileBytes;          // K + V
  static constexpr int kStages = D == 128 ? 12 : 20;
  static constexpr int kRingBytes = kStages * kStageBytes;
  static constexpr int kQOff = kRingBytes;                    // G*D floats (G <= 8)
  static constexpr int kBarOff = kQOff + 8 * D * 4;
  static constexpr int kSmemBytes = kBarOff + 2 * kStages * 8 + 16 + 1024;
};

struct DecArgs {
  const void* q;
  float* ws_acc;   // [B*Hq][nsplit][D]
  float* ws_ml;    // [B*Hq][nsplit][2]  (m in log2 units, l)
  int* status;
  int64_t S;
  int32_t Hq, Hkv, nsplit, chunk;
  float scale_log2;
};

__device__ __forceinline__ float to_float(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }

template <bool BF16>
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (BF16) {
      __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
      float2 t = __bfloat1622float2(h);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    } else {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 t = __half22float2(h);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
}

template <int D, int G, bool BF16>
__global__ void __launch_bounds__(kThreadsDec, 1)
    decode_partial_kernel(const __grid_constant__ CUtensorMap tk,
                          const __grid_constant__ CUtensorMap tv, const DecArgs a) {
  using C = DecCfg<D>;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  constexpr int DL = D / 32;  // value columns per lane
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  float* sq = reinterpret_cast<float*>(smem + C::kQOff);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* empty = full + C::kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kBarOff + 2 * C::kStages * 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x % a.nsplit;
  const int64_t pair = blockIdx.x / a.nsplit;  // b * Hkv + kh
  const int64_t b = pair / a.Hkv;
  const int kh = static_cast<int>(pair % a.Hkv);
  const int64_t k0 = static_cast<int64_t>(split) * a.chunk;
  const int64_t k1 = (k0 + a.chunk < a.S) ? k0 + a.chunk : a.S;
  const int ntiles = k1 > k0 ? static_cast<int>((k1 - k0 + kTileKeys - 1) / kTileKeys) : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  // q for the G heads of this group, fp32 in shared memory.
  const T* qg = static_cast<const T*>(a.q) + (b * a.Hq + static_cast<int64_t>(kh) * G) * D;
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) sq[i] = to_float(qg[i]);
  __syncthreads();

  if (warp == kWarpsC) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int last[C::kStages];
#pragma unroll
      for (int s = 0; s < C::kStages; ++s) last[s] = -1;
      for (int t = 0; t < ntiles; ++t) {
        const int st = t % C::kStages;
        if (!mbar_wait(empty + st, ((t / C::kStages) & 1) ^ 1, a.status, kStatusTimeoutFree, abort_flag)) break;
        mbar_expect_tx(full + st, C::kStageBytes);
        uint8_t* base = smem + st * C::kStageBytes;
        const int32_t row = static_cast<int32_t>(k0 + static_cast<int64_t>(t) * kTileKeys);
        for (int bx = 0; bx < C::kBoxes; ++bx) {
          tma_load_3d(base + bx * (kTileKeys * 128), &tk, full + st, bx * 64, row, static_cast<int32_t>(pair));
          tma_load_3d(base + C::kTileBytes + bx * (kTileKeys * 128), &tv, full + st, bx * 64, row,
                      static_cast<int32_t>(pair));
        }
        last[st] = t;
      }
#pragma unroll
      for (int s = 0; s < C::kStages; ++s)
        if (last[s] >= 0) mbar_drain(full + s, (last[s] / C::kStages) & 1);
    }
    __syncwarp();
    __syncthreads();
    return;
  }

  // -------------------------------------------------------------- compute
  float m_run[G], l_run[G], acc[G][DL];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m_run[h] = -INFINITY;
    l_run[h] = 0.f;
#pragma unroll
    for (int c = 0; c < DL; ++c) acc[h][c] = 0.f;
  }
  for (int t = warp; t < ntiles; t += kWarpsC) {
    const int st = t % C::kStages;
    bool ok = mbar_wait(full + st, (t / C::kStages) & 1, a.status, kStatusTimeoutLoad, abort_flag);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) break;
    const uint8_t* kt = smem + st * C::kStageBytes;
    const uint8_t* vt = kt + C::kTileBytes;
    // scores: lane <-> key
    float s[G];
#pragma unroll
    for (int h = 0; h < G; ++h) s[h] = 0.f;
#pragma unroll
    for (int c = 0; c < D / 8; ++c) {
      const int bx = c / 8, ch = c % 8;
      const uint4 u = *reinterpret_cast<const uint4*>(kt + bx * (kTileKeys * 128) + lane * 128 +
                                                      ((ch ^ (lane & 7)) * 16));
      float kf[8];
      unpack8<BF16>(u, kf);
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float4 q0 = *reinterpret_cast<const float4*>(sq + h * D + c * 8);
        const float4 q1 = *reinterpret_cast<const float4*>(sq + h * D + c * 8 + 4);
        s[h] = fmaf(q0.x, kf[0], s[h]);
        s[h] = fmaf(q0.y, kf[1], s[h]);
        s[h] = fmaf(q0.z, kf[2], s[h]);
        s[h] = fmaf(q0.w, kf[3], s[h]);
        s[h] = fmaf(q1.x, kf[4], s[h]);
        s[h] = fmaf(q1.y, kf[5], s[h]);
        s[h] = fmaf(q1.z, kf[6], s[h]);
        s[h] = fmaf(q1.w, kf[7], s[h]);
      }
    }
    const int64_t key = k0 + static_cast<int64_t>(t) * kTileKeys + lane;
    float p[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float x = key < k1 ? s[h] * a.scale_log2 : -INFINITY;
      float mx = x;
#pragma unroll
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_new = fmaxf(m_run[h], mx);  // finite: the tile has >= 1 valid key
      const float alpha = ex2(m_run[h] - m_new);
      p[h] = ex2(x - m_new);
      l_run[h] = l_run[h] * alpha + p[h];  // lane-local partial sum
      m_run[h] = m_new;
#pragma unroll
      for (int c = 0; c < DL; ++c) acc[h][c] *= alpha;
    }
    // P V: lane <-> value columns
#pragma unroll 4
    for (int j = 0; j < kTileKeys; ++j) {
      float vf[DL];
      {
        // columns [lane*DL, lane*DL + DL) of row j; 64-column boxes, swizzled 16-byte chunks
        const int col = lane * DL;
        const int bx = col / 64, cb = (col % 64) * 2;  // byte offset inside the 128-byte row
        const uint8_t* rowp = vt + bx * (kTileKeys * 128) + j * 128;
        const int chunk = (cb >> 4) ^ (j & 7);
        const uint8_t* src = rowp + chunk * 16 + (cb & 15);
        if (DL == 4) {
          const uint2 u = *reinterpret_cast<const uint2*>(src);
          float2 a0, a1;
          if (BF16) {
            a0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
            a1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
          } else {
            a0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
            a1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
          }
          vf[0] = a0.x;
          vf[1] = a0.y;
          vf[DL > 2 ? 2 : 0] = a1.x;
          vf[DL > 3 ? 3 : 1] = a1.y;
        } else {
          const uint32_t u = *reinterpret_cast<const uint32_t*>(src);
          float2 a0 = BF16 ? __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u))
                           : __half22float2(*reinterpret_cast<const __half2*>(&u));
          vf[0] = a0.x;
          vf[DL > 1 ? 1 : 0] = a0.y;
        }
      }
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float pj = __shfl_sync(0xffffffffu, p[h], j);
#pragma unroll
        for (int c = 0; c < DL; ++c) acc[h][c] = fmaf(pj, vf[c], acc[h][c]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + st);
  }

  // Lane-local sums -> warp sums.
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int o = 16; o; o >>= 1) l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], o);

  __syncthreads();  // every tile consumed and landed: the ring is free for the merge
  float* mw = reinterpret_cast<float*>(smem);                 // [8][G] m
  float* lw = mw + kWarpsC * G;                              // [8][G] l
  float* aw = lw + kWarpsC * G;                              // [8][G][D] acc
  if (lane == 0)
#pragma unroll
    for (int h = 0; h < G; ++h) {
      mw[warp * G + h] = m_run[h];
      lw[warp * G + h] = l_run[h];
    }
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int c = 0; c < DL; ++c) aw[(warp * G + h) * D + lane * DL + c] = acc[h][c];
  asm volatile("bar.sync 1, %0;" ::"n"(kWarpsC * 32));
  for (int i = threadIdx.x; i < G * D; i += kWarpsC * 32) {
    const int h = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarpsC; ++w) M = fmaxf(M, mw[w * G + h]);
    float o = 0.f, l = 0.f;
#pragma unroll
    for (int w = 0; w < kWarpsC; ++w) {
      const float mwv = mw[w * G + h];
      const float f = mwv == -INFINITY ? 0.f : ex2(mwv - M);
      o = fmaf(f, aw[(w * G + h) * D + d], o);
      l = fmaf(f, lw[w * G + h], l);
    }
    const int64_t qh = b * a.Hq + static_cast<int64_t>(kh) * G + h;
    const int64_t slot = qh * a.nsplit + split;
    a.ws_acc[slot * D + d] = o;
    if (d == 0) {
      a.ws_ml[slot * 2] = M;
      a.ws_ml[slot * 2 + 1] = l;
    }
  }
}

template <int D, bool BF16>
__global__ void __launch_bounds__(D) decode_combine_kernel(const float* ws_acc, const float* ws_ml,
                                                           void* out, float* lse, int nsplit) {
  const int64_t qh = blockIdx.x;
  const int d = threadIdx.x;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, ws_ml[(qh * nsplit + s) * 2]);
  float o = 0.f, l = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float ms = ws_ml[(qh * nsplit + s) * 2];
    const float f = ms == -INFINITY ? 0.f : ex2(ms - M);
    o = fmaf(f, ws_acc[(qh * nsplit + s) * D + d], o);
    l = fmaf(f, ws_ml[(qh * nsplit + s) * 2 + 1], l);
  }
  const float r = l > 0.f ? o / l : 0.f;
  if (BF16)
    static_cast<__nv_bfloat16*>(out)[qh * D + d] = __float2bfloat16_rn(r);
  else
    static_cast<__half*>(out)[qh * D + d] = __float2half_rn(r);
  if (lse && d == 0) lse[qh] = l > 0.f ? (M + __log2f(l)) * kLn2f : -INFINITY;
}

struct DecPlan {
  int64_t B, Hq, Hkv, S;
  int D, G, nsplit, chunk;
  bool bf16;
};

pa_status make_plan(const pa_sdpa_desc& d, DecPlan* p) {
  if (d.L != 1) return fail(PA_ERR_UNSUPPORTED, "decode: query length must be 1");
  if (d.dtype != PA_F16 && d.dtype != PA_BF16) return fail(PA_ERR_UNSUPPORTED, "decode: dtype must be fp16/bf16");
  if (d.E != d.Ev || (d.E != 64 && d.E != 128)) return fail(PA_ERR_UNSUPPORTED, "decode: head dim must be 64 or 128");
  if (d.mask_kind != PA_MASK_NONE || d.is_causal) return fail(PA_ERR_UNSUPPORTED, "decode: no mask / causal");
  if (d.S < 1) return fail(PA_ERR_UNSUPPORTED, "decode: needs at least one key");
  int64_t n, H, Hkv;
  if (!dense_bhsd(d, &n, &H, &Hkv)) return fail(PA_ERR_UNSUPPORTED, "decode: operands not dense (B, H, S, D)");
  const int64_t G = H / Hkv;
  if (G != 1 && G != 2 && G != 4 && G != 8) return fail(PA_ERR_UNSUPPORTED, "decode: group size must be 1, 2, 4 or 8");
  if (d.S > 0x7fffffffLL) return fail(PA_ERR_UNSUPPORTED, "decode: too many keys");
  p->B = n / H;
  p->Hq = H;
  p->Hkv = Hkv;
  p->S = d.S;
  p->D = static_cast<int>(d.E);
  p->G = static_cast<int>(G);
  p->bf16 = d.dtype == PA_BF16;
  // Split the keys so that the CTA count fills whole waves (1 CTA per SM).
  const int64_t pairs = p->B * Hkv;
  const int64_t sms = sm_count();
  const int64_t tiles = (d.S + kTileKeys - 1) / kTileKeys;
  int best = 1;
  double best_eff = 0;
  for (int ns = 1; ns <= 64 && ns <= tiles; ++ns) {
    const int64_t ctas = pairs * ns;
    const double waves = static_cast<double>(ctas) / sms;
    const double eff = waves / std::ceil(waves);
    // Prefer fewer splits unless a larger count fills waves clearly better;
    // also keep at least 8 tiles per CTA so the ring pipelines.
    if (tiles / ns < 8 && ns > 1) break;
    if (eff > best_eff + 0.02) {
      best_eff = eff;
      best = ns;
    }
  }
  p->nsplit = best;
  const int64_t per = (tiles + best - 1) / best;
  p->chunk = static_cast<int>(per * kTileKeys);
  p->nsplit = static_cast<int>((d.S + p->chunk - 1) / p->chunk);
  return PA_OK;
}

size_t plan_ws_bytes(const DecPlan& p) {
  const size_t slots = static_cast<size_t>(p.B * p.Hq) * p.nsplit;
  return slots * (p.D + 2) * sizeof(float);
}

template <int D, int G, bool BF16>
pa_status launch_dec(const DecPlan& p, const CUtensorMap& tk, const CUtensorMap& tv, DecArgs& a,
                     void* out, float* lse, cudaStream_t st) {
  auto kern = decode_partial_kernel<D, G, BF16>;
  constexpr int smem = DecCfg<D>::kSmemBytes;
  static uint64_t attr_set = 0;
  PA_TRY(set_smem_attr_once(reinterpret_cast<const void*>(kern), smem, &attr_set));
  const int64_t grid = p.B * p.Hkv * p.nsplit;
  kern<<<static_cast<unsigned>(grid), kThreadsDec, smem, st>>>(tk, tv, a);
  PA_CUDA(cudaGetLastError());
  decode_combine_kernel<D, BF16><<<static_cast<unsigned>(p.B * p.Hq), D, 0, st>>>(
      a.ws_acc, a.ws_ml, out, lse, p.nsplit);
  PA_CUDA(cudaGetLastError());
  return PA_OK;
}

template <int D, bool BF16>
pa_status launch_dec_g(const DecPlan& p, const CUtensorMap& tk, const CUtensorMap& tv, DecArgs& a,
                       void* out, float* lse, cudaStream_t st) {
  switch (p.G) {
    case 1: return launch_dec<D, 1, BF16>(p, tk, tv, a, out, lse, st);
    case 2: return launch_dec<D, 2, BF16>(p, tk, tv, a, out, lse, st);
    case 4: return launch_dec<D, 4, BF16>(p, tk, tv, a, out, lse, st);
    default: return launch_dec<D, 8, BF16>(p, tk, tv, a, out, lse, st);
  }
}

}  // namespace

// Runs the decode with the given workspace (at least decode_ws_bytes bytes);
// bounded waits that give up record their code in `status`.
pa_status run_decode_status(const pa_sdpa_desc& d, const void* q, const void* k, const void* v,
                            void* out, float* lse, void* ws, size_t ws_bytes, int* status,
                            cudaStream_t st) {
  DecPlan p;
  PA_TRY(make_plan(d, &p));
  if (ws_bytes < plan_ws_bytes(p)) return fail(PA_ERR_INVALID, "decode: workspace too small");
  const bool bf16 = p.bf16;
  const CUtensorMapDataType tdt = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tk, tv;
  const uint64_t rowb = static_cast<uint64_t>(p.D) * 2;
  const uint64_t planes = static_cast<uint64_t>(p.B * p.Hkv);
  PA_TRY(encode_tma_3d(&tk, tdt, k, p.D, p.S, planes, rowb, rowb * p.S, 64, kTileKeys, CU_TENSOR_MAP_SWIZZLE_128B));
  PA_TRY(encode_tma_3d(&tv, tdt, v, p.D, p.S, planes, rowb, rowb * p.S, 64, kTileKeys, CU_TENSOR_MAP_SWIZZLE_128B));
  DecArgs a{};
  a.q = q;
  const size_t slots = static_cast<size_t>(p.B * p.Hq) * p.nsplit;
  a.ws_acc = static_cast<float*>(ws);
  a.ws_ml = a.ws_acc + slots * p.D;
  a.status = status;
  a.S = p.S;
  a.Hq = static_cast<int32_t>(p.Hq);
  a.Hkv = static_cast<int32_t>(p.Hkv);
  a.nsplit = p.nsplit;
  a.chunk = p.chunk;
  a.scale_log2 = static_cast<float>(d.scale * 1.4426950408889634);
  if (p.B * p.Hkv * p.nsplit > 0x7fffffffLL) return fail(PA_ERR_UNSUPPORTED, "decode: grid too large");
  if (p.D == 128)
    return bf16 ? launch_dec_g<128, true>(p, tk, tv, a, out, lse, st)
                : launch_dec_g<128, false>(p, tk, tv, a, out, lse, st);
  return bf16 ? launch_dec_g<64, true>(p, tk, tv, a, out, lse, st)
              : launch_dec_g<64, false>(p, tk, tv, a, out, lse, st);
}

pa_status run_decode(const pa_sdpa_desc& d, const void* q, const void* k, const void* v, void* out,
                     float* lse, void* ws, size_t ws_bytes, cudaStream_t st) {
  int* status = device_status_word();
  if (!status) return fail(PA_ERR_CUDA, "device status word unavailable");
  return run_decode_status(d, q, k, v, out, lse, ws, ws_bytes, status, st);
}

pa_status decode_ws_bytes(const pa_sdpa_desc& d, size_t* bytes) {
  DecPlan p;
  PA_TRY(make_plan(d, &p));
  *bytes = plan_ws_bytes(p);
  return PA_OK;
}

}  // namespace pa

using namespace pa;

extern "C" pa_status pa_decode_workspace_size(const pa_sdpa_desc* desc, size_t* bytes) {
  clear_error();
  if (!desc || !bytes) return fail(PA_ERR_INVALID, "null argument");
  return decode_ws_bytes(*desc, bytes);
}

extern "C" pa_status pa_decode_fwd(const pa_sdpa_desc* desc, const void* q, const void* k,
                                   const void* v, void* out, float* lse, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  clear_error();
  PA_TRY(check_desc(desc));
  const pa_sdpa_desc& d = *desc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (lead_count(d) == 0) return PA_OK;
  size_t need = 0;
  PA_TRY(decode_ws_bytes(d, &need));
  if (workspace) {
    if (workspace_bytes < need) return fail(PA_ERR_INVALID, "decode: workspace smaller than pa_decode_workspace_size");
    return run_decode(d, q, k, v, out, lse, workspace, workspace_bytes, st);
  }
  void* ws = nullptr;
  PA_TRY(scratch_alloc(&ws, need, st));
  pa_status s = run_decode(d, q, k, v, out, lse, ws, need, st);
  scratch_free(ws, st);
  return s;
}

// ---------------------------------------------------------------------------
// Allocation-free decode: the split partials live in a file-scope device
// array instead of a workspace from cudaMallocAsync or from the caller.
//
// Some callers cannot allocate device memory at call time: code running
// under an allocator or memory budget that forbids new cudaMalloc calls once
// a model is loaded, plugin hosts whose device memory is owned by another
// runtime, and latency-critical serving loops that must not synchronise or
// fragment the pool. They pass inputs and outputs only. The scratch below is
// part of the loaded module, so every GPU that loads this library holds it
// (kStaticScratchBytes) until the process exits.
namespace pa {
namespace {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;  // 8 MiB per device
static __device__ __align__(256) uint8_t g_decode_scratch[kStaticScratchBytes];
// Status word for bounded waits when the caller passes none (write-only here).
static __device__ __align__(256) int g_decode_static_status[64];

constexpr int kMaxDev = 64;
void* g_scratch_addr[kMaxDev] = {};
int* g_status_addr[kMaxDev] = {};
std::mutex g_static_mu;

// Host code may not use the symbols' names as device addresses: fetch the
// real addresses once per device, with that device current.
pa_status static_scratch_for_current_device(void** scratch, int** status) {
  int dev = 0;
  PA_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDev) return fail(PA_ERR_UNSUPPORTED, "device index out of range");
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!g_scratch_addr[dev]) {
    void* s = nullptr;
    void* w = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&s, g_decode_scratch);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetSymbolAddress(decode scratch)");
    e = cudaGetSymbolAddress(&w, g_decode_static_status);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetSymbolAddress(decode status)");
    g_status_addr[dev] = static_cast<int*>(w);
    g_scratch_addr[dev] = s;
  }
  *scratch = g_scratch_addr[dev];
  *status = g_status_addr[dev];
  return PA_OK;
}

}  // namespace
}  // namespace pa

extern "C" pa_status pa_decode_fwd_static(const pa_sdpa_desc* desc, const void* q, const void* k,
                                          const void* v, void* out, float* lse, int32_t* status,
                                          void* stream) {
  clear_error();
  PA_TRY(check_desc(desc));
  const pa_sdpa_desc& d = *desc;
  if (lead_count(d) == 0) return PA_OK;
  size_t need = 0;
  PA_TRY(decode_ws_bytes(d, &need));
  if (need > kStaticScratchBytes) {
    char buf[192];
    snprintf(buf, sizeof buf,
             "pa_decode_fwd_static: this problem needs %zu bytes of split scratch; the static "
             "scratch holds %zu bytes (use pa_decode_fwd with a workspace)",
             need, kStaticScratchBytes);
    return fail(PA_ERR_UNSUPPORTED, buf);
  }
  void* scratch = nullptr;
  int* own_status = nullptr;
  PA_TRY(static_scratch_for_current_device(&scratch, &own_status));
  int* st_word = status ? reinterpret_cast<int*>(status) : own_status;
  return run_decode_status(d, q, k, v, out, lse, scratch, kStaticScratchBytes, st_word,
                           static_cast<cudaStream_t>(stream));
}
