// Tensor-core SDPA forward for sm_100a: TMA-fed tiles, tcgen05.mma into
// TMEM, online softmax in fp32 with one query row per thread.
//
// CTA = one 128-row query tile of one (batch, head). 192 threads:
//   warp 0      TMA producer: Q once, then K/V tiles of 128 keys into a ring
//               of shared-memory stages (128-byte swizzle, 64-column boxes).
//   warp 1      owns TMEM (512 columns) and issues the MMAs from one lane:
//                 S_j  = Q K_j^T        (SS form, M=128 N=128 K=D) -> S[j%2]
//                 O   += P_j V_j        (TS form: P_j read from TMEM) -> O
//   warps 2..5  softmax: thread <-> TMEM lane <-> query row. Loads S_j,
//               applies scale / causal / mask / key-bound, keeps a running
//               max m and sum l, writes P_j = 2^(x - m) as fp16/bf16 into the
//               first 64 columns of S[j%2] (aliasing S_j), rescales O only
//               when its row max grows by more than 2^8, and finally writes
//               O / l and the natural-log lse.
// TMEM columns: S0 [0,128), S1 [128,256), O [256, 256+D).
//
// Semantics follow src/portable_attention/reference.py:139-162: top-left
// causal alignment (key j visible to row i iff j <= i), boolean keep-masks,
// additive masks, and exact-zero output for fully-masked rows (l == 0).
// Every wait is bounded; a wait that gives up records a status code and the
// CTA drains its in-flight copies and MMAs before freeing TMEM.
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace pa {
namespace {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColS1 = 128, kColO = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
// Running max moves only when the block max exceeds it by more than this
// (log2 units): P stays <= 2^8 in fp16 and O is rescaled rarely.
constexpr float kRescaleSlack = 8.0f;

template <int D>
struct TcCfg {
  static constexpr int kBoxes = D / 64;                 // 64-column swizzle boxes per tile row
  static constexpr int kTileBytes = BN * D * 2;         // one K or V stage (== BM * D * 2)
  static constexpr int kStages = (D == 128) ? 2 : 4;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + BM * D * 2;
  static constexpr int kVOff = kKOff + kStages * kTileBytes;
  static constexpr int kBarOff = kVOff + kStages * kTileBytes;
  static constexpr int kNumBars = 1 + 4 * kStages + 2 + 2 + 1 + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kMiscOff + 16 + 1024;  // + alignment slack
};

struct TcArgs {
  void* out;
  float* lse;
  const void* mask;
  int* status;
  LeadTable mlt;  // mask offsets per slice
  int64_t L, S;
  int64_t m_rs, m_cs;
  int32_t H, Hkv, group, m_blocks;
  int64_t slices;
  int32_t causal;
  float scale_log2;
};

template <typename MaskT>
__device__ __forceinline__ float mask_add_value(const MaskT* p) {
  return static_cast<float>(*p);
}
template <>
__device__ __forceinline__ float mask_add_value<__half>(const __half* p) { return __half2float(*p); }
template <>
__device__ __forceinline__ float mask_add_value<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

template <int D, bool BF16, int MASK, typename MaskT>
__global__ void __launch_bounds__(kThreads, 1)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, const TcArgs a) {
  using C = TcCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);

  uint8_t* sQ = smem + C::kQOff;
  uint8_t* sK = smem + C::kKOff;
  uint8_t* sV = smem + C::kVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + C::kStages;
  uint64_t* v_full = k_empty + C::kStages;
  uint64_t* v_empty = v_full + C::kStages;
  uint64_t* s_full = v_empty + C::kStages;  // [2]
  uint64_t* p_full = s_full + 2;            // [2]
  uint64_t* o_done = p_full + 2;
  uint64_t* mma_done = o_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMiscOff + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Work item: heaviest (last) query tiles first for causal balance.
  const int64_t item = blockIdx.x;
  const int m_block = a.m_blocks - 1 - static_cast<int>(item / a.slices);
  const int64_t slice = item % a.slices;
  const int64_t m0 = static_cast<int64_t>(m_block) * BM;
  const int32_t zq = static_cast<int32_t>(slice);
  const int32_t zkv = static_cast<int32_t>((slice / a.H) * a.Hkv + (slice % a.H) / a.group);
  int64_t kv_end = a.S;
  if (a.causal) {
    const int64_t last_row = (m0 + BM < a.L ? m0 + BM : a.L) - 1;
    kv_end = last_row + 1 < a.S ? last_row + 1 : a.S;
  }
  const int n_blocks = static_cast<int>((kv_end + BN - 1) / BN);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(k_empty + s, 1);
      mbar_init(v_full + s, 1);
      mbar_init(v_empty + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(s_full + s, 1);
      mbar_init(p_full + s, 128);
    }
    mbar_init(o_done, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n_blocks > 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      mbar_expect_tx(q_full, BM * D * 2);
      for (int b = 0; b < C::kBoxes; ++b)
        tma_load_3d(sQ + b * (BM * 128), &tq, q_full, b * 64, static_cast<int32_t>(m0), zq);
      int last_k[C::kStages], last_v[C::kStages];
#pragma unroll
      for (int s = 0; s < C::kStages; ++s) last_k[s] = last_v[s] = -1;
      for (int j = 0; j < n_blocks; ++j) {
        const int st = j % C::kStages;
        const uint32_t ph = (j / C::kStages) & 1;
        if (!mbar_wait(k_empty + st, ph ^ 1, a.status, kStatusTimeoutFree, abort_flag)) break;
        mbar_expect_tx(k_full + st, C::kTileBytes);
        for (int b = 0; b < C::kBoxes; ++b)
          tma_load_3d(sK + st * C::kTileBytes + b * (BN * 128), &tk, k_full + st, b * 64, j * BN, zkv);
        last_k[st] = j;
        if (!mbar_wait(v_empty + st, ph ^ 1, a.status, kStatusTimeoutFree, abort_flag)) break;
        mbar_expect_tx(v_full + st, C::kTileBytes);
        for (int b = 0; b < C::kBoxes; ++b)
          tma_load_3d(sV + st * C::kTileBytes + b * (BN * 128), &tv, v_full + st, b * 64, j * BN, zkv);
        last_v[st] = j;
      }
      // Every issued copy must land before the CTA may exit. A full barrier
      // completes once per issue, so wait for the last issue of each stage.
      mbar_drain(q_full, 0);
#pragma unroll
      for (int s = 0; s < C::kStages; ++s) {
        if (last_k[s] >= 0) mbar_drain(k_full + s, (last_k[s] / C::kStages) & 1);
        if (last_v[s] >= 0) mbar_drain(v_full + s, (last_v[s] / C::kStages) & 1);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issue
    if (lane == 0 && n_blocks > 0) {
      constexpr uint32_t idS = idesc_f16(BM, BN, false, false, BF16);
      constexpr uint32_t idO = idesc_f16(BM, D, false, true, BF16);
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, a.status, kStatusTimeoutLoad, abort_flag);
      auto issue_pv = [&](int i) -> bool {
        const int st = i % C::kStages;
        const uint32_t ph = (i / C::kStages) & 1;
        const uint32_t sb = i & 1;
        if (!mbar_wait(p_full + sb, (i >> 1) & 1, a.status, kStatusTimeoutSoftmax, abort_flag)) return false;
        if (!mbar_wait(v_full + st, ph, a.status, kStatusTimeoutLoad, abort_flag)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + st * C::kTileBytes);
        const uint32_t p_col = tmem + (sb ? kColS1 : kColS0);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t bdesc = sdesc_sw128(v_addr + kk * 2048, BN * 128, 1024);
          umma_ts(tmem + kColO, p_col + kk * 8, bdesc, idO, (i > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(o_done);
        tc_commit(v_empty + st);
        return true;
      };
      for (int j = 0; ok && j < n_blocks; ++j) {
        const int st = j % C::kStages;
        const uint32_t ph = (j / C::kStages) & 1;
        const uint32_t sb = j & 1;
        if (!mbar_wait(k_full + st, ph, a.status, kStatusTimeoutLoad, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * C::kTileBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t box = kk / 4, sub = (kk % 4) * 32;
          const uint64_t adesc = sdesc_sw128(q_addr + box * (BM * 128) + sub, 16, 1024);
          const uint64_t bdesc = sdesc_sw128(k_addr + box * (BN * 128) + sub, 16, 1024);
          umma_ss(tmem + (sb ? kColS1 : kColS0), adesc, bdesc, idS, kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full + sb);
        tc_commit(k_empty + st);
        if (j >= 1 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) issue_pv(n_blocks - 1);
      // All issued tensor-core work must finish before TMEM is freed.
      tc_commit(mma_done);
      mbar_drain(mma_done, 0);
    }
    __syncwarp();
  } else {
    // --------------------------------------------------------------- softmax
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // row inside the tile == TMEM lane
    const int64_t row = m0 + r;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const bool row_ok = row < a.L;
    float m_run = -INFINITY, l_run = 0.f;
    const SliceOffsets moff = slice_offsets(a.mlt, slice);
    bool ok = true;

    for (int j = 0; j < n_blocks; ++j) {
      const uint32_t sb = j & 1;
      ok = mbar_wait(s_full + sb, (j >> 1) & 1, a.status, kStatusTimeoutMma, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t s_addr = lane_base + (sb ? kColS1 : kColS0);
      float x[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t rr[32];
        tmem_ld32(s_addr + c * 32, rr);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t) x[c * 32 + t] = __uint_as_float(rr[t]) * a.scale_log2;
      }
      const int64_t n0 = static_cast<int64_t>(j) * BN;
      const bool edge = (n0 + BN > a.S) || (a.causal && n0 + BN - 1 > m0);
      if (edge || MASK != PA_MASK_NONE) {
        const int64_t vis = a.causal ? (row + 1 < a.S ? row + 1 : a.S) : a.S;
#pragma unroll
        for (int t = 0; t < BN; ++t) {
          const int64_t col = n0 + t;
          if (col >= vis) x[t] = -INFINITY;
        }
        if (MASK != PA_MASK_NONE && row_ok) {
          const int64_t base = moff.m + row * a.m_rs;
#pragma unroll
          for (int t = 0; t < BN; ++t) {
            const int64_t col = n0 + t;
            if (col < a.S) {
              if (MASK == PA_MASK_BOOL) {
                if (!static_cast<const uint8_t*>(a.mask)[base + col * a.m_cs]) x[t] = -INFINITY;
              } else {
                x[t] += kLog2e * mask_add_value(static_cast<const MaskT*>(a.mask) + base + col * a.m_cs);
              }
            }
          }
        }
      }
      float mx = x[0];
#pragma unroll
      for (int t = 1; t < BN; ++t) mx = fmaxf(mx, x[t]);
      const float m_new = fmaxf(m_run, mx);
      const float m_use = (m_run == -INFINITY || m_new - m_run > kRescaleSlack) ? m_new : m_run;
      float rowsum = 0.f;
      uint32_t pk[BN / 2];
      if (m_use == -INFINITY) {
#pragma unroll
        for (int t = 0; t < BN / 2; ++t) pk[t] = 0u;
      } else {
#pragma unroll
        for (int t = 0; t < BN / 2; ++t) {
          const float p0 = ex2(x[2 * t] - m_use);
          const float p1 = ex2(x[2 * t + 1] - m_use);
          rowsum += p0 + p1;
          pk[t] = pack2(p0, p1, BF16);
        }
      }
      {
        uint32_t half0[32], half1[32];
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          half0[t] = pk[t];
          half1[t] = pk[32 + t];
        }
        tmem_st32(s_addr, half0);
        tmem_st32(s_addr + 32, half1);
        tmem_st_wait();
      }
      const float alpha = (m_use == m_run) ? 1.f : ((m_run == -INFINITY) ? 0.f : ex2(m_run - m_use));
      const bool need = (j > 0) && (m_use != m_run);
      if (__any_sync(0xffffffffu, need)) {
        ok = mbar_wait(o_done, (j - 1) & 1, a.status, kStatusTimeoutMma, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t rr[32];
          tmem_ld32(lane_base + kColO + c * 32, rr);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 32; ++t) rr[t] = __float_as_uint(__uint_as_float(rr[t]) * alpha);
          tmem_st32(lane_base + kColO + c * 32, rr);
        }
        tmem_st_wait();
      }
      l_run = l_run * alpha + rowsum;
      m_run = m_use;
      tc_fence_before();
      mbar_arrive(p_full + sb);
    }

    if (ok && n_blocks > 0) {
      ok = mbar_wait(o_done, (n_blocks - 1) & 1, a.status, kStatusTimeoutMma, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      uint8_t* orow = static_cast<uint8_t*>(a.out) + ((slice * a.L + row) * D) * 2;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t rr[32];
        if (n_blocks > 0) {
          tmem_ld32(lane_base + kColO + c * 32, rr);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) rr[t] = 0u;
        }
        uint32_t pk[16];
#pragma unroll
        for (int t = 0; t < 16; ++t)
          pk[t] = pack2(__uint_as_float(rr[2 * t]) * inv, __uint_as_float(rr[2 * t + 1]) * inv, BF16);
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 64);
#pragma unroll
          for (int t = 0; t < 4; ++t) dst[t] = make_uint4(pk[4 * t], pk[4 * t + 1], pk[4 * t + 2], pk[4 * t + 3]);
        }
      }
      if (row_ok && a.lse)
        a.lse[slice * a.L + row] = l_run > 0.f ? (m_run + __log2f(l_run)) * kLn2 : -INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D, bool BF16, int MASK, typename MaskT>
pa_status launch_variant(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                         const TcArgs& a, int64_t grid, cudaStream_t st) {
  auto kern = fwd_tc_kernel<D, BF16, MASK, MaskT>;
  constexpr int smem = TcCfg<D>::kSmemBytes;
  PA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  kern<<<static_cast<unsigned>(grid), kThreads, smem, st>>>(tq, tk, tv, a);
  PA_CUDA(cudaGetLastError());
  return PA_OK;
}

template <int D, bool BF16>
pa_status launch_masked(const pa_sdpa_desc& d, const CUtensorMap& tq, const CUtensorMap& tk,
                        const CUtensorMap& tv, const TcArgs& a, int64_t grid, cudaStream_t st) {
  if (d.mask_kind == PA_MASK_NONE || d.is_causal)
    return launch_variant<D, BF16, PA_MASK_NONE, float>(tq, tk, tv, a, grid, st);
  if (d.mask_kind == PA_MASK_BOOL)
    return launch_variant<D, BF16, PA_MASK_BOOL, uint8_t>(tq, tk, tv, a, grid, st);
  switch (d.mask_dtype) {
    case PA_F16: return launch_variant<D, BF16, PA_MASK_ADD, __half>(tq, tk, tv, a, grid, st);
    case PA_BF16: return launch_variant<D, BF16, PA_MASK_ADD, __nv_bfloat16>(tq, tk, tv, a, grid, st);
    case PA_F32: return launch_variant<D, BF16, PA_MASK_ADD, float>(tq, tk, tv, a, grid, st);
    default: return fail(PA_ERR_UNSUPPORTED, "additive mask dtype not supported by the tensor-core kernel");
  }
}

}  // namespace

bool dense_bhsd(const pa_sdpa_desc& d, int64_t* slices, int64_t* heads, int64_t* kv_heads) {
  const int64_t n = lead_count(d);
  const int64_t H = d.nlead > 0 ? d.lead[d.nlead - 1] : 1;
  const int64_t g = d.gqa_group > 1 ? d.gqa_group : 1;
  if (g > 1 && d.gqa_axis != d.nlead - 1) return false;
  if (H % g) return false;
  const int64_t Hkv = H / g;
  if (d.q_row_stride != d.E || d.k_row_stride != d.E || d.v_row_stride != d.Ev) return false;
  // Dense strides: q over the full lead, k/v over the lead with H -> Hkv.
  int64_t qs = d.L * d.E, ks = d.S * d.E, vs = d.S * d.Ev;
  for (int i = d.nlead - 1; i >= 0; --i) {
    const int64_t dim = d.lead[i];
    const int64_t kdim = (i == d.nlead - 1) ? Hkv : dim;
    if (dim > 1) {
      if (d.q_lead_stride[i] != qs) return false;
      if (kdim > 1 && (d.k_lead_stride[i] != ks || d.v_lead_stride[i] != vs)) return false;
    }
    qs *= dim;
    ks *= kdim;
    vs *= kdim;
  }
  *slices = n;
  *heads = H;
  *kv_heads = Hkv;
  return true;
}

bool fwd_tc_eligible(const pa_sdpa_desc& d, std::string* why) {
  auto no = [&](const char* m) {
    if (why) *why = m;
    return false;
  };
  if (d.dtype != PA_F16 && d.dtype != PA_BF16) return no("dtype is not fp16/bf16");
  if (d.E != d.Ev || (d.E != 64 && d.E != 128)) return no("head dim not 64/128 or E != Ev");
  int64_t n, H, Hkv;
  if (!dense_bhsd(d, &n, &H, &Hkv)) return no("operands are not dense (B, H, L, D)");
  if (n > 0x7fffffffLL / 64 || d.L > 0x7fffffffLL || d.S > 0x7fffffffLL) return no("too large");
  if (!d.is_causal && d.mask_kind == PA_MASK_ADD && d.mask_dtype == PA_F64)
    return no("fp64 additive mask");
  return true;
}

pa_status launch_fwd_tc(const pa_sdpa_desc& d, const void* q, const void* k, const void* v,
                        const void* mask, void* out, float* lse, cudaStream_t st) {
  int64_t n, H, Hkv;
  if (!dense_bhsd(d, &n, &H, &Hkv)) return fail(PA_ERR_INVALID, "fwd_tc: operands not dense");
  const int D = static_cast<int>(d.E);
  const bool bf16 = d.dtype == PA_BF16;
  const CUtensorMapDataType tdt = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tk, tv;
  const uint64_t rowb = static_cast<uint64_t>(D) * 2;
  PA_TRY(encode_tma_3d(&tq, tdt, q, D, d.L, n, rowb, rowb * d.L, 64, BM, CU_TENSOR_MAP_SWIZZLE_128B));
  const int64_t nkv = (n / H) * Hkv;
  PA_TRY(encode_tma_3d(&tk, tdt, k, D, d.S, nkv, rowb, rowb * d.S, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B));
  PA_TRY(encode_tma_3d(&tv, tdt, v, D, d.S, nkv, rowb, rowb * d.S, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B));
  TcArgs a{};
  a.out = out;
  a.lse = lse;
  a.mask = mask;
  a.status = device_status_word();
  if (!a.status) return fail(PA_ERR_CUDA, "device status word unavailable");
  a.mlt = make_lead_table(d);
  a.mlt.gqa_axis = -1;
  a.L = d.L;
  a.S = d.S;
  a.m_rs = d.m_row_stride;
  a.m_cs = d.m_col_stride;
  a.H = static_cast<int32_t>(H);
  a.Hkv = static_cast<int32_t>(Hkv);
  a.group = static_cast<int32_t>(H / Hkv);
  a.m_blocks = static_cast<int32_t>((d.L + BM - 1) / BM);
  a.slices = n;
  a.causal = d.is_causal;
  a.scale_log2 = static_cast<float>(d.scale * 1.4426950408889634);
  const int64_t grid = n * a.m_blocks;
  if (grid == 0) return PA_OK;
  if (grid > 0x7fffffffLL) return fail(PA_ERR_UNSUPPORTED, "fwd_tc: grid too large");
  if (D == 128)
    return bf16 ? launch_masked<128, true>(d, tq, tk, tv, a, grid, st)
                : launch_masked<128, false>(d, tq, tk, tv, a, grid, st);
  return bf16 ? launch_masked<64, true>(d, tq, tk, tv, a, grid, st)
              : launch_masked<64, false>(d, tq, tk, tv, a, grid, st);
}

}  // namespace pa
