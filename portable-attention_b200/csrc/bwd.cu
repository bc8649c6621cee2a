// Backward (VJP) of the SDPA forward on sm_100a tensor cores.
//
// With S = scale * Q K^T, P = softmax(S) (recomputed from the saved lse),
// dP = dO V^T and dS = P * (dP - rowsum(dO * O)):
//   dV = P^T dO,   dK = scale * dS^T Q,   dQ = scale * dS K.
// Three launches, no atomics (results are deterministic):
//   bwd_prep_kernel   delta = rowsum(dO * O) and lse in log2 units, per row,
//                     into a row-padded fp32 workspace (rows rounded up to 64).
//   bwd_dkdv_kernel   CTA = 128 keys of one (batch, KV head). Loops over every
//                     query head of the grouped-query group and every 64-row
//                     query block that can see those keys:
//                       S^T  = K Q^T     (SS, M=128 keys, N=64 rows)
//                       dP^T = V dO^T    (SS)
//                       softmax warps: P^T, dS^T -> fp16 into TMEM (aliasing)
//                       dV  += P^T dO    (TS, B = dO MN-major)
//                       dK  += dS^T Q    (TS, B = Q MN-major)
//                     S^T / dP^T are double-buffered so the next block's MMAs
//                     overlap this block's softmax. dK, dV stay in TMEM until
//                     the end: grouped-query heads are summed in place.
//   bwd_dq_kernel     CTA = 128 query rows of one (batch, head). Its Q and
//                     dO rows are written once into TMEM by the softmax
//                     warps (thread <-> row), then it loops over 64-key
//                     blocks:  S = Q K^T, dP = dO V^T (TS: A from TMEM, so
//                     each MMA reads only K or V from shared memory),
//                     dS -> fp16 into TMEM, dQ += dS K (TS, B = K MN-major).
// TMEM (512 columns): dkdv S^T[2] 0..127, dP^T[2] 128..255, dV, dK after;
// dq S[2] 0..127, dP[2] 128..255, dQ at 256, Q at 384, dO at 384 + D/2.
// Masking matches the forward: top-left causal (key j visible to row i iff
// j <= i), keys >= S and rows >= L contribute nothing, and rows whose lse is
// -inf (fully masked) have P = 0 and so zero gradient.
#include <math.h>

#include <functional>

#include "common.cuh"
#include "kernels.h"

namespace pa {
namespace {

// Warp 0 TMA producer, warp 1 MMA issuer, warps 2-9 two "softmax" warpgroups
// that split each block's 64 columns in halves (thread <-> TMEM lane <-> row;
// there is no row reduction in the backward, so the halves are independent).
constexpr int kThreadsB = 320;
constexpr int kSoftThreadsB = 256;
constexpr int kRowPad = 64;

struct BwdArgs {
  void* dk;
  void* dv;
  void* dq;
  // When set, the gradients are added in fp32 into these (same dense layouts as
  // dk / dv / dq) instead of being stored in the operand type: the ring
  // accumulates a chunk pair's contribution this way without extra kernels.
  float* dk_acc;
  float* dv_acc;
  float* dq_acc;
  const void* q;       // (slices_q, L, D), read row by row into tensor memory by the dQ kernel
  const void* dout;    // same layout as q
  const float* lse2;   // [slices_q][Lp], log2 units
  const float* delta;  // [slices_q][Lp]
  int* status;
  int64_t L, S, Lp;
  int32_t Hq, Hkv, group, blocks;
  int64_t slices;      // B*Hkv (dkdv) or B*Hq (dq)
  int32_t causal;
  float scale_log2, scale;
};

template <bool BF16>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  if (BF16) return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// One warp per row: delta = sum_d dO * O; lse2 = lse * log2(e); padded rows
// get delta 0 and lse2 -inf.
template <int D, bool BF16>
__global__ void bwd_prep_kernel(const void* o, const void* dout, const float* lse, float* delta,
                                float* lse2, int64_t slices, int64_t L, int64_t Lp) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  if (r >= slices * Lp) return;
  const int64_t sl = r / Lp, row = r % Lp;
  if (row >= L) {
    if (lane == 0) {
      delta[r] = 0.f;
      lse2[r] = -INFINITY;
    }
    return;
  }
  const int64_t src = (sl * L + row) * D;
  constexpr int PER = D / 32;  // elements per lane (2 or 4)
  const uint8_t* ob = static_cast<const uint8_t*>(o) + (src + lane * PER) * 2;
  const uint8_t* db = static_cast<const uint8_t*>(dout) + (src + lane * PER) * 2;
  float acc = 0.f;
  if (PER == 4) {
    const uint2 a = *reinterpret_cast<const uint2*>(ob);
    const uint2 b = *reinterpret_cast<const uint2*>(db);
    const float2 a0 = unpack2<BF16>(a.x), a1 = unpack2<BF16>(a.y);
    const float2 b0 = unpack2<BF16>(b.x), b1 = unpack2<BF16>(b.y);
    acc = a0.x * b0.x + a0.y * b0.y + a1.x * b1.x + a1.y * b1.y;
  } else {
    const float2 a0 = unpack2<BF16>(*reinterpret_cast<const uint32_t*>(ob));
    const float2 b0 = unpack2<BF16>(*reinterpret_cast<const uint32_t*>(db));
    acc = a0.x * b0.x + a0.y * b0.y;
  }
  for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    delta[r] = acc;
    const float l = lse[sl * L + row];
    lse2[r] = l == -INFINITY ? -INFINITY : l * 1.4426950408889634f;
  }
}

// Add 32 fp32 values (scaled) into 32 consecutive fp32 accumulators (16-byte aligned).
__device__ __forceinline__ void accum_row32(float* dst, const uint32_t (&rr)[32], float mul) {
  float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    float4 x = d4[t];
    x.x = fmaf(__uint_as_float(rr[4 * t]), mul, x.x);
    x.y = fmaf(__uint_as_float(rr[4 * t + 1]), mul, x.y);
    x.z = fmaf(__uint_as_float(rr[4 * t + 2]), mul, x.z);
    x.w = fmaf(__uint_as_float(rr[4 * t + 3]), mul, x.w);
    d4[t] = x;
  }
}

// Store 32 fp32 values (scaled) as 16 packed fp16/bf16 words -> 64 bytes.
template <bool BF16>
__device__ __forceinline__ void store_row32(uint8_t* dst, const uint32_t (&rr)[32], float mul) {
  uint32_t pk[16];
#pragma unroll
  for (int t = 0; t < 16; ++t)
    pk[t] = pack2(__uint_as_float(rr[2 * t]) * mul, __uint_as_float(rr[2 * t + 1]) * mul, BF16);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int t = 0; t < 4; ++t) d4[t] = make_uint4(pk[4 * t], pk[4 * t + 1], pk[4 * t + 2], pk[4 * t + 3]);
}

// ------------------------------------------------------------------ dK / dV

template <int D>
struct DkdvCfg {
  static constexpr int BQ = 64, BK = 128;
  static constexpr int kBoxes = D / 64;
  static constexpr int kKVBytes = BK * D * 2;
  static constexpr int kQBytes = BQ * D * 2;
  static constexpr int kStages = 3;
  static constexpr int kStageBytes = ((2 * kQBytes + 2 * BQ * 4) + 1023) / 1024 * 1024;
  static constexpr int kKOff = 0, kVOff = kKVBytes, kStageOff = 2 * kKVBytes;
  static constexpr int kBarOff = kStageOff + kStages * kStageBytes;
  static constexpr int kNumBars = 1 + 2 * kStages + 2 + 2 + 2;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kMiscOff + 16 + 1024;
  static constexpr uint32_t kColS = 0, kColP = 128, kColV = 256, kColK = 256 + D;
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreadsB, 1)
    bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                    const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                    const BwdArgs a) {
  using C = DkdvCfg<D>;
  constexpr int BQ = C::BQ, BK = C::BK;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sK = smem + C::kKOff;
  uint8_t* sV = smem + C::kVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* kv_full = bars;
  uint64_t* qd_full = bars + 1;
  uint64_t* qd_empty = qd_full + C::kStages;
  uint64_t* sdp_full = qd_empty + C::kStages;  // [2]
  uint64_t* ds_ready = sdp_full + 2;            // [2]
  uint64_t* acc_done = ds_ready + 2;
  uint64_t* mma_done = acc_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMiscOff + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kv_blk = static_cast<int>(blockIdx.x / a.slices);  // low blocks (most work) first
  const int64_t pair = blockIdx.x % a.slices;                  // b * Hkv + kvh
  const int64_t n0 = static_cast<int64_t>(kv_blk) * BK;
  const int64_t b = pair / a.Hkv;
  const int kvh = static_cast<int>(pair % a.Hkv);
  const int nqb = static_cast<int>((a.L + BQ - 1) / BQ);
  const int qb0 = a.causal ? static_cast<int>(n0 / BQ) : 0;
  const int per_head = nqb > qb0 ? nqb - qb0 : 0;
  const int n = per_head * a.group;
  auto stage_ptr = [&](int st) { return smem + C::kStageOff + st * C::kStageBytes; };

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(qd_full + s, 1);
      mbar_init(qd_empty + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(sdp_full + s, 1);
      mbar_init(ds_ready + s, kSoftThreadsB);
    }
    mbar_init(acc_done, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && n > 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tdo);
      mbar_expect_tx(kv_full, 2 * C::kKVBytes);
      for (int bx = 0; bx < C::kBoxes; ++bx) {
        tma_load_3d(sK + bx * (BK * 128), &tk, kv_full, bx * 64, static_cast<int32_t>(n0), static_cast<int32_t>(pair));
        tma_load_3d(sV + bx * (BK * 128), &tv, kv_full, bx * 64, static_cast<int32_t>(n0), static_cast<int32_t>(pair));
      }
      int last[C::kStages];
#pragma unroll
      for (int s = 0; s < C::kStages; ++s) last[s] = -1;
      for (int i = 0; i < n; ++i) {
        const int st = i % C::kStages;
        if (!mbar_wait(qd_empty + st, ((i / C::kStages) & 1) ^ 1, a.status, kStatusTimeoutFree, abort_flag)) break;
        const int h = i / per_head;
        const int64_t q0 = static_cast<int64_t>(qb0 + i % per_head) * BQ;
        const int64_t zq = b * a.Hq + static_cast<int64_t>(kvh) * a.group + h;
        uint8_t* sp = stage_ptr(st);
        mbar_expect_tx(qd_full + st, 2 * C::kQBytes + 2 * BQ * 4);
        for (int bx = 0; bx < C::kBoxes; ++bx) {
          tma_load_3d(sp + bx * (BQ * 128), &tq, qd_full + st, bx * 64, static_cast<int32_t>(q0), static_cast<int32_t>(zq));
          tma_load_3d(sp + C::kQBytes + bx * (BQ * 128), &tdo, qd_full + st, bx * 64, static_cast<int32_t>(q0),
                      static_cast<int32_t>(zq));
        }
        bulk_load(sp + 2 * C::kQBytes, a.lse2 + zq * a.Lp + q0, BQ * 4, qd_full + st);
        bulk_load(sp + 2 * C::kQBytes + BQ * 4, a.delta + zq * a.Lp + q0, BQ * 4, qd_full + st);
        last[st] = i;
      }
      mbar_drain(kv_full, 0);
#pragma unroll
      for (int s = 0; s < C::kStages; ++s)
        if (last[s] >= 0) mbar_drain(qd_full + s, (last[s] / C::kStages) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && n > 0) {
      constexpr uint32_t idS = idesc_f16(128, BQ, false, false, BF16);
      constexpr uint32_t idA = idesc_f16(128, D, false, true, BF16);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      bool ok = mbar_wait(kv_full, 0, a.status, kStatusTimeoutLoad, abort_flag);
      auto issue_sdp = [&](int i) -> bool {
        const int st = i % C::kStages;
        if (!mbar_wait(qd_full + st, (i / C::kStages) & 1, a.status, kStatusTimeoutLoad, abort_flag)) return false;
        tc_fence_after();
        const uint32_t sb = i & 1;
        const uint32_t q_addr = smem_u32(stage_ptr(st)), do_addr = q_addr + C::kQBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t bx = kk / 4, sub = (kk % 4) * 32;
          umma_ss(tmem + C::kColS + sb * 64, sdesc_sw128(k_addr + bx * (BK * 128) + sub, 16, 1024),
                  sdesc_sw128(q_addr + bx * (BQ * 128) + sub, 16, 1024), idS, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t bx = kk / 4, sub = (kk % 4) * 32;
          umma_ss(tmem + C::kColP + sb * 64, sdesc_sw128(v_addr + bx * (BK * 128) + sub, 16, 1024),
                  sdesc_sw128(do_addr + bx * (BQ * 128) + sub, 16, 1024), idS, kk > 0);
        }
        tc_commit(sdp_full + sb);
        return true;
      };
      if (ok) ok = issue_sdp(0);
      for (int i = 0; ok && i < n; ++i) {
        if (i + 1 < n && !issue_sdp(i + 1)) {
          ok = false;
          break;
        }
        const uint32_t sb = i & 1;
        if (!mbar_wait(ds_ready + sb, (i >> 1) & 1, a.status, kStatusTimeoutSoftmax, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int st = i % C::kStages;
        const uint32_t q_addr = smem_u32(stage_ptr(st)), do_addr = q_addr + C::kQBytes;
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          umma_ts(tmem + C::kColV, tmem + C::kColS + sb * 64 + kk * 8,
                  sdesc_sw128(do_addr + kk * 2048, BQ * 128, 1024), idA, (i > 0 || kk > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          umma_ts(tmem + C::kColK, tmem + C::kColP + sb * 64 + kk * 8,
                  sdesc_sw128(q_addr + kk * 2048, BQ * 128, 1024), idA, (i > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(qd_empty + st);
      }
      tc_commit(acc_done);
      tc_commit(mma_done);
      mbar_drain(mma_done, 0);
    }
    __syncwarp();
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // which 32 columns of each block this warpgroup owns
    const int r = quad * 32 + lane;
    const int64_t key = n0 + r;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      const uint32_t sb = i & 1;
      const int st = i % C::kStages;
      ok = mbar_wait(sdp_full + sb, (i >> 1) & 1, a.status, kStatusTimeoutMma, abort_flag);
      ok = ok && mbar_wait(qd_full + st, (i / C::kStages) & 1, a.status, kStatusTimeoutLoad, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const float* l2 = reinterpret_cast<const float*>(stage_ptr(st) + 2 * C::kQBytes);
      const float* dl = l2 + BQ;
      const int64_t q0 = static_cast<int64_t>(qb0 + i % per_head) * BQ;
      // Visible query columns of this key row: c in [cmin, cmax).
      const int64_t lo = a.causal ? key - q0 : 0;
      const int cmin = static_cast<int>(lo < 0 ? 0 : (lo > BQ ? BQ : lo));
      const int64_t hi = a.L - q0;
      const int cmax = static_cast<int>(hi < 0 ? 0 : (hi > BQ ? BQ : hi));
      const bool all_vis = __all_sync(0xffffffffu, cmin == 0 && cmax == BQ);
      {
        uint32_t sr[32], pr[32];
        tmem_ld32(lane_base + C::kColS + sb * 64 + half * 32, sr);
        tmem_ld32(lane_base + C::kColP + sb * 64 + half * 32, pr);
        tmem_ld_wait();
        reg_fence(sr);
        reg_fence(pr);
        uint32_t pk[16], dk[16];
        const uint64_t sl2x2 = f2(a.scale_log2, a.scale_log2);
#pragma unroll
        for (int v4 = 0; v4 < 8; ++v4) {
          const float4 lz = reinterpret_cast<const float4*>(l2)[half * 8 + v4];
          const float4 dd = reinterpret_cast<const float4*>(dl)[half * 8 + v4];
          const uint64_t nlz[2] = {f2(-lz.x, -lz.y), f2(-lz.z, -lz.w)};
          const uint64_t ndd[2] = {f2(-dd.x, -dd.y), f2(-dd.z, -dd.w)};
          const float lzv[4] = {lz.x, lz.y, lz.z, lz.w};
#pragma unroll
          for (int w = 0; w < 2; ++w) {
            const int e = v4 * 4 + 2 * w;      // column pair inside this half
            const int c = half * 32 + e;       // column inside the block
            // p = 2^(s * scale - lse), dS = p * (dP - delta), two columns at a time
            const uint64_t y = fma2(f2(__uint_as_float(sr[e]), __uint_as_float(sr[e + 1])), sl2x2, nlz[w]);
            float p0 = ex2(f2_lo(y)), p1 = ex2(f2_hi(y));
            if (!all_vis) {
              p0 = (c >= cmin && c < cmax && lzv[2 * w] != -INFINITY) ? p0 : 0.f;
              p1 = (c + 1 >= cmin && c + 1 < cmax && lzv[2 * w + 1] != -INFINITY) ? p1 : 0.f;
            }
            const uint64_t p2 = f2(p0, p1);
            const uint64_t d2 = mul2(p2, add2(f2(__uint_as_float(pr[e]), __uint_as_float(pr[e + 1])), ndd[w]));
            float d0 = f2_lo(d2), d1 = f2_hi(d2);
            if (!all_vis) {
              if (!(c >= cmin && c < cmax)) d0 = 0.f;
              if (!(c + 1 >= cmin && c + 1 < cmax)) d1 = 0.f;
            }
            pk[v4 * 2 + w] = pack2(p0, p1, BF16);
            dk[v4 * 2 + w] = pack2(d0, d1, BF16);
          }
        }
        tmem_st16(lane_base + C::kColS + sb * 64 + half * 16, pk);
        tmem_st16(lane_base + C::kColP + sb * 64 + half * 16, dk);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(ds_ready + sb);
    }
    if (ok && n > 0) {
      ok = mbar_wait(acc_done, 0, a.status, kStatusTimeoutMma, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      const bool row_ok = key < a.S;
      uint8_t* dvrow = static_cast<uint8_t*>(a.dv) + ((pair * a.S + key) * D) * 2;
      uint8_t* dkrow = static_cast<uint8_t*>(a.dk) + ((pair * a.S + key) * D) * 2;
#pragma unroll
      for (int c = half * (D / 64); c < (half + 1) * (D / 64); ++c) {
        uint32_t rv[32], rk[32];
        if (n > 0) {
          tmem_ld32(lane_base + C::kColV + c * 32, rv);
          tmem_ld32(lane_base + C::kColK + c * 32, rk);
          tmem_ld_wait();
          reg_fence(rv);
          reg_fence(rk);
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) rv[t] = rk[t] = 0u;
        }
        if (row_ok && a.dk_acc) {
          accum_row32(a.dv_acc + (pair * a.S + key) * D + c * 32, rv, 1.f);
          accum_row32(a.dk_acc + (pair * a.S + key) * D + c * 32, rk, a.scale);
        } else if (row_ok) {
          store_row32<BF16>(dvrow + c * 64, rv, 1.f);
          store_row32<BF16>(dkrow + c * 64, rk, a.scale);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------- dQ

template <int D>
struct DqCfg {
  static constexpr int BQ = 128, BK = 64;
  static constexpr int kBoxes = D / 64;
  static constexpr int kKBytes = BK * D * 2;
  static constexpr int kStages = 4;
  static constexpr int kStageOff = 0;
  static constexpr int kStageBytes = 2 * kKBytes;
  static constexpr int kBarOff = kStageOff + kStages * kStageBytes;
  static constexpr int kNumBars = 1 + 2 * kStages + 2 + 2 + 2;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kMiscOff + 16 + 1024;
  // TMEM columns: S and dP (two 64-column buffers each; dS overwrites dP),
  // the dQ accumulator, then the CTA's Q and dO rows as fp16/bf16 pairs
  // (D/2 columns each): S = Q K^T and dP = dO V^T take their A operand from
  // tensor memory, so each MMA reads only its K or V tile from shared memory.
  static constexpr uint32_t kColS = 0, kColP = 128, kColQ = 256, kColQa = 384, kColDOa = 384 + D / 2;
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreadsB, 1)
    bwd_dq_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                  const BwdArgs a) {
  using C = DqCfg<D>;
  constexpr int BQ = C::BQ, BK = C::BK;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* qa_ready = bars;  // Q and dO rows are in tensor memory
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + C::kStages;
  uint64_t* sdp_full = kv_empty + C::kStages;
  uint64_t* ds_ready = sdp_full + 2;
  uint64_t* acc_done = ds_ready + 2;
  uint64_t* mma_done = acc_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMiscOff + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_blk = a.blocks - 1 - static_cast<int>(blockIdx.x / a.slices);  // heaviest first
  const int64_t zq = blockIdx.x % a.slices;                                   // b * Hq + h
  const int64_t m0 = static_cast<int64_t>(m_blk) * BQ;
  const int64_t zkv = (zq / a.Hq) * a.Hkv + (zq % a.Hq) / a.group;
  int64_t kv_end = a.S;
  if (a.causal) {
    const int64_t last = (m0 + BQ < a.L ? m0 + BQ : a.L);
    kv_end = last < a.S ? last : a.S;
  }
  const int n = static_cast<int>((kv_end + BK - 1) / BK);
  auto stage_ptr = [&](int st) { return smem + C::kStageOff + st * C::kStageBytes; };

  if (threadIdx.x == 0) {
    mbar_init(qa_ready, kSoftThreadsB);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(kv_full + s, 1);
      mbar_init(kv_empty + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(sdp_full + s, 1);
      mbar_init(ds_ready + s, kSoftThreadsB);
    }
    mbar_init(acc_done, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && n > 0) {
      int last[C::kStages];
#pragma unroll
      for (int s = 0; s < C::kStages; ++s) last[s] = -1;
      for (int j = 0; j < n; ++j) {
        const int st = j % C::kStages;
        if (!mbar_wait(kv_empty + st, ((j / C::kStages) & 1) ^ 1, a.status, kStatusTimeoutFree, abort_flag)) break;
        uint8_t* sp = stage_ptr(st);
        mbar_expect_tx(kv_full + st, C::kStageBytes);
        for (int bx = 0; bx < C::kBoxes; ++bx) {
          tma_load_3d(sp + bx * (BK * 128), &tk, kv_full + st, bx * 64, j * BK, static_cast<int32_t>(zkv));
          tma_load_3d(sp + C::kKBytes + bx * (BK * 128), &tv, kv_full + st, bx * 64, j * BK,
                      static_cast<int32_t>(zkv));
        }
        last[st] = j;
      }
#pragma unroll
      for (int s = 0; s < C::kStages; ++s)
        if (last[s] >= 0) mbar_drain(kv_full + s, (last[s] / C::kStages) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && n > 0) {
      constexpr uint32_t idS = idesc_f16(128, BK, false, false, BF16);
      constexpr uint32_t idQ = idesc_f16(128, D, false, true, BF16);
      bool ok = mbar_wait(qa_ready, 0, a.status, kStatusTimeoutSoftmax, abort_flag);
      if (ok) tc_fence_after();
      auto issue_sdp = [&](int j) -> bool {
        const int st = j % C::kStages;
        if (!mbar_wait(kv_full + st, (j / C::kStages) & 1, a.status, kStatusTimeoutLoad, abort_flag)) return false;
        tc_fence_after();
        const uint32_t sb = j & 1;
        const uint32_t k_addr = smem_u32(stage_ptr(st)), v_addr = k_addr + C::kKBytes;
        // A = Q (dO) rows from tensor memory: 16 head-dim elements = 8 columns per step.
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t bx = kk / 4, sub = (kk % 4) * 32;
          umma_ts(tmem + C::kColS + sb * 64, tmem + C::kColQa + kk * 8,
                  sdesc_sw128(k_addr + bx * (BK * 128) + sub, 16, 1024), idS, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t bx = kk / 4, sub = (kk % 4) * 32;
          umma_ts(tmem + C::kColP + sb * 64, tmem + C::kColDOa + kk * 8,
                  sdesc_sw128(v_addr + bx * (BK * 128) + sub, 16, 1024), idS, kk > 0);
        }
        tc_commit(sdp_full + sb);
        return true;
      };
      if (ok) ok = issue_sdp(0);
      for (int j = 0; ok && j < n; ++j) {
        if (j + 1 < n && !issue_sdp(j + 1)) {
          ok = false;
          break;
        }
        const uint32_t sb = j & 1;
        if (!mbar_wait(ds_ready + sb, (j >> 1) & 1, a.status, kStatusTimeoutSoftmax, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int st = j % C::kStages;
        const uint32_t k_addr = smem_u32(stage_ptr(st));
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          umma_ts(tmem + C::kColQ, tmem + C::kColP + sb * 64 + kk * 8,
                  sdesc_sw128(k_addr + kk * 2048, BK * 128, 1024), idQ, (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(kv_empty + st);
      }
      tc_commit(acc_done);
      tc_commit(mma_done);
      mbar_drain(mma_done, 0);
    }
    __syncwarp();
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // which 32 columns of each block this warpgroup owns
    const int r = quad * 32 + lane;
    const int64_t row = m0 + r;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const float lz = a.lse2[zq * a.Lp + row];  // padded rows hold -inf
    const float dlt = a.delta[zq * a.Lp + row];
    const bool row_live = row < a.L && lz != -INFINITY;
    if (n > 0) {
      // This thread's row of Q (first warpgroup) or dO (second) into its TMEM
      // lane as the A operand of S = Q K^T or dP = dO V^T; rows past L are zero.
      const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(half ? a.dout : a.q) +
                                                        ((zq * a.L + row) * D) * 2);
      const uint32_t col = half ? C::kColDOa : C::kColQa;
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        uint32_t w[32];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const uint4 x = row < a.L ? src[c * 8 + u] : make_uint4(0u, 0u, 0u, 0u);
          w[4 * u] = x.x;
          w[4 * u + 1] = x.y;
          w[4 * u + 2] = x.z;
          w[4 * u + 3] = x.w;
        }
        tmem_st32(lane_base + col + c * 32, w);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(qa_ready);
    }
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const uint32_t sb = j & 1;
      ok = mbar_wait(sdp_full + sb, (j >> 1) & 1, a.status, kStatusTimeoutMma, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const int64_t k0 = static_cast<int64_t>(j) * BK;
      const int64_t vis = a.causal ? (row + 1 < a.S ? row + 1 : a.S) : a.S;
      const int64_t lim64 = row_live ? vis - k0 : 0;
      const int lim = static_cast<int>(lim64 < 0 ? 0 : (lim64 > BK ? BK : lim64));
      const bool all_vis = __all_sync(0xffffffffu, lim == BK);
      {
        uint32_t sr[32], pr[32];
        tmem_ld32(lane_base + C::kColS + sb * 64 + half * 32, sr);
        tmem_ld32(lane_base + C::kColP + sb * 64 + half * 32, pr);
        tmem_ld_wait();
        reg_fence(sr);
        reg_fence(pr);
        uint32_t dk[16];
        const uint64_t sl2x2 = f2(a.scale_log2, a.scale_log2), nlz = f2(-lz, -lz), ndl = f2(-dlt, -dlt);
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const int c = half * 32 + 2 * t;
          // p = 2^(s * scale - lse), dS = p * (dP - delta), two columns at a time
          const uint64_t y = fma2(f2(__uint_as_float(sr[2 * t]), __uint_as_float(sr[2 * t + 1])), sl2x2, nlz);
          const uint64_t p2 = f2(ex2(f2_lo(y)), ex2(f2_hi(y)));
          const uint64_t d2 = mul2(p2, add2(f2(__uint_as_float(pr[2 * t]), __uint_as_float(pr[2 * t + 1])), ndl));
          float d0 = f2_lo(d2), d1 = f2_hi(d2);
          if (!all_vis) {
            if (c >= lim) d0 = 0.f;
            if (c + 1 >= lim) d1 = 0.f;
          }
          dk[t] = pack2(d0, d1, BF16);
        }
        tmem_st16(lane_base + C::kColP + sb * 64 + half * 16, dk);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(ds_ready + sb);
    }
    if (ok && n > 0) {
      ok = mbar_wait(acc_done, 0, a.status, kStatusTimeoutMma, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      uint8_t* dqrow = static_cast<uint8_t*>(a.dq) + ((zq * a.L + row) * D) * 2;
#pragma unroll
      for (int c = half * (D / 64); c < (half + 1) * (D / 64); ++c) {
        uint32_t rq[32];
        if (n > 0) {
          tmem_ld32(lane_base + C::kColQ + c * 32, rq);
          tmem_ld_wait();
          reg_fence(rq);
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) rq[t] = 0u;
        }
        if (row < a.L && a.dq_acc) accum_row32(a.dq_acc + (zq * a.L + row) * D + c * 32, rq, a.scale);
        else if (row < a.L) store_row32<BF16>(dqrow + c * 64, rq, a.scale);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, bool BF16>
pa_status launch_bwd_tc(const pa_sdpa_desc& d, int64_t n, int64_t H, int64_t Hkv, const void* q,
                        const void* k, const void* v, const void* o, const void* dout,
                        const float* lse, void* dq, void* dk, void* dv, cudaStream_t st,
                        float* dq_acc = nullptr, float* dk_acc = nullptr, float* dv_acc = nullptr,
                        const std::function<void()>* before_dkdv = nullptr) {
  const int64_t L = d.L, S = d.S;
  const int64_t Lp = (L + kRowPad - 1) / kRowPad * kRowPad;
  const int64_t nkv = (n / H) * Hkv;
  float* ws = nullptr;
  const size_t ws_floats = 2 * static_cast<size_t>(n * Lp) + 2 * kRowPad;
  PA_TRY(scratch_alloc(reinterpret_cast<void**>(&ws), ws_floats * sizeof(float), st));
  float* delta = ws;
  float* lse2 = ws + n * Lp + kRowPad;
  pa_status rc = PA_OK;
  do {
    const int64_t rows = n * Lp;
    const int64_t threads = rows * 32;
    bwd_prep_kernel<D, BF16><<<static_cast<unsigned>((threads + 255) / 256), 256, 0, st>>>(
        o, dout, lse, delta, lse2, n, L, Lp);
    if (cudaGetLastError() != cudaSuccess) {
      rc = fail(PA_ERR_CUDA, "bwd_prep launch failed");
      break;
    }
    const CUtensorMapDataType tdt = BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint64_t rowb = D * 2;
    CUtensorMap tq64, tdo64, tk128, tv128, tk64, tv64;
    rc = encode_tma_3d(&tq64, tdt, q, D, L, n, rowb, rowb * L, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc == PA_OK) rc = encode_tma_3d(&tdo64, tdt, dout, D, L, n, rowb, rowb * L, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc == PA_OK) rc = encode_tma_3d(&tk128, tdt, k, D, S, nkv, rowb, rowb * S, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc == PA_OK) rc = encode_tma_3d(&tv128, tdt, v, D, S, nkv, rowb, rowb * S, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc == PA_OK) rc = encode_tma_3d(&tk64, tdt, k, D, S, nkv, rowb, rowb * S, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc == PA_OK) rc = encode_tma_3d(&tv64, tdt, v, D, S, nkv, rowb, rowb * S, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != PA_OK) break;
    BwdArgs a{};
    a.dk = dk;
    a.dv = dv;
    a.dq = dq;
    a.dk_acc = dk_acc;
    a.dv_acc = dv_acc;
    a.dq_acc = dq_acc;
    a.q = q;
    a.dout = dout;
    a.lse2 = lse2;
    a.delta = delta;
    a.status = device_status_word();
    if (!a.status) {
      rc = fail(PA_ERR_CUDA, "device status word unavailable");
      break;
    }
    a.L = L;
    a.S = S;
    a.Lp = Lp;
    a.Hq = static_cast<int32_t>(H);
    a.Hkv = static_cast<int32_t>(Hkv);
    a.group = static_cast<int32_t>(H / Hkv);
    a.causal = d.is_causal;
    a.scale_log2 = static_cast<float>(d.scale * 1.4426950408889634);
    a.scale = static_cast<float>(d.scale);
    auto run_dkdv = [&]() -> pa_status {
      using C = DkdvCfg<D>;
      BwdArgs b = a;
      b.slices = nkv;
      b.blocks = static_cast<int32_t>((S + C::BK - 1) / C::BK);
      const int64_t grid = nkv * b.blocks;
      auto kern = bwd_dkdv_kernel<D, BF16>;
      static uint64_t attr_set = 0;
      PA_TRY(set_smem_attr_once(reinterpret_cast<const void*>(kern), C::kSmemBytes, &attr_set));
      if (grid > 0) kern<<<static_cast<unsigned>(grid), kThreadsB, C::kSmemBytes, st>>>(tq64, tdo64, tk128, tv128, b);
      if (cudaGetLastError() != cudaSuccess) return fail(PA_ERR_CUDA, "bwd_dkdv launch failed");
      return PA_OK;
    };
    auto run_dq = [&]() -> pa_status {
      using C = DqCfg<D>;
      BwdArgs b = a;
      b.slices = n;
      b.blocks = static_cast<int32_t>((L + C::BQ - 1) / C::BQ);
      const int64_t grid = n * b.blocks;
      auto kern = bwd_dq_kernel<D, BF16>;
      static uint64_t attr_set = 0;
      PA_TRY(set_smem_attr_once(reinterpret_cast<const void*>(kern), C::kSmemBytes, &attr_set));
      if (grid > 0) kern<<<static_cast<unsigned>(grid), kThreadsB, C::kSmemBytes, st>>>(tk64, tv64, b);
      if (cudaGetLastError() != cudaSuccess) return fail(PA_ERR_CUDA, "bwd_dq launch failed");
      return PA_OK;
    };
    if (before_dkdv) {
      // Accumulating into buffers that may still be arriving: dQ first (its
      // accumulator is the caller's own), then whatever the caller must wait for,
      // then dK/dV.
      if ((rc = run_dq()) != PA_OK) break;
      if (*before_dkdv) (*before_dkdv)();
      rc = run_dkdv();
    } else {
      if ((rc = run_dkdv()) != PA_OK) break;
      rc = run_dq();
    }
  } while (false);
  scratch_free(ws, st);
  return rc;
}

}  // namespace

pa_status bwd_accumulate(const pa_sdpa_desc& d, const void* q, const void* k, const void* v,
                         const void* out, const void* dout, const float* lse, float* dq_acc,
                         float* dk_acc, float* dv_acc, cudaStream_t st,
                         const std::function<void()>& before_dkdv) {
  std::string why;
  if (d.mask_kind != PA_MASK_NONE || !fwd_tc_eligible(d, &why))
    return fail(PA_ERR_UNSUPPORTED, "backward accumulate: dense fp16/bf16 (B, H, L, D), D in {64, 128}, no mask");
  if (!dq_acc || !dk_acc || !dv_acc) return fail(PA_ERR_INVALID, "backward accumulate: null accumulator");
  int64_t n, H, Hkv;
  dense_bhsd(d, &n, &H, &Hkv);
  if (n == 0 || d.L == 0 || d.S == 0) return PA_OK;  // nothing to add
  const bool bf16 = d.dtype == PA_BF16;
  if (d.E == 128)
    return bf16 ? launch_bwd_tc<128, true>(d, n, H, Hkv, q, k, v, out, dout, lse, nullptr, nullptr, nullptr, st,
                                           dq_acc, dk_acc, dv_acc, &before_dkdv)
                : launch_bwd_tc<128, false>(d, n, H, Hkv, q, k, v, out, dout, lse, nullptr, nullptr, nullptr, st,
                                            dq_acc, dk_acc, dv_acc, &before_dkdv);
  return bf16 ? launch_bwd_tc<64, true>(d, n, H, Hkv, q, k, v, out, dout, lse, nullptr, nullptr, nullptr, st,
                                        dq_acc, dk_acc, dv_acc, &before_dkdv)
              : launch_bwd_tc<64, false>(d, n, H, Hkv, q, k, v, out, dout, lse, nullptr, nullptr, nullptr, st,
                                         dq_acc, dk_acc, dv_acc, &before_dkdv);
}

}  // namespace pa

using namespace pa;

extern "C" pa_status pa_sdpa_bwd(const pa_sdpa_desc* desc, const void* q, const void* k,
                                 const void* v, const void* out, const void* dout,
                                 const float* lse, void* dq, void* dk, void* dv, void* stream) {
  clear_error();
  PA_TRY(check_desc(desc));
  const pa_sdpa_desc& d = *desc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (d.mask_kind != PA_MASK_NONE)
    return fail(PA_ERR_UNSUPPORTED, "pa_sdpa_bwd: attn_mask is not supported by the backward yet");
  std::string why;
  if (!fwd_tc_eligible(d, &why))
    return fail(PA_ERR_UNSUPPORTED, "pa_sdpa_bwd needs dense fp16/bf16 (B, H, L, D) with D in {64, 128}: " + why);
  int64_t n, H, Hkv;
  dense_bhsd(d, &n, &H, &Hkv);
  if (n == 0 || (d.L == 0 && d.S == 0)) return PA_OK;
  if (d.S == 0 || d.L == 0) {
    // No keys: every gradient is zero; no rows: dK and dV are zero.
    const size_t es = 2;
    if (d.L) PA_CUDA(cudaMemsetAsync(dq, 0, static_cast<size_t>(n * d.L * d.E) * es, st));
    if (d.S) {
      const size_t kv = static_cast<size_t>((n / H) * Hkv * d.S * d.E) * es;
      PA_CUDA(cudaMemsetAsync(dk, 0, kv, st));
      PA_CUDA(cudaMemsetAsync(dv, 0, kv, st));
    }
    return PA_OK;
  }
  const bool bf16 = d.dtype == PA_BF16;
  if (d.E == 128)
    return bf16 ? launch_bwd_tc<128, true>(d, n, H, Hkv, q, k, v, out, dout, lse, dq, dk, dv, st)
                : launch_bwd_tc<128, false>(d, n, H, Hkv, q, k, v, out, dout, lse, dq, dk, dv, st);
  return bf16 ? launch_bwd_tc<64, true>(d, n, H, Hkv, q, k, v, out, dout, lse, dq, dk, dv, st)
              : launch_bwd_tc<64, false>(d, n, H, Hkv, q, k, v, out, dout, lse, dq, dk, dv, st);
}
