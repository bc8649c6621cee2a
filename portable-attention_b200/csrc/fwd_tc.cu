// Tensor-core SDPA forward for sm_100a: TMA-fed tiles, tcgen05.mma into
// TMEM, online softmax in fp32 with one query row per thread.
//
// CTA = two 128-row query tiles (256 rows) of one (batch, head), 384 threads:
//   warps 0-3   softmax of query tile 0; warps 4-7 softmax of tile 1. Thread
//               <-> TMEM lane <-> query row (warp w reaches lanes 32*(w%4)..).
//   warp 8      TMA producer: both Q tiles once, then 128-key K/V tiles into a
//               ring of shared-memory stages (128-byte swizzle, 64-col boxes).
//   warp 9      owns TMEM (512 columns) and issues the MMAs from one lane:
//                 S_t = Q_t K^T  (SS form, M=128 N=128 K=D)      -> S[t]
//                 O_t += P_t V   (TS form, P_t read from TMEM)    -> O[t]
//               in the order S0(i), PV1(i-1), S1(i), PV0(i), so one tile's
//               softmax overlaps the other tile's tensor-core work.
//   warps 10-11 complete the third warpgroup (registers are allocated per
//               warpgroup) and have no work.
// TMEM columns: S0 [0,128), S1 [128,256), O0 [256,256+D), O1 after.
//
// Softmax per key tile: the row max is taken on raw scores (scale > 0) with
// three-input maxima, each pair of probabilities costs one packed f32x2 FMA,
// two ex2 and one packed add, partial max/sum chains are split for ILP, and
// P is packed to fp16/bf16 into the first 64 columns
// of its S buffer (aliasing S). The running max moves only when it grows by
// more than 2^8 (log2 units), so O is rescaled rarely. Fully-masked rows keep
// l = 0 and produce exact zeros and lse = -inf.
//
// Key tiles are classified per query tile: dead (causally invisible, or a
// boolean-mask tile with no kept element: no MMA, no softmax), full (no
// per-element work) or partial (diagonal, ragged key edge, mixed mask tile:
// per-element masking, 16-byte vector mask loads when the mask row allows).
// Boolean-mask tile classes come from a pre-pass over the mask.
//
// Semantics follow src/portable_attention/reference.py:139-162 (top-left
// causal, keep-masks, additive masks, dead rows exactly zero). Every wait is
// bounded; a wait that gives up records a status code and the CTA drains its
// copies and MMAs before freeing TMEM.
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace pa {
namespace {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int kTiles = 2;
constexpr int kSoftWarps = 4 * kTiles;
constexpr int kProducerWarp = kSoftWarps;
constexpr int kMmaWarp = kSoftWarps + 1;
// Warpgroup 2 holds the producer (warp 8) and MMA (warp 9) warps and two
// idle warps: registers are allocated per warpgroup, so a 10-warp CTA would
// pay for 12 anyway, and whole warpgroups can move registers with setmaxnreg.
constexpr int kThreads = 32 * 12;
// Register split (setmaxnreg): the softmax warpgroups keep a 128-column score
// row per thread; the producer/MMA warpgroup needs few. 128 x (2 x 200 + 80)
// = 61440 registers, at most the 384 x 160 a launch of >= 160 registers per
// thread provides (checked on the host before the first launch).
constexpr int kRegsSoft = 200;
constexpr int kRegsOther = 80;
constexpr uint32_t kTmemCols = 512;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleSlack = 8.0f;

template <int D>
struct TcCfg {
  static constexpr int kBoxes = D / 64;
  static constexpr int kQBytes = BM * D * 2;
  static constexpr int kTileBytes = BN * D * 2;
  // V of key tile i stays in use until tile 1's PV, issued one iteration
  // later than tile 0's, so V gets one more stage than K.
  static constexpr int kKStages = (D == 128) ? 2 : 3;
  static constexpr int kVStages = (D == 128) ? 3 : 4;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kTiles * kQBytes;
  static constexpr int kVOff = kKOff + kKStages * kTileBytes;
  static constexpr int kBarOff = kVOff + kVStages * kTileBytes;
  static constexpr int kNumBars = 1 + 2 * kKStages + 2 * kVStages + 3 * kTiles + 2;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kMiscOff + 16 + 1024;
  static constexpr uint32_t col_s(int t) { return 128u * t; }
  static constexpr uint32_t col_o(int t) { return 256u + D * t; }
};

struct TcArgs {
  void* out;
  float* lse;
  const void* mask;
  const uint8_t* mcls;  // boolean-mask tile classes [mslice][row_tile][col_block] or null
  int* status;
  LeadTable mlt;        // mask element offsets per output slice
  int64_t L, S;
  int64_t m_rs, m_cs;
  int64_t slices, items;
  int32_t H, Hkv, group, pairs;
  int32_t row_tiles, col_blocks;
  int32_t causal;
  float scale_log2, inv_scale;
};

// Index of the mask slice an output slice reads (only non-broadcast dims count).
__host__ __device__ inline int64_t mask_slice_id(const LeadTable& t, int64_t slice) {
  int64_t id = 0, rem = slice, suffix = 1;
  for (int i = 0; i < t.n; ++i) suffix *= t.dim[i];
  for (int i = 0; i < t.n; ++i) {
    suffix /= t.dim[i];
    const int64_t idx = rem / suffix;
    rem %= suffix;
    if (t.ms[i] != 0) id = id * t.dim[i] + idx;
  }
  return id;
}

__host__ __device__ inline int64_t mask_slice_count(const LeadTable& t) {
  int64_t n = 1;
  for (int i = 0; i < t.n; ++i)
    if (t.ms[i] != 0) n *= t.dim[i];
  return n;
}

template <typename MaskT>
__device__ __forceinline__ float mask_value(const MaskT* p) { return static_cast<float>(*p); }
template <>
__device__ __forceinline__ float mask_value<__half>(const __half* p) { return __half2float(*p); }
template <>
__device__ __forceinline__ float mask_value<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

// Classify each (mask slice, 128-row tile, 128-key tile) of a boolean mask:
// 0 = no element kept, 1 = every in-range element kept, 2 = mixed.
__global__ void mask_classify_kernel(const uint8_t* mask, LeadTable mlt, int64_t L, int64_t S,
                                     int64_t m_rs, int64_t m_cs, int32_t row_tiles,
                                     int32_t col_blocks, uint8_t* cls) {
  const int64_t tile = blockIdx.x;
  const int cb = static_cast<int>(tile % col_blocks);
  const int rt = static_cast<int>((tile / col_blocks) % row_tiles);
  const int64_t ms = tile / (static_cast<int64_t>(col_blocks) * row_tiles);
  // element offset of mask slice `ms`
  int64_t off = 0, rem = ms;
  for (int i = mlt.n - 1; i >= 0; --i) {
    if (mlt.ms[i] == 0) continue;
    off += (rem % mlt.dim[i]) * mlt.ms[i];
    rem /= mlt.dim[i];
  }
  int any = 0, all = 1;
  const int64_t r0 = static_cast<int64_t>(rt) * BM, c0 = static_cast<int64_t>(cb) * BN;
  const bool vec = m_cs == 1 && c0 + BN <= S && ((off + c0) & 15) == 0 && (m_rs & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(mask) & 15) == 0;
  if (vec) {
    // 16 bytes per load; a word has a zero byte iff (w - 0x01..) & ~w & 0x80.. != 0.
    for (int e = threadIdx.x; e < BM * (BN / 16); e += blockDim.x) {
      const int64_t r = r0 + e / (BN / 16);
      if (r >= L) continue;
      const uint4 w = *reinterpret_cast<const uint4*>(mask + off + r * m_rs + c0 + (e % (BN / 16)) * 16);
      const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        any |= wd[k] != 0u;
        all &= ((wd[k] - 0x01010101u) & ~wd[k] & 0x80808080u) == 0u;
      }
    }
  } else {
    for (int e = threadIdx.x; e < BM * BN; e += blockDim.x) {
      const int64_t r = r0 + e / BN, c = c0 + e % BN;
      if (r < L && c < S) {
        const int keep = mask[off + r * m_rs + c * m_cs] != 0;
        any |= keep;
        all &= keep;
      }
    }
  }
  any = __syncthreads_or(any);
  all = __syncthreads_and(all);
  if (threadIdx.x == 0) cls[tile] = any ? (all ? 1 : 2) : 0;
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
  uint64_t* k_empty = k_full + C::kKStages;
  uint64_t* v_full = k_empty + C::kKStages;
  uint64_t* v_empty = v_full + C::kVStages;
  uint64_t* s_full = v_empty + C::kVStages;  // [kTiles]
  uint64_t* p_full = s_full + kTiles;       // [kTiles]
  uint64_t* o_done = p_full + kTiles;       // [kTiles]
  uint64_t* mma_done = o_done + kTiles;
  uint64_t* q_empty = mma_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMiscOff + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Persistent CTAs. A work item is (query-tile pair, slice); items are
  // ordered heaviest pair first (under causal masking a pair's cost grows with
  // its row index), then by slice, so the items running together share K/V
  // under GQA. Round k of CTA c takes item k * grid + c for even k and
  // k * grid + (grid - 1 - c) for odd k: this snake order evens out the CTAs'
  // total work (the plain stride left the busiest CTA ~8 % above the mean on
  // the causal prefill).
  int64_t slice = 0, m0 = 0;
  int32_t zq = 0, zkv = 0;
  int n_blocks = 0;
  const uint8_t* cls_row[kTiles] = {nullptr, nullptr};
  auto item_of = [&](int64_t k) -> int64_t {
    const int64_t g = gridDim.x;
    const int64_t item = k * g + ((k & 1) ? (g - 1 - blockIdx.x) : blockIdx.x);
    return item < a.items ? item : -1;
  };
  auto set_item = [&](int64_t item) {
    const int pair = a.pairs - 1 - static_cast<int>(item / a.slices);
    slice = item % a.slices;
    m0 = static_cast<int64_t>(pair) * (kTiles * BM);
    zq = static_cast<int32_t>(slice);
    zkv = static_cast<int32_t>((slice / a.H) * a.Hkv + (slice % a.H) / a.group);
    const int64_t last_row = (m0 + kTiles * BM < a.L ? m0 + kTiles * BM : a.L) - 1;
    int64_t kv_end = a.S;
    if (a.causal) kv_end = last_row + 1 < a.S ? last_row + 1 : a.S;
    n_blocks = static_cast<int>((kv_end + BN - 1) / BN);
    cls_row[0] = cls_row[1] = nullptr;
    if (MASK == PA_MASK_BOOL && a.mcls) {
      const int64_t ms = mask_slice_id(a.mlt, slice);
#pragma unroll
      for (int t = 0; t < kTiles; ++t) {
        const int64_t rt = (m0 / BM) + t;
        cls_row[t] = rt < a.row_tiles ? a.mcls + (ms * a.row_tiles + rt) * a.col_blocks : nullptr;
      }
    }
  };
  // 0 dead, 1 full, 2 partial -- identical in every role.
  auto tile_class = [&](int t, int j) -> int {
    const int64_t r_lo = m0 + static_cast<int64_t>(t) * BM;
    if (r_lo >= a.L) return 0;
    const int64_t r_hi = (r_lo + BM - 1 < a.L) ? r_lo + BM - 1 : a.L - 1;
    const int64_t n0 = static_cast<int64_t>(j) * BN;
    int c = 1;
    if (a.causal) {
      if (n0 > r_hi) return 0;
      if (n0 + BN - 1 > r_lo) c = 2;
    }
    if (n0 + BN > a.S) c = 2;
    if (MASK == PA_MASK_ADD) c = 2;
    if (MASK == PA_MASK_BOOL) {
      const int mc = cls_row[t] ? cls_row[t][j] : 2;
      if (mc == 0) return 0;
      if (mc == 2) c = 2;
    }
    return c;
  };
  auto block_live = [&](int j) -> bool { return tile_class(0, j) != 0 || tile_class(1, j) != 0; };
  auto last_live = [&]() -> int {
    for (int j = n_blocks - 1; j >= 0; --j)
      if (block_live(j)) return j;
    return -1;
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::kKStages; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(k_empty + s, 1);
    }
    for (int s = 0; s < C::kVStages; ++s) {
      mbar_init(v_full + s, 1);
      mbar_init(v_empty + s, 1);
    }
    for (int t = 0; t < kTiles; ++t) {
      mbar_init(s_full + t, 1);
      mbar_init(p_full + t, 128);
      mbar_init(o_done + t, 1);
    }
    mbar_init(mma_done, 1);
    mbar_init(q_empty, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp >= kSoftWarps) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsOther));
  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      int last_k[C::kKStages], last_v[C::kVStages];
#pragma unroll
      for (int s = 0; s < C::kKStages; ++s) last_k[s] = -1;
#pragma unroll
      for (int s = 0; s < C::kVStages; ++s) last_v[s] = -1;
      int it = 0, g = 0;
      bool ok = true;
      for (int64_t k = 0; ok; ++k) {
        const int64_t item = item_of(k);
        if (item < 0) break;
        set_item(item);
        if (last_live() < 0) continue;
        // Q of this item may overwrite the previous one once its S MMAs are done.
        if (!mbar_wait(q_empty, (it & 1) ^ 1, a.status, kStatusTimeoutFree, abort_flag)) break;
        mbar_expect_tx(q_full, kTiles * C::kQBytes);
        for (int t = 0; t < kTiles; ++t)
          for (int b = 0; b < C::kBoxes; ++b)
            tma_load_3d(sQ + t * C::kQBytes + b * (BM * 128), &tq, q_full, b * 64,
                        static_cast<int32_t>(m0 + t * BM), zq);
        ++it;
        for (int j = 0; j < n_blocks; ++j) {
          if (!block_live(j)) continue;
          const int ks = g % C::kKStages, vs = g % C::kVStages;
          if (!mbar_wait(k_empty + ks, ((g / C::kKStages) & 1) ^ 1, a.status, kStatusTimeoutFree, abort_flag)) {
            ok = false;
            break;
          }
          mbar_expect_tx(k_full + ks, C::kTileBytes);
          for (int b = 0; b < C::kBoxes; ++b)
            tma_load_3d(sK + ks * C::kTileBytes + b * (BN * 128), &tk, k_full + ks, b * 64, j * BN, zkv);
          last_k[ks] = g;
          if (!mbar_wait(v_empty + vs, ((g / C::kVStages) & 1) ^ 1, a.status, kStatusTimeoutFree, abort_flag)) {
            ok = false;
            break;
          }
          mbar_expect_tx(v_full + vs, C::kTileBytes);
          for (int b = 0; b < C::kBoxes; ++b)
            tma_load_3d(sV + vs * C::kTileBytes + b * (BN * 128), &tv, v_full + vs, b * 64, j * BN, zkv);
          last_v[vs] = g;
          ++g;
        }
      }
      if (it > 0) mbar_drain(q_full, (it - 1) & 1);
#pragma unroll
      for (int s = 0; s < C::kKStages; ++s)
        if (last_k[s] >= 0) mbar_drain(k_full + s, (last_k[s] / C::kKStages) & 1);
#pragma unroll
      for (int s = 0; s < C::kVStages; ++s)
        if (last_v[s] >= 0) mbar_drain(v_full + s, (last_v[s] / C::kVStages) & 1);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------- MMA issue
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16(BM, BN, false, false, BF16);
      constexpr uint32_t idO = idesc_f16(BM, D, false, true, BF16);
      const uint32_t q_addr = smem_u32(sQ);
      int pv_cnt[kTiles] = {0, 0};   // PVs issued per tile over the CTA's life
      bool first_pv[kTiles] = {true, true};
      auto issue_s = [&](int t, int st) {
        const uint32_t k_addr = smem_u32(sK + st * C::kTileBytes);
        const uint32_t qa = q_addr + t * C::kQBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t box = kk / 4, sub = (kk % 4) * 32;
          umma_ss(tmem + C::col_s(t), sdesc_sw128(qa + box * (BM * 128) + sub, 16, 1024),
                  sdesc_sw128(k_addr + box * (BN * 128) + sub, 16, 1024), idS, kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full + t);
      };
      auto issue_pv = [&](int t, int gi, bool release_v) -> bool {
        const int st = gi % C::kVStages;
        if (!mbar_wait(p_full + t, pv_cnt[t] & 1, a.status, kStatusTimeoutSoftmax, abort_flag)) return false;
        if (!mbar_wait(v_full + st, (gi / C::kVStages) & 1, a.status, kStatusTimeoutLoad, abort_flag)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + st * C::kTileBytes);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          umma_ts(tmem + C::col_o(t), tmem + C::col_s(t) + kk * 8,
                  sdesc_sw128(v_addr + kk * 2048, BN * 128, 1024), idO,
                  (!first_pv[t] || kk > 0) ? 1u : 0u);
        tc_commit(o_done + t);
        if (release_v) tc_commit(v_empty + st);
        ++pv_cnt[t];
        first_pv[t] = false;
        return true;
      };
      int it = 0, g = 0;
      bool ok = true;
      for (int64_t k = 0; ok; ++k) {
        const int64_t item = item_of(k);
        if (item < 0) break;
        set_item(item);
        const int jl = last_live();
        if (jl < 0) continue;
        if (!mbar_wait(q_full, it & 1, a.status, kStatusTimeoutLoad, abort_flag)) {
          ok = false;
          break;
        }
        ++it;
        first_pv[0] = first_pv[1] = true;
        int pend1 = -1;  // global index of tile 1's S awaiting its PV
        for (int j = 0; j <= jl; ++j) {
          if (!block_live(j)) continue;
          const int st = g % C::kKStages;
          const bool live0 = tile_class(0, j) != 0, live1 = tile_class(1, j) != 0;
          if (!mbar_wait(k_full + st, (g / C::kKStages) & 1, a.status, kStatusTimeoutLoad, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (live0) issue_s(0, st);
          if (pend1 >= 0) {
            // tile 1's previous block; its V stage is released here
            if (!issue_pv(1, pend1, true)) {
              ok = false;
              break;
            }
            pend1 = -1;
          }
          if (live1) {
            issue_s(1, st);
            pend1 = g;
          }
          // Every S of this item is issued: its Q tiles may be replaced once they finish.
          if (j == jl) tc_commit(q_empty);
          tc_commit(k_empty + st);
          if (live0 && !issue_pv(0, g, !live1)) {
            ok = false;
            break;
          }
          ++g;
        }
        if (ok && pend1 >= 0) ok = issue_pv(1, pend1, true);
      }
      tc_commit(mma_done);
      mbar_drain(mma_done, 0);
    }
    __syncwarp();
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoft));
    // --------------------------------------------------------------- softmax
    const int t = warp / 4;                 // query tile of this warpgroup
    const int quad = warp & 3;
    const int r = quad * 32 + lane;         // row inside the tile == TMEM lane
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t s_addr = lane_base + C::col_s(t);
    const uint32_t o_addr = lane_base + C::col_o(t);
    const float sl2 = a.scale_log2;
    int cnt = 0;  // softmax blocks of this tile over the CTA's life (barrier phases)
    bool ok = true;
    for (int64_t k = 0; ok; ++k) {
    const int64_t item = item_of(k);
    if (item < 0) break;
    set_item(item);
    const int64_t row = m0 + static_cast<int64_t>(t) * BM + r;
    const bool row_ok = row < a.L;
    float m_run = -INFINITY, l_run = 0.f;
    const SliceOffsets moff = slice_offsets(a.mlt, slice);
    int icnt = 0;   // blocks of this item

    for (int j = 0; j < n_blocks; ++j) {
      const int cls = tile_class(t, j);
      if (cls == 0) continue;
      ok = mbar_wait(s_full + t, cnt & 1, a.status, kStatusTimeoutMma, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      float x[BN];
      {
        uint32_t rr[BN / 32][32];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_ld32(s_addr + c * 32, rr[c]);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          reg_fence(rr[c]);
#pragma unroll
          for (int u = 0; u < 32; ++u) x[c * 32 + u] = __uint_as_float(rr[c][u]);
        }
      }
      const int64_t n0 = static_cast<int64_t>(j) * BN;
      if (cls == 2) {
        const int64_t vis = a.causal ? (row + 1 < a.S ? row + 1 : a.S) : a.S;
        const int lim = static_cast<int>(vis - n0 < 0 ? 0 : (vis - n0 > BN ? BN : vis - n0));
#pragma unroll
        for (int u = 0; u < BN; ++u)
          if (u >= lim) x[u] = -INFINITY;
        if (MASK != PA_MASK_NONE && row_ok) {
          const int64_t base = moff.m + row * a.m_rs + n0 * a.m_cs;
          if (MASK == PA_MASK_BOOL) {
            const uint8_t* mp = static_cast<const uint8_t*>(a.mask) + base;
            if (a.m_cs == 1 && n0 + BN <= a.S && (reinterpret_cast<uintptr_t>(mp) & 15) == 0) {
#pragma unroll
              for (int v = 0; v < BN / 16; ++v) {
                const uint4 w = reinterpret_cast<const uint4*>(mp)[v];
                const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int b = 0; b < 16; ++b)
                  if (((wd[b >> 2] >> (8 * (b & 3))) & 0xffu) == 0u) x[v * 16 + b] = -INFINITY;
              }
            } else {
#pragma unroll
              for (int u = 0; u < BN; ++u)
                if (u < lim && mp[u * a.m_cs] == 0) x[u] = -INFINITY;
            }
          } else {
            const MaskT* mp = static_cast<const MaskT*>(a.mask) + base;
#pragma unroll
            for (int u = 0; u < BN; ++u)
              if (u < lim) x[u] = fmaf(mask_value(mp + u * a.m_cs), a.inv_scale, x[u]);
          }
        }
      }
      // Row max of raw scores (scale > 0): eight chains of three-input maxima.
      float mx8[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mx8[u] = fmaxf(x[2 * u], x[2 * u + 1]);
#pragma unroll
      for (int u = 16; u < BN; u += 2) mx8[(u >> 1) & 7] = max3(mx8[(u >> 1) & 7], x[u], x[u + 1]);
      const float mx = max3(max3(mx8[0], mx8[1], mx8[2]), max3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])) * sl2;
      const float m_new = fmaxf(m_run, mx);
      const float m_use = (m_run == -INFINITY || m_new - m_run > kRescaleSlack) ? m_new : m_run;
      const float neg_m = m_use == -INFINITY ? 0.f : -m_use;
      // p = 2^(x * scale - m), two columns per packed FMA and packed add.
      const uint64_t sl2x2 = f2(sl2, sl2), negm2 = f2(neg_m, neg_m);
      uint64_t sum4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) sum4[u] = 0ull;
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const uint64_t y = fma2(f2(x[c * 32 + 2 * u], x[c * 32 + 2 * u + 1]), sl2x2, negm2);
          const float p0 = ex2(f2_lo(y));
          const float p1 = ex2(f2_hi(y));
          sum4[u & 3] = add2(sum4[u & 3], f2(p0, p1));
          pk[u] = pack2(p0, p1, BF16);
        }
        tmem_st16(s_addr + c * 16, pk);
      }
      tmem_st_wait();
      const uint64_t s2 = add2(add2(sum4[0], sum4[1]), add2(sum4[2], sum4[3]));
      const float rowsum = f2_lo(s2) + f2_hi(s2);
      const float alpha = (m_use == m_run) ? 1.f : ((m_run == -INFINITY) ? 0.f : ex2(m_run - m_use));
      const bool need = (icnt > 0) && (m_use != m_run);
      if (__any_sync(0xffffffffu, need)) {
        ok = mbar_wait(o_done + t, (cnt - 1) & 1, a.status, kStatusTimeoutMma, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t rr[32];
          tmem_ld32(o_addr + c * 32, rr);
          tmem_ld_wait();
          reg_fence(rr);
          const uint64_t al2 = f2(alpha, alpha);
#pragma unroll
          for (int u = 0; u < 16; ++u) {
            const uint64_t y = mul2(f2(__uint_as_float(rr[2 * u]), __uint_as_float(rr[2 * u + 1])), al2);
            rr[2 * u] = __float_as_uint(f2_lo(y));
            rr[2 * u + 1] = __float_as_uint(f2_hi(y));
          }
          tmem_st32(o_addr + c * 32, rr);
        }
        tmem_st_wait();
      }
      l_run = l_run * alpha + rowsum;
      m_run = m_use;
      tc_fence_before();
      mbar_arrive(p_full + t);
      ++cnt;
      ++icnt;
    }

    if (ok && icnt > 0) {
      ok = mbar_wait(o_done + t, (cnt - 1) & 1, a.status, kStatusTimeoutMma, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      uint8_t* orow = static_cast<uint8_t*>(a.out) + ((slice * a.L + row) * D) * 2;
      // All of the row's O columns in one batch of TMEM loads, one wait.
      uint32_t rr[D / 32][32];
      if (icnt > 0) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) tmem_ld32(o_addr + c * 32, rr[c]);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) reg_fence(rr[c]);
      } else {
#pragma unroll
        for (int c = 0; c < D / 32; ++c)
#pragma unroll
          for (int u = 0; u < 32; ++u) rr[c][u] = 0u;
      }
      const uint64_t inv2 = f2(inv, inv);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const uint64_t y = mul2(f2(__uint_as_float(rr[c][2 * u]), __uint_as_float(rr[c][2 * u + 1])), inv2);
          pk[u] = pack2(f2_lo(y), f2_hi(y), BF16);
        }
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 64);
#pragma unroll
          for (int u = 0; u < 4; ++u) dst[u] = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
      }
      if (row_ok && a.lse)
        a.lse[slice * a.L + row] = l_run > 0.f ? (m_run + __log2f(l_run)) * kLn2 : -INFINITY;
    }
      }  // item loop
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D, bool BF16, int MASK, typename MaskT>
pa_status launch_variant(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                         const TcArgs& a, int64_t grid, cudaStream_t st) {
  auto kern = fwd_tc_kernel<D, BF16, MASK, MaskT>;
  constexpr int smem = TcCfg<D>::kSmemBytes;
  static uint64_t attr_set = 0;  // one bit per device
  PA_TRY(set_smem_attr_once(reinterpret_cast<const void*>(kern), smem, &attr_set));
  // setmaxnreg.inc waits until the pool of registers the CTA was launched
  // with can cover the request: never launch a build whose per-thread count
  // is too small for the split (it would wait forever).
  static int regs = 0;
  if (regs == 0) {
    cudaFuncAttributes fa{};
    PA_CUDA(cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(kern)));
    regs = fa.numRegs;
  }
  if (regs * kThreads < 128 * (2 * kRegsSoft + kRegsOther))
    return fail(PA_ERR_UNSUPPORTED, "fwd_tc: kernel built with too few registers for its register split");
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
  if (!(d.scale > 0)) return no("scale must be positive");
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
  a.slices = n;
  a.H = static_cast<int32_t>(H);
  a.Hkv = static_cast<int32_t>(Hkv);
  a.group = static_cast<int32_t>(H / Hkv);
  a.pairs = static_cast<int32_t>((d.L + kTiles * BM - 1) / (kTiles * BM));
  a.row_tiles = static_cast<int32_t>((d.L + BM - 1) / BM);
  a.col_blocks = static_cast<int32_t>((d.S + BN - 1) / BN);
  a.causal = d.is_causal;
  a.scale_log2 = static_cast<float>(d.scale * 1.4426950408889634);
  a.inv_scale = static_cast<float>(1.0 / d.scale);
  a.items = n * a.pairs;
  if (a.items == 0) return PA_OK;
  const int64_t grid = a.items < sm_count() ? a.items : sm_count();
  uint8_t* cls = nullptr;
  if (!d.is_causal && d.mask_kind == PA_MASK_BOOL) {
    const int64_t tiles = mask_slice_count(a.mlt) * a.row_tiles * a.col_blocks;
    if (tiles > 0 && tiles <= 0x7fffffffLL) {
      PA_TRY(scratch_alloc(reinterpret_cast<void**>(&cls), static_cast<size_t>(tiles), st));
      mask_classify_kernel<<<static_cast<unsigned>(tiles), 256, 0, st>>>(
          static_cast<const uint8_t*>(mask), a.mlt, d.L, d.S, d.m_row_stride, d.m_col_stride,
          a.row_tiles, a.col_blocks, cls);
      PA_CUDA(cudaGetLastError());
      a.mcls = cls;
    }
  }
  pa_status rc;
  if (D == 128)
    rc = bf16 ? launch_masked<128, true>(d, tq, tk, tv, a, grid, st)
              : launch_masked<128, false>(d, tq, tk, tv, a, grid, st);
  else
    rc = bf16 ? launch_masked<64, true>(d, tq, tk, tv, a, grid, st)
              : launch_masked<64, false>(d, tq, tk, tv, a, grid, st);
  scratch_free(cls, st);
  return rc;
}

}  // namespace pa

namespace {
template <int D>
void fill_plan(pa_tile_plan* p) {
  using C = pa::TcCfg<D>;
  p->block_q = pa::BM;
  p->block_k = pa::BN;
  p->query_tiles = pa::kTiles;
  p->threads = pa::kThreads;
  p->shared_memory_bytes = C::kSmemBytes;
  p->tmem_columns = static_cast<int32_t>(pa::kTmemCols);
  p->k_stages = C::kKStages;
  p->v_stages = C::kVStages;
}
}  // namespace

extern "C" pa_status pa_fwd_tile_plan(int32_t head_dim, int32_t dtype_bytes, pa_tile_plan* plan) {
  pa::clear_error();
  if (!plan) return pa::fail(PA_ERR_INVALID, "null plan");
  if (dtype_bytes != 2) return pa::fail(PA_ERR_UNSUPPORTED, "the tensor-core forward takes 2-byte elements (fp16/bf16)");
  if (head_dim == 128) {
    fill_plan<128>(plan);
    return PA_OK;
  }
  if (head_dim == 64) {
    fill_plan<64>(plan);
    return PA_OK;
  }
  return pa::fail(PA_ERR_UNSUPPORTED, "the tensor-core forward takes head_dim 64 or 128");
}
