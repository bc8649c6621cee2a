// Split-KV decode forward (query length 1), HBM-bound.
//
// Work unit: (sequence b, key/value head kh, split s) -> one CTA that reads
// keys [s*chunk, min(len_b, (s+1)*chunk)) of K[b, kh] and V[b, kh] exactly
// once and serves all G = Hq / Hkv query heads that share that key/value
// head, so grouped-query K/V is never repeated.
//
// One kernel serves three cache layouts through a 4-D tensor map
// [D, page rows, kv heads, pages] with arbitrary strides:
//   dense     (B, Hkv, S, D), the reference's operand layout: page b holds
//             sequence b (pa_decode_fwd);
//   varlen    the same with a length per sequence (seq_lens);
//   paged     pages of `page_size` keys named by a block table, in any
//             (page, head, key) stride order, e.g. (pages, Hkv, page, D) or
//             (pages, page, Hkv, D).
// Key/value elements are fp16, bf16 (the query's type) or fp8 e4m3 with
// per-tensor dequantisation scales: k_scale folds into the softmax scale and
// v_scale into the final normalisation.
//
// CTA = 8 warps. Warp w owns tiles w, w+8, w+16, ... of the CTA's key range
// (a tile is 4 KB of keys + 4 KB of values: 16, 32 or 64 keys) and three
// 8 KB shared-memory stages: it keeps three tiles in flight by TMA (128-byte
// swizzle, or 64-byte for 64-byte rows; 192 KB per SM) and refills a stage as
// soon as it has used it, so no warp waits on another. For a paged cache the
// page numbers of the next tile to load are read from the block table one
// tile ahead, one piece per lane; a tile is split into pieces of 8-32 rows
// when pages are shorter than a tile.
//   compute   on tensor cores (warp-level m16n8k16, fp32 accumulators):
//             S = Q K^T for the G query heads (zero-padded to 16 rows),
//             online softmax on the accumulators, O^T += V^T P^T with P
//             straight from those accumulators. fp8 tiles are converted to
//             f16 in registers. Keys past the sequence end are masked and
//             their value rows zeroed, so stale cache contents (even NaN)
//             never reach the output.
//             The 8 warps' partial states merge in shared memory at the end
//             and the CTA writes one partial (m, l, acc[D]) per query head
//             into the workspace.
// combine     one CTA per (b, query head) merges the splits by log-sum-exp
//             and writes the fp16/bf16 output and, optionally, the lse. A
//             sequence with no keys gets a zero output and lse = -inf.
//
// The math is reference.py:139-162 for L == 1 (no mask, not causal), per
// sequence over its own keys.
#include <cuda_fp8.h>
#include <math.h>

#include <cmath>
#include <cstdio>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace pa {
namespace {

constexpr int kWarpsC = 8;                 // compute warps (each loads its own tiles)
constexpr int kThreadsDec = 32 * kWarpsC;
constexpr int kDepth = 3;                  // stages per warp
constexpr int kStages = kWarpsC * kDepth;  // 24 stages of 8 KB
constexpr int kStageBytes = 8192;          // one K tile + one V tile
constexpr float kLn2f = 0.6931471805599453f;

enum : int { kKvF16 = 0, kKvBF16 = 1, kKvE4M3 = 2 };

// Keys per tile: a stage holds 4 KB of keys and 4 KB of values.
constexpr int tile_keys(int D, int KV) { return 4096 / (D * (KV == kKvE4M3 ? 1 : 2)); }

template <int D, int KV>
struct DecCfg {
  static constexpr int kEsz = KV == kKvE4M3 ? 1 : 2;
  static constexpr int kRowBytes = D * kEsz;                        // one key row
  static constexpr int kBoxBytes = kRowBytes < 128 ? kRowBytes : 128;  // 128 (SW128) or 64 (SW64)
  static constexpr int kBoxCols = kBoxBytes / kEsz;
  static constexpr int kBoxes = kRowBytes / kBoxBytes;
  static constexpr int kTK = tile_keys(D, KV);                      // 16, 32 or 64 keys
  static constexpr int kTileBytes = kTK * kRowBytes;                // 4096: one K (or V) tile
  static_assert(2 * kTileBytes == kStageBytes, "stage = K tile + V tile");
  static constexpr int kRingBytes = kStages * kStageBytes;          // 192 KB
  static constexpr int kQOff = kRingBytes;                          // G*D floats (G <= 16)
  static constexpr int kBarOff = kQOff + 16 * D * 4;
  static constexpr int kSmemBytes = kBarOff + kStages * 8 + 16 + 1024;

  // Byte offset of byte `byte` of key row `row` inside a tile: 64-column
  // (128-byte) boxes one after another, rows 128 (or 64) bytes apart, the
  // 16-byte chunks permuted by the TMA swizzle (128B: chunk ^= row % 8;
  // 64B: chunk ^= (row / 2) % 4).
  static __device__ __forceinline__ int off(int row, int byte) {
    const int bx = byte / kBoxBytes, b = byte % kBoxBytes;
    const int sw = kBoxBytes == 128 ? (row & 7) : ((row >> 1) & 3);
    return bx * (kTK * kBoxBytes) + row * kBoxBytes + (((b >> 4) ^ sw) << 4) + (b & 15);
  }
};

struct DecArgs {
  const void* q;
  float* ws_acc;   // [B*Hq][nsplit][D]
  float* ws_ml;    // [B*Hq][nsplit][2]  (m in log2 units, l)
  int* status;
  const int32_t* block_table;  // [B][max_pages] or null (page b = sequence b)
  const int32_t* seq_lens;     // [B] or null (every sequence holds S keys)
  int64_t S;                   // bound on every sequence length
  int64_t max_pages;
  int32_t Hq, Hkv, nsplit, chunk;
  int32_t G;                   // query heads per key/value head (1..16)
  int32_t page_size, piece_rows, num_pages;
  float scale_log2;            // softmax scale * k_scale * log2(e)
};

__device__ __forceinline__ float to_float(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }

// ---- warp-level tensor-core helpers (mma.sync m16n8k16, f32 accumulate).
// The decode streams every key once and has at most 8 query heads per tile,
// so its products are tiny; warp-level MMAs from registers are enough to keep
// it HBM-bound, where CUDA-core FMAs were not (fp8 halves the bytes per key).
template <bool BF16>
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  if (BF16)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldsm_x4_t(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack_pair(float lo, float hi) {
  if (BF16) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Two e4m3 values in the low 16 bits (first value in the low byte) -> f16x2.
__device__ __forceinline__ uint32_t e4m3x2_to_h2(uint32_t two) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two & 0xffffu), __NV_E4M3);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t byte_perm(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

template <int D, int HT, bool QBF16, int KV>
__global__ void __launch_bounds__(kThreadsDec, 1)
    decode_partial_kernel(const __grid_constant__ CUtensorMap tk,
                          const __grid_constant__ CUtensorMap tv, const DecArgs a) {
  using C = DecCfg<D, KV>;
  using T = typename std::conditional<QBF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  float* sq = reinterpret_cast<float*>(smem + C::kQOff);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kBarOff + kStages * 8);
  constexpr int TK = C::kTK;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x % a.nsplit;
  const int64_t pair = blockIdx.x / a.nsplit;  // b * Hkv + kh
  const int64_t b = pair / a.Hkv;
  const int kh = static_cast<int>(pair % a.Hkv);
  const int G = a.G;  // query heads of this group: rows 0..G-1 of the HT-row head tile
  int64_t len = a.S;
  if (a.seq_lens) {
    len = a.seq_lens[b];
    if (len < 0 || len > a.S) {
      if (threadIdx.x == 0 && split == 0) atomicExch(a.status, kStatusBadSeqLen);
      len = len < 0 ? 0 : a.S;
    }
  }
  const int64_t k0 = static_cast<int64_t>(split) * a.chunk;
  const int64_t k1 = (k0 + a.chunk < len) ? k0 + a.chunk : len;
  const int ntiles = k1 > k0 ? static_cast<int>((k1 - k0 + TK - 1) / TK) : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(full + s, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  // q for the G heads of this group, fp32 in shared memory.
  const T* qg = static_cast<const T*>(a.q) + (b * a.Hq + static_cast<int64_t>(kh) * G) * D;
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) sq[i] = to_float(qg[i]);
  __syncthreads();

  // ------------------------------------------------------------ loading
  // Warp w owns tiles t = w + 8 j (j = 0, 1, ...) and stages w, w + 8, w + 16:
  // its j-th tile lands in stage w + 8 (j % 3). Each warp keeps its own three
  // tiles in flight and refills a stage as soon as it has finished with it, so
  // no warp ever waits for another (an in-order producer feeding all warps
  // stalls behind the slowest one), and a stage's barrier is never waited on
  // more than one phase ahead. Lane 0 issues the TMA copies.
  // A paged cache's page numbers for the tile issued at the end of an
  // iteration are loaded (one piece per lane) at its start, so the compute
  // hides their latency.
  const int n_own = ntiles > warp ? (ntiles - warp + kWarpsC - 1) / kWarpsC : 0;
  const int n_pc = TK / a.piece_rows;  // pieces per tile: 1, 2, 4 or 8
  auto tile_key0 = [&](int j) -> int32_t {
    return static_cast<int32_t>(k0 + static_cast<int64_t>(warp + kWarpsC * j) * TK);
  };
  // Page of piece `lane` of own tile j (lanes >= n_pc: unused), -1 past the end.
  auto load_page = [&](int j) -> int32_t {
    if (!a.block_table || lane >= n_pc || j >= n_own) return -1;
    const int32_t key = tile_key0(j) + lane * a.piece_rows;
    if (key >= len) return -1;
    const int32_t page = a.block_table[b * a.max_pages + key / a.page_size];
    if (page < 0 || page >= a.num_pages) {
      atomicExch(a.status, kStatusBadPage);
      return -1;
    }
    return page;
  };
  auto issue = [&](int j, int32_t pg) {  // all lanes call; lane 0 issues
    const int st = warp + kWarpsC * (j % kDepth);
    uint8_t* base = smem + st * kStageBytes;
    if (lane == 0) mbar_expect_tx(full + st, kStageBytes);
    const int32_t key0 = tile_key0(j);
    for (int p = 0; p < n_pc; ++p) {
      const int32_t key = key0 + p * a.piece_rows;
      int32_t page = static_cast<int32_t>(b), row = key;
      if (a.block_table) {
        page = __shfl_sync(0xffffffffu, pg, p);
        row = key % a.page_size;
      }
      if (lane == 0) {
        uint8_t* dst = base + p * a.piece_rows * C::kBoxBytes;
        for (int bx = 0; bx < C::kBoxes; ++bx) {
          tma_load_4d(dst + bx * (TK * C::kBoxBytes), &tk, full + st, bx * C::kBoxCols, row, kh, page);
          tma_load_4d(dst + C::kTileBytes + bx * (TK * C::kBoxBytes), &tv, full + st, bx * C::kBoxCols, row,
                      kh, page);
        }
      }
    }
  };
  for (int j = 0; j < kDepth && j < n_own; ++j) issue(j, load_page(j));
  int issued = n_own < kDepth ? n_own : kDepth;

  // -------------------------------------------------------------- compute
  // Per tile of TK keys, on tensor cores (m16n8k16, fp32 accumulators):
  //   S   = Q K^T    M = 16 query rows (the G heads, zero-padded), N = 8 keys
  //                  per n-tile (TK/8 n-tiles), K = head dim;
  //   O^T = V^T P^T  M = 16 value columns per m-tile (D/16 m-tiles), N = 8
  //                  heads, K = 16 keys per step (TK/16 steps).
  // The S accumulator of a thread (head g = lane/4, keys 2c, 2c+1 of each
  // n-tile, c = lane%4) is exactly its B fragment of P^T, so P never leaves
  // registers. Softmax runs on the S accumulators; each thread's per-head
  // running max/sum covers head g, and the O^T columns it owns (heads 2c,
  // 2c+1) fetch their rescale factors by two shuffles.
  // Operands: fp16/bf16 tiles by ldmatrix (K) / ldmatrix.trans (V); fp8 tiles
  // by 16-byte loads converted in registers (e4m3x2 -> f16x2). For fp8 the
  // head-dim elements are assigned to threads in a permuted order (thread c
  // owns a contiguous quarter of each key row for Q K^T, and thread g owns a
  // contiguous eighth of each value row for P V): a dot product does not
  // depend on the order of its terms, and the output columns are written
  // back to their true positions.
  // MMA type: bf16 for bf16 caches, otherwise f16 (fp8 values are exact in
  // f16; a bf16 query is scaled by a power of two into f16 range first).
  constexpr bool kMmaBf16 = KV == kKvBF16;
  constexpr bool kF8 = KV == kKvE4M3;
  constexpr int KS = D / 16;   // k-steps of Q K^T
  constexpr int MT = D / 16;   // m-tiles of P V
  constexpr int NT = TK / 8;   // n-tiles of Q K^T
  constexpr int PS = TK / 16;  // k-steps of P V
  const int g = lane >> 2, c = lane & 3;
  float sl2 = a.scale_log2;
  float qs = 1.f;
  if (QBF16 && kF8) {
    float mx = 0.f;
    for (int i = lane; i < G * D; i += 32) mx = fmaxf(mx, fabsf(sq[i]));
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (mx > 0.f && mx <= 3.0e38f) {
      int e = ((__float_as_int(mx) >> 23) & 0xff) - 127;  // floor(log2(max |q|)) for normal values
      e = e < -100 ? -100 : e;
      qs = __int_as_float((127 + 14 - e) << 23);         // max |q| * qs in [2^14, 2^15)
      sl2 = a.scale_log2 * __int_as_float((127 - 14 + e) << 23);
    }
  }
  // A fragments of Q: rows g (heads 0-7: a0, a2) and g + 8 (heads 8-15: a1, a3;
  // zero when the head tile is 8 rows). Rows past the group are zero.
  constexpr bool kTwo = HT == 16;
  uint32_t qa[KS][2], qh[KS][2];
#pragma unroll
  for (int s = 0; s < KS; ++s) {
    const int d0 = kF8 ? (D / 4) * c + 4 * s : 16 * s + 2 * c;
    const int d1 = kF8 ? d0 + 2 : d0 + 8;
    const float* qr = sq + (g < G ? g : 0) * D;
    const float z = g < G ? qs : 0.f;
    qa[s][0] = pack_pair<kMmaBf16>(qr[d0] * z, qr[d0 + 1] * z);
    qa[s][1] = pack_pair<kMmaBf16>(qr[d1] * z, qr[d1 + 1] * z);
    if (kTwo) {
      const float* q2 = sq + (g + 8 < G ? g + 8 : 0) * D;
      const float z2 = g + 8 < G ? qs : 0.f;
      qh[s][0] = pack_pair<kMmaBf16>(q2[d0] * z2, q2[d0 + 1] * z2);
      qh[s][1] = pack_pair<kMmaBf16>(q2[d1] * z2, q2[d1 + 1] * z2);
    }
  }
  auto qa_hi = [&](int s, int w) -> uint32_t { return kTwo ? qh[s][w] : 0u; };
  float o[MT][4], o2[MT][4];  // O^T for heads 0-7 and (16-row tiles) 8-15
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    o2[mt][0] = o2[mt][1] = o2[mt][2] = o2[mt][3] = 0.f;
  }
  float m_run = -INFINITY, l_run = 0.f, m_run2 = -INFINITY, l_run2 = 0.f;

  int consumed = 0;
  for (int j = 0; j < n_own; ++j) {
    const int st = warp + kWarpsC * (j % kDepth);
    bool ok = mbar_wait(full + st, (j / kDepth) & 1, a.status, kStatusTimeoutLoad, abort_flag);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) break;
    consumed = j + 1;
    const int32_t pg_next = load_page(j + kDepth);  // used after this tile's compute
    const uint8_t* kt = smem + st * kStageBytes;
    const uint8_t* vt = kt + C::kTileBytes;
    const int64_t tile0 = k0 + static_cast<int64_t>(warp + kWarpsC * j) * TK;
    const int rem = static_cast<int>(k1 - tile0 < TK ? k1 - tile0 : TK);

    // ---- S = Q K^T
    float sacc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
      if (kF8) {
        uint32_t kw[D / 16];
        const int row = 8 * nt + g;
#pragma unroll
        for (int i = 0; i < D / 64; ++i) {
          const uint4 u = *reinterpret_cast<const uint4*>(kt + C::off(row, (D / 4) * c + 16 * i));
          kw[4 * i] = u.x;
          kw[4 * i + 1] = u.y;
          kw[4 * i + 2] = u.z;
          kw[4 * i + 3] = u.w;
        }
#pragma unroll
        for (int s = 0; s < KS; ++s)
          mma16816<kMmaBf16>(sacc[nt], qa[s][0], qa_hi(s, 0), qa[s][1], qa_hi(s, 1), e4m3x2_to_h2(kw[s]),
                             e4m3x2_to_h2(kw[s] >> 16));
      } else {
        const int row = 8 * nt + (lane & 7);
#pragma unroll
        for (int s2 = 0; s2 < KS / 2; ++s2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kt + C::off(row, (4 * s2 + (lane >> 3)) * 16), b0, b1, b2, b3);
          mma16816<kMmaBf16>(sacc[nt], qa[2 * s2][0], qa_hi(2 * s2, 0), qa[2 * s2][1], qa_hi(2 * s2, 1), b0, b1);
          mma16816<kMmaBf16>(sacc[nt], qa[2 * s2 + 1][0], qa_hi(2 * s2 + 1, 0), qa[2 * s2 + 1][1],
                             qa_hi(2 * s2 + 1, 1), b2, b3);
        }
      }
    }

    // ---- online softmax: head g on accumulator columns 0-1, head g + 8 (16-row
    // head tiles) on columns 2-3; keys 8 nt + 2c + e.
    // The running max moves only when a score exceeds it by more than 2^8
    // (p <= 256 stays exact enough in f16/bf16 and fp32 sums), so after the
    // first tiles the accumulators are rarely rescaled; the max is finite
    // because the tile has at least one valid key.
    auto head_softmax = [&](int e0, float& m_h, float& l_h, uint32_t (&pbh)[PS][2], float& alpha_h) -> bool {
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float x = (8 * nt + 2 * c + e) < rem ? sacc[nt][e0 + e] * sl2 : -INFINITY;
          sacc[nt][e0 + e] = x;
          mx = fmaxf(mx, x);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const bool mv = mx > m_h + 8.f;
      const float m_new = mv ? mx : m_h;
      alpha_h = ex2(m_h - m_new);
      m_h = m_new;
      float psum = 0.f;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const float p0 = ex2(sacc[nt][e0] - m_new), p1 = ex2(sacc[nt][e0 + 1] - m_new);
        psum += p0 + p1;
        pbh[nt >> 1][nt & 1] = pack_pair<kMmaBf16>(p0, p1);
      }
      l_h = l_h * alpha_h + psum;
      return mv;
    };
    uint32_t pb[PS][2], pb2[PS][2];  // B fragments of P^T for the 16-key steps
    float alpha = 1.f, alpha2 = 1.f;
    bool moved = head_softmax(0, m_run, l_run, pb, alpha);
    if (kTwo) moved = head_softmax(2, m_run2, l_run2, pb2, alpha2) || moved;
    if (__any_sync(0xffffffffu, moved)) {
      const float al0 = __shfl_sync(0xffffffffu, alpha, 8 * c);      // head 2c
      const float al1 = __shfl_sync(0xffffffffu, alpha, 8 * c + 4);  // head 2c + 1
      const float bl0 = __shfl_sync(0xffffffffu, alpha2, 8 * c);     // head 8 + 2c
      const float bl1 = __shfl_sync(0xffffffffu, alpha2, 8 * c + 4); // head 9 + 2c
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        o[mt][0] *= al0;
        o[mt][1] *= al1;
        o[mt][2] *= al0;
        o[mt][3] *= al1;
        if (kTwo) {
          o2[mt][0] *= bl0;
          o2[mt][1] *= bl1;
          o2[mt][2] *= bl0;
          o2[mt][3] *= bl1;
        }
      }
    }

    // ---- O^T += V^T P^T
#pragma unroll
    for (int sp = 0; sp < PS; ++sp) {
      const int kb = 16 * sp;
      if (kF8) {
        constexpr int W = D / 32;  // 32-bit words of a thread's eighth of a value row
        uint32_t r[4][W];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = kb + 2 * c + (i & 1) + 8 * (i >> 1);
          const uint8_t* src = vt + C::off(row, (D / 8) * g);
          if (W == 4) {
            const uint4 u = *reinterpret_cast<const uint4*>(src);
            r[i][0] = u.x;
            r[i][W > 1 ? 1 : 0] = u.y;
            r[i][W > 2 ? 2 : 0] = u.z;
            r[i][W > 3 ? 3 : 0] = u.w;
          } else {
            const uint2 u = *reinterpret_cast<const uint2*>(src);
            r[i][0] = u.x;
            r[i][W > 1 ? 1 : 0] = u.y;
          }
          if (row >= rem)
#pragma unroll
            for (int w = 0; w < W; ++w) r[i][w] = 0u;  // rows past the end may hold anything
        }
#pragma unroll
        for (int w = 0; w < W; ++w) {
          const uint32_t x01 = byte_perm(r[0][w], r[1][w], 0x5140), y01 = byte_perm(r[0][w], r[1][w], 0x7362);
          const uint32_t x23 = byte_perm(r[2][w], r[3][w], 0x5140), y23 = byte_perm(r[2][w], r[3][w], 0x7362);
          const uint32_t ax0 = e4m3x2_to_h2(x01), ax1 = e4m3x2_to_h2(x01 >> 16);
          const uint32_t ax2 = e4m3x2_to_h2(x23), ax3 = e4m3x2_to_h2(x23 >> 16);
          const uint32_t ay0 = e4m3x2_to_h2(y01), ay1 = e4m3x2_to_h2(y01 >> 16);
          const uint32_t ay2 = e4m3x2_to_h2(y23), ay3 = e4m3x2_to_h2(y23 >> 16);
          mma16816<kMmaBf16>(o[2 * w], ax0, ax1, ax2, ax3, pb[sp][0], pb[sp][1]);
          mma16816<kMmaBf16>(o[2 * w + 1], ay0, ay1, ay2, ay3, pb[sp][0], pb[sp][1]);
          if (kTwo) {
            mma16816<kMmaBf16>(o2[2 * w], ax0, ax1, ax2, ax3, pb2[sp][0], pb2[sp][1]);
            mma16816<kMmaBf16>(o2[2 * w + 1], ay0, ay1, ay2, ay3, pb2[sp][0], pb2[sp][1]);
          }
        }
      } else {
        const int m = lane >> 3;
        const int row = kb + 8 * (m >> 1) + (lane & 7);
        // keys of this thread's A fragment halves: a0/a1 -> kb + 2c (+1), a2/a3 -> kb + 8 + 2c (+1)
        const uint32_t mlo = (kb + 2 * c < rem ? 0x0000ffffu : 0u) | (kb + 2 * c + 1 < rem ? 0xffff0000u : 0u);
        const uint32_t mhi = (kb + 8 + 2 * c < rem ? 0x0000ffffu : 0u) | (kb + 9 + 2 * c < rem ? 0xffff0000u : 0u);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4_t(vt + C::off(row, (2 * mt + (m & 1)) * 16), a0, a1, a2, a3);
          a0 &= mlo;
          a1 &= mlo;
          a2 &= mhi;
          a3 &= mhi;
          mma16816<kMmaBf16>(o[mt], a0, a1, a2, a3, pb[sp][0], pb[sp][1]);
          if (kTwo) mma16816<kMmaBf16>(o2[mt], a0, a1, a2, a3, pb2[sp][0], pb2[sp][1]);
        }
      }
    }
    // Every lane has finished reading this stage: refill it with tile j + 3.
    __syncwarp();
    if (j + kDepth < n_own) {
      issue(j + kDepth, pg_next);
      issued = j + kDepth + 1;
    }
  }
  // After an abort, wait (bounded) for this warp's copies still in flight
  // before the CTA reuses or releases the stages.
  if (lane == 0)
    for (int j = consumed; j < issued; ++j)
      mbar_drain(full + warp + kWarpsC * (j % kDepth), (j / kDepth) & 1);
  __syncwarp();

  // Per-thread sums -> per-head sums (the four threads of head g, and g + 8).
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  l_run2 += __shfl_xor_sync(0xffffffffu, l_run2, 1);
  l_run2 += __shfl_xor_sync(0xffffffffu, l_run2, 2);

  __syncthreads();  // every tile consumed and landed: the ring is free for the merge
  float* mw = reinterpret_cast<float*>(smem);                 // [8][G] m
  float* lw = mw + kWarpsC * G;                              // [8][G] l
  float* aw = lw + kWarpsC * G;                              // [8][G][D] acc
  if (c == 0 && g < G) {
    mw[warp * G + g] = m_run;
    lw[warp * G + g] = l_run;
  }
  if (kTwo && c == 0 && g + 8 < G) {
    mw[warp * G + g + 8] = m_run2;
    lw[warp * G + g + 8] = l_run2;
  }
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int h = 2 * c + (i & 1), half = i >> 1;
      const int d = kF8 ? (D / 8) * g + 2 * mt + half : 16 * mt + 8 * half + g;
      if (h < G) aw[(warp * G + h) * D + d] = o[mt][i];
      if (kTwo && h + 8 < G) aw[(warp * G + h + 8) * D + d] = o2[mt][i];
    }
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

template <int D, bool QBF16>
__global__ void __launch_bounds__(D) decode_combine_kernel(const float* ws_acc, const float* ws_ml,
                                                           void* out, float* lse, int nsplit,
                                                           float v_scale) {
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
  const float r = l > 0.f ? (o / l) * v_scale : 0.f;
  if (QBF16)
    static_cast<__nv_bfloat16*>(out)[qh * D + d] = __float2bfloat16_rn(r);
  else
    static_cast<__half*>(out)[qh * D + d] = __float2half_rn(r);
  if (lse && d == 0) lse[qh] = l > 0.f ? (M + __log2f(l)) * kLn2f : -INFINITY;
}

// A decode problem in cache terms. The dense operands of pa_decode_fwd map to
// one page per sequence (page_size = S, pages = B) and no block table.
struct DecPlan {
  int64_t B, Hq, Hkv, S;
  int D, G, nsplit, chunk;
  int tk;                       // keys per tile
  bool q_bf16;
  int kv;                       // kKvF16 / kKvBF16 / kKvE4M3
  int64_t page_size, num_pages, max_pages;
  int64_t key_stride, head_stride, page_stride;  // elements
  bool paged;
  int piece_rows;
  double scale;
  float k_scale, v_scale;
};

// Splits the keys so that the CTA count fills whole waves (1 CTA per SM).
void split_keys(DecPlan* p) {
  const int64_t pairs = p->B * p->Hkv;
  const int64_t sms = sm_count();
  const int64_t tiles = (p->S + p->tk - 1) / p->tk;
  if (tiles == 0) {
    p->nsplit = 1;
    p->chunk = p->tk;
    return;
  }
  int best = 1;
  double best_eff = 0;
  for (int ns = 1; ns <= 64 && ns <= tiles; ++ns) {
    const int64_t ctas = pairs * ns;
    const double waves = static_cast<double>(ctas) / sms;
    const double eff = waves / std::ceil(waves);
    // Prefer fewer splits unless a larger count fills waves clearly better;
    // also keep at least 4 tiles per warp so each warp's pipeline fills.
    if (tiles / ns < 4 * kWarpsC && ns > 1) break;
    if (eff > best_eff + 0.02) {
      best_eff = eff;
      best = ns;
    }
  }
  const int64_t per = (tiles + best - 1) / best;
  p->chunk = static_cast<int>(per * p->tk);
  p->nsplit = static_cast<int>((p->S + p->chunk - 1) / p->chunk);
}

pa_status check_shape(DecPlan* p) {
  if (p->D != 64 && p->D != 128) return fail(PA_ERR_UNSUPPORTED, "decode: head dim must be 64 or 128");
  if (p->Hkv < 1 || p->Hq < 1 || p->Hq % p->Hkv) return fail(PA_ERR_INVALID, "decode: q heads must be a multiple of kv heads");
  const int64_t G = p->Hq / p->Hkv;
  if (G < 1 || G > 16) return fail(PA_ERR_UNSUPPORTED, "decode: at most 16 query heads per key/value head");
  p->G = static_cast<int>(G);
  if (p->S < 0 || p->S > 0x7fffffffLL - 64) return fail(PA_ERR_UNSUPPORTED, "decode: too many keys");
  return PA_OK;
}

pa_status make_plan(const pa_sdpa_desc& d, DecPlan* p) {
  if (d.L != 1) return fail(PA_ERR_UNSUPPORTED, "decode: query length must be 1");
  if (d.dtype != PA_F16 && d.dtype != PA_BF16) return fail(PA_ERR_UNSUPPORTED, "decode: dtype must be fp16/bf16");
  if (d.E != d.Ev || (d.E != 64 && d.E != 128)) return fail(PA_ERR_UNSUPPORTED, "decode: head dim must be 64 or 128");
  if (d.mask_kind != PA_MASK_NONE || d.is_causal) return fail(PA_ERR_UNSUPPORTED, "decode: no mask / causal");
  if (d.S < 1) return fail(PA_ERR_UNSUPPORTED, "decode: needs at least one key");
  int64_t n, H, Hkv;
  if (!dense_bhsd(d, &n, &H, &Hkv)) return fail(PA_ERR_UNSUPPORTED, "decode: operands not dense (B, H, S, D)");
  *p = DecPlan{};
  p->B = n / H;
  p->Hq = H;
  p->Hkv = Hkv;
  p->S = d.S;
  p->D = static_cast<int>(d.E);
  PA_TRY(check_shape(p));
  p->q_bf16 = d.dtype == PA_BF16;
  p->kv = p->q_bf16 ? kKvBF16 : kKvF16;
  p->tk = tile_keys(p->D, p->kv);
  p->page_size = d.S;
  p->num_pages = p->B;
  p->max_pages = 1;
  p->key_stride = p->D;
  p->head_stride = d.S * p->D;
  p->page_stride = Hkv * d.S * p->D;
  p->paged = false;
  p->piece_rows = p->tk;
  p->scale = d.scale;
  p->k_scale = 1.f;
  p->v_scale = 1.f;
  split_keys(p);
  return PA_OK;
}

pa_status make_plan(const pa_kv_cache_desc& d, bool paged, DecPlan* p) {
  *p = DecPlan{};
  if (d.q_dtype != PA_F16 && d.q_dtype != PA_BF16) return fail(PA_ERR_UNSUPPORTED, "decode: q dtype must be fp16 or bf16");
  if (d.kv_dtype != d.q_dtype && d.kv_dtype != PA_FP8_E4M3)
    return fail(PA_ERR_UNSUPPORTED, "decode: the cache dtype must be the query's dtype or fp8 e4m3");
  if (d.batch < 0) return fail(PA_ERR_INVALID, "decode: negative batch");
  if (!std::isfinite(d.scale) || !std::isfinite(d.k_scale) || !std::isfinite(d.v_scale))
    return fail(PA_ERR_INVALID, "decode: scale, k_scale and v_scale must be finite");
  p->B = d.batch;
  p->Hq = d.q_heads;
  p->Hkv = d.kv_heads;
  p->S = d.max_seq_len;
  p->D = static_cast<int>(d.head_dim);
  if (d.head_dim != p->D) return fail(PA_ERR_UNSUPPORTED, "decode: head dim must be 64 or 128");
  PA_TRY(check_shape(p));
  p->q_bf16 = d.q_dtype == PA_BF16;
  p->kv = d.kv_dtype == PA_FP8_E4M3 ? kKvE4M3 : (p->q_bf16 ? kKvBF16 : kKvF16);
  p->tk = tile_keys(p->D, p->kv);
  p->page_size = d.page_size;
  p->num_pages = d.num_pages;
  p->max_pages = d.max_pages_per_seq;
  p->key_stride = d.key_stride;
  p->head_stride = d.head_stride;
  p->page_stride = d.page_stride;
  p->paged = paged;
  p->scale = d.scale;
  p->k_scale = d.k_scale;
  p->v_scale = d.v_scale;
  if (d.key_stride < p->D || d.head_stride < 1 || d.page_stride < 1)
    return fail(PA_ERR_INVALID, "decode: cache strides must be positive and key_stride >= head_dim");
  if (d.num_pages < 1 || d.num_pages > 0x7fffffffLL) return fail(PA_ERR_INVALID, "decode: num_pages must be in [1, 2^31)");
  if (paged) {
    if (d.page_size < 8 || d.page_size % 8) return fail(PA_ERR_UNSUPPORTED, "decode: page_size must be a positive multiple of 8");
    if (d.page_size > 0x7fffffffLL) return fail(PA_ERR_UNSUPPORTED, "decode: page_size too large");
    if (d.max_pages_per_seq < (d.max_seq_len + d.page_size - 1) / d.page_size)
      return fail(PA_ERR_INVALID, "decode: max_pages_per_seq * page_size must cover max_seq_len");
    // One TMA box per page piece: the largest power of two <= the tile that
    // divides the page size (at least 8 rows).
    int pr = p->tk;
    while (d.page_size % pr) pr /= 2;
    p->piece_rows = pr;
  } else {
    if (d.num_pages < d.batch) return fail(PA_ERR_INVALID, "decode: without a block table the cache needs one page per sequence");
    if (d.page_size < d.max_seq_len || d.page_size < 1 || d.page_size > 0x7fffffffLL)
      return fail(PA_ERR_INVALID, "decode: without a block table page_size must be at least max_seq_len");
    p->max_pages = 1;
    p->piece_rows = p->tk;
  }
  split_keys(p);
  return PA_OK;
}

size_t plan_ws_bytes(const DecPlan& p) {
  const size_t slots = static_cast<size_t>(p.B * p.Hq) * p.nsplit;
  return slots * (p.D + 2) * sizeof(float);
}

template <int D, int HT, bool QBF16, int KV>
pa_status launch_dec(const DecPlan& p, const CUtensorMap& tk, const CUtensorMap& tv, DecArgs& a,
                     void* out, float* lse, cudaStream_t st) {
  auto kern = decode_partial_kernel<D, HT, QBF16, KV>;
  constexpr int smem = DecCfg<D, KV>::kSmemBytes;
  static uint64_t attr_set = 0;
  PA_TRY(set_smem_attr_once(reinterpret_cast<const void*>(kern), smem, &attr_set));
  const int64_t grid = p.B * p.Hkv * p.nsplit;
  kern<<<static_cast<unsigned>(grid), kThreadsDec, smem, st>>>(tk, tv, a);
  PA_CUDA(cudaGetLastError());
  decode_combine_kernel<D, QBF16><<<static_cast<unsigned>(p.B * p.Hq), D, 0, st>>>(
      a.ws_acc, a.ws_ml, out, lse, p.nsplit, p.v_scale);
  PA_CUDA(cudaGetLastError());
  return PA_OK;
}

template <int D, bool QBF16, int KV>
pa_status launch_dec_g(const DecPlan& p, const CUtensorMap& tk, const CUtensorMap& tv, DecArgs& a,
                       void* out, float* lse, cudaStream_t st) {
  // Head tile of 8 rows (groups 1-8) or 16 rows (groups 9-16).
  if (p.G <= 8) return launch_dec<D, 8, QBF16, KV>(p, tk, tv, a, out, lse, st);
  return launch_dec<D, 16, QBF16, KV>(p, tk, tv, a, out, lse, st);
}

template <int D>
pa_status launch_dec_t(const DecPlan& p, const CUtensorMap& tk, const CUtensorMap& tv, DecArgs& a,
                       void* out, float* lse, cudaStream_t st) {
  if (p.kv == kKvE4M3)
    return p.q_bf16 ? launch_dec_g<D, true, kKvE4M3>(p, tk, tv, a, out, lse, st)
                    : launch_dec_g<D, false, kKvE4M3>(p, tk, tv, a, out, lse, st);
  return p.q_bf16 ? launch_dec_g<D, true, kKvBF16>(p, tk, tv, a, out, lse, st)
                  : launch_dec_g<D, false, kKvF16>(p, tk, tv, a, out, lse, st);
}

pa_status encode_cache_map(const DecPlan& p, const void* base, CUtensorMap* map) {
  const int esz = p.kv == kKvE4M3 ? 1 : 2;
  const int row_bytes = p.D * esz;
  const uint32_t box_bytes = row_bytes < 128 ? row_bytes : 128;
  const CUtensorMapDataType dt = p.kv == kKvE4M3 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                 : p.kv == kKvBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t dims[4] = {static_cast<uint64_t>(p.D), static_cast<uint64_t>(p.page_size),
                            static_cast<uint64_t>(p.Hkv), static_cast<uint64_t>(p.num_pages)};
  const uint64_t strides[3] = {static_cast<uint64_t>(p.key_stride) * esz,
                               static_cast<uint64_t>(p.head_stride) * esz,
                               static_cast<uint64_t>(p.page_stride) * esz};
  return encode_tma_4d(map, dt, base, dims, strides, box_bytes / esz, static_cast<uint32_t>(p.piece_rows),
                       box_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
}

pa_status run_plan(const DecPlan& p, const void* q, const void* k, const void* v,
                   const int32_t* block_table, const int32_t* seq_lens, void* out, float* lse,
                   void* ws, size_t ws_bytes, int* status, cudaStream_t st) {
  if (ws_bytes < plan_ws_bytes(p)) return fail(PA_ERR_INVALID, "decode: workspace too small");
  if (p.B * p.Hkv * p.nsplit > 0x7fffffffLL) return fail(PA_ERR_UNSUPPORTED, "decode: grid too large");
  CUtensorMap tk, tv;
  PA_TRY(encode_cache_map(p, k, &tk));
  PA_TRY(encode_cache_map(p, v, &tv));
  DecArgs a{};
  a.q = q;
  const size_t slots = static_cast<size_t>(p.B * p.Hq) * p.nsplit;
  a.ws_acc = static_cast<float*>(ws);
  a.ws_ml = a.ws_acc + slots * p.D;
  a.status = status;
  a.block_table = p.paged ? block_table : nullptr;
  a.seq_lens = seq_lens;
  a.S = p.S;
  a.max_pages = p.max_pages;
  a.Hq = static_cast<int32_t>(p.Hq);
  a.Hkv = static_cast<int32_t>(p.Hkv);
  a.G = p.G;
  a.nsplit = p.nsplit;
  a.chunk = p.chunk;
  a.page_size = static_cast<int32_t>(p.page_size);
  a.piece_rows = p.piece_rows;
  a.num_pages = static_cast<int32_t>(p.num_pages);
  a.scale_log2 = static_cast<float>(p.scale * static_cast<double>(p.k_scale) * 1.4426950408889634);
  if (p.D == 128) return launch_dec_t<128>(p, tk, tv, a, out, lse, st);
  return launch_dec_t<64>(p, tk, tv, a, out, lse, st);
}

}  // namespace

// Runs the decode with the given workspace (at least decode_ws_bytes bytes);
// bounded waits that give up record their code in `status`.
pa_status run_decode_status(const pa_sdpa_desc& d, const void* q, const void* k, const void* v,
                            void* out, float* lse, void* ws, size_t ws_bytes, int* status,
                            cudaStream_t st) {
  DecPlan p;
  PA_TRY(make_plan(d, &p));
  return run_plan(p, q, k, v, nullptr, nullptr, out, lse, ws, ws_bytes, status, st);
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
  if (!q || !k || !v || !out) return fail(PA_ERR_INVALID, "decode: null q, k, v or out pointer");
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

extern "C" pa_status pa_decode_kv_workspace_size(const pa_kv_cache_desc* desc, int32_t paged,
                                                 size_t* bytes) {
  clear_error();
  if (!desc || !bytes) return fail(PA_ERR_INVALID, "null argument");
  DecPlan p;
  PA_TRY(make_plan(*desc, paged != 0, &p));
  *bytes = plan_ws_bytes(p);
  return PA_OK;
}

extern "C" pa_status pa_decode_kv_fwd(const pa_kv_cache_desc* desc, const void* q,
                                      const void* k_cache, const void* v_cache,
                                      const int32_t* block_table, const int32_t* seq_lens,
                                      void* out, float* lse, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  clear_error();
  if (!desc) return fail(PA_ERR_INVALID, "null descriptor");
  DecPlan p;
  PA_TRY(make_plan(*desc, block_table != nullptr, &p));
  if (p.B == 0) return PA_OK;
  if (!q || !k_cache || !v_cache || !out) return fail(PA_ERR_INVALID, "decode: null q, cache or out pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* status = device_status_word();
  if (!status) return fail(PA_ERR_CUDA, "device status word unavailable");
  const size_t need = plan_ws_bytes(p);
  if (workspace) {
    if (workspace_bytes < need) return fail(PA_ERR_INVALID, "decode: workspace smaller than pa_decode_kv_workspace_size");
    return run_plan(p, q, k_cache, v_cache, block_table, seq_lens, out, lse, workspace, workspace_bytes, status, st);
  }
  void* ws = nullptr;
  PA_TRY(scratch_alloc(&ws, need, st));
  pa_status s = run_plan(p, q, k_cache, v_cache, block_table, seq_lens, out, lse, ws, need, status, st);
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
// Status word for bounded waits when the caller passes none; pa_device_status
// reads and clears it together with the library's own word.
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

pa_status take_static_decode_status(int* code) {
  *code = 0;
  int dev = 0;
  PA_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDev) return PA_OK;
  {
    // Nothing to read on a device where the static entry point never ran
    // (its word was never handed to a kernel).
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_status_addr[dev]) return PA_OK;
  }
  int v = 0;
  PA_CUDA(cudaMemcpyFromSymbol(&v, g_decode_static_status, sizeof(int)));
  if (v) {
    const int zero = 0;
    PA_CUDA(cudaMemcpyToSymbol(g_decode_static_status, &zero, sizeof(int)));
  }
  *code = v;
  return PA_OK;
}

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
  if (!q || !k || !v || !out) return fail(PA_ERR_INVALID, "decode: null q, k, v or out pointer");
  void* scratch = nullptr;
  int* own_status = nullptr;
  PA_TRY(static_scratch_for_current_device(&scratch, &own_status));
  int* st_word = status ? reinterpret_cast<int*>(status) : own_status;
  return run_decode_status(d, q, k, v, out, lse, scratch, kStaticScratchBytes, st_word,
                           static_cast<cudaStream_t>(stream));
}
