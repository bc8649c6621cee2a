// Shared host/device plumbing for libpa_b200: error reporting, the device
// status word, descriptor helpers, and the sm_100a PTX wrappers (mbarrier,
// TMA, tcgen05) the tensor-core kernels are written against.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "pa_b200.h"

namespace pa {

// ---------------------------------------------------------------- host errors

// Stores `msg` as this thread's last error and returns `code`.
pa_status fail(pa_status code, const std::string& msg);
pa_status fail_cuda(cudaError_t err, const char* what);
void clear_error();

#define PA_CUDA(call)                                        \
  do {                                                       \
    cudaError_t e_ = (call);                                 \
    if (e_ != cudaSuccess) return ::pa::fail_cuda(e_, #call); \
  } while (0)

#define PA_TRY(call)                   \
  do {                                 \
    pa_status s_ = (call);             \
    if (s_ != PA_OK) return s_;        \
  } while (0)

// Device-side status word of the current device (one int per device).
int* device_status_word();

// Stream-ordered scratch from the library pool (cudaMallocAsync).
pa_status scratch_alloc(void** p, size_t bytes, cudaStream_t s);
void scratch_free(void* p, cudaStream_t s);

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per device for `fn`
// (`mask` holds one bit per device already done).
pa_status set_smem_attr_once(const void* fn, int bytes, uint64_t* mask);

// Number of SMs of the current device (cached).
int sm_count();

// cuTensorMapEncodeTiled resolved through the runtime's driver entry point,
// so the library does not link libcuda directly.
pa_status encode_tma_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base,
                        uint64_t inner, uint64_t rows, uint64_t planes, uint64_t row_bytes,
                        uint64_t plane_bytes, uint32_t box_inner, uint32_t box_rows,
                        CUtensorMapSwizzle swz);

// 4-D map [inner, rows, heads, pages] with byte strides for the three outer
// dimensions; box = (box_inner, box_rows, 1, 1). Used for key/value caches
// that are either dense (batch, heads, keys, D) or split into pages.
pa_status encode_tma_4d(CUtensorMap* map, CUtensorMapDataType dt, const void* base,
                        const uint64_t dims[4], const uint64_t strides_bytes[3],
                        uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz);

// ------------------------------------------------------- descriptor helpers

inline int64_t lead_count(const pa_sdpa_desc& d) {
  int64_t n = 1;
  for (int i = 0; i < d.nlead; ++i) n *= d.lead[i];
  return n;
}

// Offsets of one output slice into q / k / v / mask given the broadcast
// leading shape; the grouped-query axis divides the k/v index.
struct LeadTable {
  int32_t n;
  int32_t gqa_axis;
  int32_t group;
  int32_t pad;
  int64_t dim[PA_MAX_LEAD];
  int64_t qs[PA_MAX_LEAD], ks[PA_MAX_LEAD], vs[PA_MAX_LEAD], ms[PA_MAX_LEAD];
};

inline LeadTable make_lead_table(const pa_sdpa_desc& d) {
  LeadTable t{};
  t.n = d.nlead;
  t.gqa_axis = d.gqa_group > 1 ? d.gqa_axis : -1;
  t.group = d.gqa_group > 1 ? d.gqa_group : 1;
  for (int i = 0; i < d.nlead; ++i) {
    t.dim[i] = d.lead[i];
    t.qs[i] = d.q_lead_stride[i];
    t.ks[i] = d.k_lead_stride[i];
    t.vs[i] = d.v_lead_stride[i];
    t.ms[i] = d.m_lead_stride[i];
  }
  return t;
}

struct SliceOffsets {
  int64_t q, k, v, m;
};

__host__ __device__ inline SliceOffsets slice_offsets(const LeadTable& t, int64_t slice) {
  SliceOffsets o{0, 0, 0, 0};
  for (int i = t.n - 1; i >= 0; --i) {
    int64_t idx = slice % t.dim[i];
    slice /= t.dim[i];
    int64_t kidx = (i == t.gqa_axis) ? idx / t.group : idx;
    o.q += idx * t.qs[i];
    o.k += kidx * t.ks[i];
    o.v += kidx * t.vs[i];
    o.m += idx * t.ms[i];
  }
  return o;
}

// ------------------------------------------------------------- device PTX

#if defined(__CUDACC__)

// Bound on every spin-wait in device code: give up after this many polls or
// this many nanoseconds of %globaltimer, whichever comes first.
constexpr uint32_t kWaitPolls = 1u << 28;
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s

// Codes written to the device status word.
enum : int {
  kStatusTimeoutLoad = 0x101,   // waiting for a TMA tile
  kStatusTimeoutMma = 0x102,    // waiting for a tensor-core result
  kStatusTimeoutSoftmax = 0x103,
  kStatusTimeoutFree = 0x104,   // producer waiting for a free stage
  kStatusTimeoutSelfTest = 0x105,  // pa_selftest_wait_timeout's planted wait
  kStatusBadSeqLen = 0x201,     // a sequence length outside [0, max_seq_len]
  kStatusBadPage = 0x202,       // a block-table entry outside [0, num_pages)
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase of parity `parity` to complete. On give-up it
// records `code` in the status word, raises the CTA abort flag and returns
// false; it also returns false at once when another role already aborted.
// `limit_ns` shortens the time bound (the self-test kernel uses 1 ms).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code,
                                          volatile int* abort_flag, uint64_t limit_ns = kWaitNs) {
  if (mbar_test(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0; i < kWaitPolls; ++i) {
    if (mbar_test(bar, parity)) return true;
    if ((i & 255u) == 255u) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > limit_ns) {
        *abort_flag = 1;
        atomicExch(status, code);
        return false;
      }
    }
  }
  *abort_flag = 1;
  atomicExch(status, code);
  return false;
}

// Bounded wait used on exit paths: it ignores the abort flag, because copies
// and MMAs already issued must complete before shared memory or TMEM is
// released. Gives up silently after the same poll / time bound.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  if (mbar_test(bar, parity)) return;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0; i < kWaitPolls; ++i) {
    if (mbar_test(bar, parity)) return;
    if ((i & 255u) == 255u && global_ns() - t0 > kWaitNs) return;
  }
}

// TMA: 3-D tiled load into shared memory, completion counted on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2, int32_t c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Untiled bulk copy global -> shared (16-byte aligned addresses, size % 16 == 0).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- tcgen05 / TMEM

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
// D(tmem) (+)= A(smem desc) * B(smem desc)
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D(tmem) (+)= A(tmem) * B(smem desc)
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp gets lane
// (32 * (warp % 4) + t) of the accessed quadrant, columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
// After tcgen05.wait::ld: make the compiler treat the loaded registers as
// redefined here, so no use of them is scheduled above the wait.
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i])::"memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), sm_100
// descriptor version 1, base offset 0 (tiles are 1024-byte aligned).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n, bool a_mn, bool b_mn, bool bf16) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack2(float a, float b, bool bf16) {
  if (bf16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Packed fp32 pairs (sm_100 f32x2 instructions: one issue, two lanes of math).
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// max(a, b, c) in one instruction.
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

#endif  // __CUDACC__

}  // namespace pa
