/*
 * pa_b200.h -- C ABI of the B200 (sm_100a) attention library libpa_b200.so.
 *
 * This is the drop-in boundary for the portable-attention backend seam: the
 * Python host layer (package pa_b200) binds every symbol here through ctypes
 * and registers the result with portable_attention.register_backend
 * (src/portable_attention/dispatch.py:92-120) as an SdpaBackend
 * (dispatch.py:53-76). Any other FFI (cffi, JNI, cgo) can bind the same
 * symbols: only plain pointers, sizes and the POD descriptor below cross it.
 *
 * Conventions
 *  - Every entry point returns a pa_status (0 = PA_OK). On failure a
 *    thread-local message is available from pa_last_error(); no C++ exception
 *    crosses the boundary.
 *  - Device pointers come from pa_malloc (or any CUDA allocation on the
 *    current device). A NULL stream means the legacy default stream.
 *  - Compute entry points are asynchronous on `stream`; pa_stream_sync or the
 *    synchronous copy helpers complete them. Kernels whose bounded waits give
 *    up record a code in a per-device status word read by pa_device_status.
 *  - Element strides are in elements, not bytes.
 */
#ifndef PA_B200_H
#define PA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t pa_status;
enum {
  PA_OK = 0,
  PA_ERR_INVALID = 1,     /* bad argument: mirrors the reference's ValueError */
  PA_ERR_UNSUPPORTED = 2, /* valid input this library does not handle (dropout...) */
  PA_ERR_CUDA = 3,        /* a CUDA runtime / driver call failed */
  PA_ERR_TIMEOUT = 4,     /* a bounded device-side wait gave up */
  PA_ERR_NCCL = 5,        /* an NCCL call failed or a peer timed out */
  PA_ERR_NOMEM = 6        /* device or pinned-host allocation failed */
};

/* Element types. PA_FP8_E4M3 is the OCP FP8 E4M3 format ("e4m3fn": 1 sign,
 * 4 exponent bits with bias 7, 3 mantissa bits, no infinities, 0x7f / 0xff
 * NaN, largest finite 448); it is accepted only as a decode cache type. */
enum { PA_F16 = 1, PA_BF16 = 2, PA_F32 = 3, PA_F64 = 4, PA_BOOL = 5, PA_FP8_E4M3 = 6 };

/* Mask kinds: none, boolean keep-mask (1 byte per element, nonzero = keep),
 * additive float mask (type mask_dtype) added to the scaled scores. */
enum { PA_MASK_NONE = 0, PA_MASK_BOOL = 1, PA_MASK_ADD = 2 };

#define PA_MAX_LEAD 6

/*
 * Problem descriptor for one scaled-dot-product-attention call.
 *
 * Shapes follow the reference contract (src/portable_attention/reference.py:76-82):
 * query (*, L, E), key (*, S, E), value (*, S, Ev) -> out (*, L, Ev), with the
 * leading dims `lead[0..nlead)` being the broadcast leading shape of the
 * output. Each operand gives one element stride per leading dim (0 where it
 * broadcasts) and a row stride; its last dim is contiguous. `out` is always
 * dense: out[(slice * L + i) * Ev + j], slice = row-major index over `lead`.
 *
 * Grouped-query attention (reference.py:20-53): when gqa_group > 1, key and
 * value are indexed along leading dim `gqa_axis` by (query index / gqa_group).
 *
 * Causal masking is top-left aligned: key j is visible to query i iff j <= i
 * (reference.py:141-144). A mask has one element stride per leading dim plus
 * row and column strides (column stride may be 0 for a broadcast column).
 */
typedef struct pa_sdpa_desc {
  int32_t dtype;                      /* PA_F16 / PA_BF16 / PA_F32 / PA_F64 for q,k,v,out */
  int32_t nlead;                      /* 0..PA_MAX_LEAD */
  int64_t lead[PA_MAX_LEAD];
  int64_t q_lead_stride[PA_MAX_LEAD];
  int64_t k_lead_stride[PA_MAX_LEAD];
  int64_t v_lead_stride[PA_MAX_LEAD];
  int64_t m_lead_stride[PA_MAX_LEAD];
  int64_t L, S, E, Ev;
  int64_t q_row_stride, k_row_stride, v_row_stride;
  int32_t gqa_axis;                   /* -1 when gqa_group == 1 */
  int32_t gqa_group;                  /* Hq / Hkv, >= 1 */
  int32_t mask_kind;                  /* PA_MASK_* */
  int32_t mask_dtype;                 /* PA_BOOL, or PA_F16/PA_F32/PA_F64 for additive */
  int64_t m_row_stride, m_col_stride;
  int32_t is_causal;
  int32_t reserved;
  double scale;                       /* softmax scale (caller resolves the 1/sqrt(E) default) */
} pa_sdpa_desc;

/* ---- library / device ------------------------------------------------- */

/* Library version as major*10000 + minor*100 + patch. */
int32_t pa_version(void);
/* Thread-local text of the last failure on this thread ("" if none). */
const char* pa_last_error(void);
/* Initialise the runtime and report the visible CUDA device count (0 on a
 * host without a usable GPU, with PA_ERR_CUDA). */
pa_status pa_init(int32_t* ndev);
pa_status pa_set_device(int32_t dev);
pa_status pa_get_device(int32_t* dev);
/* Read and clear the device status words of the current device (the
 * library's own and the one pa_decode_fwd_static uses when given no status
 * pointer): 0, or the code of a bounded device-side wait that gave up
 * (0x101-0x105, PA_ERR_TIMEOUT) or of an input error found on the device
 * (0x201-0x202, PA_ERR_INVALID). Allocates nothing. */
pa_status pa_device_status(int32_t* code);

/* Failure-path self-test (no reference counterpart; the reference's analogue
 * is its bounded fence wait, vkcompute.py:1031-1042). Launches one CTA on
 * `stream` whose first warp waits on an mbarrier nothing arrives on, with a
 * time bound of `limit_us` microseconds (1 to 1000000), through the same
 * bounded-wait routine every pipelined kernel uses; its second warp waits on
 * another such barrier and leaves through the CTA abort flag. The kernel ends
 * by itself: pa_device_status() then reports code 0x105 (PA_ERR_TIMEOUT) and
 * the context stays usable. */
pa_status pa_selftest_wait_timeout(int32_t limit_us, void* stream);

/* ---- memory and streams ------------------------------------------------ */

pa_status pa_malloc(void** dptr, size_t bytes);
pa_status pa_free(void* dptr);
pa_status pa_host_alloc(void** hptr, size_t bytes); /* page-locked host memory */
pa_status pa_host_free(void* hptr);
pa_status pa_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream);
pa_status pa_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream);
pa_status pa_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream);
pa_status pa_memset(void* dptr, int32_t value, size_t bytes, void* stream);
pa_status pa_stream_create(void** stream);
pa_status pa_stream_destroy(void* stream);
pa_status pa_stream_sync(void* stream);
pa_status pa_event_create(void** event);
pa_status pa_event_destroy(void* event);
pa_status pa_event_record(void* event, void* stream);
/* Block the calling host thread until `event` has completed. */
pa_status pa_event_sync(void* event);
/* *pinned = 1 when `ptr` lies in page-locked host memory the CUDA runtime knows
 * (pa_host_alloc, cudaHostAlloc, registered ranges), 0 for ordinary pageable
 * memory. The NumPy entry point stages pageable inputs through page-locked
 * buffers itself, since the driver's own staging of pageable copies is slow. */
pa_status pa_host_is_pinned(const void* ptr, int32_t* pinned);
/* Make later work on `stream` wait for `event` (cross-stream ordering). */
pa_status pa_stream_wait_event(void* stream, void* event);
pa_status pa_event_elapsed_ms(void* start, void* stop, float* ms);

/* ---- attention ---------------------------------------------------------- */

/*
 * Forward attention. Replaces the backend call of
 * src/portable_attention/dispatch.py:53-76 (SdpaBackend.__call__), whose
 * CPU implementations are reference.py:56-163 and fused.py:115-218.
 *
 * `lse` (optional, may be NULL) receives the natural-log log-sum-exp of the
 * scaled, masked scores per output row (float32, dense over lead x L);
 * fully-masked rows get -inf and an exactly-zero output row
 * (reference.py:151-160).
 *
 * Kernel choice is internal: fp16/bf16 with E == Ev in {64, 128} and dense
 * (B, H, L, E) operands runs the tcgen05/TMEM tensor-core kernel; everything
 * else runs the exact CUDA-core kernel (fp32 math for fp16/fp32, fp64 math
 * for fp64; no TF32).
 */
pa_status pa_sdpa_fwd(const pa_sdpa_desc* desc, const void* q, const void* k, const void* v,
                      const void* mask, void* out, float* lse, void* stream);

/*
 * Split-KV decode forward for L == 1 (no reference counterpart beyond the
 * same SdpaBackend call with a length-1 query: dispatch.py:53-76). Dense
 * (B, Hq, 1, D) query, (B, Hkv, S, D) key/value, D in {64, 128}, fp16/bf16,
 * no mask, not causal. `workspace` holds the per-split partial results; pass
 * NULL to let the library take it from its stream-ordered pool, or a buffer
 * of at least pa_decode_workspace_size() bytes.
 */
pa_status pa_decode_workspace_size(const pa_sdpa_desc* desc, size_t* bytes);
pa_status pa_decode_fwd(const pa_sdpa_desc* desc, const void* q, const void* k, const void* v,
                        void* out, float* lse, void* workspace, size_t workspace_bytes,
                        void* stream);

/*
 * Decode over a key/value cache: the L == 1 attention of pa_decode_fwd for a
 * batch of sequences with their own lengths, read from a contiguous or a
 * paged cache in fp16, bf16 or fp8 e4m3. No reference counterpart: the
 * reference's interface takes dense key/value tensors only
 * (dispatch.py:53-76); this is its math (reference.py:139-162) per sequence
 * over keys [0, seq_lens[b]) of that sequence.
 *
 * Cache layout. Keys and values live in pages of `page_size` keys; element
 * (page, kv head h, key row r, column d) is at
 *   page * page_stride + h * head_stride + r * key_stride + d
 * elements from the cache base (k and v share the layout), so both
 * (pages, kv_heads, page_size, D) and (pages, page_size, kv_heads, D) caches
 * are accepted as they are. Byte strides must be multiples of 16 and the
 * bases 16-byte aligned.
 *   With a block table (int32 [batch][max_pages_per_seq], device memory):
 *   key j of sequence b is row j % page_size of page
 *   block_table[b][j / page_size]; page_size is a multiple of 8. Entries past
 *   a sequence's last page are not read.
 *   Without one (NULL): page b holds sequence b from row 0, so a dense
 *   (batch, kv_heads, S, D) cache is page_size = S, num_pages = batch.
 * seq_lens (int32 [batch], device memory) gives each sequence's length, at
 * most max_seq_len; NULL means every sequence holds max_seq_len keys. A
 * sequence of length 0 gets a zero output row and lse = -inf. Cache rows past
 * a sequence's length are never used, whatever they hold.
 *
 * q and out are dense (batch, q_heads, head_dim) in q_dtype; lse (optional)
 * is float32 (batch, q_heads), natural log. Grouped-query attention shares
 * kv head h among q heads [h*G, (h+1)*G), G = q_heads / kv_heads from
 * 1 to 16; head_dim is 64 or 128.
 *
 * fp8 caches: scores use k * k_scale and the output v * v_scale (per-tensor
 * dequantisation); set both to 1.0 for fp16/bf16 caches. `scale` is the
 * softmax scale (1/sqrt(head_dim) for the reference's default).
 *
 * A sequence length outside [0, max_seq_len] or a block-table entry outside
 * [0, num_pages) is detected on the device: the keys involved are treated
 * as zeros and pa_device_status() then reports PA_ERR_INVALID (codes 0x201
 * and 0x202); no out-of-bounds memory is read.
 *
 * `workspace` as for pa_decode_fwd (NULL: stream-ordered pool), at least
 * pa_decode_kv_workspace_size() bytes; `paged` is nonzero when a block table
 * will be passed.
 */
typedef struct pa_kv_cache_desc {
  int32_t q_dtype;            /* PA_F16 / PA_BF16: q and out */
  int32_t kv_dtype;           /* q_dtype, or PA_FP8_E4M3 */
  int64_t batch;              /* sequences, one query row each */
  int64_t q_heads, kv_heads;
  int64_t head_dim;           /* 64 or 128 */
  int64_t max_seq_len;        /* bound on every seq_lens[b]; sizes the key split */
  int64_t page_size;          /* keys per page */
  int64_t num_pages;          /* pages in the cache */
  int64_t max_pages_per_seq;  /* block-table row length (ignored without one) */
  int64_t key_stride;         /* elements between consecutive keys (rows) */
  int64_t head_stride;        /* elements between kv heads */
  int64_t page_stride;        /* elements between pages */
  double scale;               /* softmax scale */
  float k_scale, v_scale;     /* dequantisation factors (1.0 unless fp8) */
} pa_kv_cache_desc;

pa_status pa_decode_kv_workspace_size(const pa_kv_cache_desc* desc, int32_t paged, size_t* bytes);
pa_status pa_decode_kv_fwd(const pa_kv_cache_desc* desc, const void* q, const void* k_cache,
                           const void* v_cache, const int32_t* block_table,
                           const int32_t* seq_lens, void* out, float* lse, void* workspace,
                           size_t workspace_bytes, void* stream);

/*
 * Allocation-free variant of pa_decode_fwd. It has no counterpart in the
 * reference (which runs on the CPU and never manages device memory).
 *
 * For callers that cannot allocate device memory while they run: hosts whose
 * allocator or memory budget forbids new cudaMalloc calls after start-up,
 * plugins whose device memory belongs to another runtime, and serving loops
 * that must not synchronise or fragment a pool mid-step. The caller passes
 * only inputs and outputs; the split partials live in a file-scope device
 * array of 8 MiB (8388608 bytes) that every GPU loading this library holds
 * until the process exits. Problems whose partials need more than that
 * (pa_decode_workspace_size reports the need) fail with PA_ERR_UNSUPPORTED
 * and a message giving both sizes; nothing is launched then.
 *
 * The first call on each device looks up the array's device address with
 * that device current (cudaGetSymbolAddress); make that first call before
 * any stream capture. With CUDA's lazy module loading that first call may
 * also load the library's device code on that device, which is when the
 * array's 8 MiB are committed: make it at start-up, before any memory budget
 * applies. The entry point calls no cudaMalloc, cudaFree or other
 * allocating routine.
 *
 * All calls on a device share the one array and it keeps the last call's
 * contents. Every partial a call reads is written earlier in the same call,
 * so nothing needs clearing, but calls that overlap on the GPU (different
 * streams, or different host threads without ordering) race on the array:
 * order them on one stream.
 *
 * `status` (device pointer, may be NULL) receives a nonzero code if a bounded
 * device-side wait gives up; the caller zeroes it beforehand. With NULL the
 * code goes to a word inside the library that pa_device_status() reads and
 * clears (without allocating), so check pa_device_status() after the stream
 * has finished: the output of a call whose wait gave up is not valid.
 * q, k, v and out must not be NULL (PA_ERR_INVALID, nothing launched).
 */
pa_status pa_decode_fwd_static(const pa_sdpa_desc* desc, const void* q, const void* k,
                               const void* v, void* out, float* lse, int32_t* status,
                               void* stream);

/*
 * One forward call spread over several GPUs of this process (batch x head
 * sharding; no reference counterpart: the reference runs one CPU call).
 * `desc` describes HOST operands exactly as for pa_sdpa_fwd; q, k, v, mask,
 * out and lse are host pointers (page-locked memory copies fastest). The
 * first leading dimension is cut into contiguous shards, one per entry of
 * `devices` (fewer if it has fewer indices); each device copies its rows in,
 * runs the same kernels as pa_sdpa_fwd (or the split-KV decode for L == 1)
 * and copies its rows of out / lse back, driven by its own host thread.
 * Operands broadcast over the first dimension (stride 0, e.g. a mask) are
 * copied whole to every device. When the first dimension is the grouped-
 * query head axis, shards hold whole groups. Blocks until every device has
 * finished; the first failure is returned with the device named.
 */
pa_status pa_shard_fwd(int32_t ndev, const int32_t* devices, const pa_sdpa_desc* desc,
                       const void* q, const void* k, const void* v, const void* mask, void* out,
                       float* lse);

/*
 * The tile plan the tensor-core forward compiles for a head dimension and
 * element size (pa_sdpa_fwd's fwd_tc kernel), in the vocabulary of the
 * reference's tile planner (tiling.py:68-121 DeviceLimits / :125-145
 * TilePlan): rows per query tile and keys per streamed tile, threads and
 * shared memory per CTA, plus what tcgen05 adds (query tiles per CTA, K/V
 * stages, TMEM columns). Returns PA_ERR_UNSUPPORTED for shapes the kernel
 * does not take (they run on the exact CUDA-core kernel).
 */
typedef struct pa_tile_plan {
  int32_t block_q;          /* query rows per tile */
  int32_t block_k;          /* keys per streamed K/V tile */
  int32_t query_tiles;      /* query tiles per CTA */
  int32_t threads;          /* threads per CTA */
  int32_t shared_memory_bytes;
  int32_t tmem_columns;
  int32_t k_stages, v_stages;
} pa_tile_plan;

pa_status pa_fwd_tile_plan(int32_t head_dim, int32_t dtype_bytes, pa_tile_plan* plan);

/*
 * Backward (VJP) of pa_sdpa_fwd: dQ, dK, dV from q, k, v, the forward output,
 * its cotangent dout and the forward's lse. The reference has no backward
 * (the autograd hook is a roadmap item, ROADMAP.md:57-58); this is the
 * gradient of reference.py:56-163. Dense (B, H, L, E) operands; dK/dV are
 * summed over each grouped-query group. fp16/bf16 with E == Ev in {64, 128}
 * run on tcgen05; fp32/fp64 run on CUDA cores.
 */
pa_status pa_sdpa_bwd(const pa_sdpa_desc* desc, const void* q, const void* k, const void* v,
                      const void* out, const void* dout, const float* lse, void* dq, void* dk,
                      void* dv, void* stream);

/* ---- multi-GPU ---------------------------------------------------------- */

typedef struct pa_comm pa_comm;

/* 128-byte NCCL unique id made on one rank and shared out of band. */
pa_status pa_comm_unique_id(uint8_t id[128]);
pa_status pa_comm_init(pa_comm** comm, const uint8_t id[128], int32_t nranks, int32_t rank);
pa_status pa_comm_destroy(pa_comm* comm);
/* Wait (host side, bounded) until `stream` and the communicator's side stream
 * are idle. On an NCCL asynchronous error or when `timeout_ms` (>= 0) passes,
 * the communicator is aborted and PA_ERR_NCCL / PA_ERR_TIMEOUT is returned, so
 * a dead peer ends in an error instead of a hang. */
pa_status pa_comm_wait(pa_comm* comm, void* stream, int32_t timeout_ms);

/* Phase timing of the ring calls on `comm` (instrumentation; no reference
 * counterpart). pa_comm_profile_start clears and enables it: the following
 * pa_ring_fwd / pa_ring_bwd calls record CUDA events at phase boundaries.
 * pa_comm_profile_read waits for those events, writes the milliseconds spent
 * per phase (indexes PA_RING_PHASE_*) and disables it again. */
enum {
  PA_RING_PHASE_REPACK = 0,      /* chunk copies, fills, output stores (compute stream) */
  PA_RING_PHASE_ATTENTION = 1,   /* tensor-core kernels of every chunk pair */
  PA_RING_PHASE_ACCUMULATE = 2,  /* fp32 log-sum-exp merges / gradient accumulation */
  PA_RING_PHASE_WAIT = 3,        /* compute stream stalled on a transfer */
  PA_RING_PHASE_NCCL = 4,        /* side stream busy in NCCL send/recv */
  PA_RING_PHASES = 5
};
pa_status pa_comm_profile_start(pa_comm* comm);
pa_status pa_comm_profile_read(pa_comm* comm, float ms[PA_RING_PHASES]);

/*
 * Ring (context-parallel) causal attention over `comm`. Each rank holds its
 * zig-zag shard of the sequence: chunks r and 2n-1-r of 2n equal chunks, laid
 * out back to back as (B, H, 2*C, D). K/V shards travel around the ring with
 * NCCL send/recv on a side stream while the local block is computed; partial
 * results merge by log-sum-exp. The backward sends fp32 dK/dV accumulators
 * along with their K/V (received while the next step's first chunk pair runs)
 * and home after the last step. No reference counterpart (the reference has
 * no distributed code); the result equals reference.py:56-163 on the gathered
 * sequence.
 */
pa_status pa_ring_fwd(pa_comm* comm, const pa_sdpa_desc* local_desc, const void* q,
                      const void* k, const void* v, void* out, float* lse, void* stream);
pa_status pa_ring_bwd(pa_comm* comm, const pa_sdpa_desc* local_desc, const void* q,
                      const void* k, const void* v, const void* out, const void* dout,
                      const float* lse, void* dq, void* dk, void* dv, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PA_B200_H */
