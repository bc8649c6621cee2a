// Library plumbing behind include/pa_b200.h: errors, devices, memory,
// streams, events, the per-device status word and the tensor-map encoder.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace pa {

namespace {
thread_local std::string g_last_error;
constexpr int kMaxDevices = 64;
int* g_status_words[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};
std::mutex g_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}
}  // namespace

pa_status fail(pa_status code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

pa_status fail_cuda(cudaError_t err, const char* what) {
  std::string m = std::string(what) + ": " + cudaGetErrorName(err) + " (" +
                  cudaGetErrorString(err) + ")";
  // Clear a sticky-free error so the next call starts clean.
  cudaGetLastError();
  return fail(err == cudaErrorMemoryAllocation ? PA_ERR_NOMEM : PA_ERR_CUDA, m);
}

void clear_error() { g_last_error.clear(); }

int* device_status_word() {
  int d = current_device();
  if (d < 0 || d >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_status_words[d]) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    cudaMemset(p, 0, sizeof(int));
    cudaDeviceSynchronize();
    g_status_words[d] = p;
  }
  return g_status_words[d];
}

int sm_count() {
  int d = current_device();
  if (d < 0 || d >= kMaxDevices) return 148;
  if (!g_sm_count[d]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
    g_sm_count[d] = n > 0 ? n : 148;
  }
  return g_sm_count[d];
}

pa_status scratch_alloc(void** p, size_t bytes, cudaStream_t s) {
  *p = nullptr;
  if (bytes == 0) return PA_OK;
  {
    // Keep freed scratch cached in the device's default pool instead of
    // returning it to the driver at every synchronisation.
    static uint64_t pool_set = 0;
    const int d = current_device();
    if (d >= 0 && d < 64 && !(pool_set & (1ull << d))) {
      std::lock_guard<std::mutex> lk(g_mu);
      cudaMemPool_t pool;
      if (cudaDeviceGetDefaultMemPool(&pool, d) == cudaSuccess) {
        uint64_t keep = ~0ull;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
      }
      cudaGetLastError();
      pool_set |= 1ull << d;
    }
  }
  PA_CUDA(cudaMallocAsync(p, bytes, s));
  return PA_OK;
}

pa_status set_smem_attr_once(const void* fn, int bytes, uint64_t* mask) {
  const int d = current_device();
  const uint64_t bit = (d >= 0 && d < 64) ? (1ull << d) : 0;
  if (bit && (__atomic_load_n(mask, __ATOMIC_ACQUIRE) & bit)) return PA_OK;
  PA_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  if (bit) __atomic_fetch_or(mask, bit, __ATOMIC_RELEASE);
  return PA_OK;
}

void scratch_free(void* p, cudaStream_t s) {
  if (p) cudaFreeAsync(p, s);
}

namespace {
pa_status encoder(PFN_cuTensorMapEncodeTiled_v12000* out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
      cudaGetLastError();
      return fail(PA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    }
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  *out = g_encode;
  return PA_OK;
}
}  // namespace

pa_status encode_tma_4d(CUtensorMap* map, CUtensorMapDataType dt, const void* base,
                        const uint64_t dims[4], const uint64_t strides_bytes[3],
                        uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
  PA_TRY(encoder(&enc));
  cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t st[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  cuuint32_t box[4] = {box_inner, box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, dt, 4, const_cast<void*>(base), d, st, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[320];
    snprintf(buf, sizeof buf,
             "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu x %llu x %llu, byte strides "
             "%llu/%llu/%llu, box %u x %u (strides must be multiples of 16 bytes and the base "
             "16-byte aligned)",
             static_cast<int>(r), (unsigned long long)dims[0], (unsigned long long)dims[1],
             (unsigned long long)dims[2], (unsigned long long)dims[3],
             (unsigned long long)strides_bytes[0], (unsigned long long)strides_bytes[1],
             (unsigned long long)strides_bytes[2], box_inner, box_rows);
    return fail(PA_ERR_INVALID, buf);
  }
  return PA_OK;
}

pa_status encode_tma_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base,
                        uint64_t inner, uint64_t rows, uint64_t planes, uint64_t row_bytes,
                        uint64_t plane_bytes, uint32_t box_inner, uint32_t box_rows,
                        CUtensorMapSwizzle swz) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
  PA_TRY(encoder(&enc));
  cuuint64_t dims[3] = {inner, rows, planes};
  cuuint64_t strides[2] = {row_bytes, plane_bytes};
  cuuint32_t box[3] = {box_inner, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[256];
    snprintf(buf, sizeof buf,
             "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu x %llu, strides %llu/%llu, "
             "box %u x %u",
             static_cast<int>(r), (unsigned long long)inner, (unsigned long long)rows,
             (unsigned long long)planes, (unsigned long long)row_bytes,
             (unsigned long long)plane_bytes, box_inner, box_rows);
    return fail(PA_ERR_CUDA, buf);
  }
  return PA_OK;
}

namespace {

// One CTA of two warps. Lane 0 of warp 0 waits on an mbarrier that nothing
// arrives on, with a time bound of `limit_ns`, and gives up: it writes
// kStatusTimeoutSelfTest and raises the CTA abort flag. Lane 0 of warp 1
// waits on a second such barrier with the default bound and must leave
// through the abort flag, long before that bound. This is the give-up path of
// every pipelined kernel, run on its own.
__global__ void __launch_bounds__(64) selftest_wait_kernel(int* status, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  const int warp = threadIdx.x / 32;
  if ((threadIdx.x & 31) == 0)
    mbar_wait(&bars[warp], 0, status, kStatusTimeoutSelfTest, &abort_flag,
              warp == 0 ? limit_ns : kWaitNs);
  __syncthreads();
}

}  // namespace

}  // namespace pa

using namespace pa;

extern "C" {

pa_status pa_selftest_wait_timeout(int32_t limit_us, void* stream) {
  clear_error();
  if (limit_us < 1 || limit_us > 1000000)
    return fail(PA_ERR_INVALID, "pa_selftest_wait_timeout: limit_us must be in [1, 1000000]");
  int* status = device_status_word();
  if (!status) return fail(PA_ERR_CUDA, "device status word unavailable");
  selftest_wait_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(
      status, static_cast<uint64_t>(limit_us) * 1000ull);
  PA_CUDA(cudaGetLastError());
  return PA_OK;
}

int32_t pa_version(void) { return 100; }  // 0.1.0

const char* pa_last_error(void) { return g_last_error.c_str(); }

pa_status pa_init(int32_t* ndev) {
  clear_error();
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (ndev) *ndev = (e == cudaSuccess) ? n : 0;
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDeviceCount");
  return PA_OK;
}

pa_status pa_set_device(int32_t dev) {
  PA_CUDA(cudaSetDevice(dev));
  return PA_OK;
}

pa_status pa_get_device(int32_t* dev) {
  int d = 0;
  PA_CUDA(cudaGetDevice(&d));
  *dev = d;
  return PA_OK;
}

pa_status pa_device_status(int32_t* code) {
  // The library's word exists once a kernel on this device has used it; no
  // kernel can have written it before, so it is not allocated here (callers
  // of the allocation-free decode may call this without allocating).
  int* w = nullptr;
  {
    const int d = current_device();
    std::lock_guard<std::mutex> lk(g_mu);
    if (d >= 0 && d < kMaxDevices) w = g_status_words[d];
  }
  int v = 0;
  if (w) {
    PA_CUDA(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost));
    if (v) PA_CUDA(cudaMemset(w, 0, sizeof(int)));
  }
  int v_static = 0;
  PA_TRY(take_static_decode_status(&v_static));
  if (!v) v = v_static;
  if (code) *code = v;
  if (v) {
    char buf[96];
    if (v == kStatusBadSeqLen)
      snprintf(buf, sizeof buf, "a sequence length was outside [0, max_seq_len] (code 0x%x)", v);
    else if (v == kStatusBadPage)
      snprintf(buf, sizeof buf, "a block-table entry was outside [0, num_pages) (code 0x%x)", v);
    else
      snprintf(buf, sizeof buf, "a bounded device-side wait gave up (code 0x%x)", v);
    return fail((v & 0xf00) == 0x200 ? PA_ERR_INVALID : PA_ERR_TIMEOUT, buf);
  }
  return PA_OK;
}

pa_status pa_malloc(void** dptr, size_t bytes) {
  if (!dptr) return fail(PA_ERR_INVALID, "pa_malloc: null output pointer");
  *dptr = nullptr;
  if (bytes == 0) bytes = 1;
  PA_CUDA(cudaMalloc(dptr, bytes));
  return PA_OK;
}

pa_status pa_free(void* dptr) {
  if (dptr) PA_CUDA(cudaFree(dptr));
  return PA_OK;
}

pa_status pa_host_alloc(void** hptr, size_t bytes) {
  if (!hptr) return fail(PA_ERR_INVALID, "pa_host_alloc: null output pointer");
  *hptr = nullptr;
  if (bytes == 0) bytes = 1;
  PA_CUDA(cudaHostAlloc(hptr, bytes, cudaHostAllocPortable));
  return PA_OK;
}

pa_status pa_host_free(void* hptr) {
  if (hptr) PA_CUDA(cudaFreeHost(hptr));
  return PA_OK;
}

pa_status pa_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes) PA_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice,
                                     static_cast<cudaStream_t>(stream)));
  return PA_OK;
}

pa_status pa_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes) PA_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost,
                                     static_cast<cudaStream_t>(stream)));
  return PA_OK;
}

pa_status pa_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes) PA_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice,
                                     static_cast<cudaStream_t>(stream)));
  return PA_OK;
}

pa_status pa_memset(void* dptr, int32_t value, size_t bytes, void* stream) {
  if (bytes) PA_CUDA(cudaMemsetAsync(dptr, value, bytes, static_cast<cudaStream_t>(stream)));
  return PA_OK;
}

pa_status pa_stream_create(void** stream) {
  cudaStream_t s;
  PA_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  *stream = s;
  return PA_OK;
}

pa_status pa_stream_destroy(void* stream) {
  if (stream) PA_CUDA(cudaStreamDestroy(static_cast<cudaStream_t>(stream)));
  return PA_OK;
}

pa_status pa_stream_sync(void* stream) {
  PA_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  return PA_OK;
}

pa_status pa_event_create(void** event) {
  cudaEvent_t e;
  PA_CUDA(cudaEventCreate(&e));
  *event = e;
  return PA_OK;
}

pa_status pa_event_destroy(void* event) {
  if (event) PA_CUDA(cudaEventDestroy(static_cast<cudaEvent_t>(event)));
  return PA_OK;
}

pa_status pa_event_sync(void* event) {
  PA_CUDA(cudaEventSynchronize(static_cast<cudaEvent_t>(event)));
  return PA_OK;
}

pa_status pa_host_is_pinned(const void* ptr, int32_t* pinned) {
  if (!pinned) return fail(PA_ERR_INVALID, "pa_host_is_pinned: null output");
  *pinned = 0;
  if (!ptr) return PA_OK;
  cudaPointerAttributes at{};
  const cudaError_t e = cudaPointerGetAttributes(&at, ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();  // an address the runtime does not know: not page-locked
    return PA_OK;
  }
  *pinned = at.type == cudaMemoryTypeHost ? 1 : 0;
  return PA_OK;
}

pa_status pa_event_record(void* event, void* stream) {
  PA_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream)));
  return PA_OK;
}

pa_status pa_stream_wait_event(void* stream, void* event) {
  PA_CUDA(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), static_cast<cudaEvent_t>(event), 0));
  return PA_OK;
}

pa_status pa_event_elapsed_ms(void* start, void* stop, float* ms) {
  PA_CUDA(cudaEventSynchronize(static_cast<cudaEvent_t>(stop)));
  PA_CUDA(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start),
                               static_cast<cudaEvent_t>(stop)));
  return PA_OK;
}

}  // extern "C"
