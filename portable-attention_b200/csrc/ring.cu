// Ring (context-parallel) causal attention over NCCL.
//
// n ranks split a sequence of 2nC rows into 2n chunks of C rows; rank r owns
// chunks r and 2n-1-r (zig-zag: every rank gets the same causal work). Its
// shard is laid out back to back, (B, H, 2C, D). Forward, for t = 0..n-1:
//   the rank holds the K/V shard of source s = (r - t) mod n; while the
//   compute stream runs the tensor-core forward for every (query chunk,
//   key chunk) pair with key chunk <= query chunk (diagonal pairs causal,
//   the others full), the side stream sends the held K/V to r+1 and receives
//   the next one from r-1 (ncclSend/ncclRecv, double-buffered). Each pair's
//   (O, lse) merges into fp32 accumulators by log-sum-exp.
// Backward: same rotation; each pair runs the tensor-core backward with the
//   global lse and O of the forward, its kernels adding the pair's dQ, dK, dV
//   in fp32 straight into accumulators (dQ local, dK/dV travelling with their
//   K/V, sent after the step's compute and received while the next step's
//   first dQ kernel runs), one extra hop bringing dK/dV home at the end.
// Chunks are copied into dense (B, H, C, D) buffers (pitched 2-D copies) so
// the single-GPU kernels run unchanged on them.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <mutex>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"
#include "kernels.h"

struct pa_comm {
  ncclComm_t nccl;
  int nranks, rank, device;
  cudaStream_t side;
  cudaEvent_t ev[4];
  // Second compute stream of the forward (query chunk 1's pairs) and its
  // fork / join events.
  cudaStream_t side2;
  cudaEvent_t fj[2];
  // Phase timing (pa_comm_profile_start / _read): events recorded at phase
  // boundaries on the compute stream (marks[0]) and the side stream (marks[1]);
  // the time from one mark to the next on a stream belongs to the first mark's
  // phase. Off unless started; events come from a pool kept for reuse.
  bool profiling;
  std::vector<std::pair<int, cudaEvent_t>> marks[2];
  std::vector<cudaEvent_t> event_pool;
  size_t pool_used;
};

namespace pa {
namespace {

// NCCL is loaded on first use, not linked: the process may already hold a
// different libnccl.so.2 (a framework's own build), and two copies under one
// soname break whichever loads second. Preference: a libnccl.so.2 already in
// the process, then $PA_B200_NCCL, then the default search path.
struct Nccl {
  decltype(&ncclGetUniqueId) GetUniqueId;
  decltype(&ncclCommInitRank) CommInitRank;
  decltype(&ncclCommDestroy) CommDestroy;
  decltype(&ncclCommAbort) CommAbort;
  decltype(&ncclCommGetAsyncError) CommGetAsyncError;
  decltype(&ncclGetErrorString) GetErrorString;
  decltype(&ncclGroupStart) GroupStart;
  decltype(&ncclGroupEnd) GroupEnd;
  decltype(&ncclSend) Send;
  decltype(&ncclRecv) Recv;
};
Nccl g_nccl;
bool g_nccl_ok = false;
std::mutex g_nccl_mu;

pa_status load_nccl() {
  std::lock_guard<std::mutex> lk(g_nccl_mu);
  if (g_nccl_ok) return PA_OK;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  const char* env = getenv("PA_B200_NCCL");
  if (!h && env && *env) h = dlopen(env, RTLD_NOW | RTLD_LOCAL);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
  if (!h) return fail(PA_ERR_NCCL, std::string("cannot load libnccl.so.2: ") + dlerror());
  bool ok = true;
  auto sym = [&](auto& fp, const char* name) {
    fp = reinterpret_cast<std::remove_reference_t<decltype(fp)>>(dlsym(h, name));
    ok = ok && fp != nullptr;
  };
  sym(g_nccl.GetUniqueId, "ncclGetUniqueId");
  sym(g_nccl.CommInitRank, "ncclCommInitRank");
  sym(g_nccl.CommDestroy, "ncclCommDestroy");
  sym(g_nccl.CommAbort, "ncclCommAbort");
  sym(g_nccl.CommGetAsyncError, "ncclCommGetAsyncError");
  sym(g_nccl.GetErrorString, "ncclGetErrorString");
  sym(g_nccl.GroupStart, "ncclGroupStart");
  sym(g_nccl.GroupEnd, "ncclGroupEnd");
  sym(g_nccl.Send, "ncclSend");
  sym(g_nccl.Recv, "ncclRecv");
  if (!ok) return fail(PA_ERR_NCCL, "libnccl.so.2 lacks a required symbol");
  g_nccl_ok = true;
  return PA_OK;
}

pa_status fail_nccl(ncclResult_t r, const char* what) {
  const char* msg = g_nccl_ok ? g_nccl.GetErrorString(r) : "NCCL not loaded";
  return fail(PA_ERR_NCCL, std::string(what) + ": " + msg);
}

#define PA_NCCL(call)                                    \
  do {                                                   \
    ncclResult_t r_ = (call);                            \
    if (r_ != ncclSuccess) return fail_nccl(r_, #call);  \
  } while (0)

// acc (fp32 rows x D, lse fp32) <- merge(acc, part (fp16/bf16 rows, lse)).
template <bool BF16>
__global__ void ring_merge_kernel(const void* part_o, const float* part_lse, float* acc_o,
                                  float* acc_lse, int64_t rows, int D) {
  const int64_t r = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const float la = acc_lse[r], lb = part_lse[r];
  const float m = fmaxf(la, lb);
  if (m == -INFINITY) return;  // nothing seen yet by either side
  const float wa = la == -INFINITY ? 0.f : __expf(la - m);
  const float wb = lb == -INFINITY ? 0.f : __expf(lb - m);
  const float inv = 1.f / (wa + wb);
  for (int c = lane; c < D; c += 32) {
    float pb;
    if (BF16) pb = __bfloat162float(static_cast<const __nv_bfloat16*>(part_o)[r * D + c]);
    else pb = __half2float(static_cast<const __half*>(part_o)[r * D + c]);
    acc_o[r * D + c] = (acc_o[r * D + c] * wa + pb * wb) * inv;
  }
  if (lane == 0) acc_lse[r] = m + __logf(wa + wb);
}

// out rows of one chunk <- acc (fp32) as fp16/bf16; chunk rows are strided
// inside the (B, H, 2C, D) shard.
template <bool BF16>
__global__ void ring_store_kernel(const float* acc, void* out, int64_t planes, int64_t C, int D,
                                  int64_t plane_stride_rows, int64_t row0) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t total = planes * C * D;
  if (i >= total) return;
  const int64_t p = i / (C * D), rem = i % (C * D);
  const int64_t dst = (p * plane_stride_rows + row0) * D + rem;
  if (BF16) static_cast<__nv_bfloat16*>(out)[dst] = __float2bfloat16_rn(acc[i]);
  else static_cast<__half*>(out)[dst] = __float2half_rn(acc[i]);
}

__global__ void fill_f32_kernel(float* p, float v, int64_t n) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < n) p[i] = v;
}

unsigned blocks_for(int64_t n, int threads) { return static_cast<unsigned>((n + threads - 1) / threads); }

// Phases of a ring call, for pa_comm_profile_read (PA_RING_PHASE_* in the header).
enum { kPhCopy = 0, kPhAttn = 1, kPhAccum = 2, kPhWait = 3, kPhNccl = 4, kPhEnd = 5 };

// Records a phase boundary on `st` (0: compute stream, 1: side stream) when
// profiling is on.
void mark(pa_comm* c, int which, int phase, cudaStream_t st) {
  if (!c->profiling) return;
  if (c->pool_used == c->event_pool.size()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) {
      cudaGetLastError();
      return;
    }
    c->event_pool.push_back(e);
  }
  cudaEvent_t e = c->event_pool[c->pool_used++];
  cudaEventRecord(e, st);
  c->marks[which].push_back({phase, e});
}

// Dense (B, H, C, D) descriptor for one chunk pair.
pa_sdpa_desc chunk_desc(const pa_sdpa_desc& d, int64_t C, int causal) {
  pa_sdpa_desc c = d;
  c.L = C;
  c.S = C;
  int64_t H = d.lead[d.nlead - 1];
  int64_t g = d.gqa_group > 1 ? d.gqa_group : 1;
  int64_t Hkv = H / g;
  int64_t qs = C * d.E, ks = C * d.E;
  for (int i = d.nlead - 1; i >= 0; --i) {
    const int64_t dim = d.lead[i];
    const int64_t kdim = (i == d.nlead - 1) ? Hkv : dim;
    c.q_lead_stride[i] = dim > 1 ? qs : 0;
    c.k_lead_stride[i] = kdim > 1 ? ks : 0;
    c.v_lead_stride[i] = kdim > 1 ? ks : 0;
    if (i == d.nlead - 1 && g > 1) {
      c.k_lead_stride[i] = ks;
      c.v_lead_stride[i] = ks;
    }
    qs *= dim;
    ks *= kdim;
  }
  c.is_causal = causal;
  return c;
}

struct RingShape {
  int64_t planes_q, planes_kv, C, D;
  size_t q_chunk, kv_chunk;  // elements per chunk buffer
};

pa_status ring_shape(const pa_comm* comm, const pa_sdpa_desc& d, RingShape* s) {
  if (!comm) return fail(PA_ERR_INVALID, "ring: null communicator");
  if (!comm->nccl) return fail(PA_ERR_NCCL, "ring: the communicator was aborted after an error or time-out");
  if (d.dtype != PA_F16 && d.dtype != PA_BF16) return fail(PA_ERR_UNSUPPORTED, "ring: fp16/bf16 only");
  if (!d.is_causal) return fail(PA_ERR_UNSUPPORTED, "ring: causal attention only");
  if (d.L != d.S || d.L % 2) return fail(PA_ERR_INVALID, "ring: local shard must be 2*C rows of q and k");
  int64_t n, H, Hkv;
  if (!dense_bhsd(d, &n, &H, &Hkv) || d.nlead < 1)
    return fail(PA_ERR_UNSUPPORTED, "ring: operands must be dense (B, H, 2C, D)");
  if (d.E != d.Ev || (d.E != 64 && d.E != 128)) return fail(PA_ERR_UNSUPPORTED, "ring: head dim 64/128");
  s->planes_q = n;
  s->planes_kv = (n / H) * Hkv;
  s->C = d.L / 2;
  s->D = d.E;
  s->q_chunk = static_cast<size_t>(n * s->C * s->D);
  s->kv_chunk = static_cast<size_t>(s->planes_kv * s->C * s->D);
  return PA_OK;
}

// Copy chunk `which` (0: rows [0,C), 1: rows [C,2C)) of every plane of a
// (planes, 2C, D) shard into a dense (planes, C, D) buffer.
pa_status chunk_copy(void* dense, const void* shard, int64_t planes, int64_t C, int64_t D, size_t es,
                     int which, cudaStream_t st) {
  const size_t w = static_cast<size_t>(C * D) * es;
  PA_CUDA(cudaMemcpy2DAsync(dense, w, static_cast<const uint8_t*>(shard) + which * w, 2 * w, w, planes,
                            cudaMemcpyDeviceToDevice, st));
  return PA_OK;
}

// Owned chunk ids of rank r: {r, 2n-1-r}.
inline int chunk_id(int n, int r, int which) { return which == 0 ? r : 2 * n - 1 - r; }

}  // namespace
}  // namespace pa

using namespace pa;

extern "C" {

pa_status pa_comm_unique_id(uint8_t id[128]) {
  clear_error();
  static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
  PA_TRY(load_nccl());
  ncclUniqueId u;
  PA_NCCL(g_nccl.GetUniqueId(&u));
  std::memcpy(id, &u, 128);
  return PA_OK;
}

pa_status pa_comm_init(pa_comm** out, const uint8_t id[128], int32_t nranks, int32_t rank) {
  clear_error();
  if (!out || !id || nranks < 1 || rank < 0 || rank >= nranks) return fail(PA_ERR_INVALID, "pa_comm_init: bad arguments");
  PA_TRY(load_nccl());
  auto* c = new pa_comm{};
  c->nranks = nranks;
  c->rank = rank;
  cudaGetDevice(&c->device);
  ncclUniqueId u;
  std::memcpy(&u, id, 128);
  ncclResult_t r = g_nccl.CommInitRank(&c->nccl, nranks, u, rank);
  if (r != ncclSuccess) {
    delete c;
    return fail_nccl(r, "ncclCommInitRank");
  }
  if (cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&c->side2, cudaStreamNonBlocking) != cudaSuccess) {
    g_nccl.CommDestroy(c->nccl);
    delete c;
    return fail(PA_ERR_CUDA, "pa_comm_init: side streams");
  }
  for (auto& e : c->ev) cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
  for (auto& e : c->fj) cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
  *out = c;
  return PA_OK;
}

pa_status pa_comm_destroy(pa_comm* c) {
  if (!c) return PA_OK;
  cudaStreamSynchronize(c->side);
  cudaStreamSynchronize(c->side2);
  for (auto& e : c->ev) cudaEventDestroy(e);
  for (auto& e : c->fj) cudaEventDestroy(e);
  cudaStreamDestroy(c->side2);
  for (auto& e : c->event_pool) cudaEventDestroy(e);
  cudaStreamDestroy(c->side);
  // An aborted communicator (pa_comm_wait) is already freed.
  ncclResult_t r = c->nccl ? g_nccl.CommDestroy(c->nccl) : ncclSuccess;
  delete c;
  if (r != ncclSuccess) return fail_nccl(r, "ncclCommDestroy");
  return PA_OK;
}

pa_status pa_comm_wait(pa_comm* c, void* stream, int32_t timeout_ms) {
  clear_error();
  if (!c) return fail(PA_ERR_INVALID, "null communicator");
  if (!c->nccl) return fail(PA_ERR_NCCL, "the communicator was aborted after an error or time-out");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t q1 = cudaStreamQuery(st), q2 = cudaStreamQuery(c->side);
    if (q1 == cudaSuccess && q2 == cudaSuccess) return PA_OK;
    if ((q1 != cudaSuccess && q1 != cudaErrorNotReady) || (q2 != cudaSuccess && q2 != cudaErrorNotReady))
      return fail_cuda(q1 != cudaSuccess && q1 != cudaErrorNotReady ? q1 : q2, "pa_comm_wait");
    ncclResult_t async = ncclSuccess;
    g_nccl.CommGetAsyncError(c->nccl, &async);
    if (async != ncclSuccess && async != ncclInProgress) {
      g_nccl.CommAbort(c->nccl);
      c->nccl = nullptr;
      return fail_nccl(async, "NCCL asynchronous error (communicator aborted)");
    }
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                        std::chrono::steady_clock::now() - t0).count();
    if (timeout_ms >= 0 && ms > timeout_ms) {
      g_nccl.CommAbort(c->nccl);
      c->nccl = nullptr;
      return fail(PA_ERR_TIMEOUT, "ring: peers did not complete in time (communicator aborted)");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

pa_status pa_comm_profile_start(pa_comm* c) {
  clear_error();
  if (!c) return fail(PA_ERR_INVALID, "null communicator");
  c->marks[0].clear();
  c->marks[1].clear();
  c->pool_used = 0;
  c->profiling = true;
  return PA_OK;
}

pa_status pa_comm_profile_read(pa_comm* c, float ms[PA_RING_PHASES]) {
  clear_error();
  if (!c || !ms) return fail(PA_ERR_INVALID, "null argument");
  for (int i = 0; i < PA_RING_PHASES; ++i) ms[i] = 0.f;
  for (int w = 0; w < 2; ++w) {
    const auto& m = c->marks[w];
    if (!m.empty()) PA_CUDA(cudaEventSynchronize(m.back().second));
    for (size_t i = 0; i + 1 < m.size(); ++i) {
      if (m[i].first == kPhEnd) continue;
      float t = 0.f;
      PA_CUDA(cudaEventElapsedTime(&t, m[i].second, m[i + 1].second));
      ms[m[i].first] += t;
    }
  }
  c->profiling = false;
  c->marks[0].clear();
  c->marks[1].clear();
  c->pool_used = 0;
  return PA_OK;
}

pa_status pa_ring_fwd(pa_comm* comm, const pa_sdpa_desc* desc, const void* q, const void* k,
                      const void* v, void* out, float* lse, void* stream) {
  clear_error();
  PA_TRY(check_desc(desc));
  const pa_sdpa_desc& d = *desc;
  RingShape sh;
  PA_TRY(ring_shape(comm, d, &sh));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int n = comm->nranks, r = comm->rank;
  const size_t es = 2;
  const bool bf16 = d.dtype == PA_BF16;
  const int64_t C = sh.C, D = sh.D;
  const size_t qb = sh.q_chunk * es, kvb = sh.kv_chunk * es;
  const int64_t rows = sh.planes_q * C;
  // scratch: q chunks [2], kv ring buffers [2] x (K0,K1,V0,V1), part out [2], part lse [2],
  // acc o [2], acc lse [2] (one part buffer per compute stream)
  const size_t bytes = 2 * qb + 2 * 4 * kvb + 2 * qb + 2 * rows * 4 + 2 * rows * D * 4 + 2 * rows * 4 + 4096;
  uint8_t* ws = nullptr;
  PA_TRY(scratch_alloc(reinterpret_cast<void**>(&ws), bytes, st));
  auto align = [](size_t x) { return (x + 255) & ~size_t(255); };
  size_t off = 0;
  auto take = [&](size_t b) { uint8_t* p = ws + off; off += align(b); return p; };
  uint8_t* qc[2] = {take(qb), take(qb)};
  uint8_t* kvbuf[2] = {take(4 * kvb), take(4 * kvb)};
  uint8_t* part_o[2] = {take(qb), take(qb)};
  float* part_lse[2] = {reinterpret_cast<float*>(take(rows * 4)), reinterpret_cast<float*>(take(rows * 4))};
  float* acc_o[2] = {reinterpret_cast<float*>(take(rows * D * 4)), reinterpret_cast<float*>(take(rows * D * 4))};
  float* acc_l[2] = {reinterpret_cast<float*>(take(rows * 4)), reinterpret_cast<float*>(take(rows * 4))};
  pa_status rc = PA_OK;
  do {
    mark(comm, 0, kPhCopy, st);
    for (int w = 0; w < 2 && rc == PA_OK; ++w) {
      rc = chunk_copy(qc[w], q, sh.planes_q, C, D, es, w, st);
      if (rc == PA_OK) rc = chunk_copy(kvbuf[0] + w * kvb, k, sh.planes_kv, C, D, es, w, st);
      if (rc == PA_OK) rc = chunk_copy(kvbuf[0] + (2 + w) * kvb, v, sh.planes_kv, C, D, es, w, st);
      fill_f32_kernel<<<blocks_for(rows * D, 256), 256, 0, st>>>(acc_o[w], 0.f, rows * D);
      fill_f32_kernel<<<blocks_for(rows, 256), 256, 0, st>>>(acc_l[w], -INFINITY, rows);
    }
    if (rc != PA_OK) break;
    for (int t = 0; t < n && rc == PA_OK; ++t) {
      const int src = ((r - t) % n + n) % n;
      const int cur = t & 1, nxt = cur ^ 1;
      if (t + 1 < n) {
        // The side stream may overwrite kvbuf[nxt] only after the compute that
        // read it (step t-1) and the copies above are done.
        cudaEventRecord(comm->ev[0], st);
        cudaStreamWaitEvent(comm->side, comm->ev[0], 0);
        mark(comm, 1, kPhNccl, comm->side);
        g_nccl.GroupStart();
        g_nccl.Send(kvbuf[cur], 4 * kvb, ncclUint8, (r + 1) % n, comm->nccl, comm->side);
        g_nccl.Recv(kvbuf[nxt], 4 * kvb, ncclUint8, (r - 1 + n) % n, comm->nccl, comm->side);
        ncclResult_t nr = g_nccl.GroupEnd();
        if (nr != ncclSuccess) {
          rc = fail_nccl(nr, "ring send/recv");
          break;
        }
        mark(comm, 1, kPhEnd, comm->side);
        cudaEventRecord(comm->ev[1], comm->side);
      }
      // The two query chunks' pairs touch disjoint accumulators: chunk 1's run on
      // a second compute stream beside chunk 0's, so one persistent launch's
      // tail overlaps the other's work.
      cudaEventRecord(comm->fj[0], st);
      cudaStreamWaitEvent(comm->side2, comm->fj[0], 0);
      for (int qw = 0; qw < 2 && rc == PA_OK; ++qw) {
        const int qid = chunk_id(n, r, qw);
        cudaStream_t sq = qw == 0 ? st : comm->side2;
        for (int kw = 0; kw < 2 && rc == PA_OK; ++kw) {
          const int kid = chunk_id(n, src, kw);
          if (kid > qid) continue;
          pa_sdpa_desc cd = chunk_desc(d, C, kid == qid);
          if (qw == 0) mark(comm, 0, kPhAttn, st);
          rc = launch_fwd_tc(cd, qc[qw], kvbuf[cur] + kw * kvb, kvbuf[cur] + (2 + kw) * kvb, nullptr,
                             part_o[qw], part_lse[qw], sq);
          if (rc != PA_OK) break;
          if (qw == 0) mark(comm, 0, kPhAccum, st);
          if (bf16)
            ring_merge_kernel<true><<<blocks_for(rows * 32, 256), 256, 0, sq>>>(part_o[qw], part_lse[qw], acc_o[qw],
                                                                                acc_l[qw], rows, static_cast<int>(D));
          else
            ring_merge_kernel<false><<<blocks_for(rows * 32, 256), 256, 0, sq>>>(part_o[qw], part_lse[qw], acc_o[qw],
                                                                                 acc_l[qw], rows, static_cast<int>(D));
        }
      }
      cudaEventRecord(comm->fj[1], comm->side2);
      mark(comm, 0, kPhAttn, st);  // waiting for chunk 1's pairs
      cudaStreamWaitEvent(st, comm->fj[1], 0);
      if (rc != PA_OK) break;
      if (t + 1 < n) {
        mark(comm, 0, kPhWait, st);
        cudaStreamWaitEvent(st, comm->ev[1], 0);
      }
    }
    if (rc != PA_OK) break;
    mark(comm, 0, kPhCopy, st);
    for (int w = 0; w < 2; ++w) {
      if (bf16)
        ring_store_kernel<true><<<blocks_for(rows * D, 256), 256, 0, st>>>(acc_o[w], out, sh.planes_q, C,
                                                                          static_cast<int>(D), 2 * C, w * C);
      else
        ring_store_kernel<false><<<blocks_for(rows * D, 256), 256, 0, st>>>(acc_o[w], out, sh.planes_q, C,
                                                                           static_cast<int>(D), 2 * C, w * C);
      if (lse)
        PA_CUDA(cudaMemcpy2DAsync(lse + w * C, 2 * C * 4, acc_l[w], C * 4, C * 4, sh.planes_q,
                                  cudaMemcpyDeviceToDevice, st));
    }
    mark(comm, 0, kPhEnd, st);
    if (cudaGetLastError() != cudaSuccess) rc = fail(PA_ERR_CUDA, "ring forward launch failed");
  } while (false);
  scratch_free(ws, st);
  return rc;
}

pa_status pa_ring_bwd(pa_comm* comm, const pa_sdpa_desc* desc, const void* q, const void* k,
                      const void* v, const void* out, const void* dout, const float* lse,
                      void* dq, void* dk, void* dv, void* stream) {
  clear_error();
  PA_TRY(check_desc(desc));
  const pa_sdpa_desc& d = *desc;
  RingShape sh;
  PA_TRY(ring_shape(comm, d, &sh));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int n = comm->nranks, r = comm->rank;
  const size_t es = 2;
  const bool bf16 = d.dtype == PA_BF16;
  const int64_t C = sh.C, D = sh.D;
  const size_t qb = sh.q_chunk * es, kvb = sh.kv_chunk * es;
  const int64_t rows = sh.planes_q * C;
  const int64_t kv_elems = static_cast<int64_t>(sh.kv_chunk);
  // Per ring buffer: K0, K1, V0, V1 (fp16) then dK0, dK1, dV0, dV1 (fp32).
  const size_t ring_bytes = 4 * kvb + 4 * sh.kv_chunk * 4;
  auto align = [](size_t x) { return (x + 255) & ~size_t(255); };
  const size_t bytes = 3 * 2 * align(qb) + 2 * align(rows * 4) + 2 * align(ring_bytes) +
                       2 * align(rows * D * 4) + 4096;
  uint8_t* ws = nullptr;
  PA_TRY(scratch_alloc(reinterpret_cast<void**>(&ws), bytes, st));
  size_t off = 0;
  auto take = [&](size_t b) { uint8_t* p = ws + off; off += align(b); return p; };
  uint8_t* qc[2] = {take(qb), take(qb)};
  uint8_t* oc[2] = {take(qb), take(qb)};
  uint8_t* doc[2] = {take(qb), take(qb)};
  float* lc[2] = {reinterpret_cast<float*>(take(rows * 4)), reinterpret_cast<float*>(take(rows * 4))};
  uint8_t* ring[2] = {take(ring_bytes), take(ring_bytes)};
  float* dq_acc[2] = {reinterpret_cast<float*>(take(rows * D * 4)), reinterpret_cast<float*>(take(rows * D * 4))};
  auto kptr = [&](int b, int w) { return ring[b] + w * kvb; };
  auto vptr = [&](int b, int w) { return ring[b] + (2 + w) * kvb; };
  auto dkacc = [&](int b, int w) { return reinterpret_cast<float*>(ring[b] + 4 * kvb) + w * kv_elems; };
  auto dvacc = [&](int b, int w) { return reinterpret_cast<float*>(ring[b] + 4 * kvb) + (2 + w) * kv_elems; };
  pa_status rc = PA_OK;
  do {
    mark(comm, 0, kPhCopy, st);
    for (int w = 0; w < 2 && rc == PA_OK; ++w) {
      rc = chunk_copy(qc[w], q, sh.planes_q, C, D, es, w, st);
      if (rc == PA_OK) rc = chunk_copy(oc[w], out, sh.planes_q, C, D, es, w, st);
      if (rc == PA_OK) rc = chunk_copy(doc[w], dout, sh.planes_q, C, D, es, w, st);
      if (rc == PA_OK) rc = chunk_copy(kptr(0, w), k, sh.planes_kv, C, D, es, w, st);
      if (rc == PA_OK) rc = chunk_copy(vptr(0, w), v, sh.planes_kv, C, D, es, w, st);
      if (rc == PA_OK)
        PA_CUDA(cudaMemcpy2DAsync(lc[w], C * 4, lse + w * C, 2 * C * 4, C * 4, sh.planes_q,
                                  cudaMemcpyDeviceToDevice, st));
      fill_f32_kernel<<<blocks_for(rows * D, 256), 256, 0, st>>>(dq_acc[w], 0.f, rows * D);
    }
    if (rc != PA_OK) break;
    PA_CUDA(cudaMemsetAsync(ring[0] + 4 * kvb, 0, 4 * sh.kv_chunk * 4, st));
    // Side-stream order (every rank the same, so the point-to-point operations
    // between neighbours match in order): at the start of step t the K/V group
    // for step t+1 (send to r+1, receive from r-1); after step t's compute the
    // dK/dV group: send the held block's fp32 accumulators on to r+1 and
    // receive, from r-1, those of the block held in step t+1 (after the last
    // step: this rank's own block, home). Each send is grouped with a receive
    // so every rank's group progresses together: a lone send waits for its
    // receiver, and a receiver queued behind its own lone send would wait in a
    // cycle. The compute stream waits for the incoming accumulators only
    // before its first accumulation into them, so the transfer overlaps the
    // next step's first chunk-pair backward.
    for (int t = 0; t < n && rc == PA_OK; ++t) {
      const int src = ((r - t) % n + n) % n;
      const int cur = t & 1, nxt = cur ^ 1;
      if (t + 1 < n) {
        // ring[nxt]'s K/V were last read by the compute of step t-1.
        cudaEventRecord(comm->ev[0], st);
        cudaStreamWaitEvent(comm->side, comm->ev[0], 0);
        mark(comm, 1, kPhNccl, comm->side);
        g_nccl.GroupStart();
        g_nccl.Send(ring[cur], 4 * kvb, ncclUint8, (r + 1) % n, comm->nccl, comm->side);
        g_nccl.Recv(ring[nxt], 4 * kvb, ncclUint8, (r - 1 + n) % n, comm->nccl, comm->side);
        ncclResult_t nr = g_nccl.GroupEnd();
        if (nr != ncclSuccess) {
          rc = fail_nccl(nr, "ring K/V send/recv");
          break;
        }
        mark(comm, 1, kPhEnd, comm->side);
        cudaEventRecord(comm->ev[3], comm->side);
      }
      bool have_acc = t == 0;  // step 0's accumulators start at zero (memset above)
      for (int qw = 0; qw < 2 && rc == PA_OK; ++qw) {
        const int qid = chunk_id(n, r, qw);
        for (int kw = 0; kw < 2 && rc == PA_OK; ++kw) {
          const int kid = chunk_id(n, src, kw);
          if (kid > qid) continue;
          pa_sdpa_desc cd = chunk_desc(d, C, kid == qid);
          mark(comm, 0, kPhAttn, st);
          // The pair's gradients are added in fp32 by the backward kernels' own
          // epilogues. Its dQ kernel runs first; before the step's first dK/dV
          // kernel the stream waits for the incoming accumulators, so their
          // transfer overlaps that dQ kernel.
          const std::function<void()> wait_acc = [&]() {
            if (have_acc) return;
            mark(comm, 0, kPhWait, st);
            cudaStreamWaitEvent(st, comm->ev[1], 0);
            mark(comm, 0, kPhAttn, st);
            have_acc = true;
          };
          rc = bwd_accumulate(cd, qc[qw], kptr(cur, kw), vptr(cur, kw), oc[qw], doc[qw], lc[qw], dq_acc[qw],
                              dkacc(cur, kw), dvacc(cur, kw), st, wait_acc);
          if (rc != PA_OK) break;
        }
      }
      if (rc != PA_OK) break;
      if (!have_acc) {
        mark(comm, 0, kPhWait, st);
        cudaStreamWaitEvent(st, comm->ev[1], 0);
      }
      if (n > 1) {
        // ring[nxt]'s accumulators were sent on in step t-1's group, earlier on
        // this same side stream, so they may be overwritten here.
        cudaEventRecord(comm->ev[2], st);
        cudaStreamWaitEvent(comm->side, comm->ev[2], 0);
        mark(comm, 1, kPhNccl, comm->side);
        g_nccl.GroupStart();
        g_nccl.Send(ring[cur] + 4 * kvb, 4 * sh.kv_chunk * 4, ncclUint8, (r + 1) % n, comm->nccl,
                    comm->side);
        g_nccl.Recv(ring[nxt] + 4 * kvb, 4 * sh.kv_chunk * 4, ncclUint8, (r - 1 + n) % n, comm->nccl,
                    comm->side);
        ncclResult_t nr = g_nccl.GroupEnd();
        if (nr != ncclSuccess) {
          rc = fail_nccl(nr, "ring dK/dV send/recv");
          break;
        }
        mark(comm, 1, kPhEnd, comm->side);
        cudaEventRecord(comm->ev[1], comm->side);
      }
      if (t + 1 < n) {
        mark(comm, 0, kPhWait, st);
        cudaStreamWaitEvent(st, comm->ev[3], 0);
      }
    }
    if (rc != PA_OK) break;
    // After the last group this rank's own accumulators sit in ring[n & 1]; with
    // one rank they never left ring[0].
    const int home = n > 1 ? (n & 1) : 0;
    if (n > 1) {
      mark(comm, 0, kPhWait, st);
      cudaStreamWaitEvent(st, comm->ev[1], 0);
    }
    mark(comm, 0, kPhCopy, st);
    for (int w = 0; w < 2; ++w) {
      if (bf16) {
        ring_store_kernel<true><<<blocks_for(rows * D, 256), 256, 0, st>>>(dq_acc[w], dq, sh.planes_q, C,
                                                                          static_cast<int>(D), 2 * C, w * C);
        ring_store_kernel<true><<<blocks_for(kv_elems, 256), 256, 0, st>>>(dkacc(home, w), dk, sh.planes_kv, C,
                                                                          static_cast<int>(D), 2 * C, w * C);
        ring_store_kernel<true><<<blocks_for(kv_elems, 256), 256, 0, st>>>(dvacc(home, w), dv, sh.planes_kv, C,
                                                                          static_cast<int>(D), 2 * C, w * C);
      } else {
        ring_store_kernel<false><<<blocks_for(rows * D, 256), 256, 0, st>>>(dq_acc[w], dq, sh.planes_q, C,
                                                                           static_cast<int>(D), 2 * C, w * C);
        ring_store_kernel<false><<<blocks_for(kv_elems, 256), 256, 0, st>>>(dkacc(home, w), dk, sh.planes_kv, C,
                                                                           static_cast<int>(D), 2 * C, w * C);
        ring_store_kernel<false><<<blocks_for(kv_elems, 256), 256, 0, st>>>(dvacc(home, w), dv, sh.planes_kv, C,
                                                                           static_cast<int>(D), 2 * C, w * C);
      }
    }
    mark(comm, 0, kPhEnd, st);
    if (cudaGetLastError() != cudaSuccess) rc = fail(PA_ERR_CUDA, "ring backward launch failed");
  } while (false);
  scratch_free(ws, st);
  return rc;
}

}  // extern "C"
