// pa_shard_fwd: one forward call spread over several GPUs of this process.
//
// The problem's first leading dimension (the batch) is cut into contiguous
// shards, one per device. Shards are independent (no data moves between
// GPUs): each device copies its rows of q, k, v (and of the mask when the
// mask has a batch dimension; a mask broadcast over the batch is copied
// whole) from host memory, runs the same kernels as pa_sdpa_fwd /
// pa_decode_fwd on them, and copies its rows of out and lse back. One host
// thread drives each device, so the copies of different devices overlap even
// from pageable host memory, each over its own PCIe link.
//
// When the first leading dimension is also the grouped-query head axis,
// shard boundaries fall on whole groups and each device gets the key/value
// heads its query heads use.
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace pa {
namespace {

size_t dtype_bytes(int32_t dt) {
  switch (dt) {
    case PA_F16:
    case PA_BF16: return 2;
    case PA_F32: return 4;
    case PA_F64: return 8;
    case PA_BOOL: return 1;
    default: return 0;
  }
}

// Elements spanned by one index of leading dim 0 (all other dims at full
// extent): 1 + sum over the other dims of (extent - 1) * stride.
int64_t inner_span(const pa_sdpa_desc& d, const int64_t* lead_stride, int64_t rows, int64_t row_stride,
                   int64_t cols, int64_t col_stride, int kv_axis_div) {
  int64_t span = 1;
  for (int i = 1; i < d.nlead; ++i) {
    int64_t ext = d.lead[i];
    if (i == kv_axis_div) ext /= d.gqa_group;
    if (ext > 0) span += (ext - 1) * lead_stride[i];
  }
  if (rows > 0) span += (rows - 1) * row_stride;
  if (cols > 0) span += (cols - 1) * col_stride;
  return span;
}

struct Operand {
  const uint8_t* host;
  size_t esz;
  int64_t stride0;  // elements between consecutive indices of leading dim 0 (0: broadcast)
  int64_t span;     // elements spanned by one index of dim 0
  bool present;
};

// Bytes [first, last) of the host buffer that rows [r0, r0 + n) of dim 0 cover.
void shard_range(const Operand& o, int64_t r0, int64_t n, size_t* off, size_t* bytes) {
  if (o.stride0 == 0) {
    *off = 0;
    *bytes = static_cast<size_t>(o.span) * o.esz;
    return;
  }
  *off = static_cast<size_t>(r0 * o.stride0) * o.esz;
  *bytes = static_cast<size_t>((n - 1) * o.stride0 + o.span) * o.esz;
}

struct Job {
  int device;
  int64_t r0, n, kr0, kn;  // query rows and key/value rows of dim 0
  pa_status status = PA_OK;
  std::string message;
};

pa_status run_shard(const pa_sdpa_desc& d, const Operand& q, const Operand& k, const Operand& v,
                    const Operand& m, uint8_t* out, float* lse, size_t out_row_bytes,
                    size_t lse_row_elems, Job& j) {
  PA_CUDA(cudaSetDevice(j.device));
  cudaStream_t st;
  PA_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  pa_sdpa_desc sd = d;
  sd.lead[0] = j.n;
  size_t qo, qb, ko, kb, vo, vb, mo = 0, mb = 0;
  shard_range(q, j.r0, j.n, &qo, &qb);
  shard_range(k, j.kr0, j.kn, &ko, &kb);
  shard_range(v, j.kr0, j.kn, &vo, &vb);
  if (m.present) shard_range(m, j.r0, j.n, &mo, &mb);
  const size_t ob = static_cast<size_t>(j.n) * out_row_bytes;
  const size_t lb = lse ? static_cast<size_t>(j.n) * lse_row_elems * sizeof(float) : 0;
  const size_t sizes[6] = {qb, kb, vb, mb, ob, lb};
  void* buf[6] = {};
  pa_status rc = PA_OK;
  for (int i = 0; i < 6 && rc == PA_OK; ++i) rc = scratch_alloc(&buf[i], sizes[i], st);
  auto h2d = [&](void* dst, const uint8_t* src, size_t bytes) -> pa_status {
    if (bytes) PA_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, st));
    return PA_OK;
  };
  if (rc == PA_OK) rc = h2d(buf[0], q.host + qo, qb);
  if (rc == PA_OK) rc = h2d(buf[1], k.host + ko, kb);
  if (rc == PA_OK) rc = h2d(buf[2], v.host + vo, vb);
  if (rc == PA_OK && m.present) rc = h2d(buf[3], m.host + mo, mb);
  if (rc == PA_OK) {
    size_t ws = 0;
    const bool decode = sd.L == 1 && decode_ws_bytes(sd, &ws) == PA_OK;
    clear_error();
    if (decode) {
      void* w = nullptr;
      rc = scratch_alloc(&w, ws, st);
      if (rc == PA_OK) rc = run_decode(sd, buf[0], buf[1], buf[2], buf[4], static_cast<float*>(buf[5]), w, ws, st);
      scratch_free(w, st);
    } else {
      rc = pa_sdpa_fwd(&sd, buf[0], buf[1], buf[2], m.present ? buf[3] : nullptr, buf[4],
                       static_cast<float*>(buf[5]), st);
    }
  }
  if (rc == PA_OK && ob) {
    cudaError_t e = cudaMemcpyAsync(out + static_cast<size_t>(j.r0) * out_row_bytes, buf[4], ob,
                                    cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) rc = fail_cuda(e, "cudaMemcpyAsync(out)");
  }
  if (rc == PA_OK && lb) {
    cudaError_t e = cudaMemcpyAsync(lse + static_cast<size_t>(j.r0) * lse_row_elems, buf[5], lb,
                                    cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) rc = fail_cuda(e, "cudaMemcpyAsync(lse)");
  }
  for (int i = 0; i < 6; ++i) scratch_free(buf[i], st);
  cudaError_t e = cudaStreamSynchronize(st);
  if (rc == PA_OK && e != cudaSuccess) rc = fail_cuda(e, "cudaStreamSynchronize(shard)");
  cudaStreamDestroy(st);
  if (rc == PA_OK) {
    int code = 0;
    rc = pa_device_status(&code);
  }
  return rc;
}

}  // namespace
}  // namespace pa

using namespace pa;

extern "C" pa_status pa_shard_fwd(int32_t ndev, const int32_t* devices, const pa_sdpa_desc* desc,
                                  const void* q, const void* k, const void* v, const void* mask,
                                  void* out, float* lse) {
  clear_error();
  PA_TRY(check_desc(desc));
  const pa_sdpa_desc& d = *desc;
  if (ndev < 1 || !devices) return fail(PA_ERR_INVALID, "pa_shard_fwd: need at least one device");
  if (!q || !k || !v || !out) return fail(PA_ERR_INVALID, "pa_shard_fwd: null operand");
  if (d.mask_kind != PA_MASK_NONE && !mask) return fail(PA_ERR_INVALID, "pa_shard_fwd: mask kind set but no mask");
  if (lead_count(d) == 0 || d.L == 0) return PA_OK;
  int count = 0;
  PA_CUDA(cudaGetDeviceCount(&count));
  for (int i = 0; i < ndev; ++i)
    if (devices[i] < 0 || devices[i] >= count) return fail(PA_ERR_INVALID, "pa_shard_fwd: device index out of range");

  const size_t esz = dtype_bytes(d.dtype);
  const int64_t rows0 = d.nlead > 0 ? d.lead[0] : 1;
  const bool gqa_on_0 = d.gqa_group > 1 && d.gqa_axis == 0;
  const int64_t unit = gqa_on_0 ? d.gqa_group : 1;  // shard boundaries fall on whole groups
  const int kv_div_axis = d.gqa_group > 1 ? d.gqa_axis : -1;
  int64_t zero[PA_MAX_LEAD] = {};
  Operand oq{static_cast<const uint8_t*>(q), esz, d.nlead > 0 ? d.q_lead_stride[0] : 0,
             inner_span(d, d.nlead ? d.q_lead_stride : zero, d.L, d.q_row_stride, d.E, 1, -1), true};
  Operand ok_{static_cast<const uint8_t*>(k), esz, d.nlead > 0 ? d.k_lead_stride[0] : 0,
              inner_span(d, d.nlead ? d.k_lead_stride : zero, d.S, d.k_row_stride, d.E, 1, kv_div_axis), true};
  Operand ov{static_cast<const uint8_t*>(v), esz, d.nlead > 0 ? d.v_lead_stride[0] : 0,
             inner_span(d, d.nlead ? d.v_lead_stride : zero, d.S, d.v_row_stride, d.Ev, 1, kv_div_axis), true};
  Operand om{static_cast<const uint8_t*>(mask), dtype_bytes(d.mask_dtype), d.nlead > 0 ? d.m_lead_stride[0] : 0,
             inner_span(d, d.nlead ? d.m_lead_stride : zero, d.L, d.m_row_stride, d.S, d.m_col_stride, -1),
             d.mask_kind != PA_MASK_NONE};
  for (const Operand* o : {&oq, &ok_, &ov, &om})
    if (o->present && o->stride0 != 0 && o->stride0 < o->span)
      return fail(PA_ERR_UNSUPPORTED, "pa_shard_fwd: rows of the first leading dimension overlap in memory");
  if (oq.stride0 == 0 && rows0 > 1) return fail(PA_ERR_UNSUPPORTED, "pa_shard_fwd: query broadcast over the first dimension");

  // Output rows of dim 0: the product of the other leading dims x L x Ev (dense).
  int64_t per = 1;
  for (int i = 1; i < d.nlead; ++i) per *= d.lead[i];
  const size_t out_row_bytes = static_cast<size_t>(per * d.L * d.Ev) * esz;
  const size_t lse_row = static_cast<size_t>(per * d.L);

  const int64_t units = rows0 / unit;
  const int use = static_cast<int>(units < ndev ? units : ndev);
  std::vector<Job> jobs(use);
  int64_t done = 0;
  for (int i = 0; i < use; ++i) {
    const int64_t take = units / use + (i < units % use ? 1 : 0);
    jobs[i].device = devices[i];
    jobs[i].r0 = done * unit;
    jobs[i].n = take * unit;
    jobs[i].kr0 = gqa_on_0 ? done : jobs[i].r0;
    jobs[i].kn = gqa_on_0 ? take : jobs[i].n;
    done += take;
  }
  int prev = 0;
  cudaGetDevice(&prev);
  std::vector<std::thread> threads;
  for (int i = 0; i < use; ++i)
    threads.emplace_back([&, i] {
      Job& j = jobs[i];
      j.status = run_shard(d, oq, ok_, ov, om, static_cast<uint8_t*>(out), lse, out_row_bytes, lse_row, j);
      if (j.status != PA_OK) j.message = pa_last_error();
    });
  for (auto& t : threads) t.join();
  cudaSetDevice(prev);
  for (const Job& j : jobs)
    if (j.status != PA_OK) return fail(static_cast<pa_status>(j.status), "device " + std::to_string(j.device) + ": " + j.message);
  return PA_OK;
}
