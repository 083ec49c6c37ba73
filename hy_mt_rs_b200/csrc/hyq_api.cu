// C ABI of libhyq (include/hyq.h): argument validation mirroring the
// reference's ensure! checks, weight handles, status reporting, and dispatch
// to the kernel translation units.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <functional>
#include <mutex>
#include <string>

#include "../../include/hyq.h"
#include "hyq_common.cuh"
#include "hyq_kernels.h"

struct hyq_weight {
  int dtype;
  int ndim;
  int64_t dims[3];
  size_t byte_len;
  const uint8_t* data;  // device
  bool owns;
};

namespace {

thread_local std::string t_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(HYQ_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool valid_dtype(int t) { return t >= HYQ_F32 && t <= HYQ_STQ1_0; }

int64_t row_bytes(int dtype, int64_t K) { return K / hyq::block_len(dtype) * hyq::block_bytes(dtype); }

// Per-device status word: a module-scope device variable (no allocation).
__device__ unsigned g_status;

constexpr int kMaxDevices = 64;
unsigned* g_status_ptr[kMaxDevices] = {};
std::mutex g_status_mu;

int status_ptr(unsigned** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(HYQ_E_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_status_mu);
  if (!g_status_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_status);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(status)");
    g_status_ptr[dev] = static_cast<unsigned*>(p);
  }
  *out = g_status_ptr[dev];
  return HYQ_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Stream-ordered workspace of the tensor-core products.  Outside stream
// capture it comes from a memory pool the library owns (one per device,
// created on first use, its release threshold at the maximum so that freed
// workspace stays cached between calls instead of going back to the driver
// at every synchronization).  The device's default pool, and its settings,
// belong to the caller and are left alone.  Under capture the allocation
// becomes a graph memory node (graph-owned memory), as cudaMallocAsync gives.
cudaError_t ws_alloc(void** p, size_t bytes, cudaStream_t st) {
  static std::mutex mu;
  static cudaMemPool_t pools[kMaxDevices] = {};
  static bool made[kMaxDevices] = {};
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(st, &cap);
  if (e != cudaSuccess) return e;
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if (cap != cudaStreamCaptureStatusNone || dev < 0 || dev >= kMaxDevices) return cudaMallocAsync(p, bytes, st);
  cudaMemPool_t pool = nullptr;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!made[dev]) {
      cudaMemPoolProps props = {};
      props.allocType = cudaMemAllocationTypePinned;
      props.location.type = cudaMemLocationTypeDevice;
      props.location.id = dev;
      if ((e = cudaMemPoolCreate(&pools[dev], &props)) != cudaSuccess) return e;
      uint64_t keep = UINT64_MAX;
      if ((e = cudaMemPoolSetAttribute(pools[dev], cudaMemPoolAttrReleaseThreshold, &keep)) != cudaSuccess) return e;
      made[dev] = true;
    }
    pool = pools[dev];
  }
  return cudaMallocFromPoolAsync(p, bytes, pool, st);
}

// hyq_set_launch_overlap: batch-1 products launch as programmatic dependents
// of the preceding grid in their stream.
std::atomic<int> g_launch_overlap{0};

// hyq_set_gemm_precision: batched products on split fp16 operands.
std::atomic<int> g_gemm_precision{HYQ_GEMM_FP16};

// Batches from this size up go to the tensor-core GEMM when the format and
// shape allow it; smaller batches run batch-1 products.
constexpr int64_t kGemmMinBatch = 16;

int check_matrix(const hyq_weight* w, const char* name) {
  if (!w) return fail(HYQ_E_INVALID, "%s: null weight", name);
  if (w->ndim != 2) return fail(HYQ_E_SHAPE, "%s is not a matrix", name);
  return HYQ_OK;
}

int launch_status(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return cuda_fail(e, what);
  return HYQ_OK;
}

int make_weight(const void* data, size_t byte_len, int dtype, int ndim, const int64_t* dims, bool device,
                hyq_weight** out) {
  if (!out) return fail(HYQ_E_INVALID, "weight: null output handle");
  *out = nullptr;
  if (!valid_dtype(dtype)) return fail(HYQ_E_INVALID, "unsupported tensor type %d", dtype);
  if (!data || !dims) return fail(HYQ_E_INVALID, "weight: null data or dims");
  if (ndim < 1 || ndim > 3) return fail(HYQ_E_SHAPE, "weight: rank %d not supported", ndim);
  int64_t d[3] = {1, 1, 1};
  for (int i = 0; i < ndim; ++i) {
    if (dims[i] <= 0) return fail(HYQ_E_SHAPE, "weight: non-positive dimension");
    d[i] = dims[i];
  }
  if (d[0] % hyq::block_len(dtype) != 0) return fail(HYQ_E_SHAPE, "weight: K=%lld is not a multiple of %d",
                                                     (long long)d[0], hyq::block_len(dtype));
  const int64_t expect = row_bytes(dtype, d[0]) * d[1] * d[2];
  if ((int64_t)byte_len != expect)
    return fail(HYQ_E_SHAPE, "weight: byte_len %zu does not match shape (expected %lld)", byte_len,
                (long long)expect);
  hyq_weight* w = new hyq_weight{};
  w->dtype = dtype;
  w->ndim = ndim;
  for (int i = 0; i < 3; ++i) w->dims[i] = i < ndim ? d[i] : 0;
  w->byte_len = byte_len;
  if (device) {
    w->data = static_cast<const uint8_t*>(data);
    w->owns = false;
  } else {
    void* p = nullptr;
    // Pad to a 16-byte multiple so bulk copies of the last rows stay inside.
    cudaError_t e = cudaMalloc(&p, (byte_len + 15) / 16 * 16 + 16);
    if (e != cudaSuccess) {
      delete w;
      return fail(HYQ_E_NOMEM, "cudaMalloc(%zu): %s", byte_len, cudaGetErrorString(e));
    }
    e = cudaMemcpy(p, data, byte_len, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      cudaFree(p);
      delete w;
      return cuda_fail(e, "cudaMemcpy(upload)");
    }
    w->data = static_cast<const uint8_t*>(p);
    w->owns = true;
  }
  *out = w;
  return HYQ_OK;
}

// Activations given either as f32 or as Q8 (values, scales).
struct Act {
  const float* x = nullptr;
  const int8_t* xq = nullptr;
  const float* xs = nullptr;
  bool quantize = false;  // x is quantized to Q8 inside the kernel
  const float* norm_w = nullptr;  // fused RMSNorm of x (hyq_gemv_*_norm)
  float eps = 0.f;
};

int run_gemv(int n_mat, const hyq_weight* const* ws, float* const* ys, const hyq_weight* up, const Act& a,
             cudaStream_t st, const char* name, bool residual = false) {
  unsigned* status = nullptr;
  int rc = status_ptr(&status);
  if (rc) return rc;
  hyq::GemvJob j;
  j.dtype = ws[0]->dtype;
  j.n_mat = n_mat;
  for (int m = 0; m < n_mat; ++m) {
    j.w[m] = ws[m]->data;
    j.y[m] = ys[m];
    j.rows[m] = ws[m]->dims[1];
  }
  j.up = up ? up->data : nullptr;
  j.K = ws[0]->dims[0];
  j.x = a.x;
  j.xq = a.xq;
  j.xs = a.xs;
  j.quantize_q8 = a.quantize;
  j.norm_w = a.norm_w;
  j.eps = a.eps;
  j.residual = residual;
  j.status = status;
  j.overlap = g_launch_overlap.load(std::memory_order_relaxed) != 0;
  if ((a.norm_w || residual) && !hyq::gemv_fusable(j))
    return fail(HYQ_E_UNSUPPORTED,
                "%s: the fused norm / residual forms need a packed format, K a multiple of 256 and at most 6144, "
                "and 16-byte aligned weights and input",
                name);
  const cudaError_t e = hyq::launch_gemv(j, st);
  if (e == cudaErrorNotSupported)
    return fail(HYQ_E_UNSUPPORTED, "%s: in-kernel Q8 needs K to be a multiple of 256 for this buffer layout", name);
  return launch_status(e, name);
}

int check_act(const Act& a, const char* name) {
  if (a.x) {
    if (!aligned(a.x, 4)) return fail(HYQ_E_ALIGN, "%s: input not 4-byte aligned", name);
    return HYQ_OK;
  }
  if (!a.xq || !a.xs) return fail(HYQ_E_INVALID, "%s: null activations", name);
  if (!aligned(a.xs, 4)) return fail(HYQ_E_ALIGN, "%s: scales not 4-byte aligned", name);
  return HYQ_OK;
}

}  // namespace

namespace hyq {

// Error and status plumbing shared with C-ABI entry points defined in other
// translation units.
int api_fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_err = buf;
  return code;
}

int api_status_word(unsigned** out) { return status_ptr(out); }

bool launch_overlap() { return g_launch_overlap.load(std::memory_order_relaxed) != 0; }
bool gemm_split() { return g_gemm_precision.load(std::memory_order_relaxed) == HYQ_GEMM_F32; }

}  // namespace hyq

extern "C" {

const char* hyq_last_error(void) { return t_err.c_str(); }

int hyq_block_len(int dtype) { return valid_dtype(dtype) ? hyq::block_len(dtype) : 0; }

int hyq_block_bytes(int dtype) { return valid_dtype(dtype) ? hyq::block_bytes(dtype) : 0; }

int hyq_dtype_from_id(uint32_t id, int profile, int* dtype_out) {
  if (!dtype_out) return fail(HYQ_E_INVALID, "dtype_from_id: null output");
  int t = -1;
  switch (id) {
    case 0: t = HYQ_F32; break;
    case 1: t = HYQ_F16; break;
    case 8: t = HYQ_Q8_0; break;
    case 12: t = HYQ_Q4_K; break;
    case 14: t = HYQ_Q6_K; break;
    case 40: t = profile == HYQ_PROFILE_TENCENT_Q2_0C ? HYQ_Q2_0C : -1; break;
    case 42: t = profile == HYQ_PROFILE_TENCENT_STQ1 ? HYQ_STQ1_0 : -1; break;
    default: break;
  }
  if (t < 0) return fail(HYQ_E_INVALID, "unsupported GGUF tensor type %u for profile %d", id, profile);
  *dtype_out = t;
  return HYQ_OK;
}

int hyq_upload(const void* packed_host, size_t byte_len, int dtype, int ndim, const int64_t* dims,
               hyq_weight** out) {
  return make_weight(packed_host, byte_len, dtype, ndim, dims, false, out);
}

int hyq_weight_wrap(const void* packed_device, size_t byte_len, int dtype, int ndim, const int64_t* dims,
                    hyq_weight** out) {
  return make_weight(packed_device, byte_len, dtype, ndim, dims, true, out);
}

int hyq_weight_expert(const hyq_weight* w, int64_t index, hyq_weight** out) {
  if (!w || !out) return fail(HYQ_E_INVALID, "expert: null argument");
  *out = nullptr;
  if (w->ndim != 3 || index < 0 || index >= w->dims[2])
    return fail(HYQ_E_SHAPE, "invalid expert %lld", (long long)index);
  hyq_weight* e = new hyq_weight{};
  e->dtype = w->dtype;
  e->ndim = 2;
  e->dims[0] = w->dims[0];
  e->dims[1] = w->dims[1];
  e->byte_len = w->byte_len / (size_t)w->dims[2];
  e->data = w->data + (size_t)index * e->byte_len;
  e->owns = false;
  *out = e;
  return HYQ_OK;
}

int hyq_weight_shard(const hyq_weight* w, int axis, int64_t part, int64_t parts, void* stream, hyq_weight** out) {
  if (!w || !out) return fail(HYQ_E_INVALID, "shard: null argument");
  *out = nullptr;
  if (w->ndim != 2) return fail(HYQ_E_SHAPE, "shard: weight is not a matrix");
  if (parts < 1 || part < 0 || part >= parts) return fail(HYQ_E_INVALID, "shard: part %lld of %lld", (long long)part,
                                                          (long long)parts);
  const int64_t K = w->dims[0], N = w->dims[1];
  const int64_t rb = row_bytes(w->dtype, K);
  if (axis == 0) {
    // Column-parallel: a contiguous range of output rows, viewed in place.
    if (N % parts != 0) return fail(HYQ_E_SHAPE, "shard: %lld rows do not split into %lld parts", (long long)N,
                                    (long long)parts);
    const int64_t n = N / parts;
    hyq_weight* s = new hyq_weight{};
    s->dtype = w->dtype;
    s->ndim = 2;
    s->dims[0] = K;
    s->dims[1] = n;
    s->byte_len = (size_t)(n * rb);
    s->data = w->data + part * n * rb;
    s->owns = false;
    *out = s;
    return HYQ_OK;
  }
  if (axis != 1) return fail(HYQ_E_INVALID, "shard: axis %d (0 = rows, 1 = input columns)", axis);
  // Row-parallel: the same K range of every row, on block boundaries, gathered
  // into a new [K / parts, N] buffer (packed bytes unchanged).
  const int bl = hyq::block_len(w->dtype);
  if (K % parts != 0 || (K / parts) % bl != 0)
    return fail(HYQ_E_SHAPE, "shard: K=%lld does not split into %lld parts of whole %d-weight blocks", (long long)K,
                (long long)parts, bl);
  const int64_t k = K / parts;
  const int64_t srb = row_bytes(w->dtype, k);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)((N * srb + 15) / 16 * 16 + 16));
  if (e != cudaSuccess) return fail(HYQ_E_NOMEM, "shard: cudaMalloc: %s", cudaGetErrorString(e));
  e = cudaMemcpy2DAsync(p, (size_t)srb, w->data + part * srb, (size_t)rb, (size_t)srb, (size_t)N,
                        cudaMemcpyDeviceToDevice, (cudaStream_t)stream);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "shard: copy");
  }
  hyq_weight* s = new hyq_weight{};
  s->dtype = w->dtype;
  s->ndim = 2;
  s->dims[0] = k;
  s->dims[1] = N;
  s->byte_len = (size_t)(N * srb);
  s->data = static_cast<const uint8_t*>(p);
  s->owns = true;
  *out = s;
  return HYQ_OK;
}

int hyq_weight_info(const hyq_weight* w, int* dtype, int* ndim, int64_t* dims, size_t* byte_len,
                    const void** device_ptr) {
  if (!w) return fail(HYQ_E_INVALID, "info: null weight");
  if (dtype) *dtype = w->dtype;
  if (ndim) *ndim = w->ndim;
  if (dims)
    for (int i = 0; i < 3; ++i) dims[i] = w->dims[i];
  if (byte_len) *byte_len = w->byte_len;
  if (device_ptr) *device_ptr = w->data;
  return HYQ_OK;
}

void hyq_free(hyq_weight* w) {
  if (!w) return;
  if (w->owns) cudaFree(const_cast<uint8_t*>(w->data));
  delete w;
}

int hyq_decode(int dtype, const void* bytes, size_t byte_len, float* out, size_t out_len, void* stream) {
  if (!valid_dtype(dtype)) return fail(HYQ_E_INVALID, "unsupported tensor type %d", dtype);
  const size_t bl = (size_t)hyq::block_len(dtype), bb = (size_t)hyq::block_bytes(dtype);
  if (out_len % bl) return fail(HYQ_E_SHAPE, "partial output block");
  if (byte_len != out_len / bl * bb) return fail(HYQ_E_SHAPE, "wrong byte count");
  if (out_len == 0) return HYQ_OK;
  if (!bytes || !out) return fail(HYQ_E_INVALID, "decode: null pointer");
  if (!aligned(out, 4)) return fail(HYQ_E_ALIGN, "decode: output not 4-byte aligned");
  return launch_status(hyq::launch_decode(dtype, bytes, out, (int64_t)out_len, (cudaStream_t)stream), "decode");
}

int hyq_weight_row_into(const hyq_weight* w, int64_t row, float* out, int64_t out_len, void* stream) {
  if (!w || !out) return fail(HYQ_E_INVALID, "row_into: null argument");
  const int64_t n = w->dims[0];
  if (out_len != n) return fail(HYQ_E_SHAPE, "out buffer length mismatch");
  const int64_t rb = row_bytes(w->dtype, n);
  if (row < 0 || row >= (int64_t)w->byte_len / rb) return fail(HYQ_E_SHAPE, "row %lld out of range", (long long)row);
  if (!aligned(out, 4)) return fail(HYQ_E_ALIGN, "row_into: output not 4-byte aligned");
  return launch_status(hyq::launch_decode(w->dtype, w->data + row * rb, out, n, (cudaStream_t)stream), "row_into");
}

int hyq_dot(const float* a, const float* b, size_t n, float* out, void* stream) {
  if (!out || (n && (!a || !b))) return fail(HYQ_E_INVALID, "dot: null pointer");
  return launch_status(hyq::launch_dot(a, b, (int64_t)n, out, (cudaStream_t)stream), "dot");
}

int hyq_matmul(const hyq_weight* w, const float* input, int64_t batch, float* out, void* stream) {
  int rc = check_matrix(w, "matmul");
  if (rc) return rc;
  if (batch <= 0) return fail(HYQ_E_SHAPE, "invalid activation shape");
  if (!input || !out) return fail(HYQ_E_INVALID, "matmul: null pointer");
  Act a;
  a.x = input;
  if ((rc = check_act(a, "matmul"))) return rc;
  const int64_t K = w->dims[0], N = w->dims[1];
  if (batch >= kGemmMinBatch && hyq::gemm_supported(w->dtype, K, N, batch, w->data) && aligned(input, 16)) {
    unsigned* status = nullptr;
    if ((rc = status_ptr(&status))) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    void* ws = nullptr;
    const bool split = hyq::gemm_split();
    cudaError_t e = ws_alloc(&ws, hyq::gemm_workspace_bytes(w->dtype, K, N, batch, split), st);
    if (e != cudaSuccess) return fail(HYQ_E_NOMEM, "matmul workspace: %s", cudaGetErrorString(e));
    e = hyq::launch_gemm(w->dtype, w->data, K, N, input, batch, out, ws, status, st, split);
    cudaError_t e2 = cudaFreeAsync(ws, st);
    if (e != cudaSuccess) return cuda_fail(e, "matmul (tensor-core GEMM)");
    if (e2 != cudaSuccess) return cuda_fail(e2, "matmul workspace free");
    return HYQ_OK;
  }
  for (int64_t b = 0; b < batch; ++b) {
    Act ab;
    ab.x = input + b * K;
    float* y = out + b * N;
    rc = run_gemv(1, &w, &y, nullptr, ab, (cudaStream_t)stream, "matmul");
    if (rc) return rc;
  }
  return HYQ_OK;
}

static int qkv_checks(const hyq_weight* q, const hyq_weight* k, const hyq_weight* v) {
  if (!q || !k || !v) return fail(HYQ_E_INVALID, "qkv: null weight");
  if (q->ndim != 2 || k->ndim != 2 || v->ndim != 2 || k->dims[0] != q->dims[0] || v->dims[0] != q->dims[0])
    return fail(HYQ_E_SHAPE, "query, key and value must be matrices that share an input width");
  return HYQ_OK;
}

static int qkv_run(const hyq_weight* q, const hyq_weight* k, const hyq_weight* v, const Act& a, float* qo,
                   float* ko, float* vo, cudaStream_t st) {
  if (!qo || !ko || !vo) return fail(HYQ_E_INVALID, "qkv: null output");
  const hyq_weight* ws[3] = {q, k, v};
  float* ys[3] = {qo, ko, vo};
  if (q->dtype == k->dtype && q->dtype == v->dtype) return run_gemv(3, ws, ys, nullptr, a, st, "qkv");
  for (int m = 0; m < 3; ++m) {
    int rc = run_gemv(1, &ws[m], &ys[m], nullptr, a, st, "qkv");
    if (rc) return rc;
  }
  return HYQ_OK;
}

int hyq_gemv_qkv(const hyq_weight* q, const hyq_weight* k, const hyq_weight* v, const float* input, float* q_out,
                 float* k_out, float* v_out, void* stream) {
  int rc = qkv_checks(q, k, v);
  if (rc) return rc;
  Act a;
  a.x = input;
  if (!input) return fail(HYQ_E_INVALID, "qkv: null input");
  if ((rc = check_act(a, "qkv"))) return rc;
  return qkv_run(q, k, v, a, q_out, k_out, v_out, (cudaStream_t)stream);
}

static int act_mode(Act& a, int act, const char* name) {
  if (act != HYQ_ACT_F32 && act != HYQ_ACT_Q8) return fail(HYQ_E_INVALID, "%s: unknown activation mode %d", name, act);
  a.quantize = act == HYQ_ACT_Q8;
  return HYQ_OK;
}

static int norm_act(Act& a, const float* hidden, const float* norm_w, float eps, int act, const char* name) {
  if (!hidden || !norm_w) return fail(HYQ_E_INVALID, "%s: null pointer", name);
  if (!aligned(norm_w, 4)) return fail(HYQ_E_ALIGN, "%s: norm weights not 4-byte aligned", name);
  int rc = act_mode(a, act, name);
  if (rc) return rc;
  a.x = hidden;
  a.norm_w = norm_w;
  a.eps = eps;
  return check_act(a, name);
}

int hyq_gemv_qkv_norm(const hyq_weight* q, const hyq_weight* k, const hyq_weight* v, const float* hidden,
                      const float* norm_w, float eps, int act, float* q_out, float* k_out, float* v_out,
                      void* stream) {
  int rc = qkv_checks(q, k, v);
  if (rc) return rc;
  Act a;
  if ((rc = norm_act(a, hidden, norm_w, eps, act, "qkv_norm"))) return rc;
  return qkv_run(q, k, v, a, q_out, k_out, v_out, (cudaStream_t)stream);
}

int hyq_gemv_norm(const hyq_weight* w, const float* hidden, const float* norm_w, float eps, int act, float* out,
                  void* stream) {
  int rc = check_matrix(w, "gemv_norm");
  if (rc) return rc;
  if (!out) return fail(HYQ_E_INVALID, "gemv_norm: null output");
  Act a;
  if ((rc = norm_act(a, hidden, norm_w, eps, act, "gemv_norm"))) return rc;
  return run_gemv(1, &w, &out, nullptr, a, (cudaStream_t)stream, "gemv_norm");
}

int hyq_gemv_residual(const hyq_weight* w, const float* input, int act, float* hidden, void* stream) {
  int rc = check_matrix(w, "gemv_residual");
  if (rc) return rc;
  if (!input || !hidden) return fail(HYQ_E_INVALID, "gemv_residual: null pointer");
  if (!aligned(hidden, 4)) return fail(HYQ_E_ALIGN, "gemv_residual: hidden not 4-byte aligned");
  Act a;
  if ((rc = act_mode(a, act, "gemv_residual"))) return rc;
  a.x = input;
  if ((rc = check_act(a, "gemv_residual"))) return rc;
  return run_gemv(1, &w, &hidden, nullptr, a, (cudaStream_t)stream, "gemv_residual", true);
}

int hyq_gemv_fusable(const hyq_weight* w, int* out) {
  int rc = check_matrix(w, "gemv_fusable");
  if (rc) return rc;
  if (!out) return fail(HYQ_E_INVALID, "gemv_fusable: null output");
  hyq::GemvJob j;
  j.dtype = w->dtype;
  j.w[0] = w->data;
  j.rows[0] = w->dims[1];
  j.K = w->dims[0];
  j.x = reinterpret_cast<const float*>(uintptr_t{256});  // any 16-byte aligned input
  *out = hyq::gemv_fusable(j) ? 1 : 0;
  return HYQ_OK;
}

static int gate_up_checks(const hyq_weight* gate, const hyq_weight* up) {
  int rc = check_matrix(gate, "gate");
  if (rc) return rc;
  if ((rc = check_matrix(up, "up"))) return rc;
  if (up->dims[0] != gate->dims[0] || up->dims[1] != gate->dims[1]) return fail(HYQ_E_SHAPE, "gate and up shape mismatch");
  if (up->dtype != gate->dtype) return fail(HYQ_E_UNSUPPORTED, "gate and up must share a tensor type");
  return HYQ_OK;
}

int hyq_matmul_gate_up_silu(const hyq_weight* gate, const hyq_weight* up, const float* input, float* out,
                            void* stream) {
  int rc = gate_up_checks(gate, up);
  if (rc) return rc;
  if (!input || !out) return fail(HYQ_E_INVALID, "gate_up_silu: null pointer");
  Act a;
  a.x = input;
  if ((rc = check_act(a, "gate_up_silu"))) return rc;
  return run_gemv(1, &gate, &out, up, a, (cudaStream_t)stream, "gate_up_silu");
}

int hyq_gemv_gate_up_silu_norm(const hyq_weight* gate, const hyq_weight* up, const float* hidden,
                               const float* norm_w, float eps, int act, float* out, void* stream) {
  int rc = gate_up_checks(gate, up);
  if (rc) return rc;
  if (!out) return fail(HYQ_E_INVALID, "gate_up_silu_norm: null output");
  Act a;
  if ((rc = norm_act(a, hidden, norm_w, eps, act, "gate_up_silu_norm"))) return rc;
  return run_gemv(1, &gate, &out, up, a, (cudaStream_t)stream, "gate_up_silu_norm");
}

// A grouped tensor-core product with a stream-ordered workspace.
static int run_gemm_job(const hyq::GemmJob& j, cudaStream_t st, const char* name) {
  unsigned* status = nullptr;
  int rc = status_ptr(&status);
  if (rc) return rc;
  hyq::GemmJob jj = j;
  jj.status = status;
  jj.split = hyq::gemm_split();
  void* ws = nullptr;
  cudaError_t e = ws_alloc(&ws, hyq::gemm_job_workspace_bytes(jj), st);
  if (e != cudaSuccess) return fail(HYQ_E_NOMEM, "%s workspace: %s", name, cudaGetErrorString(e));
  e = hyq::launch_gemm_job(jj, ws, st);
  const cudaError_t e2 = cudaFreeAsync(ws, st);
  if (e != cudaSuccess) return cuda_fail(e, name);
  if (e2 != cudaSuccess) return cuda_fail(e2, name);
  return HYQ_OK;
}

int hyq_matmul_qkv(const hyq_weight* q, const hyq_weight* k, const hyq_weight* v, const float* input, int64_t batch,
                   float* q_out, float* k_out, float* v_out, void* stream) {
  int rc = qkv_checks(q, k, v);
  if (rc) return rc;
  if (batch <= 0) return fail(HYQ_E_SHAPE, "invalid activation shape");
  if (!input || !q_out || !k_out || !v_out) return fail(HYQ_E_INVALID, "matmul_qkv: null pointer");
  Act a;
  a.x = input;
  if ((rc = check_act(a, "matmul_qkv"))) return rc;
  const int64_t K = q->dims[0];
  cudaStream_t st = (cudaStream_t)stream;
  hyq::GemmJob j;
  j.dtype = q->dtype;
  j.n_mat = 3;
  const hyq_weight* ws[3] = {q, k, v};
  float* ys[3] = {q_out, k_out, v_out};
  for (int m = 0; m < 3; ++m) {
    j.w[m] = ws[m]->data;
    j.rows[m] = ws[m]->dims[1];
    j.y[m] = ys[m];
  }
  j.K = K;
  j.M = batch;
  j.x = input;
  if (batch >= kGemmMinBatch && k->dtype == q->dtype && v->dtype == q->dtype && aligned(input, 16) &&
      hyq::gemm_job_supported(j))
    return run_gemm_job(j, st, "matmul_qkv (tensor-core GEMM)");
  for (int64_t b = 0; b < batch; ++b) {
    Act ab;
    ab.x = input + b * K;
    if ((rc = qkv_run(q, k, v, ab, q_out + b * q->dims[1], k_out + b * k->dims[1], v_out + b * v->dims[1], st)))
      return rc;
  }
  return HYQ_OK;
}

// Grouped expert products (expert mode of the tensor-core GEMM).
static int experts_job(const hyq_weight* w, const hyq_weight* up, const float* input, const int32_t* input_rows,
                       int64_t rows, const int32_t* expert_off, int64_t max_rows, float* out, hyq::GemmJob& j,
                       const char* name) {
  if (!w || !input || !expert_off || !out) return fail(HYQ_E_INVALID, "%s: null pointer", name);
  if (w->ndim != 3 || (up && (up->ndim != 3 || up->dtype != w->dtype || up->dims[0] != w->dims[0] ||
                              up->dims[1] != w->dims[1] || up->dims[2] != w->dims[2])))
    return fail(HYQ_E_SHAPE, "%s: weights must be [K, N, experts] tensors of one shape", name);
  if (rows <= 0 || max_rows <= 0) return fail(HYQ_E_SHAPE, "%s: invalid activation shape", name);
  if (!aligned(input, 16)) return fail(HYQ_E_ALIGN, "%s: input must be 16-byte aligned", name);
  j.dtype = w->dtype;
  j.n_mat = up ? 2 : 1;
  j.gate_up = up != nullptr;
  j.w[0] = w->data;
  if (up) j.w[1] = up->data;
  j.rows[0] = j.rows[1] = w->dims[1];
  j.y[0] = out;
  j.K = w->dims[0];
  j.M = rows;
  j.x = input;
  j.experts = (int)w->dims[2];
  j.expert_off = expert_off;
  j.expert_max_rows = max_rows;
  j.x_rows = input_rows;
  if (!hyq::gemm_job_supported(j))
    return fail(HYQ_E_UNSUPPORTED, "%s: the tensor-core path does not take this expert format or shape", name);
  return HYQ_OK;
}

int hyq_matmul_experts(const hyq_weight* w, const float* input, const int32_t* input_rows, int64_t rows,
                       const int32_t* expert_off, int64_t max_rows, float* out, void* stream) {
  hyq::GemmJob j;
  int rc = experts_job(w, nullptr, input, input_rows, rows, expert_off, max_rows, out, j, "matmul_experts");
  if (rc) return rc;
  return run_gemm_job(j, (cudaStream_t)stream, "matmul_experts (tensor-core GEMM)");
}

int hyq_matmul_experts_gate_up_silu(const hyq_weight* gate, const hyq_weight* up, const float* input,
                                    const int32_t* input_rows, int64_t rows, const int32_t* expert_off,
                                    int64_t max_rows, float* out, void* stream) {
  if (!up) return fail(HYQ_E_INVALID, "matmul_experts_gate_up_silu: null pointer");
  hyq::GemmJob j;
  int rc = experts_job(gate, up, input, input_rows, rows, expert_off, max_rows, out, j,
                       "matmul_experts_gate_up_silu");
  if (rc) return rc;
  return run_gemm_job(j, (cudaStream_t)stream, "matmul_experts_gate_up_silu (tensor-core GEMM)");
}

int hyq_matmul_gate_up_silu_batch(const hyq_weight* gate, const hyq_weight* up, const float* input, int64_t batch,
                                  float* out, void* stream) {
  int rc = gate_up_checks(gate, up);
  if (rc) return rc;
  if (batch <= 0) return fail(HYQ_E_SHAPE, "invalid activation shape");
  if (!input || !out) return fail(HYQ_E_INVALID, "gate_up_silu_batch: null pointer");
  Act a;
  a.x = input;
  if ((rc = check_act(a, "gate_up_silu_batch"))) return rc;
  const int64_t K = gate->dims[0], N = gate->dims[1];
  cudaStream_t st = (cudaStream_t)stream;
  hyq::GemmJob j;
  j.dtype = gate->dtype;
  j.n_mat = 2;
  j.gate_up = true;
  j.w[0] = gate->data;
  j.w[1] = up->data;
  j.rows[0] = j.rows[1] = N;
  j.y[0] = out;
  j.K = K;
  j.M = batch;
  j.x = input;
  if (batch >= kGemmMinBatch && aligned(input, 16) && hyq::gemm_job_supported(j))
    return run_gemm_job(j, st, "gate_up_silu_batch (tensor-core GEMM)");
  for (int64_t b = 0; b < batch; ++b) {
    Act ab;
    ab.x = input + b * K;
    float* y = out + b * N;
    if ((rc = run_gemv(1, &gate, &y, up, ab, st, "gate_up_silu_batch"))) return rc;
  }
  return HYQ_OK;
}

// The residual-stream input of the fused batched forms: hidden [batch, K]
// (+= delta when given), normalised with norm_w.
struct NormIn {
  float* hidden;
  const float* delta;
  const float* w;
  float eps;
};

static int norm_in_checks(const NormIn& n, int64_t batch, const char* name) {
  if (batch <= 0) return fail(HYQ_E_SHAPE, "%s: invalid activation shape", name);
  if (!n.hidden || !n.w) return fail(HYQ_E_INVALID, "%s: null pointer", name);
  if (!aligned(n.hidden, 4) || !aligned(n.w, 4) || (n.delta && !aligned(n.delta, 4)))
    return fail(HYQ_E_ALIGN, "%s: f32 buffers must be 4-byte aligned", name);
  return HYQ_OK;
}

static void set_norm(hyq::GemmJob& j, const NormIn& n) {
  j.x = n.hidden;
  j.norm_x = n.hidden;
  j.norm_delta = n.delta;
  j.norm_w = n.w;
  j.norm_eps = n.eps;
}

// The separate add + norm (or norm) kernel into a pool buffer, then `run` on
// it: the fused batched forms below 16 rows and for shapes the tensor-core
// conversion does not take.
static int norm_then(const NormIn& n, int64_t batch, int64_t K, cudaStream_t st, const char* name,
                     const std::function<int(const float*)>& run) {
  void* buf = nullptr;
  const cudaError_t e = ws_alloc(&buf, (size_t)batch * K * sizeof(float) + 16, st);
  if (e != cudaSuccess) return fail(HYQ_E_NOMEM, "%s workspace: %s", name, cudaGetErrorString(e));
  float* x = static_cast<float*>(buf);
  int rc = n.delta ? hyq_add_rms_norm(n.hidden, n.delta, n.w, K, batch, n.eps, x, st)
                   : hyq_rms_norm(n.hidden, n.w, K, batch, n.eps, x, st);
  if (!rc) rc = run(static_cast<const float*>(x));
  const cudaError_t e2 = cudaFreeAsync(buf, st);
  if (rc) return rc;
  if (e2 != cudaSuccess) return cuda_fail(e2, name);
  return HYQ_OK;
}

int hyq_matmul_qkv_norm(const hyq_weight* q, const hyq_weight* k, const hyq_weight* v, float* hidden,
                        const float* delta, const float* norm_w, float eps, int64_t batch, float* q_out,
                        float* k_out, float* v_out, void* stream) {
  int rc = qkv_checks(q, k, v);
  if (rc) return rc;
  const NormIn n{hidden, delta, norm_w, eps};
  if ((rc = norm_in_checks(n, batch, "matmul_qkv_norm"))) return rc;
  if (!q_out || !k_out || !v_out) return fail(HYQ_E_INVALID, "matmul_qkv_norm: null output");
  const int64_t K = q->dims[0];
  cudaStream_t st = (cudaStream_t)stream;
  hyq::GemmJob j;
  j.dtype = q->dtype;
  j.n_mat = 3;
  const hyq_weight* ws[3] = {q, k, v};
  float* ys[3] = {q_out, k_out, v_out};
  for (int m = 0; m < 3; ++m) {
    j.w[m] = ws[m]->data;
    j.rows[m] = ws[m]->dims[1];
    j.y[m] = ys[m];
  }
  j.K = K;
  j.M = batch;
  set_norm(j, n);
  if (batch >= kGemmMinBatch && k->dtype == q->dtype && v->dtype == q->dtype && hyq::gemm_job_supported(j))
    return run_gemm_job(j, st, "matmul_qkv_norm (tensor-core GEMM)");
  return norm_then(n, batch, K, st, "matmul_qkv_norm", [&](const float* x) {
    return hyq_matmul_qkv(q, k, v, x, batch, q_out, k_out, v_out, stream);
  });
}

int hyq_matmul_gate_up_silu_norm(const hyq_weight* gate, const hyq_weight* up, float* hidden, const float* delta,
                                 const float* norm_w, float eps, int64_t batch, float* out, void* stream) {
  int rc = gate_up_checks(gate, up);
  if (rc) return rc;
  const NormIn n{hidden, delta, norm_w, eps};
  if ((rc = norm_in_checks(n, batch, "gate_up_silu_norm"))) return rc;
  if (!out) return fail(HYQ_E_INVALID, "gate_up_silu_norm: null output");
  const int64_t K = gate->dims[0], N = gate->dims[1];
  cudaStream_t st = (cudaStream_t)stream;
  hyq::GemmJob j;
  j.dtype = gate->dtype;
  j.n_mat = 2;
  j.gate_up = true;
  j.w[0] = gate->data;
  j.w[1] = up->data;
  j.rows[0] = j.rows[1] = N;
  j.y[0] = out;
  j.K = K;
  j.M = batch;
  set_norm(j, n);
  if (batch >= kGemmMinBatch && hyq::gemm_job_supported(j))
    return run_gemm_job(j, st, "gate_up_silu_norm (tensor-core GEMM)");
  return norm_then(n, batch, K, st, "gate_up_silu_norm", [&](const float* x) {
    return hyq_matmul_gate_up_silu_batch(gate, up, x, batch, out, stream);
  });
}

int hyq_matmul_norm(const hyq_weight* w, float* hidden, const float* delta, const float* norm_w, float eps,
                    int64_t batch, float* out, void* stream) {
  int rc = check_matrix(w, "matmul_norm");
  if (rc) return rc;
  const NormIn n{hidden, delta, norm_w, eps};
  if ((rc = norm_in_checks(n, batch, "matmul_norm"))) return rc;
  if (!out) return fail(HYQ_E_INVALID, "matmul_norm: null output");
  const int64_t K = w->dims[0];
  cudaStream_t st = (cudaStream_t)stream;
  hyq::GemmJob j;
  j.dtype = w->dtype;
  j.n_mat = 1;
  j.w[0] = w->data;
  j.rows[0] = w->dims[1];
  j.y[0] = out;
  j.K = K;
  j.M = batch;
  set_norm(j, n);
  if (batch >= kGemmMinBatch && hyq::gemm_job_supported(j))
    return run_gemm_job(j, st, "matmul_norm (tensor-core GEMM)");
  return norm_then(n, batch, K, st, "matmul_norm",
                   [&](const float* x) { return hyq_matmul(w, x, batch, out, stream); });
}

int hyq_q8_quantize(const float* input, int64_t len, int8_t* values, float* scales, int8_t* values_q2c,
                    void* stream) {
  if (len < 0) return fail(HYQ_E_SHAPE, "q8: negative length");
  if (len == 0) return HYQ_OK;
  if (!input || !values || !scales) return fail(HYQ_E_INVALID, "q8: null pointer");
  if (!aligned(input, 4) || !aligned(scales, 4)) return fail(HYQ_E_ALIGN, "q8: f32 buffers must be 4-byte aligned");
  return launch_status(hyq::launch_q8_quantize(input, len, values, scales, values_q2c, (cudaStream_t)stream), "q8");
}

int hyq_gemv_q8(const hyq_weight* w, const int8_t* values, const float* scales, const int8_t* values_q2c,
                float* out, void* stream) {
  (void)values_q2c;  // the kernels permute the natural-order values themselves
  int rc = check_matrix(w, "gemv_q8");
  if (rc) return rc;
  if (!out) return fail(HYQ_E_INVALID, "gemv_q8: null output");
  Act a;
  a.xq = values;
  a.xs = scales;
  if ((rc = check_act(a, "gemv_q8"))) return rc;
  return run_gemv(1, &w, &out, nullptr, a, (cudaStream_t)stream, "gemv_q8");
}

int hyq_gemv_qkv_q8(const hyq_weight* q, const hyq_weight* k, const hyq_weight* v, const int8_t* values,
                    const float* scales, const int8_t* values_q2c, float* q_out, float* k_out, float* v_out,
                    void* stream) {
  (void)values_q2c;
  int rc = qkv_checks(q, k, v);
  if (rc) return rc;
  Act a;
  a.xq = values;
  a.xs = scales;
  if ((rc = check_act(a, "qkv_q8"))) return rc;
  return qkv_run(q, k, v, a, q_out, k_out, v_out, (cudaStream_t)stream);
}

int hyq_matmul_gate_up_silu_q8(const hyq_weight* gate, const hyq_weight* up, const int8_t* values,
                               const float* scales, const int8_t* values_q2c, float* out, void* stream) {
  (void)values_q2c;
  int rc = gate_up_checks(gate, up);
  if (rc) return rc;
  if (!out) return fail(HYQ_E_INVALID, "gate_up_silu_q8: null output");
  Act a;
  a.xq = values;
  a.xs = scales;
  if ((rc = check_act(a, "gate_up_silu_q8"))) return rc;
  return run_gemv(1, &gate, &out, up, a, (cudaStream_t)stream, "gate_up_silu_q8");
}

int hyq_gemv_int8(const hyq_weight* w, const float* input, float* out, void* stream) {
  int rc = check_matrix(w, "gemv_int8");
  if (rc) return rc;
  if (!input || !out) return fail(HYQ_E_INVALID, "gemv_int8: null pointer");
  Act a;
  a.x = input;
  a.quantize = true;
  if ((rc = check_act(a, "gemv_int8"))) return rc;
  return run_gemv(1, &w, &out, nullptr, a, (cudaStream_t)stream, "gemv_int8");
}

int hyq_gemv_qkv_int8(const hyq_weight* q, const hyq_weight* k, const hyq_weight* v, const float* input,
                      float* q_out, float* k_out, float* v_out, void* stream) {
  int rc = qkv_checks(q, k, v);
  if (rc) return rc;
  if (!input) return fail(HYQ_E_INVALID, "qkv_int8: null input");
  Act a;
  a.x = input;
  a.quantize = true;
  if ((rc = check_act(a, "qkv_int8"))) return rc;
  return qkv_run(q, k, v, a, q_out, k_out, v_out, (cudaStream_t)stream);
}

int hyq_matmul_gate_up_silu_int8(const hyq_weight* gate, const hyq_weight* up, const float* input, float* out,
                                 void* stream) {
  int rc = gate_up_checks(gate, up);
  if (rc) return rc;
  if (!input || !out) return fail(HYQ_E_INVALID, "gate_up_silu_int8: null pointer");
  Act a;
  a.x = input;
  a.quantize = true;
  if ((rc = check_act(a, "gate_up_silu_int8"))) return rc;
  return run_gemv(1, &gate, &out, up, a, (cudaStream_t)stream, "gate_up_silu_int8");
}

int hyq_set_gemm_precision(int precision) {
  if (precision != HYQ_GEMM_FP16 && precision != HYQ_GEMM_F32)
    return fail(HYQ_E_INVALID, "set_gemm_precision: unknown precision %d", precision);
  g_gemm_precision.store(precision, std::memory_order_relaxed);
  return HYQ_OK;
}

int hyq_set_launch_overlap(int enable) {
  g_launch_overlap.store(enable ? 1 : 0, std::memory_order_relaxed);
  return HYQ_OK;
}

int hyq_device_status(void* stream, uint32_t* status_out) {
  if (!status_out) return fail(HYQ_E_INVALID, "device_status: null output");
  unsigned* sp = nullptr;
  int rc = status_ptr(&sp);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  unsigned v = 0;
  e = cudaMemcpy(&v, sp, sizeof v, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read status");
  const unsigned zero = 0;
  e = cudaMemcpy(sp, &zero, sizeof zero, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "clear status");
  *status_out = v;
  if (v) return fail(HYQ_E_DEVICE, "device status 0x%x (bounded wait expired)", v);
  return HYQ_OK;
}

}  // extern "C"
