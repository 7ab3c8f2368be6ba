// ssa_capi.cu — the extern "C" boundary of libssa_b200.so (declared in include/ssa_b200.h).
//
// Validates a problem the way the reference's wrappers assert it (Hq % Hkv == 0,
// ssa_triton_kernel.py:753; head dim supported, :764-767), picks the kernel family, sizes
// and carves the caller's workspace, launches on the caller's stream and reports errors as
// status codes plus a thread-local message. It never allocates device memory.
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "ssa_internal.h"
#include "ssa_tmap.h"

namespace ssa {

__device__ unsigned int g_ssa_status;

namespace {
thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

constexpr int kMaxDevices = 64;
unsigned int* g_status_ptr[kMaxDevices] = {};
std::mutex g_mu;

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

int64_t rows_total(const ssa_problem_t* pr) {
  return pr->cu_seqlens ? (int64_t)pr->N : (int64_t)pr->B * pr->N;
}

int check_problem(const ssa_problem_t* pr) {
  if (!pr) return fail(SSA_ERR_NULL, "problem is NULL");
  if (pr->dtype < SSA_DTYPE_F32 || pr->dtype > SSA_DTYPE_BF16)
    return fail(SSA_ERR_UNSUPPORTED, "unsupported dtype %d", pr->dtype);
  if (pr->B <= 0 || pr->Hq <= 0 || pr->Hkv <= 0 || pr->N <= 0 || pr->D <= 0)
    return fail(SSA_ERR_BAD_SHAPE, "non-positive shape B=%d Hq=%d Hkv=%d N=%d D=%d", pr->B,
                pr->Hq, pr->Hkv, pr->N, pr->D);
  if (pr->Hq % pr->Hkv != 0)
    return fail(SSA_ERR_BAD_SHAPE, "Hq=%d must be divisible by Hkv=%d", pr->Hq, pr->Hkv);
  if (!generic_supports_head_dim(pr->D))
    return fail(SSA_ERR_UNSUPPORTED, "head dim D=%d not supported (16, 32, 64, 128)", pr->D);
  if (!pr->ssa_n || !pr->ssa_b) return fail(SSA_ERR_NULL, "ssa_n / ssa_b device pointer is NULL");
  if (!pr->cu_seqlens && pr->cu_seqlens_padded)
    return fail(SSA_ERR_BAD_SHAPE, "cu_seqlens_padded needs cu_seqlens (packed mode)");
  if (pr->cu_seqlens && pr->max_seqlen <= 0)
    return fail(SSA_ERR_BAD_SHAPE, "varlen needs max_seqlen > 0");
  if (!(pr->softmax_scale == pr->softmax_scale))
    return fail(SSA_ERR_BAD_SHAPE, "softmax_scale is NaN");
  if (!(pr->dropout_p >= 0.f && pr->dropout_p < 1.f))
    return fail(SSA_ERR_UNSUPPORTED, "dropout_p must be in [0, 1), got %g", (double)pr->dropout_p);
  if (pr->dropout_p > 0.f && !pr->dropout_seed)
    return fail(SSA_ERR_NULL, "dropout_p > 0 needs a dropout_seed device pointer");
  return SSA_OK;
}

int check_tensor(const ssa_tensor_t& t, const char* name) {
  if (!t.ptr) return fail(SSA_ERR_NULL, "%s is NULL", name);
  if (t.sB < 0 || t.sH < 0 || t.sN < 0)
    return fail(SSA_ERR_BAD_STRIDE, "%s has a negative stride", name);
  return SSA_OK;
}

Problem to_problem(const ssa_problem_t* pr) {
  Problem p;
  p.B = pr->B;
  p.Hq = pr->Hq;
  p.Hkv = pr->Hkv;
  p.N = pr->N;
  p.D = pr->D;
  p.gqa = pr->Hq / pr->Hkv;
  p.causal = pr->causal ? 1 : 0;
  p.scale = pr->softmax_scale;
  p.n_ptr = pr->ssa_n;
  p.n_per_head = pr->n_per_head ? 1 : 0;
  p.b_ptr = pr->ssa_b;
  p.cu_seqlens = pr->cu_seqlens;
  p.cu_seqlens_padded = pr->cu_seqlens ? pr->cu_seqlens_padded : nullptr;
  p.max_seqlen = pr->cu_seqlens ? pr->max_seqlen : pr->N;
  p.det = pr->deterministic ? 1 : 0;
  if (pr->dropout_p > 0.f) {  // p * 2^24 is exact in double: the threshold is exact too
    p.drop_thr = (uint32_t)ceil((double)pr->dropout_p * 16777216.0);
    p.drop_scale = 1.0f / (1.0f - pr->dropout_p);
    p.drop_delta_scale = 1.0f - pr->dropout_p;
    p.drop_lse_shift = (float)(-log2(1.0 - (double)pr->dropout_p));
    p.drop_seed = reinterpret_cast<const unsigned long long*>(pr->dropout_seed);
  } else {
    p.drop_thr = 0;
    p.drop_scale = 1.0f;
    p.drop_delta_scale = 1.0f;
    p.drop_lse_shift = 0.0f;
    p.drop_seed = nullptr;
  }
  return p;
}

TensorRef to_ref(const ssa_tensor_t& t) { return TensorRef{t.ptr, t.sB, t.sH, t.sN}; }

// Tensor-core family: 16-bit inputs, D in {32, 64, 128} (32 on the D = 64 kernels), positive
// scale, TMA-legal layouts.
bool use_sm100(const ssa_problem_t* pr) {
  return sm100_supports(pr->dtype, pr->D) && pr->softmax_scale > 0.f;
}
bool use_sm100_bwd(const ssa_problem_t* pr) {
  return use_sm100(pr) && sm100_bwd_supports(pr->dtype, pr->D);
}

int check_tma(const Problem& p, const ssa_tensor_t& t, int H, const char* name) {
  if (!tma_compatible(to_ref(t), p, H))
    return fail(SSA_ERR_BAD_STRIDE,
                "%s: base and B/H/N strides must be 16-byte aligned for the TMA path", name);
  return SSA_OK;
}

int finish_launch(int rc, const char* what) {
  if (rc != SSA_OK) {
    if (g_err[0] == 0) snprintf(g_err, sizeof(g_err), "%s failed with status %d", what, rc);
    return rc;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SSA_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return SSA_OK;
}

struct BwdWorkspace {
  float* delta;
  float* dn_part;
  float* db_part;
  void* sm100;
  size_t sm100_bytes;
  void* dom;  // output dropout: dout * keep / (1 - p) in the logical contiguous layout
  size_t total;
};

size_t dtype_bytes(int dtype) { return dtype == SSA_DTYPE_F32 ? 4 : 2; }

BwdWorkspace carve_bwd(const ssa_problem_t* pr, void* base) {
  const Problem p = to_problem(pr);
  BwdWorkspace w{};
  uint8_t* b = static_cast<uint8_t*>(base);
  size_t off = 0;
  const size_t delta_bytes = align256(sizeof(float) * (size_t)pr->Hq * (size_t)rows_total(pr));
  w.delta = reinterpret_cast<float*>(b ? b + off : nullptr);
  off += delta_bytes;
  if (use_sm100_bwd(pr)) {
    w.sm100_bytes = sm100_bwd_workspace_bytes(p);
    w.sm100 = b ? b + off : nullptr;
    off += align256(w.sm100_bytes);
  } else {
    const size_t part = align256(sizeof(float) * (size_t)pr->B * pr->Hq *
                                 (size_t)generic_bwd_partials_per_seq(p));
    w.dn_part = reinterpret_cast<float*>(b ? b + off : nullptr);
    off += part;
    w.db_part = reinterpret_cast<float*>(b ? b + off : nullptr);
    off += part;
  }
  w.dom = nullptr;
  if (pr->dropout_p > 0.f) {  // dout * keep, then the shifted lse (dropout_scratch_bytes)
    w.dom = b ? b + off : nullptr;
    off += dropout_scratch_bytes(p, (int)dtype_bytes(pr->dtype));
  }
  w.total = off;
  return w;
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// Makes the device that owns `ptr` current on the calling thread (its primary context). A thread
// that has not used CUDA yet (an autograd worker thread, a fresh thread of a C caller) has no
// current context: driver calls such as tensor-map encoding would fail there, and runtime calls
// would default to device 0 whatever device the caller's tensors live on.
int bind_device(const void* ptr, const char* name) {
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, ptr) != cudaSuccess) {
    cudaGetLastError();
    return fail(SSA_ERR_CUDA, "%s: cannot query the owning device of %p", name, ptr);
  }
  if (at.type != cudaMemoryTypeDevice && at.type != cudaMemoryTypeManaged)
    return fail(SSA_ERR_CUDA, "%s: %p is not device memory", name, ptr);
  if (cudaSetDevice(at.device) != cudaSuccess) {
    cudaGetLastError();
    return fail(SSA_ERR_CUDA, "%s: cannot make device %d current", name, at.device);
  }
  return SSA_OK;
}

int set_smem_limit_once(const void* func, int bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SSA_ERR_CUDA;
  static std::mutex mu;
  static std::unordered_map<const void*, int> done[kMaxDevices];  // bytes already granted
  std::lock_guard<std::mutex> lk(mu);
  auto it = done[dev].find(func);
  if (it != done[dev].end() && it->second >= bytes) return SSA_OK;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess) {
    cudaGetLastError();
    return SSA_ERR_CUDA;
  }
  done[dev][func] = bytes;
  return SSA_OK;
}

unsigned int* device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_status_ptr[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_ssa_status) != cudaSuccess) return nullptr;
    g_status_ptr[dev] = static_cast<unsigned int*>(ptr);
  }
  return g_status_ptr[dev];
}

namespace {
std::atomic<uint64_t> g_launches{0};
}
void note_launches(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

int abi_validate_problem(const ssa_problem_t* pr) {
  g_err[0] = 0;
  return check_problem(pr);
}
int abi_check_tensor(const ssa_tensor_t& t, const char* name) { return check_tensor(t, name); }
Problem abi_to_problem(const ssa_problem_t* pr) { return to_problem(pr); }
int abi_bind_device(const void* ptr, const char* name) { return bind_device(ptr, name); }
int abi_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

}  // namespace ssa

using namespace ssa;

extern "C" {

const char* ssa_last_error(void) { return g_err; }

uint64_t ssa_kernel_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

const char* ssa_version(void) { return "ssa_b200 0.1 (sm_100a tcgen05/TMA + generic fp32)"; }

int ssa_attn_kernel_family(const ssa_problem_t* prob) {
  if (check_problem(prob) != SSA_OK) return -1;
  return use_sm100(prob) ? 1 : 0;
}

size_t ssa_attn_fwd_workspace_size(const ssa_problem_t* prob) {
  (void)prob;
  return 0;
}

int ssa_attn_fwd(const ssa_problem_t* prob, ssa_tensor_t q, ssa_tensor_t k, ssa_tensor_t v,
                 ssa_tensor_t out, float* lse, void* workspace, size_t workspace_bytes,
                 void* stream) {
  (void)workspace;
  (void)workspace_bytes;
  g_err[0] = 0;
  int rc;
  if ((rc = check_problem(prob)) != SSA_OK) return rc;
  if ((rc = check_tensor(q, "q")) || (rc = check_tensor(k, "k")) || (rc = check_tensor(v, "v")) ||
      (rc = check_tensor(out, "out")))
    return rc;
  if (!lse) return fail(SSA_ERR_NULL, "lse is NULL");
  if ((rc = bind_device(q.ptr, "q")) != SSA_OK) return rc;
  const Problem p = to_problem(prob);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (use_sm100(prob)) {
    if ((rc = check_tma(p, q, p.Hq, "q")) || (rc = check_tma(p, k, p.Hkv, "k")) ||
        (rc = check_tma(p, v, p.Hkv, "v")))
      return rc;
    if ((reinterpret_cast<uintptr_t>(out.ptr) % 16) || (out.sN * 2) % 16 || (out.sH * 2) % 16 ||
        (out.sB * 2) % 16)
      return fail(SSA_ERR_BAD_STRIDE, "out: base and strides must be 16-byte aligned");
    if (!device_status_ptr()) return fail(SSA_ERR_CUDA, "cannot resolve the device status word");
    return finish_launch(launch_fwd_sm100(prob->dtype, p, to_ref(q), to_ref(k), to_ref(v),
                                          to_ref(out), lse, st),
                         "ssa_attn_fwd(sm100)");
  }
  return finish_launch(
      launch_fwd_generic(prob->dtype, p, to_ref(q), to_ref(k), to_ref(v), to_ref(out), lse, st),
      "ssa_attn_fwd(generic)");
}

int ssa_attn_bwd_preprocess(const ssa_problem_t* prob, ssa_tensor_t out, ssa_tensor_t dout,
                            float* delta, void* stream) {
  g_err[0] = 0;
  int rc;
  if ((rc = check_problem(prob)) != SSA_OK) return rc;
  if ((rc = check_tensor(out, "out")) || (rc = check_tensor(dout, "dout"))) return rc;
  if (!delta) return fail(SSA_ERR_NULL, "delta is NULL");
  if ((rc = bind_device(out.ptr, "out")) != SSA_OK) return rc;
  const Problem p = to_problem(prob);
  return finish_launch(launch_bwd_preprocess(prob->dtype, p, to_ref(out), to_ref(dout), delta,
                                             nullptr, nullptr, nullptr,
                                             static_cast<cudaStream_t>(stream)),
                       "ssa_attn_bwd_preprocess");
}

size_t ssa_attn_bwd_workspace_size(const ssa_problem_t* prob) {
  if (check_problem(prob) != SSA_OK) return 0;
  return carve_bwd(prob, nullptr).total;
}

int ssa_attn_bwd(const ssa_problem_t* prob, ssa_tensor_t q, ssa_tensor_t k, ssa_tensor_t v,
                 ssa_tensor_t out, ssa_tensor_t dout, const float* lse, ssa_tensor_t dq,
                 ssa_tensor_t dk, ssa_tensor_t dv, float* dn, float* db, void* workspace,
                 size_t workspace_bytes, void* stream) {
  g_err[0] = 0;
  int rc;
  if ((rc = check_problem(prob)) != SSA_OK) return rc;
  if ((rc = check_tensor(q, "q")) || (rc = check_tensor(k, "k")) || (rc = check_tensor(v, "v")) ||
      (rc = check_tensor(out, "out")) || (rc = check_tensor(dout, "dout")) ||
      (rc = check_tensor(dq, "dq")) || (rc = check_tensor(dk, "dk")) ||
      (rc = check_tensor(dv, "dv")))
    return rc;
  if (!lse || !dn || !db) return fail(SSA_ERR_NULL, "lse / dn / db is NULL");
  const BwdWorkspace need = carve_bwd(prob, nullptr);
  if (!workspace || workspace_bytes < need.total)
    return fail(SSA_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", need.total,
                workspace_bytes);
  if ((rc = bind_device(q.ptr, "q")) != SSA_OK) return rc;
  const BwdWorkspace w = carve_bwd(prob, workspace);
  const Problem p = to_problem(prob);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (use_sm100_bwd(prob)) {
    if ((rc = check_tma(p, q, p.Hq, "q")) || (rc = check_tma(p, k, p.Hkv, "k")) ||
        (rc = check_tma(p, v, p.Hkv, "v")) || (rc = check_tma(p, dout, p.Hq, "dout")) ||
        (rc = check_tma(p, dq, p.Hq, "dq")) || (rc = check_tma(p, dk, p.Hkv, "dk")) ||
        (rc = check_tma(p, dv, p.Hkv, "dv")))
      return rc;
    if (!device_status_ptr()) return fail(SSA_ERR_CUDA, "cannot resolve the device status word");
    if ((reinterpret_cast<uintptr_t>(out.ptr) % 16) || (out.sN * 2) % 16 || (out.sH * 2) % 16 ||
        (out.sB * 2) % 16)
      return fail(SSA_ERR_BAD_STRIDE, "out: base and strides must be 16-byte aligned");
    return finish_launch(launch_bwd_sm100(prob->dtype, p, to_ref(q), to_ref(k), to_ref(v),
                                          to_ref(out), to_ref(dout), lse, w.delta, to_ref(dq),
                                          to_ref(dk), to_ref(dv), dn, db, w.dom, w.sm100,
                                          w.sm100_bytes, st),
                         "ssa_attn_bwd(sm100)");
  }
  float* lse_sh = w.dom ? dropout_lse_buffer(p, w.dom, (int)dtype_bytes(prob->dtype)) : nullptr;
  rc = launch_bwd_preprocess(prob->dtype, p, to_ref(out), to_ref(dout), w.delta, w.dom, lse,
                             lse_sh, st);
  if ((rc = finish_launch(rc, "ssa_attn_bwd(preprocess)")) != SSA_OK) return rc;
  // with output dropout the gradient kernels read dout * keep and the shifted lse
  const TensorRef dO = w.dom ? dropout_dout_ref(p, w.dom) : to_ref(dout);
  rc = launch_bwd_generic(prob->dtype, p, to_ref(q), to_ref(k), to_ref(v), dO,
                          lse_sh ? lse_sh : lse, w.delta, to_ref(dq), to_ref(dk), to_ref(dv),
                          w.dn_part, w.db_part, st);
  if ((rc = finish_launch(rc, "ssa_attn_bwd(generic)")) != SSA_OK) return rc;
  rc = launch_dndb_reduce(w.dn_part, w.db_part, p.B, p.Hq, generic_bwd_partials_per_seq(p),
                          p.n_per_head, dn, db, st);
  return finish_launch(rc, "ssa_attn_bwd(dn/db reduce)");
}

int ssa_selftest_device_timeout(uint64_t wait_cycles, void* stream) {
  int dev = -1;
  if (cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &dev) == cudaSuccess)
    cudaSetDevice(dev);
  else
    cudaGetLastError();
  unsigned int* ptr = device_status_ptr();
  if (!ptr) return fail(SSA_ERR_CUDA, "cannot resolve the device status word");
  return finish_launch(launch_selftest_timeout(ptr, (long long)wait_cycles,
                                               static_cast<cudaStream_t>(stream)),
                       "ssa_selftest_device_timeout");
}

int ssa_device_status(void* stream) {
  g_err[0] = 0;
  int dev = -1;
  if (cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &dev) == cudaSuccess)
    cudaSetDevice(dev);
  else
    cudaGetLastError();
  cudaGetDevice(&dev);
  unsigned int* ptr = device_status_ptr();
  if (!ptr) return fail(SSA_ERR_CUDA, "cannot resolve the device status word");
  unsigned int h = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(&h, ptr, sizeof(h), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaMemsetAsync(ptr, 0, sizeof(h), st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return fail(SSA_ERR_CUDA, "reading the device status word failed");
  if (h)
    return fail(SSA_ERR_DEVICE_TIMEOUT,
                "a bounded device-side wait expired on device %d; the sm_100a kernels launched "
                "since then skipped their work and wrote NaN outputs (status now cleared)",
                dev);
  return SSA_OK;
}

}  // extern "C"
