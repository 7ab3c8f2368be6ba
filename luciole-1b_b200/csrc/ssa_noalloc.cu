// ssa_noalloc.cu — ssa_attn_bwd_noalloc: the SSA backward with no workspace argument.
//
// Who needs this: callers that cannot allocate device memory at the point where they run the
// backward — for example a binding from another host language that has no device allocator
// of its own, or a training loop whose device memory is reserved up front by a different
// allocator, where a cudaMalloc would fail or stall the device. Every other entry point asks
// the caller for a workspace; this one brings its own.
//
// What it runs: the generic (fp32-arithmetic, CUDA-core) backward kernels of ssa_generic.cu —
// delta preprocess, dK/dV with dn/db partials, dQ, and the dn/db reduction — the same kernels
// ssa_attn_bwd runs for fp32 inputs and for head dims without a tensor-core kernel. Their
// scratch (delta, and the per-tile dn/db partials) lives in the file-scope array below instead
// of a caller workspace. Inputs and outputs are still the caller's.
//
// Limits and sharing rules:
//   * the array holds kNoAllocScratchBytes (16 MiB) on every GPU that loads this library, for
//     the life of the process; a problem whose scratch needs more is rejected with
//     SSA_ERR_WORKSPACE and a message giving both sizes;
//   * every call on a device uses the same array, so two calls whose kernels overlap on the GPU
//     (different streams, or different host threads) race on it and corrupt each other: order
//     them on one stream or synchronise between them;
//   * nothing in the array needs to start at zero: each call writes every scratch element it
//     later reads, so stale contents from an earlier call are never used;
//   * the first call on each device looks up the array's device address (cudaGetSymbolAddress
//     with that device current) and caches it; make that first call before any stream capture
//     begins on the device.
#include <mutex>

#include "ssa_internal.h"

namespace ssa {
namespace {

constexpr size_t kNoAllocScratchBytes = 16u << 20;  // 16 MiB per device

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

size_t round256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Device address of g_noalloc_scratch on the current device (looked up once per device).
int scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SSA_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr) return SSA_ERR_CUDA;
    g_scratch_addr[dev] = ptr;
  }
  *out = g_scratch_addr[dev];
  return SSA_OK;
}

}  // namespace
}  // namespace ssa

using namespace ssa;

extern "C" int ssa_attn_bwd_noalloc(const ssa_problem_t* pr, ssa_tensor_t q, ssa_tensor_t k,
                                    ssa_tensor_t v, ssa_tensor_t out, ssa_tensor_t dout,
                                    const float* lse, ssa_tensor_t dq, ssa_tensor_t dk,
                                    ssa_tensor_t dv, float* dn, float* db, void* stream) {
  int rc = abi_validate_problem(pr);
  if (rc != SSA_OK) return rc;
  if ((rc = abi_check_tensor(q, "q")) || (rc = abi_check_tensor(k, "k")) ||
      (rc = abi_check_tensor(v, "v")) || (rc = abi_check_tensor(out, "out")) ||
      (rc = abi_check_tensor(dout, "dout")) || (rc = abi_check_tensor(dq, "dq")) ||
      (rc = abi_check_tensor(dk, "dk")) || (rc = abi_check_tensor(dv, "dv")))
    return rc;
  if (!lse || !dn || !db) return abi_error(SSA_ERR_NULL, "lse / dn / db is NULL");
  if (pr->dropout_p > 0.f)
    return abi_error(SSA_ERR_UNSUPPORTED,
                     "ssa_attn_bwd_noalloc: output dropout needs a workspace for the masked dout; "
                     "use ssa_attn_bwd");
  const Problem p = abi_to_problem(pr);

  // Scratch layout: delta [Hq x rows] fp32, then dn and db partials [B x Hq x tiles] fp32.
  const size_t rows = pr->cu_seqlens ? (size_t)pr->N : (size_t)pr->B * pr->N;
  const int tiles = generic_bwd_partials_per_seq(p);
  const size_t delta_bytes = round256(sizeof(float) * (size_t)pr->Hq * rows);
  const size_t part_bytes = round256(sizeof(float) * (size_t)pr->B * pr->Hq * (size_t)tiles);
  const size_t need = delta_bytes + 2 * part_bytes;
  if (need > kNoAllocScratchBytes)
    return abi_error(SSA_ERR_WORKSPACE,
                     "ssa_attn_bwd_noalloc: this problem needs %zu bytes of scratch, more than "
                     "the library's fixed %zu-byte device array; use ssa_attn_bwd with a "
                     "caller workspace",
                     need, kNoAllocScratchBytes);
  if ((rc = abi_bind_device(q.ptr, "q")) != SSA_OK) return rc;
  void* base = nullptr;
  if (scratch_address(&base) != SSA_OK)
    return abi_error(SSA_ERR_CUDA, "ssa_attn_bwd_noalloc: cudaGetSymbolAddress failed");
  unsigned char* s = static_cast<unsigned char*>(base);
  float* delta = reinterpret_cast<float*>(s);
  float* dn_part = reinterpret_cast<float*>(s + delta_bytes);
  float* db_part = reinterpret_cast<float*>(s + delta_bytes + part_bytes);

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const TensorRef tq{q.ptr, q.sB, q.sH, q.sN}, tk{k.ptr, k.sB, k.sH, k.sN},
      tv{v.ptr, v.sB, v.sH, v.sN}, to{out.ptr, out.sB, out.sH, out.sN},
      tdo{dout.ptr, dout.sB, dout.sH, dout.sN}, tdq{dq.ptr, dq.sB, dq.sH, dq.sN},
      tdk{dk.ptr, dk.sB, dk.sH, dk.sN}, tdv{dv.ptr, dv.sB, dv.sH, dv.sN};
  rc = launch_bwd_preprocess(pr->dtype, p, to, tdo, delta, nullptr, nullptr, nullptr, st);
  if (rc == SSA_OK)
    rc = launch_bwd_generic(pr->dtype, p, tq, tk, tv, tdo, lse, delta, tdq, tdk, tdv, dn_part,
                            db_part, st);
  if (rc == SSA_OK)
    rc = launch_dndb_reduce(dn_part, db_part, p.B, p.Hq, tiles, p.n_per_head, dn, db, st);
  if (rc != SSA_OK) return abi_error(rc, "ssa_attn_bwd_noalloc: launch setup failed (%d)", rc);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return abi_error(SSA_ERR_LAUNCH, "ssa_attn_bwd_noalloc: %s", cudaGetErrorString(e));
  return SSA_OK;
}
