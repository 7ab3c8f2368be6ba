// ssa_internal.h — launchers shared between the C ABI (ssa_capi.cu) and the kernel files.
#pragma once

#include "ssa_common.cuh"

namespace ssa {

// Generic fp32-compute kernels (ssa_generic.cu).
bool generic_supports_head_dim(int D);
int generic_bwd_partials_per_seq(const Problem& p);
int launch_fwd_generic(int dtype, const Problem& p, TensorRef q, TensorRef k, TensorRef v,
                       TensorRef o, float* lse, cudaStream_t st);
// delta = rowsum(o * dout); with output dropout on (p.drop_seed) and dom != nullptr it also
// writes dout * keep into dom (contiguous [B, Hq, N, D], or [T, Hq, D] packed), stores delta
// times (1 - p) and writes lse - log2(1 / (1 - p)) into lse_shifted: the inputs the gradient
// kernels take under dropout (the Problem's dropout fields).
int launch_bwd_preprocess(int dtype, const Problem& p, TensorRef o, TensorRef dout, float* delta,
                          void* dom, const float* lse, float* lse_shifted, cudaStream_t st);
int launch_bwd_generic(int dtype, const Problem& p, TensorRef q, TensorRef k, TensorRef v,
                       TensorRef dout, const float* lse, const float* delta, TensorRef dq,
                       TensorRef dk, TensorRef dv, float* dn_part, float* db_part,
                       cudaStream_t st);
int launch_dndb_reduce(const float* dn_part, const float* db_part, int Z, int Hq, int P,
                       int n_per_head, float* dn, float* db, cudaStream_t st);

// sm_100a tcgen05 / TMA kernels (ssa_sm100_fwd.cu, ssa_sm100_bwd.cu).
bool sm100_supports(int dtype, int D);
int launch_fwd_sm100(int dtype, const Problem& p, TensorRef q, TensorRef k, TensorRef v,
                     TensorRef o, float* lse, cudaStream_t st);
bool sm100_bwd_supports(int dtype, int D);
size_t sm100_bwd_workspace_bytes(const Problem& p);
// Runs its own fused preprocess (delta + dQ-accumulator zeroing, and with output dropout
// dout * keep written to `dom`, which the main kernel then reads) before the main kernel.
int launch_bwd_sm100(int dtype, const Problem& p, TensorRef q, TensorRef k, TensorRef v,
                     TensorRef out, TensorRef dout, const float* lse, float* delta, TensorRef dq,
                     TensorRef dk, TensorRef dv, float* dn, float* db, void* dom, void* ws,
                     size_t ws_bytes, cudaStream_t st);
// Output-dropout scratch, one block of the backward workspace: dout * keep in the logical
// contiguous layout (the dropout index's), then the shifted lse ([B, Hq, N] or [Hq, T] fp32).
inline size_t dropout_dout_bytes(const Problem& p, int elem_bytes) {
  const size_t rows = p.cu_seqlens ? (size_t)p.N : (size_t)p.B * p.N;
  return ((size_t)elem_bytes * rows * (size_t)p.Hq * (size_t)p.D + 255) & ~(size_t)255;
}
inline size_t dropout_scratch_bytes(const Problem& p, int elem_bytes) {
  const size_t rows = p.cu_seqlens ? (size_t)p.N : (size_t)p.B * p.N;
  return dropout_dout_bytes(p, elem_bytes) + ((sizeof(float) * rows * p.Hq + 255) & ~(size_t)255);
}
inline TensorRef dropout_dout_ref(const Problem& p, void* dom) {
  if (p.cu_seqlens) return TensorRef{dom, 0, (int64_t)p.D, (int64_t)p.Hq * p.D};
  return TensorRef{dom, (int64_t)p.Hq * p.N * p.D, (int64_t)p.N * p.D, (int64_t)p.D};
}
inline float* dropout_lse_buffer(const Problem& p, void* dom, int elem_bytes = 2) {
  return reinterpret_cast<float*>(static_cast<uint8_t*>(dom) + dropout_dout_bytes(p, elem_bytes));
}

// Device status word written by bounded waits in the sm_100a kernels.
unsigned int* device_status_ptr();

// Host-side count of kernel launches issued by this library (ssa_kernel_launch_count).
void note_launches(int n);

// Shared C-ABI helpers (ssa_capi.cu): problem validation (status code, message set on
// failure), conversion to the device-side Problem, and recording an error message that
// ssa_last_error() then returns.
int abi_validate_problem(const ssa_problem_t* pr);
// Non-NULL pointer and non-negative B/H/N strides (the rule every entry point applies).
int abi_check_tensor(const ssa_tensor_t& t, const char* name);
Problem abi_to_problem(const ssa_problem_t* pr);
int abi_error(int code, const char* fmt, ...);
// One CTA waiting on an mbarrier nobody completes, with a bounded wait of `cycles` (self-test of
// the device-timeout path; ssa_sm100_fwd.cu).
int launch_selftest_timeout(unsigned int* status, long long cycles, cudaStream_t st);
// Raises `func`'s dynamic shared-memory limit to `bytes` once per device (the attribute lives in
// the context), so later launches, including launches under CUDA stream capture, make no
// attribute call. SSA_OK or SSA_ERR_CUDA.
int set_smem_limit_once(const void* func, int bytes);
// Makes the device owning `ptr` current on the calling thread (see ssa_capi.cu).
int abi_bind_device(const void* ptr, const char* name);

}  // namespace ssa
