// ssa_common.cuh — parameter blocks, dtype helpers and the SSA logit transform shared by
// the generic (SIMT) and the sm_100a (tcgen05/TMA) kernels.
//
// The SSA transform (reference: training/train/train_ssa_triton/SSA/ssa_triton_kernel.py:96-107):
//     s  = softmax_scale * (q . k)
//     u  = b * |s|
//     t  = n * sign(s) * log1p(u)
//     t2 = t * log2(e)                      (base-2 online normaliser, :107-113)
// Backward chain rule (:378-397):
//     ds_ssa = P * (dP - Delta)
//     dL/ds  = ds_ssa * n * b / (1 + u)
//     dn    += ds_ssa * sign(s) * log1p(u)
//     db    += ds_ssa * n * sign(s) * |s| / (1 + u)  ( = ds_ssa * n * s / (1 + u) )
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "ssa_b200.h"

namespace ssa {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Device-side problem block (plain data, passed by value to every kernel).
struct Problem {
  int B, Hq, Hkv, N, D, gqa;
  int causal;
  float scale;
  const float* n_ptr;
  int n_per_head;
  const float* b_ptr;
  const int* cu_seqlens;         // nullptr: dense
  const int* cu_seqlens_padded;  // packed with padding: start row of each document, or nullptr
  int max_seqlen;                // rows a sequence can have (N when dense)
  int det;                       // tensor-core backward: bit-reproducible dq (ordered dQ adds)
  // Output dropout (0 = off): keep an element iff its Philox word >> 8 >= drop_thr
  // (= ceil(p * 2^24)); the forward scales kept elements by drop_scale (= 1 / (1 - p), fp32).
  // The backward runs on dout * keep (exact in any dtype) and moves the 1 / (1 - p) into fp32
  // quantities instead: delta is multiplied by drop_delta_scale (= 1 - p) and every lse read
  // by the backward kernels is lowered by drop_lse_shift (= log2(1 / (1 - p))), so P comes out
  // multiplied by 1 / (1 - p). Then P (dP - delta) and P^T dO are the gradients of the scaled
  // dO without a rounding of dout / (1 - p) to 16 bits. Off: 1, 1, 0.
  uint32_t drop_thr;
  float drop_scale;
  float drop_delta_scale;
  float drop_lse_shift;
  const unsigned long long* drop_seed;  // device: [0] Philox key, [1] counter offset
};

struct TensorRef {
  void* ptr;
  int64_t sB, sH, sN;
};

// Start row and length of sequence z (a batch entry, or a document when varlen).
__device__ __forceinline__ void seq_bounds(const Problem& p, int z, int& start, int& len) {
  if (p.cu_seqlens) {
    const int c0 = __ldg(p.cu_seqlens + z);
    len = __ldg(p.cu_seqlens + z + 1) - c0;
    start = p.cu_seqlens_padded ? __ldg(p.cu_seqlens_padded + z) : c0;
  } else {
    start = 0;
    len = p.N;
  }
}

// Element offset of (z, h, row) in a strided tensor; row is relative to the sequence start.
__device__ __forceinline__ int64_t row_offset(const TensorRef& t, const Problem& p, int z, int h,
                                              int seq_start, int row) {
  const int64_t zb = p.cu_seqlens ? 0 : (int64_t)z * t.sB;
  return zb + (int64_t)h * t.sH + (int64_t)(seq_start + row) * t.sN;
}

// Offset into a [B, Hq, N] (dense) or [Hq, T] (varlen) fp32 row-statistics array (lse, delta).
__device__ __forceinline__ int64_t stat_offset(const Problem& p, int z, int h, int seq_start,
                                               int row) {
  if (p.cu_seqlens) return (int64_t)h * p.N + seq_start + row;  // N == T (total tokens)
  return ((int64_t)z * p.Hq + h) * p.N + row;
}

// ---------------------------------------------------------------------------------------------
// Output dropout. The reference drops attention-output elements with nn.Dropout after its kernel
// (training/train/train_ssa_triton/SSA/ssa_triton_attention.py:110-113,186-193); here the forward
// epilogue applies the mask and the backward's delta pass applies it to dout. Keep decisions come
// from Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3",
// SC 2011): ten rounds of two 32x32->64-bit products with the paper's multipliers, the key
// advanced by the paper's Weyl increments between rounds. Element e (its position in the
// logical contiguous output: ((z * Hq + h) * N + row) * D + d dense, (t * Hq + h) * D + d
// packed) takes word e % 4 of the call with counter (e / 4, offset) and key seed.

__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

// Index of element (z, h, row, d = 0), row relative to seq_start.
__device__ __forceinline__ uint64_t dropout_index(const Problem& p, int z, int h, int seq_start,
                                                  int row) {
  if (p.cu_seqlens) return ((uint64_t)(seq_start + row) * p.Hq + h) * (uint64_t)p.D;
  return (((uint64_t)z * p.Hq + h) * p.N + row) * (uint64_t)p.D;
}

struct DropoutKey {
  uint32_t k0, k1, o0, o1, thr;
};
__device__ __forceinline__ DropoutKey dropout_key(const Problem& p) {
  const unsigned long long key = __ldg(p.drop_seed), off = __ldg(p.drop_seed + 1);
  return DropoutKey{(uint32_t)key, (uint32_t)(key >> 32), (uint32_t)off, (uint32_t)(off >> 32),
                    p.drop_thr};
}

// Keep bits of the four elements e .. e + 3 (e a multiple of 4): bit i for element e + i.
__device__ __forceinline__ uint32_t dropout_keep4(const DropoutKey& k, uint64_t e) {
  const uint64_t c = e >> 2;
  const uint4 w = philox4x32_10(make_uint4((uint32_t)c, (uint32_t)(c >> 32), k.o0, k.o1), k.k0,
                                k.k1);
  return (uint32_t)((w.x >> 8) >= k.thr) | ((uint32_t)((w.y >> 8) >= k.thr) << 1) |
         ((uint32_t)((w.z >> 8) >= k.thr) << 2) | ((uint32_t)((w.w >> 8) >= k.thr) << 3);
}

__device__ __forceinline__ float load_n(const Problem& p, int hq) {
  return __ldg(p.n_ptr + (p.n_per_head ? hq : 0));
}

// The device status word (non-zero after an expired bounded wait), read by one thread and shared
// with the block: every thread of every block reading the one word directly piles the loads onto
// a single L2 slice (that cost the dq conversion a third of its time on B200). Called by every
// thread of the block at a point they all reach; contains a __syncthreads.
__device__ __forceinline__ bool block_status_failed(const unsigned int* status) {
  __shared__ unsigned int s_status;
  if (threadIdx.x == 0) s_status = *reinterpret_cast<const volatile unsigned int*>(status);
  __syncthreads();
  return s_status != 0;
}

// Quiet NaN written into the outputs of a kernel that skipped its work because a bounded device
// wait expired (in this launch or an earlier one): a caller that never reads the status word still
// sees the failure as NaN in out / lse / dq / dk / dv / dn / db instead of stale memory.
constexpr uint32_t kNaNBf16x2 = 0x7FC07FC0u, kNaNF16x2 = 0x7E007E00u;
__device__ __forceinline__ float nan_f32() { return __uint_as_float(0x7FC00000u); }

// NaN into rows [row0, row1) (every head dim) of head h of sequence z of a 16-bit tensor whose
// rows are 16-byte aligned (true on the TMA path), and into the matching fp32 row statistics when
// stat != nullptr. Called by every thread of the block.
template <bool BF16>
__device__ __forceinline__ void nan_fill_rows16(const TensorRef& t, const Problem& p, int z, int h,
                                                int seq_start, int row0, int row1, float* stat) {
  const uint32_t w = BF16 ? kNaNBf16x2 : kNaNF16x2;
  const int per_row = p.D / 8;  // 16-byte chunks per row
  const int total = (row1 - row0) * per_row;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int r = row0 + i / per_row, c = i - (i / per_row) * per_row;
    uint16_t* rowp = reinterpret_cast<uint16_t*>(t.ptr) + row_offset(t, p, z, h, seq_start, r);
    reinterpret_cast<uint4*>(rowp)[c] = make_uint4(w, w, w, w);
  }
  if (stat)
    for (int r = row0 + (int)threadIdx.x; r < row1; r += blockDim.x)
      stat[stat_offset(p, z, h, seq_start, r)] = nan_f32();
}

template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Accurate transform used by the generic path (fp32 inputs need 1e-5 relative parity):
// returns sign(s)*log1p(b|s|) (natural log) and 1/(1+b|s|) through out-params.
__device__ __forceinline__ float ssa_signed_log1p(float s, float b, float& inv_1pu) {
  const float u = b * fabsf(s);
  inv_1pu = 1.0f / (1.0f + u);
  const float l = log1pf(u);
  return s > 0.f ? l : (s < 0.f ? -l : 0.f);
}


// dn / db: deterministic fp64 reduction of per-tile partials laid out [Z][Hq][P], by one block of
// NT threads. Block h < nh (nh = Hq for a per-head n, else 1) sums dn for head h (or, for a
// scalar n, every partial); block nh sums db. Each thread walks a fixed strided subset, then a
// fixed tree: the result does not depend on scheduling. red: NT doubles of shared memory.
template <int NT>
__device__ __forceinline__ void dndb_reduce_block(int h, const float* dn_part, const float* db_part,
                                                  int Z, int Hq, int P, int n_per_head, float* dn,
                                                  float* db, double* red) {
  const int tid = threadIdx.x;
  const int nh = n_per_head ? Hq : 1;
  const int64_t per_head = (int64_t)Z * P;
  double s = 0.0;
  if (h < nh && n_per_head) {
    for (int64_t i = tid; i < per_head; i += NT) {
      const int64_t zz = i / P, pp = i - zz * P;
      s += (double)dn_part[(zz * Hq + h) * P + pp];
    }
  } else {
    const float* src = h < nh ? dn_part : db_part;
    for (int64_t i = tid; i < per_head * Hq; i += NT) s += (double)src[i];
  }
  red[tid] = s;
  __syncthreads();
  for (int o = NT / 2; o > 0; o >>= 1) {
    if (tid < o) red[tid] += red[tid + o];
    __syncthreads();
  }
  if (tid == 0) {
    if (h < nh) dn[h] = (float)red[0];
    else db[0] = (float)red[0];
  }
}

}  // namespace ssa
