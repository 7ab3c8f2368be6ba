// ssa_tmap.h — TMA tensor maps for strided [B, H, N, D] (or packed [T, H, D]) 16-bit tensors.
//
// A map is 4-D {D, rows, H, B} with byte strides {sN, sH, sB} and a {64, box_rows, 1, 1} box
// in the 128-byte swizzle, so one box is a [box_rows x 64] slab of 128-byte rows, exactly the
// K-major SW128 operand layout tcgen05.mma reads. Rows past the end of a sequence's tensor
// extent read as zero (out-of-bounds fill). cuTensorMapEncodeTiled is fetched through the
// runtime's driver entry point, so the library does not link libcuda directly.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "ssa_common.cuh"
#include "ssa_internal.h"

namespace ssa {

PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder();

// True when a 16-bit tensor's base and strides satisfy TMA's 16-byte rules.
inline bool tma_compatible(const TensorRef& t, const Problem& p, int H) {
  const uintptr_t base = reinterpret_cast<uintptr_t>(t.ptr);
  if (base % 16) return false;
  const int64_t es = 2;
  const int rows = p.N;
  if (rows > 1 && ((t.sN * es) % 16 || t.sN <= 0)) return false;
  if (H > 1 && ((t.sH * es) % 16 || t.sH <= 0)) return false;
  if (!p.cu_seqlens && p.B > 1 && ((t.sB * es) % 16 || t.sB <= 0)) return false;
  return true;
}

inline int make_tmap_bhnd(CUtensorMap* map, const TensorRef& t, const Problem& p, int dtype,
                          int H, int box_rows) {
  auto enc = tmap_encoder();
  if (!enc) return SSA_ERR_CUDA;
  if (!tma_compatible(t, p, H))
    return abi_error(SSA_ERR_BAD_STRIDE, "tensor at %p: base and B/H/N strides must be 16-byte "
                     "aligned for TMA", t.ptr);
  const uint64_t es = 2;
  const uint64_t B = p.cu_seqlens ? 1 : (uint64_t)p.B;
  const uint64_t rows = (uint64_t)p.N;
  // Strides of extent-1 dimensions never move the address; give them a legal value.
  const uint64_t sN = rows > 1 ? (uint64_t)t.sN * es : 16;
  const uint64_t sH = H > 1 ? (uint64_t)t.sH * es : 16;
  const uint64_t sB = B > 1 ? (uint64_t)t.sB * es : 16;
  cuuint64_t dims[4] = {(cuuint64_t)p.D, rows, (cuuint64_t)H, B};
  cuuint64_t strides[3] = {sN, sH, sB};
  cuuint32_t box[4] = {64u, (cuuint32_t)box_rows, 1u, 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  const CUtensorMapDataType dt =
      dtype == SSA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, dt, 4, t.ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return abi_error(SSA_ERR_BAD_STRIDE,
                     "cuTensorMapEncodeTiled failed (CUresult %d) for ptr %p dims {%llu, %llu, "
                     "%llu, %llu} byte strides {%llu, %llu, %llu} box rows %d",
                     (int)r, t.ptr, (unsigned long long)dims[0], (unsigned long long)dims[1],
                     (unsigned long long)dims[2], (unsigned long long)dims[3],
                     (unsigned long long)sN, (unsigned long long)sH, (unsigned long long)sB,
                     box_rows);
  return SSA_OK;
}

}  // namespace ssa
