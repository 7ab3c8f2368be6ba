// ssa_generic.cu — generic SSA attention kernels: fp32 arithmetic on CUDA cores (SIMT).
//
// These serve fp32 inputs (the reference's fp32 mode, ssa_triton_kernel.py:779-784, where the
// parity bar is 1e-5 relative and tensor cores cannot help: tcgen05 has no full-fp32 MMA) and
// the head dim that has no tcgen05 kernel (D = 16). bf16/fp16 with D in {32, 64, 128} (the
// reference's own test matrix uses D = 32, check_ssa_triton_parity.py:1025) run on the sm_100a
// tcgen05 kernels instead (ssa_sm100_fwd.cu / ssa_sm100_bwd.cu).
//
// Structure follows the reference's kernel set:
//   forward            <-> _ssa_attn_fwd            (ssa_triton_kernel.py:150-260)
//   delta preprocess   <-> _ssa_attn_bwd_preprocess (ssa_triton_kernel.py:267-298)
//   dK/dV + dn/db      <-> _ssa_attn_bwd part 1     (ssa_triton_kernel.py:559-636)
//   dQ                 <-> _ssa_attn_bwd part 2     (ssa_triton_kernel.py:638-719)
//   dn/db reduce       <-> dn_partial.sum()         (ssa_triton_kernel.py:894-895)
// Every output element is written by exactly one thread (no atomics), so results are
// bit-deterministic run to run, as the reference's determinism suite requires
// (check_ssa_triton_parity.py:507-562).
#include "ssa_internal.h"

namespace ssa {

namespace {

constexpr int kBM = 64;   // query rows per tile
constexpr int kBN = 64;   // key rows per tile
constexpr int kNT = 256;  // threads per block: 64 rows x 4 lanes

template <typename T, int D>
__device__ __forceinline__ void load_tile_f32(float* dst, int ldd, const TensorRef& t,
                                              const Problem& p, int z, int h, int seq_start,
                                              int row0, int L) {
  const T* base = reinterpret_cast<const T*>(t.ptr);
  for (int idx = threadIdx.x; idx < 64 * D; idx += kNT) {
    const int rr = idx / D, d = idx - rr * D;
    const int row = row0 + rr;
    float x = 0.f;
    if (row < L) x = to_f32<T>(base[row_offset(t, p, z, h, seq_start, row) + d]);
    dst[rr * ldd + d] = x;
  }
}

__device__ __forceinline__ float quad_max(float x) {
  x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 1));
  return fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 2));
}
__device__ __forceinline__ float quad_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  return x + __shfl_xor_sync(0xffffffffu, x, 2);
}

// Block-wide deterministic sum (fixed shuffle tree, then a fixed warp order).
__device__ __forceinline__ float block_sum(float x, float* red) {
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = x;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x == 0)
    for (int i = 0; i < kNT / 32; ++i) s += red[i];
  return s;
}

// ---------------------------------------------------------------------------------------------
// Forward: one block per (64-row query tile, sequence z, q-head). Online base-2 normaliser
// exactly as ssa_triton_kernel.py:107-113; epilogue O = acc / l, M = m + log2(l) (:248-255).
template <typename T, int D>
__global__ void __launch_bounds__(kNT) fwd_generic_kernel(Problem p, TensorRef q, TensorRef k,
                                                          TensorRef v, TensorRef o, float* lse) {
  constexpr int DP = D + 1, DPT = D / 4, PP = kBN + 1;
  extern __shared__ float smem[];
  float* Qs = smem;
  float* Ks = Qs + kBM * DP;
  float* Vs = Ks + kBN * DP;
  float* Ps = Vs + kBN * DP;

  const int tid = threadIdx.x, r = tid >> 2, sub = tid & 3;
  const int z = blockIdx.y / p.Hq, hq = blockIdx.y % p.Hq, hkv = hq / p.gqa;
  int seq_start, L;
  seq_bounds(p, z, seq_start, L);
  const int m0 = (gridDim.x - 1 - blockIdx.x) * kBM;  // longest causal rows first
  if (m0 >= L) return;
  const float n = load_n(p, hq), b = __ldg(p.b_ptr);

  load_tile_f32<T, D>(Qs, DP, q, p, z, hq, seq_start, m0, L);
  const int row = m0 + r;
  float m_run = -INFINITY, l_run = 0.f;
  float acc[DPT];
#pragma unroll
  for (int e = 0; e < DPT; ++e) acc[e] = 0.f;

  const int kv_end = p.causal ? min(L, m0 + kBM) : L;
  for (int n0 = 0; n0 < kv_end; n0 += kBN) {
    __syncthreads();
    load_tile_f32<T, D>(Ks, DP, k, p, z, hkv, seq_start, n0, L);
    load_tile_f32<T, D>(Vs, DP, v, p, z, hkv, seq_start, n0, L);
    __syncthreads();
    float t2[kBN / 4];
    float bmax = -INFINITY;
#pragma unroll
    for (int c = 0; c < kBN / 4; ++c) {
      const int j = sub + 4 * c, col = n0 + j;
      float dot = 0.f;
#pragma unroll 16
      for (int d = 0; d < D; ++d) dot = fmaf(Qs[r * DP + d], Ks[j * DP + d], dot);
      const float s = dot * p.scale;
      const bool ok = (row < L) && (col < L) && (!p.causal || col <= row);
      float inv;
      const float sl = ssa_signed_log1p(s, b, inv);
      t2[c] = ok ? n * sl * kLog2e : -INFINITY;
      bmax = fmaxf(bmax, t2[c]);
    }
    bmax = quad_max(bmax);
    const float m_new = fmaxf(m_run, bmax);
    const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
    const float alpha = exp2f(m_run - m_use);
    float rs = 0.f;
#pragma unroll
    for (int c = 0; c < kBN / 4; ++c) {
      const float pv = exp2f(t2[c] - m_use);
      Ps[r * PP + sub + 4 * c] = pv;
      rs += pv;
    }
    rs = quad_sum(rs);
    l_run = l_run * alpha + rs;
    m_run = m_new;
#pragma unroll
    for (int e = 0; e < DPT; ++e) acc[e] *= alpha;
    __syncthreads();
    for (int j = 0; j < kBN; ++j) {
      const float pj = Ps[r * PP + j];
#pragma unroll
      for (int e = 0; e < DPT; ++e) acc[e] = fmaf(pj, Vs[j * DP + sub + 4 * e], acc[e]);
    }
  }
  if (row < L) {
    const float l_safe = l_run > 0.f ? l_run : 1.f;
    const float inv_l = 1.f / l_safe;
    T* ob = reinterpret_cast<T*>(o.ptr) + row_offset(o, p, z, hq, seq_start, row);
    if (p.drop_seed) {  // output dropout: column sub + 4e is word `sub` of group e's Philox call
      const DropoutKey dk = dropout_key(p);
      const uint64_t e0 = dropout_index(p, z, hq, seq_start, row);
      const float ks = inv_l * p.drop_scale;
#pragma unroll 4
      for (int e = 0; e < DPT; ++e) {
        const bool keep = (dropout_keep4(dk, e0 + 4 * e) >> sub) & 1u;
        ob[sub + 4 * e] = from_f32<T>(keep ? acc[e] * ks : 0.f);
      }
    } else {
#pragma unroll
      for (int e = 0; e < DPT; ++e) ob[sub + 4 * e] = from_f32<T>(acc[e] * inv_l);
    }
    if (sub == 0) lse[stat_offset(p, z, hq, seq_start, row)] = m_run + log2f(l_safe);
  }
}

// ---------------------------------------------------------------------------------------------
// delta = rowsum(O * dO) in fp32 (ssa_triton_kernel.py:267-298).
// With output dropout (p.drop_seed set) `o` is the dropped output and `dout` the gradient of the
// dropped output: rowsum(o * dout) is the undropped rowsum(O * dO) with dO = dout * keep / (1 - p).
// dout * keep goes to `dom` (contiguous in the logical layout), delta is stored times (1 - p) and
// lse lowered by log2(1 / (1 - p)) goes to `lse_shifted`; with these the gradient kernels produce
// the gradients of dO.
template <typename T>
__global__ void __launch_bounds__(kNT) bwd_preprocess_kernel(Problem p, TensorRef o,
                                                             TensorRef dout, float* delta, T* dom,
                                                             const float* lse,
                                                             float* lse_shifted) {
  const int r = threadIdx.x >> 2, sub = threadIdx.x & 3;
  const int z = blockIdx.y / p.Hq, hq = blockIdx.y % p.Hq;
  int seq_start, L;
  seq_bounds(p, z, seq_start, L);
  const int row = blockIdx.x * kBM + r;
  if (blockIdx.x * kBM >= L) return;
  float acc = 0.f;
  if (row < L) {
    const T* ob = reinterpret_cast<const T*>(o.ptr) + row_offset(o, p, z, hq, seq_start, row);
    const T* db = reinterpret_cast<const T*>(dout.ptr) + row_offset(dout, p, z, hq, seq_start, row);
    for (int d = sub; d < p.D; d += 4) acc = fmaf(to_f32<T>(ob[d]), to_f32<T>(db[d]), acc);
    if (dom) {
      const DropoutKey dk = dropout_key(p);
      const uint64_t e0 = dropout_index(p, z, hq, seq_start, row);
      for (int d = sub; d < p.D; d += 4) {
        const bool keep = (dropout_keep4(dk, e0 + (d - sub)) >> sub) & 1u;
        dom[e0 + d] = keep ? db[d] : from_f32<T>(0.f);
      }
      acc *= p.drop_delta_scale;
    }
  }
  acc = quad_sum(acc);
  if (row < L && sub == 0) {
    const int64_t so = stat_offset(p, z, hq, seq_start, row);
    delta[so] = acc;
    if (dom) lse_shifted[so] = lse[so] - p.drop_lse_shift;
  }
}

// ---------------------------------------------------------------------------------------------
// dK, dV (and dn/db partials): one block per (64-row key tile, sequence z, kv-head); loops the
// GQA q-heads that share the kv-head and all query tiles that can see the key tile
// (ssa_triton_kernel.py:573-623). dn/db partials: [z][hq][key tile].
template <typename T, int D>
__global__ void __launch_bounds__(kNT) bwd_dkdv_generic_kernel(
    Problem p, TensorRef q, TensorRef k, TensorRef v, TensorRef dout, const float* lse,
    const float* delta, TensorRef dk, TensorRef dv, float* dn_part, float* db_part, int ntiles) {
  constexpr int DP = D + 1, DPT = D / 4, PP = kBM + 1;
  extern __shared__ float smem[];
  float* Ks = smem;
  float* Vs = Ks + kBN * DP;
  float* Qs = Vs + kBN * DP;
  float* dOs = Qs + kBM * DP;
  float* Ps = dOs + kBM * DP;
  float* dSs = Ps + kBN * PP;
  float* lse_s = dSs + kBN * PP;
  float* del_s = lse_s + kBM;
  float* red = del_s + kBM;

  const int tid = threadIdx.x, jr = tid >> 2, sub = tid & 3;
  const int z = blockIdx.y / p.Hkv, hkv = blockIdx.y % p.Hkv;
  int seq_start, L;
  seq_bounds(p, z, seq_start, L);
  const int tile = blockIdx.x, n0 = tile * kBN;
  if (n0 >= L) {  // keep the partials well defined
    if (tid < p.gqa) {
      const int64_t pi = ((int64_t)z * p.Hq + hkv * p.gqa + tid) * ntiles + tile;
      dn_part[pi] = 0.f;
      db_part[pi] = 0.f;
    }
    return;
  }
  const float b = __ldg(p.b_ptr);
  load_tile_f32<T, D>(Ks, DP, k, p, z, hkv, seq_start, n0, L);
  load_tile_f32<T, D>(Vs, DP, v, p, z, hkv, seq_start, n0, L);
  const int col = n0 + jr;

  float dk_acc[DPT], dv_acc[DPT];
#pragma unroll
  for (int e = 0; e < DPT; ++e) dk_acc[e] = dv_acc[e] = 0.f;

  for (int g = 0; g < p.gqa; ++g) {
    const int hq = hkv * p.gqa + g;
    const float n = load_n(p, hq), nb = n * b;
    float dn_acc = 0.f, db_acc = 0.f;
    const int m_start = p.causal ? (n0 / kBM) * kBM : 0;
    for (int m0 = m_start; m0 < L; m0 += kBM) {
      __syncthreads();
      load_tile_f32<T, D>(Qs, DP, q, p, z, hq, seq_start, m0, L);
      load_tile_f32<T, D>(dOs, DP, dout, p, z, hq, seq_start, m0, L);
      if (tid < kBM) {
        const int row = m0 + tid;
        lse_s[tid] = row < L ? lse[stat_offset(p, z, hq, seq_start, row)] : 0.f;
        del_s[tid] = row < L ? delta[stat_offset(p, z, hq, seq_start, row)] : 0.f;
      }
      __syncthreads();
#pragma unroll 4
      for (int c = 0; c < kBM / 4; ++c) {
        const int i = sub + 4 * c, row = m0 + i;
        float dot = 0.f, dp = 0.f;
#pragma unroll 16
        for (int d = 0; d < D; ++d) {
          dot = fmaf(Qs[i * DP + d], Ks[jr * DP + d], dot);
          dp = fmaf(dOs[i * DP + d], Vs[jr * DP + d], dp);
        }
        const bool ok = (row < L) && (col < L) && (!p.causal || col <= row);
        float pv = 0.f, ds = 0.f;
        if (ok) {
          const float s = dot * p.scale;
          float inv;
          const float sl = ssa_signed_log1p(s, b, inv);
          pv = exp2f(n * sl * kLog2e - lse_s[i]);
          const float dss = pv * (dp - del_s[i]);
          ds = dss * nb * inv;
          dn_acc = fmaf(dss, sl, dn_acc);
          db_acc = fmaf(dss * n, s * inv, db_acc);
        }
        Ps[jr * PP + i] = pv;
        dSs[jr * PP + i] = ds * p.scale;
      }
      __syncthreads();
      for (int i = 0; i < kBM; ++i) {
        const float pv = Ps[jr * PP + i], dsv = dSs[jr * PP + i];
#pragma unroll
        for (int e = 0; e < DPT; ++e) {
          dv_acc[e] = fmaf(pv, dOs[i * DP + sub + 4 * e], dv_acc[e]);
          dk_acc[e] = fmaf(dsv, Qs[i * DP + sub + 4 * e], dk_acc[e]);
        }
      }
    }
    const float dn_blk = block_sum(dn_acc, red);
    const float db_blk = block_sum(db_acc, red);
    if (tid == 0) {
      const int64_t pi = ((int64_t)z * p.Hq + hq) * ntiles + tile;
      dn_part[pi] = dn_blk;
      db_part[pi] = db_blk;
    }
  }
  if (col < L) {
    T* dkb = reinterpret_cast<T*>(dk.ptr) + row_offset(dk, p, z, hkv, seq_start, col);
    T* dvb = reinterpret_cast<T*>(dv.ptr) + row_offset(dv, p, z, hkv, seq_start, col);
#pragma unroll
    for (int e = 0; e < DPT; ++e) {
      dkb[sub + 4 * e] = from_f32<T>(dk_acc[e]);
      dvb[sub + 4 * e] = from_f32<T>(dv_acc[e]);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// dQ: one block per (64-row query tile, sequence z, q-head), all visible key tiles
// (ssa_triton_kernel.py:643-719).
template <typename T, int D>
__global__ void __launch_bounds__(kNT) bwd_dq_generic_kernel(Problem p, TensorRef q, TensorRef k,
                                                             TensorRef v, TensorRef dout,
                                                             const float* lse,
                                                             const float* delta, TensorRef dq) {
  constexpr int DP = D + 1, DPT = D / 4, PP = kBN + 1;
  extern __shared__ float smem[];
  float* Qs = smem;
  float* dOs = Qs + kBM * DP;
  float* Ks = dOs + kBM * DP;
  float* Vs = Ks + kBN * DP;
  float* dSs = Vs + kBN * DP;

  const int tid = threadIdx.x, ir = tid >> 2, sub = tid & 3;
  const int z = blockIdx.y / p.Hq, hq = blockIdx.y % p.Hq, hkv = hq / p.gqa;
  int seq_start, L;
  seq_bounds(p, z, seq_start, L);
  const int m0 = (gridDim.x - 1 - blockIdx.x) * kBM;
  if (m0 >= L) return;
  const float n = load_n(p, hq), b = __ldg(p.b_ptr), nb = n * b;
  load_tile_f32<T, D>(Qs, DP, q, p, z, hq, seq_start, m0, L);
  load_tile_f32<T, D>(dOs, DP, dout, p, z, hq, seq_start, m0, L);
  const int row = m0 + ir;
  const float lse_r = row < L ? lse[stat_offset(p, z, hq, seq_start, row)] : 0.f;
  const float del_r = row < L ? delta[stat_offset(p, z, hq, seq_start, row)] : 0.f;

  float dq_acc[DPT];
#pragma unroll
  for (int e = 0; e < DPT; ++e) dq_acc[e] = 0.f;
  const int kv_end = p.causal ? min(L, m0 + kBM) : L;
  for (int n0 = 0; n0 < kv_end; n0 += kBN) {
    __syncthreads();
    load_tile_f32<T, D>(Ks, DP, k, p, z, hkv, seq_start, n0, L);
    load_tile_f32<T, D>(Vs, DP, v, p, z, hkv, seq_start, n0, L);
    __syncthreads();
#pragma unroll 4
    for (int c = 0; c < kBN / 4; ++c) {
      const int j = sub + 4 * c, col = n0 + j;
      float dot = 0.f, dp = 0.f;
#pragma unroll 16
      for (int d = 0; d < D; ++d) {
        dot = fmaf(Qs[ir * DP + d], Ks[j * DP + d], dot);
        dp = fmaf(dOs[ir * DP + d], Vs[j * DP + d], dp);
      }
      const bool ok = (row < L) && (col < L) && (!p.causal || col <= row);
      float ds = 0.f;
      if (ok) {
        const float s = dot * p.scale;
        float inv;
        const float sl = ssa_signed_log1p(s, b, inv);
        const float pv = exp2f(n * sl * kLog2e - lse_r);
        ds = pv * (dp - del_r) * nb * inv;
      }
      dSs[ir * PP + j] = ds * p.scale;
    }
    __syncthreads();
    for (int j = 0; j < kBN; ++j) {
      const float dsv = dSs[ir * PP + j];
#pragma unroll
      for (int e = 0; e < DPT; ++e) dq_acc[e] = fmaf(dsv, Ks[j * DP + sub + 4 * e], dq_acc[e]);
    }
  }
  if (row < L) {
    T* qb = reinterpret_cast<T*>(dq.ptr) + row_offset(dq, p, z, hq, seq_start, row);
#pragma unroll
    for (int e = 0; e < DPT; ++e) qb[sub + 4 * e] = from_f32<T>(dq_acc[e]);
  }
}

// ---------------------------------------------------------------------------------------------
// dn / db reduction as its own launch (generic path and the allocation-free backward): one block
// per dn head plus one for db (dndb_reduce_block). 1024 threads per block: the db block sums every
// partial of the call (B * Hq * P values), so its per-thread loop bounds this kernel's time.
constexpr int kRedNT = 1024;
__global__ void __launch_bounds__(kRedNT) dndb_reduce_kernel(const float* dn_part,
                                                             const float* db_part, int Z, int Hq,
                                                             int P, int n_per_head, float* dn,
                                                             float* db) {
  __shared__ double red[kRedNT];
  dndb_reduce_block<kRedNT>(blockIdx.x, dn_part, db_part, Z, Hq, P, n_per_head, dn, db, red);
}

template <typename T, int D>
int run_fwd_generic(const Problem& p, TensorRef q, TensorRef k, TensorRef v, TensorRef o,
                    float* lse, cudaStream_t st) {
  constexpr int DP = D + 1;
  const size_t smem = sizeof(float) * (size_t)(kBM * DP + 2 * kBN * DP + kBM * (kBN + 1));
  auto kern = fwd_generic_kernel<T, D>;
  if (set_smem_limit_once(reinterpret_cast<const void*>(kern), (int)smem) != SSA_OK)
    return SSA_ERR_CUDA;
  dim3 grid((p.max_seqlen + kBM - 1) / kBM, p.B * p.Hq);
  kern<<<grid, kNT, smem, st>>>(p, q, k, v, o, lse);
  note_launches(1);
  return SSA_OK;
}

template <typename T, int D>
int run_bwd_generic(const Problem& p, TensorRef q, TensorRef k, TensorRef v, TensorRef dout,
                    const float* lse, const float* delta, TensorRef dq, TensorRef dk,
                    TensorRef dv, float* dn_part, float* db_part, int ntiles, cudaStream_t st) {
  constexpr int DP = D + 1;
  const size_t smem_kv = sizeof(float) * (size_t)(2 * kBN * DP + 2 * kBM * DP +
                                                  2 * kBN * (kBM + 1) + 2 * kBM + 32);
  const size_t smem_q = sizeof(float) * (size_t)(2 * kBM * DP + 2 * kBN * DP + kBM * (kBN + 1));
  auto kkv = bwd_dkdv_generic_kernel<T, D>;
  auto kq = bwd_dq_generic_kernel<T, D>;
  if (set_smem_limit_once(reinterpret_cast<const void*>(kkv), (int)smem_kv) != SSA_OK ||
      set_smem_limit_once(reinterpret_cast<const void*>(kq), (int)smem_q) != SSA_OK)
    return SSA_ERR_CUDA;
  dim3 gkv(ntiles, p.B * p.Hkv);
  kkv<<<gkv, kNT, smem_kv, st>>>(p, q, k, v, dout, lse, delta, dk, dv, dn_part, db_part, ntiles);
  dim3 gq((p.max_seqlen + kBM - 1) / kBM, p.B * p.Hq);
  kq<<<gq, kNT, smem_q, st>>>(p, q, k, v, dout, lse, delta, dq);
  note_launches(2);
  return SSA_OK;
}

template <typename T>
int dispatch_d_fwd(const Problem& p, TensorRef q, TensorRef k, TensorRef v, TensorRef o,
                   float* lse, cudaStream_t st) {
  switch (p.D) {
    case 16: return run_fwd_generic<T, 16>(p, q, k, v, o, lse, st);
    case 32: return run_fwd_generic<T, 32>(p, q, k, v, o, lse, st);
    case 64: return run_fwd_generic<T, 64>(p, q, k, v, o, lse, st);
    case 128: return run_fwd_generic<T, 128>(p, q, k, v, o, lse, st);
    default: return SSA_ERR_UNSUPPORTED;
  }
}

template <typename T>
int dispatch_d_bwd(const Problem& p, TensorRef q, TensorRef k, TensorRef v, TensorRef dout,
                   const float* lse, const float* delta, TensorRef dq, TensorRef dk, TensorRef dv,
                   float* dn_part, float* db_part, int ntiles, cudaStream_t st) {
  switch (p.D) {
    case 16: return run_bwd_generic<T, 16>(p, q, k, v, dout, lse, delta, dq, dk, dv, dn_part, db_part, ntiles, st);
    case 32: return run_bwd_generic<T, 32>(p, q, k, v, dout, lse, delta, dq, dk, dv, dn_part, db_part, ntiles, st);
    case 64: return run_bwd_generic<T, 64>(p, q, k, v, dout, lse, delta, dq, dk, dv, dn_part, db_part, ntiles, st);
    case 128: return run_bwd_generic<T, 128>(p, q, k, v, dout, lse, delta, dq, dk, dv, dn_part, db_part, ntiles, st);
    default: return SSA_ERR_UNSUPPORTED;
  }
}

}  // namespace

bool generic_supports_head_dim(int D) { return D == 16 || D == 32 || D == 64 || D == 128; }

int generic_bwd_partials_per_seq(const Problem& p) { return (p.max_seqlen + kBN - 1) / kBN; }

int launch_fwd_generic(int dtype, const Problem& p, TensorRef q, TensorRef k, TensorRef v,
                       TensorRef o, float* lse, cudaStream_t st) {
  switch (dtype) {
    case SSA_DTYPE_F32: return dispatch_d_fwd<float>(p, q, k, v, o, lse, st);
    case SSA_DTYPE_F16: return dispatch_d_fwd<__half>(p, q, k, v, o, lse, st);
    case SSA_DTYPE_BF16: return dispatch_d_fwd<__nv_bfloat16>(p, q, k, v, o, lse, st);
    default: return SSA_ERR_UNSUPPORTED;
  }
}

int launch_bwd_preprocess(int dtype, const Problem& p, TensorRef o, TensorRef dout, float* delta,
                          void* dom, const float* lse, float* lse_shifted, cudaStream_t st) {
  dim3 grid((p.max_seqlen + kBM - 1) / kBM, p.B * p.Hq);
  switch (dtype) {
    case SSA_DTYPE_F32: bwd_preprocess_kernel<float><<<grid, kNT, 0, st>>>(p, o, dout, delta, static_cast<float*>(dom), lse, lse_shifted); break;
    case SSA_DTYPE_F16: bwd_preprocess_kernel<__half><<<grid, kNT, 0, st>>>(p, o, dout, delta, static_cast<__half*>(dom), lse, lse_shifted); break;
    case SSA_DTYPE_BF16: bwd_preprocess_kernel<__nv_bfloat16><<<grid, kNT, 0, st>>>(p, o, dout, delta, static_cast<__nv_bfloat16*>(dom), lse, lse_shifted); break;
    default: return SSA_ERR_UNSUPPORTED;
  }
  note_launches(1);
  return SSA_OK;
}

int launch_bwd_generic(int dtype, const Problem& p, TensorRef q, TensorRef k, TensorRef v,
                       TensorRef dout, const float* lse, const float* delta, TensorRef dq,
                       TensorRef dk, TensorRef dv, float* dn_part, float* db_part,
                       cudaStream_t st) {
  const int ntiles = generic_bwd_partials_per_seq(p);
  switch (dtype) {
    case SSA_DTYPE_F32: return dispatch_d_bwd<float>(p, q, k, v, dout, lse, delta, dq, dk, dv, dn_part, db_part, ntiles, st);
    case SSA_DTYPE_F16: return dispatch_d_bwd<__half>(p, q, k, v, dout, lse, delta, dq, dk, dv, dn_part, db_part, ntiles, st);
    case SSA_DTYPE_BF16: return dispatch_d_bwd<__nv_bfloat16>(p, q, k, v, dout, lse, delta, dq, dk, dv, dn_part, db_part, ntiles, st);
    default: return SSA_ERR_UNSUPPORTED;
  }
}

int launch_dndb_reduce(const float* dn_part, const float* db_part, int Z, int Hq, int P,
                       int n_per_head, float* dn, float* db, cudaStream_t st) {
  const int blocks = (n_per_head ? Hq : 1) + 1;
  dndb_reduce_kernel<<<blocks, kRedNT, 0, st>>>(dn_part, db_part, Z, Hq, P, n_per_head, dn, db);
  note_launches(1);
  return SSA_OK;
}

}  // namespace ssa
