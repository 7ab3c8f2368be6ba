// ssa_sm100_bwd.cu — SSA attention backward for sm_100a: one fused tcgen05/TMA kernel.
//
// Computes what the reference's _ssa_attn_bwd computes (ssa_triton_kernel.py:488-719, inner
// loops :305-401 and :408-481) in a single pass: for each score element the SSA transform and
// P = exp2(t2 - M) are recomputed ONCE (the reference recomputes them twice, once for dK/dV and
// once for dQ), and
//     dV += P^T dO,   dP = dO V^T,   ds_ssa = P (dP - delta),
//     dS  = ds_ssa * n b / (1 + b|s|) * scale,   dK += dS^T Q,   dQ += dS K,
//     dn += ds_ssa * sign(s) log1p(b|s|),   db += ds_ssa * n s / (1 + b|s|)    (:372-397).
//
// One CTA owns a 128-row key block of one (sequence, kv-head) and walks every q-head of its GQA
// group (ssa_triton_kernel.py:573) and every 128-row query tile that can see the block. Per query
// tile, the two 64-row halves are handled by two warp-groups side by side:
//   warp 12     TMA producer: K, V once; Q and dO tiles through a 3-stage ring; the tile's
//               lse / delta rows into shared memory with plain loads.
//   warp 13     MMA issuer (tcgen05, fp32 accumulation in TMEM):
//                 S^T  = K Q^T,    dP^T = V dO^T            (SS, M=128 keys, N=128 queries)
//                 dV  += P^T dO_h                           (TS: P^T read from TMEM)
//                 dK  += dS^T Q_h                           (SS: dS^T from shared memory)
//                 dQ   = dS K                               (SS, M=128 queries, dS from smem)
//   warps 0..3  half 0 of each tile, one thread per key row: SSA transform, P, dS, dn/db
//   warps 4..7  half 1 of each tile
//   warps 8..11 dQ drain: TMEM -> shared staging -> TMA bulk reduce-adds (fp32) into the
//               dQ accumulator in global memory; a small kernel converts it to dq's dtype.
// The roles sit on whole warpgroups so setmaxnreg can move registers to the P/dS groups.
// TMEM (512 columns): S^T of the tile [0,128) and dP^T [128,256) (half h reads columns
// [64h, 64h + 64) of each), dK [256,320), dV [320,384), dQ [384,448), P^T (packed 16-bit) of
// half h at [448 + 32h, 480 + 32h). Each half pulls its S^T / dP^T into registers half-way
// through its arithmetic and signals it, so the next tile's S^T / dP^T MMAs run under the second
// half of the arithmetic; with P^T outside the S/dP buffers and dS^T in shared memory they do
// not wait for the grads MMAs either.
//
// dn / db: per-thread fp32 sums, reduced per warp at the end of each q-head and written as
// partials [z][hq][key block][half][warp]; a deterministic fp64 kernel sums them.
// dQ accumulation order across key blocks is not fixed (L2 reduce-adds), so dq may differ in
// the last bits from run to run; dk, dv, dn, db are bit-deterministic.
//
// Every mbarrier wait is bounded (~1 s); on expiry the kernel records SSA_ERR_DEVICE_TIMEOUT in
// the device status word and unwinds (later launches then skip their work).
#include <cudaTypedefs.h>

#include "ssa_internal.h"
#include "ssa_sm100.cuh"
#include "ssa_tmap.h"

namespace ssa {
namespace sm100 {

struct BwdCfg {
  static constexpr int D = 64;
  static constexpr int BN = 128;  // key rows per CTA
  static constexpr int BT = 128;  // query rows per tile (two 64-row halves)
  static constexpr uint32_t KV_BYTES = BN * D * 2;   // 16 KB
  static constexpr uint32_t QT_BYTES = BT * D * 2;   // 16 KB
  static constexpr uint32_t HALF_BYTES = QT_BYTES / 2;
  static constexpr uint32_t DS_BYTES = BN * BT * 2;  // 32 KB: two [128 keys x 64 queries] slabs
  static constexpr uint32_t DS_SLAB = DS_BYTES / 2;
  static constexpr int STAGES = 3;                   // Q / dO / lse / delta ring
  static constexpr uint32_t DQS_WARP = 32 * 32 * 4;  // 4 KB: 32 rows x 32 fp32 per drain warp
  static constexpr uint32_t OFF_K = 0;
  static constexpr uint32_t OFF_V = OFF_K + KV_BYTES;
  static constexpr uint32_t OFF_Q = OFF_V + KV_BYTES;               // STAGES tiles
  static constexpr uint32_t OFF_DO = OFF_Q + STAGES * QT_BYTES;     // STAGES tiles
  static constexpr uint32_t OFF_DS = OFF_DO + STAGES * QT_BYTES;    // 2 buffers
  static constexpr uint32_t OFF_DQS = OFF_DS + 2 * DS_BYTES;        // 4 warps x 4 KB
  static constexpr uint32_t OFF_LSE = OFF_DQS + 4 * DQS_WARP;       // STAGES x 128 fp32
  static constexpr uint32_t OFF_DEL = OFF_LSE + STAGES * BT * 4;
  static constexpr uint32_t OFF_BAR = OFF_DEL + STAGES * BT * 4;
  static constexpr uint32_t SMEM_BYTES = OFF_BAR + 256 + 1024;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t COL_S = 0, COL_DP = 128;  // S^T / dP^T of the whole tile
  static constexpr uint32_t COL_DK = 256, COL_DV = 320, COL_DQ = 384;
  static constexpr uint32_t COL_PT = 448;  // P^T (packed 16-bit) for half h at COL_PT + 32 h
  static constexpr int THREADS = 512;
  // Warp roles (warpgroup-aligned so each group can resize its register file):
  //   warps 0..3 / 4..7  P/dS for query halves 0 / 1   (regs raised to REGS_PDS)
  //   warps 8..11        dQ drain                       (REGS_DQ)
  //   warp 12 TMA producer, warp 13 MMA issuer, 14..15 idle (REGS_CTRL)
  // Budget at launch: 512 threads x 128 = 65536; after the moves 2*128*168 + 128*96 + 128*80
  // = 65536 (no role spills at this split; the drain needs 96 for its two 32-column loads).
  static constexpr uint32_t REGS_PDS = 168, REGS_DQ = 96, REGS_CTRL = 80;
  static constexpr int WARP_PRODUCER = 12, WARP_MMA = 13;
};
static_assert(BwdCfg::SMEM_BYTES <= 232448, "shared memory budget");

struct BwdArgs {
  Problem p;
  TensorRef dk, dv;
  const float* lse;
  const float* delta;
  float* dq_accum;    // fp32, [B][Hq][rows_pad][D] dense or [Hq][T + 128][D] packed; zeroed
  int64_t dq_rows;    // rows_pad (dense) or T + 128 (packed) per head
  float* dn_part;     // [B][Hq][nkv][2 halves][4 warps]
  float* db_part;
  unsigned int* status;
  int nkv;            // key blocks per sequence (ceil(max_seqlen / 128))
  // q-head slices per key block: 1, or a divisor of the GQA ratio when the grid would leave SMs
  // idle (few sequences). A slice's CTA holds partial dK / dV, written in fp32 to dkv_part
  // [B][Hkv][nkv][hsplit][dK, dV][128 rows][D] and summed in slice order by the dq conversion.
  int hsplit;
  float* dkv_part;
  // dn / db partials per (sequence, q-head, key block): 8 (two halves x four warps), or, with
  // deterministic dq (tile-major order, heads alternating), 8 per query tile: ppk = 8 * ntq.
  int ppk;
  int ntq;      // query tiles per sequence (ceil(max_seqlen / query tile rows))
  int* dq_sem;  // deterministic dq: turn counters [B][Hq][ntq][4 drain warps], zeroed per call
};

__device__ __forceinline__ int64_t bwd_partial_index(const BwdArgs& a, int z, int hq, int kvb,
                                                     int tile_slot) {
  return ((int64_t)z * a.p.Hq + hq) * ((int64_t)a.ppk * a.nkv) + (int64_t)a.ppk * kvb +
         8 * tile_slot;
}

// Tile t of a CTA's loop -> (q-head g within its slice, query tile tt within the head). Default
// order: heads outer, tiles ascending. Deterministic-dQ order: tiles descending outer, heads inner,
// so the CTAs of all key blocks of a (sequence, slice) reach a query tile together and the
// ordered dQ adds pass along the key blocks with a short lag that does not grow.
__device__ __forceinline__ void tile_coords(int t, int T_h, int gh, int det, int& g, int& tt) {
  if (det) {
    const int k = t / gh;
    g = t - k * gh;
    tt = T_h - 1 - k;
  } else {
    g = t / T_h;
    tt = t - g * T_h;
  }
}

// CTA -> work unit. Key block 0 (the most query tiles) first, then the q-head slice, then the
// (sequence, kv-head); a slice covers q-heads [g0, g0 + gh) of the GQA group.
struct BwdUnit {
  int kvb, sp, z, hkv, g0, gh;
};
__device__ __forceinline__ BwdUnit bwd_unit(const Problem& p, int hsplit) {
  const int BHkv = p.B * p.Hkv;
  const int per_kvb = BHkv * hsplit;
  BwdUnit u;
  u.kvb = (int)(blockIdx.x / per_kvb);
  const int rem = (int)(blockIdx.x % per_kvb);
  u.sp = rem / BHkv;
  const int bh = rem % BHkv;
  u.z = bh / p.Hkv;
  u.hkv = bh % p.Hkv;
  u.gh = p.gqa / hsplit;
  u.g0 = u.sp * u.gh;
  return u;
}

// Epilogue of one key row r (global row j) of dK (h = 0) or dV (h = 1): D fp32 accumulator columns
// from TMEM at tcol, written in the output dtype, or in fp32 to the slice's partial rows.
template <bool BF16, int D>
__device__ __forceinline__ void store_dkv_row(const BwdArgs& a, const BwdUnit& u, int seq_start,
                                              int h, int r, int j, int L, uint32_t tcol) {
  using Tout = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  const Problem& p = a.p;
  const TensorRef& dst = h ? a.dv : a.dk;
  Tout* rowp = reinterpret_cast<Tout*>(dst.ptr) + row_offset(dst, p, u.z, u.hkv, seq_start, j);
  float* prow = a.dkv_part +
                (((((int64_t)u.z * p.Hkv + u.hkv) * a.nkv + u.kvb) * a.hsplit + u.sp) * 2 + h) *
                    (128 * D) + (int64_t)r * D;
#pragma unroll
  for (int c = 0; c < D / 32; ++c) {
    uint32_t o[32];
    tmem_ld32(tcol + c * 32, o);
    tmem_ld_wait(o);
    if (j < L) {
      if (a.hsplit > 1) {
        float4* d4 = reinterpret_cast<float4*>(prow + c * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          d4[i] = make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]),
                              __uint_as_float(o[4 * i + 2]), __uint_as_float(o[4 * i + 3]));
      } else if (c * 32 < p.D) {  // p.D < D when a D = 32 problem runs the D = 64 kernel
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          w[i] = pack2<BF16>(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1]));
        uint4* d4 = reinterpret_cast<uint4*>(rowp + c * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          d4[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
      }
    }
  }
}

// dn / db partials of the unit's key block and q-head slice: zero for a block past the sequence
// end (nothing to add), NaN for a block that skipped or abandoned its work after a device timeout
// (its dK / dV rows are NaN as well; with q-head slices the dq conversion, which reads the status
// word, writes them). Called by every thread of the block.
template <bool BF16>
__device__ __forceinline__ void bwd_block_partials(const BwdArgs& a, const BwdUnit& u,
                                                   int seq_start, int n0, int L, bool failed) {
  const Problem& p = a.p;
  const float v = failed ? nan_f32() : 0.f;
  for (int i = threadIdx.x; i < a.ppk * u.gh; i += blockDim.x) {
    const int g = u.g0 + i / a.ppk, sub = i % a.ppk;
    const int64_t pi = bwd_partial_index(a, u.z, u.hkv * p.gqa + g, u.kvb, 0) + sub;
    a.dn_part[pi] = v;
    a.db_part[pi] = v;
  }
  if (failed && a.hsplit == 1) {
    const int n1 = min(n0 + 128, L);
    nan_fill_rows16<BF16>(a.dk, p, u.z, u.hkv, seq_start, n0, n1, nullptr);
    nan_fill_rows16<BF16>(a.dv, p, u.z, u.hkv, seq_start, n0, n1, nullptr);
  }
}

enum BwdBar : int {
  BB_KV = 0,
  BB_QF = 1,    // 3 stages: Q/dO tile + lse/delta landed
  BB_QE = 4,    // 3 stages: tile's MMAs retired
  BB_SF = 7,    // S^T and dP^T of the tile in TMEM
  BB_SC = 8,    // both halves pulled S^T / dP^T into registers (TMEM columns free)
  BB_SM = 9,    // P^T / dS^T of both halves written (TMEM + smem), and the previous
                //   tile's dQ read out of TMEM by the drain warps (256 + 128 arrivals)
  BB_BF = 10,   // dV / dK MMAs of the tile retired
  BB_DQF = 11,  // dQ in TMEM
  BB_KVD = 12,  // all MMAs retired: dK, dV final
  BB_END = 13,
  BB_COUNT = 14
};

// One W-query chunk of one key row: recompute P from S, dS = P (dP - delta) n b scale / (1+u),
// accumulate dn/db, and pack P and dS to 16 bits. The fp32 elementwise work runs on element
// pairs with the packed f32x2 FMA/ADD/MUL instructions (half the issue slots); lrow / drow hold
// -lse and -delta so both subtractions fold into packed FMA / ADD. MASKED adds the causal /
// bounds test (valid iff the row is in range and qmin <= q < L), applied to the exponent: an
// invalid element gets t = -inf and ex2.approx returns +0 for it. NRCP takes 1/(1+u) from
// Newton steps on the FMA pipe instead of the special-function unit.
template <int W, bool BF16, bool MASKED, bool NRCP>
__device__ __forceinline__ void bwd_chunk(const uint32_t (&sx)[W], const uint32_t (&dp)[W],
                                          const float* lrow, const float* drow, float n, float cb,
                                          float nbs, int q0, int qmin, int L, bool row_ok,
                                          float2 (&dn_acc)[2], float2 (&db_acc)[2],
                                          uint32_t (&pk)[W / 2], uint32_t (&dk)[W / 2]) {
  const float2 n2 = make_float2(n, n), nbs2 = make_float2(nbs, nbs);
  float slv[W], rv[W];
  float2 prv[W / 2];
  // Three passes over the chunk: sign * log2(1 + u) and 1/(1 + u) per element, then the
  // exponentials, then the rest. The operations and results are those of one pass per element
  // pair; the phased order measured 1.5% faster in the config-2 backward.
#pragma unroll
  for (int e = 0; e < W; e += 2) {
    const float x0 = __uint_as_float(sx[e]), x1 = __uint_as_float(sx[e + 1]);
    const float a0 = fmaf(fabsf(x0), cb, 1.0f), a1 = fmaf(fabsf(x1), cb, 1.0f);
    slv[e] = copy_sign_bit(lg2_approx(a0), x0);
    slv[e + 1] = copy_sign_bit(lg2_approx(a1), x1);
    const float2 r =
        NRCP ? rcp2_newton(make_float2(a0, a1)) : make_float2(rcp_approx(a0), rcp_approx(a1));
    rv[e] = r.x;
    rv[e + 1] = r.y;
  }
#pragma unroll
  for (int e4 = 0; e4 < W / 4; ++e4) {
    const float4 nl = *reinterpret_cast<const float4*>(lrow + e4 * 4);
#pragma unroll
    for (int pi = 0; pi < 2; ++pi) {
      const int e = e4 * 4 + pi * 2;
      const float2 nlse = pi ? make_float2(nl.z, nl.w) : make_float2(nl.x, nl.y);
      float2 t = __ffma2_rn(n2, make_float2(slv[e], slv[e + 1]), nlse);
      if (MASKED) {
        const int q = q0 + e;
        t.x = (row_ok && q >= qmin && q < L) ? t.x : -INFINITY;
        t.y = (row_ok && q + 1 >= qmin && q + 1 < L) ? t.y : -INFINITY;
      }
      prv[e / 2] = make_float2(ex2_approx(t.x), ex2_approx(t.y));
    }
  }
#pragma unroll
  for (int e4 = 0; e4 < W / 4; ++e4) {
    const float4 nd = *reinterpret_cast<const float4*>(drow + e4 * 4);
#pragma unroll
    for (int pi = 0; pi < 2; ++pi) {
      const int e = e4 * 4 + pi * 2;
      const float x0 = __uint_as_float(sx[e]), x1 = __uint_as_float(sx[e + 1]);
      const float2 sl = make_float2(slv[e], slv[e + 1]);
      const float2 pr = prv[e / 2];
      const float2 ndel = pi ? make_float2(nd.z, nd.w) : make_float2(nd.x, nd.y);
      const float2 dss = __fmul2_rn(pr, __fadd2_rn(make_float2(__uint_as_float(dp[e]),
                                                               __uint_as_float(dp[e + 1])),
                                                   ndel));
      const float2 w = __fmul2_rn(dss, make_float2(rv[e], rv[e + 1]));
      dn_acc[pi] = __ffma2_rn(dss, sl, dn_acc[pi]);
      db_acc[pi] = __ffma2_rn(w, make_float2(x0, x1), db_acc[pi]);
      const float2 dsv = __fmul2_rn(w, nbs2);
      pk[e4 * 2 + pi] = pack2<BF16>(pr.x, pr.y);
      dk[e4 * 2 + pi] = pack2<BF16>(dsv.x, dsv.y);
    }
  }
}

template <bool BF16, bool DET>
__global__ void __launch_bounds__(512, 1)
    bwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ,
                     const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV,
                     const __grid_constant__ CUtensorMap tmDO,
                     const __grid_constant__ CUtensorMap tmDQ, const BwdArgs a) {
  using C = BwdCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto bar = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + 8 * BB_COUNT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* lse_s = reinterpret_cast<float*>(smem + C::OFF_LSE);
  float* del_s = reinterpret_cast<float*>(smem + C::OFF_DEL);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Problem& p = a.p;
  const BwdUnit unit = bwd_unit(p, a.hsplit);  // key block 0 (most query tiles) first
  const int kvb = unit.kvb, z = unit.z, hkv = unit.hkv;
  const int hq0 = hkv * p.gqa + unit.g0;  // first q-head of this CTA's slice
  int seq_start, L;
  seq_bounds(p, z, seq_start, L);
  const int n0 = kvb * C::BN;
  // Block-uniform exit: a block past the sequence end has nothing to add. (A device timeout
  // recorded by an earlier launch is checked during the set-up below: the block then skips its
  // work and writes NaN.)
  if (n0 >= L) {
    bwd_block_partials<BF16>(a, unit, seq_start, n0, L, false);
    return;
  }
  const int q_start = p.causal ? n0 : 0;
  const int T_h = (L - q_start + C::BT - 1) / C::BT;  // query tiles per q-head
  const int T = T_h * unit.gh;
  const int zc = p.cu_seqlens ? 0 : z;
  // Deterministic dq writes dn/db partials per query tile: start this slice's at zero (the
  // __syncthreads below orders these writes before the P/dS warps' own).
  if (DET) bwd_block_partials<BF16>(a, unit, seq_start, n0, L, false);

  volatile int* skip_flag = abort_flag + 1;
  if (threadIdx.x == 0) {
    // The device status word, read while the barriers are set up (one load per block; its
    // latency overlaps the set-up instead of preceding it).
    const unsigned int st0 = *reinterpret_cast<const volatile unsigned int*>(a.status);
    mbar_init(bar(BB_KV), 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar(BB_QF + s), 33);
      mbar_init(bar(BB_QE + s), 1);
    }
    mbar_init(bar(BB_SF), 1);
    mbar_init(bar(BB_SC), 256);
    mbar_init(bar(BB_SM), 384);
    mbar_init(bar(BB_BF), 1);
    mbar_init(bar(BB_DQF), 1);
    mbar_init(bar(BB_KVD), 1);
    mbar_init(bar(BB_END), 1);
    *abort_flag = st0 != 0 ? 1 : 0;  // an earlier timeout: skip the work, outputs NaN
    *skip_flag = st0 != 0 ? 1 : 0;
    fence_mbar_init();
  }
  if (warp == C::WARP_PRODUCER) {
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (*skip_flag) {
    // an earlier launch recorded a device timeout: no work (the epilogue below writes NaN)
  } else if (warp >= 12) {
   regs_dec<C::REGS_CTRL>();
   if (warp == C::WARP_PRODUCER) {
    // ---------------------------------------------------------------- producer (whole warp)
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      prefetch_tmap(&tmDO);
      mbar_expect_tx(bar(BB_KV), 2 * C::KV_BYTES);
      tma_load_4d(sbase + C::OFF_K, &tmK, bar(BB_KV), 0, seq_start + n0, hkv, zc);
      tma_load_4d(sbase + C::OFF_V, &tmV, bar(BB_KV), 0, seq_start + n0, hkv, zc);
    }
    int last_tile = -1;
    // lse / delta of the next tile are fetched into registers one tile ahead, so their global
    // latency overlaps the wait for a free stage.
    float pl[C::BT / 32], pd[C::BT / 32];
    auto fetch_stats = [&](int t) {
      int g, tt;
      tile_coords(t, T_h, unit.gh, DET, g, tt);
      const int hq = hq0 + g;
      const int m0 = q_start + tt * C::BT;
#pragma unroll
      for (int k = 0; k < C::BT / 32; ++k) {
        const int row = m0 + lane + 32 * k;
        pl[k] = 0.f;
        pd[k] = 0.f;
        if (row < L) {
          const int64_t o = stat_offset(p, z, hq, seq_start, row);
          pl[k] = __ldg(a.lse + o);
          pd[k] = __ldg(a.delta + o);
        }
      }
    };
    // delta comes from the preprocess kernel, which may still be running (programmatic launch);
    // the K / V loads above do not depend on it.
    griddep_wait();
    fetch_stats(0);
    for (int t = 0; t < T; ++t) {
      const int st = t % C::STAGES, u = t / C::STAGES;
      int g, tt;
      tile_coords(t, T_h, unit.gh, DET, g, tt);
      const int hq = hq0 + g;
      const int m0 = q_start + tt * C::BT;
      bool ok = true;
      if (t >= C::STAGES) ok = mbar_wait(bar(BB_QE + st), (u - 1) & 1, a.status);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || *abort_flag) {
        *abort_flag = 1;
        break;
      }
      if (lane == 0) {
        mbar_expect_tx(bar(BB_QF + st), 2 * C::QT_BYTES);
        tma_load_4d(sbase + C::OFF_Q + st * C::QT_BYTES, &tmQ, bar(BB_QF + st), 0,
                    seq_start + m0, hq, zc);
        tma_load_4d(sbase + C::OFF_DO + st * C::QT_BYTES, &tmDO, bar(BB_QF + st), 0,
                    seq_start + m0, hq, zc);
      }
#pragma unroll
      for (int k = 0; k < C::BT / 32; ++k) {
        lse_s[st * C::BT + lane + 32 * k] = -pl[k];  // stored negated for packed FMA / ADD
        del_s[st * C::BT + lane + 32 * k] = -pd[k];
      }
      mbar_arrive(bar(BB_QF + st));
      last_tile = t;
      if (t + 1 < T) fetch_stats(t + 1);
    }
    if (*abort_flag && lane == 0) {  // drain own TMA loads before shared memory is released
      mbar_wait(bar(BB_KV), 0, a.status);
      for (int t = max(0, last_tile - C::STAGES + 1); t <= last_tile; ++t)
        mbar_wait(bar(BB_QF + t % C::STAGES), (t / C::STAGES) & 1, a.status);
    }
   } else if (warp == C::WARP_MMA) {
    // ---------------------------------------------------------------- MMA issuer
    // The whole warp runs the schedule and its waits; one elected lane issues each batch of
    // tcgen05.mma / commit. The warp shares its SM sub-partition with three busy warps, so the
    // issue path is kept short: descriptors are low words (constant high word) advanced by
    // immediates, computed once per CTA or per tile.
    {
      const bool leader = elect_one() != 0;
      constexpr uint32_t id_s = idesc_f16(BF16, false, false, 128, 128);  // S^T, dP^T
      constexpr uint32_t id_g = idesc_f16(BF16, false, true, 128, 64);   // dV, dK
      constexpr uint32_t id_q = idesc_f16(BF16, true, true, 128, 64);    // dQ
      const uint32_t sK = sbase + C::OFF_K, sV = sbase + C::OFF_V;
      const uint32_t dK_s = sdesc_lo(sK, 16), dV_s = sdesc_lo(sV, 16);  // K-major K, V
      const uint32_t dK_q = sdesc_lo(sK, 8192);                         // MN-major K (dQ's B)
      auto wait_all = [&](uint32_t b, uint32_t par) {
        return __all_sync(0xffffffffu, mbar_wait(b, par, a.status));
      };
      // 16-byte units: a K step of 16 elements is 32 B within a swizzled row (2 units); a K step
      // of 16 rows of an MN-major operand is 2048 B (128 units).
      // S^T = K Q^T and dP^T = V dO^T for the whole 128-query tile: N = 128 runs at the full
      // tensor rate, while an M = 128, K = 16 MMA costs about as long for any N up to 128.
      auto issue_sdp = [&](int t) {
        if (!leader) return;
        const int st = t % C::STAGES;
        const uint32_t q_lo = sdesc_lo(sbase + C::OFF_Q + st * C::QT_BYTES, 16);
        const uint32_t o_lo = sdesc_lo(sbase + C::OFF_DO + st * C::QT_BYTES, 16);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_ss_lo(tmem + C::COL_S, dK_s + 2 * kk, q_lo + 2 * kk, id_s, kk > 0);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_ss_lo(tmem + C::COL_DP, dV_s + 2 * kk, o_lo + 2 * kk, id_s, kk > 0);
        mma_commit(bar(BB_SF));
      };
      bool ok = wait_all(bar(BB_KV), 0) && wait_all(bar(BB_QF), 0);
      if (ok) {
        tc_fence_after();
        issue_sdp(0);
        __syncwarp();
      }
      for (int t = 0; ok && t < T; ++t) {
        const int st = t % C::STAGES, dsb = t & 1;
        // The next tile's S^T / dP^T go first, as soon as both halves have pulled this tile's
        // into registers (half-way through their arithmetic): the grads below read only P^T
        // (own TMEM columns) and dS^T (shared memory).
        if (t + 1 < T) {
          ok = wait_all(bar(BB_QF + (t + 1) % C::STAGES), ((t + 1) / C::STAGES) & 1);
          if (ok) ok = wait_all(bar(BB_SC), t & 1);
          if (!ok || *abort_flag) break;
          tc_fence_after();
          issue_sdp(t + 1);
          __syncwarp();
        }
        // Both halves' P^T / dS^T written, and dQ(t-1) read out of TMEM by the drain warps
        // (they arrive on the same barrier): the grads and this tile's dQ can go.
        const uint32_t q_mn = sdesc_lo(sbase + C::OFF_Q + st * C::QT_BYTES, 8192);
        const uint32_t o_mn = sdesc_lo(sbase + C::OFF_DO + st * C::QT_BYTES, 8192);
        const uint32_t ds_k = sdesc_lo(sbase + C::OFF_DS + dsb * C::DS_BYTES, 16);
        const uint32_t ds_mn = sdesc_lo(sbase + C::OFF_DS + dsb * C::DS_BYTES, C::DS_SLAB);
        ok = wait_all(bar(BB_SM), t & 1);
        if (!ok || *abort_flag) break;
        tc_fence_after();
        if (leader) {
          // dV += P^T dO_h (P^T from TMEM); dK += dS^T Q_h (dS^T from the shared slab the dQ
          // MMA also reads: [128 keys x 64 queries] per half, K-major here, MN-major for dQ).
          // Half 0 before half 1, always: dK / dV are bit-reproducible.
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t acc0 = (t > 0 || h > 0) ? 1u : 0u;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_ts_lo(tmem + C::COL_DV, tmem + C::COL_PT + h * 32 + kk * 8,
                        o_mn + (C::HALF_BYTES >> 4) * h + 128 * kk, id_g, kk > 0 ? 1u : acc0);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_ss_lo(tmem + C::COL_DK, ds_k + (C::DS_SLAB >> 4) * h + 2 * kk,
                        q_mn + (C::HALF_BYTES >> 4) * h + 128 * kk, id_g, kk > 0 ? 1u : acc0);
          }
          mma_commit(bar(BB_BF));
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ss_lo(tmem + C::COL_DQ, ds_mn + 128 * kk, dK_q + 128 * kk, id_q, kk > 0);
          mma_commit(bar(BB_DQF));
          mma_commit(bar(BB_QE + st));
        }
        __syncwarp();
      }
      if (!ok) *abort_flag = 1;
      if (leader) {
        mma_commit(bar(BB_KVD));
        mma_commit(bar(BB_END));
      }
      __syncwarp();
      mbar_wait(bar(BB_END), 0, a.status);
    }
   }
  } else if (warp < 8) {
    // ---------------------------------------------------------------- P / dS warp-groups
    regs_inc<C::REGS_PDS>();
    const int h = warp >> 2;  // 0: warps 0..3, 1: warps 4..7
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // key row within the block
    const int j = n0 + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tS = tmem + lane_off + C::COL_S + 64 * h;
    const uint32_t tP = tmem + lane_off + C::COL_DP + 64 * h;
    const uint32_t tPT = tmem + lane_off + C::COL_PT + h * 32;
    const float bval = __ldg(p.b_ptr);
    const float cb = bval * p.scale;
    float n = 0.f, nbs = 0.f;
    float2 dn_acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    float2 db_acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    // Tile t may start once its Q / dO / lse / delta have landed (QF) and its S^T / dP^T are in
    // TMEM (SF). SF also implies that the dQ MMA of tile t - 2, which read this tile's dS^T
    // buffer, has retired: its commit follows that MMA in the issuer's order.
    auto wait_tile = [&](int t) {
      bool w = mbar_wait(bar(BB_QF + t % C::STAGES), (t / C::STAGES) & 1, a.status);
      if (w) w = mbar_wait(bar(BB_SF), t & 1, a.status);
      w = __all_sync(0xffffffffu, w);
      return w && !*abort_flag;
    };
    uint32_t sx[16], dp[16];
    bool ok = wait_tile(0);
    if (ok) {  // chunk 0 of tile 0; later tiles' chunk 0 is fetched after the previous tile's SM
      tc_fence_after();
      tmem_ld16(tS, sx);
      tmem_ld16(tP, dp);
    }
    // ring stage, q-head within the slice, query tile within the head (tile_coords order)
    int st = 0, g = 0, tt = DET ? T_h - 1 : 0;
    for (int t = 0; ok && t < T; ++t) {
      const int dsb = t & 1;
      const int hq = hq0 + g;
      if (DET || tt == 0) {  // a new q-head (the deterministic order changes head every tile)
        n = load_n(p, hq);
        nbs = n * bval * p.scale;
      }
      const int mh = q_start + tt * C::BT + h * 64;  // first query row of this half
      const bool full = (!p.causal || mh >= n0 + C::BN - 1) && (mh + 64 <= L) && (n0 + C::BN <= L);
      const float* lrow = lse_s + st * C::BT + h * 64;
      const float* drow = del_s + st * C::BT + h * 64;
      uint8_t* dsrow = smem + C::OFF_DS + dsb * C::DS_BYTES + h * C::DS_SLAB + r * 128;
      const int qmin = p.causal ? j : 0;
      tmem_ld_wait_only();
      tmem_pin_n(sx);
      tmem_pin_n(dp);
      // 4 chunks of 16 queries (16-wide chunks leave the compiler registers to overlap more
      // element pairs than 32-wide ones). Chunk c + 1's S / dP loads are issued after chunk c
      // has been computed and are in flight while chunk c's P^T and dS^T are stored. After
      // chunk 3 the tile's SM arrival goes first (the grads MMAs wait on it), then the next
      // tile's chunk 0 is loaded.
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[8], dk[8];
        // A chunk masked for every row of this warp (the lower part of a diagonal tile, or past
        // the sequence end) has P = dS = 0: its transform is skipped.
        const bool dead = !full && ((p.causal && mh + c * 16 + 15 < n0 + quad * 32) ||
                                    mh + c * 16 >= L || n0 + quad * 32 >= L);
        if (dead) {
#pragma unroll
          for (int i = 0; i < 8; ++i) pk[i] = dk[i] = 0u;
        } else if (full)
          bwd_chunk<16, BF16, false, true>(sx, dp, lrow + c * 16, drow + c * 16, n, cb, nbs,
                                           mh + c * 16, qmin, L, j < L, dn_acc, db_acc, pk, dk);
        else
          bwd_chunk<16, BF16, true, true>(sx, dp, lrow + c * 16, drow + c * 16, n, cb, nbs,
                                          mh + c * 16, qmin, L, j < L, dn_acc, db_acc, pk, dk);
        if (c < 3) {
          tmem_ld16(tS + 16 * (c + 1), sx);
          tmem_ld16(tP + 16 * (c + 1), dp);
          if (c == 0) {
            // dV(t-1) must have read this half's P^T columns before they are rewritten.
            bool okb = t == 0 || mbar_wait(bar(BB_BF), (t - 1) & 1, a.status);
            if (!__all_sync(0xffffffffu, okb)) *abort_flag = 1;
            tc_fence_after();
          }
        }
        tmem_st8(tPT + c * 8, pk);
        // dS^T row r of this half's slab: 16-byte chunks, 128-byte swizzle (chunk ^ (row & 7))
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
          const int chunk = c * 2 + q2;
          *reinterpret_cast<uint4*>(dsrow + ((chunk ^ (r & 7)) << 4)) =
              make_uint4(dk[q2 * 4], dk[q2 * 4 + 1], dk[q2 * 4 + 2], dk[q2 * 4 + 3]);
        }
        if (c < 3) {
          tmem_ld_wait_only();
          tmem_pin_n(sx);
          tmem_pin_n(dp);
          if (c == 2) {
            tc_fence_before();
            mbar_arrive(bar(BB_SC));  // this tile's S^T / dP^T columns may now be overwritten
          }
        }
      }
      tmem_st_wait();
      tc_fence_before();
      fence_proxy_async_smem();
      mbar_arrive(bar(BB_SM));
      if (t + 1 < T) {
        if (wait_tile(t + 1)) {
          tc_fence_after();
          tmem_ld16(tS, sx);
          tmem_ld16(tP, dp);
        } else {
          ok = false;
        }
      }
      // End of q-head g (deterministic order, where heads alternate: every tile): each warp
      // writes its dn/db partial.
      if (DET || tt == T_h - 1) {
        float x1 = (dn_acc[0].x + dn_acc[0].y) + (dn_acc[1].x + dn_acc[1].y);
        float x2 = (db_acc[0].x + db_acc[0].y) + (db_acc[1].x + db_acc[1].y);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          x1 += __shfl_xor_sync(0xffffffffu, x1, o);
          x2 += __shfl_xor_sync(0xffffffffu, x2, o);
        }
        if (lane == 0) {
          const int64_t pi = bwd_partial_index(a, z, hq, kvb, DET ? tt : 0) + 4 * h + quad;
          a.dn_part[pi] = x1 * kLn2;
          a.db_part[pi] = x2 * n * p.scale;
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) dn_acc[i] = db_acc[i] = make_float2(0.f, 0.f);
      }
      st = st + 1 == C::STAGES ? 0 : st + 1;
      if (DET) {
        if (++g == unit.gh) {
          g = 0;
          --tt;
        }
      } else if (++tt == T_h) {
        tt = 0;
        ++g;
      }
    }
    if (!ok) *abort_flag = 1;
    // ---- epilogue: half 0 stores dK, half 1 stores dV (one key row per thread)
    bool okd = ok && mbar_wait(bar(BB_KVD), 0, a.status);
    okd = __all_sync(0xffffffffu, okd);
    if (okd && !*abort_flag) {
      tc_fence_after();
      store_dkv_row<BF16, C::D>(a, unit, seq_start, h, r, j, L,
                                tmem + lane_off + (h ? C::COL_DV : C::COL_DK));
    }
  } else {
    // ---------------------------------------------------------------- dQ drain (warps 8..11)
    regs_dec<C::REGS_DQ>();
    // Each warp drains its own 32 query rows in two 32-column halves: TMEM -> 4 KB of staging in
    // the 128-byte swizzle -> one 2-D TMA reduce-add (fp32) per half into the dQ accumulator.
    const int quad = warp & 3;
    uint8_t* stage = smem + C::OFF_DQS + quad * C::DQS_WARP;
    const uint32_t stage_s = sbase + C::OFF_DQS + quad * C::DQS_WARP;
    const uint32_t tQ = tmem + ((uint32_t)(quad * 32) << 16) + C::COL_DQ;
    // The drain's arrival for tile t's barrier SM(t) says dQ(t-1) has left TMEM; tile 0 has no
    // predecessor.
    mbar_arrive(bar(BB_SM));
    griddep_wait();  // the dQ accumulator is zeroed by the preprocess kernel
    bool ok = true;
    for (int t = 0; t < T; ++t) {
      ok = mbar_wait(bar(BB_DQF), t & 1, a.status);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || *abort_flag) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t v0[32], v1[32];
      tmem_ld32(tQ, v0);
      tmem_ld32(tQ + 32, v1);
      tmem_ld_wait_only();
      tmem_pin(v0);
      tmem_pin(v1);
      tc_fence_before();
      mbar_arrive(bar(BB_SM));  // dQ(t) is out of TMEM: counts toward SM(t + 1)
      int g, tt;
      tile_coords(t, T_h, unit.gh, DET, g, tt);
      const int hq = hq0 + g;
      const int m0 = q_start + tt * C::BT + quad * 32;
      const int row0 = p.cu_seqlens ? (int)((int64_t)hq * a.dq_rows + seq_start + m0)
                                    : (int)(((int64_t)z * p.Hq + hq) * a.dq_rows + m0);
      // Deterministic dq: these 32 rows take their turn after key blocks 0 .. kvb - 1.
      int* sem = DET ? a.dq_sem + (((int64_t)z * p.Hq + hq) * a.ntq + q_start / C::BT + tt) * 4 +
                             quad
                       : nullptr;
      if (DET) {
        bool okw = true;
        if (lane == 0) okw = sem_wait_eq(sem, kvb, a.status);
        if (!__shfl_sync(0xffffffffu, okw ? 1 : 0, 0)) {
          ok = false;
          break;
        }
      }
#pragma unroll
      for (int hc = 0; hc < 2; ++hc) {
        const uint32_t(&v)[32] = hc ? v1 : v0;
        if (lane == 0) bulk_wait_read0();  // the staging buffer is free again
        __syncwarp();
        uint8_t* srow = stage + lane * 128;
#pragma unroll
        for (int i = 0; i < 8; ++i)
          *reinterpret_cast<uint4*>(srow + ((i ^ (lane & 7)) << 4)) =
              make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_2d(&tmDQ, stage_s, hc * 32, row0);
          bulk_commit();
        }
      }
      if (DET && lane == 0) {  // both adds performed, then the next key block's turn
        bulk_wait0();
        sem_release_next(sem);
      }
    }
    if (!ok) *abort_flag = 1;
    // The staging buffers must outlive the TMA engine's reads of them; the reduce-adds' global
    // writes need no wait here (they are performed before the grid completes).
    if (lane == 0) bulk_wait_read0();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == C::WARP_PRODUCER) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  // A wait of this CTA expired: its dK / dV rows and dn / db partials are NaN, never partial
  // results (dq is filled with NaN by the conversion kernel, which reads the status word).
  if (*abort_flag) bwd_block_partials<BF16>(a, unit, seq_start, n0, L, true);
}

// Backward preprocess for the tensor-core path, one pass: delta = rowsum(O * dO) in fp32
// (ssa_triton_kernel.py:267-298) and zeroing of the fp32 dQ accumulator rows (padding rows
// included) and, for deterministic dq, of the turn counters (sem_per_zh per sequence x q-head).
// D/8 threads per row (D: the tensors' head dim), 16-byte loads; 2048/D rows per 256-thread block.
// The accumulator rows are DACC floats wide (the kernel's head dim: 64 when D = 32 runs the D = 64
// kernel).
template <typename T, int D, int DACC>
__global__ void __launch_bounds__(256) bwd_preprocess_sm100_kernel(Problem p, TensorRef o,
                                                                   TensorRef dout, float* delta,
                                                                   float* dq_accum,
                                                                   int64_t dq_rows, int* sem,
                                                                   int sem_per_zh, T* dom,
                                                                   const float* lse,
                                                                   float* lse_shifted) {
  griddep_launch_dependents();  // the backward's setup may overlap this pass
  // Launched programmatically behind the forward (which wrote `o`): nothing global is touched
  // before that grid has completed.
  griddep_wait();
  if (sem && blockIdx.x == 0) {
    const int nz = p.cu_seqlens ? p.B : 1;  // packed: grid row = q-head, every document
    for (int zz = 0; zz < nz; ++zz) {
      const int64_t base =
          (int64_t)(p.cu_seqlens ? zz * p.Hq + (int)blockIdx.y : (int)blockIdx.y) * sem_per_zh;
      for (int i = threadIdx.x; i < sem_per_zh; i += blockDim.x) sem[base + i] = 0;
    }
  }
  constexpr int TPR = D / 8, RPB = 256 / TPR;
  constexpr int ZPT = DACC / TPR;  // accumulator floats zeroed per thread
  const int sub = threadIdx.x % TPR;
  const int rr = blockIdx.x * RPB + threadIdx.x / TPR;  // row within the head's accumulator
  const bool in_acc = rr < dq_rows;  // (no early return: every lane takes part in the shuffles)
  int z, hq, row, L;
  if (p.cu_seqlens) {  // accumulator rows are packed tokens; delta is [Hq][T]
    z = 0;
    hq = blockIdx.y;
    row = rr;
    L = p.N;
  } else {
    z = blockIdx.y / p.Hq;
    hq = blockIdx.y % p.Hq;
    row = rr;
    L = p.N;
  }
  if (in_acc) {
    float4* zdst = reinterpret_cast<float4*>(
        dq_accum + ((int64_t)blockIdx.y * dq_rows + rr) * DACC + sub * ZPT);
#pragma unroll
    for (int i = 0; i < ZPT / 4; ++i) zdst[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float acc = 0.f;
  const bool valid = in_acc && row < L;
  if (valid) {
    const int64_t oo = (p.cu_seqlens ? 0 : (int64_t)z * o.sB) + (int64_t)hq * o.sH + (int64_t)row * o.sN;
    const int64_t od = (p.cu_seqlens ? 0 : (int64_t)z * dout.sB) + (int64_t)hq * dout.sH +
                       (int64_t)row * dout.sN;
    const uint4 a = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(o.ptr) + oo + sub * 8);
    const uint4 b = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(dout.ptr) + od + sub * 8);
    const T* ae = reinterpret_cast<const T*>(&a);
    const T* be = reinterpret_cast<const T*>(&b);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc = fmaf(to_f32<T>(ae[i]), to_f32<T>(be[i]), acc);
    if (dom) {
      // Output dropout: o is the dropped output and dout the gradient of the dropped output, so
      // the sum above is the undropped rowsum(O * dO) with dO = dout * keep / (1 - p). The main
      // kernel reads dout * keep (dom, exact) with delta * (1 - p) and lse lowered by
      // log2(1 / (1 - p)) (lse_shifted, written below), which gives the gradients of dO.
      const DropoutKey dk = dropout_key(p);
      const uint64_t e0 = dropout_index(p, z, hq, 0, row) + (uint64_t)(sub * 8);
      const uint32_t keep = dropout_keep4(dk, e0) | (dropout_keep4(dk, e0 + 4) << 4);
      uint4 m = b;
      uint16_t* me = reinterpret_cast<uint16_t*>(&m);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (!((keep >> i) & 1u)) me[i] = 0;
      *reinterpret_cast<uint4*>(dom + e0) = m;
      acc *= p.drop_delta_scale;
    }
  }
#pragma unroll
  for (int o2 = 1; o2 < TPR; o2 <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o2);
  if (valid && sub == 0) {
    const int64_t so = p.cu_seqlens ? (int64_t)hq * p.N + row : ((int64_t)z * p.Hq + hq) * p.N + row;
    delta[so] = acc;
    if (dom) lse_shifted[so] = __ldg(lse + so) - p.drop_lse_shift;
  }
}

// dq (q's dtype, caller strides) = dq_accum (fp32) for the valid rows. The first grid rows
// (r.rows of them) reduce dn / db instead (dndb_reduce_block, one block per dn head plus one for
// db): dispatched first, that latency-bound work runs under the bandwidth-bound conversion
// rather than as a launch of its own or as a tail after it.
struct DndbArgs {
  const float* dn_part;
  const float* db_part;
  int P;     // partials per (sequence, q-head)
  int rows;  // leading grid rows that reduce
  float* dn;
  float* db;
  const unsigned int* status;  // device status word: non-zero after an expired bounded wait
  // dK / dV from q-head slice partials (hsplit > 1): grid rows after the dq rows, one per
  // (sequence, kv-head, dK or dV); fp32 [B][Hkv][nkv][hsplit][2][128][D] summed in slice order.
  const float* dkv_part;
  int hsplit, nkv;
  TensorRef dk, dv;
};

// D: the tensors' head dim (the columns written); DACC: the accumulator's row width.
template <typename T, int D, int DACC>
__global__ void __launch_bounds__(256) dq_convert_kernel(Problem p, const float* dq_accum,
                                                         int64_t dq_rows, TensorRef dq,
                                                         DndbArgs r) {
  griddep_wait();  // launched programmatically behind the backward kernel
  griddep_launch_dependents();  // the next forward may launch; it waits for this grid first
  // After a device timeout (this backward's or an earlier launch's) dq, dk, dv, dn and db are NaN.
  if ((int)blockIdx.y < r.rows) {
    const bool failed = block_status_failed(r.status);
    __shared__ double red[256];
    const int nred = (p.n_per_head ? p.Hq : 1) + 1;
    const int h = (int)blockIdx.y * (int)gridDim.x + (int)blockIdx.x;
    if (h < nred && failed) {
      if (threadIdx.x == 0) (h < nred - 1 ? r.dn[h] : r.db[0]) = nan_f32();
    } else if (h < nred) {  // uniform per block
      dndb_reduce_block<256>(h, r.dn_part, r.db_part, p.B, p.Hq, r.P, p.n_per_head, r.dn, r.db,
                             red);
    }
    return;
  }
  constexpr int TPR = D / 8, RPB = 256 / TPR;
  const int zh = (int)blockIdx.y - r.rows;
  if (zh >= p.B * p.Hq) {  // dK / dV rows: sum the q-head slices' partials in order
    const bool failed = block_status_failed(r.status);
    const int u = zh - p.B * p.Hq;
    const int z = u / (2 * p.Hkv), hkv = (u / 2) % p.Hkv, h = u & 1;
    int seq_start, L;
    seq_bounds(p, z, seq_start, L);
    const int row = blockIdx.x * RPB + threadIdx.x / TPR;
    const int d0 = (threadIdx.x % TPR) * 8;
    if (row >= L) return;
    const TensorRef& dst = h ? r.dv : r.dk;
    T* d = reinterpret_cast<T*>(dst.ptr) + row_offset(dst, p, z, hkv, seq_start, row) + d0;
    const uint32_t nn = std::is_same<T, __nv_bfloat16>::value ? kNaNBf16x2 : kNaNF16x2;
    if (failed) {
      *reinterpret_cast<uint4*>(d) = make_uint4(nn, nn, nn, nn);
      return;
    }
    const int kvb = row >> 7;
    const float* src = r.dkv_part +
                       ((((int64_t)z * p.Hkv + hkv) * r.nkv + kvb) * r.hsplit * 2 + h) * (128 * DACC) +
                       (int64_t)(row & 127) * DACC + d0;
    float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
    for (int sp = 0; sp < r.hsplit; ++sp) {
      const float4* s4 = reinterpret_cast<const float4*>(src + (int64_t)sp * 2 * 128 * DACC);
      const float4 b0 = s4[0], b1 = s4[1];
      a0 = make_float4(a0.x + b0.x, a0.y + b0.y, a0.z + b0.z, a0.w + b0.w);
      a1 = make_float4(a1.x + b1.x, a1.y + b1.y, a1.z + b1.z, a1.w + b1.w);
    }
    constexpr bool kBf = std::is_same<T, __nv_bfloat16>::value;
    *reinterpret_cast<uint4*>(d) =
        make_uint4(pack2<kBf>(a0.x, a0.y), pack2<kBf>(a0.z, a0.w), pack2<kBf>(a1.x, a1.y),
                   pack2<kBf>(a1.z, a1.w));
    return;
  }
  const int z = zh / p.Hq, hq = zh % p.Hq;
  int seq_start, L;
  seq_bounds(p, z, seq_start, L);
  const int row = blockIdx.x * RPB + threadIdx.x / TPR;
  const int d0 = (threadIdx.x % TPR) * 8;
  const bool valid = row < L;
  float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
  if (valid) {
    const int64_t src_row = p.cu_seqlens ? (int64_t)hq * dq_rows + seq_start + row
                                         : ((int64_t)z * p.Hq + hq) * dq_rows + row;
    const float4* s = reinterpret_cast<const float4*>(dq_accum + src_row * DACC + d0);
    a0 = s[0];
    a1 = s[1];
  }
  // The status word, read by one thread after the data loads are in flight, so its latency
  // overlaps theirs.
  __shared__ unsigned int s_fail;
  if (threadIdx.x == 0) s_fail = *reinterpret_cast<const volatile unsigned int*>(r.status);
  __syncthreads();
  const bool failed = s_fail != 0;
  if (!valid) return;
  T* d = reinterpret_cast<T*>(dq.ptr) + row_offset(dq, p, z, hq, seq_start, row) + d0;
  uint4 w;
  if (failed) {
    const uint32_t nn = std::is_same<T, __nv_bfloat16>::value ? kNaNBf16x2 : kNaNF16x2;
    *reinterpret_cast<uint4*>(d) = make_uint4(nn, nn, nn, nn);
    return;
  }
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    w = make_uint4(pack2<true>(a0.x, a0.y), pack2<true>(a0.z, a0.w), pack2<true>(a1.x, a1.y),
                   pack2<true>(a1.z, a1.w));
  } else {
    w = make_uint4(pack2<false>(a0.x, a0.y), pack2<false>(a0.z, a0.w), pack2<false>(a1.x, a1.y),
                   pack2<false>(a1.z, a1.w));
  }
  *reinterpret_cast<uint4*>(d) = w;
}

// dq conversion + dn / db reduction, one launch.
template <typename T, int D, int DACC>
int launch_dq_convert_dndb(const Problem& p, const float* dq_accum, int64_t dq_rows,
                            TensorRef dq, const float* dn_part, const float* db_part, int P,
                            float* dn, float* db, const BwdArgs& a, cudaStream_t st) {
  constexpr int RPB = 256 / (D / 8);
  const int gx = (p.max_seqlen + RPB - 1) / RPB;
  const int nred = (p.n_per_head ? p.Hq : 1) + 1;
  const int extra_rows = (nred + gx - 1) / gx;
  const int dkv_rows = a.hsplit > 1 ? p.B * p.Hkv * 2 : 0;
  dim3 gc((unsigned)gx, (unsigned)(p.B * p.Hq + extra_rows + dkv_rows));
  if (launch_pdl(dq_convert_kernel<T, D, DACC>, gc, dim3(256), 0, st, p, dq_accum, dq_rows, dq,
                 DndbArgs{dn_part, db_part, P, extra_rows, dn, db, device_status_ptr(),
                          a.dkv_part, a.hsplit, a.nkv, a.dk, a.dv}) != cudaSuccess)
    return SSA_ERR_LAUNCH;
  note_launches(1);
  return SSA_OK;
}

// ============================================================================================
// Backward for D = 128. dK and dV alone take 256 TMEM columns here, so the D = 64 layout (two
// S/dP buffers) does not fit. Instead:
//   - query tiles are 64 rows; tile t belongs to P/dS warpgroup t & 1;
//   - one S^T/dP^T buffer [0,128) is shared: the owning group pulls its 64 + 64 values per key
//     row into registers and releases it (BB2_SL) before computing, so the next tile's S^T/dP^T
//     MMAs overlap the current tile's arithmetic;
//   - dQ^T = K^T dS^T (M = D = 128 lanes, N = 64 queries) per tile, drained per warp (32 head
//     dims x 64 queries) with 2-D TMA reduce-adds into the fp32 accumulator.
// TMEM: S^T [0,64), dP^T [64,128), dK [128,256), dV [256,384), dQ^T [384,448),
//       P^T of group h (packed 16-bit) [448 + 32h, 480 + 32h).
struct Bwd128Cfg {
  static constexpr int D = 128;
  static constexpr int BN = 128;  // key rows per CTA
  static constexpr int BT = 64;   // query rows per tile
  static constexpr int STAGES = 2;
  static constexpr uint32_t KV_BYTES = BN * D * 2;   // 32 KB: two [128 x 128 B] slabs
  static constexpr uint32_t KV_SLAB = BN * 128;      // 16 KB
  static constexpr uint32_t QT_BYTES = BT * D * 2;   // 16 KB: two [64 x 128 B] slabs
  static constexpr uint32_t QT_SLAB = BT * 128;      // 8 KB
  static constexpr uint32_t DS_BYTES = BN * BT * 2;  // 16 KB: [128 keys x 64 queries]
  static constexpr uint32_t DQS_WARP = BT * 32 * 4;  // 8 KB: [64 queries x 32 head dims] fp32
  static constexpr uint32_t OFF_K = 0;
  static constexpr uint32_t OFF_V = OFF_K + KV_BYTES;
  static constexpr uint32_t OFF_Q = OFF_V + KV_BYTES;
  static constexpr uint32_t OFF_DO = OFF_Q + STAGES * QT_BYTES;
  static constexpr uint32_t OFF_DS = OFF_DO + STAGES * QT_BYTES;  // 2 buffers
  static constexpr uint32_t OFF_DQS = OFF_DS + 2 * DS_BYTES;      // 4 warps x 8 KB
  static constexpr uint32_t OFF_LSE = OFF_DQS + 4 * DQS_WARP;
  static constexpr uint32_t OFF_DEL = OFF_LSE + STAGES * BT * 4;
  static constexpr uint32_t OFF_BAR = OFF_DEL + STAGES * BT * 4;
  static constexpr uint32_t SMEM_BYTES = OFF_BAR + 256 + 1024;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t COL_S = 0, COL_DP = 64, COL_DK = 128, COL_DV = 256, COL_DQ = 384,
                            COL_PT = 448;
  static constexpr int THREADS = 512;
  static constexpr uint32_t REGS_PDS = 184, REGS_DQ = 88, REGS_CTRL = 56;  // 65536 in total
  static constexpr int WARP_PRODUCER = 12, WARP_MMA = 13;
};
static_assert(Bwd128Cfg::SMEM_BYTES <= 232448, "shared memory budget");

// Every barrier is waited on phase after phase by each of its waiters (a parity wait can only
// tell two consecutive phases apart), hence one "S^T/dP^T ready" barrier per P/dS group.
enum Bwd128Bar : int {
  B2_KV = 0,
  B2_QF = 1,    // 2 stages (stage t % 2 == group t & 1)
  B2_QE = 3,    // 2 stages
  B2_SF = 5,    // 2 groups: S^T/dP^T of the group's next tile in the shared buffer
  B2_SL = 7,    // shared buffer read out by its owner (every tile, in order)
  B2_SM = 8,    // 2 groups: P^T / dS^T written
  B2_BF = 10,   // 2 groups: dV/dK MMAs of the group's last tile retired
  B2_DSF = 12,  // 2 dS buffers: dQ^T MMA retired
  B2_DQF = 14,
  B2_DQE = 15,
  B2_KVD = 16,
  B2_END = 17,
  B2_COUNT = 18
};

template <bool BF16, bool DET>
__global__ void __launch_bounds__(512, 1)
    bwd128_sm100_kernel(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV,
                        const __grid_constant__ CUtensorMap tmDO,
                        const __grid_constant__ CUtensorMap tmDQ, const BwdArgs a) {
  using C = Bwd128Cfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto bar = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + 8 * B2_COUNT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* lse_s = reinterpret_cast<float*>(smem + C::OFF_LSE);
  float* del_s = reinterpret_cast<float*>(smem + C::OFF_DEL);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Problem& p = a.p;
  const BwdUnit unit = bwd_unit(p, a.hsplit);
  const int kvb = unit.kvb, z = unit.z, hkv = unit.hkv;
  const int hq0 = hkv * p.gqa + unit.g0;
  int seq_start, L;
  seq_bounds(p, z, seq_start, L);
  const int n0 = kvb * C::BN;
  // Block-uniform exit: a block past the sequence end has nothing to add. (A device timeout
  // recorded by an earlier launch is checked during the set-up below: the block then skips its
  // work and writes NaN.)
  if (n0 >= L) {
    bwd_block_partials<BF16>(a, unit, seq_start, n0, L, false);
    return;
  }
  const int q_start = p.causal ? n0 : 0;
  const int T_h = (L - q_start + C::BT - 1) / C::BT;
  const int T = T_h * unit.gh;
  const int zc = p.cu_seqlens ? 0 : z;
  // A P/dS group may own no tile of some q-head (tiles alternate between the groups): start
  // every partial of this block at zero; the __syncthreads below orders these writes first.
  bwd_block_partials<BF16>(a, unit, seq_start, n0, L, false);

  volatile int* skip_flag = abort_flag + 1;
  if (threadIdx.x == 0) {
    // The device status word, read while the barriers are set up (see the D = 64 kernel).
    const unsigned int st0 = *reinterpret_cast<const volatile unsigned int*>(a.status);
    mbar_init(bar(B2_KV), 1);
    for (int s2 = 0; s2 < C::STAGES; ++s2) {
      mbar_init(bar(B2_QF + s2), 33);
      mbar_init(bar(B2_QE + s2), 1);
    }
    mbar_init(bar(B2_SL), 128);
    for (int s2 = 0; s2 < 2; ++s2) {
      mbar_init(bar(B2_SF + s2), 1);
      mbar_init(bar(B2_SM + s2), 128);
      mbar_init(bar(B2_BF + s2), 1);
      mbar_init(bar(B2_DSF + s2), 1);
    }
    mbar_init(bar(B2_DQF), 1);
    mbar_init(bar(B2_DQE), 128);
    mbar_init(bar(B2_KVD), 1);
    mbar_init(bar(B2_END), 1);
    *abort_flag = st0 != 0 ? 1 : 0;  // an earlier timeout: skip the work, outputs NaN
    *skip_flag = st0 != 0 ? 1 : 0;
    fence_mbar_init();
  }
  if (warp == C::WARP_PRODUCER) {
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (*skip_flag) {
    // an earlier launch recorded a device timeout: no work (the epilogue below writes NaN)
  } else if (warp >= 12) {
    regs_dec<C::REGS_CTRL>();
    if (warp == C::WARP_PRODUCER) {
      // ------------------------------------------------------------ producer (whole warp)
      if (lane == 0) {
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
        prefetch_tmap(&tmDO);
        mbar_expect_tx(bar(B2_KV), 2 * C::KV_BYTES);
#pragma unroll
        for (int sl = 0; sl < 2; ++sl) {
          tma_load_4d(sbase + C::OFF_K + sl * C::KV_SLAB, &tmK, bar(B2_KV), sl * 64,
                      seq_start + n0, hkv, zc);
          tma_load_4d(sbase + C::OFF_V + sl * C::KV_SLAB, &tmV, bar(B2_KV), sl * 64,
                      seq_start + n0, hkv, zc);
        }
      }
      int last_tile = -1;
      float pl[2], pd[2];
      auto fetch_stats = [&](int t) {
        int g, tt;
        tile_coords(t, T_h, unit.gh, DET, g, tt);
        const int hq = hq0 + g;
        const int m0 = q_start + tt * C::BT;
#pragma unroll
        for (int k2 = 0; k2 < 2; ++k2) {
          const int row = m0 + lane + 32 * k2;
          pl[k2] = 0.f;
          pd[k2] = 0.f;
          if (row < L) {
            const int64_t o = stat_offset(p, z, hq, seq_start, row);
            pl[k2] = __ldg(a.lse + o);
            pd[k2] = __ldg(a.delta + o);
          }
        }
      };
      fetch_stats(0);
      for (int t = 0; t < T; ++t) {
        const int st = t % C::STAGES, u = t / C::STAGES;
        int g, tt;
        tile_coords(t, T_h, unit.gh, DET, g, tt);
        const int hq = hq0 + g;
        const int m0 = q_start + tt * C::BT;
        bool ok = true;
        if (t >= C::STAGES) ok = mbar_wait(bar(B2_QE + st), (u - 1) & 1, a.status);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok || *abort_flag) {
          *abort_flag = 1;
          break;
        }
        if (lane == 0) {
          mbar_expect_tx(bar(B2_QF + st), 2 * C::QT_BYTES);
#pragma unroll
          for (int sl = 0; sl < 2; ++sl) {
            tma_load_4d(sbase + C::OFF_Q + st * C::QT_BYTES + sl * C::QT_SLAB, &tmQ,
                        bar(B2_QF + st), sl * 64, seq_start + m0, hq, zc);
            tma_load_4d(sbase + C::OFF_DO + st * C::QT_BYTES + sl * C::QT_SLAB, &tmDO,
                        bar(B2_QF + st), sl * 64, seq_start + m0, hq, zc);
          }
        }
#pragma unroll
        for (int k2 = 0; k2 < 2; ++k2) {
          lse_s[st * C::BT + lane + 32 * k2] = -pl[k2];  // stored negated (packed FMA / ADD)
          del_s[st * C::BT + lane + 32 * k2] = -pd[k2];
        }
        mbar_arrive(bar(B2_QF + st));
        last_tile = t;
        if (t + 1 < T) fetch_stats(t + 1);
      }
      if (*abort_flag && lane == 0) {
        mbar_wait(bar(B2_KV), 0, a.status);
        for (int t = max(0, last_tile - C::STAGES + 1); t <= last_tile; ++t)
          mbar_wait(bar(B2_QF + t % C::STAGES), (t / C::STAGES) & 1, a.status);
      }
    } else if (warp == C::WARP_MMA) {
      // ------------------------------------------------------------ MMA issuer (converged)
      // The whole warp runs the schedule and its waits; one elected lane issues each batch.
      // Descriptors are low words (constant high word) advanced by immediates (16-byte units).
      const bool leader = elect_one() != 0;
      constexpr uint32_t id_s = idesc_f16(BF16, false, false, 128, 64);   // S^T, dP^T
      constexpr uint32_t id_g = idesc_f16(BF16, false, true, 128, 128);   // dV, dK (N = D)
      constexpr uint32_t id_q = idesc_f16(BF16, true, true, 128, 64);     // dQ^T
      const uint32_t sK = sbase + C::OFF_K, sV = sbase + C::OFF_V;
      const uint32_t dK_s = sdesc_lo(sK, 16), dV_s = sdesc_lo(sV, 16);  // K-major K, V
      const uint32_t dK_q = sdesc_lo(sK, C::KV_SLAB);                   // MN-major K (dQ^T's A)
      auto wait_all = [&](uint32_t b, uint32_t par) {
        return __all_sync(0xffffffffu, mbar_wait(b, par, a.status));
      };
      auto issue_sdp = [&](int t) {
        if (!leader) return;
        const int st = t % C::STAGES;
        const uint32_t q_lo = sdesc_lo(sbase + C::OFF_Q + st * C::QT_BYTES, 16);
        const uint32_t o_lo = sdesc_lo(sbase + C::OFF_DO + st * C::QT_BYTES, 16);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t sl = kk >> 2, off = (kk & 3) * 2;
          mma_ss_lo(tmem + C::COL_S, dK_s + sl * (C::KV_SLAB >> 4) + off,
                    q_lo + sl * (C::QT_SLAB >> 4) + off, id_s, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t sl = kk >> 2, off = (kk & 3) * 2;
          mma_ss_lo(tmem + C::COL_DP, dV_s + sl * (C::KV_SLAB >> 4) + off,
                    o_lo + sl * (C::QT_SLAB >> 4) + off, id_s, kk > 0);
        }
        mma_commit(bar(B2_SF + (t & 1)));
      };
      bool ok = wait_all(bar(B2_KV), 0) && wait_all(bar(B2_QF), 0);
      if (ok) {
        tc_fence_after();
        issue_sdp(0);
        __syncwarp();
      }
      for (int t = 0; ok && t < T; ++t) {
        const int st = t % C::STAGES, h = t & 1;
        // next tile's S^T/dP^T as soon as the owner has read the shared buffer
        ok = wait_all(bar(B2_SL), t & 1);
        if (ok && t + 1 < T) ok = wait_all(bar(B2_QF + (t + 1) % C::STAGES), ((t + 1) / C::STAGES) & 1);
        if (!ok || *abort_flag) break;
        tc_fence_after();
        if (t + 1 < T) issue_sdp(t + 1);
        __syncwarp();
        ok = wait_all(bar(B2_SM + h), (t >> 1) & 1);
        if (!ok || *abort_flag) break;
        tc_fence_after();
        if (leader) {
          const uint32_t q_mn = sdesc_lo(sbase + C::OFF_Q + st * C::QT_BYTES, C::QT_SLAB);
          const uint32_t o_mn = sdesc_lo(sbase + C::OFF_DO + st * C::QT_BYTES, C::QT_SLAB);
          const uint32_t ds_k = sdesc_lo(sbase + C::OFF_DS + h * C::DS_BYTES, 16);
          const uint32_t acc0 = t > 0 ? 1u : 0u;
          // dV += P^T dO (A: TMEM, K = 64 queries); dK += dS^T Q (A: shared dS^T, K-major)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_ts_lo(tmem + C::COL_DV, tmem + C::COL_PT + h * 32 + kk * 8, o_mn + 128 * kk, id_g,
                      kk > 0 ? 1u : acc0);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_ss_lo(tmem + C::COL_DK, ds_k + 2 * kk, q_mn + 128 * kk, id_g, kk > 0 ? 1u : acc0);
          mma_commit(bar(B2_BF + h));
        }
        __syncwarp();
        // dQ^T = K^T dS^T (A: K read MN-major, M = head dims; B: dS^T, N = queries)
        if (t >= 1) ok = wait_all(bar(B2_DQE), (t - 1) & 1);
        if (!ok) break;
        tc_fence_after();
        if (leader) {
          const uint32_t ds_mn = sdesc_lo(sbase + C::OFF_DS + h * C::DS_BYTES, 8192);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ss_lo(tmem + C::COL_DQ, dK_q + 128 * kk, ds_mn + 128 * kk, id_q, kk > 0);
          mma_commit(bar(B2_DQF));
          mma_commit(bar(B2_DSF + h));
          mma_commit(bar(B2_QE + st));
        }
        __syncwarp();
      }
      if (!ok) *abort_flag = 1;
      if (leader) {
        mma_commit(bar(B2_KVD));
        mma_commit(bar(B2_END));
      }
      __syncwarp();
      mbar_wait(bar(B2_END), 0, a.status);
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ P / dS warp-groups
    regs_inc<C::REGS_PDS>();
    const int h = warp >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int j = n0 + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tS = tmem + lane_off + C::COL_S;
    const uint32_t tP = tmem + lane_off + C::COL_DP;
    const uint32_t tPT = tmem + lane_off + C::COL_PT + h * 32;
    const float bval = __ldg(p.b_ptr);
    const float cb = bval * p.scale;
    float n = 0.f, nbs = 0.f;
    float2 dn_acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    float2 db_acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    bool ok = true;
    const int qmin = p.causal ? j : 0;
    for (int t = h; t < T; t += 2) {
      const int st = t % C::STAGES;
      int g, tt;
      tile_coords(t, T_h, unit.gh, DET, g, tt);
      const int hq = hq0 + g;
      n = load_n(p, hq);
      nbs = n * bval * p.scale;
      const int mh = q_start + tt * C::BT;
      ok = mbar_wait(bar(B2_QF + st), (t / C::STAGES) & 1, a.status);
      if (ok) ok = mbar_wait(bar(B2_SF + h), (t >> 1) & 1, a.status);
      if (ok && t >= 2) ok = mbar_wait(bar(B2_DSF + h), ((t >> 1) - 1) & 1, a.status);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || *abort_flag) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s0[32], s1[32], d0[32], d1[32];
      tmem_ld32(tS, s0);
      tmem_ld32(tS + 32, s1);
      tmem_ld32(tP, d0);
      tmem_ld32(tP + 32, d1);
      tmem_ld_wait_only();
      tmem_pin_n(s0);
      tmem_pin_n(s1);
      tmem_pin_n(d0);
      tmem_pin_n(d1);
      tc_fence_before();
      mbar_arrive(bar(B2_SL));  // the shared S^T/dP^T buffer may be overwritten now
      const bool full = (!p.causal || mh >= n0 + C::BN - 1) && (mh + C::BT <= L) && (n0 + C::BN <= L);
      const float* lrow = lse_s + st * C::BT;
      const float* drow = del_s + st * C::BT;
      uint8_t* dsrow = smem + C::OFF_DS + h * C::DS_BYTES + r * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {  // 16-query chunks: more element pairs overlap than at 32
        uint32_t pk[8], dk[8];
        const uint32_t(&cs)[16] =
            *reinterpret_cast<const uint32_t(*)[16]>(&((c >> 1) ? s1 : s0)[16 * (c & 1)]);
        const uint32_t(&cd)[16] =
            *reinterpret_cast<const uint32_t(*)[16]>(&((c >> 1) ? d1 : d0)[16 * (c & 1)]);
        // A chunk masked for every row of this warp: P = dS = 0, transform skipped.
        const bool dead = !full && ((p.causal && mh + c * 16 + 15 < n0 + quad * 32) ||
                                    mh + c * 16 >= L || n0 + quad * 32 >= L);
        if (dead) {
#pragma unroll
          for (int i = 0; i < 8; ++i) pk[i] = dk[i] = 0u;
        } else if (full)
          bwd_chunk<16, BF16, false, false>(cs, cd, lrow + c * 16, drow + c * 16, n, cb, nbs,
                                            mh + c * 16, qmin, L, j < L, dn_acc, db_acc, pk, dk);
        else
          bwd_chunk<16, BF16, true, false>(cs, cd, lrow + c * 16, drow + c * 16, n, cb, nbs,
                                           mh + c * 16, qmin, L, j < L, dn_acc, db_acc, pk, dk);
        if (c == 0) {  // dV of this group's previous tile must have read its P^T columns
          bool okb = t < 2 || mbar_wait(bar(B2_BF + h), ((t >> 1) - 1) & 1, a.status);
          if (!__all_sync(0xffffffffu, okb)) *abort_flag = 1;
          tc_fence_after();
        }
        tmem_st8(tPT + c * 8, pk);
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
          const int chunk = c * 2 + q2;
          *reinterpret_cast<uint4*>(dsrow + ((chunk ^ (r & 7)) << 4)) =
              make_uint4(dk[q2 * 4], dk[q2 * 4 + 1], dk[q2 * 4 + 2], dk[q2 * 4 + 3]);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      fence_proxy_async_smem();
      mbar_arrive(bar(B2_SM + h));
      // this group's last tile of q-head g (deterministic order, where heads alternate: every
      // tile): write its per-warp dn/db partials
      const bool head_end = DET || (tt + 2 >= T_h);
      if (head_end) {
        float x1 = (dn_acc[0].x + dn_acc[0].y) + (dn_acc[1].x + dn_acc[1].y);
        float x2 = (db_acc[0].x + db_acc[0].y) + (db_acc[1].x + db_acc[1].y);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          x1 += __shfl_xor_sync(0xffffffffu, x1, o);
          x2 += __shfl_xor_sync(0xffffffffu, x2, o);
        }
        if (lane == 0) {
          const int64_t pi = bwd_partial_index(a, z, hq, kvb, DET ? tt : 0) + 4 * h + quad;
          a.dn_part[pi] = x1 * kLn2;
          a.db_part[pi] = x2 * n * p.scale;
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) dn_acc[i] = db_acc[i] = make_float2(0.f, 0.f);
      }
    }
    if (!ok) *abort_flag = 1;
    // ---- epilogue: group 0 stores dK, group 1 stores dV (one key row per thread, 128 dims)
    bool okd = ok && mbar_wait(bar(B2_KVD), 0, a.status);
    okd = __all_sync(0xffffffffu, okd);
    if (okd && !*abort_flag) {
      tc_fence_after();
      store_dkv_row<BF16, C::D>(a, unit, seq_start, h, r, j, L,
                                tmem + lane_off + (h ? C::COL_DV : C::COL_DK));
    }
  } else {
    // ------------------------------------------------------------ dQ^T drain (warps 8..11)
    // Warp `quad` owns head dims [32 quad, 32 quad + 32) (TMEM lanes): 64 queries x 32 dims of
    // fp32 staged row-major (query-major) in its 8 KB, then one 2-D TMA reduce-add.
    regs_dec<C::REGS_DQ>();
    const int quad = warp & 3;
    float* stage = reinterpret_cast<float*>(smem + C::OFF_DQS + quad * C::DQS_WARP);
    const uint32_t stage_s = sbase + C::OFF_DQS + quad * C::DQS_WARP;
    const uint32_t tQ = tmem + ((uint32_t)(quad * 32) << 16) + C::COL_DQ;
    bool ok = true;
    for (int t = 0; t < T; ++t) {
      ok = mbar_wait(bar(B2_DQF), t & 1, a.status);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || *abort_flag) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t v0[32], v1[32];
      tmem_ld32(tQ, v0);
      tmem_ld32(tQ + 32, v1);
      tmem_ld_wait_only();
      tmem_pin(v0);
      tmem_pin(v1);
      tc_fence_before();
      mbar_arrive(bar(B2_DQE));
      if (lane == 0) bulk_wait_read0();
      __syncwarp();
#pragma unroll
      for (int qi = 0; qi < 32; ++qi) stage[qi * 32 + lane] = __uint_as_float(v0[qi]);
#pragma unroll
      for (int qi = 0; qi < 32; ++qi) stage[(32 + qi) * 32 + lane] = __uint_as_float(v1[qi]);
      fence_proxy_async_smem();
      __syncwarp();
      bool okw = true;
      if (lane == 0) {
        int g, tt;
        tile_coords(t, T_h, unit.gh, DET, g, tt);
        const int hq = hq0 + g;
        const int m0 = q_start + tt * C::BT;
        const int row0 = p.cu_seqlens ? (int)((int64_t)hq * a.dq_rows + seq_start + m0)
                                      : (int)(((int64_t)z * p.Hq + hq) * a.dq_rows + m0);
        // Deterministic dq: this warp's head dims of the tile take their turn after key blocks
        // 0 .. kvb - 1, and pass it on once the add has been performed.
        int* sem = DET ? a.dq_sem +
                               (((int64_t)z * p.Hq + hq) * a.ntq + q_start / C::BT + tt) * 4 + quad
                         : nullptr;
        if (DET) okw = sem_wait_eq(sem, kvb, a.status);
        if (okw) {
          tma_reduce_add_2d(&tmDQ, stage_s, quad * 32, row0);
          bulk_commit();
          if (DET) {
            bulk_wait0();
            sem_release_next(sem);
          }
        }
      }
      if (!__shfl_sync(0xffffffffu, okw ? 1 : 0, 0)) {
        ok = false;
        break;
      }
    }
    if (!ok) *abort_flag = 1;
    // The staging buffers must outlive the TMA engine's reads of them; the reduce-adds' global
    // writes need no wait here (they are performed before the grid completes).
    if (lane == 0) bulk_wait_read0();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == C::WARP_PRODUCER) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  // A wait of this CTA expired: its dK / dV rows and dn / db partials are NaN, never partial
  // results (dq is filled with NaN by the conversion kernel, which reads the status word).
  if (*abort_flag) bwd_block_partials<BF16>(a, unit, seq_start, n0, L, true);
}

struct BwdLayout {
  int nkv, hsplit, ntq, ppk;
  int64_t dq_rows;
  size_t dq_bytes, part_bytes, dkv_bytes, sem_bytes, total;
};

constexpr int kNumSMs = 148;      // B200
constexpr double kCtaCost = 4.0;  // per-CTA fixed cost of the backward, in query-tile periods

// q-head slices per key block (see BwdArgs::hsplit): the divisor s of the GQA ratio that
// minimises max(longest CTA, average work per SM), in query tiles of `bt` rows with a fixed cost
// of four tiles per CTA (setup, first loads, pipeline fill and the dK / dV epilogue; this value
// reproduces the measured B200 choices at config-2 shapes: B = 1 -> 2 slices, 0.203 -> 0.138 ms;
// B = 2 -> 1, where 2 slices measured 0.218 against 0.198 ms). A dense estimate (every sequence
// max_seqlen long); another s must be at least 3% better than the smaller one to be taken.
// SSA_BWD_HSPLIT overrides it (a divisor of the GQA ratio) for measurements.
int choose_hsplit(const Problem& p, int bt) {
  if (const char* e = getenv("SSA_BWD_HSPLIT")) {
    const int s = atoi(e);
    if (s >= 1 && p.gqa % s == 0) return s;
  }
  const int nkv = (p.max_seqlen + 127) / 128;
  const double units = (double)p.B * p.Hkv;
  double total = 0.0, longest = 0.0;
  for (int kvb = 0; kvb < nkv; ++kvb) {
    const int rows = p.causal ? p.max_seqlen - 128 * kvb : p.max_seqlen;
    const double th = (double)((rows + bt - 1) / bt);
    total += th;
    longest = longest > th ? longest : th;
  }
  total *= units * p.gqa;
  int best = 1;
  double best_cost = 1e300;
  for (int s = 1; s <= p.gqa && s <= 8; ++s) {
    if (p.gqa % s) continue;
    const double ctas = nkv * units * s;
    const double c1 = longest * p.gqa / s + kCtaCost, c2 = (total + kCtaCost * ctas) / kNumSMs;
    const double cost = c1 > c2 ? c1 : c2;
    if (cost < best_cost * 0.97) {
      best = s;
      best_cost = cost;
    }
  }
  return best;
}

inline size_t al256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Workspace of the tensor-core backward: the fp32 dQ accumulator (rows padded to 128 per head,
// or 128 rows after the last packed token) and the dn/db partials.
BwdLayout bwd_layout(const Problem& p) {
  BwdLayout l;
  l.nkv = (p.max_seqlen + 127) / 128;
  const int dk = p.D == 128 ? 128 : 64;  // the kernel's head dim (D = 32 runs the D = 64 kernel)
  if (p.cu_seqlens) {
    l.dq_rows = (int64_t)p.N + 128;
    l.dq_bytes = al256(sizeof(float) * (size_t)p.Hq * l.dq_rows * dk);
  } else {
    l.dq_rows = (int64_t)((p.N + 127) / 128) * 128;
    l.dq_bytes = al256(sizeof(float) * (size_t)p.B * p.Hq * l.dq_rows * dk);
  }
  const int bt = p.D == 128 ? 64 : 128;  // query tile rows of the kernel
  l.ntq = (p.max_seqlen + bt - 1) / bt;
  l.ppk = p.det ? 8 * l.ntq : 8;
  l.part_bytes = al256(sizeof(float) * (size_t)p.B * p.Hq * l.ppk * l.nkv);
  l.sem_bytes = p.det ? al256(sizeof(int) * (size_t)p.B * p.Hq * l.ntq * 4) : 0;
  l.hsplit = choose_hsplit(p, bt);
  l.dkv_bytes = l.hsplit > 1 ? al256(sizeof(float) * (size_t)p.B * p.Hkv * l.nkv * l.hsplit * 2 *
                                     128 * dk)
                             : 0;
  l.total = l.dq_bytes + 2 * l.part_bytes + l.dkv_bytes + l.sem_bytes;
  return l;
}

template <bool BF16>
int run_bwd(const Problem& p, TensorRef q, TensorRef k, TensorRef v, TensorRef out,
            TensorRef dout, const float* lse, float* delta, TensorRef dq, TensorRef dk,
            TensorRef dv, float* dn, float* db, void* dom, void* ws, size_t ws_bytes,
            cudaStream_t st) {
  using C = BwdCfg;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  const int dtype = BF16 ? SSA_DTYPE_BF16 : SSA_DTYPE_F16;
  const BwdLayout lay = bwd_layout(p);
  if (!ws || ws_bytes < lay.total) return SSA_ERR_WORKSPACE;
  if (p.drop_seed && !dom) return SSA_ERR_WORKSPACE;
  T* domT = p.drop_seed ? static_cast<T*>(dom) : nullptr;
  float* lse_sh = domT ? dropout_lse_buffer(p, dom) : nullptr;
  CUtensorMap tq, tk, tv, tdo;
  int rc;
  if ((rc = make_tmap_bhnd(&tq, q, p, dtype, p.Hq, C::BT)) != SSA_OK) return rc;
  if ((rc = make_tmap_bhnd(&tk, k, p, dtype, p.Hkv, C::BN)) != SSA_OK) return rc;
  if ((rc = make_tmap_bhnd(&tv, v, p, dtype, p.Hkv, C::BN)) != SSA_OK) return rc;
  // with output dropout the main kernel reads the masked dout the preprocess writes
  if ((rc = make_tmap_bhnd(&tdo, domT ? dropout_dout_ref(p, domT) : dout, p, dtype, p.Hq,
                           C::BT)) != SSA_OK)
    return rc;
  uint8_t* w = static_cast<uint8_t*>(ws);
  BwdArgs a;
  a.p = p;
  a.dk = dk;
  a.dv = dv;
  a.lse = lse_sh ? lse_sh : lse;
  a.delta = delta;
  a.dq_accum = reinterpret_cast<float*>(w);
  a.dq_rows = lay.dq_rows;
  a.dn_part = reinterpret_cast<float*>(w + lay.dq_bytes);
  a.db_part = reinterpret_cast<float*>(w + lay.dq_bytes + lay.part_bytes);
  a.status = device_status_ptr();
  a.nkv = lay.nkv;
  a.hsplit = lay.hsplit;
  a.dkv_part = lay.hsplit > 1
                   ? reinterpret_cast<float*>(w + lay.dq_bytes + 2 * lay.part_bytes)
                   : nullptr;
  a.ppk = lay.ppk;
  a.ntq = lay.ntq;
  a.dq_sem = p.det ? reinterpret_cast<int*>(w + lay.dq_bytes + 2 * lay.part_bytes + lay.dkv_bytes)
                   : nullptr;
  {
    const unsigned gy = p.cu_seqlens ? p.Hq : p.B * p.Hq;
    const cudaError_t e =
        p.D == 32
            ? launch_pdl(bwd_preprocess_sm100_kernel<T, 32, 64>,
                         dim3((unsigned)((lay.dq_rows + 63) / 64), gy), dim3(256), 0, st, p, out,
                         dout, delta, a.dq_accum, lay.dq_rows, a.dq_sem, 4 * lay.ntq, domT, lse,
                         lse_sh)
            : launch_pdl(bwd_preprocess_sm100_kernel<T, 64, 64>,
                         dim3((unsigned)((lay.dq_rows + 31) / 32), gy), dim3(256), 0, st, p, out,
                         dout, delta, a.dq_accum, lay.dq_rows, a.dq_sem, 4 * lay.ntq, domT, lse,
                         lse_sh);
    if (e != cudaSuccess) return SSA_ERR_LAUNCH;
    note_launches(1);
  }
  // dQ accumulator as a 2-D fp32 tensor [rows][64] for the drain's tiled reduce-adds:
  // {32 columns x 32 rows} boxes in the 128-byte swizzle.
  CUtensorMap tdq;
  {
    auto enc = tmap_encoder();
    if (!enc) return SSA_ERR_CUDA;
    const uint64_t rows = (uint64_t)(p.cu_seqlens ? p.Hq : p.B * p.Hq) * (uint64_t)lay.dq_rows;
    cuuint64_t dims[2] = {(cuuint64_t)C::D, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)C::D * 4};
    cuuint32_t box[2] = {32u, 32u};
    cuuint32_t estr[2] = {1u, 1u};
    if (enc(&tdq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.dq_accum, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return SSA_ERR_CUDA;
  }
  auto kern = p.det ? bwd_sm100_kernel<BF16, true> : bwd_sm100_kernel<BF16, false>;
  if (set_smem_limit_once(reinterpret_cast<const void*>(kern), (int)C::SMEM_BYTES) != SSA_OK)
    return SSA_ERR_CUDA;
  const long long grid = (long long)lay.nkv * p.B * p.Hkv * lay.hsplit;
  if (launch_pdl(kern, dim3((unsigned)grid), dim3(C::THREADS), C::SMEM_BYTES, st, tq, tk, tv, tdo,
                 tdq, a) != cudaSuccess)
    return SSA_ERR_LAUNCH;
  note_launches(1);
  if (p.D == 32)
    return launch_dq_convert_dndb<T, 32, 64>(p, a.dq_accum, a.dq_rows, dq, a.dn_part, a.db_part,
                                             lay.ppk * lay.nkv, dn, db, a, st);
  return launch_dq_convert_dndb<T, 64, 64>(p, a.dq_accum, a.dq_rows, dq, a.dn_part, a.db_part,
                                           lay.ppk * lay.nkv, dn, db, a, st);
}

template <bool BF16>
int run_bwd128(const Problem& p, TensorRef q, TensorRef k, TensorRef v, TensorRef out,
               TensorRef dout, const float* lse, float* delta, TensorRef dq, TensorRef dk,
               TensorRef dv, float* dn, float* db, void* dom, void* ws, size_t ws_bytes,
               cudaStream_t st) {
  using C = Bwd128Cfg;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  const int dtype = BF16 ? SSA_DTYPE_BF16 : SSA_DTYPE_F16;
  const BwdLayout lay = bwd_layout(p);
  if (!ws || ws_bytes < lay.total) return SSA_ERR_WORKSPACE;
  if (p.drop_seed && !dom) return SSA_ERR_WORKSPACE;
  T* domT = p.drop_seed ? static_cast<T*>(dom) : nullptr;
  float* lse_sh = domT ? dropout_lse_buffer(p, dom) : nullptr;
  CUtensorMap tq, tk, tv, tdo, tdq;
  int rc;
  if ((rc = make_tmap_bhnd(&tq, q, p, dtype, p.Hq, C::BT)) != SSA_OK) return rc;
  if ((rc = make_tmap_bhnd(&tk, k, p, dtype, p.Hkv, C::BN)) != SSA_OK) return rc;
  if ((rc = make_tmap_bhnd(&tv, v, p, dtype, p.Hkv, C::BN)) != SSA_OK) return rc;
  if ((rc = make_tmap_bhnd(&tdo, domT ? dropout_dout_ref(p, domT) : dout, p, dtype, p.Hq,
                           C::BT)) != SSA_OK)
    return rc;
  uint8_t* w = static_cast<uint8_t*>(ws);
  BwdArgs a;
  a.p = p;
  a.dk = dk;
  a.dv = dv;
  a.lse = lse_sh ? lse_sh : lse;
  a.delta = delta;
  a.dq_accum = reinterpret_cast<float*>(w);
  a.dq_rows = lay.dq_rows;
  a.dn_part = reinterpret_cast<float*>(w + lay.dq_bytes);
  a.db_part = reinterpret_cast<float*>(w + lay.dq_bytes + lay.part_bytes);
  a.status = device_status_ptr();
  a.nkv = lay.nkv;
  a.hsplit = lay.hsplit;
  a.dkv_part = lay.hsplit > 1
                   ? reinterpret_cast<float*>(w + lay.dq_bytes + 2 * lay.part_bytes)
                   : nullptr;
  a.ppk = lay.ppk;
  a.ntq = lay.ntq;
  a.dq_sem = p.det ? reinterpret_cast<int*>(w + lay.dq_bytes + 2 * lay.part_bytes + lay.dkv_bytes)
                   : nullptr;
  {
    dim3 gp((unsigned)((lay.dq_rows + 15) / 16), p.cu_seqlens ? p.Hq : p.B * p.Hq);
    if (launch_pdl(bwd_preprocess_sm100_kernel<T, 128, 128>, gp, dim3(256), 0, st, p, out, dout,
                   delta, a.dq_accum, lay.dq_rows, a.dq_sem, 4 * lay.ntq, domT, lse,
                   lse_sh) != cudaSuccess)
      return SSA_ERR_LAUNCH;
  }
  {  // dQ accumulator as 2-D fp32 [rows][128]; {32 head dims x 64 queries} boxes, no swizzle
    auto enc = tmap_encoder();
    if (!enc) return SSA_ERR_CUDA;
    const uint64_t rows = (uint64_t)(p.cu_seqlens ? p.Hq : p.B * p.Hq) * (uint64_t)lay.dq_rows;
    cuuint64_t dims[2] = {(cuuint64_t)C::D, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)C::D * 4};
    cuuint32_t box[2] = {32u, (cuuint32_t)C::BT};
    cuuint32_t estr[2] = {1u, 1u};
    if (enc(&tdq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.dq_accum, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return SSA_ERR_CUDA;
  }
  auto kern = p.det ? bwd128_sm100_kernel<BF16, true> : bwd128_sm100_kernel<BF16, false>;
  if (set_smem_limit_once(reinterpret_cast<const void*>(kern), (int)C::SMEM_BYTES) != SSA_OK)
    return SSA_ERR_CUDA;
  const long long grid = (long long)lay.nkv * p.B * p.Hkv * lay.hsplit;
  kern<<<(unsigned)grid, C::THREADS, C::SMEM_BYTES, st>>>(tq, tk, tv, tdo, tdq, a);
  note_launches(2);
  return launch_dq_convert_dndb<T, 128, 128>(p, a.dq_accum, a.dq_rows, dq, a.dn_part, a.db_part,
                                        lay.ppk * lay.nkv, dn, db, a, st);
}

}  // namespace sm100

bool sm100_bwd_supports(int dtype, int D) {  // D = 32 runs the D = 64 kernel (see sm100_supports)
  return (dtype == SSA_DTYPE_BF16 || dtype == SSA_DTYPE_F16) && (D == 32 || D == 64 || D == 128);
}

size_t sm100_bwd_workspace_bytes(const Problem& p) { return sm100::bwd_layout(p).total; }

int launch_bwd_sm100(int dtype, const Problem& p, TensorRef q, TensorRef k, TensorRef v,
                     TensorRef out, TensorRef dout, const float* lse, float* delta, TensorRef dq,
                     TensorRef dk, TensorRef dv, float* dn, float* db, void* dom, void* ws,
                     size_t ws_bytes, cudaStream_t st) {
  // The dQ accumulator's reduce-adds address its rows with 32-bit TMA coordinates.
  const sm100::BwdLayout lay = sm100::bwd_layout(p);
  if ((int64_t)(p.cu_seqlens ? p.Hq : p.B * p.Hq) * lay.dq_rows >= (int64_t)1 << 31)
    return SSA_ERR_BAD_SHAPE;
  if (p.D == 128)
    return dtype == SSA_DTYPE_BF16
               ? sm100::run_bwd128<true>(p, q, k, v, out, dout, lse, delta, dq, dk, dv, dn, db,
                                         dom, ws, ws_bytes, st)
               : sm100::run_bwd128<false>(p, q, k, v, out, dout, lse, delta, dq, dk, dv, dn, db,
                                          dom, ws, ws_bytes, st);
  if (p.D != 64 && p.D != 32) return SSA_ERR_UNSUPPORTED;
  return dtype == SSA_DTYPE_BF16
             ? sm100::run_bwd<true>(p, q, k, v, out, dout, lse, delta, dq, dk, dv, dn, db, dom,
                                    ws, ws_bytes, st)
             : sm100::run_bwd<false>(p, q, k, v, out, dout, lse, delta, dq, dk, dv, dn, db, dom,
                                     ws, ws_bytes, st);
}

}  // namespace ssa
