// ssa_sm100_fwd.cu — SSA attention forward for sm_100a: TMA + tcgen05 + TMEM.
//
// Computes what the reference's _ssa_attn_fwd computes (ssa_triton_kernel.py:150-260, inner
// loop :40-124): S = scale * Q K^T, the SSA transform t2 = n * sign(s) * log2(1 + b|s|)
// (= n * sign(s) * log1p(b|s|) * log2 e, :96-107), an online base-2 normaliser (:110-113),
// O = P V / l and M = m + log2 l (:248-255).
//
// One CTA = one 128-row query tile of one (sequence, q-head). 6 warps:
//   warp 0      TMEM allocator + TMA producer (Q once, K/V through a 2-stage ring)
//   warp 1      MMA issuer: S = Q K^T (SS form, fp32 in TMEM), O += P V (TS form: P read
//               straight from TMEM). P has its own columns, so S_{j+1} is issued as soon as the
//               softmax warps hold S_j in registers and runs under their work on block j.
//   warps 2..5  one thread per query row: tcgen05.ld its S row, SSA transform, running max
//               and sum, P (bf16/f16) written to TMEM, O correction, epilogue.
// Two CTAs share an SM (TMEM 2 x 256 columns, ~81 KB shared memory each), so one CTA's
// transcendental work overlaps the other's tensor-core work.
//
// Rescaling: each block's row maximum is bounded from above by U = |n| log2(1 + b max|s|)
// (t2 is monotone in s); the running reference only moves when U exceeds it by more than
// kRescaleThreshold (log2 units), so P <= 2^8 and O is corrected rarely. m, l and O always
// refer to the same reference, so the result is exact up to rounding.
//
// Every mbarrier wait is bounded (~1 s): on expiry the kernel records SSA_ERR_DEVICE_TIMEOUT in
// the device status word, unwinds, waits for its own in-flight TMA / MMA work (bounded) and
// frees its TMEM.
#include <cudaTypedefs.h>

#include "ssa_internal.h"
#include "ssa_sm100.cuh"
#include "ssa_tmap.h"

namespace ssa {
namespace sm100 {

constexpr float kRescaleThreshold = 8.0f;
// Element pairs, of every 4, whose exponential is evaluated on the FMA pipe (exp2_poly2).
// Measured on B200: D = 128 gains from 1 of 4 (2 of 4 and more lose again); at D = 64 the
// softmax is not bound by the special-function unit alone and the extra work only costs time.
template <int D>
constexpr int kEmuPairs = D == 128 ? 1 : 0;
// D = 64: every element's sign * log2(1 + b|s|) is computed in a first pass over the block (in
// place of s), the exponentials in a second. Same operations and results as one pass per element
// pair; measured on B200 the two-pass order is 1% faster at D = 64 (config 2) and 1% slower at
// D = 128, which keeps one pass.
template <int D>
constexpr bool kLogFirst = D == 64;

template <int D>
struct FwdCfg {
  static constexpr int BM = 128;
  static constexpr int BN = (D == 64) ? 128 : 64;
  static constexpr int KH = D / 64;  // 64-element (128-byte) column slabs per row
  static constexpr int STAGES = 2;
  static constexpr uint32_t Q_BYTES = BM * D * 2;
  static constexpr uint32_t KV_BYTES = BN * D * 2;
  static constexpr uint32_t OFF_Q = 0;
  static constexpr uint32_t OFF_K = Q_BYTES;
  static constexpr uint32_t OFF_V = OFF_K + STAGES * KV_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_V + STAGES * KV_BYTES;
  static constexpr uint32_t SMEM_BYTES = OFF_BAR + 256 + 1024;  // + slack for 1 KB alignment
  static constexpr uint32_t TMEM_COLS = 256;
  static constexpr uint32_t COL_S = 0;            // S (fp32, BN columns)
  static constexpr uint32_t COL_P = BN;           // P (packed 16-bit, BN / 2 columns)
  static constexpr uint32_t COL_O = BN + BN / 2;  // O accumulator (fp32, D columns)
  static constexpr int THREADS = 192;
  static_assert(BN + BN / 2 + D <= (int)TMEM_COLS, "TMEM budget");
};

struct FwdArgs {
  Problem p;
  TensorRef o;
  float* lse;
  unsigned int* status;
  int tiles_m;
};

enum FwdBar : int {
  FB_Q = 0,
  FB_KF = 1,   // 2 stages
  FB_VF = 3,   // 2 stages
  FB_KVE = 5,  // 2 stages
  FB_S = 7,    // S_j in TMEM
  FB_SC = 8,   // S_j pulled into registers by the softmax warps: its columns are free
  FB_P = 9,    // P_j in TMEM (and O corrected for block j)
  FB_O = 10,   // P_j V_j retired: O final through block j, P columns free
  FB_END = 11,
  FB_COUNT = 12
};

template <int D, bool BF16>
__global__ void __launch_bounds__(192, 2)
    fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ,
                     const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const FwdArgs a) {
  using C = FwdCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto bar = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + 8 * FB_COUNT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Problem& p = a.p;
  // Launched programmatically: the grid may be dispatched while the previous kernel on the stream
  // still runs, and waits here, before any global access (inputs that kernel may write, outputs in
  // memory it may still read, the status word it may set). The next kernel may launch as soon as
  // every CTA of this grid has started; it waits for this grid the same way.
  griddep_wait();
  griddep_launch_dependents();
  const int BH = p.B * p.Hq;
  const int tile = a.tiles_m - 1 - (int)(blockIdx.x / BH);  // longest causal rows first
  const int bh = blockIdx.x % BH;
  const int z = bh / p.Hq, hq = bh % p.Hq, hkv = hq / p.gqa;
  int seq_start, L;
  seq_bounds(p, z, seq_start, L);
  const int m0 = tile * C::BM;
  // Block-uniform exits, before any barrier or TMEM allocation: nothing to do, or an earlier
  // launch already recorded a device-side timeout (this tile's out and lse rows are then NaN).
  if (m0 >= L) return;
  if (block_status_failed(a.status)) {
    nan_fill_rows16<BF16>(a.o, p, z, hq, seq_start, m0, min(m0 + C::BM, L), a.lse);
    return;
  }
  const int kv_len = p.causal ? min(L, m0 + C::BM) : L;
  const int nblk = (kv_len + C::BN - 1) / C::BN;
  const int zc = p.cu_seqlens ? 0 : z;

  if (threadIdx.x == 0) {
    mbar_init(bar(FB_Q), 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar(FB_KF + s), 1);
      mbar_init(bar(FB_VF + s), 1);
      mbar_init(bar(FB_KVE + s), 1);
    }
    mbar_init(bar(FB_S), 1);
    mbar_init(bar(FB_SC), 128);
    mbar_init(bar(FB_P), 128);
    mbar_init(bar(FB_O), 1);
    mbar_init(bar(FB_END), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_expect_tx(bar(FB_Q), C::Q_BYTES);
#pragma unroll
      for (int h = 0; h < C::KH; ++h)
        tma_load_4d(sbase + C::OFF_Q + h * C::BM * 128, &tmQ, bar(FB_Q), h * 64, seq_start + m0,
                    hq, zc);
      int last_use[C::STAGES] = {-1, -1};
      for (int j = 0; j < nblk; ++j) {
        const int st = j & 1, u = j >> 1;
        if (j >= C::STAGES && !mbar_wait(bar(FB_KVE + st), (u - 1) & 1, a.status)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        const int r0 = seq_start + j * C::BN;
        mbar_expect_tx(bar(FB_KF + st), C::KV_BYTES);
#pragma unroll
        for (int h = 0; h < C::KH; ++h)
          tma_load_4d(sbase + C::OFF_K + st * C::KV_BYTES + h * C::BN * 128, &tmK,
                      bar(FB_KF + st), h * 64, r0, hkv, zc);
        mbar_expect_tx(bar(FB_VF + st), C::KV_BYTES);
#pragma unroll
        for (int h = 0; h < C::KH; ++h)
          tma_load_4d(sbase + C::OFF_V + st * C::KV_BYTES + h * C::BN * 128, &tmV,
                      bar(FB_VF + st), h * 64, r0, hkv, zc);
        last_use[st] = u;
      }
      if (*abort_flag) {  // drain this CTA's own loads before its shared memory is released
        mbar_wait(bar(FB_Q), 0, a.status);
        for (int s = 0; s < C::STAGES; ++s)
          if (last_use[s] >= 0) {
            mbar_wait(bar(FB_KF + s), last_use[s] & 1, a.status);
            mbar_wait(bar(FB_VF + s), last_use[s] & 1, a.status);
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp runs the schedule; one elected lane issues each tcgen05.mma / commit.
    {
      const uint32_t leader = elect_one();
      constexpr uint32_t idesc_s = idesc_f16(BF16, false, false, 128, C::BN);
      constexpr uint32_t idesc_o = idesc_f16(BF16, false, true, 128, D);
      auto wait_all = [&](uint32_t b, uint32_t par) {
        return __all_sync(0xffffffffu, mbar_wait(b, par, a.status));
      };
      auto issue_s = [&](int j) {  // S_j = Q K_j^T
        const int st = j & 1;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)(kk & 3) * 32u;  // 16 elements = 32 B within the slab
          const uint32_t slab = (uint32_t)(kk >> 2);
          const uint64_t ad = sdesc_sw128(sbase + C::OFF_Q + slab * C::BM * 128 + off, 16, 1024);
          const uint64_t bd = sdesc_sw128(
              sbase + C::OFF_K + st * C::KV_BYTES + slab * C::BN * 128 + off, 16, 1024);
          mma_ss_p(tmem + C::COL_S, ad, bd, idesc_s, kk > 0 ? 1u : 0u, leader);
        }
        mma_commit_p(bar(FB_S), leader);
      };
      bool ok = wait_all(bar(FB_Q), 0) && wait_all(bar(FB_KF), 0);
      if (ok && !*abort_flag) {
        tc_fence_after();
        issue_s(0);
      }
      for (int j = 0; ok && j < nblk; ++j) {
        const int st = j & 1, u = j >> 1;
        // S_{j+1} as soon as the softmax warps hold S_j in registers: it is computed while they
        // work on block j (P_j goes to its own columns, so S_{j+1} need not wait for P_j V_j).
        if (j + 1 < nblk) {
          ok = wait_all(bar(FB_KF + (st ^ 1)), ((j + 1) >> 1) & 1);
          if (ok) ok = wait_all(bar(FB_SC), j & 1);
          if (!ok || *abort_flag) break;
          tc_fence_after();
          issue_s(j + 1);
        }
        ok = wait_all(bar(FB_VF + st), u & 1);
        if (ok) ok = wait_all(bar(FB_P), j & 1);
        if (!ok || *abort_flag) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < C::BN / 16; ++kk) {
          const uint64_t bd = sdesc_sw128(sbase + C::OFF_V + st * C::KV_BYTES + kk * 16 * 128,
                                          C::BN * 128, 1024);
          mma_ts_p(tmem + C::COL_O, tmem + C::COL_P + kk * 8, bd, idesc_o,
                   (j > 0 || kk > 0) ? 1u : 0u, leader);
        }
        mma_commit_p(bar(FB_O), leader);
        mma_commit_p(bar(FB_KVE + st), leader);
      }
      if (!ok) *abort_flag = 1;
      mma_commit_p(bar(FB_END), leader);  // all MMAs of this CTA retired before TMEM is freed
      mbar_wait(bar(FB_END), 0, a.status);
    }
  } else {
    // ------------------------------------------------------------------ softmax rows
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int row = m0 + r;
    const uint32_t t_lane = tmem + ((uint32_t)(quad * 32) << 16);
    const float n = load_n(p, hq);
    const float cb = __ldg(p.b_ptr) * p.scale;  // b * |scale|; scale > 0 on this path
    float m_run = -INFINITY, l_run = 0.f;  // m_run: reference of l and O (log2 units)
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      ok = mbar_wait(bar(FB_S), j & 1, a.status);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || *abort_flag) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[C::BN / 32][32];
#pragma unroll
      for (int c = 0; c < C::BN / 32; ++c) tmem_ld32(t_lane + C::COL_S + c * 32, sr[c]);
      tmem_ld_wait_only();
#pragma unroll
      for (int c = 0; c < C::BN / 32; ++c) tmem_pin(sr[c]);
      tc_fence_before();
      mbar_arrive(bar(FB_SC));  // S_j is in registers: the MMA warp may write S_{j+1}

      const int n0 = j * C::BN;
      const bool full = (n0 + C::BN <= L) && (!p.causal || n0 + C::BN - 1 <= m0);
      // Normaliser reference: t2 = n sign(s) log2(1 + b|s|) <= |n| log2(1 + b max|s|) = U, so U
      // bounds the row's max from above without transforming every element first. Masked
      // elements may enter the bound (they are real scores of this row, or zero padding); only
      // the bound's tightness depends on them, never the result.
      float am0 = 0.f, am1 = 0.f, am2 = 0.f, am3 = 0.f;
#pragma unroll
      for (int c = 0; c < C::BN / 32; ++c) {
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          am0 = fmaxf(am0, fabsf(__uint_as_float(sr[c][i])));
          am1 = fmaxf(am1, fabsf(__uint_as_float(sr[c][i + 1])));
          am2 = fmaxf(am2, fabsf(__uint_as_float(sr[c][i + 2])));
          am3 = fmaxf(am3, fabsf(__uint_as_float(sr[c][i + 3])));
        }
      }
      const float ubound = fabsf(n) * lg2_approx(fmaf(fmaxf(fmaxf(am0, am1), fmaxf(am2, am3)), cb, 1.0f));
      const bool need = ubound > m_run + kRescaleThreshold;  // always true on the first block
      float alpha = 1.f;
      if (need) {
        alpha = ex2_approx(m_run - ubound);
        m_run = ubound;
      }
      // P for element pairs: t2 - m on a packed f32x2 FMA, the row sum on packed adds.
      const float2 n2 = make_float2(n, n), negm2 = make_float2(-m_run, -m_run);
      float2 rs2 = make_float2(0.f, 0.f);
      uint32_t pk[C::BN / 64][32];
      const int lim = p.causal ? min(L - 1, row) : L - 1;  // last visible key of this row
      // kEmuPairs of every 4 element pairs take 2^t from the FMA-pipe polynomial, the rest from
      // the special-function unit, which lg2 keeps busy as well.
      auto p_pair = [&](float x0, float x1, bool emu) {
        const float2 sl = make_float2(copy_sign_bit(lg2_approx(fmaf(fabsf(x0), cb, 1.0f)), x0),
                                      copy_sign_bit(lg2_approx(fmaf(fabsf(x1), cb, 1.0f)), x1));
        const float2 t = __ffma2_rn(n2, sl, negm2);
        return emu ? exp2_poly2(t) : make_float2(ex2_approx(t.x), ex2_approx(t.y));
      };
      auto p_sl = [&](uint32_t s0, uint32_t s1, bool emu, bool v0 = true, bool v1 = true) {
        float2 t = __ffma2_rn(n2, make_float2(__uint_as_float(s0), __uint_as_float(s1)), negm2);
        t.x = v0 ? t.x : -INFINITY;  // ex2.approx(-inf) = +0
        t.y = v1 ? t.y : -INFINITY;
        return emu ? exp2_poly2(t) : make_float2(ex2_approx(t.x), ex2_approx(t.y));
      };
      auto p_of = [&](uint32_t s0, uint32_t s1, bool emu) {
        if constexpr (kLogFirst<D>)
          return p_sl(s0, s1, emu);
        else
          return p_pair(__uint_as_float(s0), __uint_as_float(s1), emu);
      };
      if constexpr (kLogFirst<D>) {
#pragma unroll
        for (int c = 0; c < C::BN / 32; ++c) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float x = __uint_as_float(sr[c][i]);
            sr[c][i] = __float_as_uint(copy_sign_bit(lg2_approx(fmaf(fabsf(x), cb, 1.0f)), x));
          }
        }
      }
      if (full) {  // no masking code in interior blocks
#pragma unroll
        for (int c = 0; c < C::BN / 32; ++c) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float2 pp = p_of(sr[c][i], sr[c][i + 1], ((i >> 1) & 3) < kEmuPairs<D>);
            rs2 = __fadd2_rn(rs2, pp);
            pk[c >> 1][(c & 1) * 16 + (i >> 1)] = pack2<BF16>(pp.x, pp.y);
          }
        }
      } else {
#pragma unroll
        for (int c = 0; c < C::BN / 32; ++c) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const int col = n0 + c * 32 + i;
            float2 pp;
            if constexpr (kLogFirst<D>) {
              pp = p_sl(sr[c][i], sr[c][i + 1], false, col <= lim && row < L,
                        col + 1 <= lim && row < L);
            } else {
              pp = p_pair(__uint_as_float(sr[c][i]), __uint_as_float(sr[c][i + 1]),
                          ((i >> 1) & 3) < kEmuPairs<D>);
              pp.x = (col <= lim && row < L) ? pp.x : 0.f;
              pp.y = (col + 1 <= lim && row < L) ? pp.y : 0.f;
            }
            rs2 = __fadd2_rn(rs2, pp);
            pk[c >> 1][(c & 1) * 16 + (i >> 1)] = pack2<BF16>(pp.x, pp.y);
          }
        }
      }
      const float rs = rs2.x + rs2.y;
      l_run = l_run * alpha + rs;
      // P_{j-1} V_{j-1} must have retired before O is corrected and before P_j overwrites
      // P_{j-1}; it was issued at the end of block j - 1, so this wait rarely blocks.
      if (j > 0) {
        bool okv = mbar_wait(bar(FB_O), (j - 1) & 1, a.status);
        if (!__all_sync(0xffffffffu, okv)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      // O correction: O is final for blocks < j here.
      if (__any_sync(0xffffffffu, need && j > 0)) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(t_lane + C::COL_O + c * 32, o);
          tmem_ld_wait(o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(t_lane + C::COL_O + c * 32, o);
        }
      }
#pragma unroll
      for (int c = 0; c < C::BN / 64; ++c) tmem_st32(t_lane + C::COL_P + c * 32, pk[c]);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar(FB_P));
    }
    if (ok) {
      ok = mbar_wait(bar(FB_O), (nblk - 1) & 1, a.status);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (!ok) {
      *abort_flag = 1;
    } else {
      tc_fence_after();
      const float l_safe = l_run > 0.f ? l_run : 1.f;
      const float inv_l = 1.f / l_safe;
      using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
      T* orow = reinterpret_cast<T*>(a.o.ptr) + row_offset(a.o, p, z, hq, seq_start, row);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(t_lane + C::COL_O + c * 32, o);
        tmem_ld_wait(o);
        // p.D is the tensors' head dim: 32 when a D = 32 problem runs this D = 64 kernel (its
        // TMA boxes zero-fill columns 32..63, so those O columns are zero and not stored).
        if (row < L && c * 32 < p.D) {
          if (p.drop_seed) {  // output dropout: dropped elements 0, kept ones scaled by 1/(1-p)
            const DropoutKey dk = dropout_key(p);
            const uint64_t e0 = dropout_index(p, z, hq, seq_start, row) + (uint64_t)(c * 32);
            const float ks = inv_l * p.drop_scale;
            uint32_t keep = 0;
#pragma unroll
            for (int g = 0; g < 8; ++g) keep |= dropout_keep4(dk, e0 + 4 * g) << (4 * g);
#pragma unroll
            for (int i = 0; i < 32; ++i)
              o[i] = __float_as_uint(((keep >> i) & 1u) ? __uint_as_float(o[i]) * ks : 0.f);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * inv_l);
          }
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = pack2<BF16>(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1]));
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
      if (row < L) a.lse[stat_offset(p, z, hq, seq_start, row)] = m_run + log2f(l_safe);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  // A wait of this CTA expired: its tile's out / lse rows are NaN, never partial results.
  if (*abort_flag) nan_fill_rows16<BF16>(a.o, p, z, hq, seq_start, m0, min(m0 + C::BM, L), a.lse);
}

template <int D, bool BF16>
int run_fwd(const Problem& p, TensorRef q, TensorRef k, TensorRef v, TensorRef o, float* lse,
            cudaStream_t st) {
  using C = FwdCfg<D>;
  const int dtype = BF16 ? SSA_DTYPE_BF16 : SSA_DTYPE_F16;
  CUtensorMap tq, tk, tv;
  int rc;
  if ((rc = make_tmap_bhnd(&tq, q, p, dtype, p.Hq, C::BM)) != SSA_OK) return rc;
  if ((rc = make_tmap_bhnd(&tk, k, p, dtype, p.Hkv, C::BN)) != SSA_OK) return rc;
  if ((rc = make_tmap_bhnd(&tv, v, p, dtype, p.Hkv, C::BN)) != SSA_OK) return rc;
  FwdArgs a;
  a.p = p;
  a.o = o;
  a.lse = lse;
  a.status = device_status_ptr();
  a.tiles_m = (p.max_seqlen + C::BM - 1) / C::BM;
  auto kern = fwd_sm100_kernel<D, BF16>;
  if (set_smem_limit_once(reinterpret_cast<const void*>(kern), (int)C::SMEM_BYTES) != SSA_OK)
    return SSA_ERR_CUDA;
  const long long grid = (long long)a.tiles_m * p.B * p.Hq;
  if (launch_pdl(kern, dim3((unsigned)grid), dim3(C::THREADS), C::SMEM_BYTES, st, tq, tk, tv, a) !=
      cudaSuccess)
    return SSA_ERR_LAUNCH;
  note_launches(1);
  return SSA_OK;
}

}  // namespace sm100

namespace sm100 {
// Waits on an mbarrier that no thread arrives on: the bounded wait expires after `cycles` and
// records the timeout in the status word, exactly as in the attention kernels.
__global__ void selftest_timeout_kernel(unsigned int* status, long long cycles) {
  __shared__ __align__(8) unsigned long long b;
  const uint32_t bar = smem_u32(&b);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(bar, 0, status, cycles);
}
}  // namespace sm100

int launch_selftest_timeout(unsigned int* status, long long cycles, cudaStream_t st) {
  if (cycles < 0) return SSA_ERR_BAD_SHAPE;
  sm100::selftest_timeout_kernel<<<1, 32, 0, st>>>(status, cycles);
  note_launches(1);
  return SSA_OK;
}

// Head dims with a tensor-core kernel. D = 32 runs the D = 64 kernels: their TMA boxes are 64
// elements wide, so a D = 32 tensor's boxes read zeros in columns 32..63 (out-of-bounds fill),
// which add nothing to S, O, dQ, dK or dV; the epilogues store the first p.D columns only. The
// MMAs then do twice the needed work, but at D = 64 the special-function work per score element,
// not the tensor pipe, bounds these kernels.
bool sm100_supports(int dtype, int D) {
  return (dtype == SSA_DTYPE_BF16 || dtype == SSA_DTYPE_F16) && (D == 32 || D == 64 || D == 128);
}

int launch_fwd_sm100(int dtype, const Problem& p, TensorRef q, TensorRef k, TensorRef v,
                     TensorRef o, float* lse, cudaStream_t st) {
  const bool bf = dtype == SSA_DTYPE_BF16;
  if (p.D == 64 || p.D == 32) return bf ? sm100::run_fwd<64, true>(p, q, k, v, o, lse, st)
                                         : sm100::run_fwd<64, false>(p, q, k, v, o, lse, st);
  if (p.D == 128) return bf ? sm100::run_fwd<128, true>(p, q, k, v, o, lse, st)
                            : sm100::run_fwd<128, false>(p, q, k, v, o, lse, st);
  return SSA_ERR_UNSUPPORTED;
}

}  // namespace ssa
