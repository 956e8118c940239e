// Residual (tail) + combine on the 5th-generation tensor cores (tcgen05, TMEM, TMA).
//
// Same mathematics as residual.cu (fast_article_attention.py:437-514 and the
// combine at :596-598): for query i in block c,
//   num_i = low_i + sum_{reps of blocks < c} w_r (exp(x) - P_t(x)) v_r
//                 + sum_{j in block c, j <= i} exp(x) v_j ,   x = scale q_i.k
// and den_i the same with v -> 1; out_i = num_i / max(den_i, eps).
//
// One CTA per (128-query tile, sequence).  Key material streams in tiles of
// 64 rows: first the coreset reps of the blocks before the tile, then the keys
// of the current block(s).  Roles:
//   warp 0      TMA producer: K_hi, K_lo, V_hi, V_lo (+ rep weights) per stage
//   warp 1      TMEM owner and MMA issuer: the converged warp runs the loop, an
//               elected lane issues every tcgen05.mma and commit
//   warps 2..17 query rows: four warps per TMEM lane quarter, one row per
//               thread, each warp of a quarter owning 16 of a tile's 64 columns
//               (more warps shorten the P step that each P V product waits for);
//               they write the scaled query into TMEM, turn each S tile into
//               P = f(S), then run the epilogue
// Precision: 3xTF32.  Every fp32 operand x is carried as hi = rna_tf32(x) and
// lo = x - hi, and each product uses hi*hi + hi*lo + lo*hi, which keeps the
// result within a few fp32 ulps (a single TF32 product loses ~11 bits).
// Q (hi/lo) lives in TMEM as the A operand of S = Q K^T; P (hi/lo) is written
// back to TMEM in place of S and is the A operand of O += P V.  Both B operands
// are K-major with the 128-byte swizzle, written by TMA: K tiles from the
// row-major k split, V tiles from the transposed v split (an MN-major tf32
// operand runs markedly slower on the tensor cores).
//
// Each 8-wide K step forms the three products hi*hi + hi*lo + lo*hi (not the
// unneeded lo*lo: a tf32 MMA's time grows with N) in two MMAs, one of them
// twice as wide:
//   S' = Q_hi [K_hi ; K_lo]^T (N = 128: each 32-column K chunk holds the 64 hi
//        rows, then the 64 lo rows) + Q_lo K_hi^T into its first 64 columns;
//        S = S'[0, 64) + S'[64, 128), added by the query-row warps (for d <= 32,
//        whose S is only four K steps, three MMAs of N = 64: there the extra
//        TMEM load and adds of the query-row warps cost more than the issues
//        saved -- config 4's residual measured 18.4 against 17.2 ms)
//   O' = P_hi [V_hi | V_lo] (N = 2 dv: each 32-key chunk of the V^T tile holds
//        the dv hi rows, then the dv lo rows) + P_lo V_hi into its first dv
//        columns; O = O'[0, dv) + O'[dv, 2 dv), added in the epilogue
//        (for dv > 64, where O' would not fit in TMEM, three MMAs of N = dv)
// The tensor time is that of three MMAs of N = 64, and the MMA warp issues a
// third fewer instructions (it shares its scheduler with four query-row
// warps).  Measured with clock64 stamps in every CTA at config 3: the issuing
// of a tile's products took ~1900 cycles in the three-MMA form and ~1800 in
// this one, against 1536 of tensor work -- the issuing thread waits on a full
// tensor pipe queue -- and the main loop per 64-key tile went from ~2620 to
// ~2560 cycles; the rest is waiting for the K/V ring (~290 per tile) and for
// P (~160-260).
#include <math.h>

#include "sa_common.cuh"
#include "tc_util.cuh"

namespace sa {

namespace {

using namespace tc;

constexpr int kRowsQ = 128;    // queries per CTA = UMMA M
constexpr int kTile = 64;      // keys per tile = N of S = K of PV
constexpr int kQW = 4;          // query-row warps per TMEM lane quarter (column groups)
constexpr int kCW = kTile / kQW;        // columns of a key tile one query-row warp handles (16)
constexpr int kQueryWarps = 4 * kQW;    // 16
constexpr int kQueryThreads = 32 * kQueryWarps;
constexpr int kThreads = 64 + kQueryThreads;   // warp 0 TMA, warp 1 MMA, warps 2.. query rows

// status codes written to the launch's status word
constexpr int kErrWaitQ = 101, kErrWaitFull = 102, kErrWaitP = 104, kErrWaitS = 105,
              kErrWaitEmpty = 106, kErrWaitO = 107, kErrDrain = 108;

struct ResTCParams {
  const float* q;        // [bh, n, d] raw queries
  const float* rep_w;    // [bh, r_pad] rep weights (nullptr: every weight is 1)
  const float* low;      // [groups, bh, n, dv+1] partial low sums (summed here)
  float* out;            // [bh, n, dv]
  int* status;           // launch status word (0 = ok)
  int64_t n;
  int64_t m_blk;         // reps per completed block
  int64_t r_pad;         // per-sequence stride of rep_w
  int d, dv, bs;
  float scale, eps;
  int groups;            // partial slices in `low`
  int64_t group_stride;  // floats between slices (bh * n * (dv+1))
  int64_t c_off;         // global index of the sequence's first block (a shard of a longer sequence:
                         // rep rows and each query's active reps count from global block 0)
  uint64_t wait_ns;      // limit of one bounded wait
};

template <int DP, int DVP>
struct Layout {
  static constexpr uint32_t kKT = DP * kTile * 4;   // one K tile (hi or lo); chunk a: hi rows at
                                                    // a * 2 * kTile * 128, lo rows 64 rows further
  static constexpr uint32_t kVT = DVP * kTile * 4;  // one V tile (hi or lo); 32-key chunk a: hi rows at
                                                    // a * 2 * DVP * 128, lo rows DVP rows further
  static constexpr uint32_t kStage = 2 * kKT + 2 * kVT;
  static constexpr int kStages = (200u * 1024u / kStage) >= 4 ? 4 : (int)(200u * 1024u / kStage);
  static_assert(kStages >= 2, "at least double buffering");
  static constexpr uint32_t kW = kStages * kTile * 4;
  // TMEM columns
  static constexpr uint32_t kQhi = 0, kQlo = DP;
  static constexpr uint32_t kS0 = 2 * DP;           // buffer b: S (or S', 128 columns) at kS0 + 128 b, then
                                                    // P_hi over its first 64 columns and P_lo over the other 64
  static constexpr uint32_t kO = 2 * DP + 256;
  static constexpr bool kStackK = DP == 64;                 // S' = [S_hh + S_lh | S_hl]
  static constexpr bool kStackV = DVP <= 64;                // O' = [O_hh + O_lh | O_hl]
  static constexpr uint32_t kOCols = kStackV ? 2 * DVP : DVP;
  static_assert(kO + kOCols <= 512, "TMEM columns");
  static constexpr uint32_t kSmemBytes = kStages * kStage + kW + (2 * kStages + 11) * 8 + 64 + kQW * 128 * 4 + 1024;
};

template <int DEG>
__device__ __forceinline__ float taylor_t(float x) {
  // the reference's term recurrence (fast_article_attention.py:95-104)
  float out = 1.0f;
  if (DEG >= 1) {
    float term = x;
    out = out + term;
    if (DEG >= 2) {
      term = term * x * 0.5f;
      out = out + term;
      if (DEG >= 3) {
        term = __fdiv_rn(term * x, 3.0f);
        out = out + term;
      }
    }
  }
  return out;
}

// P_t(x) in Horner form with fused multiply-adds (within a rounding or two
// of the reference's term recurrence).
template <int DEG>
__device__ __forceinline__ float taylor_fma(float x) {
  if (DEG == 0) return 1.0f;
  if (DEG == 1) return 1.0f + x;
  if (DEG == 2) return fmaf(fmaf(x, 0.5f, 1.0f), x, 1.0f);
  return fmaf(fmaf(fmaf(x, 1.0f / 6.0f, 0.5f), x, 1.0f), x, 1.0f);
}

// exp of a score; CLAMP caps its argument at 80 (the segment-mean variant,
// triton_article_attention.py:331-333 and :359, keeps e^x finite in fp32 there)
template <bool CLAMP>
__device__ __forceinline__ float exp_score(float x) {
  return __expf(CLAMP ? fminf(x, 80.0f) : x);
}

// P = w (e^x - P_t(x)) over NC rep scores, split hi / lo; MASK zeroes j > jhi;
// w = nullptr for unit weights.
template <bool MASK, int DEG, bool CLAMP, int NC>
__device__ __forceinline__ void rep_to_p(const float (&sv)[NC], const float* w, int jhi, float& den,
                                         uint32_t (&hi)[NC], uint32_t (&lo)[NC]) {
#pragma unroll
  for (int j4 = 0; j4 < NC / 4; ++j4) {
    float ww[4] = {1.0f, 1.0f, 1.0f, 1.0f};
    if (w) {
      const float4 w4 = reinterpret_cast<const float4*>(w)[j4];
      ww[0] = w4.x; ww[1] = w4.y; ww[2] = w4.z; ww[3] = w4.w;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = 4 * j4 + u;
      const float x = sv[j];
      float e = exp_score<CLAMP>(x) - taylor_fma<DEG>(x);
      if (w) e *= ww[u];
      if (MASK && j > jhi) e = 0.0f;
      den += e;
      hi[j] = to_tf32(e);
      lo[j] = __float_as_uint(e - __uint_as_float(hi[j]));
    }
  }
}

// P = e^x over NC current-block scores; MASK keeps jlo <= j <= jhi only.
template <bool MASK, bool CLAMP, int NC>
__device__ __forceinline__ void cur_to_p(const float (&sv)[NC], int jlo, int jhi, float& den, uint32_t (&hi)[NC],
                                         uint32_t (&lo)[NC]) {
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    float e = exp_score<CLAMP>(sv[j]);
    if (MASK && (j < jlo || j > jhi)) e = 0.0f;
    den += e;
    hi[j] = to_tf32(e);
    lo[j] = __float_as_uint(e - __uint_as_float(hi[j]));
  }
}

template <int DP, int DVP, int DEG, bool CLAMP>
__global__ void __launch_bounds__(kThreads, 1)
residual_tc_kernel(const __grid_constant__ CUtensorMap tm_rkh, const __grid_constant__ CUtensorMap tm_rkl,
                   const __grid_constant__ CUtensorMap tm_rvh, const __grid_constant__ CUtensorMap tm_rvl,
                   const __grid_constant__ CUtensorMap tm_kh, const __grid_constant__ CUtensorMap tm_kl,
                   const __grid_constant__ CUtensorMap tm_vh, const __grid_constant__ CUtensorMap tm_vl,
                   const ResTCParams p) {
  using L = Layout<DP, DVP>;
  constexpr int kStages = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* wbuf = reinterpret_cast<float*>(smem + kStages * L::kStage);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * L::kStage + L::kW);
  uint64_t* full = bars;                 // [kStages]
  uint64_t* empty = bars + kStages;      // [kStages]
  uint64_t* sfull = bars + 2 * kStages;  // [2]
  uint64_t* pfull = sfull + 2;           // [2]
  uint64_t* qready = pfull + 2;
  uint64_t* ofull = qready + 1;
  uint64_t* drain = ofull + 1;
  uint64_t* lowfull = drain + 1;          // the epilogue's low-sum rows, bulk-copied into the stages
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(lowfull + 1);
  int* abort_word = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t h = blockIdx.y;
  // heavy query tiles (late in the sequence) first
  const int64_t n_qt = (p.n + kRowsQ - 1) / kRowsQ;
  const int64_t qt = n_qt - 1 - blockIdx.x;
  const int64_t q0 = qt * kRowsQ;
  const int64_t q_last = min(q0 + kRowsQ, p.n) - 1;
  const int64_t c_first = q0 / p.bs, c_last = q_last / p.bs;
  const int64_t r_end = (p.c_off + c_last) * p.m_blk;
  const int n_rep = (int)((r_end + kTile - 1) / kTile);
  const int64_t kb0 = c_first * p.bs;
  const int n_cur = (int)((q_last + 1 - kb0 + kTile - 1) / kTile);
  const int T = n_rep + n_cur;
  // Epilogue input: this CTA's rows of the `groups` low slices.  When they fit in
  // the stage buffers (free once O is complete) next to the O staging, and every
  // row block is 16-byte aligned, the producer bulk-copies them into shared
  // memory as soon as O is complete.
  const int64_t erows = min((int64_t)kRowsQ, p.n - q0);
  const int64_t lblk = erows * (int64_t)(p.dv + 1);          // floats of one slice's row block
  const uint64_t lbytes = (uint64_t)p.groups * (uint64_t)lblk * 4u;
  const uint64_t lbytes16 = (lbytes + 15) & ~uint64_t(15);
  const bool bulk_low = (lblk * 4) % 16 == 0 && (p.group_stride * 4) % 16 == 0 &&
                        ((reinterpret_cast<uintptr_t>(p.low) + (uintptr_t)((h * p.n + q0) * (int64_t)(p.dv + 1) * 4)) & 15) == 0 &&
                        lbytes16 + (uint64_t)kRowsQ * (DVP + 1) * 4 + (uint64_t)kRowsQ * 4 <= (uint64_t)kStages * L::kStage;

  // Query-row threads start loading their piece of the query row now, so that
  // the loads' latency overlaps the set-up below: 16-byte loads when the rows
  // allow them (a warp's load then touches 32 rows once, not once per float).
  float qv[16];
  if (warp >= 2) {
    const int u = (warp - 2) >> 2;                 // the column group's 16-column piece
    const int64_t iq = q0 + (warp & 3) * 32 + lane;
    const bool vq = iq < p.n && u < DP / 16;
    const float* qr = p.q + (h * p.n + (vq ? iq : 0)) * p.d + u * 16;
    if (vq && (p.d & 3) == 0 && u * 16 + 16 <= p.d && (reinterpret_cast<uintptr_t>(p.q) & 15) == 0) {
#pragma unroll
      for (int j4 = 0; j4 < 4; ++j4) {
        const float4 x = __ldg(reinterpret_cast<const float4*>(qr) + j4);
        qv[4 * j4 + 0] = x.x;
        qv[4 * j4 + 1] = x.y;
        qv[4 * j4 + 2] = x.z;
        qv[4 * j4 + 3] = x.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) qv[j] = (vq && u * 16 + j < p.d) ? __ldg(qr + j) : 0.0f;
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sfull[b], 1);
      mbar_init(&pfull[b], kQueryWarps);   // one arrival per query-row warp
    }
    mbar_init(qready, kQueryWarps);
    mbar_init(ofull, 1);
    mbar_init(drain, 1);
    mbar_init(lowfull, 1);
    *abort_word = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const Abort ab{abort_word, p.status, p.wait_ns};

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_rkh);
      tma_prefetch_desc(&tm_kh);
      // The epilogue reads this CTA's rows of every low slice, written long ago
      // by the moment kernel: start moving them into L2 now, under the main loop.
      if ((reinterpret_cast<uintptr_t>(p.low) & 15) == 0) {
        const uintptr_t base = reinterpret_cast<uintptr_t>(p.low);
        const uintptr_t end = base + (uintptr_t)p.groups * (uintptr_t)p.group_stride * 4u;
        const int64_t rows = min((int64_t)kRowsQ, p.n - q0);
        for (int gi = 0; gi < p.groups; ++gi) {
          const uintptr_t a0 =
              (base + (uintptr_t)(((h * p.n + q0) * (int64_t)(p.dv + 1) + gi * p.group_stride) * 4)) & ~uintptr_t(15);
          uintptr_t a1 = (a0 + (uintptr_t)(rows * (p.dv + 1) * 4) + 31) & ~uintptr_t(15);
          if (a1 > (end & ~uintptr_t(15))) a1 = end & ~uintptr_t(15);
          if (a1 > a0) bulk_prefetch_l2(reinterpret_cast<const void*>(a0), (uint32_t)(a1 - a0));
        }
      }
      int issued = 0;
      for (int t = 0; t < T; ++t) {
        const int s = t % kStages;
        if (t >= kStages && !mbar_wait(&empty[s], ((t / kStages) - 1) & 1, ab, kErrWaitEmpty)) break;
        const bool rep = t < n_rep;
        const int row0 = rep ? t * kTile : (int)(kb0 + (int64_t)(t - n_rep) * kTile);
        const bool with_w = rep && p.rep_w != nullptr;
        mbar_arrive_expect_tx(&full[s], L::kStage + (with_w ? kTile * 4 : 0));
        uint8_t* st = smem + s * L::kStage;
        const CUtensorMap* mkh = rep ? &tm_rkh : &tm_kh;
        const CUtensorMap* mkl = rep ? &tm_rkl : &tm_kl;
        const CUtensorMap* mvh = rep ? &tm_rvh : &tm_vh;
        const CUtensorMap* mvl = rep ? &tm_rvl : &tm_vl;
#pragma unroll
        for (int a = 0; a < DP / 32; ++a) {
          tma_load_3d(st + a * (2 * kTile * 128), mkh, &full[s], a * 32, row0, (int)h);
          tma_load_3d(st + a * (2 * kTile * 128) + kTile * 128, mkl, &full[s], a * 32, row0, (int)h);
        }
#pragma unroll
        for (int a = 0; a < kTile / 32; ++a) {
          uint8_t* vd = st + 2 * L::kKT + a * (2 * DVP * 128);
          tma_load_3d(vd, mvh, &full[s], row0 + a * 32, 0, (int)h);
          tma_load_3d(vd + DVP * 128, mvl, &full[s], row0 + a * 32, 0, (int)h);
        }
        // (a bulk copy has no bounds of its own: the weight rows must lie in the sequence's stride)
        if (with_w && SA_DEVICE_CHECK(row0 >= 0 && row0 + kTile <= p.r_pad, p.status, 921, row0))
          bulk_load(wbuf + s * kTile, p.rep_w + h * p.r_pad + row0, kTile * 4, &full[s]);
        ++issued;
      }
      // never leave with copies in flight: the last use of each stage must have landed
      for (int t = max(0, issued - kStages); t < issued; ++t) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&full[t % kStages], (t / kStages) & 1)) {
          if (globaltimer_ns() - t0 > 1000000000ull) {
            atomicCAS(p.status, 0, kErrDrain);
            break;
          }
        }
      }
      // once O is complete nothing reads the stages: bring in the epilogue's rows
      if (bulk_low && issued == T && mbar_wait(ofull, 0, ab, kErrWaitO)) {
        mbar_arrive_expect_tx(lowfull, (uint32_t)lbytes);
        for (int gi = 0; gi < p.groups; ++gi) {
          const int64_t e0 = (h * p.n + q0) * (int64_t)(p.dv + 1) + gi * p.group_stride;
          if (SA_DEVICE_CHECK(e0 >= 0 && e0 + lblk <= (gi + 1) * p.group_stride, p.status, 922, e0))
            bulk_load(reinterpret_cast<float*>(smem) + gi * lblk, p.low + e0, (uint32_t)(lblk * 4), lowfull);
        }
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(lowfull, 0)) {   // and never leave with them in flight
          if (globaltimer_ns() - t0 > 1000000000ull) {
            atomicCAS(p.status, 0, kErrDrain);
            break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // the whole warp runs the loop; the elected lane issues MMAs and commits
    {
      constexpr uint32_t idesc_qk2 = idesc_tf32(128, 2 * kTile, false, false);
      constexpr uint32_t idesc_qk = idesc_tf32(128, kTile, false, false);
      constexpr uint32_t idesc_pv2 = idesc_tf32(128, 2 * DVP, false, false);
      constexpr uint32_t idesc_pv = idesc_tf32(128, DVP, false, false);
      bool ok = mbar_wait_warp(qready, 0, ab, kErrWaitQ);
      if (ok) tc_fence_after();
      auto issue_pv = [&](int tp) -> bool {
        const int sp = tp % kStages, bp = tp & 1;
        if (!mbar_wait_warp(&pfull[bp], (tp >> 1) & 1, ab, kErrWaitP)) return false;
        tc_fence_after();
        const uint32_t vt = smem_u32(smem + sp * L::kStage + 2 * L::kKT);
        const uint32_t ph = tmem + L::kS0 + 128 * bp;
        const uint32_t pl = ph + 64;
        // one elected lane issues the tile's MMAs and commits back to back; the
        // descriptors' start address field (address >> 4) is advanced in place
        if (elect_one()) {
          const uint64_t vd = sdesc_sw128(vt, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < kTile / 8; ++kk) {
            // 8 keys of 32-key chunk kk / 4: rows = value columns (hi rows, then lo rows)
            const uint64_t bh_ = vd + (uint64_t)(((kk >> 2) * (2 * DVP * 128) + (kk & 3) * 32) >> 4);
            if (L::kStackV) {
              // [V_hi | V_lo] are the chunk's 2 dv rows from bh_ on
              mma_tf32_ts(tmem + L::kO, ph + kk * 8, bh_, idesc_pv2, (tp > 0 || kk > 0) ? 1u : 0u);
              mma_tf32_ts(tmem + L::kO, pl + kk * 8, bh_, idesc_pv, 1u);
            } else {
              const uint64_t bl_ = bh_ + (uint64_t)((DVP * 128) >> 4);
              mma_tf32_ts(tmem + L::kO, ph + kk * 8, bh_, idesc_pv, (tp > 0 || kk > 0) ? 1u : 0u);
              mma_tf32_ts(tmem + L::kO, ph + kk * 8, bl_, idesc_pv, 1u);
              mma_tf32_ts(tmem + L::kO, pl + kk * 8, bh_, idesc_pv, 1u);
            }
          }
          mma_commit(&empty[sp]);
        }
        __syncwarp();
        return true;
      };
      for (int t = 0; ok && t < T; ++t) {
        const int s = t % kStages, b = t & 1;
        if (!mbar_wait_warp(&full[s], (t / kStages) & 1, ab, kErrWaitFull)) { ok = false; break; }
        // S(t) reuses the TMEM columns that PV(t-2) reads as its A operand.  No wait:
        // tcgen05.mma operations issued by one thread execute in issue order (mma
        // after mma is an implicitly pipelined pair), and PV(t-2) was issued first.
        tc_fence_after();
        const uint32_t kh = smem_u32(smem + s * L::kStage);
        const uint32_t dS = tmem + L::kS0 + 128 * b;
        if (elect_one()) {
          const uint64_t kd = sdesc_sw128(kh, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < DP / 8; ++kk) {
            // N = 128 rows: the chunk's 64 hi rows, then its 64 lo rows
            const uint64_t bk = kd + (uint64_t)(((kk >> 2) * (2 * kTile * 128) + (kk & 3) * 32) >> 4);
            if (L::kStackK) {
              mma_tf32_ts(dS, tmem + L::kQhi + kk * 8, bk, idesc_qk2, kk > 0 ? 1u : 0u);
              mma_tf32_ts(dS, tmem + L::kQlo + kk * 8, bk, idesc_qk, 1u);
            } else {
              // K_lo rows 64 rows (8 KB) after the chunk's K_hi rows
              const uint64_t bkl = bk + (uint64_t)((kTile * 128) >> 4);
              mma_tf32_ts(dS, tmem + L::kQhi + kk * 8, bk, idesc_qk, kk > 0 ? 1u : 0u);
              mma_tf32_ts(dS, tmem + L::kQhi + kk * 8, bkl, idesc_qk, 1u);
              mma_tf32_ts(dS, tmem + L::kQlo + kk * 8, bk, idesc_qk, 1u);
            }
          }
          mma_commit(&sfull[b]);
        }
        __syncwarp();
        if (t >= 1 && !issue_pv(t - 1)) { ok = false; break; }
      }
      if (ok && T > 0) ok = issue_pv(T - 1);
      if (ok && elect_one()) mma_commit(ofull);
      // drain: nothing of ours may still write TMEM when it is freed
      if (elect_one()) mma_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0)) {
        if (globaltimer_ns() - t0 > 2000000000ull) {
          atomicCAS(p.status, 0, kErrDrain);
          break;
        }
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ query rows
    // four warps per TMEM lane quarter: column group `cgp` (warps 2 + 4 cgp ..
    // 5 + 4 cgp) owns columns [16 cgp, 16 cgp + 16) of every tile
    const int quarter = warp & 3;
    const int cgp = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int64_t i = q0 + row;
    const bool valid = i < p.n;
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    // scaled query, split hi/lo, into TMEM (16-column pieces: column group cgp
    // writes piece cgp, loaded into qv at the start)
    {
      static_assert(DP / 16 <= kQW, "one query piece per column group");
      if (cgp < DP / 16) {
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float x = qv[j] * p.scale;
          hi[j] = to_tf32(x);
          lo[j] = __float_as_uint(x - __uint_as_float(hi[j]));
        }
        tmem_st16(lane_addr + L::kQhi + cgp * 16, hi);
        tmem_st16(lane_addr + L::kQlo + cgp * 16, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(qready);
    }
    const int64_t ci = valid ? i / p.bs : 0;
    const int64_t lim = valid ? (p.c_off + ci) * p.m_blk : 0;    // reps r < lim are active for this query
    const int64_t bst = valid ? ci * p.bs : p.n;      // first key of this query's block
    float den = 0.0f;
    bool ok = true;
    for (int t = 0; t < T; ++t) {
      const int s = t % kStages, b = t & 1;
      // warp-uniform verdicts: the TMEM loads and stores below are .sync.aligned
      if (!mbar_wait_warp(&sfull[b], (t >> 1) & 1, ab, kErrWaitS)) { ok = false; break; }
      const bool rep = t < n_rep;
      const bool with_w = rep && p.rep_w != nullptr;
      if (with_w && !mbar_wait_warp(&full[s], (t / kStages) & 1, ab, kErrWaitFull)) { ok = false; break; }
      tc_fence_after();
      const uint32_t tS = lane_addr + L::kS0 + 128 * b + cgp * kCW;
      const int64_t row0 = rep ? (int64_t)t * kTile : kb0 + (int64_t)(t - n_rep) * kTile;
      const int64_t col0 = row0 + cgp * kCW;
      float sv[kCW];
      if (L::kStackK) {
        float sl[kCW];
        tmem_ld16(tS, sv);
        tmem_ld16(tS + kTile, sl);   // the Q_hi K_lo^T half
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < kCW; ++j) sv[j] += sl[j];
      } else {
        tmem_ld16(tS, sv);
        tmem_wait_ld();
      }
      uint32_t hi[kCW], lo[kCW];
      if (rep) {
        // reps col0 + j with j <= jhi are active (r < lim)
        const int64_t rel = lim - 1 - col0;
        const int jhi = rel < 0 ? -1 : (rel > kCW - 1 ? kCW - 1 : (int)rel);
        const float* w = with_w ? wbuf + s * kTile + cgp * kCW : nullptr;
        if (jhi == kCW - 1)
          rep_to_p<false, DEG, CLAMP, kCW>(sv, w, jhi, den, hi, lo);
        else
          rep_to_p<true, DEG, CLAMP, kCW>(sv, w, jhi, den, hi, lo);
      } else {
        // keys col0 + j of the query's own block up to the query: jlo <= j <= jhi
        const int64_t rlo = bst - col0, rhi = i - col0;
        const int jlo = rlo < 0 ? 0 : (rlo > kCW ? kCW : (int)rlo);
        const int jhi = !valid || rhi < 0 ? -1 : (rhi > kCW - 1 ? kCW - 1 : (int)rhi);
        if (jlo == 0 && jhi == kCW - 1)
          cur_to_p<false, CLAMP, kCW>(sv, jlo, jhi, den, hi, lo);
        else
          cur_to_p<true, CLAMP, kCW>(sv, jlo, jhi, den, hi, lo);
      }
      tmem_st16(tS, hi);
      tmem_st16(tS + 64, lo);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfull[b]);
    }
    // the column groups' denominators, added in group order
    float* den_x = reinterpret_cast<float*>(abort_word + 1);   // [kQW][128]
    den_x[cgp * 128 + row] = den;
    asm volatile("bar.sync 1, %0;" ::"n"(kQueryThreads) : "memory");
    float den_all = den_x[row];
#pragma unroll
    for (int g2 = 1; g2 < kQW; ++g2) den_all += den_x[g2 * 128 + row];
    // Epilogue.  The output rows and the moment kernel's `groups` partial
    // slices of the low term are read and written coalesced: each thread first
    // puts its row's O columns (and the row's divisor) into shared memory, over
    // the stage buffers, which no copy or product touches any more once O is
    // complete; then each warp takes whole rows, lanes on consecutive columns.
    const bool o_ok = ok && mbar_wait_warp(ofull, 0, ab, kErrWaitO);
    constexpr int OS = DVP + 1;                                  // odd row stride: conflict-free
    float* os = reinterpret_cast<float*>(smem + (bulk_low ? lbytes16 : 0));   // [128][DVP + 1]
    float* dms = os + kRowsQ * OS;                               // [128] max(den, eps)
    if (o_ok) {
      tc_fence_after();
      if (cgp == 0) {
        const float* lrow = p.low + (h * p.n + (valid ? i : 0)) * (int64_t)(p.dv + 1);
        float ldsum = 0.0f;
        for (int gi = 0; gi < p.groups; ++gi) ldsum += valid ? __ldg(lrow + gi * p.group_stride + p.dv) : 0.0f;
        const float dtot = valid ? ldsum + den_all : 1.0f;
        dms[row] = fmaxf(dtot, p.eps);
      }
#pragma unroll
      for (int u = 0; u < DVP / 16; ++u) {
        if (u % kQW != cgp) continue;
        float ov[16];
        tmem_ld16(lane_addr + L::kO + u * 16, ov);
        if (L::kStackV) {
          float o2[16];   // the P_hi V_lo half
          tmem_ld16(lane_addr + L::kO + DVP + u * 16, o2);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) ov[j] += o2[j];
        } else {
          tmem_wait_ld();
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) os[row * OS + u * 16 + j] = ov[j];
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kQueryThreads) : "memory");
    if (o_ok && bulk_low) {
      // The rows arrive by bulk copy: every read below is from shared memory.
      // Four rows per pass (rows r, r+16, r+32, r+48 of this warp), the slices'
      // loads of a pass independent of each other, so their latencies overlap
      // instead of forming one chain per element.
      if (mbar_wait_warp(lowfull, 0, ab, kErrWaitO)) {
        constexpr int kRP = 4, kNC = DVP / 32;
        const float* lb = reinterpret_cast<const float*>(smem);
        const int ls = p.dv + 1;
        const int nrows = (int)erows;
        for (int r0 = warp - 2; r0 < nrows; r0 += kQueryWarps * kRP) {
          float lv[kRP][kNC];
#pragma unroll
          for (int a = 0; a < kRP; ++a)
#pragma unroll
            for (int c = 0; c < kNC; ++c) lv[a][c] = 0.0f;
          for (int gi = 0; gi < p.groups; ++gi) {
#pragma unroll
            for (int a = 0; a < kRP; ++a) {
              const int r = r0 + kQueryWarps * a;
              const float* lr = lb + gi * lblk + (r < nrows ? r : 0) * ls;
#pragma unroll
              for (int c = 0; c < kNC; ++c) {
                const int col = c * 32 + lane;
                if (col < p.dv) lv[a][c] += lr[col];
              }
            }
          }
#pragma unroll
          for (int a = 0; a < kRP; ++a) {
            const int r = r0 + kQueryWarps * a;
            if (r >= nrows) continue;
            float* orow = p.out + (h * p.n + q0 + r) * (int64_t)p.dv;
            const float dm = dms[r];
#pragma unroll
            for (int c = 0; c < kNC; ++c) {
              const int col = c * 32 + lane;
              if (col < p.dv) orow[col] = __fdiv_rn(os[r * OS + col] + lv[a][c], dm);
            }
          }
        }
      }
    } else if (o_ok) {
      // Four rows per pass (rows r, r+16, r+32, r+48 of this warp), every load of
      // the pass issued before any store: the loads of a row do not wait for the
      // stores of the row before (the output and the slices never overlap).
      constexpr int kRP = 4, kNC = DVP / 32;
      const float* __restrict__ lowp = p.low;
      float* __restrict__ outp = p.out;
      const int nrows = (int)min((int64_t)kRowsQ, p.n - q0);
      const int64_t ls = p.dv + 1;
      for (int r0 = warp - 2; r0 < nrows; r0 += kQueryWarps * kRP) {
        float lv[kRP][kNC];
#pragma unroll
        for (int a = 0; a < kRP; ++a)
#pragma unroll
          for (int c = 0; c < kNC; ++c) lv[a][c] = 0.0f;
        for (int gi = 0; gi < p.groups; ++gi) {
#pragma unroll
          for (int a = 0; a < kRP; ++a) {
            const int r = r0 + kQueryWarps * a;
            const float* lr = lowp + (h * p.n + q0 + (r < nrows ? r : 0)) * ls + gi * p.group_stride;
#pragma unroll
            for (int c = 0; c < kNC; ++c) {
              const int col = c * 32 + lane;
              if (r < nrows && col < p.dv) lv[a][c] += __ldg(lr + col);
            }
          }
        }
#pragma unroll
        for (int a = 0; a < kRP; ++a) {
          const int r = r0 + kQueryWarps * a;
          if (r >= nrows) continue;
          float* orow = outp + (h * p.n + q0 + r) * (int64_t)p.dv;
          const float dm = dms[r];
#pragma unroll
          for (int c = 0; c < kNC; ++c) {
            const int col = c * 32 + lane;
            if (col < p.dv) orow[col] = __fdiv_rn(os[r * OS + col] + lv[a][c], dm);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int DP, int DVP, int DEG, bool CLAMP = false>
int launch_tc(const CUtensorMap* maps, const ResTCParams& prm, int64_t bh, cudaStream_t stream) {
  using L = Layout<DP, DVP>;
  auto kern = residual_tc_kernel<DP, DVP, DEG, CLAMP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kSmemBytes);
  if (e != cudaSuccess) return set_error(SA_ERR_CUDA, "residual_tc smem attribute: %s", cudaGetErrorString(e));
  dim3 grid((unsigned)((prm.n + kRowsQ - 1) / kRowsQ), (unsigned)bh);
  kern<<<grid, kThreads, L::kSmemBytes, stream>>>(maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], maps[6],
                                                  maps[7], prm);
  return check_launch("residual_tc_kernel");
}

template <int DP, int DVP>
int launch_deg(int degree, const CUtensorMap* maps, const ResTCParams& prm, int64_t bh, cudaStream_t s,
               bool clamp_exp) {
  if (clamp_exp) {  // the segment-mean variant: degree 0, 1 or 2
    switch (degree) {
      case 0: return launch_tc<DP, DVP, 0, true>(maps, prm, bh, s);
      case 1: return launch_tc<DP, DVP, 1, true>(maps, prm, bh, s);
      case 2: return launch_tc<DP, DVP, 2, true>(maps, prm, bh, s);
      default: return set_error(SA_ERR_UNSUPPORTED, "the clamped residual supports degree 0, 1 or 2");
    }
  }
  switch (degree) {
    case 0: return launch_tc<DP, DVP, 0>(maps, prm, bh, s);
    case 1: return launch_tc<DP, DVP, 1>(maps, prm, bh, s);
    case 2: return launch_tc<DP, DVP, 2>(maps, prm, bh, s);
    default: return launch_tc<DP, DVP, 3>(maps, prm, bh, s);
  }
}

}  // namespace

// Padded widths the tensor-core residual uses (0 if the shape is not supported).
int residual_tc_dp(int d) { return d <= 32 ? 32 : (d <= 64 ? 64 : 0); }
int residual_tc_dvp(int dv) { return dv <= 32 ? 32 : (dv <= 64 ? 64 : (dv <= 128 ? 128 : 0)); }

// maps: rep_k_hi, rep_k_lo, rep_v_hi, rep_v_lo, k_hi, k_lo, v_hi, v_lo (3-D, box {32, 64, 1}).
int launch_residual_tc(const CUtensorMap* maps, const float* q, const float* rep_w, int64_t r_pad, const float* low,
                       int groups, float* out, int* status, int64_t bh, int64_t n, int d, int dv, int degree, int bs,
                       int64_t m_blk, float scale, float eps, cudaStream_t stream, int64_t c_off,
                       bool clamp_exp) {
  if (bh == 0 || n == 0) return SA_OK;
  if (bh > 65535 || (n + kRowsQ - 1) / kRowsQ > 2147483647LL)
    return set_error(SA_ERR_UNSUPPORTED, "grid too large for the tensor-core residual");
  ResTCParams prm{q, rep_w, low, out, status, n, m_blk, r_pad, d, dv, bs, scale, eps, groups, bh * n * (dv + 1),
                  c_off, wait_limit_ns()};
  const int dp = residual_tc_dp(d), dvp = residual_tc_dvp(dv);
  if (dp == 32 && dvp == 32) return launch_deg<32, 32>(degree, maps, prm, bh, stream, clamp_exp);
  if (dp == 32 && dvp == 64) return launch_deg<32, 64>(degree, maps, prm, bh, stream, clamp_exp);
  if (dp == 32 && dvp == 128) return launch_deg<32, 128>(degree, maps, prm, bh, stream, clamp_exp);
  if (dp == 64 && dvp == 32) return launch_deg<64, 32>(degree, maps, prm, bh, stream, clamp_exp);
  if (dp == 64 && dvp == 64) return launch_deg<64, 64>(degree, maps, prm, bh, stream, clamp_exp);
  if (dp == 64 && dvp == 128) return launch_deg<64, 128>(degree, maps, prm, bh, stream, clamp_exp);
  return set_error(SA_ERR_UNSUPPORTED, "tensor-core residual: d=%d dv=%d not supported", d, dv);
}

}  // namespace sa
