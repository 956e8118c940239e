// Exact causal softmax attention on the 5th-generation tensor cores (tcgen05,
// TMEM, TMA): the comparator and large-N check of the approximate paths
// (the exact baseline of triton_article_attention.py:372-435 / :580-637).
//
//   out_i = sum_{j <= i} exp(x_ij - m_i) v_j / max(sum_{j <= i} exp(x_ij - m_i), 1e-20),
//   x_ij = scale q_i.k_j
//
// One CTA per (128-query tile, sequence); keys stream in tiles of 64 from key 0
// to the tile's last query.  Roles as in the residual kernel: warp 0 TMA
// producer (K_hi, K_lo, V_hi, V_lo per stage), warp 1 TMEM owner and MMA
// issuer (converged warp, elected lane), warps 2..9 two per TMEM lane quarter,
// one query row per thread, each warp of a pair owning 32 of a tile's 64
// columns.  3xTF32 with the stacked products of the residual kernel.
//
// Online softmax with a lazily moved reference maximum.  Each row keeps m, the
// maximum it subtracts; the pair of warps sharing a row agrees on the tile's
// row maximum through shared memory.  m moves only when the tile maximum
// exceeds it by more than kRescale (so every p <= 2^kRescale): then the row's
// O accumulator in TMEM (all products of earlier tiles, which the warp first
// waits for) and its running sum are multiplied by the factor of the move.
// After the first tile that is rare, so the tensor-core pipeline almost never
// waits on it.
//
// The tensor cores' fp32 accumulation in TMEM is not round-to-nearest, so O
// is not carried in TMEM over the whole sequence: every kFold tiles the query
// rows fold it (after its last product has landed) into an fp32 master in
// registers (the row's columns of this half) with round-to-nearest adds, and
// the next product restarts the TMEM chain.  The running sum l adds each tile's 32
// values pairwise before the running add.  Scores are kept in base-2 units (the query is scaled by
// scale * log2(e), as FlashAttention-2 does), so p = 2^(s - m) is one ex2.
#include <math.h>

#include "sa_common.cuh"
#include "tc_util.cuh"

namespace sa {

namespace {

using namespace tc;

constexpr int kRowsQ = 128;
constexpr int kTile = 64;
constexpr int kThreads = 320;
constexpr float kRescale = 12.0f;   // base-2 units: p <= 4096
constexpr int kFold = 16;           // key tiles per TMEM accumulation chain

constexpr int kErrWaitQ = 301, kErrWaitFull = 302, kErrWaitP = 304, kErrWaitS = 305,
              kErrWaitEmpty = 306, kErrWaitO = 307, kErrDrain = 308, kErrWaitPV = 309;

// 2^x with the SFU's ex2 (relative error about 2^-22; 2^-inf = 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct FlashParams {
  const float* q;   // [bh, n, d]
  float* out;       // [bh, n, dv]
  int* status;
  int64_t n;
  int d, dv;
  float scale;
  uint64_t wait_ns;  // limit of one bounded wait
};

template <int DP, int DVP>
struct FLayout {
  static constexpr uint32_t kKT = DP * kTile * 4;
  static constexpr uint32_t kVT = DVP * kTile * 4;
  static constexpr uint32_t kStage = 2 * kKT + 2 * kVT;
  static constexpr int kStages = (200u * 1024u / kStage) >= 4 ? 4 : (int)(200u * 1024u / kStage);
  static_assert(kStages >= 2, "at least double buffering");
  static constexpr uint32_t kQhi = 0, kQlo = DP;
  static constexpr uint32_t kS0 = 2 * DP;            // buffer b: S/P_hi at kS0 + 128 b, P_lo 64 further
  static constexpr uint32_t kO = 2 * DP + 256;
  static constexpr bool kPVStack = kO + 2 * DVP <= 512;
  static_assert(kO + DVP <= 512, "TMEM columns");
  // after the stages: row maxima [2 tiles][2 halves][128], row sums [2][128]
  static constexpr uint32_t kXmax = kStages * kStage;
  static constexpr uint32_t kBars = kXmax + (2 * 2 * 128 + 2 * 128) * 4;
  static constexpr uint32_t kSmemBytes = kBars + (2 * kStages + 10) * 8 + 64 + 1024;
};

template <int DP, int DVP>
__global__ void __launch_bounds__(kThreads, 1)
flash_tc_kernel(const __grid_constant__ CUtensorMap tm_kh, const __grid_constant__ CUtensorMap tm_kl,
                const __grid_constant__ CUtensorMap tm_vh, const __grid_constant__ CUtensorMap tm_vl,
                const FlashParams p) {
  using L = FLayout<DP, DVP>;
  constexpr int kStages = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* xmax = reinterpret_cast<float*>(smem + L::kXmax);   // [2][2][128]
  float* lsum = xmax + 2 * 2 * 128;                           // [2][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBars);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* sfull = bars + 2 * kStages;
  uint64_t* pfull = sfull + 2;
  uint64_t* sfree = pfull + 2;
  uint64_t* qready = sfree + 2;
  uint64_t* ofull = qready + 1;
  uint64_t* drain = ofull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_word = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t h = blockIdx.y;
  const int64_t n_qt = (p.n + kRowsQ - 1) / kRowsQ;
  const int64_t qt = n_qt - 1 - blockIdx.x;     // heavy (late) query tiles first
  const int64_t q0 = qt * kRowsQ;
  const int64_t q_last = min(q0 + kRowsQ, p.n) - 1;
  const int T = (int)((q_last + kTile) / kTile);  // key tiles 0 .. q_last

  // Query-row threads start loading their 32-column chunk of the query row now,
  // so that the loads' latency overlaps the set-up below: 16-byte loads when
  // the rows allow them (a warp's load then touches 32 rows once, not once per
  // float).
  float qv[32];
  if (warp >= 2) {
    const int cq = (warp - 2) >> 2;                // this warp's 32-column chunk (its half)
    const int64_t iq = q0 + (warp & 3) * 32 + lane;
    const bool vq = iq < p.n && cq < DP / 32;
    const float* qr = p.q + (h * p.n + (vq ? iq : 0)) * p.d + cq * 32;
    if (vq && (p.d & 3) == 0 && cq * 32 + 32 <= p.d && (reinterpret_cast<uintptr_t>(p.q) & 15) == 0) {
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float4 x = __ldg(reinterpret_cast<const float4*>(qr) + j4);
        qv[4 * j4 + 0] = x.x;
        qv[4 * j4 + 1] = x.y;
        qv[4 * j4 + 2] = x.z;
        qv[4 * j4 + 3] = x.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) qv[j] = (vq && cq * 32 + j < p.d) ? __ldg(qr + j) : 0.0f;
    }
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sfull[b], 1);
      mbar_init(&pfull[b], 8);   // one arrival per query-row warp
      mbar_init(&sfree[b], 1);
    }
    mbar_init(qready, 8);
    mbar_init(ofull, 1);
    mbar_init(drain, 1);
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
      tma_prefetch_desc(&tm_kh);
      tma_prefetch_desc(&tm_vh);
      int issued = 0;
      for (int t = 0; t < T; ++t) {
        const int s = t % kStages;
        if (t >= kStages && !mbar_wait(&empty[s], ((t / kStages) - 1) & 1, ab, kErrWaitEmpty)) break;
        const int row0 = t * kTile;
        mbar_arrive_expect_tx(&full[s], L::kStage);
        uint8_t* st = smem + s * L::kStage;
#pragma unroll
        for (int a = 0; a < DP / 32; ++a) {
          tma_load_3d(st + a * (2 * kTile * 128), &tm_kh, &full[s], a * 32, row0, (int)h);
          tma_load_3d(st + a * (2 * kTile * 128) + kTile * 128, &tm_kl, &full[s], a * 32, row0, (int)h);
        }
#pragma unroll
        for (int a = 0; a < kTile / 32; ++a) {
          uint8_t* vd = st + 2 * L::kKT + a * (2 * DVP * 128);
          tma_load_3d(vd, &tm_vh, &full[s], row0 + a * 32, 0, (int)h);
          tma_load_3d(vd + DVP * 128, &tm_vl, &full[s], row0 + a * 32, 0, (int)h);
        }
        ++issued;
      }
      // never leave with copies in flight
      for (int t = max(0, issued - kStages); t < issued; ++t) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&full[t % kStages], (t / kStages) & 1)) {
          if (globaltimer_ns() - t0 > 1000000000ull) {
            atomicCAS(p.status, 0, kErrDrain);
            break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_qk = idesc_tf32(128, 2 * kTile, false, false);
    constexpr uint32_t idesc_pv = idesc_tf32(128, L::kPVStack ? 2 * DVP : DVP, false, false);
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
          const uint64_t bh_ = vd + (uint64_t)(((kk >> 2) * (2 * DVP * 128) + (kk & 3) * 32) >> 4);
          // the accumulator restarts after every fold (tiles tp % kFold == 0)
          mma_tf32_ts(tmem + L::kO, ph + kk * 8, bh_, idesc_pv, (tp % kFold || kk > 0) ? 1u : 0u);
          if (L::kPVStack) {
            mma_tf32_ts(tmem + L::kO, pl + kk * 8, bh_, idesc_pv, 1u);
          } else {
            const uint64_t bl_ = bh_ + (uint64_t)((DVP * 128) >> 4);
            mma_tf32_ts(tmem + L::kO, ph + kk * 8, bl_, idesc_pv, 1u);
            mma_tf32_ts(tmem + L::kO, pl + kk * 8, bh_, idesc_pv, 1u);
          }
        }
        mma_commit(&empty[sp]);
        mma_commit(&sfree[bp]);
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
          const uint64_t bk = kd + (uint64_t)(((kk >> 2) * (2 * kTile * 128) + (kk & 3) * 32) >> 4);
          mma_tf32_ts(dS, tmem + L::kQhi + kk * 8, bk, idesc_qk, kk > 0 ? 1u : 0u);
          mma_tf32_ts(dS, tmem + L::kQlo + kk * 8, bk, idesc_qk, 1u);
        }
        mma_commit(&sfull[b]);
      }
      __syncwarp();
      if (t >= 1 && !issue_pv(t - 1)) { ok = false; break; }
    }
    if (ok && T > 0) ok = issue_pv(T - 1);
    if (ok && elect_one()) mma_commit(ofull);
    if (elect_one()) mma_commit(drain);
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(drain, 0)) {
      if (globaltimer_ns() - t0 > 2000000000ull) {
        atomicCAS(p.status, 0, kErrDrain);
        break;
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ query rows
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int64_t i = q0 + row;
    const bool valid = i < p.n;
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    const float qscale = p.scale * 1.4426950408889634f;   // log2(e): scores in base 2
    {
      // this half's 32-column chunk of the scaled query (loaded into qv at the start)
      static_assert(DP / 32 <= 2, "one query chunk per half");
      if (half < DP / 32) {
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float x = qv[j] * qscale;
          hi[j] = to_tf32(x);
          lo[j] = __float_as_uint(x - __uint_as_float(hi[j]));
        }
        tmem_st32(lane_addr + L::kQhi + half * 32, hi);
        tmem_st32(lane_addr + L::kQlo + half * 32, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(qready);
    }
    // O columns this half rescales and writes: 32-column chunks c with (c & 1) == half
    // (for DVP = 32 the single chunk belongs to half 0)
    float m = -INFINITY;   // the maximum this row subtracts
    float l = 0.0f;        // this half's running sum of exp(x - m)
    // the master: this half's 32-column chunks of the row (tiles before the last fold)
    constexpr int kMine = DVP == 32 ? 1 : DVP / 64;
    float master[kMine][32];
#pragma unroll
    for (int c = 0; c < kMine; ++c)
#pragma unroll
      for (int j = 0; j < 32; ++j) master[c][j] = 0.0f;
    bool ok = true;
    const uint32_t bar_id = 2 + quarter;   // named barrier of the warp pair
    // Waits are warp-uniform and a failed wait does not leave the loop: both
    // warps of a pair pass the same named barrier once per tile, whatever
    // happens (a failed CTA skips its work; the status word says why).
    for (int t = 0; t < T; ++t) {
      const int b = t & 1;
      if (ok && !mbar_wait_warp(&sfull[b], (t >> 1) & 1, ab, kErrWaitS)) ok = false;
      const uint32_t tS = lane_addr + L::kS0 + 128 * b + half * 32;
      const int64_t col0 = (int64_t)t * kTile + half * 32;
      // causal mask: key col0 + j is visible to row i when j <= lim
      const int64_t rel = i - col0;
      const int lim = !valid || rel < 0 ? -1 : (rel > 31 ? 31 : (int)rel);
      const bool all_on = lim >= 31;
      float sv[32];
      float pm = -INFINITY;
      if (ok) {
        tc_fence_after();
        float s2[32];
        tmem_ld32(tS, sv);
        tmem_ld32(tS + 64, s2);
        tmem_wait_ld();
        if (all_on) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            sv[j] += s2[j];
            pm = fmaxf(pm, sv[j]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            sv[j] = j <= lim ? sv[j] + s2[j] : -INFINITY;
            pm = fmaxf(pm, sv[j]);
          }
        }
      }
      // the pair's row maximum of this tile
      xmax[(b * 2 + half) * 128 + row] = pm;
      asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory");
      if (!ok) continue;
      const float tmax = fmaxf(pm, xmax[(b * 2 + (half ^ 1)) * 128 + row]);
      // move m when the tile's maximum exceeds it by more than kRescale; a
      // valid row sees key 0 in tile 0, so its m is finite from then on
      const bool move = tmax > m + kRescale;
      float alpha = 1.0f;
      if (move) {
        alpha = (m == -INFINITY) ? 0.0f : ex2_approx(m - tmax);
        m = tmax;
        l *= alpha;
      }
      // fold O into the master (every kFold tiles), or rescale it where a row
      // of this warp moved its m; both first wait for the products of tile t-1
      const bool fold = t > 0 && t % kFold == 0;
      if (t > 0 && (fold || __any_sync(0xffffffffu, move))) {
        const int tp = t - 1;
        if (!mbar_wait_warp(&sfree[tp & 1], (tp >> 1) & 1, ab, kErrWaitPV)) {
          ok = false;
          continue;
        }
        tc_fence_after();
#pragma unroll
        for (int cchunk = 0; cchunk < DVP / 32; ++cchunk) {
          if (DVP > 32 && (cchunk & 1) != half) continue;
          if (DVP == 32 && half != 0) continue;
          float (&g)[32] = master[DVP == 32 ? 0 : cchunk >> 1];
          if (fold) {
            // master = (master + O) * alpha; the TMEM chain restarts at tile t
            float ov[32];
            tmem_ld32(lane_addr + L::kO + cchunk * 32, ov);
            if (L::kPVStack) {
              float o2[32];
              tmem_ld32(lane_addr + L::kO + DVP + cchunk * 32, o2);
              tmem_wait_ld();
#pragma unroll
              for (int j = 0; j < 32; ++j) ov[j] += o2[j];
            }
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) g[j] = (g[j] + ov[j]) * alpha;
          } else {
            // O *= alpha in TMEM, and the master with it
#pragma unroll
            for (int part = 0; part < (L::kPVStack ? 2 : 1); ++part) {
              const uint32_t oa = lane_addr + L::kO + part * DVP + cchunk * 32;
              float ov[32];
              tmem_ld32(oa, ov);
              tmem_wait_ld();
              uint32_t os[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) os[j] = __float_as_uint(ov[j] * alpha);
              tmem_st32(oa, os);
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) g[j] *= alpha;
          }
        }
      }
      // masked scores are -inf: ex2 gives exactly 0 there (m is finite for a
      // valid row; an invalid row has every p = 0 below)
      const float mm = valid ? m : 0.0f;
      uint32_t hi[32], lo[32];
      float ps[16];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float e = ex2_approx(sv[j] - mm);
        if (j & 1) ps[j >> 1] += e; else ps[j >> 1] = e;
        hi[j] = to_tf32(e);
        lo[j] = __float_as_uint(e - __uint_as_float(hi[j]));
      }
#pragma unroll
      for (int w = 8; w >= 1; w >>= 1) {
#pragma unroll
        for (int j = 0; j < w; ++j) ps[j] += ps[j + w];
      }
      l += ps[0];
      tmem_st32(tS, hi);
      tmem_st32(tS + 64, lo);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfull[b]);
    }
    // both halves' sums (they share m)
    lsum[half * 128 + row] = l;
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const float l_all = lsum[row] + lsum[128 + row];
    if (ok && mbar_wait_warp(ofull, 0, ab, kErrWaitO)) {
      tc_fence_after();
      const float dmax = fmaxf(l_all, 1.0e-20f);
      float* orow = p.out + (h * p.n + (valid ? i : 0)) * (int64_t)p.dv;
#pragma unroll
      for (int cchunk = 0; cchunk < DVP / 32; ++cchunk) {
        if (DVP > 32 && (cchunk & 1) != half) continue;
        if (DVP == 32 && half != 0) continue;
        float ov[32];
        tmem_ld32(lane_addr + L::kO + cchunk * 32, ov);
        if (L::kPVStack) {
          float o2[32];
          tmem_ld32(lane_addr + L::kO + DVP + cchunk * 32, o2);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) ov[j] += o2[j];
        }
        tmem_wait_ld();
        if (valid) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int col = cchunk * 32 + j;
            if (col < p.dv) orow[col] = __fdiv_rn(master[DVP == 32 ? 0 : cchunk >> 1][j] + ov[j], dmax);
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

template <int DP, int DVP>
int launch_flash(const CUtensorMap* maps, const FlashParams& prm, int64_t bh, cudaStream_t stream) {
  using L = FLayout<DP, DVP>;
  auto kern = flash_tc_kernel<DP, DVP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kSmemBytes);
  if (e != cudaSuccess) return set_error(SA_ERR_CUDA, "flash_tc smem attribute: %s", cudaGetErrorString(e));
  dim3 grid((unsigned)((prm.n + kRowsQ - 1) / kRowsQ), (unsigned)bh);
  kern<<<grid, kThreads, L::kSmemBytes, stream>>>(maps[0], maps[1], maps[2], maps[3], prm);
  return check_launch("flash_tc_kernel");
}

}  // namespace

// maps: k_hi, k_lo (3-D [bh, n, dp], box {32, 64, 1}), v_hi, v_lo (V^T splits
// [bh, dvp, n_pad], box {32, dvp, 1}); q and out raw fp32.
int launch_flash_tc(const CUtensorMap* maps, const float* q, float* out, int* status, int64_t bh, int64_t n, int d,
                    int dv, float scale, cudaStream_t stream) {
  if (bh == 0 || n == 0) return SA_OK;
  if (bh > 65535 || (n + kRowsQ - 1) / kRowsQ > 2147483647LL)
    return set_error(SA_ERR_UNSUPPORTED, "grid too large for the tensor-core flash kernel");
  const FlashParams prm{q, out, status, n, d, dv, scale, wait_limit_ns()};
  const int dp = d <= 32 ? 32 : (d <= 64 ? 64 : 0);
  const int dvp = dv <= 32 ? 32 : (dv <= 64 ? 64 : (dv <= 128 ? 128 : 0));
  if (dp == 32 && dvp == 32) return launch_flash<32, 32>(maps, prm, bh, stream);
  if (dp == 32 && dvp == 64) return launch_flash<32, 64>(maps, prm, bh, stream);
  if (dp == 32 && dvp == 128) return launch_flash<32, 128>(maps, prm, bh, stream);
  if (dp == 64 && dvp == 32) return launch_flash<64, 32>(maps, prm, bh, stream);
  if (dp == 64 && dvp == 64) return launch_flash<64, 64>(maps, prm, bh, stream);
  if (dp == 64 && dvp == 128) return launch_flash<64, 128>(maps, prm, bh, stream);
  return set_error(SA_ERR_UNSUPPORTED, "tensor-core flash: d=%d dv=%d not supported", d, dv);
}

}  // namespace sa
