// Low-degree Taylor moments on the tensor cores (tcgen05 / TMEM / TMA), 3xTF32.
//
// Same quantity as moments.cu: for query i of block c,
//   low[i, :dv] = phi_q(scale q_i) . S_{<c},  low[i, dv] = phi_q(scale q_i) . s_{<c}
// with S = sum phi_k(k_j) v_j^T and s = sum phi_k(k_j) over the keys of the
// completed blocks before c (fast_article_attention.py:151-259,
// streaming_taylor_coreset_attention.py:118-296).
//
// Feature layout.  The monomials are enumerated in aligned runs of 8
// ("segments") that share a prefix: value = x~[p1] * x~[p2] * x~[c0 + u],
// u = 0..7, over the extended row x~ of DX = dp + 8 entries (dp = d rounded up
// to 8): x~[0,d) = x, x~[d,dp) = 0, x~[dp] = 1, the rest 0.  Rows:
//   constant + linear   p1 = p2 = dp, c over [0, DX)
//   degree 2            p1 = a, p2 = dp, c over [8 floor(a/8), dp), a < d
//   degree 3            p1 = a, p2 = b, c over [8 floor(b/8), dp), a <= b < d
// A segment position that is not a canonical monomial (c below the prefix, or
// past d) gets key coefficient 0, so its state row stays exactly zero and its
// query-side value never matters.  This spends ~10% extra MMA work (degree 2,
// d = 64) to let every feature run be produced with vector loads.  The key
// coefficient (1/prod alpha!, or 0) is applied to a state row when its change
// is folded into the master state, not to every key feature: for the
// coefficients 1/2 and 1 that scaling is exact, so the state is the same.
//
// Work split: one CTA per (group of up to FT feature tiles of 128, sequence).
// The CTA scans the sequence block by block:
//   update phase  dS_j[128 features x dv] = Phi_k^T[features x tokens] . V   (M = features)
//   query phase   Out_j[128 tokens x dv]  = Phi_q[tokens x features of j] . S_j (M = tokens)
// Both feature matrices are generated on the CUDA cores directly into TMEM
// (tcgen05.st), where they are the A operand.  Sixteen generator warps, four
// per TMEM lane quarter: thread t of each of the four column groups owns TMEM
// lane t, i.e. token t in the query phase and feature t of the tile in the
// update phase, and each column group writes a quarter of every chunk's
// columns (one 8-feature segment, or 8 tokens).  Four warps per scheduler
// hide the latency of each warp's dependent loads, products and TMEM stores.
// A warp hands a finished chunk to the MMA issuer with one arrival (after
// every lane's stores are complete).  V chunks (tf32 hi / fp32 remainder
// copies made by the transposing split pass) arrive by TMA, K-major with the
// 128-byte swizzle: dv hi rows, then dv lo rows, of 32 tokens.
//
// Each 8-wide K step takes the three products of 3xTF32 as three MMAs of
// N = DVP into one accumulator: A_hi B_hi, A_hi B_lo, A_lo B_hi (the hi and
// remainder copies of V or of the state sit one fixed stride apart in shared
// memory).  A tf32 MMA's time grows with N (M = 128: 32 cycles at N = 64,
// 64 at N = 128, measured back to back), so this costs 3/4 of the two
// doubled-width MMAs that would also form the unneeded A_lo B_lo.
//
// Accumulation: tensor-core accumulation into TMEM does not round to nearest,
// so no long sum stays there.  dS_j covers one block (3 MMAs per 8 keys) and is
// folded into an fp32 master state in global memory (L2-resident, RN adds on
// the CUDA cores) at the start of the next query phase, where the same thread
// also writes the state's hi/lo split (MN-major, 32-byte-atom swizzle) that is
// the B operand of the query product.  Out_j covers one tile (48 MMA steps)
// and lands in tile j's own TMEM columns (free after the fold); the tiles are
// summed in registers.  The denominator column is a dot product with the same
// features on the CUDA cores.  Each CTA writes its partial sums; the residual
// kernel adds the groups.
//
// Every wait is bounded, including the generator warps' own barrier (an
// mbarrier, not bar.sync): a role that gives up leaves its loops, and the
// others then give up at their next wait instead of waiting for it forever.
#include "moments_seg.cuh"
#include "sa_common.cuh"
#include "tc_util.cuh"

namespace sa {

namespace {

using namespace tc;

using namespace mseg;

constexpr int kRows = 128;      // tokens per sub-tile = features per tile = TMEM lanes
constexpr int kChunk = 32;      // K columns per staged feature chunk
constexpr int kNCG = 4;         // column groups of generator warps (warps per TMEM lane quarter)
constexpr int kGenWarps = 4 * kNCG;
constexpr int kGenThreads = 32 * kGenWarps;
constexpr int kThreads = 64 + kGenThreads;   // warp 0 TMA, warp 1 MMA, warps 2.. generators
constexpr int kCgCols = kChunk / kNCG;       // chunk columns one column group writes (8)
constexpr int kNStg = 3;        // TMEM staging buffers (32 hi + 32 lo columns each); 3 leave room
                                // for 5 state tiles, so fewer feature groups per sequence
constexpr int kXtStride = kRows + 4;   // transposed key tile row (floats)
constexpr int kTileVals = 4 * (kRows * 64 / 4) / kGenThreads;   // row-tile floats a thread prefetches (16)

constexpr int kErrMomWait = 201, kErrMomDrain = 202;

struct MomTCParams {
  const float* q;     // [bh, n, d]
  const float* k;     // [bh, n, d]
  float* part;        // [G, bh, n, dv+1] partial low sums
  float* master;      // [G, bh, FT*128, DVP] fp32 moment state
  int* status;
  int64_t n, bh;
  int d, dv, bs, degree, nseg, G;
  float scale;
  // 0: the scan (state from zero, queries of block c read the blocks before it);
  // 1 (total): also update and fold the last block, so that `master` ends as the
  //    state of every block and den_io [G, bh, FT*128] receives the feature sums;
  // 2 (frozen): `master` and den_io hold a given state; every block's queries
  //    read it and nothing is updated (the contribution of keys before the
  //    sequence, e.g. earlier shards of a split sequence).
  int mode;
  float* den_io;
  uint64_t wait_ns;   // limit of one bounded wait
};

template <int DVP>
struct MomLayout {
  // TMEM columns of a tile: one DVP-wide accumulator
  static constexpr int kTC = DVP;
  static constexpr int kFT = (512 - kNStg * 2 * kChunk) / kTC > 5 ? 5 : (512 - kNStg * 2 * kChunk) / kTC;
                                                                       // state tiles per CTA
  // TMEM columns: tile j at j*kTC (dS_j, then Out_j); staging after the tiles
  static constexpr uint32_t kStg = kFT * kTC;
  static_assert(kStg + kNStg * 2 * kChunk <= 512, "TMEM columns");
  // shared memory
  static constexpr uint32_t kSbufHalf = (DVP / 32) * kRows * 128;    // hi or lo: DVP/32 chunks x 128 rows x 128 B
  static constexpr uint32_t kSbuf = 2 * kSbufHalf;                   // hi + lo
  static constexpr uint32_t kVStage = 2 * DVP * 128;                // V^T chunk: DVP hi + DVP lo rows x 32 tokens
  static constexpr int kVStages = 2;
};

}  // namespace

// Number of 8-feature segments (see moments_seg.cuh).
__host__ __device__ int64_t mom_seg_count(int d, int t) { return mseg::seg_count(d, t); }

namespace {

// Loads of one 128-row tile of q or k rows into registers, issued one tile
// ahead of use so that their latency hides behind a phase of generation.
//
// Vector path (d % 4 == 0, 16-byte aligned rows): the first min(d, 64) columns
// of the tile are cut into blocks of 8 rows x 4 float4 (64 contiguous bytes per
// row); generator warp w (0..15) takes blocks k * 16 + w, k < 4, and lane l the
// float4 (row 8 rb + l / 4, float4 column 4 cb + l % 4) of block (rb, cb).  A
// warp access then covers eight 64-byte segments.  Scalar path: thread t of
// column group cg reads row t, columns [16 cg, 16 cg + 16).  Columns from 64 on
// are read when the tile is stored.
// The four (row, float4 column) pairs of a thread, packed as 16-bit
// (row << 8 | col4) entries of a uint2, 0xffff where the thread has no element;
// built once per CTA and kept in shared memory (not in registers across phases).
__device__ __forceinline__ uint2 tile_map_entries(int d, int wg, int l) {
  const int d4 = min(d, 64) >> 2, cb = (d4 + 3) >> 2;
  uint32_t w[2];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int b = k * kGenWarps + wg;
    const int rb = b / cb;
    const int row = 8 * rb + (l >> 2), col4 = 4 * (b - rb * cb) + (l & 3);
    const uint32_t e = (rb < 16 && col4 < d4) ? (uint32_t)((row << 8) | col4) : 0xffffu;
    if (k & 1) w[k >> 1] |= e << 16;
    else w[k >> 1] = e;
  }
  return make_uint2(w[0], w[1]);
}

__device__ __forceinline__ uint32_t tile_entry(const uint2& m, int k) {
  const uint32_t w = (k >> 1) == 0 ? m.x : m.y;
  return (k & 1) ? (w >> 16) : (w & 0xffffu);
}

__device__ __forceinline__ void rows_issue(const float* head, int64_t i0, int nvalid, int d, int t, int cg,
                                           bool vec, const uint2* tmap, float (&v)[kTileVals]) {
  if (vec) {
    const uint2 m = *tmap;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t e = tile_entry(m, k);
      const int row = (int)(e >> 8), col4 = (int)(e & 255);
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e != 0xffffu && row < nvalid)
        x = __ldg(reinterpret_cast<const float4*>(head + (i0 + row) * d) + col4);
      v[4 * k + 0] = x.x;
      v[4 * k + 1] = x.y;
      v[4 * k + 2] = x.z;
      v[4 * k + 3] = x.w;
    }
  } else {
    const int a0 = cg * 16;
    const bool valid = t < nvalid;
    const float* src = head + (i0 + (valid ? t : 0)) * d + a0;
#pragma unroll
    for (int u = 0; u < 16; ++u) v[u] = (valid && a0 + u < d) ? __ldg(src + u) : 0.0f;
  }
}

template <int DVP, bool DEG3>
__global__ void __launch_bounds__(kThreads, 1)
moments_tc_kernel(const __grid_constant__ CUtensorMap tm_vh, const __grid_constant__ CUtensorMap tm_vl,
                  const MomTCParams p) {
  using L = MomLayout<DVP>;
  constexpr int FT = L::kFT;
  constexpr int HC = DVP / kNCG;                           // state / output columns per column group
  static_assert(HC == 8 || HC == 16, "column group share of the state");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sbuf = smem;                                    // [2][hi, lo]
  uint8_t* vst = sbuf + 2 * L::kSbuf;                      // [kVStages][hi, lo]
  const int dp = dpad8(p.d);
  const int DX = dp + 8;                                   // extended row length
  const int XS = DX + 4;                                   // query tile row stride
  float* X = reinterpret_cast<float*>(vst + L::kVStages * L::kVStage);   // query: [128][XS]; update: [DX][kXtStride]
  const int xwords = max(max(kRows * XS, DX * kXtStride), kRows * (DVP + 1));
  uint32_t* segtab = reinterpret_cast<uint32_t*>(X + xwords);            // [FT*16]
  float* sden = reinterpret_cast<float*>(segtab + FT * 16);              // [FT*128]
  float* xch = sden + FT * kRows;                                        // [kNCG][128]
  float* sdx = xch + kNCG * kRows;                                       // [kNCG-1][FT*128]
  uint2* tmaps = reinterpret_cast<uint2*>(
      (reinterpret_cast<uintptr_t>(sdx + (kNCG - 1) * FT * kRows) + 15) & ~uintptr_t(15));   // [kGenThreads]
  uint2* fco = tmaps + kGenThreads;                                      // [FT][128] update-phase feature of lane t
  uint64_t* bars = reinterpret_cast<uint64_t*>(fco + FT * kRows);
  uint64_t* stg_full = bars;                // [kNStg] one arrival per generator warp
  uint64_t* stg_free = bars + kNStg;        // [kNStg] commit
  uint64_t* sb_full = bars + 2 * kNStg;     // [2] one arrival per generator warp
  uint64_t* sb_free = sb_full + 2;          // [2] commit
  uint64_t* v_full = sb_free + 2;           // [2] TMA
  uint64_t* v_free = v_full + 2;            // [2] commit
  uint64_t* out_full = v_free + 2;          // commit, once per query sub-tile
  uint64_t* out_free = out_full + 1;        // one arrival per generator warp, once per sub-tile
  uint64_t* u_done = out_free + 1;          // commit, once per update phase
  uint64_t* drain = u_done + 1;
  uint64_t* gbar = drain + 1;               // the generator warps' own barrier
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbar + 1);
  int* abort_word = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x;
  const int64_t h = blockIdx.y;
  const int seg0 = g * FT * 16;                       // first segment of this group
  const int ntiles = min(FT, (p.nseg - seg0 + 15) / 16);
  const int64_t nb = (p.n + p.bs - 1) / p.bs;
  const int sub = (p.bs + kRows - 1) / kRows;          // 128-token sub-tiles of a full block
  // which phases block c has (see MomTCParams::mode)
  auto has_update = [&](int64_t c) { return p.mode != 2 && (c + 1 < nb || p.mode == 1); };
  auto has_query = [&](int64_t c) { return c > 0 || p.mode == 2; };

  if (threadIdx.x == 0) {
    for (int b = 0; b < kNStg; ++b) {
      mbar_init(&stg_full[b], kGenWarps);
      mbar_init(&stg_free[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sb_full[b], kGenWarps);
      mbar_init(&sb_free[b], 1);
      mbar_init(&v_full[b], 1);
      mbar_init(&v_free[b], 1);
    }
    mbar_init(out_full, 1);
    mbar_init(out_free, kGenWarps);
    mbar_init(u_done, 1);
    mbar_init(drain, 1);
    mbar_init(gbar, kGenWarps);
    *abort_word = 0;
    fence_mbar_init();
  }
  for (int s = threadIdx.x; s < FT * 16; s += kThreads) {
    int p1, p2, c0;
    seg_of(seg0 + s, p.d, p.degree, p1, p2, c0);
    // every entry indexes the extended row x~ of DX floats (8 of them from c0)
    if (!SA_DEVICE_CHECK(p1 >= 0 && p1 < DX && p2 >= 0 && p2 < DX && c0 >= 0 && c0 + 8 <= DX, p.status, 911,
                         seg0 + s)) {
      p1 = p2 = c0 = 0;
    }
    segtab[s] = (uint32_t)p1 | ((uint32_t)p2 << 10) | ((uint32_t)c0 << 20);
  }
  __syncthreads();
  for (int f = threadIdx.x; f < FT * kRows; f += kThreads) {
    sden[f] = p.mode == 2 ? p.den_io[((int64_t)g * p.bh + h) * (FT * kRows) + f] : 0.0f;
    // the update-phase feature of lane t of tile j (f = j * 128 + t): its indices
    // and key coefficient
    const int j = f / kRows, t = f % kRows;
    const uint32_t sg = segtab[j * 16 + (t >> 3)];
    const int p1 = sg & 1023, p2 = (sg >> 10) & 1023, c = (int)(sg >> 20) + (t & 7);
    const float cf = j < ntiles ? seg_key_coef(p1, p2, c, p.d, p.degree) : 0.0f;
    fco[f] = make_uint2((uint32_t)p1 | ((uint32_t)p2 << 10) | ((uint32_t)c << 20), __float_as_uint(cf));
  }
  if (threadIdx.x >= 64) tmaps[threadIdx.x - 64] = tile_map_entries(p.d, (threadIdx.x >> 5) - 2, threadIdx.x & 31);
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const Abort ab{abort_word, p.status, p.wait_ns};
  const float* qh = p.q + h * p.n * p.d;
  const float* kh = p.k + h * p.n * p.d;

  if (warp == 0) {
    // -------------------------------------------------------------- V chunks
    if (lane == 0) {
      int use = 0;
      bool ok = true;
      for (int64_t c = 0; ok && c < nb; ++c) {
        if (!has_update(c)) continue;
        for (int st = 0; ok && st < sub; ++st) {
          const int64_t t0 = c * p.bs + (int64_t)st * kRows;
          for (int tc = 0; tc < kRows / kChunk; ++tc, ++use) {
            const int s = use & 1;
            if (use >= 2 && !mbar_wait(&v_free[s], ((use >> 1) - 1) & 1, ab, kErrMomWait)) { ok = false; break; }
            mbar_arrive_expect_tx(&v_full[s], L::kVStage);
            uint8_t* dst = vst + s * L::kVStage;
            const int row = (int)(t0 + tc * kChunk);
            // V^T chunk: DVP hi rows, then DVP lo rows, of 32 tokens (128 B) each
            tma_load_3d(dst, &tm_vh, &v_full[s], row, 0, (int)h);
            tma_load_3d(dst + DVP * 128, &tm_vl, &v_full[s], row, 0, (int)h);
          }
        }
      }
      for (int u = max(0, use - 2); u < use; ++u) {  // no copies left in flight
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&v_full[u & 1], (u >> 1) & 1) && globaltimer_ns() - t0 < 1000000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer
    // the whole warp runs the loop; the elected lane issues MMAs and commits
    {
      // B = the hi or the lo copy of V or of the state (N = DVP each).  The state
      // is MN-major (written by the generators); V is K-major (transposed split).
      constexpr uint32_t idesc = idesc_tf32(128, DVP, false, true);
      constexpr uint32_t idesc_v = idesc_tf32(128, DVP, false, false);
      int stg_use = 0, sb_use = 0, v_use = 0, sub_use = 0;
      bool ok = true;
      for (int64_t c = 0; ok && c < nb; ++c) {
        if (has_query(c)) {
          const int64_t b1 = min((c + 1) * (int64_t)p.bs, p.n);
          const int nsq = (int)((b1 - c * (int64_t)p.bs + kRows - 1) / kRows);  // query sub-tiles of block c
          for (int st = 0; ok && st < nsq; ++st, ++sub_use) {
            if (sub_use >= 1 && !mbar_wait_warp(out_free, (sub_use - 1) & 1, ab, kErrMomWait)) { ok = false; break; }
            tc_fence_after();
            for (int j = 0; ok && j < ntiles; ++j, ++sb_use) {
              const int sb = sb_use & 1;
              if (!mbar_wait_warp(&sb_full[sb], (sb_use >> 1) & 1, ab, kErrMomWait)) { ok = false; break; }
              tc_fence_after();
              const uint32_t bhi = smem_u32(sbuf + sb * L::kSbuf);
              const uint32_t dO = tmem + j * L::kTC;
              for (int kc = 0; kc < kRows / kChunk; ++kc, ++stg_use) {
                const int b = stg_use % kNStg;
                if (!mbar_wait_warp(&stg_full[b], (stg_use / kNStg) & 1, ab, kErrMomWait)) { ok = false; break; }
                tc_fence_after();
                // one elected lane issues the chunk's 12 MMAs and its commit back to back
                // (at N = DVP an MMA takes only ~32 cycles, so per-MMA elections and
                // descriptor arithmetic would starve the tensor pipe)
                if (elect_one()) {
                  const uint32_t ahi = tmem + L::kStg + b * 2 * kChunk;
                  const uint32_t alo = ahi + kChunk;
                  // 8 feature rows of 128 B per K step: the descriptors' start address
                  // field (address >> 4) advances by 64 per step
                  const uint64_t dbh = sdesc_sw128_atom32(bhi + kc * kChunk * 128, kRows * 128, 512);
                  const uint64_t dbl = dbh + (L::kSbufHalf >> 4);
#pragma unroll
                  for (int kk = 0; kk < kChunk / 8; ++kk) {
                    const uint64_t dk = (uint64_t)(kk * 8 * 128 / 16);
                    mma_tf32_ts(dO, ahi + kk * 8, dbh + dk, idesc, (kc > 0 || kk > 0) ? 1u : 0u);
                    mma_tf32_ts(dO, ahi + kk * 8, dbl + dk, idesc, 1u);
                    mma_tf32_ts(dO, alo + kk * 8, dbh + dk, idesc, 1u);
                  }
                  mma_commit(&stg_free[b]);
                }
                __syncwarp();
              }
              if (elect_one()) mma_commit(&sb_free[sb]);
            }
            // one commit per sub-tile: it completes once every tile's MMAs are done
            // (a waiter must never fall two phases behind an mbarrier)
            if (ok && elect_one()) mma_commit(out_full);
          }
        }
        if (ok && has_update(c)) {
          for (int st = 0; ok && st < sub; ++st) {
            for (int tc = 0; ok && tc < kRows / kChunk; ++tc, ++v_use) {
              const int vs = v_use & 1;
              if (!mbar_wait_warp(&v_full[vs], (v_use >> 1) & 1, ab, kErrMomWait)) { ok = false; break; }
              const uint32_t vhi = smem_u32(vst + vs * L::kVStage);
              for (int j = 0; ok && j < ntiles; ++j, ++stg_use) {
                const int b = stg_use % kNStg;
                if (!mbar_wait_warp(&stg_full[b], (stg_use / kNStg) & 1, ab, kErrMomWait)) { ok = false; break; }
                tc_fence_after();
                if (elect_one()) {
                  const uint32_t ahi = tmem + L::kStg + b * 2 * kChunk;
                  const uint32_t alo = ahi + kChunk;
                  const uint32_t dS = tmem + j * L::kTC;
                  // K-major V^T rows of 128 B: a K step of 8 tokens is 32 B further
                  const uint64_t dbh = sdesc_sw128(vhi, 16, 1024);
                  const uint64_t dbl = dbh + ((DVP * 128) >> 4);
#pragma unroll
                  for (int kk = 0; kk < kChunk / 8; ++kk) {
                    const uint64_t dk = (uint64_t)(kk * 32 / 16);
                    // dS_j starts from zero in every block
                    const uint32_t acc = (st > 0 || tc > 0 || kk > 0) ? 1u : 0u;
                    mma_tf32_ts(dS, ahi + kk * 8, dbh + dk, idesc_v, acc);
                    mma_tf32_ts(dS, ahi + kk * 8, dbl + dk, idesc_v, 1u);
                    mma_tf32_ts(dS, alo + kk * 8, dbh + dk, idesc_v, 1u);
                  }
                  mma_commit(&stg_free[b]);
                }
                __syncwarp();
              }
              if (elect_one()) mma_commit(&v_free[vs]);
            }
          }
          if (ok && elect_one()) mma_commit(u_done);
        }
      }
      if (elect_one()) mma_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0)) {
        if (globaltimer_ns() - t0 > 2000000000ull) {
          atomicCAS(p.status, 0, kErrMomDrain);
          break;
        }
      }
      __syncwarp();
    }
  } else {
    // -------------------------------------------------------------- generators
    // four warps per TMEM lane quarter, one per column group cg: thread t owns
    // TMEM lane t, and column group cg writes columns [8 cg, 8 cg + 8) of every
    // chunk's hi and lo halves and columns [HC cg, HC cg + HC) of every state row
    const int gi = threadIdx.x - 64;
    const int cg = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int t = quarter * 32 + lane;                   // TMEM lane = token or feature
    const uint32_t la = tmem + ((uint32_t)(quarter * 32) << 16);
    int stg_use = 0, sb_use = 0, out_use = 0;
    bool ok = true;
    const int64_t col_stride = p.dv + 1;
    // The generator warps' barrier: an mbarrier each warp arrives on once, waited
    // on with the bounded wait (a generator that gave up stops arriving, and
    // the others then give up instead of hanging).  Every wait of a generator
    // warp has one verdict for all its lanes (mbar_wait_warp), so the warp's
    // .sync.aligned TMEM instructions always run converged.
    uint32_t gphase = 0;
    // one arrival per warp, once every lane's stores (TMEM or shared) are done
    auto warp_arrive = [&](uint64_t* bar) {
      __syncwarp();
      if (lane == 0) mbar_arrive(bar);
    };
    // (one arrival per warp rather than per thread: 512 arrivals on one mbarrier
    // serialize in the shared-memory atomics unit)
    auto gen_sync = [&]() -> bool {
      warp_arrive(gbar);
      const bool r = mbar_wait_warp(gbar, gphase, ab, kErrMomWait);
      gphase ^= 1;
      return r;
    };

    float* part_h = p.part + ((int64_t)g * p.bh + h) * p.n * col_stride;
    // staged query sums of one sub-tile ([rows, dv + 1] in the state buffer)
    // and where they go; copy_out writes them once every thread has staged its row
    float* ostg = reinterpret_cast<float*>(sbuf);
    int64_t out_i0 = 0;
    int out_rows = 0;
    auto copy_out = [&]() {
      if (out_rows > 0 && !SA_DEVICE_CHECK(out_i0 >= 0 && out_i0 + out_rows <= p.n, p.status, 912, out_i0))
        out_rows = 0;
      if (out_rows > 0) {
        const int total = out_rows * (int)col_stride;
        float* dst = part_h + out_i0 * col_stride;
        for (int e = gi; e < total; e += kGenThreads) dst[e] = ostg[e];
        out_rows = 0;
      }
    };
    float* master_h = p.master + ((int64_t)g * p.bh + h) * (int64_t)(FT * kRows) * DVP;
    const bool vec = (p.d & 3) == 0 &&
                     ((reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.k)) & 15) == 0;
    // Row tiles are loaded one tile ahead, in the order the phases consume them:
    // per block c, the query sub-tiles of c (c > 0), then the key sub-tiles of c
    // (c + 1 < nb).  rowv holds this thread's share of the next tile.
    const uint2* my_map = tmaps + gi;
    float rowv[kTileVals];
    auto issue_tile = [&](int64_t uc, bool uq, int ust) {
      const int64_t i0 = uc * p.bs + (int64_t)ust * kRows;
      const int nvalid = (int)min((int64_t)kRows, min(uc * p.bs + p.bs, p.n) - i0);
      rows_issue(uq ? qh : kh, i0, nvalid, p.d, t, cg, vec, my_map, rowv);
    };
    // issue the loads of the tile after (uc, uq, ust), if there is one
    auto issue_next = [&](int64_t uc, bool uq, int ust) {
      if (uq) {
        const int64_t ub0 = uc * p.bs, ub1 = min(ub0 + p.bs, p.n);
        if ((int64_t)(ust + 1) * kRows < ub1 - ub0) issue_tile(uc, true, ust + 1);
        else if (has_update(uc)) issue_tile(uc, false, 0);
        else if (uc + 1 < nb && has_query(uc + 1)) issue_tile(uc + 1, true, 0);
      } else if (ust + 1 < sub) {
        issue_tile(uc, false, ust + 1);
      } else if (uc + 1 < nb) {
        issue_tile(uc + 1, true, 0);
      }
    };
    if (has_query(0)) issue_tile(0, true, 0);
    else if (has_update(0)) issue_tile(0, false, 0);
    // Master state: only the thread that owns feature t of a tile (and its column
    // group's columns) ever touches those entries, so they are stored in the order
    // that makes a warp's accesses contiguous: float4 u4 of (tile j, column group
    // cg, lane t) at float4 index ((j * kNCG + cg) * (HC / 4) + u4) * 128 + t.
    auto mrow_of = [&](int j) {
      return reinterpret_cast<float4*>(master_h) + (int64_t)((j * kNCG + cg) * (HC / 4)) * kRows + t;
    };
    // master state row of the next tile to fold (prefetched one tile ahead)
    float mp[HC];
    auto mload = [&](int j) {
      const float4* mrow = mrow_of(j);
#pragma unroll
      for (int u4 = 0; u4 < HC / 4; ++u4) {
        const float4 m4 = mrow[u4 * kRows];
        mp[4 * u4 + 0] = m4.x;
        mp[4 * u4 + 1] = m4.y;
        mp[4 * u4 + 2] = m4.z;
        mp[4 * u4 + 3] = m4.w;
      }
    };
    // the transposed key tile of update sub-tile st of block c into X
    // (X[a * kXtStride + token]) from the prefetched rows; then the next tile's loads
    auto stage_keys = [&](int64_t c, int st) {
      const int64_t b1 = min(c * p.bs + (int64_t)p.bs, p.n);
      const int64_t i = c * p.bs + (int64_t)st * kRows + t;
      const bool valid = i < b1;
      if (vec) {
        const uint2 m = *my_map;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t e = tile_entry(m, k);
          const int row = (int)(e >> 8), col4 = (int)(e & 255);
          if (e != 0xffffu) {
#pragma unroll
            for (int u = 0; u < 4; ++u) X[(4 * col4 + u) * kXtStride + row] = rowv[4 * k + u];
          }
        }
      } else {
        const int a0 = cg * 16;
#pragma unroll
        for (int u = 0; u < 16; ++u)
          if (a0 + u < p.d) X[(a0 + u) * kXtStride + t] = rowv[u];
      }
      const float* src = kh + (valid ? i : 0) * p.d;
      for (int a = 64 + cg; a < p.d; a += kNCG) X[a * kXtStride + t] = valid ? __ldg(src + a) : 0.0f;
      // an invalid token's extended row is all zero, so are its features
      if (cg == kNCG - 1)
        for (int a = p.d; a < DX; ++a) X[a * kXtStride + t] = (a == dp && valid) ? 1.0f : 0.0f;
      issue_next(c, false, st);
    };
    bool kstaged = false;   // the first key tile of the update phase is already in X
    for (int64_t c = 0; ok && c < nb; ++c) {
      const int64_t b0 = c * p.bs;
      const int64_t b1 = min(b0 + (int64_t)p.bs, p.n);
      // ---------------- query phase: tokens of block c read S_{<c}
      if (!has_query(c)) {
        // no earlier block: this block's low sums are zero
        float* dst = part_h + b0 * col_stride;
        const int64_t total = (b1 - b0) * col_stride;
        for (int64_t e = gi; e < total; e += kGenThreads) dst[e] = 0.0f;
      } else {
        const bool frozen = p.mode == 2;
        if (c >= 2 || frozen) mload(0);   // the state rows written by the previous query phase
        const int nsq = (int)((b1 - b0 + kRows - 1) / kRows);  // query sub-tiles of block c
        for (int st = 0; ok && st < nsq; ++st) {
          const int64_t i = b0 + (int64_t)st * kRows + t;
          const bool valid = i < b1;
          float* xr = X + t * XS;
          // X is free, and sden of the previous update phase is visible
          if (!gen_sync()) { ok = false; break; }
          {
            // x~ = [scale q_i, zeros, 1 at dp, zeros]
            if (vec) {
              const uint2 m = *my_map;
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const uint32_t e = tile_entry(m, k);
                const int row = (int)(e >> 8), col4 = (int)(e & 255);
                if (e != 0xffffu)
                  *reinterpret_cast<float4*>(X + row * XS + 4 * col4) =
                      make_float4(rowv[4 * k] * p.scale, rowv[4 * k + 1] * p.scale, rowv[4 * k + 2] * p.scale,
                                  rowv[4 * k + 3] * p.scale);
              }
            } else {
              const int a0 = cg * 16;
#pragma unroll
              for (int u = 0; u < 16; ++u)
                if (a0 + u < p.d) xr[a0 + u] = rowv[u] * p.scale;
            }
            const float* src = qh + (valid ? i : 0) * p.d;
            for (int a = 64 + cg; a < p.d; a += kNCG) xr[a] = valid ? __ldg(src + a) * p.scale : 0.0f;
            if (cg == kNCG - 1)
              for (int a = p.d; a < DX; ++a) xr[a] = (a == dp) ? 1.0f : 0.0f;
          }
          issue_next(c, true, st);
          if (!gen_sync()) { ok = false; break; }
          // the fold below reads the update products of block c - 1: wait for them
          // only now, so that staging the query tile overlaps their tail
          if (st == 0 && !frozen) {
            if (!mbar_wait_warp(u_done, (int)((c - 1) & 1), ab, kErrMomWait)) { ok = false; break; }
            tc_fence_after();
          }
          float den_acc = 0.0f;
          for (int j = 0; ok && j < ntiles; ++j, ++sb_use) {
            const int sb = sb_use & 1;
            if (sb_use >= 2 && !mbar_wait_warp(&sb_free[sb], ((sb_use >> 1) - 1) & 1, ab, kErrMomWait)) { ok = false; break; }
            {
              // State row of feature t of tile j, this column group's HC columns:
              // fold cf * dS_j (first sub-tile) into the fp32 master and write the
              // hi/lo split into the B buffer (MN-major: row t of chunk (cg HC) / 32,
              // 32-byte granule g stored at g ^ (t & 3)).
              float4* mrow = mrow_of(j);
              uint8_t* bhi = sbuf + sb * L::kSbuf + ((cg * HC) / 32) * (kRows * 128) + t * 128;
              uint8_t* blo = bhi + L::kSbufHalf;
              const int g0 = ((cg * HC) % 32) / 8;
              float sv[HC];
              if (st == 0 && !frozen) {
                tmem_ld_wait<HC>(la + j * L::kTC + cg * HC, sv);
                const float cf = __uint_as_float(fco[j * kRows + t].y);
#pragma unroll
                for (int u = 0; u < HC; ++u) sv[u] *= cf;
                if (c >= 2) {
#pragma unroll
                  for (int u = 0; u < HC; ++u) sv[u] += mp[u];
                }
#pragma unroll
                for (int u4 = 0; u4 < HC / 4; ++u4)
                  mrow[u4 * kRows] = make_float4(sv[4 * u4], sv[4 * u4 + 1], sv[4 * u4 + 2], sv[4 * u4 + 3]);
              } else {
#pragma unroll
                for (int u = 0; u < HC; ++u) sv[u] = mp[u];
              }
#pragma unroll
              for (int gg = 0; gg < HC / 8; ++gg) {
                const uint32_t off = (uint32_t)(((g0 + gg) ^ (t & 3)) * 32);
                float hv[8], lv[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                  hv[u] = __uint_as_float(tf32_trunc(sv[gg * 8 + u]));
                  lv[u] = sv[gg * 8 + u] - hv[u];
                }
                *reinterpret_cast<float4*>(bhi + off) = make_float4(hv[0], hv[1], hv[2], hv[3]);
                *reinterpret_cast<float4*>(bhi + off + 16) = make_float4(hv[4], hv[5], hv[6], hv[7]);
                *reinterpret_cast<float4*>(blo + off) = make_float4(lv[0], lv[1], lv[2], lv[3]);
                *reinterpret_cast<float4*>(blo + off + 16) = make_float4(lv[4], lv[5], lv[6], lv[7]);
              }
            }
            // prefetch the state row of the next tile to fold: tile j + 1, or tile 0 of
            // the next sub-tile (written by the fold of sub-tile 0 above)
            if (j + 1 < ntiles) {
              if (st > 0 || c >= 2 || frozen) mload(j + 1);
            } else if (st + 1 < nsq) {
              mload(0);
            }
            tc_fence_before();   // the dS_j reads are ordered before the MMAs that reuse its columns
            fence_proxy_async_smem();
            warp_arrive(&sb_full[sb]);
            // Phi_q chunks of tile j for this thread's token: one segment (8 features) each
            for (int kc = 0; kc < kRows / kChunk; ++kc, ++stg_use) {
              const int b = stg_use % kNStg;
              const int sl = j * 16 + kc * 4 + cg;    // segment within the group
              const uint32_t pk = segtab[sl];
              float pre = xr[pk & 1023];
              if (DEG3) pre *= xr[(pk >> 10) & 1023];
              const float* xc = xr + (pk >> 20);
              const float4 x0 = ld4(xc), x1 = ld4(xc + 4);
              const float4 d0 = ld4(sden + sl * 8), d1 = ld4(sden + sl * 8 + 4);
              const float ph[8] = {pre * x0.x, pre * x0.y, pre * x0.z, pre * x0.w,
                                   pre * x1.x, pre * x1.y, pre * x1.z, pre * x1.w};
              const float dd[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
              uint32_t hi[8], lo[8];
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                den_acc = fmaf(ph[u], dd[u], den_acc);
                hi[u] = tf32_trunc(ph[u]);
                lo[u] = __float_as_uint(ph[u] - __uint_as_float(hi[u]));
              }
              if (stg_use >= kNStg && !mbar_wait_warp(&stg_free[b], ((stg_use / kNStg) - 1) & 1, ab, kErrMomWait)) { ok = false; break; }
              tmem_st8(la + L::kStg + b * 2 * kChunk + cg * kCgCols, hi);
              tmem_st8(la + L::kStg + b * 2 * kChunk + kChunk + cg * kCgCols, lo);
              tmem_wait_st();
              tc_fence_before();
              warp_arrive(&stg_full[b]);
            }
          }
          if (!ok) break;
          // X (the query tile) is free once every thread has made its last Phi_q
          // chunk: stage the first key tile of the update phase now, under the
          // tail of the query products (the gen_sync after the readback below
          // orders these writes before the update phase reads them)
          if (st + 1 == nsq && has_update(c)) {
            if (!gen_sync()) { ok = false; break; }
            stage_keys(c, 0);
            kstaged = true;
          }
          // Out_j of every tile sits in the tile's own TMEM columns: once all the
          // sub-tile's MMAs are done, add them up in tile order
          if (!mbar_wait_warp(out_full, out_use & 1, ab, kErrMomWait)) { ok = false; break; }
          ++out_use;
          tc_fence_after();
          float acc[HC];
#pragma unroll
          for (int u = 0; u < HC; ++u) acc[u] = 0.0f;
          for (int j = 0; j < ntiles; ++j) {
            float ov[HC];
            tmem_ld_wait<HC>(la + j * L::kTC + cg * HC, ov);
#pragma unroll
            for (int u = 0; u < HC; ++u) acc[u] += ov[u];
          }
          tc_fence_before();
          warp_arrive(out_free);
          xch[cg * kRows + t] = den_acc;
          if (!gen_sync()) { ok = false; break; }
          {
            // Stage the sub-tile's [rows, dv + 1] sums in the state buffer (every
            // product that reads it is done; row stride dv + 1 is odd, so the
            // column writes are conflict-free).  The coalesced copy to global
            // memory (consecutive threads on consecutive words) waits until after
            // the update phase, where it overlaps the tail of the update products,
            // unless another query sub-tile's fold needs the buffer first.
            const int cs = (int)col_stride;
#pragma unroll
            for (int u = 0; u < HC; ++u)
              if (cg * HC + u < p.dv) ostg[t * cs + cg * HC + u] = acc[u];
            if (cg == 0) {
              float dsum = xch[t];
#pragma unroll
              for (int x = 1; x < kNCG; ++x) dsum += xch[x * kRows + t];
              ostg[t * cs + p.dv] = dsum;
            }
            out_i0 = b0 + (int64_t)st * kRows;
            out_rows = (int)min((int64_t)kRows, b1 - out_i0);
          }
          if (st + 1 < nsq || !has_update(c)) {
            if (!gen_sync()) { ok = false; break; }
            copy_out();
          }
        }
      }
      if (!ok || !has_update(c)) continue;
      // ---------------- update phase: dS_j of block c (unscaled key features;
      // the key coefficient is applied at the fold)
      float sd[FT];
#pragma unroll
      for (int j = 0; j < FT; ++j) sd[j] = 0.0f;
      // a chunk's TMEM stores complete under the next chunk's arithmetic
      int held = -1;
      auto hand_over = [&]() {
        if (held >= 0) {
          tmem_wait_st();
          tc_fence_before();
          warp_arrive(&stg_full[held]);
          held = -1;
        }
      };
      for (int st = 0; ok && st < sub; ++st) {
        if (!(st == 0 && kstaged)) {
          hand_over();
          if (!gen_sync()) { ok = false; break; }   // everyone is done with X
          stage_keys(c, st);
          if (!gen_sync()) { ok = false; break; }
        }
        kstaged = false;
        for (int tcn = 0; ok && tcn < kRows / kChunk; ++tcn) {
          const int tok0 = tcn * kChunk + cg * kCgCols;
#pragma unroll
          for (int j = 0; j < FT; ++j) {
            if (!ok || j >= ntiles) break;
            const int b = stg_use % kNStg;
            const uint32_t fi = fco[j * kRows + t].x;
            const float* r1 = X + (fi & 1023) * kXtStride + tok0;
            const float* rc = X + (fi >> 20) * kXtStride + tok0;
            uint32_t hi[8], lo[8];
            float fsum = 0.0f;
#pragma unroll
            for (int u4 = 0; u4 < 2; ++u4) {
              float4 a4 = ld4(r1 + 4 * u4);
              const float4 c4 = ld4(rc + 4 * u4);
              if (DEG3) {
                const float4 b4 = ld4(X + ((fi >> 10) & 1023) * kXtStride + tok0 + 4 * u4);
                a4.x *= b4.x;
                a4.y *= b4.y;
                a4.z *= b4.z;
                a4.w *= b4.w;
              }
              const float ph[4] = {a4.x * c4.x, a4.y * c4.y, a4.z * c4.z, a4.w * c4.w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                fsum += ph[u];
                hi[4 * u4 + u] = tf32_trunc(ph[u]);
                lo[4 * u4 + u] = __float_as_uint(ph[u] - __uint_as_float(hi[4 * u4 + u]));
              }
            }
            sd[j] += fsum;
            hand_over();
            if (stg_use >= kNStg && !mbar_wait_warp(&stg_free[b], ((stg_use / kNStg) - 1) & 1, ab, kErrMomWait)) { ok = false; break; }
            ++stg_use;
            tmem_st8(la + L::kStg + b * 2 * kChunk + cg * kCgCols, hi);
            tmem_st8(la + L::kStg + b * 2 * kChunk + kChunk + cg * kCgCols, lo);
            held = b;
          }
        }
      }
      hand_over();
      if (!ok) continue;
      // s += cf * (the features of this block's keys): the column groups' sums
      // meet in shared memory, added in column-group order
      if (cg > 0) {
#pragma unroll
        for (int j = 0; j < FT; ++j)
          if (j < ntiles) sdx[((cg - 1) * FT + j) * kRows + t] = sd[j];
      }
      if (!gen_sync()) { ok = false; continue; }   // all reads of sden by the query phase are done
      if (cg == 0) {
#pragma unroll
        for (int j = 0; j < FT; ++j) {
          if (j < ntiles) {
            float s4 = sd[j];
#pragma unroll
            for (int x = 0; x < kNCG - 1; ++x) s4 += sdx[(x * FT + j) * kRows + t];
            sden[j * kRows + t] += __uint_as_float(fco[j * kRows + t].y) * s4;
          }
        }
      }
      copy_out();   // the query sums of this block, staged before the update phase
    }
    if (ok && p.mode == 1) {
      // total: fold the last block's dS into the master (which then holds the
      // state of every block) and hand out the feature sums
      if (!mbar_wait_warp(u_done, (int)((nb - 1) & 1), ab, kErrMomWait)) {
        ok = false;
      } else {
        tc_fence_after();
        for (int j = 0; j < ntiles; ++j) {
          float4* mrow = mrow_of(j);
          const float cf = __uint_as_float(fco[j * kRows + t].y);
          float a[HC];
          tmem_ld_wait<HC>(la + j * L::kTC + cg * HC, a);
#pragma unroll
          for (int u4 = 0; u4 < HC / 4; ++u4) {
            float4 v4 = make_float4(cf * a[4 * u4], cf * a[4 * u4 + 1], cf * a[4 * u4 + 2], cf * a[4 * u4 + 3]);
            if (nb >= 2) {
              const float4 m4 = mrow[u4 * kRows];
              v4.x += m4.x;
              v4.y += m4.y;
              v4.z += m4.z;
              v4.w += m4.w;
            }
            mrow[u4 * kRows] = v4;
          }
        }
        // the feature sums: sden was last written by column group 0 of each lane
        if (cg == 0)
          for (int j = 0; j < ntiles; ++j)
            p.den_io[((int64_t)g * p.bh + h) * (FT * kRows) + j * kRows + t] = sden[j * kRows + t];
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

template <int DVP>
size_t mom_smem(int d) {
  using L = MomLayout<DVP>;
  const int dp = dpad8(d), DX = dp + 8, XS = DX + 4;
  const size_t xwords = (size_t)max(max(kRows * XS, DX * kXtStride), kRows * (DVP + 1));
  return 1024 + 2 * L::kSbuf + L::kVStages * L::kVStage + xwords * 4 + (size_t)L::kFT * 16 * 4 +
         (size_t)L::kFT * kRows * 4 + (size_t)kNCG * kRows * 4 + (size_t)(kNCG - 1) * L::kFT * kRows * 4 + 16 +
         (size_t)kGenThreads * 8 + (size_t)L::kFT * kRows * 8 + (2 * kNStg + 14) * 8 + 16;
}

template <int DVP, bool DEG3>
int launch_mom_tc(const CUtensorMap* maps, const MomTCParams& prm, cudaStream_t stream) {
  auto kern = moments_tc_kernel<DVP, DEG3>;
  const size_t smem = mom_smem<DVP>(prm.d);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_error(SA_ERR_CUDA, "moments_tc smem attribute: %s", cudaGetErrorString(e));
  dim3 grid((unsigned)prm.G, (unsigned)prm.bh);
  kern<<<grid, kThreads, smem, stream>>>(maps[0], maps[1], prm);
  return check_launch("moments_tc_kernel");
}

__global__ void sum_groups_kernel(const float* __restrict__ part, int groups, int64_t stride, float* __restrict__ out) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < stride; e += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.0f;
    for (int g = 0; g < groups; ++g) s += __ldg(part + g * stride + e);
    out[e] = s;
  }
}

}  // namespace

// Feature groups (CTAs per sequence) the tensor-core moment kernel uses, or 0
// when the shape is not supported (then the CUDA-core kernel runs).
int moments_tc_groups(int d, int dv, int degree) {
  if (dv > 64 || d > 128 || degree > 3) return 0;
  const int dvp = dv <= 32 ? 32 : 64;
  const int ft = dvp == 32 ? MomLayout<32>::kFT : MomLayout<64>::kFT;
  const int64_t tiles = (mom_seg_count(d, degree) + 15) / 16;
  const size_t smem = dvp == 32 ? mom_smem<32>(d) : mom_smem<64>(d);
  if (smem > 227 * 1024) return 0;
  return (int)((tiles + ft - 1) / ft);
}

// Floats of the fp32 master state: [G, bh, FT*128, dvp].
int64_t moments_tc_master_floats(int64_t bh, int d, int dv, int degree) {
  const int G = moments_tc_groups(d, dv, degree);
  if (G <= 0) return 0;
  const int dvp = dv <= 32 ? 32 : 64;
  const int ft = dvp == 32 ? MomLayout<32>::kFT : MomLayout<64>::kFT;
  return (int64_t)G * bh * ft * kRows * dvp;
}

// Floats of the feature sums that go with the master state: [G, bh, FT*128].
int64_t moments_tc_den_floats(int64_t bh, int d, int dv, int degree) {
  const int G = moments_tc_groups(d, dv, degree);
  if (G <= 0) return 0;
  const int ft = (dv <= 32 ? 32 : 64) == 32 ? MomLayout<32>::kFT : MomLayout<64>::kFT;
  return (int64_t)G * bh * ft * kRows;
}

namespace {

// The exclusive prefix of per-shard moment states: for each entry e,
// sum over r < nprev of states[r * stride + e], added in shard order; the
// first n_master entries go to the master state, the rest to the feature sums.
__global__ void state_prefix_kernel(const float* __restrict__ states, int nprev, int64_t stride,
                                    float* __restrict__ master, int64_t n_master, float* __restrict__ den,
                                    int64_t n_den) {
  const int64_t total = n_master + n_den;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    float acc = 0.0f;
    for (int r = 0; r < nprev; ++r) acc += __ldg(states + r * stride + e);
    if (e < n_master) master[e] = acc;
    else den[e - n_master] = acc;
  }
}

// The same scan 16 bytes a thread (every count a multiple of 4, every pointer
// 16-byte aligned): entry e4 of the float4 view.
__global__ void state_prefix4_kernel(const float4* __restrict__ states, int nprev, int64_t stride4,
                                     float4* __restrict__ master, int64_t n_master4, float4* __restrict__ den,
                                     int64_t n_den4) {
  const int64_t total = n_master4 + n_den4;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < nprev; ++r) {
      const float4 x = __ldg(states + r * stride4 + e);
      acc.x += x.x;
      acc.y += x.y;
      acc.z += x.z;
      acc.w += x.w;
    }
    if (e < n_master4) master[e] = acc;
    else den[e - n_master4] = acc;
  }
}

}  // namespace

int launch_state_prefix(const float* states, int nprev, int64_t n_master, int64_t n_den, float* master, float* den,
                        cudaStream_t stream) {
  const int64_t total = n_master + n_den;
  if (total == 0) return SA_OK;
  if (nprev > 0 && !states) return set_error(SA_ERR_INVALID_ARG, "null state pointer");
  const int threads = 256;
  if (n_master % 4 == 0 && n_den % 4 == 0 &&
      ((reinterpret_cast<uintptr_t>(states) | reinterpret_cast<uintptr_t>(master) |
        reinterpret_cast<uintptr_t>(den)) & 15) == 0) {
    const int64_t t4 = total / 4;
    const int64_t blocks = min((t4 + threads - 1) / threads, (int64_t)148 * 8);
    state_prefix4_kernel<<<(unsigned)blocks, threads, 0, stream>>>(
        reinterpret_cast<const float4*>(states), nprev, t4, reinterpret_cast<float4*>(master), n_master / 4,
        reinterpret_cast<float4*>(den), n_den / 4);
    return check_launch("state_prefix4_kernel");
  }
  const int64_t blocks = min((total + threads - 1) / threads, (int64_t)148 * 8);
  state_prefix_kernel<<<(unsigned)blocks, threads, 0, stream>>>(states, nprev, total, master, n_master, den, n_den);
  return check_launch("state_prefix_kernel");
}

// out[e] = sum_g part[g * stride + e]: the low sums from the per-group partials.
int launch_sum_groups(const float* part, int groups, int64_t stride, float* out, cudaStream_t stream) {
  if (stride == 0) return SA_OK;
  const int threads = 256;
  const int64_t blocks = min((stride + threads - 1) / threads, (int64_t)148 * 16);
  sum_groups_kernel<<<(unsigned)blocks, threads, 0, stream>>>(part, groups, stride, out);
  return check_launch("sum_groups_kernel");
}

// maps: split v hi / lo ([bh, n, dvp], box {32, 32, 1}, 128-byte swizzle with 32-byte atoms).
int launch_moments_tc(const CUtensorMap* maps, const float* q, const float* k, float* part, float* master,
                      int* status, int64_t bh, int64_t n, int d, int dv, int degree, int bs, float scale,
                      cudaStream_t stream, int mode, float* den_io) {
  if (bh == 0 || n == 0) return SA_OK;
  const int G = moments_tc_groups(d, dv, degree);
  if (G <= 0) return set_error(SA_ERR_UNSUPPORTED, "tensor-core moments: shape not supported");
  if (bh > 65535) return set_error(SA_ERR_UNSUPPORTED, "too many sequences for one launch");
  if (mode != 0 && !den_io) return set_error(SA_ERR_INVALID_ARG, "moment state modes need the feature-sum buffer");
  MomTCParams prm{q, k, part, master, status, n, bh, d, dv, bs, degree, (int)mom_seg_count(d, degree), G, scale,
                  mode, den_io, wait_limit_ns()};
  if (degree == 3) return dv <= 32 ? launch_mom_tc<32, true>(maps, prm, stream) : launch_mom_tc<64, true>(maps, prm, stream);
  return dv <= 32 ? launch_mom_tc<32, false>(maps, prm, stream) : launch_mom_tc<64, false>(maps, prm, stream);
}

}  // namespace sa
