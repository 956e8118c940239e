// Low-degree Taylor moments on the tensor cores (tcgen05 / TMEM / TMA), 3xTF32.
//
// Same quantity as moments.cu: for query i of block c,
//   low[i, :dv] = phi_q(scale q_i) . S_{<c},  low[i, dv] = phi_q(scale q_i) . s_{<c}
// with S = sum phi_k(k_j) v_j^T and s = sum phi_k(k_j) over the keys of the
// completed blocks before c (fast_article_attention.py:151-259,
// streaming_taylor_coreset_attention.py:118-296).
//
// Work split: one CTA per (group of up to FT feature tiles of 128, sequence).
// The CTA scans the sequence block by block:
//   update phase  dS_j[128 features x dv] = Phi_k^T[features x tokens] . V   (M = features)
//   query phase   Out_j[128 tokens x dv]  = Phi_q[tokens x features of j] . S_j (M = tokens)
// Both feature matrices are generated on the CUDA cores directly into TMEM
// (tcgen05.st), where they are the A operand.  Eight generator warps, two per
// TMEM lane quarter: thread t of each half owns TMEM lane t, i.e. token t in
// the query phase and feature t of the tile in the update phase, and each half
// writes half of every chunk's columns.  V chunks (tf32 hi / fp32 remainder copies made
// by the split pass) arrive by TMA, MN-major with the 32-byte-atom swizzle.
//
// Accumulation: tensor-core accumulation into TMEM does not round to nearest,
// so no long sum stays there.  dS_j covers one block (<= 96 MMA steps) and is
// folded into an fp32 master state in global memory (L2-resident, RN adds on
// the CUDA cores) at the start of the next query phase, where the same thread
// also writes the state's K-major hi/lo copy that is the B operand of the
// query product.  Out_j covers one tile (48 MMA steps) and lands in tile j's
// own TMEM columns (free after the fold); the tiles are summed in registers.
// The denominator column is a dot product with the same features on the CUDA
// cores.  Each CTA writes its partial sums; the residual kernel adds the groups.
#include "sa_common.cuh"
#include "tc_util.cuh"

namespace sa {

namespace {

using namespace tc;

constexpr int kRows = 128;      // tokens per sub-tile = features per tile = TMEM lanes
constexpr int kChunk = 32;      // K columns per staged feature chunk
constexpr int kThreads = 320;   // warp 0 TMA, warp 1 MMA, warps 2..9 generators

constexpr int kErrMomWait = 201, kErrMomDrain = 202;

struct MomTCParams {
  const float* q;     // [bh, n, d]
  const float* k;     // [bh, n, d]
  float* part;        // [G, bh, n, dv+1] partial low sums
  float* master;      // [G, bh, FT*128, DVP] fp32 moment state
  int* status;
  int64_t n, bh;
  int d, dv, bs, F, G;
  float scale;
};

template <int DVP>
struct MomLayout {
  static constexpr int kFT = (512 - 2 * 2 * kChunk) / DVP;          // state tiles per CTA
  // TMEM columns: tile j at j*DVP (dS_j, then Out_j); staging after the tiles
  static constexpr uint32_t kStg = kFT * DVP;
  static_assert(kStg + 4 * kChunk <= 512, "TMEM columns");
  // shared memory
  static constexpr uint32_t kSbufHalf = (kRows / 32) * DVP * 128;    // one of hi / lo: 4 atoms x DVP rows x 128 B
  static constexpr uint32_t kSbuf = 2 * kSbufHalf;                   // hi + lo
  static constexpr uint32_t kVHalf = (DVP / 32) * kChunk * 128;     // V chunk hi or lo
  static constexpr uint32_t kVStage = 2 * kVHalf;
  static constexpr int kVStages = 2;
};

__device__ __forceinline__ float key_coef_tc(int a, int b, int c, int d) {
  const bool ab = (a == b) && (a < d);
  const bool bc = (b == c) && (b < d);
  return (ab && bc) ? (1.0f / 6.0f) : ((ab || bc) ? 0.5f : 1.0f);
}

// named barrier among the 256 generator threads (warps 2..9)
__device__ __forceinline__ void gen_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// HC consecutive columns (16 or 32) of this thread's TMEM lane
template <int HC>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float (&v)[HC]) {
  if constexpr (HC == 32) {
    tmem_ld32(taddr, v);
  } else {
    static_assert(HC == 16, "16 or 32 columns");
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
  }
  tmem_wait_ld();
}

template <int DVP, bool DEG3>
__global__ void __launch_bounds__(kThreads, 1)
moments_tc_kernel(const __grid_constant__ CUtensorMap tm_vh, const __grid_constant__ CUtensorMap tm_vl,
                  const MomTCParams p) {
  using L = MomLayout<DVP>;
  constexpr int FT = L::kFT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sbuf = smem;                                   // [2][hi, lo]
  uint8_t* vst = sbuf + 2 * L::kSbuf;                     // [kVStages][hi, lo]
  const int xs = (p.d + 1) | 1;                           // odd row stride, x[d] = 1
  float* X = reinterpret_cast<float*>(vst + L::kVStages * L::kVStage);     // [128][xs]
  uint32_t* ftab = reinterpret_cast<uint32_t*>(X + kRows * xs);            // [FT*128]
  float* sden = reinterpret_cast<float*>(ftab + FT * kRows);               // [FT*128]
  // after sden: [2][128] denominator exchange, [FT*128] sden exchange (used by the generators)
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(sden + FT * kRows + 2 * kRows + FT * kRows) + 7) & ~uintptr_t(7));
  uint64_t* stg_full = bars;        // [2] 256 arrivals
  uint64_t* stg_free = bars + 2;    // [2] commit
  uint64_t* sb_full = bars + 4;     // [2] 256 arrivals
  uint64_t* sb_free = bars + 6;     // [2] commit
  uint64_t* v_full = bars + 8;      // [2] TMA
  uint64_t* v_free = bars + 10;     // [2] commit
  uint64_t* out_full = bars + 12;   // commit, once per (sub-tile, tile)
  uint64_t* out_free = bars + 13;   // 256 arrivals, once per sub-tile
  uint64_t* u_done = bars + 14;     // commit, once per update phase
  uint64_t* drain = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  int* abort_word = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x;
  const int64_t h = blockIdx.y;
  const int f0 = g * FT * kRows;                      // first feature of this group
  const int ntiles = min(FT, (p.F - f0 + kRows - 1) / kRows);
  const int64_t nb = (p.n + p.bs - 1) / p.bs;
  const int sub = (p.bs + kRows - 1) / kRows;          // 128-token sub-tiles of a full block

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&stg_full[b], 256);
      mbar_init(&stg_free[b], 1);
      mbar_init(&sb_full[b], 256);
      mbar_init(&sb_free[b], 1);
      mbar_init(&v_full[b], 1);
      mbar_init(&v_free[b], 1);
    }
    mbar_init(out_full, 1);
    mbar_init(out_free, 256);
    mbar_init(u_done, 1);
    mbar_init(drain, 1);
    *abort_word = 0;
    fence_mbar_init();
  }
  for (int f = threadIdx.x; f < FT * kRows; f += kThreads) {
    const int ff = f0 + f;
    if (ff < p.F) {
      const Monomial mo = monomial_of(ff, p.d);
      ftab[f] = (uint32_t)mo.a | ((uint32_t)mo.b << 10) | ((uint32_t)mo.c << 20);
    } else {
      ftab[f] = 0xFFFFFFFFu;  // padding feature: value 0
    }
    sden[f] = 0.0f;
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const Abort ab{abort_word, p.status};
  const float* qh = p.q + h * p.n * p.d;
  const float* kh = p.k + h * p.n * p.d;

  if (warp == 0) {
    // -------------------------------------------------------------- V chunks
    if (lane == 0) {
      int use = 0;
      bool ok = true;
      for (int64_t c = 0; ok && c + 1 < nb; ++c) {
        for (int st = 0; ok && st < sub; ++st) {
          const int64_t t0 = c * p.bs + (int64_t)st * kRows;
          for (int tc = 0; tc < kRows / kChunk; ++tc, ++use) {
            const int s = use & 1;
            if (use >= 2 && !mbar_wait(&v_free[s], ((use >> 1) - 1) & 1, ab, kErrMomWait)) { ok = false; break; }
            mbar_arrive_expect_tx(&v_full[s], L::kVStage);
            uint8_t* dst = vst + s * L::kVStage;
            const int row = (int)(t0 + tc * kChunk);
#pragma unroll
            for (int a = 0; a < DVP / 32; ++a) {
              tma_load_3d(dst + a * (kChunk * 128), &tm_vh, &v_full[s], a * 32, row, (int)h);
              tma_load_3d(dst + L::kVHalf + a * (kChunk * 128), &tm_vl, &v_full[s], a * 32, row, (int)h);
            }
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
    if (lane == 0) {
      constexpr uint32_t idesc_q = idesc_tf32(128, DVP, false, false);  // B = state copy, K-major
      constexpr uint32_t idesc_u = idesc_tf32(128, DVP, false, true);   // B = V chunk, MN-major
      int stg_use = 0, sb_use = 0, v_use = 0, sub_use = 0;
      bool ok = true;
      for (int64_t c = 0; ok && c < nb; ++c) {
        if (c > 0) {
          const int64_t b1 = min((c + 1) * (int64_t)p.bs, p.n);
          const int nsq = (int)((b1 - c * (int64_t)p.bs + kRows - 1) / kRows);  // query sub-tiles of block c
          for (int st = 0; ok && st < nsq; ++st, ++sub_use) {
            if (sub_use >= 1 && !mbar_wait(out_free, (sub_use - 1) & 1, ab, kErrMomWait)) { ok = false; break; }
            tc_fence_after();
            for (int j = 0; ok && j < ntiles; ++j, ++sb_use) {
              const int sb = sb_use & 1;
              if (!mbar_wait(&sb_full[sb], (sb_use >> 1) & 1, ab, kErrMomWait)) { ok = false; break; }
              tc_fence_after();
              const uint32_t bhi = smem_u32(sbuf + sb * L::kSbuf);
              const uint32_t blo = bhi + L::kSbufHalf;
              const uint32_t dO = tmem + j * DVP;
              for (int kc = 0; kc < kRows / kChunk; ++kc, ++stg_use) {
                const int b = stg_use & 1;
                if (!mbar_wait(&stg_full[b], (stg_use >> 1) & 1, ab, kErrMomWait)) { ok = false; break; }
                tc_fence_after();
                const uint32_t ahi = tmem + L::kStg + b * 2 * kChunk;
                const uint32_t alo = ahi + kChunk;
#pragma unroll
                for (int kk = 0; kk < kChunk / 8; ++kk) {
                  const uint32_t off = kc * (DVP * 128) + kk * 32;
                  const uint64_t dh = sdesc_sw128(bhi + off, 16, 1024);
                  const uint64_t dl = sdesc_sw128(blo + off, 16, 1024);
                  mma_tf32_ts(dO, ahi + kk * 8, dh, idesc_q, (kc > 0 || kk > 0) ? 1u : 0u);
                  mma_tf32_ts(dO, ahi + kk * 8, dl, idesc_q, 1u);
                  mma_tf32_ts(dO, alo + kk * 8, dh, idesc_q, 1u);
                }
                mma_commit(&stg_free[b]);
              }
              mma_commit(&sb_free[sb]);
              mma_commit(out_full);
            }
          }
        }
        if (ok && c + 1 < nb) {
          for (int st = 0; ok && st < sub; ++st) {
            for (int tc = 0; ok && tc < kRows / kChunk; ++tc, ++v_use) {
              const int vs = v_use & 1;
              if (!mbar_wait(&v_full[vs], (v_use >> 1) & 1, ab, kErrMomWait)) { ok = false; break; }
              const uint32_t vhi = smem_u32(vst + vs * L::kVStage);
              const uint32_t vlo = vhi + L::kVHalf;
              for (int j = 0; ok && j < ntiles; ++j, ++stg_use) {
                const int b = stg_use & 1;
                if (!mbar_wait(&stg_full[b], (stg_use >> 1) & 1, ab, kErrMomWait)) { ok = false; break; }
                tc_fence_after();
                const uint32_t ahi = tmem + L::kStg + b * 2 * kChunk;
                const uint32_t alo = ahi + kChunk;
                const uint32_t dS = tmem + j * DVP;
#pragma unroll
                for (int kk = 0; kk < kChunk / 8; ++kk) {
                  const uint64_t dh = sdesc_sw128_atom32(vhi + kk * 1024, kChunk * 128, 512);
                  const uint64_t dl = sdesc_sw128_atom32(vlo + kk * 1024, kChunk * 128, 512);
                  // dS_j starts from zero in every block
                  const uint32_t acc = (st > 0 || tc > 0 || kk > 0) ? 1u : 0u;
                  mma_tf32_ts(dS, ahi + kk * 8, dh, idesc_u, acc);
                  mma_tf32_ts(dS, ahi + kk * 8, dl, idesc_u, 1u);
                  mma_tf32_ts(dS, alo + kk * 8, dh, idesc_u, 1u);
                }
                mma_commit(&stg_free[b]);
              }
              mma_commit(&v_free[vs]);
            }
          }
          if (ok) mma_commit(u_done);
        }
      }
      mma_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0)) {
        if (globaltimer_ns() - t0 > 2000000000ull) {
          atomicCAS(p.status, 0, kErrMomDrain);
          break;
        }
      }
    }
  } else {
    // -------------------------------------------------------------- generators
    // two warps per TMEM lane quarter: `half` 0 (warps 2..5) and 1 (warps 6..9);
    // thread t owns TMEM lane t, each half owns half of every chunk's columns
    constexpr int HC = DVP / 2;                          // state / output columns per half
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int t = quarter * 32 + lane;                   // TMEM lane = token or feature
    const uint32_t la = tmem + ((uint32_t)(quarter * 32) << 16);
    int stg_use = 0, sb_use = 0, out_use = 0;
    bool ok = true;
    float* myrow = X + t * xs;
    const int dh = (p.d + 1) / 2;                        // row elements loaded by each half
    const int a0 = half * dh, a1 = min(p.d, a0 + dh);
    const int64_t col_stride = p.dv + 1;
    float* part_h = p.part + ((int64_t)g * p.bh + h) * p.n * col_stride;
    float* master_h = p.master + ((int64_t)g * p.bh + h) * (int64_t)(FT * kRows) * DVP;
    float* xch = sden + FT * kRows;                      // [2][128] exchange for the denominators
    float* sdx = xch + 2 * kRows;                        // [FT*128] exchange for the sden sums
    for (int64_t c = 0; ok && c < nb; ++c) {
      const int64_t b0 = c * p.bs;
      const int64_t b1 = min(b0 + (int64_t)p.bs, p.n);
      // ---------------- query phase: tokens of block c read S_{<c}
      if (c == 0) {
        for (int64_t i = b0 + t + half * kRows; i < b1; i += 2 * kRows) {
          float* dst = part_h + i * col_stride;
          for (int col = 0; col <= p.dv; ++col) dst[col] = 0.0f;
        }
      } else {
        if (!mbar_wait(u_done, (int)((c - 1) & 1), ab, kErrMomWait)) { ok = false; break; }
        tc_fence_after();
        const int nsq = (int)((b1 - b0 + kRows - 1) / kRows);  // query sub-tiles of block c
        for (int st = 0; ok && st < nsq; ++st) {
          const int64_t i = b0 + (int64_t)st * kRows + t;
          const bool valid = i < b1;
          gen_sync();  // X is free, and sden of the previous update phase is visible
          for (int a = a0; a < a1; ++a) myrow[a] = valid ? __ldg(qh + i * p.d + a) * p.scale : 0.0f;
          if (half == 0) myrow[p.d] = 1.0f;
          gen_sync();
          float den_acc = 0.0f;
          float acc[HC];
#pragma unroll
          for (int u = 0; u < HC; ++u) acc[u] = 0.0f;
          for (int j = 0; ok && j < ntiles; ++j, ++sb_use) {
            // state row of feature t of tile j, this half's columns: fold dS_j (first sub-tile)
            // into the fp32 master and write its hi/lo split into the K-major B buffer
            const int sb = sb_use & 1;
            if (sb_use >= 2 && !mbar_wait(&sb_free[sb], ((sb_use >> 1) - 1) & 1, ab, kErrMomWait)) { ok = false; break; }
            uint8_t* bhi = sbuf + sb * L::kSbuf;
            uint8_t* blo = bhi + L::kSbufHalf;
            const uint32_t atom = (uint32_t)(t >> 5) * (DVP * 128);
            float4* mrow = reinterpret_cast<float4*>(master_h + (int64_t)(j * kRows + t) * DVP + half * HC);
            float sv[HC];
            if (st == 0) {
              tmem_ld_cols<HC>(la + j * DVP + half * HC, sv);
              if (c >= 2) {
#pragma unroll
                for (int u4 = 0; u4 < HC / 4; ++u4) {
                  const float4 m4 = mrow[u4];
                  sv[4 * u4 + 0] += m4.x;
                  sv[4 * u4 + 1] += m4.y;
                  sv[4 * u4 + 2] += m4.z;
                  sv[4 * u4 + 3] += m4.w;
                }
              }
#pragma unroll
              for (int u4 = 0; u4 < HC / 4; ++u4)
                mrow[u4] = make_float4(sv[4 * u4], sv[4 * u4 + 1], sv[4 * u4 + 2], sv[4 * u4 + 3]);
            } else {
#pragma unroll
              for (int u4 = 0; u4 < HC / 4; ++u4) {
                const float4 m4 = mrow[u4];
                sv[4 * u4 + 0] = m4.x;
                sv[4 * u4 + 1] = m4.y;
                sv[4 * u4 + 2] = m4.z;
                sv[4 * u4 + 3] = m4.w;
              }
            }
#pragma unroll
            for (int u = 0; u < HC; ++u) {
              const int nrow = half * HC + u;
              const uint32_t chunk = ((uint32_t)((t & 31) >> 2)) ^ (uint32_t)(nrow & 7);
              const uint32_t off = atom + nrow * 128 + chunk * 16 + (t & 3) * 4;
              const float hi = __uint_as_float(to_tf32(sv[u]));
              *reinterpret_cast<float*>(bhi + off) = hi;
              *reinterpret_cast<float*>(blo + off) = sv[u] - hi;
            }
            tc_fence_before();   // the dS_j reads are ordered before the MMAs that reuse its columns
            fence_proxy_async_smem();
            mbar_arrive(&sb_full[sb]);
            // Phi_q chunks of tile j for this thread's token: 16 features per half
            for (int kc = 0; kc < kRows / kChunk; ++kc, ++stg_use) {
              const int b = stg_use & 1;
              if (stg_use >= 2 && !mbar_wait(&stg_free[b], ((stg_use >> 1) - 1) & 1, ab, kErrMomWait)) { ok = false; break; }
              uint32_t hi[16], lo[16];
              const int fl = j * kRows + kc * kChunk + half * 16;
#pragma unroll
              for (int u = 0; u < 16; ++u) {
                const uint32_t pk = ftab[fl + u];
                float phi = 0.0f;
                if (pk != 0xFFFFFFFFu) {
                  phi = myrow[pk & 1023] * myrow[(pk >> 10) & 1023];
                  if (DEG3) phi *= myrow[pk >> 20];
                }
                den_acc = fmaf(phi, sden[fl + u], den_acc);
                hi[u] = to_tf32(phi);
                lo[u] = __float_as_uint(phi - __uint_as_float(hi[u]));
              }
              tmem_st16(la + L::kStg + b * 2 * kChunk + half * 16, hi);
              tmem_st16(la + L::kStg + b * 2 * kChunk + kChunk + half * 16, lo);
              tmem_wait_st();
              tc_fence_before();
              mbar_arrive(&stg_full[b]);
            }
            if (!ok) break;
            // Out of the previous tile (its MMAs overlap this tile's generation)
            if (j >= 1) {
              if (!mbar_wait(out_full, out_use & 1, ab, kErrMomWait)) { ok = false; break; }
              ++out_use;
              tc_fence_after();
              float ov[HC];
              tmem_ld_cols<HC>(la + (j - 1) * DVP + half * HC, ov);
#pragma unroll
              for (int u = 0; u < HC; ++u) acc[u] += ov[u];
            }
          }
          if (!ok) break;
          if (!mbar_wait(out_full, out_use & 1, ab, kErrMomWait)) { ok = false; break; }
          ++out_use;
          tc_fence_after();
          {
            float ov[HC];
            tmem_ld_cols<HC>(la + (ntiles - 1) * DVP + half * HC, ov);
#pragma unroll
            for (int u = 0; u < HC; ++u) acc[u] += ov[u];
          }
          tc_fence_before();
          mbar_arrive(out_free);
          xch[half * kRows + t] = den_acc;
          gen_sync();
          if (valid) {
            float* dst = part_h + i * col_stride;
#pragma unroll
            for (int u = 0; u < HC; ++u)
              if (half * HC + u < p.dv) dst[half * HC + u] = acc[u];
            if (half == 0) dst[p.dv] = xch[t] + xch[kRows + t];
          }
        }
      }
      if (!ok || c + 1 >= nb) continue;
      // ---------------- update phase: dS_j of block c
      float sd[FT];
#pragma unroll
      for (int j = 0; j < FT; ++j) sd[j] = 0.0f;
      for (int st = 0; ok && st < sub; ++st) {
        const int64_t t0 = b0 + (int64_t)st * kRows;
        gen_sync();  // everyone is done with X
        {
          const int64_t i = t0 + t;
          const bool valid = i < b1;
          for (int a = a0; a < a1; ++a) myrow[a] = valid ? __ldg(kh + i * p.d + a) : 0.0f;
          if (half == 0) myrow[p.d] = valid ? 1.0f : 0.0f;   // an invalid token's features are all zero
        }
        gen_sync();
        for (int tcn = 0; ok && tcn < kRows / kChunk; ++tcn) {
#pragma unroll
          for (int j = 0; j < FT; ++j) {
            if (!ok || j >= ntiles) break;
            const int b = stg_use & 1;
            if (stg_use >= 2 && !mbar_wait(&stg_free[b], ((stg_use >> 1) - 1) & 1, ab, kErrMomWait)) { ok = false; break; }
            ++stg_use;
            const uint32_t pk = ftab[j * kRows + t];
            const bool live = pk != 0xFFFFFFFFu;
            const int ia = live ? (int)(pk & 1023) : 0, ib = live ? (int)((pk >> 10) & 1023) : 0,
                      ic = live ? (int)(pk >> 20) : 0;
            const float cf = live ? key_coef_tc(ia, ib, ic, p.d) : 0.0f;
            uint32_t hi[16], lo[16];
            float fsum = 0.0f;
#pragma unroll
            for (int u = 0; u < 16; ++u) {
              const float* xr = X + (tcn * kChunk + half * 16 + u) * xs;
              float phi = xr[ia] * cf * xr[ib];
              if (DEG3) phi *= xr[ic];
              fsum += phi;
              hi[u] = to_tf32(phi);
              lo[u] = __float_as_uint(phi - __uint_as_float(hi[u]));
            }
            sd[j] += fsum;
            tmem_st16(la + L::kStg + b * 2 * kChunk + half * 16, hi);
            tmem_st16(la + L::kStg + b * 2 * kChunk + kChunk + half * 16, lo);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&stg_full[b]);
          }
        }
      }
      // s += the features of this block's keys: the halves' sums meet in shared memory
      if (half == 1) {
#pragma unroll
        for (int j = 0; j < FT; ++j)
          if (j < ntiles) sdx[j * kRows + t] = sd[j];
      }
      gen_sync();  // all reads of sden by the query phase are done; sdx is written
      if (half == 0) {
#pragma unroll
        for (int j = 0; j < FT; ++j)
          if (j < ntiles) sden[j * kRows + t] += sd[j] + sdx[j * kRows + t];
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
  const int xs = (d + 1) | 1;
  return 1024 + 2 * L::kSbuf + L::kVStages * L::kVStage + (size_t)kRows * xs * 4 + (size_t)L::kFT * kRows * 12 +
         2 * kRows * 4 + 16 + 17 * 8 + 16;
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
  if (dv > 64 || d > 128) return 0;
  const int dvp = dv <= 32 ? 32 : 64;
  const int ft = dvp == 32 ? MomLayout<32>::kFT : MomLayout<64>::kFT;
  const int64_t F = feature_count(d, degree);
  const int64_t tiles = (F + kRows - 1) / kRows;
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
                      cudaStream_t stream) {
  if (bh == 0 || n == 0) return SA_OK;
  const int G = moments_tc_groups(d, dv, degree);
  if (G <= 0) return set_error(SA_ERR_UNSUPPORTED, "tensor-core moments: shape not supported");
  if (bh > 65535) return set_error(SA_ERR_UNSUPPORTED, "too many sequences for one launch");
  MomTCParams prm{q, k, part, master, status, n, bh, d, dv, bs, (int)feature_count(d, degree), G, scale};
  if (degree == 3) return dv <= 32 ? launch_mom_tc<32, true>(maps, prm, stream) : launch_mom_tc<64, true>(maps, prm, stream);
  return dv <= 32 ? launch_mom_tc<32, false>(maps, prm, stream) : launch_mom_tc<64, false>(maps, prm, stream);
}

}  // namespace sa
