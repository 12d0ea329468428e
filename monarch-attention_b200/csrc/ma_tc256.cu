// tcgen05 / TMEM MonarchAttention forward for block size b = number of
// blocks M = 256 (N = 65536), head dim D = Dv = 128.
//
// A reference item (key block m of an R-step, index j of an L / output
// step) is 256 x 256 here, so a 128-row tile of it has 256 logit columns:
// GEMM1 is one M = 128, N = 256 MMA chain whose fp32 result fills 256 TMEM
// columns.  The tile's softmax runs on those columns; its 16-bit P is
// packed in place into columns 0..127 and GEMM2 (K = 256) writes O into
// columns 128..255, so one tile needs 256 TMEM columns and two CTAs share
// an SM.  One launch per phase (the phase boundary is the all-to-all
// between the (M, b) and (b, M) views), one tile per CTA:
//
//   R   (ma_torch.py:10-23; RF adds y, :38-52): rows j of key block m,
//        softmax over the 256 keys i of the block, al = P K[m], y = P V[m]
//   LS  (first half of ar_cr_ref, :26-35): rows l of index j, the
//        log-sum-exp over key blocks k of al_j q_l - cl[k] -> lse[j][l]
//   LA  (second half): rows k of index j; P^T[k][l] = exp(al_j[k] q_l -
//        cl[k] - lse[j][l]) are the reference's L[k][l] exactly; cr[k] =
//        sum_l P^T[k][l], ar[k] = P^T q_j.  The L-step contracts over the
//        256 query rows l, which a 128-row tile of rows l cannot finish on
//        its own: the statistics pass makes the L weights column-local.
//   O   (:55-62): rows l of index j, softmax over k, z = P y_j.
//
// Warps 0-3: softmax and epilogue (thread i = TMEM lane = tile row i);
// warp 4: TMEM allocation, and lane 0 issues every TMA copy and MMA.
// Every wait is bounded (MA_STATUS_WAIT_TIMEOUT, abort flag); no named
// barriers; TMA loads without multicast.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdlib.h>
#include <string.h>

#include "ma_common.cuh"
#include "ma_tc_ptx.cuh"

namespace ma {
namespace tc256 {

using namespace ma::tc;

constexpr int kRows = 128;                    // tile rows = TMEM lanes
constexpr int kCols = 256;                    // logit columns = b = M
constexpr int kThreads = 160;                 // 4 softmax / epilogue warps + 1 issue warp
constexpr int kIssueWarp = 4;
constexpr int kAHalf = kRows * 128;           // 16 KB: 128 rows x 64 columns (SW128)
constexpr int kABytes = 2 * kAHalf;           // 32 KB
constexpr int kBHalf = kCols * 128;           // 32 KB: 256 rows x 64 columns
constexpr int kBBytes = 2 * kBHalf;           // 64 KB
constexpr uint32_t kTmemCols = 256;
// small region: barriers, TMEM address, vectors
constexpr int kOffBar = 0;
constexpr int kOffTmem = 128;
constexpr int kOffVecB = 256;                 // per-row vector (cr[j] or cl[k]): 128 fp32
// The per-column term of LS / LA / output tiles (cl[k] or lse[l]) is
// subtracted on the tensor core by a ninth K step of GEMM1: A_ext (128 rows:
// -1, -1, 0 ...) times B_ext (256 rows: the term split into a 16-bit value
// and the 16-bit rounding of its remainder, 0 ...), K-major without
// swizzle (8-row core matrices of 16-byte rows 128 B apart; the K = 8..15
// half read from a zero block).
constexpr int kOffExtA = 1024;                // A_ext: 128 x 16 B
constexpr int kOffExtB = kOffExtA + 2048;     // B_ext: 256 x 16 B (clx / lsex rows)
constexpr int kOffZero = kOffExtB + 4096;     // 4 KB of zeros
constexpr int kSmallBytes = kOffZero + 4096;
constexpr int kSmemBytes = kSmallBytes + 1024 + kABytes + kBBytes;  // + alignment pad

// barriers (8 B each)
constexpr int kBarFull = 0;     // A, B and the vectors landed
constexpr int kBarS = 8;        // GEMM1 done (S in TMEM)
constexpr int kBarP = 16;       // P written to TMEM (128 arrivals)
constexpr int kBarX = 24;       // late X tile (V or y_j) landed in B
constexpr int kBarO = 32;       // GEMM2 done (one phase per part)
constexpr int kBarStaged = 40;  // output tile staged in SMEM (128 arrivals per part)
constexpr int kBarDrain = 48;   // issued MMAs complete (after an abort)
constexpr int kBarX2 = 56;      // R-final: V rows 128..255 landed in B

enum Kind : int { K_R = 0, K_RF = 1, K_LS = 2, K_LA = 3, K_O = 4 };

struct Params {
  CUtensorMap tm_qblk;   // q (D, N, H, E): 64 x 128 token rows
  CUtensorMap tm_kblk;
  CUtensorMap tm_vblk;
  CUtensorMap tm_qstr;   // q as (D, b, M, H, E): 64 x 1 x 128 -> tokens l*b + j
  CUtensorMap tm_al;     // al rows [head][j][m]: 64 x 128
  CUtensorMap tm_ar;     // ar rows [head][m][j]
  CUtensorMap tm_y;      // y rows  [head][j][m]
  CUtensorMap tm_al_st;  // al as (D, M, heads*b): 64 x 1 x 128 (rows j of block m)
  CUtensorMap tm_y_st;
  CUtensorMap tm_ar_st;  // ar as (D, b, heads*M): rows k of index j
  CUtensorMap tm_out_st; // out as (Dv, b, M, H, E): tokens l*b + j
  float* cl;             // [head][j][m]
  uint4* clx;            // cl as B_ext rows: (hi, lo) 16-bit pair padded to 16 bytes
  float* cr;             // [head][m][j]
  uint4* lsex;           // [head][j][l]: log-sum-exp of the L-step rows, as B_ext rows
  uint32_t* abort;
  uint32_t* status;
  uint32_t* status_host;  // host mirror of the status word (optional)
  int H;
  int heads;             // E * H
  int first;             // R-step of round 0: A = q blocks, cr = 1
  float sm_scale;
  unsigned long long timeout_ns;
};

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// 128 fp32 accumulator columns of this lane -> scaled 16-bit into a 128-row
// SW128 staging tile (row r of column half h at h*hstride + r*128, 16-byte
// unit c at c ^ (r & 7)); 16-column chunks, the next one's load in flight
template <bool BF16>
__device__ __forceinline__ void stage_row(uint32_t tile, uint32_t hstride, int row, uint32_t taddr,
                                          float scale) {
  uint32_t ca[16], cb[16];
  const uint32_t rbase = tile + row * 128;
  const uint64_t sc2 = f2pack(scale, scale);
  auto put = [&](const uint32_t(&cv)[16], int ch) {
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      uint32_t w[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        w[q] = scale_pack2<BF16>(cv[8 * t + 2 * q], cv[8 * t + 2 * q + 1], sc2);
      const int u = 2 * ch + t;
      st_shared_v4(rbase + (u >> 3) * hstride + (((u & 7) ^ (row & 7)) << 4), w[0], w[1], w[2],
                   w[3]);
    }
  };
  tmem_ld16(taddr, ca);
  tmem_wait_ld();
#pragma unroll 1
  for (int ch = 0; ch < 8; ch += 2) {
    tmem_ld16(taddr + 16 * (ch + 1), cb);
    put(ca, ch);
    tmem_wait_ld();
    if (ch + 2 < 8) tmem_ld16(taddr + 16 * (ch + 2), ca);
    put(cb, ch + 1);
    tmem_wait_ld();
  }
}

template <bool BF16, int KIND>
__global__ void __launch_bounds__(kThreads, 2) tc256_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t sbase = smem_u32(smem_raw);
  const uint32_t A = (sbase + kSmallBytes + 1023u) & ~1023u;  // SW128 tiles
  const uint32_t B = A + kABytes;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const Guard guard{p.abort, p.status, p.timeout_ns, p.status_host};
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem_raw + kOffTmem);
  const float* vecB = reinterpret_cast<const float*>(smem_raw + kOffVecB);
  auto bar = [&](int off) { return sbase + kOffBar + off; };
  constexpr bool has_o = KIND != K_LS;
  constexpr int parts = KIND == K_RF ? 2 : 1;
  const int ntiles = p.heads * 2 * kCols;

  // tile -> (head, item, row tile): rows 128*rt .. 128*rt + 127 of item m
  // (R steps) or j (L / output) of a head
  struct TileId {
    int head, item, rt, eb, hh, hrow;
  };
  auto tile_id = [&](int t) {
    TileId d;
    d.head = t / (2 * kCols);
    d.item = (t >> 1) % kCols;
    d.rt = t & 1;
    d.eb = d.head / p.H;
    d.hh = d.head - d.eb * p.H;
    d.hrow = d.head * kCols;  // first row of the head in [b][M] / [M][b] arrays
    return d;
  };

  if (tid == 0) {
    mbar_init(bar(kBarFull), 1);
    mbar_init(bar(kBarS), 1);
    mbar_init(bar(kBarP), kRows);
    mbar_init(bar(kBarX), 1);
    mbar_init(bar(kBarO), 1);
    mbar_init(bar(kBarStaged), kRows);
    mbar_init(bar(kBarDrain), 1);
    mbar_init(bar(kBarX2), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = tid; i < 256; i += kThreads) {  // A_ext rows (-1, -1, 0 ...) and the zero block
    const uint32_t m1 = BF16 ? 0xBF80BF80u : 0xBC00BC00u;
    if (i < kRows) st_shared_v4(sbase + kOffExtA + i * 16, m1, 0u, 0u, 0u);
    st_shared_v4(sbase + kOffZero + i * 16, 0u, 0u, 0u, 0u);
  }
  fence_proxy_async_smem();
  if (warp == kIssueWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == kIssueWarp) {
    // ===================== TMA + MMA issue (one thread) =====================
    // The CTA walks its tiles t = blockIdx.x, + gridDim.x, ...  A tile's
    // loads are issued while the previous tile finishes: B (and the vectors)
    // as soon as the previous GEMM2 has read B, A once the previous output
    // store has read its staging in A.
    if (lane == 0) {
      const uint64_t keep = policy_evict_last(), once = policy_evict_first();
      const uint32_t fb = bar(kBarFull);
      const uint32_t va = sbase + kOffExtB, vb = sbase + kOffVecB;
      uint32_t vbytes = 0;
      if (KIND == K_R || KIND == K_RF) vbytes = p.first ? 0 : 512;  // cr[m][j-tile]
      if (KIND == K_LS || KIND == K_O) vbytes = 4096;               // cl[j][:] rows
      if (KIND == K_LA) vbytes = 4096 + 512;                        // lse[j][:] rows, cl[j][k-tile]
      auto load_vec = [&](const TileId& d) {
        if (KIND == K_R || KIND == K_RF) {
          if (!p.first)
            bulk_load(vb, p.cr + (size_t)(d.hrow + d.item) * kCols + d.rt * kRows, 512, fb);
        } else if (KIND == K_LS || KIND == K_O) {
          bulk_load(va, p.clx + (size_t)(d.hrow + d.item) * kCols, 4096, fb);
        } else {
          bulk_load(va, p.lsex + (size_t)(d.hrow + d.item) * kCols, 4096, fb);
          bulk_load(vb, p.cl + (size_t)(d.hrow + d.item) * kCols + d.rt * kRows, 512, fb);
        }
      };
      auto load_b = [&](const TileId& d) {
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2)
          for (int r2 = 0; r2 < 2; ++r2) {
            const uint32_t dst = B + h2 * kBHalf + r2 * kAHalf;
            if (KIND == K_R || KIND == K_RF)  // k block m (256 tokens)
              tma_load_4d_h(dst, &p.tm_kblk, h2 * 64, d.item * kCols + r2 * kRows, d.hh, d.eb, fb,
                            KIND == K_RF ? once : keep);
            else if (KIND == K_LS || KIND == K_O)  // al_j (rows k)
              tma_load_2d_h(dst, &p.tm_al, h2 * 64, (d.hrow + d.item) * kCols + r2 * kRows, fb,
                            KIND == K_O ? once : keep);
            else  // q_j (all 256 rows l)
              tma_load_5d_h(dst, &p.tm_qstr, h2 * 64, d.item, r2 * kRows, d.hh, d.eb, fb, keep);
          }
      };
      auto load_a = [&](const TileId& d) {
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const uint32_t dst = A + h2 * kAHalf;
          if (KIND == K_R || KIND == K_RF) {  // rows j of ar[m] (or of the q block)
            if (p.first)
              tma_load_4d_h(dst, &p.tm_qblk, h2 * 64, d.item * kCols + d.rt * kRows, d.hh, d.eb,
                            fb, keep);
            else
              tma_load_2d_h(dst, &p.tm_ar, h2 * 64, (d.hrow + d.item) * kCols + d.rt * kRows, fb,
                            once);
          } else if (KIND == K_LS || KIND == K_O) {  // q_j rows l (tokens l*b + j)
            tma_load_5d_h(dst, &p.tm_qstr, h2 * 64, d.item, d.rt * kRows, d.hh, d.eb, fb, keep);
          } else {  // al_j rows k
            tma_load_2d_h(dst, &p.tm_al, h2 * 64, (d.hrow + d.item) * kCols + d.rt * kRows, fb,
                          once);
          }
        }
      };
      constexpr uint32_t id1 = idesc_f16(BF16, false, false, kRows, kCols);
      constexpr uint32_t id2 = idesc_f16(BF16, false, true, kRows, 128);
      bool ok = true;
      bool pending = false;  // loads of the next tile in flight
      uint32_t full_phase = 0;
      int x_it = -1, x2_it = -1;  // tile iterations whose late X / X2 loads were issued
      int t = blockIdx.x;
      if (t < ntiles) {
        const TileId d0 = tile_id(t);
        mbar_expect_tx(fb, kABytes + kBBytes + vbytes);
        load_vec(d0);
        load_b(d0);
        load_a(d0);
        pending = true;
      }
      for (int it = 0; ok && t < ntiles; ++it, t += gridDim.x) {
        const TileId d = tile_id(t);
        const int tn = t + gridDim.x;
        const bool has_next = tn < ntiles;
        const TileId dn = tile_id(has_next ? tn : t);
        const uint32_t ph = it & 1;
        ok = wait_bar(fb, full_phase & 1, guard);
        ++full_phase;
        pending = false;
        if (!ok) break;
        // ---- GEMM1: S (128 x 256) = A B^T, both K-major ----
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t offa = (kk >> 2) * kAHalf + (kk & 3) * 32;
          const uint32_t offb = (kk >> 2) * kBHalf + (kk & 3) * 32;
          mma_ss(tmem, smem_desc(A + offa, 16, 1024, kSwz128),
                 smem_desc(B + offb, 16, 1024, kSwz128), id1, kk > 0);
        }
        if (KIND == K_LS || KIND == K_LA || KIND == K_O) {  // S - column term: ninth K step
          const uint32_t xa = sbase + kOffExtA, xb = sbase + kOffExtB, z = sbase + kOffZero;
          mma_ss(tmem, smem_desc(xa, z - xa, 128, kSwzNone), smem_desc(xb, z - xb, 128, kSwzNone),
                 id1, 1);
        }
        mma_commit(bar(kBarS));
        if (KIND == K_LS) {
          // no GEMM2: A and B are free once GEMM1 ran, the vectors once the
          // softmax is done with them (and with S)
          ok = wait_bar(bar(kBarS), ph, guard);
          if (ok && has_next) {
            mbar_expect_tx(fb, kABytes + kBBytes + vbytes);
            load_b(dn);
            load_a(dn);
            pending = true;
          }
          if (ok) ok = wait_bar(bar(kBarP), ph, guard);
          if (ok && has_next) load_vec(dn);
          continue;
        }
        // R-final: V rows 0..127 to A once GEMM1 has read it; out: y_j to B
        if (KIND == K_RF || KIND == K_O) {
          ok = wait_bar(bar(kBarS), ph, guard);
          if (!ok) break;
          x_it = it;
          if (KIND == K_RF) {
            mbar_expect_tx(bar(kBarX), kABytes);
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2)
              tma_load_4d_h(A + h2 * kAHalf, &p.tm_vblk, h2 * 64, d.item * kCols, d.hh, d.eb,
                            bar(kBarX), once);
          } else {
            fence_proxy_async_global();
            mbar_expect_tx(bar(kBarX), kBBytes);
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2)
              for (int r2 = 0; r2 < 2; ++r2)
                tma_load_2d_h(B + h2 * kBHalf + r2 * kAHalf, &p.tm_y, h2 * 64,
                              (d.hrow + d.item) * kCols + r2 * kRows, bar(kBarX), once);
          }
        }
        // ---- GEMM2 part(s): O (128 x 128) = P (TMEM, K = 256) X, then store ----
        for (int part = 0; ok && part < parts; ++part) {
          const uint32_t ophase = (uint32_t)(it * parts + part) & 1;
          if (part == 0) {
            ok = wait_bar(bar(kBarP), ph, guard);
            if (ok && KIND == K_O) ok = wait_bar(bar(kBarX), ph, guard);
          } else {
            // R-final second part: V rows 0..127 in A, rows 128..255 in B
            ok = wait_bar(bar(kBarX), ph, guard) && wait_bar(bar(kBarX2), ph, guard);
          }
          if (!ok) break;
          tc_fence_after();
          if (part == 0) {
#pragma unroll
            for (int kk = 0; kk < 16; ++kk)
              mma_ts(tmem + 128, tmem + kk * 8, smem_desc(B + kk * 2048, kBHalf, 1024, kSwz128),
                     id2, kk > 0);
          } else {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              mma_ts(tmem + 128, tmem + kk * 8, smem_desc(A + kk * 2048, kAHalf, 1024, kSwz128),
                     id2, kk > 0);
#pragma unroll
            for (int kk = 8; kk < 16; ++kk)
              mma_ts(tmem + 128, tmem + kk * 8,
                     smem_desc(B + kAHalf + (kk - 8) * 2048, kBHalf, 1024, kSwz128), id2, 1);
          }
          mma_commit(bar(kBarO));
          // this GEMM2 finished reading B: R-final's first part hands rows
          // 128..255 of B to V; the last part hands B to the next tile
          ok = wait_bar(bar(kBarO), ophase, guard);
          if (!ok) break;
          if (KIND == K_RF && part == 0) {
            x2_it = it;
            mbar_expect_tx(bar(kBarX2), kABytes);
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2)
              tma_load_4d_h(B + h2 * kBHalf + kAHalf, &p.tm_vblk, h2 * 64, d.item * kCols + kRows,
                            d.hh, d.eb, bar(kBarX2), once);
          }
          if (part == parts - 1 && has_next) {
            mbar_expect_tx(fb, kABytes + kBBytes + vbytes);
            load_vec(dn);
            load_b(dn);
            pending = true;
          }
          // ---- store the staged output tile ----
          ok = wait_bar(bar(kBarStaged), ophase, guard);
          if (!ok) break;
          // staging: R-final's al in the rows 0..127 of B, everything else in A
          const bool in_b = KIND == K_RF && part == 0;
          const uint32_t src = in_b ? B : A, hstride = in_b ? kBHalf : kAHalf;
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const uint32_t s2 = src + h2 * hstride;
            if (KIND == K_R || KIND == K_RF)
              tma_store_3d_h(part == 0 ? &p.tm_al_st : &p.tm_y_st, s2, h2 * 64, d.item,
                             d.hrow + d.rt * kRows, keep);
            else if (KIND == K_LA)
              tma_store_3d_h(&p.tm_ar_st, s2, h2 * 64, d.item, d.hrow + d.rt * kRows, keep);
            else
              tma_store_5d_h(&p.tm_out_st, s2, h2 * 64, d.item, d.rt * kRows, d.hh, d.eb, once);
          }
          bulk_commit();
          bulk_wait_read<0>();
        }
        if (ok && has_next) load_a(dn);  // the staging in A has been read
      }
      bulk_wait<0>();  // never leave with stores in flight
      if (!ok) {
        // After an abort: loads of the next tile may be in flight, and MMAs
        // this thread issued may still run; let both finish (bounded)
        // before the CTA releases shared memory and TMEM.
        const uint64_t t0 = globaltimer();
        while (pending && !mbar_try(fb, full_phase & 1) && globaltimer() - t0 < guard.limit) {
        }
        while (x_it >= 0 && !mbar_try(bar(kBarX), x_it & 1) && globaltimer() - t0 < guard.limit) {
        }
        while (x2_it >= 0 && !mbar_try(bar(kBarX2), x2_it & 1) && globaltimer() - t0 < guard.limit) {
        }
        mma_commit(bar(kBarDrain));
        const uint64_t t1 = globaltimer();
        while (!mbar_try(bar(kBarDrain), 0) && globaltimer() - t1 < guard.limit) {
        }
      }
    }
  } else {
    // ===================== softmax + epilogue (warps 0-3) =====================
    const int row = tid;  // TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_off, tO = tS + 128;
    bool ok = true;
    for (int it = 0, t = blockIdx.x; ok && t < ntiles; ++it, t += gridDim.x) {
      const TileId d = tile_id(t);
      const uint32_t ph = it & 1;
      ok = wait_bar_warp(bar(kBarFull), ph, guard) && wait_bar_warp(bar(kBarS), ph, guard);
      if (!ok) break;
      tc_fence_after();
      float scale_out = 1.0f;
      // per-row constant (log2 units) and exponent slope
      float u_a = kLog2e, rowc = 0.0f;
      if (KIND == K_R || KIND == K_RF) {
        const float crj = p.first ? 1.0f : vecB[row];
        u_a = p.sm_scale / (crj + kEps) * kLog2e;  // t = sm_scale * S / (cr + eps) (ma_torch.py:11-12)
      } else if (KIND == K_LA) {
        rowc = vecB[row];  // cl[k] of this row
      }
      // pass 1: row maximum of the exponent argument (not needed for LA,
      // whose normaliser lse[l] is known)
      float mx = 0.0f;
      if (KIND != K_LA) {
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t sv[64];
          tmem_ld32(tS + 64 * c, *reinterpret_cast<uint32_t(*)[32]>(sv));
          tmem_ld32(tS + 64 * c + 32, *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
          tmem_wait_ld();
          // (LS / output tiles: S already holds x = S - cl[k], from GEMM1)
#pragma unroll
          for (int i = 0; i < 64; ++i) mx4[i & 3] = fmaxf(mx4[i & 3], __uint_as_float(sv[i]));
        }
        mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      }
      // exponent in log2 units: u = u_a * S + u_b (for LS / O, S - cl[k];
      // for LA, S - lse[l]: GEMM1 subtracted the column term)
      float u_b;
      if (KIND == K_R || KIND == K_RF) {
        const float mxt = fmaxf(u_a * kLn2 * mx, kEps);  // clamp(max, eps) of t (:14-16)
        u_b = -mxt * kLog2e;
      } else if (KIND == K_LA) {
        u_b = -rowc * kLog2e;
      } else {
        u_b = -mx * kLog2e;
      }
      // pass 2 in 16-column chunks (next chunk's TMEM load in flight), two
      // columns per f32x2 instruction; P of chunk ch as packed 16-bit pairs
      // into TMEM columns 8 ch .. 8 ch + 7 (S columns already read)
      float s4[4] = {0.f, 0.f, 0.f, 0.f}, w4[4] = {0.f, 0.f, 0.f, 0.f};
      {
        uint64_t s2[2] = {0ull, 0ull}, w2[2] = {0ull, 0ull};
        const uint64_t ua2 = f2pack(u_a, u_a), ub2 = f2pack(u_b, u_b);
        uint32_t ca[16], cb[16];
        auto exp_chunk = [&](uint32_t(&cv)[16], int ch) {
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const uint64_t u2 =
                ffma2(f2pack(__uint_as_float(cv[2 * t]), __uint_as_float(cv[2 * t + 1])), ua2, ub2);
            float u0, u1;
            f2unpack(u2, u0, u1);
            const float e0 = ex2(u0), e1 = ex2(u1);
            const uint64_t e2 = f2pack(e0, e1);
            s2[t & 1] = fadd2(s2[t & 1], e2);
            if (KIND == K_R || KIND == K_RF) w2[t & 1] = ffma2(e2, u2, w2[t & 1]);
            cv[2 * t] = __float_as_uint(e0);
            cv[2 * t + 1] = __float_as_uint(e1);
          }
          if (KIND != K_LS) {
            uint32_t pk[8];
#pragma unroll
            for (int t = 0; t < 8; ++t)
              pk[t] = pack2<BF16>(__uint_as_float(cv[2 * t]), __uint_as_float(cv[2 * t + 1]));
            tmem_st8(tS + 8 * ch, pk);
          }
        };
        tmem_ld16(tS, ca);
        tmem_wait_ld();
#pragma unroll 1
        for (int ch = 0; ch < 16; ch += 2) {
          tmem_ld16(tS + 16 * (ch + 1), cb);
          exp_chunk(ca, ch);
          tmem_wait_ld();
          if (ch + 2 < 16) tmem_ld16(tS + 16 * (ch + 2), ca);
          exp_chunk(cb, ch + 1);
          tmem_wait_ld();
        }
        f2unpack(s2[0], s4[0], s4[1]);
        f2unpack(s2[1], s4[2], s4[3]);
        f2unpack(w2[0], w4[0], w4[1]);
        f2unpack(w2[1], w4[2], w4[3]);
      }
      const float sum = (s4[0] + s4[1]) + (s4[2] + s4[3]);
      if (KIND == K_R || KIND == K_RF) {
        const float wsum = (w4[0] + w4[1]) + (w4[2] + w4[3]);
        const float den = sum + kEps;  // r = e / (sum + eps), :17
        const float inv = 1.0f / den;
        // cl[j][m] = sum_i r_i log r_i (:20); this row is j = 128*rt + row;
        // fp32 for the LA tiles' rows, and as the B_ext row of the GEMM1 step
        // of LS / output tiles (16-bit value + 16-bit remainder)
        const float clv = kLn2 * inv * wsum - __logf(den) * sum * inv;
        const size_t ci = (size_t)(d.hrow + d.rt * kRows + row) * kCols + d.item;
        p.cl[ci] = clv;
        const float hi = round16<BF16>(clv);
        p.clx[ci] = make_uint4(pack2<BF16>(hi, clv - hi), 0u, 0u, 0u);
        scale_out = inv;
      } else if (KIND == K_LS) {
        // lse[j][l] = max_k x + log(sum_k exp(x - max)), as the B_ext row of
        // the GEMM1 step of LA tiles
        const float lse = mx + __logf(sum);
        const float hi = round16<BF16>(lse);
        p.lsex[(size_t)(d.hrow + d.item) * kCols + d.rt * kRows + row] =
            make_uint4(pack2<BF16>(hi, lse - hi), 0u, 0u, 0u);
      } else if (KIND == K_LA) {
        // cr[k][j] = sum_l L[k][l] (:32); this row is k = 128*rt + row
        p.cr[(size_t)(d.hrow + d.rt * kRows + row) * kCols + d.item] = sum;
      } else {
        scale_out = 1.0f / sum;
      }
      // P written (TMEM), S and the vectors no longer read
      if (has_o) tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(kBarP));
      // ---- epilogue: O -> scaled 16-bit -> staging tile -> TMA store ----
      for (int part = 0; has_o && part < parts; ++part) {
        const uint32_t ophase = (uint32_t)(it * parts + part) & 1;
        if (!wait_bar_warp(bar(kBarO), ophase, guard)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float sc = scale_out;                                       // z (:60-62), y (:51)
        if ((KIND == K_R || KIND == K_RF) && part == 0) sc = p.sm_scale * scale_out;  // al (:21)
        if (KIND == K_LA) sc = 1.0f;                                // ar (:34)
        // R-final: al into the rows 0..127 of B (A holds V rows 0..127 for
        // the second part), y into A (free once that part ran); else A
        const bool in_b = KIND == K_RF && part == 0;
        stage_row<BF16>(in_b ? B : A, in_b ? kBHalf : kAHalf, row, tO, sc);
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(bar(kBarStaged));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kIssueWarp) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

static bool encode(CUtensorMap* tm, CUtensorMapDataType dt, int rank, const void* base,
                   const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box) {
  auto fn = get_encode();
  if (!fn) return false;
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  cuuint64_t gd[5], gs[4];
  cuuint32_t bx[5];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
  }
  for (int i = 0; i < rank - 1; ++i) gs[i] = strides_bytes[i];
  return fn(tm, dt, (cuuint32_t)rank, const_cast<void*>(base), gd, gs, bx, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool BF16, int KIND>
static cudaError_t launch_kind(const Params& prm, int heads, cudaStream_t st) {
  auto kfn = tc256_kernel<BF16, KIND>;
  cudaError_t err =
      cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (err != cudaSuccess) return err;
  int dev = 0, sms = 0;
  err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (err != cudaSuccess) return err;
  const int64_t tiles = (int64_t)heads * 2 * kCols;
  const int grid = (int)(tiles < 2LL * sms ? tiles : 2LL * sms);  // two resident CTAs per SM
  kfn<<<grid, kThreads, kSmemBytes, st>>>(prm);
  return cudaGetLastError();
}

template <bool BF16>
static cudaError_t launch(Params& prm, int kind, int heads, cudaStream_t st) {
  switch (kind) {
    case K_R: return launch_kind<BF16, K_R>(prm, heads, st);
    case K_RF: return launch_kind<BF16, K_RF>(prm, heads, st);
    case K_LS: return launch_kind<BF16, K_LS>(prm, heads, st);
    case K_LA: return launch_kind<BF16, K_LA>(prm, heads, st);
    default: return launch_kind<BF16, K_O>(prm, heads, st);
  }
}

}  // namespace tc256

static bool aligned16p(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

bool tc256_supports(const ma_fwd_params* p, const Shape& s) {
  const char* off = getenv("MA_DISABLE_TC");
  if (off && off[0] == '1') return false;
  if (p->dtype != MA_DTYPE_BF16 && p->dtype != MA_DTYPE_F16) return false;
  if (s.D != 128 || s.Dv != 128 || s.b != 256 || s.M != 256 || s.N != s.Np) return false;
  if (p->mask_dtype != MA_MASK_NONE) return false;
  const int64_t* st[4] = {p->q_stride, p->k_stride, p->v_stride, p->o_stride};
  for (int t = 0; t < 4; ++t) {
    if (st[t][3] != 1) return false;
    for (int i = 0; i < 3; ++i)
      if ((st[t][i] * 2) % 16 != 0 || st[t][i] <= 0) return false;
  }
  if (p->q && !(aligned16p(p->q) && aligned16p(p->k) && aligned16p(p->v) && aligned16p(p->out)))
    return false;
  return true;
}

cudaError_t run_tc256(const ma_fwd_params* p, const Shape& s, const WsLayout& ws, cudaStream_t st,
                      int* nlaunch) {
  using namespace tc256;
  Params prm;
  memset(&prm, 0, sizeof(prm));
  const CUtensorMapDataType dt =
      p->dtype == MA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int heads = s.E * s.H;
  bool ok = true;
  const uint32_t box_blk[4] = {64, kRows, 1, 1};
  auto tok_map = [&](CUtensorMap* tm, const void* base, const int64_t* es) {
    const uint64_t dims[4] = {(uint64_t)s.D, (uint64_t)s.N, (uint64_t)s.H, (uint64_t)s.E};
    const uint64_t str[3] = {(uint64_t)es[2] * 2, (uint64_t)es[1] * 2, (uint64_t)es[0] * 2};
    ok = ok && encode(tm, dt, 4, base, dims, str, box_blk);
  };
  tok_map(&prm.tm_qblk, p->q, p->q_stride);
  tok_map(&prm.tm_kblk, p->k, p->k_stride);
  tok_map(&prm.tm_vblk, p->v, p->v_stride);
  {
    const int64_t* es = p->q_stride;
    const uint64_t dims[5] = {(uint64_t)s.D, (uint64_t)s.b, (uint64_t)s.M, (uint64_t)s.H,
                              (uint64_t)s.E};
    const uint64_t str[4] = {(uint64_t)es[2] * 2, (uint64_t)es[2] * 2 * s.b, (uint64_t)es[1] * 2,
                             (uint64_t)es[0] * 2};
    const uint32_t box[5] = {64, 1, kRows, 1, 1};
    ok = ok && encode(&prm.tm_qstr, dt, 5, p->q, dims, str, box);
  }
  char* w = reinterpret_cast<char*>(p->workspace);
  const uint64_t rows = (uint64_t)heads * s.b * s.M;
  {
    const uint64_t dims[2] = {(uint64_t)s.D, rows};
    const uint64_t str[1] = {(uint64_t)s.D * 2};
    const uint32_t box[2] = {64, kRows};
    ok = ok && encode(&prm.tm_al, dt, 2, w + ws.al, dims, str, box);
    ok = ok && encode(&prm.tm_ar, dt, 2, w + ws.ar, dims, str, box);
    ok = ok && encode(&prm.tm_y, dt, 2, w + ws.y, dims, str, box);
  }
  {
    const uint32_t box3[3] = {64, 1, kRows};
    const uint64_t dal[3] = {(uint64_t)s.D, (uint64_t)s.M, (uint64_t)heads * s.b};
    const uint64_t sal[2] = {(uint64_t)s.D * 2, (uint64_t)s.M * s.D * 2};
    ok = ok && encode(&prm.tm_al_st, dt, 3, w + ws.al, dal, sal, box3);
    ok = ok && encode(&prm.tm_y_st, dt, 3, w + ws.y, dal, sal, box3);
    const uint64_t dar[3] = {(uint64_t)s.D, (uint64_t)s.b, (uint64_t)heads * s.M};
    const uint64_t sar[2] = {(uint64_t)s.D * 2, (uint64_t)s.b * s.D * 2};
    ok = ok && encode(&prm.tm_ar_st, dt, 3, w + ws.ar, dar, sar, box3);
    const int64_t* os = p->o_stride;
    const uint64_t dout[5] = {(uint64_t)s.Dv, (uint64_t)s.b, (uint64_t)s.M, (uint64_t)s.H,
                              (uint64_t)s.E};
    const uint64_t sout[4] = {(uint64_t)os[2] * 2, (uint64_t)os[2] * 2 * s.b,
                              (uint64_t)os[1] * 2, (uint64_t)os[0] * 2};
    const uint32_t box5[5] = {64, 1, kRows, 1, 1};
    ok = ok && encode(&prm.tm_out_st, dt, 5, p->out, dout, sout, box5);
  }
  if (!ok) return cudaErrorInvalidValue;
  prm.cl = reinterpret_cast<float*>(w + ws.cl);
  prm.cr = reinterpret_cast<float*>(w + ws.cr);
  prm.clx = reinterpret_cast<uint4*>(w + ws.clx);
  prm.lsex = reinterpret_cast<uint4*>(w + ws.lsex);
  if (ws.clx == 0 || ws.lsex == 0) return cudaErrorInvalidValue;  // layout without the rows
  prm.abort = reinterpret_cast<uint32_t*>(w + ws.ctrl) + 1;
  prm.status = p->status;
  prm.status_host = p->status_host;
  prm.H = s.H;
  prm.heads = heads;
  prm.sm_scale = s.sm_scale;
  prm.timeout_ns = 2000000000ull;
  const char* tmo = getenv("MA_WAIT_TIMEOUT_NS");
  if (tmo) prm.timeout_ns = strtoull(tmo, nullptr, 10);
  cudaError_t err = cudaMemsetAsync(w + ws.ctrl, 0, 64, st);
  if (err != cudaSuccess) return err;
  const bool bf = p->dtype == MA_DTYPE_BF16;
  auto run = [&](int kind) -> cudaError_t {
    cudaError_t e = bf ? launch<true>(prm, kind, heads, st) : launch<false>(prm, kind, heads, st);
    if (e == cudaSuccess) *nlaunch += 1;
    return e;
  };
  // T-1 rounds of (R, L statistics, L accumulation), the final R-step and the output
  for (int t = 0; t + 1 < s.T && err == cudaSuccess; ++t) {
    prm.first = t == 0;
    err = run(K_R);
    if (err == cudaSuccess) err = run(K_LS);
    if (err == cudaSuccess) err = run(K_LA);
  }
  prm.first = s.T == 1;
  if (err == cudaSuccess) err = run(K_RF);
  if (err == cudaSuccess) err = run(K_O);
  return err;
}

}  // namespace ma
