// Persistent tcgen05 / TMEM MonarchAttention forward (the kernel template;
// host side and dispatch in ma_tc.cu, explicit instantiations in
// ma_tc_inst_*.cu).  Shapes: block size b = BB and number of blocks M = MM
// each 32, 64 or 128, head dim D = Dv = DD 64 or 128, bf16 / fp16, N a
// multiple of b, optional key / query validity mask.  b = 256 runs in
// ma_tc256.cu.
//
// Work decomposition.  Per head (e, h) the reference runs 2T phases
// (ma/ma_torch.py:100-105):
//   phase 2t   (t < T)  : R-step t, one item per key block m      (al_cl_ref /
//                         al_y_cl_ref when t = T-1, ma_torch.py:10-23, 38-52)
//   phase 2t+1 (t < T-1): L-step t, one item per intra-block index j (ar_cr_ref,
//                         ma_torch.py:26-35)
//   phase 2T-1          : output, one item per j                    (z_ref, :55-62)
// An R item is a b x b logit block (rows j, columns: keys i of block m), an
// L / output item an M x M block (rows: query blocks l, columns: key blocks
// k).  A work unit ("tile") is one 128-row tcgen05 tile holding 128 / b R
// items or 128 / M L / output items stacked on top of each other; both GEMMs
// run over the full tile and the softmax of a row covers only its own
// item's column block, writing zeros to the rest of P, so the off-diagonal
// products drop out.  Every phase has b * M / 128 tiles.
//
// Every phase of a head needs *all* items of the previous phase of the same
// head (the (M,B) <-> (B,M) transpose between steps is an all-to-all inside
// the head).  Instead of one launch per phase, a single persistent kernel
// claims tiles from a global counter in a wavefront order -- round r holds
// phase p of head group r - p for every p -- so a tile's producer phase was
// claimed a whole round earlier and dependency waits are rare.  Completion
// is published per (head, phase) with a release counter and awaited with
// bounded acquire spins.  The intermediates of a head live in one of a few
// workspace slots, reused round-robin (slot reuse waits for the output phase
// of the head that used it before), so the live set stays L2-resident.
//
// CTA roles (512 threads, one CTA per SM):
//   warpgroups 0, 1  softmax; group g takes the tiles n with n % 2 == g
//                    (ping-pong), thread i owns row i = TMEM lane i; the
//                    group's thread 0 issues the tile's GEMM2 once P is ready
//   warpgroup 2      epilogue (O -> 16-bit staging in shared memory)
//   warp 12          scheduler + TMA producer (3-entry ring, 2 tiles each)
//   warp 13          TMEM allocator + GEMM1 issuer
//   warps 14, 15     TMA stores + publication of alternate tiles
// The softmax and the epilogue stream each row out of TMEM in 32-column
// chunks, the next chunk's load in flight while the current one is
// processed, in small loop bodies with few live registers (the whole CTA
// gets 128 registers per thread).
// Per tile n (group g = n % 2, ring entry e = n % 3):
//   GEMM1  S[g] = A * B^T        (A, B: K-major SW128 tiles of entry e)
//   softmax over the row (fp32, exp2); P -> TMEM S[g] as 16-bit (R / out
//          tiles) or -> the B tile of entry e (free after GEMM1) in the
//          MN-major SW128 layout (L tiles, whose GEMM2 contracts over rows)
//   GEMM2  O[g] = P * X           (A from TMEM; X = K[m] or y_j)
//          O[g] = P^T * Q_j       (L tiles; and cr = P^T * 1 into S[g])
//   R-final tiles run a second part O[g] = P * V[m]; V and y_j are loaded
//   into the A tile of the entry once GEMM1 has consumed it.
//   epilogue: TMEM -> registers -> scale -> 16-bit -> shared -> TMA store
// Masks (ma_torch.py:13, 30): a per-(e, token) validity bitmap (pad
// positions and the caller's mask), read by R tiles as -inf logits for
// invalid keys and by L tiles as zero P rows for invalid queries.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include "ma_common.cuh"
#include "ma_tc_ptx.cuh"

namespace ma {
namespace tc {

constexpr int kThreads = 512;
constexpr int kEpiWarp0 = 8;       // warps 8-11: epilogue warpgroup
constexpr int kProducerWarp = 12;
constexpr int kMmaWarp = 13;
constexpr int kStoreWarp = 14;     // warps 14, 15: TMA stores + publication (alternate tiles)
constexpr int kStoreWarps = 2;
constexpr int kT = 128;                  // tile rows (and logit columns)
constexpr int kHalf = 16384;             // one 64-column half of a tile (128 rows x 128 B)
constexpr int kMaxEntries = 4;           // ring entries (tiles in flight): 3 at D = 128, 4 at D = 64
constexpr int kItemRing = 8;             // tile descriptors for the epilogue
constexpr int kScaleRing = 4;            // per-row output scales, softmax -> epilogue
// small objects at the start of dynamic shared memory
constexpr int kOffBar = 0;        // mbarriers
constexpr int kOffDesc = 256;     // tile descriptors of the ring entries (kMaxEntries x int4)
constexpr int kOffEnd = 320;      // number of tiles this CTA was given (set at the end)
constexpr int kOffTmem = 324;     // TMEM base address
constexpr int kOffItems = 384;    // tile descriptors by tile index (kItemRing x int4)
constexpr int kOffOnes = 512;     // ones operand of the cr GEMM (512 B)
constexpr int kOffScale = 1024;   // output scale per row (kScaleRing x 128 fp32)
// The cl subtraction of L / output tiles runs on the tensor core as one more
// K step of GEMM1: A_ext (128 rows x 16 columns: -1, -1, 0 ...) times B_ext
// (row k: cl_hi[k], cl_lo[k], 0 ..., cl split into two 16-bit values) adds
// -(cl_hi + cl_lo) = -cl[k] to column k of S.  Both are K-major tiles
// without swizzle: 8-row core matrices of 16 bytes per row, row groups 128 B
// apart (SBO), the K = 8..15 half read from a zero block (LBO).
constexpr int kOffExtA = 3072;    // A_ext (2 KB)
constexpr int kOffVec = 5120;     // per entry: B_ext rows of cl[j][:] (L / out, 2 KB)
                                  // or the cr[m][:] vector (R, 512 B fp32)
constexpr int kExtBytes = 2048;
constexpr int kOffZero = kOffVec + kMaxEntries * kExtBytes;  // 2 KB of zeros
constexpr int kSmallBytes = kOffZero + kExtBytes;

// bytes of one tile (128 rows of DD 16-bit values), of a ring entry (tile A,
// then tile B, which also holds the 128 x 128 16-bit P^T of an L tile: at
// least 32 KB) and of the dynamic shared memory of a CTA.  The ring has as
// many entries as fit: 3 of 64 KB at D = 128, 4 of 48 KB at D = 64 (a tile
// holds its entry from its loads to the read of its staged output, so the
// entries in flight bound the tiles per second of an SM).
__host__ __device__ constexpr int tile_bytes(int dd) { return (dd / 64) * kHalf; }
__host__ __device__ constexpr int entry_bytes(int dd) { return tile_bytes(dd) + 2 * kHalf; }
__host__ __device__ constexpr int ring_entries(int dd) { return dd == 64 ? 4 : 3; }
__host__ __device__ constexpr int smem_bytes(int dd) {
  return kSmallBytes + 1024 + ring_entries(dd) * entry_bytes(dd);  // + worst-case alignment pad
}
static_assert(smem_bytes(128) <= 232448 && smem_bytes(64) <= 232448, "shared memory budget");
static_assert(ring_entries(128) <= kMaxEntries && ring_entries(64) <= kMaxEntries, "ring layout");

// barrier offsets (8 B each)
constexpr int kBarFull = 0;      // [kMaxEntries] A/B tiles (+ vector) of the entry landed
constexpr int kBarEmpty = 32;    // [kMaxEntries] the entry's last GEMM finished
constexpr int kBarX = 64;        // [kMaxEntries] late X tile (V or y) landed
constexpr int kBarSFull = 96;    // [2] S of the group written (GEMM1 done)
constexpr int kBarPReady = 112;  // [2] P of the group written (128 arrivals)
constexpr int kBarOFull = 128;   // [2] O of the group written (one per GEMM2 part)
constexpr int kBarOFree = 144;   // [2] O of the group read (128 arrivals per part)
constexpr int kBarCrTaken = 160; // [2] cr read out of S (L tiles, 128 arrivals)
constexpr int kBarDrain = 176;   // MMA drain before the end
constexpr int kBarStaged = 184;  // [kMaxEntries] output tile(s) of the entry's tile staged (128)
constexpr int kBarG2 = 216;      // [2] GEMM2 (all parts) of the group's tile issued
constexpr int kBarDrain2 = 232;  // [2] MMAs a softmax group issued, complete (at the end)
// e4m3 inputs (FP8 builds): the item's e4m3 tiles were converted in place to
// f16 by its softmax group (128 arrivals; GEMM1 waits for it), and the late
// V tile of a final R-step likewise (per group, before GEMM2's second part)
constexpr int kBarConv = 328;    // [kMaxEntries] (after the small objects at 320..327)
constexpr int kBarVConv = 360;   // [2]

// TMEM columns (fp32, 128 lanes): per group g, S/P at 256 g and O at 256 g + 128
constexpr uint32_t kTmemCols = 512;

// control block (uint32 words in the workspace)
constexpr int kCtrlNext = 0;   // global work counter
constexpr int kCtrlAbort = 1;  // set when any bounded wait gives up
constexpr int kCtrlDone = 64;  // done[head * P + phase]

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct TcParams {
  CUtensorMap tm_qblk;  // q (E,H,N,D) boxes of 64 x 128 token rows
  CUtensorMap tm_qstr;  // q viewed (E,H,M,b,D): 64 x (tokens j, j+b, ...) boxes of M rows
  CUtensorMap tm_kblk;
  CUtensorMap tm_vblk;
  CUtensorMap tm_al;    // al rows [slot][j][m]
  CUtensorMap tm_ar;    // ar rows [slot][m][j]
  CUtensorMap tm_y;     // y rows  [slot][j][m]
  CUtensorMap tm_al_st; // al as (D, M, slots*b): 64 x 1 x b boxes = rows j of block m
  CUtensorMap tm_y_st;  // y, same view
  CUtensorMap tm_ar_st; // ar as (D, b, slots*M): 64 x 1 x M boxes = rows k of index j
  CUtensorMap tm_out_st;// out as (Dv, b, M, H, E): tokens l*b + j of index j
  char* al;
  char* ar;
  char* y;
  uint4* clx;   // cl[j][k] as B_ext rows: (hi, lo) 16-bit pair padded to 16 bytes
  float* cr;
  const uint32_t* valid;  // validity bitmap [E][N / 32] (bit n % 32 of word n / 32), or null
  // e4m3 inputs (FP8 builds): per-(e, h) dequantisation scales, x = x8 * s
  const float* qsc;
  const float* ksc;
  const float* vsc;
  uint32_t* ctrl;
  uint32_t* status;
  uint32_t* status_host;  // host mirror of the status word (optional)
  int N, H, nheads, T, P, slots;
  int hgroup;  // heads per wavefront phase slot (round r runs phase p of heads hgroup*(r-p) + i)
  int early;   // 1: claim the next tile (and await its dependency) before its ring entry frees
  int claim;   // tiles claimed per global atomic
  float sm_scale;
  unsigned long long timeout_ns;
  // test hook (MA_TEST_STALL_DEP=head,phase): the dependency wait of that
  // (head, phase) needs one more completed tile than the phase before it
  // has, so it runs out after timeout_ns; -1 = off
  int stall_head, stall_phase;
  unsigned long long* trace;  // MA_TC_TRACE builds: per-CTA tile timestamps, else null
};

enum Kind : int { KIND_R = 0, KIND_L = 1, KIND_O = 2 };

// Optional per-tile timeline (compiled in with -DMA_TC_TRACE): for the first
// kTraceItems tiles of each CTA, slot 0 holds (head, phase, tile) and the
// other slots globaltimer stamps: 1 claim, 2 dependency met (loads issued),
// 11 loads landed, 3 GEMM1 issued, 4 softmax start, 5 P ready, 8 GEMM2
// issued, 6 epilogue start, 15 output staged, 12 store issued, 9 store read,
// 10 writes complete, 7 published.
#ifdef MA_TC_TRACE
constexpr int kTraceItems = 256;
constexpr int kTraceSlots = 16;
#endif
__device__ __forceinline__ void trace_stamp(const TcParams& p, uint32_t n, int slot,
                                            unsigned long long v) {
#ifdef MA_TC_TRACE
  if (p.trace != nullptr && n < (uint32_t)kTraceItems)
    p.trace[((size_t)blockIdx.x * kTraceItems + n) * kTraceSlots + slot] = v;
#else
  (void)p; (void)n; (void)slot; (void)v;
#endif
}

// NH * 64 TMEM accumulator columns of this lane -> scaled 16-bit row of an
// output tile staged in SMEM in the SW128 layout the TMA store expects: row
// r of half h at h*16K + r*128, 16-byte unit c at position c ^ (r & 7).  The
// row is read in 32-column chunks with the next chunk's load in flight.
template <bool BF16, int NH>
__device__ __forceinline__ void stage_row(uint32_t tile, int row, uint32_t taddr, float scale) {
  constexpr int kChunks = 2 * NH;
  uint32_t ca[32], cb[32];
  const uint32_t rbase = tile + row * 128;
  const uint64_t sc2 = f2pack(scale, scale);
  // chunk ch (32 columns) = 16-byte units u = 4 ch .. 4 ch + 3
  auto put = [&](const uint32_t(&cv)[32], int ch) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      uint32_t w[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        w[q] = scale_pack2<BF16>(cv[8 * t + 2 * q], cv[8 * t + 2 * q + 1], sc2);
      const int u = 4 * ch + t;
      st_shared_v4(rbase + (u >> 3) * kHalf + (((u & 7) ^ (row & 7)) << 4), w[0], w[1], w[2], w[3]);
    }
  };
  tmem_ld32(taddr, ca);
  tmem_wait_ld();
#pragma unroll 1
  for (int ch = 0; ch < kChunks; ch += 2) {
    tmem_ld32(taddr + 32 * (ch + 1), cb);
    put(ca, ch);
    tmem_wait_ld();
    if (ch + 2 < kChunks) tmem_ld32(taddr + 32 * (ch + 2), ca);
    put(cb, ch + 1);
    tmem_wait_ld();
  }
}

// S = A B^T over K = NH * 64 (A, B: 128-row K-major SW128 tiles)
template <bool BF16, int NH>
__device__ __forceinline__ void gemm1(uint32_t tS, uint32_t A, uint32_t B) {
  constexpr uint32_t id_ss = idesc_f16(BF16, false, false, 128, 128);
#pragma unroll
  for (int kk = 0; kk < 4 * NH; ++kk) {
    const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;  // K step of 16 inside SW128 rows
    mma_ss(tS, smem_desc(A + off, 16, 1024, kSwz128), smem_desc(B + off, 16, 1024, kSwz128),
           id_ss, kk > 0);
  }
}
// O = P (TMEM, 128 x 128 16-bit) * X (SMEM, MN-major SW128 128 x DD)
template <bool BF16, int DD>
__device__ __forceinline__ void gemm2_ts(uint32_t tO, uint32_t tP, uint32_t X) {
  constexpr uint32_t id_ts = idesc_f16(BF16, false, true, 128, DD);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    mma_ts(tO, tP + kk * 8, smem_desc(X + kk * 2048, kHalf, 1024, kSwz128), id_ts, kk > 0);
}

// validity word of 32 consecutive tokens (tok0 a multiple of 32) of batch
// row e; all ones without a mask
__device__ __forceinline__ uint32_t valid_word(const TcParams& p, int e, int tok0) {
  if (p.valid == nullptr) return 0xFFFFFFFFu;
  return __ldg(p.valid + ((size_t)e * p.N + tok0) / 32);
}

// e4m3 -> f16 in place (FP8 builds): row `row` of a 128-row tile whose e4m3
// values (128 per row, SW128: 16-byte unit c at position c ^ (row & 7)) were
// loaded into its second 16 KB half; the f16 row (256 bytes) is written in
// the tile's SW128 layout (half c / 4, units 2 (c % 4) and 2 (c % 4) + 1).
// The row is read completely before anything is written, and no other
// thread touches it, so converting in place is safe.  e4m3 values are exact
// in f16.
__device__ __forceinline__ void e4m3_row_to_f16(uint32_t tile, int row) {
  const uint32_t src = tile + kHalf + row * 128;
  uint32_t in[8][4];
#pragma unroll
  for (int c = 0; c < 8; ++c)
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(in[c][0]), "=r"(in[c][1]), "=r"(in[c][2]), "=r"(in[c][3])
                 : "r"(src + ((c ^ (row & 7)) << 4))
                 : "memory");
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2_raw lo =
          __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(in[c][i] & 0xFFFFu), __NV_E4M3);
      const __half2_raw hi =
          __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(in[c][i] >> 16), __NV_E4M3);
      o[2 * i] = (uint32_t)lo.x | ((uint32_t)lo.y << 16);
      o[2 * i + 1] = (uint32_t)hi.x | ((uint32_t)hi.y << 16);
    }
    const uint32_t dst = tile + (c >> 2) * kHalf + row * 128;
    const int u = 2 * (c & 3);
    st_shared_v4(dst + ((u ^ (row & 7)) << 4), o[0], o[1], o[2], o[3]);
    st_shared_v4(dst + (((u + 1) ^ (row & 7)) << 4), o[4], o[5], o[6], o[7]);
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// MASKED: the call has a validity bitmap (p.valid); the unmasked build
// carries no mask code at all.  FP8: q, k, v are e4m3 with per-head scales
// (f16 tensor-core arithmetic, f16 intermediates, bf16 output).
template <bool BF16, int BB, int MM, int DD, bool MASKED, bool FP8>
__global__ void __launch_bounds__(kThreads, 1) ma_tc_kernel(const __grid_constant__ TcParams p) {
  constexpr int PR = kT / BB;             // R items per tile
  constexpr int PL = kT / MM;             // L / output items per tile
  constexpr int kTiles = BB * MM / kT;    // tiles per (head, phase)
  constexpr int NH = DD / 64;             // 64-column halves of a D-wide row
  constexpr int kTileBytes = tile_bytes(DD);
  constexpr int kEntryBytes = entry_bytes(DD);  // tiles A and B
  constexpr int kEntries = ring_entries(DD);     // ring entries of this head dim
  static_assert((BB == 32 || BB == 64 || BB == 128) && (MM == 32 || MM == 64 || MM == 128),
                "block size and block count 32, 64 or 128");
  static_assert(DD == 64 || DD == 128, "head dim 64 or 128");
  static_assert(kTiles >= 1, "at least one tile per phase");
  static_assert(!FP8 || (!BF16 && DD == 128), "e4m3 builds: f16 arithmetic, head dim 128");
  constexpr int kInBytes = FP8 ? kHalf : kTileBytes;  // bytes of a q / k / v tile as loaded
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t sbase = smem_u32(smem_raw);                       // small objects
  const uint32_t tbase = (sbase + kSmallBytes + 1023u) & ~1023u;   // SW128 tiles
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  uint32_t* ctrl = p.ctrl;
  const Guard guard{ctrl + kCtrlAbort, p.status, p.timeout_ns, p.status_host};
  const int P = p.P;
  const uint32_t total = (uint32_t)p.nheads * P * kTiles;

  int4* desc_slot = reinterpret_cast<int4*>(smem_raw + kOffDesc);
  int4* item_ring = reinterpret_cast<int4*>(smem_raw + kOffItems);
  volatile uint32_t* n_end_s = reinterpret_cast<volatile uint32_t*>(smem_raw + kOffEnd);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem_raw + kOffTmem);
  const float* vec0 = reinterpret_cast<const float*>(smem_raw + kOffVec);
  float* scale_ring = reinterpret_cast<float*>(smem_raw + kOffScale);
  auto bar = [&](int off, int i) { return sbase + kOffBar + off + 8 * i; };

  if (tid == 0) {
    for (int i = 0; i < kEntries; ++i) {
      mbar_init(bar(kBarFull, i), 1);
      mbar_init(bar(kBarEmpty, i), 1);
      mbar_init(bar(kBarX, i), 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(bar(kBarSFull, g), 1);
      mbar_init(bar(kBarPReady, g), 128);
      mbar_init(bar(kBarOFull, g), 1);
      mbar_init(bar(kBarOFree, g), 128);
      mbar_init(bar(kBarCrTaken, g), 128);
    }
    for (int i = 0; i < kEntries; ++i) mbar_init(bar(kBarStaged, i), 128);
    if (FP8) {
      for (int i = 0; i < kEntries; ++i) mbar_init(bar(kBarConv, i), 128);
      for (int g = 0; g < 2; ++g) mbar_init(bar(kBarVConv, g), 128);
    }
    mbar_init(bar(kBarDrain, 0), 1);
    for (int g = 0; g < 2; ++g) {
      mbar_init(bar(kBarG2, g), 1);
      mbar_init(bar(kBarDrain2, g), 1);
    }
    *n_end_s = 0xFFFFFFFFu;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid < 32) {  // ones operand of the cr GEMM: 256 x 16-bit 1.0
    const uint32_t one = BF16 ? 0x3F803F80u : 0x3C003C00u;
    st_shared_v4(sbase + kOffOnes + tid * 16, one, one, one, one);
  }
  if (tid < 128) {  // A_ext row (-1, -1, 0, ...) and the zero block
    const uint32_t m1 = BF16 ? 0xBF80BF80u : 0xBC00BC00u;
    st_shared_v4(sbase + kOffExtA + tid * 16, m1, 0u, 0u, 0u);
    st_shared_v4(sbase + kOffZero + tid * 16, 0u, 0u, 0u, 0u);
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == kProducerWarp) {
    // ===================== scheduler + TMA producer =====================
    if (lane == 0) {
      // wavefront cursor over valid (round r, phase ph, head sub) blocks of
      // kTiles tiles; blk = block index.  Head group of round r, phase ph:
      // r - ph; heads hgroup * (r - ph) + sub.
      const int G = p.hgroup;
      const int ngroups = (p.nheads + G - 1) / G;
      int r = 0, ph = 0, sub = 0;
      uint32_t blk = 0;
      uint32_t issued = 0;  // bit e: a load was issued on entry e
      uint32_t last_on[kEntries] = {};
      // Tiles are claimed p.claim at a time (one global atomic per batch), and
      // the last (head, phase) whose dependency was seen complete is
      // remembered (completion is final), so consecutive tiles of one
      // (head, phase) block cost no global round trip at all.
      uint32_t w_next = 0, w_end = 0;
      int dep_head = -1, dep_ph = -1;
      uint32_t n = 0;
      for (;; ++n) {
        const int e = n % kEntries;
        const uint32_t use = n / kEntries;
        const uint32_t fb = bar(kBarFull, e);
        if (!p.early && n >= kEntries && !wait_bar(bar(kBarEmpty, e), (use - 1) & 1, guard))
          break;
        trace_stamp(p, n, 1, globaltimer());
        if (w_next == w_end) {
          w_next = atomicAdd(ctrl + kCtrlNext, (uint32_t)p.claim);
          w_end = w_next + (uint32_t)p.claim;
        }
        const uint32_t w = w_next++;
        bool ok = w < total && !ld_relaxed(guard.abort);
        int head = -1, item = 0, kind = 0;
        if (ok) {
          const uint32_t want = w / kTiles;
          item = (int)(w % kTiles);
          while (blk < want) {
            ++sub;
            if (sub >= G || G * (r - ph) + sub >= p.nheads) {
              sub = 0;
              ++ph;
              if (ph > (r < P - 1 ? r : P - 1)) {
                ++r;
                ph = r - ngroups + 1 > 0 ? r - ngroups + 1 : 0;
              }
            }
            ++blk;
          }
          head = G * (r - ph) + sub;
          if (head < 0 || head >= p.nheads) {
            guard.raise(MA_STATUS_BAD_ITEM);
            ok = false;
          }
        }
        if (ok) {
          kind = (ph & 1) == 0 ? KIND_R : (ph == P - 1 ? KIND_O : KIND_L);
          // dependency: the previous phase of this head, or -- for phase 0 --
          // the output phase of the head that used this workspace slot before
          if (head != dep_head || ph != dep_ph) {
            const uint32_t need =
                (uint32_t)kTiles + (head == p.stall_head && ph == p.stall_phase ? 1u : 0u);
            if (ph > 0)
              ok = wait_counter(ctrl + kCtrlDone + head * P + ph - 1, need, guard);
            else if (head >= p.slots)
              ok = wait_counter(ctrl + kCtrlDone + (head - p.slots) * P + P - 1, need, guard);
            if (ok) {
              dep_head = head;
              dep_ph = ph;
            }
          }
        }
        if (p.early && n >= kEntries && !wait_bar(bar(kBarEmpty, e), (use - 1) & 1, guard))
          break;
        if (!ok) {
          *n_end_s = n;  // tiles n, n+1, ... do not exist
          mbar_arrive(fb);
          break;
        }
        desc_slot[e] = make_int4(head, ph, item, kind);
        item_ring[n % kItemRing] = make_int4(head, ph, item, kind);
        trace_stamp(p, n, 0, ((unsigned long long)head << 32) | ((unsigned)ph << 16) | item);
        trace_stamp(p, n, 2, globaltimer());
        fence_proxy_async_global();
        const int slot = head % p.slots;
        const int eb = head / p.H, hh = head - eb * p.H;
        const uint32_t A = tbase + e * kEntryBytes, B = A + kTileBytes;
        const uint32_t vdst = sbase + kOffVec + e * kExtBytes;
        // first row of the tile in the per-slot arrays ar [M][b], al / y
        // [b][M], cr [M][b], cl [b][M] (rows of D / Dv elements or floats),
        // and its first token in q / k / v (R tiles: key blocks item * PR ..)
        const int trow = slot * BB * MM + item * kT;
        const int tok0 = item * kT;
        const size_t vrow = (size_t)trow;
        // L2 policy: keep what a later phase of this head reads again (q before
        // the output phase, k before the final R-step); stream last uses and
        // the single-use intermediates
        const uint64_t keep = policy_evict_last(), once = policy_evict_first();
        if (FP8 && kind == KIND_R) {
          // e4m3 q / k tiles (128 rows x 128 bytes) into the second half of
          // their slot, converted to f16 in place by the softmax group
          const bool first = ph == 0, final_ = ph == P - 2;
          mbar_expect_tx(fb, (first ? kInBytes : kTileBytes) + kInBytes + (first ? 0 : 512));
          if (!first) bulk_load(vdst, p.cr + vrow, 512, fb);
          if (first)
            tma_load_4d_h(A + kHalf, &p.tm_qblk, 0, tok0, hh, eb, fb, keep);
          else
            for (int h2 = 0; h2 < NH; ++h2)
              tma_load_2d_h(A + h2 * kHalf, &p.tm_ar, h2 * 64, trow, fb, once);
          tma_load_4d_h(B + kHalf, &p.tm_kblk, 0, tok0, hh, eb, fb, final_ ? once : keep);
        } else if (FP8) {
          mbar_expect_tx(fb, kInBytes + kTileBytes + kExtBytes);
          bulk_load(vdst, p.clx + vrow, kExtBytes, fb);
#pragma unroll
          for (int pk = 0; pk < PL; ++pk)
            tma_load_5d_h(A + kHalf + pk * MM * 128, &p.tm_qstr, 0, item * PL + pk, 0, hh, eb, fb,
                          kind == KIND_O ? once : keep);
#pragma unroll
          for (int h2 = 0; h2 < NH; ++h2)
            tma_load_2d_h(B + h2 * kHalf, &p.tm_al, h2 * 64, trow, fb, once);
        } else if (kind == KIND_R) {
          const bool first = ph == 0, final_ = ph == P - 2;
          mbar_expect_tx(fb, 2 * kTileBytes + (first ? 0 : 512));
          if (!first) bulk_load(vdst, p.cr + vrow, 512, fb);
#pragma unroll
          for (int h2 = 0; h2 < NH; ++h2) {
            if (first)
              tma_load_4d_h(A + h2 * kHalf, &p.tm_qblk, h2 * 64, tok0, hh, eb, fb, keep);
            else
              tma_load_2d_h(A + h2 * kHalf, &p.tm_ar, h2 * 64, trow, fb, once);
            tma_load_4d_h(B + h2 * kHalf, &p.tm_kblk, h2 * 64, tok0, hh, eb, fb,
                          final_ ? once : keep);
          }
        } else {
          mbar_expect_tx(fb, 2 * kTileBytes + kExtBytes);
          bulk_load(vdst, p.clx + vrow, kExtBytes, fb);
#pragma unroll
          for (int h2 = 0; h2 < NH; ++h2) {
            // Q_j: tokens j, j + b, j + 2b, ... of each index j of the tile
#pragma unroll
            for (int pk = 0; pk < PL; ++pk)
              tma_load_5d_h(A + h2 * kHalf + pk * MM * 128, &p.tm_qstr, h2 * 64, item * PL + pk,
                            0, hh, eb, fb, kind == KIND_O ? once : keep);
            tma_load_2d_h(B + h2 * kHalf, &p.tm_al, h2 * 64, trow, fb, once);
          }
        }
        issued |= 1u << e;
        last_on[e] = use;
      }
      // never leave with copies in flight: after an abort, wait (bounded,
      // ignoring the abort flag) until the last load of each entry landed
      if (ld_relaxed(guard.abort)) {
        for (int e = 0; e < kEntries; ++e) {
          if (!(issued >> e & 1)) continue;
          const uint64_t t0 = globaltimer();
          while (!mbar_try(bar(kBarFull, e), last_on[e] & 1) && globaltimer() - t0 < guard.limit) {
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ===================== GEMM1 issuer =====================
    // GEMM1 (and the cl step) of every tile in order; GEMM2 is issued by the
    // tile's softmax group once its P is ready.  GEMM1 of tile m reuses S of
    // its group, so it waits until GEMM2 of tile m - 2 (same group) has been
    // issued (kBarG2; the tcgen05 fences around that barrier order the two).
    if (lane == 0) {
      constexpr uint32_t id_ext = idesc_f16(BF16, false, false, 128, 128);  // S -= cl
      uint32_t cr_waits[2] = {0, 0};      // cr_taken phases consumed per group
      int prev_kind[2] = {-1, -1};        // kind of the group's previous tile
      uint32_t m = 0;
      bool ok = true;
      for (;; ++m) {
        const int e = m % kEntries, gm = m & 1;
        ok = wait_bar(bar(kBarFull, e), (m / kEntries) & 1, guard);
        if (!ok) break;
        trace_stamp(p, m, 11, globaltimer());
        if (m >= *n_end_s) break;  // end marker: no tile m
        if (FP8) ok = wait_bar(bar(kBarConv, e), (m / kEntries) & 1, guard);  // e4m3 -> f16 done
        if (ok && m >= 2) ok = wait_bar(bar(kBarG2, gm), ((m - 2) >> 1) & 1, guard);
        if (ok && prev_kind[gm] == KIND_L) {  // its cr lives in S[gm]: wait until read
          ok = wait_bar(bar(kBarCrTaken, gm), cr_waits[gm] & 1, guard);
          ++cr_waits[gm];
        }
        if (!ok) break;
        const int kind1 = desc_slot[e].w;
        prev_kind[gm] = kind1;
        tc_fence_after();
        const uint32_t A = tbase + e * kEntryBytes;
        gemm1<BF16, NH>(tmem + 256 * gm, A, A + kTileBytes);
        if (kind1 != KIND_R) {  // S - cl[k] (L / output tiles): one more K step
          const uint32_t xa = sbase + kOffExtA, xb = sbase + kOffVec + e * kExtBytes;
          const uint32_t z = sbase + kOffZero;
          mma_ss(tmem + 256 * gm, smem_desc(xa, z - xa, 128, kSwzNone),
                 smem_desc(xb, z - xb, 128, kSwzNone), id_ext, 1);
        }
        mma_commit(bar(kBarSFull, gm));
        trace_stamp(p, m, 3, globaltimer());
      }
      // let the GEMM1s complete, then pass the end marker to the softmax
      // groups: one extra S-full phase each, posted only after the group's
      // last real tile was taken (its GEMM2 issued), so the phase cannot
      // alias under the group's parity wait
      mma_commit(bar(kBarDrain, 0));
      const uint64_t t0 = globaltimer();
      while (!mbar_try(bar(kBarDrain, 0), 0) && globaltimer() - t0 < guard.limit) {
      }
      if (*n_end_s == 0xFFFFFFFFu) *n_end_s = m;  // gave up: stop everyone
      const uint32_t n_end = m;
      for (int g = 0; g < 2; ++g) {
        if (ok && n_end > (uint32_t)g) {
          const uint32_t last = ((n_end - 1 - g) & ~1u) + g;  // the group's last tile
          const uint64_t t1 = globaltimer();
          while (!mbar_try(bar(kBarG2, g), (last >> 1) & 1) && globaltimer() - t1 < guard.limit) {
          }
        }
        mbar_arrive(bar(kBarSFull, g));
      }
    }
  } else if (warp < 8) {
    // ===================== softmax (warpgroups 0, 1) =====================
    const int g = warp >> 2;
    const int row = tid & 127;  // = TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + 256 * g + lane_off;
    constexpr uint32_t id_mm = idesc_f16(BF16, true, true, 128, DD);   // ar = P^T Q_j
    constexpr uint32_t id_cr = idesc_f16(BF16, true, false, 128, 16);  // cr = P^T 1
    uint32_t g2_parts = 0;  // O parts this group committed (row 0)
    uint32_t vconv = 0;     // final R-step V tiles this group converted (FP8)
    for (uint32_t k = 0;; ++k) {
      const uint32_t n = 2 * k + g;
      const int e = n % kEntries;
      if (FP8) {
        // convert this tile's e4m3 operands to f16 (row `row` of each) as
        // soon as they land; GEMM1 waits for the 128 arrivals.  The wait also
        // watches the end marker: after the last tile the producer posts it on
        // one entry only, and the tile this group waits for may not exist.
        bool ready = false;
        {
          const uint32_t fb = bar(kBarFull, e), par = (n / kEntries) & 1;
          const uint64_t t0 = globaltimer();
          for (uint32_t spin = 0;; ++spin) {
            if (mbar_try(fb, par)) {
              ready = true;
              break;
            }
            if (n >= *n_end_s) break;  // no such tile
            if ((spin & 63u) == 0) {
              if (ld_relaxed(guard.abort)) break;
              if (globaltimer() - t0 > guard.limit) {
                guard.raise(MA_STATUS_WAIT_TIMEOUT);
                break;
              }
            }
          }
        }
        if (!__all_sync(0xffffffffu, ready)) break;
        if (n >= *n_end_s) break;
        const int4 dc = desc_slot[e];
        const uint32_t At = tbase + e * kEntryBytes, Bt = At + kTileBytes;
        if (dc.w != KIND_R || dc.y == 0) e4m3_row_to_f16(At, row);  // q blocks / Q_j
        if (dc.w == KIND_R) e4m3_row_to_f16(Bt, row);               // k blocks
        fence_proxy_async_smem();
        mbar_arrive(bar(kBarConv, e));
      }
      if (!wait_bar_warp(bar(kBarSFull, g), k & 1, guard)) break;
      if (n >= *n_end_s) break;
      // the entry's vector was written by the async proxy: observe its
      // barrier (already complete -- GEMM1 consumed the entry)
      if (!wait_bar_warp(bar(kBarFull, e), (n / kEntries) & 1, guard)) break;
      tc_fence_after();
      if (row == 0) trace_stamp(p, n, 4, globaltimer());
      const int4 d = desc_slot[e];
      const int head = d.x, ph = d.y, item = d.z, kind = d.w;
      const int slot = head % p.slots;
      const bool final_ = kind == KIND_R && ph == P - 2;
      const int eb = head / p.H, hh = head - eb * p.H;
      const uint32_t A = tbase + e * kEntryBytes, B = A + kTileBytes;
      const float* vec = vec0 + e * (kExtBytes / 4);  // cr[m][:] (R tiles)
      const int trow = slot * BB * MM + item * kT;    // tile's first row in the slot arrays
      const bool rk = kind == KIND_R;
      // this row's item within the tile and its column block of S / P
      // (warp-uniform: a block is at least 32 rows = one warp wide)
      const int bw = rk ? BB : MM;                    // logit columns of the row's item
      const int pk_row = row / bw;
      const int c_lo = pk_row * bw / 32, c_hi = c_lo + bw / 32;  // 32-column chunks

      // late X tile (V[m] for R-final, y_j for out) into tile A, free after
      // GEMM1; every tile completes one phase of X[e] (a plain arrival when
      // there is no late tile), so tile n waits for phase n / kEntries
      if (!(final_ || kind == KIND_O) && row == 0) mbar_arrive(bar(kBarX, e));
      if ((final_ || kind == KIND_O) && row == 0) {
        fence_proxy_async_global();
        const uint32_t xb = bar(kBarX, e);
        const uint64_t once = policy_evict_first();  // V and y_j: single use
        if (FP8 && final_) {  // e4m3 V (converted before GEMM2's second part)
          mbar_expect_tx(xb, kInBytes);
          tma_load_4d_h(A + kHalf, &p.tm_vblk, 0, item * kT, hh, eb, xb, once);
        } else {
          mbar_expect_tx(xb, kTileBytes);
#pragma unroll
          for (int h2 = 0; h2 < NH; ++h2) {
            if (final_)
              tma_load_4d_h(A + h2 * kHalf, &p.tm_vblk, h2 * 64, item * kT, hh, eb, xb, once);
            else
              tma_load_2d_h(A + h2 * kHalf, &p.tm_y, h2 * 64, trow, xb, once);
          }
        }
      }

      // The intermediate tiles and vectors this tile read have no other
      // reader: drop them from L2 so their dirty lines are never written back
      if (kind != KIND_R || ph > 0) {
        const char* tile = (kind == KIND_R ? p.ar : p.al) + (size_t)trow * DD * 2;
#pragma unroll
        for (int h2 = 0; h2 < NH; ++h2) discard_l2(tile + (row + 128 * h2) * 128);
        if (kind == KIND_R ? row < 4 : row < kExtBytes / 128)  // the cr vector or the cl rows
          discard_l2((kind == KIND_R ? reinterpret_cast<const char*>(p.cr + trow)
                                     : reinterpret_cast<const char*>(p.clx + trow)) +
                     row * 128);
      }

      // validity: R tiles mask invalid keys of the row's block m (logit
      // -inf, ma_torch.py:13); L tiles zero the P row of an invalid query
      // token l * b + j (ma_torch.py:30); output tiles use no mask (:55-62)
      const bool kmask = MASKED && rk;
      const int kblock = item * PR + row / BB;        // R: the row's key block m
      bool row_valid = true;
      if (MASKED && kind == KIND_L) {
        const int tok = (row % MM) * BB + item * PL + row / MM;
        row_valid = (valid_word(p, eb, tok & ~31) >> (tok & 31)) & 1u;
      }
      auto chunk_valid = [&](int ch) {  // validity bits of the keys of chunk ch (R)
        return kmask ? valid_word(p, eb, kblock * BB + 32 * (ch - c_lo)) : 0xFFFFFFFFu;
      };

      // The row's logits (its own block: bw columns) are streamed out of
      // TMEM in 32-column chunks, the next chunk's load in flight while the
      // current one is processed: pass 1 takes the row maximum, pass 2
      // exponentiates and sums (P goes back to TMEM; for L tiles e goes back
      // in place), pass 3 (L only) normalises and writes P^T to shared
      // memory.  Everything outside the block is written as zero.
      float c = 1.0f;  // R: sm_scale / (cr_j + eps)
      if (rk) c = p.sm_scale / ((ph > 0 ? vec[row] : 1.0f) + kEps);
      // e4m3: S was computed on the unscaled values: R logits carry s_k
      // (and s_q in round 0), L / output logits were computed as
      // (q8 al^T - cl / s_q) and are s_q times that
      float sq = 1.0f;
      if (FP8) {
        sq = __ldg(p.qsc + head);
        if (rk) c *= __ldg(p.ksc + head) * (ph == 0 ? sq : 1.0f);
      }
      uint32_t ca[32], cb[32];
      float mx;
      {
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        // (L / output tiles: S already holds x = S - cl[k], from GEMM1)
        auto max_chunk = [&](const uint32_t(&cv)[32], int ch) {
          if (MASKED && kmask) {
            const uint32_t vw = chunk_valid(ch);
#pragma unroll
            for (int i = 0; i < 32; ++i)
              mx4[i & 3] = fmaxf(mx4[i & 3], ((vw >> i) & 1u) ? __uint_as_float(cv[i]) : -INFINITY);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) mx4[i & 3] = fmaxf(mx4[i & 3], __uint_as_float(cv[i]));
          }
        };
#pragma unroll 1
        for (int ch = c_lo; ch < c_hi; ch += 2) {  // the maximum needs no prefetch
          const bool two = ch + 1 < c_hi;
          tmem_ld32(tS + 32 * ch, ca);
          if (two) tmem_ld32(tS + 32 * (ch + 1), cb);
          tmem_wait_ld();
          max_chunk(ca, ch);
          if (two) max_chunk(cb, ch + 1);
        }
        mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      }
      // exponent arguments in log2 units: u = u_a * x + u_b
      float u_a, u_b;
      if (rk) {
        // t_i = sm_scale * S_i / (cr_j + eps); mx = max(max_i t_i, eps) (ma_torch.py:11-16);
        // a row whose keys are all masked has mx = -inf and takes eps
        const float mxt = fmaxf(c * mx, kEps);
        u_a = c * kLog2e;
        u_b = -mxt * kLog2e;
      } else {
        u_a = kLog2e;  // x = S - cl[k] (subtracted by GEMM1)
        u_b = -mx * kLog2e;
        if (FP8) {
          u_a *= sq;
          u_b *= sq;
        }
      }
      float s4[4] = {0.f, 0.f, 0.f, 0.f}, w4[4] = {0.f, 0.f, 0.f, 0.f};
      uint64_t s2[2] = {0ull, 0ull}, w2[2] = {0ull, 0ull};
      const uint64_t ua2 = f2pack(u_a, u_a), ub2 = f2pack(u_b, u_b);
      {
        // e of chunk ch (0 for masked keys); back to TMEM as fp32 in place
        // (L) or as packed 16-bit pairs into columns 16 ch .. 16 ch + 15
        // (R / out: those S columns were read already, and the chunk in
        // flight lies beyond)
        auto exp_chunk = [&](uint32_t(&cv)[32], int ch) {
          const uint32_t vw = MASKED ? chunk_valid(ch) : 0xFFFFFFFFu;
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            const uint64_t x2 = f2pack(__uint_as_float(cv[2 * t]), __uint_as_float(cv[2 * t + 1]));
            const uint64_t u2 = ffma2(x2, ua2, ub2);
            float u0, u1;
            f2unpack(u2, u0, u1);
            float e0 = ex2(u0), e1 = ex2(u1);
            if (MASKED && kmask) {
              e0 = ((vw >> (2 * t)) & 1u) ? e0 : 0.0f;
              e1 = ((vw >> (2 * t + 1)) & 1u) ? e1 : 0.0f;
            }
            const uint64_t e2 = f2pack(e0, e1);
            s2[t & 1] = fadd2(s2[t & 1], e2);
            if (rk) w2[t & 1] = ffma2(e2, u2, w2[t & 1]);
            cv[2 * t] = __float_as_uint(e0);
            cv[2 * t + 1] = __float_as_uint(e1);
          }
          if (kind == KIND_L) {
            tmem_st32(tS + 32 * ch, cv);
          } else {
            uint32_t pk[16];
#pragma unroll
            for (int t = 0; t < 16; ++t)
              pk[t] = pack2<BF16>(__uint_as_float(cv[2 * t]), __uint_as_float(cv[2 * t + 1]));
            tmem_st16(tS + 16 * ch, pk);
          }
        };
        tmem_ld32(tS + 32 * c_lo, ca);
        tmem_wait_ld();
#pragma unroll 1
        for (int ch = c_lo; ch < c_hi; ch += 2) {
          const bool two = ch + 1 < c_hi;
          if (two) tmem_ld32(tS + 32 * (ch + 1), cb);
          exp_chunk(ca, ch);
          tmem_wait_ld();
          if (ch + 2 < c_hi) tmem_ld32(tS + 32 * (ch + 2), ca);
          if (two) exp_chunk(cb, ch + 1);
          tmem_wait_ld();
        }
      }
      if (kind != KIND_L && (c_hi - c_lo) < 4) {  // P outside the row's block is zero
        uint32_t z[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) z[q] = 0u;
#pragma unroll 1
        for (int q = 0; q < 4; ++q)
          if (q < c_lo || q >= c_hi) tmem_st16(tS + 16 * q, z);
      }
      tmem_wait_st();
      f2unpack(s2[0], s4[0], s4[1]);
      f2unpack(s2[1], s4[2], s4[3]);
      f2unpack(w2[0], w4[0], w4[1]);
      f2unpack(w2[1], w4[2], w4[3]);
      const float sum = (s4[0] + s4[1]) + (s4[2] + s4[3]);
      float scale_out;
      if (rk) {
        const float wsum = (w4[0] + w4[1]) + (w4[2] + w4[3]);
        const float den = sum + kEps;  // r = e / (sum + eps), :17
        const float inv = 1.0f / den;
        // cl = sum_i r_i log r_i, log r_i = (t_i - mx) - log(den)  (:20)
        // (masked keys: r = 0; a fully masked row gives sum = wsum = 0, cl = 0)
        // cl[j][m] of this row: j = row % b, m = the row's key block; stored
        // as the B_ext row of the later GEMM that subtracts it: cl split into
        // a 16-bit value and the 16-bit rounding of the remainder (their sum
        // carries ~16 significant bits)
        float clv = kLn2 * inv * wsum - __logf(den) * sum * inv;
        if (FP8) clv /= sq;  // subtracted from q8 al^T (the unscaled logits)
        const float hi = round16<BF16>(clv);
        p.clx[(size_t)(slot * BB + row % BB) * MM + kblock] =
            make_uint4(pack2<BF16>(hi, clv - hi), 0u, 0u, 0u);
        scale_out = inv;
      } else {
        // L: a row of an invalid query token is zero (L *= qmask, :30)
        scale_out = row_valid ? 1.0f / sum : 0.0f;
      }
      scale_ring[(n % kScaleRing) * 128 + row] = scale_out;

      if (kind == KIND_L) {
        // P[l][k] = e / sum -> tile B (al_j is consumed) in the MN-major
        // SW128 layout: row l of half h at h*16K + l*128, 16-byte unit c at
        // position c ^ (l & 7).  Unit u (8 columns) of the 128-column row
        // sits in half u / 8; the row's own block is units 4 c_lo .. 4 c_hi - 1.
        const uint32_t prow = B + row * 128;
        if (c_hi - c_lo < 4) {
#pragma unroll 1
          for (int u = 0; u < 16; ++u)
            if (u < 4 * c_lo || u >= 4 * c_hi)
              st_shared_v4(prow + (u >> 3) * kHalf + (((u & 7) ^ (row & 7)) << 4), 0u, 0u, 0u, 0u);
        }
        const uint64_t so2 = f2pack(scale_out, scale_out);
        auto st_chunk = [&](const uint32_t(&cv)[32], int ch) {
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            uint32_t a[4];
#pragma unroll
            for (int q = 0; q < 4; ++q)
              a[q] = scale_pack2<BF16>(cv[8 * t + 2 * q], cv[8 * t + 2 * q + 1], so2);
            const int u = 4 * ch + t;
            st_shared_v4(prow + (u >> 3) * kHalf + (((u & 7) ^ (row & 7)) << 4), a[0], a[1], a[2],
                         a[3]);
          }
        };
        tmem_ld32(tS + 32 * c_lo, ca);
        tmem_wait_ld();
#pragma unroll 1
        for (int ch = c_lo; ch < c_hi; ch += 2) {
          const bool two = ch + 1 < c_hi;
          if (two) tmem_ld32(tS + 32 * (ch + 1), cb);
          st_chunk(ca, ch);
          tmem_wait_ld();
          if (ch + 2 < c_hi) tmem_ld32(tS + 32 * (ch + 2), ca);
          if (two) st_chunk(cb, ch + 1);
          tmem_wait_ld();
        }
        fence_proxy_async_smem();
      }
      tc_fence_before();
      mbar_arrive(bar(kBarPReady, g));
      if (row == 0) trace_stamp(p, n, 5, globaltimer());
      // GEMM2 of this tile, issued by the group's thread 0 as soon as its P
      // (all 128 rows), its late X tile and the group's O accumulator are
      // ready; then the MMA warp may reuse S of the group (kBarG2)
      auto issue_part = [&](int part) -> bool {
        bool ok = true;
        if (kind == KIND_O || part == 1) ok = wait_bar(bar(kBarX, e), (n / kEntries) & 1, guard);
        if (FP8 && ok && part == 1) ok = wait_bar(bar(kBarVConv, g), vconv & 1, guard);
        if (ok && g2_parts > 0) ok = wait_bar(bar(kBarOFree, g), (g2_parts - 1) & 1, guard);
        if (!ok) return false;
        tc_fence_after();
        const uint32_t tSg = tmem + 256 * g, tO = tSg + 128;
        if (kind == KIND_L) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t pd = smem_desc(B + kk * 2048, kHalf, 1024, kSwz128);  // P^T
            mma_ss(tO, pd, smem_desc(A + kk * 2048, kHalf, 1024, kSwz128), id_mm, kk > 0);
            mma_ss(tSg, pd, smem_desc(sbase + kOffOnes, 128, 256, kSwzNone), id_cr, kk > 0);
          }
        } else if (kind == KIND_O || part == 1) {
          gemm2_ts<BF16, DD>(tO, tSg, A);  // out: P y_j; R-final part 2: P V[m] (tile A)
        } else {
          gemm2_ts<BF16, DD>(tO, tSg, B);  // R: P K[m]
        }
        mma_commit(bar(kBarOFull, g));
        ++g2_parts;
        return true;
      };
      // e4m3 final R-step: the late V tile -> f16 before GEMM2's second part;
      // warps 1-3 of the group convert their rows right away, warp 0 once its
      // thread 0 has issued the first part (P K[m], which does not read V)
      const bool vconv_now = FP8 && final_;
      auto convert_v = [&]() -> bool {
        if (!wait_bar_warp(bar(kBarX, e), (n / kEntries) & 1, guard)) return false;
        e4m3_row_to_f16(A, row);
        fence_proxy_async_smem();
        mbar_arrive(bar(kBarVConv, g));
        return true;
      };
      if (vconv_now && (warp & 3) != 0 && !convert_v()) break;
      // (a failed wait leaves through the abort flag at the group's next
      // warp-uniform wait, so the warp's lanes stay together)
      bool ok2 = true;
      if (row == 0) {
        ok2 = wait_bar(bar(kBarPReady, g), k & 1, guard);
        const int nparts = vconv_now ? 1 : (final_ ? 2 : 1);
        for (int part = 0; ok2 && part < nparts; ++part) ok2 = issue_part(part);
      }
      if (vconv_now && (warp & 3) == 0) {
        if (!convert_v()) break;
        if (row == 0 && ok2) ok2 = issue_part(1);
      }
      if (row == 0 && ok2) {
        trace_stamp(p, n, 8, globaltimer());
        tc_fence_before();
        mbar_arrive(bar(kBarG2, g));
      }
      if (FP8 && final_) ++vconv;
    }
    if (row == 0) {
      // The epilogue may still be draining this group's last tile: post the
      // end marker on O-full only after its last real phase was released
      // (else the barrier would advance two phases under its parity wait),
      // and never leave with issued MMAs running.
      if (!ld_relaxed(guard.abort)) {
        if (g2_parts > 0) {
          const uint64_t t1 = globaltimer();
          while (!mbar_try(bar(kBarOFree, g), (g2_parts - 1) & 1) &&
                 globaltimer() - t1 < guard.limit) {
          }
        }
        mbar_arrive(bar(kBarOFull, g));
      }
      mma_commit(bar(kBarDrain2, g));
      const uint64_t t2 = globaltimer();
      while (!mbar_try(bar(kBarDrain2, g), 0) && globaltimer() - t2 < guard.limit) {
      }
    }
  } else if (warp < kEpiWarp0 + 4) {
    // ===================== epilogue (warpgroup 2) =====================
    // Drains O of both groups in tile order: TMEM -> registers -> scale ->
    // 16-bit -> SMEM staging in the tile's own ring tiles (free once its
    // GEMM2 ran); the store warp takes it from there.
    const int row = tid & 127;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    uint32_t eparts[2] = {0, 0};  // O parts consumed per group
    for (uint32_t n = 0;; ++n) {
      const int g = n & 1, e = n % kEntries;
      const uint32_t tS = tmem + 256 * g + lane_off, tO = tS + 128;
      if (!wait_bar_warp(bar(kBarOFull, g), eparts[g] & 1, guard)) break;
      if (n >= *n_end_s) break;
      tc_fence_after();
      ++eparts[g];
      if (row == 0) trace_stamp(p, n, 6, globaltimer());
      const int4 d = item_ring[n % kItemRing];
      const int head = d.x, ph = d.y, item = d.z, kind = d.w;
      const int slot = head % p.slots;
      const float scale_out = scale_ring[(n % kScaleRing) * 128 + row];
      const uint32_t A = tbase + e * kEntryBytes, B = A + kTileBytes;
      const bool final_ = kind == KIND_R && ph == P - 2;
      // One staging call site for every output (the kernel's speed follows
      // its code size): R tiles al[j][m] = sm_scale * r K[m] (ma_torch.py:21),
      // staged in tile B for R-final tiles (K is consumed) while their second
      // GEMM2 part reads V in tile A, then y[j][m] = r V[m] (:51) from a second
      // pass through O; L tiles ar[k][j] = sum_l P[l][k] q[l*b+j] (:34); output
      // tiles z[l*b + j] = (P y_j) / sum (:60-62).  e4m3: the GEMM2 operands
      // k, v, q_j were unscaled, and the output is bf16.
      bool ok_e = true;
      const int nparts = final_ ? 2 : 1;
#pragma unroll 1
      for (int part = 0; part < nparts; ++part) {
        if (part == 1) {
          tc_fence_before();
          mbar_arrive(bar(kBarOFree, g));
          if (!wait_bar_warp(bar(kBarOFull, g), eparts[g] & 1, guard)) {
            ok_e = false;
            break;
          }
          tc_fence_after();
          ++eparts[g];
        }
        if (kind == KIND_L) {
          // cr[k][j] = sum_l P[l][k] (the N = 16 GEMM into S[g]; read it first,
          // then let the next GEMM1 of this group overwrite S[g]) (:32)
          uint32_t o[32];
          tmem_ld32(tS, o);
          tmem_wait_ld();
          tc_fence_before();
          mbar_arrive(bar(kBarCrTaken, g));
          // cr[k][j] of this row: k = row % M, j = the row's index
          p.cr[(size_t)(slot * MM + row % MM) * BB + item * PL + row / MM] = __uint_as_float(o[0]);
        }
        float sc;
        if (kind == KIND_R)
          sc = part == 0 ? p.sm_scale * scale_out * (FP8 ? __ldg(p.ksc + head) : 1.0f)
                         : scale_out * (FP8 ? __ldg(p.vsc + head) : 1.0f);
        else
          sc = kind == KIND_L ? (FP8 ? __ldg(p.qsc + head) : 1.0f) : scale_out;
        const uint32_t dst = (final_ && part == 0) ? B : A;
        if (FP8 && kind == KIND_O)
          stage_row<true, NH>(dst, row, tO, sc);
        else
          stage_row<BF16, NH>(dst, row, tO, sc);
      }
      if (!ok_e) break;
      if (kind == KIND_O) {
        // y_j has no other reader: drop it from L2 (GEMM2 consumed it)
        const char* ytile = p.y + ((size_t)slot * BB * MM + item * kT) * DD * 2;
#pragma unroll
        for (int h2 = 0; h2 < NH; ++h2) discard_l2(ytile + (row + 128 * h2) * 128);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar(kBarOFree, g));
      mbar_arrive(bar(kBarStaged, e));
      if (row == 0) trace_stamp(p, n, 15, globaltimer());
    }
  } else if (warp >= kStoreWarp && warp < kStoreWarp + kStoreWarps) {
    // ===================== TMA stores + publication =====================
    // Per tile: wait until its output is staged, store it, release the ring
    // entry once the stores have read SMEM, and publish the tile once its
    // writes are complete.
    if (lane == 0) {
      // Publication is immediate: later phases of the head wait for the last
      // tile of this one, so any delay here lengthens the phase boundary.
      // The store warps take alternate tiles, so one warp's wait for its
      // writes to complete overlaps the other's stores.
      for (uint32_t n = warp - kStoreWarp;; n += kStoreWarps) {
        const int e = n % kEntries;
        bool ready = false;
        const uint64_t t0 = globaltimer();
        for (uint32_t spin = 0;; ++spin) {
          if (mbar_test(bar(kBarStaged, e), (n / kEntries) & 1)) {
            ready = true;
            break;
          }
          if (n >= *n_end_s) break;  // no such tile
          if ((spin & 63u) == 0) {
            if (ld_relaxed(guard.abort)) break;
            if (globaltimer() - t0 > guard.limit) {
              guard.raise(MA_STATUS_WAIT_TIMEOUT);
              break;
            }
          }
        }
        if (!ready) break;
        const int4 d = item_ring[n % kItemRing];
        const int head = d.x, ph = d.y, item = d.z, kind = d.w;
        const int slot = head % p.slots;
        const bool final_ = kind == KIND_R && ph == P - 2;
        const int eb = head / p.H, hh = head - eb * p.H;
        const uint32_t A = tbase + e * kEntryBytes, B = A + kTileBytes;
        // intermediates are read by the next phase soon: keep them in L2;
        // the output streams out
        const uint64_t keep = policy_evict_last(), once = policy_evict_first();
        // one box per item of the tile: al[.][m] / y[.][m] (b rows j),
        // ar[.][j] (M rows k), out tokens l*b + j (M rows l)
        const int np = kind == KIND_R ? PR : PL;
        const int rows = kind == KIND_R ? BB : MM;
#pragma unroll
        for (int h2 = 0; h2 < NH; ++h2) {
#pragma unroll 1
          for (int pk = 0; pk < np; ++pk) {
            const int it = item * np + pk;
            const uint32_t off = h2 * kHalf + pk * rows * 128;
            if (kind == KIND_R) {
              tma_store_3d_h(&p.tm_al_st, (final_ ? B : A) + off, h2 * 64, it, slot * BB, keep);
              if (final_) tma_store_3d_h(&p.tm_y_st, A + off, h2 * 64, it, slot * BB, keep);
            } else if (kind == KIND_L) {
              tma_store_3d_h(&p.tm_ar_st, A + off, h2 * 64, it, slot * MM, keep);
            } else {
              tma_store_5d_h(&p.tm_out_st, A + off, h2 * 64, it, 0, hh, eb, once);
            }
          }
        }
        bulk_commit();
        trace_stamp(p, n, 12, globaltimer());
        bulk_wait_read<0>();  // staging read: the ring entry can be refilled
        trace_stamp(p, n, 9, globaltimer());
        mbar_arrive(bar(kBarEmpty, e));
        bulk_wait<0>();       // writes complete
        trace_stamp(p, n, 10, globaltimer());
        fence_proxy_async_global();
        red_release_add(ctrl + kCtrlDone + head * P + ph, 1u);
        trace_stamp(p, n, 7, globaltimer());
      }
      bulk_wait<0>();  // never leave with stores in flight
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// Launch one forward on `grid` persistent CTAs (grid <= SM count).
template <bool BF16, int BB, int MM, int DD, bool MASKED, bool FP8>
cudaError_t launch_tc(const TcParams& tp, int grid, cudaStream_t st) {
  auto kfn = ma_tc_kernel<BF16, BB, MM, DD, MASKED, FP8>;
  cudaError_t err =
      cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes(DD));
  if (err != cudaSuccess) return err;
  kfn<<<grid, kThreads, smem_bytes(DD), st>>>(tp);
  return cudaGetLastError();
}

// The (b, M, D) shapes compiled (ma_tc_inst_*.cu); ma_tc.cu dispatches on them.
#define MA_TC_SHAPES(X) \
  X(128, 128, 128)      \
  X(64, 64, 128)        \
  X(64, 64, 64)         \
  X(64, 128, 64)        \
  X(32, 64, 64)         \
  X(128, 128, 64)

}  // namespace tc
}  // namespace ma
