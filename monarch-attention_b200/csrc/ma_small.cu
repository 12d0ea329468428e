// Fused small-block MonarchAttention forward: one thread-block cluster runs
// every phase of one (batch, head) -- the T-1 (R, L) rounds, the final
// R-step and the output step of ma/ma_torch.py:100-105 -- with a cluster
// barrier between phases and no kernel boundaries.  The cluster's CTAs (1, 2,
// 4 or 8) take turns on the items of a phase, so a head's critical path is
// shorter and the grid packs into fewer partial waves.  For block size b <= 32 and number of blocks M <= 32
// (the ViT, RoBERTa and DiT shapes), D = Dv <= 128, bf16 / fp16, any strides,
// padding and key-padding mask.
//
// Work items of a phase (key blocks m of an R-step, indices j of an L- or
// output step) are spread over the CTA's warps.  A warp stages its item's
// operands in shared memory with cp.async (zero-filled padding rows and head
// dim), computes the 32 x 32 logit tile with mma.sync m16n8k16 (fp32
// accumulate), the row softmax on the accumulator fragments (quad shuffles),
// and the output tile with a second mma.sync whose A operand is the
// probability fragment itself (R / output) or P^T re-read from shared memory
// (L-step, which contracts over rows).  Intermediates go through a per-head
// workspace that stays in L2.
#include <float.h>
#include <stdlib.h>

#include "ma_common.cuh"

namespace ma {
namespace small {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kRows = 32;  // rows / columns of an item, padded

struct SmallParams {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int64_t qs[4], ks[4], vs[4], os[4];
  const void* mask;
  int64_t ms[2];
  int mask_dtype;
  int E, H, N, D, b, M, T, pad_off;
  float sm_scale;
  char* al;   // [E*H][b][M][D]
  char* y;    // [E*H][b][M][D]
  char* ar;   // [E*H][M][b][D]
  float* cl;  // [E*H][b][M]
  float* cr;  // [E*H][M][b]
};

enum { PH_R = 0, PH_RF = 1, PH_L = 2, PH_O = 3 };

// ---------------------------------------------------------------------------
// warp-level primitives
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src),
               "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                          uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
template <bool BF16>
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  if (BF16)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  uint32_t r;
  if (BF16)
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  else
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

constexpr float kLog2eS = 1.4426950408889634f;
constexpr float kLn2S = 0.6931471805599453f;
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ bool token_valid(const SmallParams& p, int e, int pidx) {
  const int n = pidx - p.pad_off;
  if (n < 0 || n >= p.N) return false;
  if (p.mask == nullptr) return true;
  return mask_value(p.mask, p.mask_dtype, (int64_t)e * p.ms[0] + (int64_t)n * p.ms[1]);
}
// validity of padded token pidx from the CTA's bitmap (built in the prologue)
__device__ __forceinline__ bool valid_bit(const uint32_t* bits, int pidx) {
  return (bits[pidx >> 5] >> (pidx & 31)) & 1u;
}

// ---------------------------------------------------------------------------
// one work item, executed by one warp
// ---------------------------------------------------------------------------
// Shared-memory tiles of a warp: A, B, X (32 rows x RS 16-bit, RS = DP + 8 so
// that ldmatrix rows fall in distinct banks) and P^T staging (32 x 40).
template <typename TI, int DP, int ROWS>
struct WarpTiles {
  static constexpr int RS = DP + 8;
  static constexpr int kTile = ROWS * RS;   // elements
  static constexpr int kPS = ROWS + 8;      // P staging row stride (in tile X: L items have no X)
  static constexpr int kVec = ROWS * 4;     // cr / cl vector of the item (fp32)
  static constexpr int kTileX = ROWS * (RS > kPS ? RS : kPS);  // tile X doubles as P staging
  static constexpr int kBytes = (2 * kTile + kTileX) * 2 + kVec;
  static constexpr int kMaxTokens = ROWS * ROWS;  // padded sequence length N_p
  static constexpr int kBitmapBytes = kMaxTokens / 8 < 16 ? 16 : kMaxTokens / 8;
};

// Copy rows r = 0 .. ROWS-1 of an operand into a tile.  Row r starts at src +
// r * rstride bytes and is copied when r < rows and its token index n0 + r *
// nstep lies in [0, N) (workspace rows: n0 = nstep = 0, N = 1); other rows
// are zero-filled.  Only the first D columns are written; the padding
// columns D..DP stay zero from the kernel prologue.  Lane (rl, c) copies
// 16-byte chunk c of rows rl, rl + RPI, ...: every row address is affine in
// r, so a pass costs three additions and no per-chunk index arithmetic.
template <int DP, int ROWS>
__device__ __forceinline__ void stage_rows(uint32_t tile, int D, int lane, const char* src,
                                           int64_t rstride, int rows, int n0, int nstep, int N,
                                           const void* safe) {
  constexpr int RS = DP + 8;
  constexpr int CH = DP / 8;    // 16-byte chunks per padded row
  constexpr int RPI = 32 / CH;  // rows per pass of the warp
  const int rl = lane / CH, c = lane - rl * CH;
  if (rl >= RPI || c >= D / 8) return;
  const char* s = src + rl * rstride + c * 16;
  uint32_t d = tile + (uint32_t)(rl * RS + c * 8) * 2;
  int n = n0 + rl * nstep;
#pragma unroll
  for (int r0 = 0; r0 < ROWS; r0 += RPI) {
    if (r0 + RPI <= ROWS || r0 + rl < ROWS) {
      const bool ok = r0 + rl < rows && (unsigned)n < (unsigned)N;
      cp_async16(d, ok ? s : safe, ok);
    }
    s += RPI * rstride;
    d += RPI * RS * 2;
    n += RPI * nstep;
  }
}

template <int PH, bool BF16, typename TI, int DP, int ROWS>
__device__ void run_item(const SmallParams& p, int e, int h, int item, int first, uint8_t* wsm,
                         const uint32_t* vbits, int lane) {
  using WT = WarpTiles<TI, DP, ROWS>;
  constexpr int MT = ROWS / 16;  // m16 tiles of the item
  constexpr int NT = ROWS / 8;   // n8 tiles of its columns
  constexpr int RS = WT::RS;
  constexpr int NK = DP / 16;  // k16 steps over the head dim
  constexpr int ND = DP / 8;   // n8 tiles over the head dim
  const int D = p.D, b = p.b, M = p.M;
  const int eh = e * p.H + h;
  const uint32_t tA = smem_u32(wsm), tB = tA + WT::kTile * 2, tX = tB + WT::kTile * 2;
  const uint32_t tP = tX;                        // P staging of L items
  const uint32_t tV = tX + WT::kTileX * 2;       // cr[m][:] (R) or cl[j][:] (L / out)
  const float* vec = reinterpret_cast<const float*>(wsm + (tV - tA));
  const bool rph = PH == PH_R || PH == PH_RF;
  const int R = rph ? b : M;  // rows of the item
  const int C = R;            // columns
  const size_t esz = sizeof(TI);

  const char* al_h = p.al + (size_t)eh * b * M * D * esz;
  const char* y_h = p.y + (size_t)eh * b * M * D * esz;
  const char* ar_h = p.ar + (size_t)eh * M * b * D * esz;
  const float* cr_h = p.cr + (size_t)eh * M * b;
  const float* cl_h = p.cl + (size_t)eh * b * M;
  // q / k / v rows: token n0 + r * nstep of the head (padded index minus the
  // pre-padding), zero rows outside the sequence
  auto stage_tok = [&](uint32_t tile, const void* base, const int64_t* st, int n0, int nstep) {
    const char* hb = reinterpret_cast<const char*>(base) + esz * (e * st[0] + h * st[1]);
    stage_rows<DP, ROWS>(tile, D, lane, hb + (int64_t)n0 * st[2] * (int64_t)esz,
                         st[2] * (int64_t)esz * nstep, R, n0, nstep, p.N, hb);
  };
  // workspace rows: row r at base + r * D elements, all R rows valid
  auto stage_ws = [&](uint32_t tile, const char* base) {
    stage_rows<DP, ROWS>(tile, D, lane, base, (int64_t)D * esz, R, 0, 0, 1, base);
  };

  // ---- stage operands ----
  if (rph) {
    if (first)
      stage_tok(tA, p.q, p.qs, item * b - p.pad_off, 1);  // q block m
    else
      stage_ws(tA, ar_h + (size_t)item * b * D * esz);   // ar[m][.]
    stage_tok(tB, p.k, p.ks, item * b - p.pad_off, 1);    // k block m
  } else {
    stage_tok(tA, p.q, p.qs, item - p.pad_off, b);        // Q_j: tokens l * b + j
    stage_ws(tB, al_h + (size_t)item * M * D * esz);     // al[j][.]
    if (PH == PH_O) stage_ws(tX, y_h + (size_t)item * M * D * esz);  // y[j][.]
  }
  if (!(rph && first)) {  // the item's cr / cl vector (one fp32 per lane, 0 beyond it)
    const float* vsrc = rph ? cr_h + (size_t)item * b : cl_h + (size_t)item * M;
    if (lane < ROWS) {
      const bool ok = lane < (rph ? b : M);
      cp_async4(tV + lane * 4, ok ? vsrc + lane : vsrc, ok);
    }
  }
  cp_async_wait_all();
  __syncwarp();

  // The item is processed one 16-row tile (mt) at a time: S row tile ->
  // softmax -> (R / out) output row tile; the L-step first puts the
  // probabilities of every row tile in the staging tile, then computes its
  // output (rows k of P^T Q_j) one 16-row tile at a time.
  const int g = lane >> 2, t4 = lane & 3;
  bool colv[NT][2];
  float colc[NT][2];  // per-column term in log2 units: cl[j][k] * log2(e) (L / out)
  bool allv = true;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int c = nt * 8 + 2 * t4 + q;
      colv[nt][q] = c < C && (!rph || valid_bit(vbits, item * b + c));
      colc[nt][q] = (!rph && c < C) ? vec[c] * kLog2eS : 0.0f;
      allv = allv && colv[nt][q];
    }
  // every column of the item valid (no padding, no masked key): the
  // softmax below skips its masking selects
  allv = __all_sync(0xffffffffu, allv);
  float colsum[NT][2];  // L-step: column sums of P over the rows (cr)
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) colsum[nt][0] = colsum[nt][1] = 0.0f;
  const int nparts = PH == PH_RF ? 2 : 1;
  if (PH == PH_RF) {  // V[m] for the second output part, staged with the item
    stage_tok(tX, p.v, p.vs, item * b - p.pad_off, 1);
    cp_async_wait_all();
    __syncwarp();
  }

#pragma unroll 1
  for (int mt = 0; mt < MT; ++mt) {
    // ---- S row tile = A[mt] B^T : 16 x ROWS ----
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[nt][i] = 0.0f;
#pragma unroll
    for (int ks = 0; ks < NK; ++ks) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(tA + ((mt * 16 + (lane & 15)) * RS + ks * 16 + (lane >> 4) * 8) * 2, a0, a1, a2, a3);
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {  // pairs of n8 tiles
        uint32_t b0, b1, b2, b3;
        ldsm_x4(tB + ((np * 16 + (lane & 7) + (lane >> 4) * 8) * RS + ks * 16 + ((lane >> 3) & 1) * 8) * 2,
                b0, b1, b2, b3);
        mma16816<BF16>(acc[2 * np], a0, a1, a2, a3, b0, b1);
        mma16816<BF16>(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // ---- softmax over the columns of each row ----
    // fragment element (nt, i): row mt*16 + g + 8*(i>>1), col nt*8 + 2*t4 + (i&1)
    // Exponents in log2 units, u = ua * x + ub (- colc for L / out): one FMA
    // and one ex2 per element.  R and out rows keep e unnormalised; their
    // 1 / sum goes into the output scale (row_scale), as the second matmul
    // is linear in the rows of P.
    float row_scale[2], cl_row[2];
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = mt * 16 + g + 8 * hf;
      float c = 1.0f;
      if (rph) {
        const float crj = (first || r >= R) ? 1.0f : vec[r];
        c = __fdividef(p.sm_scale, crj + kEps);  // t = sm_scale * S / (cr + eps), ma_torch.py:11-12
      }
      // pass 1: row maximum (R: of S, as c > 0 gives max t = c * max S)
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          float x = acc[nt][2 * hf + q];
          if (!rph) x -= colc[nt][q] * kLn2S;
          if (!allv && !colv[nt][q]) x = -INFINITY;
          mx = fmaxf(mx, x);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      float ua, ub;
      if (rph) {
        ua = c * kLog2eS;
        ub = -fmaxf(c * mx, kEps) * kLog2eS;  // clamp(max t, min=eps), :14-16
      } else {
        ua = kLog2eS;
        ub = -mx * kLog2eS;
      }
      float sum = 0.0f, wsum = 0.0f;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          float& x = acc[nt][2 * hf + q];
          const float u = fmaf(x, ua, rph ? ub : ub - colc[nt][q]);
          float ev = ex2f(u);
          if (!allv && !colv[nt][q]) ev = 0.0f;
          sum += ev;
          if (rph) wsum = fmaf(ev, (allv || colv[nt][q]) ? u : 0.0f, wsum);
          x = ev;
        }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      if (rph) {
        wsum += __shfl_xor_sync(0xffffffffu, wsum, 1);
        wsum += __shfl_xor_sync(0xffffffffu, wsum, 2);
        const float den = sum + kEps;  // r = e / (sum + eps), :17
        const float inv = __fdividef(1.0f, den);
        // sum_i r_i log r_i, log r_i = ln2 * u_i - log(den) (:20)
        cl_row[hf] = kLn2S * inv * wsum - __logf(den) * sum * inv;
        row_scale[hf] = inv;
      } else {
        cl_row[hf] = 0.0f;
        row_scale[hf] = __fdividef(1.0f, sum);
      }
      if (PH == PH_L) {
        // the L-step's P is normalised here (its column sums are cr, and its
        // transpose is the second matmul's operand), times the query mask of
        // row l (:30)
        float sc = row_scale[hf];
        if (!(r < R && valid_bit(vbits, r * b + item))) sc = 0.0f;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int q = 0; q < 2; ++q) acc[nt][2 * hf + q] *= sc;
      }
    }
    if (rph) {  // cl[j][m] (:20)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = mt * 16 + g + 8 * hf;
        if (t4 == 0 && r < R) p.cl[(size_t)eh * b * M + (size_t)r * M + item] = cl_row[hf];
      }
    }

    if constexpr (PH == PH_L) {
      // cr partial sums and P (16-bit) -> staging tile Pst[l][k]
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int q = 0; q < 2; ++q) colsum[nt][q] += acc[nt][q] + acc[nt][2 + q];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = mt * 16 + g + 8 * hf, c = nt * 8 + 2 * t4;
          const uint32_t v2 = pack2<BF16>(acc[nt][2 * hf], acc[nt][2 * hf + 1]);
          asm volatile("st.shared.b32 [%0], %1;" ::"r"(tP + (r * WT::kPS + c) * 2), "r"(v2)
                       : "memory");
        }
    } else {
    // ---- R / out: output row tile O = P X over the item's ROWS columns ----
#pragma unroll 1
    for (int part = 0; part < nparts; ++part) {
      const uint32_t tXo = (rph && part == 0) ? tB : tX;  // K[m] / V[m] / y_j
      float o[ND][4];
#pragma unroll
      for (int nd = 0; nd < ND; ++nd)
#pragma unroll
        for (int i = 0; i < 4; ++i) o[nd][i] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < ROWS / 16; ++kk) {
        const uint32_t a0 = pack2<BF16>(acc[2 * kk][0], acc[2 * kk][1]);
        const uint32_t a1 = pack2<BF16>(acc[2 * kk][2], acc[2 * kk][3]);
        const uint32_t a2 = pack2<BF16>(acc[2 * kk + 1][0], acc[2 * kk + 1][1]);
        const uint32_t a3 = pack2<BF16>(acc[2 * kk + 1][2], acc[2 * kk + 1][3]);
#pragma unroll
        for (int np = 0; np < ND / 2; ++np) {
          uint32_t b0, b1, b2, b3;
          const int xr = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int xc = np * 16 + (lane >> 4) * 8;
          ldsm_x4_t(tXo + (xr * RS + xc) * 2, b0, b1, b2, b3);
          mma16816<BF16>(o[2 * np], a0, a1, a2, a3, b0, b1);
          mma16816<BF16>(o[2 * np + 1], a0, a1, a2, a3, b2, b3);
        }
      }
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = mt * 16 + g + 8 * hf;
        if (r >= R) continue;
        char* dst;
        float sc = row_scale[hf];  // 1 / (sum + eps) of R rows, 1 / sum of out rows
        if (rph && part == 0) {  // al[j][m] = sm_scale * (r K[m])  (:21)
          dst = p.al + ((size_t)eh * b * M + (size_t)r * M + item) * D * esz;
          sc *= p.sm_scale;
        } else if (rph) {        // y[j][m] = r V[m] (:51)
          dst = p.y + ((size_t)eh * b * M + (size_t)r * M + item) * D * esz;
        } else {                 // z at token l*b + j (:60-62, :106-108)
          const int n = r * b + item - p.pad_off;
          if (n < 0 || n >= p.N) continue;
          dst = reinterpret_cast<char*>(p.out) +
                esz * ((int64_t)e * p.os[0] + (int64_t)h * p.os[1] + (int64_t)n * p.os[2]);
        }
#pragma unroll
        for (int nd = 0; nd < ND; ++nd) {
          const int c = nd * 8 + 2 * t4;
          if (c >= D) continue;
          *reinterpret_cast<uint32_t*>(dst + c * esz) =
              pack2<BF16>(o[nd][2 * hf] * sc, o[nd][2 * hf + 1] * sc);
        }
      }
    }
    }  // R / out
  }

  if (PH == PH_L) {
    // cr[k][j] = sum_l P[l][k] (:32)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        float sm = colsum[nt][q];
        sm += __shfl_xor_sync(0xffffffffu, sm, 4);
        sm += __shfl_xor_sync(0xffffffffu, sm, 8);
        sm += __shfl_xor_sync(0xffffffffu, sm, 16);
        const int c = nt * 8 + 2 * t4 + q;
        if (g == 0 && c < C) p.cr[(size_t)eh * M * b + (size_t)c * b + item] = sm;
      }
    __syncwarp();
    // ar[k][j] = sum_l P[l][k] q[l*b+j] (:34): A = P^T read transposed from the
    // staging tile, B = Q_j (tile A), one 16-row tile of k at a time
#pragma unroll 1
    for (int mt = 0; mt < MT; ++mt) {
      float o[ND][4];
#pragma unroll
      for (int nd = 0; nd < ND; ++nd)
#pragma unroll
        for (int i = 0; i < 4; ++i) o[nd][i] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < ROWS / 16; ++kk) {
        uint32_t a0, a1, a2, a3;
        const int lrow = kk * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int kcol = mt * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4_t(tP + (lrow * WT::kPS + kcol) * 2, a0, a1, a2, a3);
#pragma unroll
        for (int np = 0; np < ND / 2; ++np) {
          uint32_t b0, b1, b2, b3;
          const int xr = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int xc = np * 16 + (lane >> 4) * 8;
          ldsm_x4_t(tA + (xr * RS + xc) * 2, b0, b1, b2, b3);
          mma16816<BF16>(o[2 * np], a0, a1, a2, a3, b0, b1);
          mma16816<BF16>(o[2 * np + 1], a0, a1, a2, a3, b2, b3);
        }
      }
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = mt * 16 + g + 8 * hf;  // k
        if (r >= R) continue;
        char* dst = p.ar + ((size_t)eh * M * b + (size_t)r * b + item) * D * esz;
#pragma unroll
        for (int nd = 0; nd < ND; ++nd) {
          const int c = nd * 8 + 2 * t4;
          if (c >= D) continue;
          *reinterpret_cast<uint32_t*>(dst + c * esz) = pack2<BF16>(o[nd][2 * hf], o[nd][2 * hf + 1]);
        }
      }
    }
  }
  __syncwarp();
}

// all threads of the cluster; orders the phase's global writes (release)
// before the next phase's reads (acquire) across the cluster's CTAs
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}

template <bool BF16, typename TI, int DP, int ROWS>
__global__ void __launch_bounds__(kThreads, ROWS == 16 ? 4 : 3) ma_small_kernel(const SmallParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  using WT = WarpTiles<TI, DP, ROWS>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t crank, csize;  // this CTA's rank in its cluster, cluster size
  asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
  asm("mov.u32 %0, %%cluster_nctarank;" : "=r"(csize));
  const int eh = blockIdx.x / csize;  // clusters are consecutive blocks
  const int e = eh / p.H, h = eh - e * p.H;
  const int wg = crank * kWarps + warp, nw = csize * kWarps;  // warp within the cluster
  uint8_t* wsm = smem + warp * WT::kBytes;
  uint32_t* vbits = reinterpret_cast<uint32_t*>(smem + kWarps * WT::kBytes);
  // zero the tiles once: padding rows/columns must read as 0
  for (int i = threadIdx.x; i < kWarps * WT::kBytes / 16; i += kThreads)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  // token validity of the padded sequence (pad positions and the mask row)
  const int Np = p.M * p.b;
  // (one lane per token, so the mask loads of a word are issued together)
  for (int w = warp; w < (WT::kMaxTokens + 31) / 32; w += kWarps) {
    const int pidx = w * 32 + lane;
    const uint32_t bits = __ballot_sync(0xffffffffu, pidx < Np && token_valid(p, e, pidx));
    if (lane == 0) vbits[w] = bits;
  }
  __syncthreads();
  for (int t = 0; t < p.T; ++t) {
    const bool final_ = t == p.T - 1;
    for (int m = wg; m < p.M; m += nw) {
      if (final_)
        run_item<PH_RF, BF16, TI, DP, ROWS>(p, e, h, m, t == 0, wsm, vbits, lane);
      else
        run_item<PH_R, BF16, TI, DP, ROWS>(p, e, h, m, t == 0, wsm, vbits, lane);
    }
    cluster_sync();
    for (int j = wg; j < p.b; j += nw) {
      if (final_)
        run_item<PH_O, BF16, TI, DP, ROWS>(p, e, h, j, 0, wsm, vbits, lane);
      else
        run_item<PH_L, BF16, TI, DP, ROWS>(p, e, h, j, 0, wsm, vbits, lane);
    }
    cluster_sync();
  }
}

// CTAs per head (1, 2, 4 or 8).  CTAs of equal length run in waves of `slots`
// (resident CTAs on the GPU), so a forward takes about
// ceil(heads * C / slots) waves of 1 / C of a head's work; each doubling of
// C costs ~10 % in cluster barriers and idle warps (a phase has only 14-32
// items).  Measured on B200: ViT (768 heads) best at 2, RoBERTa (384 heads,
// one wave) at 1, DiT (512 heads) at 4, BART-1k (48 heads) at 8.
// MA_SMALL_CLUSTER overrides.
static int cluster_size(int heads, int slots, int items) {
  const char* env = getenv("MA_SMALL_CLUSTER");
  if (env) {
    const int c = atoi(env);
    if (c == 1 || c == 2 || c == 4 || c == 8) return c;
  }
  int best_c = 1;
  double best = 1e300;
  // up to 8 CTAs, while the cluster's warps have an item each in every phase
  for (int c = 1, lg = 0; c <= 8 && (c == 1 || c * kWarps <= items); c *= 2, ++lg) {
    const int64_t waves = ((int64_t)heads * c + slots - 1) / slots;
    const double cost = (double)waves / c * (1.0 + 0.1 * lg);
    if (cost < best - 1e-9) {
      best = cost;
      best_c = c;
    }
  }
  return best_c;
}

template <bool BF16, typename TI, int DP, int ROWS>
static cudaError_t launch(const SmallParams& sp, cudaStream_t st) {
  using WT = WarpTiles<TI, DP, ROWS>;
  const size_t smem = (size_t)kWarps * WT::kBytes + WT::kBitmapBytes;
  auto kfn = ma_small_kernel<BF16, TI, DP, ROWS>;
  cudaError_t err =
      cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  int dev = 0, sms = 0;
  err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (err != cudaSuccess) return err;
  const int heads = sp.E * sp.H;
  const int csize = cluster_size(heads, sms * (ROWS == 16 ? 4 : 3), sp.b > sp.M ? sp.b : sp.M);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(heads * csize));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kfn, sp);
}

}  // namespace small

// ma_small_f32.cu: the same fused kernel in fp32 (FFMA)
bool small_f32_supports(const ma_fwd_params* p, const Shape& s);
// ma_small_res.cu: the head-resident variant (intermediates in shared memory)
bool small_res_supports(const ma_fwd_params* p, const Shape& s);
cudaError_t run_small_res(const ma_fwd_params* p, const Shape& s, cudaStream_t st, int* nlaunch);
cudaError_t run_small_f32(const ma_fwd_params* p, const Shape& s, const WsLayout& ws,
                          cudaStream_t st, int* nlaunch);

bool small_supports(const ma_fwd_params* p, const Shape& s) {
  if (p->dtype == MA_DTYPE_F32) return small_f32_supports(p, s);
  if (p->dtype != MA_DTYPE_BF16 && p->dtype != MA_DTYPE_F16) return false;
  if (s.b > small::kRows || s.M > small::kRows) return false;
  if (s.D != s.Dv || s.D % 8 != 0 || s.D > 128) return false;
  if ((int64_t)s.E * s.H * 4 > 2147483647) return false;
  const int64_t* st[4] = {p->q_stride, p->k_stride, p->v_stride, p->o_stride};
  for (int t = 0; t < 3; ++t) {  // q / k / v rows read with 16-byte copies
    if (st[t][3] != 1) return false;
    for (int i = 0; i < 3; ++i)
      if ((st[t][i] * 2) % 16 != 0) return false;
  }
  if (st[3][3] != 1 || (st[3][2] * 2) % 4 != 0) return false;
  const void* ptrs[3] = {p->q, p->k, p->v};
  for (int i = 0; i < 3; ++i)
    if (ptrs[i] && (reinterpret_cast<uintptr_t>(ptrs[i]) & 15)) return false;
  if (p->out && (reinterpret_cast<uintptr_t>(p->out) & 3)) return false;
  return true;
}

cudaError_t run_small(const ma_fwd_params* p, const Shape& s, const WsLayout& ws,
                      cudaStream_t st, int* nlaunch) {
  if (p->dtype == MA_DTYPE_F32) return run_small_f32(p, s, ws, st, nlaunch);
  if (small_res_supports(p, s)) return run_small_res(p, s, st, nlaunch);
  small::SmallParams sp{};
  sp.q = p->q; sp.k = p->k; sp.v = p->v; sp.out = p->out;
  for (int i = 0; i < 4; ++i) {
    sp.qs[i] = p->q_stride[i]; sp.ks[i] = p->k_stride[i];
    sp.vs[i] = p->v_stride[i]; sp.os[i] = p->o_stride[i];
  }
  sp.mask = p->mask_dtype == MA_MASK_NONE ? nullptr : p->mask;
  sp.ms[0] = p->mask_stride[0]; sp.ms[1] = p->mask_stride[1];
  sp.mask_dtype = p->mask_dtype;
  sp.E = s.E; sp.H = s.H; sp.N = s.N; sp.D = s.D; sp.b = s.b; sp.M = s.M; sp.T = s.T;
  sp.pad_off = s.pad_off; sp.sm_scale = s.sm_scale;
  char* w = reinterpret_cast<char*>(p->workspace);
  sp.al = w + ws.al; sp.y = w + ws.y; sp.ar = w + ws.ar;
  sp.cl = reinterpret_cast<float*>(w + ws.cl);
  sp.cr = reinterpret_cast<float*>(w + ws.cr);
  const bool bf = p->dtype == MA_DTYPE_BF16;
  const int dp = (s.D + 15) / 16 * 16;
  cudaError_t err;
  const bool r16 = s.b <= 16 && s.M <= 16;
#define MA_SMALL_CASE(DPV)                                                              \
  case DPV:                                                                             \
    if (r16)                                                                            \
      err = bf ? small::launch<true, __nv_bfloat16, DPV, 16>(sp, st)                    \
               : small::launch<false, __half, DPV, 16>(sp, st);                         \
    else                                                                                \
      err = bf ? small::launch<true, __nv_bfloat16, DPV, 32>(sp, st)                    \
               : small::launch<false, __half, DPV, 32>(sp, st);                         \
    break;
  switch (dp) {
    MA_SMALL_CASE(16)
    MA_SMALL_CASE(32)
    MA_SMALL_CASE(48)
    MA_SMALL_CASE(64)
    MA_SMALL_CASE(80)
    MA_SMALL_CASE(96)
    MA_SMALL_CASE(112)
    MA_SMALL_CASE(128)
    default: return cudaErrorInvalidValue;
  }
#undef MA_SMALL_CASE
  if (err == cudaSuccess) *nlaunch += 1;
  return err;
}

}  // namespace ma
