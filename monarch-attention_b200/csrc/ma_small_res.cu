// Head-resident small-block MonarchAttention forward (16-bit inputs, head
// dim 64 or 128, block size b <= 32, number of blocks M <= 32): one CTA runs
// every phase of one (batch, head) -- the T-1 (R, L) rounds, the final
// R-step and the output step of ma/ma_torch.py:100-105 -- and keeps all of
// the head's intermediates in shared memory:
//   al  [b][M] rows of D   R-step output, read by the L / output step (:21)
//   ary [M][b] rows of D   L-step output ar (:34), read by the next R-step;
//                          the final R-step writes y (:51) into the same rows
//                          (item m overwrites exactly the rows ar[m][.] it
//                          read), and the output step reads y[.][j] from them
//   cl  [b][M], cr [M][b]  fp32 row statistics (:20, :32)
// Only q, k and v come from global memory: a warp stages the rows of its
// item with cp.async (16-byte chunks, zero rows outside the sequence).  The
// all-to-all exchange between phases (items m write rows j of every item j
// of the next phase) is a __syncthreads, with no global round trip and no
// cluster barrier.  Used where the arrays fit (ViT, RoBERTa shapes); the
// workspace kernel in ma_small.cu covers the other b, M <= 32 shapes.
//
// Every 16-bit row in shared memory is 128-byte segments of eight 16-byte
// chunks; chunk c of an item row t sits at position c ^ ((t ^ f) & 7) of its
// segment, where f is a per-item constant (the item index for the strided
// views al[j][.], ar[m][.], y[.][j]; 0 for a staging tile), so ldmatrix reads
// of eight consecutive item rows hit distinct banks whichever view is read.
#include <float.h>
#include <stdlib.h>

#include "ma_common.cuh"
#include "ma_mma_sync.cuh"

namespace ma {
namespace smallr {

using namespace mmas;

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

struct Params {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int64_t qs[4], ks[4], vs[4], os[4];  // element strides
  const void* mask;
  int64_t ms[2];
  int mask_dtype;
  int E, H, N, b, M, T, pad_off;
  float sm_scale;
  unsigned long long* trace;  // MA_SMALL_TRACE builds: per-head phase timestamps, else null
};

// Optional per-head timeline (compiled in with -DMA_SMALL_TRACE): slot 0 the
// start, slot 1 the bitmap built, slot 2 + i the end of phase i (16 slots).
__device__ __forceinline__ void trace_stamp(const Params& p, int head, int slot) {
#ifdef MA_SMALL_TRACE
  if (p.trace != nullptr && threadIdx.x == 0 && slot < 16) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    p.trace[(size_t)head * 16 + slot] = t;
  }
#else
  (void)p; (void)head; (void)slot;
#endif
}

enum { PH_R = 0, PH_RF = 1, PH_L = 2, PH_O = 3 };

// A view of item rows t = 0, 1, ... in shared memory: row t at base + t *
// stride, 16-byte chunk c at segment c / 8, position (c % 8) ^ ((t ^ f) % 8).
// Operand reads clamp t to the item's last valid row: the padding rows and
// columns of an item (t >= b or M) then hold finite copies of valid data,
// which the softmax masks or multiplies by an exact zero, and no read leaves
// the head's arrays.
struct View {
  uint32_t base, stride;
  int f;
  __device__ __forceinline__ uint32_t chunk(int t, int c) const {
    return base + (uint32_t)t * stride + ((uint32_t)(c >> 3) << 7) +
           ((uint32_t)((c & 7) ^ ((t ^ f) & 7)) << 4);
  }
};

// Offset of the validity bitmap: behind al, ary (b M rows each) and cl, cr
// (b M floats each), rounded up to 128 bytes so that the staging tiles
// behind it stay 16-byte aligned for cp.async and ldmatrix whatever b M is.
__host__ __device__ constexpr size_t bits_offset(int np, int row_bytes) {
  return ((size_t)2 * np * row_bytes + (size_t)2 * np * 4 + 127) / 128 * 128;
}

// bytes of shared memory for a head of b x M items, tiles of RT rows
template <int DP>
__host__ __device__ constexpr size_t smem_bytes(int b, int M, int RT) {
  return bits_offset(b * M, DP * 2)     // al, ary, cl, cr
         + 128                          // validity bitmap (<= 1024 tokens)
         + (size_t)kWarps * 2 * RT * (DP * 2);  // staging tiles T0, T1 per warp
}

// validity of padded token pidx (pad positions and the mask row)
__device__ __forceinline__ bool vbit(const uint32_t* bits, int pidx) {
  return (bits[pidx >> 5] >> (pidx & 31)) & 1u;
}

// Stage rows t = 0 .. R-1 of a q / k / v operand into a tile (view f = 0):
// row t is padded token tok0 + t * tstep when t < rows, zero otherwise.
// Lane (rl, c) copies 16-byte chunk c of rows rl, rl + RPI, ...; the source
// address is affine in t, and as RPI (2 or 4) divides 8 and rl < RPI, the
// swizzled position (c ^ t) & 7 of row t0 + rl is ((c ^ rl) & 7) ^ (t0 & 7),
// a constant per pass.
template <int DP, int R>
__device__ __forceinline__ void stage(const View& dst, const char* base, int64_t stride_b,
                                      const Params& p, int tok0, int tstep, int rows, int lane) {
  constexpr int CH = DP / 8;
  constexpr int RPI = 32 / CH;  // rows per pass of the warp
  static_assert(RPI == 2 || RPI == 4, "staging passes of 2 or 4 rows");
  const int rl = lane / CH, c = lane % CH;
  int n = tok0 + rl * tstep - p.pad_off;
  const char* s = base + n * stride_b + c * 16;
  const int64_t step = RPI * tstep * stride_b;
  const uint32_t d0 = dst.base + (uint32_t)rl * dst.stride + ((uint32_t)(c >> 3) << 7);
  const uint32_t x = (uint32_t)((c ^ rl) & 7);
#pragma unroll
  for (int t0 = 0; t0 < R; t0 += RPI) {
    const bool ok = t0 + rl < rows && (unsigned)n < (unsigned)p.N;
    cp_async16(d0 + (uint32_t)t0 * dst.stride + ((x ^ (uint32_t)(t0 & 7)) << 4), ok ? s : base,
               ok);
    s += step;
    n += RPI * tstep;
  }
}

// Issue (no wait) the cp.async copies of the q / k / v rows an item reads:
// R-steps k[m] -> T1, the first round's q[m] -> T0, the final R-step's v[m]
// -> T0 (after round 0; a single-round call stages v inside the item, once
// GEMM1 has read q); L / output steps Q_j -> T0.  q, k and v are inputs, so
// a warp may stage its next item while other warps finish the current phase.
template <int PH, int DP, int RB, int RM>
__device__ __forceinline__ void stage_item(const Params& p, int e, int h, int item, bool first,
                                           uint32_t t0s, uint32_t t1s, int lane) {
  constexpr int RBY = DP * 2;
  const View T0{t0s, RBY, 0}, T1{t1s, RBY, 0};
  const char* qh = reinterpret_cast<const char*>(p.q) + 2 * (e * p.qs[0] + h * p.qs[1]);
  if (PH == PH_R || PH == PH_RF) {
    const char* kh = reinterpret_cast<const char*>(p.k) + 2 * (e * p.ks[0] + h * p.ks[1]);
    if (first) stage<DP, RB>(T0, qh, 2 * p.qs[2], p, item * p.b, 1, p.b, lane);
    stage<DP, RB>(T1, kh, 2 * p.ks[2], p, item * p.b, 1, p.b, lane);
    if (PH == PH_RF && !first) {
      const char* vh = reinterpret_cast<const char*>(p.v) + 2 * (e * p.vs[0] + h * p.vs[1]);
      stage<DP, RB>(T0, vh, 2 * p.vs[2], p, item * p.b, 1, p.b, lane);
    }
  } else {
    stage<DP, RM>(T0, qh, 2 * p.qs[2], p, item, p.b, p.M, lane);
  }
}

// One work item, executed by one warp.  R / RF: key block m (RB x RB logits:
// rows j, columns i of block m).  L / O: index j (RM x RM logits: rows l,
// columns k).  Rows and columns beyond b (R) or M (L / O) are padding.
template <int PH, bool BF16, int DP, int RB, int RM>
__device__ void run_item(const Params& p, int e, int h, int item, bool first, bool staged,
                         uint8_t* sm, uint32_t t0s, uint32_t t1s, int lane, int mt_lo = 0,
                         int mt_hi = 2) {
  constexpr bool kR = PH == PH_R || PH == PH_RF;
  constexpr int ROWS = kR ? RB : RM;
  constexpr int MT = ROWS / 16;  // m16 tiles
  constexpr int NT = ROWS / 8;   // n8 tiles of the logit columns
  constexpr int NK = DP / 16;    // k16 steps over the head dim
  constexpr int ND = DP / 8;     // n8 tiles over the head dim
  constexpr int RBY = DP * 2;
  using TI = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  const int b = p.b, M = p.M;
  const int R = kR ? b : M;  // valid rows = valid columns of the item
  const uint32_t s_al = smem_u32(sm);
  const uint32_t s_ary = s_al + (uint32_t)(b * M * RBY);
  float* cl = reinterpret_cast<float*>(sm + 2 * (size_t)b * M * RBY);
  float* cr = cl + b * M;
  const uint32_t* vbits = reinterpret_cast<const uint32_t*>(sm + bits_offset(b * M, RBY));
  const View T0{t0s, RBY, 0}, T1{t1s, RBY, 0};
  const size_t esz = sizeof(TI);
  const char* vh = reinterpret_cast<const char*>(p.v) + esz * (e * p.vs[0] + h * p.vs[1]);

  // ---- operand views (staged rows: stage_item, here or ahead) ----
  if (!staged) stage_item<PH, DP, RB, RM>(p, e, h, item, first, t0s, t1s, lane);
  View A, B, X1, X2;
  if (kR) {
    // A: q block m (first round) or ar[m][.] (resident); B, X1: k block m;
    // X2: v block m (final R-step)
    A = first ? T0 : View{s_ary + (uint32_t)(item * b * RBY), RBY, item};
    B = T1;
    X1 = T1;
    X2 = T0;
  } else {
    // A: Q_j = tokens l * b + j; B: al[j][.] (resident); X1 (output step):
    // y[.][j] (resident rows m * b + j)
    A = T0;
    B = View{s_al + (uint32_t)(item * M * RBY), RBY, item};
    X1 = View{s_ary + (uint32_t)(item * RBY), (uint32_t)(b * RBY), item};
  }
  cp_async_wait_all();
  __syncwarp();

  const int g = lane >> 2, t4 = lane & 3;
  // columns of this lane's fragments: c = nt * 8 + 2 t4 + q
  bool colv[NT][2];
  float colc[NT][2];  // L / out: cl[j][k] in log2 units
  bool allv = true;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int c = nt * 8 + 2 * t4 + q;
      colv[nt][q] = c < R && (!kR || vbit(vbits, item * b + c));
      colc[nt][q] = (!kR && c < R) ? cl[item * M + c] * kLog2e : 0.0f;
      allv = allv && colv[nt][q];
    }
  allv = __all_sync(0xffffffffu, allv);
  float colsum[NT][2];  // L: column sums of P (cr)
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) colsum[nt][0] = colsum[nt][1] = 0.0f;
  // P^T staging of L items (rows l, 16-bit, stride 80 bytes) in tile T1
  const uint32_t tP = t1s;
  constexpr int kPS = 40;  // elements per staged row

  // the final R-step's V goes into T0: at once when A is resident; in a
  // single-round call (T = 1, A = q in T0) after GEMM1, which then has one
  // row tile only (b <= 16, see small_res_supports)
  bool v_staged = PH == PH_RF && !first;
  const int rlast = R - 1;

  // 16-row tiles mt_lo .. mt_hi - 1 of the item (all of them, or one half
  // of an R item shared by a warp pair)
  if (mt_hi > MT) mt_hi = MT;
#pragma unroll 1
  for (int mt = mt_lo; mt < mt_hi; ++mt) {
    // ---- S row tile = A[mt] B^T ----
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[nt][i] = 0.0f;
#pragma unroll
    for (int ks = 0; ks < NK; ++ks) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(A.chunk(min(mt * 16 + (lane & 15), rlast), 2 * ks + (lane >> 4)), a0, a1, a2, a3);
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(B.chunk(min(np * 16 + (lane & 7) + (lane >> 4) * 8, rlast), 2 * ks + ((lane >> 3) & 1)),
                b0, b1, b2, b3);
        mma16816<BF16>(acc[2 * np], a0, a1, a2, a3, b0, b1);
        mma16816<BF16>(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // ---- softmax over the columns of each row (log2 units: one FMA + ex2) ----
    float row_scale[2], cl_row[2];
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = mt * 16 + g + 8 * hf;
      float c = 1.0f;
      if (kR) {
        const float crj = (first || r >= R) ? 1.0f : cr[item * b + r];
        c = __fdividef(p.sm_scale, crj + kEps);  // t = sm_scale * S / (cr + eps), ma_torch.py:11-12
      }
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          float x = acc[nt][2 * hf + q];
          if (!kR) x -= colc[nt][q] * kLn2;
          if (!allv && !colv[nt][q]) x = -INFINITY;
          mx = fmaxf(mx, x);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      float ua, ub;
      if (kR) {
        ua = c * kLog2e;
        ub = -fmaxf(c * mx, kEps) * kLog2e;  // clamp(max t, min=eps), :14-16
      } else {
        ua = kLog2e;
        ub = -mx * kLog2e;
      }
      float sum = 0.0f, wsum = 0.0f;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          float& x = acc[nt][2 * hf + q];
          const float u = fmaf(x, ua, kR ? ub : ub - colc[nt][q]);
          float ev = ex2f(u);
          if (!allv && !colv[nt][q]) ev = 0.0f;
          sum += ev;
          if (kR) wsum = fmaf(ev, (allv || colv[nt][q]) ? u : 0.0f, wsum);
          x = ev;
        }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      if (kR) {
        wsum += __shfl_xor_sync(0xffffffffu, wsum, 1);
        wsum += __shfl_xor_sync(0xffffffffu, wsum, 2);
        const float den = sum + kEps;  // r = e / (sum + eps), :17
        const float inv = __fdividef(1.0f, den);
        // sum_i r_i log r_i, log r_i = ln2 * u_i - log(den) (:20)
        cl_row[hf] = kLn2 * inv * wsum - __logf(den) * sum * inv;
        row_scale[hf] = inv;
      } else {
        cl_row[hf] = 0.0f;
        row_scale[hf] = __fdividef(1.0f, sum);
      }
      {
        // P is normalised before it is packed for the second matmul (the
        // reference's r.to(dtype) / l.to(dtype)): L rows times the query
        // mask of row l (:30); a plain R-step's rows also carry al's
        // sm_scale (:21), so no output scales
        float sc = row_scale[hf];
        if (PH == PH_L && !(r < R && vbit(vbits, r * b + item))) sc = 0.0f;
        if (PH == PH_R) sc *= p.sm_scale;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int q = 0; q < 2; ++q) acc[nt][2 * hf + q] *= sc;
      }
    }
    if (kR) {  // cl[j][m] (:20)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = mt * 16 + g + 8 * hf;
        if (t4 == 0 && r < R) cl[r * M + item] = cl_row[hf];
      }
    }

    if constexpr (PH == PH_L) {
      // cr partial sums and P (16-bit) -> staging P[l][k]
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int q = 0; q < 2; ++q) colsum[nt][q] += acc[nt][q] + acc[nt][2 + q];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = mt * 16 + g + 8 * hf, c = nt * 8 + 2 * t4;
          st_shared_b32(tP + (r * kPS + c) * 2, pack2<BF16>(acc[nt][2 * hf], acc[nt][2 * hf + 1]));
        }
    } else {
      // ---- R / out: output row tile O = P X ----
      const int nparts = PH == PH_RF ? 2 : 1;
#pragma unroll 1
      for (int part = 0; part < nparts; ++part) {
        if (PH == PH_RF && part == 1 && !v_staged) {
          // T = 1: the only row tile's GEMM1 has read q from T0
          stage<DP, RB>(T0, vh, esz * p.vs[2], p, item * b, 1, b, lane);
          cp_async_wait_all();
          __syncwarp();
          v_staged = true;
        }
        const View X = part == 0 ? X1 : X2;
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
            const int xr = min(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, rlast);
            ldsm_x4_t(X.chunk(xr, 2 * np + (lane >> 4)), b0, b1, b2, b3);
            mma16816<BF16>(o[2 * np], a0, a1, a2, a3, b0, b1);
            mma16816<BF16>(o[2 * np + 1], a0, a1, a2, a3, b2, b3);
          }
        }
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = mt * 16 + g + 8 * hf;
          if (r >= R) continue;
          // P is normalised already (and carries sm_scale in a plain
          // R-step): only the final R-step's al part is scaled here
          const bool scaled = PH == PH_RF && part == 0;
          const float sc = p.sm_scale;
          if (kR) {
            // al[j][m] = sm_scale * (r K[m]) (:21) -> al row (j, m);
            // y[j][m] = r V[m] (:51) -> ary row (m, j)
            const View dst = part == 0
                ? View{s_al + (uint32_t)(item * RBY), (uint32_t)(M * RBY), item}
                : View{s_ary + (uint32_t)(item * b * RBY), RBY, item};
#pragma unroll
            for (int nd = 0; nd < ND; ++nd)
              st_shared_b32(dst.chunk(r, nd) + 4 * t4,
                            scaled ? pack2<BF16>(o[nd][2 * hf] * sc, o[nd][2 * hf + 1] * sc)
                                   : pack2<BF16>(o[nd][2 * hf], o[nd][2 * hf + 1]));
          } else {
            // z at token l * b + j (:60-62, :106-108)
            const int n = r * b + item - p.pad_off;
            if (n < 0 || n >= p.N) continue;
            char* dst = reinterpret_cast<char*>(p.out) +
                        esz * ((int64_t)e * p.os[0] + (int64_t)h * p.os[1] + (int64_t)n * p.os[2]);
#pragma unroll
            for (int nd = 0; nd < ND; ++nd)
              *reinterpret_cast<uint32_t*>(dst + (nd * 8 + 2 * t4) * esz) =
                  pack2<BF16>(o[nd][2 * hf], o[nd][2 * hf + 1]);
          }
        }
      }
    }
  }

  if constexpr (PH == PH_L) {
    // cr[k][j] = sum_l P[l][k] (:32)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        float s = colsum[nt][q];
        s += __shfl_xor_sync(0xffffffffu, s, 4);
        s += __shfl_xor_sync(0xffffffffu, s, 8);
        s += __shfl_xor_sync(0xffffffffu, s, 16);
        const int c = nt * 8 + 2 * t4 + q;
        if (g == 0 && c < R) cr[c * b + item] = s;
      }
    __syncwarp();
    // ar[k][j] = sum_l P[l][k] q[l*b+j] (:34): A = P^T read transposed from
    // the staging, B = Q_j (tile T0); -> ary rows (k, j)
    const View dst{s_ary + (uint32_t)(item * RBY), (uint32_t)(b * RBY), item};
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
        ldsm_x4_t(tP + (lrow * kPS + kcol) * 2, a0, a1, a2, a3);
#pragma unroll
        for (int np = 0; np < ND / 2; ++np) {
          uint32_t b0, b1, b2, b3;
          const int xr = min(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, rlast);
          ldsm_x4_t(A.chunk(xr, 2 * np + (lane >> 4)), b0, b1, b2, b3);
          mma16816<BF16>(o[2 * np], a0, a1, a2, a3, b0, b1);
          mma16816<BF16>(o[2 * np + 1], a0, a1, a2, a3, b2, b3);
        }
      }
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = mt * 16 + g + 8 * hf;  // k
        if (r >= R) continue;
#pragma unroll
        for (int nd = 0; nd < ND; ++nd)
          st_shared_b32(dst.chunk(r, nd) + 4 * t4, pack2<BF16>(o[nd][2 * hf], o[nd][2 * hf + 1]));
      }
    }
  }
  __syncwarp();
}

__device__ __forceinline__ bool token_valid(const Params& p, int e, int pidx) {
  const int n = pidx - p.pad_off;
  if (n < 0 || n >= p.N) return false;
  if (p.mask == nullptr) return true;
  return mask_value(p.mask, p.mask_dtype, (int64_t)e * p.ms[0] + (int64_t)n * p.ms[1]);
}

// SPLIT (D = 64, 32-row R items, 16-row L / output items: the RoBERTa
// shape, whose resident arrays leave room for one CTA per SM): 16 warps in
// 8 pairs.  A pair shares one staging slot (T0, T1 of 32 rows); its two
// warps take the two 16-row halves of each R item (row-local softmax, each
// writing its own rows of al, cl, y), with a named barrier per pair after
// the shared operands landed and before they are replaced.  L / output
// items stay one per warp, in the warp's half of the slot (Q_j, then P^T).
// Twice the warps of the 8-warp layout in the same shared memory.
__device__ __forceinline__ void pair_sync(int pair) {
  asm volatile("bar.sync %0, 64;" ::"r"(1 + pair) : "memory");
}

template <bool BF16, int DP, int RB, int RM, bool SPLIT>
__global__ void __launch_bounds__(SPLIT ? 2 * kThreads : kThreads,
                                  (RB == 16 && RM == 16) ? 2 : 1)
    ma_small_res_kernel(const Params p) {
  extern __shared__ __align__(128) uint8_t sm[];
  constexpr int RT = RB > RM ? RB : RM;
  constexpr int kW = SPLIT ? 2 * kWarps : kWarps;  // warps of the CTA
  static_assert(!SPLIT || (DP == 64 && RB == 32 && RM == 16), "pair layout: RoBERTa shape");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int eh = blockIdx.x;
  const int e = eh / p.H, h = eh - e * p.H;
  const int b = p.b, M = p.M;
  const size_t res = bits_offset(b * M, DP * 2);
  uint32_t* vbits = reinterpret_cast<uint32_t*>(sm + res);
  uint8_t* tiles = sm + res + 128;
  const int slot = SPLIT ? warp >> 1 : warp;  // staging slot (T0, T1)
  const uint32_t t0s = smem_u32(tiles + (size_t)slot * 2 * RT * (DP * 2));
  const uint32_t t1s = t0s + RT * (DP * 2);
  trace_stamp(p, eh, 0);
  // token validity of the padded sequence (pad positions and the mask row)
  // (one lane per token, so the mask loads of a word are issued together)
  const int Np = M * b;
  for (int w = warp; w < (Np + 31) / 32; w += kW) {
    const int pidx = w * 32 + lane;
    const uint32_t bits = __ballot_sync(0xffffffffu, pidx < Np && token_valid(p, e, pidx));
    if (lane == 0) vbits[w] = bits;
  }
  __syncthreads();
  trace_stamp(p, eh, 1);
  if constexpr (SPLIT) {
    const int pair = warp >> 1, half = warp & 1;
    constexpr int kPairs = kW / 2;
    constexpr int RBY = DP * 2;
    // this warp's half of the slot for L / output items: Q_j, then P^T
    const uint32_t l0 = t0s + (uint32_t)half * (RT * RBY), l1 = l0 + RM * RBY;
    const char* qh = reinterpret_cast<const char*>(p.q) + 2 * (e * p.qs[0] + h * p.qs[1]);
    const char* kh = reinterpret_cast<const char*>(p.k) + 2 * (e * p.ks[0] + h * p.ks[1]);
    const char* vh = reinterpret_cast<const char*>(p.v) + 2 * (e * p.vs[0] + h * p.vs[1]);
    for (int t = 0; t < p.T; ++t) {
      const bool final_ = t == p.T - 1, first = t == 0;
      for (int m = pair; m < M; m += kPairs) {
        // half 0 stages T0 (q[m] in the first round, v[m] in the final one),
        // half 1 stages T1 (k[m])
        const View T0{t0s, RBY, 0}, T1{t1s, RBY, 0};
        if (half == 0) {
          if (first) stage<DP, RB>(T0, qh, 2 * p.qs[2], p, m * b, 1, b, lane);
          else if (final_) stage<DP, RB>(T0, vh, 2 * p.vs[2], p, m * b, 1, b, lane);
        } else {
          stage<DP, RB>(T1, kh, 2 * p.ks[2], p, m * b, 1, b, lane);
        }
        cp_async_wait_all();
        pair_sync(pair);
        if (final_)
          run_item<PH_RF, BF16, DP, RB, RM>(p, e, h, m, first, true, sm, t0s, t1s, lane, half,
                                            half + 1);
        else
          run_item<PH_R, BF16, DP, RB, RM>(p, e, h, m, first, true, sm, t0s, t1s, lane, half,
                                           half + 1);
        pair_sync(pair);
      }
      __syncthreads();
      trace_stamp(p, eh, 2 + 2 * t);
      for (int j = warp; j < b; j += kW) {
        stage_item<PH_L, DP, RB, RM>(p, e, h, j, false, l0, l1, lane);
        if (final_)
          run_item<PH_O, BF16, DP, RB, RM>(p, e, h, j, false, true, sm, l0, l1, lane);
        else
          run_item<PH_L, BF16, DP, RB, RM>(p, e, h, j, false, true, sm, l0, l1, lane);
      }
      __syncthreads();
      trace_stamp(p, eh, 3 + 2 * t);
    }
    return;
  }
  // Each warp stages the q / k / v rows of its next item as soon as the
  // current one is done -- across phase barriers too (they are inputs) -- so
  // an item waits only for copies issued an item earlier.
  if (warp < M)
    stage_item<PH_R, DP, RB, RM>(p, e, h, warp, true, t0s, t1s, lane);  // same rows as RF
  for (int t = 0; t < p.T; ++t) {
    const bool final_ = t == p.T - 1;
    for (int m = warp; m < M; m += kWarps) {
      if (final_)
        run_item<PH_RF, BF16, DP, RB, RM>(p, e, h, m, t == 0, true, sm, t0s, t1s, lane);
      else
        run_item<PH_R, BF16, DP, RB, RM>(p, e, h, m, t == 0, true, sm, t0s, t1s, lane);
      // next: this phase's next R item, else this warp's first L / output item
      if (m + kWarps < M) {
        if (final_)
          stage_item<PH_RF, DP, RB, RM>(p, e, h, m + kWarps, t == 0, t0s, t1s, lane);
        else
          stage_item<PH_R, DP, RB, RM>(p, e, h, m + kWarps, t == 0, t0s, t1s, lane);
      } else if (warp < b) {
        stage_item<PH_L, DP, RB, RM>(p, e, h, warp, false, t0s, t1s, lane);  // = output rows
      }
    }
    if (warp >= M && warp < b)
      stage_item<PH_L, DP, RB, RM>(p, e, h, warp, false, t0s, t1s, lane);
    __syncthreads();
    trace_stamp(p, eh, 2 + 2 * t);
    const bool next_final = t + 1 == p.T - 1;
    for (int j = warp; j < b; j += kWarps) {
      if (final_)
        run_item<PH_O, BF16, DP, RB, RM>(p, e, h, j, false, true, sm, t0s, t1s, lane);
      else
        run_item<PH_L, BF16, DP, RB, RM>(p, e, h, j, false, true, sm, t0s, t1s, lane);
      // next: this phase's next item, else the next round's first R item
      if (j + kWarps < b) {
        stage_item<PH_L, DP, RB, RM>(p, e, h, j + kWarps, false, t0s, t1s, lane);
      } else if (!final_ && warp < M) {
        if (next_final)
          stage_item<PH_RF, DP, RB, RM>(p, e, h, warp, false, t0s, t1s, lane);
        else
          stage_item<PH_R, DP, RB, RM>(p, e, h, warp, false, t0s, t1s, lane);
      }
    }
    if (!final_ && warp >= b && warp < M) {
      if (next_final)
        stage_item<PH_RF, DP, RB, RM>(p, e, h, warp, false, t0s, t1s, lane);
      else
        stage_item<PH_R, DP, RB, RM>(p, e, h, warp, false, t0s, t1s, lane);
    }
    __syncthreads();
    trace_stamp(p, eh, 3 + 2 * t);
  }
}

template <bool BF16, int DP, int RB, int RM, bool SPLIT = false>
static cudaError_t launch(const Params& sp, cudaStream_t st) {
  constexpr int RT = RB > RM ? RB : RM;
  const size_t smem = smem_bytes<DP>(sp.b, sp.M, RT);
  auto kfn = ma_small_res_kernel<BF16, DP, RB, RM, SPLIT>;
  cudaError_t err =
      cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  kfn<<<sp.E * sp.H, SPLIT ? 2 * kThreads : kThreads, smem, st>>>(sp);
  return cudaGetLastError();
}

static int round16(int x) { return x <= 16 ? 16 : 32; }

}  // namespace smallr

// Shapes the head-resident kernel takes: 16-bit inputs, D = Dv in {64, 128},
// b, M <= 32, the head's arrays within 200 KB of shared memory, q / k / v /
// out rows 16-byte aligned.  A single-round call (T = 1) stages V where q
// was, after GEMM1: only with one row tile per item (b <= 16).
bool small_res_supports(const ma_fwd_params* p, const Shape& s) {
  const char* off = getenv("MA_DISABLE_SMALL_RES");
  if (off && off[0] == '1') return false;
  if (p->dtype != MA_DTYPE_BF16 && p->dtype != MA_DTYPE_F16) return false;
  if (p->v_f32) return false;
  if (s.D != s.Dv || (s.D != 64 && s.D != 128)) return false;
  if (s.b > 32 || s.M > 32) return false;
  if (s.T == 1 && s.b > 16) return false;
  const int rt = smallr::round16(s.b) > smallr::round16(s.M) ? smallr::round16(s.b)
                                                             : smallr::round16(s.M);
  const size_t need = s.D == 64 ? smallr::smem_bytes<64>(s.b, s.M, rt)
                                : smallr::smem_bytes<128>(s.b, s.M, rt);
  if (need > 200 * 1024) return false;
  const int64_t* st[4] = {p->q_stride, p->k_stride, p->v_stride, p->o_stride};
  for (int t = 0; t < 3; ++t) {
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

cudaError_t run_small_res(const ma_fwd_params* p, const Shape& s, cudaStream_t st,
                          int* nlaunch) {
  smallr::Params sp{};
  sp.q = p->q; sp.k = p->k; sp.v = p->v; sp.out = p->out;
  for (int i = 0; i < 4; ++i) {
    sp.qs[i] = p->q_stride[i]; sp.ks[i] = p->k_stride[i];
    sp.vs[i] = p->v_stride[i]; sp.os[i] = p->o_stride[i];
  }
  sp.mask = p->mask_dtype == MA_MASK_NONE ? nullptr : p->mask;
  sp.ms[0] = p->mask_stride[0]; sp.ms[1] = p->mask_stride[1];
  sp.mask_dtype = p->mask_dtype;
  sp.E = s.E; sp.H = s.H; sp.N = s.N; sp.b = s.b; sp.M = s.M; sp.T = s.T;
  sp.pad_off = s.pad_off; sp.sm_scale = s.sm_scale;
#ifdef MA_SMALL_TRACE
  const char* trc = getenv("MA_SMALL_TRACE_PTR");  // device buffer of E*H x 16 u64
  if (trc) sp.trace = reinterpret_cast<unsigned long long*>(strtoull(trc, nullptr, 0));
#endif
  const bool bf = p->dtype == MA_DTYPE_BF16;
  const int rb = smallr::round16(s.b), rm = smallr::round16(s.M);
  cudaError_t err = cudaErrorInvalidValue;
#define MA_RES_CASE(DPV, RBV, RMV)                                                        \
  if (s.D == DPV && rb == RBV && rm == RMV)                                               \
    err = bf ? smallr::launch<true, DPV, RBV, RMV>(sp, st)                                \
             : smallr::launch<false, DPV, RBV, RMV>(sp, st);
  MA_RES_CASE(64, 16, 16)
  // D = 64, 32-row R items, 16-row L items (RoBERTa): the 16-warp pair
  // layout (MA_SMALL_RES_PAIRS=0 selects the 8-warp one)
  const char* pairs = getenv("MA_SMALL_RES_PAIRS");
  if (s.D == 64 && rb == 32 && rm == 16 && !(pairs && pairs[0] == '0')) {
    err = bf ? smallr::launch<true, 64, 32, 16, true>(sp, st)
             : smallr::launch<false, 64, 32, 16, true>(sp, st);
  } else
  MA_RES_CASE(64, 32, 16)
  MA_RES_CASE(64, 16, 32)
  MA_RES_CASE(64, 32, 32)
  MA_RES_CASE(128, 16, 16)
  MA_RES_CASE(128, 32, 16)
  MA_RES_CASE(128, 16, 32)
  MA_RES_CASE(128, 32, 32)
#undef MA_RES_CASE
  if (err == cudaSuccess) *nlaunch += 1;
  return err;
}

}  // namespace ma
