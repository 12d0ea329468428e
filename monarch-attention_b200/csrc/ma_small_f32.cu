// Fused small-block MonarchAttention forward in fp32 (the reference's
// default precision for its fp32 pipelines, e.g. DiT, dit/pipeline.py:147-159,
// and the fp32 parity configuration): one thread-block cluster runs every
// phase of one (batch, head) -- the T-1 (R, L) rounds, the final R-step and
// the output step of ma/ma_torch.py:100-105 -- with a cluster barrier
// between phases, like the 16-bit small-block kernel (ma_small.cu).  Block
// size b <= 32, number of blocks M <= 32, D = Dv <= 128 (multiple of 4), any
// padding and key-padding mask.
//
// The arithmetic is fp32 FFMA throughout (no TF32: the fp32 result must stay
// within 1e-4 of the reference): a warp owns one item, stages its operands
// in shared memory with cp.async, and computes the R x C logit block as a
// register tile per lane (rows ry + 8 i, columns cx + 4 j; lane = 4 ry + cx),
// the row softmax with quad shuffles, then the output block from P staged in
// shared memory (rows ry + 8 i, 8 consecutive columns per lane).
#include <float.h>
#include <stdlib.h>

#include "ma_common.cuh"

namespace ma {
namespace smallf {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;

struct Params {
  const float* q;
  const float* k;
  const float* v;
  float* out;
  int64_t qs[4], ks[4], vs[4], os[4];
  const void* mask;
  int64_t ms[2];
  int mask_dtype;
  int E, H, N, D, b, M, T, pad_off;
  float sm_scale;
  float* al;  // [E*H][b][M][D]
  float* y;   // [E*H][b][M][D]
  float* ar;  // [E*H][M][b][D]
  float* cl;  // [E*H][b][M]
  float* cr;  // [E*H][M][b]
};

enum { PH_R = 0, PH_RF = 1, PH_L = 2, PH_O = 3 };

constexpr float kLog2eS = 1.4426950408889634f;
constexpr float kLn2S = 0.6931471805599453f;

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
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ bool token_valid(const Params& p, int e, int pidx) {
  const int n = pidx - p.pad_off;
  if (n < 0 || n >= p.N) return false;
  if (p.mask == nullptr) return true;
  return mask_value(p.mask, p.mask_dtype, (int64_t)e * p.ms[0] + (int64_t)n * p.ms[1]);
}
__device__ __forceinline__ bool valid_bit(const uint32_t* bits, int pidx) {
  return (bits[pidx >> 5] >> (pidx & 31)) & 1u;
}

// Shared memory of a warp: tiles A, B, X (ROWS rows x RS floats; RS = DP + 4
// puts the rows of a quarter-warp's 16-byte loads in distinct banks), the P
// staging block (ROWS x PS floats) and the item's cr / cl vector.
template <int DP, int ROWS>
struct Tiles {
  static constexpr int RS = DP + 4;
  static constexpr int PS = ROWS + 1;
  static constexpr int kTile = ROWS * RS;  // floats
  static constexpr int kBytes = (3 * kTile + ROWS * PS + ROWS) * 4;
  static constexpr int kMaxTokens = ROWS * ROWS;
  static constexpr int kBitmapBytes = kMaxTokens / 8 < 16 ? 16 : kMaxTokens / 8;
};

// Rows r = 0 .. ROWS-1 of an operand into a tile, the first D floats of each
// row in 16-byte pieces.  Row r starts at src + r * rstride floats and is
// copied when r < rows and its token index n0 + r * nstep lies in [0, N)
// (workspace rows: n0 = nstep = 0, N = 1); other rows are zero-filled.  Lane
// (rl, c) copies piece c of rows rl, rl + RPI, ...: the row address is
// affine in r, so a pass costs three additions.
template <int DP, int ROWS>
__device__ __forceinline__ void stage_rows(uint32_t tile, int D, int lane, const float* src,
                                           int64_t rstride, int rows, int n0, int nstep, int N,
                                           const float* safe) {
  constexpr int RS = DP + 4;
  constexpr int CH = DP / 4;    // 16-byte pieces per padded row
  constexpr int RPI = 32 / CH;  // rows per pass of the warp
  const int rl = lane / CH, c = lane - rl * CH;
  if (rl >= RPI || c >= D / 4) return;
  const float* s = src + rl * rstride + c * 4;
  uint32_t d = tile + (uint32_t)(rl * RS + c * 4) * 4;
  int n = n0 + rl * nstep;
#pragma unroll 8
  for (int r0 = 0; r0 < ROWS; r0 += RPI) {
    if (r0 + RPI <= ROWS || r0 + rl < ROWS) {
      const bool ok = r0 + rl < rows && (unsigned)n < (unsigned)N;
      cp_async16(d, ok ? s : safe, ok);
    }
    s += RPI * rstride;
    d += RPI * RS * 4;
    n += RPI * nstep;
  }
}

// ---------------------------------------------------------------------------
// one work item, executed by one warp
// ---------------------------------------------------------------------------
template <int PH, int DP, int ROWS>
__device__ void run_item(const Params& p, int e, int h, int item, int first, float* wsm,
                         const uint32_t* vbits, int lane) {
  using TL = Tiles<DP, ROWS>;
  constexpr int RS = TL::RS, PS = TL::PS;
  constexpr int RT = ROWS / 8;  // rows of the logit block per lane
  constexpr int CT = ROWS / 4;  // columns per lane
  const int D = p.D, b = p.b, M = p.M;
  const int eh = e * p.H + h;
  float* A = wsm;
  float* Bt = A + TL::kTile;
  float* X = Bt + TL::kTile;
  float* Pst = X + TL::kTile;
  float* vec = Pst + ROWS * PS;
  const uint32_t tA = smem_u32(A), tB = smem_u32(Bt), tX = smem_u32(X), tV = smem_u32(vec);
  const bool rph = PH == PH_R || PH == PH_RF;
  const int R = rph ? b : M;  // rows of the item
  const int C = R;            // columns

  const float* al_h = p.al + (size_t)eh * b * M * D;
  const float* y_h = p.y + (size_t)eh * b * M * D;
  const float* ar_h = p.ar + (size_t)eh * M * b * D;
  const float* cl_h = p.cl + (size_t)eh * b * M;
  const float* cr_h = p.cr + (size_t)eh * M * b;
  // q / k / v rows: token n0 + r * nstep of the head (padded index minus the
  // pre-padding), zero rows outside the sequence
  auto stage_tok = [&](uint32_t tile, const float* base, const int64_t* st, int n0, int nstep) {
    const float* hb = base + ((int64_t)e * st[0] + (int64_t)h * st[1]);
    stage_rows<DP, ROWS>(tile, D, lane, hb + (int64_t)n0 * st[2], st[2] * nstep, R, n0, nstep,
                         p.N, hb);
  };
  // workspace rows: row r at base + r * D floats, all R rows valid
  auto stage_ws = [&](uint32_t tile, const float* base) {
    stage_rows<DP, ROWS>(tile, D, lane, base, D, R, 0, 0, 1, base);
  };

  // ---- stage operands (same roles as the 16-bit kernel) ----
  if (rph) {
    if (first)
      stage_tok(tA, p.q, p.qs, item * b - p.pad_off, 1);  // q block m
    else
      stage_ws(tA, ar_h + (size_t)item * b * D);         // ar[m][.]
    stage_tok(tB, p.k, p.ks, item * b - p.pad_off, 1);    // k block m
    if (PH == PH_RF) stage_tok(tX, p.v, p.vs, item * b - p.pad_off, 1);  // v block m
  } else {
    stage_tok(tA, p.q, p.qs, item - p.pad_off, b);        // Q_j: tokens l * b + j
    stage_ws(tB, al_h + (size_t)item * M * D);           // al[j][.]
    if (PH == PH_O) stage_ws(tX, y_h + (size_t)item * M * D);  // y[j][.]
  }
  if (!(rph && first)) {  // the item's cr / cl vector (0 beyond it)
    const float* vsrc = rph ? cr_h + (size_t)item * b : cl_h + (size_t)item * M;
    if (lane < ROWS) {
      const bool ok = lane < (rph ? b : M);
      cp_async4(tV + lane * 4, ok ? vsrc + lane : vsrc, ok);
    }
  }
  cp_async_wait_all();
  __syncwarp();

  const int ry = lane >> 2, cx = lane & 3;
  // columns c = cx + 4 j of this lane: validity (R: key padding / mask) and
  // the per-column term cl[j][k] of L / output logits
  bool colv[CT];
  float colc[CT];
#pragma unroll
  for (int j = 0; j < CT; ++j) {
    const int c = cx + 4 * j;
    colv[j] = c < C && (!rph || valid_bit(vbits, item * b + c));
    colc[j] = (!rph && c < C) ? vec[c] : 0.0f;
  }

  // ---- S = A B^T, rows ry + 8 i, columns cx + 4 j ----
  float s[RT][CT];
#pragma unroll
  for (int i = 0; i < RT; ++i)
#pragma unroll
    for (int j = 0; j < CT; ++j) s[i][j] = 0.0f;
#pragma unroll 2
  for (int d = 0; d < D; d += 4) {
    float4 a[RT];
#pragma unroll
    for (int i = 0; i < RT; ++i) a[i] = *reinterpret_cast<const float4*>(A + (ry + 8 * i) * RS + d);
#pragma unroll
    for (int j = 0; j < CT; ++j) {
      const float4 bb = *reinterpret_cast<const float4*>(Bt + (cx + 4 * j) * RS + d);
#pragma unroll
      for (int i = 0; i < RT; ++i) {
        float t = s[i][j];
        t = fmaf(a[i].x, bb.x, t);
        t = fmaf(a[i].y, bb.y, t);
        t = fmaf(a[i].z, bb.z, t);
        s[i][j] = fmaf(a[i].w, bb.w, t);
      }
    }
  }

  // ---- row softmax (ma_torch.py:11-20 R-steps, :27-29 L-step, :56-57 out) ----
  float row_scale[RT];
#pragma unroll
  for (int i = 0; i < RT; ++i) {
    const int r = ry + 8 * i;
    float c = 1.0f;
    if (rph) {
      const float crj = (first || r >= R) ? 1.0f : vec[r];
      c = __fdividef(p.sm_scale, crj + kEps);  // t = sm_scale * S / (cr + eps), :11-12
    }
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < CT; ++j) {
      const float x = rph ? s[i][j] : s[i][j] - colc[j];
      if (colv[j]) mx = fmaxf(mx, x);
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
    for (int j = 0; j < CT; ++j) {
      const float x = rph ? s[i][j] : s[i][j] - colc[j];
      const float u = fmaf(x, ua, ub);
      const float ev = colv[j] ? ex2f(u) : 0.0f;
      sum += ev;
      if (rph) wsum = fmaf(ev, colv[j] ? u : 0.0f, wsum);
      s[i][j] = ev;
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if (rph) {
      wsum += __shfl_xor_sync(0xffffffffu, wsum, 1);
      wsum += __shfl_xor_sync(0xffffffffu, wsum, 2);
      const float den = sum + kEps;  // r = e / (sum + eps), :17
      const float inv = __fdividef(1.0f, den);
      // cl[j][m] = sum_i r_i log r_i, log r_i = ln2 * u_i - log(den) (:20)
      const float clv = kLn2S * inv * wsum - __logf(den) * sum * inv;
      if (cx == 0 && r < R) p.cl[(size_t)eh * b * M + (size_t)r * M + item] = clv;
      row_scale[i] = inv;
    } else if (PH == PH_L) {
      // L: P is normalised here, times the query mask of row l (:28-30)
      const float sc = (r < R && valid_bit(vbits, r * b + item)) ? __fdividef(1.0f, sum) : 0.0f;
#pragma unroll
      for (int j = 0; j < CT; ++j) s[i][j] *= sc;
      row_scale[i] = 1.0f;
    } else {
      row_scale[i] = __fdividef(1.0f, sum);
    }
  }
  // P -> staging block Pst[r][c] (R / out: unnormalised e, L: normalised)
#pragma unroll
  for (int i = 0; i < RT; ++i)
#pragma unroll
    for (int j = 0; j < CT; ++j) Pst[(ry + 8 * i) * PS + cx + 4 * j] = s[i][j];
  __syncwarp();

  if (PH == PH_L) {  // cr[k][j] = sum_l P[l][k] (:32)
    if (lane < C) {
      float sm = 0.0f;
#pragma unroll 8
      for (int l = 0; l < ROWS; ++l) sm += Pst[l * PS + lane];
      p.cr[(size_t)eh * M * b + (size_t)lane * b + item] = sm;
    }
  }

  // ---- output block: rows ry + 8 i, columns d0 .. d0 + 7 of 32-column chunks ----
  //   R      : al[j][m] = sm_scale * r K[m]  (:21)    X = K[m]  (tile B)
  //   R-final: + y[j][m] = r V[m]           (:51)    X = V[m]  (tile X)
  //   L      : ar[k][j] = sum_l P[l][k] q_l (:34)    X = Q_j   (tile A), P transposed
  //   out    : z[l*b + j] = P y_j / sum     (:60-62) X = y_j   (tile X)
  const int nparts = PH == PH_RF ? 2 : 1;
#pragma unroll 1
  for (int part = 0; part < nparts; ++part) {
    const float* Xs = PH == PH_L ? A : ((rph && part == 0) ? Bt : X);
#pragma unroll 1
    for (int dc = 0; dc < D; dc += 32) {
      const int d0 = dc + cx * 8;
      const bool dok = d0 < D;  // D is a multiple of 8
      float o[RT][8];
#pragma unroll
      for (int i = 0; i < RT; ++i)
#pragma unroll
        for (int t = 0; t < 8; ++t) o[i][t] = 0.0f;
      if (dok) {
#pragma unroll 4
        for (int c = 0; c < ROWS; ++c) {
          const float4 x0 = *reinterpret_cast<const float4*>(Xs + c * RS + d0);
          const float4 x1 = *reinterpret_cast<const float4*>(Xs + c * RS + d0 + 4);
#pragma unroll
          for (int i = 0; i < RT; ++i) {
            const int r = ry + 8 * i;
            const float pv = PH == PH_L ? Pst[c * PS + r] : Pst[r * PS + c];
            o[i][0] = fmaf(pv, x0.x, o[i][0]);
            o[i][1] = fmaf(pv, x0.y, o[i][1]);
            o[i][2] = fmaf(pv, x0.z, o[i][2]);
            o[i][3] = fmaf(pv, x0.w, o[i][3]);
            o[i][4] = fmaf(pv, x1.x, o[i][4]);
            o[i][5] = fmaf(pv, x1.y, o[i][5]);
            o[i][6] = fmaf(pv, x1.z, o[i][6]);
            o[i][7] = fmaf(pv, x1.w, o[i][7]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < RT; ++i) {
        const int r = ry + 8 * i;
        if (!dok || r >= R) continue;
        float* dst;
        float sc = row_scale[i];
        if (PH == PH_L) {
          dst = p.ar + ((size_t)eh * M * b + (size_t)r * b + item) * D;
        } else if (rph && part == 0) {
          dst = p.al + ((size_t)eh * b * M + (size_t)r * M + item) * D;
          sc *= p.sm_scale;
        } else if (rph) {
          dst = p.y + ((size_t)eh * b * M + (size_t)r * M + item) * D;
        } else {
          const int n = r * b + item - p.pad_off;
          if (n < 0 || n >= p.N) continue;
          dst = p.out + ((int64_t)e * p.os[0] + (int64_t)h * p.os[1] + (int64_t)n * p.os[2]);
        }
        *reinterpret_cast<float4*>(dst + d0) =
            make_float4(o[i][0] * sc, o[i][1] * sc, o[i][2] * sc, o[i][3] * sc);
        *reinterpret_cast<float4*>(dst + d0 + 4) =
            make_float4(o[i][4] * sc, o[i][5] * sc, o[i][6] * sc, o[i][7] * sc);
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

template <int DP, int ROWS>
__global__ void __launch_bounds__(kThreads, 1) ma_small_f32_kernel(const Params p) {
  extern __shared__ __align__(16) uint8_t smem[];
  using TL = Tiles<DP, ROWS>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t crank, csize;  // this CTA's rank in its cluster, cluster size
  asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
  asm("mov.u32 %0, %%cluster_nctarank;" : "=r"(csize));
  const int eh = blockIdx.x / csize;  // clusters are consecutive blocks
  const int e = eh / p.H, h = eh - e * p.H;
  const int wg = crank * kWarps + warp, nw = csize * kWarps;  // warp within the cluster
  float* wsm = reinterpret_cast<float*>(smem + warp * TL::kBytes);
  uint32_t* vbits = reinterpret_cast<uint32_t*>(smem + kWarps * TL::kBytes);
  // zero the tiles once: the head-dim padding columns must read as 0
  for (int i = threadIdx.x; i < kWarps * TL::kBytes / 16; i += kThreads)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  // token validity of the padded sequence (pad positions and the mask row)
  const int Np = p.M * p.b;
  // (one lane per token, so the mask loads of a word are issued together)
  for (int w = warp; w < (TL::kMaxTokens + 31) / 32; w += kWarps) {
    const int pidx = w * 32 + lane;
    const uint32_t bits = __ballot_sync(0xffffffffu, pidx < Np && token_valid(p, e, pidx));
    if (lane == 0) vbits[w] = bits;
  }
  __syncthreads();
  for (int t = 0; t < p.T; ++t) {
    const bool final_ = t == p.T - 1;
    for (int m = wg; m < p.M; m += nw) {
      if (final_)
        run_item<PH_RF, DP, ROWS>(p, e, h, m, t == 0, wsm, vbits, lane);
      else
        run_item<PH_R, DP, ROWS>(p, e, h, m, t == 0, wsm, vbits, lane);
    }
    cluster_sync();
    for (int j = wg; j < p.b; j += nw) {
      if (final_)
        run_item<PH_O, DP, ROWS>(p, e, h, j, 0, wsm, vbits, lane);
      else
        run_item<PH_L, DP, ROWS>(p, e, h, j, 0, wsm, vbits, lane);
    }
    cluster_sync();
  }
}

// CTAs per head (1, 2, 4 or 8): waves of resident CTAs cost ceil(heads * C /
// slots) / C of a head's work each, plus ~10 % per doubling of C for cluster
// barriers and idle warps (a phase has only b or M items).  MA_SMALL_CLUSTER
// overrides.
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

template <int DP, int ROWS>
static cudaError_t launch(const Params& sp, cudaStream_t st) {
  using TL = Tiles<DP, ROWS>;
  const size_t smem = (size_t)kWarps * TL::kBytes + TL::kBitmapBytes;
  auto kfn = ma_small_f32_kernel<DP, ROWS>;
  cudaError_t err =
      cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  int dev = 0, sms = 0, per_sm = 0;
  err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (err != cudaSuccess) return err;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, kThreads, smem);
  if (err != cudaSuccess) return err;
  if (per_sm < 1) per_sm = 1;
  const int heads = sp.E * sp.H;
  const int csize = cluster_size(heads, sms * per_sm, sp.b > sp.M ? sp.b : sp.M);
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

}  // namespace smallf

static bool al16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

// fp32 shapes of the fused kernel: b, M <= 32, D = Dv a multiple of 8 up to
// 128, innermost strides 1 and 16-byte aligned rows (q / k / v read and out
// written in 16-byte pieces)
bool small_f32_supports(const ma_fwd_params* p, const Shape& s) {
  if (p->dtype != MA_DTYPE_F32) return false;
  if (s.b > 32 || s.M > 32) return false;
  if (s.D != s.Dv || s.D % 8 != 0 || s.D > 128) return false;
  if ((int64_t)s.E * s.H * 4 > 2147483647) return false;
  const int64_t* st[4] = {p->q_stride, p->k_stride, p->v_stride, p->o_stride};
  for (int t = 0; t < 4; ++t) {
    if (st[t][3] != 1) return false;
    for (int i = 0; i < 3; ++i)
      if ((st[t][i] * 4) % 16 != 0) return false;
  }
  const void* ptrs[4] = {p->q, p->k, p->v, p->out};
  for (int i = 0; i < 4; ++i)
    if (ptrs[i] && !al16(ptrs[i])) return false;
  return true;
}

cudaError_t run_small_f32(const ma_fwd_params* p, const Shape& s, const WsLayout& ws,
                          cudaStream_t st, int* nlaunch) {
  smallf::Params sp{};
  sp.q = static_cast<const float*>(p->q);
  sp.k = static_cast<const float*>(p->k);
  sp.v = static_cast<const float*>(p->v);
  sp.out = static_cast<float*>(p->out);
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
  sp.al = reinterpret_cast<float*>(w + ws.al);
  sp.y = reinterpret_cast<float*>(w + ws.y);
  sp.ar = reinterpret_cast<float*>(w + ws.ar);
  sp.cl = reinterpret_cast<float*>(w + ws.cl);
  sp.cr = reinterpret_cast<float*>(w + ws.cr);
  const int dp = (s.D + 15) / 16 * 16;
  const bool r16 = s.b <= 16 && s.M <= 16;
  cudaError_t err;
#define MA_SMALLF_CASE(DPV)                                                              \
  case DPV:                                                                              \
    err = r16 ? smallf::launch<DPV, 16>(sp, st) : smallf::launch<DPV, 32>(sp, st);       \
    break;
  switch (dp) {
    MA_SMALLF_CASE(16)
    MA_SMALLF_CASE(32)
    MA_SMALLF_CASE(48)
    MA_SMALLF_CASE(64)
    MA_SMALLF_CASE(80)
    MA_SMALLF_CASE(96)
    MA_SMALLF_CASE(112)
    MA_SMALLF_CASE(128)
    default: return cudaErrorInvalidValue;
  }
#undef MA_SMALLF_CASE
  if (err == cudaSuccess) *nlaunch += 1;
  return err;
}

}  // namespace ma
