// Generic MonarchAttention forward: one launch per algorithm phase, any
// block size / head dim / dtype / stride / mask / padding.
//
// Each phase is a set of independent "row-softmax problems".  A problem has
// R rows and C columns; a CTA takes RB rows of one problem of one (e, h):
//   1. logits  t[r][c] = f(A_r . B_c)          (SIMT dot products, fp32)
//   2. per-row softmax statistics / weights    (warp reductions)
//   3. outputs O_r = sum_c w[r][c] X_c          (tiled over output columns)
//
// Phase          problem (item)  rows r      cols c     reference
// PH_R / PH_RF   key block m     index j     key i      al_cl_ref / al_y_cl_ref
//                                                       (ma/ma_torch.py:10-23, 38-52)
// PH_LS          index j         q-block l   k-block k  softmax stats of ar_cr_ref
// PH_LA          index j         k-block k   q-block l  ar_cr_ref (ma_torch.py:26-35)
// PH_O           index j         q-block l   k-block k  z_ref (ma_torch.py:55-62)
//
// The L-step softmax runs over k for every l (dim -2 of the reference's
// [j][k][l] tensor), while its outputs ar/cr sum over l.  PH_LS computes the
// per-l statistics; PH_LA recomputes the logits with rows = k and applies
// them, so no R x C matrix ever leaves the SM.
//
// All arithmetic is fp32.  To track the reference bit-for-bit where it
// rounds, a matmul output is rounded to the input dtype before it is used
// (ma_torch.py:11, 27, 56), and every weight matrix is rounded to the input
// dtype before it becomes a matmul operand (ma_torch.py:21, 34, 50-51, 60).
#include <float.h>

#include "ma_common.cuh"

namespace ma {

enum Phase { PH_R = 0, PH_RF = 1, PH_LS = 2, PH_LA = 3, PH_O = 4 };

struct GenParams {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int64_t qs[4], ks[4], vs[4], os[4];
  const void* mask;
  int64_t ms[2];
  int mask_dtype;
  const float* qsc;  // per-(e,h) dequantisation scales (E4M3 only) or null
  const float* ksc;
  const float* vsc;
  int E, H, N, D, Dv, b, M, pad_off;
  float sm_scale;
  char* al;
  char* y;
  char* ar;
  float* cl;
  float* cr;
  float* lmax;
  float* lsum;
  int first;  // R-step reads q / cr = 1 instead of ar / cr
};

constexpr int GT = 128;  // threads per CTA (4 warps)
constexpr int RB = 16;   // rows per CTA (4 per warp)
constexpr int RW = RB / 4;
constexpr int CC = 32;   // columns per staged chunk
constexpr int OT = 128;  // output columns per tile

__host__ __device__ inline int odd_stride(int d) { return (d & 1) ? d : d + 1; }

size_t generic_smem_bytes(int D, int C) {
  const int dp = odd_stride(D);
  const int bs = dp > OT + 1 ? dp : OT + 1;
  return sizeof(float) * (size_t)(RB * dp + CC * bs + RB * C);
}

// validity of padded token index pidx of batch row e
__device__ __forceinline__ bool token_valid(const GenParams& p, int e, int pidx) {
  const int n = pidx - p.pad_off;
  if (n < 0 || n >= p.N) return false;
  if (p.mask == nullptr) return true;
  return mask_value(p.mask, p.mask_dtype, (int64_t)e * p.ms[0] + (int64_t)n * p.ms[1]);
}

// element d of the padded token pidx of a (E, H, N, X) input (0 in the padding)
template <typename TI>
__device__ __forceinline__ float load_tok(const void* base, const int64_t* st, const float* sc,
                                          const GenParams& p, int e, int h, int pidx, int d) {
  const int n = pidx - p.pad_off;
  if (n < 0 || n >= p.N) return 0.0f;
  const TI* t = reinterpret_cast<const TI*>(base);
  float x = to_f<TI>(t[(int64_t)e * st[0] + (int64_t)h * st[1] + (int64_t)n * st[2] +
                       (int64_t)d * st[3]]);
  if (sc != nullptr) x *= sc[e * p.H + h];
  return x;
}

// TI: q / k input type; TS: storage of al / ar and the rounding of the R / L
// weights; TVI: v input type; TY: storage of y, the output type, and the
// rounding of the y / output weights (the reference computes y = r.to(v.dtype)
// @ v and z = l.to(y.dtype) @ y, ma_torch.py:51, 60).
template <int PH, typename TI, typename TS, typename TVI, typename TY>
__global__ void __launch_bounds__(GT) generic_phase_kernel(const GenParams p) {
  extern __shared__ float smem[];
  const int D = p.D;
  const int dp = odd_stride(D);
  const int bstride = dp > OT + 1 ? dp : OT + 1;
  const bool rphase = (PH == PH_R || PH == PH_RF);
  const int R = rphase ? p.b : p.M;
  const int C = R;
  float* As = smem;                 // RB x dp     A rows
  float* Bs = As + RB * dp;         // CC x bstride B / X chunk
  float* Sw = Bs + CC * bstride;    // RB x C      logits -> weights

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int eh = blockIdx.z;
  const int e = eh / p.H, h = eh - e * p.H;
  const int item = blockIdx.y;
  const int r0 = blockIdx.x * RB;
  const int b = p.b, M = p.M;

  const TS* al_h = reinterpret_cast<const TS*>(p.al) + (size_t)eh * b * M * D;
  const TY* y_h = reinterpret_cast<const TY*>(p.y) + (size_t)eh * b * M * p.Dv;
  const TS* ar_h = reinterpret_cast<const TS*>(p.ar) + (size_t)eh * M * b * D;
  const float* cl_h = p.cl + (size_t)eh * b * M;
  const float* cr_h = p.cr + (size_t)eh * M * b;

  // ---- stage the RB A-rows ------------------------------------------------
  for (int idx = tid; idx < RB * D; idx += GT) {
    const int rr = idx / D, d = idx - rr * D, r = r0 + rr;
    float a = 0.0f;
    if (r < R) {
      if (rphase) {
        a = p.first ? load_tok<TI>(p.q, p.qs, p.qsc, p, e, h, item * b + r, d)
                    : to_f<TS>(ar_h[((size_t)item * b + r) * D + d]);
      } else if (PH == PH_LA) {
        a = to_f<TS>(al_h[((size_t)item * M + r) * D + d]);
      } else {  // PH_LS, PH_O: query rows l, token l*b + j
        a = load_tok<TI>(p.q, p.qs, p.qsc, p, e, h, r * b + item, d);
      }
    }
    As[rr * dp + d] = a;
  }

  // per-row scalars of this warp's rows
  float rowc[RW];
#pragma unroll
  for (int i = 0; i < RW; ++i) {
    const int r = r0 + warp * RW + i;
    rowc[i] = 0.0f;
    if (r < R) {
      if (rphase) rowc[i] = p.first ? 1.0f : cr_h[(size_t)item * b + r];
      if (PH == PH_LA) rowc[i] = cl_h[(size_t)item * M + r];
    }
  }

  // ---- 1. logits ----------------------------------------------------------
  for (int c0 = 0; c0 < C; c0 += CC) {
    __syncthreads();
    for (int idx = tid; idx < CC * D; idx += GT) {
      const int cc = idx / D, d = idx - cc * D, c = c0 + cc;
      float x = 0.0f;
      if (c < C) {
        if (rphase) x = load_tok<TI>(p.k, p.ks, p.ksc, p, e, h, item * b + c, d);
        else if (PH == PH_LA) x = load_tok<TI>(p.q, p.qs, p.qsc, p, e, h, c * b + item, d);
        else x = to_f<TS>(al_h[((size_t)item * M + c) * D + d]);
      }
      Bs[cc * bstride + d] = x;
    }
    __syncthreads();
    const int c = c0 + lane;
    float acc[RW];
#pragma unroll
    for (int i = 0; i < RW; ++i) acc[i] = 0.0f;
    const float* brow = Bs + lane * bstride;
    const float* arow = As + warp * RW * dp;
    for (int d = 0; d < D; ++d) {
      const float bv = brow[d];
#pragma unroll
      for (int i = 0; i < RW; ++i) acc[i] = fmaf(arow[i * dp + d], bv, acc[i]);
    }
    if (c < C) {
      bool cvalid = true;
      float cstat_m = 0.0f, cstat_s = 1.0f, ccl = 0.0f;
      if (rphase) {
        cvalid = token_valid(p, e, item * b + c);
      } else if (PH == PH_LA) {
        cvalid = token_valid(p, e, c * b + item);
        cstat_m = p.lmax[(size_t)eh * b * M + (size_t)item * M + c];
        cstat_s = p.lsum[(size_t)eh * b * M + (size_t)item * M + c];
      } else {
        ccl = cl_h[(size_t)item * M + c];
      }
#pragma unroll
      for (int i = 0; i < RW; ++i) {
        float t;
        const float s = rnd<TS>(acc[i]);  // matmul output in the input dtype
        if (rphase) {
          t = p.sm_scale * s;              // ma_torch.py:11
          t = t / (rowc[i] + kEps);        // :12
          if (!cvalid) t = -INFINITY;      // :13
        } else if (PH == PH_LA) {
          t = s - rowc[i];                 // l_hat - cl (row term), :27-28
          t = expf(t - cstat_m) / cstat_s; // softmax over k, :29
          if (!cvalid) t = 0.0f;           // query mask, :30
        } else {
          t = s - ccl;                     // :28 / :57
        }
        Sw[(warp * RW + i) * C + c] = t;
      }
    }
  }
  __syncthreads();

  // ---- 2. per-row statistics and weights (warp w owns rows w*RW..) -------
  for (int i = 0; i < RW; ++i) {
    const int rr = warp * RW + i, r = r0 + rr;
    float* srow = Sw + rr * C;
    if (PH == PH_LA) {
      float s = 0.0f;
      for (int c = lane; c < C; c += 32) s += srow[c];
#pragma unroll
      for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      for (int c = lane; c < C; c += 32) srow[c] = rnd<TS>(srow[c]);
      if (lane == 0 && r < R) p.cr[(size_t)eh * M * b + (size_t)r * b + item] = s;  // :32
      continue;
    }
    float mx = -INFINITY;
    for (int c = lane; c < C; c += 32) mx = fmaxf(mx, srow[c]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (rphase) mx = fmaxf(mx, kEps);  // clamp(max, min=eps), ma_torch.py:14-16
    float s = 0.0f;
    for (int c = lane; c < C; c += 32) {
      const float ex = expf(srow[c] - mx);
      srow[c] = ex;
      s += ex;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (PH == PH_LS) {
      if (lane == 0 && r < R) {
        p.lmax[(size_t)eh * b * M + (size_t)item * M + r] = mx;
        p.lsum[(size_t)eh * b * M + (size_t)item * M + r] = s;
      }
      continue;
    }
    if (rphase) {
      const float den = s + kEps;  // :17
      float cl = 0.0f;
      for (int c = lane; c < C; c += 32) {
        float w = srow[c] / den;
        w = fmaxf(w, kTiny);  // :18
        cl += w * logf(w);    // xlogy(r, r), :20
        srow[c] = w;          // rounded where it becomes a matmul operand
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) cl += __shfl_xor_sync(0xffffffffu, cl, o);
      if (lane == 0 && r < R) p.cl[(size_t)eh * b * M + (size_t)r * M + item] = cl;
    } else {  // PH_O: l.to(y.dtype), :60
      for (int c = lane; c < C; c += 32) srow[c] = rnd<TY>(srow[c] / s);
    }
  }
  if (PH == PH_LS) return;

  // ---- 3. outputs: O_r = sum_c w[r][c] X_c, tiled over output columns -----
  const int nseg = (PH == PH_RF) ? 2 : 1;
  for (int seg = 0; seg < nseg; ++seg) {
    const int X = (PH == PH_O || seg == 1) ? p.Dv : D;
    for (int x0 = 0; x0 < X; x0 += OT) {
      float acc[RW][4];
#pragma unroll
      for (int i = 0; i < RW; ++i)
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) acc[i][qd] = 0.0f;
      for (int c0 = 0; c0 < C; c0 += CC) {
        __syncthreads();
        for (int idx = tid; idx < CC * OT; idx += GT) {
          const int cc = idx / OT, d = idx - cc * OT, c = c0 + cc, xd = x0 + d;
          float x = 0.0f;
          if (c < C && xd < X) {
            if (rphase) {
              x = seg == 0 ? load_tok<TI>(p.k, p.ks, p.ksc, p, e, h, item * b + c, xd)
                           : load_tok<TVI>(p.v, p.vs, p.vsc, p, e, h, item * b + c, xd);
            } else if (PH == PH_LA) {
              x = load_tok<TI>(p.q, p.qs, p.qsc, p, e, h, c * b + item, xd);
            } else {
              x = to_f<TY>(y_h[((size_t)item * M + c) * p.Dv + xd]);
            }
          }
          Bs[cc * bstride + d] = x;
        }
        __syncthreads();
        const int ce = (C - c0) < CC ? (C - c0) : CC;
        for (int cc = 0; cc < ce; ++cc) {
          const float* xrow = Bs + cc * bstride;
          float xv[4];
#pragma unroll
          for (int qd = 0; qd < 4; ++qd) xv[qd] = xrow[lane + 32 * qd];
#pragma unroll
          for (int i = 0; i < RW; ++i) {
            float w = Sw[(warp * RW + i) * C + c0 + cc];
            // R-steps: r.to(k.dtype) for al, r.to(v.dtype) for y (:21, :51)
            if (rphase) w = seg == 0 ? rnd<TS>(w) : rnd<TY>(w);
#pragma unroll
            for (int qd = 0; qd < 4; ++qd) acc[i][qd] = fmaf(w, xv[qd], acc[i][qd]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < RW; ++i) {
        const int r = r0 + warp * RW + i;
        if (r >= R) continue;
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {
          const int xd = x0 + lane + 32 * qd;
          if (xd >= X) continue;
          const float a = acc[i][qd];
          if (rphase && seg == 0) {  // al = sm_scale * (r @ k), ma_torch.py:21
            TS* al = reinterpret_cast<TS*>(p.al) + (size_t)eh * b * M * D;
            al[((size_t)r * M + item) * D + xd] = from_f<TS>(p.sm_scale * rnd<TS>(a));
          } else if (rphase) {  // y = r @ v, :51
            TY* y = reinterpret_cast<TY*>(p.y) + (size_t)eh * b * M * p.Dv;
            y[((size_t)r * M + item) * p.Dv + xd] = from_f<TY>(a);
          } else if (PH == PH_LA) {  // ar = l @ q, :34
            TS* ar = reinterpret_cast<TS*>(p.ar) + (size_t)eh * M * b * D;
            ar[((size_t)r * b + item) * D + xd] = from_f<TS>(a);
          } else {  // z = l @ y, written at token l*b + j (unpadded), :60-62, :106-108
            const int n = r * b + item - p.pad_off;
            if (n >= 0 && n < p.N) {
              TY* o = reinterpret_cast<TY*>(p.out);
              o[(int64_t)e * p.os[0] + (int64_t)h * p.os[1] + (int64_t)n * p.os[2] +
                (int64_t)xd * p.os[3]] = from_f<TY>(a);
            }
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <int PH, typename TI, typename TS, typename TVI, typename TY>
static cudaError_t launch_phase(const GenParams& gp, cudaStream_t st) {
  const int R = (PH == PH_R || PH == PH_RF) ? gp.b : gp.M;
  const int items = (PH == PH_R || PH == PH_RF) ? gp.M : gp.b;
  const size_t smem = generic_smem_bytes(gp.D, R);
  auto kfn = generic_phase_kernel<PH, TI, TS, TVI, TY>;
  cudaError_t err = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
  if (err != cudaSuccess) return err;
  dim3 grid((R + RB - 1) / RB, items, gp.E * gp.H);
  kfn<<<grid, GT, smem, st>>>(gp);
  return cudaGetLastError();
}

template <typename TI, typename TS, typename TVI, typename TY>
static cudaError_t run_generic_t(GenParams gp, int T, cudaStream_t st, int* nlaunch) {
  cudaError_t err;
  for (int t = 0; t < T - 1; ++t) {
    gp.first = (t == 0);
    if ((err = launch_phase<PH_R, TI, TS, TVI, TY>(gp, st)) != cudaSuccess) return err;
    if ((err = launch_phase<PH_LS, TI, TS, TVI, TY>(gp, st)) != cudaSuccess) return err;
    if ((err = launch_phase<PH_LA, TI, TS, TVI, TY>(gp, st)) != cudaSuccess) return err;
    *nlaunch += 3;
  }
  gp.first = (T == 1);
  if ((err = launch_phase<PH_RF, TI, TS, TVI, TY>(gp, st)) != cudaSuccess) return err;
  if ((err = launch_phase<PH_O, TI, TS, TVI, TY>(gp, st)) != cudaSuccess) return err;
  *nlaunch += 2;
  return cudaSuccess;
}

// The forward's R and L phases with every step's intermediates kept (the
// backward pass recomputes the forward this way): R-step t reads ar[t] /
// cr[t] (t >= 1; step 0 reads q and cr = 1) and writes al[t] / cl[t] (and y
// at t = T-1); L-step t writes ar[t+1] / cr[t+1].  No output phase.
template <typename TI, typename TS>
static cudaError_t run_generic_saved_t(GenParams gp, int T, char* const* al, float* const* cl,
                                       char* const* ar, float* const* cr, cudaStream_t st,
                                       int* nlaunch) {
  cudaError_t err;
  for (int t = 0; t < T; ++t) {
    gp.first = (t == 0);
    gp.al = al[t];
    gp.cl = cl[t];
    gp.ar = t > 0 ? ar[t] : ar[1 < T ? 1 : 0];  // unused at t = 0
    gp.cr = t > 0 ? cr[t] : cr[1 < T ? 1 : 0];
    if (t == T - 1) {
      if ((err = launch_phase<PH_RF, TI, TS, TS, TS>(gp, st)) != cudaSuccess) return err;
      *nlaunch += 1;
      break;
    }
    if ((err = launch_phase<PH_R, TI, TS, TS, TS>(gp, st)) != cudaSuccess) return err;
    gp.ar = ar[t + 1];
    gp.cr = cr[t + 1];
    if ((err = launch_phase<PH_LS, TI, TS, TS, TS>(gp, st)) != cudaSuccess) return err;
    if ((err = launch_phase<PH_LA, TI, TS, TS, TS>(gp, st)) != cudaSuccess) return err;
    *nlaunch += 3;
  }
  return cudaSuccess;
}

cudaError_t run_generic_saved(const ma_fwd_params* p, const Shape& s, char* const* al,
                              float* const* cl, char* const* ar, float* const* cr, char* y,
                              float* lmax, float* lsum, cudaStream_t st, int* nlaunch) {
  GenParams gp{};
  gp.q = p->q; gp.k = p->k; gp.v = p->v; gp.out = nullptr;
  for (int i = 0; i < 4; ++i) {
    gp.qs[i] = p->q_stride[i]; gp.ks[i] = p->k_stride[i];
    gp.vs[i] = p->v_stride[i]; gp.os[i] = 0;
  }
  gp.mask = p->mask_dtype == MA_MASK_NONE ? nullptr : p->mask;
  gp.ms[0] = p->mask_stride[0]; gp.ms[1] = p->mask_stride[1];
  gp.mask_dtype = p->mask_dtype;
  gp.E = s.E; gp.H = s.H; gp.N = s.N; gp.D = s.D; gp.Dv = s.Dv; gp.b = s.b; gp.M = s.M;
  gp.pad_off = s.pad_off; gp.sm_scale = s.sm_scale;
  gp.y = y;
  gp.lmax = lmax;
  gp.lsum = lsum;
  switch (p->dtype) {
    case MA_DTYPE_F32: return run_generic_saved_t<float, float>(gp, s.T, al, cl, ar, cr, st, nlaunch);
    case MA_DTYPE_F16:
      return run_generic_saved_t<__half, __half>(gp, s.T, al, cl, ar, cr, st, nlaunch);
    case MA_DTYPE_BF16:
      return run_generic_saved_t<__nv_bfloat16, __nv_bfloat16>(gp, s.T, al, cl, ar, cr, st,
                                                               nlaunch);
    default: return cudaErrorInvalidValue;
  }
}

// Limits of the generic path (checked by the C ABI before launching).
bool generic_supports(const Shape& s) {
  if (s.D > 1024) return false;
  const int C = s.b > s.M ? s.b : s.M;
  if (generic_smem_bytes(s.D, C) > 200 * 1024) return false;
  if ((int64_t)s.E * s.H > 65535 || s.M > 65535 || s.b > 65535) return false;
  return true;
}

cudaError_t run_generic(const ma_fwd_params* p, const Shape& s, const WsLayout& ws,
                        cudaStream_t st, int* nlaunch) {
  GenParams gp{};
  gp.q = p->q; gp.k = p->k; gp.v = p->v; gp.out = p->out;
  for (int i = 0; i < 4; ++i) {
    gp.qs[i] = p->q_stride[i]; gp.ks[i] = p->k_stride[i];
    gp.vs[i] = p->v_stride[i]; gp.os[i] = p->o_stride[i];
  }
  gp.mask = p->mask_dtype == MA_MASK_NONE ? nullptr : p->mask;
  gp.ms[0] = p->mask_stride[0]; gp.ms[1] = p->mask_stride[1];
  gp.mask_dtype = p->mask_dtype;
  const bool fp8 = p->dtype == MA_DTYPE_E4M3;
  gp.qsc = fp8 ? p->q_scale : nullptr;
  gp.ksc = fp8 ? p->k_scale : nullptr;
  gp.vsc = fp8 ? p->v_scale : nullptr;
  gp.E = s.E; gp.H = s.H; gp.N = s.N; gp.D = s.D; gp.Dv = s.Dv; gp.b = s.b; gp.M = s.M;
  gp.pad_off = s.pad_off; gp.sm_scale = s.sm_scale;
  char* w = reinterpret_cast<char*>(p->workspace);
  gp.al = w + ws.al; gp.y = w + ws.y; gp.ar = w + ws.ar;
  gp.cl = reinterpret_cast<float*>(w + ws.cl);
  gp.cr = reinterpret_cast<float*>(w + ws.cr);
  gp.lmax = reinterpret_cast<float*>(w + ws.lmax);
  gp.lsum = reinterpret_cast<float*>(w + ws.lsum);
  if (p->v_f32) {  // fp32 values with 16-bit q / k (get_matrix)
    if (p->dtype == MA_DTYPE_F16)
      return run_generic_t<__half, __half, float, float>(gp, s.T, st, nlaunch);
    if (p->dtype == MA_DTYPE_BF16)
      return run_generic_t<__nv_bfloat16, __nv_bfloat16, float, float>(gp, s.T, st, nlaunch);
    return cudaErrorInvalidValue;
  }
  switch (p->dtype) {
    case MA_DTYPE_F32: return run_generic_t<float, float, float, float>(gp, s.T, st, nlaunch);
    case MA_DTYPE_F16: return run_generic_t<__half, __half, __half, __half>(gp, s.T, st, nlaunch);
    case MA_DTYPE_BF16:
      return run_generic_t<__nv_bfloat16, __nv_bfloat16, __nv_bfloat16, __nv_bfloat16>(
          gp, s.T, st, nlaunch);
    case MA_DTYPE_E4M3:
      return run_generic_t<__nv_fp8_e4m3, __nv_bfloat16, __nv_fp8_e4m3, __nv_bfloat16>(
          gp, s.T, st, nlaunch);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ma
