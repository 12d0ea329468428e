// Backward pass of the MonarchAttention forward: d<out, dout>/d(q, k, v),
// the gradients the reference obtains with PyTorch autograd over
// ma/ma_torch.py:65-108 (its training path, bart/run_summarization.py).
//
// The forward is recomputed by the generic phase kernels with every step's
// intermediates kept (al, cl, ar, cr per step, y; ma_generic.cu), then the
// phases are differentiated in reverse order, one launch per phase:
//
//   output (z_ref, ma_torch.py:55-62), item j, rows l, columns k:
//     P = softmax_k(q_l . al_k - cl_k);  z_l = sum_k P y_k
//     dy_k += sum_l P dz_l;  dS = P (dP - sum_k P dP), dP = dz_l . y_k
//     dq_l += sum_k dS al_k;  dal_k += sum_l dS q_l;  dcl_k -= sum_l dS
//   R-step (al_cl_ref / al_y_cl_ref, :10-23, :38-52), item m, rows j, keys i:
//     t = sm_scale ar_j . k_i / (cr_j + eps) (masked -inf); r = softmax with
//     the clamps; al_j = sm_scale sum_i r k_i; y_j = sum_i r v_i; cl_j =
//     sum_i r log r
//     dr = sm_scale dal_j . k_i + dy_j . v_i + dcl_j (log r + 1)
//     dt = r (dr - sum_i r dr);  dS = dt sm_scale / (cr_j + eps)
//     dar_j = sum_i dS k_i (step 0: dq);  dcr_j = -sum_i dt t / (cr_j + eps)
//     dk_i += sum_j dS ar_j + sm_scale r dal_j;  dv_i += sum_j r dy_j
//   L-step (ar_cr_ref, :26-35), item j, rows l, columns k:
//     Ps = softmax_k(al_k . q_l - cl_k);  P = Ps * qmask_l
//     ar_k = sum_l P q_l;  cr_k = sum_l P
//     dP = dar_k . q_l + dcr_k;  dS = Ps (qmask_l dP - sum_k Ps qmask_l dP)
//     dq_l += sum_k P dar_k + sum_k dS al_k;  dal_k += sum_l dS q_l;
//     dcl_k -= sum_l dS
//
// A CTA takes 16 rows of one item (like the generic forward kernels):
// logits and gradient dot products are SIMT fp32 over column chunks staged
// in shared memory, the row softmax and its gradient are warp reductions,
// row gradients are written directly (the rows of a launch are disjoint) and
// column gradients are added with fp32 atomics.  All gradient arithmetic is
// fp32; the recomputed forward rounds where the reference rounds.  The
// gradients of the max shift, of the eps terms and of r at the FLT_MIN clamp
// are zero or O(1e-12) relative and are left out.
#include <float.h>
#include <math.h>
#include <string.h>

#include <string>

#include "ma_common.cuh"

namespace ma {

// ma_generic.cu
cudaError_t run_generic_saved(const ma_fwd_params* p, const Shape& s, char* const* al,
                              float* const* cl, char* const* ar, float* const* cr, char* y,
                              float* lmax, float* lsum, cudaStream_t st, int* nlaunch);

namespace bwd {

constexpr int BT = 128;  // threads per CTA (4 warps)
constexpr int RB = 16;   // rows per CTA
constexpr int RW = RB / 4;
constexpr int CC = 32;   // columns per staged chunk
constexpr int kMaxDim = 256;  // head dims (D, Dv) and row lengths (b, M) handled

enum Kind { K_O = 0, K_R = 1, K_RF = 2, K_L = 3 };

struct Params {
  const void* q;
  const void* k;
  const void* v;
  int64_t qs[4], ks[4], vs[4];
  const void* dout;
  int64_t gs[4];
  const void* mask;
  int64_t ms[2];
  int mask_dtype;
  int E, H, N, Np, D, Dv, b, M, pad_off, first;
  float sm_scale;
  // forward intermediates of the step being differentiated (storage dtype)
  const void* al;   // [eh][b][M][D]
  const float* cl;  // [eh][b][M]
  const void* ar;   // [eh][M][b][D]
  const float* cr;  // [eh][M][b]
  const void* y;    // [eh][b][M][Dv]
  // fp32 gradients
  float* dal;  // [eh][b][M][D]
  float* dcl;  // [eh][b][M]
  float* dy;   // [eh][b][M][Dv]
  float* dar;  // [eh][M][b][D]
  float* dcr;  // [eh][M][b]
  float* dq;   // [eh][Np][D]  (padded token index)
  float* dk;   // [eh][Np][D]
  float* dv;   // [eh][Np][Dv]
};

__host__ __device__ inline int odd_stride(int d) { return (d & 1) ? d : d + 1; }

__device__ __forceinline__ bool token_valid(const Params& p, int e, int pidx) {
  const int n = pidx - p.pad_off;
  if (n < 0 || n >= p.N) return false;
  if (p.mask == nullptr) return true;
  return mask_value(p.mask, p.mask_dtype, (int64_t)e * p.ms[0] + (int64_t)n * p.ms[1]);
}

// element d of padded token pidx of an (E, H, N, X) tensor (0 in the padding)
template <typename T>
__device__ __forceinline__ float load_tok(const void* base, const int64_t* st, const Params& p,
                                          int e, int h, int pidx, int d) {
  const int n = pidx - p.pad_off;
  if (n < 0 || n >= p.N) return 0.0f;
  return to_f<T>(reinterpret_cast<const T*>(base)[(int64_t)e * st[0] + (int64_t)h * st[1] +
                                                  (int64_t)n * st[2] + (int64_t)d * st[3]]);
}

// dynamic shared memory of a CTA (floats): A rows, row gradients G and G2,
// a column chunk of B and of X, P and dS of the CTA's rows, row scalars
struct Smem {
  int dp, gp, g2p, xp;  // row strides (odd)
  int offA, offG, offG2, offB, offX, offP, offS, offRow, total;
};
__host__ __device__ inline Smem smem_layout(int kind, int D, int Dv, int C) {
  Smem m{};
  const int Dx = kind == K_L ? D : Dv;  // X columns: y (O), v (RF), dar (L)
  const int Dg = kind == K_O ? Dv : D;  // G rows: dz (O), dal (R, RF)
  m.dp = odd_stride(D);
  m.gp = odd_stride(Dg);
  m.g2p = odd_stride(Dv);
  m.xp = odd_stride(Dx);
  int off = 0;
  m.offA = off; off += RB * m.dp;
  m.offG = off; off += (kind == K_L ? 0 : RB * m.gp);
  m.offG2 = off; off += (kind == K_RF ? RB * m.g2p : 0);
  m.offB = off; off += CC * m.dp;
  m.offX = off; off += (kind == K_R ? 0 : CC * m.xp);
  m.offP = off; off += RB * C;
  m.offS = off; off += RB * C;
  m.offRow = off; off += RB * 4;
  m.total = off;
  return m;
}

template <int KIND, typename TI, typename TS>
__global__ void __launch_bounds__(BT) bwd_kernel(const Params p) {
  extern __shared__ float sm[];
  constexpr bool rk = KIND == K_R || KIND == K_RF;
  const int b = p.b, M = p.M, D = p.D, Dv = p.Dv;
  const int R = rk ? b : M, C = R;
  const Smem L = smem_layout(KIND, D, Dv, C);
  float* As = sm + L.offA;
  float* Gs = sm + L.offG;
  float* G2s = sm + L.offG2;
  float* Bs = sm + L.offB;
  float* Xs = sm + L.offX;
  float* Ps = sm + L.offP;
  float* Ss = sm + L.offS;
  float* rowv = sm + L.offRow;  // per row: [0] cr (R) / query mask (L), [1] dcl (R), [2] dcr out
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int eh = blockIdx.z, e = eh / p.H, h = eh - e * p.H;
  const int item = blockIdx.y, r0 = blockIdx.x * RB;
  const int Dg = KIND == K_O ? Dv : D;
  const TS* al_h = reinterpret_cast<const TS*>(p.al) + (size_t)eh * b * M * D;
  const TS* ar_h = reinterpret_cast<const TS*>(p.ar) + (size_t)eh * M * b * D;
  const TS* y_h = reinterpret_cast<const TS*>(p.y) + (size_t)eh * b * M * Dv;
  const float* cl_h = p.cl + (size_t)eh * b * M;
  const float* cr_h = p.cr + (size_t)eh * M * b;

  // ---- stage the CTA's rows: A (q / ar), G (dz / dal), G2 (dy), scalars ----
  for (int idx = tid; idx < RB * D; idx += BT) {
    const int rr = idx / D, d = idx - rr * D, r = r0 + rr;
    float a = 0.0f;
    if (r < R) {
      if (rk)
        a = p.first ? load_tok<TI>(p.q, p.qs, p, e, h, item * b + r, d)
                    : to_f<TS>(ar_h[((size_t)item * b + r) * D + d]);
      else
        a = load_tok<TI>(p.q, p.qs, p, e, h, r * b + item, d);
    }
    As[rr * L.dp + d] = a;
  }
  if (KIND != K_L) {
    for (int idx = tid; idx < RB * Dg; idx += BT) {
      const int rr = idx / Dg, d = idx - rr * Dg, r = r0 + rr;
      float g = 0.0f;
      if (r < R) {
        if (KIND == K_O)
          g = load_tok<TI>(p.dout, p.gs, p, e, h, r * b + item, d);
        else
          g = p.dal[((size_t)eh * b * M + (size_t)r * M + item) * D + d];
      }
      Gs[rr * L.gp + d] = g;
    }
  }
  if (KIND == K_RF) {
    for (int idx = tid; idx < RB * Dv; idx += BT) {
      const int rr = idx / Dv, d = idx - rr * Dv, r = r0 + rr;
      G2s[rr * L.g2p + d] =
          r < R ? p.dy[((size_t)eh * b * M + (size_t)r * M + item) * Dv + d] : 0.0f;
    }
  }
  if (tid < RB) {
    const int r = r0 + tid;
    float v0 = 0.0f, v1 = 0.0f;
    if (r < R) {
      if (rk) {
        v0 = p.first ? 1.0f : cr_h[(size_t)item * b + r];
        v1 = p.dcl[(size_t)eh * b * M + (size_t)r * M + item];
      } else if (KIND == K_L) {
        v0 = token_valid(p, e, r * b + item) ? 1.0f : 0.0f;
      }
    }
    rowv[tid * 4 + 0] = v0;
    rowv[tid * 4 + 1] = v1;
    rowv[tid * 4 + 2] = 0.0f;
  }

  // column chunk staging: B (k / al_j), X (y_j / v / dar_j)
  auto stage_cols = [&](int c0, bool with_x) {
    for (int idx = tid; idx < CC * D; idx += BT) {
      const int cc = idx / D, d = idx - cc * D, c = c0 + cc;
      float x = 0.0f;
      if (c < C)
        x = rk ? load_tok<TI>(p.k, p.ks, p, e, h, item * b + c, d)
               : to_f<TS>(al_h[((size_t)item * M + c) * D + d]);
      Bs[cc * L.dp + d] = x;
    }
    if (with_x) {
      const int Dx = KIND == K_L ? D : Dv;
      for (int idx = tid; idx < CC * Dx; idx += BT) {
        const int cc = idx / Dx, d = idx - cc * Dx, c = c0 + cc;
        float x = 0.0f;
        if (c < C) {
          if (KIND == K_O) x = to_f<TS>(y_h[((size_t)item * M + c) * Dv + d]);
          else if (KIND == K_RF) x = load_tok<TI>(p.v, p.vs, p, e, h, item * b + c, d);
          else x = p.dar[((size_t)eh * M * b + (size_t)c * b + item) * D + d];
        }
        Xs[cc * L.xp + d] = x;
      }
    }
  };

  // ---- 1. logits S (-> Ps) and the gradient dot products (-> Ss) ----
  for (int c0 = 0; c0 < C; c0 += CC) {
    __syncthreads();
    stage_cols(c0, KIND != K_R);
    __syncthreads();
    const int c = c0 + lane;
    float as[RW], ag[RW], ag2[RW];
#pragma unroll
    for (int i = 0; i < RW; ++i) as[i] = ag[i] = ag2[i] = 0.0f;
    const float* brow = Bs + lane * L.dp;
    const float* xrow = Xs + lane * L.xp;
    for (int d = 0; d < D; ++d) {
      const float bv = brow[d];
#pragma unroll
      for (int i = 0; i < RW; ++i) {
        as[i] = fmaf(As[(warp * RW + i) * L.dp + d], bv, as[i]);
        if (rk) ag[i] = fmaf(Gs[(warp * RW + i) * L.gp + d], bv, ag[i]);     // dal . k
        if (KIND == K_L) ag[i] = fmaf(As[(warp * RW + i) * L.dp + d], xrow[d], ag[i]);  // dar . q
      }
    }
    if (KIND == K_O || KIND == K_RF) {
      for (int d = 0; d < Dv; ++d) {
        const float xv = xrow[d];
#pragma unroll
        for (int i = 0; i < RW; ++i) {
          if (KIND == K_O) ag[i] = fmaf(Gs[(warp * RW + i) * L.gp + d], xv, ag[i]);   // dz . y
          else ag2[i] = fmaf(G2s[(warp * RW + i) * L.g2p + d], xv, ag2[i]);           // dy . v
        }
      }
    }
    if (c < C) {
      const float dcr_c =
          KIND == K_L ? p.dcr[(size_t)eh * M * b + (size_t)c * b + item] : 0.0f;
#pragma unroll
      for (int i = 0; i < RW; ++i) {
        const int rr = warp * RW + i;
        Ps[rr * C + c] = as[i];
        float g;
        if (KIND == K_O) g = ag[i];
        else if (KIND == K_R) g = p.sm_scale * ag[i];
        else if (KIND == K_RF) g = p.sm_scale * ag[i] + ag2[i];
        else g = ag[i] + dcr_c;
        Ss[rr * C + c] = g;
      }
    }
  }
  __syncthreads();

  // ---- 2. per row: the softmax recomputed, dS = the logit gradient ----
  // Ps[r][c] <- P as the forward's matmuls used it (rounded to the storage
  // dtype; R: r clamped at FLT_MIN; L: times the query mask); Ss[r][c] <- dS.
  for (int i = 0; i < RW; ++i) {
    const int rr = warp * RW + i, r = r0 + rr;
    float* prow = Ps + rr * C;
    float* srow = Ss + rr * C;
    if (r >= R) {
      for (int c = lane; c < C; c += 32) prow[c] = srow[c] = 0.0f;
      continue;
    }
    if (rk) {
      const float crv = rowv[rr * 4 + 0], dclr = rowv[rr * 4 + 1];
      const float cs = p.sm_scale / (crv + kEps);
      // t = sm_scale * S / (cr + eps), -inf for invalid keys (ma_torch.py:11-13)
      auto tval = [&](int c) {
        return token_valid(p, e, item * b + c) ? cs * rnd<TS>(prow[c]) : -INFINITY;
      };
      float mx = -INFINITY;
      for (int c = lane; c < C; c += 32) mx = fmaxf(mx, tval(c));
#pragma unroll
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float sh = fmaxf(mx, kEps);  // :14-16
      float s = 0.0f;
      for (int c = lane; c < C; c += 32) s += expf(tval(c) - sh);
#pragma unroll
      for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      const float den = s + kEps;  // :17
      // dr (gradient of the clamped r the forward used: al, y and cl), then
      // sum_i r dr for the softmax gradient
      float dot = 0.0f;
      for (int c = lane; c < C; c += 32) {
        const float t = tval(c);
        const float rv = expf(t - sh) / den;
        const float rc = fmaxf(rv, kTiny);  // :18
        const float dr = rv >= kTiny ? srow[c] + dclr * (logf(rc) + 1.0f) : 0.0f;  // :20-21, :51
        srow[c] = dr;
        dot = fmaf(rv, dr, dot);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      float dcr = 0.0f;
      for (int c = lane; c < C; c += 32) {
        const float t = tval(c);
        const float rv = expf(t - sh) / den;
        const float dt = rv * (srow[c] - dot);
        if (t != -INFINITY) dcr = fmaf(dt, t, dcr);
        srow[c] = dt * cs;
        prow[c] = rnd<TS>(fmaxf(rv, kTiny));
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) dcr += __shfl_xor_sync(0xffffffffu, dcr, o);
      if (lane == 0) rowv[rr * 4 + 2] = -dcr / (crv + kEps);  // d t / d cr = -t / (cr + eps)
    } else {
      // x = S - cl[k] (output: :56-57; L: :27-28), softmax over the columns k
      auto xval = [&](int c) { return rnd<TS>(prow[c]) - cl_h[(size_t)item * M + c]; };
      float mx = -INFINITY;
      for (int c = lane; c < C; c += 32) mx = fmaxf(mx, xval(c));
#pragma unroll
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float s = 0.0f;
      for (int c = lane; c < C; c += 32) s += expf(xval(c) - mx);
#pragma unroll
      for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      const float qm = KIND == K_L ? rowv[rr * 4 + 0] : 1.0f;  // L *= qmask (:30)
      float dot = 0.0f;
      for (int c = lane; c < C; c += 32) {
        const float pv = expf(xval(c) - mx) / s;
        const float gd = srow[c] * qm;
        srow[c] = gd;
        dot = fmaf(pv, gd, dot);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      for (int c = lane; c < C; c += 32) {
        const float pv = expf(xval(c) - mx) / s;
        srow[c] = pv * (srow[c] - dot);
        prow[c] = rnd<TS>(pv * qm);
      }
    }
  }

  // ---- 3. row gradients (dS B, L: + P X) and column gradients, per chunk ----
  constexpr int NQ = kMaxDim / 32;
  float acc[RW][NQ];
#pragma unroll
  for (int i = 0; i < RW; ++i)
#pragma unroll
    for (int qd = 0; qd < NQ; ++qd) acc[i][qd] = 0.0f;
  for (int c0 = 0; c0 < C; c0 += CC) {
    __syncthreads();
    stage_cols(c0, KIND == K_L);
    __syncthreads();
    const int ce = (C - c0) < CC ? (C - c0) : CC;
    for (int cc = 0; cc < ce; ++cc) {
      const float* brow = Bs + cc * L.dp;
      const float* xrow = Xs + cc * L.xp;
#pragma unroll
      for (int i = 0; i < RW; ++i) {
        const int rr = warp * RW + i;
        const float w = Ss[rr * C + c0 + cc];
        const float pw = KIND == K_L ? Ps[rr * C + c0 + cc] : 0.0f;
#pragma unroll
        for (int qd = 0; qd < NQ; ++qd) {
          const int d = lane + 32 * qd;
          if (d < D) {
            float a = fmaf(w, brow[d], acc[i][qd]);
            if (KIND == K_L) a = fmaf(pw, xrow[d], a);
            acc[i][qd] = a;
          }
        }
      }
    }
    // column gradients of this chunk: dB_c = sum_r dS A_r (R: + sm_scale P dal_r)
    for (int idx = tid; idx < ce * D; idx += BT) {
      const int cc = idx / D, d = idx - cc * D, c = c0 + cc;
      float sb = 0.0f;
#pragma unroll 4
      for (int rr = 0; rr < RB; ++rr) {
        sb = fmaf(Ss[rr * C + c], As[rr * L.dp + d], sb);
        if (rk) sb = fmaf(p.sm_scale * Ps[rr * C + c], Gs[rr * L.gp + d], sb);
      }
      if (rk)
        atomicAdd(p.dk + ((size_t)eh * p.Np + (size_t)item * b + c) * D + d, sb);
      else
        atomicAdd(p.dal + ((size_t)eh * b * M + (size_t)item * M + c) * D + d, sb);
    }
    // dy_k = sum_l P dz_l (output), dv_i = sum_j r dy_j (final R-step)
    if (KIND == K_O || KIND == K_RF) {
      for (int idx = tid; idx < ce * Dv; idx += BT) {
        const int cc = idx / Dv, d = idx - cc * Dv, c = c0 + cc;
        float sx = 0.0f;
#pragma unroll 4
        for (int rr = 0; rr < RB; ++rr)
          sx = fmaf(Ps[rr * C + c], KIND == K_O ? Gs[rr * L.gp + d] : G2s[rr * L.g2p + d], sx);
        if (KIND == K_O)
          atomicAdd(p.dy + ((size_t)eh * b * M + (size_t)item * M + c) * Dv + d, sx);
        else
          atomicAdd(p.dv + ((size_t)eh * p.Np + (size_t)item * b + c) * Dv + d, sx);
      }
    }
    // dcl_k = -sum_l dS (output, L)
    if (!rk) {
      for (int cc = tid; cc < ce; cc += BT) {
        float sc = 0.0f;
        for (int rr = 0; rr < RB; ++rr) sc += Ss[rr * C + c0 + cc];
        atomicAdd(p.dcl + (size_t)eh * b * M + (size_t)item * M + c0 + cc, -sc);
      }
    }
  }
  // row gradients: dq rows (output, L, R-step 0) or dar / dcr (later R-steps)
#pragma unroll
  for (int i = 0; i < RW; ++i) {
    const int rr = warp * RW + i, r = r0 + rr;
    if (r >= R) continue;
    float* dst;
    bool add = true;
    if (!rk) {
      dst = p.dq + ((size_t)eh * p.Np + (size_t)r * b + item) * D;
    } else if (p.first) {
      dst = p.dq + ((size_t)eh * p.Np + (size_t)item * b + r) * D;
    } else {
      dst = p.dar + ((size_t)eh * M * b + (size_t)item * b + r) * D;
      add = false;
      if (lane == 0) p.dcr[(size_t)eh * M * b + (size_t)item * b + r] = rowv[rr * 4 + 2];
    }
#pragma unroll
    for (int qd = 0; qd < NQ; ++qd) {
      const int d = lane + 32 * qd;
      if (d < D) dst[d] = add ? dst[d] + acc[i][qd] : acc[i][qd];
    }
  }
}

// fp32 gradient accumulator (padded token index) -> caller tensor (E, H, N, X)
template <typename T>
__global__ void cast_grad_kernel(const float* acc, int H, int N, int Np, int X, int pad_off,
                                 int64_t total, void* out, int64_t s0, int64_t s1, int64_t s2,
                                 int64_t s3) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % X);
    const int64_t rest = i / X;
    const int n = (int)(rest % N);
    const int64_t eh = rest / N;
    const int e = (int)(eh / H), h = (int)(eh % H);
    reinterpret_cast<T*>(out)[(int64_t)e * s0 + (int64_t)h * s1 + (int64_t)n * s2 +
                              (int64_t)d * s3] =
        from_f<T>(acc[((size_t)eh * Np + n + pad_off) * X + d]);
  }
}

template <int KIND, typename TI, typename TS>
static cudaError_t launch_kind(const Params& bp, cudaStream_t st) {
  const bool rk = KIND == K_R || KIND == K_RF;
  const int R = rk ? bp.b : bp.M, items = rk ? bp.M : bp.b;
  const Smem L = smem_layout(KIND, bp.D, bp.Dv, R);
  const size_t smem = (size_t)L.total * sizeof(float);
  auto kfn = bwd_kernel<KIND, TI, TS>;
  cudaError_t err =
      cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  dim3 grid((R + RB - 1) / RB, items, bp.E * bp.H);
  kfn<<<grid, BT, smem, st>>>(bp);
  return cudaGetLastError();
}

// workspace: the recomputed forward's per-step intermediates, then the fp32
// gradients
struct Layout {
  size_t al[64], cl[64], ar[64], cr[64];
  size_t y, lmax, lsum, dal, dcl, dy, dar, dcr, dq, dk, dv, total;
};
static Layout layout(const Shape& s, int sb) {
  Layout w{};
  const size_t heads = (size_t)s.E * s.H, bm = (size_t)s.b * s.M;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes, 256);
    return at;
  };
  for (int t = 0; t < s.T; ++t) {
    w.al[t] = take(heads * bm * s.D * sb);
    w.cl[t] = take(heads * bm * 4);
    w.ar[t] = t > 0 ? take(heads * bm * s.D * sb) : 0;
    w.cr[t] = t > 0 ? take(heads * bm * 4) : 0;
  }
  w.y = take(heads * bm * s.Dv * sb);
  w.lmax = take(heads * bm * 4);
  w.lsum = take(heads * bm * 4);
  w.dal = take(heads * bm * s.D * 4);
  w.dcl = take(heads * bm * 4);
  w.dy = take(heads * bm * s.Dv * 4);
  w.dar = take(heads * bm * s.D * 4);
  w.dcr = take(heads * bm * 4);
  w.dq = take(heads * s.Np * s.D * 4);
  w.dk = take(heads * s.Np * s.D * 4);
  w.dv = take(heads * s.Np * s.Dv * 4);
  w.total = off;
  return w;
}

template <typename T>
static cudaError_t run_t(const ma_bwd_params* p, const Shape& s, const Layout& w,
                         cudaStream_t st, int* nlaunch) {
  char* base = reinterpret_cast<char*>(p->workspace);
  const ma_fwd_params* f = &p->fwd;
  // 1. forward recomputation, every step kept
  char* al[64];
  float* cl[64];
  char* ar[64];
  float* cr[64];
  for (int t = 0; t < s.T; ++t) {
    al[t] = base + w.al[t];
    cl[t] = reinterpret_cast<float*>(base + w.cl[t]);
    ar[t] = t > 0 ? base + w.ar[t] : nullptr;
    cr[t] = t > 0 ? reinterpret_cast<float*>(base + w.cr[t]) : nullptr;
  }
  if (s.T == 1) {  // run_generic_saved reads ar[0] / cr[0] only as unused placeholders
    ar[0] = base + w.dar;
    cr[0] = reinterpret_cast<float*>(base + w.dcr);
  }
  cudaError_t err = run_generic_saved(f, s, al, cl, ar, cr, base + w.y,
                                      reinterpret_cast<float*>(base + w.lmax),
                                      reinterpret_cast<float*>(base + w.lsum), st, nlaunch);
  if (err != cudaSuccess) return err;

  Params bp{};
  bp.q = f->q; bp.k = f->k; bp.v = f->v;
  for (int i = 0; i < 4; ++i) {
    bp.qs[i] = f->q_stride[i]; bp.ks[i] = f->k_stride[i]; bp.vs[i] = f->v_stride[i];
    bp.gs[i] = p->dout_stride[i];
  }
  bp.dout = p->dout;
  bp.mask = f->mask_dtype == MA_MASK_NONE ? nullptr : f->mask;
  bp.ms[0] = f->mask_stride[0]; bp.ms[1] = f->mask_stride[1];
  bp.mask_dtype = f->mask_dtype;
  bp.E = s.E; bp.H = s.H; bp.N = s.N; bp.Np = s.Np; bp.D = s.D; bp.Dv = s.Dv;
  bp.b = s.b; bp.M = s.M; bp.pad_off = s.pad_off; bp.sm_scale = s.sm_scale;
  bp.y = base + w.y;
  bp.dal = reinterpret_cast<float*>(base + w.dal);
  bp.dcl = reinterpret_cast<float*>(base + w.dcl);
  bp.dy = reinterpret_cast<float*>(base + w.dy);
  bp.dar = reinterpret_cast<float*>(base + w.dar);
  bp.dcr = reinterpret_cast<float*>(base + w.dcr);
  bp.dq = reinterpret_cast<float*>(base + w.dq);
  bp.dk = reinterpret_cast<float*>(base + w.dk);
  bp.dv = reinterpret_cast<float*>(base + w.dv);
  const size_t heads = (size_t)s.E * s.H, bm = (size_t)s.b * s.M;
  // 2. zero the accumulated gradients (dq .. dv are contiguous)
  err = cudaMemsetAsync(base + w.dq, 0, w.total - w.dq, st);
  if (err == cudaSuccess) err = cudaMemsetAsync(base + w.dal, 0, heads * bm * s.D * 4, st);
  if (err == cudaSuccess) err = cudaMemsetAsync(base + w.dcl, 0, heads * bm * 4, st);
  if (err == cudaSuccess) err = cudaMemsetAsync(base + w.dy, 0, heads * bm * s.Dv * 4, st);
  if (err != cudaSuccess) return err;
  auto step_in = [&](int t) {
    bp.al = al[t];
    bp.cl = cl[t];
    bp.ar = ar[t];
    bp.cr = cr[t];
    bp.first = t == 0;
  };
  // 3. output step, final R-step, then (L-step t, R-step t) for t = T-2 .. 0
  step_in(s.T - 1);
  if ((err = launch_kind<K_O, T, T>(bp, st)) != cudaSuccess) return err;
  if ((err = launch_kind<K_RF, T, T>(bp, st)) != cudaSuccess) return err;
  *nlaunch += 2;
  for (int t = s.T - 2; t >= 0; --t) {
    step_in(t);
    err = cudaMemsetAsync(base + w.dal, 0, heads * bm * s.D * 4, st);
    if (err == cudaSuccess) err = cudaMemsetAsync(base + w.dcl, 0, heads * bm * 4, st);
    if (err != cudaSuccess) return err;
    if ((err = launch_kind<K_L, T, T>(bp, st)) != cudaSuccess) return err;
    if ((err = launch_kind<K_R, T, T>(bp, st)) != cudaSuccess) return err;
    *nlaunch += 2;
  }
  // 4. the gradients in the caller's dtype and layout
  const int64_t nd = (int64_t)heads * s.N * s.D, nv = (int64_t)heads * s.N * s.Dv;
  const int thr = 256;
  auto blocks = [&](int64_t n) { return (int)((n + thr - 1) / thr < 4096 ? (n + thr - 1) / thr : 4096); };
  cast_grad_kernel<T><<<blocks(nd), thr, 0, st>>>(bp.dq, s.H, s.N, s.Np, s.D, s.pad_off, nd, p->dq,
                                                  p->dq_stride[0], p->dq_stride[1],
                                                  p->dq_stride[2], p->dq_stride[3]);
  cast_grad_kernel<T><<<blocks(nd), thr, 0, st>>>(bp.dk, s.H, s.N, s.Np, s.D, s.pad_off, nd, p->dk,
                                                  p->dk_stride[0], p->dk_stride[1],
                                                  p->dk_stride[2], p->dk_stride[3]);
  cast_grad_kernel<T><<<blocks(nv), thr, 0, st>>>(bp.dv, s.H, s.N, s.Np, s.Dv, s.pad_off, nv,
                                                  p->dv, p->dv_stride[0], p->dv_stride[1],
                                                  p->dv_stride[2], p->dv_stride[3]);
  *nlaunch += 3;
  return cudaGetLastError();
}

}  // namespace bwd

// ma_api.cu
void set_error_detail(const std::string& detail);
void set_launch_count(int n);
bool generic_supports(const Shape& s);

}  // namespace ma

namespace {

ma::Shape bwd_shape(const ma_fwd_params* p) {
  ma::Shape s{};
  s.E = p->E; s.H = p->H; s.N = p->N; s.D = p->D; s.Dv = p->Dv;
  s.b = p->block_size;
  s.M = (p->N + p->block_size - 1) / p->block_size;
  s.Np = s.M * s.b;
  s.T = p->num_steps;
  s.pre_pad = p->pre_pad ? 1 : 0;
  s.pad_off = s.pre_pad ? s.Np - s.N : 0;
  s.sm_scale = (float)(1.0 / sqrt((double)p->D));  // ma_torch.py:79
  return s;
}

// host checks shared by ma_bwd_workspace_bytes and ma_bwd
int bwd_check(const ma_bwd_params* p) {
  if (p == nullptr) return MA_ERR_NULL_POINTER;
  if (p->struct_size != sizeof(ma_bwd_params)) {
    ma::set_error_detail("struct_size != sizeof(ma_bwd_params)");
    return MA_ERR_BAD_PARAMS;
  }
  const int sel = ma_select_impl(&p->fwd);  // validates the forward parameters
  if (sel < 0) return -sel;
  const ma_fwd_params* f = &p->fwd;
  if (f->dtype == MA_DTYPE_E4M3) {
    ma::set_error_detail("gradients through float8 e4m3 inputs are not supported");
    return MA_ERR_BAD_DTYPE;
  }
  if (f->v_f32) {
    ma::set_error_detail("gradients with fp32 values and 16-bit q / k are not supported");
    return MA_ERR_UNSUPPORTED;
  }
  const ma::Shape s = bwd_shape(f);
  if (s.D > ma::bwd::kMaxDim || s.Dv > ma::bwd::kMaxDim || s.b > ma::bwd::kMaxDim ||
      s.M > ma::bwd::kMaxDim || s.T > 64 || !ma::generic_supports(s)) {
    ma::set_error_detail("the backward kernels take D, Dv, b, M <= 256 and T <= 64");
    return MA_ERR_UNSUPPORTED;
  }
  return MA_OK;
}

}  // namespace

extern "C" size_t ma_bwd_workspace_bytes(const ma_bwd_params* p) {
  if (bwd_check(p) != MA_OK) return 0;
  const int sb = p->fwd.dtype == MA_DTYPE_F32 ? 4 : 2;
  return ma::bwd::layout(bwd_shape(&p->fwd), sb).total;
}

extern "C" int ma_bwd(const ma_bwd_params* p, void* stream) {
  ma::set_error_detail("");
  int rc = bwd_check(p);
  if (rc != MA_OK) return rc;
  const ma_fwd_params* f = &p->fwd;
  if (!f->q || !f->k || !f->v || !p->dout || !p->dq || !p->dk || !p->dv) {
    ma::set_error_detail("q/k/v/dout/dq/dk/dv is NULL");
    return MA_ERR_NULL_POINTER;
  }
  const int64_t* st[8] = {f->q_stride, f->k_stride, f->v_stride, p->dout_stride,
                          p->dq_stride, p->dk_stride, p->dv_stride, f->mask_stride};
  for (int t = 0; t < 7; ++t)
    for (int i = 0; i < 4; ++i)
      if (st[t][i] < 0) {
        ma::set_error_detail("negative stride");
        return MA_ERR_BAD_STRIDE;
      }
  const ma::Shape s = bwd_shape(f);
  const int sb = f->dtype == MA_DTYPE_F32 ? 4 : 2;
  const ma::bwd::Layout w = ma::bwd::layout(s, sb);
  if (p->workspace == nullptr || p->workspace_bytes < w.total) {
    ma::set_error_detail("workspace needs " + std::to_string(w.total) + " bytes, got " +
                         std::to_string(p->workspace_bytes));
    return MA_ERR_WORKSPACE;
  }
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  int n = 0;
  cudaError_t err;
  switch (f->dtype) {
    case MA_DTYPE_F32: err = ma::bwd::run_t<float>(p, s, w, cs, &n); break;
    case MA_DTYPE_F16: err = ma::bwd::run_t<__half>(p, s, w, cs, &n); break;
    case MA_DTYPE_BF16: err = ma::bwd::run_t<__nv_bfloat16>(p, s, w, cs, &n); break;
    default: return MA_ERR_BAD_DTYPE;
  }
  if (err != cudaSuccess) {
    ma::set_error_detail(std::string("CUDA error: ") + cudaGetErrorName(err));
    return MA_ERR_CUDA;
  }
  ma::set_launch_count(n);
  return MA_OK;
}
