// Persistent tcgen05 / TMEM MonarchAttention forward for large blocks
// (block size b = number of blocks M = head dim = 128, i.e. N = 16384).
//
// Work decomposition.  Per head (e, h) the reference runs 2T phases
// (ma/ma_torch.py:100-105):
//   phase 2t   (t < T)  : R-step t, one item per key block m      (al_cl_ref /
//                         al_y_cl_ref when t = T-1, ma_torch.py:10-23, 38-52)
//   phase 2t+1 (t < T-1): L-step t, one item per intra-block index j (ar_cr_ref,
//                         ma_torch.py:26-35)
//   phase 2T-1          : output, one item per j                    (z_ref, :55-62)
// Every phase of a head needs *all* items of the previous phase of the same
// head (the (M,B) <-> (B,M) transpose between steps is an all-to-all inside
// the head).  Instead of one launch per phase, a single persistent kernel
// claims items from a global counter in a wavefront order -- round r holds
// phase p of head r - p for every p -- so an item's producer phase was
// claimed a whole round (2T * 128 items) earlier and dependency waits are
// rare.  Completion is published per (head, phase) with a release counter
// and awaited with bounded acquire spins.  The intermediates of a head live
// in one of 2T+1 workspace slots, reused round-robin (slot reuse waits for
// the output phase of the head that used it before), so the live set stays
// L2-resident.
//
// CTA roles (192 threads, one CTA per SM):
//   warps 0-3  softmax + epilogue; thread i owns row i = TMEM lane i
//   warp 4     scheduler + TMA producer (2-stage SMEM ring)
//   warp 5     TMEM allocator + tcgen05.mma issuer
// Per item:
//   GEMM1  S = A * B^T            (both K-major, SW128 SMEM tiles) -> TMEM
//   softmax over the row (fp32, exp2), P -> TMEM as bf16 (R / out items) or
//          -> SMEM in the MN-major SW128 layout (L items, whose second GEMM
//          contracts over rows)
//   GEMM2  O = P * X  (A from TMEM)   or   O = P^T * Q_j (A MN-major SMEM)
//          plus cr = P^T * 1 on L items (N = 16 GEMM against a ones tile)
//   epilogue: TMEM -> registers -> scale -> bf16 -> global
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdlib.h>
#include <string.h>

#include "ma_common.cuh"

namespace ma {
namespace tc {

constexpr int kThreads = 192;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kT = 128;                  // tile edge: b = M = D = 128
constexpr int kHalf = 16384;             // one 64-column half of a tile (128 rows x 128 B)
constexpr int kTileBytes = 2 * kHalf;    // 32 KB
constexpr int kStageBytes = 3 * kTileBytes;
// small objects at the start of dynamic shared memory
constexpr int kOffBar = 0;        // mbarriers (16 x 8 B)
constexpr int kOffDesc = 128;     // item descriptors (2 x int4)
constexpr int kOffTmem = 160;     // TMEM base address
constexpr int kOffVec = 256;      // per stage: cr[m][:] or cl[j][:] of the item (2 x 512 B)
constexpr int kOffOnes = 1280;    // ones operand of the cr GEMM (512 B)
constexpr int kSmallBytes = 1792;
// 1024-aligned tile region (SW128 atoms): 2 stages x {A, B, X}, then P^T
constexpr int kTileOffP = 2 * kStageBytes;
constexpr int kTileRegion = kTileOffP + kTileBytes;
constexpr int kSmemBytes = kSmallBytes + 1024 + kTileRegion;  // + worst-case alignment pad
static_assert(kSmemBytes <= 232448, "shared memory budget");

// TMEM columns (fp32 accumulators, 128 lanes)
constexpr uint32_t kColS = 0;     // S, then P (bf16 pairs) in its first 64 columns
constexpr uint32_t kColO1 = 128;  // al / ar / z accumulator
constexpr uint32_t kColO2 = 256;  // y accumulator (final R-step)
constexpr uint32_t kColCr = 384;  // cr accumulator (L-step), 16 columns
constexpr uint32_t kTmemCols = 512;

// control block (uint32 words in the workspace)
constexpr int kCtrlNext = 0;   // global work counter
constexpr int kCtrlAbort = 1;  // set when any bounded wait gives up
constexpr int kCtrlDone = 64;  // done[head * P + phase]

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct TcParams {
  CUtensorMap tm_qblk;  // q (E,H,N,D) boxes of 64 x 128 token rows
  CUtensorMap tm_qstr;  // q viewed (E,H,M,b,D): 64 x (tokens j, j+b, ...) boxes
  CUtensorMap tm_kblk;
  CUtensorMap tm_vblk;
  CUtensorMap tm_al;    // al rows [slot][j][m]
  CUtensorMap tm_ar;    // ar rows [slot][m][j]
  CUtensorMap tm_y;     // y rows  [slot][j][m]
  void* out;
  int64_t os[4];
  char* al;
  char* ar;
  char* y;
  float* cl;
  float* cr;
  uint32_t* ctrl;
  uint32_t* status;
  int H, nheads, T, P, slots;
  float sm_scale;
  unsigned long long timeout_ns;
};

enum Kind : int { KIND_R = 0, KIND_L = 1, KIND_O = 2 };

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          bar),
      "r"(bytes)
      : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint32_t ld_relaxed(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* tm, int c0, int c1,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* tm, int c0, int c1,
                                            int c2, int c3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* tm, int c0, int c1,
                                            int c2, int c3, int c4, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
      "r"(bar)
      : "memory");
}

// tcgen05 shared-memory matrix descriptor
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                              uint32_t swizzle) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version (sm_100)
  d |= (uint64_t)swizzle << 61;
  return d;
}
constexpr uint32_t kSwz128 = 2;
constexpr uint32_t kSwzNone = 0;

// instruction descriptor, kind::f16, fp32 accumulate
__host__ __device__ constexpr uint32_t idesc_f16(bool bf16, bool a_mn, bool b_mn, int M, int N) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                       uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive TMEM columns of this thread's lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
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
__device__ __forceinline__ void st_global_v4(void* p, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// ---------------------------------------------------------------------------
// bounded waits: false = gave up (timeout or another role aborted)
// ---------------------------------------------------------------------------
struct Guard {
  uint32_t* abort;
  uint32_t* status;
  unsigned long long limit;
  __device__ __forceinline__ void raise(uint32_t bit) const {
    atomicOr(status, bit);
    atomicExch(abort, 1u);
  }
};

__device__ __noinline__ bool wait_bar(uint32_t bar, uint32_t parity, const Guard& g) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try(bar, parity)) return true;
    if ((spin & 63u) == 0) {
      if (ld_relaxed(g.abort)) return false;
      if (globaltimer() - t0 > g.limit) {
        g.raise(MA_STATUS_WAIT_TIMEOUT);
        return false;
      }
    }
  }
}

__device__ __noinline__ bool wait_counter(const uint32_t* ctr, uint32_t target, const Guard& g) {
  if (ld_acquire(ctr) >= target) return true;
  const uint64_t t0 = globaltimer();
  for (;;) {
    __nanosleep(128);
    if (ld_acquire(ctr) >= target) return true;
    if (ld_relaxed(g.abort)) return false;
    if (globaltimer() - t0 > g.limit) {
      g.raise(MA_STATUS_WAIT_TIMEOUT);
      return false;
    }
  }
}

// warp-uniform bounded wait: every lane waits, and the warp goes on only if
// all lanes saw the phase complete (so .sync.aligned tcgen05 ops that follow
// are executed by the whole warp or by none of it)
__device__ __forceinline__ bool wait_bar_warp(uint32_t bar, uint32_t parity, const Guard& g) {
  const bool ok = wait_bar(bar, parity, g);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// convert 32 fp32 accumulator columns * scale to 16-bit and store 64 B
template <bool BF16>
__device__ __forceinline__ void store_row32(char* dst, const uint32_t (&o)[32], float scale) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t w[4];
#pragma unroll
    for (int t = 0; t < 4; ++t)
      w[t] = pack2<BF16>(__uint_as_float(o[c * 8 + 2 * t]) * scale,
                         __uint_as_float(o[c * 8 + 2 * t + 1]) * scale);
    st_global_v4(dst + c * 16, w[0], w[1], w[2], w[3]);
  }
}

// 128 TMEM accumulator columns of this lane -> scaled 16-bit row of 256 B
template <bool BF16>
__device__ __forceinline__ void store_row128(char* dst, uint32_t taddr, float scale) {
#pragma unroll
  for (int q4 = 0; q4 < 4; ++q4) {
    uint32_t o[32];
    tmem_ld32(taddr + q4 * 32, o);
    tmem_wait_ld();
    store_row32<BF16>(dst + q4 * 64, o, scale);
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <bool BF16>
__global__ void __launch_bounds__(kThreads, 1) ma_tc_kernel(const __grid_constant__ TcParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t sbase = smem_u32(smem_raw);                       // small objects
  const uint32_t tbase = (sbase + kSmallBytes + 1023u) & ~1023u;   // SW128 tiles
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  uint32_t* ctrl = p.ctrl;
  const Guard guard{ctrl + kCtrlAbort, p.status, p.timeout_ns};
  const int P = p.P;
  const uint32_t total = (uint32_t)p.nheads * P * kT;

  const uint32_t bar_full0 = sbase + kOffBar + 0;    // +8 * stage
  const uint32_t bar_empty0 = sbase + kOffBar + 16;  // +8 * stage
  const uint32_t bar_sfull = sbase + kOffBar + 32;
  const uint32_t bar_pready = sbase + kOffBar + 40;
  const uint32_t bar_ofull = sbase + kOffBar + 48;
  const uint32_t bar_ofree = sbase + kOffBar + 56;
  const uint32_t bar_drain = sbase + kOffBar + 64;
  const uint32_t bar_epi = sbase + kOffBar + 72;
  int4* desc_slot = reinterpret_cast<int4*>(smem_raw + kOffDesc);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem_raw + kOffTmem);
  const float* vec0 = reinterpret_cast<const float*>(smem_raw + kOffVec);

  if (tid == 0) {
    mbar_init(bar_full0, 1);
    mbar_init(bar_full0 + 8, 1);
    mbar_init(bar_empty0, 1);
    mbar_init(bar_empty0 + 8, 1);
    mbar_init(bar_sfull, 1);
    mbar_init(bar_pready, 128);
    mbar_init(bar_ofull, 1);
    mbar_init(bar_ofree, 128);
    mbar_init(bar_drain, 1);
    mbar_init(bar_epi, 128);
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
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == kProducerWarp) {
    // ===================== scheduler + TMA producer =====================
    if (lane == 0) {
      // wavefront cursor over valid (round r, phase ph) blocks; blk = index
      int r = 0, ph = 0;
      uint32_t blk = 0;
      bool issued[2] = {false, false};  // a load was issued on the stage
      uint32_t last_on[2] = {0, 0};     // item counter of the last load on it
      uint32_t n = 0;
      for (;; ++n) {
        const int s = n & 1;
        const uint32_t fb = bar_full0 + 8 * s;
        if (n >= 2 && !wait_bar(bar_empty0 + 8 * s, ((n >> 1) - 1) & 1, guard)) break;
        const uint32_t w = atomicAdd(ctrl + kCtrlNext, 1u);
        bool ok = w < total && !ld_relaxed(guard.abort);
        int head = -1, item = 0, kind = 0;
        if (ok) {
          const uint32_t want = w / kT;
          item = (int)(w % kT);
          while (blk < want) {
            ++ph;
            if (ph > (r < P - 1 ? r : P - 1)) {
              ++r;
              ph = r - p.nheads + 1 > 0 ? r - p.nheads + 1 : 0;
            }
            ++blk;
          }
          head = r - ph;
          if (head < 0 || head >= p.nheads) {
            guard.raise(MA_STATUS_BAD_ITEM);
            ok = false;
          }
        }
        if (ok) {
          kind = (ph & 1) == 0 ? KIND_R : (ph == P - 1 ? KIND_O : KIND_L);
          // dependency: the previous phase of this head, or -- for phase 0 --
          // the output phase of the head that used this workspace slot before
          if (ph > 0)
            ok = wait_counter(ctrl + kCtrlDone + head * P + ph - 1, (uint32_t)kT, guard);
          else if (head >= p.slots)
            ok = wait_counter(ctrl + kCtrlDone + (head - p.slots) * P + P - 1, (uint32_t)kT,
                              guard);
        }
        if (!ok) {
          desc_slot[s] = make_int4(-1, 0, 0, 0);  // end marker
          mbar_arrive(fb);
          break;
        }
        desc_slot[s] = make_int4(head, ph, item, kind);
        fence_proxy_async_global();
        const int slot = head % p.slots;
        const int e = head / p.H, hh = head - e * p.H;
        const uint32_t A = tbase + s * kStageBytes, B = A + kTileBytes, X = B + kTileBytes;
        const uint32_t vdst = sbase + kOffVec + s * 512;
        const size_t vrow = ((size_t)slot * kT + item) * kT;  // cr[slot][m][:] / cl[slot][j][:]
        if (kind == KIND_R) {
          const bool first = ph == 0, final_ = ph == P - 2;
          mbar_expect_tx(fb, (final_ ? 3 : 2) * kTileBytes + (first ? 0 : 512));
          if (!first) bulk_load(vdst, p.cr + vrow, 512, fb);
          for (int h2 = 0; h2 < 2; ++h2) {
            if (first)
              tma_load_4d(A + h2 * kHalf, &p.tm_qblk, h2 * 64, item * kT, hh, e, fb);
            else
              tma_load_2d(A + h2 * kHalf, &p.tm_ar, h2 * 64, (slot * kT + item) * kT, fb);
            tma_load_4d(B + h2 * kHalf, &p.tm_kblk, h2 * 64, item * kT, hh, e, fb);
            if (final_) tma_load_4d(X + h2 * kHalf, &p.tm_vblk, h2 * 64, item * kT, hh, e, fb);
          }
        } else {
          const bool out = kind == KIND_O;
          mbar_expect_tx(fb, (out ? 3 : 2) * kTileBytes + 512);
          bulk_load(vdst, p.cl + vrow, 512, fb);
          for (int h2 = 0; h2 < 2; ++h2) {
            tma_load_5d(A + h2 * kHalf, &p.tm_qstr, h2 * 64, item, 0, hh, e, fb);
            tma_load_2d(B + h2 * kHalf, &p.tm_al, h2 * 64, (slot * kT + item) * kT, fb);
            if (out) tma_load_2d(X + h2 * kHalf, &p.tm_y, h2 * 64, (slot * kT + item) * kT, fb);
          }
        }
        issued[s] = true;
        last_on[s] = n;
      }
      // never leave with copies in flight: after an abort, wait (bounded,
      // ignoring the abort flag) until the last load of each stage landed
      if (ld_relaxed(guard.abort)) {
        for (int s = 0; s < 2; ++s) {
          if (!issued[s]) continue;
          const uint32_t par = (last_on[s] >> 1) & 1;
          const uint64_t t0 = globaltimer();
          while (!mbar_try(bar_full0 + 8 * s, par) && globaltimer() - t0 < guard.limit) {
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ===================== tcgen05.mma issuer =====================
    if (lane == 0) {
      constexpr uint32_t id_ss = idesc_f16(BF16, false, false, 128, 128);  // S = A B^T
      constexpr uint32_t id_ts = idesc_f16(BF16, false, true, 128, 128);   // O = P X
      constexpr uint32_t id_mm = idesc_f16(BF16, true, true, 128, 128);    // ar = P^T Q_j
      constexpr uint32_t id_cr = idesc_f16(BF16, true, false, 128, 16);    // cr = P^T 1
      const uint32_t tS = tmem + kColS, tO1 = tmem + kColO1, tO2 = tmem + kColO2,
                     tCr = tmem + kColCr;
      const uint32_t Pt = tbase + kTileOffP;
      const uint32_t ones = sbase + kOffOnes;
      int4 d = make_int4(-1, 0, 0, 0);
      if (wait_bar(bar_full0, 0, guard)) d = desc_slot[0];
      if (d.x >= 0) {
        tc_fence_after();
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
          mma_ss(tS, smem_desc(tbase + off, 16, 1024, kSwz128),
                 smem_desc(tbase + kTileBytes + off, 16, 1024, kSwz128), id_ss, kk > 0);
        }
        mma_commit(bar_sfull);
        for (uint32_t n = 0;; ++n) {
          const int s = n & 1;
          const uint32_t A = tbase + s * kStageBytes, B = A + kTileBytes, X = B + kTileBytes;
          if (!wait_bar(bar_pready, n & 1, guard)) break;
          if (n > 0 && !wait_bar(bar_ofree, (n - 1) & 1, guard)) break;
          tc_fence_after();
          if (d.w == KIND_L) {
            for (int kk = 0; kk < 8; ++kk) {
              const uint32_t off = kk * 2048;  // 16 rows l = two 8-row SW128 atoms
              const uint64_t pd = smem_desc(Pt + off, kHalf, 1024, kSwz128);
              mma_ss(tO1, pd, smem_desc(A + off, kHalf, 1024, kSwz128), id_mm, kk > 0);
              mma_ss(tCr, pd, smem_desc(ones, 128, 256, kSwzNone), id_cr, kk > 0);
            }
          } else {
            const bool final_ = d.w == KIND_R && d.y == P - 2;
            const uint32_t Xo = d.w == KIND_O ? X : B;  // R: O1 = P K[m]; out: O1 = P y_j
            for (int kk = 0; kk < 8; ++kk) {
              const uint32_t off = kk * 2048;
              mma_ts(tO1, tS + kk * 8, smem_desc(Xo + off, kHalf, 1024, kSwz128), id_ts, kk > 0);
              if (final_)
                mma_ts(tO2, tS + kk * 8, smem_desc(X + off, kHalf, 1024, kSwz128), id_ts, kk > 0);
            }
          }
          mma_commit(bar_ofull);
          mma_commit(bar_empty0 + 8 * s);
          // next item's GEMM1 into S: the tensor pipe runs MMAs in issue
          // order, so it starts after this item's GEMM2 has read P
          const int s1 = (n + 1) & 1;
          if (!wait_bar(bar_full0 + 8 * s1, ((n + 1) >> 1) & 1, guard)) break;
          d = desc_slot[s1];
          if (d.x < 0) {
            mbar_arrive(bar_sfull);  // pass the end marker to the softmax warps
            break;
          }
          tc_fence_after();
          const uint32_t A1 = tbase + s1 * kStageBytes, B1 = A1 + kTileBytes;
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
            mma_ss(tS, smem_desc(A1 + off, 16, 1024, kSwz128),
                   smem_desc(B1 + off, 16, 1024, kSwz128), id_ss, kk > 0);
          }
          mma_commit(bar_sfull);
        }
      } else {
        mbar_arrive(bar_sfull);  // nothing to do (or gave up): pass the end marker on
      }
      // let every issued MMA complete before TMEM is released
      mma_commit(bar_drain);
      const uint64_t t0 = globaltimer();
      while (!mbar_try(bar_drain, 0) && globaltimer() - t0 < guard.limit) {
      }
    }
  } else {
    // ===================== softmax + epilogue (warps 0-3) =====================
    const int row = tid;  // = TMEM lane
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const uint32_t tS = tmem + lane_off + kColS;
    const uint32_t tO1 = tmem + lane_off + kColO1;
    const uint32_t tO2 = tmem + lane_off + kColO2;
    const uint32_t tCr = tmem + lane_off + kColCr;
    for (uint32_t n = 0;; ++n) {
      if (!wait_bar_warp(bar_sfull, n & 1, guard)) break;
      const int4 d = desc_slot[n & 1];
      if (d.x < 0) break;
      // the stage's vector was written by the async proxy: observe its barrier
      // (already complete -- the MMA warp waited on it before GEMM1)
      if (!wait_bar_warp(bar_full0 + 8 * (n & 1), (n >> 1) & 1, guard)) break;
      tc_fence_after();
      const int head = d.x, ph = d.y, item = d.z, kind = d.w;
      const int slot = head % p.slots;
      const bool final_ = kind == KIND_R && ph == P - 2;
      const float* vec = vec0 + (n & 1) * 128;  // cr[m][:] (R) or cl[j][:] (L / out)

      uint32_t sv[128];
      tmem_ld32(tS + 0, *reinterpret_cast<uint32_t(*)[32]>(sv + 0));
      tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
      tmem_ld32(tS + 64, *reinterpret_cast<uint32_t(*)[32]>(sv + 64));
      tmem_ld32(tS + 96, *reinterpret_cast<uint32_t(*)[32]>(sv + 96));
      tmem_wait_ld();

      float sum = 0.0f, scale_out = 1.0f, cl_row = 0.0f;
      if (kind == KIND_R) {
        // t_i = sm_scale * S_i / (cr_j + eps); mx = max(max_i t_i, eps)
        // (ma_torch.py:11-16), carried in log2 units: u_i = (t_i - mx) log2(e)
        const float crj = ph > 0 ? vec[row] : 1.0f;
        const float c = p.sm_scale / (crj + kEps);
        float smax = -INFINITY;
#pragma unroll
        for (int i = 0; i < 128; ++i) smax = fmaxf(smax, __uint_as_float(sv[i]));
        const float mx = fmaxf(c * smax, kEps);
        const float c2 = c * kLog2e, m2 = mx * kLog2e;
        float wsum = 0.0f;
#pragma unroll
        for (int i = 0; i < 128; ++i) {
          const float u = fmaf(__uint_as_float(sv[i]), c2, -m2);
          const float e = ex2(u);
          sum += e;
          wsum = fmaf(e, u, wsum);
          sv[i] = __float_as_uint(e);
        }
        const float den = sum + kEps;  // r = e / (sum + eps), :17
        const float inv = 1.0f / den;
        // cl = sum_i r_i log r_i, log r_i = (t_i - mx) - log(den)  (:20)
        cl_row = kLn2 * inv * wsum - __logf(den) * sum * inv;
        scale_out = inv;
      } else {
        // logits S'[l][k] - cl[j][k], softmax over k (ma_torch.py:27-29, 56-58)
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < 128; i += 4) {
          const float4 c4 = *reinterpret_cast<const float4*>(vec + i);
          const float u0 = __uint_as_float(sv[i + 0]) - c4.x;
          const float u1 = __uint_as_float(sv[i + 1]) - c4.y;
          const float u2 = __uint_as_float(sv[i + 2]) - c4.z;
          const float u3 = __uint_as_float(sv[i + 3]) - c4.w;
          sv[i + 0] = __float_as_uint(u0);
          sv[i + 1] = __float_as_uint(u1);
          sv[i + 2] = __float_as_uint(u2);
          sv[i + 3] = __float_as_uint(u3);
          mx = fmaxf(mx, fmaxf(fmaxf(u0, u1), fmaxf(u2, u3)));
        }
        const float m2 = mx * kLog2e;
#pragma unroll
        for (int i = 0; i < 128; ++i) {
          const float e = ex2(fmaf(__uint_as_float(sv[i]), kLog2e, -m2));
          sum += e;
          sv[i] = __float_as_uint(e);
        }
        scale_out = 1.0f / sum;
      }

      if (kind == KIND_L) {
        // P[l][k] (normalised; every query row valid here) -> SMEM in the
        // MN-major SW128 layout: row l of half h at h*16K + l*128, 16-byte
        // chunk c at position c ^ (l & 7)
        const uint32_t prow = tbase + kTileOffP + row * 128;
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const int k0 = h2 * 64 + c * 8;
            uint32_t a[4];
#pragma unroll
            for (int t = 0; t < 4; ++t)
              a[t] = pack2<BF16>(__uint_as_float(sv[k0 + 2 * t]) * scale_out,
                                 __uint_as_float(sv[k0 + 2 * t + 1]) * scale_out);
            st_shared_v4(prow + h2 * kHalf + ((c ^ (row & 7)) << 4), a[0], a[1], a[2], a[3]);
          }
        }
        fence_proxy_async_smem();
      } else {
        // P (unnormalised) -> TMEM columns 0..63 as packed 16-bit pairs
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 32; ++c)
          pk[c] = pack2<BF16>(__uint_as_float(sv[2 * c]), __uint_as_float(sv[2 * c + 1]));
        tmem_st32(tS + 0, pk);
#pragma unroll
        for (int c = 0; c < 32; ++c)
          pk[c] = pack2<BF16>(__uint_as_float(sv[64 + 2 * c]), __uint_as_float(sv[65 + 2 * c]));
        tmem_st32(tS + 32, pk);
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(bar_pready);

      // ---------------- epilogue ----------------
      if (!wait_bar_warp(bar_ofull, n & 1, guard)) break;
      tc_fence_after();
      if (kind == KIND_R) {
        // al[j][m] = sm_scale * r K[m] (ma_torch.py:21); y[j][m] = r V[m] (:51)
        const size_t orow = (((size_t)slot * kT + row) * kT + item) * kT * 2;
        store_row128<BF16>(p.al + orow, tO1, p.sm_scale * scale_out);
        if (final_) store_row128<BF16>(p.y + orow, tO2, scale_out);
        p.cl[((size_t)slot * kT + row) * kT + item] = cl_row;  // cl[j][m]
      } else if (kind == KIND_L) {
        // ar[k][j] = sum_l P[l][k] q[l*b+j]; cr[k][j] = sum_l P[l][k] (:32-34)
        const size_t orow = (((size_t)slot * kT + row) * kT + item) * kT * 2;
        store_row128<BF16>(p.ar + orow, tO1, 1.0f);
        uint32_t o[32];
        tmem_ld32(tCr, o);  // the N = 16 accumulator; every column holds the sum
        tmem_wait_ld();
        p.cr[((size_t)slot * kT + row) * kT + item] = __uint_as_float(o[0]);
      } else {
        // z[l*b + j] = (P y_j) / sum (ma_torch.py:60-62)
        const int e = head / p.H, hh = head - e * p.H;
        char* dst = reinterpret_cast<char*>(p.out) +
                    2 * ((int64_t)e * p.os[0] + (int64_t)hh * p.os[1] +
                         (int64_t)(row * kT + item) * p.os[2]);
        store_row128<BF16>(dst, tO1, scale_out);
      }
      tc_fence_before();
      mbar_arrive(bar_ofree);
      // publish the item once all 128 rows are stored
      __threadfence();
      mbar_arrive(bar_epi);
      if (warp == 0) {  // lane 0 waits; the decision stays warp-uniform
        bool ok = true;
        if (lane == 0) {
          ok = wait_bar(bar_epi, n & 1, guard);
          if (ok) red_release_add(ctrl + kCtrlDone + head * P + ph, 1u);
        }
        if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      }
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

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
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
  CUresult r = fn(tm, dt, (cuuint32_t)rank, const_cast<void*>(base), gd, gs, bx, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace tc

static bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

bool tc_supports(const ma_fwd_params* p, const Shape& s) {
  const char* off = getenv("MA_DISABLE_TC");
  if (off && off[0] == '1') return false;
  if (p->dtype != MA_DTYPE_BF16 && p->dtype != MA_DTYPE_F16) return false;
  if (s.D != 128 || s.Dv != 128 || s.b != 128 || s.M != 128 || s.N != s.Np) return false;
  if (p->mask_dtype != MA_MASK_NONE) return false;
  const int64_t* st[4] = {p->q_stride, p->k_stride, p->v_stride, p->o_stride};
  for (int t = 0; t < 4; ++t) {
    if (st[t][3] != 1) return false;
    for (int i = 0; i < 3; ++i)
      if ((st[t][i] * 2) % 16 != 0 || st[t][i] <= 0) return false;
  }
  if (p->q && !(aligned16(p->q) && aligned16(p->k) && aligned16(p->v) && aligned16(p->out)))
    return false;
  return true;
}

size_t tc_ctrl_bytes(const Shape& s) {
  return sizeof(uint32_t) * (tc::kCtrlDone + (size_t)s.E * s.H * 2 * s.T) + 256;
}

cudaError_t run_tc(const ma_fwd_params* p, const Shape& s, const WsLayout& ws, cudaStream_t st,
                   int* nlaunch) {
  using namespace tc;
  TcParams tp;
  memset(&tp, 0, sizeof(tp));
  const CUtensorMapDataType dt =
      p->dtype == MA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int nheads = s.E * s.H;
  const int P = 2 * s.T;
  int slots = 2 * s.T + 1;
  if (slots > nheads) slots = nheads;
  const uint32_t box_blk[4] = {64, kT, 1, 1};
  const uint32_t box_str[5] = {64, 1, kT, 1, 1};
  const uint32_t box_ws[2] = {64, kT};
  bool ok = true;
  auto tok_map = [&](CUtensorMap* tm, const void* base, const int64_t* es) {
    const uint64_t dims[4] = {(uint64_t)s.D, (uint64_t)s.N, (uint64_t)s.H, (uint64_t)s.E};
    const uint64_t str[3] = {(uint64_t)es[2] * 2, (uint64_t)es[1] * 2, (uint64_t)es[0] * 2};
    ok = ok && encode(tm, dt, 4, base, dims, str, box_blk);
  };
  tok_map(&tp.tm_qblk, p->q, p->q_stride);
  tok_map(&tp.tm_kblk, p->k, p->k_stride);
  tok_map(&tp.tm_vblk, p->v, p->v_stride);
  {
    const int64_t* es = p->q_stride;
    const uint64_t dims[5] = {(uint64_t)s.D, (uint64_t)s.b, (uint64_t)s.M, (uint64_t)s.H,
                              (uint64_t)s.E};
    const uint64_t str[4] = {(uint64_t)es[2] * 2, (uint64_t)es[2] * 2 * s.b, (uint64_t)es[1] * 2,
                             (uint64_t)es[0] * 2};
    ok = ok && encode(&tp.tm_qstr, dt, 5, p->q, dims, str, box_str);
  }
  char* w = reinterpret_cast<char*>(p->workspace);
  const uint64_t rows = (uint64_t)slots * s.b * s.M;
  {
    const uint64_t dims[2] = {(uint64_t)s.D, rows};
    const uint64_t str[1] = {(uint64_t)s.D * 2};
    ok = ok && encode(&tp.tm_al, dt, 2, w + ws.al, dims, str, box_ws);
    ok = ok && encode(&tp.tm_ar, dt, 2, w + ws.ar, dims, str, box_ws);
    const uint64_t dimy[2] = {(uint64_t)s.Dv, rows};
    const uint64_t stry[1] = {(uint64_t)s.Dv * 2};
    ok = ok && encode(&tp.tm_y, dt, 2, w + ws.y, dimy, stry, box_ws);
  }
  if (!ok) return cudaErrorInvalidValue;
  tp.out = p->out;
  for (int i = 0; i < 4; ++i) tp.os[i] = p->o_stride[i];
  tp.al = w + ws.al;
  tp.ar = w + ws.ar;
  tp.y = w + ws.y;
  tp.cl = reinterpret_cast<float*>(w + ws.cl);
  tp.cr = reinterpret_cast<float*>(w + ws.cr);
  tp.ctrl = reinterpret_cast<uint32_t*>(w + ws.ctrl);
  tp.status = p->status;
  tp.H = s.H;
  tp.nheads = nheads;
  tp.T = s.T;
  tp.P = P;
  tp.slots = slots;
  tp.sm_scale = s.sm_scale;
  tp.timeout_ns = 2000000000ull;  // 2 s per bounded wait
  const char* tmo = getenv("MA_WAIT_TIMEOUT_NS");
  if (tmo) tp.timeout_ns = strtoull(tmo, nullptr, 10);

  int dev = 0, sms = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (err != cudaSuccess) return err;
  err = cudaMemsetAsync(tp.ctrl, 0, ws.ctrl_bytes, st);
  if (err != cudaSuccess) return err;
  auto kfn = p->dtype == MA_DTYPE_BF16 ? ma_tc_kernel<true> : ma_tc_kernel<false>;
  err = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (err != cudaSuccess) return err;
  const int64_t items = (int64_t)nheads * P * kT;
  const int grid = (int)(items < sms ? items : sms);
  kfn<<<grid, kThreads, kSmemBytes, st>>>(tp);
  err = cudaGetLastError();
  if (err == cudaSuccess) *nlaunch += 1;
  return err;
}

}  // namespace ma
