// Prefill GLA on the tensor cores (tcgen05 + TMEM + TMA), chunk-parallel.
//
// Replaces chunk_gla_fwd_kernel (src/chunk_gla_inlier.py:5-150) for bf16/f16
// inputs with head dim 64 or 128 and a per-head scalar decay (no log_alpha).
// Operand tiles are [128 tokens x D channels] in 64-channel column blocks of
// 128-byte swizzled rows (one TMA box each), so D = 128 uses two blocks.  The
// reference runs one program per (b,h) that walks every chunk in sequence; here
// every 128-token chunk of every (b,h) is its own CTA in two of three launches:
//
//   A  gla_tc_state_kernel   (one CTA per chunk c)
//        G   = inclusive cumsum of log_gamma over the chunk, G_C = its total
//        Kd  = K_I * exp(G_C - G_t)        (rows of the K tile, in shared memory)
//        dS  = Kd^T V                      tcgen05.mma, M = 64 or 128 (inlier rows,
//                                          padded), N = D, K = 128 tokens, A and B MN-major;
//                                          Kd as hi + lo 16-bit terms, two MMAs
//        -> workspace: dS_c [J x D] fp32 and G_C
//   B  gla_tc_scan_kernel    (one thread per state element of a head)
//        S_0 = state_init or 0;  start_c = S before chunk c;  S <- exp(G_C) S + dS_c
//        start_c overwrites dS_c in the workspace; the last S goes to state_out
//   C  gla_tc_out_kernel     (one CTA per chunk c; at D = 64 Y2 and then Y1 reuse A's
//                             upper TMEM columns once P is formed: 128 columns, 3 CTAs/SM)
//        A   = Q_I K_I^T            tcgen05.mma M=128, N=128, K=J (A/B K-major)
//        Y2  = Q_I start_c          tcgen05.mma M=128, N=D,   K=J (start_c as a bf16
//                                   MN-major operand)
//        P   = A * exp(G_i - G_j) [j <= i]  -> bf16, written back into TMEM
//        Y1  = P V                  tcgen05.mma, A = P from TMEM, V MN-major
//        y   = Y1 + exp(G_i) Y2, then (1 - mix) * gla_scale * RMSNorm(y)
//
// All decay factors are exponentials of non-positive differences of cumulative
// log decays (no overflow).  Rounding points: the masked score matrix and the
// carried state enter the output kernel's tensor-core products in the input
// dtype, as in the reference kernel; the decayed keys of the state update
// enter as a hi + lo pair of 16-bit terms (the reference rounds them once),
// accumulation is fp32 and the state carried between chunks stays fp32.
// Waits are bounded (sm100::mbar_wait); a timeout is recorded in
// g_gla_tc_status and the CTA skips its remaining issue, frees TMEM and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace hofa {

__device__ int g_gla_tc_status;

namespace {

constexpr int kC = 128;           // tokens per chunk
constexpr int kThreads = 128;
constexpr uint32_t kTile = kC * 128;  // one [128 rows x 128 B] column block (64 channels)

template <int D>
struct Geo {
  static constexpr int NB = D / 64;                      // 64-channel column blocks
  static constexpr uint32_t OP = NB * kTile;             // one operand tile (128 tokens x D)
  static constexpr uint32_t LBO = NB > 1 ? kTile : 16;   // byte distance of the column blocks
  static constexpr int STATE_M = D == 64 ? 64 : 128;     // MMA M of the state kernel
  // output kernel TMEM: D = 64 keeps A (128 columns) and lets Y2 then Y1 use A's
  // upper half once P is formed (128 columns, three CTAs per SM); D = 128 holds
  // A, Y1 and Y2 side by side (512 columns, one CTA per SM)
  static constexpr bool SHARE = D == 64;
  static constexpr uint32_t OUT_COLS = SHARE ? 128 : 512;
  static constexpr size_t STATE_SMEM = 3 * OP + 1024 + 256;   // K (then Kd hi), V, Kd lo
  // D = 64: 80 KB keeps <= 2 CTAs (2 x 256 TMEM columns) per SM; D = 128: one CTA
  static constexpr size_t OUT_SMEM = 4 * OP + 1024 + 4096;
};

__device__ __forceinline__ uint32_t pack2(float a, float b, bool bf16) {
  if (bf16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Inclusive prefix sum of one value per thread over the 128 threads.
__device__ __forceinline__ float block_scan128(float x, float* sm_warp, int tid) {
  const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sm_warp[warp] = x;
  __syncthreads();
  float add = 0.f;
  for (int w = 0; w < warp; ++w) add += sm_warp[w];
  return x + add;
}

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// A: per-chunk state contribution dS = (K * exp(G_C - G_t))^T V
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(kThreads)
gla_tc_state_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                    const GlaParams p) {
  using Gm = Geo<D>;
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC = sm100::idesc_f16(BF16, true, true, Gm::STATE_M, D);
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sK = base;
  unsigned char* sV = base + Gm::OP;
  unsigned char* sL = base + 2 * Gm::OP;   // Kd lo
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + 3 * Gm::OP);
  float* sm_warp = reinterpret_cast<float*>(bars + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm_warp + 4);
  int* err = reinterpret_cast<int*>(tmem_slot + 1);

  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = c * kC;
  const int bh = b * p.H + h;
  if (tid == 0) {
    sm100::mbar_init(&bars[0], 1);
    sm100::mbar_init(&bars[1], 1);
    *err = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tmem_slot, D);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) {
    sm100::mbar_arrive_expect_tx(&bars[0], 2 * Gm::OP);
#pragma unroll
    for (int nb = 0; nb < Gm::NB; ++nb) {
      sm100::tma_load_4d(sK + nb * kTile, &tk, p.R + 64 * nb, t0, h, b, &bars[0]);
      sm100::tma_load_4d(sV + nb * kTile, &tv, 64 * nb, t0, h, b, &bars[0]);
    }
  }
  const int t = t0 + tid;
  const float g = t < p.T ? ld_any(p.log_gamma, p.dt_lg, b * p.slg[0] + h * p.slg[1] + (int64_t)t * p.slg[2]) : 0.f;
  const float G = block_scan128(g, sm_warp, tid);
  __shared__ float sm_gc;  // the chunk's total log decay (thread 127's prefix)
  if (tid == kThreads - 1) sm_gc = G;
  volatile int* verr = err;
  if (!sm100::mbar_wait(&bars[0], 0)) atomicOr(err, 1);
  __syncthreads();
  const float gc = sm_gc;
  // Kd = K * exp(G_C - G_t) enters the tensor core as two 16-bit terms,
  // Kd = hi + lo (hi = Kd rounded, lo = the rounding remainder, rounded), so
  // the fp32 state keeps about 16 significant bits of every key instead of
  // the 8 of a single bf16 operand.  The reference rounds Kd once
  // (src/chunk_gla_inlier.py:122-125); that alone puts about 2e-2 of absolute
  // error into a state of magnitude 10 over 8192 tokens.  hi replaces the K
  // tile, lo has a tile of its own, and both products accumulate into the same
  // TMEM columns under one commit.
  {
    const float w = sm100::ex2_approx((gc - G) * kLog2e);
#pragma unroll
    for (int nb = 0; nb < Gm::NB; ++nb) {
      uint4* row = reinterpret_cast<uint4*>(sK + nb * kTile + tid * 128);
      uint4* lrow = reinterpret_cast<uint4*>(sL + nb * kTile + tid * 128);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        uint4 u = row[q], l;
        uint32_t* pu = reinterpret_cast<uint32_t*>(&u);
        uint32_t* pl = reinterpret_cast<uint32_t*>(&l);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float a, bb;
          if (BF16) bf16x2_to_f(pu[e], a, bb);
          else f16x2_to_f(pu[e], a, bb);
          const float xa = a * w, xb = bb * w;
          pu[e] = pack2(xa, xb, BF16);
          float ha, hb;
          if (BF16) bf16x2_to_f(pu[e], ha, hb);
          else f16x2_to_f(pu[e], ha, hb);
          pl[e] = pack2(xa - ha, xb - hb, BF16);
        }
        row[q] = u;
        lrow[q] = l;
      }
    }
  }
  fence_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  if (tid == 0 && !*verr) {
    sm100::tc_fence_after();
    const uint64_t adesc = sm100::smem_desc(sK, Gm::LBO, 1024, sm100::kSwizzle128);
    const uint64_t ldesc = sm100::smem_desc(sL, Gm::LBO, 1024, sm100::kSwizzle128);
    const uint64_t bdesc = sm100::smem_desc(sV, Gm::LBO, 1024, sm100::kSwizzle128);
#pragma unroll
    for (int ks = 0; ks < kC / 16; ++ks)
      sm100::mma_ss(tmem, adesc + (uint64_t)(ks * 2048 >> 4), bdesc + (uint64_t)(ks * 2048 >> 4), IDESC, ks > 0);
#pragma unroll
    for (int ks = 0; ks < kC / 16; ++ks)
      sm100::mma_ss(tmem, ldesc + (uint64_t)(ks * 2048 >> 4), bdesc + (uint64_t)(ks * 2048 >> 4), IDESC, true);
    sm100::mma_commit(&bars[1]);
  }
  if (!*verr && !sm100::mbar_wait(&bars[1], 0)) atomicOr(err, 1);
  sm100::tc_fence_after();
  // D (M = 64): row j lives in lane 32*(j/16) + j%16; (M = 128): row j in lane j
  const int j = Gm::STATE_M == 64 ? 16 * warp + lane : tid;
  const bool row_ok = (Gm::STATE_M == 64 ? lane < 16 : true) && j < p.J && !*verr;
  const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
  float* dst = p.ws_state + (((int64_t)bh * p.nseg + c) * p.J + j) * D;
#pragma unroll
  for (int half = 0; half < D / 32; ++half) {
    uint32_t r[32];
    sm100::tmem_ld32(taddr + half * 32, r);
    sm100::tc_wait_ld();
    if (row_ok) {
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(dst + half * 32 + i) =
            make_float4(__uint_as_float(r[i]), __uint_as_float(r[i + 1]), __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
    }
  }
  if (tid == 0) p.ws_decay[(int64_t)bh * p.nseg + c] = gc;
  sm100::tc_fence_before();
  __syncthreads();
  if (*err && tid == 0) atomicOr(&g_gla_tc_status, 1);
  if (warp == 0) sm100::tmem_dealloc(tmem, D);
}

// ---------------------------------------------------------------------------
// B: scan over chunks (start state of every chunk, final state)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gla_tc_scan_kernel(const GlaParams p) {
  const int e = blockIdx.x * 256 + threadIdx.x;  // element j*D + d of the head's state
  const int h = blockIdx.y, b = blockIdx.z;
  if (e >= p.J * p.D) return;
  const int j = e / p.D, d = e % p.D;
  const int64_t bh = (int64_t)b * p.H + h;
  float S = p.state_init ? p.state_init[b * p.ssi[0] + h * p.ssi[1] + j * p.ssi[2] + d] : 0.f;
  float* ws = p.ws_state + bh * p.nseg * p.J * p.D + e;
  const float* gc = p.ws_decay + bh * p.nseg;
  const int64_t cs = (int64_t)p.J * p.D;
  // 16 chunk contributions per round trip: their loads are independent, only
  // the fmaf chain is sequential.  The next batch is requested before this
  // batch's start states are stored (the compiler cannot move those loads
  // above the stores, which it must assume may alias), so round trips overlap.
  constexpr int kU = 16;
  const int full = p.nseg / kU * kU;
  float dS[kU], g[kU], dSn[kU], gn[kU];
  if (full > 0) {
#pragma unroll
    for (int u = 0; u < kU; ++u) { dSn[u] = ws[u * cs]; gn[u] = gc[u]; }
  }
  int c = 0;
  for (; c < full; c += kU) {
#pragma unroll
    for (int u = 0; u < kU; ++u) { dS[u] = dSn[u]; g[u] = gn[u]; }
    if (c + kU < full) {
#pragma unroll
      for (int u = 0; u < kU; ++u) { dSn[u] = ws[(c + kU + u) * cs]; gn[u] = gc[c + kU + u]; }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      ws[(c + u) * cs] = S;
      S = fmaf(sm100::ex2_approx(g[u] * kLog2e), S, dS[u]);
    }
  }
  for (; c < p.nseg; ++c) {
    const float dS = ws[c * cs];
    ws[c * cs] = S;
    S = fmaf(sm100::ex2_approx(gc[c] * kLog2e), S, dS);
  }
  if (p.state_out) p.state_out[b * p.sso[0] + h * p.sso[1] + j * p.sso[2] + d * p.sso[3]] = S;
}

// ---------------------------------------------------------------------------
// C: per-chunk output
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(kThreads, D == 64 ? 3 : 1)
gla_tc_out_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, const GlaParams p) {
  using Gm = Geo<D>;
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC_A = sm100::idesc_f16(BF16, false, false, 128, 128);
  constexpr uint32_t IDESC_Y = sm100::idesc_f16(BF16, false, true, 128, D);
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = base;
  unsigned char* sK = base + Gm::OP;
  unsigned char* sV = base + 2 * Gm::OP;
  unsigned char* sS = base + 3 * Gm::OP;              // start state, [128 rows j][D] bf16 MN-major blocks
  float* sG = reinterpret_cast<float*>(sS + Gm::OP);  // cumulative log2 decay per token
  float* sGS = sG + kC;                                // gla_scale[h, 0:D]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sGS + D);
  float* sm_warp = reinterpret_cast<float*>(bars + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm_warp + 4);
  int* err = reinterpret_cast<int*>(tmem_slot + 1);

  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int t0 = c * kC;
  const int bh = b * p.H + h;
  const int J = p.J, KS = (J + 15) / 16;
  if (tid == 0) {
    sm100::mbar_init(&bars[0], 1);
    sm100::mbar_init(&bars[1], 1);
    *err = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tmem_slot, Gm::OUT_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tA = tmem;
  const uint32_t tY1 = Gm::SHARE ? tmem + 64 : tmem + 128, tY2 = Gm::SHARE ? tmem + 64 : tmem + 128 + D;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  if (tid == 0) {
    sm100::mbar_arrive_expect_tx(&bars[0], 3 * Gm::OP);
#pragma unroll
    for (int nb = 0; nb < Gm::NB; ++nb) {
      sm100::tma_load_4d(sQ + nb * kTile, &tq, p.R + 64 * nb, t0, h, b, &bars[0]);
      sm100::tma_load_4d(sK + nb * kTile, &tk, p.R + 64 * nb, t0, h, b, &bars[0]);
      sm100::tma_load_4d(sV + nb * kTile, &tv, 64 * nb, t0, h, b, &bars[0]);
    }
  }
  // Every global read of the prologue is issued before the first shared-memory
  // store: the stores go through generic pointers that the compiler cannot
  // tell apart from the global sources, so a load placed after one waits for
  // the round trips before it.
  static_assert(D <= kThreads, "one gla_scale value per thread");
  const int t = t0 + tid;
  const float g = t < p.T ? ld_any(p.log_gamma, p.dt_lg, b * p.slg[0] + h * p.slg[1] + (int64_t)t * p.slg[2]) : 0.f;
  float mix = 0.f;
  if (p.fuse && t < p.T) mix = ld_any(p.mix_g, p.dt_mg, b * p.smg[0] + h * p.smg[1] + (int64_t)t * p.smg[2]);
  const float gsv = tid < D && p.fuse ? ld_any(p.gla_scale, p.dt_gs, h * p.sgs[0] + tid * p.sgs[1]) : 1.f;
  // start state of this chunk -> bf16 MN-major operand (row j = 128 bytes per block, 128B swizzle);
  // each 64-channel block of the row is read into registers at once, then packed
  if (tid < 16 * KS) {
    const int j = tid;
    const float* src = p.ws_state + (((int64_t)bh * p.nseg + c) * J + j) * D;
#pragma unroll
    for (int nb = 0; nb < Gm::NB; ++nb) {
      float4 f[16];
#pragma unroll
      for (int q = 0; q < 16; ++q)
        f[q] = j < J ? reinterpret_cast<const float4*>(src + nb * 64)[q] : make_float4(0.f, 0.f, 0.f, 0.f);
      uint4* row = reinterpret_cast<uint4*>(sS + nb * kTile + j * 128);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 a = f[2 * q], bq = f[2 * q + 1];
        uint4 u;
        u.x = pack2(a.x, a.y, BF16); u.y = pack2(a.z, a.w, BF16);
        u.z = pack2(bq.x, bq.y, BF16); u.w = pack2(bq.z, bq.w, BF16);
        row[q ^ (j & 7)] = u;
      }
    }
  }
  const float G = block_scan128(g, sm_warp, tid) * kLog2e;   // log2 units from here on
  sG[tid] = G;
  if (tid < D) sGS[tid] = gsv;
  fence_async_smem();
  volatile int* verr = err;
  if (!sm100::mbar_wait(&bars[0], 0)) atomicOr(err, 1);
  sm100::tc_fence_before();
  __syncthreads();
  if (tid == 0 && !*verr) {
    sm100::tc_fence_after();
    const uint64_t qdesc = sm100::smem_desc(sQ, 16, 1024, sm100::kSwizzle128);
    const uint64_t kdesc = sm100::smem_desc(sK, 16, 1024, sm100::kSwizzle128);
    const uint64_t sdesc = sm100::smem_desc(sS, Gm::LBO, 1024, sm100::kSwizzle128);
    // K-major steps of 16 channels: 4 per 128-byte block (32 B each), blocks kTile apart
    auto kstep = [](int ks) { return (uint64_t)(((ks >> 2) * kTile + (ks & 3) * 32) >> 4); };
    for (int ks = 0; ks < KS; ++ks) sm100::mma_ss(tA, qdesc + kstep(ks), kdesc + kstep(ks), IDESC_A, ks > 0);
    if (!Gm::SHARE)
      for (int ks = 0; ks < KS; ++ks)
        sm100::mma_ss(tY2, qdesc + kstep(ks), sdesc + (uint64_t)(ks * 2048 >> 4), IDESC_Y, ks > 0);
    sm100::mma_commit(&bars[1]);
  }
  if (!*verr && !sm100::mbar_wait(&bars[1], 0)) atomicOr(err, 1);
  sm100::tc_fence_after();

  // P = A * exp(G_i - G_j) for j <= i, as 16-bit pairs over columns [0, 64)
  const int i = tid;
#pragma unroll
  for (int cc = 0; cc < kC; cc += 64) {
    uint32_t r0[32], r1[32], pk[32];
    sm100::tmem_ld32(tA + lane_off + cc, r0);
    sm100::tmem_ld32(tA + lane_off + cc + 32, r1);
    sm100::tc_wait_ld();
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int j0 = cc + 2 * u, j1 = cc + 32 + 2 * u;
      const float a0 = j0 <= i ? __uint_as_float(r0[2 * u]) * sm100::ex2_approx(G - sG[j0]) : 0.f;
      const float a1 = j0 + 1 <= i ? __uint_as_float(r0[2 * u + 1]) * sm100::ex2_approx(G - sG[j0 + 1]) : 0.f;
      const float a2 = j1 <= i ? __uint_as_float(r1[2 * u]) * sm100::ex2_approx(G - sG[j1]) : 0.f;
      const float a3 = j1 + 1 <= i ? __uint_as_float(r1[2 * u + 1]) * sm100::ex2_approx(G - sG[j1 + 1]) : 0.f;
      pk[u] = pack2(a0, a1, BF16);
      pk[16 + u] = pack2(a2, a3, BF16);
    }
    sm100::tmem_st32(tA + lane_off + cc / 2, pk);
  }
  sm100::tc_wait_st();
  sm100::tc_fence_before();
  __syncthreads();
  // SHARE: Y2 = Q_I start_c into A's upper half (consumed above), read into
  // registers, then Y1 = P V into the same columns
  float y2r[Gm::SHARE ? D : 1];
  if constexpr (Gm::SHARE) {
    if (tid == 0 && !*verr) {
      sm100::tc_fence_after();
      const uint64_t qdesc = sm100::smem_desc(sQ, 16, 1024, sm100::kSwizzle128);
      const uint64_t sdesc = sm100::smem_desc(sS, Gm::LBO, 1024, sm100::kSwizzle128);
      auto kstep = [](int ks) { return (uint64_t)(((ks >> 2) * kTile + (ks & 3) * 32) >> 4); };
      for (int ks = 0; ks < KS; ++ks)
        sm100::mma_ss(tY2, qdesc + kstep(ks), sdesc + (uint64_t)(ks * 2048 >> 4), IDESC_Y, ks > 0);
      sm100::mma_commit(&bars[1]);
    }
    if (!*verr && !sm100::mbar_wait(&bars[1], 1)) atomicOr(err, 1);
    sm100::tc_fence_after();
#pragma unroll
    for (int cc = 0; cc < D; cc += 32) {
      uint32_t a[32];
      sm100::tmem_ld32(tY2 + lane_off + cc, a);
      sm100::tc_wait_ld();
#pragma unroll
      for (int u = 0; u < 32; ++u) y2r[cc + u] = __uint_as_float(a[u]);
    }
    sm100::tc_fence_before();
    __syncthreads();
  }
  if (tid == 0 && !*verr) {
    sm100::tc_fence_after();
    const uint64_t vdesc = sm100::smem_desc(sV, Gm::LBO, 1024, sm100::kSwizzle128);
#pragma unroll
    for (int kk = 0; kk < kC / 16; ++kk)
      sm100::mma_ts(tY1, tA + kk * 8, vdesc + (uint64_t)(kk * 2048 >> 4), IDESC_Y, kk > 0);
    sm100::mma_commit(&bars[1]);
  }
  if (!*verr && !sm100::mbar_wait(&bars[1], Gm::SHARE ? 0 : 1)) atomicOr(err, 1);
  sm100::tc_fence_after();

  // epilogue: y = Y1 + exp(G_i) Y2, fused (1 - mix) * gla_scale * RMSNorm(y); two passes over
  // 32-column chunks of TMEM (sum of squares, then the scaled store)
  const float eg = sm100::ex2_approx(G);
  float scale = 1.f;
  if (p.fuse) {
    float ss = 0.f;
#pragma unroll
    for (int cc = 0; cc < D; cc += 32) {
      uint32_t a[32], bb[32];
      sm100::tmem_ld32(tY1 + lane_off + cc, a);
      if (!Gm::SHARE) sm100::tmem_ld32(tY2 + lane_off + cc, bb);
      sm100::tc_wait_ld();
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const float y2 = Gm::SHARE ? y2r[cc + u] : __uint_as_float(bb[u]);
        const float y = fmaf(eg, y2, __uint_as_float(a[u]));
        ss = fmaf(y, y, ss);
      }
    }
    scale = rsqrtf(ss / (float)D + p.eps) * (1.f - mix);
  }
  const bool store = t < p.T && !*verr;
  T* yp = reinterpret_cast<T*>(p.y) + b * p.sy[0] + h * p.sy[1] + (int64_t)(store ? t : 0) * p.sy[2];
  const bool vec = p.sy[3] == 1 && (reinterpret_cast<uintptr_t>(yp) & 15u) == 0;
#pragma unroll
  for (int cc = 0; cc < D; cc += 32) {
    uint32_t a[32], bb[32];
    sm100::tmem_ld32(tY1 + lane_off + cc, a);  // warp-collective: every lane executes it
    if (!Gm::SHARE) sm100::tmem_ld32(tY2 + lane_off + cc, bb);
    sm100::tc_wait_ld();
    if (store) {
      float y[32];
#pragma unroll
      for (int u = 0; u < 32; ++u)
        y[u] = fmaf(eg, Gm::SHARE ? y2r[cc + u] : __uint_as_float(bb[u]), __uint_as_float(a[u])) * scale * sGS[cc + u];
      if (vec) {
#pragma unroll
        for (int d = 0; d < 32; d += 8) {
          uint4 w;
          w.x = pack2(y[d], y[d + 1], BF16);
          w.y = pack2(y[d + 2], y[d + 3], BF16);
          w.z = pack2(y[d + 4], y[d + 5], BF16);
          w.w = pack2(y[d + 6], y[d + 7], BF16);
          *reinterpret_cast<uint4*>(yp + cc + d) = w;
        }
      } else {
#pragma unroll
        for (int d = 0; d < 32; ++d) yp[(int64_t)(cc + d) * p.sy[3]] = from_f<T>(y[d]);
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (*err && tid == 0) atomicOr(&g_gla_tc_status, 1);
  if (warp == 0) sm100::tmem_dealloc(tmem, Gm::OUT_COLS);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// [B,H,T,D] operand map with a (64 channels x 128 tokens) box, 128-byte swizzle
bool make_map(CUtensorMap* m, const void* ptr, bool bf16, int64_t D, int64_t T, int64_t H, int64_t B, const int64_t* s) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0 || s[3] != 1) return false;
  const int64_t sb = B > 1 ? s[0] : 8, sh = H > 1 ? s[1] : 8;
  if (s[2] % 8 || sh % 8 || sb % 8 || s[2] <= 0 || sh <= 0 || sb <= 0) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)H, (cuuint64_t)B};  // channels past D read as 0
  cuuint64_t strides[3] = {(cuuint64_t)(s[2] * 2), (cuuint64_t)(sh * 2), (cuuint64_t)(sb * 2)};
  cuuint32_t box[4] = {64, (cuuint32_t)kC, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(ptr),
            dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T, int D>
cudaError_t launch_t(const GlaParams& p, cudaStream_t st, bool* taken) {
  using Gm = Geo<D>;
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, p.q, bf16, D, p.T, p.H, p.B, p.sq) || !make_map(&mk, p.k, bf16, D, p.T, p.H, p.B, p.sk) ||
      !make_map(&mv, p.v, bf16, D, p.T, p.H, p.B, p.sv))
    return cudaSuccess;
  auto kA = gla_tc_state_kernel<T, D>;
  auto kC_ = gla_tc_out_kernel<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kA, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Gm::STATE_SMEM);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kC_, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Gm::OUT_SMEM);
  if (e != cudaSuccess) return e;
  *taken = true;
  const dim3 grid(p.nseg, p.H, p.B);
  kA<<<grid, kThreads, Gm::STATE_SMEM, st>>>(mk, mv, p);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  gla_tc_scan_kernel<<<dim3((p.J * D + 255) / 256, p.H, p.B), 256, 0, st>>>(p);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  kC_<<<grid, kThreads, Gm::OUT_SMEM, st>>>(mq, mk, mv, p);
  return cudaGetLastError();
}

}  // namespace

// Workspace bytes of the tensor-core path (start states + chunk decays).
size_t gla_tc_workspace_bytes(int64_t B, int64_t H, int64_t T, int64_t J, int64_t D) {
  const int64_t nc = (T + kC - 1) / kC;
  return (size_t)(B * H * nc * (J * D + 1)) * sizeof(float) + 256;
}

bool gla_tc_eligible(const GlaParams& p, int dtype) {
  const char* off = getenv("HOFA_GLA_NO_TC");
  if (off != nullptr && off[0] != '\0' && off[0] != '0') return false;
  return (dtype == HOFA_DTYPE_BF16 || dtype == HOFA_DTYPE_F16) && (p.D == 64 || p.D == 128) && p.R % 8 == 0 &&
         p.R < p.D && p.log_alpha == nullptr;
}

// p.nseg must hold the chunk count ceil(T / 128), p.ws_state / p.ws_decay the
// tensor-core workspace layout.  *taken stays false when a tensor map cannot
// be built for these strides (the caller then uses the CUDA-core kernel).
cudaError_t launch_gla_tc(const GlaParams& p, int dtype, cudaStream_t st, bool* taken) {
  *taken = false;
  if (dtype == HOFA_DTYPE_BF16)
    return p.D == 64 ? launch_t<__nv_bfloat16, 64>(p, st, taken) : launch_t<__nv_bfloat16, 128>(p, st, taken);
  return p.D == 64 ? launch_t<__half, 64>(p, st, taken) : launch_t<__half, 128>(p, st, taken);
}

int gla_tc_chunk() { return kC; }

cudaError_t read_gla_tc_status(int* out, cudaStream_t st) {
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_gla_tc_status, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return e;
  const int zero = 0;
  e = cudaMemcpyToSymbolAsync(g_gla_tc_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return e;
  return cudaStreamSynchronize(st);
}

}  // namespace hofa
