// Prefill GLA on the tensor cores (tcgen05 + TMEM + TMA), chunk-parallel.
//
// Replaces chunk_gla_fwd_kernel (src/chunk_gla_inlier.py:5-150) for bf16/f16
// inputs with head dim 64 or 128, with a per-head scalar decay or a per-channel
// one (log_alpha: the ALPHA variants of A, B and C, described at C).
// Operand tiles are [128 tokens x D channels] in 64-channel column blocks of
// 128-byte swizzled rows (one TMA box each), so D = 128 uses two blocks.  The
// reference runs one program per (b,h) that walks every chunk in sequence; here
// every 128-token chunk of every (b,h) is its own CTA.  Head dim 64 runs the
// single launch F below (the chunk-to-chunk state carry done inside the launch
// by a decoupled look-back); head dim 128 runs three launches:
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
//   C  gla_tc_out_kernel     (one CTA per chunk c; at D = 64 -- the per-channel decay --
//                             Y2 and then Y1 reuse A's upper TMEM columns once P is
//                             formed: 128 columns)
//        A   = Q_I K_I^T            tcgen05.mma M=128, N=128, K=J (A/B K-major)
//        Y2  = Q_I start_c          tcgen05.mma M=128, N=D,   K=J (start_c as a bf16
//                                   MN-major operand)
//        P   = A * exp(G_i - G_j) [j <= i]  -> bf16, written back into TMEM
//        Y1  = P V                  tcgen05.mma, A = P from TMEM, V MN-major
//        y   = Y1 + exp(G_i) Y2, then (1 - mix) * gla_scale * RMSNorm(y)
//      with a per-channel decay (ALPHA) A is the reference's factored form over
//      key sub-blocks of 64 / 32 / 16 tokens (decayed Q and K as hi + lo terms),
//      P = A masked, Y2's operand Q exp(G_i a) and y = Y1 + Y2 (see the kernel);
//      A and B decay key channel c / state row j by exp(... a_c) / exp(G_C a_j)
//
// All decay factors of the scalar form are exponentials of non-positive
// differences of cumulative log decays (no overflow).  Rounding points: the masked score matrix and the
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
  static constexpr size_t STATE_SMEM = 3 * OP + 1024 + 256 + 4 * D;   // K (then Kd hi), V, Kd lo; alpha
  // D = 64: about 69 KB, three CTAs per SM; D = 128: one CTA
  static constexpr size_t OUT_SMEM = 4 * OP + 1024 + 4096 + 4 * D;
  // per-channel decay: two more tiles for the lo terms of the decayed Q and K
  // (D = 64: about 101 KB, two CTAs per SM)
  static constexpr size_t OUT_SMEM_ALPHA = 6 * OP + 1024 + 4096 + 4 * D;
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
template <typename T, int D, bool ALPHA>
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
  float* sAl = reinterpret_cast<float*>(base + 3 * Gm::OP + 256);  // alpha_c = exp(log_alpha_c) per inlier channel

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
  if constexpr (ALPHA) {
    for (int cc = tid; cc < D; cc += kThreads)
      sAl[cc] = cc < p.J ? __expf(ld_any(p.log_alpha, p.dt_la, b * p.sla[0] + h * p.sla[1] + cc * p.sla[2])) : 0.f;
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
  // With a per-channel decay (ALPHA) the factor is exp((G_C - G_t) alpha_c)
  // (src/chunk_gla_inlier.py:90-107), still <= 1.  With the rotated chunk order
  // the loop index q0 is the logical 16-byte chunk of the row (the 128-byte
  // swizzle stores logical chunk L of row r at L ^ (r & 7)), so its channels
  // are 64 nb + 8 q0 + [0, 8).
  {
    const float dG = (gc - G) * kLog2e;
    const float w = sm100::ex2_approx(dG);
    const int rot = tid & 7;  // chunk order q ^ (lane & 7): the warp's lanes spread over all banks
#pragma unroll
    for (int nb = 0; nb < Gm::NB; ++nb) {
      uint4* row = reinterpret_cast<uint4*>(sK + nb * kTile + tid * 128);
      uint4* lrow = reinterpret_cast<uint4*>(sL + nb * kTile + tid * 128);
#pragma unroll
      for (int q0 = 0; q0 < 8; ++q0) {
        const int q = q0 ^ rot;
        uint4 u = row[q], l;
        uint32_t* pu = reinterpret_cast<uint32_t*>(&u);
        uint32_t* pl = reinterpret_cast<uint32_t*>(&l);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float a, bb;
          if (BF16) bf16x2_to_f(pu[e], a, bb);
          else f16x2_to_f(pu[e], a, bb);
          float wa = w, wb = w;
          if constexpr (ALPHA) {
            const int ch = 64 * nb + 8 * q0 + 2 * e;
            wa = sm100::ex2_approx(dG * sAl[ch]);
            wb = sm100::ex2_approx(dG * sAl[ch + 1]);
          }
          const float xa = a * wa, xb = bb * wb;
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
  // row j of the state decays by exp(G_C alpha_j) per chunk (alpha = 1 without log_alpha)
  const float a2 = kLog2e * (p.log_alpha ? __expf(ld_any(p.log_alpha, p.dt_la, b * p.sla[0] + h * p.sla[1] + j * p.sla[2])) : 1.f);
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
      S = fmaf(sm100::ex2_approx(g[u] * a2), S, dS[u]);
    }
  }
  for (; c < p.nseg; ++c) {
    const float dS = ws[c * cs];
    ws[c * cs] = S;
    S = fmaf(sm100::ex2_approx(gc[c] * a2), S, dS);
  }
  if (p.state_out) p.state_out[b * p.sso[0] + h * p.sso[1] + j * p.sso[2] + d * p.sso[3]] = S;
}

// ---------------------------------------------------------------------------
// C: per-chunk output
// ---------------------------------------------------------------------------
template <typename T, int D, bool ALPHA>
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
  unsigned char* sQl = base + 4 * Gm::OP;             // ALPHA: lo terms of the decayed Q
  unsigned char* sKl = base + 5 * Gm::OP;             //        and of the decayed K
  float* sG = reinterpret_cast<float*>(base + (ALPHA ? 6 : 4) * Gm::OP);  // cumulative log2 decay per token
  float* sGS = sG + kC;                                // gla_scale[h, 0:D]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sGS + D);
  float* sm_warp = reinterpret_cast<float*>(bars + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm_warp + 4);
  int* err = reinterpret_cast<int*>(tmem_slot + 1);
  float* sAl = reinterpret_cast<float*>(err + 1);  // alpha_c = exp(log_alpha_c) (ALPHA)

  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int t0 = c * kC;
  const int bh = b * p.H + h;
  const int J = p.J, KS = (J + 15) / 16;
  if (tid == 0) {
    sm100::mbar_init(&bars[0], 1);
    sm100::mbar_init(&bars[1], 1);
    sm100::mbar_init(&bars[2], 1);
    *err = 0;
    sm100::fence_mbar_init();
  }
  if constexpr (ALPHA) {
    for (int cc = tid; cc < D; cc += kThreads)
      sAl[cc] = cc < J ? __expf(ld_any(p.log_alpha, p.dt_la, b * p.sla[0] + h * p.sla[1] + cc * p.sla[2])) : 0.f;
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
  if constexpr (ALPHA) {
    if (warp == 0) {  // largest alpha (sAl is complete: the scan above holds a barrier)
      float m = 0.f;
      for (int cc = tid; cc < D; cc += 32) m = fmaxf(m, sAl[cc]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (tid == 0) sAl[D] = m;
    }
  }
  fence_async_smem();
  volatile int* verr = err;
  if (!sm100::mbar_wait(&bars[0], 0)) atomicOr(err, 1);
  sm100::tc_fence_before();
  __syncthreads();
  // K-major steps of 16 channels: 4 per 128-byte block (32 B each), blocks kTile apart
  auto kstep = [](int ks) { return (uint64_t)(((ks >> 2) * kTile + (ks & 3) * 32) >> 4); };
  uint32_t ph1 = 0;  // completions of bars[1] waited for so far (its next parity)
  if constexpr (ALPHA) {
    // Per-channel decay: the reference's factored form (src/chunk_gla_inlier.py:
    // 90-107) over key sub-blocks of S tokens: for the keys of sub-block b (last
    // token e_b)
    //   A[:, b] = (Q exp((G_i - G_e_b) a)) (K exp((G_e_b - G_j) a))^T,  rows i before b zero.
    // Key factors are <= 1; query factors exceed 1 only within the key's own
    // sub-block, so S bounds the exponents: each CTA takes the largest S of 64
    // (the reference's chunk), 32 and 16 whose sub-blocks keep
    // (G_first - G_last) max(a) within the type's bound (log2 units), and runs kC / S
    // products of N = S.  Y2's operand is Q exp(G_i a) (<= 1).  Thread i keeps
    // its Q row in registers and rewrites Q's tile for each product; K is
    // decayed in place.  With the rotated chunk order index q0 is the logical
    // 16-byte chunk of the row (channels 64 nb + 8 q0 + [0, 8)).
    // A chunk whose 16-token sub-blocks still exceed that range (a decay of
    // more than about 2^-6 per token over 16 tokens) forms A exactly on the CUDA
    // cores instead (every A_ij = sum_c Q_ic K_jc exp((G_i - G_j) a_c), j <= i),
    // so the output stays finite where every factored form overflows.
    // The range bound is 2^100 for bf16 (range 2^+-126) and 2^10 for f16
    // (largest value 65504, smallest normal 2^-14).
    constexpr float kRange = BF16 ? 100.f : 10.f;
    const int i = tid, rot = tid & 7;
    const float Gi = sG[i], amax = sAl[D];
    int S = 0;
    for (int cand = 64; cand >= 16; cand >>= 1) {
      bool ok = true;
      for (int sb = 0; sb < kC / cand; ++sb) ok = ok && (sG[sb * cand] - sG[sb * cand + cand - 1]) * amax <= kRange;
      if (ok) {
        S = cand;
        break;
      }
    }
    uint4 qr[8 * Gm::NB];
#pragma unroll
    for (int nb = 0; nb < Gm::NB; ++nb)
#pragma unroll
      for (int q0 = 0; q0 < 8; ++q0) qr[nb * 8 + q0] = reinterpret_cast<const uint4*>(sQ + nb * kTile + i * 128)[q0 ^ rot];
    // x * exp2(dg a_c) as hi + lo 16-bit terms (hi = the rounded value, lo =
    // the rounded remainder), so that the products of the decayed operands
    // keep about 16 significant bits (three MMAs: hi*hi + hi*lo + lo*hi)
    // instead of the 8 of the reference's single rounding
    auto scaled = [&](uint4 u, int ch0, float dg, uint4& lo) {
      uint32_t pu[4] = {u.x, u.y, u.z, u.w}, pl[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float a, bb, ha, hb;
        if (BF16) bf16x2_to_f(pu[e], a, bb);
        else f16x2_to_f(pu[e], a, bb);
        a *= sm100::ex2_approx(dg * sAl[ch0 + 2 * e]);
        bb *= sm100::ex2_approx(dg * sAl[ch0 + 2 * e + 1]);
        pu[e] = pack2(a, bb, BF16);
        if (BF16) bf16x2_to_f(pu[e], ha, hb);
        else f16x2_to_f(pu[e], ha, hb);
        pl[e] = pack2(a - ha, bb - hb, BF16);
      }
      lo = make_uint4(pl[0], pl[1], pl[2], pl[3]);
      return make_uint4(pu[0], pu[1], pu[2], pu[3]);
    };
    auto write_q = [&](float dg, bool zero) {
#pragma unroll
      for (int nb = 0; nb < Gm::NB; ++nb)
#pragma unroll
        for (int q0 = 0; q0 < 8; ++q0) {
          uint4 hi = make_uint4(0u, 0u, 0u, 0u), lo = hi;
          if (!zero) hi = scaled(qr[nb * 8 + q0], 64 * nb + 8 * q0, dg, lo);
          reinterpret_cast<uint4*>(sQ + nb * kTile + i * 128)[q0 ^ rot] = hi;
          reinterpret_cast<uint4*>(sQl + nb * kTile + i * 128)[q0 ^ rot] = lo;
        }
    };
    if (S == 0) {
      // exact A on the CUDA cores from the unscaled Q row (registers) and K rows
      // (shared memory, logical chunk L of row j at L ^ (j & 7)), 32 columns at a time
#pragma unroll 1
      for (int cc = 0; cc < kC; cc += 32) {
        uint32_t out[32];
#pragma unroll 1
        for (int u = 0; u < 32; ++u) {
          const int j = cc + u;
          float acc = 0.f;
          if (j <= i) {
            const float dg = Gi - sG[j];
#pragma unroll
            for (int nb = 0; nb < Gm::NB; ++nb)
#pragma unroll
              for (int q0 = 0; q0 < 8; ++q0) {
                if (64 * nb + 8 * q0 >= J) continue;
                const uint4 kv = reinterpret_cast<const uint4*>(sK + nb * kTile + j * 128)[q0 ^ (j & 7)];
                const uint4 qv = qr[nb * 8 + q0];
                const uint32_t kk4[4] = {kv.x, kv.y, kv.z, kv.w}, qq4[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  float qa, qb, ka, kb;
                  if (BF16) {
                    bf16x2_to_f(qq4[e], qa, qb);
                    bf16x2_to_f(kk4[e], ka, kb);
                  } else {
                    f16x2_to_f(qq4[e], qa, qb);
                    f16x2_to_f(kk4[e], ka, kb);
                  }
                  const int ch = 64 * nb + 8 * q0 + 2 * e;
                  acc = fmaf(qa * ka, sm100::ex2_approx(dg * sAl[ch]), acc);
                  acc = fmaf(qb * kb, sm100::ex2_approx(dg * sAl[ch + 1]), acc);
                }
              }
          }
          out[u] = __float_as_uint(acc);
        }
        sm100::tmem_st32(tA + lane_off + cc, out);
      }
      sm100::tc_wait_st();
    } else {
      const float dk = sG[(i / S) * S + S - 1] - Gi;
#pragma unroll
      for (int nb = 0; nb < Gm::NB; ++nb)
#pragma unroll
        for (int q0 = 0; q0 < 8; ++q0) {
          uint4* kr = reinterpret_cast<uint4*>(sK + nb * kTile + i * 128);
          uint4 lo;
          kr[q0 ^ rot] = scaled(kr[q0 ^ rot], 64 * nb + 8 * q0, dk, lo);
          reinterpret_cast<uint4*>(sKl + nb * kTile + i * 128)[q0 ^ rot] = lo;
        }
    }
    const uint32_t idesc_s = sm100::idesc_f16(BF16, false, false, 128, S > 0 ? S : 16);
    for (int sb = 0; S > 0 && sb < kC / S; ++sb) {
      write_q(Gi - sG[sb * S + S - 1], i < sb * S);
      fence_async_smem();
      sm100::tc_fence_before();
      __syncthreads();
      if (tid == 0 && !*verr) {
        sm100::tc_fence_after();
        const uint64_t qdesc = sm100::smem_desc(sQ, 16, 1024, sm100::kSwizzle128);
        const uint64_t qldesc = sm100::smem_desc(sQl, 16, 1024, sm100::kSwizzle128);
        const uint64_t kdesc = sm100::smem_desc(sK + sb * S * 128, 16, 1024, sm100::kSwizzle128);
        const uint64_t kldesc = sm100::smem_desc(sKl + sb * S * 128, 16, 1024, sm100::kSwizzle128);
        for (int ks = 0; ks < KS; ++ks)
          sm100::mma_ss(tA + sb * S, qdesc + kstep(ks), kdesc + kstep(ks), idesc_s, ks > 0);
        for (int ks = 0; ks < KS; ++ks) sm100::mma_ss(tA + sb * S, qdesc + kstep(ks), kldesc + kstep(ks), idesc_s, true);
        for (int ks = 0; ks < KS; ++ks) sm100::mma_ss(tA + sb * S, qldesc + kstep(ks), kdesc + kstep(ks), idesc_s, true);
        sm100::mma_commit(&bars[2]);
      }
      if (!*verr && !sm100::mbar_wait(&bars[2], sb & 1)) atomicOr(err, 1);
      sm100::tc_fence_after();
    }
    write_q(Gi, false);
    fence_async_smem();
    if (!Gm::SHARE) {
      sm100::tc_fence_before();
      __syncthreads();
      if (tid == 0 && !*verr) {
        sm100::tc_fence_after();
        const uint64_t qdesc = sm100::smem_desc(sQ, 16, 1024, sm100::kSwizzle128);
        const uint64_t qldesc = sm100::smem_desc(sQl, 16, 1024, sm100::kSwizzle128);
        const uint64_t sdesc = sm100::smem_desc(sS, Gm::LBO, 1024, sm100::kSwizzle128);
        for (int ks = 0; ks < KS; ++ks)
          sm100::mma_ss(tY2, qdesc + kstep(ks), sdesc + (uint64_t)(ks * 2048 >> 4), IDESC_Y, ks > 0);
        for (int ks = 0; ks < KS; ++ks)
          sm100::mma_ss(tY2, qldesc + kstep(ks), sdesc + (uint64_t)(ks * 2048 >> 4), IDESC_Y, true);
        sm100::mma_commit(&bars[1]);
      }
      if (!*verr && !sm100::mbar_wait(&bars[1], ph1 & 1)) atomicOr(err, 1);
      ++ph1;
      sm100::tc_fence_after();
    }
  } else {
    if (tid == 0 && !*verr) {
      sm100::tc_fence_after();
      const uint64_t qdesc = sm100::smem_desc(sQ, 16, 1024, sm100::kSwizzle128);
      const uint64_t kdesc = sm100::smem_desc(sK, 16, 1024, sm100::kSwizzle128);
      const uint64_t sdesc = sm100::smem_desc(sS, Gm::LBO, 1024, sm100::kSwizzle128);
      for (int ks = 0; ks < KS; ++ks) sm100::mma_ss(tA, qdesc + kstep(ks), kdesc + kstep(ks), IDESC_A, ks > 0);
      if (!Gm::SHARE)
        for (int ks = 0; ks < KS; ++ks)
          sm100::mma_ss(tY2, qdesc + kstep(ks), sdesc + (uint64_t)(ks * 2048 >> 4), IDESC_Y, ks > 0);
      sm100::mma_commit(&bars[1]);
    }
    if (!*verr && !sm100::mbar_wait(&bars[1], ph1 & 1)) atomicOr(err, 1);
    ++ph1;
    sm100::tc_fence_after();
  }

  // P = A * exp(G_i - G_j) for j <= i, as 16-bit pairs over columns [0, 64)
  // (with ALPHA the decay is already inside A: P = A for j <= i)
  const int i = tid;
  auto dec = [&](int j) { return ALPHA ? 1.f : sm100::ex2_approx(G - sG[j]); };
#pragma unroll
  for (int cc = 0; cc < kC; cc += 64) {
    uint32_t r0[32], r1[32], pk[32];
    sm100::tmem_ld32(tA + lane_off + cc, r0);
    sm100::tmem_ld32(tA + lane_off + cc + 32, r1);
    sm100::tc_wait_ld();
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int j0 = cc + 2 * u, j1 = cc + 32 + 2 * u;
      const float a0 = j0 <= i ? __uint_as_float(r0[2 * u]) * dec(j0) : 0.f;
      const float a1 = j0 + 1 <= i ? __uint_as_float(r0[2 * u + 1]) * dec(j0 + 1) : 0.f;
      const float a2 = j1 <= i ? __uint_as_float(r1[2 * u]) * dec(j1) : 0.f;
      const float a3 = j1 + 1 <= i ? __uint_as_float(r1[2 * u + 1]) * dec(j1 + 1) : 0.f;
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
      for (int ks = 0; ks < KS; ++ks)
        sm100::mma_ss(tY2, qdesc + kstep(ks), sdesc + (uint64_t)(ks * 2048 >> 4), IDESC_Y, ks > 0);
      if constexpr (ALPHA) {  // lo term of Q exp(G_i a)
        const uint64_t qldesc = sm100::smem_desc(sQl, 16, 1024, sm100::kSwizzle128);
        for (int ks = 0; ks < KS; ++ks)
          sm100::mma_ss(tY2, qldesc + kstep(ks), sdesc + (uint64_t)(ks * 2048 >> 4), IDESC_Y, true);
      }
      sm100::mma_commit(&bars[1]);
    }
    if (!*verr && !sm100::mbar_wait(&bars[1], ph1 & 1)) atomicOr(err, 1);
    ++ph1;
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
  if (!*verr && !sm100::mbar_wait(&bars[1], ph1 & 1)) atomicOr(err, 1);
  sm100::tc_fence_after();

  // epilogue: y = Y1 + exp(G_i) Y2, fused (1 - mix) * gla_scale * RMSNorm(y); two passes over
  // 32-column chunks of TMEM (sum of squares, then the scaled store)
  const float eg = ALPHA ? 1.f : sm100::ex2_approx(G);  // ALPHA: the decay is inside Y2's operand
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

// ---------------------------------------------------------------------------
// F: single-launch form at head dim 64 (replaces A + B + C there)
//
// One CTA per chunk as in C, but the chunk comes from a ticket (atomic counter)
// handed out chunk-major over all (b,h), and the chunk-to-chunk state carry is
// done inside the launch by a decoupled look-back (Merrill and Garland, "Single-
// pass Parallel Prefix Scan with Decoupled Look-back", 2016):
//   1. dS_c = Kd^T V as in A (hi + lo terms), stored as the chunk's aggregate;
//      flag_c = AGG (release).  This needs nothing from other chunks.
//   2. start_c = sum over the chunks k < c back to the nearest one whose
//      inclusive state is published: exp(G_{k+1} + ... + G_{c-1}) * (dS_k, or
//      the inclusive state of the last one), or state_init when the walk
//      reaches the sequence start.  The multipliers are exponentials of sums
//      of non-positive chunk log decays.
//   3. inclusive_c = exp(G_C) start_c + dS_c; flag_c = INCL (release).
//   4. outputs as in C, with start_c as the bf16 operand of Y2.
// A CTA waits only for chunks with a lower ticket, which are resident and reach
// step 1 without waiting on anything, so every wait ends; each is bounded by
// wall time all the same, and a CTA that gives up publishes ERR, which its
// successors propagate instead of waiting.  DRAM traffic: Q, K, V read once, y
// written once; the per-chunk states live in L2 between publication and use.
//
// Four CTAs per SM: TMEM 128 columns each -- A = Q K^T in [0,128); P in
// [0,64); dS (M = 64) in [64,128), read out before Y1 = P V takes [64,128); Y2
// in [0,64) once Y1 has consumed P -- and three 16 KB tiles of shared memory:
// Q (then Kd lo, then Q again, reloaded by TMA for Y2), K (then Kd hi, then dS
// as fp32) and V (then start_c as the bf16 operand of Y2); at most 128
// registers per thread.
// ---------------------------------------------------------------------------
constexpr int kFlagAgg = 1, kFlagIncl = 2, kFlagErr = 3;
constexpr uint32_t kFusedCols = 128;
constexpr size_t kFusedSmem = 3 * (size_t)kTile + 1024 + 2048;

// flag word: state in the low 32 bits, the chunk's natural-log decay G_C (f32
// bits) in the high 32, so one acquire load returns both
__device__ __forceinline__ unsigned long long ld_acquire_gpu(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(unsigned long long* p, int state, float gc) {
  const unsigned long long v = ((unsigned long long)__float_as_uint(gc) << 32) | (unsigned)state;
  asm volatile("st.release.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

template <typename T, int NQ>
__global__ void __launch_bounds__(kThreads, 4)
gla_tc_fused_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, const GlaParams p) {
  constexpr int D = 64;
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC_A = sm100::idesc_f16(BF16, false, false, 128, 128);
  constexpr uint32_t IDESC_Y = sm100::idesc_f16(BF16, false, true, 128, D);
  constexpr uint32_t IDESC_S = sm100::idesc_f16(BF16, true, true, 64, D);
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = base;              // Q, then Kd lo, then Q again (reloaded)
  unsigned char* sK = base + kTile;      // K, then Kd hi, then dS as fp32
  unsigned char* sV = base + 2 * kTile;  // V, then start_c as the bf16 operand of Y2
  float* sG = reinterpret_cast<float*>(base + 3 * kTile);  // cumulative log2 decay per token
  float* sGS = sG + kC;                                     // gla_scale[h, 0:64]
  float* sPm = sGS + D;                                     // look-back plan: multipliers
  int* sPi = reinterpret_cast<int*>(sPm + 32);              //   and entries (4 * chunk + kind)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sPi + 32);
  float* sm_warp = reinterpret_cast<float*>(bars + 3);
  int* misc = reinterpret_cast<int*>(sm_warp + 4);  // tmem slot, err, ticket, plan size, plan final, plan valid
  float* sGC = reinterpret_cast<float*>(misc + 6);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (warp == 0) {
    sm100::tmem_alloc(reinterpret_cast<uint32_t*>(&misc[0]), kFusedCols);
    sm100::tmem_relinquish();
  }
  // the ticket is taken once the TMEM columns are held: a CTA that waits in the
  // allocation (for CTAs of another kernel on the SM) holds no place in the
  // chain that other chunks wait on
  if (tid == 0) {
    sm100::mbar_init(&bars[0], 1);
    sm100::mbar_init(&bars[1], 1);
    sm100::mbar_init(&bars[2], 1);
    misc[1] = 0;
    misc[2] = (int)atomicAdd(p.ws_ticket, 1u);
    misc[5] = 0;
    sm100::fence_mbar_init();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = static_cast<uint32_t>(misc[0]);
  const int BH = p.B * p.H;
  const int c = misc[2] / BH, bh = misc[2] % BH;
  const int b = bh / p.H, h = bh % p.H;
  const int t0 = c * kC;
  const int J = p.J, KS = (J + 15) / 16;
  const int64_t ci = (int64_t)bh * p.nseg + c;  // this chunk's slot in the workspace
  const int64_t chunk0 = (int64_t)bh * p.nseg;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  int* err = &misc[1];
  volatile int* verr = err;
  if (tid == 0) {
    sm100::mbar_arrive_expect_tx(&bars[0], 3 * kTile);
    sm100::tma_load_4d(sQ, &tq, p.R, t0, h, b, &bars[0]);
    sm100::tma_load_4d(sK, &tk, p.R, t0, h, b, &bars[0]);
    sm100::tma_load_4d(sV, &tv, 0, t0, h, b, &bars[0]);
  }
  const int t = t0 + tid;
  const float g = t < p.T ? ld_any(p.log_gamma, p.dt_lg, b * p.slg[0] + h * p.slg[1] + (int64_t)t * p.slg[2]) : 0.f;
  float mix = 0.f;
  if (p.fuse && t < p.T) mix = ld_any(p.mix_g, p.dt_mg, b * p.smg[0] + h * p.smg[1] + (int64_t)t * p.smg[2]);
  const float gsv = tid < D && p.fuse ? ld_any(p.gla_scale, p.dt_gs, h * p.sgs[0] + tid * p.sgs[1]) : 1.f;
  const float Gn = block_scan128(g, sm_warp, tid);  // natural log, inclusive over the chunk
  const float G = Gn * kLog2e;
  sG[tid] = G;
  if (tid == kThreads - 1) *sGC = Gn;
  if (tid < D) sGS[tid] = gsv;
  if (!sm100::mbar_wait(&bars[0], 0)) atomicOr(err, 1);
  sm100::tc_fence_before();
  __syncthreads();
  const float gc = *sGC;
  auto kstep = [](int ks) { return (uint64_t)((ks & 3) * 32 >> 4); };  // 16 channels in a 128-byte row
  if (tid == 0 && !*verr) {
    sm100::tc_fence_after();
    const uint64_t qdesc = sm100::smem_desc(sQ, 16, 1024, sm100::kSwizzle128);
    const uint64_t kdesc = sm100::smem_desc(sK, 16, 1024, sm100::kSwizzle128);
    for (int ks = 0; ks < KS; ++ks) sm100::mma_ss(tmem, qdesc + kstep(ks), kdesc + kstep(ks), IDESC_A, ks > 0);
    sm100::mma_commit(&bars[1]);
  }
  // Kd = K * exp(G_C - G_t) as hi + lo 16-bit terms (see A).  lo is formed in
  // registers while the A product runs; once it has read Q and K, hi goes over
  // K and lo over Q.  Lane l visits the 16-byte chunks of its row in the order
  // q ^ (l & 7), so the 32 lanes of a warp spread over all banks.
  const int rot = tid & 7;
  const float kw = sm100::ex2_approx((gc - Gn) * kLog2e);
  auto kd_hi = [&](uint32_t u, float& xa, float& xb) {
    float a, bb;
    if (BF16) bf16x2_to_f(u, a, bb);
    else f16x2_to_f(u, a, bb);
    xa = a * kw;
    xb = bb * kw;
    return pack2(xa, xb, BF16);
  };
  uint32_t klo[32];
  {
    const uint4* row = reinterpret_cast<const uint4*>(sK + tid * 128);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint4 u = row[q ^ rot];
      const uint32_t pu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float xa, xb, ha, hb;
        const uint32_t hi = kd_hi(pu[e], xa, xb);
        if (BF16) bf16x2_to_f(hi, ha, hb);
        else f16x2_to_f(hi, ha, hb);
        klo[4 * q + e] = pack2(xa - ha, xb - hb, BF16);
      }
    }
  }
  if (!*verr && !sm100::mbar_wait(&bars[1], 0)) atomicOr(err, 1);
  sm100::tc_fence_after();
  {
    uint4* row = reinterpret_cast<uint4*>(sK + tid * 128);
    uint4* qrow = reinterpret_cast<uint4*>(sQ + tid * 128);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint4 u = row[q ^ rot];
      float xa, xb;
      row[q ^ rot] = make_uint4(kd_hi(u.x, xa, xb), kd_hi(u.y, xa, xb), kd_hi(u.z, xa, xb), kd_hi(u.w, xa, xb));
      qrow[q ^ rot] = make_uint4(klo[4 * q], klo[4 * q + 1], klo[4 * q + 2], klo[4 * q + 3]);
    }
  }
  // P = A * exp(G_i - G_j) for j <= i, as 16-bit pairs over columns [0, 64),
  // 32 columns of A at a time
  const int i = tid;
#pragma unroll
  for (int cc = 0; cc < kC; cc += 32) {
    uint32_t r[32], pk[16];
    sm100::tmem_ld32(tmem + lane_off + cc, r);
    sm100::tc_wait_ld();
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int j0 = cc + 2 * u;
      const float a0 = j0 <= i ? __uint_as_float(r[2 * u]) * sm100::ex2_approx(G - sG[j0]) : 0.f;
      const float a1 = j0 + 1 <= i ? __uint_as_float(r[2 * u + 1]) * sm100::ex2_approx(G - sG[j0 + 1]) : 0.f;
      pk[u] = pack2(a0, a1, BF16);
    }
    sm100::tmem_st16(tmem + lane_off + cc / 2, pk);
  }
  sm100::tc_wait_st();
  fence_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  // dS = Kd^T V (M = 64 inlier rows, N = 64, K = 128 tokens) into columns [64, 128)
  if (tid == 0 && !*verr) {
    sm100::tc_fence_after();
    const uint64_t adesc = sm100::smem_desc(sK, 16, 1024, sm100::kSwizzle128);
    const uint64_t ldesc = sm100::smem_desc(sQ, 16, 1024, sm100::kSwizzle128);
    const uint64_t vdesc = sm100::smem_desc(sV, 16, 1024, sm100::kSwizzle128);
#pragma unroll
    for (int ks = 0; ks < kC / 16; ++ks)
      sm100::mma_ss(tmem + 64, adesc + (uint64_t)(ks * 2048 >> 4), vdesc + (uint64_t)(ks * 2048 >> 4), IDESC_S, ks > 0);
#pragma unroll
    for (int ks = 0; ks < kC / 16; ++ks)
      sm100::mma_ss(tmem + 64, ldesc + (uint64_t)(ks * 2048 >> 4), vdesc + (uint64_t)(ks * 2048 >> 4), IDESC_S, true);
    sm100::mma_commit(&bars[1]);
  }
  // look-back plan (warp 1): lanes read the flags of chunks k_hi - lane; every
  // chunk before the first one with a published inclusive state (or the
  // sequence start) enters with its aggregate, that one with its inclusive
  // state (or state_init), each with multiplier exp(sum of the log decays of
  // the aggregate entries before it, and of earlier rounds).  Without
  // may_wait, a plan that would need an unpublished aggregate is left invalid.
  const uint64_t t_start = sm100::globaltimer_ns();
  float logm = 0.f;
  auto plan_round = [&](int k_hi, bool may_wait) {
    const int kk = k_hi - lane;
    int fl = 0, s = 32;
    float gdk = 0.f;
    while (true) {
      if (kk >= 0) {
        const unsigned long long w = ld_acquire_gpu(&p.ws_flags[chunk0 + kk]);
        fl = (int)(unsigned)(w & 0xffffffffu);
        gdk = __uint_as_float((unsigned)(w >> 32));
      } else {
        fl = kFlagIncl;
      }
      const unsigned term = __ballot_sync(0xffffffffu, fl >= kFlagIncl);
      const unsigned none = __ballot_sync(0xffffffffu, fl == 0);
      s = term ? __ffs(term) - 1 : 32;
      const unsigned need = s == 32 ? 0xffffffffu : ((1u << s) - 1u);
      if ((none & need) == 0) break;
      if (!may_wait) return;
      int late = 0;
      if (lane == 0) late = sm100::globaltimer_ns() - t_start > 200000000ull;
      if (__shfl_sync(0xffffffffu, late, 0)) {
        s = -1;
        break;
      }
      __nanosleep(64);
    }
    if (s < 0 || (s < 32 && __shfl_sync(0xffffffffu, fl, s) == kFlagErr)) {
      if (lane == 0) {
        atomicOr(err, 1);
        misc[3] = 0;
        misc[4] = 1;
        misc[5] = 1;
      }
      return;
    }
    const float gd = lane < s ? gdk : 0.f;
    float pre = gd;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, pre, o);
      if (lane >= o) pre += y;
    }
    if (lane <= s) {
      const int kind = lane < s ? 0 : (kk >= 0 ? 1 : 2);  // aggregate, inclusive, state_init
      sPi[lane] = 4 * (kk >= 0 ? kk : 0) + kind;
      sPm[lane] = sm100::ex2_approx((logm + pre - gd) * kLog2e);
    }
    logm += __shfl_sync(0xffffffffu, pre, 31);
    if (lane == 0) {
      misc[3] = s < 32 ? s + 1 : 32;
      misc[4] = s < 32;
      misc[5] = 1;
    }
  };
  // a first plan while the dS product runs, taken only if nothing in it is missing
  if (warp == 1) plan_round(c - 1, false);
  if (!*verr && !sm100::mbar_wait(&bars[1], 1)) atomicOr(err, 1);
  sm100::tc_fence_after();
  // Q again for Y2 (its tile held Kd lo, which the dS product has read)
  bool reloading = false;
  if (tid == 0 && !*verr) {
    sm100::mbar_arrive_expect_tx(&bars[0], kTile);
    sm100::tma_load_4d(sQ, &tq, p.R, t0, h, b, &bars[0]);
    reloading = true;
  }
  // aggregate: dS rows (M = 64: row j in lane 32*(j/16) + j%16) into shared
  // memory over the K tile as fp32 [J][64], 16-byte chunk c of row j at
  // position c ^ (j & 15) (the row-owning lanes then spread over the banks);
  // from there to the workspace in coalesced slots
  float* sA = reinterpret_cast<float*>(sK);
  auto sa_at = [&](int j, int cq) { return sA + j * D + ((cq ^ (j & 15)) << 2); };
  {
    const int jr = 16 * warp + lane;
    const bool row_ok = lane < 16 && jr < J;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t r[32];
      sm100::tmem_ld32(tmem + 64 + lane_off + half * 32, r);
      sm100::tc_wait_ld();
      if (row_ok) {
#pragma unroll
        for (int u = 0; u < 32; u += 4)
          *reinterpret_cast<float4*>(sa_at(jr, (half * 32 + u) >> 2)) =
              make_float4(__uint_as_float(r[u]), __uint_as_float(r[u + 1]), __uint_as_float(r[u + 2]),
                          __uint_as_float(r[u + 3]));
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  const bool early_plan = misc[5] != 0;
  // Y1 = P V into columns [64, 128) (dS has been read out)
  if (tid == 0 && !*verr) {
    sm100::tc_fence_after();
    const uint64_t vdesc = sm100::smem_desc(sV, 16, 1024, sm100::kSwizzle128);
#pragma unroll
    for (int kk = 0; kk < kC / 16; ++kk)
      sm100::mma_ts(tmem + 64, tmem + kk * 8, vdesc + (uint64_t)(kk * 2048 >> 4), IDESC_Y, kk > 0);
    sm100::mma_commit(&bars[1]);
  }
  {
    float4* agg = reinterpret_cast<float4*>(p.ws_agg + ci * J * D);
    for (int f = tid; f < 16 * J; f += kThreads) agg[f] = *reinterpret_cast<const float4*>(sa_at(f >> 4, f & 15));
  }
  __syncthreads();
  // publication: a fence that waits for every store above, then the flag; left
  // to warp 3, off the paths of the MMA issue and of the look-back
  if (tid == 96) {
    __threadfence();
    st_release_gpu(&p.ws_flags[ci], *verr ? kFlagErr : kFlagAgg, gc);
  }

  // look-back for start_c: thread tid owns the float4 slots f = tid + 128 q of
  // the [J][64] state (16 per row); two planned entries per step, their loads
  // in flight together
  float4 acc[NQ];
#pragma unroll
  for (int q = 0; q < NQ; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
  const int nslot = 16 * J;
  auto src_of = [&](int code) {
    return reinterpret_cast<const float4*>(((code & 3) == 0 ? p.ws_agg : p.ws_incl) + (chunk0 + (code >> 2)) * J * D);
  };
  auto add_init = [&](float m) {
    if (p.state_init == nullptr) return;
    const float* s0 = p.state_init + b * p.ssi[0] + h * p.ssi[1];
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      const int f = tid + 128 * q;
      if (f < nslot) {
        const float* r = s0 + (f >> 4) * p.ssi[2] + (f & 15) * 4;
        acc[q].x = fmaf(m, r[0], acc[q].x);
        acc[q].y = fmaf(m, r[1], acc[q].y);
        acc[q].z = fmaf(m, r[2], acc[q].z);
        acc[q].w = fmaf(m, r[3], acc[q].w);
      }
    }
  };
  int k_hi = c - 1;
  bool first = true;
  while (true) {
    if (!(first && early_plan) && warp == 1) plan_round(k_hi, true);
    __syncthreads();
    const int n = misc[3];
    const bool fin = misc[4] != 0;
    for (int e = 0; e < n; e += 2) {
      const int c0 = sPi[e];
      const int c1 = e + 1 < n ? sPi[e + 1] : 2;  // a missing second entry reads as "state_init" with m = 0
      const float m0 = sPm[e];
      const float m1 = e + 1 < n ? sPm[e + 1] : 0.f;
      const bool g0 = (c0 & 3) != 2, g1 = (c1 & 3) != 2;
      const float4* p0 = src_of(g0 ? c0 : 0);
      const float4* p1 = src_of(g1 ? c1 : 0);
      float4 x0[NQ], x1[NQ];
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        const int f = tid + 128 * q;
        x0[q] = g0 && f < nslot ? __ldcg(p0 + f) : make_float4(0.f, 0.f, 0.f, 0.f);
        x1[q] = g1 && f < nslot ? __ldcg(p1 + f) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        acc[q].x = fmaf(m1, x1[q].x, fmaf(m0, x0[q].x, acc[q].x));
        acc[q].y = fmaf(m1, x1[q].y, fmaf(m0, x0[q].y, acc[q].y));
        acc[q].z = fmaf(m1, x1[q].z, fmaf(m0, x0[q].z, acc[q].z));
        acc[q].w = fmaf(m1, x1[q].w, fmaf(m0, x0[q].w, acc[q].w));
      }
      if (!g0) add_init(m0);
      if (!g1 && e + 1 < n) add_init(m1);
    }
    if (fin) break;
    k_hi -= 32;
    first = false;
    __syncthreads();  // warp 1 rewrites the plan next round
  }

  // Y1 complete: V's tile and P's columns are free.  inclusive_c = exp(G_C)
  // start_c + dS_c -> workspace (and the final state for the last chunk);
  // start_c -> V's tile as the bf16 operand of Y2 (rows j, 128-byte swizzled,
  // rows J .. 16*KS zero)
  if (!*verr && !sm100::mbar_wait(&bars[1], 0)) atomicOr(err, 1);
  sm100::tc_fence_after();
  const float egc = sm100::ex2_approx(gc * kLog2e);
  float* incl = p.ws_incl + ci * J * D;
  const bool last = c == p.nseg - 1 && p.state_out != nullptr;
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    const int f = tid + 128 * q;
    const int j = f >> 4, d0 = (f & 15) * 4;
    if (j < 16 * KS) {
      const float4 v = f < nslot ? acc[q] : make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<uint2*>(sV + j * 128 + (((d0 >> 3) ^ (j & 7)) << 4) + (d0 & 7) * 2) =
          make_uint2(pack2(v.x, v.y, BF16), pack2(v.z, v.w, BF16));
    }
    if (f < nslot) {
      const float4 a = *reinterpret_cast<const float4*>(sa_at(j, f & 15));
      const float4 o = make_float4(fmaf(egc, acc[q].x, a.x), fmaf(egc, acc[q].y, a.y), fmaf(egc, acc[q].z, a.z),
                                   fmaf(egc, acc[q].w, a.w));
      *reinterpret_cast<float4*>(incl + f * 4) = o;
      if (last) {
        float* so = p.state_out + b * p.sso[0] + h * p.sso[1] + j * p.sso[2] + d0 * p.sso[3];
        so[0] = o.x;
        so[p.sso[3]] = o.y;
        so[2 * p.sso[3]] = o.z;
        so[3 * p.sso[3]] = o.w;
      }
    }
  }
  fence_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  if (tid == 96) {
    __threadfence();
    st_release_gpu(&p.ws_flags[ci], *verr ? kFlagErr : kFlagIncl, gc);
  }
  // Y2 = Q_I start_c into [0, 64), once the reloaded Q has landed; on a
  // barrier of its own (a thread still on its way to an earlier wait must not
  // find bars[1] two phases ahead)
  // (a reload in flight is always waited for, so the CTA never leaves with a
  // copy into its shared memory outstanding)
  if (tid == 0 && reloading) {
    if (!sm100::mbar_wait(&bars[0], 1)) {
      atomicOr(err, 1);
    } else if (!*verr) {
      sm100::tc_fence_after();
      const uint64_t qdesc = sm100::smem_desc(sQ, 16, 1024, sm100::kSwizzle128);
      const uint64_t sdesc = sm100::smem_desc(sV, 16, 1024, sm100::kSwizzle128);
      for (int ks = 0; ks < KS; ++ks)
        sm100::mma_ss(tmem, qdesc + kstep(ks), sdesc + (uint64_t)(ks * 2048 >> 4), IDESC_Y, ks > 0);
      sm100::mma_commit(&bars[2]);
    }
  }
  if (!*verr && !sm100::mbar_wait(&bars[2], 0)) atomicOr(err, 1);
  sm100::tc_fence_after();

  // epilogue as in C: y = Y1 + exp(G_i) Y2, fused (1 - mix) * gla_scale * RMSNorm(y),
  // 16 columns of TMEM at a time
  const uint32_t tY1 = tmem + 64, tY2 = tmem;
  const float eg = sm100::ex2_approx(G);
  float scale = 1.f;
  if (p.fuse) {
    float ss = 0.f;
#pragma unroll
    for (int cc = 0; cc < D; cc += 16) {
      uint32_t a[16], bb[16];
      sm100::tmem_ld16(tY1 + lane_off + cc, a);
      sm100::tmem_ld16(tY2 + lane_off + cc, bb);
      sm100::tc_wait_ld();
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const float y = fmaf(eg, __uint_as_float(bb[u]), __uint_as_float(a[u]));
        ss = fmaf(y, y, ss);
      }
    }
    scale = rsqrtf(ss / (float)D + p.eps) * (1.f - mix);
  }
  const bool store = t < p.T && !*verr;
  T* yp = reinterpret_cast<T*>(p.y) + b * p.sy[0] + h * p.sy[1] + (int64_t)(store ? t : 0) * p.sy[2];
  const bool vec = p.sy[3] == 1 && (reinterpret_cast<uintptr_t>(yp) & 15u) == 0;
#pragma unroll
  for (int cc = 0; cc < D; cc += 16) {
    uint32_t a[16], bb[16];
    sm100::tmem_ld16(tY1 + lane_off + cc, a);  // warp-collective: every lane executes it
    sm100::tmem_ld16(tY2 + lane_off + cc, bb);
    sm100::tc_wait_ld();
    if (store) {
      float y[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) y[u] = fmaf(eg, __uint_as_float(bb[u]), __uint_as_float(a[u])) * scale * sGS[cc + u];
      if (vec) {
#pragma unroll
        for (int d = 0; d < 16; d += 8) {
          uint4 w;
          w.x = pack2(y[d], y[d + 1], BF16);
          w.y = pack2(y[d + 2], y[d + 3], BF16);
          w.z = pack2(y[d + 4], y[d + 5], BF16);
          w.w = pack2(y[d + 6], y[d + 7], BF16);
          *reinterpret_cast<uint4*>(yp + cc + d) = w;
        }
      } else {
#pragma unroll
        for (int d = 0; d < 16; ++d) yp[(int64_t)(cc + d) * p.sy[3]] = from_f<T>(y[d]);
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (*err && tid == 0) atomicOr(&g_gla_tc_status, 1);
  if (warp == 0) sm100::tmem_dealloc(tmem, kFusedCols);
}

// Workspace of the single-launch form: ticket counter, per-chunk flags and
// log decays, aggregates and inclusive states (byte offsets from the base).
struct FusedLayout {
  size_t flags, decay, agg, incl, total;
};
FusedLayout fused_layout(int64_t nch, int64_t J) {
  auto r256 = [](size_t x) { return (x + 255) / 256 * 256; };
  FusedLayout L;
  L.flags = 256;
  L.decay = L.flags + r256((size_t)nch * 8);
  L.agg = L.decay + r256((size_t)nch * 4);
  L.incl = L.agg + r256((size_t)nch * J * 64 * 4);
  L.total = L.incl + r256((size_t)nch * J * 64 * 4);
  return L;
}

// True when launch_gla_tc runs the single-launch form for `p` (the per-channel
// decay runs the three launches at every head dim).
bool gla_tc_single_launch(const GlaParams& p) { return p.D == 64 && p.log_alpha == nullptr; }

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
  if (gla_tc_single_launch(p)) {
    auto kF = p.J <= 48 ? gla_tc_fused_kernel<T, 6> : gla_tc_fused_kernel<T, 8>;
    cudaError_t e = cudaFuncSetAttribute(kF, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFusedSmem);
    if (e != cudaSuccess) return e;
    *taken = true;
    const int64_t nch = (int64_t)p.B * p.H * p.nseg;
    // ticket and flags start at zero in every call (one memset of the front of the workspace)
    e = cudaMemsetAsync(p.ws_ticket, 0, fused_layout(nch, p.J).decay, st);
    if (e != cudaSuccess) return e;
    kF<<<(unsigned)nch, kThreads, kFusedSmem, st>>>(mq, mk, mv, p);
    return cudaGetLastError();
  }
  const bool alpha = p.log_alpha != nullptr;
  auto kA = alpha ? gla_tc_state_kernel<T, D, true> : gla_tc_state_kernel<T, D, false>;
  auto kC_ = alpha ? gla_tc_out_kernel<T, D, true> : gla_tc_out_kernel<T, D, false>;
  cudaError_t e = cudaFuncSetAttribute(kA, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Gm::STATE_SMEM);
  if (e != cudaSuccess) return e;
  const size_t out_smem = alpha ? Gm::OUT_SMEM_ALPHA : Gm::OUT_SMEM;
  e = cudaFuncSetAttribute(kC_, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)out_smem);
  if (e != cudaSuccess) return e;
  *taken = true;
  const dim3 grid(p.nseg, p.H, p.B);
  kA<<<grid, kThreads, Gm::STATE_SMEM, st>>>(mk, mv, p);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  gla_tc_scan_kernel<<<dim3((p.J * D + 255) / 256, p.H, p.B), 256, 0, st>>>(p);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  kC_<<<grid, kThreads, out_smem, st>>>(mq, mk, mv, p);
  return cudaGetLastError();
}

}  // namespace

// Workspace bytes of the tensor-core path: at head dim 64 the single-launch
// form's layout, otherwise start states + chunk decays of the three-launch form.
size_t gla_tc_workspace_bytes(int64_t B, int64_t H, int64_t T, int64_t J, int64_t D) {
  const int64_t nc = (T + kC - 1) / kC;
  if (D == 64) return fused_layout(B * H * nc, J).total;
  return (size_t)(B * H * nc * (J * D + 1)) * sizeof(float) + 256;
}

// Points the workspace fields of `p` (B, H, J, D, nseg and log_alpha set) into
// `ws`: the single-launch layout or the three-launch one, as the launch will
// use.  (gla_tc_workspace_bytes covers both at head dim 64.)
void gla_tc_bind_workspace(GlaParams& p, void* ws) {
  unsigned char* base = reinterpret_cast<unsigned char*>(ws);
  if (gla_tc_single_launch(p)) {
    const FusedLayout L = fused_layout((int64_t)p.B * p.H * p.nseg, p.J);
    p.ws_ticket = reinterpret_cast<unsigned*>(base);
    p.ws_flags = reinterpret_cast<unsigned long long*>(base + L.flags);
    p.ws_decay = reinterpret_cast<float*>(base + L.decay);
    p.ws_agg = reinterpret_cast<float*>(base + L.agg);
    p.ws_incl = reinterpret_cast<float*>(base + L.incl);
    p.ws_state = nullptr;
    return;
  }
  p.ws_state = reinterpret_cast<float*>(ws);
  p.ws_decay = p.ws_state + (size_t)p.B * p.H * p.nseg * p.J * p.D;
}

bool gla_tc_eligible(const GlaParams& p, int dtype) {
  const char* off = getenv("HOFA_GLA_NO_TC");
  if (off != nullptr && off[0] != '\0' && off[0] != '0') return false;
  return (dtype == HOFA_DTYPE_BF16 || dtype == HOFA_DTYPE_F16) && (p.D == 64 || p.D == 128) && p.R % 8 == 0 &&
         p.R < p.D;
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
