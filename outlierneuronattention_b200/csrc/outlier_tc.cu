// Tensor-core outlier attention for sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces the reference's Triton kernel _fwd_kernel (src/exact_attention.py:
// 45-161): out += mix * softmax(sm_scale * q_r k_r^T, causal) v with r = R
// query/key channels and D value channels.  One CTA of 128 threads owns 128
// query rows of one (b,h); thread i owns row i, which is TMEM lane i.  Keys
// come in tiles of 64, so S/P (64 columns) and O (64 columns at head dim 64)
// fit in 128 TMEM columns and three to four CTAs share an SM.
//
//   TMA (4-D tiled maps over [B,H,T,channels], no multicast) brings the Q
//   tile once and K/V tiles of 128 keys into a two-stage shared-memory ring.
//   Q/K tiles are K-major with R*2-byte swizzled rows; V tiles are MN-major
//   with 128-byte swizzled rows (as stored in memory), so no transposition.
//   Per key tile:
//     S   = Q K^T            tcgen05.mma kind::f16, A/B from shared memory,
//                             fp32 accumulator in TMEM columns [0, 64)
//     P   = exp2(S*c - m)    every thread reads its row of S from TMEM in one
//                             round trip (row max, then exponentials), writes
//                             P as bf16/f16 pairs over columns [0, 32)
//     O  += P V              tcgen05.mma with A = P from TMEM, B = V from
//                             shared memory, fp32 accumulator in TMEM
//                             columns [64, 64 + D)
//   The running max is only raised when a row's max grows by more than 2^8
//   (then the row of O is rescaled in TMEM); otherwise P is formed against the
//   stale max, which changes nothing but the common factor removed at the end.
//
// Every mbarrier wait is bounded; on a timeout the CTA records an error in
// g_outlier_tc_status, skips the rest of its work, frees its TMEM and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace hofa {

__device__ int g_outlier_tc_status;

namespace {

constexpr int kRows = 128;        // query rows per CTA (TMEM lanes)
constexpr int kKeys = 64;         // keys per tile
constexpr int kThreads = 128;

// TMEM columns: S / P in [0, kKeys), O in [kKeys, kKeys + D), rounded up to a power of two
template <int D>
constexpr uint32_t tmem_cols() { return kKeys + D <= 128 ? 128 : 256; }

template <int D, int R>
constexpr size_t smem_bytes() {
  constexpr size_t q = ((size_t)kRows * R * 2 + 1023) & ~size_t(1023);
  constexpr size_t k = ((size_t)kKeys * R * 2 + 1023) & ~size_t(1023);
  constexpr size_t v = (size_t)kKeys * D * 2;
  return 1024 + q + 2 * k + 2 * v + 64;
}

constexpr uint32_t swizzle_mode(int row_bytes) {
  return row_bytes == 32 ? sm100::kSwizzle32 : (row_bytes == 64 ? sm100::kSwizzle64 : sm100::kSwizzle128);
}

__device__ __forceinline__ uint32_t pack2(float a, float b, bool bf16) {
  if (bf16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <typename T, int D, int R>
__global__ void __launch_bounds__(kThreads, D == 64 ? 4 : 2)
outlier_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, const OutlierParams p) {
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int RB = R * 2;                       // bytes per Q/K row
  constexpr uint32_t Q_BYTES = kRows * RB;
  constexpr uint32_t K_BYTES = kKeys * RB;
  constexpr uint32_t V_BYTES = kKeys * D * 2;
  constexpr uint32_t Q_SLOT = (Q_BYTES + 1023) & ~1023u;
  constexpr uint32_t K_SLOT = (K_BYTES + 1023) & ~1023u;
  constexpr uint32_t SWZ = swizzle_mode(RB);
  constexpr uint32_t IDESC_S = sm100::idesc_f16(BF16, false, false, kRows, kKeys);
  constexpr uint32_t IDESC_O = sm100::idesc_f16(BF16, false, true, kRows, D);
  constexpr uint32_t NCOLS = tmem_cols<D>();

  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = base;
  unsigned char* const sK0 = base + Q_SLOT;                  // slot st at sK0 + st * K_SLOT
  unsigned char* const sV0 = base + Q_SLOT + 2 * K_SLOT;     // slot st at sV0 + st * V_BYTES
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + Q_SLOT + 2 * K_SLOT + 2 * V_BYTES);
  uint64_t* bar_q = bars + 0;
  uint64_t* bar_kv = bars + 1;  // [2]
  uint64_t* bar_s = bars + 3;
  uint64_t* bar_o = bars + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6);
  int* err_flag = reinterpret_cast<int*>(bars + 7);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int nqb = (p.Tq + kRows - 1) / kRows;
  const int qb = nqb - 1 - (int)blockIdx.x;     // long causal rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int q0 = qb * kRows;
  const int last_key = min(p.Tk - 1, q0 + kRows - 1 + p.q_offset);
  const int ntiles = last_key / kKeys + 1;

  if (tid == 0) {
    sm100::mbar_init(bar_q, 1);
    sm100::mbar_init(&bar_kv[0], 1);
    sm100::mbar_init(&bar_kv[1], 1);
    sm100::mbar_init(bar_s, 1);
    sm100::mbar_init(bar_o, 1);
    *err_flag = 0;
    sm100::fence_mbar_init();
    sm100::prefetch_tmap(&tq);
    sm100::prefetch_tmap(&tk);
    sm100::prefetch_tmap(&tv);
  }
  if (warp == 0) {
    sm100::tmem_alloc(tmem_slot, NCOLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + kKeys;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;

  auto load_kv = [&](int j, int st) {
    sm100::mbar_arrive_expect_tx(&bar_kv[st], K_BYTES + V_BYTES);
    sm100::tma_load_4d(sK0 + st * K_SLOT, &tk, 0, j * kKeys, h, b, &bar_kv[st]);
#pragma unroll
    for (int g = 0; g < D / 64; ++g)
      sm100::tma_load_4d(sV0 + st * V_BYTES + g * kKeys * 128, &tv, g * 64, j * kKeys, h, b, &bar_kv[st]);
  };
  if (tid == 0) {
    sm100::mbar_arrive_expect_tx(bar_q, Q_BYTES);
    sm100::tma_load_4d(sQ, &tq, 0, q0, h, b, bar_q);
    load_kv(0, 0);
  }

  const float scale = p.qk_scale_log2;
  const int row = q0 + tid;
  const int limit = min(row + p.q_offset, p.Tk - 1);   // last visible key of this row
  float m_used = -INFINITY, l_sum = 0.f;
  // Bounded waits; after the first timeout in the CTA every later wait and
  // MMA / copy issue is skipped, while the loop keeps its uniform trip count
  // so that barriers and warp-collective TMEM accesses stay convergent.
  volatile int* verr = err_flag;
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (*verr) return;
    if (!sm100::mbar_wait(bar, parity)) atomicOr(err_flag, 1);
  };
  wait(bar_q, 0);

  const uint64_t qdesc = sm100::smem_desc(sQ, 16, 8 * RB, SWZ);
  for (int j = 0; j < ntiles; ++j) {
    const int st = j & 1;
    if (tid == 0 && j + 1 < ntiles && !*verr) load_kv(j + 1, st ^ 1);
    wait(&bar_kv[st], (j >> 1) & 1);
    if (tid == 0 && !*verr) {
      sm100::tc_fence_after();
      const uint64_t kdesc = sm100::smem_desc(sK0 + st * K_SLOT, 16, 8 * RB, SWZ);
#pragma unroll
      for (int ks = 0; ks < R / 16; ++ks) sm100::mma_ss(tS, qdesc + 2 * ks, kdesc + 2 * ks, IDESC_S, ks > 0);
      sm100::mma_commit(bar_s);
    }
    wait(bar_s, j & 1);
    sm100::tc_fence_after();

    // ---- the row's 64 scores of this tile, one TMEM round trip ------------
    uint32_t r0[32], r1[32];
    sm100::tmem_ld32(tS + lane_off, r0);
    sm100::tmem_ld32(tS + lane_off + 32, r1);
    sm100::tc_wait_ld();
    const int k0 = j * kKeys;
    const bool masked = k0 + kKeys - 1 > q0 + p.q_offset || k0 + kKeys > p.Tk;
    if (masked) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (k0 + i > limit) r0[i] = __float_as_uint(-INFINITY);
        if (k0 + 32 + i > limit) r1[i] = __float_as_uint(-INFINITY);
      }
    }
    float mt = -INFINITY;
#pragma unroll
    for (int i = 0; i < 32; ++i) mt = fmaxf(mt, fmaxf(__uint_as_float(r0[i]), __uint_as_float(r1[i])));
    const float mts = mt * scale;
    const bool raise = mts > m_used + 8.f;
    const float factor = raise ? exp2f(m_used - mts) : 1.f;  // 0 on the first tile
    l_sum *= factor;
    if (raise) m_used = mts;
    // TMEM loads/stores are warp-collective: the whole warp rescales its rows
    // of O when any of them raised its max (the others multiply by 1)
    if (j > 0 && __any_sync(0xffffffffu, raise)) {
#pragma unroll
      for (int c = 0; c < D; c += 16) {
        uint32_t r[16];
        sm100::tmem_ld16(tO + lane_off + c, r);
        sm100::tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * factor);
        sm100::tmem_st16(tO + lane_off + c, r);
      }
    }
    // ---- P = exp2(s*scale - m) as 16-bit pairs over columns [0, 32), written
    // in two halves of 16 columns to keep the register count low
    float ls = 0.f;
    {
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float e0 = exp2f(fmaf(__uint_as_float(r0[2 * i]), scale, -m_used));
        const float e1 = exp2f(fmaf(__uint_as_float(r0[2 * i + 1]), scale, -m_used));
        ls += e0 + e1;
        pk[i] = pack2(e0, e1, BF16);
      }
      sm100::tmem_st16(tS + lane_off, pk);
    }
    {
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float e2 = exp2f(fmaf(__uint_as_float(r1[2 * i]), scale, -m_used));
        const float e3 = exp2f(fmaf(__uint_as_float(r1[2 * i + 1]), scale, -m_used));
        ls += e2 + e3;
        pk[i] = pack2(e2, e3, BF16);
      }
      sm100::tmem_st16(tS + lane_off + 16, pk);
    }
    l_sum += ls;
    sm100::tc_wait_st();
    sm100::tc_fence_before();
    __syncthreads();
    if (tid == 0 && !*verr) {
      sm100::tc_fence_after();
      const uint64_t vdesc = sm100::smem_desc(sV0 + st * V_BYTES, kKeys * 128, 1024, sm100::kSwizzle128);
#pragma unroll
      for (int kk = 0; kk < kKeys / 16; ++kk)
        sm100::mma_ts(tO, tS + kk * 8, vdesc + (uint64_t)(kk * 2048 >> 4), IDESC_O, j > 0 || kk > 0);
      sm100::mma_commit(bar_o);
    }
    wait(bar_o, j & 1);
    sm100::tc_fence_after();
  }

  // ---- epilogue: out = (accumulate ? out : 0) + mix * O / l ----------------
  const bool store = row < p.Tq && !*verr;
  const float mix = store ? ld_any(p.mix_g, p.dt_mg, b * p.smg[0] + h * p.smg[1] + (int64_t)row * p.smg[2]) : 0.f;
  const float inv = l_sum > 0.f ? mix / l_sum : 0.f;
  T* og = reinterpret_cast<T*>(p.out) + b * p.so[0] + h * p.so[1] + (int64_t)(store ? row : 0) * p.so[2];
#pragma unroll
  for (int c = 0; c < D; c += 16) {
    uint32_t r[16];
    sm100::tmem_ld16(tO + lane_off + c, r);  // warp-collective: every lane executes it
    sm100::tc_wait_ld();
    if (store) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int64_t off = (int64_t)(c + i) * p.so[3];
        float o = __uint_as_float(r[i]) * inv;
        if (p.accumulate) o += to_f(og[off]);
        og[off] = from_f<T>(o);
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (*err_flag && tid == 0) atomicOr(&g_outlier_tc_status, 1);
  if (warp == 0) sm100::tmem_dealloc(tmem, NCOLS);
}

// ---------------------------------------------------------------------------
// Pipelined variant for head dim 64: three S/P buffers in TMEM and a 4-deep
// K/V ring let the tensor core run one tile ahead of the softmax:
//   iteration j:  [issuer] S_{j+1} = Q K_{j+1}^T into buffer (j+1)%3
//                 softmax of S_j -> P_j in buffer j%3
//                 [issuer] O += P_j V_j; K/V of tile j+3 -> ring slot (j+3)%4
// so neither MMA round trip sits on the softmax's critical path.  Every MMA
// group commits to its own buffer's mbarrier, so a parity wait never spans
// more than one phase.
// ---------------------------------------------------------------------------
template <typename T, int R>
__global__ void __launch_bounds__(kThreads, 2)
outlier_tc_pipe_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                       const __grid_constant__ CUtensorMap tv, const OutlierParams p) {
  constexpr int D = 64;
  constexpr int NKV = 4, NS = 3;
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int RB = R * 2;
  constexpr uint32_t Q_BYTES = kRows * RB;
  constexpr uint32_t K_BYTES = kKeys * RB;
  constexpr uint32_t V_BYTES = kKeys * D * 2;
  constexpr uint32_t Q_SLOT = (Q_BYTES + 1023) & ~1023u;
  constexpr uint32_t K_SLOT = (K_BYTES + 1023) & ~1023u;
  constexpr uint32_t SWZ = swizzle_mode(RB);
  constexpr uint32_t IDESC_S = sm100::idesc_f16(BF16, false, false, kRows, kKeys);
  constexpr uint32_t IDESC_O = sm100::idesc_f16(BF16, false, true, kRows, D);
  constexpr uint32_t NCOLS = 256;
  constexpr uint32_t COL_O = NS * kKeys;

  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = base;
  unsigned char* sK0 = base + Q_SLOT;
  unsigned char* sV0 = sK0 + NKV * K_SLOT;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV0 + NKV * V_BYTES);
  uint64_t* bar_q = bars;
  uint64_t* bar_kv = bars + 1;            // [NKV]
  uint64_t* bar_s = bar_kv + NKV;         // [NS]
  uint64_t* bar_o = bar_s + NS;           // [NS]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_o + NS);
  int* err_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int nqb = (p.Tq + kRows - 1) / kRows;
  const int qb = nqb - 1 - (int)blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int q0 = qb * kRows;
  const int last_key = min(p.Tk - 1, q0 + kRows - 1 + p.q_offset);
  const int n = last_key / kKeys + 1;

  if (tid == 0) {
    sm100::mbar_init(bar_q, 1);
    for (int i = 0; i < NKV; ++i) sm100::mbar_init(&bar_kv[i], 1);
    for (int i = 0; i < NS; ++i) { sm100::mbar_init(&bar_s[i], 1); sm100::mbar_init(&bar_o[i], 1); }
    *err_flag = 0;
    sm100::fence_mbar_init();
    sm100::prefetch_tmap(&tq);
    sm100::prefetch_tmap(&tk);
    sm100::prefetch_tmap(&tv);
  }
  if (warp == 0) {
    sm100::tmem_alloc(tmem_slot, NCOLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + COL_O;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  volatile int* verr = err_flag;
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (*verr) return;
    if (!sm100::mbar_wait(bar, parity)) atomicOr(err_flag, 1);
  };
  auto load_kv = [&](int t) {
    const int st = t % NKV;
    sm100::mbar_arrive_expect_tx(&bar_kv[st], K_BYTES + V_BYTES);
    sm100::tma_load_4d(sK0 + st * K_SLOT, &tk, 0, t * kKeys, h, b, &bar_kv[st]);
    sm100::tma_load_4d(sV0 + st * V_BYTES, &tv, 0, t * kKeys, h, b, &bar_kv[st]);
  };
  const uint64_t qdesc = sm100::smem_desc(sQ, 16, 8 * RB, SWZ);
  auto issue_s = [&](int t) {  // S_t -> buffer t % NS
    const uint64_t kdesc = sm100::smem_desc(sK0 + (t % NKV) * K_SLOT, 16, 8 * RB, SWZ);
#pragma unroll
    for (int ks = 0; ks < R / 16; ++ks)
      sm100::mma_ss(tmem + (t % NS) * kKeys, qdesc + 2 * ks, kdesc + 2 * ks, IDESC_S, ks > 0);
    sm100::mma_commit(&bar_s[t % NS]);
  };
  if (tid == 0) {
    sm100::mbar_arrive_expect_tx(bar_q, Q_BYTES);
    sm100::tma_load_4d(sQ, &tq, 0, q0, h, b, bar_q);
    for (int t = 0; t < 3 && t < n; ++t) load_kv(t);
    wait(bar_q, 0);
    wait(&bar_kv[0], 0);
    if (!*verr) {
      sm100::tc_fence_after();
      issue_s(0);
    }
  }

  const float scale = p.qk_scale_log2;
  const int row = q0 + tid;
  const int limit = min(row + p.q_offset, p.Tk - 1);
  float m_used = -INFINITY, l_sum = 0.f;

  for (int j = 0; j < n; ++j) {
    // ---- issuer: S_{j+1} into buffer (j+1)%3 (its last reader PV_{j-2} done) --
    if (tid == 0 && j + 1 < n && !*verr) {
      if (j >= 2) wait(&bar_o[(j - 2) % NS], ((j - 2) / NS) & 1);
      wait(&bar_kv[(j + 1) % NKV], ((j + 1) / NKV) & 1);
      if (!*verr) {
        sm100::tc_fence_after();
        issue_s(j + 1);
      }
    }
    // ---- softmax of S_j ------------------------------------------------------
    wait(&bar_s[j % NS], (j / NS) & 1);
    sm100::tc_fence_after();
    const uint32_t tS = tmem + (j % NS) * kKeys;
    uint32_t r0[32], r1[32];
    sm100::tmem_ld32(tS + lane_off, r0);
    sm100::tmem_ld32(tS + lane_off + 32, r1);
    sm100::tc_wait_ld();
    const int k0 = j * kKeys;
    const bool masked = k0 + kKeys - 1 > q0 + p.q_offset || k0 + kKeys > p.Tk;
    if (masked) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (k0 + i > limit) r0[i] = __float_as_uint(-INFINITY);
        if (k0 + 32 + i > limit) r1[i] = __float_as_uint(-INFINITY);
      }
    }
    float mt = -INFINITY;
#pragma unroll
    for (int i = 0; i < 32; ++i) mt = fmaxf(mt, fmaxf(__uint_as_float(r0[i]), __uint_as_float(r1[i])));
    const float mts = mt * scale;
    const bool raise = mts > m_used + 8.f;
    const float factor = raise ? exp2f(m_used - mts) : 1.f;
    l_sum *= factor;
    if (raise) m_used = mts;
    if (j > 0 && __any_sync(0xffffffffu, raise)) {
      wait(&bar_o[(j - 1) % NS], ((j - 1) / NS) & 1);  // O is stable once PV_{j-1} is done
      sm100::tc_fence_after();
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        uint32_t r[32];
        sm100::tmem_ld32(tO + lane_off + c, r);
        sm100::tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * factor);
        sm100::tmem_st32(tO + lane_off + c, r);
      }
    }
    uint32_t pk[32];
    float ls = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float e0 = exp2f(fmaf(__uint_as_float(r0[2 * i]), scale, -m_used));
      const float e1 = exp2f(fmaf(__uint_as_float(r0[2 * i + 1]), scale, -m_used));
      const float e2 = exp2f(fmaf(__uint_as_float(r1[2 * i]), scale, -m_used));
      const float e3 = exp2f(fmaf(__uint_as_float(r1[2 * i + 1]), scale, -m_used));
      ls += (e0 + e1) + (e2 + e3);
      pk[i] = pack2(e0, e1, BF16);
      pk[16 + i] = pack2(e2, e3, BF16);
    }
    l_sum += ls;
    sm100::tmem_st32(tS + lane_off, pk);
    sm100::tc_wait_st();
    sm100::tc_fence_before();
    __syncthreads();
    // ---- issuer: O += P_j V_j; next K/V load into the slot PV_{j-1} freed ----
    if (tid == 0 && !*verr) {
      sm100::tc_fence_after();
      const uint64_t vdesc = sm100::smem_desc(sV0 + (j % NKV) * V_BYTES, kKeys * 128, 1024, sm100::kSwizzle128);
#pragma unroll
      for (int kk = 0; kk < kKeys / 16; ++kk)
        sm100::mma_ts(tO, tS + kk * 8, vdesc + (uint64_t)(kk * 2048 >> 4), IDESC_O, j > 0 || kk > 0);
      sm100::mma_commit(&bar_o[j % NS]);
      if (j + 3 < n) {
        if (j >= 1) wait(&bar_o[(j - 1) % NS], ((j - 1) / NS) & 1);
        if (!*verr) load_kv(j + 3);
      }
    }
  }
  wait(&bar_o[(n - 1) % NS], ((n - 1) / NS) & 1);
  sm100::tc_fence_after();

  const bool store = row < p.Tq && !*verr;
  const float mix = store ? ld_any(p.mix_g, p.dt_mg, b * p.smg[0] + h * p.smg[1] + (int64_t)row * p.smg[2]) : 0.f;
  const float inv = l_sum > 0.f ? mix / l_sum : 0.f;
  T* og = reinterpret_cast<T*>(p.out) + b * p.so[0] + h * p.so[1] + (int64_t)(store ? row : 0) * p.so[2];
#pragma unroll
  for (int c = 0; c < D; c += 32) {
    uint32_t r[32];
    sm100::tmem_ld32(tO + lane_off + c, r);
    sm100::tc_wait_ld();
    if (store) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int64_t off = (int64_t)(c + i) * p.so[3];
        float o = __uint_as_float(r[i]) * inv;
        if (p.accumulate) o += to_f(og[off]);
        og[off] = from_f<T>(o);
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (*err_flag && tid == 0) atomicOr(&g_outlier_tc_status, 1);
  if (warp == 0) sm100::tmem_dealloc(tmem, NCOLS);
}

template <int R>
constexpr size_t pipe_smem_bytes() {
  constexpr size_t q = ((size_t)kRows * R * 2 + 1023) & ~size_t(1023);
  constexpr size_t k = ((size_t)kKeys * R * 2 + 1023) & ~size_t(1023);
  return 1024 + q + 4 * k + 4 * (size_t)kKeys * 64 * 2 + 128;
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

// 4-D map over [B, H, T, C] (dims innermost first: channels, T, H, B) with a
// (box_c x 128 x 1 x 1) box.
bool make_map(CUtensorMap* m, const void* ptr, bool bf16, int64_t C, int64_t T, int64_t H, int64_t B,
              const int64_t* stride, int box_c, int box_rows, CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[4] = {(cuuint64_t)C, (cuuint64_t)T, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(stride[2] * 2), (cuuint64_t)(stride[1] * 2), (cuuint64_t)(stride[0] * 2)};
  cuuint32_t box[4] = {(cuuint32_t)box_c, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool tma_ok(const void* ptr, const int64_t* s, int64_t B, int64_t H) {
  if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0 || s[3] != 1) return false;
  if (s[2] % 8 != 0 || s[2] <= 0) return false;
  if (H > 1 && (s[1] % 8 != 0 || s[1] <= 0)) return false;
  if (B > 1 && (s[0] % 8 != 0 || s[0] <= 0)) return false;
  return true;
}

template <typename T, int D, int R>
cudaError_t launch_dr(const OutlierParams& p, cudaStream_t st, bool* taken) {
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  // size-1 batch/head dims get a harmless legal stride
  int64_t sq[4] = {p.B > 1 ? p.sq[0] : 8, p.H > 1 ? p.sq[1] : 8, p.sq[2], p.sq[3]};
  int64_t sk[4] = {p.B > 1 ? p.sk[0] : 8, p.H > 1 ? p.sk[1] : 8, p.sk[2], p.sk[3]};
  int64_t sv[4] = {p.B > 1 ? p.sv[0] : 8, p.H > 1 ? p.sv[1] : 8, p.sv[2], p.sv[3]};
  if (!tma_ok(p.q, sq, p.B, p.H) || !tma_ok(p.k, sk, p.B, p.H) || !tma_ok(p.v, sv, p.B, p.H)) return cudaSuccess;
  CUtensorMap mq, mk, mv;
  const CUtensorMapSwizzle qk_swz = R == 16 ? CU_TENSOR_MAP_SWIZZLE_32B
                                            : (R == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
  if (!make_map(&mq, p.q, bf16, R, p.Tq, p.H, p.B, sq, R, kRows, qk_swz)) return cudaSuccess;
  if (!make_map(&mk, p.k, bf16, R, p.Tk, p.H, p.B, sk, R, kKeys, qk_swz)) return cudaSuccess;
  if (!make_map(&mv, p.v, bf16, D, p.Tk, p.H, p.B, sv, 64, kKeys, CU_TENSOR_MAP_SWIZZLE_128B)) return cudaSuccess;
  dim3 grid((p.Tq + kRows - 1) / kRows, p.H, p.B);
  // the pipelined variant (two CTAs per SM) is opt-in: the four-CTA kernel below is faster at r=16
  const char* pipe = getenv("HOFA_OUTLIER_PIPE");
  if (D == 64 && pipe != nullptr && pipe[0] != '\0' && pipe[0] != '0') {
    auto k = outlier_tc_pipe_kernel<T, R>;
    constexpr size_t smem = pipe_smem_bytes<R>();
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    *taken = true;
    k<<<grid, kThreads, smem, st>>>(mq, mk, mv, p);
    return cudaGetLastError();
  }
  auto k = outlier_tc_kernel<T, D, R>;
  constexpr size_t smem = smem_bytes<D, R>();
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  *taken = true;
  k<<<grid, kThreads, smem, st>>>(mq, mk, mv, p);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t launch_d(const OutlierParams& p, cudaStream_t st, bool* taken) {
  switch (p.R) {
    case 16: return launch_dr<T, D, 16>(p, st, taken);
    case 32: return launch_dr<T, D, 32>(p, st, taken);
    case 64: return launch_dr<T, D, 64>(p, st, taken);
    default: return cudaSuccess;
  }
}

}  // namespace

cudaError_t launch_outlier_tc(const OutlierParams& p, int dtype, cudaStream_t st, bool* taken) {
  *taken = false;
  const char* off = getenv("HOFA_OUTLIER_NO_TC");
  if (off != nullptr && off[0] != '\0' && off[0] != '0') return cudaSuccess;
  if (dtype == HOFA_DTYPE_F32) return cudaSuccess;  // fp32 inputs take the CUDA-core kernel
  if (p.D != 64 && p.D != 128) return cudaSuccess;
  if (dtype == HOFA_DTYPE_BF16) {
    return p.D == 64 ? launch_d<__nv_bfloat16, 64>(p, st, taken) : launch_d<__nv_bfloat16, 128>(p, st, taken);
  }
  return p.D == 64 ? launch_d<__half, 64>(p, st, taken) : launch_d<__half, 128>(p, st, taken);
}

cudaError_t read_outlier_tc_status(int* out, cudaStream_t st) {
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_outlier_tc_status, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return e;
  const int zero = 0;
  e = cudaMemcpyToSymbolAsync(g_outlier_tc_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return e;
  return cudaStreamSynchronize(st);
}

}  // namespace hofa
