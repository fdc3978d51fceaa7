// Tensor-core outlier attention for sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces the reference's Triton kernel _fwd_kernel (src/exact_attention.py:
// 45-161): out += mix * softmax(sm_scale * q_r k_r^T, causal) v with r = R
// query/key channels and D value channels.  One CTA owns 128 query rows of
// one (b,h): warps 0-3 run the softmax (thread i owns row i, which is TMEM
// lane i) and warp 4 issues every TMA copy and MMA.  Keys come in tiles of 64.
//
//   TMEM: one S/P buffer of 64 fp32 columns and O (D fp32 columns); 128
//   columns in all at head dim 64, so four CTAs share an SM.
//   Shared memory: the Q tile and 4-stage K and V rings filled by TMA (4-D
//   tiled maps over [B,H,T,channels], no multicast).
//
//   Issuer, step t:  once every softmax warp wrote P_{t-1}:
//                    O += P_{t-1} V_{t-1} (P from TMEM, V from shared memory),
//                    then S_t = Q K_t^T into the same buffer and one commit.
//                    MMAs issued by one thread run in issue order, so S_t
//                    overwrites P_{t-1} only after the P V product read it,
//                    and the commit's arrival means O is complete as well.
//   Softmax, tile t: two 32-column halves: load S from TMEM, P = exp2(S*c - m)
//                    as 16-bit pairs written back over the columns already
//                    consumed (P of the tile ends in columns [0, 32)), arrive.
//   While a CTA's softmax waits for its next S, the warps of the other CTAs
//   on the SM keep the exponential unit busy.
//   The 1-D grid launches the row blocks with the most keys first, across
//   all heads, so that the CTAs finishing last are short ones.
//
// The running max is raised only when a row's max grows by more than 2^64
// (bf16; 2^8 for f16, whose largest value is 65504) -- then the row of O (and
// the tile's first half of P, when the second half raised it) is rescaled in
// TMEM; otherwise P is formed against the stale max, which changes nothing
// but the common factor removed at the end.  With bf16 a half-tile computes
// its exponentials against the running max at once and only takes the row max
// when a row's sum shows a growth past 2^64.
//
// Exponentials: two of the sixteen exp2 pairs of each full (unmasked) half
// run on the FMA pipe as a cubic polynomial (exp2_pair_poly), the rest on the
// MUFU unit, so that neither unit alone bounds the softmax (HOFA_OUTLIER_EMU
// selects 0-4 of 16 at bf16, head dim 64, r = 16; two measured fastest).
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

constexpr int kRows = 128;         // query rows per CTA (TMEM lanes)
constexpr int kKeys = 64;          // keys per tile
constexpr int kHalf = 32;          // the softmax takes a tile in two halves of 32 columns
constexpr int kSoftmaxWarps = 4;
constexpr int kThreads = 32 * (kSoftmaxWarps + 1);
constexpr int kStages = 4;         // K and V ring depth
constexpr int kEmuDefault = 2;     // of the 16 exp2 pairs of a full half-tile, this many run on the FMA pipe (measured best)
const int kEmuSetting = [] {
  const char* v = getenv("HOFA_OUTLIER_EMU");
  return v != nullptr && v[0] != '\0' ? atoi(v) : kEmuDefault;
}();

// TMEM columns: the S/P buffer in [0, kKeys), O in [kKeys, kKeys + D), rounded up to a power of two
template <int D>
constexpr uint32_t tmem_cols() { return kKeys + D <= 128 ? 128 : 256; }

constexpr uint32_t round1k(uint32_t b) { return (b + 1023u) & ~1023u; }

template <int D, int R>
struct Smem {
  static constexpr uint32_t RB = R * 2;                       // bytes per Q/K row
  static constexpr uint32_t Q_BYTES = kRows * RB;
  static constexpr uint32_t K_BYTES = kKeys * RB;
  static constexpr uint32_t V_BYTES = kKeys * D * 2;
  static constexpr uint32_t K_SLOT = round1k(K_BYTES);
  static constexpr uint32_t V_SLOT = round1k(V_BYTES);
  static constexpr uint32_t OFF_K = round1k(Q_BYTES);
  static constexpr uint32_t OFF_V = OFF_K + kStages * K_SLOT;
  static constexpr uint32_t OFF_BAR = OFF_V + kStages * V_SLOT;
  static constexpr size_t BYTES = 1024 + OFF_BAR + 256;       // + alignment slack, barriers
};

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

// 2^x for two fp32 lanes without the MUFU unit (packed f32x2 FMA-pipe math).
// Range reduction 2^x = 2^n * 2^f with n = floor(x) and f = x - n in [0, 1):
// adding 1.5*2^23 with round-toward-minus-infinity leaves n in the low
// mantissa bits of t, so t - 1.5*2^23 = n exactly and (bits(t) << 23) is n
// shifted into the exponent field.  2^f is a cubic fitted to minimise the
// maximum relative error over [0, 1) (a linear programme over 4001 points):
// max relative error 7.5e-5, below the 2^-9 rounding of the 16-bit P that the
// P V product consumes.  x is clamped at -126 so that the exponent field never
// underflows into the sign bit (2^-126 is zero for every later use).
__device__ __forceinline__ void exp2_pair_poly(uint64_t x2, float& e0, float& e1) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  constexpr float kC0 = 0.99992525577545166f, kC1 = 0.69583284854888916f;
  constexpr float kC2 = 0.22606939077377319f, kC3 = 0.078023009002208710f;
  float x0, x1;
  sm100::f2_unpack(x2, x0, x1);
  const uint64_t x = sm100::f2_pack(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
  const uint64_t magic = sm100::f2_pack(kMagic, kMagic);
  const uint64_t t = sm100::f2_add_rm(x, magic);
  const uint64_t f = sm100::f2_sub(x, sm100::f2_sub(t, magic));
  uint64_t p = sm100::f2_fma(sm100::f2_pack(kC3, kC3), f, sm100::f2_pack(kC2, kC2));
  p = sm100::f2_fma(p, f, sm100::f2_pack(kC1, kC1));
  p = sm100::f2_fma(p, f, sm100::f2_pack(kC0, kC0));
  float p0, p1, t0, t1;
  sm100::f2_unpack(p, p0, p1);
  sm100::f2_unpack(t, t0, t1);
  e0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  e1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

// Row of 32 scores -> 32 probabilities packed as 16-bit pairs in pk[16]
// (pair i = columns 2i, 2i+1); returns the row sum in fp32.  E of the 16
// pairs, spread evenly (pair i when i*E mod 16 < E), use the polynomial, the
// rest the MUFU unit.
template <bool BF16, int E>
__device__ __forceinline__ float row_exp(const uint32_t (&r)[32], float scale, float m, uint32_t (&pk)[16]) {
  const uint64_t sc2 = sm100::f2_pack(scale, scale);
  const uint64_t nm2 = sm100::f2_pack(-m, -m);
  uint64_t acc[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = sm100::f2_pack(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint64_t x =
        sm100::f2_fma(sm100::f2_pack(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])), sc2, nm2);
    float e0, e1;
    if ((i * E) % 16 < E) {
      exp2_pair_poly(x, e0, e1);
    } else {
      float x0, x1;
      sm100::f2_unpack(x, x0, x1);
      e0 = sm100::ex2_approx(x0);
      e1 = sm100::ex2_approx(x1);
    }
    acc[i & 3] = sm100::f2_add(acc[i & 3], sm100::f2_pack(e0, e1));
    pk[i] = pack2(e0, e1, BF16);
  }
  const uint64_t t = sm100::f2_add(sm100::f2_add(acc[0], acc[1]), sm100::f2_add(acc[2], acc[3]));
  float a, b;
  sm100::f2_unpack(t, a, b);
  return a + b;
}

template <typename T, int D, int R, int EMU>
__global__ void __launch_bounds__(kThreads, D == 64 ? 4 : 2)
outlier_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, const OutlierParams p) {
  using L = Smem<D, R>;
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t SWZ = swizzle_mode(L::RB);
  constexpr uint32_t IDESC_S = sm100::idesc_f16(BF16, false, false, kRows, kKeys);
  constexpr uint32_t IDESC_O = sm100::idesc_f16(BF16, false, true, kRows, D);
  constexpr uint32_t NCOLS = tmem_cols<D>();
  constexpr bool SKIPMAX = BF16;  // f16 P (kRaise 8) keeps the row max on every tile
  // lazy rescale threshold (log2 units): P values stay below 2^kRaise.  bf16
  // P and the fp32 row sums and O share fp32's exponent range, so 2^64 (and
  // a row sum below 2^64 times the key count) is far from overflow; f16 P
  // (largest value 65504) keeps a margin at 2^8
  constexpr float kRaise = BF16 ? 64.f : 8.f;

  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* const sQ = base;
  unsigned char* const sK0 = base + L::OFF_K;   // slot s at sK0 + s * K_SLOT
  unsigned char* const sV0 = base + L::OFF_V;   // slot s at sV0 + s * V_SLOT
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + L::OFF_BAR);
  uint64_t* bar_q = bars + 0;
  uint64_t* bar_k = bars + 1;                 // [kStages] K_t landed
  uint64_t* bar_v = bar_k + kStages;          // [kStages] V_t landed
  uint64_t* bar_s = bar_v + kStages;          // phase t: S_t (and every earlier MMA) complete
  uint64_t* bar_p = bar_s + 1;                // phase t: every softmax warp wrote P_t
  uint64_t* bar_fin = bar_p + 1;              // the last O += P V is done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_fin + 1);
  int* err_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nqb = (p.Tq + kRows - 1) / kRows;
  // one block per (row block, head, batch), numbered so that the row blocks
  // with the most keys (the last ones) of every head launch first: the CTAs
  // that finish last are the short ones, which keeps the grid's tail short
  const int heads = p.H * p.B;
  const int qb = nqb - 1 - (int)(blockIdx.x / heads);
  const int h = (int)(blockIdx.x % heads) % p.H, b = (int)(blockIdx.x % heads) / p.H;
  const int q0 = qb * kRows;
  const int last_key = min(p.Tk - 1, q0 + kRows - 1 + p.q_offset);
  const int n = last_key / kKeys + 1;

  if (tid == 0) {
    sm100::mbar_init(bar_q, 1);
    for (int i = 0; i < kStages; ++i) {
      sm100::mbar_init(&bar_k[i], 1);
      sm100::mbar_init(&bar_v[i], 1);
    }
    sm100::mbar_init(bar_s, 1);
    sm100::mbar_init(bar_p, kSoftmaxWarps);
    sm100::mbar_init(bar_fin, 1);
    *err_flag = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tmem_slot, NCOLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + kKeys;

  // Bounded waits.  The CTA's error flag is only read when a phase is not
  // already complete; after the first timeout every later wait and every
  // MMA / copy issue is skipped, while the loops keep their trip counts so
  // that warp-collective TMEM accesses stay convergent.  Phase parities never
  // alias: a waiter of phase t of bar_s or bar_p is itself what holds back
  // phase t + 1 (the issuer issues S_{t+1} only after P_t; P_{t+1} needs
  // S_{t+1}).
  volatile int* verr = err_flag;
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (sm100::mbar_try_wait(bar, parity)) return;
    if (*verr) return;
    if (!sm100::mbar_wait(bar, parity)) atomicOr(err_flag, 1);
  };

  if (warp == kSoftmaxWarps) {
    // ---------------------------- issuer ------------------------------------
    if (lane == 0) {
      sm100::prefetch_tmap(&tq);
      sm100::prefetch_tmap(&tk);
      sm100::prefetch_tmap(&tv);
      auto load_kv = [&](int t) {
        const int s = t % kStages;
        sm100::mbar_arrive_expect_tx(&bar_k[s], L::K_BYTES);
        sm100::tma_load_4d(sK0 + s * L::K_SLOT, &tk, 0, t * kKeys, h, b, &bar_k[s]);
        sm100::mbar_arrive_expect_tx(&bar_v[s], L::V_BYTES);
#pragma unroll
        for (int g = 0; g < D / 64; ++g)
          sm100::tma_load_4d(sV0 + s * L::V_SLOT + g * kKeys * 128, &tv, g * 64, t * kKeys, h, b, &bar_v[s]);
      };
      const uint64_t qdesc = sm100::smem_desc(sQ, 16, 8 * L::RB, SWZ);
      const uint64_t kdesc0 = sm100::smem_desc(sK0, 16, 8 * L::RB, SWZ);
      const uint64_t vdesc0 = sm100::smem_desc(sV0, kKeys * 128, 1024, sm100::kSwizzle128);
      auto issue_pv = [&](int u) {  // O += P_u V_u, P_u in TMEM columns [0, kKeys / 2)
        // V_u landed long before P_u: only the MMAs follow P_u's arrival
        wait(&bar_v[u % kStages], (u / kStages) & 1);
        wait(bar_p, u & 1);
        if (*verr) return;
        sm100::tc_fence_after();
        const uint64_t vdesc = vdesc0 + (uint64_t)(((u % kStages) * L::V_SLOT) >> 4);
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk)
          sm100::mma_ts(tO, tmem + kk * 8, vdesc + (uint64_t)(kk * 2048 >> 4), IDESC_O, u > 0 || kk > 0);
      };
      sm100::mbar_arrive_expect_tx(bar_q, L::Q_BYTES);
      sm100::tma_load_4d(sQ, &tq, 0, q0, h, b, bar_q);
      for (int t = 0; t < kStages && t < n; ++t) load_kv(t);
      wait(bar_q, 0);
      for (int t = 0; t < n; ++t) {
        const int s = t % kStages;
        wait(&bar_k[s], (t / kStages) & 1);
        if (t >= 1) issue_pv(t - 1);
        if (!*verr) {
          sm100::tc_fence_after();
          const uint64_t kdesc = kdesc0 + (uint64_t)((s * L::K_SLOT) >> 4);
#pragma unroll
          for (int ks = 0; ks < R / 16; ++ks)
            sm100::mma_ss(tmem, qdesc + 2 * ks, kdesc + 2 * ks, IDESC_S, ks > 0);
          sm100::mma_commit(bar_s);
        }
        // the slot of tile t - 2 is free: O += P_{t-2} V_{t-2} completed before
        // S_{t-1}, which the softmax consumed before it wrote P_{t-1}
        if (t >= 2 && t - 2 + kStages < n && !*verr) load_kv(t - 2 + kStages);
      }
      issue_pv(n - 1);
      sm100::mma_commit(bar_fin);
    }
  } else {
    // ---------------------------- softmax -----------------------------------
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const float scale = p.qk_scale_log2;
    const int row = q0 + tid;
    const int limit = min(row + p.q_offset, p.Tk - 1);   // last visible key of this row
    const int warp_min_limit = min(q0 + warp * 32 + p.q_offset, p.Tk - 1);
    float m_used = -INFINITY, l_sum = 0.f;
    for (int t = 0; t < n; ++t) {
      wait(bar_s, t & 1);
      sm100::tc_fence_after();
#pragma unroll 1
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t r[32];
        sm100::tmem_ld32(tmem + hf * kHalf + lane_off, r);
        sm100::tc_wait_ld();

        const int k0 = t * kKeys + hf * kHalf;
        const bool masked = k0 + kHalf - 1 > warp_min_limit;   // some key of the half is past some row's limit
        if (masked) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (k0 + i > limit) r[i] = __float_as_uint(-INFINITY);
        }
        uint32_t pk[16];
        float ls = 0.f, factor = 1.f;
        bool slow = true;
        if (SKIPMAX && !masked && (t | hf) != 0) {
          // exponentials against the running max straight away; a row whose max
          // grew by more than 2^kRaise shows in its sum (>= 2^kRaise, inf or
          // NaN), and only then does the warp redo the half with the row max
          ls = row_exp<BF16, (EMU > 16 ? 0 : EMU)>(r, scale, m_used, pk);
          slow = __any_sync(0xffffffffu, !(ls < 1.8446744e19f));  // 2^64
        }
        if (slow) {
          float mx[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            mx[i] = sm100::fmax3(__uint_as_float(r[8 * i]), __uint_as_float(r[8 * i + 1]), __uint_as_float(r[8 * i + 2]));
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            mx[i] = sm100::fmax3(mx[i], __uint_as_float(r[8 * i + 3]), __uint_as_float(r[8 * i + 4]));
            mx[i] = sm100::fmax3(mx[i], __uint_as_float(r[8 * i + 5]), __uint_as_float(r[8 * i + 6]));
            mx[i] = fmaxf(mx[i], __uint_as_float(r[8 * i + 7]));
          }
          const float mts = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * scale;
          const bool raise = mts > m_used + kRaise;
          factor = raise ? sm100::ex2_approx(m_used - mts) : 1.f;  // 0 while m_used is -inf
          if (raise) m_used = mts;
          // TMEM loads/stores are warp-collective: the whole warp rescales its
          // rows when any of them raised its max (the others multiply by 1).
          // O is quiescent here: S_t's commit arrived after O += P_{t-1} V_{t-1}
          // completed, and O += P_t V_t waits for this warp's arrival.
          if (__any_sync(0xffffffffu, raise)) {
            if (t > 0) {
#pragma unroll
              for (int c = 0; c < D; c += 16) {
                uint32_t o[16];
                sm100::tmem_ld16(tO + lane_off + c, o);
                sm100::tc_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
                sm100::tmem_st16(tO + lane_off + c, o);
              }
            }
            if (hf == 1) {
              // the first half's P (16-bit pairs in columns [0, 16)) was formed
              // against the old max
              uint32_t o[16];
              sm100::tc_wait_st();
              sm100::tmem_ld16(tmem + lane_off, o);
              sm100::tc_wait_ld();
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                float a, bb;
                if (BF16) bf16x2_to_f(o[i], a, bb); else f16x2_to_f(o[i], a, bb);
                o[i] = pack2(a * factor, bb * factor, BF16);
              }
              sm100::tmem_st16(tmem + lane_off, o);
            }
          }
          ls = masked ? row_exp<BF16, 0>(r, scale, m_used, pk)   // exact zeros where masked
                      : row_exp<BF16, (EMU > 16 ? 0 : EMU)>(r, scale, m_used, pk);
        }
        l_sum = l_sum * factor + ls;
        // P of this half as 16-bit pairs over columns [16 hf, 16 hf + 16), which
        // the first half's load already consumed
        sm100::tmem_st16(tmem + hf * 16 + lane_off, pk);
      }
      sm100::tc_wait_st();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(bar_p);
    }
    wait(bar_fin, 0);
    sm100::tc_fence_after();

    // ---- epilogue: out = (accumulate ? out : 0) + mix * O / l --------------
    const bool store = row < p.Tq && !*verr;
    T* og = reinterpret_cast<T*>(p.out) + b * p.so[0] + h * p.so[1] + (int64_t)(store ? row : 0) * p.so[2];
    const bool vec = p.so[3] == 1 && (reinterpret_cast<uintptr_t>(og) & 15u) == 0;
    // the row's global reads in one round trip: its blend and, when accumulating,
    // its current output (read per column chunk, each read would wait for the
    // previous chunk's TMEM load and stores)
    const float mix = store ? ld_any(p.mix_g, p.dt_mg, b * p.smg[0] + h * p.smg[1] + (int64_t)row * p.smg[2]) : 0.f;
    uint4 oldv[D / 8];
#pragma unroll
    for (int i = 0; i < D / 8; ++i)
      oldv[i] = store && vec && p.accumulate ? reinterpret_cast<const uint4*>(og)[i] : make_uint4(0, 0, 0, 0);
    const float inv = l_sum > 0.f ? mix / l_sum : 0.f;
#pragma unroll
    for (int c = 0; c < D; c += 16) {
      uint32_t o[16];
      sm100::tmem_ld16(tO + lane_off + c, o);  // warp-collective: every lane executes it
      sm100::tc_wait_ld();
      if (store && vec) {
        uint4* dst = reinterpret_cast<uint4*>(og + c);
        uint32_t w[8];
        const uint4 old[2] = {oldv[c / 8], oldv[c / 8 + 1]};   // zeros unless accumulating
        const uint32_t* ow = reinterpret_cast<const uint32_t*>(old);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float a = __uint_as_float(o[2 * i]) * inv, bb = __uint_as_float(o[2 * i + 1]) * inv;
          if (p.accumulate) {
            float oa, ob;
            if (BF16) bf16x2_to_f(ow[i], oa, ob); else f16x2_to_f(ow[i], oa, ob);
            a += oa;
            bb += ob;
          }
          w[i] = pack2(a, bb, BF16);
        }
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
      } else if (store) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int64_t off = (int64_t)(c + i) * p.so[3];
          float v = __uint_as_float(o[i]) * inv;
          if (p.accumulate) v += to_f(og[off]);
          og[off] = from_f<T>(v);
        }
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (*err_flag && tid == 0) atomicOr(&g_outlier_tc_status, 1);
  if (warp == 0) sm100::tmem_dealloc(tmem, NCOLS);
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

// Dynamic shared memory per CTA: at least what the kernel uses, and enough
// that no more CTAs are resident on an SM than its 512 TMEM columns serve (a
// CTA beyond that would wait inside tcgen05.alloc for a neighbour to finish).
size_t residency_smem(size_t need, uint32_t tmem_cols_per_cta) {
  static int per_sm = -1, reserved = 0;
  if (per_sm < 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess) per_sm = 0;
    if (cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess) reserved = 0;
  }
  const int fit = 512 / (int)tmem_cols_per_cta;                  // CTAs whose TMEM fits
  const long cap = per_sm / (fit + 1) - reserved + 128;            // more than 1/(fit+1) of the SM each
  return cap > (long)need ? (size_t)((cap + 127) & ~127L) : need;
}

template <typename T, int D, int R, int EMU>
cudaError_t launch_kernel(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const OutlierParams& p,
                          dim3 grid, cudaStream_t st, bool* taken) {
  auto k = outlier_tc_kernel<T, D, R, EMU>;
  const size_t smem = residency_smem(Smem<D, R>::BYTES, tmem_cols<D>());
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  *taken = true;
  k<<<grid, kThreads, smem, st>>>(mq, mk, mv, p);
  return cudaGetLastError();
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
  dim3 grid((unsigned)((p.Tq + kRows - 1) / kRows) * p.H * p.B);
  // HOFA_OUTLIER_EMU (0..4, read once at library load) overrides how many of
  // the 16 exp2 pairs of a full half-tile run as the FMA-pipe polynomial
  // (bf16, head dim 64, r = 16)
  if constexpr (std::is_same<T, __nv_bfloat16>::value && D == 64 && R == 16) {
    const int e = kEmuSetting;
    if (e == 0) return launch_kernel<T, D, R, 0>(mq, mk, mv, p, grid, st, taken);
    if (e == 1) return launch_kernel<T, D, R, 1>(mq, mk, mv, p, grid, st, taken);
    if (e == 2) return launch_kernel<T, D, R, 2>(mq, mk, mv, p, grid, st, taken);
    if (e == 3) return launch_kernel<T, D, R, 3>(mq, mk, mv, p, grid, st, taken);
    if (e == 4) return launch_kernel<T, D, R, 4>(mq, mk, mv, p, grid, st, taken);
  }
  return launch_kernel<T, D, R, kEmuDefault>(mq, mk, mv, p, grid, st, taken);
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
