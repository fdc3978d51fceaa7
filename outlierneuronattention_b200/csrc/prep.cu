// Gates + RoPE + cache export: one warp per token over all heads when each
// token's heads are adjacent in memory (prep_tok_kernel: a token's q, k, v
// rows are then contiguous blocks, read with coalesced 16-byte loads), one
// thread per (token, head) with 16-byte row accesses otherwise
// (prep_vec_kernel), or one warp per (token, head) for any strides.
//
// Replaces the layer's elementwise glue around the attention core
// (src/HybridOutlierFactorizedAttention.py):
//   * _compute_gates_optimized (:67-95): gate = q.Wg[h,:D] + k.Wg[h,D:] + bg[h]
//     and mix = sigmoid(q.Wm[h,:D] + k.Wm[h,D:] + bm[h]) on the UN-rotated q, k
//     (or sigmoid(fixed_mix[h]) for the fixed-blend ablation);
//   * log_gamma = logsigmoid(-gate) (:177, :361);
//   * rotate-half RoPE of channels [0, R) of q and k in place, at absolute
//     position pos0 + n, from the module's cos/sin tables (:180-188,
//     :365-375; src/modules/modules.py:33-45);
//   * the outlier cache rows: cache_k[.., pos, :R] = rotated k,
//     cache_v[.., pos, :] = v (:196-198 prefill export, :382-384 decode append).
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace hofa {

namespace {

// HOFA_PREP_NO_TOKEN_MAJOR (read once at library load) turns the token-major
// kernel off, for comparisons.
const bool kPrepNoTokenMajor = [] {
  const char* v = getenv("HOFA_PREP_NO_TOKEN_MAJOR");
  return v != nullptr && v[0] != '\0' && v[0] != '0';
}();

int sm_count() {
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

constexpr int kPrepWarps = 8;

template <typename T, int D>
__global__ void __launch_bounds__(kPrepWarps * 32)
prep_kernel(const PrepParams p) {
  constexpr int PL = D / 32 > 0 ? D / 32 : 1;  // channels per lane
  __shared__ float xs[kPrepWarps][2][D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * kPrepWarps + warp;
  const int64_t total = (int64_t)p.B * p.H * p.N;
  if (gw >= total) return;
  const int n = (int)(gw % p.N);
  const int h = (int)((gw / p.N) % p.H);
  const int b = (int)(gw / ((int64_t)p.N * p.H));

  T* qp = reinterpret_cast<T*>(p.q) + b * p.sq[0] + h * p.sq[1] + (int64_t)n * p.sq[2];
  T* kp = reinterpret_cast<T*>(p.k) + b * p.sk[0] + h * p.sk[1] + (int64_t)n * p.sk[2];

  float qv[PL], kv[PL];
  float g = 0.f, ml = 0.f;
#pragma unroll
  for (int u = 0; u < PL; ++u) {
    const int c = lane + 32 * u;
    qv[u] = kv[u] = 0.f;
    if (c < D) {
      qv[u] = to_f(qp[(int64_t)c * p.sq[3]]);
      kv[u] = to_f(kp[(int64_t)c * p.sk[3]]);
      g = fmaf(qv[u], ld_any(p.gate_w, p.dt_gw, h * p.sgw[0] + c * p.sgw[1]), g);
      g = fmaf(kv[u], ld_any(p.gate_w, p.dt_gw, h * p.sgw[0] + (D + c) * p.sgw[1]), g);
      if (p.mix_w != nullptr) {
        ml = fmaf(qv[u], ld_any(p.mix_w, p.dt_mw, h * p.smw[0] + c * p.smw[1]), ml);
        ml = fmaf(kv[u], ld_any(p.mix_w, p.dt_mw, h * p.smw[0] + (D + c) * p.smw[1]), ml);
      }
      xs[warp][0][c] = qv[u];
      xs[warp][1][c] = kv[u];
    }
  }
  g = warp_sum(g);
  ml = warp_sum(ml);
  if (lane == 0) {
    g += ld_any(p.gate_b, p.dt_gb, h * p.sgb);
    // logsigmoid(-g) = -softplus(g) = -(max(g,0) + log1p(exp(-|g|)))
    const float lgam = -(fmaxf(g, 0.f) + log1pf(expf(-fabsf(g))));
    st_any(p.log_gamma, p.dt_lg, b * p.slg[0] + h * p.slg[1] + (int64_t)n * p.slg[2], lgam);
    if (p.mix_out != nullptr) {
      float mlog;
      if (p.mix_w != nullptr) mlog = ml + ld_any(p.mix_b, p.dt_mb, h * p.smb);
      else mlog = ld_any(p.fixed_mix, p.dt_fm, h * p.sfm);
      const float mix = 1.f / (1.f + expf(-mlog));
      st_any(p.mix_out, p.dt_mo, b * p.smo[0] + h * p.smo[1] + (int64_t)n * p.smo[2], mix);
    }
  }
  __syncwarp();

  int pos = (p.pos0_dev != nullptr ? *p.pos0_dev + p.pos0_dev_bias : p.pos0) + n;
  const int R = p.R, half = R / 2;
  if (p.rope && R > 0) {
    const int prow = pos < 0 ? 0 : (pos < p.P ? pos : p.P - 1);
#pragma unroll
    for (int u = 0; u < PL; ++u) {
      const int c = lane + 32 * u;
      if (c < R) {
        const float cs = ld_any(p.cos, p.dt_cs, (int64_t)prow * p.scos[0] + c * p.scos[1]);
        const float sn = ld_any(p.sin, p.dt_cs, (int64_t)prow * p.ssin[0] + c * p.ssin[1]);
        const float qr = (c < half) ? -xs[warp][0][c + half] : xs[warp][0][c - half];
        const float kr = (c < half) ? -xs[warp][1][c + half] : xs[warp][1][c - half];
        qv[u] = qv[u] * cs + qr * sn;
        kv[u] = kv[u] * cs + kr * sn;
        qp[(int64_t)c * p.sq[3]] = from_f<T>(qv[u]);
        kp[(int64_t)c * p.sk[3]] = from_f<T>(kv[u]);
      }
    }
  }
  if (p.cache_k != nullptr && pos >= 0 && pos < p.L) {
    T* ck = reinterpret_cast<T*>(p.cache_k) + b * p.sck[0] + h * p.sck[1] + (int64_t)pos * p.sck[2];
#pragma unroll
    for (int u = 0; u < PL; ++u) {
      const int c = lane + 32 * u;
      if (c < R) ck[(int64_t)c * p.sck[3]] = from_f<T>(kv[u]);
    }
  }
  if (p.cache_v != nullptr && pos >= 0 && pos < p.L) {
    const T* vp = reinterpret_cast<const T*>(p.v) + b * p.sv[0] + h * p.sv[1] + (int64_t)n * p.sv[2];
    T* cv = reinterpret_cast<T*>(p.cache_v) + b * p.scv[0] + h * p.scv[1] + (int64_t)pos * p.scv[2];
#pragma unroll
    for (int u = 0; u < PL; ++u) {
      const int c = lane + 32 * u;
      if (c < D) cv[(int64_t)c * p.scv[3]] = vp[(int64_t)c * p.sv[3]];
    }
  }
}

// Vector variant: one thread per (token, head), 16-byte loads/stores of whole
// rows, the head's gate / mix weights staged in shared memory.  Needs unit
// channel stride, 16-byte aligned rows and R % 8 == 0.
constexpr int kVecThreads = 128;

// Threads [0, kVecThreads) compute the gates and RoPE of one token each;
// threads [kVecThreads, 2*kVecThreads) copy the same tokens' v rows into the
// V cache meanwhile (the copy then costs no round trip of its own).
template <typename T, int D, int RMAX>  // RMAX == R (compile-time, so RoPE stays in registers)
__global__ void __launch_bounds__(2 * kVecThreads)
prep_vec_kernel(const PrepParams p) {
  constexpr int G = D / 8;  // 16-byte groups of 8 channels (2-byte types)
  __shared__ float w_gate[2 * D], w_mix[2 * D];
  const int h = blockIdx.y, b = blockIdx.z;
  if (threadIdx.x >= kVecThreads) {
    const int nv = blockIdx.x * kVecThreads + threadIdx.x - kVecThreads;
    const int posv = (p.pos0_dev != nullptr ? *p.pos0_dev + p.pos0_dev_bias : p.pos0) + nv;
    if (nv < p.N && p.cache_v != nullptr && posv >= 0 && posv < p.L) {
      const T* vp = reinterpret_cast<const T*>(p.v) + b * p.sv[0] + h * p.sv[1] + (int64_t)nv * p.sv[2];
      T* cv = reinterpret_cast<T*>(p.cache_v) + b * p.scv[0] + h * p.scv[1] + (int64_t)posv * p.scv[2];
      uint4 rowv[G];
#pragma unroll
      for (int c = 0; c < G; ++c) rowv[c] = *reinterpret_cast<const uint4*>(vp + 8 * c);
#pragma unroll
      for (int c = 0; c < G; ++c) *reinterpret_cast<uint4*>(cv + 8 * c) = rowv[c];
    }
    return;
  }
  const int n = blockIdx.x * kVecThreads + threadIdx.x;
  const bool has_mix = p.mix_w != nullptr;
  for (int i = threadIdx.x; i < 2 * D; i += kVecThreads) {
    w_gate[i] = ld_any(p.gate_w, p.dt_gw, h * p.sgw[0] + i * p.sgw[1]);
    w_mix[i] = has_mix ? ld_any(p.mix_w, p.dt_mw, h * p.smw[0] + i * p.smw[1]) : 0.f;
  }
  asm volatile("bar.sync 1, %0;" ::"n"(kVecThreads) : "memory");  // the gate/RoPE threads only
  if (n >= p.N) return;
  T* qp = reinterpret_cast<T*>(p.q) + b * p.sq[0] + h * p.sq[1] + (int64_t)n * p.sq[2];
  T* kp = reinterpret_cast<T*>(p.k) + b * p.sk[0] + h * p.sk[1] + (int64_t)n * p.sk[2];
  float qo[RMAX > 0 ? RMAX : 1], ko[RMAX > 0 ? RMAX : 1];
  float g = 0.f, ml = 0.f;
#pragma unroll
  for (int c = 0; c < G; ++c) {
    float fq[8], fk[8];
    vec8_to_f(*reinterpret_cast<const Vec8<T>*>(qp + 8 * c), fq);
    vec8_to_f(*reinterpret_cast<const Vec8<T>*>(kp + 8 * c), fk);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      g = fmaf(fq[e], w_gate[8 * c + e], g);
      g = fmaf(fk[e], w_gate[D + 8 * c + e], g);
      ml = fmaf(fq[e], w_mix[8 * c + e], ml);
      ml = fmaf(fk[e], w_mix[D + 8 * c + e], ml);
      if (8 * c + e < RMAX) { qo[8 * c + e] = fq[e]; ko[8 * c + e] = fk[e]; }
    }
  }
  g += ld_any(p.gate_b, p.dt_gb, h * p.sgb);
  st_any(p.log_gamma, p.dt_lg, b * p.slg[0] + h * p.slg[1] + (int64_t)n * p.slg[2],
         -(fmaxf(g, 0.f) + log1pf(expf(-fabsf(g)))));
  if (p.mix_out != nullptr) {
    const float mlog = has_mix ? ml + ld_any(p.mix_b, p.dt_mb, h * p.smb) : ld_any(p.fixed_mix, p.dt_fm, h * p.sfm);
    st_any(p.mix_out, p.dt_mo, b * p.smo[0] + h * p.smo[1] + (int64_t)n * p.smo[2], 1.f / (1.f + expf(-mlog)));
  }
  const int pos = (p.pos0_dev != nullptr ? *p.pos0_dev + p.pos0_dev_bias : p.pos0) + n;
  if (RMAX > 0 && p.rope) {
    constexpr int half = RMAX / 2;
    const int prow = pos < 0 ? 0 : (pos < p.P ? pos : p.P - 1);
    float qr[RMAX > 0 ? RMAX : 1], kr[RMAX > 0 ? RMAX : 1];
    float csv[RMAX > 0 ? RMAX : 1], snv[RMAX > 0 ? RMAX : 1];
    const float* cs_row = reinterpret_cast<const float*>(p.cos) + (int64_t)prow * p.scos[0];
    const float* sn_row = reinterpret_cast<const float*>(p.sin) + (int64_t)prow * p.ssin[0];
    if (RMAX % 4 == 0 && p.dt_cs == HOFA_DTYPE_F32 && p.scos[1] == 1 && p.ssin[1] == 1 &&
        ((reinterpret_cast<uintptr_t>(cs_row) | reinterpret_cast<uintptr_t>(sn_row)) & 15u) == 0) {
#pragma unroll
      for (int c = 0; c < RMAX; c += 4) {  // contiguous fp32 table rows: 16-byte loads
        const float4 a = *reinterpret_cast<const float4*>(cs_row + c);
        const float4 z = *reinterpret_cast<const float4*>(sn_row + c);
        csv[c] = a.x; csv[c + 1] = a.y; csv[c + 2] = a.z; csv[c + 3] = a.w;
        snv[c] = z.x; snv[c + 1] = z.y; snv[c + 2] = z.z; snv[c + 3] = z.w;
      }
    } else {
#pragma unroll
      for (int c = 0; c < RMAX; ++c) {
        csv[c] = ld_any(p.cos, p.dt_cs, (int64_t)prow * p.scos[0] + c * p.scos[1]);
        snv[c] = ld_any(p.sin, p.dt_cs, (int64_t)prow * p.ssin[0] + c * p.ssin[1]);
      }
    }
#pragma unroll
    for (int c = 0; c < RMAX; ++c) {
      const float cs = csv[c], sn = snv[c];
      const float qh = c < half ? -qo[c + half] : qo[c - half];
      const float kh = c < half ? -ko[c + half] : ko[c - half];
      qr[c] = qo[c] * cs + qh * sn;
      kr[c] = ko[c] * cs + kh * sn;
    }
#pragma unroll
    for (int c = 0; c < RMAX / 8; ++c) {
      T tq[8], tk[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) { tq[e] = from_f<T>(qr[8 * c + e]); tk[e] = from_f<T>(kr[8 * c + e]); }
      *reinterpret_cast<uint4*>(qp + 8 * c) = *reinterpret_cast<const uint4*>(tq);
      *reinterpret_cast<uint4*>(kp + 8 * c) = *reinterpret_cast<const uint4*>(tk);
#pragma unroll
      for (int e = 0; e < 8; ++e) ko[8 * c + e] = kr[8 * c + e];
    }
  }
  if (RMAX > 0 && p.cache_k != nullptr && pos >= 0 && pos < p.L) {
    T* ck = reinterpret_cast<T*>(p.cache_k) + b * p.sck[0] + h * p.sck[1] + (int64_t)pos * p.sck[2];
#pragma unroll
    for (int c = 0; c < RMAX / 8; ++c) {
      T tk[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) tk[e] = from_f<T>(ko[8 * c + e]);
      *reinterpret_cast<uint4*>(ck + 8 * c) = *reinterpret_cast<const uint4*>(tk);
    }
  }
}

// Token-major variant: one warp per token, all heads at once.  When every
// head's row of a token lies next to the previous head's (q, k, v views of a
// [.., T, H, D] or [.., T, 3, H, D] projection output), a token's q (and k, v)
// is one contiguous block of H*D elements, read with fully coalesced 16-byte
// loads: lane L holds 16-byte slot i = L + 32 j, i.e. channels [8g, 8g + 8)
// (g = i % (D/8)) of head i / (D/8), so each head is a group of D/8 adjacent
// lanes.  The gate and blend dot products reduce within a group; rotate-half
// RoPE exchanges the partner channels of [0, R) with one shuffle (in-lane for
// R = 8); the cache rows of a head are written by its group.  The heads'
// gate / blend weights are staged in shared memory once per CTA, and each
// warp walks tokens with a grid stride over a grid of resident CTAs.  Each
// lane copies its slots of the warp's NEXT token (and that token's cos/sin
// channels when the tables are contiguous fp32) into its own part of a
// shared-memory stage with cp.async while the current token is computed, so
// a warp always has one token's reads in flight.
constexpr int kTokWarps = 8;
constexpr int kTokMaxElems = 1024;  // H * D: at most four 16-byte slots per lane (registers)

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Bytes of one warp's stage: q, k, v slots of a token, then cos lo/hi, sin lo/hi.
template <int NJ, int RMAX>
__host__ __device__ constexpr int tok_stage_bytes() { return (3 * NJ + (RMAX > 0 ? 4 : 0)) * 32 * 16; }

template <typename T, int D, int RMAX, int NJ>   // NJ >= ceil(H * D / 256) 16-byte slots per lane
__global__ void __launch_bounds__(kTokWarps * 32, 2)
prep_tok_kernel(const PrepParams p) {
  constexpr int GL = D / 8;                 // lanes per head
  // Weights in shared memory, per head a row of 2D gate values then 2D blend
  // values; every 32 values are followed by 4 pad words, so that the 16-byte
  // reads of the 8 lanes of a quarter warp (channels 8g .. 8g + 7) hit
  // distinct banks.
  constexpr int PADROW = 2 * D + 2 * D / 8;  // one weight vector of 2D values, padded
  extern __shared__ __align__(16) float w_sm[];   // [H][2][PADROW], then kTokWarps stages
  auto widx = [](int c) { return c + 4 * (c >> 5); };
  const int H = p.H;
  const int slots = H * GL;                 // 16-byte slots of a token's row block
  const bool has_mix = p.mix_w != nullptr;
  const int lane = threadIdx.x & 31;
  const int g = lane % GL;                  // channel group of this lane within its head
  const int64_t total = (int64_t)p.B * p.N;
  const int64_t nwarps = (int64_t)gridDim.x * kTokWarps;
  const int pbase = p.pos0_dev != nullptr ? *p.pos0_dev + p.pos0_dev_bias : p.pos0;
  // this lane's stage entries: data slot (t, j) at stg[(t * NJ + j) * 32], table row q at stg[(3 NJ + q) * 32]
  uint4* stg = reinterpret_cast<uint4*>(w_sm + H * 2 * PADROW) + (threadIdx.x >> 5) * (tok_stage_bytes<NJ, RMAX>() / 16) + lane;
  const bool tab_async = RMAX > 0 && p.rope && p.dt_cs == HOFA_DTYPE_F32 && p.scos[1] == 1 && p.ssin[1] == 1 &&
                         (p.scos[0] & 3) == 0 && (p.ssin[0] & 3) == 0 &&
                         ((reinterpret_cast<uintptr_t>(p.cos) | reinterpret_cast<uintptr_t>(p.sin)) & 15) == 0;
  // Copies token t's slots into the stage.  `z` is zero, computed from the
  // values this lane last read from the stage, so that the copies cannot be
  // issued before those reads have returned.
  auto prefetch = [&](int b_, int n_, uint32_t z) {
    const T* q_ = reinterpret_cast<const T*>(p.q) + b_ * p.sq[0] + (int64_t)n_ * p.sq[2];
    const T* k_ = reinterpret_cast<const T*>(p.k) + b_ * p.sk[0] + (int64_t)n_ * p.sk[2];
    const T* v_ = reinterpret_cast<const T*>(p.v) + b_ * p.sv[0] + (int64_t)n_ * p.sv[2];
    uint4* d = stg + z;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int i = lane + 32 * j;
      if (i < slots) {
        cp_async16(d + (0 * NJ + j) * 32, q_ + 8 * i);
        cp_async16(d + (1 * NJ + j) * 32, k_ + 8 * i);
        if (p.cache_v != nullptr) cp_async16(d + (2 * NJ + j) * 32, v_ + 8 * i);
      }
    }
    if (RMAX > 0 && tab_async && g < RMAX / 8) {
      const int pos_ = pbase + n_;
      const int64_t pr = pos_ < 0 ? 0 : (pos_ < p.P ? pos_ : p.P - 1);
      const float* c_ = reinterpret_cast<const float*>(p.cos) + pr * p.scos[0] + 8 * g;
      const float* s_ = reinterpret_cast<const float*>(p.sin) + pr * p.ssin[0] + 8 * g;
      cp_async16(d + (3 * NJ + 0) * 32, c_);
      cp_async16(d + (3 * NJ + 1) * 32, c_ + 4);
      cp_async16(d + (3 * NJ + 2) * 32, s_);
      cp_async16(d + (3 * NJ + 3) * 32, s_ + 4);
    }
  };
  // tokens advance by nwarps: (b, n) are carried instead of divided per token
  const int64_t tok0 = (int64_t)blockIdx.x * kTokWarps + (threadIdx.x >> 5);
  const int step_b = (int)(nwarps / p.N), step_n = (int)(nwarps % p.N);
  int nb = (int)(tok0 / p.N), nn = (int)(tok0 % p.N);
  if (tok0 < total) prefetch(nb, nn, 0u);   // overlaps the weight staging below
  // The gate and blend of head fin_h are finalized by this lane once per
  // token: slot j = g of the token (g < NJ) belongs to that head.
  const int fin_i = lane + 32 * g;
  const bool fin_live = g < NJ && fin_i < slots;
  const int fin_h = fin_live ? fin_i / GL : 0;
  const float fin_gb = fin_live ? ld_any(p.gate_b, p.dt_gb, fin_h * p.sgb) : 0.f;
  const float fin_mb = !fin_live || p.mix_out == nullptr ? 0.f
                       : has_mix ? ld_any(p.mix_b, p.dt_mb, fin_h * p.smb) : ld_any(p.fixed_mix, p.dt_fm, fin_h * p.sfm);
  for (int i = threadIdx.x; i < H * 2 * D; i += blockDim.x) {
    const int hh = i / (2 * D), c = i % (2 * D);
    w_sm[(2 * hh) * PADROW + widx(c)] = ld_any(p.gate_w, p.dt_gw, hh * p.sgw[0] + c * p.sgw[1]);
    w_sm[(2 * hh + 1) * PADROW + widx(c)] = has_mix ? ld_any(p.mix_w, p.dt_mw, hh * p.smw[0] + c * p.smw[1]) : 0.f;
  }
  __syncthreads();
  for (int64_t tok = tok0; tok < total; tok += nwarps) {
    const int b = nb, n = nn;
    nn += step_n;
    nb += step_b;
    if (nn >= p.N) { nn -= p.N; ++nb; }
    T* qrow = reinterpret_cast<T*>(p.q) + b * p.sq[0] + (int64_t)n * p.sq[2];
    T* krow = reinterpret_cast<T*>(p.k) + b * p.sk[0] + (int64_t)n * p.sk[2];
    const int pos = pbase + n;
    const int prow = pos < 0 ? 0 : (pos < p.P ? pos : p.P - 1);
    cp_async_wait_all();   // this lane's copies of the token have landed
    // this lane's channels are the same for every head: one table row per token
    float csv[RMAX > 0 ? 8 : 1], snv[RMAX > 0 ? 8 : 1];
    uint32_t seen = 0;
    if constexpr (RMAX > 0) {
      if (p.rope && g < RMAX / 8) {
        if (tab_async) {
          const float4 c0 = *reinterpret_cast<const float4*>(stg + (3 * NJ + 0) * 32);
          const float4 c1 = *reinterpret_cast<const float4*>(stg + (3 * NJ + 1) * 32);
          const float4 s0 = *reinterpret_cast<const float4*>(stg + (3 * NJ + 2) * 32);
          const float4 s1 = *reinterpret_cast<const float4*>(stg + (3 * NJ + 3) * 32);
          csv[0] = c0.x; csv[1] = c0.y; csv[2] = c0.z; csv[3] = c0.w;
          csv[4] = c1.x; csv[5] = c1.y; csv[6] = c1.z; csv[7] = c1.w;
          snv[0] = s0.x; snv[1] = s0.y; snv[2] = s0.z; snv[3] = s0.w;
          snv[4] = s1.x; snv[5] = s1.y; snv[6] = s1.z; snv[7] = s1.w;
#pragma unroll
          for (int e = 0; e < 8; ++e) seen ^= __float_as_uint(csv[e]) ^ __float_as_uint(snv[e]);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            csv[e] = ld_any(p.cos, p.dt_cs, (int64_t)prow * p.scos[0] + (8 * g + e) * p.scos[1]);
            snv[e] = ld_any(p.sin, p.dt_cs, (int64_t)prow * p.ssin[0] + (8 * g + e) * p.ssin[1]);
          }
        }
      }
    }
    uint4 aq[NJ], ak[NJ], av[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int i = lane + 32 * j;
      aq[j] = ak[j] = av[j] = make_uint4(0, 0, 0, 0);
      if (i < slots) {
        aq[j] = stg[(0 * NJ + j) * 32];
        ak[j] = stg[(1 * NJ + j) * 32];
        if (p.cache_v != nullptr) av[j] = stg[(2 * NJ + j) * 32];
      }
      seen ^= aq[j].x ^ aq[j].y ^ aq[j].z ^ aq[j].w ^ ak[j].x ^ ak[j].y ^ ak[j].z ^ ak[j].w ^
              av[j].x ^ av[j].y ^ av[j].z ^ av[j].w;
    }
    // the next token's reads overwrite the stage only once every read above has returned
    if (tok + nwarps < total) prefetch(nb, nn, seen & p.zero);
    float fin_gs = 0.f, fin_ms = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      // keeps the weight reads of one slot from being hoisted above another's
      asm volatile("" ::: "memory");
      const int i = lane + 32 * j;
      const bool live = i < slots;
      const int hh = live ? i / GL : 0;
      uint4 uk = ak[j];
      const uint4 uv = av[j];
      Vec8<T> vq, vk;
      vq.w[0] = aq[j];
      vk.w[0] = uk;
      float fq[8], fk[8];
      vec8_to_f(vq, fq);
      vec8_to_f(vk, fk);
      // gate / blend partial dots of channels [8g, 8g + 8) on the un-rotated q, k
      const float* wg = w_sm + (2 * hh) * PADROW;
      const float* wm = wg + PADROW;
      float w[4][8];   // gate-q, gate-k, blend-q, blend-k weights of these channels
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const float* src = (v < 2 ? wg : wm) + widx((v & 1) * D + 8 * g);   // 8 values, 16-byte aligned
        const float4 a = *reinterpret_cast<const float4*>(src);
        const float4 c4 = *reinterpret_cast<const float4*>(src + 4);
        w[v][0] = a.x; w[v][1] = a.y; w[v][2] = a.z; w[v][3] = a.w;
        w[v][4] = c4.x; w[v][5] = c4.y; w[v][6] = c4.z; w[v][7] = c4.w;
      }
      float gs = 0.f, ms = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        gs = fmaf(fq[e], w[0][e], gs);
        gs = fmaf(fk[e], w[1][e], gs);
        ms = fmaf(fq[e], w[2][e], ms);
        ms = fmaf(fk[e], w[3][e], ms);
      }
#pragma unroll
      for (int o = 1; o < GL; o <<= 1) {
        gs += __shfl_xor_sync(0xffffffffu, gs, o);
        ms += __shfl_xor_sync(0xffffffffu, ms, o);
      }
      if (g == j) { fin_gs = gs; fin_ms = ms; }   // every lane of the group holds the sums
      // rotate-half RoPE of channels [0, R): the partner of channel c is c +- R/2
      if constexpr (RMAX > 0) {
        float pq[8], pk[8];
        if constexpr (RMAX >= 16) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            pq[e] = __shfl_xor_sync(0xffffffffu, fq[e], RMAX / 16);
            pk[e] = __shfl_xor_sync(0xffffffffu, fk[e], RMAX / 16);
          }
        }
        const bool in_r = live && g < RMAX / 8;
        if (in_r) {
          if (p.rope) {
            float rq[8], rk[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int c = 8 * g + e;
              const float cs = csv[e], sn = snv[e];
              float hq, hk;
              if constexpr (RMAX >= 16) {
                const bool lower = c < RMAX / 2;
                hq = lower ? -pq[e] : pq[e];
                hk = lower ? -pk[e] : pk[e];
              } else {   // R = 8: the partner is in this lane
                hq = e < 4 ? -fq[e + 4] : fq[e - 4];
                hk = e < 4 ? -fk[e + 4] : fk[e - 4];
              }
              rq[e] = fq[e] * cs + hq * sn;
              rk[e] = fk[e] * cs + hk * sn;
            }
            T tq[8], tk[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) { tq[e] = from_f<T>(rq[e]); tk[e] = from_f<T>(rk[e]); }
            *reinterpret_cast<uint4*>(qrow + 8 * i) = *reinterpret_cast<const uint4*>(tq);
            *reinterpret_cast<uint4*>(krow + 8 * i) = *reinterpret_cast<const uint4*>(tk);
            uk = *reinterpret_cast<const uint4*>(tk);
          }
          if (p.cache_k != nullptr && pos >= 0 && pos < p.L) {
            T* ck = reinterpret_cast<T*>(p.cache_k) + b * p.sck[0] + hh * p.sck[1] + (int64_t)pos * p.sck[2];
            *reinterpret_cast<uint4*>(ck + 8 * g) = uk;
          }
        }
      }
      if (live && p.cache_v != nullptr && pos >= 0 && pos < p.L) {
        T* cv = reinterpret_cast<T*>(p.cache_v) + b * p.scv[0] + hh * p.scv[1] + (int64_t)pos * p.scv[2];
        *reinterpret_cast<uint4*>(cv + 8 * g) = uv;
      }
    }
    if (fin_live) {
      const float gt = fin_gs + fin_gb;
      st_any(p.log_gamma, p.dt_lg, b * p.slg[0] + fin_h * p.slg[1] + (int64_t)n * p.slg[2],
             -(fmaxf(gt, 0.f) + log1pf(expf(-fabsf(gt)))));
      if (p.mix_out != nullptr) {
        const float mlog = (has_mix ? fin_ms : 0.f) + fin_mb;
        st_any(p.mix_out, p.dt_mo, b * p.smo[0] + fin_h * p.smo[1] + (int64_t)n * p.smo[2], 1.f / (1.f + expf(-mlog)));
      }
    }
  }
}

template <typename T>
cudaError_t launch_t(const PrepParams& p, cudaStream_t st) {
  if constexpr (sizeof(T) == 2) {
    // token-major kernel: each token's heads are adjacent (head stride D) in q, k and v
    const bool tok = p.vec && p.sq[1] == p.D && p.sk[1] == p.D && (p.cache_v == nullptr || p.sv[1] == p.D) &&
                     p.H * p.D <= kTokMaxElems && (p.R == 0 || p.R == 8 || p.R == 16 || p.R == 32 || p.R == 64);
    if (tok && !kPrepNoTokenMajor) {
      const size_t wbytes = (size_t)p.H * 2 * (2 * p.D + 2 * p.D / 8) * sizeof(float);
      const int sms = sm_count();
      // resident CTAs only (two per SM: registers), each walking its tokens with a grid stride
      const int64_t warps_needed = (int64_t)p.B * p.N;
      const int64_t blocks = std::min<int64_t>((warps_needed + kTokWarps - 1) / kTokWarps, (int64_t)sms * 2);
      PrepParams pk = p;
      pk.zero = 0;
      bool launched = true;
      const int nj = (p.H * p.D / 8 + 31) / 32;
#define HOFA_PREP_TOK_NJ(DD, RR, NJJ)                                                                          \
  {                                                                                                            \
    auto kk = prep_tok_kernel<T, DD, RR, NJJ>;                                                                 \
    const size_t smem = wbytes + (size_t)kTokWarps * tok_stage_bytes<NJJ, RR>();                              \
    if (smem > 48 * 1024) cudaFuncSetAttribute(kk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);    \
    kk<<<(unsigned)blocks, kTokWarps * 32, smem, st>>>(pk);                                                    \
  }
#define HOFA_PREP_TOK(DD, RR)                                                                                  \
  else if (p.D == DD && p.R == RR) {                                                                           \
    if (nj <= 1) HOFA_PREP_TOK_NJ(DD, RR, 1)                                                                   \
    else if (nj <= 2) HOFA_PREP_TOK_NJ(DD, RR, 2)                                                              \
    else HOFA_PREP_TOK_NJ(DD, RR, 4)                                                                           \
  }
      if (false) {}
      HOFA_PREP_TOK(64, 0) HOFA_PREP_TOK(64, 8) HOFA_PREP_TOK(64, 16) HOFA_PREP_TOK(64, 32) HOFA_PREP_TOK(64, 64)
      HOFA_PREP_TOK(128, 0) HOFA_PREP_TOK(128, 16) HOFA_PREP_TOK(128, 32) HOFA_PREP_TOK(128, 64)
      HOFA_PREP_TOK(32, 0) HOFA_PREP_TOK(32, 8) HOFA_PREP_TOK(32, 16) HOFA_PREP_TOK(32, 32)
      else launched = false;
#undef HOFA_PREP_TOK
#undef HOFA_PREP_TOK_NJ
      if (launched) return cudaGetLastError();
    }
    if (p.vec) {
      const dim3 grid((unsigned)((p.N + kVecThreads - 1) / kVecThreads), p.H, p.B);
      const int r = p.R;  // the outlier channels: rotated when p.rope, copied to cache_k either way
      bool launched = true;
#define HOFA_PREP_VEC(DD, RR) \
  else if (p.D == DD && r == RR) prep_vec_kernel<T, DD, RR><<<grid, 2 * kVecThreads, 0, st>>>(p);
      if (false) {}
      HOFA_PREP_VEC(64, 0) HOFA_PREP_VEC(64, 8) HOFA_PREP_VEC(64, 16) HOFA_PREP_VEC(64, 32)
      HOFA_PREP_VEC(128, 0) HOFA_PREP_VEC(128, 16) HOFA_PREP_VEC(128, 32) HOFA_PREP_VEC(128, 64)
      HOFA_PREP_VEC(32, 0) HOFA_PREP_VEC(32, 8) HOFA_PREP_VEC(32, 16)
      else launched = false;
#undef HOFA_PREP_VEC
      if (launched) return cudaGetLastError();
    }
  }
  const int64_t total = (int64_t)p.B * p.H * p.N;
  const dim3 grid((unsigned)((total + kPrepWarps - 1) / kPrepWarps));
  switch (p.D) {
    case 32: prep_kernel<T, 32><<<grid, kPrepWarps * 32, 0, st>>>(p); break;
    case 64: prep_kernel<T, 64><<<grid, kPrepWarps * 32, 0, st>>>(p); break;
    case 128: prep_kernel<T, 128><<<grid, kPrepWarps * 32, 0, st>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prep(const PrepParams& p, int dtype, cudaStream_t st) {
  switch (dtype) {
    case HOFA_DTYPE_BF16: return launch_t<__nv_bfloat16>(p, st);
    case HOFA_DTYPE_F16: return launch_t<__half>(p, st);
    default: return launch_t<float>(p, st);
  }
}

}  // namespace hofa
