// Fused HOFA decode: one launch per decode step.
//
// Replaces fused_hofa_decode (src/hofa_decode_triton.py:342-476), which runs
// either one (B,H) Triton program per head or a split kernel (B,H,split_k)
// plus a reduce kernel (B,H).  Here one grid (split_k, H, B) does everything:
//
//   * every CTA streams a contiguous slice of the (b,h) outlier cache
//     (K rows of R channels, V rows of D channels) with 16-byte loads: a warp
//     scores 32 tokens at a time (lane t owns token t's key row), keeps a
//     running softmax (max, sum) and accumulates p*V with each lane owning
//     8 value channels of a few tokens;
//   * the same CTA updates its share of the GLA state rows
//     (S' = gamma*S + k_I v^T, written to state_out) and the matching part of
//     the inclusive readout y_I = q_I S';
//   * partials (m, l, acc[D], y_I[D]) go to the workspace; the last CTA of a
//     (b,h) to arrive (atomic ticket, no spin-wait) combines them, applies
//     RMSNorm * gla_scale and the blend mix*y_O + (1-mix)*y_I_norm, writes Y
//     and re-arms the ticket for the next launch.
#include <float.h>

#include "common.cuh"
#include "kernels.h"

namespace hofa {

namespace {

constexpr int kDecThreads = 128;
constexpr int kDecWarps = kDecThreads / 32;

template <typename T, int D, bool VEC, bool ALPHA>
__global__ void __launch_bounds__(kDecThreads)
decode_kernel(const DecodeParams p) {
  constexpr int G = D / 8;        // 8-channel groups in one V row
  constexpr int TS = 32 / G;      // tokens covered by one warp-wide V load
  constexpr int VI = 32 / TS;     // V loads per lane for a 32-token tile
  constexpr int D4 = D / 4;       // float4 per state row
  constexpr int RSUB = kDecThreads / D4;

  const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int R = p.R, J = D - p.R;
  const int bh = b * p.H + h;

  __shared__ float sm_m[kDecWarps], sm_l[kDecWarps];
  __shared__ __align__(16) float sm_acc[kDecWarps][D];
  __shared__ __align__(16) float sm_y[RSUB][D];
  __shared__ float sm_red[kDecWarps];
  __shared__ __align__(16) float sm_q[D];
  __shared__ int sm_last;

  // ---------------- outlier softmax over this CTA's cache slice ----------
  int seq_len = p.seq_len;
  if (p.seq_len_dev != nullptr) {
    seq_len = *p.seq_len_dev;
    if (seq_len < 1 || seq_len > p.L) {
      if (s == 0 && tid == 0) atomicExch(p.ws_status, 1);
      seq_len = seq_len < 1 ? 1 : p.L;
    }
  }
  if (R == 0) seq_len = 0;
  int tps = (seq_len + p.split_k - 1) / p.split_k;
  tps = (tps + 31) & ~31;
  const int t_begin = s * tps;
  const int t_end = min(seq_len, t_begin + tps);

  // q_O pre-scaled to the base-2 logit domain; read by every lane (broadcast)
  if (tid < D) {
    sm_q[tid] = (tid < R) ? to_f(reinterpret_cast<const T*>(p.q)[b * p.sq[0] + h * p.sq[1] + tid * p.sq[2]]) *
                                p.qk_scale_log2
                          : 0.f;
  }
  __syncthreads();

  const int cg = lane % G, ts = lane / G;
  float m_run = -INFINITY, l_run = 0.f;
  float acc[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) acc[c] = 0.f;

  const T* kb = reinterpret_cast<const T*>(p.cache_k) + b * p.sck[0] + h * p.sck[1];
  const T* vb = reinterpret_cast<const T*>(p.cache_v) + b * p.scv[0] + h * p.scv[1];

  for (int t0 = t_begin + warp * 32; t0 < t_end; t0 += kDecWarps * 32) {
    const int t = t0 + lane;
    const bool valid = t < t_end;
    // value loads first: they do not depend on the scores
    Vec8<T> vr[VI];
#pragma unroll
    for (int i = 0; i < VI; ++i) {
      const int tv = t0 + i * TS + ts;
      if (tv < t_end) {
        if constexpr (VEC) vr[i] = ld_vec8<T>(vb + (int64_t)tv * p.scv[2] + cg * 8);
        else vr[i] = ld_strided8<T>(vb + (int64_t)tv * p.scv[2] + (int64_t)cg * 8 * p.scv[3], p.scv[3]);
      } else {
        vr[i] = zero_vec8<T>();
      }
    }
    float sc = -INFINITY;
    if (valid) {
      float dot = 0.f;
      if constexpr (VEC) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
          if (g * 8 < R) {
            float f[8];
            vec8_to_f(ld_vec8<T>(kb + (int64_t)t * p.sck[2] + g * 8), f);
#pragma unroll
            for (int c = 0; c < 8; ++c) dot = fmaf(sm_q[g * 8 + c], f[c], dot);
          }
        }
      } else {
#pragma unroll
        for (int c = 0; c < D; ++c)
          if (c < R) dot = fmaf(sm_q[c], to_f(kb[(int64_t)t * p.sck[2] + (int64_t)c * p.sck[3]]), dot);
      }
      sc = dot;
    }
    const float mt = warp_max(sc);
    const float mn = fmaxf(m_run, mt);
    const float corr = exp2f(m_run - mn);
    const float pl = exp2f(sc - mn);
    l_run = l_run * corr + pl;
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] *= corr;
#pragma unroll
    for (int i = 0; i < VI; ++i) {
      const float pi = __shfl_sync(0xffffffffu, pl, i * TS + ts);
      float f[8];
      vec8_to_f(vr[i], f);
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[c] = fmaf(pi, f[c], acc[c]);
    }
    m_run = mn;
  }
  // lanes sharing a channel group hold disjoint tokens: sum them
#pragma unroll
  for (int o = G; o < 32; o <<= 1) {
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], o);
  }
  l_run = warp_sum(l_run);
  if (lane < G) {
#pragma unroll
    for (int c = 0; c < 8; ++c) sm_acc[warp][lane * 8 + c] = acc[c];
  }
  if (lane == 0) { sm_m[warp] = m_run; sm_l[warp] = l_run; }

  // ---------------- GLA rows owned by this split --------------------------
  const int rows_per = (J + p.split_k - 1) / p.split_k;
  const int r0 = s * rows_per, r1 = min(J, r0 + rows_per);
  const int c4 = tid % D4, rsub = tid / D4;
  float ya[4] = {0.f, 0.f, 0.f, 0.f};
  if (r0 < r1) {
    const T* qp = reinterpret_cast<const T*>(p.q) + b * p.sq[0] + h * p.sq[1];
    const T* kp = reinterpret_cast<const T*>(p.k) + b * p.sk[0] + h * p.sk[1];
    const T* vp = reinterpret_cast<const T*>(p.v) + b * p.sv[0] + h * p.sv[1];
    float v4[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) v4[c] = to_f(vp[(int64_t)(4 * c4 + c) * p.sv[2]]);
    const float lg = ld_any(p.log_gamma, p.dt_lg, b * p.slg[0] + h * p.slg[1]);
    const float gam_h = expf(lg);
    const float* sin_ = p.state_in + b * p.sst[0] + h * p.sst[1];
    float* sout = p.state_out + b * p.sso[0] + h * p.sso[1];
    for (int row = r0 + rsub; row < r1; row += RSUB) {
      const float kr = to_f(kp[(int64_t)(R + row) * p.sk[2]]);
      const float qr = to_f(qp[(int64_t)(R + row) * p.sq[2]]);
      float gam = gam_h;
      if constexpr (ALPHA) gam = expf(lg * expf(ld_any(p.log_alpha, p.dt_la, b * p.sla[0] + h * p.sla[1] + row * p.sla[2])));
      const float4 s4 = *reinterpret_cast<const float4*>(sin_ + (int64_t)row * p.sst[2] + 4 * c4);
      float4 n4;
      n4.x = fmaf(gam, s4.x, kr * v4[0]);
      n4.y = fmaf(gam, s4.y, kr * v4[1]);
      n4.z = fmaf(gam, s4.z, kr * v4[2]);
      n4.w = fmaf(gam, s4.w, kr * v4[3]);
      *reinterpret_cast<float4*>(sout + (int64_t)row * p.sso[2] + 4 * c4) = n4;
      ya[0] = fmaf(qr, n4.x, ya[0]);
      ya[1] = fmaf(qr, n4.y, ya[1]);
      ya[2] = fmaf(qr, n4.z, ya[2]);
      ya[3] = fmaf(qr, n4.w, ya[3]);
    }
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) sm_y[rsub][4 * c4 + c] = ya[c];
  __syncthreads();

  // ---------------- CTA partial: (m, l, acc[D], y_I[D]) -------------------
  float cta_m = -INFINITY;
#pragma unroll
  for (int w = 0; w < kDecWarps; ++w) cta_m = fmaxf(cta_m, sm_m[w]);
  float cta_l = 0.f, part_acc = 0.f, part_y = 0.f;
  const int d = tid;
#pragma unroll
  for (int w = 0; w < kDecWarps; ++w) {
    const float wgt = (sm_m[w] == -INFINITY) ? 0.f : exp2f(sm_m[w] - cta_m);
    cta_l += sm_l[w] * wgt;
    if (d < D) part_acc += sm_acc[w][d] * wgt;
  }
  if (d < D) {
#pragma unroll
    for (int rr = 0; rr < RSUB; ++rr) part_y += sm_y[rr][d];
  }

  float fin_acc, fin_l, fin_y, fin_m;
  if (p.split_k == 1) {
    fin_acc = part_acc; fin_l = cta_l; fin_y = part_y; fin_m = cta_m;
  } else {
    const int PS = 4 + 2 * D;
    float* part = p.ws_part + ((int64_t)bh * p.split_k + s) * PS;
    if (tid == 0) { part[0] = cta_m; part[1] = cta_l; }
    if (d < D) { part[4 + d] = part_acc; part[4 + D + d] = part_y; }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int prev = atomicAdd(p.ws_count + bh, 1);
      sm_last = (prev == p.split_k - 1);
    }
    __syncthreads();
    if (!sm_last) return;
    __threadfence();
    const float* all = p.ws_part + (int64_t)bh * p.split_k * PS;
    float M = -INFINITY;
    for (int q = 0; q < p.split_k; ++q) M = fmaxf(M, __ldcg(all + q * PS));
    fin_acc = 0.f; fin_l = 0.f; fin_y = 0.f; fin_m = M;
    for (int q = 0; q < p.split_k; ++q) {
      const float mq = __ldcg(all + q * PS);
      const float wgt = (mq == -INFINITY) ? 0.f : exp2f(mq - M);
      fin_l += __ldcg(all + q * PS + 1) * wgt;
      if (d < D) {
        fin_acc += __ldcg(all + q * PS + 4 + d) * wgt;
        fin_y += __ldcg(all + q * PS + 4 + D + d);
      }
    }
    if (tid == 0) p.ws_count[bh] = 0;  // re-arm the ticket for the next launch
  }
  (void)fin_m;

  // ---------------- RMSNorm(y_I) * gla_scale, blend, store ---------------
  float sq = (d < D) ? fin_y * fin_y : 0.f;
  sq = warp_sum(sq);
  if (lane == 0) sm_red[warp] = sq;
  __syncthreads();
  float ss = 0.f;
#pragma unroll
  for (int w = 0; w < kDecWarps; ++w) ss += sm_red[w];
  if (d < D) {
    const float rs = rsqrtf(ss / (float)D + p.eps);
    const float nw = ld_any(p.norm_w, p.dt_nw, h * p.snw[0] + d * p.snw[1]);
    const float mix = ld_any(p.mix_g, p.dt_mg, b * p.smg[0] + h * p.smg[1]);
    const float yo = fin_l > 0.f ? fin_acc / fin_l : 0.f;
    const float out = mix * yo + (1.f - mix) * (fin_y * rs * nw);
    reinterpret_cast<T*>(p.y)[b * p.sy[0] + h * p.sy[1] + d * p.sy[2]] = from_f<T>(out);
  }
}

template <typename T, int D>
cudaError_t launch_d(const DecodeParams& p, bool vec, bool alpha, cudaStream_t st) {
  dim3 grid(p.split_k, p.H, p.B);
  if (vec) {
    if (alpha) decode_kernel<T, D, true, true><<<grid, kDecThreads, 0, st>>>(p);
    else decode_kernel<T, D, true, false><<<grid, kDecThreads, 0, st>>>(p);
  } else {
    if (alpha) decode_kernel<T, D, false, true><<<grid, kDecThreads, 0, st>>>(p);
    else decode_kernel<T, D, false, false><<<grid, kDecThreads, 0, st>>>(p);
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_t(const DecodeParams& p, bool vec, bool alpha, cudaStream_t st) {
  switch (p.D) {
    case 32: return launch_d<T, 32>(p, vec, alpha, st);
    case 64: return launch_d<T, 64>(p, vec, alpha, st);
    case 128: return launch_d<T, 128>(p, vec, alpha, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_decode(const DecodeParams& p, int dtype, bool vec, bool alpha, cudaStream_t st) {
  switch (dtype) {
    case HOFA_DTYPE_BF16: return launch_t<__nv_bfloat16>(p, vec, alpha, st);
    case HOFA_DTYPE_F16: return launch_t<__half>(p, vec, alpha, st);
    default: return launch_t<float>(p, vec, alpha, st);
  }
}

}  // namespace hofa
