// Fused HOFA decode: one launch per decode step.
//
// Replaces fused_hofa_decode (src/hofa_decode_triton.py:342-476), which runs
// either one (B,H) Triton program per head or a split kernel (B,H,split_k)
// plus a reduce kernel (B,H).  Here one grid (split_k, H, B) does everything:
//
//   * every CTA streams a contiguous slice of the (b,h) outlier cache (K rows
//     of R channels, V rows of D channels).  A warp scores 32 tokens at a time
//     (lane t owns token t's key row), keeps a running softmax (max, sum) and
//     accumulates p*V with each lane owning 8 value channels of a few tokens;
//   * the same CTA updates its share of the GLA state rows
//     (S' = gamma*S + k_I v^T, written to state_out) and the matching part of
//     the inclusive readout y_I = q_I S';
//   * partials (m, l, acc[D], y_I[D]) go to the workspace; the last CTA of a
//     (b,h) to arrive (atomic ticket, no spin-wait) combines them, applies
//     RMSNorm * gla_scale and the blend mix*y_O + (1-mix)*y_I_norm, writes Y
//     and re-arms the ticket for the next launch.
//
// Two cache-streaming variants share that structure:
//   decode_bulk_kernel  -- cache rows contiguous in memory (the layer's
//       pre-allocated [B,H,L,*] caches): a producer warp streams 64-token
//       chunks with 1-D TMA bulk copies (cp.async.bulk) into an 8-stage
//       shared-memory ring guarded by mbarriers, four consumer warps reduce
//       them; up to 80 KB per CTA is in flight.  The splits of a head run as
//       one thread-block cluster and combine through distributed shared
//       memory.
//   decode_reg_kernel   -- any strides: 16-byte (or scalar) register loads.
#include <float.h>
#include <cstdlib>

#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace cg = cooperative_groups;

namespace hofa {

namespace {

constexpr int kConsumerWarps = 4;              // warps of the register-load kernel; the GLA-row
constexpr int kConsumers = kConsumerWarps * 32;  // mapping always uses the first 128 threads
constexpr int kMaxWarps = 8;                     // consumer warps of the bulk kernel (4 or 8)
constexpr int kMaxStages = 16;
constexpr int kChunk = 32;           // tokens per warp tile
constexpr int kMaxClusterSplit = 16;  // splits combined through a thread-block cluster

struct DecShared {
  float m[kMaxWarps], l[kMaxWarps];
  float red[kMaxWarps + 2];
  int last;
};

// Online-softmax update of one warp with a 32-token tile: `sc` is this
// lane's score (log2 domain, -inf when invalid); vr[i] holds V channels
// [8cg, 8cg+8) of token i*TS+ts of the tile.
template <typename T, int D>
__device__ __forceinline__ void tile_update(float sc, const Vec8<T> (&vr)[D / 8], float& m_run, float& l_run,
                                            float (&acc)[8], int ts) {
  constexpr int G = D / 8, TS = 32 / G, VI = 32 / TS;
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

// Warp result -> shared (acc summed over the lanes that share a channel group).
template <int D>
__device__ __forceinline__ void warp_flush(float m_run, float l_run, float (&acc)[8], int lane, int warp,
                                          DecShared& sh, float (*sm_acc)[D]) {
  constexpr int G = D / 8;
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
  if (lane == 0) { sh.m[warp] = m_run; sh.l[warp] = l_run; }
}

// GLA rows [r0, r1) of (b,h): S' = gamma*S + k_I v^T -> state_out, and this
// split's part of y_I = q_I S' -> sm_y (one row of partial sums per group of
// D/4 threads).  Run by NT threads with indices t in [0, NT).
template <typename T, int D, bool ALPHA, int NT>
__device__ __forceinline__ void gla_rows(const DecodeParams& p, int s, int b, int h, int t, float (*sm_y)[D],
                                         const float* lg_smem = nullptr) {
  constexpr int D4 = D / 4;
  constexpr int RSUB = NT / D4;
  const int R = p.R, J = D - p.R;
  const int rows_per = (J + p.split_k - 1) / p.split_k;
  const int r0 = s * rows_per, r1 = min(J, r0 + rows_per);
  const int c4 = t % D4, rsub = t / D4;
  float ya[4] = {0.f, 0.f, 0.f, 0.f};
  if (r0 < r1) {
    const T* qp = reinterpret_cast<const T*>(p.q) + b * p.sq[0] + h * p.sq[1];
    const T* kp = reinterpret_cast<const T*>(p.k) + b * p.sk[0] + h * p.sk[1];
    const T* vp = reinterpret_cast<const T*>(p.v) + b * p.sv[0] + h * p.sv[1];
    float v4[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) v4[c] = to_f(vp[(int64_t)(4 * c4 + c) * p.sv[2]]);
    const float lg = lg_smem != nullptr ? *lg_smem : ld_any(p.log_gamma, p.dt_lg, b * p.slg[0] + h * p.slg[1]);
    const float gam_h = expf(lg);
    const float* sin_ = p.state_in + b * p.sst[0] + h * p.sst[1];
    float* sout = p.state_out + b * p.sso[0] + h * p.sso[1];
    // Batches of up to four rows per thread: every load of a batch is issued
    // before its first store (a store to state_out could alias a later
    // state_in load as far as the compiler knows, which would otherwise
    // serialise one memory round trip per row).
    constexpr int BAT = 4;
    for (int base = r0 + rsub; base < r1; base += BAT * RSUB) {
      float kr[BAT], qr[BAT], la[BAT];
      float4 s4[BAT];
#pragma unroll
      for (int u = 0; u < BAT; ++u) {
        const int row = base + u * RSUB;
        if (row < r1) {
          kr[u] = to_f(kp[(int64_t)(R + row) * p.sk[2]]);
          qr[u] = to_f(qp[(int64_t)(R + row) * p.sq[2]]);
          s4[u] = __ldg(reinterpret_cast<const float4*>(sin_ + (int64_t)row * p.sst[2] + 4 * c4));
          if constexpr (ALPHA) la[u] = ld_any(p.log_alpha, p.dt_la, b * p.sla[0] + h * p.sla[1] + row * p.sla[2]);
        }
      }
#pragma unroll
      for (int u = 0; u < BAT; ++u) {
        const int row = base + u * RSUB;
        if (row < r1) {
          float gam = gam_h;
          if constexpr (ALPHA) gam = expf(lg * expf(la[u]));
          float4 n4;
          n4.x = fmaf(gam, s4[u].x, kr[u] * v4[0]);
          n4.y = fmaf(gam, s4[u].y, kr[u] * v4[1]);
          n4.z = fmaf(gam, s4[u].z, kr[u] * v4[2]);
          n4.w = fmaf(gam, s4[u].w, kr[u] * v4[3]);
          *reinterpret_cast<float4*>(sout + (int64_t)row * p.sso[2] + 4 * c4) = n4;
          ya[0] = fmaf(qr[u], n4.x, ya[0]);
          ya[1] = fmaf(qr[u], n4.y, ya[1]);
          ya[2] = fmaf(qr[u], n4.z, ya[2]);
          ya[3] = fmaf(qr[u], n4.w, ya[3]);
        }
      }
    }
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) sm_y[rsub][4 * c4 + c] = ya[c];
}

// norm_w[h, d] and mix[b, h] for the epilogue, read at the start of a kernel
// (after the grid dependency) so that the epilogue does no global round trip.
struct EpiloguePrefetch {
  float nw = 0.f, mix = 0.f;
};
template <int D>
__device__ __forceinline__ EpiloguePrefetch prefetch_epilogue(const DecodeParams& p, int b, int h, int d) {
  EpiloguePrefetch e;
  if (d < D) {
    e.nw = ld_any(p.norm_w, p.dt_nw, h * p.snw[0] + d * p.snw[1]);
    if (!p.fused_prep) e.mix = ld_any(p.mix_g, p.dt_mg, b * p.smg[0] + h * p.smg[1]);  // fused: computed here
  }
  return e;
}

// CTA partial (m, l, acc[D], y_I[D]), cross-split combine, RMSNorm, blend,
// store.  Called by every thread of the CTA after a __syncthreads() that
// publishes sh / sm_acc / sm_y.  The splits of one (b,h) combine either
//   CLUSTER: the split CTAs of a head form one thread-block cluster; each
//            leaves its partial in shared memory, rank 0 reads the peers'
//            partials through distributed shared memory (no global round
//            trip, no fences, no atomics), or
//   workspace: partials go to global memory and the last CTA to take a
//            ticket combines them (any split count).
template <typename T, int D, bool CLUSTER, int NW, int RSUB>
__device__ __forceinline__ void finish(const DecodeParams& p, int s, int b, int h, int tid, int lane, int warp,
                                       int nwarps, DecShared& sh, float (*sm_acc)[D], float (*sm_y)[D],
                                       float (*sm_all)[4 + 2 * D], uint64_t* comb_bar, EpiloguePrefetch ep,
                                       const float* newtok = nullptr) {
  constexpr int PS = 4 + 2 * D;
  const int bh = b * p.H + h;
  float cta_m = -INFINITY;
#pragma unroll
  for (int w = 0; w < NW; ++w) cta_m = fmaxf(cta_m, sh.m[w]);
  float cta_l = 0.f, part_acc = 0.f, part_y = 0.f;
  const int d = tid;
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    const float wgt = (sh.m[w] == -INFINITY) ? 0.f : exp2f(sh.m[w] - cta_m);
    cta_l += sh.l[w] * wgt;
    if (d < D) part_acc += sm_acc[w][d] * wgt;
  }
  if (d < D) {
#pragma unroll
    for (int rr = 0; rr < RSUB; ++rr) part_y += sm_y[rr][d];
  }

  float fin_acc, fin_l, fin_y, M_fin = cta_m;
  if (p.split_k == 1) {
    fin_acc = part_acc; fin_l = cta_l; fin_y = part_y;
  } else if constexpr (CLUSTER) {
    // every other split CTA sends its partial into rank 0's sm_all[rank] with
    // st.async stores whose bytes complete on rank 0's comb_bar (rank 0
    // expects (split_k - 1) partials' bytes from kernel start), then exits
    // without waiting; rank 0 adds its own arrival and waits once.
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t rank = cluster.block_rank();
    sm100::cluster_wait();  // rank 0's comb_bar and its expected bytes are in place
    if (rank != 0) {
      const uint32_t rbar = sm100::mapa_shared(comb_bar, 0);
      const uint32_t rslot = sm100::mapa_shared(&sm_all[rank][0], 0);
      if (tid == 0) {
        sm100::st_async_f32(rslot, cta_m, rbar);
        sm100::st_async_f32(rslot + 4, cta_l, rbar);
      }
      if (d < D) {
        sm100::st_async_f32(rslot + 4 * (4 + d), part_acc, rbar);
        sm100::st_async_f32(rslot + 4 * (4 + D + d), part_y, rbar);
      }
      return;
    }
    if (tid == 0) { sm_all[0][0] = cta_m; sm_all[0][1] = cta_l; }
    if (d < D) { sm_all[0][4 + d] = part_acc; sm_all[0][4 + D + d] = part_y; }
    if (tid == 0) sm100::mbar_arrive(comb_bar);
    __syncthreads();
    if (!sm100::mbar_wait_cluster(comb_bar, 0) && tid == 0) atomicOr(p.ws_status, 64);
    float M = -INFINITY;
    for (int q = 0; q < p.split_k; ++q) M = fmaxf(M, sm_all[q][0]);
    M_fin = M;
    fin_acc = 0.f; fin_l = 0.f; fin_y = 0.f;
#pragma unroll 4
    for (int q = 0; q < p.split_k; ++q) {
      const float mq = sm_all[q][0];
      const float wgt = (mq == -INFINITY) ? 0.f : exp2f(mq - M);
      fin_l += sm_all[q][1] * wgt;
      if (d < D) {
        fin_acc += sm_all[q][4 + d] * wgt;
        fin_y += sm_all[q][4 + D + d];
      }
    }
  } else {
    float* part = p.ws_part + ((int64_t)bh * p.split_k + s) * PS;
    if (tid == 0) { part[0] = cta_m; part[1] = cta_l; }
    if (d < D) { part[4 + d] = part_acc; part[4 + D + d] = part_y; }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int prev = atomicAdd(p.ws_count + bh, 1);
      sh.last = (prev == p.split_k - 1);
    }
    __syncthreads();
    if (!sh.last) return;
    __threadfence();
    const float* all = p.ws_part + (int64_t)bh * p.split_k * PS;
    float M = -INFINITY;
#pragma unroll 8
    for (int q = 0; q < p.split_k; ++q) M = fmaxf(M, __ldcg(all + q * PS));
    M_fin = M;
    fin_acc = 0.f; fin_l = 0.f; fin_y = 0.f;
#pragma unroll 8
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

  if (newtok != nullptr) {
    // the new token (score newtok[4] + newtok[5], value newtok[16 + d]) joins the softmax
    const float sn = newtok[4] + newtok[5];
    const float M2 = fmaxf(M_fin, sn);
    const float wo = M_fin == -INFINITY ? 0.f : exp2f(M_fin - M2);
    const float wn = exp2f(sn - M2);
    fin_l = fin_l * wo + wn;
    if (d < D) fin_acc = fin_acc * wo + wn * newtok[16 + d];
    ep.mix = newtok[2];
  }
  float sq = (d < D) ? fin_y * fin_y : 0.f;
  sq = warp_sum(sq);
  if (lane == 0) sh.red[warp] = sq;
  __syncthreads();
  float ss = 0.f;
  for (int w = 0; w < nwarps; ++w) ss += sh.red[w];
  if (d < D) {
    const float rs = rsqrtf(ss / (float)D + p.eps);
    const float yo = fin_l > 0.f ? fin_acc / fin_l : 0.f;
    const float out = ep.mix * yo + (1.f - ep.mix) * (fin_y * rs * ep.nw);
    reinterpret_cast<T*>(p.y)[b * p.sy[0] + h * p.sy[1] + d * p.sy[2]] = from_f<T>(out);
  }
}

__device__ __forceinline__ int resolve_seq_len(const DecodeParams& p, int s, int tid) {
  int seq_len = p.seq_len;
  if (p.seq_len_dev != nullptr) {
    seq_len = *p.seq_len_dev;
    if (seq_len < 1 || seq_len > p.L) {
      if (s == 0 && tid == 0) atomicOr(p.ws_status, 1);
      seq_len = seq_len < 1 ? 1 : p.L;
    }
  }
  return p.R == 0 ? 0 : seq_len;
}

template <typename T, int D>
__device__ __forceinline__ void load_q(const DecodeParams& p, int b, int h, int tid, float* sm_q) {
  if (tid < D) {
    sm_q[tid] = (tid < p.R) ? to_f(reinterpret_cast<const T*>(p.q)[b * p.sq[0] + h * p.sq[1] + tid * p.sq[2]]) *
                                  p.qk_scale_log2
                            : 0.f;
  }
}

// ============================================================================
// Register-load variant (any strides).
// ============================================================================
template <typename T, int D, bool VEC, bool ALPHA>
__global__ void __launch_bounds__(kConsumers)
decode_reg_kernel(const DecodeParams p) {
  constexpr int G = D / 8, TS = 32 / G, VI = 32 / TS;
  constexpr int RSUB = kConsumers / (D / 4);
  const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int R = p.R;

  __shared__ DecShared sh;
  __shared__ __align__(16) float sm_acc[kConsumerWarps][D];
  __shared__ __align__(16) float sm_y[RSUB][D];
  __shared__ __align__(16) float sm_q[D];

  const int seq_len = resolve_seq_len(p, s, tid);
  int tps = (seq_len + p.split_k - 1) / p.split_k;
  tps = (tps + kChunk - 1) & ~(kChunk - 1);
  const int t_begin = s * tps;
  const int t_end = min(seq_len, t_begin + tps);
  load_q<T, D>(p, b, h, tid, sm_q);
  const EpiloguePrefetch ep = prefetch_epilogue<D>(p, b, h, tid);
  __syncthreads();

  const int cg = lane % G, ts = lane / G;
  float m_run = -INFINITY, l_run = 0.f;
  float acc[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) acc[c] = 0.f;
  const T* kb = reinterpret_cast<const T*>(p.cache_k) + b * p.sck[0] + h * p.sck[1];
  const T* vb = reinterpret_cast<const T*>(p.cache_v) + b * p.scv[0] + h * p.scv[1];

  for (int t0 = t_begin + warp * kChunk; t0 < t_end; t0 += kConsumerWarps * kChunk) {
    const int t = t0 + lane;
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
    if (t < t_end) {
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
        for (int c = 0; c < R; ++c) dot = fmaf(sm_q[c], to_f(kb[(int64_t)t * p.sck[2] + (int64_t)c * p.sck[3]]), dot);
      }
      sc = dot;
    }
    tile_update<T, D>(sc, vr, m_run, l_run, acc, ts);
  }
  warp_flush<D>(m_run, l_run, acc, lane, warp, sh, sm_acc);
  gla_rows<T, D, ALPHA, kConsumers>(p, s, b, h, tid, sm_y);
  __syncthreads();
  finish<T, D, false, kConsumerWarps, RSUB>(p, s, b, h, tid, lane, warp, kConsumerWarps, sh, sm_acc, sm_y, nullptr,
                                            nullptr, ep);
}

// ============================================================================
// TMA-bulk variant (cache rows contiguous: row stride R for K, D for V).
// ============================================================================
// The new token of a fused decode step (consumer threads, tid < NW * 32):
// gate = q.Wg[h,:D] + k.Wg[h,D:] + bg on the un-rotated q, k; log decay =
// logsigmoid(-gate); mix = sigmoid(q.Wm[h,:D] + k.Wm[h,D:] + bm) (or of the
// fixed blend logit) rounded to the activation dtype; rotate-half RoPE of
// channels [0, R) at position pos, rounded to the activation dtype as the
// separate prep kernel stores them; q -> sm_q (scaled), the new score's
// partial sums -> sm_pre[4..6), v -> sm_pre[16..); split 0 appends the cache
// row and writes the optional log_gamma / mix outputs.
template <typename T, int D, int NW>
__device__ __forceinline__ void prep_new_token(const DecodeParams& p, int s, int b, int h, int tid, int lane,
                                               int warp, int pos, float* sm_q, float* sm_pre) {
  const int R = p.R;
  float gp = 0.f, mp = 0.f;
  if (tid < D) {
    const float qf = to_f(reinterpret_cast<const T*>(p.q)[b * p.sq[0] + h * p.sq[1] + tid * p.sq[2]]);
    const float kf = to_f(reinterpret_cast<const T*>(p.k)[b * p.sk[0] + h * p.sk[1] + tid * p.sk[2]]);
    const float vf = to_f(reinterpret_cast<const T*>(p.v)[b * p.sv[0] + h * p.sv[1] + tid * p.sv[2]]);
    gp = fmaf(qf, ld_any(p.gate_w, p.dt_gw, h * p.sgw[0] + tid * p.sgw[1]),
              kf * ld_any(p.gate_w, p.dt_gw, h * p.sgw[0] + (D + tid) * p.sgw[1]));
    if (p.mix_w != nullptr)
      mp = fmaf(qf, ld_any(p.mix_w, p.dt_mw, h * p.smw[0] + tid * p.smw[1]),
                kf * ld_any(p.mix_w, p.dt_mw, h * p.smw[0] + (D + tid) * p.smw[1]));
    sm_pre[16 + tid] = vf;
    sm_pre[16 + D + tid] = qf;
    sm_pre[16 + 2 * D + tid] = kf;
  }
  gp = warp_sum(gp);
  mp = warp_sum(mp);
  if (lane == 0 && warp < (D + 31) / 32) { sm_pre[8 + warp] = gp; sm_pre[12 + warp] = mp; }
  asm volatile("bar.sync 1, %0;" ::"n"(NW * 32) : "memory");  // consumers only
  float g = ld_any(p.gate_b, p.dt_gb, h * p.sgb);
  float ml = p.mix_w != nullptr ? ld_any(p.mix_b, p.dt_mb, h * p.smb) : ld_any(p.fixed_mix, p.dt_fm, h * p.sfm);
#pragma unroll
  for (int w = 0; w < (D + 31) / 32; ++w) {
    g += sm_pre[8 + w];
    if (p.mix_w != nullptr) ml += sm_pre[12 + w];
  }
  const float lg = -(fmaxf(g, 0.f) + log1pf(expf(-fabsf(g))));
  const float mixv = to_f(from_f<T>(1.f / (1.f + expf(-ml))));
  float prod = 0.f;
  if (tid < R) {
    const int half = R / 2;
    const float qf = sm_pre[16 + D + tid], kf = sm_pre[16 + 2 * D + tid];
    const float qh = tid < half ? -sm_pre[16 + D + tid + half] : sm_pre[16 + D + tid - half];
    const float kh = tid < half ? -sm_pre[16 + 2 * D + tid + half] : sm_pre[16 + 2 * D + tid - half];
    float cs = 1.f, sn = 0.f;
    if (p.rope_rows > 0) {
      const int prow = pos < 0 ? 0 : (pos < p.rope_rows ? pos : p.rope_rows - 1);
      cs = ld_any(p.rope_cos, p.dt_cs, (int64_t)prow * p.scos[0] + tid * p.scos[1]);
      sn = ld_any(p.rope_sin, p.dt_cs, (int64_t)prow * p.ssin[0] + tid * p.ssin[1]);
    }
    const T qr = from_f<T>(qf * cs + qh * sn), kr = from_f<T>(kf * cs + kh * sn);
    sm_q[tid] = to_f(qr) * p.qk_scale_log2;
    prod = sm_q[tid] * to_f(kr);
    if (s == 0) reinterpret_cast<T*>(const_cast<void*>(p.cache_k))[b * p.sck[0] + h * p.sck[1] + (int64_t)pos * p.sck[2] + tid * p.sck[3]] = kr;
  } else if (tid < D) {
    sm_q[tid] = 0.f;
  }
  if (s == 0 && tid < D)
    reinterpret_cast<T*>(const_cast<void*>(p.cache_v))[b * p.scv[0] + h * p.scv[1] + (int64_t)pos * p.scv[2] + tid * p.scv[3]] =
        from_f<T>(sm_pre[16 + tid]);
  prod = warp_sum(prod);
  if (lane == 0 && warp < 2) sm_pre[4 + warp] = prod;
  if (tid == 0) {
    sm_pre[1] = lg;
    sm_pre[2] = mixv;
    if (s == 0 && p.log_gamma_out != nullptr) st_any(p.log_gamma_out, p.dt_lgo, b * p.slgo[0] + h * p.slgo[1], lg);
    if (s == 0 && p.mix_out != nullptr) st_any(p.mix_out, p.dt_mo, b * p.smo[0] + h * p.smo[1], mixv);
  }
}

constexpr int kBulkChunk = 64;  // tokens per bulk chunk (two warp tiles)

// Warps: NW consumers, then the TMA producer (warp NW), then the GLA warp
// (warp NW + 1), which updates this split's GLA state rows and its part of
// y_I while the consumers stream the cache.
//
// PREP (hofa_decode_step_fwd): the consumers first compute the new token's
// gates and RoPE (the layer's prep step, src/HybridOutlierFactorizedAttention.py
// :360-392) into sm_pre, split 0 appends its cache row, the GLA warp waits for
// the log decay (named barrier 2), the stream covers rows [0, seq_len - 1) and
// the new token joins the softmax in finish().
template <typename T, int D, bool ALPHA, bool CLUSTER, int NW, bool PREP>
__global__ void __launch_bounds__(NW * 32 + 64)
decode_bulk_kernel(const DecodeParams p) {
  constexpr int G = D / 8, TS = 32 / G, VI = 32 / TS;
  constexpr int RSUB = 32 / (D / 4);   // rows of sm_y written by the GLA warp
  const int NST = p.stages;
  const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int R = p.R;

  __shared__ DecShared sh;
  __shared__ __align__(16) float sm_acc[NW][D];
  __shared__ __align__(16) float sm_y[RSUB][D];
  __shared__ __align__(16) float sm_q[D];
  __shared__ __align__(16) float sm_all[CLUSTER ? kMaxClusterSplit : 1][4 + 2 * D];  // split partials (rank 0's)
  __shared__ __align__(8) uint64_t full_bar[kMaxStages], empty_bar[kMaxStages];
  __shared__ __align__(8) uint64_t comb_bar;
  __shared__ float sm_ep[D + 1];   // norm_w[h, :] and the blend weight, for the epilogue
  // PREP: [1] log decay, [2] mix, [4..6) new-token score partials, [8..12) / [12..16)
  // gate / mix dot partials, [16, 16+D) v, [16+D, 16+2D) q, [16+2D, 16+3D) k
  __shared__ __align__(16) float sm_pre[PREP ? 16 + 3 * D : 1];
  __shared__ int sm_err;
  extern __shared__ __align__(128) unsigned char ring[];  // [NST][chunk*R] K, then [NST][chunk*D] V
  T* sK = reinterpret_cast<T*>(ring);
  T* sV = reinterpret_cast<T*>(ring + (size_t)NST * kBulkChunk * R * sizeof(T));

  // Slot st of the ring holds chunks st, st+NST, ... and is consumed by warp
  // st % NW only when NST % NW == 0; otherwise a warp could wait on a phase
  // two completions ahead (mbarrier parity waits alias).  The host guarantees
  // the divisibility; a violation is reported and the CTA produces nothing.
  if (NST % NW != 0 || NST > kMaxStages) {
    if (tid == 0) atomicOr(p.ws_status, 16);
    return;
  }
  // this split's token range [t_begin, t_end) of the cache stream
  auto split_range = [&](int seq_len, int& t_begin, int& t_end) {
    const int stream_len = PREP ? seq_len - 1 : seq_len;  // PREP: the newest row comes from registers
    int tps = (stream_len + p.split_k - 1) / p.split_k;
    tps = (tps + kBulkChunk - 1) & ~(kBulkChunk - 1);
    t_begin = s * tps;
    t_end = min(stream_len, t_begin + tps);
  };
  if (tid == 0) {
    for (int i = 0; i < NST; ++i) {
      sm100::mbar_init(&full_bar[i], 1);
      sm100::mbar_init(&empty_bar[i], 1);
    }
    if (CLUSTER) {
      sm100::mbar_init(&comb_bar, 1);   // rank 0's own arrival, plus the peers' partial bytes
      if (s == 0 && p.split_k > 1) sm100::mbar_expect_tx(&comb_bar, (uint32_t)((p.split_k - 1) * (4 * (2 + 2 * D))));
    }
    sm_err = 0;
    sm100::fence_mbar_init();
  }
  // Programmatic dependent launch: this grid may have been scheduled while the
  // previous kernel of the stream was still running.  Before waiting for it,
  // the producer only asks L2 to prefetch this split's cache rows (a hint that
  // reads nothing into the SM: every load below, made after the wait, still
  // sees all of that kernel's writes), so the rows stream in while the
  // previous kernel finishes; with a device-side seq_len the range is not
  // known yet and nothing is prefetched.  Then wait for the previous kernel
  // (its writes become visible) and let the next kernel start scheduling.
  if (warp == NW && lane == 0 && p.seq_len_dev == nullptr && p.R > 0 && !p.no_l2_prefetch) {
    int tb, te;
    split_range(p.seq_len, tb, te);
    if (p.prefetch_window) te = min(te, tb + NST * kBulkChunk);  // only the chunks the ring loads first
    if (te > tb) {
      const char* kg = reinterpret_cast<const char*>(p.cache_k) + (b * p.sck[0] + h * p.sck[1] + (int64_t)tb * R) * sizeof(T);
      const char* vg = reinterpret_cast<const char*>(p.cache_v) + (b * p.scv[0] + h * p.scv[1] + (int64_t)tb * D) * sizeof(T);
      sm100::prefetch_l2(kg, (uint32_t)((te - tb) * R * sizeof(T)));
      sm100::prefetch_l2(vg, (uint32_t)((te - tb) * D * sizeof(T)));
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int seq_len = resolve_seq_len(p, s, tid);
  int t_begin, t_end;
  split_range(seq_len, t_begin, t_end);
  const int nchunks = t_end > t_begin ? (t_end - t_begin + kBulkChunk - 1) / kBulkChunk : 0;
  __syncthreads();  // barriers initialised; the producer starts streaming at once
  // cluster combine: arrive now (releasing rank 0's barrier set-up), wait just
  // before the first remote access
  if (CLUSTER && p.split_k > 1) sm100::cluster_arrive();

  float m_run = -INFINITY, l_run = 0.f;
  float acc[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) acc[c] = 0.f;

  if (warp == NW) {
    // ---------------- producer: stream chunks into the ring ----------------
    if (lane == 0) {
      const char* kg = reinterpret_cast<const char*>(p.cache_k) + (b * p.sck[0] + h * p.sck[1]) * sizeof(T);
      const char* vg = reinterpret_cast<const char*>(p.cache_v) + (b * p.scv[0] + h * p.scv[1]) * sizeof(T);
      for (int c = 0; c < nchunks; ++c) {
        const int st = c % NST;
        if (c >= NST && !sm_err && !sm100::mbar_wait(&empty_bar[st], ((c / NST) - 1) & 1)) atomicOr(&sm_err, 1);
        if (sm_err) break;
        const int t0 = t_begin + c * kBulkChunk;
        const int n = min(kBulkChunk, t_end - t0);
        const uint32_t kbytes = (uint32_t)(n * R * sizeof(T)), vbytes = (uint32_t)(n * D * sizeof(T));
        sm100::mbar_arrive_expect_tx(&full_bar[st], kbytes + vbytes);
        sm100::bulk_g2s(sK + (size_t)st * kBulkChunk * R, kg + (size_t)t0 * R * sizeof(T), kbytes, &full_bar[st]);
        sm100::bulk_g2s(sV + (size_t)st * kBulkChunk * D, vg + (size_t)t0 * D * sizeof(T), vbytes, &full_bar[st]);
      }
    }
  } else if (warp == NW + 1) {
    // ---------------- GLA warp: state rows and y_I, beside the streaming ---
    // the epilogue's norm_w row and blend weight go to shared memory first,
    // so that their global round trip is over long before the epilogue
    for (int d = lane; d < D; d += 32) sm_ep[d] = ld_any(p.norm_w, p.dt_nw, h * p.snw[0] + d * p.snw[1]);
    if (lane == 0 && !p.fused_prep) sm_ep[D] = ld_any(p.mix_g, p.dt_mg, b * p.smg[0] + h * p.smg[1]);
    if constexpr (PREP) {
      asm volatile("bar.sync 2, %0;" ::"n"(NW * 32 + 32) : "memory");  // the log decay is in sm_pre[1]
      gla_rows<T, D, ALPHA, 32>(p, s, b, h, lane, sm_y, &sm_pre[1]);
    } else {
      gla_rows<T, D, ALPHA, 32>(p, s, b, h, lane, sm_y);
    }
  } else {
    // ---------------- consumers: q, then the cache stream ------------------
    if constexpr (PREP) {
      prep_new_token<T, D, NW>(p, s, b, h, tid, lane, warp, seq_len - 1, sm_q, sm_pre);
      asm volatile("bar.sync 2, %0;" ::"n"(NW * 32 + 32) : "memory");  // consumers + GLA warp
    } else {
      load_q<T, D>(p, b, h, tid, sm_q);
      asm volatile("bar.sync 1, %0;" ::"n"(NW * 32) : "memory");  // consumers only
    }
    const int cg_ = lane % G, ts = lane / G;
    volatile int* verr = &sm_err;
    for (int c = warp; c < nchunks; c += NW) {
      const int st = c % NST;
      if (!*verr && !sm100::mbar_wait(&full_bar[st], (c / NST) & 1)) atomicOr(&sm_err, 2);
      const int t0 = t_begin + c * kBulkChunk;
      const int n = min(kBulkChunk, t_end - t0);
      const T* kc = sK + (size_t)st * kBulkChunk * R;
      const T* vc = sV + (size_t)st * kBulkChunk * D;
#pragma unroll
      for (int sub = 0; sub < kBulkChunk / kChunk; ++sub) {
        const int base = sub * kChunk;
        Vec8<T> vr[VI];
#pragma unroll
        for (int i = 0; i < VI; ++i) {
          const int tl = base + i * TS + ts;
          vr[i] = tl < n ? *reinterpret_cast<const Vec8<T>*>(vc + tl * D + cg_ * 8) : zero_vec8<T>();
        }
        float sc = -INFINITY;
        if (base + lane < n) {
          float dot = 0.f;
#pragma unroll
          for (int g = 0; g < G; ++g) {
            if (g * 8 < R) {
              float f[8];
              vec8_to_f(*reinterpret_cast<const Vec8<T>*>(kc + (base + lane) * R + g * 8), f);
#pragma unroll
              for (int cc = 0; cc < 8; ++cc) dot = fmaf(sm_q[g * 8 + cc], f[cc], dot);
            }
          }
          sc = dot;
        }
        if (base < n) tile_update<T, D>(sc, vr, m_run, l_run, acc, ts);  // consumes every value read
      }
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&empty_bar[st]);
    }
    warp_flush<D>(m_run, l_run, acc, lane, warp, sh, sm_acc);
  }
  __syncthreads();
  if (tid == 0 && sm_err) atomicOr(p.ws_status, 4 * sm_err);
  EpiloguePrefetch ep;
  if (tid < D) {
    ep.nw = sm_ep[tid];
    ep.mix = sm_ep[D];
  }
  finish<T, D, CLUSTER, NW, RSUB>(p, s, b, h, tid, lane, warp, NW + 2, sh, sm_acc, sm_y, sm_all, &comb_bar, ep,
                                  PREP ? sm_pre : nullptr);
}

template <typename T, int D, bool ALPHA, bool CLUSTER, int NW, bool PREP>
cudaError_t launch_bulk(const DecodeParams& p, cudaStream_t st) {
  const size_t smem = (size_t)p.stages * kBulkChunk * (p.R + D) * sizeof(T);
  auto k = decode_bulk_kernel<T, D, ALPHA, CLUSTER, NW, PREP>;
  // the function attributes are set once per device (and again only for a
  // larger shared-memory size): a decode step's host time is on the critical
  // path of a serving loop that synchronises every token
  static int smem_set[64] = {};
  static bool cluster_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const int slot = dev >= 0 && dev < 64 ? dev : 0;
  if (smem_set[slot] < (int)smem || dev >= 64) {
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    smem_set[slot] = (int)smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.split_k, p.H, p.B);
  cfg.blockDim = dim3(NW * 32 + 64);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (CLUSTER) {
    if (p.split_k > 8 && (!cluster_set[slot] || dev >= 64)) {
      e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return e;
      cluster_set[slot] = true;
    }
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = p.split_k;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  e = cudaLaunchKernelEx(&cfg, k, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

// HOFA_DECODE_NO_CLUSTER (read once at library load): combine the splits of a
// head through the workspace even when they would fit in one cluster.
const bool kDecodeNoCluster = [] {
  const char* v = getenv("HOFA_DECODE_NO_CLUSTER");
  return v != nullptr && v[0] != '\0' && v[0] != '0';
}();

template <typename T, int D>
cudaError_t launch_d(const DecodeParams& p, int path, bool alpha, cudaStream_t st) {
  dim3 grid(p.split_k, p.H, p.B);
  if (path == 2) {
    const bool cluster = p.split_k > 1 && p.split_k <= kMaxClusterSplit && !kDecodeNoCluster;
    if (p.fused_prep) {  // decode step with the new token's prep (4 consumer warps)
      if (cluster) return alpha ? launch_bulk<T, D, true, true, 4, true>(p, st) : launch_bulk<T, D, false, true, 4, true>(p, st);
      return alpha ? launch_bulk<T, D, true, false, 4, true>(p, st) : launch_bulk<T, D, false, false, 4, true>(p, st);
    }
    if (p.consumer_warps == 6) {
      if (cluster) return alpha ? launch_bulk<T, D, true, true, 6, false>(p, st) : launch_bulk<T, D, false, true, 6, false>(p, st);
      return alpha ? launch_bulk<T, D, true, false, 6, false>(p, st) : launch_bulk<T, D, false, false, 6, false>(p, st);
    }
    if (p.consumer_warps == 8) {
      if (cluster) return alpha ? launch_bulk<T, D, true, true, 8, false>(p, st) : launch_bulk<T, D, false, true, 8, false>(p, st);
      return alpha ? launch_bulk<T, D, true, false, 8, false>(p, st) : launch_bulk<T, D, false, false, 8, false>(p, st);
    }
    if (cluster) return alpha ? launch_bulk<T, D, true, true, 4, false>(p, st) : launch_bulk<T, D, false, true, 4, false>(p, st);
    return alpha ? launch_bulk<T, D, true, false, 4, false>(p, st) : launch_bulk<T, D, false, false, 4, false>(p, st);
  } else if (path == 1) {
    if (alpha) decode_reg_kernel<T, D, true, true><<<grid, kConsumers, 0, st>>>(p);
    else decode_reg_kernel<T, D, true, false><<<grid, kConsumers, 0, st>>>(p);
  } else {
    if (alpha) decode_reg_kernel<T, D, false, true><<<grid, kConsumers, 0, st>>>(p);
    else decode_reg_kernel<T, D, false, false><<<grid, kConsumers, 0, st>>>(p);
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_t(const DecodeParams& p, int path, bool alpha, cudaStream_t st) {
  switch (p.D) {
    case 32: return launch_d<T, 32>(p, path, alpha, st);
    case 64: return launch_d<T, 64>(p, path, alpha, st);
    case 128: return launch_d<T, 128>(p, path, alpha, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

// path: 0 = strided register loads, 1 = 16-byte register loads, 2 = TMA bulk ring
cudaError_t launch_decode(const DecodeParams& p, int dtype, int path, bool alpha, cudaStream_t st) {
  switch (dtype) {
    case HOFA_DTYPE_BF16: return launch_t<__nv_bfloat16>(p, path, alpha, st);
    case HOFA_DTYPE_F16: return launch_t<__half>(p, path, alpha, st);
    default: return launch_t<float>(p, path, alpha, st);
  }
}

}  // namespace hofa
