// Prefill, inlier path: chunked gated linear attention (GLA).
//
// Replaces chunk_gla_inlier_fwd / chunk_gla_fwd_kernel
// (src/chunk_gla_inlier.py:153-237, :5-150).  The reference runs one program
// per (b,h) walking every chunk in sequence (B*H programs: 64 at B=4,H=16,
// 16 at B=1).  Here each (b,h) sequence is cut into `nseg` segments of whole
// chunks that run in parallel:
//
//   pass A (segments 0..nseg-2): the segment's end state from a zero start,
//          S_loc = sum_t exp(G_end - G_t) k_t v_t^T, and its total log decay;
//   pass C (all segments): the start state is rebuilt from the earlier
//          segments' (S_loc, decay) -- S <- exp(decay_s) S + S_loc_s -- and
//          the segment is swept chunk by chunk:
//            A   = (Q K^T) * exp(G_i - G_j) [i >= j]
//            Y   = A V + (Q * exp(G_i)) S
//            S  <- exp(G_C) S + (K * exp(G_C - G_j))^T V
//          followed by the fused epilogue (1 - mix) * gla_scale * RMSNorm(Y).
//
// All arithmetic is fp32 (inputs of any activation dtype are widened on
// load); the decay factors are formed as differences of cumulative log decays
// that are <= 0, so no factor exceeds 1 (no overflow for strong decay, unlike
// the factored form at chunk_gla_inlier.py:90-107).
#include "common.cuh"
#include "kernels.h"

namespace hofa {

namespace {

constexpr int kGlaThreads = 256;

template <int D, int C, bool ALPHA>
struct GlaSmem {
  static constexpr int J_MAX = D;  // J = D - R <= D
  float S[J_MAX * D];
  float Q[C * (J_MAX + 1)];   // row stride J + 1 (odd: conflict-free column walks)
  float K[C * (J_MAX + 1)];
  float V[C * D];
  float A[C * C];
  float G[ALPHA ? C * J_MAX : C];
  float GC[J_MAX];
};

template <typename T, int D, int C, bool ALPHA, bool STATE_ONLY>
__global__ void __launch_bounds__(kGlaThreads)
gla_kernel(const GlaParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  auto& sm = *reinterpret_cast<GlaSmem<D, C, ALPHA>*>(smem_raw);
  const int seg = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
  const int J = p.J, R = p.R;
  const int JP = J + 1;
  const int bh = b * p.H + h;
  const int t_seg0 = seg * p.seg_len;
  const int t_seg1 = min(p.T, t_seg0 + p.seg_len);

  // ---- start state -------------------------------------------------------
  for (int e = tid; e < J * D; e += kGlaThreads) {
    const int c = e / D, d = e % D;
    float s = 0.f;
    if (!STATE_ONLY) {
      if (p.state_init != nullptr) s = p.state_init[b * p.ssi[0] + h * p.ssi[1] + c * p.ssi[2] + d];
      for (int q = 0; q < seg; ++q) {
        const float dec = p.ws_decay[((int64_t)bh * p.nseg + q) * J + c];
        const float loc = p.ws_state[(((int64_t)bh * p.nseg + q) * J + c) * D + d];
        s = fmaf(expf(dec), s, loc);
      }
    }
    sm.S[c * D + d] = s;
  }

  float total_decay = 0.f;  // sum of log decay over the segment (per channel tid when ALPHA)

  const T* qb = reinterpret_cast<const T*>(p.q) + b * p.sq[0] + h * p.sq[1];
  const T* kb = reinterpret_cast<const T*>(p.k) + b * p.sk[0] + h * p.sk[1];
  const T* vb = reinterpret_cast<const T*>(p.v) + b * p.sv[0] + h * p.sv[1];

  // register tile of the output: 4 rows x (D/16) cols per thread
  constexpr int YC = D / 16;          // columns per thread (4 for D=64)
  const int ti = tid / 16, td = tid % 16;
  constexpr int YR = C / 16;          // rows per thread

  for (int t0 = t_seg0; t0 < t_seg1; t0 += C) {
    __syncthreads();
    // ---- load the chunk (fp32) ---------------------------------------------
    for (int e = tid; e < C * J; e += kGlaThreads) {
      const int i = e / J, c = e % J;
      const int t = t0 + i;
      float qv = 0.f, kv = 0.f;
      if (t < t_seg1) {
        if (!STATE_ONLY) qv = to_f(qb[(int64_t)t * p.sq[2] + (int64_t)(R + c) * p.sq[3]]);
        kv = to_f(kb[(int64_t)t * p.sk[2] + (int64_t)(R + c) * p.sk[3]]);
      }
      sm.Q[i * JP + c] = qv;
      sm.K[i * JP + c] = kv;
    }
    for (int e = tid; e < C * D; e += kGlaThreads) {
      const int i = e / D, d = e % D;
      const int t = t0 + i;
      sm.V[e] = (t < t_seg1) ? to_f(vb[(int64_t)t * p.sv[2] + (int64_t)d * p.sv[3]]) : 0.f;
    }
    // cumulative log decay within the chunk
    if constexpr (ALPHA) {
      for (int c = tid; c < J; c += kGlaThreads) {
        const float a = expf(ld_any(p.log_alpha, p.dt_la, b * p.sla[0] + h * p.sla[1] + c * p.sla[2]));
        float g = 0.f;
        for (int i = 0; i < C; ++i) {
          const int t = t0 + i;
          const float lg = (t < t_seg1) ? ld_any(p.log_gamma, p.dt_lg, b * p.slg[0] + h * p.slg[1] + t * p.slg[2]) : 0.f;
          g += lg * a;
          sm.G[i * J + c] = g;
        }
        sm.GC[c] = g;
      }
    } else {
      if (tid < 32) {
        float carry = 0.f;
        for (int i0 = 0; i0 < C; i0 += 32) {
          const int t = t0 + i0 + tid;
          float x = (t < t_seg1) ? ld_any(p.log_gamma, p.dt_lg, b * p.slg[0] + h * p.slg[1] + t * p.slg[2]) : 0.f;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, x, o);
            if (tid >= o) x += y;
          }
          x += carry;
          sm.G[i0 + tid] = x;
          carry = __shfl_sync(0xffffffffu, x, 31);
        }
        if (tid == 0) sm.GC[0] = carry;
      }
    }
    __syncthreads();

    // ---- intra-chunk scores A = (Q K^T) * decay, causal ------------------
    if (!STATE_ONLY) {
      for (int e = tid; e < C * C; e += kGlaThreads) {
        const int i = e / C, j = e % C;
        float a = 0.f;
        if (j <= i) {
          if constexpr (ALPHA) {
            for (int c = 0; c < J; ++c)
              a = fmaf(sm.Q[i * JP + c] * sm.K[j * JP + c], expf(sm.G[i * J + c] - sm.G[j * J + c]), a);
          } else {
            for (int c = 0; c < J; ++c) a = fmaf(sm.Q[i * JP + c], sm.K[j * JP + c], a);
            a *= expf(sm.G[i] - sm.G[j]);
          }
        }
        sm.A[e] = a;
      }
      __syncthreads();
    }
    // ---- Q <- Q exp(G_i), K <- K exp(G_C - G_j) -------------------------
    for (int e = tid; e < C * J; e += kGlaThreads) {
      const int i = e / J, c = e % J;
      const float gi = ALPHA ? sm.G[i * J + c] : sm.G[i];
      const float gc = ALPHA ? sm.GC[c] : sm.GC[0];
      if (!STATE_ONLY) sm.Q[i * JP + c] *= expf(gi);
      sm.K[i * JP + c] *= expf(gc - gi);
    }
    __syncthreads();

    // ---- Y = A V + Qe S  ----------------------------------------------------
    float yv[YR][YC];
    if (!STATE_ONLY) {
#pragma unroll
      for (int a = 0; a < YR; ++a)
#pragma unroll
        for (int c = 0; c < YC; ++c) yv[a][c] = 0.f;
      for (int j = 0; j < C; ++j) {
        float vv[YC];
#pragma unroll
        for (int c = 0; c < YC; ++c) vv[c] = sm.V[j * D + td + 16 * c];
#pragma unroll
        for (int a = 0; a < YR; ++a) {
          const float aij = sm.A[(ti + 16 * a) * C + j];
#pragma unroll
          for (int c = 0; c < YC; ++c) yv[a][c] = fmaf(aij, vv[c], yv[a][c]);
        }
      }
      for (int c2 = 0; c2 < J; ++c2) {
        float sv[YC];
#pragma unroll
        for (int c = 0; c < YC; ++c) sv[c] = sm.S[c2 * D + td + 16 * c];
#pragma unroll
        for (int a = 0; a < YR; ++a) {
          const float qe = sm.Q[(ti + 16 * a) * JP + c2];
#pragma unroll
          for (int c = 0; c < YC; ++c) yv[a][c] = fmaf(qe, sv[c], yv[a][c]);
        }
      }
    }
    __syncthreads();

    // ---- S <- exp(G_C) S + Kd^T V ----------------------------------------
    for (int e = tid; e < J * D; e += kGlaThreads) {
      const int c = e / D, d = e % D;
      const float gc = ALPHA ? sm.GC[c] : sm.GC[0];
      float s = sm.S[e] * expf(gc);
      for (int j = 0; j < C; ++j) s = fmaf(sm.K[j * JP + c], sm.V[j * D + d], s);
      sm.S[e] = s;
    }
    if constexpr (ALPHA) {
      if (tid < J) total_decay += sm.GC[tid];
    } else {
      total_decay += sm.GC[0];
    }

    // ---- epilogue + store ---------------------------------------------------
    if (!STATE_ONLY) {
#pragma unroll
      for (int a = 0; a < YR; ++a) {
        const int i = ti + 16 * a;
        const int t = t0 + i;
        float o[YC];
#pragma unroll
        for (int c = 0; c < YC; ++c) o[c] = yv[a][c];
        if (p.fuse) {
          float ss = 0.f;
#pragma unroll
          for (int c = 0; c < YC; ++c) ss = fmaf(o[c], o[c], ss);
          // the 16 threads of a row are consecutive lanes of one warp
#pragma unroll
          for (int off = 8; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
          const float rs = rsqrtf(ss / (float)D + p.eps);
          const float mix = (t < t_seg1) ? ld_any(p.mix_g, p.dt_mg, b * p.smg[0] + h * p.smg[1] + t * p.smg[2]) : 0.f;
#pragma unroll
          for (int c = 0; c < YC; ++c) {
            const int d = td + 16 * c;
            const float gsv = ld_any(p.gla_scale, p.dt_gs, h * p.sgs[0] + d * p.sgs[1]);
            o[c] = o[c] * rs * gsv * (1.f - mix);
          }
        }
        if (t < t_seg1) {
          T* yp = reinterpret_cast<T*>(p.y) + b * p.sy[0] + h * p.sy[1] + (int64_t)t * p.sy[2];
#pragma unroll
          for (int c = 0; c < YC; ++c) yp[(int64_t)(td + 16 * c) * p.sy[3]] = from_f<T>(o[c]);
        }
      }
    }
  }
  __syncthreads();

  // ---- segment results ------------------------------------------------------
  if (STATE_ONLY) {
    float* ws = p.ws_state + ((int64_t)bh * p.nseg + seg) * J * D;
    for (int e = tid; e < J * D; e += kGlaThreads) ws[e] = sm.S[e];
    if constexpr (ALPHA) {
      if (tid < J) p.ws_decay[((int64_t)bh * p.nseg + seg) * J + tid] = total_decay;
    } else {
      for (int c = tid; c < J; c += kGlaThreads) p.ws_decay[((int64_t)bh * p.nseg + seg) * J + c] = total_decay;
    }
  } else if (p.state_out != nullptr && t_seg1 >= p.T) {
    for (int e = tid; e < J * D; e += kGlaThreads) {
      const int c = e / D, d = e % D;
      p.state_out[b * p.sso[0] + h * p.sso[1] + c * p.sso[2] + d * p.sso[3]] = sm.S[e];
    }
  }
}

template <typename T, int D, int C, bool ALPHA>
cudaError_t launch_dc(const GlaParams& p, cudaStream_t st) {
  const size_t smem = sizeof(GlaSmem<D, C, ALPHA>);
  auto kA = gla_kernel<T, D, C, ALPHA, true>;
  auto kC = gla_kernel<T, D, C, ALPHA, false>;
  cudaError_t e = cudaFuncSetAttribute(kA, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kC, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  if (p.nseg > 1) {
    kA<<<dim3(p.nseg - 1, p.H, p.B), kGlaThreads, smem, st>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  kC<<<dim3(p.nseg, p.H, p.B), kGlaThreads, smem, st>>>(p);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_t(const GlaParams& p, cudaStream_t st) {
  const bool alpha = p.log_alpha != nullptr;
  switch (p.D) {
    case 32: return alpha ? launch_dc<T, 32, 64, true>(p, st) : launch_dc<T, 32, 64, false>(p, st);
    case 64: return alpha ? launch_dc<T, 64, 64, true>(p, st) : launch_dc<T, 64, 64, false>(p, st);
    case 128: return alpha ? launch_dc<T, 128, 32, true>(p, st) : launch_dc<T, 128, 32, false>(p, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

int gla_internal_chunk(int D) { return D == 128 ? 32 : 64; }

cudaError_t launch_gla(const GlaParams& p, int dtype, cudaStream_t st) {
  switch (dtype) {
    case HOFA_DTYPE_BF16: return launch_t<__nv_bfloat16>(p, st);
    case HOFA_DTYPE_F16: return launch_t<__half>(p, st);
    default: return launch_t<float>(p, st);
  }
}

}  // namespace hofa
