// Prefill, outlier path: causal softmax attention over R channels with
// full-width values, scaled by the blend gate and added into the output.
//
// Replaces exact_attention_triton / _fwd_kernel (src/exact_attention.py:
// 163-188, :45-161).  This file holds the generic CUDA-core kernel (any
// activation dtype, any R <= D, D in {32, 64, 128}, any strides); it is the
// path for fp32 inputs (fp32 parity) and for shapes the tensor-core kernel
// does not take.  Math: s = (q . k) * sm_scale * log2(e), online softmax in
// base 2, out = (accumulate ? out : 0) + mix * (sum p v) / (sum p).
#include "common.cuh"
#include "kernels.h"

namespace hofa {

namespace {

constexpr int kOutThreads = 256;
constexpr int BM = 64, BN = 64;

template <typename T, int D>
__global__ void __launch_bounds__(kOutThreads)
outlier_generic_kernel(const OutlierParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int R = p.R;
  const int RP = R + 1;
  float* Qs = reinterpret_cast<float*>(smem_raw);   // [BM][RP]
  float* Ks = Qs + BM * RP;                          // [BN][RP]
  float* Vs = Ks + BN * RP;                          // [BN][D]
  float* Ps = Vs + BN * D;                           // [BM][BN+1]

  const int nqb = (p.Tq + BM - 1) / BM;
  const int qb = nqb - 1 - (int)blockIdx.x;          // long rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
  const int i = tid / 4, sub = tid % 4;              // row of this thread, lane in the row quad
  const int q0 = qb * BM;

  const T* qg = reinterpret_cast<const T*>(p.q) + b * p.sq[0] + h * p.sq[1];
  const T* kg = reinterpret_cast<const T*>(p.k) + b * p.sk[0] + h * p.sk[1];
  const T* vg = reinterpret_cast<const T*>(p.v) + b * p.sv[0] + h * p.sv[1];

  for (int e = tid; e < BM * R; e += kOutThreads) {
    const int r = e / R, c = e % R;
    const int t = q0 + r;
    Qs[r * RP + c] = (t < p.Tq) ? to_f(qg[(int64_t)t * p.sq[2] + (int64_t)c * p.sq[3]]) * p.qk_scale_log2 : 0.f;
  }

  constexpr int DC = D / 4;
  float acc[DC];
#pragma unroll
  for (int u = 0; u < DC; ++u) acc[u] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  const int qpos = q0 + i + p.q_offset;              // absolute position of this row
  const int last_key = min(p.Tk - 1, q0 + BM - 1 + p.q_offset);

  for (int k0 = 0; k0 <= last_key; k0 += BN) {
    __syncthreads();
    for (int e = tid; e < BN * R; e += kOutThreads) {
      const int r = e / R, c = e % R;
      const int t = k0 + r;
      Ks[r * RP + c] = (t < p.Tk) ? to_f(kg[(int64_t)t * p.sk[2] + (int64_t)c * p.sk[3]]) : 0.f;
    }
    for (int e = tid; e < BN * D; e += kOutThreads) {
      const int r = e / D, d = e % D;
      const int t = k0 + r;
      Vs[e] = (t < p.Tk) ? to_f(vg[(int64_t)t * p.sv[2] + (int64_t)d * p.sv[3]]) : 0.f;
    }
    __syncthreads();
    float sc[BN / 4];
    float mt = -INFINITY;
#pragma unroll
    for (int u = 0; u < BN / 4; ++u) {
      const int j = sub + 4 * u;
      const int kpos = k0 + j;
      float s = -INFINITY;
      if (kpos <= qpos && kpos < p.Tk) {
        s = 0.f;
        for (int c = 0; c < R; ++c) s = fmaf(Qs[i * RP + c], Ks[j * RP + c], s);
      }
      sc[u] = s;
      mt = fmaxf(mt, s);
    }
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
    const float mn = fmaxf(m_run, mt);
    const float corr = (mn == -INFINITY) ? 1.f : exp2f(m_run - mn);
    float ls = 0.f;
#pragma unroll
    for (int u = 0; u < BN / 4; ++u) {
      const float pv = (mn == -INFINITY) ? 0.f : exp2f(sc[u] - mn);
      ls += pv;
      Ps[i * (BN + 1) + sub + 4 * u] = pv;
    }
    ls += __shfl_xor_sync(0xffffffffu, ls, 1);
    ls += __shfl_xor_sync(0xffffffffu, ls, 2);
    l_run = l_run * corr + ls;
    m_run = mn;
    __syncwarp();
#pragma unroll
    for (int u = 0; u < DC; ++u) acc[u] *= corr;
    for (int j = 0; j < BN; ++j) {
      const float pj = Ps[i * (BN + 1) + j];
#pragma unroll
      for (int u = 0; u < DC; ++u) acc[u] = fmaf(pj, Vs[j * D + sub + 4 * u], acc[u]);
    }
  }

  const int t = q0 + i;
  if (t < p.Tq) {
    const float mix = ld_any(p.mix_g, p.dt_mg, b * p.smg[0] + h * p.smg[1] + (int64_t)t * p.smg[2]);
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    T* og = reinterpret_cast<T*>(p.out) + b * p.so[0] + h * p.so[1] + (int64_t)t * p.so[2];
#pragma unroll
    for (int u = 0; u < DC; ++u) {
      const int64_t off = (int64_t)(sub + 4 * u) * p.so[3];
      float o = mix * acc[u] * inv;
      if (p.accumulate) o += to_f(og[off]);
      og[off] = from_f<T>(o);
    }
  }
}

template <typename T, int D>
cudaError_t launch_d(const OutlierParams& p, cudaStream_t st) {
  const size_t smem = sizeof(float) * ((size_t)BM * (p.R + 1) + (size_t)BN * (p.R + 1) + (size_t)BN * D + (size_t)BM * (BN + 1));
  auto k = outlier_generic_kernel<T, D>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((p.Tq + BM - 1) / BM, p.H, p.B);
  k<<<grid, kOutThreads, smem, st>>>(p);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_t(const OutlierParams& p, cudaStream_t st) {
  switch (p.D) {
    case 32: return launch_d<T, 32>(p, st);
    case 64: return launch_d<T, 64>(p, st);
    case 128: return launch_d<T, 128>(p, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_outlier_generic(const OutlierParams& p, int dtype, cudaStream_t st) {
  switch (dtype) {
    case HOFA_DTYPE_BF16: return launch_t<__nv_bfloat16>(p, st);
    case HOFA_DTYPE_F16: return launch_t<__half>(p, st);
    default: return launch_t<float>(p, st);
  }
}

}  // namespace hofa
