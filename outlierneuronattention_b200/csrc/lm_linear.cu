// Small-batch linear layer of the decoder LM harness (decode steps, M <= 8 rows).
//
// y[m, n] = (residual[m, n] +) sum_k xin[m, k] * W[n, k], with W in the
// nn.Linear layout [N, K], and xin one of
//   mode 0: x[m, k]
//   mode 1: RMSNorm: x[m, k] * rsqrt(mean_k x[m, k]^2 + eps) * norm_w[k]  (float32, one rounding)
//   mode 2: SwiGLU:  silu(x[m, k]) * x[m, K + k]      (x holds [gate | up]; silu rounded first)
// rounded to the activation dtype, where the unfused modules round.
//
// At decode batch sizes a projection is a matrix-vector product: every weight
// is read once and used M times, so the kernel streams W at HBM speed with
// 16-byte loads and does the few FMAs per element on the CUDA cores.  Two CTAs
// of 8 warps per SM (grid-stride over row groups); a warp covers at most 1024
// columns of its rows, so larger K is split over 2 or 4 warps of a CTA (one
// warp per 4096-wide row took twice as long for the same bytes).  The kernel is launched
// with programmatic dependent launch: each warp issues its first row group's
// weight loads BEFORE waiting for the previous kernel of the stream (the
// weights are parameters: no kernel of a decode loop writes them, so they may
// be read while the kernel that produces x is still running), then waits,
// releases the next kernel, and stages the transformed input rows in shared
// memory (the norm's reduction and the SwiGLU product happen here, once per
// CTA).  So the weight fetch of every projection overlaps the end of the
// kernel before it.  Contract: the weight, norm_w and any memory other than
// x and residual must not be written by the kernel immediately preceding
// this launch on the stream.  All of a row group's loads are in flight before
// its first FMA; the warp reduction leaves one sum per (row, m) in lane m.
#include <cstdio>

#include "common.cuh"

namespace hofa {

struct LinearParams {
  const void* x; const void* w; const void* norm_w; const void* res; void* y;
  int M, N, K;
  int64_t sx, sw, sres, sy;       // row strides (elements)
  int64_t snw;                    // norm_w stride
  int dt_nw;
  float eps;
};

namespace {

constexpr int kLinWarps = 8;
constexpr int kLinThreads = kLinWarps * 32;
constexpr int kMaxM = 8;

__device__ __forceinline__ float silu(float v) { return v / (1.f + __expf(-v)); }

template <typename T>
__device__ __forceinline__ uint4 pack8(const float f[8]) {
  uint4 u;
  if constexpr (sizeof(T) == 2) {
    uint32_t* pu = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      T a = from_f<T>(f[2 * i]), b = from_f<T>(f[2 * i + 1]);
      pu[i] = (uint32_t)*reinterpret_cast<uint16_t*>(&a) | ((uint32_t)*reinterpret_cast<uint16_t*>(&b) << 16);
    }
  }
  return u;
}

// KCH: 16-byte weight chunks per lane per row segment (256 columns each);
// RG: rows per group; SEG: warps that share a group, each taking one
// contiguous K segment of KCH * 256 columns (their partial sums meet in
// shared memory).  A CTA works on 8 / SEG groups at a time, in lockstep.  All
// of a warp's RG * KCH loads are in flight together.  MAXM: the largest batch
// (rows of x) the instance serves (its accumulators are sized for it).
template <typename T, int MODE, bool RES, int KCH, int RG, int SEG, int MAXM>
__global__ void __launch_bounds__(kLinThreads, 2) lm_linear_kernel(const LinearParams p) {
  static_assert(sizeof(T) == 2, "2-byte activations");
  static_assert(kLinWarps % SEG == 0, "segments of a group share one CTA");
  constexpr int GPC = kLinWarps / SEG;   // groups per CTA step
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* sxin = reinterpret_cast<T*>(smem_raw);          // [M][K]
  __shared__ float s_part[kLinWarps][kMaxM];
  __shared__ float s_scale[kMaxM];
  __shared__ float s_red[SEG > 1 ? kLinWarps : 1][RG][MAXM];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int seg = warp % SEG, slot = warp / SEG;
  const int M = p.M, K = p.K;
  const int kbase = seg * KCH * 256;
  const T* W = reinterpret_cast<const T*>(p.w);
  const int groups = (p.N + RG - 1) / RG;
  const int step = gridDim.x * GPC;

  // first step's weights: issued before the input is staged
  uint4 wv[RG][KCH];
  auto issue = [&](int grp) {
#pragma unroll
    for (int r = 0; r < RG; ++r) {
      const int n = grp * RG + r;
#pragma unroll
      for (int c = 0; c < KCH; ++c) {
        const int k0 = kbase + (c * 32 + lane) * 8;
        wv[r][c] = (grp < groups && n < p.N && k0 < K) ? ld_stream16(W + (int64_t)n * p.sw + k0)
                                                       : make_uint4(0, 0, 0, 0);
      }
    }
  };
  int g0 = blockIdx.x * GPC;
  issue(g0 + slot);
  // RMSNorm weights of this thread's staging chunks (columns 8 kc .. 8 kc + 8
  // for kc = tid, tid + 256; K <= 4096): parameters as well, read before the wait
  float nwr[MODE == 1 ? 2 : 1][8];
  if constexpr (MODE == 1) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int kc = tid + j * kLinThreads;
#pragma unroll
      for (int e = 0; e < 8; ++e)
        nwr[j][e] = kc < K / 8 ? ld_any(p.norm_w, p.dt_nw, (int64_t)(kc * 8 + e) * p.snw) : 0.f;
    }
  }
  // x / residual come from the kernels before: wait for them, then let the
  // next kernel of the stream start its own weight fetch
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // stage the transformed input rows
  const T* X = reinterpret_cast<const T*>(p.x);
  const int K8 = K / 8;
  if constexpr (MODE == 1) {
    float ss[MAXM];
#pragma unroll
    for (int m = 0; m < MAXM; ++m) ss[m] = 0.f;
    for (int i = tid; i < K8; i += kLinThreads) {
#pragma unroll
      for (int m = 0; m < MAXM; ++m) {
        if (m < M) {
          float f[8];
          Vec8<T> v;
          v.w[0] = *reinterpret_cast<const uint4*>(X + (int64_t)m * p.sx + i * 8);
          vec8_to_f(v, f);
#pragma unroll
          for (int e = 0; e < 8; ++e) ss[m] = fmaf(f[e], f[e], ss[m]);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < MAXM; ++m) {
      const float t = warp_sum(ss[m]);
      if (lane == 0) s_part[warp][m] = t;
    }
    __syncthreads();
    if (tid < M) {
      float t = 0.f;
      for (int w = 0; w < kLinWarps; ++w) t += s_part[w][tid];
      s_scale[tid] = rsqrtf(t / (float)K + p.eps);
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int kc = tid + j * kLinThreads;
      if (kc < K8) {
#pragma unroll
        for (int m = 0; m < MAXM; ++m) {
          if (m < M) {
            float f[8];
            Vec8<T> v;
            v.w[0] = *reinterpret_cast<const uint4*>(X + (int64_t)m * p.sx + kc * 8);
            vec8_to_f(v, f);
            const float sc = s_scale[m];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = f[e] * sc * nwr[j][e];
            *reinterpret_cast<uint4*>(sxin + (int64_t)m * K + kc * 8) = pack8<T>(f);
          }
        }
      }
    }
  }
  for (int i = tid; MODE != 1 && i < M * K8; i += kLinThreads) {
    const int m = i / K8, k0 = (i - m * K8) * 8;
    float f[8];
    Vec8<T> v;
    v.w[0] = *reinterpret_cast<const uint4*>(X + (int64_t)m * p.sx + k0);
    vec8_to_f(v, f);
    if constexpr (MODE == 2) {
      float u[8];
      Vec8<T> vu;
      vu.w[0] = *reinterpret_cast<const uint4*>(X + (int64_t)m * p.sx + K + k0);
      vec8_to_f(vu, u);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = to_f(from_f<T>(silu(f[e]))) * u[e];
    }
    *reinterpret_cast<uint4*>(sxin + (int64_t)m * K + k0) = pack8<T>(f);
  }
  __syncthreads();

  // every warp of a CTA takes the same number of steps (the shared-memory
  // combine of the segments needs the whole CTA)
  for (; g0 < groups; g0 += step) {
    const int g = g0 + slot;
    float acc[RG][MAXM];
#pragma unroll
    for (int r = 0; r < RG; ++r)
#pragma unroll
      for (int m = 0; m < MAXM; ++m) acc[r][m] = 0.f;
#pragma unroll
    for (int c = 0; c < KCH; ++c) {
      const int k0 = kbase + (c * 32 + lane) * 8;
      if (k0 < K) {
        float wf[RG][8];
#pragma unroll
        for (int r = 0; r < RG; ++r) {
          Vec8<T> wq;
          wq.w[0] = wv[r][c];
          vec8_to_f(wq, wf[r]);
        }
#pragma unroll
        for (int m = 0; m < MAXM; ++m) {
          if (m < M) {
            float xf[8];
            Vec8<T> xv;
            xv.w[0] = *reinterpret_cast<const uint4*>(sxin + (int64_t)m * K + k0);
            vec8_to_f(xv, xf);
#pragma unroll
            for (int r = 0; r < RG; ++r)
#pragma unroll
              for (int e = 0; e < 8; ++e) acc[r][m] = fmaf(wf[r][e], xf[e], acc[r][m]);
          }
        }
      }
    }
    if (g0 + step < groups) issue(g0 + step + slot);   // next step's loads before the reductions
#pragma unroll
    for (int r = 0; r < RG; ++r)
#pragma unroll
      for (int m = 0; m < MAXM; ++m)
        if (m < M) acc[r][m] = warp_sum(acc[r][m]);
    if constexpr (SEG > 1) {
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < RG; ++r)
#pragma unroll
          for (int m = 0; m < MAXM; ++m) s_red[warp][r][m] = acc[r][m];
      }
      __syncthreads();
    }
    if (seg == 0) {
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        const int n = g * RG + r;
#pragma unroll
        for (int m = 0; m < MAXM; ++m) {
          if (m < M && lane == m && g < groups && n < p.N) {
            float out = acc[r][m];
            if constexpr (SEG > 1) {
#pragma unroll
              for (int sg = 1; sg < SEG; ++sg) out += s_red[warp + sg][r][m];
            }
            if constexpr (RES) out += to_f(reinterpret_cast<const T*>(p.res)[(int64_t)m * p.sres + n]);
            reinterpret_cast<T*>(p.y)[(int64_t)m * p.sy + n] = from_f<T>(out);
          }
        }
      }
    }
    if constexpr (SEG > 1) __syncthreads();   // s_red is rewritten next step
  }
}

template <typename T, int MODE, bool RES>
cudaError_t launch_k(const LinearParams& p, cudaStream_t st) {
  const size_t smem = (size_t)p.M * p.K * sizeof(T);
  int sms = 148;
  {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  auto go = [&](auto kern, int rg, int seg) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int groups = (p.N + rg - 1) / rg;
    const int gpc = kLinWarps / seg;
    int grid = (groups + gpc - 1) / gpc;
    if (grid > 2 * sms) grid = 2 * sms;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kLinThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
  };
  // each warp takes up to 1024 columns of its rows (K above that is split
  // over 2 or 4 warps); for one row of x (accumulators for one row), 4 rows a
  // warp when 2 would leave weights for a second round of loads behind the first
  const int slots = 2 * sms * kLinWarps;
  if (p.M == 1) {  // accumulators for one row of x
    if (p.K <= 1024) {
      if ((p.N + 1) / 2 > slots) return go(lm_linear_kernel<T, MODE, RES, 4, 4, 1, 1>, 4, 1);
      return go(lm_linear_kernel<T, MODE, RES, 4, 2, 1, 1>, 2, 1);
    }
    if (p.K <= 2048) return go(lm_linear_kernel<T, MODE, RES, 4, 2, 2, 1>, 2, 2);
    return go(lm_linear_kernel<T, MODE, RES, 4, 2, 4, 1>, 2, 4);
  }
  if (p.K <= 1024) return go(lm_linear_kernel<T, MODE, RES, 4, 2, 1, kMaxM>, 2, 1);
  if (p.K <= 2048) return go(lm_linear_kernel<T, MODE, RES, 4, 2, 2, kMaxM>, 2, 2);
  return go(lm_linear_kernel<T, MODE, RES, 4, 2, 4, kMaxM>, 2, 4);
}

template <typename T>
cudaError_t launch_t(const LinearParams& p, int mode, bool res, cudaStream_t st) {
  if (mode == 1) return res ? launch_k<T, 1, true>(p, st) : launch_k<T, 1, false>(p, st);
  if (mode == 2) return res ? launch_k<T, 2, true>(p, st) : launch_k<T, 2, false>(p, st);
  return res ? launch_k<T, 0, true>(p, st) : launch_k<T, 0, false>(p, st);
}

}  // namespace

int set_last_error(int code, const char* message);  // capi.cu

}  // namespace hofa

extern "C" int hofa_lm_linear_fwd(const hofa_linear_args* a, void* stream) {
  using hofa::set_last_error;
  char msg[256];
  if (a == nullptr) return set_last_error(HOFA_ERR_INVALID_ARGUMENT, "args is NULL");
  auto bad = [&](const char* what) {
    snprintf(msg, sizeof(msg), "hofa_lm_linear_fwd: %s", what);
    return set_last_error(HOFA_ERR_INVALID_ARGUMENT, msg);
  };
  const hofa_tensor &x = a->x, &w = a->weight, &y = a->y;
  if (x.data == nullptr || w.data == nullptr || y.data == nullptr) return bad("x, weight and y are required");
  if (x.ndim != 2 || w.ndim != 2 || y.ndim != 2) return bad("x [M, K], weight [N, K] and y [M, N] are 2-D");
  const int64_t M = x.shape[0], N = w.shape[0], K = w.shape[1];
  const int mode = a->input_mode;
  if (mode < 0 || mode > 2) return bad("input_mode must be 0 (plain), 1 (RMSNorm) or 2 (SwiGLU)");
  if (M < 1 || M > 8) return bad("1 <= M <= 8 rows (larger batches are GEMMs)");
  if (x.shape[1] != (mode == 2 ? 2 * K : K)) return bad("x has K columns (2K with the SwiGLU input)");
  if (y.shape[0] != M || y.shape[1] != N) return bad("y must be [M, N]");
  if (x.dtype != w.dtype || y.dtype != w.dtype || (w.dtype != HOFA_DTYPE_BF16 && w.dtype != HOFA_DTYPE_F16))
    return set_last_error(HOFA_ERR_UNSUPPORTED, "hofa_lm_linear_fwd: bf16 or f16 x, weight and y of one dtype");
  if (K % 8 || K > 4096 || x.stride[1] != 1 || w.stride[1] != 1 || y.stride[1] != 1) return bad("K % 8 == 0, K <= 4096, unit inner strides");
  auto al16 = [](const void* p, int64_t stride) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && (stride * 2) % 16 == 0;
  };
  if (!al16(x.data, x.stride[0]) || !al16(w.data, w.stride[0]))
    return set_last_error(HOFA_ERR_MISALIGNED, "hofa_lm_linear_fwd: x and weight rows must be 16-byte aligned");
  hofa::LinearParams p{};
  p.x = x.data; p.w = w.data; p.y = y.data;
  p.M = (int)M; p.N = (int)N; p.K = (int)K;
  p.sx = x.stride[0]; p.sw = w.stride[0]; p.sy = y.stride[0];
  p.eps = a->eps;
  const bool res = a->residual.data != nullptr;
  if (res) {
    const hofa_tensor& r = a->residual;
    if (r.ndim != 2 || r.shape[0] != M || r.shape[1] != N || r.dtype != w.dtype || r.stride[1] != 1)
      return bad("residual must be [M, N] with the dtype of y");
    p.res = r.data; p.sres = r.stride[0];
  }
  if (mode == 1) {
    const hofa_tensor& g = a->norm_w;
    if (g.data == nullptr || g.ndim != 1 || g.shape[0] != K) return bad("RMSNorm input needs norm_w [K]");
    p.norm_w = g.data; p.snw = g.stride[0]; p.dt_nw = g.dtype;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const cudaError_t e = w.dtype == HOFA_DTYPE_BF16 ? hofa::launch_t<__nv_bfloat16>(p, mode, res, st)
                                                   : hofa::launch_t<__half>(p, mode, res, st);
  if (e != cudaSuccess) {
    snprintf(msg, sizeof(msg), "hofa_lm_linear_fwd launch: %s", cudaGetErrorString(e));
    return set_last_error(HOFA_ERR_CUDA, msg);
  }
  return HOFA_OK;
}
