// extern "C" entry points of libhofa_b200.so (declared in include/hofa.h).
//
// Every entry point validates its arguments on the host (shapes, strides,
// dtypes, alignment, workspace size) and returns a hofa_status; nothing here
// traps, synchronises or allocates.  Kernels are launched on the caller's
// stream.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "../../include/hofa.h"
#include "kernels.h"

namespace hofa {
int gla_internal_chunk(int D);
size_t gla_tc_workspace_bytes(int64_t B, int64_t H, int64_t T, int64_t J, int64_t D);
void gla_tc_bind_workspace(GlaParams& p, void* ws);
bool gla_tc_eligible(const GlaParams& p, int dtype);
cudaError_t launch_gla_tc(const GlaParams& p, int dtype, cudaStream_t st, bool* taken);
int gla_tc_chunk();
cudaError_t read_gla_tc_status(int* out, cudaStream_t st);
cudaError_t read_outlier_tc_status(int* out, cudaStream_t st);
cudaError_t launch_outlier_generic(const OutlierParams& p, int dtype, cudaStream_t st);
cudaError_t launch_outlier_tc(const OutlierParams& p, int dtype, cudaStream_t st, bool* taken);
}  // namespace hofa

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(HOFA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool present(const hofa_tensor& t) { return t.data != nullptr; }
bool dtype_ok(int dt) { return dt == HOFA_DTYPE_F32 || dt == HOFA_DTYPE_BF16 || dt == HOFA_DTYPE_F16; }
int esize(int dt) { return dt == HOFA_DTYPE_F32 ? 4 : 2; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Checks presence, dtype validity, ndim and every shape entry that is >= 0.
int check(const hofa_tensor& t, const char* name, int ndim, const int64_t* shape) {
  if (!present(t)) return fail(HOFA_ERR_INVALID_ARGUMENT, "%s: missing (NULL data)", name);
  if (!dtype_ok(t.dtype)) return fail(HOFA_ERR_INVALID_ARGUMENT, "%s: unknown dtype code %d", name, t.dtype);
  if (t.ndim != ndim) return fail(HOFA_ERR_INVALID_ARGUMENT, "%s: expected %d dims, got %d", name, ndim, t.ndim);
  for (int i = 0; i < ndim; ++i) {
    if (t.shape[i] < 0) return fail(HOFA_ERR_INVALID_ARGUMENT, "%s: negative size in dim %d", name, i);
    if (shape[i] >= 0 && t.shape[i] != shape[i])
      return fail(HOFA_ERR_INVALID_ARGUMENT, "%s: dim %d is %lld, expected %lld", name, i,
                  (long long)t.shape[i], (long long)shape[i]);
  }
  return HOFA_OK;
}
#define CHECK(t, name, nd, ...)                              \
  do {                                                       \
    const int64_t _s[4] = {__VA_ARGS__};                     \
    int _r = check(t, name, nd, _s);                         \
    if (_r) return _r;                                       \
  } while (0)

// Per-(b,h) side tensors given as [B,H] or [B,H,1] (decode) / [B,H,T] or
// [B,H,T,1] (prefill); returns the strides of (b, h, t).
int side_bht(const hofa_tensor& t, const char* name, int64_t B, int64_t H, int64_t T, int64_t out[3]) {
  if (!present(t)) return fail(HOFA_ERR_INVALID_ARGUMENT, "%s: missing", name);
  if (!dtype_ok(t.dtype)) return fail(HOFA_ERR_INVALID_ARGUMENT, "%s: unknown dtype", name);
  int64_t tb = t.shape[0], th = t.ndim > 1 ? t.shape[1] : 1;
  int64_t tt = t.ndim > 2 ? t.shape[2] : 1;
  bool ok = (t.ndim >= 2 && t.ndim <= 4) && (tb == B || tb == 1) && th == H && tt == T &&
            (t.ndim < 4 || t.shape[3] == 1);
  if (!ok) return fail(HOFA_ERR_INVALID_ARGUMENT, "%s: expected shape [B=%lld,H=%lld,%lld(,1)]", name,
                       (long long)B, (long long)H, (long long)T);
  out[0] = tb == 1 ? 0 : t.stride[0];
  out[1] = t.stride[1];
  out[2] = t.ndim > 2 ? t.stride[2] : 0;
  return HOFA_OK;
}

// [H, X] per-head vectors (gla_scale / norm_w) given as [H,X] or [1,H,1,X].
int head_vec(const hofa_tensor& t, const char* name, int64_t H, int64_t X, int64_t out[2]) {
  if (!present(t)) return fail(HOFA_ERR_INVALID_ARGUMENT, "%s: missing", name);
  if (!dtype_ok(t.dtype)) return fail(HOFA_ERR_INVALID_ARGUMENT, "%s: unknown dtype", name);
  if (t.ndim == 2 && t.shape[0] == H && t.shape[1] == X) {
    out[0] = t.stride[0]; out[1] = t.stride[1];
    return HOFA_OK;
  }
  if (t.ndim == 4 && t.shape[0] == 1 && t.shape[1] == H && t.shape[2] == 1 && t.shape[3] == X) {
    out[0] = t.stride[1]; out[1] = t.stride[3];
    return HOFA_OK;
  }
  return fail(HOFA_ERR_INVALID_ARGUMENT, "%s: expected [H=%lld, %lld] or [1,H,1,%lld]", name, (long long)H,
              (long long)X, (long long)X);
}

// log_alpha given as [1|B,H,1,J] or [H,J]: strides of (b, h, j).
int alpha_strides(const hofa_tensor& t, int64_t B, int64_t H, int64_t J, int64_t out[3]) {
  if (!dtype_ok(t.dtype)) return fail(HOFA_ERR_INVALID_ARGUMENT, "log_alpha: unknown dtype");
  if (t.ndim == 4 && (t.shape[0] == 1 || t.shape[0] == B) && t.shape[1] == H && t.shape[2] == 1 && t.shape[3] == J) {
    out[0] = t.shape[0] > 1 ? t.stride[0] : 0; out[1] = t.stride[1]; out[2] = t.stride[3];
    return HOFA_OK;
  }
  if (t.ndim == 2 && t.shape[0] == H && t.shape[1] == J) {
    out[0] = 0; out[1] = t.stride[0]; out[2] = t.stride[1];
    return HOFA_OK;
  }
  return fail(HOFA_ERR_INVALID_ARGUMENT, "log_alpha: expected [1|B,H,1,J=%lld] or [H,J]", (long long)J);
}

int g_num_sms[64];

int num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (g_num_sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_num_sms[dev] = n;
  }
  return g_num_sms[dev];
}

// Tuning overrides for sweeps of the decode kernel, read once when the
// library is loaded (never per launch).  Unset: the measured defaults below.
int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return (v != nullptr && v[0] != '\0') ? atoi(v) : dflt;
}
const bool kDecodeNoBulk = env_int("HOFA_DECODE_NO_BULK", 0) != 0;
const int kDecodeWarps = [] {
  const int w = env_int("HOFA_DECODE_WARPS", 4);
  return (w == 6 || w == 8) ? w : 4;
}();
const bool kDecodeNoL2Prefetch = env_int("HOFA_DECODE_NO_L2_PREFETCH", 0) != 0;
const int kDecodeStages = env_int("HOFA_DECODE_STAGES", 0);  // 0: choose by shape
// Steps of up to this many MB of cache rows ask L2 to prefetch the first
// window of their ring (the chunks loaded first) before the grid dependency.
// Measured at the 4096-token config 1: B = 4 10.77 -> 10.49 us per step with
// the windowed prefetch; prefetching a split's whole range instead was slower
// above 24 MB (11.17 us at B = 4).
const int kDecodePrefetchMaxMB = env_int("HOFA_DECODE_PREFETCH_MAX_MB", 100);
const bool kDecodePrefetchWindow = env_int("HOFA_DECODE_PREFETCH_WINDOW", 1) != 0;

bool supported_d(int64_t D) { return D == 32 || D == 64 || D == 128; }

constexpr int kMaxSplit = 64;
constexpr int kAutoClusterMax = 16;
constexpr int kAutoClusterCap = 8;
constexpr int kMaxSegments = 64;

size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

namespace {

// Validation of hofa_decode_args and the kernel parameters (shared by
// hofa_decode_fwd, hofa_decode_step_fwd and the no-allocation entry point).
// With check_ws == false the workspace fields are not looked at (p.split_k
// and the size the workspace would need still come out).
int decode_setup(const hofa_decode_args* a, hofa::DecodeParams& p, int& path, bool& alpha, int& dt,
                 bool check_ws = true, size_t* ws_need = nullptr) {
  if (a == nullptr) return fail(HOFA_ERR_INVALID_ARGUMENT, "args is NULL");
  const int64_t B = a->q.shape[0], H = a->q.shape[1], D = a->q.shape[3];
  CHECK(a->q, "q", 4, -1, -1, 1, -1);
  if (B <= 0 || H <= 0) return fail(HOFA_ERR_INVALID_ARGUMENT, "q: empty batch or heads");
  if (!supported_d(D)) return fail(HOFA_ERR_UNSUPPORTED, "head dim %lld not built (32, 64, 128)", (long long)D);
  const int R = a->R;
  if (R < 0 || R > D) return fail(HOFA_ERR_INVALID_ARGUMENT, "R=%d outside [0, D=%lld]", R, (long long)D);
  const int64_t J = D - R;
  CHECK(a->k, "k", 4, B, H, 1, D);
  CHECK(a->v, "v", 4, B, H, 1, D);
  CHECK(a->y, "y", 4, B, H, 1, D);
  dt = a->q.dtype;
  if (a->k.dtype != dt || a->v.dtype != dt || a->y.dtype != dt)
    return fail(HOFA_ERR_INVALID_ARGUMENT, "q, k, v and y must share one dtype");
  int64_t L = 0;
  if (R > 0) {
    CHECK(a->cache_k, "cache_k", 4, B, H, -1, -1);
    L = a->cache_k.shape[2];
    if (a->cache_k.shape[3] < R) return fail(HOFA_ERR_INVALID_ARGUMENT, "cache_k: last dim < R");
    CHECK(a->cache_v, "cache_v", 4, B, H, L, D);
    if (a->cache_k.dtype != dt || a->cache_v.dtype != dt)
      return fail(HOFA_ERR_INVALID_ARGUMENT, "caches must have the dtype of q");
    if (L < 1) return fail(HOFA_ERR_INVALID_ARGUMENT, "empty cache");
    if (a->seq_len_dev == nullptr && (a->seq_len < 1 || a->seq_len > L))
      return fail(HOFA_ERR_INVALID_ARGUMENT, "seq_len=%d outside [1, L=%lld]", a->seq_len, (long long)L);
  }
  CHECK(a->state_in, "state_in", 4, B, H, J, D);
  CHECK(a->state_out, "state_out", 4, B, H, J, D);
  if (a->state_in.dtype != HOFA_DTYPE_F32 || a->state_out.dtype != HOFA_DTYPE_F32)
    return fail(HOFA_ERR_INVALID_ARGUMENT, "GLA states must be float32");
  for (const hofa_tensor* s : {&a->state_in, &a->state_out}) {
    if (J > 0 && (s->stride[3] != 1 || s->stride[2] % 4 || s->stride[1] % 4 || s->stride[0] % 4 || !aligned16(s->data)))
      return fail(HOFA_ERR_MISALIGNED, "GLA states need unit stride along D and 16-byte aligned rows");
  }
  if (J > 0 && a->state_in.data == a->state_out.data)
    return fail(HOFA_ERR_INVALID_ARGUMENT, "state_out must not alias state_in");

  memset(&p, 0, sizeof(p));
  int r = side_bht(a->log_gamma, "log_gamma", B, H, 1, p.slg);
  if (r) return r;
  int64_t tmp3[3];
  r = side_bht(a->mix_g, "mix_g", B, H, 1, tmp3);
  if (r) return r;
  p.smg[0] = tmp3[0]; p.smg[1] = tmp3[1];
  r = head_vec(a->norm_w, "norm_w", H, D, p.snw);
  if (r) return r;
  alpha = present(a->log_alpha);
  if (alpha) {
    r = alpha_strides(a->log_alpha, B, H, J, p.sla);
    if (r) return r;
  }

  const int sms = num_sms();
  int split = a->split_k;
  const int len_hint = a->seq_len_dev ? (int)L : a->seq_len;
  if (split <= 0) split = hofa_decode_choose_split((int)B, (int)H, len_hint, sms);
  if (split > kMaxSplit) return fail(HOFA_ERR_INVALID_ARGUMENT, "split_k=%d above %d", split, kMaxSplit);
  if (R == 0) split = 1;
  const size_t need = hofa_decode_workspace_size((int)B, (int)H, (int)D, split);
  if (ws_need != nullptr) *ws_need = need;
  if (check_ws) {
    if (a->workspace == nullptr || a->workspace_bytes < need)
      return fail(HOFA_ERR_WORKSPACE, "decode workspace needs %zu bytes, got %zu", need, a->workspace_bytes);
    if (!aligned16(a->workspace)) return fail(HOFA_ERR_MISALIGNED, "workspace must be 16-byte aligned");
  }

  p.q = a->q.data; p.k = a->k.data; p.v = a->v.data;
  p.cache_k = a->cache_k.data; p.cache_v = a->cache_v.data;
  p.state_in = (const float*)a->state_in.data; p.state_out = (float*)a->state_out.data;
  p.log_gamma = a->log_gamma.data; p.mix_g = a->mix_g.data; p.norm_w = a->norm_w.data;
  p.log_alpha = alpha ? a->log_alpha.data : nullptr;
  p.y = a->y.data;
  p.B = (int)B; p.H = (int)H; p.D = (int)D; p.R = R; p.L = (int)L;
  p.seq_len = a->seq_len; p.seq_len_dev = a->seq_len_dev;
  p.qk_scale_log2 = a->sm_scale * 1.4426950408889634f;
  p.eps = a->eps;
  p.split_k = split;
  for (int i = 0; i < 2; ++i) { p.sq[i] = a->q.stride[i]; p.sk[i] = a->k.stride[i]; p.sv[i] = a->v.stride[i]; p.sy[i] = a->y.stride[i]; }
  p.sq[2] = a->q.stride[3]; p.sk[2] = a->k.stride[3]; p.sv[2] = a->v.stride[3]; p.sy[2] = a->y.stride[3];
  if (R > 0) {
    for (int i = 0; i < 4; ++i) { p.sck[i] = a->cache_k.stride[i]; p.scv[i] = a->cache_v.stride[i]; }
  }
  for (int i = 0; i < 3; ++i) { p.sst[i] = a->state_in.stride[i]; p.sso[i] = a->state_out.stride[i]; }
  p.dt_lg = a->log_gamma.dtype; p.dt_mg = a->mix_g.dtype; p.dt_nw = a->norm_w.dtype;
  p.dt_la = alpha ? a->log_alpha.dtype : 0;
  char* ws = reinterpret_cast<char*>(a->workspace);
  p.ws_status = reinterpret_cast<int*>(ws);
  p.ws_count = reinterpret_cast<int*>(ws + 256);
  p.ws_part = reinterpret_cast<float*>(ws + 256 + round256((size_t)B * H * sizeof(int)));

  // 16-byte vector path: unit channel stride and 16-byte aligned rows
  const int es = esize(dt);
  bool vec = R > 0 && R % 8 == 0;
  if (vec) {
    for (const hofa_tensor* c : {&a->cache_k, &a->cache_v}) {
      vec = vec && c->stride[3] == 1 && aligned16(c->data);
      for (int i = 0; i < 3; ++i) vec = vec && ((c->stride[i] * es) % 16 == 0 || c->shape[i] == 1);
    }
  }
  // TMA bulk path: additionally, every (b,h) slab of cache rows is contiguous
  const bool bulk = vec && a->cache_k.stride[2] == R && a->cache_v.stride[2] == D && !kDecodeNoBulk;
  path = bulk ? 2 : (vec ? 1 : 0);
  // bulk ring: 64-token slots; a slot is always consumed by the same warp,
  // which requires stages % consumer_warps == 0
  p.consumer_warps = 4;
  p.stages = es == 4 ? 4 : 8;
  // A grid that does not fit at once with the 8-slot ring (80 KB at r=16,
  // d_h=64: two CTAs per SM) runs in waves; then the 4-slot ring, which keeps
  // more CTAs resident per SM, streams faster (measured at config 1: B=32
  // 90 -> 94 % and B=64 90 -> 97 % of the HBM roofline; one-wave grids such
  // as B=4, 8 and 16 are faster with 8 slots).
  if (es != 4) {
    const size_t ring8 = (size_t)8 * 64 * (R + D) * es;
    const int64_t per_sm8 = (int64_t)(228 * 1024 / (ring8 + 12 * 1024));
    if ((int64_t)B * H * split > (per_sm8 > 0 ? per_sm8 : 1) * (int64_t)sms) p.stages = 4;
  }
  p.consumer_warps = kDecodeWarps;
  p.no_l2_prefetch = kDecodeNoL2Prefetch ||
                     (double)B * H * (a->seq_len_dev ? L : a->seq_len) * (R + D) * es > kDecodePrefetchMaxMB * 1e6;
  p.prefetch_window = kDecodePrefetchWindow;
  if (kDecodeStages >= 2 && kDecodeStages <= 16) p.stages = kDecodeStages;
  p.stages = ((p.stages + p.consumer_warps - 1) / p.consumer_warps) * p.consumer_warps;
  const size_t ring_budget = 200 * 1024;  // dynamic shared memory of the ring (the kernel adds ~12 KB static)
  while (p.stages > p.consumer_warps && (size_t)p.stages * 64 * (R + D) * es > ring_budget) p.stages -= p.consumer_warps;
  if (p.stages > 16 || (size_t)p.stages * 64 * (R + D) * es > ring_budget) {
    p.consumer_warps = 4;
    p.stages = 4;
  }
  // rows too wide for even a 4-slot ring (float32 with large R at d_h = 128):
  // stream with 16-byte register loads instead
  if (path == 2 && (size_t)p.stages * 64 * (R + D) * es > ring_budget) path = 1;
  return HOFA_OK;
}

// Validation of hofa_prep_args and the kernel parameters (shared by
// hofa_prep_fwd and hofa_decode_step_fwd).  `empty` is set for N == 0.
int prep_setup(const hofa_prep_args* a, hofa::PrepParams& p, int& dt, bool& empty) {
  if (a == nullptr) return fail(HOFA_ERR_INVALID_ARGUMENT, "args is NULL");
  const int64_t B = a->q.shape[0], H = a->q.shape[1], N = a->q.shape[2], D = a->q.shape[3];
  CHECK(a->q, "q", 4, -1, -1, -1, -1);
  CHECK(a->k, "k", 4, B, H, N, D);
  if (!supported_d(D)) return fail(HOFA_ERR_UNSUPPORTED, "head dim %lld not built (32, 64, 128)", (long long)D);
  dt = a->q.dtype;
  if (a->k.dtype != dt) return fail(HOFA_ERR_INVALID_ARGUMENT, "q and k must share one dtype");
  const int R = a->R;
  if (R < 0 || R > D || (R % 2)) return fail(HOFA_ERR_INVALID_ARGUMENT, "R=%d must be even and in [0, D]", R);
  memset(&p, 0, sizeof(p));
  CHECK(a->gate_w, "gate_w", 2, H, 2 * D);
  CHECK(a->gate_b, "gate_b", 1, H);
  p.sgw[0] = a->gate_w.stride[0]; p.sgw[1] = a->gate_w.stride[1]; p.sgb = a->gate_b.stride[0];
  if (present(a->mix_w)) {
    CHECK(a->mix_w, "mix_w", 2, H, 2 * D);
    CHECK(a->mix_b, "mix_b", 1, H);
    p.smw[0] = a->mix_w.stride[0]; p.smw[1] = a->mix_w.stride[1]; p.smb = a->mix_b.stride[0];
  } else if (present(a->fixed_mix)) {
    CHECK(a->fixed_mix, "fixed_mix", 1, H);
    p.sfm = a->fixed_mix.stride[0];
  }
  int r = side_bht(a->log_gamma, "log_gamma", B, H, N, p.slg);
  if (r) return r;
  if (present(a->mix_out)) {
    if (!present(a->mix_w) && !present(a->fixed_mix))
      return fail(HOFA_ERR_INVALID_ARGUMENT, "mix_out requested without mix_w or fixed_mix");
    r = side_bht(a->mix_out, "mix_out", B, H, N, p.smo);
    if (r) return r;
  }
  const bool rope = a->use_rope != 0 && R > 0;
  if (rope) {
    CHECK(a->cos, "cos", 2, -1, -1);
    CHECK(a->sin, "sin", 2, a->cos.shape[0], -1);
    if (a->cos.shape[1] < R || a->sin.shape[1] < R) return fail(HOFA_ERR_INVALID_ARGUMENT, "RoPE tables narrower than R");
    if (a->sin.dtype != a->cos.dtype) return fail(HOFA_ERR_INVALID_ARGUMENT, "cos/sin dtypes differ");
    p.P = (int)a->cos.shape[0];
    if (a->pos0_dev == nullptr && a->pos0 + N > p.P)
      return fail(HOFA_ERR_INVALID_ARGUMENT, "RoPE tables hold %d positions, need %lld", p.P, (long long)(a->pos0 + N));
    p.scos[0] = a->cos.stride[0]; p.scos[1] = a->cos.stride[1];
    p.ssin[0] = a->sin.stride[0]; p.ssin[1] = a->sin.stride[1];
    p.dt_cs = a->cos.dtype;
  }
  p.L = 0;
  if (present(a->cache_k) || present(a->cache_v)) {
    if (R > 0) {
      CHECK(a->cache_k, "cache_k", 4, B, H, -1, -1);
      if (a->cache_k.shape[3] < R) return fail(HOFA_ERR_INVALID_ARGUMENT, "cache_k: last dim < R");
    }
    const int64_t L = R > 0 ? a->cache_k.shape[2] : a->cache_v.shape[2];
    CHECK(a->cache_v, "cache_v", 4, B, H, L, D);
    CHECK(a->v, "v", 4, B, H, N, D);
    if ((R > 0 && a->cache_k.dtype != dt) || a->cache_v.dtype != dt || a->v.dtype != dt)
      return fail(HOFA_ERR_INVALID_ARGUMENT, "caches and v must have the dtype of q");
    if (a->pos0_dev == nullptr && (a->pos0 < 0 || a->pos0 + N > L))
      return fail(HOFA_ERR_INVALID_ARGUMENT, "cache rows [%d, %lld) outside [0, %lld)", a->pos0,
                  (long long)(a->pos0 + N), (long long)L);
    p.L = (int)L;
    for (int i = 0; i < 4; ++i) {
      if (R > 0) p.sck[i] = a->cache_k.stride[i];
      p.scv[i] = a->cache_v.stride[i];
      p.sv[i] = a->v.stride[i];
    }
  }
  if (a->pos0 < 0) return fail(HOFA_ERR_INVALID_ARGUMENT, "pos0 must be >= 0");
  if (N == 0) { empty = true; return HOFA_OK; }
  p.q = a->q.data; p.k = a->k.data; p.v = a->v.data;
  p.gate_w = a->gate_w.data; p.gate_b = a->gate_b.data;
  p.mix_w = present(a->mix_w) ? a->mix_w.data : nullptr;
  p.mix_b = present(a->mix_w) ? a->mix_b.data : nullptr;
  p.fixed_mix = (!present(a->mix_w) && present(a->fixed_mix)) ? a->fixed_mix.data : nullptr;
  p.cos = rope ? a->cos.data : nullptr; p.sin = rope ? a->sin.data : nullptr;
  p.log_gamma = a->log_gamma.data;
  p.mix_out = present(a->mix_out) ? a->mix_out.data : nullptr;
  p.cache_k = (R > 0 && present(a->cache_k)) ? a->cache_k.data : nullptr;
  p.cache_v = present(a->cache_v) ? a->cache_v.data : nullptr;
  p.B = (int)B; p.H = (int)H; p.N = (int)N; p.D = (int)D; p.R = R;
  p.pos0 = a->pos0; p.pos0_dev = a->pos0_dev;
  p.rope = rope;
  for (int i = 0; i < 4; ++i) { p.sq[i] = a->q.stride[i]; p.sk[i] = a->k.stride[i]; }
  p.dt_gw = a->gate_w.dtype; p.dt_gb = a->gate_b.dtype;
  p.dt_mw = p.mix_w ? a->mix_w.dtype : 0; p.dt_mb = p.mix_b ? a->mix_b.dtype : 0;
  p.dt_fm = p.fixed_mix ? a->fixed_mix.dtype : 0;
  p.dt_lg = a->log_gamma.dtype; p.dt_mo = p.mix_out ? a->mix_out.dtype : 0;
  // 16-byte row path: unit channel stride and 16-byte aligned rows for q, k (and v / caches when written)
  {
    auto rows16 = [](const hofa_tensor& t) {
      if (t.stride[3] != 1 || !aligned16(t.data)) return false;
      for (int i = 0; i < 3; ++i)
        if ((t.stride[i] * 2) % 16 != 0 && t.shape[i] != 1) return false;
      return true;
    };
    bool vec = dt != HOFA_DTYPE_F32 && R % 8 == 0 && rows16(a->q) && rows16(a->k);
    if (p.cache_k) vec = vec && rows16(a->cache_k);
    if (p.cache_v) vec = vec && rows16(a->cache_v) && rows16(a->v);
    p.vec = vec;
  }
  return HOFA_OK;
}

}  // namespace

namespace hofa {
// Records `message` as the calling thread's last error and returns `code`
// (for entry points defined outside this file).
int set_last_error(int code, const char* message) {
  g_err = message;
  return code;
}

// Validates `a` exactly as hofa_decode_fwd does, except for the workspace
// fields, and returns the split count hofa_decode_fwd will launch with and
// the workspace bytes that split needs (for the no-allocation entry point,
// which sizes its built-in scratch with this before touching the device).
int decode_plan(const hofa_decode_args* a, int32_t* split, size_t* ws_need) {
  DecodeParams p;
  int path = 0, dt = 0;
  bool alpha = false;
  const int st = decode_setup(a, p, path, alpha, dt, /*check_ws=*/false, ws_need);
  if (st != HOFA_OK) return st;
  *split = p.split_k;
  return HOFA_OK;
}
}  // namespace hofa

extern "C" {

const char* hofa_last_error(void) { return g_err.c_str(); }
int32_t hofa_abi_version(void) { return HOFA_ABI_VERSION; }

// ---------------------------------------------------------------------------
// decode
// ---------------------------------------------------------------------------
int32_t hofa_decode_choose_split(int32_t B, int32_t H, int32_t seq_len, int32_t sms) {
  if (B <= 0 || H <= 0) return 1;
  if (sms <= 0) sms = 148;
  // about two resident CTAs of the cache-streaming kernel per SM, at least
  // 256 tokens a split; up to 16 splits run as one thread-block cluster per
  // head (a power of two), more splits combine through the workspace
  const int64_t heads = (int64_t)B * H;
  int64_t s = (2 * (int64_t)sms) / heads;
  const int64_t by_len = seq_len / 256 > 1 ? seq_len / 256 : 1;
  if (s > by_len) s = by_len;
  if (s > kMaxSplit) s = kMaxSplit;
  if (s < 1) s = 1;
  if (s <= kAutoClusterMax) {
    int64_t p2 = 1;
    while (p2 * 2 <= s) p2 *= 2;
    s = p2 < kAutoClusterCap ? p2 : kAutoClusterCap;  // clusters above 8 CTAs schedule poorly
    // clusters of 8 that need more CTAs than there are SMs do not all fit in
    // one wave; 6 do (measured at B=2, H=16, L=4096: 8.1 us with 6 splits,
    // 10.5 us with 8, 9.3 us with 4)
    if (s == 8 && heads * 8 > sms) s = 6;
  }
  return (int32_t)s;
}

size_t hofa_decode_workspace_size(int32_t B, int32_t H, int32_t D, int32_t max_split_k) {
  if (max_split_k <= 0 || max_split_k > kMaxSplit) max_split_k = kMaxSplit;
  const size_t heads = (size_t)(B > 0 ? B : 0) * (size_t)(H > 0 ? H : 0);
  return 256 + round256(heads * sizeof(int)) + heads * (size_t)max_split_k * (4 + 2 * (size_t)D) * sizeof(float);
}

int hofa_decode_read_status(void* workspace, void* stream, int32_t* status_out) {
  if (workspace == nullptr || status_out == nullptr) return fail(HOFA_ERR_INVALID_ARGUMENT, "NULL argument");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int32_t v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(workspace, 0, sizeof(int32_t), st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "hofa_decode_read_status");
  *status_out = v;
  return HOFA_OK;
}

int hofa_decode_fwd(const hofa_decode_args* a, void* stream) {
  hofa::DecodeParams p;
  int path = 0, dt = 0;
  bool alpha = false;
  const int st = decode_setup(a, p, path, alpha, dt);
  if (st != HOFA_OK) return st;
  cudaError_t e = hofa::launch_decode(p, dt, path, alpha, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "hofa_decode_fwd launch");
  return HOFA_OK;
}

// ---------------------------------------------------------------------------
// prefill GLA
// ---------------------------------------------------------------------------
static void gla_geometry(int64_t B, int64_t H, int64_t T, int64_t D, int nseg_req, int sms,
                        int* nseg, int* seg_len, int* chunk) {
  const int C = hofa::gla_internal_chunk((int)D);
  const int64_t nchunks = (T + C - 1) / C;
  int64_t s = nseg_req;
  if (s <= 0) s = (2 * (int64_t)sms + B * H - 1) / (B * H);
  if (s > kMaxSegments) s = kMaxSegments;
  if (s > nchunks) s = nchunks;
  if (s < 1) s = 1;
  const int64_t chunks_per = (nchunks + s - 1) / s;
  *seg_len = (int)(chunks_per * C);
  *nseg = (int)((T + *seg_len - 1) / *seg_len);
  if (*nseg < 1) *nseg = 1;
  *chunk = C;
}

size_t hofa_gla_workspace_size(int32_t B, int32_t H, int32_t T, int32_t D, int32_t R, int32_t chunk_size,
                               int32_t num_segments) {
  (void)chunk_size;
  if (B <= 0 || H <= 0 || T <= 0 || D <= 0 || R < 0 || R > D) return 0;
  const int C = hofa::gla_internal_chunk(D);
  int64_t nseg = num_segments > 0 ? num_segments : kMaxSegments;
  if (nseg > kMaxSegments) nseg = kMaxSegments;
  const int64_t nchunks = (T + C - 1) / C;
  if (nseg > nchunks) nseg = nchunks;
  const int64_t J = D - R;
  const size_t cuda_core = (size_t)B * H * nseg * (J * D + J) * sizeof(float) + 256;
  const size_t tensor_core = hofa::gla_tc_workspace_bytes(B, H, T, J, D);
  return cuda_core > tensor_core ? cuda_core : tensor_core;
}

int hofa_prefill_gla_fwd(const hofa_gla_args* a, void* stream) {
  if (a == nullptr) return fail(HOFA_ERR_INVALID_ARGUMENT, "args is NULL");
  const int64_t B = a->q.shape[0], H = a->q.shape[1], T = a->q.shape[2], D = a->q.shape[3];
  CHECK(a->q, "q", 4, -1, -1, -1, -1);
  if (B <= 0 || H <= 0) return fail(HOFA_ERR_INVALID_ARGUMENT, "q: empty batch or heads");
  if (!supported_d(D)) return fail(HOFA_ERR_UNSUPPORTED, "head dim %lld not built (32, 64, 128)", (long long)D);
  const int R = a->R;
  if (R < 0 || R >= D) return fail(HOFA_ERR_INVALID_ARGUMENT, "R=%d outside [0, D)", R);
  const int64_t J = D - R;
  CHECK(a->k, "k", 4, B, H, T, D);
  CHECK(a->v, "v", 4, B, H, T, D);
  CHECK(a->y, "y", 4, B, H, T, D);
  const int dt = a->q.dtype;
  if (a->k.dtype != dt || a->v.dtype != dt || a->y.dtype != dt)
    return fail(HOFA_ERR_INVALID_ARGUMENT, "q, k, v and y must share one dtype");
  if (a->chunk_size <= 0) return fail(HOFA_ERR_INVALID_ARGUMENT, "chunk_size must be positive");
  hofa::GlaParams p;
  memset(&p, 0, sizeof(p));
  int r = side_bht(a->log_gamma, "log_gamma", B, H, T, p.slg);
  if (r) return r;
  p.fuse = present(a->mix_g) && present(a->gla_scale);
  if (p.fuse) {
    r = side_bht(a->mix_g, "mix_g", B, H, T, p.smg);
    if (r) return r;
    r = head_vec(a->gla_scale, "gla_scale", H, D, p.sgs);
    if (r) return r;
  }
  const bool alpha = present(a->log_alpha);
  if (alpha) {
    r = alpha_strides(a->log_alpha, B, H, J, p.sla);
    if (r) return r;
  }
  if (present(a->state_init)) {
    CHECK(a->state_init, "state_init", 4, B, H, J, D);
    if (a->state_init.dtype != HOFA_DTYPE_F32 || a->state_init.stride[3] != 1)
      return fail(HOFA_ERR_INVALID_ARGUMENT, "state_init must be float32 with unit stride along D");
  }
  if (present(a->state_out)) {
    CHECK(a->state_out, "state_out", 4, B, H, J, D);
    if (a->state_out.dtype != HOFA_DTYPE_F32) return fail(HOFA_ERR_INVALID_ARGUMENT, "state_out must be float32");
  }
  if (T == 0) return HOFA_OK;
  // tensor-core path: chunk-parallel tcgen05 kernels (bf16/f16, head dim 64 or 128, scalar or per-channel decay)
  {
    hofa::GlaParams tp;
    memset(&tp, 0, sizeof(tp));
    tp.D = (int)D; tp.R = R; tp.log_alpha = alpha ? a->log_alpha.data : nullptr;
    const size_t need_tc = hofa::gla_tc_workspace_bytes(B, H, T, J, D);
    if (hofa::gla_tc_eligible(tp, dt) && a->workspace != nullptr && a->workspace_bytes >= need_tc &&
        ((reinterpret_cast<uintptr_t>(a->workspace) & 15u) == 0)) {
      tp = p;  // side-tensor strides filled above
      tp.q = a->q.data; tp.k = a->k.data; tp.v = a->v.data;
      tp.log_gamma = a->log_gamma.data;
      tp.log_alpha = alpha ? a->log_alpha.data : nullptr;
      tp.dt_la = alpha ? a->log_alpha.dtype : 0;
      tp.mix_g = p.fuse ? a->mix_g.data : nullptr;
      tp.gla_scale = p.fuse ? a->gla_scale.data : nullptr;
      tp.state_init = present(a->state_init) ? (const float*)a->state_init.data : nullptr;
      tp.y = a->y.data;
      tp.state_out = present(a->state_out) ? (float*)a->state_out.data : nullptr;
      tp.B = (int)B; tp.H = (int)H; tp.T = (int)T; tp.D = (int)D; tp.R = R; tp.J = (int)J;
      tp.chunk = hofa::gla_tc_chunk();
      tp.nseg = (int)((T + tp.chunk - 1) / tp.chunk);
      tp.seg_len = tp.chunk;
      tp.eps = a->eps;
      for (int i = 0; i < 4; ++i) {
        tp.sq[i] = a->q.stride[i]; tp.sk[i] = a->k.stride[i]; tp.sv[i] = a->v.stride[i]; tp.sy[i] = a->y.stride[i];
      }
      if (tp.state_init) for (int i = 0; i < 3; ++i) tp.ssi[i] = a->state_init.stride[i];
      if (tp.state_out) for (int i = 0; i < 4; ++i) tp.sso[i] = a->state_out.stride[i];
      tp.dt_lg = a->log_gamma.dtype;
      tp.dt_mg = p.fuse ? a->mix_g.dtype : 0;
      tp.dt_gs = p.fuse ? a->gla_scale.dtype : 0;
      hofa::gla_tc_bind_workspace(tp, a->workspace);
      bool taken = false;
      cudaError_t e = hofa::launch_gla_tc(tp, dt, reinterpret_cast<cudaStream_t>(stream), &taken);
      if (e != cudaSuccess) return cuda_fail(e, "hofa_prefill_gla_fwd launch (tensor cores)");
      if (taken) return HOFA_OK;
    }
  }
  int nseg, seg_len, C;
  gla_geometry(B, H, T, D, a->num_segments, num_sms(), &nseg, &seg_len, &C);
  const size_t need = (size_t)B * H * nseg * (J * D + J) * sizeof(float);
  if (nseg > 1 && (a->workspace == nullptr || a->workspace_bytes < need))
    return fail(HOFA_ERR_WORKSPACE, "GLA workspace needs %zu bytes, got %zu", need, a->workspace_bytes);

  p.q = a->q.data; p.k = a->k.data; p.v = a->v.data;
  p.log_gamma = a->log_gamma.data;
  p.log_alpha = alpha ? a->log_alpha.data : nullptr;
  p.mix_g = p.fuse ? a->mix_g.data : nullptr;
  p.gla_scale = p.fuse ? a->gla_scale.data : nullptr;
  p.state_init = present(a->state_init) ? (const float*)a->state_init.data : nullptr;
  p.y = a->y.data;
  p.state_out = present(a->state_out) ? (float*)a->state_out.data : nullptr;
  p.B = (int)B; p.H = (int)H; p.T = (int)T; p.D = (int)D; p.R = R; p.J = (int)J;
  p.chunk = C; p.nseg = nseg; p.seg_len = seg_len;
  p.eps = a->eps;
  for (int i = 0; i < 4; ++i) {
    p.sq[i] = a->q.stride[i]; p.sk[i] = a->k.stride[i]; p.sv[i] = a->v.stride[i]; p.sy[i] = a->y.stride[i];
  }
  if (p.state_init) for (int i = 0; i < 3; ++i) p.ssi[i] = a->state_init.stride[i];
  if (p.state_out) for (int i = 0; i < 4; ++i) p.sso[i] = a->state_out.stride[i];
  p.dt_lg = a->log_gamma.dtype;
  p.dt_mg = p.fuse ? a->mix_g.dtype : 0;
  p.dt_gs = p.fuse ? a->gla_scale.dtype : 0;
  p.dt_la = alpha ? a->log_alpha.dtype : 0;
  p.ws_state = reinterpret_cast<float*>(a->workspace);
  p.ws_decay = p.ws_state ? p.ws_state + (size_t)B * H * nseg * J * D : nullptr;
  cudaError_t e = hofa::launch_gla(p, dt, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "hofa_prefill_gla_fwd launch");
  return HOFA_OK;
}

// ---------------------------------------------------------------------------
// prefill outlier attention
// ---------------------------------------------------------------------------
int hofa_prefill_outlier_fwd(const hofa_outlier_args* a, void* stream) {
  if (a == nullptr) return fail(HOFA_ERR_INVALID_ARGUMENT, "args is NULL");
  const int64_t B = a->q.shape[0], H = a->q.shape[1], Tq = a->q.shape[2];
  CHECK(a->q, "q", 4, -1, -1, -1, -1);
  const int64_t Tk = a->k.shape[2];
  CHECK(a->k, "k", 4, B, H, -1, -1);
  const int64_t D = a->v.shape[3];
  CHECK(a->v, "v", 4, B, H, Tk, -1);
  CHECK(a->out, "out", 4, B, H, Tq, D);
  if (!supported_d(D)) return fail(HOFA_ERR_UNSUPPORTED, "value dim %lld not built (32, 64, 128)", (long long)D);
  const int R = a->R;
  if (R < 1 || R > D || R > a->q.shape[3] || R > a->k.shape[3])
    return fail(HOFA_ERR_INVALID_ARGUMENT, "R=%d outside [1, min(D, q/k channels)]", R);
  const int dt = a->q.dtype;
  if (a->k.dtype != dt || a->v.dtype != dt || a->out.dtype != dt)
    return fail(HOFA_ERR_INVALID_ARGUMENT, "q, k, v and out must share one dtype");
  if (a->q_offset < 0) return fail(HOFA_ERR_INVALID_ARGUMENT, "q_offset must be >= 0");
  hofa::OutlierParams p;
  memset(&p, 0, sizeof(p));
  int r = side_bht(a->mix_g, "mix_g", B, H, Tq, p.smg);
  if (r) return r;
  if (Tq == 0) return HOFA_OK;
  if (Tk < 1) return fail(HOFA_ERR_INVALID_ARGUMENT, "no keys");
  p.q = a->q.data; p.k = a->k.data; p.v = a->v.data; p.mix_g = a->mix_g.data; p.out = a->out.data;
  p.B = (int)B; p.H = (int)H; p.Tq = (int)Tq; p.Tk = (int)Tk; p.D = (int)D; p.R = R;
  p.q_offset = a->q_offset;
  p.qk_scale_log2 = a->sm_scale * 1.4426950408889634f;
  p.accumulate = a->accumulate != 0;
  for (int i = 0; i < 4; ++i) {
    p.sq[i] = a->q.stride[i]; p.sk[i] = a->k.stride[i]; p.sv[i] = a->v.stride[i]; p.so[i] = a->out.stride[i];
  }
  p.dt_mg = a->mix_g.dtype;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  bool taken = false;
  cudaError_t e = hofa::launch_outlier_tc(p, dt, st, &taken);
  if (!taken) e = hofa::launch_outlier_generic(p, dt, st);
  if (e != cudaSuccess) return cuda_fail(e, "hofa_prefill_outlier_fwd launch");
  return HOFA_OK;
}

int hofa_prefill_read_status(void* stream, int32_t* status_out) {
  if (status_out == nullptr) return fail(HOFA_ERR_INVALID_ARGUMENT, "NULL argument");
  int v = 0, w = 0;
  cudaError_t e = hofa::read_outlier_tc_status(&v, reinterpret_cast<cudaStream_t>(stream));
  if (e == cudaSuccess) e = hofa::read_gla_tc_status(&w, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "hofa_prefill_read_status");
  *status_out = v | (w << 1);
  return HOFA_OK;
}

// ---------------------------------------------------------------------------
// gates + RoPE + cache export
// ---------------------------------------------------------------------------
int hofa_prep_fwd(const hofa_prep_args* a, void* stream) {
  hofa::PrepParams p;
  int dt = 0;
  bool empty = false;
  const int st = prep_setup(a, p, dt, empty);
  if (st != HOFA_OK || empty) return st;
  cudaError_t e = hofa::launch_prep(p, dt, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "hofa_prep_fwd launch");
  return HOFA_OK;
}

// ---------------------------------------------------------------------------
// decode step: the new token's prep and the decode in one launch
// ---------------------------------------------------------------------------
int hofa_decode_step_fwd(const hofa_decode_args* d, const hofa_prep_args* pr, void* stream) {
  if (d == nullptr || pr == nullptr) return fail(HOFA_ERR_INVALID_ARGUMENT, "args is NULL");
  if (pr->q.data != d->q.data || pr->k.data != d->k.data || pr->v.data != d->v.data)
    return fail(HOFA_ERR_INVALID_ARGUMENT, "prep and decode must name the same q, k, v");
  if (!present(d->cache_k) || pr->cache_k.data != d->cache_k.data || pr->cache_v.data != d->cache_v.data)
    return fail(HOFA_ERR_INVALID_ARGUMENT, "prep must append to the decode's caches");
  if (!present(pr->mix_out)) return fail(HOFA_ERR_INVALID_ARGUMENT, "mix_out is required (the blend weight)");
  // the new token's position is the decode's last row: seq_len - 1
  hofa_prep_args pa = *pr;
  pa.pos0 = d->seq_len_dev != nullptr ? 0 : d->seq_len - 1;
  pa.pos0_dev = d->seq_len_dev;
  hofa::PrepParams pp;
  int pdt = 0;
  bool empty = false;
  int st = prep_setup(&pa, pp, pdt, empty);
  if (st != HOFA_OK) return st;
  if (pp.N != 1) return fail(HOFA_ERR_INVALID_ARGUMENT, "a decode step takes one token (N=1)");
  pp.pos0_dev_bias = d->seq_len_dev != nullptr ? -1 : 0;
  hofa_decode_args da = *d;
  da.log_gamma = pr->log_gamma;
  da.mix_g = pr->mix_out;
  hofa::DecodeParams dp;
  int path = 0, dt = 0;
  bool alpha = false;
  st = decode_setup(&da, dp, path, alpha, dt);
  if (st != HOFA_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool fuse = path == 2 && dp.R > 0 && pdt == dt;
  if (!fuse) {  // the same computation as two launches
    cudaError_t e = hofa::launch_prep(pp, pdt, s);
    if (e != cudaSuccess) return cuda_fail(e, "hofa_decode_step_fwd prep launch");
    e = hofa::launch_decode(dp, dt, path, alpha, s);
    if (e != cudaSuccess) return cuda_fail(e, "hofa_decode_step_fwd decode launch");
    return HOFA_OK;
  }
  dp.fused_prep = true;
  dp.consumer_warps = 4;
  dp.gate_w = pp.gate_w; dp.gate_b = pp.gate_b; dp.mix_w = pp.mix_w; dp.mix_b = pp.mix_b; dp.fixed_mix = pp.fixed_mix;
  dp.rope_cos = pp.cos; dp.rope_sin = pp.sin;
  dp.rope_rows = pp.rope ? pp.P : 0;
  dp.log_gamma_out = pp.log_gamma; dp.mix_out = pp.mix_out;
  for (int i = 0; i < 2; ++i) {
    dp.sgw[i] = pp.sgw[i]; dp.smw[i] = pp.smw[i]; dp.scos[i] = pp.scos[i]; dp.ssin[i] = pp.ssin[i];
    dp.slgo[i] = pp.slg[i]; dp.smo[i] = pp.smo[i];
  }
  dp.sgb = pp.sgb; dp.smb = pp.smb; dp.sfm = pp.sfm;
  dp.dt_gw = pp.dt_gw; dp.dt_gb = pp.dt_gb; dp.dt_mw = pp.dt_mw; dp.dt_mb = pp.dt_mb; dp.dt_fm = pp.dt_fm;
  dp.dt_cs = pp.dt_cs; dp.dt_lgo = pp.dt_lg; dp.dt_mo = pp.dt_mo;
  cudaError_t e = hofa::launch_decode(dp, dt, path, alpha, s);
  if (e != cudaSuccess) return cuda_fail(e, "hofa_decode_step_fwd launch");
  return HOFA_OK;
}

}  // extern "C"
