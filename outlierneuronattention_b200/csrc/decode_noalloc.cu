// hofa_decode_fwd_noalloc: the decode step for callers that cannot allocate.
//
// hofa_decode_fwd needs a caller-provided workspace (split partials, the
// per-head tickets of the last-CTA combine and a status word).  Some callers
// cannot provide one: code that runs where device allocation is forbidden or
// unavailable -- a host runtime that owns every allocation and exposes no
// allocator to plugins, a real-time loop that must never enter the driver's
// allocator (cudaMalloc may synchronise the device and take an unbounded
// time), or glue that only holds borrowed pointers to inputs and outputs.
// This entry point uses a fixed scratch array that lives in the library
// itself instead, so the caller passes nothing but its inputs and outputs.
//
// Limits and behaviour:
//   * the scratch is kNoAllocScratchBytes (2 MiB) of static device memory;
//     every GPU that loads the library holds it until the process exits;
//   * calls whose shapes need more scratch (hofa_decode_workspace_size() of
//     B, H, D and the split count in use) are rejected with
//     HOFA_ERR_WORKSPACE and a message naming both sizes;
//   * all calls share the one array: calls that overlap on the GPU (two
//     streams, or two host threads) race on it and must be serialised by the
//     caller;
//   * the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current) and caches it; make that
//     first call before any stream capture;
//   * the ticket and status words must start at zero; every call clears them
//     (an asynchronous memset on the caller's stream) before the kernel runs,
//     so nothing left by an earlier call can leak into the next one;
//   * no cudaMalloc, cudaFree or other allocating routine is called.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/hofa.h"

namespace hofa {
int set_last_error(int code, const char* message);  // capi.cu
}

namespace {

constexpr size_t kNoAllocScratchBytes = 2u << 20;

static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once
// per device, with that device current).
int scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return hofa::set_last_error(HOFA_ERR_CUDA, "hofa_decode_fwd_noalloc: no usable current CUDA device");
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr)
      return hofa::set_last_error(HOFA_ERR_CUDA, cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return HOFA_OK;
}

}  // namespace

extern "C" int hofa_decode_fwd_noalloc(const hofa_decode_args* args, void* stream) {
  if (args == nullptr) return hofa_decode_fwd(args, stream);
  hofa_decode_args a = *args;
  const int64_t B = a.q.shape[0], H = a.q.shape[1], D = a.q.shape[3];
  size_t zero_bytes = 256;
  if (a.q.ndim == 4 && B > 0 && H > 0 && D > 0) {
    // the split this call will use, chosen exactly as hofa_decode_fwd chooses it
    int split = a.split_k;
    if (split <= 0) {
      int dev = 0, sms = 148;
      if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      const int len_hint = a.seq_len_dev != nullptr && a.cache_k.ndim == 4 ? (int)a.cache_k.shape[2] : a.seq_len;
      split = hofa_decode_choose_split((int32_t)B, (int32_t)H, len_hint, sms);
    }
    if (a.R == 0) split = 1;
    const size_t need = (B * H > ((int64_t)1 << 24)) ? (size_t)-1
                                                     : hofa_decode_workspace_size((int32_t)B, (int32_t)H, (int32_t)D, split);
    if (need > kNoAllocScratchBytes) {
      char msg[256];
      snprintf(msg, sizeof(msg),
               "hofa_decode_fwd_noalloc: this call needs %zu bytes of scratch (B=%lld, H=%lld, D=%lld, split_k=%d) "
               "but the built-in array holds %zu; pass a workspace to hofa_decode_fwd instead",
               need, (long long)B, (long long)H, (long long)D, split, kNoAllocScratchBytes);
      return hofa::set_last_error(HOFA_ERR_WORKSPACE, msg);
    }
    a.split_k = split;
    zero_bytes = 256 + (((size_t)B * (size_t)H * sizeof(int) + 255) & ~size_t(255));  // status word + tickets
  }
  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st != HOFA_OK) return st;
  const cudaError_t e = cudaMemsetAsync(scratch, 0, zero_bytes, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return hofa::set_last_error(HOFA_ERR_CUDA, cudaGetErrorString(e));
  a.workspace = scratch;
  a.workspace_bytes = kNoAllocScratchBytes;
  return hofa_decode_fwd(&a, stream);
}
