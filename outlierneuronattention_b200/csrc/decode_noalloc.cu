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
//   * the arguments are validated exactly as hofa_decode_fwd validates them,
//     and the split count is the one hofa_decode_fwd will launch with
//     (hofa::decode_plan), before anything is issued on the device; calls
//     whose shapes need more scratch (hofa_decode_workspace_size() of B, H,
//     D and that split count) are rejected with HOFA_ERR_WORKSPACE and a
//     message naming both sizes;
//   * all calls share the one array: calls that overlap on the GPU (two
//     streams, or two host threads) race on it and must be serialised by the
//     caller;
//   * the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current) and caches it; make that
//     first call before any stream capture;
//   * the per-head tickets of the combine must start at zero; every call
//     clears them (an asynchronous memset on the caller's stream) before the
//     kernel runs, so a ticket left by an interrupted earlier call cannot leak
//     into the next one;
//   * the status word (device-side faults: a clamped seq_len_dev, a ring or
//     combine wait that ran out) collects the bits of every call since it was
//     last read; hofa_decode_noalloc_read_status() returns and clears it;
//   * no cudaMalloc, cudaFree or other allocating routine is called.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/hofa.h"

namespace hofa {
int set_last_error(int code, const char* message);                            // capi.cu
int decode_plan(const hofa_decode_args* a, int32_t* split, size_t* ws_need);  // capi.cu
}

namespace {

constexpr size_t kNoAllocScratchBytes = 2u << 20;
constexpr size_t kTicketOffset = 256;  // the status word sits at offset 0, tickets from here

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
  if (args == nullptr) return hofa::set_last_error(HOFA_ERR_INVALID_ARGUMENT, "args is NULL");
  int32_t split = 0;
  size_t need = 0;
  int st = hofa::decode_plan(args, &split, &need);  // all argument checks, nothing issued yet
  if (st != HOFA_OK) return st;
  if (need > kNoAllocScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "hofa_decode_fwd_noalloc: this call needs %zu bytes of scratch (B=%lld, H=%lld, D=%lld, split_k=%d) "
             "but the built-in array holds %zu; pass a workspace to hofa_decode_fwd instead",
             need, (long long)args->q.shape[0], (long long)args->q.shape[1], (long long)args->q.shape[3], split,
             kNoAllocScratchBytes);
    return hofa::set_last_error(HOFA_ERR_WORKSPACE, msg);
  }
  void* scratch = nullptr;
  st = scratch_address(&scratch);
  if (st != HOFA_OK) return st;
  const size_t heads = (size_t)args->q.shape[0] * (size_t)args->q.shape[1];
  const size_t ticket_bytes = (heads * sizeof(int) + 255) & ~size_t(255);
  const cudaError_t e = cudaMemsetAsync(static_cast<char*>(scratch) + kTicketOffset, 0, ticket_bytes,
                                        reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return hofa::set_last_error(HOFA_ERR_CUDA, cudaGetErrorString(e));
  hofa_decode_args a = *args;
  a.split_k = split;  // the split the scratch was sized for
  a.workspace = scratch;
  a.workspace_bytes = kNoAllocScratchBytes;
  return hofa_decode_fwd(&a, stream);
}

extern "C" int hofa_decode_noalloc_read_status(void* stream, int32_t* status_out) {
  if (status_out == nullptr) return hofa::set_last_error(HOFA_ERR_INVALID_ARGUMENT, "status_out is NULL");
  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st != HOFA_OK) return st;
  return hofa_decode_read_status(scratch, stream, status_out);
}
