// Exit head (final RMSNorm + LM head + greedy argmax) that allocates nothing.
//
// Some callers of this library cannot call cudaMalloc: code that runs while a memory pool or
// allocator is locked (a serving runtime that pre-plans every byte and forbids allocation on
// its decode path), code running inside a foreign framework's stream capture, or a plug-in that
// only receives raw input/output pointers.  eesd_head_argmax() needs a model handle and the
// caller-allocated workspace behind it; eesd_head_argmax_static() needs neither: its scratch (the
// normalised rows, the per-row argmax keys and a status word) is a file-scope __device__ array of
// fixed size, so every GPU that loads the library holds it until the process exits.
//
// Limits: bf16 only, n_rows <= kMaxRows (128), dim <= kMaxDim (8192) and a multiple of 64.
// The caller still passes the inputs (hidden states, final-norm weight, LM head) and the output
// (token ids).  All calls share the one array: calls that overlap on the GPU (different streams,
// or different host threads) race on it and must be serialised by the caller.
//
// Errors found on the device (a row index outside x, a bounded wait of the GEMM that gave up) are
// not silent: every id of the call becomes -1 and the call's status bits go to status_out, both
// written on the stream, so the caller reads them with its own synchronisation.
#include <mutex>

#include "common.cuh"
#include "gemm_tc.h"
#include "kernels.h"

namespace eesd {
namespace {

constexpr int kMaxRows = 128;
constexpr int kMaxDim = 8192;
constexpr size_t kStatusOff = 0;                         // int32 status word (256-byte slot)
constexpr size_t kKeysOff = 256;                         // kMaxRows x uint64 argmax keys
constexpr size_t kRowsOff = kKeysOff + kMaxRows * 8;     // kMaxRows x kMaxDim bf16 normalised rows
constexpr size_t kScratchBytes = kRowsOff + (size_t)kMaxRows * kMaxDim * 2;   // 2 MiB + 1280 B

static __device__ __align__(256) unsigned char g_head_scratch[kScratchBytes];

// Host-side device addresses of g_head_scratch, one per device.  In host code the symbol's name
// is only a host stand-in, so the address comes from cudaGetSymbolAddress with that device
// current; it is resolved on a device's first call.
constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_dev[kMaxDevices] = {};

}  // namespace
}  // namespace eesd

using namespace eesd;

extern "C" int eesd_head_argmax_static(const void* x, int x_rows, const int32_t* rows, int n, int dim, int vocab,
                                       const void* norm_w, const void* lm_head, float eps, int32_t* out_ids,
                                       int32_t* status_out, void* stream) {
  if (!x || !norm_w || !lm_head || !out_ids) {
    set_last_error("head_argmax_static: null pointer argument");
    return EESD_ERR_ARG;
  }
  if (x_rows < 1 || (!rows && x_rows < n)) {
    set_last_error("head_argmax_static: x_rows must be >= 1, and >= n without a row list");
    return EESD_ERR_ARG;
  }
  if (n < 1 || n > kMaxRows) {
    set_last_error("head_argmax_static: n must be in [1, 128] (size of the static scratch)");
    return EESD_ERR_ARG;
  }
  if (dim < 64 || dim > kMaxDim || dim % 64) {
    set_last_error("head_argmax_static: dim must be a multiple of 64 in [64, 8192] (static scratch)");
    return EESD_ERR_ARG;
  }
  if (vocab < 1) {
    set_last_error("head_argmax_static: vocab must be >= 1");
    return EESD_ERR_ARG;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_last_error("head_argmax_static: no usable current CUDA device");
    return EESD_ERR_CUDA;
  }
  // the scratch address below belongs to the current device: the stream must be one of its streams
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int stream_dev = -1;
  if (cudaStreamGetDevice(s, &stream_dev) != cudaSuccess || stream_dev != dev) {
    set_last_error("head_argmax_static: the stream does not belong to the current CUDA device");
    return EESD_ERR_ARG;
  }
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_dev[dev]) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_head_scratch);
      if (e != cudaSuccess || !p) {
        set_last_error("head_argmax_static: cudaGetSymbolAddress of the static scratch failed");
        return EESD_ERR_CUDA;
      }
      g_scratch_dev[dev] = p;
    }
    base = g_scratch_dev[dev];
  }
  uint8_t* b = static_cast<uint8_t*>(base);
  int* status = reinterpret_cast<int*>(b + kStatusOff);
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(b + kKeysOff);
  void* xn = b + kRowsOff;
  // the array keeps the previous call's contents: the argmax keys must start at zero
  if (cudaMemsetAsync(keys, 0, (size_t)n * 8, s) != cudaSuccess || cudaMemsetAsync(status, 0, 4, s) != cudaSuccess) {
    set_last_error("head_argmax_static: scratch reset failed");
    return EESD_ERR_CUDA;
  }
  int rc = launch_rmsnorm(EESD_BF16, x, rows, norm_w, xn, n, dim, eps, s, x_rows, status);
  if (rc) {
    set_last_error("head_argmax_static: rmsnorm launch failed");
    return rc;
  }
  CUtensorMap map;
  rc = encode_kmajor_map(&map, lm_head, vocab, dim, 128);
  if (rc) {
    set_last_error("head_argmax_static: LM head tensor map (needs a 16-byte aligned bf16 [vocab, dim])");
    return rc;
  }
  rc = tc_gemm_launch(EESD_EPI_ARGMAX_INTERNAL, map, xn, n, vocab, dim, 0, nullptr, 0, nullptr, 0, keys, status, s, 0,
                      TcScratch{});  // the head is never split: no partial-tile scratch
  if (!rc) rc = launch_keys_to_ids(keys, out_ids, n, s, status, status_out);
  if (rc) set_last_error("head_argmax_static: head GEMM / argmax launch failed");
  return rc;
}
