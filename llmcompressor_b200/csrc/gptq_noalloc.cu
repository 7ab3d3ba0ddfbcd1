// GPTQ block loop for callers that cannot allocate device memory.
//
// llmc_gptq_quantize needs a scratch workspace (a float32 copy of the
// weight, the current block's errors and per-row losses) that its caller
// allocates.  Some callers cannot do that: code running while a CUDA stream
// is being captured (cudaMalloc is not allowed there and would synchronise
// the device), runtimes embedding this library that own all device memory
// through their own pool and give it no allocator, or thin FFI bindings
// with no device allocator at hand.  For them, llmc_gptq_quantize_noalloc
// runs the same kernels with the scratch taken from a fixed array compiled
// into the library.
//
// The array is a file-scope __device__ variable of LLMC_GPTQ_NOALLOC_SCRATCH_BYTES
// (32 MiB).  Every GPU on which the library's device code is loaded holds
// those 32 MiB until the process exits.  In host code its name is only a
// host-side stand-in, never a device address, so the entry point asks the
// runtime for the device address (cudaGetSymbolAddress), with that device
// current, on every call made outside stream capture, and passes that
// address on as the workspace.
#include "llmc_common.cuh"

#include <mutex>

namespace {

constexpr int64_t kScratchBytes = LLMC_GPTQ_NOALLOC_SCRATCH_BYTES;
static_assert(kScratchBytes == (int64_t)32 << 20, "header and definition disagree");

static __device__ __align__(256) unsigned char g_gptq_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_dev[kMaxDevices] = {};

// Device address of g_gptq_scratch on the current device.  Outside stream
// capture it is looked up on every call (cheap), so the address stays right
// after a device reset reloads the module; during capture the address cached
// by the last call outside capture is used.
int scratch_address(cudaStream_t st, void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return LLMC_ECUDA;
  if (dev < 0 || dev >= kMaxDevices) return LLMC_ENOSUPPORT;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) return LLMC_ECUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  if (cap == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_gptq_scratch) != cudaSuccess || p == nullptr) return LLMC_ECUDA;
    g_scratch_dev[dev] = p;
  } else if (!g_scratch_dev[dev]) {
    return LLMC_EINVAL_ARG;  // first call on this device during capture: no address known yet
  }
  *out = g_scratch_dev[dev];
  return LLMC_OK;
}

}  // namespace

extern "C" int llmc_gptq_quantize_noalloc(const void* w_bf16, int64_t rows, int64_t cols, const float* Hinv,
                                          const float* HinvT, const uint8_t* dead, const LlmcQuantArgs* args, const void* scale_bf16,
                                          const int8_t* zp, int64_t blocksize, void* wq_bf16, float* loss,
                                          int* status, void* stream) {
  int64_t need = 0;
  int s = llmc_gptq_quantize_workspace_size(rows, cols, &need);
  if (s != LLMC_OK) return s;
  if (need > kScratchBytes) return LLMC_EINVAL_SHAPE;  // the weight does not fit the fixed scratch
  void* ws = nullptr;
  if ((s = scratch_address((cudaStream_t)stream, &ws)) != LLMC_OK) return s;
  // The workspace contents left by an earlier call are never read: the
  // float32 weight copy and the block errors are written before use, and
  // llmc_gptq_quantize zeroes the per-row losses itself.
  return llmc_gptq_quantize(w_bf16, rows, cols, Hinv, HinvT, dead, args, scale_bf16, zp, blocksize, wq_bf16, loss, ws,
                            status, stream);
}
