// Fused LM head for callers that cannot allocate device memory.
//
// b200_lm_head_bf16 needs a caller-provided workspace for its per-CTA argmax
// partials.  Some callers have nowhere to get one: a plugin host that hands
// a kernel only its input and output buffers, or code that is already
// recording a CUDA graph, where cudaMalloc is not allowed.  This entry point
// keeps that workspace in a fixed array in device memory owned by the
// library, so the caller passes only weights, input and outputs.
//
// The array is a file-scope __device__ variable of kScratchBytes (256 KiB);
// every GPU that loads the library holds one copy until the process exits.
// Host code cannot pass the array's name to a kernel (on the host it names a
// stand-in object, not device memory), so the device address is looked up
// with cudaGetSymbolAddress once per device, with that device current, on the
// first call made on that device.
#include <mutex>

#include "b200_linear.h"
#include "kernels.h"

namespace {

constexpr size_t kScratchBytes = 256 * 1024;
constexpr int kMaxPartials = int(kScratchBytes / (sizeof(float) + sizeof(int)));
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_lm_head_scratch[kScratchBytes];

std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of this device's copy of the array (looked up once).
cudaError_t scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_lm_head_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" {

size_t b200_lm_head_noalloc_max_vocab(void) {
  // Every launch shape of the LM head uses at least 8 rows per CTA.
  return size_t(kMaxPartials) * 8;
}

int b200_lm_head_bf16_noalloc(const uint16_t* weight, const uint16_t* bias,
                              const uint16_t* input, uint16_t* logits,
                              int* argmax, int vocab, int in_features,
                              b200_stream_t stream) {
  if (vocab < 0 || in_features < 0 || argmax == nullptr) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  if (size_t(vocab) > b200_lm_head_noalloc_max_vocab()) return B200_ERR_TOO_LARGE;
  if (vocab == 0) {
    cudaError_t e = cudaMemsetAsync(argmax, 0, sizeof(int), stream);
    return e == cudaSuccess ? B200_OK : int(e);
  }
  if (logits == nullptr) return B200_ERR_INVALID_ARGUMENT;
  if (in_features > 0 && (weight == nullptr || input == nullptr)) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  void* scratch = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess) return int(e);
  // Partials: kMaxPartials floats, then kMaxPartials ints.  The first kernel
  // writes every slot the second one reads, so nothing needs clearing.
  float* block_value = static_cast<float*>(scratch);
  int* block_index = reinterpret_cast<int*>(block_value + kMaxPartials);
  const auto* w = reinterpret_cast<const b200::bf16*>(weight);
  const auto* b = reinterpret_cast<const b200::bf16*>(bias);
  const auto* x = reinterpret_cast<const b200::bf16*>(input);
  auto* y = reinterpret_cast<b200::bf16*>(logits);
  // The partials array holds kMaxPartials entries: check the launch's CTA
  // count before anything is enqueued (every launch shape has >= 8 rows per
  // CTA, so the vocab limit above already keeps it within range).
  const int planned = b200::gemv_grid(false, w, nullptr, x, vocab, in_features,
                                      /*lm_head=*/true);
  if (planned > kMaxPartials) return B200_ERR_TOO_LARGE;
  int grid = 0;
  e = b200::launch_gemv(false, w, nullptr, b, x, y, vocab, in_features,
                        block_value, block_index, stream, &grid);
  if (e != cudaSuccess) return int(e);
  e = b200::launch_argmax_partials(block_value, block_index, grid, argmax,
                                   stream);
  return e == cudaSuccess ? B200_OK : int(e);
}

}  // extern "C"
