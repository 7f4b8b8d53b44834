// noalloc.cu — hexmoe_forward_noalloc: the layer forward for callers that can
// hand the library no device memory of their own.
//
// hexmoe_forward takes its scratch (routing plan, gathered activations, the
// SwiGLU activation, per-slot outputs) from a caller buffer.  Some callers have
// none to give and may not make one: a serving process whose memory pool has
// already reserved nearly all of the GPU (a cudaMalloc there fails, or takes
// memory the pool has promised elsewhere), a plugin host that owns every device
// allocation and hands a custom operator only its inputs and outputs, or a
// latency-bound loop where cudaMalloc / cudaFree would synchronise the device.
// For them this file keeps one fixed scratch array in the library itself, a
// file-scope __device__ array of kNoAllocScratchBytes (32 MiB) that every GPU
// which loads the library holds until the process exits, and runs the same
// forward over it.
//
// Rules that follow from the array being shared:
//   * The first call on a device looks the array's device address up (with
//     that device current) and caches it; make that first call before any
//     stream capture begins on the device.
//   * Every call on a device uses the same array, and it keeps whatever the
//     last call left there.  Calls whose kernels overlap on the GPU (two
//     streams, or two host threads, without ordering between them) race on it
//     and produce wrong results: order them on one stream or with events.
//   * Nothing in the array has to start at zero: every scratch word a forward
//     reads (plan, gathered rows, activations, per-slot outputs) is written
//     earlier in the same call, and padding rows are never stored to `out`.
//   * A call whose scratch need (hexmoe_forward_workspace_bytes) exceeds the
//     array returns HEXMOE_E_ARG with the sizes in the message.
// Nothing here calls cudaMalloc, cudaFree or any other allocating routine.
#include <cstdio>
#include <mutex>

#include "internal.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = HEXMOE_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// In host code `g_noalloc_scratch` only names the symbol; its device address
// comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of this device's scratch array (the current device's).
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return hexmoe::report_cuda_error(e, "hexmoe_forward_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return hexmoe::report_error(HEXMOE_E_DEVICE, "hexmoe_forward_noalloc: device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return hexmoe::report_cuda_error(e, "hexmoe_forward_noalloc: cudaGetSymbolAddress");
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return HEXMOE_OK;
}

}  // namespace

extern "C" HEXMOE_API int hexmoe_forward_noalloc(const hexmoe_layer* layer, const void* x, int32_t x_dtype,
                                                 int64_t tokens, int32_t topk, const float* topk_weights,
                                                 const void* topk_ids, int32_t ids_dtype, void* out,
                                                 int32_t out_dtype, int32_t block_m, void* stream) {
  if (!layer) return hexmoe::report_error(HEXMOE_E_ARG, "hexmoe_forward_noalloc: null layer");
  if (tokens < 0 || topk <= 0) return hexmoe::report_error(HEXMOE_E_ARG, "hexmoe_forward_noalloc: bad tokens / topk");
  const size_t need = hexmoe_forward_workspace_bytes(layer, tokens, topk, block_m, x_dtype);
  if (need > kNoAllocScratchBytes) {
    char msg[320];
    snprintf(msg, sizeof(msg),
             "hexmoe_forward_noalloc: %lld tokens x top-%d need %zu scratch bytes, more than the fixed %zu; "
             "use hexmoe_forward with a caller workspace",
             static_cast<long long>(tokens), topk, need, kNoAllocScratchBytes);
    return hexmoe::report_error(HEXMOE_E_ARG, msg);
  }
  void* scratch = nullptr;
  if (int rc = scratch_for_current_device(&scratch)) return rc;
  return hexmoe_forward(layer, x, x_dtype, tokens, topk, topk_weights, topk_ids, ids_dtype, out, out_dtype, block_m,
                        scratch, kNoAllocScratchBytes, stream);
}
