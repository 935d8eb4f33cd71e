// rkv_decode_static: rkv_decode for callers that cannot allocate device memory.
//
// Some callers of this library have no way to provide a device workspace:
// hosts that bind only this C ABI (for example through an FFI from a language
// without a CUDA allocator), or serving stacks that partition all device
// memory in advance and may not allocate once decoding has started.  This
// entry point runs exactly the same kernels as rkv_decode but takes its
// scratch from a fixed array that lives in this library's device image
// instead of a caller-supplied workspace.
//
// Limits and sharing:
// * the array is RKV_DECODE_STATIC_SCRATCH_BYTES (32 MiB) on every GPU that loads the
//   library, held until the process exits; geometries whose rkv_decode
//   workspace would be larger are rejected with RKV_ERR_WORKSPACE;
// * every call on a device shares the one array and it keeps the previous
//   call's contents: calls that may overlap on the GPU (different streams
//   without ordering between them) race and must not be issued;
// * the array's device address is looked up once per device, on the first
//   call made with that device current; make that first call before any
//   stream capture begins.  The address belongs to the CUDA context current
//   at that call: after cudaDeviceReset (or any teardown of the device's
//   primary context) the cached address is stale, so a process that resets
//   a device must not call these entry points on it again;
// * the device status word (timeouts of the kernels' bounded waits, range
//   errors in device-side inputs) lives in the array too; read it with
//   rkv_decode_static_status after the call.
// Nothing here calls cudaMalloc, cudaFree or an allocating library routine.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "refinekv_b200.h"

namespace rkv {
void set_last_error(const std::string& message);  // rkv_capi.cu; read by rkv_last_error()
}

namespace {

constexpr size_t kStaticScratchBytes = RKV_DECODE_STATIC_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the array for the current device (host code cannot use
// the symbol itself: on the host it is only a stand-in).
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) {
    rkv::set_last_error(std::string("cudaGetDevice failed: ") + cudaGetErrorString(err));
    return RKV_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    rkv::set_last_error("device index " + std::to_string(dev) + " is beyond the " +
                        std::to_string(kMaxDevices) + " devices the static array supports");
    return RKV_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (err != cudaSuccess || ptr == nullptr) {
      rkv::set_last_error(std::string("cudaGetSymbolAddress failed: ") +
                          cudaGetErrorString(err));
      return RKV_ERR_CUDA;
    }
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return RKV_OK;
}

}  // namespace

extern "C" {

int rkv_decode_static(const rkv_summary* summary, const void* query, int query_dtype,
                      int64_t group, const void* key_suffix, const void* value_suffix,
                      int64_t suffix_capacity, int64_t key_suffix_head_stride,
                      int64_t key_suffix_token_stride, int64_t value_suffix_head_stride,
                      int64_t value_suffix_token_stride, const int32_t* suffix_length,
                      int64_t suffix_length_host, const uint8_t* anchor_mask, float eps,
                      int reduction, void* output, uint8_t* selected, void* stream) {
  if (summary == nullptr) {
    rkv::set_last_error("summary is null");
    return RKV_ERR_INVALID_ARGUMENT;
  }
  const size_t need = rkv_decode_workspace_size(summary->heads, group, summary->blocks,
                                                summary->head_dim, summary->block_size);
  if (need == 0) return rkv_decode(summary, query, query_dtype, group, key_suffix, value_suffix,
                                   suffix_capacity, key_suffix_head_stride,
                                   key_suffix_token_stride, value_suffix_head_stride,
                                   value_suffix_token_stride, suffix_length, suffix_length_host,
                                   anchor_mask, eps, reduction, output, selected, nullptr, 0,
                                   RKV_PHASE_ALL, stream);  // reports the argument error
  if (need > kStaticScratchBytes) {
    rkv::set_last_error("rkv_decode_static: this geometry needs " + std::to_string(need) +
                        " bytes of scratch, more than the " +
                        std::to_string(kStaticScratchBytes) +
                        "-byte static array; call rkv_decode with a workspace instead");
    return RKV_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != RKV_OK) return rc;
  // Word 0 is the device status; it must start at zero for this call.
  const cudaError_t err = cudaMemsetAsync(scratch, 0, 256, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) {
    rkv::set_last_error(std::string("cudaMemsetAsync failed: ") + cudaGetErrorString(err));
    return RKV_ERR_CUDA;
  }
  return rkv_decode(summary, query, query_dtype, group, key_suffix, value_suffix,
                    suffix_capacity, key_suffix_head_stride, key_suffix_token_stride,
                    value_suffix_head_stride, value_suffix_token_stride, suffix_length,
                    suffix_length_host, anchor_mask, eps, reduction, output, selected, scratch,
                    kStaticScratchBytes, RKV_PHASE_ALL, stream);
}

int rkv_decode_static_status(int32_t* out, void* stream) {
  if (out == nullptr) {
    rkv::set_last_error("out is null");
    return RKV_ERR_INVALID_ARGUMENT;
  }
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != RKV_OK) return rc;
  // Word 0 of the array is the status word of the last rkv_decode_static
  // call on this device; the copy is ordered after that call on `stream`.
  const cudaError_t err = cudaMemcpyAsync(out, scratch, sizeof(int32_t), cudaMemcpyDefault,
                                          static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) {
    rkv::set_last_error(std::string("cudaMemcpyAsync failed: ") + cudaGetErrorString(err));
    return RKV_ERR_CUDA;
  }
  return RKV_OK;
}

}  // extern "C"
