// paged_decode_noalloc.cu — split-KV paged decode for callers that cannot
// allocate device memory.
//
// b200_paged_decode needs a caller-provided workspace when it splits long
// contexts across CTAs (fp32 partial outputs plus log-sum-exp per split).
// Some hosts cannot hand one over: a serving process that reserved nearly
// all of HBM for its KV pool at start-up and forbids later cudaMalloc calls,
// or a plugin host that owns every device allocation through its own pool
// and exposes no allocator across this C ABI. For them this entry point uses
// a fixed scratch area compiled into the library instead.
//
// The scratch is one file-scope __device__ array of
// B200_NOALLOC_DECODE_SCRATCH_BYTES per device. Every GPU that loads this
// library holds that memory until the process exits. In host code the
// array's name is only a host-side stand-in, never a device address, so the
// address is fetched once per device with cudaGetSymbolAddress (with that
// device current) and passed to the kernels like any workspace. The cached
// address is tied to the CUDA context that was current when it was fetched:
// a host that makes its own driver context on the device, or that reset the
// device (which destroys the primary context), gets the address looked up
// again in its own context.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/b200_paged_attn.h"
#include "paged_decode.cuh"

namespace b200 {
// Sets the message b200_last_error() returns (defined with the ABI in capi.cu).
void set_last_error(const std::string& message);
}  // namespace b200

namespace {

static __device__ __align__(256) unsigned char
    g_decode_scratch[B200_NOALLOC_DECODE_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};

// The driver's cuCtxGetCurrent, reached through the runtime (no link
// dependency on libcuda); null if the driver does not provide it.
PFN_cuCtxGetCurrent_v4000 ctx_get_current_fn() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(ptr);
    }
  });
  return fn;
}

// Device address of this device's scratch array in the current context; set
// up on the first call per device and context (the device is current here).
cudaError_t scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  CUcontext ctx = nullptr;
  PFN_cuCtxGetCurrent_v4000 get_ctx = ctx_get_current_fn();
  if (get_ctx == nullptr || get_ctx(&ctx) != CUDA_SUCCESS) return cudaErrorUnknown;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr || ctx == nullptr || g_scratch_ctx[dev] != ctx) {
    void* ptr = nullptr;
    // binds the device's primary context first if no context is current yet
    e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
    if (e != cudaSuccess) return e;
    if (ctx == nullptr && get_ctx(&ctx) != CUDA_SUCCESS) return cudaErrorUnknown;
    g_scratch_ptr[dev] = ptr;
    g_scratch_ctx[dev] = ctx;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

// Bytes of split-KV partials for this batch: fp32 [seqs, q heads, parts,
// head_dim] then fp32 LSE [seqs, q heads, parts], each rounded up to 256 B
// (the workspace layout b200_paged_decode expects).
int64_t needed_scratch(int64_t num_seqs, int64_t num_q_heads, int64_t num_parts) {
  if (num_parts <= 1) return 0;
  const int64_t slots = num_seqs * num_q_heads * num_parts;
  return (slots * b200::kHeadDim * 4 + 255) / 256 * 256 + (slots * 4 + 255) / 256 * 256;
}

}  // namespace

extern "C" {

int b200_paged_decode_noalloc(const void* q, int64_t q_seq_stride, int64_t q_head_stride,
                              const b200_paged_cache* cache, const int32_t* block_tables,
                              int64_t block_table_stride, const int32_t* seq_lens,
                              int32_t num_seqs, int32_t num_q_heads, void* out,
                              int64_t out_seq_stride, int64_t out_head_stride,
                              float softmax_scale, const b200_decode_plan* plan,
                              int32_t* status, void* stream) {
  if (plan == nullptr || num_seqs < 0 || num_q_heads < 0) {
    // let the regular entry point produce its usual message
    return b200_paged_decode(q, q_seq_stride, q_head_stride, cache, block_tables,
                             block_table_stride, seq_lens, num_seqs, num_q_heads, out,
                             out_seq_stride, out_head_stride, softmax_scale, plan, nullptr,
                             0, status, stream);
  }
  const int64_t need = needed_scratch(num_seqs, num_q_heads, plan->num_parts);
  if (need > (int64_t)B200_NOALLOC_DECODE_SCRATCH_BYTES) {
    b200::set_last_error(
        "b200_paged_decode_noalloc: this batch needs " + std::to_string(need) +
        " bytes of split-KV scratch but the built-in scratch holds " +
        std::to_string((long long)B200_NOALLOC_DECODE_SCRATCH_BYTES) +
        "; use fewer sequences or partitions per call, or b200_paged_decode with a "
        "caller workspace");
    return B200_ERR_INVALID_ARGUMENT;
  }
  void* scratch = nullptr;
  if (need > 0) {
    cudaError_t e = scratch_for_current_device(&scratch);
    if (e != cudaSuccess) {
      b200::set_last_error(
          std::string("b200_paged_decode_noalloc: cudaGetSymbolAddress failed: ") +
          cudaGetErrorString(e));
      return B200_ERR_CUDA;
    }
  }
  // The partial outputs and LSE are written by every contributing CTA before
  // the reduce reads them, so stale contents from an earlier call need no
  // clearing.
  return b200_paged_decode(q, q_seq_stride, q_head_stride, cache, block_tables,
                           block_table_stride, seq_lens, num_seqs, num_q_heads, out,
                           out_seq_stride, out_head_stride, softmax_scale, plan, scratch,
                           need > 0 ? (int64_t)B200_NOALLOC_DECODE_SCRATCH_BYTES : 0, status,
                           stream);
}

}  // extern "C"
