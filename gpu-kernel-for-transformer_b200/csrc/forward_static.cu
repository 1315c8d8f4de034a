// tfx_forward_static: the whole forward without any caller-provided or
// allocated scratch.
//
// Who needs it: callers that are not allowed to allocate device memory --
// plugins loaded into a host runtime whose memory manager owns the whole GPU
// and forbids cudaMalloc from extensions, FFI bindings that can hand the
// library input and output buffers but have no way to pass an extra
// workspace, and latency-critical serving loops that must never allocate
// after start-up. The per-op kernel chain of tfx_forward needs a workspace
// (fp16 LayerNorm output, packed QKV, attention context, fp32 residual stream
// and FFN hidden activations); here that workspace is a fixed device array
// compiled into the library instead.
//
// Limits and caveats:
// * The array is kStaticScratchBytes (32 MiB) of device memory, held on every
//   GPU that loads this library until the process exits. Inputs needing more
//   workspace than that (tfx_forward_workspace_bytes) are rejected with
//   TFX_ERR_WORKSPACE before anything is enqueued.
// * All calls on a device share the one array. Calls whose kernels overlap on
//   the GPU (different streams without ordering, several host threads)
//   corrupt each other's intermediates; serialise them on one stream.
// * Nothing in the array has to start at zero: every byte the kernels read
//   was written earlier in the same forward, so the previous call's leftover
//   contents are harmless.
// * The first call on each device that runs the per-op chain resolves the
//   array's device address (cudaGetSymbolAddress) with that device current;
//   make that first call before any stream capture begins. Calls the fused
//   whole-forward kernel serves need no scratch and skip the lookup.
#include <mutex>

#include "internal.h"

namespace tfx {
namespace {

constexpr size_t kStaticScratchBytes = size_t(32) << 20;

static __device__ __align__(256) unsigned char g_forward_scratch[kStaticScratchBytes];

void* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

// Device address of the scratch array for the current device. Host code must
// not use the symbol itself: on the host it names a stand-in object, not
// device memory.
int scratch_for_current_device(void** out) {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return fail(TFX_ERR_CUDA, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_forward_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(TFX_ERR_CUDA, "tfx_forward_static: cudaGetSymbolAddress failed: %s",
                  cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return TFX_OK;
}

}  // namespace
}  // namespace tfx

using namespace tfx;

extern "C" {

int tfx_forward_static(const tfx_model* model, const float* x, float* y, int batch, int seq,
                       const int32_t* valid_len, tfx_stream_t stream) {
  const int64_t need = tfx_forward_workspace_bytes(model, batch, seq);
  if (need < 0)
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_forward_static: invalid model or sizes");
  if (need > static_cast<int64_t>(kStaticScratchBytes))
    return fail(TFX_ERR_WORKSPACE,
                "tfx_forward_static: batch=%d seq=%d needs %lld bytes of scratch, more than the "
                "library's fixed %zu-byte array; use tfx_forward with a caller workspace",
                batch, seq, static_cast<long long>(need), kStaticScratchBytes);
  // The fused whole-forward kernel keeps every intermediate on chip: no
  // scratch, so no symbol lookup either.
  if (need == 0)
    return tfx_forward(model, x, y, batch, seq, valid_len, nullptr, 0, stream);
  void* scratch = nullptr;
  const int st = scratch_for_current_device(&scratch);
  if (st != TFX_OK) return st;
  return tfx_forward(model, x, y, batch, seq, valid_len, scratch, kStaticScratchBytes, stream);
}

}  // extern "C"
