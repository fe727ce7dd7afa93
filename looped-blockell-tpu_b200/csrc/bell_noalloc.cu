// bell_noalloc.cu — a bf16 SwiGLU forward for callers that cannot allocate
// device memory.
//
// bell_swiglu_fwd_bf16 needs two scratch buffers besides its inputs and
// outputs: the tile-schedule plan and the intermediate h = silu(x Wg) * (x Wu)
// ([T, d_ff] bf16).  Normally the caller allocates both.  Some callers
// cannot: a host that hands this library only the tensors of the layer (an
// FFI binding from a runtime with its own memory manager, or a serving process
// whose device memory is carved up once at start-up and must not grow
// afterwards).  bell_swiglu_fwd_bf16_noalloc serves them from a fixed scratch
// array compiled into this library, so the call performs no allocation at
// all.
//
// The array is a file-scope __device__ variable: every GPU that loads the
// library reserves BELL_NOALLOC_SCRATCH_BYTES (32 MiB) for it until the
// process exits.  In host code the array's name is only a host-side stand-in,
// never a device address, so its device address is looked up with
// cudaGetSymbolAddress, once per device, on that device's first call (make
// that first call before starting any stream capture).  The address stays
// cached for the life of the process's primary context on that device, so
// the library must not be used across a cudaDeviceReset.  All calls on a device
// share the one array: calls that overlap on the GPU (on different streams,
// without ordering between them) race on it.  The array keeps the last call's
// contents; nothing needs clearing because each call writes every byte of the
// plan and of h that it later reads.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "bell_host.h"

namespace bell {

static __device__ __align__(256) uint8_t g_noalloc_scratch[BELL_NOALLOC_SCRATCH_BYTES];

static constexpr int kMaxDevices = 64;
static void* g_scratch_ptr[kMaxDevices] = {nullptr};
static std::mutex g_scratch_mu;

// Device address of the scratch array on the current device (looked up once
// per device, with that device current).
static int scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(BELL_ERR_LAUNCH, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(BELL_ERR_ARG, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(BELL_ERR_LAUNCH, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return BELL_OK;
}

static size_t up256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace bell

using namespace bell;

// 0 for sizes no forward accepts (negative T or d_ff, or a block-row or slot
// count below 1), so a caller can use it to ask whether a call fits.
extern "C" size_t bell_noalloc_scratch_bytes(int64_t T, int32_t d_ff, int32_t R_gu, int32_t K_gate, int32_t K_up,
                                             int32_t R_down, int32_t K_down) {
  if (T < 0 || d_ff < 0 || R_gu < 1 || K_gate < 1 || K_up < 1 || R_down < 1 || K_down < 1) return 0;
  return up256(plan_layout(R_gu, K_gate, K_up, R_down, K_down).total) + up256(size_t(T) * size_t(d_ff) * 2);
}

extern "C" int bell_swiglu_fwd_bf16_noalloc(const BellFFNDesc* desc, void* stream) {
  if (!desc) return fail(BELL_ERR_ARG, "descriptor is NULL");
  if (desc->h || desc->plan)
    return fail(BELL_ERR_ARG, "bell_swiglu_fwd_bf16_noalloc: h and plan must be NULL (they come from the static scratch)");
  {
    // validate the whole descriptor first (stand-in h / plan addresses), so a
    // wrong shape is reported as itself, not as a scratch-size problem
    BellFFNDesc probe = *desc;
    probe.h = probe.plan = reinterpret_cast<void*>(uintptr_t(256));
    if (int rc = check_ffn(&probe, BELL_DTYPE_BF16)) return rc;
  }
  const size_t plan_b = up256(plan_layout(desc->gate.R, desc->gate.K, desc->up.K, desc->down.R, desc->down.K).total);
  const size_t need = plan_b + up256(size_t(desc->T) * size_t(desc->d_ff) * 2);
  if (need > size_t(BELL_NOALLOC_SCRATCH_BYTES))
    return fail(BELL_ERR_SHAPE, "bell_swiglu_fwd_bf16_noalloc: needs " + std::to_string(need) +
                                    " bytes of scratch (plan + T*d_ff bf16) but the static scratch holds " +
                                    std::to_string(size_t(BELL_NOALLOC_SCRATCH_BYTES)) +
                                    "; use bell_swiglu_fwd_bf16 with caller-owned buffers");
  void* base = nullptr;
  if (int rc = scratch_address(&base)) return rc;
  BellFFNDesc d = *desc;
  d.plan = base;
  d.h = static_cast<uint8_t*>(base) + plan_b;
  return bell_swiglu_fwd_bf16(&d, stream);
}
