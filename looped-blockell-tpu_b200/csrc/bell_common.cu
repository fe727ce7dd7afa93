// bell_common.cu — host helpers (errors, device info, tensor maps, status
// word, L2 persistence window) and the tile-schedule plan kernel.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "bell_host.h"
#include "bell_ptx.cuh"

namespace bell {

// ------------------------------------------------------------------ errors

static thread_local int g_last_code = 0;
static thread_local char g_last_msg[512] = {0};

int fail(int code, const std::string& msg) {
  g_last_code = code;
  std::snprintf(g_last_msg, sizeof(g_last_msg), "%s", msg.c_str());
  return code;
}

int ok() { return BELL_OK; }

// ------------------------------------------------------------- device info

static constexpr int kMaxDev = 64;
// written once per device (benign repeats), read on every launch
static std::atomic<int> g_sm_count[kMaxDev];
static std::atomic<int> g_cc_major[kMaxDev];
static std::mutex g_mu;

static int cur_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return fail(BELL_ERR_LAUNCH, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (*dev < 0 || *dev >= kMaxDev) return fail(BELL_ERR_ARG, "device ordinal out of range");
  return BELL_OK;
}

int device_sm_count(int* sm_count) {
  int dev;
  if (int rc = cur_device(&dev)) return rc;
  if (g_sm_count[dev] == 0) {
    int sms = 0, major = 0;
    cudaError_t e1 = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaError_t e2 = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e1 != cudaSuccess || e2 != cudaSuccess)
      return fail(BELL_ERR_LAUNCH, "cudaDeviceGetAttribute failed");
    g_cc_major[dev].store(major);
    g_sm_count[dev].store(sms);
  }
  *sm_count = g_sm_count[dev];
  return BELL_OK;
}

int require_sm100() {
  int sms;
  if (int rc = device_sm_count(&sms)) return rc;
  int dev;
  cur_device(&dev);
  if (g_cc_major[dev] != 10)
    return fail(BELL_ERR_ARCH, "libbell_b200 needs an sm_100 (B200) device; compute capability major is " +
                                   std::to_string(g_cc_major[dev]));
  return BELL_OK;
}

// ------------------------------------------------------------ status word

__device__ int32_t g_bell_status_word;

// The address is cached per device ordinal for the life of the process's
// primary context (the runtime API's context); a caller that resets the
// device or binds another context to the ordinal must not reuse this library
// across that change.
int32_t* default_status_ptr() {
  int dev;
  if (cur_device(&dev)) return nullptr;
  static int32_t* ptrs[kMaxDev] = {nullptr};
  std::lock_guard<std::mutex> lk(g_mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_bell_status_word);
    if (e != cudaSuccess) {
      fail(BELL_ERR_LAUNCH, std::string("cudaGetSymbolAddress(status): ") + cudaGetErrorString(e));
      return nullptr;
    }
    ptrs[dev] = static_cast<int32_t*>(p);
  }
  return ptrs[dev];
}

uint64_t wait_budget_ns() {
  static uint64_t v = [] {
    const char* s = std::getenv("BELL_WAIT_BUDGET_MS");
    uint64_t ms = s ? std::strtoull(s, nullptr, 10) : 2000ull;
    if (ms == 0) ms = 2000ull;
    return ms * 1000000ull;
  }();
  return v;
}

// ------------------------------------------------------------- tensor maps

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess) return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

int make_map_2d(CUtensorMap* map, const void* base, MapType type, uint64_t inner, uint64_t outer,
                uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer, Swz swz, bool l2_256) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(BELL_ERR_LAUNCH, "cuTensorMapEncodeTiled entry point not available");
  if (!aligned16(base)) return fail(BELL_ERR_ALIGN, "tensor base address is not 16-byte aligned");
  if (pitch_bytes % 16 != 0) return fail(BELL_ERR_ALIGN, "row pitch is not a multiple of 16 bytes");
  CUtensorMapDataType dt = type == MapType::BF16   ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                           : type == MapType::INT8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMapSwizzle sw = swz == Swz::B128  ? CU_TENSOR_MAP_SWIZZLE_128B
                          : swz == Swz::B64 ? CU_TENSOR_MAP_SWIZZLE_64B
                          : swz == Swz::B32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                            : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  l2_256 ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B : CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(BELL_ERR_LAUNCH, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(int(r)));
  return BELL_OK;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(BELL_ERR_LAUNCH, std::string(what) + ": " + cudaGetErrorString(e));
  return BELL_OK;
}

int set_smem(const void* func, int bytes) {
  cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess)
    return fail(BELL_ERR_LAUNCH, std::string("cudaFuncSetAttribute(smem): ") + cudaGetErrorString(e));
  return BELL_OK;
}

// -------------------------------------------------------------------- plan
//
// Plan entry (uint32): bits [0,16) column block, [16,24) slot in the first
// matrix (gate, or the single weight of a linear), [24,32) slot in the up
// matrix; 255 = absent.  Count word: bits [0,16) steps, bit 16 "gate has a
// live tile", bit 17 "up has a live tile".
//
// Gate/up rows are merged: a gate slot and an up slot naming the same column
// block share one step (one activation tile feeds both MMAs); unmatched
// slots become gate-only / up-only steps.  Dead slots (-1) are dropped; any
// other index outside [0, C) sets BELL_STATUS_COLIDX and is dropped.

static size_t a16(size_t v) { return (v + 15) & ~size_t(15); }

PlanLayout plan_layout(int32_t R_gu, int32_t K_g, int32_t K_u, int32_t R_d, int32_t K_d) {
  PlanLayout L;
  size_t off = 0;
  L.gu_entries = off;
  off += a16(size_t(R_gu) * size_t(K_g + K_u) * 4);
  L.gu_counts = off;
  off += a16(size_t(R_gu) * 4);
  L.d_entries = off;
  off += a16(size_t(R_d) * size_t(K_d) * 4);
  L.d_counts = off;
  off += a16(size_t(R_d) * 4);
  L.total = off < 16 ? 16 : off;
  return L;
}

struct PlanArgs {
  const int32_t* ci_g;
  const int32_t* ci_u;
  const int32_t* ci_d;
  int32_t K_g, K_u, R_gu, C_gu, K_d, R_d, C_d;
  uint32_t* gu_entries;
  int32_t* gu_counts;
  uint32_t* d_entries;
  int32_t* d_counts;
  int32_t* status;
  int32_t merge;  // 1: share a step between a gate slot and an up slot on the same column
};

__global__ void __launch_bounds__(128) bell_plan_kernel(PlanArgs a) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < a.R_gu) {
    const int32_t* cg = a.ci_g + size_t(r) * a.K_g;
    const int32_t* cu = a.ci_u + size_t(r) * a.K_u;
    uint32_t* out = a.gu_entries + size_t(r) * (a.K_g + a.K_u);
    uint32_t used[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    uint32_t gmatched[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int n = 0, gany = 0, uany = 0, bad = 0;
    for (int k = 0; k < a.K_g; ++k) {
      const int c = cg[k];
      if (c == -1) continue;
      if (c < -1 || c >= a.C_gu) {
        bad = 1;
        continue;
      }
      for (int j = 0; j < a.K_u && a.merge; ++j) {
        if ((used[j >> 5] >> (j & 31)) & 1u) continue;
        if (cu[j] == c) {  // shared step: listed first (the 2-SM kernel relies on that order)
          used[j >> 5] |= 1u << (j & 31);
          gmatched[k >> 5] |= 1u << (k & 31);
          out[n++] = uint32_t(c) | (uint32_t(k) << 16) | (uint32_t(j) << 24);
          gany = uany = 1;
          break;
        }
      }
    }
    for (int k = 0; k < a.K_g; ++k) {  // gate slots without an up partner, ascending
      const int c = cg[k];
      if (c < 0 || c >= a.C_gu || ((gmatched[k >> 5] >> (k & 31)) & 1u)) continue;
      out[n++] = uint32_t(c) | (uint32_t(k) << 16) | (255u << 24);
      gany = 1;
    }
    for (int j = 0; j < a.K_u; ++j) {
      if ((used[j >> 5] >> (j & 31)) & 1u) continue;
      const int c = cu[j];
      if (c == -1) continue;
      if (c < -1 || c >= a.C_gu) {
        bad = 1;
        continue;
      }
      out[n++] = uint32_t(c) | (255u << 16) | (uint32_t(j) << 24);
      uany = 1;
    }
    a.gu_counts[r] = n | (gany << 16) | (uany << 17);
    if (bad) atomicOr(a.status, BELL_STATUS_COLIDX);
  } else if (r < a.R_gu + a.R_d) {
    const int rd = r - a.R_gu;
    const int32_t* cd = a.ci_d + size_t(rd) * a.K_d;
    uint32_t* out = a.d_entries + size_t(rd) * a.K_d;
    int n = 0, bad = 0;
    for (int k = 0; k < a.K_d; ++k) {
      const int c = cd[k];
      if (c == -1) continue;
      if (c < -1 || c >= a.C_d) {
        bad = 1;
        continue;
      }
      out[n++] = uint32_t(c) | (uint32_t(k) << 16) | (255u << 24);
    }
    a.d_counts[rd] = n | ((n > 0 ? 1 : 0) << 16);
    if (bad) atomicOr(a.status, BELL_STATUS_COLIDX);
  }
}

int launch_plan(const int32_t* ci_g, int32_t K_g, const int32_t* ci_u, int32_t K_u, int32_t R_gu, int32_t C_gu,
                const int32_t* ci_d, int32_t K_d, int32_t R_d, int32_t C_d, void* plan, int32_t* status,
                cudaStream_t stream) {
  return launch_plan_ex(ci_g, K_g, ci_u, K_u, R_gu, C_gu, ci_d, K_d, R_d, C_d, plan, status, stream, 1);
}

int launch_plan_ex(const int32_t* ci_g, int32_t K_g, const int32_t* ci_u, int32_t K_u, int32_t R_gu, int32_t C_gu,
                   const int32_t* ci_d, int32_t K_d, int32_t R_d, int32_t C_d, void* plan, int32_t* status,
                   cudaStream_t stream, int32_t merge) {
  PlanLayout L = plan_layout(R_gu, K_g, K_u, R_d, K_d);
  PlanArgs a;
  a.merge = merge;
  a.ci_g = ci_g;
  a.ci_u = ci_u;
  a.ci_d = ci_d;
  a.K_g = K_g;
  a.K_u = K_u;
  a.R_gu = R_gu;
  a.C_gu = C_gu;
  a.K_d = K_d;
  a.R_d = R_d;
  a.C_d = C_d;
  char* base = static_cast<char*>(plan);
  a.gu_entries = reinterpret_cast<uint32_t*>(base + L.gu_entries);
  a.gu_counts = reinterpret_cast<int32_t*>(base + L.gu_counts);
  a.d_entries = reinterpret_cast<uint32_t*>(base + L.d_entries);
  a.d_counts = reinterpret_cast<int32_t*>(base + L.d_counts);
  a.status = status;
  const int rows = R_gu + R_d;
  if (rows == 0) return BELL_OK;
  bell_plan_kernel<<<(rows + 127) / 128, 128, 0, stream>>>(a);
  return check_launch("bell_plan_kernel");
}

}  // namespace bell

// ---------------------------------------------------------------- C ABI

extern "C" {

int bell_abi_version(void) { return BELL_ABI_VERSION; }

int bell_last_error(char* buf, size_t len) {
  if (buf && len) {
    std::snprintf(buf, len, "%s", bell::g_last_msg);
  }
  return bell::g_last_code;
}

size_t bell_plan_bytes(int32_t R_gu, int32_t K_gate, int32_t K_up, int32_t R_down, int32_t K_down) {
  return bell::plan_layout(R_gu, K_gate, K_up, R_down, K_down).total;
}

int bell_read_status(int32_t* value, int32_t clear, void* stream) {
  if (!value) return bell::fail(BELL_ERR_ARG, "bell_read_status: value is NULL");
  int32_t* p = bell::default_status_ptr();
  if (!p) return BELL_ERR_LAUNCH;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(value, p, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(p, 0, sizeof(int32_t), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return bell::fail(BELL_ERR_LAUNCH, std::string("bell_read_status: ") + cudaGetErrorString(e));
  return BELL_OK;
}

int bell_device_info(int32_t* sm_count, int32_t* is_sm100) {
  int sms = 0;
  if (int rc = bell::device_sm_count(&sms)) return rc;
  if (sm_count) *sm_count = sms;
  if (is_sm100) *is_sm100 = (bell::require_sm100() == BELL_OK) ? 1 : 0;
  return BELL_OK;
}

// Persisting-L2 window (reference csrc/loop/l2_policy.cu:48-155).  The
// persisting carve-out is a limit of this process's context only; it ends
// with the context and changes no device setting.
int bell_pin_l2(const void* base, size_t bytes, void* stream) {
  if (!base || bytes == 0) return bell::fail(BELL_ERR_ARG, "bell_pin_l2: empty window");
  int dev;
  if (cudaGetDevice(&dev) != cudaSuccess) return bell::fail(BELL_ERR_LAUNCH, "cudaGetDevice");
  int max_persist = 0, max_window = 0;
  cudaDeviceGetAttribute(&max_persist, cudaDevAttrMaxPersistingL2CacheSize, dev);
  cudaDeviceGetAttribute(&max_window, cudaDevAttrMaxAccessPolicyWindowSize, dev);
  size_t reserve = bytes < size_t(max_persist) ? bytes : size_t(max_persist);
  size_t window = bytes < size_t(max_window) ? bytes : size_t(max_window);
  cudaError_t e = cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, reserve);
  if (e != cudaSuccess) return bell::fail(BELL_ERR_LAUNCH, std::string("persisting L2 limit: ") + cudaGetErrorString(e));
  cudaStreamAttrValue attr;
  std::memset(&attr, 0, sizeof(attr));
  attr.accessPolicyWindow.base_ptr = const_cast<void*>(base);
  attr.accessPolicyWindow.num_bytes = window;
  attr.accessPolicyWindow.hitRatio = window > 0 ? float(double(reserve) / double(window) < 1.0 ? double(reserve) / double(window) : 1.0) : 0.f;
  attr.accessPolicyWindow.hitProp = cudaAccessPropertyPersisting;
  attr.accessPolicyWindow.missProp = cudaAccessPropertyStreaming;
  e = cudaStreamSetAttribute(static_cast<cudaStream_t>(stream), cudaStreamAttributeAccessPolicyWindow, &attr);
  if (e != cudaSuccess) return bell::fail(BELL_ERR_LAUNCH, std::string("access policy window: ") + cudaGetErrorString(e));
  return BELL_OK;
}

int bell_unpin_l2(void* stream) {
  cudaStreamAttrValue attr;
  std::memset(&attr, 0, sizeof(attr));
  attr.accessPolicyWindow.num_bytes = 0;
  attr.accessPolicyWindow.hitRatio = 0.f;
  attr.accessPolicyWindow.hitProp = cudaAccessPropertyNormal;
  attr.accessPolicyWindow.missProp = cudaAccessPropertyNormal;
  cudaError_t e =
      cudaStreamSetAttribute(static_cast<cudaStream_t>(stream), cudaStreamAttributeAccessPolicyWindow, &attr);
  if (e == cudaSuccess) e = cudaCtxResetPersistingL2Cache();
  if (e == cudaSuccess) e = cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, 0);
  if (e != cudaSuccess) return bell::fail(BELL_ERR_LAUNCH, std::string("bell_unpin_l2: ") + cudaGetErrorString(e));
  return BELL_OK;
}

}  // extern "C"
