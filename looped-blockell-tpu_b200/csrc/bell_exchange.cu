// bell_exchange.cu — the owner-side sum of the d_ff-sharded forward.
//
// In the sharded forward every rank computes a partial [Tc, d_model] output
// for all tokens of a chunk (its d_ff shard's contribution) and the rows of
// the chunk are owned 1/N per rank.  With the copy-engine exchange each rank
// copies the owner's rows of its partial into that owner's inbox (one
// cudaMemcpyAsync per peer, no SMs), and the owner adds the N slices and the
// residual here:
//   out[r, c] = bf16( ((v_0 + v_1) + ... + v_{N-1}) + residual[r, c] )
// in fp32, in ascending rank order, rounded once: the same value whatever
// the order in which the slices arrived, unlike a ring reduction.  Slice
// `local_slot` is read from the rank's own partial (no copy of it is made).
//
// HBM-bound: N + 1 reads and one write per element, 16-byte accesses, a
// grid-stride loop over rows so the launch can be capped to the SMs the GEMM
// grids leave free.
//
// The inboxes are shared between the ranks' processes with CUDA IPC: each
// rank maps every peer's inbox into its own device's context (bell_ipc_open),
// so that its copies into a peer's inbox go device to device over NVLink.
#include <algorithm>
#include <cstring>
#include <string>

#include "bell_host.h"
#include "bell_ptx.cuh"

namespace bell {
namespace xchg {

static constexpr int kThr = 512;
static constexpr int kMaxSlices = 64;

struct SumArgs {
  const __nv_bfloat16* slices;  // slice s, row r at slices + s * slice_stride + r * ld_slice
  int64_t slice_stride, ld_slice;
  int32_t n, local_slot;
  const __nv_bfloat16* local;  // slice local_slot, row r at local + r * ld_local
  int64_t ld_local;
  const __nv_bfloat16* residual;  // optional, row r at residual + r * ld_res
  int64_t ld_res;
  __nv_bfloat16* out;
  int64_t ld_out;
  int64_t rows;
  int32_t groups;  // d / 8
};

__device__ __forceinline__ void add8(float (&acc)[8], const uint4& v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16x2(w[i]);
    acc[2 * i] = __fadd_rn(acc[2 * i], f.x);
    acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], f.y);
  }
}

// CTA b sums rows b, b + gridDim, ...: its threads cover the row's 8-column
// groups, and each thread takes kItems rows gridDim apart at once, with every
// slice's loads of those rows issued together, so enough bytes are in flight
// to run a capped grid near its share of HBM.  No integer division.
static constexpr int kItems = 2;
static constexpr int kBatch = 7;

__device__ __forceinline__ const __nv_bfloat16* slice_row(const SumArgs& a, int s, int64_t r) {
  return s == a.local_slot ? a.local + r * a.ld_local : a.slices + s * a.slice_stride + r * a.ld_slice;
}

__global__ void __launch_bounds__(kThr, 1) bell_sum_slices_kernel(const SumArgs a) {
  const int64_t G = gridDim.x;
  for (int64_t r0 = blockIdx.x; r0 < a.rows; r0 += G * kItems) {
    for (int g = threadIdx.x; g < a.groups; g += blockDim.x) {
      const int64_t c = int64_t(g) * 8;
      bool in[kItems];
#pragma unroll
      for (int k = 0; k < kItems; ++k) in[k] = r0 + k * G < a.rows;
      float acc[kItems][8];
#pragma unroll
      for (int k = 0; k < kItems; ++k) {  // the first value as is: no 0 + v (that would turn -0 into +0)
        const uint4 v =
            in[k] ? __ldg(reinterpret_cast<const uint4*>(slice_row(a, 0, r0 + k * G) + c)) : make_uint4(0, 0, 0, 0);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = unpack_bf16x2(w[i]);
          acc[k][2 * i] = f.x;
          acc[k][2 * i + 1] = f.y;
        }
      }
      int s = 1;
      for (; s + kBatch <= a.n; s += kBatch) {  // kBatch slices' loads in flight at once, added in order
        uint4 v[kBatch][kItems];
#pragma unroll
        for (int q = 0; q < kBatch; ++q)
#pragma unroll
          for (int k = 0; k < kItems; ++k)
            v[q][k] = in[k] ? __ldg(reinterpret_cast<const uint4*>(slice_row(a, s + q, r0 + k * G) + c))
                            : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int q = 0; q < kBatch; ++q)
#pragma unroll
          for (int k = 0; k < kItems; ++k) add8(acc[k], v[q][k]);
      }
      for (; s < a.n; ++s) {
        uint4 v[kItems];
#pragma unroll
        for (int k = 0; k < kItems; ++k)
          v[k] = in[k] ? __ldg(reinterpret_cast<const uint4*>(slice_row(a, s, r0 + k * G) + c)) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int k = 0; k < kItems; ++k) add8(acc[k], v[k]);
      }
      if (a.residual) {
        uint4 v[kItems];
#pragma unroll
        for (int k = 0; k < kItems; ++k)
          v[k] = in[k] ? __ldg(reinterpret_cast<const uint4*>(a.residual + (r0 + k * G) * a.ld_res + c))
                       : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int k = 0; k < kItems; ++k) add8(acc[k], v[k]);
      }
#pragma unroll
      for (int k = 0; k < kItems; ++k) {
        if (!in[k]) continue;
        uint4 o;
        o.x = pack_bf16x2(acc[k][0], acc[k][1]);
        o.y = pack_bf16x2(acc[k][2], acc[k][3]);
        o.z = pack_bf16x2(acc[k][4], acc[k][5]);
        o.w = pack_bf16x2(acc[k][6], acc[k][7]);
        *reinterpret_cast<uint4*>(a.out + (r0 + k * G) * a.ld_out + c) = o;
      }
    }
  }
}

}  // namespace xchg
}  // namespace bell

using namespace bell;
using namespace bell::xchg;

extern "C" int bell_sum_slices_bf16(const void* slices, int64_t slice_stride, int64_t ld_slice, int32_t n_slices,
                                    int32_t local_slot, const void* local, int64_t ld_local, const void* residual,
                                    int64_t ld_res, void* out, int64_t ld_out, int64_t rows, int32_t d,
                                    int32_t max_ctas, void* stream) {
  if (n_slices < 1 || n_slices > kMaxSlices) return fail(BELL_ERR_SHAPE, "n_slices must be in [1, 64]");
  if (rows < 0 || d < 0 || d % 8) return fail(BELL_ERR_SHAPE, "rows >= 0 and d a multiple of 8 required");
  if (local_slot < -1 || local_slot >= n_slices) return fail(BELL_ERR_ARG, "local_slot must be -1 or a slice index");
  if (rows == 0 || d == 0) return BELL_OK;
  const bool need_slices = !(n_slices == 1 && local_slot == 0);
  if (!out || (need_slices && !slices) || (local_slot >= 0 && !local))
    return fail(BELL_ERR_ARG, "out, slices and (with local_slot >= 0) local must be non-NULL");
  if ((need_slices && !aligned16(slices)) || (local && !aligned16(local)) || (residual && !aligned16(residual)) ||
      !aligned16(out) || slice_stride % 8 || ld_slice % 8 || ld_local % 8 || ld_res % 8 || ld_out % 8)
    return fail(BELL_ERR_ALIGN, "pointers must be 16-byte aligned and strides multiples of 8 elements");
  if (ld_out < d || (need_slices && ld_slice < d) || (local && ld_local < d) || (residual && ld_res < d))
    return fail(BELL_ERR_SHAPE, "row strides must be >= d");
  SumArgs a{};
  a.slices = static_cast<const __nv_bfloat16*>(slices);
  a.slice_stride = slice_stride;
  a.ld_slice = ld_slice;
  a.n = n_slices;
  a.local_slot = local_slot;
  a.local = static_cast<const __nv_bfloat16*>(local);
  a.ld_local = ld_local;
  a.residual = static_cast<const __nv_bfloat16*>(residual);
  a.ld_res = ld_res;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ld_out = ld_out;
  a.rows = rows;
  a.groups = d / 8;
  int sms = 0;
  if (int rc = device_sm_count(&sms)) return rc;
  int threads = (a.groups + 31) / 32 * 32;  // one thread per 8-column group, up to kThr
  if (threads > kThr) threads = kThr;
  const int64_t cap = max_ctas > 0 ? max_ctas : 2 * int64_t(sms);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
static constexpr int kItems = 2;
static constexpr int kBatch = 7;
  int64_t grid = (rows + kItems - 1) / kItems;
  if (grid > cap) grid = cap;
  bell_sum_slices_kernel<<<unsigned(grid), unsigned(threads), 0, st>>>(a);
  return check_launch("bell_sum_slices_kernel");
}

// One asynchronous copy of `bytes` between any two device addresses of the
// unified address space (a peer's memory mapped into this process included:
// the copy engines move it over NVLink, no SMs involved), stream-ordered.
extern "C" int bell_memcpy_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return BELL_OK;
  if (!dst || !src) return fail(BELL_ERR_ARG, "bell_memcpy_async: NULL pointer");
  const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(BELL_ERR_LAUNCH, std::string("cudaMemcpyAsync: ") + cudaGetErrorString(e));
  return BELL_OK;
}

// Let the current device reach `peer`'s memory directly (NVLink): without it
// a copy between the two is staged through host memory.  Already enabled is
// success.
extern "C" int bell_enable_peer_access(int32_t peer) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(BELL_ERR_LAUNCH, "cudaGetDevice failed");
  if (peer == dev) return BELL_OK;
  int can = 0;
  if (cudaDeviceCanAccessPeer(&can, dev, peer) != cudaSuccess || !can)
    return fail(BELL_ERR_ARCH, "device " + std::to_string(dev) + " cannot access device " + std::to_string(peer));
  const cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();  // reset the last-error state this call left
    return BELL_OK;
  }
  if (e != cudaSuccess) return fail(BELL_ERR_LAUNCH, std::string("cudaDeviceEnablePeerAccess: ") + cudaGetErrorString(e));
  return BELL_OK;
}

// --------------------------------------------------------------- CUDA IPC

typedef CUresult (*AddrRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

// Handle of the allocation holding `ptr` (64 bytes into handle_out) and the
// offset of `ptr` in it.
extern "C" int bell_ipc_handle(const void* ptr, void* handle_out, uint64_t* offset_out) {
  if (!ptr || !handle_out || !offset_out) return fail(BELL_ERR_ARG, "bell_ipc_handle: NULL pointer");
  static AddrRangeFn range = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    const cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess) return static_cast<AddrRangeFn>(nullptr);
    return reinterpret_cast<AddrRangeFn>(p);
  }();
  if (!range) return fail(BELL_ERR_LAUNCH, "cuMemGetAddressRange entry point not available");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return fail(BELL_ERR_ARG, "cuMemGetAddressRange failed: not device memory?");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return fail(BELL_ERR_LAUNCH, std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = uint64_t(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return BELL_OK;
}

// Map another process's allocation (a handle from bell_ipc_handle) into the
// current device's address space, peer access enabled as needed; *ptr_out =
// mapped base + offset, *base_out = the mapped base (for bell_ipc_close).
extern "C" int bell_ipc_open(const void* handle, uint64_t offset, void** ptr_out, void** base_out) {
  if (!handle || !ptr_out || !base_out) return fail(BELL_ERR_ARG, "bell_ipc_open: NULL pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(BELL_ERR_LAUNCH, std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
  *base_out = base;
  *ptr_out = static_cast<char*>(base) + offset;
  return BELL_OK;
}

extern "C" int bell_ipc_close(void* base) {
  if (!base) return BELL_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return fail(BELL_ERR_LAUNCH, std::string("cudaIpcCloseMemHandle: ") + cudaGetErrorString(e));
  return BELL_OK;
}
