// bell_loop.cu — RMSNorm, diagonal SSM injection and the L-iteration
// shared-weight loop  h <- h + FFN(RMSNorm(h))  (bf16).
//
// Loop order follows the reference persistent_mlp_step
// (csrc/loop/persistent_core.cu:315-335): normalise, run the Block-ELL
// SwiGLU without fused residual, add the PRE-norm h.  RMSNorm follows
// looped_blockell/layers/norms.py:8-15 (eps default 1e-5, config.py:110).
#include <cstdlib>
#include <string>

#include "bell_host.h"
#include "bell_ptx.cuh"

namespace bell {

// One warp per token row; fp32 sum of squares, bf16 in/out.
__global__ void __launch_bounds__(256) bell_rmsnorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                           const __nv_bfloat16* __restrict__ gain,
                                                           __nv_bfloat16* __restrict__ out, int64_t T, int d,
                                                           float eps) {
  griddep_wait();  // launched behind the previous kernel of the loop: its writes first
  const int64_t row = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const __nv_bfloat16* xr = x + row * d;
  __nv_bfloat16* orow = out + row * d;
  float ss = 0.f;
  for (int i = lane * 8; i < d; i += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 f = unpack_bf16x2(w[t]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / float(d) + eps);
  for (int i = lane * 8; i < d; i += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + i);
    const uint4 gv = *reinterpret_cast<const uint4*>(gain + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    const uint32_t g[4] = {gv.x, gv.y, gv.z, gv.w};
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 f = unpack_bf16x2(w[t]);
      const float2 s = unpack_bf16x2(g[t]);
      o[t] = pack_bf16x2(f.x * inv * s.x, f.y * inv * s.y);
    }
    *reinterpret_cast<uint4*>(orow + i) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// fp32 RMSNorm (fp32 in/out, fp32 gain), one warp per token row, the
// reference layer's precision for fp32 activations (norms.py:8-15).
__global__ void __launch_bounds__(256) bell_rmsnorm_f32_kernel(const float* __restrict__ x,
                                                               const float* __restrict__ gain,
                                                               float* __restrict__ out, int64_t T, int d, float eps) {
  const int64_t row = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const float* xr = x + row * d;
  float* orow = out + row * d;
  float ss = 0.f;
  for (int i = lane * 4; i < d; i += 128) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / float(d) + eps);
  for (int i = lane * 4; i < d; i += 128) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    const float4 g = *reinterpret_cast<const float4*>(gain + i);
    *reinterpret_cast<float4*>(orow + i) = make_float4(v.x * inv * g.x, v.y * inv * g.y, v.z * inv * g.z, v.w * inv * g.w);
  }
}

// h = exp(-softplus(log_dt) * exp(log_A)) * h + softplus(log_dt) * e
// (reference diagonal_injection_kernel, persistent_core.cu:53-83).
__global__ void __launch_bounds__(256) bell_injection_kernel(const __nv_bfloat16* __restrict__ h,
                                                             const __nv_bfloat16* __restrict__ e,
                                                             const float* __restrict__ log_A,
                                                             const float* __restrict__ log_dt,
                                                             __nv_bfloat16* __restrict__ out, int64_t n, int d) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int f = int(i % d);
    const float ldt = log_dt[f];
    const float dt = ldt > 20.f ? ldt : (ldt < -20.f ? expf(ldt) : log1pf(expf(ldt)));
    const float decay = expf(-dt * expf(log_A[f]));
    out[i] = __float2bfloat16(decay * __bfloat162float(h[i]) + dt * __bfloat162float(e[i]));
  }
}

// Injection and the first RMSNorm of persistent_mlp_step in one pass: one
// warp per token row writes the injected h (bf16, the residual base) and
// normalises those bf16 values, so the result is bit-identical to the two
// kernels above run back to back.  Each lane reads back only what it wrote.
__global__ void __launch_bounds__(256) bell_inject_rmsnorm_kernel(
    const __nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ e, const float* __restrict__ log_A,
    const float* __restrict__ log_dt, const __nv_bfloat16* __restrict__ gain, __nv_bfloat16* h_out,
    __nv_bfloat16* __restrict__ normed, int64_t T, int d, float eps) {
  const int64_t row = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const __nv_bfloat16* hr = h + row * d;
  const __nv_bfloat16* er = e + row * d;
  __nv_bfloat16* hor = h_out + row * d;
  float ss = 0.f;
  for (int i = lane * 8; i < d; i += 256) {
    const uint4 hv = *reinterpret_cast<const uint4*>(hr + i);
    const uint4 ev = *reinterpret_cast<const uint4*>(er + i);
    const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w}, ew[4] = {ev.x, ev.y, ev.z, ev.w};
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 hf = unpack_bf16x2(hw[t]), ef = unpack_bf16x2(ew[t]);
      float v[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int f = i + 2 * t + u;
        const float ldt = log_dt[f];
        const float dt = ldt > 20.f ? ldt : (ldt < -20.f ? expf(ldt) : log1pf(expf(ldt)));
        const float decay = expf(-dt * expf(log_A[f]));
        v[u] = decay * (u ? hf.y : hf.x) + dt * (u ? ef.y : ef.x);
      }
      o[t] = pack_bf16x2(v[0], v[1]);
      const float2 r = unpack_bf16x2(o[t]);  // the stored (rounded) values feed the norm
      ss = fmaf(r.x, r.x, ss);
      ss = fmaf(r.y, r.y, ss);
    }
    *reinterpret_cast<uint4*>(hor + i) = make_uint4(o[0], o[1], o[2], o[3]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / float(d) + eps);
  __nv_bfloat16* nr = normed + row * d;
  for (int i = lane * 8; i < d; i += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(hor + i);
    const uint4 gv = *reinterpret_cast<const uint4*>(gain + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    const uint32_t g[4] = {gv.x, gv.y, gv.z, gv.w};
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 f = unpack_bf16x2(w[t]);
      const float2 sc = unpack_bf16x2(g[t]);
      o[t] = pack_bf16x2(f.x * inv * sc.x, f.y * inv * sc.y);
    }
    *reinterpret_cast<uint4*>(nr + i) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Sums of squares of the bf16 state per 64-column block: ss[t*parts + r] =
// sum_{j<64} h[t, 64r + j]^2 (the folded RMSNorm's input for the first
// iteration; later iterations get them from the down epilogue).  One warp per
// row; lane group g = lane/8 takes block r = 4i + g, 8 lanes x 8 columns.
__global__ void __launch_bounds__(256) bell_row_ss_kernel(const __nv_bfloat16* __restrict__ h, float* __restrict__ ss,
                                                          int64_t T, int d) {
  const int64_t row = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const int parts = d / 64;
  for (int r0 = 0; r0 < parts; r0 += 4) {
    const int r = r0 + (lane >> 3);
    float acc = 0.f;
    if (r < parts) {
      const uint4 v = *reinterpret_cast<const uint4*>(h + row * d + r * 64 + (lane & 7) * 8);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = unpack_bf16x2(w[t]);
        acc = fmaf(f.x, f.x, fmaf(f.y, f.y, acc));
      }
    }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((lane & 7) == 0 && r < parts) ss[row * parts + r] = acc;
  }
}

// out[r,k] = tile (r,k) of w with every input row i scaled by gain[c*64 + i]
// (c = cols[r,k]): RMSNorm's gain folded into a gate/up weight.  Dead slots
// keep their tile unscaled (the kernels skip them).
__global__ void __launch_bounds__(256) bell_gain_scale_kernel(const __nv_bfloat16* __restrict__ w,
                                                              const int32_t* __restrict__ cols,
                                                              const __nv_bfloat16* __restrict__ gain,
                                                              __nv_bfloat16* __restrict__ out, int64_t n8, int C,
                                                              int out_in) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t e = i * 8;               // first of 8 elements (one 16-byte group)
    const int64_t tile = e / (64 * 64);
    const int within = int(e % (64 * 64));
    const int c = cols[tile];
    uint4 v = *reinterpret_cast<const uint4*>(w + e);
    if (c >= 0 && c < C) {
      uint32_t u[4] = {v.x, v.y, v.z, v.w};
      if (out_in) {  // [B_out][B_in]: the 8 elements are consecutive inputs
        const int i0 = within % 64;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float2 f = unpack_bf16x2(u[t]);
          u[t] = pack_bf16x2(f.x * __bfloat162float(gain[c * 64 + i0 + 2 * t]),
                             f.y * __bfloat162float(gain[c * 64 + i0 + 2 * t + 1]));
        }
      } else {  // [B_in][B_out]: one input row
        const float gsc = __bfloat162float(gain[c * 64 + within / 64]);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float2 f = unpack_bf16x2(u[t]);
          u[t] = pack_bf16x2(f.x * gsc, f.y * gsc);
        }
      }
      v = make_uint4(u[0], u[1], u[2], u[3]);
    }
    *reinterpret_cast<uint4*>(out + e) = v;
  }
}

static size_t a16(size_t v) { return (v + 15) & ~size_t(15); }

LoopWs loop_ws(int64_t T, int32_t d_model, int32_t R_gu, int32_t K_g, int32_t K_u, int32_t B) {
  LoopWs L{};
  if (B != 64 || T <= 0) {
    L.total = 64;
    return L;
  }
  const int64_t n_mt = (T + 127) / 128;
  size_t off = 0;
  L.counters = off;
  off += a16(size_t(3 * n_mt) * 4);
  L.ss = off;
  off += a16(size_t(T) * size_t(d_model / 64) * 4);
  L.wg = off;
  off += a16(size_t(R_gu) * K_g * 64 * 64 * 2);
  L.wu = off;
  off += a16(size_t(R_gu) * K_u * 64 * 64 * 2);
  L.total = off;
  return L;
}

int launch_rmsnorm(const void* x, const void* gain, void* out, int64_t T, int d, float eps, cudaStream_t s,
                   bool pdl = false) {
  if (T == 0) return BELL_OK;
  const int64_t blocks = (T + 7) / 8;
  if (pdl) {  // programmatic stream serialization: the kernel waits for its predecessor first
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(blocks));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, bell_rmsnorm_kernel, static_cast<const __nv_bfloat16*>(x),
                                       static_cast<const __nv_bfloat16*>(gain), static_cast<__nv_bfloat16*>(out), T,
                                       d, eps);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return fail(BELL_ERR_LAUNCH, std::string("bell_rmsnorm_kernel: ") + cudaGetErrorString(e));
    }
    return BELL_OK;
  }
  bell_rmsnorm_kernel<<<unsigned(blocks), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                        static_cast<const __nv_bfloat16*>(gain),
                                                        static_cast<__nv_bfloat16*>(out), T, d, eps);
  return check_launch("bell_rmsnorm_kernel");
}

// BELL_LOOP_AUTO at tile size 64: the single persistent kernel (true) or the
// stream-ordered launches (false), whichever measured faster on B200.
static constexpr bool kAutoPersistent = false;

}  // namespace bell

using namespace bell;

extern "C" {

int bell_rmsnorm_bf16(int64_t T, int32_t d_model, const void* x, const void* gain, float eps, void* out,
                      void* stream) {
  if (T < 0 || d_model <= 0 || d_model % 8 != 0)
    return fail(BELL_ERR_SHAPE, "bell_rmsnorm_bf16: need T >= 0 and d_model a positive multiple of 8");
  if (!gain || (T > 0 && (!x || !out))) return fail(BELL_ERR_ARG, "bell_rmsnorm_bf16: NULL pointer");
  if (!aligned16(x) || !aligned16(gain) || !aligned16(out)) return fail(BELL_ERR_ALIGN, "bell_rmsnorm_bf16: alignment");
  if (int rc = require_sm100()) return rc;
  return launch_rmsnorm(x, gain, out, T, d_model, eps, static_cast<cudaStream_t>(stream));
}

int bell_rmsnorm_f32(int64_t T, int32_t d_model, const float* x, const float* gain, float eps, float* out,
                     void* stream) {
  if (T < 0 || d_model <= 0 || d_model % 4 != 0)
    return fail(BELL_ERR_SHAPE, "bell_rmsnorm_f32: need T >= 0 and d_model a positive multiple of 4");
  if (!gain || (T > 0 && (!x || !out))) return fail(BELL_ERR_ARG, "bell_rmsnorm_f32: NULL pointer");
  if (!aligned16(x) || !aligned16(gain) || !aligned16(out)) return fail(BELL_ERR_ALIGN, "bell_rmsnorm_f32: alignment");
  if (int rc = require_sm100()) return rc;
  if (T == 0) return BELL_OK;
  bell_rmsnorm_f32_kernel<<<unsigned((T + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, gain, out, T,
                                                                                               d_model, eps);
  return check_launch("bell_rmsnorm_f32_kernel");
}

int bell_inject_rmsnorm_bf16(int64_t T, int32_t d_model, const void* h, const void* e, const float* log_A,
                             const float* log_dt, const void* gain, float eps, void* h_out, void* normed,
                             void* stream) {
  if (T < 0 || d_model <= 0 || d_model % 8 != 0)
    return fail(BELL_ERR_SHAPE, "bell_inject_rmsnorm_bf16: need T >= 0 and d_model a positive multiple of 8");
  if (!log_A || !log_dt || !gain || (T > 0 && (!h || !e || !h_out || !normed)))
    return fail(BELL_ERR_ARG, "bell_inject_rmsnorm_bf16: NULL pointer");
  if (!aligned16(h) || !aligned16(e) || !aligned16(gain) || !aligned16(h_out) || !aligned16(normed))
    return fail(BELL_ERR_ALIGN, "bell_inject_rmsnorm_bf16: alignment");
  if (int rc = require_sm100()) return rc;
  if (T == 0) return BELL_OK;
  bell_inject_rmsnorm_kernel<<<unsigned((T + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(h), static_cast<const __nv_bfloat16*>(e), log_A, log_dt,
      static_cast<const __nv_bfloat16*>(gain), static_cast<__nv_bfloat16*>(h_out), static_cast<__nv_bfloat16*>(normed),
      T, d_model, eps);
  return check_launch("bell_inject_rmsnorm_kernel");
}

int bell_diag_injection_bf16(int64_t T, int32_t d_model, const void* h, const void* e, const float* log_A,
                             const float* log_dt, void* out, void* stream) {
  if (T < 0 || d_model <= 0) return fail(BELL_ERR_SHAPE, "bell_diag_injection_bf16: bad shape");
  if (!log_A || !log_dt || (T > 0 && (!h || !e || !out))) return fail(BELL_ERR_ARG, "bell_diag_injection_bf16: NULL pointer");
  if (int rc = require_sm100()) return rc;
  const int64_t n = T * d_model;
  if (n == 0) return BELL_OK;
  int sms = 0;
  if (int rc = device_sm_count(&sms)) return rc;
  const int64_t want = (n + 255) / 256;
  const int grid = int(want < int64_t(sms) * 16 ? want : int64_t(sms) * 16);
  bell_injection_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(h), static_cast<const __nv_bfloat16*>(e), log_A, log_dt,
      static_cast<__nv_bfloat16*>(out), n, d_model);
  return check_launch("bell_injection_kernel");
}

int bell_loop_fwd_bf16(const BellLoopDesc* d, void* stream) {
  if (!d) return fail(BELL_ERR_ARG, "descriptor is NULL");
  if (d->L < 0) return fail(BELL_ERR_ARG, "L must be >= 0");
  if (!d->norm_gain || (d->T > 0 && (!d->h_in || !d->h_out || !d->hn || !d->h_mid || !d->plan || !d->workspace)))
    return fail(BELL_ERR_ARG, "h_in, h_out, norm_gain, hn, h_mid, plan and workspace must be non-NULL");
  if (d->mode != BELL_LOOP_AUTO && d->mode != BELL_LOOP_LAUNCHES && d->mode != BELL_LOOP_PERSISTENT)
    return fail(BELL_ERR_ARG, "unknown loop mode");
  BellFFNDesc f{};
  f.T = d->T;
  f.d_model = d->d_model;
  f.d_ff = d->d_ff;
  f.dtype = BELL_DTYPE_BF16;
  f.add_residual = 1;
  f.x = d->hn;
  f.residual = d->h_out;
  f.h = d->h_mid;
  f.out = d->h_out;
  f.plan = d->plan;
  f.gate = d->gate;
  f.up = d->up;
  f.down = d->down;
  f.status = d->status;
  if (int rc = check_ffn(&f, BELL_DTYPE_BF16)) return rc;
  // The persistent kernel (tile size 64) folds RMSNorm into its GEMMs; the
  // launch loop runs the RMSNorm kernel (measured faster there: config 4,
  // 0.856 against 0.869-0.882 ms folded).
  const bool persistent = d->mode == BELL_LOOP_PERSISTENT || (d->mode == BELL_LOOP_AUTO && kAutoPersistent &&
                                                              d->gate.B == 64);
  const bool fold = persistent;
  if (persistent && d->gate.B != 64) return fail(BELL_ERR_SHAPE, "the persistent loop kernel needs tile size 64");
  if (fold && (!aligned16(d->workspace) || !aligned16(d->norm_gain) || d->d_model % 64 != 0))
    return fail(BELL_ERR_ALIGN, "loop: workspace and norm_gain must be 16-byte aligned");
  if (int rc = require_sm100()) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t bytes = size_t(d->T) * d->d_model * 2;
  if (d->h_out != d->h_in && bytes > 0) {
    cudaError_t e = cudaMemcpyAsync(d->h_out, d->h_in, bytes, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return fail(BELL_ERR_LAUNCH, std::string("loop copy: ") + cudaGetErrorString(e));
  }
  if (d->T == 0 || d->L == 0) return BELL_OK;
  int32_t* status = d->status ? d->status : default_status_ptr();
  if (!status) return BELL_ERR_LAUNCH;
  if (int rc = launch_ffn_plan(&f, status, s)) return rc;
  if (!fold) {
    // Each launch of the chain may start while its predecessor drains
    // (programmatic dependent launch): its CTAs do their set-up, then wait for
    // the predecessor's completion before touching global memory.
    // BELL_LOOP_PDL=0 launches them plainly.
    const char* pdl_env = std::getenv("BELL_LOOP_PDL");
    const bool pdl = !(pdl_env && pdl_env[0] == '0');
    for (int it = 0; it < d->L; ++it) {
      if (int rc = launch_rmsnorm(d->h_out, d->norm_gain, d->hn, d->T, d->d_model, d->eps, s, pdl)) return rc;
      if (int rc = gate_up_bf16(&f, status, s, pdl)) return rc;
      // out = h_mid Wd + h (the pre-norm state), written in place over h
      if (int rc = down_bf16(&f, status, s, pdl)) return rc;
    }
    return BELL_OK;
  }
  // folded RMSNorm: gain into the gate/up tiles, the first sums of squares
  const LoopWs W = loop_ws(d->T, d->d_model, d->gate.R, d->gate.K, d->up.K, 64);
  char* ws = static_cast<char*>(d->workspace);
  float* ss = reinterpret_cast<float*>(ws + W.ss);
  BellEll wg = d->gate, wu = d->up;
  wg.values = ws + W.wg;
  wu.values = ws + W.wu;
  int sms = 0;
  if (int rc = device_sm_count(&sms)) return rc;
  const BellEll* src[2] = {&d->gate, &d->up};
  const BellEll* dst[2] = {&wg, &wu};
  for (int k = 0; k < 2; ++k) {
    const int64_t n8 = int64_t(src[k]->R) * src[k]->K * 64 * 64 / 8;
    const int64_t grid = (n8 + 255) / 256 < int64_t(sms) * 8 ? (n8 + 255) / 256 : int64_t(sms) * 8;
    bell_gain_scale_kernel<<<unsigned(grid), 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(src[k]->values), src[k]->col_indices,
        static_cast<const __nv_bfloat16*>(d->norm_gain), static_cast<__nv_bfloat16*>(const_cast<void*>(dst[k]->values)),
        n8, src[k]->C, src[k]->layout == BELL_TILE_OUT_IN ? 1 : 0);
    if (int rc = check_launch("bell_gain_scale_kernel")) return rc;
  }
  bell_row_ss_kernel<<<unsigned((d->T + 7) / 8), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(d->h_out), ss, d->T,
                                                               d->d_model);
  if (int rc = check_launch("bell_row_ss_kernel")) return rc;
  return loop_persistent_bf16(d, wg, wu, status, s);
}

size_t bell_loop_workspace_bytes(int64_t T, int32_t d_model, int32_t R_gu, int32_t K_gate, int32_t K_up, int32_t B) {
  return loop_ws(T, d_model, R_gu, K_gate, K_up, B).total;
}

}  // extern "C"
