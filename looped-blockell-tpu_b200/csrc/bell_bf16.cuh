// bell_bf16.cuh — definitions shared by the bf16 Block-ELL kernels
// (bell_bf16.cu: token-major kernels; bell_bf16_t.cu: feature-major kernels).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "bell_ptx.cuh"

namespace bell {

static constexpr int kBM = 128;        // tokens per tile (MMA M) in the token-major kernels
static constexpr int kBK = 64;         // K elements per pipeline stage (128 B of bf16)
static constexpr int kThreads = 192;   // 6 warps
static constexpr uint32_t kNone = 255;

struct Bf16Params {
  int64_t T;
  int32_t n_mtiles;
  int32_t R;         // output block-rows
  int32_t K0, K1;    // slots per row of w0 / w1
  int32_t S;         // plan entries per row
  const uint32_t* plan;
  const int32_t* counts;
  void* out;         // GU: h [T, R*B] bf16; linear: out [T, R*B]
  int64_t ld_out;    // elements
  void* gate_pre;    // GU optional
  void* up_out;      // GU optional
  const void* residual;  // linear optional (bf16, same shape as out)
  int32_t add_residual;
  int32_t out_f32;   // linear: write fp32 instead of bf16
  int32_t band;      // block-rows per band of the unit order (see unit_mr)
  int32_t split;     // feature-major gate/up: one weight tile per plan step
  // linear with the SiLU*up backward in the epilogue (bwd_gate != NULL): the
  // accumulator is d_h; reads gate_pre / up_out [T, ld_bwd] bf16 at the same
  // feature, writes d_gate at out[t, f] and d_up at out[t, du_off + f]
  const void* bwd_gate;
  const void* bwd_up;
  int64_t ld_bwd;
  int64_t du_off;
  int32_t* status;
  uint64_t timeout_ns;
  int32_t max_ctas;  // cap on the persistent grid (0 = all SMs)
  int64_t res_lo, res_hi;  // linear: residual added to token rows [res_lo, res_hi) only
  // Token-tile dataflow (the persistent loop kernel; NULL elsewhere): before a
  // unit of token tile m loads its activations, the producer waits until
  // dep_cnt[m] >= dep_target; after a unit's stores, each epilogue warp adds 1
  // to sig_cnt[m].
  const unsigned* dep_cnt;
  unsigned dep_target;
  unsigned* sig_cnt;
  // the epilogue also waits for epi_dep_cnt[m] >= epi_dep_target (and for
  // dep_cnt[m] >= dep_target) before it reads global inputs of tile m
  const unsigned* epi_dep_cnt;
  unsigned epi_dep_target;
  // RMSNorm folded into the GEMMs (the loop at tile size 64, NULL elsewhere):
  // a gate/up epilogue scales row t's accumulators by
  // rsqrt(sum(row_ss[t*ss_parts .. +ss_parts]) * inv_d + eps) before SiLU*up;
  // a linear epilogue writes the sum of squares of row t's stored (bf16)
  // outputs of block-row r to ss_out[t*ss_parts + r].
  const float* row_ss;
  float* ss_out;
  int32_t ss_parts;
  float inv_d, eps;
  // segment of the unit sequence this launch (or loop-kernel phase) covers:
  // units [u_begin, u_end) of the n_mtiles * R (u_end == 0: all of them)
  int32_t u_begin, u_end;
  // launch with programmatic stream serialization (the engine kernel waits for
  // its predecessor after its shared-memory / TMEM set-up; tile 64/128 engine only)
  int32_t pdl;
  // gate/up of the fp32 path on the tensor cores (tile-64 engine only): with
  // h_parts > 0 the epilogue writes the exact fp32 silu(g) * u as three bf16
  // parts at out[t * ld_out + part * h_parts + f], part = 0, 1, 2
  int64_t h_parts;
};

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait (bounded) until *cnt >= target; the acquire and the proxy fence that
// follows order this thread's later loads, TMA loads included, after the
// writes the counter publishes.  Returns false on timeout or abort.
__device__ __forceinline__ bool wait_count(const unsigned* cnt, unsigned target, const Ctl& ctl) {
  if (ld_acquire_u32(cnt) < target) {
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_u32(cnt) < target) {
      if (*ctl.abort) return false;
      if (globaltimer_ns() - t0 > ctl.timeout_ns) {
        raise_status(ctl, BELL_STATUS_TIMEOUT);
        return false;
      }
      __nanosleep(32);
    }
  }
  fence_proxy_async_global();
  return true;
}

// Publish this warp's global stores (generic proxy, read later by TMA in
// other CTAs) and add one to *cnt.
__device__ __forceinline__ void signal_count(unsigned* cnt) {
  fence_proxy_async_global();
  __threadfence();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) atomicAdd(cnt, 1u);
}

// Whether token row `row` gets the residual: res_hi == 0 means every row.
__device__ __forceinline__ bool res_row(const Bf16Params& p, int64_t row) {
  return p.res_hi == 0 || (row >= p.res_lo && row < p.res_hi);
}

// Persistent grid size: min(units, SMs, max_ctas when set).
inline int grid_size(int64_t units, int sms, int32_t max_ctas) {
  int64_t g = units < sms ? units : sms;
  if (max_ctas > 0 && g > max_ctas) g = max_ctas;
  return int(g < 1 ? 1 : g);
}

// d_gate, d_up of h = silu(g) * u for an incoming d_h (the reference
// swiglu_bwd.cu:305-334 formula), fp32.  sigmoid(g) = 0.5 + 0.5 tanh(g / 2)
// on the hardware tanh (absolute error below 2^-11 on s, under the bf16
// rounding of the results); an IEEE reciprocal here made the fused backward
// epilogue the bottleneck of its kernel.
__device__ __forceinline__ void silu_mul_grad(float dh, float g, float u, float& dg, float& du) {
  const float s = fmaf(0.5f, tanh_approx(0.5f * g), 0.5f);
  dg = dh * u * (s + g * s * (1.f - s));
  du = dh * g * s;
}

// Work-unit order: bands of `band` output block-rows; inside a band, all
// token tiles, block-row fastest.  Consecutive units share a token tile (its
// activation panel stays in L2) and a band's weight tiles stay L2-resident
// while every token tile passes, instead of the whole weight set cycling
// through L2 once per token tile.
__device__ __forceinline__ void unit_mr(int u, const Bf16Params& p, int& m, int& r) {
  const int per_band = p.n_mtiles * p.band;
  const int b = u / per_band;
  const int rem = u - b * per_band;
  const int rows = min(p.band, p.R - b * p.band);
  m = rem / rows;
  r = b * p.band + (rem - m * rows);
}

// Feature-major (transposed) B = 128 kernels, bell_bf16_t.cu.  `a` is the
// activation map with 256-row boxes.
// BELL_GU_SPLIT override for the feature-major gate/up kernel: -1 automatic,
// 0 fused steps, 1 one weight tile per step (plan built without merging)
int fmajor_split_env();

// Small-tile kernels (B = 16, 32), bell_small.cu: activation map with B x 128
// boxes, weight map with one tile per box (32- / 64-byte swizzle).
int make_small_x_map(CUtensorMap* m, const void* base, int64_t cols, int64_t rows, int B);
int make_small_w_map(CUtensorMap* m, const BellEll& e);
// Tile gradients on the CUDA cores (bf16 at B = 16, 32; fp32 operands at any
// B); grad already zeroed or accumulating.
int launch_sddmm_ffma(const BellSddmmDesc* d, bool f32, int32_t* status, cudaStream_t s);
int launch_small(bool gate_up, int B, bool w_mn, const CUtensorMap& x, const CUtensorMap& w0, const CUtensorMap& w1,
                 const Bf16Params& p, cudaStream_t stream);
int launch_fmajor(bool gate_up, bool w_mn, const CUtensorMap& a, const CUtensorMap& w0, const CUtensorMap& w1,
                  const Bf16Params& p, cudaStream_t stream);

}  // namespace bell
