// bell_f32x.cu — the fp32 SwiGLU forward on the bf16 tensor cores.
//
// Each fp32 operand is split into three bf16 parts, v = v0 + v1 + v2 with
// v0 = bf16(v), v1 = bf16(v - v0), v2 = bf16(v - v0 - v1) (round to nearest,
// each difference exact in fp32), which leaves |v - v0 - v1 - v2| <= 2^-27 |v|.
// A product x w is then the six leading cross products
//   x0 w0 + x0 w1 + x1 w0 + x0 w2 + x1 w1 + x2 w0
// (the dropped x1 w2, x2 w1, x2 w2 are below 2^-26 |x w|), each an exact
// bf16 x bf16 product accumulated in fp32 in TMEM.  This is the "bf16x6"
// scheme of Henry, Tang and Heinecke, "Leveraging the bfloat16 Artificial
// Intelligence Datatype For Higher-Precision Computations" (ARITH 2019).
//
// Block-ELL form: one activation matrix A [T, 3 d_ff + 3 d_model] bf16 holds
// the parts of h (columns [0, 3 d_ff)) and of x (columns [3 d_ff, +3 d_model)),
// part p of a C-block-wide operand at column block p C + c.  A weight slot
// (r, k) with column c becomes six slots of bf16 tiles (bell_f32x_expand_ell):
//   (x part, w part) = (0,0) (0,1) (1,0) (0,2) (1,1) (2,0),
// column base + x_part * part_cols + c.  The down projection gets three
// more slots per block-row r: identity tiles on the x-region parts of column
// block r, so the residual x0 + x1 + x2 is added inside the same fp32
// accumulator.  The forward then runs on the bf16 Block-ELL kernels: gate and
// up from A's x region (at tile size 64 with enough work, one gate/up kernel
// whose epilogue writes the exact fp32 SiLU*up as three bf16 parts into A's h
// region; else two linears with fp32 output, then SiLU*up in fp32 split into
// A), and the down linear (fp32 output) from A.  Semantics: looped_blockell/layers/
// block_ell.py:149-182 and mlp.py:119-145 (the reference computes in fp32).
#include <cuda_bf16.h>

#include <cstdlib>
#include <string>

#include "bell_host.h"
#include "bell_ptx.cuh"

namespace bell {

namespace {

// The (x part, w part) pairs of the six expanded slots of one weight slot.
__constant__ int8_t kXPart[6] = {0, 0, 1, 0, 1, 2};
__constant__ int8_t kWPart[6] = {0, 1, 0, 2, 1, 0};

__device__ __forceinline__ void split3(float v, __nv_bfloat16& a, __nv_bfloat16& b, __nv_bfloat16& c) {
  float p0, p1, p2;
  split3_bf16(v, p0, p1, p2);
  a = __float2bfloat16_rn(p0);
  b = __float2bfloat16_rn(p1);
  c = __float2bfloat16_rn(p2);
}

// One thread per element of one original tile: writes that element of its
// six expanded tiles; thread (r, k, 0) also writes the six column indices.
__global__ void f32x_expand_kernel(const float* __restrict__ w, const int32_t* __restrict__ cols, int32_t R,
                                   int32_t K, int32_t B, int32_t K6, int32_t col_base, int32_t part_cols,
                                   __nv_bfloat16* __restrict__ w6, int32_t* __restrict__ cols6) {
  const int64_t per_tile = int64_t(B) * B;
  const int64_t n = int64_t(R) * K * per_tile;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t slot = i / per_tile, e = i % per_tile;
    const int64_t r = slot / K, k = slot % K;
    __nv_bfloat16 p[3];
    split3(w[i], p[0], p[1], p[2]);
    __nv_bfloat16* dst = w6 + (r * K6 + 6 * k) * per_tile + e;
#pragma unroll
    for (int j = 0; j < 6; ++j) dst[j * per_tile] = p[kWPart[j]];
    if (e == 0) {
      const int32_t c = cols[slot];
#pragma unroll
      for (int j = 0; j < 6; ++j) cols6[r * K6 + 6 * k + j] = c < 0 ? -1 : col_base + kXPart[j] * part_cols + c;
    }
  }
}

// The three identity slots of every block-row (after its 6K expanded slots).
__global__ void f32x_identity_kernel(int32_t R, int32_t K6, int32_t B, int32_t first, int32_t ident_base,
                                     int32_t ident_stride, __nv_bfloat16* __restrict__ w6,
                                     int32_t* __restrict__ cols6) {
  const int64_t per_tile = int64_t(B) * B;
  const int64_t n = int64_t(R) * 3 * per_tile;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t slot = i / per_tile, e = i % per_tile;
    const int64_t r = slot / 3, q = slot % 3;
    const int64_t row = e / B, col = e % B;
    w6[(r * K6 + first + q) * per_tile + e] = __float2bfloat16_rn(row == col ? 1.f : 0.f);
    if (e == 0) cols6[r * K6 + first + q] = ident_base + int32_t(q) * ident_stride + int32_t(r);
  }
}

// src [T, n] fp32 (row stride ld_src; NULL: zeros) -> parts at
// dst[t, col0 + p n + j] (row stride ld_dst bf16 elements); four consecutive
// elements per thread.
__global__ void f32x_split_kernel(const float* __restrict__ src, int64_t ld_src, int64_t T, int32_t n,
                                  __nv_bfloat16* __restrict__ dst, int64_t ld_dst, int64_t col0) {
  const int32_t n4 = n / 4;
  const int64_t total = T * n4;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t t = i / n4;
    const int32_t j = int32_t(i % n4) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (src) v = *reinterpret_cast<const float4*>(src + t * ld_src + j);
    __nv_bfloat16 a[4], b[4], c[4];
    split3(v.x, a[0], b[0], c[0]);
    split3(v.y, a[1], b[1], c[1]);
    split3(v.z, a[2], b[2], c[2]);
    split3(v.w, a[3], b[3], c[3]);
    __nv_bfloat16* row = dst + t * ld_dst + col0 + j;
    *reinterpret_cast<uint2*>(row) = *reinterpret_cast<const uint2*>(a);
    *reinterpret_cast<uint2*>(row + n) = *reinterpret_cast<const uint2*>(b);
    *reinterpret_cast<uint2*>(row + 2 * int64_t(n)) = *reinterpret_cast<const uint2*>(c);
  }
}

// h = silu(g) * u in fp32 (optionally stored), split into dst[t, p F + j].
__global__ void f32x_silu_split_kernel(const float* __restrict__ g, const float* __restrict__ u, int64_t T,
                                       int32_t F, float* __restrict__ h, __nv_bfloat16* __restrict__ dst,
                                       int64_t ld_dst) {
  const int32_t n4 = F / 4;
  const int64_t total = T * n4;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t t = i / n4;
    const int32_t j = int32_t(i % n4) * 4;
    const float4 gv = *reinterpret_cast<const float4*>(g + t * F + j);
    const float4 uv = *reinterpret_cast<const float4*>(u + t * F + j);
    const float4 hv = make_float4(silu_mul_exact(gv.x, uv.x), silu_mul_exact(gv.y, uv.y), silu_mul_exact(gv.z, uv.z),
                                  silu_mul_exact(gv.w, uv.w));
    if (h) *reinterpret_cast<float4*>(h + t * F + j) = hv;
    __nv_bfloat16 a[4], b[4], c[4];
    split3(hv.x, a[0], b[0], c[0]);
    split3(hv.y, a[1], b[1], c[1]);
    split3(hv.z, a[2], b[2], c[2]);
    split3(hv.w, a[3], b[3], c[3]);
    __nv_bfloat16* row = dst + t * ld_dst + j;
    *reinterpret_cast<uint2*>(row) = *reinterpret_cast<const uint2*>(a);
    *reinterpret_cast<uint2*>(row + F) = *reinterpret_cast<const uint2*>(b);
    *reinterpret_cast<uint2*>(row + 2 * int64_t(F)) = *reinterpret_cast<const uint2*>(c);
  }
}

int grid_for(int64_t n, int threads) {
  int sms = 0;
  if (device_sm_count(&sms) || sms < 1) sms = 148;
  const int64_t want = (n + threads - 1) / threads;
  const int64_t cap = int64_t(sms) * 16;
  return int(want < 1 ? 1 : (want < cap ? want : cap));
}

size_t up256(size_t v) { return (v + 255) & ~size_t(255); }

// The fused gate/up kernel (both projections in one unit, twice the steps of
// a linear's unit) once there are at least kFusedUnitsPerSm units per SM;
// with fewer the unit count leaves a tail.  Config 1's shapes on B200, fused
// against two linears: T=1024 (1.7 units per SM) 0.109 / 0.096 ms, T=4096
// 0.142 / 0.153 ms, T=8192 0.218 / 0.248 ms, T=65536 1.17 / 1.54 ms.
// BELL_F32X_FUSED=0/1 forces one or the other.
constexpr int64_t kFusedUnitsPerSm = 4;
bool fused_gate_up(int64_t T, int32_t R_gu) {
  const char* e = std::getenv("BELL_F32X_FUSED");
  if (e && (e[0] == '0' || e[0] == '1')) return e[0] == '1';
  int sms = 0;
  if (device_sm_count(&sms) || sms < 1) sms = 148;
  return ((T + 127) / 128) * int64_t(R_gu) >= kFusedUnitsPerSm * sms;
}

struct F32xWs {
  size_t a, g, u, plan, total;
};

F32xWs f32x_ws(int64_t T, int32_t d_model, int32_t d_ff, int32_t B, int32_t K_g6, int32_t K_u6, int32_t K_d6) {
  F32xWs w{};
  const int32_t R_gu = d_ff / B, R_d = d_model / B;
  // one plan buffer, used in turn by each launch: the fused gate/up's plan
  // (gate, up and down lists) or the gate / up / down linears' plans
  size_t plan = plan_layout(R_gu, K_g6, K_u6, R_d, K_d6).total;
  const size_t pg = plan_layout(0, 0, 0, R_gu, K_g6).total, pu = plan_layout(0, 0, 0, R_gu, K_u6).total,
               pd = plan_layout(0, 0, 0, R_d, K_d6).total;
  if (pg > plan) plan = pg;
  if (pu > plan) plan = pu;
  if (pd > plan) plan = pd;
  w.a = 0;
  w.g = up256(size_t(T) * (3 * size_t(d_ff) + 3 * size_t(d_model)) * 2);
  w.u = w.g + up256(size_t(T) * size_t(d_ff) * 4);
  w.plan = w.u + up256(size_t(T) * size_t(d_ff) * 4);
  w.total = w.plan + up256(plan);
  return w;
}

int linear(int64_t T, const void* a, const BellEll& w, float* out, const BellFFNDesc* d, cudaStream_t s,
           void* plan) {
  BellLinearDesc L{};
  L.T = T;
  L.dtype = BELL_DTYPE_BF16;
  L.out_dtype = BELL_DTYPE_F32;
  L.add_residual = 0;
  L.max_ctas = d->max_ctas;
  L.x = a;
  L.out = out;
  L.plan = plan;
  L.w = w;
  L.status = d->status;
  return bell_linear_bf16(&L, s);
}

}  // namespace

}  // namespace bell

using namespace bell;

extern "C" {

int32_t bell_f32x_slots(int32_t K, int32_t with_identity) { return 6 * K + (with_identity ? 3 : 0); }

int bell_f32x_expand_ell(const BellEll* w, int32_t col_base, int32_t part_cols, int32_t ident_base,
                         int32_t ident_stride, void* values6, int32_t* cols6, void* stream) {
  if (!w || !w->values || !w->col_indices || !values6 || !cols6)
    return fail(BELL_ERR_ARG, "bell_f32x_expand_ell: NULL pointer");
  if (w->R < 1 || w->K < 1 || (w->B != 16 && w->B != 32 && w->B != 64 && w->B != 128))
    return fail(BELL_ERR_SHAPE, "bell_f32x_expand_ell: need R, K >= 1 and B in {16, 32, 64, 128}");
  if (col_base < 0 || part_cols < 1 || (ident_base >= 0 && ident_stride < 1))
    return fail(BELL_ERR_ARG, "bell_f32x_expand_ell: bad column base / part stride");
  const int32_t K6 = bell_f32x_slots(w->K, ident_base >= 0);
  if (K6 > 254) return fail(BELL_ERR_SHAPE, "bell_f32x_expand_ell: the expanded row needs " + std::to_string(K6) +
                                                " slots; the forward takes at most 254");
  if (!aligned16(values6) || !aligned16(w->values)) return fail(BELL_ERR_ALIGN, "bell_f32x_expand_ell: alignment");
  if (int rc = require_sm100()) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t n = int64_t(w->R) * w->K * w->B * w->B;
  f32x_expand_kernel<<<grid_for(n, 256), 256, 0, s>>>(static_cast<const float*>(w->values), w->col_indices, w->R,
                                                      w->K, w->B, K6, col_base, part_cols,
                                                      static_cast<__nv_bfloat16*>(values6), cols6);
  if (int rc = check_launch("f32x_expand_kernel")) return rc;
  if (ident_base >= 0) {
    const int64_t ni = int64_t(w->R) * 3 * w->B * w->B;
    f32x_identity_kernel<<<grid_for(ni, 256), 256, 0, s>>>(w->R, K6, w->B, 6 * w->K, ident_base, ident_stride,
                                                           static_cast<__nv_bfloat16*>(values6), cols6);
    if (int rc = check_launch("f32x_identity_kernel")) return rc;
  }
  return BELL_OK;
}

size_t bell_f32x_workspace_bytes(int64_t T, int32_t d_model, int32_t d_ff, int32_t B, int32_t K_gate6,
                                 int32_t K_up6, int32_t K_down6) {
  if (T < 0 || B < 1 || d_model < B || d_ff < B || K_gate6 < 1 || K_up6 < 1 || K_down6 < 1) return 0;
  return f32x_ws(T, d_model, d_ff, B, K_gate6, K_up6, K_down6).total;
}

int bell_swiglu_fwd_f32x(const BellFFNDesc* d, void* workspace, void* stream) {
  if (!d) return fail(BELL_ERR_ARG, "descriptor is NULL");
  if (d->dtype != BELL_DTYPE_F32) return fail(BELL_ERR_DTYPE, "bell_swiglu_fwd_f32x: dtype must be BELL_DTYPE_F32");
  const BellEll &g = d->gate, &u = d->up, &w = d->down;
  const int32_t B = g.B;
  if (B != 16 && B != 32 && B != 64 && B != 128)
    return fail(BELL_ERR_SHAPE, "bell_swiglu_fwd_f32x: tile size B must be 16, 32, 64 or 128");
  if (d->T < 0 || d->d_model < B || d->d_ff < B || d->d_model % B || d->d_ff % B)
    return fail(BELL_ERR_SHAPE, "bell_swiglu_fwd_f32x: need T >= 0 and d_model, d_ff positive multiples of B");
  const int32_t CA = 3 * (d->d_ff / B) + 3 * (d->d_model / B);  // column blocks of A
  if (u.B != B || w.B != B || g.R != d->d_ff / B || u.R != g.R || w.R != d->d_model / B || g.C != CA || u.C != CA ||
      w.C != CA)
    return fail(BELL_ERR_SHAPE, "bell_swiglu_fwd_f32x: gate/up/down must be bell_f32x_expand_ell outputs over the " +
                                    std::to_string(CA) + " column blocks of [h parts | x parts]");
  if (g.K % 6 || u.K % 6 || (w.K % 6 != 0 && w.K % 6 != 3))
    return fail(BELL_ERR_SHAPE, "bell_swiglu_fwd_f32x: expanded rows hold 6K slots (down: 6K or 6K + 3)");
  const bool ident = w.K % 6 == 3;
  if (d->add_residual && !ident)
    return fail(BELL_ERR_ARG, "bell_swiglu_fwd_f32x: add_residual needs a down weight expanded with identity slots");
  if (d->T > 0 && (!d->x || !d->out || !workspace)) return fail(BELL_ERR_ARG, "x, out and workspace must be non-NULL");
  if (!aligned16(d->x) || !aligned16(d->out) || !aligned16(workspace) || (d->h && !aligned16(d->h)) ||
      (d->residual && !aligned16(d->residual)) || (d->gate_pre && !aligned16(d->gate_pre)) ||
      (d->up_out && !aligned16(d->up_out)))
    return fail(BELL_ERR_ALIGN, "bell_swiglu_fwd_f32x: buffers must be 16-byte aligned");
  if (int rc = require_sm100()) return rc;
  if (d->T == 0) return BELL_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t T = d->T;
  const int32_t dm = d->d_model, F = d->d_ff;
  const F32xWs W = f32x_ws(T, dm, F, B, g.K, u.K, w.K);
  char* ws = static_cast<char*>(workspace);
  __nv_bfloat16* A = reinterpret_cast<__nv_bfloat16*>(ws + W.a);
  const int64_t LA = int64_t(CA) * B;  // row stride of A, elements
  float* gb = d->gate_pre ? static_cast<float*>(d->gate_pre) : reinterpret_cast<float*>(ws + W.g);
  float* ub = d->up_out ? static_cast<float*>(d->up_out) : reinterpret_cast<float*>(ws + W.u);
  void* plan = ws + W.plan;
  const int64_t xcol = 3 * int64_t(F);  // first column of A's x region
  f32x_split_kernel<<<grid_for(T * (dm / 4), 256), 256, 0, s>>>(static_cast<const float*>(d->x), dm, T, dm, A, LA,
                                                                 xcol);
  if (int rc = check_launch("f32x_split_kernel")) return rc;
  if (B == 64 && !d->h && !d->gate_pre && !d->up_out && fused_gate_up(T, g.R)) {
    // tile 64 without fp32 intermediates: one gate/up kernel whose epilogue
    // writes the exact fp32 silu(g) * u straight into A's h parts
    int32_t* status = d->status ? d->status : default_status_ptr();
    if (!status) return BELL_ERR_LAUNCH;
    BellFFNDesc f{};
    f.T = T;
    f.d_model = int32_t(LA);  // the activation rows the gate/up kernel reads are A's
    f.d_ff = F;
    f.dtype = BELL_DTYPE_BF16;
    f.x = A;
    f.h = A;
    f.plan = plan;
    f.gate = g;
    f.up = u;
    f.down = w;
    f.max_ctas = d->max_ctas;
    if (int rc = launch_ffn_plan(&f, status, s)) return rc;
    if (int rc = gate_up_bf16(&f, status, s, false, LA, F)) return rc;
  } else {
    if (int rc = linear(T, A, g, gb, d, s, plan)) return rc;
    if (int rc = linear(T, A, u, ub, d, s, plan)) return rc;
    f32x_silu_split_kernel<<<grid_for(T * (F / 4), 256), 256, 0, s>>>(gb, ub, T, F, static_cast<float*>(d->h), A,
                                                                      LA);
    if (int rc = check_launch("f32x_silu_split_kernel")) return rc;
  }
  if (ident) {
    // the identity slots add whatever A's x region holds: x itself, the
    // caller's residual, or zeros when no residual is wanted
    const float* res = !d->add_residual ? nullptr : (d->residual ? static_cast<const float*>(d->residual)
                                                                  : static_cast<const float*>(d->x));
    if (res != d->x) {
      f32x_split_kernel<<<grid_for(T * (dm / 4), 256), 256, 0, s>>>(res, dm, T, dm, A, LA, xcol);
      if (int rc = check_launch("f32x_split_kernel")) return rc;
    }
  }
  return linear(T, A, w, static_cast<float*>(d->out), d, s, plan);
}

int bell_f32x_split_rows(int64_t T, int32_t n, const float* src, int64_t ld_src, void* dst, int64_t ld_dst,
                         int64_t col0, void* stream) {
  if (T < 0 || n < 4 || n % 4 || ld_src < n || ld_src % 4 || ld_dst < col0 + 3 * int64_t(n) || ld_dst % 4 ||
      col0 < 0 || col0 % 4)
    return fail(BELL_ERR_SHAPE, "bell_f32x_split_rows: need n, ld_src, ld_dst, col0 multiples of 4 with "
                                "ld_src >= n and ld_dst >= col0 + 3 n");
  if (T > 0 && (!src || !dst)) return fail(BELL_ERR_ARG, "bell_f32x_split_rows: NULL pointer");
  if (!aligned16(src) || (reinterpret_cast<uintptr_t>(dst) & 7u))
    return fail(BELL_ERR_ALIGN, "bell_f32x_split_rows: src must be 16-byte and dst 8-byte aligned");
  if (int rc = require_sm100()) return rc;
  if (T == 0) return BELL_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  f32x_split_kernel<<<grid_for(T * (n / 4), 256), 256, 0, s>>>(src, ld_src, T, n, static_cast<__nv_bfloat16*>(dst),
                                                                ld_dst, col0);
  return check_launch("f32x_split_kernel");
}

// One fp32 Block-ELL linear, y = x W (+ residual), the same way: A = [x parts
// | residual parts] ([T, 3 in_f + 3 out_f] bf16; [T, 3 in_f] without the
// identity slots), w expanded with col_base = 0, part_cols = C and, for the
// residual, ident_base = 3 C, ident_stride = R.
size_t bell_f32x_linear_workspace_bytes(int64_t T, int32_t in_f, int32_t out_f, int32_t R, int32_t K6) {
  if (T < 0 || in_f < 1 || out_f < 1 || R < 1 || K6 < 1) return 0;
  const size_t la = 3 * size_t(in_f) + (K6 % 6 == 3 ? 3 * size_t(out_f) : 0);
  return up256(size_t(T) * la * 2) + up256(plan_layout(0, 0, 0, R, K6).total);
}

int bell_linear_f32x(const BellLinearDesc* d, void* workspace, void* stream) {
  if (!d) return fail(BELL_ERR_ARG, "descriptor is NULL");
  if (d->dtype != BELL_DTYPE_F32 || d->out_dtype != BELL_DTYPE_F32)
    return fail(BELL_ERR_DTYPE, "bell_linear_f32x: dtype and out_dtype must be BELL_DTYPE_F32");
  const BellEll& w = d->w;
  const int32_t B = w.B;
  if (B != 16 && B != 32 && B != 64 && B != 128)
    return fail(BELL_ERR_SHAPE, "bell_linear_f32x: tile size B must be 16, 32, 64 or 128");
  const bool ident = w.K % 6 == 3;
  if (w.R < 1 || w.K < 6 || (w.K % 6 != 0 && !ident))
    return fail(BELL_ERR_SHAPE, "bell_linear_f32x: expanded rows hold 6K slots (6K + 3 with the residual's)");
  const int32_t rest = w.C - (ident ? 3 * w.R : 0);  // 3 C column blocks of x parts
  if (rest < 3 || rest % 3)
    return fail(BELL_ERR_SHAPE, "bell_linear_f32x: the weight must be a bell_f32x_expand_ell output over [x parts"
                                " | residual parts]");
  if (d->add_residual && !ident)
    return fail(BELL_ERR_ARG, "bell_linear_f32x: add_residual needs a weight expanded with identity slots");
  if (d->residual_row_lo || d->residual_row_hi)
    return fail(BELL_ERR_ARG, "bell_linear_f32x: residual row ranges are a bf16 feature");
  if (d->T < 0) return fail(BELL_ERR_SHAPE, "T must be >= 0");
  if (d->T > 0 && (!d->x || !d->out || !workspace || (d->add_residual && !d->residual)))
    return fail(BELL_ERR_ARG, "x, out, workspace (and residual with add_residual) must be non-NULL");
  if (!aligned16(d->x) || !aligned16(d->out) || !aligned16(workspace) || (d->residual && !aligned16(d->residual)))
    return fail(BELL_ERR_ALIGN, "bell_linear_f32x: buffers must be 16-byte aligned");
  if (int rc = require_sm100()) return rc;
  if (d->T == 0) return BELL_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t T = d->T;
  const int32_t in_f = rest / 3 * B, out_f = w.R * B;
  const int64_t LA = int64_t(w.C) * B;
  __nv_bfloat16* A = static_cast<__nv_bfloat16*>(workspace);
  void* plan = static_cast<char*>(workspace) + up256(size_t(T) * size_t(LA) * 2);
  f32x_split_kernel<<<grid_for(T * (in_f / 4), 256), 256, 0, s>>>(static_cast<const float*>(d->x), in_f, T, in_f, A,
                                                                   LA, 0);
  if (int rc = check_launch("f32x_split_kernel")) return rc;
  if (ident) {  // the identity slots add A's residual region: the residual, or zeros
    const float* res = d->add_residual ? static_cast<const float*>(d->residual) : nullptr;
    f32x_split_kernel<<<grid_for(T * (out_f / 4), 256), 256, 0, s>>>(res, out_f, T, out_f, A, LA, 3 * int64_t(in_f));
    if (int rc = check_launch("f32x_split_kernel")) return rc;
  }
  BellLinearDesc L{};
  L.T = T;
  L.dtype = BELL_DTYPE_BF16;
  L.out_dtype = BELL_DTYPE_F32;
  L.max_ctas = d->max_ctas;
  L.x = A;
  L.out = d->out;
  L.plan = plan;
  L.w = w;
  L.status = d->status;
  return bell_linear_bf16(&L, s);
}

}  // extern "C"
