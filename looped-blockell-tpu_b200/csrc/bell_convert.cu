// bell_convert.cu — dense weight -> Block-ELL on the GPU.
//
// The reference builds a Block-ELL weight from a dense one by keeping, per
// block-row, the K tiles of largest Frobenius norm, with the kept columns in
// ascending order (looped_blockell/layers/block_ell.py:79-116: reshape to
// [R, C, B_in, B_out], norms, argsort descending, first K, sort).  A
// block-row is B consecutive dense rows, one contiguous stretch of memory.
// Three launches:
//   1. bell_block_norms_kernel streams the matrix once (all SMs), each thread
//      summing the squares of one 16-byte column group over the B rows of a
//      block-row; lanes that share a column block reduce with shuffles;
//   2. bell_ell_select_kernel, one CTA per block-row, ranks every column
//      block against the others (larger norm first, the lower column index
//      first on equal norms: a stable descending sort) and keeps ranks < K,
//      numbered in ascending column order;
//   3. bell_ell_copy_kernel, one CTA per kept tile, copies it into
//      values[r, k] in the requested layout.
// HBM traffic: the dense matrix once, the kept tiles once more (mostly from
// L2, the block-row having just been streamed), the values once written.
#include <string>

#include "bell_host.h"
#include "bell_ptx.cuh"

namespace bell {
namespace conv {

static constexpr int kThr = 256;
static constexpr int kMaxC = 2048;  // column blocks per row held in shared memory

template <typename T>
struct Elt;
template <>
struct Elt<__nv_bfloat16> {
  static constexpr int PER16 = 8;  // elements per 16 bytes
  __device__ static float sq_sum(const uint4& v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16x2(w[i]);
      s = fmaf(f.x, f.x, s);
      s = fmaf(f.y, f.y, s);
    }
    return s;
  }
};
template <>
struct Elt<float> {
  static constexpr int PER16 = 4;
  __device__ static float sq_sum(const uint4& v) {
    const float a = __uint_as_float(v.x), b = __uint_as_float(v.y), c = __uint_as_float(v.z),
                d = __uint_as_float(v.w);
    return fmaf(a, a, fmaf(b, b, fmaf(c, c, d * d)));
  }
};

// Squared Frobenius norms: CTA (seg, r) sums the squares of 16-byte column
// groups [seg*kThrN, (seg+1)*kThrN) of block-row r over its B dense rows;
// the lanes of one column block reduce with shuffles.  sq: [R, C].
static constexpr int kThrN = 128;

template <typename T, int B>
__global__ void __launch_bounds__(kThrN) bell_block_norms_kernel(const T* __restrict__ dense, int32_t C,
                                                                float* __restrict__ sq) {
  constexpr int P = Elt<T>::PER16;
  constexpr int GROUP = B / P;  // lanes per column block (8 / 16 / 32)
  static_assert(GROUP <= 32 && (32 % GROUP) == 0, "a column block's lanes share a warp");
  const int r = blockIdx.y;
  const int64_t in_f = int64_t(C) * B;
  const int64_t groups = in_f / P;
  const int64_t g = int64_t(blockIdx.x) * kThrN + threadIdx.x;
  float s = 0.f;
  if (g < groups) {
    const T* p = dense + int64_t(r) * B * in_f + g * P;
#pragma unroll 8
    for (int i = 0; i < B; ++i) s += Elt<T>::sq_sum(ld_global_nc_v4(p + int64_t(i) * in_f));
  }
#pragma unroll
  for (int o = GROUP / 2; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o, GROUP);
  if (g < groups && (threadIdx.x % GROUP) == 0) sq[int64_t(r) * C + g / GROUP] = s;
}

// One CTA per block-row r: rank the C squared norms (larger first, the lower
// column first on equal norms: a stable descending sort), keep ranks < K,
// numbered in ascending column order (cols[r, k]), and turn the row's squared
// norms into norms.
__global__ void __launch_bounds__(kThr) bell_ell_select_kernel(int32_t C, int32_t K, float* __restrict__ norms,
                                                              int32_t* __restrict__ cols) {
  __shared__ float sq[kMaxC];
  __shared__ int32_t keep[kMaxC];
  const int r = blockIdx.x;
  for (int c = threadIdx.x; c < C; c += kThr) sq[c] = norms[int64_t(r) * C + c];
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += kThr) {
    const float v = sq[c];
    int rank = 0;
    for (int j = 0; j < C; ++j) {
      const float u = sq[j];
      rank += (u > v) || (u == v && j < c);
    }
    keep[c] = rank < K;
    norms[int64_t(r) * C + c] = sqrtf(v);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += kThr) {
    if (!keep[c]) continue;
    int p = 0;
    for (int j = 0; j < c; ++j) p += keep[j];
    cols[int64_t(r) * K + p] = c;
  }
}

// CTA (k, r) copies kept tile (r, k) into values[r, k] in the requested layout
// ([B_in, B_out] is the transpose of the dense block, staged through shared
// memory 32 dense rows at a time; [B_out, B_in] a straight row copy).
template <typename T, int B>
__global__ void __launch_bounds__(kThr) bell_ell_copy_kernel(const T* __restrict__ dense, int32_t C, int32_t K,
                                                            int32_t out_in, const int32_t* __restrict__ cols,
                                                            T* __restrict__ values) {
  constexpr int P = Elt<T>::PER16;
  constexpr int GROUP = B / P;
  constexpr int TR = 32;
  __shared__ __align__(16) T tile[TR][B + 16 / sizeof(T)];
  const int k = blockIdx.x, r = blockIdx.y;
  const int64_t in_f = int64_t(C) * B;
  const int c = cols[int64_t(r) * K + k];
  T* dst = values + (int64_t(r) * K + k) * B * B;
  const T* src = dense + int64_t(r) * B * in_f + int64_t(c) * B;
  if (out_in) {
    for (int q = threadIdx.x; q < B * GROUP; q += kThr) {
      const int o = q / GROUP, part = q % GROUP;
      *reinterpret_cast<uint4*>(dst + o * B + part * P) = ld_global_nc_v4(src + int64_t(o) * in_f + part * P);
    }
    return;
  }
  for (int o0 = 0; o0 < B; o0 += TR) {
    for (int q = threadIdx.x; q < TR * GROUP; q += kThr) {
      const int o = q / GROUP, part = q % GROUP;
      *reinterpret_cast<uint4*>(&tile[o][part * P]) = ld_global_nc_v4(src + int64_t(o0 + o) * in_f + part * P);
    }
    __syncthreads();
    for (int q = threadIdx.x; q < TR * B; q += kThr) {
      const int i = q / TR, o = q % TR;
      dst[i * B + o0 + o] = tile[o][i];
    }
    __syncthreads();
  }
}

template <typename T, int B>
int launch_b(const BellDenseToEllDesc* d, cudaStream_t s) {
  const int R = d->out_features / B, C = d->in_features / B;
  const T* dense = static_cast<const T*>(d->dense);
  const int64_t groups = int64_t(d->in_features) / Elt<T>::PER16;
  dim3 grid_n(unsigned((groups + kThrN - 1) / kThrN), unsigned(R));
  bell_block_norms_kernel<T, B><<<grid_n, kThrN, 0, s>>>(dense, C, d->norms);
  if (int rc = check_launch("bell_block_norms_kernel")) return rc;
  bell_ell_select_kernel<<<R, kThr, 0, s>>>(C, d->K, d->norms, d->col_indices);
  if (int rc = check_launch("bell_ell_select_kernel")) return rc;
  bell_ell_copy_kernel<T, B><<<dim3(unsigned(d->K), unsigned(R)), kThr, 0, s>>>(
      dense, C, d->K, d->layout == BELL_TILE_OUT_IN, d->col_indices, static_cast<T*>(d->values));
  return check_launch("bell_ell_copy_kernel");
}

template <typename T>
int launch(const BellDenseToEllDesc* d, cudaStream_t s) {
  return d->B == 64 ? launch_b<T, 64>(d, s) : launch_b<T, 128>(d, s);
}

}  // namespace conv
}  // namespace bell

using namespace bell;

extern "C" {

int bell_dense_to_ell(const BellDenseToEllDesc* d, void* stream) {
  if (!d) return fail(BELL_ERR_ARG, "descriptor is NULL");
  if (d->dtype != BELL_DTYPE_BF16 && d->dtype != BELL_DTYPE_F32)
    return fail(BELL_ERR_DTYPE, "bell_dense_to_ell: dtype must be BELL_DTYPE_BF16 or BELL_DTYPE_F32");
  if (d->B != 64 && d->B != 128) return fail(BELL_ERR_SHAPE, "bell_dense_to_ell: tile size must be 64 or 128");
  if (d->out_features <= 0 || d->in_features <= 0 || d->out_features % d->B || d->in_features % d->B)
    return fail(BELL_ERR_SHAPE, "Dimensions (" + std::to_string(d->out_features) + ", " +
                                    std::to_string(d->in_features) + ") must be divisible by tile_size " +
                                    std::to_string(d->B));
  const int C = d->in_features / d->B;
  if (C > conv::kMaxC) return fail(BELL_ERR_SHAPE, "bell_dense_to_ell: more than 2048 column blocks");
  if (d->K < 1 || d->K > C) return fail(BELL_ERR_SHAPE, "bell_dense_to_ell: need 1 <= K <= C");
  if (d->layout != BELL_TILE_IN_OUT && d->layout != BELL_TILE_OUT_IN)
    return fail(BELL_ERR_ARG, "bell_dense_to_ell: unknown tile layout");
  if (!d->dense || !d->values || !d->col_indices || !d->norms)
    return fail(BELL_ERR_ARG, "bell_dense_to_ell: NULL pointer");
  if (d->out_features / d->B > 65535) return fail(BELL_ERR_SHAPE, "bell_dense_to_ell: more than 65535 block-rows");
  if (d->K > 65535) return fail(BELL_ERR_SHAPE, "bell_dense_to_ell: K above 65535");
  if (!aligned16(d->dense) || !aligned16(d->values))
    return fail(BELL_ERR_ALIGN, "bell_dense_to_ell: dense and values must be 16-byte aligned");
  if (int rc = require_sm100()) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return d->dtype == BELL_DTYPE_BF16 ? conv::launch<__nv_bfloat16>(d, s) : conv::launch<float>(d, s);
}

}  // extern "C"
