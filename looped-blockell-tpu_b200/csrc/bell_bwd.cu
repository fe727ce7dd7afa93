// bell_bwd.cu — backward pieces of the Block-ELL SwiGLU (bf16).
//
// The reference backward (csrc/block_ell/swiglu_bwd.cu:7-35) runs five
// kernels: d_h = dy W_down, d_W_down, the SiLU*up backward, d_x = d_gate
// W_gate + d_up W_up (+ dy), d_W_gate / d_W_up.  Here:
//   * the two transposed products run on the forward linear kernels with a
//     transposed Block-ELL (same tile bytes read in the flipped layout; built
//     by the host layer), so they need no kernel of their own;
//   * bell_silu_mul_bwd_kernel: d_gate = d_h * up * silu'(gate),
//     d_up = d_h * silu(gate) (swiglu_bwd.cu:305-334);
//   * bell_sddmm_kernel: the tile gradients d_W[r, k] = a[:, c]^T b[:, r]
//     summed over tokens (swiglu_bwd.cu:13-14, 29-30), on tcgen05 with the
//     token dimension as the MMA K and both operands MN-major straight from
//     the row-major activations.  At tile size 64 a work unit is four slots
//     of one block-row in two accumulators (two slots' a features form
//     M = 128 against the row's 64 b features); at 128 it is two slots, the
//     row's b features M and the two slots' a features N = 256.  Either way
//     one b chunk serves every slot of the unit.  Tokens
//     run in ranges sized to stay in L2; each CTA takes an equal share of a
//     range and adds its fp32 partial tiles into the gradient with atomics.
#include <string>

#include "bell_bf16.cuh"
#include "bell_host.h"
#include "bell_ptx.cuh"

namespace bell {
namespace bwd {

// dh, g, u: [T, F] contiguous; dg, du: rows `ld` elements apart (so both can
// be the two halves of one [T, 2F] buffer).  f8 = F / 8; n8 = T * f8.
__global__ void __launch_bounds__(256) bell_silu_mul_bwd_kernel(const __nv_bfloat16* __restrict__ dh,
                                                                const __nv_bfloat16* __restrict__ g,
                                                                const __nv_bfloat16* __restrict__ u,
                                                                __nv_bfloat16* __restrict__ dg,
                                                                __nv_bfloat16* __restrict__ du, int64_t n8,
                                                                int64_t f8, int64_t ld) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
    const uint4 vh = ld_global_nc_v4(dh + i * 8), vg = ld_global_nc_v4(g + i * 8), vu = ld_global_nc_v4(u + i * 8);
    const uint32_t wh[4] = {vh.x, vh.y, vh.z, vh.w}, wg[4] = {vg.x, vg.y, vg.z, vg.w}, wu[4] = {vu.x, vu.y, vu.z, vu.w};
    uint32_t og[4], ou[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 h2 = unpack_bf16x2(wh[t]), g2 = unpack_bf16x2(wg[t]), u2 = unpack_bf16x2(wu[t]);
      float dg0, du0, dg1, du1;
      silu_mul_grad(h2.x, g2.x, u2.x, dg0, du0);
      silu_mul_grad(h2.y, g2.y, u2.y, dg1, du1);
      og[t] = pack_bf16x2(dg0, dg1);
      ou[t] = pack_bf16x2(du0, du1);
    }
    const int64_t row = i / f8, off = row * ld + (i - row * f8) * 8;
    st_global_v4(dg + off, og[0], og[1], og[2], og[3]);
    st_global_v4(du + off, ou[0], ou[1], ou[2], ou[3]);
  }
}

__global__ void __launch_bounds__(256) bell_f32_to_bf16_kernel(const float* __restrict__ src,
                                                               __nv_bfloat16* __restrict__ dst, int64_t n8) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
    const float4 a = *reinterpret_cast<const float4*>(src + i * 8);
    const float4 b = *reinterpret_cast<const float4*>(src + i * 8 + 4);
    st_global_v4(dst + i * 8, pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y),
                 pack_bf16x2(b.z, b.w));
  }
}

// ------------------------------------------------------------------ SDDMM

static constexpr int kTok = 64;   // tokens per stage (MMA K per stage)
static constexpr int kThr = 192;  // warp 0 producer, 1 MMA, 2-5 epilogue

// B = 64: a unit is four slots of one block-row in two accumulators; each
// accumulator's M is two slots' a features (2 x 64) against the row's 64 b
// features (N), so one b chunk serves four slots.  B = 128 (TR): a unit is
// two slots; M = the row's 128 b features, N = the two slots' a features
// (2 x 128).  Both operands are MN-major straight from the row-major
// activations: 64-token x 64-feature boxes, 128-byte swizzle, 64-feature
// groups 8 KB apart.
template <int B>
struct SCfg {
  static constexpr bool TR = B == 128;
  static constexpr int SLOTS = TR ? 2 : 4;
  static constexpr int NACC = TR ? 1 : 2;              // accumulators per unit
  static constexpr int SLOT_BYTES = TR ? 16384 : 8192; // one slot's a chunk
  static constexpr int A_BYTES = TR ? 16384 : 32768;   // B=64: four a slots; B=128: b
  static constexpr int B_BYTES = TR ? 32768 : 8192;    // B=64: b; B=128: two a slots
  static constexpr int STAGE = A_BYTES + B_BYTES;      // 40 / 48 KB
  static constexpr int N = TR ? 256 : 64;              // MMA N = accumulator columns
  static constexpr int NS = 196608 / STAGE;            // 4 / 4 stages
  static constexpr int SMEM = NS * STAGE + 1024 + 512;
  static constexpr int TMEM_COLS = 2 * NACC * N;       // double-buffered unit accumulators
  static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation");
};

struct SddmmParams {
  int64_t T;
  int32_t R, K, KP;          // rows, slots per row, slot groups per row (K / SLOTS, rounded up)
  int32_t C;                 // column blocks of a (a_cols / B)
  int32_t n_split;           // token ranges
  int64_t split_chunks;      // 64-token chunks per token range
  const int32_t* cols;       // [R, K]
  float* grad;               // [R, K, B, B] fp32, accumulated
  int32_t out_in;            // tile layout of grad: 0 [B_in, B_out], 1 [B_out, B_in]
  int32_t* status;
  uint64_t timeout_ns;
};

__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

struct Unit {
  int r;
  int k[4], c[4];    // slot and validated column (-1: absent or dead) of each slot of the unit
  int64_t ch0, ch1;  // 64-token chunks [ch0, ch1)
  bool any;
};

// a[i] with a runtime i, by selects (keeps the unit in registers)
__device__ __forceinline__ int pick4(const int (&a)[4], int i) {
  return i == 0 ? a[0] : i == 1 ? a[1] : i == 2 ? a[2] : a[3];
}

template <int SLOTS>
__device__ __forceinline__ Unit unit_of(int u, const SddmmParams& p) {
  Unit x;
  const int per = p.R * p.KP;
  const int s = u / per, rem = u - s * per;
  x.r = rem / p.KP;
  const int k0 = (rem - x.r * p.KP) * SLOTS;
  bool live = false;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int k = (j < SLOTS && k0 + j < p.K) ? k0 + j : -1;
    const int c = k >= 0 ? p.cols[size_t(x.r) * p.K + k] : -1;
    x.k[j] = k;
    x.c[j] = (c >= 0 && c < p.C) ? c : -1;
    live |= x.c[j] >= 0;
  }
  const int64_t total = (p.T + kTok - 1) / kTok;
  x.ch0 = int64_t(s) * p.split_chunks;
  x.ch1 = x.ch0 + p.split_chunks < total ? x.ch0 + p.split_chunks : total;
  x.any = live && x.ch1 > x.ch0;
  return x;
}

// Work split.  Token ranges (splits) run one after another; inside a split
// the units x chunks of the range are cut into equal contiguous shares, one
// per CTA, so every CTA streams the same tokens at the same time (the
// activation tiles are shared through L2) and no CTA waits on a longer share.
// A share may start or end inside a unit: each piece (segment) adds its
// partial tiles into the gradient like a whole unit.
struct SegIt {
  int s;
  int64_t L, L1, Ws;
};

__device__ __forceinline__ void seg_share(const SddmmParams& p, SegIt& it) {
  it.L = it.Ws * blockIdx.x / gridDim.x;
  it.L1 = it.Ws * (blockIdx.x + 1) / gridDim.x;
}

__device__ __forceinline__ SegIt seg_begin(const SddmmParams& p) {
  SegIt it;
  it.s = 0;
  it.Ws = int64_t(p.R) * p.KP * p.split_chunks;
  seg_share(p, it);
  return it;
}

// Next segment of this CTA: unit `x`, chunks [a0, a1) (empty when a1 <= a0),
// `head` when it starts at the unit's first chunk of split 0.  False at the end.
template <int SLOTS>
__device__ __forceinline__ bool seg_next(const SddmmParams& p, SegIt& it, Unit& x, int64_t& a0, int64_t& a1,
                                         bool& head) {
  while (it.L >= it.L1) {
    if (++it.s >= p.n_split) return false;
    seg_share(p, it);
  }
  const int ul = int(it.L / p.split_chunks);
  const int64_t c_lo = it.L - int64_t(ul) * p.split_chunks;
  const int64_t end = min(it.L1, int64_t(ul + 1) * p.split_chunks);
  const int64_t c_hi = end - int64_t(ul) * p.split_chunks;
  it.L = end;
  x = unit_of<SLOTS>(it.s * p.R * p.KP + ul, p);
  a0 = x.ch0 + c_lo;
  a1 = min(x.ch0 + c_hi, x.ch1);
  head = it.s == 0 && c_lo == 0;
  return true;
}

template <int B>
__global__ void __launch_bounds__(kThr, 1)
    bell_sddmm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                      const SddmmParams p) {
  using C = SCfg<B>;
  constexpr int SLOTS = C::SLOTS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::NS * C::STAGE);
  uint64_t* empty = full + C::NS;
  uint64_t* acc_full = empty + C::NS;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  Ctl ctl{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // -------------------------------------------- producer
      prefetch_tmap(&tm_a);
      prefetch_tmap(&tm_b);
      const uint64_t pol = policy_evict_normal();
      int stage = 0, last = -1;
      uint32_t phase = 0, last_phase = 0;
      bool alive = true;
      SegIt it = seg_begin(p);
      Unit x;
      int64_t a0, a1;
      bool head;
      while (alive && seg_next<SLOTS>(p, it, x, a0, a1, head)) {
        if (head) {  // once per unit: report indices outside [-1, C)
#pragma unroll
          for (int j = 0; j < SLOTS; ++j) {
            const int k = x.k[j];
            if (k >= 0) {
              const int c = p.cols[size_t(x.r) * p.K + k];
              if (c < -1 || c >= p.C) atomicOr(p.status, BELL_STATUS_COLIDX);
            }
          }
        }
        if (!x.any || a1 <= a0) continue;
        for (int64_t ch = a0; ch < a1; ++ch) {
          if (!mbar_wait(&empty[stage], phase ^ 1, ctl)) {
            alive = false;
            break;
          }
          uint8_t* st = smem + stage * C::STAGE;
          const int y = int(ch * kTok);
          uint32_t bytes = C::TR ? 16384 : 8192;  // the b chunk
#pragma unroll
          for (int j = 0; j < SLOTS; ++j) bytes += x.c[j] >= 0 ? C::SLOT_BYTES : 0;
          mbar_arrive_expect_tx(&full[stage], bytes);
          // a slots: B=64 -> A operand, 8 KB each; B=128 -> B operand, 16 KB each
          uint8_t* a_dst = st + (C::TR ? C::A_BYTES : 0);
          uint8_t* b_dst = st + (C::TR ? 0 : C::A_BYTES);
#pragma unroll
          for (int j = 0; j < SLOTS; ++j) {
            const int c = x.c[j];
            if (c < 0) continue;
#pragma unroll
            for (int h = 0; h < B / 64; ++h)
              tma_load_2d(a_dst + j * C::SLOT_BYTES + h * 8192, &tm_a, &full[stage], c * B + h * 64, y, pol);
          }
#pragma unroll
          for (int h = 0; h < B / 64; ++h)
            tma_load_2d(b_dst + h * 8192, &tm_b, &full[stage], x.r * B + h * 64, y, pol);
          last = stage;
          last_phase = phase;
          if (++stage == C::NS) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!alive && last >= 0) {  // error path: let the copies in flight land
        int st = last;
        uint32_t ph = last_phase;
        for (int i = 0; i < C::NS; ++i) {
          const uint32_t a = smem_u32(&full[st]);
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(a, ph) && globaltimer_ns() - t0 < 100000000ull) {
          }
          if (--st < 0) {
            st = C::NS - 1;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------- MMA issuer
    const bool leader = elect_one();
    constexpr uint32_t IDESC = idesc_bf16(128, C::N, true, true);
    const uint64_t a_desc0 = sdesc_sw128(smem_u32(smem), 8192, 1024);
    const uint64_t b_desc0 = sdesc_sw128(smem_u32(smem) + C::A_BYTES, 8192, 1024);
    int stage = 0, i = 0;
    uint32_t phase = 0;
    SegIt it = seg_begin(p);
    Unit x;
    int64_t a0, a1;
    bool head;
    while (seg_next<SLOTS>(p, it, x, a0, a1, head)) {
      if (!x.any || a1 <= a0) continue;
      const int buf = i & 1;
      const uint32_t use = uint32_t(i >> 1);
      ++i;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_empty[buf], (use & 1u) ^ 1u, ctl))) break;
      tc_fence_after();
      const uint32_t d = tmem + uint32_t(buf * C::NACC * C::N);
      bool ok = true;
      for (int64_t ch = a0; ch < a1; ++ch) {
        if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, ctl))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = a_desc0 + uint64_t(stage) * (C::STAGE >> 4);
        const uint64_t bd = b_desc0 + uint64_t(stage) * (C::STAGE >> 4);
        if (leader) {
#pragma unroll
          for (int ac = 0; ac < C::NACC; ++ac) {  // accumulator ac: slots 2ac, 2ac+1 (B=64)
#pragma unroll
            for (int kk = 0; kk < kTok / 16; ++kk)
              mma_bf16(d + uint32_t(ac * C::N), ad + uint64_t(ac) * (16384 >> 4) + kk * (2048 >> 4),
                       bd + kk * (2048 >> 4), IDESC, (ch > a0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == C::NS) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      if (leader) mma_commit(&acc_full[buf]);
      __syncwarp();
    }
    // every MMA has completed before TMEM is released
    if (leader) {
      mma_commit(drain);
      const uint32_t a = smem_u32(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(a, 0) && globaltimer_ns() - t0 < 100000000ull) {
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;  // accumulator row (TMEM lane)
    int i = 0;
    SegIt it = seg_begin(p);
    Unit x;
    int64_t a0, a1;
    bool head;
    while (seg_next<SLOTS>(p, it, x, a0, a1, head)) {
      if (!x.any || a1 <= a0) continue;
      const int buf = i & 1;
      const uint32_t use = uint32_t(i >> 1);
      ++i;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], use & 1u, ctl))) break;
      tc_fence_after();
      const uint32_t tb = tmem + (uint32_t(q * 32) << 16) + uint32_t(buf * C::NACC * C::N);
      if constexpr (!C::TR) {
        // B = 64: accumulator ac, row = a feature; rows 0-63 slot 2ac, 64-127
        // slot 2ac+1; columns = the row's 64 b (output) features
        const int fin = row & 63;
#pragma unroll 1
        for (int jj = 0; jj < C::NACC * (B / 32); ++jj) {
          const int ac = jj / (B / 32), j = jj % (B / 32);
          const int sl = 2 * ac + (q >= 2 ? 1 : 0);
          const int k = pick4(x.k, sl), c = pick4(x.c, sl);
          float* tile = p.grad + (size_t(x.r) * p.K + (k >= 0 ? k : 0)) * B * B;
          uint32_t v[32];
          tmem_ld32_sync(tb + uint32_t(ac * C::N) + j * 32, v);
          if (c < 0) continue;
          if (!p.out_in) {  // [B_in, B_out]: this row's 32 outputs are contiguous
            float* dst = tile + size_t(fin) * B + j * 32;
#pragma unroll
            for (int t = 0; t < 8; ++t)
              red_add_v4(dst + 4 * t, __uint_as_float(v[4 * t]), __uint_as_float(v[4 * t + 1]),
                         __uint_as_float(v[4 * t + 2]), __uint_as_float(v[4 * t + 3]));
          } else {  // [B_out, B_in]: consecutive lanes hit consecutive addresses
#pragma unroll
            for (int t = 0; t < 32; ++t) atomicAdd(tile + size_t(j * 32 + t) * B + fin, __uint_as_float(v[t]));
          }
        }
      } else {
        // B = 128: accumulator row = b (output) feature `row`; columns 0-127
        // slot k0's a (input) features, 128-255 slot k1's
#pragma unroll 1
        for (int sl = 0; sl < 2; ++sl) {
          const int k = pick4(x.k, sl);
          const int c = pick4(x.c, sl);
          if (c < 0) continue;  // warp-uniform
          float* tile = p.grad + (size_t(x.r) * p.K + k) * B * B;
#pragma unroll 1
          for (int j = 0; j < B / 32; ++j) {
            uint32_t v[32];
            tmem_ld32_sync(tb + sl * B + j * 32, v);
            if (!p.out_in) {  // [B_in, B_out]: consecutive lanes hit consecutive addresses
#pragma unroll
              for (int t = 0; t < 32; ++t) atomicAdd(tile + size_t(j * 32 + t) * B + row, __uint_as_float(v[t]));
            } else {  // [B_out, B_in]: this row's 32 inputs are contiguous
              float* dst = tile + size_t(row) * B + j * 32;
#pragma unroll
              for (int t = 0; t < 8; ++t)
                red_add_v4(dst + 4 * t, __uint_as_float(v[4 * t]), __uint_as_float(v[4 * t + 1]),
                           __uint_as_float(v[4 * t + 2]), __uint_as_float(v[4 * t + 3]));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------- host

namespace {

int grid_for(int64_t n8, int sms) {
  const int64_t want = (n8 + 255) / 256;
  const int64_t cap = int64_t(sms) * 8;
  return int(want < cap ? (want > 0 ? want : 1) : cap);
}

template <int B>
int launch_sddmm(const BellSddmmDesc* d, int32_t* status, cudaStream_t s, int sms) {
  using C = SCfg<B>;
  CUtensorMap ma, mb;
  if (int rc = make_map_2d(&ma, d->a, MapType::BF16, uint64_t(d->C) * B, uint64_t(d->T), uint64_t(d->lda) * 2, 64,
                           kTok, Swz::B128))
    return rc;
  if (int rc = make_map_2d(&mb, d->b, MapType::BF16, uint64_t(d->R) * B, uint64_t(d->T), uint64_t(d->ldb) * 2, 64,
                           kTok, Swz::B128))
    return rc;
  SddmmParams p{};
  p.T = d->T;
  p.R = d->R;
  p.K = d->K;
  p.KP = (d->K + C::SLOTS - 1) / C::SLOTS;
  p.C = d->C;
  const int64_t chunks = (d->T + kTok - 1) / kTok;
  const int64_t per = int64_t(p.R) * p.KP;
  // token ranges whose operands (a and b rows, bf16) fit in ~96 MB of the
  // 126 MB L2, so every unit of the range re-reads them from L2; 16..128
  // chunks (1024..8192 tokens) keep each CTA's partial-tile additions small
  // next to its loads
  const int64_t row_bytes = 2 * (int64_t(d->C) + d->R) * B;
  int64_t range = (int64_t(96) << 20) / (row_bytes * kTok);
  range = range < 16 ? 16 : (range > 128 ? 128 : range);
  p.split_chunks = chunks < range ? chunks : range;
  p.n_split = int32_t((chunks + p.split_chunks - 1) / p.split_chunks);
  p.cols = d->col_indices;
  p.grad = d->grad;
  p.out_in = d->layout == BELL_TILE_OUT_IN;
  p.status = status;
  p.timeout_ns = wait_budget_ns();
  if (per * p.n_split > INT32_MAX) return fail(BELL_ERR_SHAPE, "bell_sddmm_bf16: too many work units");
  auto kern = bell_sddmm_kernel<B>;
  if (int rc = set_smem(reinterpret_cast<const void*>(kern), C::SMEM)) return rc;
  const int64_t share = per * p.split_chunks;  // chunk-steps of one range
  const int grid = int(share < sms ? share : sms);
  kern<<<grid, kThr, C::SMEM, s>>>(ma, mb, p);
  return check_launch("bell_sddmm_kernel");
}

}  // namespace
}  // namespace bwd
}  // namespace bell

using namespace bell;
using namespace bell::bwd;

extern "C" {

int bell_silu_mul_bwd_bf16(int64_t T, int32_t d_ff, const void* d_h, const void* gate_pre, const void* up_out,
                           void* d_gate, void* d_up, int64_t ld_out, void* stream) {
  if (!d_h || !gate_pre || !up_out || !d_gate || !d_up) return fail(BELL_ERR_ARG, "bell_silu_mul_bwd_bf16: NULL pointer");
  if (T < 0 || d_ff <= 0 || d_ff % 8 != 0 || ld_out < d_ff || ld_out % 8 != 0)
    return fail(BELL_ERR_SHAPE, "bell_silu_mul_bwd_bf16: need T >= 0, d_ff % 8 == 0, ld_out >= d_ff, ld_out % 8 == 0");
  if (!aligned16(d_h) || !aligned16(gate_pre) || !aligned16(up_out) || !aligned16(d_gate) || !aligned16(d_up))
    return fail(BELL_ERR_ALIGN, "bell_silu_mul_bwd_bf16: pointers must be 16-byte aligned");
  if (int rc = require_sm100()) return rc;
  if (T == 0) return BELL_OK;
  int sms = 0;
  if (int rc = device_sm_count(&sms)) return rc;
  const int64_t f8 = d_ff / 8, n8 = T * f8;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  bell_silu_mul_bwd_kernel<<<grid_for(n8, sms), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(d_h), static_cast<const __nv_bfloat16*>(gate_pre),
      static_cast<const __nv_bfloat16*>(up_out), static_cast<__nv_bfloat16*>(d_gate),
      static_cast<__nv_bfloat16*>(d_up), n8, f8, ld_out);
  return check_launch("bell_silu_mul_bwd_kernel");
}

int bell_sddmm_bf16(const BellSddmmDesc* d, void* stream) {
  if (!d) return fail(BELL_ERR_ARG, "bell_sddmm_bf16: NULL descriptor");
  if (!d->col_indices || !d->grad || (d->T > 0 && (!d->a || !d->b)))
    return fail(BELL_ERR_ARG, "bell_sddmm_bf16: NULL pointer");
  if (d->B != 16 && d->B != 32 && d->B != 64 && d->B != 128)
    return fail(BELL_ERR_SHAPE, "bell_sddmm_bf16: tile size must be 16, 32, 64 or 128");
  if (d->T < 0 || d->R <= 0 || d->C <= 0 || d->K <= 0)
    return fail(BELL_ERR_SHAPE, "bell_sddmm_bf16: need T >= 0 and R, C, K > 0");
  if (d->T > INT32_MAX - 64) return fail(BELL_ERR_SHAPE, "bell_sddmm_bf16: T too large");
  if (d->lda < int64_t(d->C) * d->B || d->ldb < int64_t(d->R) * d->B)
    return fail(BELL_ERR_SHAPE, "bell_sddmm_bf16: row pitch smaller than the row");
  if (d->layout != BELL_TILE_IN_OUT && d->layout != BELL_TILE_OUT_IN)
    return fail(BELL_ERR_ARG, "bell_sddmm_bf16: unknown tile layout");
  if (!aligned16(d->grad) || (d->grad_bf16 && !aligned16(d->grad_bf16)))
    return fail(BELL_ERR_ALIGN, "bell_sddmm_bf16: gradient buffers must be 16-byte aligned");
  if (int rc = require_sm100()) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* status = d->status ? d->status : default_status_ptr();
  if (!status) return BELL_ERR_LAUNCH;
  int sms = 0;
  if (int rc = device_sm_count(&sms)) return rc;
  const size_t n = size_t(d->R) * d->K * d->B * d->B;
  if (!d->accumulate) {
    cudaError_t e = cudaMemsetAsync(d->grad, 0, n * sizeof(float), s);
    if (e != cudaSuccess) return fail(BELL_ERR_LAUNCH, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  }
  if (d->T > 0) {
    const int rc = d->B < 64     ? launch_sddmm_ffma(d, false, status, s)
                   : d->B == 64 ? launch_sddmm<64>(d, status, s, sms)
                                : launch_sddmm<128>(d, status, s, sms);
    if (rc) return rc;
  }
  if (d->grad_bf16) {
    const int64_t n8 = int64_t(n / 8);
    bell_f32_to_bf16_kernel<<<grid_for(n8, sms), 256, 0, s>>>(d->grad, static_cast<__nv_bfloat16*>(d->grad_bf16), n8);
    return check_launch("bell_f32_to_bf16_kernel");
  }
  return BELL_OK;
}

int bell_sddmm_f32(const BellSddmmDesc* d, void* stream) {
  if (!d) return fail(BELL_ERR_ARG, "bell_sddmm_f32: NULL descriptor");
  if (!d->col_indices || !d->grad || (d->T > 0 && (!d->a || !d->b)))
    return fail(BELL_ERR_ARG, "bell_sddmm_f32: NULL pointer");
  if (d->grad_bf16) return fail(BELL_ERR_ARG, "bell_sddmm_f32: grad_bf16 must be NULL (the gradient is fp32)");
  if (d->B != 16 && d->B != 32 && d->B != 64 && d->B != 128)
    return fail(BELL_ERR_SHAPE, "bell_sddmm_f32: tile size must be 16, 32, 64 or 128");
  if (d->T < 0 || d->R <= 0 || d->C <= 0 || d->K <= 0)
    return fail(BELL_ERR_SHAPE, "bell_sddmm_f32: need T >= 0 and R, C, K > 0");
  if (d->lda < int64_t(d->C) * d->B || d->ldb < int64_t(d->R) * d->B)
    return fail(BELL_ERR_SHAPE, "bell_sddmm_f32: row pitch smaller than the row");
  if (d->layout != BELL_TILE_IN_OUT && d->layout != BELL_TILE_OUT_IN)
    return fail(BELL_ERR_ARG, "bell_sddmm_f32: unknown tile layout");
  if (!aligned16(d->grad)) return fail(BELL_ERR_ALIGN, "bell_sddmm_f32: gradient buffer must be 16-byte aligned");
  if (int rc = require_sm100()) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* status = d->status ? d->status : default_status_ptr();
  if (!status) return BELL_ERR_LAUNCH;
  if (!d->accumulate) {
    const size_t n = size_t(d->R) * d->K * d->B * d->B;
    cudaError_t e = cudaMemsetAsync(d->grad, 0, n * sizeof(float), s);
    if (e != cudaSuccess) return fail(BELL_ERR_LAUNCH, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  }
  if (d->T == 0) return BELL_OK;
  return launch_sddmm_ffma(d, true, status, s);
}

}  // extern "C"
