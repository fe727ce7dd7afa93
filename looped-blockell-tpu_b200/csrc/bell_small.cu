// bell_small.cu — bf16 Block-ELL kernels for the small tiles of the reference
// model (B = 16 and 32).
//
// The reference's native op exists only for 16 x 16 tiles
// (csrc/block_ell/swiglu_fwd.cu:84, TILE = 16; schemas at
// csrc/block_ell/block_ell_ops.cpp:51-62 give [R_ff, K_g, 16, 16]) and its
// model default is tile_size = 16 (looped_blockell/config.py:63), so existing
// callers hand this library 16 x 16 (or 32 x 32) tiles.
//
// A work unit is one 128-token tile m times a group of G consecutive output
// block-rows, G * B (* 2 for gate|up) = 128 accumulator columns.  One plan
// step (column block c, gate and/or up slot) is one pipeline stage: the
// activation slice x[128 tokens, c*B : c*B+B] as a TMA box with a 32-byte (B
// = 16) or 64-byte (B = 32) swizzle — the K-major A operand — and the B x B
// weight tile(s) as the B operand (MN-major for [B_in, B_out] tiles, K-major
// for [B_out, B_in]).  Each stage is B/16 tcgen05.mma of M = 128, N = B,
// K = 16 into the block-row's columns of the unit's accumulator, fp32 in
// TMEM, double buffered (2 x 128 columns).
//
// Warps: 0, 6, 7 and 8 TMA producers (every fourth stage each; each walks the
// unit's plan steps from a two-unit-deep register prefetch), 1 TMEM owner +
// MMA issuer, 2-5 epilogue (one TMEM lane quadrant each, one token row per
// thread): SiLU(gate) * up, or + residual, with 16-byte stores.  A TMA copy
// costs its issuing thread ~225 cycles whatever its size and a step here is
// two or three small copies, so the copies are spread over four warps.
#include <string>

#include "bell_bf16.cuh"
#include "bell_host.h"
#include "bell_ptx.cuh"

namespace bell {
namespace small {

static constexpr int kM = 128;        // tokens per unit (MMA M)
static constexpr int kThr = 9 * 32;   // warps 0-8
static constexpr int kProds = 4;      // TMA producer warps: 0, 6, 7, 8
static constexpr int kProd1 = 6;      // first of the extra producer warps
static constexpr int kAcc = 128;      // accumulator columns per buffer

template <int B, bool GU>
struct SCfg {
  static constexpr int X_BYTES = kM * B * 2;  // activation slice (4 / 8 KB)
  static constexpr int W_BYTES = B * B * 2;   // one tile (512 B / 2 KB)
  static constexpr int STAGE = (X_BYTES + (GU ? 2 : 1) * W_BYTES + 1023) & ~1023;
  static constexpr int NS = B == 16 ? 16 : 12;
  static constexpr int G = kAcc / (B * (GU ? 2 : 1));  // block-rows per unit
  static constexpr int UP_COL = G * B;                  // up accumulator columns start here
  static constexpr int CTL = 1024;
  static constexpr int SMEM = NS * STAGE + 1024 + CTL;
  static_assert(G >= 1 && G <= 8, "rows per unit");
  // producer p takes the steps g with g % kProds == p, so it always uses the
  // same NS / kProds stages and waits on each one use behind (no parity aliasing)
  static_assert(NS % kProds == 0, "stages per producer");
};

// stage-info word: [0,8) row of the group, then flags
enum : uint32_t { kHas0 = 1u << 8, kHas1 = 1u << 9, kLast = 1u << 10 };

// Shared-memory matrix descriptor with the swizzle of a row of B bf16 values
// (32 bytes for B = 16, 64 bytes for B = 32).
template <int B>
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  if constexpr (B == 16) return sdesc_sw32(saddr, lbo, sbo);
  else return sdesc_sw64(saddr, lbo, sbo);
}

// Which work unit is the i-th of this CTA, as (token tile, first block-row).
__device__ __forceinline__ void unit_of(int u, int n_groups, int G, int& m, int& r0) {
  m = u / n_groups;
  r0 = (u - m * n_groups) * G;
}

// The plan steps of one unit, spread over a warp: lane l holds flat step l
// (rows of the group in order, each row's steps in plan order) as its plan
// entry and its row in the group.  `total` = steps of the unit.
struct UnitSteps {
  int total;
  uint32_t entry;
  int row;
};

// Counts of the unit's rows: lane j < G holds counts[r0 + j] & 0xFFFF.
__device__ __forceinline__ int load_counts(const Bf16Params& p, int r0, int G) {
  const int lane = threadIdx.x & 31;
  return (lane < G && r0 + lane < p.R) ? (p.counts[r0 + lane] & 0xFFFF) : 0;
}

// Given this lane's row count word `cnt_l` (lanes 0..G-1), issue the loads of
// steps [f0, f0 + 32) of the unit.
template <int G>
__device__ __forceinline__ UnitSteps load_steps(const Bf16Params& p, int r0, int cnt_l, int f0) {
  const int lane = threadIdx.x & 31;
  int n[G];
#pragma unroll
  for (int j = 0; j < G; ++j) n[j] = __shfl_sync(0xffffffffu, cnt_l, j);
  UnitSteps s;
  s.total = 0;
#pragma unroll
  for (int j = 0; j < G; ++j) s.total += n[j];
  const int f = f0 + lane;
  s.entry = 0u;
  s.row = 0;
  if (f < s.total) {
    // row = the j with end_{j-1} <= f < end_j (end_j = n[0] + ... + n[j]);
    // rows at or past R have n = 0, so row < R whenever f < total
    int start = 0, end = 0, row = 0;
#pragma unroll
    for (int j = 0; j < G; ++j) {
      end += n[j];
      if (f >= end) {
        start = end;
        row = j + 1;
      }
    }
    s.row = row;
    s.entry = p.plan[size_t(r0 + row) * size_t(p.S) + size_t(f - start)];
  }
  return s;
}

template <int B, bool GU, bool W_MN>
__global__ void __launch_bounds__(kThr, 1)
    bell_small_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w0,
                      const __grid_constant__ CUtensorMap tm_w1, const Bf16Params p) {
  using C = SCfg<B, GU>;
  constexpr int G = C::G;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ctl_base = smem + C::NS * C::STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(ctl_base);
  uint64_t* empty = full + C::NS;
  uint64_t* acc_full = empty + C::NS;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* stage_info = reinterpret_cast<uint32_t*>(ctl_base + 512);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  Ctl ctl{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kAcc);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_groups = (p.R + G - 1) / G;
  const int n_units = p.n_mtiles * n_groups;

  if (warp == 0 || warp >= kProd1) {
    // ---------------------------------------------------------- producers
    const int pid = warp == 0 ? 0 : warp - kProd1 + 1;
    if (pid == 0 && lane == 0) {
      prefetch_tmap(&tm_x);
      prefetch_tmap(&tm_w0);
      if (GU) prefetch_tmap(&tm_w1);
    }
    const uint64_t pol_x = policy_evict_normal(), pol_w = policy_evict_last();
    int stage = 0;
    uint32_t phase = 0, g = 0;
    int last_stage = -1;
    uint32_t last_phase = 0;
    bool alive = true;
    // two-deep prefetch: row counts two units ahead, first 32 steps one unit ahead
    int u = blockIdx.x;
    int m1, r1, m2, r2;
    unit_of(u, n_groups, G, m1, r1);
    int cnt_cur = u < n_units ? load_counts(p, r1, G) : 0;
    const int u2 = u + int(gridDim.x);
    unit_of(u2, n_groups, G, m2, r2);
    int cnt_next = u2 < n_units ? load_counts(p, r2, G) : 0;
    UnitSteps st_cur = load_steps<G>(p, r1, cnt_cur, 0);
    for (; u < n_units && alive; u += gridDim.x) {
      int m, r0;
      unit_of(u, n_groups, G, m, r0);
      const UnitSteps first = st_cur;
      const int cnt_this = cnt_cur;
      // prefetch: the next unit's first steps, the counts of the one after
      const int un = u + int(gridDim.x), unn = u + 2 * int(gridDim.x);
      int mn, rn, mnn, rnn;
      unit_of(un, n_groups, G, mn, rn);
      unit_of(unn, n_groups, G, mnn, rnn);
      st_cur = un < n_units ? load_steps<G>(p, rn, cnt_next, 0) : UnitSteps{0, 0u, 0};
      cnt_cur = cnt_next;
      cnt_next = unn < n_units ? load_counts(p, rnn, G) : 0;

      const int total = first.total;
      const int uses = total > 0 ? total : 1;  // a unit without live steps: one empty stage
      UnitSteps chunk = first;
      for (int f = 0; f < uses && alive; ++f, ++g) {
        if (f > 0 && (f & 31) == 0) chunk = load_steps<G>(p, r0, cnt_this, f);  // long units: next 32 steps
        const uint32_t e = __shfl_sync(0xffffffffu, chunk.entry, f & 31);
        const int j = __shfl_sync(0xffffffffu, chunk.row, f & 31);
        if (int(g % uint32_t(kProds)) == pid) {
          if (!__all_sync(0xffffffffu, mbar_wait(&empty[stage], phase ^ 1, ctl))) {
            alive = false;
            break;
          }
          if (elect_one()) {
            uint32_t info = uint32_t(j) | (f == uses - 1 ? kLast : 0u);
            if (f < total) {
              const int c = int(e & 0xFFFFu);
              const uint32_t k0 = (e >> 16) & 0xFFu, k1 = e >> 24;
              const bool has0 = k0 != kNone, has1 = GU && k1 != kNone;
              info |= (has0 ? kHas0 : 0u) | (has1 ? kHas1 : 0u);
              stage_info[stage] = info;
              uint8_t* sp = smem + stage * C::STAGE;
              const int r = r0 + j;
              mbar_arrive_expect_tx(&full[stage], C::X_BYTES + (has0 ? C::W_BYTES : 0) + (has1 ? C::W_BYTES : 0));
              tma_load_2d(sp, &tm_x, &full[stage], c * B, m * kM, pol_x);
              if (has0) tma_load_2d(sp + C::X_BYTES, &tm_w0, &full[stage], 0, (r * p.K0 + int(k0)) * B, pol_w);
              if (has1)
                tma_load_2d(sp + C::X_BYTES + C::W_BYTES, &tm_w1, &full[stage], 0, (r * p.K1 + int(k1)) * B, pol_w);
            } else {
              stage_info[stage] = info;  // empty stage: no copies
              mbar_arrive(&full[stage]);
            }
          }
          __syncwarp();
          last_stage = stage;
          last_phase = phase;
        }
        if (++stage == C::NS) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    if (!alive && last_stage >= 0 && lane == 0) {
      // error path: let this warp's copies in flight land before the CTA exits
      int s = last_stage;
      uint32_t ph = last_phase;
      for (int i = 0; i < C::NS; ++i) {
        const uint32_t a = smem_u32(&full[s]);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(a, ph) && globaltimer_ns() - t0 < 100000000ull) {
        }
        if (--s < 0) {
          s = C::NS - 1;
          ph ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------- MMA issuer
    constexpr uint32_t IDESC = idesc_bf16(kM, B, false, W_MN);
    constexpr uint32_t ROWB = B * 2;  // bytes of one swizzled row (x slice and weight tile)
    // weight tile K step of 16: 16 K-rows (MN-major) or 32 bytes of a row (K-major)
    constexpr uint64_t kWStep = W_MN ? ((16 * ROWB) >> 4) : (32 >> 4);
    const uint32_t s0 = smem_u32(smem);
    const uint64_t x_desc0 = sdesc<B>(s0, 16, 8 * ROWB);
    const uint64_t w_desc0 = W_MN ? sdesc<B>(s0 + C::X_BYTES, C::W_BYTES, 8 * ROWB)
                                  : sdesc<B>(s0 + C::X_BYTES, 16, 8 * ROWB);
    const bool leader = elect_one();
    int stage = 0, i = 0;
    uint32_t phase = 0;
    bool alive = true, issued_any = false;
    for (int u = blockIdx.x; u < n_units && alive; u += gridDim.x, ++i) {
      const int buf = i & 1;
      const uint32_t use = uint32_t(i >> 1);
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_empty[buf], (use & 1u) ^ 1u, ctl))) break;
      tc_fence_after();
      const uint32_t dacc = tmem + uint32_t(buf * kAcc);
      uint32_t init = 0;  // bit j: gate/linear accumulator of row j started; bit 8+j: up
      for (bool last = false; !last;) {
        if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, ctl))) {
          alive = false;
          break;
        }
        tc_fence_after();
        const uint32_t info = stage_info[stage];
        last = (info & kLast) != 0;
        const int j = int(info & 0xFFu);
        const bool has0 = (info & kHas0) != 0, has1 = GU && (info & kHas1) != 0;
        const uint64_t xd = x_desc0 + uint64_t(stage) * (C::STAGE >> 4);
        const uint64_t wd0 = w_desc0 + uint64_t(stage) * (C::STAGE >> 4);
        if (leader) {
          if (has0) {
            const uint32_t acc0 = (init >> j) & 1u;
#pragma unroll
            for (int kk = 0; kk < B / 16; ++kk)
              mma_bf16(dacc + uint32_t(j * B), xd + 2 * kk, wd0 + kk * kWStep, IDESC, kk > 0 ? 1u : acc0);
          }
          if (has1) {
            const uint32_t acc1 = (init >> (8 + j)) & 1u;
            const uint64_t wd1 = wd0 + (C::W_BYTES >> 4);
#pragma unroll
            for (int kk = 0; kk < B / 16; ++kk)
              mma_bf16(dacc + uint32_t(C::UP_COL + j * B), xd + 2 * kk, wd1 + kk * kWStep, IDESC, kk > 0 ? 1u : acc1);
          }
          mma_commit(&empty[stage]);
        }
        __syncwarp();
        if (has0) init |= 1u << j;
        if (has1) init |= 1u << (8 + j);
        issued_any = true;
        if (++stage == C::NS) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!alive) break;
      if (leader) mma_commit(&acc_full[buf]);
      __syncwarp();
    }
    if (leader && issued_any) {  // every MMA of this warp completes before TMEM is freed
      mma_commit(drain);
      const uint32_t a = smem_u32(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(a, 0) && globaltimer_ns() - t0 < 100000000ull) {
      }
    }
    __syncwarp();
  } else {
    // ----------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quadrant of this warp
    int i = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++i) {
      int m, r0;
      unit_of(u, n_groups, G, m, r0);
      const int buf = i & 1;
      const uint32_t use = uint32_t(i >> 1);
      // live-matrix bits of the group's rows (bit j: gate / linear, bit 8+j: up), read before the wait
      uint32_t live = 0;
#pragma unroll
      for (int j = 0; j < G; ++j) {
        if (r0 + j < p.R) {
          const int cw = p.counts[r0 + j];
          live |= (((cw >> 16) & 1) ? 1u << j : 0u) | (((cw >> 17) & 1) ? 1u << (8 + j) : 0u);
        }
      }
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], use & 1u, ctl))) break;
      tc_fence_after();
      const int64_t row = int64_t(m) * kM + q * 32 + lane;
      const bool row_ok = row < p.T;
      const uint32_t tbase = tmem + (uint32_t(q * 32) << 16) + uint32_t(buf * kAcc);
      if constexpr (GU) {
#pragma unroll 1
        for (int cc = 0; cc < C::UP_COL / 32; ++cc) {  // 32 features of the group per chunk
          uint32_t gv[32], uv[32];
          tmem_ld32x2_sync(tbase + uint32_t(cc * 32), gv, tbase + uint32_t(C::UP_COL + cc * 32), uv);
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            const int j = (cc * 32 + t) / B;
            if (!((live >> j) & 1u)) gv[t] = 0u;
            if (!((live >> (8 + j)) & 1u)) uv[t] = 0u;
          }
          if (row_ok) {
            const int64_t off = row * p.ld_out + int64_t(r0) * B + cc * 32;
#pragma unroll
            for (int v = 0; v < 4; ++v) {  // 16-byte groups of 8 features
              if (r0 + (cc * 32 + v * 8) / B >= p.R) continue;
              uint32_t hw[4];
#pragma unroll
              for (int z = 0; z < 4; ++z) {
                const int t = v * 8 + 2 * z;
                hw[z] = pack_bf16x2(silu_fast(__uint_as_float(gv[t])) * __uint_as_float(uv[t]),
                                    silu_fast(__uint_as_float(gv[t + 1])) * __uint_as_float(uv[t + 1]));
              }
              st_global_v4(static_cast<__nv_bfloat16*>(p.out) + off + v * 8, hw[0], hw[1], hw[2], hw[3]);
              if (p.gate_pre)
                st_global_v4(static_cast<__nv_bfloat16*>(p.gate_pre) + off + v * 8,
                             pack_bf16x2(__uint_as_float(gv[v * 8]), __uint_as_float(gv[v * 8 + 1])),
                             pack_bf16x2(__uint_as_float(gv[v * 8 + 2]), __uint_as_float(gv[v * 8 + 3])),
                             pack_bf16x2(__uint_as_float(gv[v * 8 + 4]), __uint_as_float(gv[v * 8 + 5])),
                             pack_bf16x2(__uint_as_float(gv[v * 8 + 6]), __uint_as_float(gv[v * 8 + 7])));
              if (p.up_out)
                st_global_v4(static_cast<__nv_bfloat16*>(p.up_out) + off + v * 8,
                             pack_bf16x2(__uint_as_float(uv[v * 8]), __uint_as_float(uv[v * 8 + 1])),
                             pack_bf16x2(__uint_as_float(uv[v * 8 + 2]), __uint_as_float(uv[v * 8 + 3])),
                             pack_bf16x2(__uint_as_float(uv[v * 8 + 4]), __uint_as_float(uv[v * 8 + 5])),
                             pack_bf16x2(__uint_as_float(uv[v * 8 + 6]), __uint_as_float(uv[v * 8 + 7])));
            }
          }
        }
      } else {
#pragma unroll 1
        for (int cc = 0; cc < kAcc / 32; ++cc) {
          uint32_t a[32];
          tmem_ld32_sync(tbase + uint32_t(cc * 32), a);
          float f[32];
#pragma unroll
          for (int t = 0; t < 32; ++t) f[t] = ((live >> ((cc * 32 + t) / B)) & 1u) ? __uint_as_float(a[t]) : 0.f;
          if (row_ok) {
            const int64_t off = row * p.ld_out + int64_t(r0) * B + cc * 32;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              if (r0 + (cc * 32 + v * 8) / B >= p.R) continue;
              float* fv = f + v * 8;
              if (p.add_residual && res_row(p, row)) {
                const uint4 rv = ld_global_v4(static_cast<const __nv_bfloat16*>(p.residual) + off + v * 8);
                const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                for (int z = 0; z < 4; ++z) {
                  const float2 x2 = unpack_bf16x2(rw[z]);
                  fv[2 * z] += x2.x;
                  fv[2 * z + 1] += x2.y;
                }
              }
              if (p.out_f32) {
                float* o = static_cast<float*>(p.out) + off + v * 8;
                st_global_v4(o, __float_as_uint(fv[0]), __float_as_uint(fv[1]), __float_as_uint(fv[2]),
                             __float_as_uint(fv[3]));
                st_global_v4(o + 4, __float_as_uint(fv[4]), __float_as_uint(fv[5]), __float_as_uint(fv[6]),
                             __float_as_uint(fv[7]));
              } else {
                st_global_v4(static_cast<__nv_bfloat16*>(p.out) + off + v * 8, pack_bf16x2(fv[0], fv[1]),
                             pack_bf16x2(fv[2], fv[3]), pack_bf16x2(fv[4], fv[5]), pack_bf16x2(fv[6], fv[7]));
              }
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
    tmem_dealloc(tmem, 2 * kAcc);
  }
}

template <int B, bool GU, bool W_MN>
static int launch_t(const CUtensorMap& x, const CUtensorMap& w0, const CUtensorMap& w1, const Bf16Params& p0,
                    cudaStream_t stream) {
  using C = SCfg<B, GU>;
  auto kern = bell_small_kernel<B, GU, W_MN>;
  if (int rc = set_smem(reinterpret_cast<const void*>(kern), C::SMEM)) return rc;
  int sms = 0;
  if (int rc = device_sm_count(&sms)) return rc;
  Bf16Params p = p0;
  p.n_mtiles = int32_t((p.T + kM - 1) / kM);
  const int64_t units = int64_t(p.n_mtiles) * ((p.R + C::G - 1) / C::G);
  if (units == 0) return BELL_OK;
  if (units > int64_t(INT32_MAX)) return fail(BELL_ERR_SHAPE, "too many work units");
  kern<<<grid_size(units, sms, p.max_ctas), kThr, C::SMEM, stream>>>(x, w0, w1, p);
  return check_launch(GU ? "bell gate/up small-tile kernel" : "bell linear small-tile kernel");
}

// ------------------------------------------------------ tile gradients
//
// grad[r, k] += a[:, c*B : c*B+B]^T b[:, r*B : r*B+B] over a token range on
// the CUDA cores, fp32 accumulation (the reference's
// block_ell_proj_backward_dw / block_ell_down_backward_dw,
// csrc/block_ell/swiglu_bwd.cu:13-14, 29-30).  Used where the tcgen05
// tile-gradient kernel does not apply: B = 16 / 32 in bf16 (a B x B product
// has no tensor-core shape; tcgen05 needs M >= 64), and fp32 operands at every
// tile size (the fp32 training path keeps full precision).  One CTA per
// (slot, token range) stages token slices of both operands in shared memory
// and each thread sums B*B/256 outputs, then adds them to the fp32 gradient
// with atomics.
static constexpr int kSdRange = 2048;  // tokens per CTA

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* f) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int z = 0; z < 4; ++z) {
    const float2 t = unpack_bf16x2(w[z]);
    f[2 * z] = t.x;
    f[2 * z + 1] = t.y;
  }
}
__device__ __forceinline__ void load8(const float* p, float* f) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
}

template <typename TIn, int B>
__global__ void __launch_bounds__(256) bell_sddmm_ffma_kernel(const TIn* __restrict__ a, const TIn* __restrict__ b,
                                                              int64_t T, int64_t lda, int64_t ldb, const int32_t* cols,
                                                              int C, int K, int out_in, float* grad,
                                                              int32_t* status) {
  constexpr int PER = B * B / 256;          // outputs per thread
  constexpr int TOK = B == 128 ? 32 : 64;   // tokens per staged slice
  __shared__ float as[TOK][B + 1];
  __shared__ float bs[TOK][B + 1];
  const int slot = blockIdx.x;
  const int r = slot / K;
  const int c = cols[slot];
  if (c < 0) return;  // dead slot: its gradient stays zero
  if (c >= C) {
    if (threadIdx.x == 0) atomicOr(status, BELL_STATUS_COLIDX);
    return;
  }
  const int64_t t0 = int64_t(blockIdx.y) * kSdRange;
  const int64_t t1 = t0 + kSdRange < T ? t0 + kSdRange : T;
  const int tid = threadIdx.x;
  const int i = (tid * PER) / B, j0 = (tid * PER) % B;  // this thread: row i, columns j0 .. j0+PER-1
  float acc[PER];
#pragma unroll
  for (int v = 0; v < PER; ++v) acc[v] = 0.f;
  constexpr int VEC = B / 8;  // 8-element groups per token row of one slice
  for (int64_t ts = t0; ts < t1; ts += TOK) {
    __syncthreads();
    for (int idx = tid; idx < TOK * VEC; idx += 256) {
      const int t = idx / VEC, v = idx % VEC;
      const int64_t tok = ts + t;
      float fa[8], fb[8];
      if (tok < t1) {
        load8(a + tok * lda + int64_t(c) * B + v * 8, fa);
        load8(b + tok * ldb + int64_t(r) * B + v * 8, fb);
      } else {
#pragma unroll
        for (int z = 0; z < 8; ++z) fa[z] = fb[z] = 0.f;
      }
#pragma unroll
      for (int z = 0; z < 8; ++z) {
        as[t][v * 8 + z] = fa[z];
        bs[t][v * 8 + z] = fb[z];
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int t = 0; t < TOK; ++t) {
      const float av = as[t][i];
#pragma unroll
      for (int v = 0; v < PER; ++v) acc[v] = fmaf(av, bs[t][j0 + v], acc[v]);
    }
  }
  float* g = grad + size_t(slot) * B * B;
#pragma unroll
  for (int v = 0; v < PER; ++v) {
    const int j = j0 + v;
    atomicAdd(g + (out_in ? j * B + i : i * B + j), acc[v]);
  }
}

}  // namespace small

// Tile gradients on the CUDA cores: bf16 operands at B = 16 / 32, or fp32
// operands (`f32`) at any tile size.  grad is already zeroed or accumulating.
int launch_sddmm_ffma(const BellSddmmDesc* d, bool f32, int32_t* status, cudaStream_t s) {
  const int vec = f32 ? 4 : 8;
  if ((d->lda % vec) || (d->ldb % vec) || !aligned16(d->a) || !aligned16(d->b))
    return fail(BELL_ERR_ALIGN, "tile gradients: a, b and their row pitches must be 16-byte aligned");
  const int64_t ranges = (d->T + small::kSdRange - 1) / small::kSdRange;
  if (ranges > 65535) return fail(BELL_ERR_SHAPE, "tile gradients: T too large for the CUDA-core kernel");
  if (int64_t(d->R) * d->K > INT32_MAX) return fail(BELL_ERR_SHAPE, "tile gradients: too many slots");
  const dim3 grid(unsigned(int64_t(d->R) * d->K), unsigned(ranges));
  const int oi = d->layout == BELL_TILE_OUT_IN ? 1 : 0;
#define BELL_SD(TY, BB)                                                                                      \
  small::bell_sddmm_ffma_kernel<TY, BB><<<grid, 256, 0, s>>>(static_cast<const TY*>(d->a),                  \
                                                             static_cast<const TY*>(d->b), d->T, d->lda,    \
                                                             d->ldb, d->col_indices, d->C, d->K, oi, d->grad, \
                                                             status)
  if (f32) {
    switch (d->B) {
      case 16: BELL_SD(float, 16); break;
      case 32: BELL_SD(float, 32); break;
      case 64: BELL_SD(float, 64); break;
      default: BELL_SD(float, 128); break;
    }
  } else if (d->B == 16) {
    BELL_SD(__nv_bfloat16, 16);
  } else {
    BELL_SD(__nv_bfloat16, 32);
  }
#undef BELL_SD
  return check_launch("bell_sddmm_ffma_kernel");
}

// Activation map for the small-tile kernels: boxes of B columns x 128 rows.
int make_small_x_map(CUtensorMap* m, const void* base, int64_t cols, int64_t rows, int B) {
  return make_map_2d(m, base, MapType::BF16, uint64_t(cols), uint64_t(rows), uint64_t(cols) * 2, uint32_t(B),
                     uint32_t(small::kM), B == 16 ? Swz::B32 : Swz::B64);
}

// Weight map for the small-tile kernels: one B x B tile per box.
int make_small_w_map(CUtensorMap* m, const BellEll& e) {
  const uint64_t rows = uint64_t(e.R) * uint64_t(e.K) * uint64_t(e.B);
  return make_map_2d(m, e.values, MapType::BF16, uint64_t(e.B), rows, uint64_t(e.B) * 2, uint32_t(e.B),
                     uint32_t(e.B), e.B == 16 ? Swz::B32 : Swz::B64);
}

int launch_small(bool gate_up, int B, bool w_mn, const CUtensorMap& x, const CUtensorMap& w0, const CUtensorMap& w1,
                 const Bf16Params& p, cudaStream_t s) {
  if (B == 16) {
    if (gate_up) return w_mn ? small::launch_t<16, true, true>(x, w0, w1, p, s) : small::launch_t<16, true, false>(x, w0, w1, p, s);
    return w_mn ? small::launch_t<16, false, true>(x, w0, w1, p, s) : small::launch_t<16, false, false>(x, w0, w1, p, s);
  }
  if (gate_up) return w_mn ? small::launch_t<32, true, true>(x, w0, w1, p, s) : small::launch_t<32, true, false>(x, w0, w1, p, s);
  return w_mn ? small::launch_t<32, false, true>(x, w0, w1, p, s) : small::launch_t<32, false, false>(x, w0, w1, p, s);
}

}  // namespace bell
