// bell_bf16_t.cu — feature-major bf16 Block-ELL kernels for B = 128.
//
// The token-major kernels (bell_bf16.cu) multiply an activation tile (M =
// tokens) by a weight tile (N = B_out = 128).  On B200 an N = 128 MMA runs at
// about half the rate of an N = 256 one, and with independent gate/up
// topologies most steps are N = 128.  These kernels compute the transposed
// product instead:  D^T[feature, token] = W^T[feature, k] x^T[k, token]
// with M = 128 output features of one block-row and N = 256 tokens, so every
// MMA is N = 256 whatever the topology.  The weight tile is the A operand
// (MN-major for [B_in, B_out] tiles, K-major for [B_out, B_in]) and the
// activation tile [256 tokens x 64 K] is the K-major B operand.
//
// TMEM holds D^T: lanes = features, columns = tokens.  Gate/up: gate in
// columns [0, 256), up in [256, 512) (single buffer); the epilogue copies
// its values into packed bf16 registers, releases TMEM, then stores while
// the next unit's MMAs run.  Linear (down): one 256-column accumulator,
// double buffered.
//
// Warps: 0 and 10 TMA producers (alternate stages), 1 TMEM owner + MMA
// issuer, 2-9 epilogue (two per TMEM lane quadrant, each owning 128 of the
// 256 tokens).
#include <string>

#include "bell_bf16.cuh"
#include "bell_host.h"
#include "bell_ptx.cuh"

namespace bell {
namespace fmaj {

static constexpr int B = 128;                  // features per block-row (MMA M)
static constexpr int TN = 256;                 // tokens per unit (MMA N)
static constexpr int X_BYTES = TN * kBK * 2;   // 32 KB activation chunk
static constexpr int W_BYTES = kBK * B * 2;    // 16 KB weight chunk
static constexpr int kThr = 352;               // 11 warps
static constexpr int kProd1 = 10;              // second producer warp

// SPLIT (gate/up): every plan step carries one weight tile (the plan is built
// without gate/up merging), so a stage is 48 KB and the ring 4 deep; fused
// stages (x + gate + up, 64 KB) allow only 3 but load x once for both.
template <bool GU, bool SPLIT = false>
struct FCfg {
  static constexpr bool TWO_W = GU && !SPLIT;
  static constexpr int STAGE = X_BYTES + W_BYTES * (TWO_W ? 2 : 1);  // 64 / 48 KB
  static constexpr int NS = TWO_W ? 3 : 4;
  static constexpr int NBUF = GU ? 1 : 2;
  // linear: a 128 x 128 bf16 identity tile (the residual is added by one more
  // MMA step, I x residual, instead of strided loads in the epilogue)
  static constexpr int ID_BYTES = GU ? 0 : B * B * 2;
  static constexpr int SMEM = NS * STAGE + ID_BYTES + 1024 + 512;
};

// Write the identity tile in the 128-byte-swizzled layout the weight chunks
// use: per 64-wide K chunk, two 64-column groups of 64 rows x 128 B, 16-byte
// chunks XOR-ed with (row & 7).  The identity is symmetric, so the bytes read
// the same whether the descriptor treats rows as K (MN-major) or as M.
__device__ __forceinline__ void fill_identity(uint8_t* id, int tid, int nthreads) {
  for (int q = tid; q < (B * B * 2) / 16; q += nthreads) {
    const int off = q * 16;
    const int kc = off / 16384, g = (off % 16384) / 8192, rem = off % 8192;
    const int k = rem / 128, pc = (rem % 128) / 16;
    const int c = pc ^ (k & 7);
    const int m0 = g * 64 + c * 8, kidx = kc * 64 + k;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    const int d = kidx - m0;
    if (d >= 0 && d < 8) w[d >> 1] = (d & 1) ? 0x3F800000u : 0x00003F80u;  // bf16 1.0 in the right half
    *reinterpret_cast<uint4*>(id + off) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

__device__ __forceinline__ void st_global_b16(void* p, uint16_t v) {
  asm volatile("st.global.b16 [%0], %1;" ::"l"(p), "h"(v) : "memory");
}

// Whether 256-token tile m gets the residual: the tile lies inside the
// residual row range (the host keeps the range on 256-row boundaries or T).
__device__ __forceinline__ bool unit_res(const Bf16Params& p, int m) {
  if (p.res_hi == 0) return true;
  const int64_t t0 = int64_t(m) * TN, t1 = t0 + TN < p.T ? t0 + TN : p.T;
  return t0 >= p.res_lo && t1 <= p.res_hi;
}

template <bool GU, bool W_MN, bool SPLIT>
__global__ void __launch_bounds__(kThr, 1)
    bell_bf16_fmajor_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w0,
                            const __grid_constant__ CUtensorMap tm_w1, const Bf16Params p) {
  using C = FCfg<GU, SPLIT>;
  // Split gate/up: the plan lists every gate step before the up steps, so the
  // gate accumulator (TMEM columns [0, 256)) is handed to the epilogue
  // (acc_full[0]) as soon as the last gate step is issued, and released by it
  // (acc_empty[0]) before the up accumulator is done (acc_full[1] /
  // acc_empty[1]).  The next unit's gate MMAs then start without waiting for
  // this unit's epilogue to read the up columns.
  constexpr bool STAG = GU && SPLIT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* id_tile = smem + C::NS * C::STAGE;  // linear only (ID_BYTES)
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::NS * C::STAGE + C::ID_BYTES);
  uint64_t* empty = full + C::NS;
  uint64_t* acc_full = empty + C::NS;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  const bool res_mma = !GU && p.add_residual;  // residual added as I x residual
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
      mbar_init(&acc_empty[b], 8);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (res_mma && warp >= 2 && warp < kProd1) {
    fill_identity(id_tile, threadIdx.x - 64, 256);
    fence_proxy_async_smem();  // generic writes -> visible to the tensor core
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_units = p.n_mtiles * p.R;  // n_mtiles counts 256-token tiles

  if (warp == 0 || warp == kProd1) {
    if (lane == 0) {  // ------------------------------------------- producers
      // Two producer warps take alternate stage uses (use g goes to warp
      // g & 1): one thread issuing every copy tops out near one stage per
      // ~450 cycles, about the MMA time of a stage.
      const int pid = warp == 0 ? 0 : 1;
      if (pid == 0) {
        prefetch_tmap(&tm_x);
        prefetch_tmap(&tm_w0);
        if (GU || res_mma) prefetch_tmap(&tm_w1);
      }
      const uint64_t pol_x = policy_evict_normal(), pol_w = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0, g = 0;
      int last_stage = -1;
      uint32_t last_phase = 0;
      bool alive = true;
      for (int u = blockIdx.x; u < n_units && alive; u += gridDim.x) {
        int m, r;
        unit_mr(u, p, m, r);
        const int n = p.counts[r] & 0xFFFF;
        const uint32_t* plan = p.plan + size_t(r) * p.S;
        const bool ures = res_mma && unit_res(p, m);
        const int n_uses = n * (B / kBK) + (ures ? B / kBK : 0);
        for (int j = 0; j < n_uses && alive; ++j, ++g) {
          if (int(g & 1u) == pid) {
            if (!mbar_wait(&empty[stage], phase ^ 1, ctl)) {
              alive = false;
              break;
            }
            uint8_t* st = smem + stage * C::STAGE;
            const int s = j >> 1, kc = j & 1;
            if (s < n) {
              const uint32_t e = plan[s];
              const int c = int(e & 0xFFFFu);
              const uint32_t k0 = (e >> 16) & 0xFFu, k1 = e >> 24;
              const bool has0 = k0 != kNone, has1 = GU && k1 != kNone;
              mbar_arrive_expect_tx(&full[stage], X_BYTES + (has0 ? W_BYTES : 0) + (has1 ? W_BYTES : 0));
              tma_load_2d(st, &tm_x, &full[stage], c * B + kc * kBK, m * TN, pol_x);
#pragma unroll
              for (int w = 0; w < 2; ++w) {
                if (w == 0 ? !has0 : !has1) continue;
                const CUtensorMap* map = w == 0 ? &tm_w0 : &tm_w1;
                const int tile = w == 0 ? r * p.K0 + int(k0) : r * p.K1 + int(k1);
                uint8_t* dst = st + X_BYTES + (C::TWO_W ? w : 0) * W_BYTES;
#pragma unroll
                for (int nb = 0; nb < 2; ++nb) {
                  if constexpr (W_MN)
                    tma_load_2d(dst + nb * 8192, map, &full[stage], nb * 64, tile * B + kc * kBK, pol_w);
                  else
                    tma_load_2d(dst + nb * 8192, map, &full[stage], kc * kBK, tile * B + nb * 64, pol_w);
                }
              }
            } else {
              // residual columns of this block-row (tm_w1 maps the residual for linear)
              mbar_arrive_expect_tx(&full[stage], X_BYTES);
              tma_load_2d(st, &tm_w1, &full[stage], r * B + kc * kBK, m * TN, pol_x);
            }
            last_stage = stage;
            last_phase = phase;
          }
          if (++stage == C::NS) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!alive && last_stage >= 0) {
        // error path: let this warp's copies in flight land before the CTA exits
        // (a stage use newer than the last one issued here belongs to the other
        // producer; walking back over NS uses covers every copy still pending)
        int st = last_stage;
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
    if (lane == 0) {  // ----------------------------------------- MMA issuer
      constexpr uint32_t IDESC = idesc_bf16(B, TN, W_MN, false);
      constexpr uint64_t kAStep = W_MN ? (2048 >> 4) : (32 >> 4);  // weight tile: K step of 16
      const uint64_t x_desc0 = sdesc_sw128(smem_u32(smem), 16, 1024);
      const uint64_t w_desc0 = W_MN ? sdesc_sw128(smem_u32(smem) + X_BYTES, 8192, 1024)
                                    : sdesc_sw128(smem_u32(smem) + X_BYTES, 16, 1024);
      const uint64_t id_desc0 = W_MN ? sdesc_sw128(smem_u32(id_tile), 8192, 1024)
                                     : sdesc_sw128(smem_u32(id_tile), 16, 1024);
      int stage = 0, i = 0;
      uint32_t phase = 0;
      bool alive = true, issued_any = false;
      for (int u = blockIdx.x; u < n_units && alive; u += gridDim.x, ++i) {
        int m, r;
        unit_mr(u, p, m, r);
        const bool ures = res_mma && unit_res(p, m);
        const int buf = C::NBUF == 2 ? (i & 1) : 0;
        const uint32_t use = C::NBUF == 2 ? uint32_t(i >> 1) : uint32_t(i);
        if (!mbar_wait(&acc_empty[buf], (use & 1u) ^ 1u, ctl)) break;
        tc_fence_after();
        const uint32_t d0 = tmem + uint32_t(buf * TN), d1 = tmem + 256u;
        const int n = p.counts[r] & 0xFFFF;
        const uint32_t* plan = p.plan + size_t(r) * p.S;
        uint32_t init0 = 0, init1 = 0;
        bool up_ready = !STAG;  // staggered: the up columns are waited for at the first up step
        for (int s = 0; s < n && alive; ++s) {
          const uint32_t e = plan[s];
          const bool has0 = ((e >> 16) & 0xFFu) != kNone;
          const bool has1 = GU && (e >> 24) != kNone;
          if (STAG && has1 && !up_ready) {  // every gate step is in: hand the gate columns over
            mma_commit(&acc_full[0]);
            if (!mbar_wait(&acc_empty[1], (uint32_t(i) & 1u) ^ 1u, ctl)) {
              alive = false;
              break;
            }
            tc_fence_after();
            up_ready = true;
          }
          for (int kc = 0; kc < B / kBK; ++kc) {
            if (!mbar_wait(&full[stage], phase, ctl)) {
              alive = false;
              break;
            }
            tc_fence_after();
            const uint64_t xd = x_desc0 + uint64_t(stage) * (C::STAGE >> 4);
            const uint64_t wd0 = w_desc0 + uint64_t(stage) * (C::STAGE >> 4);
            if (has0) {
#pragma unroll
              for (int kk = 0; kk < kBK / 16; ++kk)
                mma_bf16(d0, wd0 + kk * kAStep, xd + 2 * kk, IDESC, kk > 0 ? 1u : init0);
            }
            if (has1) {
              const uint64_t wd1 = wd0 + (C::TWO_W ? (W_BYTES >> 4) : 0);
#pragma unroll
              for (int kk = 0; kk < kBK / 16; ++kk)
                mma_bf16(d1, wd1 + kk * kAStep, xd + 2 * kk, IDESC, kk > 0 ? 1u : init1);
            }
            issued_any = true;
            if (has0) init0 = 1;
            if (has1) init1 = 1;
            mma_commit(&empty[stage]);
            if (++stage == C::NS) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
        for (int kc = 0; ures && alive && kc < B / kBK; ++kc) {  // acc += I x residual
          if (!mbar_wait(&full[stage], phase, ctl)) {
            alive = false;
            break;
          }
          tc_fence_after();
          const uint64_t xd = x_desc0 + uint64_t(stage) * (C::STAGE >> 4);
          const uint64_t idd = id_desc0 + uint64_t(kc) * (16384 >> 4);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_bf16(d0, idd + kk * kAStep, xd + 2 * kk, IDESC, (kk > 0 || kc > 0) ? 1u : init0);
          issued_any = true;
          mma_commit(&empty[stage]);
          if (++stage == C::NS) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!alive) break;
        if (STAG && !up_ready) {  // a unit without up steps
          mma_commit(&acc_full[0]);
          if (!mbar_wait(&acc_empty[1], (uint32_t(i) & 1u) ^ 1u, ctl)) break;
          tc_fence_after();
        }
        mma_commit(&acc_full[STAG ? 1 : buf]);
      }
      if (!alive && issued_any) {
        mma_commit(drain);
        const uint32_t a = smem_u32(drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(a, 0) && globaltimer_ns() - t0 < 100000000ull) {
        }
      }
    }
  } else if (warp < kProd1) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3, half = (warp - 2) >> 2;
    int i = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++i) {
      int m, r;
      unit_mr(u, p, m, r);
      const int buf = C::NBUF == 2 ? (i & 1) : 0;
      const uint32_t use = C::NBUF == 2 ? uint32_t(i >> 1) : uint32_t(i);
      const bool got = mbar_wait(&acc_full[buf], use & 1u, ctl);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const int cw = p.counts[r];
      const bool any0 = ((cw >> 16) & 1) || (res_mma && unit_res(p, m)), any1 = (cw >> 17) & 1;
      const int64_t feat = int64_t(r) * B + q * 32 + lane;
      const int64_t tok0 = int64_t(m) * TN + half * 128;
      const uint32_t lane_base = uint32_t(q * 32) << 16;
      // gate/up outputs are written token by token down this lane's feature column: the address
      // steps one row per token, and a half tile wholly inside T skips the bounds checks (the
      // linear epilogue keeps per-element indexing, measured faster for the down projection)
      const bool whole = tok0 + 128 <= p.T;
      if constexpr (STAG) {
        auto store16 = [&](void* dst, int64_t tok_start, const uint32_t (&v)[16], bool live) {
          __nv_bfloat16* ptr = static_cast<__nv_bfloat16*>(dst) + tok_start * p.ld_out + feat;
#pragma unroll
          for (int t = 0; t < 16; ++t, ptr += p.ld_out)
            if (whole || tok_start + t < p.T)
              st_global_b16(ptr, __bfloat16_as_ushort(__float2bfloat16(live ? __uint_as_float(v[t]) : 0.f)));
        };
        // gate columns (already complete): SiLU(gate) of this feature's 128
        // tokens as bf16 pairs, then the columns go back to the issuer
        uint32_t hp[64];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint32_t g[16];
          tmem_ld16_sync(tmem + lane_base + uint32_t(half * 128 + j * 16), g);
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const float g0 = any0 ? __uint_as_float(g[2 * t]) : 0.f, g1 = any0 ? __uint_as_float(g[2 * t + 1]) : 0.f;
            hp[j * 8 + t] = pack_bf16x2(silu_fast(g0), silu_fast(g1));
          }
          if (p.gate_pre) store16(p.gate_pre, tok0 + j * 16, g, any0);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[0]);
        // up columns: h = SiLU(gate) * up, in place over the pairs
        if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[1], uint32_t(i) & 1u, ctl))) break;
        tc_fence_after();
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // 16 columns at a time: the 64 pairs stay live throughout
          uint32_t v[16];
          tmem_ld16_sync(tmem + lane_base + uint32_t(256 + half * 128 + j * 16), v);
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const float u0 = any1 ? __uint_as_float(v[2 * t]) : 0.f, u1 = any1 ? __uint_as_float(v[2 * t + 1]) : 0.f;
            const float2 sg = unpack_bf16x2(hp[j * 8 + t]);
            hp[j * 8 + t] = pack_bf16x2(sg.x * u0, sg.y * u1);
          }
          if (p.up_out) store16(p.up_out, tok0 + j * 16, v, any1);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[1]);  // TMEM free: stores below overlap the next unit
        __nv_bfloat16* hptr = static_cast<__nv_bfloat16*>(p.out) + tok0 * p.ld_out + feat;
#pragma unroll
        for (int t = 0; t < 64; ++t, hptr += 2 * p.ld_out) {
          if (whole || tok0 + 2 * t < p.T) st_global_b16(hptr, uint16_t(hp[t] & 0xFFFFu));
          if (whole || tok0 + 2 * t + 1 < p.T) st_global_b16(hptr + p.ld_out, uint16_t(hp[t] >> 16));
        }
      } else if constexpr (GU) {
        uint32_t hp[64];  // 128 tokens of this feature, bf16 pairs
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t g[32], v[32];
          tmem_ld32x2_sync(tmem + lane_base + uint32_t(half * 128 + j * 32), g,
                           tmem + lane_base + uint32_t(256 + half * 128 + j * 32), v);
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            const float g0 = any0 ? __uint_as_float(g[2 * t]) : 0.f, g1 = any0 ? __uint_as_float(g[2 * t + 1]) : 0.f;
            const float u0 = any1 ? __uint_as_float(v[2 * t]) : 0.f, u1 = any1 ? __uint_as_float(v[2 * t + 1]) : 0.f;
            hp[j * 16 + t] = pack_bf16x2(silu_fast(g0) * u0, silu_fast(g1) * u1);
          }
          if (p.gate_pre || p.up_out) {  // optional intermediates, one row pointer step per token
            const int64_t tj = tok0 + j * 32;
            const int64_t o0 = tj * p.ld_out + feat;
            __nv_bfloat16* gptr = static_cast<__nv_bfloat16*>(p.gate_pre) + o0;
            __nv_bfloat16* uptr = static_cast<__nv_bfloat16*>(p.up_out) + o0;
#pragma unroll
            for (int t = 0; t < 32; ++t, gptr += p.ld_out, uptr += p.ld_out) {
              if (!whole && tj + t >= p.T) continue;
              const float gv = any0 ? __uint_as_float(g[t]) : 0.f, uv = any1 ? __uint_as_float(v[t]) : 0.f;
              if (p.gate_pre) st_global_b16(gptr, __bfloat16_as_ushort(__float2bfloat16(gv)));
              if (p.up_out) st_global_b16(uptr, __bfloat16_as_ushort(__float2bfloat16(uv)));
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);  // TMEM free: stores below overlap the next unit
        __nv_bfloat16* hptr = static_cast<__nv_bfloat16*>(p.out) + tok0 * p.ld_out + feat;
#pragma unroll
        for (int t = 0; t < 64; ++t, hptr += 2 * p.ld_out) {
          if (whole || tok0 + 2 * t < p.T) st_global_b16(hptr, uint16_t(hp[t] & 0xFFFFu));
          if (whole || tok0 + 2 * t + 1 < p.T) st_global_b16(hptr + p.ld_out, uint16_t(hp[t] >> 16));
        }
      } else {
#pragma unroll 1
        for (int j = 0; j < 4; ++j) {
          uint32_t a[32];
          tmem_ld32_sync(tmem + lane_base + uint32_t(buf * TN + half * 128 + j * 32), a);
          // the residual (when requested) is already in the accumulator
          const int64_t tokj = tok0 + j * 32;
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            const int64_t tok = tokj + t;
            if (tok >= p.T) continue;
            const int64_t off = tok * p.ld_out + feat;
            const float y = any0 ? __uint_as_float(a[t]) : 0.f;
            if (p.out_f32) static_cast<float*>(p.out)[off] = y;
            else st_global_b16(static_cast<__nv_bfloat16*>(p.out) + off, __bfloat16_as_ushort(__float2bfloat16(y)));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <bool GU, bool W_MN, bool SPLIT = false>
static int launch(const CUtensorMap& a, const CUtensorMap& w0, const CUtensorMap& w1, const Bf16Params& p0,
                  cudaStream_t stream) {
  using C = FCfg<GU, SPLIT>;
  auto kern = bell_bf16_fmajor_kernel<GU, W_MN, SPLIT>;
  if (int rc = set_smem(reinterpret_cast<const void*>(kern), C::SMEM)) return rc;
  int sms = 0;
  if (int rc = device_sm_count(&sms)) return rc;
  Bf16Params p = p0;
  p.n_mtiles = int32_t((p.T + TN - 1) / TN);
  const int64_t units = int64_t(p.n_mtiles) * p.R;
  if (units == 0) return BELL_OK;
  kern<<<grid_size(units, sms, p.max_ctas), kThr, C::SMEM, stream>>>(a, w0, w1, p);
  return check_launch(GU ? "bell gate/up feature-major kernel" : "bell linear feature-major kernel");
}

}  // namespace fmaj

int fmajor_split_env() {
  static const int v = [] {
    const char* e = std::getenv("BELL_GU_SPLIT");
    return e ? (e[0] == '1' ? 1 : 0) : -1;
  }();
  return v;
}

int launch_fmajor(bool gate_up, bool w_mn, const CUtensorMap& a, const CUtensorMap& w0, const CUtensorMap& w1,
                  const Bf16Params& p, cudaStream_t s) {
  if (gate_up && p.split)
    return w_mn ? fmaj::launch<true, true, true>(a, w0, w1, p, s) : fmaj::launch<true, false, true>(a, w0, w1, p, s);
  if (gate_up) return w_mn ? fmaj::launch<true, true>(a, w0, w1, p, s) : fmaj::launch<true, false>(a, w0, w1, p, s);
  return w_mn ? fmaj::launch<false, true>(a, w0, w1, p, s) : fmaj::launch<false, false>(a, w0, w1, p, s);
}

}  // namespace bell
