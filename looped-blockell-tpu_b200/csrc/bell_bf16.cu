// bell_bf16.cu — bf16 Block-ELL kernels for sm_100a.
//
//   * gate/up kernel: h = silu(x Wg) * (x Wu), the SiLU*up epilogue fused;
//     replaces block_ell_gate_up_silu_kernel (reference
//     csrc/block_ell/swiglu_fwd.cu:140-402).
//   * linear kernel: out = a W (+ residual); the down projection with its
//     residual epilogue, replacing block_ell_down_residual_kernel
//     (swiglu_fwd.cu:413-559), and the generic block_ell_matmul
//     (looped_blockell/layers/block_ell.py:149-182).
//
// The token-major kernels (tile sizes 64 and 128) are one phase of the
// engine in bell_engine.cuh: one persistent CTA per SM walks work units
// (128-token tile m, output block-row r), activation tiles [128 tokens x
// 64 K] (K-major) times weight tiles [64 K x B] (MN-major for [B_in,B_out]
// tiles, K-major for [B_out,B_in]).  The tile-size-128 default is the
// feature-major kernel (bell_bf16_t.cu); the CTA-pair kernel below is the
// other tile-size-128 variant.
#include <string>

#include "bell_bf16.cuh"
#include "bell_engine.cuh"
#include "bell_host.h"
#include "bell_ptx.cuh"
#include "bell_sched.cuh"

namespace bell {

// Token-major gate/up or linear kernel: one phase of the engine
// (bell_engine.cuh) over all units.
template <int B, bool GU, bool W_MN, bool SB = false>
__global__ void __launch_bounds__(eng::kThreads, 1)
    bell_bf16_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w0,
                     const __grid_constant__ CUtensorMap tm_w1, const Bf16Params p) {
  using G = eng::Geo<B, GU, SB>;
  extern __shared__ uint8_t smem_raw[];
  const eng::Smem s = eng::carve<G>(smem_raw);
  const uint32_t tmem = eng::setup<G>(s);
  // launched behind the previous kernel (programmatic dependent launch): the
  // set-up above touched only this CTA's shared memory and TMEM; every global
  // read and write comes after the predecessor has completed
  griddep_wait();
  griddep_launch();
  Ctl ctl{s.abort_flag, p.status, p.timeout_ns};
  const int warp = threadIdx.x >> 5;
  switch (eng::role_of(warp)) {
    case eng::kProducer: {
      const int pid = eng::producer_id(warp);
      if (pid == 0 && (threadIdx.x & 31) == 0) {
        prefetch_tmap(&tm_a);
        prefetch_tmap(&tm_w0);
        if (GU) prefetch_tmap(&tm_w1);
      }
      eng::ProdState st;
      if (!eng::produce<B, GU, W_MN, G>(p, &tm_a, &tm_w0, &tm_w1, s, st, 0, pid, ctl, policy_evict_normal(),
                                        policy_evict_last()))
        eng::producer_drain<G>(s, st, pid);
      break;
    }
    case eng::kIssuer: {
      const int k = warp == 1 ? 0 : 1;
      const bool leader = elect_one();
      eng::IssueState st;
      eng::issue<B, GU, W_MN, G>(p, s, tmem, st, 0, k, leader, ctl);
      eng::issuer_drain(s, k, leader);
      break;
    }
    case eng::kEpilogue:
      eng::epilogue<B, GU, G, SB>(p, s, tmem, 0, ctl, SB ? &tm_w1 : nullptr);  // SB: tm_w1 maps the output
      break;
  }
  eng::teardown<G>(tmem);
}

// ================================================================ 2-SM kernel
//
// B = 128 only.  A cluster of two CTAs works on one unit of 256 tokens x one
// output block-row; CTA c owns tokens [256m + 128c, +128).  The even CTA
// issues tcgen05.mma.cta_group::2 with M = 256: A comes from each CTA's own
// rows, B is split by N — on a shared gate|up step (N = 256) CTA 0 supplies
// the gate tile and CTA 1 the up tile; on an N = 128 step each CTA supplies
// 64 columns.  Per CTA, a stage is 16 KB of x plus at most 16 KB of weights,
// half the weight bytes of the single-CTA kernel, and the MMA reads half the
// B operand from each CTA's shared memory.  Both CTAs' TMA loads complete on
// the even CTA's `full` barrier; its MMA commits release the stage and the
// accumulator in both CTAs; both epilogues free an accumulator by arriving
// on the even CTA's `acc_empty` (count 8).
namespace pair {

static constexpr int B = 128;
static constexpr int A_BYTES = kBM * kBK * 2;  // 16 KB of this CTA's 128 token rows
static constexpr int W_BYTES = kBK * 128 * 2;  // 16 KB: one [64 K x 128 N] box pair
template <bool GU>
struct PCfg {
  static constexpr int STAGE = A_BYTES + W_BYTES;  // 32 KB (linear steps use half of W)
  static constexpr int NS = 7;
  static constexpr int ACC_COLS = GU ? 256 : 128;
  static constexpr int TMEM_COLS = 2 * ACC_COLS;
  static constexpr int SMEM = NS * STAGE + 1024 + 512;
};

template <bool GU, bool W_MN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    bell_bf16_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w0,
                          const __grid_constant__ CUtensorMap tm_w1, const Bf16Params p) {
  using C = PCfg<GU>;
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
  const uint32_t rank = cluster_ctarank();
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
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int pairs = gridDim.x >> 1, pid = blockIdx.x >> 1;
  const int n_units = p.n_mtiles * p.R;  // n_mtiles counts 256-token tiles here

  if (warp == 0) {
    if (lane == 0) {  // -------------------------------------------- producer
      prefetch_tmap(&tm_a);
      prefetch_tmap(&tm_w0);
      if (GU) prefetch_tmap(&tm_w1);
      const uint64_t pol_a = policy_evict_normal(), pol_w = policy_evict_last();
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      bool alive = true;
      for (int u = pid; u < n_units && alive; u += pairs) {
        int m, r;
        unit_mr(u, p, m, r);
        const int n = p.counts[r] & 0xFFFF;
        const uint32_t* plan = p.plan + size_t(r) * p.S;
        for (int s = 0; s < n && alive; ++s) {
          const uint32_t e = plan[s];
          const int c = int(e & 0xFFFFu);
          const uint32_t k0 = (e >> 16) & 0xFFu, k1 = e >> 24;
          const bool has0 = k0 != kNone, has1 = GU && k1 != kNone;
          const bool fused = has0 && has1;
          // both CTAs' bytes land on the even CTA's barrier
          const uint32_t step_bytes = 2 * A_BYTES + (fused ? 2 * W_BYTES : W_BYTES);
          for (int kc = 0; kc < B / kBK; ++kc) {
            if (!mbar_wait(&empty[stage], phase ^ 1, ctl)) {
              alive = false;
              break;
            }
            uint8_t* st = smem + stage * C::STAGE;
            const uint32_t bar0 = mapa_shared(smem_u32(&full[stage]), 0);
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], step_bytes);
            tma_load_2d_pair(st, &tm_a, bar0, c * B + kc * kBK, m * 256 + int(rank) * kBM, pol_a);
            // this CTA's half of B
            const CUtensorMap* wm;
            int tile, n_off, n_len;
            if (fused) {  // CTA 0: the whole gate tile, CTA 1: the whole up tile
              wm = rank == 0 ? &tm_w0 : &tm_w1;
              tile = rank == 0 ? r * p.K0 + int(k0) : r * p.K1 + int(k1);
              n_off = 0;
              n_len = 128;
            } else {  // one tile, columns split 64 / 64
              wm = has0 ? &tm_w0 : &tm_w1;
              tile = has0 ? r * p.K0 + int(k0) : r * p.K1 + int(k1);
              n_off = int(rank) * 64;
              n_len = 64;
            }
            if constexpr (W_MN) {
              for (int nb = 0; nb < n_len / 64; ++nb)
                tma_load_2d_pair(st + A_BYTES + nb * 8192, wm, bar0, n_off + nb * 64, tile * B + kc * kBK, pol_w);
            } else {
              // [B_out, B_in] tiles: rows are N; box of 64 K x 64 rows, twice for 128 rows
              for (int nb = 0; nb < n_len / 64; ++nb)
                tma_load_2d_pair(st + A_BYTES + nb * 8192, wm, bar0, kc * kBK, tile * B + n_off + nb * 64, pol_w);
            }
            ++issued;
            if (++stage == C::NS) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
      }
      (void)issued;
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {  // --------------------- MMA issuer (even CTA)
      constexpr uint32_t IDESC_N128 = idesc_bf16(256, 128, false, W_MN);
      constexpr uint32_t IDESC_N256 = idesc_bf16(256, 256, false, W_MN);
      // K step of 16 elements: +32 B inside a K-major row, +16 rows (2048 B) for MN-major B
      constexpr uint64_t kBStep = W_MN ? (2048 >> 4) : (32 >> 4);
      const uint64_t a_desc0 = sdesc_sw128(smem_u32(smem), 16, 1024);
      const uint64_t b_desc0 = W_MN ? sdesc_sw128(smem_u32(smem) + A_BYTES, 8192, 1024)
                                    : sdesc_sw128(smem_u32(smem) + A_BYTES, 16, 1024);
      const uint32_t empty_c0 = mapa_shared(smem_u32(&empty[0]), 0);
      const uint32_t empty_c1 = mapa_shared(smem_u32(&empty[0]), 1);
      int stage = 0, i = 0;
      uint32_t phase = 0;
      bool alive = true, issued_any = false;
      for (int u = pid; u < n_units && alive; u += pairs, ++i) {
        int m_unused, r;
        unit_mr(u, p, m_unused, r);
        const int buf = i & 1;
        const uint32_t use = uint32_t(i >> 1);
        if (!mbar_wait(&acc_empty[buf], (use & 1u) ^ 1u, ctl)) break;
        tc_fence_after();
        const uint32_t d0 = tmem + uint32_t(buf * C::ACC_COLS), d1 = d0 + 128;
        const int n = p.counts[r] & 0xFFFF;
        const uint32_t* plan = p.plan + size_t(r) * p.S;
        uint32_t init0 = 0, init1 = 0;
        for (int s = 0; s < n && alive; ++s) {
          const uint32_t e = plan[s];
          const bool has0 = ((e >> 16) & 0xFFu) != kNone;
          const bool has1 = GU && (e >> 24) != kNone;
          const bool fused = has0 && has1;
          for (int kc = 0; kc < B / kBK; ++kc) {
            if (!mbar_wait(&full[stage], phase, ctl)) {
              alive = false;
              break;
            }
            tc_fence_after();
            // Straight-line issue: descriptors are the stage-0 descriptors plus
            // constant offsets in their 16-byte start-address field.
            const uint64_t ad = a_desc0 + uint64_t(stage) * (C::STAGE >> 4);
            const uint64_t bd = b_desc0 + uint64_t(stage) * (C::STAGE >> 4);
            if (fused) {
              // The plan lists a row's shared steps before its single ones, so gate and
              // up are always in the same state here (one N=256 MMA spans both CTAs'
              // halves and cannot initialise one accumulator and add to the other).
              mma_bf16_pair(d0, ad, bd, IDESC_N256, init0);
              mma_bf16_pair(d0, ad + 2, bd + kBStep, IDESC_N256, 1u);
              mma_bf16_pair(d0, ad + 4, bd + 2 * kBStep, IDESC_N256, 1u);
              mma_bf16_pair(d0, ad + 6, bd + 3 * kBStep, IDESC_N256, 1u);
              if (init0 != init1) atomicOr(p.status, BELL_STATUS_INTERNAL);
            } else {
              const uint32_t dd = has0 ? d0 : d1;
              mma_bf16_pair(dd, ad, bd, IDESC_N128, has0 ? init0 : init1);
              mma_bf16_pair(dd, ad + 2, bd + kBStep, IDESC_N128, 1u);
              mma_bf16_pair(dd, ad + 4, bd + 2 * kBStep, IDESC_N128, 1u);
              mma_bf16_pair(dd, ad + 6, bd + 3 * kBStep, IDESC_N128, 1u);
            }
            issued_any = true;
            if (has0) init0 = 1;
            if (has1) init1 = 1;
            mma_commit_pair(empty_c0 + uint32_t(stage) * 8u);
            mma_commit_pair(empty_c1 + uint32_t(stage) * 8u);
            if (++stage == C::NS) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
        if (!alive) break;
        mma_commit_pair(mapa_shared(smem_u32(&acc_full[buf]), 0));
        mma_commit_pair(mapa_shared(smem_u32(&acc_full[buf]), 1));
      }
      if (!alive && issued_any) {
        mma_commit_pair(mapa_shared(smem_u32(drain), 0));
        const uint32_t a = smem_u32(drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(a, 0) && globaltimer_ns() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const uint64_t pol_out = policy_evict_first();
    int i = 0;
    for (int u = pid; u < n_units; u += pairs, ++i) {
      int m, r;
        unit_mr(u, p, m, r);
      const int buf = i & 1;
      const uint32_t use = uint32_t(i >> 1);
      const bool got = mbar_wait(&acc_full[buf], use & 1u, ctl);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const int cw = p.counts[r];
      const bool any0 = (cw >> 16) & 1, any1 = (cw >> 17) & 1;
      const int64_t row = int64_t(m) * 256 + int64_t(rank) * kBM + q * 32 + lane;
      const bool row_ok = row < p.T;
      const uint32_t tbase = tmem + (uint32_t(q * 32) << 16) + uint32_t(buf * C::ACC_COLS);
#pragma unroll 1
      for (int j = 0; j < B / 32; ++j) {
        if constexpr (GU) {
          uint32_t g[32], v[32];
          tmem_ld32x2_sync(tbase + j * 32, g, tbase + 128 + j * 32, v);
          uint32_t hp[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            const float g0 = any0 ? __uint_as_float(g[2 * t]) : 0.f, g1 = any0 ? __uint_as_float(g[2 * t + 1]) : 0.f;
            const float u0 = any1 ? __uint_as_float(v[2 * t]) : 0.f, u1 = any1 ? __uint_as_float(v[2 * t + 1]) : 0.f;
            hp[t] = pack_bf16x2(silu_fast(g0) * u0, silu_fast(g1) * u1);
          }
          if (row_ok) {
            const int64_t off = row * p.ld_out + int64_t(r) * B + j * 32;
            __nv_bfloat16* hrow = static_cast<__nv_bfloat16*>(p.out) + off;
#pragma unroll
            for (int t = 0; t < 4; ++t)
              st_global_v4_hint(hrow + t * 8, hp[4 * t], hp[4 * t + 1], hp[4 * t + 2], hp[4 * t + 3], pol_out);
            if (p.gate_pre) {
              __nv_bfloat16* grow = static_cast<__nv_bfloat16*>(p.gate_pre) + off;
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                uint32_t w[4];
#pragma unroll
                for (int z = 0; z < 4; ++z)
                  w[z] = any0 ? pack_bf16x2(__uint_as_float(g[8 * t + 2 * z]), __uint_as_float(g[8 * t + 2 * z + 1])) : 0u;
                st_global_v4(grow + t * 8, w[0], w[1], w[2], w[3]);
              }
            }
            if (p.up_out) {
              __nv_bfloat16* urow = static_cast<__nv_bfloat16*>(p.up_out) + off;
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                uint32_t w[4];
#pragma unroll
                for (int z = 0; z < 4; ++z)
                  w[z] = any1 ? pack_bf16x2(__uint_as_float(v[8 * t + 2 * z]), __uint_as_float(v[8 * t + 2 * z + 1])) : 0u;
                st_global_v4(urow + t * 8, w[0], w[1], w[2], w[3]);
              }
            }
          }
        } else {
          uint32_t a[32];
          tmem_ld32_sync(tbase + j * 32, a);
          float f[32];
#pragma unroll
          for (int t = 0; t < 32; ++t) f[t] = any0 ? __uint_as_float(a[t]) : 0.f;
          if (row_ok) {
            const int64_t off = row * p.ld_out + int64_t(r) * B + j * 32;
            if (p.add_residual && res_row(p, row)) {
              const __nv_bfloat16* rrow = static_cast<const __nv_bfloat16*>(p.residual) + off;
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                const uint4 rv = ld_global_v4(rrow + t * 8);
                const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                  const float2 x2 = unpack_bf16x2(rw[w]);
                  f[8 * t + 2 * w] += x2.x;
                  f[8 * t + 2 * w + 1] += x2.y;
                }
              }
            }
            if (p.out_f32) {
              float* orow = static_cast<float*>(p.out) + off;
#pragma unroll
              for (int t = 0; t < 8; ++t)
                st_global_v4_hint(orow + t * 4, __float_as_uint(f[4 * t]), __float_as_uint(f[4 * t + 1]),
                                  __float_as_uint(f[4 * t + 2]), __float_as_uint(f[4 * t + 3]), pol_out);
            } else {
              __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.out) + off;
#pragma unroll
              for (int t = 0; t < 4; ++t)
                st_global_v4_hint(orow + t * 8, pack_bf16x2(f[8 * t], f[8 * t + 1]), pack_bf16x2(f[8 * t + 2], f[8 * t + 3]),
                                  pack_bf16x2(f[8 * t + 4], f[8 * t + 5]), pack_bf16x2(f[8 * t + 6], f[8 * t + 7]),
                                  pol_out);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&acc_empty[buf]), 0));
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the pair may still touch its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::TMEM_COLS);
  }
}

}  // namespace pair

// ------------------------------------------------------------------- host

struct EllArgs {
  const BellEll* e;
  const char* name;
};

static int check_ell(const BellEll& e, const char* name) {
  if (!e.values || !e.col_indices) return fail(BELL_ERR_ARG, std::string(name) + ": NULL values/col_indices");
  if (e.R < 1 || e.C < 1 || e.K < 1) return fail(BELL_ERR_SHAPE, std::string(name) + ": R, C, K must be >= 1");
  if (e.B != 16 && e.B != 32 && e.B != 64 && e.B != 128)
    return fail(BELL_ERR_SHAPE, std::string(name) + ": tile size B must be 16, 32, 64 or 128");
  if (e.K > 254) return fail(BELL_ERR_SHAPE, std::string(name) + ": K must be <= 254");
  if (e.C > 65535) return fail(BELL_ERR_SHAPE, std::string(name) + ": C must be <= 65535");
  if (e.layout != BELL_TILE_IN_OUT && e.layout != BELL_TILE_OUT_IN)
    return fail(BELL_ERR_ARG, std::string(name) + ": unknown tile layout");
  if (!aligned16(e.values)) return fail(BELL_ERR_ALIGN, std::string(name) + ": values not 16-byte aligned");
  return BELL_OK;
}

// Weight tensor map: values [R, K, B, B] viewed as 2-D [R*K*B rows, B cols].
int make_w_map(CUtensorMap* m, const BellEll& e) {
  const uint64_t rows = uint64_t(e.R) * uint64_t(e.K) * uint64_t(e.B);
  // both layouts: boxes of 64 x 64 (128-byte rows); a [B_out, B_in] tile is
  // fetched as B/64 boxes of 64 N-rows
  return make_map_2d(m, e.values, MapType::BF16, e.B, rows, uint64_t(e.B) * 2, 64, 64, Swz::B128);
}

static int unit_band(bool gate_up, const Bf16Params& p, int B);

// B = 128 kernel family: 0 feature-major (default), 1 CTA-pair token-major,
// 2 single-CTA token-major (BELL_BF16_KERNEL=fmajor|pair|single).
static int b128_kernel() {
  static const int k = [] {
    const char* s = std::getenv("BELL_BF16_KERNEL");
    if (s && std::string(s) == "pair") return 1;
    if (s && std::string(s) == "single") return 2;
    const char* old = std::getenv("BELL_SINGLE_CTA");
    if (old && old[0] == '1') return 2;
    return 0;
  }();
  return k;
}

static bool pair_enabled() { return b128_kernel() == 1; }

// Rows of the activation TMA box: the feature-major kernels take 256 tokens.
static uint32_t a_box_rows(int B) { return (B == 128 && b128_kernel() == 0) ? 256u : uint32_t(kBM); }

template <bool GU, bool W_MN>
static int launch_pair(const CUtensorMap& a, const CUtensorMap& w0, const CUtensorMap& w1, const Bf16Params& p0,
                       cudaStream_t stream) {
  using C = pair::PCfg<GU>;
  auto kern = pair::bell_bf16_pair_kernel<GU, W_MN>;
  if (int rc = set_smem(reinterpret_cast<const void*>(kern), C::SMEM)) return rc;
  int sms = 0;
  if (int rc = device_sm_count(&sms)) return rc;
  Bf16Params p = p0;
  p.n_mtiles = int32_t((p.T + 255) / 256);
  p.band = unit_band(GU, p, 128);
  const int64_t units = int64_t(p.n_mtiles) * p.R;
  if (units == 0) return BELL_OK;
  // persistent grid: as many CTA pairs as can be resident at once
  static int max_pairs[2][2] = {{0, 0}, {0, 0}};
  int& mp = max_pairs[GU][W_MN];
  if (mp == 0) {
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(unsigned(sms & ~1));
    lc.blockDim = dim3(kThreads);
    lc.dynamicSmemBytes = C::SMEM;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, reinterpret_cast<const void*>(kern), &lc) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sms / 2;
    }
    mp = n < sms / 2 ? n : sms / 2;
  }
  int64_t pairs = units < mp ? units : mp;
  if (p.max_ctas > 0 && pairs > p.max_ctas / 2) pairs = p.max_ctas / 2 > 0 ? p.max_ctas / 2 : 1;
  kern<<<int(2 * pairs), kThreads, C::SMEM, stream>>>(a, w0, w1, p);
  return check_launch(GU ? "bell gate/up pair kernel" : "bell linear pair kernel");
}

// Rows per band of the unit order.  While the gate/up weight tiles of all
// block-rows fit in kBandBudget bytes (about 3/4 of the 126 MB L2), the order
// is unbanded: every token tile passes all block-rows, so its activation panel
// is read from DRAM once and the weights stay L2-resident.  Larger weight sets
// are cut into bands of that many bytes, each L2-resident while all token
// tiles pass.  Unbanded measured faster than 32-row bands on every benchmark
// shape (config 5, 67 MB of gate/up tiles: 26.0 against 27.5-28.0 ms, the
// power-capped clock higher with the DRAM re-reads gone; config 2: 0.682
// against 0.699 ms).  The down projection is unbanded.  BELL_BAND_ROWS
// overrides the gate/up band.
static constexpr int64_t kBandBudget = int64_t(96) << 20;
static int unit_band(bool gate_up, const Bf16Params& p, int B) {
  static const int env = [] {
    const char* s = std::getenv("BELL_BAND_ROWS");
    return s ? std::atoi(s) : 0;
  }();
  const int R = p.R;
  int band = R;
  if (gate_up) {
    const int64_t row_bytes = int64_t(p.K0 + p.K1) * B * B * 2;
    if (row_bytes > 0 && kBandBudget / row_bytes < R) band = int(kBandBudget / row_bytes);
    if (env > 0) band = env;
  }
  return band < 1 ? 1 : (band > R ? R : band);
}

template <int B, bool GU, bool W_MN, bool SB = false>
static int launch_bf16(const CUtensorMap& a, const CUtensorMap& w0, const CUtensorMap& w1, const Bf16Params& p0,
                       cudaStream_t stream) {
  using G = eng::Geo<B, GU, SB>;
  Bf16Params p = p0;
  p.band = unit_band(GU, p, B);
  auto kern = bell_bf16_kernel<B, GU, W_MN, SB>;
  if (int rc = set_smem(reinterpret_cast<const void*>(kern), G::SMEM_BYTES)) return rc;
  int sms = 0;
  if (int rc = device_sm_count(&sms)) return rc;
  const int64_t units = int64_t(p.n_mtiles) * p.R;
  if (units == 0) return BELL_OK;
  if (p.pdl) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(grid_size(units, sms, p.max_ctas)));
    cfg.blockDim = dim3(eng::kThreads);
    cfg.dynamicSmemBytes = G::SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a, w0, w1, p);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return fail(BELL_ERR_LAUNCH, std::string(GU ? "bell gate/up kernel: " : "bell linear kernel: ") +
                                       cudaGetErrorString(e));
    }
    return BELL_OK;
  }
  kern<<<grid_size(units, sms, p.max_ctas), eng::kThreads, G::SMEM_BYTES, stream>>>(a, w0, w1, p);
  return check_launch(GU ? "bell gate/up kernel" : "bell linear kernel");
}

template <bool GU>
static int dispatch_bf16(int B, int layout, const CUtensorMap& a, const CUtensorMap& w0, const CUtensorMap& w1,
                         const Bf16Params& p, cudaStream_t s) {
  const bool mn = layout == BELL_TILE_IN_OUT;
  if (B == 64) return mn ? launch_bf16<64, GU, true>(a, w0, w1, p, s) : launch_bf16<64, GU, false>(a, w0, w1, p, s);
  if (b128_kernel() == 0) {
    Bf16Params q = p;
    q.band = unit_band(GU, p, 128);
    if (!GU && p.add_residual) {  // the feature-major linear reads the residual with TMA
      CUtensorMap mr;
      if (int rc = make_map_2d(&mr, p.residual, MapType::BF16, uint64_t(p.ld_out), uint64_t(p.T),
                               uint64_t(p.ld_out) * 2, 64, 256, Swz::B128))
        return rc;
      return launch_fmajor(GU, mn, a, w0, mr, q, s);
    }
    return launch_fmajor(GU, mn, a, w0, w1, q, s);
  }
  if (pair_enabled()) return mn ? launch_pair<GU, true>(a, w0, w1, p, s) : launch_pair<GU, false>(a, w0, w1, p, s);
  return mn ? launch_bf16<128, GU, true>(a, w0, w1, p, s) : launch_bf16<128, GU, false>(a, w0, w1, p, s);
}

// Tile-schedule plan of one bf16 SwiGLU forward.  Gate/up slots on the same
// column share a step unless the B = 128 gate/up kernel runs one weight tile
// per step (feature-major split mode).
// Split mode (one weight tile per gate/up step, 48-KB stages, 4 deep) suits
// independent gate/up topologies; fused steps (x loaded once for both
// projections) suit shared ones.
static bool use_split(const BellFFNDesc* d) {
  if (d->gate.B != 128 || b128_kernel() != 0) return false;
  const int env = fmajor_split_env();
  if (env >= 0) return env == 1;
  const bool same = (d->gate.flags & BELL_ELL_SAME_COLS_AS_UP) || d->gate.col_indices == d->up.col_indices;
  return !same;
}

int launch_ffn_plan(const BellFFNDesc* d, int32_t* status, cudaStream_t s) {
  const int merge = use_split(d) ? 0 : 1;
  return launch_plan_ex(d->gate.col_indices, d->gate.K, d->up.col_indices, d->up.K, d->gate.R, d->gate.C,
                        d->down.col_indices, d->down.K, d->down.R, d->down.C, d->plan, status, s, merge);
}

int check_ffn(const BellFFNDesc* d, int dtype) {
  if (!d) return fail(BELL_ERR_ARG, "descriptor is NULL");
  if (d->dtype != dtype) return fail(BELL_ERR_DTYPE, "descriptor dtype does not match the entry point");
  if (d->T < 0) return fail(BELL_ERR_SHAPE, "T must be >= 0");
  if (int rc = check_ell(d->gate, "gate")) return rc;
  if (int rc = check_ell(d->up, "up")) return rc;
  if (int rc = check_ell(d->down, "down")) return rc;
  const BellEll &g = d->gate, &u = d->up, &w = d->down;
  if (g.B != u.B || g.B != w.B) return fail(BELL_ERR_SHAPE, "gate, up and down must share the tile size");
  if (g.R != u.R) return fail(BELL_ERR_SHAPE, "gate and up must have same R_ff");
  if (g.C != u.C) return fail(BELL_ERR_SHAPE, "gate and up must have the same number of input column blocks");
  if (g.layout != u.layout) return fail(BELL_ERR_SHAPE, "gate and up must use the same tile layout");
  if (int64_t(g.C) * g.B != d->d_model) return fail(BELL_ERR_SHAPE, "gate C*B inconsistent with d_model");
  if (int64_t(g.R) * g.B != d->d_ff) return fail(BELL_ERR_SHAPE, "gate R*B inconsistent with d_ff");
  if (int64_t(w.R) * w.B != d->d_model)
    return fail(BELL_ERR_SHAPE, "values_down R_model=" + std::to_string(w.R) + " inconsistent with d_model=" +
                                    std::to_string(d->d_model));
  if (int64_t(w.C) * w.B != d->d_ff) return fail(BELL_ERR_SHAPE, "down C*B inconsistent with d_ff");
  if (d->T > 0 && (!d->x || !d->h || !d->out || !d->plan))
    return fail(BELL_ERR_ARG, "x, h, out and plan must be non-NULL");
  if (!aligned16(d->x) || !aligned16(d->h) || !aligned16(d->out) || !aligned16(d->plan))
    return fail(BELL_ERR_ALIGN, "x, h, out and plan must be 16-byte aligned");
  if ((d->gate_pre && !aligned16(d->gate_pre)) || (d->up_out && !aligned16(d->up_out)) ||
      (d->residual && !aligned16(d->residual)))
    return fail(BELL_ERR_ALIGN, "optional buffers must be 16-byte aligned");
  if (d->T > (int64_t(1) << 31) - 256) return fail(BELL_ERR_SHAPE, "T too large");
  if (d->max_ctas < 0) return fail(BELL_ERR_ARG, "max_ctas must be >= 0");
  return BELL_OK;
}

int gate_up_bf16(const BellFFNDesc* d, int32_t* status, cudaStream_t s, bool pdl, int64_t ld_h, int64_t h_parts) {
  const BellEll &g = d->gate, &u = d->up;
  const bool sm = g.B < 64;  // small tiles: bell_small.cu
  CUtensorMap ma, mg, mu;
  if (sm) {
    if (int rc = make_small_x_map(&ma, d->x, d->d_model, d->T, g.B)) return rc;
    if (int rc = make_small_w_map(&mg, g)) return rc;
    if (int rc = make_small_w_map(&mu, u)) return rc;
  } else {
    if (int rc = make_map_2d(&ma, d->x, MapType::BF16, d->d_model, d->T, uint64_t(d->d_model) * 2, 64,
                             a_box_rows(g.B), Swz::B128))
      return rc;
    if (int rc = make_w_map(&mg, g)) return rc;
    if (int rc = make_w_map(&mu, u)) return rc;
  }
  PlanLayout L = plan_layout(g.R, g.K, u.K, d->down.R, d->down.K);
  Bf16Params p{};
  p.T = d->T;
  p.n_mtiles = int32_t((d->T + kBM - 1) / kBM);
  p.R = g.R;
  p.K0 = g.K;
  p.K1 = u.K;
  p.S = g.K + u.K;
  p.plan = reinterpret_cast<const uint32_t*>(static_cast<const char*>(d->plan) + L.gu_entries);
  p.counts = reinterpret_cast<const int32_t*>(static_cast<const char*>(d->plan) + L.gu_counts);
  p.out = d->h;
  p.ld_out = ld_h > 0 ? ld_h : d->d_ff;
  p.h_parts = h_parts;
  p.gate_pre = d->gate_pre;
  p.up_out = d->up_out;
  p.status = status;
  p.timeout_ns = wait_budget_ns();
  p.split = use_split(d) ? 1 : 0;  // must match the plan built by launch_ffn_plan
  p.max_ctas = d->max_ctas;
  if (sm) return launch_small(true, g.B, g.layout == BELL_TILE_IN_OUT, ma, mg, mu, p, s);
  p.pdl = pdl ? 1 : 0;
  return dispatch_bf16<true>(g.B, g.layout, ma, mg, mu, p, s);
}

int down_bf16(const BellFFNDesc* d, int32_t* status, cudaStream_t s, bool pdl) {
  const BellEll& w = d->down;
  const bool sm = w.B < 64;
  CUtensorMap ma, mw;
  if (sm) {
    if (int rc = make_small_x_map(&ma, d->h, d->d_ff, d->T, w.B)) return rc;
    if (int rc = make_small_w_map(&mw, w)) return rc;
  } else {
    if (int rc = make_map_2d(&ma, d->h, MapType::BF16, d->d_ff, d->T, uint64_t(d->d_ff) * 2, 64, a_box_rows(w.B),
                             Swz::B128))
      return rc;
    if (int rc = make_w_map(&mw, w)) return rc;
  }
  PlanLayout L = plan_layout(d->gate.R, d->gate.K, d->up.K, w.R, w.K);
  Bf16Params p{};
  p.T = d->T;
  p.n_mtiles = int32_t((d->T + kBM - 1) / kBM);
  p.R = w.R;
  p.K0 = w.K;
  p.K1 = 0;
  p.S = w.K;
  p.plan = reinterpret_cast<const uint32_t*>(static_cast<const char*>(d->plan) + L.d_entries);
  p.counts = reinterpret_cast<const int32_t*>(static_cast<const char*>(d->plan) + L.d_counts);
  p.out = d->out;
  p.ld_out = d->d_model;
  p.residual = d->residual ? d->residual : d->x;
  p.add_residual = d->add_residual ? 1 : 0;
  p.out_f32 = 0;
  p.max_ctas = d->max_ctas;
  p.status = status;
  p.timeout_ns = wait_budget_ns();
  p.pdl = pdl ? 1 : 0;
  if (sm) return launch_small(false, w.B, w.layout == BELL_TILE_IN_OUT, ma, mw, mw, p, s);
  return dispatch_bf16<false>(w.B, w.layout, ma, mw, mw, p, s);
}

}  // namespace bell

using namespace bell;

extern "C" {

int bell_swiglu_fwd_bf16(const BellFFNDesc* d, void* stream) {
  if (int rc = check_ffn(d, BELL_DTYPE_BF16)) return rc;
  if (int rc = require_sm100()) return rc;
  if (d->T == 0) return BELL_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* status = d->status ? d->status : default_status_ptr();
  if (!status) return BELL_ERR_LAUNCH;
  if (int rc = launch_ffn_plan(d, status, s)) return rc;
  if (int rc = gate_up_bf16(d, status, s)) return rc;
  return down_bf16(d, status, s);
}

int bell_gate_up_bf16(const BellFFNDesc* d, void* stream) {
  if (int rc = check_ffn(d, BELL_DTYPE_BF16)) return rc;
  if (int rc = require_sm100()) return rc;
  if (d->T == 0) return BELL_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* status = d->status ? d->status : default_status_ptr();
  if (!status) return BELL_ERR_LAUNCH;
  if (int rc = launch_ffn_plan(d, status, s)) return rc;
  return gate_up_bf16(d, status, s);
}

int bell_down_bf16(const BellFFNDesc* d, void* stream) {
  if (int rc = check_ffn(d, BELL_DTYPE_BF16)) return rc;
  if (int rc = require_sm100()) return rc;
  if (d->T == 0) return BELL_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* status = d->status ? d->status : default_status_ptr();
  if (!status) return BELL_ERR_LAUNCH;
  if (int rc = launch_ffn_plan(d, status, s)) return rc;
  return down_bf16(d, status, s);
}

int bell_linear_bf16(const BellLinearDesc* d, void* stream) {
  if (!d) return fail(BELL_ERR_ARG, "descriptor is NULL");
  if (d->dtype != BELL_DTYPE_BF16) return fail(BELL_ERR_DTYPE, "bell_linear_bf16: dtype must be BELL_DTYPE_BF16");
  if (d->out_dtype != BELL_DTYPE_BF16 && d->out_dtype != BELL_DTYPE_F32)
    return fail(BELL_ERR_DTYPE, "bell_linear_bf16: out_dtype must be BELL_DTYPE_BF16 or BELL_DTYPE_F32");
  if (int rc = check_ell(d->w, "weight")) return rc;
  if (d->T < 0) return fail(BELL_ERR_SHAPE, "T must be >= 0");
  if (d->T > 0 && (!d->x || !d->out || !d->plan)) return fail(BELL_ERR_ARG, "x, out and plan must be non-NULL");
  if (d->T > 0 && d->add_residual && !d->residual) return fail(BELL_ERR_ARG, "add_residual needs a residual pointer");
  if (!aligned16(d->x) || !aligned16(d->out) || !aligned16(d->plan) || (d->residual && !aligned16(d->residual)))
    return fail(BELL_ERR_ALIGN, "x, out, residual and plan must be 16-byte aligned");
  const bool res_all = d->residual_row_lo == 0 && d->residual_row_hi == 0;
  if (!res_all && (d->residual_row_lo < 0 || d->residual_row_hi < d->residual_row_lo || d->residual_row_hi > d->T))
    return fail(BELL_ERR_SHAPE, "residual rows must satisfy 0 <= lo <= hi <= T");
  if (!res_all && d->w.B == 128 && ((d->residual_row_lo % 256) || (d->residual_row_hi % 256 && d->residual_row_hi != d->T)))
    return fail(BELL_ERR_SHAPE, "at tile size 128 the residual rows must start and end on 256-row boundaries (or T)");
  if (d->max_ctas < 0) return fail(BELL_ERR_ARG, "max_ctas must be >= 0");
  if (int rc = require_sm100()) return rc;
  if (d->T == 0) return BELL_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* status = d->status ? d->status : default_status_ptr();
  if (!status) return BELL_ERR_LAUNCH;
  const BellEll& w = d->w;
  if (int rc = launch_plan(nullptr, 0, nullptr, 0, 0, 0, w.col_indices, w.K, w.R, w.C, d->plan, status, s)) return rc;
  const int64_t in_f = int64_t(w.C) * w.B, out_f = int64_t(w.R) * w.B;
  const bool sm = w.B < 64;
  CUtensorMap ma, mw;
  if (sm) {
    if (int rc = make_small_x_map(&ma, d->x, in_f, d->T, w.B)) return rc;
    if (int rc = make_small_w_map(&mw, w)) return rc;
  } else {
    if (int rc = make_map_2d(&ma, d->x, MapType::BF16, in_f, d->T, uint64_t(in_f) * 2, 64, a_box_rows(w.B),
                             Swz::B128))
      return rc;
    if (int rc = make_w_map(&mw, w)) return rc;
  }
  PlanLayout L = plan_layout(0, 0, 0, w.R, w.K);
  Bf16Params p{};
  p.T = d->T;
  p.n_mtiles = int32_t((d->T + kBM - 1) / kBM);
  p.R = w.R;
  p.K0 = w.K;
  p.S = w.K;
  p.plan = reinterpret_cast<const uint32_t*>(static_cast<const char*>(d->plan) + L.d_entries);
  p.counts = reinterpret_cast<const int32_t*>(static_cast<const char*>(d->plan) + L.d_counts);
  p.out = d->out;
  p.ld_out = out_f;
  p.residual = d->residual;
  p.add_residual = d->add_residual ? 1 : 0;
  p.out_f32 = d->out_dtype == BELL_DTYPE_F32 ? 1 : 0;
  p.status = status;
  p.timeout_ns = wait_budget_ns();
  p.max_ctas = d->max_ctas;
  if (!res_all) {  // hi >= 1 here; [k, k) adds the residual to no row
    p.res_lo = d->residual_row_lo;
    p.res_hi = d->residual_row_hi;
  }
  if (sm) return launch_small(false, w.B, w.layout == BELL_TILE_IN_OUT, ma, mw, mw, p, s);
  return dispatch_bf16<false>(w.B, w.layout, ma, mw, mw, p, s);
}

int bell_down_silu_bwd_bf16(const BellDownBwdDesc* d, void* stream) {
  if (!d) return fail(BELL_ERR_ARG, "descriptor is NULL");
  if (int rc = check_ell(d->w_t, "w_t")) return rc;
  if (d->w_t.B < 64)
    return fail(BELL_ERR_SHAPE, "bell_down_silu_bwd_bf16: tile size must be 64 or 128 (use bell_linear_bf16 + "
                                "bell_silu_mul_bwd_bf16 for smaller tiles)");
  if (d->T < 0) return fail(BELL_ERR_SHAPE, "T must be >= 0");
  if (d->T > 0 && (!d->grad_out || !d->gate_pre || !d->up_out || !d->d_gate_up || !d->plan))
    return fail(BELL_ERR_ARG, "grad_out, gate_pre, up_out, d_gate_up and plan must be non-NULL");
  if (!aligned16(d->grad_out) || !aligned16(d->gate_pre) || !aligned16(d->up_out) || !aligned16(d->d_gate_up) ||
      !aligned16(d->plan))
    return fail(BELL_ERR_ALIGN, "bell_down_silu_bwd_bf16: pointers must be 16-byte aligned");
  if (int rc = require_sm100()) return rc;
  if (d->T == 0) return BELL_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* status = d->status ? d->status : default_status_ptr();
  if (!status) return BELL_ERR_LAUNCH;
  const BellEll& w = d->w_t;
  if (int rc = launch_plan(nullptr, 0, nullptr, 0, 0, 0, w.col_indices, w.K, w.R, w.C, d->plan, status, s)) return rc;
  const int64_t in_f = int64_t(w.C) * w.B, F = int64_t(w.R) * w.B;
  CUtensorMap ma, mw;
  if (int rc = make_map_2d(&ma, d->grad_out, MapType::BF16, in_f, d->T, uint64_t(in_f) * 2, 64, kBM, Swz::B128))
    return rc;
  if (int rc = make_w_map(&mw, w)) return rc;
  PlanLayout L = plan_layout(0, 0, 0, w.R, w.K);
  Bf16Params p{};
  p.T = d->T;
  p.n_mtiles = int32_t((d->T + kBM - 1) / kBM);
  p.R = w.R;
  p.K0 = w.K;
  p.S = w.K;
  p.plan = reinterpret_cast<const uint32_t*>(static_cast<const char*>(d->plan) + L.d_entries);
  p.counts = reinterpret_cast<const int32_t*>(static_cast<const char*>(d->plan) + L.d_counts);
  p.out = d->d_gate_up;
  p.ld_out = 2 * F;
  p.bwd_gate = d->gate_pre;
  p.bwd_up = d->up_out;
  p.ld_bwd = F;
  p.du_off = F;
  p.status = status;
  p.timeout_ns = wait_budget_ns();
  // token-major engine at both tile sizes: its epilogue owns whole token
  // rows, so the gate/up rows are staged with 16-byte copies; at B = 64 the
  // results leave through TMA stores (the third map, unused by a linear)
  const bool mn = w.layout == BELL_TILE_IN_OUT;
  if (w.B == 64) {
    CUtensorMap mo;
    if (int rc = make_map_2d(&mo, d->d_gate_up, MapType::BF16, uint64_t(2 * F), uint64_t(d->T), uint64_t(2 * F) * 2,
                             64, 32, Swz::B128))
      return rc;
    return mn ? launch_bf16<64, false, true, true>(ma, mw, mo, p, s) : launch_bf16<64, false, false, true>(ma, mw, mo, p, s);
  }
  return mn ? launch_bf16<128, false, true, true>(ma, mw, mw, p, s) : launch_bf16<128, false, false, true>(ma, mw, mw, p, s);
}

}  // extern "C"
