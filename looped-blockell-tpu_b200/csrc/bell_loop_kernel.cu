// bell_loop_kernel.cu — the L-iteration shared-weight loop in ONE persistent
// kernel:  for it < L:  hn = RMSNorm(h);  h_mid = silu(hn Wg) * (hn Wu);
//                        h = h_mid Wd + h
// (the order of the reference persistent_mlp_step, csrc/loop/
// persistent_core.cu:315-335, with one weight set repeated L times).
//
// One CTA per SM (cooperative launch, so every CTA is resident and the
// grid-wide barriers between phases cannot deadlock).  Warp roles inside the
// GEMM phases are those of the single-CTA token-major bf16 kernel: warps 0
// and 6 TMA producers, warp 1 TMEM owner + MMA issuer, warps 2-5 epilogue;
// the TMA ring and the TMEM accumulator ring carry over from phase to phase.  The RMSNorm
// phase uses every warp, one token row per warp.  Weight tiles are loaded with
// an L2 evict-last policy, so the 2.6 MB of gate/up/down tiles (config 4) stay
// L2-resident across all iterations.  Every wait — mbarrier or grid barrier —
// is bounded by the status/abort machinery of bell_ptx.cuh.
//
// Tile size 64, either tile layout; other tile sizes use the multi-launch loop.
#include <string>

#include "bell_bf16.cuh"
#include "bell_host.h"
#include "bell_ptx.cuh"

namespace bell {
namespace loopk {

static constexpr int B = 64;
static constexpr int A_BYTES = kBM * kBK * 2;      // 16 KB: 128 tokens x 64 K
static constexpr int W_BYTES = kBK * B * 2;        // 8 KB: 64 K x 64 N
static constexpr int STAGE = A_BYTES + 2 * W_BYTES;  // 32 KB
static constexpr int NS = 6;
static constexpr int ACC = 2 * B;                  // gate | up columns per accumulator
static constexpr int SMEM = NS * STAGE + 1024 + 512;
static constexpr int kLoopThreads = 224;  // warps 0, 6 producers; 1 MMA; 2-5 epilogue
static constexpr int kProd1 = 6;

struct LoopParams {
  int64_t T;
  int32_t L, n_mtiles, d_model, d_ff;
  float eps;
  int32_t R_gu, K_g, K_u, S_gu, R_d, K_d;
  const uint32_t* plan_gu;
  const int32_t* cnt_gu;
  const uint32_t* plan_d;
  const int32_t* cnt_d;
  __nv_bfloat16* h;           // state, updated in place
  __nv_bfloat16* hn;          // normalised state
  __nv_bfloat16* hmid;        // silu(gate) * up
  const __nv_bfloat16* gain;  // RMSNorm scale [d_model]
  unsigned int* gbar;         // grid barrier counter (zeroed by the host)
  int32_t* status;
  uint64_t timeout_ns;
};

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier: every CTA arrives once per call; `target` is the
// cumulative arrival count to wait for.  Generic-proxy stores made before it
// (RMSNorm output, epilogue stores) are fenced for the async proxy so the
// TMA loads of other CTAs after it see them.  Bounded: on timeout it records
// BELL_STATUS_TIMEOUT.  Returns false (uniformly across the CTA) when this
// CTA must stop: a role of it failed (`failed`), or the barrier timed out.
__device__ __forceinline__ bool grid_sync(const LoopParams& p, unsigned target, const Ctl& ctl, bool failed) {
  fence_proxy_async_global();
  __threadfence();
  if (__syncthreads_or(failed || *ctl.abort)) return false;
  bool timed_out = false;
  if (threadIdx.x == 0) {
    __threadfence();  // release this CTA's writes (ordered before it by the CTA barrier)
    atomicAdd(p.gbar, 1u);
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_gpu(p.gbar) < target) {
      if (globaltimer_ns() - t0 > ctl.timeout_ns) {
        raise_status(ctl, BELL_STATUS_TIMEOUT);
        timed_out = true;
        break;
      }
      __nanosleep(64);
    }
    __threadfence();  // acquire side: later loads of the CTA see the other CTAs' writes
  }
  if (__syncthreads_or(timed_out)) return false;
  fence_proxy_async_global();
  return true;
}

// One warp per token row: hn = h * rsqrt(mean(h^2) + eps) * gain.
__device__ __forceinline__ void norm_phase(const LoopParams& p) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int64_t row = int64_t(blockIdx.x) * warps + (threadIdx.x >> 5); row < p.T;
       row += int64_t(gridDim.x) * warps) {
    const __nv_bfloat16* x = p.h + row * p.d_model;
    float ss = 0.f;
    for (int i = lane * 8; i < p.d_model; i += 256) {
      const uint4 v = *reinterpret_cast<const uint4*>(x + i);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = unpack_bf16x2(w[t]);
        ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss / float(p.d_model) + p.eps);
    __nv_bfloat16* y = p.hn + row * p.d_model;
    for (int i = lane * 8; i < p.d_model; i += 256) {
      const uint4 v = *reinterpret_cast<const uint4*>(x + i);
      const uint4 g = *reinterpret_cast<const uint4*>(p.gain + i);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w}, gw[4] = {g.x, g.y, g.z, g.w};
      uint32_t o[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = unpack_bf16x2(w[t]), s = unpack_bf16x2(gw[t]);
        o[t] = pack_bf16x2(f.x * inv * s.x, f.y * inv * s.y);
      }
      *reinterpret_cast<uint4*>(y + i) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

struct PhaseArgs {
  int32_t R, K0, K1, S;
  const uint32_t* plan;
  const int32_t* cnt;
};

__device__ __forceinline__ PhaseArgs phase_args(const LoopParams& p, bool gu) {
  return gu ? PhaseArgs{p.R_gu, p.K_g, p.K_u, p.S_gu, p.plan_gu, p.cnt_gu}
            : PhaseArgs{p.R_d, p.K_d, 0, p.K_d, p.plan_d, p.cnt_d};
}

// TMA producer for one GEMM phase (tile size 64: one K chunk per plan step).
// Two producer warps take alternate stage uses (use g goes to producer g & 1);
// `last_stage`/`last_phase` record this producer's newest copy for the
// error-path drain.
__device__ __forceinline__ bool produce(bool gu, const CUtensorMap* ta, const CUtensorMap* tw0, const CUtensorMap* tw1,
                                       const LoopParams& p, uint8_t* smem, uint64_t* full, uint64_t* empty, int& stage,
                                       uint32_t& phase, uint32_t& g, int pid, int& last_stage, uint32_t& last_phase,
                                       const Ctl& ctl, uint64_t pol_a, uint64_t pol_w) {
  const PhaseArgs a = phase_args(p, gu);
  const int n_units = p.n_mtiles * a.R;
  for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
    const int m = u / a.R, r = u % a.R;
    const int n = a.cnt[r] & 0xFFFF;
    for (int s = 0; s < n; ++s, ++g) {
      if (int(g & 1u) == pid) {
        const uint32_t e = a.plan[size_t(r) * a.S + s];
        const int c = int(e & 0xFFFFu);
        const uint32_t k0 = (e >> 16) & 0xFFu, k1 = e >> 24;
        const bool has0 = k0 != kNone, has1 = gu && k1 != kNone;
        if (!mbar_wait(&empty[stage], phase ^ 1, ctl)) return false;
        uint8_t* st = smem + stage * STAGE;
        mbar_arrive_expect_tx(&full[stage], A_BYTES + (has0 ? W_BYTES : 0) + (has1 ? W_BYTES : 0));
        tma_load_2d(st, ta, &full[stage], c * B, m * kBM, pol_a);
        // a 64 x 64 tile is one box in either layout: coordinates (0, tile * 64)
        if (has0) tma_load_2d(st + A_BYTES, tw0, &full[stage], 0, (r * a.K0 + int(k0)) * B, pol_w);
        if (has1) tma_load_2d(st + A_BYTES + W_BYTES, tw1, &full[stage], 0, (r * a.K1 + int(k1)) * B, pol_w);
        last_stage = stage;
        last_phase = phase;
      }
      if (++stage == NS) {
        stage = 0;
        phase ^= 1;
      }
    }
  }
  return true;
}

template <bool W_MN>
__device__ __forceinline__ bool mma_phase(bool gu, const LoopParams& p, uint8_t* smem, uint64_t* full,
                                          uint64_t* empty, uint64_t* acc_full, uint64_t* acc_empty, uint32_t tmem,
                                          int& stage, uint32_t& phase, int& acc_i, const Ctl& ctl) {
  constexpr uint32_t IDESC_1 = idesc_bf16(kBM, B, false, W_MN);
  constexpr uint32_t IDESC_2 = idesc_bf16(kBM, 2 * B, false, W_MN);
  constexpr uint64_t kBStep = W_MN ? (2048 >> 4) : (32 >> 4);
  const uint64_t a_desc0 = sdesc_sw128(smem_u32(smem), 16, 1024);
  const uint64_t b_desc0 = W_MN ? sdesc_sw128(smem_u32(smem) + A_BYTES, 8192, 1024)
                                : sdesc_sw128(smem_u32(smem) + A_BYTES, 16, 1024);
  const PhaseArgs a = phase_args(p, gu);
  const int n_units = p.n_mtiles * a.R;
  for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++acc_i) {
    const int r = u % a.R;
    const int buf = acc_i & 1;
    const uint32_t use = uint32_t(acc_i >> 1);
    if (!mbar_wait(&acc_empty[buf], (use & 1u) ^ 1u, ctl)) return false;
    tc_fence_after();
    const uint32_t d0 = tmem + uint32_t(buf * ACC), d1 = d0 + B;
    const int n = a.cnt[r] & 0xFFFF;
    uint32_t init0 = 0, init1 = 0;
    for (int s = 0; s < n; ++s) {
      const uint32_t e = a.plan[size_t(r) * a.S + s];
      const bool has0 = ((e >> 16) & 0xFFu) != kNone, has1 = gu && (e >> 24) != kNone;
      if (!mbar_wait(&full[stage], phase, ctl)) return false;
      tc_fence_after();
      const uint64_t ad = a_desc0 + uint64_t(stage) * (STAGE >> 4);
      const uint64_t bd0 = b_desc0 + uint64_t(stage) * (STAGE >> 4), bd1 = bd0 + (W_BYTES >> 4);
      if (has0 && has1 && init0 == init1) {  // gate | up side by side: one N = 128 MMA
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) mma_bf16(d0, ad + 2 * kk, bd0 + kk * kBStep, IDESC_2, kk ? 1u : init0);
      } else {
        if (has0) {
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) mma_bf16(d0, ad + 2 * kk, bd0 + kk * kBStep, IDESC_1, kk ? 1u : init0);
        }
        if (has1) {
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) mma_bf16(d1, ad + 2 * kk, bd1 + kk * kBStep, IDESC_1, kk ? 1u : init1);
        }
      }
      if (has0) init0 = 1;
      if (has1) init1 = 1;
      mma_commit(&empty[stage]);
      if (++stage == NS) {
        stage = 0;
        phase ^= 1;
      }
    }
    mma_commit(&acc_full[buf]);
  }
  return true;
}

__device__ __forceinline__ bool epilogue_phase(bool gu, const LoopParams& p, uint64_t* acc_full, uint64_t* acc_empty,
                                               uint32_t tmem, int& acc_i, const Ctl& ctl) {
  const int q = (threadIdx.x >> 5) & 3, lane = threadIdx.x & 31;
  const PhaseArgs a = phase_args(p, gu);
  const int n_units = p.n_mtiles * a.R;
  for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++acc_i) {
    const int m = u / a.R, r = u % a.R;
    const int buf = acc_i & 1;
    const uint32_t use = uint32_t(acc_i >> 1);
    const bool got = mbar_wait(&acc_full[buf], use & 1u, ctl);
    if (!__all_sync(0xffffffffu, got)) return false;
    tc_fence_after();
    const int cw = a.cnt[r];
    const bool any0 = (cw >> 16) & 1, any1 = (cw >> 17) & 1;
    const int64_t row = int64_t(m) * kBM + q * 32 + lane;
    const uint32_t tb = tmem + (uint32_t(q * 32) << 16) + uint32_t(buf * ACC);
#pragma unroll 1
    for (int j = 0; j < B / 32; ++j) {
      uint32_t g[32], v[32];
      __syncwarp();
      tmem_ld32(tb + j * 32, g);
      if (gu) tmem_ld32(tb + B + j * 32, v);
      tmem_ld_wait();
      if (row >= p.T) {
      } else if (gu) {
        uint32_t hp[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const float g0 = any0 ? __uint_as_float(g[2 * t]) : 0.f, g1 = any0 ? __uint_as_float(g[2 * t + 1]) : 0.f;
          const float u0 = any1 ? __uint_as_float(v[2 * t]) : 0.f, u1 = any1 ? __uint_as_float(v[2 * t + 1]) : 0.f;
          hp[t] = pack_bf16x2(silu_fast(g0) * u0, silu_fast(g1) * u1);
        }
        __nv_bfloat16* dst = p.hmid + row * p.d_ff + int64_t(r) * B + j * 32;
#pragma unroll
        for (int t = 0; t < 4; ++t) st_global_v4(dst + t * 8, hp[4 * t], hp[4 * t + 1], hp[4 * t + 2], hp[4 * t + 3]);
      } else {
        __nv_bfloat16* hrow = p.h + row * p.d_model + int64_t(r) * B + j * 32;  // residual in, result out
        uint32_t o[16];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const uint4 rv = ld_global_v4(hrow + t * 8);
          const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const float2 x2 = unpack_bf16x2(rw[w]);
            const float a0 = any0 ? __uint_as_float(g[8 * t + 2 * w]) : 0.f;
            const float a1 = any0 ? __uint_as_float(g[8 * t + 2 * w + 1]) : 0.f;
            o[4 * t + w] = pack_bf16x2(a0 + x2.x, a1 + x2.y);
          }
        }
#pragma unroll
        for (int t = 0; t < 4; ++t) st_global_v4(hrow + t * 8, o[4 * t], o[4 * t + 1], o[4 * t + 2], o[4 * t + 3]);
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&acc_empty[buf]);
  }
  return true;
}

template <bool W_MN>
__global__ void __launch_bounds__(kLoopThreads, 1)
    loop_kernel(const __grid_constant__ CUtensorMap tm_hn, const __grid_constant__ CUtensorMap tm_hmid,
                const __grid_constant__ CUtensorMap tm_wg, const __grid_constant__ CUtensorMap tm_wu,
                const __grid_constant__ CUtensorMap tm_wd, const LoopParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * STAGE);
  uint64_t* empty = full + NS;
  uint64_t* acc_full = empty + NS;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  Ctl ctl{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
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
    tmem_alloc(tmem_slot, 2 * ACC);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tm_hn);
    prefetch_tmap(&tm_hmid);
    prefetch_tmap(&tm_wg);
    prefetch_tmap(&tm_wu);
    prefetch_tmap(&tm_wd);
  }
  const uint64_t pol_a = policy_evict_normal();
  const uint64_t pol_w = policy_evict_last();

  // pipeline state, carried from phase to phase (each role uses its own copy)
  int stage = 0, acc_i = 0, last_stage = -1;
  uint32_t phase = 0, g = 0, last_phase = 0;
  bool ok = true;
  const unsigned G = gridDim.x;
  for (int it = 0; it < p.L && ok; ++it) {
    norm_phase(p);
    if (!grid_sync(p, unsigned(3 * it + 1) * G, ctl, false)) {
      ok = false;
      break;
    }
#pragma unroll 1
    for (int ph = 0; ph < 2; ++ph) {
      const bool gu = ph == 0;
      bool role_ok = true;
      if (warp == 0 || warp == kProd1) {
        if (lane == 0)
          role_ok = produce(gu, gu ? &tm_hn : &tm_hmid, gu ? &tm_wg : &tm_wd, &tm_wu, p, smem, full, empty, stage,
                            phase, g, warp == 0 ? 0 : 1, last_stage, last_phase, ctl, pol_a, pol_w);
      } else if (warp == 1) {
        if (lane == 0)
          role_ok = mma_phase<W_MN>(gu, p, smem, full, empty, acc_full, acc_empty, tmem, stage, phase, acc_i, ctl);
      } else {
        role_ok = epilogue_phase(gu, p, acc_full, acc_empty, tmem, acc_i, ctl);
      }
      if (!grid_sync(p, unsigned(3 * it + 2 + ph) * G, ctl, !role_ok)) {
        ok = false;
        break;
      }
    }
  }

  if (!ok) {
    // error path: let this CTA's copies and MMAs in flight land (bounded)
    if ((warp == 0 || warp == kProd1) && lane == 0 && last_stage >= 0) {
      int st = last_stage;
      uint32_t ph = last_phase;
      for (int i = 0; i < NS; ++i) {
        const uint32_t a = smem_u32(&full[st]);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(a, ph) && globaltimer_ns() - t0 < 100000000ull) {
        }
        if (--st < 0) {
          st = NS - 1;
          ph ^= 1;
        }
      }
    } else if (warp == 1 && lane == 0) {
      mma_commit(drain);
      const uint32_t a = smem_u32(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(a, 0) && globaltimer_ns() - t0 < 100000000ull) {
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * ACC);
  }
}

}  // namespace loopk

// Host side of the persistent loop.  Preconditions checked by the caller:
// bf16 descriptor validated by check_ffn, tile size 64, h_out already holds
// h_in, plan built.  Returns BELL_ERR_LAUNCH when the cooperative grid cannot
// be formed (the caller then runs the multi-launch loop).
int loop_persistent_bf16(const BellLoopDesc* d, int32_t* status, cudaStream_t s) {
  using namespace loopk;
  if (!aligned16(d->norm_gain) || !aligned16(d->hn) || !aligned16(d->h_mid) || !aligned16(d->h_out) ||
      !aligned16(d->barrier))
    return fail(BELL_ERR_ALIGN, "loop buffers must be 16-byte aligned");
  const BellEll &g = d->gate, &u = d->up, &w = d->down;
  CUtensorMap m_hn, m_hmid, m_wg, m_wu, m_wd;
  if (int rc = make_map_2d(&m_hn, d->hn, MapType::BF16, d->d_model, d->T, uint64_t(d->d_model) * 2, 64, kBM,
                           Swz::B128))
    return rc;
  if (int rc = make_map_2d(&m_hmid, d->h_mid, MapType::BF16, d->d_ff, d->T, uint64_t(d->d_ff) * 2, 64, kBM,
                           Swz::B128))
    return rc;
  if (int rc = make_w_map(&m_wg, g)) return rc;
  if (int rc = make_w_map(&m_wu, u)) return rc;
  if (int rc = make_w_map(&m_wd, w)) return rc;
  const PlanLayout PL = plan_layout(g.R, g.K, u.K, w.R, w.K);
  const char* plan = static_cast<const char*>(d->plan);
  LoopParams p{};
  p.T = d->T;
  p.L = d->L;
  p.n_mtiles = int32_t((d->T + kBM - 1) / kBM);
  p.d_model = d->d_model;
  p.d_ff = d->d_ff;
  p.eps = d->eps;
  p.R_gu = g.R;
  p.K_g = g.K;
  p.K_u = u.K;
  p.S_gu = g.K + u.K;
  p.R_d = w.R;
  p.K_d = w.K;
  p.plan_gu = reinterpret_cast<const uint32_t*>(plan + PL.gu_entries);
  p.cnt_gu = reinterpret_cast<const int32_t*>(plan + PL.gu_counts);
  p.plan_d = reinterpret_cast<const uint32_t*>(plan + PL.d_entries);
  p.cnt_d = reinterpret_cast<const int32_t*>(plan + PL.d_counts);
  p.h = static_cast<__nv_bfloat16*>(d->h_out);
  p.hn = static_cast<__nv_bfloat16*>(d->hn);
  p.hmid = static_cast<__nv_bfloat16*>(d->h_mid);
  p.gain = static_cast<const __nv_bfloat16*>(d->norm_gain);
  p.gbar = static_cast<unsigned int*>(d->barrier);
  p.status = status;
  p.timeout_ns = wait_budget_ns();

  const bool w_mn = g.layout == BELL_TILE_IN_OUT;
  const void* fn = w_mn ? reinterpret_cast<const void*>(&loop_kernel<true>)
                        : reinterpret_cast<const void*>(&loop_kernel<false>);
  if (int rc = set_smem(fn, SMEM)) return rc;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kLoopThreads, SMEM);
  if (e != cudaSuccess || per_sm < 1)
    return fail(BELL_ERR_LAUNCH, "loop kernel: no resident CTA per SM");
  int sms = 0;
  if (int rc = device_sm_count(&sms)) return rc;
  const int grid = sms;  // one CTA per SM: every CTA resident, one TMEM owner per SM
  e = cudaMemsetAsync(d->barrier, 0, 64, s);
  if (e != cudaSuccess) return fail(BELL_ERR_LAUNCH, std::string("loop barrier reset: ") + cudaGetErrorString(e));

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(kLoopThreads);
  cfg.dynamicSmemBytes = SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (w_mn)
    e = cudaLaunchKernelEx(&cfg, loop_kernel<true>, m_hn, m_hmid, m_wg, m_wu, m_wd, p);
  else
    e = cudaLaunchKernelEx(&cfg, loop_kernel<false>, m_hn, m_hmid, m_wg, m_wu, m_wd, p);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(BELL_ERR_LAUNCH, std::string("loop kernel launch: ") + cudaGetErrorString(e));
  }
  return BELL_OK;
}

}  // namespace bell
