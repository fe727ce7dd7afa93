// bell_loop_kernel.cu — the L-iteration shared-weight loop in ONE persistent
// kernel:  for it < L:  hn = RMSNorm(h);  h_mid = silu(hn Wg) * (hn Wu);
//                        h = h_mid Wd + h
// (the order of the reference persistent_mlp_step, csrc/loop/
// persistent_core.cu:315-335, with one weight set repeated L times).
//
// One CTA per SM (cooperative launch, so every CTA is resident and the
// grid-wide barriers between phases cannot deadlock).  The two GEMM phases
// are phases of the token-major engine (bell_engine.cuh) with its warp roles;
// the TMA rings, TMEM accumulators and per-warp pipeline state carry over
// from phase to phase.  The RMSNorm phase uses every warp, one token row per
// warp.  Weight tiles are loaded with an L2 evict-last policy, so the 2.6 MB
// of gate/up/down tiles (config 4) stay L2-resident across all iterations.
// Every wait — mbarrier or grid barrier — is bounded by the status/abort
// machinery of bell_ptx.cuh.
//
// Tile size 64, either tile layout; other tile sizes use the multi-launch loop.
#include <string>

#include "bell_bf16.cuh"
#include "bell_engine.cuh"
#include "bell_host.h"
#include "bell_ptx.cuh"

namespace bell {
namespace loopk {

static constexpr int B = 64;
using G = eng::Geo<B, true>;  // ring / accumulator geometry of both phases

struct LoopParams {
  int64_t T;
  int32_t L, d_model;
  float eps;
  __nv_bfloat16* h;           // state, updated in place
  __nv_bfloat16* hn;          // normalised state
  const __nv_bfloat16* gain;  // RMSNorm scale [d_model]
  unsigned int* gbar;         // grid barrier counter (zeroed by the host)
  int32_t* status;
  uint64_t timeout_ns;
  Bf16Params gu;              // hn -> h_mid = silu(hn Wg) * (hn Wu)
  Bf16Params dn;              // h_mid -> h = h_mid Wd + h
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

// The engine's role functions are called through these non-inlined wrappers.
// With the producer, issuer and epilogue of both phases all inlined into one
// kernel body, the down phase computed wrong results (while each phase alone
// was exact); any one role kept out of line gives exact results, so all are.
template <bool GU, bool W_MN>
__device__ __noinline__ bool loop_produce(const Bf16Params& p, const CUtensorMap* ta, const CUtensorMap* tw0,
                                          const CUtensorMap* tw1, const eng::Smem& s, eng::ProdState& st, int i_base,
                                          int pid, const Ctl& ctl, uint64_t pol_a, uint64_t pol_w) {
  return eng::produce<B, GU, W_MN, G>(p, ta, tw0, tw1, s, st, i_base, pid, ctl, pol_a, pol_w);
}
template <bool GU, bool W_MN>
__device__ __noinline__ bool loop_issue(const Bf16Params& p, const eng::Smem& s, uint32_t tmem, eng::IssueState& st,
                                        int i_base, int k, bool leader, const Ctl& ctl) {
  return eng::issue<B, GU, W_MN, G>(p, s, tmem, st, i_base, k, leader, ctl);
}
template <bool GU>
__device__ __noinline__ bool loop_epilogue(const Bf16Params& p, const eng::Smem& s, uint32_t tmem, int i_base,
                                           const Ctl& ctl) {
  return eng::epilogue<B, GU, G>(p, s, tmem, i_base, ctl);
}

template <bool W_MN>
__global__ void __launch_bounds__(eng::kThreads, 1)
    loop_kernel(const __grid_constant__ CUtensorMap tm_hn, const __grid_constant__ CUtensorMap tm_hmid,
                const __grid_constant__ CUtensorMap tm_wg, const __grid_constant__ CUtensorMap tm_wu,
                const __grid_constant__ CUtensorMap tm_wd, const __grid_constant__ LoopParams p) {
  extern __shared__ uint8_t smem_raw[];
  const eng::Smem s = eng::carve<G>(smem_raw);
  const uint32_t tmem = eng::setup<G>(s);
  Ctl ctl{s.abort_flag, p.status, p.timeout_ns};
  const int warp = threadIdx.x >> 5;
  const eng::Role role = eng::role_of(warp);
  const int pid = eng::producer_id(warp), k = warp == 1 ? 0 : 1;
  const bool leader = elect_one();
  if (warp == 0 && (threadIdx.x & 31) == 0) {
    prefetch_tmap(&tm_hn);
    prefetch_tmap(&tm_hmid);
    prefetch_tmap(&tm_wg);
    prefetch_tmap(&tm_wu);
    prefetch_tmap(&tm_wd);
  }
  const uint64_t pol_a = policy_evict_normal();
  const uint64_t pol_w = policy_evict_last();
  eng::ProdState ps;
  eng::IssueState is;
  const int nl_gu = eng::local_units(p.gu.n_mtiles * p.gu.R);
  const int nl_dn = eng::local_units(p.dn.n_mtiles * p.dn.R);
  const unsigned nG = gridDim.x;
  bool ok = true;
  for (int it = 0; it < p.L && ok; ++it) {
    norm_phase(p);
    if (!grid_sync(p, unsigned(3 * it + 1) * nG, ctl, false)) {
      ok = false;
      break;
    }
    const int base = it * (nl_gu + nl_dn);  // units this CTA took in earlier phases
#pragma unroll 1
    for (int ph = 0; ph < 2; ++ph) {
      bool role_ok = true;
      if (role == eng::kProducer) {
        role_ok = ph == 0 ? loop_produce<true, W_MN>(p.gu, &tm_hn, &tm_wg, &tm_wu, s, ps, base, pid, ctl, pol_a, pol_w)
                          : loop_produce<false, W_MN>(p.dn, &tm_hmid, &tm_wd, &tm_wd, s, ps, base + nl_gu, pid, ctl,
                                                      pol_a, pol_w);
      } else if (role == eng::kIssuer) {
        role_ok = ph == 0 ? loop_issue<true, W_MN>(p.gu, s, tmem, is, base, k, leader, ctl)
                          : loop_issue<false, W_MN>(p.dn, s, tmem, is, base + nl_gu, k, leader, ctl);
      } else {
        role_ok = ph == 0 ? loop_epilogue<true>(p.gu, s, tmem, base, ctl)
                          : loop_epilogue<false>(p.dn, s, tmem, base + nl_gu, ctl);
      }
      if (!grid_sync(p, unsigned(3 * it + 2 + ph) * nG, ctl, !role_ok)) {
        ok = false;
        break;
      }
    }
  }
  if (role == eng::kProducer && !ok) eng::producer_drain<G>(s, ps, pid);
  if (role == eng::kIssuer) eng::issuer_drain(s, k, leader);
  eng::teardown<G>(tmem);
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
  p.d_model = d->d_model;
  p.eps = d->eps;
  p.h = static_cast<__nv_bfloat16*>(d->h_out);
  p.hn = static_cast<__nv_bfloat16*>(d->hn);
  p.gain = static_cast<const __nv_bfloat16*>(d->norm_gain);
  p.gbar = static_cast<unsigned int*>(d->barrier);
  p.status = status;
  p.timeout_ns = wait_budget_ns();
  Bf16Params& gu = p.gu;  // hn -> h_mid
  gu.T = d->T;
  gu.n_mtiles = int32_t((d->T + kBM - 1) / kBM);
  gu.R = g.R;
  gu.K0 = g.K;
  gu.K1 = u.K;
  gu.S = g.K + u.K;
  gu.plan = reinterpret_cast<const uint32_t*>(plan + PL.gu_entries);
  gu.counts = reinterpret_cast<const int32_t*>(plan + PL.gu_counts);
  gu.out = d->h_mid;
  gu.ld_out = d->d_ff;
  gu.band = g.R < 32 ? g.R : 32;  // weight bands stay L2-resident while the token tiles pass
  gu.status = status;
  gu.timeout_ns = p.timeout_ns;
  Bf16Params& dn = p.dn;  // h_mid -> h = h_mid Wd + h, in place
  dn.T = d->T;
  dn.n_mtiles = gu.n_mtiles;
  dn.R = w.R;
  dn.K0 = w.K;
  dn.K1 = 0;
  dn.S = w.K;
  dn.plan = reinterpret_cast<const uint32_t*>(plan + PL.d_entries);
  dn.counts = reinterpret_cast<const int32_t*>(plan + PL.d_counts);
  dn.out = d->h_out;
  dn.ld_out = d->d_model;
  dn.residual = d->h_out;
  dn.add_residual = 1;
  dn.band = w.R;
  dn.status = status;
  dn.timeout_ns = p.timeout_ns;

  const bool w_mn = g.layout == BELL_TILE_IN_OUT;
  const void* fn = w_mn ? reinterpret_cast<const void*>(&loop_kernel<true>)
                        : reinterpret_cast<const void*>(&loop_kernel<false>);
  if (int rc = set_smem(fn, G::SMEM_BYTES)) return rc;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, eng::kThreads, G::SMEM_BYTES);
  if (e != cudaSuccess || per_sm < 1)
    return fail(BELL_ERR_LAUNCH, "loop kernel: no resident CTA per SM");
  int sms = 0;
  if (int rc = device_sm_count(&sms)) return rc;
  const int grid = sms;  // one CTA per SM: every CTA resident, one TMEM owner per SM
  e = cudaMemsetAsync(d->barrier, 0, 64, s);
  if (e != cudaSuccess) return fail(BELL_ERR_LAUNCH, std::string("loop barrier reset: ") + cudaGetErrorString(e));

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(eng::kThreads);
  cfg.dynamicSmemBytes = G::SMEM_BYTES;
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
