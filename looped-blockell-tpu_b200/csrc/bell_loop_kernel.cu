// bell_loop_kernel.cu — the L-iteration shared-weight loop in ONE persistent
// kernel:  for it < L:  h_mid = silu(RMSNorm(h) Wg) * (RMSNorm(h) Wu);
//                        h = h_mid Wd + h
// (the order of the reference persistent_mlp_step, csrc/loop/
// persistent_core.cu:315-335, with one weight set repeated L times).
//
// One CTA per SM (cooperative launch, so every CTA is resident).  The two
// GEMM phases of every iteration are phases of the token-major engine
// (bell_engine.cuh) with its warp roles; the TMA rings, TMEM accumulators and
// per-warp pipeline state carry over from phase to phase.  RMSNorm has no
// phase of its own: RMSNorm(h) W = diag(1/rms) h diag(gain) W, so the gate/up
// GEMMs read h itself against gain-scaled tiles (made by the host entry point)
// and the epilogue multiplies each token row by its 1/rms, from per-row sums
// of squares that the down epilogue of the previous iteration wrote next to
// the new h (the first ones come from a small kernel before this one).
//
// There is no grid barrier: the FFN is token-local, so each 128-token tile m
// only waits for its own producers, through two per-tile counters:
//   gu[m]  +1 per epilogue warp per gate/up unit of tile m (h_mid stored);
//   dn[m]  +1 per epilogue warp per down unit of tile m (h and its sums of
//          squares stored).
// A gate/up unit of iteration `it` loads h[m] once dn[m] >= 4 R_model it; a
// down unit loads h_mid[m] once gu[m] >= 4 R_ff (it+1).  These conditions also
// cover the write-after-read hazards of the in-place buffers: a tile's next
// writer waits, through the chain, for every reader of its previous contents.
// Epilogues acquire the counters themselves before reading what they publish.
// Every role works through its phases in order and only waits on work of an
// earlier phase, and every CTA is resident, so the waits always end; each is
// still bounded by the status/abort machinery of bell_ptx.cuh.  Weight tiles
// are loaded with an L2 evict-last policy, so the gate/up/down tiles (config
// 4: 6.3 MB) stay L2-resident across all iterations.
//
// Tile size 64, either tile layout; other tile sizes use the launch loop.
#include <cstdlib>
#include <string>

#include "bell_bf16.cuh"
#include "bell_engine.cuh"
#include "bell_host.h"
#include "bell_ptx.cuh"

namespace bell {
namespace loopk {

static constexpr int B = 64;
using G = eng::Geo<B, true>;  // ring / accumulator geometry of both phases
// Token tiles per wave.  Config 4 (64 tiles): 4 -> 2.23 ms, 8 -> 1.77 ms,
// 16 -> 1.51 ms, 32 -> 1.48 ms; 16 keeps four waves per iteration.
static constexpr int kWaveTiles = 16;

struct LoopParams {
  int64_t T;
  int32_t L, d_model;
  float eps;
  __nv_bfloat16* h;           // state, updated in place
  unsigned* cnt_gu;           // per-tile counters [n_mtiles] each (zeroed by the host)
  unsigned* cnt_dn;
  int32_t n_seg, seg_tiles;   // waves per iteration, token tiles per wave
  int32_t* status;
  uint64_t timeout_ns;
  Bf16Params gu;              // h -> h_mid = silu(RMSNorm(h) Wg) * (RMSNorm(h) Wu)
  Bf16Params dn;              // h_mid -> h = h_mid Wd + h
};

// The engine's role functions are called through these non-inlined wrappers.
// With the producer, issuer and epilogue of both phases all inlined into one
// kernel body, the down phase computed wrong results (while each phase alone
// was exact); any one role kept out of line gives exact results, so all are.
// A reference argument of a non-inlined function points into the caller's
// stack frame (local memory), and the role loops store through generic
// pointers that the compiler cannot tell apart from it, so every field read
// would be a local-memory load inside the issue, copy and store loops.  Each
// wrapper therefore copies its arguments into locals once per call (they stay
// in registers) and writes the pipeline state back when the phase ends.
template <bool GU, bool W_MN>
__device__ __noinline__ bool loop_produce(const Bf16Params& p_in, const CUtensorMap* ta, const CUtensorMap* tw0,
                                          const CUtensorMap* tw1, const eng::Smem& s_in, eng::ProdState& st_io,
                                          int i_base, int pid, const Ctl& ctl_in, uint64_t pol_a, uint64_t pol_w) {
  const Bf16Params p = p_in;
  const eng::Smem s = s_in;
  const Ctl ctl = ctl_in;
  eng::ProdState st = st_io;
  const bool ok = eng::produce<B, GU, W_MN, G>(p, ta, tw0, tw1, s, st, i_base, pid, ctl, pol_a, pol_w);
  st_io = st;
  return ok;
}
template <bool GU, bool W_MN>
__device__ __noinline__ bool loop_issue(const Bf16Params& p_in, const eng::Smem& s_in, uint32_t tmem,
                                        eng::IssueState& st_io, int i_base, int k, bool leader, const Ctl& ctl_in) {
  const Bf16Params p = p_in;
  const eng::Smem s = s_in;
  const Ctl ctl = ctl_in;
  eng::IssueState st = st_io;
  const bool ok = eng::issue<B, GU, W_MN, G>(p, s, tmem, st, i_base, k, leader, ctl);
  st_io = st;
  return ok;
}
template <bool GU>
__device__ __noinline__ bool loop_epilogue(const Bf16Params& p_in, const eng::Smem& s_in, uint32_t tmem, int i_base,
                                           const Ctl& ctl_in) {
  const Bf16Params p = p_in;
  const eng::Smem s = s_in;
  const Ctl ctl = ctl_in;
  return eng::epilogue<B, GU, G>(p, s, tmem, i_base, ctl);
}

template <bool W_MN>
__global__ void __launch_bounds__(eng::kThreads, 1)
    loop_kernel(const __grid_constant__ CUtensorMap tm_h, const __grid_constant__ CUtensorMap tm_hmid,
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
    prefetch_tmap(&tm_h);
    prefetch_tmap(&tm_hmid);
    prefetch_tmap(&tm_wg);
    prefetch_tmap(&tm_wu);
    prefetch_tmap(&tm_wd);
  }
  const uint64_t pol_a = policy_evict_normal();
  const uint64_t pol_w = policy_evict_last();
  eng::ProdState ps;
  eng::IssueState is;
  // The work runs in waves of `seg_tiles` token tiles: wave w = it * S + s
  // covers tiles [s * seg_tiles, (s+1) * seg_tiles) of iteration it.  Every
  // role walks, for w = 0 .. L*S, the gate/up units of wave w, then the down
  // units of wave w-1: a down wave waits on the gate/up wave before it, with
  // the next gate/up wave's work in between, and a gate/up wave waits on the
  // down wave of the same tiles one iteration earlier (S >= 2 waves earlier).
  // Every unit only waits on units earlier in this one global order.
  const int S = p.n_seg;
  const int st = p.seg_tiles;
  const int n_mt = p.gu.n_mtiles;
  int base = 0;  // units this CTA took in earlier segments
  bool ok = true;
  for (int w = 0; w <= p.L * S && ok; ++w) {
#pragma unroll 1
    for (int part = 0; part < 2 && ok; ++part) {
      const int wv = part == 0 ? w : w - 1;  // gate/up of wave w, then down of wave w-1
      if (wv < 0 || wv >= p.L * S) continue;
      const int it = wv / S, sg = wv % S;
      const int t0 = sg * st, t1 = (sg + 1) * st < n_mt ? (sg + 1) * st : n_mt;
      if (t0 >= t1) continue;
      const bool gu_part = part == 0;
      Bf16Params q = gu_part ? p.gu : p.dn;
      q.u_begin = t0 * q.R;
      q.u_end = t1 * q.R;
      unsigned* sig = gu_part ? p.cnt_gu : p.cnt_dn;  // signalled once per wave, below
      // The wave's inputs: every tile of the wave ready before any of its
      // units load (one parallel acquire per tile instead of one per unit).
      // Gate/up reads h[m] and its sums of squares (down of the previous
      // iteration); down reads h_mid[m] (gate/up of this iteration) and the
      // residual h[m] (down of the previous iteration).
      if (role == eng::kProducer || role == eng::kEpilogue) {
        const unsigned tgt_dn = 4u * unsigned(p.dn.R) * unsigned(it);
        const unsigned tgt_gu = 4u * unsigned(p.gu.R) * unsigned(it + 1);
        const int lane = threadIdx.x & 31;
        bool w_ok = true;
        for (int t = t0 + lane; t < t1; t += 32) {
          if (gu_part) w_ok = w_ok && wait_count(p.cnt_dn + t, tgt_dn, ctl);
          else w_ok = w_ok && wait_count(p.cnt_gu + t, tgt_gu, ctl) && wait_count(p.cnt_dn + t, tgt_dn, ctl);
        }
        if (!__all_sync(0xffffffffu, w_ok)) {
          ok = false;
          break;
        }
        fence_proxy_async_global();  // the issuing lanes' TMA loads after every lane's acquire
      }
      if (role == eng::kProducer) {
        ok = gu_part ? loop_produce<true, W_MN>(q, &tm_h, &tm_wg, &tm_wu, s, ps, base, pid, ctl, pol_a, pol_w)
                     : loop_produce<false, W_MN>(q, &tm_hmid, &tm_wd, &tm_wd, s, ps, base, pid, ctl, pol_a, pol_w);
      } else if (role == eng::kIssuer) {
        ok = gu_part ? loop_issue<true, W_MN>(q, s, tmem, is, base, k, leader, ctl)
                     : loop_issue<false, W_MN>(q, s, tmem, is, base, k, leader, ctl);
      } else {
        ok = gu_part ? loop_epilogue<true>(q, s, tmem, base, ctl) : loop_epilogue<false>(q, s, tmem, base, ctl);
        if (ok) {
          // one release per warp and wave: every unit of the wave this warp
          // stored adds one to its tile's counter
          fence_proxy_async_global();
          __threadfence();
          __syncwarp();
          if ((threadIdx.x & 31) == 0) {
            const int nu = eng::seg_count(q);
            for (int i = 0; i < nu; ++i) {
              int m, r;
              unit_mr(eng::unit_at(q, i), q, m, r);
              atomicAdd(sig + m, 1u);
            }
          }
          __syncwarp();
        }
      }
      base += eng::seg_count(q);
    }
  }
  if (!ok && *ctl.abort == 0) raise_status(ctl, BELL_STATUS_INTERNAL);  // a role stopped: stop the others
  if (role == eng::kProducer && !ok) eng::producer_drain<G>(s, ps, pid);
  if (role == eng::kIssuer) eng::issuer_drain(s, k, leader);
  eng::teardown<G>(tmem);
}

}  // namespace loopk

// Host side of the persistent loop.  Preconditions checked by the caller:
// bf16 descriptor validated by check_ffn, tile size 64, h_out already holds
// h_in, plan built, `barrier` holds bell_loop_barrier_bytes(T) bytes.
int loop_persistent_bf16(const BellLoopDesc* d, const BellEll& g, const BellEll& u, int32_t* status,
                         cudaStream_t s) {
  using namespace loopk;
  if (!aligned16(d->h_mid) || !aligned16(d->h_out) || !aligned16(d->workspace))
    return fail(BELL_ERR_ALIGN, "loop buffers must be 16-byte aligned");
  const BellEll& w = d->down;
  CUtensorMap m_h, m_hmid, m_wg, m_wu, m_wd;
  // the gate/up GEMMs read the pre-norm state h (RMSNorm is folded in)
  if (int rc = make_map_2d(&m_h, d->h_out, MapType::BF16, d->d_model, d->T, uint64_t(d->d_model) * 2, 64, kBM,
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
  const int64_t n_mt = (d->T + kBM - 1) / kBM;
  const LoopWs W = loop_ws(d->T, d->d_model, g.R, g.K, u.K, 64);
  p.cnt_gu = reinterpret_cast<unsigned*>(static_cast<char*>(d->workspace) + W.counters);
  p.cnt_dn = p.cnt_gu + n_mt;
  float* ss = reinterpret_cast<float*>(static_cast<char*>(d->workspace) + W.ss);
  // waves of kWaveTiles token tiles, at least two waves per iteration (see
  // the kernel); BELL_LOOP_WAVE_TILES overrides, read per call
  const char* wave_env = std::getenv("BELL_LOOP_WAVE_TILES");
  const int64_t want = wave_env && std::atoi(wave_env) > 0 ? std::atoi(wave_env) : kWaveTiles;
  p.seg_tiles = n_mt >= 2 * want ? int32_t(want) : int32_t((n_mt + 1) / 2);
  p.n_seg = int32_t((n_mt + p.seg_tiles - 1) / p.seg_tiles);
  if (p.n_seg < 2) p.n_seg = 2;
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
  gu.band = g.R;  // token-tile-major unit order: tiles become ready, and are consumed, in order
  gu.status = status;
  gu.timeout_ns = p.timeout_ns;
  gu.row_ss = ss;
  gu.ss_parts = d->d_model / 64;
  gu.inv_d = 1.0f / float(d->d_model);
  gu.eps = d->eps;
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
  dn.ss_out = ss;
  dn.ss_parts = gu.ss_parts;

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
  e = cudaMemsetAsync(p.cnt_gu, 0, size_t(2 * n_mt) * sizeof(unsigned), s);
  if (e != cudaSuccess) return fail(BELL_ERR_LAUNCH, std::string("loop counters reset: ") + cudaGetErrorString(e));

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
    e = cudaLaunchKernelEx(&cfg, loop_kernel<true>, m_h, m_hmid, m_wg, m_wu, m_wd, p);
  else
    e = cudaLaunchKernelEx(&cfg, loop_kernel<false>, m_h, m_hmid, m_wg, m_wu, m_wd, p);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(BELL_ERR_LAUNCH, std::string("loop kernel launch: ") + cudaGetErrorString(e));
  }
  return BELL_OK;
}

}  // namespace bell
