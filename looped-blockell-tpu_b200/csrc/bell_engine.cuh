// bell_engine.cuh — the token-major bf16 Block-ELL GEMM engine, shared by
// the stand-alone gate/up and linear kernels (bell_bf16.cu) and the
// persistent loop kernel (bell_loop_kernel.cu).
//
// A phase multiplies 128-token activation tiles by the Block-ELL tiles of
// one matrix (gate/up together, or one linear matrix).  A work unit is
// (token tile m, output block-row r); the CTA walks units
// u = blockIdx.x + i * gridDim.x (of a segment [u_begin, u_end) of the
// phase when one is set) and its i-th unit (counted across phases)
// goes to MMA issuer i & 1.  Warp roles:
//   warps 0, 6, 7, 8  TMA producers: 0/6 fill ring 0, 7/8 fill ring 1; the
//                     two of a ring take its stage uses alternately.  Each
//                     warp stages its plan rows through shared memory one
//                     unit ahead (bell_sched.cuh) and writes a stage-info
//                     word per stage for the issuer.
//   warps 1, 9        MMA issuers (warp 1 also owns TMEM): issuer k reads
//                     ring k and accumulates into its own TMEM accumulators
//                     (gate | up side by side, so a shared column block is
//                     one N = 2B MMA), double buffered where TMEM allows.
//   warps 2-5         epilogue: tcgen05.ld, SiLU*up or +residual, stores.
// At tile size 64 a single thread issuing every MMA, or every TMA copy, is
// slower than the tensor core; hence two issuers and four producers.  The
// issue loops run on whole warps (state stays warp-uniform) and an elected
// lane issues.  Every wait is bounded (bell_ptx.cuh).
#pragma once

#include "bell_bf16.cuh"
#include "bell_ptx.cuh"
#include "bell_sched.cuh"

namespace bell {
namespace eng {

static constexpr int kProds = 4;
static constexpr int kProd1 = 6;                 // first of the extra producer warps
static constexpr int kMma1 = kProd1 + kProds - 1;  // second MMA issuer warp (9)
static constexpr int kThreads = 32 * (kMma1 + 1);  // 10 warps

// Ring and accumulator geometry for tile size B; GU sizes a stage for two
// weight tiles and an accumulator for gate | up.
// SB (linear with the SiLU*up backward epilogue) reserves EPI_BYTES for the
// epilogue's gate/up staging: per epilogue warp, EPI_NSLOT slots of 32 rows x
// B features of gate and of up — two at B = 64 (this unit's and the next
// one's copy in flight), one at B = 128 (copied during the accumulator wait),
// so that the stage ring keeps NR >= 2.
template <int B, bool GU, bool SB = false>
struct Geo {
  static constexpr int A_BYTES = kBM * kBK * 2;  // 16 KB
  static constexpr int W_BYTES = kBK * B * 2;    // 8 / 16 KB
  static constexpr int STAGE_BYTES = A_BYTES + W_BYTES * (GU ? 2 : 1);
  static constexpr int EPI_SLOT = SB ? 32 * B * 2 * 2 : 0;  // one warp, one unit: gate | up rows
  static constexpr int EPI_NSLOT = B == 64 ? 2 : 1;
  static constexpr int EPI_BYTES = 4 * EPI_NSLOT * EPI_SLOT;
  static constexpr int NS_FIT = ((196608 - EPI_BYTES) / STAGE_BYTES) & ~1;
  static constexpr int NS = NS_FIT < 8 ? NS_FIT : 8;
  static constexpr int NR = NS / 2;              // stages per ring
  static constexpr int ACC_COLS = GU ? 2 * B : B;  // fp32 columns of one accumulator
  // two issuers, each double buffered when the four accumulators fit
  static constexpr int NBUF = 4 * ACC_COLS <= 512 ? 2 : 1;
  static constexpr int TMEM_COLS = 2 * NBUF * ACC_COLS < 128 ? 128 : 2 * NBUF * ACC_COLS;
  // align + barriers (512) + stage info (64) + one staged plan row per producer
  // the staging area starts 1024-aligned (its slots are 128-byte-swizzled TMA boxes at B = 64)
  static constexpr int EPI_OFF = ((576 + kProds * kRowMax * 4) + 1023) & ~1023;
  static constexpr int SMEM_BYTES = NS * STAGE_BYTES + 1024 + EPI_OFF + EPI_BYTES;
  // the two producers of a ring take alternate steps; with one stage per
  // ring a producer could wait on a phase two ahead of the stage (parity
  // aliasing), so each ring needs at least two stages
  static_assert(NR >= 2, "stage ring");
  static_assert(TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation");
  static_assert(NS % 2 == 0, "the stage ring is split between two MMA issuers");
};

struct Smem {
  uint8_t* stages;
  uint64_t *full, *empty;          // [ring * NR + stage]
  uint64_t *acc_full, *acc_empty;  // [issuer * 2 + buf]
  uint64_t* drain;                 // one per issuer
  uint32_t* tmem_slot;
  volatile int* abort_flag;
  uint32_t* stage_info;            // [ring * NR + stage]
  uint32_t* rows;                  // [producer][kRowMax]
  uint8_t* epi;                    // SB: [epilogue warp][slot][gate | up rows], 1024-byte aligned
};

template <class G>
__device__ __forceinline__ Smem carve(uint8_t* smem_raw) {
  Smem s;
  s.stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ctl = s.stages + G::NS * G::STAGE_BYTES;
  s.full = reinterpret_cast<uint64_t*>(ctl);
  s.empty = s.full + G::NS;
  s.acc_full = s.empty + G::NS;
  s.acc_empty = s.acc_full + 4;
  s.drain = s.acc_empty + 4;
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.drain + 2);
  s.abort_flag = reinterpret_cast<volatile int*>(s.tmem_slot + 1);
  s.stage_info = reinterpret_cast<uint32_t*>(ctl + 512);
  s.rows = reinterpret_cast<uint32_t*>(ctl + 576);
  s.epi = ctl + G::EPI_OFF;
  return s;
}

// Barrier init and TMEM allocation (all threads; ends with a CTA barrier).
template <class G>
__device__ __forceinline__ uint32_t setup(const Smem& s) {
  if (threadIdx.x == 0) {
    for (int i = 0; i < G::NS; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int b = 0; b < 4; ++b) {
      mbar_init(&s.acc_full[b], 1);
      mbar_init(&s.acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(&s.drain[0], 1);
    mbar_init(&s.drain[1], 1);
    *s.abort_flag = 0;
    fence_mbar_init();
  }
  if ((threadIdx.x >> 5) == 1) {
    tmem_alloc(s.tmem_slot, G::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  return *s.tmem_slot;
}

template <class G>
__device__ __forceinline__ void teardown(uint32_t tmem) {
  tc_fence_before();
  __syncthreads();
  if ((threadIdx.x >> 5) == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, G::TMEM_COLS);
  }
}

// Role of this warp.
enum Role { kProducer, kIssuer, kEpilogue };
__device__ __forceinline__ Role role_of(int warp) {
  if (warp == 1 || warp == kMma1) return kIssuer;
  if (warp >= 2 && warp < 6) return kEpilogue;
  return kProducer;
}
__device__ __forceinline__ int producer_id(int warp) { return warp == 0 ? 0 : warp - kProd1 + 1; }

// Load one [64 K x B] weight chunk of tile `tile` (global tile index r*K+k).
template <int B, bool W_MN>
__device__ __forceinline__ void load_w_chunk(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int tile, int kc,
                                             uint64_t pol) {
  if constexpr (W_MN) {
    // [B_in, B_out] tile rows are K; two 64-wide boxes when B = 128.
#pragma unroll
    for (int nh = 0; nh < B / 64; ++nh) tma_load_2d(dst + nh * 8192, map, bar, nh * 64, tile * B + kc * kBK, pol);
  } else {
    // [B_out, B_in] tile rows are N; boxes of 64 K x 64 rows stacked along N.
#pragma unroll
    for (int nb = 0; nb < B / 64; ++nb) tma_load_2d(dst + nb * 8192, map, bar, kc * kBK, tile * B + nb * 64, pol);
  }
}

// Per-warp pipeline state carried from phase to phase.
struct ProdState {
  int stage = 0;  // within the ring
  uint32_t phase = 0, g = 0;
  int last_slot = -1;
  uint32_t last_phase = 0;
};
struct IssueState {
  int stage = 0;
  uint32_t phase = 0;
};

// Number of units this CTA takes in a phase of n_units units.
__device__ __forceinline__ int local_units(int n_units) {
  return int(blockIdx.x) < n_units ? (n_units - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x) : 0;
}

// This CTA's units of the segment [u_begin, u_end) of a phase: the ordinals
// i of u = blockIdx.x + i * gridDim.x inside the segment start at seg_lo and
// number seg_count; unit_at gives the i-th of them.
__device__ __forceinline__ int seg_lo(const Bf16Params& p) {
  const int b = p.u_begin - int(blockIdx.x);
  return b <= 0 ? 0 : (b + int(gridDim.x) - 1) / int(gridDim.x);
}
__device__ __forceinline__ int seg_count(const Bf16Params& p) {
  const int hi = local_units(p.u_end > 0 ? p.u_end : p.n_mtiles * p.R);
  const int lo = seg_lo(p);
  return hi > lo ? hi - lo : 0;
}
__device__ __forceinline__ int unit_at(const Bf16Params& p, int i) {
  return int(blockIdx.x) + (seg_lo(p) + i) * int(gridDim.x);
}

// ------------------------------------------------------------------ producer
// One producer warp for one phase.  `i_base` = units this CTA took in
// earlier phases.  Returns false (warp-uniform) when a wait gave up.
template <int B, bool GU, bool W_MN, class G>
__device__ bool produce(const Bf16Params& p, const CUtensorMap* ta, const CUtensorMap* tw0, const CUtensorMap* tw1,
                        const Smem& s, ProdState& st, int i_base, int pid, const Ctl& ctl, uint64_t pol_a,
                        uint64_t pol_w) {
  constexpr int KC = B / kBK;  // stages per plan step
  const int ring = pid >> 1, sub = pid & 1;
  uint32_t* row = s.rows + pid * kRowMax;
  const int nl = seg_count(p);
  const int i0 = (ring - i_base) & 1;
  RowAhead ahead;
  if (i0 < nl) {
    int m0, r0;
    unit_mr(unit_at(p, i0), p, m0, r0);
    row_fetch(ahead, p.plan, p.counts, p.S, r0);
  }
  for (int i = i0; i < nl; i += 2) {
    int m, r;
    unit_mr(unit_at(p, i), p, m, r);
    const int real = (ahead.cnt & 0xFFFF) * KC;
    row_put(ahead, row, p.S);
    __syncwarp();
    if (i + 2 < nl) {
      int m2, r2;
      unit_mr(unit_at(p, i + 2), p, m2, r2);
      row_fetch(ahead, p.plan, p.counts, p.S, r2);
    }
    if (p.dep_cnt) {  // dataflow: this token tile's activations must be complete
      bool ok = true;
      if (elect_one()) ok = wait_count(p.dep_cnt + m, p.dep_target, ctl);
      if (!__all_sync(0xffffffffu, ok)) return false;
    }
    const int uses = real > 1 ? real : 1;  // a unit without live steps: one empty stage
    for (int j = 0; j < uses; ++j, ++st.g) {
      if (int(st.g & 1u) == sub) {
        const int slot = ring * G::NR + st.stage;
        if (!__all_sync(0xffffffffu, mbar_wait(&s.empty[slot], st.phase ^ 1, ctl))) return false;
        uint32_t info = (j == 0 ? kSiFirst : 0u) | (j == uses - 1 ? kSiLast : 0u);
        if (j < real) {
          const uint32_t e = row[j / KC];
          const int kc = j % KC;
          const int c = int(e & 0xFFFFu);
          const uint32_t k0 = (e >> 16) & 0xFFu, k1 = e >> 24;
          const bool has0 = k0 != kNone, has1 = GU && k1 != kNone;
          info |= (has0 ? kSiHas0 : 0u) | (has1 ? kSiHas1 : 0u);
          if (elect_one()) {
            s.stage_info[slot] = info;
            uint8_t* sp = s.stages + slot * G::STAGE_BYTES;
            mbar_arrive_expect_tx(&s.full[slot], G::A_BYTES + (has0 ? G::W_BYTES : 0) + (has1 ? G::W_BYTES : 0));
            tma_load_2d(sp, ta, &s.full[slot], c * B + kc * kBK, m * kBM, pol_a);
            if (has0) load_w_chunk<B, W_MN>(sp + G::A_BYTES, tw0, &s.full[slot], r * p.K0 + int(k0), kc, pol_w);
            if (has1)
              load_w_chunk<B, W_MN>(sp + G::A_BYTES + G::W_BYTES, tw1, &s.full[slot], r * p.K1 + int(k1), kc, pol_w);
          }
          st.last_slot = slot;
          st.last_phase = st.phase;
        } else if (elect_one()) {
          s.stage_info[slot] = info;  // empty stage: no copies
          mbar_arrive(&s.full[slot]);
        }
        __syncwarp();
      }
      if (++st.stage == G::NR) {
        st.stage = 0;
        st.phase ^= 1;
      }
    }
    __syncwarp();
  }
  return true;
}

// Error path: let this producer's copies in flight land before the CTA exits.
template <class G>
__device__ __forceinline__ void producer_drain(const Smem& s, const ProdState& st, int pid) {
  if ((threadIdx.x & 31) != 0 || st.last_slot < 0) return;
  const int ring = pid >> 1;
  int stg = st.last_slot - ring * G::NR;
  uint32_t ph = st.last_phase;
  for (int i = 0; i < G::NR; ++i) {
    const uint32_t a = smem_u32(&s.full[ring * G::NR + stg]);
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(a, ph) && globaltimer_ns() - t0 < 100000000ull) {
    }
    if (--stg < 0) {
      stg = G::NR - 1;
      ph ^= 1;
    }
  }
}

// -------------------------------------------------------------- MMA issuer
// Issuer k (warp 1 or 9) for one phase; `leader` = this warp's elected lane
// (the same lane for the whole kernel, so its commits track its MMAs).
template <int B, bool GU, bool W_MN, class G>
__device__ bool issue(const Bf16Params& p, const Smem& s, uint32_t tmem, IssueState& st, int i_base, int k,
                      bool leader, const Ctl& ctl) {
  constexpr uint32_t IDESC_1 = idesc_bf16(kBM, B, false, W_MN);
  constexpr uint32_t IDESC_2 = idesc_bf16(kBM, 2 * B, false, W_MN);
  constexpr uint64_t kBStep = W_MN ? (2048 >> 4) : (32 >> 4);
  const uint64_t a_desc0 = sdesc_sw128(smem_u32(s.stages), 16, 1024);
  const uint64_t b_desc0 = W_MN ? sdesc_sw128(smem_u32(s.stages) + G::A_BYTES, 8192, 1024)
                                : sdesc_sw128(smem_u32(s.stages) + G::A_BYTES, 16, 1024);
  const int nl = seg_count(p);
  for (int i = (k - i_base) & 1; i < nl; i += 2) {
    const int ik = (i_base + i) >> 1;  // units of this issuer so far
    const int buf = G::NBUF == 2 ? (ik & 1) : 0;
    const uint32_t use = G::NBUF == 2 ? uint32_t(ik >> 1) : uint32_t(ik);
    const int ab = k * 2 + buf;
    if (!__all_sync(0xffffffffu, mbar_wait(&s.acc_empty[ab], (use & 1u) ^ 1u, ctl))) return false;
    tc_fence_after();
    const uint32_t d0 = tmem + uint32_t((k * G::NBUF + buf) * G::ACC_COLS);
    const uint32_t d1 = d0 + B;
    uint32_t init0 = 0, init1 = 0;
    for (bool last = false; !last;) {
      const int slot = k * G::NR + st.stage;
      if (!__all_sync(0xffffffffu, mbar_wait(&s.full[slot], st.phase, ctl))) return false;
      tc_fence_after();
      const uint32_t info = s.stage_info[slot];
      last = (info & kSiLast) != 0;
      const bool has0 = (info & kSiHas0) != 0, has1 = GU && (info & kSiHas1) != 0;
      // stage descriptors = stage-0 descriptors + constant start-address offsets
      const uint64_t ad = a_desc0 + uint64_t(slot) * (G::STAGE_BYTES >> 4);
      const uint64_t bd0 = b_desc0 + uint64_t(slot) * (G::STAGE_BYTES >> 4);
      const uint64_t bd1 = bd0 + (G::W_BYTES >> 4);
      if (leader) {
        if (GU && has0 && has1 && init0 == init1) {  // gate | up side by side: one MMA of N = 2B
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_bf16(d0, ad + 2 * kk, bd0 + kk * kBStep, IDESC_2, kk > 0 ? 1u : init0);
        } else {
          if (has0) {
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              mma_bf16(d0, ad + 2 * kk, bd0 + kk * kBStep, IDESC_1, kk > 0 ? 1u : init0);
          }
          if (has1) {
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              mma_bf16(d1, ad + 2 * kk, bd1 + kk * kBStep, IDESC_1, kk > 0 ? 1u : init1);
          }
        }
        mma_commit(&s.empty[slot]);
      }
      __syncwarp();
      if (has0) init0 = 1;
      if (has1) init1 = 1;
      if (++st.stage == G::NR) {
        st.stage = 0;
        st.phase ^= 1;
      }
    }
    if (leader) mma_commit(&s.acc_full[ab]);
    __syncwarp();
  }
  return true;
}

// Every MMA of this issuer has completed before TMEM is released (always run).
__device__ __forceinline__ void issuer_drain(const Smem& s, int k, bool leader) {
  if (leader) {
    mma_commit(&s.drain[k]);
    const uint32_t a = smem_u32(&s.drain[k]);
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(a, 0) && globaltimer_ns() - t0 < 100000000ull) {
    }
  }
  __syncwarp();
}

// ---------------------------------------------------------------- epilogue
// One epilogue warp (2-5) for one phase: units in CTA order, unit i_base + i
// from issuer (i_base + i) & 1.  GU: out = silu(gate) * up (bf16, optional
// bf16 copies of gate/up); linear: out = acc (+ residual), bf16 or fp32.
// `residual` may alias `out` (each element is read, then written, by the same
// thread).
// SB: copy this lane's row of gate_pre and up_out for unit (m, r) — B
// features each — into slot `slot` of the warp's staging area.  Layout per
// slot: gate rows [32][B*2 bytes] then up rows; 16-byte chunk c of a row sits
// at position c ^ (lane & 7), so the lane-per-row reads hit distinct banks.
template <int B, class G>
__device__ __forceinline__ void stage_gate_up(const Bf16Params& p, const Smem& s, int m, int r, int q, int lane,
                                              int slot) {
  const int64_t row = int64_t(m) * kBM + q * 32 + lane;
  if (row >= p.T) return;
  uint8_t* dst = s.epi + (q * G::EPI_NSLOT + slot) * G::EPI_SLOT + lane * (B * 2);
  const char* g = static_cast<const char*>(p.bwd_gate) + (row * p.ld_bwd + int64_t(r) * B) * 2;
  const char* u = static_cast<const char*>(p.bwd_up) + (row * p.ld_bwd + int64_t(r) * B) * 2;
#pragma unroll
  for (int c = 0; c < B / 8; ++c) {
    const int pos = c ^ (lane & 7);
    cp_async16(dst + pos * 16, g + c * 16);
    cp_async16(dst + 32 * B * 2 + pos * 16, u + c * 16);
  }
}

// SB: the linear's epilogue applies the SiLU*up backward (p.bwd_gate).  At
// B = 64 a lane's staged gate row and up row are 128 bytes with 16-byte chunk
// c at c ^ (lane & 7) — the 128-byte-swizzled layout of a TMA box of 32 rows
// x 64 columns — so d_gate / d_up are written over them in place and leave
// as two TMA stores through `tm_out` ([T, 2 d_ff] bf16, 64 x 32 boxes).
template <int B, bool GU, class G, bool SB = false>
__device__ bool epilogue(const Bf16Params& p, const Smem& s, uint32_t tmem, int i_base, const Ctl& ctl,
                         const CUtensorMap* tm_out = nullptr) {
  static_assert(!(GU && SB), "the SiLU*up backward epilogue is a linear mode");
  constexpr bool TSTORE = SB && B == 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = warp & 3;  // TMEM lane quadrant this warp may access
  const int nl = seg_count(p);
  int cw_next = 0;  // count word of the next unit, loaded one unit ahead
  if (nl > 0) {
    int m0, r0;
    unit_mr(unit_at(p, 0), p, m0, r0);
    cw_next = p.counts[r0];
  }
  for (int i = 0; i < nl; ++i) {
    int m, r;
    unit_mr(unit_at(p, i), p, m, r);
    const int cw = cw_next;
    if (i + 1 < nl) {
      int m2, r2;
      unit_mr(unit_at(p, i + 1), p, m2, r2);
      cw_next = p.counts[r2];
    }
    const int iG = i_base + i;
    const int k = iG & 1, ik = iG >> 1;
    const int buf = G::NBUF == 2 ? (ik & 1) : 0;
    const uint32_t use = G::NBUF == 2 ? uint32_t(ik >> 1) : uint32_t(ik);
    const int ab = k * 2 + buf;
    const int64_t row = int64_t(m) * kBM + q * 32 + lane;
    const bool row_ok = row < p.T;
    // SiLU*up backward: this unit's gate/up rows were copied to shared memory
    // (cp.async, one slot per unit) while the previous unit ran; start the
    // next unit's copy, then wait for this one's (per-thread groups)
    const bool sb = SB && row_ok;
    const uint8_t* gu_row = nullptr;
    if constexpr (SB) {
      if constexpr (G::EPI_NSLOT == 2) {
        if (i == 0) {
          stage_gate_up<B, G>(p, s, m, r, q, lane, 0);
          cp_async_commit();
        }
        if (i + 1 < nl) {
          if constexpr (TSTORE) {  // slot (i+1)&1 is the source of unit i-1's stores
            if (lane == 0) bulk_wait_group_read0();
            __syncwarp();
          }
          int m2, r2;
          unit_mr(unit_at(p, i + 1), p, m2, r2);
          stage_gate_up<B, G>(p, s, m2, r2, q, lane, (i + 1) & 1);
        }
        cp_async_commit();
        cp_async_wait_group<1>();
      } else {  // one slot: this unit's copy overlaps the accumulator wait
        stage_gate_up<B, G>(p, s, m, r, q, lane, 0);
        cp_async_commit();
      }
      gu_row = s.epi + (q * G::EPI_NSLOT + (G::EPI_NSLOT == 2 ? (i & 1) : 0)) * G::EPI_SLOT + lane * (B * 2);
    }
    // dataflow: this thread's own acquire of the writes it is about to read
    // (the sums of squares, the residual) before touching them; done while
    // the unit's MMAs run
    if (p.dep_cnt && !__all_sync(0xffffffffu, wait_count(p.dep_cnt + m, p.dep_target, ctl))) return false;
    if (p.epi_dep_cnt && !__all_sync(0xffffffffu, wait_count(p.epi_dep_cnt + m, p.epi_dep_target, ctl))) return false;
    // folded RMSNorm (GU): 1 / rms of this token row from the partial sums of
    // squares (independent loads, four partial sums, a fixed order)
    float rs = 1.f;
    if (GU && p.row_ss && row_ok) {
      const float* sp = p.row_ss + row * p.ss_parts;
      float a4[4] = {0.f, 0.f, 0.f, 0.f};
      int k2 = 0;
#pragma unroll 4
      for (; k2 + 4 <= p.ss_parts; k2 += 4) {
        a4[0] += sp[k2];
        a4[1] += sp[k2 + 1];
        a4[2] += sp[k2 + 2];
        a4[3] += sp[k2 + 3];
      }
      for (; k2 < p.ss_parts; ++k2) a4[0] += sp[k2];
      rs = rsqrtf(((a4[0] + a4[1]) + (a4[2] + a4[3])) * p.inv_d + p.eps);
    }
    // warp-uniform before the collective tcgen05.ld
    if (!__all_sync(0xffffffffu, mbar_wait(&s.acc_full[ab], use & 1u, ctl))) {
      if constexpr (SB) cp_async_wait_group<0>();  // no copy into shared memory outlives the CTA
      if constexpr (TSTORE) {
        if (lane == 0) bulk_wait_group0();
      }
      return false;
    }
    tc_fence_after();
    const bool any0 = (cw >> 16) & 1;
    const bool any1 = (cw >> 17) & 1;
    if constexpr (SB && G::EPI_NSLOT == 1) cp_async_wait_group<0>();
    float ssq = 0.f;  // linear: squares of this row's stored outputs (folded RMSNorm of the next step)
    const uint32_t tbase = tmem + (uint32_t(q * 32) << 16) + uint32_t((k * G::NBUF + buf) * G::ACC_COLS);
#pragma unroll 1
    for (int j = 0; j < B / 32; ++j) {
      if constexpr (GU) {
        uint32_t g[32], v[32];
        tmem_ld32x2_sync(tbase + j * 32, g, tbase + B + j * 32, v);
        if (!any0 || !any1) {  // a projection with no live tile is zero, so is h
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            if (!any0) g[t] = 0u;
            if (!any1) v[t] = 0u;
          }
        }
        if (p.h_parts) {  // fp32 path on the tensor cores: exact SiLU*up, stored as three bf16 parts
          if (row_ok) {
            __nv_bfloat16* hrow = static_cast<__nv_bfloat16*>(p.out) + row * p.ld_out + int64_t(r) * B + j * 32;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              uint32_t w0[4], w1[4], w2[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int c0 = 8 * t + 2 * e;
                float a0, b0, z0, a1, b1, z1;
                split3_bf16(silu_mul_exact(__uint_as_float(g[c0]) * rs, __uint_as_float(v[c0]) * rs), a0, b0, z0);
                split3_bf16(silu_mul_exact(__uint_as_float(g[c0 + 1]) * rs, __uint_as_float(v[c0 + 1]) * rs), a1, b1,
                            z1);
                w0[e] = pack_bf16x2(a0, a1);
                w1[e] = pack_bf16x2(b0, b1);
                w2[e] = pack_bf16x2(z0, z1);
              }
              st_global_v4(hrow + t * 8, w0[0], w0[1], w0[2], w0[3]);
              st_global_v4(hrow + p.h_parts + t * 8, w1[0], w1[1], w1[2], w1[3]);
              st_global_v4(hrow + 2 * p.h_parts + t * 8, w2[0], w2[1], w2[2], w2[3]);
            }
          }
          continue;
        }
        uint32_t hp[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const float g0 = __uint_as_float(g[2 * t]) * rs, g1 = __uint_as_float(g[2 * t + 1]) * rs;
          const float u0 = __uint_as_float(v[2 * t]) * rs, u1 = __uint_as_float(v[2 * t + 1]) * rs;
          hp[t] = pack_bf16x2(silu_fast(g0) * u0, silu_fast(g1) * u1);
        }
        if (row_ok) {
          const int64_t off = row * p.ld_out + int64_t(r) * B + j * 32;
          __nv_bfloat16* hrow = static_cast<__nv_bfloat16*>(p.out) + off;
#pragma unroll
          for (int t = 0; t < 4; ++t) st_global_v4(hrow + t * 8, hp[4 * t], hp[4 * t + 1], hp[4 * t + 2], hp[4 * t + 3]);
          if (p.gate_pre) {  // optional intermediates: packed only when requested
            __nv_bfloat16* grow = static_cast<__nv_bfloat16*>(p.gate_pre) + off;
#pragma unroll
            for (int t = 0; t < 4; ++t)
              st_global_v4(grow + t * 8, pack_bf16x2(__uint_as_float(g[8 * t]), __uint_as_float(g[8 * t + 1])),
                           pack_bf16x2(__uint_as_float(g[8 * t + 2]), __uint_as_float(g[8 * t + 3])),
                           pack_bf16x2(__uint_as_float(g[8 * t + 4]), __uint_as_float(g[8 * t + 5])),
                           pack_bf16x2(__uint_as_float(g[8 * t + 6]), __uint_as_float(g[8 * t + 7])));
          }
          if (p.up_out) {
            __nv_bfloat16* urow = static_cast<__nv_bfloat16*>(p.up_out) + off;
#pragma unroll
            for (int t = 0; t < 4; ++t)
              st_global_v4(urow + t * 8, pack_bf16x2(__uint_as_float(v[8 * t]), __uint_as_float(v[8 * t + 1])),
                           pack_bf16x2(__uint_as_float(v[8 * t + 2]), __uint_as_float(v[8 * t + 3])),
                           pack_bf16x2(__uint_as_float(v[8 * t + 4]), __uint_as_float(v[8 * t + 5])),
                           pack_bf16x2(__uint_as_float(v[8 * t + 6]), __uint_as_float(v[8 * t + 7])));
          }
        }
      } else {
        uint32_t a[32];
        tmem_ld32_sync(tbase + j * 32, a);
        float f[32];
#pragma unroll
        for (int t = 0; t < 32; ++t) f[t] = any0 ? __uint_as_float(a[t]) : 0.f;
        if (sb) {  // SiLU*up backward: f = d_h; gate/up from this lane's staged row
          const int64_t col = int64_t(r) * B + j * 32;
          __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.out) + row * p.ld_out + col;
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int c = (j * 4 + t) ^ (lane & 7);  // swizzled 16-byte chunk
            const uint4 gv = *reinterpret_cast<const uint4*>(gu_row + c * 16);
            const uint4 uv = *reinterpret_cast<const uint4*>(gu_row + 32 * B * 2 + c * 16);
            const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
            uint32_t og[4], ou[4];
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              const float2 g2 = unpack_bf16x2(gw[w]), u2 = unpack_bf16x2(uw[w]);
              float dg0, du0, dg1, du1;
              silu_mul_grad(f[8 * t + 2 * w], g2.x, u2.x, dg0, du0);
              silu_mul_grad(f[8 * t + 2 * w + 1], g2.y, u2.y, dg1, du1);
              og[w] = pack_bf16x2(dg0, dg1);
              ou[w] = pack_bf16x2(du0, du1);
            }
            if constexpr (TSTORE) {  // in place over the staged gate / up chunk
              *reinterpret_cast<uint4*>(const_cast<uint8_t*>(gu_row) + c * 16) = make_uint4(og[0], og[1], og[2], og[3]);
              *reinterpret_cast<uint4*>(const_cast<uint8_t*>(gu_row) + 32 * B * 2 + c * 16) =
                  make_uint4(ou[0], ou[1], ou[2], ou[3]);
            } else {
              st_global_v4(orow + t * 8, og[0], og[1], og[2], og[3]);
              st_global_v4(orow + p.du_off + t * 8, ou[0], ou[1], ou[2], ou[3]);
            }
          }
        } else if (row_ok) {
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
              st_global_v4(orow + t * 4, __float_as_uint(f[4 * t]), __float_as_uint(f[4 * t + 1]),
                           __float_as_uint(f[4 * t + 2]), __float_as_uint(f[4 * t + 3]));
          } else {
            __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.out) + off;
            uint32_t ow[16];
#pragma unroll
            for (int t = 0; t < 16; ++t) ow[t] = pack_bf16x2(f[2 * t], f[2 * t + 1]);
#pragma unroll
            for (int t = 0; t < 4; ++t) st_global_v4(orow + t * 8, ow[4 * t], ow[4 * t + 1], ow[4 * t + 2], ow[4 * t + 3]);
            if (p.ss_out) {
#pragma unroll
              for (int t = 0; t < 16; ++t) {
                const float2 r2 = unpack_bf16x2(ow[t]);
                ssq = fmaf(r2.x, r2.x, fmaf(r2.y, r2.y, ssq));
              }
            }
          }
        }
      }
    }
    if (!GU && p.ss_out && row_ok) p.ss_out[row * p.ss_parts + r] = ssq;
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&s.acc_empty[ab]);
    if (p.sig_cnt) signal_count(p.sig_cnt + m);  // dataflow: this warp's rows of the unit are stored
    if constexpr (TSTORE) {  // this warp's 32 rows of d_gate and d_up, out of the staging slot
      const int64_t row0 = int64_t(m) * kBM + q * 32;
      fence_proxy_async_smem();  // the in-place writes above -> visible to the TMA engine
      __syncwarp();
      if (lane == 0 && row0 < p.T) {  // rows past T are clipped by the map
        const uint8_t* slot = s.epi + (q * G::EPI_NSLOT + (G::EPI_NSLOT == 2 ? (i & 1) : 0)) * G::EPI_SLOT;
        tma_store_2d(tm_out, slot, int32_t(r) * B, int32_t(row0));
        tma_store_2d(tm_out, slot + 32 * B * 2, int32_t(p.du_off + int64_t(r) * B), int32_t(row0));
        bulk_commit_group();
      }
      __syncwarp();
    }
  }
  if constexpr (TSTORE) {
    if (lane == 0) bulk_wait_group0();
  }
  return true;
}

}  // namespace eng
}  // namespace bell
