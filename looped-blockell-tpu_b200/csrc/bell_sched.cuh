// bell_sched.cuh — how the warp roles of the Block-ELL kernels learn their
// work without waiting on global memory in the issue loops.
//
// A plan row (the steps of one output block-row) is fetched by a whole warp
// one work unit ahead into registers (lane l holds entries l, l+32, ...) and
// put into shared memory when its unit starts, so the single issuing thread
// reads its steps from shared memory.  The producer tells the MMA issuer what
// each stage holds through a stage-info word written next to the stage
// before its `full` barrier is armed; the MMA issuer never reads the plan.
// A unit with no live step still gets one (empty) stage, so the MMA issuer
// commits its accumulator and the epilogue sees the unit.
#pragma once

#include <cstdint>

namespace bell {

enum : uint32_t {
  kSiHas0 = 1u,   // the stage holds a tile of weight 0 (gate / the only weight)
  kSiHas1 = 2u,   // the stage holds a tile of weight 1 (up)
  kSiFirst = 4u,  // first stage of a unit
  kSiLast = 8u,   // last stage of a unit
  kSiRes = 16u,   // residual stage (feature-major linear kernel)
};

// Largest plan row (entries) a warp stages: K_gate + K_up <= 2 * 254.
static constexpr int kRowRegs = 16;
static constexpr int kRowMax = 32 * kRowRegs;

struct RowAhead {
  uint32_t v[kRowRegs];
  int32_t cnt;
};

// Issue the loads of plan row r (all lanes of the warp); the values are
// consumed by row_put one unit later, so the load latency is hidden.
__device__ __forceinline__ void row_fetch(RowAhead& a, const uint32_t* plan, const int32_t* counts, int S, int r) {
  const int lane = threadIdx.x & 31;
  a.cnt = counts[r];
  const uint32_t* row = plan + size_t(r) * size_t(S);
#pragma unroll
  for (int t = 0; t < kRowRegs; ++t) {
    const int j = lane + 32 * t;
    a.v[t] = j < S ? row[j] : 0u;
  }
}

__device__ __forceinline__ void row_put(const RowAhead& a, uint32_t* dst, int S) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int t = 0; t < kRowRegs; ++t) {
    const int j = lane + 32 * t;
    if (j < S) dst[j] = a.v[t];
  }
}

}  // namespace bell
