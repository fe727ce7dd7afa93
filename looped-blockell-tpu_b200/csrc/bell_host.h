// bell_host.h — host-side helpers shared by the entry points: error state,
// device info, tensor-map encoding, launch checks.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>

#include "../../include/bell.h"

namespace bell {

// Record `code` with a message as this thread's last error and return it.
int fail(int code, const std::string& msg);
int ok();

// SM count / sm_100 check of the current device (cached per device).
int device_sm_count(int* sm_count);
int require_sm100();

// Library-owned status word of the current device (statically allocated
// __device__ int; no cudaMalloc).
int32_t* default_status_ptr();

// Encode a 2-D tiled tensor map: `inner` contiguous elements per row,
// `outer` rows, `pitch_bytes` between rows, box = box_inner x box_outer.
enum class MapType { BF16, INT8, F32 };
enum class Swz { NONE, B32, B64, B128 };
int make_map_2d(CUtensorMap* map, const void* base, MapType type, uint64_t inner, uint64_t outer,
                uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer, Swz swz, bool l2_256 = true);

// Check the last launch; maps errors to BELL_ERR_LAUNCH with a message.
int check_launch(const char* what);

// Set the max dynamic shared memory of `func` (once per device).
int set_smem(const void* func, int bytes);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Plan workspace layout (all offsets 16-byte aligned).
struct PlanLayout {
  size_t gu_entries, gu_counts, d_entries, d_counts, total;
};
PlanLayout plan_layout(int32_t R_gu, int32_t K_g, int32_t K_u, int32_t R_d, int32_t K_d);

// Launch the plan kernel (defined in bell_plan.cu).
int launch_plan(const int32_t* ci_g, int32_t K_g, const int32_t* ci_u, int32_t K_u, int32_t R_gu,
                int32_t C_gu, const int32_t* ci_d, int32_t K_d, int32_t R_d, int32_t C_d, void* plan,
                int32_t* status, cudaStream_t stream);
// merge = 0: gate slots then up slots, each in ascending slot order, never
// sharing a step (the ternary path needs that exact per-matrix order).
int launch_plan_ex(const int32_t* ci_g, int32_t K_g, const int32_t* ci_u, int32_t K_u, int32_t R_gu,
                   int32_t C_gu, const int32_t* ci_d, int32_t K_d, int32_t R_d, int32_t C_d, void* plan,
                   int32_t* status, cudaStream_t stream, int32_t merge);

// bf16 building blocks (bell_bf16.cu): descriptor checks, the gate/up launch
// and the down (linear + residual) launch, on an already-built plan.
int check_ffn(const BellFFNDesc* d, int dtype);
int launch_ffn_plan(const BellFFNDesc* d, int32_t* status, cudaStream_t s);
// pdl: launch with programmatic stream serialization (honoured by the tile-64/
// 128 token-major engine, which waits for its predecessor after its set-up).
// ld_h > 0: row stride of h in elements (default d_ff); h_parts > 0: write
// h as three bf16 parts of the exact fp32 value (tile 64 only, see Bf16Params).
int gate_up_bf16(const BellFFNDesc* d, int32_t* status, cudaStream_t s, bool pdl = false, int64_t ld_h = 0,
                 int64_t h_parts = 0);
int down_bf16(const BellFFNDesc* d, int32_t* status, cudaStream_t s, bool pdl = false);

// Workspace of the loop: per-tile counters, per-row partial sums of squares
// and the gain-scaled gate/up tiles (tile size 64; other sizes need none).
struct LoopWs {
  size_t counters, ss, wg, wu, total;
};
LoopWs loop_ws(int64_t T, int32_t d_model, int32_t R_gu, int32_t K_g, int32_t K_u, int32_t B);
// Weight tensor map of a bf16 Block-ELL matrix: 64 x 64 boxes, 128-byte swizzle.
int make_w_map(CUtensorMap* m, const BellEll& e);

// The L-iteration loop as one persistent cooperative kernel (tile size 64;
// bell_loop_kernel.cu).  h_out must already hold h_in and the plan be built.
int loop_persistent_bf16(const BellLoopDesc* d, const BellEll& wg, const BellEll& wu, int32_t* status,
                         cudaStream_t s);

// Wait budget for device-side bounded waits (ns).
uint64_t wait_budget_ns();

}  // namespace bell
