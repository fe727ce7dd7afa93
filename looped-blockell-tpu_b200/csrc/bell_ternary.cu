// bell_ternary.cu — ternary (2-bit weights, int8 activations) Block-ELL SwiGLU.
#include "bell_host.h"
#include "bell_ptx.cuh"

using namespace bell;

extern "C" int bell_swiglu_fwd_ternary(const BellTernaryFFNDesc* d, void* stream) {
  (void)stream;
  if (!d) return fail(BELL_ERR_ARG, "descriptor is NULL");
  return fail(BELL_ERR_DTYPE, "ternary path not available in this build");
}
