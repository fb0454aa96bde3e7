// Device copies of the integer-exp2 constants (exp2_tables.h), one per translation unit.
#pragma once
#include <stdint.h>

#include "exp2_tables.h"

namespace ea {
static __device__ const uint64_t g_ta64[256] = EA_EXP2_TA64_INIT;
static __device__ const uint64_t g_tb64[256] = EA_EXP2_TB64_INIT;
static __device__ const uint64_t g_ta128[512] = EA_EXP2_TA128_INIT;
static __device__ const uint64_t g_tb128[512] = EA_EXP2_TB128_INIT;
}  // namespace ea
