// placeholder replaced below
#include "common.cuh"
#include "errwords.h"
namespace b200 { namespace { __device__ int g_err_gdn_prefill = 0; } }
B200_DEFINE_ERR_TAKER(gdn_prefill, b200::g_err_gdn_prefill)
extern "C" size_t gdn_prefill_sm100_workspace(int, int, int, int, int, int) { return 0; }
extern "C" int gdn_prefill_sm100(const void*, const void*, const void*, const float*, const float*,
                                 float*, void*, int, int, int, int, int, int, int, float, int, int,
                                 void*, size_t, void*) { return B200LAB_ERR_UNSUPPORTED; }
