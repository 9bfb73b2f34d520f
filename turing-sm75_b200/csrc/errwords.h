// errwords.h -- each kernel translation unit owns one device error word
// (a static __device__ int).  These host functions read it back, clear it and
// return its value (B200LAB_OK when no kernel of that unit gave up a wait);
// B200LAB_ERR_CUDA when the copy itself failed.
#pragma once
namespace b200 {
int take_err_attn();
int take_err_attn_gated();
int take_err_gdn_prefill();
int take_err_gdn_decode();
int take_err_watchdog();
}  // namespace b200

// Defines take_err_<name>() for the translation unit's error word `sym`.
#define B200_DEFINE_ERR_TAKER(name, sym)                                              \
    namespace b200 {                                                                 \
    int take_err_##name() {                                                          \
        int v = 0, z = 0;                                                            \
        if (cudaMemcpyFromSymbol(&v, sym, sizeof(int)) != cudaSuccess) return B200LAB_ERR_CUDA; \
        if (v != 0 && cudaMemcpyToSymbol(sym, &z, sizeof(int)) != cudaSuccess)       \
            return B200LAB_ERR_CUDA;                                                 \
        return v;                                                                    \
    }                                                                                \
    }
