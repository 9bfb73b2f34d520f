// ref_attn.cu -- builds the reference's attention source file where it lies
// (REF_ATTN_SRC, given by the Makefile) for sm_100a and exports a C-ABI
// launcher for its naive_attn_kernel (src/attn_sm75.cu:55-94), the
// reference's own correctness oracle.  TEST INFRASTRUCTURE ONLY: the GPU
// parity tests use it to pin the fp64 CPU restatement in oracle.c.
//
// Layout: Q,K,V,O fp16 [B*H][S][D] on the device.  One block per (b,h) with
// S threads, so S <= 1024, the reference's own limit (src/attn_sm75.cu:457).
#define main reference_attn_main
#include REF_ATTN_SRC
#undef main

extern "C" int ref_naive_attn(const void* Q, const void* K, const void* V, void* O, int BH,
                              int S, int D, float scale, int causal) {
    if (BH < 1 || S < 1 || S > 1024 || D < 1) return -1;
    naive_attn_kernel<<<BH, S>>>(static_cast<const half*>(Q), static_cast<const half*>(K),
                                 static_cast<const half*>(V), static_cast<half*>(O), S, D,
                                 scale, causal);
    if (cudaGetLastError() != cudaSuccess) return -3;
    if (cudaDeviceSynchronize() != cudaSuccess) return -3;
    return 0;
}
