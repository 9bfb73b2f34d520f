// attn_sm100 -- command-line drop-in for the reference's attn_sm75 binary
// (src/attn_sm75.cu:442-554), running the sm_100a kernel through the C ABI.
//
//   attn_sm100 [B H S D] [--causal 0|1] [--hkv N] [--bf16] [--iters N] [--no-check]
//
// Same positional arguments, defaults (B=2 H=8 S=512 D=128, causal, scale
// 1/sqrt(D)), input generator (std::mt19937(42), N(0, 0.5) per tensor, fp16),
// report lines and exit codes (0 = PASS, 1 = FAIL, 2 = usage) as the
// reference.  The correctness check compares against a naive on-device
// kernel of this tool (one thread per query row, fp32), with the reference's
// bar max-abs < 2e-2; like the reference it needs S <= 1024.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "../../include/b200lab.h"

#define CHECK_CUDA(x)                                                                 \
    do {                                                                              \
        cudaError_t e_ = (x);                                                         \
        if (e_ != cudaSuccess) {                                                      \
            fprintf(stderr, "CUDA %s:%d: %s\n", __FILE__, __LINE__, cudaGetErrorString(e_)); \
            return 1;                                                                 \
        }                                                                             \
    } while (0)

template <typename T> __device__ float tof(T x);
template <> __device__ float tof<__half>(__half x) { return __half2float(x); }
template <> __device__ float tof<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> __device__ T fromf(float x);
template <> __device__ __half fromf<__half>(float x) { return __float2half(x); }
template <> __device__ __nv_bfloat16 fromf<__nv_bfloat16>(float x) { return __float2bfloat16(x); }

// Naive check kernel: block = one (b, q-head), thread = one query row.
// Pass 1: row max of the scaled scores; pass 2: softmax-weighted V sum.
template <typename T, int D>
__global__ void __launch_bounds__(1024) naive_check_kernel(const T* Q, const T* K, const T* V, T* O, int Hq, int Hkv, int S,
                                   float scale, int causal) {
    const int bh = blockIdx.x;
    const int b = bh / Hq, h = bh % Hq;
    const int hk = h / (Hq / Hkv);
    const int qi = threadIdx.x;
    if (qi >= S) return;
    const T* q = Q + ((size_t)bh * S + qi) * D;
    const T* Kh = K + ((size_t)b * Hkv + hk) * S * D;
    const T* Vh = V + ((size_t)b * Hkv + hk) * S * D;
    const int nk = causal ? qi + 1 : S;
    float m = -INFINITY;
    for (int j = 0; j < nk; ++j) {
        float dot = 0.f;
        for (int d = 0; d < D; ++d) dot += tof(q[d]) * tof(Kh[(size_t)j * D + d]);
        m = fmaxf(m, dot * scale);
    }
    float acc[D];
    for (int d = 0; d < D; ++d) acc[d] = 0.f;
    float l = 0.f;
    for (int j = 0; j < nk; ++j) {
        float dot = 0.f;
        for (int d = 0; d < D; ++d) dot += tof(q[d]) * tof(Kh[(size_t)j * D + d]);
        const float p = expf(dot * scale - m);
        l += p;
        for (int d = 0; d < D; ++d) acc[d] += p * tof(Vh[(size_t)j * D + d]);
    }
    T* o = O + ((size_t)bh * S + qi) * D;
    for (int d = 0; d < D; ++d) o[d] = fromf<T>(acc[d] / l);
}

template <typename T>
static int run(int B, int H, int Hkv, int S, int D, int causal, int iters, bool check, int dtype) {
    const float scale = 1.f / std::sqrt(static_cast<float>(D));
    const size_t nq = (size_t)B * H * S * D, nkv = (size_t)B * Hkv * S * D;
    std::mt19937 rng(42);
    auto make = [&](size_t n) {
        std::normal_distribution<float> dist(0.f, 0.5f);  // a fresh distribution per tensor
        std::vector<T> h(n);
        for (size_t i = 0; i < n; ++i) h[i] = T(dist(rng));
        return h;
    };
    std::vector<T> hQ = make(nq), hK = make(nkv), hV = make(nkv);
    T *Q, *K, *V, *O, *On;
    CHECK_CUDA(cudaMalloc(&Q, nq * sizeof(T)));
    CHECK_CUDA(cudaMalloc(&K, nkv * sizeof(T)));
    CHECK_CUDA(cudaMalloc(&V, nkv * sizeof(T)));
    CHECK_CUDA(cudaMalloc(&O, nq * sizeof(T)));
    CHECK_CUDA(cudaMalloc(&On, nq * sizeof(T)));
    CHECK_CUDA(cudaMemcpy(Q, hQ.data(), nq * sizeof(T), cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(K, hK.data(), nkv * sizeof(T), cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(V, hV.data(), nkv * sizeof(T), cudaMemcpyHostToDevice));
    const size_t ws_bytes = attn_fwd_sm100_workspace(B, H, Hkv, S, S, D, causal);
    void* ws = nullptr;
    if (ws_bytes) CHECK_CUDA(cudaMalloc(&ws, ws_bytes));

    auto fast = [&]() {
        return attn_fwd_sm100(Q, K, V, O, B, H, Hkv, S, S, D, scale, causal, dtype, ws, ws_bytes, nullptr);
    };
    int st = fast();
    if (st != B200LAB_OK) {
        fprintf(stderr, "attn_fwd_sm100: %s\n", b200lab_strerror(st));
        return 1;
    }
    st = b200lab_device_status(nullptr);
    if (st != B200LAB_OK) {
        fprintf(stderr, "device status: %s\n", b200lab_strerror(st));
        return 1;
    }
    float err = 0.f;
    if (check) {
        if (D == 64)
            naive_check_kernel<T, 64><<<B * H, S>>>(Q, K, V, On, H, Hkv, S, scale, causal);
        else if (D == 128)
            naive_check_kernel<T, 128><<<B * H, S>>>(Q, K, V, On, H, Hkv, S, scale, causal);
        else
            naive_check_kernel<T, 256><<<B * H, S>>>(Q, K, V, On, H, Hkv, S, scale, causal);
        CHECK_CUDA(cudaGetLastError());
        CHECK_CUDA(cudaDeviceSynchronize());
        std::vector<T> a(nq), r(nq);
        CHECK_CUDA(cudaMemcpy(a.data(), O, nq * sizeof(T), cudaMemcpyDeviceToHost));
        CHECK_CUDA(cudaMemcpy(r.data(), On, nq * sizeof(T), cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < nq; ++i) err = std::max(err, std::fabs(float(a[i]) - float(r[i])));
        printf("max |tcgen05-naive| : %.5f   %s\n", err, err < 2e-2f ? "OK" : "FAIL");
    }
    cudaEvent_t e0, e1;
    CHECK_CUDA(cudaEventCreate(&e0));
    CHECK_CUDA(cudaEventCreate(&e1));
    for (int i = 0; i < 3; ++i) fast();  // warm-up (the reference times cold)
    CHECK_CUDA(cudaEventRecord(e0));
    for (int i = 0; i < iters; ++i) fast();
    CHECK_CUDA(cudaEventRecord(e1));
    CHECK_CUDA(cudaEventSynchronize(e1));
    float ms = 0.f;
    CHECK_CUDA(cudaEventElapsedTime(&ms, e0, e1));
    ms /= iters;
    const double dense = 4.0 * B * H * (double)S * S * D;
    const double exec = causal ? 2.0 * B * H * (double)S * (S + 1.0) * D : dense;
    printf("tcgen05 (sm_100a) : %8.4f ms   %7.1f TFLOP/s dense-eq   %7.1f %s\n", ms,
           dense / (ms * 1e-3) / 1e12, exec / (ms * 1e-3) / 1e12, causal ? "causal-exec" : "exec");
    cudaFree(Q);
    cudaFree(K);
    cudaFree(V);
    cudaFree(O);
    cudaFree(On);
    if (ws) cudaFree(ws);
    return (check && !(err < 2e-2f)) ? 1 : 0;
}

int main(int argc, char** argv) {
    int B = 2, H = 8, S = 512, D = 128, causal = 1, Hkv = -1, iters = 20;
    bool bf16 = false, check = true;
    std::vector<int> pos;
    for (int i = 1; i < argc; ++i) {
        std::string a = argv[i];
        if (a == "--causal" && i + 1 < argc) causal = std::atoi(argv[++i]);
        else if (a == "--hkv" && i + 1 < argc) Hkv = std::atoi(argv[++i]);
        else if (a == "--iters" && i + 1 < argc) iters = std::atoi(argv[++i]);
        else if (a == "--bf16") bf16 = true;
        else if (a == "--no-check") check = false;
        else if (!a.empty() && a[0] != '-') pos.push_back(std::atoi(a.c_str()));
        else {
            fprintf(stderr, "usage: %s [B H S D] [--causal 0|1] [--hkv N] [--bf16] [--iters N] [--no-check]\n", argv[0]);
            return 2;
        }
    }
    if (pos.size() == 4) {
        B = pos[0]; H = pos[1]; S = pos[2]; D = pos[3];
    } else if (!pos.empty()) {
        fprintf(stderr, "usage: %s [B H S D]\n", argv[0]);
        return 2;
    }
    if (Hkv < 0) Hkv = H;
    if (D != 64 && D != 128 && D != 256) {
        fprintf(stderr, "D=64, 128 and 256 only\n");
        return 2;
    }
    if (B < 1 || H < 1 || S < 1 || Hkv < 1 || H % Hkv || iters < 1 || (causal != 0 && causal != 1)) {
        fprintf(stderr, "bad shape\n");
        return 2;
    }
    if (check && S > 1024) {
        fprintf(stderr, "naive check is O(S^2 D); keep S <= 1024 (or pass --no-check)\n");
        return 2;
    }
    cudaDeviceProp prop{};
    CHECK_CUDA(cudaGetDeviceProperties(&prop, 0));
    printf("GPU             : %s  (sm_%d%d)\n", prop.name, prop.major, prop.minor);
    printf("shape           : B=%d H=%d Hkv=%d S=%d D=%d  causal=%d  %s\n", B, H, Hkv, S, D, causal,
           bf16 ? "bf16" : "fp16");
    if (D == 256)
        printf("tile            : 128x64 tcgen05.mma, S double-buffered in TMEM, TMA 128B-swizzled K/V ring\n");
    else
        printf("tile            : 128x128 tcgen05.mma (TMEM accumulators), TMA 128B-swizzled K/V ring\n");
    return bf16 ? run<__nv_bfloat16>(B, H, Hkv, S, D, causal, iters, check, B200LAB_BF16)
                : run<__half>(B, H, Hkv, S, D, causal, iters, check, B200LAB_F16);
}
