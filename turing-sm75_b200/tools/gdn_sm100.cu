// gdn_sm100 -- command-line drop-in for the reference's gdn_sm75 binary
// (src/gdn_sm75.cu:1246-1412), running the sm_100a kernels through the C ABI.
//
//   gdn_sm100 [T] [--hq N] [--hv N] [--b N] [--iters N]
//
// Same positional argument (T, default 64, 1..2048), shape defaults (Sv=128,
// Hq=16, Hv=48, v-head h reads q/k head h % Hq), input generator (the LCG of
// src/gdn_sm75.cu:1270-1279, drawn in the order q, k, v, g, beta), scale
// 1/sqrt(128), report lines and exit codes (0 = all variants within 2e-2 of
// the CPU recurrence, 1 = a variant failed, 2 = usage).  q/k/v go to the
// library as fp32, the reference kernels' const float* (the prefill rounds
// them to bf16 copies in its workspace), and the CPU check runs on the same
// unrounded values.  Variants:
//   prefill  gdn_prefill_sm100 (chunked, tcgen05)
//   decode   gdn_decode_sm100 called once per token (token-serial)
// Unlike the reference, the final state is checked too.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
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

static constexpr int kSv = 128;

// CPU token-serial recurrence (src/gdn_sm75.cu:6-11) in double, used as the check.
static void cpu_recurrence(const std::vector<float>& q, const std::vector<float>& k,
                           const std::vector<float>& v, const std::vector<float>& g,
                           const std::vector<float>& b, std::vector<double>& S,
                           std::vector<double>& out, int B, int T, int Hq, int Hv, float scale) {
    for (int bb = 0; bb < B; ++bb)
        for (int h = 0; h < Hv; ++h) {
            const int hq = h % Hq;
            double* Sh = S.data() + ((size_t)bb * Hv + h) * kSv * kSv;
            for (int t = 0; t < T; ++t) {
                const size_t bt = (size_t)bb * T + t;
                const float* qt = q.data() + (bt * Hq + hq) * kSv;
                const float* kt = k.data() + (bt * Hq + hq) * kSv;
                const float* vt = v.data() + (bt * Hv + h) * kSv;
                const double gg = std::exp((double)g[bt * Hv + h]);
                const double be = b[bt * Hv + h];
                for (int c = 0; c < kSv; ++c) {
                    double* row = Sh + (size_t)c * kSv;
                    double kv = 0;
                    for (int i = 0; i < kSv; ++i) kv += row[i] * kt[i];
                    const double d = (vt[c] - gg * kv) * be;
                    double o = 0;
                    for (int i = 0; i < kSv; ++i) {
                        row[i] = gg * row[i] + kt[i] * d;
                        o += row[i] * qt[i];
                    }
                    out[(bt * Hv + h) * kSv + c] = o * scale;
                }
            }
        }
}

int main(int argc, char** argv) {
    int T = 64, Hq = 16, Hv = 48, B = 1, iters = 20;
    std::vector<int> pos;
    for (int i = 1; i < argc; ++i) {
        std::string a = argv[i];
        if (a == "--hq" && i + 1 < argc) Hq = std::atoi(argv[++i]);
        else if (a == "--hv" && i + 1 < argc) Hv = std::atoi(argv[++i]);
        else if (a == "--b" && i + 1 < argc) B = std::atoi(argv[++i]);
        else if (a == "--iters" && i + 1 < argc) iters = std::atoi(argv[++i]);
        else if (!a.empty() && a[0] != '-') pos.push_back(std::atoi(a.c_str()));
        else pos.push_back(-1);
    }
    if (pos.size() == 1) T = pos[0];
    if (pos.size() > 1 || T < 1 || T > 2048 || Hq < 1 || Hv < 1 || B < 1 || iters < 1) {
        fprintf(stderr, "usage: %s [T] [--hq N] [--hv N] [--b N] [--iters N]   (1 <= T <= 2048)\n", argv[0]);
        return 2;
    }
    cudaDeviceProp prop{};
    CHECK_CUDA(cudaGetDeviceProperties(&prop, 0));
    printf("GPU             : %s  (sm_%d%d)\n", prop.name, prop.major, prop.minor);
    printf("GDN shape       : Sv=%d  Hq=%d  Hv=%d  T=%d  B=%d  chunk=64\n", kSv, Hq, Hv, T, B);

    const float scale = 1.f / std::sqrt((float)kSv);
    const size_t nq = (size_t)B * T * Hq * kSv, nv = (size_t)B * T * Hv * kSv, ng = (size_t)B * T * Hv;
    const size_t ns = (size_t)B * Hv * kSv * kSv;
    std::vector<float> q(nq), k(nq), v(nv), g(ng), bt(ng);
    unsigned seed = 1;
    auto rnd = [&]() {
        seed = seed * 1664525u + 1013904223u;
        return ((seed >> 8) / 16777216.f) - 0.5f;
    };
    for (auto& x : q) x = rnd() * 0.2f;
    for (auto& x : k) x = rnd() * 0.2f;
    for (auto& x : v) x = rnd() * 0.2f;
    for (auto& x : g) x = -0.2f + rnd() * 0.05f;
    for (auto& x : bt) x = 0.4f + (rnd() + 0.5f) * 0.4f;

    std::vector<double> S_ref(ns, 0.0), o_ref(nv);
    cpu_recurrence(q, k, v, g, bt, S_ref, o_ref, B, T, Hq, Hv, scale);

    float *dq, *dk, *dv;
    float *dg, *db, *dS, *dO;
    CHECK_CUDA(cudaMalloc(&dq, nq * 4));
    CHECK_CUDA(cudaMalloc(&dk, nq * 4));
    CHECK_CUDA(cudaMalloc(&dv, nv * 4));
    CHECK_CUDA(cudaMalloc(&dg, ng * 4));
    CHECK_CUDA(cudaMalloc(&db, ng * 4));
    CHECK_CUDA(cudaMalloc(&dS, ns * 4));
    CHECK_CUDA(cudaMalloc(&dO, nv * 4));
    CHECK_CUDA(cudaMemcpy(dq, q.data(), nq * 4, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(dk, k.data(), nq * 4, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(dv, v.data(), nv * 4, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(dg, g.data(), ng * 4, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(db, bt.data(), ng * 4, cudaMemcpyHostToDevice));
    const size_t ws_bytes = gdn_prefill_sm100_workspace_ex(B, T, Hq, Hv, kSv, kSv, B200LAB_F32);
    void* ws = nullptr;
    CHECK_CUDA(cudaMalloc(&ws, ws_bytes));

    // token-serial variant: gdn_decode_sm100 per token on strided views needs contiguous
    // per-token tensors, so the inputs are regrouped [t][b][...] once.
    float *tq, *tk, *tv;
    float *tg, *tb, *tO;
    CHECK_CUDA(cudaMalloc(&tq, nq * 4));
    CHECK_CUDA(cudaMalloc(&tk, nq * 4));
    CHECK_CUDA(cudaMalloc(&tv, nv * 4));
    CHECK_CUDA(cudaMalloc(&tg, ng * 4));
    CHECK_CUDA(cudaMalloc(&tb, ng * 4));
    CHECK_CUDA(cudaMalloc(&tO, nv * 4));
    for (int bb = 0; bb < B; ++bb)
        for (int t = 0; t < T; ++t) {
            const size_t src = (size_t)bb * T + t, dst = (size_t)t * B + bb;
            CHECK_CUDA(cudaMemcpy(tq + dst * Hq * kSv, dq + src * Hq * kSv, Hq * kSv * 4, cudaMemcpyDeviceToDevice));
            CHECK_CUDA(cudaMemcpy(tk + dst * Hq * kSv, dk + src * Hq * kSv, Hq * kSv * 4, cudaMemcpyDeviceToDevice));
            CHECK_CUDA(cudaMemcpy(tv + dst * Hv * kSv, dv + src * Hv * kSv, Hv * kSv * 4, cudaMemcpyDeviceToDevice));
            CHECK_CUDA(cudaMemcpy(tg + dst * Hv, dg + src * Hv, Hv * 4, cudaMemcpyDeviceToDevice));
            CHECK_CUDA(cudaMemcpy(tb + dst * Hv, db + src * Hv, Hv * 4, cudaMemcpyDeviceToDevice));
        }

    auto prefill = [&]() {
        return gdn_prefill_sm100(dq, dk, dv, dg, db, dS, dO, B, T, Hq, Hv, kSv, kSv, 0, scale,
                                 B200LAB_F32, B200LAB_F32, ws, ws_bytes, nullptr);
    };
    auto serial = [&]() {
        int st = B200LAB_OK;
        for (int t = 0; t < T && st == B200LAB_OK; ++t)
            st = gdn_decode_sm100(tq + (size_t)t * B * Hq * kSv, tk + (size_t)t * B * Hq * kSv,
                                  tv + (size_t)t * B * Hv * kSv, tg + (size_t)t * B * Hv,
                                  tb + (size_t)t * B * Hv, dS, tO + (size_t)t * B * Hv * kSv, B, Hq,
                                  Hv, kSv, kSv, 0, scale, B200LAB_F32, B200LAB_F32, nullptr);
        return st;
    };

    std::vector<float> o(nv), S(ns);
    float worst = 0.f;
    auto bench = [&](auto fn, const char* name, bool token_major) -> int {
        CHECK_CUDA(cudaMemset(dS, 0, ns * 4));
        int st = fn();
        if (st == B200LAB_OK) st = b200lab_device_status(nullptr);
        if (st != B200LAB_OK) {
            fprintf(stderr, "%s: %s\n", name, b200lab_strerror(st));
            worst = INFINITY;
            return 1;
        }
        CHECK_CUDA(cudaMemcpy(o.data(), token_major ? tO : dO, nv * 4, cudaMemcpyDeviceToHost));
        CHECK_CUDA(cudaMemcpy(S.data(), dS, ns * 4, cudaMemcpyDeviceToHost));
        float eo = 0.f, es = 0.f;
        for (int bb = 0; bb < B; ++bb)
            for (int t = 0; t < T; ++t)
                for (int j = 0; j < Hv * kSv; ++j) {
                    const size_t ri = ((size_t)bb * T + t) * Hv * kSv + j;
                    const size_t gi = token_major ? ((size_t)t * B + bb) * Hv * kSv + j : ri;
                    eo = std::max(eo, (float)std::fabs(o[gi] - o_ref[ri]));
                }
        for (size_t i = 0; i < ns; ++i) es = std::max(es, (float)std::fabs(S[i] - S_ref[i]));
        printf("max |%s-cpu| : out %.6f  state %.6f   %s\n", name, eo, es,
               (eo < 2e-2f && es < 2e-2f) ? "OK" : "FAIL");
        worst = std::max(worst, std::max(eo, es));
        cudaEvent_t e0, e1;
        CHECK_CUDA(cudaEventCreate(&e0));
        CHECK_CUDA(cudaEventCreate(&e1));
        CHECK_CUDA(cudaEventRecord(e0));
        for (int i = 0; i < iters; ++i) fn();
        CHECK_CUDA(cudaEventRecord(e1));
        CHECK_CUDA(cudaEventSynchronize(e1));
        float ms = 0.f;
        CHECK_CUDA(cudaEventElapsedTime(&ms, e0, e1));
        ms /= iters;
        printf("%-16s: %8.4f ms   x48 layers %8.3f ms   %.3g tok/s\n", name, ms, ms * 48,
               (double)B * T / (ms * 1e-3));
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        return 0;
    };
    bench(prefill, "prefill", false);
    bench(serial, "decode-serial", true);

    cudaFree(dq); cudaFree(dk); cudaFree(dv); cudaFree(dg); cudaFree(db); cudaFree(dS); cudaFree(dO);
    cudaFree(tq); cudaFree(tk); cudaFree(tv); cudaFree(tg); cudaFree(tb); cudaFree(tO); cudaFree(ws);
    return worst < 2e-2f ? 0 : 1;
}
