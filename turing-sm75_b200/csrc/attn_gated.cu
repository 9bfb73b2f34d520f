// attn_gated.cu -- softmax attention forward with head dim 256 and an optional output
// gate, for sm_100a (tcgen05 + TMEM + TMA).
//
//   O = (softmax(scale * Q K^T, causal k <= q) V) * sigmoid(G)      (G optional)
//
// The softmax semantics are the reference's (naive_attn_kernel, src/attn_sm75.cu:55-94;
// online form flash_attn_sm75_wmma, :239-375: masked scores -inf, l == 0 -> 0).  D = 256
// and the gate after the softmax are the model's gated-attention layer (24 q-heads / 4
// kv-heads, head dim 256, docs/qwen38-27b.md:13), which the reference does not build.
//
// Design: one CTA per (128-row query tile, q-head, batch), 192 threads.
//   TMEM (512 columns): S in two 64-column buffers (64 keys a tile), O in 256, and Q in
//   128 (copied there once by the softmax warps, so QK^T reads only K from shared memory).
//   Two query tiles would need 768 columns, so the overlap comes from S instead: the
//   tensor core computes S(j+1) while the softmax works on S(j), and PV(j) runs as soon
//   as P(j) is in TMEM.  Per 64-key tile the tensor work (QK^T and PV, 8.4 MFLOP) is
//   ~1320 cycles (the N = 64 QK^T instructions run at two thirds of the full rate)
//   against ~1000 of softmax.
//   warp 4: TMA producer (Q once; K(0), K(1); then per tile the stage {V(j), K(j+2)} into
//           slot j & 1 of two rings of 128-byte-swizzled 64-column boxes).
//   warp 5: TMEM owner and MMA issuer: QK(0), QK(1), then per tile PV(j), QK(j+2).
//   warps 0-3: softmax, thread = query row = TMEM lane; P(j) packed to 16 bits over the
//           first 32 columns of its S buffer; lazy O rescale (max grows by > 2^8) after
//           waiting for PV(j-1); epilogue O / l * sigmoid(G).
// The issuing thread keeps the tensor pipe busy only while it is issuing: every barrier
// wait or commit it makes between MMAs idles the pipe for ~50-150 cycles, wherever it is
// placed.  Per tile the MMA thread therefore waits once (P(j), which the softmax warps
// publish only after they have seen stage j land) and commits once: done[j & 1] marks
// PV(j) and QK(j+2) complete, which is at once "S(j+2) ready" for the softmax, "slots of
// V(j) and K(j+2) free" for the producer, and "PV(j) done" for a rescale of O.
// Every mbarrier wait is bounded (common.cuh).
#include "common.cuh"
#include "errwords.h"

namespace b200 {
namespace {

__device__ int g_err_attn_gated = 0;

constexpr int D = 256;
constexpr int BM = 128;   // query rows per CTA
constexpr int BN = 64;    // keys per tile
constexpr int kThreads = 192;
constexpr int kWarpProducer = 4, kWarpMma = 5;
constexpr uint32_t kTmemCols = 512;
// S buffers at 0 and 64, O at 128..383, Q at 384..511 (two 16-bit values a column): the
// QK^T products take Q from TMEM, so per key tile shared memory carries only K and V
constexpr uint32_t kColS = 0, kColO = 128, kColQ = 384;
constexpr float kRescaleThreshold = 8.0f;

// shared layout: Q [4 boxes of 128 rows x 64 cols], K and V rings [2][4 boxes of 64 x 64]
constexpr int kQBytes = BM * D * 2;      // 64 KiB
constexpr int kKVBytes = BN * D * 2;     // 32 KiB a stage
constexpr int kQ = 0, kK = kQ + kQBytes, kV = kK + 2 * kKVBytes, kBar = kV + 2 * kKVBytes;

// done[s] completes its n-th phase when QK(s + 2n) has completed, together with every MMA
// issued before it (PV(s + 2n - 2) among them); the prologue commits QK(0) and QK(1).
struct Bars {
    uint64_t q_full;
    uint64_t k_pro;       // K(0) and K(1) landed
    uint64_t kv_full[2];  // stage j: V(j) (and K(j+2)) landed in slot j & 1
    uint64_t done[2];
    uint64_t p_full[2];
    uint64_t q_tmem;  // the softmax warps have copied Q into TMEM
    uint64_t o_final, drain;
    uint32_t tmem_base;
    int abort;
};
constexpr int kAlloc = kBar + (int)sizeof(Bars) + 1024;
static_assert(kAlloc <= 232448, "shared memory budget");

struct Params {
    const void* G;  // gate [B][Hq][Sq][D] or null
    void* O;
    int Hq, Sq, Skv, group, n_ctas, causal;
    int tail_groups;  // causal: groups whose query tiles are dispatched level-major
    float scale_log2;
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    attn_gated_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(smem + kBar);
    volatile int* abort = &bars->abort;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // causal: the linear block index follows causal_unit_order (common.cuh), heaviest query
    // tile of a group first and the last groups level-major, so the last wave is the lightest
    int cta, hq, b;
    if (p.causal) {
        const int lin = (int)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z));
        int unit, g;
        causal_unit_order(lin, p.n_ctas, (int)(gridDim.y * gridDim.z), p.tail_groups, unit, g);
        cta = p.n_ctas - 1 - unit;
        hq = g % (int)gridDim.y;
        b = g / (int)gridDim.y;
    } else {
        cta = (int)blockIdx.x;
        hq = blockIdx.y;
        b = blockIdx.z;
    }
    const int q0 = cta * BM;
    const int off = p.Skv - p.Sq;
    const int nkv_all = (p.Skv + BN - 1) / BN;
    int nkv = nkv_all;
    if (p.causal) {
        const long long lim = (long long)min(q0 + BM, p.Sq) - 1 + off;  // last visible key
        nkv = lim < 0 ? 0 : min(nkv_all, (int)(lim / BN) + 1);
    }

    if (threadIdx.x == 0) {
        mbar_init(&bars->q_full, 1);
        mbar_init(&bars->k_pro, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars->kv_full[i], 1);
            mbar_init(&bars->done[i], 1);
            mbar_init(&bars->p_full[i], 4);  // one arrival per softmax warp
        }
        mbar_init(&bars->q_tmem, 4);
        mbar_init(&bars->o_final, 1);
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_barrier_init();
    }
    if (warp == kWarpMma) {
        tmem_alloc(&bars->tmem_base, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == kWarpProducer) {
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            const int bh_q = b * p.Hq + hq;
            const int bh_kv = b * (p.Hq / p.group) + hq / p.group;
            mbar_arrive_expect_tx(&bars->q_full, kQBytes);
#pragma unroll
            for (int a = 0; a < D / 64; ++a)
                tma_load_3d(smem + kQ + a * BM * 128, &tmQ, &bars->q_full, a * 64, q0, bh_q);
            auto load_k = [&](int j, int slot, uint64_t* bar) {
#pragma unroll
                for (int a = 0; a < D / 64; ++a)
                    tma_load_3d(smem + kK + slot * kKVBytes + a * BN * 128, &tmK, bar, a * 64, j * BN, bh_kv);
            };
            const int npro = min(2, nkv);
            if (npro > 0) {
                mbar_arrive_expect_tx(&bars->k_pro, npro * kKVBytes);
                for (int j = 0; j < npro; ++j) load_k(j, j, &bars->k_pro);
            }
            int issued = 0;  // stages whose loads were issued
            for (int j = 0; j < nkv; ++j) {
                const int st = j & 1;
                const bool with_k = j + 2 < nkv;
                // slot st of V held V(j-2) (read by PV(j-2)) and slot st of K holds K(j)
                // (read by QK(j)): both are free once done[st] has completed phase j >> 1
                if (j >= 2 && !mbar_wait(&bars->done[st], (j >> 1) & 1, abort, &g_err_attn_gated)) break;
                mbar_arrive_expect_tx(&bars->kv_full[st], with_k ? 2 * kKVBytes : kKVBytes);
#pragma unroll
                for (int a = 0; a < D / 64; ++a)
                    tma_load_3d(smem + kV + st * kKVBytes + a * BN * 128, &tmV, &bars->kv_full[st], a * 64,
                                j * BN, bh_kv);
                issued = j + 1;
                if (with_k) {
                    if (j < 2 && !mbar_wait(&bars->done[st], 0, abort, &g_err_attn_gated)) break;
                    load_k(j + 2, st, &bars->kv_full[st]);
                }
            }
            // drain: every TMA load issued has landed before exit (a stage whose K load was
            // skipped by an abort never completes; its wait gives up on the abort flag)
            mbar_wait(&bars->q_full, 0, abort, &g_err_attn_gated);
            if (npro > 0) mbar_wait(&bars->k_pro, 0, abort, &g_err_attn_gated);
            for (int j = max(0, issued - 2); j < issued; ++j)
                mbar_wait(&bars->kv_full[j & 1], (j >> 1) & 1, abort, &g_err_attn_gated);
        }
    } else if (warp == kWarpMma) {
        if (lane == 0) {
            constexpr uint32_t kFmt = Elem<T>::kFmt;
            constexpr uint32_t idesc_qk = make_idesc(kFmt, BM, BN, false, false);
            constexpr uint32_t idesc_pv = make_idesc(kFmt, BM, D, false, true);
            const uint64_t dk = smem_desc(smem_u32(smem + kK), 16, 1024, kLayoutSW128);
            const uint64_t dv = smem_desc(smem_u32(smem + kV), BN * 128, 1024, kLayoutSW128);
            auto qk = [&](int j) {  // S[j & 1] = Q K_j^T  (M=128, N=64, K=256), Q from TMEM
                const uint64_t ka = dk + (((j & 1) * kKVBytes) >> 4);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t ko = ((kk >> 2) * (BN * 128) + (kk & 3) * 32) >> 4;
                    mma_f16_ts(tmem + kColS + (j & 1) * BN, tmem + kColQ + kk * 8, ka + ko, idesc_qk,
                               kk > 0 ? 1u : 0u);
                }
            };
            // (no key tile: the softmax warps copy no Q and nothing waits for it)
            bool ok = nkv == 0 || (mbar_wait(&bars->q_tmem, 0, abort, &g_err_attn_gated) &&
                                   mbar_wait(&bars->k_pro, 0, abort, &g_err_attn_gated));
            if (ok && nkv > 0) {
                tc_fence_after();
                qk(0);
                mma_commit(&bars->done[0]);
                if (nkv > 1) {
                    qk(1);
                    mma_commit(&bars->done[1]);
                }
            }
            for (int j = 0; ok && j < nkv; ++j) {
                const int st = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                // P(j) implies stage j: the softmax warps saw it land before publishing P(j)
                if (!mbar_wait(&bars->p_full[st], ph, abort, &g_err_attn_gated)) break;
                tc_fence_after();
                // O += P(j) V_j: P from TMEM (16 keys = 8 packed columns a step), V MN-major,
                // its four 64-column boxes BN*128 bytes apart
                const uint64_t va = dv + ((st * kKVBytes) >> 4);
#pragma unroll
                for (int kk = 0; kk < BN / 16; ++kk)
                    mma_f16_ts(tmem + kColO, tmem + kColS + st * BN + kk * 8, va + ((kk * 16 * 128) >> 4),
                               idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
                // S buffer st is free once PV(j) has read P(j); the tensor pipe runs in order
                if (j + 2 < nkv) qk(j + 2);
                mma_commit(&bars->done[st]);
            }
            mma_commit(&bars->o_final);
            mma_commit(&bars->drain);
            mbar_wait(&bars->drain, 0, abort, &g_err_attn_gated);
        }
    } else {
        // ---------------- softmax: thread = query row r = TMEM lane ----------------
        const int r = warp * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
        const int qrow = q0 + r;
        const int key_lim = p.causal ? min(p.Skv - 1, qrow + off) : (p.Skv - 1);
        const float sl2 = p.scale_log2;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        if (nkv > 0) {
            // Q row r (four 128B-swizzled 64-column boxes) -> TMEM columns kColQ.., two 16-bit
            // values a column (low half = even k), the A layout of the QK^T MMAs
            ok = __all_sync(0xffffffffu, mbar_wait(&bars->q_full, 0, abort, &g_err_attn_gated));
#pragma unroll
            for (int a = 0; a < D / 64; ++a) {
                uint32_t w[32];
                const uint8_t* qrow_s = smem + kQ + a * BM * 128 + r * 128;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint4 v4 = *reinterpret_cast<const uint4*>(qrow_s + ((c ^ (r & 7)) << 4));
                    w[4 * c + 0] = v4.x;
                    w[4 * c + 1] = v4.y;
                    w[4 * c + 2] = v4.z;
                    w[4 * c + 3] = v4.w;
                }
                tmem_st32(tmem + lane_base + kColQ + a * 32, w);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->q_tmem);
        }
        for (int j = 0; ok && j < nkv; ++j) {
            const int st = j & 1;
            // S(j) = QK(j) complete: phase j >> 1 of done[st]
            if (!__all_sync(0xffffffffu, mbar_wait(&bars->done[st], (j >> 1) & 1, abort, &g_err_attn_gated))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t tS = tmem + lane_base + kColS + st * BN;
            uint32_t sr[BN];
            tmem_ld32(tS, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
            tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
            tmem_ld_wait();
            const int k0 = j * BN;
            if (k0 + BN - 1 > key_lim) {
#pragma unroll
                for (int c = 0; c < BN; ++c)
                    if (k0 + c > key_lim) sr[c] = __float_as_uint(-INFINITY);
            }
            float mx[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) mx[u] = -INFINITY;
#pragma unroll
            for (int c = 0; c < BN; ++c) mx[c & 3] = fmaxf(mx[c & 3], __uint_as_float(sr[c]));
            const float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * sl2;
            float alpha = 1.f;
            bool rescale = false;
            if (mt > m + kRescaleThreshold) {
                if (m != -INFINITY) {
                    alpha = ex2(m - mt);
                    rescale = true;
                }
                m = mt;
            }
            const float neg_mb = (m == -INFINITY) ? 0.f : -m;
            float2 rs[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};  // packed f32x2 partials
            uint32_t pk[32];
#pragma unroll
            for (int c2 = 0; c2 < BN / 2; ++c2) {
                const float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[2 * c2]), __uint_as_float(sr[2 * c2 + 1])),
                                            make_float2(sl2, sl2), make_float2(neg_mb, neg_mb));
                const float2 e = make_float2(ex2(x.x), ex2(x.y));
                rs[c2 & 1] = __fadd2_rn(rs[c2 & 1], e);
                pk[c2] = Elem<T>::pack2(e.x, e.y);
            }
            tmem_st32(tS, pk);
            // O may be rescaled only once PV(j-1) has finished (S(j) was computed earlier)
            if (j > 0 && __any_sync(0xffffffffu, rescale)) {
                // PV(j-1) complete: phase ((j - 1) >> 1) + 1 of done[(j - 1) & 1]
                const int jp = j - 1;
                if (!__all_sync(0xffffffffu, mbar_wait(&bars->done[jp & 1], ((jp >> 1) + 1) & 1, abort,
                                                       &g_err_attn_gated))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t tO = tmem + lane_base + kColO;
#pragma unroll 1
                for (int c = 0; c < D / 32; ++c) {
                    uint32_t o[32];
                    tmem_ld32(tO + c * 32, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int u = 0; u < 32; ++u) o[u] = __float_as_uint(__uint_as_float(o[u]) * alpha);
                    tmem_st32(tO + c * 32, o);
                }
            }
            tmem_st_wait();
            l = l * alpha + ((rs[0].x + rs[0].y) + (rs[1].x + rs[1].y));
            // P(j) is published only once stage j (V(j), K(j+2)) has landed, so the MMA thread
            // waits once a tile (each wait it makes idles the tensor pipe)
            if (!__all_sync(0xffffffffu, mbar_wait(&bars->kv_full[st], (j >> 1) & 1, abort, &g_err_attn_gated))) {
                ok = false;
                break;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->p_full[st]);
        }

        // ---------------- epilogue: O / l * sigmoid(G) -------------------------------
        if (ok && nkv > 0) {
            ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_final, 0, abort, &g_err_attn_gated));
            tc_fence_after();
        }
        const bool have = ok && nkv > 0;
        const float inv_l = (have && l > 0.f && m != -INFINITY) ? 1.f / l : 0.f;
        const size_t row_off = ((size_t)(b * p.Hq + hq) * p.Sq + qrow) * D;
        T* orow = static_cast<T*>(p.O) + row_off;
        const T* grow = p.G ? static_cast<const T*>(p.G) + row_off : nullptr;
        const uint32_t tO = tmem + lane_base + kColO;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            if (have) {
                tmem_ld32(tO + c * 32, o);
                tmem_ld_wait();
            } else {
#pragma unroll
                for (int u = 0; u < 32; ++u) o[u] = 0u;
            }
            if (qrow < p.Sq) {
                float gate[32];
                if (grow) {
#pragma unroll
                    for (int v4 = 0; v4 < 4; ++v4) {
                        const uint4 raw = *reinterpret_cast<const uint4*>(grow + c * 32 + v4 * 8);
                        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
                        for (int u = 0; u < 8; ++u)
                            gate[v4 * 8 + u] = 1.f / (1.f + __expf(-Elem<T>::to_f(e[u])));
                    }
                } else {
#pragma unroll
                    for (int u = 0; u < 32; ++u) gate[u] = 1.f;
                }
#pragma unroll
                for (int v4 = 0; v4 < 4; ++v4) {
                    uint4 q4;
                    uint32_t* pw = &q4.x;
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int i0 = v4 * 8 + 2 * u;
                        pw[u] = Elem<T>::pack2(__uint_as_float(o[i0]) * inv_l * gate[i0],
                                               __uint_as_float(o[i0 + 1]) * inv_l * gate[i0 + 1]);
                    }
                    *reinterpret_cast<uint4*>(orow + c * 32 + v4 * 8) = q4;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

template <typename T>
int launch(const void* Q, const void* K, const void* V, const void* G, void* O, int B, int Hq, int Hkv,
           int Sq, int Skv, float scale, int causal, cudaStream_t st) {
    const CUtensorMapDataType dt = Elem<T>::kFmt == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap tq, tk, tv;
    int rc = make_tmap_3d(&tq, Q, dt, 2, D, Sq, (uint64_t)B * Hq, 64, BM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap_3d(&tk, K, dt, 2, D, Skv, (uint64_t)B * Hkv, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap_3d(&tv, V, dt, 2, D, Skv, (uint64_t)B * Hkv, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    Params p;
    p.G = G;
    p.O = O;
    p.Hq = Hq;
    p.Sq = Sq;
    p.Skv = Skv;
    p.group = Hq / Hkv;
    p.n_ctas = (Sq + BM - 1) / BM;
    p.causal = causal;
    p.tail_groups = causal_tail_groups(p.n_ctas, B * Hq);
    p.scale_log2 = scale * 1.4426950408889634f;
    auto kern = attn_gated_kernel<T>;
    B200_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kAlloc));
    kern<<<dim3(p.n_ctas, Hq, B), kThreads, kAlloc, st>>>(tq, tk, tv, p);
    count_launch(1);
    B200_TRY_CUDA(cudaGetLastError());
    return B200LAB_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// Shared by attn_gated_fwd_sm100 and the D = 256 case of attn_fwd_sm100.
int attn_d256_launch(const void* Q, const void* K, const void* V, const void* G, void* O, int B, int Hq,
                     int Hkv, int Sq, int Skv, float scale, int causal, int dtype, void* stream) {
    if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O) || (G && !aligned16(G)))
        return B200LAB_ERR_INVALID;
    int rc = check_device_sm100();
    if (rc != B200LAB_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return dtype == B200LAB_BF16
               ? launch<__nv_bfloat16>(Q, K, V, G, O, B, Hq, Hkv, Sq, Skv, scale, causal, st)
               : launch<__half>(Q, K, V, G, O, B, Hq, Hkv, Sq, Skv, scale, causal, st);
}

}  // namespace b200

B200_DEFINE_ERR_TAKER(attn_gated, b200::g_err_attn_gated)

extern "C" int attn_gated_fwd_sm100(const void* Q, const void* K, const void* V, const void* G, void* O,
                                    int B, int Hq, int Hkv, int Sq, int Skv, int D, float scale,
                                    int causal, int dtype, void* stream) {
    if (!Q || !K || !V || !O) return B200LAB_ERR_INVALID;
    if (B < 1 || Hq < 1 || Hkv < 1 || Sq < 1 || Skv < 1 || Hq % Hkv != 0) return B200LAB_ERR_INVALID;
    if (dtype != B200LAB_F16 && dtype != B200LAB_BF16) return B200LAB_ERR_INVALID;
    if (causal != 0 && causal != 1) return B200LAB_ERR_INVALID;
    if (!(scale > 0.f) || !(scale < 1e30f)) return B200LAB_ERR_INVALID;
    if (D != 256) return B200LAB_ERR_UNSUPPORTED;
    if (B > 65535 || Hq > 65535) return B200LAB_ERR_UNSUPPORTED;
    return b200::attn_d256_launch(Q, K, V, G, O, B, Hq, Hkv, Sq, Skv, scale, causal, dtype, stream);
}
