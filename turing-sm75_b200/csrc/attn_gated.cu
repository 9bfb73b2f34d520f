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
//   TMEM (512 columns): S in two 64-column buffers (64 keys a tile) and O in 256.
//   Two query tiles would need 768 columns, so the overlap comes from S instead: the
//   tensor core computes S(j+1) while the softmax works on S(j), and PV(j) runs as soon
//   as P(j) is in TMEM.  Per 64-key tile the tensor work (QK^T and PV, 8.4 MFLOP) is
//   ~1024 cycles against ~950 of softmax, so the two can keep each other busy.
//   warp 4: TMA producer (Q once; K_j, V_j into two-stage rings of 128-byte-swizzled
//           64-column boxes).
//   warp 5: TMEM owner and MMA issuer: QK(0), QK(1), then per tile PV(j), QK(j+2).
//   warps 0-3: softmax, thread = query row = TMEM lane; P(j) packed to 16 bits over the
//           first 32 columns of its S buffer; lazy O rescale (max grows by > 2^8) after
//           waiting for PV(j-1); epilogue O / l * sigmoid(G).
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
constexpr uint32_t kColS = 0, kColO = 128;  // S buffers at 0 and 64, O at 128..383
constexpr float kRescaleThreshold = 8.0f;

// shared layout: Q [4 boxes of 128 rows x 64 cols], K and V rings [2][4 boxes of 64 x 64]
constexpr int kQBytes = BM * D * 2;      // 64 KiB
constexpr int kKVBytes = BN * D * 2;     // 32 KiB a stage
constexpr int kQ = 0, kK = kQ + kQBytes, kV = kK + 2 * kKVBytes, kBar = kV + 2 * kKVBytes;

struct Bars {
    uint64_t q_full;
    uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
    uint64_t s_full[2], p_full[2];
    uint64_t pv_done, o_final, drain;
    uint32_t tmem_base;
    int abort;
};
constexpr int kAlloc = kBar + (int)sizeof(Bars) + 1024;
static_assert(kAlloc <= 232448, "shared memory budget");

struct Params {
    const void* G;  // gate [B][Hq][Sq][D] or null
    void* O;
    int Hq, Sq, Skv, group, n_ctas, causal;
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
    const int cta = p.causal ? (p.n_ctas - 1 - (int)blockIdx.x) : (int)blockIdx.x;
    const int hq = blockIdx.y;
    const int b = blockIdx.z;
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
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars->k_full[i], 1);
            mbar_init(&bars->k_empty[i], 1);
            mbar_init(&bars->v_full[i], 1);
            mbar_init(&bars->v_empty[i], 1);
            mbar_init(&bars->s_full[i], 1);
            mbar_init(&bars->p_full[i], 4);  // one arrival per softmax warp
        }
        mbar_init(&bars->pv_done, 1);
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
            int nk = 0, nv = 0;
            for (int j = 0; j < nkv; ++j) {
                const int st = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                if (!mbar_wait(&bars->k_empty[st], ph ^ 1, abort, &g_err_attn_gated)) break;
                mbar_arrive_expect_tx(&bars->k_full[st], kKVBytes);
#pragma unroll
                for (int a = 0; a < D / 64; ++a)
                    tma_load_3d(smem + kK + st * kKVBytes + a * BN * 128, &tmK, &bars->k_full[st], a * 64,
                                j * BN, bh_kv);
                nk = j + 1;
                if (!mbar_wait(&bars->v_empty[st], ph ^ 1, abort, &g_err_attn_gated)) break;
                mbar_arrive_expect_tx(&bars->v_full[st], kKVBytes);
#pragma unroll
                for (int a = 0; a < D / 64; ++a)
                    tma_load_3d(smem + kV + st * kKVBytes + a * BN * 128, &tmV, &bars->v_full[st], a * 64,
                                j * BN, bh_kv);
                nv = j + 1;
            }
            // drain: every TMA load issued has landed before exit
            mbar_wait(&bars->q_full, 0, abort, &g_err_attn_gated);
            for (int j = max(0, nk - 2); j < nk; ++j)
                mbar_wait(&bars->k_full[j & 1], (j >> 1) & 1, abort, &g_err_attn_gated);
            for (int j = max(0, nv - 2); j < nv; ++j)
                mbar_wait(&bars->v_full[j & 1], (j >> 1) & 1, abort, &g_err_attn_gated);
        }
    } else if (warp == kWarpMma) {
        if (lane == 0) {
            constexpr uint32_t kFmt = Elem<T>::kFmt;
            constexpr uint32_t idesc_qk = make_idesc(kFmt, BM, BN, false, false);
            constexpr uint32_t idesc_pv = make_idesc(kFmt, BM, D, false, true);
            const uint64_t dq = smem_desc(smem_u32(smem + kQ), 16, 1024, kLayoutSW128);
            const uint64_t dk = smem_desc(smem_u32(smem + kK), 16, 1024, kLayoutSW128);
            const uint64_t dv = smem_desc(smem_u32(smem + kV), BN * 128, 1024, kLayoutSW128);
            auto qk = [&](int j) {  // S[j & 1] = Q K_j^T  (M=128, N=64, K=256)
                const uint64_t ka = dk + (((j & 1) * kKVBytes) >> 4);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t qo = ((kk >> 2) * (BM * 128) + (kk & 3) * 32) >> 4;
                    const uint32_t ko = ((kk >> 2) * (BN * 128) + (kk & 3) * 32) >> 4;
                    mma_f16_ss(tmem + kColS + (j & 1) * BN, dq + qo, ka + ko, idesc_qk, kk > 0 ? 1u : 0u);
                }
                mma_commit(&bars->s_full[j & 1]);
                mma_commit(&bars->k_empty[j & 1]);
            };
            bool ok = mbar_wait(&bars->q_full, 0, abort, &g_err_attn_gated);
            for (int j = 0; ok && j < min(2, nkv); ++j) {
                ok = mbar_wait(&bars->k_full[j & 1], (j >> 1) & 1, abort, &g_err_attn_gated);
                if (ok) {
                    tc_fence_after();
                    qk(j);
                }
            }
            for (int j = 0; ok && j < nkv; ++j) {
                const int st = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                if (!mbar_wait(&bars->p_full[st], ph, abort, &g_err_attn_gated)) break;
                if (!mbar_wait(&bars->v_full[st], ph, abort, &g_err_attn_gated)) break;
                tc_fence_after();
                // O += P(j) V_j: P from TMEM (16 keys = 8 packed columns a step), V MN-major,
                // its four 64-column boxes BN*128 bytes apart
                const uint64_t va = dv + ((st * kKVBytes) >> 4);
#pragma unroll
                for (int kk = 0; kk < BN / 16; ++kk)
                    mma_f16_ts(tmem + kColO, tmem + kColS + st * BN + kk * 8, va + ((kk * 16 * 128) >> 4),
                               idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
                mma_commit(&bars->v_empty[st]);
                mma_commit(&bars->pv_done);
                // S buffer st is free once PV(j) has read P(j); the tensor pipe runs in order
                if (j + 2 < nkv) {
                    if (!mbar_wait(&bars->k_full[st], ((j + 2) >> 1) & 1, abort, &g_err_attn_gated)) break;
                    tc_fence_after();
                    qk(j + 2);
                }
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
        for (int j = 0; j < nkv; ++j) {
            const int st = j & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&bars->s_full[st], (j >> 1) & 1, abort, &g_err_attn_gated))) {
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
            float rs[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t pk[32];
#pragma unroll
            for (int c2 = 0; c2 < BN / 2; ++c2) {
                const float e0 = ex2(fmaf(__uint_as_float(sr[2 * c2]), sl2, neg_mb));
                const float e1 = ex2(fmaf(__uint_as_float(sr[2 * c2 + 1]), sl2, neg_mb));
                rs[c2 & 3] += e0 + e1;
                pk[c2] = Elem<T>::pack2(e0, e1);
            }
            tmem_st32(tS, pk);
            // O may be rescaled only once PV(j-1) has finished (S(j) was computed earlier)
            if (j > 0 && __any_sync(0xffffffffu, rescale)) {
                if (!__all_sync(0xffffffffu, mbar_wait(&bars->pv_done, (j - 1) & 1, abort, &g_err_attn_gated))) {
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
            l = l * alpha + ((rs[0] + rs[1]) + (rs[2] + rs[3]));
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
