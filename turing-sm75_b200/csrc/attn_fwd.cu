// attn_fwd.cu -- softmax attention forward for sm_100a (tcgen05 + TMEM + TMA).
//
// Reference semantics: flash_attn_sm75_wmma<D> / flash_attn_sm75_ffma<D>
// (src/attn_sm75.cu:107-375), checked there against naive_attn_kernel
// (src/attn_sm75.cu:55-94): O = softmax(scale * Q K^T, causal k <= q) V,
// online softmax with running (m, l, O), masked scores = -inf, l == 0 -> 0.
//
// Design (one CTA per (128-row query tile, q-head, batch)):
//   warp 4      TMA producer: Q tile once, then K_j / V_j tiles into a
//               two-stage ring (128-byte swizzled boxes of 64 columns).
//   warp 5      MMA issuer (one thread) and TMEM owner:
//                 S_j = Q K_j^T   -> TMEM columns [128*(j%2), +128)  (M=128,N=128)
//                 O  += P_j V_j   -> TMEM columns [256, 256+D)        (M=128,N=D)
//               issue order QK_0, QK_1, PV_0, QK_2, PV_1, ... so the tensor
//               core computes S_{j+1} while the softmax warps work on S_j.
//   warps 0-3   softmax + epilogue; thread t owns query row t (= TMEM lane t).
//               Reads S_j with tcgen05.ld, masks, keeps the running max m in
//               log2 units and rescales O only when the max grows by more
//               than 2^8 (exact: the final 1/l uses the same m), writes
//               P_j = exp2(s*scale*log2e - m) as 16-bit values into a
//               swizzled shared tile (double-buffered) for the PV MMA.
// Causal tiles above the diagonal are skipped; only tiles that straddle the
// diagonal or the key end are masked.  GQA: q-head h reads kv-head
// h / (Hq/Hkv).  Every mbarrier wait is bounded (common.cuh).
#include "common.cuh"
#include "errwords.h"

namespace b200 {
namespace {

__device__ int g_err_attn = 0;

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int kThreads = 192;
constexpr int kWarpProducer = 4;
constexpr int kWarpMma = 5;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemO = 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P <= 2^8 between rescales

struct Bars {
    uint64_t q_full;
    uint64_t k_full[2], k_empty[2];
    uint64_t v_full[2], v_empty[2];
    uint64_t s_full[2], s_empty[2];
    uint64_t p_full[2];
    uint64_t o_done;
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

template <int D>
struct Layout {
    static constexpr int kQBytes = BM * D * 2;
    static constexpr int kKVBytes = BN * D * 2;
    static constexpr int kPBytes = BM * BN * 2;
    static constexpr int kQ = 0;
    static constexpr int kK = kQ + kQBytes;
    static constexpr int kV = kK + 2 * kKVBytes;
    static constexpr int kP = kV + 2 * kKVBytes;
    static constexpr int kBar = kP + 2 * kPBytes;
    static constexpr int kBytes = kBar + (int)sizeof(Bars);
    static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
    static_assert(kAlloc <= 232448, "shared memory budget");
};

struct Params {
    void* O;
    int Hq, Sq, Skv, group, n_qtiles, causal;
    float scale_log2;
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int D, typename T>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const Params p) {
    using L = Layout<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(smem + L::kBar);
    volatile int* abort = &bars->abort;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int qt = p.causal ? (p.n_qtiles - 1 - (int)blockIdx.x) : (int)blockIdx.x;
    const int hq = blockIdx.y;
    const int b = blockIdx.z;
    const int q0 = qt * BM;
    const int off = p.Skv - p.Sq;

    // number of key tiles this query tile needs
    const int nkv_all = (p.Skv + BN - 1) / BN;
    int nkv = nkv_all;
    if (p.causal) {
        const long long lim = (long long)q0 + BM - 1 + off;  // last row's last visible key
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
            mbar_init(&bars->s_empty[i], 128);
            mbar_init(&bars->p_full[i], 128);
        }
        mbar_init(&bars->o_done, 1);
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

    const uint32_t sQ = smem_u32(smem + L::kQ);
    const uint32_t sK0 = smem_u32(smem + L::kK);
    const uint32_t sV0 = smem_u32(smem + L::kV);
    const uint32_t sP0 = smem_u32(smem + L::kP);

    if (warp == kWarpProducer) {
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            const int bh_q = b * p.Hq + hq;
            const int bh_kv = b * (p.Hq / p.group) + hq / p.group;
            mbar_arrive_expect_tx(&bars->q_full, L::kQBytes);
#pragma unroll
            for (int a = 0; a < D / 64; ++a)
                tma_load_3d(smem + L::kQ + a * BM * 128, &tmQ, &bars->q_full, a * 64, q0, bh_q);
            int issued = 0;
            for (int j = 0; j < nkv; ++j) {
                const int st = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                if (!mbar_wait(&bars->k_empty[st], ph ^ 1, abort, &g_err_attn)) break;
                mbar_arrive_expect_tx(&bars->k_full[st], L::kKVBytes);
#pragma unroll
                for (int a = 0; a < D / 64; ++a)
                    tma_load_3d(smem + L::kK + st * L::kKVBytes + a * BN * 128, &tmK,
                                &bars->k_full[st], a * 64, j * BN, bh_kv);
                if (!mbar_wait(&bars->v_empty[st], ph ^ 1, abort, &g_err_attn)) {
                    issued = -(j + 1);  // K_j issued, V_j not
                    break;
                }
                mbar_arrive_expect_tx(&bars->v_full[st], L::kKVBytes);
#pragma unroll
                for (int a = 0; a < D / 64; ++a)
                    tma_load_3d(smem + L::kV + st * L::kKVBytes + a * BN * 128, &tmV,
                                &bars->v_full[st], a * 64, j * BN, bh_kv);
                issued = j + 1;
            }
            // Drain: every TMA load this thread issued has landed before exit.
            mbar_wait(&bars->q_full, 0, abort, &g_err_attn);
            const int nk = issued >= 0 ? issued : -issued;
            const int nv = issued >= 0 ? issued : -issued - 1;
            for (int j = max(0, nk - 2); j < nk; ++j)
                mbar_wait(&bars->k_full[j & 1], (j >> 1) & 1, abort, &g_err_attn);
            for (int j = max(0, nv - 2); j < nv; ++j)
                mbar_wait(&bars->v_full[j & 1], (j >> 1) & 1, abort, &g_err_attn);
        }
    } else if (warp == kWarpMma) {
        if (lane == 0) {
            constexpr uint32_t kFmt = Elem<T>::kFmt;
            constexpr uint32_t idesc_qk = make_idesc(kFmt, BM, BN, false, false);
            constexpr uint32_t idesc_pv = make_idesc(kFmt, BM, D, false, true);
            bool ok = mbar_wait(&bars->q_full, 0, abort, &g_err_attn);
            auto issue_pv = [&](int i) -> bool {
                const int st = i & 1;
                const uint32_t ph = (i >> 1) & 1;
                if (!mbar_wait(&bars->v_full[st], ph, abort, &g_err_attn)) return false;
                if (!mbar_wait(&bars->p_full[st], ph, abort, &g_err_attn)) return false;
                tc_fence_after();
                const uint32_t pa = sP0 + st * L::kPBytes;
                const uint32_t va = sV0 + st * L::kKVBytes;
#pragma unroll
                for (int kk = 0; kk < BN / 16; ++kk) {
                    // A = P tile, K-major, 128B-swizzled atoms of 64 keys.
                    const uint64_t a = smem_desc(pa + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 16,
                                                 1024, kLayoutSW128);
                    // B = V tile [key][d], MN-major: 16 keys = 2 groups of 8 rows.
                    const uint64_t bd = smem_desc(va + kk * 16 * 128, BN * 128, 1024, kLayoutSW128);
                    mma_f16_ss(tmem + kTmemO, a, bd, idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
                }
                mma_commit(&bars->v_empty[st]);
                mma_commit(&bars->o_done);
                return true;
            };
            for (int j = 0; ok && j < nkv; ++j) {
                const int st = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                if (!mbar_wait(&bars->k_full[st], ph, abort, &g_err_attn)) { ok = false; break; }
                if (!mbar_wait(&bars->s_empty[st], ph ^ 1, abort, &g_err_attn)) { ok = false; break; }
                tc_fence_after();
                const uint32_t ka = sK0 + st * L::kKVBytes;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint64_t a =
                        smem_desc(sQ + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 16, 1024, kLayoutSW128);
                    const uint64_t bd =
                        smem_desc(ka + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 16, 1024, kLayoutSW128);
                    mma_f16_ss(tmem + st * BN, a, bd, idesc_qk, kk > 0 ? 1u : 0u);
                }
                mma_commit(&bars->s_full[st]);
                mma_commit(&bars->k_empty[st]);
                if (j > 0 && !issue_pv(j - 1)) { ok = false; break; }
            }
            if (ok && nkv > 0) issue_pv(nkv - 1);
            // Drain: all MMAs issued by this thread are complete before TMEM is freed.
            mma_commit(&bars->drain);
            mbar_wait(&bars->drain, 0, abort, &g_err_attn);
        }
    } else {
        // ---------------- softmax warps 0..3: thread owns query row r -------------
        const int r = warp * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
        const int qrow = q0 + r;
        const int key_lim = p.causal ? min(p.Skv - 1, qrow + off) : (p.Skv - 1);
        const float sl2 = p.scale_log2;
        float m = -INFINITY;  // running max of scaled scores, log2 units
        float l = 0.f;
        uint8_t* sP = smem + L::kP;
        bool ok = true;
        for (int j = 0; j < nkv; ++j) {
            const int st = j & 1;
            const uint32_t ph = (j >> 1) & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&bars->s_full[st], ph, abort, &g_err_attn))) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t sr[BN];
#pragma unroll
            for (int c = 0; c < BN / 32; ++c)
                tmem_ld32(tmem + lane_base + st * BN + c * 32,
                          *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(&bars->s_empty[st]);

            const int k0 = j * BN;
            const bool need_mask = k0 + BN - 1 > key_lim;
            // row max as 8 independent chains (a single 128-long fmax chain is
            // latency bound with one warp per SM sub-partition)
            float mx[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) mx[u] = -INFINITY;
            if (need_mask) {
#pragma unroll
                for (int c = 0; c < BN; ++c) {
                    float s = __uint_as_float(sr[c]);
                    if (k0 + c > key_lim) s = -INFINITY;
                    sr[c] = __float_as_uint(s);
                    mx[c & 7] = fmaxf(mx[c & 7], s);
                }
            } else {
#pragma unroll
                for (int c = 0; c < BN; ++c) mx[c & 7] = fmaxf(mx[c & 7], __uint_as_float(sr[c]));
            }
            const float smax = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                     fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
            const float mt = smax * sl2;
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

            // P_j -> shared (swizzled 128B rows), 8 keys per 16-byte chunk.
            uint8_t* prow = sP + st * L::kPBytes + r * 128;
            float rs[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) rs[u] = 0.f;
#pragma unroll
            for (int ch = 0; ch < BN / 8; ++ch) {
                float e[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    e[u] = ex2(fmaf(__uint_as_float(sr[ch * 8 + u]), sl2, neg_mb));
                    rs[u] += e[u];
                }
                uint4 pk;
                pk.x = Elem<T>::pack2(e[0], e[1]);
                pk.y = Elem<T>::pack2(e[2], e[3]);
                pk.z = Elem<T>::pack2(e[4], e[5]);
                pk.w = Elem<T>::pack2(e[6], e[7]);
                const int atom = ch >> 3;
                const int c16 = (ch & 7) ^ (r & 7);
                *reinterpret_cast<uint4*>(prow + atom * (BM * 128) + c16 * 16) = pk;
            }
            fence_proxy_async_smem();
            const float rowsum = ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));

            // PV_{j-1} must be complete before O is touched and before P[(j+1)%2]
            // is rewritten next iteration.
            if (j > 0) {
                if (!__all_sync(0xffffffffu, mbar_wait(&bars->o_done, (j - 1) & 1, abort, &g_err_attn))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
                    for (int c = 0; c < D / 32; ++c) {
                        uint32_t o[32];
                        tmem_ld32(tmem + lane_base + kTmemO + c * 32, o);
                        tmem_ld_wait();
#pragma unroll
                        for (int u = 0; u < 32; ++u) o[u] = __float_as_uint(__uint_as_float(o[u]) * alpha);
                        tmem_st32(tmem + lane_base + kTmemO + c * 32, o);
                    }
                    tmem_st_wait();
                }
            }
            l = l * alpha + rowsum;
            tc_fence_before();
            mbar_arrive(&bars->p_full[st]);
        }

        // ---------------- epilogue: O / l -> global -------------------------------
        if (ok && nkv > 0) {
            ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_done, (nkv - 1) & 1, abort, &g_err_attn));
            tc_fence_after();
        }
        const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
        T* orow = static_cast<T*>(p.O) + ((size_t)(b * p.Hq + hq) * p.Sq + qrow) * D;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            if (ok && nkv > 0) {
                tmem_ld32(tmem + lane_base + kTmemO + c * 32, o);
                tmem_ld_wait();
            } else {
#pragma unroll
                for (int u = 0; u < 32; ++u) o[u] = 0u;
            }
            if (qrow < p.Sq) {
#pragma unroll
                for (int v4 = 0; v4 < 4; ++v4) {
                    uint4 pk;
                    pk.x = Elem<T>::pack2(__uint_as_float(o[v4 * 8 + 0]) * inv_l,
                                          __uint_as_float(o[v4 * 8 + 1]) * inv_l);
                    pk.y = Elem<T>::pack2(__uint_as_float(o[v4 * 8 + 2]) * inv_l,
                                          __uint_as_float(o[v4 * 8 + 3]) * inv_l);
                    pk.z = Elem<T>::pack2(__uint_as_float(o[v4 * 8 + 4]) * inv_l,
                                          __uint_as_float(o[v4 * 8 + 5]) * inv_l);
                    pk.w = Elem<T>::pack2(__uint_as_float(o[v4 * 8 + 6]) * inv_l,
                                          __uint_as_float(o[v4 * 8 + 7]) * inv_l);
                    *reinterpret_cast<uint4*>(orow + c * 32 + v4 * 8) = pk;
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

template <int D, typename T>
int launch(const void* Q, const void* K, const void* V, void* O, int B, int Hq, int Hkv, int Sq,
           int Skv, float scale, int causal, cudaStream_t st) {
    using L = Layout<D>;
    const CUtensorMapDataType dt = Elem<T>::kFmt == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap tq, tk, tv;
    int rc = make_tmap_3d(&tq, Q, dt, 2, D, Sq, (uint64_t)B * Hq, 64, BM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap_3d(&tk, K, dt, 2, D, Skv, (uint64_t)B * Hkv, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap_3d(&tv, V, dt, 2, D, Skv, (uint64_t)B * Hkv, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    auto kern = attn_fwd_kernel<D, T>;
    B200_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc));
    Params p;
    p.O = O;
    p.Hq = Hq;
    p.Sq = Sq;
    p.Skv = Skv;
    p.group = Hq / Hkv;
    p.n_qtiles = (Sq + BM - 1) / BM;
    p.causal = causal;
    p.scale_log2 = scale * 1.4426950408889634f;
    dim3 grid(p.n_qtiles, Hq, B);
    kern<<<grid, kThreads, L::kAlloc, st>>>(tq, tk, tv, p);
    count_launch(1);
    return cudaGetLastError() == cudaSuccess ? B200LAB_OK : B200LAB_ERR_CUDA;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace b200

B200_DEFINE_ERR_TAKER(attn, b200::g_err_attn)

extern "C" size_t attn_fwd_sm100_workspace(int B, int Hq, int Hkv, int Sq, int Skv, int D,
                                           int causal) {
    (void)B; (void)Hq; (void)Hkv; (void)Sq; (void)Skv; (void)D; (void)causal;
    return 0;
}

extern "C" int attn_fwd_sm100(const void* Q, const void* K, const void* V, void* O, int B, int Hq,
                              int Hkv, int Sq, int Skv, int D, float scale, int causal, int dtype,
                              void* workspace, size_t ws_bytes, void* stream) {
    using namespace b200;
    (void)workspace;
    (void)ws_bytes;
    if (!Q || !K || !V || !O) return B200LAB_ERR_INVALID;
    if (B < 1 || Hq < 1 || Hkv < 1 || Sq < 1 || Skv < 1 || Hq % Hkv != 0) return B200LAB_ERR_INVALID;
    if (dtype != B200LAB_F16 && dtype != B200LAB_BF16) return B200LAB_ERR_INVALID;
    if (causal != 0 && causal != 1) return B200LAB_ERR_INVALID;
    if (!(scale > 0.f) || !(scale < 1e30f)) return B200LAB_ERR_INVALID;
    if (D != 64 && D != 128) return B200LAB_ERR_UNSUPPORTED;
    if (B > 65535 || Hq > 65535) return B200LAB_ERR_UNSUPPORTED;
    if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O)) return B200LAB_ERR_INVALID;
    int rc = check_device_sm100();
    if (rc != B200LAB_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (dtype == B200LAB_BF16) {
        return D == 128 ? launch<128, __nv_bfloat16>(Q, K, V, O, B, Hq, Hkv, Sq, Skv, scale, causal, st)
                        : launch<64, __nv_bfloat16>(Q, K, V, O, B, Hq, Hkv, Sq, Skv, scale, causal, st);
    }
    return D == 128 ? launch<128, __half>(Q, K, V, O, B, Hq, Hkv, Sq, Skv, scale, causal, st)
                    : launch<64, __half>(Q, K, V, O, B, Hq, Hkv, Sq, Skv, scale, causal, st);
}
