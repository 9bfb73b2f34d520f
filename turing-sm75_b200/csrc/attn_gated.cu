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
// Design: one CTA per (128-row query tile, q-head, batch), 192 threads, 128-key tiles.
//   TMEM (512 columns): S in two 128-column buffers, O in 256.  Q, K and V sit in shared
//   memory (64 KiB each, one slot each); both QK^T operands come from shared memory, so the
//   QK^T products run at N = 128 (the full rate; 64-key tiles with Q in TMEM ran them at
//   N = 64, two thirds of it).  Two query tiles would need 768 TMEM columns, so the overlap
//   comes from S: the tensor core computes S(j+1) while the softmax works on S(j), then
//   PV(j).  Per key tile: QK^T and PV 16.8 MFLOP, ~2048 cycles of tensor work.
//   warp 4: TMA producer -- lane 0: Q once, then K(j) as soon as QK(j-1) has read K(j-1);
//           lane 1: V(j) as soon as PV(j-1) has read V(j-1) (128-byte-swizzled 64-column
//           boxes of 128 rows).
//   warp 5: TMEM owner and MMA issuer: QK(0), then per tile QK(j+1) (once K(j+1) landed)
//           and PV(j) (once P(j) is published).
//   warps 0-3: softmax, thread = query row = TMEM lane; P(j) packed to 16 bits over the
//           first 64 columns of its S buffer; lazy O rescale (max grows by > 2^8) after
//           waiting for PV(j-1); epilogue O / l * sigmoid(G).
// The issuing thread keeps the tensor pipe busy only while it is issuing: every barrier
// wait or commit it makes between MMAs idles the pipe for ~50-150 cycles, wherever it is
// placed.  Per 128-key tile it waits twice (K(j+1) landed; P(j), which the softmax warps
// publish only after they have seen V(j) land) and commits twice (S(j+1) ready, which also
// frees the K slot; PV(j) done, which frees the V slot and lets O be rescaled).
// Every mbarrier wait is bounded (common.cuh).
#include "common.cuh"
#include "errwords.h"

namespace b200 {
namespace {

__device__ int g_err_attn_gated = 0;

constexpr int D = 256;
constexpr int BM = 128;   // query rows per CTA
constexpr int BN = 128;   // keys per tile
constexpr int kThreads = 192;
constexpr int kWarpProducer = 4, kWarpMma = 5;
constexpr uint32_t kTmemCols = 512;
// S in two 128-column buffers (columns 0 and 128), O at 256..511; Q stays in shared memory
constexpr uint32_t kColS = 0, kColO = 256;
constexpr float kRescaleThreshold = 8.0f;

// shared layout: Q, K and V, each four 128-byte-swizzled boxes of 128 rows x 64 columns, one
// slot each: K(j+1) streams in once QK(j) has read K(j), V(j+1) once PV(j) has read V(j)
constexpr int kQBytes = BM * D * 2;    // 64 KiB
constexpr int kKVBytes = BN * D * 2;   // 64 KiB
constexpr int kQ = 0, kK = kQ + kQBytes, kV = kK + kKVBytes, kBar = kV + kKVBytes;

struct Bars {
    uint64_t q_full;
    uint64_t k_full;     // K(j) landed: phase j
    uint64_t v_full;     // V(j) landed: phase j
    uint64_t s_full[2];  // QK(j) complete (S(j) ready, K slot free): buffer j & 1, phase j >> 1
    uint64_t pv_done;    // PV(j) complete (V slot free, O up to date): phase j
    uint64_t p_full;     // P(j) written, V(j) seen landed: phase j
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

__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float y;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(a), "f"(b), "f"(c));
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
        mbar_init(&bars->k_full, 1);
        mbar_init(&bars->v_full, 1);
        mbar_init(&bars->s_full[0], 1);
        mbar_init(&bars->s_full[1], 1);
        mbar_init(&bars->pv_done, 1);
        mbar_init(&bars->p_full, 4);  // one arrival per softmax warp
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
        // lane 0 streams Q and the K tiles, lane 1 the V tiles: each waits only for the
        // product that frees its slot
        const int bh_q = b * p.Hq + hq;
        const int bh_kv = b * (p.Hq / p.group) + hq / p.group;
        auto load4 = [&](uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int row, int z) {
#pragma unroll
            for (int a = 0; a < D / 64; ++a) tma_load_3d(dst + a * BN * 128, map, bar, a * 64, row, z);
        };
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            mbar_arrive_expect_tx(&bars->q_full, kQBytes);
            load4(smem + kQ, &tmQ, &bars->q_full, q0, bh_q);
            int issued = 0;
            for (int j = 0; j < nkv; ++j) {
                // the K slot held K(j-1): free once QK(j-1) has completed
                if (j > 0 && !mbar_wait(&bars->s_full[(j - 1) & 1], ((j - 1) >> 1) & 1, abort, &g_err_attn_gated))
                    break;
                mbar_arrive_expect_tx(&bars->k_full, kKVBytes);
                load4(smem + kK, &tmK, &bars->k_full, j * BN, bh_kv);
                issued = j + 1;
            }
            // drain: every load issued has landed before exit (one K load is in flight at most)
            mbar_wait(&bars->q_full, 0, abort, &g_err_attn_gated);
            if (issued > 0) mbar_wait(&bars->k_full, (issued - 1) & 1, abort, &g_err_attn_gated);
        } else if (lane == 1) {
            prefetch_tmap(&tmV);
            int issued = 0;
            for (int j = 0; j < nkv; ++j) {
                // the V slot held V(j-1): free once PV(j-1) has completed
                if (j > 0 && !mbar_wait(&bars->pv_done, (j - 1) & 1, abort, &g_err_attn_gated)) break;
                mbar_arrive_expect_tx(&bars->v_full, kKVBytes);
                load4(smem + kV, &tmV, &bars->v_full, j * BN, bh_kv);
                issued = j + 1;
            }
            if (issued > 0) mbar_wait(&bars->v_full, (issued - 1) & 1, abort, &g_err_attn_gated);
        }
    } else if (warp == kWarpMma) {
        if (lane == 0) {
            constexpr uint32_t kFmt = Elem<T>::kFmt;
            constexpr uint32_t idesc_qk = make_idesc(kFmt, BM, BN, false, false);
            constexpr uint32_t idesc_pv = make_idesc(kFmt, BM, D, false, true);
            const uint64_t dq = smem_desc(smem_u32(smem + kQ), 16, 1024, kLayoutSW128);
            const uint64_t dk = smem_desc(smem_u32(smem + kK), 16, 1024, kLayoutSW128);
            const uint64_t dv = smem_desc(smem_u32(smem + kV), BN * 128, 1024, kLayoutSW128);
            auto qk = [&](int j) {  // S[j & 1] = Q K_j^T  (M=128, N=128, K=256), both from shared
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t o = ((kk >> 2) * (BM * 128) + (kk & 3) * 32) >> 4;  // BM == BN
                    mma_f16_ss(tmem + kColS + (j & 1) * BN, dq + o, dk + o, idesc_qk, kk > 0 ? 1u : 0u);
                }
            };
            bool ok = nkv == 0 || (mbar_wait(&bars->q_full, 0, abort, &g_err_attn_gated) &&
                                   mbar_wait(&bars->k_full, 0, abort, &g_err_attn_gated));
            if (ok && nkv > 0) {
                tc_fence_after();
                qk(0);
                mma_commit(&bars->s_full[0]);
            }
            for (int j = 0; ok && j < nkv; ++j) {
                if (j + 1 < nkv) {
                    // S buffer (j+1) & 1 held P(j-1), which PV(j-1), issued before, has read
                    if (!mbar_wait(&bars->k_full, (j + 1) & 1, abort, &g_err_attn_gated)) break;
                    tc_fence_after();
                    qk(j + 1);
                    mma_commit(&bars->s_full[(j + 1) & 1]);
                }
                // P(j) implies V(j): the softmax warps saw it land before publishing P(j)
                if (!mbar_wait(&bars->p_full, j & 1, abort, &g_err_attn_gated)) break;
                tc_fence_after();
                // O += P(j) V_j: P from TMEM (16 keys = 8 packed columns a step), V MN-major,
                // its four 64-column boxes BN*128 bytes apart
                const uint32_t tP = tmem + kColS + (j & 1) * BN;
#pragma unroll
                for (int kk = 0; kk < BN / 16; ++kk)
                    mma_f16_ts(tmem + kColO, tP + kk * 8, dv + ((kk * 16 * 128) >> 4), idesc_pv,
                               (j > 0 || kk > 0) ? 1u : 0u);
                mma_commit(&bars->pv_done);
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
        for (int j = 0; ok && j < nkv; ++j) {
            const int st = j & 1;
            // S(j) = QK(j) complete: phase j >> 1 of s_full[st]
            if (!__all_sync(0xffffffffu, mbar_wait(&bars->s_full[st], (j >> 1) & 1, abort, &g_err_attn_gated))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t tS = tmem + lane_base + kColS + st * BN;
            uint32_t sr[BN];
#pragma unroll
            for (int c = 0; c < BN / 32; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
            tmem_ld_wait();
            const int k0 = j * BN;
            if (k0 + BN - 1 > key_lim) {
#pragma unroll
                for (int c = 0; c < BN; ++c)
                    if (k0 + c > key_lim) sr[c] = __float_as_uint(-INFINITY);
            }
            // row max: three-input max, eight independent chains (8 deep)
            float mx[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) mx[u] = -INFINITY;
#pragma unroll
            for (int c = 0; c < BN; c += 16)
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    mx[u] = fmax3(mx[u], __uint_as_float(sr[c + 2 * u]), __uint_as_float(sr[c + 2 * u + 1]));
            const float mt =
                fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7])) * sl2;
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
            float2 rs[4];  // row-sum partials, packed f32x2 adds
#pragma unroll
            for (int u = 0; u < 4; ++u) rs[u] = make_float2(0.f, 0.f);
#pragma unroll
            for (int half = 0; half < 2; ++half) {  // 64 keys -> 32 packed columns at a time
                uint32_t pk[32];
#pragma unroll
                for (int c2 = 0; c2 < 32; ++c2) {
                    const int c = half * 64 + 2 * c2;
                    const float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])),
                                                make_float2(sl2, sl2), make_float2(neg_mb, neg_mb));
                    const float2 e = make_float2(ex2(x.x), ex2(x.y));
                    rs[c2 & 3] = __fadd2_rn(rs[c2 & 3], e);
                    pk[c2] = Elem<T>::pack2(e.x, e.y);
                }
                tmem_st32(tS + half * 32, pk);
            }
            // O may be rescaled only once PV(j-1) has finished
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
            l = l * alpha + (((rs[0].x + rs[0].y) + (rs[1].x + rs[1].y)) + ((rs[2].x + rs[2].y) + (rs[3].x + rs[3].y)));
            // P(j) is published only once V(j) has landed, so the MMA thread waits once for PV(j)
            if (!__all_sync(0xffffffffu, mbar_wait(&bars->v_full, j & 1, abort, &g_err_attn_gated))) {
                ok = false;
                break;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->p_full);
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
