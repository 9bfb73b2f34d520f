// attn_fwd.cu -- softmax attention forward for sm_100a (tcgen05 + TMEM + TMA).
//
// Reference semantics: flash_attn_sm75_wmma<D> / flash_attn_sm75_ffma<D>
// (src/attn_sm75.cu:107-375), checked there against naive_attn_kernel
// (src/attn_sm75.cu:55-94): O = softmax(scale * Q K^T, causal k <= q) V,
// online softmax with running (m, l, O), masked scores = -inf, l == 0 -> 0.
//
// Design: one CTA per (256 query rows = two 128-row tiles, q-head, batch),
// 320 threads, every K/V tile loaded once and used by both query tiles.
//   warp 8      TMA producer: Q0, Q1 once, then K_j / V_j into a two-stage
//               ring (128-byte swizzled boxes of 64 columns).
//   warp 9      MMA issuer (one thread) and owner of all 512 TMEM columns:
//                 S_t  = Q_t K_j^T      TMEM cols [128 t, 128 t + 128)   (M=N=128)
//                 O_t += P_t V_j        TMEM cols [256 + D t, +D)        (M=128, N=D)
//               P_t is read from TMEM (the ".kind::f16 [d], [a], b" form) where
//               the softmax wrote it over the first 64 columns of S_t.  Issue
//               order per key tile: PV_0(j), QK_0(j+1), PV_1(j), QK_1(j+1), so
//               the tensor core always has the other tile's work queued while a
//               softmax warpgroup works.
//   warps 0-3   softmax of tile 0, warps 4-7 softmax of tile 1: thread = query
//               row = TMEM lane.  tcgen05.ld S, mask, running max in log2
//               units with lazy O rescale (only when the max grows by > 2^8;
//               exact since the final 1/l uses the same max), P = exp2(s*c - m)
//               packed to 16 bits and stored back with tcgen05.st, then the
//               epilogue O / l -> HBM.
// Ordering without extra barriers: tcgen05.commit tracks every earlier MMA of
// the issuing thread, so "S_t(j) ready" also means PV_t(j-1) has finished --
// O_t may be rescaled and P_t's columns rewritten.
// Causal tiles above the diagonal are skipped; only tiles that straddle the
// diagonal or the key end are masked.  GQA: q-head h reads kv-head
// h / (Hq/Hkv).  Split-KV: when the (query-tile pair, head, batch) grid cannot
// fill the GPU (short queries), the key tiles are split over extra CTAs that
// write fp32 partials (O, max, sum) to the caller's workspace, merged by
// attn_combine_kernel.  Every mbarrier wait is bounded (common.cuh).
#include "common.cuh"
#include "errwords.h"

#include <type_traits>
#include <vector>

namespace b200 {
namespace {

__device__ int g_err_attn = 0;

constexpr int BM = 128;  // rows per query tile
constexpr int BN = 128;  // keys per K/V tile
constexpr int kQTiles = 2;
constexpr int kThreads = 320;
constexpr int kWarpProducer = 8;
constexpr int kWarpMma = 9;
constexpr int kStages = 2;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P <= 2^8 between rescales

// The MMA thread keeps the tensor pipe fed only while it issues: each barrier wait or commit
// it makes between MMAs idles the pipe (~50-150 cycles, measured, wherever it is placed).
// Per key tile it therefore waits three times (the stage, P_0, P_1) and commits twice:
// s_full0 after QK_0(j+1), and done[j&1] after the whole step, which completes
// when PV(j) and QK(j+1) of both tiles have: "S_1(j+1) ready" for the second softmax
// warpgroup and "V slot j&1 and K slot (j+1)&1 free" for the producer, which loads V(j)
// and K(j+1) as one stage under one barrier.
struct Bars {
    uint64_t q_full;
    uint64_t k_pro;               // K(0) landed
    uint64_t kv_full[kStages];    // stage j: V(j) (and K(j+1)) landed
    uint64_t done[kStages];       // step j's MMAs complete
    uint64_t s_full0;             // S_0(j) ready
    uint64_t s1_pro;              // S_1(0) ready (QK of both tiles on K(0) complete)
    uint64_t p_full[kQTiles];
    uint64_t o_final;
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

template <int D>
struct Layout {
    static constexpr int kQTileBytes = BM * D * 2;
    static constexpr int kKVBytes = BN * D * 2;
    static constexpr int kQ = 0;
    static constexpr int kK = kQ + kQTiles * kQTileBytes;
    static constexpr int kV = kK + kStages * kKVBytes;
    // Head dim 64: the row sums of P come from the PV product itself, N = D + 16, whose
    // columns D .. D+15 read a 64-column swizzle block of ones placed after the V stages (the
    // descriptor's leading byte offset, one descriptor a stage); O_t column D is then the
    // running sum, rescaled with O.  The MMAs have slack at D = 64, the softmax (issue-bound)
    // drops its packed add a pair.  At D = 128 TMEM has no room for the extra columns.
    static constexpr bool kRowSumMma = D == 64;
    static constexpr int kOnes = kV + kStages * kKVBytes;
    static constexpr int kOnesBytes = kRowSumMma ? BN * 128 : 0;
    static constexpr int kBar = kOnes + kOnesBytes;
    static constexpr int kBytes = kBar + (int)sizeof(Bars);
    static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
    static_assert(kAlloc <= 232448, "shared memory budget");
    static constexpr int kOCols = kRowSumMma ? D + 16 : D;  // TMEM columns of an O tile
    static constexpr uint32_t kTmemO = 256;                  // O_t at kTmemO + t*kOCols
    static_assert(kTmemO + kQTiles * kOCols <= kTmemCols, "TMEM columns");
    static_assert(kOnes % 1024 == 0, "swizzled operand base");
};

struct Params {
    void* O;
    const int* cu_q;  // varlen: [B+1] token offsets of the sequences in Q/O (device)
    const int* cu_k;  // varlen: [B+1] token offsets in K/V
    float* part_o;   // split-KV partials: [B*Hq*Sq][nsplit][D] fp32 (unnormalised)
    float* part_ml;  // [B*Hq*Sq][nsplit][2]: running max (log2 units), row sum
    int Hq, Sq, Skv, group, n_ctas, causal;
    int nsplit, tiles_per_split;
    int total_q, total_k, max_sq;  // varlen: the buffers' token counts and the grid's sizing
    int pack_sq;  // > 0: GQA-packed rows (row r is query r % pack_sq); 0: row = query
    int tail_groups;  // causal: groups whose query pairs are dispatched level-major
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

// 2^x for a pair of values on the FMA pipe (packed f32x2 ops), so that a quarter of
// the exponentials leave the MUFU pipe (4 lanes a clock per SM sub-partition), which
// otherwise bounds the softmax.  x = n + f by round-to-nearest through the 1.5*2^23
// shifter, 2^f by a degree-3 polynomial fitted for this kernel (Remez exchange,
// minimax relative error 7.5e-5 on [-1/2, 1/2], well below the 2^-9 rounding of the
// 16-bit P), 2^n added into the exponent field.  x is clamped to >= -125 so the
// result stays a normal float: a masked key gives 2^-125 instead of 0, and a row
// that never sees a key is zeroed from its max in the epilogue.  More than a quarter
// costs more issue slots (the packed ops take two) than it saves MUFU time.
__device__ __forceinline__ float2 exp2_fma2(float2 x) {
    constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
    constexpr float kP0 = 9.999280572e-01f, kP1 = 6.932609677e-01f, kP2 = 2.426111251e-01f,
                    kP3 = 5.517166853e-02f;
    x.x = fmaxf(x.x, -125.f);
    x.y = fmaxf(x.y, -125.f);
    const float2 t = __fadd2_rn(x, make_float2(kShift, kShift));
    const float2 n = __fadd2_rn(t, make_float2(-kShift, -kShift));
    const float2 f = __ffma2_rn(n, make_float2(-1.f, -1.f), x);
    float2 q = __ffma2_rn(make_float2(kP3, kP3), f, make_float2(kP2, kP2));
    q = __ffma2_rn(q, f, make_float2(kP1, kP1));
    q = __ffma2_rn(q, f, make_float2(kP0, kP0));
    // the shifter's low mantissa bits hold n (two's complement); its own exponent
    // and leading bits shift out above bit 31
    return make_float2(__uint_as_float(__float_as_uint(q.x) + (__float_as_uint(t.x) << 23)),
                       __uint_as_float(__float_as_uint(q.y) + (__float_as_uint(t.y) << 23)));
}

// kVarlen: packed sequences in the token-major layout Q/O [total_q][Hq][D], K/V
// [total_k][Hkv][D] with per-sequence offsets cu_q / cu_k (blockIdx.z = sequence); the
// tensor maps are (D, heads, tokens) with (64, 1, rows) boxes, which land in shared
// memory exactly like the head-major boxes.  Rows of a box past the sequence belong to the
// next one: keys there are masked, query rows there are not stored.
template <int D, typename T, bool kSplit, bool kVarlen = false>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const Params p) {
    static_assert(!(kSplit && kVarlen), "no key splits for packed sequences");
    using L = Layout<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(smem + L::kBar);
    volatile int* abort = &bars->abort;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // Causal CTAs differ in work (a pair's key tiles grow with its row index): the linear
    // block index follows causal_unit_order (common.cuh), the last groups level-major so the
    // last wave holds the shortest CTAs.  Splits of one pair stay adjacent.  Packed sequences
    // keep the plain order (blockIdx.z is the sequence).
    int split, cta_lin, hq, b;
    if (p.causal && !kVarlen) {
        const int lin = (int)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z));
        split = lin % p.nsplit;
        int g;
        causal_unit_order(lin / p.nsplit, p.n_ctas, (int)(gridDim.y * gridDim.z), p.tail_groups, cta_lin, g);
        hq = g % (int)gridDim.y;
        b = g / (int)gridDim.y;
    } else {
        split = (int)blockIdx.x % p.nsplit;
        cta_lin = (int)blockIdx.x / p.nsplit;
        hq = blockIdx.y;
        b = blockIdx.z;
    }
    int Sq = p.Sq, Skv = p.Skv, n_ctas = p.n_ctas;  // this sequence's lengths
    int q_tok0 = 0, k_tok0 = 0;                      // varlen: its first token in Q/O, K/V
    if constexpr (kVarlen) {
        q_tok0 = p.cu_q[b];
        k_tok0 = p.cu_k[b];
        Sq = p.cu_q[b + 1] - q_tok0;
        Skv = p.cu_k[b + 1] - k_tok0;
        // a caller's offsets are checked before anything is read or written through them
        if (q_tok0 < 0 || Sq < 0 || Sq > p.max_sq || q_tok0 > p.total_q - Sq || k_tok0 < 0 || Skv < 0 ||
            k_tok0 > p.total_k - Skv) {
            if (threadIdx.x == 0 && cta_lin == 0 && hq == 0) atomicExch(&g_err_attn, B200LAB_ERR_INVALID);
            return;
        }
        n_ctas = (Sq + kQTiles * BM - 1) / (kQTiles * BM);
        if (cta_lin >= n_ctas) return;  // the grid covers the longest sequence
    }
    const int cta = p.causal ? (n_ctas - 1 - cta_lin) : cta_lin;
    const int q0 = cta * (kQTiles * BM);
    // the causal mask: row r is query r (or r % pack_sq when a GQA group's q-heads are packed
    // into the rows), aligned at the bottom right of the key range
    const int sq_mask = p.pack_sq ? p.pack_sq : Sq;
    const int off = Skv - sq_mask;

    // key tiles this CTA needs: enough for its last valid query row, then the
    // part [j0, j0 + nkv) of them that belongs to this CTA's key split
    const int nkv_all = (Skv + BN - 1) / BN;
    int nkv_need = nkv_all;
    if (p.causal) {
        const long long last_row = p.pack_sq ? p.pack_sq - 1 : min(q0 + kQTiles * BM, Sq) - 1;
        const long long lim = last_row + off;  // last visible key of that row
        nkv_need = lim < 0 ? 0 : min(nkv_all, (int)(lim / BN) + 1);
    }
    const int j0 = split * p.tiles_per_split;
    const int nkv = max(0, min(nkv_need - j0, p.tiles_per_split));
    // the second query tile holds rows (false only for short queries: its products are skipped)
    const bool tile1 = q0 + BM < Sq;
    // the combine kernel that follows a split grid may be scheduled now: it waits for this
    // grid to complete before reading the partials (griddepcontrol.wait)
    if constexpr (kSplit) allow_dependent_launch();

    if (threadIdx.x == 0) {
        mbar_init(&bars->q_full, 1);
        mbar_init(&bars->k_pro, 1);
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&bars->kv_full[i], 1);
            mbar_init(&bars->done[i], 1);
        }
        mbar_init(&bars->s_full0, 1);
        mbar_init(&bars->s1_pro, 1);
        for (int t = 0; t < kQTiles; ++t) mbar_init(&bars->p_full[t], 4);  // one arrival a warp
        mbar_init(&bars->o_final, 1);
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_barrier_init();
    }
    if constexpr (L::kRowSumMma) {  // the tile of ones, made visible to the tensor core
        const uint32_t one2 = Elem<T>::pack2(1.f, 1.f);
        uint4* ones = reinterpret_cast<uint4*>(smem + L::kOnes);
        for (int i = threadIdx.x; i < L::kOnesBytes / 16; i += kThreads) ones[i] = make_uint4(one2, one2, one2, one2);
        fence_proxy_async_smem();
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

    if (warp == kWarpProducer) {
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            const int bh_q = b * p.Hq + hq;
            const int bh_kv = b * (p.Hq / p.group) + hq / p.group;
            mbar_arrive_expect_tx(&bars->q_full, kQTiles * L::kQTileBytes);
#pragma unroll
            for (int t = 0; t < kQTiles; ++t)
#pragma unroll
                for (int a = 0; a < D / 64; ++a)
                    if constexpr (kVarlen)
                        tma_load_4d(smem + L::kQ + t * L::kQTileBytes + a * BM * 128, &tmQ, &bars->q_full,
                                    a * 64, hq, q_tok0 + q0 + t * BM, 0);
                    else
                        tma_load_3d(smem + L::kQ + t * L::kQTileBytes + a * BM * 128, &tmQ, &bars->q_full,
                                    a * 64, q0 + t * BM, bh_q);
            auto load_kv = [&](const CUtensorMap* map, int base, int slot, int j, uint64_t* bar) {
#pragma unroll
                for (int a = 0; a < D / 64; ++a)
                    if constexpr (kVarlen)
                        tma_load_4d(smem + base + slot * L::kKVBytes + a * BN * 128, map, bar, a * 64,
                                    hq / p.group, k_tok0 + j * BN, 0);
                    else
                        tma_load_3d(smem + base + slot * L::kKVBytes + a * BN * 128, map, bar, a * 64,
                                    (j0 + j) * BN, bh_kv);
            };
            if (nkv > 0) {
                mbar_arrive_expect_tx(&bars->k_pro, L::kKVBytes);
                load_kv(&tmK, L::kK, 0, 0, &bars->k_pro);
            }
            int issued = 0;  // stages whose loads were issued
            for (int j = 0; j < nkv; ++j) {
                const int st = j & 1;
                const bool with_k = j + 1 < nkv;
                // V slot st held V(j-2) and K slot (j+1)&1 held K(j-1): both were read by
                // step j-2, whose MMAs done[st] tracks (commit (j>>1)-1 on it); K(1)'s slot
                // is free from the start, K(2)'s once the QKs on K(0) completed
                if (j >= 2 && !mbar_wait(&bars->done[st], ((j >> 1) & 1) ^ 1, abort, &g_err_attn)) break;
                mbar_arrive_expect_tx(&bars->kv_full[st], with_k ? 2 * L::kKVBytes : L::kKVBytes);
                load_kv(&tmV, L::kV, st, j, &bars->kv_full[st]);
                issued = j + 1;
                if (with_k) {
                    if (j == 1 && !mbar_wait(&bars->s1_pro, 0, abort, &g_err_attn)) break;
                    load_kv(&tmK, L::kK, (j + 1) & 1, j + 1, &bars->kv_full[st]);
                }
            }
            // Drain: every TMA load this thread issued has landed before exit (a stage whose
            // K load an abort skipped never completes; its wait gives up on the abort flag).
            mbar_wait(&bars->q_full, 0, abort, &g_err_attn);
            if (nkv > 0) mbar_wait(&bars->k_pro, 0, abort, &g_err_attn);
            for (int j = max(0, issued - 2); j < issued; ++j)
                mbar_wait(&bars->kv_full[j & 1], (j >> 1) & 1, abort, &g_err_attn);
        }
    } else if (warp == kWarpMma) {
        if (lane == 0) {
            constexpr uint32_t kFmt = Elem<T>::kFmt;
            constexpr uint32_t idesc_qk = make_idesc(kFmt, BM, BN, false, false);
            constexpr uint32_t idesc_pv = make_idesc(kFmt, BM, L::kOCols, false, true);
            // Descriptors are built once; per K-step only the start-address field
            // (bits 0-13, address >> 4) advances, by a plain 64-bit add.
            const uint64_t dq0 = smem_desc(sQ, 16, 1024, kLayoutSW128);
            const uint64_t dk0 = smem_desc(sK0, 16, 1024, kLayoutSW128);
            const uint64_t dv0 = smem_desc(sV0, BN * 128, 1024, kLayoutSW128);
            // D = 64: the block after each V stage's columns is the tile of ones
            const uint64_t dv1s[2] = {smem_desc(sV0, L::kOnes - L::kV, 1024, kLayoutSW128),
                                      smem_desc(sV0 + L::kKVBytes, L::kOnes - L::kV - L::kKVBytes, 1024,
                                                kLayoutSW128)};
            auto qk = [&](int t, int j) {  // S_t = Q_t K_j^T
                const uint64_t qa = dq0 + ((t * L::kQTileBytes) >> 4);
                const uint64_t ka = dk0 + (((j & 1) * L::kKVBytes) >> 4);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t o = ((kk >> 2) * (BM * 128) + (kk & 3) * 32) >> 4;
                    mma_f16_ss(tmem + t * BN, qa + o, ka + o, idesc_qk, kk > 0 ? 1u : 0u);
                }
            };
            auto pv = [&](int t, int j) {  // O_t += P_t V_j, P from TMEM
                // B = V tile [key][d], MN-major: 16 keys = two 8-row groups; 64-column
                // boxes BN*128 bytes apart (the descriptor's leading byte offset).
                const uint64_t va = L::kRowSumMma ? dv1s[j & 1] : dv0 + (((j & 1) * L::kKVBytes) >> 4);
#pragma unroll
                for (int kk = 0; kk < BN / 16; ++kk) {
                    mma_f16_ts(tmem + L::kTmemO + t * L::kOCols, tmem + t * BN + kk * 8,
                               va + ((kk * 16 * 128) >> 4), idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
                }
            };
            bool ok = mbar_wait(&bars->q_full, 0, abort, &g_err_attn);
            if (ok && nkv > 0) {
                ok = mbar_wait(&bars->k_pro, 0, abort, &g_err_attn);
                if (ok) {
                    tc_fence_after();
                    qk(0, 0);
                    mma_commit(&bars->s_full0);
                    if (tile1) qk(1, 0);
                    mma_commit(&bars->s1_pro);
                }
            }
            for (int j = 0; ok && j < nkv; ++j) {
                const int st = j & 1;
                const int jn = j + 1;
                if (!mbar_wait(&bars->kv_full[st], (j >> 1) & 1, abort, &g_err_attn)) break;
                // tile 0
                if (!mbar_wait(&bars->p_full[0], j & 1, abort, &g_err_attn)) break;
                tc_fence_after();
                pv(0, j);
                if (jn < nkv) {
                    qk(0, jn);
                    mma_commit(&bars->s_full0);
                }
                // tile 1
                if (tile1) {
                    if (!mbar_wait(&bars->p_full[1], j & 1, abort, &g_err_attn)) break;
                    tc_fence_after();
                    pv(1, j);
                    if (jn < nkv) qk(1, jn);
                }
                mma_commit(&bars->done[st]);
            }
            mma_commit(&bars->o_final);
            // Drain: all MMAs issued by this thread are complete before TMEM is freed.
            mma_commit(&bars->drain);
            mbar_wait(&bars->drain, 0, abort, &g_err_attn);
        }
    } else {
        // ---------------- softmax warpgroups: tile t, thread owns query row r ------------
        const int t = warp >> 2;
        const int r = (warp & 3) * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + lane_base + t * BN;
        const uint32_t tO = tmem + lane_base + L::kTmemO + t * L::kOCols;
        const int qrow = q0 + t * BM + r;
        const int key_lim = p.causal ? min(Skv - 1, (p.pack_sq ? qrow % p.pack_sq : qrow) + off) : (Skv - 1);
        const float sl2 = p.scale_log2;
        float m = -INFINITY;  // running max of scaled scores, log2 units
        float l = 0.f;  // (D = 64: O_t column D holds it, read in the epilogue)
        bool ok = true;
        // a warp whose 32 rows all lie past the queries (short or GQA-packed queries) writes no
        // P: it only keeps step with the tiles, so that its arrival is counted for the right one.
        // A second tile with no rows at all is not computed: its warps skip the key loop.
        const bool warp_rows = __any_sync(0xffffffffu, qrow < Sq);
        const int nkv_t = (t == 1 && !tile1) ? 0 : nkv;
        for (int j = 0; j < nkv_t; ++j) {
            // S_0(j): commit j on s_full0.  S_1(j): the prologue's s1_pro, then step j-1's
            // commit on done[(j-1)&1] (its ((j-1)>>1)-th)
            uint64_t* s_bar = t == 0 ? &bars->s_full0 : (j == 0 ? &bars->s1_pro : &bars->done[(j - 1) & 1]);
            const uint32_t s_par = t == 0 ? (uint32_t)(j & 1) : (j == 0 ? 0u : (uint32_t)(((j - 1) >> 1) & 1));
            if (!__all_sync(0xffffffffu, mbar_wait(s_bar, s_par, abort, &g_err_attn))) {
                ok = false;
                break;
            }
            tc_fence_after();
            if (!warp_rows) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->p_full[t]);
                continue;
            }
            uint32_t sr[BN];
#pragma unroll
            for (int c = 0; c < BN / 32; ++c)
                tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
            tmem_ld_wait();

            const int k0 = (j0 + j) * BN;
            const bool need_mask = k0 + BN - 1 > key_lim;
            if (need_mask) {
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
            const float smax = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
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

            // P = exp2(s*c - m), packed two per 32-bit column, over S's first 64 columns
            float2 rs[4];  // row-sum partials, pairs added with packed f32x2 adds
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
                    float2 e;
                    if ((c2 & 7) >= 6) {  // two pairs in every eight on the FMA pipe
                        e = exp2_fma2(x);
                    } else {
                        e.x = ex2(x.x);
                        e.y = ex2(x.y);
                    }
                    if constexpr (!L::kRowSumMma) rs[c2 & 3] = __fadd2_rn(rs[c2 & 3], e);
                    pk[c2] = Elem<T>::pack2(e.x, e.y);
                }
                tmem_st32(tS + half * 32, pk);
            }
            const float rowsum =
                ((rs[0].x + rs[0].y) + (rs[1].x + rs[1].y)) + ((rs[2].x + rs[2].y) + (rs[3].x + rs[3].y));

            // O_t is idle here: PV_t(j-1) finished before S_t(j) was signalled.
            if (j > 0 && __any_sync(0xffffffffu, rescale)) {
#pragma unroll
                for (int c = 0; c < D / 32; ++c) {
                    uint32_t o[32];
                    tmem_ld32(tO + c * 32, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int u = 0; u < 32; ++u) o[u] = __float_as_uint(__uint_as_float(o[u]) * alpha);
                    tmem_st32(tO + c * 32, o);
                }
                if constexpr (L::kRowSumMma) {  // the running row sum in column D
                    uint32_t lc;
                    tmem_ld1(tO + D, lc);
                    tmem_ld_wait();
                    tmem_st1(tO + D, __float_as_uint(__uint_as_float(lc) * alpha));
                }
            }
            tmem_st_wait();
            if constexpr (!L::kRowSumMma) l = l * alpha + rowsum;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->p_full[t]);
        }

        // ---------------- epilogue -------------------------------------------------
        if (ok && nkv > 0) {
            ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_final, 0, abort, &g_err_attn));
            tc_fence_after();
        }
        if constexpr (L::kRowSumMma) {  // the row sum from O_t column D (warp-uniform condition)
            if (ok && nkv > 0) {
                uint32_t lc;
                tmem_ld1(tO + D, lc);
                tmem_ld_wait();
                l = __uint_as_float(lc);
            }
        }
        if constexpr (kSplit) {
            // split-KV partial: unnormalised O, running max and sum, fp32
            if (qrow < p.Sq) {
                const size_t prow = ((size_t)(b * p.Hq + hq) * p.Sq + qrow) * p.nsplit + split;
                float2 ml = make_float2(m, l);
                if (!(ok && nkv > 0) || m == -INFINITY) ml = make_float2(-INFINITY, 0.f);
                *reinterpret_cast<float2*>(p.part_ml + prow * 2) = ml;
            }
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
                uint32_t o[32];
                if (ok && nkv > 0) {
                    tmem_ld32(tO + c * 32, o);
                    tmem_ld_wait();
                } else {
#pragma unroll
                    for (int u = 0; u < 32; ++u) o[u] = 0u;
                }
                if (qrow < p.Sq) {
                    float* po = p.part_o + (((size_t)(b * p.Hq + hq) * p.Sq + qrow) * p.nsplit + split) * D;
#pragma unroll
                    for (int v4 = 0; v4 < 8; ++v4)
                        *reinterpret_cast<uint4*>(po + c * 32 + v4 * 4) =
                            make_uint4(o[v4 * 4], o[v4 * 4 + 1], o[v4 * 4 + 2], o[v4 * 4 + 3]);
                }
            }
        } else {
            // a row that never saw a key (max still -inf) is 0, as with l == 0
            const float inv_l = (l > 0.f && m != -INFINITY) ? 1.f / l : 0.f;
            T* orow = static_cast<T*>(p.O) +
                      (kVarlen ? ((size_t)(q_tok0 + qrow) * p.Hq + hq) * D
                               : ((size_t)(b * p.Hq + hq) * p.Sq + qrow) * D);
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
                uint32_t o[32];
                if (ok && nkv > 0) {
                    tmem_ld32(tO + c * 32, o);
                    tmem_ld_wait();
                } else {
#pragma unroll
                    for (int u = 0; u < 32; ++u) o[u] = 0u;
                }
                if (qrow < Sq) {
#pragma unroll
                    for (int v4 = 0; v4 < 4; ++v4) {
                        uint4 q4;
                        q4.x = Elem<T>::pack2(__uint_as_float(o[v4 * 8 + 0]) * inv_l,
                                              __uint_as_float(o[v4 * 8 + 1]) * inv_l);
                        q4.y = Elem<T>::pack2(__uint_as_float(o[v4 * 8 + 2]) * inv_l,
                                              __uint_as_float(o[v4 * 8 + 3]) * inv_l);
                        q4.z = Elem<T>::pack2(__uint_as_float(o[v4 * 8 + 4]) * inv_l,
                                              __uint_as_float(o[v4 * 8 + 5]) * inv_l);
                        q4.w = Elem<T>::pack2(__uint_as_float(o[v4 * 8 + 6]) * inv_l,
                                              __uint_as_float(o[v4 * 8 + 7]) * inv_l);
                        *reinterpret_cast<uint4*>(orow + c * 32 + v4 * 8) = q4;
                    }
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

// Split-KV combine: the nsplit (<= 64) partials of a query row are merged as
//   M = max_s m_s,  O = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s   (0 if no key seen).
// A row gets wpr = 2^wpr_log2 warps (wpr >= nsplit / 8); warp `sub` of the row owns the
// splits sub, sub + wpr, ... (at most 8) and issues all of their O loads before anything
// else, so a row costs one memory round trip; the row's (max, sum) pairs are staged in
// shared memory, reduced with shuffles, and the wpr warps' weighted sums are added in shared
// memory.  Launched as a programmatic dependent of the split kernel: it waits for that grid
// to complete (griddepcontrol.wait) before reading the partials.
template <int D, typename T>
__global__ void __launch_bounds__(256) attn_combine_kernel(const float* __restrict__ part_o,
                                                           const float* __restrict__ part_ml,
                                                           T* __restrict__ O, long long rows, int nsplit,
                                                           int wpr_log2) {
    constexpr int kPer = D / 32;  // values per lane (4 or 2)
    static_assert(kPer == 4 || kPer == 2, "head dim 64 or 128");
    using Vec = typename std::conditional<kPer == 4, float4, float2>::type;
    __shared__ float2 s_ml[8][64];
    __shared__ float s_acc[8][D];
    grid_dependency_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wpr = 1 << wpr_log2;
    const int rpb = 8 >> wpr_log2;  // rows per block
    const int slot = warp >> wpr_log2, sub = warp & (wpr - 1);
    const long long row0 = (long long)blockIdx.x * rpb;
    const long long row = row0 + slot;
    const bool live = row < rows;

    Vec v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int sp = sub + i * wpr;
        v[i] = Vec{};
        if (live && sp < nsplit)
            v[i] = *reinterpret_cast<const Vec*>(part_o + (row * nsplit + sp) * D + lane * kPer);
    }
    const float2* ml = reinterpret_cast<const float2*>(part_ml);
    for (int i = threadIdx.x; i < rpb * nsplit; i += blockDim.x) {
        const int r = i / nsplit, sp = i % nsplit;
        float2 e = make_float2(-INFINITY, 0.f);
        if (row0 + r < rows) e = ml[(row0 + r) * nsplit + sp];
        if (!(e.y > 0.f)) e = make_float2(-INFINITY, 0.f);  // an empty split takes no part
        s_ml[r][sp] = e;
    }
    __syncthreads();

    const float2 e0 = lane < nsplit ? s_ml[slot][lane] : make_float2(-INFINITY, 0.f);
    const float2 e1 = lane + 32 < nsplit ? s_ml[slot][lane + 32] : make_float2(-INFINITY, 0.f);
    float M = fmaxf(e0.x, e1.x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.f;
    if (M != -INFINITY) {
        L = (e0.y > 0.f ? ex2(e0.x - M) * e0.y : 0.f) + (e1.y > 0.f ? ex2(e1.x - M) * e1.y : 0.f);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    }
    float acc[kPer];
#pragma unroll
    for (int c = 0; c < kPer; ++c) acc[c] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int sp = sub + i * wpr;
        if (sp < nsplit && M != -INFINITY) {
            const float2 e = s_ml[slot][sp];
            if (e.y > 0.f) {
                const float w = ex2(e.x - M);
                const float* pv = reinterpret_cast<const float*>(&v[i]);
#pragma unroll
                for (int c = 0; c < kPer; ++c) acc[c] = fmaf(w, pv[c], acc[c]);
            }
        }
    }
#pragma unroll
    for (int c = 0; c < kPer; ++c) s_acc[warp][lane * kPer + c] = acc[c];
    __syncthreads();

    if (live) {
        const float inv = L > 0.f ? 1.f / L : 0.f;
        T* orow = O + row * D;
        for (int pr = sub * 32 + lane; pr < D / 2; pr += wpr * 32) {  // column pairs
            float a0 = 0.f, a1 = 0.f;
            for (int k = 0; k < wpr; ++k) {
                a0 += s_acc[slot * wpr + k][2 * pr];
                a1 += s_acc[slot * wpr + k][2 * pr + 1];
            }
            *reinterpret_cast<uint32_t*>(orow + 2 * pr) = Elem<T>::pack2(a0 * inv, a1 * inv);
        }
    }
}

// Packed sequences (token-major Q/O [total_q][Hq][D], K/V [total_k][Hkv][D]): tensor
// maps over (D, heads, tokens) with one head's rows per box; one grid column per
// sequence, sized for the longest one.
template <int D, typename T>
int launch_varlen(const void* Q, const void* K, const void* V, void* O, const int* cu_q, const int* cu_k,
                  int max_sq, int total_q, int total_k, int B, int Hq, int Hkv, float scale, int causal,
                  cudaStream_t st) {
    using L = Layout<D>;
    const CUtensorMapDataType dt = Elem<T>::kFmt == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap tq, tk, tv;
    int rc = make_tmap_4d(&tq, Q, dt, 2, D, Hq, total_q, 1, 64, 1, BM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap_4d(&tk, K, dt, 2, D, Hkv, total_k, 1, 64, 1, BN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap_4d(&tv, V, dt, 2, D, Hkv, total_k, 1, 64, 1, BN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    Params p{};
    p.O = O;
    p.cu_q = cu_q;
    p.cu_k = cu_k;
    p.part_o = nullptr;
    p.part_ml = nullptr;
    p.Hq = Hq;
    p.Sq = 0;   // per sequence, from cu_q
    p.Skv = 0;  // per sequence, from cu_k
    p.group = Hq / Hkv;
    p.n_ctas = (max_sq + kQTiles * BM - 1) / (kQTiles * BM);
    p.causal = causal;
    p.nsplit = 1;
    p.tiles_per_split = 1 << 30;
    p.total_q = total_q;
    p.total_k = total_k;
    p.max_sq = max_sq;
    p.scale_log2 = scale * 1.4426950408889634f;
    auto kern = attn_fwd_kernel<D, T, false, true>;
    B200_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc));
    kern<<<dim3(p.n_ctas, Hq, B), kThreads, L::kAlloc, st>>>(tq, tk, tv, p);
    count_launch(1);
    B200_TRY_CUDA(cudaGetLastError());
    return B200LAB_OK;
}

inline size_t align_up_floats(size_t n) { return (n + 63) / 64 * 64; }  // 256-byte steps

// Key splits for a launch: split the key tiles only when the (query-tile pair,
// q-head, batch) grid cannot fill the GPU; each split gets >= 2 key tiles.
struct SplitPlan {
    int nsplit, tiles_per_split;
};
SplitPlan plan_splits(int B, int Hq, int Sq, int Skv) {
    const int sms = device_sm_count();
    const long long base = (long long)((Sq + kQTiles * BM - 1) / (kQTiles * BM)) * Hq * B;
    const int nkv = (Skv + BN - 1) / BN;
    SplitPlan sp{1, nkv};
    if (base >= sms || nkv < 4) return sp;
    long long want_ll = sms / base;  // one wave: at most one CTA an SM
    if (want_ll > 64) want_ll = 64;
    int want = (int)want_ll;
    want = min(want, nkv / 2);
    if (want < 2) return sp;
    sp.tiles_per_split = (nkv + want - 1) / want;
    sp.nsplit = (nkv + sp.tiles_per_split - 1) / sp.tiles_per_split;
    return sp;
}

// Short queries of a GQA group are packed into the rows of one query tile pair: the q-heads
// of a kv group are adjacent, so [B][Hq][Sq][D] is [B*Hkv][group*Sq][D], and row r of kv-head
// h is query r % Sq of q-head h*group + r / Sq.  The kernel then runs with Hkv "heads" of
// group*Sq rows: K/V are read once per group, the 128-row tiles are filled, and the causal
// mask takes the query index r % Sq.  Partial and output rows keep their addresses.
struct RowShape {
    int Hq, Sq, pack_sq;
};
RowShape row_shape(int Hq, int Hkv, int Sq) {
    const int group = Hq / Hkv;
    if (group > 1 && Sq < kQTiles * BM) return RowShape{Hkv, group * Sq, Sq};
    return RowShape{Hq, Sq, 0};
}

size_t split_workspace_bytes(int B, int Hq, int Sq, int Skv, int D) {
    const SplitPlan sp = plan_splits(B, Hq, Sq, Skv);
    if (sp.nsplit <= 1) return 0;
    const size_t rows = (size_t)B * Hq * Sq;
    return rows * sp.nsplit * ((size_t)D + 2) * sizeof(float) + 256;
}

template <int D, typename T>
int launch(const void* Q, const void* K, const void* V, void* O, int B, int Hq, int Hkv, int Sq,
           int Skv, float scale, int causal, void* ws, size_t ws_bytes, cudaStream_t st) {
    using L = Layout<D>;
    const CUtensorMapDataType dt = Elem<T>::kFmt == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const int group = Hq / Hkv;
    const RowShape rs = row_shape(Hq, Hkv, Sq);
    Hq = rs.Hq;
    Sq = rs.Sq;
    CUtensorMap tq, tk, tv;
    int rc = make_tmap_3d(&tq, Q, dt, 2, D, Sq, (uint64_t)B * Hq, 64, BM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap_3d(&tk, K, dt, 2, D, Skv, (uint64_t)B * Hkv, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap_3d(&tv, V, dt, 2, D, Skv, (uint64_t)B * Hkv, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    Params p{};
    p.O = O;
    p.Hq = Hq;
    p.Sq = Sq;
    p.Skv = Skv;
    p.group = rs.pack_sq ? 1 : group;
    p.pack_sq = rs.pack_sq;
    p.n_ctas = (Sq + kQTiles * BM - 1) / (kQTiles * BM);
    p.causal = causal;
    p.scale_log2 = scale * 1.4426950408889634f;
    SplitPlan sp = plan_splits(B, Hq, Sq, Skv);
    const size_t need = split_workspace_bytes(B, Hq, Sq, Skv, D);
    if (sp.nsplit > 1 && (ws == nullptr || ws_bytes < need)) sp = SplitPlan{1, (Skv + BN - 1) / BN};
    p.nsplit = sp.nsplit;
    p.tiles_per_split = sp.tiles_per_split;
    p.tail_groups = causal_tail_groups(p.n_ctas * p.nsplit, B * Hq);
    const size_t rows = (size_t)B * Hq * Sq;
    p.part_o = nullptr;
    p.part_ml = nullptr;
    if (sp.nsplit > 1) {
        p.part_ml = static_cast<float*>(ws);
        p.part_o = p.part_ml + align_up_floats(rows * sp.nsplit * 2);
    }
    dim3 grid(p.n_ctas * p.nsplit, Hq, B);
    auto kern = sp.nsplit > 1 ? attn_fwd_kernel<D, T, true> : attn_fwd_kernel<D, T, false>;
    B200_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc));
    kern<<<grid, kThreads, L::kAlloc, st>>>(tq, tk, tv, p);
    count_launch(1);
    B200_TRY_CUDA(cudaGetLastError());
    if (sp.nsplit > 1) {
        // a programmatic dependent of the split kernel: its launch overlaps that grid's
        // drain, and griddepcontrol.wait in the kernel orders its reads after the partials
        cudaLaunchConfig_t cc = {};
        // warps per row: enough that a warp owns at most 8 splits, then more (up to
        // min(nsplit, 8)) while the grid has fewer than ~16 warps an SM
        int wpr_log2 = 0;
        while ((8 << wpr_log2) < sp.nsplit) ++wpr_log2;
        while (wpr_log2 < 3 && (1 << wpr_log2) < sp.nsplit &&
               (long long)rows * (1 << wpr_log2) < 16LL * device_sm_count())
            ++wpr_log2;
        const int rpb = 8 >> wpr_log2;
        cc.gridDim = dim3((unsigned)((rows + rpb - 1) / rpb));
        cc.blockDim = dim3(256);
        cc.stream = st;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        cc.attrs = at;
        cc.numAttrs = 1;
        B200_TRY_CUDA(cudaLaunchKernelEx(&cc, attn_combine_kernel<D, T>, (const float*)p.part_o,
                                         (const float*)p.part_ml, static_cast<T*>(O), (long long)rows,
                                         sp.nsplit, wpr_log2));
        count_launch(1);
        B200_TRY_CUDA(cudaGetLastError());
    }
    return B200LAB_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace b200

B200_DEFINE_ERR_TAKER(attn, b200::g_err_attn)

namespace b200 {
// attn_gated.cu: head dim 256 (one query tile per CTA, double-buffered S)
int attn_d256_launch(const void* Q, const void* K, const void* V, const void* G, void* O, int B, int Hq,
                     int Hkv, int Sq, int Skv, float scale, int causal, int dtype, void* stream);
}  // namespace b200

extern "C" size_t attn_fwd_sm100_workspace(int B, int Hq, int Hkv, int Sq, int Skv, int D,
                                           int causal) {
    (void)causal;
    if (B < 1 || Hq < 1 || Hkv < 1 || Hq % Hkv || Sq < 1 || Skv < 1 || (D != 64 && D != 128)) return 0;
    const b200::RowShape rs = b200::row_shape(Hq, Hkv, Sq);
    return b200::split_workspace_bytes(B, rs.Hq, rs.Sq, Skv, D);
}

extern "C" int attn_fwd_sm100(const void* Q, const void* K, const void* V, void* O, int B, int Hq,
                              int Hkv, int Sq, int Skv, int D, float scale, int causal, int dtype,
                              void* workspace, size_t ws_bytes, void* stream) {
    using namespace b200;
    if (!Q || !K || !V || !O) return B200LAB_ERR_INVALID;
    if (B < 1 || Hq < 1 || Hkv < 1 || Sq < 1 || Skv < 1 || Hq % Hkv != 0) return B200LAB_ERR_INVALID;
    if (dtype != B200LAB_F16 && dtype != B200LAB_BF16) return B200LAB_ERR_INVALID;
    if (causal != 0 && causal != 1) return B200LAB_ERR_INVALID;
    if (!(scale > 0.f) || !(scale < 1e30f)) return B200LAB_ERR_INVALID;
    if (D != 64 && D != 128 && D != 256) return B200LAB_ERR_UNSUPPORTED;
    if (B > 65535 || Hq > 65535) return B200LAB_ERR_UNSUPPORTED;
    if (D == 256)  // no split-KV for this head dim: the workspace is not used
        return attn_d256_launch(Q, K, V, nullptr, O, B, Hq, Hkv, Sq, Skv, scale, causal, dtype, stream);
    if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O)) return B200LAB_ERR_INVALID;
    int rc = check_device_sm100();
    if (rc != B200LAB_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (dtype == B200LAB_BF16) {
        return D == 128 ? launch<128, __nv_bfloat16>(Q, K, V, O, B, Hq, Hkv, Sq, Skv, scale, causal, workspace, ws_bytes, st)
                        : launch<64, __nv_bfloat16>(Q, K, V, O, B, Hq, Hkv, Sq, Skv, scale, causal, workspace, ws_bytes, st);
    }
    return D == 128 ? launch<128, __half>(Q, K, V, O, B, Hq, Hkv, Sq, Skv, scale, causal, workspace, ws_bytes, st)
                    : launch<64, __half>(Q, K, V, O, B, Hq, Hkv, Sq, Skv, scale, causal, workspace, ws_bytes, st);
}

namespace {
// Streams and events of the host-buffer pipeline.  A host thread creates them on its first
// call for a device and keeps them until it exits: creating two streams and up to 130 events
// on every call cost ~0.25 ms of a C5 call, all of it while the GPU waited at the call's first
// event.  Kept per thread, so callers on different threads never share them; calls from one
// thread on one device share the two copy streams, so their copies run in call order.
struct HostPipe {
    static constexpr int kEvents = 64;
    cudaStream_t s_in = nullptr, s_out = nullptr;
    cudaEvent_t ev_start = nullptr, ev_end = nullptr;
    cudaEvent_t ev_in[kEvents] = {}, ev_done[kEvents] = {};
    bool ready = false;
    int create() {
        bool ok = cudaStreamCreateWithFlags(&s_in, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaStreamCreateWithFlags(&s_out, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaEventCreateWithFlags(&ev_start, cudaEventDisableTiming) == cudaSuccess &&
                  cudaEventCreateWithFlags(&ev_end, cudaEventDisableTiming) == cudaSuccess;
        for (int i = 0; ok && i < kEvents; ++i)
            ok = cudaEventCreateWithFlags(&ev_in[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&ev_done[i], cudaEventDisableTiming) == cudaSuccess;
        if (!ok) {
            destroy();
            return B200LAB_ERR_CUDA;
        }
        ready = true;
        return B200LAB_OK;
    }
    void destroy() {
        for (int i = 0; i < kEvents; ++i) {
            if (ev_in[i]) cudaEventDestroy(ev_in[i]);
            if (ev_done[i]) cudaEventDestroy(ev_done[i]);
            ev_in[i] = ev_done[i] = nullptr;
        }
        if (ev_start) cudaEventDestroy(ev_start);
        if (ev_end) cudaEventDestroy(ev_end);
        if (s_in) cudaStreamDestroy(s_in);
        if (s_out) cudaStreamDestroy(s_out);
        ev_start = ev_end = nullptr;
        s_in = s_out = nullptr;
        ready = false;
    }
    ~HostPipe() { destroy(); }
};
constexpr int kPipeDevices = 16;
thread_local HostPipe t_host_pipes[kPipeDevices];
}  // namespace

// Host-buffer pipeline over attn_fwd_sm100: chunks of whole (batch, kv-head) units.  Units
// are numbered b * Hkv + kv-head; any run of consecutive units is one contiguous slab of Q/O
// ([B][Hq][Sq][D], the q-heads of a kv group adjacent) and of K/V, so a chunk is one call with
// B = 1, Hq = n * group, Hkv = n over its slab, whatever batch boundaries it spans.
extern "C" int attn_fwd_sm100_host(const void* Qh, const void* Kh, const void* Vh, void* Oh, void* Qd, void* Kd,
                                   void* Vd, void* Od, int B, int Hq, int Hkv, int Sq, int Skv, int D, float scale,
                                   int causal, int dtype, void* stream) {
    using namespace b200;
    if (!Qh || !Kh || !Vh || !Oh || !Qd || !Kd || !Vd || !Od) return B200LAB_ERR_INVALID;
    if (B < 1 || Hq < 1 || Hkv < 1 || Sq < 1 || Skv < 1 || Hq % Hkv != 0) return B200LAB_ERR_INVALID;
    if (dtype != B200LAB_F16 && dtype != B200LAB_BF16) return B200LAB_ERR_INVALID;
    if (causal != 0 && causal != 1) return B200LAB_ERR_INVALID;
    if (!(scale > 0.f) || !(scale < 1e30f)) return B200LAB_ERR_INVALID;
    if (D != 64 && D != 128 && D != 256) return B200LAB_ERR_UNSUPPORTED;
    if (B > 65535 || Hq > 65535) return B200LAB_ERR_UNSUPPORTED;
    int rc = check_device_sm100();
    if (rc != B200LAB_OK) return rc;
    const int group = Hq / Hkv;
    // Chunk schedule, in units: about an eighth of the units a chunk, and the last two such
    // chunks' worth split into halves then quarters.  The copies in run back to back; what
    // follows the last of them (that chunk's kernel and copy out) is the pipeline's tail,
    // which the small final chunks shorten.  C5 (32 units): 4 x 6, 2, 2, 1 x 4 took 18.05 ms
    // against 18.98 ms for eight chunks of 4 (the copies alone, pipelined: ~17 ms); chunks of
    // 1 or 2 units throughout were slower (smaller copies move fewer bytes a second).
    const long long units = (long long)B * Hkv;
    if (units > (1LL << 30)) return B200LAB_ERR_UNSUPPORTED;
    const int nunits = static_cast<int>(units);
    std::vector<int> sched;
    {
        int c = nunits / 8 > 1 ? nunits / 8 : 1;
        if (c > 65535 / Hq * Hkv) c = 65535 / Hq * Hkv;  // a chunk's q-heads stay a grid dimension
        if (c < 1) c = 1;
        const int tail = nunits < 2 * c ? nunits : 2 * c;
        const int head = nunits - tail;
        for (int u = 0; u < head; u += c) sched.push_back(c < head - u ? c : head - u);
        const int half = c / 2 > 1 ? c / 2 : 1, quarter = c / 4 > 1 ? c / 4 : 1;
        int rem = tail;
        for (int k = 0; k < 2 && rem > 0; ++k) {
            const int n = half < rem ? half : rem;
            sched.push_back(n);
            rem -= n;
        }
        while (rem > 0) {
            const int n = quarter < rem ? quarter : rem;
            sched.push_back(n);
            rem -= n;
        }
    }
    const int nchunks = static_cast<int>(sched.size());
    const size_t esz = 2;
    const size_t q_unit = (size_t)group * Sq * D * esz;  // Q or O bytes of a unit
    const size_t kv_unit = (size_t)Skv * D * esz;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int nev = nchunks < HostPipe::kEvents ? nchunks : HostPipe::kEvents;  // reused round-robin past that
    auto fail = [&](int code) { rc = code; };
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return B200LAB_ERR_CUDA;
    HostPipe per_call;  // devices past the per-thread cache get their own, destroyed on return
    HostPipe& pipe = (dev >= 0 && dev < kPipeDevices) ? t_host_pipes[dev] : per_call;
    if (!pipe.ready && pipe.create() != B200LAB_OK) return B200LAB_ERR_CUDA;
    cudaStream_t s_in = pipe.s_in, s_out = pipe.s_out;
    cudaEvent_t ev_start = pipe.ev_start, ev_end = pipe.ev_end;
    cudaEvent_t* ev_in = pipe.ev_in;
    cudaEvent_t* ev_done = pipe.ev_done;
    if (rc == B200LAB_OK) {
        // the device buffers may still be in use by earlier work on `stream`
        if (cudaEventRecord(ev_start, st) != cudaSuccess || cudaStreamWaitEvent(s_in, ev_start, 0) != cudaSuccess ||
            cudaStreamWaitEvent(s_out, ev_start, 0) != cudaSuccess)
            fail(B200LAB_ERR_CUDA);
    }
    const char* qh = static_cast<const char*>(Qh);
    const char* kh = static_cast<const char*>(Kh);
    const char* vh = static_cast<const char*>(Vh);
    char* oh = static_cast<char*>(Oh);
    char* qd = static_cast<char*>(Qd);
    char* kd = static_cast<char*>(Kd);
    char* vd = static_cast<char*>(Vd);
    char* od = static_cast<char*>(Od);
    size_t u0 = 0;  // first unit of chunk i
    for (int i = 0; rc == B200LAB_OK && i < nchunks; u0 += sched[i], ++i) {
        const int hc = sched[i];  // units (kv-heads) of this chunk
        const size_t qo = u0 * q_unit, ko = u0 * kv_unit;
        const size_t q_chunk = (size_t)hc * q_unit, kv_chunk = (size_t)hc * kv_unit;
        cudaEvent_t ein = ev_in[i % nev], edone = ev_done[i % nev];
        if (cudaMemcpyAsync(qd + qo, qh + qo, q_chunk, cudaMemcpyHostToDevice, s_in) != cudaSuccess ||
            cudaMemcpyAsync(kd + ko, kh + ko, kv_chunk, cudaMemcpyHostToDevice, s_in) != cudaSuccess ||
            cudaMemcpyAsync(vd + ko, vh + ko, kv_chunk, cudaMemcpyHostToDevice, s_in) != cudaSuccess ||
            cudaEventRecord(ein, s_in) != cudaSuccess || cudaStreamWaitEvent(st, ein, 0) != cudaSuccess) {
            fail(B200LAB_ERR_CUDA);
            break;
        }
        const int lrc = attn_fwd_sm100(qd + qo, kd + ko, vd + ko, od + qo, 1, hc * group, hc, Sq, Skv, D, scale,
                                       causal, dtype, nullptr, 0, stream);
        if (lrc != B200LAB_OK) {
            fail(lrc);
            break;
        }
        if (cudaEventRecord(edone, st) != cudaSuccess || cudaStreamWaitEvent(s_out, edone, 0) != cudaSuccess ||
            cudaMemcpyAsync(oh + qo, od + qo, q_chunk, cudaMemcpyDeviceToHost, s_out) != cudaSuccess) {
            fail(B200LAB_ERR_CUDA);
            break;
        }
    }
    // join: `stream` continues after every copy of this call, whatever happened above
    bool joined = cudaEventRecord(ev_end, s_in) == cudaSuccess && cudaStreamWaitEvent(st, ev_end, 0) == cudaSuccess;
    joined = cudaEventRecord(ev_start, s_out) == cudaSuccess && cudaStreamWaitEvent(st, ev_start, 0) == cudaSuccess &&
             joined;
    // a CUDA failure on the cached streams or events (e.g. after cudaDeviceReset, which
    // invalidates them) drops the cache, so the next call on this thread creates them anew
    if ((rc == B200LAB_ERR_CUDA || !joined) && &pipe != &per_call) pipe.destroy();
    return joined ? rc : B200LAB_ERR_CUDA;
}

extern "C" int attn_fwd_sm100_varlen(const void* Q, const void* K, const void* V, void* O, const int* cu_seqlens_q,
                                     const int* cu_seqlens_k, int max_seqlen_q, int total_q, int total_k, int B,
                                     int Hq, int Hkv, int D, float scale, int causal, int dtype, void* stream) {
    using namespace b200;
    if (!Q || !K || !V || !O || !cu_seqlens_q || !cu_seqlens_k) return B200LAB_ERR_INVALID;
    if (B < 1 || Hq < 1 || Hkv < 1 || Hq % Hkv != 0 || max_seqlen_q < 1 || total_q < 1 || total_k < 1)
        return B200LAB_ERR_INVALID;
    if (dtype != B200LAB_F16 && dtype != B200LAB_BF16) return B200LAB_ERR_INVALID;
    if (causal != 0 && causal != 1) return B200LAB_ERR_INVALID;
    if (!(scale > 0.f) || !(scale < 1e30f)) return B200LAB_ERR_INVALID;
    if (D != 64 && D != 128) return B200LAB_ERR_UNSUPPORTED;
    if (B > 65535 || Hq > 65535) return B200LAB_ERR_UNSUPPORTED;
    if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O)) return B200LAB_ERR_INVALID;
    int rc = check_device_sm100();
    if (rc != B200LAB_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (dtype == B200LAB_BF16)
        return D == 128 ? launch_varlen<128, __nv_bfloat16>(Q, K, V, O, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                                            total_q, total_k, B, Hq, Hkv, scale, causal, st)
                        : launch_varlen<64, __nv_bfloat16>(Q, K, V, O, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                                           total_q, total_k, B, Hq, Hkv, scale, causal, st);
    return D == 128 ? launch_varlen<128, __half>(Q, K, V, O, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, total_q,
                                                 total_k, B, Hq, Hkv, scale, causal, st)
                    : launch_varlen<64, __half>(Q, K, V, O, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, total_q,
                                                total_k, B, Hq, Hkv, scale, causal, st);
}
