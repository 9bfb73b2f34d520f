// gdn_prefill.cu -- chunked Gated DeltaNet prefill for sm_100a (tcgen05 + TMA).
//
// Reference semantics: the recurrence of src/gdn_sm75.cu:6-11 (gdn_cpu,
// :1078-1106), computed with the chunked WY/UT algebra of gdn_chunked_cpu
// (:1109-1244) and the reference's two-pass split gdn_prep_kernel /
// gdn_apply_kernel (:896-1073).  The triangular solve here is the exact
// (I + A)^-1, so the chunked result equals the recurrence (the reference's
// own solve loop is not exact; see oracle/oracle.c).
//
// Chunk C = 64 tokens.  Per chunk, with gcs = cumsum(g_log), Gam = e^gcs:
//   A[t][s]  = beta_t (k_t.k_s) e^{gcs_t-gcs_s}      s < t
//   T        = (I + A)^-1
//   W        = T diag(beta Gam) K          U = T diag(beta) V
//   Aqk[t][s]= (q_t.k_s) e^{gcs_t-gcs_s}              s <= t
//   Vn       = U - W S^T                    (state-dependent, sequential)
//   o_t      = scale (Gam_t (S q_t) + sum_s Aqk[t][s] Vn_s)
//   S       <- e^{gcs_last} S + sum_t e^{gcs_last-gcs_t} Vn_t k_t^T
//
// Kernel 1, gdn_prep_kernel: one CTA per (b, v-head, chunk), fully parallel.
//   TMA loads K, Q, V chunk tiles; ONE M=128 tcgen05 MMA gives [K;Q] K^T
//   (lanes 0-63: K K^T, lanes 64-127: Q K^T); the threads form A and Aqk,
//   invert (I + A) as a 2 x 2 block inverse in fp32, and two M=128, N=128 MMAs give
//   [T diag(beta Gam); T diag(beta)] K -> W and [...] V -> U.  A last MMA gives
//   M = W K_prev^T diag(e^{gcs_last,prev - gcs_prev}) against the previous chunk's keys.
//   W, U, Aqk, M (16-bit) and gcs (fp32) go to the workspace.
// Kernel 2, gdn_state_kernel: one CTA per (b, v-head, 32-column slice of the
//   state), sequential over chunks, with the chain carried by Vn:
//     Vn_{c+1} = U_{c+1} - e^{gcs_last,c} W_{c+1} S_c^T - M_{c+1} Vn_c
//   so that between Vn_c and Vn_{c+1} sits one 64-deep MMA ([Aqk_c; M_{c+1}] Vn_c,
//   which also gives the intra-chunk output), while the 128-deep [Q_c; W_{c+1}] S_c^T
//   and the state update S_{c+1} = e^{gcs_last} S_c + K_c^T diag(..) Vn_c run beside it
//   on their own warps and MMA thread.
// Every wait is bounded (common.cuh).
#include <algorithm>

#include "common.cuh"
#include "errwords.h"

namespace b200 {
namespace {

__device__ int g_err_gdn_prefill = 0;

constexpr int kC = 64;    // chunk length
constexpr int kD = 128;   // dk = dv
constexpr int kSlice = 32;  // state columns (v dim) per kernel-2 CTA

// ---- workspace layout ------------------------------------------------------
struct WsLayout {
    size_t w, u, aqk, m, gcs, rq, rk, total;
};
__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
__host__ __device__ inline WsLayout ws_layout(size_t nbhc) {
    WsLayout L;
    L.w = 0;
    L.u = align_up(L.w + nbhc * kC * kD * 2, 1024);
    L.aqk = align_up(L.u + nbhc * kC * kD * 2, 1024);
    L.m = align_up(L.aqk + nbhc * kC * kC * 2, 1024);
    L.gcs = align_up(L.m + nbhc * kC * kC * 2, 1024);
    L.rq = align_up(L.gcs + nbhc * kC * 4, 1024);   // 1/|q_t|, 1/|k_t| (fused entry only)
    L.rk = align_up(L.rq + nbhc * kC * 4, 1024);
    L.total = align_up(L.rk + nbhc * kC * 4, 1024);
    return L;
}

struct PrepParams {
    uint8_t* ws;
    const float* g_log;    // fused: the gate logits a
    const float* beta;     // fused: the beta logits b
    const float* A_log;    // fused: [Hv] or null
    const float* dt_bias;  // fused: [Hv] or null
    size_t ws_u, ws_aqk, ws_gcs, ws_rq, ws_rk;
    const int* cu;  // packed sequences: [B+1] token offsets (device), or null: B x T dense
    int T, Hqk, Hv, nch, head_map;  // with cu, T is the longest sequence; nch = ceil(T / 64)
    int ntok;                       // tokens in the flattened dimension (B*T, or cu[B])
};

// Tokens are addressed in one flattened sequence dimension ([B*T] dense, [total] packed), so
// chunk c of sequence b starts at token seq_start + 64 c.  The last chunk of a sequence may
// read the next sequence's rows (or zero fill past the end): those tokens get g = beta = 0,
// which zeroes every product they could enter (their A, W and U rows, their columns of W and
// U through beta, their Vn rows), and their outputs are not stored.
struct SeqSpan {
    int start, len;
};
__device__ __forceinline__ SeqSpan seq_span(const int* cu, int T, int b) {
    if (cu) return SeqSpan{cu[b], cu[b + 1] - cu[b]};
    return SeqSpan{b * T, T};
}
// A packed sequence must lie inside [0, ntok) and be no longer than the T the grid and the
// workspace were sized for; a caller's offsets that break this are reported, not followed.
__device__ __forceinline__ bool seq_ok(SeqSpan s, int T, int ntok) {
    return s.start >= 0 && s.len >= 0 && s.len <= T && s.start <= ntok - s.len;
}

// Fused pre-processing (gdn_prefill_sm100_fused): q, k arrive raw and are L2-normalised,
// x * rsqrt(sum x^2 + kNormEps) over dk; the gates come as logits,
// g_log = -exp(A_log[h]) softplus(a + dt_bias[h]), beta = sigmoid(b).  The tensor-core
// tiles stay the raw 16-bit q, k: the per-token factors 1/|q_t|, 1/|k_t| enter where the
// products are scaled anyway (A, Aqk, the column scale of W, M, the decayed V_new rows and
// the Q S^T output term).
constexpr float kNormEps = 1e-6f;
__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(__expf(x)); }
__device__ __forceinline__ float fused_gate(float a, const PrepParams& p, int h) {
    const float decay = p.A_log ? __expf(p.A_log[h]) : 1.f;
    return -decay * softplus(a + (p.dt_bias ? p.dt_bias[h] : 0.f));
}
// 1/|row| of a 64-token x 128-dim 16-bit tile held as two 128B-swizzled 64-column boxes
template <typename T16>
__device__ __forceinline__ float row_rnorm(const uint8_t* box0, const uint8_t* box1, int r) {
    float acc = 0.f;
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        const uint8_t* row = (b ? box1 : box0) + r * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint4 raw = *reinterpret_cast<const uint4*>(row + ((c ^ (r & 7)) << 4));
            const T16* e = reinterpret_cast<const T16*>(&raw);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float x = Elem<T16>::to_f(e[u]);
                acc = fmaf(x, x, acc);
            }
        }
    }
    return rsqrtf(acc + kNormEps);
}

__device__ __forceinline__ int qk_head(int h, int Hqk, int Hv, int head_map) {
    return head_map == 0 ? h % Hqk : h / (Hv / Hqk);
}

// ===========================================================================
// Kernel 1: per-chunk preparation
// ===========================================================================
namespace prep {
constexpr int kThreads = 128;
// shared layout (bytes)
// [K0|Q0|K1|Q1], 8 KiB each (64 tokens x 64 dims); V0/V1 are loaded over Q0/Q1 once the
// first MMA has read Q (so the first TMA wait covers K and Q only)
constexpr int kTiles = 0;
constexpr int kK0 = 0, kQ0 = 8192, kK1 = 16384, kQ1 = 24576, kV0 = kQ0, kV1 = kQ1;
constexpr int kLd = 68;            // fp32 row pitch of A and T (16-byte aligned, fewer conflicts)
// One region, in turn: A, then T = (I + A)^-1 in place (fp32 64 x kLd; the block inverse's
// 32 x 32 scratch sits in its upper-right block, zero in A and in T); then, once every thread
// holds its row of T in registers, AT = [T diag(beta Gam); T diag(beta)] (16-bit 128 x 64, the
// A operand of the W and U products); after those, the previous chunk's K (for M); last, M
// staged for its store.
constexpr int kAs = 32768;
constexpr int kAT = kAs;
constexpr int kMisc = kAs + kC * kLd * 4;
constexpr int kBytes = kMisc + 3072;
constexpr int kAlloc = kBytes + 1024;
static_assert(4 * (kAlloc + 1024) <= 233472, "four prep CTAs per SM");
// 128 columns: four CTAs per SM fit the 512 TMEM columns without one waiting in
// tcgen05.alloc for another to exit (W and U are produced one after the other)
constexpr uint32_t kTmemCols = 128;

struct Misc {
    float gcs[kC];   // natural log units (stored to the workspace)
    float g2[kC];    // gcs * log2(e), for ex2
    float beta[kC];
    float colscale[2 * kC];  // [beta Gam | beta], the column scales of T' and T''
    float gprev[kC];         // cumsum of g_log over the previous chunk (for M)
    float rk[kC], rq[kC];    // 1/|k_t|, 1/|q_t| (fused; else 1)
    float rkp[kC];           // 1/|k_s| of the previous chunk (fused; else 1)
    float mdecay[kC];        // e^{gprev_last - gprev_s}, the column decay of M
    uint64_t bar_tma, bar_v, bar_mma1, bar_mma2, bar_kp, bar_m, drain;
    uint32_t tmem_base;
    int abort;
};
static_assert(sizeof(Misc) <= kBytes - kMisc, "prep Misc overflows its slot");
}  // namespace prep

__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// T = (I + A)^-1 for a strictly lower 64 x 64 A (fp32, shared, row pitch kLd)
// as a 2 x 2 block inverse of 32 x 32 blocks:
//   T11 = (I + A11)^-1, T22 = (I + A22)^-1      (warp 0 / warp 1: one column per
//                                                lane, forward substitution)
//   T21 = -T22 (A21 T11),  T12 = 0              (all 128 threads, 8 outputs each)
// In place: T overwrites A (fp32, row pitch kLd; the upper triangle of A is zero and stays
// so); X (32 x 32) is scratch.  The diagonal blocks are done by the warp that built their
// rows of A (diag_block_inverse, right after that warp's rows are written, while the other
// two warps still build Aqk); the off-diagonal block after a CTA barrier.
__device__ __forceinline__ void diag_block_inverse(float* As, int warp, int lane) {
    using prep::kLd;
    float* Ts = As;
    {
        const int o = warp * 32;  // diagonal block origin
        const int j = lane;       // column within the block
        float col[32];
#pragma unroll
        for (int b = 0; b < 4; ++b) {   // rows in blocks of 8: 8 independent chains
            const int t0 = b * 8;
            float acc[8];
#pragma unroll
            for (int r = 0; r < 8; ++r) acc[r] = 0.f;
#pragma unroll
            for (int s = 0; s < t0; s += 4) {
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    const float4 a = *reinterpret_cast<const float4*>(As + (o + t0 + r) * kLd + o + s);
                    acc[r] = fmaf(a.x, col[s], acc[r]);
                    acc[r] = fmaf(a.y, col[s + 1], acc[r]);
                    acc[r] = fmaf(a.z, col[s + 2], acc[r]);
                    acc[r] = fmaf(a.w, col[s + 3], acc[r]);
                }
            }
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                const int t = t0 + r;
                float x = acc[r];
#pragma unroll
                for (int s = 0; s < r; ++s) x = fmaf(As[(o + t) * kLd + o + t0 + s], col[t0 + s], x);
                col[t] = t < j ? 0.f : (t == j ? 1.f : -x);
            }
        }
        __syncwarp();  // every lane has read its block of A before any column is replaced
#pragma unroll
        for (int t = 0; t < 32; ++t) Ts[(o + t) * kLd + o + j] = col[t];
    }
}

// T21 = -T22 (A21 T11) once both diagonal blocks are inverted (all 128 threads; the caller
// has synchronised the CTA after diag_block_inverse).
__device__ __forceinline__ void offdiag_block_inverse(float* As, float* X, int xld, int tid) {
    using prep::kLd;
    float* Ts = As;
    // 128 threads x 8 outputs: row r = tid / 4, columns c0 .. c0 + 7 with c0 = (tid % 4) * 8
    const int r = tid >> 2, c0 = (tid & 3) * 8;
    {   // X = A21 T11
        float acc[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) acc[u] = 0.f;
#pragma unroll
        for (int s = 0; s < 32; ++s) {
            const float a = As[(32 + r) * kLd + s];
            const float4 t0 = *reinterpret_cast<const float4*>(Ts + s * kLd + c0);
            const float4 t1 = *reinterpret_cast<const float4*>(Ts + s * kLd + c0 + 4);
            acc[0] = fmaf(a, t0.x, acc[0]); acc[1] = fmaf(a, t0.y, acc[1]);
            acc[2] = fmaf(a, t0.z, acc[2]); acc[3] = fmaf(a, t0.w, acc[3]);
            acc[4] = fmaf(a, t1.x, acc[4]); acc[5] = fmaf(a, t1.y, acc[5]);
            acc[6] = fmaf(a, t1.z, acc[6]); acc[7] = fmaf(a, t1.w, acc[7]);
        }
        *reinterpret_cast<float4*>(X + r * xld + c0) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        *reinterpret_cast<float4*>(X + r * xld + c0 + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
    __syncthreads();
    {   // T21 = -T22 X
        float acc[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) acc[u] = 0.f;
#pragma unroll
        for (int s = 0; s < 32; ++s) {
            const float a = Ts[(32 + r) * kLd + 32 + s];
            const float4 x0 = *reinterpret_cast<const float4*>(X + s * xld + c0);
            const float4 x1 = *reinterpret_cast<const float4*>(X + s * xld + c0 + 4);
            acc[0] = fmaf(a, x0.x, acc[0]); acc[1] = fmaf(a, x0.y, acc[1]);
            acc[2] = fmaf(a, x0.z, acc[2]); acc[3] = fmaf(a, x0.w, acc[3]);
            acc[4] = fmaf(a, x1.x, acc[4]); acc[5] = fmaf(a, x1.y, acc[5]);
            acc[6] = fmaf(a, x1.z, acc[6]); acc[7] = fmaf(a, x1.w, acc[7]);
        }
        *reinterpret_cast<float4*>(Ts + (32 + r) * kLd + c0) = make_float4(-acc[0], -acc[1], -acc[2], -acc[3]);
        *reinterpret_cast<float4*>(Ts + (32 + r) * kLd + c0 + 4) = make_float4(-acc[4], -acc[5], -acc[6], -acc[7]);
    }
    __syncthreads();
}

template <typename T16, bool kFused>
__global__ void __launch_bounds__(prep::kThreads, 4)
    gdn_prep_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmW,
                    const __grid_constant__ CUtensorMap tmU, const __grid_constant__ CUtensorMap tmAqk,
                    const __grid_constant__ CUtensorMap tmM, const PrepParams p) {
    using namespace prep;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Misc* ms = reinterpret_cast<Misc*>(smem + kMisc);
    float* As = reinterpret_cast<float*>(smem + kAs);
    const float* Ts = As;  // T replaces A in place
    volatile int* abort = &ms->abort;

    const int c = blockIdx.x;   // chunk of the sequence
    const int h = blockIdx.y;   // v-head
    const int b = blockIdx.z;   // sequence
    const SeqSpan seq = seq_span(p.cu, p.T, b);
    if (!seq_ok(seq, p.T, p.ntok)) {
        if (threadIdx.x == 0 && c == 0) atomicExch(&g_err_gdn_prefill, B200LAB_ERR_INVALID);
        return;
    }
    const int t0 = c * kC;
    if (t0 >= seq.len) return;  // packed: a shorter sequence has fewer chunks
    const int hq = qk_head(h, p.Hqk, p.Hv, p.head_map);
    const int tok0 = seq.start + t0;  // first token of the chunk in the flattened dimension
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const size_t bhc = ((size_t)b * p.Hv + h) * p.nch + c;
    // the state pass may be scheduled once every prep CTA is running; it waits for this
    // grid's results itself (grid_dependency_wait)
    allow_dependent_launch();
    // gate inputs, loaded first so their latency overlaps the setup: threads 0-63 this
    // chunk's g_log and beta (padded tokens keep g = 0, beta = 0), threads 64-127 the
    // previous (always full) chunk's g_log, for M
    float g_in = 0.f, be_in = 0.f;
    if (tid < kC) {
        if (t0 + tid < seq.len) {
            const size_t gi = ((size_t)tok0 + tid) * p.Hv + h;
            g_in = p.g_log[gi];
            be_in = p.beta[gi];
        }
    } else if (c > 0) {
        g_in = p.g_log[((size_t)tok0 - kC + tid - kC) * p.Hv + h];
    }

    if (tid == 0) {
        mbar_init(&ms->bar_tma, 1);
        mbar_init(&ms->bar_v, 1);
        mbar_init(&ms->bar_mma1, 1);
        mbar_init(&ms->bar_mma2, 1);
        mbar_init(&ms->bar_kp, 1);
        mbar_init(&ms->bar_m, 1);
        mbar_init(&ms->drain, 1);
        ms->abort = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(&ms->tmem_base, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ms->tmem_base;

    if (tid == 0) {
        mbar_arrive_expect_tx(&ms->bar_tma, 4 * 8192);
        tma_load_4d(smem + kK0, &tmK, &ms->bar_tma, 0, hq, tok0, 0);
        tma_load_4d(smem + kK1, &tmK, &ms->bar_tma, 64, hq, tok0, 0);
        tma_load_4d(smem + kQ0, &tmQ, &ms->bar_tma, 0, hq, tok0, 0);
        tma_load_4d(smem + kQ1, &tmQ, &ms->bar_tma, 64, hq, tok0, 0);
    }
    // gates: gcs = inclusive prefix sum of g_log over the chunk (padded tokens: g=0, beta=0)
    if (tid < kC) {
        float g = g_in, be = be_in;
        if constexpr (kFused) {
            if (t0 + tid < seq.len) {
                g = fused_gate(g, p, h);
                be = 1.f / (1.f + __expf(-be));
            }
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, g, o);
            if (lane >= o) g += y;
        }
        ms->gcs[tid] = g;  // per-warp inclusive scan; warp 1 adds warp 0's total below
        ms->beta[tid] = be;
    } else if (c > 0) {
        // warps 2-3: the same scan over the previous (always full) chunk, for M
        float g = g_in;
        if constexpr (kFused) g = fused_gate(g, p, h);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, g, o);
            if (lane >= o) g += y;
        }
        ms->gprev[tid - kC] = g;
    }
    __syncthreads();
    if (tid < kC) {
        const float g = tid >= 32 ? ms->gcs[tid] + ms->gcs[31] : ms->gcs[tid];
        __syncwarp();
        ms->gcs[tid] = g;
        ms->g2[tid] = g * 1.4426950408889634f;
    } else if (c > 0) {
        const int t = tid - kC;
        const float g = t >= 32 ? ms->gprev[t] + ms->gprev[31] : ms->gprev[t];
        __syncwarp();
        ms->gprev[t] = g;
    }
    __syncthreads();
    if (tid >= kC && c > 0) ms->mdecay[tid - kC] = __expf(ms->gprev[kC - 1] - ms->gprev[tid - kC]);

    // MMA1: [K;Q] K^T  (M=128, N=64, K=128)
    bool ok = true;
    if (tid == 0) {
        ok = mbar_wait(&ms->bar_tma, 0, abort, &g_err_gdn_prefill);
        if (ok) {
            tc_fence_after();
            constexpr uint32_t idesc = make_idesc(Elem<T16>::kFmt, 128, 64, false, false);
            const uint32_t base = smem_u32(smem + kTiles);
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk) {
                const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                mma_f16_ss(tmem, smem_desc(base + off, 16, 1024, kLayoutSW128),
                           smem_desc(base + off, 16, 1024, kLayoutSW128), idesc, kk > 0 ? 1u : 0u);
            }
            mma_commit(&ms->bar_mma1);
        }
    }
    if constexpr (kFused) {
        // per-token 1/|q_t| from the Q tile while MMA1 runs (warps 2-3); these reads of Q come
        // before the V load's writes over it
        ok = __all_sync(0xffffffffu, mbar_wait(&ms->bar_tma, 0, abort, &g_err_gdn_prefill));
        if (tid >= kC) ms->rq[tid - kC] = row_rnorm<T16>(smem + kQ0, smem + kQ1, tid - kC);
        fence_proxy_async_smem();
    }
    ok = __all_sync(0xffffffffu, mbar_wait(&ms->bar_mma1, 0, abort, &g_err_gdn_prefill)) && ok;
    if constexpr (kFused) {
        // 1/|k_t| from the diagonal of K K^T, which MMA1 has just made (lanes 0-63): warp w holds
        // rows 32w .. 32w + 31, so its diagonal lies in columns 32w .. 32w + 31
        if (warp < 2) {
            tc_fence_after();
            uint32_t d[32];
            tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + warp * 32, d);
            tmem_ld_wait();
            float kk = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) kk = (i == lane) ? __uint_as_float(d[i]) : kk;
            ms->rk[tid] = ok ? rsqrtf(kk + kNormEps) : 1.f;
        }
        __syncthreads();
    }
    if (tid == 0 && ok) {
        // Q has been read: V goes over it (needed only by MMA2, after the solve)
        mbar_arrive_expect_tx(&ms->bar_v, 2 * 8192);
        tma_load_4d(smem + kV0, &tmV, &ms->bar_v, 0, h, tok0, 0);
        tma_load_4d(smem + kV1, &tmV, &ms->bar_v, 64, h, tok0, 0);
    }
    tc_fence_after();
    const int row = (warp & 1) * 32 + lane;  // token within the chunk
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const float gcs_r = ms->gcs[row];
    const float g2_r = ms->g2[row];
    if (ok) {
        uint32_t v[64];
        tmem_ld32(tmem + lane_base + 0, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tmem_ld32(tmem + lane_base + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tmem_ld_wait();
        if (warp < 2) {
            // A row (strictly lower), fp32, to shared
            const float be = ms->beta[row];
#pragma unroll
            for (int s = 0; s < kC; s += 4) {
                float4 a;
                float* pa = &a.x;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int ss = s + u;
                    float x = be * __uint_as_float(v[ss]) * ex2f(g2_r - ms->g2[ss]);
                    if constexpr (kFused) x *= ms->rk[row] * ms->rk[ss];
                    pa[u] = ss < row ? x : 0.f;
                }
                *reinterpret_cast<float4*>(As + row * kLd + s) = a;
            }
            __syncwarp();  // this warp's 32 rows of A, which hold its whole diagonal block
            diag_block_inverse(As, warp, lane);
        } else {
            // Aqk row (lower incl. diagonal), 16-bit, straight to the workspace (row-major
            // [64][64] a chunk item; the state pass loads it by TMA after this grid completes)
            uint4* dst = reinterpret_cast<uint4*>(p.ws + p.ws_aqk + ((size_t)bhc * kC + row) * kC * 2);
#pragma unroll
            for (int s = 0; s < kC; s += 8) {
                uint4 pk;
                uint32_t* pw = &pk.x;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int s0 = s + 2 * u, s1 = s0 + 1;
                    float a0 = s0 <= row ? __uint_as_float(v[s0]) * ex2f(g2_r - ms->g2[s0]) : 0.f;
                    float a1 = s1 <= row ? __uint_as_float(v[s1]) * ex2f(g2_r - ms->g2[s1]) : 0.f;
                    if constexpr (kFused) {
                        a0 *= ms->rq[row] * ms->rk[s0];
                        a1 *= ms->rq[row] * ms->rk[s1];
                    }
                    pw[u] = Elem<T16>::pack2(a0, a1);
                }
                dst[s >> 3] = pk;
            }
        }
    }
    __syncthreads();

    {
        const int j = tid & 63;
        float sc = tid < kC ? ms->beta[j] * ex2f(ms->g2[j]) : ms->beta[j];
        if constexpr (kFused)
            if (tid < kC) sc *= ms->rk[j];  // W = T diag(beta Gam / |k|) K
        ms->colscale[tid] = sc;
    }
    // the block inverse's scratch X is the upper-right 32 x 32 block (zero in A and in T)
    offdiag_block_inverse(As, As + 32, kLd, tid);  // contains __syncthreads: every thread calls it
    {
        // AT rows 0-63 <- T diag(beta Gam), rows 64-127 <- T diag(beta). Thread = AT row: its
        // row of T (the upper-right block read as the zero it is in T) into registers, then,
        // once every thread holds its row, eight 16-byte swizzled chunks of 8 columns over the
        // same bytes (broadcast reads of the column scales)
        const int r = tid;
        const float* trow = Ts + (r & (kC - 1)) * kLd;
        const float* sc = ms->colscale + (r < kC ? 0 : kC);
        float4 tr[kC / 4];
#pragma unroll
        for (int c4 = 0; c4 < kC / 4; ++c4)
            tr[c4] = ((r & (kC - 1)) < 32 && c4 >= 8) ? make_float4(0.f, 0.f, 0.f, 0.f)
                                                      : *reinterpret_cast<const float4*>(trow + c4 * 4);
        __syncthreads();
        uint8_t* at = smem + kAT + r * 128;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
            const float4 a = tr[2 * c8];
            const float4 b = tr[2 * c8 + 1];
            const float4 sa = *reinterpret_cast<const float4*>(sc + c8 * 8);
            const float4 sb = *reinterpret_cast<const float4*>(sc + c8 * 8 + 4);
            uint4 pk;
            pk.x = Elem<T16>::pack2(a.x * sa.x, a.y * sa.y);
            pk.y = Elem<T16>::pack2(a.z * sa.z, a.w * sa.w);
            pk.z = Elem<T16>::pack2(b.x * sb.x, b.y * sb.y);
            pk.w = Elem<T16>::pack2(b.z * sb.z, b.w * sb.w);
            *reinterpret_cast<uint4*>(at + ((c8 ^ (r & 7)) << 4)) = pk;
        }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // MMA2 in two steps through the same 128 TMEM columns (M=128, N=128, K=64; B operands
    // MN-major, their two 64-column chunks 16 KiB apart, [K0|V0|K1|V1]):
    //   [T'; T''] K -> W in lanes 0-63, then [T'; T''] V -> U in lanes 64-127
    // (the other half of each product is not used).
    if (tid == 0 && ok) {
        ok = mbar_wait(&ms->bar_v, 0, abort, &g_err_gdn_prefill);
    }
    constexpr uint32_t idesc2 = make_idesc(Elem<T16>::kFmt, 128, 128, false, true);
    const uint32_t a0 = smem_u32(smem + kAT);
    if (tid == 0 && ok) {
        tc_fence_after();
        const uint32_t bk = smem_u32(smem + kK0);
#pragma unroll
        for (int kk = 0; kk < kC / 16; ++kk)
            mma_f16_ss(tmem, smem_desc(a0 + kk * 32, 16, 1024, kLayoutSW128),
                       smem_desc(bk + kk * 2048, 16384, 1024, kLayoutSW128), idesc2, kk > 0 ? 1u : 0u);
        mma_commit(&ms->bar_mma2);
    }
    // 64 rows x 128 columns of TMEM -> 16-bit, 128B-swizzled as two 64-column boxes 16 KiB
    // apart, for TMA stores: W over the K boxes (free once the W product is done; V, still
    // needed by the U product, sits in the other two), U over the V boxes afterwards
    auto stage_rows = [&](uint8_t* base) {
        uint8_t* stg = base + row * 128;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            uint32_t v[32];
            tmem_ld32(tmem + lane_base + cc * 32, v);
            tmem_ld_wait();
#pragma unroll
            for (int q8 = 0; q8 < 4; ++q8) {
                uint4 pk;
                pk.x = Elem<T16>::pack2(__uint_as_float(v[q8 * 8 + 0]), __uint_as_float(v[q8 * 8 + 1]));
                pk.y = Elem<T16>::pack2(__uint_as_float(v[q8 * 8 + 2]), __uint_as_float(v[q8 * 8 + 3]));
                pk.z = Elem<T16>::pack2(__uint_as_float(v[q8 * 8 + 4]), __uint_as_float(v[q8 * 8 + 5]));
                pk.w = Elem<T16>::pack2(__uint_as_float(v[q8 * 8 + 6]), __uint_as_float(v[q8 * 8 + 7]));
                const int q = cc * 4 + q8;  // 16-byte chunk 0..15 of the 256-byte row
                *reinterpret_cast<uint4*>(stg + (q >> 3) * 16384 + (((q & 7) ^ (row & 7)) << 4)) = pk;
            }
        }
        fence_proxy_async_smem();
    };
    ok = __all_sync(0xffffffffu, mbar_wait(&ms->bar_mma2, 0, abort, &g_err_gdn_prefill)) && ok;
    tc_fence_after();
    if (ok && warp < 2) {
        stage_rows(smem + kK0);  // W -> [K0 | . | K1 | .]
        reinterpret_cast<float*>(p.ws + p.ws_gcs)[bhc * kC + row] = gcs_r;
        if constexpr (kFused) {
            reinterpret_cast<float*>(p.ws + p.ws_rk)[bhc * kC + row] = ms->rk[row];
            reinterpret_cast<float*>(p.ws + p.ws_rq)[bhc * kC + row] = ms->rq[row];
        }
    }
    tc_fence_before();
    __syncthreads();  // W is out of TMEM
    if (tid == 0 && ok) {
        tc_fence_after();
        const uint32_t bv = smem_u32(smem + kV0);
#pragma unroll
        for (int kk = 0; kk < kC / 16; ++kk)
            mma_f16_ss(tmem, smem_desc(a0 + kk * 32, 16, 1024, kLayoutSW128),
                       smem_desc(bv + kk * 2048, 16384, 1024, kLayoutSW128), idesc2, kk > 0 ? 1u : 0u);
        mma_commit(&ms->bar_mma2);
    }
    ok = __all_sync(0xffffffffu, mbar_wait(&ms->bar_mma2, 1, abort, &g_err_gdn_prefill)) && ok;
    tc_fence_after();
    if (tid == 0 && ok && c > 0) {
        // the W and U products have read AT: the previous chunk's K goes over it, for M below
        // (in flight while warps 2-3 stage U)
        mbar_arrive_expect_tx(&ms->bar_kp, 2 * 8192);
        tma_load_4d(smem + kAs, &tmK, &ms->bar_kp, 0, hq, tok0 - kC, 0);
        tma_load_4d(smem + kAs + 8192, &tmK, &ms->bar_kp, 64, hq, tok0 - kC, 0);
    }
    if (ok && warp >= 2) stage_rows(smem + kV0);  // U -> [. | V0 | . | V1]
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && ok) {
        tma_store_3d(&tmW, smem + kK0, 0, 0, (int)bhc);
        tma_store_3d(&tmW, smem + kK1, 64, 0, (int)bhc);
        tma_store_3d(&tmU, smem + kV0, 0, 0, (int)bhc);
        tma_store_3d(&tmU, smem + kV1, 64, 0, (int)bhc);
        bulk_commit();
        // M = W K_prev^T (M=128, N=64, K=128): A = the staged W (K-major, its two
        // 64-column boxes 16 KiB apart; rows 64-127 of the product are not used),
        // B = K of the previous chunk.  Result in TMEM cols 0-63, lanes 0-63.
        if (c > 0) {
            ok = mbar_wait(&ms->bar_kp, 0, abort, &g_err_gdn_prefill);
            if (ok) {
                tc_fence_after();
                constexpr uint32_t idesc = make_idesc(Elem<T16>::kFmt, 128, 64, false, false);
                const uint64_t dw = smem_desc(smem_u32(smem + kK0), 16, 1024, kLayoutSW128);
                const uint64_t dk = smem_desc(smem_u32(smem + kAs), 16, 1024, kLayoutSW128);
#pragma unroll
                for (int kk = 0; kk < kD / 16; ++kk) {
                    const uint32_t offw = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
                    const uint32_t offk = ((kk >> 2) * 8192 + (kk & 3) * 32) >> 4;
                    mma_f16_ss(tmem, dw + offw, dk + offk, idesc, kk > 0 ? 1u : 0u);
                }
                mma_commit(&ms->bar_m);
            }
        }
    }
    // M[t][s] = (W K_prev^T)[t][s] e^{gprev_last - gprev_s}: the previous chunk's
    // decayed keys as seen through this chunk's W.  Staged over AT (free since
    // MMA2), stored next to Aqk.  Chunk 0 of a sequence stores zeros.
    if constexpr (kFused) {
        // 1/|k_s| of the previous chunk's keys, from its tile
        if (c > 0) {
            ok = __all_sync(0xffffffffu, mbar_wait(&ms->bar_kp, 0, abort, &g_err_gdn_prefill)) && ok;
            if (tid < kC) ms->rkp[tid] = row_rnorm<T16>(smem + kAs, smem + kAs + 8192, tid);
        }
        __syncthreads();
    }
    if (c > 0)
        ok = __all_sync(0xffffffffu, mbar_wait(&ms->bar_m, 0, abort, &g_err_gdn_prefill)) && ok;
    tc_fence_after();
    if (warp < 2) {
        uint32_t v[64];
        if (c > 0 && ok) {
            tmem_ld32(tmem + lane_base + 0, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
            tmem_ld32(tmem + lane_base + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
            tmem_ld_wait();
        }
        uint8_t* stg = smem + kAT + row * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            uint4 pk = make_uint4(0, 0, 0, 0);
            if (c > 0 && ok) {
                uint32_t* pw = &pk.x;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int s0 = q * 8 + 2 * u;
                    float m0 = __uint_as_float(v[s0]) * ms->mdecay[s0];
                    float m1 = __uint_as_float(v[s0 + 1]) * ms->mdecay[s0 + 1];
                    if constexpr (kFused) {
                        m0 *= ms->rkp[s0];
                        m1 *= ms->rkp[s0 + 1];
                    }
                    pw[u] = Elem<T16>::pack2(m0, m1);
                }
            }
            *reinterpret_cast<uint4*>(stg + ((q ^ (row & 7)) << 4)) = pk;
        }
        fence_proxy_async_smem();
    }
    __syncthreads();
    if (tid == 0 && ok) {
        tma_store_3d(&tmM, smem + kAT, 0, 0, (int)bhc);
        bulk_commit();
        // shared memory must outlive only the stores' reads of it: their writes are complete
        // when the grid is, which the state pass waits for (griddepcontrol.wait)
        bulk_wait_read();
    }
    if (tid == 0) {
        mma_commit(&ms->drain);
        mbar_wait(&ms->drain, 0, abort, &g_err_gdn_prefill);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ===========================================================================
// Kernel 2: sequential state pass
// ===========================================================================
// The chain runs on Vn, not on S.  With R_{c+1} = W_{c+1} S_c^T and
// M_{c+1} = W_{c+1} K_c^T diag(e^{gcs_last,c - gcs_c}) (from kernel 1),
//   Vn_{c+1} = U_{c+1} - W_{c+1} S_{c+1}^T = U_{c+1} - e^{gcs_last,c} R_{c+1} - M_{c+1} Vn_c,
// so the only MMA between Vn_c and Vn_{c+1} is the 64-deep M_{c+1} Vn_c; the 128-deep
// products with S (R_{c+1} and Q_c S_c^T) run a chunk ahead, off the chain.
namespace st {
// warps 0-3 state (thread = key row of the slice), 4-5 outputs (TMEM lanes 0-63),
// 6-7 Vn (lanes 64-127), 8 TMA producer, 9 chain MMAs, 10 state MMAs
constexpr int kThreads = 352;
constexpr int kWarpOut = 4, kWarpVn = 6, kWarpProducer = 8, kWarpMmaA = 9, kWarpMmaB = 10;
// one stage of chunk c (69 KiB):
//   A1  [Q_c b0 | W_{c+1} b0 | Q_c b1 | W_{c+1} b1]  32 KiB: A of [Q_c; W_{c+1}] S_c^T
//   Kt  [K_c b0 | K_c b1]                              16 KiB: A of K_c^T Vt_c (MN-major)
//   AM  [Aqk_c | M_{c+1}]                              16 KiB: A of [Aqk_c; M_{c+1}] Vn_c
//   U   this CTA's 32 columns of U_c (64-byte swizzle)  4 KiB;  G  gcs_c  256 B
// (b0/b1: 64-column boxes).  Three stages; the prologue's W_0 borrows stage 2's A1.
constexpr int kStage = 70656;
constexpr int kA1 = 0, kKt = 32768, kAM = 49152, kU = 65536, kG = 69632;
constexpr int kStageTx = 8 * 8192 + 4096 + kC * 4;
constexpr int kStages = 3;
// B operands, MN-major with 64-byte swizzle: one 64-byte row (32 state columns,
// 16-bit) per K index, so each thread writes its row as four 16-byte chunks
constexpr int kSt = kStages * kStage;    // S^T tile: 128 keys x 32 v, 8 KiB
constexpr int kVn = kSt + 8192;          // Vn tile: 64 tokens x 32 v, 4 KiB
constexpr int kVt = kVn + 4096;          // decayed Vn tile, 4 KiB
constexpr int kMisc = kVt + 4096;
constexpr int kBytes = kMisc + 256;
constexpr int kAlloc = kBytes + 1024;
static_assert(kAlloc <= 232448, "state kernel shared memory above the 227 KiB per-CTA limit");
constexpr uint32_t kTmemCols = 256;
// TMEM, two buffers each by chunk parity (32 columns a buffer):
//   X1 = [Aqk_c; M_{c+1}] Vn_c   lanes 0-63 intra-chunk output, 64-127 chain term
//   DS = K_c^T Vt_c              lane = key: the state increment
//   RQ = [Q_c; W_{c+1}] S_c^T    lanes 0-63 Q S^T, 64-127 R_{c+1}
constexpr uint32_t kColX1 = 0, kColDS = 64, kColRQ = 128;

struct Misc {
    uint64_t full[kStages], empty[kStages];
    uint64_t pro_full, pro_done;
    uint64_t s_ready[2];
    uint64_t vn_ready;  // Vn_c written: the chain product X1(c) may run
    uint64_t vt_ready;  // decayed Vn_c written: the state increment DS(c) may run
    uint64_t x1_full[2], ds_full[2], rq_full[2];
    uint64_t o_done[2];  // the output warps have read X1 / RQ buffer (c & 1) of chunk c
    uint64_t drain_a, drain_b;
    uint32_t tmem_base;
    int abort;
};
static_assert(sizeof(Misc) <= kBytes - kMisc, "state Misc overflows its slot");

// rq_full[c & 1] completes for the prologue product (counted as c = -1, buffer 1)
// and then for c = 0, 1, 2, ...: the parity of the completion that belongs to c
__device__ __forceinline__ uint32_t rq_parity(int c) {
    return c < 0 ? 0u : (uint32_t)(((c & 1) ? (c + 1) >> 1 : c >> 1) & 1);
}
}  // namespace st

// byte offset of 16-byte chunk q (columns 8q..8q+7) of row r in a 64-byte-swizzled tile
__device__ __forceinline__ uint32_t sw64_chunk(int r, int q) {
    return (uint32_t)(r * 64 + ((q ^ ((r >> 1) & 3)) << 4));
}

struct StateParams {
    const uint8_t* ws;
    float* state;
    void* o;
    size_t ws_gcs, ws_rq, ws_rk;
    const int* cu;  // as PrepParams
    int T, Hqk, Hv, nch, head_map;
    int ntok;
    float scale;
    // Segmented chain (nseg > 1, dense sequences only): segment g covers chunks
    // [g seg_len, (g + 1) seg_len).  Segment 0 runs from the caller's state as usual; later
    // segments run from a zero state and carry 128 more state columns (slices 4-7) that start
    // as the identity with zero values, so that their end state is the segment's transition
    // product P_g and their outputs are R = (the output map) P.  End states go to seg_x
    // ([B][Hv][nseg][256 v][128 k], segment 0's real columns its true end state); outputs of
    // segments g >= 1 go to seg_o (zero-state outputs, fp32 [tokens][Hv][128]) and seg_r (R,
    // bf16 [tokens][Hv][128], an MMA operand).  gdn_seg_link_kernel and gdn_seg_fix_kernel
    // then chain the segment starts and add R S_start.
    int seg_len, nseg;
    float* seg_x;
    float* seg_o;
    __nv_bfloat16* seg_r;
};

// 32 consecutive outputs of one thread as 16-byte vector stores
template <typename TOut>
__device__ __forceinline__ void store_row32(TOut* dst, const float (&v)[32]) {
    if constexpr (sizeof(TOut) == 4) {
#pragma unroll
        for (int q = 0; q < 8; ++q)
            reinterpret_cast<float4*>(dst)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint4 pk;
            pk.x = Elem<TOut>::pack2(v[8 * q + 0], v[8 * q + 1]);
            pk.y = Elem<TOut>::pack2(v[8 * q + 2], v[8 * q + 3]);
            pk.z = Elem<TOut>::pack2(v[8 * q + 4], v[8 * q + 5]);
            pk.w = Elem<TOut>::pack2(v[8 * q + 6], v[8 * q + 7]);
            reinterpret_cast<uint4*>(dst)[q] = pk;
        }
    }
}

// kSeg: the segmented chain (StateParams); the plain instantiation compiles without any of it
template <typename T16, typename TOut, bool kFused, bool kSeg>
__global__ void __launch_bounds__(st::kThreads, 1)
    gdn_state_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmAqk,
                     const __grid_constant__ CUtensorMap tmM, const __grid_constant__ CUtensorMap tmU,
                     const StateParams p) {
    using namespace st;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Misc* ms = reinterpret_cast<Misc*>(smem + kMisc);
    volatile int* abort = &ms->abort;

    const int slice = blockIdx.x;
    const int h = blockIdx.y;
    const int b = kSeg ? (int)blockIdx.z / p.nseg : (int)blockIdx.z;
    const int g = kSeg ? (int)blockIdx.z % p.nseg : 0;  // segment
    const bool aug = kSeg && slice >= kD / kSlice;      // transition columns of a later segment
    if (aug && g == 0) return;
    const SeqSpan seq = seq_span(p.cu, p.T, b);
    if (!seq_ok(seq, p.T, p.ntok)) return;    // recorded by the prep grid; state left as it is
    const int cs = kSeg ? g * p.seg_len : 0;  // the segment's first chunk
    // this segment's chunks (the sequence's chunks, p.nch for the longest, when plain)
    const int nch = kSeg ? min(p.seg_len, (seq.len + kC - 1) / kC - cs) : (seq.len + kC - 1) / kC;
    if (nch <= 0) return;                     // an empty sequence: its state stays as it is
    // segmented: the link kernel, launched as a programmatic dependent, may be scheduled now
    // (it waits for this grid to complete before reading the end states)
    if constexpr (kSeg) allow_dependent_launch();
    const int tok0 = seq.start + cs * kC;     // the segment's first token
    const int seq_left = seq.len - cs * kC;   // tokens of the sequence from there on
    const int c0 = slice * kSlice;
    const int hq = qk_head(h, p.Hqk, p.Hv, p.head_map);
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const size_t bh = (size_t)b * p.Hv + h;  // workspace slots: p.nch chunks a (sequence, head)
    const size_t bhcs = bh * p.nch + cs;     // the segment's first chunk slot

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&ms->full[i], 1);
            mbar_init(&ms->empty[i], 2);  // one commit from each MMA thread
        }
        mbar_init(&ms->pro_full, 1);
        mbar_init(&ms->pro_done, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&ms->s_ready[i], 4);  // one arrival per state warp
            mbar_init(&ms->x1_full[i], 1);
            mbar_init(&ms->ds_full[i], 1);
            mbar_init(&ms->rq_full[i], 1);
            mbar_init(&ms->o_done[i], 2);   // one per output warp
        }
        mbar_init(&ms->vn_ready, 2);        // one per Vn warp
        mbar_init(&ms->vt_ready, 2);
        mbar_init(&ms->drain_a, 1);
        mbar_init(&ms->drain_b, 1);
        ms->abort = 0;
        fence_barrier_init();
    }
    if (warp == kWarpMmaA) {
        tmem_alloc(&ms->tmem_base, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ms->tmem_base;
    constexpr uint32_t kFmt = Elem<T16>::kFmt;

    if (warp == kWarpProducer) {
        if (lane == 0) {
            const float* gcs_all = reinterpret_cast<const float*>(p.ws + p.ws_gcs);
            const int bhc0 = (int)bhcs;
            grid_dependency_wait();  // W, U, Aqk, M, gcs come from the prep grid
            // prologue: W_0 into the W rows of stage 2's A1 tile
            uint8_t* pro = smem + (kStages - 1) * kStage + kA1;
            mbar_arrive_expect_tx(&ms->pro_full, 2 * 8192);
            tma_load_3d(pro + 8192, &tmW, &ms->pro_full, 0, 0, bhc0);
            tma_load_3d(pro + 24576, &tmW, &ms->pro_full, 64, 0, bhc0);
            int issued = 0;
            for (int c = 0; c < nch; ++c) {
                const int s = c % kStages;
                if (!mbar_wait(&ms->empty[s], ((c / kStages) & 1) ^ 1, abort, &g_err_gdn_prefill)) break;
                if (c == kStages - 1 && !mbar_wait(&ms->pro_done, 0, abort, &g_err_gdn_prefill)) break;
                uint8_t* stg = smem + s * kStage;
                uint64_t* bar = &ms->full[s];
                const int bhc = bhc0 + c;
                // W_{c+1}, M_{c+1} of the last chunk read the next sequence's first chunk (or
                // zero fill past the end): those rows of the products are not used
                // (transition columns have zero values: no U tile)
                mbar_arrive_expect_tx(bar, aug ? kStageTx - 4096 : kStageTx);
                tma_load_4d(stg + kA1 + 0, &tmQ, bar, 0, hq, tok0 + c * kC, 0);
                tma_load_3d(stg + kA1 + 8192, &tmW, bar, 0, 0, bhc + 1);
                tma_load_4d(stg + kA1 + 16384, &tmQ, bar, 64, hq, tok0 + c * kC, 0);
                tma_load_3d(stg + kA1 + 24576, &tmW, bar, 64, 0, bhc + 1);
                tma_load_4d(stg + kKt, &tmK, bar, 0, hq, tok0 + c * kC, 0);
                tma_load_4d(stg + kKt + 8192, &tmK, bar, 64, hq, tok0 + c * kC, 0);
                tma_load_3d(stg + kAM, &tmAqk, bar, 0, 0, bhc);
                tma_load_3d(stg + kAM + 8192, &tmM, bar, 0, 0, bhc + 1);
                if (!aug) tma_load_3d(stg + kU, &tmU, bar, c0, 0, bhc);
                bulk_load_1d(stg + kG, gcs_all + (size_t)bhc * kC, kC * 4, bar);
                issued = c + 1;
            }
            mbar_wait(&ms->pro_full, 0, abort, &g_err_gdn_prefill);
            for (int c = max(0, issued - kStages); c < issued; ++c)
                mbar_wait(&ms->full[c % kStages], (c / kStages) & 1, abort, &g_err_gdn_prefill);
        }
    } else if (warp == kWarpMmaA) {
        // chain MMAs: X1 = [Aqk_c; M_{c+1}] Vn_c, then DS = K_c^T Vt_c
        if (lane == 0) {
            constexpr uint32_t id_kb = make_idesc(kFmt, 128, kSlice, false, true);  // A K-major, B MN
            constexpr uint32_t id_mn = make_idesc(kFmt, 128, kSlice, true, true);   // both MN-major
            const uint64_t dAM = smem_desc(smem_u32(smem + kAM), 16, 1024, kLayoutSW128);
            const uint64_t dK = smem_desc(smem_u32(smem + kKt), 8192, 1024, kLayoutSW128);
            const uint64_t dVn = smem_desc(smem_u32(smem + kVn), 4096, 512, kLayoutSW64);
            const uint64_t dVt = smem_desc(smem_u32(smem + kVt), 4096, 512, kLayoutSW64);
            for (int c = 0; c < nch; ++c) {
                const int s = c % kStages;
                const uint32_t so = (s * kStage) >> 4;
                const uint32_t buf = (c & 1) * 32;
                // Vn_c is the chain dependency, so it is waited for last: every wait between
                // it and the MMAs would lengthen the chain
                if (!mbar_wait(&ms->full[s], (c / kStages) & 1, abort, &g_err_gdn_prefill)) break;
                if (c >= 2 && !mbar_wait(&ms->o_done[c & 1], ((c - 2) >> 1) & 1, abort, &g_err_gdn_prefill)) break;
                if (!mbar_wait(&ms->vn_ready, c & 1, abort, &g_err_gdn_prefill)) break;
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < kC / 16; ++kk)
                    mma_f16_ss(tmem + kColX1 + buf, dAM + so + ((kk * 32) >> 4), dVn + ((kk * 1024) >> 4), id_kb,
                               kk > 0 ? 1u : 0u);
                mma_commit(&ms->x1_full[c & 1]);
                if (!mbar_wait(&ms->vt_ready, c & 1, abort, &g_err_gdn_prefill)) break;
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < kC / 16; ++kk)
                    mma_f16_ss(tmem + kColDS + buf, dK + so + ((kk * 2048) >> 4), dVt + ((kk * 1024) >> 4), id_mn,
                               kk > 0 ? 1u : 0u);
                mma_commit(&ms->ds_full[c & 1]);
                mma_commit(&ms->empty[s]);
            }
            mma_commit(&ms->drain_a);
            mbar_wait(&ms->drain_a, 0, abort, &g_err_gdn_prefill);
        }
    } else if (warp == kWarpMmaB) {
        // state MMAs: RQ = [Q_c; W_{c+1}] S_c^T, one chunk ahead of the chain
        if (lane == 0) {
            constexpr uint32_t id_kb = make_idesc(kFmt, 128, kSlice, false, true);
            const uint64_t dA1 = smem_desc(smem_u32(smem + kA1), 16, 1024, kLayoutSW128);
            const uint64_t dS = smem_desc(smem_u32(smem + kSt), 8192, 512, kLayoutSW64);
            auto rq = [&](uint32_t so, uint32_t buf) {
#pragma unroll
                for (int kk = 0; kk < kD / 16; ++kk) {
                    const uint32_t ao = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
                    mma_f16_ss(tmem + kColRQ + buf, dA1 + so + ao, dS + ((kk * 1024) >> 4), id_kb,
                               kk > 0 ? 1u : 0u);
                }
            };
            // prologue: R_0 = W_0 S_0^T (rows 64-127; rows 0-63 read stage 2's unused Q slot)
            bool ok = mbar_wait(&ms->pro_full, 0, abort, &g_err_gdn_prefill) &&
                      mbar_wait(&ms->s_ready[0], 0, abort, &g_err_gdn_prefill);
            if (ok) {
                tc_fence_after();
                rq(((kStages - 1) * kStage) >> 4, 32);
                mma_commit(&ms->rq_full[1]);
                mma_commit(&ms->pro_done);
            }
            for (int c = 0; ok && c < nch; ++c) {
                const int s = c % kStages;
                if (!mbar_wait(&ms->full[s], (c / kStages) & 1, abort, &g_err_gdn_prefill)) break;
                if (c > 0 && !mbar_wait(&ms->s_ready[c & 1], (c >> 1) & 1, abort, &g_err_gdn_prefill)) break;
                if (c >= 2 && !mbar_wait(&ms->o_done[c & 1], ((c - 2) >> 1) & 1, abort, &g_err_gdn_prefill)) break;
                tc_fence_after();
                rq((s * kStage) >> 4, (c & 1) * 32);
                mma_commit(&ms->rq_full[c & 1]);
                mma_commit(&ms->empty[s]);
            }
            mma_commit(&ms->drain_b);
            mbar_wait(&ms->drain_b, 0, abort, &g_err_gdn_prefill);
        }
    } else {
        // ---------------- compute warps: three roles, each on its own chain -------
        const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const float* gcs_all = reinterpret_cast<const float*>(p.ws + p.ws_gcs);
        const size_t bhc0 = bhcs;
        if (warp >= kWarpOut) grid_dependency_wait();  // gcs comes from the prep grid
        auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
            return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, &g_err_gdn_prefill));
        };
        // 32 values -> one 64-byte row of an MN-major B tile (16-bit)
        auto put_row = [&](uint8_t* tile, int r, const float* x) {
#pragma unroll
            for (int q = 0; q < kSlice / 8; ++q) {
                uint4 pk;
                pk.x = Elem<T16>::pack2(x[8 * q + 0], x[8 * q + 1]);
                pk.y = Elem<T16>::pack2(x[8 * q + 2], x[8 * q + 3]);
                pk.z = Elem<T16>::pack2(x[8 * q + 4], x[8 * q + 5]);
                pk.w = Elem<T16>::pack2(x[8 * q + 6], x[8 * q + 7]);
                *reinterpret_cast<uint4*>(tile + sw64_chunk(r, q)) = pk;
            }
        };
        if (warp < kWarpOut) {
            // ---- state: S_{c+1} = e^{gcs_last} S_c + K_c^T Vt_c, thread i = key i ----
            const int i = tid;
            float S[kSlice];
            float* Sg = p.state + (bh * kD + c0) * kD + i;
            if (g == 0) {
#pragma unroll
                for (int cc = 0; cc < kSlice; ++cc) S[cc] = Sg[(size_t)cc * kD];
            } else {  // a later segment: zero state, the transition columns the identity
#pragma unroll
                for (int cc = 0; cc < kSlice; ++cc) S[cc] = (aug && i == c0 - kD + cc) ? 1.f : 0.f;
            }
            grid_dependency_wait();  // (the state itself is an input, not a prep result)
            uint8_t* sS = smem + kSt;
            // S (16-bit) -> shared (B operand of the RQ product), then S_c is announced
            auto publish_S = [&](int c) {
                put_row(sS, i, S);
                fence_proxy_async_smem();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&ms->s_ready[c & 1]);
            };
            bool ok = true;
            publish_S(0);
            float glast_nx = gcs_all[bhc0 * kC + kC - 1];
            for (int c = 0; c < nch; ++c) {
                const float gam = __expf(glast_nx);
                if (c + 1 < nch) glast_nx = gcs_all[(bhc0 + c + 1) * kC + kC - 1];
                if (!wait_all(&ms->ds_full[c & 1], (c >> 1) & 1)) { ok = false; break; }
                tc_fence_after();
                uint32_t ds[32];
                tmem_ld32(tmem + lane_base + kColDS + (c & 1) * 32, ds);
                tmem_ld_wait();
#pragma unroll
                for (int cc = 0; cc < kSlice; ++cc) S[cc] = fmaf(gam, S[cc], __uint_as_float(ds[cc]));
                if (c + 1 < nch) {
                    // the S tile is rewritten only once the RQ product that reads S_c is done
                    if (!wait_all(&ms->rq_full[c & 1], st::rq_parity(c))) { ok = false; break; }
                    tc_fence_after();
                    publish_S(c + 1);
                }
            }
            if (ok && !kSeg) {
#pragma unroll
                for (int cc = 0; cc < kSlice; ++cc) Sg[(size_t)cc * kD] = S[cc];
            } else if (ok) {
                float* X = p.seg_x + ((bh * p.nseg + g) * 2 * kD + c0) * kD + i;
#pragma unroll
                for (int cc = 0; cc < kSlice; ++cc) X[(size_t)cc * kD] = S[cc];
            }
        } else if (warp < kWarpVn) {
            // ---- outputs: o_c = scale (e^{gcs} Q_c S_c^T + Aqk_c Vn_c), token row ----
            const int row = tid - kWarpOut * 32;  // 0..63 = TMEM lane
            const float* rq_all = reinterpret_cast<const float*>(p.ws + p.ws_rq);
            float gcs_nx = gcs_all[bhc0 * kC + row];
            float rq_nx = kFused ? rq_all[bhc0 * kC + row] : 1.f;
            for (int c = 0; c < nch; ++c) {
                const float gcs_t = gcs_nx;
                const float rq_t = rq_nx;  // 1/|q_t| (fused pre-processing)
                if (c + 1 < nch) {
                    gcs_nx = gcs_all[(bhc0 + c + 1) * kC + row];
                    if constexpr (kFused) rq_nx = rq_all[(bhc0 + c + 1) * kC + row];
                }
                if (!wait_all(&ms->rq_full[c & 1], st::rq_parity(c))) break;
                if (!wait_all(&ms->x1_full[c & 1], (c >> 1) & 1)) break;
                tc_fence_after();
                uint32_t pq[32], oi[32];
                tmem_ld32(tmem + lane_base + kColRQ + (c & 1) * 32, pq);
                tmem_ld32(tmem + lane_base + kColX1 + (c & 1) * 32, oi);
                tmem_ld_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&ms->o_done[c & 1]);
                const int tt = c * kC + row;  // token from the segment's start
                if (tt < seq_left) {
                    const float eg = __expf(gcs_t) * rq_t;
                    float ov[kSlice];
#pragma unroll
                    for (int cc = 0; cc < kSlice; ++cc)
                        ov[cc] = p.scale * fmaf(eg, __uint_as_float(pq[cc]), __uint_as_float(oi[cc]));
                    const size_t orow = ((size_t)tok0 + tt) * p.Hv + h;
                    if (g == 0)
                        store_row32(static_cast<TOut*>(p.o) + orow * kD + c0, ov);
                    else if (!aug)
                        store_row32(p.seg_o + orow * kD + c0, ov);
                    else
                        store_row32(p.seg_r + orow * kD + (c0 - kD), ov);
                }
            }
        } else {
            // ---- Vn_c = U_c - e^{gcs_last,c-1} R_c - M_c Vn_{c-1}   (c = 0: U_0 - W_0 S_0^T)
            const int row = tid - kWarpVn * 32;  // token; TMEM lane 64 + row
            uint8_t* sVn = smem + kVn;
            uint8_t* sVt = smem + kVt;
            const float* rk_all = reinterpret_cast<const float*>(p.ws + p.ws_rk);
            float rk_nx = kFused ? rk_all[bhc0 * kC + row] : 1.f;
            float gam_prev = 1.f;
            for (int c = 0; c < nch; ++c) {
                const float rk_t = rk_nx;  // 1/|k_t|: K^T diag(1/|k|) Vt is the normalised keys' product
                if (kFused && c + 1 < nch) rk_nx = rk_all[(bhc0 + c + 1) * kC + row];
                const int s = c % kStages;
                // chunk c's U row and gates from its stage (released only after vt_ready(c))
                if (!wait_all(&ms->full[s], (c / kStages) & 1)) break;
                const uint8_t* stg = smem + s * kStage;
                const float gcs_t = reinterpret_cast<const float*>(stg + kG)[row];
                const float g_last = reinterpret_cast<const float*>(stg + kG)[kC - 1];
                float u[kSlice];
#pragma unroll
                for (int q8 = 0; q8 < kSlice / 8; ++q8) {
                    uint4 raw = make_uint4(0u, 0u, 0u, 0u);  // transition columns: zero values
                    if (!aug) raw = *reinterpret_cast<const uint4*>(stg + kU + sw64_chunk(row, q8));
                    const T16* e = reinterpret_cast<const T16*>(&raw);
#pragma unroll
                    for (int u8 = 0; u8 < 8; ++u8) u[q8 * 8 + u8] = Elem<T16>::to_f(e[u8]);
                }
                if (!wait_all(&ms->rq_full[(c - 1) & 1], st::rq_parity(c - 1))) break;
                if (c > 0 && !wait_all(&ms->x1_full[(c - 1) & 1], ((c - 1) >> 1) & 1)) break;
                tc_fence_after();
                uint32_t rr[32], xx[32];
                tmem_ld32(tmem + lane_base + kColRQ + ((c - 1) & 1) * 32, rr);
                if (c > 0) tmem_ld32(tmem + lane_base + kColX1 + ((c - 1) & 1) * 32, xx);
                tmem_ld_wait();
                const float dec = __expf(g_last - gcs_t) * rk_t;
                float vt[kSlice];
#pragma unroll
                for (int cc = 0; cc < kSlice; ++cc) {
                    float vn = fmaf(-gam_prev, __uint_as_float(rr[cc]), u[cc]);
                    if (c > 0) vn -= __uint_as_float(xx[cc]);
                    u[cc] = vn;
                    vt[cc] = vn * dec;
                }
                // Vn_c first (its tile was read by X1(c-1), whose result is in hand), so the
                // chain product X1(c) can start; then decayed Vn_c, once K^T Vt of chunk c-1
                // has read the Vt tile
                put_row(sVn, row, u);
                fence_proxy_async_smem();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&ms->vn_ready);
                if (c > 0 && !wait_all(&ms->ds_full[(c - 1) & 1], ((c - 1) >> 1) & 1)) break;
                put_row(sVt, row, vt);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&ms->vt_ready);
                gam_prev = __expf(g_last);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kWarpMmaA) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ===========================================================================
// Segmented chain: linking the segments and correcting their outputs
// ===========================================================================
// Every state column evolves on its own and linearly in (its values, its initial column), so
// a segment run from a zero state has the true end state S_zero_g + P_g S_start(g) and the
// true outputs O_zero + R S_start(g), with P_g and R from the identity-started columns.

// 16-byte asynchronous copies global -> shared (no register staging); a thread's copies
// are complete after cp_wait<n> leaves at most n of its newest groups in flight.
__device__ __forceinline__ void cp16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// S_start(1) = segment 0's end state; S_start(g + 1) = S_zero_g + P_g S_start(g).  One CTA
// per (8 state columns j, v-head, sequence) of 256 threads: key row k = tid % 128, and the
// two halves of the threads take the product's inner index kp in [0, 64) and [64, 128),
// their sums added through shared memory; packed f32x2 FMAs.  The starts of segments
// 1 .. nseg-1 go to sst ([B][Hv][nseg][k][j], bf16: the correction's MMA operand), the last
// segment's end state to the caller's state ([v][k] as everywhere else).  P_g (64 KiB, the
// transition columns' end states, contiguous in seg_x) and the CTA's 8 rows of S_zero_g (4 KiB)
// are double-buffered in shared memory: step g+1's operands stream in while step g runs, so no
// step waits on a global load.
namespace seglink {
constexpr int kThreads = 2 * kD;
constexpr int kZero = 2 * kD * kD;              // float offset of the S_zero rows, 2 x [8][kD]
constexpr int kCur = kZero + 2 * 8 * kD;        // S_start(g) [kD][8]
constexpr int kPart = kCur + kD * 8;            // second half's sums [kD][8]
constexpr int kSmem = (kPart + kD * 8) * 4;
static_assert(kThreads * 4 == 8 * kD, "one 16-byte copy a thread moves the 8 S_zero rows");
}  // namespace seglink
__global__ void __launch_bounds__(seglink::kThreads) gdn_seg_link_kernel(const float* __restrict__ seg_x,
                                                                         __nv_bfloat16* __restrict__ sst,
                                                                         float* __restrict__ state, int Hv,
                                                                         int nseg) {
    extern __shared__ __align__(16) float lsm[];
    float (*cur)[8] = reinterpret_cast<float (*)[8]>(lsm + seglink::kCur);    // S_start(g)[k'][j0 ..]
    float (*part)[8] = reinterpret_cast<float (*)[8]>(lsm + seglink::kPart);  // second half's sums
    grid_dependency_wait();    // the state pass's end states (a programmatic dependent launch)
    allow_dependent_launch();  // the correction kernel waits for this grid in turn
    const int j0 = blockIdx.x * 8, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, k = tid & (kD - 1), half = tid >> 7;
    const size_t bh = (size_t)b * Hv + h;
    auto fetch = [&](int g, int buf) {  // P_g^T (row kp = column kp's end state), S_zero_g rows j0 ..
        const float4* src = reinterpret_cast<const float4*>(seg_x + ((bh * nseg + g) * 2 + 1) * kD * kD);
        float4* dst = reinterpret_cast<float4*>(lsm + buf * kD * kD);
#pragma unroll
        for (int m = 0; m < kD * kD / 4 / seglink::kThreads; ++m)
            cp16(dst + m * seglink::kThreads + tid, src + m * seglink::kThreads + tid);
        const int zr = tid >> 5, zc = 4 * (tid & 31);  // row j0 + zr, keys zc .. zc + 3
        cp16(lsm + seglink::kZero + buf * 8 * kD + zr * kD + zc,
             seg_x + (bh * nseg + g) * 2 * kD * kD + (size_t)(j0 + zr) * kD + zc);
        cp_commit();
    };
    fetch(1, 0);
    const float* X0 = seg_x + bh * nseg * 2 * kD * kD;  // X^T rows v, columns k
    float sv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) sv[u] = X0[(size_t)(j0 + u) * kD + k];
    for (int g = 1; g < nseg; ++g) {
        const int buf = (g - 1) & 1;
        if (g + 1 < nseg) fetch(g + 1, buf ^ 1);
        else cp_commit();  // an empty group keeps the count: step g's group is then the second newest
        if (half == 0) {
#pragma unroll
            for (int u = 0; u < 8; ++u) cur[k][u] = sv[u];
            uint4 pk;
            pk.x = Elem<__nv_bfloat16>::pack2(sv[0], sv[1]);
            pk.y = Elem<__nv_bfloat16>::pack2(sv[2], sv[3]);
            pk.z = Elem<__nv_bfloat16>::pack2(sv[4], sv[5]);
            pk.w = Elem<__nv_bfloat16>::pack2(sv[6], sv[7]);
            *reinterpret_cast<uint4*>(sst + ((bh * nseg + g) * kD + k) * kD + j0) = pk;
        }
        cp_wait<1>();
        __syncthreads();  // every thread's copies of P_g, S_zero_g and the rows of cur are visible
        float2 acc[4];
        const float* Z = lsm + seglink::kZero + buf * 8 * kD;
#pragma unroll
        for (int u = 0; u < 4; ++u)  // S_zero_g[k][j] seeds the first half's sums
            acc[u] = half == 0 ? make_float2(Z[(2 * u) * kD + k], Z[(2 * u + 1) * kD + k]) : make_float2(0.f, 0.f);
        const float* sP = lsm + buf * kD * kD;
        const int kp0 = half * (kD / 2);
#pragma unroll 8
        for (int kp = kp0; kp < kp0 + kD / 2; ++kp) {
            const float pk = sP[kp * kD + k];  // P_g[k][kp]
            const float2 p2 = make_float2(pk, pk);
            const float4 c0 = *reinterpret_cast<const float4*>(&cur[kp][0]);
            const float4 c1 = *reinterpret_cast<const float4*>(&cur[kp][4]);
            acc[0] = __ffma2_rn(p2, make_float2(c0.x, c0.y), acc[0]);
            acc[1] = __ffma2_rn(p2, make_float2(c0.z, c0.w), acc[1]);
            acc[2] = __ffma2_rn(p2, make_float2(c1.x, c1.y), acc[2]);
            acc[3] = __ffma2_rn(p2, make_float2(c1.z, c1.w), acc[3]);
        }
        if (half == 1) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                part[k][2 * u] = acc[u].x;
                part[k][2 * u + 1] = acc[u].y;
            }
        }
        __syncthreads();  // the second half's sums are in; this buffer and cur are rewritten next
        if (half == 0) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                sv[2 * u] = acc[u].x + part[k][2 * u];
                sv[2 * u + 1] = acc[u].y + part[k][2 * u + 1];
            }
        }
    }
    cp_wait<0>();
    if (half == 0) {
#pragma unroll
        for (int u = 0; u < 8; ++u) state[(bh * kD + j0 + u) * kD + k] = sv[u];
    }
}

// o = O_zero + R S_start(g) for a tile of 128 tokens (two chunks) of a segment g >= 1 and one
// v-head (dense sequences, T tokens each), on the tensor core: A = R (bf16 [token][k],
// K-major, two 64-column boxes), B = S_start(g) (bf16 [k][j], MN-major, two 64-column boxes
// 16 KiB apart), D = 128 lanes x 128 fp32 columns of TMEM; thread = token row then adds
// O_zero (fp32) and stores.  Rows past the segment (an odd segment length) or past T are
// computed but not stored.  128 threads; every wait is bounded.
namespace segfix {
constexpr int kThreads = 128;
constexpr int kA = 0, kB = 32768, kBar = 65536;
constexpr int kAlloc = kBar + 64 + 1024;
}  // namespace segfix
template <typename TOut>
__global__ void __launch_bounds__(segfix::kThreads) gdn_seg_fix_kernel(const __grid_constant__ CUtensorMap tmR,
                                                                       const __grid_constant__ CUtensorMap tmS,
                                                                       const float* __restrict__ seg_o,
                                                                       TOut* __restrict__ o, int T, int Hv,
                                                                       int seg_len, int nseg) {
    using namespace segfix;
    extern __shared__ uint8_t xsm_raw[];
    // Launched as a programmatic dependent of the link kernel, whose CTAs allow this launch only
    // after their own griddepcontrol.wait on the state pass: the state pass has completed and
    // flushed by the time any CTA here starts, so R and O_zero are read at once; the segment
    // starts (the link kernel's results) only after this grid's own wait.
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(xsm_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bar_ld = reinterpret_cast<uint64_t*>(smem + kBar);
    uint64_t* bar_mma = bar_ld + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_ld + 2);
    volatile int* abort = reinterpret_cast<volatile int*>(bar_ld + 3);
    const int h = blockIdx.y;
    const int b = blockIdx.z / (nseg - 1);
    const int g = 1 + blockIdx.z % (nseg - 1);
    const int cs = g * seg_len;                                   // the segment's first chunk
    const int c_end = min((g + 1) * seg_len, (T + kC - 1) / kC);  // one past its last
    const int c_tile = cs + 2 * (int)blockIdx.x;                  // the tile's first chunk
    if (c_tile >= c_end) return;
    const int rows = min(2 * kC, min(c_end * kC, T) - c_tile * kC);  // tokens of the tile to store
    const int tid = threadIdx.x, warp = tid >> 5;
    const size_t bh = (size_t)b * Hv + h;
    if (tid == 0) {
        mbar_init(bar_ld, 1);
        mbar_init(bar_mma, 1);
        *abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 128);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;
    if (tid == 0) {
        const int tok = b * T + c_tile * kC;
        const int sg = (int)(bh * nseg + g);
        mbar_arrive_expect_tx(bar_ld, 4 * 16384);
        tma_load_4d(smem + kA, &tmR, bar_ld, 0, h, tok, 0);
        tma_load_4d(smem + kA + 16384, &tmR, bar_ld, 64, h, tok, 0);
        grid_dependency_wait();  // the segment starts
        tma_load_3d(smem + kB, &tmS, bar_ld, 0, 0, sg);
        tma_load_3d(smem + kB + 16384, &tmS, bar_ld, 64, 0, sg);
        ok = mbar_wait(bar_ld, 0, abort, &g_err_gdn_prefill);
        if (ok) {
            tc_fence_after();
            constexpr uint32_t idesc = make_idesc(Elem<__nv_bfloat16>::kFmt, 128, 128, false, true);
            const uint64_t da = smem_desc(smem_u32(smem + kA), 16, 1024, kLayoutSW128);
            const uint64_t db = smem_desc(smem_u32(smem + kB), 16384, 1024, kLayoutSW128);
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk)
                mma_f16_ss(tmem, da + (uint64_t)((((kk >> 2) * 16384) + (kk & 3) * 32) >> 4),
                           db + (uint64_t)((kk * 2048) >> 4), idesc, kk > 0 ? 1u : 0u);
        }
        mma_commit(bar_mma);  // also after a failed load wait: the epilogue's wait then ends
    }
    // this thread's O_zero row (token row = TMEM lane), every load issued while the MMAs run
    const int r = tid;
    const bool live = r < rows;
    const size_t row = ((size_t)b * T + (size_t)c_tile * kC + r) * Hv + h;
    float4 zr[kD / 4];
#pragma unroll
    for (int q = 0; q < kD / 4; ++q)
        zr[q] = live ? reinterpret_cast<const float4*>(seg_o + row * kD)[q] : make_float4(0.f, 0.f, 0.f, 0.f);
    grid_dependency_wait();  // (thread 0 passed it above) nothing is stored before the link kernel ends
    // (a load that timed out set the abort flag: then nothing is stored)
    ok = __all_sync(0xffffffffu, mbar_wait(bar_mma, 0, abort, &g_err_gdn_prefill) && *abort == 0);
    tc_fence_after();
    if (ok) {  // (warp-uniform: every lane takes part in the TMEM loads, only rows < rows store)
        TOut* dst = o + row * kD;
        const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
#pragma unroll
        for (int cc = 0; cc < kD / 32; ++cc) {
            uint32_t v[32];
            tmem_ld32(tmem + lane_base + cc * 32, v);
            tmem_ld_wait();
            if (live) {
                float ov[32];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 zz = zr[cc * 8 + q];
                    ov[4 * q + 0] = __uint_as_float(v[4 * q + 0]) + zz.x;
                    ov[4 * q + 1] = __uint_as_float(v[4 * q + 1]) + zz.y;
                    ov[4 * q + 2] = __uint_as_float(v[4 * q + 2]) + zz.z;
                    ov[4 * q + 3] = __uint_as_float(v[4 * q + 3]) + zz.w;
                }
                store_row32(dst + cc * 32, ov);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 128);
    }
}

// ===========================================================================
// host side
// ===========================================================================
// Pre-processing options of the fused entry (A_log, dt_bias may be null)
struct Fuse {
    bool on;
    const float* A_log;
    const float* dt_bias;
};

// The segmented chain (StateParams): segment length and count, and the workspace area of its
// buffers (end states, fp32 outputs, segment starts).  nseg == 1: the plain chain.
struct Seg {
    int seg_len, nseg;
    uint8_t* area;
};

// Segments pay when the plain chain leaves SMs idle (few sequences x v-heads, as on each GPU
// of a multi-GPU split).  Costs are counted in chain steps (~1.2 us each): a state pass of
// one wave costs its chain length plus ~4 steps of prologue and epilogue; a segmented plan
// must fit in one wave (a second wave repays everything) and adds the link kernel (~1.5
// steps a segment) and the output correction (~3 steps).  Packed sequences keep the plain
// chain.
Seg seg_plan(int B, int Hv, int nch, bool packed) {
    Seg best{nch, 1, nullptr};
    if (packed || nch < 8) return best;
    const long long sms = device_sm_count();
    const long long plain_ctas = (long long)B * Hv * (kD / kSlice);
    double best_cost = (double)((plain_ctas + sms - 1) / sms) * (nch + 4);
    for (int G = 2; G <= 8; G *= 2) {
        const int L = (nch + G - 1) / G;
        if (L < 4) break;
        const int nseg = (nch + L - 1) / L;
        if ((long long)B * nseg > 65535) break;
        // segment 0: the usual 4 slice-CTAs a head; later segments 8 (the transition columns)
        const long long ctas = (long long)B * Hv * (2LL * (kD / kSlice) * nseg - kD / kSlice);
        if (ctas > sms) break;
        const double cost = L + 4 + 1.5 * (nseg - 1) + 3;
        if (cost < best_cost) {
            best = Seg{L, nseg, nullptr};
            best_cost = cost;
        }
    }
    return best;
}

// The segment buffers, in this order: end states [B][Hv][nseg][256][128] fp32, zero-state
// outputs [ntok][Hv][128] fp32, R [ntok][Hv][128] bf16, segment starts [B][Hv][nseg][128][128]
// bf16.
struct SegLayout {
    size_t x, o, r, s, total;
};
SegLayout seg_layout(int nseg, int B, size_t ntok, int Hv) {
    SegLayout L{};
    if (nseg <= 1) return L;
    L.x = 0;
    L.o = align_up((size_t)B * Hv * nseg * 2 * kD * kD * 4, 1024);
    L.r = L.o + align_up(ntok * Hv * kD * 4, 1024);
    L.s = L.r + align_up(ntok * Hv * kD * 2, 1024);
    L.total = L.s + align_up((size_t)B * Hv * nseg * kD * kD * 2, 1024);
    return L;
}
size_t seg_bytes(const Seg& sg, int B, size_t ntok, int Hv) { return seg_layout(sg.nseg, B, ntok, Hv).total; }

// Packed sequences: cu is the device [B+1] token-offset array and ntok its last entry; dense
// B x T: cu = null, ntok = B * T.  T is the (longest) sequence length.
template <typename T16, typename TOut>
int launch(const void* q, const void* k, const void* v, const float* g_log, const float* beta,
           float* state, void* o, int B, int T, int Hqk, int Hv, int head_map, float scale,
           void* ws, cudaStream_t stream, Fuse fuse, const int* cu, int ntok, Seg sg) {
    const int nch = (T + kC - 1) / kC;
    const size_t nbhc = (size_t)B * Hv * nch;
    const WsLayout L = ws_layout(nbhc);
    const CUtensorMapDataType dt = Elem<T16>::kFmt == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap tq, tk, tv, tw, ta;
    int rc;
    if ((rc = make_tmap_4d(&tq, q, dt, 2, kD, Hqk, ntok, 1, 64, 1, kC, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
    if ((rc = make_tmap_4d(&tk, k, dt, 2, kD, Hqk, ntok, 1, 64, 1, kC, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
    if ((rc = make_tmap_4d(&tv, v, dt, 2, kD, Hv, ntok, 1, 64, 1, kC, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
    uint8_t* wsb = static_cast<uint8_t*>(ws);
    if ((rc = make_tmap_3d(&tw, wsb + L.w, dt, 2, kD, kC, nbhc, 64, kC, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
    if ((rc = make_tmap_3d(&ta, wsb + L.aqk, dt, 2, kC, kC, nbhc, 64, kC, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
    CUtensorMap tu, tus, tm;
    if ((rc = make_tmap_3d(&tm, wsb + L.m, dt, 2, kC, kC, nbhc, 64, kC, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
    if ((rc = make_tmap_3d(&tu, wsb + L.u, dt, 2, kD, kC, nbhc, 64, kC, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
    if ((rc = make_tmap_3d(&tus, wsb + L.u, dt, 2, kD, kC, nbhc, kSlice, kC, CU_TENSOR_MAP_SWIZZLE_64B)))
        return rc;

    PrepParams pp;
    pp.ws = wsb;
    pp.g_log = g_log;
    pp.beta = beta;
    pp.ws_u = L.u;
    pp.ws_aqk = L.aqk;
    pp.ws_gcs = L.gcs;
    pp.ws_rq = L.rq;
    pp.ws_rk = L.rk;
    pp.A_log = fuse.A_log;
    pp.dt_bias = fuse.dt_bias;
    pp.cu = cu;
    pp.ntok = ntok;
    pp.T = T;
    pp.Hqk = Hqk;
    pp.Hv = Hv;
    pp.nch = nch;
    pp.head_map = head_map;
    auto k1 = fuse.on ? gdn_prep_kernel<T16, true> : gdn_prep_kernel<T16, false>;
    B200_TRY_CUDA(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, prep::kAlloc));
    k1<<<dim3(nch, Hv, B), prep::kThreads, prep::kAlloc, stream>>>(tq, tk, tv, tw, tu, ta, tm, pp);
    B200_TRY_CUDA(cudaGetLastError());

    StateParams sp;
    sp.ws = wsb;
    sp.state = state;
    sp.o = o;
    sp.ws_gcs = L.gcs;
    sp.ws_rq = L.rq;
    sp.ws_rk = L.rk;
    sp.cu = cu;
    sp.ntok = ntok;
    sp.T = T;
    sp.Hqk = Hqk;
    sp.Hv = Hv;
    sp.nch = nch;
    sp.head_map = head_map;
    sp.scale = scale;
    sp.seg_len = sg.nseg > 1 ? sg.seg_len : nch;
    sp.nseg = sg.nseg > 1 ? sg.nseg : 1;
    const SegLayout SL = seg_layout(sp.nseg, B, (size_t)ntok, Hv);
    float* seg_x = sp.nseg > 1 ? reinterpret_cast<float*>(sg.area + SL.x) : nullptr;
    float* seg_o = sp.nseg > 1 ? reinterpret_cast<float*>(sg.area + SL.o) : nullptr;
    __nv_bfloat16* seg_r = sp.nseg > 1 ? reinterpret_cast<__nv_bfloat16*>(sg.area + SL.r) : nullptr;
    __nv_bfloat16* seg_s = sp.nseg > 1 ? reinterpret_cast<__nv_bfloat16*>(sg.area + SL.s) : nullptr;
    CUtensorMap tr, tss;
    if (sp.nseg > 1) {
        if ((rc = make_tmap_4d(&tr, seg_r, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kD, Hv, ntok, 1, 64, 1, 2 * kC,
                               CU_TENSOR_MAP_SWIZZLE_128B)))
            return rc;
        if ((rc = make_tmap_3d(&tss, seg_s, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kD, kD, (uint64_t)B * Hv * sp.nseg,
                               64, kD, CU_TENSOR_MAP_SWIZZLE_128B)))
            return rc;
    }
    sp.seg_x = seg_x;
    sp.seg_o = seg_o;
    sp.seg_r = seg_r;
    auto k2 = sp.nseg > 1 ? (fuse.on ? gdn_state_kernel<T16, TOut, true, true> : gdn_state_kernel<T16, TOut, false, true>)
                          : (fuse.on ? gdn_state_kernel<T16, TOut, true, false> : gdn_state_kernel<T16, TOut, false, false>);
    B200_TRY_CUDA(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, st::kAlloc));
    // launched with programmatic stream serialisation: its prologue (barriers, TMEM, the
    // initial state) overlaps the prep grid's last CTAs
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sp.nseg > 1 ? 2 * kD / kSlice : kD / kSlice, Hv, B * sp.nseg);
    cfg.blockDim = dim3(st::kThreads);
    cfg.dynamicSmemBytes = st::kAlloc;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    B200_TRY_CUDA(cudaLaunchKernelEx(&cfg, k2, tq, tk, tw, ta, tm, tus, sp));
    count_launch(2);
    B200_TRY_CUDA(cudaGetLastError());
    if (sp.nseg > 1) {
        // both as programmatic dependents of the kernel before them (each waits for it with
        // griddepcontrol.wait before reading its results), so their launches overlap its drain
        B200_TRY_CUDA(cudaFuncSetAttribute(gdn_seg_link_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           seglink::kSmem));
        cudaLaunchConfig_t lc = {};
        lc.gridDim = dim3(kD / 8, Hv, B);
        lc.blockDim = dim3(seglink::kThreads);
        lc.dynamicSmemBytes = seglink::kSmem;
        lc.stream = stream;
        lc.attrs = attr;
        lc.numAttrs = 1;
        B200_TRY_CUDA(cudaLaunchKernelEx(&lc, gdn_seg_link_kernel, (const float*)seg_x, seg_s, state, Hv, sp.nseg));
        B200_TRY_CUDA(cudaGetLastError());
        auto k4 = gdn_seg_fix_kernel<TOut>;
        B200_TRY_CUDA(cudaFuncSetAttribute(k4, cudaFuncAttributeMaxDynamicSharedMemorySize, segfix::kAlloc));
        cudaLaunchConfig_t fc = {};
        fc.gridDim = dim3((sp.seg_len + 1) / 2, Hv, B * (sp.nseg - 1));
        fc.blockDim = dim3(segfix::kThreads);
        fc.dynamicSmemBytes = segfix::kAlloc;
        fc.stream = stream;
        fc.attrs = attr;
        fc.numAttrs = 1;
        B200_TRY_CUDA(cudaLaunchKernelEx(&fc, k4, tr, tss, (const float*)seg_o, static_cast<TOut*>(o), T, Hv,
                                         sp.seg_len, sp.nseg));
        count_launch(2);
        B200_TRY_CUDA(cudaGetLastError());
    }
    return B200LAB_OK;
}

// fp32 q / k / v: one pass converts them to bf16 copies in the workspace, which the chunked
// kernels then read like 16-bit inputs (the tensor-core operands are 16-bit either way).
// blockIdx.y picks the tensor; 8 elements a thread per step (two 16-byte loads, one store).
struct F32Copies {
    const float* src[3];
    __nv_bfloat16* dst[3];
    size_t n8[3];  // elements / 8
};
__global__ void __launch_bounds__(256) f32_to_bf16_kernel(const F32Copies a) {
    const int t = blockIdx.y;
    const float4* src = reinterpret_cast<const float4*>(a.src[t]);
    uint4* dst = reinterpret_cast<uint4*>(a.dst[t]);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < a.n8[t];
         i += (size_t)gridDim.x * blockDim.x) {
        const float4 x = src[2 * i], y = src[2 * i + 1];
        uint4 o;
        o.x = Elem<__nv_bfloat16>::pack2(x.x, x.y);
        o.y = Elem<__nv_bfloat16>::pack2(x.z, x.w);
        o.z = Elem<__nv_bfloat16>::pack2(y.x, y.y);
        o.w = Elem<__nv_bfloat16>::pack2(y.z, y.w);
        dst[i] = o;
    }
}

// bytes of the bf16 copies of fp32 q, k, v for ntok tokens (each 1 KiB-aligned)
size_t f32_copy_bytes(size_t ntok, int Hqk, int Hv) {
    return 2 * align_up(ntok * Hqk * kD * 2, 1024) + align_up(ntok * Hv * kD * 2, 1024);
}

template <typename T16>
int dispatch_out(int out_dtype, const void* q, const void* k, const void* v, const float* g,
                 const float* be, float* state, void* o, int B, int T, int Hqk, int Hv, int hm,
                 float scale, void* ws, cudaStream_t s, Fuse f, const int* cu, int ntok, Seg sg) {
    switch (out_dtype) {
        case B200LAB_F16:
            return launch<T16, __half>(q, k, v, g, be, state, o, B, T, Hqk, Hv, hm, scale, ws, s, f, cu, ntok, sg);
        case B200LAB_BF16:
            return launch<T16, __nv_bfloat16>(q, k, v, g, be, state, o, B, T, Hqk, Hv, hm, scale, ws, s, f, cu,
                                              ntok, sg);
        case B200LAB_F32:
            return launch<T16, float>(q, k, v, g, be, state, o, B, T, Hqk, Hv, hm, scale, ws, s, f, cu, ntok, sg);
    }
    return B200LAB_ERR_UNSUPPORTED;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace
}  // namespace b200

B200_DEFINE_ERR_TAKER(gdn_prefill, b200::g_err_gdn_prefill)

namespace b200 {
namespace {
// the chunk items of the prep pass (the smallest workspace the entries accept, with the fp32
// copies for fp32 inputs); the segmented chain's buffers follow them
size_t prefill_base_bytes(int B, int T, int Hv) {
    if (B < 1 || T < 1 || Hv < 1) return 0;
    const size_t nch = ((size_t)T + kC - 1) / kC;
    return ws_layout((size_t)B * Hv * nch).total;
}
size_t prefill_min_bytes(int B, int T, int Hqk, int Hv, int in_dtype) {
    const size_t base = prefill_base_bytes(B, T, Hv);
    if (base == 0 || in_dtype != B200LAB_F32 || Hqk < 1) return base;
    return base + f32_copy_bytes((size_t)B * T, Hqk, Hv);
}
size_t prefill_seg_bytes(int B, int T, int Hv) {
    if (B < 1 || T < 1 || Hv < 1) return 0;
    const int nch = (T + kC - 1) / kC;
    return seg_bytes(seg_plan(B, Hv, nch, false), B, (size_t)B * T, Hv);
}
}  // namespace
}  // namespace b200

extern "C" size_t gdn_prefill_sm100_workspace(int B, int T, int Hqk, int Hv, int dk, int dv) {
    (void)dk;
    (void)dv;
    const size_t base = b200::prefill_min_bytes(B, T, Hqk, Hv, B200LAB_BF16);
    return base == 0 ? 0 : base + b200::prefill_seg_bytes(B, T, Hv);
}

extern "C" size_t gdn_prefill_sm100_workspace_ex(int B, int T, int Hqk, int Hv, int dk, int dv, int in_dtype) {
    (void)dk;
    (void)dv;
    const size_t base = b200::prefill_min_bytes(B, T, Hqk, Hv, in_dtype);
    return base == 0 ? 0 : base + b200::prefill_seg_bytes(B, T, Hv);
}

extern "C" size_t gdn_prefill_sm100_workspace_min(int B, int T, int Hqk, int Hv, int dk, int dv, int in_dtype) {
    (void)dk;
    (void)dv;
    return b200::prefill_min_bytes(B, T, Hqk, Hv, in_dtype);
}

namespace b200 {
namespace {
// cu / ntok: packed sequences (T = the longest), or null / unused for dense B x T
int prefill_entry(const void* q, const void* k, const void* v, const float* g_log, const float* beta,
                  float* state, void* o, int B, int T, int Hqk, int Hv, int dk, int dv, int head_map,
                  float scale, int in_dtype, int out_dtype, void* workspace, size_t ws_bytes, void* stream,
                  Fuse fuse, const int* cu = nullptr, int ntok = 0) {
    if (!q || !k || !v || !g_log || !beta || !state || !o) return B200LAB_ERR_INVALID;
    if (B < 1 || T < 0 || Hqk < 1 || Hv < 1 || dk < 1 || dv < 1) return B200LAB_ERR_INVALID;
    if (cu && ntok < 1) return B200LAB_ERR_INVALID;
    if (!cu && (long long)B * T > 0x7fffffffLL) return B200LAB_ERR_UNSUPPORTED;
    if (head_map != 0 && head_map != 1) return B200LAB_ERR_INVALID;
    if (head_map == 1 && Hv % Hqk != 0) return B200LAB_ERR_INVALID;
    if (in_dtype < B200LAB_F16 || in_dtype > B200LAB_F32) return B200LAB_ERR_INVALID;
    if (out_dtype < B200LAB_F16 || out_dtype > B200LAB_F32) return B200LAB_ERR_INVALID;
    if (dk != 128 || dv != 128) return B200LAB_ERR_UNSUPPORTED;
    if (B > 65535 || Hv > 65535) return B200LAB_ERR_UNSUPPORTED;
    if (T == 0) return B200LAB_OK;
    if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(state, 16) ||
        !aligned(o, 16))
        return B200LAB_ERR_INVALID;
    // fp32 inputs: the bf16 copies are sized by B * max_seqlen tokens, which bounds total_tokens
    if (in_dtype == B200LAB_F32 && cu && (long long)ntok > (long long)B * T) return B200LAB_ERR_INVALID;
    // the chunk items (and fp32 copies) are required; the segmented chain's buffers are used
    // when the workspace also holds them (the size gdn_prefill_sm100_workspace reports)
    const size_t need = prefill_min_bytes(B, T, Hqk, Hv, in_dtype);
    if (!workspace || ws_bytes < need || !aligned(workspace, 256)) return B200LAB_ERR_WORKSPACE;
    int rc = check_device_sm100();
    if (rc != B200LAB_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!cu) ntok = B * T;
    Seg sg = seg_plan(B, Hv, (T + kC - 1) / kC, cu != nullptr);
    if (ws_bytes - need < seg_bytes(sg, B, (size_t)ntok, Hv)) sg = Seg{(T + kC - 1) / kC, 1, nullptr};
    sg.area = static_cast<uint8_t*>(workspace) + need;
    if (in_dtype == B200LAB_F32) {
        // bf16 copies after the chunk items, then the 16-bit path on them
        uint8_t* conv = static_cast<uint8_t*>(workspace) + prefill_base_bytes(B, T, Hv);
        const size_t nqk = (size_t)ntok * Hqk * kD, nv = (size_t)ntok * Hv * kD;
        F32Copies cp;
        cp.src[0] = static_cast<const float*>(q);
        cp.src[1] = static_cast<const float*>(k);
        cp.src[2] = static_cast<const float*>(v);
        cp.dst[0] = reinterpret_cast<__nv_bfloat16*>(conv);
        cp.dst[1] = reinterpret_cast<__nv_bfloat16*>(conv + align_up(nqk * 2, 1024));
        cp.dst[2] = reinterpret_cast<__nv_bfloat16*>(conv + 2 * align_up(nqk * 2, 1024));
        cp.n8[0] = cp.n8[1] = nqk / 8;
        cp.n8[2] = nv / 8;
        const size_t most = nqk > nv ? nqk : nv;
        const unsigned gx = (unsigned)std::min<size_t>((most / 8 + 255) / 256, 148 * 16);
        f32_to_bf16_kernel<<<dim3(gx, 3), 256, 0, s>>>(cp);
        B200_TRY_CUDA(cudaGetLastError());
        count_launch(1);
        return dispatch_out<__nv_bfloat16>(out_dtype, cp.dst[0], cp.dst[1], cp.dst[2], g_log, beta, state, o, B,
                                           T, Hqk, Hv, head_map, scale, workspace, s, fuse, cu, ntok, sg);
    }
    if (in_dtype == B200LAB_BF16)
        return dispatch_out<__nv_bfloat16>(out_dtype, q, k, v, g_log, beta, state, o, B, T, Hqk, Hv,
                                           head_map, scale, workspace, s, fuse, cu, ntok, sg);
    return dispatch_out<__half>(out_dtype, q, k, v, g_log, beta, state, o, B, T, Hqk, Hv, head_map,
                                scale, workspace, s, fuse, cu, ntok, sg);
}
}  // namespace
}  // namespace b200

extern "C" int gdn_prefill_sm100(const void* q, const void* k, const void* v, const float* g_log,
                                 const float* beta, float* state, void* o, int B, int T, int Hqk,
                                 int Hv, int dk, int dv, int head_map, float scale, int in_dtype,
                                 int out_dtype, void* workspace, size_t ws_bytes, void* stream) {
    return b200::prefill_entry(q, k, v, g_log, beta, state, o, B, T, Hqk, Hv, dk, dv, head_map, scale,
                               in_dtype, out_dtype, workspace, ws_bytes, stream,
                               b200::Fuse{false, nullptr, nullptr});
}

extern "C" int gdn_prefill_sm100_varlen(const void* q, const void* k, const void* v, const float* g_log,
                                        const float* beta, float* state, void* o, const int* cu_seqlens,
                                        int max_seqlen, int total_tokens, int B, int Hqk, int Hv, int dk,
                                        int dv, int head_map, float scale, int in_dtype, int out_dtype,
                                        void* workspace, size_t ws_bytes, void* stream) {
    if (!cu_seqlens) return B200LAB_ERR_INVALID;
    if (max_seqlen < 1 || total_tokens < 1) return B200LAB_ERR_INVALID;
    return b200::prefill_entry(q, k, v, g_log, beta, state, o, B, max_seqlen, Hqk, Hv, dk, dv, head_map, scale,
                               in_dtype, out_dtype, workspace, ws_bytes, stream,
                               b200::Fuse{false, nullptr, nullptr}, cu_seqlens, total_tokens);
}

extern "C" int gdn_prefill_sm100_fused_varlen(const void* q, const void* k, const void* v, const float* a,
                                              const float* b, const float* A_log, const float* dt_bias,
                                              float* state, void* o, const int* cu_seqlens, int max_seqlen,
                                              int total_tokens, int B, int Hqk, int Hv, int dk, int dv,
                                              int head_map, float scale, int in_dtype, int out_dtype,
                                              void* workspace, size_t ws_bytes, void* stream) {
    if (!cu_seqlens) return B200LAB_ERR_INVALID;
    if (max_seqlen < 1 || total_tokens < 1) return B200LAB_ERR_INVALID;
    return b200::prefill_entry(q, k, v, a, b, state, o, B, max_seqlen, Hqk, Hv, dk, dv, head_map, scale, in_dtype,
                               out_dtype, workspace, ws_bytes, stream, b200::Fuse{true, A_log, dt_bias},
                               cu_seqlens, total_tokens);
}

extern "C" int gdn_prefill_sm100_fused(const void* q, const void* k, const void* v, const float* a,
                                       const float* b, const float* A_log, const float* dt_bias,
                                       float* state, void* o, int B, int T, int Hqk, int Hv, int dk,
                                       int dv, int head_map, float scale, int in_dtype, int out_dtype,
                                       void* workspace, size_t ws_bytes, void* stream) {
    return b200::prefill_entry(q, k, v, a, b, state, o, B, T, Hqk, Hv, dk, dv, head_map, scale, in_dtype,
                               out_dtype, workspace, ws_bytes, stream, b200::Fuse{true, A_log, dt_bias});
}

// ===========================================================================
// Allocation-free entry (gdn_prefill_sm100_noalloc): scratch in a file-scope
// device array instead of a caller workspace.  In host code the array's name
// is only a host-side stand-in, so its device address is looked up with
// cudaGetSymbolAddress on every call, with the caller's device current (the
// first lookup on a device loads the module there; later ones are cheap, and
// a module reloaded after cudaDeviceReset is found at its new address).
// ===========================================================================
static __device__ __align__(256) unsigned char g_prefill_noalloc_scratch[B200LAB_NOALLOC_SCRATCH_BYTES];

extern "C" int gdn_prefill_sm100_noalloc(const void* q, const void* k, const void* v,
                                         const float* g_log, const float* beta, float* state,
                                         void* o, int B, int T, int Hqk, int Hv, int dk, int dv,
                                         int head_map, float scale, int in_dtype, int out_dtype,
                                         void* stream) {
    int rc = b200::check_device_sm100();
    if (rc != B200LAB_OK) return rc;
    void* scratch = nullptr;
    if (cudaGetSymbolAddress(&scratch, g_prefill_noalloc_scratch) != cudaSuccess || !scratch)
        return B200LAB_ERR_CUDA;
    // the workspace entry checks the arguments first, then that the problem's workspace fits
    // in the array (B200LAB_ERR_WORKSPACE otherwise)
    return gdn_prefill_sm100(q, k, v, g_log, beta, state, o, B, T, Hqk, Hv, dk, dv, head_map,
                             scale, in_dtype, out_dtype, scratch,
                             (size_t)B200LAB_NOALLOC_SCRATCH_BYTES, stream);
}
