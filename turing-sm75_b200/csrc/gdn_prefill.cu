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
#include "common.cuh"
#include "errwords.h"

namespace b200 {
namespace {

__device__ int g_err_gdn_prefill = 0;

constexpr int kC = 64;    // chunk length
constexpr int kD = 128;   // dk = dv

// ---- workspace layout ------------------------------------------------------
struct WsLayout {
    size_t w, u, aqk, m, qt, gcs, vdec, total;
};
__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
__host__ __device__ inline WsLayout ws_layout(size_t nbhc) {
    WsLayout L;
    L.w = 0;
    L.u = align_up(L.w + nbhc * kC * kD * 2, 1024);
    L.aqk = align_up(L.u + nbhc * kC * kD * 2, 1024);
    L.m = align_up(L.aqk + nbhc * kC * kC * 2, 1024);
    L.qt = align_up(L.m + nbhc * kC * kC * 2, 1024);
    L.gcs = align_up(L.qt + nbhc * kC * kD * 2, 1024);
    L.vdec = align_up(L.gcs + nbhc * kC * 4, 1024);  // e^{gcs_last - gcs_t} (/ |k_t| fused)
    L.total = align_up(L.vdec + nbhc * kC * 4, 1024);
    return L;
}

struct PrepParams {
    uint8_t* ws;
    const float* g_log;    // fused: the gate logits a
    const float* beta;     // fused: the beta logits b
    const float* A_log;    // fused: [Hv] or null
    const float* dt_bias;  // fused: [Hv] or null
    size_t ws_u, ws_aqk, ws_gcs, ws_vdec;
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
constexpr int kAT = 32768;         // [T diag(beta Gam); T diag(beta)] 128 x 64, 16 KiB
constexpr int kLd = 68;            // fp32 row pitch of A and T (16-byte aligned, fewer conflicts)
constexpr int kAs = 49152;         // A, then T = (I + A)^-1 in place, fp32 64 x kLd
constexpr int kMisc = kAs + kC * kLd * 4;
constexpr int kXs = kMisc + 3072;  // 32 x 36 fp32 scratch of the block inverse (its own
                                   // slot: AT is still being read by the Aqk store then)
constexpr int kBytes = kXs + 32 * 36 * 4;
constexpr int kAlloc = kBytes + 1024;
static_assert(3 * (kAlloc + 1024) <= 233472, "three prep CTAs per SM");
static_assert(kAlloc <= 232448, "state kernel shared memory above the 227 KiB per-CTA limit");
// 128 columns: three CTAs per SM fit the 512 TMEM columns without one waiting in
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
static_assert(sizeof(Misc) <= kXs - kMisc, "prep Misc overflows its slot");
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
__device__ __forceinline__ void offdiag_block_inverse(float* As, float* X, int tid) {
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
        *reinterpret_cast<float4*>(X + r * 36 + c0) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        *reinterpret_cast<float4*>(X + r * 36 + c0 + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
    __syncthreads();
    {   // T21 = -T22 X
        float acc[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) acc[u] = 0.f;
#pragma unroll
        for (int s = 0; s < 32; ++s) {
            const float a = Ts[(32 + r) * kLd + 32 + s];
            const float4 x0 = *reinterpret_cast<const float4*>(X + s * 36 + c0);
            const float4 x1 = *reinterpret_cast<const float4*>(X + s * 36 + c0 + 4);
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
__global__ void __launch_bounds__(prep::kThreads, 3)
    gdn_prep_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmW,
                    const __grid_constant__ CUtensorMap tmU, const __grid_constant__ CUtensorMap tmAqk,
                    const __grid_constant__ CUtensorMap tmM, const __grid_constant__ CUtensorMap tmQt,
                    const PrepParams p) {
    using namespace prep;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Misc* ms = reinterpret_cast<Misc*>(smem + kMisc);
    float* As = reinterpret_cast<float*>(smem + kAs);
    const float* Ts = As;  // T replaces A in place
    float* Xs = reinterpret_cast<float*>(smem + kXs);
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
    ok = __all_sync(0xffffffffu, mbar_wait(&ms->bar_mma1, 0, abort, &g_err_gdn_prefill));
    if constexpr (kFused) {
        // per-token 1/|k_t| and 1/|q_t| from the tiles, before V is loaded over Q
        ok = __all_sync(0xffffffffu, mbar_wait(&ms->bar_tma, 0, abort, &g_err_gdn_prefill)) && ok;
        if (tid < kC) ms->rk[tid] = row_rnorm<T16>(smem + kK0, smem + kK1, tid);
        else ms->rq[tid - kC] = row_rnorm<T16>(smem + kQ0, smem + kQ1, tid - kC);
        __syncthreads();
    }
    // Qt = diag(e^{gcs_t} / |q_t|) Q, scaled in place over the Q tile (MMA1 has read it) and
    // stored to the workspace: the state pass's output product takes it as is.  Thread =
    // (row, 64-column box); scaling whole rows commutes with the 128-byte swizzle.
    ok = __all_sync(0xffffffffu, mbar_wait(&ms->bar_tma, 0, abort, &g_err_gdn_prefill)) && ok;
    tc_fence_after();
    {
        const int r = tid & (kC - 1);
        uint8_t* qrow = smem + (tid < kC ? kQ0 : kQ1) + r * 128;
        float f = ex2f(ms->g2[r]);
        if constexpr (kFused) f *= ms->rq[r];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            uint4 raw = *reinterpret_cast<const uint4*>(qrow + q * 16);
            uint32_t* w = &raw.x;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const T16* e = reinterpret_cast<const T16*>(&w[u]);
                w[u] = Elem<T16>::pack2(Elem<T16>::to_f(e[0]) * f, Elem<T16>::to_f(e[1]) * f);
            }
            *reinterpret_cast<uint4*>(qrow + q * 16) = raw;
        }
        fence_proxy_async_smem();
    }
    __syncthreads();
    if (tid == 0 && ok) {
        tma_store_3d(&tmQt, smem + kQ0, 0, 0, (int)bhc);
        tma_store_3d(&tmQt, smem + kQ1, 64, 0, (int)bhc);
        bulk_commit();
        bulk_wait_read();  // Qt has left shared memory: V goes over it (needed only by MMA2)
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
            // Aqk row (lower incl. diagonal), 16-bit, staged 128B-swizzled in the (not yet
            // used) AT tile and written to the workspace by one TMA store
            uint8_t* stg = smem + kAT + row * 128;
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
                *reinterpret_cast<uint4*>(stg + (((s >> 3) ^ (row & 7)) << 4)) = pk;
            }
            fence_proxy_async_smem();
        }
    }
    __syncthreads();
    if (tid == 64 && ok) {
        tma_store_3d(&tmAqk, smem + kAT, 0, 0, (int)bhc);
        bulk_commit();
    }

    {
        const int j = tid & 63;
        float sc = tid < kC ? ms->beta[j] * ex2f(ms->g2[j]) : ms->beta[j];
        if constexpr (kFused)
            if (tid < kC) sc *= ms->rk[j];  // W = T diag(beta Gam / |k|) K
        ms->colscale[tid] = sc;
    }
    offdiag_block_inverse(As, Xs, tid);  // contains __syncthreads: every thread calls it
    if (tid == 64 && ok) {
        bulk_wait_read();  // the Aqk store has read the AT tile, which is rewritten next
    }
    __syncthreads();
    {
        // AT rows 0-63 <- T diag(beta Gam), rows 64-127 <- T diag(beta). Thread = AT row:
        // eight 16-byte swizzled chunks of 8 columns each (conflict-free row reads of Ts,
        // broadcast reads of the column scales)
        const int r = tid;
        const float* trow = Ts + (r & (kC - 1)) * kLd;
        const float* sc = ms->colscale + (r < kC ? 0 : kC);
        uint8_t* at = smem + kAT + r * 128;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
            const float4 a = *reinterpret_cast<const float4*>(trow + c8 * 8);
            const float4 b = *reinterpret_cast<const float4*>(trow + c8 * 8 + 4);
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
        if (c > 0) {
            // K of the previous chunk into the (now dead) A tile, for M below
            mbar_arrive_expect_tx(&ms->bar_kp, 2 * 8192);
            tma_load_4d(smem + kAs, &tmK, &ms->bar_kp, 0, hq, tok0 - kC, 0);
            tma_load_4d(smem + kAs + 8192, &tmK, &ms->bar_kp, 64, hq, tok0 - kC, 0);
        }
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
        float vdec = __expf(ms->gcs[kC - 1] - gcs_r);  // the state update's row decay
        if constexpr (kFused) vdec *= ms->rk[row];     // K^T diag(1/|k|): normalised keys
        reinterpret_cast<float*>(p.ws + p.ws_vdec)[bhc * kC + row] = vdec;
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
    if (ok && warp >= 2) stage_rows(smem + kV0);  // U -> [. | V0 | . | V1]
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && ok) {
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
    // The state pass uses W only as e^{gcs_last of the previous chunk} W: the staged W (read
    // unscaled by the M product above) is rescaled in place before it is stored.  Thread =
    // (row, 64-column box), as for Qt.
    if (c > 0 && ok) {
        const float gam = __expf(ms->gprev[kC - 1]);
        uint8_t* wrow = smem + (tid < kC ? kK0 : kK1) + (tid & (kC - 1)) * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            uint4 raw = *reinterpret_cast<const uint4*>(wrow + q * 16);
            uint32_t* w = &raw.x;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const T16* e = reinterpret_cast<const T16*>(&w[u]);
                w[u] = Elem<T16>::pack2(Elem<T16>::to_f(e[0]) * gam, Elem<T16>::to_f(e[1]) * gam);
            }
            *reinterpret_cast<uint4*>(wrow + q * 16) = raw;
        }
        fence_proxy_async_smem();
    }
    __syncthreads();
    if (tid == 0 && ok) {
        tma_store_3d(&tmW, smem + kK0, 0, 0, (int)bhc);
        tma_store_3d(&tmW, smem + kK1, 64, 0, (int)bhc);
        tma_store_3d(&tmM, smem + kAT, 0, 0, (int)bhc);
        bulk_commit();
        bulk_wait_all();   // the next kernel reads Qt, W, U, Aqk, M
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
// Kernel 2: sequential state pass, one CTA per (sequence, v-head)
// ===========================================================================
// Transposed form: the v column j of the state is the MMA's M dimension (TMEM lane j), so
// every product has N = 128 (the full tensor rate) and the state itself never leaves TMEM.
// With S_c the state at the start of chunk c ([dv][dk], fp32), Vn_c = U_c - W_c S_c^T and
// gam_c = e^{gcs_last,c}, per chunk:
//   Y_c   = S_c [Qt_c; Wp_{c+1}]^T + Vn_c^T [Aqk_c; M_{c+1}]^T       (lane j, 128 columns)
//           columns 0-63:   o_c^T / scale     (Qt_c = diag(e^{gcs}) Q_c from the prep pass)
//           columns 64-127: U_{c+1} - Vn_{c+1}  (Wp_{c+1} = gam_c W_{c+1}, M_{c+1} as below)
//   S_{c+1} = gam_c S_c + Vt_c^T K_c,   Vt_c = diag(e^{gcs_last - gcs}) Vn_c
// where M_{c+1} = W_{c+1} K_c^T diag(e^{gcs_last,c - gcs_c}) (prep pass) carries the chain
// through Vn: Vn_{c+1} = U_{c+1} - gam_c W_{c+1} S_c^T - M_{c+1} Vn_c.  The A operands (S_c,
// Vn_c, Vt_c as 16-bit) are written to TMEM by the threads; the B operands come by TMA.
namespace ch {
// warps 0-3: the state (thread = v column j = TMEM lane): S16_c and gam_c S_c into TMEM;
// warps 4-7: Vn_{c+1}, Vt_{c+1} from Y_c and U_{c+1}, then the outputs o_c;
// warp 8: TMA producer; warp 9: TMEM owner and MMA issuer.
constexpr int kThreads = 320;
constexpr int kWarpVn = 4, kWarpProducer = 8, kWarpMma = 9;
// one stage (the inputs of chunk c's products), 81 KiB:
//   B1 [Qt_c b0 | Wp_{c+1} b0 | Qt_c b1 | Wp_{c+1} b1]  32 KiB  B of Y p1 (K-major, 128 rows)
//   B2 [Aqk_c | M_{c+1}]                                16 KiB  B of Y p2 (K-major)
//   Kt [K_c b0 | K_c b1]                                16 KiB  B of the state update (MN-major)
//   U  [U_{c+1} b0 | U_{c+1} b1]                        16 KiB  read by the Vn warps
//   G  gcs_c | gcs_{c+1} | 1/|k| of chunk c+1 (fp32 x 64 each)
// (b0/b1: 64-column boxes, 128-byte swizzle).  The prologue stage carries Wp_0, U_0, gcs_0.
constexpr int kB1 = 0, kB2 = 32768, kKt = 49152, kU = 65536, kG = 81920;
constexpr int kStage = 82944;
constexpr int kStages = 2;
constexpr int kMisc = kStages * kStage;
constexpr int kBytes = kMisc + 512;
constexpr int kAlloc = kBytes + 1024;
static_assert(kAlloc <= 232448, "chain kernel shared memory above the 227 KiB per-CTA limit");
// TMEM columns: S fp32 [0,128); Y buffers [128,256), [256,384); A operands S16 (64 cols),
// Vn16 (32), Vt16 (32)
constexpr uint32_t kColS = 0, kColY = 128, kColS16 = 384, kColVn = 448, kColVt = 480;
constexpr uint32_t kTmemCols = 512;

struct Misc {
    uint64_t full[kStages], empty[kStages];
    uint64_t s_ready;      // S16_c and gam_c S_c are in TMEM (4 state-warp arrivals)
    uint64_t vn_ready;     // Vn_c, Vt_c are in TMEM (4 Vn-warp arrivals)
    uint64_t ds_done;      // the state update of chunk c has completed (MMA commit)
    uint64_t y_full[2];    // Y buffer complete (MMA commit)
    uint64_t y_empty[2];   // Y buffer read out (4 Vn-warp arrivals)
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};
static_assert(sizeof(Misc) <= kBytes - kMisc, "chain Misc overflows its slot");
// arrivals on a stage's `empty` barrier: the MMA thread's commit, 4 Vn warps, 4 state warps
constexpr uint32_t kEmptyCount = 9;
}  // namespace ch

struct ChainParams {
    const uint8_t* ws;
    float* state;
    void* o;
    size_t ws_gcs, ws_vdec;
    const int* cu;  // as PrepParams
    int T, Hqk, Hv, nch, head_map;
    int ntok;
    float scale;
};

// Stage of chunk c: slot c & 1; slot 1 holds the prologue first, so both slots' use counts
// are (c + 1) >> 1 and the barrier parities follow from it.
__device__ __forceinline__ uint32_t ch_use(int c) { return (uint32_t)((c + 1) >> 1); }

// 16-bit element (t, j) of a 64-token x 128-column tile held as two 128B-swizzled boxes
template <typename T16>
__device__ __forceinline__ float tile_elem(const uint8_t* tile, int t, int j) {
    const int off = (j >> 6) * 8192 + t * 128 + ((((j & 63) >> 3) ^ (t & 7)) << 4) + (j & 7) * 2;
    return Elem<T16>::to_f(*reinterpret_cast<const T16*>(tile + off));
}

template <typename T16, typename TOut>
__global__ void __launch_bounds__(ch::kThreads, 1)
    gdn_chain_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQt,
                     const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmAqk,
                     const __grid_constant__ CUtensorMap tmM, const __grid_constant__ CUtensorMap tmU,
                     const ChainParams p) {
    using namespace ch;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Misc* ms = reinterpret_cast<Misc*>(smem + kMisc);
    volatile int* abort = &ms->abort;

    const int h = blockIdx.x;
    const int b = blockIdx.y;
    const SeqSpan seq = seq_span(p.cu, p.T, b);
    if (!seq_ok(seq, p.T, p.ntok)) return;    // recorded by the prep grid; state left as it is
    const int nch = (seq.len + kC - 1) / kC;  // this sequence's chunks (p.nch for the longest)
    if (nch == 0) return;                     // an empty sequence: its state stays as it is
    const int hq = qk_head(h, p.Hqk, p.Hv, p.head_map);
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const size_t bh = (size_t)b * p.Hv + h;
    const int bhc0 = (int)(bh * p.nch);  // workspace slots: p.nch chunks a (sequence, head)

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&ms->full[i], 1);
            mbar_init(&ms->empty[i], kEmptyCount);
            mbar_init(&ms->y_full[i], 1);
            mbar_init(&ms->y_empty[i], 4);
        }
        mbar_init(&ms->s_ready, 4);
        mbar_init(&ms->vn_ready, 4);
        mbar_init(&ms->ds_done, 1);
        mbar_init(&ms->drain, 1);
        ms->abort = 0;
        fence_barrier_init();
    }
    if (warp == kWarpMma) {
        tmem_alloc(&ms->tmem_base, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ms->tmem_base;
    constexpr uint32_t kFmt = Elem<T16>::kFmt;
    volatile int no_abort = 0;  // drain waits ignore the abort flag: copies in flight land first

    if (warp == kWarpProducer) {
        if (lane == 0) {
            const float* gcs_all = reinterpret_cast<const float*>(p.ws + p.ws_gcs);
            const float* vdec_all = reinterpret_cast<const float*>(p.ws + p.ws_vdec);
            int last_use[kStages] = {-1, 0};  // slot 1 carries the prologue (use 0)
            grid_dependency_wait();  // Qt, W, U, Aqk, M, gcs come from the prep grid
            {   // prologue stage (slot 1): Wp_0 in the W rows of B1, U_0, gcs_0 and decays
                uint8_t* stg = smem + kStage;
                uint64_t* bar = &ms->full[1];
                mbar_arrive_expect_tx(bar, 4 * 8192 + 2 * 256);
                tma_load_3d(stg + kB1 + 8192, &tmW, bar, 0, 0, bhc0);
                tma_load_3d(stg + kB1 + 24576, &tmW, bar, 64, 0, bhc0);
                tma_load_3d(stg + kU, &tmU, bar, 0, 0, bhc0);
                tma_load_3d(stg + kU + 8192, &tmU, bar, 64, 0, bhc0);
                bulk_load_1d(stg + kG + 256, gcs_all + (size_t)bhc0 * kC, kC * 4, bar);
                bulk_load_1d(stg + kG + 512, vdec_all + (size_t)bhc0 * kC, kC * 4, bar);
            }
            for (int c = 0; c < nch; ++c) {
                const int s = c & 1;
                const uint32_t u = ch_use(c);
                if (u >= 1 && !mbar_wait(&ms->empty[s], (u - 1) & 1, abort, &g_err_gdn_prefill)) break;
                uint8_t* stg = smem + s * kStage;
                uint64_t* bar = &ms->full[s];
                const int bhc = bhc0 + c;
                const int tok = seq.start + c * kC;
                const bool next = c + 1 < nch;  // the last chunk has no successor to prepare
                mbar_arrive_expect_tx(bar, 5 * 8192 + 256 + (next ? 5 * 8192 + 2 * 256 : 0));
                tma_load_3d(stg + kB1, &tmQt, bar, 0, 0, bhc);
                tma_load_3d(stg + kB1 + 16384, &tmQt, bar, 64, 0, bhc);
                tma_load_3d(stg + kB2, &tmAqk, bar, 0, 0, bhc);
                tma_load_4d(stg + kKt, &tmK, bar, 0, hq, tok, 0);
                tma_load_4d(stg + kKt + 8192, &tmK, bar, 64, hq, tok, 0);
                bulk_load_1d(stg + kG, gcs_all + (size_t)bhc * kC, kC * 4, bar);
                if (next) {
                    tma_load_3d(stg + kB1 + 8192, &tmW, bar, 0, 0, bhc + 1);
                    tma_load_3d(stg + kB1 + 24576, &tmW, bar, 64, 0, bhc + 1);
                    tma_load_3d(stg + kB2 + 8192, &tmM, bar, 0, 0, bhc + 1);
                    tma_load_3d(stg + kU, &tmU, bar, 0, 0, bhc + 1);
                    tma_load_3d(stg + kU + 8192, &tmU, bar, 64, 0, bhc + 1);
                    bulk_load_1d(stg + kG + 256, gcs_all + (size_t)(bhc + 1) * kC, kC * 4, bar);
                    bulk_load_1d(stg + kG + 512, vdec_all + (size_t)(bhc + 1) * kC, kC * 4, bar);
                }
                last_use[s] = (int)u;
            }
            // every copy issued has landed before the CTA exits
            for (int s = 0; s < kStages; ++s)
                if (last_use[s] >= 0) mbar_wait(&ms->full[s], last_use[s] & 1, &no_abort, &g_err_gdn_prefill);
        }
    } else if (warp == kWarpMma) {
        if (lane == 0) {
            constexpr uint32_t id_y = make_idesc(kFmt, 128, 128, false, false);   // B K-major
            constexpr uint32_t id_ds = make_idesc(kFmt, 128, 128, false, true);   // B MN-major
            const uint64_t dB1 = smem_desc(smem_u32(smem + kB1), 16, 1024, kLayoutSW128);
            const uint64_t dB2 = smem_desc(smem_u32(smem + kB2), 16, 1024, kLayoutSW128);
            const uint64_t dKt = smem_desc(smem_u32(smem + kKt), 8192, 1024, kLayoutSW128);
            // Y p1 = S_c [Qt_c; Wp_{c+1}]^T  (A = S16 from TMEM, K = dk = 128)
            auto p1 = [&](uint32_t so, uint32_t ycol) {
#pragma unroll
                for (int kk = 0; kk < kD / 16; ++kk) {
                    const uint32_t off = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
                    mma_f16_ts(tmem + ycol, tmem + kColS16 + kk * 8, dB1 + so + off, id_y, kk > 0 ? 1u : 0u);
                }
            };
            bool ok = mbar_wait(&ms->full[1], 0, abort, &g_err_gdn_prefill) &&
                      mbar_wait(&ms->s_ready, 0, abort, &g_err_gdn_prefill);
            if (ok) {  // prologue: W_0 S_0^T into Y buffer 1 (its Qt half reads nothing loaded)
                tc_fence_after();
                p1(kStage >> 4, kColY + 128);
                mma_commit(&ms->y_full[1]);
                mma_commit(&ms->empty[1]);
            }
            for (int c = 0; ok && c < nch; ++c) {
                const int s = c & 1;
                const uint32_t so = (uint32_t)(s * kStage) >> 4;
                const uint32_t ycol = kColY + (c & 1) * 128;
                if (!mbar_wait(&ms->full[s], ch_use(c) & 1, abort, &g_err_gdn_prefill)) break;
                if (!mbar_wait(&ms->s_ready, c & 1, abort, &g_err_gdn_prefill)) break;
                if (c >= 1 && !mbar_wait(&ms->y_empty[c & 1], ((c - 1) >> 1) & 1, abort, &g_err_gdn_prefill))
                    break;
                tc_fence_after();
                p1(so, ycol);
                // Vn_c is the chain dependency: waited for last
                if (!mbar_wait(&ms->vn_ready, c & 1, abort, &g_err_gdn_prefill)) break;
                tc_fence_after();
                // S += Vt_c^T K_c  (A = Vt16 from TMEM, K = 64 tokens; the threads put gam_c S_c there)
#pragma unroll
                for (int kk = 0; kk < kC / 16; ++kk)
                    mma_f16_ts(tmem + kColS, tmem + kColVt + kk * 8, dKt + so + ((kk * 2048) >> 4), id_ds, 1u);
                mma_commit(&ms->ds_done);
                // Y p2 += Vn_c^T [Aqk_c; M_{c+1}]^T  (A = Vn16 from TMEM, K = 64 tokens)
#pragma unroll
                for (int kk = 0; kk < kC / 16; ++kk)
                    mma_f16_ts(tmem + ycol, tmem + kColVn + kk * 8, dB2 + so + ((kk * 32) >> 4), id_y, 1u);
                mma_commit(&ms->y_full[c & 1]);
                mma_commit(&ms->empty[s]);
            }
            mma_commit(&ms->drain);
            mbar_wait(&ms->drain, 0, &no_abort, &g_err_gdn_prefill);
        }
    } else if (warp < kWarpVn) {
        // ---- state warps: thread j = v column j = TMEM lane j ----
        const int j = tid;
        const uint32_t lb = static_cast<uint32_t>(warp * 32) << 16;
        float* Srow = p.state + (bh * kD + j) * kD;  // S[j][0..127], 512 contiguous bytes
        auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
            return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, &g_err_gdn_prefill));
        };
        // the prologue stage is not read here: its arrivals are made at once
        __syncwarp();
        if (lane == 0) mbar_arrive(&ms->empty[1]);
        bool ok = true;
        for (int c = 0; c < nch; ++c) {
            const int s = c & 1;
            if (!wait_all(&ms->full[s], ch_use(c) & 1)) { ok = false; break; }
            const float gam = __expf(reinterpret_cast<const float*>(smem + s * kStage + kG)[kC - 1]);
            __syncwarp();
            if (lane == 0) mbar_arrive(&ms->empty[s]);
            if (c > 0) {
                if (!wait_all(&ms->ds_done, (c - 1) & 1)) { ok = false; break; }
                tc_fence_after();
            }
            // S_c -> S16_c (A operand of Y p1) and gam_c S_c (the update accumulates onto it)
#pragma unroll
            for (int cc = 0; cc < kD / 32; ++cc) {
                uint32_t r[32];
                if (c == 0) {
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const float4 x = reinterpret_cast<const float4*>(Srow + cc * 32)[q];
                        r[4 * q] = __float_as_uint(x.x);
                        r[4 * q + 1] = __float_as_uint(x.y);
                        r[4 * q + 2] = __float_as_uint(x.z);
                        r[4 * q + 3] = __float_as_uint(x.w);
                    }
                } else {
                    tmem_ld32(tmem + lb + kColS + cc * 32, r);
                    tmem_ld_wait();
                }
                uint32_t h16[16];
#pragma unroll
                for (int u = 0; u < 16; ++u)
                    h16[u] = Elem<T16>::pack2(__uint_as_float(r[2 * u]), __uint_as_float(r[2 * u + 1]));
                tmem_st16(tmem + lb + kColS16 + cc * 16, h16);
#pragma unroll
                for (int u = 0; u < 32; ++u) r[u] = __float_as_uint(__uint_as_float(r[u]) * gam);
                tmem_st32(tmem + lb + kColS + cc * 32, r);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ms->s_ready);
        }
        if (ok && wait_all(&ms->ds_done, (nch - 1) & 1)) {
            tc_fence_after();
#pragma unroll
            for (int cc = 0; cc < kD / 32; ++cc) {
                uint32_t r[32];
                tmem_ld32(tmem + lb + kColS + cc * 32, r);
                tmem_ld_wait();
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    reinterpret_cast<float4*>(Srow + cc * 32)[q] =
                        make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                    __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
            }
        }
    } else {
        // ---- Vn / output warps: thread j = v column j = TMEM lane j ----
        const int j = tid - kWarpVn * 32;
        const uint32_t lb = static_cast<uint32_t>((warp & 3) * 32) << 16;
        auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
            return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, &g_err_gdn_prefill));
        };
        // offsets of column j of a 128B-swizzled 64-row tile, by row mod 8 (row t adds 128 t)
        uint32_t uoff[8];
#pragma unroll
        for (int r = 0; r < 8; ++r)
            uoff[r] = (uint32_t)((j >> 6) * 8192 + ((((j & 63) >> 3) ^ r) << 4) + (j & 7) * 2);
        // Vn = U - y (y = the chain half of Y) and Vt = Vn * vdec into TMEM, then announced.
        // vdec_t = e^{gcs_last - gcs_t} (/ |k_t| with the fused pre-processing), from the prep pass.
        auto make_vn = [&](const uint8_t* stg, const uint32_t (&y)[64]) {
            const float* vdec = reinterpret_cast<const float*>(stg + kG + 512);
            uint32_t pv[32], pt[32];
#pragma unroll
            for (int t2 = 0; t2 < kC / 2; ++t2) {
                const int t = 2 * t2;
                const float u0 = Elem<T16>::to_f(*reinterpret_cast<const T16*>(stg + kU + uoff[t & 7] + t * 128));
                const float u1 =
                    Elem<T16>::to_f(*reinterpret_cast<const T16*>(stg + kU + uoff[(t + 1) & 7] + (t + 1) * 128));
                const float v0 = u0 - __uint_as_float(y[t]);
                const float v1 = u1 - __uint_as_float(y[t + 1]);
                pv[t2] = Elem<T16>::pack2(v0, v1);
                pt[t2] = Elem<T16>::pack2(v0 * vdec[t], v1 * vdec[t + 1]);
            }
            tmem_st32(tmem + lb + kColVn, pv);
            tmem_st32(tmem + lb + kColVt, pt);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ms->vn_ready);
        };
        auto load_y = [&](uint32_t col, uint32_t (&y)[64]) {
            tmem_ld32(tmem + lb + col, *reinterpret_cast<uint32_t(*)[32]>(&y[0]));
            tmem_ld32(tmem + lb + col + 32, *reinterpret_cast<uint32_t(*)[32]>(&y[32]));
            tmem_ld_wait();
        };
        bool ok = wait_all(&ms->full[1], 0) && wait_all(&ms->y_full[1], 0);
        if (ok) {  // prologue: Vn_0 = U_0 - W_0 S_0^T
            tc_fence_after();
            uint32_t y[64];
            load_y(kColY + 128 + 64, y);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ms->y_empty[1]);
            make_vn(smem + kStage, y);
            __syncwarp();
            if (lane == 0) mbar_arrive(&ms->empty[1]);
        }
        TOut* obase = static_cast<TOut*>(p.o) + ((size_t)seq.start * p.Hv + h) * kD + j;
        const size_t tstride = (size_t)p.Hv * kD;
        for (int c = 0; ok && c < nch; ++c) {
            const int s = c & 1;
            const uint32_t ycol = kColY + (c & 1) * 128;
            if (!wait_all(&ms->y_full[c & 1], ((c + 1) >> 1) & 1)) break;
            if (!wait_all(&ms->full[s], ch_use(c) & 1)) break;  // U_{c+1} and the decays
            tc_fence_after();
            const uint8_t* stg = smem + s * kStage;
            if (c + 1 < nch) {  // Vn_{c+1} = U_{c+1} - (Y_c columns 64-127)
                uint32_t y[64];
                load_y(ycol + 64, y);
                make_vn(stg, y);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&ms->empty[s]);
            uint32_t o[64];
            load_y(ycol, o);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ms->y_empty[c & 1]);
            // o_c[t][j] = scale * Y_c[j][t] for the chunk's tokens of this sequence
            const int nt = min(kC, seq.len - c * kC);
            TOut* op = obase + (size_t)c * kC * tstride;
#pragma unroll
            for (int t = 0; t < kC; ++t)
                if (t < nt) op[(size_t)t * tstride] = Elem<TOut>::from_f(p.scale * __uint_as_float(o[t]));
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
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

// Packed sequences: cu is the device [B+1] token-offset array and ntok its last entry; dense
// B x T: cu = null, ntok = B * T.  T is the (longest) sequence length.
template <typename T16, typename TOut>
int launch(const void* q, const void* k, const void* v, const float* g_log, const float* beta,
           float* state, void* o, int B, int T, int Hqk, int Hv, int head_map, float scale,
           void* ws, cudaStream_t stream, Fuse fuse, const int* cu, int ntok) {
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
    CUtensorMap tu, tm, tqt;
    if ((rc = make_tmap_3d(&tm, wsb + L.m, dt, 2, kC, kC, nbhc, 64, kC, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
    if ((rc = make_tmap_3d(&tu, wsb + L.u, dt, 2, kD, kC, nbhc, 64, kC, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
    if ((rc = make_tmap_3d(&tqt, wsb + L.qt, dt, 2, kD, kC, nbhc, 64, kC, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;

    PrepParams pp;
    pp.ws = wsb;
    pp.g_log = g_log;
    pp.beta = beta;
    pp.ws_u = L.u;
    pp.ws_aqk = L.aqk;
    pp.ws_gcs = L.gcs;
    pp.ws_vdec = L.vdec;
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
    k1<<<dim3(nch, Hv, B), prep::kThreads, prep::kAlloc, stream>>>(tq, tk, tv, tw, tu, ta, tm, tqt, pp);
    B200_TRY_CUDA(cudaGetLastError());

    ChainParams cp;
    cp.ws = wsb;
    cp.state = state;
    cp.o = o;
    cp.ws_gcs = L.gcs;
    cp.ws_vdec = L.vdec;
    cp.cu = cu;
    cp.ntok = ntok;
    cp.T = T;
    cp.Hqk = Hqk;
    cp.Hv = Hv;
    cp.nch = nch;
    cp.head_map = head_map;
    cp.scale = scale;
    auto k2 = gdn_chain_kernel<T16, TOut>;
    B200_TRY_CUDA(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, ch::kAlloc));
    // launched with programmatic stream serialisation: its prologue (barriers, TMEM) overlaps
    // the prep grid's last CTAs; its producer waits for the prep grid's results
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(Hv, B);
    cfg.blockDim = dim3(ch::kThreads);
    cfg.dynamicSmemBytes = ch::kAlloc;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    B200_TRY_CUDA(cudaLaunchKernelEx(&cfg, k2, tk, tqt, tw, ta, tm, tu, cp));
    count_launch(2);
    return cudaGetLastError() == cudaSuccess ? B200LAB_OK : B200LAB_ERR_CUDA;
}

template <typename T16>
int dispatch_out(int out_dtype, const void* q, const void* k, const void* v, const float* g,
                 const float* be, float* state, void* o, int B, int T, int Hqk, int Hv, int hm,
                 float scale, void* ws, cudaStream_t s, Fuse f, const int* cu, int ntok) {
    switch (out_dtype) {
        case B200LAB_F16:
            return launch<T16, __half>(q, k, v, g, be, state, o, B, T, Hqk, Hv, hm, scale, ws, s, f, cu, ntok);
        case B200LAB_BF16:
            return launch<T16, __nv_bfloat16>(q, k, v, g, be, state, o, B, T, Hqk, Hv, hm, scale, ws, s, f, cu,
                                              ntok);
        case B200LAB_F32:
            return launch<T16, float>(q, k, v, g, be, state, o, B, T, Hqk, Hv, hm, scale, ws, s, f, cu, ntok);
    }
    return B200LAB_ERR_UNSUPPORTED;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace
}  // namespace b200

B200_DEFINE_ERR_TAKER(gdn_prefill, b200::g_err_gdn_prefill)

extern "C" size_t gdn_prefill_sm100_workspace(int B, int T, int Hqk, int Hv, int dk, int dv) {
    (void)Hqk;
    (void)dk;
    (void)dv;
    if (B < 1 || T < 1 || Hv < 1) return 0;
    const size_t nch = ((size_t)T + b200::kC - 1) / b200::kC;
    return b200::ws_layout((size_t)B * Hv * nch).total;
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
    if (in_dtype == B200LAB_F32) return B200LAB_ERR_UNSUPPORTED;  // 16-bit operands only
    if (B > 65535 || Hv > 65535) return B200LAB_ERR_UNSUPPORTED;
    if (T == 0) return B200LAB_OK;
    if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(state, 16) ||
        !aligned(o, 16))
        return B200LAB_ERR_INVALID;
    const size_t need = gdn_prefill_sm100_workspace(B, T, Hqk, Hv, dk, dv);
    if (!workspace || ws_bytes < need || !aligned(workspace, 256)) return B200LAB_ERR_WORKSPACE;
    int rc = check_device_sm100();
    if (rc != B200LAB_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!cu) ntok = B * T;
    if (in_dtype == B200LAB_BF16)
        return dispatch_out<__nv_bfloat16>(out_dtype, q, k, v, g_log, beta, state, o, B, T, Hqk, Hv,
                                           head_map, scale, workspace, s, fuse, cu, ntok);
    return dispatch_out<__half>(out_dtype, q, k, v, g_log, beta, state, o, B, T, Hqk, Hv, head_map,
                                scale, workspace, s, fuse, cu, ntok);
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
