// gdn_decode.cu -- Gated DeltaNet single-token decode step for sm_100a.
//
// Reference semantics: the token-serial kernels of src/gdn_sm75.cu run with
// T = 1 (gdn_occ8_kernel, src/gdn_sm75.cu:722-789; gdn_occ_kernel :135-188):
//   g = exp(g_log); kv = S k; d = (v - g*kv)*beta; S = g*S + d k^T;
//   o = scale * S q,  per (sequence b, v-head h), state row c = v column.
//
// The step is memory-bound: the fp32 state (dv*dk*4 = 64 KiB per (b,h)) is
// read once and written once, everything else is < 2% of the bytes.  Layout
// in HBM is the reference's [B][Hv][dv][dk] with dk innermost, so a state row
// is 512 contiguous bytes = one warp x one float4 per lane: every load and
// store is a fully coalesced 128-bit access.  One CTA of 8 warps owns half a
// (b, h) (64 rows); each warp owns 8 rows and issues all 8 row loads before the
// first reduction.  Small CTAs keep 64 warps resident per SM and make the last
// partial wave short.  Loads and
// stores use the streaming (evict-first) cache policy: a step touches each
// state byte exactly once.
#include "common.cuh"
#include "errwords.h"

namespace b200 {
namespace {

__device__ int g_err_gdn_decode = 0;

constexpr int kD = 128;           // dk = dv
constexpr int kThreads = 256;
// 8 warps x 8 rows = 64 rows, half a (b, h) per CTA, for either state type (a 16-bit
// state with 16 rows a warp keeps more bytes in flight but leaves a 1.7-wave grid)
template <typename TS>
struct Rows {
    static constexpr int kPerWarp = 8;
    static constexpr int kCtasPerHead = kD / (kPerWarp * 8);
};

// Streaming loads / stores of four state entries (one lane's share of a row): 128-bit
// for an fp32 state, 64-bit for a 16-bit one.  asm volatile keeps a warp's row loads
// issued back to back, ahead of the first reduction that consumes them.
__device__ __forceinline__ float4 ld_stream(const float* p) {
    float4 v;
    asm volatile("ld.global.cs.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ void st_stream(float* p, float4 v) {
    asm volatile("st.global.cs.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w)
                 : "memory");
}
template <typename TS>
__device__ __forceinline__ float4 ld_stream(const TS* p) {
    uint32_t a, b;
    asm volatile("ld.global.cs.v2.b32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "l"(p));
    const TS* e0 = reinterpret_cast<const TS*>(&a);
    const TS* e1 = reinterpret_cast<const TS*>(&b);
    return make_float4(Elem<TS>::to_f(e0[0]), Elem<TS>::to_f(e0[1]), Elem<TS>::to_f(e1[0]),
                       Elem<TS>::to_f(e1[1]));
}
template <typename TS>
__device__ __forceinline__ void st_stream(TS* p, float4 v) {
    const uint32_t a = Elem<TS>::pack2(v.x, v.y), b = Elem<TS>::pack2(v.z, v.w);
    asm volatile("st.global.cs.v2.b32 [%0], {%1, %2};" ::"l"(p), "r"(a), "r"(b) : "memory");
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) x += __shfl_xor_sync(0xffffffffu, x, m);
    return x;
}

template <typename T>
__device__ __forceinline__ float4 load4(const T* p) {
    if constexpr (sizeof(T) == 4) {
        return *reinterpret_cast<const float4*>(p);
    } else {
        const uint2 raw = *reinterpret_cast<const uint2*>(p);
        const T* e = reinterpret_cast<const T*>(&raw);
        return make_float4(Elem<T>::to_f(e[0]), Elem<T>::to_f(e[1]), Elem<T>::to_f(e[2]),
                           Elem<T>::to_f(e[3]));
    }
}

// Fused pre-processing (gdn_decode_sm100_fused): q and k arrive raw and are L2-normalised
// here, x * rsqrt(sum x^2 + kNormEps) over dk; g_log and beta then carry the logits a and b,
// g = -exp(A_log[h]) * softplus(a + dt_bias[h]), beta = sigmoid(b).
struct Pre {
    const float* A_log;    // [Hv] or null (0)
    const float* dt_bias;  // [Hv] or null (0)
    int fused;
    // Continuous batching (gdn_decode_sm100_slots): sequence b's state is
    // state[slots[b]] of a pool of pool_size [Hv][dv][dk] states; slots[b] < 0 is padding
    // (skipped); slots[b] >= pool_size is reported as ERR_INVALID and skipped.
    const int* slots = nullptr;
    int pool_size = 0;
};
constexpr float kNormEps = 1e-6f;

__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

template <typename TIn, typename TOut, typename TS, bool kFused>
__global__ void __launch_bounds__(kThreads, 4) gdn_decode_kernel(
    const TIn* __restrict__ q, const TIn* __restrict__ k, const TIn* __restrict__ v,
    const float* __restrict__ g_log, const float* __restrict__ beta, TS* __restrict__ state,
    TOut* __restrict__ o, int Hqk, int Hv, int head_map, float scale, Pre pre) {
    constexpr int kRowsPerWarp = Rows<TS>::kPerWarp;
    constexpr int kCtasPerHead = Rows<TS>::kCtasPerHead;
    const int bh = blockIdx.x / kCtasPerHead;  // b * Hv + h
    const int b = bh / Hv;
    const int h = bh - b * Hv;
    const int hq = head_map == 0 ? h % Hqk : h / (Hv / Hqk);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x % kCtasPerHead) * (kRowsPerWarp * 8) + warp * kRowsPerWarp;
    // launched with programmatic stream serialisation (launch_step): nothing global is read or
    // written before the previous grid in the stream has completed; the next one may then be
    // scheduled onto the SMs this grid's last CTAs free
    grid_dependency_wait();
    allow_dependent_launch();

    size_t sh = (size_t)bh;  // state index of (b, h)
    if (pre.slots) {
        const int slot = pre.slots[b];
        if (slot < 0) return;  // padding entry: no state, no output (uniform over the CTA)
        if (slot >= pre.pool_size) {  // outside the pool: reported, never followed
            if (threadIdx.x == 0) atomicExch(&g_err_gdn_decode, B200LAB_ERR_INVALID);
            return;
        }
        sh = (size_t)slot * Hv + h;
    }
    TS* S = state + sh * kD * kD + (size_t)row0 * kD + 4 * lane;
    float4 s[kRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) s[r] = ld_stream(S + r * kD);

    const size_t qk_off = ((size_t)b * Hqk + hq) * kD + 4 * lane;
    float4 kk = load4(k + qk_off);
    float4 qq = load4(q + qk_off);
    float g, be;
    if constexpr (kFused) {
        const float kr = rsqrtf(warp_sum(kk.x * kk.x + kk.y * kk.y + kk.z * kk.z + kk.w * kk.w) + kNormEps);
        const float qr = rsqrtf(warp_sum(qq.x * qq.x + qq.y * qq.y + qq.z * qq.z + qq.w * qq.w) + kNormEps);
        kk = make_float4(kk.x * kr, kk.y * kr, kk.z * kr, kk.w * kr);
        qq = make_float4(qq.x * qr, qq.y * qr, qq.z * qr, qq.w * qr);
        const float a = g_log[bh] + (pre.dt_bias ? pre.dt_bias[h] : 0.f);
        const float decay = pre.A_log ? __expf(pre.A_log[h]) : 1.f;
        g = __expf(-decay * softplus(a));
        be = 1.f / (1.f + __expf(-beta[bh]));
    } else {
        g = expf(g_log[bh]);
        be = beta[bh];
    }
    const float vr = lane < kRowsPerWarp ? Elem<TIn>::to_f(v[(size_t)bh * kD + row0 + lane]) : 0.f;
    static_assert(kRowsPerWarp <= 32, "one v entry per lane");

    float out = 0.f;
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
        float kv = s[r].x * kk.x + s[r].y * kk.y + s[r].z * kk.z + s[r].w * kk.w;
        kv = warp_sum(kv);
        const float vv = __shfl_sync(0xffffffffu, vr, r);
        const float d = (vv - g * kv) * be;
        s[r].x = g * s[r].x + kk.x * d;
        s[r].y = g * s[r].y + kk.y * d;
        s[r].z = g * s[r].z + kk.z * d;
        s[r].w = g * s[r].w + kk.w * d;
        float od = s[r].x * qq.x + s[r].y * qq.y + s[r].z * qq.z + s[r].w * qq.w;
        od = warp_sum(od);
        if (lane == r) out = od * scale;
        st_stream(S + r * kD, s[r]);
    }
    if (lane < kRowsPerWarp) o[(size_t)bh * kD + row0 + lane] = Elem<TOut>::from_f(out);
}

// ---------------------------------------------------------------------------
// 16-bit state: a 256-byte row is one 16-byte load for each of 16 lanes, so a warp
// works on two rows at a time (lanes 0-15 / 16-31) with 16-lane reductions, and each
// lane converts 8 entries a load.  CTA = 8 warps x 8 rows = half a (b, h).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
    uint4 v;
    asm volatile("ld.global.cs.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ void st_stream16(void* p, uint4 v) {
    asm volatile("st.global.cs.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ float half_warp_sum(float x) {
#pragma unroll
    for (int m = 8; m > 0; m >>= 1) x += __shfl_xor_sync(0xffffffffu, x, m);
    return x;
}
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&x)[8]) {
    if constexpr (sizeof(T) == 4) {
        const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    } else {
        const uint4 raw = *reinterpret_cast<const uint4*>(p);
        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int u = 0; u < 8; ++u) x[u] = Elem<T>::to_f(e[u]);
    }
}

template <typename TIn, typename TOut, typename TS>
__global__ void __launch_bounds__(kThreads, 4) gdn_decode16_kernel(
    const TIn* __restrict__ q, const TIn* __restrict__ k, const TIn* __restrict__ v,
    const float* __restrict__ g_log, const float* __restrict__ beta, TS* __restrict__ state,
    TOut* __restrict__ o, int Hqk, int Hv, int head_map, float scale) {
    // one CTA per (sequence, v-head): 8 warps x 16 rows, as 8 pairs (more bytes in flight a
    // warp and fewer CTAs to start than 2 CTAs of 8-row warps: 24.7 vs 26.6 us a C4 step)
    constexpr int kRows = 16;
    const int bh = blockIdx.x;
    const int b = bh / Hv;
    const int h = bh - b * Hv;
    const int hq = head_map == 0 ? h % Hqk : h / (Hv / Hqk);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int half = lane >> 4, l16 = lane & 15;
    const int row0 = warp * kRows;
    grid_dependency_wait();  // as in gdn_decode_kernel
    allow_dependent_launch();
    TS* S = state + (size_t)bh * kD * kD + (size_t)(row0 + half) * kD + 8 * l16;
    uint4 raw[kRows / 2];
#pragma unroll
    for (int i = 0; i < kRows / 2; ++i) raw[i] = ld_stream16(S + (size_t)(2 * i) * kD);
    const size_t qk_off = ((size_t)b * Hqk + hq) * kD + 8 * l16;
    float kk[8], qq[8];
    load8(k + qk_off, kk);
    load8(q + qk_off, qq);
    const float g = expf(g_log[bh]);
    const float be = beta[bh];
    const float vr = lane < kRows ? Elem<TIn>::to_f(v[(size_t)bh * kD + row0 + lane]) : 0.f;
#pragma unroll
    for (int i = 0; i < kRows / 2; ++i) {
        const TS* e = reinterpret_cast<const TS*>(&raw[i]);
        float sv[8];
        float kv = 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            sv[u] = Elem<TS>::to_f(e[u]);
            kv = fmaf(sv[u], kk[u], kv);
        }
        kv = half_warp_sum(kv);
        const float vv = __shfl_sync(0xffffffffu, vr, 2 * i + half);
        const float d = (vv - g * kv) * be;
        float od = 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            sv[u] = fmaf(g, sv[u], kk[u] * d);
            od = fmaf(sv[u], qq[u], od);
        }
        od = half_warp_sum(od);
        uint4 w;
        w.x = Elem<TS>::pack2(sv[0], sv[1]);
        w.y = Elem<TS>::pack2(sv[2], sv[3]);
        w.z = Elem<TS>::pack2(sv[4], sv[5]);
        w.w = Elem<TS>::pack2(sv[6], sv[7]);
        st_stream16(S + (size_t)(2 * i) * kD, w);
        if (l16 == 0) o[(size_t)bh * kD + row0 + 2 * i + half] = Elem<TOut>::from_f(od * scale);
    }
}

// One decode step as a programmatic dependent launch: consecutive steps on a stream (each
// waits for the previous grid before touching memory) then start without the launch gap.
template <typename Kern, typename... Args>
int launch_step(Kern kern, int grid, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, args...) != cudaSuccess) return B200LAB_ERR_CUDA;
    count_launch(1);
    return cudaGetLastError() == cudaSuccess ? B200LAB_OK : B200LAB_ERR_CUDA;
}

template <typename TIn, typename TOut, typename TS>
int launch(const void* q, const void* k, const void* v, const float* g_log, const float* beta,
           void* state, void* o, int B, int Hqk, int Hv, int head_map, float scale,
           cudaStream_t st, Pre pre) {
    if constexpr (sizeof(TS) == 2) {
        return launch_step(gdn_decode16_kernel<TIn, TOut, TS>, B * Hv, st, static_cast<const TIn*>(q),
                           static_cast<const TIn*>(k), static_cast<const TIn*>(v), g_log, beta,
                           static_cast<TS*>(state), static_cast<TOut*>(o), Hqk, Hv, head_map, scale);
    }
    // the fused pre-processing is its own instantiation: the plain step keeps its registers
    auto kern = pre.fused ? gdn_decode_kernel<TIn, TOut, TS, true> : gdn_decode_kernel<TIn, TOut, TS, false>;
    return launch_step(kern, B * Hv * Rows<TS>::kCtasPerHead, st, static_cast<const TIn*>(q),
                       static_cast<const TIn*>(k), static_cast<const TIn*>(v), g_log, beta,
                       static_cast<TS*>(state), static_cast<TOut*>(o), Hqk, Hv, head_map, scale, pre);
}

template <typename TIn, typename TS>
int dispatch_out(int out_dtype, const void* q, const void* k, const void* v, const float* g_log,
                 const float* beta, void* state, void* o, int B, int Hqk, int Hv, int head_map,
                 float scale, cudaStream_t st, Pre pre) {
    switch (out_dtype) {
        case B200LAB_F16:
            return launch<TIn, __half, TS>(q, k, v, g_log, beta, state, o, B, Hqk, Hv, head_map, scale, st, pre);
        case B200LAB_BF16:
            return launch<TIn, __nv_bfloat16, TS>(q, k, v, g_log, beta, state, o, B, Hqk, Hv, head_map,
                                                  scale, st, pre);
        case B200LAB_F32:
            return launch<TIn, float, TS>(q, k, v, g_log, beta, state, o, B, Hqk, Hv, head_map, scale, st, pre);
    }
    return B200LAB_ERR_UNSUPPORTED;
}

template <typename TS>
int dispatch_in(int in_dtype, int out_dtype, const void* q, const void* k, const void* v,
                const float* g_log, const float* beta, void* state, void* o, int B, int Hqk, int Hv,
                int head_map, float scale, cudaStream_t st, Pre pre = Pre{nullptr, nullptr, 0}) {
    switch (in_dtype) {
        case B200LAB_F16:
            return dispatch_out<__half, TS>(out_dtype, q, k, v, g_log, beta, state, o, B, Hqk, Hv,
                                            head_map, scale, st, pre);
        case B200LAB_BF16:
            return dispatch_out<__nv_bfloat16, TS>(out_dtype, q, k, v, g_log, beta, state, o, B, Hqk,
                                                   Hv, head_map, scale, st, pre);
        default:
            return dispatch_out<float, TS>(out_dtype, q, k, v, g_log, beta, state, o, B, Hqk, Hv,
                                           head_map, scale, st, pre);
    }
}

// argument checks shared by both entries (state alignment checked by the caller)
int check_args(const void* q, const void* k, const void* v, const float* g_log, const float* beta,
               const void* state, const void* o, int B, int Hqk, int Hv, int dk, int dv, int head_map,
               int in_dtype, int out_dtype) {
    if (!q || !k || !v || !g_log || !beta || !state || !o) return B200LAB_ERR_INVALID;
    if (B < 1 || Hqk < 1 || Hv < 1 || dk < 1 || dv < 1) return B200LAB_ERR_INVALID;
    if (head_map != 0 && head_map != 1) return B200LAB_ERR_INVALID;
    if (head_map == 1 && Hv % Hqk != 0) return B200LAB_ERR_INVALID;
    if (in_dtype < B200LAB_F16 || in_dtype > B200LAB_F32) return B200LAB_ERR_INVALID;
    if (out_dtype < B200LAB_F16 || out_dtype > B200LAB_F32) return B200LAB_ERR_INVALID;
    if (dk != 128 || dv != 128) return B200LAB_ERR_UNSUPPORTED;
    if ((long long)B * Hv > 0x7fffffffLL) return B200LAB_ERR_UNSUPPORTED;
    return B200LAB_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace
}  // namespace b200

B200_DEFINE_ERR_TAKER(gdn_decode, b200::g_err_gdn_decode)

extern "C" int gdn_decode_sm100(const void* q, const void* k, const void* v, const float* g_log,
                                const float* beta, float* state, void* o, int B, int Hqk, int Hv,
                                int dk, int dv, int head_map, float scale, int in_dtype,
                                int out_dtype, void* stream) {
    using namespace b200;
    int rc = check_args(q, k, v, g_log, beta, state, o, B, Hqk, Hv, dk, dv, head_map, in_dtype, out_dtype);
    if (rc != B200LAB_OK) return rc;
    const uintptr_t in_align = in_dtype == B200LAB_F32 ? 16 : 8;
    if (!aligned(q, in_align) || !aligned(k, in_align) || !aligned(state, 16))
        return B200LAB_ERR_INVALID;
    rc = check_device_sm100();
    if (rc != B200LAB_OK) return rc;
    return dispatch_in<float>(in_dtype, out_dtype, q, k, v, g_log, beta, state, o, B, Hqk, Hv, head_map,
                              scale, static_cast<cudaStream_t>(stream));
}

extern "C" int gdn_decode_sm100_state16(const void* q, const void* k, const void* v,
                                        const float* g_log, const float* beta, void* state,
                                        int state_dtype, void* o, int B, int Hqk, int Hv, int dk,
                                        int dv, int head_map, float scale, int in_dtype,
                                        int out_dtype, void* stream) {
    using namespace b200;
    int rc = check_args(q, k, v, g_log, beta, state, o, B, Hqk, Hv, dk, dv, head_map, in_dtype, out_dtype);
    if (rc != B200LAB_OK) return rc;
    if (state_dtype != B200LAB_F16 && state_dtype != B200LAB_BF16) return B200LAB_ERR_INVALID;
    // 16-byte loads of q, k and the state rows
    if (!aligned(q, 16) || !aligned(k, 16) || !aligned(state, 16)) return B200LAB_ERR_INVALID;
    rc = check_device_sm100();
    if (rc != B200LAB_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return state_dtype == B200LAB_F16
               ? dispatch_in<__half>(in_dtype, out_dtype, q, k, v, g_log, beta, state, o, B, Hqk, Hv,
                                     head_map, scale, st)
               : dispatch_in<__nv_bfloat16>(in_dtype, out_dtype, q, k, v, g_log, beta, state, o, B,
                                            Hqk, Hv, head_map, scale, st);
}

extern "C" int gdn_decode_sm100_fused(const void* q, const void* k, const void* v, const float* a,
                                      const float* b, const float* A_log, const float* dt_bias,
                                      float* state, void* o, int B, int Hqk, int Hv, int dk, int dv,
                                      int head_map, float scale, int in_dtype, int out_dtype,
                                      void* stream) {
    using namespace b200;
    int rc = check_args(q, k, v, a, b, state, o, B, Hqk, Hv, dk, dv, head_map, in_dtype, out_dtype);
    if (rc != B200LAB_OK) return rc;
    const uintptr_t in_align = in_dtype == B200LAB_F32 ? 16 : 8;
    if (!aligned(q, in_align) || !aligned(k, in_align) || !aligned(state, 16))
        return B200LAB_ERR_INVALID;
    rc = check_device_sm100();
    if (rc != B200LAB_OK) return rc;
    return dispatch_in<float>(in_dtype, out_dtype, q, k, v, a, b, state, o, B, Hqk, Hv, head_map, scale,
                              static_cast<cudaStream_t>(stream), Pre{A_log, dt_bias, 1});
}

extern "C" int gdn_decode_sm100_slots(const void* q, const void* k, const void* v, const float* g_log,
                                      const float* beta, float* state_pool, const int* slots, int pool_size,
                                      void* o, int B, int Hqk, int Hv, int dk, int dv, int head_map,
                                      float scale, int in_dtype, int out_dtype, void* stream) {
    using namespace b200;
    if (!slots || pool_size < 1) return B200LAB_ERR_INVALID;
    int rc = check_args(q, k, v, g_log, beta, state_pool, o, B, Hqk, Hv, dk, dv, head_map, in_dtype,
                        out_dtype);
    if (rc != B200LAB_OK) return rc;
    const uintptr_t in_align = in_dtype == B200LAB_F32 ? 16 : 8;
    if (!aligned(q, in_align) || !aligned(k, in_align) || !aligned(state_pool, 16))
        return B200LAB_ERR_INVALID;
    rc = check_device_sm100();
    if (rc != B200LAB_OK) return rc;
    Pre pre{nullptr, nullptr, 0};
    pre.slots = slots;
    pre.pool_size = pool_size;
    return dispatch_in<float>(in_dtype, out_dtype, q, k, v, g_log, beta, state_pool, o, B, Hqk, Hv,
                              head_map, scale, static_cast<cudaStream_t>(stream), pre);
}
