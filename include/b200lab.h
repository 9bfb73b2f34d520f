/*
 * b200lab.h -- C ABI of the B200-native (sm_100a) attention and Gated
 * DeltaNet kernels.
 *
 * The reference (cookys/turing-sm75) has no library; its drop-in surface is
 * the raw __global__ signatures called from each binary's main() and the
 * per-binary CLI.  Each entry point below replaces one of those kernel
 * families; the comment on each names the reference interface (file:line).
 *
 * Conventions shared by every entry point:
 *   - All tensor pointers are DEVICE pointers owned by the caller.  Nothing
 *     is allocated; scratch space, where an entry needs it, is passed in
 *     through (workspace, ws_bytes) and sized by the matching *_workspace()
 *     query.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream).  Each call enqueues its launches on that stream and returns
 *     without synchronising.  The caller selects the device (cudaSetDevice).
 *   - The return value is a status code (B200LAB_OK or a negative error);
 *     the library never prints and never exits.  Arguments are validated
 *     before anything is launched, so an error return means nothing ran
 *     (except B200LAB_ERR_CUDA, which reports a failed launch).
 *   - Device-side bounded waits that run out set a device error word instead
 *     of hanging; b200lab_device_status() reads and clears it.
 *   - Entry points are stateless and re-entrant apart from that error word
 *     (and attn_fwd_sm100_host's per-thread copy streams, described there).
 */
#ifndef B200LAB_H
#define B200LAB_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define B200LAB_OK               0
#define B200LAB_ERR_INVALID     -1  /* null pointer or inconsistent shape     */
#define B200LAB_ERR_UNSUPPORTED -2  /* well-formed but not built (e.g. D=96)  */
#define B200LAB_ERR_CUDA        -3  /* a CUDA runtime call / launch failed    */
#define B200LAB_ERR_TIMEOUT     -4  /* a device-side bounded wait ran out     */
#define B200LAB_ERR_WORKSPACE   -5  /* workspace missing or too small         */
#define B200LAB_ERR_DEVICE      -6  /* current device is not sm_100 (B200)    */

/* ---- element types ----------------------------------------------------- */
#define B200LAB_F16  0
#define B200LAB_BF16 1
#define B200LAB_F32  2

/* ---- softmax attention forward ------------------------------------------
 * Replaces flash_attn_sm75_wmma<D> / flash_attn_sm75_ffma<D>
 * (src/attn_sm75.cu:107-112, 239-244) and their launchers launch_wmma /
 * launch_ffma (src/attn_sm75.cu:421-440):
 *   (const half* Q, const half* K, const half* V, half* O, int S,
 *    float scale, int causal), grid (ceil(S/16), B*H).
 * Generalised with GQA (Hkv divides Hq; q-head h reads kv-head h/(Hq/Hkv)),
 * separate query / key lengths and a bf16 variant.
 *   Q, O : [B][Hq ][Sq ][D]  dtype (F16 or BF16)
 *   K, V : [B][Hkv][Skv][D]  dtype
 *   D    : 64, 128 or 256.  fp32 accumulation; O = softmax(scale*Q K^T [+mask]) V.
 *          (D = 256 runs the kernel of attn_gated_fwd_sm100 without a gate; it
 *          splits no key range and leaves the workspace unused.)
 *   causal: key j is visible to query i iff j <= i + (Skv - Sq); with
 *           Sq == Skv this is the reference's k <= q (src/attn_sm75.cu:69).
 *           A query row that sees no key is written as 0 (the reference's
 *           l == 0 rule, src/attn_sm75.cu:372).
 *   Base pointers must be 16-byte aligned.
 *   workspace: may be NULL when attn_fwd_sm100_workspace() returns 0. */
int attn_fwd_sm100(const void* Q, const void* K, const void* V, void* O,
                   int B, int Hq, int Hkv, int Sq, int Skv, int D,
                   float scale, int causal, int dtype,
                   void* workspace, size_t ws_bytes, void* stream);
size_t attn_fwd_sm100_workspace(int B, int Hq, int Hkv, int Sq, int Skv, int D,
                                int causal);

/* Host-buffer form of attn_fwd_sm100 (no counterpart in the reference, whose
 * main() copies whole tensors in, launches, and copies O back, serially,
 * src/attn_sm75.cu:404, 489-497): Qh, Kh, Vh, Oh are HOST buffers in the same
 * layouts (pinned memory lets the copies overlap), Qd, Kd, Vd, Od caller-owned
 * device buffers of the full sizes.  The (batch, kv-head) units are cut into
 * about eight contiguous chunks; chunk i+1 is copied in while chunk i is
 * computed and chunk i-1 copied out (two internal streams, joined back into
 * `stream` before return; no device memory is allocated).  The two streams and
 * their events are created on a host thread's first call for a device and kept
 * until that thread exits; calls from one thread on one device share them, so
 * their copies run in call order.  Oh is complete once
 * `stream` reaches the point of the call.  Same arguments and status codes as
 * attn_fwd_sm100, no workspace (no key splits). */
int attn_fwd_sm100_host(const void* Qh, const void* Kh, const void* Vh, void* Oh,
                        void* Qd, void* Kd, void* Vd, void* Od,
                        int B, int Hq, int Hkv, int Sq, int Skv, int D,
                        float scale, int causal, int dtype, void* stream);

/* Packed variable-length sequences (the cu_seqlens convention serving callers
 * use; no counterpart in the reference, whose batches are dense):
 *   Q, O : [total_q][Hq][D] token-major; K, V : [total_k][Hkv][D]
 *   cu_seqlens_q, cu_seqlens_k : [B+1] device int32 prefix sums; sequence b is
 *   tokens [cu[b], cu[b+1]) of each; max_seqlen_q bounds the grid.
 *   Causal is aligned per sequence: key j visible to query i iff
 *   j <= i + (Skv_b - Sq_b).  D = 64 or 128; no workspace (no key splits).
 *   The kernel checks the offsets before using them: a sequence outside the
 *   buffers or longer than max_seqlen_q is skipped and b200lab_device_status()
 *   then returns B200LAB_ERR_INVALID. */
int attn_fwd_sm100_varlen(const void* Q, const void* K, const void* V, void* O,
                          const int* cu_seqlens_q, const int* cu_seqlens_k,
                          int max_seqlen_q, int total_q, int total_k, int B, int Hq,
                          int Hkv, int D, float scale, int causal, int dtype, void* stream);

/* Gated softmax attention, head dim 256: O = softmax(scale*Q K^T [+mask]) V *
 * sigmoid(G), the gate applied elementwise after the softmax.  No counterpart
 * in the reference, which builds D = 64/128 only; this is the model layer its
 * notes describe (24 q-heads / 4 kv-heads, head dim 256, gate after softmax,
 * docs/qwen38-27b.md:13), with the same softmax semantics as attn_fwd_sm100.
 *   Q, G, O : [B][Hq][Sq][256]; K, V : [B][Hkv][Skv][256]; G may be NULL (no
 *   gate).  D must be 256.  16-byte aligned pointers.  No workspace. */
int attn_gated_fwd_sm100(const void* Q, const void* K, const void* V, const void* G,
                         void* O, int B, int Hq, int Hkv, int Sq, int Skv, int D,
                         float scale, int causal, int dtype, void* stream);

/* ---- Gated DeltaNet chunked prefill --------------------------------------
 * Replaces the chunked GDN kernels gdn_wmma_kernel (src/gdn_sm75.cu:361-369)
 * and gdn_prep_kernel + gdn_apply_kernel (src/gdn_sm75.cu:896-905, 981-992):
 *   (const float* q, k, v, g_log, beta, float* state, float* out, int T,
 *    float scale) with Sv=128, Hq=16, Hv=48 compiled in.
 * Same recurrence (src/gdn_sm75.cu:6-11): per token
 *   g = exp(g_log); kv = S k; d = (v - g*kv)*beta; S = g*S + d k^T;
 *   o = scale * S q
 * computed by the chunked (WY/UT) algebra with chunk 64.
 *   q, k  : [B][T][Hqk][dk]  in_dtype (F16, BF16 or F32)
 *   v     : [B][T][Hv ][dv]  in_dtype
 *   g_log, beta : [B][T][Hv] fp32
 *   state : [B][Hv][dv][dk] fp32, read and updated in place; element
 *           state[c*dk + i] multiplies k[i] (the reference's layout,
 *           src/gdn_sm75.cu:1094)
 *   o     : [B][T][Hv][dv]  out_dtype (F16, BF16 or F32)
 *   head_map: 0 -> v-head h reads q/k head h % Hqk (the reference,
 *             src/gdn_sm75.cu:1083); 1 -> h / (Hv/Hqk).
 *   dk = dv = 128.  workspace: gdn_prefill_sm100_workspace_ex(..., in_dtype)
 *   bytes (gdn_prefill_sm100_workspace() for 16-bit inputs).  fp32 q, k, v
 *   (the reference kernels' const float*) are converted once to bf16 copies in
 *   the workspace; the tensor-core operands are 16-bit for every in_dtype.
 *   With few sequences x v-heads (fewer state-pass CTAs than SMs, as on each GPU
 *   of a multi-GPU split) the chunk chain is cut into segments that run side by
 *   side and are then linked (two more kernels); the queried size includes their
 *   buffers.  Any workspace of at least gdn_prefill_sm100_workspace_min() bytes
 *   is accepted: one too small for the segment buffers runs the unsegmented
 *   chain (same results up to rounding). */
int gdn_prefill_sm100(const void* q, const void* k, const void* v,
                      const float* g_log, const float* beta, float* state, void* o,
                      int B, int T, int Hqk, int Hv, int dk, int dv, int head_map,
                      float scale, int in_dtype, int out_dtype,
                      void* workspace, size_t ws_bytes, void* stream);
size_t gdn_prefill_sm100_workspace(int B, int T, int Hqk, int Hv, int dk, int dv);
/* Workspace for a given in_dtype: the 16-bit size plus, for B200LAB_F32, the
 * bf16 copies of q, k, v (B*T*(2*Hqk + Hv)*dk*2 bytes, rounded up).  Packed
 * sequences (the varlen entries) use B and max_seqlen, as for the 16-bit size. */
size_t gdn_prefill_sm100_workspace_ex(int B, int T, int Hqk, int Hv, int dk, int dv, int in_dtype);
/* The smallest workspace the prefill entries accept (the chunk items, plus the
 * fp32 copies for B200LAB_F32 inputs): the unsegmented chain. */
size_t gdn_prefill_sm100_workspace_min(int B, int T, int Hqk, int Hv, int dk, int dv, int in_dtype);

/* Packed variable-length sequences (no counterpart in the reference, whose
 * prefill runs one sequence, src/gdn_sm75.cu:1246-1412): q, k [total][Hqk][dk],
 * v, o [total][Hv][dv], g_log, beta [total][Hv]; cu_seqlens device int32 [B+1]
 * (sequence b is tokens [cu[b], cu[b+1]), total_tokens = cu[B]); state
 * [B][Hv][dv][dk], one per sequence, updated in place (an empty sequence keeps
 * its state).  Chunks start at each sequence's first token, so sequence b's
 * outputs and state are those of a B = 1 call on it alone.  Workspace:
 * gdn_prefill_sm100_workspace(B, max_seqlen, ...).  The kernels check the
 * offsets before using them: a sequence outside [0, total_tokens) or longer
 * than max_seqlen is skipped and b200lab_device_status() then returns
 * B200LAB_ERR_INVALID. */
int gdn_prefill_sm100_varlen(const void* q, const void* k, const void* v,
                             const float* g_log, const float* beta, float* state, void* o,
                             const int* cu_seqlens, int max_seqlen, int total_tokens,
                             int B, int Hqk, int Hv, int dk, int dv, int head_map,
                             float scale, int in_dtype, int out_dtype,
                             void* workspace, size_t ws_bytes, void* stream);

/* ---- Gated DeltaNet chunked prefill without any allocation ----------------
 * No counterpart in the reference: it has no library, so nothing there
 * allocates on a caller's behalf.  This entry is for callers that cannot call
 * cudaMalloc or provide a workspace -- e.g. a host framework whose graph
 * allocator plans every buffer ahead of time and hands an operator only its
 * inputs and outputs, or a serving loop that must not hit cudaMalloc's
 * implicit device-wide synchronisation.
 * Same arguments and results as gdn_prefill_sm100, minus the workspace: the
 * scratch is a file-scope device array of B200LAB_NOALLOC_SCRATCH_BYTES
 * (64 MiB) that every GPU loading the prefill kernels holds until the process
 * exits.  A problem whose gdn_prefill_sm100_workspace_min() exceeds that size is
 * rejected with B200LAB_ERR_WORKSPACE before anything is launched (the
 * segmented chain runs when gdn_prefill_sm100_workspace_ex() fits; about
 * 50 KB per (sequence, v-head, 64-token chunk): B*Hv*ceil(T/64) <= 1344,
 * e.g. Hv=48 up to T=1792, Hv=32 up to T=2688).
 * Every call looks up the array's device address with the caller's device
 * current; the first call on a device also loads the library's kernels there,
 * so make that first call before any stream capture.  All calls on a device share the one array, so calls that overlap
 * on the GPU (other streams, other host threads) race and must be
 * serialised by the caller.  Nothing in the scratch needs to start at zero:
 * the preparation kernel writes every byte the state kernel reads. */
#define B200LAB_NOALLOC_SCRATCH_BYTES (64u << 20)
int gdn_prefill_sm100_noalloc(const void* q, const void* k, const void* v,
                              const float* g_log, const float* beta, float* state,
                              void* o, int B, int T, int Hqk, int Hv, int dk, int dv,
                              int head_map, float scale, int in_dtype, int out_dtype,
                              void* stream);

/* The prefill with the model's pre-processing fused in (no C entry of the
 * reference corresponds; the steps either side of the path in the llama.cpp
 * graph it targets, docs/ggml-turing.md:13-17), same conventions as
 * gdn_decode_sm100_fused: q, k raw, L2-normalised over dk in the kernels
 * (x * rsqrt(sum x^2 + 1e-6)); a, b : [B][T][Hv] fp32 logits,
 * g_log = -exp(A_log[h]) * softplus(a + dt_bias[h]), beta = sigmoid(b);
 * A_log, dt_bias : [Hv] fp32 or NULL.  Workspace as gdn_prefill_sm100. */
int gdn_prefill_sm100_fused(const void* q, const void* k, const void* v,
                            const float* a, const float* b, const float* A_log,
                            const float* dt_bias, float* state, void* o, int B, int T,
                            int Hqk, int Hv, int dk, int dv, int head_map, float scale,
                            int in_dtype, int out_dtype, void* workspace, size_t ws_bytes,
                            void* stream);
/* The same with packed sequences (cu_seqlens, as gdn_prefill_sm100_varlen):
 * raw q, k [total][Hqk][dk], logits a, b [total][Hv]. */
int gdn_prefill_sm100_fused_varlen(const void* q, const void* k, const void* v,
                                   const float* a, const float* b,
                                   const float* A_log, const float* dt_bias,
                                   float* state, void* o, const int* cu_seqlens,
                                   int max_seqlen, int total_tokens, int B, int Hqk, int Hv,
                                   int dk, int dv, int head_map, float scale,
                                   int in_dtype, int out_dtype,
                                   void* workspace, size_t ws_bytes, void* stream);

/* ---- Gated DeltaNet single-token decode ----------------------------------
 * Replaces the token-serial kernels with T = 1, e.g. gdn_occ8_kernel
 * (src/gdn_sm75.cu:722-730) and gdn_occ_kernel (src/gdn_sm75.cu:135-145),
 * batched over B sequences.  Same per-token math as gdn_prefill_sm100.
 *   q, k : [B][Hqk][dk] in_dtype;  v : [B][Hv][dv] in_dtype
 *   g_log, beta : [B][Hv] fp32;  state : [B][Hv][dv][dk] fp32 in place
 *   o : [B][Hv][dv] out_dtype.   dk = dv = 128. */
int gdn_decode_sm100(const void* q, const void* k, const void* v,
                     const float* g_log, const float* beta, float* state, void* o,
                     int B, int Hqk, int Hv, int dk, int dv, int head_map,
                     float scale, int in_dtype, int out_dtype, void* stream);

/* The decode step with the model's pre-processing fused in (the steps either
 * side of the path in the llama.cpp graph the reference targets,
 * docs/ggml-turing.md:13-17; no C entry of the reference corresponds):
 *   q, k raw; each is L2-normalised over dk in the kernel,
 *       x * rsqrt(sum x^2 + 1e-6);
 *   a, b : [B][Hv] fp32 logits; g_log = -exp(A_log[h]) * softplus(a + dt_bias[h])
 *       (softplus(x) = x for x > 20), beta = sigmoid(b);
 *   A_log, dt_bias : [Hv] fp32, either may be NULL (taken as 0).
 * Otherwise as gdn_decode_sm100 (fp32 state in place). */
int gdn_decode_sm100_fused(const void* q, const void* k, const void* v,
                           const float* a, const float* b, const float* A_log,
                           const float* dt_bias, float* state, void* o, int B, int Hqk,
                           int Hv, int dk, int dv, int head_map, float scale, int in_dtype,
                           int out_dtype, void* stream);

/* The decode step for continuous batching (no C entry of the reference
 * corresponds; the paged batching serving callers need): the states live in a
 * pool [pool_size][Hv][dv][dk] fp32 and sequence b uses state_pool[slots[b]]
 * (slots: B device ints); slots[b] < 0 marks a padding entry, whose state and
 * output are not touched; slots[b] >= pool_size is skipped the same way and
 * b200lab_device_status() then returns B200LAB_ERR_INVALID.  Otherwise as
 * gdn_decode_sm100. */
int gdn_decode_sm100_slots(const void* q, const void* k, const void* v,
                           const float* g_log, const float* beta, float* state_pool,
                           const int* slots, int pool_size, void* o, int B, int Hqk,
                           int Hv, int dk, int dv, int head_map, float scale,
                           int in_dtype, int out_dtype, void* stream);

/* The same decode step with a 16-bit recurrent state in HBM (state_dtype
 * B200LAB_F16 or B200LAB_BF16; [B][Hv][dv][dk], updated in place; q, k and
 * state 16-byte aligned): half the bytes of the fp32 step,
 * which is bound by them.  The
 * update is done in fp32 registers and rounded once per step on the store.
 * No C entry of the reference corresponds; the reference's own kernels keep
 * the state in fp16 within a launch (gdn_smem_kernel, src/gdn_sm75.cu:95-133;
 * gdn_wmma_kernel, src/gdn_sm75.cu:378, 543-573), which is the precision
 * precedent.  fp16 keeps 3 more mantissa bits than bf16: prefer it unless the
 * state can exceed 65504 in magnitude. */
int gdn_decode_sm100_state16(const void* q, const void* k, const void* v,
                             const float* g_log, const float* beta, void* state,
                             int state_dtype, void* o, int B, int Hqk, int Hv, int dk,
                             int dv, int head_map, float scale, int in_dtype,
                             int out_dtype, void* stream);

/* ---- utilities ----------------------------------------------------------- */
/* Message for a status code (static storage). */
const char* b200lab_strerror(int status);
/* Synchronises `stream`, then returns B200LAB_ERR_TIMEOUT (and clears the
 * flag) if any kernel of this library on the current device gave up a
 * bounded wait since the last call, B200LAB_ERR_CUDA on a CUDA error, else
 * B200LAB_OK.  The reference's equivalent is CUDA_CHECK -> exit(1)
 * (src/attn_sm75.cu:40-48); this library reports instead of exiting. */
int b200lab_device_status(void* stream);
/* Failure-path self-test (no counterpart in the reference): launches on
 * `stream` a one-thread kernel whose bounded wait is on a barrier that nothing
 * completes, so it gives up after the wait limit (1 s of GPU time) and records
 * B200LAB_ERR_TIMEOUT, exactly as a kernel of this library does when a
 * partner it waits for never arrives; the next b200lab_device_status() returns
 * that status and the context stays usable.  Nothing faults or traps.  Returns
 * the launch status. */
int b200lab_watchdog_selftest(void* stream);
/* Library version, major*10000 + minor*100 + patch. */
int b200lab_version(void);
/* Number of kernels this library has enqueued in this process (all devices,
 * all threads) since it was loaded.  Benchmarks read it before and after a
 * timed region to count their own launches. */
unsigned long long b200lab_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* B200LAB_H */
