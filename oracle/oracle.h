/*
 * oracle.h -- CPU fp64 restatement of the reference's hot-path math.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links this code.
 * It is loaded by tests/, by __graft_entry__.smoke() and by bench.py's
 * cpu_baseline / --impl reference legs, always as the checker or the timed
 * CPU baseline, never as a fallback for the CUDA path.
 *
 * Reference being restated (cookys/turing-sm75):
 *   attention : naive_attn_kernel          src/attn_sm75.cu:55-94
 *   GDN serial: gdn_cpu                    src/gdn_sm75.cu:1078-1106
 *   GDN chunk : gdn_chunked_cpu            src/gdn_sm75.cu:1109-1244 (algebra),
 *               with the triangular solve done as a true inverse (see oracle.c).
 *
 * Layouts (all row-major, innermost last):
 *   attention: Q,O [B][Hq][Sq][D]; K,V [B][Hkv][Skv][D]  (the reference's
 *              [B*H][S][D] when Hkv == Hq and Sq == Skv)
 *   GDN      : q,k [B][T][Hqk][dk]; v,o [B][T][Hv][dv]; g_log,beta [B][T][Hv];
 *              state [B][Hv][dv][dk]; element state[c*dk + i] multiplies k[i]
 *              (the reference's layout, src/gdn_sm75.cu:1094, plus a batch dim).
 *
 * Parity status: pinned.  The GDN restatement is checked against the
 * reference's own gdn_cpu compiled from its sources (oracle/_ref) and against
 * golden vectors produced by it (tests/golden/).  The attention restatement is
 * checked against the reference's naive_attn_kernel compiled from its sources
 * and run on the GPU (tests/test_attn_gpu.py), and against closed-form cases.
 */
#ifndef B200LAB_ORACLE_H
#define B200LAB_ORACLE_H

#ifdef __cplusplus
extern "C" {
#endif

/* Softmax attention forward, fp64.
 * causal: key j is visible to query i iff j <= i + (Skv - Sq) (bottom-right
 * alignment; equals the reference's k <= q when Sq == Skv).  A query row with
 * no visible key produces 0, as the reference's flash kernels do
 * (src/attn_sm75.cu:372).
 * rows/nrows: if rows != NULL only those query rows are computed for every
 * (b, h) and O is laid out [B][Hq][nrows][D].  Returns 0, or -1 on bad args. */
int orc_attn_fwd(const float* Q, const float* K, const float* V, double* O,
                 int B, int Hq, int Hkv, int Sq, int Skv, int D, double scale,
                 int causal, const int* rows, int nrows, int nthreads);

/* Gated DeltaNet, token-serial recurrence (src/gdn_sm75.cu:1078-1106), fp64:
 *   g = exp(g_log); kv = S k; d = (v - g*kv)*beta; S = g*S + d k^T;
 *   o = scale * S q.
 * state is read and updated in place.  head_map 0: v-head h uses q/k head
 * h % Hqk (the reference, src/gdn_sm75.cu:1083); 1: h / (Hv/Hqk). */
int orc_gdn_recurrent(const float* q, const float* k, const float* v,
                      const float* g_log, const float* beta, double* state,
                      double* out, int B, int T, int Hqk, int Hv, int dk, int dv,
                      int head_map, double scale, int nthreads);

/* Same result through the chunked (WY/UT) algebra of src/gdn_sm75.cu:1109-1244
 * with chunk length C.  Exact in real arithmetic; agrees with
 * orc_gdn_recurrent to ~1e-12. */
int orc_gdn_chunked(const float* q, const float* k, const float* v,
                    const float* g_log, const float* beta, double* state,
                    double* out, int B, int T, int Hqk, int Hv, int dk, int dv,
                    int head_map, double scale, int C, int nthreads);

/* The reference's chunk algebra with its own triangular-solve loop
 * (src/gdn_sm75.cu:1160-1180) kept as written, in fp64.  Used only by a test
 * that documents how far that loop's result is from the recurrence. */
int orc_gdn_chunked_refsolve(const float* q, const float* k, const float* v,
                             const float* g_log, const float* beta, double* state,
                             double* out, int B, int T, int Hqk, int Hv, int dk,
                             int dv, int head_map, double scale, int C,
                             int nthreads);

/* Number of hardware threads the oracle would use for nthreads <= 0. */
int orc_default_threads(void);

#ifdef __cplusplus
}
#endif
#endif
