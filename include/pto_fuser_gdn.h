/*
 * pto_fuser_gdn.h — C ABI of the B200 (sm_100a) chunked Gated DeltaNet kernels.
 *
 * This library replaces the Ascend kernel .so files that pto-fuser loads with
 * ctypes (src/pto_fuser/fused.py:58-77, registry.py:96-104). It keeps their
 * setup / exec / teardown discipline (fused.py:93-115): `*_setup` allocates the
 * library-owned workspace once, `*_exec` only launches on the caller's stream
 * (no host synchronisation, so calls can be captured into a CUDA graph), and
 * `*_teardown` frees the workspace.
 *
 * Differences from the reference ABI, by design:
 *   - shapes are runtime parameters (the reference rebuilds one .so per shape
 *     through -D defines, fused.py:66-76);
 *   - every exec returns a status code (the reference's exec functions return
 *     void and report nothing);
 *   - chunk batches are keyed on M = B*H*nc (the reference's native launchers
 *     drop B, fused.py:256,264).
 *
 * All tensor arguments are device pointers; the caller owns inputs and outputs.
 * Pointers must be 16-byte aligned and rows contiguous in the innermost dim.
 */
#ifndef PTO_FUSER_GDN_H
#define PTO_FUSER_GDN_H

#include <stdint.h>

#if defined(__GNUC__)
#define PTOF_API __attribute__((visibility("default")))
#else
#define PTOF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes returned by every exec / check call ---------------------- */
enum {
  PTOF_OK = 0,
  PTOF_EINVAL = 1,       /* bad shape / null pointer / bad dtype code           */
  PTOF_EALIGN = 2,       /* pointer not 16-byte aligned                          */
  PTOF_ECUDA = 3,        /* a CUDA runtime / driver call failed                  */
  PTOF_EUNSUPPORTED = 4, /* valid request this build does not implement          */
  PTOF_ETIMEOUT = 5      /* a device-side bounded wait gave up (see check_status) */
};

/* ---- element type codes ---------------------------------------------------- */
enum { PTOF_F32 = 0, PTOF_F16 = 1, PTOF_BF16 = 2 };

/* ---- memory layouts of q/k/v/o ([.., D] innermost) and of beta/g ------------ */
enum {
  PTOF_LAYOUT_BHTD = 0, /* q [B,H,T,D], beta/g [B,H,T]  (== reference [B,H,nc,C,D]) */
  PTOF_LAYOUT_BTHD = 1  /* q [B,T,H,D], beta/g [B,T,H]  (reference "mega" layout)   */
};

/* ---- gate modes -------------------------------------------------------------- */
enum {
  PTOF_GATE_RAW = 0,    /* g is the per-token log decay; kernels do the chunk-local cumsum */
  PTOF_GATE_CUMSUM = 1, /* g already holds the chunk-local inclusive cumsum (g_native)     */
  PTOF_GATE_NONE = 2    /* ungated DeltaNet: g ignored (may be NULL)                        */
};

/* Shape / dtype description of one chunked GDN forward. */
typedef struct ptof_gdn_params {
  int32_t B, H, T;    /* batch, heads, tokens (T a multiple of C)          */
  int32_t C;          /* chunk length; 64                                 */
  int32_t Dk, Dv;     /* key / value head dims                            */
  int32_t in_dtype;   /* q, k, v element type (PTOF_F32/F16/BF16)         */
  int32_t beta_dtype; /* beta element type                                */
  int32_t out_dtype;  /* o element type                                   */
  int32_t gate_mode;  /* PTOF_GATE_*; g is always fp32                    */
  int32_t layout;     /* PTOF_LAYOUT_*                                    */
  float scale;        /* output scale (reference: D^-0.5)                 */
} ptof_gdn_params;

/* ---------------------------------------------------------------------------
 * Full fused chunk forward:
 *   cumsum -> A = tril(beta*KK^T*exp(dg), -1) -> T = (I+A)^-1 -> W, U ->
 *   state scan -> o = scale*(exp(g)*(Q S) + tril(QK^T*exp(min(dg,0))) V_new)
 * Replaces the whole lowered chain kkt_gated_native_v2 -> tri_inv_rec_unroll ->
 * W/U einsums -> chunk_h_scan -> qkv_flash_native_v2 (fused.py:446-569,
 * registry.py:96-140) and matches gdn_reference (examples/attention/_gdn_full.py:57-97)
 * plus the final state and an optional initial state.
 *   q,k: [.., Dk] in_dtype; v: [.., Dv] in_dtype; beta: in beta_dtype; g: fp32;
 *   S0: [B,H,Dk,Dv] fp32 or NULL (zero state); o: [.., Dv] out_dtype;
 *   S_final: [B,H,Dk,Dv] fp32 or NULL.
 * fp32 inputs run the fp32 SIMT kernel (reference tolerance 1e-4); fp16/bf16
 * inputs run the tcgen05 kernel (fp32 accumulate, tolerance 1e-2).
 */
PTOF_API void* ptof_gdn_fwd_setup(const ptof_gdn_params* p);
PTOF_API int ptof_gdn_fwd_exec(void* ws, const void* q, const void* k, const void* v, const void* beta,
                      const float* g, const float* S0, void* o, float* S_final, void* stream);
PTOF_API void ptof_gdn_fwd_teardown(void* ws);

/* Variable-length sequences with grouped query/key heads (the production layout the
 * reference leaves out: registry.py:124 passes cu_seqlens=None; gdn_mega.py:49-50).
 * N sequences packed token-major: q, k [T_total, Hg, Dk]; v, o [T_total, H, Dv];
 * beta, g [T_total, H]; sequence n spans tokens [cu_seqlens[n], cu_seqlens[n+1])
 * (device int32 [N+1], non-decreasing, every length <= max_len; a longer one is cut
 * at max_len and reported by ptof_check_status). Value head h reads query/key head
 * h / (H / Hg). Chunks start at each sequence's first token; the last chunk of a
 * sequence may be partial. S0 / S_final [N, H, Dk, Dv] fp32 (optional). f16/bf16
 * operands, Dk = Dv = 64 or 128. Empty sequences return S_final = S0 (or 0). */
typedef struct ptof_gdn_varlen_params {
  int32_t N, H, Hg;    /* sequences, value heads, query/key heads (H % Hg == 0) */
  int32_t T_total;     /* packed tokens                                        */
  int32_t max_len;     /* upper bound of every sequence length                 */
  int32_t Dk, Dv;
  int32_t in_dtype, beta_dtype, out_dtype, gate_mode;
  float scale;
} ptof_gdn_varlen_params;
PTOF_API void* ptof_gdn_fwd_varlen_setup(const ptof_gdn_varlen_params* p);
PTOF_API int ptof_gdn_fwd_varlen_exec(void* ws, const void* q, const void* k, const void* v,
                                      const void* beta, const float* g, const int* cu_seqlens,
                                      const float* S0, void* o, float* S_final, void* stream);

/* The same f16/bf16 tensor-core forward without a workspace and without any device
 * allocation. It has no counterpart in the reference. It is for callers that cannot
 * call cudaMalloc, e.g. code inside a device-memory allocator or arena that owns all
 * device memory, or code replaying a fixed memory plan. Its per-chunk scratch (the gate
 * coefficient records) lives in a fixed array in the library's device memory, reserved
 * on every GPU that loads the library until the process exits:
 *   - B*H*T/64 must not exceed 4096 chunks (7.4 MB of records); larger problems
 *     are rejected with PTOF_EINVAL, and unsupported shapes or dtypes
 *     (fp32, Dk = Dv other than 64 or 128) with PTOF_EUNSUPPORTED;
 *   - the first call on a device looks up the array's device address with that
 *     device current (cudaGetSymbolAddress); make it before any stream capture;
 *   - every call shares the one array, so calls whose kernels overlap on the GPU
 *     (other streams, other host threads) race and corrupt each other's results;
 *   - its bounded device waits report to a library status word of its own, read
 *     with ptof_gdn_fwd_noalloc_status (ptof_check_status takes a workspace).
 * Inputs and outputs are as for ptof_gdn_fwd_exec; the call launches on `stream`
 * and does not synchronise. */
PTOF_API int ptof_gdn_fwd_exec_noalloc(const ptof_gdn_params* p, const void* q, const void* k,
                                       const void* v, const void* beta, const float* g,
                                       const float* S0, void* o, float* S_final, void* stream);

/* Status of the allocation-free forwards on the current device: synchronises `stream`,
 * then reads and clears the status word they share. PTOF_OK, or PTOF_ETIMEOUT when a
 * bounded device wait of one of them gave up since the last read (its outputs are then
 * undefined). Allocates nothing. */
PTOF_API int ptof_gdn_fwd_noalloc_status(void* stream);

/* ---------------------------------------------------------------------------
 * Kernels behind the reference's finer-grained fused-node keys. They share one
 * library-owned workspace (status word) from ptof_ws_setup / ptof_ws_teardown,
 * replacing the per-kernel setup/teardown pairs kkt_setup, scan_setup and qkv_setup
 * (kernels/kkt_fused_lib.cpp:401-443, scan_lib.cpp:343-365, qkv_fused_lib.cpp:296-344).
 * All chunk batches are native [M, C, ...] with M = B*H*nc; C <= 128, D <= 256.
 */
PTOF_API void* ptof_ws_setup(void);
PTOF_API void ptof_ws_teardown(void* ws);

/* Gated masked a b^T per chunk (replaces kkt_exec / kkt_exec_v2,
 * kernels/kkt_fused_lib.cpp:411-441):
 *   L[m,i,j] = (a_i . b_j) * exp(min(g_i + log beta_i - g_j, 0)) * mask(i,j)
 * mask: strict lower (causal = 0, the kkt A) or lower incl. diagonal (causal = 1).
 * a, b [M,C,D] in_dtype; g [M,C] fp32; beta [M,C] beta_dtype; L [M,C,C] fp16. */
PTOF_API int ptof_gated_qk_exec(void* ws, const void* a, const void* b, const float* g,
                                const void* beta, void* L, int M, int C, int D, int in_dtype,
                                int beta_dtype, int causal, void* stream);

/* The kkt + triangular-inverse stage alone, fused: per chunk of
 * 64 tokens A = tril(beta_i k_i.k_j exp(g_i - g_j), -1) and T = (I + A)^-1, written
 * as fp32 T_out [B, H, T/64, 64, 64] (chunk order b, h, c). k [B,H,T,D] or [B,T,H,D]
 * (layout) in f16/bf16, D = 64 or 128; beta like g; g fp32 raw / chunk-local cumsum /
 * ignored (gate_mode). Replaces the reference's kkt_exec (kernels/kkt_fused_lib.cpp:
 * 401-443) followed by the external tri_inv (registry.py:96-140); matches
 * _gdn_full.py:73-78. ws: a workspace from ptof_ws_setup (its status word records
 * device wait timeouts) or NULL. */
PTOF_API int ptof_kkt_inv_exec(void* ws, const void* k, const void* beta, const float* g,
                               float* T_out, int B, int H, int T, int D, int in_dtype,
                               int beta_dtype, int gate_mode, int layout, void* stream);

/* Per-channel-gate chunk_o flash (KDA / GLA): o = tril((q * P)(k * invP)^T, 0) v per
 * chunk, the score kept on chip. q/k/P/invP [M, C, D], v [M, C, Dv] (f16/bf16/f32),
 * o [M, C, Dv] fp32. Replaces qkvp_exec / qkvp_exec_v2 (the qkvp_flash_native[_v2]
 * keys, src/pto_fuser/fused.py:396-441, 570-585). C <= 128, D <= 256. */
PTOF_API int ptof_qkvp_flash_exec(void* ws, const void* q, const void* k, const void* v,
                                  const void* P, const void* invP, float* o, int M, int C,
                                  int D, int Dv, int in_dtype, void* stream);

/* Per-channel-gate intra-chunk score of the chunked linear-attention family (GLA):
 * L = tril((q * P) (k * invP)^T, 0) per chunk, q/k/P/invP [M, C, D] (f16/bf16/f32),
 * L [M, C, C] fp16. Replaces pro_exec / pro_exec_v2 (the qk_prologue[_v2] keys,
 * src/pto_fuser/fused.py:286-311, 532-553). C <= 128, D <= 256. */
PTOF_API int ptof_qk_prologue_exec(void* ws, const void* q, const void* k, const void* P,
                                   const void* invP, void* L, int M, int C, int D, int in_dtype,
                                   void* stream);

/* (I + A)^-1 for strictly-lower A [M,C,C] (a_dtype), fp32 out [M,C,C]; replaces the
 * opaque tri_inv_rec_unroll kernel (registry.py:96-140). Unlike the reference it takes
 * A lower-triangular directly (no transpose round trip). ws may be NULL. */
PTOF_API int ptof_tri_inv_exec(void* ws, const void* A, int a_dtype, float* T, int M, int C,
                               void* stream);

/* Resident-state chunk recurrence (replaces scan_exec, kernels/scan_lib.cpp:354-361):
 *   h_out[b,c,h] = S; S = decay[b,h,c] * S + k_c^T (u_c - w_c S); final = S.
 * w, k [B,nc,C,H,D], u [B,nc,C,H,Dv] in_dtype; decay [B,H,nc] fp32;
 * h_out [B,nc,H,D,Dv], final [B,H,D,Dv] in out_dtype (fp16 / bf16 / fp32). */
PTOF_API int ptof_chunk_h_scan_exec(void* ws, const void* w, const void* u, const void* k,
                                    const float* decay, void* h_out, void* final_state, int B,
                                    int H, int nc, int C, int D, int Dv, int in_dtype,
                                    int out_dtype, void* stream);

/* The same scan with a per-key-dimension decay (the KDA scan: chunk_h_scan built with
 * perdim_decay=True, transforms/kda.py:19-70; scan_fused.h:136-180): decay is fp32
 * [B, H, nc, D] and row d of the state decays by decay[b, h, c, d]. */
PTOF_API int ptof_chunk_h_scan_perdim_exec(void* ws, const void* w, const void* u, const void* k,
                                           const float* decay, void* h_out, void* final_state,
                                           int B, int H, int nc, int C, int D, int Dv,
                                           int in_dtype, int out_dtype, void* stream);

/* chunk_o score -> output in one launch (replaces qkv_exec / qkv_exec_v2,
 * kernels/qkv_fused_lib.cpp:296-344): o = tril(q k^T * exp(min(g_i - g_j, 0))) v.
 * q, k [M,C,D], v [M,C,Dv] in_dtype; g [M,C] fp32; o [M,C,Dv] fp32. */
PTOF_API int ptof_qkv_flash_exec(void* ws, const void* q, const void* k, const void* v,
                                 const float* g, float* o, int M, int C, int D, int Dv,
                                 int in_dtype, void* stream);

/* Stage timing trace (no counterpart in the reference, which attributes cost with
 * compile-time knock-out flags, kernels/kkt_fused.h:49-56): while set, every
 * tensor-core launch on this workspace writes, for CTA 0 and its first `chunks`
 * chunks, 24 globaltimer stamps (ns) per chunk into the caller's device buffer
 * dev_buf[chunks][24], followed by one record {start ns, end ns, SM id, 0} per CTA
 * (B*H records). chunks = 0 turns tracing off. */
PTOF_API int ptof_gdn_fwd_set_trace(void* ws, void* dev_buf, int chunks);

/* Fused chunked KDA forward (Kimi Delta Attention: a per-key-dimension gate) on the
 * tensor cores. Replaces the reference's lowered KDA chain — the per-dim scan
 * (scan_exec with perdim_decay, kernels/scan_fused.h:136-180) plus the per-dim
 * prologue/flash keys (pro_exec / qkvp_exec, kernels/prologue_fused.h:1-28,
 * kernels/qkv_prologue_fused.h:1-24) — with one operand pre-pass and one fused
 * launch, the semantics of kda_reference (examples/attention/_kda_full.py:38-77)
 * plus an optional initial state and the final state.
 * q, k, v bf16 [B,H,T,64]; beta [B,H,T] (beta_dtype); g fp32 [B,H,T,64] per-token
 * per-dimension log decay; S0 / S_final fp32 [B,H,64,64] (optional); o [B,H,T,64]
 * (out_dtype). Requires C = 64, Dk = Dv = 64, in_dtype BF16, layout BHTD. The gate is
 * applied to the operands (k e^g, q e^g, k e^-g with g the chunk-local cumsum), as in
 * the reference's factorised form: a chunk whose total decay in some dimension
 * exceeds about 80 overflows the bf16 operands, as it does there. */
PTOF_API void* ptof_kda_fwd_setup(const ptof_gdn_params* p);
PTOF_API int ptof_kda_fwd_exec(void* ws, const void* q, const void* k, const void* v,
                               const void* beta, const float* g, const float* S0, void* o,
                               float* S_final, void* stream);

/* Limit of every bounded device wait of the tensor-core forward launched on this
 * workspace, in nanoseconds (default 2 s). No counterpart in the reference, whose
 * kernels have no wait limit. A wait that exceeds it ends the launch early, records
 * its site in the status word and makes ptof_check_status return PTOF_ETIMEOUT; the
 * outputs of that launch are then undefined. Lowering it is for fault-path tests
 * (a limit below the time one chunk takes makes a wait run out on purpose). */
PTOF_API int ptof_ws_set_wait_limit(void* ws, unsigned long long ns);

/* Strided views for the tensor-core forward on this workspace (no counterpart in the
 * reference, whose operands are always dense): with the heads-outer layout, head (b, h)
 * of q, k, beta and g starts at token b * qk_pair + h * qk_seg of its buffer, of v at
 * b * v_pair + h * v_seg, of o at b * o_pair + h * o_seg (strides in tokens; T tokens
 * from there). All zero restores the dense [B,H,T,D] layout. Used by the chunk-segment
 * scan inside one GPU, which runs segments of the caller's sequences in place. */
PTOF_API int ptof_gdn_fwd_set_view(void* ws, long long qk_pair, long long qk_seg,
                                   long long v_pair, long long v_seg, long long o_pair,
                                   long long o_seg);

/* Fault-path test hook (no counterpart in the reference): while `on` is nonzero, each
 * tensor-core forward launched on this workspace first waits on a device barrier that
 * nothing arrives at, so that wait runs out after the wait limit, the launch ends early
 * (site 99 in the status word) and ptof_check_status returns PTOF_ETIMEOUT. No trap,
 * fault or unbounded spin is involved. */
PTOF_API int ptof_gdn_fwd_inject_stall(void* ws, int on);

/* Reads (and clears) the workspace's device status word after synchronising
 * `stream`: PTOF_OK, or PTOF_ETIMEOUT when a bounded device wait gave up. */
PTOF_API int ptof_check_status(void* ws, void* stream);

/* ---------------------------------------------------------------------------
 * Segment-state combine for a chunk-segment scan of one long sequence (no
 * counterpart in the reference: it runs each head's recurrence serially over the
 * whole sequence, scan_fused.h:198-262, and its own notes place few-head long
 * contexts outside its winning regime, docs/DESIGN.md:336-340).
 * Over a chunk-aligned token segment the state map is affine, S_out = A S_in + B:
 * A [D,D] is the final state of ptof_gdn_fwd_exec started from S0 = I with v = 0,
 * B [D,Dv] the final state started from S0 = 0. For every head this applies the
 * maps of segments j = 0..nseg-1 in order:
 *   X_0 = X0 (NULL: zero),  X_{j+1} = A_j X_j + B_j  (Bv NULL: no offset)
 * and writes the entry state X_j of each segment to Xout (NULL: not written) and
 * X_nseg to Xfinal (NULL: not written). All fp32; every matrix is row-major with
 * rows of D (A) or Dv (B, X) floats; the *_stride arguments give, in floats, the
 * distance between heads and between segments (multiples of 4; pointers 16-byte
 * aligned). D in {64, 128}, Dv a multiple of 32, nseg >= 0. Launches on `stream`, no host synchronisation. Outputs must not
 * overlap the inputs.
 */
PTOF_API int ptof_seg_scan_exec(const float* A, int64_t a_head_stride, int64_t a_seg_stride,
                                const float* Bv, int64_t b_head_stride, int64_t b_seg_stride,
                                const float* X0, int64_t x0_head_stride, float* Xout,
                                int64_t xout_head_stride, int64_t xout_seg_stride,
                                float* Xfinal, int64_t xfinal_head_stride, int heads, int nseg,
                                int D, int Dv, void* stream);

/* Output fix-up of the chunk-segment scan (no counterpart in the reference; see
 * ptof_seg_scan_exec). A segment's output is affine in its entry state X:
 * o = o^B + o^A X, with o^B the forward's output from a zero state (held in `o` on
 * entry) and o^A its output from S0 = I with v = 0. For every unit u (one token
 * segment of one (b, h) pair) and token t < Tseg:
 *   o[u][t][:] += oa[u][t][:] @ X[u]      (fp32 accumulate, result rounded to dtype)
 * o, oa: [units][Tseg][D] in dtype (PTOF_BF16 / PTOF_F16), oa distinct from o;
 * X: [units][D][D] fp32 (rounded to dtype for the tensor-core product). Tseg a
 * multiple of 128, D 64 or 128, pointers 16-byte aligned. `ws` (from ptof_ws_setup,
 * or NULL) receives the status of bounded device waits (ptof_check_status).
 * Launches on `stream`, no host synchronisation. */
PTOF_API int ptof_seg_fix_exec(void* ws, void* o, const void* oa, const float* X, int units,
                               int Tseg, int D, int dtype, void* stream);

/* The same fix-up with o a strided view (no counterpart in the reference): unit
 * (pair, seg) of o starts at token pair * o_pair_stride + seg * o_seg_stride of o's
 * buffer; o^A [pairs * segs, Tseg, D] and X [pairs * segs, D, D] are contiguous. */
PTOF_API int ptof_seg_fix_exec_view(void* ws, void* o, const void* oa, const float* X, int pairs,
                                    int segs, int Tseg, int D, int dtype,
                                    long long o_pair_stride, long long o_seg_stride,
                                    void* stream);

/* Human-readable text of the last host-side error on this thread. */
PTOF_API const char* ptof_last_error(void);

/* ---------------------------------------------------------------------------
 * Self-tests of the sm_100a building blocks (no counterpart in the reference).
 * selftest_umma: D[M,N] = (+-)A[M,K] * B[N,K]^T through one UMMA, A/B fp32 device
 *   arrays rounded to bf16. mode bit0: A MN-major in smem; bit1: B MN-major;
 *   bit2: A from TMEM; bit3: negate A. M in {64,128}, N%16==0 <= 256, K%32==0 <= 128.
 * selftest_tma: TMA SWIZZLE_128B load of the [64 x 64] bf16 box at column x0,
 *   row y0 of a row-major [rows, cols] bf16 matrix, de-swizzled into out[64*64].
 * selftest_umma_rate: issue-rate probe. `issuers` threads (1-4) each issue `n`
 *   back-to-back UMMAs (M=128, N, K=16; n a multiple of 8; a_tmem = mode bits: 1 A from
 *   TMEM, 2 warp-uniform issue, 4 incremented descriptors, 8 unrolled) into their own
 *   accumulator; out (device int64 [3*issuers]) receives per issuer the issue
 *   cycles, issue-to-completion cycles and one single UMMA's round trip (cycles).
 * `status` is a device int that receives a nonzero code if a bounded wait gave up.
 */
PTOF_API int ptof_selftest_umma(const float* A, const float* B, float* D, int M, int N, int K,
                                int mode, int* status, void* stream);
PTOF_API int ptof_selftest_umma_rate(int N, int n, int issuers, int a_tmem, long long* out,
                                     int* status, void* stream);
PTOF_API int ptof_selftest_tma(const void* src, int rows, int cols, int x0, int y0, void* out,
                               int* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PTO_FUSER_GDN_H */
