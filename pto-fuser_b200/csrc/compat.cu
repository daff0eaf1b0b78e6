// Kernels behind the reference's finer-grained fused-node keys, so that programs
// lowered the reference's way (kkt epilogue, opaque tri-inv, resident scan,
// chunk_o flash as separate nodes) run unchanged on B200. The fused forward
// (gdn_fwd_tc.cu) subsumes all of them on the hot path; these serve the IR's
// staged / partially fused lowerings and accept any chunk length C <= 128 and head
// dim D <= 256. fp32 accumulation throughout (the reference accumulates in fp32
// and stores fp16).
//
//   gated_qk : L = a b^T * exp(min(g_i + log beta_i - g_j, 0)) * mask   per chunk
//              (src/pto_fuser/kernels/kkt_fused.h:10-13, 154-185)
//   tri_inv  : T = (I + A)^-1, A strictly lower                          per matrix
//              (src/pto_fuser/registry.py:107-127)
//   scan     : h_c = S; S = decay_c S + k_c^T (u_c - w_c S)             per (b, h)
//              (src/pto_fuser/kernels/scan_fused.h:13-17, 217-261)
//   qkv_flash: o = tril(q k^T * exp(min(g_i - g_j, 0))) v                per chunk
//              (src/pto_fuser/kernels/qkv_fused.h:5-18)
//   qk_prologue: L = tril((q * P) (k * invP)^T, 0)                         per chunk
//              (per-channel-gate intra score of the chunked linear family,
//               src/pto_fuser/fused.py:286-311, 532-553)
#include <cuda_runtime.h>

#include "capi_internal.h"
#include "common.cuh"

namespace ptof {
namespace compat {

constexpr int kThreads = 256;

template <typename T>
__device__ __forceinline__ float ldf(const T* p, int64_t i) { return to_f32(p[i]); }

// ------------------------------------------------------------------ gated_qk ----
// One CTA per chunk m. a, b: [M, C, D]; g, beta: [M, C]; L: [M, C, C] (TO).
// mask: 0 strictly lower (kkt), 1 causal incl. diagonal (chunk_o score).
template <typename TI, typename TB, typename TO>
__global__ void __launch_bounds__(kThreads) gated_qk_kernel(const TI* a, const TI* b,
                                                            const float* g, const TB* beta,
                                                            TO* L, int C, int D, int causal) {
  extern __shared__ float sm[];
  const int m = blockIdx.x;
  const int ld = D + 1;
  float* sa = sm;
  float* sb = sm + C * ld;
  float* gv = sb + C * ld;   // g_i + log(beta_i)
  float* gs = gv + C;        // g_j
  const int64_t base = static_cast<int64_t>(m) * C * D;
  for (int idx = threadIdx.x; idx < C * D; idx += kThreads) {
    const int i = idx / D, d = idx % D;
    sa[i * ld + d] = ldf(a, base + idx);
    sb[i * ld + d] = ldf(b, base + idx);
  }
  for (int i = threadIdx.x; i < C; i += kThreads) {
    const float gi = g[static_cast<int64_t>(m) * C + i];
    gs[i] = gi;
    gv[i] = gi + logf(ldf(beta, static_cast<int64_t>(m) * C + i));
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < C * C; idx += kThreads) {
    const int i = idx / C, j = idx % C;
    float out = 0.f;
    if (causal ? (j <= i) : (j < i)) {
      float acc = 0.f;
      for (int d = 0; d < D; ++d) acc = fmaf(sa[i * ld + d], sb[j * ld + d], acc);
      out = acc * expf(fminf(gv[i] - gs[j], 0.f));
    }
    L[static_cast<int64_t>(m) * C * C + idx] = from_f32<TO>(out);
  }
}

// --------------------------------------------------------------- qk_prologue ----
// One CTA per chunk m: the per-channel decay rides on the operands, prescaled while
// staging into shared memory. q, k, P, invP: [M, C, D]; L: [M, C, C] fp16, causal
// (j <= i) incl. the diagonal, zeros above.
template <typename TI>
__global__ void __launch_bounds__(kThreads) qk_prologue_kernel(const TI* q, const TI* k,
                                                               const TI* P, const TI* invP,
                                                               __half* L, int C, int D) {
  extern __shared__ float sm[];
  const int m = blockIdx.x;
  const int ld = D + 1;
  float* sq = sm;
  float* sk = sm + C * ld;
  const int64_t base = static_cast<int64_t>(m) * C * D;
  for (int idx = threadIdx.x; idx < C * D; idx += kThreads) {
    const int i = idx / D, d = idx % D;
    sq[i * ld + d] = ldf(q, base + idx) * ldf(P, base + idx);
    sk[i * ld + d] = ldf(k, base + idx) * ldf(invP, base + idx);
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < C * C; idx += kThreads) {
    const int i = idx / C, j = idx % C;
    float acc = 0.f;
    if (j <= i)
      for (int d = 0; d < D; ++d) acc = fmaf(sq[i * ld + d], sk[j * ld + d], acc);
    L[static_cast<int64_t>(m) * C * C + idx] = __float2half_rn(acc);
  }
}

// ------------------------------------------------------------------- tri_inv ----
// One CTA per matrix; thread j solves column j by forward substitution.
template <typename TA>
__global__ void __launch_bounds__(128) tri_inv_kernel(const TA* A, float* T, int C) {
  extern __shared__ float sm[];
  const int m = blockIdx.x;
  const int ld = C + 1;
  float* sa = sm;
  float* st = sm + C * ld;
  const int64_t base = static_cast<int64_t>(m) * C * C;
  for (int idx = threadIdx.x; idx < C * C; idx += blockDim.x) {
    const int i = idx / C, j = idx % C;
    sa[i * ld + j] = (j < i) ? ldf(A, base + idx) : 0.f;
  }
  __syncthreads();
  const int j = threadIdx.x;
  if (j < C) {
    for (int i = 0; i < C; ++i) st[i * ld + j] = (i == j) ? 1.f : 0.f;
    for (int i = j + 1; i < C; ++i) {
      float acc = 0.f;
      for (int k = j; k < i; ++k) acc = fmaf(sa[i * ld + k], st[k * ld + j], acc);
      st[i * ld + j] = -acc;
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < C * C; idx += blockDim.x)
    T[base + idx] = st[(idx / C) * ld + idx % C];
}

// --------------------------------------------------------------------- scan ----
// One CTA per (b, h, value block of 32). w, k: [B, nc, C, H, D]; u: [B, nc, C, H, Dv];
// decay: [B, H, nc] fp32, or per key dimension [B, H, nc, D] (perdim: row d of S decays
// by decay[.., d], the KDA scan, scan_fused.h:136-180); h_out: [B, nc, H, D, Dv];
// final: [B, H, D, Dv] (TO).
template <typename TI, typename TO>
__global__ void __launch_bounds__(kThreads) scan_kernel(const TI* w, const TI* u, const TI* k,
                                                        const float* decay, TO* h_out,
                                                        TO* final_state, int B, int H, int nc,
                                                        int C, int D, int Dv, int perdim) {
  constexpr int BV = 32;
  extern __shared__ float sm[];
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int v0 = blockIdx.y * BV;
  const int nv = min(BV, Dv - v0);
  const int ld = D + 1;
  float* S = sm;                    // [D][BV]
  float* sw = S + D * BV;           // [C][ld]
  float* sk = sw + C * ld;          // [C][ld]
  float* su = sk + C * ld;          // [C][BV]
  for (int idx = threadIdx.x; idx < D * BV; idx += kThreads) S[idx] = 0.f;
  for (int c = 0; c < nc; ++c) {
    __syncthreads();
    // h_out[b, c, h] = S (before the update)
    for (int idx = threadIdx.x; idx < D * BV; idx += kThreads) {
      const int d = idx / BV, jv = idx % BV;
      if (jv < nv)
        h_out[(((static_cast<int64_t>(b) * nc + c) * H + h) * D + d) * Dv + v0 + jv] =
            from_f32<TO>(S[idx]);
    }
    for (int idx = threadIdx.x; idx < C * D; idx += kThreads) {
      const int i = idx / D, d = idx % D;
      const int64_t off = ((static_cast<int64_t>(b) * nc + c) * C + i) * H * D + h * D + d;
      sw[i * ld + d] = ldf(w, off);
      sk[i * ld + d] = ldf(k, off);
    }
    for (int idx = threadIdx.x; idx < C * BV; idx += kThreads) {
      const int i = idx / BV, jv = idx % BV;
      const int64_t off = ((static_cast<int64_t>(b) * nc + c) * C + i) * H * Dv + h * Dv + v0 + jv;
      su[idx] = jv < nv ? ldf(u, off) : 0.f;
    }
    __syncthreads();
    // vc = u - w S  (into su)
    for (int idx = threadIdx.x; idx < C * BV; idx += kThreads) {
      const int i = idx / BV, jv = idx % BV;
      float acc = 0.f;
      for (int d = 0; d < D; ++d) acc = fmaf(sw[i * ld + d], S[d * BV + jv], acc);
      su[idx] -= acc;
    }
    __syncthreads();
    const int64_t dbase = (static_cast<int64_t>(b) * H + h) * nc + c;
    for (int idx = threadIdx.x; idx < D * BV; idx += kThreads) {
      const int d = idx / BV, jv = idx % BV;
      const float dec = perdim ? decay[dbase * D + d] : decay[dbase];
      float acc = 0.f;
      for (int i = 0; i < C; ++i) acc = fmaf(sk[i * ld + d], su[i * BV + jv], acc);
      S[idx] = dec * S[idx] + acc;
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < D * BV; idx += kThreads) {
    const int d = idx / BV, jv = idx % BV;
    if (jv < nv)
      final_state[((static_cast<int64_t>(b) * H + h) * D + d) * Dv + v0 + jv] = from_f32<TO>(S[idx]);
  }
}

// ---------------------------------------------------------------- qkv_flash ----
// One CTA per chunk m. q, k: [M, C, D]; v: [M, C, Dv]; g: [M, C]; o: [M, C, Dv] fp32.
template <typename TI>
__global__ void __launch_bounds__(kThreads) qkv_flash_kernel(const TI* q, const TI* k,
                                                             const TI* v, const float* g,
                                                             float* o, int C, int D, int Dv) {
  extern __shared__ float sm[];
  const int m = blockIdx.x;
  const int ld = D + 1, lds = C + 1;
  float* sq = sm;
  float* sk = sq + C * ld;
  float* ss = sk + C * ld;     // [C][C+1] gated causal score
  float* gs = ss + C * lds;
  const int64_t b = static_cast<int64_t>(m) * C * D;
  for (int idx = threadIdx.x; idx < C * D; idx += kThreads) {
    const int i = idx / D, d = idx % D;
    sq[i * ld + d] = ldf(q, b + idx);
    sk[i * ld + d] = ldf(k, b + idx);
  }
  for (int i = threadIdx.x; i < C; i += kThreads) gs[i] = g[static_cast<int64_t>(m) * C + i];
  __syncthreads();
  for (int idx = threadIdx.x; idx < C * C; idx += kThreads) {
    const int i = idx / C, j = idx % C;
    float s = 0.f;
    if (j <= i) {
      for (int d = 0; d < D; ++d) s = fmaf(sq[i * ld + d], sk[j * ld + d], s);
      s *= expf(fminf(gs[i] - gs[j], 0.f));
    }
    ss[i * lds + j] = s;
  }
  __syncthreads();
  const int64_t bv = static_cast<int64_t>(m) * C * Dv;
  for (int idx = threadIdx.x; idx < C * Dv; idx += kThreads) {
    const int i = idx / Dv, e = idx % Dv;
    float acc = 0.f;
    for (int j = 0; j <= i; ++j) acc = fmaf(ss[i * lds + j], ldf(v, bv + j * Dv + e), acc);
    o[bv + idx] = acc;
  }
}

// --------------------------------------------------------------- qkvp_flash ----
// Per-channel-gate chunk_o flash, one CTA per chunk m: the decay rides on the
// operands (q P, k invP, prescaled while staging), then the causal score (j <= i)
// and its product with v, the score staying in shared memory.
// q, k, P, invP: [M, C, D]; v: [M, C, Dv]; o: [M, C, Dv] fp32.
template <typename TI>
__global__ void __launch_bounds__(kThreads) qkvp_flash_kernel(const TI* q, const TI* k,
                                                              const TI* v, const TI* P,
                                                              const TI* invP, float* o, int C,
                                                              int D, int Dv) {
  extern __shared__ float sm[];
  const int m = blockIdx.x;
  const int ld = D + 1, lds = C + 1;
  float* sq = sm;
  float* sk = sq + C * ld;
  float* ss = sk + C * ld;     // [C][C+1] causal score
  const int64_t b = static_cast<int64_t>(m) * C * D;
  for (int idx = threadIdx.x; idx < C * D; idx += kThreads) {
    const int i = idx / D, d = idx % D;
    sq[i * ld + d] = ldf(q, b + idx) * ldf(P, b + idx);
    sk[i * ld + d] = ldf(k, b + idx) * ldf(invP, b + idx);
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < C * C; idx += kThreads) {
    const int i = idx / C, j = idx % C;
    float s = 0.f;
    if (j <= i)
      for (int d = 0; d < D; ++d) s = fmaf(sq[i * ld + d], sk[j * ld + d], s);
    ss[i * lds + j] = s;
  }
  __syncthreads();
  const int64_t bv = static_cast<int64_t>(m) * C * Dv;
  for (int idx = threadIdx.x; idx < C * Dv; idx += kThreads) {
    const int i = idx / Dv, e = idx % Dv;
    float acc = 0.f;
    for (int j = 0; j <= i; ++j) acc = fmaf(ss[i * lds + j], ldf(v, bv + j * Dv + e), acc);
    o[bv + idx] = acc;
  }
}

template <typename K>
cudaError_t prep(K kern, size_t smem) {
  return set_smem_once(kern, static_cast<int>(smem));
}

}  // namespace compat

// ------------------------------------------------------------------ launchers ----
int launch_gated_qk(int in_dtype, int beta_dtype, const void* a, const void* b, const float* g,
                    const void* beta, void* L, int M, int C, int D, int causal,
                    cudaStream_t st) {
  using namespace compat;
  const size_t smem = (2 * static_cast<size_t>(C) * (D + 1) + 2 * C) * sizeof(float);
  if (smem > 227 * 1024) return fail(PTOF_EUNSUPPORTED, "gated_qk: C=%d D=%d too large", C, D);
  cudaError_t e;
#define PTOF_GQK(TI, TB)                                                                   \
  {                                                                                        \
    auto kern = gated_qk_kernel<TI, TB, __half>;                                           \
    e = prep(kern, smem);                                                                  \
    if (e == cudaSuccess)                                                                  \
      kern<<<M, kThreads, smem, st>>>(static_cast<const TI*>(a), static_cast<const TI*>(b), g, \
                                      static_cast<const TB*>(beta), static_cast<__half*>(L), C, D, causal); \
  }
  if (in_dtype == PTOF_BF16) {
    if (beta_dtype == PTOF_F32) PTOF_GQK(__nv_bfloat16, float) else if (beta_dtype == PTOF_F16) PTOF_GQK(__nv_bfloat16, __half) else PTOF_GQK(__nv_bfloat16, __nv_bfloat16)
  } else if (in_dtype == PTOF_F16) {
    if (beta_dtype == PTOF_F32) PTOF_GQK(__half, float) else if (beta_dtype == PTOF_F16) PTOF_GQK(__half, __half) else PTOF_GQK(__half, __nv_bfloat16)
  } else {
    if (beta_dtype == PTOF_F32) PTOF_GQK(float, float) else if (beta_dtype == PTOF_F16) PTOF_GQK(float, __half) else PTOF_GQK(float, __nv_bfloat16)
  }
#undef PTOF_GQK
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? PTOF_OK : cuda_fail(e, "gated_qk launch");
}

int launch_tri_inv(int a_dtype, const void* A, float* T, int M, int C, cudaStream_t st) {
  using namespace compat;
  const size_t smem = 2 * static_cast<size_t>(C) * (C + 1) * sizeof(float);
  cudaError_t e;
  if (a_dtype == PTOF_F32) {
    e = prep(tri_inv_kernel<float>, smem);
    if (e == cudaSuccess) tri_inv_kernel<float><<<M, 128, smem, st>>>(static_cast<const float*>(A), T, C);
  } else if (a_dtype == PTOF_F16) {
    e = prep(tri_inv_kernel<__half>, smem);
    if (e == cudaSuccess) tri_inv_kernel<__half><<<M, 128, smem, st>>>(static_cast<const __half*>(A), T, C);
  } else {
    e = prep(tri_inv_kernel<__nv_bfloat16>, smem);
    if (e == cudaSuccess)
      tri_inv_kernel<__nv_bfloat16><<<M, 128, smem, st>>>(static_cast<const __nv_bfloat16*>(A), T, C);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? PTOF_OK : cuda_fail(e, "tri_inv launch");
}

int launch_scan(int in_dtype, int out_dtype, const void* w, const void* u, const void* k,
                const float* decay, void* h_out, void* final_state, int B, int H, int nc, int C,
                int D, int Dv, int perdim, cudaStream_t st) {
  using namespace compat;
  const size_t smem = (static_cast<size_t>(D) * 32 + 2 * static_cast<size_t>(C) * (D + 1) +
                       static_cast<size_t>(C) * 32) * sizeof(float);
  if (smem > 227 * 1024) return fail(PTOF_EUNSUPPORTED, "scan: C=%d D=%d too large", C, D);
  dim3 grid(B * H, (Dv + 31) / 32);
  cudaError_t e = cudaErrorInvalidValue;
#define PTOF_SCAN(TI, TO)                                                                   \
  {                                                                                         \
    auto kern = scan_kernel<TI, TO>;                                                        \
    e = prep(kern, smem);                                                                   \
    if (e == cudaSuccess)                                                                   \
      kern<<<grid, kThreads, smem, st>>>(static_cast<const TI*>(w), static_cast<const TI*>(u), \
                                         static_cast<const TI*>(k), decay, static_cast<TO*>(h_out), \
                                         static_cast<TO*>(final_state), B, H, nc, C, D, Dv, perdim); \
  }
  if (in_dtype == PTOF_F16) {
    if (out_dtype == PTOF_F32) PTOF_SCAN(__half, float) else PTOF_SCAN(__half, __half)
  } else if (in_dtype == PTOF_BF16) {
    if (out_dtype == PTOF_F32) PTOF_SCAN(__nv_bfloat16, float) else PTOF_SCAN(__nv_bfloat16, __nv_bfloat16)
  } else {
    if (out_dtype == PTOF_F32) PTOF_SCAN(float, float) else PTOF_SCAN(float, __half)
  }
#undef PTOF_SCAN
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? PTOF_OK : cuda_fail(e, "chunk_h_scan launch");
}

int launch_qkv_flash(int in_dtype, const void* q, const void* k, const void* v, const float* g,
                     float* o, int M, int C, int D, int Dv, cudaStream_t st) {
  using namespace compat;
  const size_t smem = (2 * static_cast<size_t>(C) * (D + 1) + static_cast<size_t>(C) * (C + 1) + C) *
                      sizeof(float);
  if (smem > 227 * 1024) return fail(PTOF_EUNSUPPORTED, "qkv_flash: C=%d D=%d too large", C, D);
  cudaError_t e;
  if (in_dtype == PTOF_F16) {
    e = prep(qkv_flash_kernel<__half>, smem);
    if (e == cudaSuccess)
      qkv_flash_kernel<__half><<<M, kThreads, smem, st>>>(
          static_cast<const __half*>(q), static_cast<const __half*>(k), static_cast<const __half*>(v), g, o, C, D, Dv);
  } else if (in_dtype == PTOF_BF16) {
    e = prep(qkv_flash_kernel<__nv_bfloat16>, smem);
    if (e == cudaSuccess)
      qkv_flash_kernel<__nv_bfloat16><<<M, kThreads, smem, st>>>(
          static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
          static_cast<const __nv_bfloat16*>(v), g, o, C, D, Dv);
  } else {
    e = prep(qkv_flash_kernel<float>, smem);
    if (e == cudaSuccess)
      qkv_flash_kernel<float><<<M, kThreads, smem, st>>>(
          static_cast<const float*>(q), static_cast<const float*>(k), static_cast<const float*>(v), g, o, C, D, Dv);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? PTOF_OK : cuda_fail(e, "qkv_flash launch");
}

int launch_qkvp_flash(int in_dtype, const void* q, const void* k, const void* v, const void* P,
                      const void* invP, float* o, int M, int C, int D, int Dv, cudaStream_t st) {
  using namespace compat;
  const size_t smem = (2 * static_cast<size_t>(C) * (D + 1) + static_cast<size_t>(C) * (C + 1)) *
                      sizeof(float);
  if (smem > 227 * 1024) return fail(PTOF_EUNSUPPORTED, "qkvp_flash: C=%d D=%d too large", C, D);
  cudaError_t e;
#define PTOF_QKVP(TI)                                                                        \
  {                                                                                          \
    auto kern = qkvp_flash_kernel<TI>;                                                       \
    e = prep(kern, smem);                                                                    \
    if (e == cudaSuccess)                                                                    \
      kern<<<M, kThreads, smem, st>>>(static_cast<const TI*>(q), static_cast<const TI*>(k),   \
                                      static_cast<const TI*>(v), static_cast<const TI*>(P),   \
                                      static_cast<const TI*>(invP), o, C, D, Dv);             \
  }
  if (in_dtype == PTOF_BF16) PTOF_QKVP(__nv_bfloat16) else if (in_dtype == PTOF_F16) PTOF_QKVP(__half) else PTOF_QKVP(float)
#undef PTOF_QKVP
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? PTOF_OK : cuda_fail(e, "qkvp_flash launch");
}

int launch_qk_prologue(int in_dtype, const void* q, const void* k, const void* P,
                       const void* invP, void* L, int M, int C, int D, cudaStream_t st) {
  using namespace compat;
  const size_t smem = 2 * static_cast<size_t>(C) * (D + 1) * sizeof(float);
  if (smem > 227 * 1024) return fail(PTOF_EUNSUPPORTED, "qk_prologue: C=%d D=%d too large", C, D);
  cudaError_t e;
#define PTOF_QKP(TI)                                                                        \
  {                                                                                         \
    auto kern = qk_prologue_kernel<TI>;                                                     \
    e = prep(kern, smem);                                                                   \
    if (e == cudaSuccess)                                                                   \
      kern<<<M, kThreads, smem, st>>>(static_cast<const TI*>(q), static_cast<const TI*>(k),  \
                                      static_cast<const TI*>(P), static_cast<const TI*>(invP), \
                                      static_cast<__half*>(L), C, D);                       \
  }
  if (in_dtype == PTOF_BF16) PTOF_QKP(__nv_bfloat16) else if (in_dtype == PTOF_F16) PTOF_QKP(__half) else PTOF_QKP(float)
#undef PTOF_QKP
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? PTOF_OK : cuda_fail(e, "qk_prologue launch");
}

}  // namespace ptof
