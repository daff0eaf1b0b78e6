// fp32 SIMT chunk forward of Gated DeltaNet.
//
// The full-precision path (fp32 inputs, reference tolerance 1e-4): every
// contraction accumulates in fp32 FMA on the CUDA cores (value-column products in
// register tiles of four columns), the (I+A)^-1 solve is a forward substitution
// per column (a warp per eight columns, shuffles only, no block barrier), the
// per-token exponentials are computed once per chunk, and the state S[Dk, BV] of one
// (batch, head, value-block) stays resident in shared memory across all chunks.
// It restates, step for step, gdn_reference (examples/attention/_gdn_full.py:57-97):
//   A   = tril((k k^T) * safe_exp(g_i - g_j) * beta_i, -1)          :73-75
//   T   = solve_triangular(I + A, I, unitriangular)                   :76-78
//   W   = T (k * beta * exp(g)),  U = T (v * beta)                     :79-82
//   vn  = U - W S ; S = exp(g_last) S + k^T (vn * exp(g_last - g))    :83-87
//   o   = (q S) * exp(g) + (q k^T * exp(min(g_i - g_j, 0)) * causal) vn  :88-94
// with two additions the reference lacks: an initial state S0 and the final state.
//
// One CTA per (b*h, value block of kBV columns); the chunk loop is sequential.
#include <cuda_runtime.h>

#include "capi_internal.h"
#include "common.cuh"

namespace ptof {

namespace simt {

constexpr int kThreads = 256;
constexpr int kBV = 32;       // value columns per CTA
constexpr int kMaxDk = 128;
constexpr int kC = kChunk;    // 64

struct Args {
  const void* q;
  const void* k;
  const void* v;
  const void* beta;
  const float* g;
  const float* S0;
  void* o;
  float* S_final;
  int B, H, T, Dk, Dv;
  int gate_mode;
  float scale;
  Strides4 sq, sv;   // q/k strides (Dk) and v/o strides (Dv)
  Strides3 sg;       // beta / g strides
};

// shared-memory carve-up (floats); padded rows break bank conflicts
struct __align__(16) Smem {
  // rows padded to a multiple of 4 floats (float4 access) plus 4 (bank spread)
  static constexpr int kLdK = kMaxDk + 4;
  static constexpr int kLdC = kC + 1;
  static constexpr int kLdV = kBV + 4;
  float K[kC * kLdK];
  float Q[kC * kLdK];
  float W[kC * kLdK];
  float V[kC * kLdV];
  float U[kC * kLdV];
  float Vn[kC * kLdV];
  float A[kC * kLdC];
  float Tm[kC * kLdC];
  float Aqk[kC * kLdC];
  float S[kMaxDk * kLdV];
  float g[kC];
  float beta[kC];
  float eg[kC];    // e^{g_i}
  float wk[kC];    // beta_j e^{g_j}   (W operand scale)
  float gam[kC];   // e^{g_last - g_i} (state update scale)
};

template <typename TI, typename TB, typename TO>
__global__ void __launch_bounds__(kThreads) gdn_fwd_simt_kernel(Args a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>(smem_raw);
  const int tid = threadIdx.x;
  const int bh = blockIdx.x;
  const int b = bh / a.H, h = bh % a.H;
  const int v0 = blockIdx.y * kBV;
  const int nv = min(kBV, a.Dv - v0);
  const int Dk = a.Dk;
  constexpr int ldk = Smem::kLdK, ldc = Smem::kLdC, ldv = Smem::kLdV;

  const TI* qp = static_cast<const TI*>(a.q) + b * a.sq.b + h * a.sq.h;
  const TI* kp = static_cast<const TI*>(a.k) + b * a.sq.b + h * a.sq.h;
  const TI* vp = static_cast<const TI*>(a.v) + b * a.sv.b + h * a.sv.h + v0;
  TO* op = static_cast<TO*>(a.o) + b * a.sv.b + h * a.sv.h + v0;
  const TB* bp = static_cast<const TB*>(a.beta) + b * a.sg.b + h * a.sg.h;
  const float* gp = a.g ? a.g + b * a.sg.b + h * a.sg.h : nullptr;
  const int64_t sbase = static_cast<int64_t>(bh) * Dk * a.Dv;

  // K and Q rows are read as float4 up to the next multiple of 4: zero that tail once
  // (the chunk loads below write columns d < Dk only)
  const int dk4 = (Dk + 3) / 4;
  for (int idx = tid; idx < kC * (4 * dk4 - Dk); idx += kThreads) {
    const int i = idx / (4 * dk4 - Dk), d = Dk + idx % (4 * dk4 - Dk);
    s.K[i * ldk + d] = 0.f;
    s.Q[i * ldk + d] = 0.f;
  }
  // initial state
  for (int idx = tid; idx < Dk * kBV; idx += kThreads) {
    const int d = idx / kBV, j = idx % kBV;
    float x = 0.f;
    if (a.S0 && j < nv) x = a.S0[sbase + static_cast<int64_t>(d) * a.Dv + v0 + j];
    s.S[d * ldv + j] = x;
  }

  const int nc = a.T / kC;
  for (int c = 0; c < nc; ++c) {
    const int t0 = c * kC;
    __syncthreads();
    // ---- load the chunk -------------------------------------------------
    for (int idx = tid; idx < kC * Dk; idx += kThreads) {
      const int i = idx / Dk, d = idx % Dk;
      const int64_t off = static_cast<int64_t>(t0 + i) * a.sq.t + d;
      s.K[i * ldk + d] = to_f32(kp[off]);
      s.Q[i * ldk + d] = to_f32(qp[off]);
    }
    for (int idx = tid; idx < kC * kBV; idx += kThreads) {
      const int i = idx / kBV, j = idx % kBV;
      s.V[i * ldv + j] = j < nv ? to_f32(vp[static_cast<int64_t>(t0 + i) * a.sv.t + j]) : 0.f;
    }
    if (tid < 32) {
      // chunk-local inclusive cumsum of g, two tokens per lane (_gdn_full.py:63)
      float x0 = 0.f, x1 = 0.f;
      if (a.gate_mode != PTOF_GATE_NONE) {
        x0 = gp[static_cast<int64_t>(t0 + 2 * tid) * a.sg.t];
        x1 = gp[static_cast<int64_t>(t0 + 2 * tid + 1) * a.sg.t];
      }
      if (a.gate_mode == PTOF_GATE_RAW) {
        x1 += x0;
        float run = x1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, run, o);
          if (tid >= o) run += y;
        }
        const float excl = run - x1;
        x0 += excl;
        x1 = run;
      }
      s.g[2 * tid] = x0;
      s.g[2 * tid + 1] = x1;
      s.beta[2 * tid] = to_f32(bp[static_cast<int64_t>(t0 + 2 * tid) * a.sg.t]);
      s.beta[2 * tid + 1] = to_f32(bp[static_cast<int64_t>(t0 + 2 * tid + 1) * a.sg.t]);
    }
    __syncthreads();
    if (tid < kC) {
      // per-token exponentials, once per chunk (not per product term)
      const float gi = s.g[tid], e = expf(gi);
      s.eg[tid] = e;
      s.wk[tid] = s.beta[tid] * e;
      s.gam[tid] = expf(s.g[kC - 1] - gi);
    }

    // ---- A (strictly lower, gated) and Aqk (causal, gated) ----------------
    // Register tiles: thread (ti, tj) owns rows ti + 16 r and columns tj + 16 c
    // (r, c < 4) of both products and walks d four at a time; the 16 column rows a
    // warp reads are consecutive, so its float4 loads of K rows are conflict-free
    // (rows 4 apart would put 8 lanes on one bank with the 132-float row pitch).
    // Column block c > row block r lies wholly above the diagonal (j - i >= 1), so
    // those 6 of the 16 tiles are skipped.
    {
      const int ti = tid >> 4, tj = tid & 15;
      float ak[4][4], aq[4][4];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) ak[r][c] = aq[r][c] = 0.f;
#pragma unroll 2
      for (int d = 0; d < 4 * dk4; d += 4) {
        float4 ki[4], qi[4], kj[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          ki[r] = *reinterpret_cast<const float4*>(&s.K[(ti + 16 * r) * ldk + d]);
          qi[r] = *reinterpret_cast<const float4*>(&s.Q[(ti + 16 * r) * ldk + d]);
          kj[r] = *reinterpret_cast<const float4*>(&s.K[(tj + 16 * r) * ldk + d]);
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int c = 0; c <= r; ++c) {
            float x = ak[r][c], y = aq[r][c];
            x = fmaf(ki[r].x, kj[c].x, x); y = fmaf(qi[r].x, kj[c].x, y);
            x = fmaf(ki[r].y, kj[c].y, x); y = fmaf(qi[r].y, kj[c].y, y);
            x = fmaf(ki[r].z, kj[c].z, x); y = fmaf(qi[r].z, kj[c].z, y);
            x = fmaf(ki[r].w, kj[c].w, x); y = fmaf(qi[r].w, kj[c].w, y);
            ak[r][c] = x;
            aq[r][c] = y;
          }
      }
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int i = ti + 16 * r, j = tj + 16 * c;
          float akk = 0.f, aqk = 0.f;
          if (j <= i) {
            const float x = s.g[i] - s.g[j];
            if (j < i) akk = ak[r][c] * (x <= 0.f ? expf(x) : 0.f) * s.beta[i];
            aqk = aq[r][c] * expf(fminf(x, 0.f));
          }
          s.A[i * ldc + j] = akk;
          s.Aqk[i * ldc + j] = aqk;
        }
    }
    __syncthreads();

    // ---- T = (I + A)^-1: column j of T solves (I + A) x = e_j, and the 64 columns
    //      are independent. Warp w owns columns w + 8 m (m < 8), lane l rows l and
    //      l + 32 of each; a right-looking forward substitution walks k = 0..63: x_k is
    //      final once every row above it has been applied, is broadcast by a shuffle,
    //      and every row takes x_i -= A[i][k] x_k (A is strictly lower, so rows i <= k
    //      take zero). No block barrier inside the solve. ----
    {
      const int w = tid >> 5, l = tid & 31;
      constexpr int kCols = kC / (kThreads / 32);   // columns per warp
      float x0[kCols], x1[kCols];
#pragma unroll
      for (int m = 0; m < kCols; ++m) {
        const int j = w + 8 * m;
        x0[m] = (l == j) ? 1.f : 0.f;
        x1[m] = (l + 32 == j) ? 1.f : 0.f;
      }
#pragma unroll 2
      for (int k = 0; k < kC; ++k) {
        const float a0 = s.A[l * ldc + k], a1 = s.A[(l + 32) * ldc + k];
#pragma unroll
        for (int m = 0; m < kCols; ++m) {
          const float xk = __shfl_sync(0xffffffffu, k < 32 ? x0[m] : x1[m], k & 31);
          x0[m] = fmaf(-a0, xk, x0[m]);
          x1[m] = fmaf(-a1, xk, x1[m]);
        }
      }
#pragma unroll
      for (int m = 0; m < kCols; ++m) {
        const int j = w + 8 * m;
        s.Tm[l * ldc + j] = x0[m];
        s.Tm[(l + 32) * ldc + j] = x1[m];
      }
    }
    __syncthreads();

    // ---- W = T (k * beta * exp(g)),  U = T (v * beta) ----------------------
    // Every product below gives a thread rows i and i + 32 (or four state rows) of
    // one 4-column group: several independent accumulator chains per thread, one
    // float4 shared load of the shared operand feeding both rows. T, Aqk are zero
    // above the diagonal, so both rows run the longer row's j range; each output
    // element sums its terms in the same order as a plain row loop.
    for (int idx = tid; idx < (kC / 2) * dk4; idx += kThreads) {
      const int i = idx / dk4, d = (idx % dk4) * 4;
      float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
#pragma unroll 4
      for (int j = 0; j <= i + kC / 2; ++j) {
        const float wj = s.wk[j];
        const float t0 = s.Tm[i * ldc + j] * wj, t1 = s.Tm[(i + kC / 2) * ldc + j] * wj;
        const float4 kv = *reinterpret_cast<const float4*>(&s.K[j * ldk + d]);
        a0.x = fmaf(t0, kv.x, a0.x); a0.y = fmaf(t0, kv.y, a0.y);
        a0.z = fmaf(t0, kv.z, a0.z); a0.w = fmaf(t0, kv.w, a0.w);
        a1.x = fmaf(t1, kv.x, a1.x); a1.y = fmaf(t1, kv.y, a1.y);
        a1.z = fmaf(t1, kv.z, a1.z); a1.w = fmaf(t1, kv.w, a1.w);
      }
      *reinterpret_cast<float4*>(&s.W[i * ldk + d]) = a0;
      *reinterpret_cast<float4*>(&s.W[(i + kC / 2) * ldk + d]) = a1;
    }
    static_assert((kC / 2) * (kBV / 4) == kThreads, "one row pair and column group per thread");
    const int pi = tid / (kBV / 4), pj = (tid % (kBV / 4)) * 4;   // rows pi, pi + 32
    {
      float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
#pragma unroll 4
      for (int j = 0; j <= pi + kC / 2; ++j) {
        const float bj = s.beta[j];
        const float t0 = s.Tm[pi * ldc + j] * bj, t1 = s.Tm[(pi + kC / 2) * ldc + j] * bj;
        const float4 vv = *reinterpret_cast<const float4*>(&s.V[j * ldv + pj]);
        a0.x = fmaf(t0, vv.x, a0.x); a0.y = fmaf(t0, vv.y, a0.y);
        a0.z = fmaf(t0, vv.z, a0.z); a0.w = fmaf(t0, vv.w, a0.w);
        a1.x = fmaf(t1, vv.x, a1.x); a1.y = fmaf(t1, vv.y, a1.y);
        a1.z = fmaf(t1, vv.z, a1.z); a1.w = fmaf(t1, vv.w, a1.w);
      }
      *reinterpret_cast<float4*>(&s.U[pi * ldv + pj]) = a0;
      *reinterpret_cast<float4*>(&s.U[(pi + kC / 2) * ldv + pj]) = a1;
    }
    __syncthreads();

    // ---- v_new = U - W S --------------------------------------------------
    {
      float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
#pragma unroll 4
      for (int d = 0; d < Dk; ++d) {
        const float w0 = s.W[pi * ldk + d], w1 = s.W[(pi + kC / 2) * ldk + d];
        const float4 sv = *reinterpret_cast<const float4*>(&s.S[d * ldv + pj]);
        a0.x = fmaf(w0, sv.x, a0.x); a0.y = fmaf(w0, sv.y, a0.y);
        a0.z = fmaf(w0, sv.z, a0.z); a0.w = fmaf(w0, sv.w, a0.w);
        a1.x = fmaf(w1, sv.x, a1.x); a1.y = fmaf(w1, sv.y, a1.y);
        a1.z = fmaf(w1, sv.z, a1.z); a1.w = fmaf(w1, sv.w, a1.w);
      }
      const float4 u0 = *reinterpret_cast<const float4*>(&s.U[pi * ldv + pj]);
      const float4 u1 = *reinterpret_cast<const float4*>(&s.U[(pi + kC / 2) * ldv + pj]);
      *reinterpret_cast<float4*>(&s.Vn[pi * ldv + pj]) =
          make_float4(u0.x - a0.x, u0.y - a0.y, u0.z - a0.z, u0.w - a0.w);
      *reinterpret_cast<float4*>(&s.Vn[(pi + kC / 2) * ldv + pj]) =
          make_float4(u1.x - a1.x, u1.y - a1.y, u1.z - a1.z, u1.w - a1.w);
    }
    __syncthreads();

    // ---- o = scale * ((q S) * exp(g) + Aqk v_new) -------------------------
    {
      float qs[2][4] = {}, in[2][4] = {};
#pragma unroll 4
      for (int d = 0; d < Dk; ++d) {
        const float q0 = s.Q[pi * ldk + d], q1 = s.Q[(pi + kC / 2) * ldk + d];
        const float4 sv = *reinterpret_cast<const float4*>(&s.S[d * ldv + pj]);
        qs[0][0] = fmaf(q0, sv.x, qs[0][0]); qs[0][1] = fmaf(q0, sv.y, qs[0][1]);
        qs[0][2] = fmaf(q0, sv.z, qs[0][2]); qs[0][3] = fmaf(q0, sv.w, qs[0][3]);
        qs[1][0] = fmaf(q1, sv.x, qs[1][0]); qs[1][1] = fmaf(q1, sv.y, qs[1][1]);
        qs[1][2] = fmaf(q1, sv.z, qs[1][2]); qs[1][3] = fmaf(q1, sv.w, qs[1][3]);
      }
#pragma unroll 4
      for (int j = 0; j <= pi + kC / 2; ++j) {
        const float aq0 = s.Aqk[pi * ldc + j], aq1 = s.Aqk[(pi + kC / 2) * ldc + j];
        const float4 vn = *reinterpret_cast<const float4*>(&s.Vn[j * ldv + pj]);
        in[0][0] = fmaf(aq0, vn.x, in[0][0]); in[0][1] = fmaf(aq0, vn.y, in[0][1]);
        in[0][2] = fmaf(aq0, vn.z, in[0][2]); in[0][3] = fmaf(aq0, vn.w, in[0][3]);
        in[1][0] = fmaf(aq1, vn.x, in[1][0]); in[1][1] = fmaf(aq1, vn.y, in[1][1]);
        in[1][2] = fmaf(aq1, vn.z, in[1][2]); in[1][3] = fmaf(aq1, vn.w, in[1][3]);
      }
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int i = pi + h2 * (kC / 2);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float ov = a.scale * (qs[h2][e] * s.eg[i] + in[h2][e]);
          if (pj + e < nv) op[static_cast<int64_t>(t0 + i) * a.sv.t + pj + e] = from_f32<TO>(ov);
        }
      }
    }
    __syncthreads();

    // ---- S = exp(g_last) S + k^T (v_new * exp(g_last - g)) ----------------
    // thread: state rows d0 + 32 m (m < 4) of one 4-column group
    {
      const float egl = expf(s.g[kC - 1]);
      const int d0 = tid / (kBV / 4), jv = (tid % (kBV / 4)) * 4;
      float4 acc[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) acc[m] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 2
      for (int i = 0; i < kC; ++i) {
        const float gm = s.gam[i];
        const float4 vn = *reinterpret_cast<const float4*>(&s.Vn[i * ldv + jv]);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const float kg = s.K[i * ldk + d0 + 32 * m] * gm;
          acc[m].x = fmaf(kg, vn.x, acc[m].x); acc[m].y = fmaf(kg, vn.y, acc[m].y);
          acc[m].z = fmaf(kg, vn.z, acc[m].z); acc[m].w = fmaf(kg, vn.w, acc[m].w);
        }
      }
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int d = d0 + 32 * m;
        if (d < Dk) {
          float4* sp = reinterpret_cast<float4*>(&s.S[d * ldv + jv]);
          const float4 o = *sp;
          *sp = make_float4(fmaf(egl, o.x, acc[m].x), fmaf(egl, o.y, acc[m].y),
                            fmaf(egl, o.z, acc[m].z), fmaf(egl, o.w, acc[m].w));
        }
      }
    }
  }
  __syncthreads();
  if (a.S_final) {
    for (int idx = tid; idx < Dk * kBV; idx += kThreads) {
      const int d = idx / kBV, j = idx % kBV;
      if (j < nv) a.S_final[sbase + static_cast<int64_t>(d) * a.Dv + v0 + j] = s.S[d * ldv + j];
    }
  }
}

template <typename TI, typename TB, typename TO>
cudaError_t launch_typed(const Args& a, cudaStream_t stream) {
  auto kern = gdn_fwd_simt_kernel<TI, TB, TO>;
  const int smem = static_cast<int>(sizeof(Smem));
  cudaError_t e = set_smem_once(kern, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(a.B * a.H, (a.Dv + kBV - 1) / kBV);
  kern<<<grid, kThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

template <typename TI, typename TB>
cudaError_t launch_out(const Args& a, int out_dtype, cudaStream_t st) {
  switch (out_dtype) {
    case PTOF_F32: return launch_typed<TI, TB, float>(a, st);
    case PTOF_F16: return launch_typed<TI, TB, __half>(a, st);
    default: return launch_typed<TI, TB, __nv_bfloat16>(a, st);
  }
}
template <typename TI>
cudaError_t launch_beta(const Args& a, int beta_dtype, int out_dtype, cudaStream_t st) {
  switch (beta_dtype) {
    case PTOF_F32: return launch_out<TI, float>(a, out_dtype, st);
    case PTOF_F16: return launch_out<TI, __half>(a, out_dtype, st);
    default: return launch_out<TI, __nv_bfloat16>(a, out_dtype, st);
  }
}

}  // namespace simt

// Host entry used by the C ABI. Shapes are validated by the caller.
cudaError_t launch_gdn_fwd_simt(const ptof_gdn_params& p, const void* q, const void* k,
                                const void* v, const void* beta, const float* g,
                                const float* S0, void* o, float* S_final, cudaStream_t stream) {
  simt::Args a;
  a.q = q; a.k = k; a.v = v; a.beta = beta; a.g = g; a.S0 = S0; a.o = o; a.S_final = S_final;
  a.B = p.B; a.H = p.H; a.T = p.T; a.Dk = p.Dk; a.Dv = p.Dv;
  a.gate_mode = p.gate_mode;
  a.scale = p.scale;
  a.sq = make_strides4(p.layout, p.H, p.T, p.Dk);
  a.sv = make_strides4(p.layout, p.H, p.T, p.Dv);
  a.sg = make_strides3(p.layout, p.H, p.T);
  switch (p.in_dtype) {
    case PTOF_F32: return simt::launch_beta<float>(a, p.beta_dtype, p.out_dtype, stream);
    case PTOF_F16: return simt::launch_beta<__half>(a, p.beta_dtype, p.out_dtype, stream);
    default: return simt::launch_beta<__nv_bfloat16>(a, p.beta_dtype, p.out_dtype, stream);
  }
}

bool gdn_fwd_simt_supports(const ptof_gdn_params& p) {
  return p.C == kChunk && p.Dk >= 1 && p.Dk <= simt::kMaxDk && p.Dv >= 1;
}

}  // namespace ptof
