// Segment-state combine of the chunked GDN recurrence (affine prefix over segments).
//
// Over one contiguous token segment the delta-rule state map is affine in the entry
// state: S_out = A S_in + B, with A [Dk,Dk] the segment's transition (the final state
// of a forward started from S0 = I with v = 0) and B [Dk,Dv] its offset (the final
// state started from S0 = 0). Given (A_j, B_j) for segments j = 0..nseg-1 of every
// head, this kernel applies them in order to an entry state X0:
//
//   X_0 = X0 (or 0),   X_{j+1} = A_j X_j (+ B_j)
//
// writing the entry state X_j of every segment (Xout) and the exit state X_nseg
// (Xfinal). One CTA owns 32 state columns of one head: the columns stay in shared
// memory across segments and A_j is staged into shared memory once per segment, so
// the work per segment is one [Dk,Dk] x [Dk,32] fp32 product. The same kernel
// composes two maps (A1,B1) o (A0,B0) = (A1 A0, A1 B0 + B1) by scanning X0 = A0 with
// no offset and X0 = B0 with offset B1.
#include <cstdint>

#include "capi_internal.h"

namespace ptof {
namespace segscan {

struct Params {
  const float* A; int64_t a_hs, a_ss;      // [heads][nseg][D][D] by strides (floats)
  const float* Bv; int64_t b_hs, b_ss;     // [heads][nseg][D][Dv] or null (no offset)
  const float* X0; int64_t x0_hs;          // [heads][D][Dv] or null (zero entry state)
  float* Xout; int64_t xo_hs, xo_ss;       // [heads][nseg][D][Dv] entry states or null
  float* Xf; int64_t xf_hs;                // [heads][D][Dv] exit state or null
  int nseg, Dv;
};

constexpr int kCols = 32;
constexpr int kThreads = 256;

template <int D>
__global__ void __launch_bounds__(kThreads) seg_scan_kernel(Params p) {
  extern __shared__ float smem[];
  float* As = smem;               // [D][D] transition of the current segment
  float* cur = smem + D * D;      // [D][kCols] running state columns
  constexpr int R = D / (kThreads / kCols);   // rows per thread
  const int head = blockIdx.x;
  const int c0 = blockIdx.y * kCols;
  const int t = threadIdx.x;
  const int c = t % kCols;
  const int r0 = (t / kCols) * R;
  const int Dv = p.Dv;

  const float* x0 = p.X0 ? p.X0 + head * p.x0_hs : nullptr;
#pragma unroll
  for (int i = 0; i < R; ++i)
    cur[(r0 + i) * kCols + c] = x0 ? x0[(int64_t)(r0 + i) * Dv + c0 + c] : 0.f;
  __syncthreads();

  for (int j = 0; j < p.nseg; ++j) {
    if (p.Xout) {
      float* xo = p.Xout + head * p.xo_hs + j * p.xo_ss;
#pragma unroll
      for (int i = 0; i < R; ++i) xo[(int64_t)(r0 + i) * Dv + c0 + c] = cur[(r0 + i) * kCols + c];
    }
    const float* a = p.A + head * p.a_hs + j * p.a_ss;
    for (int e = t; e < D * D; e += kThreads) As[e] = a[e];
    float acc[R];
    if (p.Bv) {
      const float* b = p.Bv + head * p.b_hs + j * p.b_ss;
#pragma unroll
      for (int i = 0; i < R; ++i) acc[i] = b[(int64_t)(r0 + i) * Dv + c0 + c];
    } else {
#pragma unroll
      for (int i = 0; i < R; ++i) acc[i] = 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int k = 0; k < D; ++k) {
      const float s = cur[k * kCols + c];
#pragma unroll
      for (int i = 0; i < R; ++i) acc[i] = fmaf(As[(r0 + i) * D + k], s, acc[i]);
    }
    __syncthreads();   // every thread has read cur and As
#pragma unroll
    for (int i = 0; i < R; ++i) cur[(r0 + i) * kCols + c] = acc[i];
    __syncthreads();
  }
  if (p.Xf) {
    float* xf = p.Xf + head * p.xf_hs;
#pragma unroll
    for (int i = 0; i < R; ++i) xf[(int64_t)(r0 + i) * Dv + c0 + c] = cur[(r0 + i) * kCols + c];
  }
}

template <int D>
int launch(const Params& p, int heads, cudaStream_t st) {
  const int smem = (D * D + D * kCols) * static_cast<int>(sizeof(float));
  cudaError_t e = set_smem_once(seg_scan_kernel<D>, smem);
  if (e != cudaSuccess) return cuda_fail(e, "seg_scan smem attribute");
  seg_scan_kernel<D><<<dim3(heads, p.Dv / kCols), kThreads, smem, st>>>(p);
  e = cudaGetLastError();
  return e == cudaSuccess ? PTOF_OK : cuda_fail(e, "seg_scan launch");
}

}  // namespace segscan
}  // namespace ptof

using namespace ptof;

int ptof_seg_scan_exec(const float* A, int64_t a_head_stride, int64_t a_seg_stride,
                       const float* Bv, int64_t b_head_stride, int64_t b_seg_stride,
                       const float* X0, int64_t x0_head_stride, float* Xout,
                       int64_t xout_head_stride, int64_t xout_seg_stride, float* Xfinal,
                       int64_t xfinal_head_stride, int heads, int nseg, int D, int Dv,
                       void* stream) {
  if (heads < 1 || heads > 65535 || nseg < 0 || (D != 64 && D != 128) || Dv < segscan::kCols ||
      Dv % segscan::kCols || Dv / segscan::kCols > 65535)
    return fail(PTOF_EINVAL, "seg_scan shape heads=%d nseg=%d D=%d Dv=%d (D in {64,128}, "
                "Dv a multiple of 32)", heads, nseg, D, Dv);
  if (nseg > 0 && !A) return fail(PTOF_EINVAL, "seg_scan: A is NULL with nseg=%d", nseg);
  if (!Xout && !Xfinal) return fail(PTOF_EINVAL, "seg_scan: no output (Xout and Xfinal NULL)");
  if (a_head_stride < 0 || a_seg_stride < 0 || b_head_stride < 0 || b_seg_stride < 0 ||
      x0_head_stride < 0 || xout_head_stride < 0 || xout_seg_stride < 0 || xfinal_head_stride < 0)
    return fail(PTOF_EINVAL, "seg_scan: negative stride");
  segscan::Params p{A, a_head_stride, a_seg_stride, Bv, b_head_stride, b_seg_stride,
                    X0, x0_head_stride, Xout, xout_head_stride, xout_seg_stride,
                    Xfinal, xfinal_head_stride, nseg, Dv};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return D == 128 ? segscan::launch<128>(p, heads, st) : segscan::launch<64>(p, heads, st);
}
