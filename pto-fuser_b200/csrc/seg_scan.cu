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
// (Xfinal). One CTA owns 16 or 32 state columns of one head: the columns stay in
// shared memory across segments and A_j streams into shared memory (double-buffered)
// once per segment, so the work per segment is one [Dk,Dk] x [Dk,cols] fp32 product. The same kernel
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

constexpr int kThreads = 256;
constexpr int kMinCols = 16;           // Dv granularity

// 16-byte asynchronous global -> shared copy (completion by cp.async.wait_group)
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Thread tile: R = D (COLS / 4) / 256 rows x 4 columns (thread t: columns
// 4 (t % (COLS / 4)), rows R (t / (COLS / 4))); a head's state spreads over Dv / COLS
// CTAs. Every CTA streams the whole A_j, so fewer columns per CTA only pay while the
// grid would leave SMs idle (the launch picks 16 then, else 32). A_j rows are padded
// to D + 4 floats so the R rows a warp reads at one k fall in different banks; A_{j+1}
// streams into the second buffer (cp.async) while A_j is applied.
template <int D, int COLS>
struct SLayout {
  static constexpr int AP = D + 4;                       // padded A row (floats)
  static constexpr int A_FLOATS = D * AP;
  static constexpr int BYTES = (2 * A_FLOATS + D * COLS) * 4;
};

template <int D>
__device__ __forceinline__ void load_a_async(float* As, const float* a, int t) {
  constexpr int AP = D + 4;
#pragma unroll 4
  for (int e = t; e < D * D / 4; e += kThreads) {
    const int row = e / (D / 4), c4 = e % (D / 4);
    cp_async16(As + row * AP + 4 * c4, a + static_cast<int64_t>(row) * D + 4 * c4);
  }
  cp_async_commit();
}

template <int D, int COLS>
__global__ void __launch_bounds__(kThreads) seg_scan_kernel(Params p) {
  using SL = SLayout<D, COLS>;
  constexpr int AP = SL::AP;
  constexpr int kCols = COLS, kGroups = COLS / 4;        // 4-column thread groups
  constexpr int R = D * kGroups / kThreads;              // rows per thread
  extern __shared__ __align__(16) float smem[];
  float* Abuf = smem;                                    // 2 x [D][AP]
  float* cur = smem + 2 * SL::A_FLOATS;                  // [D][kCols] running state columns
  const int head = blockIdx.x;
  const int c0 = blockIdx.y * kCols;
  const int t = threadIdx.x;
  const int cq = (t % kGroups) * 4;                      // this thread's 4 columns
  const int r0 = (t / kGroups) * R;                      // and R rows
  const int Dv = p.Dv;

  if (p.nseg > 0) load_a_async<D>(Abuf, p.A + head * p.a_hs, t);
  const float* x0 = p.X0 ? p.X0 + head * p.x0_hs : nullptr;
  for (int e = t; e < D * kCols / 4; e += kThreads) {
    const int row = e / (kCols / 4), c4 = (e % (kCols / 4)) * 4;
    const float4 x = x0 ? *reinterpret_cast<const float4*>(x0 + static_cast<int64_t>(row) * Dv + c0 + c4)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4*>(cur + row * kCols + c4) = x;
  }

  for (int j = 0; j < p.nseg; ++j) {
    float* As = Abuf + (j & 1) * SL::A_FLOATS;
    cp_async_wait_all();
    __syncthreads();                                     // A_j and cur complete
    if (j + 1 < p.nseg)
      load_a_async<D>(Abuf + ((j + 1) & 1) * SL::A_FLOATS, p.A + head * p.a_hs + (j + 1) * p.a_ss, t);
    if (p.Xout) {
      float* xo = p.Xout + head * p.xo_hs + j * p.xo_ss;
#pragma unroll
      for (int i = 0; i < R; ++i)
        *reinterpret_cast<float4*>(xo + static_cast<int64_t>(r0 + i) * Dv + c0 + cq) =
            *reinterpret_cast<const float4*>(cur + (r0 + i) * kCols + cq);
    }
    float acc[R][4];
    if (p.Bv) {
      const float* b = p.Bv + head * p.b_hs + j * p.b_ss;
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const float4 v = *reinterpret_cast<const float4*>(b + static_cast<int64_t>(r0 + i) * Dv + c0 + cq);
        acc[i][0] = v.x; acc[i][1] = v.y; acc[i][2] = v.z; acc[i][3] = v.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < R; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    }
#pragma unroll 2
    for (int k = 0; k < D; k += 4) {
      float4 s4[4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) s4[kk] = *reinterpret_cast<const float4*>(cur + (k + kk) * kCols + cq);
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const float4 a = *reinterpret_cast<const float4*>(As + (r0 + i) * AP + k);
        const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          acc[i][0] = fmaf(av[kk], s4[kk].x, acc[i][0]);
          acc[i][1] = fmaf(av[kk], s4[kk].y, acc[i][1]);
          acc[i][2] = fmaf(av[kk], s4[kk].z, acc[i][2]);
          acc[i][3] = fmaf(av[kk], s4[kk].w, acc[i][3]);
        }
      }
    }
    __syncthreads();                                     // every thread has read cur
#pragma unroll
    for (int i = 0; i < R; ++i)
      *reinterpret_cast<float4*>(cur + (r0 + i) * kCols + cq) =
          make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
  }
  __syncthreads();
  if (p.Xf) {
    float* xf = p.Xf + head * p.xf_hs;
#pragma unroll
    for (int i = 0; i < R; ++i)
      *reinterpret_cast<float4*>(xf + static_cast<int64_t>(r0 + i) * Dv + c0 + cq) =
          *reinterpret_cast<const float4*>(cur + (r0 + i) * kCols + cq);
  }
}

template <int D, int COLS>
int launch_c(const Params& p, int heads, cudaStream_t st) {
  const int smem = SLayout<D, COLS>::BYTES;
  cudaError_t e = set_smem_once(seg_scan_kernel<D, COLS>, smem);
  if (e != cudaSuccess) return cuda_fail(e, "seg_scan smem attribute");
  seg_scan_kernel<D, COLS><<<dim3(heads, p.Dv / COLS), kThreads, smem, st>>>(p);
  e = cudaGetLastError();
  return e == cudaSuccess ? PTOF_OK : cuda_fail(e, "seg_scan launch");
}

template <int D>
int launch(const Params& p, int heads, cudaStream_t st) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // one CTA per SM (the A double buffer fills shared memory)
  const bool wide = p.Dv % 32 == 0 && static_cast<int64_t>(heads) * (p.Dv / 32) >= sms;
  return wide ? launch_c<D, 32>(p, heads, st) : launch_c<D, 16>(p, heads, st);
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
  if (heads < 1 || heads > 65535 || nseg < 0 || (D != 64 && D != 128) || Dv < segscan::kMinCols ||
      Dv % segscan::kMinCols || Dv / segscan::kMinCols > 65535)
    return fail(PTOF_EINVAL, "seg_scan shape heads=%d nseg=%d D=%d Dv=%d (D in {64,128}, "
                "Dv a multiple of 16)", heads, nseg, D, Dv);
  if (nseg > 0 && !A) return fail(PTOF_EINVAL, "seg_scan: A is NULL with nseg=%d", nseg);
  if (!Xout && !Xfinal) return fail(PTOF_EINVAL, "seg_scan: no output (Xout and Xfinal NULL)");
  if (a_head_stride < 0 || a_seg_stride < 0 || b_head_stride < 0 || b_seg_stride < 0 ||
      x0_head_stride < 0 || xout_head_stride < 0 || xout_seg_stride < 0 || xfinal_head_stride < 0)
    return fail(PTOF_EINVAL, "seg_scan: negative stride");
  if ((a_head_stride | a_seg_stride | b_head_stride | b_seg_stride | x0_head_stride |
       xout_head_stride | xout_seg_stride | xfinal_head_stride) & 3)
    return fail(PTOF_EALIGN, "seg_scan: strides must be multiples of 4 floats");
  for (const void* q : {static_cast<const void*>(A), static_cast<const void*>(Bv),
                        static_cast<const void*>(X0), static_cast<const void*>(Xout),
                        static_cast<const void*>(Xfinal)})
    if (reinterpret_cast<uintptr_t>(q) & 15) return fail(PTOF_EALIGN, "seg_scan: pointer not 16-byte aligned");
  segscan::Params p{A, a_head_stride, a_seg_stride, Bv, b_head_stride, b_seg_stride,
                    X0, x0_head_stride, Xout, xout_head_stride, xout_seg_stride,
                    Xfinal, xfinal_head_stride, nseg, Dv};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return D == 128 ? segscan::launch<128>(p, heads, st) : segscan::launch<64>(p, heads, st);
}
