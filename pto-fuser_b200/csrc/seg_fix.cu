// Output fix-up of the chunk-segment scan: o += o^A X per token segment.
//
// The GDN output of a segment is affine in its entry state: o = o^B + o^A X, where
// o^B is the forward's output started from a zero state and o^A [Tseg, Dk] its output
// started from S0 = I with v = 0 (both written by the fused forward), and X [Dk, Dv]
// is the segment's true entry state. This kernel applies the linear part in place on
// o (holding o^B), per 128-token tile on the tensor cores:
//
//   D[128, Dv] (TMEM, fp32) = o^A tile [128, Dk] (bf16/f16, K-major, TMA)
//                             x X [Dk, Dv] (fp32 -> bf16/f16, MN-major, staged once per
//                               segment a CTA touches)
//   o tile = o^B tile (TMA) + D, stored back with a TMA tensor store.
//
// Persistent CTAs (one per SM) walk contiguous tile ranges, so a CTA restages X only
// when its range crosses a segment boundary. Roles (320 threads):
//   warp 4  producer: TMA loads of o^A and o^B tiles (2 stages for D = 128, 4 for D = 64)
//   warp 5  TMEM owner and UMMA issuer (one thread; two accumulators)
//   warps 6-9 X staging: fp32 -> 16-bit, two buffers
//   warps 0-3 epilogue: TMEM -> registers, + o^B from shared memory, TMA store.
// HBM-bound: per token 2 Dk bytes of o^A read, 2 Dv bytes of o read and written.
#include <cuda_runtime.h>

#include "capi_internal.h"
#include "common.cuh"
#include "ptx.cuh"

namespace ptof {
namespace segfix {

constexpr int kRows = 128;
constexpr int kThreads = 320;

template <int D>
struct FLayout {
  static constexpr int NKB = D / 64;
  static constexpr int TILE = NKB * kRows * 128;   // [128 tokens x D] 16-bit, SW128 blocks
  static constexpr int XT = NKB * D * 128;         // X [D k-rows x D n], n-blocks of 64
  // input stages (o^A and o^B tiles) and X buffers (double-buffered, so X restaging
  // overlaps the previous unit's tiles): four stages for D = 64, two for D = 128
  // (three beside a single X measured no faster once X staging had its own warps)
  static constexpr int NS = (D == 128) ? 2 : 4;
  static constexpr int NX = 2;
  static constexpr int OFF_OA = 0;
  static constexpr int OFF_OB = NS * TILE;
  static constexpr int OFF_X = 2 * NS * TILE;
  static constexpr int OFF_BAR = OFF_X + NX * XT;
  static constexpr int BYTES = OFF_BAR + 256 + 1024;
  static_assert(BYTES <= 227 * 1024, "seg_fix shared memory");
  static constexpr int TCOLS = 2 * D;
};

enum FBar { F_FULL0 = 0, F_EMPTY0 = 4, F_TFULL0 = 8, F_TFREE0 = 10, F_XFULL0 = 12, F_XFREE0 = 14,
            F_DONE = 16, F_COUNT = 17 };
static_assert(F_COUNT * 8 + 8 <= 256, "barrier area");

struct FParams {
  CUtensorMap mapOA, mapO;
  const float* X;      // [units][D][D] fp32 entry states
  int* status;
  int64_t tiles;       // units * tiles_per_unit
  int tiles_per_unit;
  int view_segs;       // > 0: o is a strided view, mapO 4D {D, Tseg, segs, pairs}
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreads, 1) seg_fix_kernel(const __grid_constant__ FParams P) {
  using L = FLayout<D>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t sbase = smem_u32(smem_raw);
  unsigned char* sm = smem_raw + (((sbase + 1023u) & ~1023u) - sbase);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + F_COUNT);
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t t0 = P.tiles * blockIdx.x / gridDim.x;
  const int64_t cnt = P.tiles * (blockIdx.x + 1) / gridDim.x - t0;

  if (tid == 0) {
    abort_flag = 0;
    for (int i = 0; i < F_COUNT; ++i) mbar_init(&bars[i], 1);
    mbar_init(&bars[F_TFREE0], 4);   // one arrival per epilogue warp
    mbar_init(&bars[F_TFREE0 + 1], 4);
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, L::TCOLS);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto wait = [&](uint64_t* bar, uint32_t par, int site) {
    if (mbar_try_wait(bar, par)) return true;
    return mbar_wait(bar, par, &abort_flag, P.status, site);
  };
  auto unit_of = [&](int64_t i) { return static_cast<int>((t0 + i) / P.tiles_per_unit); };

  if (warp == 4) {
    // ================================ producer ================================
    if (lane == 0) {
      prefetch_tmap(&P.mapOA);
      prefetch_tmap(&P.mapO);
    }
    int64_t issued = 0;    // tiles whose loads were issued
    for (int64_t i = 0; i < cnt; ++i) {
      const int s = static_cast<int>(i % L::NS);
      // after a wait gave up (here or in another warp) no further load is issued; the
      // decision is warp-uniform
      bool ok = i < L::NS ||
                wait(&bars[F_EMPTY0 + s], static_cast<uint32_t>(((i / L::NS) + 1) & 1), 1);
      if (!__all_sync(0xffffffffu, ok && !abort_flag)) break;
      issued = i + 1;
      if (lane == 0) {
        const int y = static_cast<int>((t0 + i) * kRows);
        mbar_arrive_expect_tx(&bars[F_FULL0 + s], 2 * L::TILE);
        const int64_t tile = t0 + i;
        const int u = static_cast<int>(tile / P.tiles_per_unit);
        const int r = static_cast<int>(tile % P.tiles_per_unit) * kRows;
#pragma unroll
        for (int kb = 0; kb < L::NKB; ++kb) {
          tma_load_2d(sm + L::OFF_OA + s * L::TILE + kb * kRows * 128, &P.mapOA,
                      &bars[F_FULL0 + s], kb * 64, y);
          if (P.view_segs > 0)
            tma_load_4d(sm + L::OFF_OB + s * L::TILE + kb * kRows * 128, &P.mapO,
                        &bars[F_FULL0 + s], kb * 64, r, u % P.view_segs, u / P.view_segs);
          else
            tma_load_2d(sm + L::OFF_OB + s * L::TILE + kb * kRows * 128, &P.mapO,
                        &bars[F_FULL0 + s], kb * 64, y);
        }
      }
    }
    // drain: the CTA must not exit (or release its shared memory) with TMA loads in
    // flight, so wait (bounded, also after an abort) for the last NS tiles' loads
    if (lane == 0) {
      for (int64_t i = issued > L::NS ? issued - L::NS : 0; i < issued; ++i) {
        const uint64_t t_0 = globaltimer_ns();
        while (!mbar_try_wait(&bars[F_FULL0 + i % L::NS], static_cast<uint32_t>((i / L::NS) & 1)) &&
               globaltimer_ns() - t_0 < kWaitTimeoutNs) {
        }
      }
    }
  } else if (warp == 5) {
    // ============================== UMMA issuer ===============================
    if (lane == 0) {
      constexpr uint32_t ID = idesc_f16(kRows, D, false, true, BF16);
      int cur = -1, f = -1;
      for (int64_t i = 0; i < cnt; ++i) {
        const int s = static_cast<int>(i % L::NS), b = static_cast<int>(i & 1);
        const int u = unit_of(i);
        if (u != cur) {
          if (f >= 0) umma_commit(&bars[F_XFREE0 + f % L::NX]);   // old X no longer read
          ++f;
          if (!wait(&bars[F_XFULL0 + f % L::NX], static_cast<uint32_t>((f / L::NX) & 1), 3)) break;
          cur = u;
        }
        if (!wait(&bars[F_FULL0 + s], static_cast<uint32_t>((i / L::NS) & 1), 4)) break;
        if (i >= 2 && !wait(&bars[F_TFREE0 + b], static_cast<uint32_t>(((i >> 1) + 1) & 1), 5))
          break;
        tc_fence_after();
        const uint32_t a = smem_u32(sm + L::OFF_OA + s * L::TILE);
        const uint32_t x = smem_u32(sm + L::OFF_X + (f % L::NX) * L::XT);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          umma_ss(tmem + b * D, sdesc_sw128(a + (ks >> 2) * (kRows * 128) + (ks & 3) * 32, 16, 1024),
                  sdesc_sw128(x + ks * 2048, D * 128, 1024), ID, ks > 0);
        umma_commit(&bars[F_TFULL0 + b]);
      }
      if (f >= 0) umma_commit(&bars[F_XFREE0 + f % L::NX]);
      umma_commit(&bars[F_DONE]);   // arrives once every UMMA issued above has retired
    }
  } else if (warp >= 6) {
    // ================================ X staging ===============================
    // one fill per unit the CTA's tile range touches, in the issuer's order; the
    // break decisions are uniform over the group (barrier OR)
    const int xt = tid - 6 * 32;
    const int u_first = unit_of(0), u_end = cnt > 0 ? unit_of(cnt - 1) + 1 : u_first;
    for (int u = u_first, f = 0; u < u_end; ++u, ++f) {
      const int xb = f % L::NX;
      const bool ok = f < L::NX ||
                      wait(&bars[F_XFREE0 + xb], static_cast<uint32_t>(((f / L::NX) + 1) & 1), 2);
      if (named_bar_or(2, 128, !ok || abort_flag != 0)) break;
      // X[k][n] fp32 -> 16-bit, MN-major SW128: n-block n/64, row k, byte 2 (n % 64)
      unsigned char* xs = sm + L::OFF_X + xb * L::XT;
      const float4* xg = reinterpret_cast<const float4*>(P.X + static_cast<int64_t>(u) * D * D);
      constexpr int PER = D * D / 4 / 128;   // float4s per thread
      static_assert(PER % 8 == 0, "X staging batches");
#pragma unroll 1
      for (int j0 = 0; j0 < PER; j0 += 8) {
        float4 x[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) x[j] = __ldg(xg + (j0 + j) * 128 + xt);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int idx = (j0 + j) * 128 + xt;
          const int k = idx / (D / 4), n = (idx % (D / 4)) * 4;
          const uint32_t lo = BF16 ? pack_bf16(x[j].x, x[j].y) : pack_f16(x[j].x, x[j].y);
          const uint32_t hi = BF16 ? pack_bf16(x[j].z, x[j].w) : pack_f16(x[j].z, x[j].w);
          *reinterpret_cast<uint2*>(xs + (n >> 6) * (D * 128) + sw128_off(k, (n & 63) * 2)) =
              make_uint2(lo, hi);
        }
      }
      fence_async_smem();
      named_bar_sync(3, 128);
      if (xt == 0) mbar_arrive(&bars[F_XFULL0 + xb]);
    }
  } else {
    // =============================== epilogue =================================
    const int r = tid;   // tile row = TMEM lane
    for (int64_t i = 0; i < cnt; ++i) {
      const int s = static_cast<int>(i % L::NS), b = static_cast<int>(i & 1);
      // o^B visible, then the product (after an abort the waits return at once and
      // the barrier below ends the loop for the whole warpgroup)
      wait(&bars[F_FULL0 + s], static_cast<uint32_t>((i / L::NS) & 1), 6);
      wait(&bars[F_TFULL0 + b], static_cast<uint32_t>((i >> 1) & 1), 7);
      tc_fence_after();
      unsigned char* ob = sm + L::OFF_OB + s * L::TILE;
#pragma unroll 1
      for (int cc = 0; cc < D / 16; ++cc) {
        float v[16];
        tmem_ld16(tmem + b * D + cc * 16 + ((32u * warp) << 16), v);
        tmem_wait_ld();
        unsigned char* row = ob + (cc >> 2) * (kRows * 128);
        const uint32_t o0 = sw128_off(r, (cc & 3) * 32), o1 = sw128_off(r, (cc & 3) * 32 + 16);
        uint4 p0 = *reinterpret_cast<const uint4*>(row + o0);
        uint4 p1 = *reinterpret_cast<const uint4*>(row + o1);
        uint32_t* w0 = reinterpret_cast<uint32_t*>(&p0);
        uint32_t* w1 = reinterpret_cast<uint32_t*>(&p1);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 a0 = BF16 ? unpack_bf16(w0[e]) : unpack_f16(w0[e]);
          const float2 a1 = BF16 ? unpack_bf16(w1[e]) : unpack_f16(w1[e]);
          w0[e] = BF16 ? pack_bf16(a0.x + v[2 * e], a0.y + v[2 * e + 1])
                       : pack_f16(a0.x + v[2 * e], a0.y + v[2 * e + 1]);
          w1[e] = BF16 ? pack_bf16(a1.x + v[8 + 2 * e], a1.y + v[9 + 2 * e])
                       : pack_f16(a1.x + v[8 + 2 * e], a1.y + v[9 + 2 * e]);
        }
        *reinterpret_cast<uint4*>(row + o0) = p0;
        *reinterpret_cast<uint4*>(row + o1) = p1;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[F_TFREE0 + b]);
      fence_async_smem();
      // the tile is complete in shared memory; the OR over the warpgroup gives every
      // thread the same answer, so an abort never stores a partial tile
      if (named_bar_or(1, 128, abort_flag != 0)) break;
      if (tid == 0) {
        const int y = static_cast<int>((t0 + i) * kRows);
        const int64_t tile = t0 + i;
        const int u = static_cast<int>(tile / P.tiles_per_unit);
        const int r = static_cast<int>(tile % P.tiles_per_unit) * kRows;
#pragma unroll
        for (int kb = 0; kb < L::NKB; ++kb) {
          if (P.view_segs > 0)
            tma_store_4d(&P.mapO, ob + kb * kRows * 128, kb * 64, r, u % P.view_segs,
                         u / P.view_segs);
          else
            tma_store_2d(&P.mapO, ob + kb * kRows * 128, kb * 64, y);
        }
        bulk_commit();
        bulk_wait_read0();
        mbar_arrive(&bars[F_EMPTY0 + s]);
      }
    }
    if (tid == 0) bulk_wait0();
  }
  if (warp == 5 && lane == 0) {
    // every UMMA has retired before TMEM is released (bounded, also after an abort)
    const uint64_t t_0 = globaltimer_ns();
    while (!mbar_try_wait(&bars[F_DONE], 0) && globaltimer_ns() - t_0 < kWaitTimeoutNs) {
    }
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, L::TCOLS);
}

template <int D, bool BF16>
int launch_t(int* status, void* o, const void* oa, const float* X, int units, int Tseg,
             cudaStream_t st, int view_segs = 0, long long o_pair = 0, long long o_seg = 0) {
  FParams P;
  const CUtensorMapDataType t = BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t rows = static_cast<uint64_t>(units) * Tseg;
  int rc = make_tmap_2d(&P.mapOA, oa, t, 2, D, rows, static_cast<uint64_t>(D) * 2, 64, kRows,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) {
    if (view_segs > 0) {
      // o strided: unit (pair, seg) starts at token pair*o_pair + seg*o_seg
      const uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(Tseg),
                                static_cast<uint64_t>(view_segs),
                                static_cast<uint64_t>(units / view_segs)};
      const uint64_t strides[3] = {static_cast<uint64_t>(D) * 2,
                                   static_cast<uint64_t>(o_seg) * D * 2,
                                   static_cast<uint64_t>(o_pair) * D * 2};
      const uint32_t box[4] = {64, static_cast<uint32_t>(kRows), 1, 1};
      rc = make_tmap_4d(&P.mapO, o, t, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    } else {
      rc = make_tmap_2d(&P.mapO, o, t, 2, D, rows, static_cast<uint64_t>(D) * 2, 64, kRows,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    }
  }
  if (rc) return rc;
  P.view_segs = view_segs;
  P.X = X;
  P.status = status;
  P.tiles_per_unit = Tseg / kRows;
  P.tiles = static_cast<int64_t>(units) * P.tiles_per_unit;
  auto kern = seg_fix_kernel<D, BF16>;
  const int bytes = FLayout<D>::BYTES;
  cudaError_t e = set_smem_once(kern, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "seg_fix smem attribute");
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t grid = P.tiles < sms ? P.tiles : sms;
  kern<<<static_cast<unsigned>(grid), kThreads, bytes, st>>>(P);
  e = cudaGetLastError();
  return e == cudaSuccess ? PTOF_OK : cuda_fail(e, "seg_fix launch");
}

}  // namespace segfix
}  // namespace ptof

using namespace ptof;

int ptof_seg_fix_exec(void* ws, void* o, const void* oa, const float* X, int units, int Tseg,
                      int D, int dtype, void* stream) {
  Workspace* w = static_cast<Workspace*>(ws);
  if (units < 1 || Tseg < segfix::kRows || Tseg % segfix::kRows || (D != 64 && D != 128) ||
      static_cast<int64_t>(units) * Tseg > (1LL << 31) - segfix::kRows)
    return fail(PTOF_EINVAL, "seg_fix shape units=%d Tseg=%d D=%d (Tseg a multiple of 128, "
                "D 64 or 128)", units, Tseg, D);
  if (dtype != PTOF_BF16 && dtype != PTOF_F16) return fail(PTOF_EINVAL, "seg_fix dtype");
  int rc = check_ptrs({o, oa, X}, {});
  if (rc) return rc;
  int* status = w ? w->d_status : nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf = dtype == PTOF_BF16;
  if (D == 128)
    return bf ? segfix::launch_t<128, true>(status, o, oa, X, units, Tseg, st)
              : segfix::launch_t<128, false>(status, o, oa, X, units, Tseg, st);
  return bf ? segfix::launch_t<64, true>(status, o, oa, X, units, Tseg, st)
            : segfix::launch_t<64, false>(status, o, oa, X, units, Tseg, st);
}

// The same fix-up with o a strided view (the chunk-segment scan inside one GPU writes
// its tail segments straight into the caller's o): o^A and X are contiguous
// [pairs * segs, Tseg, D] / [pairs * segs, D, D]; unit (pair, seg) of o starts at token
// pair * o_pair_stride + seg * o_seg_stride of o's buffer.
int ptof_seg_fix_exec_view(void* ws, void* o, const void* oa, const float* X, int pairs, int segs,
                           int Tseg, int D, int dtype, long long o_pair_stride,
                           long long o_seg_stride, void* stream) {
  Workspace* w = static_cast<Workspace*>(ws);
  if (pairs < 1 || segs < 1 || Tseg < segfix::kRows || Tseg % segfix::kRows ||
      (D != 64 && D != 128) || o_pair_stride < 1 || o_seg_stride < 1 ||
      static_cast<int64_t>(pairs) * segs * Tseg > (1LL << 31) - segfix::kRows)
    return fail(PTOF_EINVAL, "seg_fix view shape pairs=%d segs=%d Tseg=%d D=%d", pairs, segs,
                Tseg, D);
  if (dtype != PTOF_BF16 && dtype != PTOF_F16) return fail(PTOF_EINVAL, "seg_fix dtype");
  int rc = check_ptrs({o, oa, X}, {});
  if (rc) return rc;
  int* status = w ? w->d_status : nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf = dtype == PTOF_BF16;
  const int units = pairs * segs;
  if (D == 128)
    return bf ? segfix::launch_t<128, true>(status, o, oa, X, units, Tseg, st, segs, o_pair_stride, o_seg_stride)
              : segfix::launch_t<128, false>(status, o, oa, X, units, Tseg, st, segs, o_pair_stride, o_seg_stride);
  return bf ? segfix::launch_t<64, true>(status, o, oa, X, units, Tseg, st, segs, o_pair_stride, o_seg_stride)
            : segfix::launch_t<64, false>(status, o, oa, X, units, Tseg, st, segs, o_pair_stride, o_seg_stride);
}
