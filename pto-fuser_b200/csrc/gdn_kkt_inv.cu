// The kkt + triangular-inverse stage on its own (the first two stages of the chunked
// GDN forward, run as a standalone op): per chunk of C = 64 tokens,
//   A = tril(beta_i * k_i.k_j * safe_exp(g_i - g_j), -1)      T = (I + A)^-1  (fp32 out)
// with g the chunk-local cumsum of the log decay, following gdn_reference
// (examples/attention/_gdn_full.py:73-78) and replacing the reference's kkt_exec +
// external tri_inv pair (kernels/kkt_fused_lib.cpp:401-443, registry.py:96-140).
//
// Persistent CTAs, three per SM, each walking chunks m = blockIdx.x + k * gridDim.x:
//   warp 4      one thread: TMA producer of K tiles (2-stage ring) and UMMA issuer of
//               KK^T (M = N = 64, fp32 accumulators in two TMEM buffers)
//   warps 0-3   gate cumsum and coefficients (warp 1 during the inverse of the previous
//               chunk, g and beta prefetched one chunk ahead; two record buffers), KK^T epilogue from TMEM -> fp16 A tile: beta_i e^{g_i - g_0}
//               e^{g_0 - g_j} for monotone chunks with total decay < 80, else the exact
//               per-element safe_exp,
//               (I + A)^-1 in place on warp-level MMAs, T -> fp32 staging tile ->
//               one asynchronous bulk store per chunk
// HBM-bound: per chunk 16 KB of K in, 16 KB of T out, 384 B of g and beta.
#include <cuda_runtime.h>

#include "capi_internal.h"
#include "common.cuh"
#include "ptx.cuh"
#include "tri_inv_warp.cuh"

namespace ptof {
namespace kktinv {

constexpr int kC = kChunk;   // 64
constexpr int kThreads = 160;
constexpr int kNS = 2;       // K ring depth
// four CTAs per SM: TMEM 4 x 128 columns; T is stored straight from the inverse's tile
constexpr int kCtasPerSm = 4;
constexpr int kAllBar = 1;   // named barriers: 1 = the four compute warps, 2-3 = pairs

template <int D>
struct KLayout {
  static constexpr int NKB = D / 64;
  static constexpr int STAGE = NKB * kC * 128;       // K rows x (64 d) per 128B-swizzled region
  static constexpr int OFF_A = kNS * STAGE;          // fp16 A -> T tile, 8 KB
  // fp32 gcum[64], beta[64], rowfb[64] = beta_i e^{g_i - g_0}, colf[64] = e^{g_0 - g_j},
  // then the chunk's fast-path flag
  // (two buffers: the next chunk's are written during the inverse of the current one)
  static constexpr int G_BYTES = 1024 + 16;
  static constexpr int OFF_G = OFF_A + kC * 128;
  static constexpr int OFF_BAR = OFF_G + 2 * G_BYTES;
  static constexpr int BYTES = OFF_BAR + 256 + 1024;
  static constexpr int TCOLS = 2 * kC;               // two fp32 64x64 accumulators
};

enum KBar { K_FULL0 = 0, K_MDONE0 = kNS, K_TFULL0 = 2 * kNS, K_TFREE0 = 2 * kNS + 2, K_COUNT = 2 * kNS + 4 };

struct KParams {
  CUtensorMap mapK;
  const float* g;          // may be null (ungated)
  const void* beta;
  float* Tout;             // [M][64][64], M = B*H*nc in (b, h, chunk) order
  int* status;
  int B, H, T, nc;
  int64_t M;
  int gate_mode, beta_dtype, layout;
  int64_t gs_b, gs_h, gs_t;
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) gdn_kkt_inv_kernel(const __grid_constant__ KParams P) {
  using L = KLayout<D>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t sbase = smem_u32(smem_raw);
  unsigned char* sm = smem_raw + (((sbase + 1023u) & ~1023u) - sbase);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + K_COUNT);
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t cnt = (P.M > blockIdx.x) ? (P.M - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;

  if (tid == 0) {
    abort_flag = 0;
    for (int i = 0; i < K_COUNT; ++i) mbar_init(&bars[i], 1);
    mbar_init(&bars[K_TFREE0], 4);   // one arrival per compute warp
    mbar_init(&bars[K_TFREE0 + 1], 4);
    fence_mbar_init();
  }
  if (warp == 4) {
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
  auto chunk_of = [&](int64_t k) { return static_cast<int64_t>(blockIdx.x) + k * gridDim.x; };

  if (warp == 4) {
    if (lane == 0) {
      prefetch_tmap(&P.mapK);
      const bool bhtd = (P.layout == PTOF_LAYOUT_BHTD);
      auto load = [&](int64_t k) {
        const int s = static_cast<int>(k % kNS);
        const int64_t m = chunk_of(k);
        const int bh = static_cast<int>(m / P.nc), c = static_cast<int>(m % P.nc);
        const int b = bh / P.H, h = bh % P.H, t0 = c * kC;
        const int y = bhtd ? t0 : h, z = bhtd ? bh : b * P.T + t0;
        mbar_arrive_expect_tx(&bars[K_FULL0 + s], L::STAGE);
#pragma unroll
        for (int kb = 0; kb < L::NKB; ++kb)
          tma_load_3d(sm + s * L::STAGE + kb * kC * 128, &P.mapK, &bars[K_FULL0 + s], kb * 64, y, z);
      };
      constexpr uint32_t ID = idesc_f16(64, kC, false, false, BF16);
      for (int64_t k = 0; k < cnt && k < kNS; ++k) load(k);
      for (int64_t k = 0; k < cnt; ++k) {
        const int s = static_cast<int>(k % kNS), bb = static_cast<int>(k & 1);
        // a wait that gives up raises the abort flag; the loop still runs to its end so
        // that every warp passes the same barriers (results are then invalid)
        wait(&bars[K_FULL0 + s], static_cast<uint32_t>((k / kNS) & 1), 1);
        if (k >= 2) wait(&bars[K_TFREE0 + bb], static_cast<uint32_t>(((k >> 1) + 1) & 1), 2);
        tc_fence_after();
        const uint32_t kt = smem_u32(sm + s * L::STAGE);
#pragma unroll 1
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint64_t d = sdesc_sw128(kt + (ks >> 2) * (kC * 128) + (ks & 3) * 32, 16, 1024);
          umma_ss(tmem + bb * kC, d, d, ID, ks > 0);
        }
        umma_commit(&bars[K_TFULL0 + bb]);
        umma_commit(&bars[K_MDONE0 + s]);
        // refill the stage of chunk k - 1 once its UMMA has read it
        if (k >= 1 && k - 1 + kNS < cnt) {
          const int sp = static_cast<int>((k - 1) % kNS);
          wait(&bars[K_MDONE0 + sp], static_cast<uint32_t>(((k - 1) / kNS) & 1), 3);
          load(k - 1 + kNS);
        }
      }
      // every UMMA has completed before TMEM is released
      if (cnt > 0) {
        const int64_t kl = cnt - 1;
        wait(&bars[K_MDONE0 + (kl % kNS)], static_cast<uint32_t>((kl / kNS) & 1), 4);
      }
    }
  } else {
    // ============================ compute warps 0-3 ============================
    const int w = warp, l = lane;
    unsigned char* at = sm + L::OFF_A;
    // gate records of chunk k in buffer k & 1: gcum[64], beta[64], rowfb[64], colf[64], fast
    auto gbuf = [&](int64_t k) { return reinterpret_cast<float*>(sm + L::OFF_G + (k & 1) * L::G_BYTES); };
    // warp 1: g and beta of a chunk, two tokens per lane (prefetched one chunk ahead)
    float pg0 = 0.f, pg1 = 0.f, pb0 = 0.f, pb1 = 0.f;
    auto fetch = [&](int64_t k) {
      const int64_t m = chunk_of(k);
      const int bh = static_cast<int>(m / P.nc), c = static_cast<int>(m % P.nc);
      const int b = bh / P.H, h = bh % P.H;
      const int64_t i0 = b * P.gs_b + h * P.gs_h + (static_cast<int64_t>(c) * kC + 2 * l) * P.gs_t;
      pg0 = pg1 = 0.f;
      if (P.gate_mode != PTOF_GATE_NONE) {
        pg0 = P.g[i0];
        pg1 = P.g[i0 + P.gs_t];
      }
      pb0 = ld_beta_any(P.beta, P.beta_dtype, i0);
      pb1 = ld_beta_any(P.beta, P.beta_dtype, i0 + P.gs_t);
    };
    // the gate records of chunk k from the prefetched registers, then the prefetch of
    // chunk k + 1 (whole warp 1)
    auto gate = [&](int64_t k) {
      float* gr = gbuf(k);
      float g0 = pg0, g1 = pg1;
      const float b0 = pb0, b1 = pb1;
      bool mono = true;   // the chunk-local cumsum never increases
      if (P.gate_mode == PTOF_GATE_RAW) {
        mono = (g0 <= 0.f) && (g1 <= 0.f);
        g1 += g0;
        float run = g1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, run, o);
          if (l >= o) run += y;
        }
        g0 += run - g1;
        g1 = run;
      } else if (P.gate_mode == PTOF_GATE_CUMSUM) {
        const float prev = __shfl_up_sync(0xffffffffu, g1, 1);
        mono = (g1 <= g0) && (l == 0 || g0 <= prev);
      }
      // exp(g_i - g_j) = exp(g_i - g_0) exp(g_0 - g_j): overflow-free when the cumsum is
      // monotone and the chunk's total decay is below 80; otherwise the exact form
      const float gfirst = __shfl_sync(0xffffffffu, g0, 0);
      const float gl = __shfl_sync(0xffffffffu, g1, 31);
      const bool fast = __all_sync(0xffffffffu, mono) && (gfirst - gl < 80.f);
      reinterpret_cast<float2*>(gr)[l] = make_float2(g0, g1);
      reinterpret_cast<float2*>(gr + kC)[l] = make_float2(b0, b1);
      reinterpret_cast<float2*>(gr + 2 * kC)[l] =
          make_float2(b0 * __expf(g0 - gfirst), b1 * __expf(g1 - gfirst));
      reinterpret_cast<float2*>(gr + 3 * kC)[l] = make_float2(__expf(gfirst - g0), __expf(gfirst - g1));
      if (l == 0) *reinterpret_cast<int*>(gr + 4 * kC) = fast ? 1 : 0;
      if (k + 1 < cnt) fetch(k + 1);
    };
    if (w == 1 && cnt > 0) {
      fetch(0);
      gate(0);
    }
    named_bar_sync(kAllBar, 128);   // gate records of chunk 0
    for (int64_t k = 0; k < cnt; ++k) {
      const int bb = static_cast<int>(k & 1);
      const int64_t m = chunk_of(k);
      const float* gcum = gbuf(k);
      const float* bsm = gcum + kC;
      const float* rowfb = gcum + 2 * kC;
      const float* colf = gcum + 3 * kC;
      const int* fastp = reinterpret_cast<const int*>(gcum + 4 * kC);
      // ---- KK^T row i = 16 w + (l & 15) (M = 64 accumulator: lanes 32w .. 32w + 15);
      //      lanes 0-15 take columns 0-31 of their row, lanes 16-31 columns 32-63 ----
      wait(&bars[K_TFULL0 + bb], static_cast<uint32_t>((k >> 1) & 1), 10);
      tc_fence_after();
      const int i = 16 * w + (l & 15), jb = 32 * (l >> 4);
      const uint32_t tacc = tmem + bb * kC + ((32u * w) << 16);
      const bool fast = *fastp != 0;
      const float gi = gcum[i], bi = bsm[i], rb = rowfb[i];
      {
        float v[32];
        tmem_ld16_split<32>(tacc, *reinterpret_cast<float(*)[16]>(v));
        tmem_ld16_split<32>(tacc + 16, *reinterpret_cast<float(*)[16]>(v + 16));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (l == 0) mbar_arrive(&bars[K_TFREE0 + bb]);
#pragma unroll
        for (int j0 = 0; j0 < 32; j0 += 8) {
          uint32_t pk[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float a2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int j = jb + j0 + 2 * u + e;
              const float cf = fast ? rb * colf[j] : bi * kkt_coef(gi, gcum[j]);
              a2[e] = (j < i) ? v[j0 + 2 * u + e] * cf : 0.f;
            }
            pk[u] = pack_f16(a2[0], a2[1]);
          }
          const int jj = jb + j0;
          *reinterpret_cast<uint4*>(at + i * 128 + (((jj >> 3) ^ (i & 7)) << 4)) =
              make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
      named_bar_sync(kAllBar, 128);   // A complete
      // warp 1 is idle during the inverse's 16 -> 32 level: it writes the next chunk's
      // gate records into the other buffer (visible to all four warps after the level)
      tri_inv64_inplace_idle(at, w, l, 2, kAllBar, [&] {
        if (w == 1 && k + 1 < cnt) gate(k + 1);
      });
      // ---- T (fp16 tile) -> fp32 rows of T in global memory: float4 f = tid + 128 it is
      //      row f / 16, columns 4 (f % 16) .. (each row 256 contiguous bytes) ----
      float4* tg = reinterpret_cast<float4*>(P.Tout + m * (kC * kC));
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int f = tid + 128 * it, row = f >> 4, col = (f & 15) * 4;
        const uint2 u = *reinterpret_cast<const uint2*>(
            at + row * 128 + ((((col >> 3) ^ (row & 7)) << 4) | ((col & 7) << 1)));
        const float2 lo = unpack_f16(u.x), hi = unpack_f16(u.y);
        tg[f] = make_float4(lo.x, lo.y, hi.x, hi.y);
      }
      named_bar_sync(kAllBar, 128);   // A tile free again
    }
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 4) tmem_dealloc(tmem, L::TCOLS);
}

}  // namespace kktinv

namespace {
template <int D, bool BF16>
int launch_kkt_inv_t(const ptof_gdn_params& p, int* status, const void* k, const void* beta,
                     const float* g, float* Tout, cudaStream_t st) {
  using L = kktinv::KLayout<D>;
  kktinv::KParams P;
  const CUtensorMapDataType t = BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  uint64_t dims[3], strides[2];
  uint32_t box[3] = {64, 64, 1};
  if (p.layout == PTOF_LAYOUT_BHTD) {
    dims[0] = D; dims[1] = p.T; dims[2] = static_cast<uint64_t>(p.B) * p.H;
    strides[0] = static_cast<uint64_t>(D) * 2;
    strides[1] = static_cast<uint64_t>(p.T) * D * 2;
  } else {
    dims[0] = D; dims[1] = p.H; dims[2] = static_cast<uint64_t>(p.B) * p.T;
    strides[0] = static_cast<uint64_t>(D) * 2;
    strides[1] = static_cast<uint64_t>(p.H) * D * 2;
    box[1] = 1; box[2] = 64;
  }
  int rc = make_tmap_3d(&P.mapK, k, t, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  P.g = (p.gate_mode == PTOF_GATE_NONE) ? nullptr : g;
  P.beta = beta;
  P.Tout = Tout;
  P.status = status;
  P.B = p.B; P.H = p.H; P.T = p.T; P.nc = p.T / kChunk;
  P.M = static_cast<int64_t>(p.B) * p.H * P.nc;
  P.gate_mode = p.gate_mode;
  P.beta_dtype = p.beta_dtype;
  P.layout = p.layout;
  const Strides3 sg = make_strides3(p.layout, p.H, p.T);
  P.gs_b = sg.b; P.gs_h = sg.h; P.gs_t = sg.t;
  auto kern = kktinv::gdn_kkt_inv_kernel<D, BF16>;
  cudaError_t e = set_smem_once(kern, L::BYTES);
  if (e != cudaSuccess) return cuda_fail(e, "kkt_inv smem attribute");
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t grid = P.M < kktinv::kCtasPerSm * static_cast<int64_t>(sms)
                           ? P.M : kktinv::kCtasPerSm * static_cast<int64_t>(sms);
  kern<<<static_cast<unsigned>(grid), kktinv::kThreads, L::BYTES, st>>>(P);
  e = cudaGetLastError();
  return e == cudaSuccess ? PTOF_OK : cuda_fail(e, "kkt_inv launch");
}
}  // namespace

int launch_kkt_inv(const ptof_gdn_params& p, int* status, const void* k, const void* beta,
                   const float* g, float* Tout, cudaStream_t st) {
  const bool bf = (p.in_dtype == PTOF_BF16);
  if (p.Dk == 128) return bf ? launch_kkt_inv_t<128, true>(p, status, k, beta, g, Tout, st)
                             : launch_kkt_inv_t<128, false>(p, status, k, beta, g, Tout, st);
  return bf ? launch_kkt_inv_t<64, true>(p, status, k, beta, g, Tout, st)
            : launch_kkt_inv_t<64, false>(p, status, k, beta, g, Tout, st);
}

}  // namespace ptof
