// Self-tests of the sm_100a building blocks the GDN kernels are made of.
//
//  * selftest_umma: one UMMA D = (+-)A * B^T with A [M,K] and B [N,K] written
//    into shared memory in a chosen canonical layout (K-major or MN-major, 128-byte
//    swizzle) or A placed in TMEM, then D read back from TMEM with the 32x32b
//    load pattern the kernels use. Checks descriptors, instruction descriptor
//    fields, the M=64 / M=128 accumulator lane maps and the TMEM A-operand packing.
//  * selftest_tma: a TMA SWIZZLE_128B tile load, read back through sw128_off, so the
//    software swizzle the kernels use for their own smem tiles matches the hardware.
#include <cuda_runtime.h>

#include <utility>

#include "common.cuh"
#include "ptx.cuh"

namespace ptof {

namespace selftest {

constexpr int kMaxM = 128, kMaxN = 256, kMaxK = 128;

__global__ void __launch_bounds__(128) umma_kernel(const float* A, const float* B, float* D,
                                                   int M, int N, int K, int mode, int* status) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-align the dynamic smem base for the swizzle phase
  const uint32_t base = smem_u32(smem_raw);
  unsigned char* sm = smem_raw + (((base + 1023u) & ~1023u) - base);
  unsigned char* sA = sm;                                  // up to 128x128 bf16 = 32 KB
  unsigned char* sB = sm + kMaxM * kMaxK * 2;              // up to 256x128 bf16 = 64 KB
  uint64_t* bar = reinterpret_cast<uint64_t*>(sB + kMaxN * kMaxK * 2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  __shared__ int abort_flag;

  const bool a_mn = mode & 1, b_mn = mode & 2, a_tmem = mode & 4, neg = mode & 8;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    abort_flag = 0;
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t d_tmem = tmem;          // columns [0, N)
  const uint32_t a_col = tmem + 256;     // A operand columns [256, 256 + K/2)

  // ---- operands into smem (bf16) in the requested canonical layout ----
  for (int idx = tid; idx < M * K; idx += 128) {
    const int m = idx / K, k = idx % K;
    const __nv_bfloat16 x = __float2bfloat16_rn(A[idx]);
    uint32_t off;
    if (!a_mn) off = (k / 64) * (M * 128) + sw128_off(m, (k % 64) * 2);
    else off = (m / 64) * (K * 128) + sw128_off(k, (m % 64) * 2);
    *reinterpret_cast<__nv_bfloat16*>(sA + off) = x;
  }
  for (int idx = tid; idx < N * K; idx += 128) {
    const int n = idx / K, k = idx % K;
    const __nv_bfloat16 x = __float2bfloat16_rn(B[idx]);
    uint32_t off;
    if (!b_mn) off = (k / 64) * (N * 128) + sw128_off(n, (k % 64) * 2);
    else off = (n / 64) * (K * 128) + sw128_off(k, (n % 64) * 2);
    *reinterpret_cast<__nv_bfloat16*>(sB + off) = x;
  }
  if (a_tmem) {
    // row m -> lane m (M == 128); column c holds K elements 2c (low half), 2c+1 (high)
    const int m = tid;
    for (int c0 = 0; c0 < K / 2; c0 += 16) {
      uint32_t r[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int k = 2 * (c0 + j);
        r[j] = (m < M && k + 1 < K) ? pack_bf16(A[m * K + k], A[m * K + k + 1]) : 0u;
      }
      tmem_st16(a_col + ((32u * warp) << 16) + c0, r);
    }
    tmem_wait_st();
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (tid == 0) {
    const uint32_t idesc = idesc_f16(M, N, a_mn, b_mn, true, neg);
    const uint32_t sa = smem_u32(sA), sb = smem_u32(sB);
    for (int ks = 0; ks < K / 16; ++ks) {
      const int k0 = ks * 16;
      uint64_t bdesc;
      if (!b_mn) bdesc = sdesc_sw128(sb + (k0 / 64) * (N * 128) + (k0 % 64) * 2, 16, 1024);
      else bdesc = sdesc_sw128(sb + k0 * 128, K * 128, 1024);
      if (a_tmem) {
        umma_ts(d_tmem, a_col + ks * 8, bdesc, idesc, ks > 0);
      } else {
        uint64_t adesc;
        if (!a_mn) adesc = sdesc_sw128(sa + (k0 / 64) * (M * 128) + (k0 % 64) * 2, 16, 1024);
        else adesc = sdesc_sw128(sa + k0 * 128, K * 128, 1024);
        umma_ss(d_tmem, adesc, bdesc, idesc, ks > 0);
      }
    }
    umma_commit(bar);
  }
  __syncwarp();
  mbar_wait(bar, 0, &abort_flag, status, 100);
  tc_fence_after();

  // ---- read D back: M=128 -> lane m; M=64 -> lane 16*(m/16) + m%16 ----
  int row = -1;
  if (M == 128) row = warp * 32 + lane;
  else if (lane < 16) row = warp * 16 + lane;
  for (int c0 = 0; c0 < N; c0 += 16) {
    float v[16];
    tmem_ld16(d_tmem + ((32u * warp) << 16) + c0, v);
    tmem_wait_ld();
    if (row >= 0 && row < M) {
#pragma unroll
      for (int j = 0; j < 16; ++j) D[row * N + c0 + j] = v[j];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// TMA SWIZZLE_128B load of a [64 x 64] bf16 box at (x0, y0), de-swizzled in software.
__global__ void tma_kernel(const __grid_constant__ CUtensorMap map, int x0, int y0,
                           __nv_bfloat16* out, int* status) {
  __shared__ __align__(1024) unsigned char tile[64 * 128];
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  const int tid = threadIdx.x;
  if (tid == 0) {
    abort_flag = 0;
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    mbar_arrive_expect_tx(&bar, 64 * 128);
    tma_load_2d(tile, &map, &bar, x0, y0);
  }
  mbar_wait(&bar, 0, &abort_flag, status, 200);
  for (int idx = tid; idx < 64 * 64; idx += blockDim.x) {
    const int r = idx / 64, c = idx % 64;
    out[idx] = *reinterpret_cast<const __nv_bfloat16*>(tile + sw128_off(r, c * 2));
  }
}

// Issue-rate probe: `issuers` warps each issue `n` back-to-back UMMAs (M = 128, N,
// K = 16 each) into their own accumulator, commit, and wait. Operand contents are
// irrelevant (zeros). MODE bit 0: A from TMEM (else shared memory); bit 1: the whole
// warp runs the loop and one elected lane issues (else lane 0 alone); bit 2: the
// descriptors are formed once and advanced by constant increments (else rebuilt per
// UMMA); bit 3: the 8 K-steps of the loop are unrolled.
// out[3 i + 0..2] = issue cycles, issue-to-completion cycles, and the cycles of one
// further UMMA issued alone and waited for (its round trip), for issuer i.
template <int MODE>
__global__ void __launch_bounds__(128) umma_rate_kernel(int N, int n, int issuers,
                                                         long long* out, int* status) {
  constexpr bool kTmemA = MODE & 1, kUniform = MODE & 2, kIncr = MODE & 4, kUnroll = MODE & 8;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t base = smem_u32(smem_raw);
  unsigned char* sm = smem_raw + (((base + 1023u) & ~1023u) - base);
  unsigned char* sA = sm;                       // 128 x 128 bf16
  unsigned char* sB = sm + 32768;               // 256 x 128 bf16
  uint64_t* bar = reinterpret_cast<uint64_t*>(sB + 65536);   // 4 x 2 barriers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 8);
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < (32768 + 65536) / 16; i += 128)
    reinterpret_cast<uint4*>(sm)[i] = make_uint4(0, 0, 0, 0);
  if (tid == 0) {
    abort_flag = 0;
    for (int i = 0; i < 8; ++i) mbar_init(&bar[i], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp < issuers && (kUniform || lane == 0)) {
    const uint32_t idesc = idesc_f16(128, N, false, false, true);
    const uint32_t d = tmem + warp * N;          // accumulator of this issuer
    const uint32_t a_t = tmem + 448;             // TMEM A operand (64 columns)
    const uint32_t sa = smem_u32(sA), sb = smem_u32(sB);
    const uint64_t a0 = sdesc_sw128(sa, 16, 1024), b0 = sdesc_sw128(sb, 16, 1024);
    const uint32_t bstep = (N * 128) >> 4;       // next 64-wide K block of B
    const bool leader = kUniform ? elect_one() : true;
    auto issue = [&](int ks) {
      uint64_t ad, bd;
      if (kIncr) {
        ad = a0 + static_cast<uint64_t>((ks >> 2) * 1024 + (ks & 3) * 2);
        bd = b0 + static_cast<uint64_t>((ks >> 2) * bstep + (ks & 3) * 2);
      } else {
        ad = sdesc_sw128(sa + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024);
        bd = sdesc_sw128(sb + (ks >> 2) * (N * 128) + (ks & 3) * 32, 16, 1024);
      }
      if (leader) {
        if (kTmemA) umma_ts(d, a_t + ks * 8, bd, idesc, 1);
        else umma_ss(d, ad, bd, idesc, 1);
      }
    };
    const long long t0 = clock64();
    for (int i = 0; i < n; i += 8) {
      if (kUnroll) {
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) issue(ks);
      } else {
#pragma unroll 1
        for (int ks = 0; ks < 8; ++ks) issue(ks);
      }
    }
    const long long t1 = clock64();
    if (leader) umma_commit(&bar[2 * warp]);
    mbar_wait(&bar[2 * warp], 0, &abort_flag, status, 300);
    const long long t2 = clock64();
    if (leader) {
      if (kTmemA) umma_ts(d, a_t, b0, idesc, 1);
      else umma_ss(d, a0, b0, idesc, 1);
      umma_commit(&bar[2 * warp + 1]);
    }
    mbar_wait(&bar[2 * warp + 1], 0, &abort_flag, status, 301);
    const long long t3 = clock64();
    if (leader) {
      out[3 * warp + 0] = t1 - t0;
      out[3 * warp + 1] = t2 - t0;
      out[3 * warp + 2] = t3 - t2;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

template <int MODE>
cudaError_t launch_rate(int N, int n, int issuers, long long* out, int* status, cudaStream_t st) {
  const int smem = 32768 + 65536 + 256 + 1024;
  cudaError_t e = cudaFuncSetAttribute(umma_rate_kernel<MODE>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  umma_rate_kernel<MODE><<<1, 128, smem, st>>>(N, n, issuers, out, status);
  return cudaGetLastError();
}

template <int... M>
cudaError_t launch_rate_mode(int mode, int N, int n, int issuers, long long* out, int* status,
                             cudaStream_t st, std::integer_sequence<int, M...>) {
  cudaError_t e = cudaErrorInvalidValue;
  ((mode == M ? (e = launch_rate<M>(N, n, issuers, out, status, st), 0) : 0), ...);
  return e;
}

}  // namespace selftest

cudaError_t launch_selftest_umma_rate(int N, int n, int issuers, int mode, long long* out,
                                      int* status, cudaStream_t stream) {
  return selftest::launch_rate_mode(mode, N, n, issuers, out, status, stream,
                                    std::make_integer_sequence<int, 16>{});
}

cudaError_t launch_selftest_umma(const float* A, const float* B, float* D, int M, int N, int K,
                                 int mode, int* status, cudaStream_t stream) {
  const int smem = selftest::kMaxM * selftest::kMaxK * 2 + selftest::kMaxN * selftest::kMaxK * 2 +
                   64 + 1024;
  cudaError_t e = cudaFuncSetAttribute(selftest::umma_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  selftest::umma_kernel<<<1, 128, smem, stream>>>(A, B, D, M, N, K, mode, status);
  return cudaGetLastError();
}

cudaError_t launch_selftest_tma(const CUtensorMap& map, int x0, int y0, void* out, int* status,
                                cudaStream_t stream) {
  selftest::tma_kernel<<<1, 128, 0, stream>>>(map, x0, y0, static_cast<__nv_bfloat16*>(out),
                                              status);
  return cudaGetLastError();
}

}  // namespace ptof
