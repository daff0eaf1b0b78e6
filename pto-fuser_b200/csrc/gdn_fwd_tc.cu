// Fused chunked Gated DeltaNet forward on B200 tensor cores (tcgen05 + TMEM + TMA).
//
// One CTA owns one (batch, head) pair and walks its chunks (C = 64 tokens) in order.
// Per chunk c, with g the chunk-local cumsum of the log decay and gl = g[63]:
//   A    = tril(beta_i * k_i.k_j * exp(g_i - g_j), -1)      T = (I + A)^-1
//   W^T  = K^T (T * (beta e^g)_j)^T        U^T = V^T (T * beta_j)^T
//   Vn^T = U^T - S^T W^T                                  (S = state [Dk, Dv])
//   O^T  = S^T (Q * e^g)^T + Vn^T Aqk^T,   Aqk = tril(q_i.k_j * exp(min(g_i - g_j, 0)))
//   S^T  = e^gl S^T + (Vn^T * e^(gl - g)) K
// which is the reference's gdn_reference (examples/attention/_gdn_full.py:57-97) with
// every contraction transposed so the value dimension Dv is the UMMA M dimension:
// all chain MMAs have M = Dv (128 -> full datapath), the state lives in TMEM as
// fp32 S^T (TMEM lane = value column), and its bf16 copy feeds the next chunk's
// MMAs straight from TMEM.
//
// Warp roles (512 threads):
//   warp 0       TMA producer: [K|Q] tiles, g, beta -> 3-stage ring; V -> 2-stage ring
//   warps 1-3    single-thread UMMA issuers, one in-order stream each: chain (V_new,
//                state update), prep ([K;Q]K^T, W^T / U^T), output (S^T Q'^T, Vn^T Aqk^T);
//                warp 2 also owns the TMEM allocation
//   warps 4-11   prep: kkt/qk epilogue from TMEM, (I + A)^-1, T' and T'' for the WY
//                UMMAs, W^T readout; software-pipelined one chunk ahead of the chain
//   warps 12-15  scan: V_new readout, state copy / decay, output epilogue
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>

#include "capi_internal.h"
#include "common.cuh"
#include "ptx.cuh"
#include "tri_inv_warp.cuh"

namespace ptof {
namespace tcfwd {

constexpr int kC = kChunk;  // 64
// Threads per CTA. The D = 64 kernel adds a fifth warpgroup (warps 16-19) that writes
// the output, so the scan group's V_new conversion and state pass (the per-chunk
// recurrence) never wait behind output stores (330 -> 300 us).
// The D = 128 kernel needs up to 128 registers per thread, which 640 threads do not
// leave (it measured slower with spills), so its scan group writes the output itself.
template <int DK>
struct Roles {
  static constexpr bool OUT_GROUP = (DK == 64);
  static constexpr int THREADS = OUT_GROUP ? 640 : 512;
};
// named barrier ids: P = warps 4-7 (inverse, T', W^T readout), Q = warps 8-11
// (kkt/qk epilogue), scan = warps 12-15, output = warps 16-19 (D = 64); 4 and 5 pair
// warps 4-5 and 6-7
constexpr int kPBar = 1, kScanBar = 2, kQBar = 3, kOutBar = 6;

// ------------------------------------------------------ coefficient records ----
// Per chunk (64 tokens), computed once by gdn_coef_kernel from g and beta, byte
// offsets of fp32 arrays [64] and scalars; g is the chunk-local cumsum, gl = g[63].
namespace coef {
constexpr int GCUM = 0;      // g_i
constexpr int EG = 256;      // e^{g_i}
constexpr int BK = 512;      // beta_i e^{g_i}
constexpr int BV = 768;      // beta_i
constexpr int GAM = 1024;    // gamma_i = e^{gl - g_i}
constexpr int ROWFB = 1280;  // beta_i e^{g_i - g_0}
constexpr int COLF = 1536;   // e^{g_0 - g_j}
constexpr int EGL = 1792;    // e^{gl}
constexpr int FAST = 1796;   // int: the factorised (fast) path applies to this chunk
constexpr int ENGL = 1800;   // e^{-gl} (fast chunks)
constexpr int BYTES = 1808;  // multiple of 16 (bulk copies)
}  // namespace coef

// ------------------------------------------------------------------ layout ----
template <int DK, int DV, bool KDA = false>
struct Layout {
  static constexpr int NKB = DK / 64;               // 64-wide d blocks
  static constexpr int NVB = DV / 64;
  // bf16 S^T and bf16 V_new^T (+ V_new^T gamma) as TMEM A operands (M = DV = 128);
  // the DV = 64 variant keeps them in shared memory
  static constexpr bool SA_TMEM = (DV == 128);
  static constexpr bool VN_TMEM = SA_TMEM;
  // input ring (4 stages): [K | Q] per 64-wide d block, then the per-token arrays
  static constexpr int NIN = (DK == 128) ? 3 : 4;
  // K rows 0-63 | Q rows 64-127 (16 KB); KDA adds K e^{-g} in rows 128-191 (24 KB)
  static constexpr int KQ_REGION = (KDA ? 3 : 2) * kC * 128;
  static constexpr int OFF_K2 = 2 * kC * 128;        // KDA: K e^{-g} within a region
  static constexpr int OFF_KQ = 0;                   // within an input stage
  static constexpr int IN_STAGE = NKB * KQ_REGION;
  // per-chunk coefficient records written by gdn_coef_kernel (one per input stage,
  // in their own region below)
  static constexpr int M_GCUM = coef::GCUM, M_EG = coef::EG, M_BK = coef::BK, M_BV = coef::BV,
                       M_GAM = coef::GAM, M_ROWFB = coef::ROWFB, M_COLF = coef::COLF,
                       M_EGL = coef::EGL, M_FAST = coef::FAST, M_ENGL = coef::ENGL;
  static constexpr int MISC_BYTES = coef::BYTES;
  // V ring (2 stages)
  static constexpr int V_REGION = kC * 128;          // 8 KB per 64-wide block
  static constexpr int OFF_V = NIN * IN_STAGE;
  static constexpr int V_STAGE = NVB * V_REGION;
  // Aqk (3 buffers), W^T (1 buffer)
  static constexpr int OFF_AQK = OFF_V + V_STAGE;
  static constexpr int WT_BYTES = DK * 128;
  static constexpr int OFF_WT = OFF_AQK + 3 * kC * 128;
  // prep buffers: T' and T'' (bf16 WY operands), A (fp16, 2 buffers; the inverse
  // overwrites A with T in place)
  static constexpr int OFF_TP = OFF_WT + WT_BYTES;
  static constexpr int OFF_TPP = OFF_TP + 8192;
  static constexpr int OFF_TA = OFF_TPP + 8192;
  // shared-memory chain operands of the DV = 64 variant: Vn^T, Vn^T gamma, S^T
  static constexpr int VNT_BYTES = VN_TMEM ? 0 : DV * 128;
  static constexpr int OFF_VNT = OFF_TA + 2 * 8192;
  static constexpr int OFF_VNG = OFF_VNT + VNT_BYTES;
  static constexpr int OFF_SA = OFF_VNG + VNT_BYTES;
  static constexpr int SA_BYTES = SA_TMEM ? 0 : NKB * DV * 128;
  static constexpr int OFF_MISC = OFF_SA + SA_BYTES;  // NIN x MISC_BYTES
  // fp32 [2][64] output multipliers by chunk parity (written by the scan group at
  // V_new time, read by the output stores of the same chunk)
  // KDA: per input stage, the per-dimension decay e^{g_tot} of the PREVIOUS chunk
  static constexpr int EGLD_BYTES = KDA ? DK * 4 : 0;
  static constexpr int OFF_EGLD = OFF_MISC + NIN * MISC_BYTES;
  static constexpr int OFF_OSC = OFF_EGLD + NIN * EGLD_BYTES;
  static constexpr int OFF_BAR = OFF_OSC + 512;
  static constexpr int BYTES = OFF_BAR + 512 + 1024;  // + alignment slack
  // TMEM columns
  static constexpr int T_SM = 0;                     // fp32 S^T master: DK columns
  static constexpr int T_SA = DK;                    // bf16 S^T: DK/2 columns
  static constexpr int T_VN0 = DK + (SA_TMEM ? DK / 2 : 0);  // U^T -> V_new^T, 2 buffers
  static constexpr int T_VN1 = T_VN0 + kC;
  static constexpr int T_O = T_VN1 + kC;
  static constexpr int T_KQ = T_O + kC;             // [K;Q] K^T of the chunk in prep
  static constexpr int T_RW = T_KQ + kC;             // W^T of the chunk in prep
  static constexpr int T_COLS = 512;
  static_assert(T_RW + kC <= T_COLS, "TMEM budget");
  // the kernel's static shared memory (1 KB) counts against the 227 KB opt-in
  static_assert(BYTES <= 227 * 1024 - 1024, "smem budget");
};

// barrier slots (uint64 each) inside the BAR area. Hand-offs between groups that
// can run two chunks apart use one barrier per buffer, so a phase parity never
// aliases a later chunk.
enum Bar {
  B_FULL0 = 0, B_FULL1, B_FULL2, B_FULL3, B_EMPTY0, B_EMPTY1, B_EMPTY2, B_EMPTY3,
  B_VFULL, B_WREADY, B_WTFREE,
  B_AREADY0, B_AREADY1, B_TAFREE0, B_TAFREE1,
  B_KQFULL, B_TREADY, B_WUFULL, B_RWFREE, B_VNFREE0, B_VNFREE1, B_SREADY, B_VNFULL,
  B_VNREADY, B_SFULL, B_OFULL0, B_OFULL1, B_OFULL2, B_OFREE, B_DONE, B_KQFREE, B_O1DONE,
  B_NEVER,   // never arrived at: the injected stall of the fault-path test waits on it
  B_COUNT
};
static_assert(B_COUNT * 8 + 8 <= 512, "barrier area");

struct Params {
  CUtensorMap mapK, mapQ, mapV;   // 3D maps, box = 64 d x 64 tokens
  CUtensorMap mapK2;               // KDA: k e^{-g} (mapK, mapQ: k e^{g}, q e^{g})
  const float* egl;                // KDA: [B*H][nc + 1][DK] e^{g_tot} of chunk c - 1 at c
  const unsigned char* coef;       // [B*H][nc] coefficient records (gdn_coef_kernel)
  const float* S0;                 // [B,H,DK,DV] or null
  void* o;
  float* S_final;                  // or null
  int* status;
  unsigned long long* trace;       // optional [chunks x kTraceSlots] timestamps of CTA 0
  int trace_chunks;
  int B, H, T, nc;
  int layout;
  // variable-length sequences: B sequences packed token-major, sequence b spans tokens
  // [cu_seqlens[b], cu_seqlens[b+1]) of every tensor; null for fixed length T
  const int* cu_seqlens;
  int mnc;                         // coefficient records per (b, h) (>= chunks of any sequence)
  int gqa;                         // value heads per query/key head (q, k have H / gqa heads)
  int64_t os_b, os_h, os_t;        // o strides (elements)
  float scale;
  unsigned long long wait_ns;      // limit of every bounded wait
  int inject_stall;                // test only: the chain waits on B_NEVER before chunk 0
  int view;                        // strided view: 4D maps {D, T, H, B}, coordinates (x, t, h, b)
};

// Optional stage timestamps (globaltimer, ns) of CTA 0: slot layout per chunk.
constexpr int kTraceSlots = 24;
enum TraceSlot {
  TR_TMA_ISSUE = 0, TR_PREP_FULL, TR_PREP_KQ, TR_PREP_EPI, TR_PREP_INV, TR_PREP_TREADY,
  TR_PREP_WU, TR_PREP_END, TR_SCAN_VNFULL, TR_SCAN_VNREADY, TR_SCAN_SFULL, TR_SCAN_SREADY,
  TR_SCAN_OFULL, TR_SCAN_END, TR_MMA_C1, TR_MMA_C2, TR_INV_START, TR_INV_L0, TR_INV_L1,
  TR_INV_L2, TR_PREP_COEF, TR_PREP_OFULL, TR_X0, TR_X1
};
// Compiled only into the traced instantiation (TRACE = true), so the production
// kernel's loops carry no trace code.
template <bool TRACE>
__device__ __forceinline__ void trace_mark(const Params& P, int c, int slot) {
  if (TRACE && blockIdx.x == 0 && c < P.trace_chunks)
    P.trace[c * kTraceSlots + slot] = globaltimer_ns();
}

// ------------------------------------------------------------ small helpers ----
struct Sync {
  volatile int* abort;
  int* status;
  unsigned long long limit;
  // one inlined probe, the bounded loop out of line. After an abort every wait
  // returns false at once: the roles run out their loops without blocking, no new
  // TMA load is issued, and the teardown drains what is in flight.
  __device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity, int site) const {
    if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait(bar, parity, abort, status, site, limit);
  }
};

// Bounded spin on a phase (teardown drains, not subject to the abort flag).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity) && globaltimer_ns() - t0 < kWaitTimeoutNs) {
  }
}

__device__ __forceinline__ float ld_beta(const void* p, int dt, int64_t i) {
  if (dt == PTOF_F32) return static_cast<const float*>(p)[i];
  if (dt == PTOF_F16) return __half2float(static_cast<const __half*>(p)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

template <bool F16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  return F16 ? pack_f16(a, b) : pack_bf16(a, b);
}
template <bool F16>
__device__ __forceinline__ float2 unpack2(uint32_t u) {
  return F16 ? unpack_f16(u) : unpack_bf16(u);
}

// Output rows of a partial last chunk: tokens [0, lim) of O^T row v (TMEM, 64 columns,
// scaled by osc) to o; kept out of line so the full-chunk store loop stays unchanged.
template <typename TO>
__device__ __noinline__ void store_tail(uint32_t t_o, TO* op, const float* osc, int64_t os_t,
                                        int lim, bool active) {
#pragma unroll 1
  for (int c0 = 0; c0 < 64; c0 += 16) {
    float x[16];
    tmem_ld16(t_o + c0, x);
    tmem_wait_ld();
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      if (active && c0 + m < lim) *op = from_f32<TO>(x[m] * osc[c0 + m]);
      op += os_t;
    }
  }
}

// ------------------------------------------------------ coefficient pre-pass ----
struct CoefParams {
  const float* g;        // [B,H,T] / [B,T,H] fp32, raw or chunk-local cumsum (null: ungated)
  const void* beta;
  unsigned char* out;    // [B*H][nc][coef::BYTES]
  int B, H, nc;          // nc: records per (b, h)
  int gate_mode, beta_dtype, allow_fast;
  int64_t gs_b, gs_h, gs_t;
  const int* cu_seqlens; // variable-length sequences (token-major), or null
  int T;                 // fixed sequence length (cu_seqlens null)
};

// One warp per chunk, lane l owns tokens 2l and 2l+1: chunk-local cumsum of the
// log decay (warp scan), the exponentials every later stage needs, and the fast-path
// test: exp(g_i - g_j) = exp(g_i - g_0) exp(g_0 - g_j) is overflow-free when the
// cumsum is monotone and the chunk's total decay is below 80 (fp16 operands always
// take the exact path). Mirrors gdn_reference's per-chunk gate handling
// (examples/attention/_gdn_full.py:63-66, 108).
__global__ void __launch_bounds__(256) gdn_coef_kernel(const __grid_constant__ CoefParams P) {
  const int l = threadIdx.x & 31;
  const int64_t chunk = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (chunk >= static_cast<int64_t>(P.B) * P.H * P.nc) return;
  const int bh = static_cast<int>(chunk / P.nc), c = static_cast<int>(chunk % P.nc);
  const int b = bh / P.H, h = bh % P.H;
  int len = P.T;
  int64_t gb = b * P.gs_b;
  if (P.cu_seqlens != nullptr) {
    const int st = P.cu_seqlens[b], en = P.cu_seqlens[b + 1];
    len = en > st ? en - st : 0;
    if (c * kC >= len) return;   // beyond this sequence: record unused
    gb = static_cast<int64_t>(st) * P.gs_t;
  }
  gb += h * P.gs_h + static_cast<int64_t>(c) * kC * P.gs_t;
  const int64_t i0 = gb + static_cast<int64_t>(2 * l) * P.gs_t, i1 = i0 + P.gs_t;
  // tokens past the end of the sequence (the ragged last chunk) get beta = 0 and
  // g = 0: their rows of A, W, U and V_new vanish and the state is not decayed
  const bool ok0 = c * kC + 2 * l < len, ok1 = c * kC + 2 * l + 1 < len;
  float g0 = 0.f, g1 = 0.f;
  if (P.gate_mode != PTOF_GATE_NONE) {
    // a raw decay of 0 past the end keeps the cumsum flat; a given cumsum repeats the
    // sequence's last value there
    float gpad = 0.f;
    if (P.gate_mode == PTOF_GATE_CUMSUM && !ok1)
      gpad = P.g[gb + static_cast<int64_t>(len - 1 - c * kC) * P.gs_t];
    g0 = ok0 ? P.g[i0] : gpad;
    g1 = ok1 ? P.g[i1] : gpad;
  }
  bool mono = true;  // the chunk-local cumsum never increases
  if (P.gate_mode == PTOF_GATE_RAW) {
    mono = (g1 <= 0.f) && (g0 <= 0.f);
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
  const float gfirst = __shfl_sync(0xffffffffu, g0, 0);
  const float gl = __shfl_sync(0xffffffffu, g1, 31);
  const bool fast = P.allow_fast && __all_sync(0xffffffffu, mono) && (gfirst - gl < 80.f);
  const float b0 = ok0 ? ld_beta(P.beta, P.beta_dtype, i0) : 0.f;
  const float b1 = ok1 ? ld_beta(P.beta, P.beta_dtype, i1) : 0.f;
  const float e0 = __expf(g0), e1 = __expf(g1);
  const float rf0 = __expf(g0 - gfirst), rf1 = __expf(g1 - gfirst);
  unsigned char* rec = P.out + chunk * coef::BYTES;
  auto put = [&](int off, float x, float y) {
    reinterpret_cast<float2*>(rec + off)[l] = make_float2(x, y);
  };
  put(coef::GCUM, g0, g1);
  put(coef::EG, e0, e1);
  put(coef::BK, b0 * e0, b1 * e1);
  put(coef::BV, b0, b1);
  put(coef::GAM, __expf(gl - g0), __expf(gl - g1));
  put(coef::ROWFB, rf0 * b0, rf1 * b1);
  put(coef::COLF, __expf(gfirst - g0), __expf(gfirst - g1));
  if (l == 0) {
    *reinterpret_cast<float*>(rec + coef::EGL) = __expf(gl);
    *reinterpret_cast<int*>(rec + coef::FAST) = fast ? 1 : 0;
    *reinterpret_cast<float*>(rec + coef::ENGL) = fast ? __expf(-gl) : 0.f;
  }
}

// ------------------------------------------------------------------ kernel ----
template <int DK, int DV, bool F16, typename TO, bool TRACE, bool VARLEN, bool KDA = false>
__global__ void __launch_bounds__(Roles<DK>::THREADS, 1) gdn_fwd_tc_kernel(const __grid_constant__ Params P) {
  using L = Layout<DK, DV, KDA>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t sbase = smem_u32(smem_raw);
  unsigned char* sm = smem_raw + (((sbase + 1023u) & ~1023u) - sbase);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B_COUNT);
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x, b = bh / P.H, h = bh % P.H;
  // sequence bounds: fixed length, or from cu_seqlens (a sequence longer than the
  // workspace's maximum is cut at mnc chunks and flagged in the status word). They are
  // kept in shared memory and read where used, so no warp holds them in registers.
  __shared__ int s_nc, s_len, s_tok0;
  int nc0 = P.nc, len0 = P.T, tok00 = b * P.T;
  if (VARLEN) {
    const int st = P.cu_seqlens[b], en = P.cu_seqlens[b + 1];
    tok00 = st;
    len0 = en > st ? en - st : 0;
    nc0 = (len0 + kC - 1) / kC;
    if (nc0 > P.mnc) {
      nc0 = P.mnc;
      len0 = nc0 * kC;
      if (tid == 0 && P.status != nullptr) atomicCAS(P.status, 0, 90);
    }
  }
  if (tid == 0) {
    s_nc = nc0;
    s_len = len0;
    s_tok0 = tok00;
  }
  if (nc0 == 0) {  // empty sequence: the final state is the initial one (CTA-uniform exit)
    if (P.S_final != nullptr) {
      const int64_t base = static_cast<int64_t>(bh) * DK * DV;
      for (int i = tid; i < DK * DV; i += Roles<DK>::THREADS)
        P.S_final[base + i] = P.S0 != nullptr ? P.S0[base + i] : 0.f;
    }
    return;
  }
  Sync sy{&abort_flag, P.status, P.wait_ns};

  if (tid == 0) {
    abort_flag = 0;
    for (int i = 0; i < B_COUNT; ++i) mbar_init(&bars[i], 1);
    for (int i = 0; i < L::NIN; ++i) mbar_init(&bars[B_EMPTY0 + i], 3);  // 2 issuers + scan
    mbar_init(&bars[B_DONE], 3);  // the three UMMA issuers
    if (L::VN_TMEM) {             // the chain and output UMMAs read V_new^T from TMEM
      mbar_init(&bars[B_VNFREE0], 2);
      mbar_init(&bars[B_VNFREE1], 2);
    }
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, L::T_COLS);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // fixed length: the kernel parameters themselves (no register held for them)
  const int nc = VARLEN ? s_nc : P.nc;
  const int tok0 = VARLEN ? s_tok0 : b * P.T;
  const uint64_t t_start = (TRACE && tid == 0) ? globaltimer_ns() : 0;

  // chunk c lives in input stage c % NIN (use index c / NIN) and Aqk buffer c % 3
  auto stage = [&](int c) { return sm + (c % L::NIN) * L::IN_STAGE; };
  auto misc = [&](int c) { return reinterpret_cast<float*>(sm + L::OFF_MISC + (c % L::NIN) * L::MISC_BYTES); };
  auto aqk = [&](int c) { return sm + L::OFF_AQK + (c % 3) * (kC * 128); };
  auto in_par = [&](int c) { return static_cast<uint32_t>((c / L::NIN) & 1); };
  auto aq_par = [&](int c) { return static_cast<uint32_t>((c / 3) & 1); };

  // ---- output of chunk c: O^T row v -> o[t0 + i, v], scaled by the chunk's output
  //      multipliers; run by the scan group (D = 128) or the output group (D = 64),
  //      `s` the thread's index in its group and `bar` that group's named barrier ----
  auto output_chunk = [&](int c, int s, int bar) {
    const int q = warp & 3;
    const int v = (DV == 128) ? (32 * q + lane) : (lane < 16 ? 16 * q + lane : -1);
    const uint32_t t_o = tmem + L::T_O + ((32u * q) << 16);
    TO* obase = static_cast<TO*>(P.o) +
                (VARLEN ? static_cast<int64_t>(tok0) * P.os_t : b * P.os_b) + h * P.os_h;
    sy.wait(&bars[B_OFULL0 + (c % 3)], aq_par(c), 34);
    tc_fence_after();
    if (s == 0) trace_mark<TRACE>(P, c, TR_SCAN_OFULL);
    const float* osc = reinterpret_cast<const float*>(sm + L::OFF_OSC) + (c & 1) * kC;
    if (!VARLEN || c + 1 < nc || s_len == nc * kC) {
      TO* op = obase + static_cast<int64_t>(c * kC) * P.os_t + (v >= 0 ? v : 0);
#pragma unroll 1
      for (int c0 = 0; c0 < kC; c0 += 16) {
        float x[16];
        tmem_ld16(t_o + c0, x);
        tmem_wait_ld();
        if (v >= 0) {
          if constexpr (Roles<DK>::OUT_GROUP) {
            // the output group has registers to spare: vector loads of the multipliers
            float sc[16];
#pragma unroll
            for (int m = 0; m < 16; m += 4)
              *reinterpret_cast<float4*>(sc + m) = *reinterpret_cast<const float4*>(osc + c0 + m);
#pragma unroll
            for (int m = 0; m < 16; ++m) {
              *op = from_f32<TO>(x[m] * sc[m]);
              op += P.os_t;
            }
          } else {
#pragma unroll
            for (int m = 0; m < 16; ++m) {
              *op = from_f32<TO>(x[m] * osc[c0 + m]);
              op += P.os_t;
            }
          }
        }
      }
    } else {   // the partial last chunk of a variable-length sequence (out of line)
      store_tail<TO>(t_o, obase + static_cast<int64_t>(c * kC) * P.os_t + (v >= 0 ? v : 0),
                     osc, P.os_t, s_len - c * kC, v >= 0);
    }
    tc_fence_before();
    named_bar_sync(bar, 128);
    if (s == 0) {
      mbar_arrive(&bars[B_OFREE]);
      trace_mark<TRACE>(P, c, TR_SCAN_END);
    }
  };


  // ================================================================ TMA ====
  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&P.mapK);
      prefetch_tmap(&P.mapQ);
      prefetch_tmap(&P.mapV);
    }
    const bool bhtd = (P.layout == PTOF_LAYOUT_BHTD);
    const unsigned char* crec = P.coef + static_cast<int64_t>(bh) * P.mnc * L::MISC_BYTES;
    const int Hg = P.H / P.gqa, hk = h / P.gqa;   // this value head's query/key head
    int issued = 0;   // chunks whose loads were issued
    for (int c = 0; c < nc; ++c) {
      const int s = c % L::NIN;
      const bool ok = c < L::NIN || sy.wait(&bars[B_EMPTY0 + s], in_par(c) ^ 1, 1);
      // after an abort no further load is issued (warp-uniform decision)
      if (!__all_sync(0xffffffffu, ok && !abort_flag)) break;
      issued = c + 1;
      unsigned char* st = stage(c);
      const int t0 = c * kC;
      // q, k: heads-outer {D, T, B*Hg} or token-major {D, Hg, tokens}
      const int y = bhtd ? t0 : hk;
      const int z = bhtd ? b * Hg + hk : static_cast<int>(tok0 + t0);
      if (lane == 0) {
        mbar_arrive_expect_tx(&bars[B_FULL0 + s], (KDA ? 3 : 2) * DK * kC * 2 + L::MISC_BYTES +
                                                      L::EGLD_BYTES);
#pragma unroll
        for (int kb = 0; kb < L::NKB; ++kb) {
          if (P.view) {
            tma_load_4d(st + L::OFF_KQ + kb * L::KQ_REGION, &P.mapK, &bars[B_FULL0 + s], kb * 64,
                        t0, h, b);
            tma_load_4d(st + L::OFF_KQ + kb * L::KQ_REGION + kC * 128, &P.mapQ,
                        &bars[B_FULL0 + s], kb * 64, t0, h, b);
            continue;
          }
          tma_load_3d(st + L::OFF_KQ + kb * L::KQ_REGION, &P.mapK, &bars[B_FULL0 + s], kb * 64, y, z);
          tma_load_3d(st + L::OFF_KQ + kb * L::KQ_REGION + kC * 128, &P.mapQ, &bars[B_FULL0 + s],
                      kb * 64, y, z);
          if constexpr (KDA)
            tma_load_3d(st + L::OFF_KQ + kb * L::KQ_REGION + L::OFF_K2, &P.mapK2,
                        &bars[B_FULL0 + s], kb * 64, y, z);
        }
        bulk_load(misc(c), crec + static_cast<int64_t>(c) * L::MISC_BYTES, L::MISC_BYTES,
                  &bars[B_FULL0 + s]);
        if constexpr (KDA)
          bulk_load(sm + L::OFF_EGLD + s * L::EGLD_BYTES,
                    P.egl + (static_cast<int64_t>(bh) * (P.nc + 1) + c) * DK, L::EGLD_BYTES,
                    &bars[B_FULL0 + s]);
        trace_mark<TRACE>(P, c, TR_TMA_ISSUE);
      }
      __syncwarp();
    }
    // the loads of the last NIN issued chunks may still be in flight after an abort:
    // the CTA does not exit (or release its shared memory) before they land
    if (lane == 0)
      for (int c = issued > L::NIN ? issued - L::NIN : 0; c < issued; ++c)
        drain_wait(&bars[B_FULL0 + (c % L::NIN)], in_par(c));
  }
  // ================================================================ MMA ====
  // Three UMMA issuer warps, each blocking on its own in-order stream (a commit
  // tracks only the issuing thread's UMMAs, so the streams stay independent):
  //   warp 1, chain:  Vn^T = U^T - S^T W^T ; S^T += (Vn^T g) K
  //   warp 2, prep:   [K;Q] K^T ; W^T = K^T T'^T, U^T = V^T T''^T
  //   warp 3, output: O = S^T Q'^T ; O += Vn^T Aqk^T
  // The whole warp runs each issue loop (the descriptors are then warp-uniform
  // values) and one elected lane issues and commits; the K-step loops are unrolled.
  // Measured on B200 (ptof_selftest_umma_rate): a lone lane in a rolled loop issues
  // one UMMA per ~120 cycles, a warp-uniform unrolled loop one per ~35-45 cycles, and
  // the commit-to-wait round trip drops from ~410 to ~280 cycles.
  else if (warp >= 1 && warp <= 3) {
    const bool leader = elect_one();
    constexpr uint32_t ID_KQ = idesc_f16(128, kC, false, false, !F16);
    constexpr uint32_t ID_WT = idesc_f16(DK, kC, true, false, !F16);
    constexpr uint32_t ID_UT = idesc_f16(DV, kC, true, false, !F16);
    constexpr uint32_t ID_VN = idesc_f16(DV, kC, false, true, !F16, true);   // -S^T W^T
    constexpr uint32_t ID_O1 = idesc_f16(DV, kC, false, false, !F16);        //  S^T Q'^T
    constexpr uint32_t ID_S = idesc_f16(DV, DK, false, true, !F16);          // (Vn g) K
    constexpr uint32_t ID_O2 = idesc_f16(DV, kC, false, false, !F16);        //  Vn^T Aqk^T
    const uint32_t t_sm = tmem + L::T_SM, t_sa = tmem + L::T_SA, t_o = tmem + L::T_O,
                   t_kq = tmem + L::T_KQ, t_rw = tmem + L::T_RW;
    const uint32_t s_tp = smem_u32(sm + L::OFF_TP), s_tpp = smem_u32(sm + L::OFF_TPP);
    const uint32_t s_vnt = smem_u32(sm + L::OFF_VNT), s_vng = smem_u32(sm + L::OFF_VNG);
    const uint32_t s_wt = smem_u32(sm + L::OFF_WT), s_sa = smem_u32(sm + L::OFF_SA);
    auto a_desc_sa = [&](int ks) {  // smem S^T (K-major, DV rows x DK)
      return sdesc_sw128(s_sa + (ks >> 2) * (DV * 128) + (ks & 3) * 32, 16, 1024);
    };
    auto t_vn = [&](int c) { return tmem + ((c & 1) ? L::T_VN1 : L::T_VN0); };
    auto commit = [&](uint64_t* bar) {
      if (leader) umma_commit(bar);
    };
    if (warp == 1) {
      // fault-path test: a wait on a barrier nothing arrives at runs out, aborts the CTA
      if (P.inject_stall) sy.wait(&bars[B_NEVER], 0, 99);
      for (int c = 0; c < nc; ++c) {
        sy.wait(&bars[B_SREADY], c & 1, 14);
        sy.wait(&bars[B_WREADY], c & 1, 15);
        __syncwarp();
        tc_fence_after();
        if (leader) trace_mark<TRACE>(P, c, TR_MMA_C1);
        const uint32_t vn = t_vn(c);
#pragma unroll
        for (int ks = 0; ks < DK / 16; ++ks) {
          const uint64_t bd = sdesc_sw128(s_wt + ks * 2048, DK * 128, 1024);
          if (leader) {
            if constexpr (L::SA_TMEM) umma_ts(vn, t_sa + ks * 8, bd, ID_VN, 1);
            else umma_ss(vn, a_desc_sa(ks), bd, ID_VN, 1);
          }
        }
        commit(&bars[B_VNFULL]);
        commit(&bars[B_WTFREE]);
        sy.wait(&bars[B_VNREADY], c & 1, 17);
        __syncwarp();
        tc_fence_after();
        if (leader) trace_mark<TRACE>(P, c, TR_MMA_C2);
        const uint32_t kq = smem_u32(stage(c) + L::OFF_KQ);
        // fast chunks: gamma is folded into U^T and W^T, so Vn^T itself; slow chunks:
        // the separate Vn^T gamma operand
        const bool fastc = reinterpret_cast<const int*>(misc(c))[L::M_FAST / 4] != 0;
        if constexpr (L::VN_TMEM) {
          const uint32_t a0 = vn + (fastc ? 0 : kC / 2);
#pragma unroll
          for (int ks = 0; ks < kC / 16; ++ks) {
            const uint64_t bd = sdesc_sw128(kq + (KDA ? L::OFF_K2 : 0) + ks * 2048, L::KQ_REGION, 1024);
            if (leader) umma_ts(t_sm, a0 + ks * 8, bd, ID_S, 1);
          }
        } else {
          const uint32_t s_vs = fastc ? s_vnt : s_vng;
#pragma unroll
          for (int ks = 0; ks < kC / 16; ++ks) {
            const uint64_t ad = sdesc_sw128(s_vs + ks * 32, 16, 1024);
            // KDA: the state update reads K e^-g (the per-dimension e^{g_tot} is applied
            // to the whole state afterwards, in the state pass)
            const uint64_t bd = sdesc_sw128(kq + (KDA ? L::OFF_K2 : 0) + ks * 2048, L::KQ_REGION, 1024);
            if (leader) umma_ss(t_sm, ad, bd, ID_S, 1);
          }
        }
        commit(&bars[B_SFULL]);
        commit(&bars[B_EMPTY0 + (c % L::NIN)]);
        if (L::VN_TMEM) commit(&bars[B_VNFREE0 + (c & 1)]);
      }
    } else if (warp == 3) {
      for (int c = 0; c < nc; ++c) {
        sy.wait(&bars[B_SREADY], c & 1, 40);
        // Q' of slow chunks is written before A(c) is handed over, long before W^T(c)
        sy.wait(&bars[B_WREADY], c & 1, 42);
        if (c >= 1) sy.wait(&bars[B_OFREE], (c - 1) & 1, 16);
        __syncwarp();
        tc_fence_after();
        const uint32_t kq = smem_u32(stage(c) + L::OFF_KQ);
#pragma unroll
        for (int ks = 0; ks < DK / 16; ++ks) {
          const uint64_t bd =
              sdesc_sw128(kq + (ks >> 2) * L::KQ_REGION + kC * 128 + (ks & 3) * 32, 16, 1024);
          if (leader) {
            if constexpr (L::SA_TMEM) umma_ts(t_o, t_sa + ks * 8, bd, ID_O1, ks > 0);
            else umma_ss(t_o, a_desc_sa(ks), bd, ID_O1, ks > 0);
          }
        }
        commit(&bars[B_O1DONE]);   // the bf16 S^T copy may be overwritten after this
        sy.wait(&bars[B_VNREADY], c & 1, 41);
        __syncwarp();
        tc_fence_after();
        const uint32_t aq = smem_u32(aqk(c));
        const uint32_t vn = t_vn(c);
#pragma unroll
        for (int ks = 0; ks < kC / 16; ++ks) {
          const uint64_t bd = sdesc_sw128(aq + ks * 32, 16, 1024);
          if (leader) {
            if constexpr (L::VN_TMEM) umma_ts(t_o, vn + ks * 8, bd, ID_O2, 1);
            else umma_ss(t_o, sdesc_sw128(s_vnt + ks * 32, 16, 1024), bd, ID_O2, 1);
          }
        }
        commit(&bars[B_OFULL0 + (c % 3)]);
        commit(&bars[B_EMPTY0 + (c % L::NIN)]);
        if (L::VN_TMEM) commit(&bars[B_VNFREE0 + (c & 1)]);
      }
    } else {
      // P0(c) = [K;Q] K^T -> KQ, then P1(c - 1) = (W^T, U^T) of the previous chunk:
      // P0(c) needs only E(c - 1) to have drained KQ, P1(c - 1) needs T'(c - 1)
      for (int c = 0; c <= nc; ++c) {
        if (c < nc) {
          sy.wait(&bars[B_FULL0 + (c % L::NIN)], in_par(c), 10);
          if (c >= 1) sy.wait(&bars[B_KQFREE], (c - 1) & 1, 11);
          __syncwarp();
          tc_fence_after();
          const uint32_t kq = smem_u32(stage(c) + L::OFF_KQ);
#pragma unroll
          for (int ks = 0; ks < DK / 16; ++ks) {
            const uint64_t d = sdesc_sw128(kq + (ks >> 2) * L::KQ_REGION + (ks & 3) * 32, 16, 1024);
            // KDA: [K e^g; Q e^g] (K e^-g)^T, the gate on the operands
            const uint64_t db = KDA ? sdesc_sw128(kq + (ks >> 2) * L::KQ_REGION + L::OFF_K2 +
                                                  (ks & 3) * 32, 16, 1024)
                                    : d;
            if (leader) umma_ss(t_kq, d, db, ID_KQ, ks > 0);
          }
          commit(&bars[B_KQFULL]);
        }
        if (c >= 1) {
          const int cp = c - 1;
          sy.wait(&bars[B_TREADY], cp & 1, 13);
          sy.wait(&bars[B_VFULL], cp & 1, 18);
          if (cp >= 2) sy.wait(&bars[B_VNFREE0 + (cp & 1)], ((cp >> 1) + 1) & 1, 19);
          if (cp >= 1) sy.wait(&bars[B_RWFREE], (cp - 1) & 1, 9);
          __syncwarp();
          tc_fence_after();
          const uint32_t kq = smem_u32(stage(cp) + L::OFF_KQ);
          const uint32_t vt = smem_u32(sm + L::OFF_V);
          const uint32_t t_u = t_vn(cp);
#pragma unroll
          for (int ks = 0; ks < kC / 16; ++ks) {
            const uint64_t ka = sdesc_sw128(kq + ks * 2048, L::KQ_REGION, 1024);
            const uint64_t tb = sdesc_sw128(s_tp + ks * 32, 16, 1024);
            const uint64_t va = sdesc_sw128(vt + ks * 2048, L::V_REGION, 1024);
            const uint64_t ub = sdesc_sw128(s_tpp + ks * 32, 16, 1024);
            if (leader) {
              umma_ss(t_rw, ka, tb, ID_WT, ks > 0);
              umma_ss(t_u, va, ub, ID_UT, ks > 0);
            }
          }
          commit(&bars[B_WUFULL]);
        }
      }
    }
    commit(&bars[B_DONE]);
  }
  // =============================================================== PREP ====
  // Two warpgroups, each one chunk at a time, handing chunks over through mbarriers:
  //   Q (warps 8-11)  E(c): coefficients, [K;Q]K^T epilogue -> A (fp16, 2 buffers)
  //                   and Aqk (2 buffers), slow chunks: Q' = Q e^g
  //   P (warps 4-7)   I(c): (I + A)^-1, T' and T'' -> UMMA W^T, U^T;
  //                   R(c - 1): W^T readout (2 buffers) -> chain of chunk c - 1
  // so E(c + 1) runs beside I(c) and the readout lags one chunk behind its UMMA.
  // Warp quadrant q = warp & 3 selects TMEM lanes 32q..32q+31 (row r = 32q + lane).
  else if (warp >= 8 && warp < 12) {
    const int qp = tid - 256, q = warp & 3, l = lane;
    const int r = 32 * q + l;
    const uint32_t t_kq = tmem + L::T_KQ + ((32u * q) << 16);
    const uint32_t t_rw = tmem + L::T_RW + ((32u * q) << 16);
    // V tile of chunk cv (read by the U^T UMMA only; single buffer, loaded once the
    // previous chunk's WY UMMAs have completed)
    auto issue_v = [&](int cv) {
      const int t0 = cv * kC;
      const bool bhtd = (P.layout == PTOF_LAYOUT_BHTD);
      const int y = bhtd ? t0 : h, z = bhtd ? bh : static_cast<int>(tok0 + t0);
      mbar_arrive_expect_tx(&bars[B_VFULL], DV * kC * 2);
#pragma unroll
      for (int vb = 0; vb < L::NVB; ++vb) {
        if (P.view)
          tma_load_4d(sm + L::OFF_V + vb * L::V_REGION, &P.mapV, &bars[B_VFULL], vb * 64, t0, h, b);
        else
          tma_load_3d(sm + L::OFF_V + vb * L::V_REGION, &P.mapV, &bars[B_VFULL], vb * 64, y, z);
      }
    };
    int v_issued = -1;   // last chunk whose V load was issued (drained at exit)
    if (qp == 0) {
      prefetch_tmap(&P.mapV);
      issue_v(0);
      v_issued = 0;
    }
    // E(c), then R(c - 1): the W^T readout follows its WY UMMAs as closely as the
    // epilogue allows, so the chain of chunk c - 1 starts early
    for (int c = 0; c <= nc; ++c) {
      if (c < nc) {
      unsigned char* st = stage(c);
      float* ms = misc(c);
      const float* gcum = ms + L::M_GCUM / 4;
      sy.wait(&bars[B_FULL0 + (c % L::NIN)], in_par(c), 20);
      if (qp == 0) trace_mark<TRACE>(P, c, TR_PREP_FULL);
      const bool fast = reinterpret_cast<const int*>(ms)[L::M_FAST / 4] != 0;
      // A buffer c & 1 last held A(c - 2) / T(c - 2); Aqk buffer c % 3 last fed O(c - 3)
      if (c >= 2) sy.wait(&bars[B_TAFREE0 + (c & 1)], ((c >> 1) + 1) & 1, 23);
      if (c >= 3) sy.wait(&bars[B_OFULL0 + (c % 3)], aq_par(c) ^ 1, 24);
      if (qp == 0) trace_mark<TRACE>(P, c, TR_PREP_OFULL);
      sy.wait(&bars[B_KQFULL], c & 1, 21);
      tc_fence_after();
      if (qp == 0) trace_mark<TRACE>(P, c, TR_PREP_KQ);
      // ---- A = gated strict-lower KK^T (rows 0-63), Aqk = gated causal QK^T (64-127),
      //      16 columns per iteration (rolled: the per-chunk code of all warps must
      //      fit the SM's instruction cache) ----
      const int i = r & 63;
      const bool is_k = r < 64;
      const int lim = is_k ? i : i + 1;       // strict lower (A) / causal (Aqk)
      // fast chunks: A = rowf_i beta_i colf_j KK^T and Aqk = e^{-gl} QK^T (the e^{g_i}
      // of the score is applied at the output)
      const float rowm = is_k ? ms[L::M_ROWFB / 4 + i] : ms[L::M_ENGL / 4];
      unsigned char* dst = is_k ? (sm + L::OFF_TA + (c & 1) * 8192) : aqk(c);
#pragma unroll 1
      for (int j0 = 0; j0 < kC; j0 += 16) {
        float v[16];
        tmem_ld16(t_kq + j0, v);
        tmem_wait_ld();
        if (fast) {
          if constexpr (DK == 64) {
            // D = 64: vector loads of the column factors (measured faster there; the
            // D = 128 kernel measured slower with them and keeps the scalar loads)
            float cl[16];
#pragma unroll
            for (int m = 0; m < 16; m += 4)
              *reinterpret_cast<float4*>(cl + m) =
                  *reinterpret_cast<const float4*>(ms + L::M_COLF / 4 + j0 + m);
#pragma unroll
            for (int m = 0; m < 16; ++m) {
              const float cf = is_k ? rowm * cl[m] : rowm;
              v[m] = (j0 + m < lim) ? v[m] * cf : 0.f;
            }
          } else {
#pragma unroll
            for (int m = 0; m < 16; ++m) {
              const float cf = is_k ? rowm * ms[L::M_COLF / 4 + j0 + m] : rowm;
              v[m] = (j0 + m < lim) ? v[m] * cf : 0.f;
            }
          }
        } else {
          // exact per-element coefficients: K rows beta_i * kkt_coef, Q rows qk_coef
          // (one exponential each: both are exp(min(x, 0)) up to the x > 0 cut of kkt)
          const float gi = gcum[i], bi = is_k ? ms[L::M_BV / 4 + i] : 1.f;
          const float xcut = is_k ? 0.f : 3.0e38f;
#pragma unroll
          for (int m = 0; m < 16; ++m) {
            const float x = gi - gcum[j0 + m];
            const float cf = (x <= xcut) ? __expf(fminf(x, 0.f)) * bi : 0.f;
            v[m] = (j0 + m < lim) ? v[m] * cf : 0.f;
          }
        }
        // A in fp16 (operand of the inverse), Aqk in the input type (score UMMA operand)
        uint32_t pk[8];
#pragma unroll
        for (int m = 0; m < 8; ++m)
          pk[m] = is_k ? pack_f16(v[2 * m], v[2 * m + 1]) : pack2<F16>(v[2 * m], v[2 * m + 1]);
        st_chunk(dst, i, j0 / 8, make_uint4(pk[0], pk[1], pk[2], pk[3]));
        st_chunk(dst, i, j0 / 8 + 1, make_uint4(pk[4], pk[5], pk[6], pk[7]));
      }
      tc_fence_before();
      if (!fast) {
        // slow chunks: Q' = Q e^g in place (P0 has read Q: KQFULL)
        const float* eg = ms + L::M_EG / 4;
        constexpr int NCH = DK / 8;
        for (int idx = qp; idx < kC * NCH; idx += 128) {
          const int ii = idx / NCH, ch = idx % NCH;
          unsigned char* reg = st + L::OFF_KQ + (ch >> 3) * L::KQ_REGION + kC * 128;
          uint4 u4 = ld_chunk(reg, ii, ch & 7);
          uint32_t* w = reinterpret_cast<uint32_t*>(&u4);
          const float e = eg[ii];
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const float2 f = unpack2<F16>(w[m]);
            w[m] = pack2<F16>(f.x * e, f.y * e);
          }
          st_chunk(reg, ii, ch & 7, u4);
        }
      }
      fence_async_smem();   // Aqk and Q' are read by the UMMA unit
      named_bar_sync(kQBar, 128);
      if (qp == 0) {
        mbar_arrive(&bars[B_KQFREE]);
        mbar_arrive(&bars[B_AREADY0 + (c & 1)]);
        trace_mark<TRACE>(P, c, TR_PREP_EPI);
      }
      }
      if (c >= 1) {
        // ================= R(c - 1): W^T readout =================
        const int cp = c - 1;
        const bool wu = sy.wait(&bars[B_WUFULL], cp & 1, 27);
        // P1(cp) has read V(cp), so the single V buffer takes V(cp + 1); never after an
        // abort (a V load still in flight would be armed twice)
        if (cp + 1 < nc && qp == 0 && wu && !abort_flag) {
          issue_v(cp + 1);
          v_issued = cp + 1;
        }
        // the W^T tile was last read by the chain UMMA of chunk cp - 1
        if (cp >= 1) sy.wait(&bars[B_WTFREE], (cp - 1) & 1, 28);
        tc_fence_after();
        if (qp == 0) trace_mark<TRACE>(P, cp, TR_PREP_WU);
        unsigned char* wt = sm + L::OFF_WT;
        if constexpr (DK == 128) {
          const int d = 32 * q + l;
#pragma unroll 1
          for (int j0 = 0; j0 < kC; j0 += 16) {
            float a0[16];
            tmem_ld16(t_rw + j0, a0);
            tmem_wait_ld();
            uint32_t pk[8];
#pragma unroll
            for (int m = 0; m < 8; ++m) pk[m] = pack2<F16>(a0[2 * m], a0[2 * m + 1]);
            st_chunk(wt, d, j0 / 8, make_uint4(pk[0], pk[1], pk[2], pk[3]));
            st_chunk(wt, d, j0 / 8 + 1, make_uint4(pk[4], pk[5], pk[6], pk[7]));
          }
        } else {
          // M = 64 accumulator: lanes 0-15 read columns 0-31 of row 16q + l, lanes
          // 16-31 columns 32-63 of row 16q + l - 16 (16x32bx2 loads)
          const int d = 16 * q + (l & 15), jb = 32 * (l >> 4);
#pragma unroll 1
          for (int j0 = 0; j0 < 32; j0 += 16) {
            float a0[16];
            tmem_ld16_split<32>(t_rw + j0, a0);
            tmem_wait_ld();
            uint32_t pk[8];
#pragma unroll
            for (int m = 0; m < 8; ++m) pk[m] = pack2<F16>(a0[2 * m], a0[2 * m + 1]);
            st_chunk(wt, d, (jb + j0) / 8, make_uint4(pk[0], pk[1], pk[2], pk[3]));
            st_chunk(wt, d, (jb + j0) / 8 + 1, make_uint4(pk[4], pk[5], pk[6], pk[7]));
          }
        }
        tc_fence_before();
        fence_async_smem();
        named_bar_sync(kQBar, 128);
        if (qp == 0) {
          mbar_arrive(&bars[B_WREADY]);
          mbar_arrive(&bars[B_RWFREE]);
          trace_mark<TRACE>(P, cp, TR_PREP_END);
        }
      }
    }
    if (qp == 0 && v_issued >= 0) drain_wait(&bars[B_VFULL], v_issued & 1);
  } else if (warp >= 4 && warp < 8) {
    const int pp = tid - 128, q = warp & 3, l = lane;
    unsigned char* s_tp = sm + L::OFF_TP;
    unsigned char* s_tpp = sm + L::OFF_TPP;
    for (int c = 0; c < nc; ++c) {
      float* ms = misc(c);
      // A(c) in, T(c) out, in place (the strictly upper blocks of A are zero)
      unsigned char* s_td = sm + L::OFF_TA + (c & 1) * 8192;
      if (c < nc) {
        // ================= I(c): T = (I + A)^-1 =================
        sy.wait(&bars[B_AREADY0 + (c & 1)], (c >> 1) & 1, 25);
        const unsigned char* s_ta = s_td;
        if (pp == 0) trace_mark<TRACE>(P, c, TR_INV_START);
        (void)s_ta;
        tri_inv64_inplace(s_td, warp - 4, l, 4, kPBar);
        if (pp == 0) trace_mark<TRACE>(P, c, TR_PREP_INV);
      }
      if (c < nc) {
        const bool fast = reinterpret_cast<const int*>(ms)[L::M_FAST / 4] != 0;
        // ---- T' = T * (beta e^g)_j, T'' = T * beta_j (K-major B operands); fast
        //      chunks also scale row i by gamma_i so the UMMAs yield W^T g, U^T g.
        //      T' / T'' of chunk c - 1 must have been consumed (WUFULL(c - 1)). ----
        if (c >= 1) sy.wait(&bars[B_WUFULL], (c - 1) & 1, 26);
        {
          const int i = pp >> 1;
          const float gi = fast ? ms[L::M_GAM / 4 + i] : 1.f;
#pragma unroll 1
          for (int j0 = 32 * (pp & 1); j0 < 32 * (pp & 1) + 32; j0 += 16) {
            float tv[16];
            {
              const uint4 u0 = ld_chunk(s_td, i, j0 / 8), u1 = ld_chunk(s_td, i, j0 / 8 + 1);
              const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
              for (int m = 0; m < 8; ++m) {
                const float2 f = unpack_f16(w[m]);
                tv[2 * m] = f.x * gi;
                tv[2 * m + 1] = f.y * gi;
              }
            }
            uint32_t a[8], bb[8];
            if constexpr (DK == 64) {   // vector loads at D = 64 only (as for the column factors)
              float bk[16], bv[16];
#pragma unroll
              for (int m = 0; m < 16; m += 4) {
                *reinterpret_cast<float4*>(bk + m) = *reinterpret_cast<const float4*>(ms + L::M_BK / 4 + j0 + m);
                *reinterpret_cast<float4*>(bv + m) = *reinterpret_cast<const float4*>(ms + L::M_BV / 4 + j0 + m);
              }
#pragma unroll
              for (int m = 0; m < 8; ++m) {
                a[m] = pack2<F16>(tv[2 * m] * bk[2 * m], tv[2 * m + 1] * bk[2 * m + 1]);
                bb[m] = pack2<F16>(tv[2 * m] * bv[2 * m], tv[2 * m + 1] * bv[2 * m + 1]);
              }
            } else {
              const float* bk = ms + L::M_BK / 4 + j0;
              const float* bv = ms + L::M_BV / 4 + j0;
#pragma unroll
              for (int m = 0; m < 8; ++m) {
                a[m] = pack2<F16>(tv[2 * m] * bk[2 * m], tv[2 * m + 1] * bk[2 * m + 1]);
                bb[m] = pack2<F16>(tv[2 * m] * bv[2 * m], tv[2 * m + 1] * bv[2 * m + 1]);
              }
            }
            st_chunk(s_tp, i, j0 / 8, make_uint4(a[0], a[1], a[2], a[3]));
            st_chunk(s_tp, i, j0 / 8 + 1, make_uint4(a[4], a[5], a[6], a[7]));
            st_chunk(s_tpp, i, j0 / 8, make_uint4(bb[0], bb[1], bb[2], bb[3]));
            st_chunk(s_tpp, i, j0 / 8 + 1, make_uint4(bb[4], bb[5], bb[6], bb[7]));
          }
        }
        fence_async_smem();
        named_bar_sync(kPBar, 128);
        if (pp == 0) {
          mbar_arrive(&bars[B_TAFREE0 + (c & 1)]);   // T(c) fully read
          mbar_arrive(&bars[B_TREADY]);
          trace_mark<TRACE>(P, c, TR_PREP_TREADY);
        }
      }
    }
  }
  // =============================================================== SCAN ====
  else if (warp >= 12 && warp < 16) {
    const int s = tid - 384, q = warp & 3, l = lane;
    const int v = (DV == 128) ? (32 * q + l) : (l < 16 ? 16 * q + l : -1);
    const uint32_t lane_off = (32u * q) << 16;
    const uint32_t t_sm = tmem + L::T_SM + lane_off, t_sa = tmem + L::T_SA + lane_off;
    const uint32_t t_o = tmem + L::T_O + lane_off;
    unsigned char* s_vnt = sm + L::OFF_VNT;
    unsigned char* s_vng = sm + L::OFF_VNG;
    unsigned char* s_sa = sm + L::OFF_SA;
    (void)s_sa;
    float* osc = reinterpret_cast<float*>(sm + L::OFF_OSC);
    const int64_t sbase = static_cast<int64_t>(bh) * DK * DV;

    // smem variant of the bf16 S^T copy (K-major A operand, rows v, DK columns)
    auto put_sa = [&](int d0, const float (&x)[16]) {
      if (v >= 0) {
        uint32_t pk[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) pk[m] = pack2<F16>(x[2 * m], x[2 * m + 1]);
        unsigned char* reg = s_sa + (d0 >> 6) * (DV * 128);
        st_chunk(reg, v, (d0 & 63) / 8, make_uint4(pk[0], pk[1], pk[2], pk[3]));
        st_chunk(reg, v, (d0 & 63) / 8 + 1, make_uint4(pk[4], pk[5], pk[6], pk[7]));
      }
    };
    // One pass over S^T row v in 32-column pieces: optional source (global S0),
    // bf16 copy -> SA, then master <- scale * value.
    // KDA: `md` (per key dimension d) scales the state first: the per-dimension decay
    // of the chunk just completed, so S_{c+1} = e^{g_tot} (S_c + (K e^-g)^T V_new)
    auto state_pass = [&](bool from_global, float mult, float* final_out, const float* md) {
      if constexpr (!L::SA_TMEM && DK == 64) {
        // M = 64 master (lanes 32q .. 32q + 15): lanes 0-15 take key columns 0-31 of
        // row 16q + l, lanes 16-31 columns 32-63 of row 16q + l - 16 (16x32bx2 shape)
        const int vr = 16 * q + (l & 15), db = 32 * (l >> 4);
        float x[32];
        if (from_global) {
#pragma unroll
          for (int m = 0; m < 32; ++m)
            x[m] = P.S0 ? P.S0[sbase + static_cast<int64_t>(db + m) * DV + vr] : 0.f;
        } else {
          tmem_ld16_split<32>(t_sm, *reinterpret_cast<float(*)[16]>(x));
          tmem_ld16_split<32>(t_sm + 16, *reinterpret_cast<float(*)[16]>(x + 16));
          tmem_wait_ld();
        }
        if constexpr (KDA) {
          if (md != nullptr) {
#pragma unroll
            for (int m = 0; m < 32; ++m) x[m] *= md[db + m];
          }
        }
        if (final_out) {
#pragma unroll
          for (int m = 0; m < 32; ++m) final_out[sbase + static_cast<int64_t>(db + m) * DV + vr] = x[m];
          return;
        }
        uint32_t pk[16];
#pragma unroll
        for (int m = 0; m < 16; ++m) pk[m] = pack2<F16>(x[2 * m], x[2 * m + 1]);
        st_chunk(s_sa, vr, db / 8, make_uint4(pk[0], pk[1], pk[2], pk[3]));
        st_chunk(s_sa, vr, db / 8 + 1, make_uint4(pk[4], pk[5], pk[6], pk[7]));
        st_chunk(s_sa, vr, db / 8 + 2, make_uint4(pk[8], pk[9], pk[10], pk[11]));
        st_chunk(s_sa, vr, db / 8 + 3, make_uint4(pk[12], pk[13], pk[14], pk[15]));
        float y0[16], y1[16];
#pragma unroll
        for (int m = 0; m < 16; ++m) { y0[m] = x[m] * mult; y1[m] = x[16 + m] * mult; }
        tmem_st16f_split<32>(t_sm, y0);
        tmem_st16f_split<32>(t_sm + 16, y1);
        tmem_wait_st();
        return;
      }
#pragma unroll 1
      for (int d0 = 0; d0 < DK; d0 += 32) {
        float x[32];
        if (from_global) {
#pragma unroll
          for (int m = 0; m < 32; ++m)
            x[m] = (P.S0 && v >= 0) ? P.S0[sbase + static_cast<int64_t>(d0 + m) * DV + v] : 0.f;
        } else {
          float a[16], bq[16];
          tmem_ld16(t_sm + d0, a);
          tmem_ld16(t_sm + d0 + 16, bq);
          tmem_wait_ld();
#pragma unroll
          for (int m = 0; m < 16; ++m) { x[m] = a[m]; x[16 + m] = bq[m]; }
        }
        if constexpr (KDA) {
          if (md != nullptr) {
#pragma unroll
            for (int m = 0; m < 32; ++m) x[m] *= md[d0 + m];
          }
        }
        if (final_out) {
          if (v >= 0) {
#pragma unroll
            for (int m = 0; m < 32; ++m) final_out[sbase + static_cast<int64_t>(d0 + m) * DV + v] = x[m];
          }
          continue;
        }
        if constexpr (L::SA_TMEM) {
          uint32_t pk[16];
#pragma unroll
          for (int m = 0; m < 16; ++m) pk[m] = pack2<F16>(x[2 * m], x[2 * m + 1]);
          tmem_st16(t_sa + d0 / 2, pk);
        } else {
          float lo[16], hi[16];
#pragma unroll
          for (int m = 0; m < 16; ++m) { lo[m] = x[m]; hi[m] = x[16 + m]; }
          put_sa(d0, lo);
          put_sa(d0 + 16, hi);
        }
        float y0[16], y1[16];
#pragma unroll
        for (int m = 0; m < 16; ++m) { y0[m] = x[m] * mult; y1[m] = x[16 + m] * mult; }
        tmem_st16f(t_sm + d0, y0);
        tmem_st16f(t_sm + d0 + 16, y1);
      }
      tmem_wait_st();
    };

    sy.wait(&bars[B_FULL0], 0, 30);  // chunk 0
    // initial state: S^T <- S0 (or 0); GDN pre-scales the master by e^{g_last} of chunk
    // 0, KDA applies its per-dimension decays after each chunk's update instead
    state_pass(true, KDA ? 1.f : misc(0)[L::M_EGL / 4], nullptr, nullptr);
    tc_fence_before();
    if (!L::SA_TMEM) fence_async_smem();
    named_bar_sync(kScanBar, 128);
    if (s == 0) mbar_arrive(&bars[B_SREADY]);

    for (int c = 0; c < nc; ++c) {
      const float* ms = misc(c);
      // ---- (a) V_new^T row v -> bf16 A operands Vn^T and Vn^T*gamma ----
      sy.wait(&bars[B_VNFULL], c & 1, 31);
      tc_fence_after();
      if (s == 0) trace_mark<TRACE>(P, c, TR_SCAN_VNFULL);
      const bool fastc = reinterpret_cast<const int*>(ms)[L::M_FAST / 4] != 0;
      if (s < kC) osc[(c & 1) * kC + s] = fastc ? P.scale * ms[L::M_EG / 4 + s] : P.scale;
      const uint32_t t_vn = tmem + ((c & 1) ? L::T_VN1 : L::T_VN0) + lane_off;
      const float* gam = ms + L::M_GAM / 4;
      if constexpr (L::VN_TMEM) {
        // in place: the fp32 row (64 columns) becomes bf16 Vn^T in columns 0-31 and,
        // for slow chunks, bf16 Vn^T gamma in columns 32-63 (TMEM A operands)
        float x[kC];
#pragma unroll
        for (int c0 = 0; c0 < kC; c0 += 16) tmem_ld16(t_vn + c0, *reinterpret_cast<float(*)[16]>(x + c0));
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
          for (int m = 0; m < 16; ++m) pk[m] = pack2<F16>(x[32 * hh + 2 * m], x[32 * hh + 2 * m + 1]);
          tmem_st16(t_vn + 16 * hh, pk);
        }
        if (!fastc) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
            for (int m = 0; m < 16; ++m) {
              const int t = 32 * hh + 2 * m;
              pk[m] = pack2<F16>(x[t] * gam[t], x[t + 1] * gam[t + 1]);
            }
            tmem_st16(t_vn + kC / 2 + 16 * hh, pk);
          }
        }
        tmem_wait_st();
      } else {
        // M = 64 accumulator (lanes 32q .. 32q + 15): lanes 0-15 convert columns 0-31 of
        // row 16q + l, lanes 16-31 columns 32-63 of row 16q + l - 16 (16x32bx2 loads)
        const int vr = 16 * q + (l & 15), cb = 32 * (l >> 4);
#pragma unroll 1
        for (int c0 = 0; c0 < 32; c0 += 16) {
          float x[16];
          tmem_ld16_split<32>(t_vn + c0, x);
          tmem_wait_ld();
          const int cc = cb + c0;
          uint32_t a[8];
#pragma unroll
          for (int m = 0; m < 8; ++m) a[m] = pack2<F16>(x[2 * m], x[2 * m + 1]);
          st_chunk(s_vnt, vr, cc / 8, make_uint4(a[0], a[1], a[2], a[3]));
          st_chunk(s_vnt, vr, cc / 8 + 1, make_uint4(a[4], a[5], a[6], a[7]));
          if (!fastc) {
            uint32_t gq[8];
#pragma unroll
            for (int m = 0; m < 8; ++m)
              gq[m] = pack2<F16>(x[2 * m] * gam[cc + 2 * m], x[2 * m + 1] * gam[cc + 2 * m + 1]);
            st_chunk(s_vng, vr, cc / 8, make_uint4(gq[0], gq[1], gq[2], gq[3]));
            st_chunk(s_vng, vr, cc / 8 + 1, make_uint4(gq[4], gq[5], gq[6], gq[7]));
          }
        }
        fence_async_smem();
      }
      tc_fence_before();
      named_bar_sync(kScanBar, 128);
      if (s == 0) {
        mbar_arrive(&bars[B_VNREADY]);
        trace_mark<TRACE>(P, c, TR_SCAN_VNREADY);
        if (!L::VN_TMEM) mbar_arrive(&bars[B_VNFREE0 + (c & 1)]);
        mbar_arrive(&bars[B_EMPTY0 + (c % L::NIN)]);
      }
      // ---- (b) state: S^T_{c+1} ready -> bf16 copy, pre-scale by e^{gl_{c+1}} ----
      sy.wait(&bars[B_SFULL], c & 1, 32);
      sy.wait(&bars[B_O1DONE], c & 1, 35);  // the output UMMA has read the bf16 S^T copy
      tc_fence_after();
      if (s == 0) trace_mark<TRACE>(P, c, TR_SCAN_SFULL);
      if (c + 1 < nc) {
        sy.wait(&bars[B_FULL0 + ((c + 1) % L::NIN)], in_par(c + 1), 33);
        // KDA: the stage of chunk c + 1 carries the decay of chunk c
        state_pass(false, KDA ? 1.f : misc(c + 1)[L::M_EGL / 4], nullptr,
                   KDA ? reinterpret_cast<const float*>(sm + L::OFF_EGLD +
                                                        ((c + 1) % L::NIN) * L::EGLD_BYTES)
                       : nullptr);
        tc_fence_before();
        if (!L::SA_TMEM) fence_async_smem();
        named_bar_sync(kScanBar, 128);
        if (s == 0) {
          mbar_arrive(&bars[B_SREADY]);
          trace_mark<TRACE>(P, c, TR_SCAN_SREADY);
        }
      } else if (P.S_final) {
        state_pass(false, 1.f, P.S_final,
                   KDA ? P.egl + (static_cast<int64_t>(bh) * (P.nc + 1) + nc) * DK : nullptr);
      }
      if constexpr (!Roles<DK>::OUT_GROUP) output_chunk(c, s, kScanBar);
    }
  }
  // ============================================================= OUTPUT ====
  // (D = 64 only) a group of its own for the output stores
  else if (Roles<DK>::OUT_GROUP) {
    for (int c = 0; c < nc; ++c) output_chunk(c, tid - 512, kOutBar);
  }

  // ============================================================ teardown ====
  if (warp >= 1 && warp <= 3 && lane == 0) {
    // every UMMA has retired before TMEM is released (bounded, even after an abort)
    drain_wait(&bars[B_DONE], 0);
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem, L::T_COLS);
  if (TRACE && tid == 0) {
    // per-CTA record after the chunk table: start ns, end ns, SM id
    unsigned long long* rec = P.trace + P.trace_chunks * kTraceSlots + 4 * blockIdx.x;
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    rec[0] = t_start;
    rec[1] = globaltimer_ns();
    rec[2] = smid;
  }
}

// ---------------------------------------------------------- KDA operand pre-pass ----
// Kimi Delta Attention gates every key dimension separately (per-token log decay g
// [B,H,T,DK]), so the gate cannot ride on the scores as GDN's does: it rides on the
// operands, as in the reference's factorised chunk form (examples/attention/
// _kda_full.py:38-77, the prologue keys of kernels/qkv_prologue_fused.h). Per chunk
// with G the chunk-local cumsum, this pass writes K e^G, Q e^G, K e^-G (bf16) and the
// chunk's per-dimension decay e^{G_last} into slot c + 1 of `egl` (slot 0 = 1), so
// the fused kernel runs the ungated GDN chain on these operands. One thread per key
// dimension and token group covers 16 tokens of one chunk (coalesced rows of g, k, q).
struct KdaPrepParams {
  const __nv_bfloat16 *q, *k;
  const float* g;
  __nv_bfloat16 *q1, *k1, *k2;
  float* egl;
  int nc, T;
};
// 4 DK threads: thread (j, d2) handles the dimension pair 2 d2, 2 d2 + 1 of the 8
// tokens 8 j .. 8 j + 7 (4-byte loads and stores; every load of q, k and g is issued
// before the prefix), the 8 token groups joined by a prefix over shared memory.
template <int DK>
__global__ void __launch_bounds__(4 * DK) kda_prep_kernel(const __grid_constant__ KdaPrepParams P) {
  constexpr int ND = DK / 2;          // dimension pairs
  constexpr int NG = 4 * DK / ND;     // token groups
  constexpr int TPG = kC / NG;        // tokens per group
  static_assert(NG * TPG == kC, "token groups");
  __shared__ float2 part[NG][ND];
  const int d2 = threadIdx.x % ND, j = threadIdx.x / ND;
  const int bh = blockIdx.x / P.nc, c = blockIdx.x % P.nc;
  const int64_t row0 =
      static_cast<int64_t>(bh) * P.T + static_cast<int64_t>(c) * kC + TPG * j;
  const int64_t base = row0 * ND + d2;   // in dimension pairs
  const float2* g2 = reinterpret_cast<const float2*>(P.g) + base;
  const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(P.k) + base;
  const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(P.q) + base;
  float2 gl[TPG];
  __nv_bfloat162 kk[TPG], qq[TPG];
#pragma unroll
  for (int i = 0; i < TPG; ++i) {
    gl[i] = g2[i * ND];
    kk[i] = k2[i * ND];
    qq[i] = q2[i * ND];
  }
#pragma unroll
  for (int i = 1; i < TPG; ++i) {
    gl[i].x += gl[i - 1].x;
    gl[i].y += gl[i - 1].y;
  }
  part[j][d2] = gl[TPG - 1];
  __syncthreads();
  float2 off = make_float2(0.f, 0.f);
  for (int jj = 0; jj < j; ++jj) {
    off.x += part[jj][d2].x;
    off.y += part[jj][d2].y;
  }
  __nv_bfloat162* k1o = reinterpret_cast<__nv_bfloat162*>(P.k1) + base;
  __nv_bfloat162* q1o = reinterpret_cast<__nv_bfloat162*>(P.q1) + base;
  __nv_bfloat162* k2o = reinterpret_cast<__nv_bfloat162*>(P.k2) + base;
#pragma unroll
  for (int i = 0; i < TPG; ++i) {
    const float Gx = gl[i].x + off.x, Gy = gl[i].y + off.y;
    const float ux = __expf(Gx), uy = __expf(Gy), dx = __expf(-Gx), dy = __expf(-Gy);
    const float2 kf = __bfloat1622float2(kk[i]), qf = __bfloat1622float2(qq[i]);
    k1o[i * ND] = __floats2bfloat162_rn(kf.x * ux, kf.y * uy);
    q1o[i * ND] = __floats2bfloat162_rn(qf.x * ux, qf.y * uy);
    k2o[i * ND] = __floats2bfloat162_rn(kf.x * dx, kf.y * dy);
  }
  if (j == NG - 1) {
    float2* eg = reinterpret_cast<float2*>(P.egl + static_cast<int64_t>(bh) * (P.nc + 1) * DK);
    eg[static_cast<int64_t>(c + 1) * ND + d2] =
        make_float2(__expf(gl[TPG - 1].x + off.x), __expf(gl[TPG - 1].y + off.y));
    if (c == 0) eg[d2] = make_float2(1.f, 1.f);
  }
}

}  // namespace tcfwd

// ------------------------------------------------------------------- host ----
namespace {

// 3D TMA map over a [.., D]-innermost activation so that one box is 64 tokens x 64
// features of one (batch, head): heads-outer layout -> dims {D, T, B*H};
// token-major layout -> dims {D, H, B*T}.
// 3D TMA map over a [.., D]-innermost activation with `heads` heads so that one box
// is 64 tokens x 64 features of one head: heads-outer layout -> dims {D, T, B*heads};
// token-major layout -> dims {D, heads, tokens} with tokens = B*T or the packed total.
int make_act_map(CUtensorMap* m, const void* base, int dt, const ptof_gdn_params& p, int D,
                 int heads, int64_t tokens) {
  const CUtensorMapDataType t =
      dt == PTOF_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  uint64_t dims[3], strides[2];
  uint32_t box[3];
  if (p.layout == PTOF_LAYOUT_BHTD) {
    dims[0] = D; dims[1] = p.T; dims[2] = static_cast<uint64_t>(p.B) * heads;
    strides[0] = static_cast<uint64_t>(D) * 2;
    strides[1] = static_cast<uint64_t>(p.T) * D * 2;
    box[0] = 64; box[1] = 64; box[2] = 1;
  } else {
    dims[0] = D; dims[1] = heads; dims[2] = static_cast<uint64_t>(tokens);
    strides[0] = static_cast<uint64_t>(D) * 2;
    strides[1] = static_cast<uint64_t>(heads) * D * 2;
    box[0] = 64; box[1] = 1; box[2] = 64;
  }
  return make_tmap_3d(m, base, t, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// 4D TMA map of a strided view of a heads-outer activation: dims {D, T, H, B}, head
// (b, h) at token b*pair + h*seg of the buffer (strides in tokens).
int make_view_map(CUtensorMap* m, const void* base, int dt, const ptof_gdn_params& p, int D,
                  long long pair, long long seg) {
  const CUtensorMapDataType t =
      dt == PTOF_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(p.T),
                            static_cast<uint64_t>(p.H), static_cast<uint64_t>(p.B)};
  const uint64_t strides[3] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(seg) * D * 2,
                               static_cast<uint64_t>(pair) * D * 2};
  const uint32_t box[4] = {64, 64, 1, 1};
  return make_tmap_4d(m, base, t, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int DK, int DV, bool F16, typename TO>
int launch_t(Workspace* w, const void* q, const void* k, const void* v, const void* beta,
             const float* g, const float* S0, void* o, float* S_final, const int* cu_seqlens,
             cudaStream_t stream) {
  using L = tcfwd::Layout<DK, DV>;
  const ptof_gdn_params& p = w->p;
  // variable-length / grouped-query workspaces: ex[0] = 1, ex[1] = q/k heads,
  // ex[2] = packed tokens (p.B sequences of at most p.T tokens, token-major)
  const bool varlen = (w->ex[0] == 1);
  const int Hg = varlen ? w->ex[1] : p.H;
  const int64_t tokens = varlen ? w->ex[2] : static_cast<int64_t>(p.B) * p.T;
  tcfwd::Params P;
  const long long* vw = w->view;
  P.view = (vw[0] != 0) ? 1 : 0;
  int rc;
  if (P.view) {
    // strided view: head (b, h) starts at token b*pair + h*seg of its buffer
    rc = make_view_map(&P.mapK, k, p.in_dtype, p, DK, vw[0], vw[1]);
    if (!rc) rc = make_view_map(&P.mapQ, q, p.in_dtype, p, DK, vw[0], vw[1]);
    if (!rc) rc = make_view_map(&P.mapV, v, p.in_dtype, p, DV, vw[2], vw[3]);
  } else {
    rc = make_act_map(&P.mapK, k, p.in_dtype, p, DK, Hg, tokens);
    if (!rc) rc = make_act_map(&P.mapQ, q, p.in_dtype, p, DK, Hg, tokens);
    if (!rc) rc = make_act_map(&P.mapV, v, p.in_dtype, p, DV, p.H, tokens);
  }
  if (rc) return rc;
  // per-chunk coefficient records, then the fused forward (same stream)
  if (!w->d_scratch || w->scratch_bytes < gdn_fwd_tc_scratch_bytes(p))
    return fail(PTOF_EINVAL, "gdn_fwd workspace has no coefficient buffer");
  {
    tcfwd::CoefParams C;
    C.g = (p.gate_mode == PTOF_GATE_NONE) ? nullptr : g;
    C.beta = beta;
    C.out = static_cast<unsigned char*>(w->d_scratch);
    C.B = p.B; C.H = p.H; C.nc = (p.T + kChunk - 1) / kChunk;
    C.gate_mode = p.gate_mode;
    C.beta_dtype = p.beta_dtype;
    C.allow_fast = F16 ? 0 : 1;
    const Strides3 sg = make_strides3(p.layout, p.H, p.T);
    C.gs_b = sg.b; C.gs_h = sg.h; C.gs_t = sg.t;
    if (P.view) {
      C.gs_b = vw[0]; C.gs_h = vw[1]; C.gs_t = 1;
    }
    C.cu_seqlens = varlen ? cu_seqlens : nullptr;
    C.T = p.T;
    const int64_t chunks = static_cast<int64_t>(p.B) * p.H * C.nc;
    tcfwd::gdn_coef_kernel<<<static_cast<unsigned>((chunks + 7) / 8), 256, 0, stream>>>(C);
  }
  P.coef = static_cast<const unsigned char*>(w->d_scratch);
  P.S0 = S0;
  P.o = o;
  P.S_final = S_final;
  P.status = w->d_status;
  P.trace = static_cast<unsigned long long*>(w->trace);
  P.trace_chunks = w->trace_chunks;
  P.B = p.B; P.H = p.H; P.T = p.T; P.nc = p.T / kChunk;
  P.layout = p.layout;
  const Strides4 so = make_strides4(p.layout, p.H, p.T, DV);
  P.os_b = so.b; P.os_h = so.h; P.os_t = so.t;
  if (P.view) {
    P.os_b = vw[4] * DV; P.os_h = vw[5] * DV; P.os_t = DV;
  }
  P.cu_seqlens = varlen ? cu_seqlens : nullptr;
  P.mnc = (p.T + kChunk - 1) / kChunk;
  P.gqa = p.H / Hg;
  P.scale = p.scale;
  P.wait_ns = w->wait_ns;
  P.inject_stall = w->inject_stall;
  auto kern = varlen    ? tcfwd::gdn_fwd_tc_kernel<DK, DV, F16, TO, false, true>
              : P.trace ? tcfwd::gdn_fwd_tc_kernel<DK, DV, F16, TO, true, false>
                        : tcfwd::gdn_fwd_tc_kernel<DK, DV, F16, TO, false, false>;
  cudaError_t e = set_smem_once(kern, L::BYTES);
  if (e != cudaSuccess) return cuda_fail(e, "gdn_fwd_tc smem attribute");
  kern<<<p.B * p.H, tcfwd::Roles<DK>::THREADS, L::BYTES, stream>>>(P);
  e = cudaGetLastError();
  return e == cudaSuccess ? PTOF_OK : cuda_fail(e, "gdn_fwd_tc launch");
}

template <int DK, int DV, bool F16>
int launch_o(Workspace* w, const void* q, const void* k, const void* v, const void* beta,
             const float* g, const float* S0, void* o, float* S_final, const int* cu,
             cudaStream_t st) {
  switch (w->p.out_dtype) {
    case PTOF_F32: return launch_t<DK, DV, F16, float>(w, q, k, v, beta, g, S0, o, S_final, cu, st);
    case PTOF_F16: return launch_t<DK, DV, F16, __half>(w, q, k, v, beta, g, S0, o, S_final, cu, st);
    default: return launch_t<DK, DV, F16, __nv_bfloat16>(w, q, k, v, beta, g, S0, o, S_final, cu, st);
  }
}

template <int DK, int DV>
int launch_d(Workspace* w, const void* q, const void* k, const void* v, const void* beta,
             const float* g, const float* S0, void* o, float* S_final, const int* cu,
             cudaStream_t st) {
  if (w->p.in_dtype == PTOF_F16) return launch_o<DK, DV, true>(w, q, k, v, beta, g, S0, o, S_final, cu, st);
  return launch_o<DK, DV, false>(w, q, k, v, beta, g, S0, o, S_final, cu, st);
}

// KDA forward (DK = DV = 64, bf16 q/k/v, heads-outer): the operand pre-pass, then the
// fused kernel's ungated chain on K e^g, Q e^g, K e^-g with the per-dimension decay
// applied to the state after every chunk.
struct KdaScratch {
  size_t coef, egl, ops, total;   // byte offsets of the parts and the total
};
KdaScratch kda_scratch_layout(const ptof_gdn_params& p) {
  auto up = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
  const size_t nc = p.T / kChunk, pairs = static_cast<size_t>(p.B) * p.H;
  KdaScratch s;
  s.coef = 0;
  s.egl = up(pairs * nc * tcfwd::coef::BYTES);
  s.ops = s.egl + up(pairs * (nc + 1) * 64 * sizeof(float));
  const size_t one = up(pairs * p.T * 64 * 2);   // one bf16 operand [B,H,T,64]
  s.total = s.ops + 3 * one;
  return s;
}

template <typename TO>
int launch_kda_t(Workspace* w, const void* q, const void* k, const void* v, const void* beta,
                 const float* g, const float* S0, void* o, float* S_final, cudaStream_t stream) {
  constexpr int D = 64;
  using L = tcfwd::Layout<D, D, true>;
  const ptof_gdn_params& p = w->p;
  const KdaScratch ks = kda_scratch_layout(p);
  if (!w->d_scratch || w->scratch_bytes < ks.total)
    return fail(PTOF_EINVAL, "kda_fwd workspace has no scratch buffer");
  unsigned char* base = static_cast<unsigned char*>(w->d_scratch);
  const int nc = p.T / kChunk;
  const size_t one = (ks.total - ks.ops) / 3;
  auto* k1 = reinterpret_cast<__nv_bfloat16*>(base + ks.ops);
  auto* q1 = reinterpret_cast<__nv_bfloat16*>(base + ks.ops + one);
  auto* k2 = reinterpret_cast<__nv_bfloat16*>(base + ks.ops + 2 * one);
  float* egl = reinterpret_cast<float*>(base + ks.egl);
  {
    tcfwd::CoefParams C;   // beta only: the gate is on the operands
    C.g = nullptr;
    C.beta = beta;
    C.out = base + ks.coef;
    C.B = p.B; C.H = p.H; C.nc = nc;
    C.gate_mode = PTOF_GATE_NONE;
    C.beta_dtype = p.beta_dtype;
    C.allow_fast = 1;
    const Strides3 sg = make_strides3(PTOF_LAYOUT_BHTD, p.H, p.T);
    C.gs_b = sg.b; C.gs_h = sg.h; C.gs_t = sg.t;
    C.cu_seqlens = nullptr;
    C.T = p.T;
    const int64_t chunks = static_cast<int64_t>(p.B) * p.H * nc;
    tcfwd::gdn_coef_kernel<<<static_cast<unsigned>((chunks + 7) / 8), 256, 0, stream>>>(C);
    tcfwd::KdaPrepParams K;
    K.q = static_cast<const __nv_bfloat16*>(q);
    K.k = static_cast<const __nv_bfloat16*>(k);
    K.g = g;
    K.q1 = q1; K.k1 = k1; K.k2 = k2;
    K.egl = egl;
    K.nc = nc; K.T = p.T;
    tcfwd::kda_prep_kernel<D><<<static_cast<unsigned>(chunks), 4 * D, 0, stream>>>(K);
  }
  const int64_t tokens = static_cast<int64_t>(p.B) * p.T;
  tcfwd::Params P;
  int rc = make_act_map(&P.mapK, k1, PTOF_BF16, p, D, p.H, tokens);
  if (!rc) rc = make_act_map(&P.mapQ, q1, PTOF_BF16, p, D, p.H, tokens);
  if (!rc) rc = make_act_map(&P.mapK2, k2, PTOF_BF16, p, D, p.H, tokens);
  if (!rc) rc = make_act_map(&P.mapV, v, PTOF_BF16, p, D, p.H, tokens);
  if (rc) return rc;
  P.egl = egl;
  P.coef = base + ks.coef;
  P.S0 = S0;
  P.o = o;
  P.S_final = S_final;
  P.status = w->d_status;
  P.trace = nullptr;
  P.trace_chunks = 0;
  P.B = p.B; P.H = p.H; P.T = p.T; P.nc = nc;
  P.layout = PTOF_LAYOUT_BHTD;
  const Strides4 so = make_strides4(PTOF_LAYOUT_BHTD, p.H, p.T, D);
  P.os_b = so.b; P.os_h = so.h; P.os_t = so.t;
  P.cu_seqlens = nullptr;
  P.mnc = nc;
  P.gqa = 1;
  P.scale = p.scale;
  P.wait_ns = w->wait_ns;
  P.inject_stall = 0;
  P.view = 0;
  auto kern = tcfwd::gdn_fwd_tc_kernel<D, D, false, TO, false, false, true>;
  cudaError_t e = set_smem_once(kern, L::BYTES);
  if (e != cudaSuccess) return cuda_fail(e, "kda_fwd smem attribute");
  kern<<<p.B * p.H, tcfwd::Roles<D>::THREADS, L::BYTES, stream>>>(P);
  e = cudaGetLastError();
  return e == cudaSuccess ? PTOF_OK : cuda_fail(e, "kda_fwd launch");
}

}  // namespace

size_t gdn_fwd_tc_scratch_bytes(const ptof_gdn_params& p) {
  return static_cast<size_t>(p.B) * p.H * ((p.T + kChunk - 1) / kChunk) * tcfwd::coef::BYTES;
}

bool gdn_fwd_tc_supports(const ptof_gdn_params& p) {
  if (p.in_dtype != PTOF_F16 && p.in_dtype != PTOF_BF16) return false;
  if (p.C != kChunk) return false;
  return (p.Dk == 128 && p.Dv == 128) || (p.Dk == 64 && p.Dv == 64);
}

int launch_gdn_fwd_tc(Workspace* w, const void* q, const void* k, const void* v, const void* beta,
                      const float* g, const float* S0, void* o, float* S_final, const int* cu,
                      cudaStream_t stream) {
  const ptof_gdn_params& p = w->p;
  if (p.Dk == 128) return launch_d<128, 128>(w, q, k, v, beta, g, S0, o, S_final, cu, stream);
  return launch_d<64, 64>(w, q, k, v, beta, g, S0, o, S_final, cu, stream);
}

// ----------------------------------------------- allocation-free entry point ----
// For callers that cannot allocate device memory: code running where cudaMalloc is
// off limits (inside a host allocator or an arena that owns all device memory, or
// between the set-up and replay of a fixed memory plan) cannot create a workspace.
// ptof_gdn_fwd_exec_noalloc runs the same tensor-core forward with its coefficient
// records in this file-scope array instead of a workspace buffer, and its bounded
// waits report to a file-scope status word (ptof_gdn_fwd_noalloc_status). The array's
// size is fixed: every GPU that loads the library reserves it until the process exits.
namespace {
constexpr int64_t kNoAllocMaxChunks = 4096;   // B * H * T / 64, i.e. 262,144 head-tokens
static __device__ __align__(256) unsigned char
    g_noalloc_coef[kNoAllocMaxChunks * tcfwd::coef::BYTES];   // 7.4 MB
static __device__ int g_noalloc_status;
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};
void* g_noalloc_status_ptr[kMaxDevices] = {};

// The device addresses of the array and the status word on the current device, looked
// up once per device with that device current (in host code the symbols themselves are
// only host-side stand-ins). Returns PTOF_OK or an error.
int noalloc_symbols(int* dev_out, void** coef, int** status) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(PTOF_EUNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* c = nullptr;
    void* st = nullptr;
    e = cudaGetSymbolAddress(&c, g_noalloc_coef);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&st, g_noalloc_status);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(allocation-free arrays)");
    g_noalloc_status_ptr[dev] = st;
    g_noalloc_ptr[dev] = c;
  }
  *dev_out = dev;
  *coef = g_noalloc_ptr[dev];
  *status = static_cast<int*>(g_noalloc_status_ptr[dev]);
  return PTOF_OK;
}
}  // namespace

}  // namespace ptof

extern "C" int ptof_gdn_fwd_exec_noalloc(const ptof_gdn_params* p, const void* q, const void* k,
                                         const void* v, const void* beta, const float* g,
                                         const float* S0, void* o, float* S_final, void* stream) {
  using namespace ptof;
  if (!p) return fail(PTOF_EINVAL, "null params");
  int rc = validate_gdn(*p);
  if (rc) return rc;
  if (p->in_dtype == PTOF_F32 || !gdn_fwd_tc_supports(*p))
    return fail(PTOF_EUNSUPPORTED,
                "ptof_gdn_fwd_exec_noalloc covers the f16/bf16 tensor-core forward only "
                "(C = 64, Dk = Dv = 64 or 128)");
  const int64_t chunks = static_cast<int64_t>(p->B) * p->H * (p->T / kChunk);
  if (chunks > kNoAllocMaxChunks)
    return fail(PTOF_EINVAL,
                "ptof_gdn_fwd_exec_noalloc: B*H*T/64 = %lld chunks exceeds its fixed maximum of "
                "%lld (use ptof_gdn_fwd_setup / ptof_gdn_fwd_exec)",
                static_cast<long long>(chunks), static_cast<long long>(kNoAllocMaxChunks));
  rc = check_ptrs({q, k, v, beta, o}, {S0, S_final});
  if (rc) return rc;
  if (p->gate_mode != PTOF_GATE_NONE && !g) return fail(PTOF_EINVAL, "g is NULL for a gated forward");
  int dev = -1;
  void* base = nullptr;
  int* status = nullptr;
  rc = noalloc_symbols(&dev, &base, &status);
  if (rc) return rc;
  // A workspace on the stack pointing at the file-scope array and status word, no
  // trace. The coefficient pre-pass rewrites every record the forward reads, so
  // nothing in the array has to start at zero.
  Workspace w;
  w.kind = kWsGdnFwd;
  w.device = dev;
  w.p = *p;
  w.d_status = status;
  w.d_scratch = base;
  w.scratch_bytes = static_cast<size_t>(kNoAllocMaxChunks) * tcfwd::coef::BYTES;
  return launch_gdn_fwd_tc(&w, q, k, v, beta, g, S0, o, S_final, nullptr,
                           static_cast<cudaStream_t>(stream));
}

extern "C" int ptof_gdn_fwd_noalloc_status(void* stream) {
  using namespace ptof;
  int dev = -1;
  void* base = nullptr;
  int* status = nullptr;
  int rc = noalloc_symbols(&dev, &base, &status);
  if (rc) return rc;
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "stream synchronize");
  int h = 0;
  e = cudaMemcpy(&h, status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "status read");
  if (h != 0) {
    e = cudaMemset(status, 0, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "status clear");
    return fail(PTOF_ETIMEOUT, "allocation-free forward: device wait gave up at site %d", h);
  }
  return PTOF_OK;
}

// ----------------------------------------------------------------- KDA C ABI ----
extern "C" void* ptof_kda_fwd_setup(const ptof_gdn_params* p) {
  using namespace ptof;
  if (!p) {
    fail(PTOF_EINVAL, "null params");
    return nullptr;
  }
  if (validate_gdn(*p) != PTOF_OK) return nullptr;
  if (p->Dk != 64 || p->Dv != 64 || p->in_dtype != PTOF_BF16 || p->layout != PTOF_LAYOUT_BHTD) {
    fail(PTOF_EUNSUPPORTED, "kda_fwd: Dk = Dv = 64, bf16 q/k/v, heads-outer layout only "
         "(got Dk=%d Dv=%d in_dtype=%d layout=%d)", p->Dk, p->Dv, p->in_dtype, p->layout);
    return nullptr;
  }
  Workspace* w = ws_create(kWsKdaFwd, p);
  if (!w) return nullptr;
  w->scratch_bytes = kda_scratch_layout(*p).total;
  const cudaError_t e = cudaMalloc(&w->d_scratch, w->scratch_bytes);
  if (e != cudaSuccess) {
    cuda_fail(e, "kda_fwd scratch buffer");
    ws_destroy(w);
    return nullptr;
  }
  return w;
}

extern "C" int ptof_kda_fwd_exec(void* wsv, const void* q, const void* k, const void* v,
                                 const void* beta, const float* g, const float* S0, void* o,
                                 float* S_final, void* stream) {
  using namespace ptof;
  Workspace* w = static_cast<Workspace*>(wsv);
  if (!w || w->kind != kWsKdaFwd) return fail(PTOF_EINVAL, "not a kda_fwd workspace");
  int rc = check_ptrs({q, k, v, beta, g, o}, {S0, S_final});
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (w->p.out_dtype) {
    case PTOF_F32: return launch_kda_t<float>(w, q, k, v, beta, g, S0, o, S_final, st);
    case PTOF_F16: return launch_kda_t<__half>(w, q, k, v, beta, g, S0, o, S_final, st);
    default: return launch_kda_t<__nv_bfloat16>(w, q, k, v, beta, g, S0, o, S_final, st);
  }
}
