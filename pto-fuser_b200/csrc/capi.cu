// C ABI of the GDN kernel library: argument validation, library-owned
// workspaces, TMA descriptor encoding and kernel selection. No function here
// synchronises the caller's stream except ptof_check_status.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "capi_internal.h"
#include "common.cuh"

namespace ptof {

// ---------------------------------------------------------------- errors ----
static thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(PTOF_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

// ------------------------------------------------------ TMA descriptors ----
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes,
                 uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(PTOF_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return fail(PTOF_EALIGN, "TMA base address not 16-byte aligned");
  if (row_stride_bytes % 16 != 0)
    return fail(PTOF_EALIGN, "TMA row stride %llu not a multiple of 16 bytes",
                (unsigned long long)row_stride_bytes);
  (void)elem_bytes;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PTOF_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return PTOF_OK;
}

int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(PTOF_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return fail(PTOF_EALIGN, "TMA base address not 16-byte aligned");
  for (int i = 0; i < 2; ++i)
    if (strides_bytes[i] % 16 != 0)
      return fail(PTOF_EALIGN, "TMA stride %llu not a multiple of 16 bytes",
                  (unsigned long long)strides_bytes[i]);
  cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t s[2] = {strides_bytes[0], strides_bytes[1]};
  cuuint32_t b[3] = {box[0], box[1], box[2]};
  cuuint32_t e[3] = {1, 1, 1};
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PTOF_ECUDA, "cuTensorMapEncodeTiled(3d) failed (%d)", (int)r);
  return PTOF_OK;
}

int make_tmap_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(PTOF_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return fail(PTOF_EALIGN, "TMA base address not 16-byte aligned");
  for (int i = 0; i < 3; ++i)
    if (strides_bytes[i] % 16 != 0 || strides_bytes[i] == 0)
      return fail(PTOF_EALIGN, "TMA stride %llu not a positive multiple of 16 bytes",
                  (unsigned long long)strides_bytes[i]);
  cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t s[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  cuuint32_t b[4] = {box[0], box[1], box[2], box[3]};
  cuuint32_t e[4] = {1, 1, 1, 1};
  CUresult r = fn(map, dt, 4, const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PTOF_ECUDA, "cuTensorMapEncodeTiled(4d) failed (%d)", (int)r);
  return PTOF_OK;
}

cudaError_t set_smem_attr_once(const void* kern, int bytes) {
  static std::mutex mu;
  static std::unordered_map<const void*, int> done;
  std::lock_guard<std::mutex> lock(mu);
  auto it = done.find(kern);
  if (it != done.end() && it->second >= bytes) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done[kern] = bytes;
  return e;
}

// ------------------------------------------------------------ workspace ----
Workspace* ws_create(int kind, const ptof_gdn_params* p) {
  Workspace* w = new Workspace();
  w->kind = kind;
  if (p) w->p = *p;
  if (cudaGetDevice(&w->device) != cudaSuccess) {
    fail(PTOF_ECUDA, "cudaGetDevice failed");
    delete w;
    return nullptr;
  }
  cudaError_t e = cudaMalloc(&w->d_status, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(w->d_status, 0, sizeof(int));
  if (e != cudaSuccess) {
    cuda_fail(e, "workspace allocation");
    delete w;
    return nullptr;
  }
  return w;
}

void ws_destroy(Workspace* w) {
  if (!w) return;
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != w->device) cudaSetDevice(w->device);
  if (w->d_status) cudaFree(w->d_status);
  if (w->d_scratch) cudaFree(w->d_scratch);
  if (cur >= 0 && cur != w->device) cudaSetDevice(cur);
  delete w;
}

static bool dtype_ok(int d) { return d == PTOF_F32 || d == PTOF_F16 || d == PTOF_BF16; }
static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int validate_gdn(const ptof_gdn_params& p) {
  if (p.B < 1 || p.H < 1 || p.T < 1) return fail(PTOF_EINVAL, "B, H, T must be >= 1");
  if (p.C != kChunk) return fail(PTOF_EUNSUPPORTED, "chunk length C=%d (only 64)", p.C);
  if (p.T % p.C != 0) return fail(PTOF_EINVAL, "T=%d is not a multiple of C=%d", p.T, p.C);
  if (p.Dk < 1 || p.Dv < 1) return fail(PTOF_EINVAL, "Dk, Dv must be >= 1");
  if (!dtype_ok(p.in_dtype) || !dtype_ok(p.beta_dtype) || !dtype_ok(p.out_dtype))
    return fail(PTOF_EINVAL, "bad dtype code");
  if (p.gate_mode < PTOF_GATE_RAW || p.gate_mode > PTOF_GATE_NONE)
    return fail(PTOF_EINVAL, "bad gate_mode %d", p.gate_mode);
  if (p.layout != PTOF_LAYOUT_BHTD && p.layout != PTOF_LAYOUT_BTHD)
    return fail(PTOF_EINVAL, "bad layout %d", p.layout);
  return PTOF_OK;
}

int check_ptrs(std::initializer_list<const void*> required,
               std::initializer_list<const void*> optional) {
  int i = 0;
  for (const void* q : required) {
    if (!q) return fail(PTOF_EINVAL, "required pointer #%d is NULL", i);
    if (!aligned16(q)) return fail(PTOF_EALIGN, "pointer #%d not 16-byte aligned", i);
    ++i;
  }
  for (const void* q : optional) {
    if (q && !aligned16(q)) return fail(PTOF_EALIGN, "optional pointer not 16-byte aligned");
  }
  return PTOF_OK;
}

}  // namespace ptof

using namespace ptof;

extern "C" {

const char* ptof_last_error(void) { return g_err; }

// ------------------------------------------------------------ gdn forward ----
void* ptof_gdn_fwd_setup(const ptof_gdn_params* p) {
  if (!p) {
    fail(PTOF_EINVAL, "null params");
    return nullptr;
  }
  if (validate_gdn(*p) != PTOF_OK) return nullptr;
  Workspace* w = ws_create(kWsGdnFwd, p);
  if (!w) return nullptr;
  // tensor-core path: per-chunk coefficient records; fp32 path: the two-phase
  // kernels' per-chunk records when they apply (else nothing)
  const bool tc = p->in_dtype != PTOF_F32 && gdn_fwd_tc_supports(*p);
  w->scratch_bytes = tc ? gdn_fwd_tc_scratch_bytes(*p) : gdn_fwd_simt_split_bytes(*p);
  if (w->scratch_bytes) {
    const cudaError_t e = cudaMalloc(&w->d_scratch, w->scratch_bytes);
    if (e != cudaSuccess) {
      cuda_fail(e, "gdn_fwd workspace buffer");
      ws_destroy(w);
      return nullptr;
    }
  }
  return w;
}

int ptof_gdn_fwd_exec(void* wsv, const void* q, const void* k, const void* v, const void* beta,
                      const float* g, const float* S0, void* o, float* S_final, void* stream) {
  Workspace* w = static_cast<Workspace*>(wsv);
  if (!w || w->kind != kWsGdnFwd) return fail(PTOF_EINVAL, "not a gdn_fwd workspace");
  const ptof_gdn_params& p = w->p;
  int rc = check_ptrs({q, k, v, beta, o}, {S0, S_final});
  if (rc) return rc;
  if (p.gate_mode != PTOF_GATE_NONE && !g) return fail(PTOF_EINVAL, "g is NULL for a gated forward");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (p.in_dtype == PTOF_F32 || !gdn_fwd_tc_supports(p)) {
    if (!gdn_fwd_simt_supports(p))
      return fail(PTOF_EUNSUPPORTED, "no kernel for Dk=%d Dv=%d", p.Dk, p.Dv);
    const size_t split = gdn_fwd_simt_split_bytes(p);
    if (split && w->d_scratch && w->scratch_bytes >= split)
      e = launch_gdn_fwd_simt_split(p, q, k, v, beta, g, S0, o, S_final, w->d_scratch, st);
    else
      e = launch_gdn_fwd_simt(p, q, k, v, beta, g, S0, o, S_final, st);
    if (e != cudaSuccess) return cuda_fail(e, "gdn_fwd_simt launch");
    return PTOF_OK;
  }
  return launch_gdn_fwd_tc(w, q, k, v, beta, g, S0, o, S_final, nullptr, st);
}

void* ptof_gdn_fwd_varlen_setup(const ptof_gdn_varlen_params* v) {
  if (!v) {
    fail(PTOF_EINVAL, "null params");
    return nullptr;
  }
  if (v->N < 1 || v->H < 1 || v->Hg < 1 || v->H % v->Hg || v->T_total < 0 || v->max_len < 1) {
    fail(PTOF_EINVAL, "varlen shape N=%d H=%d Hg=%d T_total=%d max_len=%d (H a multiple of Hg)",
         v->N, v->H, v->Hg, v->T_total, v->max_len);
    return nullptr;
  }
  ptof_gdn_params p{};
  p.B = v->N; p.H = v->H; p.T = v->max_len; p.C = kChunk; p.Dk = v->Dk; p.Dv = v->Dv;
  p.in_dtype = v->in_dtype; p.beta_dtype = v->beta_dtype; p.out_dtype = v->out_dtype;
  p.gate_mode = v->gate_mode; p.layout = PTOF_LAYOUT_BTHD; p.scale = v->scale;
  if (p.in_dtype == PTOF_F32 || !gdn_fwd_tc_supports(p)) {
    fail(PTOF_EUNSUPPORTED, "varlen forward: f16/bf16 operands, Dk = Dv = 64 or 128");
    return nullptr;
  }
  if (!dtype_ok(p.beta_dtype) || !dtype_ok(p.out_dtype) || p.gate_mode < PTOF_GATE_RAW ||
      p.gate_mode > PTOF_GATE_NONE) {
    fail(PTOF_EINVAL, "varlen dtype / gate");
    return nullptr;
  }
  Workspace* w = ws_create(kWsGdnFwd, &p);
  if (!w) return nullptr;
  w->ex[0] = 1;
  w->ex[1] = v->Hg;
  w->ex[2] = v->T_total;
  w->scratch_bytes = gdn_fwd_tc_scratch_bytes(p);
  const cudaError_t e = cudaMalloc(&w->d_scratch, w->scratch_bytes);
  if (e != cudaSuccess) {
    cuda_fail(e, "gdn_fwd coefficient buffer");
    ws_destroy(w);
    return nullptr;
  }
  return w;
}

int ptof_gdn_fwd_varlen_exec(void* wsv, const void* q, const void* k, const void* v,
                             const void* beta, const float* g, const int* cu_seqlens,
                             const float* S0, void* o, float* S_final, void* stream) {
  Workspace* w = static_cast<Workspace*>(wsv);
  if (!w || w->kind != kWsGdnFwd || w->ex[0] != 1)
    return fail(PTOF_EINVAL, "not a varlen gdn_fwd workspace");
  if (!cu_seqlens) return fail(PTOF_EINVAL, "cu_seqlens is NULL");
  int rc = check_ptrs({q, k, v, beta, o}, {S0, S_final});
  if (rc) return rc;
  if (w->p.gate_mode != PTOF_GATE_NONE && !g) return fail(PTOF_EINVAL, "g is NULL for a gated forward");
  return launch_gdn_fwd_tc(w, q, k, v, beta, g, S0, o, S_final, cu_seqlens,
                           static_cast<cudaStream_t>(stream));
}

void ptof_gdn_fwd_teardown(void* ws) { ws_destroy(static_cast<Workspace*>(ws)); }

int ptof_gdn_fwd_set_trace(void* wsv, void* dev_buf, int chunks) {
  Workspace* w = static_cast<Workspace*>(wsv);
  if (!w || w->kind != kWsGdnFwd) return fail(PTOF_EINVAL, "not a gdn_fwd workspace");
  if (chunks < 0 || (chunks > 0 && !dev_buf)) return fail(PTOF_EINVAL, "bad trace buffer");
  w->trace = chunks > 0 ? dev_buf : nullptr;
  w->trace_chunks = chunks;
  return PTOF_OK;
}

int ptof_ws_set_wait_limit(void* wsv, unsigned long long ns) {
  Workspace* w = static_cast<Workspace*>(wsv);
  if (!w || w->kind != kWsGdnFwd) return fail(PTOF_EINVAL, "not a gdn_fwd workspace");
  if (ns == 0) return fail(PTOF_EINVAL, "wait limit must be positive");
  w->wait_ns = ns;
  return PTOF_OK;
}

int ptof_gdn_fwd_set_view(void* wsv, long long qk_pair, long long qk_seg, long long v_pair,
                          long long v_seg, long long o_pair, long long o_seg) {
  Workspace* w = static_cast<Workspace*>(wsv);
  if (!w || w->kind != kWsGdnFwd) return fail(PTOF_EINVAL, "not a gdn_fwd workspace");
  const long long all[6] = {qk_pair, qk_seg, v_pair, v_seg, o_pair, o_seg};
  bool any = false;
  for (long long x : all) {
    if (x < 0) return fail(PTOF_EINVAL, "view strides must be >= 0");
    any = any || x != 0;
  }
  if (any) {
    if (w->p.layout != PTOF_LAYOUT_BHTD || w->ex[0] == 1)
      return fail(PTOF_EUNSUPPORTED, "views need the heads-outer layout (not varlen)");
    if (w->p.in_dtype == PTOF_F32 || !gdn_fwd_tc_supports(w->p))
      return fail(PTOF_EUNSUPPORTED, "views are served by the tensor-core forward only");
    for (long long x : all)
      if (x == 0) return fail(PTOF_EINVAL, "every view stride must be positive");
  }
  for (int i = 0; i < 6; ++i) w->view[i] = all[i];
  return PTOF_OK;
}

int ptof_gdn_fwd_inject_stall(void* wsv, int on) {
  Workspace* w = static_cast<Workspace*>(wsv);
  if (!w || w->kind != kWsGdnFwd) return fail(PTOF_EINVAL, "not a gdn_fwd workspace");
  w->inject_stall = on ? 1 : 0;
  return PTOF_OK;
}

int ptof_check_status(void* wsv, void* stream) {
  Workspace* w = static_cast<Workspace*>(wsv);
  if (!w) return fail(PTOF_EINVAL, "null workspace");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "stream synchronize");
  int h = 0;
  e = cudaMemcpy(&h, w->d_status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "status read");
  if (h != 0) {
    cudaMemset(w->d_status, 0, sizeof(int));
    return fail(PTOF_ETIMEOUT, "device wait gave up at site %d", h);
  }
  return PTOF_OK;
}

// ------------------------------------------------- reference-key kernels ----
void* ptof_ws_setup(void) { return ws_create(kWsGeneric, nullptr); }
void ptof_ws_teardown(void* ws) { ws_destroy(static_cast<Workspace*>(ws)); }

static bool dt16(int d) { return d == PTOF_F16 || d == PTOF_BF16 || d == PTOF_F32; }

int ptof_gated_qk_exec(void* ws, const void* a, const void* b, const float* g, const void* beta,
                       void* L, int M, int C, int D, int in_dtype, int beta_dtype, int causal,
                       void* stream) {
  (void)ws;
  if (M < 1 || C < 1 || C > 128 || D < 1 || D > 256) return fail(PTOF_EINVAL, "gated_qk shape");
  if (!dt16(in_dtype) || !dt16(beta_dtype)) return fail(PTOF_EINVAL, "gated_qk dtype");
  if (!a || !b || !g || !beta || !L) return fail(PTOF_EINVAL, "gated_qk: NULL pointer");
  return launch_gated_qk(in_dtype, beta_dtype, a, b, g, beta, L, M, C, D, causal,
                         static_cast<cudaStream_t>(stream));
}

int ptof_kkt_inv_exec(void* ws, const void* k, const void* beta, const float* g, float* T_out,
                      int B, int H, int T, int D, int in_dtype, int beta_dtype, int gate_mode,
                      int layout, void* stream) {
  Workspace* w = static_cast<Workspace*>(ws);
  if (B < 1 || H < 1 || T < kChunk || T % kChunk || (D != 64 && D != 128))
    return fail(PTOF_EINVAL, "kkt_inv shape B=%d H=%d T=%d D=%d (T a multiple of 64, D 64 or 128)",
                B, H, T, D);
  if ((in_dtype != PTOF_F16 && in_dtype != PTOF_BF16) || !dtype_ok(beta_dtype))
    return fail(PTOF_EINVAL, "kkt_inv dtype");
  if (gate_mode < PTOF_GATE_RAW || gate_mode > PTOF_GATE_NONE || (layout != PTOF_LAYOUT_BHTD &&
                                                                  layout != PTOF_LAYOUT_BTHD))
    return fail(PTOF_EINVAL, "kkt_inv gate/layout");
  int rc = check_ptrs({k, beta, T_out}, {g});
  if (rc) return rc;
  if (gate_mode != PTOF_GATE_NONE && !g) return fail(PTOF_EINVAL, "g is NULL for a gated kkt_inv");
  ptof_gdn_params p{};
  p.B = B; p.H = H; p.T = T; p.C = kChunk; p.Dk = D; p.Dv = D;
  p.in_dtype = in_dtype; p.beta_dtype = beta_dtype; p.out_dtype = PTOF_F32;
  p.gate_mode = gate_mode; p.layout = layout; p.scale = 1.f;
  return launch_kkt_inv(p, w ? w->d_status : nullptr, k, beta, g, T_out,
                        static_cast<cudaStream_t>(stream));
}

int ptof_qk_prologue_exec(void* ws, const void* q, const void* k, const void* P,
                          const void* invP, void* L, int M, int C, int D, int in_dtype,
                          void* stream) {
  (void)ws;
  if (M < 1 || C < 1 || C > 128 || D < 1 || D > 256) return fail(PTOF_EINVAL, "qk_prologue shape");
  if (!dtype_ok(in_dtype)) return fail(PTOF_EINVAL, "qk_prologue dtype");
  if (!q || !k || !P || !invP || !L) return fail(PTOF_EINVAL, "qk_prologue: NULL pointer");
  return launch_qk_prologue(in_dtype, q, k, P, invP, L, M, C, D, static_cast<cudaStream_t>(stream));
}

int ptof_qkvp_flash_exec(void* ws, const void* q, const void* k, const void* v, const void* P,
                         const void* invP, float* o, int M, int C, int D, int Dv, int in_dtype,
                         void* stream) {
  (void)ws;
  if (M < 1 || C < 1 || C > 128 || D < 1 || D > 256 || Dv < 1)
    return fail(PTOF_EINVAL, "qkvp_flash shape");
  if (!dtype_ok(in_dtype)) return fail(PTOF_EINVAL, "qkvp_flash dtype");
  if (!q || !k || !v || !P || !invP || !o) return fail(PTOF_EINVAL, "qkvp_flash: NULL pointer");
  return launch_qkvp_flash(in_dtype, q, k, v, P, invP, o, M, C, D, Dv,
                           static_cast<cudaStream_t>(stream));
}

int ptof_tri_inv_exec(void* ws, const void* A, int a_dtype, float* T, int M, int C, void* stream) {
  (void)ws;
  if (M < 1 || C < 1 || C > 128) return fail(PTOF_EINVAL, "tri_inv shape M=%d C=%d", M, C);
  if (!dt16(a_dtype)) return fail(PTOF_EINVAL, "tri_inv dtype");
  if (!A || !T) return fail(PTOF_EINVAL, "tri_inv: NULL pointer");
  return launch_tri_inv(a_dtype, A, T, M, C, static_cast<cudaStream_t>(stream));
}

int ptof_chunk_h_scan_exec(void* ws, const void* w, const void* u, const void* k,
                           const float* decay, void* h_out, void* final_state, int B, int H,
                           int nc, int C, int D, int Dv, int in_dtype, int out_dtype,
                           void* stream) {
  (void)ws;
  if (B < 1 || H < 1 || nc < 1 || C < 1 || C > 128 || D < 1 || D > 128 || Dv < 1)
    return fail(PTOF_EINVAL, "chunk_h_scan shape");
  if (!dt16(in_dtype) || !dt16(out_dtype)) return fail(PTOF_EINVAL, "chunk_h_scan dtype");
  if (!w || !u || !k || !decay || !h_out || !final_state)
    return fail(PTOF_EINVAL, "chunk_h_scan: NULL pointer");
  return launch_scan(in_dtype, out_dtype, w, u, k, decay, h_out, final_state, B, H, nc, C, D,
                     Dv, 0, static_cast<cudaStream_t>(stream));
}

int ptof_chunk_h_scan_perdim_exec(void* ws, const void* w, const void* u, const void* k,
                                  const float* decay, void* h_out, void* final_state, int B,
                                  int H, int nc, int C, int D, int Dv, int in_dtype,
                                  int out_dtype, void* stream) {
  (void)ws;
  if (B < 1 || H < 1 || nc < 1 || C < 1 || C > 128 || D < 1 || D > 128 || Dv < 1)
    return fail(PTOF_EINVAL, "chunk_h_scan shape");
  if (!dt16(in_dtype) || !dt16(out_dtype)) return fail(PTOF_EINVAL, "chunk_h_scan dtype");
  if (!w || !u || !k || !decay || !h_out || !final_state)
    return fail(PTOF_EINVAL, "chunk_h_scan: NULL pointer");
  return launch_scan(in_dtype, out_dtype, w, u, k, decay, h_out, final_state, B, H, nc, C, D,
                     Dv, 1, static_cast<cudaStream_t>(stream));
}

int ptof_qkv_flash_exec(void* ws, const void* q, const void* k, const void* v, const float* g,
                        float* o, int M, int C, int D, int Dv, int in_dtype, void* stream) {
  (void)ws;
  if (M < 1 || C < 1 || C > 128 || D < 1 || D > 256 || Dv < 1 || Dv > 256)
    return fail(PTOF_EINVAL, "qkv_flash shape");
  if (!dt16(in_dtype)) return fail(PTOF_EINVAL, "qkv_flash dtype");
  if (!q || !k || !v || !g || !o) return fail(PTOF_EINVAL, "qkv_flash: NULL pointer");
  return launch_qkv_flash(in_dtype, q, k, v, g, o, M, C, D, Dv, static_cast<cudaStream_t>(stream));
}

// --------------------------------------------------------------- selftests ----
int ptof_selftest_umma(const float* A, const float* B, float* D, int M, int N, int K, int mode,
                       int* status, void* stream) {
  if (!(M == 64 || M == 128) || N < 16 || N > 256 || N % 16 || K < 32 || K > 128 || K % 32)
    return fail(PTOF_EINVAL, "selftest shape M=%d N=%d K=%d", M, N, K);
  if ((mode & 4) && M != 128) return fail(PTOF_EINVAL, "TMEM A operand needs M=128");
  if ((mode & 1) && M % 64) return fail(PTOF_EINVAL, "MN-major A needs M%%64==0");
  if ((mode & 2) && N % 64) return fail(PTOF_EINVAL, "MN-major B needs N%%64==0");
  cudaError_t e = launch_selftest_umma(A, B, D, M, N, K, mode, status,
                                       static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? PTOF_OK : cuda_fail(e, "selftest_umma launch");
}

int ptof_selftest_umma_rate(int N, int n, int issuers, int a_tmem, long long* out, int* status,
                            void* stream) {
  if (N < 16 || N > 256 || N % 16 || n < 8 || n % 8 || issuers < 1 || issuers > 4 ||
      issuers * N > 448 || a_tmem < 0 || a_tmem > 15 || !out)
    return fail(PTOF_EINVAL, "selftest_umma_rate N=%d n=%d issuers=%d", N, n, issuers);
  cudaError_t e = launch_selftest_umma_rate(N, n, issuers, a_tmem, out, status,
                                            static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? PTOF_OK : cuda_fail(e, "selftest_umma_rate launch");
}

int ptof_selftest_tma(const void* src, int rows, int cols, int x0, int y0, void* out, int* status,
                      void* stream) {
  CUtensorMap map;
  int rc = make_tmap_2d(&map, src, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, cols, rows,
                        static_cast<uint64_t>(cols) * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  cudaError_t e = launch_selftest_tma(map, x0, y0, out, status, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? PTOF_OK : cuda_fail(e, "selftest_tma launch");
}

}  // extern "C"
