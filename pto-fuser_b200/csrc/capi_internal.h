// Internal declarations shared by the C-ABI implementation and the kernel files.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <initializer_list>

#include "../../include/pto_fuser_gdn.h"

namespace ptof {

// Raise a kernel's dynamic shared-memory limit once per kernel (keyed by its
// address). The first launch of every kernel happens outside stream capture (warm-up),
// so no attribute call is ever recorded into a graph.
cudaError_t set_smem_attr_once(const void* kern, int bytes);
template <typename K>
inline cudaError_t set_smem_once(K kern, int bytes) {
  return set_smem_attr_once(reinterpret_cast<const void*>(kern), bytes);
}

enum WsKind { kWsGdnFwd = 1, kWsGeneric = 2, kWsKdaFwd = 3 };

// Library-owned per-setup state.
struct Workspace {
  int kind = 0;
  int device = 0;
  ptof_gdn_params p{};
  int* d_status = nullptr;       // device status word written by bounded waits
  void* d_scratch = nullptr;     // optional kernel scratch, owned here
  size_t scratch_bytes = 0;
  int ex[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // per-kind extra integers
  void* trace = nullptr;         // caller-owned device buffer of stage timestamps
  int trace_chunks = 0;
  unsigned long long wait_ns = 2000000000ull;  // limit of every bounded device wait
  int inject_stall = 0;          // test only: make one device wait run out
  // strided view (tokens): head (b, h) of q/k/beta/g starts at token b*view[0] + h*view[1]
  // of its buffer, of v at b*view[2] + h*view[3], of o at b*view[4] + h*view[5]; all 0 =
  // the contiguous [B,H,T,D] layout
  long long view[6] = {0, 0, 0, 0, 0, 0};
};

int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes,
                 uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle swz);
int make_tmap_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz);
int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz);
Workspace* ws_create(int kind, const ptof_gdn_params* p);
void ws_destroy(Workspace* w);
int validate_gdn(const ptof_gdn_params& p);
int check_ptrs(std::initializer_list<const void*> required,
               std::initializer_list<const void*> optional);

// kernels
cudaError_t launch_gdn_fwd_simt(const ptof_gdn_params& p, const void* q, const void* k,
                                const void* v, const void* beta, const float* g,
                                const float* S0, void* o, float* S_final, cudaStream_t stream);
bool gdn_fwd_simt_supports(const ptof_gdn_params& p);
// Two-phase fp32 path (gdn_simt_split.cu): its per-chunk record bytes for these
// params, 0 when it does not apply (then the single-kernel path runs).
size_t gdn_fwd_simt_split_bytes(const ptof_gdn_params& p);
cudaError_t launch_gdn_fwd_simt_split(const ptof_gdn_params& p, const void* q, const void* k,
                                      const void* v, const void* beta, const float* g,
                                      const float* S0, void* o, float* S_final, void* scratch,
                                      cudaStream_t stream);
bool gdn_fwd_tc_supports(const ptof_gdn_params& p);
// bytes of the per-chunk coefficient records the tensor-core forward keeps in the
// workspace (allocated by ptof_gdn_fwd_setup)
size_t gdn_fwd_tc_scratch_bytes(const ptof_gdn_params& p);
// cu_seqlens: device int32 [p.B + 1] for variable-length workspaces (ex[0] = 1), else null
int launch_gdn_fwd_tc(Workspace* w, const void* q, const void* k, const void* v,
                      const void* beta, const float* g, const float* S0, void* o,
                      float* S_final, const int* cu_seqlens, cudaStream_t stream);

int launch_kkt_inv(const ptof_gdn_params& p, int* status, const void* k, const void* beta,
                   const float* g, float* Tout, cudaStream_t st);
int launch_gated_qk(int in_dtype, int beta_dtype, const void* a, const void* b, const float* g,
                    const void* beta, void* L, int M, int C, int D, int causal, cudaStream_t st);
int launch_qkvp_flash(int in_dtype, const void* q, const void* k, const void* v, const void* P,
                      const void* invP, float* o, int M, int C, int D, int Dv, cudaStream_t st);
int launch_qk_prologue(int in_dtype, const void* q, const void* k, const void* P,
                       const void* invP, void* L, int M, int C, int D, cudaStream_t st);
int launch_tri_inv(int a_dtype, const void* A, float* T, int M, int C, cudaStream_t st);
int launch_scan(int in_dtype, int out_dtype, const void* w, const void* u, const void* k,
                const float* decay, void* h_out, void* final_state, int B, int H, int nc, int C,
                int D, int Dv, int perdim, cudaStream_t st);
int launch_qkv_flash(int in_dtype, const void* q, const void* k, const void* v, const float* g,
                     float* o, int M, int C, int D, int Dv, cudaStream_t st);

cudaError_t launch_selftest_umma(const float* A, const float* B, float* D, int M, int N, int K,
                                 int mode, int* status, cudaStream_t stream);
cudaError_t launch_selftest_umma_rate(int N, int n, int issuers, int a_tmem, long long* out,
                                      int* status, cudaStream_t stream);
cudaError_t launch_selftest_tma(const CUtensorMap& map, int x0, int y0, void* out, int* status,
                                cudaStream_t stream);

}  // namespace ptof
