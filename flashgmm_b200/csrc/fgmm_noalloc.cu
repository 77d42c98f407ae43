// fgmm_em_fused_static: one fused EM iteration that allocates no device memory.
//
// Some callers cannot call cudaMalloc at all -- code that runs inside another
// framework's allocator or memory pool (allocating behind its back breaks its
// accounting or is forbidden), or a process that must keep a fixed memory footprint
// after start-up.  For them this entry point takes its scratch from a file-scope
// device array of fixed size instead of a caller-provided workspace.  It runs the
// generic fp32 CUDA-core kernels (fgmm_simt.cu) followed by the M-step update.
//
// The array is part of this library's device image: every GPU that loads the library
// holds FGMM_STATIC_SCRATCH_BYTES of it until the process exits.  All calls share it
// and it keeps the last call's contents; nothing in it needs to start at zero (every
// value a call reads was written earlier in the same call).  Calls whose work overlaps
// on the GPU (different streams, or different host threads) race on it.
#include <mutex>
#include "fgmm_common.cuh"

namespace fgmm {
namespace {

static __device__ __align__(256) unsigned char g_static_scratch[FGMM_STATIC_SCRATCH_BYTES];

// Device address of g_static_scratch per device.  In host code the array's name is
// only a host-side stand-in, so the address is looked up with cudaGetSymbolAddress on
// the first call made with each device current.
constexpr int kMaxDevices = 64;
void *g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

int scratch_for_current_device(void **out) {
  int dev = 0;
  FGMM_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(FGMM_ERR_INVALID, "device index out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return FGMM_OK;
}

}  // namespace
}  // namespace fgmm

using namespace fgmm;

extern "C" int fgmm_em_fused_static(const float *X, int64_t N, int32_t d, const float *mu,
                                    const float *var, const float *log_pi, int32_t K,
                                    float *new_mu, float *new_var, float *new_log_pi,
                                    float *log_normalizer, void *stream) {
  if (N < 1 || K < 1 || d < 1)
    return fail(FGMM_ERR_INVALID, "N, K and d must all be >= 1");
  if (d > 256) return fail(FGMM_ERR_UNSUPPORTED, "d > 256 is not supported");
  if (!X || !mu || !var || !log_pi || !new_mu || !new_var || !new_log_pi || !log_normalizer)
    return fail(FGMM_ERR_INVALID, "null pointer argument");
  const size_t ws = align_up(simt_workspace_bytes(N, d, K), 256);
  const size_t stats = (size_t)((int64_t)K * (2 * (int64_t)d + 1) + 1) * sizeof(double);
  if (ws + stats > (size_t)FGMM_STATIC_SCRATCH_BYTES)
    return fail(FGMM_ERR_WORKSPACE,
                "fgmm_em_fused_static: this shape needs " + std::to_string(ws + stats) +
                    " bytes of scratch, more than the fixed " +
                    std::to_string((size_t)FGMM_STATIC_SCRATCH_BYTES) +
                    " bytes; use fgmm_em_fused with a caller-provided workspace");
  void *scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  double *stats_ptr = reinterpret_cast<double *>(static_cast<char *>(scratch) + ws);
  const UpdateOut up{(double)N, new_mu, new_var, new_log_pi, true};
  return simt_em_stats(X, N, d, mu, var, log_pi, K, stats_ptr, log_normalizer, scratch, st, &up);
}
