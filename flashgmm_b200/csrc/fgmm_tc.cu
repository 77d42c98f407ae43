// tcgen05 tensor-core family (placeholder until the kernels land).
#include "fgmm_common.cuh"
namespace fgmm {
int tc_launches(int64_t, int, int) { return 0; }
bool tc_supported(int64_t, int, int) { return false; }
size_t tc_points_bytes(int64_t, int) { return 0; }
size_t tc_workspace_bytes(int64_t, int, int) { return 0; }
int tc_prepare_points(const float *, int64_t, int, void *, cudaStream_t) {
  return fail(FGMM_ERR_UNSUPPORTED, "tcgen05 family not built");
}
int tc_em_stats(const float *, const void *, int64_t, int, const float *, const float *,
                const float *, int, double *, float *, void *, cudaStream_t) {
  return fail(FGMM_ERR_UNSUPPORTED, "tcgen05 family not built");
}
}  // namespace fgmm
