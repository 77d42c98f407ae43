// Reduction of per-block partial statistics and the M-step update.
//
// The M-step follows the reference's update (flash_gmm/csrc/flash_gmm_cuda.cu:298-322
// update_params_kernel, floors as in flash_gmm/csrc/flash_gmm_cpu.cpp:270-284):
//   mu = s * (1 / max(n, 1e-8)),  var = max(sq/n - mu^2, 1e-6),  log_pi = log(max(n/N, 1e-8))
// but is evaluated in fp64 from fp64 statistics and rounded once to fp32.
#include "fgmm_common.cuh"

namespace fgmm {

// partials: [slots][K][W] fp32 with W = 2d+1 laid out [s (d) | sq (d) | n];
// stats: [n (K) | s (K d) | sq (K d) | sum ln].  One thread per (k, c).
__global__ void reduce_partials_kernel(const float *__restrict__ part, int slots, int K, int d,
                                       double *__restrict__ stats) {
  const int W = 2 * d + 1;
  const int64_t total = (int64_t)K * W;
  const int64_t slot_stride = total;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    double acc = 0.0;
    for (int s = 0; s < slots; ++s) acc += (double)part[s * slot_stride + i];
    const int k = (int)(i / W), c = (int)(i % W);
    int64_t dst;
    if (c < d)            dst = K + (int64_t)k * d + c;                       // s_k
    else if (c < 2 * d)   dst = K + (int64_t)K * d + (int64_t)k * d + (c - d); // sq_k
    else                  dst = k;                                            // n_k
    stats[dst] = acc;
  }
}

__global__ void reduce_ln_kernel(const double *__restrict__ lnp, int n, double *__restrict__ out) {
  __shared__ double sh[256];
  double a = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) a += lnp[i];
  sh[threadIdx.x] = a;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) sh[threadIdx.x] += sh[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) *out = sh[0];
}

int reduce_partials(const float *partials, int slots, int K, int d, const double *ln_partials,
                    int ln_slots, double *stats, cudaStream_t stream) {
  const int64_t total = (int64_t)K * (2 * d + 1);
  int blocks = (int)std::min<int64_t>(cdiv(total, 256), 4 * num_sms());
  reduce_partials_kernel<<<blocks, 256, 0, stream>>>(partials, slots, K, d, stats);
  FGMM_LAUNCH_CHECK("reduce_partials_kernel");
  mark(stream, "reduce_partials_kernel");
  reduce_ln_kernel<<<1, 256, 0, stream>>>(ln_partials, ln_slots, stats + K + 2 * (int64_t)K * d);
  FGMM_LAUNCH_CHECK("reduce_ln_kernel");
  mark(stream, "reduce_ln_kernel");
  return FGMM_OK;
}

__global__ void em_update_kernel(const double *__restrict__ stats, double n_total, int K, int d,
                                 float *__restrict__ new_mu, float *__restrict__ new_var,
                                 float *__restrict__ new_log_pi) {
  const int k = blockIdx.x;
  const double nk = stats[k];
  const double inv = 1.0 / fmax(nk, 1e-8);
  const double *s = stats + K + (int64_t)k * d;
  const double *q = stats + K + (int64_t)K * d + (int64_t)k * d;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    const double m = s[j] * inv;
    new_mu[(int64_t)k * d + j] = (float)m;
    new_var[(int64_t)k * d + j] = (float)fmax(q[j] * inv - m * m, 1e-6);
  }
  if (threadIdx.x == 0) new_log_pi[k] = (float)log(fmax(nk / n_total, 1e-8));
}

int em_update(const double *stats, double n_total, int K, int d, float *new_mu, float *new_var,
              float *new_log_pi, cudaStream_t stream) {
  int threads = d >= 128 ? 128 : (d >= 64 ? 64 : 32);
  em_update_kernel<<<K, threads, 0, stream>>>(stats, n_total, K, d, new_mu, new_var, new_log_pi);
  FGMM_LAUNCH_CHECK("em_update_kernel");
  return FGMM_OK;
}

}  // namespace fgmm
