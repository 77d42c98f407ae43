// Reduction of per-block partial statistics and the M-step update.
//
// The M-step follows the reference's update (flash_gmm/csrc/flash_gmm_cuda.cu:298-322
// update_params_kernel, floors as in flash_gmm/csrc/flash_gmm_cpu.cpp:270-284):
//   mu = s * (1 / max(n, 1e-8)),  var = max(sq/n - mu^2, 1e-6),  log_pi = log(max(n/N, 1e-8))
// but is evaluated in fp64 from fp64 statistics and rounded once to fp32.
#include "fgmm_common.cuh"

namespace fgmm {

// partials: [slots][K][W] fp32, each row laid out [s (ds) | sq (ds) | n | ...] where only
// the first d of each ds-wide run are meaningful; stats: [n (K) | s (K d) | sq (K d) | sum ln].
// One thread per output value; the slots are summed in a fixed order with eight
// independent loads in flight (deterministic).  Block 0 also sums the per-block
// log-normalizer partials into the last entry.
__global__ void reduce_partials_kernel(const float *__restrict__ part, int slots, int K, int d,
                                       int ds, int W, const double *__restrict__ lnp, int ln_slots,
                                       double *__restrict__ stats) {
  const int V = 2 * d + 1;
  const int64_t total = (int64_t)K * V;
  const int64_t slot_stride = (int64_t)K * W;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(i / V), c = (int)(i % V);
    int src;
    int64_t dst;
    if (c < d)          { src = c;               dst = K + (int64_t)k * d + c; }
    else if (c < 2 * d) { src = ds + (c - d);    dst = K + (int64_t)K * d + (int64_t)k * d + (c - d); }
    else                { src = 2 * ds;          dst = k; }
    const float *p = part + (int64_t)k * W + src;
    double acc = 0.0;
    int s = 0;
    for (; s + 8 <= slots; s += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldg(p + (int64_t)(s + u) * slot_stride);
#pragma unroll
      for (int u = 0; u < 8; ++u) acc += (double)v[u];
    }
    for (; s < slots; ++s) acc += (double)__ldg(p + (int64_t)s * slot_stride);
    stats[dst] = acc;
  }
  if (blockIdx.x == 0) {
    __shared__ double sh[256];
    double a = 0.0;
    for (int j = threadIdx.x; j < ln_slots; j += blockDim.x) a += lnp[j];
    sh[threadIdx.x] = a;
    __syncthreads();
    for (int o = blockDim.x / 2; o > 0; o >>= 1) {
      if (threadIdx.x < o) sh[threadIdx.x] += sh[threadIdx.x + o];
      __syncthreads();
    }
    if (threadIdx.x == 0) stats[total] = sh[0];
  }
}

int reduce_partials(const float *partials, int slots, int K, int d, int ds, int W,
                    const double *ln_partials, int ln_slots, double *stats, cudaStream_t stream) {
  const int64_t total = (int64_t)K * (2 * d + 1);
  int blocks = (int)std::min<int64_t>(cdiv(total, 256), 8 * num_sms());
  reduce_partials_kernel<<<blocks, 256, 0, stream>>>(partials, slots, K, d, ds, W, ln_partials,
                                                     ln_slots, stats);
  FGMM_LAUNCH_CHECK("reduce_partials_kernel");
  mark(stream, "reduce_partials_kernel");
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
