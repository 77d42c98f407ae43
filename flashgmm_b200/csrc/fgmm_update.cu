// Reduction of per-block partial statistics and the M-step update.
//
// The M-step follows the reference's update (flash_gmm/csrc/flash_gmm_cuda.cu:298-322
// update_params_kernel, floors as in flash_gmm/csrc/flash_gmm_cpu.cpp:270-284):
//   mu = s * (1 / max(n, 1e-8)),  var = max(sq/n - mu^2, 1e-6),  log_pi = log(max(n/N, 1e-8))
// but is evaluated in fp64 from fp64 statistics and rounded once to fp32.
#include "fgmm_common.cuh"

namespace fgmm {

// partials: [K][slots][W] fp32 (a component's rows contiguous), each row laid out
// [s (ds) | sq (ds) | n | ...] where only
// the first d of each ds-wide run are meaningful; stats: [n (K) | s (K d) | sq (K d) | sum ln].
// A block takes 32 consecutive output values (lane = value, so the loads of a warp are
// contiguous) and splits the slots over its 8 warps (warp g sums slots g, g + 8, ... with
// every load in flight before the adds); the 8 warp sums are then added in a fixed order,
// so the result does not depend on timing.  Block 0 also sums the per-block
// log-normalizer partials into the last entry.
constexpr int kRedGroups = 8;
constexpr int kRedUnroll = 10;  // loads in flight per thread (one round trip up to 80 slots)
__global__ void __launch_bounds__(32 * kRedGroups, 6)  // six blocks (1536 threads) per SM
reduce_partials_kernel(const float *__restrict__ part, int slots, int K, int d, int ds, int W,
                       const double *__restrict__ lnp, int ln_slots, double *__restrict__ stats) {
  __shared__ double sh[kRedGroups][32];
  griddep_launch();
  griddep_wait();
  const int V = 2 * d + 1;
  const int64_t total = (int64_t)K * V;
  const int64_t slot_stride = W;
  const int lane = threadIdx.x & 31, g = threadIdx.x >> 5;
  for (int64_t base = (int64_t)blockIdx.x * 32; base < total; base += (int64_t)gridDim.x * 32) {
    const int64_t i = base + lane;
    const bool live = i < total;
    const int k = live ? (int)(i / V) : 0, c = live ? (int)(i % V) : 0;
    const int src = c < d ? c : (c < 2 * d ? ds + (c - d) : 2 * ds);
    const float *p = part + (int64_t)k * slots * W + src;
    double acc = 0.0;
    const int n_mine = live && g < slots ? (slots - g + kRedGroups - 1) / kRedGroups : 0;
    const float *q = p + (int64_t)g * slot_stride;
    const int step = kRedGroups * (int)slot_stride;
    for (int s = 0; s < n_mine; s += kRedUnroll) {  // all loads of a batch, then the adds
      float v[kRedUnroll];
#pragma unroll
      for (int u = 0; u < kRedUnroll; ++u) v[u] = s + u < n_mine ? __ldg(q + (s + u) * step) : 0.0f;
#pragma unroll
      for (int u = 0; u < kRedUnroll; ++u) acc += (double)v[u];
    }
    sh[g][lane] = acc;
    __syncthreads();
    if (g == 0 && live) {
      double t = 0.0;
#pragma unroll
      for (int u = 0; u < kRedGroups; ++u) t += sh[u][lane];
      const int64_t dst = c < d ? K + (int64_t)k * d + c
                        : (c < 2 * d ? K + (int64_t)K * d + (int64_t)k * d + (c - d) : (int64_t)k);
      stats[dst] = t;
    }
    __syncthreads();
  }
  if (blockIdx.x == 0) {
    double a = 0.0;
    for (int j = threadIdx.x; j < ln_slots; j += blockDim.x) a += lnp[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) sh[g][0] = a;
    __syncthreads();
    if (threadIdx.x == 0) {
      double t = 0.0;
      for (int u = 0; u < kRedGroups; ++u) t += sh[u][0];
      stats[total] = t;
    }
  }
}

int reduce_partials(const float *partials, int slots, int K, int d, int ds, int W,
                    const double *ln_partials, int ln_slots, double *stats, cudaStream_t stream) {
  const int64_t total = (int64_t)K * (2 * d + 1);
#ifndef FGMM_RED_BLOCKS_PER_SM
#define FGMM_RED_BLOCKS_PER_SM 16
#endif
  int blocks = (int)std::min<int64_t>(cdiv(total, 32), FGMM_RED_BLOCKS_PER_SM * num_sms());
  FGMM_CUDA_TRY(launch_pdl(reduce_partials_kernel, blocks, 32 * kRedGroups, 0, stream, partials,
                           slots, K, d, ds, W, ln_partials, ln_slots, stats));
  mark(stream, "reduce_partials_kernel");
  return FGMM_OK;
}

// floors = 1: the fused path's update (flash_gmm_cpu.cpp:270-284): n_k and the weight
// floored at 1e-8.  floors = 0: the reference's standard M-step
// (flash_gmm/csrc/binding.cpp:82-90, flash_gmm_cpu.cpp:292-311): plain division by n_k and
// log(n_k / N), only the variance clamped (a NaN stays NaN, as torch's clamp_min keeps it).
__global__ void em_update_kernel(const double *__restrict__ stats, double n_total, int K, int d,
                                 float *__restrict__ new_mu, float *__restrict__ new_var,
                                 float *__restrict__ new_log_pi, int floors) {
  griddep_launch();
  griddep_wait();
  const int k = blockIdx.x;
  const double nk = stats[k];
  const double inv = 1.0 / (floors ? fmax(nk, 1e-8) : nk);
  const double *s = stats + K + (int64_t)k * d;
  const double *q = stats + K + (int64_t)K * d + (int64_t)k * d;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    const double m = s[j] * inv;
    const double v = q[j] * inv - m * m;
    new_mu[(int64_t)k * d + j] = (float)m;
    new_var[(int64_t)k * d + j] = (float)(v < 1e-6 ? 1e-6 : v);
  }
  if (threadIdx.x == 0)
    new_log_pi[k] = (float)(floors ? log(fmax(nk / n_total, 1e-8)) : log(nk / n_total));
}

int em_update(const double *stats, double n_total, int K, int d, float *new_mu, float *new_var,
              float *new_log_pi, cudaStream_t stream, bool floors) {
  int threads = d >= 128 ? 128 : (d >= 64 ? 64 : 32);
  FGMM_CUDA_TRY(launch_pdl(em_update_kernel, K, threads, 0, stream, stats, n_total, K, d, new_mu,
                           new_var, new_log_pi, floors ? 1 : 0));
  return FGMM_OK;
}

}  // namespace fgmm
