// Reduction of per-block partial statistics and the M-step update.
//
// The M-step follows the reference's update (flash_gmm/csrc/flash_gmm_cuda.cu:298-322
// update_params_kernel, floors as in flash_gmm/csrc/flash_gmm_cpu.cpp:270-284):
//   mu = s * (1 / max(n, 1e-8)),  var = max(sq/n - mu^2, 1e-6),  log_pi = log(max(n/N, 1e-8))
// but is evaluated in fp64 from fp64 statistics and rounded once to fp32.
#include "fgmm_common.cuh"

namespace fgmm {

// partials: [K][slots][W] fp32 (a component's rows contiguous), each row laid out
// [s (ds) | sq (ds) | n | ...] where only the first d of each ds-wide run are meaningful;
// stats: [n (K) | s (K d) | sq (K d) | sum ln].
// One block per component (block K sums the per-block log-normalizer partials).  The
// 512 threads are G slot groups x DT dimension lanes: thread (g, j) sums dimension j's
// s and sq over slots g, g + G, ... with kRedBatch slots' loads in flight, so a warp reads
// 128 contiguous bytes per load; warp 0 first sums n_k.  The G group sums are added in a
// fixed order (deterministic) in fp64.  With `up`, the same block then applies the
// M-step to its component (em_update_kernel's arithmetic), which saves the update launch.
constexpr int kRedThreads = 512;
#ifndef FGMM_RED_BATCH
#define FGMM_RED_BATCH 8
#endif
constexpr int kRedBatch = FGMM_RED_BATCH;
struct UpdateArgs {
  double n_total;
  float *mu, *var, *log_pi;
  int floors, on;
  TcParamOps tc;  // next iteration's tensor-core operands (tc.kbp > 0)
};

__device__ __forceinline__ float2 update_component(double nk, double s, double q, double n_total,
                                                   int floors, float *mu, float *var) {
  const double inv = 1.0 / (floors ? fmax(nk, 1e-8) : nk);
  const double m = s * inv;
  const double v = q * inv - m * m;
  const float2 r = make_float2((float)m, (float)(v < 1e-6 ? 1e-6 : v));
  *mu = r.x;
  *var = r.y;
  return r;
}

__global__ void __launch_bounds__(kRedThreads)
reduce_partials_kernel(const float *__restrict__ part, int slots, int K, int d, int ds, int W,
                       const double *__restrict__ lnp, int ln_slots, double *__restrict__ stats,
                       UpdateArgs up) {
  __shared__ double sh_s[kRedThreads], sh_q[kRedThreads];
  __shared__ double sh_n;
  griddep_launch();
  griddep_wait();
  const int k = blockIdx.x, t = threadIdx.x, lane = t & 31;
  if (k == K) {  // the log-normalizer sum
    double a = 0.0;
    for (int j = t; j < ln_slots; j += kRedThreads) a += lnp[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) sh_s[t >> 5] = a;
    __syncthreads();
    if (t == 0) {
      double tot = 0.0;
      for (int w = 0; w < kRedThreads / 32; ++w) tot += sh_s[w];
      stats[K + 2 * (int64_t)K * d] = tot;
    }
    return;
  }
  const float *pk = part + (int64_t)k * slots * W;
  if (t < 32) {  // n_k: lanes over slots, fixed-order tree
    double a = 0.0;
    for (int sl = lane; sl < slots; sl += 32) a += (double)__ldg(pk + (int64_t)sl * W + 2 * ds);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) sh_n = a;
  }
  const int DT = d >= 128 ? 128 : (d + 31) / 32 * 32;  // dimension lanes
  const int G = kRedThreads / DT;                        // slot groups
  const int g = t / DT, jl = t - g * DT;
  for (int j0 = 0; j0 < d; j0 += DT) {
    const int j = j0 + jl;
    double as = 0.0, aq = 0.0;
    if (j < d) {
      const float *ps = pk + j, *pq = pk + ds + j;
      for (int sl = g; sl < slots; sl += G * kRedBatch) {
        float vs[kRedBatch], vq[kRedBatch];
#pragma unroll
        for (int u = 0; u < kRedBatch; ++u) {
          const int su = sl + u * G;
          vs[u] = su < slots ? __ldg(ps + (int64_t)su * W) : 0.0f;
          vq[u] = su < slots ? __ldg(pq + (int64_t)su * W) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kRedBatch; ++u) { as += (double)vs[u]; aq += (double)vq[u]; }
      }
    }
    sh_s[t] = as;
    sh_q[t] = aq;
    __syncthreads();
    if (g == 0 && j < d) {
      double s = 0.0, q = 0.0;
      for (int u = 0; u < G; ++u) { s += sh_s[u * DT + jl]; q += sh_q[u * DT + jl]; }
      stats[K + (int64_t)k * d + j] = s;
      stats[K + (int64_t)K * d + (int64_t)k * d + j] = q;
      if (up.on)
        update_component(sh_n, s, q, up.n_total, up.floors, up.mu + (int64_t)k * d + j,
                         up.var + (int64_t)k * d + j);
    }
    __syncthreads();
  }
  if (t == 0) {
    const double nk = sh_n;
    stats[k] = nk;
    if (up.on)
      up.log_pi[k] = (float)(up.floors ? log(fmax(nk / up.n_total, 1e-8)) : log(nk / up.n_total));
  }
}

// The same reduction for rows whose statistics runs are 16-byte aligned (ds and W
// multiples of 4, as the tensor-core family writes them): warp w of the block sums slots
// w, w + 16, ... with float4 loads (lane: four consecutive dimensions), four slots' loads
// in flight per lane, and the 16 warp sums are added in a fixed order.
// With the update on, the first 128 threads (thread j: dimension j, d <= 128) also write
// the next iteration's tensor-core parameter operands of component k's updated values
// (tc_prep_component, the same arithmetic tc_prep_params_kernel uses).
constexpr int kRed4Warps = 16;
__global__ void __launch_bounds__(32 * kRed4Warps)
reduce_rows4_kernel(const float *__restrict__ part, int slots, int K, int d, int ds, int W,
                    const double *__restrict__ lnp, int ln_slots, double *__restrict__ stats,
                    UpdateArgs up) {
  __shared__ double sh_s[kRed4Warps][128], sh_q[kRed4Warps][128];
  __shared__ double sh_n[kRed4Warps];
  griddep_launch();
  griddep_wait();
  const int k = blockIdx.x, t = threadIdx.x, lane = t & 31, w = t >> 5;
  if (k == K) {  // the log-normalizer sum
    double a = 0.0;
    for (int j = t; j < ln_slots; j += 32 * kRed4Warps) a += lnp[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) sh_n[w] = a;
    __syncthreads();
    if (t == 0) {
      double tot = 0.0;
      for (int u = 0; u < kRed4Warps; ++u) tot += sh_n[u];
      stats[K + 2 * (int64_t)K * d] = tot;
    }
    return;
  }
  const float *pk = part + (int64_t)k * slots * W;
  double nk = 0.0;
  for (int j0 = 0; j0 < d; j0 += 128) {
    const int j = j0 + 4 * lane;
    const bool in = j < d;
    double as[4] = {0.0, 0.0, 0.0, 0.0}, aq[4] = {0.0, 0.0, 0.0, 0.0}, an = 0.0;
    for (int sl = w; sl < slots; sl += 4 * kRed4Warps) {
      float4 vs[4], vq[4];
      float vn[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int su = sl + u * kRed4Warps;
        const bool live = su < slots;
        const float *row = pk + (int64_t)(live ? su : 0) * W;
        vs[u] = live && in ? __ldg(reinterpret_cast<const float4 *>(row + j)) : make_float4(0.f, 0.f, 0.f, 0.f);
        vq[u] = live && in ? __ldg(reinterpret_cast<const float4 *>(row + ds + j)) : make_float4(0.f, 0.f, 0.f, 0.f);
        vn[u] = live && j0 == 0 && lane == 0 ? __ldg(row + 2 * ds) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        as[0] += (double)vs[u].x; as[1] += (double)vs[u].y; as[2] += (double)vs[u].z; as[3] += (double)vs[u].w;
        aq[0] += (double)vq[u].x; aq[1] += (double)vq[u].y; aq[2] += (double)vq[u].z; aq[3] += (double)vq[u].w;
        an += (double)vn[u];
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) { sh_s[w][4 * lane + e] = as[e]; sh_q[w][4 * lane + e] = aq[e]; }
    if (j0 == 0 && lane == 0) sh_n[w] = an;
    __syncthreads();
    if (j0 == 0) {
      for (int u = 0; u < kRed4Warps; ++u) nk += sh_n[u];  // every thread, same order
    }
    float2 mv = make_float2(0.0f, 1.0f);
    if (t < 128 && j0 + t < d) {
      double sv = 0.0, qv = 0.0;
      for (int u = 0; u < kRed4Warps; ++u) { sv += sh_s[u][t]; qv += sh_q[u][t]; }
      const int jj = j0 + t;
      stats[K + (int64_t)k * d + jj] = sv;
      stats[K + (int64_t)K * d + (int64_t)k * d + jj] = qv;
      if (up.on)
        mv = update_component(nk, sv, qv, up.n_total, up.floors, up.mu + (int64_t)k * d + jj,
                              up.var + (int64_t)k * d + jj);
    }
    if (up.on && up.tc.kbp > 0 && t < 128) {  // d <= 128: one pass; operands of the new values
      const float lp32 = (float)(up.floors ? log(fmax(nk / up.n_total, 1e-8)) : log(nk / up.n_total));
      tc_prep_component(k, K, d, t, mv.x, mv.y, lp32, up.tc, 2);
    }
    __syncthreads();
  }
  if (t == 0) {
    stats[k] = nk;
    if (up.on)
      up.log_pi[k] = (float)(up.floors ? log(fmax(nk / up.n_total, 1e-8)) : log(nk / up.n_total));
  }
}

int reduce_partials(const float *partials, int slots, int K, int d, int ds, int W,
                    const double *ln_partials, int ln_slots, double *stats, cudaStream_t stream,
                    const UpdateOut *update) {
  UpdateArgs up{};
  if (update) {
    up.n_total = update->n_total;
    up.mu = update->mu;
    up.var = update->var;
    up.log_pi = update->log_pi;
    up.floors = update->floors ? 1 : 0;
    up.on = 1;
    up.tc = update->tc;
  }
  if (up.tc.kbp > 0 && !(ds % 4 == 0 && W % 4 == 0 && d <= 128 && reinterpret_cast<uintptr_t>(partials) % 16 == 0))
    return fail(FGMM_ERR_UNSUPPORTED, "fused parameter preparation needs the aligned row reduction");
  if (up.tc.kbp > 0 || (ds % 4 == 0 && W % 4 == 0 && reinterpret_cast<uintptr_t>(partials) % 16 == 0))
    FGMM_CUDA_TRY(launch_pdl(reduce_rows4_kernel, K + 1, 32 * kRed4Warps, 0, stream, partials,
                             slots, K, d, ds, W, ln_partials, ln_slots, stats, up));
  else
    FGMM_CUDA_TRY(launch_pdl(reduce_partials_kernel, K + 1, kRedThreads, 0, stream, partials,
                             slots, K, d, ds, W, ln_partials, ln_slots, stats, up));
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
  const double *s = stats + K + (int64_t)k * d;
  const double *q = stats + K + (int64_t)K * d + (int64_t)k * d;
  for (int j = threadIdx.x; j < d; j += blockDim.x)
    update_component(nk, s[j], q[j], n_total, floors, new_mu + (int64_t)k * d + j,
                     new_var + (int64_t)k * d + j);
  if (threadIdx.x == 0)
    new_log_pi[k] = (float)(floors ? log(fmax(nk / n_total, 1e-8)) : log(nk / n_total));
}

// em_update_kernel's M-step for d <= 128 (thread j: dimension j, 128 threads), which also
// writes the next iteration's tensor-core operands of the new values (tc_prep_component):
// the update step of a sharded fit, after the statistics all-reduce, in one launch.
// Blocks k >= K (padding components) only rewrite their padding operands.
__global__ void __launch_bounds__(128)
em_update_prep_kernel(const double *__restrict__ stats, double n_total, int K, int d,
                      float *__restrict__ new_mu, float *__restrict__ new_var,
                      float *__restrict__ new_log_pi, int floors, TcParamOps op) {
  griddep_launch();
  griddep_wait();
  const int k = blockIdx.x, j = threadIdx.x;
  float2 mv = make_float2(0.0f, 1.0f);
  float lp32 = 0.0f;
  if (k < K) {
    const double nk = stats[k];
    if (j < d)
      mv = update_component(nk, stats[K + (int64_t)k * d + j], stats[K + (int64_t)K * d + (int64_t)k * d + j],
                            n_total, floors, new_mu + (int64_t)k * d + j, new_var + (int64_t)k * d + j);
    lp32 = (float)(floors ? log(fmax(nk / n_total, 1e-8)) : log(nk / n_total));
    if (j == 0) new_log_pi[k] = lp32;
  }
  tc_prep_component(k, K, d, j, mv.x, mv.y, lp32, op, 1);
}

int em_update_prep(const double *stats, double n_total, int K, int Kp, int d, float *new_mu,
                   float *new_var, float *new_log_pi, const TcParamOps &op, cudaStream_t stream) {
  if (d > 128) return fail(FGMM_ERR_UNSUPPORTED, "operand preparation needs d <= 128");
  FGMM_CUDA_TRY(launch_pdl(em_update_prep_kernel, Kp, 128, 0, stream, stats, n_total, K, d, new_mu,
                           new_var, new_log_pi, 1, op));
  return FGMM_OK;
}

int em_update(const double *stats, double n_total, int K, int d, float *new_mu, float *new_var,
              float *new_log_pi, cudaStream_t stream, bool floors) {
  int threads = d >= 128 ? 128 : (d >= 64 ? 64 : 32);
  FGMM_CUDA_TRY(launch_pdl(em_update_kernel, K, threads, 0, stream, stats, n_total, K, d, new_mu,
                           new_var, new_log_pi, floors ? 1 : 0));
  return FGMM_OK;
}

}  // namespace fgmm
