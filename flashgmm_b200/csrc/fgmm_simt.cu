// Generic fp32 CUDA-core ("SIMT") family of the fused EM statistics kernels.
//
// Runs every shape with 1 <= d <= 256 (the tensor-core family covers the common
// d <= 160 shapes).  Numerics follow the direct form of the reference's CPU path
// (flash_gmm/csrc/flash_gmm_cpu.cpp:30-45): each Mahalanobis term is evaluated
// as w = x*s - mu*s with s = var^{-1/2} (one FMA, no cancellation), summed as
// w*w; the log-sum-exp is the reference's online update
// (flash_gmm/csrc/flash_gmm_cpu.cpp:210-216) with accurate expf.
//
// Pass 1: one warp per point, lanes striped over the dimensions; components
// staged through shared memory in tiles.  Pass 2: a block owns a tile of TK
// components and a slice of the points; each warp keeps its own register
// accumulators for n_k, s_k, sq_k and the block combines warps in a fixed
// order, writing one fp32 partial per block (no atomics: deterministic).
#include <float.h>
#include <algorithm>
#include "fgmm_common.cuh"

namespace fgmm {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kP1Tile = 16;   // components per shared-memory tile in pass 1
constexpr int kP1Points = 4;  // points per warp per tile sweep in pass 1
constexpr int kTK = 8;        // components per block in pass 2

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// s = var^{-1/2}, ms = mu * s, lc = log_pi - 0.5 (d log 2pi + sum_j log var)
__global__ void simt_prep_kernel(const float *__restrict__ mu, const float *__restrict__ var,
                                 const float *__restrict__ log_pi, int K, int d,
                                 float *__restrict__ sc, float *__restrict__ ms,
                                 float *__restrict__ lc) {
  const int k = blockIdx.x;
  __shared__ double red[32];
  double ld = 0.0;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    const double v = var[(int64_t)k * d + j];
    const double s = 1.0 / sqrt(v);
    sc[(int64_t)k * d + j] = (float)s;
    ms[(int64_t)k * d + j] = (float)((double)mu[(int64_t)k * d + j] * s);
    ld += log(v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ld += __shfl_xor_sync(0xffffffffu, ld, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ld;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    lc[k] = (float)((double)log_pi[k] - 0.5 * (d * kLog2Pi + t));
  }
}

template <int DPL>
__device__ __forceinline__ void load_x(const float *__restrict__ X, int64_t n, int d, int lane,
                                       float (&x)[DPL]) {
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    const int j = lane + 32 * i;
    x[i] = (j < d) ? __ldg(X + n * d + j) : 0.0f;
  }
}

template <int DPL>
__device__ __forceinline__ float mahal(const float (&x)[DPL], const float *s, const float *m,
                                       int d, int lane) {
  float p = 0.0f;
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    const int j = lane + 32 * i;
    if (j < d) {
      const float w = fmaf(x[i], s[j], -m[j]);
      p = fmaf(w, w, p);
    }
  }
  return warp_sum(p);
}

// grid: cdiv(N, kWarps*kP1Points); each warp owns kP1Points consecutive points.
template <int DPL>
__global__ void __launch_bounds__(kThreads)
simt_pass1_kernel(const float *__restrict__ X, int64_t N, int d, const float *__restrict__ sc,
                  const float *__restrict__ ms, const float *__restrict__ lc, int K,
                  float *__restrict__ ln_out, double *__restrict__ ln_part) {
  extern __shared__ float sm[];
  float *s_t = sm;                    // [kP1Tile][d]
  float *m_t = s_t + kP1Tile * d;     // [kP1Tile][d]
  float *c_t = m_t + kP1Tile * d;     // [kP1Tile]
  __shared__ double wsum[kWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t n0 = ((int64_t)blockIdx.x * kWarps + warp) * kP1Points;

  float x[kP1Points][DPL];
  float rm[kP1Points], rs[kP1Points];
#pragma unroll
  for (int p = 0; p < kP1Points; ++p) {
    rm[p] = -FLT_MAX;
    rs[p] = 0.0f;
    if (n0 + p < N) load_x<DPL>(X, n0 + p, d, lane, x[p]);
    else {
#pragma unroll
      for (int i = 0; i < DPL; ++i) x[p][i] = 0.0f;
    }
  }
  for (int t = 0; t < K; t += kP1Tile) {
    const int tk = min(kP1Tile, K - t);
    __syncthreads();
    for (int i = threadIdx.x; i < tk * d; i += kThreads) {
      s_t[i] = sc[(int64_t)t * d + i];
      m_t[i] = ms[(int64_t)t * d + i];
    }
    if (threadIdx.x < tk) c_t[threadIdx.x] = lc[t + threadIdx.x];
    __syncthreads();
    for (int kk = 0; kk < tk; ++kk) {
#pragma unroll
      for (int p = 0; p < kP1Points; ++p) {
        const float ll = c_t[kk] - 0.5f * mahal<DPL>(x[p], s_t + kk * d, m_t + kk * d, d, lane);
        if (ll > rm[p]) { rs[p] = rs[p] * expf(rm[p] - ll) + 1.0f; rm[p] = ll; }
        else            { rs[p] += expf(ll - rm[p]); }
      }
    }
  }
  double acc = 0.0;
#pragma unroll
  for (int p = 0; p < kP1Points; ++p) {
    if (n0 + p < N) {
      const float l = rm[p] + logf(rs[p]);
      if (lane == 0) ln_out[n0 + p] = l;
      acc += (double)l;
    }
  }
  if (lane == 0) wsum[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < kWarps; ++w) t += wsum[w];
    ln_part[blockIdx.x] = t;
  }
}

// grid: (slots, cdiv(K, kTK)).  Block (s, ct) accumulates components
// [ct*kTK, ct*kTK + kTK) over points [s*chunk, (s+1)*chunk) and writes
// partial[k][s][0..2d] = [s_k | sq_k | n_k].
// GIN: the responsibilities are given (gamma[N][K], the standard M-step) instead of
// being recomputed from the parameters and the log-normalizer.
template <int DPL, bool GIN>
__global__ void __launch_bounds__(kThreads)
simt_pass2_kernel(const float *__restrict__ X, int64_t N, int d, const float *__restrict__ sc,
                  const float *__restrict__ ms, const float *__restrict__ lc, int K,
                  const float *__restrict__ ln, int64_t chunk, float *__restrict__ partial,
                  const float *__restrict__ gamma) {
  extern __shared__ float sm[];
  float *s_t = sm;                   // [kTK][d]
  float *m_t = s_t + kTK * d;        // [kTK][d]
  float *c_t = m_t + kTK * d;        // [kTK]
  float *acc_sm = c_t + kTK;         // [kTK][2d+1]
  const int W = 2 * d + 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int k0 = blockIdx.y * kTK;
  const int tk = min(kTK, K - k0);
  if (!GIN) {
    for (int i = threadIdx.x; i < tk * d; i += kThreads) {
      s_t[i] = sc[(int64_t)k0 * d + i];
      m_t[i] = ms[(int64_t)k0 * d + i];
    }
    if (threadIdx.x < tk) c_t[threadIdx.x] = lc[k0 + threadIdx.x];
  }
  for (int i = threadIdx.x; i < kTK * W; i += kThreads) acc_sm[i] = 0.0f;
  __syncthreads();

  float an[kTK], as[kTK][DPL], aq[kTK][DPL];
#pragma unroll
  for (int kk = 0; kk < kTK; ++kk) {
    an[kk] = 0.0f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) { as[kk][i] = 0.0f; aq[kk][i] = 0.0f; }
  }
  const int64_t pbeg = (int64_t)blockIdx.x * chunk;
  const int64_t pend = (pbeg + chunk < N) ? pbeg + chunk : N;
  for (int64_t n = pbeg + warp; n < pend; n += kWarps) {
    float x[DPL];
    load_x<DPL>(X, n, d, lane, x);
    const float l = GIN ? 0.0f : __ldg(ln + n);
#pragma unroll
    for (int kk = 0; kk < kTK; ++kk) {
      if (kk < tk) {
        float g;
        if (GIN) {
          g = __ldg(gamma + n * K + k0 + kk);
        } else {
          const float ll = c_t[kk] - 0.5f * mahal<DPL>(x, s_t + kk * d, m_t + kk * d, d, lane);
          g = expf(ll - l);
        }
        an[kk] += g;
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          const float gx = g * x[i];
          as[kk][i] += gx;
          aq[kk][i] = fmaf(gx, x[i], aq[kk][i]);
        }
      }
    }
  }
  // combine warps in a fixed order (deterministic)
  for (int w = 0; w < kWarps; ++w) {
    if (warp == w) {
#pragma unroll
      for (int kk = 0; kk < kTK; ++kk) {
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          const int j = lane + 32 * i;
          if (j < d) {
            acc_sm[kk * W + j] += as[kk][i];
            acc_sm[kk * W + d + j] += aq[kk][i];
          }
        }
        if (lane == 0) acc_sm[kk * W + 2 * d] += an[kk];
      }
    }
    __syncthreads();
  }
  for (int kk = 0; kk < tk; ++kk) {  // partial[k][slot][0..2d]
    float *dst = partial + ((int64_t)(k0 + kk) * gridDim.x + blockIdx.x) * W;
    for (int i = threadIdx.x; i < W; i += kThreads) dst[i] = acc_sm[kk * W + i];
  }
}

struct SimtWs {
  float *sc, *ms, *lc, *partial;
  double *ln_part;
  int slots, p1_blocks;
  int64_t chunk;
  size_t bytes;
};

SimtWs simt_layout(void *ws, int64_t N, int d, int K) {
  SimtWs w{};
  Carve c(ws);
  const int n_ct = (int)cdiv(K, kTK);
  const int target = 4 * num_sms();
  int slots = std::max(1, target / n_ct);
  slots = (int)std::min<int64_t>(slots, std::max<int64_t>(1, cdiv(N, 64)));
  w.slots = slots;
  w.chunk = cdiv(N, slots);
  w.p1_blocks = (int)cdiv(N, kWarps * kP1Points);
  w.sc = c.take<float>((size_t)K * d);
  w.ms = c.take<float>((size_t)K * d);
  w.lc = c.take<float>(K);
  w.partial = c.take<float>((size_t)slots * K * (2 * d + 1));
  w.ln_part = c.take<double>(w.p1_blocks);
  w.bytes = c.bytes();
  return w;
}

template <int DPL>
int simt_launch(const float *X, int64_t N, int d, int K, const SimtWs &w, float *ln,
                cudaStream_t st) {
  const size_t sm1 = (size_t)(2 * kP1Tile * d + kP1Tile) * sizeof(float);
  simt_pass1_kernel<DPL><<<w.p1_blocks, kThreads, sm1, st>>>(X, N, d, w.sc, w.ms, w.lc, K, ln,
                                                             w.ln_part);
  FGMM_LAUNCH_CHECK("simt_pass1_kernel");
  mark(st, "simt_pass1_kernel");
  const size_t sm2 = (size_t)(2 * kTK * d + kTK + kTK * (2 * d + 1)) * sizeof(float);
  if (sm2 > 48 * 1024)
    FGMM_CUDA_TRY(cudaFuncSetAttribute(simt_pass2_kernel<DPL, false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2));
  dim3 grid(w.slots, (unsigned)cdiv(K, kTK));
  simt_pass2_kernel<DPL, false><<<grid, kThreads, sm2, st>>>(X, N, d, w.sc, w.ms, w.lc, K, ln,
                                                             w.chunk, w.partial, nullptr);
  FGMM_LAUNCH_CHECK("simt_pass2_kernel");
  mark(st, "simt_pass2_kernel");
  return FGMM_OK;
}

template <int DPL>
int mstep_launch(const float *X, int64_t N, int d, const float *gamma, int K, const SimtWs &w,
                 cudaStream_t st) {
  const size_t sm2 = (size_t)(2 * kTK * d + kTK + kTK * (2 * d + 1)) * sizeof(float);
  if (sm2 > 48 * 1024)
    FGMM_CUDA_TRY(cudaFuncSetAttribute(simt_pass2_kernel<DPL, true>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2));
  dim3 grid(w.slots, (unsigned)cdiv(K, kTK));
  simt_pass2_kernel<DPL, true><<<grid, kThreads, sm2, st>>>(X, N, d, nullptr, nullptr, nullptr, K,
                                                            nullptr, w.chunk, w.partial, gamma);
  FGMM_LAUNCH_CHECK("simt_mstep_kernel");
  return FGMM_OK;
}

}  // namespace

int prep_direct_params(const float *mu, const float *var, const float *log_pi, int K, int d,
                       float *sc, float *ms, float *lc, cudaStream_t st) {
  simt_prep_kernel<<<K, 64, 0, st>>>(mu, var, log_pi, K, d, sc, ms, lc);
  FGMM_LAUNCH_CHECK("simt_prep_kernel");
  return FGMM_OK;
}

size_t mstep_workspace_bytes(int64_t N, int d, int K) { return simt_layout(nullptr, N, d, K).bytes; }

int mstep_stats(const float *X, int64_t N, int d, const float *gamma, int K, double *stats,
                void *ws, cudaStream_t st) {
  SimtWs w = simt_layout(ws, N, d, K);
  const int dpl = (d + 31) / 32;
  int rc;
  switch (dpl) {
    case 1: rc = mstep_launch<1>(X, N, d, gamma, K, w, st); break;
    case 2: rc = mstep_launch<2>(X, N, d, gamma, K, w, st); break;
    case 3: rc = mstep_launch<3>(X, N, d, gamma, K, w, st); break;
    case 4: rc = mstep_launch<4>(X, N, d, gamma, K, w, st); break;
    case 5: case 6: rc = mstep_launch<6>(X, N, d, gamma, K, w, st); break;
    default: rc = mstep_launch<8>(X, N, d, gamma, K, w, st); break;
  }
  if (rc != FGMM_OK) return rc;
  return reduce_partials(w.partial, w.slots, K, d, d, 2 * d + 1, w.ln_part, 0, stats, st);
}

int simt_launches() { return 4; }

size_t simt_workspace_bytes(int64_t N, int d, int K) { return simt_layout(nullptr, N, d, K).bytes; }

int simt_em_stats(const float *X, int64_t N, int d, const float *mu, const float *var,
                  const float *log_pi, int K, double *stats, float *log_norm, void *ws,
                  cudaStream_t st, const UpdateOut *update) {
  SimtWs w = simt_layout(ws, N, d, K);
  simt_prep_kernel<<<K, 64, 0, st>>>(mu, var, log_pi, K, d, w.sc, w.ms, w.lc);
  FGMM_LAUNCH_CHECK("simt_prep_kernel");
  mark(st, "simt_prep_kernel");
  const int dpl = (d + 31) / 32;
  int rc;
  switch (dpl) {
    case 1: rc = simt_launch<1>(X, N, d, K, w, log_norm, st); break;
    case 2: rc = simt_launch<2>(X, N, d, K, w, log_norm, st); break;
    case 3: rc = simt_launch<3>(X, N, d, K, w, log_norm, st); break;
    case 4: rc = simt_launch<4>(X, N, d, K, w, log_norm, st); break;
    case 5: case 6: rc = simt_launch<6>(X, N, d, K, w, log_norm, st); break;
    default: rc = simt_launch<8>(X, N, d, K, w, log_norm, st); break;
  }
  if (rc != FGMM_OK) return rc;
  return reduce_partials(w.partial, w.slots, K, d, d, 2 * d + 1, w.ln_part, w.p1_blocks, stats, st,
                         update);
}

}  // namespace fgmm
