// Low-K family: one fused statistics launch for K <= 16 components, d <= 128.
//
// With few components the tensor-core family pads the component tile to 128 (K = 8
// does 16x the needed contraction work) and runs four to five launches; the SIMT family
// walks X twice.  Here one kernel does the whole E-step and the block-level M-step
// statistics, and the shared row reduction (reduce_rows4_kernel, with the M-step fused)
// finishes the iteration: two launches per EM iteration.
//
// Per block (256 threads, persistent over 64-point tiles):
//   prologue  the direct-form parameters s = var^-1/2, m = mu s (fp64, rounded once) and
//             lc = log_pi - 1/2 (d log 2pi + sum log var) of all K components into
//             shared memory (what simt_prep_kernel computes, per block: no launch);
//   stage     the tile's rows of X into shared memory with cp.async (16-byte pieces when
//             d % 4 == 0), double-buffered: the next tile's copies run during this one;
//   phase 1   four threads per point (interleaved quarters of the dimensions, summed by
//             a shuffle tree, so no fp32 sum runs longer than d/4 terms) evaluate the K
//             log-likelihoods in the reference's direct form
//             (flash_gmm/csrc/flash_gmm_cpu.cpp:30-45: w = x s - m, one FMA, summed as
//             w w), then the log-sum-exp (max, then sum of expf) and
//             gamma_k = expf(l_k - ln) into shared memory, ln to the output;
//   phase 2   threads own (component group, 4 dimensions, point residue) cells and
//             accumulate n_k, s_k = sum gamma x and sq_k = sum gamma x^2 in fp32 over
//             at most 16 points, then fold them into their own fp64 slots in shared
//             memory, across all of the block's tiles (replaces the reference's
//             per-block shared accumulators and global atomics,
//             flash_gmm/csrc/flash_gmm_cuda.cu:179-292).
// At the end the point-residue groups' fp64 sums are added in a fixed order into one fp32
// partial row per (component, block), in reduce_rows4_kernel's layout [s (dp4) | sq (dp4)
// | n | pad], and one fp64 log-normalizer sum per block.  Deterministic: no atomics.
#include <float.h>
#include <algorithm>
#include "fgmm_common.cuh"

namespace fgmm {
namespace {

constexpr int kLkThreads = 256;
constexpr int kLkTPP = 4;                     // phase-1 threads per point
constexpr int kLkTile = kLkThreads / kLkTPP;  // points per tile
constexpr int kLkMaxK = 16;
constexpr int kLkMaxD = 128;
constexpr int kLkGS = kLkMaxK + 1;  // gamma row stride in shared memory

struct LkGeom {
  int dp4, D4, XS, W;  // d rounded to 4, float4 groups, X row stride, partial row width
};
__host__ __device__ inline LkGeom lk_geom(int d) {
  LkGeom g;
  g.dp4 = (d + 3) & ~3;
  g.D4 = g.dp4 / 4;
  // float4-aligned rows with XS = 16 (mod 32) words: a 128-bit phase of 8 threads (two
  // points x four interleaved dimension groups) reads 8 distinct 16-byte bank groups
  g.XS = g.dp4 + ((16 - g.dp4 % 32) + 32) % 32;
  g.W = 2 * g.dp4 + 4;
  return g;
}
constexpr int kLkFold = 16;  // points a thread sums in fp32 before folding into fp64
inline int lk_cpt(int d, int K) { return (K * lk_geom(d).D4 + kLkThreads - 1) / kLkThreads; }
// [X tile x 2 | gamma tile | s | m | lc] floats, then per-thread fp64 accumulators
// [cpt * 9][256] (an even float count precedes them: 8-byte aligned).
inline size_t lk_smem_floats(int d, int K) {
  const LkGeom g = lk_geom(d);
  return 2 * (size_t)kLkTile * g.XS + (size_t)kLkTile * kLkGS + 2 * (size_t)K * g.dp4 + kLkMaxK +
         2 * (size_t)lk_cpt(d, K) * 9 * kLkThreads;
}

// Asynchronous global -> shared copies (cp.async); src_bytes = 0 writes zeros.
__device__ __forceinline__ void cpa16(float *dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src),
               "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cpa4(float *dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src),
               "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cpa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cpa_wait_prev() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// CPT: components per phase-2 thread, ceil(K * D4 / 256) (1 or 2); KM: the most
// components the build handles (8: a 64-register build, four blocks per SM; 16: three
// blocks per SM with one component per phase-2 thread, two with two).
template <int CPT, int KM>
__global__ void __launch_bounds__(kLkThreads, KM <= 8 ? 4 : (CPT == 1 ? 3 : 2))
lowk_stats_kernel(const float *__restrict__ X, int64_t N, int d, const float *__restrict__ mu,
                  const float *__restrict__ var, const float *__restrict__ log_pi, int K,
                  float *__restrict__ ln_out, float *__restrict__ partial,
                  double *__restrict__ ln_part, int vec) {
  extern __shared__ __align__(16) float lk_sm[];
  const LkGeom g = lk_geom(d);
  float *x_s = lk_sm;                        // [2][kLkTile][XS] (double buffer)
  float *gm_s = x_s + 2 * kLkTile * g.XS;    // [kLkTile][kLkGS]
  float *s_s = gm_s + kLkTile * kLkGS;       // [K][dp4]
  float *m_s = s_s + K * g.dp4;              // [K][dp4]
  float *lc_s = m_s + K * g.dp4;             // [kLkMaxK]
  double *a64 = reinterpret_cast<double *>(lc_s + kLkMaxK);  // [CPT * 9][256], per thread
  __shared__ double wsum[kLkThreads / 32];
  griddep_launch();
  griddep_wait();
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;

  // ---- prologue: direct-form parameters (fp64, rounded once to fp32)
  for (int i = t; i < K * g.dp4; i += kLkThreads) {
    const int k = i / g.dp4, j = i - k * g.dp4;
    float sv = 0.0f, mv = 0.0f;
    if (j < d) {
      const double v = var[(int64_t)k * d + j];
      const double s = 1.0 / sqrt(v);
      sv = (float)s;
      mv = (float)((double)mu[(int64_t)k * d + j] * s);
    }
    s_s[i] = sv;
    m_s[i] = mv;
  }
  for (int k = warp; k < K; k += kLkThreads / 32) {
    double ld = 0.0;
    for (int j = lane; j < d; j += 32) ld += log((double)var[(int64_t)k * d + j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ld += __shfl_xor_sync(0xffffffffu, ld, o);
    if (lane == 0) lc_s[k] = (float)((double)log_pi[k] - 0.5 * (d * kLog2Pi + ld));
  }

  // ---- phase-2 cell of this thread
  const int NCG = (K + CPT - 1) / CPT;
  const int PS = kLkThreads / (g.D4 * NCG);
  const int j4 = t % g.D4, u = t / g.D4;
  const int cg = u % NCG, ps = u / NCG;
  const bool cell = ps < PS;
  // fp32 sums over at most kLkFold points, folded into this thread's own fp64 slots
  // (element e of component slot c at a64[(c * 9 + e) * 256 + t]: s 0-3, sq 4-7, n 8)
#pragma unroll
  for (int e = 0; e < CPT * 9; ++e) a64[e * kLkThreads + t] = 0.0;
  // ---- phase-1 role: point p1 of the tile, dimension groups sub, sub + 4, ...
  const int p1 = t / kLkTPP, sub = t % kLkTPP;
  double lnacc = 0.0;

  const int64_t ntiles = (N + kLkTile - 1) / kLkTile;
  // stage a tile's rows into buffer b (zero-filled past N and past d); one commit group
  auto stage = [&](int64_t tl, int b) {
    if (tl < ntiles) {
      const int64_t m0 = tl * kLkTile;
      const int mp = N - m0 < kLkTile ? (int)(N - m0) : kLkTile;
      float *dst = x_s + b * kLkTile * g.XS;
      if (vec) {
        const float4 *src = reinterpret_cast<const float4 *>(X + m0 * d);
        for (int i = t; i < kLkTile * g.D4; i += kLkThreads) {
          const int p = i / g.D4, q = i - p * g.D4;
          const bool in = p < mp;
          cpa16(dst + p * g.XS + 4 * q, in ? (const void *)(src + (int64_t)p * g.D4 + q) : (const void *)X,
                in ? 16u : 0u);
        }
      } else {
        for (int i = t; i < kLkTile * g.dp4; i += kLkThreads) {
          const int p = i / g.dp4, j = i - p * g.dp4;
          const bool in = p < mp && j < d;
          cpa4(dst + p * g.XS + j, in ? (const void *)(X + (m0 + p) * d + j) : (const void *)X,
               in ? 4u : 0u);
        }
      }
    }
    cpa_commit();
  };
  stage(blockIdx.x, 0);
  int cur = 0;
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, cur ^= 1) {
    const int64_t n0 = tile * kLkTile;
    const int np = N - n0 < kLkTile ? (int)(N - n0) : kLkTile;
    __syncthreads();  // the previous tile's phases are done with gm_s and the other buffer
    stage(tile + gridDim.x, cur ^ 1);  // the next tile's rows fly during this tile
    cpa_wait_prev();                   // this thread's copies of the current tile landed
    __syncthreads();
    const float *xb = x_s + cur * kLkTile * g.XS;

    // phase 1
    {
      float acc[KM];
#pragma unroll
      for (int k = 0; k < KM; ++k) acc[k] = 0.0f;
      const float *xr = xb + p1 * g.XS;
      for (int i = sub; i < g.D4; i += kLkTPP) {
        const float4 xv = *reinterpret_cast<const float4 *>(xr + 4 * i);
#pragma unroll
        for (int k = 0; k < KM; ++k) {
          if (k < K) {
            const float4 sv = *reinterpret_cast<const float4 *>(s_s + k * g.dp4 + 4 * i);
            const float4 mv = *reinterpret_cast<const float4 *>(m_s + k * g.dp4 + 4 * i);
            float w = fmaf(xv.x, sv.x, -mv.x);
            acc[k] = fmaf(w, w, acc[k]);
            w = fmaf(xv.y, sv.y, -mv.y);
            acc[k] = fmaf(w, w, acc[k]);
            w = fmaf(xv.z, sv.z, -mv.z);
            acc[k] = fmaf(w, w, acc[k]);
            w = fmaf(xv.w, sv.w, -mv.w);
            acc[k] = fmaf(w, w, acc[k]);
          }
        }
      }
      // the four quarters' sums by a tree (the same value in all four threads), each
      // thread's exponentials for components k = sub (mod 4) only
      float mx = -FLT_MAX;
#pragma unroll
      for (int k = 0; k < KM; ++k) {
        if (k < K) {
          acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], 1);
          acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], 2);
          acc[k] = lc_s[k] - 0.5f * acc[k];  // log-likelihood
          mx = fmaxf(mx, acc[k]);
        }
      }
      float sum = 0.0f;
#pragma unroll
      for (int k = 0; k < KM; ++k)
        if (k < K && (k & 3) == sub) sum += expf(acc[k] - mx);
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      const float ln = mx + logf(sum);
      const bool live = p1 < np;
#pragma unroll
      for (int k = 0; k < KM; ++k)
        if (k < K && (k & 3) == sub) gm_s[p1 * kLkGS + k] = live ? expf(acc[k] - ln) : 0.0f;
      if (live && sub == 0) {
        ln_out[n0 + p1] = ln;
        lnacc += (double)ln;
      }
    }
    __syncthreads();

    // phase 2
    if (cell) {
      for (int pb = ps; pb < np; pb += kLkFold * PS) {
        const int pe = min(np, pb + kLkFold * PS);
        float an[CPT], as[CPT][4], aq[CPT][4];
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
          an[c] = 0.0f;
#pragma unroll
          for (int e = 0; e < 4; ++e) { as[c][e] = 0.0f; aq[c][e] = 0.0f; }
        }
        for (int p = pb; p < pe; p += PS) {
          const float4 xv = *reinterpret_cast<const float4 *>(xb + p * g.XS + 4 * j4);
#pragma unroll
          for (int c = 0; c < CPT; ++c) {
            const int k = cg * CPT + c;
            if (k < K) {
              const float gk = gm_s[p * kLkGS + k];
              an[c] += gk;
              float gx = gk * xv.x; as[c][0] += gx; aq[c][0] = fmaf(gx, xv.x, aq[c][0]);
              gx = gk * xv.y; as[c][1] += gx; aq[c][1] = fmaf(gx, xv.y, aq[c][1]);
              gx = gk * xv.z; as[c][2] += gx; aq[c][2] = fmaf(gx, xv.z, aq[c][2]);
              gx = gk * xv.w; as[c][3] += gx; aq[c][3] = fmaf(gx, xv.w, aq[c][3]);
            }
          }
        }
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
          double *a = a64 + c * 9 * kLkThreads + t;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            a[e * kLkThreads] += (double)as[c][e];
            a[(4 + e) * kLkThreads] += (double)aq[c][e];
          }
          a[8 * kLkThreads] += (double)an[c];
        }
      }
    }
  }

  // ---- one partial row per component: the point-residue groups' fp64 sums added in a
  // fixed order, rounded once to fp32; row [s (dp4) | sq (dp4) | n | pad]
  __syncthreads();
  for (int i = t; i < K * g.W; i += kLkThreads) {
    const int k = i / g.W, col = i - k * g.W;
    const int kg = k / CPT, c = k - kg * CPT;
    int e = -1, jj = 0;
    if (col < g.dp4) { e = col & 3; jj = col >> 2; }
    else if (col < 2 * g.dp4) { e = 4 + ((col - g.dp4) & 3); jj = (col - g.dp4) >> 2; }
    else if (col == 2 * g.dp4) { e = 8; jj = 0; }
    double v = 0.0;
    if (e >= 0)
      for (int r = 0; r < PS; ++r) v += a64[(c * 9 + e) * kLkThreads + (r * NCG + kg) * g.D4 + jj];
    partial[((int64_t)k * gridDim.x + blockIdx.x) * g.W + col] = (float)v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) lnacc += __shfl_xor_sync(0xffffffffu, lnacc, o);
  if (lane == 0) wsum[warp] = lnacc;
  __syncthreads();
  if (t == 0) {
    double s = 0.0;
    for (int w = 0; w < kLkThreads / 32; ++w) s += wsum[w];
    ln_part[blockIdx.x] = s;
  }
}

int lowk_blocks_per_sm(int d, int K) {
  const size_t smem = lk_smem_floats(d, K) * sizeof(float);
  const int by_regs = K <= 8 ? 4 : (lk_cpt(d, K) == 1 ? 3 : 2);  // the builds' launch bounds
  return (int)std::max<size_t>(1, std::min<size_t>(by_regs, (size_t)(220 * 1024) / smem));
}

int lowk_blocks(int64_t N, int d, int K) {
  return (int)std::min<int64_t>(cdiv(N, kLkTile), (int64_t)lowk_blocks_per_sm(d, K) * num_sms());
}

struct LkWs {
  float *partial;
  double *ln_part;
  int slots;
  size_t bytes;
};

LkWs lk_layout(void *ws, int64_t N, int d, int K) {
  LkWs w{};
  Carve c(ws);
  w.slots = lowk_blocks(N, d, K);
  w.partial = c.take<float>((size_t)w.slots * K * lk_geom(d).W);
  w.ln_part = c.take<double>(w.slots);
  w.bytes = c.bytes();
  return w;
}

}  // namespace

bool lowk_supported(int64_t N, int d, int K) {
  return N >= 1 && K >= 1 && K <= kLkMaxK && d >= 1 && d <= kLkMaxD;
}

int lowk_launches() { return 2; }

size_t lowk_workspace_bytes(int64_t N, int d, int K) { return lk_layout(nullptr, N, d, K).bytes; }

int lowk_em_stats(const float *X, int64_t N, int d, const float *mu, const float *var,
                  const float *log_pi, int K, double *stats, float *log_norm, void *ws,
                  cudaStream_t st, const UpdateOut *update) {
  if (!lowk_supported(N, d, K)) return fail(FGMM_ERR_UNSUPPORTED, "low-K family: K <= 16, d <= 128");
  const LkWs w = lk_layout(ws, N, d, K);
  const LkGeom g = lk_geom(d);
  const size_t smem = lk_smem_floats(d, K) * sizeof(float);
  const int vec = (d % 4 == 0 && reinterpret_cast<uintptr_t>(X) % 16 == 0) ? 1 : 0;
  const int cpt = lk_cpt(d, K);
  auto go = [&](auto kernel, int slot) -> int {
    std::atomic<bool> &done = device_once_flag(slot);
    if (!done) {
      FGMM_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
      FGMM_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
      done = true;
    }
    FGMM_CUDA_TRY(launch_pdl(kernel, w.slots, kLkThreads, smem, st, X, N, d, mu, var, log_pi, K,
                             log_norm, w.partial, w.ln_part, vec));
    return FGMM_OK;
  };
  int rc;
  if (K <= 8) rc = go(lowk_stats_kernel<1, 8>, 0);
  else if (cpt == 1) rc = go(lowk_stats_kernel<1, 16>, 1);
  else rc = go(lowk_stats_kernel<2, 16>, 2);
  if (rc) return rc;
  mark(st, "lowk_stats_kernel");
  return reduce_partials(w.partial, w.slots, K, d, g.dp4, g.W, w.ln_part, w.slots, stats, st, update);
}

}  // namespace fgmm
