// tcgen05 tensor-core family of the fused EM statistics kernels (sm_100a).
//
// Both passes evaluate the Mahalanobis term through the expansion
//   sum_j (x_j - mu_kj)^2 / var_kj = sum_j x_j^2 iv_kj - 2 sum_j x_j mu_kj iv_kj + sum_j mu_kj^2 iv_kj
// as one GEMM per (point tile, component tile):
//   acc[n,k] = P[n,:] . Q[k,:],   P[n] = [x^2 | x],  Q[k] = [iv | -2 mu iv]
// with the constant folded into cst2_k = log2(e) (log_pi - 1/2 (d log 2pi + sum log var + sum mu^2 iv)),
// so that log2-likelihood = cst2_k - (log2(e)/2) acc.  The GEMM runs in 3xTF32: every
// operand is split v = hi + lo with hi, lo tf32, and acc += lo_P.hi_Q + hi_P.lo_Q + hi_P.hi_Q.
// (Reference: the direct form in flash_gmm/csrc/flash_gmm_cuda.cu:135-156 and
// flash_gmm/csrc/flash_gmm_cpu.cpp:30-45.)
//
// Pass 1 (log-normalizer): persistent CTAs over (point tile, component group) units;
//   the accumulator lives in TMEM and eight epilogue warps run the online log-sum-exp of
//   flash_gmm/csrc/flash_gmm_cuda.cu:145-155 in base 2, writing one (max, sum) partial
//   per point and component group.
// Pass 2 (statistics): CTA (component tile ct, slot) walks a contiguous range of point
//   tiles.  Per tile: the distance GEMM again -> gamma = 2^(l2 - ln2) computed by the
//   epilogue from TMEM and stored to shared memory -> a second GEMM
//   S[k, f] = sum_n gamma[n,k] F[n,f],  F[n] = [x^2 | x] (hi + lo), and
//   n_k = sum_n gamma[n,k] on the CUDA cores.  gamma is split into tf32 hi + lo (three
//   products) and staged in two 64-point rounds; S restarts every tile and is added
//   (fp32, round-to-nearest) into one partial row per CTA; the partials are reduced in
//   fp64 afterwards: deterministic, no atomics between CTAs.  (Reference: flash_accumulate_stats_v2_kernel,
//   flash_gmm/csrc/flash_gmm_cuda.cu:179-292, which accumulates with global atomics.)
//
// Warp roles (320 threads): warp 0 issues TMA loads, warp 1 owns TMEM and issues
// tcgen05.mma (one thread), warps 2-9 are the epilogue: warp w reads TMEM lanes
// 32*(w%4) .. +31, and warps w and w+4 split the 128 columns of a tile.  No cluster
// multicast anywhere.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <algorithm>
#include <cmath>
#include <mutex>

#include "fgmm_common.cuh"
#include "sm100_ptx.cuh"

namespace fgmm {
using namespace ptx;

namespace {

constexpr int BM = 128;                       // points per tile
constexpr int NC = 128;                       // components per tile
constexpr int KC = 32;                        // fp32 elements per K chunk (one 128-byte row)
constexpr int kEpiWarps = 16;                 // four warps per TMEM lane quarter
constexpr int kThreads = 64 + 32 * kEpiWarps; // warp 0 TMA, warp 1 MMA, warps 2.. epilogue
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kPart = 32;                     // columns of a tile owned by one epilogue warp
constexpr int kParts = NC / kPart;            // epilogue warps per lane quarter
constexpr int kStages1 = 3;
constexpr int kTileBytes = BM * KC * 4;       // 16 KB: 128 rows x 128 B
constexpr int kStageBytes = 4 * kTileBytes;   // 64 KB
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kMaxDp = 128;                   // d <= 128 runs here

// Points buffer: P_hi and P_lo, each [Npad][2 dp] fp32 with Npad = N rounded up to a
// whole 128-row tile (rows >= N are zero), so no TMA box ever leaves the tensor.
inline int dp_of(int d) { return (d + KC - 1) / KC * KC; }
inline int64_t npad_of(int64_t N) { return cdiv(N, BM) * BM; }
inline size_t points_half_floats(int64_t N, int d) {
  return align_up((size_t)npad_of(N) * 2 * dp_of(d), 256);
}

__device__ __forceinline__ uint8_t *align1024(uint8_t *p) {
  uintptr_t a = reinterpret_cast<uintptr_t>(p);
  return reinterpret_cast<uint8_t *>((a + 1023) & ~uintptr_t(1023));
}

// --------------------------------------------------------------------------- prep
// P[n] = [x^2 (dp) | x (dp)] split into tf32 hi/lo (zero for j >= d and rows n >= N).
__global__ void tc_prep_points_kernel(const float *__restrict__ X, int64_t N, int64_t Npad, int d,
                                      int dp, float *__restrict__ phi, float *__restrict__ plo) {
  const int KA = 2 * dp;
  const int64_t total = Npad * dp;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / dp;
    const int j = (int)(i - n * dp);
    const float x = (j < d && n < N) ? __ldg(X + n * d + j) : 0.0f;
    const float x2 = x * x;
    const float x2h = to_tf32(x2), xh = to_tf32(x);
    phi[n * KA + j] = x2h;
    plo[n * KA + j] = to_tf32(x2 - x2h);
    phi[n * KA + dp + j] = xh;
    plo[n * KA + dp + j] = to_tf32(x - xh);
  }
}

// Q[k] = [iv (dp) | -2 mu iv (dp)] (hi/lo of the fp64 value), cst2[k]; rows k >= K are
// zero with cst2 = -inf (padding components never receive responsibility).
// Also writes the direct-form parameters the refinement uses: sc = var^{-1/2},
// ms = mu sc, lc = log_pi - 1/2 (d log 2pi + sum log var)  ([K][d], [K][d], [K]).
__global__ void tc_prep_params_kernel(const float *__restrict__ mu, const float *__restrict__ var,
                                      const float *__restrict__ log_pi, int K, int d, int dp,
                                      float *__restrict__ qhi, float *__restrict__ qlo,
                                      float *__restrict__ cst2, float *__restrict__ sc,
                                      float *__restrict__ ms, float *__restrict__ lc) {
  griddep_launch();
  griddep_wait();
  const int k = blockIdx.x;
  const int KA = 2 * dp;
  __shared__ double red[8], red2[8];
  double acc = 0.0;   // sum_j (log var + mu^2 / var)
  double acc2 = 0.0;  // sum_j log var
  for (int j = threadIdx.x; j < dp; j += blockDim.x) {
    double iv = 0.0, b = 0.0;
    if (k < K && j < d) {
      const double v = var[(int64_t)k * d + j];
      const double m = mu[(int64_t)k * d + j];
      iv = 1.0 / v;
      b = -2.0 * m * iv;
      acc += log(v) + m * m * iv;
      acc2 += log(v);
      const double sv = 1.0 / sqrt(v);
      sc[(int64_t)k * d + j] = (float)sv;
      ms[(int64_t)k * d + j] = (float)(m * sv);
    }
    const float ivh = to_tf32((float)iv), bh = to_tf32((float)b);
    qhi[(int64_t)k * KA + j] = ivh;
    qlo[(int64_t)k * KA + j] = to_tf32((float)(iv - (double)ivh));
    qhi[(int64_t)k * KA + dp + j] = bh;
    qlo[(int64_t)k * KA + dp + j] = to_tf32((float)(b - (double)bh));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc += __shfl_xor_sync(0xffffffffu, acc, o);
    acc2 += __shfl_xor_sync(0xffffffffu, acc2, o);
  }
  if ((threadIdx.x & 31) == 0) { red[threadIdx.x >> 5] = acc; red2[threadIdx.x >> 5] = acc2; }
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0, t2 = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) { t += red[w]; t2 += red2[w]; }
    cst2[k] = (k < K) ? (float)(1.4426950408889634 *
                                ((double)log_pi[k] - 0.5 * (d * kLog2Pi + t)))
                      : -INFINITY;
    if (k < K) lc[k] = (float)((double)log_pi[k] - 0.5 * (d * kLog2Pi + t2));
  }
}

// ------------------------------------------------------------- shared pieces
// Named barrier 1 across the epilogue warps that also ANDs a flag, so every epilogue
// warp takes the same early-exit decision (no warp is left waiting at a barrier).
__device__ __forceinline__ bool epi_sync_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kEpiThreads)
      : "memory");
  return r != 0;
}

// The distance GEMM is accumulated per 32-column K group (one staged chunk): each group
// goes into a fresh TMEM buffer, the 8 small cross products (lo.hi, hi.lo) first and the
// 4 hi.hi products last, and the epilogue adds the groups in fp32 registers.
// Tensor-memory accumulation does not round to nearest, so one long accumulation at the
// magnitude of the expanded form (|x|^2/var ~ thousands) drifts by ~1e-2; short groups
// with the small terms summed first, added on the CUDA cores, match a direct fp32
// evaluation of the Mahalanobis sum.

// K group size in staged 32-column chunks (divides NKC).
#ifndef FGMM_GROUP_CHUNKS
#define FGMM_GROUP_CHUNKS 1
#endif
template <int NKC>
__host__ __device__ constexpr int group_chunks() {
  constexpr int g = FGMM_GROUP_CHUNKS < NKC ? FGMM_GROUP_CHUNKS : NKC;
  return NKC % g == 0 ? g : (NKC % 2 == 0 ? 2 : 1);
}

// MMA side: one staged 32-column chunk of a K group that rotates over NB TMEM buffers;
// gfirst / glast mark the group's first / last chunk.
// `desc` is the stage's shared-memory descriptor (SWIZZLE_128B K-major, stage base); the
// operand tiles and k-steps are fixed offsets of its 16-byte address field, so the issuing
// thread (which shares its scheduler with a quarter of the epilogue warps) spends one add
// per operand.
template <int NB>
__device__ __forceinline__ bool issue_dist_chunk(uint64_t desc, uint32_t tmem, uint32_t &gcount,
                                                 uint32_t tfull0, uint32_t tempty0, bool gfirst,
                                                 bool glast) {
  constexpr uint32_t idesc = idesc_tf32(BM, NC, 0, 0);
  constexpr uint64_t kT = kTileBytes >> 4, kK = 32 >> 4;  // tile and k-step offsets
  const uint32_t buf = gcount % NB, use = gcount / NB;
  if (gfirst && !mbar_wait(tempty0 + 8u * buf, (use & 1u) ^ 1u, kErrWaitTmemEmpty)) return false;
  tc_fence_after();
  const uint32_t d = tmem + buf * NC;
#pragma unroll
  for (int kk = 0; kk < KC / 8; ++kk) {
    mma_tf32(d, desc + kT + kk * kK, desc + 2 * kT + kk * kK, idesc, (kk != 0 || !gfirst) ? 1u : 0u);
    mma_tf32(d, desc + kk * kK, desc + 3 * kT + kk * kK, idesc, 1u);
  }
#pragma unroll
  for (int kk = 0; kk < KC / 8; ++kk) mma_tf32(d, desc + kk * kK, desc + 2 * kT + kk * kK, idesc, 1u);
  if (glast) {
    mma_commit(tfull0 + 8u * buf);
    ++gcount;
  }
  return true;
}

// Epilogue side: add the next group buffer into acc (this warp's 32 rows, its 32 columns;
// lane_tmem already points at the warp's lane quarter and column part).
template <int NB, bool kFirst>
__device__ __forceinline__ bool drain_group(uint32_t lane_tmem, uint32_t &gcount, uint32_t tfull0,
                                            uint32_t tempty0, float (&acc)[kPart], int lane) {
  const uint32_t buf = gcount % NB, use = gcount / NB;
  if (!__all_sync(0xffffffffu, mbar_wait(tfull0 + 8u * buf, use & 1u, kErrWaitTmemFull)))
    return false;
  tc_fence_after();
  float v[kPart];
  tmem_ld32(lane_tmem + buf * NC, v);
  tmem_wait_ld();
#pragma unroll
  for (int e = 0; e < kPart; ++e) acc[e] = kFirst ? v[e] : acc[e] + v[e];
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(tempty0 + 8u * buf);
  ++gcount;
  return true;
}

// ------------------------------------------------------------------------- pass 1
template <int NKC>
__global__ void __launch_bounds__(kThreads, 1)
tc_pass1_kernel(const __grid_constant__ CUtensorMap tm_phi, const __grid_constant__ CUtensorMap tm_plo,
                const __grid_constant__ CUtensorMap tm_qhi, const __grid_constant__ CUtensorMap tm_qlo,
                const float *__restrict__ cst2, int64_t N, int n_pt, int n_ct, int G, int tpg,
                float *__restrict__ part_m, float *__restrict__ part_s,
                float2 *__restrict__ part_tv, int2 *__restrict__ part_ti,
                float *__restrict__ Lt, int64_t Npad) {
  constexpr int S = kStages1;
  constexpr int NB = 4;  // TMEM group buffers (4 x 128 columns)
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + S * kStageBytes);
  // bars: full[S] empty[S] tfull[NB] tempty[NB] done
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * S + 2 * NB + 1);
  struct Part { float m, s, v1, v2; int i1, i2; };
  Part *lse_x = reinterpret_cast<Part *>(tmem_slot + 2);  // [kParts - 1][128] row exchange
  const uint32_t bar0 = smem_u32(bars);
  auto FULL = [&](int s) { return bar0 + 8u * s; };
  auto EMPTY = [&](int s) { return bar0 + 8u * (S + s); };
  const uint32_t TFULL0 = bar0 + 8u * (2 * S), TEMPTY0 = bar0 + 8u * (2 * S + NB);
  const uint32_t DONE = bar0 + 8u * (2 * S + 2 * NB);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(FULL(s), 1); mbar_init(EMPTY(s), 1); }
    for (int b = 0; b < NB; ++b) {
      mbar_init(TFULL0 + 8u * b, 1);
      mbar_init(TEMPTY0 + 8u * b, kEpiWarps);
    }
    mbar_init(DONE, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  griddep_launch();
  griddep_wait();  // the parameter operands and Lt of earlier launches
  const uint32_t tmem = *tmem_slot;
  const int n_units = n_pt * G;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm_phi); prefetch_tmap(&tm_plo); prefetch_tmap(&tm_qhi); prefetch_tmap(&tm_qlo);
      // the points stream through once per component group; the parameters are re-read
      const uint64_t pol_p = policy_evict_first(), pol_q = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0, armed = 0, armed_par = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const int pt = u / G, g = u % G;
        const int t1 = min(n_ct, (g + 1) * tpg);
        for (int t = g * tpg; t < t1 && ok; ++t) {
          for (int c = 0; c < NKC; ++c) {
            if (!mbar_wait(EMPTY(stage), phase ^ 1, kErrWaitEmpty)) { ok = false; break; }
            const uint32_t base = smem_u32(smem + stage * kStageBytes);
            mbar_arrive_expect_tx(FULL(stage), kStageBytes);
            tma_load_2d_hint(base, &tm_phi, c * KC, pt * BM, FULL(stage), pol_p);
            tma_load_2d_hint(base + kTileBytes, &tm_plo, c * KC, pt * BM, FULL(stage), pol_p);
            tma_load_2d_hint(base + 2 * kTileBytes, &tm_qhi, c * KC, t * NC, FULL(stage), pol_q);
            tma_load_2d_hint(base + 3 * kTileBytes, &tm_qlo, c * KC, t * NC, FULL(stage), pol_q);
            armed |= 1u << stage;
            armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
            if (++stage == S) { stage = 0; phase ^= 1; }
          }
        }
      }
      // never leave the CTA with bulk copies in flight
      for (int s = 0; s < S; ++s)
        if (armed & (1u << s)) mbar_wait(FULL(s), (armed_par >> s) & 1u, kErrWaitDrain);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, gcount = 0;
      bool ok = true;
      const uint64_t desc0 = sdesc_sw128(smem_u32(smem), 16, 1024);
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const int g = u % G;
        const int t1 = min(n_ct, (g + 1) * tpg);
        for (int t = g * tpg; t < t1 && ok; ++t) {
          for (int c = 0; c < NKC; ++c) {
            if (!mbar_wait(FULL(stage), phase, kErrWaitFull)) { ok = false; break; }
            tc_fence_after();
            constexpr int GC = group_chunks<NKC>();
            if (!issue_dist_chunk<NB>(desc0 + (uint64_t)((stage * kStageBytes) >> 4), tmem, gcount,
                                      TFULL0, TEMPTY0, c % GC == 0, c % GC == GC - 1)) {
              ok = false;
              break;
            }
            mma_commit(EMPTY(stage));
            if (++stage == S) { stage = 0; phase ^= 1; }
          }
        }
      }
      mma_commit(DONE);
      mbar_wait(DONE, 0, kErrWaitDrain);
    }
    __syncwarp();
  } else {
    const int q = warp & 3, part = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const uint64_t pol_l = policy_evict_last();
    const uint32_t lane_tmem = tmem + ((uint32_t)(q * 32) << 16) + part * kPart;
    uint32_t gcount = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
      const int pt = u / G, g = u % G;
      const int t1 = min(n_ct, (g + 1) * tpg);
      float m = -INFINITY, s = 0.0f;
      float v1 = -INFINITY, v2 = -INFINITY;  // the row's two largest log2-likelihoods
      int i1 = -1, i2 = -1;
      const int64_t n_row = (int64_t)pt * BM + row;
      for (int t = g * tpg; t < t1 && ok; ++t) {
        const int kb = t * NC + part * kPart;
        float acc[kPart];
        ok = drain_group<NB, true>(lane_tmem, gcount, TFULL0, TEMPTY0, acc, lane);
#pragma unroll 1
        for (int grp = 1; grp < NKC / group_chunks<NKC>() && ok; ++grp)
          ok = drain_group<NB, false>(lane_tmem, gcount, TFULL0, TEMPTY0, acc, lane);
        if (!ok) break;
        float cst[kPart];  // this warp's 32 log-coefficients (uniform loads, L1-resident)
#pragma unroll
        for (int e = 0; e < kPart; e += 4)
          *reinterpret_cast<float4 *>(cst + e) = __ldg(reinterpret_cast<const float4 *>(cst2 + kb + e));
        float c4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // independent chains
#pragma unroll
        for (int e = 0; e < kPart; ++e) {
          acc[e] = fmaf(acc[e], -0.5f * kLog2e, cst[e]);
          c4[e & 3] = fmaxf(c4[e & 3], acc[e]);
        }
        const float cm = fmaxf(fmaxf(c4[0], c4[1]), fmaxf(c4[2], c4[3]));
        {  // the log2-likelihood matrix feeds the statistics pass; stored transposed
           // (Lt [component][point]) so that each store of a warp is 32 consecutive points
          // kept in L2 for the statistics pass (evict_last)
          float *lp = Lt + (int64_t)kb * Npad + n_row;
#pragma unroll
          for (int e = 0; e < kPart; ++e) st_hint(lp + (int64_t)e * Npad, acc[e], pol_l);
        }
        const float mn = fmaxf(m, cm);
        const float mr = (mn == -INFINITY) ? 0.0f : mn;
        float a4[4] = {s * ex2(m - mr), 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int e = 0; e < kPart; ++e) a4[e & 3] += ex2(acc[e] - mr);
        s = (a4[0] + a4[1]) + (a4[2] + a4[3]);
        m = mn;
        if (cm > v2) {  // the tile's two largest, without data-dependent branches
          int e1 = kPart;  // first column at the maximum
#pragma unroll
          for (int e = kPart - 1; e >= 0; --e) e1 = acc[e] == cm ? e : e1;
          float t4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
          int k4[4] = {-1, -1, -1, -1};
#pragma unroll
          for (int e = 0; e < kPart; ++e) {
            const bool take = e != e1 && acc[e] > t4[e & 3];
            t4[e & 3] = take ? acc[e] : t4[e & 3];
            k4[e & 3] = take ? e : k4[e & 3];
          }
          float t2 = t4[0];
          int e2 = k4[0];
#pragma unroll
          for (int c = 1; c < 4; ++c)
            if (t4[c] > t2 || (t4[c] == t2 && k4[c] >= 0 && (e2 < 0 || k4[c] < e2))) { t2 = t4[c]; e2 = k4[c]; }
          auto insert = [&](float x, int ix) {
            if (x > v2) {
              if (x > v1) { v2 = v1; i2 = i1; v1 = x; i1 = ix; }
              else        { v2 = x; i2 = ix; }
            }
          };
          if (e1 < kPart) {
            insert(cm, kb + e1);
            if (e2 >= 0) insert(t2, kb + e2);
          }
        }
      }
      // merge the column parts of each row
      if (part > 0) lse_x[(part - 1) * BM + row] = Part{m, s, v1, v2, i1, i2};
      ok = epi_sync_and(ok);
      if (part == 0) {
        Part o[kParts];
        o[0] = Part{m, s, v1, v2, i1, i2};
#pragma unroll
        for (int r = 1; r < kParts; ++r) o[r] = lse_x[(r - 1) * BM + row];
        float mn = -INFINITY;
#pragma unroll
        for (int r = 0; r < kParts; ++r) mn = fmaxf(mn, o[r].m);
        const float mr = (mn == -INFINITY) ? 0.0f : mn;
        float sm = 0.0f;
        float b1 = -INFINITY, b2 = -INFINITY;
        int j1 = -1, j2 = -1;
#pragma unroll
        for (int r = 0; r < kParts; ++r) {
          sm += o[r].s * ex2(o[r].m - mr);
          const float c[2] = {o[r].v1, o[r].v2};
          const int ci[2] = {o[r].i1, o[r].i2};
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            if (c[e] > b2) {
              if (c[e] > b1) { b2 = b1; j2 = j1; b1 = c[e]; j1 = ci[e]; }
              else           { b2 = c[e]; j2 = ci[e]; }
            }
          }
        }
        const int64_t n = (int64_t)pt * BM + row;
        if (ok && n < N) {
          part_m[(int64_t)g * N + n] = mn;
          part_s[(int64_t)g * N + n] = sm;
          part_tv[(int64_t)g * N + n] = make_float2(b1, b2);
          part_ti[(int64_t)g * N + n] = make_int2(j1, j2);
        }
      }
      ok = epi_sync_and(ok);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------- refine
// Exact re-evaluation of each point's two leading components.  The tensor-core
// log-likelihoods carry an absolute error of ~1e-4..1e-3 (the expanded form's terms
// |x|^2/var are far larger than the Mahalanobis distance they cancel down to), while
// responsibility mass sits on one or two components per point.  This kernel merges the
// pass-1 partials of the component groups, recomputes the two leading log-likelihoods in
// the direct form of flash_gmm/csrc/flash_gmm_cpu.cpp:30-45 (fp32, with
// w = x var^{-1/2} - mu var^{-1/2} formed by one FMA), swaps them into the log-sum-exp,
// and writes the log-normalizer (output and log2 form for pass 2), the two exact
// log2-likelihoods over their tensor-core values in L, and one log-normalizer sum per
// block.
// Eight lanes per point (four points per warp), lanes striped over the dimensions; all
// loads of a point are issued before its reductions.
// Blocks per SM (register budget): five for 16 dimensions per lane, four below (measured).
template <int DPL, bool VEC>  // dimensions per lane: ceil(d / 8); VEC: float4 loads
__global__ void __launch_bounds__(256, DPL >= 16 ? 5 : 4)
tc_refine_kernel(const float *__restrict__ X, int64_t N, int d, const float *__restrict__ sc,
                 const float *__restrict__ ms, const float *__restrict__ lc,
                 const float *__restrict__ part_m, const float *__restrict__ part_s,
                 const float2 *__restrict__ part_tv, const int2 *__restrict__ part_ti, int G,
                 float *__restrict__ ln2x, float *__restrict__ Lt, int64_t Npad,
                 float *__restrict__ ln_out, double *__restrict__ ln_part, int acc_ln) {
  __shared__ double wsum[8];
  griddep_launch();
  griddep_wait();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane & 7;           // lane within the point's group of 8
  double acc = 0.0;
  const int64_t stride = (int64_t)gridDim.x * 32;  // points per grid sweep
  for (int64_t n = ((int64_t)blockIdx.x * 8 + warp) * 4 + (lane >> 3); n - (lane >> 3) < N;
       n += stride) {
    const bool live = n < N;
    const int64_t nn = live ? n : 0;
    // the point's row first (independent of everything below), so its latency overlaps
    // the partial loads and the parameter gathers
    float x[DPL], s1[DPL], m1[DPL], s2[DPL], m2[DPL];
    if (VEC) {  // d == 8 DPL, DPL % 4 == 0, 16-byte aligned rows; lane takes float4 i * 8 + sub
      const float4 *xp = reinterpret_cast<const float4 *>(X + nn * d) + sub;
#pragma unroll
      for (int i = 0; i < DPL / 4; ++i) {
        const float4 a = __ldg(xp + 8 * i);
        x[4 * i] = a.x; x[4 * i + 1] = a.y; x[4 * i + 2] = a.z; x[4 * i + 3] = a.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        const int j = i * 8 + sub;
        x[i] = j < d ? __ldg(X + nn * d + j) : 0.0f;
      }
    }
    // merge the component groups' partials: online log-sum-exp and top-2
    float mx = -INFINITY, sm = 0.0f, b1 = -INFINITY, b2 = -INFINITY;
    int j1 = -1, j2 = -1;
#pragma unroll 4
    for (int g = 0; g < G; ++g) {
      const float pm = __ldg(part_m + (int64_t)g * N + nn);
      const float ps = __ldg(part_s + (int64_t)g * N + nn);
      const float2 tv = part_tv[(int64_t)g * N + nn];
      const int2 ti = part_ti[(int64_t)g * N + nn];
      const float mn = fmaxf(mx, pm);
      const float mr = mn == -INFINITY ? 0.0f : mn;
      sm = sm * ex2(mx - mr) + ps * ex2(pm - mr);
      mx = mn;
      if (ti.x >= 0 && tv.x > b2) {
        if (tv.x > b1) { b2 = b1; j2 = j1; b1 = tv.x; j1 = ti.x; }
        else           { b2 = tv.x; j2 = ti.x; }
      }
      if (ti.y >= 0 && tv.y > b2) {
        if (tv.y > b1) { b2 = b1; j2 = j1; b1 = tv.y; j1 = ti.y; }
        else           { b2 = tv.y; j2 = ti.y; }
      }
    }
    // the runner-up only matters when it is within 2^-40 of the leader (otherwise its
    // responsibility is below 1e-12 and its tensor-core value is kept)
    if (j2 >= 0 && b2 < b1 - 40.0f) j2 = -1;
    const int k1 = j1 >= 0 ? j1 : 0, k2 = j2 >= 0 ? j2 : 0;
    const bool need2 = __any_sync(0xffffffffu, j2 >= 0);
    // the 8 lanes of a point read each row in consecutive 16-byte (VEC) or 4-byte pieces,
    // so a load instruction of the warp touches whole 128-byte lines
    const bool use2 = need2 && j2 >= 0;
    if (VEC) {
      const float4 *s1p = reinterpret_cast<const float4 *>(sc + (int64_t)k1 * d) + sub;
      const float4 *m1p = reinterpret_cast<const float4 *>(ms + (int64_t)k1 * d) + sub;
      const float4 *s2p = reinterpret_cast<const float4 *>(sc + (int64_t)k2 * d) + sub;
      const float4 *m2p = reinterpret_cast<const float4 *>(ms + (int64_t)k2 * d) + sub;
#pragma unroll
      for (int i = 0; i < DPL / 4; ++i) {
        const float4 b = __ldg(s1p + 8 * i), c = __ldg(m1p + 8 * i);
        const float4 e = use2 ? __ldg(s2p + 8 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 f = use2 ? __ldg(m2p + 8 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
        s1[4 * i] = b.x; s1[4 * i + 1] = b.y; s1[4 * i + 2] = b.z; s1[4 * i + 3] = b.w;
        m1[4 * i] = c.x; m1[4 * i + 1] = c.y; m1[4 * i + 2] = c.z; m1[4 * i + 3] = c.w;
        s2[4 * i] = e.x; s2[4 * i + 1] = e.y; s2[4 * i + 2] = e.z; s2[4 * i + 3] = e.w;
        m2[4 * i] = f.x; m2[4 * i + 1] = f.y; m2[4 * i + 2] = f.z; m2[4 * i + 3] = f.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        const int j = i * 8 + sub;
        const bool in = j < d;
        s1[i] = in ? __ldg(sc + (int64_t)k1 * d + j) : 0.0f;
        m1[i] = in ? __ldg(ms + (int64_t)k1 * d + j) : 0.0f;
        s2[i] = in && use2 ? __ldg(sc + (int64_t)k2 * d + j) : 0.0f;
        m2[i] = in && use2 ? __ldg(ms + (int64_t)k2 * d + j) : 0.0f;
      }
    }
    float p1 = 0.0f, p2 = 0.0f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const float w1 = fmaf(x[i], s1[i], -m1[i]);
      const float w2 = fmaf(x[i], s2[i], -m2[i]);
      p1 = fmaf(w1, w1, p1);
      p2 = fmaf(w2, w2, p2);
    }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
      p1 += __shfl_xor_sync(0xffffffffu, p1, o);
      p2 += __shfl_xor_sync(0xffffffffu, p2, o);
    }
    const float e1 = j1 >= 0 ? (__ldg(lc + k1) - 0.5f * p1) * kLog2e : -INFINITY;
    const float e2 = j2 >= 0 ? (__ldg(lc + k2) - 0.5f * p2) * kLog2e : -INFINITY;
    // swap the approximate leading terms of the sum for the exact ones
    const float m = fmaxf(mx, fmaxf(e1, e2));
    float rest = sm * ex2(mx - m);
    if (j1 >= 0) rest -= ex2(b1 - m);
    if (j2 >= 0) rest -= ex2(b2 - m);
    float tot = fmaxf(rest, 0.0f);
    if (j1 >= 0) tot += ex2(e1 - m);
    if (j2 >= 0) tot += ex2(e2 - m);
    const float ln2 = m + __log2f(tot);
    if (live && sub == 0) {
      ln2x[n] = ln2;
      if (j1 >= 0) Lt[(int64_t)j1 * Npad + n] = e1;
      if (j2 >= 0) Lt[(int64_t)j2 * Npad + n] = e2;
      const float l = ln2 * kLn2;
      ln_out[n] = l;
      acc += (double)l;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) wsum[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < 8; ++w) t += wsum[w];
    ln_part[blockIdx.x] = acc_ln ? ln_part[blockIdx.x] + t : t;  // chunks add up in order
  }
}

// ------------------------------------------------------------------------- pass 2
// Statistics GEMM S[k, f] = sum_n gamma[n, k] F[n, f] with F = [x^2 | x] (3xTF32), the
// only tensor-core work left once pass 1 has stored the log2-likelihood matrix L (with
// the refined leading components written over their tensor-core values).  A CTA owns
// 128 components (the M of the MMA, on the TMEM lanes) and a contiguous range of points,
// taken in slices of 16 points (the K of two MMA k-steps).  Warp roles (16 warps):
//   warp 9 lane 0 (producer): per slice, TMA of F hi and F lo from the prepared points
//     buffer (one 3-D box each: 16 points x all 32-feature atoms, MN-major
//     SWIZZLE_128B_ATOM_32B), of the slice's L tile [16 points][128 components] and of
//     its 16 log2-normalizers, into a ring of kStages slices;
//   warps 0-7 (gamma): warp w computes gamma = 2^(L - ln2) for components
//     32 (w % 4) .. +31 (its TMEM lane quarter) at 8 of the slice's 16 points, splits it
//     into tf32 hi / lo and stores both to a TMEM gamma buffer (ring of kGBufs), the
//     MMA's A operand;
//   warp 8 lane 0 (MMA): six MMAs per slice (gamma_lo F_hi, gamma_hi F_lo, then
//     gamma_hi F_hi, two k-steps each) into the statistics accumulator;
//   all 16 warps: every kSlicesFlush slices (128 points) the accumulator is added into
//     fp32 registers (warp w: lane quarter w % 4, a quarter of the columns), because
//     tensor-memory accumulation does not round to nearest.  With two accumulator
//     regions (KA <= 192) the tensor pipe fills one while the other drains; at KA = 256
//     the single region is drained between tiles.  Warps waiting only for a drain sleep
//     between polls.
// Every hand-off is an mbarrier; no barrier spans the CTA inside the loop.
constexpr int kSlicePts = 16;
constexpr int kSlicesFlush = 8;
constexpr int kGBufs = 4;
constexpr int kThreads2 = 512;
constexpr int kGammaWarps = 8;
constexpr int kGCols = 2 * kSlicePts;  // TMEM columns of one gamma buffer (hi | lo)

template <int KA>
struct StatsShape {
  static constexpr int kAtom = kSlicePts * 128;                // 2 KB: 16 points x 32 fp32
  static constexpr int kFPart = (KA / 32) * kAtom;             // F hi (or lo) of a slice
  static constexpr int kLOff = 2 * kFPart;                     // L tile [128][16], 64B-swizzled
  static constexpr int kNOff = kLOff + kSlicePts * NC * 4;     // ln2 [16]
  static constexpr int kStage = (kNOff + kSlicePts * 4 + 1023) / 1024 * 1024;
  static constexpr int kStagesFit = (220 * 1024) / kStage;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int kSmem = 1024 + kStages * kStage + 512;
};

__device__ __forceinline__ bool cta_sync_and(bool v) {
  return __syncthreads_and(v ? 1 : 0) != 0;
}

// Partial statistics row (per component and CTA slot, partial[k][slot]):
// [s (DP) | sq (DP) | n | pad], stride 2 DP + 4.
template <int NKC>
__global__ void __launch_bounds__(kThreads2, 1)
tc_stats_kernel(const __grid_constant__ CUtensorMap tm_fhi, const __grid_constant__ CUtensorMap tm_flo,
                const __grid_constant__ CUtensorMap tm_l, const float *__restrict__ ln2x, int64_t N,
                int S_slots, int K, float *__restrict__ partial, int accum) {
  constexpr int KA = NKC * KC;
  constexpr int DP = KA / 2;
  constexpr int PSTRIDE = 2 * DP + 4;
  constexpr int SEG = KA / 4;  // statistics columns per warp
  constexpr int NSR = 2 * KA + kGBufs * kGCols <= 512 ? 2 : 1;  // accumulator regions
  constexpr uint32_t kGBase = NSR * KA;                           // TMEM column of gamma buffer 0
  using Sh = StatsShape<KA>;
  constexpr int NST = Sh::kStages;
  static_assert(NSR * KA + kGBufs * kGCols <= 512, "TMEM budget");
  static_assert(SEG % 16 == 0, "statistics segment of whole 16-column loads");
  static_assert(NST >= 2, "shared-memory budget");
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + NST * Sh::kStage);
  // bars: full[NST] empty[NST] gfull[G] gempty[G] sfull[2] sempty[2] done
  const uint32_t bar0 = smem_u32(bars);
  auto FULL = [&](int s) { return bar0 + 8u * s; };
  auto EMPTY = [&](int s) { return bar0 + 8u * (NST + s); };
  auto GFULL = [&](int g) { return bar0 + 8u * (2 * NST + g); };
  auto GEMPTY = [&](int g) { return bar0 + 8u * (2 * NST + kGBufs + g); };
  auto SFULL = [&](int r) { return bar0 + 8u * (2 * NST + 2 * kGBufs + r); };
  auto SEMPTY = [&](int r) { return bar0 + 8u * (2 * NST + 2 * kGBufs + 2 + r); };
  const uint32_t DONE = bar0 + 8u * (2 * NST + 2 * kGBufs + 4);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * NST + 2 * kGBufs + 5);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ct = blockIdx.x / S_slots, slot = blockIdx.x % S_slots;
  const int64_t n_sl = (N + kSlicePts - 1) / kSlicePts;
  const int64_t s0 = slot * n_sl / S_slots, s1 = (slot + 1) * n_sl / S_slots;
  const int S = (int)(s1 - s0);                        // slices of this CTA
  const int T = (S + kSlicesFlush - 1) / kSlicesFlush;  // flush tiles

  if (threadIdx.x == 0) {
    for (int i = 0; i < NST; ++i) { mbar_init(FULL(i), 1); mbar_init(EMPTY(i), 1 + kGammaWarps); }
    for (int g = 0; g < kGBufs; ++g) { mbar_init(GFULL(g), kGammaWarps); mbar_init(GEMPTY(g), 1); }
    for (int r = 0; r < 2; ++r) { mbar_init(SFULL(r), 1); mbar_init(SEMPTY(r), 16); }
    mbar_init(DONE, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  griddep_launch();
  griddep_wait();  // Lt, ln2x and the partial rows of earlier launches
  const uint32_t tmem = *tmem_slot;

  const int q = warp & 3, seg = warp >> 2;  // TMEM lane quarter, column segment
  const uint32_t lane_tmem = tmem + ((uint32_t)(q * 32) << 16);
  const int cl = q * 32 + lane;             // component of this lane within the CTA's 128
  float sacc[SEG];
#pragma unroll
  for (int e = 0; e < SEG; ++e) sacc[e] = 0.0f;
  int nf = 0;  // next tile this warp drains
  bool ok = true;

  // Adds accumulator region of tile nf into sacc (whole warp).
  auto flush_next = [&](bool sleep) {
    const int j = nf++;
    const int reg = NSR == 2 ? (j & 1) : 0;
    ok = ok && __all_sync(0xffffffffu, sleep ? mbar_wait_sleep(SFULL(reg), (j / NSR) & 1, kErrWaitStatsDone)
                                             : mbar_wait(SFULL(reg), (j / NSR) & 1, kErrWaitStatsDone));
    if (!ok) return;
    tc_fence_after();
#pragma unroll
    for (int c = 0; c < SEG / 32; ++c) {  // two loads in flight per wait
      float v[32];
      tmem_ld16(lane_tmem + reg * KA + seg * SEG + c * 32, *reinterpret_cast<float(*)[16]>(v));
      tmem_ld16(lane_tmem + reg * KA + seg * SEG + c * 32 + 16, *reinterpret_cast<float(*)[16]>(v + 16));
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 32; ++e) sacc[c * 32 + e] += v[e];
    }
    if (SEG % 32) {
      float v[16];
      tmem_ld16(lane_tmem + reg * KA + seg * SEG + SEG - 16, v);
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 16; ++e) sacc[SEG - 16 + e] += v[e];
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(SEMPTY(reg));
  };

  // Warp-uniform probe: have the MMAs of tile j completed?
  auto tile_done = [&](int j) -> bool {
    return __all_sync(0xffffffffu, mbar_test(SFULL(NSR == 2 ? (j & 1) : 0), (j / NSR) & 1));
  };

  float nk = 0.0f;
  if (warp < kGammaWarps) {
    // ---------------- gamma warps
    const int p0 = (warp >> 2) * 8;  // this warp's 8 points of each slice
    for (int s = 0; s < S && ok; ++s) {
      // Tile j is drained once this warp is kGBufs slices into tile j + 1: having waited
      // for the MMAs of slice 8j + 7 it finds tile j complete, and the drain comes before
      // this warp could need the MMA to have started tile j + NSR.
      while (nf < T && s >= kSlicesFlush * (nf + 1) + kGBufs && ok) flush_next(false);
      if (nf < T && s >= kSlicesFlush * (nf + 1) && tile_done(nf)) flush_next(false);  // early
      const int st = s % NST, gb = s % kGBufs;
      ok = ok && __all_sync(0xffffffffu, mbar_wait(FULL(st), (s / NST) & 1, kErrWaitFull));
      ok = ok && __all_sync(0xffffffffu, mbar_wait(GEMPTY(gb), ((s / kGBufs) & 1) ^ 1, kErrWaitGammaEmpty));
      if (!ok) break;
      tc_fence_after();
      const uint8_t *stg = smem + st * Sh::kStage;
      // this lane's component row of the L tile: 16 points = four 16-byte chunks, chunk c
      // stored at c ^ ((row >> 1) & 3) (SWIZZLE_64B)
      const float4 *Lrow = reinterpret_cast<const float4 *>(stg + Sh::kLOff + cl * 64);
      const int sw = (cl >> 1) & 3;
      const float4 *ln4 = reinterpret_cast<const float4 *>(stg + Sh::kNOff);
      const int64_t nb = (s0 + s) * kSlicePts;
      const int live = (N - nb < kSlicePts ? (int)(N - nb) : kSlicePts) - p0;
      float gh[8], gl[8];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const float4 l4 = ln4[p0 / 4 + c];
        const float4 v4 = Lrow[(p0 / 4 + c) ^ sw];
        const float ln2[4] = {l4.x, l4.y, l4.z, l4.w};
        const float lv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int p = c * 4 + e;
          const float g = p < live ? ex2(lv[e] - ln2[e]) : 0.0f;
          nk += g;
          gh[p] = to_tf32(g);
          gl[p] = to_tf32(g - gh[p]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(EMPTY(st));  // this warp is done with the slice's L
      const uint32_t ga = lane_tmem + kGBase + gb * kGCols + p0;
      tmem_st8(ga, gh);
      tmem_st8(ga + kSlicePts, gl);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(GFULL(gb));
    }
  } else if (warp == kGammaWarps) {
    // ---------------- MMA warp
    constexpr uint32_t idesc = idesc_tf32(NC, KA, 0, 1);  // A from TMEM, B MN-major
    const uint64_t fdesc0 = sdesc(smem_u32(smem), Sh::kAtom, 512, kSw128Base32);
    for (int s = 0; s < S && ok; ++s) {
      const int j = s / kSlicesFlush, reg = NSR == 2 ? (j & 1) : 0;
      const bool tile_first = s % kSlicesFlush == 0;
      if (tile_first && j >= NSR) {
        while (nf <= j - NSR && ok) flush_next(false);
        ok = ok && __all_sync(0xffffffffu, mbar_wait(SEMPTY(reg), ((j / NSR) & 1) ^ 1, kErrWaitStatsDone));
      }
      const int st = s % NST, gb = s % kGBufs;
      ok = ok && __all_sync(0xffffffffu, mbar_wait(FULL(st), (s / NST) & 1, kErrWaitFull));
      ok = ok && __all_sync(0xffffffffu, mbar_wait(GFULL(gb), (s / kGBufs) & 1, kErrWaitGammaFull));
      if (!ok) break;
      if (lane == 0) {
        tc_fence_after();
        const uint32_t gbuf = tmem + kGBase + gb * kGCols;
        const uint32_t dst = tmem + reg * KA;
        // the stage's descriptor; F lo and the second k-step are fixed address offsets
        const uint64_t fd = fdesc0 + (uint64_t)((st * Sh::kStage) >> 4);
        constexpr uint64_t kLo = Sh::kFPart >> 4, kK = 1024 >> 4;
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          mma_tf32_ta(dst, gbuf + kSlicePts + kk * 8, fd + kk * kK, idesc, (tile_first && kk == 0) ? 0u : 1u);
          mma_tf32_ta(dst, gbuf + kk * 8, fd + kLo + kk * kK, idesc, 1u);
        }
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) mma_tf32_ta(dst, gbuf + kk * 8, fd + kk * kK, idesc, 1u);
        mma_commit(EMPTY(st));
        mma_commit(GEMPTY(gb));
        if (s % kSlicesFlush == kSlicesFlush - 1 || s == S - 1) mma_commit(SFULL(reg));
      }
      __syncwarp();
    }
    if (lane == 0 && S > 0) {  // every MMA of this CTA has completed before the teardown
      mma_commit(DONE);
      mbar_wait_drain(DONE, 0);
    }
    __syncwarp();
  } else if (warp == kGammaWarps + 1) {
    // ---------------- producer warp
    if (lane == 0) {
      prefetch_tmap(&tm_fhi);
      prefetch_tmap(&tm_flo);
      prefetch_tmap(&tm_l);
    }
    // L is read exactly once
    const uint64_t pol_l = policy_evict_first();
    for (int s = 0; s < S && ok; ++s) {
      // same rule as the gamma warps, NST slices ahead (before the EMPTY wait below)
      while (nf < T && s >= kSlicesFlush * (nf + 1) + NST && ok) flush_next(false);
      if (nf < T && s >= kSlicesFlush * (nf + 1) && tile_done(nf)) flush_next(false);  // early
      const int st = s % NST;
      if (s >= NST) ok = ok && __all_sync(0xffffffffu, mbar_wait(EMPTY(st), ((s / NST) & 1) ^ 1, kErrWaitEmpty));
      if (!ok) break;
      if (lane == 0) {
        const uint32_t base = smem_u32(smem + st * Sh::kStage);
        const int64_t nb = (s0 + s) * kSlicePts;
        mbar_arrive_expect_tx(FULL(st), 2 * Sh::kFPart + kSlicePts * NC * 4 + kSlicePts * 4);
        tma_load_3d(base, &tm_fhi, 0, (int32_t)nb, 0, FULL(st));
        tma_load_3d(base + Sh::kFPart, &tm_flo, 0, (int32_t)nb, 0, FULL(st));
        tma_load_2d_hint(base + Sh::kLOff, &tm_l, (int32_t)nb, ct * NC, FULL(st), pol_l);
        bulk_load(base + Sh::kNOff, ln2x + nb, kSlicePts * 4, FULL(st));
      }
      __syncwarp();
    }
    // no copy may land after the CTA ends: the last NST slices' loads must be complete
    if (lane == 0)
      for (int s = (S > NST ? S - NST : 0); s < S; ++s) mbar_wait_drain(FULL(s % NST), (s / NST) & 1);
    __syncwarp();
  }
  // every warp drains the tiles it has not drained yet (the drain-only warps sleep between
  // polls)
  while (nf < T && ok) flush_next(warp > kGammaWarps + 1);

  ok = cta_sync_and(ok);
  const int k = ct * NC + cl;
  if (k < K) {
    float *dst = partial + ((int64_t)k * S_slots + slot) * PSTRIDE;
#pragma unroll
    for (int e = 0; e < SEG; e += 4) {
      const int f = seg * SEG + e;  // feature column: x^2 part first, then x
      float4 *o = reinterpret_cast<float4 *>(dst + (f < DP ? DP + f : f - DP));
      float4 v = ok ? make_float4(sacc[e], sacc[e + 1], sacc[e + 2], sacc[e + 3])
                    : make_float4(0.f, 0.f, 0.f, 0.f);
      if (accum) {  // a later chunk of the same iteration: this CTA slot's row adds up
        const float4 o0 = *o;
        v = make_float4(o0.x + v.x, o0.y + v.y, o0.z + v.z, o0.w + v.w);
      }
      *o = v;
    }
  }
  // n_k: the two gamma warps of a lane quarter add up their halves of the points
  float *nk_s = reinterpret_cast<float *>(smem);  // [128], the stage ring is idle now
  if (warp >= 4 && warp < kGammaWarps) nk_s[cl] = nk;
  __syncthreads();
  if (warp < 4 && k < K) {
    float *o = partial + ((int64_t)k * S_slots + slot) * PSTRIDE + 2 * DP;
    const float v = ok ? nk + nk_s[cl] : 0.0f;
    *o = accum ? *o + v : v;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------- host
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Row-major fp32 [rows][cols] matrix, box [box_rows][box_cols] with the given swizzle.
// Row-major fp32 [rows][cols] matrix (cols a multiple of 32) seen as 32-column atoms:
// box = 32 rows x all atoms, landing as [atom][row][32] with SWIZZLE_128B_ATOM_32B (the
// MN-major operand layout of the statistics GEMM).
int make_map_atoms(CUtensorMap *m, const float *base, int64_t rows, int cols, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(FGMM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)KC, (cuuint64_t)rows, (cuuint64_t)(cols / KC)};
  cuuint64_t strides[2] = {(cuuint64_t)cols * sizeof(float), (cuuint64_t)KC * sizeof(float)};
  cuuint32_t box[3] = {(cuuint32_t)KC, (cuuint32_t)box_rows, (cuuint32_t)(cols / KC)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FGMM_ERR_CUDA, "cuTensorMapEncodeTiled (atoms) failed: " + std::to_string((int)r));
  return FGMM_OK;
}

int make_map(CUtensorMap *m, const float *base, int64_t rows, int cols, int box_rows,
             CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B, int box_cols = KC) {
  auto fn = encode_fn();
  if (!fn) return fail(FGMM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * sizeof(float)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FGMM_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return FGMM_OK;
}

// The points are processed in chunks whose log2-likelihood block Lt [Kp][chunk] fits a
// fixed budget, so the workspace stays bounded for any N: pass 1 writes the block, the
// refine kernel patches it and the statistics kernel reads it back.  Chunks run in order
// on the stream; the per-slot statistics rows and the log-normalizer block sums add up
// across chunks.  The budget (256 MB, twice the L2) is set by the per-chunk cost of three
// launches and their pipeline fill and drain, which outweighs keeping the block
// L2-resident: against 64 MB, config 4 (K = 1024) runs 21 % and config 5 13 % faster;
// larger budgets measured no further change.
#ifndef FGMM_L_CHUNK_MB
#define FGMM_L_CHUNK_MB 256
#endif
constexpr int64_t kLChunkBytes = (int64_t)FGMM_L_CHUNK_MB << 20;

// Launch geometry of one chunk of Nc points.
struct TcChunk {
  int64_t Nc;
  int n_pt, G, tpg, S, grid1, grid2;
};

struct TcPlan {
  int64_t N, Nc;  // all points; points per chunk (a multiple of 128, the last may be short)
  int d, dp, KA, nkc, K, Kp, n_ct, chunks;
  TcChunk first;
};

TcChunk chunk_plan(int64_t Nc, int n_ct) {
  TcChunk c{};
  c.Nc = Nc;
  c.n_pt = (int)cdiv(Nc, BM);
  const int sms = num_sms();
  const int G = (int)std::min<int64_t>(n_ct, std::max<int64_t>(1, cdiv(4 * sms, c.n_pt)));
  c.tpg = (int)cdiv(n_ct, G);
  c.G = (int)cdiv(n_ct, c.tpg);
  c.grid1 = (int)std::min<int64_t>((int64_t)c.n_pt * c.G, sms);
  c.S = (int)std::max<int64_t>(1, std::min<int64_t>(sms / std::max(1, n_ct), cdiv(Nc, 32)));
  c.grid2 = n_ct * c.S;
  return c;
}

TcPlan plan(int64_t N, int d, int K) {
  TcPlan p{};
  p.N = N; p.d = d; p.K = K;
  p.dp = dp_of(d);
  p.KA = 2 * p.dp;
  p.nkc = p.KA / KC;
  p.n_ct = (int)cdiv(K, NC);
  p.Kp = p.n_ct * NC;
  const int64_t fit = std::max<int64_t>(BM, kLChunkBytes / ((int64_t)p.Kp * 4) / BM * BM);
  p.Nc = std::min<int64_t>(npad_of(N), fit);
  p.chunks = (int)cdiv(N, p.Nc);
  p.first = chunk_plan(std::min<int64_t>(N, p.Nc), p.n_ct);
  return p;
}

struct TcWs {
  float *qhi, *qlo, *cst2, *sc, *ms, *lc, *part_m, *part_s, *ln2x, *partial, *L;
  float2 *part_tv;
  int2 *part_ti;
  double *ln_part;
  size_t bytes;
};

constexpr int kRefineBlocks = 8192;  // 32 points per block
inline int refine_blocks(int64_t N) { return (int)std::min<int64_t>(kRefineBlocks, cdiv(N, 32)); }

// Per-chunk buffers are sized for the first (largest) chunk; the component-group
// partials for n_ct groups, the most any chunk uses.
TcWs tc_layout(void *ws, const TcPlan &p) {
  TcWs w{};
  Carve c(ws);
  const int64_t Nc = p.first.Nc;
  w.qhi = c.take<float>((size_t)p.Kp * p.KA);
  w.qlo = c.take<float>((size_t)p.Kp * p.KA);
  w.cst2 = c.take<float>(p.Kp);
  w.sc = c.take<float>((size_t)p.K * p.d);
  w.ms = c.take<float>((size_t)p.K * p.d);
  w.lc = c.take<float>(p.K);
  w.part_m = c.take<float>((size_t)p.n_ct * Nc);
  w.part_s = c.take<float>((size_t)p.n_ct * Nc);
  w.part_tv = c.take<float2>((size_t)p.n_ct * Nc);
  w.part_ti = c.take<int2>((size_t)p.n_ct * Nc);
  w.ln2x = c.take<float>(npad_of(Nc));
  w.partial = c.take<float>((size_t)p.first.S * p.K * (2 * p.dp + 4));
  w.ln_part = c.take<double>(kRefineBlocks);
  w.L = c.take<float>((size_t)npad_of(Nc) * p.Kp);  // Lt [Kp][chunk]
  w.bytes = c.bytes();
  return w;
}

size_t smem1_bytes() { return 1024 + kStages1 * kStageBytes + 256 + (kParts - 1) * BM * 24; }
size_t smem2_bytes(int KA) {
  switch (KA) {
    case 64: return StatsShape<64>::kSmem;
    case 128: return StatsShape<128>::kSmem;
    case 192: return StatsShape<192>::kSmem;
    default: return StatsShape<256>::kSmem;
  }
}

// Pass 1, refine and statistics for the chunk of points [n0, n0 + c.Nc).
template <int NKC>
int tc_launch_chunk(const TcPlan &p, const TcChunk &c, int64_t n0, bool first, const float *X,
                    const float *pts, const TcWs &w, float *ln, cudaStream_t st) {
  const float *phi = pts + n0 * p.KA;
  const float *plo = pts + points_half_floats(p.N, p.d) + n0 * p.KA;
  const int64_t rows = npad_of(c.Nc);
  const int64_t lcols = npad_of(c.Nc);
  const float *Xc = X + n0 * p.d;
  CUtensorMap m_phi, m_plo, m_qhi, m_qlo;
  int rc;
  if ((rc = make_map(&m_phi, phi, rows, p.KA, BM))) return rc;
  if ((rc = make_map(&m_plo, plo, rows, p.KA, BM))) return rc;
  if ((rc = make_map(&m_qhi, w.qhi, p.Kp, p.KA, NC))) return rc;
  if ((rc = make_map(&m_qlo, w.qlo, p.Kp, p.KA, NC))) return rc;
  FGMM_CUDA_TRY(launch_pdl(tc_pass1_kernel<NKC>, c.grid1, kThreads, smem1_bytes(), st, m_phi, m_plo,
                           m_qhi, m_qlo, w.cst2, c.Nc, c.n_pt, p.n_ct, c.G, c.tpg, w.part_m,
                           w.part_s, w.part_tv, w.part_ti, w.L, lcols));
  mark(st, "tc_pass1_kernel");
  {
    const int blocks = refine_blocks(c.Nc);
    const int dpl = (p.d + 7) / 8;
    const bool vec = p.d % 32 == 0 && reinterpret_cast<uintptr_t>(Xc) % 16 == 0;  // d = 8 DPL
    const int acc = first ? 0 : 1;
#define FGMM_REFINE(D)                                                                             \
  do {                                                                                             \
    if (vec && (D) % 4 == 0 && 8 * (D) == p.d)                                                     \
      FGMM_CUDA_TRY(launch_pdl(tc_refine_kernel<D, true>, blocks, 256, 0, st, Xc, c.Nc, p.d, w.sc, \
                               w.ms, w.lc, w.part_m, w.part_s, w.part_tv, w.part_ti, c.G, w.ln2x,  \
                               w.L, lcols, ln + n0, w.ln_part, acc));                              \
    else                                                                                           \
      FGMM_CUDA_TRY(launch_pdl(tc_refine_kernel<D, false>, blocks, 256, 0, st, Xc, c.Nc, p.d, w.sc,\
                               w.ms, w.lc, w.part_m, w.part_s, w.part_tv, w.part_ti, c.G, w.ln2x,  \
                               w.L, lcols, ln + n0, w.ln_part, acc));                              \
  } while (0)
    if (dpl <= 1) FGMM_REFINE(1);
    else if (dpl <= 2) FGMM_REFINE(2);
    else if (dpl <= 4) FGMM_REFINE(4);
    else if (dpl <= 8) FGMM_REFINE(8);
    else if (dpl <= 12) FGMM_REFINE(12);
    else FGMM_REFINE(16);
#undef FGMM_REFINE
    FGMM_LAUNCH_CHECK("tc_refine_kernel");
    mark(st, "tc_refine_kernel");
  }
  CUtensorMap m_fhi, m_flo, m_l;
  if ((rc = make_map_atoms(&m_fhi, phi, rows, p.KA, kSlicePts))) return rc;
  if ((rc = make_map_atoms(&m_flo, plo, rows, p.KA, kSlicePts))) return rc;
  if ((rc = make_map(&m_l, w.L, p.Kp, (int)lcols, NC, CU_TENSOR_MAP_SWIZZLE_64B, kSlicePts))) return rc;
  FGMM_CUDA_TRY(launch_pdl(tc_stats_kernel<NKC>, c.grid2, kThreads2, smem2_bytes(NKC * KC), st,
                           m_fhi, m_flo, m_l, w.ln2x, c.Nc, c.S, p.K, w.partial, first ? 0 : 1));
  mark(st, "tc_stats_kernel");
  return FGMM_OK;
}

template <int NKC>
int tc_launch(const TcPlan &p, const float *X, const float *pts, const TcWs &w, float *ln,
              cudaStream_t st) {
  std::atomic<bool> &done = device_once_flag(8 + NKC / 2);
  if (!done) {
    FGMM_CUDA_TRY(cudaFuncSetAttribute(tc_pass1_kernel<NKC>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1_bytes()));
    FGMM_CUDA_TRY(cudaFuncSetAttribute(tc_stats_kernel<NKC>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2_bytes(NKC * KC)));
    done = true;
  }
  for (int i = 0; i < p.chunks; ++i) {
    const int64_t n0 = (int64_t)i * p.Nc;
    const int64_t nc = std::min<int64_t>(p.Nc, p.N - n0);
    const TcChunk c = nc == p.first.Nc ? p.first : chunk_plan(nc, p.n_ct);
    const int rc = tc_launch_chunk<NKC>(p, c, n0, i == 0, X, pts, w, ln, st);
    if (rc) return rc;
  }
  return FGMM_OK;
}

}  // namespace

int tc_launches(int64_t N, int d, int K) { return 2 + 3 * plan(N, d, K).chunks; }

bool tc_supported(int64_t N, int d, int K) { return N >= 1 && K >= 1 && d >= 1 && d <= kMaxDp; }

size_t tc_points_bytes(int64_t N, int d) { return points_half_floats(N, d) * sizeof(float) * 2; }

size_t tc_workspace_bytes(int64_t N, int d, int K) { return tc_layout(nullptr, plan(N, d, K)).bytes; }

int tc_prepare_points(const float *X, int64_t N, int d, void *points, cudaStream_t st) {
  const int dp = dp_of(d);
  float *phi = static_cast<float *>(points);
  float *plo = phi + points_half_floats(N, d);
  const int64_t total = npad_of(N) * dp;
  const int blocks = (int)std::min<int64_t>(cdiv(total, 256), 16 * num_sms());
  tc_prep_points_kernel<<<blocks, 256, 0, st>>>(X, N, npad_of(N), d, dp, phi, plo);
  FGMM_LAUNCH_CHECK("tc_prep_points_kernel");
  return FGMM_OK;
}

int tc_em_stats(const float *X, const void *points, int64_t N, int d, const float *mu,
                const float *var, const float *log_pi, int K, double *stats, float *log_norm,
                void *ws, cudaStream_t st, const UpdateOut *update, bool prepared) {
  const TcPlan p = plan(N, d, K);
  const TcWs w = tc_layout(ws, p);
  // `prepared`: the workspace already holds the operands of (mu, var, log_pi), written by
  // the previous call's fused update
  if (!prepared) {
    FGMM_CUDA_TRY(launch_pdl(tc_prep_params_kernel, p.Kp, 128, 0, st, mu, var, log_pi, K, d, p.dp,
                             w.qhi, w.qlo, w.cst2, w.sc, w.ms, w.lc));
    mark(st, "tc_prep_params_kernel");
  }
  UpdateOut up{};
  if (update) {  // the update also prepares the next iteration's operands
    up = *update;
    up.qhi = w.qhi; up.qlo = w.qlo; up.cst2 = w.cst2; up.sc = w.sc; up.ms = w.ms; up.lc = w.lc;
    up.dp = p.dp;
  }
  const float *pts = static_cast<const float *>(points);
  int rc;
  switch (p.nkc) {
    case 2: rc = tc_launch<2>(p, X, pts, w, log_norm, st); break;
    case 4: rc = tc_launch<4>(p, X, pts, w, log_norm, st); break;
    case 6: rc = tc_launch<6>(p, X, pts, w, log_norm, st); break;
    case 8: rc = tc_launch<8>(p, X, pts, w, log_norm, st); break;
    default: return fail(FGMM_ERR_UNSUPPORTED, "tcgen05 family: d > 128");
  }
  if (rc) return rc;
  return reduce_partials(w.partial, p.first.S, K, d, p.dp, 2 * p.dp + 4, w.ln_part,
                         refine_blocks(p.first.Nc), stats, st, update ? &up : nullptr);
}

int tc_device_error(bool reset) {
  int v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    int z = 0;
    cudaMemcpyToSymbol(g_dev_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace fgmm
