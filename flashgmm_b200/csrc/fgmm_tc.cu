// tcgen05 tensor-core family of the fused EM statistics kernels (sm_100a).
//
// Per iteration, over chunks of points:
//   tc_pass1_kernel   distance GEMM D = P Q^T (kind::f16, fp16 hi/lo operands, the
//                     per-dimension [x^2, x, 1] . [iv, -2 mu iv, mu^2 iv] layout of
//                     fgmm_tcops.cuh), the online log-sum-exp of
//                     flash_gmm/csrc/flash_gmm_cuda.cu:145-155 in base 2, the four
//                     leading components of every point, and the log2-likelihood block
//                     Lt [component][point] that the statistics pass reads;
//   tc_refine_kernel  merges the component groups, re-evaluates the leading components
//                     exactly in the reference's direct form, writes the log-normalizer;
//   tc_stats_kernel   S[k, f] = sum_n gamma[n, k] F[n, f], F = [x^2 | x] (kind::f16,
//                     gamma from tensor memory), one partial row per (component, CTA).
// (Reference: flash_log_normalizer_v2_kernel and flash_accumulate_stats_v2_kernel,
// flash_gmm/csrc/flash_gmm_cuda.cu:72-292, and the direct form of
// flash_gmm/csrc/flash_gmm_cpu.cpp:30-45.)  No cluster multicast anywhere.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <algorithm>
#include <atomic>
#include <cmath>
#include <mutex>

#include "fgmm_common.cuh"
#include "sm100_ptx.cuh"

namespace fgmm {
using namespace ptx;

namespace {

constexpr int BM = 128;                        // points per pass-1 tile (MMA M)
constexpr int KCH = 64;                        // fp16 K elements per staged chunk (128-byte rows)
constexpr int kEpiWarps = 16;                  // four warps per TMEM lane quarter
constexpr int kThreads1 = 64 + 32 * kEpiWarps; // warp 0 TMA, warp 1 MMA, warps 2.. epilogue
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kMaxD = 128;                     // d <= 128 runs here
// Leading components more than kNear below a point's largest base-2 log-likelihood have
// responsibilities below 2^-kNear relative to the leader and are not re-evaluated.
constexpr float kNear = 32.0f;

inline int64_t npad_of(int64_t N) { return cdiv(N, BM) * BM; }

// Layout shared by pass 1 and the statistics pass: the statistics CTAs own 128 components
// each and take points in slices of 32; bit p of word
// xmask[(tile * n_slices + slice) * 128 + c] is set when component c of the tile is one of
// the exactly evaluated leading components of point p of the slice.
constexpr int NC2_ref = 128;
constexpr int kSlice_ref = 32;

// Prepared points: header (column exponents, max |x|), then P hi / lo [Npad][KBp] and
// F hi / lo [Npad][KA], fp16.  Rows >= N are zero, so no TMA box leaves the tensor.
inline size_t p_elems(int64_t N, int d) { return align_up((size_t)npad_of(N) * tc_kbp(d), 128); }
inline size_t f_elems(int64_t N, int d) { return align_up((size_t)npad_of(N) * 2 * tc_dp(d), 128); }
struct PtsPtrs {
  const int *aexp;
  uint32_t *xmax;
  __half *phi, *plo, *fhi, *flo;
};
inline PtsPtrs pts_ptrs(const void *pts, int64_t N, int d) {
  char *b = static_cast<char *>(const_cast<void *>(pts));
  PtsPtrs p;
  p.aexp = reinterpret_cast<const int *>(b + kPtsAexpOff);
  p.xmax = reinterpret_cast<uint32_t *>(b + kPtsXmaxOff);
  p.phi = reinterpret_cast<__half *>(b + kPtsHeader);
  p.plo = p.phi + p_elems(N, d);
  p.fhi = p.plo + p_elems(N, d);
  p.flo = p.fhi + f_elems(N, d);
  return p;
}

__device__ __forceinline__ uint8_t *align1024(uint8_t *p) {
  uintptr_t a = reinterpret_cast<uintptr_t>(p);
  return reinterpret_cast<uint8_t *>((a + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ void split_f16f(float v, __half &hi, __half &lo) {
  hi = __float2half_rn(v);
  lo = __float2half_rn(v - __half2float(hi));
}

// --------------------------------------------------------------------------- prep
// max |x_j| over the points.  A block takes a contiguous row range; thread t owns
// dimension t % d of rows t / d, t / d + R, ... (R = blockDim / d rows per pass), four
// loads in flight; the block's maxima meet in shared memory before one global atomic per
// dimension.
__global__ void __launch_bounds__(256) tc_xmax_kernel(const float *__restrict__ X, int64_t N, int d,
                                                      int64_t rows_per_block, uint32_t *__restrict__ xmax) {
  __shared__ uint32_t s_max[kMaxD];
  for (int j = threadIdx.x; j < d; j += blockDim.x) s_max[j] = 0u;
  __syncthreads();
  const int R = blockDim.x / d;
  const int j = threadIdx.x % d, r = threadIdx.x / d;
  const int64_t n0 = (int64_t)blockIdx.x * rows_per_block;
  const int64_t n1 = n0 + rows_per_block < N ? n0 + rows_per_block : N;
  if (r < R) {
    float m[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int64_t n = n0 + r;
    for (; n + 3 * R < n1; n += 4 * R) {
#pragma unroll
      for (int u = 0; u < 4; ++u) m[u] = fmaxf(m[u], fabsf(__ldg(X + (n + u * R) * d + j)));
    }
    for (; n < n1; n += R) m[0] = fmaxf(m[0], fabsf(__ldg(X + n * d + j)));
    // non-negative floats order like their bit patterns
    atomicMax(s_max + j, __float_as_uint(fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]))));
  }
  __syncthreads();
  for (int c = threadIdx.x; c < d; c += blockDim.x) atomicMax(xmax + c, s_max[c]);
}

// P[n][c] (c = 3 j + t: x^2, x, 1) and F[n][f] (f < dp: x^2, else x), scaled by the
// column exponents and split into fp16 hi / lo; block 0 also records the exponents of P.
// A block stages kPrepRows rows of X in shared memory, next to a per-column table (source
// dimension and kind, and the exact power of two 2^a_c: the product rounds exactly as
// ldexpf does), and writes four columns per thread as 8-byte stores.  Rows >= N and
// columns past the data are zero.
constexpr int kPrepRows = 16;  // divides the 128-row padding of Npad
__host__ __device__ inline int tc_prep_smem(int kbp, int ka, int d) {
  return (kbp + ka) * 8 + kPrepRows * d * 4;
}
__global__ void __launch_bounds__(256) tc_prep_points_kernel(const float *__restrict__ X, int64_t N, int64_t Npad, int d,
                                      int kbp, int ka, const uint32_t *__restrict__ xmax,
                                      int *__restrict__ aexp, __half *__restrict__ phi,
                                      __half *__restrict__ plo, __half *__restrict__ fhi,
                                      __half *__restrict__ flo) {
  extern __shared__ __align__(16) uint8_t prep_smem[];
  const int W = kbp + ka, dp = ka / 2, Q = W / 4;  // columns, quads of columns per row
  int *s_code = reinterpret_cast<int *>(prep_smem);            // j << 2 | t (t = 3: zero column)
  float *s_scale = reinterpret_cast<float *>(prep_smem) + W;   // 2^a_c
  float *xs = reinterpret_cast<float *>(prep_smem) + 2 * W;    // [kPrepRows][d]
  for (int c = threadIdx.x; c < W; c += blockDim.x) {
    int j, t;
    if (c < kbp) { j = c / 3; t = c - 3 * j; }
    else { const int f = c - kbp; t = f < dp ? 0 : 1; j = t == 0 ? f : f - dp; }
    const bool in = j < d;
    const int a = in ? tc_p_col_exp(3 * j + t, d, xmax) : 0;  // |a| <= 100
    s_code[c] = in ? (j << 2 | t) : 3;
    s_scale[c] = __int_as_float((a + 127) << 23);
    if (blockIdx.x == 0 && c < kbp) aexp[c] = a;
  }
  const int64_t nd = N * (int64_t)d;
  for (int64_t r0 = (int64_t)blockIdx.x * kPrepRows; r0 < Npad; r0 += (int64_t)gridDim.x * kPrepRows) {
    __syncthreads();  // the table is written / the previous rows are consumed
    for (int i = threadIdx.x; i < kPrepRows * d; i += blockDim.x) {
      const int64_t g = r0 * d + i;
      xs[i] = g < nd ? __ldg(X + g) : 0.0f;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kPrepRows * Q; i += blockDim.x) {
      const int r = i / Q, c = 4 * (i - r * Q);
      const int64_t n = r0 + r;
      const bool live = n < N;
      __half h[4], l[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int code = s_code[c + u], t = code & 3;
        const float x = xs[r * d + (code >> 2)];
        float v = t == 0 ? x * x : (t == 1 ? x : (t == 2 ? 1.0f : 0.0f));
        v = live ? v * s_scale[c + u] : 0.0f;
        split_f16f(v, h[u], l[u]);
      }
      uint2 hv, lv;
      hv.x = (uint32_t)__half_as_ushort(h[0]) | ((uint32_t)__half_as_ushort(h[1]) << 16);
      hv.y = (uint32_t)__half_as_ushort(h[2]) | ((uint32_t)__half_as_ushort(h[3]) << 16);
      lv.x = (uint32_t)__half_as_ushort(l[0]) | ((uint32_t)__half_as_ushort(l[1]) << 16);
      lv.y = (uint32_t)__half_as_ushort(l[2]) | ((uint32_t)__half_as_ushort(l[3]) << 16);
      if (c < kbp) {
        *reinterpret_cast<uint2 *>(phi + n * kbp + c) = hv;
        *reinterpret_cast<uint2 *>(plo + n * kbp + c) = lv;
      } else {
        *reinterpret_cast<uint2 *>(fhi + n * ka + (c - kbp)) = hv;
        *reinterpret_cast<uint2 *>(flo + n * ka + (c - kbp)) = lv;
      }
    }
  }
}

// The same operands for d a multiple of 64 (3 d = KBp and d = dp: no padding columns) and
// 16-byte aligned rows.  Thread t owns the dimension quad q = t % (d / 4) of rows
// t / (d / 4), + 256 / (d / 4), ...: its twelve P columns 12 q .. 12 q + 11 and its eight F
// columns keep their scales in registers, x comes as one float4, and the outputs leave as
// 8-byte stores.  Values and rounding are those of tc_prep_points_kernel.
__global__ void __launch_bounds__(256) tc_prep_points_q_kernel(const float *__restrict__ X, int64_t N, int64_t Npad, int d,
                                        const uint32_t *__restrict__ xmax, int *__restrict__ aexp,
                                        __half *__restrict__ phi, __half *__restrict__ plo,
                                        __half *__restrict__ fhi, __half *__restrict__ flo) {
  const int nq = d / 4, rpp = blockDim.x / nq;  // quads per row, rows per pass
  const int q = threadIdx.x % nq, r = threadIdx.x / nq;
  const int kbp = 3 * d, ka = 2 * d;
  float sp[12], sf[8];  // 2^a of P columns 12 q + i and of F columns (x^2 of 4 q + i, then x)
#pragma unroll
  for (int i = 0; i < 12; ++i) {
    const int a = tc_p_col_exp(12 * q + i, d, xmax);
    sp[i] = __int_as_float((a + 127) << 23);
    if (blockIdx.x == 0 && r == 0) aexp[12 * q + i] = a;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    sf[i] = sp[3 * i];          // x^2 of dimension 4 q + i
    sf[4 + i] = sp[3 * i + 1];  // x
  }
  if (r >= rpp) return;
  for (int64_t n = (int64_t)blockIdx.x * rpp + r; n < Npad; n += (int64_t)gridDim.x * rpp) {
    const bool live = n < N;
    float4 x4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live) x4 = __ldg(reinterpret_cast<const float4 *>(X + n * d) + q);
    const float xs[4] = {x4.x, x4.y, x4.z, x4.w};
    __half h[20], l[20];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float x = xs[i];
      split_f16f(x * x * sp[3 * i], h[3 * i], l[3 * i]);
      split_f16f(x * sp[3 * i + 1], h[3 * i + 1], l[3 * i + 1]);
      split_f16f(live ? sp[3 * i + 2] : 0.0f, h[3 * i + 2], l[3 * i + 2]);
      split_f16f(x * x * sf[i], h[12 + i], l[12 + i]);
      split_f16f(x * sf[4 + i], h[16 + i], l[16 + i]);
    }
    auto pack = [](const __half *v) {
      uint2 u;
      u.x = (uint32_t)__half_as_ushort(v[0]) | ((uint32_t)__half_as_ushort(v[1]) << 16);
      u.y = (uint32_t)__half_as_ushort(v[2]) | ((uint32_t)__half_as_ushort(v[3]) << 16);
      return u;
    };
    uint2 *ph = reinterpret_cast<uint2 *>(phi + n * kbp + 12 * q);
    uint2 *pl = reinterpret_cast<uint2 *>(plo + n * kbp + 12 * q);
#pragma unroll
    for (int i = 0; i < 3; ++i) { ph[i] = pack(h + 4 * i); pl[i] = pack(l + 4 * i); }
    *reinterpret_cast<uint2 *>(fhi + n * ka + 4 * q) = pack(h + 12);
    *reinterpret_cast<uint2 *>(flo + n * ka + 4 * q) = pack(l + 12);
    *reinterpret_cast<uint2 *>(fhi + n * ka + d + 4 * q) = pack(h + 16);
    *reinterpret_cast<uint2 *>(flo + n * ka + d + 4 * q) = pack(l + 16);
  }
}

// One block of 128 threads per component (rows k >= K are padding: zero operands,
// cst2 = -inf, so they never receive responsibility).
__global__ void __launch_bounds__(128)
tc_prep_params_kernel(const float *__restrict__ mu, const float *__restrict__ var,
                      const float *__restrict__ log_pi, int K, int d, TcParamOps op) {
  griddep_launch();
  griddep_wait();
  const int k = blockIdx.x, j = threadIdx.x;
  const bool live = k < K && j < d;
  const float m32 = live ? mu[(int64_t)k * d + j] : 0.0f;
  const float v32 = live ? var[(int64_t)k * d + j] : 1.0f;
  const float lp = k < K ? log_pi[k] : 0.0f;
  tc_prep_component(k, K, d, j, m32, v32, lp, op, 1);
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

// Pushes (x, ix) into (tv, ti), the four largest values seen in descending order (ties:
// first seen), and returns in (dv, di) the one of the five that drops out (di = -1 for
// an empty slot, whose value is -inf).
__device__ __forceinline__ void top_push(float (&tv)[kTcTop], int (&ti)[kTcTop], float x, int ix,
                                         float &dv, int &di) {
  if (!(x > tv[3])) { dv = x; di = ix; return; }
  dv = tv[3]; di = ti[3];
  if (x > tv[1]) {
    tv[3] = tv[2]; ti[3] = ti[2];
    tv[2] = tv[1]; ti[2] = ti[1];
    if (x > tv[0]) { tv[1] = tv[0]; ti[1] = ti[0]; tv[0] = x; ti[0] = ix; }
    else           { tv[1] = x; ti[1] = ix; }
  } else if (x > tv[2]) {
    tv[3] = tv[2]; ti[3] = ti[2]; tv[2] = x; ti[2] = ix;
  } else {
    tv[3] = x; ti[3] = ix;
  }
}

// Adds 2^v to the base-2 log-sum-exp state (m, s) = 2^m s.
__device__ __forceinline__ void lse_add(float &m, float &s, float v) {
  const float mn = fmaxf(m, v);
  const float r = mn == -INFINITY ? 0.0f : mn;
  s = s * ex2(m - r) + ex2(v - r);
  m = mn;
}

// Merges (m2, s2) into (m, s).
__device__ __forceinline__ void lse_merge(float &m, float &s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  const float r = mn == -INFINITY ? 0.0f : mn;
  s = s * ex2(m - r) + s2 * ex2(m2 - r);
  m = mn;
}

// A point's running summary over the components seen so far: the four largest
// log2-likelihoods with their components, and the base-2 log-sum-exp (m, s) of all the
// others.  Keeping the two apart (every value that leaves the four joins the rest) lets
// the refinement replace the four by exactly evaluated values without subtracting them
// from a total, which loses everything when an approximate leader was far too large.
__device__ __forceinline__ void summary_push(float (&tv)[kTcTop], int (&ti)[kTcTop], float &m, float &s,
                                             float x, int ix) {
  float dv;
  int di;
  top_push(tv, ti, x, ix, dv, di);
  if (di >= 0) lse_add(m, s, dv);
}

// ------------------------------------------------------------------------- pass 1
// Persistent CTAs over (point tile, component group) units; a group is `tpg` component
// tiles of NC.  Per tile the MMA thread accumulates all NKC chunks into one TMEM buffer
// (two buffers, so the next tile's MMAs run while the epilogue drains this one):
// per chunk four k-steps of lo.hi and hi.lo, then four of hi.hi (small products first).
// Epilogue warp w owns TMEM lane quarter w % 4 (32 points) and a quarter of the tile's
// columns; it turns accumulators into log2-likelihoods l2 = cst2 + coef D, stores them
// into Lt (transposed, evict_last: the statistics pass reads them back), and keeps per
// point a summary: the four largest l2 within 2^-kNear of the point's running maximum,
// with their components, and the log-sum-exp of the rest.
template <int NKC, int NC>
struct Pass1Shape {
  static constexpr int S = NC == 256 ? 2 : 3;             // stages
  static constexpr int kPBytes = BM * 128;                 // P tile of one chunk (hi or lo)
  static constexpr int kQBytes = NC * 128;                 // Q tile of one chunk (hi or lo)
  static constexpr int kStage = 2 * kPBytes + 2 * kQBytes;
  static constexpr int kCols = NC / 4;                     // columns per epilogue warp
  struct Part { float m, s; float v[kTcTop]; int i[kTcTop]; };
  static constexpr int kBarOff = S * kStage;
  static constexpr int kXOff = kBarOff + 8 * (2 * S + 5) + 8;
  static constexpr int kSmem = 1024 + kXOff + 3 * BM * (int)sizeof(Part);
};

template <int NKC, int NC>
__global__ void __launch_bounds__(kThreads1, 1)
tc_pass1_kernel(const __grid_constant__ CUtensorMap tm_phi, const __grid_constant__ CUtensorMap tm_plo,
                const __grid_constant__ CUtensorMap tm_qhi, const __grid_constant__ CUtensorMap tm_qlo,
                const float *__restrict__ coef, const float *__restrict__ cst2, int64_t N, int n_pt,
                int n_ct, int G, int tpg, float *__restrict__ part_m, float *__restrict__ part_s,
                float4 *__restrict__ part_tv, int4 *__restrict__ part_ti, float *__restrict__ Lt,
                int64_t Npad, uint32_t *__restrict__ xmask, int64_t xmask_words) {
  using Sh = Pass1Shape<NKC, NC>;
  constexpr int S = Sh::S;
  using Part = typename Sh::Part;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Sh::kBarOff);
  // bars: full[S] empty[S] tfull[2] tempty[2] done
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * S + 5);
  Part *lse_x = reinterpret_cast<Part *>(smem + Sh::kXOff);  // [3][128] row exchange
  const uint32_t bar0 = smem_u32(bars);
  auto FULL = [&](int s) { return bar0 + 8u * s; };
  auto EMPTY = [&](int s) { return bar0 + 8u * (S + s); };
  const uint32_t TFULL0 = bar0 + 8u * (2 * S), TEMPTY0 = bar0 + 8u * (2 * S + 2);
  const uint32_t DONE = bar0 + 8u * (2 * S + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(FULL(s), 1); mbar_init(EMPTY(s), 1); }
    for (int b = 0; b < 2; ++b) {
      mbar_init(TFULL0 + 8u * b, 1);
      mbar_init(TEMPTY0 + 8u * b, kEpiWarps);
    }
    mbar_init(DONE, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 2 * NC);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  griddep_launch();
  // The prepared points do not change between launches: the producer starts loading the
  // first unit's point tiles before waiting for the earlier launches (which write the
  // parameter operands, Lt's readers and the bit words); every other thread waits first.
  const int n_units = n_pt * G;
  const int npre = (warp == 0 && lane == 0 && (int)blockIdx.x < n_units) ? min(S, NKC) : 0;
  if (npre > 0) {
    const int pt0 = blockIdx.x / G;
    for (int c = 0; c < npre; ++c) {
      const uint32_t base = smem_u32(smem + c * Sh::kStage);
      mbar_arrive_expect_tx(FULL(c), Sh::kStage);
      tma_load_2d_hint(base, &tm_phi, c * KCH, pt0 * BM, FULL(c), policy_evict_first());
      tma_load_2d_hint(base + Sh::kPBytes, &tm_plo, c * KCH, pt0 * BM, FULL(c), policy_evict_first());
    }
  }
  griddep_wait();  // the parameter operands and Lt of earlier launches
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane != 0) {  // the idle lanes clear the exact-component words the refinement sets
      for (int64_t i = (int64_t)blockIdx.x * 31 + lane - 1; i < xmask_words; i += (int64_t)gridDim.x * 31)
        xmask[i] = 0u;
    } else {
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
            const uint32_t base = smem_u32(smem + stage * Sh::kStage);
            const bool pre = u == (int)blockIdx.x && t == g * tpg && c < npre;  // P already on its way
            if (!pre) {
              mbar_arrive_expect_tx(FULL(stage), Sh::kStage);
              tma_load_2d_hint(base, &tm_phi, c * KCH, pt * BM, FULL(stage), pol_p);
              tma_load_2d_hint(base + Sh::kPBytes, &tm_plo, c * KCH, pt * BM, FULL(stage), pol_p);
            }
            tma_load_2d_hint(base + 2 * Sh::kPBytes, &tm_qhi, c * KCH, t * NC, FULL(stage), pol_q);
            tma_load_2d_hint(base + 2 * Sh::kPBytes + Sh::kQBytes, &tm_qlo, c * KCH, t * NC,
                             FULL(stage), pol_q);
            armed |= 1u << stage;
            armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
            if (++stage == S) { stage = 0; phase ^= 1; }
          }
        }
      }
      // never leave the CTA with bulk copies in flight
      for (int s = 0; s < S; ++s)
        if (armed & (1u << s)) mbar_wait_drain(FULL(s), (armed_par >> s) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(BM, NC, 0, 0);
      constexpr uint64_t kPl = Sh::kPBytes >> 4, kQh = (2 * Sh::kPBytes) >> 4,
                         kQl = (2 * Sh::kPBytes + Sh::kQBytes) >> 4;
      const uint64_t desc0 = sdesc_sw128(smem_u32(smem), 16, 1024);
      int stage = 0;
      uint32_t phase = 0, tcount = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const int g = u % G;
        const int t1 = min(n_ct, (g + 1) * tpg);
        for (int t = g * tpg; t < t1 && ok; ++t) {
          const uint32_t buf = tcount & 1u, use = tcount >> 1;
          if (!mbar_wait(TEMPTY0 + 8u * buf, (use & 1u) ^ 1u, kErrWaitTmemEmpty)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d = tmem + buf * NC;
          for (int c = 0; c < NKC; ++c) {
            if (!mbar_wait(FULL(stage), phase, kErrWaitFull)) { ok = false; break; }
            tc_fence_after();
            const uint64_t ds = desc0 + (uint64_t)((stage * Sh::kStage) >> 4);
#pragma unroll
            for (int kk = 0; kk < KCH / 16; ++kk) {  // k-step kk: +32 bytes = +2
              mma_f16(d, ds + kPl + 2 * kk, ds + kQh + 2 * kk, idesc, (c != 0 || kk != 0) ? 1u : 0u);
              mma_f16(d, ds + 2 * kk, ds + kQl + 2 * kk, idesc, 1u);
            }
#pragma unroll
            for (int kk = 0; kk < KCH / 16; ++kk) mma_f16(d, ds + 2 * kk, ds + kQh + 2 * kk, idesc, 1u);
            mma_commit(EMPTY(stage));
            if (++stage == S) { stage = 0; phase ^= 1; }
          }
          if (!ok) break;
          mma_commit(TFULL0 + 8u * buf);
          ++tcount;
        }
      }
      mma_commit(DONE);
      mbar_wait_drain(DONE, 0);
    }
    __syncwarp();
  } else {
    constexpr int kC = Sh::kCols;
    const int q = warp & 3, part = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const uint64_t pol_l = policy_evict_last();
    const uint32_t lane_tmem = tmem + ((uint32_t)(q * 32) << 16) + part * kC;
    uint32_t tcount = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
      const int pt = u / G, g = u % G;
      const int t1 = min(n_ct, (g + 1) * tpg);
      const int64_t n_row = (int64_t)pt * BM + row;
      float m = -INFINITY, s = 0.0f;
      float tv[kTcTop] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      int ti[kTcTop] = {-1, -1, -1, -1};
      for (int t = g * tpg; t < t1 && ok; ++t) {
        const uint32_t buf = tcount & 1u, use = tcount >> 1;
        ok = __all_sync(0xffffffffu, mbar_wait(TFULL0 + 8u * buf, use & 1u, kErrWaitTmemFull));
        if (!ok) break;
        tc_fence_after();
        const int kb = t * NC + part * kC;
#pragma unroll 1
        for (int h = 0; h < kC / 32; ++h) {  // 32 columns at a time (register budget)
          float w[32];
          tmem_ld32(lane_tmem + buf * NC + h * 32, w);
          tmem_wait_ld();
          if (h == kC / 32 - 1) {  // the buffer is drained: the MMA may refill it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(TEMPTY0 + 8u * buf);
            ++tcount;
          }
          const int k0 = kb + h * 32;
          float c4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // independent chains
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const float4 a = __ldg(reinterpret_cast<const float4 *>(coef + k0 + e));
            const float4 b = __ldg(reinterpret_cast<const float4 *>(cst2 + k0 + e));
            w[e] = fmaf(w[e], a.x, b.x);
            w[e + 1] = fmaf(w[e + 1], a.y, b.y);
            w[e + 2] = fmaf(w[e + 2], a.z, b.z);
            w[e + 3] = fmaf(w[e + 3], a.w, b.w);
#pragma unroll
            for (int r = 0; r < 4; ++r) c4[r] = fmaxf(c4[r], w[e + r]);
          }
          const float cm = fmaxf(fmaxf(c4[0], c4[1]), fmaxf(c4[2], c4[3]));
          {  // the log2-likelihood block, transposed: a warp's store is 32 consecutive points
            float *lp = Lt + (int64_t)k0 * Npad + n_row;
#pragma unroll
            for (int e = 0; e < 32; ++e, lp += Npad) st_hint(lp, w[e], pol_l);
          }
          // A value enters the leading four only if it lies within kNear of the point's
          // running maximum (the refinement re-evaluates nothing further below).  Only a
          // half whose maximum comes that close is scanned: its qualifying values are
          // pushed in turn and w[] then holds the values that drop out.  Every other value
          // joins the rest, whose reference is its true maximum (so its sum never
          // underflows to zero).
          float mn;
          if (cm > tv[0] - kNear) {
            const float thr = fmaxf(tv[0], cm) - kNear;
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              if (w[e] > thr && w[e] > tv[3]) {
                int di;
                top_push(tv, ti, w[e], k0 + e, w[e], di);  // w[e] becomes the dropped value
              }
            }
            float r4[4] = {m, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int e = 0; e < 32; ++e) r4[e & 3] = fmaxf(r4[e & 3], w[e]);
            mn = fmaxf(fmaxf(r4[0], r4[1]), fmaxf(r4[2], r4[3]));
          } else {
            mn = fmaxf(m, cm);
          }
          const float mr = (mn == -INFINITY) ? 0.0f : mn;
          float a4[4] = {s * ex2(m - mr), 0.0f, 0.0f, 0.0f};
#pragma unroll
          for (int e = 0; e < 32; ++e) a4[e & 3] += ex2(w[e] - mr);  // a dropped empty slot: -inf
          s = (a4[0] + a4[1]) + (a4[2] + a4[3]);
          m = mn;
        }
      }
      // merge the four column parts of each row
      if (part > 0) {
        Part &o = lse_x[(part - 1) * BM + row];
        o.m = m; o.s = s;
#pragma unroll
        for (int r = 0; r < kTcTop; ++r) { o.v[r] = tv[r]; o.i[r] = ti[r]; }
      }
      ok = epi_sync_and(ok);
      if (part == 0) {
#pragma unroll
        for (int r = 0; r < 3; ++r) {
          const Part &o = lse_x[r * BM + row];
          lse_merge(m, s, o.m, o.s);
#pragma unroll
          for (int c = 0; c < kTcTop; ++c)
            if (o.i[c] >= 0) summary_push(tv, ti, m, s, o.v[c], o.i[c]);
        }
        const int64_t n = (int64_t)pt * BM + row;
        if (ok && n < N) {
          part_m[(int64_t)g * N + n] = m;
          part_s[(int64_t)g * N + n] = s;
          part_tv[(int64_t)g * N + n] = make_float4(tv[0], tv[1], tv[2], tv[3]);
          part_ti[(int64_t)g * N + n] = make_int4(ti[0], ti[1], ti[2], ti[3]);
        }
      }
      ok = epi_sync_and(ok);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * NC);
  }
}

// Exact squared distances of one point (eight lanes, dimension i * 8 + sub per lane) to
// two components (index -1: none): sum_j ((x_j - mu_j) var_j^-1/2)^2, each term from the
// fp32 inputs in fp64 (fp32 terms leave ~10x the error in the variances), reduced over the
// point's eight lanes.
template <int DPL, bool VEC>
__device__ __forceinline__ void exact_pair(const float (&x)[DPL], int sub, int d,
                                           const float *__restrict__ sc, const float *__restrict__ mu,
                                           int k0, int k1, double (&p)[2]) {
  const int kk[2] = {k0, k1};
  float m[2][DPL], sv[2][DPL];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const bool need = kk[u] >= 0;
    const int64_t base = (int64_t)(need ? kk[u] : 0) * d;
    if (VEC) {
#pragma unroll
      for (int i = 0; i < DPL / 4; ++i) {
        const int64_t q = base + (int64_t)(i * 8 + sub) * 4;
        const float4 m4 = need ? __ldg(reinterpret_cast<const float4 *>(mu + q)) : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 s4 = need ? __ldg(reinterpret_cast<const float4 *>(sc + q)) : make_float4(0.f, 0.f, 0.f, 0.f);
        m[u][4 * i] = m4.x; m[u][4 * i + 1] = m4.y; m[u][4 * i + 2] = m4.z; m[u][4 * i + 3] = m4.w;
        sv[u][4 * i] = s4.x; sv[u][4 * i + 1] = s4.y; sv[u][4 * i + 2] = s4.z; sv[u][4 * i + 3] = s4.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        const int j = i * 8 + sub;
        const bool in = need && j < d;
        m[u][i] = in ? __ldg(mu + base + j) : 0.0f;
        sv[u][i] = in ? __ldg(sc + base + j) : 0.0f;
      }
    }
  }
  // the second component's arithmetic only where some point of the warp needs it
  const bool any1 = __any_sync(0xffffffffu, k1 >= 0);
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    p[u] = 0.0;
    if (u == 1 && !any1) break;
    double a0 = 0.0, a1 = 0.0;  // two chains
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const double t = ((double)x[i] - (double)m[u][i]) * (double)sv[u][i];
      if (i & 1) a1 = fma(t, t, a1); else a0 = fma(t, t, a0);
    }
    p[u] = a0 + a1;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) p[u] += __shfl_xor_sync(0xffffffffu, p[u], o);
  }
}

// ------------------------------------------------------------------------- refine
// Exact re-evaluation of each point's leading components.  The tensor-core
// log-likelihoods carry an absolute error of ~1e-4 (the products are fp16 hi/lo pairs
// and tensor-memory accumulation truncates), while the responsibility mass of a point
// sits on its few leading components.  This kernel merges the pass-1 summaries of the
// component groups and re-evaluates every one of the four leading log-likelihoods that
// lies within 2^-kNear of the leader: sum_j ((x_j - mu_j) var_j^-1/2)^2 from the fp32
// inputs, evaluated and summed in fp64 (the direct form of
// flash_gmm/csrc/flash_gmm_cpu.cpp:30-45, which the reference evaluates in fp32).  The point's log-normalizer is formed in fp64 from them and the rest's sum.
// Outputs per point: the log-normalizer (fp32 output, a fp64 block sum, and its base-2
// form for the statistics pass), and the re-evaluated components with their base-2
// log-responsibilities l2 - ln2 (fp32 of the fp64 difference: these small numbers keep
// full precision, where an fp32 l2 of magnitude ~300 would not), which the statistics
// pass substitutes for its tensor-core values.
// Eight lanes per point (four points per warp), lanes striped over the dimensions; the
// point's row is loaded first so its latency overlaps the partial loads.
template <int DPL, bool VEC>  // dimensions per lane: ceil(d / 8); VEC: vector loads
__global__ void __launch_bounds__(256, DPL >= 12 ? 2 : 4)
tc_refine_kernel(const float *__restrict__ X, int64_t N, int d, const float *__restrict__ sc,
                 const float *__restrict__ mu, const double *__restrict__ lc,
                 const float *__restrict__ part_m, const float *__restrict__ part_s,
                 const float4 *__restrict__ part_tv, const int4 *__restrict__ part_ti, int G,
                 float *__restrict__ ln2x, int4 *__restrict__ top_i, float4 *__restrict__ top_d,
                 uint32_t *__restrict__ xmask, int64_t msl, float *__restrict__ ln_out,
                 double *__restrict__ ln_part, int acc_ln) {
  __shared__ double wsum[8];
  griddep_launch();
  bool waited = false;  // X is an input: its first rows load before waiting for pass 1
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane & 7;  // lane within the point's group of 8
  double acc = 0.0;
  const int64_t stride = (int64_t)gridDim.x * 32;  // points per grid sweep
  for (int64_t n = ((int64_t)blockIdx.x * 8 + warp) * 4 + (lane >> 3); n - (lane >> 3) < N;
       n += stride) {
    const bool live = n < N;
    const int64_t nn = live ? n : 0;
    float x[DPL];
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
    if (!waited) {
      griddep_wait();
      waited = true;
    }
    // merge the component groups' summaries: leading four and the log-sum-exp of the rest
    float mx = -INFINITY, sm = 0.0f;
    float b[kTcTop] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    int jx[kTcTop] = {-1, -1, -1, -1};
    if (G == 1) {  // one group: its summary is already the point's
      const float4 tv = __ldg(part_tv + nn);
      const int4 ti = __ldg(part_ti + nn);
      mx = __ldg(part_m + nn); sm = __ldg(part_s + nn);
      b[0] = tv.x; b[1] = tv.y; b[2] = tv.z; b[3] = tv.w;
      jx[0] = ti.x; jx[1] = ti.y; jx[2] = ti.z; jx[3] = ti.w;
    } else
#pragma unroll 2
    for (int g = 0; g < G; ++g) {
      const float4 tv = __ldg(part_tv + (int64_t)g * N + nn);
      const int4 ti = __ldg(part_ti + (int64_t)g * N + nn);
      lse_merge(mx, sm, __ldg(part_m + (int64_t)g * N + nn), __ldg(part_s + (int64_t)g * N + nn));
      if (ti.x >= 0) summary_push(b, jx, mx, sm, tv.x, ti.x);
      if (ti.y >= 0) summary_push(b, jx, mx, sm, tv.y, ti.y);
      if (ti.z >= 0) summary_push(b, jx, mx, sm, tv.z, ti.z);
      if (ti.w >= 0) summary_push(b, jx, mx, sm, tv.w, ti.w);
    }
    // the components within 2^-kNear of the leader are re-evaluated (the others carry
    // responsibilities below 2e-10 of the leader's and keep their tensor-core values)
    double v[kTcTop];
    bool ex[kTcTop];
#pragma unroll
    for (int c = 0; c < kTcTop; ++c) {
      ex[c] = jx[c] >= 0 && b[c] >= b[0] - kNear;
      v[c] = jx[c] >= 0 ? (double)b[c] : -INFINITY;
    }
    // two components at a time, all their loads issued before the arithmetic
#pragma unroll
    for (int c = 0; c < kTcTop; c += 2) {
      if (!__any_sync(0xffffffffu, ex[c] || ex[c + 1])) continue;
      double p[2];
      exact_pair<DPL, VEC>(x, sub, d, sc, mu, ex[c] ? jx[c] : -1, ex[c + 1] ? jx[c + 1] : -1, p);
#pragma unroll
      for (int u = 0; u < 2; ++u)
        if (ex[c + u]) v[c + u] = (__ldg(lc + jx[c + u]) - 0.5 * p[u]) * 1.4426950408889634;
    }
    // the sum: the rest (fp32 tensor-core values), plus the leading four; terms relative to
    // the maximum in fp32, the maximum itself kept in fp64
    double m = (double)mx;
#pragma unroll
    for (int c = 0; c < kTcTop; ++c) m = fmax(m, v[c]);
    const double mr = m == -INFINITY ? 0.0 : m;
    float tot = sm * exp2f((float)((double)mx - mr));
#pragma unroll
    for (int c = 0; c < kTcTop; ++c) tot += exp2f((float)(v[c] - mr));
    const float lt = log2f(tot);
    const double ln2 = mr + (double)lt;
    if (live && sub == 0) {
      ln2x[n] = (float)(ln2 - kTcGammaExp);  // the statistics pass works with gamma 2^14
      top_i[n] = make_int4(ex[0] ? jx[0] : -1, ex[1] ? jx[1] : -1, ex[2] ? jx[2] : -1, ex[3] ? jx[3] : -1);
      top_d[n] = make_float4((float)(v[0] - mr) - lt, (float)(v[1] - mr) - lt, (float)(v[2] - mr) - lt,
                             (float)(v[3] - mr) - lt);
      // mark the point in the (component tile, slice) words of its exact components
#pragma unroll
      for (int c = 0; c < kTcTop; ++c)
        if (ex[c])
          atomicOr(xmask + ((int64_t)(jx[c] / NC2_ref) * msl + n / kSlice_ref) * NC2_ref + jx[c] % NC2_ref,
                   1u << (n % kSlice_ref));
      const double l = ln2 * 0.6931471805599453;
      ln_out[n] = (float)l;
      acc += l;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (!waited) griddep_wait();
  if (lane == 0) wsum[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < 8; ++w) t += wsum[w];
    ln_part[blockIdx.x] = acc_ln ? ln_part[blockIdx.x] + t : t;  // chunks add up in order
  }
}

// The same refinement with one lane per point for the per-point work, for d <= 64: the
// (point, component) pairs to re-evaluate are listed in shared memory and taken four at a
// time, eight lanes per pair striped over the dimensions.  It executes fewer instructions
// than eight lanes per point repeating the per-point merge, which pays at small d (configs
// 3 and 4: 78 -> 59 and 31 -> 23 us); at d = 128 the per-point kernel measured faster
// (37 against 45 us at config 2).
constexpr int kRefWarps = 8;
constexpr int kRefPts = 16;  // points per warp (lanes 0-15; more warps in flight for small N)
template <int DPL, bool VEC>  // dimensions per lane of a pair: ceil(d / 8); VEC: float4 loads
__global__ void __launch_bounds__(32 * kRefWarps, DPL >= 12 ? 3 : 4)
tc_refine_items_kernel(const float *__restrict__ X, int64_t N, int d, const float *__restrict__ sc,
                 const float *__restrict__ mu, const double *__restrict__ lc,
                 const float *__restrict__ part_m, const float *__restrict__ part_s,
                 const float4 *__restrict__ part_tv, const int4 *__restrict__ part_ti, int G,
                 float *__restrict__ ln2x, int4 *__restrict__ top_i, float4 *__restrict__ top_d,
                 uint32_t *__restrict__ xmask, int64_t msl, float *__restrict__ ln_out,
                 double *__restrict__ ln_part, int acc_ln) {
  __shared__ int s_item[kRefWarps][32 * kTcTop];     // (lane << 2) | c
  __shared__ double s_val[kRefWarps][32 * kTcTop];   // exact base-2 log-likelihoods
  __shared__ double wsum[kRefWarps];
  griddep_launch();
  griddep_wait();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, sub = lane & 7;
  const unsigned lt_mask = (1u << lane) - 1u;
  double acc = 0.0;
  for (int64_t base = ((int64_t)blockIdx.x * kRefWarps + warp) * kRefPts; base < N;
       base += (int64_t)gridDim.x * kRefWarps * kRefPts) {
    const int64_t n = base + (lane & (kRefPts - 1));
    const bool live = lane < kRefPts && n < N;
    // merge the component groups' summaries: leading four and the log-sum-exp of the rest
    float mx = -INFINITY, sm = 0.0f;
    float b[kTcTop] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    int jx[kTcTop] = {-1, -1, -1, -1};
    if (live && G == 1) {  // one group: its summary is already the point's
      const float4 tv = __ldg(part_tv + n);
      const int4 ti = __ldg(part_ti + n);
      mx = __ldg(part_m + n); sm = __ldg(part_s + n);
      b[0] = tv.x; b[1] = tv.y; b[2] = tv.z; b[3] = tv.w;
      jx[0] = ti.x; jx[1] = ti.y; jx[2] = ti.z; jx[3] = ti.w;
    } else if (live) {
      for (int g = 0; g < G; ++g) {
        const float4 tv = __ldg(part_tv + (int64_t)g * N + n);
        const int4 ti = __ldg(part_ti + (int64_t)g * N + n);
        lse_merge(mx, sm, __ldg(part_m + (int64_t)g * N + n), __ldg(part_s + (int64_t)g * N + n));
        if (ti.x >= 0) summary_push(b, jx, mx, sm, tv.x, ti.x);
        if (ti.y >= 0) summary_push(b, jx, mx, sm, tv.y, ti.y);
        if (ti.z >= 0) summary_push(b, jx, mx, sm, tv.z, ti.z);
        if (ti.w >= 0) summary_push(b, jx, mx, sm, tv.w, ti.w);
      }
    }
    // the components within 2^-kNear of the leader are re-evaluated (the others carry
    // responsibilities below 2e-10 of the leader's and keep their tensor-core values);
    // list them: item pos[c] of this warp
    bool ex[kTcTop];
    int pos[kTcTop];
    int nitems = 0;
#pragma unroll
    for (int c = 0; c < kTcTop; ++c) {
      ex[c] = live && jx[c] >= 0 && b[c] >= b[0] - kNear;
      const unsigned bal = __ballot_sync(0xffffffffu, ex[c]);
      pos[c] = nitems + __popc(bal & lt_mask);
      if (ex[c]) s_item[warp][pos[c]] = (lane << 2) | c;
      nitems += __popc(bal);
    }
    __syncwarp();
    for (int i0 = 0; i0 < nitems; i0 += 4) {
      const int item = i0 + (lane >> 3);
      const bool valid = item < nitems;
      const int code = valid ? s_item[warp][item] : 0;
      const int pl = code >> 2, c = code & 3;
      // the component of that lane's leading slot c
      const int k0 = __shfl_sync(0xffffffffu, jx[0], pl), k1 = __shfl_sync(0xffffffffu, jx[1], pl);
      const int k2 = __shfl_sync(0xffffffffu, jx[2], pl), k3 = __shfl_sync(0xffffffffu, jx[3], pl);
      const int k = c == 0 ? k0 : (c == 1 ? k1 : (c == 2 ? k2 : k3));
      const int64_t xrow = (base + pl) * d, krow = (int64_t)(valid ? k : 0) * d;
      double a0 = 0.0, a1 = 0.0;  // two chains
      if (VEC) {  // d == 8 DPL, DPL % 4 == 0, 16-byte aligned rows; lane takes float4 i * 8 + sub
#pragma unroll
        for (int i = 0; i < DPL / 4; ++i) {
          const int64_t q = (int64_t)(i * 8 + sub) * 4;
          float4 x4 = make_float4(0.f, 0.f, 0.f, 0.f), m4 = x4, s4 = x4;
          if (valid) {
            x4 = __ldg(reinterpret_cast<const float4 *>(X + xrow + q));
            m4 = __ldg(reinterpret_cast<const float4 *>(mu + krow + q));
            s4 = __ldg(reinterpret_cast<const float4 *>(sc + krow + q));
          }
          const double t0 = ((double)x4.x - (double)m4.x) * (double)s4.x;
          const double t1 = ((double)x4.y - (double)m4.y) * (double)s4.y;
          const double t2 = ((double)x4.z - (double)m4.z) * (double)s4.z;
          const double t3 = ((double)x4.w - (double)m4.w) * (double)s4.w;
          a0 = fma(t0, t0, a0); a1 = fma(t1, t1, a1); a0 = fma(t2, t2, a0); a1 = fma(t3, t3, a1);
        }
      } else {
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          const int j = i * 8 + sub;
          const bool in = valid && j < d;
          const float xv = in ? __ldg(X + xrow + j) : 0.0f;
          const float mv = in ? __ldg(mu + krow + j) : 0.0f;
          const float sv = in ? __ldg(sc + krow + j) : 0.0f;
          const double t = ((double)xv - (double)mv) * (double)sv;
          if (i & 1) a1 = fma(t, t, a1); else a0 = fma(t, t, a0);
        }
      }
      double pq = a0 + a1;
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) pq += __shfl_xor_sync(0xffffffffu, pq, o);
      if (valid && sub == 0) s_val[warp][item] = (__ldg(lc + k) - 0.5 * pq) * 1.4426950408889634;
    }
    __syncwarp();
    if (live) {
      // the sum: the rest (fp32 tensor-core values), plus the leading four (exact where
      // re-evaluated); terms relative to the maximum in fp32, the maximum kept in fp64
      double v[kTcTop];
      double m = (double)mx;
#pragma unroll
      for (int c = 0; c < kTcTop; ++c) {
        v[c] = ex[c] ? s_val[warp][pos[c]] : (jx[c] >= 0 ? (double)b[c] : -INFINITY);
        m = fmax(m, v[c]);
      }
      const double mr = m == -INFINITY ? 0.0 : m;
      float tot = sm * exp2f((float)((double)mx - mr));
#pragma unroll
      for (int c = 0; c < kTcTop; ++c) tot += exp2f((float)(v[c] - mr));
      const float lt = log2f(tot);
      const double ln2 = mr + (double)lt;
      ln2x[n] = (float)(ln2 - kTcGammaExp);  // the statistics pass works with gamma 2^14
      top_i[n] = make_int4(ex[0] ? jx[0] : -1, ex[1] ? jx[1] : -1, ex[2] ? jx[2] : -1, ex[3] ? jx[3] : -1);
      top_d[n] = make_float4((float)(v[0] - mr) - lt, (float)(v[1] - mr) - lt, (float)(v[2] - mr) - lt,
                             (float)(v[3] - mr) - lt);
      // mark the point in the (component tile, slice) words of its exact components
#pragma unroll
      for (int c = 0; c < kTcTop; ++c)
        if (ex[c])
          atomicOr(xmask + ((int64_t)(jx[c] / NC2_ref) * msl + n / kSlice_ref) * NC2_ref + jx[c] % NC2_ref,
                   1u << (n % kSlice_ref));
      const double l = ln2 * 0.6931471805599453;
      ln_out[n] = (float)l;
      acc += l;
    }
    __syncwarp();  // s_item / s_val are reused by the next 32 points
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) wsum[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < kRefWarps; ++w) t += wsum[w];
    ln_part[blockIdx.x] = acc_ln ? ln_part[blockIdx.x] + t : t;  // chunks add up in order
  }
}

// ------------------------------------------------------------------------- pass 2
// Statistics GEMM S[k, f] = sum_n gamma[n, k] F[n, f] with F = [x^2 | x] (fp16 hi/lo,
// column-scaled), the tensor-core work left once pass 1 has stored the log2-likelihood
// block Lt and the refinement the exact leading components of every point.
// A CTA owns 128 components (the M of the MMA, on the TMEM lanes) and a contiguous range
// of points, taken in slices of 32 points (two kind::f16 k-steps).  Roles:
//   warp 9 lane 0 (producer): per slice, TMA of F hi and F lo (one 3-D box each: 32 points
//     x all 64-feature atoms, MN-major SWIZZLE_128B), of the slice's Lt tile
//     [128 components][32 points], its 32 log2-normalizers (shifted by the gamma scale),
//     the points' exact leaders and the slice's exact-component bit words;
//   warps 0-7 (gamma): warp w computes gamma 2^14 = 2^(l2 - ln2 + 14) for components
//     32 (w % 4) .. +31 (its TMEM lane quarter) at 16 of the slice's 32 points, taking
//     the exact value where the component's bit is set, splits it into fp16 hi / lo and
//     stores the pairs into a TMEM gamma buffer (two points per 32-bit column), the MMA's
//     A operand;
//   warp 8 lane 0 (MMA): six MMAs per slice (gamma_lo F_hi, gamma_hi F_lo, gamma_hi F_hi,
//     two k-steps each) into the statistics accumulator;
//   all 16 warps: every kSlicesFlush slices (256 points) the accumulator is added into
//     fp32 registers (warp w: lane quarter w % 4, a quarter of the columns), because
//     tensor-memory accumulation does not round to nearest.  With two accumulator regions
//     (KA <= 192) the tensor pipe fills one while the other drains.
// Every hand-off is an mbarrier; no barrier spans the CTA inside the loop.
constexpr int kSlicePts = 32;
constexpr int kSlicesFlush = 8;  // drains every 256 points
constexpr int kGBufs = 4;
constexpr int kThreads2 = 512;
constexpr int kGammaWarps = 8;
constexpr int kGPts = kSlicePts / 2;  // points of a slice per gamma warp
constexpr int kGCols = kSlicePts;     // TMEM columns of one gamma buffer: hi 16 | lo 16
constexpr int NC2 = NC2_ref;  // components per statistics CTA
static_assert(kSlicePts == kSlice_ref, "one bit per point of a slice");

template <int KA>
struct StatsShape {
  static constexpr int kAtom = kSlicePts * 128;                // 4 KB: 32 points x 64 fp16
  static constexpr int kFPart = (KA / 64) * kAtom;             // F hi (or lo) of a slice
  static constexpr int kLOff = 2 * kFPart;                     // Lt tile [128][32], 128B-swizzled
  static constexpr int kNOff = kLOff + kSlicePts * NC2 * 4;    // ln2 [32]
  static constexpr int kTOff = kNOff + kSlicePts * 4;          // exact leaders: int4 [32], float4 [32]
  static constexpr int kMOff = kTOff + kSlicePts * 32;         // exact-component bit words [128]
  static constexpr int kStage = (kMOff + NC2 * 4 + 1023) / 1024 * 1024;
  static constexpr int kStagesFit = (220 * 1024) / kStage;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int kSmem = 1024 + kStages * kStage + 512;
  static_assert(kStages * kStage >= NC2 * (KA + 4) * 4 + NC2 * 4, "partial rows staged in the ring");
};

__device__ __forceinline__ bool cta_sync_and(bool v) {
  return __syncthreads_and(v ? 1 : 0) != 0;
}

// Partial statistics row (per component and CTA slot, partial[k][slot]):
// [s (DP) | sq (DP) | n | pad], stride 2 DP + 4, unscaled fp32.
template <int NKCF>
__global__ void __launch_bounds__(kThreads2, 1)
tc_stats_kernel(const __grid_constant__ CUtensorMap tm_fhi, const __grid_constant__ CUtensorMap tm_flo,
                const __grid_constant__ CUtensorMap tm_l, const float *__restrict__ ln2x,
                const int4 *__restrict__ top_i, const float4 *__restrict__ top_d,
                const uint32_t *__restrict__ xmask, int64_t msl, int64_t N, int S_slots, int K, int d,
                const int *__restrict__ aexp, float *__restrict__ partial, int accum,
                const float *__restrict__ Lt, int64_t Npad) {
  constexpr int KA = NKCF * 64;
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
  // F (prepared points) does not change between launches: the producer starts loading the
  // first slices' F before waiting for the earlier launches; every other thread waits first.
  const int fpre = (warp == kGammaWarps + 1 && lane == 0) ? min(S, NST) : 0;
  for (int sp = 0; sp < fpre; ++sp) {
    const uint32_t base = smem_u32(smem + sp * Sh::kStage);
    const int64_t nb = (s0 + sp) * kSlicePts;
    mbar_arrive_expect_tx(FULL(sp), 2 * Sh::kFPart + kSlicePts * NC2 * 4 + kSlicePts * 36 + NC2 * 4);
    tma_load_3d(base, &tm_fhi, 0, (int32_t)nb, 0, FULL(sp));
    tma_load_3d(base + Sh::kFPart, &tm_flo, 0, (int32_t)nb, 0, FULL(sp));
  }
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
    const int p0 = (warp >> 2) * kGPts;  // this warp's points of each slice
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
      // this lane's component row of the Lt tile: 32 points = eight 16-byte chunks, chunk c
      // stored at c ^ (row & 7) (SWIZZLE_128B)
      const float4 *Lrow = reinterpret_cast<const float4 *>(stg + Sh::kLOff + cl * 128);
      const int sw = cl & 7;
      const float4 *ln4 = reinterpret_cast<const float4 *>(stg + Sh::kNOff);
      const int4 *ti_s = reinterpret_cast<const int4 *>(stg + Sh::kTOff);
      const float4 *td_s = reinterpret_cast<const float4 *>(stg + Sh::kTOff + kSlicePts * 16);
      const int kabs = ct * NC2 + cl;
      const uint32_t xw = reinterpret_cast<const uint32_t *>(stg + Sh::kMOff)[cl] >> p0;
      const int64_t nb = (s0 + s) * kSlicePts;
      const int live = (N - nb < kSlicePts ? (int)(N - nb) : kSlicePts) - p0;
      float g[kGPts];
#pragma unroll
      for (int c = 0; c < kGPts / 4; ++c) {
        const float4 l4 = ln4[p0 / 4 + c];
        const float4 v4 = Lrow[(p0 / 4 + c) ^ sw];
        const float ln2[4] = {l4.x, l4.y, l4.z, l4.w};
        const float lv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int p = c * 4 + e;
          // base-2 log-responsibility (scaled by 2^14): the tensor-core value, or, for the
          // point's exactly evaluated leading components (marked in xw), the exact one
          float dl = lv[e] - ln2[e];
          if ((xw >> p) & 1u) {
            const int4 ti = ti_s[p0 + p];
            const float4 td = td_s[p0 + p];
            dl = (kabs == ti.x ? td.x : (kabs == ti.y ? td.y : (kabs == ti.z ? td.z : td.w))) +
                 (float)kTcGammaExp;
          }
          g[p] = p < live ? ex2(dl) : 0.0f;
          nk += g[p];
        }
      }
      uint32_t hi8[kGPts / 2], lo8[kGPts / 2];
#pragma unroll
      for (int i = 0; i < kGPts / 2; ++i) {  // fp16 hi / lo pairs, two points per 32-bit column
        const __half2 h = __floats2half2_rn(g[2 * i], g[2 * i + 1]);
        const float2 hf = __half22float2(h);
        const __half2 l = __floats2half2_rn(g[2 * i] - hf.x, g[2 * i + 1] - hf.y);
        hi8[i] = *reinterpret_cast<const uint32_t *>(&h);
        lo8[i] = *reinterpret_cast<const uint32_t *>(&l);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(EMPTY(st));  // this warp is done with the slice's Lt
      const uint32_t ga = lane_tmem + kGBase + gb * kGCols + p0 / 2;
      tmem_st8(ga, *reinterpret_cast<const float(*)[8]>(hi8));
      tmem_st8(ga + kSlicePts / 2, *reinterpret_cast<const float(*)[8]>(lo8));
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(GFULL(gb));
    }
  } else if (warp == kGammaWarps) {
    // ---------------- MMA warp
    constexpr uint32_t idesc = idesc_f16(NC2, KA, 0, 1);  // A from TMEM, B MN-major
    // B: 64-feature atoms of kSlicePts points each: LBO = atom stride, SBO = 8 points (1 KB)
    const uint64_t fdesc0 = sdesc(smem_u32(smem), Sh::kAtom, 1024, kSw128);
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
        const uint64_t fd = fdesc0 + (uint64_t)((st * Sh::kStage) >> 4);
        constexpr uint64_t kLo = Sh::kFPart >> 4, kK = (16 * 128) >> 4;  // k-step: 16 points
        constexpr uint32_t kGLo = kSlicePts / 2;                          // gamma lo columns
#pragma unroll
        for (int kk = 0; kk < kSlicePts / 16; ++kk) {
          mma_f16_ta(dst, gbuf + kGLo + kk * 8, fd + kk * kK, idesc, (tile_first && kk == 0) ? 0u : 1u);
          mma_f16_ta(dst, gbuf + kk * 8, fd + kLo + kk * kK, idesc, 1u);
        }
#pragma unroll
        for (int kk = 0; kk < kSlicePts / 16; ++kk) mma_f16_ta(dst, gbuf + kk * 8, fd + kk * kK, idesc, 1u);
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
    // Lt is read exactly once: once a slice's tile has been consumed, its lines are dropped
    // from L2 without being written back, so a block that stayed in L2 from pass 1 to here
    // never reaches DRAM
    const uint64_t pol_l = policy_evict_first();
    auto discard_lt_slice = [&](int sd) {
      const float *row0 = Lt + (int64_t)ct * NC2 * Npad + (s0 + sd) * kSlicePts;
#pragma unroll
      for (int r = lane; r < NC2; r += 32) discard_l2_line(row0 + (int64_t)r * Npad);
    };
    for (int s = 0; s < S && ok; ++s) {
      // same rule as the gamma warps, NST slices ahead (before the EMPTY wait below)
      while (nf < T && s >= kSlicesFlush * (nf + 1) + NST && ok) flush_next(false);
      if (nf < T && s >= kSlicesFlush * (nf + 1) && tile_done(nf)) flush_next(false);  // early
      const int st = s % NST;
      if (s >= NST) {
        ok = ok && __all_sync(0xffffffffu, mbar_wait(EMPTY(st), ((s / NST) & 1) ^ 1, kErrWaitEmpty));
        if (ok) discard_lt_slice(s - NST);
      }
      if (!ok) break;
      if (lane == 0) {
        const uint32_t base = smem_u32(smem + st * Sh::kStage);
        const int64_t nb = (s0 + s) * kSlicePts;
        if (s >= fpre) {  // F, Lt, ln2, leaders, exact-component words (F of the first slices is on its way)
          mbar_arrive_expect_tx(FULL(st), 2 * Sh::kFPart + kSlicePts * NC2 * 4 + kSlicePts * 36 + NC2 * 4);
          tma_load_3d(base, &tm_fhi, 0, (int32_t)nb, 0, FULL(st));
          tma_load_3d(base + Sh::kFPart, &tm_flo, 0, (int32_t)nb, 0, FULL(st));
        }
        tma_load_2d_hint(base + Sh::kLOff, &tm_l, (int32_t)nb, ct * NC2, FULL(st), pol_l);
        bulk_load(base + Sh::kNOff, ln2x + nb, kSlicePts * 4, FULL(st));
        bulk_load(base + Sh::kTOff, top_i + nb, kSlicePts * 16, FULL(st));
        bulk_load(base + Sh::kTOff + kSlicePts * 16, top_d + nb, kSlicePts * 16, FULL(st));
        bulk_load(base + Sh::kMOff, xmask + ((int64_t)ct * msl + s0 + s) * NC2, NC2 * 4, FULL(st));
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
  if (warp == kGammaWarps + 1 && ok) {  // the producer drops the last slices' Lt lines
    for (int sd = (S > NST ? S - NST : 0); sd < S; ++sd) {
      const float *row0 = Lt + (int64_t)ct * NC2 * Npad + (s0 + sd) * kSlicePts;
      for (int r = lane; r < NC2; r += 32) discard_l2_line(row0 + (int64_t)r * Npad);
    }
  }
  // The tile's partial rows go through shared memory (the stage ring is idle now), so the
  // global writes are whole coalesced rows: row c = component ct * 128 + c, laid out
  // [s (DP) | sq (DP) | n | pad].  The column and responsibility scales are undone by exact
  // power-of-two multiplies.
  float *rows_s = reinterpret_cast<float *>(smem);         // [128][PSTRIDE]
  float *nk_s = rows_s + NC2 * PSTRIDE;                     // [128]
#pragma unroll
  for (int e = 0; e < SEG; e += 4) {
    const int f = seg * SEG + e;  // feature column: x^2 part first, then x
    const int j0 = f < DP ? f : f - DP, t = f < DP ? 0 : 1;
    float r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int ex = (j0 + i < d ? __ldg(aexp + 3 * (j0 + i) + t) : 0) + kTcGammaExp;
      r[i] = (ok && j0 + i < d) ? sacc[e + i] * __int_as_float((127 - ex) << 23) : 0.0f;
    }
    *reinterpret_cast<float4 *>(rows_s + cl * PSTRIDE + (f < DP ? DP + f : f - DP)) =
        make_float4(r[0], r[1], r[2], r[3]);
  }
  // n_k: the two gamma warps of a lane quarter add up their halves of the points
  if (warp >= 4 && warp < kGammaWarps) nk_s[cl] = nk;
  __syncthreads();
  if (warp < 4)
    *reinterpret_cast<float4 *>(rows_s + cl * PSTRIDE + 2 * DP) =
        make_float4(ok ? (nk + nk_s[cl]) * (1.0f / (float)(1 << kTcGammaExp)) : 0.0f, 0.f, 0.f, 0.f);
  __syncthreads();
  {
    constexpr int Q = PSTRIDE / 4;  // float4 per row
    const int rows = min(NC2, K - ct * NC2);
    for (int i = threadIdx.x; i < rows * Q; i += kThreads2) {
      const int c = i / Q, q = i - c * Q;
      float4 *o = reinterpret_cast<float4 *>(partial + ((int64_t)(ct * NC2 + c) * S_slots + slot) * PSTRIDE) + q;
      float4 v = reinterpret_cast<const float4 *>(rows_s + c * PSTRIDE)[q];
      if (accum) {  // a later chunk of the same iteration: this CTA slot's row adds up
        const float4 o0 = *o;
        v = make_float4(o0.x + v.x, o0.y + v.y, o0.z + v.z, o0.w + v.w);
      }
      *o = v;
    }
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

// Row-major fp16 [rows][cols] matrix (cols a multiple of 64) seen as 64-column atoms:
// box = box_rows x all atoms, landing as [atom][row][64] with SWIZZLE_128B (the MN-major
// operand layout of the statistics GEMM).
int make_map_atoms16(CUtensorMap *m, const __half *base, int64_t rows, int cols, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(FGMM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)KCH, (cuuint64_t)rows, (cuuint64_t)(cols / KCH)};
  cuuint64_t strides[2] = {(cuuint64_t)cols * 2, (cuuint64_t)KCH * 2};
  cuuint32_t box[3] = {(cuuint32_t)KCH, (cuuint32_t)box_rows, (cuuint32_t)(cols / KCH)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half *>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FGMM_ERR_CUDA, "cuTensorMapEncodeTiled (atoms) failed: " + std::to_string((int)r));
  return FGMM_OK;
}

// Row-major [rows][cols] matrix of `dtype` (element size `es`), box [box_rows][box_cols].
int make_map(CUtensorMap *m, const void *base, CUtensorMapDataType dtype, int es, int64_t rows,
             int64_t cols, int box_rows, int box_cols, CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return fail(FGMM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * es};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dtype, 2, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FGMM_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return FGMM_OK;
}

// The points are processed in chunks whose log2-likelihood block Lt [Kp][chunk] fits a
// fixed budget, so the workspace stays bounded for any N: pass 1 writes the block, the
// refine kernel patches it and the statistics kernel reads it back.  Chunks run in order
// on the stream; the per-slot statistics rows and the log-normalizer block sums add up
// across chunks.
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
  int d, dp, KA, kbp, nkc, nkcf, K, NC, Kp, n_ct, n_ct2, chunks;
  TcChunk first;
};

TcChunk chunk_plan(int64_t Nc, int n_ct, int n_ct2) {
  TcChunk c{};
  c.Nc = Nc;
  c.n_pt = (int)cdiv(Nc, BM);
  const int sms = num_sms();
  const int G = (int)std::min<int64_t>(n_ct, std::max<int64_t>(1, cdiv(4 * sms, c.n_pt)));
  c.tpg = (int)cdiv(n_ct, G);
  c.G = (int)cdiv(n_ct, c.tpg);
  c.grid1 = (int)std::min<int64_t>((int64_t)c.n_pt * c.G, sms);
  c.S = (int)std::max<int64_t>(1, std::min<int64_t>(sms / std::max(1, n_ct2), cdiv(Nc, 32)));
  c.grid2 = n_ct2 * c.S;
  return c;
}

TcPlan plan(int64_t N, int d, int K) {
  TcPlan p{};
  p.N = N; p.d = d; p.K = K;
  p.dp = tc_dp(d);
  p.KA = 2 * p.dp;
  p.kbp = tc_kbp(d);
  p.nkc = p.kbp / KCH;
  p.nkcf = p.KA / KCH;
  p.NC = K <= 128 ? 128 : 256;
  p.n_ct = (int)cdiv(K, p.NC);
  p.Kp = p.n_ct * p.NC;
  p.n_ct2 = (int)cdiv(K, NC2);
  const int64_t fit = std::max<int64_t>(BM, kLChunkBytes / ((int64_t)p.Kp * 4) / BM * BM);
  p.Nc = std::min<int64_t>(npad_of(N), fit);
  p.chunks = (int)cdiv(N, p.Nc);
  p.first = chunk_plan(std::min<int64_t>(N, p.Nc), p.n_ct, p.n_ct2);
  return p;
}

struct TcWs {
  __half *qhi, *qlo;
  float *coef, *cst2, *sc, *mu, *part_m, *part_s, *ln2x, *partial, *L;
  double *lc;
  float4 *part_tv, *top_d;
  int4 *part_ti, *top_i;
  uint32_t *xmask;
  int64_t msl;  // slices of 32 points per chunk (the bit words' stride)
  double *ln_part;
  size_t bytes;
};

constexpr int kRefineBlocks = 8192;  // 32 points per block per sweep
// Blocks of the refinement launch (and log-normalizer block sums): the per-point kernel
// takes 32 points per block and sweep, the pair-list kernel (d <= 64) 128.
inline int refine_blocks(int64_t N, int d) {
  return (int)std::min<int64_t>(kRefineBlocks, (d + 7) / 8 <= 8 ? cdiv(N, 128) : cdiv(N, 32));
}

// Per-chunk buffers are sized for the first (largest) chunk; the component-group
// partials for n_ct groups, the most any chunk uses.
TcWs tc_layout(void *ws, const TcPlan &p) {
  TcWs w{};
  Carve c(ws);
  const int64_t Nc = p.first.Nc;
  w.qhi = c.take<__half>((size_t)p.Kp * p.kbp);
  w.qlo = c.take<__half>((size_t)p.Kp * p.kbp);
  w.coef = c.take<float>(p.Kp);
  w.cst2 = c.take<float>(p.Kp);
  w.sc = c.take<float>((size_t)p.K * p.d);
  w.mu = c.take<float>((size_t)p.K * p.d);
  w.lc = c.take<double>(p.K);
  w.part_m = c.take<float>((size_t)p.n_ct * Nc);
  w.part_s = c.take<float>((size_t)p.n_ct * Nc);
  w.part_tv = c.take<float4>((size_t)p.n_ct * Nc);
  w.part_ti = c.take<int4>((size_t)p.n_ct * Nc);
  w.ln2x = c.take<float>(npad_of(Nc));
  w.top_i = c.take<int4>(npad_of(Nc));
  w.top_d = c.take<float4>(npad_of(Nc));
  w.msl = npad_of(Nc) / kSlice_ref;
  w.xmask = c.take<uint32_t>((size_t)p.n_ct2 * w.msl * NC2_ref);
  w.partial = c.take<float>((size_t)p.first.S * p.K * (2 * p.dp + 4));
  w.ln_part = c.take<double>(kRefineBlocks);
  w.L = c.take<float>((size_t)npad_of(Nc) * p.Kp);  // Lt [Kp][chunk]
  w.bytes = c.bytes();
  return w;
}

TcParamOps param_ops(const TcWs &w, const TcPlan &p, const void *points) {
  TcParamOps op;
  op.qhi = w.qhi; op.qlo = w.qlo; op.coef = w.coef; op.cst2 = w.cst2;
  op.sc = w.sc; op.mu = w.mu; op.lc = w.lc;
  op.aexp = pts_ptrs(points, p.N, p.d).aexp;
  op.kbp = p.kbp;
  return op;
}

// Kernel attributes are per device and per kernel: `Tag` (one type per kernel
// instantiation) keeps one flag per device.
template <typename Tag, typename F>
int set_smem_once(F *kernel, int bytes) {
  static std::atomic<bool> done[64];
  int dev = 0;
  FGMM_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) dev = 0;
  if (!done[dev].load(std::memory_order_acquire)) {
    FGMM_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done[dev].store(true, std::memory_order_release);
  }
  return FGMM_OK;
}

template <int NKC, int NC>
int launch_pass1(const TcPlan &p, const TcChunk &c, const PtsPtrs &pp, int64_t n0, const TcWs &w,
                 cudaStream_t st) {
  using Sh = Pass1Shape<NKC, NC>;
  int rc = set_smem_once<Sh>(tc_pass1_kernel<NKC, NC>, Sh::kSmem);
  if (rc) return rc;
  const int64_t rows = npad_of(c.Nc);
  CUtensorMap m_phi, m_plo, m_qhi, m_qlo;
  const auto F16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
  if ((rc = make_map(&m_phi, pp.phi + n0 * p.kbp, F16, 2, rows, p.kbp, BM, KCH, SW))) return rc;
  if ((rc = make_map(&m_plo, pp.plo + n0 * p.kbp, F16, 2, rows, p.kbp, BM, KCH, SW))) return rc;
  if ((rc = make_map(&m_qhi, w.qhi, F16, 2, p.Kp, p.kbp, NC, KCH, SW))) return rc;
  if ((rc = make_map(&m_qlo, w.qlo, F16, 2, p.Kp, p.kbp, NC, KCH, SW))) return rc;
  FGMM_CUDA_TRY(launch_pdl(tc_pass1_kernel<NKC, NC>, c.grid1, kThreads1, Sh::kSmem, st, m_phi, m_plo,
                           m_qhi, m_qlo, w.coef, w.cst2, c.Nc, c.n_pt, p.n_ct, c.G, c.tpg, w.part_m,
                           w.part_s, w.part_tv, w.part_ti, w.L, rows, w.xmask,
                           (int64_t)p.n_ct2 * w.msl * NC2_ref));
  mark(st, "tc_pass1_kernel");
  return FGMM_OK;
}

template <int NKC>
int launch_pass1_nc(const TcPlan &p, const TcChunk &c, const PtsPtrs &pp, int64_t n0, const TcWs &w,
                    cudaStream_t st) {
  return p.NC == 128 ? launch_pass1<NKC, 128>(p, c, pp, n0, w, st)
                     : launch_pass1<NKC, 256>(p, c, pp, n0, w, st);
}

template <int NKCF>
int launch_stats(const TcPlan &p, const TcChunk &c, const PtsPtrs &pp, int64_t n0, const TcWs &w,
                 bool first, cudaStream_t st) {
  constexpr int KA = NKCF * 64;
  int rc = set_smem_once<StatsShape<KA>>(tc_stats_kernel<NKCF>, (int)StatsShape<KA>::kSmem);
  if (rc) return rc;
  const int64_t rows = npad_of(c.Nc);
  CUtensorMap m_fhi, m_flo, m_l;
  if ((rc = make_map_atoms16(&m_fhi, pp.fhi + n0 * p.KA, rows, p.KA, kSlicePts))) return rc;
  if ((rc = make_map_atoms16(&m_flo, pp.flo + n0 * p.KA, rows, p.KA, kSlicePts))) return rc;
  if ((rc = make_map(&m_l, w.L, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.Kp, rows, NC2, kSlicePts,
                     CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  FGMM_CUDA_TRY(launch_pdl(tc_stats_kernel<NKCF>, c.grid2, kThreads2, StatsShape<KA>::kSmem, st,
                           m_fhi, m_flo, m_l, w.ln2x, w.top_i, w.top_d, w.xmask, w.msl, c.Nc, c.S,
                           p.K, p.d, pp.aexp,
                           w.partial, first ? 0 : 1, w.L, rows));
  mark(st, "tc_stats_kernel");
  return FGMM_OK;
}

// Pass 1, refine and statistics for the chunk of points [n0, n0 + c.Nc).
int tc_launch_chunk(const TcPlan &p, const TcChunk &c, int64_t n0, bool first, const float *X,
                    const PtsPtrs &pp, const TcWs &w, float *ln, cudaStream_t st) {
  int rc;
  switch (p.nkc) {
    case 1: rc = launch_pass1_nc<1>(p, c, pp, n0, w, st); break;
    case 2: rc = launch_pass1_nc<2>(p, c, pp, n0, w, st); break;
    case 3: rc = launch_pass1_nc<3>(p, c, pp, n0, w, st); break;
    case 4: rc = launch_pass1_nc<4>(p, c, pp, n0, w, st); break;
    case 5: rc = launch_pass1_nc<5>(p, c, pp, n0, w, st); break;
    case 6: rc = launch_pass1_nc<6>(p, c, pp, n0, w, st); break;
    default: return fail(FGMM_ERR_UNSUPPORTED, "tcgen05 family: d > 128");
  }
  if (rc) return rc;
  {
    const float *Xc = X + n0 * p.d;
    const int blocks = refine_blocks(c.Nc, p.d);
    const int dpl = (p.d + 7) / 8;
    const bool vec = p.d % 32 == 0 && reinterpret_cast<uintptr_t>(Xc) % 16 == 0;  // d = 8 DPL
    const int acc = first ? 0 : 1;
#define FGMM_REFINE(D)                                                                             \
  do {                                                                                             \
    if (vec && (D) % 4 == 0 && 8 * (D) == p.d)                                                     \
      FGMM_CUDA_TRY(launch_pdl(tc_refine_kernel<D, true>, blocks, 256, 0, st, Xc, c.Nc, p.d, w.sc, \
                               w.mu, w.lc, w.part_m, w.part_s, w.part_tv, w.part_ti, c.G, w.ln2x,  \
                               w.top_i, w.top_d, w.xmask, w.msl, ln + n0, w.ln_part, acc));        \
    else                                                                                           \
      FGMM_CUDA_TRY(launch_pdl(tc_refine_kernel<D, false>, blocks, 256, 0, st, Xc, c.Nc, p.d, w.sc,\
                               w.mu, w.lc, w.part_m, w.part_s, w.part_tv, w.part_ti, c.G, w.ln2x,  \
                               w.top_i, w.top_d, w.xmask, w.msl, ln + n0, w.ln_part, acc));        \
  } while (0)
#define FGMM_REFINE_ITEMS(D)                                                                       \
  do {                                                                                             \
    const int ib = blocks;                                                                         \
    if (vec && (D) % 4 == 0 && 8 * (D) == p.d)                                                     \
      FGMM_CUDA_TRY(launch_pdl(tc_refine_items_kernel<D, true>, ib, 32 * kRefWarps, 0, st, Xc,     \
                               c.Nc, p.d, w.sc, w.mu, w.lc, w.part_m, w.part_s, w.part_tv,         \
                               w.part_ti, c.G, w.ln2x, w.top_i, w.top_d, w.xmask, w.msl, ln + n0,  \
                               w.ln_part, acc));                                                   \
    else                                                                                           \
      FGMM_CUDA_TRY(launch_pdl(tc_refine_items_kernel<D, false>, ib, 32 * kRefWarps, 0, st, Xc,    \
                               c.Nc, p.d, w.sc, w.mu, w.lc, w.part_m, w.part_s, w.part_tv,         \
                               w.part_ti, c.G, w.ln2x, w.top_i, w.top_d, w.xmask, w.msl, ln + n0,  \
                               w.ln_part, acc));                                                   \
  } while (0)
    if (dpl <= 1) FGMM_REFINE_ITEMS(1);
    else if (dpl <= 2) FGMM_REFINE_ITEMS(2);
    else if (dpl <= 4) FGMM_REFINE_ITEMS(4);
    else if (dpl <= 8) FGMM_REFINE_ITEMS(8);
    else if (dpl <= 12) FGMM_REFINE(12);
    else FGMM_REFINE(16);
#undef FGMM_REFINE_ITEMS
#undef FGMM_REFINE
    FGMM_LAUNCH_CHECK("tc_refine_kernel");
    mark(st, "tc_refine_kernel");
  }
  switch (p.nkcf) {
    case 1: return launch_stats<1>(p, c, pp, n0, w, first, st);
    case 2: return launch_stats<2>(p, c, pp, n0, w, first, st);
    case 3: return launch_stats<3>(p, c, pp, n0, w, first, st);
    case 4: return launch_stats<4>(p, c, pp, n0, w, first, st);
    default: return fail(FGMM_ERR_UNSUPPORTED, "tcgen05 family: d > 128");
  }
}

}  // namespace

int tc_launches(int64_t N, int d, int K) { return 2 + 3 * plan(N, d, K).chunks; }

bool tc_supported(int64_t N, int d, int K) { return N >= 1 && K >= 1 && d >= 1 && d <= kMaxD; }

size_t tc_points_bytes(int64_t N, int d) {
  return kPtsHeader + 2 * (p_elems(N, d) + f_elems(N, d)) * sizeof(__half);
}

size_t tc_workspace_bytes(int64_t N, int d, int K) { return tc_layout(nullptr, plan(N, d, K)).bytes; }

int tc_prepare_points(const float *X, int64_t N, int d, void *points, cudaStream_t st) {
  const PtsPtrs pp = pts_ptrs(points, N, d);
  FGMM_CUDA_TRY(cudaMemsetAsync(points, 0, kPtsHeader, st));
  const int sms = num_sms();
  {
    const int64_t blocks = std::min<int64_t>(cdiv(N, 32), 8 * sms);  // 64 warps per SM
    const int64_t rows = cdiv(N, blocks);
    tc_xmax_kernel<<<(unsigned)cdiv(N, rows), 256, 0, st>>>(X, N, d, rows, pp.xmax);
  }
  FGMM_LAUNCH_CHECK("tc_xmax_kernel");
  const int kbp = tc_kbp(d), ka = 2 * tc_dp(d);
  if (d % 64 == 0 && reinterpret_cast<uintptr_t>(X) % 16 == 0) {  // kbp == 3 d, ka == 2 d
    const int rpp = 256 / (d / 4);
    const int blocks = (int)std::min<int64_t>(cdiv(npad_of(N), rpp), 8 * sms);
    tc_prep_points_q_kernel<<<blocks, 256, 0, st>>>(X, N, npad_of(N), d, pp.xmax,
                                                    const_cast<int *>(pp.aexp), pp.phi, pp.plo,
                                                    pp.fhi, pp.flo);
    FGMM_LAUNCH_CHECK("tc_prep_points_q_kernel");
    return FGMM_OK;
  }
  const int blocks = (int)std::min<int64_t>(npad_of(N) / kPrepRows, 8 * sms);
  tc_prep_points_kernel<<<blocks, 256, tc_prep_smem(kbp, ka, d), st>>>(X, N, npad_of(N), d, kbp, ka, pp.xmax,
                                                const_cast<int *>(pp.aexp), pp.phi, pp.plo, pp.fhi,
                                                pp.flo);
  FGMM_LAUNCH_CHECK("tc_prep_points_kernel");
  return FGMM_OK;
}

int tc_em_stats(const float *X, const void *points, int64_t N, int d, const float *mu,
                const float *var, const float *log_pi, int K, double *stats, float *log_norm,
                void *ws, cudaStream_t st, const UpdateOut *update, bool prepared) {
  const TcPlan p = plan(N, d, K);
  const TcWs w = tc_layout(ws, p);
  const PtsPtrs pp = pts_ptrs(points, N, d);
  const TcParamOps ops = param_ops(w, p, points);
  // `prepared`: the workspace already holds the operands of (mu, var, log_pi), written by
  // the previous call's fused update
  if (!prepared) {
    FGMM_CUDA_TRY(launch_pdl(tc_prep_params_kernel, p.Kp, 128, 0, st, mu, var, log_pi, K, d, ops));
    mark(st, "tc_prep_params_kernel");
  }
  UpdateOut up{};
  if (update) {  // the update also prepares the next iteration's operands
    up = *update;
    up.tc = ops;
  }
  for (int i = 0; i < p.chunks; ++i) {
    const int64_t n0 = (int64_t)i * p.Nc;
    const int64_t nc = std::min<int64_t>(p.Nc, p.N - n0);
    const TcChunk c = nc == p.first.Nc ? p.first : chunk_plan(nc, p.n_ct, p.n_ct2);
    const int rc = tc_launch_chunk(p, c, n0, i == 0, X, pp, w, log_norm, st);
    if (rc) return rc;
  }
  return reduce_partials(w.partial, p.first.S, K, d, p.dp, 2 * p.dp + 4, w.ln_part,
                         refine_blocks(p.first.Nc, p.d), stats, st, update ? &up : nullptr);
}

int tc_update_prepare(const double *stats, double n_total, const void *points, int64_t N, int d,
                      int K, float *new_mu, float *new_var, float *new_log_pi, void *ws,
                      cudaStream_t st) {
  const TcPlan p = plan(N, d, K);
  const TcWs w = tc_layout(ws, p);
  return em_update_prep(stats, n_total, K, p.Kp, d, new_mu, new_var, new_log_pi,
                        param_ops(w, p, points), st);
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
