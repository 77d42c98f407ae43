// Operand formats of the tensor-core family (shared by fgmm_tc.cu and fgmm_update.cu).
//
// The distance GEMM evaluates the Mahalanobis sum as ONE dot product per (point,
// component) over 3 d columns, one triple per dimension j:
//   P[n] = [.., x_j^2, x_j, 1, ..],   Q[k] = [.., iv_kj, -2 mu_kj iv_kj, mu_kj^2 iv_kj, ..]
//   P[n] . Q[k] = sum_j iv_kj (x_nj - mu_kj)^2            (iv = 1 / var)
// so every triple adds a non-negative term and the running sum only grows towards the
// distance itself: the tensor-memory accumulation (which does not round to nearest)
// never works at the magnitude of |x|^2 / var, which is far larger than the distance
// it would otherwise cancel down to.  The statistics GEMM reads F[n] = [x^2 (dp) | x (dp)].
//
// Both operands are fp16 hi/lo pairs (v ~ hi + lo, 22 significant bits; the products
// lo.hi + hi.lo + hi.hi of kind::f16 MMAs carry them to fp32-level accuracy at twice the
// tf32 rate).  fp16 has a narrow exponent range, so every column is scaled by a power of
// two, which is exact: point column c by 2^a_c (a_c from the data's largest magnitude in
// that column, so every value is below 2^15), component row k additionally by 2^-E_k
// after the column scale 2^-a_c (E_k from the row's largest value).  The MMA result is
// then 2^-E_k times the distance; the epilogue's coefficient carries 2^E_k back.
#pragma once
#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>

namespace fgmm {

constexpr int kTcTop = 4;        // leading components per point evaluated exactly
constexpr int kTcColMax = 14;    // scaled magnitudes stay below 2^(kTcColMax + 1)
constexpr int kTcGammaExp = 14;  // responsibilities enter the statistics GEMM as gamma 2^14

// Prepared-points buffer: header, then P hi / lo [Npad][KBp] and F hi / lo [Npad][KA],
// all fp16 (KBp = 3 d rounded up to 64, KA = 2 dp, dp = d rounded up to 32).
constexpr size_t kPtsHeader = 4096;
constexpr size_t kPtsAexpOff = 0;     // int32 [KBp]: column exponents a_c of P
constexpr size_t kPtsXmaxOff = 2048;  // uint32 [d]: bit patterns of max |x_j| (non-negative)

__host__ __device__ inline int tc_kbp(int d) { return (3 * d + 63) / 64 * 64; }
__host__ __device__ inline int tc_dp(int d) { return (d + 31) / 32 * 32; }

// Exponent a of a column whose largest magnitude is `m` (>= 0): m 2^a < 2^(kTcColMax+1).
__device__ __forceinline__ int tc_col_exp(float m) {
  if (!(m > 0.0f) || !isfinite(m)) return 0;
  int e = ilogbf(m);
  e = kTcColMax - e;
  return e > 100 ? 100 : (e < -100 ? -100 : e);
}

// Exponent of P column c (c = 3 j + t) from max |x_j|.
__device__ __forceinline__ int tc_p_col_exp(int c, int d, const uint32_t *xmax_bits) {
  const int j = c / 3, t = c - 3 * j;
  if (j >= d) return 0;
  const float m = __uint_as_float(xmax_bits[j]);
  if (t == 0) return tc_col_exp(m * m);
  if (t == 1) return tc_col_exp(m);
  return kTcColMax;
}

__device__ __forceinline__ void split_f16(double v, __half &hi, __half &lo) {
  hi = __double2half(v);
  lo = __double2half(v - (double)__half2float(hi));
}

// Parameter-side operands of the tensor-core family for component k.
struct TcParamOps {
  __half *qhi = nullptr, *qlo = nullptr;  // [Kp][KBp]
  float *coef = nullptr;                  // [Kp]: -1/2 log2(e) 2^E_k
  float *cst2 = nullptr;                  // [Kp]: log2(e) (log_pi - 1/2 (d log 2pi + sum log var))
  float *sc = nullptr;                    // [K][d]: var^-1/2 (exact re-evaluation)
  float *mu = nullptr;                    // [K][d]: the means (fp32 copy)
  double *lc = nullptr;                   // [K]: log_pi - 1/2 (d log 2pi + sum log var), fp64
  const int *aexp = nullptr;              // [KBp]: column exponents of the prepared points
  int kbp = 0;                            // 0: not in use
};

// Writes component k's operands from its fp32 parameters.  Called by 128 threads of a
// block (thread j: dimension j, d <= 128), which must all arrive: `bar_id` is a named
// barrier reserved for them.  The fp64 arithmetic and its summation order are the same
// wherever it is called, so preparing the operands at the start of an iteration and
// writing them from the previous iteration's update give identical bits.
__device__ inline void tc_prep_component(int k, int K, int d, int j, float mu32, float var32,
                                         float lp32, const TcParamOps &op, int bar_id) {
  __shared__ double s_red[4];
  __shared__ int s_emax[4];
  const int lane = j & 31, w = j >> 5;
  const bool live = k < K && j < d;
  double q[3] = {0.0, 0.0, 0.0};
  double lv = 0.0;
  int e = -1000;
  if (live) {
    const double v = var32, m = mu32;
    const double iv = 1.0 / v;
    q[0] = iv;
    q[1] = -2.0 * m * iv;
    q[2] = m * m * iv;
    lv = log(v);
    op.sc[(int64_t)k * d + j] = (float)(1.0 / sqrt(v));
    op.mu[(int64_t)k * d + j] = mu32;
#pragma unroll
    for (int t = 0; t < 3; ++t) {
      q[t] = ldexp(q[t], -op.aexp[3 * j + t]);
      if (q[t] != 0.0) e = max(e, ilogb(q[t]));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lv += __shfl_xor_sync(0xffffffffu, lv, o);
    e = max(e, __shfl_xor_sync(0xffffffffu, e, o));
  }
  if (lane == 0) { s_red[w] = lv; s_emax[w] = e; }
  asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
  const int emax = max(max(s_emax[0], s_emax[1]), max(s_emax[2], s_emax[3]));
  const int E = emax == -1000 ? 0 : emax - kTcColMax;
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    const int c = 3 * j + t;
    if (c < op.kbp) {
      __half hi, lo;
      split_f16(ldexp(q[t], -E), hi, lo);
      op.qhi[(int64_t)k * op.kbp + c] = hi;
      op.qlo[(int64_t)k * op.kbp + c] = lo;
    }
  }
  if (j == 0) {
    const double t2 = s_red[0] + s_red[1] + s_red[2] + s_red[3];
    if (k < K) {
      const double lc = (double)lp32 - 0.5 * (d * 1.8378770664093453 + t2);
      op.lc[k] = lc;
      op.cst2[k] = (float)(1.4426950408889634 * lc);
      op.coef[k] = (float)ldexp(-0.5 * 1.4426950408889634, E);
    } else {
      op.cst2[k] = -INFINITY;
      op.coef[k] = 0.0f;
    }
  }
  asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");  // s_red / s_emax reusable
}

}  // namespace fgmm
