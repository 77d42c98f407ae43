/*
 * flashgmm_oracle.c -- CPU restatement of the reference's diagonal-covariance
 * EM path.  TEST INFRASTRUCTURE ONLY: this file is the checker that the CUDA
 * product is compared against and the "port" CPU baseline; nothing in the
 * shipped library links or calls it.
 *
 * Every function states the reference lines it follows (paths relative to the
 * reference project root).  The fp32 variants keep the reference's operation
 * order (per-element log-likelihood with logf inside the d-loop, online
 * log-sum-exp with the branchy update, per-thread statistics buffers reduced in
 * thread order) so that, with the same OpenMP thread count and the same libm,
 * they reproduce the reference's C++/OpenMP outputs bit for bit.  The fp64
 * variants run the same algorithm in double precision and serve as the
 * accuracy yardstick both fp32 paths are measured against.
 */
#include <math.h>
#include <float.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

#define LOG_2PI_F 1.8378770664093453f
#define LOG_2PI_D 1.8378770664093453

/* flash_gmm/csrc/flash_gmm_cpu.cpp:30-45 compute_log_likelihood */
static inline float ll_f32(const float *x, const float *mu, const float *var,
                           float log_pi, int d) {
    float log_det = 0.0f, mahal = 0.0f;
    for (int j = 0; j < d; j++) {
        log_det += logf(var[j]);
        float diff = x[j] - mu[j];
        mahal += diff * diff / var[j];
    }
    return log_pi - 0.5f * (d * LOG_2PI_F + log_det + mahal);
}

static inline double ll_f64(const float *x, const float *mu, const float *var,
                            float log_pi, int d) {
    double log_det = 0.0, mahal = 0.0;
    for (int j = 0; j < d; j++) {
        double v = (double)var[j];
        log_det += log(v);
        double diff = (double)x[j] - (double)mu[j];
        mahal += diff * diff / v;
    }
    return (double)log_pi - 0.5 * (d * LOG_2PI_D + log_det + mahal);
}

/* Pass 1 online log-sum-exp, flash_gmm/csrc/flash_gmm_cpu.cpp:199-219
 * (identical loop in flash_e_step_cpu, :129-151). */
static void pass1_f32(const float *X, int64_t N, int d, const float *mu,
                      const float *var, const float *lp, int K, int BK,
                      int nthreads, float *ln) {
    if (BK < 1) BK = 1;
    #pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t n = 0; n < N; n++) {
        float rm = -FLT_MAX, rs = 0.0f;
        for (int t = 0; t < K; t += BK) {
            int te = t + BK < K ? t + BK : K;
            for (int k = t; k < te; k++) {
                float ll = ll_f32(X + n * d, mu + (int64_t)k * d, var + (int64_t)k * d, lp[k], d);
                if (ll > rm) { rs = rs * expf(rm - ll) + 1.0f; rm = ll; }
                else         { rs += expf(ll - rm); }
            }
        }
        ln[n] = rm + logf(rs);
    }
}

/* flash_gmm/csrc/flash_gmm_cpu.cpp:177-287 flash_em_fused_cpu (fp32, bitwise order). */
void oracle_flash_em_fused_f32(const float *X, int64_t N, int d,
                               const float *mu, const float *var, const float *lp,
                               int K, int BK, int nthreads,
                               float *new_mu, float *new_var, float *new_lp,
                               float *ln) {
    if (nthreads < 1) nthreads = 1;
    if (BK < 1) BK = 1;
    pass1_f32(X, N, d, mu, var, lp, K, BK, nthreads, ln);

    /* Pass 2 with per-thread buffers, :221-254 */
    size_t kd = (size_t)K * d;
    float *all_n = (float *)calloc((size_t)nthreads * K, sizeof(float));
    float *all_s = (float *)calloc((size_t)nthreads * kd, sizeof(float));
    float *all_q = (float *)calloc((size_t)nthreads * kd, sizeof(float));
    #pragma omp parallel num_threads(nthreads)
    {
        int tid = omp_get_thread_num();
        float *ln_k = all_n + (size_t)tid * K;
        float *ls_k = all_s + (size_t)tid * kd;
        float *lq_k = all_q + (size_t)tid * kd;
        #pragma omp for schedule(static)
        for (int64_t n = 0; n < N; n++) {
            for (int t = 0; t < K; t += BK) {
                int te = t + BK < K ? t + BK : K;
                for (int k = t; k < te; k++) {
                    float ll = ll_f32(X + n * d, mu + (int64_t)k * d, var + (int64_t)k * d, lp[k], d);
                    float g = expf(ll - ln[n]);
                    ln_k[k] += g;
                    for (int j = 0; j < d; j++) {
                        float xv = X[n * d + j];
                        ls_k[(size_t)k * d + j] += g * xv;
                        lq_k[(size_t)k * d + j] += g * xv * xv;
                    }
                }
            }
        }
    }
    /* serial reduction in thread order, :256-268 */
    float *n_k = (float *)calloc(K, sizeof(float));
    float *s_k = (float *)calloc(kd, sizeof(float));
    float *q_k = (float *)calloc(kd, sizeof(float));
    for (int t = 0; t < nthreads; t++) {
        for (int k = 0; k < K; k++) n_k[k] += all_n[(size_t)t * K + k];
        for (size_t i = 0; i < kd; i++) {
            s_k[i] += all_s[(size_t)t * kd + i];
            q_k[i] += all_q[(size_t)t * kd + i];
        }
    }
    /* update, :270-284 */
    for (int k = 0; k < K; k++) {
        float inv = 1.0f / fmaxf(n_k[k], 1e-8f);
        for (int j = 0; j < d; j++) {
            float m = s_k[(size_t)k * d + j] * inv;
            new_mu[(size_t)k * d + j] = m;
            float v = q_k[(size_t)k * d + j] * inv - m * m;
            new_var[(size_t)k * d + j] = fmaxf(v, 1e-6f);
        }
        new_lp[k] = logf(fmaxf(n_k[k] / N, 1e-8f));
    }
    free(all_n); free(all_s); free(all_q); free(n_k); free(s_k); free(q_k);
}

/* Same algorithm as oracle_flash_em_fused_f32 in double precision; also returns
 * the raw sufficient statistics n_k[K], s_k[K*d], sq_k[K*d] (may be NULL). */
void oracle_flash_em_fused_f64(const float *X, int64_t N, int d,
                               const float *mu, const float *var, const float *lp,
                               int K, int nthreads,
                               double *new_mu, double *new_var, double *new_lp,
                               double *ln, double *n_out, double *s_out, double *q_out) {
    if (nthreads < 1) nthreads = 1;
    #pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t n = 0; n < N; n++) {
        double m = -DBL_MAX, s = 0.0;
        for (int k = 0; k < K; k++) {
            double ll = ll_f64(X + n * d, mu + (int64_t)k * d, var + (int64_t)k * d, lp[k], d);
            if (ll > m) { s = s * exp(m - ll) + 1.0; m = ll; }
            else        { s += exp(ll - m); }
        }
        ln[n] = m + log(s);
    }
    size_t kd = (size_t)K * d;
    double *all_n = (double *)calloc((size_t)nthreads * K, sizeof(double));
    double *all_s = (double *)calloc((size_t)nthreads * kd, sizeof(double));
    double *all_q = (double *)calloc((size_t)nthreads * kd, sizeof(double));
    #pragma omp parallel num_threads(nthreads)
    {
        int tid = omp_get_thread_num();
        double *ln_k = all_n + (size_t)tid * K;
        double *ls_k = all_s + (size_t)tid * kd;
        double *lq_k = all_q + (size_t)tid * kd;
        #pragma omp for schedule(static)
        for (int64_t n = 0; n < N; n++) {
            for (int k = 0; k < K; k++) {
                double ll = ll_f64(X + n * d, mu + (int64_t)k * d, var + (int64_t)k * d, lp[k], d);
                double g = exp(ll - ln[n]);
                ln_k[k] += g;
                for (int j = 0; j < d; j++) {
                    double xv = X[n * d + j];
                    ls_k[(size_t)k * d + j] += g * xv;
                    lq_k[(size_t)k * d + j] += g * xv * xv;
                }
            }
        }
    }
    double *n_k = (double *)calloc(K, sizeof(double));
    double *s_k = (double *)calloc(kd, sizeof(double));
    double *q_k = (double *)calloc(kd, sizeof(double));
    for (int t = 0; t < nthreads; t++) {
        for (int k = 0; k < K; k++) n_k[k] += all_n[(size_t)t * K + k];
        for (size_t i = 0; i < kd; i++) {
            s_k[i] += all_s[(size_t)t * kd + i];
            q_k[i] += all_q[(size_t)t * kd + i];
        }
    }
    for (int k = 0; k < K; k++) {
        double inv = 1.0 / fmax(n_k[k], 1e-8);
        for (int j = 0; j < d; j++) {
            double m = s_k[(size_t)k * d + j] * inv;
            new_mu[(size_t)k * d + j] = m;
            double v = q_k[(size_t)k * d + j] * inv - m * m;
            new_var[(size_t)k * d + j] = fmax(v, 1e-6);
        }
        new_lp[k] = log(fmax(n_k[k] / (double)N, 1e-8));
    }
    if (n_out) memcpy(n_out, n_k, K * sizeof(double));
    if (s_out) memcpy(s_out, s_k, kd * sizeof(double));
    if (q_out) memcpy(q_out, q_k, kd * sizeof(double));
    free(all_n); free(all_s); free(all_q); free(n_k); free(s_k); free(q_k);
}

/* flash_gmm/csrc/flash_gmm_cpu.cpp:51-100 standard_e_step_cpu: materialised L,
 * two-pass max / sum-exp per row, gamma = exp(L - ln). */
void oracle_standard_e_step_f32(const float *X, int64_t N, int d,
                                const float *mu, const float *var, const float *lp,
                                int K, int nthreads, float *gamma, float *ln) {
    if (nthreads < 1) nthreads = 1;
    #pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t n = 0; n < N; n++) {
        float *L = gamma + n * K;      /* L is staged in the gamma row */
        for (int k = 0; k < K; k++)
            L[k] = ll_f32(X + n * d, mu + (int64_t)k * d, var + (int64_t)k * d, lp[k], d);
        float mx = -FLT_MAX;
        for (int k = 0; k < K; k++) mx = L[k] > mx ? L[k] : mx;
        float se = 0.0f;
        for (int k = 0; k < K; k++) se += expf(L[k] - mx);
        float l = mx + logf(se);
        ln[n] = l;
        for (int k = 0; k < K; k++) L[k] = expf(L[k] - l);
    }
}

/* flash_gmm/csrc/flash_gmm_cpu.cpp:108-168 flash_e_step_cpu: pass 1 online LSE,
 * pass 2 recompute gamma = exp(ll - ln). */
void oracle_flash_e_step_f32(const float *X, int64_t N, int d,
                             const float *mu, const float *var, const float *lp,
                             int K, int BK, int nthreads, float *gamma, float *ln) {
    if (nthreads < 1) nthreads = 1;
    if (BK < 1) BK = 1;
    pass1_f32(X, N, d, mu, var, lp, K, BK, nthreads, ln);
    #pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t n = 0; n < N; n++)
        for (int k = 0; k < K; k++)
            gamma[n * K + k] = expf(ll_f32(X + n * d, mu + (int64_t)k * d,
                                           var + (int64_t)k * d, lp[k], d) - ln[n]);
}

/* flash_gmm/csrc/flash_gmm_cpu.cpp:292-311 standard_m_step_cpu.  The reference
 * uses ATen GEMMs (BLAS summation order); this restatement accumulates the
 * products in double and rounds once, so it agrees with the reference to fp32
 * rounding, not bit for bit.  Note the reference applies no floor to n_k here. */
void oracle_standard_m_step_f32(const float *X, int64_t N, int d,
                                const float *gamma, int K, int nthreads,
                                float *new_mu, float *new_var, float *new_lp) {
    if (nthreads < 1) nthreads = 1;
    #pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int k = 0; k < K; k++) {
        double nk = 0.0;
        for (int64_t n = 0; n < N; n++) nk += gamma[n * K + k];
        float nkf = (float)nk;
        for (int j = 0; j < d; j++) {
            double s = 0.0, q = 0.0;
            for (int64_t n = 0; n < N; n++) {
                double g = gamma[n * K + k], x = X[n * d + j];
                s += g * x;
                q += g * (double)((float)x * (float)x);
            }
            float m = (float)s / nkf;
            new_mu[(size_t)k * d + j] = m;
            float v = (float)q / nkf - m * m;
            new_var[(size_t)k * d + j] = v > 1e-6f ? v : 1e-6f;
        }
        new_lp[k] = logf(nkf / (float)N);
    }
}

int oracle_max_threads(void) { return omp_get_max_threads(); }
