/*
 * gfield_oracle.c -- CPU restatement of GUASS's cuda_field renderer.
 *
 * TEST INFRASTRUCTURE ONLY: this file is the checker that the CUDA product
 * path (guass_b200/csrc) is compared against, and the "port" CPU baseline
 * timed by bench.py.  Nothing in guass_b200/ links or imports it.
 *
 * Floating-point model.  The reference kernels are compiled by nvcc with its
 * default floating-point contraction (-fmad=true), so some a*b+c
 * expressions become single fused multiply-adds.  This file is compiled with
 * -ffp-contract=off and writes those fused operations out explicitly with
 * fmaf(), so the operation sequence is pinned independent of the host
 * compiler.  Which expressions nvcc fuses is established on the GPU by the
 * parity tests against the reference's own extension (oracle/_ref), not by
 * reading compiler output.  expf/log1pf/sqrtf come from the host libm; CUDA's
 * expf/log1pf may differ from them by an ulp, which the tests' tolerances
 * cover.
 *
 * Reductions in gfo_backward accumulate in double: the reference reduces in
 * an order that depends on its launch shape (CTA tree + CUB reduce-by-key),
 * so the checker uses an order-insensitive accumulation and the tests
 * compare with a stated tolerance.
 */
#include "gfield_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* forward.cu:15-17 / backward.cu:16-18 */
#define GFO_CHOLESKY_EPS 1e-5f
#define GFO_COV_FLOOR 1e-8f
#define GFO_TWO_PI 6.28318530717958647692

int gfo_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void gfo_set_threads(int n) {
#ifdef _OPENMP
  if (n >= 1) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* forward.cu:25-27 (softplus_stable_scalar). */
static float softplus_stable(float x) {
  return log1pf(expf(-fabsf(x))) + fmaxf(x, 0.0f);
}

/* backward.cu:28-30 */
static float sigmoid_scalar(float x) { return 1.0f / (1.0f + expf(-x)); }

/* CUDA float->int64 conversion (cvt.rzi.s64.f32) saturates and maps NaN to
 * 0; C leaves those cases undefined, so spell them out. */
static int64_t f2i64_rz(float x) {
  if (x != x) return 0;
  if (x >= 9.2233720368547758e18f) return INT64_MAX;
  if (x <= -9.2233720368547758e18f) return INT64_MIN;
  return (int64_t)x;
}

static int64_t clamp_i64(int64_t v, int64_t lo, int64_t hi) {
  return v < lo ? lo : (v > hi ? hi : v);
}

static int64_t max_i64(int64_t a, int64_t b) { return a > b ? a : b; }

/* forward.cu:134-209 (preprocess_geometry_kernel), one Gaussian. */
static void preprocess_one(int64_t idx, int64_t out_features,
                           int64_t in_features, int64_t tile_out,
                           int64_t tile_in, int64_t num_tile_rows,
                           int64_t num_tile_cols, float sigma,
                           const float* mu, const float* chol_raw,
                           float* inv_cov, float* det_out, int64_t* r0,
                           int64_t* r1, int64_t* c0, int64_t* c1,
                           int64_t* touched) {
  const float mu_row = mu[idx * 2 + 0];
  const float mu_col = mu[idx * 2 + 1];
  const float raw11 = chol_raw[idx * 3 + 0];
  const float raw21 = chol_raw[idx * 3 + 1];
  const float raw22 = chol_raw[idx * 3 + 2];

  const float l11 = softplus_stable(raw11) + GFO_CHOLESKY_EPS;
  const float l21 = raw21;
  const float l22 = softplus_stable(raw22) + GFO_CHOLESKY_EPS;

  const float cov00 = l11 * l11;
  const float cov01 = l11 * l21;
  const float cov11 = fmaf(l21, l21, l22 * l22);           /* :170 */
  const float det = fmaxf(fmaf(cov00, cov11, -(cov01 * cov01)),
                          GFO_COV_FLOOR);                   /* :171 */

  inv_cov[idx * 4 + 0] = cov11 / det;
  inv_cov[idx * 4 + 1] = -cov01 / det;
  inv_cov[idx * 4 + 2] = -cov01 / det;
  inv_cov[idx * 4 + 3] = cov00 / det;
  det_out[idx] = det;

  const float std_row = sqrtf(fmaxf(cov00, GFO_COV_FLOOR));
  const float std_col = sqrtf(fmaxf(cov11, GFO_COV_FLOOR));
  const float row_scale = 0.5f * (float)max_i64(out_features - 1, 1);
  const float col_scale = 0.5f * (float)max_i64(in_features - 1, 1);
  const float row_a = mu_row + 1.0f;
  const float col_a = mu_col + 1.0f;
  const float row_radius = (sigma * std_row) * row_scale;
  const float col_radius = (sigma * std_col) * col_scale;

  /* :189-192, center = a*scale fused into the +/- radius. */
  int64_t row_min = f2i64_rz(floorf(fmaf(row_a, row_scale, -row_radius)));
  int64_t row_max = f2i64_rz(ceilf(fmaf(row_a, row_scale, row_radius)));
  int64_t col_min = f2i64_rz(floorf(fmaf(col_a, col_scale, -col_radius)));
  int64_t col_max = f2i64_rz(ceilf(fmaf(col_a, col_scale, col_radius)));

  row_min = max_i64(0, row_min < out_features - 1 ? row_min : out_features - 1);
  row_max = max_i64(0, row_max < out_features - 1 ? row_max : out_features - 1);
  col_min = max_i64(0, col_min < in_features - 1 ? col_min : in_features - 1);
  col_max = max_i64(0, col_max < in_features - 1 ? col_max : in_features - 1);

  const int64_t tr0 = clamp_i64(row_min / tile_out, 0, num_tile_rows - 1);
  const int64_t tr1 = clamp_i64(row_max / tile_out, 0, num_tile_rows - 1);
  const int64_t tc0 = clamp_i64(col_min / tile_in, 0, num_tile_cols - 1);
  const int64_t tc1 = clamp_i64(col_max / tile_in, 0, num_tile_cols - 1);
  r0[idx] = tr0;
  r1[idx] = tr1;
  c0[idx] = tc0;
  c1[idx] = tc1;
  touched[idx] = (tr1 - tr0 + 1) * (tc1 - tc0 + 1);
}

void gfo_preprocess(int64_t out_features, int64_t in_features, int64_t k,
                    int64_t tile_out, int64_t tile_in, double sigma_multiplier,
                    const float* mu, const float* chol_raw, float* inv_cov,
                    float* det_cov, int64_t* r0, int64_t* r1, int64_t* c0,
                    int64_t* c1, int64_t* tiles_touched) {
  const int64_t ntr = (out_features + tile_out - 1) / tile_out;
  const int64_t ntc = (in_features + tile_in - 1) / tile_in;
  const float sigma = (float)sigma_multiplier;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < k; ++i) {
    preprocess_one(i, out_features, in_features, tile_out, tile_in, ntr, ntc,
                   sigma, mu, chol_raw, inv_cov, det_cov, r0, r1, c0, c1,
                   tiles_touched);
  }
}

int64_t gfo_count_pairs(int64_t k, const int64_t* tiles_touched) {
  int64_t total = 0;
  for (int64_t i = 0; i < k; ++i) total += tiles_touched[i];
  return total;
}

/*
 * forward.cu:211-241 emits (tile_key, gaussian_id) pairs in ascending id
 * order, :481-482 sorts them with a stable radix sort on the key, :243-252
 * and :483-493 turn the sorted keys into tile_ptr.  A stable counting sort on
 * the tile key yields the identical permutation.
 */
void gfo_bin(int64_t k, int64_t num_tile_rows, int64_t num_tile_cols,
             const int64_t* r0, const int64_t* r1, const int64_t* c0,
             const int64_t* c1, int64_t* tile_ptr, int64_t* ids_sorted) {
  const int64_t num_tiles = num_tile_rows * num_tile_cols;
  memset(tile_ptr, 0, sizeof(int64_t) * (size_t)(num_tiles + 1));
  for (int64_t g = 0; g < k; ++g)
    for (int64_t tr = r0[g]; tr <= r1[g]; ++tr)
      for (int64_t tc = c0[g]; tc <= c1[g]; ++tc)
        tile_ptr[tr * num_tile_cols + tc + 1] += 1;
  for (int64_t t = 0; t < num_tiles; ++t) tile_ptr[t + 1] += tile_ptr[t];
  int64_t* cursor = (int64_t*)malloc(sizeof(int64_t) * (size_t)(num_tiles + 1));
  memcpy(cursor, tile_ptr, sizeof(int64_t) * (size_t)(num_tiles + 1));
  for (int64_t g = 0; g < k; ++g)
    for (int64_t tr = r0[g]; tr <= r1[g]; ++tr)
      for (int64_t tc = c0[g]; tc <= c1[g]; ++tc)
        ids_sorted[cursor[tr * num_tile_cols + tc]++] = g;
  free(cursor);
}

/* forward.cu:316-367: per element, Gaussians accumulated in sorted order. */
void gfo_forward(int64_t out_features, int64_t in_features, int64_t tile_out,
                 int64_t tile_in, const float* row_coords,
                 const float* col_coords, const float* mu, const float* amp,
                 const float* inv_cov, const float* det_cov,
                 const int64_t* tile_ptr, const int64_t* ids_sorted,
                 int normalize, int has_clamp_quad, double clamp_quad,
                 float* delta) {
  const int64_t ntr = (out_features + tile_out - 1) / tile_out;
  const int64_t ntc = (in_features + tile_in - 1) / tile_in;
  const int64_t num_tiles = ntr * ntc;
  const float clampf = (float)clamp_quad;
  /* forward.cu:530: delta starts at zero; tiles with no pairs stay zero. */
  memset(delta, 0, sizeof(float) * (size_t)(out_features * in_features));
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t t = 0; t < num_tiles; ++t) {
    const int64_t start = tile_ptr[t], end = tile_ptr[t + 1];
    if (end <= start) continue;
    const int64_t row_start = (t / ntc) * tile_out;
    const int64_t col_start = (t % ntc) * tile_in;
    const int64_t row_end = row_start + tile_out < out_features ? row_start + tile_out : out_features;
    const int64_t col_end = col_start + tile_in < in_features ? col_start + tile_in : in_features;
    for (int64_t r = row_start; r < row_end; ++r) {
      const float cr = row_coords[r];
      for (int64_t c = col_start; c < col_end; ++c) {
        const float cc = col_coords[c];
        float value = 0.0f;
        for (int64_t p = start; p < end; ++p) {
          const int64_t g = ids_sorted[p];
          const float* A = inv_cov + g * 4;
          const float dx = cr - mu[g * 2 + 0];
          const float dy = cc - mu[g * 2 + 1];
          /* :349-350 */
          float quad = fmaf(dx, fmaf(A[0], dx, A[1] * dy),
                            dy * fmaf(A[2], dx, A[3] * dy));
          quad = fmaxf(quad, 0.0f);
          if (has_clamp_quad) quad = fminf(quad, clampf);
          float basis = expf(-0.5f * quad);
          if (normalize) {
            const float d = fmaxf(det_cov[g], GFO_COV_FLOOR);
            basis *= 1.0f / ((float)GFO_TWO_PI * sqrtf(d));
          }
          value = fmaf(amp[g], basis, value); /* :361 */
        }
        delta[r * in_features + c] = value;
      }
    }
  }
}

/* backward.cu:234-388 for one pair, accumulating its 8 partial sums. */
static void pair_partials(int64_t t, int64_t g, int64_t out_features,
                          int64_t in_features, int64_t tile_out,
                          int64_t tile_in, int64_t ntc, const float* grad,
                          const float* row_coords, const float* col_coords,
                          const float* mu, const float* amp,
                          const float* inv_cov, const float* det_cov,
                          int normalize, int has_clamp_quad, float clampf,
                          double out[8], double out_abs[8]) {
  const int64_t row_start = (t / ntc) * tile_out;
  const int64_t col_start = (t % ntc) * tile_in;
  const int64_t row_end = row_start + tile_out < out_features ? row_start + tile_out : out_features;
  const int64_t col_end = col_start + tile_in < in_features ? col_start + tile_in : in_features;
  const float mu_row = mu[g * 2 + 0], mu_col = mu[g * 2 + 1];
  const float a = amp[g];
  const float i00 = inv_cov[g * 4 + 0], i01 = inv_cov[g * 4 + 1];
  const float i10 = inv_cov[g * 4 + 2], i11 = inv_cov[g * 4 + 3];
  const float det = det_cov[g];
  double acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  double mag[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int64_t r = row_start; r < row_end; ++r) {
    for (int64_t c = col_start; c < col_end; ++c) {
      const float go = grad[r * in_features + c];
      if (go == 0.0f) continue; /* :309-311 */
      const float dx = row_coords[r] - mu_row;
      const float dy = col_coords[c] - mu_col;
      float quad = fmaf(dx, fmaf(i00, dx, i01 * dy), dy * fmaf(i10, dx, i11 * dy));
      quad = fmaxf(quad, 0.0f);
      int q_active = 1;
      if (has_clamp_quad && quad >= clampf) { /* :318-321 */
        quad = clampf;
        q_active = 0;
      }
      float basis = expf(-0.5f * quad);
      if (normalize) {
        const float sd = fmaxf(det, GFO_COV_FLOOR);
        basis *= 1.0f / ((float)GFO_TWO_PI * sqrtf(sd));
      }
      float term[8];
      int nterm = 1;
      term[0] = go * basis;
      const float common = go * a * basis;
      term[7] = 0.0f;
      if (normalize) {
        const float sd = fmaxf(det, GFO_COV_FLOOR);
        term[7] = common * (-0.5f / sd);
      }
      if (q_active) {
        const float coeff = common * -0.5f;
        const float sym01 = i01 + i10;
        /* :338-339 as the reference's nvcc build contracts them (one fma,
         * the dy product inside it); tests/test_gpu_reference_ext.py pins this
         * rounding against the reference extension on single-element fields */
        const float dq0 = -fmaf(sym01, dy, 2.0f * i00 * dx);
        const float dq1 = -fmaf(2.0f * i11, dy, sym01 * dx);
        const float dxdy = dx * dy;
        term[1] = coeff * dq0;
        term[2] = coeff * dq1;
        term[3] = coeff * dx * dx;
        term[4] = coeff * dxdy;
        term[5] = coeff * dxdy;
        term[6] = coeff * dy * dy;
        nterm = 7;
      }
      for (int j = 0; j < nterm; ++j) {
        acc[j] += (double)term[j];
        mag[j] += fabs((double)term[j]);
      }
      acc[7] += (double)term[7];
      mag[7] += fabs((double)term[7]);
    }
  }
  memcpy(out, acc, sizeof(acc));
  if (out_abs) memcpy(out_abs, mag, sizeof(mag));
}

/* backward.cu:436-496 (cov_chain_to_chol_raw_kernel), one Gaussian. */
static void cov_chain(const float* chol_raw_g, const float* inv, float det,
                      const float gi[4], float gdet, float out[3]) {
  const float raw11 = chol_raw_g[0], raw21 = chol_raw_g[1], raw22 = chol_raw_g[2];
  const float l11 = softplus_stable(raw11) + GFO_CHOLESKY_EPS;
  const float l21 = raw21;
  const float l22 = softplus_stable(raw22) + GFO_CHOLESKY_EPS;
  const float at00 = inv[0], at01 = inv[2], at10 = inv[1], at11 = inv[3];
  const float b00 = gi[0] * at00 + gi[1] * at10;
  const float b01 = gi[0] * at01 + gi[1] * at11;
  const float b10 = gi[2] * at00 + gi[3] * at10;
  const float b11 = gi[2] * at01 + gi[3] * at11;
  float g00 = -(at00 * b00 + at01 * b10);
  float g01 = -(at00 * b01 + at01 * b11);
  float g10 = -(at10 * b00 + at11 * b10);
  float g11 = -(at10 * b01 + at11 * b11);
  g00 += gdet * det * at00;
  g01 += gdet * det * at01;
  g10 += gdet * det * at10;
  g11 += gdet * det * at11;
  const float d_l11 = g00 * (2.0f * l11) + g01 * l21 + g10 * l21;
  const float d_l21 = g01 * l11 + g10 * l11 + g11 * (2.0f * l21);
  const float d_l22 = g11 * (2.0f * l22);
  out[0] = d_l11 * sigmoid_scalar(raw11);
  out[1] = d_l21;
  out[2] = d_l22 * sigmoid_scalar(raw22);
}

void gfo_backward(int64_t out_features, int64_t in_features, int64_t k,
                  int64_t tile_out, int64_t tile_in, double sigma_multiplier,
                  const float* grad, const float* row_coords,
                  const float* col_coords, const float* mu,
                  const float* chol_raw, const float* amp,
                  const int64_t* tile_ptr, const int64_t* ids_sorted,
                  int64_t num_pairs, int normalize, int has_clamp_quad,
                  double clamp_quad, float* d_mu, float* d_chol_raw,
                  float* d_amp) {
  const int64_t ntr = (out_features + tile_out - 1) / tile_out;
  const int64_t ntc = (in_features + tile_in - 1) / tile_in;
  const int64_t num_tiles = ntr * ntc;
  float* inv = (float*)malloc(sizeof(float) * (size_t)(k * 4 + 1));
  float* det = (float*)malloc(sizeof(float) * (size_t)(k + 1));
  int64_t* box = (int64_t*)malloc(sizeof(int64_t) * (size_t)(k * 5 + 1));
  /* backward.cu:552-557 rebuilds the geometry from the saved inputs. */
  gfo_preprocess(out_features, in_features, k, tile_out, tile_in,
                 sigma_multiplier, mu, chol_raw, inv, det, box, box + k,
                 box + 2 * k, box + 3 * k, box + 4 * k);
  /* fill_pair_tile_ids_range_kernel (backward.cu:209-232). */
  int64_t* pair_tile = (int64_t*)malloc(sizeof(int64_t) * (size_t)(num_pairs + 1));
  for (int64_t t = 0; t < num_tiles; ++t)
    for (int64_t p = tile_ptr[t]; p < tile_ptr[t + 1] && p < num_pairs; ++p)
      pair_tile[p] = t;
  double* part = (double*)malloc(sizeof(double) * 8 * (size_t)(num_pairs + 1));
  const float clampf = (float)clamp_quad;
#pragma omp parallel for schedule(dynamic, 4)
  for (int64_t p = 0; p < num_pairs; ++p) {
    pair_partials(pair_tile[p], ids_sorted[p], out_features, in_features,
                  tile_out, tile_in, ntc, grad, row_coords, col_coords, mu,
                  amp, inv, det, normalize, has_clamp_quad, clampf,
                  part + 8 * p, NULL);
  }
  /* reduce-by-key + scatter (backward.cu:635-701): sum partials per id. */
  double* sum = (double*)calloc((size_t)(k * 8 + 1), sizeof(double));
  for (int64_t p = 0; p < num_pairs; ++p) {
    const int64_t g = ids_sorted[p];
    for (int j = 0; j < 8; ++j) sum[g * 8 + j] += part[8 * p + j];
  }
  for (int64_t g = 0; g < k; ++g) {
    const double* s = sum + g * 8;
    d_amp[g] = (float)s[0];
    d_mu[g * 2 + 0] = (float)s[1];
    d_mu[g * 2 + 1] = (float)s[2];
    const float gi[4] = {(float)s[3], (float)s[4], (float)s[5], (float)s[6]};
    cov_chain(chol_raw + g * 3, inv + g * 4, det[g], gi, (float)s[7],
              d_chol_raw + g * 3);
  }
  free(sum);
  free(part);
  free(pair_tile);
  free(box);
  free(det);
  free(inv);
}

/*
 * Checker variant of gfo_backward: the same float per-element terms, but the
 * reductions and the covariance chain are evaluated in double, and for every
 * output it also returns S, the same computation applied to the absolute
 * values of the summands.  A float implementation that sums in another order
 * (or evaluates the chain in float) differs from the double result by a small
 * multiple of u*S; S >> |result| marks an ill-conditioned output (the chain
 * -A*G*A cancels for elongated Gaussians), where no fp32 ordering can agree
 * to 1e-5 of the result itself.
 */
void gfo_backward_f64(int64_t out_features, int64_t in_features, int64_t k,
                      int64_t tile_out, int64_t tile_in, double sigma_multiplier,
                      const float* grad, const float* row_coords,
                      const float* col_coords, const float* mu,
                      const float* chol_raw, const float* amp,
                      const int64_t* tile_ptr, const int64_t* ids_sorted,
                      int64_t num_pairs, int normalize, int has_clamp_quad,
                      double clamp_quad, double* d_mu, double* d_chol_raw,
                      double* d_amp, double* s_mu, double* s_chol_raw,
                      double* s_amp, const float* geo_inv,
                      const float* geo_det) {
  const int64_t ntr = (out_features + tile_out - 1) / tile_out;
  const int64_t ntc = (in_features + tile_in - 1) / tile_in;
  const int64_t num_tiles = ntr * ntc;
  float* inv = (float*)malloc(sizeof(float) * (size_t)(k * 4 + 1));
  float* det = (float*)malloc(sizeof(float) * (size_t)(k + 1));
  int64_t* box = (int64_t*)malloc(sizeof(int64_t) * (size_t)(k * 5 + 1));
  gfo_preprocess(out_features, in_features, k, tile_out, tile_in,
                 sigma_multiplier, mu, chol_raw, inv, det, box, box + k,
                 box + 2 * k, box + 3 * k, box + 4 * k);
  if (geo_inv) memcpy(inv, geo_inv, sizeof(float) * (size_t)(k * 4));
  if (geo_det) memcpy(det, geo_det, sizeof(float) * (size_t)k);
  int64_t* pair_tile = (int64_t*)malloc(sizeof(int64_t) * (size_t)(num_pairs + 1));
  for (int64_t t = 0; t < num_tiles; ++t)
    for (int64_t p = tile_ptr[t]; p < tile_ptr[t + 1] && p < num_pairs; ++p)
      pair_tile[p] = t;
  double* part = (double*)malloc(sizeof(double) * 16 * (size_t)(num_pairs + 1));
  const float clampf = (float)clamp_quad;
#pragma omp parallel for schedule(dynamic, 4)
  for (int64_t p = 0; p < num_pairs; ++p) {
    pair_partials(pair_tile[p], ids_sorted[p], out_features, in_features,
                  tile_out, tile_in, ntc, grad, row_coords, col_coords, mu,
                  amp, inv, det, normalize, has_clamp_quad, clampf,
                  part + 16 * p, part + 16 * p + 8);
  }
  double* sum = (double*)calloc((size_t)(k * 16 + 1), sizeof(double));
  for (int64_t p = 0; p < num_pairs; ++p) {
    const int64_t g = ids_sorted[p];
    for (int j = 0; j < 16; ++j) sum[g * 16 + j] += part[16 * p + j];
  }
  for (int64_t g = 0; g < k; ++g) {
    const double* v = sum + g * 16;
    const double* m = v + 8;
    d_amp[g] = v[0];
    s_amp[g] = m[0];
    d_mu[g * 2 + 0] = v[1];
    d_mu[g * 2 + 1] = v[2];
    s_mu[g * 2 + 0] = m[1];
    s_mu[g * 2 + 1] = m[2];
    const float* cr = chol_raw + g * 3;
    const double l11 = (double)(softplus_stable(cr[0]) + GFO_CHOLESKY_EPS);
    const double l21 = (double)cr[1];
    const double l22 = (double)(softplus_stable(cr[2]) + GFO_CHOLESKY_EPS);
    const double A[2][2] = {{inv[g * 4 + 0], inv[g * 4 + 1]}, {inv[g * 4 + 2], inv[g * 4 + 3]}};
    const double G[2][2] = {{v[3], v[4]}, {v[5], v[6]}};
    const double M[2][2] = {{m[3], m[4]}, {m[5], m[6]}};
    const double dt = (double)det[g];
    double gc[2][2], sc[2][2];
    for (int i = 0; i < 2; ++i)
      for (int j = 0; j < 2; ++j) {
        double acc = 0.0, mag = 0.0;
        /* dSigma = -A^T G A^T (A symmetric) + gdet * det * A^T */
        for (int a = 0; a < 2; ++a)
          for (int b = 0; b < 2; ++b) {
            acc += A[a][i] * G[a][b] * A[j][b];
            mag += fabs(A[a][i]) * M[a][b] * fabs(A[j][b]);
          }
        gc[i][j] = -acc + v[7] * dt * A[j][i];
        sc[i][j] = mag + m[7] * fabs(dt * A[j][i]);
      }
    const double sg0 = 1.0 / (1.0 + exp(-(double)cr[0]));
    const double sg2 = 1.0 / (1.0 + exp(-(double)cr[2]));
    d_chol_raw[g * 3 + 0] = (gc[0][0] * 2.0 * l11 + (gc[0][1] + gc[1][0]) * l21) * sg0;
    d_chol_raw[g * 3 + 1] = (gc[0][1] + gc[1][0]) * l11 + gc[1][1] * 2.0 * l21;
    d_chol_raw[g * 3 + 2] = gc[1][1] * 2.0 * l22 * sg2;
    s_chol_raw[g * 3 + 0] = (sc[0][0] * 2.0 * fabs(l11) + (sc[0][1] + sc[1][0]) * fabs(l21)) * sg0;
    s_chol_raw[g * 3 + 1] = (sc[0][1] + sc[1][0]) * fabs(l11) + sc[1][1] * 2.0 * fabs(l21);
    s_chol_raw[g * 3 + 2] = sc[1][1] * 2.0 * fabs(l22) * sg2;
  }
  free(sum);
  free(part);
  free(pair_tile);
  free(box);
  free(det);
  free(inv);
}
