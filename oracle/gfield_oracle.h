/*
 * gfield_oracle.h -- CPU restatement of GUASS's cuda_field Gaussian-field
 * renderer, used ONLY as a test checker and as the timed CPU baseline.
 *
 * This is test infrastructure. Product code (guass_b200/) never links it.
 *
 * Each function follows one part of the reference implementation
 * (paths relative to the GUASS project root):
 *   gfo_preprocess  gaussian_peft/cuda_field/csrc/forward.cu:134-209
 *   gfo_bin         gaussian_peft/cuda_field/csrc/forward.cu:211-252,428-511
 *   gfo_forward     gaussian_peft/cuda_field/csrc/forward.cu:254-368,513-569
 *   gfo_backward    gaussian_peft/cuda_field/csrc/backward.cu:234-388,541-716
 *                   (pair partials, reduce-by-key, cov chain :436-496)
 */
#ifndef GFIELD_ORACLE_H
#define GFIELD_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Per-Gaussian geometry: inv_cov [K*4] (row-major 2x2), det [K],
 * tile box r0,r1,c0,c1 and tiles_touched [K]. */
void gfo_preprocess(int64_t out_features, int64_t in_features, int64_t k,
                    int64_t tile_out, int64_t tile_in, double sigma_multiplier,
                    const float* mu, const float* chol_raw,
                    float* inv_cov, float* det_cov,
                    int64_t* r0, int64_t* r1, int64_t* c0, int64_t* c1,
                    int64_t* tiles_touched);

/* Number of (tile, gaussian) pairs = sum of tiles_touched. */
int64_t gfo_count_pairs(int64_t k, const int64_t* tiles_touched);

/* Stable binning: tile_ptr [T+1], gaussian_ids_sorted [P] (ascending id
 * inside each tile, tiles in row-major order). */
void gfo_bin(int64_t k, int64_t num_tile_rows, int64_t num_tile_cols,
             const int64_t* r0, const int64_t* r1, const int64_t* c0,
             const int64_t* c1, int64_t* tile_ptr, int64_t* ids_sorted);

/* Forward render of delta [out*in] fp32 (row-major [out,in]). */
void gfo_forward(int64_t out_features, int64_t in_features, int64_t tile_out,
                 int64_t tile_in, const float* row_coords,
                 const float* col_coords, const float* mu, const float* amp,
                 const float* inv_cov, const float* det_cov,
                 const int64_t* tile_ptr, const int64_t* ids_sorted,
                 int normalize, int has_clamp_quad, double clamp_quad,
                 float* delta);

/* Backward: grad [out*in] fp32 -> d_mu [K*2], d_chol_raw [K*3], d_amp [K].
 * Recomputes the geometry from mu/chol_raw exactly like the reference. */
void gfo_backward(int64_t out_features, int64_t in_features, int64_t k,
                  int64_t tile_out, int64_t tile_in, double sigma_multiplier,
                  const float* grad, const float* row_coords,
                  const float* col_coords, const float* mu,
                  const float* chol_raw, const float* amp,
                  const int64_t* tile_ptr, const int64_t* ids_sorted,
                  int64_t num_pairs, int normalize, int has_clamp_quad,
                  double clamp_quad, float* d_mu, float* d_chol_raw,
                  float* d_amp);

/* Checker variant: double reductions and chain, plus summand magnitudes
 * S (same shapes as the gradients) for condition-aware tolerances.
 * geo_inv [K,4] / geo_det [K], when non-NULL, replace the host-computed
 * inverse covariance and det (for example with a device's own preprocess:
 * its log1pf/expf may differ from the host's by an ulp, which the det
 * cancellation of an elongated Gaussian amplifies to ~1e-5 of the inverse). */
void gfo_backward_f64(int64_t out_features, int64_t in_features, int64_t k,
                      int64_t tile_out, int64_t tile_in, double sigma_multiplier,
                      const float* grad, const float* row_coords,
                      const float* col_coords, const float* mu,
                      const float* chol_raw, const float* amp,
                      const int64_t* tile_ptr, const int64_t* ids_sorted,
                      int64_t num_pairs, int normalize, int has_clamp_quad,
                      double clamp_quad, double* d_mu, double* d_chol_raw,
                      double* d_amp, double* s_mu, double* s_chol_raw,
                      double* s_amp, const float* geo_inv, const float* geo_det);

/* Threads used by the OpenMP loops (1 when built without OpenMP). */
int gfo_max_threads(void);

/* Set the OpenMP thread count of subsequent calls (n >= 1). */
void gfo_set_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
