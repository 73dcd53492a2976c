// gfield.cu -- B200 (sm_100a) Gaussian-field weight-delta renderer.
//
// Five kernels implement the whole path (forward: bin + render; backward:
// prep + render + finalize), for one field or a batch of fields in the same
// launches.  Layout and math are described per kernel below; the C ABI is in
// include/gfield.h.
//
// Parity model.  The reference kernels (gaussian_peft/cuda_field/csrc/
// forward.cu, backward.cu) are plain fp32 CUDA compiled with nvcc's default
// contraction.  The parity-relevant arithmetic here (preprocess, quadratic
// form, basis, accumulation) is written with explicit __f*_rn intrinsics so
// that the operation sequence is fixed and equal to the one the reference
// compiles to; the GPU parity tests check this bit-for-bit against the
// reference's own extension.  expf/log1pf are CUDA's, as in the reference.
// The library must be built WITHOUT --use_fast_math.

#include "gfield.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>

namespace gf {

// forward.cu:15-17
constexpr float kCholEps = 1e-5f;
constexpr float kCovFloor = 1e-8f;
constexpr double kTwoPi = 6.28318530717958647692;

constexpr int kBinThreads = 512;
constexpr int kRenderThreads = 256;  // 8 warps; fast path tile = 32x32
constexpr int kChunk = 256;          // tile-list entries (or candidates) taken per pass
constexpr int kBinSmemCapInts = 24 * 1024;          // 96 KB diff array in smem
constexpr int kBwdSmemCapFloats = 24 * 1024;        // 96 KB grad tile in smem

struct Cfg {
  int32_t tile_out, tile_in;
  float sigma;      // (float)sigma_multiplier, as forward.cu:186
  float nclamp;     // -0.5f * (float)clamp_quad (exact scaling)
  float out_scale;
  int32_t has_clamp, normalize;
  uint32_t flags;   // gf_config.flags
};

// One field as the kernels see it (kernel-parameter space, read via LDC).
struct DevField {
  const float* row;
  const float* col;
  const float* mu;
  const float* chol;
  const float* amp;
  void* delta;
  int64_t* tile_ptr;
  int64_t* ids;
  const void* grad;
  const void* base;   // [out*in] out dtype or nullptr: forward stores base + value
  unsigned long long mc;  // NVLS multicast address of delta or 0: forward stores go through multimem.st
  float* d_mu;
  float* d_chol;
  float* d_amp;
  int64_t ids_cap;    // per-field id mode: capacity (fwd) / pair count (bwd)
  int64_t part_base;  // per-field id mode: first partial slot of this field
  int32_t out_f, in_f, K, ntr, ntc;
  int32_t tile_base;  // first global tile index
  int32_t g_base;     // first global Gaussian index
  int32_t diff_base;  // first int of this field's global diff array
  int32_t bits;       // kFieldVecOk | kFieldGradVecOk
  int32_t pad_;
};
constexpr int32_t kFieldVecOk = 1;      // delta (and base) rows are 16-byte aligned for vector access
constexpr int32_t kFieldGradVecOk = 2;  // grad rows are 16-byte aligned for vector access

// Load balance: a 32x32 tile with more than kHeavyPairs Gaussians (clusters,
// densified layers) is rendered by kHeavyWarps warps of 32/kHeavyWarps rows
// each instead of the one or two warps of a regular tile, in a second launch.
// Every element still sums its Gaussians in ascending order.
constexpr int kHeavyPairs = 128;
constexpr int kHeavyWarps = 4;
constexpr int kHeavyGridCap = 2 * 148;
// below this many warps of the regular width a 32x32 forward takes
// kSmallGridWarps warps per tile (8 rows each): latency hiding needs warps
constexpr int kSmallGridMinWarps = 148 * 24;
constexpr int kSmallGridWarps = 4;
constexpr int kHeavyChunk = 32;  // backward: pairs of a heavy tile per work item

template <int NF>
struct Params {
  Cfg cfg;
  int32_t n;
  int32_t total_tiles;
  int32_t total_g;
  int32_t tile_offset;   // render kernels: first global tile of the launch (field-range renders)
  int32_t tile_end;      // render kernels: end of the launch's global tile range
  int32_t pad2_;
  uint32_t* status;
  uint32_t* done;
  uint32_t* heavy_count;  // entries in `heavy` (reset before each binning / backward)
  int32_t* heavy;         // forward: global indices of the tiles with more than kHeavyPairs pairs;
                          // backward: (tile, chunk) int2 work items of those tiles
  int32_t heavy_cap;      // backward: capacity of the work-item list
  int32_t pad3_;
  float4* records;       // [total_g][2]
  int4* boxes;           // [total_g]  (r0, r1, c0, c1)
  int64_t* goff;         // [total_g]  first partial slot of each Gaussian
  int64_t* field_pairs;  // [n]
  int32_t* diff;         // global fallback for large tile grids
  int32_t* cursor;       // forward: per tile, the next free slot of its id list (pair emission)
  float4* partials;      // [part_cap][2]
  int64_t part_cap;      // slots in partials (backward)
  int64_t* batch_ids;    // shared-id mode or nullptr
  int64_t batch_cap;
  int64_t* pair_base;    // [n+1] (shared-id mode)
  DevField f[NF];
};
// __grid_constant__ parameters are limited to 32764 bytes per launch.
static_assert(sizeof(Params<GF_MAX_FIELDS>) <= 32764, "descriptor block exceeds the kernel-parameter limit");

// Bounds checks of the debug build (-DGF_CHECK, libgfield_check.so): every
// shape-derived global access is tested against its extent; a failure sets
// GF_FLAG_BOUNDS in the workspace and the access is skipped (never a trap).
// In the release build the check is the constant true and compiles away.
#ifdef GF_CHECK
__device__ __forceinline__ bool gf_bounds_ok(bool ok, uint32_t* status) {
  if (!ok) atomicOr(status, GF_FLAG_BOUNDS);
  return ok;
}
#define GF_IN_BOUNDS(cond) gf_bounds_ok((cond), p.status)
#else
#define GF_IN_BOUNDS(cond) ((void)sizeof(cond), true)  // unevaluated: names its operands, costs nothing
#endif

// ---------------------------------------------------------------------------
// Geometry (forward.cu:134-209), bit-exact.

__device__ __forceinline__ float softplus_stable(float x) {
  // forward.cu:25-27
  return __fadd_rn(log1pf(expf(-fabsf(x))), fmaxf(x, 0.0f));
}

struct Geo {
  float i00, i01, i11, det;  // inverse covariance (i10 == i01) and det
  float l11, l21, l22;
  int4 box;                  // tile_r0, tile_r1, tile_c0, tile_c1
};

__device__ __forceinline__ int64_t clamp64(int64_t v, int64_t lo, int64_t hi) {
  return v < lo ? lo : (v > hi ? hi : v);
}

__device__ __forceinline__ Geo geometry(float mu_r, float mu_c, float raw11, float raw21,
                                        float raw22, const DevField& F, const Cfg& c) {
  Geo o;
  o.l11 = __fadd_rn(softplus_stable(raw11), kCholEps);
  o.l21 = raw21;
  o.l22 = __fadd_rn(softplus_stable(raw22), kCholEps);
  const float cov00 = __fmul_rn(o.l11, o.l11);
  const float cov01 = __fmul_rn(o.l11, o.l21);
  const float cov11 = __fmaf_rn(o.l21, o.l21, __fmul_rn(o.l22, o.l22));  // :170
  o.det = fmaxf(__fmaf_rn(cov00, cov11, -__fmul_rn(cov01, cov01)), kCovFloor);  // :171
  o.i00 = __fdiv_rn(cov11, o.det);
  o.i01 = __fdiv_rn(-cov01, o.det);
  o.i11 = __fdiv_rn(cov00, o.det);
  const float std_r = __fsqrt_rn(fmaxf(cov00, kCovFloor));
  const float std_c = __fsqrt_rn(fmaxf(cov11, kCovFloor));
  const float rs = __fmul_rn(0.5f, (float)max(F.out_f - 1, 1));
  const float cs = __fmul_rn(0.5f, (float)max(F.in_f - 1, 1));
  const float ra = __fadd_rn(mu_r, 1.0f);
  const float ca = __fadd_rn(mu_c, 1.0f);
  const float rrad = __fmul_rn(__fmul_rn(c.sigma, std_r), rs);
  const float crad = __fmul_rn(__fmul_rn(c.sigma, std_c), cs);
  // :189-192; the centre product is fused into the +/- radius
  int64_t rmin = __float2ll_rz(floorf(__fmaf_rn(ra, rs, -rrad)));
  int64_t rmax = __float2ll_rz(ceilf(__fmaf_rn(ra, rs, rrad)));
  int64_t cmin = __float2ll_rz(floorf(__fmaf_rn(ca, cs, -crad)));
  int64_t cmax = __float2ll_rz(ceilf(__fmaf_rn(ca, cs, crad)));
  rmin = clamp64(rmin, 0, F.out_f - 1);
  rmax = clamp64(rmax, 0, F.out_f - 1);
  cmin = clamp64(cmin, 0, F.in_f - 1);
  cmax = clamp64(cmax, 0, F.in_f - 1);
  o.box.x = (int)clamp64(rmin / c.tile_out, 0, F.ntr - 1);
  o.box.y = (int)clamp64(rmax / c.tile_out, 0, F.ntr - 1);
  o.box.z = (int)clamp64(cmin / c.tile_in, 0, F.ntc - 1);
  o.box.w = (int)clamp64(cmax / c.tile_in, 0, F.ntc - 1);
  return o;
}

// forward.cu:357-360: basis *= 1 / (2*pi*sqrt(max(det, floor)))
__device__ __forceinline__ float norm_factor(float det) {
  return __fdiv_rn(1.0f, __fmul_rn((float)kTwoPi, __fsqrt_rn(fmaxf(det, kCovFloor))));
}

// Fused weight epilogue: with a base weight W0 the forward stores
// out(float(W0[i]) + value[i]), one rounding to the output type, so a layer
// can use W0 + delta as a single weight (one GEMM instead of the reference's
// base GEMM plus row-chunked delta GEMMs, gaussian_linear.py:222-242).
// `i` indexes the field's elements; value already carries out_scale.
template <int OUTT>
__device__ __forceinline__ float base_at(const void* b, size_t i) {
  if (OUTT == GF_F32) return reinterpret_cast<const float*>(b)[i];
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(b)[i]);
}
__device__ __forceinline__ float4 add_base4(const float* b, float4 x) {
  const float4 w = *reinterpret_cast<const float4*>(b);
  return make_float4(__fadd_rn(w.x, x.x), __fadd_rn(w.y, x.y), __fadd_rn(w.z, x.z), __fadd_rn(w.w, x.w));
}
// 8 bf16 of the base at b (16-byte aligned) added to x[0..7] in place.
__device__ __forceinline__ void add_base8(const __nv_bfloat16* b, float* x) {
  const uint4 u = *reinterpret_cast<const uint4*>(b);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
    x[2 * k] = __fadd_rn(f.x, x[2 * k]);
    x[2 * k + 1] = __fadd_rn(f.y, x[2 * k + 1]);
  }
}

// 16-byte output store: to the local delta, or with F.mc to the NVLS
// multicast address of the same element, so the NVSwitch writes every GPU's
// copy of the gathered buffer (this one's included) as the tile is produced.
__device__ __forceinline__ void store16(void* local, unsigned long long mc, size_t byte_off, uint4 v) {
  if (mc) {
    asm volatile("multimem.st.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc + byte_off), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
  } else {
    *reinterpret_cast<uint4*>(static_cast<char*>(local) + byte_off) = v;
  }
}
__device__ __forceinline__ uint4 as_u4(float4 x) {
  return make_uint4(__float_as_uint(x.x), __float_as_uint(x.y), __float_as_uint(x.z), __float_as_uint(x.w));
}

// Render-side record of one Gaussian: two float4.
//   a = (mu_row, mu_col, amp, norm_factor)
//   b = (-0.5*i00, -0.5*i01, -0.5*i11, det)
// Scaling the inverse by -0.5 is exact, so the quadratic form evaluated from
// it is exactly -0.5*quad of the reference and expf() sees the same operand.
__device__ __forceinline__ void store_record(float4* rec, float mu_r, float mu_c, float amp,
                                             const Geo& g) {
  rec[0] = make_float4(mu_r, mu_c, amp, norm_factor(g.det));
  rec[1] = make_float4(-0.5f * g.i00, -0.5f * g.i01, -0.5f * g.i11, g.det);
}

// q' = -0.5 * dx^T A dx with the reference's association
// (forward.cu:349-350: dx*(A00*dx + A01*dy) + dy*(A10*dx + A11*dy)).
__device__ __forceinline__ float quad_scaled(float dx, float dy, float h00, float a01,
                                            float h01, float a11) {
  const float t1 = __fmaf_rn(h00, dx, a01);  // a01 = h01*dy
  const float t2 = __fmaf_rn(h01, dx, a11);  // a11 = h11*dy
  return __fmaf_rn(dx, t1, __fmul_rn(dy, t2));
}

template <int NF>
__device__ __forceinline__ int field_of_tile(const Params<NF>& p, int t) {
  int lo = 0, hi = p.n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.f[mid].tile_base <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

template <int NF>
__device__ __forceinline__ int field_of_gaussian(const Params<NF>& p, int g) {
  int lo = 0, hi = p.n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.f[mid].g_base <= g) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Block-wide exclusive scan of one int64 per thread (blockDim multiple of 32).
__device__ __forceinline__ int64_t block_exclusive_scan(int64_t v, int64_t* s_warp, int64_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int64_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int64_t w = lane < nw ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) s_warp[lane] = w;  // inclusive warp prefix
  }
  __syncthreads();
  const int64_t before = warp > 0 ? s_warp[warp - 1] : 0;
  *total = s_warp[nw - 1];
  __syncthreads();
  return before + x - v;
}

// Lower bound of the scaled form q' = -0.5*quad at one tile corner, minus
// the evaluation-error margin (h* are the -0.5-scaled inverse entries).
__device__ __forceinline__ float corner_bound(float dx, float dy, float h00, float h01, float h11) {
  const float q = dx * (h00 * dx + h01 * dy) + dy * (h01 * dx + h11 * dy);
  const float s = fabsf(h00) * dx * dx + 2.0f * fabsf(h01) * fabsf(dx * dy) + fabsf(h11) * dy * dy;
  return q - 1e-5f * s;
}

// ---------------------------------------------------------------------------
// Kernel 0 of both passes: per-Gaussian preprocess (forward.cu:134-209; the
// reference's backward rebuilds it too, backward.cu:552-557), one thread per
// Gaussian of every field: the render record and the tile box.
constexpr int kGeoThreads = 256;

//
// Backward (CLAMP_FLAG): may any element of any of the Gaussian's tiles reach
// the clamp?  The form is convex, so over the rectangle of its tile-aligned
// box it is largest at a corner -- with monotonic axes the rectangle is
// spanned by the end rows and columns (bwd_prep_kernel checks the axes and
// flags every Gaussian of a field whose axes are not).  The answer travels as
// the sign of the record's (positive) normalisation factor: negative = test
// per tile.
template <int NF, bool CLAMP_FLAG>
__global__ void __launch_bounds__(kGeoThreads) geometry_kernel(const __grid_constant__ Params<NF> p) {
  const int G = blockIdx.x * kGeoThreads + threadIdx.x;
  if (G >= p.total_g) return;
  const int fi = field_of_gaussian(p, G);
  const DevField& F = p.f[fi];
  const int g = G - F.g_base;
  const float mu_r = F.mu[2 * g], mu_c = F.mu[2 * g + 1];
  const Geo geo = geometry(mu_r, mu_c, F.chol[3 * g], F.chol[3 * g + 1], F.chol[3 * g + 2], F, p.cfg);
  float4* rec = p.records + 2 * (size_t)G;
  store_record(rec, mu_r, mu_c, F.amp[g], geo);
  p.boxes[G] = geo.box;
  if (CLAMP_FLAG && p.cfg.has_clamp) {
    const int4 box = geo.box;
    const int ra = box.x * p.cfg.tile_out, rb = min((box.y + 1) * p.cfg.tile_out, F.out_f) - 1;
    const int ca = box.z * p.cfg.tile_in, cb = min((box.w + 1) * p.cfg.tile_in, F.in_f) - 1;
    const float h00 = -0.5f * geo.i00, h01 = -0.5f * geo.i01, h11 = -0.5f * geo.i11;
    const float x0 = F.row[ra] - mu_r, x1 = F.row[rb] - mu_r, y0 = F.col[ca] - mu_c, y1 = F.col[cb] - mu_c;
    const float lo = fminf(fminf(corner_bound(x0, y0, h00, h01, h11), corner_bound(x0, y1, h00, h01, h11)),
                           fminf(corner_bound(x1, y0, h00, h01, h11), corner_bound(x1, y1, h00, h01, h11)));
    if (!(lo > p.cfg.nclamp)) rec[0].w = -rec[0].w;
  }
}

// In-place inclusive prefix sums of `lines` lines of `len` ints each (line l,
// element i at D[l * lstride + i * estride]) by the whole CTA.  When there are
// fewer lines than threads, each line is cut into up to 32 segments summed by
// separate threads (segment totals in s_seg, then one pass adding each
// segment's offset), so a long line is not one thread's serial walk.
// Integer sums: the result does not depend on the split.
__device__ __forceinline__ void line_prefix(int* D, int lines, int len, int lstride, int estride, int* s_seg) {
  const int tid = threadIdx.x, bs = blockDim.x;
  int S = lines > 0 ? bs / lines : 1;
  S = S < 1 ? 1 : (S > 32 ? 32 : S);
  if (S > len) S = len > 0 ? len : 1;
  const int seg = (len + S - 1) / S;
  for (int w = tid; w < lines * S; w += bs) {
    const int l = w / S, k = w % S;
    const int i0 = k * seg, i1 = min(len, i0 + seg);
    int* base = D + (size_t)l * lstride;
    int acc = 0;
    for (int i = i0; i < i1; ++i) {
      acc += base[i * estride];
      base[i * estride] = acc;
    }
    if (S > 1) s_seg[w] = acc;
  }
  __syncthreads();
  if (S == 1) return;
  for (int l = tid; l < lines; l += bs) {  // exclusive scan of each line's segment totals
    int acc = 0;
    for (int k = 0; k < S; ++k) {
      const int v = s_seg[l * S + k];
      s_seg[l * S + k] = acc;
      acc += v;
    }
  }
  __syncthreads();
  for (int w = tid; w < lines * S; w += bs) {
    const int l = w / S, k = w % S;
    const int add = s_seg[w];
    if (k == 0 || add == 0) continue;
    const int i0 = k * seg, i1 = min(len, i0 + seg);
    int* base = D + (size_t)l * lstride;
    for (int i = i0; i < i1; ++i) base[i * estride] += add;
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Forward kernel 1: stable binning counts, one CTA per field.
//
// Each Gaussian's tile box adds +1/-1 at its four corners of a
// (ntr+1) x (ntc+1) difference array; a 2-D prefix sum gives every tile's
// pair count, and an exclusive scan of the counts in row-major tile order
// gives tile_ptr.  This replaces the reference's scan -> host sync -> pair
// emission -> 64-bit radix sort -> atomic count -> scan chain
// (forward.cu:428-511) with O(K + T) work and no host round trip.  In
// shared-id mode the last CTA to finish turns the per-field pair counts into
// pair_base.
template <int NF>
__global__ void __launch_bounds__(kBinThreads)
bin_kernel(const __grid_constant__ Params<NF> p, int smem_cap_ints) {
  extern __shared__ int s_dyn[];
  __shared__ int64_t s_warp[32];
  __shared__ int s_seg[kBinThreads];
  __shared__ int s_last;
  const int fi = blockIdx.x;
  const DevField& F = p.f[fi];
  const int tid = threadIdx.x, bs = blockDim.x;
  const int W = F.ntc + 1, H = F.ntr + 1, nd = H * W;
  int* D = (nd <= smem_cap_ints) ? s_dyn : (p.diff + F.diff_base);
  for (int i = tid; i < nd; i += bs) D[i] = 0;
  __syncthreads();
  for (int g = tid; g < F.K; g += bs) {  // boxes from geometry_kernel
    const int4 b = p.boxes[F.g_base + g];
    atomicAdd(&D[b.x * W + b.z], 1);
    atomicAdd(&D[b.x * W + b.w + 1], -1);
    atomicAdd(&D[(b.y + 1) * W + b.z], -1);
    atomicAdd(&D[(b.y + 1) * W + b.w + 1], 1);
  }
  __syncthreads();
  line_prefix(D, H, W, W, 1, s_seg);  // along each row
  line_prefix(D, W, H, 1, W, s_seg);  // along each column
  const int T = F.ntr * F.ntc;
  const int per = (T + bs - 1) / bs;
  const int t0 = min(T, tid * per), t1 = min(T, t0 + per);
  int64_t local = 0;
  for (int t = t0; t < t1; ++t) local += D[(t / F.ntc) * W + (t % F.ntc)];
  int64_t total;
  int64_t off = block_exclusive_scan(local, s_warp, &total);
  for (int t = t0; t < t1; ++t) {
    F.tile_ptr[t] = off;
    const int c = D[(t / F.ntc) * W + (t % F.ntc)];
    off += c;
    p.cursor[F.tile_base + t] = 0;
    if (c > kHeavyPairs) p.heavy[atomicAdd(p.heavy_count, 1u)] = F.tile_base + t;
  }
  if (tid == 0) {
    F.tile_ptr[T] = total;
    p.field_pairs[fi] = total;
    if (p.batch_ids == nullptr && total > F.ids_cap) atomicOr(p.status, GF_FLAG_CAPACITY);
  }
  if (p.batch_ids != nullptr) {
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(p.done, 1u) == gridDim.x - 1);
    __syncthreads();
    if (s_last && tid < 32) {  // exclusive scan of the fields' pair counts, 32 at a time
      __threadfence();
      int64_t acc = 0;
      for (int i0 = 0; i0 < p.n; i0 += 32) {
        const int i = i0 + tid;
        const int64_t c = i < p.n ? *((volatile int64_t*)&p.field_pairs[i]) : 0;
        int64_t x = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
          if (tid >= o) x += y;
        }
        if (i < p.n) p.pair_base[i] = acc + x - c;
        acc += __shfl_sync(0xffffffffu, x, 31);
      }
      if (tid == 0) {
        p.pair_base[p.n] = acc;
        if (acc > p.batch_cap) atomicOr(p.status, GF_FLAG_CAPACITY);
        *p.done = 0u;
      }
    }
  }
}

// Tile list of (tile t, its ids slot): where the BIN stage writes the tile's
// Gaussian ids and how many fit (less than the count when the caller's id
// buffer is too small; the capacity flag is raised by bin_kernel then).
template <int NF>
struct TileIds {
  int64_t* ids;
  int64_t count, cap_left;
  __device__ __forceinline__ bool complete() const { return count <= cap_left; }
};
template <int NF>
__device__ __forceinline__ TileIds<NF> tile_ids(const Params<NF>& p, int fi, int t) {
  const DevField& F = p.f[fi];
  const int64_t start = F.tile_ptr[t];
  TileIds<NF> r;
  r.count = F.tile_ptr[t + 1] - start;
  if (p.batch_ids != nullptr) {
    const int64_t b = p.pair_base[fi];
    r.ids = p.batch_ids + b + start;
    r.cap_left = p.batch_cap - b - start;
  } else {
    r.ids = F.ids + start;
    r.cap_left = F.ids_cap - start;
  }
  return r;
}

// ---------------------------------------------------------------------------
// Forward kernel 1b: pair emission.  One warp per Gaussian walks the tiles of
// its box; each (tile, Gaussian) pair takes the next slot of the tile's list
// from a per-tile cursor (zeroed by bin_kernel).  Slots within a tile come out
// in arbitrary order; sort_tiles_kernel / sort_heavy_kernel restore ascending
// id order, which is the reference's stable (tile, id) sort order
// (forward.cu:211-241, 469).  O(pairs), no per-tile candidate scan.
constexpr int kEmitWarps = 8;

template <int NF>
__global__ void __launch_bounds__(32 * kEmitWarps) emit_pairs_kernel(const __grid_constant__ Params<NF> p) {
  const int G = blockIdx.x * kEmitWarps + (threadIdx.x >> 5);
  if (G >= p.total_g) return;  // whole warps
  const int lane = threadIdx.x & 31;
  const int fi = field_of_gaussian(p, G);
  const DevField& F = p.f[fi];
  const int g = G - F.g_base;
  const int4 b = p.boxes[G];
  const int bw = b.w - b.z + 1;
  const int nb = (b.y - b.x + 1) * bw;
  int64_t* base;
  int64_t cap;
  if (p.batch_ids != nullptr) {
    const int64_t pb = p.pair_base[fi];
    base = p.batch_ids + pb;
    cap = p.batch_cap - pb;
  } else {
    base = F.ids;
    cap = F.ids_cap;
  }
  for (int j = lane; j < nb; j += 32) {
    const int t = (b.x + j / bw) * F.ntc + b.z + j % bw;
    const int64_t at = F.tile_ptr[t] + atomicAdd(&p.cursor[F.tile_base + t], 1);
    if (at < cap) base[at] = g;
  }
}

struct BlockSync {
  __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

// Bitonic sort of s[0, n) ascending (n a power of two), by `nt` cooperating
// threads of index `i0`; `sync` orders the stages.
template <typename Sync>
__device__ __forceinline__ void bitonic_sort(int32_t* s, int n, int i0, int nt, Sync sync) {
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = i0; i < n; i += nt) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const int32_t a = s[i], c = s[ixj];
          if ((a > c) == ((i & k) == 0)) {
            s[i] = c;
            s[ixj] = a;
          }
        }
      }
      sync();
    }
  }
}

// The ordered scan of a tile's candidates (every box of the field, 32 at a
// time, in ascending id order) -- the fallback for a tile list too long to
// sort in shared memory.  One warp; writes the list.
template <int NF>
__device__ __forceinline__ void scan_tile_list(const Params<NF>& p, const DevField& F, int tr, int tc, const TileIds<NF>& L) {
  const int lane = threadIdx.x & 31;
  const int4* box = p.boxes + F.g_base;
  int64_t found = 0;
  for (int k0 = 0; k0 < F.K && found < L.count; k0 += 32) {
    const int g = k0 + lane;
    bool hit = false;
    if (g < F.K && GF_IN_BOUNDS(F.g_base + g < p.total_g)) {
      const int4 b = box[g];
      hit = (b.x <= tr) & (tr <= b.y) & (b.z <= tc) & (tc <= b.w);
    }
    const unsigned m = __ballot_sync(0xffffffffu, hit);
    if (hit) {
      const int64_t pos = found + __popc(m & ((1u << lane) - 1u));
      if (pos < L.cap_left) L.ids[pos] = g;
    }
    found += __popc(m);
  }
  if (lane == 0 && found != L.count) atomicOr(p.status, GF_FLAG_INTERNAL);
}

// Bitonic sort of 32*R keys held by one warp, key i = v[i / 32] of lane
// i % 32: partners closer than 32 apart are exchanged by shuffles, farther
// ones sit in the same lane's registers.  Ascending.
template <int R>
__device__ __forceinline__ void warp_bitonic_sort(int32_t (&v)[R], int lane) {
  constexpr int N = 32 * R;
#pragma unroll
  for (int k = 2; k <= N; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= 32) {
        const int rj = j >> 5;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int q = r ^ rj;
          if (q > r) {
            const bool up = ((r * 32 + lane) & k) == 0;
            const int32_t lo = min(v[r], v[q]), hi = max(v[r], v[q]);
            v[r] = up ? lo : hi;
            v[q] = up ? hi : lo;
          }
        }
      } else {
        const bool lower = (lane & j) == 0;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int32_t o = __shfl_xor_sync(0xffffffffu, v[r], j);
          const bool up = ((r * 32 + lane) & k) == 0;
          v[r] = (lower == up) ? min(v[r], o) : max(v[r], o);
        }
      }
    }
  }
}

// Loads a tile list of n <= 32*R ids into the warp's registers (padding with
// INT32_MAX), sorts it unless it is already ascending, and writes it back.
template <int R, int NF>
__device__ __forceinline__ void sort_list_in_registers(const TileIds<NF>& L, int n, int lane) {
  int32_t v[R];
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = (r * 32 + lane < n) ? (int32_t)L.ids[r * 32 + lane] : INT32_MAX;
  bool descent = false;  // any key smaller than its predecessor
#pragma unroll
  for (int r = 0; r < R; ++r) {
    int32_t prev = __shfl_up_sync(0xffffffffu, v[r], 1);
    if (r > 0) {
      const int32_t last = __shfl_sync(0xffffffffu, v[r - 1], 31);
      if (lane == 0) prev = last;
    }
    const int i = r * 32 + lane;
    descent |= (i > 0 && i < n && prev > v[r]);
  }
  if (__ballot_sync(0xffffffffu, descent) == 0u) return;
  warp_bitonic_sort<R>(v, lane);
#pragma unroll
  for (int r = 0; r < R; ++r)
    if (r * 32 + lane < n) L.ids[r * 32 + lane] = v[r];
}

// Forward kernel 1c: sort every tile list of at most kHeavyPairs ids
// (ids are < 2^31), one warp per tile, in registers: 32, 64 or 128 keys by
// the list's length.  Lists beyond kHeavyPairs ids are in the heavy list and
// sorted by sort_heavy_kernel.
constexpr int kSortWarps = 4;
static_assert(kHeavyPairs <= 128, "sort_tiles_kernel sorts at most 128 ids in registers");

template <int NF>
__global__ void __launch_bounds__(32 * kSortWarps) sort_tiles_kernel(const __grid_constant__ Params<NF> p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tg = blockIdx.x * kSortWarps + warp;
  if (tg >= p.total_tiles) return;  // whole warps
  const int fi = field_of_tile(p, tg);
  const TileIds<NF> L = tile_ids(p, fi, tg - p.f[fi].tile_base);
  const int n = (int)L.count;
  if (n <= 1 || n > kHeavyPairs || !L.complete()) return;
  if (n <= 32) sort_list_in_registers<1>(L, n, lane);
  else if (n <= 64) sort_list_in_registers<2>(L, n, lane);
  else sort_list_in_registers<4>(L, n, lane);
}

// The heavy tiles' lists (more than kHeavyPairs ids): one CTA per tile,
// striding over the heavy list; lists beyond kSortCap ids are rebuilt by the
// ordered scan instead.
constexpr int kSortCap = 8192;
constexpr int kSortThreads = 512;

template <int NF>
__global__ void __launch_bounds__(kSortThreads) sort_heavy_kernel(const __grid_constant__ Params<NF> p) {
  __shared__ int32_t s[kSortCap];
  const int nh = (int)*reinterpret_cast<volatile uint32_t*>(p.heavy_count);
  for (int h = blockIdx.x; h < nh; h += gridDim.x) {
    const int tg = p.heavy[h];
    const int fi = field_of_tile(p, tg);
    const DevField& F = p.f[fi];
    const int t = tg - F.tile_base;
    const TileIds<NF> L = tile_ids(p, fi, t);
    const int64_t n0 = L.count;
    if (!L.complete()) continue;
    if (n0 > kSortCap) {
      if (threadIdx.x < 32) scan_tile_list(p, F, t / F.ntc, t % F.ntc, L);
      __syncthreads();
      continue;
    }
    int n = 32;
    while (n < n0) n <<= 1;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s[i] = i < n0 ? (int32_t)L.ids[i] : INT32_MAX;
    __syncthreads();
    bitonic_sort(s, n, (int)threadIdx.x, (int)blockDim.x, BlockSync{});
    for (int i = threadIdx.x; i < n0; i += blockDim.x) L.ids[i] = s[i];
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Forward kernel 2: tile render, one CTA (8 warps) per tile.
//
// Work is split into 32x32 sub-blocks (one for the default tile).  Lane =
// column, warp w owns rows w, w+8, w+16, w+24, so the column offset dy and the
// two products that depend on it are hoisted per Gaussian.  The tile's
// Gaussian list is rebuilt here from the boxes: candidates are tested 256 at a
// time and compacted with warp ballots, which keeps ascending id order, i.e.
// exactly the reference's stable-sorted order (forward.cu:481-482).  The first
// sub-block also writes the ids.  Each element sums amp*basis over that list
// sequentially in fp32, as forward.cu:326-362 does, so fp32 output is
// bit-identical.  Output goes through shared memory to 128-bit stores.
template <int NF, bool NORM, bool CLAMP, int OUTT>
__global__ void __launch_bounds__(kRenderThreads, 3)
render_fwd_kernel(const __grid_constant__ Params<NF> p) {
  __shared__ float4 s_rec[2 * kChunk];
  __shared__ int s_list[kChunk];
  __shared__ int s_wcnt[8];
  __shared__ float s_out[32][33];
  const int tg = blockIdx.x + p.tile_offset;
  const int fi = field_of_tile(p, tg);
  const DevField& F = p.f[fi];
  const int t = tg - F.tile_base;
  const int tr = t / F.ntc, tc = t % F.ntc;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row0 = tr * p.cfg.tile_out, col0 = tc * p.cfg.tile_in;
  const int th = min(p.cfg.tile_out, F.out_f - row0);
  const int tw = min(p.cfg.tile_in, F.in_f - col0);
  const int64_t start = F.tile_ptr[t];
  const int64_t count = F.tile_ptr[t + 1] - start;
  int64_t* ids;
  int64_t cap_left;
  if (p.batch_ids != nullptr) {
    const int64_t b = p.pair_base[fi];
    ids = p.batch_ids + b + start;
    cap_left = p.batch_cap - b - start;
  } else {
    ids = F.ids + start;
    cap_left = F.ids_cap - start;
  }
  const float4* rec = p.records + 2 * (size_t)F.g_base;
  const int4* box = p.boxes + F.g_base;
  const float nclamp = p.cfg.nclamp;
  // the tile's sorted list from the BIN stage; if the id buffer could not
  // hold it, the ordered scan of every box of the field (same order)
  const bool listed = count <= cap_left;
  const int ncand = listed ? (int)count : F.K;

  for (int rb = 0; rb < th; rb += 32) {
    for (int cb = 0; cb < tw; cb += 32) {
      const int c = cb + lane;
      const float cc = (c < tw) ? F.col[col0 + c] : 0.0f;
      float cr[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = rb + warp + 8 * j;
        cr[j] = (r < th) ? F.row[row0 + r] : 0.0f;
      }
      float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      int64_t found = 0;
      for (int k0 = 0; k0 < ncand && found < count; k0 += kChunk) {
        int g = 0;
        bool hit = false;
        if (k0 + tid < ncand) {
          if (listed) {
            const int64_t v = ids[k0 + tid];
            g = (int)v;
            hit = v >= 0 && v < F.K;
          } else if (GF_IN_BOUNDS(F.g_base + k0 + tid < p.total_g)) {
            g = k0 + tid;
            const int4 b = box[g];
            hit = (b.x <= tr) & (tr <= b.y) & (b.z <= tc) & (tc <= b.w);
          }
        }
        const unsigned m = __ballot_sync(0xffffffffu, hit);
        if (lane == 0) s_wcnt[warp] = __popc(m);
        __syncthreads();
        int before = 0, total = 0;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          const int cw = s_wcnt[w];
          before += (w < warp) ? cw : 0;
          total += cw;
        }
        if (hit) {
          const int pos = before + __popc(m & ((1u << lane) - 1u));
          s_list[pos] = g;
        }
        __syncthreads();
        if (tid < total) {
          const int gg = s_list[tid];
          s_rec[2 * tid] = rec[2 * gg];
          s_rec[2 * tid + 1] = rec[2 * gg + 1];
        }
        __syncthreads();
        for (int j = 0; j < total; ++j) {
          const float4 a = s_rec[2 * j];
          const float4 h = s_rec[2 * j + 1];
          const float dy = __fsub_rn(cc, a.y);
          const float a01 = __fmul_rn(h.y, dy);
          const float a11 = __fmul_rn(h.z, dy);
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const float dx = __fsub_rn(cr[jj], a.x);
            float q = quad_scaled(dx, dy, h.x, a01, h.y, a11);
            q = fminf(q, 0.0f);                 // quad = max(quad, 0)
            if (CLAMP) q = fmaxf(q, nclamp);    // quad = min(quad, clamp)
            float e = expf(q);
            if (NORM) e = __fmul_rn(e, a.w);
            v[jj] = __fmaf_rn(a.z, e, v[jj]);   // forward.cu:361
          }
        }
        found += total;
        __syncthreads();
      }
      if (rb == 0 && cb == 0 && tid == 0 && found != count) atomicOr(p.status, GF_FLAG_INTERNAL);

      // Store the 32x32 sub-block.
      const float sc = p.cfg.out_scale;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float val = v[j];
        if (sc != 1.0f) val = __fmul_rn(val, sc);
        s_out[warp + 8 * j][lane] = val;
      }
      __syncthreads();
      const int bh = min(32, th - rb), bw = min(32, tw - cb);
      const size_t base = (size_t)(row0 + rb) * F.in_f + (col0 + cb);
      if (OUTT == GF_F32) {
        float* out = reinterpret_cast<float*>(F.delta) + base;
        const int r = tid >> 3, q4 = (tid & 7) * 4;
        if (r < bh) {
          const size_t o = (size_t)r * F.in_f + q4;
          const size_t nel = (size_t)F.out_f * F.in_f;
          if ((F.bits & kFieldVecOk) && q4 + 3 < bw && GF_IN_BOUNDS(base + o + 3 < nel)) {
            float4 x = make_float4(s_out[r][q4], s_out[r][q4 + 1], s_out[r][q4 + 2], s_out[r][q4 + 3]);
            if (F.base) x = add_base4(reinterpret_cast<const float*>(F.base) + base + o, x);
            store16(F.delta, F.mc, 4 * (base + o), as_u4(x));
          } else {
            if (F.mc) atomicOr(p.status, GF_FLAG_INTERNAL);  // excluded on the host (vec_ok)
            for (int k = 0; k < 4; ++k)
              if (!F.mc && q4 + k < bw && GF_IN_BOUNDS(base + o + k < nel)) {
                float x = s_out[r][q4 + k];
                if (F.base) x = __fadd_rn(base_at<GF_F32>(F.base, base + o + k), x);
                out[o + k] = x;
              }
          }
        }
      } else {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(F.delta) + base;
        if (tid < 128) {
          const int r = tid >> 2, q8 = (tid & 3) * 8;
          if (r < bh) {
            const size_t o = (size_t)r * F.in_f + q8;
            const size_t nel = (size_t)F.out_f * F.in_f;
            if ((F.bits & kFieldVecOk) && q8 + 7 < bw && GF_IN_BOUNDS(base + o + 7 < nel)) {
              float x[8];
#pragma unroll
              for (int k = 0; k < 8; ++k) x[k] = s_out[r][q8 + k];
              if (F.base) add_base8(reinterpret_cast<const __nv_bfloat16*>(F.base) + base + o, x);
              uint32_t w[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const __nv_bfloat162 h2 = __floats2bfloat162_rn(x[2 * k], x[2 * k + 1]);
                w[k] = *reinterpret_cast<const uint32_t*>(&h2);
              }
              store16(F.delta, F.mc, 2 * (base + o), make_uint4(w[0], w[1], w[2], w[3]));
            } else {
              if (F.mc) atomicOr(p.status, GF_FLAG_INTERNAL);  // excluded on the host (vec_ok)
              for (int k = 0; k < 8; ++k)
                if (!F.mc && q8 + k < bw && GF_IN_BOUNDS(base + o + k < nel)) {
                  float x = s_out[r][q8 + k];
                  if (F.base) x = __fadd_rn(base_at<GF_BF16>(F.base, base + o + k), x);
                  out[o + k] = __float2bfloat16_rn(x);
                }
            }
          }
        }
      }
      // multicast stores are published before the caller's group barrier
      if (F.mc) __threadfence_system();
      __syncthreads();
    }
  }
}

// Hardware base-2 exponential (MUFU.EX2, ftz): a few 1e-7 relative error.
constexpr float kLog2e = 1.44269504088896340736f;
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// ---------------------------------------------------------------------------
// Packed fp32x2 arithmetic (sm_100: one issue slot for two IEEE fp32
// operations, each rounded exactly like the scalar instruction).

typedef unsigned long long f2;

__device__ __forceinline__ f2 pk2(float a, float b) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void up2(f2 x, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(x));
}
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
  f2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
  f2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
  f2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 sub2(f2 a, f2 b) {
  f2 d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// 2^x of both halves; one asm block so that the result stays in the input's
// register pair (no moves to re-pack the two MUFU results)
__device__ __forceinline__ f2 ex2_2(f2 x) {
  f2 r;
  asm("{\n\t.reg .f32 a, b;\n\tmov.b64 {a, b}, %1;\n\tex2.approx.ftz.f32 a, a;\n\tex2.approx.ftz.f32 b, b;\n\t"
      "mov.b64 %0, {a, b};\n\t}"
      : "=l"(r) : "l"(x));
  return r;
}

// ---------------------------------------------------------------------------
// Forward kernel 2, 32x32-tile fast path: one CTA of kFwd32Warps warps per
// tile, warp w owning rows [w*R, (w+1)*R) and lane = column.  Each warp walks
// the candidate Gaussians 32 at a time, tests their boxes, and consumes the
// warp ballot's set bits in ascending order -- the reference's stable-sorted
// order -- so no shared list and no CTA barrier are needed.  Per Gaussian the
// column terms (dy and the two products with it) are computed once per lane;
// per pair of rows the quadratic form is evaluated with packed fp32x2
// instructions in exactly the reference's association, expf and the
// accumulation stay scalar and sequential: the fp32 output is bit-identical
// to the generic kernel's and to the reference's.
#ifndef GF_FWD32_WARPS
#define GF_FWD32_WARPS 2
#endif
constexpr int kFwd32Warps = GF_FWD32_WARPS;
// the base-2 variant does less work per element, so each warp takes more rows
// to amortise its per-Gaussian set-up
#ifndef GF_FWD32_WARPS_EX2
#define GF_FWD32_WARPS_EX2 1
#endif
constexpr int kFwd32WarpsEx2 = GF_FWD32_WARPS_EX2;
template <bool EX2>
__host__ __device__ constexpr int fwd32_warps() { return EX2 ? kFwd32WarpsEx2 : kFwd32Warps; }

template <int NF, bool NORM, bool CLAMP, int OUTT, bool EX2, int NW>
__device__ __forceinline__ void fwd32_tile(const Params<NF>& p, int tg, bool skip_heavy,
                                           float (*s_out)[32 / NW][36]) {
  constexpr int R = 32 / NW;  // rows per warp
  const int fi = field_of_tile(p, tg);
  const DevField& F = p.f[fi];
  const int t = tg - F.tile_base;
  const int tr = t / F.ntc, tc = t % F.ntc;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int row0 = tr * 32, col0 = tc * 32;
  const int th = min(32, F.out_f - row0), tw = min(32, F.in_f - col0);
  const int64_t start = F.tile_ptr[t];
  const int64_t count = F.tile_ptr[t + 1] - start;
  if (skip_heavy && count > kHeavyPairs) return;  // rendered by render_fwd32_heavy_kernel
  int64_t* ids;
  int64_t cap_left;
  if (p.batch_ids != nullptr) {
    const int64_t b = p.pair_base[fi];
    ids = p.batch_ids + b + start;
    cap_left = p.batch_cap - b - start;
  } else {
    ids = F.ids + start;
    cap_left = F.ids_cap - start;
  }
  const float4* rec = p.records + 2 * (size_t)F.g_base;
  const int4* box = p.boxes + F.g_base;
  const float nclamp = p.cfg.nclamp;
  const int rw0 = warp * R;
  const float cc = (lane < tw) ? F.col[col0 + lane] : 0.0f;
  const float myr = (lane < R && rw0 + lane < th) ? F.row[row0 + rw0 + lane] : 0.0f;
  f2 CR[R / 2];
#pragma unroll
  for (int i = 0; i < R / 2; ++i)
    CR[i] = pk2(__shfl_sync(0xffffffffu, myr, 2 * i), __shfl_sync(0xffffffffu, myr, 2 * i + 1));
  // row pairs (2i, 2i+1) accumulate in packed registers: fma.rn.f32x2 rounds
  // each half exactly like the scalar fmaf of forward.cu:361
  f2 V[R / 2];
#pragma unroll
  for (int i = 0; i < R / 2; ++i) V[i] = pk2(0.0f, 0.0f);

  // the tile's sorted list from the BIN stage; if the id buffer could not
  // hold it, the ordered scan of every box of the field (same order)
  const bool listed = count <= cap_left;
  const int ncand = listed ? (int)count : F.K;
  int64_t found = 0;
  for (int k0 = 0; k0 < ncand && found < count; k0 += 32) {
    int g = 0;
    bool hit = false;
    if (k0 + lane < ncand) {
      if (listed) {
        const int64_t v = ids[k0 + lane];
        g = (int)v;
        hit = v >= 0 && v < F.K;
      } else if (GF_IN_BOUNDS(F.g_base + k0 + lane < p.total_g)) {
        g = k0 + lane;
        const int4 b = box[g];
        hit = (b.x <= tr) & (tr <= b.y) & (b.z <= tc) & (tc <= b.w);
      }
    }
    unsigned m = __ballot_sync(0xffffffffu, hit);
    found += __popc(m);
    // Every hit's record is fetched by the lane that tested it, all lanes at
    // once, and handed to the warp by shuffles in ascending order: one load
    // latency per 32 candidates instead of one per Gaussian.
    float4 ra = make_float4(0.f, 0.f, 0.f, 0.f), rh = ra;
    if (hit) {
      ra = rec[2 * g];
      rh = rec[2 * g + 1];
    }
    if constexpr (EX2) {
      // bf16 output (GF_CFG_FWD_EXP2): the form in base 2 with the column
      // terms hoisted, q2 = dx*(g00*dx + 2*g01*dy) + g11*dy^2 (g = log2e*h),
      // and the basis 2^q2 from MUFU.EX2; the normalisation folds into the
      // amplitude.  Relative error per term ~1e-5 at worst (cancelling terms
      // of very elongated Gaussians), far below bf16's 3.9e-3 ulp.  The owner
      // lane precomputes the Gaussian's constants before the hand-over.
      const float o00 = rh.x * kLog2e, o01 = 2.0f * (rh.y * kLog2e), o11 = rh.z * kLog2e;
      const float oamp = NORM ? ra.z * ra.w : ra.z;
      const float nclamp2 = nclamp * kLog2e;
      // As in the base-2 backward, a clamp at quad >= 64 is not applied: the
      // clamp only raises a term beyond it to amp * e^(-clamp/2), so leaving
      // it out changes an element by less than |amp| * e^-32 = 1.3e-14 |amp|
      // per Gaussian, in absolute terms.
      const bool clamp_terms = CLAMP && nclamp > -32.0f;
      while (m) {
        const int src = __ffs(m) - 1;
        m &= m - 1;
        const float mur = __shfl_sync(0xffffffffu, ra.x, src), muc = __shfl_sync(0xffffffffu, ra.y, src);
        const float g00 = __shfl_sync(0xffffffffu, o00, src), g01x2 = __shfl_sync(0xffffffffu, o01, src);
        const float g11 = __shfl_sync(0xffffffffu, o11, src), ampn = __shfl_sync(0xffffffffu, oamp, src);
        const float dy = cc - muc;
        const float b1 = g01x2 * dy, c0 = g11 * dy * dy;
        const f2 G00 = pk2(g00, g00), B1 = pk2(b1, b1), C0 = pk2(c0, c0), MUR = pk2(mur, mur);
        const f2 AMP = pk2(ampn, ampn);
        if (clamp_terms) {
#pragma unroll
          for (int i = 0; i < R / 2; ++i) {
            const f2 DX = sub2(CR[i], MUR);
            f2 Q = fma2(DX, fma2(G00, DX, B1), C0);
            float q0, q1;
            up2(Q, q0, q1);
            Q = pk2(fmaxf(q0, nclamp2), fmaxf(q1, nclamp2));
            V[i] = fma2(AMP, ex2_2(Q), V[i]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < R / 2; ++i) {
            const f2 DX = sub2(CR[i], MUR);
            V[i] = fma2(AMP, ex2_2(fma2(DX, fma2(G00, DX, B1), C0)), V[i]);
          }
        }
      }
    } else {
      while (m) {
        const int src = __ffs(m) - 1;
        m &= m - 1;
        float4 a, h;
        a.x = __shfl_sync(0xffffffffu, ra.x, src);
        a.y = __shfl_sync(0xffffffffu, ra.y, src);
        a.z = __shfl_sync(0xffffffffu, ra.z, src);
        a.w = NORM ? __shfl_sync(0xffffffffu, ra.w, src) : 0.0f;
        h.x = __shfl_sync(0xffffffffu, rh.x, src);
        h.y = __shfl_sync(0xffffffffu, rh.y, src);
        h.z = __shfl_sync(0xffffffffu, rh.z, src);
        const float dy = __fsub_rn(cc, a.y);
        const float a01 = __fmul_rn(h.y, dy);
        const float a11 = __fmul_rn(h.z, dy);
        const f2 H00 = pk2(h.x, h.x), H01 = pk2(h.y, h.y), A01 = pk2(a01, a01), A11 = pk2(a11, a11);
        const f2 DY = pk2(dy, dy), MUR = pk2(a.x, a.x), AMP = pk2(a.z, a.z);
#pragma unroll
        for (int i = 0; i < R / 2; ++i) {
          const f2 DX = sub2(CR[i], MUR);
          const f2 T1 = fma2(H00, DX, A01);
          const f2 T2 = fma2(H01, DX, A11);
          const f2 Q = fma2(DX, T1, mul2(DY, T2));
          float q0, q1;
          up2(Q, q0, q1);
          q0 = fminf(q0, 0.0f);
          q1 = fminf(q1, 0.0f);
          if (CLAMP) {
            q0 = fmaxf(q0, nclamp);
            q1 = fmaxf(q1, nclamp);
          }
          float e0 = expf(q0), e1 = expf(q1);
          if (NORM) {
            e0 = __fmul_rn(e0, a.w);
            e1 = __fmul_rn(e1, a.w);
          }
          V[i] = fma2(AMP, pk2(e0, e1), V[i]);
        }
      }
    }
  }
  if (warp == 0 && lane == 0 && found != count) atomicOr(p.status, GF_FLAG_INTERNAL);

  // Stage the warp's R x 32 block and store it with 128-bit stores.
  const float sc = p.cfg.out_scale;
#pragma unroll
  for (int i = 0; i < R / 2; ++i) {
    float v0, v1;
    up2(V[i], v0, v1);
    s_out[warp][2 * i][lane] = (sc != 1.0f) ? __fmul_rn(v0, sc) : v0;
    s_out[warp][2 * i + 1][lane] = (sc != 1.0f) ? __fmul_rn(v1, sc) : v1;
  }
  __syncwarp();
  const int bh = min(R, th - rw0);
  if (bh <= 0) return;
  const size_t base = (size_t)(row0 + rw0) * F.in_f + col0;
  if (OUTT == GF_F32) {
    float* out = reinterpret_cast<float*>(F.delta) + base;
#pragma unroll
    for (int k = 0; k < R / 4; ++k) {
      const int r = k * 4 + (lane >> 3), q4 = (lane & 7) * 4;
      if (r < bh) {
        const size_t o = (size_t)r * F.in_f + q4;
        const size_t nel = (size_t)F.out_f * F.in_f;
        if ((F.bits & kFieldVecOk) && q4 + 3 < tw && GF_IN_BOUNDS(base + o + 3 < nel)) {
          float4 x = *reinterpret_cast<const float4*>(&s_out[warp][r][q4]);
          if (F.base) x = add_base4(reinterpret_cast<const float*>(F.base) + base + o, x);
          store16(F.delta, F.mc, 4 * (base + o), as_u4(x));
        } else {
          if (F.mc) atomicOr(p.status, GF_FLAG_INTERNAL);  // excluded on the host (vec_ok)
          for (int j = 0; j < 4; ++j)
            if (!F.mc && q4 + j < tw && GF_IN_BOUNDS(base + o + j < nel)) {
              float x = s_out[warp][r][q4 + j];
              if (F.base) x = __fadd_rn(base_at<GF_F32>(F.base, base + o + j), x);
              out[o + j] = x;
            }
        }
      }
    }
  } else {
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(F.delta) + base;
#pragma unroll
    for (int k = 0; k < R / 8; ++k) {
      const int r = k * 8 + (lane >> 2), q8 = (lane & 3) * 8;
      if (r < bh) {
        const size_t o = (size_t)r * F.in_f + q8;
        const size_t nel = (size_t)F.out_f * F.in_f;
        if ((F.bits & kFieldVecOk) && q8 + 7 < tw && GF_IN_BOUNDS(base + o + 7 < nel)) {
          float4 x0 = *reinterpret_cast<const float4*>(&s_out[warp][r][q8]);
          float4 x1 = *reinterpret_cast<const float4*>(&s_out[warp][r][q8 + 4]);
          if (F.base) {
            float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            add_base8(reinterpret_cast<const __nv_bfloat16*>(F.base) + base + o, x);
            x0 = make_float4(x[0], x[1], x[2], x[3]);
            x1 = make_float4(x[4], x[5], x[6], x[7]);
          }
          const __nv_bfloat162 h0 = __floats2bfloat162_rn(x0.x, x0.y), h1 = __floats2bfloat162_rn(x0.z, x0.w);
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(x1.x, x1.y), h3 = __floats2bfloat162_rn(x1.z, x1.w);
          store16(F.delta, F.mc, 2 * (base + o),
                  make_uint4(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                             *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3)));
        } else {
          if (F.mc) atomicOr(p.status, GF_FLAG_INTERNAL);  // excluded on the host (vec_ok)
          for (int j = 0; j < 8; ++j)
            if (!F.mc && q8 + j < tw && GF_IN_BOUNDS(base + o + j < nel)) {
              float x = s_out[warp][r][q8 + j];
              if (F.base) x = __fadd_rn(base_at<GF_BF16>(F.base, base + o + j), x);
              out[o + j] = __float2bfloat16_rn(x);
            }
        }
      }
    }
  }
  // multicast stores are published before the caller's group barrier
  if (F.mc) __threadfence_system();
}

// NW warps per tile: fwd32_warps<EX2>() normally, kSmallGridWarps when the
// launch has too few tiles to fill the GPU with that many warps.
template <int NF, bool NORM, bool CLAMP, int OUTT, bool EX2, int NW>
__global__ void __launch_bounds__(32 * NW, (EX2 ? 20 : 12) * fwd32_warps<EX2>() / NW)
render_fwd32_kernel(const __grid_constant__ Params<NF> p) {
  __shared__ __align__(16) float s_out[NW][32 / NW][36];
  fwd32_tile<NF, NORM, CLAMP, OUTT, EX2, NW>(p, blockIdx.x + p.tile_offset, true, s_out);
}

// The tiles the binning listed as heavy (within the launch's tile range),
// kHeavyWarps warps each, CTAs striding over the list.
template <int NF, bool NORM, bool CLAMP, int OUTT, bool EX2>
__global__ void __launch_bounds__(32 * kHeavyWarps) render_fwd32_heavy_kernel(const __grid_constant__ Params<NF> p) {
  __shared__ __align__(16) float s_out[kHeavyWarps][32 / kHeavyWarps][36];
  const int n = (int)*reinterpret_cast<volatile uint32_t*>(p.heavy_count);
  for (int i = blockIdx.x; i < n; i += gridDim.x) {
    const int tg = p.heavy[i];
    if (tg < p.tile_offset || tg >= p.tile_end) continue;
    fwd32_tile<NF, NORM, CLAMP, OUTT, EX2, kHeavyWarps>(p, tg, false, s_out);
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Backward kernel 1: per field, after geometry_kernel, each Gaussian's first
// slot in the pair-partial buffer:
// an exclusive scan of tiles_touched, i.e. the reference's pair emission
// order (forward.cu:211-241).  Also checks that the saved pair count matches.
template <int NF>
__global__ void __launch_bounds__(kBinThreads)
bwd_prep_kernel(const __grid_constant__ Params<NF> p) {
  __shared__ int64_t s_warp[32];
  const int fi = blockIdx.x;
  const DevField& F = p.f[fi];
  const int tid = threadIdx.x, bs = blockDim.x;
  // Are the axes monotonic?  Then the coordinates of any range of rows (or
  // columns) lie between the range's end values, which geometry_kernel's
  // clamp bounds use.
  bool mono = true;
  if (p.cfg.has_clamp) {
    bool up_r = true, dn_r = true, up_c = true, dn_c = true;
    for (int i = tid; i + 1 < F.out_f; i += bs) {
      const float a = F.row[i], b = F.row[i + 1];
      up_r &= a <= b; dn_r &= a >= b;
    }
    for (int i = tid; i + 1 < F.in_f; i += bs) {
      const float a = F.col[i], b = F.col[i + 1];
      up_c &= a <= b; dn_c &= a >= b;
    }
    const int ur = __syncthreads_and(up_r), dr = __syncthreads_and(dn_r);
    const int uc = __syncthreads_and(up_c), dc = __syncthreads_and(dn_c);
    mono = (ur || dr) && (uc || dc);
  }
  const int per = (F.K + bs - 1) / bs;
  const int g0 = min(F.K, tid * per), g1 = min(F.K, g0 + per);
  int64_t local = 0;
  for (int g = g0; g < g1; ++g) {  // boxes from geometry_kernel
    const int4 box = p.boxes[F.g_base + g];
    if (!mono) {  // the clamp test of geometry_kernel assumed monotonic axes: test every tile
      float4* rec = p.records + 2 * (size_t)(F.g_base + g);
      rec[0].w = -fabsf(rec[0].w);
    }
    local += (int64_t)(box.y - box.x + 1) * (box.w - box.z + 1);
  }
  int64_t total;
  int64_t off = block_exclusive_scan(local, s_warp, &total);
  int64_t base, npairs;
  if (p.batch_ids != nullptr) {
    base = p.pair_base[fi];
    npairs = p.pair_base[fi + 1] - base;
  } else {
    base = F.part_base;
    npairs = F.ids_cap;
  }
  for (int g = g0; g < g1; ++g) {
    p.goff[F.g_base + g] = base + off;
    const int4 b = p.boxes[F.g_base + g];
    off += (int64_t)(b.y - b.x + 1) * (b.w - b.z + 1);
  }
  if (tid == 0) {
    const int64_t T = (int64_t)F.ntr * F.ntc;
    if (total != npairs || F.tile_ptr[T] != npairs || F.tile_ptr[0] != 0)
      atomicOr(p.status, GF_FLAG_STATE);
  }
  // work items of the heavy tiles (32x32 tiles only: the generic backward has
  // no heavy path)
  if (p.cfg.tile_out == 32 && p.cfg.tile_in == 32) {
    int2* items = reinterpret_cast<int2*>(p.heavy);
    const int T = F.ntr * F.ntc;
    for (int t = tid; t < T; t += bs) {
      const int64_t c = F.tile_ptr[t + 1] - F.tile_ptr[t];
      if (c <= kHeavyPairs || c > F.K) continue;  // (an impossible count is flagged by the render)
      const int nch = (int)((c + kHeavyChunk - 1) / kHeavyChunk);
      const unsigned at = atomicAdd(p.heavy_count, (unsigned)nch);
      for (int j = 0; j < nch; ++j)
        if (at + j < (unsigned)p.heavy_cap) items[at + j] = make_int2(F.tile_base + t, j);
    }
  }
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

template <int GT>
__device__ __forceinline__ float load_grad(const void* g, size_t i) {
  if (GT == GF_F32) return reinterpret_cast<const float*>(g)[i];
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(g)[i]);
}

// ---------------------------------------------------------------------------
// Backward kernel 2: per-pair partial gradients, one CTA (8 warps) per tile.
//
// The tile's dL/d(delta) is read from HBM once into shared memory (the
// reference re-reads it once per pair, backward.cu:301-308).  Warp i handles
// the tile's pairs i, i+8, ...; lane = column, so dy is fixed per lane and the
// per-element work is the basis plus six running sums (gba = g*b where the
// q-gradient is active, 0 where the form is clamped):
//   T0 = sum g*b,  U0 = sum gba,  U1 = sum gba*dx,  U2 = sum gba*dx^2,
//   M0 = sum gba*fma(h01, dy, h00*dx),  M1 = sum gba*fma(h11, dy, h01*dx)
// (h = -0.5*A), from which the reference's per-pair channels follow
// (backward.cu:330-351, with A01 == A10):
//   amp: T0    mu0: -2*M0    mu1: -2*M1
//   A00: U2    A01 = A10: dy*U1    A11: dy^2*U0      (times amp, -0.5 later)
// The mu factors are evaluated per element with the reference's roundings
// (its build contracts dq/dmu0 = -(2*A00*dx + 2*A01*dy) to
// -fma(2*A01, dy, 2*A00*dx)): for an elongated Gaussian A00*dx and A01*dy
// nearly cancel, and a sum factored as A00*U1 + A01*dy*U0 would carry their
// rounding, not that of the (much smaller) per-element terms.  The A factors
// carry no such cancellation (dy is exact per lane), so they stay factored.
// Lanes are reduced with a fixed xor-shuffle tree and lane 0 writes the six
// channels to the pair's slot, goff[g] + (its tile's index in g's box), so the
// finalize kernel reads each Gaussian's pairs contiguously.
// Saved-state checks: id in range, strictly ascending inside the tile, tile
// inside the Gaussian's box; a failing pair sets GF_FLAG_STATE and is skipped.
template <int NF, bool NORM, bool CLAMP, int GT>
__global__ void __launch_bounds__(kRenderThreads)
render_bwd_kernel(const __grid_constant__ Params<NF> p) {
  extern __shared__ float s_g[];  // [tile_out][tile_in] then [tile_out] row coords
  const int tg = blockIdx.x;
  const int fi = field_of_tile(p, tg);
  const DevField& F = p.f[fi];
  const int t = tg - F.tile_base;
  const int tr = t / F.ntc, tc = t % F.ntc;
  const int64_t start = F.tile_ptr[t];
  const int64_t count = F.tile_ptr[t + 1] - start;
  if (count <= 0) return;
  // The saved binning is caller data: never index outside the id buffer.
  const int64_t id_base = (p.batch_ids != nullptr) ? p.pair_base[fi] : 0;
  const int64_t id_limit = (p.batch_ids != nullptr) ? p.batch_cap : F.ids_cap;
  if (start < 0 || id_base < 0 || id_base + start + count > id_limit) {
    if (threadIdx.x == 0) atomicOr(p.status, GF_FLAG_STATE);
    return;
  }
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int TO = p.cfg.tile_out, TI = p.cfg.tile_in;
  const int row0 = tr * TO, col0 = tc * TI;
  const int th = min(TO, F.out_f - row0), tw = min(TI, F.in_f - col0);
  float* s_row = s_g + TO * TI;
  for (int e = tid; e < TO * TI; e += blockDim.x) {
    const int r = e / TI, c = e - r * TI;
    s_g[e] = (r < th && c < tw && GF_IN_BOUNDS((size_t)(row0 + r) * F.in_f + col0 + c < (size_t)F.out_f * F.in_f))
                 ? load_grad<GT>(F.grad, (size_t)(row0 + r) * F.in_f + col0 + c)
                 : 0.0f;
  }
  for (int r = tid; r < TO; r += blockDim.x) s_row[r] = (r < th) ? F.row[row0 + r] : 0.0f;
  __syncthreads();
  const int64_t* ids = ((p.batch_ids != nullptr) ? p.batch_ids : F.ids) + id_base + start;
  const float4* rec = p.records + 2 * (size_t)F.g_base;
  const int4* box = p.boxes + F.g_base;
  const float nclamp = p.cfg.nclamp;

  for (int64_t i = warp; i < count; i += 8) {
    const int64_t gid = ids[i];
    bool ok = (gid >= 0) && (gid < F.K);
    if (ok && i > 0) ok = ids[i - 1] < gid;
    int4 b = make_int4(0, -1, 0, -1);
    if (ok) {
      b = box[gid];
      ok = (b.x <= tr) & (tr <= b.y) & (b.z <= tc) & (tc <= b.w);
    }
    if (!ok) {
      if (lane == 0) atomicOr(p.status, GF_FLAG_STATE);
      continue;
    }
    const float4 a = rec[2 * gid];
    const float4 h = rec[2 * gid + 1];
    float ch[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int cb = 0; cb < tw; cb += 32) {
      const int c = cb + lane;
      const bool cval = c < tw;
      const float cc = cval ? F.col[col0 + c] : 0.0f;
      const float dy = cval ? __fsub_rn(cc, a.y) : 0.0f;
      const float a01 = __fmul_rn(h.y, dy);
      const float a11 = __fmul_rn(h.z, dy);
      // running sums: [0] T0, [1] U0, [2] U1, [3] U2, [4] M0, [5] M1; rows are
      // summed in blocks of 8 and the blocks added, so the rounding error grows
      // with 8 + th/8 terms instead of th
      float acc[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      const float* gcol = s_g + (cval ? c : 0);
      for (int r8 = 0; r8 < th; r8 += 8) {
        float blk[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        const int rend = min(th, r8 + 8);
        for (int r = r8; r < rend; ++r) {
          const float dx = __fsub_rn(s_row[r], a.x);
          float q = quad_scaled(dx, dy, h.x, a01, h.y, a11);
          q = fminf(q, 0.0f);
          bool act = true;
          if (CLAMP) {
            act = q > nclamp;          // reference: quad < clamp
            q = fmaxf(q, nclamp);
          }
          float e = expf(q);
          if (NORM) e = __fmul_rn(e, fabsf(a.w));  // the sign carries a clamp flag
          const float gb = __fmul_rn(cval ? gcol[r * TI] : 0.0f, e);
          const float gba = act ? gb : 0.0f;
          blk[0] = __fadd_rn(blk[0], gb);
          blk[1] = __fadd_rn(blk[1], gba);
          blk[2] = __fmaf_rn(gba, dx, blk[2]);
          blk[3] = __fmaf_rn(__fmul_rn(gba, dx), dx, blk[3]);
          // the reference's per-element mu factors (backward.cu:338-340) as
          // its build rounds them, dq/dmu0 = -fma(2*A01, dy, 2*A00*dx), here
          // scaled by -1/4 (exact): fma(h01, dy, h00*dx), fma(h11, dy, h01*dx)
          blk[4] = __fmaf_rn(gba, __fmaf_rn(h.y, dy, __fmul_rn(h.x, dx)), blk[4]);
          blk[5] = __fmaf_rn(gba, __fmaf_rn(h.z, dy, __fmul_rn(h.y, dx)), blk[5]);
        }
#pragma unroll
        for (int k = 0; k < 6; ++k) acc[k] = __fadd_rn(acc[k], blk[k]);
      }
      const float dyU0 = __fmul_rn(dy, acc[1]);
      ch[0] = __fadd_rn(ch[0], acc[0]);
      ch[1] = __fadd_rn(ch[1], -2.0f * acc[4]);
      ch[2] = __fadd_rn(ch[2], -2.0f * acc[5]);
      ch[3] = __fadd_rn(ch[3], acc[3]);
      ch[4] = __fadd_rn(ch[4], __fmul_rn(dy, acc[2]));
      ch[5] = __fadd_rn(ch[5], __fmul_rn(dy, dyU0));
    }
#pragma unroll
    for (int k = 0; k < 6; ++k) ch[k] = warp_sum(ch[k]);
    if (lane == 0) {
      const int64_t slot = p.goff[F.g_base + gid] + (int64_t)(tr - b.x) * (b.w - b.z + 1) + (tc - b.z);
      if (slot >= 0 && slot < p.part_cap) {
        p.partials[2 * slot] = make_float4(ch[0], ch[1], ch[2], ch[3]);
        p.partials[2 * slot + 1] = make_float4(ch[4], ch[5], 0.0f, 0.0f);
      } else {
        atomicOr(p.status, GF_FLAG_STATE);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Backward kernel 2, 32x32-tile fast path: one CTA of kBwd32Warps warps per
// tile; warp w handles the tile's pairs w, w+W, ...  The tile's dL/d(delta)
// is staged once in shared memory, transposed (s_gt[col][row], row stride 36
// floats so each lane's 128-bit read of four consecutive rows is aligned and
// conflict free), next to the 32 row coordinates.  Lane = column; rows go in
// pairs through packed fp32x2 arithmetic; the quadratic form is evaluated
// exactly as in the forward.  Per pair, the terms that depend on the row only
// (dx and the reference-rounded products h00*dx, h01*dx) are computed once,
// lane = row, into the warp's slice of shared memory and read back as
// broadcasts.  Two warps per CTA: with ~14 pairs per tile, wider CTAs leave
// warps idle at the tile's end.  The six per-pair channels are reduced across the warp with a
// reduce-scatter (9 shuffles instead of 30); lanes 0, 4, ..., 28 then hold
// channels 0..7 and write the pair's slot with one 32-byte store.
//
// Clamped elements (quad >= clamp_quad) lose their q-gradient
// (backward.cu:318-321), which costs a max, a compare and a select per
// element.  The quadratic form is convex, so over the rectangle spanned by the
// tile's row and column coordinates (min to max, whatever their order) it is
// largest at a corner; four lanes evaluate one corner each, and when every
// corner is below the clamp by more than 1e-5 of the sum of its absolute terms
// (about 20x the worst fp32 evaluation error of the element formula), no
// element of the pair can be clamped and the loop without that bookkeeping
// runs.  Results are identical either way.  The next pair's id, box and record
// are loaded while the current pair computes.
#ifndef GF_BWD32_WARPS
#define GF_BWD32_WARPS 2
#endif
// row stride of the transposed dL/d(delta) tile: 36 floats keeps every
// column 16-byte aligned and the lanes' 128-bit reads conflict-free
constexpr int kGtStride = 36;
constexpr int kBwd32Warps = GF_BWD32_WARPS;

struct PairSums {
  f2 T0, U0, U1, U2, M0, M1;
};

// Backward basis with GF_CFG_BWD_EXP2: exp(q) = 2^(q * log2 e), one
// multiply and the hardware base-2 approximation (ex2.approx.ftz).  The
// rounding of the product costs a relative error of about |q| * 6e-8 in the
// basis, i.e. at most ~2e-8 of the largest term once weighted by e^q (q <= 0);
// ex2.approx adds a few 1e-7.  Every gradient term keeps its relative
// accuracy to ~3e-7, inside the backward's tolerance.  The forward always
// uses CUDA's expf, which the bit parity of delta requires.
__device__ __forceinline__ float exp_via_ex2(float q) { return ex2_approx(__fmul_rn(q, kLog2e)); }

// One row pair (rows 2k, 2k+1 in the two halves of each argument): the row
// terms DX = row - mu_r, P0 = round(h00 * DX) and P1 = round(h01 * DX) (the
// same for every lane, computed once per row by bwd32_pairs) and the rows'
// dL/d(delta) G2 of this lane's column.
template <bool NORM, bool TRACK_CLAMP, bool EX2>
__device__ __forceinline__ void bwd32_row_pair(PairSums& S, f2 DX, f2 P0, f2 P1, f2 G2, f2 H00, f2 H01, f2 H11,
                                               f2 A01, f2 A11, f2 DY, float nclamp, float nf) {
  const f2 T1 = fma2(H00, DX, A01);
  const f2 T2 = fma2(H01, DX, A11);
  const f2 Q = fma2(DX, T1, mul2(DY, T2));
  float q0, q1;
  f2 E2 = 0;
  if (EX2 && !TRACK_CLAMP) {
    // base-2 basis: one packed scaling; the max(quad, 0) of the reference
    // only removes rounding noise of order 1e-7 here (2^q = 1 + O(q))
    E2 = ex2_2(mul2(Q, pk2(kLog2e, kLog2e)));
  } else {
    up2(Q, q0, q1);
    q0 = fminf(q0, 0.0f);
    q1 = fminf(q1, 0.0f);
  }
  bool act0 = true, act1 = true;
  if (TRACK_CLAMP) {
    act0 = q0 > nclamp;  // reference: quad < clamp
    act1 = q1 > nclamp;
    q0 = fmaxf(q0, nclamp);
    q1 = fmaxf(q1, nclamp);
  }
  if (!(EX2 && !TRACK_CLAMP)) {
    float e0, e1;
    if (EX2) {
      e0 = exp_via_ex2(q0);
      e1 = exp_via_ex2(q1);
    } else {
      e0 = expf(q0);
      e1 = expf(q1);
    }
    E2 = pk2(e0, e1);
  }
  if (NORM) E2 = mul2(E2, pk2(nf, nf));
  const f2 GB = mul2(G2, E2);
  if (TRACK_CLAMP) S.T0 = add2(S.T0, GB);  // without clamped elements T0 == U0 (same terms, same order)
  f2 GBA = GB;
  if (TRACK_CLAMP) {
    float b0, b1;
    up2(GB, b0, b1);
    GBA = pk2(act0 ? b0 : 0.0f, act1 ? b1 : 0.0f);
  }
  S.U0 = add2(S.U0, GBA);
  S.U1 = fma2(GBA, DX, S.U1);
  S.U2 = fma2(mul2(GBA, DX), DX, S.U2);
  // per-element mu factors with the reference's roundings (see render_bwd_kernel)
  S.M0 = fma2(GBA, fma2(H01, DY, P0), S.M0);
  S.M1 = fma2(GBA, fma2(H11, DY, P1), S.M1);
}

// Sum over the 32 rows of one lane's column for one pair: the row terms
// (s_rt: DX[32], P0[32], P1[32] of this warp) and the column's dL/d(delta)
// come from shared memory four rows at a time (128-bit loads; the row terms
// are broadcasts, the column is this lane's own).
template <bool NORM, bool TRACK_CLAMP, bool EX2>
__device__ __forceinline__ PairSums bwd32_pair_rows(const float* s_rt, const float* s_gcol, f2 H00, f2 H01,
                                                   f2 H11, f2 A01, f2 A11, f2 DY, float nclamp, float nf) {
  const f2 zero2 = pk2(0.0f, 0.0f);
  PairSums S{zero2, zero2, zero2, zero2, zero2, zero2};
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float4 dx = *reinterpret_cast<const float4*>(&s_rt[4 * k]);
    const float4 p0 = *reinterpret_cast<const float4*>(&s_rt[32 + 4 * k]);
    const float4 p1 = *reinterpret_cast<const float4*>(&s_rt[64 + 4 * k]);
    const float4 gg = *reinterpret_cast<const float4*>(&s_gcol[4 * k]);
    bwd32_row_pair<NORM, TRACK_CLAMP, EX2>(S, pk2(dx.x, dx.y), pk2(p0.x, p0.y), pk2(p1.x, p1.y), pk2(gg.x, gg.y),
                                           H00, H01, H11, A01, A11, DY, nclamp, nf);
    bwd32_row_pair<NORM, TRACK_CLAMP, EX2>(S, pk2(dx.z, dx.w), pk2(p0.z, p0.w), pk2(p1.z, p1.w), pk2(gg.z, gg.w),
                                           H00, H01, H11, A01, A11, DY, nclamp, nf);
  }
  if (!TRACK_CLAMP) S.T0 = S.U0;
  return S;
}

// One tile's work in the 32x32 backward: its field, position, pair range in
// the id list and whether its dL/d(delta) block can be staged with 16-byte
// copies.  False when the tile has nothing to do here (no pairs, a heavy tile
// left to render_bwd32_heavy_kernel, or inconsistent saved state, which
// raises GF_FLAG_STATE).  Every thread of the CTA computes the same job.
struct Bwd32Job {
  int fi, tr, tc, th, tw, count;
  int64_t start, id_base;
  bool vec;
};

template <int NF>
__device__ __forceinline__ bool bwd32_job(const Params<NF>& p, int tg, bool skip_heavy, Bwd32Job& j) {
  j.fi = field_of_tile(p, tg);
  const DevField& F = p.f[j.fi];
  const int t = tg - F.tile_base;
  j.tr = t / F.ntc;
  j.tc = t % F.ntc;
  j.start = F.tile_ptr[t];
  const int64_t count64 = F.tile_ptr[t + 1] - j.start;
  if (count64 <= 0) return false;
  j.id_base = (p.batch_ids != nullptr) ? p.pair_base[j.fi] : 0;
  const int64_t id_limit = (p.batch_ids != nullptr) ? p.batch_cap : F.ids_cap;
  // a tile holds at most K pairs (one per Gaussian), K < 2^30
  if (j.start < 0 || j.id_base < 0 || j.id_base + j.start + count64 > id_limit || count64 > F.K) {
    if (threadIdx.x == 0) atomicOr(p.status, GF_FLAG_STATE);
    return false;
  }
  j.count = (int)count64;
  if (skip_heavy && j.count > kHeavyPairs) return false;  // chunks of it go to render_bwd32_heavy_kernel
  const int row0 = j.tr * 32, col0 = j.tc * 32;
  j.th = min(32, F.out_f - row0);
  j.tw = min(32, F.in_f - col0);
  const size_t gbase = (size_t)row0 * F.in_f + col0;
  j.vec = j.th == 32 && j.tw == 32 && (F.bits & kFieldGradVecOk) &&
          GF_IN_BOUNDS(gbase + (size_t)31 * F.in_f + 31 < (size_t)F.out_f * F.in_f);
  return true;
}

// Stages the tile's row coordinates and its dL/d(delta) block, transposed to
// s_gt[col][row], with plain loads (the caller synchronises afterwards).
template <int NF, int GT>
__device__ __forceinline__ void bwd32_stage_sync(const Params<NF>& p, const Bwd32Job& j, float* s_rows,
                                                 float* s_gt) {
  const DevField& F = p.f[j.fi];
  const int th = j.th, tw = j.tw;
  const int row0 = j.tr * 32, col0 = j.tc * 32;
  if (threadIdx.x < 32) s_rows[threadIdx.x] = (threadIdx.x < th) ? F.row[row0 + threadIdx.x] : 0.0f;
  // dL/d(delta) of the tile, transposed into s_gt[col][row]
  const size_t gbase = (size_t)row0 * F.in_f + col0;
  if (j.vec) {
    if (GT == GF_F32) {
#pragma unroll
      for (int k = 0; k < (256 + 32 * kBwd32Warps - 1) / (32 * kBwd32Warps); ++k) {  // 256 16-byte loads of 4 floats
        const int q = threadIdx.x + k * (32 * kBwd32Warps);
        if (q < 256) {
          const int r = q >> 3, c = (q & 7) * 4;
          const float4 v = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(F.grad) + gbase +
                                                            (size_t)r * F.in_f + c);
          s_gt[(c + 0) * kGtStride + r] = v.x;
          s_gt[(c + 1) * kGtStride + r] = v.y;
          s_gt[(c + 2) * kGtStride + r] = v.z;
          s_gt[(c + 3) * kGtStride + r] = v.w;
        }
      }
    } else {
      for (int q = threadIdx.x; q < 128; q += 32 * kBwd32Warps) {  // 128 16-byte loads of 8 bf16
        const int r = q >> 2, c = (q & 3) * 8;
        const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(F.grad) + gbase +
                                                        (size_t)r * F.in_f + c);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
          s_gt[(c + 2 * k) * kGtStride + r] = f.x;
          s_gt[(c + 2 * k + 1) * kGtStride + r] = f.y;
        }
      }
    }
  } else {
    for (int e = threadIdx.x; e < 1024; e += blockDim.x) {
      const int r = e >> 5, c = e & 31;
      s_gt[c * kGtStride + r] =
          (r < th && c < tw && GF_IN_BOUNDS((size_t)(row0 + r) * F.in_f + col0 + c < (size_t)F.out_f * F.in_f))
              ? load_grad<GT>(F.grad, (size_t)(row0 + r) * F.in_f + col0 + c)
              : 0.0f;
    }
  }
}

// Sums pairs [lo, hi) of the tile (warp w takes lo + w, lo + w + kBwd32Warps,
// ...) over its staged block and stores each pair's eight partial channels.
template <int NF, bool NORM, bool CLAMP, int GT, bool EX2>
__device__ __forceinline__ void bwd32_pairs(const Params<NF>& p, const Bwd32Job& j, int lo, int hi,
                                            const float* s_rows, const float* s_gt, float* s_rt) {
  const DevField& F = p.f[j.fi];
  const int tr = j.tr, tc = j.tc, th = j.th, tw = j.tw;
  const int64_t start = j.start, id_base = j.id_base;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int col0 = tc * 32;
  if (lo + warp >= hi) return;
  const bool cval = lane < tw;
  const float cc = cval ? F.col[col0 + lane] : 0.0f;
  // Per-tile clamp test for Gaussians flagged by bwd_prep (record norm < 0):
  // lanes 0..3 each evaluate one corner of the tile's coordinate rectangle
  // (the flag is only clear when the axes are monotonic, so the rectangle is
  // spanned by the first and last row and column; otherwise flagged
  // Gaussians always take the clamp bookkeeping).
  const float corner_r = s_rows[(lane & 1) ? th - 1 : 0];
  const float corner_c = F.col[col0 + ((lane & 2) ? tw - 1 : 0)];
  const float* s_gcol = &s_gt[lane * kGtStride];
  const int64_t* ids = ((p.batch_ids != nullptr) ? p.batch_ids : F.ids) + id_base + start;
  const float4* rec = p.records + 2 * (size_t)F.g_base;
  const int4* box = p.boxes + F.g_base;
  const int64_t* goff = p.goff + F.g_base;
  const float nclamp = p.cfg.nclamp;
  // channel held by this lane after the reduce-scatter: bits 4,3,2 of lane
  const int my_ch = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);

  // software pipeline: the next pair's id, box and record load while this one computes
  const int i0 = lo + warp;
  int gid = (int)ids[i0];
  bool okn = (ids[i0] >= 0) && (ids[i0] < F.K) && (i0 == 0 || ids[i0 - 1] < ids[i0]);
  int4 bn = okn ? box[gid] : make_int4(0, -1, 0, -1);
  float4 an = okn ? rec[2 * gid] : make_float4(0.f, 0.f, 0.f, 0.f);
  float4 hn = okn ? rec[2 * gid + 1] : make_float4(0.f, 0.f, 0.f, 0.f);
  int64_t gon = okn ? goff[gid] : -1;
  for (int i = i0; i < hi; i += kBwd32Warps) {
    const int4 b = bn;
    const float4 a = an, h = hn;
    const int64_t go = gon;
    const bool ok = okn && (b.x <= tr) & (tr <= b.y) & (b.z <= tc) & (tc <= b.w);
    const int inext = i + kBwd32Warps;
    if (inext < hi) {
      const int64_t idn = ids[inext], idp = ids[inext - 1];
      okn = (idn >= 0) && (idn < F.K) && (idp < idn);
      gid = (int)idn;
      if (okn) {
        bn = box[gid];
        an = rec[2 * gid];
        hn = rec[2 * gid + 1];
        gon = goff[gid];
      }
    }
    if (!ok) {
      if (lane == 0) atomicOr(p.status, GF_FLAG_STATE);
      continue;
    }
    const float dy = cval ? __fsub_rn(cc, a.y) : 0.0f;
    const float a01 = __fmul_rn(h.y, dy);
    const float a11 = __fmul_rn(h.z, dy);
    const f2 H00 = pk2(h.x, h.x), H01 = pk2(h.y, h.y), A01 = pk2(a01, a01), A11 = pk2(a11, a11);
    const f2 DY = pk2(dy, dy);
    // the row terms of this pair, one row per lane, for the whole warp
    __syncwarp();
    {
      const float dxl = __fsub_rn(s_rows[lane], a.x);
      s_rt[lane] = dxl;
      s_rt[32 + lane] = __fmul_rn(h.x, dxl);
      s_rt[64 + lane] = __fmul_rn(h.y, dxl);
    }
    __syncwarp();
    bool track = false;
    // With the base-2 basis (tolerance-bound) a clamp at quad >= 64 is not
    // tracked: a clamped element's basis is below e^-32 = 1.3e-14 of the
    // Gaussian's peak, under the fp32 resolution of every term that matters.
    if (CLAMP && a.w < 0.0f && !(EX2 && nclamp <= -32.0f)) {  // flagged by bwd_prep: test this tile's corners
      const bool far = corner_bound(corner_r - a.x, corner_c - a.y, h.x, h.y, h.z) > nclamp;
      track = !__all_sync(0xffffffffu, far || lane >= 4);
    }
    const f2 H11 = pk2(h.z, h.z);
    const float nf = fabsf(a.w);
    PairSums S = track
                     ? bwd32_pair_rows<NORM, true, EX2>(s_rt, s_gcol, H00, H01, H11, A01, A11, DY, nclamp, nf)
                     : bwd32_pair_rows<NORM, false, EX2>(s_rt, s_gcol, H00, H01, H11, A01, A11, DY, nclamp, nf);
    float t0a, t0b, u0a, u0b, u1a, u1b, u2a, u2b, m0a, m0b, m1a, m1b;
    up2(S.T0, t0a, t0b);
    up2(S.U0, u0a, u0b);
    up2(S.U1, u1a, u1b);
    up2(S.U2, u2a, u2b);
    up2(S.M0, m0a, m0b);
    up2(S.M1, m1a, m1b);
    const float u0 = __fadd_rn(u0a, u0b), u1 = __fadd_rn(u1a, u1b);
    const float dyU0 = __fmul_rn(dy, u0);
    float ch[8] = {__fadd_rn(t0a, t0b), -2.0f * __fadd_rn(m0a, m0b), -2.0f * __fadd_rn(m1a, m1b),
                   __fadd_rn(u2a, u2b), __fmul_rn(dy, u1), __fmul_rn(dy, dyU0), 0.0f, 0.0f};
    // reduce-scatter over the warp: 8 -> 4 -> 2 -> 1 channels, then 4-lane sums
    {
      const bool hi = (lane >> 4) & 1;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float keep = hi ? ch[4 + k] : ch[k];
        const float send = hi ? ch[k] : ch[4 + k];
        ch[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
      }
    }
    {
      const bool hi = (lane >> 3) & 1;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const float keep = hi ? ch[2 + k] : ch[k];
        const float send = hi ? ch[k] : ch[2 + k];
        ch[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
      }
    }
    {
      const bool hi = (lane >> 2) & 1;
      const float keep = hi ? ch[1] : ch[0];
      const float send = hi ? ch[0] : ch[1];
      ch[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    ch[0] += __shfl_xor_sync(0xffffffffu, ch[0], 2);
    ch[0] += __shfl_xor_sync(0xffffffffu, ch[0], 1);
    const int64_t slot = go + (tr - b.x) * (b.w - b.z + 1) + (tc - b.z);
    if (slot >= 0 && slot < p.part_cap) {
      if ((lane & 3) == 0) reinterpret_cast<float*>(p.partials)[8 * slot + my_ch] = ch[0];
    } else if (lane == 0) {
      atomicOr(p.status, GF_FLAG_STATE);
    }
  }
}

// One tile (or one chunk of a heavy tile's pairs), staged with plain loads.
template <int NF, bool NORM, bool CLAMP, int GT, bool EX2>
__device__ __forceinline__ void bwd32_tile(const Params<NF>& p, int tg, int pair_lo, int pair_hi, bool skip_heavy,
                                           float* s_rows, float* s_gt, float* s_rt) {
  Bwd32Job j;
  if (!bwd32_job(p, tg, skip_heavy, j)) return;
  const int lo = pair_lo, hi = min(pair_hi, j.count);
  if (lo >= hi) return;
  bwd32_stage_sync<NF, GT>(p, j, s_rows, s_gt);
  __syncthreads();
  bwd32_pairs<NF, NORM, CLAMP, GT, EX2>(p, j, lo, hi, s_rows, s_gt, s_rt + 96 * (threadIdx.x >> 5));
}

template <int NF, bool NORM, bool CLAMP, int GT, bool EX2>
__global__ void __launch_bounds__(32 * kBwd32Warps)
render_bwd32_kernel(const __grid_constant__ Params<NF> p) {
  __shared__ __align__(16) float s_rows[32];
  __shared__ __align__(16) float s_gt[32 * kGtStride];
  __shared__ __align__(16) float s_rt[kBwd32Warps * 96];
  bwd32_tile<NF, NORM, CLAMP, GT, EX2>(p, blockIdx.x, 0, INT32_MAX, true, s_rows, s_gt, s_rt);
}

// Chunks of kHeavyChunk pairs of the heavy tiles (listed by bwd_prep), CTAs
// striding over the list: a tile with hundreds of pairs is spread over many
// CTAs instead of its own four warps.
template <int NF, bool NORM, bool CLAMP, int GT, bool EX2>
__global__ void __launch_bounds__(32 * kBwd32Warps)
render_bwd32_heavy_kernel(const __grid_constant__ Params<NF> p) {
  __shared__ __align__(16) float s_rows[32];
  __shared__ __align__(16) float s_gt[32 * kGtStride];
  __shared__ __align__(16) float s_rt[kBwd32Warps * 96];
  const int n = min((int)*reinterpret_cast<volatile uint32_t*>(p.heavy_count), p.heavy_cap);
  const int2* items = reinterpret_cast<const int2*>(p.heavy);
  for (int i = blockIdx.x; i < n; i += gridDim.x) {
    const int2 it = items[i];
    bwd32_tile<NF, NORM, CLAMP, GT, EX2>(p, it.x, it.y * kHeavyChunk, (it.y + 1) * kHeavyChunk, false, s_rows, s_gt,
                                         s_rt);
    __syncthreads();  // the next chunk restages the shared tile
  }
}

// Backward kernel 3: one warp per Gaussian.  Sums the Gaussian's pair
// partials (contiguous, fixed order) in fp64, applies amp and -0.5, and
// evaluates the covariance chain of backward.cu:436-496 in fp64 before the
// final fp32 store.  The chain dSigma = -A G A cancels strongly for
// elongated Gaussians (|A| up to ~1e5); in fp32 that cancellation costs up to
// ~1e-4 of the result, in fp64 nothing measurable.  Per Gaussian this is a
// few dozen fp64 operations.
template <int NF, bool NORM>
__global__ void __launch_bounds__(kRenderThreads)
bwd_finalize_kernel(const __grid_constant__ Params<NF> p) {
  const int lane = threadIdx.x & 31;
  const int G = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (G >= p.total_g) return;
  const int fi = field_of_gaussian(p, G);
  const DevField& F = p.f[fi];
  const int g = G - F.g_base;
  const int4 b = p.boxes[G];
  const int64_t n = (int64_t)(b.y - b.x + 1) * (b.w - b.z + 1);
  const int64_t o = p.goff[G];
  double s[6] = {0.0, 0.0, 0.0, 0.0, 0.0, 0.0};
  const int64_t jn = (o >= 0 && o + n <= p.part_cap) ? n : 0;  // inconsistent state was flagged already
  for (int64_t j = lane; j < jn; j += 32) {
    const float4 x = p.partials[2 * (o + j)];
    const float4 y = p.partials[2 * (o + j) + 1];
    s[0] += x.x; s[1] += x.y; s[2] += x.z; s[3] += x.w; s[4] += y.x; s[5] += y.y;
  }
#pragma unroll
  for (int k = 0; k < 6; ++k) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s[k] += __shfl_xor_sync(0xffffffffu, s[k], off);
  }
  if (lane != 0) return;
  const float mu_r = F.mu[2 * g], mu_c = F.mu[2 * g + 1];
  const float raw11 = F.chol[3 * g], raw21 = F.chol[3 * g + 1], raw22 = F.chol[3 * g + 2];
  const Geo geo = geometry(mu_r, mu_c, raw11, raw21, raw22, F, p.cfg);
  const double amp = F.amp[g];
  F.d_amp[g] = (float)s[0];
  F.d_mu[2 * g] = (float)(amp * s[1]);
  F.d_mu[2 * g + 1] = (float)(amp * s[2]);
  const double m = -0.5 * amp;
  const double g00 = m * s[3], g01 = m * s[4], g10 = g01, g11 = m * s[5];
  const double det = geo.det;
  double gdet = 0.0;
  if (NORM) gdet = amp * (-0.5 / (double)fmaxf(geo.det, kCovFloor)) * s[0];
  // backward.cu:469-495 with A^T = A (A01 == A10)
  const double a00 = geo.i00, a01 = geo.i01, a11 = geo.i11;
  const double b00 = g00 * a00 + g01 * a01;
  const double b01 = g00 * a01 + g01 * a11;
  const double b10 = g10 * a00 + g11 * a01;
  const double b11 = g10 * a01 + g11 * a11;
  const double c00 = -(a00 * b00 + a01 * b10) + gdet * det * a00;
  const double c01 = -(a00 * b01 + a01 * b11) + gdet * det * a01;
  const double c10 = -(a01 * b00 + a11 * b10) + gdet * det * a01;
  const double c11 = -(a01 * b01 + a11 * b11) + gdet * det * a11;
  const double l11 = geo.l11, l21 = geo.l21, l22 = geo.l22;
  const double d_l11 = c00 * (2.0 * l11) + c01 * l21 + c10 * l21;
  const double d_l21 = c01 * l11 + c10 * l11 + c11 * (2.0 * l21);
  const double d_l22 = c11 * (2.0 * l22);
  const double sg11 = 1.0 / (1.0 + exp(-(double)raw11));
  const double sg22 = 1.0 / (1.0 + exp(-(double)raw22));
  F.d_chol[3 * g] = (float)(d_l11 * sg11);
  F.d_chol[3 * g + 1] = (float)d_l21;
  F.d_chol[3 * g + 2] = (float)(d_l22 * sg22);
}

// ---------------------------------------------------------------------------
// Host side.

thread_local std::string g_last_error;

// Process-wide: an autograd backward runs on its own thread, and its trace
// events belong to the same step as the forward's.
struct Trace {
  void* const* ev = nullptr;
  int n = 0;
  int used = 0;
};
Trace g_trace;
std::mutex g_trace_mu;

// NVTX range over the host-side enqueue of one stage ("gfield.<stage>"), so a
// timeline profiler shows each entry point and kernel launch by name.  A
// no-op unless a tool is attached.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

inline void trace_mark(cudaStream_t st) {
  std::lock_guard<std::mutex> lock(g_trace_mu);
  if (g_trace.used < g_trace.n) {
    cudaEventRecord(reinterpret_cast<cudaEvent_t>(g_trace.ev[g_trace.used]), st);
    ++g_trace.used;
  }
}

gf_status fail(gf_status s, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
gf_status fail(gf_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return s;
}

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Layout {
  size_t hdr, records, boxes, goff, field_pairs, diff, cursor, heavy, partials, total;
  int64_t total_tiles, total_g, diff_ints, pair_cap;
  int64_t heavy_items; // backward: capacity of the heavy-tile work items
};

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

gf_status validate(const gf_config* cfg, const gf_batch* batch, gf_pass pass, bool data = true) {
  if (!cfg || !batch) return fail(GF_ERR_INVALID_ARG, "cfg and batch must be non-null");
  if (cfg->tile_out <= 0) return fail(GF_ERR_INVALID_ARG, "tile_out must be positive");
  if (cfg->tile_in <= 0) return fail(GF_ERR_INVALID_ARG, "tile_in must be positive");
  if (!(cfg->sigma_multiplier > 0.0)) return fail(GF_ERR_INVALID_ARG, "sigma_multiplier must be positive");
  if (cfg->out_dtype != GF_F32 && cfg->out_dtype != GF_BF16) return fail(GF_ERR_INVALID_ARG, "out_dtype must be GF_F32 or GF_BF16");
  if (cfg->grad_dtype != GF_F32 && cfg->grad_dtype != GF_BF16) return fail(GF_ERR_INVALID_ARG, "grad_dtype must be GF_F32 or GF_BF16");
  if (cfg->flags & ~(GF_CFG_BWD_EXP2 | GF_CFG_FWD_EXP2)) return fail(GF_ERR_INVALID_ARG, "unknown gf_config.flags bits 0x%x", cfg->flags);
  if (batch->num_fields < 1 || batch->num_fields > GF_MAX_FIELDS)
    return fail(GF_ERR_INVALID_ARG, "num_fields must be in [1, %d], got %d", GF_MAX_FIELDS, batch->num_fields);
  if (!batch->fields) return fail(GF_ERR_INVALID_ARG, "fields must be non-null");
  if (batch->ids && !batch->pair_base) return fail(GF_ERR_INVALID_ARG, "pair_base is required with a shared ids buffer");
  if (pass == GF_PASS_BACKWARD && (int64_t)cfg->tile_out * cfg->tile_in > kBwdSmemCapFloats - cfg->tile_out)
    return fail(GF_ERR_UNSUPPORTED, "tile_out*tile_in too large for the backward shared-memory tile");
  int64_t tiles = 0, gs = 0;
  for (int i = 0; i < batch->num_fields; ++i) {
    const gf_field& f = batch->fields[i];
    if (f.out_features <= 0 || f.in_features <= 0)
      return fail(GF_ERR_INVALID_ARG, "field %d: out_features and in_features must be positive", i);
    if (f.num_gaussians < 0) return fail(GF_ERR_INVALID_ARG, "field %d: num_gaussians must be >= 0", i);
    if (f.out_features > INT32_MAX / 2 || f.in_features > INT32_MAX / 2 || f.num_gaussians > INT32_MAX / 2)
      return fail(GF_ERR_UNSUPPORTED, "field %d: dimensions exceed the 32-bit index envelope", i);
    if (!data) {
      tiles += ceil_div(f.out_features, cfg->tile_out) * ceil_div(f.in_features, cfg->tile_in);
      gs += f.num_gaussians;
      continue;
    }
    if (!f.row_coords || !f.col_coords || !f.tile_ptr)
      return fail(GF_ERR_INVALID_ARG, "field %d: row_coords, col_coords and tile_ptr must be non-null", i);
    if (f.num_gaussians > 0 && (!f.mu || !f.chol_raw || !f.amp))
      return fail(GF_ERR_INVALID_ARG, "field %d: mu, chol_raw and amp must be non-null", i);
    if (!batch->ids && f.ids_capacity > 0 && !f.gaussian_ids)
      return fail(GF_ERR_INVALID_ARG, "field %d: gaussian_ids must be non-null", i);
    if (!batch->ids && f.ids_capacity < 0) return fail(GF_ERR_INVALID_ARG, "field %d: ids_capacity must be >= 0", i);
    if (pass == GF_PASS_FORWARD && !f.delta) return fail(GF_ERR_INVALID_ARG, "field %d: delta must be non-null", i);
    if (pass == GF_PASS_FORWARD && f.delta_multicast) {
      const int64_t vec = cfg->out_dtype == GF_F32 ? 4 : 8;  // elements per 16-byte store
      if (((reinterpret_cast<uintptr_t>(f.delta) | reinterpret_cast<uintptr_t>(f.delta_multicast)) & 15u) ||
          f.in_features % vec || cfg->tile_in % vec)
        return fail(GF_ERR_UNSUPPORTED,
                    "field %d: delta_multicast needs 16-byte aligned delta rows (aligned delta and multicast "
                    "address, in_features and tile_in multiples of %lld)", i, (long long)vec);
    }
    if (pass == GF_PASS_BACKWARD) {
      if (!f.grad_delta) return fail(GF_ERR_INVALID_ARG, "field %d: grad_delta must be non-null", i);
      if (f.num_gaussians > 0 && (!f.d_mu || !f.d_chol_raw || !f.d_amp))
        return fail(GF_ERR_INVALID_ARG, "field %d: d_mu, d_chol_raw and d_amp must be non-null", i);
    }
    tiles += ceil_div(f.out_features, cfg->tile_out) * ceil_div(f.in_features, cfg->tile_in);
    gs += f.num_gaussians;
  }
  if (tiles > INT32_MAX / 2 || gs > INT32_MAX / 2) return fail(GF_ERR_UNSUPPORTED, "batch exceeds the 32-bit index envelope");
  return GF_OK;
}

Layout layout(const gf_config* cfg, const gf_batch* batch, gf_pass pass) {
  Layout L{};
  for (int i = 0; i < batch->num_fields; ++i) {
    const gf_field& f = batch->fields[i];
    const int64_t ntr = ceil_div(f.out_features, cfg->tile_out), ntc = ceil_div(f.in_features, cfg->tile_in);
    L.total_tiles += ntr * ntc;
    L.total_g += f.num_gaussians;
    const int64_t nd = (ntr + 1) * (ntc + 1);
    if (nd > kBinSmemCapInts) L.diff_ints += nd;
    if (!batch->ids) L.pair_cap += f.ids_capacity;
  }
  if (batch->ids) L.pair_cap = batch->ids_capacity;
  size_t off = 0;
  L.hdr = off; off += 256;
  L.records = off; off = align256(off + 32 * (size_t)L.total_g);
  L.boxes = off; off = align256(off + 16 * (size_t)L.total_g);
  L.goff = off; off = align256(off + 8 * (size_t)L.total_g);
  L.field_pairs = off; off = align256(off + 8 * (size_t)batch->num_fields);
  L.diff = off; off = align256(off + 4 * (size_t)L.diff_ints);
  L.cursor = off;
  if (pass == GF_PASS_FORWARD) off = align256(off + 4 * (size_t)L.total_tiles);
  L.heavy = off;
  if (pass == GF_PASS_FORWARD) {
    off = align256(off + 4 * (size_t)L.total_tiles);
  } else {  // (tile, chunk) items: at most pairs / kHeavyChunk + one partial chunk per tile
    L.heavy_items = L.pair_cap / kHeavyChunk + L.total_tiles;
    if (L.heavy_items > INT32_MAX) L.heavy_items = INT32_MAX;
    off = align256(off + 8 * (size_t)L.heavy_items);
  }
  L.partials = off;
  if (pass == GF_PASS_BACKWARD) off = align256(off + 32 * (size_t)L.pair_cap);
  L.total = off;
  return L;
}

template <int NF>
void fill_params(Params<NF>& P, const gf_config* cfg, const gf_batch* batch, const Layout& L, char* ws) {
  memset(&P, 0, sizeof(P));
  P.cfg.tile_out = (int32_t)cfg->tile_out;
  P.cfg.tile_in = (int32_t)cfg->tile_in;
  P.cfg.sigma = (float)cfg->sigma_multiplier;
  P.cfg.nclamp = -0.5f * (float)cfg->clamp_quad;
  P.cfg.out_scale = cfg->out_scale;
  P.cfg.has_clamp = cfg->has_clamp_quad != 0;
  P.cfg.normalize = cfg->normalize != 0;
  P.cfg.flags = cfg->flags;
  P.n = batch->num_fields;
  P.total_tiles = (int32_t)L.total_tiles;
  P.total_g = (int32_t)L.total_g;
  P.status = reinterpret_cast<uint32_t*>(ws + L.hdr);
  P.done = reinterpret_cast<uint32_t*>(ws + L.hdr + 4);
  P.heavy_count = reinterpret_cast<uint32_t*>(ws + L.hdr + 8);
  P.heavy = reinterpret_cast<int32_t*>(ws + L.heavy);
  P.tile_end = (int32_t)L.total_tiles;
  P.heavy_cap = (int32_t)L.heavy_items;
  P.records = reinterpret_cast<float4*>(ws + L.records);
  P.boxes = reinterpret_cast<int4*>(ws + L.boxes);
  P.goff = reinterpret_cast<int64_t*>(ws + L.goff);
  P.field_pairs = reinterpret_cast<int64_t*>(ws + L.field_pairs);
  P.diff = reinterpret_cast<int32_t*>(ws + L.diff);
  P.cursor = reinterpret_cast<int32_t*>(ws + L.cursor);
  P.partials = reinterpret_cast<float4*>(ws + L.partials);
  P.part_cap = L.pair_cap;
  P.batch_ids = batch->ids;
  P.batch_cap = batch->ids_capacity;
  P.pair_base = batch->pair_base;
  int32_t tile_base = 0, g_base = 0, diff_base = 0;
  int64_t part_base = 0;
  const size_t esz = cfg->out_dtype == GF_BF16 ? 2 : 4;
  for (int i = 0; i < batch->num_fields; ++i) {
    const gf_field& s = batch->fields[i];
    DevField& d = P.f[i];
    d.row = s.row_coords; d.col = s.col_coords; d.mu = s.mu; d.chol = s.chol_raw; d.amp = s.amp;
    d.delta = s.delta; d.tile_ptr = s.tile_ptr; d.ids = s.gaussian_ids; d.grad = s.grad_delta;
    d.d_mu = s.d_mu; d.d_chol = s.d_chol_raw; d.d_amp = s.d_amp;
    d.base = s.base_weight;
    d.mc = reinterpret_cast<unsigned long long>(s.delta_multicast);
    d.ids_cap = s.ids_capacity;
    d.part_base = part_base;
    if (!batch->ids) part_base += s.ids_capacity;
    d.out_f = (int32_t)s.out_features;
    d.in_f = (int32_t)s.in_features;
    d.K = (int32_t)s.num_gaussians;
    d.ntr = (int32_t)ceil_div(s.out_features, cfg->tile_out);
    d.ntc = (int32_t)ceil_div(s.in_features, cfg->tile_in);
    d.tile_base = tile_base;
    d.g_base = g_base;
    const int32_t nd = (d.ntr + 1) * (d.ntc + 1);
    d.diff_base = diff_base;
    if (nd > kBinSmemCapInts) diff_base += nd;
    tile_base += d.ntr * d.ntc;
    g_base += d.K;
    const size_t vec = 16 / esz;
    d.bits = 0;
    if (((reinterpret_cast<uintptr_t>(s.delta) & 15u) == 0) &&
        ((reinterpret_cast<uintptr_t>(s.base_weight) & 15u) == 0) && (s.in_features % (int64_t)vec == 0) &&
        (cfg->tile_in % (int64_t)vec == 0))
      d.bits |= kFieldVecOk;
    const int64_t gvec = cfg->grad_dtype == GF_BF16 ? 8 : 4;
    if (((reinterpret_cast<uintptr_t>(s.grad_delta) & 15u) == 0) && (s.in_features % gvec == 0) &&
        (cfg->tile_in % gvec == 0))
      d.bits |= kFieldGradVecOk;
  }
}

#define GF_LAUNCH_CHECK(what)                                                         \
  do {                                                                                \
    cudaError_t e_ = cudaGetLastError();                                              \
    if (e_ != cudaSuccess) return fail(GF_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e_)); \
  } while (0)

// Opt a kernel in to more than 48 KB of dynamic shared memory.  The attribute
// is per device, so it is set once per (kernel, device), under a per-kernel
// flag array that concurrent host threads may race on harmlessly (setting it
// twice is idempotent).  Devices beyond the table get the call every time.
constexpr int kAttrDevices = 64;
template <auto Kernel>
cudaError_t allow_dynamic_smem(int bytes) {
  static std::atomic<int> done[kAttrDevices];
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const bool tracked = dev >= 0 && dev < kAttrDevices;
  if (tracked && done[dev].load(std::memory_order_acquire) == bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && tracked) done[dev].store(bytes, std::memory_order_release);
  return e;
}

// The per-tile id lists of the BIN stage: pair emission, then the sorts.
template <int NF>
gf_status launch_tile_lists(const Params<NF>& p, const Layout& L, cudaStream_t st) {
  if (L.total_g > 0) {
    emit_pairs_kernel<NF><<<(int)ceil_div(L.total_g, kEmitWarps), 32 * kEmitWarps, 0, st>>>(p);
    GF_LAUNCH_CHECK("emit_pairs_kernel");
  }
  sort_tiles_kernel<NF><<<(int)ceil_div(L.total_tiles, kSortWarps), 32 * kSortWarps, 0, st>>>(p);
  GF_LAUNCH_CHECK("sort_tiles_kernel");
  const int hg = L.total_tiles < kHeavyGridCap ? (int)L.total_tiles : kHeavyGridCap;
  sort_heavy_kernel<NF><<<hg, kSortThreads, 0, st>>>(p);
  GF_LAUNCH_CHECK("sort_heavy_kernel");
  return GF_OK;
}

template <int NF>
gf_status run_forward(const gf_config* cfg, const gf_batch* batch, const Layout& L, char* ws, cudaStream_t st,
                      unsigned stages = GF_STAGE_BIN | GF_STAGE_RENDER, int first_field = 0, int num_fields = -1) {
  // The descriptor block is large; keep one per thread instead of on the stack.
  thread_local Params<NF>* tp = nullptr;
  if (!tp) tp = new Params<NF>();
  Params<NF>& p = *tp;
  fill_params(p, cfg, batch, L, ws);
  int max_nd = 0;
  for (int i = 0; i < p.n; ++i) {
    const int nd = (p.f[i].ntr + 1) * (p.f[i].ntc + 1);
    if (nd <= kBinSmemCapInts && nd > max_nd) max_nd = nd;
  }
  const size_t smem = sizeof(int) * (size_t)max_nd;
  {
    const cudaError_t e = allow_dynamic_smem<bin_kernel<NF>>(kBinSmemCapInts * 4);
    if (e != cudaSuccess) return fail(GF_ERR_CUDA, "bin_kernel: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  }
  if (stages & GF_STAGE_BIN) {
    NvtxRange r("gfield.bin");
    trace_mark(st);
    if (cudaMemsetAsync(p.heavy_count, 0, sizeof(uint32_t), st) != cudaSuccess)
      return fail(GF_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(cudaGetLastError()));
    if (L.total_g > 0) {
      geometry_kernel<NF, false><<<(int)ceil_div(L.total_g, kGeoThreads), kGeoThreads, 0, st>>>(p);
      GF_LAUNCH_CHECK("geometry_kernel");
    }
    bin_kernel<NF><<<p.n, kBinThreads, smem, st>>>(p, kBinSmemCapInts);
    GF_LAUNCH_CHECK("bin_kernel");
    const gf_status sl = launch_tile_lists(p, L, st);
    if (sl != GF_OK) return sl;
    trace_mark(st);
  }
  if (!(stages & GF_STAGE_RENDER)) return GF_OK;
  NvtxRange r("gfield.render_fwd");
  const bool norm = p.cfg.normalize, clamp = p.cfg.has_clamp;
  int grid = (int)L.total_tiles;
  if (num_fields >= 0) {  // a field range: its tiles are contiguous in the global tile order
    const int t0 = p.f[first_field].tile_base;
    const int t1 = first_field + num_fields < p.n ? p.f[first_field + num_fields].tile_base : (int)L.total_tiles;
    p.tile_offset = t0;
    p.tile_end = t1;
    grid = t1 - t0;
    if (grid <= 0) return GF_OK;
  }
#define GF_FWD(N, C, O)                                                                         \
  do {                                                                                          \
    if (fast32 && O == GF_BF16 && (p.cfg.flags & GF_CFG_FWD_EXP2)) {                             \
      constexpr bool X = (O == GF_BF16);                                                        \
      if (grid * fwd32_warps<X>() < kSmallGridMinWarps)                                         \
        render_fwd32_kernel<NF, N, C, O, X, kSmallGridWarps><<<grid, 32 * kSmallGridWarps, 0, st>>>(p); \
      else                                                                                      \
        render_fwd32_kernel<NF, N, C, O, X, fwd32_warps<X>()><<<grid, 32 * fwd32_warps<X>(), 0, st>>>(p); \
      render_fwd32_heavy_kernel<NF, N, C, O, X><<<heavy_grid, 32 * kHeavyWarps, 0, st>>>(p);   \
    } else if (fast32) {                                                                        \
      if (grid * kFwd32Warps < kSmallGridMinWarps)                                              \
        render_fwd32_kernel<NF, N, C, O, false, kSmallGridWarps><<<grid, 32 * kSmallGridWarps, 0, st>>>(p); \
      else                                                                                      \
        render_fwd32_kernel<NF, N, C, O, false, kFwd32Warps><<<grid, 32 * kFwd32Warps, 0, st>>>(p); \
      render_fwd32_heavy_kernel<NF, N, C, O, false><<<heavy_grid, 32 * kHeavyWarps, 0, st>>>(p); \
    } else render_fwd_kernel<NF, N, C, O><<<grid, kRenderThreads, 0, st>>>(p);                  \
  } while (0)
  const bool fast32 = cfg->tile_out == 32 && cfg->tile_in == 32;
  const int heavy_grid = grid < kHeavyGridCap ? grid : kHeavyGridCap;  // CTAs striding over the heavy tiles
  if (cfg->out_dtype == GF_F32) {
    if (norm) { if (clamp) GF_FWD(true, true, GF_F32); else GF_FWD(true, false, GF_F32); }
    else { if (clamp) GF_FWD(false, true, GF_F32); else GF_FWD(false, false, GF_F32); }
  } else {
    if (norm) { if (clamp) GF_FWD(true, true, GF_BF16); else GF_FWD(true, false, GF_BF16); }
    else { if (clamp) GF_FWD(false, true, GF_BF16); else GF_FWD(false, false, GF_BF16); }
  }
#undef GF_FWD
  GF_LAUNCH_CHECK("render_fwd_kernel");
  trace_mark(st);
  return GF_OK;
}

template <int NF, bool N, bool C, int G, bool X>
cudaError_t launch_bwd32(const Params<NF>& p, int grid, cudaStream_t st) {
  const int hgrid = grid < kHeavyGridCap ? grid : kHeavyGridCap;
  render_bwd32_kernel<NF, N, C, G, X><<<grid, 32 * kBwd32Warps, 0, st>>>(p);
  render_bwd32_heavy_kernel<NF, N, C, G, X><<<hgrid, 32 * kBwd32Warps, 0, st>>>(p);
  return cudaSuccess;
}

template <int NF, bool N, bool C, int G>
cudaError_t launch_bwd_render(const Params<NF>& p, int grid, size_t smem, cudaStream_t st) {
  if (p.cfg.tile_out == 32 && p.cfg.tile_in == 32) {
    if (p.cfg.flags & GF_CFG_BWD_EXP2) return launch_bwd32<NF, N, C, G, true>(p, grid, st);
    return launch_bwd32<NF, N, C, G, false>(p, grid, st);
  }
  const cudaError_t e = allow_dynamic_smem<render_bwd_kernel<NF, N, C, G>>(kBwdSmemCapFloats * 4);
  if (e != cudaSuccess) return e;
  render_bwd_kernel<NF, N, C, G><<<grid, kRenderThreads, smem, st>>>(p);
  return cudaSuccess;
}

template <int NF>
gf_status run_backward(const gf_config* cfg, const gf_batch* batch, const Layout& L, char* ws, cudaStream_t st) {
  thread_local Params<NF>* tp = nullptr;
  if (!tp) tp = new Params<NF>();
  Params<NF>& p = *tp;
  fill_params(p, cfg, batch, L, ws);
  {
    NvtxRange r("gfield.bwd_prep");
    trace_mark(st);
    if (cudaMemsetAsync(p.heavy_count, 0, sizeof(uint32_t), st) != cudaSuccess)
      return fail(GF_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(cudaGetLastError()));
    if (L.total_g > 0) {
      geometry_kernel<NF, true><<<(int)ceil_div(L.total_g, kGeoThreads), kGeoThreads, 0, st>>>(p);
      GF_LAUNCH_CHECK("geometry_kernel");
    }
    bwd_prep_kernel<NF><<<p.n, kBinThreads, 0, st>>>(p);
    GF_LAUNCH_CHECK("bwd_prep_kernel");
    trace_mark(st);
  }
  const bool norm = p.cfg.normalize, clamp = p.cfg.has_clamp;
  const int grid = (int)L.total_tiles;
  const size_t smem = sizeof(float) * ((size_t)cfg->tile_out * cfg->tile_in + cfg->tile_out);
  NvtxRange r("gfield.render_bwd+finalize");
  cudaError_t attr_err = cudaSuccess;
#define GF_BWD(N, C, G) attr_err = launch_bwd_render<NF, N, C, G>(p, grid, smem, st)
  if (cfg->grad_dtype == GF_F32) {
    if (norm) { if (clamp) GF_BWD(true, true, GF_F32); else GF_BWD(true, false, GF_F32); }
    else { if (clamp) GF_BWD(false, true, GF_F32); else GF_BWD(false, false, GF_F32); }
  } else {
    if (norm) { if (clamp) GF_BWD(true, true, GF_BF16); else GF_BWD(true, false, GF_BF16); }
    else { if (clamp) GF_BWD(false, true, GF_BF16); else GF_BWD(false, false, GF_BF16); }
  }
#undef GF_BWD
  if (attr_err != cudaSuccess)
    return fail(GF_ERR_CUDA, "render_bwd_kernel: cudaFuncSetAttribute: %s", cudaGetErrorString(attr_err));
  GF_LAUNCH_CHECK("render_bwd_kernel");
  trace_mark(st);
  if (L.total_g > 0) {
    const int wpb = kRenderThreads / 32;
    const int fgrid = (int)ceil_div(L.total_g, wpb);
    if (norm) bwd_finalize_kernel<NF, true><<<fgrid, kRenderThreads, 0, st>>>(p);
    else bwd_finalize_kernel<NF, false><<<fgrid, kRenderThreads, 0, st>>>(p);
    GF_LAUNCH_CHECK("bwd_finalize_kernel");
  }
  trace_mark(st);
  return GF_OK;
}

}  // namespace gf

// ---------------------------------------------------------------------------
// C ABI

extern "C" {

int gf_abi_version(void) { return GF_ABI_VERSION; }

const char* gf_last_error(void) { return gf::g_last_error.c_str(); }

int64_t gf_num_tiles(int64_t out_features, int64_t in_features, int64_t tile_out, int64_t tile_in) {
  if (out_features <= 0 || in_features <= 0 || tile_out <= 0 || tile_in <= 0) return 0;
  return gf::ceil_div(out_features, tile_out) * gf::ceil_div(in_features, tile_in);
}

size_t gf_workspace_bytes(const gf_config* cfg, const gf_batch* batch, gf_pass pass) {
  if (gf::validate(cfg, batch, pass, /*data=*/false) != GF_OK) return 0;
  return gf::layout(cfg, batch, pass).total;
}

static gf_status gf_dispatch(const gf_config* cfg, const gf_batch* batch, void* workspace, size_t workspace_bytes,
                             gf_stream stream, gf_pass pass, unsigned stages = GF_STAGE_BIN | GF_STAGE_RENDER,
                             int first_field = 0, int num_fields = -1) {
  gf_status s = gf::validate(cfg, batch, pass);
  if (s != GF_OK) return s;
  const gf::Layout L = gf::layout(cfg, batch, pass);
  if (!workspace) return gf::fail(GF_ERR_INVALID_ARG, "workspace must be non-null");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return gf::fail(GF_ERR_INVALID_ARG, "workspace must be 256-byte aligned");
  if (workspace_bytes < L.total)
    return gf::fail(GF_ERR_INVALID_ARG, "workspace too small: %zu bytes given, %zu needed", workspace_bytes, L.total);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  const int n = batch->num_fields;
  gf::NvtxRange r(pass == GF_PASS_FORWARD ? "gfield.forward" : "gfield.backward");
  if (pass == GF_PASS_FORWARD) {
    if (n == 1) return gf::run_forward<1>(cfg, batch, L, ws, st, stages, first_field, num_fields);
    if (n <= 16) return gf::run_forward<16>(cfg, batch, L, ws, st, stages, first_field, num_fields);
    return gf::run_forward<GF_MAX_FIELDS>(cfg, batch, L, ws, st, stages, first_field, num_fields);
  }
  if (n == 1) return gf::run_backward<1>(cfg, batch, L, ws, st);
  if (n <= 16) return gf::run_backward<16>(cfg, batch, L, ws, st);
  return gf::run_backward<GF_MAX_FIELDS>(cfg, batch, L, ws, st);
}

gf_status gf_forward(const gf_config* cfg, const gf_batch* batch, void* workspace, size_t workspace_bytes,
                     gf_stream stream) {
  return gf_dispatch(cfg, batch, workspace, workspace_bytes, stream, GF_PASS_FORWARD);
}

gf_status gf_forward_stages(const gf_config* cfg, const gf_batch* batch, void* workspace, size_t workspace_bytes,
                            unsigned stages, gf_stream stream) {
  if (stages == 0 || (stages & ~(GF_STAGE_BIN | GF_STAGE_RENDER)))
    return gf::fail(GF_ERR_INVALID_ARG, "stages must be GF_STAGE_BIN, GF_STAGE_RENDER or both");
  return gf_dispatch(cfg, batch, workspace, workspace_bytes, stream, GF_PASS_FORWARD, stages);
}

gf_status gf_forward_render_fields(const gf_config* cfg, const gf_batch* batch, void* workspace,
                                   size_t workspace_bytes, int32_t first_field, int32_t num_fields, gf_stream stream) {
  if (!batch) return gf::fail(GF_ERR_INVALID_ARG, "cfg and batch must be non-null");
  if (first_field < 0 || num_fields < 1 || first_field > batch->num_fields - num_fields)
    return gf::fail(GF_ERR_INVALID_ARG, "field range [%d, %d) outside the batch's %d fields", first_field,
                    first_field + num_fields, batch->num_fields);
  return gf_dispatch(cfg, batch, workspace, workspace_bytes, stream, GF_PASS_FORWARD, GF_STAGE_RENDER, first_field,
                     num_fields);
}

gf_status gf_backward(const gf_config* cfg, const gf_batch* batch, void* workspace, size_t workspace_bytes,
                      gf_stream stream) {
  return gf_dispatch(cfg, batch, workspace, workspace_bytes, stream, GF_PASS_BACKWARD);
}

gf_status gf_workspace_status(void* workspace, gf_stream stream, int reset, uint32_t* flags_out) {
  if (!workspace || !flags_out) return gf::fail(GF_ERR_INVALID_ARG, "workspace and flags_out must be non-null");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint32_t flags = 0;
  cudaError_t e = cudaMemcpyAsync(&flags, workspace, sizeof(flags), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && reset) {
    e = cudaMemsetAsync(workspace, 0, sizeof(uint32_t), st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  }
  if (e != cudaSuccess) return gf::fail(GF_ERR_CUDA, "gf_workspace_status: %s", cudaGetErrorString(e));
  *flags_out = flags;
  return GF_OK;
}

gf_status gf_trace_events(void* const* events, int n) {
  if (n < 0 || (n > 0 && !events)) return gf::fail(GF_ERR_INVALID_ARG, "gf_trace_events: bad event array");
  std::lock_guard<std::mutex> lock(gf::g_trace_mu);
  gf::g_trace.ev = events;
  gf::g_trace.n = n;
  gf::g_trace.used = 0;
  return GF_OK;
}

int gf_trace_count(void) {
  std::lock_guard<std::mutex> lock(gf::g_trace_mu);
  return gf::g_trace.used;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Multicast publish: each thread streams 16-byte chunks from local memory to
// the NVLS multicast address (multimem.st); the switch replicates every store
// to all GPUs bound to the multicast object.

__global__ void multicast_store_kernel(const uint4* __restrict__ src, unsigned long long mc_dst, size_t n16) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n16; i += stride) {
    const uint4 v = src[i];
    const unsigned long long a = mc_dst + 16ull * i;
    asm volatile("multimem.st.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(a), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
  }
  __threadfence_system();
}

extern "C" gf_status gf_multicast_store(const void* src, void* mc_dst, size_t bytes, int max_blocks,
                                        gf_stream stream) {
  if (bytes == 0) return GF_OK;
  if (!src || !mc_dst) return gf::fail(GF_ERR_INVALID_ARG, "gf_multicast_store: src and mc_dst must be non-null");
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(mc_dst) | bytes) & 15u)
    return gf::fail(GF_ERR_INVALID_ARG, "gf_multicast_store: src, mc_dst and bytes must be multiples of 16");
  if (max_blocks <= 0) return gf::fail(GF_ERR_INVALID_ARG, "gf_multicast_store: max_blocks must be positive");
  gf::NvtxRange r("gfield.multicast_store");
  const size_t n16 = bytes / 16;
  const int threads = 512;
  const size_t need = (n16 + threads - 1) / threads;
  const int blocks = (int)(need < (size_t)max_blocks ? need : (size_t)max_blocks);
  multicast_store_kernel<<<blocks, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), reinterpret_cast<unsigned long long>(mc_dst), n16);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return gf::fail(GF_ERR_CUDA, "gf_multicast_store: %s", cudaGetErrorString(e));
  return GF_OK;
}

// ---------------------------------------------------------------------------
// Densify statistics (gf_grad_stats_accumulate): one thread per Gaussian, one
// grid row per layer.  Each plane update is the reference's fp32 add_ of a
// per-Gaussian score (controllers/stats.py:58-66).

namespace gf {
struct StatsParams {
  int32_t n;
  int32_t pad_;
  gf_stats_layer l[GF_MAX_FIELDS];
};
static_assert(sizeof(StatsParams) <= 32764, "stats descriptor block exceeds the kernel-parameter limit");

__global__ void __launch_bounds__(256) grad_stats_kernel(const __grid_constant__ StatsParams p) {
  const gf_stats_layer& L = p.l[blockIdx.y];
  const int64_t K = L.num_gaussians;
  float* s = L.stats;
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < K; k += (int64_t)gridDim.x * blockDim.x) {
    if (L.d_mu_raw) {
      const float a = L.d_mu_raw[2 * k], b = L.d_mu_raw[2 * k + 1];
      s[k] = __fadd_rn(s[k], __fsqrt_rn(__fmaf_rn(b, b, __fmul_rn(a, a))));
    }
    if (L.d_chol_raw) {
      const float a = L.d_chol_raw[3 * k], b = L.d_chol_raw[3 * k + 1], c = L.d_chol_raw[3 * k + 2];
      s[K + k] = __fadd_rn(s[K + k], __fsqrt_rn(__fmaf_rn(c, c, __fmaf_rn(b, b, __fmul_rn(a, a)))));
    }
    if (L.d_amp) s[2 * K + k] = __fadd_rn(s[2 * K + k], fabsf(L.d_amp[k]));
    if (L.amp) s[3 * K + k] = __fadd_rn(s[3 * K + k], fabsf(L.amp[k]));
    s[4 * K + k] = __fadd_rn(s[4 * K + k], 1.0f);
  }
}
}  // namespace gf

extern "C" gf_status gf_grad_stats_accumulate(int32_t num_layers, const gf_stats_layer* layers, gf_stream stream) {
  if (num_layers == 0) return GF_OK;
  if (num_layers < 0 || num_layers > GF_MAX_FIELDS || !layers)
    return gf::fail(GF_ERR_INVALID_ARG, "gf_grad_stats_accumulate: num_layers must be in 0..%d with a layer array",
                    GF_MAX_FIELDS);
  gf::NvtxRange r("gfield.grad_stats");
  thread_local gf::StatsParams* tp = nullptr;
  if (!tp) tp = new gf::StatsParams();
  gf::StatsParams& p = *tp;
  p.n = num_layers;
  int64_t kmax = 0;
  for (int i = 0; i < num_layers; ++i) {
    const gf_stats_layer& L = layers[i];
    if (L.num_gaussians < 0) return gf::fail(GF_ERR_INVALID_ARG, "gf_grad_stats_accumulate: layer %d: K < 0", i);
    if (L.num_gaussians > 0 && !L.stats)
      return gf::fail(GF_ERR_INVALID_ARG, "gf_grad_stats_accumulate: layer %d: stats must be non-null", i);
    p.l[i] = L;
    if (L.num_gaussians > kmax) kmax = L.num_gaussians;
  }
  if (kmax == 0) return GF_OK;
  const int threads = 256;
  const int64_t bx = (kmax + threads - 1) / threads;
  const dim3 grid((unsigned)(bx < 64 ? bx : 64), (unsigned)num_layers);
  gf::grad_stats_kernel<<<grid, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return gf::fail(GF_ERR_CUDA, "gf_grad_stats_accumulate: %s", cudaGetErrorString(e));
  return GF_OK;
}

// ---------------------------------------------------------------------------
// Forward render without caller scratch (gf_forward_noalloc).
//
// For callers that are handed their input and output buffers by a host that
// owns all device memory (an inference-engine plugin, a framework custom call,
// a runtime with a fixed memory budget) and that may not call cudaMalloc or
// ask for a workspace.  The forward's scratch then lives in this file-scope
// array, which every GPU that loads the library holds until the process
// exits.  All calls share it: two calls whose work overlaps on the GPU (other
// streams, other host threads) race on it and must be ordered by the caller.

static __device__ __align__(256) unsigned char g_noalloc_scratch[GF_NOALLOC_SCRATCH_BYTES];

namespace gf {

constexpr int kNoallocMaxDevices = 64;
void* g_noalloc_ptr[kNoallocMaxDevices];  // device address of the array, per device
std::mutex g_noalloc_mutex;               // guards the pointers and the static descriptors
Params<1> g_noalloc_p1;                    // launch descriptors in static storage:
Params<16> g_noalloc_p16;                  // no heap allocation on this path
Params<GF_MAX_FIELDS> g_noalloc_pmax;

template <int NF>
gf_status noalloc_launch(Params<NF>& p, const gf_config* cfg, const gf_batch* batch, const Layout& L, char* ws,
                         cudaStream_t st) {
  fill_params(p, cfg, batch, L, ws);
  int max_nd = 0;
  for (int i = 0; i < p.n; ++i) {
    const int nd = (p.f[i].ntr + 1) * (p.f[i].ntc + 1);
    if (nd <= kBinSmemCapInts && nd > max_nd) max_nd = nd;
  }
  cudaError_t e = cudaFuncSetAttribute(bin_kernel<NF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kBinSmemCapInts * 4);
  if (e != cudaSuccess) return fail(GF_ERR_CUDA, "gf_forward_noalloc: %s", cudaGetErrorString(e));
  if (L.total_g > 0) {
    geometry_kernel<NF, false><<<(int)ceil_div(L.total_g, kGeoThreads), kGeoThreads, 0, st>>>(p);
    GF_LAUNCH_CHECK("geometry_kernel");
  }
  bin_kernel<NF><<<p.n, kBinThreads, sizeof(int) * (size_t)max_nd, st>>>(p, kBinSmemCapInts);
  GF_LAUNCH_CHECK("bin_kernel");
  const gf_status sl = launch_tile_lists(p, L, st);
  if (sl != GF_OK) return sl;
  const bool norm = p.cfg.normalize, clamp = p.cfg.has_clamp;
  const int grid = (int)L.total_tiles;
#define GF_FWD(N, C, O)                                                                         \
  do {                                                                                          \
    if (fast32 && O == GF_BF16 && (p.cfg.flags & GF_CFG_FWD_EXP2)) {                             \
      constexpr bool X = (O == GF_BF16);                                                        \
      if (grid * fwd32_warps<X>() < kSmallGridMinWarps)                                         \
        render_fwd32_kernel<NF, N, C, O, X, kSmallGridWarps><<<grid, 32 * kSmallGridWarps, 0, st>>>(p); \
      else                                                                                      \
        render_fwd32_kernel<NF, N, C, O, X, fwd32_warps<X>()><<<grid, 32 * fwd32_warps<X>(), 0, st>>>(p); \
      render_fwd32_heavy_kernel<NF, N, C, O, X><<<heavy_grid, 32 * kHeavyWarps, 0, st>>>(p);   \
    } else if (fast32) {                                                                        \
      if (grid * kFwd32Warps < kSmallGridMinWarps)                                              \
        render_fwd32_kernel<NF, N, C, O, false, kSmallGridWarps><<<grid, 32 * kSmallGridWarps, 0, st>>>(p); \
      else                                                                                      \
        render_fwd32_kernel<NF, N, C, O, false, kFwd32Warps><<<grid, 32 * kFwd32Warps, 0, st>>>(p); \
      render_fwd32_heavy_kernel<NF, N, C, O, false><<<heavy_grid, 32 * kHeavyWarps, 0, st>>>(p); \
    } else render_fwd_kernel<NF, N, C, O><<<grid, kRenderThreads, 0, st>>>(p);                  \
  } while (0)
  const bool fast32 = cfg->tile_out == 32 && cfg->tile_in == 32;
  const int heavy_grid = grid < kHeavyGridCap ? grid : kHeavyGridCap;  // CTAs striding over the heavy tiles
  if (cfg->out_dtype == GF_F32) {
    if (norm) { if (clamp) GF_FWD(true, true, GF_F32); else GF_FWD(true, false, GF_F32); }
    else { if (clamp) GF_FWD(false, true, GF_F32); else GF_FWD(false, false, GF_F32); }
  } else {
    if (norm) { if (clamp) GF_FWD(true, true, GF_BF16); else GF_FWD(true, false, GF_BF16); }
    else { if (clamp) GF_FWD(false, true, GF_BF16); else GF_FWD(false, false, GF_BF16); }
  }
#undef GF_FWD
  GF_LAUNCH_CHECK("render_fwd_kernel");
  return GF_OK;
}

}  // namespace gf

extern "C" gf_status gf_forward_noalloc(const gf_config* cfg, const gf_batch* batch, gf_stream stream) {
  gf_status s = gf::validate(cfg, batch, GF_PASS_FORWARD);
  if (s != GF_OK) return s;
  const gf::Layout L = gf::layout(cfg, batch, GF_PASS_FORWARD);
  if (L.total > (size_t)GF_NOALLOC_SCRATCH_BYTES)
    return gf::fail(GF_ERR_UNSUPPORTED,
                    "gf_forward_noalloc: this batch needs %zu bytes of scratch but the static scratch holds %zu; "
                    "use gf_forward with a caller workspace",
                    L.total, (size_t)GF_NOALLOC_SCRATCH_BYTES);
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return gf::fail(GF_ERR_CUDA, "gf_forward_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= gf::kNoallocMaxDevices)
    return gf::fail(GF_ERR_UNSUPPORTED, "gf_forward_noalloc: device %d beyond the supported %d", dev,
                    gf::kNoallocMaxDevices);
  std::lock_guard<std::mutex> lock(gf::g_noalloc_mutex);
  if (gf::g_noalloc_ptr[dev] == nullptr) {
    // One-time set-up on this device (the device is current): the array's
    // name is only a host-side stand-in, so fetch its device address.
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return gf::fail(GF_ERR_CUDA, "gf_forward_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    gf::g_noalloc_ptr[dev] = ptr;
  }
  char* ws = static_cast<char*>(gf::g_noalloc_ptr[dev]);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // The array keeps the previous call's contents; the status word and the
  // completion counter in its header must start at zero.
  e = cudaMemsetAsync(ws + L.hdr, 0, 256, st);
  if (e != cudaSuccess) return gf::fail(GF_ERR_CUDA, "gf_forward_noalloc: cudaMemsetAsync: %s", cudaGetErrorString(e));
  const int n = batch->num_fields;
  if (n == 1) return gf::noalloc_launch(gf::g_noalloc_p1, cfg, batch, L, ws, st);
  if (n <= 16) return gf::noalloc_launch(gf::g_noalloc_p16, cfg, batch, L, ws, st);
  return gf::noalloc_launch(gf::g_noalloc_pmax, cfg, batch, L, ws, st);
}
