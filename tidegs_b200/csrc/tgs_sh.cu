// Spherical-harmonics colors of the render path (gsplat 1.0.0
// spherical_harmonics, called by strategies/tide_engine/engine.py:508-520):
// colors[n, c] = sum_k coeffs[n, k, c] Y_k(dirs[n] / |dirs[n]|) over the
// first (degree + 1)^2 real SH basis functions, and its vector-Jacobian
// product with respect to coeffs and dirs
// (submodules/gsplat/gsplat/cuda/csrc/compute_sh_fwd.cu, compute_sh_bwd.cu,
// spherical_harmonics.cuh).
//
// Basis: the orthonormal real SH of degree <= 4 in the order and sign
// convention of 3D Gaussian splatting (Kerbl et al. 2023) that gsplat
// evaluates (l-major, m = -l..l, Y_1 = -C1 y, C1 z, -C1 x, ...), written
// here as polynomials in the unit direction (x, y, z); constants are the
// standard normalizations, e.g. C0 = 1 / (2 sqrt(pi)), C1 = sqrt(3 / (4 pi)).
// The backward differentiates those polynomials and projects the gradient
// onto the sphere's tangent plane, (g - (g . n) n) / |d|: any polynomial
// equal to Y_k on the sphere gives the same result.
//
// One thread per Gaussian; a block stages its Gaussians' coefficient rows
// (K x 3 floats each, contiguous in memory) through shared memory with
// coalesced loads and stores, padded to an odd row stride so the per-thread
// reads hit distinct banks.
#include "tidegs_b200.h"
#include "tgs_common.cuh"

namespace tgs {
namespace {

constexpr int kShThreads = 128;
constexpr int kShMaxK = 25;  // degree 4

// Calls f(k, Y_k, dY_k/dx, dY_k/dy, dY_k/dz) for k < (degree + 1)^2 at the
// unit direction (x, y, z). The derivatives are those of the polynomial
// forms below (not of the unit-sphere restriction); callers that need the
// direction gradient project them onto the tangent plane.
template <class F>
__device__ __forceinline__ void sh_terms(int degree, float x, float y, float z, F&& f) {
  f(0, 0.28209479177387814f, 0.f, 0.f, 0.f);
  if (degree < 1) return;
  constexpr float C1 = 0.4886025119029199f;
  f(1, -C1 * y, 0.f, -C1, 0.f);
  f(2, C1 * z, 0.f, 0.f, C1);
  f(3, -C1 * x, -C1, 0.f, 0.f);
  if (degree < 2) return;
  constexpr float C2a = 1.0925484305920792f, C2c = 0.31539156525252005f,
                  C2e = 0.5462742152960396f;
  const float xx = x * x, yy = y * y, zz = z * z;
  f(4, C2a * x * y, C2a * y, C2a * x, 0.f);
  f(5, -C2a * y * z, 0.f, -C2a * z, -C2a * y);
  f(6, C2c * (3.f * zz - 1.f), 0.f, 0.f, 6.f * C2c * z);
  f(7, -C2a * x * z, -C2a * z, 0.f, -C2a * x);
  f(8, C2e * (xx - yy), 2.f * C2e * x, -2.f * C2e * y, 0.f);
  if (degree < 3) return;
  constexpr float C3a = -0.5900435899266435f, C3b = 2.890611442640554f,
                  C3c = -0.4570457994644658f, C3d = 0.3731763325901154f,
                  C3f = 1.445305721320277f;
  const float z5 = 5.f * zz - 1.f;
  f(9, C3a * y * (3.f * xx - yy), 6.f * C3a * x * y, 3.f * C3a * (xx - yy), 0.f);
  f(10, C3b * x * y * z, C3b * y * z, C3b * x * z, C3b * x * y);
  f(11, C3c * y * z5, 0.f, C3c * z5, 10.f * C3c * y * z);
  f(12, C3d * z * (5.f * zz - 3.f), 0.f, 0.f, C3d * (15.f * zz - 3.f));
  f(13, C3c * x * z5, C3c * z5, 0.f, 10.f * C3c * x * z);
  f(14, C3f * z * (xx - yy), 2.f * C3f * x * z, -2.f * C3f * y * z, C3f * (xx - yy));
  f(15, C3a * x * (xx - 3.f * yy), 3.f * C3a * (xx - yy), -6.f * C3a * x * y, 0.f);
  if (degree < 4) return;
  constexpr float C4a = 2.5033429417967046f, C4b = -1.7701307697799304f,
                  C4c = 0.9461746957575601f, C4d = -0.6690465435572892f,
                  C4e = 0.10578554691520431f, C4g = 0.47308734787878004f,
                  C4i = 0.6258357354491761f;
  const float z7a = 7.f * zz - 1.f, z7b = 7.f * zz - 3.f;
  f(16, C4a * x * y * (xx - yy), C4a * y * (3.f * xx - yy), C4a * x * (xx - 3.f * yy), 0.f);
  f(17, C4b * y * z * (3.f * xx - yy), 6.f * C4b * x * y * z, 3.f * C4b * z * (xx - yy),
    C4b * y * (3.f * xx - yy));
  f(18, C4c * x * y * z7a, C4c * y * z7a, C4c * x * z7a, 14.f * C4c * x * y * z);
  f(19, C4d * y * z * z7b, 0.f, C4d * z * z7b, C4d * y * (21.f * zz - 3.f));
  f(20, C4e * (zz * (35.f * zz - 30.f) + 3.f), 0.f, 0.f, C4e * z * (140.f * zz - 60.f));
  f(21, C4d * x * z * z7b, C4d * z * z7b, 0.f, C4d * x * (21.f * zz - 3.f));
  f(22, C4g * (xx - yy) * z7a, 2.f * C4g * x * z7a, -2.f * C4g * y * z7a,
    14.f * C4g * z * (xx - yy));
  f(23, C4b * x * z * (xx - 3.f * yy), 3.f * C4b * z * (xx - yy), -6.f * C4b * x * y * z,
    C4b * x * (xx - 3.f * yy));
  f(24, C4i * (xx * (xx - 3.f * yy) - yy * (3.f * xx - yy)), 4.f * C4i * x * (xx - 3.f * yy),
    4.f * C4i * y * (yy - 3.f * xx), 0.f);
}

// Row of flat element e of a block's [rows, row_floats] chunk: e is at most
// 128 * 75 and row_floats at most 75, so (e + 0.5) / row_floats stays at
// least 0.5 / 75 away from an integer and the float product truncates to
// the exact quotient.
__device__ __forceinline__ int row_of(int e, float inv_row) {
  return __float2int_rz((static_cast<float>(e) + 0.5f) * inv_row);
}

// Copies the block's coefficient rows [n0, n0 + rows) x (3K) floats from
// global memory into shared memory rows of stride 3K + 1: coalesced loads,
// kStageUnroll of them in flight per thread before the stores.
constexpr int kStageUnroll = 8;
__device__ __forceinline__ void stage_rows(const float* __restrict__ src, float* dst, int rows,
                                           int row_floats, float inv_row) {
  const int total = rows * row_floats;
  for (int base = threadIdx.x; base < total; base += kShThreads * kStageUnroll) {
    float v[kStageUnroll];
#pragma unroll
    for (int u = 0; u < kStageUnroll; ++u) {
      const int e = base + u * kShThreads;
      v[u] = e < total ? src[e] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kStageUnroll; ++u) {
      const int e = base + u * kShThreads;
      if (e < total) dst[e + row_of(e, inv_row)] = v[u];
    }
  }
}

__global__ void __launch_bounds__(kShThreads) sh_fwd_kernel(const TgsShArgs a) {
  extern __shared__ float sh_smem[];
  const int row_floats = 3 * a.K;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kShThreads;
  const int rows = static_cast<int>(a.n - n0 < kShThreads ? a.n - n0 : kShThreads);
  stage_rows(a.coeffs + n0 * row_floats, sh_smem, rows, row_floats, 1.f / row_floats);
  __syncthreads();
  const int t = threadIdx.x;
  if (t >= rows) return;
  const int64_t n = n0 + t;
  float col[3] = {0.f, 0.f, 0.f};
  if (a.masks == nullptr || a.masks[n]) {
    const float* row = sh_smem + t * (row_floats + 1);
    const float dx = a.dirs[3 * n], dy = a.dirs[3 * n + 1], dz = a.dirs[3 * n + 2];
    float x = 0.f, y = 0.f, z = 0.f;
    if (a.degree >= 1) {
      const float inv = rsqrtf(dx * dx + dy * dy + dz * dz);
      x = dx * inv, y = dy * inv, z = dz * inv;
    }
    sh_terms(a.degree, x, y, z, [&](int k, float Y, float, float, float) {
#pragma unroll
      for (int c = 0; c < 3; ++c) col[c] += Y * row[3 * k + c];
    });
  }
#pragma unroll
  for (int c = 0; c < 3; ++c) a.colors[3 * n + c] = col[c];
}

__global__ void __launch_bounds__(kShThreads) sh_bwd_kernel(const TgsShBwdArgs b) {
  const TgsShArgs& a = b.fwd;
  extern __shared__ float sh_smem[];
  const int row_floats = 3 * a.K;
  const int stride = row_floats + 1;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kShThreads;
  const int rows = static_cast<int>(a.n - n0 < kShThreads ? a.n - n0 : kShThreads);
  const bool want_dirs = b.v_dirs != nullptr;
  const float inv_row = 1.f / row_floats;
  if (want_dirs) stage_rows(a.coeffs + n0 * row_floats, sh_smem, rows, row_floats, inv_row);
  __syncthreads();
  const int t = threadIdx.x;
  if (t < rows) {
    const int64_t n = n0 + t;
    float* row = sh_smem + t * stride;
    const bool on = a.masks == nullptr || a.masks[n];
    const float vc[3] = {b.v_colors[3 * n], b.v_colors[3 * n + 1], b.v_colors[3 * n + 2]};
    const float dx = a.dirs[3 * n], dy = a.dirs[3 * n + 1], dz = a.dirs[3 * n + 2];
    float x = 0.f, y = 0.f, z = 0.f, inv = 0.f;
    if (a.degree >= 1) {
      inv = rsqrtf(dx * dx + dy * dy + dz * dz);
      x = dx * inv, y = dy * inv, z = dz * inv;
    }
    float g[3] = {0.f, 0.f, 0.f};
    const int used = on ? (a.degree + 1) * (a.degree + 1) : 0;
    if (on) {
      sh_terms(a.degree, x, y, z, [&](int k, float Y, float gx, float gy, float gz) {
        if (want_dirs) {
          const float w = vc[0] * row[3 * k] + vc[1] * row[3 * k + 1] + vc[2] * row[3 * k + 2];
          g[0] += w * gx;
          g[1] += w * gy;
          g[2] += w * gz;
        }
#pragma unroll
        for (int c = 0; c < 3; ++c) row[3 * k + c] = vc[c] * Y;  // v_coeffs, in place
      });
    }
    for (int e = 3 * used; e < row_floats; ++e) row[e] = 0.f;
    if (want_dirs) {
      float vd[3] = {0.f, 0.f, 0.f};
      if (on && a.degree >= 1) {
        const float dot = g[0] * x + g[1] * y + g[2] * z;
        vd[0] = (g[0] - dot * x) * inv;
        vd[1] = (g[1] - dot * y) * inv;
        vd[2] = (g[2] - dot * z) * inv;
      }
#pragma unroll
      for (int c = 0; c < 3; ++c) b.v_dirs[3 * n + c] = vd[c];
    }
  }
  __syncthreads();
  // coalesced store of the block's v_coeffs rows
  const int total = rows * row_floats;
  float* dst = b.v_coeffs + n0 * row_floats;
  for (int e = threadIdx.x; e < total; e += kShThreads) dst[e] = sh_smem[e + row_of(e, inv_row)];
}

int check_sh(const TgsShArgs* a, const char* who) {
  TGS_CHECK_ARG(a != nullptr, "%s: args is NULL", who);
  TGS_CHECK_ARG(a->n >= 0 && a->K >= 1 && a->K <= kShMaxK, "%s: bad sizes (n %lld, K %d)", who,
                static_cast<long long>(a->n), a->K);
  TGS_CHECK_ARG(a->degree >= 0 && a->degree <= 4 && (a->degree + 1) * (a->degree + 1) <= a->K,
                "%s: degree %d needs (degree + 1)^2 <= K = %d coefficients", who, a->degree, a->K);
  TGS_CHECK_ARG(a->n == 0 || (a->dirs && a->coeffs), "%s: NULL pointer", who);
  return TGS_OK;
}

size_t sh_smem_bytes(int K) { return static_cast<size_t>(kShThreads) * (3 * K + 1) * sizeof(float); }

}  // namespace
}  // namespace tgs

using namespace tgs;

extern "C" int tgs_sh_fwd(const TgsShArgs* a, void* stream) {
  if (int rc = check_sh(a, "tgs_sh_fwd")) return rc;
  if (a->n == 0) return TGS_OK;
  TGS_CHECK_ARG(a->colors != nullptr, "tgs_sh_fwd: NULL pointer");
  const size_t smem = sh_smem_bytes(a->K);
  TGS_CUDA(cudaFuncSetAttribute(sh_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem)));
  sh_fwd_kernel<<<static_cast<unsigned>(ceil_div<int64_t>(a->n, kShThreads)), kShThreads, smem,
                  as_stream(stream)>>>(*a);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int tgs_sh_bwd(const TgsShBwdArgs* b, void* stream) {
  TGS_CHECK_ARG(b != nullptr, "tgs_sh_bwd: args is NULL");
  if (int rc = check_sh(&b->fwd, "tgs_sh_bwd")) return rc;
  if (b->fwd.n == 0) return TGS_OK;
  TGS_CHECK_ARG(b->v_colors && b->v_coeffs, "tgs_sh_bwd: NULL pointer");
  const size_t smem = sh_smem_bytes(b->fwd.K);
  TGS_CUDA(cudaFuncSetAttribute(sh_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem)));
  sh_bwd_kernel<<<static_cast<unsigned>(ceil_div<int64_t>(b->fwd.n, kShThreads)), kShThreads,
                  smem, as_stream(stream)>>>(*b);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}
