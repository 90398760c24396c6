// Render path of the step before the optimizer: Gaussian projection, tile
// intersection and alpha-composited rasterization, forward and backward
// (the engine's gsplat 1.0.0 calls, strategies/tide_engine/engine.py:481-561;
// gsplat/cuda/csrc fully_fused_projection_{fwd,bwd}.cu, isect_tiles.cu,
// rasterize_to_pixels_{fwd,bwd}.cu, utils.cuh).
//
// Algorithms (3D Gaussian splatting, Kerbl et al. 2023; the gradients as
// derived in the gsplat report, Ye et al. 2024):
// * projection: world -> camera (p_c = R p + t), covariance R_q S S R_q^T
//   rotated into the camera, EWA perspective Jacobian (with the 1.3 x FOV
//   clamp of the tangent), 2D covariance + eps2d blur, conic = inverse, radius
//   = ceil(3 sqrt(largest eigenvalue)), culled outside [near, far], at
//   det <= 0, at radius <= radius_clip or off the image;
// * tile intersection: one key per (camera, tile, Gaussian) =
//   camera | tile | depth bits, sorted (stable) so that each tile lists its
//   Gaussians front to back; offsets = first key of every (camera, tile);
// * rasterization: per 16 x 16 tile, batches of Gaussians staged in shared
//   memory, alpha = min(0.999, o exp(-sigma)), skipped below 1/255, a pixel
//   stops when its transmittance would fall to 1e-4 or below;
// * backward: the same traversal back to front, transmittance recovered by
//   division; per Gaussian the warp's partial gradients are summed with
//   shuffles and lane 0 adds them to global memory (atomics; combining the
//   tile's warps in shared memory first measured slower).
#include <math.h>

#include "tgs_common.cuh"

#include <algorithm>

#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>
#include <thrust/iterator/counting_iterator.h>
#include <thrust/iterator/transform_iterator.h>

namespace tgs {
// Tiles of the j-th Gaussian in depth order, as a 64-bit value for the scan
// (a named namespace: it is a template argument of the library's kernels).
struct OrderedTileCount {
  const int32_t* tiles;
  const int32_t* order;
  __host__ __device__ int64_t operator()(int64_t j) const {
    return static_cast<int64_t>(tiles[order[j]]);
  }
};

namespace {

constexpr int kProjThreads = 256;

// 3x3 matrices are row-major float[9] here.
__device__ __forceinline__ void mat3_mul(const float* a, const float* b, float* c) {
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j)
      c[i * 3 + j] = a[i * 3] * b[j] + a[i * 3 + 1] * b[3 + j] + a[i * 3 + 2] * b[6 + j];
}
// c = a * b^T
__device__ __forceinline__ void mat3_mul_bt(const float* a, const float* b, float* c) {
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j)
      c[i * 3 + j] = a[i * 3] * b[j * 3] + a[i * 3 + 1] * b[j * 3 + 1] + a[i * 3 + 2] * b[j * 3 + 2];
}
// c = a^T * b
__device__ __forceinline__ void mat3_mul_at(const float* a, const float* b, float* c) {
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j)
      c[i * 3 + j] = a[i] * b[j] + a[3 + i] * b[3 + j] + a[6 + i] * b[6 + j];
}

// Rotation of the normalized quaternion q = (w, x, y, z).
__device__ __forceinline__ void quat_rotation(const float* q, float* R, float* qn) {
  const float inv = rsqrtf(q[1] * q[1] + q[2] * q[2] + q[3] * q[3] + q[0] * q[0]);
  const float w = q[0] * inv, x = q[1] * inv, y = q[2] * inv, z = q[3] * inv;
  qn[0] = w, qn[1] = x, qn[2] = y, qn[3] = z;
  R[0] = 1.f - 2.f * (y * y + z * z); R[1] = 2.f * (x * y - w * z);       R[2] = 2.f * (x * z + w * y);
  R[3] = 2.f * (x * y + w * z);       R[4] = 1.f - 2.f * (x * x + z * z); R[5] = 2.f * (y * z - w * x);
  R[6] = 2.f * (x * z - w * y);       R[7] = 2.f * (y * z + w * x);       R[8] = 1.f - 2.f * (x * x + y * y);
}

struct ProjectGeom {
  float Rv[9], t[3];  // world -> camera
  float Rq[9], qn[4];
  float M[9];         // Rq * diag(scale)
  float cov_c[9];     // camera-space covariance
  float pc[3];        // camera-space mean
};

__device__ __forceinline__ void project_geometry(const TgsProjectArgs& a, int64_t cam, int64_t g,
                                                 ProjectGeom& G) {
  const float* V = a.viewmats + cam * 16;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    G.Rv[i * 3] = V[i * 4];
    G.Rv[i * 3 + 1] = V[i * 4 + 1];
    G.Rv[i * 3 + 2] = V[i * 4 + 2];
    G.t[i] = V[i * 4 + 3];
  }
  const float* p = a.means + g * 3;
#pragma unroll
  for (int i = 0; i < 3; ++i)
    G.pc[i] = G.Rv[i * 3] * p[0] + G.Rv[i * 3 + 1] * p[1] + G.Rv[i * 3 + 2] * p[2] + G.t[i];
  quat_rotation(a.quats + g * 4, G.Rq, G.qn);
  const float* s = a.scales + g * 3;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    G.M[i * 3] = G.Rq[i * 3] * s[0];
    G.M[i * 3 + 1] = G.Rq[i * 3 + 1] * s[1];
    G.M[i * 3 + 2] = G.Rq[i * 3 + 2] * s[2];
  }
  float cov[9], tmp[9];
  mat3_mul_bt(G.M, G.M, cov);       // Rq S S Rq^T
  mat3_mul(G.Rv, cov, tmp);         // Rv cov
  mat3_mul_bt(tmp, G.Rv, G.cov_c);  // Rv cov Rv^T
}

// EWA Jacobian rows J0 = (fx/z, 0, -fx tx/z^2), J1 = (0, fy/z, -fy ty/z^2).
struct Persp {
  float fx, fy, cx, cy, rz, rz2, tx, ty, lim_x, lim_y;
};

__device__ __forceinline__ Persp persp_setup(const TgsProjectArgs& a, int64_t cam, const float* pc) {
  const float* K = a.Ks + cam * 9;
  Persp P;
  P.fx = K[0], P.fy = K[4], P.cx = K[2], P.cy = K[5];
  const float tan_x = 0.5f * a.image_width / P.fx, tan_y = 0.5f * a.image_height / P.fy;
  P.lim_x = 1.3f * tan_x, P.lim_y = 1.3f * tan_y;
  P.rz = 1.f / pc[2];
  P.rz2 = P.rz * P.rz;
  P.tx = pc[2] * fminf(P.lim_x, fmaxf(-P.lim_x, pc[0] * P.rz));
  P.ty = pc[2] * fminf(P.lim_y, fmaxf(-P.lim_y, pc[1] * P.rz));
  return P;
}

__global__ void __launch_bounds__(kProjThreads) project_fwd_kernel(const TgsProjectArgs a) {
  const int64_t idx = blockIdx.x * static_cast<int64_t>(kProjThreads) + threadIdx.x;
  const int64_t total = static_cast<int64_t>(a.n_cameras) * a.n_gaussians;
  if (idx >= total) return;
  const int64_t cam = idx / a.n_gaussians, g = idx - cam * a.n_gaussians;
  // culled entries: radius 0 and zero outputs
  auto cull = [&]() {
    a.radii[idx] = 0;
    a.means2d[idx * 2] = 0.f;
    a.means2d[idx * 2 + 1] = 0.f;
    a.depths[idx] = 0.f;
    a.conics[idx * 3] = 0.f;
    a.conics[idx * 3 + 1] = 0.f;
    a.conics[idx * 3 + 2] = 0.f;
    if (a.compensations != nullptr) a.compensations[idx] = 0.f;
  };
  ProjectGeom G;
  project_geometry(a, cam, g, G);
  if (G.pc[2] < a.near_plane || G.pc[2] > a.far_plane) {
    cull();
    return;
  }
  const Persp P = persp_setup(a, cam, G.pc);
  const float J02 = -P.fx * P.tx * P.rz2, J12 = -P.fy * P.ty * P.rz2;
  const float J00 = P.fx * P.rz, J11 = P.fy * P.rz;
  // cov2d = J cov_c J^T (J is 2x3 with J01 = J10 = 0)
  const float* C3 = G.cov_c;
  const float a0 = J00 * C3[0] + J02 * C3[6], a1 = J00 * C3[1] + J02 * C3[7], a2 = J00 * C3[2] + J02 * C3[8];
  // (the (1, 0) entry equals the (0, 1) entry: cov2d is symmetric)
  const float b1 = J11 * C3[4] + J12 * C3[7], b2 = J11 * C3[5] + J12 * C3[8];
  float c00 = a0 * J00 + a2 * J02;
  const float c01 = a1 * J11 + a2 * J12;
  float c11 = b1 * J11 + b2 * J12;
  const float det_orig = c00 * c11 - c01 * c01;
  c00 += a.eps2d;
  c11 += a.eps2d;
  const float det = c00 * c11 - c01 * c01;
  if (!(det > 0.f)) {
    cull();
    return;
  }
  const float inv_det = 1.f / det;
  const float bmid = 0.5f * (c00 + c11);
  const float v1 = bmid + sqrtf(fmaxf(0.01f, bmid * bmid - det));
  const float radius = ceilf(3.f * sqrtf(v1));
  if (radius <= a.radius_clip) {
    cull();
    return;
  }
  const float mx = P.fx * G.pc[0] * P.rz + P.cx, my = P.fy * G.pc[1] * P.rz + P.cy;
  if (mx + radius <= 0.f || mx - radius >= a.image_width || my + radius <= 0.f ||
      my - radius >= a.image_height) {
    cull();
    return;
  }
  a.radii[idx] = static_cast<int32_t>(radius);
  a.means2d[idx * 2] = mx;
  a.means2d[idx * 2 + 1] = my;
  a.depths[idx] = G.pc[2];
  a.conics[idx * 3] = c11 * inv_det;
  a.conics[idx * 3 + 1] = -c01 * inv_det;
  a.conics[idx * 3 + 2] = c00 * inv_det;
  if (a.compensations != nullptr) a.compensations[idx] = sqrtf(fmaxf(0.f, det_orig / det));
}

__global__ void __launch_bounds__(kProjThreads) project_bwd_kernel(const TgsProjectBwdArgs b) {
  const TgsProjectArgs& a = b.fwd;
  const int64_t idx = blockIdx.x * static_cast<int64_t>(kProjThreads) + threadIdx.x;
  const int64_t total = static_cast<int64_t>(a.n_cameras) * a.n_gaussians;
  if (idx >= total || a.radii[idx] <= 0) return;
  const int64_t cam = idx / a.n_gaussians, g = idx - cam * a.n_gaussians;

  // conic P = inverse(cov2d): dL/dcov2d = -P dL/dP P (symmetric; the
  // off-diagonal conic gradient is shared by both entries)
  const float p00 = a.conics[idx * 3], p01 = a.conics[idx * 3 + 1], p11 = a.conics[idx * 3 + 2];
  const float w00 = b.v_conics[idx * 3], w01 = 0.5f * b.v_conics[idx * 3 + 1],
              w11 = b.v_conics[idx * 3 + 2];
  // -P W P
  const float t00 = p00 * w00 + p01 * w01, t01 = p00 * w01 + p01 * w11;
  const float t10 = p01 * w00 + p11 * w01, t11 = p01 * w01 + p11 * w11;
  float g00 = -(t00 * p00 + t01 * p01), g01 = -(t00 * p01 + t01 * p11);
  float g10 = -(t10 * p00 + t11 * p01), g11 = -(t10 * p01 + t11 * p11);
  if (b.v_compensations != nullptr && a.compensations != nullptr) {
    // comp = sqrt(det(cov) / det(cov + eps I)):
    // dcomp^2/dcov = (1 - comp^2) conic - eps det(conic) I
    const float comp = a.compensations[idx];
    const float half_v = b.v_compensations[idx] * 0.5f / (comp + 1e-6f);
    const float one_m = 1.f - comp * comp;
    const float det_p = p00 * p11 - p01 * p01;
    g00 += half_v * (one_m * p00 - a.eps2d * det_p);
    g01 += half_v * (one_m * p01);
    g10 += half_v * (one_m * p01);
    g11 += half_v * (one_m * p11 - a.eps2d * det_p);
  }

  ProjectGeom G;
  project_geometry(a, cam, g, G);
  const Persp P = persp_setup(a, cam, G.pc);
  float J[6] = {P.fx * P.rz, 0.f, -P.fx * P.tx * P.rz2, 0.f, P.fy * P.rz, -P.fy * P.ty * P.rz2};
  const float Gm[4] = {g00, g01, g10, g11};
  // dL/dcov_c = J^T G J
  float v_cov_c[9];
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      float s = 0.f;
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int c = 0; c < 2; ++c) s += J[r * 3 + i] * Gm[r * 2 + c] * J[c * 3 + j];
      v_cov_c[i * 3 + j] = s;
    }
  // dL/dJ = G J cov^T + G^T J cov (cov symmetric)
  float vJ[6];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      float s = 0.f;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const float gsum = Gm[r * 2 + c] + Gm[c * 2 + r];
#pragma unroll
        for (int k = 0; k < 3; ++k) s += gsum * J[c * 3 + k] * G.cov_c[j * 3 + k];
      }
      vJ[r * 3 + j] = s;
    }
  const float vm0 = b.v_means2d[idx * 2], vm1 = b.v_means2d[idx * 2 + 1];
  const float x = G.pc[0], y = G.pc[1];
  const float rz3 = P.rz2 * P.rz;
  float v_pc[3] = {P.fx * P.rz * vm0, P.fy * P.rz * vm1,
                   -(P.fx * x * vm0 + P.fy * y * vm1) * P.rz2};
  // J02 = -fx tx / z^2 with tx = x unclamped, z * limit when clamped
  if (x * P.rz <= P.lim_x && x * P.rz >= -P.lim_x) v_pc[0] += -P.fx * P.rz2 * vJ[2];
  else v_pc[2] += -P.fx * rz3 * vJ[2] * P.tx;
  if (y * P.rz <= P.lim_y && y * P.rz >= -P.lim_y) v_pc[1] += -P.fy * P.rz2 * vJ[5];
  else v_pc[2] += -P.fy * rz3 * vJ[5] * P.ty;
  v_pc[2] += -P.fx * P.rz2 * vJ[0] - P.fy * P.rz2 * vJ[4] + 2.f * P.fx * P.tx * rz3 * vJ[2] +
             2.f * P.fy * P.ty * rz3 * vJ[5];
  v_pc[2] += b.v_depths[idx];

  // p_c = Rv p + t  ->  dL/dp = Rv^T dL/dp_c
  float v_mean[3];
#pragma unroll
  for (int i = 0; i < 3; ++i)
    v_mean[i] = G.Rv[i] * v_pc[0] + G.Rv[3 + i] * v_pc[1] + G.Rv[6 + i] * v_pc[2];
  // cov_c = Rv cov Rv^T  ->  dL/dcov = Rv^T dL/dcov_c Rv
  float tmp[9], v_cov[9];
  mat3_mul_at(G.Rv, v_cov_c, tmp);
  mat3_mul(tmp, G.Rv, v_cov);
  // cov = M M^T  ->  dL/dM = (V + V^T) M
  float vs[9], v_M[9];
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) vs[i * 3 + j] = v_cov[i * 3 + j] + v_cov[j * 3 + i];
  mat3_mul(vs, G.M, v_M);
  // M = Rq diag(s): dL/dRq = dL/dM diag(s), dL/ds_j = sum_i Rq_ij dL/dM_ij
  const float* s = a.scales + g * 3;
  float v_scale[3], v_R[9];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    v_scale[j] = G.Rq[j] * v_M[j] + G.Rq[3 + j] * v_M[3 + j] + G.Rq[6 + j] * v_M[6 + j];
#pragma unroll
    for (int i = 0; i < 3; ++i) v_R[i * 3 + j] = v_M[i * 3 + j] * s[j];
  }
  // Rq(qn): dL/dqn_k = sum_ij dL/dR_ij dR_ij/dqn_k, then through the
  // normalization qn = q / |q|: dL/dq = (v - (v . qn) qn) / |q|
  const float w = G.qn[0], qx = G.qn[1], qy = G.qn[2], qz = G.qn[3];
  const float* V = v_R;
  float vq[4];
  vq[0] = 2.f * (qx * (V[7] - V[5]) + qy * (V[2] - V[6]) + qz * (V[3] - V[1]));
  vq[1] = 2.f * (-2.f * qx * (V[4] + V[8]) + qy * (V[3] + V[1]) + qz * (V[6] + V[2]) +
                 w * (V[7] - V[5]));
  vq[2] = 2.f * (qx * (V[3] + V[1]) - 2.f * qy * (V[0] + V[8]) + qz * (V[7] + V[5]) +
                 w * (V[2] - V[6]));
  vq[3] = 2.f * (qx * (V[6] + V[2]) + qy * (V[7] + V[5]) - 2.f * qz * (V[0] + V[4]) +
                 w * (V[3] - V[1]));
  const float* q = a.quats + g * 4;
  const float inv = rsqrtf(q[1] * q[1] + q[2] * q[2] + q[3] * q[3] + q[0] * q[0]);
  const float dot = vq[0] * w + vq[1] * qx + vq[2] * qy + vq[3] * qz;
  const float qn4[4] = {w, qx, qy, qz};
#pragma unroll
  for (int k = 0; k < 4; ++k) atomicAdd(b.v_quats + g * 4 + k, (vq[k] - dot * qn4[k]) * inv);
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    atomicAdd(b.v_means + g * 3 + k, v_mean[k]);
    atomicAdd(b.v_scales + g * 3 + k, v_scale[k]);
  }
}

// ---------------------------------------------------------------------------
// Tile intersection
// ---------------------------------------------------------------------------
struct TileRect {
  int x0, y0, x1, y1;  // [x0, x1) x [y0, y1)
};

__device__ __forceinline__ TileRect tile_rect(float mx, float my, float radius, int tile_size,
                                              int tile_width, int tile_height) {
  const float tr = radius / static_cast<float>(tile_size);
  const float tx = mx / static_cast<float>(tile_size), ty = my / static_cast<float>(tile_size);
  auto clampi = [](float v, int hi) {
    const float f = v < 0.f ? 0.f : v;
    return min(static_cast<int>(fminf(f, 2147483520.f)), hi);
  };
  TileRect r;
  r.x0 = clampi(floorf(tx - tr), tile_width);
  r.y0 = clampi(floorf(ty - tr), tile_height);
  r.x1 = clampi(ceilf(tx + tr), tile_width);
  r.y1 = clampi(ceilf(ty + tr), tile_height);
  return r;
}

__global__ void isect_count_kernel(const float* __restrict__ means2d, const int32_t* __restrict__ radii,
                                   int64_t n, int tile_size, int tile_width, int tile_height,
                                   int32_t* __restrict__ tiles_per_gauss) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= n) return;
  const int32_t r = radii[i];
  if (r <= 0) {
    tiles_per_gauss[i] = 0;
    return;
  }
  const TileRect t = tile_rect(means2d[i * 2], means2d[i * 2 + 1], static_cast<float>(r),
                               tile_size, tile_width, tile_height);
  tiles_per_gauss[i] = (t.y1 - t.y0) * (t.x1 - t.x0);
}

__global__ void isect_write_kernel(const float* __restrict__ means2d, const int32_t* __restrict__ radii,
                                   const float* __restrict__ depths, int64_t n, int64_t per_camera,
                                   int tile_size, int tile_width, int tile_height, int tile_bits,
                                   const int64_t* __restrict__ cum, int64_t* __restrict__ keys,
                                   int32_t* __restrict__ flatten) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= n) return;
  const int32_t r = radii[i];
  if (r <= 0) return;
  const TileRect t = tile_rect(means2d[i * 2], means2d[i * 2 + 1], static_cast<float>(r),
                               tile_size, tile_width, tile_height);
  const int64_t cam = i / per_camera;
  const int64_t depth_bits = static_cast<int64_t>(__float_as_int(depths[i]));
  const int64_t hi = cam << (32 + tile_bits);
  int64_t out = i == 0 ? 0 : cum[i - 1];
  for (int y = t.y0; y < t.y1; ++y)
    for (int x = t.x0; x < t.x1; ++x) {
      keys[out] = hi | (static_cast<int64_t>(y * tile_width + x) << 32) | depth_bits;
      flatten[out] = static_cast<int32_t>(i);
      ++out;
    }
}

// Depth-ordered intersection (the sort that is not a 64-bit key sort).
// The reference sorts keys camera | tile | depth bits with cub over their
// low 32 + tile_bits + camera_bits bits, stably: within one (camera, tile)
// the entries come by the depth's bits (as an unsigned number), then in
// write order (Gaussian index). The same order results from
//   1. a stable sort of all C*N Gaussians by the depth bits (C*N items),
//   2. emitting each Gaussian's tiles in that order with the key bits
//      [32, 32 + tile_bits + camera_bits) of its reference key (16-bit keys
//      when those are at most 16 bits, else 32-bit),
//   3. a stable sort of those keys (tile_bits + camera_bits bits),
// after which the reference's 64-bit keys are put back (expand). A negative
// depth sign-extends into the reference key, whose bits 32 and up are then
// all ones: such entries get the all-ones key here, as they do there.
__global__ void iota_kernel(int32_t* __restrict__ out, int64_t n) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < n) out[i] = static_cast<int32_t>(i);
}

// One warp per 32 consecutive Gaussians in depth order. Their entries are
// one contiguous output range (cum is the prefix sum in that order), so the
// lanes write entries lane, lane + 32, ... of the range (coalesced, every
// lane busy whatever the Gaussians' sizes); an entry's Gaussian is found by
// binary search over the warp's inclusive entry counts in shared memory.
constexpr int kWriteThreads = 256;
template <typename KeyT>
__global__ void __launch_bounds__(kWriteThreads) isect_write_ordered_kernel(
    const float* __restrict__ means2d, const int32_t* __restrict__ radii,
    const float* __restrict__ depths, const int32_t* __restrict__ order, int64_t n,
    int64_t per_camera, int tile_size, int tile_width, int tile_height, int tile_bits,
    uint32_t key_mask, const int64_t* __restrict__ cum, KeyT* __restrict__ tile_keys,
    int32_t* __restrict__ flatten) {
  constexpr unsigned kAll = 0xffffffffu;
  constexpr int kWarps = kWriteThreads / 32;
  __shared__ int s_end[kWarps][32];
  __shared__ int s_x0[kWarps][32], s_y0[kWarps][32], s_w[kWarps][32];
  __shared__ uint32_t s_hi[kWarps][32];
  __shared__ int32_t s_id[kWarps][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t j = blockIdx.x * static_cast<int64_t>(kWriteThreads) + threadIdx.x;
  const int64_t j0 = j - lane;
  int32_t i = 0;
  int count = 0, x0 = 0, y0 = 0, w = 1;
  uint32_t hi = 0;
  if (j < n) {
    i = order[j];
    const int32_t r = radii[i];
    if (r > 0) {
      const TileRect t = tile_rect(means2d[2 * static_cast<int64_t>(i)],
                                   means2d[2 * static_cast<int64_t>(i) + 1],
                                   static_cast<float>(r), tile_size, tile_width, tile_height);
      count = (t.y1 - t.y0) * (t.x1 - t.x0);
      x0 = t.x0;
      y0 = t.y0;
      w = max(t.x1 - t.x0, 1);
      // all ones for a negative depth (the sign-extended reference key)
      hi = __float_as_int(depths[i]) < 0 ? key_mask
                                         : static_cast<uint32_t>(i / per_camera) << tile_bits;
    }
  }
  int incl = count;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(kAll, incl, o);
    if (lane >= o) incl += v;
  }
  s_end[warp][lane] = incl;
  s_x0[warp][lane] = x0;
  s_y0[warp][lane] = y0;
  s_w[warp][lane] = w;
  s_hi[warp][lane] = hi;
  s_id[warp][lane] = i;
  __syncwarp();
  const int total = __shfl_sync(kAll, incl, 31);
  if (j0 >= n || total == 0) return;
  const int64_t base = j0 == 0 ? 0 : cum[j0 - 1];
  for (int e = lane; e < total; e += 32) {
    // owner: the number of Gaussians whose entries end at or before e
    int g = 0;
#pragma unroll
    for (int step = 16; step >= 1; step >>= 1)
      if (s_end[warp][g + step - 1] <= e) g += step;
    const int local = e - (g == 0 ? 0 : s_end[warp][g - 1]);
    const int sw = s_w[warp][g];
    const int row = local / sw;
    const uint32_t tile = static_cast<uint32_t>((s_y0[warp][g] + row) * tile_width +
                                                s_x0[warp][g] + (local - row * sw));
    const uint32_t sh = s_hi[warp][g];
    tile_keys[base + e] = static_cast<KeyT>(sh == key_mask ? key_mask : (sh | tile));
    flatten[base + e] = s_id[warp][g];
  }
}

template <typename KeyT>
__device__ __forceinline__ int64_t expand_key(KeyT key, int32_t d) {
  return d < 0 ? static_cast<int64_t>(d)
               : static_cast<int64_t>((static_cast<uint64_t>(key) << 32) | static_cast<uint32_t>(d));
}

// Four entries per thread (vector loads of keys and ids, two 16-byte stores).
template <typename KeyT>
__global__ void isect_expand_kernel(const KeyT* __restrict__ tile_keys,
                                    const int32_t* __restrict__ flatten,
                                    const float* __restrict__ depths, int64_t n,
                                    int64_t* __restrict__ keys) {
  const int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t k = 4 * q;
  if (k >= n) return;
  if (k + 4 <= n) {
    const int4 f = *reinterpret_cast<const int4*>(flatten + k);
    KeyT kk[4];
    if constexpr (sizeof(KeyT) == 2) {
      const uint2 v = *reinterpret_cast<const uint2*>(tile_keys + k);
      kk[0] = static_cast<KeyT>(v.x & 0xffffu);
      kk[1] = static_cast<KeyT>(v.x >> 16);
      kk[2] = static_cast<KeyT>(v.y & 0xffffu);
      kk[3] = static_cast<KeyT>(v.y >> 16);
    } else {
      const uint4 v = *reinterpret_cast<const uint4*>(tile_keys + k);
      kk[0] = v.x;
      kk[1] = v.y;
      kk[2] = v.z;
      kk[3] = v.w;
    }
    const int32_t d0 = __float_as_int(depths[f.x]), d1 = __float_as_int(depths[f.y]);
    const int32_t d2 = __float_as_int(depths[f.z]), d3 = __float_as_int(depths[f.w]);
    longlong2* dst = reinterpret_cast<longlong2*>(keys + k);
    dst[0] = make_longlong2(expand_key(kk[0], d0), expand_key(kk[1], d1));
    dst[1] = make_longlong2(expand_key(kk[2], d2), expand_key(kk[3], d3));
  } else {
    for (int64_t e = k; e < n; ++e)
      keys[e] = expand_key(tile_keys[e], __float_as_int(depths[flatten[e]]));
  }
}

// offsets[k] = number of keys whose (camera, tile) index is below k.
__global__ void isect_offsets_kernel(const int64_t* __restrict__ keys, int64_t n_keys, int64_t n_ids,
                                     int n_tiles, int tile_bits, int32_t* __restrict__ offsets) {
  const int64_t k = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (k >= n_ids) return;
  int64_t lo = 0, hi = n_keys;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    const int64_t id = keys[mid] >> 32;
    const int64_t flat = (id >> tile_bits) * n_tiles + (id & ((1ll << tile_bits) - 1));
    if (flat < k) lo = mid + 1;
    else hi = mid;
  }
  offsets[k] = static_cast<int32_t>(lo);
}

// ---------------------------------------------------------------------------
// Rasterization
// ---------------------------------------------------------------------------
struct TileSpan {
  int start, end;
};

__device__ __forceinline__ TileSpan tile_span(const TgsRasterArgs& a, int cam, int tile_id) {
  const int n_tiles = a.tile_width * a.tile_height;
  const int32_t* offs = a.tile_offsets + static_cast<int64_t>(cam) * n_tiles;
  TileSpan s;
  s.start = offs[tile_id];
  s.end = (cam == a.n_cameras - 1 && tile_id == n_tiles - 1) ? static_cast<int>(a.n_isects)
                                                             : offs[tile_id + 1];
  return s;
}

// Forward, front to back; each thread composites P vertically adjacent
// pixels of its column, reading each staged Gaussian once for them.
template <int D, int P>
__global__ void raster_fwd_kernel(const TgsRasterArgs a) {
  extern __shared__ __align__(16) unsigned char raster_smem[];
  const int nthreads = blockDim.x * blockDim.y;
  int32_t* ids = reinterpret_cast<int32_t*>(raster_smem);
  float3* xyo = reinterpret_cast<float3*>(ids + nthreads);
  float3* con = xyo + nthreads;
  float* rgb = reinterpret_cast<float*>(con + nthreads);

  const int cam = blockIdx.x;
  const int tile_id = blockIdx.y * a.tile_width + blockIdx.z;
  const int j = blockIdx.z * a.tile_size + threadIdx.x;
  const int tr = threadIdx.y * blockDim.x + threadIdx.x;
  const int64_t pix_base = static_cast<int64_t>(cam) * a.image_height * a.image_width;
  const float px = static_cast<float>(j) + 0.5f;
  bool done[P];
  float py[P], T[P], acc[P][D];
  int cur[P];
#pragma unroll
  for (int q = 0; q < P; ++q) {
    const int i = blockIdx.y * a.tile_size + threadIdx.y * P + q;
    done[q] = !(i < a.image_height && j < a.image_width);
    py[q] = static_cast<float>(i) + 0.5f;
    T[q] = 1.f;
    cur[q] = 0;
#pragma unroll
    for (int k = 0; k < D; ++k) acc[q][k] = 0.f;
  }

  const TileSpan span = tile_span(a, cam, tile_id);
  const int n_batches = (span.end - span.start + nthreads - 1) / nthreads;

  for (int b = 0; b < n_batches; ++b) {
    bool all_done = true;
#pragma unroll
    for (int q = 0; q < P; ++q) all_done &= done[q];
    if (__syncthreads_count(all_done) >= nthreads) break;
    const int batch_start = span.start + b * nthreads;
    const int idx = batch_start + tr;
    if (idx < span.end) {
      const int32_t g = a.flatten_ids[idx];
      ids[tr] = g;
      xyo[tr] = make_float3(a.means2d[2 * static_cast<int64_t>(g)], a.means2d[2 * static_cast<int64_t>(g) + 1],
                            a.opacities[g]);
      con[tr] = make_float3(a.conics[3 * static_cast<int64_t>(g)], a.conics[3 * static_cast<int64_t>(g) + 1],
                            a.conics[3 * static_cast<int64_t>(g) + 2]);
#pragma unroll
      for (int k = 0; k < D; ++k) rgb[tr * D + k] = a.colors[static_cast<int64_t>(g) * D + k];
    }
    __syncthreads();
    const int batch_size = min(nthreads, span.end - batch_start);
    for (int t = 0; t < batch_size && !all_done; ++t) {
      const float3 c = con[t];
      const float3 xo = xyo[t];
      const float dx = xo.x - px;
      all_done = true;
#pragma unroll
      for (int q = 0; q < P; ++q) {
        if (!done[q]) {
          const float dy = xo.y - py[q];
          const float sigma = 0.5f * (c.x * dx * dx + c.z * dy * dy) + c.y * dx * dy;
          const float alpha = fminf(0.999f, xo.z * __expf(-sigma));
          if (sigma >= 0.f && alpha >= 1.f / 255.f) {
            const float next_T = T[q] * (1.f - alpha);
            if (next_T <= 1e-4f) {
              done[q] = true;
            } else {
              const float vis = alpha * T[q];
#pragma unroll
              for (int k = 0; k < D; ++k) acc[q][k] += rgb[t * D + k] * vis;
              cur[q] = batch_start + t;
              T[q] = next_T;
            }
          }
        }
        all_done &= done[q];
      }
    }
  }
#pragma unroll
  for (int q = 0; q < P; ++q) {
    const int i = blockIdx.y * a.tile_size + threadIdx.y * P + q;
    if (i < a.image_height && j < a.image_width) {
      const int64_t pix = pix_base + static_cast<int64_t>(i) * a.image_width + j;
      a.render_alphas[pix] = 1.f - T[q];
      const float* bg = a.backgrounds != nullptr ? a.backgrounds + cam * D : nullptr;
#pragma unroll
      for (int k = 0; k < D; ++k)
        a.render_colors[pix * D + k] = bg ? acc[q][k] + T[q] * bg[k] : acc[q][k];
      a.last_ids[pix] = cur[q];
    }
  }
}

// Warp reduce-scatter of 16 values: afterwards lane L holds the warp total
// of value L >> 1 (lanes L and L ^ 1 hold the same total). Each halving
// step sends half of the lane's values to its partner and keeps the other
// half: 8 + 4 + 2 + 1 + 1 = 16 shuffles for all 16 totals, where 16
// separate butterfly sums take 80.
__device__ __forceinline__ float warp_reduce_scatter16(const float (&v)[16], int lane) {
  constexpr unsigned kAll = 0xffffffffu;
  float w8[8], w4[4], w2[2];
  const bool u16 = lane & 16, u8 = lane & 8, u4 = lane & 4, u2 = lane & 2;
#pragma unroll
  for (int k = 0; k < 8; ++k)
    w8[k] = (u16 ? v[k + 8] : v[k]) + __shfl_xor_sync(kAll, u16 ? v[k] : v[k + 8], 16);
#pragma unroll
  for (int k = 0; k < 4; ++k)
    w4[k] = (u8 ? w8[k + 4] : w8[k]) + __shfl_xor_sync(kAll, u8 ? w8[k] : w8[k + 4], 8);
#pragma unroll
  for (int k = 0; k < 2; ++k)
    w2[k] = (u4 ? w4[k + 2] : w4[k]) + __shfl_xor_sync(kAll, u4 ? w4[k] : w4[k + 2], 4);
  float w1 = (u2 ? w2[1] : w2[0]) + __shfl_xor_sync(kAll, u2 ? w2[0] : w2[1], 2);
  return w1 + __shfl_xor_sync(kAll, w1, 1);
}

// Backward, back to front. Each thread handles P vertically adjacent pixels
// of its column (a warp covers a 16 x (2P) patch of a 16-pixel tile): the
// Gaussian is read from shared memory once for the P pixels, its per-pixel
// gradients are added in registers, and one warp reduce-scatter plus one
// set of atomics serves 32 P pixels.
template <int D, int P>
__global__ void raster_bwd_kernel(const TgsRasterBwdArgs b) {
  const TgsRasterArgs& a = b.fwd;
  // per-Gaussian gradient: means2d (2), conic (3), colors (D), opacity,
  // |means2d| (2)
  constexpr int K = 2 + 3 + D + 1 + 2;
  static_assert(K <= 16, "one reduce-scatter holds 16 values");
  extern __shared__ __align__(16) unsigned char raster_smem[];
  const int nthreads = blockDim.x * blockDim.y;
  int32_t* ids = reinterpret_cast<int32_t*>(raster_smem);
  float3* xyo = reinterpret_cast<float3*>(ids + nthreads);
  float3* con = xyo + nthreads;
  float* rgb = reinterpret_cast<float*>(con + nthreads);

  const int cam = blockIdx.x;
  const int tile_id = blockIdx.y * a.tile_width + blockIdx.z;
  const int j = blockIdx.z * a.tile_size + threadIdx.x;
  const int tr = threadIdx.y * blockDim.x + threadIdx.x;
  const int lane = tr & 31;
  const int64_t plane = static_cast<int64_t>(a.image_height) * a.image_width;
  const float px = static_cast<float>(j) + 0.5f;
  const bool absgrad = b.v_means2d_abs != nullptr;

  // the gradient component this lane adds to global memory after the
  // reduce-scatter (lane 2k holds component k)
  const int comp = lane >> 1;
  const bool adds = (lane & 1) == 0 && comp < (absgrad ? K : K - 2);
  float* comp_base = nullptr;
  int comp_stride = 0;
  if (adds) {
    if (comp < 2) comp_base = b.v_means2d + comp, comp_stride = 2;
    else if (comp < 5) comp_base = b.v_conics + (comp - 2), comp_stride = 3;
    else if (comp < 5 + D) comp_base = b.v_colors + (comp - 5), comp_stride = D;
    else if (comp == 5 + D) comp_base = b.v_opacities, comp_stride = 1;
    else comp_base = b.v_means2d_abs + (comp - 6 - D), comp_stride = 2;
  }

  const TileSpan span = tile_span(a, cam, tile_id);
  const int n_batches = (span.end - span.start + nthreads - 1) / nthreads;

  bool inside[P];
  float py[P], T_final[P], T[P], buffer[P][D], v_out[P][D], v_alpha_out[P], bg_dot[P];
  int bin_final[P];
  int warp_bin_final = 0;
#pragma unroll
  for (int q = 0; q < P; ++q) {
    const int i = blockIdx.y * a.tile_size + threadIdx.y * P + q;
    inside[q] = i < a.image_height && j < a.image_width;
    py[q] = static_cast<float>(i) + 0.5f;
    const int64_t pix = static_cast<int64_t>(cam) * plane +
                        min(static_cast<int64_t>(i) * a.image_width + j, plane - 1);
    T_final[q] = 1.f - a.render_alphas[pix];
    T[q] = T_final[q];
    bin_final[q] = inside[q] ? a.last_ids[pix] : 0;
    warp_bin_final = max(warp_bin_final, bin_final[q]);
#pragma unroll
    for (int k = 0; k < D; ++k) {
      buffer[q][k] = 0.f;
      v_out[q][k] = b.v_render_colors[pix * D + k];
    }
    v_alpha_out[q] = b.v_render_alphas[pix];
    bg_dot[q] = 0.f;
    if (a.backgrounds != nullptr) {
#pragma unroll
      for (int k = 0; k < D; ++k) bg_dot[q] += a.backgrounds[cam * D + k] * v_out[q][k];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    warp_bin_final = max(warp_bin_final, __shfl_xor_sync(0xffffffffu, warp_bin_final, o));

  for (int bt = 0; bt < n_batches; ++bt) {
    __syncthreads();
    // back to front: slot 0 is the farthest Gaussian of the batch
    const int batch_end = span.end - 1 - bt * nthreads;
    const int batch_size = min(nthreads, batch_end + 1 - span.start);
    const int idx = batch_end - tr;
    if (idx >= span.start) {
      const int32_t g = a.flatten_ids[idx];
      ids[tr] = g;
      xyo[tr] = make_float3(a.means2d[2 * static_cast<int64_t>(g)], a.means2d[2 * static_cast<int64_t>(g) + 1],
                            a.opacities[g]);
      con[tr] = make_float3(a.conics[3 * static_cast<int64_t>(g)], a.conics[3 * static_cast<int64_t>(g) + 1],
                            a.conics[3 * static_cast<int64_t>(g) + 2]);
#pragma unroll
      for (int k = 0; k < D; ++k) rgb[tr * D + k] = a.colors[static_cast<int64_t>(g) * D + k];
    }
    __syncthreads();
    for (int t = max(0, batch_end - warp_bin_final); t < batch_size; ++t) {
      const float3 c = con[t];
      const float3 xo = xyo[t];
      const float opac = xo.z;
      const float dx = xo.x - px;
      bool valid[P];
      float vis[P], alpha[P], dy[P];
      bool any = false;
#pragma unroll
      for (int q = 0; q < P; ++q) {
        dy[q] = xo.y - py[q];
        const float sigma = 0.5f * (c.x * dx * dx + c.z * dy[q] * dy[q]) + c.y * dx * dy[q];
        vis[q] = __expf(-sigma);
        alpha[q] = fminf(0.999f, opac * vis[q]);
        valid[q] = inside[q] && (batch_end - t <= bin_final[q]) && sigma >= 0.f &&
                   alpha[q] >= 1.f / 255.f;
        any |= valid[q];
      }
      if (!__any_sync(0xffffffffu, any)) continue;
      float gv[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) gv[k] = 0.f;
      float col[D];
#pragma unroll
      for (int k = 0; k < D; ++k) col[k] = rgb[t * D + k];
#pragma unroll
      for (int q = 0; q < P; ++q) {
        if (!valid[q]) continue;
        // fast reciprocal (the render path is compared within tolerance)
        const float ra = __fdividef(1.f, 1.f - alpha[q]);
        T[q] *= ra;
        const float fac = alpha[q] * T[q];
        float v_alpha = 0.f;
#pragma unroll
        for (int k = 0; k < D; ++k) {
          gv[5 + k] += fac * v_out[q][k];
          v_alpha += (col[k] * T[q] - buffer[q][k] * ra) * v_out[q][k];
        }
        v_alpha += T_final[q] * ra * v_alpha_out[q];
        if (a.backgrounds != nullptr) v_alpha += -T_final[q] * ra * bg_dot[q];
        if (opac * vis[q] <= 0.999f) {
          const float v_sigma = -opac * vis[q] * v_alpha;
          const float gx = v_sigma * (c.x * dx + c.y * dy[q]);
          const float gy = v_sigma * (c.y * dx + c.z * dy[q]);
          gv[0] += gx;
          gv[1] += gy;
          gv[2] += 0.5f * v_sigma * dx * dx;
          gv[3] += v_sigma * dx * dy[q];
          gv[4] += 0.5f * v_sigma * dy[q] * dy[q];
          gv[5 + D] += vis[q] * v_alpha;
          gv[6 + D] += fabsf(gx);
          gv[7 + D] += fabsf(gy);
        }
#pragma unroll
        for (int k = 0; k < D; ++k) buffer[q][k] += col[k] * fac;
      }
      const float total = warp_reduce_scatter16(gv, lane);
      if (adds) atomicAdd(comp_base + static_cast<int64_t>(comp_stride) * ids[t], total);
    }
  }
}

template <int D>
size_t raster_smem_bytes(int nthreads) {
  // per staged Gaussian: id, (x, y, opacity), conic, D colors
  return nthreads * (sizeof(int32_t) + 2 * sizeof(float3) + sizeof(float) * D);
}

template <int D>
int launch_raster(const TgsRasterArgs& a, const TgsRasterBwdArgs* bwd, cudaStream_t s) {
  const int nthreads = a.tile_size * a.tile_size;
  const dim3 grid(a.n_cameras, a.tile_height, a.tile_width);
  // two pixels per thread: tile_size^2 is a multiple of 32, so tile_size
  // is a multiple of 8 and half a tile is whole warps
  const size_t smem2 = raster_smem_bytes<D>(nthreads / 2);
  if (bwd == nullptr) {
    TGS_CUDA(cudaFuncSetAttribute(raster_fwd_kernel<D, 2>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(smem2)));
    raster_fwd_kernel<D, 2><<<grid, dim3(a.tile_size, a.tile_size / 2, 1), smem2, s>>>(a);
  } else {
    TGS_CUDA(cudaFuncSetAttribute(raster_bwd_kernel<D, 2>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(smem2)));
    raster_bwd_kernel<D, 2><<<grid, dim3(a.tile_size, a.tile_size / 2, 1), smem2, s>>>(*bwd);
  }
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

int check_raster(const TgsRasterArgs* a) {
  TGS_CHECK_ARG(a != nullptr, "rasterize: args is NULL");
  TGS_CHECK_ARG(a->n_cameras >= 0 && a->n_cameras <= 65535, "rasterize: bad camera count");
  TGS_CHECK_ARG(a->tile_size >= 1 && a->tile_size * a->tile_size <= 1024 &&
                    (a->tile_size * a->tile_size) % 32 == 0,
                "rasterize: tile_size^2 must be a multiple of 32 and at most 1024");
  TGS_CHECK_ARG(a->tile_width >= 1 && a->tile_height >= 1 && a->tile_height <= 65535 &&
                    a->tile_width <= 65535,
                "rasterize: bad tile grid");
  TGS_CHECK_ARG(static_cast<int64_t>(a->tile_width) * a->tile_size >= a->image_width &&
                    static_cast<int64_t>(a->tile_height) * a->tile_size >= a->image_height,
                "rasterize: the tile grid does not cover the image");
  TGS_CHECK_ARG(a->channels >= 1 && a->channels <= 4, "rasterize: channels must be 1..4 (got %d)",
                a->channels);
  TGS_CHECK_ARG(a->n_isects >= 0 && a->n_isects < (1ll << 31), "rasterize: bad n_isects");
  return TGS_OK;
}

}  // namespace
}  // namespace tgs

using namespace tgs;

extern "C" int tgs_project_fwd(const TgsProjectArgs* a, void* stream) {
  TGS_CHECK_ARG(a != nullptr, "tgs_project_fwd: args is NULL");
  TGS_CHECK_ARG(a->n_cameras >= 0 && a->n_gaussians >= 0, "tgs_project_fwd: negative size");
  const int64_t total = static_cast<int64_t>(a->n_cameras) * a->n_gaussians;
  if (total == 0) return TGS_OK;
  TGS_CHECK_ARG(a->means && a->quats && a->scales && a->viewmats && a->Ks && a->radii &&
                    a->means2d && a->depths && a->conics,
                "tgs_project_fwd: NULL pointer");
  project_fwd_kernel<<<static_cast<unsigned>(ceil_div<int64_t>(total, kProjThreads)), kProjThreads, 0,
                       as_stream(stream)>>>(*a);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int tgs_project_bwd(const TgsProjectBwdArgs* b, void* stream) {
  TGS_CHECK_ARG(b != nullptr, "tgs_project_bwd: args is NULL");
  const TgsProjectArgs& a = b->fwd;
  const int64_t total = static_cast<int64_t>(a.n_cameras) * a.n_gaussians;
  if (total == 0) return TGS_OK;
  TGS_CHECK_ARG(a.means && a.quats && a.scales && a.viewmats && a.Ks && a.radii && a.conics,
                "tgs_project_bwd: NULL forward pointer");
  TGS_CHECK_ARG(b->v_means2d && b->v_depths && b->v_conics && b->v_means && b->v_quats &&
                    b->v_scales,
                "tgs_project_bwd: NULL gradient pointer");
  project_bwd_kernel<<<static_cast<unsigned>(ceil_div<int64_t>(total, kProjThreads)), kProjThreads, 0,
                       as_stream(stream)>>>(*b);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int tgs_isect_count(const float* means2d, const int32_t* radii, int64_t n, int32_t tile_size,
                               int32_t tile_width, int32_t tile_height, int32_t* tiles_per_gauss,
                               void* stream) {
  TGS_CHECK_ARG(n >= 0 && tile_size > 0 && tile_width > 0 && tile_height > 0,
                "tgs_isect_count: bad sizes");
  if (n == 0) return TGS_OK;
  TGS_CHECK_ARG(means2d && radii && tiles_per_gauss, "tgs_isect_count: NULL pointer");
  isect_count_kernel<<<static_cast<unsigned>(ceil_div<int64_t>(n, 256)), 256, 0, as_stream(stream)>>>(
      means2d, radii, n, tile_size, tile_width, tile_height, tiles_per_gauss);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int32_t tgs_isect_tile_bits(int32_t n_tiles) {
  int32_t bits = 0;
  while ((1ll << bits) <= n_tiles) ++bits;  // floor(log2(n_tiles)) + 1
  return bits;
}

extern "C" int tgs_isect_write(const float* means2d, const int32_t* radii, const float* depths,
                               int64_t n, int64_t n_per_camera, int32_t tile_size, int32_t tile_width,
                               int32_t tile_height, const int64_t* cum_tiles, int64_t* isect_ids,
                               int32_t* flatten_ids, void* stream) {
  TGS_CHECK_ARG(n >= 0 && n_per_camera > 0 && tile_size > 0 && tile_width > 0 && tile_height > 0,
                "tgs_isect_write: bad sizes");
  TGS_CHECK_ARG(n < (1ll << 31), "tgs_isect_write: more than 2^31 projected Gaussians");
  if (n == 0) return TGS_OK;
  TGS_CHECK_ARG(means2d && radii && depths && cum_tiles && isect_ids && flatten_ids,
                "tgs_isect_write: NULL pointer");
  const int n_tiles = tile_width * tile_height;
  const int tile_bits = tgs_isect_tile_bits(n_tiles);
  const int cam_bits = tgs_isect_tile_bits(static_cast<int32_t>(n / n_per_camera));
  TGS_CHECK_ARG(tile_bits + cam_bits <= 32, "tgs_isect_write: camera and tile ids need %d bits",
                tile_bits + cam_bits);
  isect_write_kernel<<<static_cast<unsigned>(ceil_div<int64_t>(n, 256)), 256, 0, as_stream(stream)>>>(
      means2d, radii, depths, n, n_per_camera, tile_size, tile_width, tile_height, tile_bits,
      cum_tiles, isect_ids, flatten_ids);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

namespace {
constexpr size_t kScratchAlign = 256;
size_t align_up(size_t v) { return (v + kScratchAlign - 1) / kScratchAlign * kScratchAlign; }

int isect_key_bits(int64_t n_cameras, int32_t n_tiles) {
  return tgs_isect_tile_bits(n_tiles) + tgs_isect_tile_bits(static_cast<int32_t>(n_cameras));
}

// cub's scratch for a stable (key, int32 value) sort of n items over `bits` bits.
template <typename KeyT>
cudaError_t pair_sort_temp_bytes(int64_t n, int bits, size_t* bytes) {
  *bytes = 0;
  return cub::DeviceRadixSort::SortPairs(nullptr, *bytes, static_cast<const KeyT*>(nullptr),
                                         static_cast<KeyT*>(nullptr),
                                         static_cast<const int32_t*>(nullptr),
                                         static_cast<int32_t*>(nullptr), static_cast<int>(n), 0,
                                         bits);
}

cudaError_t ordered_scan_temp_bytes(int64_t n, size_t* bytes) {
  *bytes = 0;
  const auto it = thrust::make_transform_iterator(thrust::counting_iterator<int64_t>(0),
                                                  OrderedTileCount{nullptr, nullptr});
  return cub::DeviceScan::InclusiveSum(nullptr, *bytes, it, static_cast<int64_t*>(nullptr),
                                       static_cast<int>(n));
}

// Layout of tgs_isect_depth_order's scratch: [temp | keys out (n u32) | iota (n i32)].
int depth_order_layout(int64_t n, size_t* temp, size_t* total) {
  size_t sort_temp = 0, scan_temp = 0;
  TGS_CUDA(pair_sort_temp_bytes<uint32_t>(n, 32, &sort_temp));
  TGS_CUDA(ordered_scan_temp_bytes(n, &scan_temp));
  *temp = align_up(std::max(sort_temp, scan_temp));
  *total = *temp + 2 * align_up(static_cast<size_t>(n) * 4);
  return TGS_OK;
}
}  // namespace

extern "C" int32_t tgs_isect_key_bytes(int32_t n_cameras, int32_t tile_width,
                                       int32_t tile_height) {
  if (n_cameras <= 0 || tile_width <= 0 || tile_height <= 0) return 0;
  const int bits = isect_key_bits(n_cameras, tile_width * tile_height);
  return bits <= 16 ? 2 : bits <= 32 ? 4 : 0;
}

extern "C" int tgs_isect_depth_order_scratch_bytes(int64_t n, size_t* bytes) {
  TGS_CHECK_ARG(bytes && n >= 0 && n < (1ll << 31), "tgs_isect_depth_order_scratch_bytes: bad n");
  size_t temp = 0;
  return depth_order_layout(n, &temp, bytes);
}

extern "C" int tgs_isect_depth_order(const float* depths, const int32_t* tiles_per_gauss,
                                     int64_t n, int32_t* order, int64_t* cum_tiles, void* scratch,
                                     size_t scratch_bytes, void* stream) {
  TGS_CHECK_ARG(n >= 0 && n < (1ll << 31), "tgs_isect_depth_order: bad n");
  if (n == 0) return TGS_OK;
  TGS_CHECK_ARG(depths && tiles_per_gauss && order && cum_tiles && scratch,
                "tgs_isect_depth_order: NULL pointer");
  size_t temp = 0, need = 0;
  if (depth_order_layout(n, &temp, &need) != TGS_OK) return TGS_ERR_CUDA;
  TGS_CHECK_ARG(scratch_bytes >= need, "tgs_isect_depth_order: scratch holds %zu bytes, needs %zu",
                scratch_bytes, need);
  char* base = static_cast<char*>(scratch);
  uint32_t* keys_out = reinterpret_cast<uint32_t*>(base + temp);
  int32_t* iota = reinterpret_cast<int32_t*>(base + temp + align_up(static_cast<size_t>(n) * 4));
  cudaStream_t s = as_stream(stream);
  iota_kernel<<<static_cast<unsigned>(ceil_div<int64_t>(n, 256)), 256, 0, s>>>(iota, n);
  TGS_LAUNCH_CHECK();
  size_t sort_temp = temp;
  TGS_CUDA(cub::DeviceRadixSort::SortPairs(base, sort_temp,
                                           reinterpret_cast<const uint32_t*>(depths), keys_out,
                                           iota, order, static_cast<int>(n), 0, 32, s));
  size_t scan_temp = temp;
  const auto it = thrust::make_transform_iterator(thrust::counting_iterator<int64_t>(0),
                                                  OrderedTileCount{tiles_per_gauss, order});
  TGS_CUDA(cub::DeviceScan::InclusiveSum(base, scan_temp, it, cum_tiles, static_cast<int>(n), s));
  return TGS_OK;
}

extern "C" int tgs_isect_write_ordered(const float* means2d, const int32_t* radii,
                                       const float* depths, const int32_t* order, int64_t n,
                                       int64_t n_per_camera, int32_t tile_size, int32_t tile_width,
                                       int32_t tile_height, const int64_t* cum_tiles,
                                       void* tile_keys, int32_t* flatten_ids, void* stream) {
  TGS_CHECK_ARG(n >= 0 && n_per_camera > 0 && tile_size > 0 && tile_width > 0 && tile_height > 0,
                "tgs_isect_write_ordered: bad sizes");
  TGS_CHECK_ARG(n < (1ll << 31), "tgs_isect_write_ordered: more than 2^31 projected Gaussians");
  if (n == 0) return TGS_OK;
  TGS_CHECK_ARG(means2d && radii && depths && order && cum_tiles && tile_keys && flatten_ids,
                "tgs_isect_write_ordered: NULL pointer");
  const int n_tiles = tile_width * tile_height;
  const int64_t n_cameras = ceil_div<int64_t>(n, n_per_camera);
  TGS_CHECK_ARG(n_cameras <= 65535, "tgs_isect_write_ordered: too many cameras");
  const int bits = isect_key_bits(n_cameras, n_tiles);
  TGS_CHECK_ARG(bits <= 32, "tgs_isect_write_ordered: camera and tile ids need %d bits", bits);
  const uint32_t mask = static_cast<uint32_t>((1ull << bits) - 1);
  const unsigned grid = static_cast<unsigned>(ceil_div<int64_t>(n, kWriteThreads));
  cudaStream_t s = as_stream(stream);
  if (bits <= 16)
    isect_write_ordered_kernel<uint16_t><<<grid, kWriteThreads, 0, s>>>(
        means2d, radii, depths, order, n, n_per_camera, tile_size, tile_width, tile_height,
        tgs_isect_tile_bits(n_tiles), mask, cum_tiles, static_cast<uint16_t*>(tile_keys),
        flatten_ids);
  else
    isect_write_ordered_kernel<uint32_t><<<grid, kWriteThreads, 0, s>>>(
        means2d, radii, depths, order, n, n_per_camera, tile_size, tile_width, tile_height,
        tgs_isect_tile_bits(n_tiles), mask, cum_tiles, static_cast<uint32_t*>(tile_keys),
        flatten_ids);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int tgs_isect_sort_tiles_scratch_bytes(int64_t n_isects, int32_t n_cameras,
                                                  int32_t tile_width, int32_t tile_height,
                                                  size_t* bytes) {
  const int32_t key_bytes = tgs_isect_key_bytes(n_cameras, tile_width, tile_height);
  TGS_CHECK_ARG(bytes && n_isects >= 0 && n_isects < (1ll << 31) && key_bytes > 0,
                "tgs_isect_sort_tiles_scratch_bytes: bad sizes");
  const int bits = isect_key_bits(n_cameras, tile_width * tile_height);
  if (key_bytes == 2) TGS_CUDA(pair_sort_temp_bytes<uint16_t>(n_isects, bits, bytes));
  else TGS_CUDA(pair_sort_temp_bytes<uint32_t>(n_isects, bits, bytes));
  return TGS_OK;
}

extern "C" int tgs_isect_sort_tiles(const void* tile_keys_in, const int32_t* flatten_in,
                                    int64_t n_isects, int32_t n_cameras, int32_t tile_width,
                                    int32_t tile_height, void* tile_keys_out,
                                    int32_t* flatten_out, void* scratch, size_t scratch_bytes,
                                    void* stream) {
  const int32_t key_bytes = tgs_isect_key_bytes(n_cameras, tile_width, tile_height);
  TGS_CHECK_ARG(n_isects >= 0 && n_isects < (1ll << 31) && key_bytes > 0,
                "tgs_isect_sort_tiles: bad sizes");
  if (n_isects == 0) return TGS_OK;
  TGS_CHECK_ARG(tile_keys_in && flatten_in && tile_keys_out && flatten_out && scratch,
                "tgs_isect_sort_tiles: NULL pointer");
  const int bits = isect_key_bits(n_cameras, tile_width * tile_height);
  size_t temp = 0;
  cudaStream_t s = as_stream(stream);
  if (key_bytes == 2) {
    TGS_CUDA(pair_sort_temp_bytes<uint16_t>(n_isects, bits, &temp));
    TGS_CHECK_ARG(scratch_bytes >= temp, "tgs_isect_sort_tiles: scratch holds %zu bytes, needs %zu",
                  scratch_bytes, temp);
    TGS_CUDA(cub::DeviceRadixSort::SortPairs(
        scratch, temp, static_cast<const uint16_t*>(tile_keys_in),
        static_cast<uint16_t*>(tile_keys_out), flatten_in, flatten_out,
        static_cast<int>(n_isects), 0, bits, s));
  } else {
    TGS_CUDA(pair_sort_temp_bytes<uint32_t>(n_isects, bits, &temp));
    TGS_CHECK_ARG(scratch_bytes >= temp, "tgs_isect_sort_tiles: scratch holds %zu bytes, needs %zu",
                  scratch_bytes, temp);
    TGS_CUDA(cub::DeviceRadixSort::SortPairs(
        scratch, temp, static_cast<const uint32_t*>(tile_keys_in),
        static_cast<uint32_t*>(tile_keys_out), flatten_in, flatten_out,
        static_cast<int>(n_isects), 0, bits, s));
  }
  return TGS_OK;
}

extern "C" int tgs_isect_expand_ids(const void* tile_keys, int32_t key_bytes,
                                    const int32_t* flatten_ids, const float* depths,
                                    int64_t n_isects, int64_t* isect_ids, void* stream) {
  TGS_CHECK_ARG(n_isects >= 0 && (key_bytes == 2 || key_bytes == 4),
                "tgs_isect_expand_ids: bad sizes");
  if (n_isects == 0) return TGS_OK;
  TGS_CHECK_ARG(tile_keys && flatten_ids && depths && isect_ids, "tgs_isect_expand_ids: NULL pointer");
  TGS_CHECK_ARG(reinterpret_cast<uintptr_t>(tile_keys) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(flatten_ids) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(isect_ids) % 16 == 0,
                "tgs_isect_expand_ids: arrays must start on 16-byte boundaries");
  const unsigned grid = static_cast<unsigned>(ceil_div<int64_t>(ceil_div<int64_t>(n_isects, 4), 256));
  cudaStream_t s = as_stream(stream);
  if (key_bytes == 2)
    isect_expand_kernel<uint16_t><<<grid, 256, 0, s>>>(static_cast<const uint16_t*>(tile_keys),
                                                       flatten_ids, depths, n_isects, isect_ids);
  else
    isect_expand_kernel<uint32_t><<<grid, 256, 0, s>>>(static_cast<const uint32_t*>(tile_keys),
                                                       flatten_ids, depths, n_isects, isect_ids);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int tgs_isect_offsets(const int64_t* isect_ids, int64_t n_isects, int32_t n_cameras,
                                 int32_t tile_width, int32_t tile_height, int32_t* offsets,
                                 void* stream) {
  TGS_CHECK_ARG(n_isects >= 0 && n_cameras >= 0 && tile_width > 0 && tile_height > 0,
                "tgs_isect_offsets: bad sizes");
  const int64_t n_ids = static_cast<int64_t>(n_cameras) * tile_width * tile_height;
  if (n_ids == 0) return TGS_OK;
  TGS_CHECK_ARG(offsets && (n_isects == 0 || isect_ids), "tgs_isect_offsets: NULL pointer");
  const int n_tiles = tile_width * tile_height;
  isect_offsets_kernel<<<static_cast<unsigned>(ceil_div<int64_t>(n_ids, 256)), 256, 0,
                         as_stream(stream)>>>(isect_ids, n_isects, n_ids, n_tiles,
                                              tgs_isect_tile_bits(n_tiles), offsets);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int tgs_rasterize_fwd(const TgsRasterArgs* a, void* stream) {
  const int rc = check_raster(a);
  if (rc != TGS_OK) return rc;
  if (a->n_cameras == 0 || a->image_width <= 0 || a->image_height <= 0) return TGS_OK;
  TGS_CHECK_ARG(a->tile_offsets && a->render_colors && a->render_alphas && a->last_ids,
                "tgs_rasterize_fwd: NULL pointer");
  TGS_CHECK_ARG(a->n_isects == 0 || (a->flatten_ids && a->means2d && a->conics && a->colors &&
                                     a->opacities),
                "tgs_rasterize_fwd: NULL Gaussian pointer");
  cudaStream_t s = as_stream(stream);
  switch (a->channels) {
    case 1: return launch_raster<1>(*a, nullptr, s);
    case 2: return launch_raster<2>(*a, nullptr, s);
    case 3: return launch_raster<3>(*a, nullptr, s);
    default: return launch_raster<4>(*a, nullptr, s);
  }
}

extern "C" int tgs_rasterize_bwd(const TgsRasterBwdArgs* b, void* stream) {
  TGS_CHECK_ARG(b != nullptr, "tgs_rasterize_bwd: args is NULL");
  const int rc = check_raster(&b->fwd);
  if (rc != TGS_OK) return rc;
  const TgsRasterArgs& a = b->fwd;
  if (a.n_cameras == 0 || a.image_width <= 0 || a.image_height <= 0) return TGS_OK;
  TGS_CHECK_ARG(a.tile_offsets && a.render_alphas && a.last_ids && b->v_render_colors &&
                    b->v_render_alphas,
                "tgs_rasterize_bwd: NULL pointer");
  TGS_CHECK_ARG(a.n_isects == 0 || (a.flatten_ids && a.means2d && a.conics && a.colors &&
                                    a.opacities && b->v_means2d && b->v_conics && b->v_colors &&
                                    b->v_opacities),
                "tgs_rasterize_bwd: NULL Gaussian pointer");
  cudaStream_t s = as_stream(stream);
  switch (a.channels) {
    case 1: return launch_raster<1>(a, b, s);
    case 2: return launch_raster<2>(a, b, s);
    case 3: return launch_raster<3>(a, b, s);
    default: return launch_raster<4>(a, b, s);
  }
}
