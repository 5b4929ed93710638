// Scale-safe RMSNorm, forward and backward (the reference's column.RMSNorm, vesper/column.py:159-188,
// and its gradient vesper/kernels/norm_triton.py:47-82).
//
// Forward: one warp per row, the row held in registers (16-byte vector loads when the width
// allows), one read and one write of the row. Backward: one warp per row for dx, the next row's
// raw 16-byte words in flight and two CTAs of eight warps per SM; the gain gradient is summed per
// warp in registers, per CTA in warp order, then across CTAs in CTA order by a second kernel: no
// atomics, the same bits on every run.
#include <initializer_list>
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace vb {
namespace {

constexpr int WARPS = 8;          // warps per CTA (forward rows in flight; backward warps)
constexpr int FWD_ROWS_PER_WARP = 2;   // rows each forward warp loads before computing
constexpr int BWD_WARPS = 8;
constexpr int BWD_ROWS_PER_WARP = 8;
constexpr int BWD_ROWS_PER_CTA = BWD_WARPS * BWD_ROWS_PER_WARP;

// 16-byte vector loads of E = 16/sizeof(T) elements; VPL vectors per lane cover 32*E*VPL channels
template <typename T, int VPL>
__device__ __forceinline__ void load_row(const T* __restrict__ row, int nv, int lane, float (&v)[VPL][16 / sizeof(T)]) {
  constexpr int E = 16 / sizeof(T);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nv) load_vec<T, E>(row + vi * E, v[i]);
    else {
#pragma unroll
      for (int e = 0; e < E; ++e) v[i][e] = 0.f;
    }
  }
}

// the raw 16-byte words of a row (zero past the width) and their conversion to floats
template <int VPL>
__device__ __forceinline__ void load_raw(const void* __restrict__ row, int nv, int lane, uint4 (&r)[VPL]) {
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = lane + 32 * i;
    r[i] = vi < nv ? __ldg(reinterpret_cast<const uint4*>(row) + vi) : make_uint4(0u, 0u, 0u, 0u);
  }
}
// the raw 8-byte words of a row of 8-byte element groups (zero past the width)
template <int VPL>
__device__ __forceinline__ void load_raw(const void* __restrict__ row, int nv, int lane, uint2 (&r)[VPL]) {
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = lane + 32 * i;
    r[i] = vi < nv ? __ldg(reinterpret_cast<const uint2*>(row) + vi) : make_uint2(0u, 0u);
  }
}
// E elements of T from a raw word group (16 or 8 bytes)
template <typename T, int E, typename W>
__device__ __forceinline__ void unpack_e(const W& raw, float (&f)[E]) {
  static_assert(sizeof(W) == E * sizeof(T), "the raw group holds E elements");
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < E; ++i) f[i] = to_f32<T>(e[i]);
}
template <typename T>
__device__ __forceinline__ void unpack(const uint4& raw, float (&f)[16 / sizeof(T)]) {
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < (int)(16 / sizeof(T)); ++i) f[i] = to_f32<T>(e[i]);
}
// the gain at 16-byte vector vi of a row (E = 16 / sizeof(T) floats)
template <int E>
__device__ __forceinline__ void load_gain(const float* __restrict__ w, int vi, float (&g)[E]) {
  const float4* gp = reinterpret_cast<const float4*>(w + vi * E);
#pragma unroll
  for (int q = 0; q < E / 4; ++q) {
    const float4 g4 = __ldg(gp + q);
    g[4 * q] = g4.x; g[4 * q + 1] = g4.y; g[4 * q + 2] = g4.z; g[4 * q + 3] = g4.w;
  }
}

// E consecutive elements of T (E * sizeof(T) = 16 or 8 bytes, aligned to that) as floats, and back
template <typename T, int E>
__device__ __forceinline__ void ld_e(const T* __restrict__ p, float (&out)[E]) {
  if constexpr (E * sizeof(T) == 16) {
    load_vec<T, E>(p, out);
  } else {
    static_assert(E * sizeof(T) == 8, "8- or 16-byte element groups");
    const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < E; ++i) out[i] = to_f32<T>(e[i]);
  }
}
template <typename T, int E>
__device__ __forceinline__ void st_e(T* __restrict__ p, const float (&in)[E]) {
  if constexpr (E * sizeof(T) == 16) {
    store_vec<T, E>(p, in);
  } else {
    static_assert(E * sizeof(T) == 8, "8- or 16-byte element groups");
    uint2 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < E; ++i) e[i] = from_f32<T>(in[i]);
    *reinterpret_cast<uint2*>(p) = raw;
  }
}

// TX: the input's element type, TY: the output's (TX itself, or a 16-bit type for a float32 input,
// the output then rounded once from the float32 result, as a cast of it would round it)
template <typename TX, typename TY, int VPL>
__global__ void __launch_bounds__(WARPS * 32) rms_fwd_vec_kernel(const TX* __restrict__ x,
                                                                 const float* __restrict__ w,
                                                                 TY* __restrict__ y, float* __restrict__ inv,
                                                                 int64_t rows, int width, float floor_,
                                                                 float eps) {
  constexpr int E = 16 / sizeof(TX);
  const int lane = threadIdx.x & 31;
  const int64_t row0 = ((int64_t)blockIdx.x * WARPS + (threadIdx.x >> 5)) * FWD_ROWS_PER_WARP;
  const int nv = width / E;
  float v[FWD_ROWS_PER_WARP][VPL][E];
#pragma unroll
  for (int r = 0; r < FWD_ROWS_PER_WARP; ++r)
    if (row0 + r < rows) load_row<TX, VPL>(x + (row0 + r) * width, nv, lane, v[r]);
#pragma unroll
  for (int r = 0; r < FWD_ROWS_PER_WARP; ++r) {
    const int64_t row = row0 + r;
    if (row >= rows) break;
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i)
#pragma unroll
      for (int e = 0; e < E; ++e) amax = fmaxf(amax, fabsf(v[r][i][e]));
    const float scale = fmaxf(warp_max(amax), floor_);
    // one reciprocal per row, then products: z = x / scale and y = z / rms * g to within a few
    // ulps of the quotients (no decision depends on them), z in [-1, 1] so no product underflows
    const float rscale = 1.0f / scale;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i)
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float z = v[r][i][e] * rscale;
        v[r][i][e] = z;
        ss += z * z;
      }
    const float rms = sqrtf(warp_sum(ss) / (float)width + eps / (scale * scale));
    const float rrms = 1.0f / rms;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nv) {
        float g[E], o[E];
        const float4* gp = reinterpret_cast<const float4*>(w + vi * E);
#pragma unroll
        for (int q = 0; q < E / 4; ++q) {
          float4 g4 = __ldg(gp + q);
          g[4 * q] = g4.x; g[4 * q + 1] = g4.y; g[4 * q + 2] = g4.z; g[4 * q + 3] = g4.w;
        }
#pragma unroll
        for (int e = 0; e < E; ++e) o[e] = v[r][i][e] * (rrms * g[e]);
        st_e<TY, E>(y + row * width + vi * E, o);
      }
    }
    if (lane == 0) inv[row] = 1.0f / (scale * rms);
  }
}

template <typename T, typename TY>
__global__ void __launch_bounds__(WARPS * 32) rms_fwd_kernel(const T* __restrict__ x,
                                                             const float* __restrict__ w,
                                                             TY* __restrict__ y, float* __restrict__ inv,
                                                             int64_t rows, int width, float floor_,
                                                             float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * width;
  TY* yr = y + row * width;
  float amax = 0.f;
  for (int j = lane; j < width; j += 32) amax = fmaxf(amax, fabsf(to_f32<T>(xr[j])));
  const float scale = fmaxf(warp_max(amax), floor_);
  const float rscale = 1.0f / scale;  // as the vector kernel: one reciprocal per row
  float ss = 0.f;
  for (int j = lane; j < width; j += 32) {
    const float z = to_f32<T>(xr[j]) * rscale;
    ss += z * z;
  }
  const float rms = sqrtf(warp_sum(ss) / (float)width + eps / (scale * scale));
  const float rrms = 1.0f / rms;
  for (int j = lane; j < width; j += 32) yr[j] = from_f32<TY>(to_f32<T>(xr[j]) * rscale * (rrms * __ldg(w + j)));
  if (lane == 0) inv[row] = 1.0f / (scale * rms);
}

// Vector backward: each warp walks BWD_ROWS_PER_WARP rows with the next row's x and dy loaded
// while the current one is computed; the gain gradient stays in registers per lane, then is
// summed over the CTA's warps in warp order into partial[blockIdx.x][width].
// TD: the incoming gradient's element type (T itself, or a 16-bit type for a float32 input whose
// output was rounded to it); dx in T.
template <typename T, typename TD, int VPL>
__global__ void __launch_bounds__(BWD_WARPS * 32, 2) rms_bwd_vec_kernel(const T* __restrict__ x,
                                                                        const float* __restrict__ w,
                                                                        const TD* __restrict__ dy,
                                                                        const float* __restrict__ inv,
                                                                        T* __restrict__ dx,
                                                                        float* __restrict__ partial,
                                                                        int64_t rows, int width) {
  constexpr int E = 16 / sizeof(T);
  extern __shared__ float acc_s[];  // [BWD_WARPS][width]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nv = width / E;
  float acc[VPL][E];
#pragma unroll
  for (int i = 0; i < VPL; ++i)
#pragma unroll
    for (int e = 0; e < E; ++e) acc[i][e] = 0.f;
  const int64_t row0 = (int64_t)blockIdx.x * BWD_ROWS_PER_CTA;
  using DRaw = typename std::conditional<E * sizeof(TD) == 16, uint4, uint2>::type;
  uint4 xr[2][VPL];
  DRaw dr[2][VPL];
  int64_t row = row0 + warp;
  if (row < rows) {
    load_raw<VPL>(x + row * width, nv, lane, xr[0]);
    load_raw<VPL>(dy + row * width, nv, lane, dr[0]);
  }
#pragma unroll 2
  for (int k = 0; k < BWD_ROWS_PER_WARP; ++k) {
    const int cur = k & 1;
    row = row0 + (int64_t)k * BWD_WARPS + warp;
    if (row >= rows) break;
    const int64_t nrow = row + BWD_WARPS;
    if (k + 1 < BWD_ROWS_PER_WARP && nrow < rows) {
      load_raw<VPL>(x + nrow * width, nv, lane, xr[cur ^ 1]);
      load_raw<VPL>(dy + nrow * width, nv, lane, dr[cur ^ 1]);
    }
    const float iv = __ldg(inv + row);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nv) {
        float xv[E], dv[E], g[E];
        unpack<T>(xr[cur][i], xv);
        unpack_e<TD, E>(dr[cur][i], dv);
        load_gain<E>(w, vi, g);
#pragma unroll
        for (int e = 0; e < E; ++e) s += dv[e] * g[e] * (xv[e] * iv);
      }
    }
    const float mean = warp_sum(s) / (float)width;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nv) {
        float xv[E], dv[E], g[E], o[E];
        unpack<T>(xr[cur][i], xv);
        unpack_e<TD, E>(dr[cur][i], dv);
        load_gain<E>(w, vi, g);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float xh = xv[e] * iv;
          o[e] = iv * (dv[e] * g[e] - xh * mean);
          acc[i][e] += dv[e] * xh;
        }
        store_vec<T, E>(dx + row * width + vi * E, o);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nv) {
#pragma unroll
      for (int e = 0; e < E; ++e) acc_s[(size_t)warp * width + vi * E + e] = acc[i][e];
    }
  }
  __syncthreads();
  for (int j = threadIdx.x; j < width; j += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < BWD_WARPS; ++q) t += acc_s[(size_t)q * width + j];
    partial[(size_t)blockIdx.x * width + j] = t;
  }
}

// ---- residual add fused with the norm that reads its sum (float32 residual stream) -------------
// Forward: s = x + r (float32: x + float(r), one IEEE addition as torch's mixed add makes it), the
// sum stored, then y = RMSNorm(s) in TY. Backward: d = RMSNorm'(s) dy + ds (the sum's gradient
// from its other reader), dx = d and dr = d rounded to r's dtype (as autograd's add backward
// casts it). One read of the residual stream less than the add followed by the norm, and no
// separate gradient add or cast.
template <typename TR, typename TY, int VPL>
__global__ void __launch_bounds__(WARPS * 32) add_rms_fwd_kernel(const float* __restrict__ x, const TR* __restrict__ r,
                                                                 const float* __restrict__ w, float* __restrict__ sum,
                                                                 TY* __restrict__ y, float* __restrict__ inv,
                                                                 int64_t rows, int width, float floor_, float eps) {
  constexpr int E = 4;  // float32 elements per 16-byte vector
  const int lane = threadIdx.x & 31;
  const int64_t row0 = ((int64_t)blockIdx.x * WARPS + (threadIdx.x >> 5)) * FWD_ROWS_PER_WARP;
  const int nv = width / E;
  float v[FWD_ROWS_PER_WARP][VPL][E];
#pragma unroll
  for (int q = 0; q < FWD_ROWS_PER_WARP; ++q) {
    const int64_t row = row0 + q;
    if (row >= rows) break;
    load_row<float, VPL>(x + row * width, nv, lane, v[q]);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nv) {
        float rv[E];
        ld_e<TR, E>(r + row * width + vi * E, rv);
#pragma unroll
        for (int e = 0; e < E; ++e) v[q][i][e] += rv[e];
        st_e<float, E>(sum + row * width + vi * E, v[q][i]);
      }
    }
  }
#pragma unroll
  for (int q = 0; q < FWD_ROWS_PER_WARP; ++q) {
    const int64_t row = row0 + q;
    if (row >= rows) break;
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i)
#pragma unroll
      for (int e = 0; e < E; ++e) amax = fmaxf(amax, fabsf(v[q][i][e]));
    const float scale = fmaxf(warp_max(amax), floor_);
    const float rscale = 1.0f / scale;  // as rms_fwd_vec_kernel: the same products, the same bits
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i)
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float z = v[q][i][e] * rscale;
        v[q][i][e] = z;
        ss += z * z;
      }
    const float rms = sqrtf(warp_sum(ss) / (float)width + eps / (scale * scale));
    const float rrms = 1.0f / rms;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nv) {
        float g[E], o[E];
        load_gain<E>(w, vi, g);
#pragma unroll
        for (int e = 0; e < E; ++e) o[e] = v[q][i][e] * (rrms * g[e]);
        st_e<TY, E>(y + row * width + vi * E, o);
      }
    }
    if (lane == 0) inv[row] = 1.0f / (scale * rms);
  }
}

template <typename TD, typename TR, int VPL>
__global__ void __launch_bounds__(BWD_WARPS * 32, 2) add_rms_bwd_kernel(const float* __restrict__ x,
                                                                        const float* __restrict__ w,
                                                                        const TD* __restrict__ dy,
                                                                        const float* __restrict__ inv,
                                                                        const float* __restrict__ dsum,
                                                                        float* __restrict__ dx, TR* __restrict__ dr,
                                                                        float* __restrict__ partial, int64_t rows,
                                                                        int width) {
  constexpr int E = 4;
  extern __shared__ float acc_s[];  // [BWD_WARPS][width]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nv = width / E;
  float acc[VPL][E];
#pragma unroll
  for (int i = 0; i < VPL; ++i)
#pragma unroll
    for (int e = 0; e < E; ++e) acc[i][e] = 0.f;
  const int64_t row0 = (int64_t)blockIdx.x * BWD_ROWS_PER_CTA;
  using DRaw = typename std::conditional<E * sizeof(TD) == 16, uint4, uint2>::type;
  uint4 xr[2][VPL];
  DRaw drw[2][VPL];
  int64_t row = row0 + warp;
  if (row < rows) {
    load_raw<VPL>(x + row * width, nv, lane, xr[0]);
    load_raw<VPL>(dy + row * width, nv, lane, drw[0]);
  }
#pragma unroll 2
  for (int k = 0; k < BWD_ROWS_PER_WARP; ++k) {
    const int cur = k & 1;
    row = row0 + (int64_t)k * BWD_WARPS + warp;
    if (row >= rows) break;
    const int64_t nrow = row + BWD_WARPS;
    if (k + 1 < BWD_ROWS_PER_WARP && nrow < rows) {
      load_raw<VPL>(x + nrow * width, nv, lane, xr[cur ^ 1]);
      load_raw<VPL>(dy + nrow * width, nv, lane, drw[cur ^ 1]);
    }
    const float iv = __ldg(inv + row);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nv) {
        float xv[E], dv[E], g[E];
        unpack<float>(xr[cur][i], xv);
        unpack_e<TD, E>(drw[cur][i], dv);
        load_gain<E>(w, vi, g);
#pragma unroll
        for (int e = 0; e < E; ++e) s += dv[e] * g[e] * (xv[e] * iv);
      }
    }
    const float mean = warp_sum(s) / (float)width;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nv) {
        float xv[E], dv[E], g[E], o[E];
        unpack<float>(xr[cur][i], xv);
        unpack_e<TD, E>(drw[cur][i], dv);
        load_gain<E>(w, vi, g);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float xh = xv[e] * iv;
          o[e] = iv * (dv[e] * g[e] - xh * mean);
          acc[i][e] += dv[e] * xh;
        }
        if (dsum != nullptr) {
          float ds[E];
          ld_e<float, E>(dsum + row * width + vi * E, ds);
#pragma unroll
          for (int e = 0; e < E; ++e) o[e] += ds[e];
        }
        st_e<float, E>(dx + row * width + vi * E, o);
        if (dr != nullptr) st_e<TR, E>(dr + row * width + vi * E, o);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nv) {
#pragma unroll
      for (int e = 0; e < E; ++e) acc_s[(size_t)warp * width + vi * E + e] = acc[i][e];
    }
  }
  __syncthreads();
  for (int j = threadIdx.x; j < width; j += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < BWD_WARPS; ++q) t += acc_s[(size_t)q * width + j];
    partial[(size_t)blockIdx.x * width + j] = t;
  }
}

// Scalar backward for widths without a 16-byte vector path.
template <typename T, typename TD>
__global__ void __launch_bounds__(BWD_WARPS * 32) rms_bwd_kernel(const T* __restrict__ x,
                                                                 const float* __restrict__ w,
                                                                 const TD* __restrict__ dy,
                                                                 const float* __restrict__ inv,
                                                                 T* __restrict__ dx,
                                                                 float* __restrict__ partial,
                                                                 int64_t rows, int width) {
  extern __shared__ float acc[];  // [BWD_WARPS][width]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* mine = acc + (size_t)warp * width;
  for (int j = lane; j < width; j += 32) mine[j] = 0.f;
  const int64_t row0 = (int64_t)blockIdx.x * BWD_ROWS_PER_CTA;
  for (int k = 0; k < BWD_ROWS_PER_WARP; ++k) {
    const int64_t row = row0 + (int64_t)k * BWD_WARPS + warp;
    if (row >= rows) break;
    const T* xr = x + row * width;
    const TD* dr = dy + row * width;
    const float iv = __ldg(inv + row);
    float s = 0.f;
    for (int j = lane; j < width; j += 32) {
      const float xh = to_f32<T>(xr[j]) * iv;
      s += to_f32<TD>(dr[j]) * __ldg(w + j) * xh;
    }
    const float mean = warp_sum(s) / (float)width;
    T* out = dx + row * width;
    for (int j = lane; j < width; j += 32) {
      const float xh = to_f32<T>(xr[j]) * iv;
      const float d = to_f32<TD>(dr[j]);
      out[j] = from_f32<T>(iv * (d * __ldg(w + j) - xh * mean));
      mine[j] += d * xh;
    }
  }
  __syncthreads();
  for (int j = threadIdx.x; j < width; j += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < BWD_WARPS; ++q) t += acc[(size_t)q * width + j];
    partial[(size_t)blockIdx.x * width + j] = t;
  }
}

// out[j] = sum over p of partial[p][j]: lane <-> column; warp w of 32 sums parts w, w+32, ... into
// four interleaved accumulators (four loads in flight), then the 32 warp sums are added in warp
// order (a fixed tree: the same bits on every run)
constexpr int CS_WARPS = 32;
__global__ void __launch_bounds__(CS_WARPS * 32) column_sum_kernel(const float* __restrict__ partial,
                                                                   float* __restrict__ out, int parts, int width) {
  __shared__ float acc[CS_WARPS][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int j = blockIdx.x * 32 + lane;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  if (j < width) {
    const float* p = partial + j;
    int r = warp;
    for (; r + 3 * CS_WARPS < parts; r += 4 * CS_WARPS) {
      a0 += __ldg(p + (size_t)r * width);
      a1 += __ldg(p + (size_t)(r + CS_WARPS) * width);
      a2 += __ldg(p + (size_t)(r + 2 * CS_WARPS) * width);
      a3 += __ldg(p + (size_t)(r + 3 * CS_WARPS) * width);
    }
    for (; r < parts; r += CS_WARPS) a0 += __ldg(p + (size_t)r * width);
  }
  acc[warp][lane] = (a0 + a1) + (a2 + a3);
  __syncthreads();
  if (warp == 0 && j < width) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < CS_WARPS; ++w) s += acc[w][lane];
    out[j] = s;
  }
}

int bwd_ctas(int64_t rows) { return (int)((rows + BWD_ROWS_PER_CTA - 1) / BWD_ROWS_PER_CTA); }

// vectors per lane of the vector paths: 16-byte vectors of E elements, 32 lanes
template <typename T>
int vpl_for(int width) {
  constexpr int E = 16 / sizeof(T);
  if (width % E) return 0;
  const int nv = width / E;
  for (int v : {1, 2, 4, 8})
    if (nv <= 32 * v) return v;
  return 0;
}

#define VB_VPL_DISPATCH(vpl, VPL, ...)                               \
  [&]() -> int {                                                     \
    switch (vpl) {                                                   \
      case 1: { constexpr int VPL = 1; return __VA_ARGS__(); }       \
      case 2: { constexpr int VPL = 2; return __VA_ARGS__(); }       \
      case 4: { constexpr int VPL = 4; return __VA_ARGS__(); }       \
      default: { constexpr int VPL = 8; return __VA_ARGS__(); }      \
    }                                                                \
  }()

}  // namespace

// Sums `parts` rows of `partial [parts, width]` in row order into out[width].
int column_sum(const float* partial, float* out, int parts, int width, cudaStream_t st) {
  column_sum_kernel<<<(width + 31) / 32, CS_WARPS * 32, 0, st>>>(partial, out, parts, width);
  VB_LAUNCH_CHECK("column_sum");
  return VB_OK;
}

// Dispatches (input, other) element types: the same type, or a float32 input with a bf16 or f16
// other side (the output of the forward, the incoming gradient of the backward).
#define VB_DISPATCH_PAIR(xcode, ocode, TX, TO, ...)                                                      \
  [&]() -> int {                                                                                          \
    if ((xcode) == (ocode)) return VB_DISPATCH_DTYPE(xcode, TX, [&]() -> int { using TO = TX; return __VA_ARGS__(); }); \
    if ((xcode) == VB_F32 && (ocode) == VB_BF16) { using TX = float; using TO = __nv_bfloat16; return __VA_ARGS__(); } \
    if ((xcode) == VB_F32 && (ocode) == VB_F16) { using TX = float; using TO = __half; return __VA_ARGS__(); }        \
    ::vb::set_error("rms_norm: element types %d and %d: the same type, or float32 with bf16 or f16", (int)(xcode), \
                    (int)(ocode));                                                                       \
    return VB_ERR_INVALID;                                                                                \
  }()

// y (in TY) and inv (vector path when the width allows)
int launch_fwd(const void* x, const float* weight, void* y, float* inv, int64_t rows, int width, float floor_,
               float eps, int xcode, int ycode, cudaStream_t st) {
  return VB_DISPATCH_PAIR(xcode, ycode, T, TY, [&]() -> int {
    const int vpl = vpl_for<T>(width);
    if (vpl && aligned16(x) && aligned16(y) && aligned16(weight)) {
      const int64_t per = (int64_t)WARPS * FWD_ROWS_PER_WARP;
      const int ctas = (int)((rows + per - 1) / per);
      VB_VPL_DISPATCH(vpl, VPL, [&]() -> int {
        rms_fwd_vec_kernel<T, TY, VPL><<<ctas, WARPS * 32, 0, st>>>((const T*)x, weight, (TY*)y, inv, rows,
                                                                    width, floor_, eps);
        return 0;
      });
    } else {
      const int ctas = (int)((rows + WARPS - 1) / WARPS);
      rms_fwd_kernel<T, TY><<<ctas, WARPS * 32, 0, st>>>((const T*)x, weight, (TY*)y, inv, rows, width,
                                                         floor_, eps);
    }
    VB_LAUNCH_CHECK("rms_norm_fwd");
    return VB_OK;
  });
}

// dx (in x's type) and the per-CTA gain partials (vector path when the width allows), then the
// fixed-order sum
int launch_bwd(const void* x, const float* weight, const void* dy, const float* inv, void* dx, float* dweight,
               float* partial, int64_t rows, int width, int xcode, int dycode, cudaStream_t st) {
  const int ctas = bwd_ctas(rows);
  const size_t smem = sizeof(float) * BWD_WARPS * width;
  return VB_DISPATCH_PAIR(xcode, dycode, T, TD, [&]() -> int {
    const int vpl = vpl_for<T>(width);
    if (vpl && aligned16(x) && aligned16(dy) && aligned16(dx)) {
      VB_VPL_DISPATCH(vpl, VPL, [&]() -> int {
        if (smem > 48 * 1024)
          cudaFuncSetAttribute(rms_bwd_vec_kernel<T, TD, VPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        rms_bwd_vec_kernel<T, TD, VPL><<<ctas, BWD_WARPS * 32, smem, st>>>((const T*)x, weight, (const TD*)dy,
                                                                           inv, (T*)dx, partial, rows, width);
        return 0;
      });
    } else {
      if (smem > 48 * 1024)
        cudaFuncSetAttribute(rms_bwd_kernel<T, TD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      rms_bwd_kernel<T, TD><<<ctas, BWD_WARPS * 32, smem, st>>>((const T*)x, weight, (const TD*)dy, inv, (T*)dx,
                                                                partial, rows, width);
    }
    VB_LAUNCH_CHECK("rms_norm_bwd");
    return column_sum(partial, dweight, ctas, width, st);
  });
}

// the vectors per lane of the fused add + norm (float32 residual stream), 0 where the width or an
// address does not allow the 16-byte path
int add_vpl(int width, std::initializer_list<const void*> ptrs) {
  for (const void* p : ptrs)
    if (p != nullptr && !aligned16(p)) return 0;
  return vpl_for<float>(width);
}

#define VB_DISPATCH_16(code, T, ...)                                                                 \
  [&]() -> int {                                                                                     \
    switch (code) {                                                                                  \
      case VB_F32: { using T = float; return __VA_ARGS__(); }                                        \
      case VB_BF16: { using T = __nv_bfloat16; return __VA_ARGS__(); }                               \
      case VB_F16: { using T = __half; return __VA_ARGS__(); }                                       \
      default: ::vb::set_error("add_rms_norm: unsupported dtype code %d", (int)(code)); return VB_ERR_INVALID; \
    }                                                                                                \
  }()

}  // namespace vb

using namespace vb;

extern "C" int vb_add_rms_norm_fwd(const float* x, const void* r, const float* weight, float* sum, void* y,
                                   float* inv, int64_t rows, int width, float floor_, float eps, int r_dtype,
                                   int y_dtype, void* stream) {
  VB_REQUIRE(rows >= 0 && width > 0, "add_rms_norm_fwd: bad shape rows=%lld width=%d", (long long)rows, width);
  if (rows == 0) return VB_OK;
  VB_REQUIRE(x && r && weight && sum && y && inv, "add_rms_norm_fwd: null pointer");
  const int vpl = add_vpl(width, {x, r, weight, sum, y});
  VB_REQUIRE(vpl != 0, "add_rms_norm_fwd: width %d must be a multiple of 4 up to 1024 and every tensor 16-byte "
             "aligned", width);
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t per = (int64_t)WARPS * FWD_ROWS_PER_WARP;
  const int ctas = (int)((rows + per - 1) / per);
  return VB_DISPATCH_16(r_dtype, TR, [&]() -> int {
    return VB_DISPATCH_16(y_dtype, TY, [&]() -> int {
      VB_VPL_DISPATCH(vpl, VPL, [&]() -> int {
        add_rms_fwd_kernel<TR, TY, VPL><<<ctas, WARPS * 32, 0, st>>>(x, (const TR*)r, weight, sum, (TY*)y, inv,
                                                                     rows, width, floor_, eps);
        return 0;
      });
      VB_LAUNCH_CHECK("add_rms_norm_fwd");
      return VB_OK;
    });
  });
}

extern "C" int vb_add_rms_norm_bwd(const float* sum, const float* weight, const void* dy, const float* inv,
                                   const float* dsum, float* dx, void* dr, float* dweight, void* workspace,
                                   int64_t rows, int width, int dy_dtype, int r_dtype, void* stream) {
  VB_REQUIRE(rows >= 0 && width > 0, "add_rms_norm_bwd: bad shape rows=%lld width=%d", (long long)rows, width);
  VB_REQUIRE(width <= 4096, "add_rms_norm_bwd: width %d exceeds the kernel's 4096", width);
  cudaStream_t st = (cudaStream_t)stream;
  if (rows == 0) {
    VB_CUDA_CHECK(cudaMemsetAsync(dweight, 0, sizeof(float) * width, st), "add_rms_norm_bwd");
    return VB_OK;
  }
  VB_REQUIRE(sum && weight && dy && inv && dx && dweight && workspace, "add_rms_norm_bwd: null pointer");
  const int vpl = add_vpl(width, {sum, weight, dy, dsum, dx, dr});
  VB_REQUIRE(vpl != 0, "add_rms_norm_bwd: width %d must be a multiple of 4 up to 1024 and every tensor 16-byte "
             "aligned", width);
  const int ctas = bwd_ctas(rows);
  const size_t smem = sizeof(float) * BWD_WARPS * width;
  float* partial = (float*)workspace;
  return VB_DISPATCH_16(dy_dtype, TD, [&]() -> int {
    return VB_DISPATCH_16(r_dtype, TR, [&]() -> int {
      VB_VPL_DISPATCH(vpl, VPL, [&]() -> int {
        if (smem > 48 * 1024)
          cudaFuncSetAttribute(add_rms_bwd_kernel<TD, TR, VPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        add_rms_bwd_kernel<TD, TR, VPL><<<ctas, BWD_WARPS * 32, smem, st>>>(sum, weight, (const TD*)dy, inv, dsum,
                                                                            dx, (TR*)dr, partial, rows, width);
        return 0;
      });
      VB_LAUNCH_CHECK("add_rms_norm_bwd");
      return column_sum(partial, dweight, ctas, width, st);
    });
  });
}

extern "C" int vb_rms_norm_fwd(const void* x, const float* weight, void* y, float* inv, int64_t rows,
                               int width, float floor_, float eps, int dtype, void* stream) {
  VB_REQUIRE(rows >= 0 && width > 0, "rms_norm_fwd: bad shape rows=%lld width=%d", (long long)rows, width);
  if (rows == 0) return VB_OK;
  VB_REQUIRE(x && weight && y && inv, "rms_norm_fwd: null pointer");
  return launch_fwd(x, weight, y, inv, rows, width, floor_, eps, dtype, dtype, (cudaStream_t)stream);
}

extern "C" int vb_rms_norm_fwd_cast(const void* x, const float* weight, void* y, float* inv, int64_t rows,
                                    int width, float floor_, float eps, int x_dtype, int y_dtype, void* stream) {
  VB_REQUIRE(rows >= 0 && width > 0, "rms_norm_fwd_cast: bad shape rows=%lld width=%d", (long long)rows, width);
  if (rows == 0) return VB_OK;
  VB_REQUIRE(x && weight && y && inv, "rms_norm_fwd_cast: null pointer");
  return launch_fwd(x, weight, y, inv, rows, width, floor_, eps, x_dtype, y_dtype, (cudaStream_t)stream);
}

extern "C" size_t vb_rms_norm_bwd_workspace(int64_t rows, int width) {
  return (size_t)(rows > 0 ? bwd_ctas(rows) : 1) * (size_t)width * sizeof(float);
}

extern "C" int vb_rms_norm_bwd(const void* x, const float* weight, const void* dy, const float* inv,
                               void* dx, float* dweight, void* workspace, int64_t rows, int width,
                               int dtype, void* stream) {
  VB_REQUIRE(rows >= 0 && width > 0, "rms_norm_bwd: bad shape rows=%lld width=%d", (long long)rows, width);
  VB_REQUIRE(width <= 4096, "rms_norm_bwd: width %d exceeds the kernel's 4096", width);
  cudaStream_t st = (cudaStream_t)stream;
  if (rows == 0) {
    VB_CUDA_CHECK(cudaMemsetAsync(dweight, 0, sizeof(float) * width, st), "rms_norm_bwd");
    return VB_OK;
  }
  VB_REQUIRE(x && weight && dy && inv && dx && dweight && workspace, "rms_norm_bwd: null pointer");
  return launch_bwd(x, weight, dy, inv, dx, dweight, (float*)workspace, rows, width, dtype, dtype, st);
}

extern "C" int vb_rms_norm_bwd_cast(const void* x, const float* weight, const void* dy, const float* inv,
                                    void* dx, float* dweight, void* workspace, int64_t rows, int width,
                                    int x_dtype, int dy_dtype, void* stream) {
  VB_REQUIRE(rows >= 0 && width > 0, "rms_norm_bwd_cast: bad shape rows=%lld width=%d", (long long)rows, width);
  VB_REQUIRE(width <= 4096, "rms_norm_bwd_cast: width %d exceeds the kernel's 4096", width);
  cudaStream_t st = (cudaStream_t)stream;
  if (rows == 0) {
    VB_CUDA_CHECK(cudaMemsetAsync(dweight, 0, sizeof(float) * width, st), "rms_norm_bwd_cast");
    return VB_OK;
  }
  VB_REQUIRE(x && weight && dy && inv && dx && dweight && workspace, "rms_norm_bwd_cast: null pointer");
  return launch_bwd(x, weight, dy, inv, dx, dweight, (float*)workspace, rows, width, x_dtype, dy_dtype, st);
}

// ---- RMSNorm backward without allocation ------------------------------------------------------
// For callers that cannot call cudaMalloc or take memory from an allocator (a plugin host whose
// device memory is planned up front, a real-time loop that must not allocate, code that runs
// where an allocation would break a graph capture or a fixed memory plan): the gain gradient's
// per-CTA partial sums live in this file-scope array instead of a caller-provided workspace.
// Every GPU that loads the library holds the 4 MiB until the process exits.
namespace vb {
namespace {
constexpr size_t NOALLOC_PARTIAL_FLOATS = size_t(1) << 20;  // 4 MiB of float partial sums
static __device__ __align__(256) float g_rms_bwd_scratch[NOALLOC_PARTIAL_FLOATS];
constexpr int NOALLOC_MAX_DEVICES = 64;
std::mutex g_scratch_mutex;
float* g_scratch_device[NOALLOC_MAX_DEVICES] = {};

// The array's device address on the current device, looked up once per device: in host code
// the array's name is only a stand-in, not a device address.
int scratch_on_current_device(float** out) {
  int dev = -1;
  VB_CUDA_CHECK(cudaGetDevice(&dev), "rms_norm_bwd_noalloc: cudaGetDevice");
  VB_REQUIRE(dev >= 0 && dev < NOALLOC_MAX_DEVICES, "rms_norm_bwd_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_device[dev] == nullptr) {
    void* p = nullptr;
    VB_CUDA_CHECK(cudaGetSymbolAddress(&p, g_rms_bwd_scratch), "rms_norm_bwd_noalloc: cudaGetSymbolAddress");
    g_scratch_device[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_device[dev];
  return VB_OK;
}
}  // namespace
}  // namespace vb

extern "C" int vb_rms_norm_bwd_noalloc(const void* x, const float* weight, const void* dy,
                                       const float* inv, void* dx, float* dweight, int64_t rows,
                                       int width, int dtype, void* stream) {
  VB_REQUIRE(rows >= 0 && width > 0, "rms_norm_bwd_noalloc: bad shape rows=%lld width=%d", (long long)rows, width);
  VB_REQUIRE(width <= 4096, "rms_norm_bwd_noalloc: width %d exceeds the kernel's 4096", width);
  const int ctas = rows > 0 ? bwd_ctas(rows) : 0;
  VB_REQUIRE((size_t)ctas * (size_t)width <= NOALLOC_PARTIAL_FLOATS,
             "rms_norm_bwd_noalloc: %lld rows of width %d need %zu partial sums, above the fixed "
             "scratch of %zu floats (at this width at most %lld rows); use vb_rms_norm_bwd with a "
             "workspace",
             (long long)rows, width, (size_t)ctas * (size_t)width, NOALLOC_PARTIAL_FLOATS,
             (long long)(NOALLOC_PARTIAL_FLOATS / (size_t)width) * BWD_ROWS_PER_CTA);
  cudaStream_t st = (cudaStream_t)stream;
  if (rows == 0) {
    VB_CUDA_CHECK(cudaMemsetAsync(dweight, 0, sizeof(float) * width, st), "rms_norm_bwd_noalloc");
    return VB_OK;
  }
  VB_REQUIRE(x && weight && dy && inv && dx && dweight, "rms_norm_bwd_noalloc: null pointer");
  float* partial = nullptr;
  int rc = scratch_on_current_device(&partial);
  if (rc) return rc;
  // every partial row this call reads is written by this call first: nothing needs clearing
  return launch_bwd(x, weight, dy, inv, dx, dweight, partial, rows, width, dtype, dtype, st);
}
