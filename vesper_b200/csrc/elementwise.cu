// Elementwise sublayer ops of the column, fused: the squared ReLU of the FFN and the rotary
// embedding of the attention, forward and backward, each one pass over HBM with 16-byte vectors.
//
// Both reproduce the reference's op sequence in the activation dtype exactly (every product,
// sum and difference rounded to the dtype where the reference's separate torch ops round), so
// the fused results equal the unfused ones bit for bit:
//   relu_square (vesper/ffn.py:44-56, h = relu(z), h * h):  y = rnd(h * h);
//       dz = z > 0 ? rnd(2 rnd(dy h)) : 0      (the product's two operand gradients, summed)
//   rotary (vesper/attention.py:178-217): pairs (x1, x2) = (x[2j], x[2j+1]),
//       c = rnd(float(cos(pos w_j))), s = rnd(float(sin(pos w_j))), phase and cosine in float64,
//       y1 = rnd(rnd(x1 c) - rnd(x2 s)),  y2 = rnd(rnd(x1 s) + rnd(x2 c));
//       dx1 = rnd(rnd(g1 c) + rnd(g2 s)),   dx2 = rnd(rnd(g2 c) + rnd(-g1 s)).
#include "common.cuh"

namespace vb {
namespace {

template <typename T> __device__ __forceinline__ float rnd(float v) { return to_f32<T>(from_f32<T>(v)); }
// a float64 value cast to T the way torch casts it: to float first, then to T
template <typename T> __device__ __forceinline__ float rnd64(double v) { return rnd<T>((float)v); }
// a product that is never contracted into a fused multiply-add (each of the reference's products
// is its own op, rounded before the sum)
__device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }

template <typename T>
__global__ void relu_square_fwd_kernel(const T* __restrict__ z, T* __restrict__ y, int64_t n) {
  constexpr int V = 16 / sizeof(T);
  const int64_t nv = n / V;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += stride) {
    float a[V], r[V];
    load_vec<T, V>(z + i * V, a);
#pragma unroll
    for (int e = 0; e < V; ++e) {
      const float h = a[e] > 0.f || a[e] != a[e] ? a[e] : 0.f;  // relu, NaN propagated as torch does
      r[e] = mul(h, h);
    }
    store_vec<T, V>(y + i * V, r);
  }
  for (int64_t i = nv * V + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float zz = to_f32<T>(z[i]);
    const float h = zz > 0.f || zz != zz ? zz : 0.f;
    y[i] = from_f32<T>(mul(h, h));
  }
}

template <typename T>
__device__ __forceinline__ float relu_square_grad(float zz, float g) {
  if (!(zz > 0.f || zz != zz)) return 0.f;  // the ReLU's gradient passes where its output is not <= 0
  const float p = rnd<T>(mul(g, zz));
  return p + p;
}

template <typename T>
__global__ void relu_square_bwd_kernel(const T* __restrict__ z, const T* __restrict__ dy, T* __restrict__ dz,
                                       int64_t n) {
  constexpr int V = 16 / sizeof(T);
  const int64_t nv = n / V;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += stride) {
    float a[V], g[V], r[V];
    load_vec<T, V>(z + i * V, a);
    load_vec<T, V>(dy + i * V, g);
#pragma unroll
    for (int e = 0; e < V; ++e) r[e] = relu_square_grad<T>(a[e], g[e]);
    store_vec<T, V>(dz + i * V, r);
  }
  for (int64_t i = nv * V + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    dz[i] = from_f32<T>(relu_square_grad<T>(to_f32<T>(z[i]), to_f32<T>(dy[i])));
}

// one thread per (token, pair group of 4 pairs = 8 elements, run of `hpt` heads): the group's four
// phases and their cosines and sines (float64, the costly part) are formed once and turn that
// group of each head of the run (every head when there are tokens enough to fill the GPU, one
// head per thread for the few tokens of a decode step, where latency rules)
template <typename T, bool BWD>
__global__ void rotary_kernel(const T* __restrict__ x, const int64_t* __restrict__ pos,
                              const double* __restrict__ inv_freq, T* __restrict__ y, int64_t tokens, int heads,
                              int dk, int hpt) {
  const int groups = dk / 8;  // 8 elements (4 pairs) per group
  const int runs = (heads + hpt - 1) / hpt;
  const int64_t total = tokens * groups * runs;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < total; w += stride) {
    const int64_t tr = w / groups;  // (token, run); the group varies fastest: coalesced rows
    const int gi = (int)(w - tr * groups);
    const int64_t tok = tr / runs;
    const int h0 = (int)(tr - tok * runs) * hpt, h1 = min(heads, h0 + hpt);
    const double p = (double)pos[tok];
    float c[4], s[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const double ang = p * inv_freq[gi * 4 + q];
      c[q] = rnd64<T>(cos(ang));
      s[q] = rnd64<T>(sin(ang));
    }
    for (int hd = h0; hd < h1; ++hd) {
      const int64_t off = (tok * heads + hd) * dk + gi * 8;
      float a[8], r[8];
      load_vec<T, 8>(x + off, a);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float x1 = a[2 * q], x2 = a[2 * q + 1];
        if constexpr (!BWD) {
          r[2 * q] = rnd<T>(mul(x1, c[q])) - rnd<T>(mul(x2, s[q]));
          r[2 * q + 1] = rnd<T>(mul(x1, s[q])) + rnd<T>(mul(x2, c[q]));
        } else {  // x1, x2 hold the output gradient pair (g1, g2)
          r[2 * q] = rnd<T>(mul(x1, c[q])) + rnd<T>(mul(x2, s[q]));
          r[2 * q + 1] = rnd<T>(mul(x2, c[q])) + rnd<T>(mul(-x1, s[q]));
        }
      }
      store_vec<T, 8>(y + off, r);
    }
  }
}

unsigned grid_for(int64_t items) {
  const int64_t blocks = (items + 255) / 256;
  return (unsigned)(blocks < 148 * 32 ? (blocks > 0 ? blocks : 1) : 148 * 32);
}

// The residual add at the end of a column over the float32 residual stream, with the loop's
// zeroing of halted rows fused in: out = keep[row] ? x + float(f) : 0 (one IEEE float32 addition,
// as torch's mixed-dtype add makes it); the backward writes dx = keep ? g : 0 and the same rounded
// to f's dtype (autograd's add backward casts it). keep NULL keeps every row. W: the row width.
constexpr int RA_WARPS = 8;  // rows per CTA of the residual kernels: a warp per row
template <typename TF>
__device__ __forceinline__ void ld4(const TF* __restrict__ p, float (&v)[4]) {
  if constexpr (sizeof(TF) == 4) {
    load_vec<float, 4>(reinterpret_cast<const float*>(p), v);
  } else {
    const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
    const TF* e = reinterpret_cast<const TF*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = to_f32<TF>(e[j]);
  }
}
template <typename TF>
__device__ __forceinline__ void st4(TF* __restrict__ p, const float (&v)[4]) {
  if constexpr (sizeof(TF) == 4) {
    store_vec<float, 4>(reinterpret_cast<float*>(p), v);
  } else {
    uint2 raw;
    TF* e = reinterpret_cast<TF*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) e[j] = from_f32<TF>(v[j]);
    *reinterpret_cast<uint2*>(p) = raw;
  }
}

template <typename TF>
__global__ void __launch_bounds__(RA_WARPS * 32) residual_add_kernel(const float* __restrict__ x,
                                                                     const TF* __restrict__ f,
                                                                     const uint8_t* __restrict__ keep,
                                                                     float* __restrict__ out, int64_t rows, int W) {
  const int64_t row = (int64_t)blockIdx.x * RA_WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  const bool k = keep == nullptr || keep[row] != 0;
  const int64_t base = row * W;
  for (int c = (threadIdx.x & 31) * 4; c < W; c += 128) {
    float a[4] = {0.f, 0.f, 0.f, 0.f};
    if (k) {  // a halted row is zero: its inputs are not read
      float b[4];
      load_vec<float, 4>(x + base + c, a);
      ld4<TF>(f + base + c, b);
#pragma unroll
      for (int j = 0; j < 4; ++j) a[j] += b[j];
    }
    store_vec<float, 4>(out + base + c, a);
  }
}

template <typename TF>
__global__ void __launch_bounds__(RA_WARPS * 32) residual_add_bwd_kernel(const float* __restrict__ g,
                                                                         const uint8_t* __restrict__ keep,
                                                                         float* __restrict__ dx, TF* __restrict__ df,
                                                                         int64_t rows, int W) {
  const int64_t row = (int64_t)blockIdx.x * RA_WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  const bool k = keep == nullptr || keep[row] != 0;
  const int64_t base = row * W;
  for (int c = (threadIdx.x & 31) * 4; c < W; c += 128) {
    float a[4];
    if (k) {
      load_vec<float, 4>(g + base + c, a);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) a[j] = 0.f;
    }
    if (dx != nullptr) store_vec<float, 4>(dx + base + c, a);
    if (df != nullptr) st4<TF>(df + base + c, a);
  }
}

}  // namespace
}  // namespace vb

using namespace vb;

extern "C" int vb_relu_square_fwd(const void* z, void* y, long long n, int dtype, void* stream) {
  VB_REQUIRE(n >= 0, "relu_square_fwd: negative size");
  if (n == 0) return VB_OK;
  VB_REQUIRE(z && y && aligned16(z) && aligned16(y), "relu_square_fwd: null or unaligned tensor");
  VB_REQUIRE(dtype == VB_F32 || dtype == VB_BF16 || dtype == VB_F16, "relu_square_fwd: bad dtype %d", dtype);
  return VB_DISPATCH_DTYPE(dtype, T, [&]() -> int {
    relu_square_fwd_kernel<T><<<grid_for(n / (16 / sizeof(T)) + 1), 256, 0, (cudaStream_t)stream>>>((const T*)z, (T*)y, n);
    VB_LAUNCH_CHECK("relu_square_fwd");
    return VB_OK;
  });
}

extern "C" int vb_relu_square_bwd(const void* z, const void* dy, void* dz, long long n, int dtype, void* stream) {
  VB_REQUIRE(n >= 0, "relu_square_bwd: negative size");
  if (n == 0) return VB_OK;
  VB_REQUIRE(z && dy && dz && aligned16(z) && aligned16(dy) && aligned16(dz), "relu_square_bwd: null or unaligned tensor");
  VB_REQUIRE(dtype == VB_F32 || dtype == VB_BF16 || dtype == VB_F16, "relu_square_bwd: bad dtype %d", dtype);
  return VB_DISPATCH_DTYPE(dtype, T, [&]() -> int {
    relu_square_bwd_kernel<T><<<grid_for(n / (16 / sizeof(T)) + 1), 256, 0, (cudaStream_t)stream>>>(
        (const T*)z, (const T*)dy, (T*)dz, n);
    VB_LAUNCH_CHECK("relu_square_bwd");
    return VB_OK;
  });
}

extern "C" int vb_rotary(const void* x, const long long* pos, const double* inv_freq, void* y, long long tokens,
                         int heads, int dk, int backward, int dtype, void* stream) {
  VB_REQUIRE(tokens >= 0 && heads > 0 && dk > 0, "rotary: bad shape tokens=%lld heads=%d dk=%d", tokens, heads, dk);
  VB_REQUIRE(dk % 8 == 0, "rotary: head dimension %d must be a multiple of 8", dk);
  if (tokens == 0) return VB_OK;
  VB_REQUIRE(x && pos && inv_freq && y && aligned16(x) && aligned16(y), "rotary: null or unaligned tensor");
  VB_REQUIRE(dtype == VB_F32 || dtype == VB_BF16 || dtype == VB_F16, "rotary: bad dtype %d", dtype);
  // every head of a token per thread once there are threads enough for two waves of 256 per SM
  const int hpt = tokens * (dk / 8) >= 148 * 256 * 2 ? heads : 1;
  const int64_t items = tokens * (dk / 8) * ((heads + hpt - 1) / hpt);
  return VB_DISPATCH_DTYPE(dtype, T, [&]() -> int {
    if (backward)
      rotary_kernel<T, true><<<grid_for(items), 256, 0, (cudaStream_t)stream>>>(
          (const T*)x, (const int64_t*)pos, inv_freq, (T*)y, tokens, heads, dk, hpt);
    else
      rotary_kernel<T, false><<<grid_for(items), 256, 0, (cudaStream_t)stream>>>(
          (const T*)x, (const int64_t*)pos, inv_freq, (T*)y, tokens, heads, dk, hpt);
    VB_LAUNCH_CHECK("rotary");
    return VB_OK;
  });
}

extern "C" int vb_residual_add(const float* x, const void* f, const unsigned char* keep, float* out, long long rows,
                               int width, int f_dtype, void* stream) {
  VB_REQUIRE(rows >= 0 && width > 0 && width % 4 == 0, "residual_add: bad shape rows=%lld width=%d (a multiple of 4)",
             rows, width);
  if (rows == 0) return VB_OK;
  VB_REQUIRE(x && f && out && aligned16(x) && aligned16(f) && aligned16(out), "residual_add: null or unaligned tensor");
  const unsigned ctas = (unsigned)((rows + RA_WARPS - 1) / RA_WARPS);
  return VB_DISPATCH_DTYPE(f_dtype, T, [&]() -> int {
    residual_add_kernel<T><<<ctas, RA_WARPS * 32, 0, (cudaStream_t)stream>>>(x, (const T*)f, keep, out, rows, width);
    VB_LAUNCH_CHECK("residual_add");
    return VB_OK;
  });
}

extern "C" int vb_residual_add_bwd(const float* g, const unsigned char* keep, float* dx, void* df, long long rows,
                                   int width, int f_dtype, void* stream) {
  VB_REQUIRE(rows >= 0 && width > 0 && width % 4 == 0,
             "residual_add_bwd: bad shape rows=%lld width=%d (a multiple of 4)", rows, width);
  if (rows == 0) return VB_OK;
  VB_REQUIRE(g && aligned16(g) && (!dx || aligned16(dx)) && (!df || aligned16(df)),
             "residual_add_bwd: null or unaligned tensor");
  const unsigned ctas = (unsigned)((rows + RA_WARPS - 1) / RA_WARPS);
  return VB_DISPATCH_DTYPE(f_dtype, T, [&]() -> int {
    residual_add_bwd_kernel<T><<<ctas, RA_WARPS * 32, 0, (cudaStream_t)stream>>>(g, keep, dx, (T*)df, rows, width);
    VB_LAUNCH_CHECK("residual_add_bwd");
    return VB_OK;
  });
}
