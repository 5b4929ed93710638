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

// one thread per (token, pair group of 4 pairs = 8 elements) across all heads of the token
template <typename T, bool BWD>
__global__ void rotary_kernel(const T* __restrict__ x, const int64_t* __restrict__ pos,
                              const double* __restrict__ inv_freq, T* __restrict__ y, int64_t tokens, int heads,
                              int dk) {
  const int groups = dk / 8;  // 8 elements (4 pairs) per group
  const int64_t per_token = (int64_t)heads * groups;
  const int64_t total = tokens * per_token;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < total; w += stride) {
    const int64_t tok = w / per_token;
    const int rem = (int)(w % per_token);
    const int hd = rem / groups, gi = rem % groups;
    const double p = (double)pos[tok];
    const T* src = x + (tok * heads + hd) * dk + gi * 8;
    float a[8], r[8];
    load_vec<T, 8>(src, a);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const double ang = p * inv_freq[gi * 4 + q];
      const float c = rnd64<T>(cos(ang)), s = rnd64<T>(sin(ang));
      const float x1 = a[2 * q], x2 = a[2 * q + 1];
      if constexpr (!BWD) {
        r[2 * q] = rnd<T>(mul(x1, c)) - rnd<T>(mul(x2, s));
        r[2 * q + 1] = rnd<T>(mul(x1, s)) + rnd<T>(mul(x2, c));
      } else {  // x1, x2 hold the output gradient pair (g1, g2)
        r[2 * q] = rnd<T>(mul(x1, c)) + rnd<T>(mul(x2, s));
        r[2 * q + 1] = rnd<T>(mul(x2, c)) + rnd<T>(mul(-x1, s));
      }
    }
    store_vec<T, 8>(y + (tok * heads + hd) * dk + gi * 8, r);
  }
}

unsigned grid_for(int64_t items) {
  const int64_t blocks = (items + 255) / 256;
  return (unsigned)(blocks < 148 * 32 ? (blocks > 0 ? blocks : 1) : 148 * 32);
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
  const int64_t items = tokens * heads * (dk / 8);
  return VB_DISPATCH_DTYPE(dtype, T, [&]() -> int {
    if (backward)
      rotary_kernel<T, true><<<grid_for(items), 256, 0, (cudaStream_t)stream>>>(
          (const T*)x, (const int64_t*)pos, inv_freq, (T*)y, tokens, heads, dk);
    else
      rotary_kernel<T, false><<<grid_for(items), 256, 0, (cudaStream_t)stream>>>(
          (const T*)x, (const int64_t*)pos, inv_freq, (T*)y, tokens, heads, dk);
    VB_LAUNCH_CHECK("rotary");
    return VB_OK;
  });
}
