// The head's per-row next-token loss without float32 vocabulary copies (the row steps of
// vesper/kernels/nll.py:48-169, linear_nll; its Triton rows vesper/kernels/nll_triton.py:24-103).
//
// Given the logits [rows, V] in the matmul's own dtype (bf16 under autocast), the forward reduces
// each row to float32 statistics -- its maximum `top` and the shifted log-sum-exp
// log_total = log sum exp(x - top) -- and its loss nll = (top - x[target]) + log_total; the
// backward overwrites the logits IN PLACE with g * (exp((x - top) - log_total) - onehot), computed
// in float32 and rounded to the logits' dtype. Both keep the statistics shifted, so a common
// offset of a row cancels exactly. One 256-thread CTA per row walks it in 16-byte vectors: the
// forward holds a running (max, sum) per thread and combines them across the CTA; HBM-bound
// (2V bytes read per row forward, 2V read + 2V written backward for bf16).
#include <cmath>

#include "common.cuh"

namespace vb {
namespace {

constexpr int NT = 256;

// (m, s) <- the combination of two running (max, sum of exp(x - max)) pairs
__device__ __forceinline__ void merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;  // both empty
  s = s * expf(m - mn) + s2 * expf(m2 - mn);
  m = mn;
}

template <typename T>
__global__ void __launch_bounds__(NT) nll_stats_kernel(const T* __restrict__ logits, int64_t stride,
                                                       const int64_t* __restrict__ targets, float* __restrict__ top,
                                                       float* __restrict__ log_total, float* __restrict__ nll, int V,
                                                       int vec) {
  constexpr int E = 16 / sizeof(T);
  const int64_t row = blockIdx.x;
  const T* x = logits + row * stride;
  float m = -INFINITY, s = 0.f;
  if (vec) {
    const int nv = V / E;
    for (int i = threadIdx.x; i < nv; i += NT) {
      float v[E];
      load_vec<T, E>(x + (int64_t)i * E, v);
      float bm = v[0];
#pragma unroll
      for (int e = 1; e < E; ++e) bm = fmaxf(bm, v[e]);
      float bs = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) bs += expf(v[e] - bm);
      merge(m, s, bm, bs);
    }
    for (int j = nv * E + threadIdx.x; j < V; j += NT) merge(m, s, to_f32<T>(x[j]), 1.f);
  } else {
    for (int j = threadIdx.x; j < V; j += NT) merge(m, s, to_f32<T>(x[j]), 1.f);
  }
  // warp, then CTA combination in a fixed order (deterministic)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    merge(m, s, m2, s2);
  }
  __shared__ float wm[NT / 32], ws[NT / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { wm[warp] = m; ws[warp] = s; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = wm[0], S = ws[0];
    for (int w = 1; w < NT / 32; ++w) merge(M, S, wm[w], ws[w]);
    const float lt = logf(S);
    const float picked = to_f32<T>(x[targets[row]]);
    top[row] = M;
    log_total[row] = lt;
    nll[row] = (M - picked) + lt;
  }
}

template <typename T>
__global__ void __launch_bounds__(NT) nll_grad_kernel(T* __restrict__ logits, int64_t stride,
                                                      const int64_t* __restrict__ targets,
                                                      const float* __restrict__ top,
                                                      const float* __restrict__ log_total,
                                                      const float* __restrict__ grad, int V, int vec) {
  constexpr int E = 16 / sizeof(T);
  const int64_t row = blockIdx.x;
  T* x = logits + row * stride;
  const float tp = top[row], lt = log_total[row], g = grad[row];
  const int64_t tgt = targets[row];
  auto value = [&](float xv, int64_t j) {
    const float p = expf((xv - tp) - lt) * g;
    return j == tgt ? p - g : p;
  };
  if (vec) {
    const int nv = V / E;
    for (int i = threadIdx.x; i < nv; i += NT) {
      float v[E];
      load_vec<T, E>(x + (int64_t)i * E, v);
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] = value(v[e], (int64_t)i * E + e);
      store_vec<T, E>(x + (int64_t)i * E, v);
    }
    for (int j = nv * E + threadIdx.x; j < V; j += NT) x[j] = from_f32<T>(value(to_f32<T>(x[j]), j));
  } else {
    for (int j = threadIdx.x; j < V; j += NT) x[j] = from_f32<T>(value(to_f32<T>(x[j]), j));
  }
}

int check(const char* what, const void* logits, int64_t rows, int V, int64_t stride, int dtype) {
  VB_REQUIRE(rows >= 0 && V > 0 && stride >= V, "%s: bad shape rows=%lld V=%d stride=%lld", what, (long long)rows, V,
             (long long)stride);
  VB_REQUIRE(rows < (int64_t(1) << 31), "%s: %lld rows exceed 2^31", what, (long long)rows);
  VB_REQUIRE(dtype_size(dtype) > 0, "%s: unsupported dtype code %d", what, dtype);
  (void)logits;
  return VB_OK;
}

// 16-byte vectors when the base and every row start are 16-byte aligned
bool vectorizable(const void* logits, int64_t stride, int dtype) {
  return aligned16(logits) && (stride * dtype_size(dtype)) % 16 == 0;
}

}  // namespace
}  // namespace vb

using namespace vb;

extern "C" int vb_nll_row_stats(const void* logits, int64_t stride, const int64_t* targets, float* top,
                                float* log_total, float* nll, int64_t rows, int V, int dtype, void* stream) {
  int rc = check("nll_row_stats", logits, rows, V, stride, dtype);
  if (rc) return rc;
  if (rows == 0) return VB_OK;
  VB_REQUIRE(logits && targets && top && log_total && nll, "nll_row_stats: null pointer");
  const int vec = vectorizable(logits, stride, dtype) ? 1 : 0;
  cudaStream_t st = (cudaStream_t)stream;
  return VB_DISPATCH_DTYPE(dtype, T, [&]() -> int {
    nll_stats_kernel<T><<<(unsigned)rows, NT, 0, st>>>((const T*)logits, stride, targets, top, log_total, nll, V, vec);
    VB_LAUNCH_CHECK("nll_row_stats");
    return VB_OK;
  });
}

extern "C" int vb_nll_row_grad(void* logits, int64_t stride, const int64_t* targets, const float* top,
                               const float* log_total, const float* grad, int64_t rows, int V, int dtype,
                               void* stream) {
  int rc = check("nll_row_grad", logits, rows, V, stride, dtype);
  if (rc) return rc;
  if (rows == 0) return VB_OK;
  VB_REQUIRE(logits && targets && top && log_total && grad, "nll_row_grad: null pointer");
  const int vec = vectorizable(logits, stride, dtype) ? 1 : 0;
  cudaStream_t st = (cudaStream_t)stream;
  return VB_DISPATCH_DTYPE(dtype, T, [&]() -> int {
    nll_grad_kernel<T><<<(unsigned)rows, NT, 0, st>>>((T*)logits, stride, targets, top, log_total, grad, V, vec);
    VB_LAUNCH_CHECK("nll_row_grad");
    return VB_OK;
  });
}
