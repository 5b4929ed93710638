// Sliding-window attention in float32 on CUDA cores (FFMA), the float32 mode of
// vb_window_attn_fwd / vb_window_attn_bwd (dtype VB_F32): the reference's float32 path,
// vesper/attention.py:340-407 (WindowedAttention.attend over its blocked, masked softmax), computed
// without a tensor core so that float32 parity holds at float32 rounding.
//
// Semantics as the bf16 kernels: query row r at key index p (p = L - NQ + r, or qpos[b][r] for
// compacted rows, of which counts[b] are live) attends the keys j with p - window < j <= p,
// scale 1/sqrt(DK), query head h reading key head h / (H / HKV). lse [B,H,NQ] is the natural
// log-sum-exp of the scaled scores, saved for the backward.
//
// One warp per (batch, query row, head) in the forward and for dq, one warp per (batch, key row,
// key head) for dk and dv: lane l holds elements l, l + 32, ... of every DK-vector, a score is a
// warp sum, keys (or queries) are taken four at a time so that four reductions are in flight.
// Every gradient is a fixed-order sum: no atomics, deterministic.
#include <cmath>

#include "common.cuh"

namespace vb {
namespace {

constexpr int NE = 4;  // elements of a DK <= 128 vector per lane
constexpr int WARPS = 8;

struct Geometry {
  const int* qpos;
  const int* counts;
  int B, NQ, L, H, HKV, DK, win;
  float scale;
};

__device__ __forceinline__ void load_vec(const float* __restrict__ p, int DK, float (&x)[NE]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int e = 0; e < NE; ++e) {
    const int d = lane + 32 * e;
    x[e] = d < DK ? __ldg(p + d) : 0.f;
  }
}

__device__ __forceinline__ float dot_part(const float (&a)[NE], const float (&b)[NE]) {
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < NE; ++e) s = fmaf(a[e], b[e], s);
  return s;
}

// the position of query row r of batch b, or -1 for a padding row of a compacted batch
__device__ __forceinline__ int query_pos(const Geometry& g, int b, int r) {
  if (g.qpos == nullptr) return g.L - g.NQ + r;
  const int live = g.counts != nullptr ? g.counts[b] : g.NQ;
  return r < live ? g.qpos[(int64_t)b * g.NQ + r] : -1;
}

__global__ void __launch_bounds__(WARPS * 32) attn_f32_fwd_kernel(const float* __restrict__ q,
                                                                 const float* __restrict__ keys,
                                                                 const float* __restrict__ values,
                                                                 float* __restrict__ o, float* __restrict__ lse,
                                                                 Geometry g) {
  const int lane = threadIdx.x & 31;
  const int64_t w = (int64_t)blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (w >= (int64_t)g.B * g.NQ * g.H) return;
  const int h = (int)(w % g.H), r = (int)((w / g.H) % g.NQ), b = (int)(w / ((int64_t)g.H * g.NQ));
  const int kh = h / (g.H / g.HKV);
  const int64_t qrow = ((int64_t)b * g.NQ + r) * g.H + h;
  const int p = query_pos(g, b, r);
  if (p < 0) {  // padding row: zero output
#pragma unroll
    for (int e = 0; e < NE; ++e)
      if (lane + 32 * e < g.DK) o[qrow * g.DK + lane + 32 * e] = 0.f;
    if (lane == 0) lse[((int64_t)b * g.H + h) * g.NQ + r] = -INFINITY;
    return;
  }
  float qv[NE];
  load_vec(q + qrow * g.DK, g.DK, qv);
  const int j0 = max(0, p - g.win + 1), j1 = p;
  float m = -INFINITY, l = 0.f, acc[NE] = {0.f, 0.f, 0.f, 0.f};
  auto kv_row = [&](int j) { return (((int64_t)b * g.L + j) * g.HKV + kh) * g.DK; };
  for (int j = j0; j <= j1; j += 4) {
    float s[4], vv[4][NE];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int jj = j + u;
      float kv[NE];
      if (jj <= j1) {
        load_vec(keys + kv_row(jj), g.DK, kv);
        load_vec(values + kv_row(jj), g.DK, vv[u]);
      } else {
#pragma unroll
        for (int e = 0; e < NE; ++e) kv[e] = vv[u][e] = 0.f;
      }
      s[u] = dot_part(qv, kv);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int u = 0; u < 4; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], off);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (j + u > j1) break;
      const float sc = s[u] * g.scale;
      const float mn = fmaxf(m, sc);
      const float c = expf(m - mn), pj = expf(sc - mn);
      l = fmaf(l, c, pj);
#pragma unroll
      for (int e = 0; e < NE; ++e) acc[e] = fmaf(acc[e], c, pj * vv[u][e]);
      m = mn;
    }
  }
  const float inv = 1.0f / l;
#pragma unroll
  for (int e = 0; e < NE; ++e)
    if (lane + 32 * e < g.DK) o[qrow * g.DK + lane + 32 * e] = acc[e] * inv;
  if (lane == 0) lse[((int64_t)b * g.H + h) * g.NQ + r] = m + logf(l);
}

// delta[b][h][r] = do . o over the head dimension
__global__ void __launch_bounds__(WARPS * 32) attn_f32_delta_kernel(const float* __restrict__ o,
                                                                   const float* __restrict__ dout,
                                                                   float* __restrict__ delta, Geometry g) {
  const int lane = threadIdx.x & 31;
  const int64_t w = (int64_t)blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (w >= (int64_t)g.B * g.NQ * g.H) return;
  const int h = (int)(w % g.H), r = (int)((w / g.H) % g.NQ), b = (int)(w / ((int64_t)g.H * g.NQ));
  float ov[NE], gv[NE];
  load_vec(o + w * g.DK, g.DK, ov);
  load_vec(dout + w * g.DK, g.DK, gv);
  const float s = warp_sum(dot_part(ov, gv));
  if (lane == 0) delta[((int64_t)b * g.H + h) * g.NQ + r] = s;
}

__global__ void __launch_bounds__(WARPS * 32) attn_f32_dq_kernel(
    const float* __restrict__ q, const float* __restrict__ keys, const float* __restrict__ values,
    const float* __restrict__ dout, const float* __restrict__ lse, const float* __restrict__ delta,
    float* __restrict__ dq, Geometry g) {
  const int lane = threadIdx.x & 31;
  const int64_t w = (int64_t)blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (w >= (int64_t)g.B * g.NQ * g.H) return;
  const int h = (int)(w % g.H), r = (int)((w / g.H) % g.NQ), b = (int)(w / ((int64_t)g.H * g.NQ));
  const int kh = h / (g.H / g.HKV);
  const int p = query_pos(g, b, r);
  float acc[NE] = {0.f, 0.f, 0.f, 0.f};
  if (p >= 0) {
    float qv[NE], gv[NE];
    load_vec(q + w * g.DK, g.DK, qv);
    load_vec(dout + w * g.DK, g.DK, gv);
    const int64_t sidx = ((int64_t)b * g.H + h) * g.NQ + r;
    const float ls = lse[sidx], dl = delta[sidx];
    const int j0 = max(0, p - g.win + 1), j1 = p;
    auto kv_row = [&](int j) { return (((int64_t)b * g.L + j) * g.HKV + kh) * g.DK; };
    for (int j = j0; j <= j1; j += 4) {
      float s[4], dp[4], kv[4][NE];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float vv[NE];
        if (j + u <= j1) {
          load_vec(keys + kv_row(j + u), g.DK, kv[u]);
          load_vec(values + kv_row(j + u), g.DK, vv);
        } else {
#pragma unroll
          for (int e = 0; e < NE; ++e) kv[u][e] = vv[e] = 0.f;
        }
        s[u] = dot_part(qv, kv[u]);
        dp[u] = dot_part(gv, vv);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          s[u] += __shfl_xor_sync(0xffffffffu, s[u], off);
          dp[u] += __shfl_xor_sync(0xffffffffu, dp[u], off);
        }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (j + u > j1) break;
        const float pr = expf(s[u] * g.scale - ls);
        const float ds = pr * (dp[u] - dl) * g.scale;
#pragma unroll
        for (int e = 0; e < NE; ++e) acc[e] = fmaf(ds, kv[u][e], acc[e]);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < NE; ++e)
    if (lane + 32 * e < g.DK) dq[w * g.DK + lane + 32 * e] = acc[e];
}

// the first live row of batch b (positions ascending) whose position is at least `pos`
__device__ __forceinline__ int first_at_or_after(const int* __restrict__ qp, int live, int pos) {
  int lo = 0, hi = live;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (qp[mid] < pos) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

// the query rows [r0, r1) of batch b whose window holds key j: positions in [j, j + win)
__device__ __forceinline__ void query_range(const Geometry& g, int b, int j, int& r0, int& r1) {
  if (g.qpos == nullptr) {
    const int off = g.L - g.NQ;  // row r sits at position off + r
    r0 = max(0, j - off);
    r1 = max(r0, min(g.NQ, j - off + g.win));
    return;
  }
  const int live = g.counts != nullptr ? g.counts[b] : g.NQ;
  const int* qp = g.qpos + (int64_t)b * g.NQ;
  r0 = first_at_or_after(qp, live, j);
  r1 = first_at_or_after(qp, live, j + g.win);
}

__global__ void __launch_bounds__(WARPS * 32) attn_f32_dkv_kernel(
    const float* __restrict__ q, const float* __restrict__ keys, const float* __restrict__ values,
    const float* __restrict__ dout, const float* __restrict__ lse, const float* __restrict__ delta,
    float* __restrict__ dkeys, float* __restrict__ dvalues, Geometry g) {
  const int lane = threadIdx.x & 31;
  const int64_t w = (int64_t)blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (w >= (int64_t)g.B * g.L * g.HKV) return;
  const int kh = (int)(w % g.HKV), j = (int)((w / g.HKV) % g.L), b = (int)(w / ((int64_t)g.HKV * g.L));
  const int G = g.H / g.HKV;
  float kv[NE], vv[NE], dk[NE] = {0.f, 0.f, 0.f, 0.f}, dv[NE] = {0.f, 0.f, 0.f, 0.f};
  load_vec(keys + w * g.DK, g.DK, kv);
  load_vec(values + w * g.DK, g.DK, vv);
  int r0, r1;
  query_range(g, b, j, r0, r1);
  for (int hh = 0; hh < G; ++hh) {
    const int h = kh * G + hh;
    for (int r = r0; r < r1; r += 4) {
      float s[4], dp[4], qv[4][NE], gv[4][NE];
      bool live[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int rr = r + u;
        const int p = rr < r1 ? query_pos(g, b, rr) : -1;
        live[u] = p >= j && p - g.win < j;
        if (live[u]) {
          const int64_t row = ((int64_t)b * g.NQ + rr) * g.H + h;
          load_vec(q + row * g.DK, g.DK, qv[u]);
          load_vec(dout + row * g.DK, g.DK, gv[u]);
        } else {
#pragma unroll
          for (int e = 0; e < NE; ++e) qv[u][e] = gv[u][e] = 0.f;
        }
        s[u] = dot_part(qv[u], kv);
        dp[u] = dot_part(gv[u], vv);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          s[u] += __shfl_xor_sync(0xffffffffu, s[u], off);
          dp[u] += __shfl_xor_sync(0xffffffffu, dp[u], off);
        }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (!live[u]) continue;
        const int64_t sidx = ((int64_t)b * g.H + h) * g.NQ + r + u;
        const float pr = expf(s[u] * g.scale - lse[sidx]);
        const float ds = pr * (dp[u] - delta[sidx]) * g.scale;
#pragma unroll
        for (int e = 0; e < NE; ++e) {
          dv[e] = fmaf(pr, gv[u][e], dv[e]);
          dk[e] = fmaf(ds, qv[u][e], dk[e]);
        }
      }
    }
  }
#pragma unroll
  for (int e = 0; e < NE; ++e)
    if (lane + 32 * e < g.DK) {
      dkeys[w * g.DK + lane + 32 * e] = dk[e];
      dvalues[w * g.DK + lane + 32 * e] = dv[e];
    }
}

unsigned warps_grid(int64_t warps) { return (unsigned)((warps + WARPS - 1) / WARPS); }

}  // namespace

// the float32 forward (dtype VB_F32 of vb_window_attn_fwd; shapes already checked)
int window_attn_f32_fwd(const float* q, const int* qpos, const int* counts, const float* keys, const float* values,
                        float* o, float* lse, int B, int NQ, int L, int H, int HKV, int DK, int window,
                        cudaStream_t st) {
  const Geometry g{qpos, counts, B, NQ, L, H, HKV, DK, window > L ? L + 1 : window, 1.0f / sqrtf((float)DK)};
  attn_f32_fwd_kernel<<<warps_grid((int64_t)B * NQ * H), WARPS * 32, 0, st>>>(q, keys, values, o, lse, g);
  VB_LAUNCH_CHECK("window_attn_fwd f32");
  return VB_OK;
}

// the float32 backward; `delta` holds B*NQ*H floats
int window_attn_f32_bwd(const float* q, const int* qpos, const int* counts, const float* keys, const float* values,
                        const float* o, const float* lse, const float* dout, float* dq, float* dkeys, float* dvalues,
                        float* delta, int B, int NQ, int L, int H, int HKV, int DK, int window, cudaStream_t st) {
  const Geometry g{qpos, counts, B, NQ, L, H, HKV, DK, window > L ? L + 1 : window, 1.0f / sqrtf((float)DK)};
  const int64_t rows = (int64_t)B * NQ * H;
  attn_f32_delta_kernel<<<warps_grid(rows), WARPS * 32, 0, st>>>(o, dout, delta, g);
  VB_LAUNCH_CHECK("window_attn_bwd f32 delta");
  attn_f32_dq_kernel<<<warps_grid(rows), WARPS * 32, 0, st>>>(q, keys, values, dout, lse, delta, dq, g);
  VB_LAUNCH_CHECK("window_attn_bwd f32 dq");
  attn_f32_dkv_kernel<<<warps_grid((int64_t)B * L * HKV), WARPS * 32, 0, st>>>(q, keys, values, dout, lse, delta,
                                                                               dkeys, dvalues, g);
  VB_LAUNCH_CHECK("window_attn_bwd f32 dkv");
  return VB_OK;
}

}  // namespace vb
