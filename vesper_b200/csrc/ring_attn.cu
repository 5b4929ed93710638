// One decoding token per batch row attending over its fixed-capacity ring window and itself, then
// written into the ring (vesper/attention.py:298-338 attend_ring with :63-139 RingKVCache and
// kv_ring_write), batched over every row of a decode step.
//
// The ring holds `window` slots per row, k and v [B, W, HKV, DK] (keys already rotated),
// pos [B, W] int64 and valid [B, W] (one byte per slot); a token at position p lives in slot
// p % W and slots are not in age order: a slot is visible to the new token at position p when it
// is valid and p - window < pos <= p, and the new token always sees itself. Its own slot p % W is
// skipped while reading (its occupant, if any, is window or more positions old and not visible)
// and rewritten afterwards with the new key, value, position and valid flag, so the CTAs of one
// row never read what another is writing.
//
// One CTA of 16 warps per (row, key head), in three phases over the W + 1 candidate keys (the
// ring's slots and the new token, index W): (1) each warp takes a share of the slots and forms
// the group's scores for each (lane l holding channels l, l + 32, ... of the queries and the key
// row; the scores are warp sums), -inf for a slot that is not visible; (2) warp g reduces head g's scores to their max
// and sum and turns them into probabilities; (3) each warp takes a share of the slots and sums
// probability x value for every head of the group (lane l holding channels l, l + 32, ...: the
// value rows read coalesced), and the warps' partial sums are added in warp order.
// Deterministic (fixed-order sums), no atomics.
#include <cmath>
#include <type_traits>

#include "common.cuh"

namespace vb {
namespace {

constexpr int NT = 512;
constexpr int GMAX = 8;     // query heads per key head
constexpr int WMAX = 1024;  // ring slots
constexpr int DKMAX = 128;

template <typename E>
__global__ void __launch_bounds__(NT) ring_attn_kernel(
    const E* __restrict__ q, const E* __restrict__ k_new, const E* __restrict__ v_new, E* ring_k, E* ring_v,
    int64_t* ring_pos, uint8_t* ring_valid, const int64_t* __restrict__ pos, E* __restrict__ o, int W, int H,
    int HKV, int DK, int window, float scale) {
  extern __shared__ float smem[];
  const int G = H / HKV;
  float* qs = smem;             // [G][DK]
  float* ps = smem + G * DK;    // [G][W + 1]
  const int b = blockIdx.x, kh = blockIdx.y, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int64_t p = pos[b];
  const int own = (int)(p % W);
  for (int e = tid; e < G * DK; e += NT) qs[e] = to_f32<E>(q[((int64_t)b * H + kh * G) * DK + e]);
  __syncthreads();
  // (1) scores. The visibility of every slot first, from coalesced loads of the positions and
  // flags (a per-slot chain of dependent loads would serialise the walk); then warp w takes slots
  // w, w + NW, ... four at a time (the new token is index W): lane l holds channels l, l + 32, ...
  // of the queries (registers) and of each key row, and the 4 x G scores are warp sums in flight
  // together. Every key row is loaded (an unwritten slot holds finite zeros); a slot that is not
  // visible scores -inf.
  constexpr int NE = DKMAX / 32, NW = NT / 32, U = 4;
  uint8_t* vis = reinterpret_cast<uint8_t*>(ps + G * (W + 1) + NW * G * DK);  // [W + 1]
  for (int s = tid; s <= W; s += NT) {
    bool v = s == W;
    if (!v && s != own && ring_valid[(int64_t)b * W + s]) {
      const int64_t kp = ring_pos[(int64_t)b * W + s];
      v = kp <= p && kp > p - window;
    }
    vis[s] = v ? 1 : 0;
  }
  float qv[GMAX][NE];
#pragma unroll
  for (int g = 0; g < GMAX; ++g)
#pragma unroll
    for (int e = 0; e < NE; ++e) qv[g][e] = (g < G && lane + 32 * e < DK) ? qs[g * DK + lane + 32 * e] : 0.f;
  __syncthreads();
  for (int s0 = warp * U; s0 <= W; s0 += NW * U) {
    float sc[U][GMAX];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int s = s0 + u;
      const E* krow = s == W ? k_new + ((int64_t)b * HKV + kh) * DK
                             : ring_k + (((int64_t)b * W + min(s, W - 1)) * HKV + kh) * DK;
      float kv[NE];
#pragma unroll
      for (int e = 0; e < NE; ++e) kv[e] = (s <= W && lane + 32 * e < DK) ? to_f32<E>(krow[lane + 32 * e]) : 0.f;
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
        float a = 0.f;
#pragma unroll
        for (int e = 0; e < NE; ++e) a = fmaf(qv[g][e], kv[e], a);
        sc[u][g] = a;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int g = 0; g < GMAX; ++g)
          if (g < G) sc[u][g] += __shfl_xor_sync(0xffffffffu, sc[u][g], off);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int s = s0 + u;
#pragma unroll
      for (int g = 0; g < GMAX; ++g)
        if (g < G && lane == g && s <= W) ps[g * (W + 1) + s] = vis[s] ? sc[u][g] * scale : -INFINITY;
    }
  }
  __syncthreads();
  // (2) probabilities, head g by warp g
  if (warp < G) {
    float* row = ps + warp * (W + 1);
    float m = -INFINITY;
    for (int s = lane; s <= W; s += 32) m = fmaxf(m, row[s]);
    m = warp_max(m);
    float l = 0.f;
    for (int s = lane; s <= W; s += 32) {
      const float e = row[s] == -INFINITY ? 0.f : expf(row[s] - m);
      row[s] = e;
      l += e;
    }
    l = warp_sum(l);
    const float inv = 1.0f / l;
    for (int s = lane; s <= W; s += 32) row[s] *= inv;
  }
  __syncthreads();
  // (3) outputs: warp w sums its share of the slots (s = w, w + NW, ...) for every head of the
  // group, lane l holding channels l, l + 32, ...; the warps' partial sums are added in warp order
  float acc[GMAX][NE];
#pragma unroll
  for (int g = 0; g < GMAX; ++g)
#pragma unroll
    for (int e = 0; e < NE; ++e) acc[g][e] = 0.f;
  const int64_t stride = (int64_t)HKV * DK;
  const E* vbase = ring_v + ((int64_t)b * W * HKV + kh) * DK;
  auto add_row = [&](const E* vrow, int s) {
    float vv[NE];
#pragma unroll
    for (int e = 0; e < NE; ++e) vv[e] = lane + 32 * e < DK ? to_f32<E>(vrow[lane + 32 * e]) : 0.f;
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      if (g < G) {
        const float pr = ps[g * (W + 1) + s];
#pragma unroll
        for (int e = 0; e < NE; ++e) acc[g][e] = fmaf(pr, vv[e], acc[g][e]);
      }
    }
  };
  if (warp == 0) add_row(v_new + ((int64_t)b * HKV + kh) * DK, W);
  // unconditional loads (a slot that is not visible has probability exactly 0 and finite values)
#pragma unroll 4
  for (int s = warp; s < W; s += NW) add_row(vbase + s * stride, s);  // unrolled: four rows in flight
  float* part = ps + G * (W + 1);  // [NW][G][DK]
#pragma unroll
  for (int g = 0; g < GMAX; ++g)
    if (g < G)
#pragma unroll
      for (int e = 0; e < NE; ++e)
        if (lane + 32 * e < DK) part[(warp * G + g) * DK + lane + 32 * e] = acc[g][e];
  __syncthreads();
  for (int e = tid; e < G * DK; e += NT) {
    float sum = 0.f;
    for (int w = 0; w < NW; ++w) sum += part[w * G * DK + e];
    o[((int64_t)b * H + kh * G) * DK + e] = from_f32<E>(sum);
  }
  __syncthreads();  // every thread has read the ring
  // the new token takes its slot (no CTA of this row reads that slot)
  for (int d = tid; d < DK; d += NT) {
    const int64_t base = (((int64_t)b * W + own) * HKV + kh) * DK;
    ring_k[base + d] = k_new[((int64_t)b * HKV + kh) * DK + d];
    ring_v[base + d] = v_new[((int64_t)b * HKV + kh) * DK + d];
  }
  if (kh == 0 && tid == 0) {
    ring_pos[(int64_t)b * W + own] = p;
    ring_valid[(int64_t)b * W + own] = 1;
  }
}

}  // namespace
}  // namespace vb

using namespace vb;

extern "C" int vb_ring_attend(const void* q, const void* k_new, const void* v_new, void* ring_k, void* ring_v,
                              int64_t* ring_pos, uint8_t* ring_valid, const int64_t* pos, void* o, int B, int W,
                              int H, int HKV, int DK, int window, int dtype, void* stream) {
  VB_REQUIRE(B >= 0 && W >= 1 && H >= 1 && HKV >= 1 && H % HKV == 0 && H / HKV <= GMAX,
             "ring_attend: bad shape B=%d W=%d H=%d HKV=%d", B, W, H, HKV);
  VB_REQUIRE(DK >= 1 && DK <= DKMAX, "ring_attend: head dimension %d must lie in [1, %d]", DK, DKMAX);
  VB_REQUIRE(window >= 1, "ring_attend: window %d must be at least 1", window);
  VB_REQUIRE(dtype == VB_F32 || dtype == VB_BF16 || dtype == VB_F16, "ring_attend: unsupported dtype %d", dtype);
  if (B == 0) return VB_OK;
  VB_REQUIRE(q && k_new && v_new && ring_k && ring_v && ring_pos && ring_valid && pos && o,
             "ring_attend: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  VB_REQUIRE(W <= WMAX, "ring_attend: %d slots exceed %d", W, WMAX);
  const dim3 grid(B, HKV);
  const float scale = 1.0f / sqrtf((float)DK);
  const int G = H / HKV;
  const size_t smem = sizeof(float) * ((size_t)G * DK + (size_t)G * (W + 1) + (size_t)(NT / 32) * G * DK) +
                      (size_t)(W + 1);
  return VB_DISPATCH_DTYPE(dtype, T, [&]() -> int {
    VB_CUDA_CHECK(cudaFuncSetAttribute(ring_attn_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                  "ring_attend: smem attribute");
    ring_attn_kernel<T><<<grid, NT, smem, st>>>((const T*)q, (const T*)k_new, (const T*)v_new, (T*)ring_k,
                                               (T*)ring_v, ring_pos, ring_valid, pos, (T*)o, W, H, HKV, DK, window,
                                               scale);
    VB_LAUNCH_CHECK("ring_attend");
    return VB_OK;
  });
}
