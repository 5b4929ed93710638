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
// One CTA of eight warps per (row, key head): the warps split the ring's slots and each walks its
// share for every query head of the group at once (a slot's key and value are loaded once, with
// lane l holding elements l, l + 32, ... of each DK-vector; the group's scores are warp sums in
// flight together), keeping a running float32 (max, sum, output) per head; the warps' partial
// results are then merged in a fixed order.
#include <cmath>
#include <type_traits>

#include "common.cuh"

namespace vb {
namespace {

constexpr int NE = 4;      // DK <= 128
constexpr int WARPS = 8;   // slot-splitting warps per CTA
constexpr int GMAX = 8;    // query heads per key head

template <typename E>
__device__ __forceinline__ void load_row(const E* __restrict__ p, int DK, float (&x)[NE]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int e = 0; e < NE; ++e) {
    const int d = lane + 32 * e;
    x[e] = d < DK ? to_f32<E>(p[d]) : 0.f;
  }
}

template <typename E, int G>
__global__ void __launch_bounds__(WARPS * 32) ring_attn_kernel(
    const E* __restrict__ q, const E* __restrict__ k_new, const E* __restrict__ v_new, E* ring_k, E* ring_v,
    int64_t* ring_pos, uint8_t* ring_valid, const int64_t* __restrict__ pos, E* __restrict__ o, int W, int H,
    int HKV, int DK, int window, float scale) {
  __shared__ float sm_m[WARPS][G], sm_l[WARPS][G], sm_acc[WARPS][G][32 * NE];
  const int b = blockIdx.x, kh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t p = pos[b];
  const int own = (int)(p % W);
  float qv[G][NE], m[G], l[G], acc[G][NE];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    load_row(q + ((int64_t)b * H + kh * G + g) * DK, DK, qv[g]);
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < NE; ++e) acc[g][e] = 0.f;
  }
  auto visit = [&](const float (&kv)[NE], const float (&vv)[NE]) {
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float a = 0.f;
#pragma unroll
      for (int e = 0; e < NE; ++e) a = fmaf(qv[g][e], kv[e], a);
      s[g] = a;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int g = 0; g < G; ++g) s[g] += __shfl_xor_sync(0xffffffffu, s[g], off);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float sc = s[g] * scale;
      const float mn = fmaxf(m[g], sc);
      const float c = expf(m[g] - mn), pj = expf(sc - mn);
      l[g] = fmaf(l[g], c, pj);
#pragma unroll
      for (int e = 0; e < NE; ++e) acc[g][e] = fmaf(acc[g][e], c, pj * vv[e]);
      m[g] = mn;
    }
  };
  float kv[NE], vv[NE];
  if (warp == 0) {  // the new token: always visible
    load_row(k_new + ((int64_t)b * HKV + kh) * DK, DK, kv);
    load_row(v_new + ((int64_t)b * HKV + kh) * DK, DK, vv);
    visit(kv, vv);
  }
  for (int slot = warp; slot < W; slot += WARPS) {
    if (slot == own || !ring_valid[(int64_t)b * W + slot]) continue;
    const int64_t kp = ring_pos[(int64_t)b * W + slot];
    if (kp > p || kp <= p - window) continue;
    const int64_t base = (((int64_t)b * W + slot) * HKV + kh) * DK;
    load_row(ring_k + base, DK, kv);
    load_row(ring_v + base, DK, vv);
    visit(kv, vv);
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) { sm_m[warp][g] = m[g]; sm_l[warp][g] = l[g]; }
#pragma unroll
    for (int e = 0; e < NE; ++e) sm_acc[warp][g][lane + 32 * e] = acc[g][e];
  }
  __syncthreads();  // every warp has read the ring and left its partial result
  if (warp < G) {  // warp g merges head g's partials in warp order
    const int g = warp;
    float M = -INFINITY;
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, sm_m[w][g]);
    float L = 0.f, out[NE] = {0.f, 0.f, 0.f, 0.f};
    for (int w = 0; w < WARPS; ++w) {
      const float f = sm_m[w][g] == -INFINITY ? 0.f : expf(sm_m[w][g] - M);
      L = fmaf(sm_l[w][g], f, L);
#pragma unroll
      for (int e = 0; e < NE; ++e) out[e] = fmaf(sm_acc[w][g][lane + 32 * e], f, out[e]);
    }
    const float inv = 1.0f / L;
#pragma unroll
    for (int e = 0; e < NE; ++e) {
      const int d = lane + 32 * e;
      if (d < DK) o[((int64_t)b * H + kh * G + g) * DK + d] = from_f32<E>(out[e] * inv);
    }
  }
  if (warp == WARPS - 1) {  // the new token takes its slot (no warp of any CTA reads that slot)
    const int64_t base = (((int64_t)b * W + own) * HKV + kh) * DK;
    for (int d = lane; d < DK; d += 32) {
      ring_k[base + d] = k_new[((int64_t)b * HKV + kh) * DK + d];
      ring_v[base + d] = v_new[((int64_t)b * HKV + kh) * DK + d];
    }
    if (kh == 0 && lane == 0) {
      ring_pos[(int64_t)b * W + own] = p;
      ring_valid[(int64_t)b * W + own] = 1;
    }
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
  VB_REQUIRE(DK >= 1 && DK <= 32 * NE, "ring_attend: head dimension %d must lie in [1, %d]", DK, 32 * NE);
  VB_REQUIRE(window >= 1, "ring_attend: window %d must be at least 1", window);
  VB_REQUIRE(dtype == VB_F32 || dtype == VB_BF16 || dtype == VB_F16, "ring_attend: unsupported dtype %d", dtype);
  if (B == 0) return VB_OK;
  VB_REQUIRE(q && k_new && v_new && ring_k && ring_v && ring_pos && ring_valid && pos && o,
             "ring_attend: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid(B, HKV);
  const float scale = 1.0f / sqrtf((float)DK);
  const int G = H / HKV;
  return VB_DISPATCH_DTYPE(dtype, T, [&]() -> int {
    auto launch = [&](auto gc) -> int {
      constexpr int GG = decltype(gc)::value;
      ring_attn_kernel<T, GG><<<grid, WARPS * 32, 0, st>>>((const T*)q, (const T*)k_new, (const T*)v_new,
                                                           (T*)ring_k, (T*)ring_v, ring_pos, ring_valid, pos, (T*)o,
                                                           W, H, HKV, DK, window, scale);
      VB_LAUNCH_CHECK("ring_attend");
      return VB_OK;
    };
    switch (G) {
      case 1: return launch(std::integral_constant<int, 1>{});
      case 2: return launch(std::integral_constant<int, 2>{});
      case 3: return launch(std::integral_constant<int, 3>{});
      case 4: return launch(std::integral_constant<int, 4>{});
      case 5: return launch(std::integral_constant<int, 5>{});
      case 6: return launch(std::integral_constant<int, 6>{});
      case 7: return launch(std::integral_constant<int, 7>{});
      default: return launch(std::integral_constant<int, 8>{});
    }
  });
}
