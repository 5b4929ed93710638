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
// A row's window is split into ranges of 128 slots, one CTA of eight warps per (row, key head,
// range). Rows of a multiple of 16 bytes take the staged kernel (every key and value row of the
// range copied into shared memory at once, one thread per candidate for the scores and one per
// head and channel for the weighted values); other rows the kernel below, in which (1) the warps
// share the range's candidates
// and form the group's scores for each (lane l holding channels l, l + 32, ... of the queries and
// the key row; the scores are warp sums), -inf for a slot that is not visible; (2) warp g reduces
// head g's scores to the range's max and the unnormalised weights and their sum; (3) the warps
// share the candidates again for weight x value (the value rows read coalesced). A second kernel
// merges the ranges in order per (row, key head) and then writes the new token into its slot.
// Deterministic (fixed-order sums), no atomics.
#include <cmath>
#include <type_traits>

#include "common.cuh"

namespace vb {
namespace {

constexpr int NT = 256;
constexpr int GMAX = 8;     // query heads per key head
constexpr int WMAX = 1024;  // ring slots
constexpr int DKMAX = 128;

constexpr int SPLIT_SLOTS = 128;  // ring slots per CTA: a row's window is split over several CTAs

int splits(int W) { return (W + SPLIT_SLOTS - 1) / SPLIT_SLOTS; }

// Partial attention of one (row, key head, slot range): the range's slots (and, for the last
// range, the new token), written as each head's local max m, local sum l and unnormalised output
// acc [DK] to part [B][HKV][nsplit][G][DK + 2].
template <typename E, int GC, int NEC>
__global__ void __launch_bounds__(NT) ring_attn_part_kernel(
    const E* __restrict__ q, const E* __restrict__ k_new, const E* __restrict__ v_new, const E* __restrict__ ring_k,
    const E* __restrict__ ring_v, const int64_t* __restrict__ ring_pos, const uint8_t* __restrict__ ring_valid,
    const int64_t* __restrict__ pos, float* __restrict__ part, int W, int H, int HKV, int DK, int window,
    float scale) {
  extern __shared__ float smem[];
  // GC: the query heads per key head, NEC: channels per lane (ceil(DK / 32)), both compile-time so
  // that no lane computes for a head or a channel that does not exist
  constexpr int G = GC, GMAX = GC, NE = NEC;
  const int nsplit = gridDim.z;
  const int b = blockIdx.x, kh = blockIdx.y, z = blockIdx.z, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int lo = z * SPLIT_SLOTS, hi = min(W, lo + SPLIT_SLOTS);
  const bool last = z == nsplit - 1;
  const int L = hi - lo + (last ? 1 : 0);  // candidates: local index i is slot lo + i, or the new token
  float* qs = smem;                   // [G][DK]
  float* ps = smem + G * DK;          // [G][L]
  constexpr int NW = NT / 32, U = 4;
  float* red = ps + G * L;            // [NW][G][DK]
  uint8_t* vis = reinterpret_cast<uint8_t*>(red + NW * G * DK);  // [L]
  const int64_t p = pos[b];
  const int own = (int)(p % W);
  auto slot_of = [&](int i) { return i < hi - lo ? lo + i : W; };
  for (int e = tid; e < G * DK; e += NT) qs[e] = to_f32<E>(q[((int64_t)b * H + kh * G) * DK + e]);
  // the visibility of every candidate from one coalesced pass (a per-slot chain of dependent
  // loads would serialise the walk)
  for (int i = tid; i < L; i += NT) {
    const int s = slot_of(i);
    bool v = s == W;
    if (!v && s != own && ring_valid[(int64_t)b * W + s]) {
      const int64_t kp = ring_pos[(int64_t)b * W + s];
      v = kp <= p && kp > p - window;
    }
    vis[i] = v ? 1 : 0;
  }
  __syncthreads();
  // (1) scores: warp w takes candidates w*U .. w*U + U-1, then NW*U on; lane l holds channels
  // l, l + 32, ... of the queries and of each key row; the U x G scores are warp sums in flight
  // together; every key row is loaded (an unwritten slot holds finite zeros)
  float qv[GMAX][NE];
#pragma unroll
  for (int g = 0; g < GMAX; ++g)
#pragma unroll
    for (int e = 0; e < NE; ++e) qv[g][e] = (g < G && lane + 32 * e < DK) ? qs[g * DK + lane + 32 * e] : 0.f;
  for (int i0 = warp * U; i0 < L; i0 += NW * U) {
    float sc[U][GMAX];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u, s = slot_of(min(i, L - 1));
      const E* krow = s == W ? k_new + ((int64_t)b * HKV + kh) * DK : ring_k + (((int64_t)b * W + s) * HKV + kh) * DK;
      float kv[NE];
#pragma unroll
      for (int e = 0; e < NE; ++e) kv[e] = (i < L && lane + 32 * e < DK) ? to_f32<E>(krow[lane + 32 * e]) : 0.f;
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
      const int i = i0 + u;
#pragma unroll
      for (int g = 0; g < GMAX; ++g)
        if (g < G && lane == g && i < L) ps[g * L + i] = vis[i] ? sc[u][g] * scale : -INFINITY;
    }
  }
  __syncthreads();
  // (2) head g (warp g): the local max and the unnormalised weights exp(score - max), their sum
  float* stats = part + ((((int64_t)b * HKV + kh) * nsplit + z) * G) * (DK + 2);
  if (warp < G) {
    float* row = ps + warp * L;
    float m = -INFINITY;
    for (int i = lane; i < L; i += 32) m = fmaxf(m, row[i]);
    m = warp_max(m);
    float l = 0.f;
    for (int i = lane; i < L; i += 32) {
      const float e = row[i] == -INFINITY ? 0.f : expf(row[i] - m);
      row[i] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      stats[warp * (DK + 2) + DK] = m;
      stats[warp * (DK + 2) + DK + 1] = l;
    }
  }
  __syncthreads();
  // (3) warp w sums weight x value over its candidates for every head of the group, lane l holding
  // channels l, l + 32, ...; the warps' partials are added in warp order
  float acc[GMAX][NE];
#pragma unroll
  for (int g = 0; g < GMAX; ++g)
#pragma unroll
    for (int e = 0; e < NE; ++e) acc[g][e] = 0.f;
#pragma unroll 4
  for (int i = warp; i < L; i += NW) {  // unrolled: four value rows in flight
    const int s = slot_of(i);
    const E* vrow = s == W ? v_new + ((int64_t)b * HKV + kh) * DK : ring_v + (((int64_t)b * W + s) * HKV + kh) * DK;
    float vv[NE];
#pragma unroll
    for (int e = 0; e < NE; ++e) vv[e] = lane + 32 * e < DK ? to_f32<E>(vrow[lane + 32 * e]) : 0.f;
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      if (g < G) {
        const float pr = ps[g * L + i];
#pragma unroll
        for (int e = 0; e < NE; ++e) acc[g][e] = fmaf(pr, vv[e], acc[g][e]);
      }
    }
  }
#pragma unroll
  for (int g = 0; g < GMAX; ++g)
    if (g < G)
#pragma unroll
      for (int e = 0; e < NE; ++e)
        if (lane + 32 * e < DK) red[(warp * G + g) * DK + lane + 32 * e] = acc[g][e];
  __syncthreads();
  for (int e = tid; e < G * DK; e += NT) {
    const int g = e / DK, d = e % DK;
    float sum = 0.f;
    for (int w = 0; w < NW; ++w) sum += red[(w * G + g) * DK + d];
    stats[g * (DK + 2) + d] = sum;
  }
}

// The same partials from rows staged in shared memory (rows of a multiple of 16 bytes): every key
// and value row of the range (and, in the last range, the new token's) is copied at once by
// cp.async into an XOR-swizzled tile (16-byte chunk c of row r at c ^ (r mod 8)), the visibility
// pass runs while they land, then one thread per candidate forms the group's scores over the whole
// row and one thread per (head, channel) sums weight x value over the candidates: no shuffles and
// no cross-warp reduction, and only one round trip to memory per CTA.
__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}

template <typename E, int GC>
__global__ void __launch_bounds__(NT) ring_attn_part_staged_kernel(
    const E* __restrict__ q, const E* __restrict__ k_new, const E* __restrict__ v_new, const E* __restrict__ ring_k,
    const E* __restrict__ ring_v, const int64_t* __restrict__ ring_pos, const uint8_t* __restrict__ ring_valid,
    const int64_t* __restrict__ pos, float* __restrict__ part, int W, int H, int HKV, int DK, int window,
    float scale) {
  extern __shared__ __align__(16) uint8_t sraw[];
  constexpr int G = GC;
  const int nsplit = gridDim.z;
  const int b = blockIdx.x, kh = blockIdx.y, z = blockIdx.z, tid = threadIdx.x;
  const int lo = z * SPLIT_SLOTS, hi = min(W, lo + SPLIT_SLOTS);
  const bool last = z == nsplit - 1;
  const int L = hi - lo + (last ? 1 : 0);  // candidates: local index i is slot lo + i, or the new token
  const int RB = DK * (int)sizeof(E), NCH = RB / 16, SWM = (NCH < 8 ? NCH : 8) - 1;
  constexpr int EPC = 16 / (int)sizeof(E);
  uint8_t* ks = sraw;                                                      // [L][RB]
  uint8_t* vs = ks + (size_t)(SPLIT_SLOTS + 1) * RB;                       // [L][RB]
  float* qs = reinterpret_cast<float*>(vs + (size_t)(SPLIT_SLOTS + 1) * RB);  // [G][DK]
  float* ps = qs + G * DK;                                                 // [G][L]
  uint8_t* vis = reinterpret_cast<uint8_t*>(ps + G * (SPLIT_SLOTS + 1));   // [L]
  auto row_k = [&](int i) -> const E* {
    return i < hi - lo ? ring_k + (((int64_t)b * W + lo + i) * HKV + kh) * DK : k_new + ((int64_t)b * HKV + kh) * DK;
  };
  auto row_v = [&](int i) -> const E* {
    return i < hi - lo ? ring_v + (((int64_t)b * W + lo + i) * HKV + kh) * DK : v_new + ((int64_t)b * HKV + kh) * DK;
  };
  for (int c = tid; c < L * NCH; c += NT) {
    const int i = c / NCH, ch = c - i * NCH, at = (i * NCH + (ch ^ (i & SWM))) * 16;
    cp16(ks + at, reinterpret_cast<const uint8_t*>(row_k(i)) + ch * 16);
    cp16(vs + at, reinterpret_cast<const uint8_t*>(row_v(i)) + ch * 16);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  const int64_t p = pos[b];
  const int own = (int)(p % W);
  for (int e = tid; e < G * DK; e += NT) qs[e] = to_f32<E>(q[((int64_t)b * H + kh * G) * DK + e]);
  for (int i = tid; i < L; i += NT) {
    const int s = i < hi - lo ? lo + i : W;
    bool v = s == W;
    if (!v && s != own && ring_valid[(int64_t)b * W + s]) {
      const int64_t kp = ring_pos[(int64_t)b * W + s];
      v = kp <= p && kp > p - window;
    }
    vis[i] = v ? 1 : 0;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  // scores: one thread per candidate, the whole row against each head's query
  for (int i = tid; i < L; i += NT) {
    float acc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = 0.f;
    for (int ch = 0; ch < NCH; ++ch) {
      const uint4 raw = *reinterpret_cast<const uint4*>(ks + (i * NCH + (ch ^ (i & SWM))) * 16);
      const E* e = reinterpret_cast<const E*>(&raw);
#pragma unroll
      for (int u = 0; u < EPC; ++u) {
        const float kv = to_f32<E>(e[u]);
#pragma unroll
        for (int g = 0; g < G; ++g) acc[g] = fmaf(qs[g * DK + ch * EPC + u], kv, acc[g]);
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) ps[g * L + i] = vis[i] ? acc[g] * scale : -INFINITY;
  }
  __syncthreads();
  // head g (warp g): the local max and the unnormalised weights exp(score - max), their sum
  float* stats = part + ((((int64_t)b * HKV + kh) * nsplit + z) * G) * (DK + 2);
  const int warp = tid >> 5, lane = tid & 31;
  for (int g = warp; g < G; g += NT / 32) {
    float* row = ps + g * L;
    float m = -INFINITY;
    for (int i = lane; i < L; i += 32) m = fmaxf(m, row[i]);
    m = warp_max(m);
    float l = 0.f;
    for (int i = lane; i < L; i += 32) {
      const float e = row[i] == -INFINITY ? 0.f : expf(row[i] - m);
      row[i] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      stats[g * (DK + 2) + DK] = m;
      stats[g * (DK + 2) + DK + 1] = l;
    }
  }
  __syncthreads();
  // weight x value: one thread per (head, channel), the candidates in order
  for (int e = tid; e < G * DK; e += NT) {
    const int g = e / DK, d = e - g * DK, ch = d / EPC, u = d - ch * EPC;
    const float* w = ps + g * L;
    float a = 0.f;
    for (int i = 0; i < L; ++i) {
      const E* vr = reinterpret_cast<const E*>(vs + (i * NCH + (ch ^ (i & SWM))) * 16);
      a = fmaf(w[i], to_f32<E>(vr[u]), a);
    }
    stats[g * (DK + 2) + d] = a;
  }
}

// Merges a (row, key head)'s range partials in range order into the output, then writes the new
// token into its slot: the partial kernel has finished every read of the ring.
template <typename E>
__global__ void ring_attn_merge_kernel(const E* __restrict__ k_new, const E* __restrict__ v_new, E* ring_k, E* ring_v,
                                       int64_t* ring_pos, uint8_t* ring_valid, const int64_t* __restrict__ pos,
                                       const float* __restrict__ part, E* __restrict__ o, int nsplit, int W, int H,
                                       int HKV, int DK) {
  const int G = H / HKV;
  const int b = blockIdx.x, kh = blockIdx.y, tid = threadIdx.x;
  const float* base = part + (((int64_t)b * HKV + kh) * nsplit) * G * (DK + 2);
  for (int e = tid; e < G * DK; e += blockDim.x) {
    const int g = e / DK, d = e % DK;
    float M = -INFINITY;
    for (int z = 0; z < nsplit; ++z) M = fmaxf(M, base[((int64_t)z * G + g) * (DK + 2) + DK]);
    float Lsum = 0.f, out = 0.f;
    for (int z = 0; z < nsplit; ++z) {
      const float* st = base + ((int64_t)z * G + g) * (DK + 2);
      const float f = st[DK] == -INFINITY ? 0.f : expf(st[DK] - M);
      Lsum = fmaf(st[DK + 1], f, Lsum);
      out = fmaf(st[d], f, out);
    }
    o[((int64_t)b * H + kh * G + g) * DK + d] = from_f32<E>(out / Lsum);
  }
  const int64_t p = pos[b];
  const int own = (int)(p % W);
  for (int d = tid; d < DK; d += blockDim.x) {
    const int64_t dst = (((int64_t)b * W + own) * HKV + kh) * DK;
    ring_k[dst + d] = k_new[((int64_t)b * HKV + kh) * DK + d];
    ring_v[dst + d] = v_new[((int64_t)b * HKV + kh) * DK + d];
  }
  if (kh == 0 && tid == 0) {
    ring_pos[(int64_t)b * W + own] = p;
    ring_valid[(int64_t)b * W + own] = 1;
  }
}

}  // namespace
}  // namespace vb

using namespace vb;

extern "C" size_t vb_ring_attend_workspace(int B, int W, int H, int HKV, int DK) {
  if (B <= 0 || W <= 0 || H <= 0 || HKV <= 0 || DK <= 0) return 16;
  return sizeof(float) * (size_t)B * HKV * splits(W) * (H / HKV) * (DK + 2);
}

extern "C" int vb_ring_attend(const void* q, const void* k_new, const void* v_new, void* ring_k, void* ring_v,
                              int64_t* ring_pos, uint8_t* ring_valid, const int64_t* pos, void* o, void* workspace,
                              int B, int W, int H, int HKV, int DK, int window, int dtype, void* stream) {
  VB_REQUIRE(B >= 0 && W >= 1 && H >= 1 && HKV >= 1 && H % HKV == 0 && H / HKV <= GMAX,
             "ring_attend: bad shape B=%d W=%d H=%d HKV=%d", B, W, H, HKV);
  VB_REQUIRE(DK >= 1 && DK <= DKMAX, "ring_attend: head dimension %d must lie in [1, %d]", DK, DKMAX);
  VB_REQUIRE(window >= 1, "ring_attend: window %d must be at least 1", window);
  VB_REQUIRE(dtype == VB_F32 || dtype == VB_BF16 || dtype == VB_F16, "ring_attend: unsupported dtype %d", dtype);
  VB_REQUIRE(W <= WMAX, "ring_attend: %d slots exceed %d", W, WMAX);
  if (B == 0) return VB_OK;
  VB_REQUIRE(q && k_new && v_new && ring_k && ring_v && ring_pos && ring_valid && pos && o && workspace,
             "ring_attend: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const int G = H / HKV, nsplit = splits(W);
  const float scale = 1.0f / sqrtf((float)DK);
  const int L = SPLIT_SLOTS + 1;
  const size_t smem = sizeof(float) * ((size_t)G * DK + (size_t)G * L + (size_t)(NT / 32) * G * DK) + (size_t)L;
  float* part = (float*)workspace;
  const int ne = (DK + 31) / 32;
  return VB_DISPATCH_DTYPE(dtype, T, [&]() -> int {
    auto part_launch = [&](auto gc, auto nec) -> int {
      constexpr int GG = decltype(gc)::value, NN = decltype(nec)::value;
      if ((DK * (int)sizeof(T)) % 16 == 0 && aligned16(ring_k) && aligned16(ring_v) && aligned16(k_new) &&
          aligned16(v_new)) {
        const size_t sm2 = 2 * (size_t)L * DK * sizeof(T) + sizeof(float) * ((size_t)GG * DK + (size_t)GG * L) + L;
        VB_CUDA_CHECK(cudaFuncSetAttribute(ring_attn_part_staged_kernel<T, GG>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2),
                      "ring_attend: smem attribute");
        ring_attn_part_staged_kernel<T, GG><<<dim3(B, HKV, nsplit), NT, sm2, st>>>(
            (const T*)q, (const T*)k_new, (const T*)v_new, (const T*)ring_k, (const T*)ring_v, ring_pos, ring_valid,
            pos, part, W, H, HKV, DK, window, scale);
        VB_LAUNCH_CHECK("ring_attend part");
        return VB_OK;
      }
      VB_CUDA_CHECK(cudaFuncSetAttribute(ring_attn_part_kernel<T, GG, NN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                    "ring_attend: smem attribute");
      ring_attn_part_kernel<T, GG, NN><<<dim3(B, HKV, nsplit), NT, smem, st>>>(
          (const T*)q, (const T*)k_new, (const T*)v_new, (const T*)ring_k, (const T*)ring_v, ring_pos, ring_valid,
          pos, part, W, H, HKV, DK, window, scale);
      VB_LAUNCH_CHECK("ring_attend part");
      return VB_OK;
    };
    auto by_ne = [&](auto gc) -> int {
      switch (ne) {
        case 1: return part_launch(gc, std::integral_constant<int, 1>{});
        case 2: return part_launch(gc, std::integral_constant<int, 2>{});
        case 3: return part_launch(gc, std::integral_constant<int, 3>{});
        default: return part_launch(gc, std::integral_constant<int, 4>{});
      }
    };
    int rc = VB_OK;
    switch (G) {
      case 1: rc = by_ne(std::integral_constant<int, 1>{}); break;
      case 2: rc = by_ne(std::integral_constant<int, 2>{}); break;
      case 3: rc = by_ne(std::integral_constant<int, 3>{}); break;
      case 4: rc = by_ne(std::integral_constant<int, 4>{}); break;
      case 5: rc = by_ne(std::integral_constant<int, 5>{}); break;
      case 6: rc = by_ne(std::integral_constant<int, 6>{}); break;
      case 7: rc = by_ne(std::integral_constant<int, 7>{}); break;
      default: rc = by_ne(std::integral_constant<int, 8>{}); break;
    }
    if (rc) return rc;
    const int threads = G * DK < 1024 ? ((G * DK + 31) / 32) * 32 : 1024;
    ring_attn_merge_kernel<T><<<dim3(B, HKV), threads, 0, st>>>((const T*)k_new, (const T*)v_new, (T*)ring_k,
                                                                 (T*)ring_v, ring_pos, ring_valid, pos, part, (T*)o,
                                                                 nsplit, W, H, HKV, DK);
    VB_LAUNCH_CHECK("ring_attend merge");
    return VB_OK;
  });
}
