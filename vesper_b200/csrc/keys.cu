// The causal key filter with its key normalisation, forward and backward
// (vesper/column.py:255-289 RecurrentSublayer.keys; vesper/recurrence.py:91-115 normalize_keys).
//
// Layout: one warp walks a run of consecutive tokens of one (batch row, head); each lane holds
// EPL = head_dim/32 adjacent channels. The last K rows of the filter input stay in registers, so
// every element of z is read from HBM once (plus K-1 rows of overlap per run), and the key is
// written once. The backward walks its run in reverse with the next K-1 input gradients in
// registers, recomputing the filter output, and fuses dz, the taps' gradient (per-warp partial
// sums, reduced in a fixed order) and the history's gradient into the same pass. The forward can
// save each token's normalisation statistics (the reciprocals of scale and den, 8 bytes per token
// and head); the backward then skips recomputing them (two warp reductions, a square root and
// every quotient per token) and takes the clamp decision from them.
#include "common.cuh"

namespace vb {
int column_sum(const float* partial, float* out, int parts, int width, cudaStream_t st);

namespace {

constexpr int RUN = 64;        // tokens per warp
constexpr int WARPS = 4;       // warps per CTA
constexpr int PF = 8;          // input rows staged ahead of their use (a power of two)

// EPL consecutive elements at p (aligned to their total size, up to 16 bytes) as one access per
// 16 bytes, or one narrower access when they are fewer
template <typename T, int EPL>
__device__ __forceinline__ void ld_elems(const T* __restrict__ p, float (&out)[EPL]) {
  constexpr int BYTES = EPL * (int)sizeof(T);
  if constexpr (BYTES % 16 == 0) {
    load_vec<T, EPL>(p, out);
  } else if constexpr (BYTES == 8) {
    const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < EPL; ++i) out[i] = to_f32<T>(e[i]);
  } else if constexpr (BYTES == 4) {
    const unsigned raw = __ldg(reinterpret_cast<const unsigned*>(p));
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < EPL; ++i) out[i] = to_f32<T>(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) out[i] = to_f32<T>(p[i]);
  }
}
template <typename T, int EPL>
__device__ __forceinline__ void st_elems(T* __restrict__ p, const float (&in)[EPL]) {
  constexpr int BYTES = EPL * (int)sizeof(T);
  if constexpr (BYTES % 16 == 0) {
    store_vec<T, EPL>(p, in);
  } else if constexpr (BYTES == 8 || BYTES == 4) {
    T e[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) e[i] = from_f32<T>(in[i]);
    if constexpr (BYTES == 8) *reinterpret_cast<uint2*>(p) = *reinterpret_cast<const uint2*>(e);
    else *reinterpret_cast<unsigned*>(p) = *reinterpret_cast<const unsigned*>(e);
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) p[i] = from_f32<T>(in[i]);
  }
}

// ---- staging of input rows through shared memory (cp.async: the copies hold no registers) -----
template <int BYTES>
__device__ __forceinline__ void cp_async_bytes(uint32_t dst, const void* src) {
  static_assert(BYTES == 4 || BYTES == 8 || BYTES == 16, "cp.async copies 4, 8 or 16 bytes");
  asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(dst), "l"(src), "n"(BYTES) : "memory");
}
__device__ __forceinline__ void cp_async_commit_group() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// a lane's EPL elements of T from shared memory as floats
template <typename T, int EPL>
__device__ __forceinline__ void ld_staged(const uint8_t* p, float (&out)[EPL]) {
  const T* e = reinterpret_cast<const T*>(p);
#pragma unroll
  for (int i = 0; i < EPL; ++i) out[i] = to_f32<T>(e[i]);
}

// loads EPL channels [c, c+EPL) of row `t` of the filter input (z for t >= 0, else history)
template <typename T, int EPL>
__device__ __forceinline__ void load_in(const T* __restrict__ z, const float* __restrict__ hist,
                                        int b, int t, int T_, int W, int K, int c, bool live,
                                        float (&out)[EPL]) {
#pragma unroll
  for (int e = 0; e < EPL; ++e) out[e] = 0.f;
  if (!live) return;
  if (t >= 0) {
    ld_elems<T, EPL>(z + ((int64_t)b * T_ + t) * W + c, out);
  } else if (t >= -(K - 1)) {
    ld_elems<float, EPL>(hist + ((int64_t)b * (K - 1) + (K - 1 + t)) * W + c, out);
  }
}

// normalize_keys of one head vector spread over the warp: returns scale, s = u / scale (each
// quotient computed once and reused by the caller), den, sq
template <int EPL>
__device__ __forceinline__ void norm_stats(const float (&u)[EPL], float floor_, float& scale, float (&s)[EPL],
                                           float& den, float& sq) {
  float amax = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) amax = fmaxf(amax, fabsf(u[e]));
  scale = fmaxf(warp_max(amax), floor_);
  float s2 = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    s[e] = u[e] / scale;
    s2 += s[e] * s[e];
  }
  sq = warp_sum(s2);
  den = sqrtf(fmaxf(sq, 1.0f));
}

// normalize_keys of one head vector with one reduction of (max |u|, sum u^2) pairs. When the
// largest magnitude reaches the floor it IS the scale, its own quotient is exactly 1 and the sum
// of squared quotients is therefore at least 1: the clamp passes gradient with no quotient needed
// to decide it, and s = u * (1 / scale), sq = (sum u^2) / scale^2 (within an ulp or two of the
// quotients). Below the floor (a nearly zero vector) the exact quotients decide, as in
// norm_stats. Returns scale, 1 / scale, s, den, and whether the clamp passes gradient.
template <int EPL>
__device__ __forceinline__ void norm_stats_fast(const float (&u)[EPL], float floor_, float& scale, float& rscale,
                                                float (&s)[EPL], float& den, bool& clamped) {
  float amax = 0.f, ss = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    amax = fmaxf(amax, fabsf(u[e]));
    ss = fmaf(u[e], u[e], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
  }
  if (amax >= floor_) {  // warp-uniform
    scale = amax;
    rscale = 1.0f / scale;
#pragma unroll
    for (int e = 0; e < EPL; ++e) s[e] = u[e] * rscale;
    den = sqrtf(fmaxf(ss * rscale * rscale, 1.0f));
    clamped = true;
  } else {
    float sq;
    norm_stats<EPL>(u, floor_, scale, s, den, sq);
    rscale = 1.0f / scale;
    clamped = sq >= 1.0f;
  }
}

// EPL channels [c, c+EPL) of key-gradient row t (zero when the row is not needed)
template <typename T, int EPL>
__device__ __forceinline__ void load_g(const T* __restrict__ gk, int b, int t, int T_, int W, int c, bool need,
                                       float (&out)[EPL]) {
#pragma unroll
  for (int e = 0; e < EPL; ++e) out[e] = 0.f;
  if (!need || t < 0 || t >= T_) return;
  ld_elems<T, EPL>(gk + ((int64_t)b * T_ + t) * W + c, out);
}

// the filter input's gradient du of one token from its window w[r] = row t - r and its key
// gradient g (the normalisation's backward: (g / den - s (g . s) / den^3 [sq >= 1]) / scale).
// STATS: the forward's (1 / scale, 1 / den) of the token, the second negated when sq >= 1 (the
// clamp decision, taken from the forward's exact quotients); otherwise they are recomputed here.
template <int EPL, int K, bool STATS>
__device__ __forceinline__ void token_du(const float (&tp)[K][EPL], const float (&w)[K][EPL], const float (&g)[EPL],
                                         float floor_, float2 stat, float (&du)[EPL]) {
  float u[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    float a = 0.f;
#pragma unroll
    for (int r = 0; r < K; ++r) a = fmaf(tp[r][e], w[r][e], a);
    u[e] = a;
  }
  float s[EPL], rscale, rden;
  bool clamped;
  if constexpr (STATS) {
    rscale = stat.x;
    rden = fabsf(stat.y);
    clamped = stat.y < 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) s[e] = u[e] * rscale;  // within an ulp of u / scale: gradient only
  } else {
    float scale, den;
    norm_stats_fast<EPL>(u, floor_, scale, rscale, s, den, clamped);  // the forward's decision
    rden = 1.0f / den;
  }
  float dot = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) dot += g[e] * s[e];
  dot = warp_sum(dot);
  // the gradient's own quotients are products with the reciprocals of den and scale
  const float q = dot * (rden * rden * rden);
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    const float through = clamped ? s[e] * q : 0.f;
    du[e] = (g[e] * rden - through) * rscale;
  }
}

template <typename T, int EPL, int K>
__global__ void __launch_bounds__(WARPS * 32) keys_fwd_kernel(const T* __restrict__ z,
                                                              const float* __restrict__ hist,
                                                              const float* __restrict__ taps,
                                                              T* __restrict__ out,
                                                              float2* __restrict__ stats, int B,
                                                              int T_, int W, int heads, int runs,
                                                              float floor_) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (gw >= B * heads * runs) return;
  const int run = gw % runs, head = (gw / runs) % heads, b = gw / (runs * heads);
  const int hd = W / heads;
  const bool live = lane * EPL < hd;  // head widths below 32 leave lanes idle
  const int c = head * hd + lane * EPL;
  float tp[K][EPL];
#pragma unroll
  for (int r = 0; r < K; ++r)
#pragma unroll
    for (int e = 0; e < EPL; ++e) tp[r][e] = live ? __ldg(taps + (int64_t)r * W + c + e) : 0.f;
  const int t0 = run * RUN, t1 = min(T_, t0 + RUN);
  float win[K][EPL];  // win[r] = input row t - r
  float2 st_pair = make_float2(0.f, 0.f);
#pragma unroll
  for (int r = 1; r < K; ++r) load_in<T, EPL>(z, hist, b, t0 - r, T_, W, K, c, live, win[r]);
  // the run's input rows stream PF rows ahead of their use through a per-warp ring in shared
  // memory (each lane copies and later reads only its own EPL elements): the copies hold no
  // registers, so the load latency leaves the per-token chain without costing occupancy
  constexpr int BYTES = EPL * (int)sizeof(T);
  constexpr bool STAGED = BYTES == 4 || BYTES == 8 || BYTES == 16;
  __shared__ __align__(16) uint8_t ring[WARPS][PF][32][STAGED ? BYTES : 16];
  uint8_t(*mine)[32][STAGED ? BYTES : 16] = ring[threadIdx.x >> 5];
  auto issue = [&](int t) {
    if constexpr (STAGED) {
      if (live && t < t1) cp_async_bytes<BYTES>(smem_addr(mine[(t - t0) & (PF - 1)][lane]), z + ((int64_t)b * T_ + t) * W + c);
      cp_async_commit_group();
    }
  };
#pragma unroll
  for (int i = 0; i < PF; ++i) issue(t0 + i);
  for (int t = t0; t < t1; ++t) {
    if constexpr (STAGED) {
      cp_async_wait_group<PF - 1>();  // row t's group is the oldest of PF in flight
      if (live) ld_staged<T, EPL>(mine[(t - t0) & (PF - 1)][lane], win[0]);
      else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) win[0][e] = 0.f;
      }
      issue(t + PF);  // the slot's row has been read into registers
    } else {
      load_in<T, EPL>(z, hist, b, t, T_, W, K, c, live, win[0]);
    }
    float u[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      float a = 0.f;
#pragma unroll
      for (int r = 0; r < K; ++r) a = fmaf(tp[r][e], win[r][e], a);
      u[e] = a;
    }
    float scale, rscale, s[EPL], den;
    bool clamped;
    norm_stats_fast<EPL>(u, floor_, scale, rscale, s, den, clamped);
    const float rden = 1.0f / den;  // k = s / den to within an ulp or two of the quotient
    if (live) {
      float o[EPL];
#pragma unroll
      for (int e = 0; e < EPL; ++e) o[e] = s[e] * rden;
      st_elems<T, EPL>(out + ((int64_t)b * T_ + t) * W + c, o);
    }
    // (1 / scale, 1 / den), the second negated where the clamp passes gradient: token t's pair
    // waits in lane (t - t0) % 32, and each 32 tokens leave as one contiguous warp store
    // ([B, heads, T, 2])
    const int slot = (t - t0) & 31;
    if (lane == slot) st_pair = make_float2(rscale, clamped ? -rden : rden);
    if (stats != nullptr && (slot == 31 || t + 1 == t1) && lane <= slot)
      stats[((int64_t)b * heads + head) * T_ + (t - slot + lane)] = st_pair;
#pragma unroll
    for (int r = K - 1; r > 0; --r)
#pragma unroll
      for (int e = 0; e < EPL; ++e) win[r][e] = win[r - 1][e];
  }
}

// Backward over one run in reverse. partial: [B * runs, K, W] taps-gradient partial sums; stats:
// the forward's per-token (scale, +-den) when STATS, else recomputed.
template <typename T, int EPL, int K, bool STATS>
__global__ void __launch_bounds__(WARPS * 32) keys_bwd_kernel(
    const T* __restrict__ z, const float* __restrict__ hist, const float* __restrict__ taps,
    const T* __restrict__ gk, const float2* __restrict__ stats, T* __restrict__ dz, float* __restrict__ dhist,
    float* __restrict__ partial, int B, int T_, int W, int heads, int runs, float floor_) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (gw >= B * heads * runs) return;
  const int run = gw % runs, head = (gw / runs) % heads, b = gw / (runs * heads);
  const int hd = W / heads;
  const bool live = lane * EPL < hd;
  const int c = head * hd + lane * EPL;
  float tp[K][EPL];
#pragma unroll
  for (int r = 0; r < K; ++r)
#pragma unroll
    for (int e = 0; e < EPL; ++e) tp[r][e] = live ? __ldg(taps + (int64_t)r * W + c + e) : 0.f;
  const int t0 = run * RUN, t1 = min(T_, t0 + RUN);
  const int thi = min(T_ - 1, t1 + K - 2);  // the next run's first K-1 gradients are recomputed
  float win[K][EPL];   // win[r] = input row t - r
  float dring[K][EPL]; // dring[r] = du at t + r
  float dt[K][EPL];    // taps gradient over this run
#pragma unroll
  for (int r = 0; r < K; ++r)
#pragma unroll
    for (int e = 0; e < EPL; ++e) { dring[r][e] = 0.f; dt[r][e] = 0.f; }
  // before the step for token t the window holds the rows of step t + 1: win[r] = row t + 1 - r
#pragma unroll
  for (int r = 0; r < K; ++r) load_in<T, EPL>(z, hist, b, thi + 1 - r, T_, W, K, c, live && r > 0, win[r]);
  // tokens go in pairs: the two tokens' input gradients (their reductions independent) are formed
  // together, then each enters the ring in turn, in the order of a one-token walk
  auto step = [&](int t, const float (&du)[EPL], const float (&w)[K][EPL]) {
    // shift the gradient ring: dring[r] <- du at t + r
#pragma unroll
    for (int r = K - 1; r > 0; --r)
#pragma unroll
      for (int e = 0; e < EPL; ++e) dring[r][e] = dring[r - 1][e];
#pragma unroll
    for (int e = 0; e < EPL; ++e) dring[0][e] = du[e];
    if (t < t1) {
#pragma unroll
      for (int r = 0; r < K; ++r)
#pragma unroll
        for (int e = 0; e < EPL; ++e) dt[r][e] = fmaf(dring[0][e], w[r][e], dt[r][e]);
      float o[EPL];
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        float a = 0.f;
#pragma unroll
        for (int r = 0; r < K; ++r)
          if (t + r < T_) a = fmaf(tp[r][e], dring[r][e], a);
        o[e] = a;
      }
      if (live) st_elems<T, EPL>(dz + ((int64_t)b * T_ + t) * W + c, o);
    }
  };
  // the walk's inputs stream PF tokens ahead through a per-warp ring in shared memory: item t
  // (t = thi, thi - 1, ..., t0) is input row t - K + 1 (history rows, t - K + 1 < 0, are read
  // directly), key-gradient row t and, with STATS, the token's saved pair (copied by lane 0)
  constexpr int BYTES = EPL * (int)sizeof(T);
  constexpr bool STAGED = BYTES == 4 || BYTES == 8 || BYTES == 16;
  constexpr int SB = STAGED ? BYTES : 16;
  __shared__ __align__(16) uint8_t ring[WARPS][PF][2][32][SB];
  __shared__ __align__(8) float2 sring[WARPS][PF];
  const int wi = threadIdx.x >> 5;
  const float2* st_row = STATS ? stats + ((int64_t)b * heads + head) * T_ : nullptr;
  auto issue = [&](int t) {
    if constexpr (STAGED) {
      if (t >= t0) {
        const int slot = (thi - t) & (PF - 1), zr = t - K + 1;
        if (live && zr >= 0) cp_async_bytes<BYTES>(smem_addr(ring[wi][slot][0][lane]), z + ((int64_t)b * T_ + zr) * W + c);
        if (live) cp_async_bytes<BYTES>(smem_addr(ring[wi][slot][1][lane]), gk + ((int64_t)b * T_ + t) * W + c);
        if (STATS && lane == 0) cp_async_bytes<8>(smem_addr(&sring[wi][slot]), st_row + t);
      }
      cp_async_commit_group();
    }
  };
  // token t's new window row (t - K + 1), key gradient and saved pair
  auto take = [&](int t, float (&zrow)[EPL], float (&g)[EPL], float2& stat) {
    if constexpr (STAGED) {
      cp_async_wait_group<PF - 1>();  // item t's group is the oldest of PF in flight
      __syncwarp();                   // lane 0's copy of the pair is visible to the warp
      const int slot = (thi - t) & (PF - 1), zr = t - K + 1;
      if (live && zr >= 0) ld_staged<T, EPL>(ring[wi][slot][0][lane], zrow);
      else load_in<T, EPL>(z, hist, b, zr, T_, W, K, c, live, zrow);
      if (live) ld_staged<T, EPL>(ring[wi][slot][1][lane], g);
      else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) g[e] = 0.f;
      }
      if constexpr (STATS) stat = sring[wi][slot];
      __syncwarp();  // every lane has read the slot before it is refilled
      issue(t - PF);
    } else {
      load_in<T, EPL>(z, hist, b, t - K + 1, T_, W, K, c, live, zrow);
      load_g<T, EPL>(gk, b, t, T_, W, c, live, g);
      if constexpr (STATS) stat = __ldg(st_row + t);
    }
  };
#pragma unroll
  for (int i = 0; i < PF; ++i) issue(thi - i);
  for (int t = thi; t >= t0; t -= 2) {
    const bool two = t - 1 >= t0;
    // token t's window: win[r] = row t - r (one row older than before); token t - 1's: wb
#pragma unroll
    for (int r = 0; r < K - 1; ++r)
#pragma unroll
      for (int e = 0; e < EPL; ++e) win[r][e] = win[r + 1][e];
    float ga[EPL], gb[EPL];
    float2 sa = make_float2(1.f, 1.f), sb = sa;
    take(t, win[K - 1], ga, sa);
    float wb[K][EPL];
#pragma unroll
    for (int r = 0; r < K - 1; ++r)
#pragma unroll
      for (int e = 0; e < EPL; ++e) wb[r][e] = win[r + 1][e];
    if (two) take(t - 1, wb[K - 1], gb, sb);
    else {
#pragma unroll
      for (int e = 0; e < EPL; ++e) { wb[K - 1][e] = 0.f; gb[e] = 0.f; }
    }
    float da[EPL], db[EPL];
    token_du<EPL, K, STATS>(tp, win, ga, floor_, sa, da);
    token_du<EPL, K, STATS>(tp, wb, gb, floor_, sb, db);
    step(t, da, win);
    if (two) {
#pragma unroll
      for (int r = 0; r < K; ++r)
#pragma unroll
        for (int e = 0; e < EPL; ++e) win[r][e] = wb[r][e];
      step(t - 1, db, win);
    }
  }
  if constexpr (STAGED) cp_async_wait_group<0>();
  if (live) {
    float* p = partial + (((int64_t)b * runs + run) * K) * W + c;
#pragma unroll
    for (int r = 0; r < K; ++r)
#pragma unroll
      for (int e = 0; e < EPL; ++e) p[(int64_t)r * W + e] = dt[r][e];
  }
  // history rows p = 0..K-2 feed u[t] for t = p - (K-1) + r >= 0; dring[r] = du at t0 + r = r
  if (dhist != nullptr && run == 0 && live) {
#pragma unroll
    for (int p = 0; p < K - 1; ++p) {
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        float a = 0.f;
#pragma unroll
        for (int r = 0; r < K; ++r) {
          const int t = p - (K - 1) + r;
          if (t >= 0 && t < T_) a = fmaf(tp[r][e], dring[t][e], a);
        }
        dhist[((int64_t)b * (K - 1) + p) * W + c + e] = a;
      }
    }
  }
}

template <typename T, int EPL>
int launch_fwd(const void* z, const float* hist, const float* taps, void* out, float* stats, int B, int T_,
               int W, int heads, int K, float floor_, cudaStream_t st) {
  const int runs = (T_ + RUN - 1) / RUN;
  const int warps = B * heads * runs;
  const int ctas = (warps + WARPS - 1) / WARPS;
#define VB_KEYS_FWD(KK)                                                                          \
  case KK:                                                                                       \
    keys_fwd_kernel<T, EPL, KK><<<ctas, WARPS * 32, 0, st>>>((const T*)z, hist, taps, (T*)out,  \
                                                             (float2*)stats, B, T_, W, heads,   \
                                                             runs, floor_);                     \
    break;
  switch (K) {
    VB_KEYS_FWD(1) VB_KEYS_FWD(2) VB_KEYS_FWD(3) VB_KEYS_FWD(4)
    VB_KEYS_FWD(5) VB_KEYS_FWD(6) VB_KEYS_FWD(7) VB_KEYS_FWD(8)
    default: set_error("keys: filter width %d not in [1, 8]", K); return VB_ERR_INVALID;
  }
#undef VB_KEYS_FWD
  VB_LAUNCH_CHECK("keys_fwd");
  return VB_OK;
}

template <typename T, int EPL>
int launch_bwd(const void* z, const float* hist, const float* taps, const void* gk, const float* stats,
               void* dz, float* dtaps, float* dhist, float* partial, int B, int T_, int W, int heads,
               int K, float floor_, cudaStream_t st) {
  const int runs = (T_ + RUN - 1) / RUN;
  const int warps = B * heads * runs;
  const int ctas = (warps + WARPS - 1) / WARPS;
#define VB_KEYS_BWD(KK)                                                                            \
  case KK:                                                                                         \
    if (stats != nullptr)                                                                          \
      keys_bwd_kernel<T, EPL, KK, true><<<ctas, WARPS * 32, 0, st>>>(                              \
          (const T*)z, hist, taps, (const T*)gk, (const float2*)stats, (T*)dz, dhist, partial, B, T_, \
          W, heads, runs, floor_);                                                                 \
    else                                                                                           \
      keys_bwd_kernel<T, EPL, KK, false><<<ctas, WARPS * 32, 0, st>>>(                             \
          (const T*)z, hist, taps, (const T*)gk, nullptr, (T*)dz, dhist, partial, B, T_, W, heads, \
          runs, floor_);                                                                           \
    break;
  switch (K) {
    VB_KEYS_BWD(1) VB_KEYS_BWD(2) VB_KEYS_BWD(3) VB_KEYS_BWD(4)
    VB_KEYS_BWD(5) VB_KEYS_BWD(6) VB_KEYS_BWD(7) VB_KEYS_BWD(8)
    default: set_error("keys: filter width %d not in [1, 8]", K); return VB_ERR_INVALID;
  }
#undef VB_KEYS_BWD
  VB_LAUNCH_CHECK("keys_bwd");
  return column_sum(partial, dtaps, B * runs, K * W, st);
}

int check_shape(int B, int T_, int W, int heads, int K) {
  VB_REQUIRE(B >= 0 && T_ >= 0 && W > 0 && heads > 0 && W % heads == 0,
             "keys: bad shape B=%d T=%d W=%d heads=%d", B, T_, W, heads);
  const int hd = W / heads;
  VB_REQUIRE((hd & (hd - 1)) == 0 && hd >= 1 && hd <= 256,
             "keys: head width %d must be a power of two up to 256", hd);
  VB_REQUIRE(K >= 1 && K <= 8, "keys: filter width %d not in [1, 8]", K);
  return VB_OK;
}

}  // namespace
}  // namespace vb

using namespace vb;

#define VB_KEYS_EPL_DISPATCH(hd, EPL, ...)       \
  [&]() -> int {                                 \
    if (hd <= 32) { constexpr int EPL = 1; return __VA_ARGS__(); } \
    if (hd == 64) { constexpr int EPL = 2; return __VA_ARGS__(); } \
    if (hd == 128) { constexpr int EPL = 4; return __VA_ARGS__(); } \
    { constexpr int EPL = 8; return __VA_ARGS__(); }               \
  }()

extern "C" int vb_keys_fwd(const void* z, const float* hist, const float* taps, void* keys, float* stats,
                           int B, int T, int width, int heads, int taps_count, float floor_, int dtype,
                           void* stream) {
  int rc = check_shape(B, T, width, heads, taps_count);
  if (rc) return rc;
  if (B == 0 || T == 0) return VB_OK;
  VB_REQUIRE(z && taps && keys && (hist || taps_count == 1), "keys_fwd: null pointer");
  VB_REQUIRE(aligned16(z) && aligned16(keys) && (!hist || aligned16(hist)),
             "keys_fwd: z, keys and history must start on 16-byte boundaries");
  VB_REQUIRE(((uintptr_t)stats & 7u) == 0, "keys_fwd: stats must start on an 8-byte boundary");
  const int hd = width / heads;
  cudaStream_t st = (cudaStream_t)stream;
  return VB_DISPATCH_DTYPE(dtype, Tt, [&]() -> int {
    return VB_KEYS_EPL_DISPATCH(hd, EPL, [&]() -> int {
      return launch_fwd<Tt, EPL>(z, hist, taps, keys, stats, B, T, width, heads, taps_count, floor_, st);
    });
  });
}

extern "C" size_t vb_keys_bwd_workspace(int B, int T, int width, int heads, int taps_count) {
  const int runs = (T + RUN - 1) / RUN;
  const size_t parts = (size_t)(B > 0 ? B : 1) * (size_t)(runs > 0 ? runs : 1);
  return parts * (size_t)(taps_count > 0 ? taps_count : 1) * (size_t)(width > 0 ? width : 1) * sizeof(float);
}

extern "C" int vb_keys_bwd(const void* z, const float* hist, const float* taps, const void* grad_keys,
                           const float* stats, void* grad_z, float* grad_taps, float* grad_hist,
                           void* workspace, int B, int T, int width, int heads, int taps_count,
                           float floor_, int dtype, void* stream) {
  int rc = check_shape(B, T, width, heads, taps_count);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  if (B == 0 || T == 0) {
    VB_CUDA_CHECK(cudaMemsetAsync(grad_taps, 0, sizeof(float) * taps_count * width, st), "keys_bwd");
    if (grad_hist && B > 0)
      VB_CUDA_CHECK(cudaMemsetAsync(grad_hist, 0, sizeof(float) * B * (taps_count - 1) * width, st),
                    "keys_bwd");
    return VB_OK;
  }
  VB_REQUIRE(z && taps && grad_keys && grad_z && grad_taps && workspace && (hist || taps_count == 1),
             "keys_bwd: null pointer");
  VB_REQUIRE(aligned16(z) && aligned16(grad_keys) && aligned16(grad_z) && (!hist || aligned16(hist)),
             "keys_bwd: z, the key gradient, dz and history must start on 16-byte boundaries");
  VB_REQUIRE(((uintptr_t)stats & 7u) == 0, "keys_bwd: stats must start on an 8-byte boundary");
  const int hd = width / heads;
  return VB_DISPATCH_DTYPE(dtype, Tt, [&]() -> int {
    return VB_KEYS_EPL_DISPATCH(hd, EPL, [&]() -> int {
      return launch_bwd<Tt, EPL>(z, hist, taps, grad_keys, stats, grad_z, grad_taps, grad_hist,
                                 (float*)workspace, B, T, width, heads, taps_count, floor_, st);
    });
  });
}
