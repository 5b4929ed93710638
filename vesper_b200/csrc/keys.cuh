// The causal key filter with its key normalisation, forward and backward
// (vesper/column.py:255-289 RecurrentSublayer.keys; vesper/recurrence.py:91-115 normalize_keys).
//
// The key of a head vector u (the filter output) is u / max(||u||, floor). The reference forms it
// scale-safely: prescaled by s = max(max|u|, floor), then divided by max(sqrt(sum (u / s)^2), 1).
// Wherever sum u^2 lies in [2 floor^2, 2^100] no square overflows, the reference's squared
// quotient sum is at least 1 (the clamp passes gradient) and its key is u / ||u||: the forward
// forms k = u rsqrt(sum u^2) with no branch, and a head vector outside that range (nearly zero, or
// huge) is redone with the reference's prescaled steps and exact quotients after its group of
// tokens. With r = 1 / max(||u||, floor) and the clamp decision c, the key is u r and the
// normalisation's backward is du = r (g - c k (g . k)): the forward saves (r, +-1) per token and
// head (-1 where c holds), and the backward needs nothing else from it.
//
// Layout: a warp walks a run of tokens over a span of 32 * EPL channels: whole heads, G = hd / EPL
// lanes per head, 32 / G heads per warp (the forward takes 16-byte rows per lane: two heads of 128
// bf16 channels per warp; the backward 8 or 16 bytes, one head). Every per-token reduction is over
// the G lanes of a head. The filter window (the last K input rows) is a ring of registers indexed
// at compile time (the token loop is unrolled by K, so the window never moves). Input rows stream
// through a per-warp ring in shared memory by cp.async, about 16 rows ahead of their use, so the
// copies hold no registers. Each element of z is read from HBM once (plus K-1 rows of overlap per
// run, mostly from L2) and each key is written once.
//
// The backward walks its run forward: token t's input gradient du[t] adds taps[r] du[t] to
// dz[t - r] in a register ring of K accumulators, and dz[t - K] is complete (and stored) when token
// t starts its slot. A run recomputes du for the next run's first K-1 tokens, the taps' gradient is
// a per-warp partial sum (reduced in a fixed order afterwards), and run 0 writes the history's
// gradient from the ring.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace vb {
int column_sum(const float* partial, float* out, int parts, int width, cudaStream_t st);

namespace {

constexpr int WARPS = 4;      // warps per CTA
constexpr int RUN_F = 64;     // tokens per forward warp (rounded up to a multiple of K)
constexpr int RUN_B = 128;    // tokens per backward warp (rounded up to a multiple of K)
constexpr float FAST_MAX = 0x1p50f;  // max|u| up to here: sum u^2 is a normal float (backward)

// the run length of a warp: at least `base` tokens, a multiple of the unrolled step
__host__ __device__ constexpr int run_len(int base, int step) { return step * ((base + step - 1) / step); }

// ---- one lane's EPL elements of a row, raw (converted at use) --------------------------------
template <typename T, int EPL>
struct Raw {
  static constexpr int BYTES = EPL * (int)sizeof(T);
  static constexpr int WORDS = BYTES >= 16 ? BYTES / 16 : 1;
  uint4 w[WORDS];
};

template <typename T, int EPL>
__device__ __forceinline__ void raw_load(Raw<T, EPL>& r, const T* p, bool ok) {
  constexpr int BYTES = Raw<T, EPL>::BYTES;
  if constexpr (BYTES >= 16) {
#pragma unroll
    for (int i = 0; i < Raw<T, EPL>::WORDS; ++i)
      r.w[i] = ok ? __ldg(reinterpret_cast<const uint4*>(p) + i) : make_uint4(0u, 0u, 0u, 0u);
  } else if constexpr (BYTES == 8) {
    const uint2 v = ok ? __ldg(reinterpret_cast<const uint2*>(p)) : make_uint2(0u, 0u);
    r.w[0] = make_uint4(v.x, v.y, 0u, 0u);
  } else if constexpr (BYTES == 4) {
    r.w[0] = make_uint4(ok ? __ldg(reinterpret_cast<const unsigned*>(p)) : 0u, 0u, 0u, 0u);
  } else {
    r.w[0] = make_uint4(ok ? (unsigned)__ldg(reinterpret_cast<const unsigned short*>(p)) : 0u, 0u, 0u, 0u);
  }
}

template <typename T, int EPL>
__device__ __forceinline__ void raw_f32(const Raw<T, EPL>& r, float (&out)[EPL]) {
  const T* e = reinterpret_cast<const T*>(r.w);
#pragma unroll
  for (int i = 0; i < EPL; ++i) out[i] = to_f32<T>(e[i]);
}

// ---- rows staged through shared memory by cp.async (the copies hold no registers) -----------
// A warp's ring holds PF rows of one stream (each lane copies and later reads only its own
// bytes, so no barrier is needed); one commit group per token, so waiting until at most PF - 1
// groups are pending makes the oldest row visible to the lane that copied it.
template <int BYTES>
__device__ __forceinline__ void cp_async_row(uint32_t dst, const void* src, bool ok) {
  if constexpr (BYTES == 16 || BYTES == 32) {
#pragma unroll
    for (int i = 0; i < BYTES / 16; ++i)
      asm volatile("{ .reg .pred p; setp.ne.b32 p, %2, 0;\n @p cp.async.cg.shared.global [%0], [%1], 16; }"
                   ::"r"(dst + 16 * i), "l"((const uint8_t*)src + 16 * i), "r"((int)ok) : "memory");
  } else {
    asm volatile("{ .reg .pred p; setp.ne.b32 p, %2, 0;\n @p cp.async.ca.shared.global [%0], [%1], %3; }"
                 ::"r"(dst), "l"(src), "r"((int)ok), "n"(BYTES) : "memory");
  }
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// a lane's staged row: zero where the copy was skipped is not needed (skipped rows are never read)
template <typename T, int EPL>
__device__ __forceinline__ void staged_f32(uint32_t src, float (&out)[EPL]) {
  constexpr int BYTES = EPL * (int)sizeof(T);
  Raw<T, EPL> r;
  if constexpr (BYTES >= 16) {
#pragma unroll
    for (int i = 0; i < BYTES / 16; ++i)
      asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(r.w[i].x), "=r"(r.w[i].y), "=r"(r.w[i].z), "=r"(r.w[i].w) : "r"(src + 16 * i));
  } else if constexpr (BYTES == 8) {
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(r.w[0].x), "=r"(r.w[0].y) : "r"(src));
  } else {
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(r.w[0].x) : "r"(src));
  }
  raw_f32<T, EPL>(r, out);
}

// rows in flight per warp and stream: 8 KB of ring per warp in all (at most 16 rows)
template <int BYTES, int STREAMS>
__host__ __device__ constexpr int ring_rows() {
  return (8192 / STREAMS) / (32 * BYTES) > 16 ? 16 : (8192 / STREAMS) / (32 * BYTES);
}
template <int BYTES>
__host__ __device__ constexpr bool stageable() { return BYTES == 4 || BYTES == 8 || BYTES == 16 || BYTES == 32; }

// EPL consecutive floats at p (aligned to their total size, at most 16 bytes per access)
template <int EPL>
__device__ __forceinline__ void ld_f32(const float* __restrict__ p, float (&out)[EPL]) {
  if constexpr (EPL % 4 == 0) {
#pragma unroll
    for (int i = 0; i < EPL / 4; ++i) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p) + i);
      out[4 * i] = v.x; out[4 * i + 1] = v.y; out[4 * i + 2] = v.z; out[4 * i + 3] = v.w;
    }
  } else if constexpr (EPL == 2) {
    const float2 v = __ldg(reinterpret_cast<const float2*>(p));
    out[0] = v.x; out[1] = v.y;
  } else {
    out[0] = __ldg(p);
  }
}

template <typename T, int EPL>
__device__ __forceinline__ void st_row(T* __restrict__ p, const float (&in)[EPL]) {
  constexpr int BYTES = EPL * (int)sizeof(T);
  if constexpr (BYTES % 16 == 0) {
    store_vec<T, EPL>(p, in);
  } else {
    T e[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) e[i] = from_f32<T>(in[i]);
    if constexpr (BYTES == 8) *reinterpret_cast<uint2*>(p) = *reinterpret_cast<const uint2*>(e);
    else if constexpr (BYTES == 4) *reinterpret_cast<unsigned*>(p) = *reinterpret_cast<const unsigned*>(e);
    else *p = e[0];
  }
}

template <int EPL>
__device__ __forceinline__ void st_f32(float* __restrict__ p, const float (&in)[EPL]) {
  if constexpr (EPL % 4 == 0) {
#pragma unroll
    for (int i = 0; i < EPL / 4; ++i)
      reinterpret_cast<float4*>(p)[i] = make_float4(in[4 * i], in[4 * i + 1], in[4 * i + 2], in[4 * i + 3]);
  } else if constexpr (EPL == 2) {
    *reinterpret_cast<float2*>(p) = make_float2(in[0], in[1]);
  } else {
    *p = in[0];
  }
}

// sums / maxima over the G lanes of a head (G a power of two up to 32, the same on every lane)
// Element-wise float32 arithmetic over a row of EPL values, two lanes of the row per instruction
// where EPL is even (the packed f32x2 FMA and product of sm_100: each lane rounds exactly as
// fmaf / a product do, so the results equal the scalar ones bit for bit).
// d = a * b + c
template <int N>
__device__ __forceinline__ void fma_row(float (&d)[N], const float (&a)[N], const float (&b)[N], const float (&c)[N]) {
  if constexpr (N % 2 == 0) {
#pragma unroll
    for (int e = 0; e < N; e += 2) {
      const float2 r = __ffma2_rn(make_float2(a[e], a[e + 1]), make_float2(b[e], b[e + 1]), make_float2(c[e], c[e + 1]));
      d[e] = r.x;
      d[e + 1] = r.y;
    }
  } else {
#pragma unroll
    for (int e = 0; e < N; ++e) d[e] = fmaf(a[e], b[e], c[e]);
  }
}
// d = s * b + c (s one value for the row)
template <int N>
__device__ __forceinline__ void fma_row(float (&d)[N], float s, const float (&b)[N], const float (&c)[N]) {
  if constexpr (N % 2 == 0) {
#pragma unroll
    for (int e = 0; e < N; e += 2) {
      const float2 r = __ffma2_rn(make_float2(s, s), make_float2(b[e], b[e + 1]), make_float2(c[e], c[e + 1]));
      d[e] = r.x;
      d[e + 1] = r.y;
    }
  } else {
#pragma unroll
    for (int e = 0; e < N; ++e) d[e] = fmaf(s, b[e], c[e]);
  }
}
// d = a * b
template <int N>
__device__ __forceinline__ void mul_row(float (&d)[N], const float (&a)[N], const float (&b)[N]) {
  if constexpr (N % 2 == 0) {
#pragma unroll
    for (int e = 0; e < N; e += 2) {
      const float2 r = __fmul2_rn(make_float2(a[e], a[e + 1]), make_float2(b[e], b[e + 1]));
      d[e] = r.x;
      d[e + 1] = r.y;
    }
  } else {
#pragma unroll
    for (int e = 0; e < N; ++e) d[e] = a[e] * b[e];
  }
}
// d = s * b
template <int N>
__device__ __forceinline__ void mul_row(float (&d)[N], float s, const float (&b)[N]) {
  if constexpr (N % 2 == 0) {
#pragma unroll
    for (int e = 0; e < N; e += 2) {
      const float2 r = __fmul2_rn(make_float2(s, s), make_float2(b[e], b[e + 1]));
      d[e] = r.x;
      d[e + 1] = r.y;
    }
  } else {
#pragma unroll
    for (int e = 0; e < N; ++e) d[e] = s * b[e];
  }
}

__device__ __forceinline__ float group_sum(float v, int G) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    if (o < G) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float group_max(float v, int G) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    if (o < G) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// normalize_keys of a head vector spread over G lanes: the key k (in place of u), r and c. Every
// lane of the warp calls it (the reductions are warp-wide shuffles).
template <int EPL>
__device__ __forceinline__ void normalize(float (&k)[EPL], int G, float floor_, float& r, bool& clamp) {
  float amax = 0.f, ss = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    amax = fmaxf(amax, fabsf(k[e]));
    ss = fmaf(k[e], k[e], ss);
  }
  amax = group_max(amax, G);
  ss = group_sum(ss, G);
  const bool fast = amax >= floor_ && amax <= FAST_MAX;
  r = rsqrtf(ss);
  clamp = true;
  if (__any_sync(0xffffffffu, !fast)) {
    // the reference's prescaled steps with exact quotients (a head vector below the floor or huge)
    const float scale = fmaxf(amax, floor_);
    float s[EPL], s2 = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      s[e] = k[e] / scale;
      s2 = fmaf(s[e], s[e], s2);
    }
    const float sq = group_sum(s2, G);
    const float den = sqrtf(fmaxf(sq, 1.0f));
    if (!fast) {
#pragma unroll
      for (int e = 0; e < EPL; ++e) k[e] = s[e] / den;
      r = (1.0f / scale) * (1.0f / den);
      clamp = sq >= 1.0f;
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < EPL; ++e) k[e] *= r;
}

// Which warp does what: warp gw -> (b, span, run), runs fastest (neighbouring runs share rows in L2)
struct Walk {
  int b, span, run, c, head, G;
  bool live;
};
__device__ __forceinline__ Walk walk_of(int gw, int spans, int runs, int W, int hd, int epl) {
  Walk w;
  w.run = gw % runs;
  w.span = (gw / runs) % spans;
  w.b = gw / (runs * spans);
  const int lane = threadIdx.x & 31;
  w.c = w.span * 32 * epl + lane * epl;
  w.live = w.c < W;
  w.head = min(w.c, W - 1) / hd;
  w.G = hd / epl;
  return w;
}

// the window rows t0-K+1 .. t0-1 into slots 1..K-1 (z rows, history rows before token 0, zeros
// for a lane past the width); slot 0 is filled by token t0
template <typename T, int EPL, int K>
__device__ __forceinline__ void window_init(float (&win)[K][EPL], const T* __restrict__ z, const float* __restrict__ hist,
                                            const Walk& w, int t0, int T_, int W) {
#pragma unroll
  for (int s = 0; s < K; ++s) {
#pragma unroll
    for (int e = 0; e < EPL; ++e) win[s][e] = 0.f;
    const int row = t0 - K + s;
    if (s == 0 || !w.live) continue;
    if (row >= 0) {
      Raw<T, EPL> raw;
      raw_load<T, EPL>(raw, z + ((int64_t)w.b * T_ + row) * W + w.c, true);
      raw_f32<T, EPL>(raw, win[s]);
    } else {
      ld_f32<EPL>(hist + ((int64_t)w.b * (K - 1) + (K - 1 + row)) * W + w.c, win[s]);
    }
  }
}

// The fast path of normalize_keys for one token, with no branch: k = u rsqrt(sum u^2), and
// whether that is the reference's key (`fast`). It is wherever sum u^2 >= 2 floor^2: then the
// reference's squared quotient sum (over max|u| or the floor) is at least 1 with room for its
// rounding, the clamp passes gradient and its key u / (scale sqrt(sum (u / scale)^2)) is
// u / ||u||; and wherever sum u^2 <= 2^100, which no square or sum overflows.
template <int EPL>
__device__ __forceinline__ void normalize_fast(float (&k)[EPL], int G, float floor_, float& r, bool& fast) {
  float s0 = 0.f, s1 = 0.f;  // two partial sums: half the dependent chain
#pragma unroll
  for (int e = 0; e < EPL; e += 2) {
    s0 = fmaf(k[e], k[e], s0);
    if (e + 1 < EPL) s1 = fmaf(k[e + 1], k[e + 1], s1);
  }
  const float ss = group_sum(s0 + s1, G);
  fast = ss >= 2.0f * floor_ * floor_ && ss <= 0x1p100f;
  r = rsqrtf(ss);
#pragma unroll
  for (int e = 0; e < EPL; ++e) k[e] *= r;
}

// Token tok again for the heads of this warp whose vector left the fast range (`mine`): the
// window reloaded, the reference's prescaled steps, the key and its (r, +-1) stored over the fast
// path's. Every lane of the warp calls it (rare: nearly zero or huge head vectors).
template <typename T, int EPL, int K>
__device__ __noinline__ void fix_token(const T* __restrict__ z, const float* __restrict__ hist,
                                       const float* __restrict__ taps, T* __restrict__ out, float2* __restrict__ sp,
                                       int b, int tok, int T_, int W, int c, bool live, int G, float floor_,
                                       bool mine) {
  float k[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) k[e] = 0.f;
  if (live) {
    for (int r = 0; r < K; ++r) {
      const int row = tok - r;
      float v[EPL];
#pragma unroll
      for (int e = 0; e < EPL; ++e) v[e] = 0.f;
      if (row >= 0) {
        Raw<T, EPL> raw;
        raw_load<T, EPL>(raw, z + ((int64_t)b * T_ + row) * W + c, true);
        raw_f32<T, EPL>(raw, v);
      } else if (row >= -(K - 1)) {
        ld_f32<EPL>(hist + ((int64_t)b * (K - 1) + (K - 1 + row)) * W + c, v);
      }
#pragma unroll
      for (int e = 0; e < EPL; ++e) k[e] = fmaf(__ldg(taps + (int64_t)r * W + c + e), v[e], k[e]);
    }
  }
  float rr;
  bool clamp;
  normalize<EPL>(k, G, floor_, rr, clamp);
  if (mine && live) {
    st_row<T, EPL>(out + ((int64_t)b * T_ + tok) * W + c, k);
    if (sp != nullptr && (threadIdx.x & (G - 1)) == 0) sp[tok] = make_float2(rr, clamp ? -1.f : 1.f);
  }
}

// GT: the lanes per head when fixed at compile time (0: read from the shape)
template <typename T, int EPL, int K, int GT>
__global__ void __launch_bounds__(WARPS * 32, 4) keys_fwd_kernel(const T* __restrict__ z, const float* __restrict__ hist,
                                                                 const float* __restrict__ taps, T* __restrict__ out,
                                                                 float2* __restrict__ stats, int B, int T_, int W,
                                                                 int hd, int spans, int runs, float floor_) {
  constexpr int BYTES = EPL * (int)sizeof(T);
  constexpr bool STAGED = stageable<BYTES>() && ring_rows<BYTES, 1>() >= K;
  constexpr int NS = STAGED ? ring_rows<BYTES, 1>() / K : 1;  // steps in flight
  constexpr int SB = STAGED ? BYTES : 16;
  constexpr uint32_t ROW = 32 * SB;  // one row of the warp's ring
  __shared__ __align__(16) uint8_t ring[WARPS][NS * K][32 * SB];
  const int gw = blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (gw >= B * spans * runs) return;
  const Walk w = walk_of(gw, spans, runs, W, hd, EPL);
  const int lane = threadIdx.x & 31;
  const int G = GT ? GT : w.G, gl = lane & (G - 1);
  const int c = w.live ? w.c : 0;  // a lane past the width loads channel 0's rows and stores nothing
  float tp[K][EPL];
#pragma unroll
  for (int r = 0; r < K; ++r)
#pragma unroll
    for (int e = 0; e < EPL; ++e) tp[r][e] = __ldg(taps + (int64_t)r * W + c + e);
  const int t0 = w.run * run_len(RUN_F, K), t1 = min(T_, t0 + run_len(RUN_F, K));
  float win[K][EPL];
  window_init<T, EPL, K>(win, z, hist, w, t0, T_, W);
  const T* zq = z + ((int64_t)w.b * T_ + t0) * W + c;  // the first row of the next step to copy
  const uint32_t ring0 = static_cast<uint32_t>(__cvta_generic_to_shared(&ring[threadIdx.x >> 5][0][lane * SB]));
  // a step's K rows go in as one commit group, NS steps ahead of their use
  auto copy_step = [&](uint32_t at, int first) {
#pragma unroll
    for (int j = 0; j < K; ++j) cp_async_row<BYTES>(at + j * ROW, zq + (int64_t)j * W, first + j < t1);
    cp_async_commit();
    zq += (int64_t)K * W;
  };
  if constexpr (STAGED) {
#pragma unroll 1
    for (int i = 0; i < NS; ++i) copy_step(ring0 + i * K * ROW, t0 + i * K);
  }
  int sidx = 0;  // the ring step of the current step
  T* oq = out + ((int64_t)w.b * T_ + t0) * W + c;
  float2* sp = stats != nullptr ? stats + ((int64_t)w.b * (W / hd) + w.head) * T_ : nullptr;
  const bool st_stats = sp != nullptr && w.live && gl == 0;
  // one unrolled step of K tokens; CLEAN: every token of the step is inside the run
  auto step = [&](auto clean, int t) -> unsigned {
    constexpr bool CLEAN = decltype(clean)::value;
    unsigned slow = 0u;
    [[maybe_unused]] const uint32_t at = ring0 + sidx * K * ROW;
    if constexpr (STAGED) cp_async_wait<NS - 1>();  // this step's rows are the oldest of NS groups in flight
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const int tok = t + j;
      // row tok enters the window in slot j (the row it replaces, tok - K, is no longer needed)
      if constexpr (STAGED) {
        staged_f32<T, EPL>(at + j * ROW, win[j]);
      } else {
        Raw<T, EPL> raw;
        raw_load<T, EPL>(raw, zq + (int64_t)j * W, CLEAN || tok < t1);
        raw_f32<T, EPL>(raw, win[j]);
      }
      float k[EPL];
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        float a = 0.f;
#pragma unroll
        for (int r = 0; r < K; ++r) a = fmaf(tp[r][e], win[(j - r + K) % K][e], a);
        k[e] = a;
      }
      float rr;
      bool fast;
      normalize_fast<EPL>(k, G, floor_, rr, fast);
      if (CLEAN || tok < t1) {
        if (w.live) st_row<T, EPL>(oq, k);
        if (st_stats) sp[tok] = make_float2(rr, -1.f);
      }
      oq += W;
      slow |= fast ? 0u : 1u << j;
    }
    if constexpr (STAGED) {
      copy_step(at, t + NS * K);  // NS steps ahead, into the slots just read
      sidx = sidx + 1 == NS ? 0 : sidx + 1;
    } else {
      zq += (int64_t)K * W;
    }
    return slow;
  };
  for (int t = t0; t < t1; t += K) {
    const unsigned slow = t + K <= t1 ? step(std::true_type{}, t) : step(std::false_type{}, t);
    if (__any_sync(0xffffffffu, slow != 0u)) {
      for (int j = 0; j < K && t + j < t1; ++j)
        if (__any_sync(0xffffffffu, (slow >> j) & 1u))
          fix_token<T, EPL, K>(z, hist, taps, out, sp, w.b, t + j, T_, W, c, w.live, G, floor_, (slow >> j) & 1u);
    }
  }
  if constexpr (STAGED) cp_async_wait<0>();
}

// the dz accumulator of time tau is complete: a z row of this run, a history row (run 0), or
// nothing (a row of the neighbouring run)
template <typename T, int EPL, int K>
__device__ __forceinline__ void flush(int tau, const float (&v)[EPL], T* __restrict__ dzp, float* __restrict__ dhp,
                                      int t0, int t1, int W, bool live) {
  if (!live) return;
  if (tau >= t0 && tau < t1) st_row<T, EPL>(dzp + (int64_t)tau * W, v);
  else if (tau < 0 && tau >= -(K - 1) && dhp != nullptr) st_f32<EPL>(dhp + (int64_t)(K - 1 + tau) * W, v);
}

// Backward over one run. partial: [B * runs, K, W] taps-gradient partial sums; stats: the forward's
// per-token (r, +-1) when STATS, else recomputed.
template <typename T, int EPL, int K, bool STATS, int GT>
__global__ void __launch_bounds__(WARPS * 32, 4) keys_bwd_kernel(
    const T* __restrict__ z, const float* __restrict__ hist, const float* __restrict__ taps, const T* __restrict__ gk,
    const float2* __restrict__ stats, T* __restrict__ dz, float* __restrict__ dhist, float* __restrict__ partial,
    int B, int T_, int W, int hd, int spans, int runs, float floor_) {
  constexpr int BYTES = EPL * (int)sizeof(T);
  constexpr bool STAGED = stageable<BYTES>();
  constexpr int PF = STAGED ? ring_rows<BYTES, 2>() : 1;  // rows in flight per warp and stream
  constexpr int SB = STAGED ? BYTES : 16;
  constexpr uint32_t ROW = 32 * SB;  // one row of a warp's ring
  __shared__ __align__(16) uint8_t ring[WARPS][2][PF][32 * SB];
  const int gw = blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (gw >= B * spans * runs) return;
  const Walk w = walk_of(gw, spans, runs, W, hd, EPL);
  const int lane = threadIdx.x & 31;
  const int G = GT ? GT : w.G;
  const int c = w.live ? w.c : 0;  // a lane past the width loads channel 0's rows and stores nothing
  float tp[K][EPL];
#pragma unroll
  for (int r = 0; r < K; ++r)
#pragma unroll
    for (int e = 0; e < EPL; ++e) tp[r][e] = __ldg(taps + (int64_t)r * W + c + e);
  const int t0 = w.run * run_len(RUN_B, K), t1 = min(T_, t0 + run_len(RUN_B, K));
  const int te = min(T_, t1 + K - 1);  // the next run's first K-1 input gradients are recomputed
  float win[K][EPL];
  window_init<T, EPL, K>(win, z, hist, w, t0, T_, W);
  float acc[K][EPL];  // acc[s]: dz of the time tau = s (mod K) being accumulated
  float dt[K][EPL];   // the taps' gradient over this run
#pragma unroll
  for (int r = 0; r < K; ++r)
#pragma unroll
    for (int e = 0; e < EPL; ++e) { acc[r][e] = 0.f; dt[r][e] = 0.f; }
  const int64_t base = (int64_t)w.b * T_ * W + c;
  T* dzp = dz + base;
  float* dhp = (dhist != nullptr && w.run == 0) ? dhist + (int64_t)w.b * (K - 1) * W + c : nullptr;
  const float2* sp = STATS ? stats + ((int64_t)w.b * (W / hd) + w.head) * T_ : nullptr;
  const T* zq = z + base + (int64_t)t0 * W;   // the first z row of the next step to copy
  const T* gq = gk + base + (int64_t)t0 * W;  // the first key-gradient row of the next step to copy
  T* dq = dzp + (int64_t)(t0 - K) * W;        // dz row of the time a token's slot completes
  const uint32_t zring = static_cast<uint32_t>(__cvta_generic_to_shared(&ring[threadIdx.x >> 5][0][0][lane * SB]));
  const uint32_t gring = static_cast<uint32_t>(__cvta_generic_to_shared(&ring[threadIdx.x >> 5][1][0][lane * SB]));
  // one commit group per token: waiting until at most PF - 1 are pending makes the oldest visible
  if constexpr (STAGED) {
#pragma unroll 1
    for (int i = 0; i < PF; ++i, zq += W, gq += W) {
      cp_async_row<BYTES>(zring + i * ROW, zq, t0 + i < te);
      cp_async_row<BYTES>(gring + i * ROW, gq, t0 + i < te);
      cp_async_commit();
    }
  }
  int slot = 0;  // the ring row of the current token
  float2 rs[K];  // the statistics of the next K tokens, loaded a step ahead
#pragma unroll
  for (int j = 0; j < K; ++j)
    if constexpr (STATS) rs[j] = t0 + j < te ? __ldg(sp + t0 + j) : make_float2(0.f, 1.f);
  // one unrolled step of K tokens; CLEAN: every token of the step is below t1 and every completed
  // slot's time inside [t0, t1)
  auto step = [&](auto clean, int t) {
    constexpr bool CLEAN = decltype(clean)::value;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const int tok = t + j;
      float g[EPL];
      // row tok enters the window in slot j (the row it replaces, tok - K, is no longer needed)
      if constexpr (STAGED) {
        cp_async_wait<PF - 1>();  // token tok's rows are the oldest of PF in flight
        const uint32_t off = slot * ROW;
        staged_f32<T, EPL>(zring + off, win[j]);
        staged_f32<T, EPL>(gring + off, g);
        if constexpr (!CLEAN) {
          if (tok >= te) {  // a token past the walk: its ring slots were never filled
#pragma unroll
            for (int e = 0; e < EPL; ++e) { win[j][e] = 0.f; g[e] = 0.f; }
          }
        }
        const bool in = tok + PF < te;  // PF tokens ahead, into the slots just read
        cp_async_row<BYTES>(zring + off, zq, in);
        cp_async_row<BYTES>(gring + off, gq, in);
        cp_async_commit();
        slot = slot + 1 == PF ? 0 : slot + 1;
      } else {
        const bool in = tok < te;
        Raw<T, EPL> raw;
        raw_load<T, EPL>(raw, zq, in);
        raw_f32<T, EPL>(raw, win[j]);
        raw_load<T, EPL>(raw, gq, in);
        raw_f32<T, EPL>(raw, g);
      }
      zq += W;
      gq += W;
      float rr = 0.f;
      bool clamp = true;
      if constexpr (STATS) {
        rr = rs[j].x;
        clamp = rs[j].y < 0.f;
        rs[j] = tok + K < te ? __ldg(sp + tok + K) : make_float2(0.f, 1.f);
      }
      float k[EPL];
#pragma unroll
      for (int e = 0; e < EPL; ++e) k[e] = 0.f;
#pragma unroll
      for (int r = 0; r < K; ++r) fma_row<EPL>(k, tp[r], win[(j - r + K) % K], k);
      if constexpr (STATS) {
        mul_row<EPL>(k, rr, k);
      } else {
        normalize<EPL>(k, G, floor_, rr, clamp);
      }
      float dot = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) dot = fmaf(g[e], k[e], dot);
      dot = group_sum(dot, G);  // every lane takes part; a head whose clamp holds drops it below
      if (!clamp) dot = 0.f;
      float du[EPL];
      fma_row<EPL>(du, -dot, k, g);
      mul_row<EPL>(du, rr, du);
      // slot j held dz of tok - K, complete with token tok - 1; it restarts with tok's own term
      if constexpr (CLEAN) {
        if (w.live) st_row<T, EPL>(dq, acc[j]);
      } else {
        flush<T, EPL, K>(tok - K, acc[j], dzp, dhp, t0, t1, W, w.live);
      }
      dq += W;
      mul_row<EPL>(acc[j], tp[0], du);
#pragma unroll
      for (int r = 1; r < K; ++r) fma_row<EPL>(acc[(j - r + K) % K], tp[r], du, acc[(j - r + K) % K]);
      if (CLEAN || tok < t1) {
#pragma unroll
        for (int r = 0; r < K; ++r) fma_row<EPL>(dt[r], du, win[(j - r + K) % K], dt[r]);
      }
    }
  };
  int t = t0;
  for (; t < te; t += K) {
    if (t >= t0 + K && t + K <= t1) step(std::true_type{}, t);
    else step(std::false_type{}, t);
  }
  if constexpr (STAGED) cp_async_wait<0>();
  // slot s now holds dz of t - K + s, complete (later input gradients are zero or not this run's)
#pragma unroll
  for (int s = 0; s < K; ++s) flush<T, EPL, K>(t - K + s, acc[s], dzp, dhp, t0, t1, W, w.live);
  if (w.live) {
    float* p = partial + (((int64_t)w.b * runs + w.run) * K) * W + c;
#pragma unroll
    for (int r = 0; r < K; ++r) st_f32<EPL>(p + (int64_t)r * W, dt[r]);
  }
}

// elements per lane: 16-byte accesses in the forward, 8 (bf16) or 16 bytes (float32) in the
// backward, never more than a head and at least a head over 32 lanes
template <typename T>
int epl_fwd(int hd) {
  const int v = 16 / (int)sizeof(T);
  return hd / 32 > v ? hd / 32 : (hd < v ? hd : v);
}
inline int epl_bwd(int hd) { return hd / 32 > 4 ? hd / 32 : (hd < 4 ? hd : 4); }

#define VB_EPL_DISPATCH(epl, EPL, ...)                               \
  [&]() -> int {                                                     \
    switch (epl) {                                                   \
      case 1: { constexpr int EPL = 1; return __VA_ARGS__(); }       \
      case 2: { constexpr int EPL = 2; return __VA_ARGS__(); }       \
      case 4: { constexpr int EPL = 4; return __VA_ARGS__(); }       \
      default: { constexpr int EPL = 8; return __VA_ARGS__(); }      \
    }                                                                \
  }()

#define VB_K_DISPATCH(k, KK, ...)                                    \
  [&]() -> int {                                                     \
    switch (k) {                                                     \
      case 1: { constexpr int KK = 1; return __VA_ARGS__(); }        \
      case 2: { constexpr int KK = 2; return __VA_ARGS__(); }        \
      case 3: { constexpr int KK = 3; return __VA_ARGS__(); }        \
      case 4: { constexpr int KK = 4; return __VA_ARGS__(); }        \
      case 5: { constexpr int KK = 5; return __VA_ARGS__(); }        \
      case 6: { constexpr int KK = 6; return __VA_ARGS__(); }        \
      case 7: { constexpr int KK = 7; return __VA_ARGS__(); }        \
      default: { constexpr int KK = 8; return __VA_ARGS__(); }       \
    }                                                                \
  }()

inline int check_shape(int B, int T_, int W, int heads, int K) {
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
