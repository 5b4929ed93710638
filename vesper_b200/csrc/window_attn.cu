// Sliding-window softmax attention on tcgen05 (the contract of vesper/kernels/window_attn.py:27-39,
// window_attention; the semantics of vesper/attention.py:340-407, WindowedAttention.attend).
//
// Keys and values are [B, L, HKV, DK] (a cache of m rows first, then the chunk); query row r of
// q [B, NQ, H, DK] sits at key index qpos(b, r) and attends the keys j with
// qpos - window < j <= qpos (j < L), scale 1/sqrt(DK), query head h reading key head h / (H / HKV).
// Without a position array qpos(b, r) = L - NQ + r (the dense call: the chunk follows the cache).
// With one, the rows are the loop's compacted active tokens: positions ascend along each batch row,
// and `counts[b]` rows of the NQ are live (the rest are padding: zero output, no gradient), so a
// graph can be captured at the worst-case size while the kernels read the live count.
//
// Forward: one CTA per (b, h, 128-query tile); S = Q K^T per 128-key tile into tensor memory,
// online softmax with one thread per query row (float32, base-2 exponent), P staged in shared
// memory in the input type, O += P V accumulated in tensor memory; outputs O and the row
// log-sum-exp (base 2, of S * scale), which the backward uses to rebuild P.
// Backward (deterministic, no atomics): delta = rowsum(dO * O); dQ per (b, h, query tile) walking
// its key tiles; dK, dV per (b, key head, key tile) walking every query head of the group and every
// query tile that reaches the tile, accumulated in tensor memory.
// Waits are bounded (2 s); a wait that gives up ORs 2 into the caller's status word.
#include <climits>
#include <cmath>
#include <type_traits>

#include "common.cuh"
#include "tmap.cuh"
#include "umma.cuh"

namespace vb {
namespace {

constexpr int BQ = 128;  // queries per tile (the products' M)
constexpr int BK = 128;  // keys per tile
constexpr int NT = 256;  // two threads per query (or key) row, each taking half of the row's columns
constexpr float LOG2E = 1.4426950408889634f;

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return (uint8_t*)(((uintptr_t)p + 1023) & ~(uintptr_t)1023);
}

// kind::f16 instruction descriptor for bf16 (is_bf16) or f16 operands, f32 accumulate
__host__ __device__ constexpr uint32_t idesc_16(int M, int N, int a_mn, int b_mn, bool is_bf16) {
  return (1u << 4) | ((is_bf16 ? 1u : 0u) << 7) | ((is_bf16 ? 1u : 0u) << 10) | ((uint32_t)a_mn << 15) |
         ((uint32_t)b_mn << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

template <typename E> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) { return pack_bf16(lo, hi); }
template <> __device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <typename E>
__device__ __forceinline__ uint4 pack8(const float* v, float s) {
  uint4 w;
  w.x = pack2<E>(v[0] * s, v[1] * s);
  w.y = pack2<E>(v[2] * s, v[3] * s);
  w.z = pack2<E>(v[4] * s, v[5] * s);
  w.w = pack2<E>(v[6] * s, v[7] * s);
  return w;
}
// 32 floats into row r, columns [c0, c0 + 32) of a swizzled tile of `rows` rows
template <typename E>
__device__ __forceinline__ void st_row32(uint8_t* tile, int rows, int r, int c0, const float* v) {
#pragma unroll
  for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(tile + sw_chunk(rows, r, c0 / 8 + j)) = pack8<E>(v + 8 * j, 1.f);
}

// STEPS k-steps of one product with descriptors computed once (K-major or MN-major operands)
template <int STEPS, int A_MN, int A_ROWS, int B_MN, int B_ROWS>
__device__ __forceinline__ void mma_seq(uint32_t d, uint32_t a, uint32_t b, uint32_t idesc, uint32_t acc_first) {
  const uint64_t a0 = A_MN ? desc_mn(a, A_ROWS, 0) : desc_k(a, A_ROWS, 0);
  const uint64_t b0 = B_MN ? desc_mn(b, B_ROWS, 0) : desc_k(b, B_ROWS, 0);
#pragma unroll
  for (int s = 0; s < STEPS; ++s) {
    const uint64_t ao = A_MN ? (uint64_t)(s * 128) : (uint64_t)(((s >> 2) * A_ROWS * 128 + (s & 3) * 32) >> 4);
    const uint64_t bo = B_MN ? (uint64_t)(s * 128) : (uint64_t)(((s >> 2) * B_ROWS * 128 + (s & 3) * 32) >> 4);
    umma_bf16(d, a0 + ao, b0 + bo, idesc, (s > 0 || acc_first) ? 1u : 0u);
  }
}

// bounded wait on phase `phase` of `bar` (flipped afterwards); a timeout flags the status word
__device__ __forceinline__ bool wait_flag(uint64_t* bar, uint32_t& phase, int* status) {
  const bool ok = mbar_wait(bar, phase);
  phase ^= 1u;
  if (!ok) atomicOr(status, 2);
  tc_fence_after();
  return ok;
}

// shared-memory writes and tensor-memory stores of every thread, then one elected issue;
// returns whether every thread's waits succeeded (uniform across the CTA)
__device__ __forceinline__ bool publish(bool ok) {
  fence_async_smem();
  tc_fence_before();
  ok = __syncthreads_and(ok ? 1 : 0) != 0;
  tc_fence_after();
  return ok;
}

// a [128 row][DK] tile (64-channel atoms of 128-byte rows) at row r0 of (b, head): 2 boxes per atom
template <int ATOMS>
__device__ __forceinline__ void tma_rows(uint8_t* tile, const CUtensorMap* map, uint64_t* bar, int head, int r0,
                                         int b) {
#pragma unroll
  for (int a = 0; a < ATOMS; ++a) {
    tma_load_4d(tile + a * (128 * 128), map, bar, 64 * a, head, r0, b);
    tma_load_4d(tile + a * (128 * 128) + 64 * 128, map, bar, 64 * a, head, r0 + 64, b);
  }
}

// query positions: the dense convention or a compacted list with per-batch live counts
struct QPos {
  const int* pos;     // [B, NQ] or null
  const int* counts;  // [B] or null
  int NQ, m;
  __device__ __forceinline__ int live(int b) const { return counts ? min(max(counts[b], 0), NQ) : NQ; }
  __device__ __forceinline__ int at(int b, int r) const { return pos ? pos[(int64_t)b * NQ + r] : m + r; }
};

template <int DK, typename E>
__device__ __forceinline__ void store_row(E* dst, const float (&v)[32], int c0, float s) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if (c0 + 8 * j < DK) *reinterpret_cast<uint4*>(dst + c0 + 8 * j) = pack8<E>(v + 8 * j, s);
}
template <int DK, typename E>
__device__ __forceinline__ void zero_row(E* dst) {
#pragma unroll
  for (int d = 0; d < DK; d += 8) *reinterpret_cast<uint4*>(dst + d) = make_uint4(0, 0, 0, 0);
}

constexpr int cols32(int dk) { return dk < 32 ? 32 : dk; }
// 32-column chunks of a DK-wide accumulator and the chunks [lo, hi) of one half-row thread
constexpr int chunks32(int dk) { return (cols32(dk) + 31) / 32; }
__device__ __forceinline__ int chunk_lo(int n, int half) { return half ? (n + 1) / 2 : 0; }
__device__ __forceinline__ int chunk_hi(int n, int half) { return half ? n : (n + 1) / 2; }

// 2^x on the special-function unit (PTX ex2.approx.ftz: about 2^-22 relative error; 2^-inf = +0)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ------------------------------------------------------------------------------------------
// forward
// ------------------------------------------------------------------------------------------
template <int DK, typename E>
__global__ void __launch_bounds__(NT) attn_fwd_kernel(
    const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
    const __grid_constant__ CUtensorMap vmap, const QPos qpos, E* __restrict__ o, float* __restrict__ lse,
    int L, int H, int HKV, int window, float sl2, int* status) {
  constexpr int ATOMS = (DK + 63) / 64;
  constexpr uint32_t TQ = BQ * 128 * ATOMS;  // a [128][DK] tile
  constexpr bool BF = std::is_same<E, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  // Q, K double-buffered, V single-buffered (V_i is read only by tile i's second product, which
  // runs after the tile's softmax: its copy is issued once the previous tile's product is done),
  // P: 96 KB at DK 64, so two CTAs share an SM and one's products overlap the other's softmax
  uint8_t* Qt = sm;
  auto Kt = [&](int i) { return sm + (1 + (i & 1)) * TQ; };
  uint8_t* Vt = sm + 3 * TQ;
  uint8_t* Pt = sm + 4 * TQ;  // P [128 q][128 keys]
  __shared__ uint64_t barS, barO, lbarQ, lbar[2], lbarV;
  __shared__ uint32_t tbase;
  __shared__ float xch[2][BQ];  // the two half-row threads' partial maxima, then sums
  const int NQ = qpos.NQ;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;  // warps w and w+4 share lane quadrant w % 4
  const int r128 = quarter * 32 + lane;             // this thread's row of the tile (its TMEM lane)
  const int qtile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int r0 = qtile * BQ, row = r0 + r128;
  const int nb = qpos.live(b);
  E* orow = o + (((int64_t)b * NQ + row) * H + h) * DK;
  float* lrow = lse + ((int64_t)b * H + h) * NQ + row;
  if (r0 >= nb) {  // a tile of padding rows only
    if (row < NQ && half == 0) { zero_row<DK>(orow); *lrow = 0.f; }
    return;
  }
  const bool live = row < nb;
  const int qp = live ? qpos.at(b, row) : INT_MIN / 2;
  const int qp_first = qpos.at(b, r0), qp_last = qpos.at(b, min(nb, r0 + BQ) - 1);
  const int g = h / (H / HKV);
  if (tid == 0) {
    mbar_init(&barS, 1); mbar_init(&barO, 1); mbar_init(&lbarQ, 1); mbar_init(&lbar[0], 1); mbar_init(&lbar[1], 1);
    mbar_init(&lbarV, 1);
    mbar_fence_init();
  }
  if (warp == 0) { tmem_alloc(&tbase, 256); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tbase;
  const uint32_t lane_tm = taddr(tm, quarter * 32, 0);
  constexpr int C_O = BK;  // S in columns [0, 128), O in [128, 128 + DK)
  constexpr int OCH = chunks32(DK);
  const int c_lo = chunk_lo(OCH, half), c_hi = chunk_hi(OCH, half);
  const int klo = max(0, qp_first - window + 1), khi = min(L - 1, qp_last);
  const int kt_lo = klo / BK;
  const int ntiles = khi >= klo ? khi / BK - kt_lo + 1 : 0;
  auto load_k = [&](int i) {
    uint64_t* lb = &lbar[i & 1];
    mbar_arrive_expect_tx(lb, TQ);
    tma_rows<ATOMS>(Kt(i), &kmap, lb, g, (kt_lo + i) * BK, b);
  };
  auto load_v = [&](int i) {
    mbar_arrive_expect_tx(&lbarV, TQ);
    tma_rows<ATOMS>(Vt, &vmap, &lbarV, g, (kt_lo + i) * BK, b);
  };
  if (tid == 0) {
    mbar_arrive_expect_tx(&lbarQ, TQ);
    tma_rows<ATOMS>(Qt, &qmap, &lbarQ, h, r0, b);
    if (ntiles > 0) { load_k(0); load_v(0); }
  }
  uint32_t lph[2] = {0u, 0u}, pS = 0, pO = 0, pQ = 0, pV = 0;
  bool ok = wait_flag(&lbarQ, pQ, status);
  const uint32_t id_s = idesc_16(BQ, BK, 0, 0, BF);
  const uint32_t id_o = idesc_16(BQ, DK, 0, 1, BF);
  float m2 = -INFINITY, l = 0.f;  // running max (base-2 units) and this half's denominator
  const int kc = half * (BK / 2);  // this thread's 64 keys of each tile
  for (int i = 0; i < ntiles && ok; ++i) {
    ok = wait_flag(&lbar[i & 1], lph[i & 1], status) && ok;
    if (tid == 0) {
      mma_seq<DK / 16, 0, BQ, 0, BK>(tm, smem_u32(Qt), smem_u32(Kt(i)), id_s, 0u);
      umma_commit(&barS);
    }
    ok = wait_flag(&barS, pS, status) && ok;
    // every earlier product is complete: the other K buffer, V and P are free
    if (i > 0) ok = wait_flag(&barO, pO, status) && ok;
    if (tid == 0) {
      if (i > 0) load_v(i);  // V_0 was copied with K_0
      if (i + 1 < ntiles) load_k(i + 1);
    }
    const int k0 = (kt_lo + i) * BK;
    // a tile inside every row's window needs no mask (rows ascend in position)
    const bool interior = k0 + BK - 1 <= qp_first && k0 > qp_last - window && k0 + BK <= L && r0 + BQ <= nb;
    float sv[BK / 2];
    tmem_ld32(lane_tm + kc, *reinterpret_cast<float(*)[32]>(sv));
    tmem_ld32(lane_tm + kc + 32, *reinterpret_cast<float(*)[32]>(sv + 32));
    tmem_wait_ld();
    float mt = -INFINITY;
    if (interior) {  // the scaling two lanes per packed f32x2 product (each rounds as a product)
#pragma unroll
      for (int j = 0; j < BK / 2; j += 2) {
        const float2 v = __fmul2_rn(make_float2(sv[j], sv[j + 1]), make_float2(sl2, sl2));
        sv[j] = v.x;
        sv[j + 1] = v.y;
        mt = fmaxf(mt, fmaxf(v.x, v.y));
      }
    } else {
#pragma unroll
      for (int j = 0; j < BK / 2; ++j) {
        const int kp = k0 + kc + j;
        const bool in = kp <= qp && kp > qp - window && kp < L;
        sv[j] = in ? sv[j] * sl2 : -INFINITY;
        mt = fmaxf(mt, sv[j]);
      }
    }
    xch[half][r128] = mt;
    __syncthreads();
    mt = fmaxf(xch[0][r128], xch[1][r128]);
    const float mnew = fmaxf(m2, mt);
    const float mref = mnew == -INFINITY ? 0.f : mnew;  // all masked so far: every p is 2^-inf = 0
    const float corr = ex2(m2 - mref);
    // the subtraction and the four running sums two lanes per packed f32x2 add (x - m is
    // x + (-m) exactly, and each lane rounds as a scalar add: the same values as scalar code)
    float2 l01 = make_float2(0.f, 0.f), l23 = make_float2(0.f, 0.f);
    const float2 nm = make_float2(-mref, -mref);
#pragma unroll
    for (int j = 0; j < BK / 2; j += 4) {
      const float2 d01 = __fadd2_rn(make_float2(sv[j], sv[j + 1]), nm);
      const float2 d23 = __fadd2_rn(make_float2(sv[j + 2], sv[j + 3]), nm);
      sv[j] = ex2(d01.x);
      sv[j + 1] = ex2(d01.y);
      sv[j + 2] = ex2(d23.x);
      sv[j + 3] = ex2(d23.y);
      l01 = __fadd2_rn(l01, make_float2(sv[j], sv[j + 1]));
      l23 = __fadd2_rn(l23, make_float2(sv[j + 2], sv[j + 3]));
    }
    l = l * corr + ((l01.x + l01.y) + (l23.x + l23.y));
    m2 = mnew;
    st_row32<E>(Pt, BQ, r128, kc, sv);
    st_row32<E>(Pt, BQ, r128, kc + 32, sv + 32);
    if (i > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
      for (int ch = c_lo; ch < c_hi; ++ch) {
        float ov[32];
        tmem_ld32(lane_tm + C_O + 32 * ch, ov);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) ov[e] *= corr;
        tmem_st32(lane_tm + C_O + 32 * ch, ov);
      }
      tmem_wait_st();
    }
    ok = publish(ok);
    if (tid == 0 && ok) {
      if (wait_flag(&lbarV, pV, status)) {  // V_i has landed
        mma_seq<BK / 16, 0, BQ, 1, BK>(tm + C_O, smem_u32(Pt), smem_u32(Vt), id_o, i > 0 ? 1u : 0u);
        umma_commit(&barO);
      } else {
        ok = false;
      }
    }
  }
  if (ntiles > 0 && ok) ok = wait_flag(&barO, pO, status);
  xch[half][r128] = l;
  __syncthreads();
  const float lt = xch[0][r128] + xch[1][r128];
  const float inv_l = lt > 0.f ? 1.f / lt : 0.f;
  for (int ch = c_lo; ch < c_hi; ++ch) {
    float ov[32];
    tmem_ld32(lane_tm + C_O + 32 * ch, ov);
    tmem_wait_ld();
    if (live && lt > 0.f) store_row<DK, E>(orow, ov, 32 * ch, inv_l);
  }
  if (half == 0) {
    if (live) {
      if (!(lt > 0.f)) zero_row<DK>(orow);
      *lrow = lt > 0.f ? m2 + log2f(lt) : 0.f;
    } else if (row < NQ) {
      zero_row<DK>(orow);
      *lrow = 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tm, 256);
}

// ------------------------------------------------------------------------------------------
// backward: delta = rowsum(dO * O) per (b, h, row), float32; a team of lanes per (b, row, h), each
// lane one 16-byte vector of both rows (DK / 8 lanes, rounded up to a power of two), the products
// summed in the lane and then across the team
// ------------------------------------------------------------------------------------------
template <int DK, typename E>
__global__ void attn_delta_kernel(const E* __restrict__ o, const E* __restrict__ dout, float* __restrict__ delta,
                                  int rows, int NQ, int H) {
  constexpr int VEC = 16 / (int)sizeof(E);
  constexpr int NV = DK / VEC;  // 16-byte vectors per row
  constexpr int LPR = NV <= 1 ? 1 : NV <= 2 ? 2 : NV <= 4 ? 4 : NV <= 8 ? 8 : NV <= 16 ? 16 : 32;
  static_assert(DK % VEC == 0 && NV <= 32, "a row is whole 16-byte vectors, at most 32 of them");
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  const int r = g / LPR, l = g % LPR;
  float a = 0.f;
  if (r < rows && l < NV) {
    const uint4 x = *reinterpret_cast<const uint4*>(o + (size_t)r * DK + l * VEC);
    const uint4 y = *reinterpret_cast<const uint4*>(dout + (size_t)r * DK + l * VEC);
    const E* xe = reinterpret_cast<const E*>(&x);
    const E* ye = reinterpret_cast<const E*>(&y);
#pragma unroll
    for (int i = 0; i < VEC; ++i) a = fmaf(to_f32(xe[i]), to_f32(ye[i]), a);
  }
#pragma unroll
  for (int off = LPR / 2; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
  if (r < rows && l == 0) {
    const int h = r % H, bn = r / H;
    delta[((size_t)(bn / NQ) * H + h) * NQ + bn % NQ] = a;
  }
}

// ------------------------------------------------------------------------------------------
// backward: dQ per (b, h, query tile), walking its key tiles:
//   P = exp2(S * scale*log2e - lse), dP = dO V^T, dS = P (dP - delta), dQ = scale * sum dS K
// ------------------------------------------------------------------------------------------
template <int DK, typename E>
__global__ void __launch_bounds__(NT) attn_dq_kernel(
    const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
    const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap gmap, const QPos qpos,
    const float* __restrict__ lse, const float* __restrict__ delta, E* __restrict__ dq, int L, int H, int HKV,
    int window, float sl2, float scale, int* status) {
  constexpr int ATOMS = (DK + 63) / 64;
  constexpr uint32_t TQ = BQ * 128 * ATOMS;
  constexpr bool BF = std::is_same<E, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* Qt = sm;
  uint8_t* Gt = sm + TQ;
  auto Kt = [&](int i) { return sm + (2 + 2 * (i & 1)) * TQ; };
  auto Vt = [&](int i) { return sm + (3 + 2 * (i & 1)) * TQ; };
  uint8_t* dSt = sm + 6 * TQ;  // dS [128 q][128 keys]
  __shared__ uint64_t barS, barQ, lbarQ, lbar[2];
  __shared__ uint32_t tbase;
  const int NQ = qpos.NQ;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;
  const int r128 = quarter * 32 + lane;
  const int qtile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int r0 = qtile * BQ, row = r0 + r128;
  const int nb = qpos.live(b);
  E* dqrow = dq + (((int64_t)b * NQ + row) * H + h) * DK;
  if (r0 >= nb) {
    if (row < NQ && half == 0) zero_row<DK>(dqrow);
    return;
  }
  const bool live = row < nb;
  const int qp = live ? qpos.at(b, row) : INT_MIN / 2;
  const float lse_r = live ? lse[((int64_t)b * H + h) * NQ + row] : 0.f;
  const float dl_r = live ? delta[((int64_t)b * H + h) * NQ + row] : 0.f;
  const int qp_first = qpos.at(b, r0), qp_last = qpos.at(b, min(nb, r0 + BQ) - 1);
  const int g = h / (H / HKV);
  if (tid == 0) {
    mbar_init(&barS, 1); mbar_init(&barQ, 1); mbar_init(&lbarQ, 1); mbar_init(&lbar[0], 1); mbar_init(&lbar[1], 1);
    mbar_fence_init();
  }
  if (warp == 0) { tmem_alloc(&tbase, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tbase;
  const uint32_t lane_tm = taddr(tm, quarter * 32, 0);
  constexpr int C_S = 0, C_P = BK, C_Q = 2 * BK;  // S, dP, dQ
  constexpr int OCH = chunks32(DK);
  const int c_lo = chunk_lo(OCH, half), c_hi = chunk_hi(OCH, half);
  const int klo = max(0, qp_first - window + 1), khi = min(L - 1, qp_last);
  const int kt_lo = klo / BK;
  const int ntiles = khi >= klo ? khi / BK - kt_lo + 1 : 0;
  auto load_kv = [&](int i) {
    uint64_t* lb = &lbar[i & 1];
    mbar_arrive_expect_tx(lb, 2 * TQ);
    tma_rows<ATOMS>(Kt(i), &kmap, lb, g, (kt_lo + i) * BK, b);
    tma_rows<ATOMS>(Vt(i), &vmap, lb, g, (kt_lo + i) * BK, b);
  };
  if (tid == 0) {
    mbar_arrive_expect_tx(&lbarQ, 2 * TQ);
    tma_rows<ATOMS>(Qt, &qmap, &lbarQ, h, r0, b);
    tma_rows<ATOMS>(Gt, &gmap, &lbarQ, h, r0, b);
    if (ntiles > 0) load_kv(0);
  }
  uint32_t lph[2] = {0u, 0u}, pS = 0, pQ = 0, pL = 0;
  bool ok = wait_flag(&lbarQ, pL, status);
  const uint32_t id_s = idesc_16(BQ, BK, 0, 0, BF);
  const uint32_t id_q = idesc_16(BQ, DK, 0, 1, BF);
  for (int i = 0; i < ntiles && ok; ++i) {
    ok = wait_flag(&lbar[i & 1], lph[i & 1], status) && ok;
    if (tid == 0) {
      mma_seq<DK / 16, 0, BQ, 0, BK>(tm + C_S, smem_u32(Qt), smem_u32(Kt(i)), id_s, 0u);  // S
      mma_seq<DK / 16, 0, BQ, 0, BK>(tm + C_P, smem_u32(Gt), smem_u32(Vt(i)), id_s, 0u);  // dP
      umma_commit(&barS);
    }
    ok = wait_flag(&barS, pS, status) && ok;
    if (i > 0) ok = wait_flag(&barQ, pQ, status) && ok;
    if (tid == 0 && i + 1 < ntiles) load_kv(i + 1);
    const int k0 = (kt_lo + i) * BK;
    const bool interior = k0 + BK - 1 <= qp_first && k0 > qp_last - window && k0 + BK <= L && r0 + BQ <= nb;
#pragma unroll
    for (int c0 = half * (BK / 2); c0 < half * (BK / 2) + BK / 2; c0 += 32) {
      float s[32], dp[32];
      tmem_ld32(lane_tm + C_S + c0, s);
      tmem_ld32(lane_tm + C_P + c0, dp);
      tmem_wait_ld();
      if (interior) {
#pragma unroll
        for (int e = 0; e < 32; ++e) s[e] = ex2(s[e] * sl2 - lse_r) * (dp[e] - dl_r);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int kp = k0 + c0 + e;
          const bool in = kp <= qp && kp > qp - window && kp < L;
          const float p = in ? ex2(s[e] * sl2 - lse_r) : 0.f;
          s[e] = p * (dp[e] - dl_r);
        }
      }
      st_row32<E>(dSt, BQ, r128, c0, s);
    }
    ok = publish(ok);
    if (tid == 0 && ok) {
      mma_seq<BK / 16, 0, BQ, 1, BK>(tm + C_Q, smem_u32(dSt), smem_u32(Kt(i)), id_q, i > 0 ? 1u : 0u);
      umma_commit(&barQ);
    }
  }
  if (ntiles > 0 && ok) ok = wait_flag(&barQ, pQ, status);
  for (int ch = c_lo; ch < c_hi; ++ch) {
    float v[32];
    tmem_ld32(lane_tm + C_Q + 32 * ch, v);
    tmem_wait_ld();
    if (live && ntiles > 0) store_row<DK, E>(dqrow, v, 32 * ch, scale);
  }
  if (row < NQ && half == 0 && !(live && ntiles > 0)) zero_row<DK>(dqrow);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tm, 512);
}

// ------------------------------------------------------------------------------------------
// backward: dK, dV per (b, key head g, key tile), walking the group's query heads and the query
// tiles that reach the tile: S^T = K Q^T, P^T = exp2(S^T * scale*log2e - lse), dV += P^T dO,
// dP^T = V dO^T, dS^T = P^T (dP^T - delta), dK += scale * dS^T Q.
// NBUF query/dO buffers (2: the next step's tiles load during this step's work).
// ------------------------------------------------------------------------------------------
template <int DK, typename E, int NBUF>
__global__ void __launch_bounds__(NT) attn_dkv_kernel(
    const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
    const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap gmap, const QPos qpos,
    const float* __restrict__ lse, const float* __restrict__ delta, E* __restrict__ dk, E* __restrict__ dv, int L,
    int H, int HKV, int window, float sl2, float scale, int* status) {
  constexpr int ATOMS = (DK + 63) / 64;
  constexpr uint32_t TQ = BQ * 128 * ATOMS;
  constexpr bool BF = std::is_same<E, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* Kt = sm;
  uint8_t* Vt = sm + TQ;
  auto Qt = [&](int buf) { return sm + (2 + 2 * buf) * TQ; };
  auto Gt = [&](int buf) { return sm + (3 + 2 * buf) * TQ; };
  uint8_t* Pt = sm + (2 + 2 * NBUF) * TQ;  // P^T [128 keys][128 q]
  uint8_t* dSt = Pt + BK * 128 * 2;        // dS^T [128 keys][128 q]
  __shared__ uint64_t barS, barA, lbarK, lbar[2];
  __shared__ uint32_t tbase;
  __shared__ float lse_s[NBUF][BQ], dl_s[NBUF][BQ];
  __shared__ int qp_s[NBUF][BQ];
  __shared__ int inner_s[NBUF];  // the step's query tile lies inside every key's window: no mask
  const int NQ = qpos.NQ;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;
  const int r128 = quarter * 32 + lane;
  const int ktile = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int groups = H / HKV;
  const int k0 = ktile * BK;
  const int kp = k0 + r128;  // this thread's key
  const int nb = qpos.live(b);
  // rows whose positions reach this key tile: qpos in [k0, k0 + BK - 1 + window - 1]; positions
  // ascend along a batch row, so the rows form one range, found by bisection
  auto first_row_ge = [&](int v) {
    int lo = 0, hi = nb;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (qpos.at(b, mid) >= v) hi = mid; else lo = mid + 1;
    }
    return lo;
  };
  const int row_lo = first_row_ge(k0);
  const int row_hi = first_row_ge(k0 + BK - 1 + window);
  const int qt_lo = row_lo / BQ;
  const int nqt = row_hi > row_lo ? (row_hi - 1) / BQ - qt_lo + 1 : 0;
  const int nsteps = nqt * groups;  // step s: query head g*groups + s / nqt, query tile qt_lo + s % nqt
  if (tid == 0) {
    mbar_init(&barS, 1); mbar_init(&barA, 1); mbar_init(&lbarK, 1); mbar_init(&lbar[0], 1); mbar_init(&lbar[1], 1);
    mbar_fence_init();
  }
  if (warp == 0) { tmem_alloc(&tbase, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tbase;
  const uint32_t lane_tm = taddr(tm, quarter * 32, 0);
  constexpr int C_S = 0, C_P = BK, C_K = 2 * BK, C_V = 2 * BK + cols32(DK);  // S^T, dP^T, dK, dV
  constexpr int OCH = chunks32(DK);
  const int c_lo = chunk_lo(OCH, half), c_hi = chunk_hi(OCH, half);
  static_assert(2 * BK + 2 * cols32(DK) <= 512, "tensor memory");
  auto load_q = [&](int s) {
    const int hh = g * groups + s / nqt, qt = qt_lo + s % nqt;
    const int buf = s % NBUF;
    if (tid == 0) {
      uint64_t* lb = &lbar[buf];
      mbar_arrive_expect_tx(lb, 2 * TQ);
      tma_rows<ATOMS>(Qt(buf), &qmap, lb, hh, qt * BQ, b);
      tma_rows<ATOMS>(Gt(buf), &gmap, lb, hh, qt * BQ, b);
    }
    if (tid < BQ) {
      const int r = qt * BQ + tid;
      const bool in = r < nb;
      qp_s[buf][tid] = in ? qpos.at(b, r) : INT_MAX / 2;
      lse_s[buf][tid] = in ? lse[((int64_t)b * H + hh) * NQ + r] : 0.f;
      dl_s[buf][tid] = in ? delta[((int64_t)b * H + hh) * NQ + r] : 0.f;
    }
    if (tid == 0) {
      const int q_lo = qpos.at(b, qt * BQ), q_hi = qpos.at(b, min(nb, qt * BQ + BQ) - 1);
      inner_s[buf] = k0 + BK - 1 <= q_lo && k0 > q_hi - window && k0 + BK <= L && qt * BQ + BQ <= nb;
    }
  };
  if (tid == 0) {
    mbar_arrive_expect_tx(&lbarK, 2 * TQ);
    tma_rows<ATOMS>(Kt, &kmap, &lbarK, g, k0, b);
    tma_rows<ATOMS>(Vt, &vmap, &lbarK, g, k0, b);
  }
  if (nsteps > 0) load_q(0);
  uint32_t lph[2] = {0u, 0u}, pS = 0, pA = 0, pK = 0;
  bool ok = wait_flag(&lbarK, pK, status);
  const uint32_t id_s = idesc_16(BK, BQ, 0, 0, BF);
  const uint32_t id_a = idesc_16(BK, DK, 0, 1, BF);
  for (int s = 0; s < nsteps && ok; ++s) {
    const int buf = s % NBUF;
    if (!__syncthreads_and(ok ? 1 : 0)) break;  // qp_s / lse_s / dl_s of step s are visible
    ok = wait_flag(&lbar[buf], lph[buf], status) && ok;
    if (tid == 0) {
      mma_seq<DK / 16, 0, BK, 0, BQ>(tm + C_S, smem_u32(Kt), smem_u32(Qt(buf)), id_s, 0u);  // S^T
      mma_seq<DK / 16, 0, BK, 0, BQ>(tm + C_P, smem_u32(Vt), smem_u32(Gt(buf)), id_s, 0u);  // dP^T
      umma_commit(&barS);
    }
    ok = wait_flag(&barS, pS, status) && ok;
    if (NBUF == 2) {
      if (s > 0) ok = wait_flag(&barA, pA, status) && ok;  // step s-1's products: the other buffer is free
      if (s + 1 < nsteps) load_q(s + 1);
    }
    const bool inner = inner_s[buf] != 0;
#pragma unroll
    for (int c0 = half * (BQ / 2); c0 < half * (BQ / 2) + BQ / 2; c0 += 32) {
      float sv[32], dp[32];
      tmem_ld32(lane_tm + C_S + c0, sv);
      tmem_ld32(lane_tm + C_P + c0, dp);
      tmem_wait_ld();
      if (inner) {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int q = c0 + e;
          const float p = ex2(sv[e] * sl2 - lse_s[buf][q]);
          sv[e] = p;
          dp[e] = p * (dp[e] - dl_s[buf][q]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int q = c0 + e;
          const int qpv = qp_s[buf][q];
          const bool in = kp <= qpv && kp > qpv - window && kp < L;
          const float p = in ? ex2(sv[e] * sl2 - lse_s[buf][q]) : 0.f;
          sv[e] = p;
          dp[e] = p * (dp[e] - dl_s[buf][q]);
        }
      }
      st_row32<E>(Pt, BK, r128, c0, sv);
      st_row32<E>(dSt, BK, r128, c0, dp);
    }
    ok = publish(ok);
    if (tid == 0 && ok) {
      mma_seq<BQ / 16, 0, BK, 1, BQ>(tm + C_V, smem_u32(Pt), smem_u32(Gt(buf)), id_a, s > 0 ? 1u : 0u);   // dV
      mma_seq<BQ / 16, 0, BK, 1, BQ>(tm + C_K, smem_u32(dSt), smem_u32(Qt(buf)), id_a, s > 0 ? 1u : 0u);  // dK
      umma_commit(&barA);
    }
    if (NBUF == 1 && ok) {
      ok = wait_flag(&barA, pA, status);  // the single buffer is free again
      if (s + 1 < nsteps) load_q(s + 1);
    }
  }
  if (NBUF == 2 && nsteps > 0 && ok) ok = wait_flag(&barA, pA, status);
  const bool live = kp < L;
  E* dkr = dk + (((int64_t)b * L + kp) * HKV + g) * DK;
  E* dvr = dv + (((int64_t)b * L + kp) * HKV + g) * DK;
  for (int ch = c_lo; ch < c_hi; ++ch) {
    float kv[32], vv[32];
    tmem_ld32(lane_tm + C_K + 32 * ch, kv);
    tmem_ld32(lane_tm + C_V + 32 * ch, vv);
    tmem_wait_ld();
    if (live && nsteps > 0) {
      store_row<DK, E>(dkr, kv, 32 * ch, scale);
      store_row<DK, E>(dvr, vv, 32 * ch, 1.f);
    }
  }
  if (live && nsteps == 0 && half == 0) {
    zero_row<DK>(dkr);
    zero_row<DK>(dvr);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tm, 512);
}

template <int DK> constexpr int dkv_nbuf() { return DK > 64 ? 1 : 2; }
template <int DK> constexpr size_t fwd_smem() { return (size_t)4 * BQ * 128 * ((DK + 63) / 64) + BQ * 256 + 1024; }
template <int DK> constexpr size_t dq_smem() { return (size_t)6 * BQ * 128 * ((DK + 63) / 64) + BQ * 256 + 1024; }
template <int DK> constexpr size_t dkv_smem() {
  return (size_t)(2 + 2 * dkv_nbuf<DK>()) * BQ * 128 * ((DK + 63) / 64) + 2 * BK * 256 + 1024;
}

int check(const char* what, int B, int NQ, int L, int H, int HKV, int DK, int window, int dtype, const int* qpos) {
  VB_REQUIRE(B >= 0 && NQ >= 0 && L >= 0 && H > 0 && HKV > 0 && H % HKV == 0,
             "%s: bad shape B=%d NQ=%d L=%d H=%d HKV=%d", what, B, NQ, L, H, HKV);
  VB_REQUIRE(DK % 16 == 0 && DK >= 16 && DK <= 128, "%s: head dimension %d must be a multiple of 16 in [16, 128]",
             what, DK);
  VB_REQUIRE(window >= 1, "%s: window %d must be at least 1", what, window);
  VB_REQUIRE(dtype == VB_BF16 || dtype == VB_F16 || dtype == VB_F32, "%s: dtype must be bfloat16, float16 or float32",
             what);
  VB_REQUIRE(qpos != nullptr || L >= NQ, "%s: dense queries need L >= NQ (L=%d, NQ=%d)", what, L, NQ);
  VB_REQUIRE(L < (1 << 29) && NQ < (1 << 29), "%s: length exceeds 2^29", what);
  return VB_OK;
}

// compile-time head dimension and element type
template <typename F>
int dispatch(int DK, int dtype, F&& f) {
  auto by_dk = [&](auto e) -> int {
    using E = decltype(e);
    switch (DK) {
      case 16: return f(std::integral_constant<int, 16>{}, E{});
      case 32: return f(std::integral_constant<int, 32>{}, E{});
      case 48: return f(std::integral_constant<int, 48>{}, E{});
      case 64: return f(std::integral_constant<int, 64>{}, E{});
      case 80: return f(std::integral_constant<int, 80>{}, E{});
      case 96: return f(std::integral_constant<int, 96>{}, E{});
      case 112: return f(std::integral_constant<int, 112>{}, E{});
      default: return f(std::integral_constant<int, 128>{}, E{});
    }
  };
  return dtype == VB_F16 ? by_dk(__half{}) : by_dk(__nv_bfloat16{});
}

}  // namespace

// float32 attention on CUDA cores (window_attn_f32.cu)
int window_attn_f32_fwd(const float* q, const int* qpos, const int* counts, const float* keys, const float* values,
                        float* o, float* lse, int B, int NQ, int L, int H, int HKV, int DK, int window,
                        cudaStream_t st);
int window_attn_f32_bwd(const float* q, const int* qpos, const int* counts, const float* keys, const float* values,
                        const float* o, const float* lse, const float* dout, float* dq, float* dkeys, float* dvalues,
                        float* delta, int B, int NQ, int L, int H, int HKV, int DK, int window, cudaStream_t st);
}  // namespace vb

using namespace vb;

extern "C" int vb_window_attn_fwd(const void* q, const int* qpos, const int* counts, const void* keys,
                                  const void* values, void* o, float* lse, int* status, int B, int NQ, int L, int H,
                                  int HKV, int DK, int window, int dtype, void* stream) {
  int rc = check("window_attn_fwd", B, NQ, L, H, HKV, DK, window, dtype, qpos);
  if (rc) return rc;
  if (B == 0 || NQ == 0) return VB_OK;
  VB_REQUIRE(q && keys && values && o && lse && status, "window_attn_fwd: null pointer");
  VB_REQUIRE(L > 0, "window_attn_fwd: no keys for %d queries", NQ);
  if (dtype == VB_F32)
    return window_attn_f32_fwd((const float*)q, qpos, counts, (const float*)keys, (const float*)values, (float*)o, lse,
                               B, NQ, L, H, HKV, DK, window, (cudaStream_t)stream);
  const bool f16 = dtype == VB_F16;
  CUtensorMap qm, km, vm;
  if ((rc = make_token_map(&qm, q, B, NQ, H, DK, f16)) || (rc = make_token_map(&km, keys, B, L, HKV, DK, f16)) ||
      (rc = make_token_map(&vm, values, B, L, HKV, DK, f16)))
    return rc;
  VB_REQUIRE(aligned16(o), "window_attn_fwd: output not 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  const QPos qp{qpos, counts, NQ, L - NQ};
  const float sl2 = LOG2E / sqrtf((float)DK);
  const int win = window > L ? L + 1 : window;
  const dim3 grid((NQ + BQ - 1) / BQ, H, B);
  return dispatch(DK, dtype, [&](auto dkc, auto e) -> int {
    constexpr int D = decltype(dkc)::value;
    using E = decltype(e);
    const size_t sm = fwd_smem<D>();
    VB_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel<D, E>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
                  "window_attn_fwd: smem attribute");
    attn_fwd_kernel<D, E><<<grid, NT, sm, st>>>(qm, km, vm, qp, (E*)o, lse, L, H, HKV, win, sl2, status);
    VB_LAUNCH_CHECK("window_attn_fwd");
    return VB_OK;
  });
}

extern "C" size_t vb_window_attn_bwd_workspace(int B, int NQ, int H) {
  const size_t n = (size_t)(B > 0 ? B : 0) * (size_t)(NQ > 0 ? NQ : 0) * (size_t)(H > 0 ? H : 0);
  return (n > 0 ? n : 4) * sizeof(float);
}

extern "C" int vb_window_attn_bwd(const void* q, const int* qpos, const int* counts, const void* keys,
                                  const void* values, const void* o, const float* lse, const void* dout, void* dq,
                                  void* dkeys, void* dvalues, void* workspace, int* status, int B, int NQ, int L,
                                  int H, int HKV, int DK, int window, int dtype, void* stream) {
  int rc = check("window_attn_bwd", B, NQ, L, H, HKV, DK, window, dtype, qpos);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  if (B == 0 || L == 0) return VB_OK;
  VB_REQUIRE(dkeys && dvalues, "window_attn_bwd: null pointer");
  const size_t esize = dtype == VB_F32 ? 4 : 2;
  if (NQ == 0) {
    VB_CUDA_CHECK(cudaMemsetAsync(dkeys, 0, (size_t)B * L * HKV * DK * esize, st), "window_attn_bwd");
    VB_CUDA_CHECK(cudaMemsetAsync(dvalues, 0, (size_t)B * L * HKV * DK * esize, st), "window_attn_bwd");
    return VB_OK;
  }
  VB_REQUIRE(q && keys && values && o && lse && dout && dq && workspace && status, "window_attn_bwd: null pointer");
  if (dtype == VB_F32)
    return window_attn_f32_bwd((const float*)q, qpos, counts, (const float*)keys, (const float*)values,
                               (const float*)o, lse, (const float*)dout, (float*)dq, (float*)dkeys, (float*)dvalues,
                               (float*)workspace, B, NQ, L, H, HKV, DK, window, st);
  VB_REQUIRE(aligned16(o) && aligned16(dout) && aligned16(dq) && aligned16(dkeys) && aligned16(dvalues),
             "window_attn_bwd: tensor not 16-byte aligned");
  const bool f16 = dtype == VB_F16;
  CUtensorMap qm, km, vm, gm;
  if ((rc = make_token_map(&qm, q, B, NQ, H, DK, f16)) || (rc = make_token_map(&km, keys, B, L, HKV, DK, f16)) ||
      (rc = make_token_map(&vm, values, B, L, HKV, DK, f16)) || (rc = make_token_map(&gm, dout, B, NQ, H, DK, f16)))
    return rc;
  const QPos qp{qpos, counts, NQ, L - NQ};
  const float scale = 1.0f / sqrtf((float)DK);
  const float sl2 = LOG2E * scale;
  const int win = window > L ? L + 1 : window;
  float* delta = (float*)workspace;
  return dispatch(DK, dtype, [&](auto dkc, auto e) -> int {
    constexpr int D = decltype(dkc)::value;
    using E = decltype(e);
    const int64_t rows = (int64_t)B * NQ * H;
    constexpr int NV = D * (int)sizeof(E) / 16, LPR = NV <= 1 ? 1 : NV <= 2 ? 2 : NV <= 4 ? 4 : NV <= 8 ? 8 : NV <= 16 ? 16 : 32;
    VB_REQUIRE(rows * LPR <= 0x7fffffff, "window_attn_bwd: %lld query rows exceed the delta kernel's int32 indices",
               (long long)rows);
    attn_delta_kernel<D, E><<<(unsigned)((rows * LPR + 255) / 256), 256, 0, st>>>((const E*)o, (const E*)dout, delta,
                                                                                  (int)rows, NQ, H);
    VB_LAUNCH_CHECK("window_attn_bwd delta");
    const size_t sq = dq_smem<D>();
    VB_CUDA_CHECK(cudaFuncSetAttribute(attn_dq_kernel<D, E>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sq),
                  "window_attn_bwd: smem attribute");
    attn_dq_kernel<D, E><<<dim3((NQ + BQ - 1) / BQ, H, B), NT, sq, st>>>(qm, km, vm, gm, qp, lse, delta, (E*)dq, L,
                                                                          H, HKV, win, sl2, scale, status);
    VB_LAUNCH_CHECK("window_attn_bwd dq");
    constexpr int NB = dkv_nbuf<D>();
    const size_t skv = dkv_smem<D>();
    VB_CUDA_CHECK(
        cudaFuncSetAttribute(attn_dkv_kernel<D, E, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)skv),
        "window_attn_bwd: smem attribute");
    attn_dkv_kernel<D, E, NB><<<dim3((L + BK - 1) / BK, HKV, B), NT, skv, st>>>(
        qm, km, vm, gm, qp, lse, delta, (E*)dkeys, (E*)dvalues, L, H, HKV, win, sl2, scale, status);
    VB_LAUNCH_CHECK("window_attn_bwd dkv");
    return VB_OK;
  });
}
