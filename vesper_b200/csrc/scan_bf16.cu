// The chunked delta-rule scan in bfloat16 on tcgen05 tensor cores (the contract of
// vesper/kernels/delta_scan.py:132-153 delta_scan_fused; the blocked WY form of
// vesper/recurrence.py:166-217).
//
// Per (batch, head) sequence and 64-token chunk c with keys K, queries Q, values V [64 x d]:
//   A = strictly_lower(diag(beta) K K^T),  X = (I + A)^-1,  T' = X diag(beta)
//   W = T' K,  U = T' V,  delta = U - W H_c,  O = Q H_c + P delta,  H_{c+1} = H_c + K^T delta
// with P = lower_inclusive(Q K^T) and H [key i, value j] the state at the chunk's start.
//
// Substituting delta, the state step and the output are linear in H_c with chunk-local matrices
//   M = -W^T K (d x d),  Q' = Q - P W:   H_{c+1} = H_c + M^T H_c + K^T U,   O = Q' H_c + P U,
// and the backward's state step dH_c = dH_{c+1} + Q^T dO - W^T ddelta (ddelta = P^T dO + K dH_{c+1})
// is dH_c = dH_{c+1} + M dH_{c+1} + Q'^T dO. Only these one-product steps stay on the sequential
// chains; everything else is chunk-parallel.
//
// Kernels (every product is a tcgen05.mma from 128B-swizzled shared-memory tiles into tensor
// memory; the head dimension is zero-padded to 128 inside the tiles):
//   prep     chunk-parallel: K K^T and Q K^T, the unit-lower-triangular solve for X (float32,
//            one thread per column), then U, W, M, Q'; a bf16 tile image per chunk.
//   forward  one CTA per sequence walks its chunks; H^T lives in tensor memory (fp32, 128 lanes =
//            value index j, 128 columns = key index i). The bf16 copy of H_c that fed the chunk's
//            products is checkpointed (the backward reuses it, no recomputation of the chain).
//   backward one CTA per sequence walks the chunks in reverse for the state gradient,
//            checkpointing the bf16 dH_{c+1}; then a chunk-parallel kernel forms every local
//            gradient from (H_c, dH_{c+1}) in one pass: dq, dk, dv, dbeta.
// Waits on the tensor core are bounded (2 s): a timeout sets bit 1 of *status and the kernel
// leaves after releasing its tensor memory.
#include <cstring>

#include "common.cuh"
#include "tmap.cuh"
#include "umma.cuh"

namespace vb {
namespace {

using bf16 = __nv_bfloat16;

constexpr int C = 64;    // tokens per chunk
constexpr int DP = 128;  // padded head dimension inside the tiles
constexpr uint32_t TILE_TD = 64 * 128 * 2;   // [64 tokens][128 d]
constexpr uint32_t TILE_JI = 128 * 128 * 2;  // [128][128]
constexpr uint32_t TILE_TT = 64 * 64 * 2;    // [64][64]
constexpr uint32_t TILE_JT = 128 * 64 * 2;   // [128 rows][64]

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return (uint8_t*)(((uintptr_t)p + 1023) & ~(uintptr_t)1023);
}

// beta of this thread's token (threads < 64) as a raw load whose latency overlaps later work;
// the value is stored to shared memory only where it is first needed
__device__ __forceinline__ bf16 fetch_beta(const bf16* __restrict__ beta, int64_t row0, int H, int valid) {
  const int t = threadIdx.x;
  return (t < C && t < valid) ? beta[(row0 + t) * H] : __float2bfloat16_rn(0.f);
}

// TMA loads of one [64 token][128 d] tile (two 64-channel boxes) of chunk t0 of (b, h)
__device__ __forceinline__ void tma_tile(uint8_t* tile, const CUtensorMap* map, uint64_t* bar, int h, int t0, int b) {
  tma_load_4d(tile, map, bar, 0, h, t0, b);
  tma_load_4d(tile + TILE_TD / 2, map, bar, 64, h, t0, b);
}

__device__ __forceinline__ void ld64(uint32_t tm, int col, float (&v)[64]) {
  float* a = v;
  tmem_ld32(tm + (uint32_t)col, *reinterpret_cast<float(*)[32]>(a));
  tmem_ld32(tm + (uint32_t)col + 32, *reinterpret_cast<float(*)[32]>(a + 32));
  tmem_wait_ld();
}

// One MMA of K = 16 * STEPS, D (+)= A x B: the k-step descriptors are the step-0 descriptor plus a
// compile-time offset (the start-address field counts 16-byte units), so each step costs one
// add and the issue. A_MN / B_MN select the MN-major form (tile rows = K index) over the K-major
// one (tile rows = the M or N index, `A_ROWS` / `B_ROWS` rows per 64-element atom).
template <int STEPS, int A_MN, int A_ROWS, int B_MN, int B_ROWS>
__device__ __forceinline__ void mma_seq(uint32_t d, uint32_t a, uint32_t b, uint32_t idesc,
                                        uint32_t accumulate_first) {
  const uint64_t a0 = A_MN ? desc_mn(a, A_ROWS, 0) : desc_k(a, A_ROWS, 0);
  const uint64_t b0 = B_MN ? desc_mn(b, B_ROWS, 0) : desc_k(b, B_ROWS, 0);
#pragma unroll
  for (int s = 0; s < STEPS; ++s) {
    const uint64_t ao = A_MN ? (uint64_t)(s * 128) : (uint64_t)(((s >> 2) * A_ROWS * 128 + (s & 3) * 32) >> 4);
    const uint64_t bo = B_MN ? (uint64_t)(s * 128) : (uint64_t)(((s >> 2) * B_ROWS * 128 + (s & 3) * 32) >> 4);
    umma_bf16(d, a0 + ao, b0 + bo, idesc, (s > 0 || accumulate_first) ? 1u : 0u);
  }
}

// all threads: bounded wait on the MMA barrier; flips the phase; any thread that gives up flags it
__device__ __forceinline__ bool mma_wait(uint64_t* bar, uint32_t& phase, int* status) {
  const bool ok = mbar_wait(bar, phase);
  phase ^= 1u;
  if (!ok) atomicOr(status, 2);
  tc_fence_after();
  return ok;
}

// writes made by threads (smem operands, tensor-memory reads) complete before the next MMA
__device__ __forceinline__ void publish() {
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

// writes made by threads, as publish(); returns whether every thread's waits succeeded
__device__ __forceinline__ bool publish_ok(bool ok) {
  fence_async_smem();
  tc_fence_before();
  ok = __syncthreads_and(ok ? 1 : 0) != 0;
  tc_fence_after();
  return ok;
}

// every bulk store group of this thread but the newest has finished reading shared memory
__device__ __forceinline__ void bulk_wait_read_but_newest() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

// row r, columns [c0, c0 + 32) of a swizzled bf16 tile: x <- bf16(x - v)
__device__ __forceinline__ void sub_row32_bf16(uint8_t* tile, int rows, int r, int c0, const float* v) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4* p = reinterpret_cast<uint4*>(tile + sw_chunk(rows, r, c0 / 8 + j));
    uint4 w = *p;
    const bf16* e = reinterpret_cast<const bf16*>(&w);
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = __bfloat162float(e[i]) - v[8 * j + i];
    w.x = pack_bf16(o[0], o[1]);
    w.y = pack_bf16(o[2], o[3]);
    w.z = pack_bf16(o[4], o[5]);
    w.w = pack_bf16(o[6], o[7]);
    *p = w;
  }
}

// ------------------------------------------------------------------------------------------
// prep, chunk-parallel (two 256-thread CTAs per SM): everything of a chunk that does not depend
// on the state.
//   [K; Q] K^T (one M=128 product): A = strictly_lower(diag(beta) K K^T), P = lower_inclusive(Q K^T)
//   X = (I + A)^-1 by float32 forward substitution (one thread per column), T' = X diag(beta)
//   U = T' V, W = T' K        (the stacked operand [T'; T'] puts a token row on every lane)
//   M = -W^T K  (d x d),  Q' = Q - P W
// Substituting delta = U - W H_c, the chunk's state step and output become
//   H_{c+1} = H_c + M^T H_c + K^T U,   O = Q' H_c + P U,
// and the backward's state step dH_c = dH_{c+1} + Q^T dO - W^T ddelta becomes
//   dH_c = dH_{c+1} + M dH_{c+1} + Q'^T dO:
// one product per chunk on each chain. Per chunk the image holds the bf16 tiles
// [X 8K][P 8K][T' 8K][U 16K][Q' 16K][M 32K] (M: 128 rows i, 128 columns i').
// ------------------------------------------------------------------------------------------
constexpr uint32_t PREP_X = 0, PREP_P = TILE_TT, PREP_T = 2 * TILE_TT, PREP_U = 3 * TILE_TT,
                   PREP_Q = PREP_U + TILE_TD, PREP_M = PREP_Q + TILE_TD, PREP_BYTES = PREP_M + TILE_JI;
struct PrepSmem {
  // KQ [128 rows][128 d]: K in rows 0-63, Q in rows 64-127 of each atom (Q' replaces Q in place);
  // Vt: V, then U; AF: float32 A [64][65], then atom 0 of M; Ws: the X image, then W, then atom 1
  // of M; TT: [T'; T'] (128 rows x 64); Ps: P. During the solve Ws and TT hold the float32 X
  // [64][68] and the block products (3 x [16][20]).
  static constexpr uint32_t KQ = 0, Vt = TILE_JI, AF = Vt + TILE_TD, Ws = AF + 17 * 1024, TT = Ws + TILE_TD,
                            Ps = TT + TILE_JT, END = Ps + TILE_TT;
};
constexpr int NP = 256;

// X = (I + A)^-1 for the strictly lower A (float32 [64][65]) into X (float32 [64][68]), 256
// threads: the four 16 x 16 diagonal blocks by forward substitution (a thread per column), then
// the blocks below them one block diagonal at a time, X_ij = -X_ii sum_{j <= k < i} A_ik X_kj,
// each thread a 1 x 4 strip of an output block. Entries above the diagonal blocks are not written.
constexpr int XS = 68;  // row stride of X (16-byte aligned rows)
__device__ __forceinline__ void invert_unit_lower(const float* A, float* X, float* Tm, int tid) {
  if (tid < C) {
    const int o = 16 * (tid >> 4), j = tid & 15;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int s = 0; s < r; ++s) {
        if (s & 1) s1 = fmaf(A[(o + r) * 65 + o + s], x[s], s1);
        else s0 = fmaf(A[(o + r) * 65 + o + s], x[s], s0);
      }
      x[r] = (r == j ? 1.f : 0.f) - (s0 + s1);
      X[(o + r) * XS + o + j] = x[r];
    }
  }
  __syncthreads();
  const int jb = tid >> 6, r = (tid >> 2) & 15, q4 = 4 * (tid & 3);
#pragma unroll
  for (int d = 1; d < 4; ++d) {
    const int i = jb + d;
    const bool act = i < 4;
    if (act) {  // T = sum_k A_ik X_kj, rows r, columns q4 .. q4 + 3
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int k = jb; k < i; ++k)
#pragma unroll
        for (int s = 0; s < 16; ++s) {
          const float a = A[(16 * i + r) * 65 + 16 * k + s];
          const float4 x = *reinterpret_cast<const float4*>(X + (16 * k + s) * XS + 16 * jb + q4);
          t.x = fmaf(a, x.x, t.x); t.y = fmaf(a, x.y, t.y); t.z = fmaf(a, x.z, t.z); t.w = fmaf(a, x.w, t.w);
        }
      *reinterpret_cast<float4*>(Tm + jb * 320 + r * 20 + q4) = t;
    }
    __syncthreads();
    if (act) {  // X_ij = -X_ii T
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int s = 0; s < 16; ++s) {
        const float a = X[(16 * i + r) * XS + 16 * i + s];
        const float4 t = *reinterpret_cast<const float4*>(Tm + jb * 320 + s * 20 + q4);
        x.x = fmaf(a, t.x, x.x); x.y = fmaf(a, t.y, x.y); x.z = fmaf(a, t.z, x.z); x.w = fmaf(a, t.w, x.w);
      }
      *reinterpret_cast<float4*>(X + (16 * i + r) * XS + 16 * jb + q4) = make_float4(-x.x, -x.y, -x.z, -x.w);
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(NP, 2) scan_prep_kernel(
    const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
    const __grid_constant__ CUtensorMap vmap, const bf16* __restrict__ beta, uint8_t* __restrict__ xt, int T,
    int H, int NC, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t *KQ = sm + PrepSmem::KQ, *Vt = sm + PrepSmem::Vt, *Ws = sm + PrepSmem::Ws, *TT = sm + PrepSmem::TT;
  uint8_t* Ps = sm + PrepSmem::Ps;
  float* A = reinterpret_cast<float*>(sm + PrepSmem::AF);
  uint8_t* M0 = sm + PrepSmem::AF;  // M columns 0-63 once A is dead
  uint8_t* M1 = Ws;                 // M columns 64-127 once W is dead
  __shared__ float bsm[C];
  __shared__ uint64_t bar, lbar;
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;
  const int lane128 = quarter * 32 + lane;
  const int c = blockIdx.x % NC, bh = blockIdx.x / NC, b = bh / H, h = bh % H;
  const int t0 = c * C, valid = min(C, T - t0);
  const int64_t row0 = (int64_t)b * T + t0;
  uint8_t* img = xt + (size_t)blockIdx.x * PREP_BYTES;
  if (tid == 0) { mbar_init(&bar, 1); mbar_init(&lbar, 1); mbar_fence_init(); }
  __syncthreads();
  if (tid == 0) {
    mbar_arrive_expect_tx(&lbar, 3 * TILE_TD);
    tma_load_4d(KQ, &kmap, &lbar, 0, h, t0, b);
    tma_load_4d(KQ + TILE_JI / 2, &kmap, &lbar, 64, h, t0, b);
    tma_load_4d(KQ + TILE_TD / 2, &qmap, &lbar, 0, h, t0, b);
    tma_load_4d(KQ + TILE_JI / 2 + TILE_TD / 2, &qmap, &lbar, 64, h, t0, b);
    tma_tile(Vt, &vmap, &lbar, h, t0, b);
  }
  const bf16 bv = fetch_beta(beta + h, row0, H, valid);
  if (warp == 0) { tmem_alloc(&tbase, 256); tmem_relinquish(); }
  bool ok = mbar_wait(&lbar, 0);
  if (!ok) atomicOr(status, 4);
  if (tid < C) bsm[tid] = __bfloat162float(bv);  // after the tile wait: both loads in flight together
  ok = publish_ok(ok);
  const uint32_t tm = tbase;
  const uint32_t lane_tm = taddr(tm, quarter * 32, 0);
  const uint32_t sKQ = smem_u32(KQ), sV = smem_u32(Vt), sW = smem_u32(Ws), sTT = smem_u32(TT), sP = smem_u32(Ps);
  uint32_t phase = 0;
  // 1. [K; Q] K^T into columns 0-63
  if (tid == 0 && ok) {
    mma_seq<DP / 16, 0, 128, 0, 128>(tm, sKQ, sKQ, idesc_bf16(128, 64, 0, 0), 0u);
    umma_commit(&bar);
  }
  if (ok) ok = mma_wait(&bar, phase, status);
  {
    float v[32];
    const int c0 = half * 32;
    tmem_ld32(lane_tm + (uint32_t)c0, v);
    tmem_wait_ld();
    if (lane128 < C) {
      const int t = lane128;
#pragma unroll
      for (int e = 0; e < 32; ++e) A[t * 65 + c0 + e] = c0 + e < t ? bsm[t] * v[e] : 0.f;
    } else {
      const int t = lane128 - C;
#pragma unroll
      for (int e = 0; e < 32; ++e) v[e] = c0 + e <= t ? v[e] : 0.f;
      st_row32_bf16(Ps, 64, t, c0, v);
    }
  }
  ok = publish_ok(ok);
  // 2. X (float32 over Ws and TT), then the bf16 X image into Ws and T' = bf16(X beta) into both
  //    halves of TT; every thread reads its 16 entries of X before any is overwritten
  {
    float* Xf = reinterpret_cast<float*>(Ws);
    invert_unit_lower(A, Xf, Xf + 64 * XS, tid);
    float xv[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int idx = tid + NP * e, t = idx >> 6, j = idx & 63;
      xv[e] = (j >> 4) > (t >> 4) ? 0.f : Xf[t * XS + j];
    }
    __syncthreads();
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int idx = tid + NP * e, t = idx >> 6, j = idx & 63;
      const bf16 xb = __float2bfloat16_rn(xv[e]);
      const bf16 tb = __float2bfloat16_rn(__bfloat162float(xb) * bsm[j]);
      *reinterpret_cast<bf16*>(Ws + sw_offset(64, t, j)) = xb;
      *reinterpret_cast<bf16*>(TT + sw_offset(128, t, j)) = tb;
      *reinterpret_cast<bf16*>(TT + sw_offset(128, t + 64, j)) = tb;
    }
  }
  ok = publish_ok(ok);
  // 3. the X, P and T' images; U = [T'; T'] V (columns 0-127), W = [T'; T'] K (128-255)
  if (tid == 0) {
    bulk_store(img + PREP_X, Ws, TILE_TT);
    bulk_store(img + PREP_P, Ps, TILE_TT);
    bulk_store(img + PREP_T, TT, TILE_TT);
    bulk_commit();
    if (ok) {
      mma_seq<4, 0, 128, 1, 64>(tm, sTT, sV, idesc_bf16(128, 128, 0, 1), 0u);
      mma_seq<4, 0, 128, 1, 128>(tm + 128, sTT, sKQ, idesc_bf16(128, 128, 0, 1), 0u);
      umma_commit(&bar);
    }
    bulk_wait_read();  // Ws (the X image) is rewritten with W below
  }
  if (ok) ok = mma_wait(&bar, phase, status);
  __syncthreads();
  {
    // lanes 0-63 (the first copy of the token rows) read U, lanes 64-127 read W; the two warps of
    // a lane quarter split the 128 columns
    const int t = lane128 & 63;
    const bool w_rows = lane128 >= 64;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      float v[32];
      const int c0 = half * 64 + 32 * k;
      tmem_ld32(lane_tm + (uint32_t)((w_rows ? 128 : 0) + c0), v);
      tmem_wait_ld();
      st_row32_bf16(w_rows ? Ws : Vt, 64, t, c0, v);
    }
  }
  ok = publish_ok(ok);
  // 4. the U image; M = -W^T K (columns 0-127), P W (M=64, columns 128-255)
  if (tid == 0) {
    bulk_store(img + PREP_U, Vt, TILE_TD);
    bulk_commit();
    if (ok) {
      mma_seq<4, 1, 64, 1, 128>(tm, sW, sKQ, idesc_bf16(128, 128, 1, 1, 1), 0u);
      mma_seq<4, 0, 64, 1, 64>(tm + 128, sP, sW, idesc_bf16(64, 128, 0, 1), 0u);
      umma_commit(&bar);
    }
  }
  if (ok) ok = mma_wait(&bar, phase, status);
  __syncthreads();
  {
    // M row i = lane: columns [64 half, 64 half + 64) are atom `half` of the M image
    uint8_t* Ma = half ? M1 : M0;
    const int t = quarter * 16 + (lane & 15);  // P W row of this lane (M=64 layout, lanes 0-15)
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      float m[32], pw[32];
      tmem_ld32(lane_tm + (uint32_t)(half * 64 + 32 * k), m);
      tmem_ld32(lane_tm + (uint32_t)(128 + half * 64 + 32 * k), pw);
      tmem_wait_ld();
      st_row32_bf16(Ma, 128, lane128, 32 * k, m);
      if (lane < 16) sub_row32_bf16(KQ, 128, 64 + t, half * 64 + 32 * k, pw);  // Q' = Q - P W
    }
  }
  fence_async_smem();
  __syncthreads();
  if (tid == 0) {
    bulk_store(img + PREP_Q, KQ + TILE_TD / 2, TILE_TD / 2);  // Q' columns 0-63: rows 64-127 of atom 0
    bulk_store(img + PREP_Q + TILE_TD / 2, KQ + TILE_JI / 2 + TILE_TD / 2, TILE_TD / 2);
    bulk_store(img + PREP_M, M0, TILE_JI / 2);
    bulk_store(img + PREP_M + TILE_JI / 2, M1, TILE_JI / 2);
    bulk_commit();
    bulk_wait_read();  // shared memory stays valid until the copies have read it
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tm, 256);
}

// ------------------------------------------------------------------------------------------
// forward: two CTAs per (b, h) walk its chunks, each owning half of the value index j (rows of
// H^T): H^T_J lives in tensor memory (fp32, M=64 layout: row r at lane 32 (r / 16) + r % 16,
// column i = key index) and, for the products, as the bf16 tile Hs [64 j][128 i]:
//   H^T_J += Hs M + U_J^T K,  O_J = Q' Hs   (one commit: Q' Hs has read Hs when H^T_J is complete)
//   O_J += P U_J                            (M=64 x N=64, double-buffered in tensor memory)
// Splitting the value index halves what each SM stores per chunk (its half of the checkpoint and
// of O) and spreads a sequence's copies over two SMs; M, K, Q' and P are read by both (the second
// read mostly from L2). Warp 8 issues every product and load; warps 0-7 read H^T_J back into Hs
// and O_J into the staging tile Ot (lanes 0-15 of warp w's quarter w % 4, the two warps of a
// quarter splitting the columns); thread 0 copies Hs (the checkpoint) and Ot out with bulk
// stores. The O readout of chunk c-1 overlaps the chain products of chunk c. Mbarriers order the
// two roles; every wait is bounded.
// ------------------------------------------------------------------------------------------
constexpr int NT2 = 256;         // threads of the sequential backward
constexpr int NF = 288;          // forward: eight reading warps and the issuing warp
constexpr int NR = 256;          // the forward's reading threads
constexpr uint32_t TILE_HALF = 64 * 128 * 2;  // [64 j][128 i]
constexpr uint32_t TILE_OJ = 64 * 64 * 2;     // [64 t][64 j]
struct FwdSmem {
  // per-chunk set: P, this CTA's half of U (one 64-column atom), then [Q' | M] in the prep
  // image's order (one bulk copy), then K
  static constexpr uint32_t Pt = 0, Ut = TILE_TT, Qt = Ut + TILE_OJ, Mt = Qt + TILE_TD, Kt = Mt + TILE_JI;
  static constexpr uint32_t SET = Kt + TILE_TD;                                     // 80 KB
  static constexpr uint32_t Hs = 2 * SET, Ot = Hs + TILE_HALF, Zt = Ot + TILE_OJ;
  static constexpr uint32_t END = Zt + TILE_HALF / 2;  // 192 KB; Zt: zeros for the padding half
};
constexpr int F_H = 0, F_O = 128;  // O of chunk c at columns F_O + 64 (c & 1)

struct ChunkAt {
  int t0, valid;
  int64_t row0;
};
__device__ __forceinline__ ChunkAt chunk_at(int b, int c, int T) {
  ChunkAt a;
  a.t0 = c * C;
  a.valid = min(C, T - a.t0);
  a.row0 = (int64_t)b * T + a.t0;
  return a;
}

// bounded wait by one thread; a timeout ORs `code` into the status word
__device__ __forceinline__ bool wait_or_flag(uint64_t* bar, uint32_t& phase, int* status, int code) {
  const bool ok = mbar_wait(bar, phase);
  phase ^= 1u;
  if (!ok) atomicOr(status, code);
  return ok;
}

// the 64-row half jh of a [128 j][128 i] state image: two 8 KB pieces (one per 64-column atom);
// with a single value half (d <= 64) rows 64-127 are padding, stored as zeros from the 8 KB
// zero tile `zero` (the local-gradient kernel multiplies over all 128 rows)
__device__ __forceinline__ void store_state_half(uint8_t* img, const uint8_t* half_tile, int jh, int halves,
                                                 const uint8_t* zero) {
  bulk_store(img + (uint32_t)jh * (TILE_HALF / 2), half_tile, TILE_HALF / 2);
  bulk_store(img + TILE_JI / 2 + (uint32_t)jh * (TILE_HALF / 2), half_tile + TILE_HALF / 2, TILE_HALF / 2);
  if (halves == 1) {
    bulk_store(img + TILE_HALF / 2, zero, TILE_HALF / 2);
    bulk_store(img + TILE_JI / 2 + TILE_HALF / 2, zero, TILE_HALF / 2);
  }
}
// zeros an 8 KB shared tile (all threads of the caller's group, before a proxy fence and barrier)
__device__ __forceinline__ void zero_tile8k(uint8_t* tile, int t, int n) {
  for (int i = t; i < (int)(TILE_HALF / 2 / 16); i += n) reinterpret_cast<uint4*>(tile)[i] = make_uint4(0u, 0u, 0u, 0u);
}

// Row jl (0..63) of a state half in the M=64 layout: column j = 64 jh + jl of the float32 [D][D]
// matrix (zero past D) into tensor memory at column `col`, and as bf16 into row jl of the
// [64][128] tile. Warps 0-3 call it; lanes 16-31 write unused tensor-memory lanes and no tile row.
__device__ __forceinline__ void state_row_m64(const float* mat, int D, int jh, uint32_t lane_tm, int col,
                                              uint8_t* tile) {
  const int lane = threadIdx.x & 31, jl = 16 * ((threadIdx.x >> 5) & 3) + (lane & 15);
  const int j = lane < 16 ? 64 * jh + jl : D;
#pragma unroll
  for (int c0 = 0; c0 < DP; c0 += 32) {
    float v[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = (mat != nullptr && c0 + e < D && j < D) ? mat[(int64_t)(c0 + e) * D + j] : 0.f;
    tmem_st32(lane_tm + (uint32_t)(col + c0), v);
    if (lane < 16) st_row32_bf16(tile, 64, jl, c0, v);
  }
  tmem_wait_st();
}

__global__ void __launch_bounds__(NF, 1) scan_fwd_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap omap,
    const float* __restrict__ s0, const uint8_t* __restrict__ xt, float* __restrict__ sn,
    uint8_t* __restrict__ hck, int T, int H, int D, int NC, int halves, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t *Hs = sm + FwdSmem::Hs, *Ot = sm + FwdSmem::Ot, *Zt = sm + FwdSmem::Zt;
  __shared__ uint64_t barH, barO[2], barOR[2], barHs, lbar[2];
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x / halves, jh = blockIdx.x % halves, b = bh / H, h = bh % H;
  auto set = [&](int c) { return sm + (uint32_t)(c & 1) * FwdSmem::SET; };
  if (tid == 0) {
    mbar_init(&barH, 1); mbar_init(&barO[0], 1); mbar_init(&barO[1], 1);
    mbar_init(&barOR[0], NR); mbar_init(&barOR[1], NR); mbar_init(&barHs, NR);
    mbar_init(&lbar[0], 1); mbar_init(&lbar[1], 1);
    mbar_fence_init();
  }
  if (warp == 0) { tmem_alloc(&tbase, 256); tmem_relinquish(); }
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tbase;
  if (warp == 8) {
    // ---------------- issuing warp (lane 0) ----------------
    if (lane == 0) {
      auto load_chunk = [&](int c) {
        const ChunkAt a = chunk_at(b, c, T);
        uint8_t* s = set(c);
        uint64_t* lb = &lbar[c & 1];
        const uint8_t* img = xt + ((size_t)bh * NC + c) * PREP_BYTES;
        mbar_arrive_expect_tx(lb, FwdSmem::SET);
        bulk_load(s + FwdSmem::Pt, img + PREP_P, TILE_TT, lb);
        bulk_load(s + FwdSmem::Ut, img + PREP_U + (uint32_t)jh * TILE_OJ, TILE_OJ, lb);
        bulk_load(s + FwdSmem::Qt, img + PREP_Q, TILE_TD + TILE_JI, lb);
        tma_tile(s + FwdSmem::Kt, &kmap, lb, h, a.t0, b);
      };
      if (NC > 0) load_chunk(0);
      if (NC > 1) load_chunk(1);
      uint32_t pl[2] = {0u, 0u}, pOR[2] = {0u, 0u}, pO[2] = {0u, 0u}, pHs = 0;
      const uint32_t sH = smem_u32(Hs);
      for (int c = 0; c < NC; ++c) {
        if (!wait_or_flag(&lbar[c & 1], pl[c & 1], status, 4)) break;
        if (!wait_or_flag(&barHs, pHs, status, 2)) break;                          // Hs = H_c
        if (c >= 2 && !wait_or_flag(&barOR[c & 1], pOR[c & 1], status, 2)) break;  // O of c-2 read
        tc_fence_after();
        const uint8_t* s = set(c);
        const uint32_t sU = smem_u32(s + FwdSmem::Ut), dO = tm + F_O + 64 * (c & 1);
        mma_seq<8, 0, 64, 1, 128>(tm + F_H, sH, smem_u32(s + FwdSmem::Mt), idesc_bf16(64, 128, 0, 1), 1u);
        mma_seq<8, 0, 64, 0, 64>(dO, smem_u32(s + FwdSmem::Qt), sH, idesc_bf16(64, 64, 0, 0), 0u);
        mma_seq<4, 1, 64, 1, 64>(tm + F_H, sU, smem_u32(s + FwdSmem::Kt), idesc_bf16(64, 128, 1, 1), 1u);
        umma_commit(&barH);
        mma_seq<4, 0, 64, 1, 64>(dO, smem_u32(s + FwdSmem::Pt), sU, idesc_bf16(64, 64, 0, 1), 1u);
        umma_commit(&barO[c & 1]);
        if (c + 2 < NC) {  // the set is free once every product of chunk c is done
          if (!wait_or_flag(&barO[c & 1], pO[c & 1], status, 2)) break;
          load_chunk(c + 2);
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- reading warps 0-7 ----------------
    const int quarter = warp & 3, half = warp >> 2;
    const int jl = quarter * 16 + (lane & 15);  // this lane's row of the M=64 accumulators
    const bool rowlane = lane < 16;
    const uint32_t lane_tm = taddr(tm, quarter * 32, 0);
    // H^T_J from the initial state (warps 0-3); its bf16 copy is the first checkpoint
    if (half == 0) state_row_m64(s0 + (int64_t)bh * D * D, D, jh, lane_tm, F_H, Hs);
    zero_tile8k(Zt, tid, NR);
    fence_async_smem();
    bar_sync_named(1, NR);
    if (tid == 0 && NC > 0) {
      store_state_half(hck + (size_t)bh * NC * TILE_JI, Hs, jh, halves, Zt);
      bulk_commit();
    }
    tc_fence_before();
    mbar_arrive(&barHs);
    uint32_t pH = 0, pO[2] = {0u, 0u};
    bool ok = true;
    // O_J of chunk c: tensor memory -> registers -> Ot -> one TMA store
    auto out_rows = [&](int c) -> bool {
      if (!wait_or_flag(&barO[c & 1], pO[c & 1], status, 2)) return false;
      tc_fence_after();
      float v[32];
      tmem_ld32(lane_tm + (uint32_t)(F_O + 64 * (c & 1) + half * 32), v);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&barOR[c & 1]);
      if (tid == 0) bulk_wait_read_but_newest();  // the previous O store has left Ot
      bar_sync_named(1, NR);
      if (rowlane) st_row32_bf16(Ot, 64, jl, half * 32, v);
      fence_async_smem();
      bar_sync_named(1, NR);
      if (tid == 0) {
        const ChunkAt a = chunk_at(b, c, T);
        tma_store_4d(&omap, Ot, 64 * jh, h, a.t0, b);
        bulk_commit();
      }
      return true;
    };
    for (int c = 0; c < NC && ok; ++c) {
      if (c > 0 && !(ok = out_rows(c - 1))) break;
      if (!(ok = wait_or_flag(&barH, pH, status, 2))) break;
      tc_fence_after();
      if (tid == 0) {  // the checkpoint of H_c has left Hs (the newest group, O of c - 1, may not)
        if (c == 0) bulk_wait_read();
        else bulk_wait_read_but_newest();
      }
      bar_sync_named(1, NR);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float v[32];
        const int c0 = half * 64 + 32 * k;
        tmem_ld32(lane_tm + (uint32_t)(F_H + c0), v);
        tmem_wait_ld();
        if (rowlane) {
          st_row32_bf16(Hs, 64, jl, c0, v);
          const int j = 64 * jh + jl;
          if (c + 1 == NC && j < D) {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (c0 + e < D) sn[(int64_t)bh * D * D + (int64_t)(c0 + e) * D + j] = v[e];
          }
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&barHs);
      if (c + 1 < NC) {  // checkpoint H_{c+1} for chunk c + 1 while the next products run
        bar_sync_named(1, NR);
        if (tid == 0) {
          store_state_half(hck + ((size_t)bh * NC + c + 1) * TILE_JI, Hs, jh, halves, Zt);
          bulk_commit();
        }
      }
    }
    if (ok && NC > 0) out_rows(NC - 1);
    if (NC == 0 && half == 0 && rowlane) {
      const int j = 64 * jh + jl;
      if (j < D)
        for (int i = 0; i < D; ++i) sn[(int64_t)bh * D * D + (int64_t)i * D + j] = s0[(int64_t)bh * D * D + (int64_t)i * D + j];
    }
    if (tid == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tm, 256);
}

// ------------------------------------------------------------------------------------------
// backward, sequential (256 threads): two CTAs per (b, h), each owning half of the value index j,
// walk the dH^T chain in tensor memory (M=64 layout) in reverse chunk order,
//   dH^T_J += dHs M^T + dO_J^T Q'      (12 k-steps; dHs = bf16 dH^T_{J, c+1}, [64 j][128 i])
// dHs is double-buffered, so its bulk-copied half of the checkpoint never waits on the chain;
// three input sets are in flight.
// ------------------------------------------------------------------------------------------
struct DhSmem {
  // per-chunk set: [Q' | M] as the prep image holds them, then this CTA's 64 columns of dO
  static constexpr uint32_t Qt = 0, Mt = TILE_TD, Gt = Mt + TILE_JI;
  static constexpr uint32_t SET = Gt + TILE_OJ;  // 56 KB
  static constexpr int NSET = 3;
  static constexpr uint32_t Ha = NSET * SET, Zt = Ha + 2 * TILE_HALF, END = Zt + TILE_HALF / 2;  // 208 KB
};
constexpr int G_H = 0;

__global__ void __launch_bounds__(NT2, 1) scan_dh_kernel(
    const __grid_constant__ CUtensorMap gmap, const uint8_t* __restrict__ xt, const float* __restrict__ dsn,
    float* __restrict__ ds0, uint8_t* __restrict__ dhck, int T, int H, int D, int NC, int halves, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t *Ha = sm + DhSmem::Ha, *Zt = sm + DhSmem::Zt;
  __shared__ uint64_t barH, lbar[DhSmem::NSET];
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;
  const int jl = quarter * 16 + (lane & 15);  // this lane's row of the M=64 accumulator
  const bool rowlane = lane < 16;
  const int bh = blockIdx.x / halves, jh = blockIdx.x % halves, b = bh / H, h = bh % H;
  uint32_t lphase[DhSmem::NSET] = {0u, 0u, 0u}, pH = 0;
  auto set = [&](int c) { return sm + (uint32_t)(c % DhSmem::NSET) * DhSmem::SET; };
  auto load_chunk = [&](int c) {  // thread 0
    const ChunkAt a = chunk_at(b, c, T);
    uint8_t* s = set(c);
    uint64_t* lb = &lbar[c % DhSmem::NSET];
    mbar_arrive_expect_tx(lb, DhSmem::SET);
    bulk_load(s + DhSmem::Qt, xt + ((size_t)bh * NC + c) * PREP_BYTES + PREP_Q, TILE_TD + TILE_JI, lb);
    tma_load_4d(s + DhSmem::Gt, &gmap, lb, 64 * jh, h, a.t0, b);
  };
  auto wait_chunk = [&](int c) -> bool {
    const int k = c % DhSmem::NSET;
    const bool r = mbar_wait(&lbar[k], lphase[k]);
    lphase[k] ^= 1u;
    if (!r) atomicOr(status, 4);
    return r;
  };
  if (tid == 0) {
    mbar_init(&barH, 1);
    for (int k = 0; k < DhSmem::NSET; ++k) mbar_init(&lbar[k], 1);
    mbar_fence_init();
  }
  if (warp == 0) { tmem_alloc(&tbase, 128); tmem_relinquish(); }
  __syncthreads();
  if (tid == 0)
    for (int k = 1; k <= DhSmem::NSET && NC - k >= 0; ++k) load_chunk(NC - k);
  tc_fence_after();
  const uint32_t tm = tbase;
  const uint32_t lane_tm = taddr(tm, quarter * 32, 0);
  auto dhs = [&](int c) { return Ha + (uint32_t)(c & 1) * TILE_HALF; };  // dH_{c+1}, read by chunk c
  if (half == 0 && NC > 0)
    state_row_m64(dsn != nullptr ? dsn + (int64_t)bh * D * D : nullptr, D, jh, lane_tm, G_H, dhs(NC - 1));
  zero_tile8k(Zt, tid, NT2);
  bool ok = publish_ok(true);
  for (int c = NC - 1; c >= 0 && ok; --c) {
    uint8_t* hb = dhs(c);
    if (tid == 0) {  // checkpoint dH_{c+1} for chunk c (this CTA's half)
      store_state_half(dhck + ((size_t)bh * NC + c) * TILE_JI, hb, jh, halves, Zt);
      bulk_commit();
    }
    ok = wait_chunk(c) && ok;
    if (tid == 0 && ok) {
      const uint8_t* s = set(c);
      mma_seq<8, 0, 64, 0, 128>(tm + G_H, smem_u32(hb), smem_u32(s + DhSmem::Mt), idesc_bf16(64, 128, 0, 0), 1u);  // += dHs M^T
      mma_seq<4, 1, 64, 1, 64>(tm + G_H, smem_u32(s + DhSmem::Gt), smem_u32(s + DhSmem::Qt),
                               idesc_bf16(64, 128, 1, 1), 1u);                                          // += dO^T Q'
      umma_commit(&barH);
    }
    if (ok) ok = mma_wait(&barH, pH, status);
    if (tid == 0) bulk_wait_read_but_newest();  // the checkpoint of chunk c + 1 has left the other buffer
    __syncthreads();
    // the set of chunk c is free; it is re-armed only now that every thread has waited on its
    // load barrier (re-armed earlier, a late waiter could see the barrier two phases on and stall)
    if (tid == 0 && ok && c - DhSmem::NSET >= 0) load_chunk(c - DhSmem::NSET);
    uint8_t* nb = dhs(c - 1);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      float v[32];
      const int c0 = half * 64 + 32 * k;
      tmem_ld32(lane_tm + (uint32_t)(G_H + c0), v);
      tmem_wait_ld();
      if (rowlane) {
        st_row32_bf16(nb, 64, jl, c0, v);
        const int j = 64 * jh + jl;
        if (c == 0 && j < D) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (c0 + e < D) ds0[(int64_t)bh * D * D + (int64_t)(c0 + e) * D + j] = v[e];
        }
      }
    }
    ok = publish_ok(ok);
  }
  if (NC == 0 && half == 0 && rowlane) {
    const int j = 64 * jh + jl;
    if (j < D)
      for (int i = 0; i < D; ++i)
        ds0[(int64_t)bh * D * D + (int64_t)i * D + j] = dsn ? dsn[(int64_t)bh * D * D + (int64_t)i * D + j] : 0.f;
  }
  if (tid == 0) bulk_wait_all();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tm, 128);
}

// ------------------------------------------------------------------------------------------
// backward, chunk-parallel: every local gradient of one chunk from (H_c, dH_{c+1})
// ------------------------------------------------------------------------------------------
struct GrSmem {
  static constexpr uint32_t Qt = 0, Kt = Qt + TILE_TD, Vt = Kt + TILE_TD, Gt = Vt + TILE_TD,
                            Ht = Gt + TILE_TD, dHt = Ht + TILE_JI, Xt = dHt + TILE_JI,
                            Tt = Xt + TILE_TT, Pt = Tt + TILE_TT, Dt = Pt + TILE_TT,
                            dDt = Dt + TILE_JT, Wr = dDt + TILE_JT, dPt = Wr + TILE_JT,
                            END = dPt + TILE_TT;
  // reuse: dW [t][i] over Wr (W^T is dead once H^T W^T is formed), dX over dDt (dead after dT'),
  // Y over Vt (dead after dT'), dGs over Pt (dead after ddelta), float scratch over Ht (dead
  // after dQ and dW)
};
constexpr int R_KK = 0, R_W = 128, R_U = 192, R_DD = 256, R_X = 320;   // batches 1-2
constexpr int R_DP = 64, R_DW = 128, R_DV = 256, R_DT = 384;                      // batch 3
constexpr int R_DQ = 128, R_Y = 256, R_Z = 320, R_DK = 128;                       // batches 4-7

constexpr int NG = 256;  // threads of the local-gradient kernel: two warps per lane quadrant
// one [64 t][128] bf16 tile to (b, h, tokens t0..) of a [B, T, H, D] tensor (rows past T and
// columns past D are not written)
__device__ __forceinline__ void store_tile(const CUtensorMap* map, const uint8_t* tile, int h, int t0, int b, int D) {
  tma_store_4d(map, tile, 0, h, t0, b);
  if (D > 64) tma_store_4d(map, tile + TILE_TD / 2, 64, h, t0, b);
  bulk_commit();
}
__device__ __forceinline__ void ld32w(uint32_t tm, int col, float (&v)[32]) {
  tmem_ld32(tm + (uint32_t)col, v);
  tmem_wait_ld();
}

__global__ void __launch_bounds__(NG, 1) scan_grad_kernel(
    const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
    const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap gmap,
    const __grid_constant__ CUtensorMap dqmap, const __grid_constant__ CUtensorMap dkmap,
    const __grid_constant__ CUtensorMap dvmap, const bf16* __restrict__ beta, const uint8_t* __restrict__ xt,
    const uint8_t* __restrict__ hck, const uint8_t* __restrict__ dhck, bf16* __restrict__ dbeta, int T, int H,
    int D, int NC, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t *Qt = sm + GrSmem::Qt, *Kt = sm + GrSmem::Kt, *Vt = sm + GrSmem::Vt, *Gt = sm + GrSmem::Gt;
  uint8_t *Ht = sm + GrSmem::Ht, *dHt = sm + GrSmem::dHt, *Xt = sm + GrSmem::Xt, *Tt = sm + GrSmem::Tt;
  uint8_t *Pt = sm + GrSmem::Pt, *Dt = sm + GrSmem::Dt, *dDt = sm + GrSmem::dDt, *Wr = sm + GrSmem::Wr;
  uint8_t *dPt = sm + GrSmem::dPt;
  uint8_t* dWt = Wr;   // [64 t][128 i] fits the 16 KB of Wr
  uint8_t* dXt = dDt;  // [64][64]
  uint8_t* Yt = Vt;    // [64][64]
  uint8_t* dGt = Pt;   // [64][64]
  float* scr = reinterpret_cast<float*>(Ht);  // [64][65] floats
  __shared__ float bsm[C], db1[C], db2s[2][C];
  __shared__ uint64_t bar, lbar[3];
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // warps w and w + 4 share tensor-memory lane quadrant w % 4 and split the columns (half)
  const int quarter = warp & 3, half = warp >> 2;
  const int lane128 = quarter * 32 + lane;
  const int c = blockIdx.x % NC, bh = blockIdx.x / NC, b = bh / H, h = bh % H;
  const int t0 = c * C, valid = min(C, T - t0);
  const int64_t row0 = (int64_t)b * T + t0;
  const int trow = quarter * 16 + (lane & 15);  // token row of an M=64 accumulator (lane < 16)
  const bool rowlane = lane < 16;
  const size_t chunk = (size_t)bh * NC + c;
  if (tid == 0) {
    mbar_init(&bar, 1); mbar_init(&lbar[0], 1); mbar_init(&lbar[1], 1); mbar_init(&lbar[2], 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (tid == 0) {  // in the order of first use: batch 1's operands, batch 2's, then X and Q
    const uint8_t* pre = xt + chunk * PREP_BYTES;
    mbar_arrive_expect_tx(&lbar[0], 2 * TILE_TD + TILE_JI + TILE_TT);
    tma_tile(Kt, &kmap, &lbar[0], h, t0, b);
    bulk_load(Tt, pre + PREP_T, TILE_TT, &lbar[0]);
    tma_tile(Vt, &vmap, &lbar[0], h, t0, b);
    bulk_load(dHt, dhck + chunk * TILE_JI, TILE_JI, &lbar[0]);
    mbar_arrive_expect_tx(&lbar[1], TILE_TD + TILE_JI + TILE_TT);
    bulk_load(Ht, hck + chunk * TILE_JI, TILE_JI, &lbar[1]);
    tma_tile(Gt, &gmap, &lbar[1], h, t0, b);
    bulk_load(Pt, pre + PREP_P, TILE_TT, &lbar[1]);
    mbar_arrive_expect_tx(&lbar[2], TILE_TD + TILE_TT);
    bulk_load(Xt, pre + PREP_X, TILE_TT, &lbar[2]);
    tma_tile(Qt, &qmap, &lbar[2], h, t0, b);
  }
  auto loaded = [&](int k) -> bool {
    const bool r = mbar_wait(&lbar[k], 0);
    if (!r) atomicOr(status, 4);
    return r;
  };
  const bf16 bv = fetch_beta(beta + h, row0, H, valid);
  if (warp == 0) { tmem_alloc(&tbase, 512); tmem_relinquish(); }
  bool ok = loaded(0);
  if (tid < C) bsm[tid] = __bfloat162float(bv);  // after the tile wait: both loads in flight together
  publish();
  const uint32_t tm = tbase;
  const uint32_t lane_tm = taddr(tm, quarter * 32, 0);
  const uint32_t sQ = smem_u32(Qt), sK = smem_u32(Kt), sV = smem_u32(Vt), sG = smem_u32(Gt);
  const uint32_t sH = smem_u32(Ht), sdH = smem_u32(dHt), sX = smem_u32(Xt), sT = smem_u32(Tt);
  const uint32_t sP = smem_u32(Pt), sD = smem_u32(Dt), sdD = smem_u32(dDt), sW = smem_u32(Wr);
  const uint32_t sdP = smem_u32(dPt), sdW = smem_u32(dWt), sdX = smem_u32(dXt), sY = smem_u32(Yt);
  const uint32_t sdG = smem_u32(dGt);
  uint32_t phase = 0;
  // batch 1: K K^T, W^T, U^T, ddelta^T = dH'^T K^T
  if (tid == 0 && ok) {
    const uint32_t id64 = idesc_bf16(64, 64, 0, 0);
    mma_seq<8, 0, 64, 0, 64>(tm + R_KK, sK, sK, id64, 0u);
    const uint32_t id_tn = idesc_bf16(128, 64, 1, 0);
    mma_seq<4, 1, 64, 0, 64>(tm + R_W, sK, sT, id_tn, 0u);
    mma_seq<4, 1, 64, 0, 64>(tm + R_U, sV, sT, id_tn, 0u);
    const uint32_t id_hk = idesc_bf16(128, 64, 0, 0);
    mma_seq<8, 0, 128, 0, 64>(tm + R_DD, sdH, sK, id_hk, 0u);
    umma_commit(&bar);
  }
  ok = ok && mma_wait(&bar, phase, status);
  {
    float w[32];
    ld32w(lane_tm, R_W + half * 32, w);
    st_row32_bf16(Wr, 128, lane128, half * 32, w);
  }
  ok = loaded(1) && ok;
  publish();
  // batch 2: X = H^T W^T; ddelta^T += dO^T P
  if (tid == 0 && ok) {
    const uint32_t id_hw = idesc_bf16(128, 64, 0, 1);
    mma_seq<8, 0, 128, 1, 128>(tm + R_X, sH, sW, id_hw, 0u);
    const uint32_t id_op = idesc_bf16(128, 64, 1, 1);
    mma_seq<4, 1, 64, 1, 64>(tm + R_DD, sG, sP, id_op, 1u);
    umma_commit(&bar);
  }
  ok = ok && mma_wait(&bar, phase, status);
  {
    float u[32], x[32];
    tmem_ld32(lane_tm + (uint32_t)(R_U + half * 32), u);
    tmem_ld32(lane_tm + (uint32_t)(R_X + half * 32), x);
    tmem_wait_ld();
#pragma unroll
    for (int s = 0; s < 32; ++s) u[s] -= x[s];
    st_row32_bf16(Dt, 128, lane128, half * 32, u);  // delta^T [j][t]
    ld32w(lane_tm, R_DD + half * 32, x);
    st_row32_bf16(dDt, 128, lane128, half * 32, x);  // ddelta^T [j][t]
  }
  publish();
  // batch 3: dP = dO delta^T; dW = -ddelta H^T; dV = T'^T ddelta; dT' = ddelta V^T
  if (tid == 0 && ok) {
    const uint32_t id_dp = idesc_bf16(64, 64, 0, 1);
    mma_seq<8, 0, 64, 1, 128>(tm + R_DP, sG, sD, id_dp, 0u);
    const uint32_t id_dw = idesc_bf16(64, 128, 1, 1, 1);
    mma_seq<8, 1, 128, 1, 128>(tm + R_DW, sdD, sH, id_dw, 0u);
    const uint32_t id_dv = idesc_bf16(64, 128, 1, 0);
    mma_seq<4, 1, 64, 0, 128>(tm + R_DV, sT, sdD, id_dv, 0u);
    const uint32_t id_dt = idesc_bf16(64, 64, 1, 0);
    mma_seq<8, 1, 128, 0, 64>(tm + R_DT, sdD, sV, id_dt, 0u);
    umma_commit(&bar);
  }
  ok = ok && mma_wait(&bar, phase, status);
  {
    float a[32];
    ld32w(lane_tm, R_DP + half * 32, a);
    if (rowlane) {
#pragma unroll
      for (int e = 0; e < 32; ++e) a[e] = half * 32 + e <= trow ? a[e] : 0.f;
      st_row32_bf16(dPt, 64, trow, half * 32, a);
    }
    float r[64];
    ld64(lane_tm, R_DW + half * 64, r);
    if (rowlane) st_row64_bf16(dWt, 64, trow, half, r);
    ld64(lane_tm, R_DV + half * 64, r);
    if (rowlane) st_row64_bf16(Vt, 64, trow, half, r);  // dV staged over V (its products are done)
  }
  publish();
  if (tid == 0) store_tile(&dvmap, Vt, h, t0, b, D);
  // batch 4: dQ = dO H^T + dP K; dT' += dW K^T
  if (tid == 0 && ok) {
    const uint32_t id_oh = idesc_bf16(64, 128, 0, 1);
    mma_seq<8, 0, 64, 1, 128>(tm + R_DQ, sG, sH, id_oh, 0u);
    const uint32_t id_pk = idesc_bf16(64, 128, 0, 1);
    mma_seq<4, 0, 64, 1, 64>(tm + R_DQ, sdP, sK, id_pk, 1u);
    const uint32_t id_wk = idesc_bf16(64, 64, 0, 0);
    mma_seq<8, 0, 64, 0, 64>(tm + R_DT, sdW, sK, id_wk, 1u);
    umma_commit(&bar);
  }
  ok = ok && mma_wait(&bar, phase, status);
  {
    float r[64];
    ld64(lane_tm, R_DQ + half * 64, r);
    if (rowlane) st_row64_bf16(Gt, 64, trow, half, r);  // dQ staged over dO (its products are done)
    ok = loaded(2) && ok;
    // dT' row t: dX = dT' diag(beta) (bf16 operand), dT' * X products for dbeta's first part
    float dt[32];
    ld32w(lane_tm, R_DT + half * 32, dt);
    if (rowlane) {
      float dx[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int s2 = half * 32 + e;
        const float xr = __bfloat162float(*reinterpret_cast<const bf16*>(Xt + sw_offset(64, trow, s2)));
        dx[e] = dt[e] * bsm[s2];
        scr[trow * 65 + s2] = dt[e] * xr;
      }
      st_row32_bf16(dXt, 64, trow, half * 32, dx);
    }
  }
  publish();
  if (tid == 0) {
    store_tile(&dqmap, Gt, h, t0, b, D);
    bulk_wait_read_but_newest();  // dV has left V, which Y overwrites below
  }
  // batch 5: Y = dX X^T (issued before the dbeta column sums below, which do not feed it)
  if (tid == 0 && ok) {
    const uint32_t id = idesc_bf16(64, 64, 0, 0);
    mma_seq<4, 0, 64, 0, 64>(tm + R_Y, sdX, sX, id, 0u);
    umma_commit(&bar);
  }
  if (tid < C) {
    float a = 0.f;
    for (int t = 0; t < C; ++t) a += scr[t * 65 + tid];
    db1[tid] = a;
  }
  ok = ok && mma_wait(&bar, phase, status);
  {
    float y[32];
    ld32w(lane_tm, R_Y + half * 32, y);
    if (rowlane) st_row32_bf16(Yt, 64, trow, half * 32, y);
  }
  publish();
  // batch 6: Z = X^T Y; dA = -Z (strictly lower)
  if (tid == 0 && ok) {
    const uint32_t id = idesc_bf16(64, 64, 1, 1);
    mma_seq<4, 1, 64, 1, 64>(tm + R_Z, sX, sY, id, 0u);
    umma_commit(&bar);
  }
  ok = ok && mma_wait(&bar, phase, status);
  {
    float z[32], kk[32];
    tmem_ld32(lane_tm + (uint32_t)(R_Z + half * 32), z);
    tmem_ld32(lane_tm + (uint32_t)(R_KK + half * 32), kk);
    tmem_wait_ld();
    if (rowlane) {
      const float bt = bsm[trow];
      float db2 = 0.f;
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int s2 = half * 32 + e;
        const float da = s2 < trow ? -z[e] : 0.f;
        db2 = fmaf(da, kk[e], db2);
        scr[trow * 65 + s2] = bt * da;  // dG
      }
      db2s[half][trow] = db2;
    }
  }
  __syncthreads();
  if (rowlane) {
    float g[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const int s2 = half * 32 + e;
      g[e] = scr[trow * 65 + s2] + scr[s2 * 65 + trow];
    }
    st_row32_bf16(dGt, 64, trow, half * 32, g);
    if (half == 0 && trow < valid)
      dbeta[(row0 + trow) * H + h] = __float2bfloat16_rn(db1[trow] + db2s[0][trow] + db2s[1][trow]);
  }
  publish();
  // batch 7: dK = dP^T Q + delta dH'^T + T'^T dW + (dG + dG^T) K
  if (tid == 0 && ok) {
    const uint32_t id_mn = idesc_bf16(64, 128, 1, 1);
    mma_seq<4, 1, 64, 1, 64>(tm + R_DK, sdP, sQ, id_mn, 0u);
    mma_seq<8, 1, 128, 1, 128>(tm + R_DK, sD, sdH, id_mn, 1u);
    mma_seq<4, 1, 64, 1, 64>(tm + R_DK, sT, sdW, id_mn, 1u);
    const uint32_t id_gk = idesc_bf16(64, 128, 0, 1);
    mma_seq<4, 0, 64, 1, 64>(tm + R_DK, sdG, sK, id_gk, 1u);
    umma_commit(&bar);
  }
  ok = ok && mma_wait(&bar, phase, status);
  {
    float r[64];
    ld64(lane_tm, R_DK + half * 64, r);
    if (rowlane) st_row64_bf16(Kt, 64, trow, half, r);  // dK staged over K (its products are done)
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    store_tile(&dkmap, Kt, h, t0, b, D);
    bulk_wait_read();
  }
  if (warp == 0) tmem_dealloc(tm, 512);
}

size_t smem_bytes(uint32_t end) { return (size_t)end + 1024; }

int check(const void* const* ptrs, int n, int B, int T, int H, int D) {
  VB_REQUIRE(B >= 0 && T >= 0 && H >= 0 && D > 0, "delta_scan_bf16: bad shape B=%d T=%d H=%d D=%d", B, T, H, D);
  VB_REQUIRE(D <= DP, "delta_scan_bf16: head dimension %d exceeds the kernel's %d", D, DP);
  VB_REQUIRE(D % 8 == 0, "delta_scan_bf16: head dimension %d must be a multiple of 8", D);
  for (int i = 0; i < n; ++i)
    VB_REQUIRE(ptrs[i] == nullptr || aligned16(ptrs[i]), "delta_scan_bf16: tensor %d is not 16-byte aligned", i);
  return VB_OK;
}

int nchunks(int T) { return (T + C - 1) / C; }

}  // namespace
}  // namespace vb

using namespace vb;

extern "C" size_t vb_delta_scan_bf16_saved_bytes(int B, int T, int H, int D) {
  (void)D;
  const size_t seqs = (size_t)(B > 0 ? B : 0) * (size_t)(H > 0 ? H : 0);
  const size_t nc = (size_t)nchunks(T > 0 ? T : 0);
  const size_t n = seqs * nc * (PREP_BYTES + TILE_JI);
  return n > 0 ? n : 16;
}

extern "C" size_t vb_delta_scan_bf16_bwd_workspace(int B, int T, int H, int D) {
  (void)D;
  const size_t seqs = (size_t)(B > 0 ? B : 0) * (size_t)(H > 0 ? H : 0);
  const size_t n = seqs * (size_t)nchunks(T > 0 ? T : 0) * TILE_JI;
  return n > 0 ? n : 16;
}

extern "C" int vb_delta_scan_bf16_fwd(const void* q, const void* k, const void* v, const void* beta,
                                      const float* state0, void* o, float* state_n, void* saved,
                                      int* status, int B, int T, int H, int D, void* stream) {
  const void* ptrs[] = {q, k, v, o, saved};
  int rc = check(ptrs, 5, B, T, H, D);
  if (rc) return rc;
  if (B == 0 || H == 0) return VB_OK;
  VB_REQUIRE(q && k && v && beta && state0 && o && state_n && saved && status, "delta_scan_bf16_fwd: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const int NC = nchunks(T);
  uint8_t* xt = (uint8_t*)saved;
  uint8_t* hck = xt + (size_t)B * H * NC * PREP_BYTES;
  CUtensorMap qm, km, vm, om;
  memset(&om, 0, sizeof(om));
  if (NC > 0) {
    if ((rc = make_token_map(&qm, q, B, T, H, D)) || (rc = make_token_map(&km, k, B, T, H, D)) ||
        (rc = make_token_map(&vm, v, B, T, H, D)) || (rc = make_token_map(&om, o, B, T, H, D)))
      return rc;
    const size_t sp = smem_bytes(PrepSmem::END);
    VB_CUDA_CHECK(cudaFuncSetAttribute(scan_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sp), "prep attr");
    scan_prep_kernel<<<B * H * NC, NP, sp, st>>>(qm, km, vm, (const bf16*)beta, xt, T, H, NC, status);
    VB_LAUNCH_CHECK("delta_scan_bf16 prep");
  } else {
    memset(&qm, 0, sizeof(qm)); memset(&km, 0, sizeof(km)); memset(&vm, 0, sizeof(vm));
  }
  const size_t sf = smem_bytes(FwdSmem::END);
  const int halves = D > 64 ? 2 : 1;  // value halves: the second is all padding when D <= 64
  VB_CUDA_CHECK(cudaFuncSetAttribute(scan_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sf), "fwd attr");
  scan_fwd_kernel<<<B * H * halves, NF, sf, st>>>(km, om, state0, xt, state_n, hck, T, H, D, NC, halves, status);
  VB_LAUNCH_CHECK("delta_scan_bf16 fwd");
  return VB_OK;
}

extern "C" int vb_delta_scan_bf16_bwd(const void* q, const void* k, const void* v, const void* beta,
                                      const void* saved, const void* dout, const float* dstate_n,
                                      void* dq, void* dk, void* dv, void* dbeta, float* dstate0,
                                      void* workspace, int* status, int B, int T, int H, int D,
                                      void* stream) {
  const void* ptrs[] = {q, k, v, saved, dout, dq, dk, dv, workspace};
  int rc = check(ptrs, 9, B, T, H, D);
  if (rc) return rc;
  if (B == 0 || H == 0) return VB_OK;
  VB_REQUIRE(q && k && v && beta && saved && dout && dq && dk && dv && dbeta && dstate0 && workspace && status,
             "delta_scan_bf16_bwd: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const int NC = nchunks(T);
  const uint8_t* xt = (const uint8_t*)saved;
  const uint8_t* hck = xt + (size_t)B * H * NC * PREP_BYTES;
  uint8_t* dhck = (uint8_t*)workspace;
  CUtensorMap qm, km, vm, gm;
  if (NC > 0) {
    if ((rc = make_token_map(&qm, q, B, T, H, D)) || (rc = make_token_map(&km, k, B, T, H, D)) ||
        (rc = make_token_map(&vm, v, B, T, H, D)) || (rc = make_token_map(&gm, dout, B, T, H, D)))
      return rc;
  } else {
    memset(&qm, 0, sizeof(qm)); memset(&km, 0, sizeof(km)); memset(&vm, 0, sizeof(vm)); memset(&gm, 0, sizeof(gm));
  }
  const size_t sd = smem_bytes(DhSmem::END);
  VB_CUDA_CHECK(cudaFuncSetAttribute(scan_dh_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sd), "dh attr");
  const int halves = D > 64 ? 2 : 1;  // value halves: the second is all padding when D <= 64
  scan_dh_kernel<<<B * H * halves, NT2, sd, st>>>(gm, xt, dstate_n, dstate0, dhck, T, H, D, NC, halves, status);
  VB_LAUNCH_CHECK("delta_scan_bf16 dh");
  if (NC > 0) {
    const size_t sg = smem_bytes(GrSmem::END);
    VB_CUDA_CHECK(cudaFuncSetAttribute(scan_grad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sg), "grad attr");
    CUtensorMap dqm, dkm, dvm;
    if ((rc = make_token_map(&dqm, dq, B, T, H, D)) || (rc = make_token_map(&dkm, dk, B, T, H, D)) ||
        (rc = make_token_map(&dvm, dv, B, T, H, D)))
      return rc;
    scan_grad_kernel<<<B * H * NC, NG, sg, st>>>(qm, km, vm, gm, dqm, dkm, dvm, (const bf16*)beta, xt, hck, dhck,
                                                 (bf16*)dbeta, T, H, D, NC, status);
    VB_LAUNCH_CHECK("delta_scan_bf16 grad");
  }
  return VB_OK;
}
