// The chunked delta-rule scan in bfloat16 on tcgen05 tensor cores (the contract of
// vesper/kernels/delta_scan.py:132-153 delta_scan_fused; the blocked WY form of
// vesper/recurrence.py:166-217).
//
// Per (batch, head) sequence and 64-token chunk c with keys K, queries Q, values V [64 x d]:
//   A = strictly_lower(diag(beta) K K^T),  X = (I + A)^-1,  T' = X diag(beta)
//   W = T' K,  U = T' V,  delta = U - W H_c,  O = Q H_c + P delta,  H_{c+1} = H_c + K^T delta
// with P = lower_inclusive(Q K^T) and H [key i, value j] the state at the chunk's start.
//
// Kernels (every product is a tcgen05.mma from 128B-swizzled shared-memory tiles into tensor
// memory; the head dimension is zero-padded to 128 inside the tiles):
//   prep     chunk-parallel: K K^T (M=64) and the unit-lower-triangular solve for X (float32,
//            one thread per column), stored as a bf16 tile image per chunk.
//   forward  one CTA per sequence walks its chunks; H^T lives in tensor memory (fp32, 128 lanes =
//            value index j, 128 columns = key index i); per chunk: U^T, W^T, Q K^T, then
//            H^T W^T and Q H, then H^T += delta^T K and O += P delta. The bf16 copy of H_c that
//            fed the chunk's products is checkpointed (the backward reuses it, no recomputation
//            of the state chain).
//   backward one CTA per sequence walks the chunks in reverse for the state gradient
//            dH_c = dH_{c+1} + Q^T dO - W^T ddelta, ddelta = P^T dO + K dH_{c+1}, checkpointing
//            the bf16 dH_{c+1}; then a chunk-parallel kernel forms every local gradient from
//            (H_c, dH_{c+1}) in one pass: dq, dk, dv, dbeta.
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
constexpr int NT = 128;  // threads per CTA

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

// Column j of a float32 [D][D] matrix (zero-padded to 128) -> tensor-memory row and bf16 tile row
__device__ __forceinline__ void column_to_tmem_and_tile(const float* mat, int D, int j, uint32_t lane_tm,
                                                        int col, uint8_t* tile) {
#pragma unroll
  for (int c0 = 0; c0 < DP; c0 += 32) {
    float v[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = (mat != nullptr && c0 + e < D && j < D) ? mat[(int64_t)(c0 + e) * D + j] : 0.f;
    tmem_st32(lane_tm + (uint32_t)(col + c0), v);
    st_row32_bf16(tile, 128, j, c0, v);
  }
  tmem_wait_st();
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

// all threads: bounded wait on the MMA barrier; flips the phase
__device__ __forceinline__ bool mma_wait(uint64_t* bar, uint32_t& phase, int* status) {
  const bool ok = mbar_wait(bar, phase);
  phase ^= 1u;
  if (!ok && threadIdx.x == 0) atomicOr(status, 2);
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

// T' = X diag(beta) written twice: rows 0-63 and rows 64-127 of a 128-row tile; thread t of n
__device__ __forceinline__ void scale_columns_twice(uint8_t* TT, const uint8_t* Xt, const float* bsm, int t, int n) {
  for (int q = t; q < 64 * 8; q += n) {
    const int r = q >> 3, j = q & 7;
    uint4 w = *reinterpret_cast<const uint4*>(Xt + sw_chunk(64, r, j));
    bf16* e = reinterpret_cast<bf16*>(&w);
#pragma unroll
    for (int i = 0; i < 8; ++i) e[i] = __float2bfloat16_rn(__bfloat162float(e[i]) * bsm[8 * j + i]);
    *reinterpret_cast<uint4*>(TT + sw_chunk(128, r, j)) = w;
    *reinterpret_cast<uint4*>(TT + sw_chunk(128, r + 64, j)) = w;
  }
}

// ------------------------------------------------------------------------------------------
// prep, chunk-parallel: one stacked product [K; Q] K^T (M=128) gives K K^T (rows 0-63) and Q K^T
// (rows 64-127). From K K^T: X = (I + strictly_lower(diag(beta) K K^T))^-1 by float32 forward
// substitution (one thread per column); from Q K^T: P = lower_inclusive(Q K^T). Per chunk the
// scratch holds the bf16 tile images [X 8 KB][P 8 KB][T'; T' 16 KB], T' = bf16(bf16(X) beta).
// ------------------------------------------------------------------------------------------
// per chunk: X [64][64], P [64][64], then T' = X diag(beta) written twice ([T'; T'], 128 rows): the
// forward's stacked [T';T'] operand, whose first 8 KB is the plain T' tile the backward reads
constexpr uint32_t PREP_X = 0, PREP_P = TILE_TT, PREP_T = 2 * TILE_TT, PREP_BYTES = 4 * TILE_TT;

__global__ void __launch_bounds__(NT) scan_prep_kernel(const __grid_constant__ CUtensorMap qmap,
                                                       const __grid_constant__ CUtensorMap kmap,
                                                       const bf16* __restrict__ beta,
                                                       uint8_t* __restrict__ xt, int T, int H,
                                                       int D, int NC, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* KQ = sm;  // [128 rows][128 d]: K rows 0-63, Q rows 64-127; dead once the product is read
  uint8_t* Xs = sm;  // then the output image over it: [X 8 KB][P 8 KB][T'; T' 16 KB]
  uint8_t* Ps = Xs + PREP_P;
  uint8_t* TTs = Xs + PREP_T;
  float* A = reinterpret_cast<float*>(sm + PREP_BYTES);  // [64][65]
  __shared__ float bsm[C];
  __shared__ uint64_t bar, lbar;
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int c = blockIdx.x % NC, bh = blockIdx.x / NC, b = bh / H, h = bh % H;
  const int t0 = c * C, valid = min(C, T - t0);
  const int64_t row0 = (int64_t)b * T + t0;
  if (tid == 0) { mbar_init(&bar, 1); mbar_init(&lbar, 1); mbar_fence_init(); }
  __syncthreads();
  if (tid == 0) {
    mbar_arrive_expect_tx(&lbar, 2 * TILE_TD);
    tma_load_4d(KQ, &kmap, &lbar, 0, h, t0, b);
    tma_load_4d(KQ + TILE_JI / 2, &kmap, &lbar, 64, h, t0, b);
    tma_load_4d(KQ + TILE_TD / 2, &qmap, &lbar, 0, h, t0, b);
    tma_load_4d(KQ + TILE_JI / 2 + TILE_TD / 2, &qmap, &lbar, 64, h, t0, b);
  }
  const bf16 bv = fetch_beta(beta + h, row0, H, valid);
  if (warp == 0) { tmem_alloc(&tbase, 64); tmem_relinquish(); }
  if (!mbar_wait(&lbar, 0) && tid == 0) atomicOr(status, 4);
  if (tid < C) bsm[tid] = __bfloat162float(bv);  // after the tile wait: both loads in flight together
  publish();
  const uint32_t tm = tbase;
  if (tid == 0) {
    mma_seq<DP / 16, 0, 128, 0, 128>(tm, smem_u32(KQ), smem_u32(KQ), idesc_bf16(128, 64, 0, 0), 0u);
    umma_commit(&bar);
  }
  uint32_t phase = 0;
  const bool ok = mma_wait(&bar, phase, status);
  {
    const int row = tid;  // M=128 layout: thread <-> lane <-> row
#pragma unroll
    for (int c0 = 0; c0 < 64; c0 += 32) {
      float v[32];
      tmem_ld32(taddr(tm, warp * 32, c0), v);
      tmem_wait_ld();
      if (row < C) {
#pragma unroll
        for (int e = 0; e < 32; ++e) A[row * 65 + c0 + e] = c0 + e < row ? bsm[row] * v[e] : 0.f;
      } else {
        const int t = row - C;
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = c0 + e <= t ? v[e] : 0.f;
        st_row32_bf16(Ps, 64, t, c0, v);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tm, 64);
  if (!ok) return;
  if (tid < 64) {
    const int j = tid;
    float x[64];
#pragma unroll
    for (int t = 0; t < 64; ++t) {
      float acc = (t == j) ? 1.f : 0.f;
#pragma unroll
      for (int s = 0; s < t; ++s) acc = fmaf(-A[t * 65 + s], x[s], acc);
      x[t] = acc;
    }
#pragma unroll
    for (int t = 0; t < 64; ++t) *reinterpret_cast<bf16*>(Xs + sw_offset(64, t, j)) = __float2bfloat16_rn(x[t]);
  }
  __syncthreads();
  scale_columns_twice(TTs, Xs, bsm, tid, NT);
  fence_async_smem();
  __syncthreads();
  if (tid == 0) {
    bulk_store(xt + (size_t)blockIdx.x * PREP_BYTES, Xs, PREP_BYTES);
    bulk_commit();
    bulk_wait_all();
  }
}

// ------------------------------------------------------------------------------------------
// forward: one CTA (256 threads) per (b, h). H^T lives in tensor memory (lane j = value index,
// column i = key index); the chunk's products run in the "rows t" form with the token rows
// duplicated over both halves of the 128 lanes, so all eight warps share every readout:
//   [U | W] = [T'; T'] [V | K]         (N = 256, issued during the previous chunk)
//   X = [W; W] H,  O = Q H              (batch B)  -> delta = U - X        (rows t)
//   H^T += delta^T K                    (batch C1) -> bf16 copy of H for the next chunk
//   O += P delta, [U | W] of chunk c+1  (batch C2) -> O stored, W of chunk c+1 staged
// Warp w reads lane quarter w % 4; the two warps of a quarter split the columns (w / 4).
// ------------------------------------------------------------------------------------------
constexpr int NT2 = 256;
struct FwdSmem {
  // per-chunk input set: [V | K] adjacent (the MN-major B operand [V | K]), Q, then P and
  // [T'; T'] (128 rows x 64) as the prep wrote them
  static constexpr uint32_t Vt = 0, Kt = TILE_TD, Qt = 2 * TILE_TD, Pt = 3 * TILE_TD, TT = Pt + TILE_TT;
  static constexpr uint32_t SET = TT + TILE_JT;  // 72 KB
  static constexpr uint32_t WW = 2 * SET,            // [W; W] 128 rows x 128
      Ha = WW + TILE_JI,                             // H^T bf16 [j][i]
      Dr = Ha + TILE_JI,                             // delta rows [t][j]
      END = Dr + TILE_TD;
};
constexpr int F_H = 0, F_U = 128, F_W = 256, F_X = 256, F_O = 384;

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

__global__ void __launch_bounds__(NT2, 1) scan_fwd_kernel(
    const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
    const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap omap,
    const bf16* __restrict__ beta, const float* __restrict__ s0, const uint8_t* __restrict__ xt,
    float* __restrict__ sn, uint8_t* __restrict__ hck, int T, int H, int D,
    int NC, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t *WW = sm + FwdSmem::WW, *Ha = sm + FwdSmem::Ha, *Dr = sm + FwdSmem::Dr;
  __shared__ uint64_t barB, barH, barC, lbar[2];
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;
  const int lane128 = quarter * 32 + lane;   // this thread's tensor-memory lane
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  uint32_t lphase[2] = {0u, 0u};
  auto set = [&](int c) { return sm + (uint32_t)(c & 1) * FwdSmem::SET; };
  auto load_chunk = [&](int c) {
    const ChunkAt a = chunk_at(b, c, T);
    uint8_t* s = set(c);
    if (tid == 0) {
      uint64_t* lb = &lbar[c & 1];
      mbar_arrive_expect_tx(lb, 3 * TILE_TD + PREP_BYTES - PREP_P);
      tma_tile(s + FwdSmem::Vt, &vmap, lb, h, a.t0, b);
      tma_tile(s + FwdSmem::Kt, &kmap, lb, h, a.t0, b);
      tma_tile(s + FwdSmem::Qt, &qmap, lb, h, a.t0, b);
      bulk_load(s + FwdSmem::Pt, xt + ((size_t)bh * NC + c) * PREP_BYTES + PREP_P, PREP_BYTES - PREP_P, lb);
    }
  };
  auto wait_chunk = [&](int c) -> bool {
    const bool r = mbar_wait(&lbar[c & 1], lphase[c & 1]);
    lphase[c & 1] ^= 1u;
    if (!r && tid == 0) atomicOr(status, 4);
    return r;
  };
  if (tid == 0) {
    mbar_init(&barB, 1); mbar_init(&barH, 1); mbar_init(&barC, 1);
    mbar_init(&lbar[0], 1); mbar_init(&lbar[1], 1);
    mbar_fence_init();
  }
  if (warp == 0) { tmem_alloc(&tbase, 512); tmem_relinquish(); }
  __syncthreads();
  if (NC > 0) load_chunk(0);
  tc_fence_after();
  const uint32_t tm = tbase;
  const uint32_t lane_tm = taddr(tm, quarter * 32, 0);
  // H^T row j = column j of the initial state (warps 0-3; warps 4-7 idle here)
  if (half == 0) column_to_tmem_and_tile(s0 + (int64_t)bh * D * D, D, lane128, lane_tm, F_H, Ha);
  const uint32_t sWW = smem_u32(WW), sH = smem_u32(Ha), sD = smem_u32(Dr);
  const uint32_t id_uw = idesc_bf16(128, 256, 0, 1);  // [T';T'] (K) x [V|K] (MN)
  const uint32_t id_xo = idesc_bf16(128, 128, 0, 0);  // X = [W;W] H: both K-major
  const uint32_t id_qh = idesc_bf16(64, 128, 0, 0);   // O = Q H
  const uint32_t id_hk = idesc_bf16(128, 128, 1, 1);  // H^T += delta^T K: both MN-major
  const uint32_t id_pd = idesc_bf16(64, 128, 0, 1);   // O += P delta
  // token row of this thread in the duplicated "rows t" layout, and its 32-column slice
  const int trow = lane128 & 63;
  const int upper = lane128 >> 6;  // 0: lanes 0-63, 1: lanes 64-127
  auto readout_w = [&]() {         // W rows (duplicated lanes) -> [W; W]
    const int c0 = half * 64;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      float v[32];
      tmem_ld32(lane_tm + (uint32_t)(F_W + c0 + 32 * k), v);
      tmem_wait_ld();
      st_row32_bf16(WW, 128, upper * 64 + trow, c0 + 32 * k, v);
    }
  };
  uint32_t pB = 0, pH = 0, pC = 0;
  bool ok = true;
  if (NC > 0) {
    ok = wait_chunk(0);
    publish();
    if (tid == 0) {
      mma_seq<4, 0, 128, 1, 64>(tm + F_U, smem_u32(set(0) + FwdSmem::TT), smem_u32(set(0) + FwdSmem::Vt), id_uw, 0u);
      umma_commit(&barC);
    }
    ok = mma_wait(&barC, pC, status) && ok;
    if (NC > 1) load_chunk(1);
    readout_w();
    publish();
  }
  for (int c = 0; c < NC && ok; ++c) {
    const ChunkAt a = chunk_at(b, c, T);
    const bool more = c + 1 < NC;
    if (tid == 0) {  // checkpoint H_c (the bf16 copy the chunk's products read)
      bulk_store(hck + ((size_t)bh * NC + c) * TILE_JI, Ha, TILE_JI);
      bulk_commit();
    }
    const uint32_t sQ = smem_u32(set(c) + FwdSmem::Qt), sK = smem_u32(set(c) + FwdSmem::Kt);
    const uint32_t sP = smem_u32(set(c) + FwdSmem::Pt);
    if (tid == 0) {
      mma_seq<8, 0, 128, 0, 128>(tm + F_X, sWW, sH, id_xo, 0u);  // X = [W;W] H
      umma_commit(&barB);
      mma_seq<8, 0, 64, 0, 128>(tm + F_O, sQ, sH, id_qh, 0u);    // O = Q H (waited on with C2)
    }
    ok = mma_wait(&barB, pB, status) && ok;
    {
      // delta = U - X, rows t (Dr was released by the previous chunk's O store before the
      // barrier that ended that chunk); lanes 0-63 take columns 0-63, lanes 64-127 columns 64-127
      const int c0 = upper * 64 + half * 32;
      float u[32], x[32];
      tmem_ld32(lane_tm + (uint32_t)(F_U + c0), u);
      tmem_ld32(lane_tm + (uint32_t)(F_X + c0), x);
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 32; ++e) u[e] -= x[e];
      st_row32_bf16(Dr, 64, trow, c0, u);
    }
    if (more) ok = wait_chunk(c + 1) && ok;
    if (tid == 0) bulk_wait_read();  // the checkpoint has left Ha before it is rewritten
    publish();
    if (tid == 0 && ok) {
      mma_seq<4, 1, 64, 1, 64>(tm + F_H, sD, sK, id_hk, 1u);     // H^T += delta^T K
      umma_commit(&barH);
      mma_seq<4, 0, 64, 1, 64>(tm + F_O, sP, sD, id_pd, 1u);     // O += P delta
      if (more)
        mma_seq<4, 0, 128, 1, 64>(tm + F_U, smem_u32(set(c + 1) + FwdSmem::TT), smem_u32(set(c + 1) + FwdSmem::Vt), id_uw, 0u);
      umma_commit(&barC);
    }
    ok = ok && mma_wait(&barH, pH, status);
    {
      // H^T row j -> bf16 Ha (and the final state)
      const int c0 = half * 64;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float v[32];
        tmem_ld32(lane_tm + (uint32_t)(F_H + c0 + 32 * k), v);
        tmem_wait_ld();
        st_row32_bf16(Ha, 128, lane128, c0 + 32 * k, v);
        if (!more && lane128 < D) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (c0 + 32 * k + e < D) sn[(int64_t)bh * D * D + (int64_t)(c0 + 32 * k + e) * D + lane128] = v[e];
        }
      }
    }
    ok = ok && mma_wait(&barC, pC, status);
    if (c + 2 < NC) load_chunk(c + 2);  // set (c & 1) is free: every product of chunk c is done
    {
      // O rows (M=64 layout: lanes 0-15 of each quarter hold t = 16 quarter + lane) staged in
      // Dr (free once the state update has completed) for one TMA store
      const int t = quarter * 16 + (lane & 15);
      const int c0 = half * 64;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float v[32];
        tmem_ld32(lane_tm + (uint32_t)(F_O + c0 + 32 * k), v);
        tmem_wait_ld();
        if (lane < 16) st_row32_bf16(Dr, 64, t, c0 + 32 * k, v);
      }
    }
    if (more) readout_w();
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {
      tma_store_4d(&omap, Dr, 0, h, a.t0, b);
      if (D > 64) tma_store_4d(&omap, Dr + TILE_TD / 2, 64, h, a.t0, b);
      bulk_commit();
      bulk_wait_read();  // Dr is rewritten by the next chunk's delta readout
    }
    publish();
  }
  if (NC == 0 && half == 0) {
    const int j = lane128;
    if (j < D)
      for (int i = 0; i < D; ++i) sn[(int64_t)bh * D * D + (int64_t)i * D + j] = s0[(int64_t)bh * D * D + (int64_t)i * D + j];
  }
  if (tid == 0) bulk_wait_all();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tm, 512);
}

// ------------------------------------------------------------------------------------------
// backward, sequential (256 threads): the dH^T chain in tensor memory, in reverse chunk order,
// checkpointing the bf16 dH_{c+1} per chunk:
//   B:  ddelta^T = dH^T K^T;  [ddelta^T | dH^T] += dO^T [P | Q]    (N = 192)
//   C1: dH^T -= ddelta^T W                                          -> bf16 copy of dH
//   C2: W of chunk c-1 = T' K                                       -> staged for the next C1
// ------------------------------------------------------------------------------------------
struct DhSmem {
  // per-chunk input set: T', then P immediately before Q (the MN-major B operand [P | Q]), K, dO
  static constexpr uint32_t Tt = 0, Pt = TILE_TT, Qt = 2 * TILE_TT, Kt = Qt + TILE_TD, Gt = Kt + TILE_TD;
  static constexpr uint32_t SET = Gt + TILE_TD;  // 64 KB
  static constexpr uint32_t Wk = 2 * SET, Ha = Wk + TILE_TD, Da = Ha + TILE_JI, END = Da + TILE_JT;
};
constexpr int G_D = 0, G_H = 64, G_W = 192;

__global__ void __launch_bounds__(NT2, 1) scan_dh_kernel(
    const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
    const __grid_constant__ CUtensorMap gmap, const bf16* __restrict__ beta,
    const uint8_t* __restrict__ xt, const float* __restrict__ dsn,
    float* __restrict__ ds0, uint8_t* __restrict__ dhck, int T, int H, int D, int NC, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t *Wk = sm + DhSmem::Wk, *Ha = sm + DhSmem::Ha, *Da = sm + DhSmem::Da;
  __shared__ uint64_t barB, barH, barC, lbar[2];
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;
  const int lane128 = quarter * 32 + lane;
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  uint32_t lphase[2] = {0u, 0u};
  auto set = [&](int c) { return sm + (uint32_t)(c & 1) * DhSmem::SET; };
  auto load_chunk = [&](int c) {
    const ChunkAt a = chunk_at(b, c, T);
    uint8_t* s = set(c);
    if (tid == 0) {
      uint64_t* lb = &lbar[c & 1];
      mbar_arrive_expect_tx(lb, 3 * TILE_TD + 2 * TILE_TT);
      const uint8_t* pre = xt + ((size_t)bh * NC + c) * PREP_BYTES;
      bulk_load(s + DhSmem::Tt, pre + PREP_T, TILE_TT, lb);
      bulk_load(s + DhSmem::Pt, pre + PREP_P, TILE_TT, lb);
      tma_tile(s + DhSmem::Qt, &qmap, lb, h, a.t0, b);
      tma_tile(s + DhSmem::Kt, &kmap, lb, h, a.t0, b);
      tma_tile(s + DhSmem::Gt, &gmap, lb, h, a.t0, b);
    }
  };
  auto wait_chunk = [&](int c) -> bool {
    const bool r = mbar_wait(&lbar[c & 1], lphase[c & 1]);
    lphase[c & 1] ^= 1u;
    if (!r && tid == 0) atomicOr(status, 4);
    return r;
  };
  if (tid == 0) {
    mbar_init(&barB, 1); mbar_init(&barH, 1); mbar_init(&barC, 1);
    mbar_init(&lbar[0], 1); mbar_init(&lbar[1], 1);
    mbar_fence_init();
  }
  if (warp == 0) { tmem_alloc(&tbase, 512); tmem_relinquish(); }
  __syncthreads();
  if (NC > 0) load_chunk(NC - 1);
  tc_fence_after();
  const uint32_t tm = tbase;
  const uint32_t lane_tm = taddr(tm, quarter * 32, 0);
  if (half == 0)
    column_to_tmem_and_tile(dsn != nullptr ? dsn + (int64_t)bh * D * D : nullptr, D, lane128, lane_tm, G_H, Ha);
  const uint32_t sW = smem_u32(Wk), sH = smem_u32(Ha), sD = smem_u32(Da);
  const uint32_t id_hk = idesc_bf16(128, 64, 0, 0);       // ddelta^T = dH^T K^T
  const uint32_t id_opq = idesc_bf16(128, 192, 1, 1);     // [ddelta^T | dH^T] += dO^T [P | Q]
  const uint32_t id_dw = idesc_bf16(128, 128, 0, 1, 1);   // dH^T -= ddelta^T W
  const uint32_t id_tk = idesc_bf16(64, 128, 0, 1);       // W = T' K
  auto readout_w = [&]() {  // W rows (M=64 layout) -> Wk [t][i]
    const int t = quarter * 16 + (lane & 15);
    const int c0 = half * 64;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      float v[32];
      tmem_ld32(lane_tm + (uint32_t)(G_W + c0 + 32 * k), v);
      tmem_wait_ld();
      if (lane < 16) st_row32_bf16(Wk, 64, t, c0 + 32 * k, v);
    }
  };
  uint32_t pB = 0, pH = 0, pC = 0;
  bool ok = true;
  if (NC > 0) {
    ok = wait_chunk(NC - 1);
    publish();
    if (tid == 0) {
      mma_seq<4, 0, 64, 1, 64>(tm + G_W, smem_u32(set(NC - 1) + DhSmem::Tt), smem_u32(set(NC - 1) + DhSmem::Kt),
                               id_tk, 0u);
      umma_commit(&barC);
    }
    ok = mma_wait(&barC, pC, status) && ok;
    if (NC > 1) load_chunk(NC - 2);
    readout_w();
    publish();
  }
  for (int c = NC - 1; c >= 0 && ok; --c) {
    const bool more = c > 0;
    if (tid == 0) {  // checkpoint dH_{c+1}
      bulk_store(dhck + ((size_t)bh * NC + c) * TILE_JI, Ha, TILE_JI);
      bulk_commit();
    }
    const uint32_t sK = smem_u32(set(c) + DhSmem::Kt), sP = smem_u32(set(c) + DhSmem::Pt);
    const uint32_t sG = smem_u32(set(c) + DhSmem::Gt);
    if (tid == 0) {
      mma_seq<8, 0, 128, 0, 64>(tm + G_D, sH, sK, id_hk, 0u);   // ddelta^T = dH^T K^T
      mma_seq<4, 1, 64, 1, 64>(tm + G_D, sG, sP, id_opq, 1u);   // [ddelta^T | dH^T] += dO^T [P | Q]
      umma_commit(&barB);
    }
    ok = mma_wait(&barB, pB, status) && ok;
    {
      const int c0 = half * 32;
      float v[32];
      tmem_ld32(lane_tm + (uint32_t)(G_D + c0), v);
      tmem_wait_ld();
      st_row32_bf16(Da, 128, lane128, c0, v);  // ddelta^T row j
    }
    if (more) ok = wait_chunk(c - 1) && ok;
    if (tid == 0) bulk_wait_read();
    publish();
    if (tid == 0 && ok) {
      mma_seq<4, 0, 128, 1, 64>(tm + G_H, sD, sW, id_dw, 1u);   // dH^T -= ddelta^T W
      umma_commit(&barH);
      if (more)
        mma_seq<4, 0, 64, 1, 64>(tm + G_W, smem_u32(set(c - 1) + DhSmem::Tt), smem_u32(set(c - 1) + DhSmem::Kt),
                                 id_tk, 0u);
      umma_commit(&barC);
    }
    ok = ok && mma_wait(&barH, pH, status);
    {
      const int c0 = half * 64;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float v[32];
        tmem_ld32(lane_tm + (uint32_t)(G_H + c0 + 32 * k), v);
        tmem_wait_ld();
        st_row32_bf16(Ha, 128, lane128, c0 + 32 * k, v);
        if (c == 0 && lane128 < D) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (c0 + 32 * k + e < D) ds0[(int64_t)bh * D * D + (int64_t)(c0 + 32 * k + e) * D + lane128] = v[e];
        }
      }
    }
    ok = ok && mma_wait(&barC, pC, status);
    if (c >= 2) load_chunk(c - 2);  // set (c & 1) is free: every product of chunk c is done
    if (more) readout_w();
    publish();
  }
  if (NC == 0 && half == 0) {
    const int j = lane128;
    if (j < D)
      for (int i = 0; i < D; ++i)
        ds0[(int64_t)bh * D * D + (int64_t)i * D + j] = dsn ? dsn[(int64_t)bh * D * D + (int64_t)i * D + j] : 0.f;
  }
  if (tid == 0) bulk_wait_all();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tm, 512);
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
__device__ __forceinline__ void ld32w(uint32_t tm, int col, float (&v)[32]) {
  tmem_ld32(tm + (uint32_t)col, v);
  tmem_wait_ld();
}
// row `r` of a float32 accumulator (64 of its columns from `c0`) as bf16 at columns c0.. of a
// [64 t][128] global row (dq, dk, dv); columns at or past D are skipped
__device__ __forceinline__ void store_row64(bf16* dst, const float* r, int c0, int D) {
#pragma unroll
  for (int i = 0; i < 64; i += 8) {
    if (c0 + i >= D) break;
    uint4 w4;
    w4.x = pack_bf16(r[i], r[i + 1]); w4.y = pack_bf16(r[i + 2], r[i + 3]);
    w4.z = pack_bf16(r[i + 4], r[i + 5]); w4.w = pack_bf16(r[i + 6], r[i + 7]);
    *reinterpret_cast<uint4*>(dst + c0 + i) = w4;
  }
}

__global__ void __launch_bounds__(NG, 1) scan_grad_kernel(
    const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
    const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap gmap,
    const bf16* __restrict__ beta, const uint8_t* __restrict__ xt, const uint8_t* __restrict__ hck,
    const uint8_t* __restrict__ dhck, bf16* __restrict__ dq,
    bf16* __restrict__ dk, bf16* __restrict__ dv, bf16* __restrict__ dbeta, int T, int H, int D,
    int NC, int* status) {
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
  __shared__ uint64_t bar, lbar;
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // warps w and w + 4 share tensor-memory lane quadrant w % 4 and split the columns (half)
  const int quarter = warp & 3, half = warp >> 2;
  const int lane128 = quarter * 32 + lane;
  const int c = blockIdx.x % NC, bh = blockIdx.x / NC, b = bh / H, h = bh % H;
  const int t0 = c * C, valid = min(C, T - t0);
  const int64_t ld = (int64_t)H * D;
  const int64_t row0 = (int64_t)b * T + t0;
  const int trow = quarter * 16 + (lane & 15);  // token row of an M=64 accumulator (lane < 16)
  const bool rowlane = lane < 16;
  const size_t chunk = (size_t)bh * NC + c;
  if (tid == 0) { mbar_init(&bar, 1); mbar_init(&lbar, 1); mbar_fence_init(); }
  __syncthreads();
  if (tid == 0) {
    mbar_arrive_expect_tx(&lbar, 4 * TILE_TD + 2 * TILE_JI + 3 * TILE_TT);
    tma_tile(Qt, &qmap, &lbar, h, t0, b);
    tma_tile(Kt, &kmap, &lbar, h, t0, b);
    tma_tile(Vt, &vmap, &lbar, h, t0, b);
    tma_tile(Gt, &gmap, &lbar, h, t0, b);
    bulk_load(Ht, hck + chunk * TILE_JI, TILE_JI, &lbar);
    bulk_load(dHt, dhck + chunk * TILE_JI, TILE_JI, &lbar);
    bulk_load(Xt, xt + chunk * PREP_BYTES + PREP_X, TILE_TT, &lbar);
    bulk_load(Pt, xt + chunk * PREP_BYTES + PREP_P, TILE_TT, &lbar);
    bulk_load(Tt, xt + chunk * PREP_BYTES + PREP_T, TILE_TT, &lbar);
  }
  const bf16 bv = fetch_beta(beta + h, row0, H, valid);
  if (warp == 0) { tmem_alloc(&tbase, 512); tmem_relinquish(); }
  if (!mbar_wait(&lbar, 0) && tid == 0) atomicOr(status, 4);
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
  bool ok = true;
  // batch 1: K K^T, Q K^T, W^T, U^T, ddelta^T = dH'^T K^T
  if (tid == 0) {
    const uint32_t id64 = idesc_bf16(64, 64, 0, 0);
    mma_seq<8, 0, 64, 0, 64>(tm + R_KK, sK, sK, id64, 0u);
    const uint32_t id_tn = idesc_bf16(128, 64, 1, 0);
    mma_seq<4, 1, 64, 0, 64>(tm + R_W, sK, sT, id_tn, 0u);
    mma_seq<4, 1, 64, 0, 64>(tm + R_U, sV, sT, id_tn, 0u);
    const uint32_t id_hk = idesc_bf16(128, 64, 0, 0);
    mma_seq<8, 0, 128, 0, 64>(tm + R_DD, sdH, sK, id_hk, 0u);
    umma_commit(&bar);
  }
  ok = mma_wait(&bar, phase, status);
  {
    float w[32];
    ld32w(lane_tm, R_W + half * 32, w);
    st_row32_bf16(Wr, 128, lane128, half * 32, w);
  }
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
    if (rowlane && trow < valid) store_row64(dv + (row0 + trow) * ld + (int64_t)h * D, r, half * 64, D);
  }
  publish();
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
    if (rowlane && trow < valid) store_row64(dq + (row0 + trow) * ld + (int64_t)h * D, r, half * 64, D);
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
  if (tid < C) {
    float a = 0.f;
    for (int t = 0; t < C; ++t) a += scr[t * 65 + tid];
    db1[tid] = a;
  }
  // batch 5: Y = dX X^T
  if (tid == 0 && ok) {
    const uint32_t id = idesc_bf16(64, 64, 0, 0);
    mma_seq<4, 0, 64, 0, 64>(tm + R_Y, sdX, sX, id, 0u);
    umma_commit(&bar);
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
    if (rowlane && trow < valid) store_row64(dk + (row0 + trow) * ld + (int64_t)h * D, r, half * 64, D);
  }
  tc_fence_before();
  __syncthreads();
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
    const size_t sp = smem_bytes(PREP_BYTES + 64 * 65 * 4);
    VB_CUDA_CHECK(cudaFuncSetAttribute(scan_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sp), "prep attr");
    scan_prep_kernel<<<B * H * NC, NT, sp, st>>>(qm, km, (const bf16*)beta, xt, T, H, D, NC, status);
    VB_LAUNCH_CHECK("delta_scan_bf16 prep");
  } else {
    memset(&qm, 0, sizeof(qm)); memset(&km, 0, sizeof(km)); memset(&vm, 0, sizeof(vm));
  }
  const size_t sf = smem_bytes(FwdSmem::END);
  VB_CUDA_CHECK(cudaFuncSetAttribute(scan_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sf), "fwd attr");
  scan_fwd_kernel<<<B * H, NT2, sf, st>>>(qm, km, vm, om, (const bf16*)beta,
                                         state0, xt, state_n, hck, T, H, D, NC, status);
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
  scan_dh_kernel<<<B * H, NT2, sd, st>>>(qm, km, gm, (const bf16*)beta, xt,
                                        dstate_n, dstate0, dhck, T, H, D, NC, status);
  VB_LAUNCH_CHECK("delta_scan_bf16 dh");
  if (NC > 0) {
    const size_t sg = smem_bytes(GrSmem::END);
    VB_CUDA_CHECK(cudaFuncSetAttribute(scan_grad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sg), "grad attr");
    scan_grad_kernel<<<B * H * NC, NG, sg, st>>>(qm, km, vm, gm, (const bf16*)beta,
                                                 xt, hck, dhck, (bf16*)dq, (bf16*)dk, (bf16*)dv,
                                                 (bf16*)dbeta, T, H, D, NC, status);
    VB_LAUNCH_CHECK("delta_scan_bf16 grad");
  }
  return VB_OK;
}
